// Host side of the C ABI declared in include/llm_fa_b200.h: argument checks,
// TMA tensor-map encoding, persistent-grid sizing and the launch of
// llmfa::llm_fa_kernel_sm100 on the caller's stream.
//
// Mirrors the reference launcher llm_fa_forward (llm_fa.cu:1418-1475) with
// three differences: (1) no allocation and no device synchronisation — O is
// the caller's buffer and the launch is stream-ordered; (2) errors are status
// codes instead of TORCH_CHECK exceptions; (3) [B, S, H, 128] strided views
// instead of 2-D contiguous tensors, encoded as 4-D tensor maps (D, H, S, B)
// so that out-of-range rows are zero-filled on load and clipped on store.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "../../include/llm_fa_b200.h"
#include "fa_fwd_kernel.cuh"

namespace {

constexpr int kVersion = 100;  // 0.1.0
constexpr int kMaxDevices = 64;
constexpr int kSiteSelftest = 15;

__device__ int g_device_status = 0;

struct DeviceSetup {
  std::once_flag once;
  int err = LLMFA_OK;
  int* status_ptr = nullptr;  // device address of g_device_status on this device
  int max_clusters = 0;
};
DeviceSetup g_setup[kMaxDevices];

std::atomic<unsigned long long> g_timeout_ns{0};

unsigned long long wait_timeout_ns() {
  unsigned long long t = g_timeout_ns.load(std::memory_order_relaxed);
  if (t == 0) {
    unsigned long long ms = 2000;
    if (const char* e = std::getenv("LLMFA_WAIT_TIMEOUT_MS")) {
      const long long v = std::atoll(e);
      if (v > 0) ms = static_cast<unsigned long long>(v);
    }
    t = ms * 1000000ull;
    unsigned long long expected = 0;
    g_timeout_ns.compare_exchange_strong(expected, t);
    t = g_timeout_ns.load(std::memory_order_relaxed);
  }
  return t;
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      ptr = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }();
  return fn;
}

// Once per device (with that device current): opt in to the kernel's shared
// memory, look up the device address of the status word, size the grid.
int device_setup(int* dev_out, DeviceSetup** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return LLMFA_ERR_CUDA;
  }
  DeviceSetup& s = g_setup[dev];
  std::call_once(s.once, [&] {
    if (cudaFuncSetAttribute(llmfa::llm_fa_kernel_sm100<false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(llmfa::kSmemBytes)) != cudaSuccess ||
        cudaFuncSetAttribute(llmfa::llm_fa_kernel_sm100<true>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(llmfa::kSmemBytes)) != cudaSuccess ||
        cudaFuncSetAttribute(llmfa::llm_fa_combine_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(llmfa::kCombineMaxRound *
                                              llmfa::kCombinePieceBytes)) != cudaSuccess) {
      cudaGetLastError();
      s.err = LLMFA_ERR_CUDA;
      return;
    }
    void* sp = nullptr;
    if (cudaGetSymbolAddress(&sp, g_device_status) != cudaSuccess) {
      cudaGetLastError();
      s.err = LLMFA_ERR_CUDA;
      return;
    }
    s.status_ptr = static_cast<int*>(sp);
    int n = 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(llmfa::kThreads, 1, 1);
    cfg.dynamicSmemBytes = llmfa::kSmemBytes;
    if (cudaOccupancyMaxActiveClusters(&n, llmfa::llm_fa_kernel_sm100<false>, &cfg) != cudaSuccess ||
        n <= 0) {
      cudaGetLastError();
      int sms = 0;
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      n = sms / 2;
    }
    s.max_clusters = n > 0 ? n : 1;
  });
  if (s.err != LLMFA_OK) return s.err;
  *dev_out = dev;
  *out = &s;
  return LLMFA_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Checks one [B, S, H, 128] view; returns a status code.
int check_view(const void* ptr, const int64_t* st, int64_t seq, int64_t heads, int64_t batch) {
  if (ptr == nullptr || st == nullptr) return LLMFA_ERR_INVALID_ARGUMENT;
  if (!aligned16(ptr)) return LLMFA_ERR_UNSUPPORTED;
  const int64_t dims[3] = {batch, seq, heads};
  for (int i = 0; i < 3; ++i) {
    if (dims[i] == 1) continue;  // stride of a size-1 dimension is never used
    if (st[i] <= 0 || (st[i] % 8) != 0 || st[i] >= (int64_t(1) << 38))
      return LLMFA_ERR_UNSUPPORTED;
  }
  return LLMFA_OK;
}

// 4-D map over (D=128, H, S, B) with a (64, 1, rows, 1) box and 128-byte swizzle.
int encode_bshd(CUtensorMap* m, const void* ptr, const int64_t* st, int64_t seq, int64_t heads,
                int64_t batch, uint32_t box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = get_encode_fn();
  if (enc == nullptr) return LLMFA_ERR_CUDA;
  // Size-1 dimensions get a canonical stride (their stride is never applied).
  const uint64_t sh = heads == 1 ? 128 : static_cast<uint64_t>(st[2]);
  const uint64_t ss = seq == 1 ? sh * static_cast<uint64_t>(heads) : static_cast<uint64_t>(st[1]);
  const uint64_t sb = batch == 1 ? ss * static_cast<uint64_t>(seq) : static_cast<uint64_t>(st[0]);
  cuuint64_t dims[4] = {128, static_cast<cuuint64_t>(heads), static_cast<cuuint64_t>(seq),
                        static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[3] = {sh * 2, ss * 2, sb * 2};
  cuuint32_t box[4] = {64, 1, box_rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(ptr), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? LLMFA_OK : LLMFA_ERR_TENSOR_MAP;
}

// The units of a stream-K launch that were cut across clusters, with their
// pieces, in the combine kernel's table; returns how many.
int list_split_units(const llmfa::FwdParams& p, llmfa::CombineParams* cp) {
  int n = 0, most = 0;
  for (int u = p.dp_units; u < p.n_units; ++u) {
    const llmfa::UnitPieces pc = llmfa::unit_pieces(p, u);
    if (pc.c_lo == pc.c_hi) continue;  // one cluster computed the whole unit
    const int np = pc.c_hi - pc.c_lo + 1;
    most = np > most ? np : most;
    if (cp != nullptr) {
      cp->unit[n] = u;
      cp->c_lo[n] = static_cast<short>(pc.c_lo);
      cp->np[n] = static_cast<short>(np);
      cp->slot_lo[n] = static_cast<short>(pc.slot_lo);
    }
    ++n;
  }
  if (cp != nullptr) cp->round_pieces = most < llmfa::kCombineMaxRound ? most : llmfa::kCombineMaxRound;
  return n;
}

__global__ void llmfa_wait_selftest_kernel(unsigned long long timeout_ns, int* status) {
  __shared__ __align__(8) uint64_t bar;
  const uint32_t b = llmfa::ptx::smem_u32(&bar);
  if (threadIdx.x == 0) {
    llmfa::ptx::mbar_init(b, 1);
    llmfa::g_cta_abort = 0u;
    llmfa::ptx::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const llmfa::WaitCtl c{status, timeout_ns};
    // Nothing arrives on `bar`: phase 0 never completes and the wait gives up.
    if (!llmfa::mbar_wait(b, 0, c, kSiteSelftest, false)) {
      // the status word already holds the wait site
    }
  }
}

}  // namespace

extern "C" {

int llmfa_version(void) { return kVersion; }

int llmfa_build_config(int* ablation, int* trace) {
  if (ablation == nullptr || trace == nullptr) return LLMFA_ERR_INVALID_ARGUMENT;
  *ablation = llmfa::kAblate;
  *trace = LLMFA_TRACE;
  return LLMFA_OK;
}

const char* llmfa_error_string(int status) {
  switch (status) {
    case LLMFA_OK: return "ok";
    case LLMFA_ERR_INVALID_ARGUMENT: return "invalid argument";
    case LLMFA_ERR_UNSUPPORTED: return "unsupported layout (alignment/stride)";
    case LLMFA_ERR_TENSOR_MAP: return "tensor map encoding failed";
    case LLMFA_ERR_LAUNCH: return "kernel launch failed";
    case LLMFA_ERR_CUDA: return "CUDA runtime error";
    case LLMFA_ERR_DEVICE_TIMEOUT: return "in-kernel wait timed out";
    default: return "unknown status";
  }
}

int llmfa_set_wait_timeout_ms(uint32_t ms) {
  if (ms == 0) return LLMFA_ERR_INVALID_ARGUMENT;
  g_timeout_ns.store(static_cast<unsigned long long>(ms) * 1000000ull);
  return LLMFA_OK;
}

int llmfa_workspace_size(uint64_t* bytes) {
  if (bytes == nullptr) return LLMFA_ERR_INVALID_ARGUMENT;
  int dev = 0;
  DeviceSetup* s = nullptr;
  int rc = device_setup(&dev, &s);
  if (rc != LLMFA_OK) return rc;
  *bytes = static_cast<uint64_t>(2 * s->max_clusters) * llmfa::kSlotBytes;
  return LLMFA_OK;
}

int llmfa_forward(const void* q, const int64_t q_strides[3], const void* k,
                  const int64_t k_strides[3], const void* v, const int64_t v_strides[3], void* o,
                  const int64_t o_strides[3], int64_t batch, int64_t heads, int64_t seq_q,
                  int64_t seq_k, float softmax_scale, void* workspace, uint64_t workspace_bytes,
                  void* stream) {
  return llmfa_forward_lse(q, q_strides, k, k_strides, v, v_strides, o, o_strides, nullptr,
                           nullptr, batch, heads, seq_q, seq_k, softmax_scale, workspace,
                           workspace_bytes, stream);
}

}  // extern "C"

namespace {

// Argument checks shared by every compute entry point; makes no CUDA call.
int check_forward_args(const void* q, const int64_t q_strides[3], const void* k,
                       const int64_t k_strides[3], const void* v, const int64_t v_strides[3],
                       const void* o, const int64_t o_strides[3], const float* lse,
                       const int64_t lse_strides[2], int64_t batch, int64_t heads, int64_t seq_q,
                       int64_t seq_k, float softmax_scale) {
  if (batch < 1 || heads < 1 || seq_q < 1 || seq_k < 1) return LLMFA_ERR_INVALID_ARGUMENT;
  if (!(softmax_scale > 0.f) || !std::isfinite(softmax_scale)) return LLMFA_ERR_INVALID_ARGUMENT;
  if (seq_q >= (int64_t(1) << 31) || seq_k >= (int64_t(1) << 31) || heads >= (1 << 24) ||
      batch >= (1 << 24))
    return LLMFA_ERR_UNSUPPORTED;
  const int64_t n_qblk = (seq_q + llmfa::kUnitRows - 1) / llmfa::kUnitRows;
  if (batch * heads * n_qblk >= (int64_t(1) << 31)) return LLMFA_ERR_UNSUPPORTED;
  int rc;
  if ((rc = check_view(q, q_strides, seq_q, heads, batch)) != LLMFA_OK) return rc;
  if ((rc = check_view(k, k_strides, seq_k, heads, batch)) != LLMFA_OK) return rc;
  if ((rc = check_view(v, v_strides, seq_k, heads, batch)) != LLMFA_OK) return rc;
  if ((rc = check_view(o, o_strides, seq_q, heads, batch)) != LLMFA_OK) return rc;
  if (lse != nullptr) {  // [batch, heads, seq_q] fp32, rows contiguous
    if (lse_strides == nullptr || (reinterpret_cast<uintptr_t>(lse) & 3u) != 0)
      return LLMFA_ERR_INVALID_ARGUMENT;
    if ((batch > 1 && lse_strides[0] < 1) || (heads > 1 && lse_strides[1] < 1))
      return LLMFA_ERR_INVALID_ARGUMENT;
  }
  return LLMFA_OK;
}

// Everything that determines the tensor maps and the launch plan of a call.
struct LaunchKey {
  const void *q, *k, *v, *o, *ws;
  const float* lse;
  int64_t qs[3], ks[3], vs[3], os[3], ls[2];
  int64_t batch, heads, seq_q, seq_k;
  uint64_t ws_bytes;
  uint32_t scale_bits;
};

// What one forward launches: the attention kernel's tensor maps and
// parameters, and the combine kernel's parameters when KV ranges are split.
struct LaunchSpec {
  CUtensorMap tq, tk, tv, to, tw;
  llmfa::FwdParams p;
  llmfa::CombineParams cp;
  int nclusters;
  bool combine;
};

// A few recent launch specs per device (round-robin replacement), so that a
// loop of calls on the same buffers skips the tensor-map encoding and the
// stream-K planning (host time that bounds small shapes).
class LaunchCache {
 public:
  bool lookup(const LaunchKey& key, LaunchSpec& out) {
    std::lock_guard<std::mutex> lock(mu_);
    for (int i = 0; i < kEntries; ++i) {
      if (valid_[i] && std::memcmp(&keys_[i], &key, sizeof(LaunchKey)) == 0) {
        out = specs_[i];
        return true;
      }
    }
    return false;
  }
  void insert(const LaunchKey& key, const LaunchSpec& spec) {
    std::lock_guard<std::mutex> lock(mu_);
    keys_[next_] = key;
    specs_[next_] = spec;
    valid_[next_] = true;
    next_ = (next_ + 1) % kEntries;
  }

 private:
  static constexpr int kEntries = 8;
  std::mutex mu_;
  LaunchKey keys_[kEntries];
  LaunchSpec specs_[kEntries];
  bool valid_[kEntries] = {};
  int next_ = 0;
};
LaunchCache g_cache[kMaxDevices];

// Encodes the tensor maps and plans the launch (persistent clusters, stream-K
// cut and the combine kernel's piece table) for checked arguments.
int make_launch_spec(const LaunchKey& a, const DeviceSetup& s, LaunchSpec& spec) {
  int rc;
  if ((rc = encode_bshd(&spec.tq, a.q, a.qs, a.seq_q, a.heads, a.batch, llmfa::kBlockM)) != LLMFA_OK)
    return rc;
  if ((rc = encode_bshd(&spec.tk, a.k, a.ks, a.seq_k, a.heads, a.batch,
                        llmfa::kBlockN / llmfa::kPair)) != LLMFA_OK)
    return rc;
  if ((rc = encode_bshd(&spec.tv, a.v, a.vs, a.seq_k, a.heads, a.batch, llmfa::kBlockN)) != LLMFA_OK)
    return rc;
  if ((rc = encode_bshd(&spec.to, a.o, a.os, a.seq_q, a.heads, a.batch, llmfa::kBlockM)) != LLMFA_OK)
    return rc;

  llmfa::FwdParams& p = spec.p;
  p = llmfa::FwdParams{};
  const int64_t n_qblk = (a.seq_q + llmfa::kUnitRows - 1) / llmfa::kUnitRows;
  float scale;
  std::memcpy(&scale, &a.scale_bits, sizeof(float));
  p.B = static_cast<int>(a.batch);
  p.H = static_cast<int>(a.heads);
  p.Sq = static_cast<int>(a.seq_q);
  p.Sk = static_cast<int>(a.seq_k);
  p.n_qblk = static_cast<int>(n_qblk);
  p.n_kv = static_cast<int>((a.seq_k + llmfa::kBlockN - 1) / llmfa::kBlockN);
  p.n_units = static_cast<int>(a.batch * a.heads * n_qblk);
  p.kv_tail = static_cast<int>(a.seq_k - int64_t(p.n_kv - 1) * llmfa::kBlockN);
  p.scale_log2 = scale * 1.4426950408889634f;
  p.lse = const_cast<float*>(a.lse);
  p.lse_sb = a.lse != nullptr ? a.ls[0] : 0;
  p.lse_sh = a.lse != nullptr ? a.ls[1] : 0;
  p.wait.timeout_ns = wait_timeout_ns();
  p.wait.status = s.status_ptr;

  const int G = s.max_clusters;
  const uint64_t need = static_cast<uint64_t>(2 * G) * llmfa::kSlotBytes;
  spec.nclusters =
      llmfa::make_plan(p, G, a.ws != nullptr && a.ws_bytes >= need && aligned16(a.ws));
  spec.combine = false;
  spec.cp = llmfa::CombineParams{};
  if (p.sk_mode) {
    p.ws_ml = reinterpret_cast<float*>(static_cast<char*>(const_cast<void*>(a.ws)) +
                                       static_cast<uint64_t>(2 * G) * llmfa::kSlotOBytes);
    // the O parts of all slots as one [2G * 512, 128] bf16 matrix
    const int64_t ws_rows = int64_t(2 * G) * llmfa::kSlotRows;
    const int64_t ws_strides[3] = {ws_rows * 128, 128, 128};
    if ((rc = encode_bshd(&spec.tw, a.ws, ws_strides, ws_rows, 1, 1, llmfa::kBlockM)) != LLMFA_OK)
      return rc;
    llmfa::CombineParams& cp = spec.cp;
    cp.ws_o = static_cast<const uint16_t*>(a.ws);
    cp.ws_ml = p.ws_ml;
    cp.o = static_cast<uint16_t*>(const_cast<void*>(a.o));
    cp.o_sb = a.os[0];
    cp.o_ss = a.os[1];
    cp.o_sh = a.os[2];
    cp.lse = p.lse;
    cp.lse_sb = p.lse_sb;
    cp.lse_sh = p.lse_sh;
    cp.wait = p.wait;
    cp.H = p.H;
    cp.Sq = p.Sq;
    cp.n_qblk = p.n_qblk;
    cp.n_split = list_split_units(p, &cp);
    spec.combine = cp.n_split > 0;
  } else {
    spec.tw = spec.to;  // not read without split units
  }
  return LLMFA_OK;
}

int launch_spec(const LaunchSpec& spec, cudaStream_t st) {
  const dim3 grid(2 * spec.nclusters, 1, 1), block(llmfa::kThreads, 1, 1);
  if (spec.p.lse != nullptr)
    llmfa::llm_fa_kernel_sm100<true><<<grid, block, llmfa::kSmemBytes, st>>>(
        spec.tq, spec.tk, spec.tv, spec.to, spec.tw, spec.p);
  else
    llmfa::llm_fa_kernel_sm100<false><<<grid, block, llmfa::kSmemBytes, st>>>(
        spec.tq, spec.tk, spec.tv, spec.to, spec.tw, spec.p);
  if (cudaGetLastError() != cudaSuccess) return LLMFA_ERR_LAUNCH;
  if (spec.combine) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(spec.cp.n_split * llmfa::kCombineBlocksPerUnit);
    cfg.blockDim = dim3(llmfa::kCombineThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(spec.cp.round_pieces) * llmfa::kCombinePieceBytes;
    cfg.stream = st;
    // Programmatic dependent launch: the combine grid is scheduled while the
    // attention kernel's last CTAs finish and waits (griddepcontrol.wait)
    // for that kernel's completion before reading the partial results.
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, llmfa::llm_fa_combine_kernel, spec.cp) != cudaSuccess) {
      cudaGetLastError();
      return LLMFA_ERR_LAUNCH;
    }
  }
  return LLMFA_OK;
}

}  // namespace

extern "C" {

int llmfa_forward_lse(const void* q, const int64_t q_strides[3], const void* k,
                      const int64_t k_strides[3], const void* v, const int64_t v_strides[3],
                      void* o, const int64_t o_strides[3], float* lse,
                      const int64_t lse_strides[2], int64_t batch, int64_t heads, int64_t seq_q,
                      int64_t seq_k, float softmax_scale, void* workspace,
                      uint64_t workspace_bytes, void* stream) {
  // ---- argument checks (no CUDA call before they pass)
  int rc = check_forward_args(q, q_strides, k, k_strides, v, v_strides, o, o_strides, lse,
                              lse_strides, batch, heads, seq_q, seq_k, softmax_scale);
  if (rc != LLMFA_OK) return rc;
  int dev = 0;
  DeviceSetup* s = nullptr;
  if ((rc = device_setup(&dev, &s)) != LLMFA_OK) return rc;

  // Tensor maps and launch plan depend only on the arguments: repeated calls
  // with the same buffers and sizes reuse them (LaunchCache).
  LaunchKey key;
  std::memset(&key, 0, sizeof(key));  // padding too: keys compare bytewise
  key.q = q; key.k = k; key.v = v; key.o = o; key.lse = lse; key.ws = workspace;
  for (int i = 0; i < 3; ++i) {
    key.qs[i] = q_strides[i]; key.ks[i] = k_strides[i];
    key.vs[i] = v_strides[i]; key.os[i] = o_strides[i];
  }
  if (lse != nullptr) { key.ls[0] = lse_strides[0]; key.ls[1] = lse_strides[1]; }
  key.batch = batch; key.heads = heads; key.seq_q = seq_q; key.seq_k = seq_k;
  std::memcpy(&key.scale_bits, &softmax_scale, sizeof(float));
  key.ws_bytes = workspace_bytes;

  LaunchSpec spec;
  if (!g_cache[dev].lookup(key, spec)) {
    if ((rc = make_launch_spec(key, *s, spec)) != LLMFA_OK) return rc;
    g_cache[dev].insert(key, spec);
  }
  spec.p.wait.timeout_ns = wait_timeout_ns();  // may change between calls
  spec.cp.wait = spec.p.wait;
  return launch_spec(spec, static_cast<cudaStream_t>(stream));
}

int llmfa_forward_2d(const void* q, const void* k, const void* v, void* o, int64_t seq_q,
                     int64_t seq_k, void* workspace, uint64_t workspace_bytes, void* stream) {
  const int64_t sq[3] = {seq_q * 128, 128, 128};
  const int64_t sk[3] = {seq_k * 128, 128, 128};
  return llmfa_forward(q, sq, k, sk, v, sk, o, sq, 1, 1, seq_q, seq_k,
                       1.0f / std::sqrt(128.0f), workspace, workspace_bytes, stream);
}

int llmfa_device_status(int* out_status, void* stream) {
  if (out_status == nullptr) return LLMFA_ERR_INVALID_ARGUMENT;
  int dev = 0;
  DeviceSetup* s = nullptr;
  int rc = device_setup(&dev, &s);
  if (rc != LLMFA_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(out_status, s->status_ptr, sizeof(int), cudaMemcpyDeviceToHost, st) !=
          cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess) {
    cudaGetLastError();
    return LLMFA_ERR_CUDA;
  }
  return LLMFA_OK;
}

int llmfa_reset_device_status(void* stream) {
  int dev = 0;
  DeviceSetup* s = nullptr;
  int rc = device_setup(&dev, &s);
  if (rc != LLMFA_OK) return rc;
  if (cudaMemsetAsync(s->status_ptr, 0, sizeof(int), static_cast<cudaStream_t>(stream)) !=
      cudaSuccess) {
    cudaGetLastError();
    return LLMFA_ERR_CUDA;
  }
  return LLMFA_OK;
}

int llmfa_launch_plan(int64_t batch, int64_t heads, int64_t seq_q, int64_t seq_k,
                      uint64_t workspace_bytes, int* kernels, int* clusters, int* split_units) {
  if (kernels == nullptr || clusters == nullptr || split_units == nullptr || batch < 1 ||
      heads < 1 || seq_q < 1 || seq_k < 1)
    return LLMFA_ERR_INVALID_ARGUMENT;
  int dev = 0;
  DeviceSetup* s = nullptr;
  int rc = device_setup(&dev, &s);
  if (rc != LLMFA_OK) return rc;
  const int64_t n_qblk = (seq_q + llmfa::kUnitRows - 1) / llmfa::kUnitRows;
  const int n_units = static_cast<int>(batch * heads * n_qblk);
  const int n_kv = static_cast<int>((seq_k + llmfa::kBlockN - 1) / llmfa::kBlockN);
  const int G = s->max_clusters;
  llmfa::FwdParams p{};
  p.n_units = n_units;
  p.n_kv = n_kv;
  const int nclusters =
      llmfa::make_plan(p, G, workspace_bytes >= static_cast<uint64_t>(2 * G) * llmfa::kSlotBytes);
  const int n_split = p.sk_mode ? list_split_units(p, nullptr) : 0;
  *kernels = n_split > 0 ? 2 : 1;
  *clusters = nclusters;
  *split_units = n_split;
  return LLMFA_OK;
}

int llmfa_max_active_clusters(int* out_clusters) {
  if (out_clusters == nullptr) return LLMFA_ERR_INVALID_ARGUMENT;
  int dev = 0;
  DeviceSetup* s = nullptr;
  int rc = device_setup(&dev, &s);
  if (rc != LLMFA_OK) return rc;
  *out_clusters = s->max_clusters;
  return LLMFA_OK;
}

int llmfa_trace_read(void* dst_host, uint64_t capacity_bytes, uint64_t* written_bytes) {
  if (dst_host == nullptr || written_bytes == nullptr) return LLMFA_ERR_INVALID_ARGUMENT;
  *written_bytes = 0;
#if LLMFA_TRACE
  const uint64_t bytes = sizeof(llmfa::TraceRecord) * llmfa::kTraceRecords;
  const uint64_t seg_bytes = sizeof(llmfa::g_seg_trace);
  if (capacity_bytes < bytes) return LLMFA_ERR_INVALID_ARGUMENT;
  if (cudaDeviceSynchronize() != cudaSuccess ||
      cudaMemcpyFromSymbol(dst_host, llmfa::g_trace, bytes) != cudaSuccess) {
    cudaGetLastError();
    return LLMFA_ERR_CUDA;
  }
  *written_bytes = bytes;
  if (capacity_bytes >= bytes + seg_bytes) {  // followed by the segment timeline
    if (cudaMemcpyFromSymbol(static_cast<char*>(dst_host) + bytes, llmfa::g_seg_trace,
                             seg_bytes) != cudaSuccess) {
      cudaGetLastError();
      return LLMFA_ERR_CUDA;
    }
    *written_bytes = bytes + seg_bytes;
    const uint64_t wait_bytes = sizeof(llmfa::g_wait_stats);
    if (capacity_bytes >= bytes + seg_bytes + wait_bytes) {  // then the wait-site statistics
      static const unsigned long long zeros[2 * llmfa::kWaitSlots] = {};
      if (cudaMemcpyFromSymbol(static_cast<char*>(dst_host) + bytes + seg_bytes,
                               llmfa::g_wait_stats, wait_bytes) != cudaSuccess ||
          cudaMemcpyToSymbol(llmfa::g_wait_stats, zeros, wait_bytes) != cudaSuccess) {
        cudaGetLastError();
        return LLMFA_ERR_CUDA;
      }
      *written_bytes = bytes + seg_bytes + wait_bytes;
    }
  }
  return LLMFA_OK;
#else
  (void)capacity_bytes;
  return LLMFA_ERR_UNSUPPORTED;
#endif
}

int llmfa_selftest_wait_timeout(uint32_t timeout_us, void* stream) {
  if (timeout_us == 0 || timeout_us > 10000000u) return LLMFA_ERR_INVALID_ARGUMENT;
  int dev = 0;
  DeviceSetup* s = nullptr;
  int rc = device_setup(&dev, &s);
  if (rc != LLMFA_OK) return rc;
  llmfa_wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<unsigned long long>(timeout_us) * 1000ull, s->status_ptr);
  if (cudaGetLastError() != cudaSuccess) return LLMFA_ERR_LAUNCH;
  return LLMFA_OK;
}

}  // extern "C"

// ---------------------------------------------------------------- allocation-free entry point
// For callers that cannot allocate device memory themselves: a foreign-language
// host (Go, Java, Rust over FFI) that was handed device pointers but has no
// CUDA allocator of its own, or a serving framework that pre-plans every byte
// of device memory at start-up and forbids allocations on the request path.
// They get the split-KV scratch from this fixed array instead of a workspace
// argument. It is sized for one 148-SM B200 (two partial-result slots per
// 2-SM cluster, 74 clusters): 148 x 135,168 bytes = 20.0 MB, held by every
// GPU that loads this library until the process exits.
namespace {

constexpr int kStaticScratchSlots = 148;
static __device__ __align__(256) float g_static_scratch[kStaticScratchSlots * llmfa::kSlotBytes / 4];

struct StaticScratch {
  std::once_flag once;
  int err = LLMFA_OK;
  float* ptr = nullptr;  // device address of g_static_scratch on this device
};
StaticScratch g_static_scratch_dev[kMaxDevices];

}  // namespace

extern "C" int llmfa_forward_static_scratch(const void* q, const int64_t q_strides[3], const void* k,
                                            const int64_t k_strides[3], const void* v,
                                            const int64_t v_strides[3], void* o,
                                            const int64_t o_strides[3], int64_t batch,
                                            int64_t heads, int64_t seq_q, int64_t seq_k,
                                            float softmax_scale, void* stream) {
  // The same checks as llmfa_forward, before any CUDA call (the symbol lookup
  // below loads the module and its 20 MB array).
  const int arg_rc = check_forward_args(q, q_strides, k, k_strides, v, v_strides, o, o_strides,
                                        nullptr, nullptr, batch, heads, seq_q, seq_k,
                                        softmax_scale);
  if (arg_rc != LLMFA_OK) return arg_rc;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return LLMFA_ERR_CUDA;
  }
  // Once per device, with that device current: the host-side name of the
  // array is not a device address, so look the address up and keep it.
  StaticScratch& ss = g_static_scratch_dev[dev];
  std::call_once(ss.once, [&] {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_static_scratch) != cudaSuccess || ptr == nullptr) {
      cudaGetLastError();
      ss.err = LLMFA_ERR_CUDA;
      return;
    }
    ss.ptr = static_cast<float*>(ptr);
  });
  if (ss.err != LLMFA_OK) return ss.err;
  // The split needs two slots per cluster of this device; refuse rather than
  // overrun the fixed array on a GPU with more SMs than it was sized for.
  uint64_t need = 0;
  const int rc = llmfa_workspace_size(&need);
  if (rc != LLMFA_OK) return rc;
  if (need > sizeof(g_static_scratch)) return LLMFA_ERR_UNSUPPORTED;
  // Nothing in the scratch needs to start at zero: every slot the combine
  // kernel reads is written by the attention kernel earlier in the same call.
  return llmfa_forward(q, q_strides, k, k_strides, v, v_strides, o, o_strides, batch, heads, seq_q,
                       seq_k, softmax_scale, ss.ptr, sizeof(g_static_scratch), stream);
}
