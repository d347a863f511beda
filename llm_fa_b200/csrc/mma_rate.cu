// Tensor-core rate of the tcgen05.mma forms the attention kernel issues, measured
// in isolation: one warp per CTA (of the leader CTA of a pair for cta_group::2;
// one lane elected per instruction, as in the attention kernel) issues `n_mma`
// MMAs back to back on shared-memory / tensor-memory operands of
// the attention kernel's layouts, commits them to an mbarrier and waits; the
// SM clock (%clock64) before the first issue, after the last issue and after
// completion gives cycles per MMA and the issue rate.
//
//   form 0  QK:  SS  cta_group::2  M=256 N=128  A K-major, B K-major (SW128)
//   form 1  PV:  TS  cta_group::2  M=256 N=128  A from TMEM, B MN-major (SW128)
//   form 2       SS  cta_group::1  M=128 N=128
//   form 3       SS  cta_group::2  M=256 N=256
//   form 4       SS  cta_group::2  M=256 N=64
//   form 5       SS  cta_group::2  M=256 N=128  A K-major, B MN-major (PV's B layout)
//
// Every operand uses a layout the attention kernel itself uses (K-major SW128
// panels of up to 128 rows; one MN-major SW128 panel of 128 K rows per CTA).
// Operand contents are a fixed pattern of small bf16 values (the rate does not
// depend on them); every operand address stays inside the CTA's 64 KB operand
// area and 512 allocated TMEM columns. The completion wait gives up after one
// second and reports it. A measurement tool, built into its own library file
// (libllm_fa_b200_mmarate.so); the attention library does not contain it.
#include <cuda_runtime.h>

#include <cstdint>

#include "ptx.cuh"

namespace {

constexpr uint32_t kOperandBytes = 64 * 1024;  // A [0, 32K), B [32K, 64K)
constexpr uint32_t kSmemBytes = kOperandBytes + 1024 + 1024;
constexpr uint32_t kPanel = 128 * 128;          // 128 rows x 128 B (one SW128 panel)
constexpr uint64_t kTimeoutNs = 1000000000ull;  // 1 s

struct Form {
  int cg, m, n;
  bool a_tmem, b_mn;
};
__host__ __device__ constexpr Form form_of(int f) {
  return f == 0   ? Form{2, 256, 128, false, false}
         : f == 1 ? Form{2, 256, 128, true, true}
         : f == 2 ? Form{1, 128, 128, false, false}
         : f == 3 ? Form{2, 256, 256, false, false}
         : f == 4 ? Form{2, 256, 64, false, false}
                  : Form{2, 256, 128, false, true};
}

// Warp-converged issue: the whole warp executes the call and the lane that
// elect.sync picks issues the instruction (the attention kernel's issue form).
template <int CG>
__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                       uint32_t acc) {
  if constexpr (CG == 2)
    llmfa::ptx::mma_ss_warp(d, a, b, idesc, acc);
  else
    asm volatile(
        "{\n\t.reg .pred p, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void mma_ts2(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc,
                                        uint32_t acc) {
  llmfa::ptx::mma_ts_warp(d, a, b, idesc, acc);
}
template <int CG>
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  if constexpr (CG == 2)
    llmfa::ptx::mma_commit_warp(bar);
  else
    asm volatile(
        "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(
            bar)
        : "memory");
}

// out[4 * block + {0, 1, 2, 3}] = cycles from the first issue to completion, to the
// last issue, to the eighth issue, and 1 if the completion wait gave up (leader CTAs
// only; the other CTAs write zeros). The form is a template parameter and the eight
// K-step descriptors are computed before the clock starts, so the issue loop is as
// short as the attention kernel's unrolled MMA groups.
template <int FORM, bool kRuntimeLoop>
__global__ void __launch_bounds__(128, 1)
    mma_rate_kernel(int form_rt, int n_groups, unsigned long long* out) {
  constexpr Form f = form_of(FORM);
  constexpr int CG = f.cg;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t base = (llmfa::ptx::smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* gen = smem_raw + (base - llmfa::ptx::smem_u32(smem_raw));
  const uint32_t bar = base + kOperandBytes;
  const uint32_t slot = bar + 8;
  const int warp = threadIdx.x >> 5;
  const uint32_t rank = CG == 2 ? llmfa::ptx::cluster_ctarank() : 0u;

  // operands: small bf16 values (|x| < 1) in a fixed pattern
  for (uint32_t i = threadIdx.x; i < kOperandBytes / 4; i += blockDim.x) {
    const uint32_t h = (i * 2654435761u) >> 20;
    const uint32_t lo = 0x3C00u | (h & 0x7Fu), hi = 0xBC00u | ((h >> 7) & 0x7Fu);
    reinterpret_cast<uint32_t*>(gen)[i] = lo | (hi << 16);
  }
  if (warp == 0) {
    llmfa::ptx::tmem_alloc<CG>(slot, 512);
    llmfa::ptx::tmem_relinquish<CG>();
  }
  if (threadIdx.x == 32) {
    llmfa::ptx::mbar_init(bar, 1);
    llmfa::ptx::fence_mbar_init();
  }
  llmfa::ptx::fence_proxy_async_smem();  // operand stores -> tensor-core reads
  llmfa::ptx::tc_fence_before();
  __syncthreads();
  if constexpr (CG == 2) llmfa::ptx::cluster_sync();
  llmfa::ptx::tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(gen + kOperandBytes + 8);

  unsigned long long total = 0, issue = 0, first8 = 0, timed_out = 0;
  if (rank == 0 && warp == 0) {
    const uint32_t idesc = llmfa::ptx::idesc_bf16_f32(f.m, f.n, false, f.b_mn);
    const uint32_t hi = llmfa::ptx::smem_desc_sw128_hi(1024);
    const uint32_t a_lo = llmfa::ptx::smem_desc_lo(base, 16);
    // B: K-major (QK's K tile: 2 panels of N / cg rows) or MN-major (PV's V tile: one
    // 64-wide panel of 128 K rows per CTA, as in the attention kernel)
    const uint32_t b_lo = llmfa::ptx::smem_desc_lo(base + 32 * 1024, f.b_mn ? kPanel : 16);
    const uint32_t d = tmem;          // accumulator columns [0, N)
    const uint32_t a_t = tmem + 256;  // TS: A in columns [256, 320)
    uint64_t adesc[8], bdesc[8];
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {  // the 8 K-steps of a 128-deep tile
      const uint32_t a_off = ((kk >> 2) * kPanel + (kk & 3) * 32) >> 4;
      const uint32_t b_off = f.b_mn ? ((kk * 16 * 128) >> 4) : a_off;
      adesc[kk] = llmfa::ptx::make_desc(a_lo + a_off, hi);
      bdesc[kk] = llmfa::ptx::make_desc(b_lo + b_off, hi);
    }
    __syncwarp();
    const long long t0 = clock64();
    long long t8 = t0;
    if constexpr (kRuntimeLoop) {
      // a rolled loop that looks the form up at run time and builds both descriptors
      // for every MMA from the run-time K-step index
      const Form rf = form_of(form_rt);
      for (int i = 0; i < 8 * n_groups; ++i) {
        const int k = i & 7;
        const uint32_t acc = i > 0 ? 1u : 0u;
        const uint32_t a_off = ((k >> 2) * kPanel + (k & 3) * 32) >> 4;
        const uint32_t b_off = rf.b_mn ? ((k * 16 * 128) >> 4) : a_off;
        const uint64_t b = llmfa::ptx::make_desc(b_lo + b_off, hi);
        if (rf.a_tmem) {
          if constexpr (CG == 2) mma_ts2(d, a_t + k * 8, b, idesc, acc);
        } else {
          mma_ss<CG>(d, llmfa::ptx::make_desc(a_lo + a_off, hi), b, idesc, acc);
        }
        if (i == 7) t8 = clock64();
      }
    } else {
      for (int g = 0; g < n_groups; ++g) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t acc = (g | kk) != 0 ? 1u : 0u;
          if constexpr (f.a_tmem)
            mma_ts2(d, a_t + kk * 8, bdesc[kk], idesc, acc);
          else
            mma_ss<CG>(d, adesc[kk], bdesc[kk], idesc, acc);
        }
        if (g == 0) t8 = clock64();
      }
    }
    const long long t1 = clock64();
    mma_commit<CG>(bar);
    const uint64_t g0 = llmfa::ptx::globaltimer_ns();
    while (!llmfa::ptx::mbar_try_wait(bar, 0)) {
      if (llmfa::ptx::globaltimer_ns() - g0 > kTimeoutNs) {
        timed_out = 1;
        break;
      }
    }
    const long long t2 = clock64();
    total = static_cast<unsigned long long>(t2 - t0);
    issue = static_cast<unsigned long long>(t1 - t0);
    first8 = static_cast<unsigned long long>(t8 - t0);
  }
  if (threadIdx.x == 0) {
    out[4 * blockIdx.x + 0] = total;
    out[4 * blockIdx.x + 1] = issue;
    out[4 * blockIdx.x + 2] = first8;
    out[4 * blockIdx.x + 3] = timed_out;
  }
  llmfa::ptx::tc_fence_before();
  __syncthreads();
  if constexpr (CG == 2) llmfa::ptx::cluster_sync();
  if (warp == 0) {
    llmfa::ptx::tc_fence_after();
    llmfa::ptx::tmem_dealloc<CG>(tmem, 512);
  }
}

template <int FORM, bool kRuntimeLoop>
cudaError_t launch_form(int n_groups, int ctas, unsigned long long* out, cudaStream_t stream) {
  constexpr Form f = form_of(FORM);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3(ctas);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  if (f.cg == 2) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  cudaError_t e = cudaFuncSetAttribute(mma_rate_kernel<FORM, kRuntimeLoop>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e == cudaSuccess)
    e = cudaLaunchKernelEx(&cfg, mma_rate_kernel<FORM, kRuntimeLoop>, FORM, n_groups, out);
  return e;
}

}  // namespace

template <bool kRuntimeLoop>
cudaError_t launch(int form, int g, int ctas, unsigned long long* out, cudaStream_t stream) {
  switch (form) {
    case 0: return launch_form<0, kRuntimeLoop>(g, ctas, out, stream);
    case 1: return launch_form<1, kRuntimeLoop>(g, ctas, out, stream);
    case 2: return launch_form<2, kRuntimeLoop>(g, ctas, out, stream);
    case 3: return launch_form<3, kRuntimeLoop>(g, ctas, out, stream);
    case 4: return launch_form<4, kRuntimeLoop>(g, ctas, out, stream);
    default: return launch_form<5, kRuntimeLoop>(g, ctas, out, stream);
  }
}

// Runs `form` (0-5 above) with `n_mma` MMAs (a multiple of 8) per issuing CTA on `ctas`
// CTAs (an even number for the cta_group::2 forms: one pair per cluster). With
// `runtime_loop` nonzero the MMAs come from a rolled loop that selects the form and
// builds both descriptors at run time for every MMA (about ten more instructions per
// MMA on the issue path) instead of the unrolled groups with descriptors in registers.
// `out` is a device array of 4 * ctas unsigned 64-bit values. Returns a cudaError_t
// code (0 = launched).
extern "C" int llmfa_mma_rate(int form, int n_mma, int ctas, int runtime_loop,
                              unsigned long long* out, cudaStream_t stream) {
  if (form < 0 || form > 5 || n_mma < 8 || (n_mma & 7) || ctas < 1 || out == nullptr)
    return static_cast<int>(cudaErrorInvalidValue);
  if (form_of(form).cg == 2 && (ctas & 1)) return static_cast<int>(cudaErrorInvalidValue);
  const int g = n_mma / 8;
  const cudaError_t e = runtime_loop ? launch<true>(form, g, ctas, out, stream)
                                     : launch<false>(form, g, ctas, out, stream);
  return static_cast<int>(e);
}
