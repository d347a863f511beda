/*
 * llm_fa_b200 — C ABI of the B200 (sm_100a) FlashAttention forward.
 *
 * Plain pointers and sizes only: no torch types cross this boundary. Every
 * entry point returns an llmfa status code (0 = success) and never aborts the
 * process. Compute entry points are asynchronous on the caller's stream and
 * allocate nothing; the caller owns every buffer.
 *
 * The reference exposes its path through one pybind function,
 *   std::vector<torch::Tensor> llm_fa_forward(Tensor Q, Tensor K, Tensor V)
 *   (llm_fa.cu:1418-1475, bound in llm_fa.py:37-54),
 * which checks shapes with TORCH_CHECK, encodes the TMA tensor maps, allocates
 * O, launches `llm_fa_kernel` on the legacy default stream and synchronises
 * the device. The functions below split that into an allocation-free launch
 * on an explicit stream plus status queries.
 */
#ifndef LLM_FA_B200_H_
#define LLM_FA_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define LLMFA_OK 0
#define LLMFA_ERR_INVALID_ARGUMENT 1 /* null pointer, non-positive size, bad scale */
#define LLMFA_ERR_UNSUPPORTED 2      /* alignment/stride outside what the TMA path accepts */
#define LLMFA_ERR_TENSOR_MAP 3       /* cuTensorMapEncodeTiled rejected a descriptor */
#define LLMFA_ERR_LAUNCH 4           /* kernel launch failed */
#define LLMFA_ERR_CUDA 5             /* other CUDA runtime/driver failure (no device, ...) */
#define LLMFA_ERR_DEVICE_TIMEOUT 6   /* a bounded in-kernel wait gave up (see llmfa_device_status) */

/*
 * O = softmax(Q K^T * softmax_scale) V for bf16 tensors with head dim 128,
 * non-causal, fp32 softmax state, bf16 output.
 *
 * Replaces llm_fa_forward (llm_fa.cu:1418-1475) and generalises its 2-D
 * (q,128)/(sk,128) inputs to the [B, S, H, 128] layout:
 *   q: [batch, seq_q, heads, 128]   k, v: [batch, seq_k, heads, 128]
 *   o: [batch, seq_q, heads, 128]   (written; may not alias q, k or v)
 * Each *_strides array holds the element strides of the (batch, seq, head)
 * dimensions; the head-dim stride must be 1. Base pointers must be 16-byte
 * aligned and strides multiples of 8 elements (16 bytes). Any seq_q >= 1 and
 * seq_k >= 1 are accepted (the reference requires q % 512 == 0,
 * sk % 128 == 0, sk >= 256; llm_fa.cu:1421-1428).
 * `workspace` (optional, 16-byte aligned, at least llmfa_workspace_size()
 * bytes; may be NULL) is scratch for the partial results of query blocks
 * whose KV range is split across SMs when there are too few blocks to fill
 * the GPU (two launches then: the attention kernel and a combine kernel).
 * Without it every query block is computed by one SM pair. Its contents
 * are not read across calls; calls that share a workspace must not overlap.
 * `stream` is a cudaStream_t (NULL = legacy default stream). No device
 * synchronisation; no allocation.
 */
int llmfa_forward(const void* q, const int64_t q_strides[3], const void* k,
                  const int64_t k_strides[3], const void* v, const int64_t v_strides[3], void* o,
                  const int64_t o_strides[3], int64_t batch, int64_t heads, int64_t seq_q,
                  int64_t seq_k, float softmax_scale, void* workspace, uint64_t workspace_bytes,
                  void* stream);

/*
 * llmfa_forward that also writes the natural-log log-sum-exp of every query
 * row's scaled scores, lse[b, h, s] = log(sum_k exp(q_s . k_k * softmax_scale)),
 * fp32, at lse + b * lse_strides[0] + h * lse_strides[1] + s (rows contiguous;
 * 4-byte aligned). This is the per-row softmax normaliser that split-KV merges
 * and a backward pass consume; for query blocks whose KV range is split it
 * comes from the combine step. lse = NULL behaves as llmfa_forward. No
 * counterpart in the reference (its launcher returns O only, llm_fa.cu:1475).
 */
int llmfa_forward_lse(const void* q, const int64_t q_strides[3], const void* k,
                      const int64_t k_strides[3], const void* v, const int64_t v_strides[3],
                      void* o, const int64_t o_strides[3], float* lse,
                      const int64_t lse_strides[2], int64_t batch, int64_t heads, int64_t seq_q,
                      int64_t seq_k, float softmax_scale, void* workspace,
                      uint64_t workspace_bytes, void* stream);

/* Workspace bytes that let llmfa_forward split KV ranges on the current
 * device (depends on the device's SM count only, not on the shapes). No
 * counterpart in the reference, which always launches one cluster per 512
 * query rows (llm_fa.cu:1465). */
int llmfa_workspace_size(uint64_t* bytes);

/*
 * The reference call shape exactly: contiguous row-major Q (seq_q,128),
 * K/V (seq_k,128), O (seq_q,128) bf16, softmax_scale = 1/sqrt(128)
 * (llm_fa.py:57-65, llm_fa.cu:1418-1475). Asynchronous; O (and the optional
 * workspace, as for llmfa_forward) must be allocated by the caller.
 */
int llmfa_forward_2d(const void* q, const void* k, const void* v, void* o, int64_t seq_q,
                     int64_t seq_k, void* workspace, uint64_t workspace_bytes, void* stream);

/* Reads (and keeps) the device status word of the current device after
 * synchronising `stream`: 0, or LLMFA_DEVICE_STATUS_TIMEOUT_BASE + wait-site
 * id when an in-kernel wait gave up. No counterpart in the reference, whose
 * waits are unbounded (llm_fa.cu:197-209). */
#define LLMFA_DEVICE_STATUS_TIMEOUT_BASE 0x1000
int llmfa_device_status(int* out_status, void* stream);
/* Clears the device status word of the current device (stream-ordered). */
int llmfa_reset_device_status(void* stream);

/* Upper bound, in milliseconds, on every in-kernel wait (default 2000;
 * environment variable LLMFA_WAIT_TIMEOUT_MS overrides the default). */
int llmfa_set_wait_timeout_ms(uint32_t ms);

/* Number of 2-CTA clusters of the attention kernel that can be resident at
 * once on the current device (the persistent grid size). */
int llmfa_max_active_clusters(int* out_clusters);

/* What llmfa_forward would launch for these sizes and this much workspace on
 * the current device: number of kernels (1, or 2 with the combine kernel),
 * grid size in 2-CTA clusters, and how many 512-row query blocks get their
 * KV range split. No counterpart in the reference. */
int llmfa_launch_plan(int64_t batch, int64_t heads, int64_t seq_q, int64_t seq_k,
                      uint64_t workspace_bytes, int* kernels, int* clusters, int* split_units);

/* Human-readable text for a status code. */
const char* llmfa_error_string(int status);

/* Library version (major*10000 + minor*100 + patch). */
int llmfa_version(void);

/*
 * Compile-time configuration of this library build: `*ablation` = the
 * ablation-ladder rung (0 = the product; 1 = TMA + MMA floor, 2 = no softmax
 * math, 3 = no exponentials: the output of rungs 1-3 is not attention) and
 * `*trace` = the event-trace level (0 = none; 1 = event trace and segment
 * timeline, -DLLMFA_TRACE=1; 2 = also per-wait-site statistics). Replaces
 * the reference's separate ladder kernels (scaffolding.cu with SKIP_SM_FULL,
 * faux.cu) and its ENABLE_PROF build flag (llm_fa.py:46-51), which it reports
 * nowhere at run time.
 */
int llmfa_build_config(int* ablation, int* trace);

/*
 * Event trace of the last launch (library built with -DLLMFA_TRACE=1 or 2
 * only; otherwise returns LLMFA_ERR_UNSUPPORTED): copies the trace records
 * ({uint64 globaltimer_ns, int64 clock64} per [cta rank][Q tile][event]
 * [iteration]) to host memory after synchronising the device, followed, when
 * `capacity_bytes` allows, by the per-cluster segment timeline (uint64
 * [160 clusters][32 segments][4]) and then by the per-wait-site statistics
 * of every launch since the last read (uint64 [16][2], all zero below level
 * 2: entry 0 = summed CTA run time in SM cycles and the CTA count; entry s =
 * the SM cycles that lane 0 of the waiting warps spent in those bounded waits
 * of site s that took more than 64 cycles, and their number), which the read
 * clears. Replaces the reference's
 * profiler ring flush (profiler.cuh:85-108) and the prof_buf / prof_count
 * outputs of llm_fa_forward (llm_fa.cu:1461-1474).
 */
int llmfa_trace_read(void* dst_host, uint64_t capacity_bytes, uint64_t* written_bytes);

/*
 * llmfa_forward without a workspace argument and without allocating: for
 * callers that cannot allocate device memory themselves (a foreign-language
 * host that only holds device pointers handed to it, or a framework that
 * plans all device memory up front and forbids allocation on the request
 * path). The split-KV scratch comes from a fixed 20.0 MB array inside this
 * library (148 partial-result slots: two per 2-SM cluster of a 148-SM B200),
 * which every GPU that loads the library keeps until the process exits.
 * Returns LLMFA_ERR_UNSUPPORTED on a device that would need more slots than
 * that (more than 74 two-SM clusters resident), for every shape, including
 * shapes that would not split any KV range. Arguments are checked as for
 * llmfa_forward before any CUDA call. The first call on each device looks up
 * the array's device address (cudaGetSymbolAddress, with that device
 * current); make that first call before any stream capture. All calls share the one array, so calls that
 * overlap on the GPU (other streams, other host threads) race on it and must
 * be serialised by the caller. The array's contents from the last call are
 * left in place; nothing in it has to start at zero. Other arguments and
 * results as for llmfa_forward. No counterpart in the reference.
 */
int llmfa_forward_static_scratch(const void* q, const int64_t q_strides[3], const void* k,
                                 const int64_t k_strides[3], const void* v,
                                 const int64_t v_strides[3], void* o, const int64_t o_strides[3],
                                 int64_t batch, int64_t heads, int64_t seq_q, int64_t seq_k,
                                 float softmax_scale, void* stream);

/*
 * Failure-detection self test: launches one CTA whose single mbarrier wait can
 * never complete (nothing arrives on it); the bounded wait gives up after
 * `timeout_us` microseconds and records LLMFA_DEVICE_STATUS_TIMEOUT_BASE +
 * 15 in the device status word. The GPU context stays usable. No counterpart
 * in the reference.
 */
int llmfa_selftest_wait_timeout(uint32_t timeout_us, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LLM_FA_B200_H_ */
