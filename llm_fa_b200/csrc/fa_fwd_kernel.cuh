// Warp-specialised FlashAttention forward for sm_100a (B200):
// BF16 Q/K/V, head_dim 128, non-causal, BF16 O, FP32 softmax state.
//
// Replaces the reference kernel `llm_fa_kernel` (llm_fa.cu:589-1413) and keeps
// its computation: O = softmax(Q K^T * scale) V with an online (streaming)
// softmax over 128-key tiles, P rounded to bf16 before the PV product, lazy
// rescaling of the O accumulator only when the running row maximum grows by
// more than kRescaleThreshold (log2 units; the reference uses the same 8.0,
// llm_fa.cu:857-866), and a final division by the row sum
// (llm_fa.cu:1348-1406). One deliberate difference: the row sum of each KV
// tile also takes the bf16 rounding of the tile's largest probability, the
// weight P V uses for it (the reference sums the fp32 probabilities only,
// llm_fa.cu:1019-1031); see dominant_rounding.
//
// Work unit: 512 query rows of one (batch, head), processed by a cluster of
// two CTAs (a CTA pair). The pair issues tcgen05 MMAs with cta_group::2 and
// M = 256: CTA rank r owns query rows [r*128, r*128+128) of each 256-row
// "Q tile"; every CTA holds two Q tiles (tile 0, tile 1) that take turns on
// the tensor core while the other tile's softmax runs.
//
//   S_t = Q_t K_j^T   (SS MMA 256x128x128; B = K_j, 64 keys from each CTA)
//   P_t = exp2(S_t * scale*log2e - m_t)  (bf16, written over S_t in TMEM)
//   O_t += P_t V_j    (TS MMA; A = P_t from TMEM, B = V_j, 64 dims per CTA)
//
// Tensor memory (512 columns x 128 lanes per CTA):
//   S_0 [0,128)  S_1 [128,256)  O_0 [256,384)  O_1 [384,512); P_t = S_t[0,64).
//
// Warp roles (16 warps, 512 threads):
//   0-3  softmax, tile 0          4-7  softmax, tile 1
//   8-11 correction (O rescale, exponentials of keys 96-127) + epilogue (x 1/l, bf16, TMA store)
//   12   MMA issue (leader CTA, whole warp, one elected lane issues) + TMEM allocation
//   13   TMA producer             14-15 idle
//
// The pair is persistent: cluster c processes units c, c + nclusters, ... in
// (batch, head, query-block) order, so concurrently resident clusters share
// K/V tiles in L2; with a workspace, and where the planner's cost model
// (make_plan) says it pays, the last partial wave of units is cut into KV
// ranges across all clusters (stream-K, SegIter) and merged by
// llm_fa_combine_kernel.
//
// No wait in this kernel is unbounded: every hand-off is an mbarrier, every
// mbarrier wait gives up after `timeout_ns`, records the wait site in the
// device status word, raises a CTA-wide abort flag, and every role then runs
// to the common teardown (drain MMAs, cluster barrier, TMEM dealloc). No
// cluster-multicast form of any instruction is used.
#pragma once
#include <cuda.h>

#include <cstdint>

#include "ptx.cuh"
#include "softmax_exp2.cuh"

namespace llmfa {

constexpr int kHeadDim = 128;
constexpr int kBlockM = 128;  // query rows per CTA per Q tile
constexpr int kQTiles = 2;    // Q tiles per CTA (ping-pong)
constexpr int kPair = 2;      // CTAs per cluster (cta_group::2)
constexpr int kUnitRows = kBlockM * kPair * kQTiles;  // 512 query rows per unit
constexpr int kBlockN = 128;  // keys per KV tile
constexpr int kStages = 6;    // K/V ring stages (K and V alternate)
constexpr int kThreads = 512;

constexpr uint32_t kQTileBytes = kBlockM * kHeadDim * 2;            // 32 KB
constexpr uint32_t kKVStageBytes = kBlockN * kHeadDim * 2 / kPair;  // 16 KB
constexpr uint32_t kOStageBytes = kBlockM * kHeadDim * 2;           // 32 KB
constexpr uint32_t kPanelBytes = kBlockM * 128;                     // 128 rows x 128 B

constexpr uint32_t kSmemQ = 0;
constexpr uint32_t kSmemKV = kSmemQ + kQTiles * kQTileBytes;    // 64 KB
constexpr uint32_t kSmemO = kSmemKV + kStages * kKVStageBytes;  // 160 KB
constexpr uint32_t kSmemBar = kSmemO + kOStageBytes;            // 192 KB

// mbarrier indices (8 B each)
constexpr int kBarQFull = 0;                        // [2] leader: both CTAs' Q tile landed
constexpr int kBarQEmpty = kBarQFull + 2;           // [2] each: last QK of the unit done
constexpr int kBarKVFull = kBarQEmpty + 2;          // [S] leader: both halves landed
constexpr int kBarKVEmpty = kBarKVFull + kStages;   // [S] each: MMAs done reading the stage
constexpr int kBarSFull = kBarKVEmpty + kStages;    // [2] each: S_t in TMEM
constexpr int kBarPHalf = kBarSFull + 2;            // [2] leader: P_t keys 0-63 written, O_t corrected
constexpr int kBarPFull = kBarPHalf + 2;            // [2] leader: P_t keys 64-127 written
constexpr int kBarOFull = kBarPFull + 2;            // [2] each: last PV of the unit done
constexpr int kBarStat = kBarOFull + 2;             // [2x4] softmax warp -> correction warp
constexpr int kBarLsum = kBarStat + 8;              // [2 parity][2x4] end-of-segment row sum/max
constexpr int kBarOStageFull = kBarLsum + 16;       // [1] 4 correction warps wrote staging
constexpr int kBarOStageEmpty = kBarOStageFull + 1; // [1] TMA store finished reading staging
constexpr int kBarDrain = kBarOStageEmpty + 1;      // [1] leader: teardown MMA drain
constexpr int kNumBars = kBarDrain + 1;

constexpr uint32_t kSmemScale = kSmemBar + 512;                 // float [2][128]
// End-of-segment row sum and row max, double-buffered by segment parity: the
// softmax of a one-tile segment can finish before the correction warps have
// read the previous segment's values (nothing orders a segment's QK after the
// previous epilogue), but never two segments ahead (the next segment's PV
// waits for that epilogue). float [parity][tile][128] each.
constexpr uint32_t kSmemLsum = kSmemScale + kQTiles * kBlockM * 4;
constexpr uint32_t kSmemMrow = kSmemLsum + 2 * kQTiles * kBlockM * 4;
// Row max the softmax used for this KV tile's P (the correction warp computes
// the exponentials of keys 96-127 with it). float [tile][128]
constexpr uint32_t kSmemMcur = kSmemMrow + 2 * kQTiles * kBlockM * 4;
constexpr uint32_t kSmemTmemSlot = kSmemMcur + kQTiles * kBlockM * 4;
constexpr uint32_t kSmemUsed = kSmemTmemSlot + 4;
constexpr uint32_t kSmemBytes = kSmemUsed + 1024;  // + base-alignment slack
static_assert(kNumBars * 8 <= 512, "barrier area");
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

// setmaxnreg split of the 65536 registers (launch: 512 threads x 128):
// 2 softmax warpgroups x 128 x 168 + correction 128 x 80 + control 128 x 96.
constexpr uint32_t kRegsSoftmax = 168;
constexpr uint32_t kRegsCorrection = 80;
constexpr uint32_t kRegsControl = 96;
static_assert(2 * 128 * kRegsSoftmax + 128 * kRegsCorrection + 128 * kRegsControl <= 65536,
              "register split exceeds the launch allocation");

constexpr float kRescaleThreshold = 8.0f;  // log2 units
// Pairs (bit k = columns 2k, 2k+1) of each 32-column chunk whose exp2 runs on
// the FMA pipe (softmax_exp2.cuh) instead of MUFU; the rest use ex2.approx.
// Default: pair 7 of each chunk (1/16 of the exponentials). Measured on B200
// against all-MUFU and against 1/8 and 1/4 offloads at several positions, in
// one process with interleaved runs: +4% (Sq=Sk=16384) and +5.6% (Sq=32768,
// Sk=131072) over all-MUFU; pair 7 is a further ~+0.8% over pair 15 since the
// correction warps took keys 96-127; larger fractions lose to the extra
// FMA-pipe issue.
#ifndef LLMFA_SOFTMAX_POLY_MASK
#define LLMFA_SOFTMAX_POLY_MASK 0x0080u
#endif
constexpr uint32_t kSoftmaxPolyMask = LLMFA_SOFTMAX_POLY_MASK;

// Ablation ladder (compile-time; 0 in the product build). Each rung removes one
// phase of the softmax so that its cost can be read off as a time difference,
// as the reference's ladder kernels do (scaffolding.cu with SKIP_SM_FULL: the
// TMA + MMA floor; faux.cu: no softmax math). The output of every rung other
// than 0 is not attention; llmfa_build_config reports the rung, and the bench
// refuses to time such a library as the product.
//   1 floor     softmax and correction warps only take part in the barrier
//               hand-offs (no TMEM loads or stores): TMA + MMA + epilogue
//   2 faux      P = bf16(S): scores loaded and stored back, no row max, no
//               scale, no exponentials, no row sums, no O rescale
//   3 noexp     the full softmax (row max, rescale, row sums) with exp2(x)
//               replaced by x: what the exponentials cost
#ifndef LLMFA_ABLATE
#define LLMFA_ABLATE 0
#endif
constexpr int kAblate = LLMFA_ABLATE;
static_assert(kAblate >= 0 && kAblate <= 3, "LLMFA_ABLATE must be 0..3");

// Device status word: 0 = ok; otherwise kStatusTimeoutBase + wait-site id.
constexpr int kStatusTimeoutBase = 0x1000;
enum WaitSite : int {
  kSiteProdQEmpty = 1,
  kSiteProdKVEmpty = 2,
  kSiteMmaQFull = 3,
  kSiteMmaKVFull = 4,
  kSiteMmaPFull = 5,
  kSiteSoftSFull = 6,
  kSiteCorrStat = 7,
  kSiteCorrLsum = 8,
  kSiteEpiOFull = 9,
  kSiteEpiStage = 10,
  kSiteDrain = 11,
  kSiteCombine = 12,
};

// ---------------------------------------------------------------- event trace
// Intra-kernel event trace, compiled out unless LLMFA_TRACE=1. Cluster 0
// records, for KV iterations [kTraceFirst, kTraceFirst + kTraceIters) of its
// first unit, the %globaltimer (ns) and %clock64 of each hand-off below, for
// both Q tiles, in both CTAs of the pair.
// Layout: [cta rank][Q tile][event][iteration].
#ifndef LLMFA_TRACE
#define LLMFA_TRACE 0
#endif
constexpr int kTraceFirst = 32;
constexpr int kTraceIters = 16;
enum TraceEvent : int {
  kEvSReady = 0,     // softmax: S_t(j) visible (after the s_full wait)
  kEvLdDone,         // softmax: 128 scores in registers
  kEvStat,           // softmax: rescale factor published
  kEvPHalf,          // softmax: P keys 0-63 published
  kEvPFull,          // softmax: P keys 64-127 published
  kEvMmaPHalf,       // MMA: saw P half (about to issue PV k-steps 0-3)
  kEvMmaPFull,       // MMA: saw P full (about to issue PV k-steps 4-7)
  kEvMmaQK,          // MMA: QK_t(j+1) issued and committed
  kEvCorrStat,       // correction: saw the rescale factor
  kEvCorrArrive,     // correction: arrived on P half
  kEvMmaKV,          // MMA: V_j ready (tile 0 slot) / K_{j+1} ready (tile 1 slot)
  kEvProdLoad,       // producer: V_j load issued (tile 0 slot) / K_{j+1} (tile 1 slot)
  kEvKVLanded,       // observer: V_j landed (tile 0 slot) / K_{j+1} landed (tile 1 slot)
  kEvMmaLoopTop,     // MMA: top of iteration j (tile 0) / QK_1(j+1) issued, not committed (tile 1)
  kEvCorrPFull,      // correction: arrived on P full (its keys 96-127 written)
  kNumTraceEvents
};
struct TraceRecord {
  unsigned long long globaltimer_ns;
  long long clock;
};
constexpr int kTraceRecords = 2 * kQTiles * kNumTraceEvents * kTraceIters;
#if LLMFA_TRACE
__device__ TraceRecord g_trace[kTraceRecords];
__device__ __forceinline__ void trace_event(int ev, int tile, int j, uint32_t rank, int cluster,
                                            int u) {
  if (cluster == 0 && u == 0 && j >= kTraceFirst && j < kTraceFirst + kTraceIters) {
    long long c;
    asm volatile("mov.u64 %0, %%clock64;" : "=l"(c));
    g_trace[((rank * kQTiles + tile) * kNumTraceEvents + ev) * kTraceIters + (j - kTraceFirst)] =
        TraceRecord{ptx::globaltimer_ns(), c};
  }
}
#define LLMFA_TRACE_EVENT(ev, tile, j) trace_event((ev), (tile), (j), rank, cluster, u)
// Segment timeline of every cluster (leader CTA): per segment, %globaltimer
// when the MMA warp issues its first QK, when the epilogue sees O complete
// (Q tile 0), when the epilogue has written Q tile 1, and u * 65536 + len.
constexpr int kSegTraceClusters = 160;
constexpr int kSegTraceSegs = 32;
__device__ unsigned long long g_seg_trace[kSegTraceClusters * kSegTraceSegs * 4];
__device__ __forceinline__ void seg_trace(int cluster, int seg, int field, unsigned long long v) {
  if (cluster < kSegTraceClusters && seg < kSegTraceSegs)
    g_seg_trace[(cluster * kSegTraceSegs + seg) * 4 + field] = v;
}
#define LLMFA_SEG_TRACE(seg, field, v) seg_trace(cluster, (seg), (field), (v))
#else
#define LLMFA_SEG_TRACE(seg, field, v) ((void)0)
#define LLMFA_TRACE_EVENT(ev, tile, j) ((void)0)
#endif

// Where a bounded wait reports a timeout and how long it waits (read only on
// the slow path, from the kernel's grid-constant parameters).
struct WaitCtl {
  int* status;
  unsigned long long timeout_ns;
};

// CTA-wide abort flag of the bounded waits (static shared memory: a constant
// address, so waits keep no register for it).
__shared__ uint32_t g_cta_abort;
__device__ __forceinline__ uint32_t cta_aborted() {
  return *static_cast<volatile uint32_t*>(&g_cta_abort);
}
__device__ __forceinline__ void cta_abort() { *static_cast<volatile uint32_t*>(&g_cta_abort) = 1u; }

constexpr int kMaxSkParts = 160;  // stream-K ranges (<= clusters of the grid)
constexpr int kCombineMaxUnits = 160;  // > clusters of any B200 grid (split units < clusters)
constexpr int kSegmentCost = 2;   // a segment switch costs about this many KV tiles

struct FwdParams {
  int B, H, Sq, Sk;
  int n_qblk;        // ceil(Sq / 512)
  int n_kv;          // ceil(Sk / 128)
  int n_units;       // B * H * n_qblk
  int kv_tail;       // valid keys in the last KV tile (1..128)
  float scale_log2;  // softmax_scale * log2(e)
  WaitCtl wait;      // device status word and wait limit
  // Work split (see SegIter): units [0, dp_units) round-robin over the
  // clusters; with sk_mode the remaining units' sk_total = units * n_kv
  // iterations are cut into sk_clusters contiguous ranges.
  int sk_mode;
  int dp_units;
  int sk_clusters;
  long long sk_total;
  long long sk_bound[kMaxSkParts + 1];  // range c = [sk_bound[c], sk_bound[c + 1])
  float* ws_ml;      // row max m and row sum l of every partial-result slot (sk_mode only)
  // Optional natural-log log-sum-exp of every query row's scaled scores,
  // lse[b * lse_sb + h * lse_sh + row] = log(sum_k exp(s_k * scale)); null = not written.
  float* lse;
  long long lse_sb, lse_sh;
};

// Partial-result slot of a unit split across clusters: the piece's O
// normalised by its own row sum (512 rows x 128, bf16, written by TMA like
// the final O), and its row max m (log2 units) and row sum l (fp32). A
// workspace holds the O parts of all slots first, as one [slots*512, 128]
// bf16 matrix, then [slots][m 512, l 512] fp32.
constexpr int kSlotRows = kUnitRows;
constexpr long long kSlotOBytes = static_cast<long long>(kSlotRows) * kHeadDim * 2;
constexpr long long kSlotMLFloats = 2 * kSlotRows;
constexpr long long kSlotBytes = kSlotOBytes + kSlotMLFloats * 4;

// Slow path of a bounded wait. With honor_abort, returns early once another
// role of this CTA has given up.
__device__ __forceinline__ bool mbar_wait_slow(uint32_t bar, uint32_t parity, const WaitCtl& c,
                                            int site, bool honor_abort) {
  const uint64_t t0 = ptx::globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0) {
      if (honor_abort && cta_aborted()) return false;
      if (ptx::globaltimer_ns() - t0 > c.timeout_ns) {
        cta_abort();
        atomicCAS(c.status, 0, kStatusTimeoutBase + site);
        return false;
      }
    }
  }
}
#if LLMFA_TRACE
// Per-wait-site statistics of the attention kernel (LLMFA_TRACE=2 builds): lane
// 0 of the waiting warp reads %clock before the wait's first probe and after
// it completes; a wait that took more than kWaitFast cycles (one whose phase
// had already completed returns within a few) adds its cycles and a count to
// its own warp's slot of the site (plain shared-memory updates: each warp owns
// its slots). The CTA's totals go to g_wait_stats at teardown; slot 0 holds
// the CTAs' own run time (cycles, CTA count).
constexpr int kWaitSlots = 16;
constexpr uint32_t kWaitFast = 64;
struct WaitSlot {
  unsigned long long cycles;
  unsigned long long count;
};
__device__ unsigned long long g_wait_stats[kWaitSlots * 2];
#if LLMFA_TRACE >= 2
__shared__ WaitSlot g_wait_slot[kThreads / 32][kWaitSlots];
#endif
#endif

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const WaitCtl& c,
                                          int site, bool honor_abort = true) {
#if LLMFA_TRACE >= 2
  if (site <= kSiteDrain) {  // the attention kernel's sites (its prologue clears the slots)
    const uint32_t t0 = static_cast<uint32_t>(clock());
    const bool ok = ptx::mbar_try_wait(bar, parity) ||
                    mbar_wait_slow(bar, parity, c, site, honor_abort);
    const uint32_t dt = static_cast<uint32_t>(clock()) - t0;
    if ((threadIdx.x & 31u) == 0 && dt > kWaitFast) {
      WaitSlot& w = g_wait_slot[threadIdx.x >> 5][site];
      w.cycles += dt;
      w.count += 1ull;
    }
    return ok;
  }
#endif
  if (ptx::mbar_try_wait(bar, parity)) return true;
  return mbar_wait_slow(bar, parity, c, site, honor_abort);
}

// Bounded wait executed by all 32 lanes of a warp; the result is
// warp-uniform so warp-collective instructions can follow it.
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity, const WaitCtl& c,
                                               int site) {
  const bool ok = mbar_wait(bar, parity, c, site);
  return __all_sync(0xffffffffu, ok);
}

struct UnitCoord {
  int b, h, row0;
};
__device__ __forceinline__ UnitCoord decode_unit(const FwdParams& p, int u) {
  const int bh = u / p.n_qblk;
  const int qb = u - bh * p.n_qblk;
  return {bh / p.H, bh % p.H, qb * kUnitRows};
}

// ---------------------------------------------------------------- work split
// Work is (unit, KV tile) iterations. Full waves of units go to the clusters
// round-robin (cluster c: units c, c + G, ...), the classic persistent
// schedule, which keeps concurrently running clusters on the same (batch,
// head) so K/V tiles are shared in L2. In stream-K mode the units of the
// last, partial wave are flattened into their units * n_kv iterations and cut
// into contiguous ranges, one per cluster, of equal cost (plan_sk_bounds);
// a unit cut across clusters is finished by llm_fa_combine_kernel from the
// partial results (normalised O, row max, row sum) of each piece.
struct Segment {
  int u;     // unit
  int j0;    // first KV tile
  int len;   // number of KV tiles
  int slot;  // partial-result slot, or -1 when this cluster computes the whole unit
};

__host__ __device__ __forceinline__ long long sk_begin(const FwdParams& p, int c) {
  return c >= p.sk_clusters ? p.sk_total : p.sk_bound[c];
}
// Cluster whose stream-K range holds iteration `it` (0 <= it < sk_total).
__host__ __device__ __forceinline__ int sk_owner(const FwdParams& p, long long it) {
  int lo = 0, hi = p.sk_clusters - 1;  // largest c with sk_bound[c] <= it
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.sk_bound[mid] <= it) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// Host planner of the stream-K ranges: cuts sk_total iterations into at most
// `parts` contiguous non-empty ranges. A range costs its KV tiles plus
// kSegmentCost for every unit boundary inside it (the pipeline drain and
// refill of a segment switch). Two cuts are compared by their largest range
// cost: equal lengths, and cut points where the cumulative cost
// F(pos) = pos + kSegmentCost * (unit boundaries before pos) reaches
// (c + 1) / parts of F(sk_total). Sets sk_clusters to the number of ranges.
inline long long sk_max_cost(const long long* b, int n, int n_kv) {
  long long worst = 0;
  for (int c = 0; c < n; ++c) {
    const long long inside = (b[c + 1] - 1) / n_kv - b[c] / n_kv;
    const long long cost = b[c + 1] - b[c] + static_cast<long long>(kSegmentCost) * inside;
    worst = cost > worst ? cost : worst;
  }
  return worst;
}
inline void plan_sk_bounds(FwdParams& p, int parts, int n_kv) {
  const long long T = p.sk_total;
  long long even[kMaxSkParts + 1], bal[kMaxSkParts + 1];
  for (int c = 0; c <= parts; ++c) even[c] = T * c / parts;
  // F takes the values u (n_kv + X) + 1 .. u (n_kv + X) + n_kv on unit u's
  // positions u n_kv + 1 .. u n_kv + n_kv (X = kSegmentCost) and skips the next
  // X values, so the smallest pos with F(pos) >= t has a closed form.
  const long long w = static_cast<long long>(n_kv) + kSegmentCost;
  auto F = [&](long long pos) -> long long {
    return pos + static_cast<long long>(kSegmentCost) * ((pos - 1) / n_kv);
  };
  auto F_inverse = [&](long long t) -> long long {
    const long long u = (t - 1) / w, r = t - u * w;
    return r <= n_kv ? u * n_kv + r : (u + 1) * n_kv + 1;
  };
  const long long FT = F(T);
  int used = 0;
  long long prev = 0;
  for (int c = 1; c <= parts && prev < T; ++c) {
    const long long target = (FT * c + parts - 1) / parts;  // ceil(FT * c / parts)
    long long pos = F_inverse(target);                      // smallest pos > prev with F(pos) >= target
    pos = pos > prev ? pos : prev + 1;
    bal[used++] = prev;
    prev = pos < T ? pos : T;
  }
  bal[used] = T;
  const bool use_bal = sk_max_cost(bal, used, n_kv) <= sk_max_cost(even, parts, n_kv);
  p.sk_clusters = use_bal ? used : parts;
  for (int c = 0; c <= kMaxSkParts; ++c)
    p.sk_bound[c] = c <= p.sk_clusters ? (use_bal ? bal[c] : even[c]) : T;
}

// Launch plan of one forward: classic persistent schedule, or stream-K over
// the last partial wave of units when a large enough workspace is given, the
// classic schedule would leave more than 2% of the clusters idle, and the
// KV-tile steps the cut saves the busiest cluster outweigh what the split
// costs. Cost model, fitted to 22 shapes timed both ways on B200 (it picks
// the faster schedule for all of them): a KV-tile step ~2 us; the split
// ~1 us plus ~0.15 us per cut unit (combine kernel, the pieces' epilogues).
// Fills the work-split fields of `p` (n_units, n_kv set) and returns the grid
// size in 2-CTA clusters.
inline int make_plan(FwdParams& p, int G, bool have_workspace) {
  p.sk_mode = 0;
  const int n_units = p.n_units;
  const int waves = (n_units + G - 1) / G;
  const double classic_eff = static_cast<double>(n_units) / (static_cast<double>(G) * waves);
  const int classic = n_units < G ? n_units : G;
  if (!have_workspace || classic_eff >= 0.98) return classic;
  const int dp_units = (n_units / G) * G;
  const long long sk_total = static_cast<long long>(n_units - dp_units) * p.n_kv;
  long long parts = sk_total / 4;  // at least 4 KV tiles per piece
  if (parts > G) parts = G;
  if (parts > kMaxSkParts) parts = kMaxSkParts;
  if (parts < 2 || n_units - dp_units > kCombineMaxUnits) return classic;
  // KV-tile steps of the busiest cluster: classic = waves x n_kv; stream-K =
  // the full waves, an even share of the cut iterations and a segment switch.
  const long long classic_steps = static_cast<long long>(waves) * p.n_kv;
  const long long sk_steps = static_cast<long long>(dp_units / G) * p.n_kv +
                             (sk_total + parts - 1) / parts + kSegmentCost;
  const double saved_us = 2.0 * static_cast<double>(classic_steps - sk_steps);
  const double split_us = 1.0 + 0.15 * static_cast<double>(n_units - dp_units);
  if (saved_us <= split_us) return classic;
  p.sk_mode = 1;
  p.dp_units = dp_units;
  p.sk_total = sk_total;
  plan_sk_bounds(p, static_cast<int>(parts), p.n_kv);
  if (p.sk_clusters < 2) {
    p.sk_mode = 0;
    return classic;
  }
  return dp_units > 0 ? G : p.sk_clusters;
}

struct SegIter {
  int c, G, k;
  long long it, end;
  bool first_sk;
  __host__ __device__ __forceinline__ SegIter(const FwdParams& p, int cluster, int nclusters)
      : c(cluster), G(nclusters), k(0), it(0), end(0), first_sk(true) {
    if (p.sk_mode) {
      const long long base = static_cast<long long>(p.dp_units) * p.n_kv;
      it = base + sk_begin(p, c);
      end = base + sk_begin(p, c + 1);
    }
  }
  __host__ __device__ __forceinline__ bool next(const FwdParams& p, Segment& s) {
    const int classic_units = p.sk_mode ? p.dp_units : p.n_units;
    const int uc = c + k * G;
    if (uc < classic_units) {
      s = Segment{uc, 0, p.n_kv, -1};
      ++k;
      return true;
    }
    if (!p.sk_mode || it >= end) return false;
    const int u = static_cast<int>(it / p.n_kv);
    const int j0 = static_cast<int>(it - static_cast<long long>(u) * p.n_kv);
    const long long rest = end - it;
    const int len = (p.n_kv - j0) < rest ? (p.n_kv - j0) : static_cast<int>(rest);
    const bool whole = (j0 == 0 && len == p.n_kv);
    s = Segment{u, j0, len, whole ? -1 : 2 * c + (first_sk ? 0 : 1)};
    it += len;
    first_sk = false;
    return true;
  }
  __host__ __device__ __forceinline__ bool has_next(const FwdParams& p) const {
    SegIter copy = *this;
    Segment s;
    return copy.next(p, s);
  }
};

// Maximum of 32 scores (raw bits) with independent 3-input max chains.
__device__ __forceinline__ float chunk_max(const uint32_t (&r)[32]) {
  float a0 = ptx::fmax3(__uint_as_float(r[0]), __uint_as_float(r[1]), __uint_as_float(r[2]));
  float a1 = ptx::fmax3(__uint_as_float(r[3]), __uint_as_float(r[4]), __uint_as_float(r[5]));
#pragma unroll
  for (int k = 6; k < 30; k += 4) {
    a0 = ptx::fmax3(a0, __uint_as_float(r[k + 0]), __uint_as_float(r[k + 1]));
    a1 = ptx::fmax3(a1, __uint_as_float(r[k + 2]), __uint_as_float(r[k + 3]));
  }
  return ptx::fmax3(a0, a1, fmaxf(__uint_as_float(r[30]), __uint_as_float(r[31])));
}

// Scores of keys at or past the end of the sequence (last KV tile only) -> -inf.
__device__ __forceinline__ void mask_tail(uint32_t (&r)[32], int col0, int kv_tail) {
  if (kv_tail >= col0 + 32) return;
#pragma unroll
  for (int k = 0; k < 32; ++k)
    if (col0 + k >= kv_tail) r[k] = __float_as_uint(-INFINITY);
}

// 32 scores -> 16 bf16x2 probabilities stored to TMEM at `t_p`; adds the fp32
// probabilities to the running pair sum. (Ablation rungs: faux stores bf16(s)
// and sums nothing; noexp stores and sums x = s * scale*log2e - m.)
__device__ __forceinline__ void exp_chunk(const uint32_t (&r)[32], uint64_t c2, uint64_t neg_m2,
                                          uint64_t& lsum2, uint32_t t_p) {
  uint32_t pk[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    if constexpr (kAblate == 2) {
      pk[k] = ptx::bf16x2_pack(__uint_as_float(r[2 * k]), __uint_as_float(r[2 * k + 1]));
      continue;
    }
    const uint64_t x2 = ptx::f2_fma(
        ptx::f2_pack(__uint_as_float(r[2 * k]), __uint_as_float(r[2 * k + 1])), c2, neg_m2);
    uint64_t e2;
    if constexpr (kAblate == 3) e2 = x2;
    else e2 = ((kSoftmaxPolyMask >> k) & 1u) ? exp2_poly_x2(x2) : exp2_mufu_x2(x2);
    lsum2 = ptx::f2_add(lsum2, e2);
    float e0, e1;
    ptx::f2_unpack(e2, e0, e1);
    pk[k] = ptx::bf16x2_pack(e0, e1);
  }
  ptx::tmem_st16(t_p, pk);
}

// Whether a score equal to the row maximum `smax` sits in one of the columns
// whose exp2 runs on the FMA pipe (kSoftmaxPolyMask) in this 32-column chunk.
__device__ __forceinline__ bool max_in_poly_columns(const uint32_t (&r)[32], float smax) {
  bool hit = false;
#pragma unroll
  for (int k = 0; k < 16; ++k)
    if ((kSoftmaxPolyMask >> k) & 1u)
      hit |= (__uint_as_float(r[2 * k]) == smax) | (__uint_as_float(r[2 * k + 1]) == smax);
  return hit;
}

// bf16(p) - p for the tile's largest probability p = exp2(smax * scale*log2e - m),
// computed exactly as exp_chunk computes that element (same fma, and the FMA-pipe
// exp2 when the maximum sits in one of its columns). Added to the fp32 row sum it
// makes the sum use the weight P V uses for the row's dominant key, so that a row
// dominated by one key returns that key's V row without the key's bf16 rounding
// error (up to 2^-9 relative, which bounds the max-abs error at logit ranges of
// +-200); the other keys' rounding errors average out. Costs a few instructions
// per row and tile instead of rounding every probability a second time.
__device__ __forceinline__ float dominant_rounding(float smax, float scale_log2, float m,
                                                   bool in_poly) {
  const float x = fmaf(smax, scale_log2, -m);
  float pm;
  if constexpr (kAblate == 3) {
    pm = x;
  } else {
    float p0, p1;
    ptx::f2_unpack(exp2_poly_x2(ptx::f2_pack(x, x)), p0, p1);
    pm = in_poly ? p0 : ptx::ex2_mufu(x);
  }
  return __uint_as_float(ptx::bf16x2_pack(pm, 0.f) << 16) - pm;
}

// kWithLse: also write the per-row log-sum-exp (FwdParams::lse). A separate
// instantiation, so the plain forward's code is not touched by it (the
// correction warps' register allocation moved the plain path by ~3%).
template <bool kWithLse>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    llm_fa_kernel_sm100(const __grid_constant__ CUtensorMap tmQ,
                        const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV,
                        const __grid_constant__ CUtensorMap tmO,
                        const __grid_constant__ CUtensorMap tmW,
                        const __grid_constant__ FwdParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t smem_base = (ptx::smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* smem_gen = smem_raw + (smem_base - ptx::smem_u32(smem_raw));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = ptx::cluster_ctarank();
  const bool leader = (rank == 0);
  const int cluster = static_cast<int>(ptx::cluster_id_x());
  const int nclusters = static_cast<int>(ptx::ncluster_x());

  auto bar = [&](int idx) -> uint32_t { return smem_base + kSmemBar + 8u * idx; };
  float* sm_scale = reinterpret_cast<float*>(smem_gen + kSmemScale);
  float* sm_lsum = reinterpret_cast<float*>(smem_gen + kSmemLsum);
  float* sm_mrow = reinterpret_cast<float*>(smem_gen + kSmemMrow);
  float* sm_mcur = reinterpret_cast<float*>(smem_gen + kSmemMcur);
  const WaitCtl& wc = p.wait;

  // ------------------------------------------------------------ prologue
  if (warp == 0 && lane == 0) {
    for (int t = 0; t < 2; ++t) {
      ptx::mbar_init(bar(kBarQFull + t), 1);
      ptx::mbar_init(bar(kBarQEmpty + t), 1);
      ptx::mbar_init(bar(kBarSFull + t), 1);
      ptx::mbar_init(bar(kBarPHalf + t), 16);  // 4 softmax + 4 correction warps x 2 CTAs
      ptx::mbar_init(bar(kBarPFull + t), 16);  // 4 softmax + 4 correction warps x 2 CTAs
      ptx::mbar_init(bar(kBarOFull + t), 1);
    }
    for (int s = 0; s < kStages; ++s) {
      ptx::mbar_init(bar(kBarKVFull + s), 1);
      ptx::mbar_init(bar(kBarKVEmpty + s), 1);
    }
    for (int k = 0; k < 8; ++k) {
      ptx::mbar_init(bar(kBarStat + k), 1);
      ptx::mbar_init(bar(kBarLsum + k), 1);
      ptx::mbar_init(bar(kBarLsum + 8 + k), 1);
    }
    ptx::mbar_init(bar(kBarOStageFull), 4);
    ptx::mbar_init(bar(kBarOStageEmpty), 1);
    ptx::mbar_init(bar(kBarDrain), 1);
    g_cta_abort = 0u;
    ptx::fence_mbar_init();
  }
#if LLMFA_TRACE >= 2
  const long long cta_t0 = clock64();
  if (threadIdx.x < (kThreads / 32) * kWaitSlots)
    (&g_wait_slot[0][0])[threadIdx.x] = WaitSlot{0ull, 0ull};
#endif
  if (warp == 12) {
    ptx::tmem_alloc<2>(smem_base + kSmemTmemSlot, 512);
    ptx::tmem_relinquish<2>();
  }
  if (warp == 13 && lane == 0) {
    ptx::prefetch_tmap(&tmQ);
    ptx::prefetch_tmap(&tmK);
    ptx::prefetch_tmap(&tmV);
    ptx::prefetch_tmap(&tmO);
    if (p.sk_mode) ptx::prefetch_tmap(&tmW);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::cluster_sync();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(smem_gen + kSmemTmemSlot);

  const int n = p.n_kv;  // KV tiles per unit (a segment may cover fewer)

  if (warp < 8) {
    // ========================================================== softmax
    ptx::setmaxnreg_inc<kRegsSoftmax>();
    const int tile = warp >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t t_s = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + tile * 128;
    const uint32_t phalf_leader = ptx::mapa(bar(kBarPHalf + tile), 0);
    const uint32_t pfull_leader = ptx::mapa(bar(kBarPFull + tile), 0);
    const uint32_t stat_bar = bar(kBarStat + tile * 4 + quarter);
    uint32_t seg_parity = 0;  // selects the row sum/max buffer and barrier of this segment
    const uint64_t c2 = ptx::f2_pack(p.scale_log2, p.scale_log2);
    uint32_t s_phase = 0;
    bool ok = true;
    SegIter si(p, cluster, nclusters);
    Segment sg;
    while (ok && si.next(p, sg)) {
      const int u = sg.u;
      float m = 0.f, l = 0.f;
      for (int j = 0; j < sg.len; ++j) {
        const bool last_tile = (sg.j0 + j == n - 1);
        if (!mbar_wait_warp(bar(kBarSFull + tile), s_phase, wc, kSiteSoftSFull)) {
          ok = false;
          break;
        }
        s_phase ^= 1u;
        if (quarter == 0 && lane == 0) LLMFA_TRACE_EVENT(kEvSReady, tile, j);
        if constexpr (kAblate == 1) {  // floor: the hand-offs only
          if (lane == 0) {
            ptx::mbar_arrive(stat_bar);
            ptx::mbar_arrive_cluster(phalf_leader);
            ptx::mbar_arrive_cluster(pfull_leader);
          }
          continue;
        }
        ptx::tc_fence_after();
        // Pass 1: all 128 scores -> row max. Chunks 0-1 stay in registers;
        // chunks 2-3 (columns 64-127, never overwritten by P) are re-read from
        // TMEM in pass 2 behind the exponentials of chunks 0-1, which keeps
        // the live set small enough for the softmax register budget.
        uint32_t s0[32], s1[32];
        float mt, smax;
        bool max_poly = false;
        {
          uint32_t s2[32], s3[32];
          ptx::tmem_ld32(t_s + 0, s0);
          ptx::tmem_ld32(t_s + 32, s1);
          ptx::tmem_ld32(t_s + 64, s2);
          ptx::tmem_ld32(t_s + 96, s3);
          ptx::tmem_wait_ld();
          ptx::reg_fence32(s0);
          ptx::reg_fence32(s1);
          ptx::reg_fence32(s2);
          ptx::reg_fence32(s3);
          if (quarter == 0 && lane == 0) LLMFA_TRACE_EVENT(kEvLdDone, tile, j);
          if (last_tile) {
            mask_tail(s0, 0, p.kv_tail);
            mask_tail(s1, 32, p.kv_tail);
            mask_tail(s2, 64, p.kv_tail);
            mask_tail(s3, 96, p.kv_tail);
          }
          if constexpr (kAblate == 2) {  // faux: no row max
            smax = 0.f;
            mt = 0.f;
          } else {
            smax = fmaxf(fmaxf(chunk_max(s0), chunk_max(s1)), fmaxf(chunk_max(s2), chunk_max(s3)));
            mt = smax * p.scale_log2;
            max_poly = max_in_poly_columns(s0, smax) | max_in_poly_columns(s1, smax) |
                       max_in_poly_columns(s2, smax) | max_in_poly_columns(s3, smax);
          }
        }
        float sc = 1.f;
        if (j == 0) {
          m = mt;
        } else if (mt > m + kRescaleThreshold) {
          sc = ptx::ex2_mufu(m - mt);
          m = mt;
          l *= sc;
        }
        // rescale factor (for O and the correction warp's row sum) and the max
        // used for this tile's P, for the correction warp
        sm_scale[tile * kBlockM + row] = sc;
        sm_mcur[tile * kBlockM + row] = m;
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(stat_bar);
        if (quarter == 0 && lane == 0) LLMFA_TRACE_EVENT(kEvStat, tile, j);
        // Pass 2: P = exp2(s * scale*log2e - m) -> bf16 -> TMEM columns [0, 64),
        // published in two halves so the first four PV k-steps (keys 0-63)
        // overlap the exponentials of keys 64-127. This warp computes keys
        // 0-95; the correction warp on the same scheduler computes keys 96-127
        // in parallel (its own MUFU instructions fill this warp's gaps) and
        // keeps their row sum.
        const uint64_t neg_m2 = ptx::f2_pack(-m, -m);
        uint64_t lsum_a = ptx::f2_pack(0.f, 0.f), lsum_b = lsum_a;
        {
          uint32_t s2[32];
          ptx::tmem_ld32(t_s + 64, s2);
          exp_chunk(s0, c2, neg_m2, lsum_a, t_s + 0);
          exp_chunk(s1, c2, neg_m2, lsum_b, t_s + 16);
          ptx::tmem_wait_st();
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive_cluster(phalf_leader);
          if (quarter == 0 && lane == 0) LLMFA_TRACE_EVENT(kEvPHalf, tile, j);
          ptx::tmem_wait_ld();
          ptx::reg_fence32(s2);
          if (last_tile) mask_tail(s2, 64, p.kv_tail);
          exp_chunk(s2, c2, neg_m2, lsum_a, t_s + 32);
        }
        float l0, l1;
        ptx::f2_unpack(ptx::f2_add(lsum_a, lsum_b), l0, l1);
        if constexpr (kAblate == 2)
          l += l0 + l1;
        else
          l += l0 + l1 + dominant_rounding(smax, p.scale_log2, m, max_poly);
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive_cluster(pfull_leader);
        if (quarter == 0 && lane == 0) LLMFA_TRACE_EVENT(kEvPFull, tile, j);
      }
      if (!ok) break;
      (void)u;
      sm_lsum[(seg_parity * kQTiles + tile) * kBlockM + row] = l;
      sm_mrow[(seg_parity * kQTiles + tile) * kBlockM + row] = m;
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar(kBarLsum + seg_parity * 8 + tile * 4 + quarter));
      seg_parity ^= 1u;
    }
    if (!ok) cta_abort();
    // every role returns to the launch register count before the shared teardown
    ptx::setmaxnreg_dec<128>();
  } else if (warp < 12) {
    // ========================================================== correction + epilogue
    ptx::setmaxnreg_dec<kRegsCorrection>();
    const int quarter = warp - 8;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t sO = smem_base + kSmemO;
    uint32_t stat_phase = 0;  // bit t: phase parity of the tile-t stat barrier
    uint32_t seg_count = 0, o_phase = 0, stage_phase = 0;
    const uint64_t c2 = ptx::f2_pack(p.scale_log2, p.scale_log2);
    float lc0 = 0.f, lc1 = 0.f;  // row sums of keys 96-127 (this warp's exponentials), per tile
    bool ok = true;
    bool first = true;
    SegIter si(p, cluster, nclusters);
    Segment sg;
    while (ok && si.next(p, sg)) {
      const int u = sg.u;
      const UnitCoord uc = decode_unit(p, u);
      if (first) {
        // j = 0 needs no correction: O_t is overwritten by the unit's first PV.
        if (lane == 0) {
          ptx::mbar_arrive_cluster(ptx::mapa(bar(kBarPHalf + 0), 0));
          ptx::mbar_arrive_cluster(ptx::mapa(bar(kBarPHalf + 1), 0));
        }
        __syncwarp();
        first = false;
      }
      for (int j = 0; j < sg.len && ok; ++j) {
        const bool last_tile = (sg.j0 + j == p.n_kv - 1);
#pragma unroll 1
        for (int tile = 0; tile < 2; ++tile) {
          if (!mbar_wait_warp(bar(kBarStat + tile * 4 + quarter), (stat_phase >> tile) & 1u, wc,
                              kSiteCorrStat)) {
            ok = false;
            break;
          }
          stat_phase ^= 1u << tile;
          if (warp == 8 && lane == 0) LLMFA_TRACE_EVENT(kEvCorrStat, tile, j);
          if constexpr (kAblate == 1) {  // floor: the hand-offs only
            if (lane == 0) {
              if (j > 0) ptx::mbar_arrive_cluster(ptx::mapa(bar(kBarPHalf + tile), 0));
              ptx::mbar_arrive_cluster(ptx::mapa(bar(kBarPFull + tile), 0));
            }
            continue;
          }
          const float sc = sm_scale[tile * kBlockM + row];
          const float mcur = sm_mcur[tile * kBlockM + row];
          if (j > 0 && __any_sync(0xffffffffu, sc != 1.f)) {
            // O_t is quiescent here: PV_t(j-1) completed before S_t(j) was
            // signalled, and PV_t(j) waits for this warp's arrival below.
            ptx::tc_fence_after();
            const uint32_t t_o = tmem_base + lane_off + 256 + tile * 128;
            const uint64_t sc2 = ptx::f2_pack(sc, sc);
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
              uint32_t r[32];
              ptx::tmem_ld32(t_o + 32 * c, r);
              ptx::tmem_wait_ld();
              ptx::reg_fence32(r);
#pragma unroll
              for (int k = 0; k < 32; k += 2) {
                uint64_t v = ptx::f2_pack(__uint_as_float(r[k]), __uint_as_float(r[k + 1]));
                v = ptx::f2_mul(v, sc2);
                r[k] = static_cast<uint32_t>(v);
                r[k + 1] = static_cast<uint32_t>(v >> 32);
              }
              ptx::tmem_st32(t_o + 32 * c, r);
            }
            ptx::tmem_wait_st();
          }
          if (j > 0) {  // (j = 0: arrived at the segment's start)
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive_cluster(ptx::mapa(bar(kBarPHalf + tile), 0));
            if (warp == 8 && lane == 0) LLMFA_TRACE_EVENT(kEvCorrArrive, tile, j);
          }
          // P for keys 96-127 of this tile (TMEM columns 48-63 of S_t; the
          // softmax warp wrote columns 0-47 and read every score before the
          // rescale factor was published).
          {
            ptx::tc_fence_after();
            const uint32_t t_s = tmem_base + lane_off + tile * 128;
            uint32_t r[32];
            ptx::tmem_ld32(t_s + 96, r);
            ptx::tmem_wait_ld();
            ptx::reg_fence32(r);
            if (last_tile) mask_tail(r, 96, p.kv_tail);
            uint64_t ls = ptx::f2_pack(0.f, 0.f);
            exp_chunk(r, c2, ptx::f2_pack(-mcur, -mcur), ls, t_s + 48);
            float a, b;
            ptx::f2_unpack(ls, a, b);
            if (tile == 0) lc0 = (j == 0 ? 0.f : lc0 * sc) + (a + b);
            else lc1 = (j == 0 ? 0.f : lc1 * sc) + (a + b);
            ptx::tmem_wait_st();
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive_cluster(ptx::mapa(bar(kBarPFull + tile), 0));
            if (warp == 8 && lane == 0) LLMFA_TRACE_EVENT(kEvCorrPFull, tile, j);
          }
        }
      }
      if (!ok) break;
      const bool has_next = si.has_next(p);
#pragma unroll 1
      for (int tile = 0; tile < 2; ++tile) {
        // buffer seg_count & 1, barrier phase (seg_count >> 1) & 1
        const uint32_t sp = seg_count & 1u;
        if (!mbar_wait_warp(bar(kBarLsum + sp * 8 + tile * 4 + quarter), (seg_count >> 1) & 1u, wc,
                            kSiteCorrLsum) ||
            !mbar_wait_warp(bar(kBarOFull + tile), o_phase, wc, kSiteEpiOFull) ||
            !mbar_wait_warp(bar(kBarOStageEmpty), stage_phase ^ 1u, wc, kSiteEpiStage)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        if (warp == 8 && lane == 0 && rank == 0 && tile == 0) {
          LLMFA_SEG_TRACE(static_cast<int>(seg_count), 1, ptx::globaltimer_ns());
          LLMFA_SEG_TRACE(static_cast<int>(seg_count), 3,
                          static_cast<unsigned long long>(u) * 65536ull + sg.len);
        }
        const uint32_t t_o = tmem_base + lane_off + 256 + tile * 128;
        // O / l in bf16 through the swizzled staging buffer and a TMA store: to
        // O for a whole unit, to the unit's partial-result slot (with m and l)
        // for a piece of a unit split across clusters (llm_fa_combine_kernel
        // merges the pieces).
        const float lsum = sm_lsum[(sp * kQTiles + tile) * kBlockM + row] + (tile == 0 ? lc0 : lc1);
        // (floor and faux rungs keep no row sum: no final division, as faux.cu)
        const float inv_l = (kAblate == 1 || kAblate == 2) ? 1.f : __frcp_rn(lsum);
        const int row_blk = tile * (kBlockM * kPair) + static_cast<int>(rank) * kBlockM;
        if (kWithLse && sg.slot < 0 && uc.row0 + row_blk + row < p.Sq) {
          // sum_k exp(s_k * scale) = 2^m * l with m in log2 units
          const float m2 = sm_mrow[(sp * kQTiles + tile) * kBlockM + row];
          p.lse[uc.b * p.lse_sb + uc.h * p.lse_sh + uc.row0 + row_blk + row] =
              (m2 + __log2f(lsum)) * 0.6931471805599453f;
        }
        if (sg.slot >= 0) {
          float* ml = p.ws_ml + static_cast<long long>(sg.slot) * kSlotMLFloats;
          ml[row_blk + row] = sm_mrow[(sp * kQTiles + tile) * kBlockM + row];
          ml[kSlotRows + row_blk + row] = lsum;
        }
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          ptx::tmem_ld32(t_o + 32 * c, r);
          ptx::tmem_wait_ld();
          ptx::reg_fence32(r);
          uint32_t pk[16];
#pragma unroll
          for (int k = 0; k < 16; ++k)
            pk[k] = ptx::bf16x2_pack(__uint_as_float(r[2 * k]) * inv_l,
                                     __uint_as_float(r[2 * k + 1]) * inv_l);
          // 128-byte-swizzled staging, the layout the SWIZZLE_128B TMA store reads.
          const uint32_t rowaddr = sO + (c >> 1) * kPanelBytes + row * 128;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t chunk = static_cast<uint32_t>(((c & 1) * 4 + q) ^ (row & 7));
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(rowaddr + chunk * 16),
                         "r"(pk[4 * q]), "r"(pk[4 * q + 1]), "r"(pk[4 * q + 2]),
                         "r"(pk[4 * q + 3])
                         : "memory");
          }
        }
        // O_t has been read: the next unit's first PV may overwrite it.
        ptx::tc_fence_before();
        ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (has_next) ptx::mbar_arrive_cluster(ptx::mapa(bar(kBarPHalf + tile), 0));
          ptx::mbar_arrive(bar(kBarOStageFull));
        }
        int stored = 1;
        if (warp == 8 && lane == 0) {
          stored = mbar_wait(bar(kBarOStageFull), stage_phase, wc, kSiteEpiStage) ? 1 : 0;
          if (stored) {
            const bool split = sg.slot >= 0;
            const CUtensorMap* tm = split ? &tmW : &tmO;
            const int srow = split ? sg.slot * kSlotRows + row_blk : uc.row0 + row_blk;
            const int sh = split ? 0 : uc.h, sb = split ? 0 : uc.b;
            ptx::tma_store_4d(tm, sO, 0, sh, srow, sb);
            ptx::tma_store_4d(tm, sO + kPanelBytes, 64, sh, srow, sb);
            ptx::bulk_commit_group();
            ptx::bulk_wait_group_read0();
            ptx::mbar_arrive(bar(kBarOStageEmpty));
          }
        }
        stored = __shfl_sync(0xffffffffu, stored, 0);
        stage_phase ^= 1u;
        if (!stored) {
          ok = false;
          break;
        }
      }
      if (warp == 8 && lane == 0 && rank == 0)
        LLMFA_SEG_TRACE(static_cast<int>(seg_count), 2, ptx::globaltimer_ns());
      ++seg_count;
      o_phase ^= 1u;
    }
    if (!ok) cta_abort();
    if (warp == 8 && lane == 0) ptx::bulk_wait_group0();
    __syncwarp();
    ptx::setmaxnreg_inc<128>();
  } else {
    ptx::setmaxnreg_dec<kRegsControl>();
    if (warp == 12 && leader) {
      // The whole warp runs this role; one elected lane issues each tcgen05
      // instruction (ptx::mma_*_warp), which keeps the issue path short.
      // ======================================================== MMA issue
      const uint32_t idesc_qk = ptx::idesc_bf16_f32(kBlockM * kPair, kBlockN, false, false);
      const uint32_t idesc_pv = ptx::idesc_bf16_f32(kBlockM * kPair, kHeadDim, false, true);
      // Barrier addresses in this CTA and, for the commits that signal both
      // CTAs, the same offsets in the peer CTA's window.
      const uint32_t bar_local = bar(0);
      const uint32_t bar_peer = ptx::mapa(bar_local, 1);
      auto commit_both = [&](uint32_t b) {
        ptx::mma_commit_warp(bar_local + 8u * b);
        ptx::mma_commit_warp(bar_peer + 8u * b);
      };
      // Descriptors: the high half (SBO 1024 B, version, 128-byte swizzle) is
      // shared; the low half advances by (byte offset >> 4) per K step and by
      // kKVStageBytes >> 4 per K/V stage.
      const uint32_t dhi = ptx::smem_desc_sw128_hi(1024);
      const uint32_t q_lo = ptx::smem_desc_lo(smem_base + kSmemQ, 16);
      const uint32_t k_lo = ptx::smem_desc_lo(smem_base + kSmemKV, 16);
      const uint32_t v_lo = ptx::smem_desc_lo(smem_base + kSmemKV, kKVStageBytes);
      auto qk = [&](int tile, uint32_t stage) {
        const uint32_t d = tmem_base + tile * 128;
        const uint32_t alo = q_lo + tile * (kQTileBytes >> 4);
        const uint32_t blo = k_lo + stage * (kKVStageBytes >> 4);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t aoff = ((kk >> 2) * kPanelBytes + (kk & 3) * 32) >> 4;
          const uint32_t boff = ((kk >> 2) * (kKVStageBytes / 2) + (kk & 3) * 32) >> 4;
          ptx::mma_ss_warp(d, ptx::make_desc(alo + aoff, dhi), ptx::make_desc(blo + boff, dhi),
                         idesc_qk, kk > 0 ? 1u : 0u);
        }
      };
      // PV k-steps [k0, k0+4): keys 16*k0 .. 16*k0+63 of the tile.
      auto pv_half = [&](int tile, uint32_t stage, bool acc, int k0) {
        const uint32_t d = tmem_base + 256 + tile * 128;
        const uint32_t pa = tmem_base + tile * 128;
        const uint32_t vlo = v_lo + stage * (kKVStageBytes >> 4);
#pragma unroll
        for (int kk = k0; kk < k0 + 4; ++kk) {
          ptx::mma_ts_warp(d, pa + kk * 8, ptx::make_desc(vlo + ((kk * 16 * 128) >> 4), dhi),
                         idesc_pv, (acc || kk > 0) ? 1u : 0u);
        }
      };
      // K/V ring: stages are consumed in load order (K_0, V_0, K_1, V_1, ...);
      // bit s of kv_par is the parity of the next kv_full phase of stage s.
      uint32_t kv_stage = 0, kv_par = 0;
      auto kv_take = [&](uint32_t& stage) -> bool {
        stage = kv_stage;
        kv_stage = (kv_stage + 1 == kStages) ? 0u : kv_stage + 1;
        const bool r = mbar_wait_warp(bar_local + 8u * (kBarKVFull + stage), (kv_par >> stage) & 1u, wc,
                                 kSiteMmaKVFull);
        kv_par ^= 1u << stage;
        return r;
      };
      uint32_t q_use = 0;
      uint32_t p_phase = 0;  // bit t: phase parity of tile t's P barriers
      bool ok = true;
      SegIter si(p, cluster, nclusters);
      Segment sg;
      // The thread blocks in tcgen05.mma while the tensor pipe's queue is
      // full, so work placed between two MMA groups is a pipe bubble unless
      // MMAs are still queued. Waits on data that landed long ago (K/V tiles)
      // are therefore taken before the preceding group is issued, and stage
      // releases are committed after the following group's first MMAs.
      while (ok && si.next(p, sg)) {
        const int n = sg.len;  // KV tiles of this segment
        const int u = sg.u;
        (void)u;
        uint32_t sk, sv;
        if (!mbar_wait_warp(bar_local + 8u * (kBarQFull + 0), q_use & 1u, wc, kSiteMmaQFull) ||
            !kv_take(sk)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        LLMFA_SEG_TRACE(static_cast<int>(q_use), 0, ptx::globaltimer_ns());
        qk(0, sk);
        commit_both(kBarSFull + 0);
        if (!mbar_wait_warp(bar_local + 8u * (kBarQFull + 1), q_use & 1u, wc, kSiteMmaQFull)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        qk(1, sk);
        commit_both(kBarSFull + 1);
        if (n == 1) {
          commit_both(kBarQEmpty + 0);
          commit_both(kBarQEmpty + 1);
        }
        if (!kv_take(sv)) {  // V_0
          ok = false;
          break;
        }
        uint32_t sv_prev = kStages;  // no V stage to release yet
        for (int j = 0; j < n; ++j) {
          const bool more = (j + 1 < n);
          LLMFA_TRACE_EVENT(kEvMmaLoopTop, 0, j);
          if (!mbar_wait_warp(bar_local + 8u * (kBarPHalf + 0), p_phase & 1u, wc, kSiteMmaPFull)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          LLMFA_TRACE_EVENT(kEvMmaPHalf, 0, j);
          pv_half(0, sv, j > 0, 0);
          // K_j (last read by QK_1(j)) and V_{j-1} (last read by PV_1(j-1)) are free.
          commit_both(kBarKVEmpty + sk);
          if (sv_prev < kStages) commit_both(kBarKVEmpty + sv_prev);
          if (!mbar_wait_warp(bar_local + 8u * (kBarPFull + 0), p_phase & 1u, wc, kSiteMmaPFull)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          LLMFA_TRACE_EVENT(kEvMmaPFull, 0, j);
          pv_half(0, sv, true, 4);
          p_phase ^= 1u;
          if (!more) commit_both(kBarOFull + 0);
          if (more) {
            if (!kv_take(sk)) {  // K_{j+1}
              ok = false;
              break;
            }
            LLMFA_TRACE_EVENT(kEvMmaKV, 1, j);
            ptx::tc_fence_after();
            qk(0, sk);
            commit_both(kBarSFull + 0);
            LLMFA_TRACE_EVENT(kEvMmaQK, 0, j);
            if (j + 2 == n) commit_both(kBarQEmpty + 0);
          }
          if (!mbar_wait_warp(bar_local + 8u * (kBarPHalf + 1), (p_phase >> 1) & 1u, wc, kSiteMmaPFull)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          LLMFA_TRACE_EVENT(kEvMmaPHalf, 1, j);
          pv_half(1, sv, j > 0, 0);
          if (!mbar_wait_warp(bar_local + 8u * (kBarPFull + 1), (p_phase >> 1) & 1u, wc, kSiteMmaPFull)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          LLMFA_TRACE_EVENT(kEvMmaPFull, 1, j);
          pv_half(1, sv, true, 4);
          p_phase ^= 2u;
          if (!more) {
            commit_both(kBarOFull + 1);
            commit_both(kBarKVEmpty + sv);  // V_{n-1}; K_{n-1} was released above
            break;
          }
          sv_prev = sv;
          if (!kv_take(sv)) {  // V_{j+1}
            ok = false;
            break;
          }
          LLMFA_TRACE_EVENT(kEvMmaKV, 0, j + 1);
          qk(1, sk);
          LLMFA_TRACE_EVENT(kEvMmaLoopTop, 1, j);
          commit_both(kBarSFull + 1);
          LLMFA_TRACE_EVENT(kEvMmaQK, 1, j);
          if (j + 2 == n) commit_both(kBarQEmpty + 1);
        }
        ++q_use;
      }
      if (!ok) cta_abort();
      // Drain: every MMA issued above completes before TMEM is released.
      ptx::mma_commit_warp(bar(kBarDrain));
      mbar_wait(bar(kBarDrain), 0, wc, kSiteDrain, /*honor_abort=*/false);
      __syncwarp();
    } else if (warp == 13 && lane == 0) {
      // ======================================================== TMA producer
      const uint64_t pol_q = ptx::policy_evict_first();
      const uint64_t pol_kv = ptx::policy_evict_last();
      uint32_t kv_t = 0, q_use = 0;
      bool ok = true;
      SegIter si(p, cluster, nclusters);
      Segment sg;
      while (ok && si.next(p, sg)) {
        const UnitCoord uc = decode_unit(p, sg.u);
        const int n = sg.len;
        const int j0 = sg.j0;
        auto load_q = [&](int tile) -> bool {
          if (!mbar_wait(bar(kBarQEmpty + tile), (q_use & 1u) ^ 1u, wc, kSiteProdQEmpty))
            return false;
          const uint32_t full = ptx::mapa(bar(kBarQFull + tile), 0);
          if (leader) ptx::mbar_arrive_expect_tx(bar(kBarQFull + tile), kPair * kQTileBytes);
          const int qrow = uc.row0 + tile * (kBlockM * kPair) + static_cast<int>(rank) * kBlockM;
          const uint32_t dst = smem_base + kSmemQ + tile * kQTileBytes;
          ptx::tma_load_4d<true>(dst, &tmQ, full, 0, uc.h, qrow, uc.b, pol_q);
          ptx::tma_load_4d<true>(dst + kPanelBytes, &tmQ, full, 64, uc.h, qrow, uc.b, pol_q);
          return true;
        };
        auto acquire = [&](uint32_t& stage, uint32_t& full) -> bool {
          const uint32_t t = kv_t++;
          stage = t % kStages;
          if (!mbar_wait(bar(kBarKVEmpty + stage), ((t / kStages) & 1u) ^ 1u, wc,
                         kSiteProdKVEmpty))
            return false;
          full = ptx::mapa(bar(kBarKVFull + stage), 0);
          if (leader) ptx::mbar_arrive_expect_tx(bar(kBarKVFull + stage), kPair * kKVStageBytes);
          return true;
        };
        auto load_k = [&](int j) -> bool {
          uint32_t stage, full;
          if (!acquire(stage, full)) return false;
          const uint32_t dst = smem_base + kSmemKV + stage * kKVStageBytes;
          const int krow = (j0 + j) * kBlockN + static_cast<int>(rank) * (kBlockN / kPair);
          ptx::tma_load_4d<true>(dst, &tmK, full, 0, uc.h, krow, uc.b, pol_kv);
          ptx::tma_load_4d<true>(dst + kKVStageBytes / 2, &tmK, full, 64, uc.h, krow, uc.b,
                                 pol_kv);
          return true;
        };
        auto load_v = [&](int j) -> bool {
          uint32_t stage, full;
          if (!acquire(stage, full)) return false;
          const uint32_t dst = smem_base + kSmemKV + stage * kKVStageBytes;
          ptx::tma_load_4d<true>(dst, &tmV, full, static_cast<int>(rank) * 64, uc.h,
                                 (j0 + j) * kBlockN, uc.b, pol_kv);
          return true;
        };
        ok = load_q(0) && load_k(0) && load_q(1);
        for (int j = 0; j < n && ok; ++j) {
          ok = load_v(j);
          const int u = sg.u;
          (void)u;
          LLMFA_TRACE_EVENT(kEvProdLoad, 0, j);
          if (ok && j + 1 < n) {
            ok = load_k(j + 1);
            LLMFA_TRACE_EVENT(kEvProdLoad, 1, j);
          }
        }
        ++q_use;
      }
      if (!ok) {
        cta_abort();
        // let copies already issued land before the CTA's shared memory is released
        const uint64_t t0 = ptx::globaltimer_ns();
        while (ptx::globaltimer_ns() - t0 < 20000ull) {
        }
      }
    }
#if LLMFA_TRACE
    else if (warp == 14 && lane == 0 && leader && cluster == 0) {
      // Trace-only observer: when the K/V stages of the traced window land.
      SegIter si(p, cluster, nclusters);
      Segment sg;
      if (si.next(p, sg)) {
        const int u = sg.u;
        const int jmax = min(sg.len, kTraceFirst + kTraceIters);
        for (int j = 0; j < jmax; ++j) {
          const uint32_t tv = 2 * j + 1, tk = 2 * j + 2;
          if (!mbar_wait(bar(kBarKVFull + tv % kStages), (tv / kStages) & 1u, wc, kSiteMmaKVFull))
            break;
          LLMFA_TRACE_EVENT(kEvKVLanded, 0, j);
          if (j + 1 < sg.len) {
            if (!mbar_wait(bar(kBarKVFull + tk % kStages), (tk / kStages) & 1u, wc, kSiteMmaKVFull))
              break;
            LLMFA_TRACE_EVENT(kEvKVLanded, 1, j);
          }
        }
      }
    }
#endif
    __syncwarp();
    ptx::setmaxnreg_inc<128>();
  }
  __syncwarp();

  // ------------------------------------------------------------ teardown
  // A programmatically dependent launch (the combine kernel) may be scheduled
  // once every CTA got here; it still waits for this grid to complete.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  ptx::tc_fence_before();
  __syncthreads();
#if LLMFA_TRACE >= 2
  if (threadIdx.x < kWaitSlots) {
    unsigned long long cyc = 0, cnt = 0;
    if (threadIdx.x == 0) {
      cyc = static_cast<unsigned long long>(clock64() - cta_t0);
      cnt = 1;
    } else {
      for (int w = 0; w < kThreads / 32; ++w) {
        cyc += g_wait_slot[w][threadIdx.x].cycles;
        cnt += g_wait_slot[w][threadIdx.x].count;
      }
    }
    atomicAdd(&g_wait_stats[2 * threadIdx.x], cyc);
    atomicAdd(&g_wait_stats[2 * threadIdx.x + 1], cnt);
  }
#endif
  ptx::cluster_sync();
  if (warp == 12) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc<2>(tmem_base, 512);
  }
}

// ---------------------------------------------------------------- combine
// Pieces of stream-K unit u: the clusters [c_lo, c_hi] whose ranges meet it.
// A piece's slot is 2c when the unit is the first segment of cluster c's
// range and 2c + 1 when it is the last (a range holds at most two partial
// segments); only c_lo's range can start before the unit.
struct UnitPieces {
  int c_lo, c_hi, slot_lo;
};
__host__ __device__ __forceinline__ UnitPieces unit_pieces(const FwdParams& p, int u) {
  const long long base = static_cast<long long>(p.dp_units) * p.n_kv;
  const long long it_lo = static_cast<long long>(u) * p.n_kv - base;
  UnitPieces r;
  r.c_lo = sk_owner(p, it_lo);
  r.c_hi = sk_owner(p, it_lo + p.n_kv - 1);
  r.slot_lo = 2 * r.c_lo + (sk_begin(p, r.c_lo) < it_lo ? 1 : 0);
  return r;
}
__host__ __device__ __forceinline__ int piece_slot(int c_lo, int slot_lo, int c) {
  return c == c_lo ? slot_lo : 2 * c;
}

// Finishes the units that stream-K mode cut across clusters: for every query
// row, O = sum_p w_p O_p / sum_p w_p with w_p = l_p 2^(m_p - m) over the
// pieces p (O_p normalised by l_p, m = max_p m_p), the standard merge of
// partial softmax states. The host lists the split units and their pieces.
// A CTA merges 32 rows of one unit: one thread issues bulk copies of those
// rows of every piece (8 KB of O plus m and l each, up to 8 pieces per round)
// into shared memory, so a CTA has all its bytes in flight at once; each of
// the 256 threads then merges 16 columns of one row. Pieces are folded in
// groups of four with a running maximum.
constexpr int kCombineRows = 32;       // query rows per CTA
constexpr int kCombineThreads = 256;   // 8 threads per row
constexpr int kCombineBlocksPerUnit = kUnitRows / kCombineRows;
constexpr uint32_t kCombineOBytes = kCombineRows * kHeadDim * 2;            // 8 KB
constexpr uint32_t kCombinePieceBytes = kCombineOBytes + 2 * kCombineRows * 4;  // + m, l
constexpr int kCombineMaxRound = 8;    // pieces per load round
struct CombineParams {
  const uint16_t* ws_o;         // [slots * 512, 128] bf16 normalised partial O
  const float* ws_ml;           // [slots][m 512, l 512]
  uint16_t* o;                  // bf16 output, [B, Sq, H, 128] element strides below
  long long o_sb, o_ss, o_sh;
  float* lse;                   // optional log-sum-exp output (see FwdParams)
  long long lse_sb, lse_sh;
  WaitCtl wait;
  int H, Sq, n_qblk, n_split;
  int round_pieces;             // pieces per load round: min(most pieces of a unit, 8)
  int unit[kCombineMaxUnits];   // split units
  short c_lo[kCombineMaxUnits], np[kCombineMaxUnits], slot_lo[kCombineMaxUnits];
};

__global__ void __launch_bounds__(kCombineThreads)
    llm_fa_combine_kernel(const __grid_constant__ CombineParams p) {
  extern __shared__ __align__(128) uint8_t cmb_smem[];
  __shared__ __align__(8) uint64_t cmb_bar;
  const uint32_t sbase = ptx::smem_u32(cmb_smem);
  const uint32_t bar = ptx::smem_u32(&cmb_bar);
  const int tid = static_cast<int>(threadIdx.x);
  if (tid == 0) {
    ptx::mbar_init(bar, 1);
    ptx::fence_mbar_init();
  }
  __syncthreads();
  // Launched as a programmatic dependent of the attention kernel: everything
  // before this wait overlaps that kernel's tail; nothing is read before it.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int i = static_cast<int>(blockIdx.x) / kCombineBlocksPerUnit;
  if (i >= p.n_split) return;
  const int row0 = (static_cast<int>(blockIdx.x) - i * kCombineBlocksPerUnit) * kCombineRows;
  const int u = p.unit[i];
  const int c_lo = p.c_lo[i], np = p.np[i], slot_lo = p.slot_lo[i];
  const int r = tid >> 3;        // row of this CTA's 32
  const int ca = tid & 7;        // 16-byte column chunks ca and ca + 8 (columns 8 ca.., 64 + 8 ca..)
  float m = -INFINITY, wsum = 0.f, acc[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) acc[e] = 0.f;
  uint32_t phase = 0;
  bool ok = true;
  for (int g0 = 0; g0 < np && ok; g0 += p.round_pieces) {
    const int n_here = np - g0 < p.round_pieces ? np - g0 : p.round_pieces;
    if (tid == 0) {
      ptx::mbar_arrive_expect_tx(bar, static_cast<uint32_t>(n_here) * kCombinePieceBytes);
      for (int k = 0; k < n_here; ++k) {
        const long long slot = piece_slot(c_lo, slot_lo, c_lo + g0 + k);
        const uint32_t dst = sbase + static_cast<uint32_t>(k) * kCombinePieceBytes;
        const float* ml = p.ws_ml + slot * kSlotMLFloats + row0;
        ptx::bulk_load(dst, p.ws_o + (slot * kSlotRows + row0) * kHeadDim, kCombineOBytes, bar);
        ptx::bulk_load(dst + kCombineOBytes, ml, kCombineRows * 4, bar);
        ptx::bulk_load(dst + kCombineOBytes + kCombineRows * 4, ml + kSlotRows, kCombineRows * 4,
                       bar);
      }
    }
    ok = mbar_wait(bar, phase, p.wait, kSiteCombine, false);
    phase ^= 1u;
    if (ok) {
      for (int g = 0; g < n_here; g += 4) {
        float pm[4], pl[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t pb = sbase + static_cast<uint32_t>(g + k) * kCombinePieceBytes + kCombineOBytes;
          const bool have = g + k < n_here;
          pm[k] = have ? ptx::ld_shared_f32(pb + r * 4) : -INFINITY;
          pl[k] = have ? ptx::ld_shared_f32(pb + (kCombineRows + r) * 4) : 0.f;
        }
        const float mn = fmaxf(fmaxf(m, fmaxf(pm[0], pm[1])), fmaxf(pm[2], pm[3]));
        const float sc = ptx::ex2_mufu(m - mn);  // 0 on the first group (m = -inf)
        wsum *= sc;
#pragma unroll
        for (int e = 0; e < 16; ++e) acc[e] *= sc;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (g + k >= n_here) break;
          const float w = pl[k] * ptx::ex2_mufu(pm[k] - mn);
          wsum += w;
          const uint32_t ob = sbase + static_cast<uint32_t>(g + k) * kCombinePieceBytes +
                              r * (kHeadDim * 2);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint4 v = ptx::ld_shared_v4(ob + (ca + 8 * h) * 16);
            const uint32_t x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              acc[8 * h + 2 * e] += w * __uint_as_float(x[e] << 16);
              acc[8 * h + 2 * e + 1] += w * __uint_as_float(x[e] & 0xFFFF0000u);
            }
          }
        }
        m = mn;
      }
    }
    ok = __syncthreads_and(ok) != 0;  // the round's shared memory has been read
  }
  if (!ok) return;
  const int bh = u / p.n_qblk;
  const int qb = u - bh * p.n_qblk;
  const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
  const int srow = qb * kUnitRows + row0 + r;
  if (srow >= p.Sq) return;
  const float inv = 1.f / wsum;
  uint16_t* orow = p.o + b * p.o_sb + srow * p.o_ss + h * p.o_sh;
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    uint4 pk;
    pk.x = ptx::bf16x2_pack(acc[8 * hh + 0] * inv, acc[8 * hh + 1] * inv);
    pk.y = ptx::bf16x2_pack(acc[8 * hh + 2] * inv, acc[8 * hh + 3] * inv);
    pk.z = ptx::bf16x2_pack(acc[8 * hh + 4] * inv, acc[8 * hh + 5] * inv);
    pk.w = ptx::bf16x2_pack(acc[8 * hh + 6] * inv, acc[8 * hh + 7] * inv);
    *reinterpret_cast<uint4*>(orow + (ca + 8 * hh) * 8) = pk;
  }
  if (p.lse != nullptr && ca == 0)  // sum = 2^m * sum_p w_p
    p.lse[b * p.lse_sb + h * p.lse_sh + srow] = (m + __log2f(wsum)) * 0.6931471805599453f;
}

}  // namespace llmfa
