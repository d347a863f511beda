// Host-side check of the work split used by the attention kernel (SegIter,
// sk_owner, unit_pieces, piece_slot from fa_fwd_kernel.cuh, compiled here as
// host code): for many (units, KV tiles, clusters) it checks that every
// (unit, KV tile) iteration is processed exactly once, that pieces of split
// units get distinct partial-result slots, and that the combine kernel's slot
// lookup finds exactly the pieces the kernel wrote. The planner's cut points
// are checked against a brute-force restatement (linear search over the
// cumulative cost). The launch planner's choice between the classic schedule
// and stream-K is checked against shapes timed both ways on a B200 (74
// clusters). Prints "ok" and exits 0 on success.
#include <cstdio>
#include <map>
#include <set>
#include <vector>

#include "../../llm_fa_b200/csrc/fa_fwd_kernel.cuh"

// Brute-force cut: range c starts at the smallest pos > start of range c - 1
// with F(pos) >= ceil(F(T) c / parts), F(pos) = pos + kSegmentCost *
// floor((pos - 1) / n_kv); the even cut is floor(T c / parts). The planner
// keeps the cut whose largest range cost is smaller (ties: balanced).
static std::vector<long long> brute_bounds(long long T, int parts, int n_kv) {
  auto F = [&](long long pos) -> long long {
    return pos <= 0 ? 0 : pos + llmfa::kSegmentCost * ((pos - 1) / n_kv);
  };
  auto max_cost = [&](const std::vector<long long>& b) {
    long long worst = 0;
    for (size_t c = 0; c + 1 < b.size(); ++c) {
      long long cost = 0;
      for (long long it = b[c]; it < b[c + 1]; ++it)
        cost += 1 + (it > b[c] && it % n_kv == 0 ? llmfa::kSegmentCost : 0);
      worst = cost > worst ? cost : worst;
    }
    return worst;
  };
  std::vector<long long> even(parts + 1), bal(1, 0);
  for (int c = 0; c <= parts; ++c) even[c] = T * c / parts;
  for (int c = 1; c <= parts && bal.back() < T; ++c) {
    const long long target = (F(T) * c + parts - 1) / parts;
    long long pos = bal.back() + 1;
    while (pos < T && F(pos) < target) ++pos;
    bal.push_back(pos);
  }
  bal.back() = T;
  return max_cost(bal) <= max_cost(even) ? bal : even;
}

static int check(int n_units, int n_kv, int G, bool sk) {
  llmfa::FwdParams p{};
  p.n_units = n_units;
  p.n_kv = n_kv;
  int grid = n_units < G ? n_units : G;
  if (sk) {
    const int dp = (n_units / G) * G;
    const long long total = static_cast<long long>(n_units - dp) * n_kv;
    long long parts = total / 4;
    if (parts > G) parts = G;
    if (parts < 2) return 0;  // the host would not choose stream-K
    p.sk_mode = 1;
    p.dp_units = dp;
    p.sk_total = total;
    llmfa::plan_sk_bounds(p, static_cast<int>(parts), n_kv);
    if (p.sk_clusters < 2 || p.sk_clusters > parts) return 9;
    for (int c = 0; c < p.sk_clusters; ++c)  // non-empty ranges
      if (p.sk_bound[c + 1] <= p.sk_bound[c] && c + 1 < p.sk_clusters) return 10;
    const std::vector<long long> b = brute_bounds(total, static_cast<int>(parts), n_kv);
    if (static_cast<int>(b.size()) != p.sk_clusters + 1) return 11;
    for (int c = 0; c <= p.sk_clusters; ++c)
      if (p.sk_bound[c] != b[c]) return 11;
    grid = dp > 0 ? G : p.sk_clusters;
  }
  std::vector<int> seen(static_cast<size_t>(n_units) * n_kv, 0);
  std::map<int, std::set<int>> written;  // unit -> slots written by the kernel
  std::set<int> slots;
  for (int c = 0; c < grid; ++c) {
    llmfa::SegIter it(p, c, grid);
    llmfa::Segment s;
    while (it.next(p, s)) {
      if (s.len <= 0 || s.j0 < 0 || s.j0 + s.len > n_kv) return 1;
      for (int j = s.j0; j < s.j0 + s.len; ++j) seen[static_cast<size_t>(s.u) * n_kv + j]++;
      const bool whole = (s.j0 == 0 && s.len == n_kv);
      if (whole != (s.slot < 0)) return 2;
      if (s.slot >= 0) {
        if (s.slot >= 2 * grid || !slots.insert(s.slot).second) return 3;
        written[s.u].insert(s.slot);
      }
    }
  }
  for (int v : seen)
    if (v != 1) return 4;
  if (sk) {
    const long long base = static_cast<long long>(p.dp_units) * n_kv;
    int n_split = 0;
    for (int u = p.dp_units; u < n_units; ++u) {
      const long long lo = static_cast<long long>(u) * n_kv - base;
      const llmfa::UnitPieces pc = llmfa::unit_pieces(p, u);
      if (pc.c_lo != llmfa::sk_owner(p, lo)) return 6;
      std::set<int> found;
      if (pc.c_lo != pc.c_hi) {
        ++n_split;
        for (int c = pc.c_lo; c <= pc.c_hi; ++c) found.insert(llmfa::piece_slot(pc.c_lo, pc.slot_lo, c));
      }
      if (found != written[u]) return 5;
      if (pc.c_hi - pc.c_lo + 1 > 32767 || pc.slot_lo > 32767) return 7;  // short fields of the table
    }
    if (n_split > llmfa::kCombineMaxUnits) return 8;
  }
  return 0;
}

// (B, H, Sq, Sk) and whether stream-K measured faster than the classic
// schedule on one B200 (CUDA events, L2 flushed, median of 10 calls each).
struct Timed {
  int B, H, Sq, Sk;
  bool sk_faster;
};
static const Timed kTimed[] = {
    {1, 2, 1024, 1024, true},    {1, 1, 2048, 2048, true},   {1, 1, 4096, 4096, true},
    {1, 2, 2048, 8192, true},    {1, 4, 4096, 2048, true},   {1, 8, 2048, 2048, true},
    {1, 16, 1024, 4096, true},   {2, 16, 2048, 2048, false}, {1, 1, 8192, 8192, true},
    {1, 1, 16384, 16384, true},  {2, 16, 2048, 4096, true},  {2, 16, 2048, 8192, true},
    {2, 16, 2048, 16384, true},  {1, 40, 2048, 2048, true},  {3, 16, 2048, 2048, true},
    {4, 16, 2048, 2048, true},   {1, 80, 1024, 1024, true},  {1, 100, 1024, 4096, true},
    {1, 50, 2048, 1024, false},  {1, 3, 1024, 1024, true},   {1, 6, 1024, 2048, true},
    {1, 1, 1024, 4096, true},
};

static int check_plan_choices() {
  for (const Timed& t : kTimed) {
    llmfa::FwdParams p{};
    p.n_units = t.B * t.H * ((t.Sq + llmfa::kUnitRows - 1) / llmfa::kUnitRows);
    p.n_kv = (t.Sk + llmfa::kBlockN - 1) / llmfa::kBlockN;
    llmfa::make_plan(p, 74, true);
    if ((p.sk_mode != 0) != t.sk_faster) {
      std::printf("FAIL plan B%d H%d %dx%d: stream-K %d, measured faster %d\n", t.B, t.H, t.Sq,
                  t.Sk, p.sk_mode, t.sk_faster ? 1 : 0);
      return 1;
    }
    llmfa::FwdParams q{};  // without a workspace: always classic
    q.n_units = p.n_units;
    q.n_kv = p.n_kv;
    llmfa::make_plan(q, 74, false);
    if (q.sk_mode) return 1;
  }
  return 0;
}

int main() {
  if (check_plan_choices()) return 1;
  int cases = 0;
  const int Gs[] = {1, 2, 3, 7, 74, 148};  // grids above kMaxSkParts are not planned
  for (int G : Gs)
    for (int n_units = 1; n_units <= 600; n_units += (n_units < 40 ? 1 : 37))
      for (int n_kv : {1, 2, 3, 5, 17, 64, 128, 1024})
        for (int sk = 0; sk < 2; ++sk) {
          const int rc = check(n_units, n_kv, G, sk != 0);
          if (rc) {
            std::printf("FAIL rc=%d units=%d n_kv=%d G=%d sk=%d\n", rc, n_units, n_kv, G, sk);
            return 1;
          }
          ++cases;
        }
  std::printf("ok %d cases\n", cases);
  return 0;
}
