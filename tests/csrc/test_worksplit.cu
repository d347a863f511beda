// Host-side check of the work split used by the attention kernel (SegIter,
// sk_owner, unit_pieces, piece_slot from fa_fwd_kernel.cuh, compiled here as
// host code): for many (units, KV tiles, clusters) it checks that every
// (unit, KV tile) iteration is processed exactly once, that pieces of split
// units get distinct partial-result slots, and that the combine kernel's slot
// lookup finds exactly the pieces the kernel wrote. Prints "ok" and exits 0 on
// success.
#include <cstdio>
#include <map>
#include <set>
#include <vector>

#include "../../llm_fa_b200/csrc/fa_fwd_kernel.cuh"

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

int main() {
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
