// akv_tree.cu — device replica of the shared radix tree and match_prefix.
//
// The host tree (SharedNode table, agentkv/core/radix_tree.py:82-103) is
// mirrored as flat arrays in HBM:
//   node_edge_off[id], node_edge_len[id] — each node's edge as a range of the
//       append-only token arena (an edge split only narrows ranges);
//   slots — every node's `children` dict (first edge token → child id) as one
//       open-addressing hash table keyed by (parent id, first token), 16 bytes
//       per slot {parent, token, child, child's edge length}, linear probing,
//       -1 = empty, -2 = deleted.
// The host applies every tree mutation to its mirror and ships the changed
// slots / node ranges as a delta (akv_tree_apply); new edge tokens are
// appended to the arena with a plain copy.
//
// match_prefix runs one warp per query and restates
// DualRadixTree._match_prefix_locked (radix_tree.py:513-570):
//   from the root, look up the child keyed by the next query token; compare
//   the child's edge with the query (__ballot_sync + __ffs find the first
//   mismatch); stop on a missing child, a mismatch anywhere in the edge or a
//   query that ends inside the edge (a partial edge earns no credit);
//   otherwise descend.  The match is floored to the block size; a zero match
//   reports (-1, 0).  The walk chases up to 32 hops ahead and verifies their
//   edges together (see k_match).
#include "akv_common.cuh"

namespace {

constexpr int kEmpty = -1;  // a deleted slot holds parent -2 and never matches
constexpr int kMatchWarpsPerCta = 4;
// Warps (queries) per CTA of the whole-query lookup, k_match.  A CTA's slot
// on the SM frees only when its last query ends, so fewer warps per CTA hand
// the SM to the next queries sooner; the register cap stays 20 warps per SM.
// One query per CTA: 0.0446 ms per 4,096-query batch on the match stress
// tree against 0.0585 ms with two and 0.0583 ms with four.
#ifndef AKV_MATCH_WHOLE_WARPS
#define AKV_MATCH_WHOLE_WARPS 1
#endif
constexpr int kWholeWarpsPerCta = AKV_MATCH_WHOLE_WARPS;
static_assert(20 % kWholeWarpsPerCta == 0, "k_match: warps per CTA must divide 20");

AKV_DEV uint32_t tree_hash(int32_t parent, int32_t token) {
  // MurmurHash3's 64-bit finalizer over (parent, token).
  uint64_t k = (static_cast<uint64_t>(static_cast<uint32_t>(parent)) << 32) |
               static_cast<uint64_t>(static_cast<uint32_t>(token));
  k ^= k >> 33;
  k *= 0xff51afd7ed558ccdull;
  k ^= k >> 33;
  k *= 0xc4ceb9fe1a85ec53ull;
  k ^= k >> 33;
  return static_cast<uint32_t>(k);
}

// Warp-cooperative lookup of (parent, token): each step reads kProbe
// consecutive slots (one 128-byte line), lane i the i-th; the first matching
// slot wins; an empty slot before any match ends the probe.  The table is at
// most half full, so a key almost always sits in the first line.  Returns the
// child id (or -1) and its edge length.
constexpr int kProbe = 8;

AKV_DEV int32_t warp_lookup(const int4* __restrict__ slots, int32_t mask, int32_t parent,
                            int32_t token, int lane, int32_t& child_len) {
  const uint32_t h = tree_hash(parent, token);
  const int32_t windows = (mask + 1) / kProbe + 1;
  for (int32_t w = 0; w < windows; ++w) {
    int4 s = make_int4(kEmpty + 1, 0, 0, 0);  // lanes >= kProbe hold a non-matching, non-empty slot
    if (lane < kProbe) {
      const uint32_t idx = (h + static_cast<uint32_t>(w) * kProbe + static_cast<uint32_t>(lane)) &
                           static_cast<uint32_t>(mask);
      s = __ldg(&slots[idx]);
    }
    const uint32_t hit = __ballot_sync(0xffffffffu, lane < kProbe && s.x == parent && s.y == token);
    const uint32_t empty = __ballot_sync(0xffffffffu, lane < kProbe && s.x == kEmpty);
    if (hit) {
      const int first_hit = __ffs(hit) - 1;
      const int first_empty = empty ? __ffs(empty) - 1 : 32;
      const int32_t c = __shfl_sync(0xffffffffu, s.z, first_hit);
      child_len = __shfl_sync(0xffffffffu, s.w, first_hit);
      return first_hit < first_empty ? c : -1;
    }
    if (empty) return -1;
  }
  return -1;
}

constexpr int kWinPerLane = 8;  // query tokens a lane keeps: a 256-token window per warp
constexpr int kSegment = 32;    // hops chased before their edges are verified (one per lane)

// Where the reference's walk over one query stops, as seen from one range of
// its token positions.  key = 2 * position + mismatch: the walk compares
// every position before `position`, plus the mismatching token when
// `mismatch` is 1, so the comparison count is position + mismatch.  The
// stops of one walk are ordered by key, so over several ranges of a query
// the smallest key is the reference's stop.  `matched` is the depth the walk
// credits before flooring (the start of the stopping edge, or the end of the
// last full edge) and `node` the node at that depth.
struct MatchStop {
  int64_t key;
  int64_t matched;
  int32_t node;
};
constexpr int64_t kNoStop = INT64_MAX;  // the range ends before the walk does

// The query's tokens around the chase's position, for the hash-probe hops:
// a 256-token window held in registers (8 per lane), reloaded when the
// position leaves it.  Positions are warp-uniform and < L.
struct QueryWindow {
  const int32_t* __restrict__ Q;
  int64_t L;
  int lane;
  int32_t win[kWinPerLane];
  int64_t wbase = -(1LL << 40);

  AKV_DEV QueryWindow(const int32_t* q, int64_t l, int ln) : Q(q), L(l), lane(ln) {}

  AKV_DEV int32_t operator()(int64_t pos) {
    if (pos < wbase || pos >= wbase + 32 * kWinPerLane) {
      wbase = pos;
#pragma unroll
      for (int u = 0; u < kWinPerLane; ++u) {
        const int64_t i = pos + u * 32 + lane;
        win[u] = i < L ? Q[i] : 0;
      }
    }
    const int64_t r = pos - wbase;
    const int u = static_cast<int>(r >> 5);
    int32_t v = 0;
#pragma unroll
    for (int uu = 0; uu < kWinPerLane; ++uu) v = (uu == u) ? win[uu] : v;
    return __shfl_sync(0xffffffffu, v, static_cast<int>(r & 31));
  }
};

// One segment of the chase phase, for one warp: up to 32 hops from `cur` at
// depth `matched`, using only each edge's first token.  Lane i gets hop i
// (child, edge length, depth, and the edge's offset and length in the token
// arena when the hop came from a run, else -1).  The walk stops at a missing
// child, at the end of the query, at an edge that is empty or runs past the
// end of the query (taken, then the walk stops), or past b.  Returns false
// (after recording AKV_ERR_TREE) on a malformed tree.
struct Chase {
  int n = 0;                   // hops in this segment
  int64_t d = 0;               // depth after the last hop
  int32_t node = 0;            // node after the last hop
  bool last_segment = false;   // the walk ends with this segment's hops
  bool range_end = false;      // the hops reach past b < L
  int32_t my_child = -1, my_len = 0;
  int64_t my_d = 0;
  int64_t my_off = -1;         // from a run: the edge's offset (else -1, read later)
  int32_t my_elen = -1;        // from a run: the edge's length in the node array
  // When a segment ends at its 32nd hop inside a unary chain, the next
  // segment's run is the next consecutive entries of the same run (a run
  // starting inside a chain is a suffix of it): its entries are fetched at
  // the end of this segment and land while the caller works on its hops.
  int32_t carry_rp = -1;
  int4 carry_e = make_int4(-1, 0, 0, 0);
};

// kProbeEdges: a hop found by a hash probe loads its edge's offset and
// length at once (the loads are consumed only when the caller uses them);
// else they are left at -1 for the caller to read.
template <bool kProbeEdges, typename QToken>
AKV_DEV bool chase_segment(Chase& c, const AkvTreeView& tree, const int4* __restrict__ slots,
                           const int4* __restrict__ runs, const int32_t* __restrict__ Q, int64_t L,
                           int64_t b, int64_t matched, int32_t cur, int32_t q, AkvStatus* st, int lane,
                           QToken& qtoken) {
  constexpr uint32_t kFull = 0xffffffffu;
  int n = 0;
  int64_t d = matched;
  int32_t node = cur;
  c.last_segment = false;
  c.range_end = false;
  c.my_child = -1;
  c.my_len = 0;
  c.my_d = 0;
  c.my_off = -1;
  c.my_elen = -1;
  while (n < kSegment) {
    if (d >= L) {
      c.last_segment = true;
      break;
    }
    if (d >= b) {
      c.range_end = true;
      break;
    }
    // A node with exactly one child starts a run of its unary chain: up to
    // 32 hops come from one load of consecutive run entries (each lane one
    // entry), their depths from a prefix sum of the edge lengths, and each
    // hop is taken only if the query's token at its depth is the entry's
    // first token — what the hash lookup of that hop would have decided.
    int32_t rp = -1;
    int4 e = make_int4(-1, 0, 0, 0);
    if (c.carry_rp >= 0 && n == 0) {  // fetched at the end of the previous segment
      rp = c.carry_rp;
      e = c.carry_e;
    } else if (runs != nullptr && node < tree.run_nodes) {
      rp = __ldg(&tree.run_head[node]);
      // The run's next 32 entries in one load (each lane one; those past
      // the array's end read nothing), the run length from the first.
      if (rp >= 0 && static_cast<int64_t>(rp) + lane < tree.n_runs) e = __ldg(&runs[rp + lane]);
    }
    c.carry_rp = -1;
    if (rp >= 0) {
      const int32_t rem = __shfl_sync(kFull, e.w, 0);
      if (rem < 1 || static_cast<int64_t>(rp) + rem > tree.n_runs) {
        if (lane == 0) akv_fail(st, AKV_ERR_TREE, q, node, rp);
        return false;
      }
      const int k = rem < kSegment - n ? rem : kSegment - n;
      if (lane >= k) e = make_int4(-1, 0, 0, 0);
      const uint32_t malformed =
          __ballot_sync(kFull, lane < k && (e.x < 0 || e.x >= tree.n_nodes || e.z < 0));
      if (malformed) {
        if (lane == 0) akv_fail(st, AKV_ERR_TREE, q, node, rp);
        return false;
      }
      int64_t incl = lane < k ? e.z : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int64_t y = __shfl_up_sync(kFull, incl, o);
        if (lane >= o) incl += y;
      }
      const int64_t di = d + incl - (lane < k ? e.z : 0);  // depth where entry `lane` starts
      int32_t qt = 0;
      if (lane < k && di < L) qt = Q[di];
      // independent of the query token above: both loads are in flight at once
      int64_t e_off = -1;
      int32_t e_len = -1;
      if (lane < k) {
        e_off = __ldg(&tree.node_edge_off[e.x]);
        e_len = __ldg(&tree.node_edge_len[e.x]);
      }
      const uint32_t pass = __ballot_sync(kFull, lane < k && di < L && qt == e.y);
      const uint32_t in_run = k == 32 ? kFull : ((1u << k) - 1u);
      const uint32_t fail = ~pass & in_run;
      const int first_fail = fail ? __ffs(fail) - 1 : k;  // hops [0, first_fail) found their child
      const uint32_t upto = first_fail == 32 ? kFull : ((1u << first_fail) - 1u);
      // an empty edge or one running past the query end is taken, then the walk stops
      const uint32_t stop_m = __ballot_sync(kFull, lane < k && (e.z == 0 || di + e.z > L)) & upto;
      int taken = first_fail;
      bool stop = first_fail < k;
      if (stop_m) {
        taken = __ffs(stop_m);
        stop = true;
      }
      const int src = (lane - n) & 31;
      const int32_t c_s = __shfl_sync(kFull, e.x, src);
      const int32_t l_s = __shfl_sync(kFull, e.z, src);
      const int64_t d_s = __shfl_sync(kFull, di, src);
      const int64_t o_s = __shfl_sync(kFull, e_off, src);
      const int32_t el_s = __shfl_sync(kFull, e_len, src);
      if (lane >= n && lane < n + taken) {
        c.my_child = c_s;
        c.my_len = l_s;
        c.my_d = d_s;
        c.my_off = o_s;
        c.my_elen = el_s;
      }
      if (taken > 0) {
        node = __shfl_sync(kFull, e.x, taken - 1);
        d = __shfl_sync(kFull, di, taken - 1) + __shfl_sync(kFull, e.z, taken - 1);
      }
      n += taken;
      if (stop) {
        c.last_segment = true;
        break;
      }
      if (n == kSegment && taken == k && rem > k) {  // the chain goes on past this segment
        c.carry_rp = rp + k;
        c.carry_e = make_int4(-1, 0, 0, 0);
        if (static_cast<int64_t>(c.carry_rp) + lane < tree.n_runs) c.carry_e = __ldg(&runs[c.carry_rp + lane]);
      }
      continue;
    }
    const int32_t t = qtoken(d);
    int32_t clen = 0;
    const int32_t child = warp_lookup(slots, tree.slot_mask, node, t, lane, clen);
    if (child < 0) {
      c.last_segment = true;
      break;
    }
    if (child >= tree.n_nodes || clen < 0) {
      if (lane == 0) akv_fail(st, AKV_ERR_TREE, q, child, tree.n_nodes);
      return false;
    }
    if (lane == n) {
      c.my_child = child;
      c.my_len = clen;
      c.my_d = d;
      if (kProbeEdges) {
        c.my_off = __ldg(&tree.node_edge_off[child]);
        c.my_elen = __ldg(&tree.node_edge_len[child]);
      } else {
        c.my_off = -1;  // read at the verify phase
      }
    }
    ++n;
    if (clen == 0 || d + clen > L) {  // empty edge / edge past the query end: the walk ends here
      c.last_segment = true;
      break;
    }
    d += clen;
    node = child;
  }
  c.n = n;
  c.d = d;
  c.node = node;
  return true;
}

// One verify round of 512 positions [b0, b0 + 512) of a single contiguous
// range in 16-byte loads: the query token of position p at Q[qd + p], the
// arena token at arena[oe + p], with oe + b0 a multiple of 4 so that the
// arena loads are aligned; the query side (any alignment) is loaded as
// aligned quads and realigned with lane shuffles.  Positions outside
// [lo, hi) count as equal.  A quad that would reach past the query's end (L)
// or the arena's (arena_n) is read element by element.  Needs Q's buffer and
// the arena 16-byte aligned (so an address rounded down to 16 bytes stays
// inside the buffer).  Returns the first mismatching position, or -1.
AKV_DEV bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

AKV_DEV int4 ld_quad(const int32_t* __restrict__ base, int64_t idx, int64_t end) {
  if (idx + 3 < end) return __ldg(reinterpret_cast<const int4*>(base + idx));
  int4 v = make_int4(0, 0, 0, 0);
  if (idx < end) v.x = __ldg(base + idx);
  if (idx + 1 < end) v.y = __ldg(base + idx + 1);
  if (idx + 2 < end) v.z = __ldg(base + idx + 2);
  return v;
}

AKV_DEV int4 shfl_quad(const int4& v, int src) {
  return make_int4(__shfl_sync(0xffffffffu, v.x, src), __shfl_sync(0xffffffffu, v.y, src),
                   __shfl_sync(0xffffffffu, v.z, src), __shfl_sync(0xffffffffu, v.w, src));
}

AKV_DEV int32_t verify_round_vec(const int32_t* __restrict__ Q, int64_t qd, int64_t L,
                                 const int32_t* __restrict__ arena, int64_t arena_n, int64_t oe, int32_t b0,
                                 int32_t lo, int32_t hi, int lane) {
  constexpr uint32_t kFull = 0xffffffffu;
  // the query's quads: Q index qa + 128 u + 4 lane, qa = (qd + b0) rounded down
  // to a 16-byte address; the wanted values start r tokens into them
  const int64_t qabs = static_cast<int64_t>(reinterpret_cast<uintptr_t>(Q) >> 2) + qd + b0;
  const int r = static_cast<int>(qabs & 3);
  const int64_t qa = qd + b0 - r;
  int4 tq[4], qq[5];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    tq[u] = ld_quad(arena, oe + b0 + 128 * u + 4 * lane, arena_n);
    qq[u] = ld_quad(Q, qa + 128 * u + 4 * lane, L);
  }
  qq[4] = make_int4(0, 0, 0, 0);
  if (r != 0 && lane == 0) qq[4] = ld_quad(Q, qa + 512, L);  // lane 31's last tokens
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    int4 qv = qq[u];
    if (r != 0) {  // warp-uniform
      const int4 w0 = shfl_quad(qq[u], (lane + 1) & 31);
      const int4 w1 = shfl_quad(qq[u + 1], (lane + 1) & 31);
      const int4 nx = lane == 31 ? w1 : w0;  // the next quad in the query
      if (r == 1) qv = make_int4(qv.y, qv.z, qv.w, nx.x);
      else if (r == 2) qv = make_int4(qv.z, qv.w, nx.x, nx.y);
      else qv = make_int4(qv.w, nx.x, nx.y, nx.z);
    }
    const int32_t p0 = b0 + 128 * u + 4 * lane;
    int j = 4;  // this lane's first mismatching position in the quad
    if (p0 + 3 >= lo && p0 < hi) {
      if (qv.w != tq[u].w && p0 + 3 >= lo && p0 + 3 < hi) j = 3;
      if (qv.z != tq[u].z && p0 + 2 >= lo && p0 + 2 < hi) j = 2;
      if (qv.y != tq[u].y && p0 + 1 >= lo && p0 + 1 < hi) j = 1;
      if (qv.x != tq[u].x && p0 >= lo && p0 < hi) j = 0;
    }
    const uint32_t m = __ballot_sync(kFull, j < 4);
    if (m) {
      const int l = __ffs(m) - 1;
      return b0 + 128 * u + 4 * l + __shfl_sync(kFull, j, l);
    }
  }
  return -1;
}

// The reference's walk (radix_tree.py:513-570) over query Q[0, L), checked
// on positions [a, b) only; one warp, all lanes.  The walk alternates two
// phases:
//  chase  — follow up to 32 hops using only each edge's first token: the next
//           token position is the current depth plus the child's edge length,
//           which the hash slot carries, and the query's tokens come from a
//           256-token window held in registers, so a hop costs one dependent
//           probe.  It stops at a missing child, at the end of the query, at
//           an edge that runs past the end of the query, or past b.
//  verify — compare the chased edges' tokens that lie in [a, b) at once (their
//           positions flattened across the warp) and find the first mismatch.
//           The reference's loop would have stopped at the first edge that
//           mismatches or only partly fits; everything before it is matched.
// Hops past a stop are speculation and are discarded.  Mismatches before a
// are not looked for: the range that holds them reports them, and the
// smallest key over all ranges wins.  With a = 0 and b = L this is the whole
// lookup.
template <int kVerifyChunks, bool kPipelined>
AKV_DEV MatchStop match_range(const AkvTreeView& tree, const int32_t* __restrict__ Q, int64_t L,
                              int64_t a, int64_t b, int32_t q, AkvStatus* st, int lane, bool prefetch,
                              bool vec) {
  constexpr uint32_t kFull = 0xffffffffu;
  if (prefetch) {
    // Ask L2 for the range's query tokens now (one request per 128-byte
    // line, spread over the lanes): the verify rounds then find them there
    // instead of waiting on DRAM one round at a time.
    for (int64_t i = a + 32 * static_cast<int64_t>(lane); i < b; i += 32 * 32)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(Q + i));
  }
  const int4* __restrict__ slots = reinterpret_cast<const int4*>(tree.slots);
  const int4* __restrict__ runs =
      tree.run_head != nullptr ? reinterpret_cast<const int4*>(tree.run_entries) : nullptr;

  // (Prefetching the next 256-token window while the current one is chased
  // measured no faster: 0.182 against 0.179 ms per 4,096-query batch.)
  QueryWindow qtoken{Q, L, lane};

  int32_t cur = 0;  // ROOT_NODE_ID
  int64_t matched = 0;
  Chase c;
  while (true) {
    if (!chase_segment<false>(c, tree, slots, runs, Q, L, b, matched, cur, q, st, lane, qtoken))
      return MatchStop{0, 0, -1};
    const int n = c.n;
    const bool last_segment = c.last_segment, range_end = c.range_end;
    const int32_t my_child = c.my_child, my_len = c.my_len;
    const int64_t my_d = c.my_d;
    int64_t my_off = c.my_off;
    int32_t my_elen = c.my_elen;
    if (n == 0) {  // a missing child at `matched`, the query's end, or the range's end
      if (range_end) return MatchStop{kNoStop, 0, -1};
      return MatchStop{2 * matched, matched, cur};
    }
    // ── verify ──
    bool my_bad = false;
    if (lane < n) {
      if (my_off < 0) {  // a hop found by a hash probe
        my_off = tree.node_edge_off[my_child];
        my_elen = tree.node_edge_len[my_child];
      }
      my_bad = my_off < 0 || my_off + my_len > tree.n_tokens || my_elen != my_len;
    }
    const uint32_t badm = __ballot_sync(kFull, my_bad);
    if (badm) {
      if (lane == __ffs(badm) - 1) akv_fail(st, AKV_ERR_TREE, q, my_child, my_len, my_off);
      return MatchStop{0, 0, -1};
    }
    const int32_t lim = lane < n ? static_cast<int32_t>(my_len < L - my_d ? my_len : L - my_d) : 0;
    int32_t incl = lim;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += y;
    }
    const int32_t excl = incl - lim;
    const int32_t total = __shfl_sync(kFull, incl, 31);
    // The chased edges are consecutive in depth: flattened position p is
    // query position matched + p.  Only [a, b) is compared here.
    const int32_t p_lo = a > matched ? static_cast<int32_t>(a - matched < total ? a - matched : total) : 0;
    const int32_t p_hi = static_cast<int32_t>(b - matched < total ? b - matched : total);
    // entry holding flattened position p: the last e < n with excl_e <= p
    auto entry_of = [&](int32_t p) -> int {
      int lo = 0, hi = n - 1;
#pragma unroll
      for (int k = 0; k < 5; ++k) {
        const int mid = (lo + hi + 1) >> 1;
        const int32_t v = __shfl_sync(kFull, excl, mid);
        if (lo < hi) {
          if (v <= p) lo = mid;
          else hi = mid - 1;
        }
      }
      return lo;
    };
    int32_t first = -1;
    constexpr int32_t kStep = 32 * kVerifyChunks;
    // One verify round: kVerifyChunks x 32 consecutive flattened positions
    // from `base`, query tokens into av, edge tokens into bv.
    // Edges that lie back to back in the token arena, as the nodes of a
    // chain split from one committed edge do (a split keeps the tokens in
    // place): flattened position p is then arena position shift + matched + p
    // across the whole segment, and every round reads two contiguous ranges.
    const int64_t shift = __shfl_sync(kFull, my_off - my_d, 0);
    const bool contiguous = __all_sync(kFull, lane >= n || my_off - my_d == shift);
    auto load_round = [&](int32_t base, int32_t (&av)[kVerifyChunks], int32_t (&bv)[kVerifyChunks]) {
      // Fast path: the whole round lies inside one edge (long edges), or the
      // edges are contiguous.
      int64_t de = matched, oe = shift + matched;
      bool one_range = contiguous;
      if (!one_range) {
        const int e0 = entry_of(base);
        const int32_t ex0 = __shfl_sync(kFull, excl, e0);
        const int32_t lim0 = __shfl_sync(kFull, lim, e0);
        one_range = ex0 + lim0 >= base + kStep || e0 == n - 1;
        de = __shfl_sync(kFull, my_d, e0) - ex0;
        oe = __shfl_sync(kFull, my_off, e0) - ex0;
      }
      if (one_range) {
#pragma unroll
        for (int u = 0; u < kVerifyChunks; ++u) {
          const int32_t p = base + u * 32 + lane;
          const bool ok = p < p_hi;
          av[u] = ok ? Q[de + p] : 0;
          bv[u] = ok ? __ldg(&tree.tokens[oe + p]) : 0;
        }
      } else {
#pragma unroll
        for (int u = 0; u < kVerifyChunks; ++u) {
          const int32_t p = base + u * 32 + lane;
          const int e = entry_of(p < p_hi ? p : p_hi - 1);
          const int32_t j = p - __shfl_sync(kFull, excl, e);
          const int64_t de = __shfl_sync(kFull, my_d, e);
          const int64_t oe = __shfl_sync(kFull, my_off, e);
          const bool ok = p < p_hi;
          av[u] = ok ? Q[de + j] : 0;
          bv[u] = ok ? __ldg(&tree.tokens[oe + j]) : 0;
        }
      }
    };
    auto check_round = [&](int32_t base, const int32_t (&av)[kVerifyChunks],
                           const int32_t (&bv)[kVerifyChunks]) {
#pragma unroll
      for (int u = 0; u < kVerifyChunks; ++u) {
        const uint32_t m = __ballot_sync(kFull, av[u] != bv[u]);
        if (m && first < 0) first = base + u * 32 + __ffs(m) - 1;
      }
    };
    if constexpr (kPipelined) {
      // Two rounds in flight: the next round's loads are issued before this
      // round's compare (a round past a mismatch is loaded and discarded;
      // every position loaded lies below p_hi, inside the query and the
      // edge).
      int32_t a0[kVerifyChunks], b0[kVerifyChunks], a1[kVerifyChunks], b1[kVerifyChunks];
      if (p_lo < p_hi) load_round(p_lo, a0, b0);
      for (int32_t base = p_lo; base < p_hi; base += 2 * kStep) {
        if (base + kStep < p_hi) load_round(base + kStep, a1, b1);
        check_round(base, a0, b0);
        if (first >= 0 || base + kStep >= p_hi) break;
        if (base + 2 * kStep < p_hi) load_round(base + 2 * kStep, a0, b0);
        check_round(base + kStep, a1, b1);
        if (first >= 0) break;
      }
    } else {
      for (int32_t base = p_lo; base < p_hi;) {
        if constexpr (kVerifyChunks == 8) {
          // 512 positions of one range per round in 16-byte loads: the
          // segment's edges are contiguous, or the next 512 positions lie in
          // one edge (or the last)
          if (vec) {
            int64_t oe = shift + matched;
            bool one = contiguous;
            if (!one) {
              const int e0 = entry_of(base);
              const int32_t ex0 = __shfl_sync(kFull, excl, e0);
              one = ex0 + __shfl_sync(kFull, lim, e0) >= base + 512 || e0 == n - 1;
              oe = __shfl_sync(kFull, my_off, e0) - ex0;
            }
            const int32_t b0 = base - static_cast<int32_t>((oe + base) & 3);
            // (the query's quads start at or after the packing's first token)
            if (one && matched + b0 >= 0) {
              first = verify_round_vec(Q, matched, L, tree.tokens, tree.n_tokens, oe, b0, base, p_hi, lane);
              if (first >= 0) break;
              base = b0 + 512;
              continue;
            }
          }
        }
        int32_t av[kVerifyChunks], bv[kVerifyChunks];
        load_round(base, av, bv);
        check_round(base, av, bv);
        if (first >= 0) break;
        base += kStep;
      }
    }
    // the first entry the reference would stop in
    const int e_mis = first >= 0 ? entry_of(first) : kSegment;
    const uint32_t short_m = __ballot_sync(kFull, lane < n && (lim < my_len || my_len == 0));
    const int e_short = short_m ? __ffs(short_m) - 1 : kSegment;
    const int e_stop = e_mis < e_short ? e_mis : e_short;
    if (e_stop == kSegment) {  // every chased edge matched in [a, b)
      const int64_t end = __shfl_sync(kFull, my_d, n - 1) + __shfl_sync(kFull, my_len, n - 1);
      const int32_t last = __shfl_sync(kFull, my_child, n - 1);
      if (last_segment) return MatchStop{2 * end, end, last};
      matched = end;
      cur = last;
      if (range_end) return MatchStop{kNoStop, 0, -1};
      continue;
    }
    const int32_t ex = __shfl_sync(kFull, excl, e_stop);
    const bool mism = e_mis == e_stop;
    const int32_t em = mism ? first - ex : __shfl_sync(kFull, lim, e_stop);
    const int64_t stop_d = __shfl_sync(kFull, my_d, e_stop);
    const int32_t prev_child = __shfl_sync(kFull, my_child, e_stop > 0 ? e_stop - 1 : 0);
    return MatchStop{2 * (matched + ex + em) + (mism ? 1 : 0), stop_d, e_stop > 0 ? prev_child : cur};
  }
}

AKV_DEV void match_write(const MatchStop& s, int32_t q, int32_t block_size, int32_t* out_node,
                         int32_t* out_len, int64_t* out_compared) {
  const int64_t m = (s.matched / block_size) * block_size;
  out_node[q] = m == 0 ? -1 : s.node;
  out_len[q] = static_cast<int32_t>(m);
  if (out_compared != nullptr) out_compared[q] = (s.key >> 1) + (s.key & 1);
}

// One warp per query (the whole query is one range).  `order` (optional)
// lists the queries longest first, so the long walks start early and spread
// over the SMs.  At most 96 registers (20 warps per SM): the 16-byte verify
// rounds alone would take 126 and measured slower for it (0.0729 against
// 0.0585 ms per batch on the stress tree; without those rounds, 80 registers,
// 0.0631 ms; capped at 80 with them, 0.0603 ms with spills).
template <int kVerifyChunks, bool kPipelined>
__global__ void __launch_bounds__(kWholeWarpsPerCta * 32, 20 / kWholeWarpsPerCta)
k_match(AkvTreeView tree, const int32_t* __restrict__ tokens, const int64_t* __restrict__ q_off,
        int32_t nq, int32_t block_size, int32_t* __restrict__ out_node,
        int32_t* __restrict__ out_len, int64_t* __restrict__ out_compared,
        const int32_t* __restrict__ order, AkvStatus* st, bool prefetch) {
  const int lane = threadIdx.x & 31;
  const int32_t w = blockIdx.x * kWholeWarpsPerCta + (threadIdx.x >> 5);
  if (w >= nq) return;
  const int32_t q = order != nullptr ? order[w] : w;
  if (static_cast<uint32_t>(q) >= static_cast<uint32_t>(nq)) {
    if (lane == 0) akv_fail(st, AKV_ERR_INVALID_ARG, w, q, nq);
    return;
  }
  const int64_t qlo = q_off[q];
  const int64_t L = q_off[q + 1] - qlo;
  const MatchStop s = match_range<kVerifyChunks, kPipelined>(tree, tokens + qlo, L, 0, L, q, st, lane, prefetch,
                                                             aligned16(tokens) && aligned16(tree.tokens));
  if (lane == 0) match_write(s, q, block_size, out_node, out_len, out_compared);
}

// ── split lookups: a query's positions in ranges of R tokens, one warp each ──
// A batch is bounded by its longest query when one warp walks each query
// (an 8,192-token query is 32 dependent verify rounds of 256 tokens).  Here
// query q is cut into k_q = max(1, ceil(L_q / R)) ranges; the warp of range
// j walks the tree up to position (j + 1) R and compares positions
// [j R, (j + 1) R) only, so every warp compares at most R tokens and the
// SMs stay evenly loaded.  Each range reports the first stop it sees
// (MatchStop); the warp that finishes a query's last range picks the
// smallest key among them, which is the stop of the reference's loop.
//
// The queries are launched longest first (`order`), so range j exists for
// exactly the first n_j ranks: warp w takes range j of rank w - start[j],
// where start[j] = n_0 + ... + n_{j-1}; the host passes start[] (it knows
// the lengths), so no list of ranges is built on the device.
//
// Scratch (caller-owned, akv_match_scratch_bytes): one 16-byte stop record
// per range, then a per-query count of finished ranges (cleared by the
// entry point before the launch).
constexpr int kMaxSplitRanges = AKV_MATCH_MAX_RANGES;

struct SplitRanges {
  int64_t start[kMaxSplitRanges + 1];  // start[j]: first warp of range j; start[n] = total
  int32_t n;                           // ranges of the longest query
  int32_t R;                           // tokens per range
};

AKV_HD int64_t split_items_max(int32_t nq, int64_t n_tokens, int32_t R) {
  return static_cast<int64_t>(nq) + n_tokens / R;  // sum of max(1, ceil(L/R)) <= nq + sum(L)/R
}

AKV_HD int64_t split_scratch_bytes(int32_t nq, int64_t w_max) {
  const int64_t b = 16 * w_max + 4 * static_cast<int64_t>(nq);
  return (b + 255) / 256 * 256;
}

AKV_DEV int32_t split_count(int64_t L, int32_t R) {
  return L <= 0 ? 1 : static_cast<int32_t>((L + R - 1) / R);
}

template <int kVerifyChunks, bool kPipelined>
__global__ void __launch_bounds__(kMatchWarpsPerCta * 32, 5)
k_match_split(AkvTreeView tree, const int32_t* __restrict__ tokens, const int64_t* __restrict__ q_off,
              int32_t nq, int32_t block_size, const __grid_constant__ SplitRanges rg,
              const int32_t* __restrict__ order, int4* __restrict__ stops, int32_t* __restrict__ done,
              int32_t* __restrict__ out_node, int32_t* __restrict__ out_len,
              int64_t* __restrict__ out_compared, AkvStatus* st, bool prefetch) {
  constexpr uint32_t kFull = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const int64_t it = static_cast<int64_t>(blockIdx.x) * kMatchWarpsPerCta + (threadIdx.x >> 5);
  if (it >= rg.start[rg.n]) return;
  int j = 0;  // range index: the last j with start[j] <= it
  while (j + 1 < rg.n && rg.start[j + 1] <= it) ++j;
  const int64_t r = it - rg.start[j];
  const int32_t q = order[r];
  if (static_cast<uint32_t>(q) >= static_cast<uint32_t>(nq)) {
    if (lane == 0) akv_fail(st, AKV_ERR_INVALID_ARG, static_cast<int32_t>(r), q, nq);
    return;
  }
  const int64_t qlo = q_off[q];
  const int64_t L = q_off[q + 1] - qlo;
  const int32_t R = rg.R;
  const int32_t k = split_count(L, R);
  // rank r must hold ranges 0 .. k-1 and no more: r < n_{k-1} and r >= n_k
  const bool listed = k <= rg.n && r < rg.start[k] - rg.start[k - 1] &&
                      (k == rg.n || r >= rg.start[k + 1] - rg.start[k]);
  if (!listed || L > INT32_MAX) {
    if (lane == 0 && j == 0) akv_fail(st, AKV_ERR_INVALID_ARG, static_cast<int32_t>(r), q, k, L);
    return;
  }
  const int64_t a = static_cast<int64_t>(j) * R;
  const int64_t b = a + R < L ? a + R : L;
  const MatchStop s = match_range<kVerifyChunks, kPipelined>(tree, tokens + qlo, L, a, b, q, st, lane, prefetch,
                                                             aligned16(tokens) && aligned16(tree.tokens));
  if (k == 1) {
    if (lane == 0) match_write(s, q, block_size, out_node, out_len, out_compared);
    return;
  }
  int32_t prior = 0;
  if (lane == 0) {
    __stcg(&stops[it], make_int4(static_cast<int32_t>(s.key & 0xffffffff), static_cast<int32_t>(s.key >> 32),
                                 static_cast<int32_t>(s.matched), s.node));
    __threadfence();
    prior = atomicAdd(&done[q], 1);
  }
  prior = __shfl_sync(kFull, prior, 0);
  if (prior != k - 1) return;  // another range of this query finishes last
  __threadfence();
  // the last range of query q: the smallest key over its k stop records
  int64_t best = kNoStop;
  int32_t b_matched = 0, b_node = -1;
  for (int32_t i = lane; i < k; i += 32) {
    const int4 rec = __ldcg(&stops[rg.start[i] + r]);
    const int64_t key = (static_cast<int64_t>(rec.y) << 32) | static_cast<uint32_t>(rec.x);
    if (key < best) {
      best = key;
      b_matched = rec.z;
      b_node = rec.w;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const int64_t ok = __shfl_xor_sync(kFull, best, o);
    const int32_t om = __shfl_xor_sync(kFull, b_matched, o);
    const int32_t on = __shfl_xor_sync(kFull, b_node, o);
    if (ok < best) {
      best = ok;
      b_matched = om;
      b_node = on;
    }
  }
  if (lane == 0) {
    if (best == kNoStop) {  // cannot happen for a well-formed walk; never report a match then
      akv_fail(st, AKV_ERR_TREE, q, -1, k);
      best = 0;
      b_matched = 0;
    }
    match_write(MatchStop{best, b_matched, b_node}, q, block_size, out_node, out_len, out_compared);
  }
}

// ── staged lookups: every query chased first, its edges then verified in
// windows spread over the whole grid ──
// With one warp per query a batch lasts as long as its longest walk: an
// 8,192-token query that matches a cached sequence is 32 dependent verify
// rounds of 256 tokens, while most warps have long finished.  Here the
// lookup is two launches:
//  k_match_chase  — one warp per query runs the chase phase alone over the
//                   whole query (chase_segment: hops decided by each edge's
//                   first token, every hop's edge range loaded as it is
//                   found) and writes its hops and, for every W-token window
//                   of the chased span [0, D), a record of the window with
//                   the hop that holds its first position;
//  k_match_verify — one warp per window compares the query's tokens in it
//                   with the hops' edge tokens: a window inside one edge
//                   (most of them) goes from its record straight to the
//                   token loads.  The first mismatch over all windows of a
//                   query (an atomic min on position) is the reference
//                   loop's stop, and the warp that finishes the query's last
//                   window writes its answer.
// The answer is the one-warp walk's: the walk stops at the first hop along
// the chased path that mismatches or only partly fits (only the last hop can
// partly fit); hops past it are speculation and are discarded.  The chase may
// run further ahead than the one-warp walk (up to the query's end), so on a
// malformed tree it can report AKV_ERR_TREE where that walk would not.
//
// Scratch (caller-owned, akv_match_staged_scratch_bytes):
//   hops  int4 [n_tokens]   {child, edge length, depth, edge offset}: query
//                           q's hops at q_off[q] + h (a query of L tokens has
//                           at most L hops, as every hop before the last
//                           takes at least one token)
//   wins  2 x int4 [n_tokens / W + nq + 1]  {q, hop, window, q_off[q]} and
//                           {hop depth, edge length, edge offset, L}, or q = -1
//                           for an unused slot: query q's windows from slot
//                           q_off[q] / W + q (so no prefix sum is needed)
//   qinfo int4 [nq]         {hops, D, windows, 0}
//   stop  uint64 [nq]       (position << 32) | hop of the first mismatch
//   left  int32 [nq]        windows of the query not finished yet
// Every slot is written by the chase, so the scratch needs no clearing.
// Token counts and edge offsets must fit in int32 (checked on the host).
struct StagedScratch {
  int4* hops;
  int4* wins;
  int4* qinfo;
  unsigned long long* stop;
  int32_t* left;
};

AKV_HD int64_t staged_round256(int64_t b) { return (b + 255) / 256 * 256; }

AKV_HD int64_t staged_slots(int32_t nq, int64_t n_tokens, int32_t W) { return n_tokens / W + nq + 1; }

// Carves the scratch at `base` (nullptr: only sizes it); returns its bytes.
AKV_HD int64_t staged_layout(char* base, int32_t nq, int64_t n_tokens, int32_t W, StagedScratch* sc) {
  int64_t o = 0;
  auto take = [&](int64_t bytes) {
    char* p = base != nullptr ? base + o : nullptr;
    o += staged_round256(bytes);
    return p;
  };
  char* hops = take(16 * n_tokens);
  char* wins = take(32 * staged_slots(nq, n_tokens, W));
  char* qinfo = take(16 * static_cast<int64_t>(nq));
  char* stop = take(8 * static_cast<int64_t>(nq));
  char* left = take(4 * static_cast<int64_t>(nq));
  if (sc != nullptr) {
    sc->hops = reinterpret_cast<int4*>(hops);
    sc->wins = reinterpret_cast<int4*>(wins);
    sc->qinfo = reinterpret_cast<int4*>(qinfo);
    sc->stop = reinterpret_cast<unsigned long long*>(stop);
    sc->left = reinterpret_cast<int32_t*>(left);
  }
  return o;
}

constexpr unsigned long long kNoMismatch = ~0ull;
constexpr int64_t kCheckMinTokens = 64;  // edges the chase checks 32 tokens into

// The answer of query q from its hops, the first mismatch (or kNoMismatch)
// and the query length.
AKV_DEV void staged_finish(const int4* __restrict__ hops, int32_t n_hops, int64_t L, unsigned long long stop,
                           int32_t q, int32_t block_size, int32_t* out_node, int32_t* out_len,
                           int64_t* out_compared) {
  MatchStop s{0, 0, 0};  // no hop: nothing matched at the root
  if (stop != kNoMismatch) {  // the hop holding the first mismatch stops the walk
    const int64_t P = static_cast<int64_t>(stop >> 32);
    const int32_t h = static_cast<int32_t>(stop & 0xffffffffu);
    s = MatchStop{2 * P + 1, hops[h].z, h > 0 ? hops[h - 1].x : 0};
  } else if (n_hops > 0) {
    const int4 last = hops[n_hops - 1];
    const int64_t lim = last.y < L - last.z ? last.y : L - last.z;
    if (lim < last.y || last.y == 0)  // the last edge only partly fits: the walk stops at its start
      s = MatchStop{2 * (last.z + lim), last.z, n_hops > 1 ? hops[n_hops - 2].x : 0};
    else  // every hop matched in full
      s = MatchStop{2 * (static_cast<int64_t>(last.z) + last.y), static_cast<int64_t>(last.z) + last.y, last.x};
  }
  match_write(s, q, block_size, out_node, out_len, out_compared);
}

template <int kW>
__global__ void __launch_bounds__(kMatchWarpsPerCta * 32)
k_match_chase(AkvTreeView tree, const int32_t* __restrict__ tokens, const int64_t* __restrict__ q_off,
              int32_t nq, int64_t n_tokens, int32_t block_size, const int32_t* __restrict__ order,
              StagedScratch sc, int32_t* __restrict__ out_node, int32_t* __restrict__ out_len,
              int64_t* __restrict__ out_compared, AkvStatus* st) {
  constexpr uint32_t kFull = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const int32_t w = blockIdx.x * kMatchWarpsPerCta + (threadIdx.x >> 5);
  if (w >= nq) return;
  const int32_t q = order != nullptr ? order[w] : w;
  if (static_cast<uint32_t>(q) >= static_cast<uint32_t>(nq)) {
    if (lane == 0) akv_fail(st, AKV_ERR_INVALID_ARG, w, q, nq);
    return;
  }
  const int64_t qlo = q_off[q], qhi = q_off[q + 1];
  if (qlo < 0 || qhi < qlo || qhi > n_tokens) {
    if (lane == 0) akv_fail(st, AKV_ERR_INVALID_ARG, w, q, static_cast<int32_t>(qhi - qlo), qlo);
    return;
  }
  const int64_t L = qhi - qlo;
  const int32_t* __restrict__ Q = tokens + qlo;
  const int4* __restrict__ slots = reinterpret_cast<const int4*>(tree.slots);
  const int4* __restrict__ runs =
      tree.run_head != nullptr ? reinterpret_cast<const int4*>(tree.run_entries) : nullptr;
  int4* __restrict__ hops = sc.hops + qlo;
  int4* __restrict__ wins = sc.wins + 2 * (qlo / kW + q);
  QueryWindow qtoken{Q, L, lane};
  Chase c;
  int32_t cur = 0, h = 0;  // node reached, hops written
  int64_t matched = 0, D = 0;
  while (true) {
    if (!chase_segment<true>(c, tree, slots, runs, Q, L, L, matched, cur, q, st, lane, qtoken)) return;
    const int n = c.n;
    if (n == 0) break;
    const bool bad = lane < n && (c.my_off < 0 || c.my_off + c.my_len > tree.n_tokens || c.my_elen != c.my_len);
    const uint32_t badm = __ballot_sync(kFull, bad);
    if (badm) {
      if (lane == __ffs(badm) - 1) akv_fail(st, AKV_ERR_TREE, q, c.my_child, c.my_len, c.my_off);
      return;
    }
    int64_t lim = lane < n ? (c.my_len < L - c.my_d ? c.my_len : L - c.my_d) : 0;
    // A long edge whose first tokens already differ from the query holds
    // the walk's stop: the chase ends there, and the windows stop at the
    // mismatch instead of covering the edge and the speculation after it.
    // (Siblings that share a first token and part of a block are common:
    // the block-aligned split keeps one child per first token, so a query
    // often takes an edge that differs a few tokens in.)  One warp-wide
    // compare of the first 32 tokens per long edge.
    int keep = n;
    bool cut = false;
    uint32_t longm = __ballot_sync(kFull, lane < n && lim >= kCheckMinTokens);
    while (longm) {
      const int e = __ffs(longm) - 1;
      longm &= longm - 1;
      const int64_t de = __shfl_sync(kFull, c.my_d, e);
      const int64_t oe = __shfl_sync(kFull, c.my_off, e);
      const uint32_t mm = __ballot_sync(kFull, Q[de + lane] != __ldg(&tree.tokens[oe + lane]));
      if (mm) {
        keep = e + 1;
        cut = true;
        const int64_t end = de + __ffs(mm);  // through the mismatching position
        if (lane == e) lim = end - de;
        break;
      }
    }
    if (lane < keep) {
      const int32_t d32 = static_cast<int32_t>(c.my_d), off32 = static_cast<int32_t>(c.my_off);
      hops[h + lane] = make_int4(c.my_child, c.my_len, d32, off32);
      // the windows whose first position lies in this hop
      for (int64_t k = (c.my_d + kW - 1) / kW; k * kW < c.my_d + lim; ++k) {
        wins[2 * k] = make_int4(q, h + lane, static_cast<int32_t>(k), static_cast<int32_t>(qlo));
        wins[2 * k + 1] = make_int4(d32, c.my_len, off32, static_cast<int32_t>(L));
      }
    }
    h += keep;
    D = __shfl_sync(kFull, c.my_d + lim, keep - 1);
    if (c.last_segment || cut) break;
    matched = c.d;
    cur = c.node;
  }
  const int64_t nw = (D + kW - 1) / kW;
  // this query's unused slots, up to the next query's first; the last query
  // in the packing also clears the slots after it, and the first those before
  const bool packed_last = qhi == q_off[nq];
  const int64_t s_hi = packed_last ? n_tokens / kW + nq + 1 - (qlo / kW + q) : qhi / kW + 1 - qlo / kW;
  for (int64_t k = nw + lane; k < s_hi; k += 32) wins[2 * k] = make_int4(-1, 0, 0, 0);
  if (qlo == q_off[0])
    for (int64_t k = lane; k < qlo / kW; k += 32) sc.wins[2 * k] = make_int4(-1, 0, 0, 0);
  __syncwarp();
  if (lane == 0) {
    sc.qinfo[q] = make_int4(h, static_cast<int32_t>(D), static_cast<int32_t>(nw), 0);
    sc.stop[q] = kNoMismatch;
    sc.left[q] = static_cast<int32_t>(nw);
    if (nw == 0) staged_finish(hops, h, L, kNoMismatch, q, block_size, out_node, out_len, out_compared);
  }
}

// One window of a staged lookup (record r0, r1), one warp.  Returns false
// after recording an error.
template <int kW>
AKV_DEV bool verify_window(const AkvTreeView& tree, const int32_t* __restrict__ tokens, const int4& r0,
                           const int4& r1, const StagedScratch& sc, int32_t block_size,
                           int32_t* __restrict__ out_node, int32_t* __restrict__ out_len,
                           int64_t* __restrict__ out_compared, AkvStatus* st, int lane) {
  constexpr uint32_t kFull = 0xffffffffu;
  constexpr int32_t kRound = kW < 512 ? kW : 512;  // positions per round inside one edge
  constexpr int kRC = kRound / 32;
  constexpr int kChunks = 8;  // rounds of 256 positions across several edges
  constexpr int32_t kStep = 32 * kChunks;
  const int32_t q = r0.x, h0 = r0.y, pw = r0.z * kW, qlo = r0.w;
  const int32_t d0 = r1.x, L = r1.w;
  const int32_t end0 = d0 + (r1.y < L - d0 ? r1.y : L - d0);  // end of hop h0's positions
  const int32_t* __restrict__ Q = tokens + qlo;
  const int4* __restrict__ hops = sc.hops + qlo;
  int4 qi = make_int4(0, 0, 0, 0);  // {hops, D, windows}: needed only past hop h0
  int32_t pe = pw + kW;
  if (end0 < pe) {
    qi = sc.qinfo[q];
    pe = pe < qi.y ? pe : qi.y;
  }
  int32_t first = -1, first_hop = -1;
  if (end0 >= pe) {  // the window lies in one edge: straight to the tokens
    const int64_t oe = static_cast<int64_t>(r1.z) - d0;
    for (int32_t base = pw; base < pe && first < 0; base += kRound) {
      int32_t av[kRC], bv[kRC];
#pragma unroll
      for (int u = 0; u < kRC; ++u) {
        const int32_t x = base + u * 32 + lane;
        const bool ok = x < pe;
        av[u] = ok ? Q[x] : 0;
        bv[u] = ok ? __ldg(&tree.tokens[oe + x]) : 0;
      }
#pragma unroll
      for (int u = 0; u < kRC; ++u) {
        const uint32_t m = __ballot_sync(kFull, av[u] != bv[u]);
        if (m && first < 0) first = base + u * 32 + __ffs(m) - 1;
      }
    }
    if (first >= 0) first_hop = h0;
  } else {  // several edges: the hops 32 at a time, one per lane
    int32_t p = pw;
    for (int32_t g = h0; p < pe && first < 0; g += 32) {
      const int nh = qi.x - g < 32 ? qi.x - g : 32;
      if (nh <= 0) {  // positions left but no hop for them: the scratch does not hold this batch's chase
        if (lane == 0) akv_fail(st, AKV_ERR_TREE, q, g, qi.x);
        return false;
      }
      int4 hp = make_int4(-1, 0, INT32_MAX, 0);
      if (lane < nh) hp = hops[g + lane];
      const int32_t lim = lane < nh ? (hp.y < L - hp.z ? hp.y : L - hp.z) : 0;
      const int32_t gend_all = __shfl_sync(kFull, hp.z + lim, nh - 1);
      const int32_t gend = gend_all < pe ? gend_all : pe;
      // hop holding position x: the last lane with depth <= x
      auto hop_of = [&](int32_t x) -> int {
        int lo = 0, hi = nh - 1;
#pragma unroll
        for (int k = 0; k < 5; ++k) {
          const int mid = (lo + hi + 1) >> 1;
          const int32_t v = __shfl_sync(kFull, hp.z, mid);
          if (lo < hi) {
            if (v <= x) lo = mid;
            else hi = mid - 1;
          }
        }
        return lo;
      };
      // hops whose edges lie back to back in the arena read one range
      const int32_t shift = __shfl_sync(kFull, hp.w - hp.z, 0);
      const bool contiguous = __all_sync(kFull, lane >= nh || hp.w - hp.z == shift);
      for (int32_t base = p; base < gend; base += kStep) {
        int32_t av[kChunks], bv[kChunks];
#pragma unroll
        for (int u = 0; u < kChunks; ++u) {
          const int32_t x = base + u * 32 + lane;
          const bool ok = x < gend;
          int64_t oe = shift;
          if (!contiguous) {
            const int e = hop_of(ok ? x : gend - 1);
            oe = static_cast<int64_t>(__shfl_sync(kFull, hp.w, e)) - __shfl_sync(kFull, hp.z, e);
          }
          av[u] = ok ? Q[x] : 0;
          bv[u] = ok ? __ldg(&tree.tokens[oe + x]) : 0;
        }
#pragma unroll
        for (int u = 0; u < kChunks; ++u) {
          const uint32_t m = __ballot_sync(kFull, av[u] != bv[u]);
          if (m && first < 0) first = base + u * 32 + __ffs(m) - 1;
        }
        if (first >= 0) {
          first_hop = g + hop_of(first);
          break;
        }
      }
      p = gend;
    }
  }
  int32_t prior = 0;
  if (lane == 0) {
    if (first >= 0)
      atomicMin(&sc.stop[q], (static_cast<unsigned long long>(first) << 32) | static_cast<uint32_t>(first_hop));
    __threadfence();
    prior = atomicSub(&sc.left[q], 1);
  }
  prior = __shfl_sync(kFull, prior, 0);
  if (prior != 1) return true;  // another window of this query finishes last
  __threadfence();
  if (lane == 0)
    staged_finish(hops, sc.qinfo[q].x, L, atomicAdd(&sc.stop[q], 0ull), q, block_size, out_node, out_len,
                  out_compared);
  return true;
}

// One warp per window slot.  (Fewer warps looping over the slots, each
// loading its next record while comparing, measured slower: 0.089 against
// 0.055 ms per 4,096-query batch, cold.)
template <int kW>
__global__ void __launch_bounds__(kMatchWarpsPerCta * 32)
k_match_verify(AkvTreeView tree, const int32_t* __restrict__ tokens, int64_t n_slots, int32_t block_size,
               StagedScratch sc, int32_t* __restrict__ out_node, int32_t* __restrict__ out_len,
               int64_t* __restrict__ out_compared, AkvStatus* st) {
  const int lane = threadIdx.x & 31;
  const int64_t slot = static_cast<int64_t>(blockIdx.x) * kMatchWarpsPerCta + (threadIdx.x >> 5);
  if (slot >= n_slots || akv_failed(st)) return;
  const int4 r0 = sc.wins[2 * slot];
  if (r0.x < 0) return;
  const int4 r1 = sc.wins[2 * slot + 1];
  verify_window<kW>(tree, tokens, r0, r1, sc, block_size, out_node, out_len, out_compared, st, lane);
}

// ── tree changes built on the device ───────────────────────────────────────
// The host tree's structural changes (DualRadixTree._insert_shared_locked,
// radix_tree.py:572-686, and the prune in _dec_shared_ref_locked, :695-717)
// restated as commands that a replica applies to its own arrays, so that a
// commit ships its tokens and a few ids instead of the slot, node and token
// rows the change wrote.  One warp applies the commands in order.
//   insert {parent, first new node id, offset and count of its tokens in the
//          payload, arena length before it}: walk from `parent` by first
//          token; a missing child gets a new leaf; a fully matched edge is
//          descended; an edge that matches to its end with the tokens also
//          ending changes nothing (the host replaces the node's blocks);
//          otherwise the edge splits at the block boundary at or below the
//          common prefix — at 0 the new leaf takes the parent's slot for that
//          first token (the old child stays, unreachable from the parent), else
//          a new middle node takes the common blocks and the rest goes to a
//          new leaf under it.  New nodes take consecutive ids from the given
//          one, new edge tokens go to the arena in the order the host appends
//          them, and slots are claimed as the host's probe claims them: the
//          key's own slot when present, else the first deleted slot on the
//          probe path, else the empty slot that ends it.
//   prune  {parent, node}: the parent's slot for the node's first token is
//          deleted when it holds the node (parent -1: no parent left), and
//          the node's edge is cleared.
// The host keeps the arrays large enough (it grows and rehashes them with a
// full upload); the kernel still bounds every index and reports
// AKV_ERR_TREE (and stops) instead of writing out of range.  Arrays written
// here are read back through volatile loads: a later command reads what an
// earlier one wrote.
constexpr int64_t kCmdInsert = 1, kCmdPrune = 2;
constexpr int kCmdWords = 8;  // {kind, parent, node / first new id, src, n, arena, block size, 0}
constexpr int32_t kSlotDeleted = -2;

struct TreeArrays {
  volatile int32_t* tokens;
  volatile int64_t* off;
  volatile int32_t* len;
  volatile int4* slots;
  int4* slots_w;  // the same slots, for whole-slot stores
  int64_t token_cap;
  int32_t n_nodes, mask;
};

// (slot holding (parent, token) or -1, first reusable slot on the probe
// path or -1): the host's DeviceTree._probe, 32 slots per step.
AKV_DEV void cmd_probe(const TreeArrays& t, int32_t parent, int32_t token, int lane, int32_t& found,
                       int32_t& reusable) {
  constexpr uint32_t kFull = 0xffffffffu;
  const uint32_t h = tree_hash(parent, token);
  found = -1;
  reusable = -1;
  for (int64_t base = 0; base <= t.mask; base += 32) {
    const uint32_t idx = (h + static_cast<uint32_t>(base) + static_cast<uint32_t>(lane)) & static_cast<uint32_t>(t.mask);
    const bool in = base + lane <= t.mask;
    int32_t p = 0, tk = 0;
    if (in) {
      p = t.slots[idx].x;
      tk = t.slots[idx].y;
    }
    const uint32_t hit = __ballot_sync(kFull, in && p == parent && tk == token);
    const uint32_t empty = __ballot_sync(kFull, in && p == kEmpty);
    const uint32_t del = __ballot_sync(kFull, in && p == kSlotDeleted);
    const uint32_t stop = hit | empty;
    const int first_stop = stop ? __ffs(stop) - 1 : 32;
    const uint32_t del_before = first_stop == 32 ? del : (del & ((1u << first_stop) - 1u));
    if (reusable < 0 && del_before)
      reusable = static_cast<int32_t>(__shfl_sync(kFull, idx, __ffs(del_before) - 1));
    if (stop) {
      const int32_t at = static_cast<int32_t>(__shfl_sync(kFull, idx, first_stop));
      if ((hit >> first_stop) & 1u) found = at;
      else if (reusable < 0) reusable = at;
      return;
    }
  }
}

// children[parent][token] = child (edge length clen), claiming a slot as the
// host does; false when the table has no room.
AKV_DEV bool cmd_set_child(const TreeArrays& t, int32_t parent, int32_t token, int32_t child, int32_t clen, int lane) {
  int32_t found, reusable;
  cmd_probe(t, parent, token, lane, found, reusable);
  const int32_t s = found >= 0 ? found : reusable;
  if (s < 0) return false;
  if (lane == 0) t.slots_w[s] = make_int4(parent, token, child, clen);
  __syncwarp();
  return true;
}

AKV_DEV bool cmd_set_node(const TreeArrays& t, int32_t nid, int64_t off, int32_t len, int lane) {
  if (nid < 0 || nid >= t.n_nodes) return false;
  if (lane == 0) {
    t.off[nid] = off;
    t.len[nid] = len;
  }
  __syncwarp();
  return true;
}

__global__ void __launch_bounds__(32)
k_tree_commands(TreeArrays t, const int64_t* __restrict__ cmds, int32_t n_cmds, const int32_t* __restrict__ payload,
                int64_t payload_len, AkvStatus* st) {
  constexpr uint32_t kFull = 0xffffffffu;
  const int lane = threadIdx.x;
  for (int32_t c = 0; c < n_cmds; ++c) {
    const int64_t* cm = cmds + static_cast<int64_t>(kCmdWords) * c;
    const int64_t kind = cm[0];
    if (kind == kCmdPrune) {
      const int32_t parent = static_cast<int32_t>(cm[1]), nid = static_cast<int32_t>(cm[2]);
      if (nid < 0 || nid >= t.n_nodes) {
        if (lane == 0) akv_fail(st, AKV_ERR_TREE, c, nid, t.n_nodes);
        return;
      }
      const int64_t eo = t.off[nid];
      const int32_t el = t.len[nid];
      if (parent >= 0 && el > 0 && eo >= 0 && eo < t.token_cap) {
        int32_t found, reusable;
        cmd_probe(t, parent, t.tokens[eo], lane, found, reusable);
        if (found >= 0 && t.slots[found].z == nid) {
          if (lane == 0) t.slots_w[found] = make_int4(kSlotDeleted, 0, 0, 0);
          __syncwarp();
        }
      }
      cmd_set_node(t, nid, 0, 0, lane);
      continue;
    }
    if (kind != kCmdInsert) {
      if (lane == 0) akv_fail(st, AKV_ERR_TREE, c, static_cast<int32_t>(kind), 0);
      return;
    }
    int32_t node = static_cast<int32_t>(cm[1]);
    int32_t next_id = static_cast<int32_t>(cm[2]);
    const int64_t src = cm[3], n = cm[4];
    int64_t arena = cm[5];
    const int64_t block_size = cm[6];
    if (src < 0 || n < 0 || src + n > payload_len || arena < 0 || block_size < 1) {
      if (lane == 0) akv_fail(st, AKV_ERR_TREE, c, static_cast<int32_t>(n), 0, src);
      return;
    }
    const int32_t* __restrict__ toks = payload + src;
    // appends toks[pos, n) to the arena; its offset, or -1 without room
    auto append = [&](int64_t pos) -> int64_t {
      const int64_t m = n - pos, at = arena;
      if (at + m > t.token_cap) return -1;
      for (int64_t i = lane; i < m; i += 32) t.tokens[at + i] = toks[pos + i];
      __syncwarp();
      arena += m;
      return at;
    };
    bool ok = true;
    int64_t pos = 0;
    while (ok && pos < n) {
      const int32_t first = toks[pos];
      int32_t found, reusable;
      cmd_probe(t, node, first, lane, found, reusable);
      if (found < 0) {  // a new leaf under `node`
        const int64_t o = append(pos);
        ok = o >= 0 && cmd_set_node(t, next_id, o, static_cast<int32_t>(n - pos), lane) &&
             cmd_set_child(t, node, first, next_id, static_cast<int32_t>(n - pos), lane);
        break;
      }
      const int32_t child = t.slots[found].z;
      if (child < 0 || child >= t.n_nodes) {
        ok = false;
        break;
      }
      const int64_t co = t.off[child];
      const int32_t cl = t.len[child];
      if (co < 0 || co + cl > t.token_cap) {
        ok = false;
        break;
      }
      // common prefix of the child's edge and toks[pos, n)
      const int64_t lim = cl < n - pos ? cl : n - pos;
      int64_t common = lim;
      for (int64_t i0 = 0; i0 < lim; i0 += 32) {
        const int64_t i = i0 + lane;
        const uint32_t diff = __ballot_sync(kFull, i < lim && t.tokens[co + i] != toks[pos + i]);
        if (diff) {
          common = i0 + __ffs(diff) - 1;
          break;
        }
      }
      if (common == cl && common == n - pos) break;  // the same edge again: nothing moves
      if (common == cl) {                            // descend
        node = child;
        pos += common;
        continue;
      }
      const int64_t split = (common / block_size) * block_size;
      if (split == 0) {  // a new leaf takes the parent's slot for `first`
        const int64_t o = append(pos);
        ok = o >= 0 && cmd_set_node(t, next_id, o, static_cast<int32_t>(n - pos), lane) &&
             cmd_set_child(t, node, first, next_id, static_cast<int32_t>(n - pos), lane);
        break;
      }
      const int32_t mid = next_id++;
      ok = cmd_set_node(t, mid, co, static_cast<int32_t>(split), lane) &&
           cmd_set_node(t, child, co + split, static_cast<int32_t>(cl - split), lane) &&
           cmd_set_child(t, mid, t.tokens[co + split], child, static_cast<int32_t>(cl - split), lane) &&
           cmd_set_child(t, node, first, mid, static_cast<int32_t>(split), lane);
      if (!ok || split == n - pos) break;
      const int64_t o = append(pos + split);
      ok = o >= 0 && cmd_set_node(t, next_id, o, static_cast<int32_t>(n - pos - split), lane) &&
           cmd_set_child(t, mid, toks[pos + split], next_id, static_cast<int32_t>(n - pos - split), lane);
      break;
    }
    if (!ok) {
      if (lane == 0) akv_fail(st, AKV_ERR_TREE, c, node, next_id, pos);
      return;
    }
  }
}

__global__ void k_tree_apply(AkvTreeView tree, const int32_t* __restrict__ su, int32_t n_slot,
                             const int64_t* __restrict__ nu, int32_t n_node, AkvStatus* st) {
  int4* slots = reinterpret_cast<int4*>(const_cast<int32_t*>(tree.slots));
  int64_t* off = const_cast<int64_t*>(tree.node_edge_off);
  int32_t* len = const_cast<int32_t*>(tree.node_edge_len);
  const int32_t stride = gridDim.x * blockDim.x;
  for (int32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n_slot; i += stride) {
    const int32_t slot = su[5 * i];
    if (slot < 0 || slot > tree.slot_mask) {
      akv_fail(st, AKV_ERR_TREE, i, slot, tree.slot_mask);
      continue;
    }
    slots[slot] = make_int4(su[5 * i + 1], su[5 * i + 2], su[5 * i + 3], su[5 * i + 4]);
  }
  for (int32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n_node; i += stride) {
    const int64_t node = nu[3 * i];
    if (node < 0 || node >= tree.n_nodes) {
      akv_fail(st, AKV_ERR_TREE, i, static_cast<int32_t>(node), tree.n_nodes);
      continue;
    }
    off[node] = nu[3 * i + 1];
    len[node] = static_cast<int32_t>(nu[3 * i + 2]);
  }
}

}  // namespace

// Every (verify width, pipelining) instantiation, in one table: the entry
// points dispatch through it and akv_prepare loads it.
struct MatchKernels {
  int chunks;
  bool pipelined;
  decltype(&k_match<1, false>) whole;
  decltype(&k_match_split<1, false>) split;
};
#define AKV_MATCH_ROW(c, p) {c, p, &k_match<c, p>, &k_match_split<c, p>}
constexpr MatchKernels kMatchKernels[] = {
    AKV_MATCH_ROW(1, false), AKV_MATCH_ROW(2, false), AKV_MATCH_ROW(4, false), AKV_MATCH_ROW(8, false),
    AKV_MATCH_ROW(16, false), AKV_MATCH_ROW(2, true), AKV_MATCH_ROW(4, true), AKV_MATCH_ROW(8, true),
};
#undef AKV_MATCH_ROW

const MatchKernels* match_kernels(int32_t chunks) {
  const bool pipelined = (chunks & AKV_MATCH_PIPELINED) != 0;
  const int c = chunks & ~(AKV_MATCH_PIPELINED | AKV_MATCH_PREFETCH);
  for (const MatchKernels& k : kMatchKernels)
    if (k.chunks == c && k.pipelined == pipelined) return &k;
  return nullptr;
}

// The staged lookup's kernels, per window size.
struct StagedKernels {
  int32_t window;
  decltype(&k_match_chase<256>) chase;
  decltype(&k_match_verify<256>) verify;
};
constexpr StagedKernels kStagedKernels[] = {
    {256, &k_match_chase<256>, &k_match_verify<256>},
    {512, &k_match_chase<512>, &k_match_verify<512>},
    {1024, &k_match_chase<1024>, &k_match_verify<1024>},
};
constexpr int32_t kStagedDefaultWindow = 512;

const StagedKernels* staged_kernels(int32_t window_tokens) {
  const int32_t w = window_tokens == 0 ? kStagedDefaultWindow : window_tokens;
  for (const StagedKernels& k : kStagedKernels)
    if (k.window == w) return &k;
  return nullptr;
}

template <typename F>
int for_each_match_kernel(F&& f) {
  for (const MatchKernels& k : kMatchKernels) {
    if (int rc = f(reinterpret_cast<const void*>(k.whole), "akv_prepare: k_match")) return rc;
    if (int rc = f(reinterpret_cast<const void*>(k.split), "akv_prepare: k_match_split")) return rc;
  }
  for (const StagedKernels& k : kStagedKernels) {
    if (int rc = f(reinterpret_cast<const void*>(k.chase), "akv_prepare: k_match_chase")) return rc;
    if (int rc = f(reinterpret_cast<const void*>(k.verify), "akv_prepare: k_match_verify")) return rc;
  }
  return AKV_OK;
}

int akv_tree_prepare() {
#define AKV_LOAD(fn) if (int rc = akv_load_kernel(reinterpret_cast<const void*>(fn), "akv_prepare: " #fn)) return rc
  if (int rc = for_each_match_kernel([](const void* fn, const char* name) {
        return akv_load_kernel(fn, name);
      }))
    return rc;
  AKV_LOAD(k_tree_apply);
  AKV_LOAD(k_tree_commands);
#undef AKV_LOAD
  return AKV_OK;
}

extern "C" uint32_t akv_tree_hash(int32_t parent, int32_t token) {
  uint64_t k = (static_cast<uint64_t>(static_cast<uint32_t>(parent)) << 32) |
               static_cast<uint64_t>(static_cast<uint32_t>(token));
  k ^= k >> 33;
  k *= 0xff51afd7ed558ccdull;
  k ^= k >> 33;
  k *= 0xc4ceb9fe1a85ec53ull;
  k ^= k >> 33;
  return static_cast<uint32_t>(k);
}

extern "C" int akv_tree_apply(const AkvTreeView* tree, const int32_t* slot_updates, int32_t n_slot,
                              const int64_t* node_updates, int32_t n_node, AkvStatus* status,
                              void* stream) {
  AKV_ARG_CHECK(tree != nullptr && tree->slots && tree->node_edge_off && tree->node_edge_len,
                "akv_tree_apply: incomplete tree view");
  AKV_ARG_CHECK(n_slot >= 0 && n_node >= 0, "akv_tree_apply: negative count");
  AKV_ARG_CHECK(n_slot == 0 || slot_updates != nullptr, "akv_tree_apply: slot_updates is NULL");
  AKV_ARG_CHECK(n_node == 0 || node_updates != nullptr, "akv_tree_apply: node_updates is NULL");
  if (n_slot == 0 && n_node == 0) return AKV_OK;
  const int32_t work = n_slot > n_node ? n_slot : n_node;
  const int grid = std::min(akv_ceil_div(work, 256), kAkvSMs * 4);
  k_tree_apply<<<grid, 256, 0, akv_stream(stream)>>>(*tree, slot_updates, n_slot, node_updates,
                                                       n_node, status);
  AKV_LAUNCH_CHECK("akv_tree_apply");
  return AKV_OK;
}

namespace {

constexpr int32_t kSplitDefaultTokens = 1024;  // tokens per item (R)
constexpr int kSplitDefaultChunks = 4;        // 128 tokens compared per verify round
constexpr int kWholeDefaultChunks = 8;        // 256 (measured fastest on the match stress tree)

int match_args_ok(const AkvTreeView* tree, const int32_t* tokens, const int64_t* q_off, int32_t nq,
                  int32_t block_size, const int32_t* out_node, const int32_t* out_len, int32_t chunks,
                  const char* fn) {
  AKV_ARG_CHECK(tree != nullptr && tree->tokens && tree->node_edge_off && tree->node_edge_len &&
                    tree->slots,
                "%s: incomplete tree view", fn);
  AKV_ARG_CHECK(tree->n_nodes > 0, "%s: n_nodes=%d", fn, tree->n_nodes);
  AKV_ARG_CHECK(tree->run_head == nullptr ||
                    (tree->run_entries != nullptr && tree->n_runs > 0 && tree->run_nodes >= 0),
                "%s: run_head set without run_entries / n_runs (%d) / run_nodes (%d)", fn,
                tree->n_runs, tree->run_nodes);
  AKV_ARG_CHECK(tree->slot_mask >= 31 && ((tree->slot_mask + 1) & tree->slot_mask) == 0,
                "%s: slot count %d is not a power of two >= 32", fn, tree->slot_mask + 1);
  AKV_ARG_CHECK(nq >= 0, "%s: nq=%d < 0", fn, nq);
  AKV_ARG_CHECK(block_size > 0, "%s: block_size=%d", fn, block_size);
  AKV_ARG_CHECK((chunks & ~(AKV_MATCH_PIPELINED | AKV_MATCH_PREFETCH)) == 0 ||
                    match_kernels(chunks) != nullptr,
                "%s: chunks=%d is not a verify width (1, 2, 4, 8 or 16; 2, 4 or 8 with "
                "AKV_MATCH_PIPELINED)", fn, chunks);
  AKV_ARG_CHECK(nq == 0 || (tokens != nullptr && q_off != nullptr && out_node != nullptr &&
                            out_len != nullptr),
                "%s: NULL query or output array", fn);
  return AKV_OK;
}

}  // namespace

extern "C" int akv_match_prefix_variant(const AkvTreeView* tree, const int32_t* tokens,
                                        const int64_t* q_off, int32_t nq, int32_t block_size,
                                        int32_t* out_node, int32_t* out_len, int64_t* out_compared,
                                        const int32_t* order, AkvStatus* status, int32_t chunks,
                                        void* stream) {
  if (int rc = match_args_ok(tree, tokens, q_off, nq, block_size, out_node, out_len, chunks,
                             "akv_match_prefix"))
    return rc;
  if (nq == 0) return AKV_OK;
  if ((chunks & ~(AKV_MATCH_PIPELINED | AKV_MATCH_PREFETCH)) == 0) chunks |= kWholeDefaultChunks;
  const MatchKernels* k = match_kernels(chunks);
  const int grid = akv_ceil_div(nq, kWholeWarpsPerCta);
  k->whole<<<grid, kWholeWarpsPerCta * 32, 0, akv_stream(stream)>>>(*tree, tokens, q_off, nq, block_size, out_node,
                                                                    out_len, out_compared, order, status,
                                                                    (chunks & AKV_MATCH_PREFETCH) != 0);
  AKV_LAUNCH_CHECK("akv_match_prefix");
  return AKV_OK;
}

extern "C" int akv_match_prefix(const AkvTreeView* tree, const int32_t* tokens, const int64_t* q_off,
                                int32_t nq, int32_t block_size, int32_t* out_node,
                                int32_t* out_len, int64_t* out_compared, AkvStatus* status,
                                void* stream) {
  return akv_match_prefix_variant(tree, tokens, q_off, nq, block_size, out_node, out_len, out_compared,
                                  nullptr, status, 0, stream);
}

extern "C" int64_t akv_match_scratch_bytes(int32_t nq, int64_t n_tokens, int32_t tokens_per_range) {
  const int32_t R = tokens_per_range == 0 ? kSplitDefaultTokens : tokens_per_range;
  if (nq < 0 || n_tokens < 0 || R < 32 || R % 32 != 0) return -1;
  return split_scratch_bytes(nq, split_items_max(nq, n_tokens, R));
}

extern "C" int akv_match_split_plan(const int64_t* lengths, int32_t nq, int32_t tokens_per_range,
                                    int64_t* range_starts, int32_t* n_ranges) {
  AKV_ARG_CHECK(nq >= 0 && (nq == 0 || lengths != nullptr) && range_starts != nullptr && n_ranges != nullptr,
                "akv_match_split_plan: bad arguments");
  const int32_t R = tokens_per_range == 0 ? kSplitDefaultTokens : tokens_per_range;
  AKV_ARG_CHECK(R >= 32 && R % 32 == 0, "akv_match_split_plan: tokens_per_range=%d is not a multiple of 32",
                tokens_per_range);
  int64_t kmax = 1;
  for (int32_t i = 0; i < nq; ++i) {
    AKV_ARG_CHECK(lengths[i] >= 0 && (i == 0 || lengths[i] <= lengths[i - 1]),
                  "akv_match_split_plan: lengths must be >= 0 and longest first (entry %d)", i);
  }
  if (nq > 0) kmax = lengths[0] <= 0 ? 1 : (lengths[0] + R - 1) / R;
  AKV_ARG_CHECK(kmax <= kMaxSplitRanges,
                "akv_match_split_plan: a %lld-token query needs %lld ranges of %d (at most %d)",
                static_cast<long long>(nq > 0 ? lengths[0] : 0), static_cast<long long>(kmax), R,
                kMaxSplitRanges);
  // n_j = queries longer than j R (all of them for j = 0); lengths fall, so
  // each n_j is found by walking down from n_{j-1}
  range_starts[0] = 0;
  int32_t n_j = nq;
  for (int64_t j = 0; j < kmax; ++j) {
    if (j > 0)
      while (n_j > 0 && lengths[n_j - 1] <= j * R) --n_j;
    range_starts[j + 1] = range_starts[j] + n_j;
  }
  *n_ranges = static_cast<int32_t>(kmax);
  return AKV_OK;
}

extern "C" int akv_match_prefix_split(const AkvTreeView* tree, const int32_t* tokens, const int64_t* q_off,
                                      int32_t nq, int32_t block_size, int32_t* out_node, int32_t* out_len,
                                      int64_t* out_compared, const int32_t* order, const int64_t* range_starts,
                                      int32_t n_ranges, int32_t tokens_per_range, void* scratch,
                                      int64_t scratch_bytes, int32_t chunks, AkvStatus* status, void* stream) {
  if (int rc = match_args_ok(tree, tokens, q_off, nq, block_size, out_node, out_len, chunks,
                             "akv_match_prefix_split"))
    return rc;
  const int32_t R = tokens_per_range == 0 ? kSplitDefaultTokens : tokens_per_range;
  AKV_ARG_CHECK(R >= 32 && R % 32 == 0, "akv_match_prefix_split: tokens_per_range=%d is not a multiple of 32",
                tokens_per_range);
  if (nq == 0) return AKV_OK;
  AKV_ARG_CHECK(order != nullptr && range_starts != nullptr,
                "akv_match_prefix_split: order and range_starts are required");
  AKV_ARG_CHECK(n_ranges >= 1 && n_ranges <= kMaxSplitRanges, "akv_match_prefix_split: n_ranges=%d not in [1, %d]",
                n_ranges, kMaxSplitRanges);
  SplitRanges rg{};
  rg.n = n_ranges;
  rg.R = R;
  AKV_ARG_CHECK(range_starts[0] == 0 && range_starts[1] == nq,
                "akv_match_prefix_split: range_starts must begin 0, nq (%lld, %lld)",
                static_cast<long long>(range_starts[0]), static_cast<long long>(range_starts[1]));
  for (int32_t j = 0; j <= n_ranges; ++j) {
    rg.start[j] = range_starts[j];
    if (j >= 2) {
      const int64_t nj = range_starts[j] - range_starts[j - 1], nprev = range_starts[j - 1] - range_starts[j - 2];
      AKV_ARG_CHECK(nj >= 1 && nj <= nprev,
                    "akv_match_prefix_split: range %d holds %lld queries (range %d: %lld)", j - 1,
                    static_cast<long long>(nj), j - 2, static_cast<long long>(nprev));
    }
  }
  const int64_t w = rg.start[n_ranges];
  const int64_t need = split_scratch_bytes(nq, w);
  AKV_ARG_CHECK(scratch != nullptr && scratch_bytes >= need,
                "akv_match_prefix_split: scratch of %lld bytes, %lld needed", static_cast<long long>(scratch_bytes),
                static_cast<long long>(need));
  AKV_ARG_CHECK(reinterpret_cast<uintptr_t>(scratch) % 16 == 0,
                "akv_match_prefix_split: scratch is not 16-byte aligned");
  AKV_ARG_CHECK(w / kMatchWarpsPerCta < INT32_MAX, "akv_match_prefix_split: %lld ranges", static_cast<long long>(w));
  if ((chunks & ~(AKV_MATCH_PIPELINED | AKV_MATCH_PREFETCH)) == 0) chunks |= kSplitDefaultChunks;
  int4* stops = static_cast<int4*>(scratch);
  int32_t* done = reinterpret_cast<int32_t*>(static_cast<char*>(scratch) + 16 * w);
  // The counters' place depends on this batch's range count, so they are
  // cleared here (the stop records are written before they are read).
  const cudaError_t e = cudaMemsetAsync(done, 0, 4 * static_cast<size_t>(nq), akv_stream(stream));
  if (e != cudaSuccess) return akv_cuda_fail(e, "akv_match_prefix_split: clear counters");
  const int grid = akv_ceil_div(w, kMatchWarpsPerCta);
  match_kernels(chunks)->split<<<grid, kMatchWarpsPerCta * 32, 0, akv_stream(stream)>>>(
      *tree, tokens, q_off, nq, block_size, rg, order, stops, done, out_node, out_len, out_compared, status,
      (chunks & AKV_MATCH_PREFETCH) != 0);
  AKV_LAUNCH_CHECK("akv_match_prefix_split");
  return AKV_OK;
}

extern "C" int akv_tree_commands(const AkvTreeView* tree, int64_t token_cap, const int64_t* cmds, int32_t n_cmds,
                                 const int32_t* payload, int64_t payload_len, AkvStatus* status, void* stream) {
  AKV_ARG_CHECK(tree != nullptr && tree->tokens && tree->node_edge_off && tree->node_edge_len && tree->slots,
                "akv_tree_commands: incomplete tree view");
  AKV_ARG_CHECK(tree->slot_mask >= 31 && ((tree->slot_mask + 1) & tree->slot_mask) == 0,
                "akv_tree_commands: slot count %d is not a power of two >= 32", tree->slot_mask + 1);
  AKV_ARG_CHECK(n_cmds >= 0 && payload_len >= 0 && token_cap >= tree->n_tokens,
                "akv_tree_commands: n_cmds=%d payload_len=%lld token_cap=%lld", n_cmds,
                static_cast<long long>(payload_len), static_cast<long long>(token_cap));
  if (n_cmds == 0) return AKV_OK;
  AKV_ARG_CHECK(cmds != nullptr && (payload_len == 0 || payload != nullptr), "akv_tree_commands: NULL commands");
  TreeArrays t;
  t.tokens = const_cast<int32_t*>(tree->tokens);
  t.off = const_cast<int64_t*>(tree->node_edge_off);
  t.len = const_cast<int32_t*>(tree->node_edge_len);
  t.slots = reinterpret_cast<volatile int4*>(const_cast<int32_t*>(tree->slots));
  t.slots_w = reinterpret_cast<int4*>(const_cast<int32_t*>(tree->slots));
  t.token_cap = token_cap;
  t.n_nodes = tree->n_nodes;
  t.mask = tree->slot_mask;
  k_tree_commands<<<1, 32, 0, akv_stream(stream)>>>(t, cmds, n_cmds, payload, payload_len, status);
  AKV_LAUNCH_CHECK("akv_tree_commands");
  return AKV_OK;
}

extern "C" int64_t akv_match_staged_scratch_bytes(int32_t nq, int64_t n_tokens, int32_t window_tokens) {
  const StagedKernels* k = staged_kernels(window_tokens);
  if (k == nullptr || nq < 0 || n_tokens < 0 || n_tokens > INT32_MAX) return -1;
  return staged_layout(nullptr, nq, n_tokens, k->window, nullptr);
}

extern "C" int akv_match_prefix_staged(const AkvTreeView* tree, const int32_t* tokens, const int64_t* q_off,
                                       int32_t nq, int64_t n_tokens, int32_t block_size, int32_t* out_node,
                                       int32_t* out_len, int64_t* out_compared, const int32_t* order,
                                       int32_t window_tokens, void* scratch, int64_t scratch_bytes,
                                       AkvStatus* status, void* stream) {
  if (int rc = match_args_ok(tree, tokens, q_off, nq, block_size, out_node, out_len, 0,
                             "akv_match_prefix_staged"))
    return rc;
  const StagedKernels* k = staged_kernels(window_tokens);
  AKV_ARG_CHECK(k != nullptr, "akv_match_prefix_staged: window_tokens=%d is not 256, 512 or 1024",
                window_tokens);
  AKV_ARG_CHECK(n_tokens >= 0 && n_tokens <= INT32_MAX,
                "akv_match_prefix_staged: n_tokens=%lld not in [0, INT32_MAX]", static_cast<long long>(n_tokens));
  AKV_ARG_CHECK(tree->n_tokens <= INT32_MAX, "akv_match_prefix_staged: the tree holds %lld tokens (at most INT32_MAX)",
                static_cast<long long>(tree->n_tokens));
  if (nq == 0) return AKV_OK;
  AKV_ARG_CHECK(status != nullptr, "akv_match_prefix_staged: status is NULL");
  AKV_ARG_CHECK(scratch != nullptr && reinterpret_cast<uintptr_t>(scratch) % 256 == 0,
                "akv_match_prefix_staged: scratch is NULL or not 256-byte aligned");
  const int64_t need = staged_layout(nullptr, nq, n_tokens, k->window, nullptr);
  AKV_ARG_CHECK(scratch_bytes >= need, "akv_match_prefix_staged: scratch of %lld bytes, %lld needed",
                static_cast<long long>(scratch_bytes), static_cast<long long>(need));
  StagedScratch sc{};
  staged_layout(static_cast<char*>(scratch), nq, n_tokens, k->window, &sc);
  const int64_t n_slots = staged_slots(nq, n_tokens, k->window);
  cudaStream_t s = akv_stream(stream);
  k->chase<<<akv_ceil_div(nq, kMatchWarpsPerCta), kMatchWarpsPerCta * 32, 0, s>>>(
      *tree, tokens, q_off, nq, n_tokens, block_size, order, sc, out_node, out_len, out_compared, status);
  AKV_LAUNCH_CHECK("akv_match_prefix_staged(chase)");
  const int64_t grid = (n_slots + kMatchWarpsPerCta - 1) / kMatchWarpsPerCta;
  k->verify<<<static_cast<unsigned>(grid), kMatchWarpsPerCta * 32, 0, s>>>(
      *tree, tokens, n_slots, block_size, sc, out_node, out_len, out_compared, status);
  AKV_LAUNCH_CHECK("akv_match_prefix_staged(verify)");
  return AKV_OK;
}
