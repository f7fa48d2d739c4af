// akv_fanout.cu — plan of one fork level on device-resident block tables.
//
// A Tree-of-Thought level forks each of P parents `fanout` times; every child
// then copy-on-writes the last block it inherited and appends `append` fresh
// blocks.  In the reference that is, per child in order, fork()
// (agentkv/core/radix_tree.py:222-264: inc_ref of every inherited block),
// ensure_mutable_block(child, -1) (:286-314: the block is shared, so alloc,
// copy_block, dec_ref) and `append` allocate_block() calls (:266-284).
//
// After a fork the last block always has refcount >= 2, so every child copies.
// No refcount reaches zero during the level, so the only order-sensitive
// state is which free ids each child receives: child c gets the (1+append)
// ids popped at positions (1+append)*c ... (1+append)*c + append — the CoW
// block first, then its appended blocks.  Given those ids (one
// akv_alloc_batch of (1+append)*fanout*P), this kernel writes in one launch:
//   child_tables / child_off  — each child's residual table
//   inc_ids                   — every parent block once per child (the forks)
//   pairs                     — (parent's last block, child's CoW block)
//   dec_ids                   — the parent's last block once per child
// which akv_incref_batch / akv_copy_blocks / akv_decref_batch then apply.
#include "akv_common.cuh"

namespace {

__global__ void k_fanout_plan(const int32_t* __restrict__ parent_tables,
                              const int64_t* __restrict__ parent_off, int32_t P, int32_t K,
                              int32_t A, const int32_t* __restrict__ fresh,
                              int32_t* __restrict__ child_tables, int64_t* __restrict__ child_off,
                              int32_t* __restrict__ inc_ids, int32_t* __restrict__ pairs,
                              int32_t* __restrict__ dec_ids) {
  const int64_t n_children = static_cast<int64_t>(P) * K;
  for (int64_t c = blockIdx.x; c < n_children; c += gridDim.x) {
    const int32_t p = static_cast<int32_t>(c / K);
    const int32_t k = static_cast<int32_t>(c - static_cast<int64_t>(p) * K);
    const int64_t base = parent_off[0];
    const int64_t lo = parent_off[p] - base;
    const int64_t Lp = parent_off[p + 1] - parent_off[p];
    if (Lp < 1) continue;  // a parent without residual blocks has nothing to copy-on-write
    const int32_t* __restrict__ src = parent_tables + lo;
    const int64_t coff = static_cast<int64_t>(K) * lo + static_cast<int64_t>(K) * A * p + k * (Lp + A);
    const int64_t ioff = static_cast<int64_t>(K) * lo + k * Lp;
    const int32_t* __restrict__ mine = fresh + static_cast<int64_t>(1 + A) * c;
    for (int64_t j = threadIdx.x; j < Lp; j += blockDim.x) {
      const int32_t b = src[j];
      child_tables[coff + j] = (j == Lp - 1) ? mine[0] : b;
      inc_ids[ioff + j] = b;
    }
    for (int64_t j = threadIdx.x; j < A; j += blockDim.x) child_tables[coff + Lp + j] = mine[1 + j];
    if (threadIdx.x == 0) {
      pairs[2 * c] = src[Lp - 1];
      pairs[2 * c + 1] = mine[0];
      dec_ids[c] = src[Lp - 1];
      child_off[c] = coff;
      if (c == n_children - 1) child_off[n_children] = coff + Lp + A;
    }
  }
}

// All levels of a fan-out in one launch, for append >= 1.  With appended
// blocks every child's table follows from the root's table and the fresh ids
// of its ancestors alone: for a child x at level l with ancestors a_0..a_l
// (a_l = x),
//   T(x) = root[:-1] ++ [cow(a_0)] ++ app(a_0)[:-1] ++ ... ++ [cow(a_l)] ++ app(a_l)
// (each child drops its parent's last block, an appended block, for its CoW
// copy and adds `append` blocks), so no level waits for the previous one.
// Child g (global index, levels back to back, (parent, child) order within
// a level) owns fresh ids [(1+A) g, (1+A)(g+1)): its CoW block, then its
// appended blocks — the ids the per-child calls take.  Child tables, pairs
// and dec_ref ids are laid out exactly as the per-level launches of
// k_fanout_plan would write them, level after level; the inc_ref ids (a
// multiset: their order does not change the batch's result) are
// position-major, see below.
struct TreeShape {
  int32_t levels, K, A, R;
  int64_t first[kAkvMaxFanoutLevels + 1];  // first global child of each level
  int64_t kpow[kAkvMaxFanoutLevels + 1];   // K^l
  int64_t tab_base[kAkvMaxFanoutLevels];   // level l's child tables in child_tables
  int64_t inc_base[kAkvMaxFanoutLevels + 1];  // level l's fork inc_ref ids in inc_ids; [levels] = total
};

__global__ void k_fanout_tree_plan(const int32_t* __restrict__ root_tables, const int64_t* __restrict__ root_off,
                                   const int32_t* __restrict__ fresh, TreeShape sh,
                                   int32_t* __restrict__ child_tables, int32_t* __restrict__ inc_ids,
                                   int32_t* __restrict__ pairs, int32_t* __restrict__ dec_ids) {
  const int64_t total = sh.first[sh.levels];
  const int32_t A = sh.A;
  const int64_t base = root_off[0];
  for (int64_t g = blockIdx.x; g < total; g += gridDim.x) {
    int l = 0;
    while (g >= sh.first[l + 1]) ++l;
    const int64_t c = g - sh.first[l];
    const int64_t per_root = sh.kpow[l + 1];
    const int32_t r = static_cast<int32_t>(c / per_root);
    const int64_t i_r = c - r * per_root;
    const int64_t lo = root_off[r] - base;
    const int64_t L0 = root_off[r + 1] - root_off[r];
    const int32_t* __restrict__ root = root_tables + lo;
    // fresh-id base of the ancestor at level m: (1+A) * (first[m] + c / K^(l-m))
    auto anc = [&](int m) -> int64_t { return (1 + A) * (sh.first[m] + c / sh.kpow[l - m]); };
    // element j of the table of the ancestor at level `top` (a table of
    // L0 + (top+1) A entries)
    auto elem = [&](int top, int64_t j) -> int32_t {
      if (j < L0 - 1) return root[j];
      const int64_t k = j - (L0 - 1);
      int64_t m = k / A, e = k - m * A;
      if (m > top) {
        m = top;
        e = A;
      }
      return fresh[anc(static_cast<int>(m)) + e];
    };
    const int64_t len_x = L0 + static_cast<int64_t>(l + 1) * A;
    const int64_t toff = sh.tab_base[l] + per_root * (lo + static_cast<int64_t>(r) * (l + 1) * A) + i_r * len_x;
    for (int64_t j = threadIdx.x; j < len_x; j += blockDim.x) child_tables[toff + j] = elem(l, j);
    if (threadIdx.x == 0) {
      const int32_t src = l == 0 ? root[L0 - 1] : fresh[anc(l - 1) + A];
      pairs[2 * g] = src;
      pairs[2 * g + 1] = fresh[anc(l)];
      dec_ids[g] = src;
    }
  }
  // The forks' inc_ref ids, position-major: within level l and root r, entry
  // j of every child's parent table in turn (children in order), so that the
  // children of one parent — and, for the root's blocks, all children of a
  // root — hold the same id in consecutive slots, which the inc_ref batch
  // folds into one atomic per warp.  Written in output order (coalesced).
  const int64_t n_inc = sh.inc_base[sh.levels];
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t o = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; o < n_inc; o += stride) {
    int l = 0;
    while (o >= sh.inc_base[l + 1]) ++l;
    const int64_t per_root = sh.kpow[l + 1];
    // root r's region starts at inc_base[l] + per_root (lo_r + r l A)
    int32_t r_lo = 0, r_hi = sh.R - 1;
    while (r_lo < r_hi) {
      const int32_t mid = (r_lo + r_hi + 1) >> 1;
      const int64_t start = sh.inc_base[l] + per_root * (root_off[mid] - base + static_cast<int64_t>(mid) * l * A);
      if (start <= o) r_lo = mid;
      else r_hi = mid - 1;
    }
    const int32_t r = r_lo;
    const int64_t lo = root_off[r] - base;
    const int64_t L0 = root_off[r + 1] - root_off[r];
    const int64_t rem = o - (sh.inc_base[l] + per_root * (lo + static_cast<int64_t>(r) * l * A));
    const int64_t j = rem / per_root, i_r = rem - j * per_root;
    const int32_t* __restrict__ root = root_tables + lo;
    int32_t v;
    if (l == 0 || j < L0 - 1) {
      v = root[j];
    } else {
      // the parent's table entry j (level l-1, ancestors of child c)
      const int64_t c = static_cast<int64_t>(r) * per_root + i_r;
      const int64_t k = j - (L0 - 1);
      int64_t m = k / A, e = k - m * A;
      if (m > l - 1) {
        m = l - 1;
        e = A;
      }
      v = fresh[(1 + A) * (sh.first[m] + c / sh.kpow[l - m]) + e];
    }
    inc_ids[o] = v;
  }
}

}  // namespace

int akv_fanout_prepare() {
  if (int rc = akv_load_kernel(reinterpret_cast<const void*>(k_fanout_tree_plan), "akv_prepare: k_fanout_tree_plan"))
    return rc;
  return akv_load_kernel(reinterpret_cast<const void*>(k_fanout_plan), "akv_prepare: k_fanout_plan");
}

extern "C" int akv_fanout_tree_plan(const int32_t* root_tables, const int64_t* root_off, int32_t n_roots,
                                    int64_t root_blocks, int32_t fanout, int32_t append, int32_t levels,
                                    const int32_t* fresh_ids, int32_t* child_tables, int32_t* inc_ids,
                                    int32_t* pairs, int32_t* dec_ids, void* stream) {
  AKV_ARG_CHECK(n_roots >= 0 && fanout >= 0 && levels >= 0 && root_blocks >= n_roots,
                "akv_fanout_tree_plan: roots=%d root_blocks=%lld fanout=%d levels=%d", n_roots,
                static_cast<long long>(root_blocks), fanout, levels);
  AKV_ARG_CHECK(append >= 1, "akv_fanout_tree_plan: append=%d (needs >= 1; use akv_fanout_plan per level)",
                append);
  AKV_ARG_CHECK(levels <= kAkvMaxFanoutLevels, "akv_fanout_tree_plan: %d levels > %d", levels,
                kAkvMaxFanoutLevels);
  if (n_roots == 0 || fanout == 0 || levels == 0) return AKV_OK;
  AKV_ARG_CHECK(root_tables && root_off && fresh_ids && child_tables && inc_ids && pairs && dec_ids,
                "akv_fanout_tree_plan: NULL array argument");
  TreeShape sh{};
  sh.levels = levels;
  sh.K = fanout;
  sh.A = append;
  sh.R = n_roots;
  sh.kpow[0] = 1;
  int64_t tab = 0, inc = 0;
  sh.first[0] = 0;
  for (int l = 0; l < levels; ++l) {
    sh.kpow[l + 1] = sh.kpow[l] * fanout;
    AKV_ARG_CHECK(sh.kpow[l + 1] * n_roots < (int64_t{1} << 31), "akv_fanout_tree_plan: too many children");
    const int64_t kids = sh.kpow[l + 1] * n_roots;
    sh.first[l + 1] = sh.first[l] + kids;
    sh.tab_base[l] = tab;
    sh.inc_base[l] = inc;
    tab += sh.kpow[l + 1] * (root_blocks + static_cast<int64_t>(n_roots) * (l + 1) * append);
    inc += sh.kpow[l + 1] * (root_blocks + static_cast<int64_t>(n_roots) * l * append);
  }
  sh.inc_base[levels] = inc;
  const int64_t total = sh.first[levels];
  const int grid = static_cast<int>(total < kAkvSMs * 8 ? total : kAkvSMs * 8);
  k_fanout_tree_plan<<<grid, 256, 0, akv_stream(stream)>>>(root_tables, root_off, fresh_ids, sh, child_tables,
                                                            inc_ids, pairs, dec_ids);
  AKV_LAUNCH_CHECK("akv_fanout_tree_plan");
  return AKV_OK;
}

extern "C" int akv_fanout_plan(const int32_t* parent_tables, const int64_t* parent_off, int32_t n_parents,
                               int32_t fanout, int32_t append, const int32_t* fresh_ids,
                               int32_t* child_tables, int64_t* child_off, int32_t* inc_ids,
                               int32_t* pairs, int32_t* dec_ids, void* stream) {
  AKV_ARG_CHECK(n_parents >= 0 && fanout >= 0 && append >= 0,
                "akv_fanout_plan: negative count (parents=%d fanout=%d append=%d)", n_parents, fanout,
                append);
  if (n_parents == 0 || fanout == 0) return AKV_OK;
  AKV_ARG_CHECK(parent_tables && parent_off && fresh_ids && child_tables && child_off && inc_ids &&
                    pairs && dec_ids,
                "akv_fanout_plan: NULL array argument");
  const int64_t n_children = static_cast<int64_t>(n_parents) * fanout;
  const int grid = static_cast<int>(n_children < kAkvSMs * 8 ? n_children : kAkvSMs * 8);
  k_fanout_plan<<<grid, 256, 0, akv_stream(stream)>>>(parent_tables, parent_off, n_parents, fanout,
                                                       append, fresh_ids, child_tables, child_off,
                                                       inc_ids, pairs, dec_ids);
  AKV_LAUNCH_CHECK("akv_fanout_plan");
  return AKV_OK;
}
