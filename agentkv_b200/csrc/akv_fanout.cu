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

}  // namespace

int akv_fanout_prepare() {
  return akv_load_kernel(reinterpret_cast<const void*>(k_fanout_plan), "akv_prepare: k_fanout_plan");
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
