// akv_tree.cu — device replica of the shared radix tree and match_prefix.
//
// The host tree (SharedNode table, agentkv/core/radix_tree.py:82-103) is
// mirrored as flat arrays in HBM:
//   node_edge_off[id], node_edge_len[id] — each node's edge as a range of the
//       append-only token arena (an edge split only narrows ranges);
//   slots — every node's `children` dict (first edge token → child id) as one
//       open-addressing hash table keyed by (parent id, first token), 16 bytes
//       per slot, linear probing, -1 = empty, -2 = deleted.
// The host applies every tree mutation to its mirror and ships the changed
// slots / node ranges as a delta (akv_tree_apply); new edge tokens are
// appended to the arena with a plain copy.
//
// match_prefix runs one warp per query and restates
// DualRadixTree._match_prefix_locked (radix_tree.py:513-570):
//   from the root, look up the child keyed by the next query token; compare
//   the child's edge with the query (32 tokens per step, __ballot_sync +
//   __ffs find the first mismatch); stop on a missing child, a mismatch
//   anywhere in the edge or a query that ends inside the edge (a partial edge
//   earns no credit); otherwise descend.  The match is floored to the block
//   size; a zero match reports (-1, 0).
#include "akv_common.cuh"

namespace {

constexpr int kEmpty = -1;  // a deleted slot holds parent -2 and never matches
constexpr int kMatchWarpsPerCta = 8;

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

// Warp-cooperative lookup of (parent, token): each step reads 32 consecutive
// slots (512 B), the first matching lane wins; an empty slot before any match
// ends the probe.  Returns the child id or -1.
AKV_DEV int32_t warp_lookup(const int4* __restrict__ slots, int32_t mask, int32_t parent,
                            int32_t token, int lane) {
  const uint32_t h = tree_hash(parent, token);
  const int32_t windows = (mask >> 5) + 1;
  for (int32_t w = 0; w < windows; ++w) {
    const uint32_t idx = (h + static_cast<uint32_t>(w) * 32u + static_cast<uint32_t>(lane)) &
                         static_cast<uint32_t>(mask);
    const int4 s = __ldg(&slots[idx]);
    const uint32_t hit = __ballot_sync(0xffffffffu, s.x == parent && s.y == token);
    const uint32_t empty = __ballot_sync(0xffffffffu, s.x == kEmpty);
    if (hit) {
      // A key is only ever placed before the first empty slot of its probe.
      const int first_hit = __ffs(hit) - 1;
      const int first_empty = empty ? __ffs(empty) - 1 : 32;
      const int32_t c = __shfl_sync(0xffffffffu, s.z, first_hit);
      return first_hit < first_empty ? c : -1;
    }
    if (empty) return -1;
  }
  return -1;
}

__global__ void __launch_bounds__(kMatchWarpsPerCta * 32)
k_match(AkvTreeView tree, const int32_t* __restrict__ tokens, const int64_t* __restrict__ q_off,
        int32_t nq, int32_t block_size, int32_t* __restrict__ out_node,
        int32_t* __restrict__ out_len, int64_t* __restrict__ out_compared, AkvStatus* st) {
  const int lane = threadIdx.x & 31;
  const int32_t q = blockIdx.x * kMatchWarpsPerCta + (threadIdx.x >> 5);
  if (q >= nq) return;
  const int64_t qlo = q_off[q];
  const int64_t L = q_off[q + 1] - qlo;
  const int32_t* __restrict__ Q = tokens + qlo;
  const int4* __restrict__ slots = reinterpret_cast<const int4*>(tree.slots);
  int32_t cur = 0;  // ROOT_NODE_ID
  int64_t matched = 0, compared = 0;
  bool bad = false;
  while (matched < L) {
    const int32_t t = Q[matched];
    const int32_t child = warp_lookup(slots, tree.slot_mask, cur, t, lane);
    if (child < 0) break;
    if (child >= tree.n_nodes) {
      bad = true;
      if (lane == 0) akv_fail(st, AKV_ERR_TREE, q, child, tree.n_nodes);
      break;
    }
    const int64_t eoff = tree.node_edge_off[child];
    const int64_t elen = tree.node_edge_len[child];
    if (eoff < 0 || elen < 0 || eoff + elen > tree.n_tokens) {
      bad = true;
      if (lane == 0) akv_fail(st, AKV_ERR_TREE, q, child, static_cast<int32_t>(elen), eoff);
      break;
    }
    const int32_t* __restrict__ E = tree.tokens + eoff;
    const int32_t* __restrict__ Qm = Q + matched;
    const int64_t rem = L - matched;
    const int64_t lim = elen < rem ? elen : rem;
    int64_t em = lim;
    bool mismatch = false;
    // Two 32-token chunks per step keep two loads per array in flight.
    for (int64_t base = 0; base < lim; base += 64) {
      const int64_t i0 = base + lane, i1 = base + 32 + lane;
      const bool ok0 = i0 < lim, ok1 = i1 < lim;
      const int32_t a0 = ok0 ? Qm[i0] : 0, b0 = ok0 ? __ldg(&E[i0]) : 0;
      const int32_t a1 = ok1 ? Qm[i1] : 0, b1 = ok1 ? __ldg(&E[i1]) : 0;
      const uint32_t m0 = __ballot_sync(0xffffffffu, ok0 && a0 != b0);
      const uint32_t m1 = __ballot_sync(0xffffffffu, ok1 && a1 != b1);
      if (m0) {
        em = base + __ffs(m0) - 1;
        mismatch = true;
        break;
      }
      if (m1) {
        em = base + 32 + __ffs(m1) - 1;
        mismatch = true;
        break;
      }
    }
    // The reference evaluates `tokens[matched + i] != et` once per matched
    // token plus once for the token that differs.
    compared += em + (mismatch ? 1 : 0);
    if (em == 0 || em < elen) break;
    matched += elen;
    cur = child;
  }
  if (lane == 0) {
    int64_t m = bad ? 0 : (matched / block_size) * block_size;
    out_node[q] = m == 0 ? -1 : cur;
    out_len[q] = static_cast<int32_t>(m);
    if (out_compared != nullptr) out_compared[q] = compared;
  }
}

__global__ void k_tree_apply(AkvTreeView tree, const int32_t* __restrict__ su, int32_t n_slot,
                             const int64_t* __restrict__ nu, int32_t n_node, AkvStatus* st) {
  int4* slots = reinterpret_cast<int4*>(const_cast<int32_t*>(tree.slots));
  int64_t* off = const_cast<int64_t*>(tree.node_edge_off);
  int32_t* len = const_cast<int32_t*>(tree.node_edge_len);
  const int32_t stride = gridDim.x * blockDim.x;
  for (int32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n_slot; i += stride) {
    const int32_t slot = su[4 * i];
    if (slot < 0 || slot > tree.slot_mask) {
      akv_fail(st, AKV_ERR_TREE, i, slot, tree.slot_mask);
      continue;
    }
    slots[slot] = make_int4(su[4 * i + 1], su[4 * i + 2], su[4 * i + 3], 0);
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

extern "C" int akv_match_prefix(const AkvTreeView* tree, const int32_t* tokens, const int64_t* q_off,
                                int32_t nq, int32_t block_size, int32_t* out_node,
                                int32_t* out_len, int64_t* out_compared, AkvStatus* status,
                                void* stream) {
  AKV_ARG_CHECK(tree != nullptr && tree->tokens && tree->node_edge_off && tree->node_edge_len &&
                    tree->slots,
                "akv_match_prefix: incomplete tree view");
  AKV_ARG_CHECK(tree->n_nodes > 0, "akv_match_prefix: n_nodes=%d", tree->n_nodes);
  AKV_ARG_CHECK(tree->slot_mask >= 31 && ((tree->slot_mask + 1) & tree->slot_mask) == 0,
                "akv_match_prefix: slot count %d is not a power of two >= 32",
                tree->slot_mask + 1);
  AKV_ARG_CHECK(nq >= 0, "akv_match_prefix: nq=%d < 0", nq);
  AKV_ARG_CHECK(block_size > 0, "akv_match_prefix: block_size=%d", block_size);
  if (nq == 0) return AKV_OK;
  AKV_ARG_CHECK(tokens != nullptr && q_off != nullptr && out_node != nullptr && out_len != nullptr,
                "akv_match_prefix: NULL query or output array");
  const int grid = akv_ceil_div(nq, kMatchWarpsPerCta);
  k_match<<<grid, kMatchWarpsPerCta * 32, 0, akv_stream(stream)>>>(
      *tree, tokens, q_off, nq, block_size, out_node, out_len, out_compared, status);
  AKV_LAUNCH_CHECK("akv_match_prefix");
  return AKV_OK;
}
