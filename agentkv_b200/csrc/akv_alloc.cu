// akv_alloc.cu — the slab allocator's free list and refcounts on the device.
//
// State (all caller-owned device memory, see AkvAllocState):
//   ref[N]         refcounts                (slab_allocator.py:168-170)
//   ring[N]        free deque as a ring     (slab_allocator.py:173): ids live
//                  at ring[(left + i) mod N], i < size; alloc() pops the right
//                  end (:213), recycled ids are pushed on the left (:416-422)
//   limbo ids/tags retired ids not yet free, FIFO with three monotonic
//                  cursors head <= rel <= tail: [head, rel) is the reference's
//                  `_deferred_free` (released, drained to the free list at the
//                  next tick), [rel, tail) its reclaimer `_pending` queue
//                  (reclamation.py:74) with the epoch each id retired in.
//   ctl[16]        cursors and counters (AKV_CTL_*).
//
// Semantics restated from the reference (single-threaded order):
//   alloc   : pop right; ref = 1; tick                      (:194-220)
//   inc_ref : ref > 0 else error; ref += 1; tick            (:222-243)
//   dec_ref : ref > 0 else error; ref -= 1; at 0 retire; tick (:245-278)
//   retire  : pending.append((epoch, id)); try_retire       (reclamation.py:114-127)
//   try_retire: move pending ids with epoch < safe to deferred, FIFO, where
//             safe = min(reader epochs) or epoch + 1 when no reader (:147-173)
//   tick    : ops += 1; every epoch_interval ops maybe_advance (epoch += 1
//             unless a reader holds the current epoch; try_retire); then
//             drain deferred to the LEFT of the free list, keeping its order
//             (slab_allocator.py:424-437, 416-422)
// Consequences used by the batched kernels (the reader set is fixed during a
// batch, the host holds the allocator lock):
//   * with no reader, pending is always empty and every retirement reaches
//     the free list at its own tick, i.e. each recycled id is pushed left;
//   * with readers, try_retire inside a batch never releases anything, so
//     retirements only append to pending;
//   * whatever sat in deferred when the batch started is drained at the
//     batch's first tick — after op 0 has done its own pop / retire.
#include <algorithm>
#include <mutex>

#include "akv_common.cuh"

namespace {

constexpr int kCtlWords = 16;
enum : int {
  C_LEFT = AKV_CTL_FREE_LEFT,
  C_SIZE = AKV_CTL_FREE_SIZE,
  C_HEAD = AKV_CTL_LIMBO_HEAD,
  C_REL = AKV_CTL_LIMBO_REL,
  C_TAIL = AKV_CTL_LIMBO_TAIL,
  C_OPS = AKV_CTL_OPS,
  C_EPOCH = AKV_CTL_EPOCH,
  C_ALLOCS = AKV_CTL_ALLOCS,
  C_FREES = AKV_CTL_FREES,
  C_PEAK = AKV_CTL_PEAK,
  C_LAST_RETIRED = AKV_CTL_LAST_RETIRED,
  C_LAST_COPIED = AKV_CTL_LAST_COPIED,
  C_DONE = AKV_CTL_DONE,
  C_ADVANCES = AKV_CTL_ADVANCES,
  C_RELEASED = AKV_CTL_RELEASED,
};

// Dec_ref batches use a fixed number of CTAs, each owning a contiguous range
// of batch positions, so that CTA order is batch order.
constexpr int kDecThreads = 256;
constexpr int kDecMaxCtas = 2 * kAkvSMs * 2;  // 592
// Inc_ref / dec_ref batches of at most kSmallBatch ids run as one CTA of
// kSmallThreads in a single launch (instead of two / four launches over the
// grid): the per-call API's batches are a handful of ids.
constexpr int kSmallThreads = 512;
constexpr int32_t kSmallBatch = 2048;
// The CoW planner runs in one CTA over at most this many requests per launch.
constexpr int kCowThreads = 1024;
constexpr int kCowChunk = 4096;

AKV_DEV int64_t wrap(int64_t i, int64_t n) {
  int64_t r = i % n;
  return r < 0 ? r + n : r;
}

// Advances ops/epoch for n ticks starting from the batch's entry state.
AKV_DEV void apply_ticks(int64_t* ctl, int64_t n, const AkvTick& tk) {
  const int64_t ops = ctl[C_OPS];
  const int64_t iv = tk.epoch_interval;
  const bool allowed = !tk.readers_active || ctl[C_EPOCH] > tk.readers_max;
  if (allowed && n > 0) {
    const int64_t adv = (ops + n) / iv - ops / iv;
    ctl[C_EPOCH] += adv;
    ctl[C_ADVANCES] += adv;
  }
  ctl[C_OPS] = ops + n;
}

// Epoch in force when op p (0-based) of a batch starts.
AKV_DEV int64_t epoch_at(int64_t epoch0, int64_t ops0, int64_t p, const AkvTick& tk, bool allowed) {
  if (!allowed) return epoch0;
  const int64_t iv = tk.epoch_interval;
  return epoch0 + (ops0 + p) / iv - ops0 / iv;
}

// k-th id handed out by a run of pops whose first pop happens before the
// deferred ids are drained (k = 0 pops F's right end; later pops see
// merged = deferred ++ F[0 .. f-2]).
AKV_DEV int32_t popped_id(const int32_t* ring, const int32_t* limbo, int64_t n_blocks, int64_t left,
                          int64_t f, int64_t head, int64_t d, int64_t k) {
  if (k == 0) return ring[wrap(left + f - 1, n_blocks)];
  const int64_t m = (f - 1 + d) - k;  // index into merged, from its left
  if (m < d) return limbo[wrap(head + m, n_blocks)];
  return ring[wrap(left + (m - d), n_blocks)];
}

// Block-wide exclusive scan of one int per thread (blockDim.x <= 1024).
AKV_DEV int block_exclusive_scan(int v, int* warp_sums, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nwarps ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nwarps) warp_sums[lane] = w;  // inclusive
  }
  __syncthreads();
  const int before = (warp > 0 ? warp_sums[warp - 1] : 0) + x - v;
  total = warp_sums[nwarps - 1];
  __syncthreads();
  return before;
}

// "Last CTA finishes" handshake: returns true in exactly one CTA, after every
// CTA has passed this point.  No waiting involved.
AKV_DEV bool last_cta(int64_t* ctl) {
  __shared__ int is_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned long long prev =
        atomicAdd(reinterpret_cast<unsigned long long*>(&ctl[C_DONE]), 1ull);
    is_last = (prev == gridDim.x - 1) ? 1 : 0;
  }
  __syncthreads();
  if (is_last) {
    __threadfence();
    if (threadIdx.x == 0) ctl[C_DONE] = 0;
  }
  return is_last != 0;
}

// ── init ───────────────────────────────────────────────────────────────────
__global__ void k_init(AkvAllocState st) {
  const int64_t n = st.total_blocks;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    st.ref_counts[i] = 0;
    st.free_ring[i] = static_cast<int32_t>(i);
    st.limbo_ids[i] = -1;
    st.limbo_epochs[i] = 0;
    st.scratch_count[i] = 0;
    st.scratch_last[i] = 0;
  }
  if (blockIdx.x == 0 && threadIdx.x < kCtlWords) {
    int64_t v = 0;
    if (threadIdx.x == C_SIZE) v = n;
    st.ctl[threadIdx.x] = v;
  }
}

// ── alloc ──────────────────────────────────────────────────────────────────
__global__ void k_alloc(AkvAllocState st, int32_t n, int32_t* __restrict__ out, AkvTick tk,
                        AkvStatus* status) {
  if (akv_failed(status)) return;
  int64_t* ctl = st.ctl;
  const int64_t N = st.total_blocks;
  const int64_t left = ctl[C_LEFT], f = ctl[C_SIZE];
  const int64_t head = ctl[C_HEAD], d = ctl[C_REL] - head;
  if (f < 1 || f + d < n) {
    if (blockIdx.x == 0 && threadIdx.x == 0)
      akv_fail(status, AKV_ERR_EXHAUSTED, static_cast<int32_t>(f < 1 ? 0 : f + d), -1,
               static_cast<int32_t>(f));
    return;
  }
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  for (int64_t k = tid; k < n; k += stride) {
    const int32_t id = popped_id(st.free_ring, st.limbo_ids, N, left, f, head, d, k);
    out[k] = id;
    st.ref_counts[id] = 1;
  }
  // Drained deferred ids land just left of the old free region.
  for (int64_t j = tid; j < d; j += stride)
    st.free_ring[wrap(left - d + j, N)] = st.limbo_ids[wrap(head + j, N)];
  if (last_cta(ctl) && threadIdx.x == 0) {
    ctl[C_LEFT] = wrap(left - d, N);
    ctl[C_SIZE] = f + d - n;
    ctl[C_HEAD] = head + d;
    apply_ticks(ctl, n, tk);
    ctl[C_ALLOCS] += n;
    const int64_t cur = ctl[C_ALLOCS] - ctl[C_FREES];
    if (cur > ctl[C_PEAK]) ctl[C_PEAK] = cur;
  }
}

// ── inc_ref ────────────────────────────────────────────────────────────────
// Validation of ids [cta*blockDim + tid, n) strided over n_ctas CTAs; returns
// true when this thread found a bad id.
AKV_DEV bool incref_check_body(const AkvAllocState& st, const int32_t* __restrict__ ids, int32_t n,
                               int32_t cta, int32_t n_ctas, AkvStatus* status) {
  bool bad = false;
  for (int32_t k = cta * blockDim.x + threadIdx.x; k < n; k += n_ctas * blockDim.x) {
    const int32_t x = ids[k];
    if (static_cast<uint32_t>(x) >= static_cast<uint32_t>(st.total_blocks)) {
      akv_fail(status, AKV_ERR_OUT_OF_RANGE, k, x, st.total_blocks);
      bad = true;
      continue;
    }
    const int32_t r = st.ref_counts[x];
    if (r <= 0) {
      akv_fail(status, AKV_ERR_NOT_ALLOCATED, k, x, r);
      bad = true;
    }
  }
  return bad;
}

// The increments and the drain of the deferred ids, strided over n_ctas CTAs
// (the cursors are read by every thread before any CTA moves them).
AKV_DEV void incref_apply_body(const AkvAllocState& st, const int32_t* __restrict__ ids, int32_t n,
                               int64_t left, int64_t head, int64_t d, int32_t cta, int32_t n_ctas) {
  const int64_t N = st.total_blocks;
  const int64_t stride = static_cast<int64_t>(n_ctas) * blockDim.x;
  const int64_t tid = cta * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  // Warp-aggregated increments: lanes holding the same id add their count
  // with one atomic (a fork increments every inherited block once per child,
  // so a batch repeats ids; the fan-out planner lists them so that equal ids
  // share warps).  The loop is warp-uniform: stride is a multiple of 32.
  const int lane = threadIdx.x & 31;
  for (int64_t k0 = tid - lane; k0 < n; k0 += stride) {
    const int64_t k = k0 + lane;
    const int32_t x = k < n ? ids[k] : -1;
    const uint32_t peers = __match_any_sync(0xffffffffu, x);
    if (x >= 0 && lane == __ffs(peers) - 1) atomicAdd(&st.ref_counts[x], __popc(peers));
  }
  for (int64_t j = tid; j < d; j += stride)
    st.free_ring[wrap(left - d + j, N)] = st.limbo_ids[wrap(head + j, N)];
}

AKV_DEV void incref_finish(int64_t* ctl, int32_t n, int64_t left, int64_t head, int64_t d, int64_t N,
                           const AkvTick& tk) {
  ctl[C_LEFT] = wrap(left - d, N);
  ctl[C_SIZE] += d;
  ctl[C_HEAD] = head + d;
  apply_ticks(ctl, n, tk);
}

__global__ void k_incref_check(AkvAllocState st, const int32_t* __restrict__ ids, int32_t n,
                               AkvStatus* status) {
  if (akv_failed(status)) return;
  incref_check_body(st, ids, n, blockIdx.x, gridDim.x, status);
}

__global__ void k_incref_apply(AkvAllocState st, const int32_t* __restrict__ ids, int32_t n,
                               AkvTick tk, AkvStatus* status) {
  if (akv_failed(status)) return;
  int64_t* ctl = st.ctl;
  const int64_t left = ctl[C_LEFT], head = ctl[C_HEAD], d = ctl[C_REL] - head;
  incref_apply_body(st, ids, n, left, head, d, blockIdx.x, gridDim.x);
  if (last_cta(ctl) && threadIdx.x == 0) incref_finish(ctl, n, left, head, d, st.total_blocks, tk);
}

// Batches of at most kSmallBatch ids: check and apply in one CTA, one launch.
__global__ void __launch_bounds__(kSmallThreads)
k_incref_small(AkvAllocState st, const int32_t* __restrict__ ids, int32_t n, AkvTick tk,
               AkvStatus* status) {
  if (akv_failed(status)) return;
  const bool bad = incref_check_body(st, ids, n, 0, 1, status);
  if (__syncthreads_or(bad)) return;
  int64_t* ctl = st.ctl;
  const int64_t left = ctl[C_LEFT], head = ctl[C_HEAD], d = ctl[C_REL] - head;
  incref_apply_body(st, ids, n, left, head, d, 0, 1);
  __syncthreads();  // every thread has read the cursors
  if (threadIdx.x == 0) incref_finish(ctl, n, left, head, d, st.total_blocks, tk);
}

// ── dec_ref ────────────────────────────────────────────────────────────────
// Layout of the plan that the dec_ref stages share (in the aux words of the
// allocator's scratch, or in shared memory for the single-CTA form).
struct DecPlan {
  int64_t left_new;     // ring index of the new leftmost free id
  int64_t n_ret;        // retirements in this batch
  int64_t z;            // 1 when position 0 retires (no-reader case)
  int64_t d;            // deferred ids drained at tick 0
  int64_t head;         // limbo head before the batch
  int64_t tail;         // limbo tail before the batch
  int64_t epoch0, ops0;
  int32_t readers, allowed;
};

// Stage 1: per-id occurrence count and last position (1-based), strided over
// n_ctas CTAs.  Warp-aggregated: lanes holding the same id add their count
// with one atomic, and the highest of them (the latest position) sets the
// last position.  The loop is warp-uniform (blockDim.x is a multiple of 32).
AKV_DEV void dec_count_body(const AkvAllocState& st, const int32_t* __restrict__ ids, int32_t n,
                            int32_t cta, int32_t n_ctas, AkvStatus* status) {
  const int lane = threadIdx.x & 31;
  const int32_t stride = n_ctas * blockDim.x;
  for (int32_t k0 = cta * blockDim.x + threadIdx.x - lane; k0 < n; k0 += stride) {
    const int32_t k = k0 + lane;
    int32_t x = k < n ? ids[k] : -1;
    if (k < n && static_cast<uint32_t>(x) >= static_cast<uint32_t>(st.total_blocks)) {
      akv_fail(status, AKV_ERR_OUT_OF_RANGE, k, x, st.total_blocks);
      x = -1;
    }
    const uint32_t peers = __match_any_sync(0xffffffffu, x);
    if (x >= 0 && lane == 31 - __clz(peers)) {
      atomicAdd(&st.scratch_count[x], __popc(peers));
      atomicMax(&st.scratch_last[x], k + 1);
    }
  }
}

// Stage 2: validate positions [lo, hi) at last occurrences; returns the
// retirements among them (to every thread).
AKV_DEV int dec_flag_body(const AkvAllocState& st, const int32_t* __restrict__ ids, int32_t lo,
                          int32_t hi, AkvStatus* status, int* ws) {
  int local = 0;
  if (!akv_failed(status)) {
    for (int32_t k = lo + threadIdx.x; k < hi; k += blockDim.x) {
      const int32_t x = ids[k];
      if (static_cast<uint32_t>(x) >= static_cast<uint32_t>(st.total_blocks)) continue;
      if (st.scratch_last[x] != k + 1) continue;
      const int32_t c = st.scratch_count[x], r = st.ref_counts[x];
      if (c > r) {
        akv_fail(status, AKV_ERR_DOUBLE_FREE, k, x, r);
        continue;
      }
      local += (c == r);
    }
  }
  int total;
  block_exclusive_scan(local, ws, total);
  return total;
}

// Stage 3 (one thread): the new cursors and the plan for stage 4, given the
// batch's n_ret retirements.
AKV_DEV DecPlan dec_plan_body(const AkvAllocState& st, int32_t n, int64_t n_ret,
                              const int32_t* __restrict__ ids, const AkvTick& tk) {
  int64_t* ctl = st.ctl;
  const int64_t N = st.total_blocks;
  const int64_t left = ctl[C_LEFT], f = ctl[C_SIZE];
  const int64_t head = ctl[C_HEAD], rel = ctl[C_REL], tail = ctl[C_TAIL];
  const int64_t d = rel - head;
  // Does position 0 retire?
  int64_t z = 0;
  {
    const int32_t x0 = ids[0];
    if (static_cast<uint32_t>(x0) < static_cast<uint32_t>(N) && st.scratch_last[x0] == 1 &&
        st.scratch_count[x0] == st.ref_counts[x0])
      z = 1;
  }
  DecPlan p;
  p.n_ret = n_ret;
  p.z = z;
  p.d = d;
  p.head = head;
  p.tail = tail;
  p.epoch0 = ctl[C_EPOCH];
  p.ops0 = ctl[C_OPS];
  p.readers = tk.readers_active;
  p.allowed = (!tk.readers_active || ctl[C_EPOCH] > tk.readers_max) ? 1 : 0;
  if (!tk.readers_active) {
    // No reader: every retirement passes straight through the reclaimer's
    // release (_try_retire counts it in _freed_count) to the free list.
    p.left_new = wrap(left - d - n_ret, N);
    ctl[C_LEFT] = p.left_new;
    ctl[C_SIZE] = f + d + n_ret;
    ctl[C_HEAD] = rel;
    ctl[C_RELEASED] += n_ret;
  } else {
    p.left_new = wrap(left - d, N);
    ctl[C_LEFT] = p.left_new;
    ctl[C_SIZE] = f + d;
    ctl[C_HEAD] = rel;
    ctl[C_TAIL] = tail + n_ret;
  }
  apply_ticks(ctl, n, tk);
  ctl[C_FREES] += n_ret;
  ctl[C_LAST_RETIRED] = n_ret;
  return p;
}

// Stage 4: place the retirements of positions [lo, hi) (numbered from
// q_base in batch order), apply the refcounts, clear the scratch; then drain
// the deferred ids, strided over n_ctas CTAs.  n_ret < 0 (an error) only
// clears the scratch.
AKV_DEV void dec_apply_body(const AkvAllocState& st, const int32_t* __restrict__ ids, int32_t lo,
                            int32_t hi, int64_t q_base, const DecPlan& p,
                            int32_t* __restrict__ retired_out, const AkvTick& tk, int32_t cta,
                            int32_t n_ctas, int* ws) {
  const int64_t N = st.total_blocks;
  const bool apply = p.n_ret >= 0;
  for (int32_t base = lo; base < hi; base += blockDim.x) {
    const int32_t k = base + threadIdx.x;
    int32_t x = -1, c = 0, r = 0;
    bool last = false;
    if (k < hi) {
      x = ids[k];
      if (static_cast<uint32_t>(x) < static_cast<uint32_t>(N) && st.scratch_last[x] == k + 1) {
        last = true;
        c = st.scratch_count[x];
        r = st.ref_counts[x];
      }
    }
    const int flag = (apply && last && c == r) ? 1 : 0;
    int total;
    const int ex = block_exclusive_scan(flag, ws, total);
    if (last) {
      if (apply) {
        st.ref_counts[x] = r - c;
        if (flag) {
          const int64_t q = q_base + ex;  // retirement number in batch order
          if (retired_out != nullptr) retired_out[q] = x;
          if (!p.readers) {
            int64_t slot;  // offset from the new leftmost free slot
            if (q == 0 && p.z) slot = p.n_ret - 1 + p.d;
            else slot = p.n_ret - 1 - q;
            st.free_ring[wrap(p.left_new + slot, N)] = x;
          } else {
            const int64_t pos = wrap(p.tail + q, N);
            st.limbo_ids[pos] = x;
            st.limbo_epochs[pos] = epoch_at(p.epoch0, p.ops0, k, tk, p.allowed != 0);
          }
        }
      }
      st.scratch_count[x] = 0;
      st.scratch_last[x] = 0;
    }
    q_base += total;
  }
  if (!apply) return;
  // Deferred ids from before the batch: right of the retirements pushed after
  // op 0, left of op 0's own retirement (no-reader case); at the far left when
  // readers keep new retirements pending.
  const int64_t dstart = p.readers ? 0 : (p.n_ret - p.z);
  const int64_t stride = static_cast<int64_t>(n_ctas) * blockDim.x;
  for (int64_t j = cta * static_cast<int64_t>(blockDim.x) + threadIdx.x; j < p.d; j += stride)
    st.free_ring[wrap(p.left_new + dstart + j, N)] = st.limbo_ids[wrap(p.head + j, N)];
}

// K1: count.
__global__ void k_dec_count(AkvAllocState st, const int32_t* __restrict__ ids, int32_t n,
                            AkvStatus* status) {
  if (akv_failed(status)) return;
  dec_count_body(st, ids, n, blockIdx.x, gridDim.x, status);
}

// K2: validate at last occurrences, count retirements per CTA.
__global__ void __launch_bounds__(kDecThreads)
k_dec_flag(AkvAllocState st, const int32_t* __restrict__ ids, int32_t n, int32_t chunk,
           int32_t* __restrict__ cta_counts, AkvStatus* status) {
  const int32_t lo = blockIdx.x * chunk;
  const int32_t hi = min(n, lo + chunk);
  __shared__ int ws[32];
  const int total = dec_flag_body(st, ids, lo, hi, status, ws);
  if (threadIdx.x == 0) cta_counts[blockIdx.x] = total;
}

// K3: one CTA — offsets per CTA, new cursors, plan for K4.
__global__ void k_dec_plan(AkvAllocState st, int32_t n, int32_t n_ctas, int32_t* __restrict__ cta_counts,
                           const int32_t* __restrict__ ids, DecPlan* plan, AkvTick tk,
                           AkvStatus* status) {
  __shared__ int ws[32];
  __shared__ int64_t carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  // Exclusive scan of cta_counts in place (n_ctas <= kDecMaxCtas).
  for (int base = 0; base < n_ctas; base += blockDim.x) {
    const int i = base + threadIdx.x;
    const int v = i < n_ctas ? cta_counts[i] : 0;
    int total;
    const int ex = block_exclusive_scan(v, ws, total);
    if (i < n_ctas) cta_counts[i] = static_cast<int>(carry) + ex;
    __syncthreads();
    if (threadIdx.x == 0) carry += total;
    __syncthreads();
  }
  if (threadIdx.x != 0) return;
  if (akv_failed(status)) {
    plan->n_ret = -1;  // K4 only clears scratch
    return;
  }
  *plan = dec_plan_body(st, n, carry, ids, tk);
}

// K4: place retirements, apply refcounts, drain deferred, clear scratch.
__global__ void __launch_bounds__(kDecThreads)
k_dec_apply(AkvAllocState st, const int32_t* __restrict__ ids, int32_t n, int32_t chunk,
            const int32_t* __restrict__ cta_offsets, const DecPlan* __restrict__ plan_p,
            int32_t* __restrict__ retired_out, AkvTick tk) {
  const DecPlan p = *plan_p;
  const int32_t lo = blockIdx.x * chunk;
  const int32_t hi = min(n, lo + chunk);
  __shared__ int ws[32];
  const int64_t q_base = p.n_ret >= 0 ? cta_offsets[blockIdx.x] : 0;
  dec_apply_body(st, ids, lo, hi, q_base, p, retired_out, tk, blockIdx.x, gridDim.x, ws);
}

// Batches of at most kSmallBatch ids: the four stages in one CTA, one launch.
// __syncthreads between the stages makes each stage's global writes (the
// scratch atomics, the cursors) visible to the next.
__global__ void __launch_bounds__(kSmallThreads)
k_dec_small(AkvAllocState st, const int32_t* __restrict__ ids, int32_t n,
            int32_t* __restrict__ retired_out, AkvTick tk, AkvStatus* status) {
  __shared__ int ws[32];
  __shared__ DecPlan plan;
  if (akv_failed(status)) return;  // nothing counted, nothing to clear
  dec_count_body(st, ids, n, 0, 1, status);
  __syncthreads();
  const int n_ret = dec_flag_body(st, ids, 0, n, status, ws);
  if (threadIdx.x == 0) {
    if (akv_failed(status)) plan.n_ret = -1;  // stage 4 only clears scratch
    else plan = dec_plan_body(st, n, n_ret, ids, tk);
  }
  __syncthreads();
  const DecPlan p = plan;
  dec_apply_body(st, ids, 0, n, 0, p, retired_out, tk, 0, 1, ws);
}

// ── reclaimer ──────────────────────────────────────────────────────────────
// Releases pending ids with epoch < safe (FIFO prefix; epochs are
// non-decreasing along the queue).
AKV_DEV void try_retire(AkvAllocState& st, int64_t safe) {
  int64_t* ctl = st.ctl;
  const int64_t N = st.total_blocks;
  int64_t lo = ctl[C_REL], hi = ctl[C_TAIL];
  const int64_t rel0 = lo;
  while (lo < hi) {  // first index with epoch >= safe
    const int64_t mid = lo + (hi - lo) / 2;
    if (st.limbo_epochs[wrap(mid, N)] < safe) lo = mid + 1;
    else hi = mid;
  }
  ctl[C_REL] = lo;
  ctl[C_RELEASED] += lo - rel0;
}

__global__ void k_release(AkvAllocState st, int64_t safe) {
  if (blockIdx.x == 0 && threadIdx.x == 0) try_retire(st, safe);
}

__global__ void k_advance(AkvAllocState st, AkvTick tk) {
  if (blockIdx.x != 0 || threadIdx.x != 0) return;
  int64_t* ctl = st.ctl;
  if (!tk.readers_active || ctl[C_EPOCH] > tk.readers_max) {
    ctl[C_EPOCH] += 1;
    ctl[C_ADVANCES] += 1;
  }
  const int64_t safe = tk.readers_active ? tk.readers_min : ctl[C_EPOCH] + 1;
  try_retire(st, safe);
}

// ── copy-on-write planner ──────────────────────────────────────────────────
// One CTA over n <= kCowChunk requests in order.  Request i on block x copies
// iff ref[x] - (copies of x by earlier requests) > 1, i.e. iff its rank among
// the requests on x is < ref[x] - 1.
__global__ void __launch_bounds__(kCowThreads)
k_cow_plan(AkvAllocState st, const int32_t* __restrict__ blocks, int32_t n,
           int32_t* __restrict__ out_blocks, int32_t* __restrict__ out_copied,
           int32_t* __restrict__ pairs, AkvTick tk, AkvStatus* status) {
  __shared__ int32_t s_blk[kCowChunk];
  __shared__ int ws[32];
  __shared__ int s_fail;
  __shared__ int64_t s_left, s_f, s_head, s_d;
  constexpr int kPer = kCowChunk / kCowThreads;  // requests per thread (contiguous)
  if (threadIdx.x == 0) s_fail = akv_failed(status) ? 1 : 0;
  __syncthreads();
  if (s_fail) {
    if (threadIdx.x == 0) st.ctl[C_LAST_COPIED] = 0;
    return;
  }
  const int64_t N = st.total_blocks;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int32_t x = blocks[i];
    s_blk[i] = x;
    if (static_cast<uint32_t>(x) >= static_cast<uint32_t>(N)) {
      akv_fail(status, AKV_ERR_OUT_OF_RANGE, i, x, static_cast<int32_t>(N));
      s_fail = 1;
    } else {
      atomicAdd(&st.scratch_count[x], 1);
    }
  }
  __syncthreads();
  if (s_fail) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const int32_t x = s_blk[i];
      if (static_cast<uint32_t>(x) < static_cast<uint32_t>(N)) st.scratch_count[x] = 0;
    }
    if (threadIdx.x == 0) st.ctl[C_LAST_COPIED] = 0;
    return;
  }
  // Decide per request; thread t owns requests [t*kPer, t*kPer + kPer).
  int copy_flags = 0, local = 0;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int i = threadIdx.x * kPer + j;
    if (i >= n) break;
    const int32_t x = s_blk[i];
    const int32_t c = st.scratch_count[x];
    const int32_t r = st.ref_counts[x];
    const int32_t q = r > 1 ? r - 1 : 0;  // copies x can take in this batch
    bool cp;
    if (c <= q) {
      cp = q > 0;
    } else {
      int rank = 0;  // contested block: count earlier requests on x
      for (int jj = 0; jj < i; ++jj) rank += (s_blk[jj] == x);
      cp = rank < q;
    }
    if (cp) {
      copy_flags |= 1 << j;
      ++local;
    }
  }
  int n_copies;
  const int slot0 = block_exclusive_scan(local, ws, n_copies);
  if (threadIdx.x == 0) {
    int64_t* ctl = st.ctl;
    s_left = ctl[C_LEFT];
    s_f = ctl[C_SIZE];
    s_head = ctl[C_HEAD];
    s_d = ctl[C_REL] - s_head;
    if (n_copies > 0 && (s_f < 1 || s_f + s_d < n_copies)) {
      akv_fail(status, AKV_ERR_EXHAUSTED, 0, -1, static_cast<int32_t>(s_f));
      s_fail = 1;
    }
  }
  __syncthreads();
  if (!s_fail) {
    int slot = slot0;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int i = threadIdx.x * kPer + j;
      if (i >= n) break;
      const int32_t x = s_blk[i];
      if (copy_flags & (1 << j)) {
        const int32_t fresh =
            popped_id(st.free_ring, st.limbo_ids, N, s_left, s_f, s_head, s_d, slot);
        st.ref_counts[fresh] = 1;
        atomicSub(&st.ref_counts[x], 1);
        pairs[2 * slot] = x;
        pairs[2 * slot + 1] = fresh;
        out_blocks[i] = fresh;
        out_copied[i] = 1;
        ++slot;
      } else {
        out_blocks[i] = x;
        out_copied[i] = 0;
      }
    }
    if (n_copies > 0)
      for (int64_t j = threadIdx.x; j < s_d; j += blockDim.x)
        st.free_ring[wrap(s_left - s_d + j, N)] = st.limbo_ids[wrap(s_head + j, N)];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) st.scratch_count[s_blk[i]] = 0;
  if (threadIdx.x == 0) {
    int64_t* ctl = st.ctl;
    if (s_fail) {
      ctl[C_LAST_COPIED] = 0;
    } else {
      ctl[C_LAST_COPIED] = n_copies;
      if (n_copies > 0) {
        ctl[C_LEFT] = wrap(s_left - s_d, N);
        ctl[C_SIZE] = s_f + s_d - n_copies;
        ctl[C_HEAD] = s_head + s_d;
        apply_ticks(ctl, 2 * static_cast<int64_t>(n_copies), tk);
        ctl[C_ALLOCS] += n_copies;
        const int64_t cur = ctl[C_ALLOCS] - ctl[C_FREES];
        if (cur > ctl[C_PEAK]) ctl[C_PEAK] = cur;
      }
    }
  }
}

bool state_ok(const AkvAllocState* st) {
  return st != nullptr && st->ref_counts && st->free_ring && st->limbo_ids && st->limbo_epochs &&
         st->ctl && st->scratch_count && st->scratch_last && st->scratch_aux &&
         st->total_blocks > 0;
}

int grid_for(int64_t work, int threads, int max_ctas) {
  int64_t g = (work + threads - 1) / threads;
  if (g < 1) g = 1;
  if (g > max_ctas) g = max_ctas;
  return static_cast<int>(g);
}

}  // namespace

int akv_alloc_prepare() {
#define AKV_LOAD(fn) if (int rc = akv_load_kernel(reinterpret_cast<const void*>(fn), "akv_prepare: " #fn)) return rc
  AKV_LOAD(k_init);
  AKV_LOAD(k_alloc);
  AKV_LOAD(k_incref_check);
  AKV_LOAD(k_incref_apply);
  AKV_LOAD(k_dec_count);
  AKV_LOAD(k_dec_flag);
  AKV_LOAD(k_dec_plan);
  AKV_LOAD(k_dec_apply);
  AKV_LOAD(k_incref_small);
  AKV_LOAD(k_dec_small);
  AKV_LOAD(k_release);
  AKV_LOAD(k_advance);
  AKV_LOAD(k_cow_plan);
#undef AKV_LOAD
  return AKV_OK;
}

// Shared with the block-movement launcher in akv_blocks.cu.
int akv_launch_copy_counted(void* pool, int64_t bpb, int32_t total, const int32_t* pairs,
                            int32_t n_max, const int64_t* n_dev, AkvStatus* st, cudaStream_t s);

// ── C ABI ───────────────────────────────────────────────────────────────────
extern "C" int akv_alloc_init(const AkvAllocState* st, void* stream) {
  AKV_ARG_CHECK(state_ok(st), "akv_alloc_init: incomplete allocator state");
  k_init<<<grid_for(st->total_blocks, 256, kAkvSMs * 8), 256, 0, akv_stream(stream)>>>(*st);
  AKV_LAUNCH_CHECK("akv_alloc_init");
  return AKV_OK;
}

extern "C" int akv_alloc_batch(const AkvAllocState* st, int32_t n, int32_t* out_ids,
                               const AkvTick* tick, AkvStatus* status, void* stream) {
  AKV_ARG_CHECK(state_ok(st), "akv_alloc_batch: incomplete allocator state");
  AKV_ARG_CHECK(tick != nullptr && tick->epoch_interval > 0, "akv_alloc_batch: bad tick");
  AKV_ARG_CHECK(status != nullptr, "akv_alloc_batch: status is NULL");
  AKV_ARG_CHECK(n >= 0, "akv_alloc_batch: n=%d < 0", n);
  if (n == 0) return AKV_OK;
  AKV_ARG_CHECK(out_ids != nullptr, "akv_alloc_batch: out_ids is NULL");
  k_alloc<<<grid_for(std::max<int64_t>(n, 1), 256, kAkvSMs * 4), 256, 0, akv_stream(stream)>>>(
      *st, n, out_ids, *tick, status);
  AKV_LAUNCH_CHECK("akv_alloc_batch");
  return AKV_OK;
}

extern "C" int akv_incref_batch(const AkvAllocState* st, const int32_t* ids, int32_t n,
                                const AkvTick* tick, AkvStatus* status, void* stream) {
  AKV_ARG_CHECK(state_ok(st), "akv_incref_batch: incomplete allocator state");
  AKV_ARG_CHECK(tick != nullptr && tick->epoch_interval > 0, "akv_incref_batch: bad tick");
  AKV_ARG_CHECK(status != nullptr, "akv_incref_batch: status is NULL");
  AKV_ARG_CHECK(n >= 0, "akv_incref_batch: n=%d < 0", n);
  if (n == 0) return AKV_OK;
  AKV_ARG_CHECK(ids != nullptr, "akv_incref_batch: ids is NULL");
  cudaStream_t s = akv_stream(stream);
  if (n <= kSmallBatch) {
    k_incref_small<<<1, kSmallThreads, 0, s>>>(*st, ids, n, *tick, status);
    AKV_LAUNCH_CHECK("akv_incref_batch(small)");
    return AKV_OK;
  }
  const int g = grid_for(n, 256, kAkvSMs * 4);
  k_incref_check<<<g, 256, 0, s>>>(*st, ids, n, status);
  AKV_LAUNCH_CHECK("akv_incref_batch(check)");
  k_incref_apply<<<g, 256, 0, s>>>(*st, ids, n, *tick, status);
  AKV_LAUNCH_CHECK("akv_incref_batch(apply)");
  return AKV_OK;
}

extern "C" int akv_decref_batch(const AkvAllocState* st, const int32_t* ids, int32_t n,
                                const AkvTick* tick, int32_t* retired_out, AkvStatus* status,
                                void* stream) {
  AKV_ARG_CHECK(state_ok(st), "akv_decref_batch: incomplete allocator state");
  AKV_ARG_CHECK(tick != nullptr && tick->epoch_interval > 0, "akv_decref_batch: bad tick");
  AKV_ARG_CHECK(status != nullptr, "akv_decref_batch: status is NULL");
  AKV_ARG_CHECK(n >= 0, "akv_decref_batch: n=%d < 0", n);
  if (n == 0) return AKV_OK;
  AKV_ARG_CHECK(ids != nullptr, "akv_decref_batch: ids is NULL");
  cudaStream_t s = akv_stream(stream);
  if (n <= kSmallBatch) {
    k_dec_small<<<1, kSmallThreads, 0, s>>>(*st, ids, n, retired_out, *tick, status);
    AKV_LAUNCH_CHECK("akv_decref_batch(small)");
    return AKV_OK;
  }
  const int n_ctas = grid_for(n, kDecThreads, kDecMaxCtas);
  const int32_t chunk = akv_ceil_div(n, n_ctas);
  int32_t* cta_counts = st->scratch_aux;
  DecPlan* plan = reinterpret_cast<DecPlan*>(st->scratch_aux + AKV_AUX_PLAN_OFFSET);
  k_dec_count<<<grid_for(n, 256, kAkvSMs * 4), 256, 0, s>>>(*st, ids, n, status);
  AKV_LAUNCH_CHECK("akv_decref_batch(count)");
  k_dec_flag<<<n_ctas, kDecThreads, 0, s>>>(*st, ids, n, chunk, cta_counts, status);
  AKV_LAUNCH_CHECK("akv_decref_batch(flag)");
  k_dec_plan<<<1, 1024, 0, s>>>(*st, n, n_ctas, cta_counts, ids, plan, *tick, status);
  AKV_LAUNCH_CHECK("akv_decref_batch(plan)");
  k_dec_apply<<<n_ctas, kDecThreads, 0, s>>>(*st, ids, n, chunk, cta_counts, plan, retired_out,
                                               *tick);
  AKV_LAUNCH_CHECK("akv_decref_batch(apply)");
  return AKV_OK;
}

extern "C" int akv_limbo_release(const AkvAllocState* st, int64_t safe_before_epoch, void* stream) {
  AKV_ARG_CHECK(state_ok(st), "akv_limbo_release: incomplete allocator state");
  k_release<<<1, 32, 0, akv_stream(stream)>>>(*st, safe_before_epoch);
  AKV_LAUNCH_CHECK("akv_limbo_release");
  return AKV_OK;
}

extern "C" int akv_epoch_advance(const AkvAllocState* st, const AkvTick* tick, void* stream) {
  AKV_ARG_CHECK(state_ok(st), "akv_epoch_advance: incomplete allocator state");
  AKV_ARG_CHECK(tick != nullptr, "akv_epoch_advance: tick is NULL");
  k_advance<<<1, 32, 0, akv_stream(stream)>>>(*st, *tick);
  AKV_LAUNCH_CHECK("akv_epoch_advance");
  return AKV_OK;
}

extern "C" int akv_cow_batch(const AkvAllocState* st, void* pool, int64_t bytes_per_block,
                             const int32_t* blocks, int32_t n, int32_t* out_blocks,
                             int32_t* out_copied, int32_t* pairs_scratch, const AkvTick* tick,
                             AkvStatus* status, void* stream) {
  AKV_ARG_CHECK(state_ok(st), "akv_cow_batch: incomplete allocator state");
  AKV_ARG_CHECK(tick != nullptr && tick->epoch_interval > 0, "akv_cow_batch: bad tick");
  AKV_ARG_CHECK(status != nullptr, "akv_cow_batch: status is NULL");
  AKV_ARG_CHECK(n >= 0, "akv_cow_batch: n=%d < 0", n);
  if (n == 0) return AKV_OK;
  AKV_ARG_CHECK(blocks && out_blocks && out_copied && pairs_scratch,
                "akv_cow_batch: NULL array argument");
  AKV_ARG_CHECK(pool != nullptr || bytes_per_block == 0,
                "akv_cow_batch: NULL pool with bytes_per_block=%lld",
                static_cast<long long>(bytes_per_block));
  cudaStream_t s = akv_stream(stream);
  // Requests are applied in order, kCowChunk at a time.
  for (int32_t off = 0; off < n; off += kCowChunk) {
    const int32_t m = std::min(kCowChunk, n - off);
    k_cow_plan<<<1, kCowThreads, 0, s>>>(*st, blocks + off, m, out_blocks + off, out_copied + off,
                                         pairs_scratch + 2 * off, *tick, status);
    AKV_LAUNCH_CHECK("akv_cow_batch(plan)");
    if (pool != nullptr && bytes_per_block > 0) {
      const int rc = akv_launch_copy_counted(pool, bytes_per_block, st->total_blocks,
                                             pairs_scratch + 2 * off, m,
                                             st->ctl + AKV_CTL_LAST_COPIED, status, s);
      if (rc != AKV_OK) return rc;
    }
  }
  return AKV_OK;
}

// ── dec_ref batch without caller-provided scratch ──────────────────────────
// For callers that cannot allocate device memory at the point where they free
// blocks: a block manager running inside a serving engine's memory-pool hook
// or after the engine has reserved all free GPU memory up front, where a
// cudaMalloc (or a framework allocation) would fail or re-enter the pool.
// The per-id work space of the dec_ref batch lives in this file-scope device
// array instead of the AkvAllocState's scratch pointers.  Every GPU that loads
// the library holds it (2 MiB + 8 KiB) until the process exits.
namespace {

constexpr int32_t kNoAllocMaxBlocks = AKV_NOALLOC_MAX_BLOCKS;
constexpr int64_t kNoAllocWords = 2 * static_cast<int64_t>(kNoAllocMaxBlocks) + AKV_AUX_WORDS;

static __device__ __align__(256) int32_t g_noalloc_scratch[kNoAllocWords];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mutex;
int32_t* g_noalloc_ptr[kNoAllocMaxDevices] = {nullptr};

// Device address of g_noalloc_scratch on the current device, looked up once
// per device.  In host code the symbol itself is only a host-side stand-in:
// passing it to a kernel would fault, so kernels get this address.
int noalloc_scratch(int32_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return akv_cuda_fail(e, "akv_decref_batch_noalloc: cudaGetDevice");
  AKV_ARG_CHECK(dev >= 0 && dev < kNoAllocMaxDevices, "akv_decref_batch_noalloc: device %d", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return akv_cuda_fail(e, "akv_decref_batch_noalloc: cudaGetSymbolAddress");
    g_noalloc_ptr[dev] = static_cast<int32_t*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return AKV_OK;
}

}  // namespace

extern "C" int akv_decref_batch_noalloc(const AkvAllocState* st, const int32_t* ids, int32_t n,
                                        const AkvTick* tick, int32_t* retired_out,
                                        AkvStatus* status, void* stream) {
  AKV_ARG_CHECK(st != nullptr && st->ref_counts && st->free_ring && st->limbo_ids &&
                    st->limbo_epochs && st->ctl && st->total_blocks > 0,
                "akv_decref_batch_noalloc: incomplete allocator state");
  AKV_ARG_CHECK(st->total_blocks <= kNoAllocMaxBlocks,
                "akv_decref_batch_noalloc: total_blocks=%d exceeds the %d blocks its static "
                "scratch covers; use akv_decref_batch with caller-provided scratch",
                st->total_blocks, kNoAllocMaxBlocks);
  AKV_ARG_CHECK(tick != nullptr && tick->epoch_interval > 0, "akv_decref_batch_noalloc: bad tick");
  AKV_ARG_CHECK(status != nullptr, "akv_decref_batch_noalloc: status is NULL");
  AKV_ARG_CHECK(n >= 0, "akv_decref_batch_noalloc: n=%d < 0", n);
  if (n == 0) return AKV_OK;
  AKV_ARG_CHECK(ids != nullptr, "akv_decref_batch_noalloc: ids is NULL");
  int32_t* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != AKV_OK) return rc;
  AkvAllocState s2 = *st;
  s2.scratch_count = scratch;
  s2.scratch_last = scratch + kNoAllocMaxBlocks;
  s2.scratch_aux = scratch + 2 * static_cast<int64_t>(kNoAllocMaxBlocks);
  cudaStream_t s = akv_stream(stream);
  // The array keeps whatever the previous call left; the counters must start
  // at zero.
  const size_t bytes = static_cast<size_t>(st->total_blocks) * sizeof(int32_t);
  cudaError_t e = cudaMemsetAsync(s2.scratch_count, 0, bytes, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(s2.scratch_last, 0, bytes, s);
  if (e != cudaSuccess) return akv_cuda_fail(e, "akv_decref_batch_noalloc: clear scratch");
  if (n <= kSmallBatch) {
    k_dec_small<<<1, kSmallThreads, 0, s>>>(s2, ids, n, retired_out, *tick, status);
    AKV_LAUNCH_CHECK("akv_decref_batch_noalloc(small)");
    return AKV_OK;
  }
  const int n_ctas = grid_for(n, kDecThreads, kDecMaxCtas);
  const int32_t chunk = akv_ceil_div(n, n_ctas);
  int32_t* cta_counts = s2.scratch_aux;
  DecPlan* plan = reinterpret_cast<DecPlan*>(s2.scratch_aux + AKV_AUX_PLAN_OFFSET);
  k_dec_count<<<grid_for(n, 256, kAkvSMs * 4), 256, 0, s>>>(s2, ids, n, status);
  AKV_LAUNCH_CHECK("akv_decref_batch_noalloc(count)");
  k_dec_flag<<<n_ctas, kDecThreads, 0, s>>>(s2, ids, n, chunk, cta_counts, status);
  AKV_LAUNCH_CHECK("akv_decref_batch_noalloc(flag)");
  k_dec_plan<<<1, 1024, 0, s>>>(s2, n, n_ctas, cta_counts, ids, plan, *tick, status);
  AKV_LAUNCH_CHECK("akv_decref_batch_noalloc(plan)");
  k_dec_apply<<<n_ctas, kDecThreads, 0, s>>>(s2, ids, n, chunk, cta_counts, plan, retired_out, *tick);
  AKV_LAUNCH_CHECK("akv_decref_batch_noalloc(apply)");
  return AKV_OK;
}
