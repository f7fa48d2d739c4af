/*
 * agentkv_b200.h — C ABI of the B200 block-movement and prefix-lookup path.
 *
 * Every entry point takes plain device pointers and sizes, enqueues work on
 * the caller's CUDA stream (`stream` is a cudaStream_t; NULL means the legacy
 * default stream) and returns an AKV_* host status.  A host status other than
 * AKV_OK means nothing was enqueued; `akv_last_error` then describes why.
 *
 * Errors that only the device can see (a block id out of range, a refcount
 * that would go below zero, an exhausted free list, a destination that is not
 * exclusively owned) are written into an AkvStatus record in device memory
 * that the caller owns.  The first error sticks: every mutating kernel reads
 * the record on entry and does nothing while it holds an error, so a failed
 * batch never half-applies the batches queued behind it.  The caller reads
 * the record after synchronising the stream and clears it with
 * cudaMemsetAsync (or akv_status_clear).
 *
 * The library allocates no memory on any path: the pool, ids, refcounts,
 * free list, tree arrays and outputs are all owned by the caller (PyTorch
 * tensors in the Python package).  Functions keep no mutable host state
 * except a thread-local last-error string, so they are reentrant.
 *
 * Reference interfaces each group replaces are cited by file:line within the
 * agentkv project.
 */
#ifndef AGENTKV_B200_H
#define AGENTKV_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define AKV_API __attribute__((visibility("default")))
#else
#define AKV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ── status codes ───────────────────────────────────────────────────────── */
enum {
  AKV_OK = 0,
  AKV_ERR_INVALID_ARG = 1,     /* bad pointer / size / alignment (host) */
  AKV_ERR_OUT_OF_RANGE = 2,    /* block id outside [0, total_blocks) */
  AKV_ERR_EXHAUSTED = 3,       /* free list has fewer ids than requested */
  AKV_ERR_DOUBLE_FREE = 4,     /* dec_ref of a block whose ref_count <= 0 */
  AKV_ERR_NOT_ALLOCATED = 5,   /* inc_ref of a block whose ref_count <= 0 */
  AKV_ERR_NOT_EXCLUSIVE = 6,   /* copy/zero destination with ref_count != 1 */
  AKV_ERR_DEPENDENT_PAIRS = 7, /* a batch's dst is another pair's src/dst */
  AKV_ERR_CUDA = 8,            /* a CUDA runtime call failed (host) */
  AKV_ERR_TIMEOUT = 9,         /* a bounded device wait gave up */
  AKV_ERR_TREE = 10,           /* malformed tree replica (bad node index) */
  AKV_ERR_MIRROR = 11          /* a replayed op log disagrees with the device state */
};

/* Device-side status record (32 bytes).  code = first AKV_ERR_* seen,
 * index = batch position of the offending element, id = offending block id
 * (or node id), observed = the refcount (or other value) that failed the
 * check, aux = extra detail (e.g. the iteration count of a timed-out wait).
 * _reserved is the work counter of the claimed block copies
 * (akv_copy_blocks_variant 14-18), zero between their launches; a record
 * belongs to one stream at a time. */
typedef struct AkvStatus {
  int32_t code;
  int32_t index;
  int32_t id;
  int32_t observed;
  int64_t aux;
  int64_t _reserved;
} AkvStatus;

/* ── library ────────────────────────────────────────────────────────────── */
AKV_API int akv_version(void);                     /* (major << 16) | minor */
AKV_API int akv_last_error(char* buf, int len);    /* copies the thread's last message */
AKV_API int akv_status_clear(AkvStatus* status, void* stream);
/* One-time set-up of the current device's kernel attributes (shared-memory
 * limits).  The entry points do it on first use; call this first when the
 * first use would happen inside a CUDA stream capture. */
AKV_API int akv_prepare(void);

/* A copy of `bytes` between a host buffer (pinned for an asynchronous copy)
 * and device memory on `stream` (to_host = 1: device -> host), then, with
 * wait = 1, a wait for the stream.  No counterpart in the reference (whose
 * metadata lives on the host): the per-call API's one round trip — a call's
 * inputs up, or its status, outputs and counters back — in one call from
 * the host language. */
AKV_API int akv_copy_wait(void* dst, const void* src, int64_t bytes, int32_t to_host, int32_t wait,
                          void* stream);

/* Gather n host int32 arrays (src[i]: address, lens[i] tokens) back to back
 * into `dst` (host; pinned for an asynchronous upload) with `threads` host
 * threads (1-64; one for fewer than 65,536 tokens), then, with d_dst
 * non-NULL, one asynchronous copy of the packing to d_dst on `stream`.  The
 * host side of a batched lookup: the reference's callers hold one token list
 * per query.  Returns after enqueuing the copy. */
AKV_API int akv_gather_upload(const uint64_t* src, const int64_t* lens, int32_t n, int32_t* dst,
                              int32_t* d_dst, int32_t threads, void* stream);

/* ── block movement ─────────────────────────────────────────────────────────
 * The pool is the reference's `_kv_data` tensor
 * [total_blocks, L, 2, H_kv, block_size, D] (agentkv/core/slab_allocator.py:155-164)
 * seen as total_blocks contiguous spans of bytes_per_block bytes
 * (agentkv/core/config.py:95-98).
 *
 * akv_copy_blocks replaces triton_kernels.copy_block / _copy_block_kernel
 * (agentkv/core/triton_kernels.py:171-203, :107-132), which moves ONE block
 * per launch, with one launch for a batch of (src, dst) pairs.  `pairs` is a
 * device int32 array [n_pairs][2].  The pairs must be independent: no dst is
 * repeated and no dst is another pair's src (the batch is applied in
 * parallel; akv_check_pairs verifies this on the device).  When `ref_counts`
 * is non-NULL every dst must have ref_count == 1, the check
 * SlabAllocator.copy_block makes under its lock
 * (agentkv/core/slab_allocator.py:307-313); an offending pair is skipped and
 * reported.
 */
AKV_API int akv_copy_blocks(void* pool, int64_t bytes_per_block, int32_t total_blocks,
                    const int32_t* pairs, int32_t n_pairs,
                    const int32_t* ref_counts, AkvStatus* status, void* stream);

/* Same, with an explicit kernel choice: 0 = automatic, 1 = 16-byte vector
 * loads/stores, 2 = bulk-async (TMA) copies staged through shared memory
 * (16 KiB chunks x 12 in flight for blocks >= 2 MiB, 32 KiB x 6 below, one
 * CTA per SM); 3-13 = fixed bulk shapes for tuning
 * (32 KiB x 6; 32 KiB x 3 with 2 CTAs per SM; 64 KiB x 3; 16 KiB x 6 with
 * 2 CTAs per SM; 8 KiB x 24; chunk-major order (chunk c of every pair before
 * chunk c + 1) with 32 KiB x 3, 16 KiB x 12, 32 KiB x 6; 32 KiB x 3;
 * 16 KiB x 6 and 32 KiB x 3 on grids of 8 CTAs per SM, 2 resident at a
 * time, the rest placed on whichever SM frees up first); 14-15 = 16 KiB x 12
 * and 32 KiB x 6 with items handed out dynamically, 128 KiB per claim, from a
 * counter kept in the status record's last word (zero between launches;
 * status must be non-NULL, and launches sharing one status record must not
 * overlap on the GPU); 16-18 = the same with other claim sizes: 32 KiB x 6
 * claiming 256 KiB, 16 KiB x 12 claiming 256 KiB and 32 KiB. */
AKV_API int akv_copy_blocks_variant(void* pool, int64_t bytes_per_block, int32_t total_blocks,
                            const int32_t* pairs, int32_t n_pairs,
                            const int32_t* ref_counts, AkvStatus* status,
                            int32_t variant, void* stream);

/* Copy of a batch of (src, dst) block pairs across a serving engine's
 * per-layer KV caches: cache c holds block b at
 * cache_bases[c] + b * block_stride (block_bytes bytes), and every pair is
 * copied in every cache, all in one launch.  This is what vLLM's
 * copy_blocks(key_caches, value_caches, block_mapping) does with the
 * blocks_to_copy list that the reference's vLLM adapter returns from
 * append_slots (integrations/vllm/block_manager.py:134-167); the caches'
 * layout (one K and one V tensor per layer) differs from the AgentKV pool's.
 * cache_bases is a DEVICE array of n_caches addresses; each must be 16-byte
 * aligned (the kernel checks and reports AKV_ERR_INVALID_ARG), as must
 * block_bytes and block_stride (checked here).  Pairs must be independent;
 * ref_counts, when non-NULL, is checked as in akv_copy_blocks.  variant:
 * 0 = automatic (= 4), 1/2/3/4 = bulk chunks of 16/32/64/32 KiB, 12/6/3/3
 * in flight per SM. */
AKV_API int akv_copy_blocks_layers(const uint64_t* cache_bases, int32_t n_caches, int64_t block_bytes,
                           int64_t block_stride, int32_t total_blocks, const int32_t* pairs,
                           int32_t n_pairs, const int32_t* ref_counts, AkvStatus* status,
                           int32_t variant, void* stream);

/* akv_copy_blocks with the pair count in device memory: `pairs` has room for
 * n_max pairs and the kernel reads the int64 *n_dev (written by an earlier
 * kernel, a copy or a broadcast) and copies the first min(*n_dev, n_max).
 * No counterpart in the reference, which copies one pair per call
 * (agentkv/core/triton_kernels.py:171-203): it lets a batch of variable size
 * travel as one buffer (count and pairs) in one broadcast to the ranks of a
 * head-sharded pool, and a captured launch replay batches of any size up to
 * n_max.  Same checks and errors as akv_copy_blocks. */
AKV_API int akv_copy_blocks_counted(void* pool, int64_t bytes_per_block, int32_t total_blocks,
                            const int32_t* pairs, int32_t n_max, const int64_t* n_dev,
                            const int32_t* ref_counts, AkvStatus* status, void* stream);

/* One model layer's K and V out of the pool as contiguous tensors: for a
 * sequence whose blocks are block_ids[0..n_blocks) (device array), writes
 * out_k and out_v, each [num_kv_heads, n_tokens, head_dim] (row_bytes =
 * head_dim x element size per row), from layer `layer` of those blocks;
 * n_tokens <= n_blocks x block_size (the last block may be partly used).
 * Replaces the gather + permute + reshape + truncation of
 * AgentKVCache.update / to_legacy_cache
 * (agentkv/hf_cache.py:129-153, :196-215) with one launch.  Out-of-range
 * ids are reported (AKV_ERR_OUT_OF_RANGE) and their tiles skipped. */
AKV_API int akv_kv_gather(const void* pool, int32_t total_blocks, int32_t num_layers, int32_t num_kv_heads,
                  int32_t block_size, int64_t row_bytes, int32_t layer, const int32_t* block_ids,
                  int32_t n_blocks, int64_t n_tokens, void* out_k, void* out_v, AkvStatus* status,
                  void* stream);

/* New tokens' K and V rows of one layer into the pool: token i's rows go to
 * block slots[i] / block_size, position slots[i] % block_size (slots is a
 * device array).  k_src / v_src hold head h, token i at
 * base + h * src_stride_head + i * src_stride_token (strides in BYTES, the
 * head_dim row contiguous).  Replaces AgentKVCache.update's per-token row
 * writes (agentkv/hf_cache.py:100-127) with one launch; the caller does the
 * copy-on-write checks before it, as the reference does. */
AKV_API int akv_kv_scatter(void* pool, int32_t total_blocks, int32_t num_layers, int32_t num_kv_heads,
                   int32_t block_size, int64_t row_bytes, int32_t layer, const int32_t* slots, int32_t n_new,
                   const void* k_src, const void* v_src, int64_t src_stride_head, int64_t src_stride_token,
                   AkvStatus* status, void* stream);

/* akv_zero_blocks replaces triton_kernels.zero_block / _zero_block_kernel
 * (agentkv/core/triton_kernels.py:206-229, :134-162) and
 * SlabAllocator.zero_block (agentkv/core/slab_allocator.py:321-334).  It
 * writes +0.0 (all-zero bits), the result of the reference's CPU path
 * `block.zero_()`; the reference's Triton path stores `x * 0`, which keeps the
 * sign of negative inputs and propagates NaN.  Write-only: no read of the
 * old contents. */
AKV_API int akv_zero_blocks(void* pool, int64_t bytes_per_block, int32_t total_blocks,
                    const int32_t* ids, int32_t n, const int32_t* ref_counts,
                    AkvStatus* status, void* stream);

AKV_API int akv_zero_blocks_variant(void* pool, int64_t bytes_per_block, int32_t total_blocks,
                            const int32_t* ids, int32_t n, const int32_t* ref_counts,
                            AkvStatus* status, int32_t variant, void* stream);

/* Verify on the device that a pair batch is independent (see
 * akv_copy_blocks) and in range; sets AKV_ERR_DEPENDENT_PAIRS /
 * AKV_ERR_OUT_OF_RANGE.  `mark` is caller-owned scratch of total_blocks
 * int32 that must be all zero on entry; it is all zero again on return. */
AKV_API int akv_check_pairs(const int32_t* pairs, int32_t n_pairs, int32_t total_blocks,
                    int32_t* mark, AkvStatus* status, void* stream);

/* ── slab allocator: device free list and refcounts ─────────────────────────
 * Replaces SlabAllocator.alloc / inc_ref / dec_ref / _do_free /
 * _drain_deferred / _tick (agentkv/core/slab_allocator.py:194-278, 387-437)
 * and the id-moving half of EpochReclaimer (agentkv/core/reclamation.py:
 * 114-173).  All state lives in caller-owned device arrays:
 *
 *   ref_counts[N]     int32 — the reference's `_ref_counts`
 *   free_ring[N]      int32 — the `_free_list` deque as a ring; initially
 *                     0..N-1, pops from the right, recycled ids pushed left
 *   limbo_ids[N]      int32 — retired ids not yet on the free list, FIFO with
 *                     monotonic cursors head <= rel <= tail: [head, rel) is
 *                     the reference's `_deferred_free`, [rel, tail) the
 *                     reclaimer's `_pending` queue
 *   limbo_epochs[N]   int64 — epoch each pending id retired in
 *   ctl[AKV_CTL_WORDS] int64 — cursors and counters, see AKV_CTL_*
 *   scratch_count[N], scratch_last[N] int32 — per-id work space; all zero
 *                     on entry and again on return of every call
 *   scratch_aux[AKV_AUX_WORDS] int32 — per-launch work space
 *
 * Batches follow the reference's sequential semantics op by op: ids come
 * off the free list in the order repeated alloc() calls return them, and
 * retired ids reach the free list in the order repeated dec_ref() calls put
 * them there, including the deferred-drain and epoch rules.  The op counter
 * and the epoch are device counters; the host describes its reader set in
 * AkvTick.  A batch is validated as a whole before anything is mutated.
 * Calls on one allocator state must be ordered on one stream.
 */
enum {
  AKV_CTL_FREE_LEFT = 0,    /* ring index of the leftmost free id */
  AKV_CTL_FREE_SIZE = 1,    /* number of free ids (len(_free_list)) */
  AKV_CTL_LIMBO_HEAD = 2,   /* limbo cursors (monotonic, index mod N) */
  AKV_CTL_LIMBO_REL = 3,
  AKV_CTL_LIMBO_TAIL = 4,
  AKV_CTL_OPS = 5,          /* SlabAllocator._op_count */
  AKV_CTL_EPOCH = 6,        /* EpochReclaimer._epoch */
  AKV_CTL_ALLOCS = 7,       /* _alloc_count */
  AKV_CTL_FREES = 8,        /* _free_count (blocks retired) */
  AKV_CTL_PEAK = 9,         /* _peak_allocated */
  AKV_CTL_LAST_RETIRED = 10,/* ids retired by the last dec_ref batch */
  AKV_CTL_LAST_COPIED = 11, /* copies made by the last CoW batch chunk */
  AKV_CTL_DONE = 12,        /* internal CTA completion counter */
  AKV_CTL_ADVANCES = 13,    /* EpochReclaimer._advance_count */
  AKV_CTL_RELEASED = 14,    /* EpochReclaimer._freed_count */
  AKV_CTL_WORDS = 16
};

#define AKV_AUX_PLAN_OFFSET 1024
#define AKV_AUX_WORDS 2048

typedef struct AkvAllocState {
  int32_t* ref_counts;
  int32_t* free_ring;
  int32_t* limbo_ids;
  int64_t* limbo_epochs;
  int64_t* ctl;
  int32_t* scratch_count;
  int32_t* scratch_last;
  int32_t* scratch_aux;
  int32_t total_blocks;
  int32_t _pad;
} AkvAllocState;

/* The host's reader set when the batch starts (EpochReclaimer's
 * `_active_reader_epochs`, reclamation.py:79) and PoolConfig.epoch_interval
 * (agentkv/core/config.py:62), which must be > 0. */
typedef struct AkvTick {
  int64_t readers_min;    /* smallest epoch holding a reader */
  int64_t readers_max;    /* largest epoch holding a reader */
  int32_t epoch_interval;
  int32_t readers_active; /* 0: no read section open */
} AkvTick;

/* Reset to the constructor state: refcounts 0, free ring 0..N-1, limbo empty,
 * counters 0, scratch zeroed. */
AKV_API int akv_alloc_init(const AkvAllocState* st, void* stream);

/* n alloc() calls: out_ids[k] receives the k-th id, its refcount set to 1.
 * AKV_ERR_EXHAUSTED (nothing mutated) if the calls would run dry. */
AKV_API int akv_alloc_batch(const AkvAllocState* st, int32_t n, int32_t* out_ids,
                    const AkvTick* tick, AkvStatus* status, void* stream);

/* n inc_ref() calls (ids may repeat).  AKV_ERR_NOT_ALLOCATED if any id has
 * ref_count <= 0 on entry. */
AKV_API int akv_incref_batch(const AkvAllocState* st, const int32_t* ids, int32_t n,
                     const AkvTick* tick, AkvStatus* status, void* stream);

/* n dec_ref() calls (ids may repeat).  AKV_ERR_DOUBLE_FREE if an id would go
 * below zero.  Ids reaching zero retire at the position of their last
 * occurrence; `retired_out` (optional, n entries) receives them in
 * retirement order and ctl[AKV_CTL_LAST_RETIRED] their count. */
AKV_API int akv_decref_batch(const AkvAllocState* st, const int32_t* ids, int32_t n,
                     const AkvTick* tick, int32_t* retired_out,
                     AkvStatus* status, void* stream);

/* akv_decref_batch for callers that cannot allocate device memory where they
 * free blocks (a block manager called from a serving engine's memory-pool
 * hook, or running after the engine reserved all free GPU memory up front,
 * where a cudaMalloc would fail or re-enter the pool).  No counterpart in the
 * reference.  Same arguments and results as akv_decref_batch; the state's
 * scratch_count / scratch_last / scratch_aux pointers are ignored (they may
 * be NULL) and a static device array inside the library is used instead:
 *   - it covers total_blocks <= AKV_NOALLOC_MAX_BLOCKS; larger states are
 *     rejected with AKV_ERR_INVALID_ARG and nothing is enqueued;
 *   - every GPU that loads the library holds it (2 MiB + 8 KiB) until exit;
 *   - the first call on a device looks up its device address, so make that
 *     first call before any stream capture;
 *   - all calls in the process share it: calls whose kernels can overlap on
 *     the GPU (different streams, or concurrent host threads) race; issue
 *     them on one stream.
 * Allocates nothing: no cudaMalloc, no cudaFree, no allocating library call. */
#define AKV_NOALLOC_MAX_BLOCKS 262144
AKV_API int akv_decref_batch_noalloc(const AkvAllocState* st, const int32_t* ids, int32_t n,
                                     const AkvTick* tick, int32_t* retired_out,
                                     AkvStatus* status, void* stream);

/* EpochReclaimer._try_retire (reclamation.py:147-173): release every pending
 * id whose epoch is < safe_before_epoch, in FIFO order (INT64_MAX releases
 * all).  Released ids join the free list at the next allocator op. */
AKV_API int akv_limbo_release(const AkvAllocState* st, int64_t safe_before_epoch, void* stream);

/* EpochReclaimer.maybe_advance (reclamation.py:129-143): bump the epoch unless
 * a reader holds it, then try_retire. */
AKV_API int akv_epoch_advance(const AkvAllocState* st, const AkvTick* tick, void* stream);

/* CoW of a batch of residual blocks — DualRadixTree.ensure_mutable_block
 * (agentkv/core/radix_tree.py:286-314) for n requests on distinct
 * (handle, index) slots whose current block ids are `blocks[n]`, applied in
 * request order: a request copies iff its block's refcount is > 1 at that
 * point; it then allocates a fresh id, copies the block into it and dec_refs
 * the old one.  out_blocks[i] receives the block request i ends up owning
 * (the fresh id, or blocks[i] when no copy was needed); out_copied[i] is 1
 * when a copy happened.  `pairs_scratch` (int32 [n][2], caller-owned)
 * receives the (src, dst) pairs.  With pool == NULL (a metadata-only pool)
 * nothing is copied. */
AKV_API int akv_cow_batch(const AkvAllocState* st, void* pool, int64_t bytes_per_block,
                  const int32_t* blocks, int32_t n, int32_t* out_blocks,
                  int32_t* out_copied, int32_t* pairs_scratch,
                  const AkvTick* tick, AkvStatus* status, void* stream);

/* One fork level on device-resident block tables (a Tree-of-Thought level):
 * each of n_parents parents (residual tables concatenated in parent_tables,
 * offsets parent_off[n_parents + 1], every table non-empty) is forked
 * `fanout` times and each child copy-on-writes its last inherited block and
 * appends `append` blocks — per child, the reference's fork()
 * (agentkv/core/radix_tree.py:222-264), ensure_mutable_block(child, -1)
 * (:286-314) and `append` allocate_block() calls (:266-284).  `fresh_ids`
 * holds the (1 + append) * fanout * n_parents ids of one akv_alloc_batch.
 * Writes the children's tables (child_tables, child_off[n_children + 1]),
 * the fork's inc_ref list (inc_ids: every parent block once per child), the
 * CoW pairs (pairs [n_children][2]) and the CoW dec_ref list (dec_ids), which
 * akv_incref_batch, akv_copy_blocks and akv_decref_batch then apply. */
AKV_API int akv_fanout_plan(const int32_t* parent_tables, const int64_t* parent_off,
                            int32_t n_parents, int32_t fanout, int32_t append,
                            const int32_t* fresh_ids, int32_t* child_tables, int64_t* child_off,
                            int32_t* inc_ids, int32_t* pairs, int32_t* dec_ids, void* stream);

/* Every level of a fan-out in one launch (append >= 1): `levels` levels of
 * akv_fanout_plan from the roots (tables root_tables, offsets root_off
 * [n_roots + 1], root_blocks = their total length), children of a level
 * being the parents of the next.  fresh_ids holds the ids of one
 * akv_alloc_batch of (1 + append) x (all children) — the ids the per-child
 * calls take, level after level.  child_tables, pairs and dec_ids receive
 * what the levels' akv_fanout_plan launches would write, level after level;
 * inc_ids receives the same ids (the same multiset per level), position-
 * major within each level and root (entry j of every child's parent table,
 * children in order, then entry j + 1), so that equal ids sit in adjacent
 * slots and akv_incref_batch folds them into one atomic per warp.  With
 * appended blocks a child's table depends only on its root's
 * table and its ancestors' fresh ids, so no level waits for another.  No
 * counterpart in the reference beyond the per-child calls it replaces
 * (agentkv/core/radix_tree.py:222-314). */
#define AKV_MAX_FANOUT_LEVELS 16
AKV_API int akv_fanout_tree_plan(const int32_t* root_tables, const int64_t* root_off, int32_t n_roots,
                         int64_t root_blocks, int32_t fanout, int32_t append, int32_t levels,
                         const int32_t* fresh_ids, int32_t* child_tables, int32_t* inc_ids,
                         int32_t* pairs, int32_t* dec_ids, void* stream);

/* ── agents stepped on the device ────────────────────────────────────────────
 * A batch of the per-call steps the reference's multi-agent pattern makes,
 * applied by one warp to agents whose residual block tables live in device
 * memory (tables[n_agents][capacity], lens[n_agents]), with the reference's
 * sequential allocator semantics op by op.  actions: int32 [n][3] {kind,
 * slot, target}, step s = actions [step_off[s], step_off[s+1]) (device):
 *   0 fork     free agent `target`, then fork agent `slot` into it
 *              (DualRadixTree.free + fork, agentkv/core/radix_tree.py:
 *              351-377, 222-264)
 *   1 cow      ensure_mutable_block(agent, -1) (:286-314): a shared tail block
 *              is replaced by a fresh copy (alloc, the pair, dec_ref); an agent
 *              without blocks allocates one instead (:266-284)
 *   2 free     free agent `slot`, restart it as a fork of the root table
 *   3 advance  EpochReclaimer.maybe_advance (reclamation.py:129-143)
 *   4 append   allocate_block(agent)
 * Tables hold distinct ids (as a handle's residual blocks do).  Step s's
 * copy-on-write pairs go to pairs_out + s * (2 + 2 * pairs_cap) as an int64
 * count then the pairs (the akv_copy_blocks_counted format).  An action
 * that fails changes nothing, every earlier one stays applied (as the
 * reference's calls would), the error goes to `status` and the kernel stops.
 * Shared-tree references of the agents are the caller's (they do not change
 * the allocator).  One launch. */
AKV_API int akv_agent_steps(const AkvAllocState* st, const AkvTick* tick, int32_t* tables, int32_t* lens,
                            int32_t n_agents, int32_t capacity, const int32_t* root_table, int32_t root_len,
                            const int32_t* actions, const int32_t* step_off, int32_t n_steps,
                            int32_t* pairs_out, int32_t pairs_cap, AkvStatus* status, void* stream);

/* ── shared radix tree: device replica and match_prefix ─────────────────────
 * Replaces DualRadixTree._match_prefix_locked (agentkv/core/radix_tree.py:
 * 513-570), reached from create_root (:203) and match_prefix (:379-416).
 * The replica mirrors the host tree's SharedNode table (:82-103):
 *   node_edge_off[cap] int64 — start of the node's edge in `tokens`
 *   node_edge_len[cap] int32 — edge length (0 for the root / unused ids)
 *   slots[mask+1]      int32x4 {parent, first_token, child, child_edge_len}
 *                      — the `children` dicts of all nodes as one
 *                      open-addressing hash table; parent = -1 empty,
 *                      -2 deleted
 *   run_head[run_nodes] int32 — optional (NULL = none): for a node with
 *                      exactly one child, the index of its run in
 *                      run_entries, else -1
 *   run_entries[n_runs] int32x4 {child, first_token, edge_len, remaining} —
 *                      unary chains: a node's run lists its only child, that
 *                      child's only child, ... up to and including the first
 *                      node without exactly one child; `remaining` counts the
 *                      entries from this one to the end of its chain, so a
 *                      run starting inside a chain is a suffix of it.  The
 *                      lookup then follows up to 32 hops of a chain with one
 *                      load instead of one hash probe per hop.
 * Node ids are the tree's own ids (root = 0).  Callers that do not use runs
 * set run_head = run_entries = NULL and n_runs = run_nodes = 0.
 */
typedef struct AkvTreeView {
  const int32_t* tokens;
  const int64_t* node_edge_off;
  const int32_t* node_edge_len;
  const int32_t* slots;
  int64_t n_tokens;
  int32_t n_nodes;     /* capacity of the node arrays */
  int32_t slot_mask;   /* number of slots - 1, a power of two minus one */
  const int32_t* run_head;
  const int32_t* run_entries;
  int32_t n_runs;
  int32_t run_nodes;
} AkvTreeView;

/* Hash of (parent, first_token) into the slot table; the host builder and
 * the device lookup both use this function. */
AKV_API uint32_t akv_tree_hash(int32_t parent, int32_t token);

/* Apply a batch of replica updates: slot_updates int32 [n_slot][5]
 * {slot, parent, first_token, child, child_edge_len}; node_updates int64 [n_node][3]
 * {node, edge_off, edge_len}.  (Token arena appends are plain copies.) */
AKV_API int akv_tree_apply(const AkvTreeView* tree, const int32_t* slot_updates, int32_t n_slot,
                   const int64_t* node_updates, int32_t n_node,
                   AkvStatus* status, void* stream);

/* The host tree's inserts and prunes, applied by the replica itself
 * (DualRadixTree._insert_shared_locked, agentkv/core/radix_tree.py:572-686,
 * with its block-aligned split, split == 0 overwrite and exact re-commit;
 * the prune of _dec_shared_ref_locked, :695-717), so that a commit ships its
 * tokens and a few ids instead of the rows it changed.  cmds: device int64
 * [n_cmds][8], applied in order by one warp:
 *   {1, parent, first new node id, payload offset, token count, arena length
 *    before the insert, block size, 0}  insert the payload's tokens under
 *                                       `parent`
 *   {2, parent or -1, node, 0, ...}     prune `node`
 * payload: device int32, every insert's tokens.  New nodes take consecutive
 * ids, new edge tokens are appended to the arena and hash slots are claimed
 * exactly as the host mirror does, so the arrays end byte-equal to the host
 * mirror's.  The caller keeps the arrays large enough (token_cap = the
 * arena's capacity); an index out of range sets AKV_ERR_TREE and stops. */
AKV_API int akv_tree_commands(const AkvTreeView* tree, int64_t token_cap, const int64_t* cmds, int32_t n_cmds,
                              const int32_t* payload, int64_t payload_len, AkvStatus* status, void* stream);

/* One warp per query.  Query q is tokens[q_off[q] .. q_off[q+1]).  Writes
 * the reference's (node_id, match_len) — (-1, 0) when nothing matched — and
 * the number of token comparisons the reference loop performs. */
AKV_API int akv_match_prefix(const AkvTreeView* tree, const int32_t* tokens, const int64_t* q_off,
                     int32_t nq, int32_t block_size, int32_t* out_node, int32_t* out_len,
                     int64_t* out_compared, AkvStatus* status, void* stream);

/* Same, with an optional processing order (`order[nq]`, a permutation of
 * the query indices; launching the longest queries first balances the SMs)
 * and the number of 32-token chunks a warp compares per verify round (1, 2,
 * 4, 8 or 16; 0 = default 8), optionally OR-ed with AKV_MATCH_PIPELINED
 * (widths 2, 4 and 8: the next round's loads are issued before the current
 * round's compare).  Outputs stay indexed by query. */
#define AKV_MATCH_PIPELINED 0x100
/* OR-ed into `chunks` as well: each warp first asks L2 for its query's
 * tokens (prefetch.global.L2), so that the verify rounds wait on L2 rather
 * than DRAM. */
#define AKV_MATCH_PREFETCH 0x200
AKV_API int akv_match_prefix_variant(const AkvTreeView* tree, const int32_t* tokens,
                                     const int64_t* q_off, int32_t nq, int32_t block_size,
                                     int32_t* out_node, int32_t* out_len, int64_t* out_compared,
                                     const int32_t* order, AkvStatus* status, int32_t chunks,
                                     void* stream);

/* Bytes of scratch akv_match_prefix_split needs at most for nq queries
 * holding n_tokens tokens in all, at tokens_per_range (0 = default, 1024);
 * -1 for arguments it would refuse.  Pure host function. */
AKV_API int64_t akv_match_scratch_bytes(int32_t nq, int64_t n_tokens, int32_t tokens_per_range);

/* Longest query a split lookup takes, in ranges. */
#define AKV_MATCH_MAX_RANGES 64

/* The range plan of a split lookup (pure host function): `lengths` are the
 * queries' token counts in launch order, longest first; writes
 * range_starts[0 .. n_ranges] (range_starts[j+1] - range_starts[j] = the
 * number of queries longer than j * tokens_per_range, all nq for j = 0) and
 * n_ranges = the longest query's range count, at most AKV_MATCH_MAX_RANGES
 * (use longer ranges for longer queries). */
AKV_API int akv_match_split_plan(const int64_t* lengths, int32_t nq, int32_t tokens_per_range,
                                 int64_t* range_starts, int32_t* n_ranges);

/* The same answers as akv_match_prefix_variant (the reference's
 * _match_prefix_locked, agentkv/core/radix_tree.py:513-570, per query),
 * with each query's token positions cut into ranges of tokens_per_range
 * tokens (a multiple of 32; 0 = 1024), one warp per range, so that a long
 * query no longer holds the batch: each warp walks the tree to the end of
 * its range, compares that range only, and the last warp of a query to
 * finish picks the earliest stop among its ranges.
 *   order         required: the launch order, longest query first
 *   range_starts  HOST array from akv_match_split_plan (copied into the
 *                 launch; n_ranges + 1 entries)
 *   scratch       caller-owned device memory of at least
 *                 akv_match_scratch_bytes(nq, total tokens, tokens_per_range)
 *                 bytes, 16-byte aligned; no initial contents needed (the
 *                 call clears what it counts with, one memset); calls
 *                 sharing it must be ordered (one stream)
 *   chunks        as in akv_match_prefix_variant (0 = 4)
 * A rank whose ranges disagree with range_starts sets AKV_ERR_INVALID_ARG in
 * `status` and gets no answer.  One memset and one launch. */
AKV_API int akv_match_prefix_split(const AkvTreeView* tree, const int32_t* tokens,
                                   const int64_t* q_off, int32_t nq, int32_t block_size,
                                   int32_t* out_node, int32_t* out_len, int64_t* out_compared,
                                   const int32_t* order, const int64_t* range_starts,
                                   int32_t n_ranges, int32_t tokens_per_range, void* scratch,
                                   int64_t scratch_bytes, int32_t chunks, AkvStatus* status,
                                   void* stream);

/* Scratch bytes of a staged lookup (akv_match_prefix_staged) of nq queries
 * in a packing of n_tokens tokens, at window_tokens (0 = default, 512);
 * -1 for arguments it would refuse.  Pure host function. */
AKV_API int64_t akv_match_staged_scratch_bytes(int32_t nq, int64_t n_tokens, int32_t window_tokens);

/* The same answers as akv_match_prefix_variant (the reference's
 * _match_prefix_locked, agentkv/core/radix_tree.py:513-570, per query), in
 * two launches: one warp per query follows the tree by each edge's first
 * token only and records its hops; then one warp per window_tokens-token
 * window of every query's followed path compares the query with the edges,
 * and the first mismatch over a query's windows decides its answer.  A long
 * query is spread over many warps without being walked twice.
 *   n_tokens      tokens in the packing: q_off[nq] <= n_tokens <= INT32_MAX
 *   order         optional launch order of the queries, longest first
 *   window_tokens 256, 512 or 1024 (0 = 512)
 *   scratch       caller-owned device memory of at least
 *                 akv_match_staged_scratch_bytes(nq, n_tokens, window_tokens)
 *                 bytes, 256-byte aligned; no initial contents needed; calls
 *                 sharing it must be ordered (one stream)
 * The tree's token arena must hold at most INT32_MAX tokens.  Two launches. */
AKV_API int akv_match_prefix_staged(const AkvTreeView* tree, const int32_t* tokens,
                                    const int64_t* q_off, int32_t nq, int64_t n_tokens,
                                    int32_t block_size, int32_t* out_node, int32_t* out_len,
                                    int64_t* out_compared, const int32_t* order,
                                    int32_t window_tokens, void* scratch, int64_t scratch_bytes,
                                    AkvStatus* status, void* stream);

/* ── per-call operations on a host mirror ──────────────────────────────── */
/* A host copy of the allocator state that answers the per-call API at once
 * (SlabAllocator.alloc / inc_ref / dec_ref, ensure_mutable_block, the
 * reclaimer's release and advance: agentkv/core/slab_allocator.py:194-278,
 * 416-437; reclamation.py:88-173), in the reference's sequential order, and
 * logs each call for akv_alloc_replay.  Errors are returned at the call
 * (nothing changed, nothing logged) with `err` filled as the device status
 * would be.  Not thread-safe: the caller serialises calls (one lock). */
typedef struct AkvMirror AkvMirror;

/* Op log records: AKV_LOG_HEADER_WORDS int32 words {op, n, readers_min lo,
 * hi, readers_max lo, hi, epoch_interval, readers_active}, then n words:
 * ALLOC the ids handed out; INCREF / DECREF the ids; COW {block, the block
 * owned afterwards (itself when no copy was needed)};
 * RELEASE (n = 0) the safe epoch in the readers_min words; ADVANCE (n = 0). */
#define AKV_LOG_HEADER_WORDS 8
enum {
  AKV_OP_ALLOC = 1,
  AKV_OP_INCREF = 2,
  AKV_OP_DECREF = 3,
  AKV_OP_COW = 4,
  AKV_OP_RELEASE = 5,
  AKV_OP_ADVANCE = 6
};

/* A mirror in the constructor state (akv_alloc_init's); NULL on failure. */
AKV_API AkvMirror* akv_mirror_create(int32_t total_blocks);
AKV_API void akv_mirror_destroy(AkvMirror* m);
/* Replace the mirror's state with host copies of the device arrays
 * (ref_counts, free_ring, limbo_ids [N] int32, limbo_epochs [N] int64,
 * ctl [AKV_CTL_WORDS]); clears the log. */
AKV_API int akv_mirror_load(AkvMirror* m, const int32_t* ref_counts, const int32_t* free_ring,
                            const int32_t* limbo_ids, const int64_t* limbo_epochs, const int64_t* ctl);
/* n alloc() calls: out_ids[n]; AKV_ERR_EXHAUSTED when they would run dry. */
AKV_API int akv_mirror_alloc(AkvMirror* m, int32_t n, const AkvTick* tick, int32_t* out_ids, AkvStatus* err);
/* n inc_ref() calls, all or nothing. */
AKV_API int akv_mirror_incref(AkvMirror* m, const int32_t* ids, int32_t n, const AkvTick* tick, AkvStatus* err);
/* n dec_ref() calls, all or nothing; the retired ids in order and their count. */
AKV_API int akv_mirror_decref(AkvMirror* m, const int32_t* ids, int32_t n, const AkvTick* tick,
                              int32_t* retired_out, int32_t* n_retired, AkvStatus* err);
/* ensure_mutable on one block: *out_block is the block itself when its
 * count is 1 (or 0), else a fresh block (alloc, then dec_ref of the old one;
 * the data copy is the caller's). */
AKV_API int akv_mirror_cow(AkvMirror* m, int32_t block, const AkvTick* tick, int32_t* out_block, AkvStatus* err);
/* The reclaimer's release of pending ids older than safe_before_epoch. */
AKV_API int akv_mirror_release(AkvMirror* m, int64_t safe_before_epoch);
/* EpochReclaimer.maybe_advance. */
AKV_API int akv_mirror_advance(AkvMirror* m, const AkvTick* tick);
/* Copies of the state, in the device arrays' layout: the control words
 * (AKV_CTL_WORDS int64), refcounts, free ring, limbo ids ([N] int32) and
 * limbo epochs ([N] int64); any may be NULL. */
AKV_API int akv_mirror_read(const AkvMirror* m, int64_t* ctl, int32_t* ref_counts, int32_t* free_ring,
                            int32_t* limbo_ids, int64_t* limbo_epochs);
/* One block's refcount (INT32_MIN for a bad id). */
AKV_API int32_t akv_mirror_ref(const AkvMirror* m, int32_t block);
/* Words logged since the last take; copy them out (cap >= the count) and clear. */
AKV_API int64_t akv_mirror_log_words(const AkvMirror* m);
AKV_API int akv_mirror_take_log(AkvMirror* m, int32_t* dst, int64_t cap);
/* Apply an op log (device memory, n_words int32) to the device state with
 * the same rules, one warp, checking each logged id against its own:
 * AKV_ERR_MIRROR in `status` at the first difference.  ctl's LAST_RETIRED /
 * LAST_COPIED words end as the last DECREF / COW record left them.  One
 * launch. */
AKV_API int akv_alloc_replay(const AkvAllocState* st, const int32_t* log, int64_t n_words, AkvStatus* status,
                             void* stream);

#ifdef __cplusplus
}
#endif

#endif /* AGENTKV_B200_H */
