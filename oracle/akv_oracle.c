/*
 * akv_oracle.c — CPU restatement of AgentKV's block-movement, allocator and
 * match_prefix algorithms.  TEST INFRASTRUCTURE ONLY: the tests, the smoke
 * check and the CPU-baseline leg of bench.py use it to check results and to
 * time the reference algorithm on the host; the agentkv_b200 package never
 * links or calls it.
 *
 * Every function follows the reference's own single-threaded code path, one
 * operation at a time (file:line within the agentkv project):
 *   copy / zero ........ triton_kernels.py:194-196 (dst.copy_(src)),
 *                        :222-224 (block.zero_(), +0.0)
 *   allocator .......... slab_allocator.py:155-278 (alloc / inc_ref /
 *                        dec_ref), :387-437 (_do_free, _drain_deferred, _tick)
 *   reclaimer .......... reclamation.py:87-173 (read sections, retire,
 *                        maybe_advance, _try_retire)
 *   ensure_mutable ..... radix_tree.py:286-314
 *   match_prefix ....... radix_tree.py:513-570 (_match_prefix_locked)
 *
 * The batch entry points (orc_*_batch) run the per-op functions in order and,
 * when an op fails, restore the state from before the batch: the same
 * all-or-nothing contract the device batches give.  Without errors a batch
 * equals the reference's sequence of single calls.
 */
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_OK 0
#define ORC_ERR_OUT_OF_RANGE 2
#define ORC_ERR_EXHAUSTED 3
#define ORC_ERR_DOUBLE_FREE 4
#define ORC_ERR_NOT_ALLOCATED 5
#define ORC_ERR_NOT_EXCLUSIVE 6

/* ── block movement ─────────────────────────────────────────────────────── */

/* Sequential dst.copy_(src) per pair (triton_kernels.py:194-196). */
void orc_copy_blocks(char* pool, int64_t bpb, const int32_t* pairs, int32_t n) {
  for (int32_t p = 0; p < n; ++p)
    memmove(pool + (int64_t)pairs[2 * p + 1] * bpb, pool + (int64_t)pairs[2 * p] * bpb,
            (size_t)bpb);
}

/* Same order, each block split across `threads` workers, the way torch's CPU
 * copy_ parallelises one large copy: the workers take equal slices of pair p
 * and meet at a barrier before pair p + 1. */
typedef struct {
  char* pool;
  int64_t bpb;
  const int32_t* ids;   /* pairs [n][2] (copy) or ids [n] (zero) */
  int32_t n;
  int threads;
  int zero;
  pthread_barrier_t* bar;
  int t;
} OrcJob;

static void* orc_worker(void* arg) {
  const OrcJob* j = (const OrcJob*)arg;
  const int64_t slice = ((j->bpb + j->threads - 1) / j->threads + 63) & ~(int64_t)63;
  const int64_t off = slice * j->t;
  const int64_t len = off >= j->bpb ? 0 : ((j->bpb - off) < slice ? (j->bpb - off) : slice);
  for (int32_t p = 0; p < j->n; ++p) {
    if (len > 0) {
      if (j->zero) {
        memset(j->pool + (int64_t)j->ids[p] * j->bpb + off, 0, (size_t)len);
      } else {
        char* d = j->pool + (int64_t)j->ids[2 * p + 1] * j->bpb + off;
        const char* s = j->pool + (int64_t)j->ids[2 * p] * j->bpb + off;
        if (d != s) memcpy(d, s, (size_t)len);
      }
    }
    pthread_barrier_wait(j->bar);
  }
  return NULL;
}

static void orc_run_mt(char* pool, int64_t bpb, const int32_t* ids, int32_t n, int threads,
                       int zero) {
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  pthread_barrier_t bar;
  pthread_barrier_init(&bar, NULL, (unsigned)threads);
  pthread_t th[256];
  OrcJob jobs[256];
  for (int t = 0; t < threads; ++t) {
    jobs[t] = (OrcJob){pool, bpb, ids, n, threads, zero, &bar, t};
    if (t > 0) pthread_create(&th[t], NULL, orc_worker, &jobs[t]);
  }
  orc_worker(&jobs[0]);
  for (int t = 1; t < threads; ++t) pthread_join(th[t], NULL);
  pthread_barrier_destroy(&bar);
}

void orc_copy_blocks_mt(char* pool, int64_t bpb, const int32_t* pairs, int32_t n, int threads) {
  orc_run_mt(pool, bpb, pairs, n, threads, 0);
}

/* block.zero_() per id (triton_kernels.py:222-224): +0.0, all bits clear. */
void orc_zero_blocks(char* pool, int64_t bpb, const int32_t* ids, int32_t n) {
  for (int32_t i = 0; i < n; ++i) memset(pool + (int64_t)ids[i] * bpb, 0, (size_t)bpb);
}

void orc_zero_blocks_mt(char* pool, int64_t bpb, const int32_t* ids, int32_t n, int threads) {
  orc_run_mt(pool, bpb, ids, n, threads, 1);
}

/* ── slab allocator + epoch reclaimer ───────────────────────────────────── */

typedef struct {
  int32_t n;
  int32_t epoch_interval;
  int32_t* ref;         /* _ref_counts */
  int32_t* fl;          /* _free_list deque as a ring */
  int64_t fl_left, fl_size;
  int32_t* pend_id;     /* reclaimer _pending: (epoch, id) FIFO ring */
  int64_t* pend_ep;
  int64_t pend_head, pend_size;
  int32_t* deferred;    /* _deferred_free */
  int64_t def_size;
  int64_t* readers;     /* _active_reader_epochs (a set) */
  int32_t n_readers;
  int64_t op_count, epoch, alloc_count, free_count, peak, advance_count, freed_count;
} OrcAlloc;

static int64_t wrap64(int64_t i, int64_t n) {
  int64_t r = i % n;
  return r < 0 ? r + n : r;
}

OrcAlloc* orc_alloc_new(int32_t n, int32_t epoch_interval) {
  OrcAlloc* a = (OrcAlloc*)calloc(1, sizeof(OrcAlloc));
  a->n = n;
  a->epoch_interval = epoch_interval;
  a->ref = (int32_t*)calloc((size_t)n, 4);
  a->fl = (int32_t*)malloc((size_t)n * 4);
  a->pend_id = (int32_t*)malloc((size_t)n * 4);
  a->pend_ep = (int64_t*)malloc((size_t)n * 8);
  a->deferred = (int32_t*)malloc((size_t)n * 4);
  a->readers = (int64_t*)malloc(64 * 8);
  for (int32_t i = 0; i < n; ++i) a->fl[i] = i; /* deque(range(N)) */
  a->fl_size = n;
  return a;
}

void orc_alloc_delete(OrcAlloc* a) {
  if (!a) return;
  free(a->ref);
  free(a->fl);
  free(a->pend_id);
  free(a->pend_ep);
  free(a->deferred);
  free(a->readers);
  free(a);
}

/* Deep copy used to make batches all-or-nothing. */
static void orc_copy_state(OrcAlloc* dst, const OrcAlloc* src) {
  int32_t* ref = dst->ref; int32_t* fl = dst->fl; int32_t* pid = dst->pend_id;
  int64_t* pep = dst->pend_ep; int32_t* def = dst->deferred; int64_t* rd = dst->readers;
  *dst = *src;
  dst->ref = ref; dst->fl = fl; dst->pend_id = pid; dst->pend_ep = pep; dst->deferred = def;
  dst->readers = rd;
  const size_t n = (size_t)src->n;
  memcpy(dst->ref, src->ref, n * 4);
  memcpy(dst->fl, src->fl, n * 4);
  memcpy(dst->pend_id, src->pend_id, n * 4);
  memcpy(dst->pend_ep, src->pend_ep, n * 8);
  memcpy(dst->deferred, src->deferred, n * 4);
  memcpy(dst->readers, src->readers, 64 * 8);
}

OrcAlloc* orc_alloc_clone(const OrcAlloc* a) {
  OrcAlloc* c = orc_alloc_new(a->n, a->epoch_interval);
  orc_copy_state(c, a);
  return c;
}

static int orc_has_reader(const OrcAlloc* a, int64_t e) {
  for (int32_t i = 0; i < a->n_readers; ++i)
    if (a->readers[i] == e) return 1;
  return 0;
}

/* EpochReclaimer._try_retire (reclamation.py:147-173) with _do_free
 * (slab_allocator.py:387-414) appending to _deferred_free. */
static void orc_try_retire(OrcAlloc* a) {
  if (a->pend_size == 0) return;
  int64_t safe;
  if (a->n_readers > 0) {
    safe = a->readers[0];
    for (int32_t i = 1; i < a->n_readers; ++i)
      if (a->readers[i] < safe) safe = a->readers[i];
  } else {
    safe = a->epoch + 1;
  }
  while (a->pend_size > 0) {
    const int64_t h = wrap64(a->pend_head, a->n);
    if (a->pend_ep[h] < safe) {
      a->deferred[a->def_size++] = a->pend_id[h];
      a->pend_head = h + 1;
      a->pend_size--;
      a->freed_count++;
    } else {
      break;
    }
  }
}

/* EpochReclaimer.maybe_advance (reclamation.py:129-143). */
void orc_maybe_advance(OrcAlloc* a) {
  if (!orc_has_reader(a, a->epoch)) {
    a->epoch++;
    a->advance_count++;
  }
  orc_try_retire(a);
}

/* _drain_deferred: appendleft(deferred.pop()) until empty (:416-422). */
static void orc_drain(OrcAlloc* a) {
  while (a->def_size > 0) {
    const int32_t id = a->deferred[--a->def_size];
    a->fl_left = wrap64(a->fl_left - 1, a->n);
    a->fl[a->fl_left] = id;
    a->fl_size++;
  }
}

/* _tick (:424-437). */
static void orc_tick(OrcAlloc* a) {
  a->op_count++;
  if (a->op_count % a->epoch_interval == 0) orc_maybe_advance(a);
  orc_drain(a);
}

/* alloc (:194-220).  Returns the id, or -ORC_ERR_EXHAUSTED. */
int32_t orc_alloc_one(OrcAlloc* a) {
  if (a->fl_size == 0) return -ORC_ERR_EXHAUSTED;
  const int32_t id = a->fl[wrap64(a->fl_left + a->fl_size - 1, a->n)];
  a->fl_size--;
  a->ref[id] = 1;
  a->alloc_count++;
  const int64_t cur = a->alloc_count - a->free_count;
  if (cur > a->peak) a->peak = cur;
  orc_tick(a);
  return id;
}

/* inc_ref (:222-243). */
int orc_incref(OrcAlloc* a, int32_t id) {
  if (id < 0 || id >= a->n) return ORC_ERR_OUT_OF_RANGE;
  if (a->ref[id] <= 0) return ORC_ERR_NOT_ALLOCATED;
  a->ref[id]++;
  orc_tick(a);
  return ORC_OK;
}

/* dec_ref (:245-278).  *retired = 1 when the count reached zero. */
int orc_decref(OrcAlloc* a, int32_t id, int32_t* retired) {
  if (id < 0 || id >= a->n) return ORC_ERR_OUT_OF_RANGE;
  if (a->ref[id] <= 0) return ORC_ERR_DOUBLE_FREE;
  a->ref[id]--;
  *retired = 0;
  if (a->ref[id] == 0) {
    /* EpochReclaimer.retire (reclamation.py:114-127) */
    const int64_t t = wrap64(a->pend_head + a->pend_size, a->n);
    a->pend_id[t] = id;
    a->pend_ep[t] = a->epoch;
    a->pend_size++;
    orc_try_retire(a);
    a->free_count++;
    *retired = 1;
  }
  orc_tick(a);
  return ORC_OK;
}

/* Read sections (reclamation.py:87-112); the reader set is a set. */
int64_t orc_enter_read(OrcAlloc* a) {
  const int64_t tok = a->epoch;
  if (!orc_has_reader(a, tok) && a->n_readers < 64) a->readers[a->n_readers++] = tok;
  return tok;
}

void orc_leave_read(OrcAlloc* a, int64_t tok) {
  for (int32_t i = 0; i < a->n_readers; ++i) {
    if (a->readers[i] == tok) {
      a->readers[i] = a->readers[--a->n_readers];
      break;
    }
  }
  orc_try_retire(a);
}

/* State export.  free_out receives the free list left to right; ctl_out:
 * [0] free size [1] pending [2] deferred [3] op_count [4] epoch
 * [5] alloc_count [6] free_count [7] peak [8] advance_count [9] freed_count
 * [10] allocated (ref > 0) */
void orc_alloc_state(const OrcAlloc* a, int32_t* ref_out, int32_t* free_out, int64_t* ctl_out) {
  if (ref_out) memcpy(ref_out, a->ref, (size_t)a->n * 4);
  if (free_out)
    for (int64_t i = 0; i < a->fl_size; ++i) free_out[i] = a->fl[wrap64(a->fl_left + i, a->n)];
  if (ctl_out) {
    int64_t allocated = 0;
    for (int32_t i = 0; i < a->n; ++i) allocated += a->ref[i] > 0;
    ctl_out[0] = a->fl_size;
    ctl_out[1] = a->pend_size;
    ctl_out[2] = a->def_size;
    ctl_out[3] = a->op_count;
    ctl_out[4] = a->epoch;
    ctl_out[5] = a->alloc_count;
    ctl_out[6] = a->free_count;
    ctl_out[7] = a->peak;
    ctl_out[8] = a->advance_count;
    ctl_out[9] = a->freed_count;
    ctl_out[10] = allocated;
  }
}

/* One block's refcount (the reference's int(self._ref_counts[bid].item())). */
int32_t orc_ref_count(const OrcAlloc* a, int32_t id) {
  return (id >= 0 && id < a->n) ? a->ref[id] : -1;
}

/* Pending ids (FIFO order) and deferred ids (append order). */
void orc_alloc_limbo(const OrcAlloc* a, int32_t* pend_out, int64_t* pend_ep_out, int32_t* def_out) {
  for (int64_t i = 0; i < a->pend_size; ++i) {
    const int64_t h = wrap64(a->pend_head + i, a->n);
    if (pend_out) pend_out[i] = a->pend_id[h];
    if (pend_ep_out) pend_ep_out[i] = a->pend_ep[h];
  }
  if (def_out) memcpy(def_out, a->deferred, (size_t)a->def_size * 4);
}

/* ── sequential runs (the reference's single calls in a loop) ───────────── */
/* Stop at the first failing op, leaving the ops before it applied, exactly
 * as a loop of reference calls that raises would.  Return the number of ops
 * applied. */
int32_t orc_alloc_seq(OrcAlloc* a, int32_t n, int32_t* out) {
  for (int32_t k = 0; k < n; ++k) {
    const int32_t id = orc_alloc_one(a);
    if (id < 0) return k;
    out[k] = id;
  }
  return n;
}

int32_t orc_incref_seq(OrcAlloc* a, const int32_t* ids, int32_t n) {
  for (int32_t k = 0; k < n; ++k)
    if (orc_incref(a, ids[k]) != ORC_OK) return k;
  return n;
}

int32_t orc_decref_seq(OrcAlloc* a, const int32_t* ids, int32_t n) {
  int32_t r;
  for (int32_t k = 0; k < n; ++k)
    if (orc_decref(a, ids[k], &r) != ORC_OK) return k;
  return n;
}

/* ── all-or-nothing batches ─────────────────────────────────────────────── */

/* Returns ORC_OK, or the error code with *fail_index = failing position. */
int orc_alloc_batch(OrcAlloc* a, int32_t n, int32_t* out, int32_t* fail_index) {
  OrcAlloc* snap = orc_alloc_clone(a);
  for (int32_t k = 0; k < n; ++k) {
    const int32_t id = orc_alloc_one(a);
    if (id < 0) {
      orc_copy_state(a, snap);
      orc_alloc_delete(snap);
      if (fail_index) *fail_index = k;
      return -id;
    }
    out[k] = id;
  }
  orc_alloc_delete(snap);
  return ORC_OK;
}

int orc_incref_batch(OrcAlloc* a, const int32_t* ids, int32_t n, int32_t* fail_index) {
  OrcAlloc* snap = orc_alloc_clone(a);
  for (int32_t k = 0; k < n; ++k) {
    const int rc = orc_incref(a, ids[k]);
    if (rc != ORC_OK) {
      orc_copy_state(a, snap);
      orc_alloc_delete(snap);
      if (fail_index) *fail_index = k;
      return rc;
    }
  }
  orc_alloc_delete(snap);
  return ORC_OK;
}

int orc_decref_batch(OrcAlloc* a, const int32_t* ids, int32_t n, int32_t* retired_out,
                     int32_t* n_retired, int32_t* fail_index) {
  OrcAlloc* snap = orc_alloc_clone(a);
  int32_t nr = 0;
  for (int32_t k = 0; k < n; ++k) {
    int32_t r = 0;
    const int rc = orc_decref(a, ids[k], &r);
    if (rc != ORC_OK) {
      orc_copy_state(a, snap);
      orc_alloc_delete(snap);
      if (fail_index) *fail_index = k;
      if (n_retired) *n_retired = 0;
      return rc;
    }
    if (r) {
      if (retired_out) retired_out[nr] = ids[k];
      nr++;
    }
  }
  orc_alloc_delete(snap);
  if (n_retired) *n_retired = nr;
  return ORC_OK;
}

/* ensure_mutable_block over n requests, in order (radix_tree.py:286-314):
 * if ref_count(b) > 1: new = alloc(); copy_block(b, new); dec_ref(b).  The
 * pool may be NULL (metadata only). */
int orc_cow_batch(OrcAlloc* a, char* pool, int64_t bpb, const int32_t* blocks, int32_t n,
                  int32_t* out_blocks, int32_t* out_copied, int32_t* fail_index) {
  OrcAlloc* snap = orc_alloc_clone(a);
  for (int32_t i = 0; i < n; ++i) {
    const int32_t b = blocks[i];
    if (b < 0 || b >= a->n) {
      orc_copy_state(a, snap);
      orc_alloc_delete(snap);
      if (fail_index) *fail_index = i;
      return ORC_ERR_OUT_OF_RANGE;
    }
    if (a->ref[b] > 1) {
      const int32_t nb = orc_alloc_one(a);
      if (nb < 0) {
        orc_copy_state(a, snap);
        orc_alloc_delete(snap);
        if (fail_index) *fail_index = i;
        return -nb;
      }
      if (pool) memmove(pool + (int64_t)nb * bpb, pool + (int64_t)b * bpb, (size_t)bpb);
      int32_t r;
      orc_decref(a, b, &r);
      out_blocks[i] = nb;
      out_copied[i] = 1;
    } else {
      out_blocks[i] = b;
      out_copied[i] = 0;
    }
  }
  orc_alloc_delete(snap);
  return ORC_OK;
}

/* ── match_prefix over a CSR view of the shared tree ────────────────────── */
/* child_ptr[node]..child_ptr[node+1] index child_key (sorted) / child_id;
 * node ids are the tree's own ids; edge of node = edge_tokens[edge_off[node]
 * .. + edge_len[node]]. */
static int32_t csr_child(const int64_t* child_ptr, const int32_t* child_key,
                         const int32_t* child_id, int32_t node, int32_t tok) {
  int64_t lo = child_ptr[node], hi = child_ptr[node + 1];
  while (lo < hi) {
    const int64_t mid = lo + (hi - lo) / 2;
    if (child_key[mid] < tok) lo = mid + 1;
    else hi = mid;
  }
  if (lo < child_ptr[node + 1] && child_key[lo] == tok) return child_id[lo];
  return -1;
}

/* _match_prefix_locked (radix_tree.py:513-570), plus the number of
 * `tokens[matched + i] != et` evaluations its edge loop performs. */
void orc_match_prefix(const int64_t* child_ptr, const int32_t* child_key, const int32_t* child_id,
                      const int64_t* edge_off, const int32_t* edge_len,
                      const int32_t* edge_tokens, const int32_t* tokens, const int64_t* q_off,
                      int32_t nq, int32_t block_size, int32_t* out_node, int32_t* out_len,
                      int64_t* out_compared) {
  for (int32_t q = 0; q < nq; ++q) {
    const int32_t* t = tokens + q_off[q];
    const int64_t len = q_off[q + 1] - q_off[q];
    int32_t cur = 0;
    int64_t matched = 0, compared = 0;
    while (matched < len) {
      const int32_t child = csr_child(child_ptr, child_key, child_id, cur, t[matched]);
      if (child < 0) break;
      const int32_t* e = edge_tokens + edge_off[child];
      const int64_t el = edge_len[child];
      int64_t em = 0;
      for (int64_t i = 0; i < el; ++i) {
        if (matched + i >= len) break;
        compared++;
        if (t[matched + i] != e[i]) break;
        em++;
      }
      if (em == 0) break;
      if (em < el) break; /* partial edge: no credit */
      matched += em;
      cur = child;
    }
    matched = (matched / block_size) * block_size;
    out_node[q] = matched == 0 ? -1 : cur;
    out_len[q] = (int32_t)matched;
    if (out_compared) out_compared[q] = compared;
  }
}


