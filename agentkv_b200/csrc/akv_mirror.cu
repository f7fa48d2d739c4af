// akv_mirror.cu — the allocator's per-call operations answered on the host.
//
// The reference's per-call API (SlabAllocator.alloc / inc_ref / dec_ref,
// DualRadixTree.ensure_mutable_block, EpochReclaimer.enter/leave/maybe_advance:
// agentkv/core/slab_allocator.py:194-278, 416-437; reclamation.py:88-173)
// returns block ids and raises its errors at the call.  On the device each
// such call would be a launch and a wait for the answer; here a host copy of
// the allocator state (the mirror) applies the call at once, in the
// reference's sequential order, and appends it to an op log.  The device
// state catches up when something on the device needs it: the log is
// replayed by akv_alloc_replay, one warp applying the same operations with
// the same rules and checking every id the host handed out against its own
// (AKV_ERR_MIRROR on any difference).  After device batches the mirror is
// reloaded from the device arrays (akv_mirror_load).
//
// Layout follows AkvAllocState: refcounts; the free deque as a ring (ids at
// ring[(left + i) mod N], i < size, popped on the right, pushed on the left);
// retired ids in a FIFO with cursors head <= rel <= tail ([head, rel) deferred,
// [rel, tail) pending with the epoch each retired in); counters as AKV_CTL_*.
//
// Log records (int32 words): an 8-word header {op, n, readers_min lo/hi,
// readers_max lo/hi, epoch_interval, readers_active} and n payload words:
//   ALLOC   the n ids handed out         INCREF  the n ids
//   DECREF  the n ids                    COW     {block, block owned after}
//                                        (the same block: no copy)
//   RELEASE n = 0, safe epoch in the readers_min words
//   ADVANCE n = 0
#include <algorithm>
#include <cstring>
#include <new>
#include <unordered_map>
#include <vector>

#include "akv_common.cuh"

struct AkvMirror {
  int32_t n;
  std::vector<int32_t> ref, ring, limbo_ids;
  std::vector<int64_t> limbo_epochs;
  int64_t ctl[AKV_CTL_WORDS];
  std::vector<int32_t> log;
};

namespace {

int64_t wrap_h(int64_t i, int64_t n) {
  const int64_t r = i % n;
  return r < 0 ? r + n : r;
}

void fail(AkvStatus* err, int32_t code, int32_t index, int32_t id, int32_t observed) {
  if (err == nullptr) return;
  std::memset(err, 0, sizeof(*err));
  err->code = code;
  err->index = index;
  err->id = id;
  err->observed = observed;
}

void log_header(AkvMirror* m, int32_t op, int32_t n, const AkvTick* tk) {
  const int64_t rmin = tk != nullptr ? tk->readers_min : 0, rmax = tk != nullptr ? tk->readers_max : 0;
  const int32_t h[AKV_LOG_HEADER_WORDS] = {op,
                                    n,
                                    static_cast<int32_t>(rmin & 0xffffffff),
                                    static_cast<int32_t>(rmin >> 32),
                                    static_cast<int32_t>(rmax & 0xffffffff),
                                    static_cast<int32_t>(rmax >> 32),
                                    tk != nullptr ? tk->epoch_interval : 0,
                                    tk != nullptr ? tk->readers_active : 0};
  m->log.insert(m->log.end(), h, h + AKV_LOG_HEADER_WORDS);
}

// EpochReclaimer._try_retire with the given safe epoch.
void try_retire(AkvMirror* m, int64_t safe) {
  int64_t* c = m->ctl;
  while (c[AKV_CTL_LIMBO_REL] < c[AKV_CTL_LIMBO_TAIL] &&
         m->limbo_epochs[wrap_h(c[AKV_CTL_LIMBO_REL], m->n)] < safe) {
    ++c[AKV_CTL_LIMBO_REL];
    ++c[AKV_CTL_RELEASED];
  }
}

int64_t safe_epoch(const AkvMirror* m, const AkvTick* tk) {
  return tk->readers_active ? tk->readers_min : m->ctl[AKV_CTL_EPOCH] + 1;
}

// EpochReclaimer.maybe_advance: the epoch moves unless a reader holds it (a
// reader's epoch is never above the current one, so "no reader in the
// current epoch" is "the current epoch is above every reader's").
void maybe_advance(AkvMirror* m, const AkvTick* tk) {
  int64_t* c = m->ctl;
  if (!tk->readers_active || c[AKV_CTL_EPOCH] > tk->readers_max) {
    ++c[AKV_CTL_EPOCH];
    ++c[AKV_CTL_ADVANCES];
  }
  try_retire(m, safe_epoch(m, tk));
}

// SlabAllocator._drain_deferred: deferred ids to the left of the free deque,
// in their order.
void drain(AkvMirror* m) {
  int64_t* c = m->ctl;
  const int64_t d = c[AKV_CTL_LIMBO_REL] - c[AKV_CTL_LIMBO_HEAD];
  for (int64_t j = d - 1; j >= 0; --j) {
    c[AKV_CTL_FREE_LEFT] = wrap_h(c[AKV_CTL_FREE_LEFT] - 1, m->n);
    m->ring[c[AKV_CTL_FREE_LEFT]] = m->limbo_ids[wrap_h(c[AKV_CTL_LIMBO_HEAD] + j, m->n)];
  }
  c[AKV_CTL_FREE_SIZE] += d;
  c[AKV_CTL_LIMBO_HEAD] = c[AKV_CTL_LIMBO_REL];
}

// SlabAllocator._tick.
void tick(AkvMirror* m, const AkvTick* tk) {
  if (++m->ctl[AKV_CTL_OPS] % tk->epoch_interval == 0) maybe_advance(m, tk);
  drain(m);
}

// EpochReclaimer.retire.
void retire(AkvMirror* m, int32_t id, const AkvTick* tk) {
  int64_t* c = m->ctl;
  const int64_t pos = wrap_h(c[AKV_CTL_LIMBO_TAIL], m->n);
  m->limbo_ids[pos] = id;
  m->limbo_epochs[pos] = c[AKV_CTL_EPOCH];
  ++c[AKV_CTL_LIMBO_TAIL];
  try_retire(m, safe_epoch(m, tk));
}

// SlabAllocator.alloc after its checks.
int32_t pop(AkvMirror* m, const AkvTick* tk) {
  int64_t* c = m->ctl;
  const int32_t id = m->ring[wrap_h(c[AKV_CTL_FREE_LEFT] + c[AKV_CTL_FREE_SIZE] - 1, m->n)];
  --c[AKV_CTL_FREE_SIZE];
  m->ref[id] = 1;
  ++c[AKV_CTL_ALLOCS];
  c[AKV_CTL_PEAK] = std::max(c[AKV_CTL_PEAK], c[AKV_CTL_ALLOCS] - c[AKV_CTL_FREES]);
  tick(m, tk);
  return id;
}

// Can `k` more pops run one after another?  The first needs a free id; the
// later ones also see the deferred ids, which the first pop's tick drains
// (ticks release nothing new: a pending id always carries an epoch at or
// above the oldest reader's).
bool can_pop(const AkvMirror* m, int64_t k) {
  const int64_t f = m->ctl[AKV_CTL_FREE_SIZE];
  const int64_t d = m->ctl[AKV_CTL_LIMBO_REL] - m->ctl[AKV_CTL_LIMBO_HEAD];
  return k <= 0 || (f >= 1 && f + d >= k);
}

bool tick_ok(const AkvTick* tk) { return tk != nullptr && tk->epoch_interval > 0; }

}  // namespace

extern "C" AkvMirror* akv_mirror_create(int32_t total_blocks) {
  if (total_blocks <= 0) {
    akv_set_error("akv_mirror_create: total_blocks=%d", total_blocks);
    return nullptr;
  }
  AkvMirror* m = new (std::nothrow) AkvMirror();
  if (m == nullptr) {
    akv_set_error("akv_mirror_create: out of host memory");
    return nullptr;
  }
  try {
    m->n = total_blocks;
    m->ref.assign(total_blocks, 0);
    m->ring.resize(total_blocks);
    for (int32_t i = 0; i < total_blocks; ++i) m->ring[i] = i;
    m->limbo_ids.assign(total_blocks, -1);
    m->limbo_epochs.assign(total_blocks, 0);
  } catch (...) {
    delete m;
    akv_set_error("akv_mirror_create: out of host memory");
    return nullptr;
  }
  std::memset(m->ctl, 0, sizeof(m->ctl));
  m->ctl[AKV_CTL_FREE_SIZE] = total_blocks;
  return m;
}

extern "C" void akv_mirror_destroy(AkvMirror* m) { delete m; }

extern "C" int akv_mirror_load(AkvMirror* m, const int32_t* ref_counts, const int32_t* free_ring,
                               const int32_t* limbo_ids, const int64_t* limbo_epochs, const int64_t* ctl) {
  AKV_ARG_CHECK(m != nullptr && ref_counts && free_ring && limbo_ids && limbo_epochs && ctl,
                "akv_mirror_load: NULL argument");
  const size_t n = static_cast<size_t>(m->n);
  std::memcpy(m->ref.data(), ref_counts, 4 * n);
  std::memcpy(m->ring.data(), free_ring, 4 * n);
  std::memcpy(m->limbo_ids.data(), limbo_ids, 4 * n);
  std::memcpy(m->limbo_epochs.data(), limbo_epochs, 8 * n);
  std::memcpy(m->ctl, ctl, sizeof(m->ctl));
  m->ctl[AKV_CTL_DONE] = 0;
  m->log.clear();
  return AKV_OK;
}

extern "C" int akv_mirror_alloc(AkvMirror* m, int32_t n, const AkvTick* tk, int32_t* out_ids, AkvStatus* err) {
  AKV_ARG_CHECK(m != nullptr && tick_ok(tk) && n >= 0 && (n == 0 || out_ids != nullptr),
                "akv_mirror_alloc: bad arguments");
  if (n == 0) return AKV_OK;
  if (!can_pop(m, n)) {
    fail(err, AKV_ERR_EXHAUSTED, 0, -1, static_cast<int32_t>(m->ctl[AKV_CTL_FREE_SIZE]));
    return AKV_ERR_EXHAUSTED;
  }
  log_header(m, AKV_OP_ALLOC, n, tk);
  for (int32_t i = 0; i < n; ++i) {
    out_ids[i] = pop(m, tk);
    m->log.push_back(out_ids[i]);
  }
  return AKV_OK;
}

extern "C" int akv_mirror_incref(AkvMirror* m, const int32_t* ids, int32_t n, const AkvTick* tk, AkvStatus* err) {
  AKV_ARG_CHECK(m != nullptr && tick_ok(tk) && n >= 0 && (n == 0 || ids != nullptr),
                "akv_mirror_incref: bad arguments");
  for (int32_t k = 0; k < n; ++k) {  // all or nothing, as the batch does
    const int32_t x = ids[k];
    if (static_cast<uint32_t>(x) >= static_cast<uint32_t>(m->n)) {
      fail(err, AKV_ERR_OUT_OF_RANGE, k, x, m->n);
      return AKV_ERR_OUT_OF_RANGE;
    }
    if (m->ref[x] <= 0) {
      fail(err, AKV_ERR_NOT_ALLOCATED, k, x, m->ref[x]);
      return AKV_ERR_NOT_ALLOCATED;
    }
  }
  if (n == 0) return AKV_OK;
  log_header(m, AKV_OP_INCREF, n, tk);
  m->log.insert(m->log.end(), ids, ids + n);
  for (int32_t k = 0; k < n; ++k) {
    ++m->ref[ids[k]];
    tick(m, tk);
  }
  return AKV_OK;
}

extern "C" int akv_mirror_decref(AkvMirror* m, const int32_t* ids, int32_t n, const AkvTick* tk,
                                 int32_t* retired_out, int32_t* n_retired, AkvStatus* err) {
  AKV_ARG_CHECK(m != nullptr && tick_ok(tk) && n >= 0 && (n == 0 || ids != nullptr),
                "akv_mirror_decref: bad arguments");
  if (n_retired != nullptr) *n_retired = 0;
  // all or nothing: the first call that would find a count at zero refuses
  // the batch (counts of repeated ids taken in order)
  std::unordered_map<int32_t, int32_t> seen;
  for (int32_t k = 0; k < n; ++k) {
    const int32_t x = ids[k];
    if (static_cast<uint32_t>(x) >= static_cast<uint32_t>(m->n)) {
      fail(err, AKV_ERR_OUT_OF_RANGE, k, x, m->n);
      return AKV_ERR_OUT_OF_RANGE;
    }
    const int32_t left = m->ref[x] - seen[x];
    if (left <= 0) {
      fail(err, AKV_ERR_DOUBLE_FREE, k, x, left);
      return AKV_ERR_DOUBLE_FREE;
    }
    ++seen[x];
  }
  if (n == 0) return AKV_OK;
  int64_t* c = m->ctl;
  c[AKV_CTL_LAST_RETIRED] = 0;
  log_header(m, AKV_OP_DECREF, n, tk);
  m->log.insert(m->log.end(), ids, ids + n);
  for (int32_t k = 0; k < n; ++k) {
    const int32_t x = ids[k];
    if (--m->ref[x] == 0) {
      retire(m, x, tk);
      ++c[AKV_CTL_FREES];
      if (retired_out != nullptr) retired_out[c[AKV_CTL_LAST_RETIRED]] = x;
      ++c[AKV_CTL_LAST_RETIRED];
    }
    tick(m, tk);
  }
  if (n_retired != nullptr) *n_retired = static_cast<int32_t>(c[AKV_CTL_LAST_RETIRED]);
  return AKV_OK;
}

extern "C" int akv_mirror_cow(AkvMirror* m, int32_t block, const AkvTick* tk, int32_t* out_block, AkvStatus* err) {
  AKV_ARG_CHECK(m != nullptr && tick_ok(tk) && out_block != nullptr, "akv_mirror_cow: bad arguments");
  if (static_cast<uint32_t>(block) >= static_cast<uint32_t>(m->n)) {
    fail(err, AKV_ERR_OUT_OF_RANGE, 0, block, m->n);
    return AKV_ERR_OUT_OF_RANGE;
  }
  *out_block = block;
  if (m->ref[block] <= 1) {  // exclusively owned (or free): nothing to do
    m->ctl[AKV_CTL_LAST_COPIED] = 0;
    log_header(m, AKV_OP_COW, 2, tk);
    m->log.push_back(block);
    m->log.push_back(block);
    return AKV_OK;
  }
  if (!can_pop(m, 1)) {
    fail(err, AKV_ERR_EXHAUSTED, 0, -1, static_cast<int32_t>(m->ctl[AKV_CTL_FREE_SIZE]));
    return AKV_ERR_EXHAUSTED;
  }
  // ensure_mutable_block: alloc(), copy, dec_ref(old) — the old count stays
  // above zero
  const int32_t fresh = pop(m, tk);
  --m->ref[block];
  tick(m, tk);
  m->ctl[AKV_CTL_LAST_COPIED] = 1;
  *out_block = fresh;
  log_header(m, AKV_OP_COW, 2, tk);
  m->log.push_back(block);
  m->log.push_back(fresh);
  return AKV_OK;
}

extern "C" int akv_mirror_release(AkvMirror* m, int64_t safe_before_epoch) {
  AKV_ARG_CHECK(m != nullptr, "akv_mirror_release: NULL mirror");
  try_retire(m, safe_before_epoch);
  AkvTick t{safe_before_epoch, 0, 0, 0};
  log_header(m, AKV_OP_RELEASE, 0, &t);
  return AKV_OK;
}

extern "C" int akv_mirror_advance(AkvMirror* m, const AkvTick* tk) {
  AKV_ARG_CHECK(m != nullptr && tk != nullptr, "akv_mirror_advance: bad arguments");
  maybe_advance(m, tk);
  log_header(m, AKV_OP_ADVANCE, 0, tk);
  return AKV_OK;
}

extern "C" int akv_mirror_read(const AkvMirror* m, int64_t* ctl, int32_t* ref_counts, int32_t* free_ring,
                               int32_t* limbo_ids, int64_t* limbo_epochs) {
  AKV_ARG_CHECK(m != nullptr, "akv_mirror_read: NULL mirror");
  const size_t n = static_cast<size_t>(m->n);
  if (ctl != nullptr) std::memcpy(ctl, m->ctl, sizeof(m->ctl));
  if (ref_counts != nullptr) std::memcpy(ref_counts, m->ref.data(), 4 * n);
  if (free_ring != nullptr) std::memcpy(free_ring, m->ring.data(), 4 * n);
  if (limbo_ids != nullptr) std::memcpy(limbo_ids, m->limbo_ids.data(), 4 * n);
  if (limbo_epochs != nullptr) std::memcpy(limbo_epochs, m->limbo_epochs.data(), 8 * n);
  return AKV_OK;
}

extern "C" int32_t akv_mirror_ref(const AkvMirror* m, int32_t block) {
  if (m == nullptr || static_cast<uint32_t>(block) >= static_cast<uint32_t>(m->n)) return INT32_MIN;
  return m->ref[block];
}

extern "C" int64_t akv_mirror_log_words(const AkvMirror* m) {
  return m != nullptr ? static_cast<int64_t>(m->log.size()) : -1;
}

extern "C" int akv_mirror_take_log(AkvMirror* m, int32_t* dst, int64_t cap) {
  AKV_ARG_CHECK(m != nullptr && (m->log.empty() || dst != nullptr), "akv_mirror_take_log: bad arguments");
  AKV_ARG_CHECK(cap >= static_cast<int64_t>(m->log.size()), "akv_mirror_take_log: %lld words, room for %lld",
                static_cast<long long>(m->log.size()), static_cast<long long>(cap));
  if (!m->log.empty()) std::memcpy(dst, m->log.data(), 4 * m->log.size());
  m->log.clear();
  return AKV_OK;
}
