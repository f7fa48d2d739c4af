// akv_agents.cu — a batch of agents' per-call steps applied on the device.
//
// The ReAct-style multi-agent pattern drives the pool one call at a time:
// per agent slot and step, fork another agent into a slot (free the slot's
// agent, fork), copy-on-write the tail block, free an agent and restart it
// from the shared root, advance the epoch, or append a block
// (DualRadixTree.free / fork / ensure_mutable_block(h, -1) / allocate_block,
// EpochReclaimer.maybe_advance: agentkv/core/radix_tree.py:222-314,351-377;
// reclamation.py:129-143).  Here the agents' residual block tables live in
// device memory and one warp applies a whole batch of steps, with the
// reference's sequential allocator semantics op by op (slab_allocator.py:
// 194-278, 416-437; reclamation.py:114-173): ids popped from the right of
// the free deque, refcounts, retirements through the reclaimer, a tick per
// op with the epoch advanced every epoch_interval ops unless a reader holds
// it, retired ids drained to the left of the free deque.  Each step's
// copy-on-write pairs are written in the counted-copy batch format (an
// int64 count, then the pairs), ready for akv_copy_blocks_counted.
//
// The allocator's cursors and counters are held in registers by every lane
// (all lanes compute the same values); lane 0 reads and writes the shared
// words and broadcasts what it read.  A fork's increments and a free's
// decrements are spread over the lanes, 32 ids at a time.  Every action is
// validated before it mutates anything, so a failing action changes nothing
// and leaves every earlier one applied, as the reference's calls would; the
// kernel then records the error (status) and stops.
#include "akv_common.cuh"

namespace {

constexpr uint32_t kFull = 0xffffffffu;

struct Cursors {
  int64_t left, size, head, rel, tail, ops, epoch, allocs, frees, peak, advances, released;
};

struct Agents {
  AkvAllocState st;
  AkvTick tk;
  int64_t N;
  int32_t* tables;  // [n_agents][cap]
  int32_t* lens;    // [n_agents]
  int32_t n_agents, cap;
  const int32_t* root;
  int32_t root_len;
  AkvStatus* status;
  int lane;
};

AKV_DEV int64_t wrapn(int64_t i, int64_t n) {
  const int64_t r = i % n;
  return r < 0 ? r + n : r;
}

// Loads of words this kernel may have written earlier (another lane's store,
// ordered by __syncwarp) go around L1.
AKV_DEV int32_t vload(const int32_t* p) { return *reinterpret_cast<const volatile int32_t*>(p); }

AKV_DEV int32_t lane0_load(const int32_t* p, int lane) {
  int32_t v = 0;
  if (lane == 0) v = *reinterpret_cast<const volatile int32_t*>(p);
  return __shfl_sync(kFull, v, 0);
}

AKV_DEV int64_t lane0_load64(const int64_t* p, int lane) {
  int64_t v = 0;
  if (lane == 0) v = *reinterpret_cast<const volatile int64_t*>(p);
  return __shfl_sync(kFull, v, 0);
}

AKV_DEV Cursors load_cursors(const Agents& g) {
  const int64_t* ctl = g.st.ctl;
  Cursors c;
  c.left = lane0_load64(&ctl[AKV_CTL_FREE_LEFT], g.lane);
  c.size = lane0_load64(&ctl[AKV_CTL_FREE_SIZE], g.lane);
  c.head = lane0_load64(&ctl[AKV_CTL_LIMBO_HEAD], g.lane);
  c.rel = lane0_load64(&ctl[AKV_CTL_LIMBO_REL], g.lane);
  c.tail = lane0_load64(&ctl[AKV_CTL_LIMBO_TAIL], g.lane);
  c.ops = lane0_load64(&ctl[AKV_CTL_OPS], g.lane);
  c.epoch = lane0_load64(&ctl[AKV_CTL_EPOCH], g.lane);
  c.allocs = lane0_load64(&ctl[AKV_CTL_ALLOCS], g.lane);
  c.frees = lane0_load64(&ctl[AKV_CTL_FREES], g.lane);
  c.peak = lane0_load64(&ctl[AKV_CTL_PEAK], g.lane);
  c.advances = lane0_load64(&ctl[AKV_CTL_ADVANCES], g.lane);
  c.released = lane0_load64(&ctl[AKV_CTL_RELEASED], g.lane);
  return c;
}

// Lane 0 only.
AKV_DEV void store_cursors(const Cursors& c, int64_t* ctl) {
  ctl[AKV_CTL_FREE_LEFT] = c.left;
  ctl[AKV_CTL_FREE_SIZE] = c.size;
  ctl[AKV_CTL_LIMBO_HEAD] = c.head;
  ctl[AKV_CTL_LIMBO_REL] = c.rel;
  ctl[AKV_CTL_LIMBO_TAIL] = c.tail;
  ctl[AKV_CTL_OPS] = c.ops;
  ctl[AKV_CTL_EPOCH] = c.epoch;
  ctl[AKV_CTL_ALLOCS] = c.allocs;
  ctl[AKV_CTL_FREES] = c.frees;
  ctl[AKV_CTL_PEAK] = c.peak;
  ctl[AKV_CTL_ADVANCES] = c.advances;
  ctl[AKV_CTL_RELEASED] = c.released;
}

AKV_DEV bool advance_allowed(const Cursors& c, const AkvTick& tk) {
  // a reader always holds the current epoch: the epoch moves only when none is open
  return !tk.readers_active || c.epoch > tk.readers_max;
}

// The reclaimer's _try_retire: pending ids retired before the oldest reader
// (all of them when no reader is open) become deferred, in FIFO order.
AKV_DEV void try_retire_to(Cursors& c, const Agents& g, int64_t safe) {
  while (c.rel < c.tail && lane0_load64(&g.st.limbo_epochs[wrapn(c.rel, g.N)], g.lane) < safe) {
    ++c.rel;
    ++c.released;
  }
}

AKV_DEV void try_retire(Cursors& c, const Agents& g) {
  try_retire_to(c, g, g.tk.readers_active ? g.tk.readers_min : c.epoch + 1);
}

// _drain_deferred: the deferred ids go to the left of the free deque, keeping
// their order.
AKV_DEV void drain(Cursors& c, const Agents& g) {
  const int64_t d = c.rel - c.head;
  if (d <= 0) return;
  for (int64_t j = g.lane; j < d; j += 32)
    g.st.free_ring[wrapn(c.left - d + j, g.N)] = vload(&g.st.limbo_ids[wrapn(c.head + j, g.N)]);
  __syncwarp();
  c.left = wrapn(c.left - d, g.N);
  c.size += d;
  c.head = c.rel;
}

// n consecutive _tick()s with no retirement among them (an advance's
// try_retire then has nothing new to release, so one drain at the end
// leaves the state the n ticks would).
AKV_DEV void ticks(Cursors& c, const Agents& g, int64_t n) {
  if (n <= 0) return;
  if (advance_allowed(c, g.tk)) {
    const int64_t iv = g.tk.epoch_interval;
    const int64_t adv = (c.ops + n) / iv - c.ops / iv;
    c.epoch += adv;
    c.advances += adv;
  }
  c.ops += n;
  drain(c, g);
}

// EpochReclaimer.retire: the id joins the pending queue with the current
// epoch and the release runs.
AKV_DEV void retire(Cursors& c, const Agents& g, int32_t id) {
  ++c.frees;
  if (g.lane == 0) {
    const int64_t pos = wrapn(c.tail, g.N);
    g.st.limbo_ids[pos] = id;
    g.st.limbo_epochs[pos] = c.epoch;
  }
  __syncwarp();
  ++c.tail;
  try_retire(c, g);
}

// alloc(): the rightmost free id, refcount 1, a tick.  -1 when the pool is
// exhausted (nothing changed).
AKV_DEV int32_t op_alloc(Cursors& c, const Agents& g) {
  if (c.size == 0) return -1;
  const int32_t id = lane0_load(&g.st.free_ring[wrapn(c.left + c.size - 1, g.N)], g.lane);
  --c.size;
  if (g.lane == 0) g.st.ref_counts[id] = 1;
  __syncwarp();
  ++c.allocs;
  const int64_t cur = c.allocs - c.frees;
  if (cur > c.peak) c.peak = cur;
  ticks(c, g, 1);
  return id;
}

// fork's inc_ref of every block of `src` (n ids), then `dst` holds the same
// table.  Validated first: AKV_ERR_NOT_ALLOCATED / OUT_OF_RANGE change nothing.
// With dst == nullptr only the increments and their ticks (the inc_ref
// batch of a replayed log).
AKV_DEV int fork_into(Cursors& c, const Agents& g, const int32_t* src, int32_t n, int32_t* dst, int32_t* dst_len,
                      int32_t& bad_id) {
  if (dst != nullptr && n > g.cap) {
    bad_id = n;
    return AKV_ERR_INVALID_ARG;
  }
  for (int32_t i0 = 0; i0 < n; i0 += 32) {
    const int32_t i = i0 + g.lane;
    int32_t x = -1, r = 1;
    if (i < n) {
      x = vload(&src[i]);
      r = static_cast<uint32_t>(x) < static_cast<uint32_t>(g.N) ? vload(&g.st.ref_counts[x]) : -1;
    }
    const uint32_t badm = __ballot_sync(kFull, i < n && r <= 0);
    if (badm) {
      bad_id = __shfl_sync(kFull, x, __ffs(badm) - 1);
      const int32_t br = __shfl_sync(kFull, r, __ffs(badm) - 1);
      return br < 0 ? AKV_ERR_OUT_OF_RANGE : AKV_ERR_NOT_ALLOCATED;
    }
  }
  for (int32_t i0 = 0; i0 < n; i0 += 32) {
    const int32_t i = i0 + g.lane;
    const int32_t x = i < n ? vload(&src[i]) : -1;
    const uint32_t peers = __match_any_sync(kFull, x);
    if (x >= 0 && g.lane == __ffs(peers) - 1) atomicAdd(&g.st.ref_counts[x], __popc(peers));
    if (i < n && dst != nullptr) dst[i] = x;
  }
  __syncwarp();
  if (g.lane == 0 && dst_len != nullptr) *dst_len = n;
  __syncwarp();
  ticks(c, g, n);
  return AKV_OK;
}

// n dec_ref() calls in order (ids may repeat): a block whose count reaches
// zero retires at its own op.  32 ids at a time; a chunk holding a repeated
// id goes one id at a time, so that the retirement lands on the id's last
// occurrence.  A count already at zero is AKV_ERR_DOUBLE_FREE (the counts
// before it are applied: the host validated the batch, so this means the
// states differ).
AKV_DEV int dec_ids(Cursors& c, const Agents& g, const int32_t* ids, int32_t n, int32_t& bad_id) {
  int64_t done = 0;  // ops ticked so far
  const int64_t frees0 = c.frees;
  for (int32_t i0 = 0; i0 < n; i0 += 32) {
    const int32_t i = i0 + g.lane;
    int32_t x = i < n ? ids[i] : -1;
    const uint32_t oob = __ballot_sync(kFull, i < n && static_cast<uint32_t>(x) >= static_cast<uint32_t>(g.N));
    if (oob) {
      bad_id = __shfl_sync(kFull, x, __ffs(oob) - 1);
      return AKV_ERR_OUT_OF_RANGE;
    }
    const uint32_t peers = __match_any_sync(kFull, x);
    const bool repeated = __any_sync(kFull, i < n && __popc(peers) > 1);
    if (!repeated) {
      const int32_t old = i < n ? atomicSub(&g.st.ref_counts[x], 1) : 1;
      const uint32_t badm = __ballot_sync(kFull, old < 1);
      if (badm) {
        bad_id = __shfl_sync(kFull, x, __ffs(badm) - 1);
        return AKV_ERR_DOUBLE_FREE;
      }
      uint32_t ret = __ballot_sync(kFull, i < n && old == 1);
      while (ret) {
        const int l = __ffs(ret) - 1;
        ret &= ret - 1;
        const int32_t p = i0 + l;
        ticks(c, g, p - done);
        retire(c, g, __shfl_sync(kFull, x, l));
        ticks(c, g, 1);
        done = p + 1;
      }
    } else {
      const int32_t m = n - i0 < 32 ? n - i0 : 32;
      for (int l = 0; l < m; ++l) {
        const int32_t xl = __shfl_sync(kFull, x, l);
        int32_t old = 0;
        if (g.lane == 0) {
          old = *reinterpret_cast<volatile int32_t*>(&g.st.ref_counts[xl]);
          if (old >= 1) g.st.ref_counts[xl] = old - 1;
        }
        old = __shfl_sync(kFull, old, 0);
        __syncwarp();
        if (old < 1) {
          bad_id = xl;
          return AKV_ERR_DOUBLE_FREE;
        }
        if (old == 1) {
          const int32_t p = i0 + l;
          ticks(c, g, p - done);
          retire(c, g, xl);
          ticks(c, g, 1);
          done = p + 1;
        }
      }
    }
  }
  ticks(c, g, n - done);
  if (g.lane == 0) g.st.ctl[AKV_CTL_LAST_RETIRED] = c.frees - frees0;
  __syncwarp();
  return AKV_OK;
}

// free's dec_ref of every block of the table (n distinct ids, as a handle's
// residual blocks are), in order: a block whose count reaches zero retires
// at its own op.  Validated first: AKV_ERR_DOUBLE_FREE changes nothing.
AKV_DEV int free_table(Cursors& c, const Agents& g, const int32_t* tab, int32_t* len, int32_t& bad_id) {
  const int32_t n = lane0_load(len, g.lane);
  for (int32_t i0 = 0; i0 < n; i0 += 32) {
    const int32_t i = i0 + g.lane;
    int32_t x = -1, r = 1;
    if (i < n) {
      x = vload(&tab[i]);
      r = static_cast<uint32_t>(x) < static_cast<uint32_t>(g.N) ? vload(&g.st.ref_counts[x]) : -1;
    }
    const uint32_t badm = __ballot_sync(kFull, i < n && r <= 0);
    if (badm) {
      bad_id = __shfl_sync(kFull, x, __ffs(badm) - 1);
      return __shfl_sync(kFull, r, __ffs(badm) - 1) < 0 ? AKV_ERR_OUT_OF_RANGE : AKV_ERR_DOUBLE_FREE;
    }
  }
  int64_t done = 0;  // ops ticked so far
  for (int32_t i0 = 0; i0 < n; i0 += 32) {
    const int32_t i = i0 + g.lane;
    const int32_t x = i < n ? vload(&tab[i]) : -1;
    const int32_t old = i < n ? atomicSub(&g.st.ref_counts[x], 1) : 0;
    uint32_t ret = __ballot_sync(kFull, i < n && old == 1);
    while (ret) {
      const int l = __ffs(ret) - 1;
      ret &= ret - 1;
      const int32_t p = i0 + l;
      ticks(c, g, p - done);  // the ops before this one
      retire(c, g, __shfl_sync(kFull, x, l));
      ticks(c, g, 1);
      done = p + 1;
    }
  }
  ticks(c, g, n - done);
  if (g.lane == 0) *len = 0;
  __syncwarp();
  return AKV_OK;
}

enum : int32_t { kActFork = 0, kActCow = 1, kActFree = 2, kActAdvance = 3, kActAppend = 4 };

__global__ void __launch_bounds__(32)
k_agent_steps(Agents g, const int32_t* __restrict__ actions, const int32_t* __restrict__ step_off, int32_t n_steps,
              int32_t* __restrict__ pairs_out, int32_t pairs_cap) {
  g.lane = threadIdx.x;
  if (akv_failed(g.status)) return;
  int64_t* ctl = g.st.ctl;
  Cursors c = load_cursors(g);
  const int64_t stride = 2 + 2 * static_cast<int64_t>(pairs_cap);
  int rc = AKV_OK;
  int32_t fail_at = 0, bad_id = -1, observed = 0;
  for (int32_t s = 0; s < n_steps && rc == AKV_OK; ++s) {
    int32_t* out = pairs_out + s * stride;
    int64_t n_pairs = 0;
    const int32_t a0 = step_off[s], a1 = step_off[s + 1];
    for (int32_t a = a0; a < a1; ++a) {
      const int32_t kind = actions[3 * a], sl = actions[3 * a + 1], tl = actions[3 * a + 2];
      const bool sl_ok = static_cast<uint32_t>(sl) < static_cast<uint32_t>(g.n_agents);
      const bool tl_ok = static_cast<uint32_t>(tl) < static_cast<uint32_t>(g.n_agents);
      int32_t* ts = g.tables + static_cast<int64_t>(sl) * g.cap;
      int32_t* tt = g.tables + static_cast<int64_t>(tl) * g.cap;
      fail_at = a;
      if (kind == kActAdvance) {  // maybe_advance: no tick
        if (advance_allowed(c, g.tk)) {
          ++c.epoch;
          ++c.advances;
        }
        try_retire(c, g);
        continue;
      }
      if (!sl_ok || (kind == kActFork && (!tl_ok || tl == sl)) || kind < 0 || kind > kActAppend) {
        rc = AKV_ERR_INVALID_ARG;
        bad_id = sl;
        observed = kind;
        break;
      }
      if (kind == kActFork) {  // free agent tl, then fork agent sl into slot tl
        rc = free_table(c, g, tt, &g.lens[tl], bad_id);
        if (rc == AKV_OK) rc = fork_into(c, g, ts, lane0_load(&g.lens[sl], g.lane), tt, &g.lens[tl], bad_id);
      } else if (kind == kActFree) {  // free agent sl, restart it as a fork of the root
        rc = free_table(c, g, ts, &g.lens[sl], bad_id);
        if (rc == AKV_OK) rc = fork_into(c, g, g.root, g.root_len, ts, &g.lens[sl], bad_id);
      } else {
        const int32_t n = lane0_load(&g.lens[sl], g.lane);
        if (kind == kActCow && n > 0) {  // ensure_mutable_block(agent, -1)
          const int32_t x = lane0_load(&ts[n - 1], g.lane);
          const int32_t r = static_cast<uint32_t>(x) < static_cast<uint32_t>(g.N) ? lane0_load(&g.st.ref_counts[x], g.lane)
                                                                                    : -1;
          if (r < 1) {
            rc = r < 0 ? AKV_ERR_OUT_OF_RANGE : AKV_ERR_DOUBLE_FREE;
            bad_id = x;
            observed = r;
            break;
          }
          if (r > 1) {  // shared: alloc, copy (the pair), dec_ref
            if (n_pairs >= pairs_cap) {
              rc = AKV_ERR_INVALID_ARG;
              observed = pairs_cap;
              break;
            }
            const int32_t nb = op_alloc(c, g);
            if (nb < 0) {
              rc = AKV_ERR_EXHAUSTED;
              break;
            }
            if (g.lane == 0) {
              out[2 + 2 * n_pairs] = x;
              out[3 + 2 * n_pairs] = nb;
              g.st.ref_counts[x] = r - 1;  // r > 1: no retirement
              ts[n - 1] = nb;
            }
            __syncwarp();
            ++n_pairs;
            ticks(c, g, 1);
          }
        } else {  // allocate_block (append, or a copy-on-write of an empty agent)
          if (n >= g.cap) {
            rc = AKV_ERR_INVALID_ARG;
            bad_id = sl;
            observed = n;
            break;
          }
          const int32_t nb = op_alloc(c, g);
          if (nb < 0) {
            rc = AKV_ERR_EXHAUSTED;
            break;
          }
          if (g.lane == 0) {
            ts[n] = nb;
            g.lens[sl] = n + 1;
          }
          __syncwarp();
        }
      }
      if (rc != AKV_OK) break;
    }
    if (g.lane == 0) reinterpret_cast<int64_t*>(out)[0] = n_pairs;
    __syncwarp();
  }
  if (g.lane == 0) {
    store_cursors(c, ctl);
    if (rc != AKV_OK) akv_fail(g.status, rc, fail_at, bad_id, observed);
  }
}


// ── replay of the host mirror's op log ─────────────────────────────────────
// The per-call operations the host mirror (akv_mirror.cu) answered, applied
// here in order with the same rules; every id the host handed out is checked
// against the one this replay hands out.  Any difference, or an operation
// the device state refuses, is AKV_ERR_MIRROR (the replay stops there).
__global__ void __launch_bounds__(32)
k_alloc_replay(Agents g, const int32_t* __restrict__ log, int64_t n_words) {
  g.lane = threadIdx.x;
  if (akv_failed(g.status)) return;
  Cursors c = load_cursors(g);
  int rc = AKV_OK;
  int32_t bad_id = -1, observed = 0;
  int64_t w = 0;
  while (w < n_words && rc == AKV_OK) {
    rc = AKV_ERR_MIRROR;  // until the record is applied
    if (w + AKV_LOG_HEADER_WORDS > n_words) break;
    const int32_t* h = log + w;
    const int32_t op = h[0], n = h[1];
    if (n < 0 || w + AKV_LOG_HEADER_WORDS + n > n_words) break;
    g.tk.readers_min = (static_cast<int64_t>(h[3]) << 32) | static_cast<uint32_t>(h[2]);
    g.tk.readers_max = (static_cast<int64_t>(h[5]) << 32) | static_cast<uint32_t>(h[4]);
    g.tk.epoch_interval = h[6];
    g.tk.readers_active = h[7];
    const int32_t* p = h + AKV_LOG_HEADER_WORDS;
    bad_id = op;
    if ((op == AKV_OP_ALLOC || op == AKV_OP_INCREF || op == AKV_OP_DECREF || op == AKV_OP_COW ||
         op == AKV_OP_ADVANCE) && g.tk.epoch_interval <= 0)
      break;
    if (op == AKV_OP_ALLOC) {
      int32_t i = 0;
      for (; i < n; ++i) {
        const int32_t want = p[i];
        const int32_t got = op_alloc(c, g);
        if (got != want) {
          bad_id = want;
          observed = got;
          break;
        }
      }
      if (i < n) break;
    } else if (op == AKV_OP_INCREF) {
      int32_t bad = -1;
      if (fork_into(c, g, p, n, nullptr, nullptr, bad) != AKV_OK) {
        bad_id = bad;
        break;
      }
    } else if (op == AKV_OP_DECREF) {
      int32_t bad = -1;
      if (dec_ids(c, g, p, n, bad) != AKV_OK) {
        bad_id = bad;
        break;
      }
    } else if (op == AKV_OP_COW) {
      if (n != 2) break;
      const int32_t x = p[0], want = p[1];
      const int32_t r = static_cast<uint32_t>(x) < static_cast<uint32_t>(g.N) ? lane0_load(&g.st.ref_counts[x], g.lane)
                                                                                : -1;
      if (r < 0 || (r <= 1) != (want == x)) {  // the host's decision must be the device's
        bad_id = x;
        observed = r;
        break;
      }
      if (g.lane == 0) g.st.ctl[AKV_CTL_LAST_COPIED] = want == x ? 0 : 1;
      __syncwarp();
      if (want == x) {
        rc = AKV_OK;
        w += AKV_LOG_HEADER_WORDS + n;
        continue;
      }
      const int32_t got = op_alloc(c, g);
      if (got != want) {
        bad_id = want;
        observed = got;
        break;
      }
      if (g.lane == 0) g.st.ref_counts[x] = r - 1;
      __syncwarp();
      ticks(c, g, 1);
    } else if (op == AKV_OP_RELEASE) {
      try_retire_to(c, g, g.tk.readers_min);
    } else if (op == AKV_OP_ADVANCE) {
      if (advance_allowed(c, g.tk)) {
        ++c.epoch;
        ++c.advances;
      }
      try_retire(c, g);
    } else {
      break;
    }
    rc = AKV_OK;
    w += AKV_LOG_HEADER_WORDS + n;
  }
  if (g.lane == 0) {
    store_cursors(c, g.st.ctl);
    if (rc != AKV_OK) akv_fail(g.status, rc, static_cast<int32_t>(w), bad_id, observed, w);
  }
}

}  // namespace

int akv_agents_prepare() {
  if (int rc = akv_load_kernel(reinterpret_cast<const void*>(k_agent_steps), "akv_prepare: k_agent_steps"))
    return rc;
  return akv_load_kernel(reinterpret_cast<const void*>(k_alloc_replay), "akv_prepare: k_alloc_replay");
}

extern "C" int akv_alloc_replay(const AkvAllocState* st, const int32_t* log, int64_t n_words, AkvStatus* status,
                                void* stream) {
  AKV_ARG_CHECK(st != nullptr && st->ref_counts && st->free_ring && st->limbo_ids && st->limbo_epochs && st->ctl &&
                    st->total_blocks > 0,
                "akv_alloc_replay: incomplete allocator state");
  AKV_ARG_CHECK(status != nullptr, "akv_alloc_replay: status is NULL");
  AKV_ARG_CHECK(n_words >= 0 && (n_words == 0 || log != nullptr), "akv_alloc_replay: bad log");
  if (n_words == 0) return AKV_OK;
  Agents g{};
  g.st = *st;
  g.N = st->total_blocks;
  g.status = status;
  k_alloc_replay<<<1, 32, 0, akv_stream(stream)>>>(g, log, n_words);
  AKV_LAUNCH_CHECK("akv_alloc_replay");
  return AKV_OK;
}

extern "C" int akv_agent_steps(const AkvAllocState* st, const AkvTick* tick, int32_t* tables, int32_t* lens,
                               int32_t n_agents, int32_t capacity, const int32_t* root_table, int32_t root_len,
                               const int32_t* actions, const int32_t* step_off, int32_t n_steps,
                               int32_t* pairs_out, int32_t pairs_cap, AkvStatus* status, void* stream) {
  AKV_ARG_CHECK(st != nullptr && st->ref_counts && st->free_ring && st->limbo_ids && st->limbo_epochs && st->ctl &&
                    st->total_blocks > 0,
                "akv_agent_steps: incomplete allocator state");
  AKV_ARG_CHECK(tick != nullptr && tick->epoch_interval > 0, "akv_agent_steps: bad tick");
  AKV_ARG_CHECK(status != nullptr, "akv_agent_steps: status is NULL");
  AKV_ARG_CHECK(n_agents > 0 && capacity > 0 && root_len >= 0 && root_len <= capacity && n_steps >= 0 &&
                    pairs_cap >= 0,
                "akv_agent_steps: agents=%d capacity=%d root_len=%d steps=%d pairs_cap=%d", n_agents, capacity,
                root_len, n_steps, pairs_cap);
  if (n_steps == 0) return AKV_OK;
  AKV_ARG_CHECK(tables && lens && actions && step_off && pairs_out && (root_len == 0 || root_table),
                "akv_agent_steps: NULL array");
  Agents g;
  g.st = *st;
  g.tk = *tick;
  g.N = st->total_blocks;
  g.tables = tables;
  g.lens = lens;
  g.n_agents = n_agents;
  g.cap = capacity;
  g.root = root_table;
  g.root_len = root_len;
  g.status = status;
  g.lane = 0;
  k_agent_steps<<<1, 32, 0, akv_stream(stream)>>>(g, actions, step_off, n_steps, pairs_out, pairs_cap);
  AKV_LAUNCH_CHECK("akv_agent_steps");
  return AKV_OK;
}
