// Expert-slot cache manager: the host-side bookkeeping of GpuExpertCache and
// the fills it submits to the copy engines.
//
// Replaces the slot bookkeeping of the reference's GpuExpertCache
// (src/specfit/runtime/gpu_expert_cache.py:75-745: acquire :196-266, LRU
// victim :495-518, probability victim :520-541, assign + submit :543-589,
// completion polling :591-609, release :684-718) with a native object the
// Python class drives through the C ABI.  The contract kept is the
// observable one: which slot an expert lands in, generations, the hit /
// join / submission / eviction counters, the last-used sequence, the order
// fills are submitted and published in, and the use-event rules that keep a
// refill behind the kernels still reading a slot.
//
// Data structures (own design):
//   * per expert: a location code (absent / in flight / resident), its slot
//     and the submission number of its fill — O(1) lookups instead of
//     dictionaries;
//   * the unleased slots in an ordered index keyed (occupied, last use,
//     slot id): the LRU victim is its first element, a ready-only probe walks
//     it in order;
//   * outstanding fills in a FIFO (submission order), retired from the front
//     while their ready events have completed;
//   * use guards: per slot at most one (stream, event) pair per consumer
//     stream, events drawn from a recycled pool owned here;
//   * fills: for every miss of one acquire call, the copy stream waits on the
//     victim slot's guards, one cudaMemcpyAsync moves the packed expert from
//     its page-locked source into the slot, and the caller's ready event is
//     recorded right behind it — a wave of misses is one native call, and
//     each expert's consumer waits for its own copy only.
// Ready events belong to the caller (torch.cuda.Event objects the Python
// layer exposes on leases, observer records and snapshots); they are
// recorded and queried here through their handles.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <deque>
#include <mutex>
#include <set>
#include <tuple>
#include <vector>

#include "common.cuh"

namespace sf {
namespace {

constexpr int8_t kAbsent = 0, kInFlight = 1, kResident = 2;

struct Guard {
  uint64_t stream;
  cudaEvent_t event;
};

struct Slot {
  int32_t expert = -1;
  uint32_t generation = 0;
  int32_t leases = 0;
  uint64_t stamp = 0;            // last-used sequence
  cudaEvent_t ready = nullptr;   // event of the slot's latest fill (caller-owned)
  std::vector<Guard> guards;     // use events of released leases
};

struct Fill {
  int32_t expert, slot;
  uint32_t generation;
  int64_t seq;
  cudaEvent_t ready;
};

using IdleKey = std::tuple<int, uint64_t, int32_t>;  // (occupied, stamp, slot)

struct Manager {
  std::mutex mu;
  int32_t nslots = 0, nexperts = 0;
  std::vector<Slot> slot;
  std::vector<int8_t> where;
  std::vector<int32_t> home;
  std::vector<int64_t> fill_seq;
  std::deque<Fill> fills;
  std::set<IdleKey> idle;
  std::vector<cudaEvent_t> spare;  // recycled guard events
  int64_t h2d = 0, hits = 0, joins = 0, evictions = 0;
  uint64_t seq = 0;
  int64_t submission = 0;
  uint64_t version = 0;
  uint8_t* storage = nullptr;
  size_t slot_bytes = 0;
  std::vector<const void*> source;
  cudaStream_t copy_stream = nullptr;

  IdleKey key_of(int32_t s) const { return IdleKey(slot[s].expert >= 0, slot[s].stamp, s); }
  void unindex(int32_t s) { idle.erase(key_of(s)); }
  void index(int32_t s) {
    if (slot[s].leases == 0) idle.insert(key_of(s));
  }
  // Changes a slot's last use, keeping the idle index ordered.
  void touch(int32_t s) {
    const bool indexed = slot[s].leases == 0;
    if (indexed) unindex(s);
    slot[s].stamp = ++seq;
    if (indexed) index(s);
    ++version;
  }
};

// cudaEventQuery as a tri-state: 1 complete, 0 pending, -1 error (recorded).
int event_done(cudaEvent_t ev) {
  if (!ev) return 1;
  const cudaError_t e = cudaEventQuery(ev);
  if (e == cudaSuccess) return 1;
  if (e == cudaErrorNotReady) {
    (void)cudaGetLastError();  // not-ready is not a sticky error; clear it
    return 0;
  }
  set_error(SF_ERR_CUDA, "cudaEventQuery failed: %s", cudaGetErrorString(e));
  return -1;
}

// Publishes every fill at the front of the queue whose copy has completed.
int retire(Manager& m) {
  bool changed = false;
  while (!m.fills.empty()) {
    const Fill f = m.fills.front();
    const int d = event_done(f.ready);
    if (d < 0) return SF_ERR_CUDA;
    if (!d) break;
    m.fills.pop_front();
    const Slot& s = m.slot[f.slot];
    if (s.expert == f.expert && s.generation == f.generation && m.where[f.expert] == kInFlight &&
        m.fill_seq[f.expert] == f.seq)
      m.where[f.expert] = kResident;
    changed = true;
  }
  if (changed) ++m.version;
  return SF_OK;
}

// Drops the completed use guards of every slot (returns their events to the pool).
int retire_guards(Manager& m) {
  bool changed = false;
  for (Slot& s : m.slot) {
    for (size_t i = 0; i < s.guards.size();) {
      const int d = event_done(s.guards[i].event);
      if (d < 0) return SF_ERR_CUDA;
      if (d) {
        m.spare.push_back(s.guards[i].event);
        s.guards[i] = s.guards.back();
        s.guards.pop_back();
        changed = true;
      } else {
        ++i;
      }
    }
  }
  if (changed) ++m.version;
  return SF_OK;
}

// 1 when the slot's fill is done (or it holds a published expert) and no
// guard is pending: a copy into it would not have to wait.  -1 on error.
int writable(Manager& m, int32_t s) {
  const Slot& sl = m.slot[s];
  const bool published = sl.expert >= 0 && m.where[sl.expert] == kResident && m.home[sl.expert] == s;
  if (!published) {
    const int d = event_done(sl.ready);
    if (d <= 0) return d;
  }
  for (const Guard& g : sl.guards) {
    const int d = event_done(g.event);
    if (d <= 0) return d;
  }
  return 1;
}

int pick_lru(Manager& m, bool ready_only, int32_t* out) {
  *out = -1;
  for (const IdleKey& k : m.idle) {
    const int32_t s = std::get<2>(k);
    if (!ready_only) {
      *out = s;
      return SF_OK;
    }
    const int w = writable(m, s);
    if (w < 0) return SF_ERR_CUDA;
    if (w) {
      *out = s;
      return SF_OK;
    }
  }
  return SF_OK;
}

// Lowest-probability replacement: unleased slots ordered (occupied,
// probability of the held expert, last use, slot); stops at the first
// occupied slot whose expert is at least as likely as the incoming one.
int pick_by_probability(Manager& m, const float* prob, int32_t incoming, int32_t* out) {
  *out = -1;
  const float pin = prob[incoming];
  std::vector<std::tuple<int, float, uint64_t, int32_t>> order;
  order.reserve(m.idle.size());
  for (const IdleKey& k : m.idle) {
    const int32_t s = std::get<2>(k);
    const int32_t e = m.slot[s].expert;
    order.emplace_back(e >= 0, e >= 0 ? prob[e] : 0.f, m.slot[s].stamp, s);
  }
  std::sort(order.begin(), order.end());
  for (const auto& o : order) {
    const int32_t s = std::get<3>(o);
    if (m.slot[s].expert >= 0 && std::get<1>(o) >= pin) break;
    const int w = writable(m, s);
    if (w < 0) return SF_ERR_CUDA;
    if (w) {
      *out = s;
      return SF_OK;
    }
  }
  return SF_OK;
}

// Moves `expert` into slot `s` and queues its copy behind the slot's readers.
int assign(Manager& m, int32_t s, int32_t expert, cudaEvent_t ready, int32_t* victim) {
  Slot& sl = m.slot[s];
  const bool indexed = sl.leases == 0;
  if (indexed) m.unindex(s);
  *victim = sl.expert;
  if (sl.expert >= 0) {
    m.where[sl.expert] = kAbsent;
    ++m.evictions;
  }
  ++sl.generation;
  sl.expert = expert;
  for (const Guard& g : sl.guards) {
    SF_CHECK_CUDA(cudaStreamWaitEvent(m.copy_stream, g.event, 0));
    m.spare.push_back(g.event);  // the wait is enqueued; the event may be recorded again
  }
  sl.guards.clear();
  SF_CHECK_CUDA(cudaMemcpyAsync(m.storage + (size_t)s * m.slot_bytes, m.source[expert], m.slot_bytes,
                                cudaMemcpyHostToDevice, m.copy_stream));
  SF_CHECK_CUDA(cudaEventRecord(ready, m.copy_stream));
  sl.ready = ready;
  m.where[expert] = kInFlight;
  m.home[expert] = s;
  m.fill_seq[expert] = m.submission;
  m.fills.push_back(Fill{expert, s, sl.generation, m.submission, ready});
  ++m.submission;
  ++m.h2d;
  if (indexed) m.index(s);
  return SF_OK;
}

void grant_lease(Manager& m, int32_t s, bool defer_touch) {
  Slot& sl = m.slot[s];
  if (sl.leases == 0) m.unindex(s);
  ++sl.leases;
  if (defer_touch) {
    ++m.version;
  } else {
    sl.stamp = ++m.seq;
    ++m.version;
  }
}

int check_lease(Manager& m, int32_t expert, int32_t s, uint32_t generation) {
  SF_CHECK_ARG(s >= 0 && s < m.nslots, "slot %d out of range", s);
  const Slot& sl = m.slot[s];
  if (sl.expert != expert || sl.generation != generation || sl.leases <= 0)
    return set_error(SF_ERR_STATE, "expert lease refers to a reused GPU slot");
  return SF_OK;
}

Manager* as_mgr(void* h) { return static_cast<Manager*>(h); }

}  // namespace
}  // namespace sf

using sf::Manager;

extern "C" int sf_cache_create(int slots, int experts, void* storage, size_t slot_bytes,
                               const void* const* sources, void* copy_stream, void** out) {
  using namespace sf;
  SF_CHECK_ARG(out, "null output handle");
  *out = nullptr;
  SF_CHECK_ARG(slots > 0, "slot_count must be positive");
  SF_CHECK_ARG(experts > 0, "cpu_sources must contain at least one expert");
  SF_CHECK_ARG(storage && sources && slot_bytes > 0, "null storage or sources");
  auto* m = new Manager();
  m->nslots = slots;
  m->nexperts = experts;
  m->slot.resize(slots);
  m->where.assign(experts, kAbsent);
  m->home.assign(experts, -1);
  m->fill_seq.assign(experts, -1);
  m->storage = static_cast<uint8_t*>(storage);
  m->slot_bytes = slot_bytes;
  m->source.assign(sources, sources + experts);
  m->copy_stream = as_stream(copy_stream);
  for (int32_t s = 0; s < slots; ++s) m->index(s);
  *out = m;
  return SF_OK;
}

extern "C" void sf_cache_destroy(void* h) {
  Manager* m = sf::as_mgr(h);
  if (!m) return;
  for (cudaEvent_t e : m->spare) cudaEventDestroy(e);
  for (sf::Slot& s : m->slot)
    for (const sf::Guard& g : s.guards) cudaEventDestroy(g.event);
  delete m;
}

extern "C" int sf_cache_set_copy_stream(void* h, void* stream) {
  Manager* m = sf::as_mgr(h);
  std::lock_guard<std::mutex> lock(m->mu);
  m->copy_stream = sf::as_stream(stream);
  return SF_OK;
}

extern "C" int sf_cache_acquire(void* h, const int32_t* experts, int n, int mode, int defer_touch,
                                const uint64_t* fresh_events, const float* probabilities,
                                SfCacheGrant* grants, int* granted) {
  using namespace sf;
  Manager& m = *as_mgr(h);
  std::lock_guard<std::mutex> lock(m.mu);
  SF_CHECK_ARG(n >= 0 && experts && grants && granted, "invalid acquire arguments");
  SF_CHECK_ARG(mode >= SF_CACHE_ACQUIRE && mode <= SF_CACHE_PROBABILITY, "unknown acquire mode %d", mode);
  SF_CHECK_ARG(mode != SF_CACHE_PROBABILITY || probabilities, "probability mode needs probabilities");
  *granted = 0;
  for (int i = 0; i < n; ++i) {
    SF_CHECK_ARG(experts[i] >= 0 && experts[i] < m.nexperts, "expert index %d out of range", experts[i]);
    grants[i] = SfCacheGrant{SF_GRANT_NONE, -1, 0u, -1, -1, 0};
  }
  for (int i = 0; i < n; ++i) {
    const int32_t e = experts[i];
    if (int rc = retire(m)) return rc;
    SfCacheGrant& g = grants[i];
    if (m.where[e] != kAbsent) {
      const int32_t s = m.home[e];
      if (m.where[e] == kInFlight) {
        g.kind = SF_GRANT_JOIN;
        g.submission = m.fill_seq[e];
        ++m.joins;
      } else {
        g.kind = SF_GRANT_HIT;
        ++m.hits;
      }
      grant_lease(m, s, defer_touch != 0);
      g.slot = s;
      g.generation = m.slot[s].generation;
      g.ready_event = reinterpret_cast<uint64_t>(m.slot[s].ready);
      ++*granted;
      continue;
    }
    if (mode == SF_CACHE_RESIDENT_ONLY) continue;  // not granted
    int32_t s = -1;
    int rc = mode == SF_CACHE_PROBABILITY ? pick_by_probability(m, probabilities, e, &s)
                                          : pick_lru(m, mode == SF_CACHE_NONBLOCKING, &s);
    if (rc) return rc;
    if (s < 0) {
      if (mode == SF_CACHE_ACQUIRE) {
        if (*granted == 0) return set_error(SF_ERR_NO_SLOT, "all GPU expert slots have active leases");
        return SF_OK;  // a partial wave: the caller runs what it holds first
      }
      continue;
    }
    SF_CHECK_ARG(fresh_events && fresh_events[i], "a fill needs a ready event");
    int32_t victim = -1;
    if ((rc = assign(m, s, e, reinterpret_cast<cudaEvent_t>(fresh_events[i]), &victim))) return rc;
    grant_lease(m, s, defer_touch != 0);
    g.kind = SF_GRANT_MISS;
    g.slot = s;
    g.generation = m.slot[s].generation;
    g.victim = victim;
    g.submission = m.fill_seq[e];
    g.ready_event = fresh_events[i];
    ++*granted;
  }
  return SF_OK;
}

extern "C" int sf_cache_touch(void* h, int32_t expert, int32_t slot, uint32_t generation) {
  using namespace sf;
  Manager& m = *as_mgr(h);
  std::lock_guard<std::mutex> lock(m.mu);
  if (int rc = check_lease(m, expert, slot, generation)) return rc;
  m.touch(slot);
  return SF_OK;
}

extern "C" int sf_cache_check(void* h, int32_t expert, int32_t slot, uint32_t generation) {
  using namespace sf;
  Manager& m = *as_mgr(h);
  std::lock_guard<std::mutex> lock(m.mu);
  return check_lease(m, expert, slot, generation);
}

extern "C" int sf_cache_wait(void* h, int32_t expert, int32_t slot, uint32_t generation, void* stream,
                             int touch) {
  using namespace sf;
  Manager& m = *as_mgr(h);
  std::lock_guard<std::mutex> lock(m.mu);
  if (int rc = check_lease(m, expert, slot, generation)) return rc;
  const Slot& sl = m.slot[slot];
  const bool published = m.where[expert] == kResident && m.home[expert] == slot;
  if (!published && sl.ready) SF_CHECK_CUDA(cudaStreamWaitEvent(as_stream(stream), sl.ready, 0));
  if (touch) m.touch(slot);
  return SF_OK;
}

extern "C" int sf_cache_release(void* h, int32_t expert, int32_t slot, uint32_t generation,
                                const uint64_t* streams, int n_streams) {
  using namespace sf;
  Manager& m = *as_mgr(h);
  std::lock_guard<std::mutex> lock(m.mu);
  if (int rc = check_lease(m, expert, slot, generation)) return rc;
  Slot& sl = m.slot[slot];
  for (int i = 0; i < n_streams; ++i) {
    cudaEvent_t ev;
    if (!m.spare.empty()) {
      ev = m.spare.back();
      m.spare.pop_back();
    } else {
      SF_CHECK_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    }
    SF_CHECK_CUDA(cudaEventRecord(ev, reinterpret_cast<cudaStream_t>(streams[i])));
    bool replaced = false;
    for (Guard& g : sl.guards) {
      if (g.stream == streams[i]) {  // a later use on the same stream covers the earlier one
        m.spare.push_back(g.event);
        g.event = ev;
        replaced = true;
        break;
      }
    }
    if (!replaced) sl.guards.push_back(Guard{streams[i], ev});
  }
  --sl.leases;
  sl.stamp = ++m.seq;
  ++m.version;
  if (sl.leases == 0) m.index(slot);
  return SF_OK;
}

extern "C" int sf_cache_state(void* h, int refresh, SfCacheCounters* c, SfCacheSlot* slots,
                              int32_t* where, int32_t* home, int64_t* fill_seq) {
  using namespace sf;
  Manager& m = *as_mgr(h);
  std::lock_guard<std::mutex> lock(m.mu);
  if (refresh & 1)
    if (int rc = retire(m)) return rc;
  if (refresh & 2)
    if (int rc = retire_guards(m)) return rc;
  if (c) {
    c->h2d_submissions = m.h2d;
    c->resident_hits = m.hits;
    c->inflight_joins = m.joins;
    c->evictions = m.evictions;
    int64_t guards = 0;
    for (const Slot& s : m.slot) guards += (int64_t)s.guards.size();
    c->pending_use_guards = guards;
    c->sequence = (int64_t)m.seq;
    c->submission_sequence = m.submission;
    c->state_version = (int64_t)m.version;
    c->outstanding_fills = (int64_t)m.fills.size();
  }
  if (slots) {
    for (int32_t s = 0; s < m.nslots; ++s) {
      const Slot& sl = m.slot[s];
      SfCacheSlot& o = slots[s];
      o.expert = sl.expert;
      o.generation = sl.generation;
      o.leases = sl.leases;
      o.stamp = (int64_t)sl.stamp;
      o.ready_event = reinterpret_cast<uint64_t>(sl.ready);
      int pending = 0;
      for (const Guard& g : sl.guards) {
        const int d = event_done(g.event);
        if (d < 0) return SF_ERR_CUDA;
        pending += !d;
      }
      o.guards = (int32_t)sl.guards.size();
      o.guards_pending = pending;
    }
  }
  if (where)
    for (int32_t e = 0; e < m.nexperts; ++e) where[e] = m.where[e];
  if (home)
    for (int32_t e = 0; e < m.nexperts; ++e) home[e] = m.where[e] == kAbsent ? -1 : m.home[e];
  if (fill_seq)
    for (int32_t e = 0; e < m.nexperts; ++e) fill_seq[e] = m.where[e] == kInFlight ? m.fill_seq[e] : -1;
  return SF_OK;
}

extern "C" int sf_cache_fills(void* h, SfCacheFill* out, int cap, int* n) {
  using namespace sf;
  Manager& m = *as_mgr(h);
  std::lock_guard<std::mutex> lock(m.mu);
  SF_CHECK_ARG(n, "null count");
  *n = (int)m.fills.size();
  if (!out) return SF_OK;
  SF_CHECK_ARG(cap >= *n, "fill buffer holds %d of %d", cap, *n);
  int i = 0;
  for (const Fill& f : m.fills) {
    const int d = event_done(f.ready);
    if (d < 0) return SF_ERR_CUDA;
    out[i++] = SfCacheFill{f.expert, f.slot, f.generation, d, f.seq, reinterpret_cast<uint64_t>(f.ready)};
  }
  return SF_OK;
}

extern "C" int sf_cache_quiescent(void* h, int* quiescent) {
  using namespace sf;
  Manager& m = *as_mgr(h);
  std::lock_guard<std::mutex> lock(m.mu);
  *quiescent = 0;
  for (const Fill& f : m.fills) {
    const int d = event_done(f.ready);
    if (d < 0) return SF_ERR_CUDA;
    if (!d) return SF_OK;
  }
  for (const Slot& s : m.slot)
    for (const Guard& g : s.guards) {
      const int d = event_done(g.event);
      if (d < 0) return SF_ERR_CUDA;
      if (!d) return SF_OK;
    }
  *quiescent = 1;
  return SF_OK;
}

extern "C" int sf_cache_resident_table(void* h, int32_t* table, int* complete) {
  using namespace sf;
  Manager& m = *as_mgr(h);
  std::lock_guard<std::mutex> lock(m.mu);
  *complete = 0;
  if (m.nslots < m.nexperts) return SF_OK;
  if (int rc = retire(m)) return rc;
  for (int32_t e = 0; e < m.nexperts; ++e) {
    if (m.where[e] != kResident) return SF_OK;
    table[e] = m.home[e];
  }
  *complete = 1;
  return SF_OK;
}

extern "C" int sf_cache_add_hits(void* h, int64_t hits) {
  Manager& m = *sf::as_mgr(h);
  std::lock_guard<std::mutex> lock(m.mu);
  m.hits += hits;
  return SF_OK;
}

// Edits used by the reset paths and by callers that invalidate a cache's
// contents in place (every slot emptied, generations advanced, counters
// kept), and by checkpoint restoration.
extern "C" int sf_cache_reset(void* h, int mode) {
  using namespace sf;
  Manager& m = *as_mgr(h);
  std::lock_guard<std::mutex> lock(m.mu);
  SF_CHECK_ARG(mode == SF_CACHE_RESET_COLD || mode == SF_CACHE_RESET_DISCARD, "unknown reset mode");
  m.idle.clear();
  m.fills.clear();
  for (int32_t e = 0; e < m.nexperts; ++e) {
    m.where[e] = kAbsent;
    m.home[e] = -1;
    m.fill_seq[e] = -1;
  }
  for (int32_t s = 0; s < m.nslots; ++s) {
    Slot& sl = m.slot[s];
    for (const Guard& g : sl.guards) m.spare.push_back(g.event);
    sl.guards.clear();
    sl.expert = -1;
    sl.ready = nullptr;
    sl.stamp = 0;
    if (mode == SF_CACHE_RESET_COLD) {
      sl.generation = 0;
      sl.leases = 0;
    } else {
      ++sl.generation;
    }
  }
  for (int32_t s = 0; s < m.nslots; ++s) m.index(s);
  if (mode == SF_CACHE_RESET_COLD) {
    m.h2d = m.hits = m.joins = m.evictions = 0;
    m.seq = 0;
    m.submission = 0;
    m.version = 0;
  } else {
    ++m.version;
  }
  return SF_OK;
}

// Field edits of one slot, for in-place invalidation by callers outside the
// cache (e.g. emptying a slot's expert, advancing its generation, clearing
// its last use, forgetting its ready event or its use guards).
extern "C" int sf_cache_slot_edit(void* h, int32_t slot, int field, int64_t value) {
  using namespace sf;
  Manager& m = *as_mgr(h);
  std::lock_guard<std::mutex> lock(m.mu);
  SF_CHECK_ARG(slot >= 0 && slot < m.nslots, "slot %d out of range", slot);
  Slot& sl = m.slot[slot];
  const bool indexed = sl.leases == 0;
  if (indexed) m.unindex(slot);
  switch (field) {
    case SF_SLOT_EXPERT:
      SF_CHECK_ARG(value == -1, "a slot's expert can only be cleared");
      if (sl.expert >= 0 && m.home[sl.expert] == slot) {
        m.where[sl.expert] = kAbsent;
        m.home[sl.expert] = -1;
      }
      sl.expert = -1;
      break;
    case SF_SLOT_GENERATION: sl.generation = (uint32_t)value; break;
    case SF_SLOT_STAMP: sl.stamp = (uint64_t)value; break;
    case SF_SLOT_READY:
      SF_CHECK_ARG(value == 0, "a slot's ready event can only be cleared");
      sl.ready = nullptr;
      break;
    case SF_SLOT_GUARDS:
      SF_CHECK_ARG(value == 0, "a slot's use guards can only be cleared");
      for (const Guard& g : sl.guards) m.spare.push_back(g.event);
      sl.guards.clear();
      break;
    default:
      if (indexed) m.index(slot);
      return set_error(SF_ERR_INVALID_ARGUMENT, "unknown slot field %d", field);
  }
  if (indexed) m.index(slot);
  ++m.version;
  return SF_OK;
}

// Clears the expert-location index (`which` = 1 resident, 2 in flight, 4 the
// fill queue) without touching the slots: the in-place edits callers make
// next to the slot edits above.
extern "C" int sf_cache_forget(void* h, int which) {
  using namespace sf;
  Manager& m = *as_mgr(h);
  std::lock_guard<std::mutex> lock(m.mu);
  for (int32_t e = 0; e < m.nexperts; ++e) {
    const bool drop = (m.where[e] == kResident && (which & 1)) || (m.where[e] == kInFlight && (which & 2));
    if (drop) {
      m.where[e] = kAbsent;
      m.home[e] = -1;
      m.fill_seq[e] = -1;
    }
  }
  if (which & 4) m.fills.clear();
  ++m.version;
  return SF_OK;
}

extern "C" int sf_cache_set_version(void* h, int64_t version) {
  Manager& m = *sf::as_mgr(h);
  std::lock_guard<std::mutex> lock(m.mu);
  m.version = (uint64_t)version;
  return SF_OK;
}

// Checkpoint of the bookkeeping (not the weights): a flat image the caller
// keeps and hands back to sf_cache_import on the same cache.  Use guards are
// not part of it (a checkpoint is only taken at a quiescent point).
namespace {
struct ImageHeader {
  int32_t nslots, nexperts;
  int64_t h2d, hits, joins, evictions, submission;
  uint64_t seq, version;
  int64_t nfills;
};
}  // namespace

extern "C" int sf_cache_export(void* h, void* image, size_t capacity, size_t* needed) {
  using namespace sf;
  Manager& m = *as_mgr(h);
  std::lock_guard<std::mutex> lock(m.mu);
  const size_t need = sizeof(ImageHeader) + m.nslots * (sizeof(int32_t) * 2 + sizeof(uint64_t) * 2) +
                      m.nexperts * (1 + sizeof(int32_t) + sizeof(int64_t)) + m.fills.size() * sizeof(Fill);
  *needed = need;
  if (!image) return SF_OK;
  SF_CHECK_ARG(capacity >= need, "checkpoint image needs %zu bytes", need);
  uint8_t* p = static_cast<uint8_t*>(image);
  ImageHeader hd{m.nslots, m.nexperts, m.h2d, m.hits, m.joins, m.evictions, m.submission, m.seq,
                 m.version, (int64_t)m.fills.size()};
  memcpy(p, &hd, sizeof hd);
  p += sizeof hd;
  for (const Slot& s : m.slot) {
    const uint64_t ready = reinterpret_cast<uint64_t>(s.ready);
    memcpy(p, &s.expert, 4); p += 4;
    memcpy(p, &s.generation, 4); p += 4;
    memcpy(p, &s.stamp, 8); p += 8;
    memcpy(p, &ready, 8); p += 8;
  }
  memcpy(p, m.where.data(), m.nexperts); p += m.nexperts;
  memcpy(p, m.home.data(), 4 * m.nexperts); p += 4 * m.nexperts;
  memcpy(p, m.fill_seq.data(), 8 * m.nexperts); p += 8 * m.nexperts;
  for (const Fill& f : m.fills) {
    memcpy(p, &f, sizeof f);
    p += sizeof f;
  }
  return SF_OK;
}

extern "C" int sf_cache_import(void* h, const void* image, size_t size) {
  using namespace sf;
  Manager& m = *as_mgr(h);
  std::lock_guard<std::mutex> lock(m.mu);
  SF_CHECK_ARG(image && size >= sizeof(ImageHeader), "invalid checkpoint image");
  const uint8_t* p = static_cast<const uint8_t*>(image);
  ImageHeader hd;
  memcpy(&hd, p, sizeof hd);
  p += sizeof hd;
  SF_CHECK_ARG(hd.nslots == m.nslots && hd.nexperts == m.nexperts, "checkpoint shape differs");
  for (Slot& s : m.slot) {
    SF_CHECK_ARG(s.leases == 0, "checkpoint boundary cannot contain active leases");
  }
  m.idle.clear();
  for (Slot& s : m.slot) {
    uint64_t ready;
    memcpy(&s.expert, p, 4); p += 4;
    memcpy(&s.generation, p, 4); p += 4;
    memcpy(&s.stamp, p, 8); p += 8;
    memcpy(&ready, p, 8); p += 8;
    s.ready = reinterpret_cast<cudaEvent_t>(ready);
    for (const Guard& g : s.guards) m.spare.push_back(g.event);
    s.guards.clear();
  }
  memcpy(m.where.data(), p, m.nexperts); p += m.nexperts;
  memcpy(m.home.data(), p, 4 * m.nexperts); p += 4 * m.nexperts;
  memcpy(m.fill_seq.data(), p, 8 * m.nexperts); p += 8 * m.nexperts;
  m.fills.clear();
  for (int64_t i = 0; i < hd.nfills; ++i) {
    Fill f;
    memcpy(&f, p, sizeof f);
    p += sizeof f;
    m.fills.push_back(f);
  }
  m.h2d = hd.h2d;
  m.hits = hd.hits;
  m.joins = hd.joins;
  m.evictions = hd.evictions;
  m.submission = hd.submission;
  m.seq = hd.seq;
  m.version = hd.version;
  for (int32_t s = 0; s < m.nslots; ++s) m.index(s);
  return SF_OK;
}

// State hand-over with the device-resident directory (expert_directory.cu):
// export writes the slots, the expert->slot map of published experts, the
// LRU clock and the counters (h2d, hits, joins, evictions); it needs no
// lease and no fill still in flight.  adopt installs such a state back: every
// assigned slot holds a published expert, no fill is outstanding, no guard
// is pending (the caller synchronised the device).
extern "C" int sf_cache_export_slots(void* h, int32_t* slot_expert, int32_t* slot_gen, int64_t* slot_stamp,
                                     int32_t* expert_slot, int64_t* clock, int64_t* counters) {
  using namespace sf;
  Manager& m = *as_mgr(h);
  std::lock_guard<std::mutex> lock(m.mu);
  if (int rc = retire(m)) return rc;
  if (int rc = retire_guards(m)) return rc;
  for (const Slot& s : m.slot)
    if (s.leases) return set_error(SF_ERR_STATE, "device-managed mode cannot start with an active lease");
  for (int32_t e = 0; e < m.nexperts; ++e)
    if (m.where[e] == kInFlight)
      return set_error(SF_ERR_STATE, "device-managed mode needs every expert fill complete");
  for (int32_t s = 0; s < m.nslots; ++s) {
    slot_expert[s] = m.slot[s].expert;
    slot_gen[s] = (int32_t)m.slot[s].generation;
    slot_stamp[s] = (int64_t)m.slot[s].stamp;
  }
  for (int32_t e = 0; e < m.nexperts; ++e) expert_slot[e] = m.where[e] == kResident ? m.home[e] : -1;
  *clock = (int64_t)m.seq;
  counters[0] = m.h2d;
  counters[1] = m.hits;
  counters[2] = m.joins;
  counters[3] = m.evictions;
  return SF_OK;
}

extern "C" int sf_cache_adopt_slots(void* h, const int32_t* slot_expert, const int32_t* slot_gen,
                                    const int64_t* slot_stamp, int64_t clock, const int64_t* counters) {
  using namespace sf;
  Manager& m = *as_mgr(h);
  std::lock_guard<std::mutex> lock(m.mu);
  for (const Slot& s : m.slot)
    if (s.leases) return set_error(SF_ERR_STATE, "cannot adopt a device state while a lease is active");
  for (int32_t s = 0; s < m.nslots; ++s)
    SF_CHECK_ARG(slot_expert[s] >= -1 && slot_expert[s] < m.nexperts, "slot %d holds an unknown expert", s);
  m.idle.clear();
  m.fills.clear();
  for (int32_t e = 0; e < m.nexperts; ++e) {
    m.where[e] = kAbsent;
    m.home[e] = -1;
    m.fill_seq[e] = -1;
  }
  for (int32_t s = 0; s < m.nslots; ++s) {
    Slot& sl = m.slot[s];
    for (const Guard& g : sl.guards) m.spare.push_back(g.event);
    sl.guards.clear();
    sl.expert = slot_expert[s];
    sl.generation = (uint32_t)slot_gen[s];
    sl.stamp = (uint64_t)slot_stamp[s];
    sl.ready = nullptr;
    if (sl.expert >= 0) {
      SF_CHECK_ARG(m.where[sl.expert] == kAbsent, "expert %d is in two slots", sl.expert);
      m.where[sl.expert] = kResident;
      m.home[sl.expert] = s;
    }
  }
  for (int32_t s = 0; s < m.nslots; ++s) m.index(s);
  m.seq = (uint64_t)clock;
  m.h2d = counters[0];
  m.hits = counters[1];
  m.joins = counters[2];
  m.evictions = counters[3];
  ++m.version;
  return SF_OK;
}
