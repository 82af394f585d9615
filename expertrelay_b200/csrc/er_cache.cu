// er_cache.cu -- HBM expert cache: store records of (layer, expert) in slots
// of one device arena, filled from pinned host memory.
//
// Reference: cache/expert_cache.py:92-402 (CachedExpertSource). Same policy:
// whole slots, LRU eviction of ready slots nobody holds, pinned experts never
// evicted, a load whose copy is in flight is waited for rather than repeated,
// prefetches skipped when no slot is evictable or over the read budget, and
// the SourceStats counters. What changes on the GPU:
//   * a "read" is a cudaMemcpyAsync from pinned host memory on the cache's
//     copy stream, followed by the slot's ready event; nothing blocks the
//     host, and a compute stream that uses the slot waits on the event;
//   * the reference's in-use reference count becomes "held by layer L until
//     end_layer(L)", and end_layer records the slot's last-use event on the
//     compute stream, which the next refill of that slot waits on;
//   * the reference's QUEUED state has no counterpart: a copy handed to the
//     stream is not withdrawn (prefetches_cancelled stays 0).
#include <list>
#include <unordered_map>
#include <vector>

#include "er_internal.cuh"

namespace {

struct Slot {
  uint8_t* dev = nullptr;
  long long key = -1;
  int state = ER_SLOT_FREE;
  int held_layer = -1;      // layer whose forward pass holds it (until end_layer)
  bool pinned = false;
  bool prefetched = false;  // filled by a prefetch and not used since
  bool used_recorded = false;
  long long fill_call = -1;  // the er_cache_prefetch call that filled it
  bool counting = false;     // a prefetch copy not yet seen complete (prefetch_reads)
  cudaEvent_t ready = nullptr;  // recorded on the copy stream after the fill
  cudaEvent_t used = nullptr;   // recorded on the compute stream at end_layer
  bool in_lru = false;
  std::list<int>::iterator lru_it;
};

long long make_key(int layer, int expert) { return ((long long)layer << 32) | (unsigned)expert; }

}  // namespace

struct er_cache {
  bool dry = false;
  bool own_arena = false;
  size_t record_bytes = 0;
  uint8_t* arena = nullptr;
  int min_free_slots = 1;
  std::vector<Slot> slots;
  std::unordered_map<long long, int> map;
  std::list<int> lru;          // unpinned slots holding a key, least recently used first
  std::vector<int> free_list;  // back() is the next free slot
  int layers = 0, experts = 0;
  std::vector<const void*> host;
  cudaStream_t copy = nullptr;
  er_cache_stats stats{};
  long long prefetch_call = 0;  // numbers er_cache_prefetch calls
};

namespace {

using er::cuda_check;
using er::fail;

void touch(er_cache* c, int i) {
  Slot& s = c->slots[i];
  if (s.pinned) return;
  if (s.in_lru) c->lru.erase(s.lru_it);
  s.lru_it = c->lru.insert(c->lru.end(), i);
  s.in_lru = true;
}

void drop(er_cache* c, int i) {  // forget the slot's key
  Slot& s = c->slots[i];
  if (s.key >= 0) {
    auto it = c->map.find(s.key);
    if (it != c->map.end() && it->second == i) c->map.erase(it);
  }
  if (s.in_lru) c->lru.erase(s.lru_it);
  s.in_lru = false;
  s.key = -1;
  s.state = ER_SLOT_FREE;
  s.prefetched = false;
  s.fill_call = -1;
  s.counting = false;
}

// LOADING -> READY once the slot's copy has completed
int poll(er_cache* c, int i) {
  Slot& s = c->slots[i];
  if (s.state != ER_SLOT_LOADING) return ER_OK;
  const cudaError_t q = cudaEventQuery(s.ready);
  if (q == cudaErrorNotReady) return ER_OK;
  if (int rc = cuda_check(q, "er_cache: copy of a record")) return rc;
  s.state = ER_SLOT_READY;
  if (s.counting) c->stats.prefetch_reads += 1;  // used by now or not: the copy completed
  s.counting = false;
  return ER_OK;
}

// A slot to reuse: a free one, else the least recently used ready slot that
// no layer holds (expert_cache.py:172-191), never one filled by the prefetch
// call `call` itself (the reference's queued reads are not evicted by
// prefetches). -1 when there is none.
int victim(er_cache* c, int* out, long long call = -2) {
  *out = -1;
  if (!c->free_list.empty()) {
    *out = c->free_list.back();
    c->free_list.pop_back();
    return ER_OK;
  }
  for (int i : c->lru) {
    if (int rc = poll(c, i)) return rc;
    Slot& s = c->slots[i];
    if (s.state == ER_SLOT_READY && s.held_layer < 0 && !s.pinned && s.fill_call != call) {
      if (s.prefetched) c->stats.prefetches_wasted += 1;
      drop(c, i);
      *out = i;
      return ER_OK;
    }
  }
  return ER_OK;
}

int fill(er_cache* c, int i, int layer, int expert, bool prefetched) {
  if (layer < 0 || layer >= c->layers || expert < 0 || expert >= c->experts)
    return fail(ER_EINVAL, "er_cache: (layer %d, expert %d) outside the source's %d x %d records", layer, expert,
                c->layers, c->experts);
  const void* src = c->host[(size_t)layer * c->experts + expert];
  Slot& s = c->slots[i];
  s.key = make_key(layer, expert);
  c->map[s.key] = i;
  s.prefetched = prefetched;
  touch(c, i);
  if (c->dry) {
    s.state = ER_SLOT_READY;
    if (prefetched) c->stats.prefetch_reads += 1;
    return ER_OK;
  }
  s.state = ER_SLOT_LOADING;
  s.counting = prefetched;
  // kernels still reading the slot's previous record finish first
  if (s.used_recorded)
    if (int rc = cuda_check(cudaStreamWaitEvent(c->copy, s.used, 0), "er_cache: wait for the slot's last use")) return rc;
  if (int rc = cuda_check(cudaMemcpyAsync(s.dev, src, c->record_bytes, cudaMemcpyHostToDevice, c->copy),
                          "er_cache: record copy"))
    return rc;
  return cuda_check(cudaEventRecord(s.ready, c->copy), "er_cache: ready event");
}

}  // namespace

extern "C" int er_cache_create(int slots, size_t record_bytes, int min_free_slots, void* arena, int flags,
                               er_cache** out) {
  if (!out) return fail(ER_EINVAL, "er_cache_create: null out");
  *out = nullptr;
  if (slots < 1 || record_bytes == 0 || record_bytes % 256)
    return fail(ER_EINVAL, "er_cache_create: %d slots of %zu bytes (need >= 1 slot, a multiple of 256 bytes)", slots,
                record_bytes);
  if (min_free_slots < 0 || slots < min_free_slots)
    return fail(ER_ENOSPACE, "er_cache_create: %d slots; need %d free", slots, min_free_slots);
  if ((uintptr_t)arena & 255) return fail(ER_EINVAL, "er_cache_create: arena must be 256-byte aligned");
  er_cache* c = new er_cache();
  c->dry = (flags & ER_CACHE_DRY) != 0;
  c->record_bytes = record_bytes;
  c->min_free_slots = min_free_slots;
  c->slots.resize(slots);
  for (int i = slots - 1; i >= 0; --i) c->free_list.push_back(i);
  auto bail = [&](int rc) {
    er_cache_destroy(c);
    return rc;
  };
  if (!c->dry) {
    if (arena) {
      c->arena = static_cast<uint8_t*>(arena);
    } else {
      void* p = nullptr;
      if (int rc = cuda_check(cudaMalloc(&p, (size_t)slots * record_bytes), "er_cache_create: arena")) return bail(rc);
      c->arena = static_cast<uint8_t*>(p);
      c->own_arena = true;
    }
    if (int rc = cuda_check(cudaStreamCreateWithFlags(&c->copy, cudaStreamNonBlocking), "er_cache_create: copy stream"))
      return bail(rc);
    for (int i = 0; i < slots; ++i) {
      Slot& s = c->slots[i];
      s.dev = c->arena + (size_t)i * record_bytes;
      if (int rc = cuda_check(cudaEventCreateWithFlags(&s.ready, cudaEventDisableTiming), "er_cache_create: event"))
        return bail(rc);
      if (int rc = cuda_check(cudaEventCreateWithFlags(&s.used, cudaEventDisableTiming), "er_cache_create: event"))
        return bail(rc);
    }
  } else {
    c->arena = static_cast<uint8_t*>(arena);
    for (int i = 0; i < slots; ++i) c->slots[i].dev = c->arena ? c->arena + (size_t)i * record_bytes : nullptr;
  }
  *out = c;
  return ER_OK;
}

extern "C" int er_cache_destroy(er_cache* c) {
  if (!c) return ER_OK;
  int rc = ER_OK;
  if (!c->dry) {
    // copies in flight land before their memory and events go away
    if (c->copy) rc = cuda_check(cudaStreamSynchronize(c->copy), "er_cache_destroy: copy stream");
    for (Slot& s : c->slots) {
      if (s.ready) cudaEventDestroy(s.ready);
      if (s.used) cudaEventDestroy(s.used);
    }
    if (c->copy) cudaStreamDestroy(c->copy);
    if (c->own_arena && c->arena) cudaFree(c->arena);
  }
  delete c;
  return rc;
}

extern "C" int er_cache_info(const er_cache* c, void** arena, int* slots, size_t* record_bytes, void** copy_stream) {
  if (!c) return fail(ER_EINVAL, "er_cache_info: null cache");
  if (arena) *arena = c->arena;
  if (slots) *slots = (int)c->slots.size();
  if (record_bytes) *record_bytes = c->record_bytes;
  if (copy_stream) *copy_stream = c->copy;
  return ER_OK;
}

extern "C" int er_cache_set_source(er_cache* c, int layers, int experts, const void* const* host_records) {
  if (!c || !host_records || layers < 1 || experts < 1)
    return fail(ER_EINVAL, "er_cache_set_source: null cache or records, or empty source");
  std::vector<const void*> h(host_records, host_records + (size_t)layers * experts);
  for (const void* p : h)
    if (!p) return fail(ER_EINVAL, "er_cache_set_source: null record address");
  c->host.swap(h);
  c->layers = layers;
  c->experts = experts;
  return ER_OK;
}

extern "C" int er_cache_pin(er_cache* c, int layer, int expert) {
  if (!c) return fail(ER_EINVAL, "er_cache_pin: null cache");
  int pinned = 0;
  for (const Slot& s : c->slots) pinned += s.pinned;
  const long long key = make_key(layer, expert);
  auto it = c->map.find(key);
  if (it != c->map.end() && c->slots[it->second].pinned) return ER_OK;
  if (pinned + 1 + c->min_free_slots > (int)c->slots.size())
    return fail(ER_ENOSPACE, "er_cache_pin: %zu slots hold %d pinned + 1 + %d free", c->slots.size(), pinned,
                c->min_free_slots);
  int i = -1;
  if (it != c->map.end()) {
    i = it->second;
  } else {
    if (int rc = victim(c, &i)) return rc;
    if (i < 0) return fail(ER_ENOSPACE, "er_cache_pin: no evictable slot");
    if (int rc = fill(c, i, layer, expert, false)) return rc;  // like the reference's _pin: not in the stats
  }
  Slot& s = c->slots[i];
  if (s.in_lru) c->lru.erase(s.lru_it);
  s.in_lru = false;
  s.pinned = true;
  return ER_OK;
}

extern "C" int er_cache_acquire(er_cache* c, int layer, const int* experts, int count, void* stream,
                                uint64_t* records_out) {
  if (!c || (count > 0 && (!experts || !records_out)) || count < 0)
    return fail(ER_EINVAL, "er_cache_acquire: null cache or arrays");
  cudaStream_t st = (cudaStream_t)stream;
  for (int j = 0; j < count; ++j) {
    const int e = experts[j];
    const long long key = make_key(layer, e);
    auto it = c->map.find(key);
    int i;
    if (it != c->map.end()) {
      i = it->second;
      Slot& s = c->slots[i];
      if (int rc = poll(c, i)) return rc;
      if (s.held_layer != layer) {  // a repeat within this layer's list is not a second load
        if (s.prefetched) {
          if (s.state == ER_SLOT_READY)
            c->stats.prefetch_hits += 1;
          else
            c->stats.prefetch_waits += 1;  // the stream waits for that copy below
          s.prefetched = false;
        } else {
          c->stats.cache_hits += 1;
        }
        c->stats.loads += 1;
      }
    } else {
      if (int rc = victim(c, &i)) return rc;
      if (i < 0) return fail(ER_ENOSPACE, "er_cache_acquire: no evictable slot for a demand load (cache too small)");
      if (int rc = fill(c, i, layer, e, false)) {
        drop(c, i);
        c->free_list.push_back(i);
        return rc;
      }
      c->stats.demand_reads += 1;
      c->stats.bytes_read += (long long)c->record_bytes;
      c->stats.loads += 1;
    }
    Slot& s = c->slots[i];
    s.held_layer = layer;
    touch(c, i);
    records_out[j] = (uint64_t)(uintptr_t)s.dev;
    if (!c->dry)
      if (int rc = cuda_check(cudaStreamWaitEvent(st, s.ready, 0), "er_cache_acquire: wait for the record")) return rc;
  }
  return ER_OK;
}

extern "C" int er_cache_prefetch(er_cache* c, int layer, const int* experts, int count, const int* keep,
                                 int keep_count, int max_new_reads) {
  if (!c || count < 0 || keep_count < 0 || (count > 0 && !experts) || (keep_count > 0 && !keep))
    return fail(ER_EINVAL, "er_cache_prefetch: null cache or arrays");
  for (int j = 0; j < keep_count; ++j) {
    auto it = c->map.find(make_key(keep[2 * j], keep[2 * j + 1]));
    if (it != c->map.end()) touch(c, it->second);
  }
  int new_reads = 0;
  const long long call = ++c->prefetch_call;
  for (int j = 0; j < count; ++j) {
    const long long key = make_key(layer, experts[j]);
    auto it = c->map.find(key);
    if (it != c->map.end()) {
      touch(c, it->second);
      continue;
    }
    if (max_new_reads >= 0 && new_reads >= max_new_reads) {
      c->stats.prefetches_skipped_budget += 1;
      continue;
    }
    int i = -1;
    if (int rc = victim(c, &i, call)) return rc;
    if (i < 0) {
      c->stats.prefetches_skipped_full += 1;
      continue;
    }
    if (int rc = fill(c, i, layer, experts[j], true)) {
      drop(c, i);
      c->free_list.push_back(i);
      return rc;
    }
    c->slots[i].fill_call = call;
    c->stats.prefetches_issued += 1;
    c->stats.prefetch_bytes += (long long)c->record_bytes;
    new_reads += 1;
  }
  return ER_OK;
}

extern "C" int er_cache_end_layer(er_cache* c, int layer, void* stream) {
  if (!c) return fail(ER_EINVAL, "er_cache_end_layer: null cache");
  for (Slot& s : c->slots) {
    if (s.held_layer != layer) continue;
    s.held_layer = -1;
    if (!c->dry) {
      if (int rc = cuda_check(cudaEventRecord(s.used, (cudaStream_t)stream), "er_cache_end_layer: last-use event"))
        return rc;
      s.used_recorded = true;
    }
  }
  return ER_OK;
}

extern "C" int er_cache_resize(er_cache* c, int slots, void* new_arena, int* slots_out) {
  if (!c) return fail(ER_EINVAL, "er_cache_resize: null cache");
  int pinned = 0;
  for (const Slot& s : c->slots) pinned += s.pinned;
  if (slots < 1 || slots < pinned + c->min_free_slots)
    return fail(ER_ENOSPACE, "er_cache_resize: %d slots; need %d pinned + %d free", slots, pinned, c->min_free_slots);
  const int n = (int)c->slots.size();
  if (!c->dry && !c->own_arena && !new_arena)
    return fail(ER_EINVAL, "er_cache_resize: the arena is the caller's: pass the new one");
  if ((uintptr_t)new_arena & 255) return fail(ER_EINVAL, "er_cache_resize: arena must be 256-byte aligned");
  for (const Slot& s : c->slots)
    if (s.held_layer >= 0) return fail(ER_EINVAL, "er_cache_resize: layer %d still holds slots", s.held_layer);
  // copies in flight land, and kernels using any slot finish, before records move
  if (!c->dry) {
    if (int rc = cuda_check(cudaStreamSynchronize(c->copy), "er_cache_resize: copy stream")) return rc;
    for (Slot& s : c->slots)
      if (s.used_recorded)
        if (int rc = cuda_check(cudaEventSynchronize(s.used), "er_cache_resize: last use")) return rc;
  }
  for (int i = 0; i < n; ++i)
    if (int rc = poll(c, i)) return rc;
  // kept: pinned slots, then the most recently used others (expert_cache.py:322-337)
  std::vector<int> kept;
  for (int i = 0; i < n; ++i)
    if (c->slots[i].pinned) kept.push_back(i);
  std::vector<int> recent(c->lru.rbegin(), c->lru.rend());
  for (int i : recent) {
    if ((int)kept.size() >= slots) {
      if (c->slots[i].prefetched) c->stats.prefetches_wasted += 1;
      continue;
    }
    kept.push_back(i);
  }
  // records move into a new arena, never onto one another
  uint8_t* arena = static_cast<uint8_t*>(new_arena);
  const bool own_new = !new_arena;
  if (!c->dry && !new_arena) {
    void* p = nullptr;
    if (int rc = cuda_check(cudaMalloc(&p, (size_t)slots * c->record_bytes), "er_cache_resize: arena")) return rc;
    arena = static_cast<uint8_t*>(p);
  }
  std::vector<Slot> next(slots);
  std::unordered_map<long long, int> map;
  for (int j = 0; j < (int)kept.size(); ++j) {
    const Slot& o = c->slots[kept[j]];
    Slot& s = next[j];
    s.key = o.key;
    s.state = ER_SLOT_READY;
    s.pinned = o.pinned;
    s.prefetched = o.prefetched;
    map[s.key] = j;
  }
  if (!c->dry) {
    for (int j = 0; j < slots; ++j) {
      Slot& s = next[j];
      s.dev = arena + (size_t)j * c->record_bytes;
      if (int rc = cuda_check(cudaEventCreateWithFlags(&s.ready, cudaEventDisableTiming), "er_cache_resize: event"))
        return rc;
      if (int rc = cuda_check(cudaEventCreateWithFlags(&s.used, cudaEventDisableTiming), "er_cache_resize: event"))
        return rc;
    }
    for (int j = 0; j < (int)kept.size(); ++j)
      if (next[j].dev != c->slots[kept[j]].dev)
        if (int rc = cuda_check(cudaMemcpyAsync(next[j].dev, c->slots[kept[j]].dev, c->record_bytes,
                                                cudaMemcpyDeviceToDevice, c->copy),
                                "er_cache_resize: move a record"))
          return rc;
    if (int rc = cuda_check(cudaStreamSynchronize(c->copy), "er_cache_resize: moves")) return rc;
    for (Slot& s : c->slots) {
      cudaEventDestroy(s.ready);
      cudaEventDestroy(s.used);
    }
    if (c->own_arena) cudaFree(c->arena);
  } else {
    for (int j = 0; j < slots; ++j) next[j].dev = arena ? arena + (size_t)j * c->record_bytes : nullptr;
  }
  c->arena = arena;
  c->own_arena = !c->dry && own_new;
  c->slots.swap(next);
  c->map.swap(map);
  c->lru.clear();
  for (Slot& s : c->slots) s.in_lru = false;
  // least recently used first, as before the move
  for (int j = (int)kept.size() - 1; j >= 0; --j)
    if (!c->slots[j].pinned) touch(c, j);
  c->free_list.clear();
  for (int j = slots - 1; j >= (int)kept.size(); --j) c->free_list.push_back(j);
  if (slots_out) *slots_out = slots;
  return ER_OK;
}

extern "C" int er_cache_lookup(er_cache* c, int layer, int expert, int* slot, int* state) {
  if (!c) return fail(ER_EINVAL, "er_cache_lookup: null cache");
  auto it = c->map.find(make_key(layer, expert));
  if (it == c->map.end()) {
    if (slot) *slot = -1;
    if (state) *state = ER_SLOT_FREE;
    return ER_OK;
  }
  if (int rc = poll(c, it->second)) return rc;
  if (slot) *slot = it->second;
  if (state) *state = c->slots[it->second].state;
  return ER_OK;
}

extern "C" int er_cache_stats_get(er_cache* c, er_cache_stats* out) {
  if (!c || !out) return fail(ER_EINVAL, "er_cache_stats_get: null argument");
  for (int i = 0; i < (int)c->slots.size(); ++i)
    if (int rc = poll(c, i)) return rc;
  *out = c->stats;
  return ER_OK;
}
