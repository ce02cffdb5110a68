// Expert prefetch session: a per-layer HBM slot cache of expert blobs filled
// from a pinned host store by cudaMemcpyAsync on a session-owned side stream,
// with the expert -> slot tables the layer kernel reads (slot -1 = not
// resident: the layer kernel then reads the blob from the host store itself).
//
// Replaces the reference's payloadless producer session
// (microbench/premap_kernel_consumer/premap_payload_cache_inprocess_native_producer_stub.hip:
// session_create_v1 505, destroy_v1 570, update_v1 800: opaque u64 handle with
// a magic word, int status codes, a result struct with safe defaults) with one
// that moves the bytes, and keeps the bookkeeping of the reference's cache
// managers (runtime/cache_manager.py: ControlledExpertCacheManager 208-279,
// counters of CacheManagerSnapshot 193-205, ready-late misses of
// ReadyTimeExpertCacheManager 298-578), one LRU of slots_per_layer entries per
// layer:
//   issue(layer, e)   resident or in flight -> refresh its LRU position, not
//                     issued; else issued += 1, take a free slot or evict the
//                     least recently used one (evicted_before_use += 1 if it
//                     held a prefetched, never demanded expert), copy.
//   demand(layer, e)  demand += 1; resident and its copy complete -> hit (and
//                     used += 1 the first time a prefetched entry is demanded);
//                     else miss (ready_late += 1 when the copy is still in
//                     flight); with insert_on_miss a missing expert is copied
//                     in as a demand entry (prefetched = false, used = true).
//
// Ordering on the side stream, per copy into slot s of layer l:
//   wait for the compute stream's last use of layer l (mtp_prefetch_layer_used),
//   unpublish the slot's old expert (table entry -> -1), copy the blob,
//   publish the new expert (table entry -> s), record the slot's event.
// A layer kernel reads the table once at its start, so it sees either the old
// state or a published slot whose bytes are complete.
#include "internal.cuh"

#include <cstring>
#include <mutex>
#include <unordered_set>
#include <vector>

namespace mtp {

namespace {

constexpr uint32_t kSessionMagic = 0x4d545046u;  // "MTPF"

__global__ void set_entry_kernel(int32_t* table, int idx, int value) { table[idx] = value; }

struct Slot {
  int expert = -1;
  bool prefetched = false;
  bool used = false;
  bool inflight = false;
  uint64_t tick = 0;
};

struct Layer {
  std::vector<int> slot_of;  // [E] -> slot or -1
  std::vector<Slot> slots;   // [S]
  cudaEvent_t used_event = nullptr;
  bool used_recorded = false;
};

struct Session {
  uint32_t magic = kSessionMagic;
  MtpPrefetchConfig cfg;
  std::vector<Layer> layers;
  std::vector<cudaEvent_t> events;  // [L * S]
  cudaStream_t side = nullptr;
  uint64_t tick = 0;
  MtpPrefetchStats st;
};

// Live sessions: a handle is only dereferenced when it is one of these, so a
// stale or made-up handle returns MTP_ERR_HANDLE instead of faulting.
std::mutex g_sessions_mutex;
std::unordered_set<const void*> g_sessions;

Session* get(uint64_t h) {
  auto* s = reinterpret_cast<Session*>(h);
  {
    std::lock_guard<std::mutex> lock(g_sessions_mutex);
    if (g_sessions.count(s) == 0) return nullptr;
  }
  return s->magic == kSessionMagic ? s : nullptr;
}

bool sim(const Session* s) { return s->cfg.simulate != 0; }

int set_device(const Session* s) {
  if (sim(s)) return MTP_OK;
  return cudaSetDevice(s->cfg.device) == cudaSuccess ? MTP_OK : MTP_ERR_CUDA;
}

// Completed copies become plain residents.
void refresh(Session* s, Layer& L, int slot) {
  Slot& sl = L.slots[slot];
  if (!sl.inflight) return;
  if (sim(s)) {
    sl.inflight = false;
    return;
  }
  const cudaError_t e = cudaEventQuery(s->events[(&L - s->layers.data()) * s->cfg.slots_per_layer + slot]);
  if (e == cudaSuccess) sl.inflight = false;
  else if (e != cudaErrorNotReady) cudaGetLastError();
}

int victim(const Layer& L) {
  int best = -1;
  for (int i = 0; i < static_cast<int>(L.slots.size()); ++i) {
    if (L.slots[i].expert < 0) return i;
    if (best < 0 || L.slots[i].tick < L.slots[best].tick) best = i;
  }
  return best;
}

// Put expert e of layer l into a slot (evicting the LRU one) and start its copy.
int fill(Session* s, int l, int e, bool prefetched) {
  Layer& L = s->layers[l];
  const int v = victim(L);
  if (v < 0) return MTP_ERR_CAPACITY;
  Slot& sl = L.slots[v];
  const int32_t E = s->cfg.num_experts, S = s->cfg.slots_per_layer;
  const int old = sl.expert;
  if (old >= 0) {
    if (sl.prefetched && !sl.used) s->st.evicted_before_use_count += 1;
    L.slot_of[old] = -1;
  }
  sl.expert = e;
  sl.prefetched = prefetched;
  sl.used = !prefetched;
  sl.inflight = true;
  sl.tick = ++s->tick;
  L.slot_of[e] = v;
  s->st.bytes_copied += s->cfg.expert_bytes;
  if (sim(s)) return MTP_OK;
  cudaStream_t st = s->side;
  if (L.used_recorded && cudaStreamWaitEvent(st, L.used_event, 0) != cudaSuccess) return MTP_ERR_CUDA;
  int32_t* table = s->cfg.slot_tables + static_cast<int64_t>(l) * E;
  if (old >= 0) set_entry_kernel<<<1, 1, 0, st>>>(table, old, -1);
  const int64_t eb = s->cfg.expert_bytes;
  // host_layer_stride: 0 = one [experts][bytes] block per layer, -1 = every
  // layer reads the same block, > 0 = that many bytes between layers
  const int64_t hstride = s->cfg.host_layer_stride == 0 ? static_cast<int64_t>(E) * eb
                                                        : (s->cfg.host_layer_stride < 0 ? 0 : s->cfg.host_layer_stride);
  if (cudaMemcpyAsync(s->cfg.cache_base + (static_cast<int64_t>(l) * S + v) * eb,
                      s->cfg.host_store + static_cast<int64_t>(l) * hstride + static_cast<int64_t>(e) * eb,
                      static_cast<size_t>(eb),
                      cudaMemcpyHostToDevice, st) != cudaSuccess)
    return MTP_ERR_CUDA;
  set_entry_kernel<<<1, 1, 0, st>>>(table, e, v);
  if (cudaGetLastError() != cudaSuccess) return MTP_ERR_LAUNCH;
  if (cudaEventRecord(s->events[static_cast<size_t>(l) * S + v], st) != cudaSuccess) return MTP_ERR_CUDA;
  return MTP_OK;
}

void destroy_resources(Session* s) {
  if (sim(s)) return;
  for (cudaEvent_t e : s->events)
    if (e) cudaEventDestroy(e);
  for (Layer& L : s->layers)
    if (L.used_event) cudaEventDestroy(L.used_event);
  if (s->side) cudaStreamDestroy(s->side);
  cudaGetLastError();
}

}  // namespace

}  // namespace mtp

using namespace mtp;

extern "C" {

int mtp_prefetch_session_create(const MtpPrefetchConfig* cfg, uint64_t* out_handle) {
  if (!out_handle) return MTP_ERR_NULL;
  *out_handle = 0;
  if (!cfg) return MTP_ERR_NULL;
  if (cfg->num_layers < 1 || cfg->num_experts < 1 || cfg->slots_per_layer < 1 || cfg->expert_bytes < 1 ||
      cfg->num_layers > 4096 || cfg->num_experts > 4096 || cfg->slots_per_layer > cfg->num_experts)
    return MTP_ERR_SHAPE;
  if (!cfg->simulate && (!cfg->host_store || !cfg->cache_base || !cfg->slot_tables)) return MTP_ERR_NULL;
  if (cfg->host_layer_stride < -1) return MTP_ERR_SHAPE;
  auto* s = new Session();
  s->cfg = *cfg;
  std::memset(&s->st, 0, sizeof(s->st));
  s->layers.resize(cfg->num_layers);
  for (Layer& L : s->layers) {
    L.slot_of.assign(cfg->num_experts, -1);
    L.slots.assign(cfg->slots_per_layer, Slot());
  }
  if (!cfg->simulate) {
    int r = set_device(s);
    const size_t n = static_cast<size_t>(cfg->num_layers) * cfg->slots_per_layer;
    s->events.assign(n, nullptr);
    bool ok = r == MTP_OK && cudaStreamCreateWithFlags(&s->side, cudaStreamNonBlocking) == cudaSuccess;
    for (size_t i = 0; ok && i < n; ++i) ok = cudaEventCreateWithFlags(&s->events[i], cudaEventDisableTiming) == cudaSuccess;
    for (Layer& L : s->layers)
      if (ok) ok = cudaEventCreateWithFlags(&L.used_event, cudaEventDisableTiming) == cudaSuccess;
    // every expert starts not resident
    if (ok) ok = cudaMemsetAsync(cfg->slot_tables, 0xff,
                                 static_cast<size_t>(cfg->num_layers) * cfg->num_experts * sizeof(int32_t),
                                 s->side) == cudaSuccess;
    if (ok) ok = cudaStreamSynchronize(s->side) == cudaSuccess;
    if (!ok) {
      destroy_resources(s);
      s->magic = 0;
      delete s;
      cudaGetLastError();
      return MTP_ERR_CUDA;
    }
  }
  {
    std::lock_guard<std::mutex> lock(g_sessions_mutex);
    g_sessions.insert(s);
  }
  *out_handle = reinterpret_cast<uint64_t>(s);
  return MTP_OK;
}

int mtp_prefetch_session_destroy(uint64_t handle) {
  Session* s = get(handle);
  if (!s) return MTP_ERR_HANDLE;
  if (!sim(s)) {
    set_device(s);
    if (s->side) cudaStreamSynchronize(s->side);
  }
  {
    std::lock_guard<std::mutex> lock(g_sessions_mutex);
    g_sessions.erase(s);
  }
  destroy_resources(s);
  s->magic = 0;
  delete s;
  return MTP_OK;
}

int mtp_prefetch_layer_used(uint64_t handle, int32_t layer, void* compute_stream) {
  Session* s = get(handle);
  if (!s) return MTP_ERR_HANDLE;
  if (layer < 0 || layer >= s->cfg.num_layers) return MTP_ERR_SHAPE;
  if (sim(s)) return MTP_OK;
  if (set_device(s) != MTP_OK) return MTP_ERR_CUDA;
  Layer& L = s->layers[layer];
  if (cudaEventRecord(L.used_event, static_cast<cudaStream_t>(compute_stream)) != cudaSuccess) return MTP_ERR_CUDA;
  L.used_recorded = true;
  return MTP_OK;
}

int mtp_prefetch_issue(uint64_t handle, int32_t layer, const int32_t* experts, int32_t count, int32_t* out_issued) {
  Session* s = get(handle);
  if (!s) return MTP_ERR_HANDLE;
  if (out_issued) *out_issued = 0;
  if (layer < 0 || layer >= s->cfg.num_layers || count < 0) return MTP_ERR_SHAPE;
  if (count > 0 && !experts) return MTP_ERR_NULL;
  if (set_device(s) != MTP_OK) return MTP_ERR_CUDA;
  Layer& L = s->layers[layer];
  int issued = 0;
  for (int i = 0; i < count; ++i) {
    const int e = experts[i];
    if (e < 0 || e >= s->cfg.num_experts) return MTP_ERR_ARG;
    const int slot = L.slot_of[e];
    if (slot >= 0) {  // resident or in flight: refresh its LRU position
      L.slots[slot].tick = ++s->tick;
      continue;
    }
    s->st.issued_fetch_count += 1;
    const int r = fill(s, layer, e, true);
    if (r != MTP_OK) return r;
    ++issued;
  }
  if (out_issued) *out_issued = issued;
  return MTP_OK;
}

int mtp_prefetch_demand(uint64_t handle, int32_t layer, const int32_t* experts, int32_t count, int32_t insert_on_miss,
                        int32_t* out_hits) {
  Session* s = get(handle);
  if (!s) return MTP_ERR_HANDLE;
  if (out_hits) *out_hits = 0;
  if (layer < 0 || layer >= s->cfg.num_layers || count < 0) return MTP_ERR_SHAPE;
  if (count > 0 && !experts) return MTP_ERR_NULL;
  if (set_device(s) != MTP_OK) return MTP_ERR_CUDA;
  Layer& L = s->layers[layer];
  int hits = 0;
  for (int i = 0; i < count; ++i) {
    const int e = experts[i];
    if (e < 0 || e >= s->cfg.num_experts) return MTP_ERR_ARG;
    s->st.demand_count += 1;
    const int slot = L.slot_of[e];
    if (slot >= 0) {
      refresh(s, L, slot);
      Slot& sl = L.slots[slot];
      sl.tick = ++s->tick;
      if (!sl.inflight) {
        s->st.demand_hit_count += 1;
        if (sl.prefetched && !sl.used) s->st.used_fetch_count += 1;
        sl.used = true;
        ++hits;
        continue;
      }
      // still in flight: a ready-late miss; the entry becomes a demand entry
      s->st.demand_miss_count += 1;
      s->st.ready_late_miss_count += 1;
      sl.prefetched = false;
      sl.used = true;
      continue;
    }
    s->st.demand_miss_count += 1;
    if (insert_on_miss) {
      const int r = fill(s, layer, e, false);
      if (r != MTP_OK) return r;
    }
  }
  if (out_hits) *out_hits = hits;
  return MTP_OK;
}

int mtp_prefetch_wait(uint64_t handle, int32_t layer, const int32_t* experts, int32_t count, void* compute_stream) {
  Session* s = get(handle);
  if (!s) return MTP_ERR_HANDLE;
  if (layer < 0 || layer >= s->cfg.num_layers || count < 0) return MTP_ERR_SHAPE;
  if (count > 0 && !experts) return MTP_ERR_NULL;
  if (sim(s)) return MTP_OK;
  if (set_device(s) != MTP_OK) return MTP_ERR_CUDA;
  Layer& L = s->layers[layer];
  const cudaStream_t cs = static_cast<cudaStream_t>(compute_stream);
  for (int i = 0; i < count; ++i) {
    const int e = experts[i];
    if (e < 0 || e >= s->cfg.num_experts) return MTP_ERR_ARG;
    const int slot = L.slot_of[e];
    if (slot < 0) continue;
    refresh(s, L, slot);
    if (!L.slots[slot].inflight) continue;
    if (cudaStreamWaitEvent(cs, s->events[static_cast<size_t>(layer) * s->cfg.slots_per_layer + slot], 0) !=
        cudaSuccess)
      return MTP_ERR_CUDA;
  }
  return MTP_OK;
}

int mtp_prefetch_poll(uint64_t handle, MtpPrefetchStats* out) {
  Session* s = get(handle);
  if (!s) return MTP_ERR_HANDLE;
  if (!out) return MTP_ERR_NULL;
  if (set_device(s) != MTP_OK) return MTP_ERR_CUDA;
  int64_t inflight = 0, resident = 0, unused = 0;
  for (Layer& L : s->layers)
    for (int i = 0; i < static_cast<int>(L.slots.size()); ++i) {
      if (L.slots[i].expert < 0) continue;
      refresh(s, L, i);
      const Slot& sl = L.slots[i];
      if (sl.inflight) ++inflight;
      else ++resident;
      if (sl.prefetched && !sl.used) ++unused;
    }
  *out = s->st;
  out->inflight_count = inflight;
  out->resident_count = resident;
  out->unused_fetch_count = unused;
  return MTP_OK;
}

int mtp_prefetch_sync(uint64_t handle) {
  Session* s = get(handle);
  if (!s) return MTP_ERR_HANDLE;
  if (sim(s)) return MTP_OK;
  if (set_device(s) != MTP_OK) return MTP_ERR_CUDA;
  return cudaStreamSynchronize(s->side) == cudaSuccess ? MTP_OK : MTP_ERR_CUDA;
}

}  // extern "C"
