// HBM expert slot pool for streaming decode (the B200 counterpart of slotio's Pool + Ensurer,
// slotio/include/slotio/pool.hpp:23-160, slotio/src/ensure.cpp).
//
// Records live in fixed-size slots carved out of 1 GiB device chunks. Two device tables let the kernels find
// them: map[layer * experts + e] -> slot (-1: absent) and slot_ptr[slot] -> record address; the decode kernels
// already resolve every expert through them. ensure(layer, experts) makes a layer's experts resident before the
// layer runs: hits are marked referenced, misses take CLOCK victims (never a slot this call needs) and are
// filled by host-to-device copies on a copy stream; one small kernel on the same stream then unpublishes the
// victims' old owners and publishes the new map entries, and the compute stream waits on an event recorded after
// it. Instead of slotio's generation pins, release(layer) records an event on the compute stream after the
// layer's kernels; a copy into a victim slot first makes the copy stream wait on the event of that slot's last
// reader, so a record is never overwritten while a kernel may still read it and the host never blocks for it.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "registry.h"

struct ssb_pool {
  int dev = 0;
  int64_t record_bytes = 0, chunk_bytes = 0;
  int slots_per_chunk = 0, layers = 0, experts = 0, max_slots = 0;
  int slots = 0;
  std::vector<void*> chunks;
  int32_t* map_dev = nullptr;
  int64_t* slot_ptr_dev = nullptr;
  std::vector<int32_t> map_host, owner;
  std::vector<int64_t> slot_ptr_host;
  std::vector<uint8_t> ref;
  int hand = 0;
  // readers: event ring recorded by release(); last_use[slot] = ring index of the slot's last reader (-1: none)
  std::vector<cudaEvent_t> ring;
  int ring_next = 0;
  std::vector<int> last_use;
  std::vector<int32_t> pending;   // slots used since the last release
  cudaEvent_t ready = nullptr;
  std::mutex mu;
  int64_t hits = 0, misses = 0, bytes = 0;
};

namespace {

constexpr int RING = 256;
constexpr int PUB_MAX = 32;

struct PoolUpdates {
  int32_t n;
  int32_t idx[PUB_MAX];
  int32_t val[PUB_MAX];
};

// map[idx[i]] = val[i], in order (an unpublish of a victim's old owner comes before the new owner's publish)
__global__ void k_pool_publish(int32_t* map, PoolUpdates u) {
  if (threadIdx.x == 0)
    for (int i = 0; i < u.n; ++i) map[u.idx[i]] = u.val[i];
}

int publish(ssb_pool* p, const std::vector<std::pair<int32_t, int32_t>>& upd, cudaStream_t st) {
  for (size_t b = 0; b < upd.size(); b += PUB_MAX) {
    PoolUpdates u{};
    u.n = (int32_t)std::min<size_t>(PUB_MAX, upd.size() - b);
    for (int i = 0; i < u.n; ++i) {
      u.idx[i] = upd[b + i].first;
      u.val[i] = upd[b + i].second;
    }
    k_pool_publish<<<1, 32, 0, st>>>(p->map_dev, u);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return (int)e;
  }
  return SSB_OK;
}

}  // namespace

extern "C" ssb_pool* ssb_pool_create(int64_t record_bytes, int64_t chunk_bytes, int32_t layers, int32_t experts,
                                     int32_t max_slots) {
  if (record_bytes <= 0 || record_bytes % 16 || chunk_bytes < record_bytes || layers < 1 || experts < 1 ||
      max_slots < 1)
    return nullptr;
  ssb_pool* p = new ssb_pool();
  cudaGetDevice(&p->dev);
  p->record_bytes = record_bytes;
  p->chunk_bytes = chunk_bytes;
  p->slots_per_chunk = (int)(chunk_bytes / record_bytes);
  p->layers = layers;
  p->experts = experts;
  p->max_slots = max_slots;
  const size_t map_len = (size_t)layers * experts;
  p->map_host.assign(map_len, -1);
  p->owner.assign(max_slots, -1);
  p->slot_ptr_host.assign(max_slots, 0);
  p->ref.assign(max_slots, 0);
  p->last_use.assign(max_slots, -1);
  bool ok = cudaMalloc(&p->map_dev, map_len * 4) == cudaSuccess &&
            cudaMalloc(&p->slot_ptr_dev, (size_t)max_slots * 8) == cudaSuccess &&
            cudaMemset(p->map_dev, 0xFF, map_len * 4) == cudaSuccess &&
            cudaMemset(p->slot_ptr_dev, 0, (size_t)max_slots * 8) == cudaSuccess &&
            cudaEventCreateWithFlags(&p->ready, cudaEventDisableTiming) == cudaSuccess;
  p->ring.assign(RING, nullptr);
  for (int i = 0; ok && i < RING; ++i) ok = cudaEventCreateWithFlags(&p->ring[i], cudaEventDisableTiming) == cudaSuccess;
  if (!ok) {
    (void)cudaGetLastError();
    ssb_pool_destroy(p);
    return nullptr;
  }
  return p;
}

extern "C" void ssb_pool_destroy(ssb_pool* p) {
  if (!p) return;
  cudaDeviceSynchronize();
  for (void* c : p->chunks) cudaFree(c);
  if (p->map_dev) cudaFree(p->map_dev);
  if (p->slot_ptr_dev) cudaFree(p->slot_ptr_dev);
  for (cudaEvent_t e : p->ring)
    if (e) cudaEventDestroy(e);
  if (p->ready) cudaEventDestroy(p->ready);
  delete p;
}

extern "C" int ssb_pool_resize(ssb_pool* p, int32_t n_slots) {
  if (!p || n_slots < 0 || n_slots > p->max_slots) return SSB_EINVAL;
  std::lock_guard<std::mutex> g(p->mu);
  if (n_slots < p->slots) return SSB_EUNSUPPORTED;   // this pool only grows
  const int need = (n_slots + p->slots_per_chunk - 1) / p->slots_per_chunk;
  while ((int)p->chunks.size() < need) {
    void* c = nullptr;
    cudaError_t e = cudaMalloc(&c, (size_t)p->chunk_bytes);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      return (int)e;
    }
    p->chunks.push_back(c);
  }
  for (int s = p->slots; s < n_slots; ++s)
    p->slot_ptr_host[s] = (int64_t)((uint8_t*)p->chunks[s / p->slots_per_chunk] +
                                    (int64_t)(s % p->slots_per_chunk) * p->record_bytes);
  cudaError_t e = cudaMemcpy(p->slot_ptr_dev + p->slots, p->slot_ptr_host.data() + p->slots,
                             (size_t)(n_slots - p->slots) * 8, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return (int)e;
  p->slots = n_slots;
  return SSB_OK;
}

extern "C" int ssb_pool_tables(ssb_pool* p, int32_t** map_dev, int64_t** slot_ptr_dev, int64_t* map_len,
                               int32_t* n_slots, int32_t* chunks) {
  if (!p) return SSB_EINVAL;
  if (map_dev) *map_dev = p->map_dev;
  if (slot_ptr_dev) *slot_ptr_dev = p->slot_ptr_dev;
  if (map_len) *map_len = (int64_t)p->layers * p->experts;
  if (n_slots) *n_slots = p->slots;
  if (chunks) *chunks = (int32_t)p->chunks.size();
  return SSB_OK;
}

extern "C" int ssb_pool_ensure(ssb_pool* p, int32_t layer, const int32_t* experts, int32_t n,
                               const void* const* host_table, void* copy_stream, void* compute_stream,
                               int32_t* out_slots, int64_t* stats) {
  if (!p || !experts || n < 0 || !host_table) return SSB_EINVAL;
  if (layer < 0 || layer >= p->layers) return SSB_EINVAL;
  std::lock_guard<std::mutex> g(p->mu);
  const cudaStream_t cs = (cudaStream_t)copy_stream, ks = (cudaStream_t)compute_stream;
  // (1) validate and dedupe, first-seen order
  std::vector<int32_t> uniq;
  std::unordered_map<int32_t, int32_t> pos;
  for (int i = 0; i < n; ++i) {
    const int32_t e = experts[i];
    if (e < 0 || e >= p->experts) return SSB_EINVAL;
    if (pos.emplace(e, (int32_t)uniq.size()).second) uniq.push_back(e);
  }
  // (2) hits and misses; the slots this call needs may not be victims
  std::vector<int32_t> slot_of(uniq.size(), -1);
  std::vector<uint8_t> needed(p->slots, 0);
  size_t n_miss = 0;
  for (size_t i = 0; i < uniq.size(); ++i) {
    const int32_t s = p->map_host[(size_t)layer * p->experts + uniq[i]];
    if (s >= 0) {
      slot_of[i] = s;
      needed[s] = 1;
      p->ref[s] = 1;
    } else {
      ++n_miss;
    }
  }
  size_t n_hit = uniq.size() - n_miss;
  if (n_miss > (size_t)p->slots - n_hit) return SSB_ETOOBIG;   // no state has changed
  // (3) victims by CLOCK (free slots first, referenced slots get a second chance), copies, map updates
  std::vector<std::pair<int32_t, int32_t>> upd;
  for (size_t i = 0; i < uniq.size(); ++i) {
    if (slot_of[i] >= 0) continue;
    int victim = -1;
    for (long scan = 0; scan < 3L * p->slots && victim < 0; ++scan) {
      const int s = p->hand;
      p->hand = (p->hand + 1) % p->slots;
      if (needed[s]) continue;
      if (p->owner[s] >= 0 && p->ref[s]) {
        p->ref[s] = 0;
        continue;
      }
      victim = s;
    }
    if (victim < 0) return SSB_ETOOBIG;
    const int32_t idx = layer * p->experts + uniq[i];
    if (p->owner[victim] >= 0) {
      upd.emplace_back(p->owner[victim], -1);
      p->map_host[p->owner[victim]] = -1;
    }
    if (p->last_use[victim] >= 0) {   // its last reader must be done before the copy overwrites it
      cudaError_t e = cudaStreamWaitEvent(cs, p->ring[p->last_use[victim]], 0);
      if (e != cudaSuccess) return (int)e;
    }
    const void* src = host_table[idx];
    if (!src) return SSB_EINVAL;
    cudaError_t e = cudaMemcpyAsync((void*)p->slot_ptr_host[victim], src, (size_t)p->record_bytes,
                                    cudaMemcpyHostToDevice, cs);
    if (e != cudaSuccess) return (int)e;
    upd.emplace_back(idx, victim);
    p->map_host[idx] = victim;
    p->owner[victim] = idx;
    p->ref[victim] = 1;
    needed[victim] = 1;
    slot_of[i] = victim;
    p->bytes += p->record_bytes;
  }
  p->hits += (int64_t)n_hit;
  p->misses += (int64_t)n_miss;
  int rc = publish(p, upd, cs);
  if (rc) return rc;
  cudaError_t e = cudaEventRecord(p->ready, cs);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(ks, p->ready, 0);   // ks 0 = the default stream
  if (e != cudaSuccess) return (int)e;
  for (size_t i = 0; i < uniq.size(); ++i) p->pending.push_back(slot_of[i]);
  if (out_slots)
    for (int i = 0; i < n; ++i) out_slots[i] = slot_of[pos[experts[i]]];
  if (stats) {
    stats[0] = (int64_t)n_hit;
    stats[1] = (int64_t)n_miss;
    stats[2] = (int64_t)n_miss * p->record_bytes;
  }
  return SSB_OK;
}

extern "C" int ssb_pool_release(ssb_pool* p, void* compute_stream) {
  if (!p) return SSB_EINVAL;
  std::lock_guard<std::mutex> g(p->mu);
  const int k = p->ring_next;
  p->ring_next = (p->ring_next + 1) % RING;
  cudaError_t e = cudaEventRecord(p->ring[k], (cudaStream_t)compute_stream);
  if (e != cudaSuccess) return (int)e;
  for (int32_t s : p->pending) p->last_use[s] = k;
  p->pending.clear();
  return SSB_OK;
}

extern "C" int ssb_pool_counters(ssb_pool* p, int64_t* hits, int64_t* misses, int64_t* bytes) {
  if (!p) return SSB_EINVAL;
  std::lock_guard<std::mutex> g(p->mu);
  if (hits) *hits = p->hits;
  if (misses) *misses = p->misses;
  if (bytes) *bytes = p->bytes;
  return SSB_OK;
}

// One streaming decode layer with the host side in native code: router logits + select on the compute stream,
// the chosen ids to the host (the only synchronisation), ensure, the expert kernels through the pool's tables,
// release. Every kernel is the one the separate entry points launch, so the results are theirs bit for bit.
extern "C" int ssb_pool_decode_layer(ssb_pool* p, int32_t layer, const uint16_t* x, int64_t rows, int32_t topk,
                                     int32_t hidden, int32_t inter, int32_t experts, const uint16_t* w_router,
                                     const uint16_t* sh_gate_w, const float* bias, const void* const* host_table,
                                     const void* shared_record, float* logits_ws, int32_t* ids, float* w,
                                     float* sh_gate, int32_t* ids_host, float* h_buf, float* o_buf, float* out,
                                     uint16_t* y, int32_t* err, void* copy_stream, void* compute_stream,
                                     int64_t* stats) {
  if (!p || !x || !w_router || !sh_gate_w || !host_table || !logits_ws || !ids || !w || !sh_gate || !ids_host)
    return SSB_EINVAL;
  if (rows < 0 || topk < 1 || experts != p->experts || layer < 0 || layer >= p->layers) return SSB_EINVAL;
  if (rows == 0) return SSB_OK;
  const cudaStream_t ks = (cudaStream_t)compute_stream;
  int rc = ssb_router_logits(x, w_router, sh_gate_w, rows, hidden, experts, experts + 1, logits_ws, compute_stream);
  if (rc) return rc;
  rc = ssb_router_select(logits_ws, experts + 1, rows, experts, topk, bias, SSB_ROUTER_SHARED_GATE, ids, w, nullptr,
                         sh_gate, compute_stream);
  if (rc) return rc;
  cudaError_t e = cudaMemcpyAsync(ids_host, ids, (size_t)rows * topk * 4, cudaMemcpyDeviceToHost, ks);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ks);
  if (e != cudaSuccess) return (int)e;
  rc = ssb_pool_ensure(p, layer, ids_host, (int32_t)(rows * topk), host_table, copy_stream, compute_stream, nullptr,
                       stats);
  if (rc) return rc;
  int32_t* map_dev = nullptr;
  int64_t* slot_ptr_dev = nullptr;
  int64_t map_len = 0;
  int32_t n_slots = 0;
  rc = ssb_pool_tables(p, &map_dev, &slot_ptr_dev, &map_len, &n_slots, nullptr);
  if (rc) return rc;
  rc = ssb_moe_decode_layer(x, ids, w, rows, topk, hidden, inter, layer, map_dev, map_len, slot_ptr_dev, n_slots,
                            shared_record, sh_gate, nullptr, h_buf, o_buf, out, y, 0, err, compute_stream);
  if (rc) return rc;
  return ssb_pool_release(p, compute_stream);
}

extern "C" int ssb_copy_async(void* dst, const void* src, int64_t bytes, void* stream) {
  if (!dst || !src || bytes < 0) return SSB_EINVAL;
  if (bytes == 0) return SSB_OK;
  const cudaError_t e = cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyDefault, (cudaStream_t)stream);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return (int)e;
  }
  return SSB_OK;
}
