// Router readback signal of the CUDA-graph decode path (slotstream_spark/kernels/signal.py:15-37) and the host-side
// wait that pairs with it (the acquire spin of runtime/readback.py:40-46).
//
// At the end of a layer's segment one warp copies the layer's chosen expert ids and routing weights into that
// layer's slot of pinned host buffers the GPU writes through its mapping, then publishes seq = base + layer with a
// system-scope release exchange (base = ctrl[1], which the host sets before the step's graphs launch). A host thread
// that observes seq >= base + layer with an acquire load therefore also sees the ids: the engine's host loop can
// ensure the next layer's experts while the graph keeps running, without a stream synchronisation.
#include <atomic>
#include <chrono>
#include <thread>

#include "common.cuh"
#include "registry.h"

namespace {

constexpr int SIGNAL_SLOT = 32;   // elements per layer slot (kernels/signal.py:11)

__global__ void __launch_bounds__(32) k_signal(const int32_t* __restrict__ ids, const float* __restrict__ w, int n,
                                               int32_t* slot_ids, float* slot_w, int64_t* seq,
                                               const int64_t* __restrict__ ctrl, int layer) {
  pdl_wait();
  const int lane = threadIdx.x;
  if (lane < n) {
    slot_ids[(int64_t)layer * SIGNAL_SLOT + lane] = ids[lane];
    slot_w[(int64_t)layer * SIGNAL_SLOT + lane] = w[lane];
  }
  __syncwarp();
  if (lane == 0) {
    const long long base = *reinterpret_cast<const volatile long long*>(ctrl + 1);
    // every lane's slot stores happen before the exchange (warp barrier, then a system-scope fence), and the release
    // exchange orders them before seq for an acquiring reader on the host
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    long long old;
    asm volatile("atom.exch.release.sys.global.b64 %0, [%1], %2;" : "=l"(old) : "l"(seq), "l"(base + layer) : "memory");
    (void)old;
  }
  pdl_trigger();
}

// Byte copy by the SMs: 16-byte pieces when both ends and the size allow, else bytes; grid-stride.
__global__ void __launch_bounds__(256) k_copy_sm(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                                 int64_t bytes, int vec) {
  pdl_wait();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (vec) {
    const int64_t n16 = bytes >> 4;
    for (int64_t i = i0; i < n16; i += stride)
      reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
  } else {
    for (int64_t i = i0; i < bytes; i += stride) dst[i] = src[i];
  }
  pdl_trigger();
}

// L2 prefetch of [p, p + bytes): each lane issues bulk prefetches of 64 KB pieces (16-byte aligned inside).
__global__ void __launch_bounds__(32) k_prefetch_l2(const uint8_t* p, int64_t bytes) {
  const uintptr_t lo = ((uintptr_t)p + 15) & ~(uintptr_t)15;
  const uintptr_t hi = ((uintptr_t)p + (uintptr_t)bytes) & ~(uintptr_t)15;
  if (hi <= lo) return;
  constexpr uintptr_t PIECE = 64 * 1024;
  for (uintptr_t a = lo + (uintptr_t)threadIdx.x * PIECE; a < hi; a += 32 * PIECE) {
    const uint32_t n = (uint32_t)((hi - a) < PIECE ? (hi - a) : PIECE);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"(n) : "memory");
  }
}

}  // namespace

extern "C" int ssb_prefetch_l2(const void* p, int64_t bytes, void* stream) {
  SSB_CHECK_ARG(bytes >= 0);
  if (bytes == 0) return SSB_OK;
  SSB_CHECK_ARG(p);
  ssb_note_smem("prefetch_l2", k_prefetch_l2, 0);
  return ssb_launch(k_prefetch_l2, dim3(1), dim3(32), 0, (cudaStream_t)stream, false, (const uint8_t*)p, bytes);
}

extern "C" int ssb_copy_sm(void* dst, const void* src, int64_t bytes, void* stream) {
  SSB_CHECK_ARG(bytes >= 0 && bytes <= (int64_t(1) << 24));
  if (bytes == 0) return SSB_OK;
  SSB_CHECK_ARG(dst && src);
  const int vec = ((((uintptr_t)dst | (uintptr_t)src | (uintptr_t)bytes) & 15) == 0) ? 1 : 0;
  const int64_t units = vec ? bytes / 16 : bytes;
  const int64_t blocks = (units + 255) / 256;
  ssb_note_smem("copy_sm", k_copy_sm, 0);
  return ssb_launch(k_copy_sm, dim3((unsigned)(blocks < 148 ? blocks : 148)), dim3(256), 0, (cudaStream_t)stream, false,
                    (const uint8_t*)src, (uint8_t*)dst, bytes, vec);
}

extern "C" int ssb_signal(const int32_t* ids, const float* w, int32_t n, int32_t* slot_ids, float* slot_w, int64_t* seq,
                          const int64_t* ctrl, int32_t layer, void* stream) {
  SSB_CHECK_ARG(n >= 0 && n <= SIGNAL_SLOT && layer >= 0 && slot_ids && slot_w && seq && ctrl);
  SSB_CHECK_ARG(n == 0 || (ids && w));
  SSB_CHECK_ARG(((uintptr_t)seq & 7) == 0);
  ssb_note_smem("signal", k_signal, 0);
  return ssb_launch(k_signal, dim3(1), dim3(32), 0, (cudaStream_t)stream, true, ids, w, (int)n, slot_ids, slot_w, seq,
                    ctrl, (int)layer);
}

extern "C" int ssb_wait_seq(const int64_t* seq, int64_t target, int64_t timeout_ns) {
  SSB_CHECK_ARG(seq && timeout_ns >= 0 && ((uintptr_t)seq & 7) == 0);
  const auto* word = reinterpret_cast<const std::atomic<int64_t>*>(seq);
  const auto t0 = std::chrono::steady_clock::now();
  for (uint32_t i = 0;; ++i) {
    if (word->load(std::memory_order_acquire) >= target) return SSB_OK;
    if ((i & 255u) == 255u) {
      if (std::chrono::steady_clock::now() - t0 > std::chrono::nanoseconds(timeout_ns)) return SSB_ETIMEDOUT;
      std::this_thread::yield();
    }
  }
}
