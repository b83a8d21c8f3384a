// Shared device helpers of the sm_100a MoE kernels: bf16 bit tricks, nibble decoding, warp reductions,
// programmatic-dependent-launch (PDL) controls, L2 bulk prefetch and the launch helper.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/slotstream_b200.h"

#define SSB_DEV __device__ __forceinline__

// ---------------------------------------------------------------- bf16 <-> fp32 (bit level, exact)
SSB_DEV float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
SSB_DEV float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
SSB_DEV float bf16_at(const uint16_t* p) { return __uint_as_float(((uint32_t)*p) << 16); }
SSB_DEV float bf16_bits(uint16_t h) { return __uint_as_float(((uint32_t)h) << 16); }

// Round-to-nearest-even fp32 -> bf16 bits (the hardware cvt.rn.bf16.f32).
SSB_DEV uint16_t f32_to_bf16(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }
SSB_DEV float round_bf16(float f) { return __uint_as_float(((uint32_t)f32_to_bf16(f)) << 16); }

// ---------------------------------------------------------------- 4-bit codes
// Element j (0..7) of a little-endian word sits in bits [4j, 4j+4). Returns float(q_j) exactly.
SSB_DEV float nib(uint32_t w, int j) { return (float)((w >> (4 * j)) & 0xFu); }

// Sum over the 8 elements of one word: sum_j q_j * x[j], fp32 FMA in element order.
SSB_DEV float dot8(uint32_t w, const float* x) {
  float a = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) a = fmaf(nib(w, j), x[j], a);
  return a;
}

// ---------------------------------------------------------------- warp helpers
SSB_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}
SSB_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}
SSB_DEV unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long w = __shfl_xor_sync(0xFFFFFFFFu, v, o);
    v = w > v ? w : v;
  }
  return v;
}
SSB_DEV uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// ---------------------------------------------------------------- PDL (griddepcontrol, sm_90+)
// pdl_wait: block until the grids this one depends on have completed and their writes are visible.
// pdl_trigger: allow the next PDL-launched grid in the stream to start its prologue. Every kernel here calls
// pdl_trigger only after pdl_wait, so a grid that starts early can rely on everything two launches back
// being complete. Both are no-ops when the kernel was launched without the PDL attribute.
SSB_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
SSB_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// L2 prefetch of [p, p + bytes): bytes multiple of 16, p 16-byte aligned. Safe before pdl_wait: L2 is the
// GPU's point of coherence, so a later load never sees stale data because of it.
SSB_DEV void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Loads through L2 only (no L1 allocation): for values another grid wrote.
SSB_DEV int ld_cg_i32(const int32_t* p) { return __ldcg(p); }
SSB_DEV long long ld_cg_i64(const int64_t* p) { return __ldcg((const long long*)p); }

// Streaming 8/16-byte loads of weights that are read once (no L1 allocation).
SSB_DEV uint2 ld_stream_u2(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
SSB_DEV uint4 ld_stream_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// ---------------------------------------------------------------- error word
// Device-side problems (an expert id outside [0, 512), a map entry of -1, a slot outside the table) set a
// bit in the caller's error word instead of reading garbage; the affected row's contribution is zero.
SSB_DEV void set_err(int32_t* err, int bit) {
  if (err) atomicOr(err, bit);
}

// ---------------------------------------------------------------- launch helper (host)
// Launches `kern` on `stream`, with programmatic stream serialization when `pdl` is set.
template <typename... KArgs, typename... Args>
static inline int ssb_launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                             bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return (int)e;
  }
  return SSB_OK;
}

#define SSB_CHECK_ARG(cond)      \
  do {                           \
    if (!(cond)) return SSB_EINVAL; \
  } while (0)
