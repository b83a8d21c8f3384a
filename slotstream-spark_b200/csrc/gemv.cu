// Dense GEMV of the reference's gemv() API (slotstream_spark/kernels/gemv_affine.py:214-262): MLX affine
// 4/8-bit (gs 32/64) and bf16 dense weights, fp32 accumulation, fp32 output.
//
// Each warp owns one weight row. The row is walked in chunks of 32*NU units (16 elements each); a chunk is
// loaded into registers once and applied to every activation row, and chunk partials are added to
// out[r, row] in chunk order by the same lane. One output is therefore the same op sequence whatever the
// number of activation rows (the reference's row invariance, tests/t0/test_affine_kernels.py:43-75). With
// k <= 32*NU*16 (every shape of the MoE path) there is one chunk and the weights are loaded before the grid
// waits on its producer. No split-K and no workspace.
#include "affine.cuh"
#include "registry.h"

namespace {

constexpr int GV_WARPS = 8;

SSB_DEV void load_x_unit(const void* x, int x_f32, int64_t r, int64_t k, int u, float* x16) {
  if (x_f32) {
    const float4* p = reinterpret_cast<const float4*>((const float*)x + r * k + (int64_t)u * 16);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float4 v = __ldg(p + q);
      x16[4 * q] = v.x;
      x16[4 * q + 1] = v.y;
      x16[4 * q + 2] = v.z;
      x16[4 * q + 3] = v.w;
    }
  } else {
    const uint4* p = reinterpret_cast<const uint4*>((const uint16_t*)x + r * k + (int64_t)u * 16);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      uint4 v = __ldg(p + q);
      x16[8 * q + 0] = bf16_lo(v.x);
      x16[8 * q + 1] = bf16_hi(v.x);
      x16[8 * q + 2] = bf16_lo(v.y);
      x16[8 * q + 3] = bf16_hi(v.y);
      x16[8 * q + 4] = bf16_lo(v.z);
      x16[8 * q + 5] = bf16_hi(v.z);
      x16[8 * q + 6] = bf16_lo(v.w);
      x16[8 * q + 7] = bf16_hi(v.w);
    }
  }
}

// 8-bit codes: sum_j q_j x_j over the four bytes of w, exact products (bytes 2,3 come from w >> 16).
SSB_DEV float dot_word8(uint32_t w, const float* x4) {
  const uint32_t M = 0x4B000000u;
  const uint32_t w2 = w >> 16;
  float2 a = make_float2(__uint_as_float((w & 0xFFu) | M), __uint_as_float((w & 0xFF00u) | M));
  float2 c = make_float2(__uint_as_float((w2 & 0xFFu) | M), __uint_as_float((w2 & 0xFF00u) | M));
  const float2 m = make_float2(-8388608.f, -8388608.f);
  a = __fadd2_rn(a, m);
  c = __fadd2_rn(c, m);
  float2 acc = __fmul2_rn(a, make_float2(x4[0], x4[1] * 0.00390625f));
  acc = __ffma2_rn(c, make_float2(x4[2], x4[3] * 0.00390625f), acc);
  return acc.x + acc.y;
}

template <int NU, int BITS>
__global__ void __launch_bounds__(GV_WARPS * 32) k_gemv_affine(const void* __restrict__ x, int x_f32, int64_t R,
                                                              const uint32_t* __restrict__ q,
                                                              const uint16_t* __restrict__ s,
                                                              const uint16_t* __restrict__ b, int n, int k, int gs,
                                                              float* __restrict__ out) {
  constexpr int WPU = BITS == 4 ? 2 : 4;  // words per 16-element unit
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * GV_WARPS + (threadIdx.x >> 5);
  const int nunits = k / 16, ng = k / gs;
  const int64_t wpr = (int64_t)k * BITS / 32;  // words per row
  bool waited = false;
  for (int c0 = 0; c0 < nunits; c0 += 32 * NU) {
    uint32_t wv[NU][WPU];
    float sv[NU], bv[NU];
    if (row < n) {
#pragma unroll
      for (int i = 0; i < NU; ++i) {
        int u = c0 + lane + 32 * i;
        if (u < nunits) {
          const uint32_t* src = q + row * wpr + (int64_t)u * WPU;
          if constexpr (BITS == 4) {
            uint2 v = ld_stream_u2(src);
            wv[i][0] = v.x;
            wv[i][1] = v.y;
          } else {
            uint4 v = ld_stream_u4(src);
            wv[i][0] = v.x;
            wv[i][1] = v.y;
            wv[i][2] = v.z;
            wv[i][3] = v.w;
          }
          int g = (u * 16) / gs;
          sv[i] = bf16_bits(s[row * ng + g]);
          bv[i] = bf16_bits(b[row * ng + g]);
        }
      }
    }
    if (!waited) {
      pdl_wait();
      pdl_trigger();
      waited = true;
    }
    if (row >= n) return;
    for (int64_t r = 0; r < R; ++r) {
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < NU; ++i) {
        int u = c0 + lane + 32 * i;
        if (u < nunits) {
          float x16[16];
          load_x_unit(x, x_f32, r, k, u, x16);
          if constexpr (BITS == 4) {
            XUnit xu;
            xunit_from_f32(xu, x16);
            acc = unit_dot(make_uint2(wv[i][0], wv[i][1]), sv[i], bv[i], xu, acc);
          } else {
            float xs = 0.f;
#pragma unroll
            for (int j = 0; j < 16; ++j) xs += x16[j];
            float qx = 0.f;
#pragma unroll
            for (int w = 0; w < WPU; ++w) qx += dot_word8(wv[i][w], x16 + 4 * w);
            acc = fmaf(sv[i], qx, fmaf(bv[i], xs, acc));
          }
        }
      }
      acc = warp_sum(acc);
      if (lane == 0) out[r * n + row] = (c0 == 0) ? acc : out[r * n + row] + acc;
    }
  }
}

// dense bf16: unit = 16 elements = 32 bytes
template <int NU>
__global__ void __launch_bounds__(GV_WARPS * 32) k_gemv_dense(const void* __restrict__ x, int x_f32, int64_t R,
                                                             const uint16_t* __restrict__ w, int n, int k,
                                                             float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * GV_WARPS + (threadIdx.x >> 5);
  const int nunits = k / 16;
  bool waited = false;
  for (int c0 = 0; c0 < nunits; c0 += 32 * NU) {
    uint4 wv[NU][2];
    if (row < n) {
#pragma unroll
      for (int i = 0; i < NU; ++i) {
        int u = c0 + lane + 32 * i;
        if (u < nunits) {
          wv[i][0] = ld_stream_u4(w + row * k + (int64_t)u * 16);
          wv[i][1] = ld_stream_u4(w + row * k + (int64_t)u * 16 + 8);
        }
      }
    }
    if (!waited) {
      pdl_wait();
      pdl_trigger();
      waited = true;
    }
    if (row >= n) return;
    for (int64_t r = 0; r < R; ++r) {
      float2 acc = make_float2(0.f, 0.f);
#pragma unroll
      for (int i = 0; i < NU; ++i) {
        int u = c0 + lane + 32 * i;
        if (u < nunits) {
          float x16[16];
          load_x_unit(x, x_f32, r, k, u, x16);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t ww[4] = {wv[i][h].x, wv[i][h].y, wv[i][h].z, wv[i][h].w};
#pragma unroll
            for (int c = 0; c < 4; ++c)
              acc = __ffma2_rn(make_float2(bf16_lo(ww[c]), bf16_hi(ww[c])),
                               make_float2(x16[8 * h + 2 * c], x16[8 * h + 2 * c + 1]), acc);
          }
        }
      }
      float a = warp_sum(acc.x + acc.y);
      if (lane == 0) out[r * n + row] = (c0 == 0) ? a : out[r * n + row] + a;
    }
  }
}

}  // namespace

extern "C" int ssb_gemv_affine(const void* x, int32_t x_dtype, int64_t rows, const int32_t* q, const uint16_t* s,
                               const uint16_t* b, int32_t n, int32_t k, int32_t bits, int32_t gs, float* out,
                               void* stream) {
  SSB_CHECK_ARG(rows >= 0 && n >= 1 && k >= 1 && (x_dtype == SSB_BF16 || x_dtype == SSB_F32));
  SSB_CHECK_ARG(bits == 4 || bits == 8);
  SSB_CHECK_ARG(gs == 32 || gs == 64);
  if (k % 16 || k % gs) return SSB_EUNSUPPORTED;
  if (rows == 0) return SSB_OK;
  SSB_CHECK_ARG(x && q && s && b && out);
  cudaStream_t st = (cudaStream_t)stream;
  dim3 grid((unsigned)((n + GV_WARPS - 1) / GV_WARPS));
  const uint32_t* qq = (const uint32_t*)q;
  const int xf = x_dtype == SSB_F32;
  if (bits == 4) {
    ssb_note_smem("gemv_affine4", k_gemv_affine<8, 4>, 0);
    return ssb_launch(k_gemv_affine<8, 4>, grid, dim3(GV_WARPS * 32), 0, st, true, x, xf, rows, qq, s, b, n, k, gs,
                      out);
  }
  ssb_note_smem("gemv_affine8", k_gemv_affine<4, 8>, 0);
  return ssb_launch(k_gemv_affine<4, 8>, grid, dim3(GV_WARPS * 32), 0, st, true, x, xf, rows, qq, s, b, n, k, gs,
                    out);
}

extern "C" int ssb_gemv_dense(const void* x, int32_t x_dtype, int64_t rows, const uint16_t* w, int32_t n, int32_t k,
                              float* out, void* stream) {
  SSB_CHECK_ARG(rows >= 0 && n >= 1 && k >= 1 && (x_dtype == SSB_BF16 || x_dtype == SSB_F32));
  if (k % 16) return SSB_EUNSUPPORTED;
  if (rows == 0) return SSB_OK;
  SSB_CHECK_ARG(x && w && out);
  dim3 grid((unsigned)((n + GV_WARPS - 1) / GV_WARPS));
  ssb_note_smem("gemv_dense", k_gemv_dense<4>, 0);
  return ssb_launch(k_gemv_dense<4>, grid, dim3(GV_WARPS * 32), 0, (cudaStream_t)stream, true, x,
                    (int)(x_dtype == SSB_F32), rows, w, n, k, out);
}
