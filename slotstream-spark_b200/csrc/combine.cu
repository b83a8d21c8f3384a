// Rank-order combine (slotstream_spark/kernels/fused_moe_affine.py:164-172): out[t] = rows[t*k] + rows[t*k+1]
// + ... sequentially in fp32, bit-equal to the reference's torch loop. The layer variant adds the shared
// expert the way the reference's callers do (model/layers.py:402: routed.to(bf16) + sh) and writes bf16.
#include "common.cuh"
#include "registry.h"

namespace {

__global__ void __launch_bounds__(256) k_combine(const float4* __restrict__ rows, int64_t T, int K, int H4,
                                                 const float4* __restrict__ sh, float4* __restrict__ out,
                                                 uint2* __restrict__ y) {
  pdl_wait();
  pdl_trigger();
  const int64_t n = T * H4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / H4, c = i - t * H4;
    const float4* base = rows + t * K * H4 + c;
    float4 acc = __ldcs(base);
    for (int k = 1; k < K; ++k) {
      float4 v = __ldcs(base + (int64_t)k * H4);
      acc.x = acc.x + v.x;
      acc.y = acc.y + v.y;
      acc.z = acc.z + v.z;
      acc.w = acc.w + v.w;
    }
    if (out) out[i] = acc;
    if (y) {
      float4 s = sh ? sh[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      uint32_t a = f32_to_bf16(round_bf16(acc.x) + round_bf16(s.x));
      uint32_t b = f32_to_bf16(round_bf16(acc.y) + round_bf16(s.y));
      uint32_t c2 = f32_to_bf16(round_bf16(acc.z) + round_bf16(s.z));
      uint32_t d = f32_to_bf16(round_bf16(acc.w) + round_bf16(s.w));
      y[i] = make_uint2(a | (b << 16), c2 | (d << 16));
    }
  }
}

int launch(const float* rows, int64_t tokens, int32_t k, int32_t hidden, const float* sh, float* out, uint16_t* y,
           void* stream) {
  SSB_CHECK_ARG(tokens >= 0 && k >= 1 && hidden >= 1);
  if (hidden % 4) return SSB_EUNSUPPORTED;
  if (tokens == 0) return SSB_OK;
  SSB_CHECK_ARG(rows && (out || y));
  const int64_t n = tokens * (hidden / 4);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int64_t blocks = (n + 255) / 256;
  blocks = blocks < (int64_t)sms * 8 ? blocks : (int64_t)sms * 8;
  ssb_note_smem("combine_rank_order", k_combine, 0);
  return ssb_launch(k_combine, dim3((unsigned)blocks), dim3(256), 0, (cudaStream_t)stream, true,
                    (const float4*)rows, tokens, k, hidden / 4, (const float4*)sh, (float4*)out, (uint2*)y);
}

}  // namespace

extern "C" int ssb_combine_rank_order(const float* rows, int64_t tokens, int32_t k, int32_t hidden, float* out,
                                      void* stream) {
  if (tokens > 0 && !out) return SSB_EINVAL;   // empty tensors may come with null pointers
  return launch(rows, tokens, k, hidden, nullptr, out, nullptr, stream);
}

extern "C" int ssb_combine_layer(const float* rows, int64_t tokens, int32_t k, int32_t hidden, const float* sh,
                                 float* out, uint16_t* y, void* stream) {
  if (tokens > 0 && !y) return SSB_EINVAL;
  return launch(rows, tokens, k, hidden, sh, out, y, stream);
}
