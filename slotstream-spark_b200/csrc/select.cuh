// Router selection shared by the router kernels and the fused decode layer: softmax over one token's logits,
// stable top-k on the probabilities and the rank-order sum used to renormalise, all inside one warp.
//
// Selection rule (slotstream_spark/kernels/topk_stable.py:1-13): scores map to order-preserving uint32
// keys (positive: flip the sign bit; negative: bitwise not; NaN: 0, the lowest), larger keys first,
// ties to the lower index. Each candidate becomes the 64-bit composite (key << 32) | ~index, so
// "largest composite first" is exactly that order and every composite is distinct.
#pragma once
#include "common.cuh"

SSB_DEV uint32_t order_key(float f) {
  uint32_t b = __float_as_uint(f);
  if ((b & 0x7FFFFFFFu) > 0x7F800000u) return 0u;  // NaN: lowest
  return (b & 0x80000000u) ? ~b : (b ^ 0x80000000u);
}
SSB_DEV unsigned long long composite(uint32_t key, uint32_t idx) {
  return ((unsigned long long)key << 32) | (unsigned long long)(0xFFFFFFFFu - idx);
}

SSB_DEV void cswap_desc(unsigned long long& a, unsigned long long& b) {
  const unsigned long long hi = a > b ? a : b, lo = a > b ? b : a;
  a = hi;
  b = lo;
}
// Sort 16 composites descending (bitonic network, fully unrolled).
SSB_DEV void bitonic_sort_desc16(unsigned long long* x) {
#pragma unroll
  for (int size = 2; size <= 16; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int j = i ^ stride;
        if (j > i) {
          if ((i & size) == 0) cswap_desc(x[i], x[j]);
          else cswap_desc(x[j], x[i]);
        }
      }
    }
  }
}
// A bitonic sequence of 16 -> descending.
SSB_DEV void bitonic_merge_desc16(unsigned long long* x) {
#pragma unroll
  for (int stride = 8; stride > 0; stride >>= 1) {
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if ((i & stride) == 0) cswap_desc(x[i], x[i + stride]);
  }
}
// The fp32 value whose order key is `key` (inverse of order_key for non-NaN values).
SSB_DEV float key_value(uint32_t key) {
  return __uint_as_float((key & 0x80000000u) ? (key ^ 0x80000000u) : ~key);
}

constexpr int RS_CAND = 64;   // candidate slots per warp

// Shared-memory scratch of one selecting warp.
template <int EPL>
struct SelectScratch {
  float v[32 * EPL];                  // logits, then exponentials, then probabilities
  unsigned long long c[32 * EPL];     // composites
  unsigned long long cand[RS_CAND];
  unsigned long long top[16];
};

// Rarely taken paths (more than RS_CAND candidates, or k > 16), kept out of line so the common path stays
// short: this code runs once per token and per launch, so its size -- not its speed once cached -- is what the
// instruction fetch pays for.
template <int EPL>
__device__ __noinline__ void warp_select_fallback(SelectScratch<EPL>& S, int experts, int k, int lane,
                                                  unsigned long long& mine, float& my_p, float& sum) {
  unsigned long long c[EPL];
  float v[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    c[i] = S.c[lane + 32 * i];
    v[i] = S.v[lane + 32 * i];
  }
  if (EPL <= 16 && k <= 16) {
    // Warp-wide top 16: each lane sorts its composites, then five butterfly steps merge the lanes' sorted
    // lists (top 16 of two sorted lists = bitonic max, then a bitonic merge); every lane ends with the global
    // top 16 in (value desc, index asc) order.
    unsigned long long L[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) L[i] = i < EPL ? c[i < EPL ? i : 0] : 0ull;
    bitonic_sort_desc16(L);
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      unsigned long long o[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) o[i] = __shfl_xor_sync(0xFFFFFFFFu, L[i], off);
#pragma unroll
      for (int i = 0; i < 16; ++i) L[i] = L[i] > o[15 - i] ? L[i] : o[15 - i];
      bitonic_merge_desc16(L);
    }
    sum = 0.f;
    my_p = 0.f;
    mine = 0ull;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float pj = key_value((uint32_t)(L[j] >> 32));
      if (j < k) sum += pj;
      if (j == lane) {
        mine = L[j];
        my_p = pj;
      }
    }
    return;
  }
  // k rounds of warp arg-max; round j's winner is the j-th output (value desc, index asc)
  mine = 0ull;
  my_p = 0.f;
  for (int j = 0; j < k; ++j) {
    unsigned long long lmx = 0ull;
#pragma unroll
    for (int i = 0; i < EPL; ++i) lmx = c[i] > lmx ? c[i] : lmx;
    const unsigned long long g = warp_max_u64(lmx);
    const uint32_t e = 0xFFFFFFFFu - (uint32_t)(g & 0xFFFFFFFFull);
    float p = 0.f;
    if ((int)(e & 31) == lane) {
#pragma unroll
      for (int i = 0; i < EPL; ++i)
        if (lane + 32 * i == (int)e) {
          p = v[i];
          c[i] = 0ull;
        }
    }
    p = __shfl_sync(0xFFFFFFFFu, p, e & 31);
    if (lane == j) {
      mine = g;
      my_p = p;
    }
  }
  sum = 0.f;  // sequential in rank order
  for (int j = 0; j < k; ++j) sum += __shfl_sync(0xFFFFFFFFu, my_p, j);
}

// Candidate filter and renormalisation over a filled scratch (S.c composites, S.v probabilities, expert e at
// index e = lane + 32 i): lane j < k ends with the rank-j composite `mine` and its probability `my_p`, every
// lane with `sum`, the rank-order fp32 sum of the k probabilities. The k-th largest lane maximum T0 bounds the
// k-th largest composite from below (k lanes each hold an element >= T0), so only elements >= T0 can be chosen;
// those candidates (usually a few more than k) are ranked against each other through shared memory.
template <int EPL>
SSB_DEV void warp_select_finish(SelectScratch<EPL>& S, int experts, int k, int lane, unsigned long long& mine,
                                float& my_p, float& sum) {
  if (k <= 16) {
    unsigned long long c[EPL];
    unsigned long long lm = 0ull;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      c[i] = S.c[lane + 32 * i];
      lm = c[i] > lm ? c[i] : lm;
    }
    int rk = 0;
#pragma unroll
    for (int d = 1; d < 32; ++d) {
      const unsigned long long o = __shfl_sync(0xFFFFFFFFu, lm, (lane + d) & 31);
      rk += o > lm;
    }
    const unsigned at = __ballot_sync(0xFFFFFFFFu, rk == k - 1 && lm != 0ull);
    if (at) {
      const unsigned long long T0 = __shfl_sync(0xFFFFFFFFu, lm, __ffs(at) - 1);
      int n = 0;
#pragma unroll
      for (int i = 0; i < EPL; ++i) n += c[i] >= T0;
      int incl = n;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += y;
      }
      const int total = __shfl_sync(0xFFFFFFFFu, incl, 31);
      if (total <= RS_CAND) {
        int pos = incl - n;
#pragma unroll
        for (int i = 0; i < EPL; ++i)
          if (c[i] >= T0) S.cand[pos++] = c[i];
        __syncwarp();
        const unsigned long long a0 = lane < total ? S.cand[lane] : 0ull;
        const unsigned long long a1 = lane + 32 < total ? S.cand[lane + 32] : 0ull;
        int r0 = 0, r1 = 0;
#pragma unroll 4
        for (int q = 0; q < total; ++q) {
          const unsigned long long o = S.cand[q];
          r0 += o > a0;
          r1 += o > a1;
        }
        if (lane < total && r0 < k) S.top[r0] = a0;
        if (lane + 32 < total && r1 < k) S.top[r1] = a1;
        __syncwarp();
        sum = 0.f;   // renormalise: sequential sum in rank order
        my_p = 0.f;
        mine = 0ull;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (j < k) {
            const unsigned long long cj = S.top[j];
            const float pj = key_value((uint32_t)(cj >> 32));
            sum += pj;
            if (j == lane) {
              mine = cj;
              my_p = pj;
            }
          }
        }
        __syncwarp();
        return;
      }
    }
  }
  __syncwarp();
  warp_select_fallback<EPL>(S, experts, k, lane, mine, my_p, sum);
}

// One warp selects for the logits row `lrow` (experts entries; + bias; bf16-rounded first when flags has
// SSB_ROUTER_ROUND_BF16), results as warp_select_finish. probs_row (nullable) gets all probabilities. Lane l
// handles experts l, l + 32, ... in that order in every pass, so every sum has a fixed order.
template <int EPL>
SSB_DEV void warp_select(const float* lrow, int experts, int k, const float* bias, int flags, float* probs_row,
                         SelectScratch<EPL>& S, int lane, unsigned long long& mine, float& my_p, float& sum) {
  float v[EPL];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {   // all loads in flight at once
    const int e = lane + 32 * i;
    float l = -INFINITY;
    if (e < experts) {
      l = __ldcg(lrow + e);
      if (bias) l = l + __ldg(bias + e);
      if (flags & SSB_ROUTER_ROUND_BF16) l = round_bf16(l);
      m = fmaxf(m, l);
    }
    v[i] = l;
  }
  m = warp_max(m);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    const float ex = e < experts ? expf(v[i] - m) : 0.f;
    v[i] = ex;
    s += ex;
  }
  s = warp_sum(s);
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    const float p = v[i] / s;
    S.v[e] = p;
    S.c[e] = (e < experts) ? composite(order_key(p), (uint32_t)e) : 0ull;
    if (probs_row && e < experts) probs_row[e] = p;
  }
  __syncwarp();
  warp_select_finish<EPL>(S, experts, k, lane, mine, my_p, sum);
}
