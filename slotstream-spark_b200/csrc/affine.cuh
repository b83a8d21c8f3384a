// Affine 4-bit dot products, bulk-copy staging and expert resolution shared by the decode and GEMV kernels.
//
// Exact nibble decoding without a shift per element: for a 32-bit word w,
//   float((w & (0xF << 4j)) | 0x4B000000) - 2^23 = q_j * 16^j      (exact for j <= 4, q*16^4 < 2^23)
// and nibbles 5..7 come the same way from w >> 12 (q_j * 16^(j-3)). The matching activation is pre-scaled
// by the inverse power of two (exact), so each product q_j * x_j is formed exactly and accumulated in
// fp32, two lanes at a time with the sm_100 packed f32x2 FMA.
#pragma once
#include "common.cuh"

// Per-(16-element unit) activation registers: 8 float2 holding x * {1, 1/16, 1/256, 1/4096, 1/65536,
// 1/256, 1/4096, 1/65536} for each of the unit's two words, plus the unit's plain sum.
struct XUnit {
  float2 v[8];
  float sum;
};

SSB_DEV void xunit_from_f32(XUnit& u, const float* x16) {
  const float sc[8] = {1.f, 0.0625f, 0.00390625f, 0.000244140625f, 1.52587890625e-05f,
                       0.00390625f, 0.000244140625f, 1.52587890625e-05f};
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < 2; ++w) {
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      float a = x16[8 * w + 2 * p], b = x16[8 * w + 2 * p + 1];
      u.v[4 * w + p] = make_float2(a * sc[2 * p], b * sc[2 * p + 1]);
    }
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) s += x16[j];
  u.sum = s;
}

SSB_DEV void xunit_zero(XUnit& u) {
#pragma unroll
  for (int p = 0; p < 8; ++p) u.v[p] = make_float2(0.f, 0.f);
  u.sum = 0.f;
}

// sum_j q_j * x_j over the 8 elements of word w against the pre-scaled pairs xp[0..3]
SSB_DEV float2 dot_word(uint32_t w, const float2* xp, float2 acc) {
  const uint32_t M = 0x4B000000u;
  const uint32_t w5 = w >> 12;
  float2 a = make_float2(__uint_as_float((w & 0xFu) | M), __uint_as_float((w & 0xF0u) | M));
  float2 b = make_float2(__uint_as_float((w & 0xF00u) | M), __uint_as_float((w & 0xF000u) | M));
  float2 c = make_float2(__uint_as_float((w & 0xF0000u) | M), __uint_as_float((w5 & 0xF00u) | M));
  float2 d = make_float2(__uint_as_float((w5 & 0xF000u) | M), __uint_as_float((w5 & 0xF0000u) | M));
  const float2 m = make_float2(-8388608.f, -8388608.f);
  a = __fadd2_rn(a, m);
  b = __fadd2_rn(b, m);
  c = __fadd2_rn(c, m);
  d = __fadd2_rn(d, m);
  acc = __ffma2_rn(a, xp[0], acc);
  acc = __ffma2_rn(b, xp[1], acc);
  acc = __ffma2_rn(c, xp[2], acc);
  acc = __ffma2_rn(d, xp[3], acc);
  return acc;
}

// One unit (two words) of a row: s * sum(q x) + b * sum(x), accumulated into acc.
SSB_DEV float unit_dot(uint2 wv, float s, float b, const XUnit& x, float acc) {
  float2 a2 = dot_word(wv.x, x.v, make_float2(0.f, 0.f));
  a2 = dot_word(wv.y, x.v + 4, a2);
  float qx = a2.x + a2.y;
  return fmaf(s, qx, fmaf(b, x.sum, acc));
}

// The same dot product with the unit's codes decoded once (q_j * 16^j' as float pairs, in dot_word's order), for a
// unit that several activations meet: unit_dot_dec(unit_decode(wv), s, b, x, acc) == unit_dot(wv, s, b, x, acc).
struct WUnit {
  float2 v[8];
};
SSB_DEV WUnit unit_decode(uint2 wv) {
  const uint32_t M = 0x4B000000u;
  const float2 m = make_float2(-8388608.f, -8388608.f);
  WUnit d;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t w = h ? wv.y : wv.x, w5 = w >> 12;
    d.v[4 * h + 0] = __fadd2_rn(make_float2(__uint_as_float((w & 0xFu) | M), __uint_as_float((w & 0xF0u) | M)), m);
    d.v[4 * h + 1] = __fadd2_rn(make_float2(__uint_as_float((w & 0xF00u) | M), __uint_as_float((w & 0xF000u) | M)), m);
    d.v[4 * h + 2] = __fadd2_rn(make_float2(__uint_as_float((w & 0xF0000u) | M), __uint_as_float((w5 & 0xF00u) | M)), m);
    d.v[4 * h + 3] = __fadd2_rn(make_float2(__uint_as_float((w5 & 0xF000u) | M), __uint_as_float((w5 & 0xF0000u) | M)), m);
  }
  return d;
}
SSB_DEV float unit_dot_dec(const WUnit& d, float s, float b, const XUnit& x, float acc) {
  float2 a2 = make_float2(0.f, 0.f);
#pragma unroll
  for (int q = 0; q < 8; ++q) a2 = __ffma2_rn(d.v[q], x.v[q], a2);
  float qx = a2.x + a2.y;
  return fmaf(s, qx, fmaf(b, x.sum, acc));
}

// ---------------------------------------------------------------- mbarrier + bulk copies (async proxy)
SSB_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

SSB_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
SSB_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
SSB_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

SSB_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
SSB_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Returns true when phase `parity` completed; gives up after `limit` polls (each try_wait itself blocks
// for a bounded, hardware-chosen time).
SSB_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t limit) {
  uint32_t a = smem_u32(bar);
  for (uint32_t i = 0; i < limit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(parity), "r"(20000u)
        : "memory");
    if (done) return true;
  }
  return false;
}
// Global -> shared bulk copy, completion counted in bytes on `bar`. dst, src 16-byte aligned; bytes % 16 == 0.
SSB_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Bound on mbarrier polls: far above any real copy time, small enough that a lost arrival ends the kernel
// with an error bit instead of hanging the GPU.
constexpr uint32_t SSB_WAIT_LIMIT = 1u << 16;   // polls of up to 20 us each

// ---------------------------------------------------------------- expert resolution through the slot tables

// slot = map[layer*512 + e], base = slot_ptr[slot]  (slotstream_spark/kernels/moe_gemv_affine.py:66-69)
SSB_DEV const uint8_t* resolve_expert(int e, int layer, const int32_t* map, int64_t map_len, const int64_t* slot_ptr,
                                      int64_t n_slots, int32_t* err) {
  if (e < 0 || e >= 512) {
    set_err(err, SSB_ERR_EXPERT_RANGE);
    return nullptr;
  }
  int64_t mi = (int64_t)layer * 512 + e;
  if (mi < 0 || mi >= map_len) {
    set_err(err, SSB_ERR_UNMAPPED);
    return nullptr;
  }
  int slot = ld_cg_i32(map + mi);
  if (slot < 0) {
    set_err(err, SSB_ERR_UNMAPPED);
    return nullptr;
  }
  if (slot >= n_slots) {
    set_err(err, SSB_ERR_SLOT_RANGE);
    return nullptr;
  }
  long long p = ld_cg_i64(slot_ptr + slot);
  if (p & 15) {
    set_err(err, SSB_ERR_MISALIGNED);
    return nullptr;
  }
  return (const uint8_t*)p;
}

// Byte offsets of the nine record pieces for a (hidden, inter, gs) shape.
struct RecOffs {
  int64_t gw, gsc, gb, uw, usc, ub, dw, dsc, db;
};
static inline RecOffs rec_offsets(int hidden, int inter, int gs) {
  int64_t w = (int64_t)inter * hidden / 2, sb = (int64_t)inter * hidden / gs * 2, p = w + 2 * sb;
  RecOffs o;
  o.gw = 0;
  o.gsc = w;
  o.gb = w + sb;
  o.uw = p;
  o.usc = p + w;
  o.ub = p + w + sb;
  o.dw = 2 * p;
  o.dsc = 2 * p + w;
  o.db = 2 * p + w + sb;
  return o;
}
