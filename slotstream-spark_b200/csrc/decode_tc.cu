// Fused decode MoE layer for one or two tokens with the expert products on the tensor cores, in ONE cooperative
// launch (one CTA per SM, two grid barriers): router logits, select, expert resolution, gate_up + SwiGLU,
// down + rank-order sum + shared expert.
//
// At batch 1-2 a layer reads ~20-37 MB of 4-bit weights once; the CUDA-core version of this kernel spent ~8
// thread instructions per weight (exact fp32 nibble algebra, one FMA per product) and was bound by instruction
// issue. Here each warp dequantises a 16-row x 64-column weight tile into bf16 registers -- a 4-bit code q becomes
// the exact bf16 value 128 + q with one LOP3 per pair of codes -- and multiplies it with one mma.sync
// m16n8k16 per 16 columns (bf16 x bf16 products are exact, fp32 accumulation). The 128 offset and the affine
// scale/bias of each 64-column group fold in afterwards in fp32:
//   sum_k (q_k s + b) v_k = s * sum_k (128 + q_k) v_k + (b - 128 s) * sum_k v_k        (per group of 64)
// Column n of the mma is token n (gate_up), so the two tokens of an MTP verify share every weight tile, and each
// distinct routed expert of the call is read once. The down projection keeps h in fp32 as the reference's
// decode does (kernels/moe_gemv_affine.py:76-97): h = hi + lo with hi = bf16(h), lo = bf16(h - hi), the two
// halves in adjacent mma columns, so the products are those of h to 2^-17.
//
//  phase 1  x into smem (raw and in the mma K order), router logits (a warp per weight row, the summation order of
//           k_router_logits), expert resolution, and -- independent of routing -- the shared expert's gate/up
//           units (8 gate + 8 up rows each) on the CTAs that own one;
//  barrier
//  phase 2  select per token (the CTA-wide passes of the CUDA-core kernel, bit-identical to ssb_router_select),
//           the distinct chosen experts U, and this CTA's contiguous share of the units (u in U, 8-row block):
//           one lane per unit bulk-copies its 16 weight rows (padded rows: conflict-free fragment reads) and the
//           scales/biases onto the unit's mbarrier; the down rows of this CTA's output columns go to L2;
//  phase 3  unit K-splits on all warps as their copies land, partial sums combined in a fixed order, h written;
//  barrier
//  phase 4  down for this CTA's output columns, one task per (expert, 16-column tile, K-split), then one thread
//           per (token, column) forms the rank-order sum w_0 o_0 + w_1 o_1 + ..., the shared add and bf16 y.
// Every wait is bounded (SSB_ERR_TIMEOUT); the grid barrier is the ticket barrier of the CUDA-core kernel on the
// caller's sync word.
#include <algorithm>

#include "decode_internal.h"
#include "registry.h"
#include "select.cuh"
#include "tc_common.cuh"

namespace {

constexpr int TT = 512;               // threads per CTA
constexpr int TW = TT / 32;
constexpr int T_MAXR = 2;             // tokens
constexpr int T_MAXK = 16;
constexpr int T_MAXE = 512;
constexpr int T_MAXU = T_MAXR * T_MAXK;   // distinct routed experts of a call
constexpr int T_MAXUNITS = 24;            // gate/up units (16 rows x H) resident in one CTA
constexpr int T_MAXCOL = 32;              // output columns of one CTA: two 16-row tiles of the down weights
constexpr int T_EPL = 16;                 // experts per lane of the select scratch (E <= 512)

struct TcArgs {
  const uint16_t* x;
  int R, k, H, I, E;
  const uint16_t* w_router;
  const uint16_t* sh_gate_w;
  const float* bias;
  int flags;
  int layer;
  const int32_t* map;
  int64_t map_len;
  const int64_t* slot_ptr;
  int64_t n_slots;
  const uint8_t* shared_rec;
  RecOffs o;
  float* logits;   // [R, E + 1]
  int32_t* out_idx;
  float* out_w;
  float* out_sh_gate;
  int64_t* out_base;   // nullable
  float* h_buf;        // [R * k + R, I]
  float* o_buf;        // nullable [R, k, H]
  float* out;          // [R, H]
  uint16_t* y;         // [R, H]
  uint32_t* sync;      // [2]
  int32_t* err;
  int split_gu, split_d;   // K-splits of a gate/up unit and of a down task
  uint32_t pitch;          // bytes of one staged weight row (H / 2 + 16)
  uint32_t stage_bytes;    // one staged unit: 16 rows + gate/up scales and biases
  uint32_t off_xp, off_xsum, off_bases, off_bias, off_part, off_stage;
  uint64_t barrier_ns;     // grid-barrier wait bound (ssb_set_wait_limit_ns)
};

SSB_DEV void mma16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// codes j and j + 4 of word w (j = sh / 4) as the bf16 pair (128 + q_j, 128 + q_{j+4}), exact
SSB_DEV uint32_t npair(uint32_t w, int sh) { return ((w >> sh) & 0x000F000Fu) | 0x43004300u; }
// two floats -> bf16x2 (lo in the low half), round to nearest even
SSB_DEV uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// One 64-column group of a 16-row tile: c = sum over the group of (128 + q) * b for rows g (codes wa: words 2tq and
// 2tq + 1 of the group) and g + 8 (wb), against B columns whose K-ordered pairs are xb[0..7]. The K order inside
// a group: mma step s uses word 2tq + s/2, codes (2(s&1), 2(s&1) + 4) and (2(s&1) + 1, 2(s&1) + 5) -- the
// (0,4,1,5,2,6,3,7) order of every 8 elements, in which xb holds the activations.
// The four 16-column steps go to four independent accumulators (their latencies overlap), summed in a fixed order.
SSB_DEV void group_mma(float* c, uint2 wa, uint2 wb, const uint32_t* xb) {
  float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f}, c2[4] = {0.f, 0.f, 0.f, 0.f},
        c3[4] = {0.f, 0.f, 0.f, 0.f};
  mma16816(c0, npair(wa.x, 0), npair(wb.x, 0), npair(wa.x, 4), npair(wb.x, 4), xb[0], xb[1]);
  mma16816(c1, npair(wa.x, 8), npair(wb.x, 8), npair(wa.x, 12), npair(wb.x, 12), xb[2], xb[3]);
  mma16816(c2, npair(wa.y, 0), npair(wb.y, 0), npair(wa.y, 4), npair(wb.y, 4), xb[4], xb[5]);
  mma16816(c3, npair(wa.y, 8), npair(wb.y, 8), npair(wa.y, 12), npair(wb.y, 12), xb[6], xb[7]);
#pragma unroll
  for (int i = 0; i < 4; ++i) c[i] = (c0[i] + c1[i]) + (c2[i] + c3[i]);
}
// bf16 pairs of 8 consecutive values -> the same 8 values in the K order (0,4,1,5,2,6,3,7)
SSB_DEV uint4 kperm8_t(uint4 v) {
  return make_uint4(__byte_perm(v.x, v.z, 0x5410), __byte_perm(v.x, v.z, 0x7632), __byte_perm(v.y, v.w, 0x5410),
                    __byte_perm(v.y, v.w, 0x7632));
}

// Ticket grid barrier (see decode_fused.cu): false when the bounded wait gave up (SSB_ERR_TIMEOUT is set).
SSB_DEV bool grid_sync_tc(uint32_t* sync, int32_t* err, int* s_ok, uint64_t limit_ns) {
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    uint32_t old;
    asm volatile("atom.add.release.gpu.global.u32 %0, [%1], 1;" : "=r"(old) : "l"(sync) : "memory");
    const uint32_t target = old - old % gridDim.x + gridDim.x;
    const uint64_t t0 = globaltimer_ns();
    uint32_t polls = 0;
    for (;;) {
      uint32_t cur;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(cur) : "l"(sync) : "memory");
      if ((int32_t)(cur - target) >= 0) break;
      if ((++polls & 7u) == 0 && globaltimer_ns() - t0 > limit_ns) {
        ok = 0;
        set_err(err, SSB_ERR_TIMEOUT);
        break;
      }
    }
    *s_ok = ok;
  }
  __syncthreads();
  return *s_ok != 0;
}

// Gate/up unit (8 gate rows j0..j0+7 and the same 8 up rows of one expert) staged at `st`: rows 0..7 gate, 8..15
// up (pitch bytes apart), then gate scales, gate biases, up scales, up biases ([8 rows][ng] bf16 each). Partial
// sums over groups [g0, g1) for the tokens: acc[0..1] gate row (lane>>2) of tokens 2tq, 2tq+1; acc[2..3] up.
__device__ __noinline__ void gu_task(const uint8_t* st, uint32_t pitch, int ng, int g0, int g1, const uint4* xp,
                                     const float* xsum, int R, int lane, float* acc) {
  const int g = lane >> 2, tq = lane & 3;
  const int tb = g < R ? g : R - 1;           // B column g is token g (columns past R repeat the last token)
  const int c0 = 2 * tq < R ? 2 * tq : R - 1, c1 = 2 * tq + 1 < R ? 2 * tq + 1 : R - 1;
  const uint8_t* rg = st + (size_t)g * pitch + 8 * tq;
  const uint8_t* ru = st + (size_t)(g + 8) * pitch + 8 * tq;
  const uint16_t* sb = reinterpret_cast<const uint16_t*>(st + 16 * (size_t)pitch);
  const uint16_t *gs = sb + g * ng, *gb = gs + 8 * ng, *us = gb + 8 * ng, *ub = us + 8 * ng;
  const uint4* xr = xp + (size_t)tb * (ng * 8) + tq * 2;   // token tb's K-ordered row: 8 uint4 per group
  acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
#pragma unroll 2
  for (int grp = g0; grp < g1; ++grp) {
    const uint2 wa = *reinterpret_cast<const uint2*>(rg + grp * 32);
    const uint2 wb = *reinterpret_cast<const uint2*>(ru + grp * 32);
    const uint4 xa = xr[grp * 8], xb = xr[grp * 8 + 1];
    const uint32_t bv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
    float c[4];
    group_mma(c, wa, wb, bv);
    const float sg = bf16_bits(gs[grp]), su = bf16_bits(us[grp]);
    const float bg = fmaf(-128.f, sg, bf16_bits(gb[grp])), bu = fmaf(-128.f, su, bf16_bits(ub[grp]));
    const float x0 = xsum[c0 * ng + grp], x1 = xsum[c1 * ng + grp];
    acc[0] = fmaf(sg, c[0], fmaf(bg, x0, acc[0]));
    acc[1] = fmaf(sg, c[1], fmaf(bg, x1, acc[1]));
    acc[2] = fmaf(su, c[2], fmaf(bu, x0, acc[2]));
    acc[3] = fmaf(su, c[3], fmaf(bu, x1, acc[3]));
  }
}

// A gate/up unit (rows j0..j0+7 of gate and of up of the record at `b`) arrives in 20 bulk copies: pieces 0..7 the
// gate rows, 8..15 the up rows (one padded row each), 16..19 the gate scales, gate biases, up scales, up biases.
constexpr int GU_PIECES = 20;
SSB_DEV uint32_t gu_bytes(int H) { return 16u * (uint32_t)(H / 2) + 4u * (uint32_t)(8 * (H / 64) * 2); }
SSB_DEV void gu_piece(uint8_t* st, uint32_t pitch, const uint8_t* b, const RecOffs& o, int H, int j0, int pc,
                      uint64_t* bar) {
  const int ng = H / 64;
  const uint32_t hb = (uint32_t)H / 2, sbb = (uint32_t)(8 * ng * 2);
  if (pc < 16) {
    const int r = pc & 7;
    bulk_g2s(st + (size_t)pc * pitch, b + (pc < 8 ? o.gw : o.uw) + (int64_t)(j0 + r) * hb, hb, bar);
  } else {
    const int64_t off = pc == 16 ? o.gsc : pc == 17 ? o.gb : pc == 18 ? o.usc : o.ub;
    bulk_g2s(st + 16 * (size_t)pitch + (pc - 16) * sbb, b + off + (int64_t)j0 * ng * 2, sbb, bar);
  }
}
// One warp issues units [0, n) of the list: lane i < n arms unit i's barrier (a null record arrives with no bytes,
// its sums are then zero), then the lanes issue the 20 n pieces between them.
template <typename BaseOf, typename J0Of>
SSB_DEV void gu_issue_warp(uint8_t* stage, uint32_t stage_bytes, uint32_t pitch, const RecOffs& o, int H, int n,
                           BaseOf base_of, J0Of j0_of, uint64_t* bars, int lane) {
  for (int i = lane; i < n; i += 32) {
    if (base_of(i)) mbar_expect_tx(&bars[i], gu_bytes(H));
    else mbar_arrive(&bars[i]);
  }
  __syncwarp();
  for (int w = lane; w < n * GU_PIECES; w += 32) {
    const int i = w / GU_PIECES, pc = w - i * GU_PIECES;
    const uint8_t* b = base_of(i);
    if (b) gu_piece(stage + (size_t)i * stage_bytes, pitch, b, o, H, j0_of(i), pc, &bars[i]);
  }
}

// One down task: rows rt*16 .. rt*16 + 15 of an expert's staged column block `de` (padded rows of codes, then scales,
// then biases), groups [g0, g1) of its inter columns. The B operand is h of each token that chose the expert, staged
// per h_buf entry as bf16 hi / lo halves already in the mma fragment order (hp: [group][half][lane quad][8 pairs]),
// with the group sums of hi + lo beside it (hsum: [group]). Writes the partial column sums
// dd[(column * S + q) * T_MAXR + token].
__device__ __noinline__ void down_task(const uint8_t* de, uint32_t dpitch, uint32_t drows_b, uint32_t dsb_b, bool real,
                                       int ncol, int ngd, int rt, int g0, int g1, const uint4* hp, const float* hsum,
                                       const int* uent, int R, int lane, float* dd, int S, int q) {
  const int g = lane >> 2, tq = lane & 3;
  const int tok = g >> 1, hl = g & 1;           // B column g: half hl (0 = hi, 1 = lo) of token tok
  const int ent = tok < R ? uent[tok] : -1;      // its staged h, -1: the token did not choose this expert
  const int ent_c = tq < R ? uent[tq] : -1;      // the token of this lane's C columns (2 tq: hi, 2 tq + 1: lo)
  const int l0 = rt * 16 + g, l1 = l0 + 8;      // rows of this CTA's column block
  const bool v0 = real && l0 < ncol, v1 = real && l1 < ncol;
  const uint8_t* rw0 = de + (size_t)(v0 ? l0 : 0) * dpitch + 8 * tq;
  const uint8_t* rw1 = de + (size_t)(v1 ? l1 : 0) * dpitch + 8 * tq;
  const uint16_t* sc = reinterpret_cast<const uint16_t*>(de + drows_b);
  const uint16_t* bi = reinterpret_cast<const uint16_t*>(de + drows_b + dsb_b);
  float y0 = 0.f, y1 = 0.f;
  for (int grp = g0; grp < g1; ++grp) {
    const uint2 wa = v0 ? *reinterpret_cast<const uint2*>(rw0 + grp * 32) : make_uint2(0, 0);
    const uint2 wb = v1 ? *reinterpret_cast<const uint2*>(rw1 + grp * 32) : make_uint2(0, 0);
    uint4 b0 = make_uint4(0, 0, 0, 0), b1 = b0;
    if (ent >= 0) {
      const uint4* src = hp + (((size_t)ent * ngd + grp) * 2 + hl) * 8 + tq * 2;
      b0 = src[0];
      b1 = src[1];
    }
    const uint32_t bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    float c[4];
    group_mma(c, wa, wb, bv);
    const float hsv = ent_c >= 0 ? hsum[(size_t)ent_c * ngd + grp] : 0.f;
    if (v0) {
      const float s0 = bf16_bits(sc[l0 * ngd + grp]), b0f = fmaf(-128.f, s0, bf16_bits(bi[l0 * ngd + grp]));
      y0 = fmaf(s0, c[0] + c[1], fmaf(b0f, hsv, y0));
    }
    if (v1) {
      const float s1 = bf16_bits(sc[l1 * ngd + grp]), b1f = fmaf(-128.f, s1, bf16_bits(bi[l1 * ngd + grp]));
      y1 = fmaf(s1, c[2] + c[3], fmaf(b1f, hsv, y1));
    }
  }
  if (tq < R) {
    dd[((size_t)l0 * S + q) * T_MAXR + tq] = y0;
    dd[((size_t)l1 * S + q) * T_MAXR + tq] = y1;
  }
}

// NUX: H / 512 (16-byte chunks of a router row per lane, halved)
template <int NUX>
__global__ void __launch_bounds__(TT, 1) k_dec_tc(TcArgs a) {
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ int s_ok, s_fail;
  __shared__ int32_t s_ids[T_MAXR][T_MAXK];
  __shared__ float s_w[T_MAXR][T_MAXK];
  __shared__ float s_shg[T_MAXR];
  __shared__ SelectScratch<T_EPL> s_sel[T_MAXR];
  __shared__ float s_red[T_MAXR][TW];
  __shared__ int s_nu;                              // distinct routed experts (in order of first choice)
  __shared__ const uint8_t* s_ubase[T_MAXU + 1];   // their records; the shared expert last
  __shared__ int s_uent[T_MAXU + 1][T_MAXR];        // h_buf entry of (expert, token), -1: not chosen by it
  __shared__ int s_uidx[T_MAXR][T_MAXK];            // distinct-expert index of every choice
  __shared__ uint64_t s_full[T_MAXUNITS], s_shfull;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int R = a.R, k = a.k, H = a.H, I = a.I, E = a.E;
  const int ng = H / 64, ngd = I / 64, nj8 = I / 8;
  const RecOffs o = a.o;
  uint16_t* xs = reinterpret_cast<uint16_t*>(sm);                     // x, raw bf16 [R, H]
  uint4* xp = reinterpret_cast<uint4*>(sm + a.off_xp);                // x in the mma K order [R, H]
  float* xsum = reinterpret_cast<float*>(sm + a.off_xsum);            // [R, ng] group sums of x
  const uint8_t** bases = reinterpret_cast<const uint8_t**>(sm + a.off_bases);
  float* bias_s = reinterpret_cast<float*>(sm + a.off_bias);
  float* part = reinterpret_cast<float*>(sm + a.off_part);            // [unit][split][16 rows][R]
  uint8_t* stage = sm + a.off_stage;
  const int G = gridDim.x;
  // this CTA's output columns
  const int c0 = (int)((int64_t)blockIdx.x * H / G), c1 = (int)((int64_t)(blockIdx.x + 1) * H / G);
  const int ncol = c1 - c0, nrt = (ncol + 15) >> 4;
  // this CTA's unit of the shared expert (phase 1), if any
  const int sh_j8 = blockIdx.x < nj8 ? (int)blockIdx.x : -1;
  if (tid == 0) {
    s_fail = 0;
    for (int i = 0; i < T_MAXUNITS; ++i) mbar_init(&s_full[i], 1);
    mbar_init(&s_shfull, 1);
    fence_mbar_init();
  }
  __syncthreads();

  // ---------------- phase 1
  if (warp == 1 && sh_j8 >= 0)
    gu_issue_warp(stage, a.stage_bytes, a.pitch, o, H, 1, [&](int) { return a.shared_rec; }, [&](int) { return sh_j8 * 8; },
                  &s_shfull, lane);
  const int nrows = E + 1;   // router rows, then the shared-expert gate row
  const int rpc = (nrows + G - 1) / G;
  uint4 wr[2 * NUX];
  const int row0 = blockIdx.x * rpc + warp;
  if (warp < 4 && warp < rpc && row0 < nrows) {   // the router rows are static: load them first
    const uint16_t* wrow = row0 < E ? a.w_router + (int64_t)row0 * H : a.sh_gate_w;
#pragma unroll
    for (int i = 0; i < 2 * NUX; ++i) wr[i] = ld_stream_u4(wrow + (size_t)(lane + 32 * i) * 8);
  }
  if (warp < 4) {
    for (int e = tid; e < E; e += 4 * 32) bias_s[e] = a.bias ? __ldg(a.bias + e) : 0.f;
  } else {   // resolve every expert of the layer (unchosen misses are not errors)
    for (int e = tid - 4 * 32; e < E; e += TT - 4 * 32) {
      const int64_t m = (int64_t)a.layer * 512 + e;
      const int s = m < a.map_len ? ld_cg_i32(a.map + m) : -1;
      const long long p = s >= 0 && s < a.n_slots ? ld_cg_i64(a.slot_ptr + s) : 0;
      bases[e] = (p & 15) ? nullptr : (const uint8_t*)p;
    }
  }
  for (int c = tid; c < R * H / 8; c += TT) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(a.x) + c);
    reinterpret_cast<uint4*>(xs)[c] = v;
    xp[c] = kperm8_t(v);
  }
  __syncthreads();
  for (int c = warp; c < R * ng; c += TW) {   // group sums of x: lane pairs, then the butterfly (a fixed order)
    const uint32_t v = reinterpret_cast<const uint32_t*>(xs + (size_t)c * 64)[lane];
    const float s = warp_sum(bf16_lo(v) + bf16_hi(v));
    if (lane == 0) xsum[c] = s;
  }
  __syncthreads();
  if (warp < 4) {   // router logits: warp per row, the summation order of k_router_logits
    for (int rr = warp; rr < rpc; rr += 4) {
      const int row = blockIdx.x * rpc + rr;
      if (row >= nrows) break;
      if (rr != warp) {
        const uint16_t* wrow = row < E ? a.w_router + (int64_t)row * H : a.sh_gate_w;
#pragma unroll
        for (int i = 0; i < 2 * NUX; ++i) wr[i] = ld_stream_u4(wrow + (size_t)(lane + 32 * i) * 8);
      }
      for (int t = 0; t < R; ++t) {
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < 2 * NUX; ++i) {
          const uint4 xv = reinterpret_cast<const uint4*>(xs + (size_t)t * H)[lane + 32 * i];
          const uint4 wv = wr[i];
          acc = fmaf(bf16_lo(wv.x), bf16_lo(xv.x), acc);
          acc = fmaf(bf16_hi(wv.x), bf16_hi(xv.x), acc);
          acc = fmaf(bf16_lo(wv.y), bf16_lo(xv.y), acc);
          acc = fmaf(bf16_hi(wv.y), bf16_hi(xv.y), acc);
          acc = fmaf(bf16_lo(wv.z), bf16_lo(xv.z), acc);
          acc = fmaf(bf16_hi(wv.z), bf16_hi(xv.z), acc);
          acc = fmaf(bf16_lo(wv.w), bf16_lo(xv.w), acc);
          acc = fmaf(bf16_hi(wv.w), bf16_hi(xv.w), acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) a.logits[(int64_t)t * (E + 1) + row] = acc;
      }
    }
  } else if (sh_j8 >= 0 && warp >= 8 && warp < 8 + a.split_gu) {   // the shared expert's unit, K split over warps
    const int q = warp - 8;
    if (!mbar_wait_ns(&s_shfull, 0, SSB_WAIT_NS)) {
      s_fail = 1;
    } else {
      float acc[4];
      gu_task(stage, a.pitch, ng, q * ng / a.split_gu, (q + 1) * ng / a.split_gu, xp, xsum, R, lane, acc);
      const int g = lane >> 2, tq = lane & 3;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int t = 2 * tq + c;
        if (t < R) {
          part[((q * 16) + g) * R + t] = acc[c];
          part[((q * 16) + 8 + g) * R + t] = acc[2 + c];
        }
      }
    }
  }
  __syncthreads();
  if (sh_j8 >= 0 && !s_fail && tid < 8 * R) {   // shared h: lin() returns bf16, silu and the product round to bf16
    const int j = tid / R, t = tid % R;              // (model/layers.py:398-402)
    float gs = 0.f, us = 0.f;
    for (int q = 0; q < a.split_gu; ++q) {
      gs += part[((q * 16) + j) * R + t];
      us += part[((q * 16) + 8 + j) * R + t];
    }
    const float gbv = round_bf16(gs), ubv = round_bf16(us);
    a.h_buf[(int64_t)(R * k + t) * I + sh_j8 * 8 + j] = round_bf16(round_bf16(gbv / (1.f + expf(-gbv))) * ubv);
  }
  if (tid == 64 && ncol > 0) {   // the shared expert's down rows of this CTA's columns into L2 for phase 4
    const uint8_t* b = a.shared_rec;
    auto pf = [&](const uint8_t* s, int64_t bytes) {
      const uintptr_t s0 = (uintptr_t)s & ~(uintptr_t)15, s1 = ((uintptr_t)s + bytes + 15) & ~(uintptr_t)15;
      prefetch_l2((const void*)s0, (uint32_t)(s1 - s0));
    };
    pf(b + o.dw + (int64_t)c0 * (I / 2), (int64_t)ncol * (I / 2));
    pf(b + o.dsc + (int64_t)c0 * ngd * 2, (int64_t)ncol * ngd * 2);
    pf(b + o.db + (int64_t)c0 * ngd * 2, (int64_t)ncol * ngd * 2);
  }
  if (s_fail) {   // a copy never landed: the others may still be in flight
    if (tid == 0 && sh_j8 >= 0) mbar_wait_ns(&s_shfull, 0, SSB_WAIT_NS);
    if (tid == 0) set_err(a.err, SSB_ERR_TIMEOUT);
    return;
  }
  if (!grid_sync_tc(a.sync, a.err, &s_ok, a.barrier_ns)) return;

  // ---------------- phase 2: select (each CTA). The per-expert passes of warp_select run on all threads of the CTA --
  // element e of token t sits at index e = lane + 32 i of the token's scratch exactly as in warp_select, and the
  // denominator is summed lane-sequentially over i by one warp per token -- so every value and the chosen experts
  // are bit-identical to the router kernels; warp t then runs the candidate filter for token t.
  {
    constexpr int EW = 32 * T_EPL;
    float tmax0 = -INFINITY, tmax1 = -INFINITY;
    for (int idx = tid; idx < R * EW; idx += TT) {
      const int t = idx / EW, e = idx - t * EW;
      float l = -INFINITY;
      if (e < E) {
        l = __ldcg(a.logits + (int64_t)t * (E + 1) + e);
        if (a.bias) l = l + bias_s[e];
        if (a.flags & SSB_ROUTER_ROUND_BF16) l = round_bf16(l);
        if (t == 0) tmax0 = fmaxf(tmax0, l);
        else tmax1 = fmaxf(tmax1, l);
      }
      s_sel[t].v[e] = l;
    }
    {
      const float w0 = warp_max(tmax0), w1 = warp_max(tmax1);
      if (lane == 0) {
        s_red[0][warp] = w0;
        s_red[1][warp] = w1;
      }
    }
    __syncthreads();
    float m0 = s_red[0][0], m1 = s_red[1][0];
    for (int w = 1; w < TW; ++w) {
      m0 = fmaxf(m0, s_red[0][w]);
      m1 = fmaxf(m1, s_red[1][w]);
    }
    for (int idx = tid; idx < R * EW; idx += TT) {
      const int t = idx / EW, e = idx - t * EW;
      s_sel[t].v[e] = e < E ? expf(s_sel[t].v[e] - (t == 0 ? m0 : m1)) : 0.f;
    }
    __syncthreads();
    if (warp < R) {   // the denominator in warp_select's order: lane-sequential over i, then the butterfly
      float sl = 0.f;
#pragma unroll
      for (int i = 0; i < T_EPL; ++i) sl += s_sel[warp].v[lane + 32 * i];
      sl = warp_sum(sl);
      if (lane == 0) s_red[warp][0] = sl;
    }
    __syncthreads();
    for (int idx = tid; idx < R * EW; idx += TT) {
      const int t = idx / EW, e = idx - t * EW;
      const float pv = s_sel[t].v[e] / s_red[t][0];
      s_sel[t].v[e] = pv;
      s_sel[t].c[e] = (e < E) ? composite(order_key(pv), (uint32_t)e) : 0ull;
    }
    __syncthreads();
  }
  if (warp < R) {
    const float* lrow = a.logits + (int64_t)warp * (E + 1);
    unsigned long long mine;
    float my_p, sum;
    warp_select_finish<T_EPL>(s_sel[warp], E, k, lane, mine, my_p, sum);
    if (lane < k) {
      s_ids[warp][lane] = (int)(0xFFFFFFFFu - (uint32_t)(mine & 0xFFFFFFFFull));
      s_w[warp][lane] = my_p / sum;
    }
    if (lane == 0) {   // sigmoid(lin(x, shared_expert_gate)), bf16 output and bf16 sigmoid (model/layers.py:401)
      const float gl = round_bf16(__ldcg(lrow + E));
      s_shg[warp] = round_bf16(1.f / (1.f + expf(-gl)));
    }
  }
  __syncthreads();
  if (warp == 0) {   // the distinct chosen experts, in (token, rank) order of first appearance
    const int n = R * k;   // <= 32: lane l holds choice (l / k, l % k)
    const int e = lane < n ? s_ids[lane / k][lane % k] : -1 - lane;
    const unsigned same = __match_any_sync(0xFFFFFFFFu, e);
    const int leader = __ffs(same) - 1;
    const unsigned first = __ballot_sync(0xFFFFFFFFu, lane < n && leader == lane);
    const int u = __popc(first & ((1u << leader) - 1u));
    const int nu = __popc(first);
    for (int i = lane; i < (T_MAXU + 1) * T_MAXR; i += 32) (&s_uent[0][0])[i] = -1;
    __syncwarp();
    if (lane < n) {
      s_uidx[lane / k][lane % k] = u;
      s_uent[u][lane / k] = lane;   // the h_buf entry t * k + j of this (expert, token)
      if (leader == lane) s_ubase[u] = (e >= 0 && e < E) ? bases[e] : nullptr;
    }
    if (lane < R) s_uent[nu][lane] = R * k + lane;
    if (lane == 0) {
      s_nu = nu;
      s_ubase[nu] = a.shared_rec;
    }
  }
  __syncthreads();
  const int nu = s_nu;
  const int64_t NU = (int64_t)nu * nj8;
  const int u_lo = (int)(blockIdx.x * NU / G), u_hi = (int)((blockIdx.x + 1) * NU / G);
  const int n_my = u_hi - u_lo;
  if (warp == TW - 1) {   // this CTA's units: bulk copies spread over the lanes
    fence_proxy_async_smem();   // the stages were read by generic loads in phase 1
    gu_issue_warp(stage, a.stage_bytes, a.pitch, o, H, n_my, [&](int i) { return s_ubase[(u_lo + i) / nj8]; },
                  [&](int i) { return ((u_lo + i) % nj8) * 8; }, s_full, lane);
  } else if (warp == TW - 2 && ncol > 0) {   // the down rows of this CTA's columns of every chosen expert into L2
    for (int u = lane; u < nu; u += 32) {
      const uint8_t* b = s_ubase[u];
      if (!b) continue;
      auto pf = [&](const uint8_t* s, int64_t bytes) {
        const uintptr_t s0 = (uintptr_t)s & ~(uintptr_t)15, s1 = ((uintptr_t)s + bytes + 15) & ~(uintptr_t)15;
        prefetch_l2((const void*)s0, (uint32_t)(s1 - s0));
      };
      pf(b + o.dw + (int64_t)c0 * (I / 2), (int64_t)ncol * (I / 2));
      pf(b + o.dsc + (int64_t)c0 * ngd * 2, (int64_t)ncol * ngd * 2);
      pf(b + o.db + (int64_t)c0 * ngd * 2, (int64_t)ncol * ngd * 2);
    }
  } else if (warp == TW - 3 && blockIdx.x == 0) {
    if (lane < R * k) {
      const int r = lane / k, j = lane % k;
      const int e = s_ids[r][j];
      a.out_idx[lane] = e;
      a.out_w[lane] = s_w[r][j];
      // report an unusable choice with the precise reason (resolution errors of unchosen experts are normal)
      const uint8_t* b = resolve_expert(e, a.layer, a.map, a.map_len, a.slot_ptr, a.n_slots, a.err);
      if (a.out_base) a.out_base[lane] = (int64_t)b;
    }
    if (lane < R) a.out_sh_gate[lane] = s_shg[lane];
  }

  // ---------------- phase 3: gate/up units of this CTA, K-split over the warps as their copies land
  {
    const int S = a.split_gu;
    bool ok = true;
    const int lgS = __ffs(S) - 1;
    for (int tau = warp; tau < n_my * S && ok; tau += TW) {
      const int i = tau >> lgS, q = tau & (S - 1);
      if (!mbar_wait_ns(&s_full[i], 0, SSB_WAIT_NS)) {
        ok = false;
        break;
      }
      float acc[4];
      gu_task(stage + (size_t)i * a.stage_bytes, a.pitch, ng, q * ng / S, (q + 1) * ng / S, xp, xsum, R, lane, acc);
      const int g = lane >> 2, tq = lane & 3;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int t = 2 * tq + c;
        if (t < R) {
          part[(((size_t)i * S + q) * 16 + g) * R + t] = acc[c];
          part[(((size_t)i * S + q) * 16 + 8 + g) * R + t] = acc[2 + c];
        }
      }
    }
    if (__syncthreads_or(!ok)) {   // a copy never landed: let this CTA's copies land, then leave
      if (tid == 0) {
        set_err(a.err, SSB_ERR_TIMEOUT);
        for (int i = 0; i < n_my; ++i) mbar_wait_ns(&s_full[i], 0, SSB_WAIT_NS);
      }
      return;
    }
    // h = silu(g) * u in fp32 (kernels/moe_gemv_affine.py:76); the K-split sums in split order
    for (int idx = tid; idx < n_my * 8 * R; idx += TT) {
      const int i = idx / (8 * R), rem = idx - i * 8 * R, j = rem / R, t = rem - j * R;
      const int ug = u_lo + i, ui = ug / nj8, j8 = ug % nj8;
      const int p = s_uent[ui][t];
      if (p < 0) continue;   // (expert, token) not chosen: no h entry
      float gs = 0.f, us = 0.f;
      for (int q = 0; q < S; ++q) {
        gs += part[(((size_t)i * S + q) * 16 + j) * R + t];
        us += part[(((size_t)i * S + q) * 16 + 8 + j) * R + t];
      }
      a.h_buf[(int64_t)p * I + j8 * 8 + j] = s_ubase[ui] ? gs / (1.f + expf(-gs)) * us : 0.f;
    }
  }
  if (!grid_sync_tc(a.sync, a.err, &s_ok, a.barrier_ns)) return;

  // ---------------- phase 4: down for columns [c0, c1) of every distinct expert and the shared one
  {
    const int S = a.split_d;
    const int nud = nu + 1;
    const int np = R * k + R;                                  // h_buf entries: routed (t, j), then shared per token
    const uint32_t dpitch = (uint32_t)I / 2 + 16;            // one staged down row (padded: conflict-free reads)
    const uint32_t drows_b = (uint32_t)ncol * dpitch;
    const uint32_t dsb_b = (uint32_t)ncol * ngd * 2;          // one expert's scales (or biases) of these columns
    const uint32_t dexp_b = (drows_b + 2 * dsb_b + 15) & ~15u;
    float* dd = reinterpret_cast<float*>(stage);              // [expert][column][split][token]; stages are free now
    float* os = dd + (size_t)nud * T_MAXCOL * S * T_MAXR;     // [token][rank][column]: the weighted expert rows
    uint8_t* dst = reinterpret_cast<uint8_t*>(os + (size_t)T_MAXR * T_MAXK * T_MAXCOL);
    uint4* hp = reinterpret_cast<uint4*>(dst + (size_t)nud * dexp_b);   // [entry][group][half][quad lane][2]
    float* hsum = reinterpret_cast<float*>(hp + (size_t)np * ngd * 16);  // [entry][group]
    // the down rows of this CTA's columns of every expert (prefetched into L2 in phase 2): warp per expert,
    // 16-byte copies in flight together, one wait
    const bool sb16 = ((c0 * ngd * 2) & 15) == 0 && (dsb_b & 15) == 0;
    for (int ud = warp; ud < nud; ud += TW) {
      const uint8_t* b = s_ubase[ud];
      uint8_t* de = dst + (size_t)ud * dexp_b;
      const void* zero = a.x;
      for (int row = 0; row < ncol; ++row)
        for (int c = lane; c < I / 32; c += 32)
          cp_async16(smem_u32(de + row * dpitch + c * 16), b ? (const void*)(b + o.dw + (int64_t)(c0 + row) * (I / 2) + c * 16)
                                                              : zero, b ? 16u : 0u);
      for (int kind = 0; kind < 2; ++kind) {
        const uint8_t* sp = b ? b + (kind ? o.db : o.dsc) + (int64_t)c0 * ngd * 2 : nullptr;
        uint8_t* dp = de + drows_b + kind * dsb_b;
        if (sb16) {
          for (uint32_t c = lane; c < dsb_b / 16; c += 32)
            cp_async16(smem_u32(dp + c * 16), sp ? (const void*)(sp + c * 16) : zero, sp ? 16u : 0u);
        } else {
          for (uint32_t c = lane; c < dsb_b / 4; c += 32)
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dp + c * 4)),
                         "l"(sp ? (const void*)(sp + c * 4) : zero), "r"(sp ? 4 : 0) : "memory");
        }
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    // h of every entry as bf16 hi / lo halves in the mma fragment order, and the group sums of hi + lo: warp per
    // entry, lane l holding elements 16 l .. 16 l + 15 of each 512 (group l / 4, quad lane l % 4)
    for (int p = warp; p < np; p += TW) {
      for (int base = 0; base < I; base += 512) {
        const int grp = (base >> 6) + (lane >> 2), tq = lane & 3;
        float hv[16];
        const float4* src = reinterpret_cast<const float4*>(a.h_buf + (int64_t)p * I + base + 16 * lane);
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
          const float4 v = __ldcg(src + qq);
          hv[4 * qq] = v.x;
          hv[4 * qq + 1] = v.y;
          hv[4 * qq + 2] = v.z;
          hv[4 * qq + 3] = v.w;
        }
        uint32_t hi[8], lo[8];
        float hs = 0.f;
#pragma unroll
        for (int wd = 0; wd < 2; ++wd) {
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {   // pair (element jj, element jj + 4) of word wd: the mma step order
            const float p0 = hv[8 * wd + jj], p1 = hv[8 * wd + jj + 4];
            const uint32_t h2 = pack_bf16x2(p0, p1);
            const uint32_t l2 = pack_bf16x2(p0 - bf16_lo(h2), p1 - bf16_hi(h2));
            hi[4 * wd + jj] = h2;
            lo[4 * wd + jj] = l2;
            hs += (bf16_lo(h2) + bf16_lo(l2)) + (bf16_hi(h2) + bf16_hi(l2));
          }
        }
        uint4* d = hp + (((size_t)p * ngd + grp) * 2) * 8 + tq * 2;
        d[0] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        d[1] = make_uint4(hi[4], hi[5], hi[6], hi[7]);
        d[8] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        d[9] = make_uint4(lo[4], lo[5], lo[6], lo[7]);
        hs += __shfl_xor_sync(0xFFFFFFFFu, hs, 1);
        hs += __shfl_xor_sync(0xFFFFFFFFu, hs, 2);
        if (tq == 0) hsum[(size_t)p * ngd + grp] = hs;
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    const int lgS = __ffs(S) - 1, lgT = lgS + (nrt == 2 ? 1 : 0);
    for (int tau = warp; tau < (nud << lgT); tau += TW) {
      const int u = tau >> lgT, rem = tau & ((1 << lgT) - 1), rt = rem >> lgS, q = rem & (S - 1);
      down_task(dst + (size_t)u * dexp_b, dpitch, drows_b, dsb_b, s_ubase[u] != nullptr, ncol, ngd, rt, q * ngd / S,
                (q + 1) * ngd / S, hp, hsum, s_uent[u], R, lane, dd + ((size_t)u * T_MAXCOL) * S * T_MAXR, S, q);
    }
    __syncthreads();
    // the weighted row of every (token, rank, column), the splits summed in split order
    for (int idx = tid; idx < R * k * ncol; idx += TT) {
      const int r = idx / (k * ncol), rem = idx - r * k * ncol, j = rem / ncol, cl = rem - j * ncol;
      const int u = s_uidx[r][j];
      float v = 0.f;
      for (int q = 0; q < S; ++q) v += dd[(((size_t)u * T_MAXCOL + cl) * S + q) * T_MAXR + r];
      const float o_ = v * (s_ubase[u] ? s_w[r][j] : 0.f);   // acc * w, kernels/moe_gemv_affine.py:96-97
      os[((size_t)r * T_MAXK + j) * T_MAXCOL + cl] = o_;
      if (a.o_buf) a.o_buf[((int64_t)r * k + j) * H + c0 + cl] = o_;
    }
    __syncthreads();
    // one thread per (token, column): routed ranks in order, then the shared expert
    for (int idx = tid; idx < R * ncol; idx += TT) {
      const int r = idx / ncol, cl = idx - r * ncol, m = c0 + cl;
      float acc = os[((size_t)r * T_MAXK) * T_MAXCOL + cl];
      for (int j = 1; j < k; ++j) acc = acc + os[((size_t)r * T_MAXK + j) * T_MAXCOL + cl];   // rank order, :108-109
      float vs = 0.f;
      for (int q = 0; q < S; ++q) vs += dd[(((size_t)nu * T_MAXCOL + cl) * S + q) * T_MAXR + r];
      const float shv = round_bf16(s_shg[r] * round_bf16(vs));   // bf16(gate * bf16(h D^T))
      a.out[(int64_t)r * H + m] = acc;
      a.y[(int64_t)r * H + m] = f32_to_bf16(round_bf16(acc) + shv);   // routed.to(bf16) + sh
    }
  }
}

constexpr size_t T_SMEM_MAX = 227 * 1024;

}  // namespace

// Tensor-core fused decode layer; SSB_EUNSUPPORTED when the shape or the call's resident units do not fit.
static int decode_tc(const uint16_t* x, int64_t rows, int32_t topk, int32_t hidden, int32_t inter, int32_t experts,
                     const uint16_t* w_router, const uint16_t* sh_gate_w, const float* bias, int32_t flags,
                     int32_t layer, const int32_t* map_t, int64_t map_len, const int64_t* slot_ptr_t, int64_t n_slots,
                     const void* shared_record, float* logits_ws, int32_t* out_idx, float* out_w, float* out_sh_gate,
                     int64_t* out_base, float* h_buf, float* o_buf, float* out, uint16_t* y, uint32_t* sync,
                     int32_t* err, void* stream) {
  if (rows > T_MAXR || topk > T_MAXK || experts > T_MAXE || (hidden != 2048 && hidden != 2560 && hidden != 4096) ||
      inter % 128 || inter > 2048)
    return SSB_EUNSUPPORTED;
  if (((uintptr_t)h_buf & 15) != 0) return SSB_EUNSUPPORTED;
  static thread_local int sms_dev = -1, sms = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev != sms_dev) {
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    sms_dev = dev;
  }
  const int G = sms;
  if (G < 1) return SSB_EUNSUPPORTED;
  const int R = (int)rows;
  const int ng = hidden / 64, ngd = inter / 64;
  const int max_cols = (hidden + G - 1) / G;
  if (max_cols > T_MAXCOL) return SSB_EUNSUPPORTED;
  // units resident at once: the worst case of R * topk distinct experts, and the shared expert in phase 1
  const int64_t nu_max = (int64_t)R * topk * (inter / 8);
  const int units = (int)((nu_max + G - 1) / G);
  if (units > T_MAXUNITS) return SSB_EUNSUPPORTED;
  const uint32_t pitch = (uint32_t)hidden / 2 + 16;
  const uint32_t stage_bytes = (16 * pitch + 4 * 8 * ng * 2 + 127) & ~127u;
  const int split_gu = ng % 8 == 0 ? 8 : (ng % 4 == 0 ? 4 : (ng % 2 == 0 ? 2 : 1));
  const int split_d = ngd % 4 == 0 ? 4 : (ngd % 2 == 0 ? 2 : 1);
  // phase 4 reuses the gate/up stages: partial columns, weighted rows, the staged down rows and (if room) h
  const int nud_max = R * topk + 1;
  const size_t dexp_b = ((size_t)max_cols * (inter / 2 + 16) + 2 * (size_t)max_cols * ngd * 2 + 15) & ~(size_t)15;
  const size_t p4_fixed = (size_t)nud_max * T_MAXCOL * split_d * T_MAXR * 4 + (size_t)T_MAXR * T_MAXK * T_MAXCOL * 4 +
                          (size_t)nud_max * dexp_b;
  const size_t p4_h = (size_t)(R * topk + R) * ngd * (256 + 4);   // h halves (mma order) and group sums per entry
  const size_t part_bytes = (size_t)(units > 1 ? units : 1) * split_gu * 16 * T_MAXR * 4;
  uint32_t off = (uint32_t)((size_t)T_MAXR * hidden * 2);
  const uint32_t off_xp = off;
  off += (uint32_t)((size_t)T_MAXR * hidden * 2);
  const uint32_t off_xsum = off;
  off += (uint32_t)((size_t)T_MAXR * ng * 4);
  off = (off + 15) & ~15u;
  const uint32_t off_bases = off;
  off += T_MAXE * 8;
  const uint32_t off_bias = off;
  off += T_MAXE * 4;
  const uint32_t off_part = off;
  off += (uint32_t)part_bytes;
  off = (off + 127) & ~127u;
  const uint32_t off_stage = off;
  size_t stage_units = (size_t)(units > 1 ? units : 1) * stage_bytes;
  const size_t stage_region = std::max(stage_units, p4_fixed + p4_h);
  const size_t smem = off + stage_region;
  void (*kern)(TcArgs) = hidden == 2048 ? k_dec_tc<4> : hidden == 2560 ? k_dec_tc<5> : hidden == 4096 ? k_dec_tc<8>
                                                                                                : nullptr;
  if (!kern) return SSB_EUNSUPPORTED;
  cudaFuncAttributes fa;
  e = cudaFuncGetAttributes(&fa, kern);
  if (e != cudaSuccess) return (int)e;
  if (fa.sharedSizeBytes + smem + 1024 > T_SMEM_MAX) return SSB_EUNSUPPORTED;
  static thread_local size_t attr_smem[64][3] = {};
  const int ki = hidden == 2048 ? 0 : hidden == 2560 ? 1 : 2;
  if (dev >= 64 || attr_smem[dev][ki] < smem) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    if (dev < 64) attr_smem[dev][ki] = smem;
  }
  ssb_note_smem_bytes("moe_decode_fused", (int)(fa.sharedSizeBytes + smem));
  TcArgs a{};
  a.x = x;
  a.R = R;
  a.k = topk;
  a.H = hidden;
  a.I = inter;
  a.E = experts;
  a.w_router = w_router;
  a.sh_gate_w = sh_gate_w;
  a.bias = bias;
  a.flags = flags;
  a.layer = layer;
  a.map = map_t;
  a.map_len = map_len;
  a.slot_ptr = slot_ptr_t;
  a.n_slots = n_slots;
  a.shared_rec = (const uint8_t*)shared_record;
  a.o = rec_offsets(hidden, inter, 64);
  a.logits = logits_ws;
  a.out_idx = out_idx;
  a.out_w = out_w;
  a.out_sh_gate = out_sh_gate;
  a.out_base = out_base;
  a.h_buf = h_buf;
  a.o_buf = o_buf;
  a.out = out;
  a.y = y;
  a.sync = sync;
  a.err = err;
  a.split_gu = split_gu;
  a.split_d = split_d;
  a.pitch = pitch;
  a.stage_bytes = stage_bytes;
  a.off_xp = off_xp;
  a.off_xsum = off_xsum;
  a.off_bases = off_bases;
  a.off_bias = off_bias;
  a.off_part = off_part;
  a.off_stage = off_stage;
  a.barrier_ns = ssb_barrier_wait_ns();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)G);   // one CTA per SM, all resident (the cooperative launch fails otherwise)
  cfg.blockDim = dim3(TT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, a);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return (int)e;
  }
  return SSB_OK;
}

extern "C" int ssb_moe_decode_fused(const uint16_t* x, int64_t rows, int32_t topk, int32_t hidden, int32_t inter,
                                    int32_t experts, const uint16_t* w_router, const uint16_t* sh_gate_w,
                                    const float* bias, int32_t flags, int32_t layer, const int32_t* map_t,
                                    int64_t map_len, const int64_t* slot_ptr_t, int64_t n_slots,
                                    const void* shared_record, float* logits_ws, int32_t* out_idx, float* out_w,
                                    float* out_sh_gate, int64_t* out_base, float* h_buf, float* o_buf, float* out,
                                    uint16_t* y, uint32_t* sync, int32_t* err, void* stream) {
  SSB_CHECK_ARG(rows >= 0 && topk >= 1 && topk <= experts && experts >= 1 && layer >= 0);
  SSB_CHECK_ARG((flags & ~(SSB_ROUTER_ROUND_BF16 | SSB_DECODE_FUSED_CUDA_CORES | SSB_DECODE_FUSED_TENSOR_CORES)) == 0 &&
                (flags & (SSB_DECODE_FUSED_CUDA_CORES | SSB_DECODE_FUSED_TENSOR_CORES)) !=
                    (SSB_DECODE_FUSED_CUDA_CORES | SSB_DECODE_FUSED_TENSOR_CORES) &&
                map_len >= 0 && n_slots >= 0);
  const int32_t rflags = flags & SSB_ROUTER_ROUND_BF16;
  // which kernel: as asked, else by batch -- measured in the 48-layer decode graph on B200, one token runs faster on
  // CUDA cores (26.6 us per layer against 31.6: its phases are latency-bound either way), two tokens on the tensor
  // cores (38.3 us against 47: each distinct expert is read once for both)
  const bool tc = (flags & SSB_DECODE_FUSED_TENSOR_CORES) || (!(flags & SSB_DECODE_FUSED_CUDA_CORES) && rows >= 2);
  if (tc) {
    if (rows == 0) return SSB_OK;
    SSB_CHECK_ARG(x && w_router && sh_gate_w && map_t && slot_ptr_t && shared_record && logits_ws && out_idx &&
                  out_w && out_sh_gate && h_buf && out && y && sync);
    SSB_CHECK_ARG(((uintptr_t)shared_record & 15) == 0 && ((uintptr_t)x & 15) == 0 &&
                  ((uintptr_t)w_router & 15) == 0);
    const int rc = decode_tc(x, rows, topk, hidden, inter, experts, w_router, sh_gate_w, bias, rflags, layer, map_t,
                             map_len, slot_ptr_t, n_slots, shared_record, logits_ws, out_idx, out_w, out_sh_gate,
                             out_base, h_buf, o_buf, out, y, sync, err, stream);
    if (rc != SSB_EUNSUPPORTED) return rc;
  }
  return decode_fused_cuda_cores(x, rows, topk, hidden, inter, experts, w_router, sh_gate_w, bias, rflags, layer,
                                 map_t, map_len, slot_ptr_t, n_slots, shared_record, logits_ws, out_idx, out_w,
                                 out_sh_gate, out_base, h_buf, o_buf, out, y, sync, err, stream);
}
