// Fused decode MoE layer for one or two tokens: router logits, select, expert resolution, gate_up + SwiGLU,
// down + rank-order sum + shared expert in ONE cooperative launch with one CTA per SM and two grid barriers,
// instead of four dependent launches (router_logits -> router_select -> gate_up -> down).
//
// At batch 1 the layer is a chain of small dependent phases, so the kernel is arranged to keep every phase's
// memory traffic in flight early and every warp of the CTA busy:
//  phase 1  (inputs that do not depend on routing) every CTA computes ~(E + 1) / #SMs router logits (warp
//           per weight row; the shared-gate row last), its ~I / #SMs rows of the SHARED expert's gate/up
//           (h of the shared entries, both tokens from one read of the weights), resolves every expert of the
//           layer through the slot tables, preloads the router bias, and starts the bulk copy of its columns
//           of the shared expert's down rows;
//  barrier
//  phase 2  every CTA runs the select for every token itself (identical results everywhere); warp 0 then
//           issues the bulk copies of this CTA's slice of the routed gate/up rows in three chunks, each
//           completing on its own mbarrier, followed by its columns of every routed entry's down rows;
//  phase 3  routed gate_up: one warp item = one (entry, row): g and u dot products and h = silu(g) * u; an
//           item waits only for its own chunk, so the math on the first rows overlaps the later copies;
//  barrier
//  phase 4  h of every entry into the pre-scaled unit form; warp items = (entry, 4 output columns) write
//           their dot products to shared memory; then one thread per (token, column) forms the rank-order
//           sum, the shared add and the bf16 output.
// Every dot product keeps the summation order of the separate kernels (lane-sequential over 16-element units,
// then a butterfly), so the fused layer reproduces router_logits + router_select + moe_decode_layer bit for
// bit. Grid barriers spin with a bounded wait on a caller-owned counter word and give up with
// SSB_ERR_TIMEOUT; the word must be zero before the first call and again after a timeout.
#include "decode_internal.h"
#include "registry.h"
#include "select.cuh"
#include "tc_common.cuh"

namespace {

constexpr int FT = 512;   // threads per CTA
constexpr int FW = FT / 32;
constexpr int F_MAXR = 2;
constexpr int F_MAXK = 16;
constexpr int F_MAXE = 512;
constexpr int F_GS = 64;                       // group size of the affine codes
constexpr int F_MAXC = 32;                     // output columns per CTA
constexpr int F_MAXP = F_MAXR * (F_MAXK + 1);  // entries: routed, then one shared entry per token

struct FusedArgs {
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
  int rows_per_cta;    // gate/up rows of the flattened (routed entries, shared expert) list per CTA
  int stage_rows;      // rows one staging round holds
  int down_stage;      // 1: this CTA's columns of every entry's down rows are bulk-copied into shared memory
  uint32_t gstage_off, dstage_off;   // staged gate/up rows, later the h units; staged down rows
  uint64_t barrier_ns;               // grid-barrier wait bound (ssb_set_wait_limit_ns)
};

struct __align__(16) XUnitS {
  float2 v[8];
  float sum, pad0, pad1, pad2;
};

// All CTAs meet; false when the wait gave up (then SSB_ERR_TIMEOUT is set and the caller must stop).
// Ticket barrier on one monotonically increasing word: each CTA adds 1 with release semantics and waits
// (acquire loads) until the word reaches the end of its round, so nothing has to be reset between rounds and
// the release costs one atomic per CTA. Wrap-around is harmless (signed difference).
SSB_DEV bool grid_sync(uint32_t* sync, int32_t* err, int* s_ok, uint64_t limit_ns) {
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

SSB_DEV void xunit_store(XUnitS& d, const float* v16) {
  XUnit xu;
  xunit_from_f32(xu, v16);
#pragma unroll
  for (int q = 0; q < 8; ++q) d.v[q] = xu.v[q];
  d.sum = xu.sum;
}
SSB_DEV void xunit_load(XUnit& xu, const XUnitS& s) {
#pragma unroll
  for (int q = 0; q < 8; ++q) xu.v[q] = s.v[q];
  xu.sum = s.sum;
}

SSB_DEV void warp_sum2f(float& a, float& b) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xFFFFFFFFu, a, o);
    b += __shfl_xor_sync(0xFFFFFFFFu, b, o);
  }
}
SSB_DEV void warp_sum4f(float& a, float& b, float& c, float& d) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xFFFFFFFFu, a, o);
    b += __shfl_xor_sync(0xFFFFFFFFu, b, o);
    c += __shfl_xor_sync(0xFFFFFFFFu, c, o);
    d += __shfl_xor_sync(0xFFFFFFFFu, d, o);
  }
}

// Non-arriving expect-tx: adds `bytes` to the barrier's pending transaction count.
SSB_DEV void mbar_expect_only(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// NUX: 16-element units of x per lane (H / 512); NUI: units of h per lane (I / 512); EPL: experts per lane.
// One gate/up row of an expert in registers: codes of the lane's units and (scale | bias << 16) of their groups.
template <int NUX>
struct GuRow {
  uint2 g[NUX], u[NUX];
  uint32_t gsb[NUX], usb[NUX];
};
// g = x G_j^T and u = x U_j^T for one token, lane-sequential over the lane's units then the butterfly.
template <int NUX>
SSB_DEV void gu_row_dots(const GuRow<NUX>& w, const XUnitS* xt, int lane, float& ga, float& ua) {
  ga = 0.f;
  ua = 0.f;
#pragma unroll
  for (int i = 0; i < NUX; ++i) {
    XUnit xu;
    xunit_load(xu, xt[lane + 32 * i]);
    ga = unit_dot(w.g[i], bf16_lo(w.gsb[i]), bf16_hi(w.gsb[i]), xu, ga);
    ua = unit_dot(w.u[i], bf16_lo(w.usb[i]), bf16_hi(w.usb[i]), xu, ua);
  }
  warp_sum2f(ga, ua);
}

// NUX: 16-element units of x per lane (H / 512); NUI: units of h per lane (I / 512); EPL: experts per lane.
template <int NUX, int NUI, int EPL>
__global__ void __launch_bounds__(FT, 1) k_dec_fused(FusedArgs a) {
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ int s_ok;
  __shared__ int32_t s_ids[F_MAXR][F_MAXK];
  __shared__ float s_w[F_MAXR][F_MAXK];
  __shared__ float s_shg[F_MAXR];
  __shared__ SelectScratch<EPL> s_sel[F_MAXR];
  __shared__ float s_red[F_MAXR][FW];
  __shared__ const uint8_t* s_ebase[F_MAXP];
  __shared__ float s_dd[F_MAXP][F_MAXC];
  __shared__ uint64_t s_bar_d, s_bar_sh, s_bar_w[FW];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int R = a.R, k = a.k, H = a.H, I = a.I, E = a.E;
  const int P = R * k + R;   // entries: routed (r, j) at r*k + j, shared of token r at R*k + r
  constexpr int nux = NUX * 32, nui = NUI * 32;   // 16-element units of x, of h
  const int HB = H / 2, ng = H / F_GS;            // bytes of one gate/up row's codes; its groups
  const int ngd = I / F_GS;
  const int DRB = I / 2 + 2 * ngd * 2;            // bytes of one staged down row (codes, scales, biases)
  const int logI = __ffs(I) - 1;
  const RecOffs o = a.o;
  // shared memory: x (bf16 raw) | x units | expert bases | router bias | h units | down stage
  uint16_t* xs = reinterpret_cast<uint16_t*>(sm);
  XUnitS* xu_s = reinterpret_cast<XUnitS*>(sm + (size_t)F_MAXR * H * 2);
  const uint8_t** bases = reinterpret_cast<const uint8_t**>(xu_s + (size_t)F_MAXR * nux);
  float* bias_s = reinterpret_cast<float*>(bases + F_MAXE);
  XUnitS* hx = reinterpret_cast<XUnitS*>(sm + a.gstage_off);
  uint8_t* dst = sm + a.dstage_off;
  // this CTA's output columns
  const int c0 = (int)((int64_t)blockIdx.x * H / gridDim.x), c1 = (int)((int64_t)(blockIdx.x + 1) * H / gridDim.x);
  const int ncol = c1 - c0;
  const uint32_t dslot_b = (uint32_t)ncol * (uint32_t)DRB;   // one entry's staged down rows
  // this CTA's slice of the flattened gate/up row list: row j of routed entry p at p*I + j, then the rows of the
  // shared expert (computed for every token at once) at R*k*I + j
  const int64_t q_total = (int64_t)(R * k + 1) * I;
  const int64_t q_begin = (int64_t)blockIdx.x * a.rows_per_cta;
  const int64_t q_end = q_begin + a.rows_per_cta < q_total ? q_begin + a.rows_per_cta : q_total;
  if (tid == 0) {
    mbar_init(&s_bar_d, 1);
    mbar_init(&s_bar_sh, 1);
    for (int w = 0; w < FW; ++w) mbar_init(&s_bar_w[w], 1);
    fence_mbar_init();
  }

  // ---------------- phase 1: x, router logits, expert bases, bias; the shared expert's rows start moving
  const int nrows = E + 1;   // router rows, then the shared-expert gate row
  const int rpc = (nrows + gridDim.x - 1) / gridDim.x;
  uint4 wr[2 * NUX];
  const int row0 = blockIdx.x * rpc + warp;
  if (warp < 4 && warp < rpc && row0 < nrows) {   // the weights are static: load them first
    const uint16_t* wrow = row0 < E ? a.w_router + (int64_t)row0 * H : a.sh_gate_w;
#pragma unroll
    for (int i = 0; i < 2 * NUX; ++i) wr[i] = ld_stream_u4(wrow + (size_t)(lane + 32 * i) * 8);
  }
  if (warp == 3 && lane == 0 && q_end > (int64_t)R * k * I) {   // this CTA's shared gate/up rows into L2
    const int64_t s0 = (q_begin > (int64_t)R * k * I ? q_begin : (int64_t)R * k * I) - (int64_t)R * k * I;
    const int64_t s1 = q_end - (int64_t)R * k * I;
    const uint8_t* b = a.shared_rec;
    prefetch_l2(b + o.gw + s0 * HB, (uint32_t)((s1 - s0) * HB));
    prefetch_l2(b + o.uw + s0 * HB, (uint32_t)((s1 - s0) * HB));
    const uint32_t sb = (uint32_t)((s1 - s0) * ng * 2);
    if ((sb & 15u) == 0) {
      prefetch_l2(b + o.gsc + s0 * ng * 2, sb);
      prefetch_l2(b + o.gb + s0 * ng * 2, sb);
      prefetch_l2(b + o.usc + s0 * ng * 2, sb);
      prefetch_l2(b + o.ub + s0 * ng * 2, sb);
    }
  }
  if (warp < 4) {   // the router bias (static) into shared memory
    for (int e = tid; e < E; e += 4 * 32) bias_s[e] = a.bias ? __ldg(a.bias + e) : 0.f;
  } else {   // resolve every expert of the layer (unchosen misses are not errors): map, then slot_ptr, both
             // experts of a thread in flight together
    constexpr int NRT = FT - 4 * 32;
    for (int e0 = tid - 4 * 32; e0 < E; e0 += 2 * NRT) {
      const int e1 = e0 + NRT;
      const int64_t m0 = (int64_t)a.layer * 512 + e0, m1 = (int64_t)a.layer * 512 + e1;
      const int s0 = m0 < a.map_len ? ld_cg_i32(a.map + m0) : -1;
      const int s1 = e1 < E && m1 < a.map_len ? ld_cg_i32(a.map + m1) : -1;
      const long long p0 = s0 >= 0 && s0 < a.n_slots ? ld_cg_i64(a.slot_ptr + s0) : 0;
      const long long p1 = s1 >= 0 && s1 < a.n_slots ? ld_cg_i64(a.slot_ptr + s1) : 0;
      bases[e0] = (p0 & 15) ? nullptr : (const uint8_t*)p0;
      if (e1 < E) bases[e1] = (p1 & 15) ? nullptr : (const uint8_t*)p1;
    }
  }
  for (int c = tid; c < R * H / 8; c += FT)
    reinterpret_cast<uint4*>(xs)[c] = __ldg(reinterpret_cast<const uint4*>(a.x) + c);
  __syncthreads();
  if (a.down_stage && tid == 32 && ncol > 0) {   // this CTA's columns of the shared expert's down rows
    uint8_t* d = dst + (size_t)(R * k) * dslot_b;
    const uint8_t* b = a.shared_rec;
    mbar_expect_tx(&s_bar_sh, dslot_b);
    bulk_g2s(d, b + o.dw + (int64_t)c0 * (I / 2), (uint32_t)ncol * (I / 2), &s_bar_sh);
    bulk_g2s(d + ncol * (I / 2), b + o.dsc + (int64_t)c0 * ngd * 2, (uint32_t)ncol * ngd * 2, &s_bar_sh);
    bulk_g2s(d + ncol * (I / 2) + ncol * ngd * 2, b + o.db + (int64_t)c0 * ngd * 2, (uint32_t)ncol * ngd * 2,
             &s_bar_sh);
  }
  // x in the pre-scaled unit form for the gate/up dot products (every CTA)
  for (int idx = tid; idx < R * nux; idx += FT) {
    const int t = idx / nux, u = idx - t * nux;
    float v16[16];
    const uint4* p = reinterpret_cast<const uint4*>(xs + (size_t)t * H + u * 16);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const uint4 v = p[q];
      v16[8 * q + 0] = bf16_lo(v.x);
      v16[8 * q + 1] = bf16_hi(v.x);
      v16[8 * q + 2] = bf16_lo(v.y);
      v16[8 * q + 3] = bf16_hi(v.y);
      v16[8 * q + 4] = bf16_lo(v.z);
      v16[8 * q + 5] = bf16_hi(v.z);
      v16[8 * q + 6] = bf16_lo(v.w);
      v16[8 * q + 7] = bf16_hi(v.w);
    }
    xunit_store(xu_s[idx], v16);
  }
  __syncthreads();
  if (warp < 4) {
    for (int rr = warp; rr < rpc; rr += 4) {
      const int row = blockIdx.x * rpc + rr;
      if (row >= nrows) break;
      if (rr != warp) {
        const uint16_t* wrow = row < E ? a.w_router + (int64_t)row * H : a.sh_gate_w;
#pragma unroll
        for (int i = 0; i < 2 * NUX; ++i) wr[i] = ld_stream_u4(wrow + (size_t)(lane + 32 * i) * 8);
      }
      for (int t = 0; t < R; ++t) {   // the summation order of k_router_logits
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
  }
  if (!grid_sync(a.sync, a.err, &s_ok, a.barrier_ns)) {
    if (tid == 0 && a.down_stage && ncol > 0) mbar_wait_ns(&s_bar_sh, 0, SSB_WAIT_NS);
    return;
  }

  // ---------------- phase 2: select (each CTA). The per-expert passes of warp_select run on all threads of the
  // CTA -- element e of token t sits at index e = lane + 32 i of the token's scratch exactly as in warp_select,
  // and the denominator is summed lane-sequentially over i by one warp per token -- so every value and the
  // chosen experts are bit-identical to the router kernels; warp t then runs the candidate filter for token t.
  {
    constexpr int EW = 32 * EPL;
    float tmax0 = -INFINITY, tmax1 = -INFINITY;
    for (int idx = tid; idx < R * EW; idx += FT) {
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
    for (int w = 1; w < FW; ++w) {
      m0 = fmaxf(m0, s_red[0][w]);
      m1 = fmaxf(m1, s_red[1][w]);
    }
    for (int idx = tid; idx < R * EW; idx += FT) {
      const int t = idx / EW, e = idx - t * EW;
      s_sel[t].v[e] = e < E ? expf(s_sel[t].v[e] - (t == 0 ? m0 : m1)) : 0.f;
    }
    __syncthreads();
    if (warp < R) {   // the denominator in warp_select's order: lane-sequential over i, then the butterfly
      float sl = 0.f;
#pragma unroll
      for (int i = 0; i < EPL; ++i) sl += s_sel[warp].v[lane + 32 * i];
      sl = warp_sum(sl);
      if (lane == 0) s_red[warp][0] = sl;
    }
    __syncthreads();
    for (int idx = tid; idx < R * EW; idx += FT) {
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
    warp_select_finish<EPL>(s_sel[warp], E, k, lane, mine, my_p, sum);
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
  auto routed_base = [&](int p) -> const uint8_t* {
    const int e = s_ids[p / k][p % k];
    return (e >= 0 && e < E) ? bases[e] : nullptr;
  };
  const bool down_routed = a.down_stage && ncol > 0;
  if (warp == FW - 1) {
    // the last warp moves this CTA's columns of every routed entry's down rows (needed after the next barrier)
    // and publishes the entry bases, while the other warps start on the gate/up rows
    if (down_routed) {
      const uint8_t* b = lane < R * k ? routed_base(lane) : nullptr;
      if (b) mbar_expect_only(&s_bar_d, dslot_b);
      __syncwarp();
      if (b) {
        uint8_t* d = dst + (size_t)lane * dslot_b;
        bulk_g2s(d, b + o.dw + (int64_t)c0 * (I / 2), (uint32_t)ncol * (I / 2), &s_bar_d);
        bulk_g2s(d + ncol * (I / 2), b + o.dsc + (int64_t)c0 * ngd * 2, (uint32_t)ncol * ngd * 2, &s_bar_d);
        bulk_g2s(d + ncol * (I / 2) + ncol * ngd * 2, b + o.db + (int64_t)c0 * ngd * 2, (uint32_t)ncol * ngd * 2,
                 &s_bar_d);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_bar_d);
    } else if (ncol > 0) {   // no room to stage: L2 prefetch of the down rows
      for (int p = lane; p < R * k + 1; p += 32) {
        const uint8_t* b = p < R * k ? routed_base(p) : a.shared_rec;
        if (!b) continue;
        auto pf = [&](const uint8_t* s, int64_t bytes) {
          const uintptr_t s0 = (uintptr_t)s & ~(uintptr_t)15;
          const uintptr_t s1 = ((uintptr_t)s + bytes + 15) & ~(uintptr_t)15;
          prefetch_l2((const void*)s0, (uint32_t)(s1 - s0));
        };
        pf(b + o.dw + (int64_t)c0 * (I / 2), (int64_t)ncol * (I / 2));
        pf(b + o.dsc + (int64_t)c0 * ngd * 2, (int64_t)ncol * ngd * 2);
        pf(b + o.db + (int64_t)c0 * ngd * 2, (int64_t)ncol * ngd * 2);
      }
    }
    for (int p = lane; p < P; p += 32) s_ebase[p] = p < R * k ? routed_base(p) : a.shared_rec;
    if (blockIdx.x == 0) {
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
  }
  // ---------------- phase 3: gate_up rows of this CTA's slice. Warp w owns a contiguous block of rows and stages
  // them itself (lane 0 issues the bulk copies of each entry segment onto the warp's own barrier), so every
  // warp's rows are in flight at once and the math on them starts as soon as they land.
  {
    constexpr int HB3 = 256 * NUX, SB3 = 16 * NUX;          // bytes of one row's codes, of one scale array
    constexpr uint32_t RBS = 2 * HB3 + 4 * SB3;             // bytes of one staged row
    const int n_cta = q_end > q_begin ? (int)(q_end - q_begin) : 0;
    const int rpw = (n_cta + FW - 1) / FW;                   // rows per warp
    const int cap = a.stage_rows;                            // rows one warp's region holds
    const int w0 = warp * rpw, w1 = w0 + rpw < n_cta ? w0 + rpw : n_cta;
    uint8_t* wst = sm + a.gstage_off + (size_t)warp * cap * RBS;
    int wround = 0;
    bool ok = true;
    for (int r0 = w0; r0 < w1 && ok; r0 += cap, ++wround) {
      const int nr = w1 - r0 < cap ? w1 - r0 : cap;
      // rows [r0, r0 + nr) of the slice: one or two entry segments; lane s issues segment s
      const int64_t f0 = q_begin + r0, f1 = f0 + nr;
      const int64_t split = ((f0 >> logI) + 1) << logI;
      const int64_t sa = lane == 0 ? f0 : split, sb_ = lane == 0 ? (split < f1 ? split : f1) : f1;
      const uint8_t* b = nullptr;
      if (lane < 2 && sa < sb_) {
        const int p = (int)(sa >> logI);
        b = p < R * k ? routed_base(p) : a.shared_rec;
      }
      const uint32_t bytes = b ? (uint32_t)(sb_ - sa) * RBS : 0u;
      const uint32_t tot = __shfl_sync(0xFFFFFFFFu, bytes, 0) + __shfl_sync(0xFFFFFFFFu, bytes, 1);
      if (lane == 0) mbar_expect_tx(&s_bar_w[warp], tot);   // arrives; the copies below complete the phase
      __syncwarp();
      if (b) {
        const int j0 = (int)(sa & (I - 1)), n = (int)(sb_ - sa);
        uint8_t* d = wst + (size_t)(sa - f0) * RBS;
        // staged row layout: G codes | U codes | Gs | Gb | Us | Ub, as separate per-piece blocks of n rows
        bulk_g2s(d, b + o.gw + (int64_t)j0 * HB3, (uint32_t)n * HB3, &s_bar_w[warp]);
        bulk_g2s(d + (size_t)n * HB3, b + o.uw + (int64_t)j0 * HB3, (uint32_t)n * HB3, &s_bar_w[warp]);
        uint8_t* ds = d + (size_t)2 * n * HB3;
        bulk_g2s(ds, b + o.gsc + (int64_t)j0 * SB3, (uint32_t)n * SB3, &s_bar_w[warp]);
        bulk_g2s(ds + (size_t)n * SB3, b + o.gb + (int64_t)j0 * SB3, (uint32_t)n * SB3, &s_bar_w[warp]);
        bulk_g2s(ds + (size_t)2 * n * SB3, b + o.usc + (int64_t)j0 * SB3, (uint32_t)n * SB3, &s_bar_w[warp]);
        bulk_g2s(ds + (size_t)3 * n * SB3, b + o.ub + (int64_t)j0 * SB3, (uint32_t)n * SB3, &s_bar_w[warp]);
      }
      ok = mbar_wait_ns(&s_bar_w[warp], (uint32_t)(wround & 1), SSB_WAIT_NS);
      if (!ok) break;
      for (int rr = r0; rr < r0 + nr; ++rr) {
        const int64_t f = q_begin + rr;
        const int p = (int)(f >> logI), j = (int)(f & (I - 1));
        const uint8_t* rb = p < R * k ? routed_base(p) : a.shared_rec;
        // the row inside its segment's blocks
        const int64_t segs = (f < split) ? f0 : split;
        const int64_t sege = (f < split) ? (split < f1 ? split : f1) : f1;
        const int sn = (int)(sege - segs), si = (int)(f - segs);
        const uint8_t* d = wst + (size_t)(segs - f0) * RBS;
        const bool shared_row = p >= R * k;
        const int nt = shared_row ? R : 1;
#pragma unroll 1
        for (int qt = 0; qt < nt; ++qt) {
          const int t = shared_row ? qt : p / k;
          float ga = 0.f, ua = 0.f;
          if (rb) {
            GuRow<NUX> cur;
            const uint16_t* sc = reinterpret_cast<const uint16_t*>(d + (size_t)2 * sn * HB3);
#pragma unroll
            for (int i = 0; i < NUX; ++i) {
              const int u = lane + 32 * i, g = u >> 2;
              cur.g[i] = reinterpret_cast<const uint2*>(d + (size_t)si * HB3)[u];
              cur.u[i] = reinterpret_cast<const uint2*>(d + (size_t)(sn + si) * HB3)[u];
              const int gi = si * (SB3 / 2) + g, seg = sn * (SB3 / 2);
              cur.gsb[i] = (uint32_t)sc[gi] | ((uint32_t)sc[seg + gi] << 16);
              cur.usb[i] = (uint32_t)sc[2 * seg + gi] | ((uint32_t)sc[3 * seg + gi] << 16);
            }
            gu_row_dots<NUX>(cur, xu_s + (size_t)t * nux, lane, ga, ua);
          }
          if (lane == 0) {
            if (shared_row) {   // lin() returns bf16, silu and the product round to bf16 (model/layers.py:398-402)
              const float gbv = round_bf16(ga), ubv = round_bf16(ua);
              a.h_buf[(int64_t)(R * k + t) * I + j] = round_bf16(round_bf16(gbv / (1.f + expf(-gbv))) * ubv);
            } else {   // silu(g) * u in fp32, kernels/moe_gemv_affine.py:76
              a.h_buf[(int64_t)p * I + j] = rb ? ga / (1.f + expf(-ga)) * ua : 0.f;
            }
          }
        }
      }
      __syncwarp();   // the region is reused by the warp's next round
    }
    if (__syncthreads_or(!ok)) {   // a copy never landed: let the others land, then leave
      if (lane == 0 && !ok) mbar_wait_ns(&s_bar_w[warp], (uint32_t)(wround & 1), SSB_WAIT_NS);
      if (tid == 0) {
        set_err(a.err, SSB_ERR_TIMEOUT);
        if (down_routed) mbar_wait_ns(&s_bar_d, 0, SSB_WAIT_NS);
        if (a.down_stage && ncol > 0) mbar_wait_ns(&s_bar_sh, 0, SSB_WAIT_NS);
      }
      return;
    }
  }
  if (!grid_sync(a.sync, a.err, &s_ok, a.barrier_ns)) {
    if (tid == 0) {   // let this CTA's copies in flight land before it leaves
      if (down_routed) mbar_wait_ns(&s_bar_d, 0, SSB_WAIT_NS);
      if (a.down_stage && ncol > 0) mbar_wait_ns(&s_bar_sh, 0, SSB_WAIT_NS);
    }
    return;
  }

  // ---------------- phase 4: down for columns [c0, c1) of every entry, rank-order sum, shared add
  for (int idx = tid; idx < P * nui; idx += FT) {
    const int p = idx / nui, u = idx - p * nui;
    float v16[16];
    const float4* hp = reinterpret_cast<const float4*>(a.h_buf + (int64_t)p * I + u * 16);
#pragma unroll
    for (int qq = 0; qq < 4; ++qq) {
      const float4 v = __ldcg(hp + qq);
      v16[4 * qq] = v.x;
      v16[4 * qq + 1] = v.y;
      v16[4 * qq + 2] = v.z;
      v16[4 * qq + 3] = v.w;
    }
    xunit_store(hx[idx], v16);
  }
  if (a.down_stage && ncol > 0) {
    bool ok = mbar_wait_ns(&s_bar_sh, 0, SSB_WAIT_NS);
    if (down_routed) ok = mbar_wait_ns(&s_bar_d, 0, SSB_WAIT_NS) && ok;
    if (__syncthreads_or(!ok)) {
      if (tid == 0) {
        set_err(a.err, SSB_ERR_TIMEOUT);
        mbar_wait_spin(&s_bar_sh, 0, SSB_WAIT_NS);
        mbar_wait_spin(&s_bar_d, 0, SSB_WAIT_NS);
      }
      return;
    }
  } else {
    __syncthreads();
  }
  // warp items: (entry p, a group of 4 columns); the entry's h units are loaded once per item
  const int ncg = (ncol + 3) >> 2;
  for (int it = warp; it < P * ncg; it += FW) {
    const int p = it / ncg, cg = it - p * ncg;
    const uint8_t* eb = s_ebase[p];
    const int slot = p < R * k ? p : R * k;
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    if (eb) {
#pragma unroll
      for (int i = 0; i < NUI; ++i) {
        const int u = lane + 32 * i, g = u >> 2;
        XUnit xu;
        xunit_load(xu, hx[(size_t)p * nui + u]);
        if (a.down_stage) {   // row cl of the entry's staged codes, scales and biases
          const uint8_t* ds = dst + (size_t)slot * dslot_b;
          const uint8_t* dsc = ds + (size_t)ncol * (I / 2);
          const uint8_t* dbi = dsc + (size_t)ncol * ngd * 2;
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            const int cl = cg * 4 + cc;
            if (cl < ncol) {
              const uint2 wv = reinterpret_cast<const uint2*>(ds + (size_t)cl * (I / 2))[u];
              const float sv = bf16_bits(reinterpret_cast<const uint16_t*>(dsc + (size_t)cl * ngd * 2)[g]);
              const float bv = bf16_bits(reinterpret_cast<const uint16_t*>(dbi + (size_t)cl * ngd * 2)[g]);
              d[cc] = unit_dot(wv, sv, bv, xu, d[cc]);
            }
          }
        } else {
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            const int cl = cg * 4 + cc;
            if (cl < ncol) {
              const int64_t m = c0 + cl;
              const uint2 wv = __ldcg(reinterpret_cast<const uint2*>(eb + o.dw + m * (I / 2)) + u);
              const float sv = bf16_bits(__ldcg(reinterpret_cast<const unsigned short*>(eb + o.dsc + m * ngd * 2) + g));
              const float bv = bf16_bits(__ldcg(reinterpret_cast<const unsigned short*>(eb + o.db + m * ngd * 2) + g));
              d[cc] = unit_dot(wv, sv, bv, xu, d[cc]);
            }
          }
        }
      }
      warp_sum4f(d[0], d[1], d[2], d[3]);
    }
    if (lane < 4 && cg * 4 + lane < ncol) {
      const float v = lane == 0 ? d[0] : lane == 1 ? d[1] : lane == 2 ? d[2] : d[3];
      s_dd[p][cg * 4 + lane] = v;
    }
  }
  __syncthreads();
  // one thread per (token, column): routed ranks in order, then the shared expert
  for (int idx = tid; idx < R * ncol; idx += FT) {
    const int r = idx / ncol, cl = idx - r * ncol, m = c0 + cl;
    float acc = 0.f;
    for (int j = 0; j < k; ++j) {
      const int p = r * k + j;
      const float o_ = s_dd[p][cl] * (s_ebase[p] ? s_w[r][j] : 0.f);   // acc * w, kernels/moe_gemv_affine.py:96-97
      acc = (j == 0) ? o_ : acc + o_;                                    // rank order, :108-109
      if (a.o_buf) a.o_buf[((int64_t)r * k + j) * H + m] = o_;
    }
    const float shv = round_bf16(s_shg[r] * round_bf16(s_dd[R * k + r][cl]));   // bf16(gate * bf16(h D^T))
    a.out[(int64_t)r * H + m] = acc;
    a.y[(int64_t)r * H + m] = f32_to_bf16(round_bf16(acc) + shv);   // routed.to(bf16) + sh
  }
}

template <int NUX, int NUI>
void* pick_epl(int epl) {
  return epl <= 4 ? (void*)k_dec_fused<NUX, NUI, 4> : epl <= 8 ? (void*)k_dec_fused<NUX, NUI, 8>
                                                                : (void*)k_dec_fused<NUX, NUI, 16>;
}
template <int NUX>
void* pick_nui(int nui, int epl) {
  switch (nui) {
    case 1: return pick_epl<NUX, 1>(epl);
    case 2: return pick_epl<NUX, 2>(epl);
    case 4: return pick_epl<NUX, 4>(epl);
    default: return nullptr;
  }
}

constexpr size_t F_SMEM_MAX = 227 * 1024;   // opt-in shared memory per CTA on sm_100

}  // namespace

int decode_fused_cuda_cores(const uint16_t* x, int64_t rows, int32_t topk, int32_t hidden, int32_t inter,
                            int32_t experts, const uint16_t* w_router, const uint16_t* sh_gate_w, const float* bias,
                            int32_t flags, int32_t layer, const int32_t* map_t, int64_t map_len,
                            const int64_t* slot_ptr_t, int64_t n_slots, const void* shared_record, float* logits_ws,
                            int32_t* out_idx, float* out_w, float* out_sh_gate, int64_t* out_base, float* h_buf,
                            float* o_buf, float* out, uint16_t* y, uint32_t* sync, int32_t* err, void* stream) {
  SSB_CHECK_ARG(rows >= 0 && topk >= 1 && topk <= F_MAXK && topk <= experts && experts >= 1 && layer >= 0);
  if (rows > F_MAXR || experts > F_MAXE || hidden % 512 || hidden <= 0 || hidden > 4096 || inter % 512 ||
      inter <= 0 || inter > 2048 || inter == 1536)
    return SSB_EUNSUPPORTED;
  SSB_CHECK_ARG((flags & ~SSB_ROUTER_ROUND_BF16) == 0 && map_len >= 0 && n_slots >= 0);
  if (rows == 0) return SSB_OK;
  SSB_CHECK_ARG(x && w_router && sh_gate_w && map_t && slot_ptr_t && shared_record && logits_ws && out_idx && out_w &&
                out_sh_gate && h_buf && out && y && sync);
  SSB_CHECK_ARG(((uintptr_t)shared_record & 15) == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)w_router & 15) == 0);
  const int nux = hidden / 512, nui = inter / 512, epl = (experts + 31) / 32;
  void* kern = nullptr;
  switch (nux) {
    case 1: kern = pick_nui<1>(nui, epl); break;
    case 2: kern = pick_nui<2>(nui, epl); break;
    case 4: kern = pick_nui<4>(nui, epl); break;
    case 8: kern = pick_nui<8>(nui, epl); break;
    default: break;
  }
  if (!kern) return SSB_EUNSUPPORTED;
  // per (device, kernel) setup once: static shared memory, the SM count (host calls that would otherwise sit
  // between every launch), and the dynamic shared-memory attribute (raised when a call needs more)
  struct Prepared {
    int dev;
    void* kern;
    size_t static_smem;
    size_t smem;   // dynamic bytes the attribute allows
    int sms;
  };
  static thread_local Prepared prep[16];
  static thread_local int n_prep = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  Prepared* pp = nullptr;
  for (int i = 0; i < n_prep; ++i)
    if (prep[i].dev == dev && prep[i].kern == kern) pp = &prep[i];
  Prepared fresh{};
  if (!pp) {
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return (int)e;
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms < 1) return SSB_EUNSUPPORTED;
    fresh = Prepared{dev, kern, fa.sharedSizeBytes, 0, sms};
    if (n_prep < 16) pp = &prep[n_prep++];
    else pp = &fresh;
    *pp = fresh;
  }
  const int G = pp->sms;
  const int R = (int)rows, P = R * topk + R;
  const int64_t q_total = (int64_t)(R * topk + 1) * inter;   // gate/up rows: routed entries, then the shared expert
  const int rows_per_cta = (int)((q_total + G - 1) / G);
  const int max_cols = (hidden + G - 1) / G;
  if (max_cols > F_MAXC) return SSB_EUNSUPPORTED;
  const size_t DRB = (size_t)inter / 2 + 2 * (size_t)(inter / 64) * 2;   // one staged down row
  const size_t fixed = (size_t)F_MAXR * hidden * 2 + sizeof(XUnitS) * (size_t)F_MAXR * (hidden / 16) +
                       (size_t)F_MAXE * sizeof(void*) + (size_t)F_MAXE * sizeof(float);
  const size_t RB = (size_t)hidden + (size_t)hidden / 8;                  // one staged gate/up row
  const size_t hx_b = sizeof(XUnitS) * (size_t)P * (inter / 16);
  const size_t dstage_b = (size_t)(R * topk + 1) * max_cols * DRB;
  if (pp->static_smem + fixed + 1024 > F_SMEM_MAX) return SSB_EUNSUPPORTED;
  const size_t avail = F_SMEM_MAX - pp->static_smem - 1024 - fixed;
  // the stage holds the CTA's gate/up rows (in rounds when they do not all fit), later the h units
  auto stage_bytes = [&](int sr) {
    const size_t b = (size_t)sr * RB > hx_b ? (size_t)sr * RB : hx_b;
    return (b + 127) & ~(size_t)127;
  };
  // every warp stages its own block of ceil(rows_per_cta / 16) rows, in rounds of stage_rows when they do not fit
  int stage_rows = (rows_per_cta + FW - 1) / FW;
  if (stage_bytes(FW * stage_rows) > avail) stage_rows = (int)(avail / RB) / FW;
  if (stage_rows < 1 || stage_bytes(FW * stage_rows) > avail) return SSB_EUNSUPPORTED;
  const size_t stage_b = stage_bytes(FW * stage_rows);
  // this CTA's columns of every entry's down rows are staged in shared memory when they fit beside
  const int down_stage = stage_b + dstage_b <= avail ? 1 : 0;
  const size_t smem = fixed + stage_b + (down_stage ? dstage_b : 0);
  if (pp->smem < smem) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, FT, smem);
    if (e != cudaSuccess) return (int)e;
    if (per_sm < 1) return SSB_EUNSUPPORTED;
    pp->smem = smem;
  }
  ssb_note_smem_bytes("moe_decode_fused_cc", (int)(pp->static_smem + smem));
  FusedArgs a{};
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
  a.rows_per_cta = rows_per_cta;
  a.stage_rows = stage_rows;
  a.down_stage = down_stage;
  a.gstage_off = (uint32_t)fixed;
  a.dstage_off = (uint32_t)(fixed + stage_b);
  a.barrier_ns = ssb_barrier_wait_ns();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)G);   // one CTA per SM: all resident (the launch fails otherwise)
  cfg.blockDim = dim3(FT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, (void (*)(FusedArgs))kern, a);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return (int)e;
  }
  return SSB_OK;
}
