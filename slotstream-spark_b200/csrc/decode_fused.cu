// Fused decode MoE layer for one or two tokens: router logits, select, expert resolution, gate_up + SwiGLU,
// down + rank-order sum + shared expert in ONE cooperative launch with one CTA per SM and two grid barriers,
// instead of four dependent launches (router_logits -> router_select -> gate_up -> down).
//
// At batch 1 the layer is a chain of four tiny dependent phases; separate launches pay a grid drain and a
// launch for each, which dominated the old path. Here:
//  phase 1  every CTA computes ~(E + 1) / #SMs router logits (warp per weight row; the shared-gate row last)
//           while its other warps resolve the record base of every expert of the layer through the slot
//           tables into shared memory (static inputs: this overlaps the logits instead of following select);
//  barrier
//  phase 2  every CTA runs the warp select for every token itself (identical results everywhere, no extra
//           barrier); CTA 0 writes ids / weights / shared gate; each CTA issues L2 prefetches for the down
//           rows it will need in phase 4;
//  phase 3  gate_up: the (entry, row pair) items are split evenly over the CTAs, each warp streams its weight
//           words straight from HBM into registers and forms h = silu(G x) * (U x) (shared expert: bf16 chain);
//  barrier
//  phase 4  every CTA owns a contiguous slice of output columns for ALL entries, so the rank-order sum, the
//           shared add and the bf16 output need no further exchange.
// Every dot product keeps the summation order of the separate kernels (lane-sequential over 16-element units,
// then a butterfly), so the fused layer reproduces router_logits + router_select + moe_decode_layer bit for
// bit. Grid barriers spin with a bounded wait on a caller-owned counter word and give up with
// SSB_ERR_TIMEOUT; the word must be zero before the first call and again after a timeout.
#include "registry.h"
#include "select.cuh"
#include "tc_common.cuh"

namespace {

constexpr int FT = 512;   // threads per CTA
constexpr int FW = FT / 32;
constexpr int F_MAXR = 2;
constexpr int F_MAXK = 16;
constexpr int F_MAXE = 512;

struct FusedArgs {
  const uint16_t* x;
  int R, k, H, I, E, gs;
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
  int stage_pairs;     // gate/up row pairs one staging round of a CTA holds
  int down_stage;      // 1: this CTA's down rows of every entry are bulk-copied into shared memory after select
  uint32_t dstage_off; // their offset in the dynamic shared memory
};

struct __align__(16) XUnitS {
  float2 v[8];
  float sum, pad0, pad1, pad2;
};

// All CTAs meet; false when the wait gave up (then SSB_ERR_TIMEOUT is set and the caller must stop).
// Ticket barrier on one monotonically increasing word: each CTA adds 1 with release semantics and waits
// (acquire loads) until the word reaches the end of its round, so nothing has to be reset between rounds and
// the release costs one atomic per CTA. Wrap-around is harmless (signed difference).
SSB_DEV bool grid_sync(uint32_t* sync, int32_t* err, int* s_ok) {
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
      if ((++polls & 255u) == 0 && globaltimer_ns() - t0 > SSB_WAIT_NS) {
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

SSB_DEV void warp_sum4f(float& a, float& b, float& c, float& d) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xFFFFFFFFu, a, o);
    b += __shfl_xor_sync(0xFFFFFFFFu, b, o);
    c += __shfl_xor_sync(0xFFFFFFFFu, c, o);
    d += __shfl_xor_sync(0xFFFFFFFFu, d, o);
  }
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
  __shared__ uint64_t s_bar, s_bar_d;
  __shared__ int s_seg_p[4], s_seg_q0[4], s_seg_n[4];
  __shared__ uint32_t s_seg_off[4];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int R = a.R, k = a.k, H = a.H, I = a.I, E = a.E, gs = a.gs;
  const int P = R * k + R;                      // entries: routed (r, j) at r*k + j, shared of token r at R*k + r
  const int nux = H / 16, nui = I / 16;
  // shared memory: x (bf16 raw) | x units | expert bases | stage: the gate/up rows of phase 3, then the h units of
  // phase 4 in the same bytes
  uint16_t* xs = reinterpret_cast<uint16_t*>(sm);
  XUnitS* xu_s = reinterpret_cast<XUnitS*>(sm + (size_t)F_MAXR * H * 2);
  const uint8_t** bases = reinterpret_cast<const uint8_t**>(xu_s + (size_t)F_MAXR * nux);
  uint8_t* stage = reinterpret_cast<uint8_t*>(bases + F_MAXE);
  XUnitS* hx = reinterpret_cast<XUnitS*>(stage);
  uint8_t* dstage = sm + a.dstage_off;
  if (tid == 0) {
    mbar_init(&s_bar, 1);
    mbar_init(&s_bar_d, 1);
    fence_mbar_init();
  }

  // ---------------- phase 1: x, router logits, expert bases
  const int nrows = E + 1;   // router rows, then the shared-expert gate row
  const int rpc = (nrows + gridDim.x - 1) / gridDim.x;
  const int cpl = (H >> 3) >> 5;   // 16-byte chunks of a weight row per lane
  uint4 wr[2 * NUX];
  const int row0 = blockIdx.x * rpc + warp;
  if (warp < 4 && warp < rpc && row0 < nrows) {   // the weights are static: load them first
    const uint16_t* wrow = row0 < E ? a.w_router + (int64_t)row0 * H : a.sh_gate_w;
#pragma unroll
    for (int i = 0; i < 2 * NUX; ++i)
      if (i < cpl) wr[i] = ld_stream_u4(wrow + (size_t)(lane + 32 * i) * 8);
  }
  for (int c = tid; c < R * H / 8; c += FT)
    reinterpret_cast<uint4*>(xs)[c] = __ldg(reinterpret_cast<const uint4*>(a.x) + c);
  __syncthreads();
  if (warp < 4) {
    for (int rr = warp; rr < rpc; rr += 4) {
      const int row = blockIdx.x * rpc + rr;
      if (row >= nrows) break;
      if (rr != warp) {
        const uint16_t* wrow = row < E ? a.w_router + (int64_t)row * H : a.sh_gate_w;
#pragma unroll
        for (int i = 0; i < 2 * NUX; ++i)
          if (i < cpl) wr[i] = ld_stream_u4(wrow + (size_t)(lane + 32 * i) * 8);
      }
      for (int t = 0; t < R; ++t) {   // the summation order of k_router_logits
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < 2 * NUX; ++i) {
          if (i < cpl) {
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
        }
        acc = warp_sum(acc);
        if (lane == 0) a.logits[(int64_t)t * (E + 1) + row] = acc;
      }
    }
  } else {   // the other warps resolve every expert of the layer meanwhile (unchosen misses are not errors)
    for (int e = tid - 4 * 32; e < E; e += FT - 4 * 32)
      bases[e] = resolve_expert(e, a.layer, a.map, a.map_len, a.slot_ptr, a.n_slots, nullptr);
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
  if (!grid_sync(a.sync, a.err, &s_ok)) return;

  // ---------------- phase 2: select (each CTA). The per-expert passes of warp_select run on all threads of the
  // CTA -- element e of token t sits at index e = lane + 32 i of the token's scratch exactly as in warp_select,
  // and the denominator is summed lane-sequentially over i by one warp per token -- so every value and the
  // chosen experts are bit-identical to the router kernels; warp t then runs the candidate filter for token t.
  {
    constexpr int EW = 32 * EPL;
    float tmax[F_MAXR];
#pragma unroll
    for (int t = 0; t < F_MAXR; ++t) tmax[t] = -INFINITY;
    for (int idx = tid; idx < R * EW; idx += FT) {
      const int t = idx / EW, e = idx - t * EW;
      float l = -INFINITY;
      if (e < E) {
        l = __ldcg(a.logits + (int64_t)t * (E + 1) + e);
        if (a.bias) l = l + __ldg(a.bias + e);
        if (a.flags & SSB_ROUTER_ROUND_BF16) l = round_bf16(l);
        tmax[t] = fmaxf(tmax[t], l);
      }
      s_sel[t].v[e] = l;
    }
#pragma unroll
    for (int t = 0; t < F_MAXR; ++t) {
      const float wm = warp_max(tmax[t]);
      if (lane == 0) s_red[t][warp] = wm;
    }
    __syncthreads();
    float m[F_MAXR];
#pragma unroll
    for (int t = 0; t < F_MAXR; ++t) {
      m[t] = s_red[t][0];
      for (int w = 1; w < FW; ++w) m[t] = fmaxf(m[t], s_red[t][w]);
    }
    for (int idx = tid; idx < R * EW; idx += FT) {
      const int t = idx / EW, e = idx - t * EW;
      s_sel[t].v[e] = e < E ? expf(s_sel[t].v[e] - m[t]) : 0.f;
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
  auto entry_base = [&](int p) -> const uint8_t* {
    if (p >= R * k) return a.shared_rec;
    const int e = s_ids[p / k][p % k];
    return (e >= 0 && e < E) ? bases[e] : nullptr;
  };
  if (blockIdx.x == 0 && tid < R * k) {
    const int r = tid / k, j = tid % k;
    const int e = s_ids[r][j];
    a.out_idx[tid] = e;
    a.out_w[tid] = s_w[r][j];
    // report an unusable choice with the precise reason (resolution errors of unchosen experts are normal)
    const uint8_t* b = resolve_expert(e, a.layer, a.map, a.map_len, a.slot_ptr, a.n_slots, a.err);
    if (a.out_base) a.out_base[tid] = (int64_t)b;
  }
  if (blockIdx.x == 0 && tid < R) a.out_sh_gate[tid] = s_shg[tid];
  // this CTA's output columns, and L2 prefetches of their down rows (needed after the next barrier)
  const int c0 = (int)((int64_t)blockIdx.x * H / gridDim.x), c1 = (int)((int64_t)(blockIdx.x + 1) * H / gridDim.x);
  const int ncol = c1 - c0;
  const int ngd = I / gs;
  const uint32_t d_ebytes = (uint32_t)ncol * ((uint32_t)I / 2 + 2u * (uint32_t)ngd * 2u);   // one entry's down rows
  if (a.down_stage && tid == 32) {   // every entry's rows c0 .. c1-1 of D (codes, scales, biases) into dstage
    uint32_t bytes = 0;
    for (int pe = 0; pe < P; ++pe)
      if (entry_base(pe) && ncol > 0) bytes += d_ebytes;
    mbar_expect_tx(&s_bar_d, bytes);
    for (int pe = 0; pe < P && ncol > 0; ++pe) {
      const uint8_t* base = entry_base(pe);
      if (!base) continue;
      uint8_t* d = dstage + (size_t)pe * d_ebytes;
      bulk_g2s(d, base + a.o.dw + (int64_t)c0 * I / 2, (uint32_t)ncol * I / 2, &s_bar_d);
      bulk_g2s(d + ncol * I / 2, base + a.o.dsc + (int64_t)c0 * ngd * 2, (uint32_t)ncol * ngd * 2, &s_bar_d);
      bulk_g2s(d + ncol * I / 2 + ncol * ngd * 2, base + a.o.db + (int64_t)c0 * ngd * 2, (uint32_t)ncol * ngd * 2,
               &s_bar_d);
    }
  }
  for (int pe = lane; !a.down_stage && warp == FW - 1 && pe < P && c1 > c0; pe += 32) {
    const uint8_t* base = entry_base(pe);
    if (base) {
      const int ng = I / gs;
      auto pf = [&](const uint8_t* p, int64_t bytes) {
        const uintptr_t s0 = (uintptr_t)p & ~(uintptr_t)15;
        const uintptr_t s1 = ((uintptr_t)p + bytes + 15) & ~(uintptr_t)15;
        prefetch_l2((const void*)s0, (uint32_t)(s1 - s0));
      };
      pf(base + a.o.dw + (int64_t)c0 * I / 2, (int64_t)(c1 - c0) * I / 2);
      pf(base + a.o.dsc + (int64_t)c0 * ng * 2, (int64_t)(c1 - c0) * ng * 2);
      pf(base + a.o.db + (int64_t)c0 * ng * 2, (int64_t)(c1 - c0) * ng * 2);
    }
  }

  // ---------------- phase 3: gate_up. CTA b owns the (entry p, row pair q) items [b*ipc, (b+1)*ipc) of the
  // flattened list (a few contiguous row ranges of at most a few experts) and brings all of their codes, scales
  // and biases into shared memory with one set of bulk copies per round, so the whole expert traffic of the
  // layer is in flight at once; the warps then form h from shared memory.
  {
    const int pairs = I / 2;
    const int ng = H / gs;
    const uint32_t wrow = (uint32_t)H / 2, srow = (uint32_t)ng * 2;   // bytes of one row's codes, scales
    const int64_t items = (int64_t)P * pairs;
    const int64_t ipc = (items + gridDim.x - 1) / gridDim.x;
    const int64_t i_begin = (int64_t)blockIdx.x * ipc;
    const int64_t i_end = i_begin + ipc < items ? i_begin + ipc : items;
    int round = 0;
    for (int64_t r0 = i_begin; r0 < i_end; r0 += a.stage_pairs, ++round) {
      const int64_t r1 = r0 + a.stage_pairs < i_end ? r0 + a.stage_pairs : i_end;
      if (tid == 0) {   // segments (one per entry) of this round, their copies, one completion barrier
        int ns = 0;
        uint32_t off = 0, bytes = 0;
        for (int64_t it = r0; it < r1 && ns < 4;) {
          const int pe = (int)(it / pairs), q0 = (int)(it - (int64_t)pe * pairs);
          const int n = (int)((r1 - it) < (pairs - q0) ? (r1 - it) : (pairs - q0));
          s_seg_p[ns] = pe;
          s_seg_q0[ns] = q0;
          s_seg_n[ns] = n;
          s_seg_off[ns] = off;
          const uint8_t* base = entry_base(pe);
          const uint32_t rows = 2u * (uint32_t)n;
          if (base) bytes += rows * (2 * wrow + 4 * srow);
          off += rows * (2 * wrow + 4 * srow);
          it += n;
          ++ns;
        }
        for (int q = ns; q < 4; ++q) s_seg_n[q] = 0;
        mbar_expect_tx(&s_bar, bytes);
        for (int q = 0; q < ns; ++q) {
          const uint8_t* base = entry_base(s_seg_p[q]);
          if (!base) continue;
          const uint32_t rows = 2u * (uint32_t)s_seg_n[q];
          const int64_t j0 = 2 * (int64_t)s_seg_q0[q];
          uint8_t* d = stage + s_seg_off[q];
          bulk_g2s(d, base + a.o.gw + j0 * wrow, rows * wrow, &s_bar);
          bulk_g2s(d + rows * wrow, base + a.o.uw + j0 * wrow, rows * wrow, &s_bar);
          bulk_g2s(d + rows * 2 * wrow, base + a.o.gsc + j0 * srow, rows * srow, &s_bar);
          bulk_g2s(d + rows * (2 * wrow + srow), base + a.o.gb + j0 * srow, rows * srow, &s_bar);
          bulk_g2s(d + rows * (2 * wrow + 2 * srow), base + a.o.usc + j0 * srow, rows * srow, &s_bar);
          bulk_g2s(d + rows * (2 * wrow + 3 * srow), base + a.o.ub + j0 * srow, rows * srow, &s_bar);
        }
      }
      __syncthreads();
      // every thread waits for the copies; a CTA-wide decision to give up keeps the barrier below reachable
      if (__syncthreads_or(!mbar_wait_spin(&s_bar, (uint32_t)(round & 1), SSB_WAIT_NS))) {
        if (tid == 0) set_err(a.err, SSB_ERR_TIMEOUT);
        mbar_wait_spin(&s_bar, (uint32_t)(round & 1), SSB_WAIT_NS);   // let the copies land before leaving
        if (a.down_stage) mbar_wait_spin(&s_bar_d, 0, SSB_WAIT_NS);
        return;
      }
      for (int64_t it = r0 + warp; it < r1; it += FW) {
        // locate the segment of item `it`: segments are consecutive runs of the round's items
        int64_t first = r0;
        int q = 0;
        while (q < 3 && s_seg_n[q + 1] > 0 && it >= first + s_seg_n[q]) {
          first += s_seg_n[q];
          ++q;
        }
        const int pe = s_seg_p[q];
        const int lq = (int)(it - first);              // pair within the segment
        const int j0 = 2 * (s_seg_q0[q] + lq);
        float* hrow = a.h_buf + (int64_t)pe * I;
        if (!entry_base(pe)) {
          if (lane < 2) hrow[j0 + lane] = 0.f;
          continue;
        }
        const uint32_t rows = 2u * (uint32_t)s_seg_n[q];
        const uint8_t* d = stage + s_seg_off[q];
        const uint2* g0r = reinterpret_cast<const uint2*>(d + (2 * lq) * wrow);
        const uint2* g1r = reinterpret_cast<const uint2*>(d + (2 * lq + 1) * wrow);
        const uint2* u0r = reinterpret_cast<const uint2*>(d + rows * wrow + (2 * lq) * wrow);
        const uint2* u1r = reinterpret_cast<const uint2*>(d + rows * wrow + (2 * lq + 1) * wrow);
        const uint16_t* gsc = reinterpret_cast<const uint16_t*>(d + rows * 2 * wrow) + 2 * lq * ng;
        const uint16_t* gbi = reinterpret_cast<const uint16_t*>(d + rows * (2 * wrow + srow)) + 2 * lq * ng;
        const uint16_t* usc = reinterpret_cast<const uint16_t*>(d + rows * (2 * wrow + 2 * srow)) + 2 * lq * ng;
        const uint16_t* ubi = reinterpret_cast<const uint16_t*>(d + rows * (2 * wrow + 3 * srow)) + 2 * lq * ng;
        const int t = pe >= R * k ? pe - R * k : pe / k;
        float ga0 = 0.f, ua0 = 0.f, ga1 = 0.f, ua1 = 0.f;
#pragma unroll
        for (int i = 0; i < NUX; ++i) {
          const int u = lane + 32 * i;
          const int g = (u * 16) / gs;
          XUnit xu;
          xunit_load(xu, xu_s[(size_t)t * nux + u]);
          ga0 = unit_dot(g0r[u], bf16_bits(gsc[g]), bf16_bits(gbi[g]), xu, ga0);
          ua0 = unit_dot(u0r[u], bf16_bits(usc[g]), bf16_bits(ubi[g]), xu, ua0);
          ga1 = unit_dot(g1r[u], bf16_bits(gsc[ng + g]), bf16_bits(gbi[ng + g]), xu, ga1);
          ua1 = unit_dot(u1r[u], bf16_bits(usc[ng + g]), bf16_bits(ubi[ng + g]), xu, ua1);
        }
        warp_sum4f(ga0, ua0, ga1, ua1);
        if (lane < 2) {
          const float ga = lane ? ga1 : ga0, ua = lane ? ua1 : ua0;
          float h;
          if (pe >= R * k) {   // shared expert: lin() returns bf16, silu and the product round to bf16
            const float gbv = round_bf16(ga), ubv = round_bf16(ua);
            h = round_bf16(round_bf16(gbv / (1.f + expf(-gbv))) * ubv);
          } else {
            h = ga / (1.f + expf(-ga)) * ua;   // silu(g) * u in fp32, kernels/moe_gemv_affine.py:76
          }
          hrow[j0 + lane] = h;
        }
      }
      __syncthreads();   // the stage is reused by the next round (and by phase 4)
    }
  }
  if (!grid_sync(a.sync, a.err, &s_ok)) return;

  // ---------------- phase 4: down for columns [c0, c1) of every entry, rank-order sum, shared add
  for (int idx = tid; idx < P * nui; idx += FT) {
    const int p = idx / nui, u = idx - p * nui;
    float v16[16];
    const float4* hp = reinterpret_cast<const float4*>(a.h_buf + (int64_t)p * I + u * 16);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 v = __ldcg(hp + q);
      v16[4 * q] = v.x;
      v16[4 * q + 1] = v.y;
      v16[4 * q + 2] = v.z;
      v16[4 * q + 3] = v.w;
    }
    xunit_store(hx[idx], v16);
  }
  if (a.down_stage && __syncthreads_or(!mbar_wait_spin(&s_bar_d, 0, SSB_WAIT_NS))) {
    if (tid == 0) set_err(a.err, SSB_ERR_TIMEOUT);
    mbar_wait_spin(&s_bar_d, 0, SSB_WAIT_NS);
    return;
  }
  __syncthreads();
  const int ng4 = I / gs;
  for (int m = c0 + warp; m < c1; m += FW) {
    for (int r = 0; r < R; ++r) {
      const int nexp = k + 1;   // the token's routed entries in rank order, then its shared entry
      float acc = 0.f, shv = 0.f;
      // chunks of four entries: their words in flight together, one batched reduction; a rolled loop keeps the
      // code this once-per-launch phase fetches short
#pragma unroll 1
      for (int c = 0; c < nexp; c += 4) {
        const uint8_t* eb[4];
        uint2 wv[4][NUI];
        float sc[4][NUI], bi[4][NUI];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int j = c + jj;
          const int p = j < k ? r * k + j : R * k + r;
          eb[jj] = j < nexp ? entry_base(p) : nullptr;
#pragma unroll
          for (int i = 0; i < NUI; ++i) {
            const int u = lane + 32 * i;
            const int g = (u * 16) / gs;
            wv[jj][i] = make_uint2(0u, 0u);
            sc[jj][i] = bi[jj][i] = 0.f;
            if (eb[jj] && u < nui) {
              if (a.down_stage) {   // row m - c0 of the entry's staged codes, scales and biases
                const uint8_t* d = dstage + (size_t)p * d_ebytes;
                const int mi = m - c0;
                wv[jj][i] = reinterpret_cast<const uint2*>(d + (size_t)mi * I / 2)[u];
                sc[jj][i] = bf16_bits(reinterpret_cast<const uint16_t*>(d + (size_t)ncol * I / 2)[mi * ng4 + g]);
                bi[jj][i] = bf16_bits(
                    reinterpret_cast<const uint16_t*>(d + (size_t)ncol * I / 2 + (size_t)ncol * ng4 * 2)[mi * ng4 + g]);
              } else {
                wv[jj][i] = __ldcg(reinterpret_cast<const uint2*>(eb[jj] + a.o.dw + (int64_t)m * I / 2) + u);
                sc[jj][i] =
                    bf16_bits(__ldcg(reinterpret_cast<const uint16_t*>(eb[jj] + a.o.dsc) + (int64_t)m * ng4 + g));
                bi[jj][i] =
                    bf16_bits(__ldcg(reinterpret_cast<const uint16_t*>(eb[jj] + a.o.db) + (int64_t)m * ng4 + g));
              }
            }
          }
        }
        float d[4];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          d[jj] = 0.f;
          const int j = c + jj;
          const int p = j < k ? r * k + j : R * k + r;
#pragma unroll
          for (int i = 0; i < NUI; ++i) {
            const int u = lane + 32 * i;
            if (eb[jj] && u < nui) {
              XUnit xu;
              xunit_load(xu, hx[(size_t)p * nui + u]);
              d[jj] = unit_dot(wv[jj][i], sc[jj][i], bi[jj][i], xu, d[jj]);
            }
          }
        }
        warp_sum4f(d[0], d[1], d[2], d[3]);
        if (lane == 0) {
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const int j = c + jj;
            if (j >= nexp) break;
            const bool ok = eb[jj] != nullptr;
            if (j >= k) {
              shv = round_bf16((ok ? s_shg[r] : 0.f) * round_bf16(d[jj]));   // bf16(sigmoid gate * bf16(h D^T))
            } else {
              const float o = d[jj] * (ok ? s_w[r][j] : 0.f);   // acc * w, kernels/moe_gemv_affine.py:96-97
              acc = (j == 0) ? o : acc + o;                      // rank order, kernels/moe_gemv_affine.py:108-109
              if (a.o_buf) a.o_buf[((int64_t)r * k + j) * H + m] = o;
            }
          }
        }
      }
      if (lane == 0) {
        a.out[(int64_t)r * H + m] = acc;
        a.y[(int64_t)r * H + m] = f32_to_bf16(round_bf16(acc) + shv);   // routed.to(bf16) + sh
      }
    }
  }
}

// dynamic shared memory: x, x units, expert bases, then the stage (gate/up rows of one round, or the h units)
size_t fused_fixed_smem(int H) {
  return (size_t)F_MAXR * H * 2 + sizeof(XUnitS) * (size_t)F_MAXR * (H / 16) + (size_t)F_MAXE * sizeof(void*);
}
size_t fused_pair_bytes(int H, int gs) { return (size_t)2 * (2 * (H / 2) + 4 * (H / gs) * 2); }
size_t fused_hx_bytes(int I) { return sizeof(XUnitS) * (size_t)F_MAXR * (F_MAXK + 1) * (I / 16); }
constexpr size_t F_SMEM_BUDGET = 200 * 1024;

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

}  // namespace

extern "C" int ssb_moe_decode_fused(const uint16_t* x, int64_t rows, int32_t topk, int32_t hidden, int32_t inter,
                                    int32_t experts, const uint16_t* w_router, const uint16_t* sh_gate_w,
                                    const float* bias, int32_t flags, int32_t layer, const int32_t* map_t,
                                    int64_t map_len, const int64_t* slot_ptr_t, int64_t n_slots,
                                    const void* shared_record, float* logits_ws, int32_t* out_idx, float* out_w,
                                    float* out_sh_gate, int64_t* out_base, float* h_buf, float* o_buf, float* out,
                                    uint16_t* y, uint32_t* sync, int32_t* err, void* stream) {
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
  // pairs of gate/up rows one staging round holds: all of the CTA's share when it fits the budget
  int sms0 = 0, dev0 = 0;
  cudaGetDevice(&dev0);
  cudaDeviceGetAttribute(&sms0, cudaDevAttrMultiProcessorCount, dev0);
  if (sms0 < 1) sms0 = 148;
  const size_t fixed = fused_fixed_smem(hidden), pair_b = fused_pair_bytes(hidden, 64);
  const int64_t per_cta = ((int64_t)rows * (topk + 1) * (inter / 2) + sms0 - 1) / sms0;
  int64_t stage_pairs = (int64_t)((F_SMEM_BUDGET - fixed) / pair_b);
  if (stage_pairs > per_cta) stage_pairs = per_cta;
  if (stage_pairs > inter / 2) stage_pairs = inter / 2;   // a round then spans at most two entries
  if (stage_pairs < 1) return SSB_EUNSUPPORTED;
  size_t stage_b = (size_t)stage_pairs * pair_b;
  if (stage_b < fused_hx_bytes(inter)) stage_b = fused_hx_bytes(inter);
  size_t smem = fixed + stage_b;
  if (smem > 212 * 1024) return SSB_EUNSUPPORTED;   // with the static scratch, one CTA per SM must still fit
  // the down rows of every entry for this CTA's output columns, when they fit beside the stage
  const int max_cols = (hidden + sms0 - 1) / sms0;
  const size_t dstage_b = (size_t)rows * (topk + 1) * max_cols * ((size_t)inter / 2 + 2 * (size_t)(inter / 64) * 2);
  const int down_stage = fixed + stage_b + dstage_b <= 212 * 1024 ? 1 : 0;
  const uint32_t dstage_off = (uint32_t)(fixed + stage_b);
  if (down_stage) smem += dstage_b;
  // per (device, kernel) setup once: the dynamic shared-memory attribute (raised when a call needs more), an
  // occupancy check, the SM count (host calls that would otherwise sit between every launch)
  struct Prepared {
    int dev;
    void* kern;
    size_t smem;
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
  if (!pp || pp->smem < smem) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    ssb_note_smem("moe_decode_fused", (void (*)(FusedArgs))kern, smem);
    int per_sm = 0, sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, FT, smem);
    if (e != cudaSuccess) return (int)e;
    if (per_sm < 1 || sms < 1) return SSB_EUNSUPPORTED;
    if (!pp && n_prep < 16) pp = &prep[n_prep++];
    if (pp) *pp = Prepared{dev, kern, smem, sms};
  }
  const int sms = pp ? pp->sms : sms0;
  FusedArgs a{};
  a.x = x;
  a.R = (int)rows;
  a.k = topk;
  a.H = hidden;
  a.I = inter;
  a.E = experts;
  a.gs = 64;
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
  a.stage_pairs = (int)stage_pairs;
  a.down_stage = down_stage;
  a.dstage_off = dstage_off;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)sms);   // one CTA per SM: all resident (the launch fails otherwise)
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
