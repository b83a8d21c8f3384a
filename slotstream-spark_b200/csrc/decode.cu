// Decode grouped GEMV over routed experts addressed through the slot tables
// (slotstream_spark/kernels/moe_gemv_affine.py:113-147), plus the fused shared expert of the decode layer.
//
// Two launches:
//  * gate_up: CTA = (pair p = (row, rank) or the shared expert, 16 rows of inter). One thread copies the
//    slice of gate/up codes, scales and biases into shared memory with six bulk async copies; each of the
//    eight warps forms two rows of h = silu(G x) * (U x) in fp32, four independent dot products at once, with
//    the activation held in registers.
//  * down   : CTA = (row, 8 rows of hidden). It stages the down slices of all of the row's experts with bulk
//    copies issued BEFORE waiting on the gate_up grid (the records are static and the expert ids were
//    written two launches back), so under programmatic dependent launch the down weights stream in while
//    gate_up runs. The staged activations h_k are converted once per CTA into the pre-scaled per-unit form;
//    each warp then owns one output row and all experts, forms o_k = w_k * (D_k h_k) with the per-expert warp
//    reductions batched, and sums the ranks in order (out = o_0 + o_1 + ...), fusing the reference's
//    separate _rank_sum kernel.
// Every (row, rank, output) value is the same op sequence whatever the row count or slot placement, so a
// 3-row call equals three 1-row calls bit for bit.
#include "affine.cuh"
#include "registry.h"

namespace {

constexpr int GU_ROWS = 16;    // inter rows per gate_up CTA (two per warp)
constexpr int GU_WARPS = 8;
constexpr int DN_ROWS = 8;     // hidden rows per down CTA (one per warp)
constexpr int DN_WARPS = 8;
constexpr int DN_CHUNK = 8;    // experts whose warp reductions are batched together

struct DecodeArgs {
  const void* x;
  int x_f32;
  const int32_t* ids;
  const float* wts;
  int64_t R;
  int topk;
  int H, I, gs;
  int layer;
  const int32_t* map;
  int64_t map_len;
  const int64_t* slot_ptr;
  int64_t n_slots;
  const uint8_t* shared_rec;
  const float* sh_gate;
  const int64_t* bases;   // nullable: record base of each (row, rank), already resolved by the router
  RecOffs o;
  float* h_buf;
  float* o_buf;
  float* out;
  uint16_t* y;
  int32_t* err;
  int run;   // grouped gate_up: entries per run (<= GU_RUN), sized so the run's staged activations fit
};

// XUnit as stored in shared memory: 16-byte aligned, 80 bytes.
struct __align__(16) XUnitS {
  float2 v[8];
  float sum, pad0, pad1, pad2;
};

SSB_DEV void load_x16(const DecodeArgs& a, int64_t r, int u, float* x16) {
  if (a.x_f32) {
    const float4* p = reinterpret_cast<const float4*>((const float*)a.x + r * a.H + (int64_t)u * 16);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float4 v = p[q];
      x16[4 * q] = v.x;
      x16[4 * q + 1] = v.y;
      x16[4 * q + 2] = v.z;
      x16[4 * q + 3] = v.w;
    }
  } else {
    const uint4* p = reinterpret_cast<const uint4*>((const uint16_t*)a.x + r * a.H + (int64_t)u * 16);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      uint4 v = p[q];
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

// four independent warp sums, interleaved
SSB_DEV void warp_sum4(float& a, float& b, float& c, float& d) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xFFFFFFFFu, a, o);
    b += __shfl_xor_sync(0xFFFFFFFFu, b, o);
    c += __shfl_xor_sync(0xFFFFFFFFu, c, o);
    d += __shfl_xor_sync(0xFFFFFFFFu, d, o);
  }
}

// ------------------------------------------------------------------ gate/up
template <int NUX>
__global__ void __launch_bounds__(GU_WARPS * 32) k_dec_gate_up(DecodeArgs a) {
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ uint64_t bar;
  __shared__ const uint8_t* s_base;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t n_routed = a.R * a.topk;
  const int64_t p = blockIdx.y;
  const int n0 = blockIdx.x * GU_ROWS;
  const int H = a.H, gs = a.gs;
  const uint32_t wbytes = (uint32_t)GU_ROWS * H / 2, sbytes = (uint32_t)GU_ROWS * (H / gs) * 2;
  uint8_t* gw = sm;
  uint8_t* uw = gw + wbytes;
  uint8_t* gsc = uw + wbytes;
  uint8_t* gb = gsc + sbytes;
  uint8_t* usc = gb + sbytes;
  uint8_t* ub = usc + sbytes;
  const bool is_shared = p >= n_routed;
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](const uint8_t* base) {
    mbar_expect_tx(&bar, 2 * wbytes + 4 * sbytes);
    bulk_g2s(gw, base + a.o.gw + (int64_t)n0 * H / 2, wbytes, &bar);
    bulk_g2s(uw, base + a.o.uw + (int64_t)n0 * H / 2, wbytes, &bar);
    bulk_g2s(gsc, base + a.o.gsc + (int64_t)n0 * (H / gs) * 2, sbytes, &bar);
    bulk_g2s(gb, base + a.o.gb + (int64_t)n0 * (H / gs) * 2, sbytes, &bar);
    bulk_g2s(usc, base + a.o.usc + (int64_t)n0 * (H / gs) * 2, sbytes, &bar);
    bulk_g2s(ub, base + a.o.ub + (int64_t)n0 * (H / gs) * 2, sbytes, &bar);
  };
  if (tid == 0 && is_shared) {  // the shared record is static: start its copies before the wait
    s_base = a.shared_rec;
    issue(a.shared_rec);
  }
  pdl_wait();
  pdl_trigger();
  if (tid == 0 && !is_shared) {
    const uint8_t* base = a.bases ? (const uint8_t*)ld_cg_i64(a.bases + p)
                                  : resolve_expert(a.ids[p], a.layer, a.map, a.map_len, a.slot_ptr, a.n_slots, a.err);
    s_base = base;
    if (base) issue(base);
  }
  const int64_t r = is_shared ? p - n_routed : p / a.topk;
  const int nunits = H / 16;
  XUnit xu[NUX];
#pragma unroll
  for (int i = 0; i < NUX; ++i) {
    int u = lane + 32 * i;
    if (u < nunits) {
      float x16[16];
      load_x16(a, r, u, x16);
      xunit_from_f32(xu[i], x16);
    } else {
      xunit_zero(xu[i]);
    }
  }
  __syncthreads();
  const uint8_t* base = s_base;
  float* hrow = a.h_buf + p * a.I;
  if (!base) {
    for (int j = tid; j < GU_ROWS; j += blockDim.x) hrow[n0 + j] = 0.f;
    return;
  }
  if (!mbar_wait(&bar, 0, SSB_WAIT_LIMIT)) {
    set_err(a.err, SSB_ERR_TIMEOUT);
    mbar_wait(&bar, 0, SSB_WAIT_LIMIT);  // let the copies land before the CTA's shared memory is released
    return;
  }
  const int ng = H / gs;
  const int j0 = 2 * warp, j1 = j0 + 1;
  const uint2* g0r = reinterpret_cast<const uint2*>(gw + (size_t)j0 * H / 2);
  const uint2* u0r = reinterpret_cast<const uint2*>(uw + (size_t)j0 * H / 2);
  const uint2* g1r = reinterpret_cast<const uint2*>(gw + (size_t)j1 * H / 2);
  const uint2* u1r = reinterpret_cast<const uint2*>(uw + (size_t)j1 * H / 2);
  const uint16_t* gs16 = reinterpret_cast<const uint16_t*>(gsc);
  const uint16_t* gb16 = reinterpret_cast<const uint16_t*>(gb);
  const uint16_t* us16 = reinterpret_cast<const uint16_t*>(usc);
  const uint16_t* ub16 = reinterpret_cast<const uint16_t*>(ub);
  float ga0 = 0.f, ua0 = 0.f, ga1 = 0.f, ua1 = 0.f;
#pragma unroll
  for (int i = 0; i < NUX; ++i) {
    int u = lane + 32 * i;
    if (u < nunits) {
      const int g = (u * 16) / gs;
      ga0 = unit_dot(g0r[u], bf16_bits(gs16[j0 * ng + g]), bf16_bits(gb16[j0 * ng + g]), xu[i], ga0);
      ua0 = unit_dot(u0r[u], bf16_bits(us16[j0 * ng + g]), bf16_bits(ub16[j0 * ng + g]), xu[i], ua0);
      ga1 = unit_dot(g1r[u], bf16_bits(gs16[j1 * ng + g]), bf16_bits(gb16[j1 * ng + g]), xu[i], ga1);
      ua1 = unit_dot(u1r[u], bf16_bits(us16[j1 * ng + g]), bf16_bits(ub16[j1 * ng + g]), xu[i], ua1);
    }
  }
  warp_sum4(ga0, ua0, ga1, ua1);
  if (lane < 2) {
    const float ga = lane ? ga1 : ga0, ua = lane ? ua1 : ua0;
    float h;
    if (is_shared) {
      // shared expert: lin() returns bf16, silu and the product round to bf16 (model/layers.py:398-400)
      const float gbv = round_bf16(ga), ubv = round_bf16(ua);
      h = round_bf16(round_bf16(gbv / (1.f + expf(-gbv))) * ubv);
    } else {
      h = ga / (1.f + expf(-ga)) * ua;   // silu(g) * u in fp32, kernels/moe_gemv_affine.py:76
    }
    hrow[n0 + j0 + lane] = h;
  }
}

// ------------------------------------------------------------------ down + rank-order combine (+ shared)
template <int NUI>
__global__ void __launch_bounds__(DN_WARPS * 32) k_dec_down(DecodeArgs a) {
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ uint64_t bar, bar_h;
  __shared__ const uint8_t* s_base[33];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t r = blockIdx.y;
  const int m0 = blockIdx.x * DN_ROWS;
  const int I = a.I, gs = a.gs, H = a.H;
  const bool has_sh = a.shared_rec != nullptr;
  const int nexp = a.topk + (has_sh ? 1 : 0);
  const int nunits = I / 16, ng = I / gs;
  const uint32_t wbytes = (uint32_t)DN_ROWS * I / 2, sbytes = (uint32_t)DN_ROWS * (I / gs) * 2;
  const uint32_t ebytes = wbytes + 2 * sbytes;
  float* hraw = reinterpret_cast<float*>(sm + (size_t)nexp * ebytes);                  // [nexp][I]
  XUnitS* hx = reinterpret_cast<XUnitS*>(sm + (size_t)nexp * ebytes + (size_t)nexp * I * 4);  // [nexp][nunits]
  if (tid == 0) {
    mbar_init(&bar, 1);
    mbar_init(&bar_h, 1);
    fence_mbar_init();
  }
  // One thread per expert resolves its record. The expert ids were written before the previous (gate_up)
  // grid started, and every grid here triggers its dependents only after its own wait, so they are complete
  // and visible now (read through L2).
  if (tid < nexp) {
    if (tid >= a.topk) s_base[tid] = a.shared_rec;
    else if (a.bases) s_base[tid] = (const uint8_t*)ld_cg_i64(a.bases + r * a.topk + tid);
    else s_base[tid] = resolve_expert(ld_cg_i32(a.ids + r * a.topk + tid), a.layer, a.map, a.map_len, a.slot_ptr,
                                      a.n_slots, nullptr);
  }
  __syncthreads();
  if (tid == 0) {
    uint32_t total = 0;
    for (int j = 0; j < nexp; ++j) total += s_base[j] ? ebytes : 0u;
    mbar_expect_tx(&bar, total);
    for (int j = 0; j < nexp; ++j) {
      const uint8_t* base = s_base[j];
      if (!base) continue;
      uint8_t* dst = sm + (size_t)j * ebytes;
      bulk_g2s(dst, base + a.o.dw + (int64_t)m0 * I / 2, wbytes, &bar);
      bulk_g2s(dst + wbytes, base + a.o.dsc + (int64_t)m0 * (I / gs) * 2, sbytes, &bar);
      bulk_g2s(dst + wbytes + sbytes, base + a.o.db + (int64_t)m0 * (I / gs) * 2, sbytes, &bar);
    }
  }
  pdl_wait();
  pdl_trigger();
  if (tid == 0) {   // h was written by the gate_up grid: stage it only after the wait
    uint32_t total = 0;
    for (int j = 0; j < nexp; ++j) total += s_base[j] ? (uint32_t)I * 4u : 0u;
    mbar_expect_tx(&bar_h, total);
    for (int j = 0; j < nexp; ++j) {
      if (!s_base[j]) continue;
      const int64_t pair = j >= a.topk ? a.R * a.topk + r : r * a.topk + j;
      bulk_g2s(hraw + (size_t)j * I, a.h_buf + pair * I, (uint32_t)I * 4u, &bar_h);
    }
  }
  // the decision to give up is made for the whole CTA, so no thread is left at the barrier below
  if (__syncthreads_or(!mbar_wait(&bar_h, 0, SSB_WAIT_LIMIT))) {
    if (tid == 0) set_err(a.err, SSB_ERR_TIMEOUT);
    mbar_wait(&bar, 0, SSB_WAIT_LIMIT);
    mbar_wait(&bar_h, 0, SSB_WAIT_LIMIT);
    return;
  }
  // pre-scaled per-unit form of every expert's activation, once per CTA
  for (int idx = tid; idx < nexp * nunits; idx += DN_WARPS * 32) {
    const int j = idx / nunits, u = idx - j * nunits;
    XUnit xu;
    if (s_base[j]) {
      float h16[16];
      const float4* hp = reinterpret_cast<const float4*>(hraw + (size_t)j * I + u * 16);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float4 v = hp[q];
        h16[4 * q] = v.x;
        h16[4 * q + 1] = v.y;
        h16[4 * q + 2] = v.z;
        h16[4 * q + 3] = v.w;
      }
      xunit_from_f32(xu, h16);
    } else {
      xunit_zero(xu);
    }
    XUnitS& d = hx[idx];
#pragma unroll
    for (int q = 0; q < 8; ++q) d.v[q] = xu.v[q];
    d.sum = xu.sum;
  }
  __syncthreads();
  if (!mbar_wait(&bar, 0, SSB_WAIT_LIMIT)) {
    if (tid == 0) set_err(a.err, SSB_ERR_TIMEOUT);
    mbar_wait(&bar, 0, SSB_WAIT_LIMIT);
    return;
  }
  const int row = warp;
  const int m = m0 + row;
  float acc = 0.f, shv = 0.f;
  for (int c0 = 0; c0 < nexp; c0 += DN_CHUNK) {
    float d[DN_CHUNK];
#pragma unroll
    for (int jj = 0; jj < DN_CHUNK; ++jj) {
      d[jj] = 0.f;
      const int j = c0 + jj;
      if (j < nexp && s_base[j]) {
        const uint8_t* ew = sm + (size_t)j * ebytes;
        const uint2* wr = reinterpret_cast<const uint2*>(ew + (size_t)row * I / 2);
        const uint16_t* sr = reinterpret_cast<const uint16_t*>(ew + wbytes) + row * ng;
        const uint16_t* br = reinterpret_cast<const uint16_t*>(ew + wbytes + sbytes) + row * ng;
#pragma unroll
        for (int i = 0; i < NUI; ++i) {
          const int u = lane + 32 * i;
          if (u < nunits) {
            const XUnitS& xs = hx[(size_t)j * nunits + u];
            XUnit xu;
#pragma unroll
            for (int q = 0; q < 8; ++q) xu.v[q] = xs.v[q];
            xu.sum = xs.sum;
            const int g = (u * 16) / gs;
            d[jj] = unit_dot(wr[u], bf16_bits(sr[g]), bf16_bits(br[g]), xu, d[jj]);
          }
        }
      }
    }
#pragma unroll
    for (int jj = 0; jj < DN_CHUNK; jj += 4) warp_sum4(d[jj], d[jj + 1], d[jj + 2], d[jj + 3]);
    if (lane == 0) {
#pragma unroll
      for (int jj = 0; jj < DN_CHUNK; ++jj) {
        const int j = c0 + jj;
        if (j >= nexp) break;
        const bool shared_j = j >= a.topk;
        float wt = 0.f;
        if (s_base[j]) wt = shared_j ? a.sh_gate[r] : a.wts[r * a.topk + j];
        if (shared_j) {
          // shared expert with the reference's bf16 roundings: lin(h, D) -> bf16, then sigmoid-gate * sh -> bf16
          // (model/layers.py:398-402); sh_gate already holds bf16(sigmoid(bf16(x . g)))
          shv = round_bf16(wt * round_bf16(d[jj]));
        } else {
          const float o = d[jj] * wt;   // acc * w, kernels/moe_gemv_affine.py:96-97
          acc = (j == 0) ? o : acc + o;   // rank order, kernels/moe_gemv_affine.py:108-109
          if (a.o_buf) a.o_buf[(r * a.topk + j) * H + m] = o;
        }
      }
    }
  }
  if (lane == 0) {
    a.out[r * H + m] = acc;
    if (a.y) a.y[r * H + m] = f32_to_bf16(round_bf16(acc) + shv);   // routed.to(bf16) + sh
  }
}

// ------------------------------------------------------------------ grouped path (rows >= 3)
// Routed entries that chose the same expert form a group (the shared expert's rows form one more); a group's
// entries are cut, in entry order, into runs of GRP_TOK, and the CTA of entry p computes the run that starts
// at p against ONE staged copy of the expert's slice (CTAs of other entries exit at once). The weights of an
// expert chosen by several rows are read once per layer instead of once per row. Every (entry, output) value
// is the op sequence of the per-row kernels above, and the rank-order sum moves to its own small kernel
// (the reference's _rank_sum), so the grouped path equals the per-row path bit for bit.
constexpr int GRP_TOK = 8;      // entries one grouped down CTA computes
constexpr int GU_RUN = 4;       // entries one grouped gate_up CTA computes (their activations staged per CTA)
constexpr int GRP_MAX = 1024;   // routed entries (rows * topk) the grouped path takes
constexpr int GD_ROWS = 64;     // hidden rows per grouped down CTA (eight per warp)

// Warp-wide: the entries of the run that starts at routed entry p (none when p does not start a run), in
// entry order, into s_list; returns their count.
SSB_DEV int group_run(const int32_t* s_ids, int n_routed, int p, int* s_list, int lane, int run) {
  const int e = s_ids[p];
  int occ = 0;
  for (int q0 = 0; q0 < p; q0 += 32) {
    const int q = q0 + lane;
    occ += __popc(__ballot_sync(0xFFFFFFFFu, q < p && s_ids[q] == e));
  }
  if (occ % run) return 0;
  int n = 0;
  for (int q0 = p; q0 < n_routed && n < run; q0 += 32) {
    const int q = q0 + lane;
    const bool m = q < n_routed && s_ids[q] == e;
    const unsigned b = __ballot_sync(0xFFFFFFFFu, m);
    const int before = __popc(b & ((1u << lane) - 1u));
    if (m && n + before < run) s_list[n + before] = q;
    n += __popc(b);
  }
  return n < run ? n : run;
}

template <int NUX>
__global__ void __launch_bounds__(GU_WARPS * 32) k_dec_gate_up_g(DecodeArgs a) {
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ uint64_t bar;
  __shared__ const uint8_t* s_base;
  __shared__ int s_list[GU_RUN];
  __shared__ int s_n;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n_routed = (int)(a.R * a.topk);
  const int p = blockIdx.y;
  const int n0 = blockIdx.x * GU_ROWS;
  const int H = a.H, gs = a.gs;
  const uint32_t wbytes = (uint32_t)GU_ROWS * H / 2, sbytes = (uint32_t)GU_ROWS * (H / gs) * 2;
  uint8_t* gw = sm;
  uint8_t* uw = gw + wbytes;
  uint8_t* gsc = uw + wbytes;
  uint8_t* gb = gsc + sbytes;
  uint8_t* usc = gb + sbytes;
  uint8_t* ub = usc + sbytes;
  int32_t* s_ids = reinterpret_cast<int32_t*>(ub + sbytes);
  XUnitS* xs = reinterpret_cast<XUnitS*>(ub + sbytes + (((size_t)n_routed * 4 + 15) & ~(size_t)15));   // [run][H/16]
  const bool is_shared = p >= n_routed;
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    s_n = 0;
    s_base = nullptr;
  }
  __syncthreads();
  auto issue = [&](const uint8_t* base) {
    mbar_expect_tx(&bar, 2 * wbytes + 4 * sbytes);
    bulk_g2s(gw, base + a.o.gw + (int64_t)n0 * H / 2, wbytes, &bar);
    bulk_g2s(uw, base + a.o.uw + (int64_t)n0 * H / 2, wbytes, &bar);
    bulk_g2s(gsc, base + a.o.gsc + (int64_t)n0 * (H / gs) * 2, sbytes, &bar);
    bulk_g2s(gb, base + a.o.gb + (int64_t)n0 * (H / gs) * 2, sbytes, &bar);
    bulk_g2s(usc, base + a.o.usc + (int64_t)n0 * (H / gs) * 2, sbytes, &bar);
    bulk_g2s(ub, base + a.o.ub + (int64_t)n0 * (H / gs) * 2, sbytes, &bar);
  };
  if (is_shared) {
    const int occ = p - n_routed;
    if (occ % a.run) return;
    if (tid == 0) {   // the shared record is static: start its copies before the wait
      const int n = (int)(a.R - occ) < a.run ? (int)(a.R - occ) : a.run;
      for (int i = 0; i < n; ++i) s_list[i] = p + i;
      s_n = n;
      s_base = a.shared_rec;
      issue(a.shared_rec);
    }
    pdl_wait();
    pdl_trigger();
  } else {
    pdl_wait();
    pdl_trigger();
    for (int q = tid; q < n_routed; q += blockDim.x) s_ids[q] = ld_cg_i32(a.ids + q);
    __syncthreads();
    if (warp == 0) {
      const int n = group_run(s_ids, n_routed, p, s_list, lane, a.run);
      if (lane == 0 && n) {
        const uint8_t* base = a.bases ? (const uint8_t*)ld_cg_i64(a.bases + p)
                                      : resolve_expert(s_ids[p], a.layer, a.map, a.map_len, a.slot_ptr, a.n_slots,
                                                       a.err);
        s_base = base;
        s_n = n;
        if (base) issue(base);
      }
    }
  }
  __syncthreads();
  const int n = s_n;
  if (n == 0) return;
  const uint8_t* base = s_base;
  if (!base) {
    for (int idx = tid; idx < n * GU_ROWS; idx += blockDim.x)
      a.h_buf[(int64_t)s_list[idx / GU_ROWS] * a.I + n0 + idx % GU_ROWS] = 0.f;
    return;
  }
  const int ng = H / gs, nunits = H / 16;
  // the run's activations in the pre-scaled per-unit form, once per CTA (every warp reads every token's units)
  for (int idx = tid; idx < n * nunits; idx += blockDim.x) {
    const int t = idx / nunits, u = idx - t * nunits;
    const int q = s_list[t];
    float x16[16];
    load_x16(a, is_shared ? q - n_routed : q / a.topk, u, x16);
    XUnit xu;
    xunit_from_f32(xu, x16);
    XUnitS& d = xs[idx];
#pragma unroll
    for (int c = 0; c < 8; ++c) d.v[c] = xu.v[c];
    d.sum = xu.sum;
  }
  __syncthreads();
  if (!mbar_wait(&bar, 0, SSB_WAIT_LIMIT)) {
    set_err(a.err, SSB_ERR_TIMEOUT);
    mbar_wait(&bar, 0, SSB_WAIT_LIMIT);
    return;
  }
  const int j0 = 2 * warp, j1 = j0 + 1;
  const uint2* g0r = reinterpret_cast<const uint2*>(gw + (size_t)j0 * H / 2);
  const uint2* u0r = reinterpret_cast<const uint2*>(uw + (size_t)j0 * H / 2);
  const uint2* g1r = reinterpret_cast<const uint2*>(gw + (size_t)j1 * H / 2);
  const uint2* u1r = reinterpret_cast<const uint2*>(uw + (size_t)j1 * H / 2);
  const uint16_t* gs16 = reinterpret_cast<const uint16_t*>(gsc);
  const uint16_t* gb16 = reinterpret_cast<const uint16_t*>(gb);
  const uint16_t* us16 = reinterpret_cast<const uint16_t*>(usc);
  const uint16_t* ub16 = reinterpret_cast<const uint16_t*>(ub);
  // each unit's codes are decoded once and met by every token of the run; per (row, token) the units are
  // accumulated in the order of the per-row kernel, so the bits are the same
  float acc[4][GU_RUN];
#pragma unroll
  for (int t = 0; t < GU_RUN; ++t) acc[0][t] = acc[1][t] = acc[2][t] = acc[3][t] = 0.f;
#pragma unroll
  for (int i = 0; i < NUX; ++i) {
    const int u = lane + 32 * i;
    if (u < nunits) {
      const int g = (u * 16) / gs;
      const WUnit dg0 = unit_decode(g0r[u]), du0 = unit_decode(u0r[u]), dg1 = unit_decode(g1r[u]),
                  du1 = unit_decode(u1r[u]);
      const float sg0 = bf16_bits(gs16[j0 * ng + g]), bg0 = bf16_bits(gb16[j0 * ng + g]);
      const float su0 = bf16_bits(us16[j0 * ng + g]), bu0 = bf16_bits(ub16[j0 * ng + g]);
      const float sg1 = bf16_bits(gs16[j1 * ng + g]), bg1 = bf16_bits(gb16[j1 * ng + g]);
      const float su1 = bf16_bits(us16[j1 * ng + g]), bu1 = bf16_bits(ub16[j1 * ng + g]);
#pragma unroll
      for (int t = 0; t < GU_RUN; ++t) {
        if (t < n) {
          const XUnitS& xt = xs[t * nunits + u];
          XUnit xu;
#pragma unroll
          for (int c = 0; c < 8; ++c) xu.v[c] = xt.v[c];
          xu.sum = xt.sum;
          acc[0][t] = unit_dot_dec(dg0, sg0, bg0, xu, acc[0][t]);
          acc[1][t] = unit_dot_dec(du0, su0, bu0, xu, acc[1][t]);
          acc[2][t] = unit_dot_dec(dg1, sg1, bg1, xu, acc[2][t]);
          acc[3][t] = unit_dot_dec(du1, su1, bu1, xu, acc[3][t]);
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < GU_RUN; ++t) {
    if (t < n) {
      float ga0 = acc[0][t], ua0 = acc[1][t], ga1 = acc[2][t], ua1 = acc[3][t];
      warp_sum4(ga0, ua0, ga1, ua1);
      if (lane < 2) {
        const float ga = lane ? ga1 : ga0, ua = lane ? ua1 : ua0;
        float h;
        if (is_shared) {
          const float gbv = round_bf16(ga), ubv = round_bf16(ua);
          h = round_bf16(round_bf16(gbv / (1.f + expf(-gbv))) * ubv);
        } else {
          h = ga / (1.f + expf(-ga)) * ua;
        }
        a.h_buf[(int64_t)s_list[t] * a.I + n0 + j0 + lane] = h;
      }
    }
  }
}

// o[entry, m] = w * (D h) for the run's entries over GD_ROWS hidden rows; the shared expert's gated value
// bf16(sh_gate * bf16(D_s h_s)) goes to out[r, m], which k_dec_rank_sum reads before overwriting it.
template <int NUI>
__global__ void __launch_bounds__(DN_WARPS * 32) k_dec_down_g(DecodeArgs a) {
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ uint64_t bar;
  __shared__ const uint8_t* s_base;
  __shared__ int s_list[GRP_TOK];
  __shared__ int s_n;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n_routed = (int)(a.R * a.topk);
  const int p = blockIdx.y;
  const int m0 = blockIdx.x * GD_ROWS;
  const int I = a.I, gs = a.gs, H = a.H;
  const int nunits = I / 16, ng = I / gs;
  const uint32_t wbytes = (uint32_t)GD_ROWS * I / 2, sbytes = (uint32_t)GD_ROWS * ng * 2;
  uint8_t* dw = sm;
  uint8_t* dsc = dw + wbytes;
  uint8_t* db = dsc + sbytes;
  XUnitS* hx = reinterpret_cast<XUnitS*>(db + sbytes);   // [GRP_TOK][nunits]
  int32_t* s_ids = reinterpret_cast<int32_t*>(hx + GRP_TOK * nunits);
  const bool is_shared = p >= n_routed;
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    s_n = 0;
    s_base = nullptr;
  }
  __syncthreads();
  auto issue = [&](const uint8_t* base) {
    mbar_expect_tx(&bar, wbytes + 2 * sbytes);
    bulk_g2s(dw, base + a.o.dw + (int64_t)m0 * I / 2, wbytes, &bar);
    bulk_g2s(dsc, base + a.o.dsc + (int64_t)m0 * ng * 2, sbytes, &bar);
    bulk_g2s(db, base + a.o.db + (int64_t)m0 * ng * 2, sbytes, &bar);
  };
  // The weights are staged before the wait on the gate_up grid: the expert ids were written before that grid
  // started, and every grid here triggers its dependents only after its own wait, so they are visible now.
  if (is_shared) {
    const int occ = p - n_routed;
    if (occ % GRP_TOK) return;
    if (tid == 0) {
      const int n = (int)(a.R - occ) < GRP_TOK ? (int)(a.R - occ) : GRP_TOK;
      for (int i = 0; i < n; ++i) s_list[i] = p + i;
      s_n = n;
      s_base = a.shared_rec;
      issue(a.shared_rec);
    }
  } else {
    for (int q = tid; q < n_routed; q += blockDim.x) s_ids[q] = ld_cg_i32(a.ids + q);
    __syncthreads();
    if (warp == 0) {
      const int n = group_run(s_ids, n_routed, p, s_list, lane, GRP_TOK);
      if (lane == 0 && n) {
        const uint8_t* base = a.bases ? (const uint8_t*)ld_cg_i64(a.bases + p)
                                      : resolve_expert(s_ids[p], a.layer, a.map, a.map_len, a.slot_ptr, a.n_slots,
                                                       nullptr);
        s_base = base;
        s_n = n;
        if (base) issue(base);
      }
    }
  }
  __syncthreads();
  const int n = s_n;
  if (n == 0) return;
  pdl_wait();
  pdl_trigger();
  const uint8_t* base = s_base;
  if (!base) {   // an unmapped routed expert contributes zero
    for (int idx = tid; idx < n * GD_ROWS; idx += blockDim.x)
      a.o_buf[(int64_t)s_list[idx / GD_ROWS] * H + m0 + idx % GD_ROWS] = 0.f;
    return;
  }
  // the run's activations h in the pre-scaled per-unit form (h was written by the gate_up grid)
  for (int idx = tid; idx < n * nunits; idx += DN_WARPS * 32) {
    const int t = idx / nunits, u = idx - t * nunits;
    const float4* hp = reinterpret_cast<const float4*>(a.h_buf + (int64_t)s_list[t] * I + u * 16);
    float h16[16];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 v = __ldcg(hp + q);
      h16[4 * q] = v.x;
      h16[4 * q + 1] = v.y;
      h16[4 * q + 2] = v.z;
      h16[4 * q + 3] = v.w;
    }
    XUnit xu;
    xunit_from_f32(xu, h16);
    XUnitS& d = hx[idx];
#pragma unroll
    for (int q = 0; q < 8; ++q) d.v[q] = xu.v[q];
    d.sum = xu.sum;
  }
  __syncthreads();
  if (!mbar_wait(&bar, 0, SSB_WAIT_LIMIT)) {
    if (tid == 0) set_err(a.err, SSB_ERR_TIMEOUT);
    mbar_wait(&bar, 0, SSB_WAIT_LIMIT);
    return;
  }
  constexpr int RPW = GD_ROWS / DN_WARPS;
  for (int rr = 0; rr < RPW; ++rr) {
    const int row = warp * RPW + rr;
    const int m = m0 + row;
    const uint2* wr = reinterpret_cast<const uint2*>(dw + (size_t)row * I / 2);
    const uint16_t* sr = reinterpret_cast<const uint16_t*>(dsc) + row * ng;
    const uint16_t* br = reinterpret_cast<const uint16_t*>(db) + row * ng;
    // each unit's codes decoded once for all of the run's tokens; per token the units keep their order
    float d[GRP_TOK];
#pragma unroll
    for (int t = 0; t < GRP_TOK; ++t) d[t] = 0.f;
#pragma unroll
    for (int i = 0; i < NUI; ++i) {
      const int u = lane + 32 * i;
      if (u < nunits) {
        const int g = (u * 16) / gs;
        const WUnit dw = unit_decode(wr[u]);
        const float sv = bf16_bits(sr[g]), bv = bf16_bits(br[g]);
#pragma unroll
        for (int t = 0; t < GRP_TOK; ++t) {
          if (t < n) {
            const XUnitS& xs = hx[t * nunits + u];
            XUnit xu;
#pragma unroll
            for (int q = 0; q < 8; ++q) xu.v[q] = xs.v[q];
            xu.sum = xs.sum;
            d[t] = unit_dot_dec(dw, sv, bv, xu, d[t]);
          }
        }
      }
    }
    warp_sum4(d[0], d[1], d[2], d[3]);
    warp_sum4(d[4], d[5], d[6], d[7]);
    float v = d[0];
#pragma unroll
    for (int t = 1; t < GRP_TOK; ++t) v = lane == t ? d[t] : v;
    if (lane < n) {
      const int q = s_list[lane];
      if (is_shared) {
        const int64_t r = q - n_routed;
        a.out[r * H + m] = round_bf16(a.sh_gate[r] * round_bf16(v));
      } else {
        a.o_buf[(int64_t)q * H + m] = v * a.wts[q];   // acc * w, kernels/moe_gemv_affine.py:96-97
      }
    }
  }
}

// out[r, :] = o[r, 0, :] + o[r, 1, :] + ... in rank order (kernels/moe_gemv_affine.py:100-110); with the
// shared expert, y = bf16(bf16(out) + sh) where sh is the value k_dec_down_g left in out.
__global__ void __launch_bounds__(256) k_dec_rank_sum(DecodeArgs a) {
  pdl_wait();
  pdl_trigger();
  const int64_t i4 = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (i4 * 4 >= a.R * a.H) return;
  const int64_t r = i4 * 4 / a.H, m = i4 * 4 - r * a.H;
  const float4* o = reinterpret_cast<const float4*>(a.o_buf + r * a.topk * a.H + m);
  const int64_t st4 = a.H / 4;
  float4 acc = __ldcg(o);
  for (int j = 1; j < a.topk; ++j) {
    const float4 v = __ldcg(o + j * st4);
    acc.x = acc.x + v.x;
    acc.y = acc.y + v.y;
    acc.z = acc.z + v.z;
    acc.w = acc.w + v.w;
  }
  float4* out = reinterpret_cast<float4*>(a.out + r * a.H + m);
  if (a.y) {
    const float4 sh = __ldcg(out);
    uint2 yv;
    yv.x = (uint32_t)f32_to_bf16(round_bf16(acc.x) + sh.x) | ((uint32_t)f32_to_bf16(round_bf16(acc.y) + sh.y) << 16);
    yv.y = (uint32_t)f32_to_bf16(round_bf16(acc.z) + sh.z) | ((uint32_t)f32_to_bf16(round_bf16(acc.w) + sh.w) << 16);
    *reinterpret_cast<uint2*>(a.y + r * a.H + m) = yv;
  }
  *out = acc;
}

int launch_decode_grouped(DecodeArgs a, cudaStream_t st, bool pdl) {
  const int nux = (a.H / 16 + 31) / 32;
  const int nui = (a.I / 16 + 31) / 32;
  const int64_t n_routed = a.R * a.topk;
  const int64_t pairs = n_routed + (a.shared_rec ? a.R : 0);
  const size_t ids_bytes = ((size_t)n_routed * 4 + 15) & ~(size_t)15;
  const size_t gu_fixed = (size_t)2 * GU_ROWS * a.H / 2 + (size_t)4 * GU_ROWS * (a.H / a.gs) * 2 + ids_bytes;
  // entries per gate_up run: as many as fit with their activations staged in shared memory
  const size_t xs_unit = (size_t)(a.H / 16) * sizeof(XUnitS);
  a.run = GU_RUN;
  while (a.run > 1 && gu_fixed + (size_t)a.run * xs_unit > 100 * 1024) a.run /= 2;   // two CTAs per SM
  const size_t gu_smem = gu_fixed + (size_t)a.run * xs_unit;
  const size_t dn_smem = (size_t)GD_ROWS * a.I / 2 + (size_t)2 * GD_ROWS * (a.I / a.gs) * 2 +
                         (size_t)GRP_TOK * (a.I / 16) * sizeof(XUnitS) + ids_bytes;
  if (gu_smem > 200 * 1024 || dn_smem > 200 * 1024) return SSB_EUNSUPPORTED;
  void (*gu)(DecodeArgs) = nullptr;
  void (*dn)(DecodeArgs) = nullptr;
  switch (nux) {
    case 1: gu = k_dec_gate_up_g<1>; break;
    case 2: gu = k_dec_gate_up_g<2>; break;
    case 3: gu = k_dec_gate_up_g<3>; break;
    case 4: gu = k_dec_gate_up_g<4>; break;
    case 5: gu = k_dec_gate_up_g<5>; break;
    case 6: gu = k_dec_gate_up_g<6>; break;
    case 8: gu = k_dec_gate_up_g<8>; break;
    default: return SSB_EUNSUPPORTED;
  }
  switch (nui) {
    case 1: dn = k_dec_down_g<1>; break;
    case 2: dn = k_dec_down_g<2>; break;
    case 3: dn = k_dec_down_g<3>; break;
    case 4: dn = k_dec_down_g<4>; break;
    default: return SSB_EUNSUPPORTED;
  }
  cudaFuncSetAttribute(gu, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gu_smem);
  cudaFuncSetAttribute(dn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dn_smem);
  ssb_note_smem("moe_gate_up_grouped", gu, gu_smem);
  ssb_note_smem("moe_down_grouped", dn, dn_smem);
  int rc = ssb_launch(gu, dim3(a.I / GU_ROWS, (unsigned)pairs), dim3(GU_WARPS * 32), gu_smem, st, pdl, a);
  if (rc) return rc;
  rc = ssb_launch(dn, dim3(a.H / GD_ROWS, (unsigned)pairs), dim3(DN_WARPS * 32), dn_smem, st, true, a);
  if (rc) return rc;
  const int64_t n4 = a.R * a.H / 4;
  return ssb_launch(k_dec_rank_sum, dim3((unsigned)((n4 + 255) / 256)), dim3(256), 0, st, true, a);
}

int launch_decode(DecodeArgs a, cudaStream_t st, bool pdl) {
  if (a.R >= 3 && a.o_buf && a.R * a.topk <= GRP_MAX && a.H % GD_ROWS == 0 && a.I % 16 == 0) {
    const int rc = launch_decode_grouped(a, st, pdl);
    if (rc != SSB_EUNSUPPORTED) return rc;
  }
  const int nux = (a.H / 16 + 31) / 32;
  const int nui = (a.I / 16 + 31) / 32;
  const int nexp = a.topk + (a.shared_rec ? 1 : 0);
  const int64_t pairs = a.R * a.topk + (a.shared_rec ? a.R : 0);
  const size_t gu_smem = (size_t)2 * GU_ROWS * a.H / 2 + (size_t)4 * GU_ROWS * (a.H / a.gs) * 2;
  const size_t dn_smem = (size_t)nexp * ((size_t)DN_ROWS * a.I / 2 + (size_t)2 * DN_ROWS * (a.I / a.gs) * 2 +
                                         (size_t)a.I * 4 + (size_t)(a.I / 16) * sizeof(XUnitS));
  if (gu_smem > 200 * 1024 || dn_smem > 200 * 1024) return SSB_EUNSUPPORTED;
  if (pairs > 65535 || a.R > 65535) return SSB_EUNSUPPORTED;
  void (*gu)(DecodeArgs) = nullptr;
  void (*dn)(DecodeArgs) = nullptr;
  switch (nux) {
    case 1: gu = k_dec_gate_up<1>; break;
    case 2: gu = k_dec_gate_up<2>; break;
    case 3: gu = k_dec_gate_up<3>; break;
    case 4: gu = k_dec_gate_up<4>; break;
    case 5: gu = k_dec_gate_up<5>; break;
    case 6: gu = k_dec_gate_up<6>; break;
    case 8: gu = k_dec_gate_up<8>; break;
    default: return SSB_EUNSUPPORTED;
  }
  switch (nui) {
    case 1: dn = k_dec_down<1>; break;
    case 2: dn = k_dec_down<2>; break;
    case 3: dn = k_dec_down<3>; break;
    case 4: dn = k_dec_down<4>; break;
    default: return SSB_EUNSUPPORTED;
  }
  cudaFuncSetAttribute(gu, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gu_smem);
  cudaFuncSetAttribute(dn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dn_smem);
  ssb_note_smem("moe_gate_up", gu, gu_smem);
  ssb_note_smem("moe_down", dn, dn_smem);
  int rc = ssb_launch(gu, dim3(a.I / GU_ROWS, (unsigned)pairs), dim3(GU_WARPS * 32), gu_smem, st, pdl, a);
  if (rc) return rc;
  return ssb_launch(dn, dim3(a.H / DN_ROWS, (unsigned)a.R), dim3(DN_WARPS * 32), dn_smem, st, true, a);
}

int check_shape(int64_t rows, int topk, int hidden, int inter) {
  if (rows < 0 || topk < 1 || topk > 32) return SSB_EINVAL;
  if (hidden % 512 || hidden <= 0 || hidden > 8192) return SSB_EUNSUPPORTED;
  if (inter % GU_ROWS || inter <= 0 || inter > 2048 || inter % 64) return SSB_EUNSUPPORTED;
  if (hidden % DN_ROWS) return SSB_EUNSUPPORTED;
  return SSB_OK;
}

}  // namespace

extern "C" int ssb_moe_decode(const void* x, int32_t x_dtype, const int32_t* expert_ids, const float* weights,
                              int64_t rows, int32_t topk, int32_t hidden, int32_t inter, int32_t layer,
                              const int32_t* map_t, int64_t map_len, const int64_t* slot_ptr_t, int64_t n_slots,
                              float* h_buf, float* o_buf, float* out, int32_t* err, void* stream) {
  int rc = check_shape(rows, topk, hidden, inter);
  if (rc) return rc;
  SSB_CHECK_ARG(x_dtype == SSB_BF16 || x_dtype == SSB_F32);
  SSB_CHECK_ARG(layer >= 0 && map_len >= 0 && n_slots >= 0);
  if (rows == 0) return SSB_OK;
  SSB_CHECK_ARG(x && expert_ids && weights && map_t && slot_ptr_t && h_buf && out);
  DecodeArgs a{};
  a.x = x;
  a.x_f32 = x_dtype == SSB_F32;
  a.ids = expert_ids;
  a.wts = weights;
  a.R = rows;
  a.topk = topk;
  a.H = hidden;
  a.I = inter;
  a.gs = 64;
  a.layer = layer;
  a.map = map_t;
  a.map_len = map_len;
  a.slot_ptr = slot_ptr_t;
  a.n_slots = n_slots;
  a.o = rec_offsets(hidden, inter, 64);
  a.h_buf = h_buf;
  a.o_buf = o_buf;
  a.out = out;
  a.err = err;
  return launch_decode(a, (cudaStream_t)stream, true);
}

extern "C" int ssb_moe_decode_layer(const uint16_t* x, const int32_t* expert_ids, const float* weights, int64_t rows,
                                    int32_t topk, int32_t hidden, int32_t inter, int32_t layer, const int32_t* map_t,
                                    int64_t map_len, const int64_t* slot_ptr_t, int64_t n_slots,
                                    const void* shared_record, const float* sh_gate, const int64_t* expert_base,
                                    float* h_buf, float* o_buf, float* out, uint16_t* y, int32_t flags,
                                    int32_t* err, void* stream) {
  int rc = check_shape(rows, topk, hidden, inter);
  if (rc) return rc;
  SSB_CHECK_ARG(layer >= 0 && map_len >= 0 && n_slots >= 0);
  if (rows == 0) return SSB_OK;
  SSB_CHECK_ARG(x && expert_ids && weights && map_t && slot_ptr_t && h_buf && out && shared_record && sh_gate && y);
  SSB_CHECK_ARG(((uintptr_t)shared_record & 15) == 0);
  DecodeArgs a{};
  a.x = x;
  a.x_f32 = 0;
  a.ids = expert_ids;
  a.wts = weights;
  a.R = rows;
  a.topk = topk;
  a.H = hidden;
  a.I = inter;
  a.gs = 64;
  a.layer = layer;
  a.map = map_t;
  a.map_len = map_len;
  a.slot_ptr = slot_ptr_t;
  a.n_slots = n_slots;
  a.shared_rec = (const uint8_t*)shared_record;
  a.sh_gate = sh_gate;
  a.bases = expert_base;
  a.o = rec_offsets(hidden, inter, 64);
  a.h_buf = h_buf;
  a.o_buf = o_buf;
  a.out = out;
  a.y = y;
  a.err = err;
  return launch_decode(a, (cudaStream_t)stream, (flags & SSB_DECODE_PDL) != 0);
}
