// Expert-parallel prefill: the device side of dispatch and combine.
//
// Rank g of G owns the experts [g * epr, (g + 1) * epr). A token is sent once to every rank that owns at least
// one of its top-k experts (deduplicated per (token, rank)), with k metadata words per row: the local expert
// of each rank-k choice that rank owns (-1 otherwise) and the routing weight. The receiving rank runs the
// grouped GEMMs on what it received and sends back, per received row, either the fp32 partial sum of its
// entries in rank-k order or (exact mode) the k per-entry rows, so that the home rank can sum every token's
// expert outputs in router-rank order bit for bit like the one-GPU layer (kernels/fused_moe_affine.py:164-172).
//
// Send order: rows for destination 0 first, then 1, ...; inside a destination by ascending token. The plan runs
// on a cluster of CTAs (one CTA when clusters are unavailable): each CTA owns a contiguous token range and each
// of its threads a contiguous chunk of it (the next token's choices loaded while the current one is handled);
// per-destination counts are block-scanned, the CTAs exchange their totals through distributed shared memory,
// and a second pass writes every row to its final position, so the order is deterministic.
#include <cooperative_groups.h>
#include <cub/block/block_scan.cuh>

#include "common.cuh"
#include "registry.h"

namespace {

constexpr int EP_MAXG = 8;     // ranks (one node of B200s)
constexpr int PLAN_THREADS = 512;

// Expert placement: contiguous (rank e / epr, local e % epr) or strided (rank e % G, local e / G).
struct Placement {
  int epr, G, strided;
  SSB_DEV bool valid(int e) const { return e >= 0 && e < epr * G; }
  SSB_DEV int rank(int e) const { return strided ? e % G : e / epr; }
  SSB_DEV int local(int e) const { return strided ? e / G : e % epr; }
};

struct Counts {
  int c[2 * EP_MAXG];   // rows, then entries, per destination
};
struct CountsSum {
  SSB_DEV Counts operator()(const Counts& a, const Counts& b) const {
    Counts r;
#pragma unroll
    for (int d = 0; d < 2 * EP_MAXG; ++d) r.c[d] = a.c[d] + b.c[d];
    return r;
  }
};

// One token's choices in registers (k <= 15): the ids, and (with_w) the weights.
struct TokChoices {
  int e[16];
  float w[16];
};
template <bool WITH_W>
SSB_DEV void load_choices(const int32_t* ids, const float* w, int64_t t, int k, TokChoices& c) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    c.e[j] = j < k ? __ldcg(ids + t * k + j) : -1;
    if (WITH_W) c.w[j] = j < k ? __ldcg(w + t * k + j) : 0.f;
  }
}
// Per-destination entry counts (4 bits each; k <= 15 entries per destination fit) and the destination mask.
SSB_DEV uint32_t choice_dests(const TokChoices& c, int k, const Placement& pl, uint64_t* ecnt, int32_t* err) {
  uint32_t m = 0;
  uint64_t n = 0;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    if (j >= k) break;
    const int e = c.e[j];
    if (!pl.valid(e)) {
      set_err(err, SSB_ERR_EXPERT_RANGE);
      continue;
    }
    const int d = pl.rank(e);
    m |= 1u << d;
    n += 1ull << (4 * d);
  }
  *ecnt = n;
  return m;
}

// Both passes walk a thread's token chunk with the next token's choices loaded while the current one is handled.
__global__ void __launch_bounds__(PLAN_THREADS) k_ep_plan(const int32_t* __restrict__ ids,
                                                          const float* __restrict__ w, int64_t T, int k,
                                                          Placement pl, int32_t* __restrict__ dest_count,
                                                          int32_t* __restrict__ send_token,
                                                          int32_t* __restrict__ send_meta,
                                                          int32_t* __restrict__ tok_slot,
                                                          int32_t* __restrict__ tok_entry, int32_t* err) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  using Scan = cub::BlockScan<Counts, PLAN_THREADS>;
  __shared__ typename Scan::TempStorage tmp;
  __shared__ int s_off[EP_MAXG];
  __shared__ int s_tot[2 * EP_MAXG], s_before[2 * EP_MAXG], s_grand[2 * EP_MAXG];
  pdl_wait();
  pdl_trigger();
  const int tid = threadIdx.x, G = pl.G;
  const int crank = (int)cluster.block_rank(), csize = (int)cluster.num_blocks();
  const int mw = 2 * k + 2;
  const int64_t cchunk = (T + csize - 1) / csize;
  const int64_t c0 = (int64_t)crank * cchunk < T ? (int64_t)crank * cchunk : T;
  const int64_t c1 = c0 + cchunk < T ? c0 + cchunk : T;
  const int64_t chunk = (c1 - c0 + PLAN_THREADS - 1) / PLAN_THREADS;
  const int64_t t0 = c0 + tid * chunk < c1 ? c0 + tid * chunk : c1, t1 = t0 + chunk < c1 ? t0 + chunk : c1;
  Counts mine;
#pragma unroll
  for (int d = 0; d < 2 * EP_MAXG; ++d) mine.c[d] = 0;
  {
    TokChoices cur, nxt;
    if (t0 < t1) load_choices<false>(ids, w, t0, k, cur);
    for (int64_t t = t0; t < t1; ++t) {
      if (t + 1 < t1) load_choices<false>(ids, w, t + 1, k, nxt);
      uint64_t ec;
      const uint32_t m = choice_dests(cur, k, pl, &ec, nullptr);
#pragma unroll
      for (int d = 0; d < EP_MAXG; ++d) {
        mine.c[d] += (m >> d) & 1u;
        mine.c[EP_MAXG + d] += (int)((ec >> (4 * d)) & 15u);
      }
      cur = nxt;
    }
  }
  Counts excl, total, zero;
#pragma unroll
  for (int d = 0; d < 2 * EP_MAXG; ++d) zero.c[d] = 0;
  Scan(tmp).ExclusiveScan(mine, excl, zero, CountsSum(), total);
  if (tid == 0) {
#pragma unroll
    for (int d = 0; d < 2 * EP_MAXG; ++d) s_tot[d] = total.c[d];
  }
  cluster.sync();   // every CTA's totals are complete
  if (tid < 2 * EP_MAXG) {   // rows and entries of the earlier CTAs, and of all of them
    int b = 0, g = 0;
    for (int c = 0; c < csize; ++c) {
      const int v = *cluster.map_shared_rank(s_tot + tid, c);
      b += c < crank ? v : 0;
      g += v;
    }
    s_before[tid] = b;
    s_grand[tid] = g;
  }
  cluster.sync();   // no CTA leaves while another may still read its totals
  if (tid == 0) {
    int off = 0;
    for (int d = 0; d < G; ++d) {
      s_off[d] = off;
      if (crank == 0) {
        dest_count[2 * d] = s_grand[d];
        dest_count[2 * d + 1] = s_grand[EP_MAXG + d];
      }
      off += s_grand[d];
    }
  }
  __syncthreads();
  int pos[EP_MAXG], epos[EP_MAXG];
#pragma unroll
  for (int d = 0; d < EP_MAXG; ++d) {
    pos[d] = d < G ? s_off[d] + s_before[d] + excl.c[d] : 0;
    epos[d] = s_before[EP_MAXG + d] + excl.c[EP_MAXG + d];
  }
  TokChoices cur, nxt;
  if (t0 < t1) load_choices<true>(ids, w, t0, k, cur);
  for (int64_t t = t0; t < t1; ++t) {
    if (t + 1 < t1) load_choices<true>(ids, w, t + 1, k, nxt);
    uint64_t ec;
    const uint32_t m = choice_dests(cur, k, pl, &ec, err);
#pragma unroll
    for (int d = 0; d < EP_MAXG; ++d) {
      if (d >= G) break;
      if (!((m >> d) & 1u)) {
        tok_slot[t * G + d] = -1;
        tok_entry[t * G + d] = -1;
        continue;
      }
      const int p = pos[d]++;
      const int n = (int)((ec >> (4 * d)) & 15u);
      tok_slot[t * G + d] = p;
      tok_entry[t * G + d] = epos[d];
      send_token[p] = (int32_t)t;
      int32_t* meta = send_meta + (int64_t)p * mw;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        if (j >= k) break;
        const int e = cur.e[j];
        const bool here = pl.valid(e) && pl.rank(e) == d;
        meta[j] = here ? pl.local(e) : -1;
        meta[k + j] = here ? __float_as_int(cur.w[j]) : 0;
      }
      meta[2 * k] = epos[d];
      meta[2 * k + 1] = n;
      epos[d] += n;
    }
    cur = nxt;
  }
}

int plan_cluster_size() {   // 16 CTAs when the device runs such clusters, else 8, else 1
  static int cl = -1;
  if (cl < 0) {
    cl = 1;
    if (cudaFuncSetAttribute(k_ep_plan, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
      (void)cudaGetLastError();
    for (int want : {16, 8}) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(want);
      cfg.blockDim = dim3(PLAN_THREADS);
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = want;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, k_ep_plan, &cfg) == cudaSuccess && n >= 1) {
        cl = want;
        break;
      }
      (void)cudaGetLastError();
    }
  }
  return cl;
}

// dst[i, :] = src[idx[i], :] for rows of `row_bytes` (a multiple of 16) bytes.
__global__ void __launch_bounds__(256) k_gather_rows(const uint4* __restrict__ src, int64_t src_rows,
                                                     const int32_t* __restrict__ idx, int64_t n, int64_t row_vecs,
                                                     uint4* __restrict__ dst, int32_t* err) {
  pdl_wait();
  pdl_trigger();
  const int64_t total = n * row_vecs;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < total; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = v / row_vecs, c = v - r * row_vecs;
    const int64_t s = __ldcg(idx + r);
    if (s < 0 || s >= src_rows) {
      if (c == 0) set_err(err, SSB_ERR_EXPERT_RANGE);
      dst[v] = make_uint4(0, 0, 0, 0);
      continue;
    }
    dst[v] = __ldcs(src + s * row_vecs + c);
  }
}

// Received rows -> the grouped GEMM's compacted entry arrays. Rows from source s occupy
// [src_row_off[s], src_row_off[s + 1]) and their entries [src_entry_off[s], src_entry_off[s + 1]); entry p of
// row r is (local expert, row r, weight), entries of a row contiguous in rank-k order.
__global__ void k_ep_unpack(const int32_t* __restrict__ meta, int64_t n, int k, const int32_t* __restrict__ src_row_off,
                            const int64_t* __restrict__ src_entry_off, int G, int64_t n_entries,
                            int32_t* __restrict__ row_expert, int32_t* __restrict__ row_token,
                            float* __restrict__ row_weight, int64_t* __restrict__ row_e0, int32_t* __restrict__ row_cnt,
                            int32_t* err) {
  pdl_wait();
  pdl_trigger();
  const int mw = 2 * k + 2;
  for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n; r += (int64_t)gridDim.x * blockDim.x) {
    int s = 0;
    while (s + 1 < G && r >= __ldg(src_row_off + s + 1)) ++s;
    const int32_t* m = meta + r * mw;
    const int64_t e0 = __ldg(src_entry_off + s) + __ldcg(m + 2 * k);
    const int cnt = __ldcg(m + 2 * k + 1);
    row_e0[r] = e0;
    row_cnt[r] = cnt;
    int64_t p = e0;
    for (int j = 0; j < k; ++j) {
      const int le = __ldcg(m + j);
      if (le < 0) continue;
      if (p >= e0 + cnt || p >= n_entries) {
        set_err(err, SSB_ERR_EXPERT_RANGE);
        break;
      }
      row_expert[p] = le;
      row_token[p] = (int32_t)r;
      row_weight[p] = __int_as_float(__ldcg(m + k + j));
      ++p;
    }
  }
}

// partial[r, :] = rows[e0] + rows[e0 + 1] + ... + rows[e0 + cnt - 1] (e0 = row_e0[r]), sequential fp32; stored as
// fp32 (float4) or rounded to bf16 (uint2: four bf16, round to nearest even) for a half-size return.
SSB_DEV void store4(float4* p, float4 v) { *p = v; }
SSB_DEV void store4(uint2* p, float4 v) {
  *p = make_uint2((uint32_t)f32_to_bf16(v.x) | ((uint32_t)f32_to_bf16(v.y) << 16),
                  (uint32_t)f32_to_bf16(v.z) | ((uint32_t)f32_to_bf16(v.w) << 16));
}
SSB_DEV float4 load4(const float4* p) { return __ldcs(p); }
SSB_DEV float4 load4(const uint2* p) {
  const uint2 b = __ldcs(p);
  return make_float4(bf16_lo(b.x), bf16_hi(b.x), bf16_lo(b.y), bf16_hi(b.y));
}

template <typename P4>
__global__ void __launch_bounds__(256) k_combine_rows(const float4* __restrict__ rows, const int64_t* __restrict__ row_e0,
                                                      const int32_t* __restrict__ row_cnt, int64_t n, int64_t h4,
                                                      P4* __restrict__ partial) {
  pdl_wait();
  pdl_trigger();
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < n * h4; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = v / h4, c = v - r * h4;
    const int64_t e0 = __ldcg(row_e0 + r);
    const int cnt = __ldcg(row_cnt + r);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i = 0; i < cnt; ++i) {
      const float4 x = __ldcs(rows + (e0 + i) * h4 + c);
      acc.x += x.x;
      acc.y += x.y;
      acc.z += x.z;
      acc.w += x.w;
    }
    store4(partial + v, acc);
  }
}

// Home-side combine. exact == 0: routed[t] = sum over destinations d (ascending) holding t of ret[tok_slot[t, d]]
// (the partial row that d returned for t); exact != 0: routed[t] = sum over j (router rank order) of the entry
// row ret[ret_entry_off[d] + tok_entry[t, d] + i], d the rank of ids[t, j] and i the count of t's earlier
// choices on d. out (fp32 [T, H], nullable) gets routed; y (nullable) = bf16(bf16(routed) + bf16(sh)).
template <typename R4>
__global__ void __launch_bounds__(256) k_ep_combine(const R4* __restrict__ ret, const int32_t* __restrict__ tok_slot,
                                                    const int32_t* __restrict__ tok_entry,
                                                    const int64_t* __restrict__ ret_entry_off,
                                                    const int32_t* __restrict__ ids, int64_t T, int k, Placement pl,
                                                    int exact, int64_t h4, const float4* __restrict__ sh,
                                                    float4* __restrict__ out, uint2* __restrict__ y) {
  pdl_wait();
  pdl_trigger();
  const int G = pl.G;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < T * h4; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = v / h4, c = v - t * h4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (exact) {
      uint64_t seen = 0;   // 4-bit count of t's choices already taken per destination
      for (int j = 0; j < k; ++j) {
        const int e = __ldcg(ids + t * k + j);
        if (!pl.valid(e)) continue;
        const int d = pl.rank(e);
        const int i = (int)((seen >> (4 * d)) & 15u);
        seen += 1ull << (4 * d);
        const int64_t row = __ldg(ret_entry_off + d) + __ldcg(tok_entry + t * G + d) + i;
        const float4 x = load4(ret + row * h4 + c);
        acc.x += x.x;
        acc.y += x.y;
        acc.z += x.z;
        acc.w += x.w;
      }
    } else {
      for (int d = 0; d < G; ++d) {
        const int sl = __ldcg(tok_slot + t * G + d);
        if (sl < 0) continue;
        const float4 x = load4(ret + (int64_t)sl * h4 + c);
        acc.x += x.x;
        acc.y += x.y;
        acc.z += x.z;
        acc.w += x.w;
      }
    }
    if (out) out[v] = acc;
    if (y) {
      const float4 s4 = sh ? __ldcs(sh + v) : make_float4(0.f, 0.f, 0.f, 0.f);
      const float a0 = round_bf16(round_bf16(acc.x) + round_bf16(s4.x));
      const float a1 = round_bf16(round_bf16(acc.y) + round_bf16(s4.y));
      const float a2 = round_bf16(round_bf16(acc.z) + round_bf16(s4.z));
      const float a3 = round_bf16(round_bf16(acc.w) + round_bf16(s4.w));
      y[v] = make_uint2((uint32_t)f32_to_bf16(a0) | ((uint32_t)f32_to_bf16(a1) << 16),
                        (uint32_t)f32_to_bf16(a2) | ((uint32_t)f32_to_bf16(a3) << 16));
    }
  }
}

int grid_for(int64_t work, int threads) {
  int64_t g = (work + threads - 1) / threads;
  return (int)(g < 148 * 16 ? (g < 1 ? 1 : g) : 148 * 16);
}

bool placement_ok(int32_t epr, int32_t n_ranks, int32_t strided) {
  return epr >= 1 && n_ranks >= 1 && n_ranks <= EP_MAXG && (strided == 0 || strided == 1);
}

}  // namespace

extern "C" int ssb_ep_plan(const int32_t* ids, const float* w, int64_t tokens, int32_t k, int32_t experts_per_rank,
                           int32_t n_ranks, int32_t strided, int32_t* dest_count, int32_t* send_token,
                           int32_t* send_meta, int32_t* tok_slot, int32_t* tok_entry, int32_t* err, void* stream) {
  SSB_CHECK_ARG(tokens >= 0 && k >= 1 && k <= 15 && placement_ok(experts_per_rank, n_ranks, strided));
  if (tokens == 0) {   // an empty part still reports its (zero) counts; its other outputs are empty
    SSB_CHECK_ARG(dest_count);
    return (int)cudaMemsetAsync(dest_count, 0, sizeof(int32_t) * 2 * (size_t)n_ranks, (cudaStream_t)stream);
  }
  SSB_CHECK_ARG(ids && w && dest_count && send_token && send_meta && tok_slot && tok_entry);
  SSB_CHECK_ARG(tokens <= 0x7fffffffLL / k);
  ssb_note_smem("ep_plan", k_ep_plan, 0);
  const Placement pl{experts_per_rank, n_ranks, strided};
  const int cl = tokens >= 4096 ? plan_cluster_size() : 1;
  if (cl > 1) {   // one CTA per 1/cl of the tokens
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cl);
    cfg.blockDim = dim3(PLAN_THREADS);
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = cl;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 2;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_ep_plan, ids, w, tokens, k, pl, dest_count, send_token, send_meta,
                                       tok_slot, tok_entry, err);
    if (e == cudaSuccess) return SSB_OK;
    (void)cudaGetLastError();   // fall back to one CTA
  }
  return ssb_launch(k_ep_plan, dim3(1), dim3(PLAN_THREADS), 0, (cudaStream_t)stream, true, ids, w, tokens, k, pl,
                    dest_count, send_token, send_meta, tok_slot, tok_entry, err);
}

extern "C" int ssb_gather_rows(const void* src, int64_t src_rows, const int32_t* idx, int64_t n, int64_t row_bytes,
                               void* dst, int32_t* err, void* stream) {
  SSB_CHECK_ARG(n >= 0 && src_rows >= 0 && row_bytes > 0 && row_bytes % 16 == 0);
  if (n == 0) return SSB_OK;
  SSB_CHECK_ARG(src && idx && dst && ((((uintptr_t)src) | ((uintptr_t)dst)) & 15) == 0);
  const int64_t vecs = row_bytes / 16;
  return ssb_launch(k_gather_rows, dim3(grid_for(n * vecs, 256)), dim3(256), 0, (cudaStream_t)stream, true,
                    (const uint4*)src, src_rows, idx, n, vecs, (uint4*)dst, err);
}

extern "C" int ssb_ep_unpack(const int32_t* meta, int64_t rows, int32_t k, const int32_t* src_row_off,
                             const int64_t* src_entry_off, int32_t n_ranks, int64_t n_entries, int32_t* row_expert,
                             int32_t* row_token, float* row_weight, int64_t* row_e0, int32_t* row_cnt, int32_t* err,
                             void* stream) {
  SSB_CHECK_ARG(rows >= 0 && k >= 1 && k <= 15 && n_ranks >= 1 && n_ranks <= EP_MAXG && n_entries >= 0);
  if (rows == 0) return SSB_OK;
  SSB_CHECK_ARG(meta && src_row_off && src_entry_off && row_expert && row_token && row_weight && row_e0 && row_cnt);
  return ssb_launch(k_ep_unpack, dim3(grid_for(rows, 256)), dim3(256), 0, (cudaStream_t)stream, true, meta, rows, k,
                    src_row_off, src_entry_off, n_ranks, n_entries, row_expert, row_token, row_weight, row_e0,
                    row_cnt, err);
}

extern "C" int ssb_combine_rows(const float* rows, const int64_t* row_e0, const int32_t* row_cnt, int64_t n,
                                int32_t hidden, float* partial, void* stream) {
  SSB_CHECK_ARG(n >= 0 && hidden > 0 && hidden % 4 == 0);
  if (n == 0) return SSB_OK;
  SSB_CHECK_ARG(rows && row_e0 && row_cnt && partial && ((((uintptr_t)rows) | ((uintptr_t)partial)) & 15) == 0);
  const int64_t h4 = hidden / 4;
  return ssb_launch(k_combine_rows<float4>, dim3(grid_for(n * h4, 256)), dim3(256), 0, (cudaStream_t)stream, true,
                    (const float4*)rows, row_e0, row_cnt, n, h4, (float4*)partial);
}

extern "C" int ssb_combine_rows_bf16(const float* rows, const int64_t* row_e0, const int32_t* row_cnt, int64_t n,
                                     int32_t hidden, uint16_t* partial, void* stream) {
  SSB_CHECK_ARG(n >= 0 && hidden > 0 && hidden % 4 == 0);
  if (n == 0) return SSB_OK;
  SSB_CHECK_ARG(rows && row_e0 && row_cnt && partial && ((uintptr_t)rows & 15) == 0 && ((uintptr_t)partial & 7) == 0);
  const int64_t h4 = hidden / 4;
  return ssb_launch(k_combine_rows<uint2>, dim3(grid_for(n * h4, 256)), dim3(256), 0, (cudaStream_t)stream, true,
                    (const float4*)rows, row_e0, row_cnt, n, h4, (uint2*)partial);
}

extern "C" int ssb_ep_combine(const float* ret, const int32_t* tok_slot, const int32_t* tok_entry,
                              const int64_t* ret_entry_off, const int32_t* ids, int64_t tokens, int32_t k,
                              int32_t experts_per_rank, int32_t n_ranks, int32_t strided, int32_t exact,
                              int32_t hidden, const float* sh, float* out, uint16_t* y, void* stream) {
  SSB_CHECK_ARG(tokens >= 0 && k >= 1 && k <= 15 && placement_ok(experts_per_rank, n_ranks, strided));
  SSB_CHECK_ARG(hidden > 0 && hidden % 4 == 0 && (out || y));
  if (tokens == 0) return SSB_OK;
  SSB_CHECK_ARG(ret && ids && (exact ? (tok_entry && ret_entry_off) : tok_slot != nullptr));
  SSB_CHECK_ARG((((uintptr_t)ret | (uintptr_t)sh | (uintptr_t)out) & 15) == 0 && ((uintptr_t)y & 7) == 0);
  const int64_t h4 = hidden / 4;
  return ssb_launch(k_ep_combine<float4>, dim3(grid_for(tokens * h4, 256)), dim3(256), 0, (cudaStream_t)stream, true,
                    (const float4*)ret, tok_slot, tok_entry, ret_entry_off, ids, tokens, k,
                    Placement{experts_per_rank, n_ranks, strided}, exact, h4, (const float4*)sh, (float4*)out,
                    (uint2*)y);
}

extern "C" int ssb_ep_combine_bf16(const uint16_t* ret, const int32_t* tok_slot, const int32_t* ids, int64_t tokens,
                                   int32_t k, int32_t experts_per_rank, int32_t n_ranks, int32_t strided,
                                   int32_t hidden, const float* sh, float* out, uint16_t* y, void* stream) {
  SSB_CHECK_ARG(tokens >= 0 && k >= 1 && k <= 15 && placement_ok(experts_per_rank, n_ranks, strided));
  SSB_CHECK_ARG(hidden > 0 && hidden % 4 == 0);
  if (tokens == 0) return SSB_OK;
  SSB_CHECK_ARG(ret && ids && tok_slot && (out || y));
  SSB_CHECK_ARG((((uintptr_t)ret & 7) | (((uintptr_t)sh | (uintptr_t)out) & 15)) == 0 && ((uintptr_t)y & 7) == 0);
  const int64_t h4 = hidden / 4;
  return ssb_launch(k_ep_combine<uint2>, dim3(grid_for(tokens * h4, 256)), dim3(256), 0, (cudaStream_t)stream, true,
                    (const uint2*)ret, tok_slot, (const int32_t*)nullptr, (const int64_t*)nullptr, ids, tokens, k,
                    Placement{experts_per_rank, n_ranks, strided}, 0, h4, (const float4*)sh, (float4*)out, (uint2*)y);
}
