// moe_align: deterministic stable counting sort of rows by local expert, each expert padded to block_m
// with the sentinel R (slotstream_spark/kernels/moe_align.py:17-48), with align_rows' expert_map gather
// (slotstream_spark/kernels/fused_moe_affine.py:130-133) fused in. No global atomics, no host sync.
//
// One CTA of 32 warps. Warp w owns the contiguous row range [w*chunk, (w+1)*chunk). Pass 1 counts rows per
// (warp, expert) in shared memory; a column scan turns the counts into per-(warp, expert) destinations;
// pass 2 re-reads the rows in order and ranks equal experts inside each 32-row batch with match_any, so
// the order inside an expert is the row order -- exactly the stable sort of the reference.
#include <cooperative_groups.h>

#include "common.cuh"
#include "registry.h"

namespace {

constexpr int AL_WARPS = 32;
constexpr int AL_THREADS = AL_WARPS * 32;
constexpr int AL_MAX_LOCAL = 1280;
constexpr int AL_UNR = 16;      // 32-row batches whose loads one warp keeps in flight
constexpr int64_t AL_CLUSTER_MIN_ROWS = 32768;   // from here on the sort runs on a cluster of CTAs

SSB_DEV int local_of(const int32_t* __restrict__ row_expert, const int32_t* __restrict__ emap, int map_len,
                     int64_t i) {
  int v = row_expert[i];
  if (emap) v = (v >= 0 && v < map_len) ? emap[v] : -1;
  return v;
}

__global__ void __launch_bounds__(AL_THREADS) k_moe_align(const int32_t* __restrict__ row_expert, int64_t R,
                                                           const int32_t* __restrict__ emap, int map_len, int NL,
                                                           int bm, int64_t P, int32_t* __restrict__ sorted_rows,
                                                           int32_t* __restrict__ block_expert,
                                                           int32_t* __restrict__ num_padded) {
  extern __shared__ int sm[];
  int* cnt = sm;                       // [AL_WARPS][NL]: counts, then destinations
  int* tot = cnt + AL_WARPS * NL;      // [NL]
  int* pend = tot + NL;                // [NL] inclusive scan of padded counts
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_wait();
  pdl_trigger();
  for (int i = tid; i < AL_WARPS * NL; i += AL_THREADS) cnt[i] = 0;
  __syncthreads();
  const int64_t chunk = (R + AL_WARPS - 1) / AL_WARPS;
  const int64_t lo0 = (int64_t)warp * chunk;
  const int64_t lo = lo0 < R ? lo0 : R, hi = lo + chunk < R ? lo + chunk : R;
  int* mycnt = cnt + warp * NL;
  // AL_UNR batches of 32 rows per step: their loads are issued together, then the batches are used in order
  for (int64_t base = lo; base < hi; base += 32 * AL_UNR) {
    int v[AL_UNR];
#pragma unroll
    for (int j = 0; j < AL_UNR; ++j) {
      const int64_t i = base + 32 * j + lane;
      v[j] = i < hi ? local_of(row_expert, emap, map_len, i) : -1;
    }
#pragma unroll
    for (int j = 0; j < AL_UNR; ++j)
      if (v[j] >= 0 && v[j] < NL) atomicAdd(&mycnt[v[j]], 1);
  }
  __syncthreads();
  for (int e = tid; e < NL; e += AL_THREADS) {
    int run = 0;
    for (int w = 0; w < AL_WARPS; ++w) {
      int c = cnt[w * NL + e];
      cnt[w * NL + e] = run;
      run += c;
    }
    tot[e] = run;
  }
  __syncthreads();
  if (warp == 0) {  // inclusive scan of padded counts over experts, one contiguous segment per lane
    const int seg = (NL + 31) / 32;
    const int e0 = lane * seg, e1 = min(NL, e0 + seg);
    int s = 0;
    for (int e = e0; e < e1; ++e) s += (tot[e] + bm - 1) / bm * bm;
    int incl = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += y;
    }
    int run = incl - s;
    for (int e = e0; e < e1; ++e) {
      run += (tot[e] + bm - 1) / bm * bm;
      pend[e] = run;
    }
  }
  __syncthreads();
  for (int i = tid; i < AL_WARPS * NL; i += AL_THREADS) {
    int e = i % NL;
    int padded = (tot[e] + bm - 1) / bm * bm;
    cnt[i] += pend[e] - padded;
  }
  __syncthreads();
  for (int64_t base = lo; base < hi; base += 32 * AL_UNR) {
    int vv[AL_UNR];
#pragma unroll
    for (int j = 0; j < AL_UNR; ++j) {
      const int64_t i = base + 32 * j + lane;
      vv[j] = i < hi ? local_of(row_expert, emap, map_len, i) : -1;
    }
#pragma unroll
    for (int j = 0; j < AL_UNR; ++j) {   // batches in row order, rows in lane order: the sort stays stable
      const int64_t i = base + 32 * j + lane;
      const int v = vv[j];
      bool valid = v >= 0 && v < NL;
      int key = valid ? v : -1 - lane;  // invalid lanes never match anyone
      unsigned peers = __match_any_sync(0xFFFFFFFFu, key);
      unsigned below = peers & lanemask_lt();
      if (valid) sorted_rows[mycnt[v] + __popc(below)] = (int32_t)i;
      __syncwarp();
      if (valid && below == 0) mycnt[v] += __popc(peers);
      __syncwarp();
    }
  }
  // padding inside each expert's span, then the tail past num_padded
  for (int e = tid; e < NL; e += AL_THREADS) {
    int padded = (tot[e] + bm - 1) / bm * bm;
    for (int p = pend[e] - padded + tot[e]; p < pend[e]; ++p) sorted_rows[p] = (int32_t)R;
  }
  const int total = pend[NL - 1];
  for (int64_t p = total + tid; p < P; p += AL_THREADS) sorted_rows[p] = (int32_t)R;
  const int64_t nb = P / bm;
  for (int64_t b = tid; b < nb; b += AL_THREADS) {
    const int64_t pos = b * bm;
    int e;  // first expert whose padded span ends after pos (searchsorted right)
    int l = 0, h = NL;
    while (l < h) {
      int mid = (l + h) >> 1;
      if (pend[mid] <= pos) l = mid + 1; else h = mid;
    }
    e = l;
    block_expert[b] = e < NL ? e : -1;
  }
  if (tid == 0) num_padded[0] = total;
}

// The same sort spread over a cluster of CL CTAs (CL x 32 warps, each owning a contiguous row range in order):
// every CTA counts its warps' rows, the CTAs exchange their per-expert totals through distributed shared
// memory, and each CTA then knows where its rows go (rows of earlier CTAs first), so the result is the
// single-CTA kernel's bit for bit. Padding, the tail and block_expert are split over the CTAs.
__global__ void __launch_bounds__(AL_THREADS) k_moe_align_cluster(const int32_t* __restrict__ row_expert, int64_t R,
                                                                   const int32_t* __restrict__ emap, int map_len,
                                                                   int NL, int bm, int64_t P,
                                                                   int32_t* __restrict__ sorted_rows,
                                                                   int32_t* __restrict__ block_expert,
                                                                   int32_t* __restrict__ num_padded) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ int sm[];
  int* cnt = sm;                       // [AL_WARPS][NL]: counts, then destinations
  int* tot = cnt + AL_WARPS * NL;      // [NL] this CTA's totals (read by the other CTAs)
  int* pend = tot + NL;                // [NL] inclusive scan of padded counts
  int* before = pend + NL;             // [NL] rows of each expert in earlier CTAs
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int crank = (int)cluster.block_rank(), csize = (int)cluster.num_blocks();
  pdl_wait();
  pdl_trigger();
  for (int i = tid; i < AL_WARPS * NL; i += AL_THREADS) cnt[i] = 0;
  __syncthreads();
  const int64_t nw = (int64_t)csize * AL_WARPS;
  const int64_t chunk = (R + nw - 1) / nw;
  const int64_t lo0 = ((int64_t)crank * AL_WARPS + warp) * chunk;
  const int64_t lo = lo0 < R ? lo0 : R, hi = lo + chunk < R ? lo + chunk : R;
  int* mycnt = cnt + warp * NL;
  for (int64_t base = lo; base < hi; base += 32 * AL_UNR) {
    int v[AL_UNR];
#pragma unroll
    for (int j = 0; j < AL_UNR; ++j) {
      const int64_t i = base + 32 * j + lane;
      v[j] = i < hi ? local_of(row_expert, emap, map_len, i) : -1;
    }
#pragma unroll
    for (int j = 0; j < AL_UNR; ++j)
      if (v[j] >= 0 && v[j] < NL) atomicAdd(&mycnt[v[j]], 1);
  }
  __syncthreads();
  for (int e = tid; e < NL; e += AL_THREADS) {
    int run = 0;
    for (int w = 0; w < AL_WARPS; ++w) {
      int c = cnt[w * NL + e];
      cnt[w * NL + e] = run;
      run += c;
    }
    tot[e] = run;
  }
  cluster.sync();   // every CTA's totals are complete
  for (int e = tid; e < NL; e += AL_THREADS) {
    int b = 0, g = 0;
    for (int c = 0; c < csize; ++c) {
      const int t = *cluster.map_shared_rank(tot + e, c);
      b += c < crank ? t : 0;
      g += t;
    }
    before[e] = b;
    pend[e] = g;   // grand total, turned into the padded scan below
  }
  cluster.sync();   // no CTA leaves (or overwrites tot) while another may still read it
  if (warp == 0) {  // inclusive scan of padded grand counts over experts, one contiguous segment per lane
    const int seg = (NL + 31) / 32;
    const int e0 = lane * seg, e1 = min(NL, e0 + seg);
    int s = 0;
    for (int e = e0; e < e1; ++e) s += (pend[e] + bm - 1) / bm * bm;
    int incl = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += y;
    }
    int run = incl - s;
    for (int e = e0; e < e1; ++e) {
      const int g = pend[e];
      run += (g + bm - 1) / bm * bm;
      pend[e] = run;
      tot[e] = g;   // from here on: the grand total of expert e
    }
  }
  __syncthreads();
  for (int i = tid; i < AL_WARPS * NL; i += AL_THREADS) {
    int e = i % NL;
    int padded = (tot[e] + bm - 1) / bm * bm;
    cnt[i] += pend[e] - padded + before[e];
  }
  __syncthreads();
  for (int64_t base = lo; base < hi; base += 32 * AL_UNR) {
    int vv[AL_UNR];
#pragma unroll
    for (int j = 0; j < AL_UNR; ++j) {
      const int64_t i = base + 32 * j + lane;
      vv[j] = i < hi ? local_of(row_expert, emap, map_len, i) : -1;
    }
#pragma unroll
    for (int j = 0; j < AL_UNR; ++j) {
      const int64_t i = base + 32 * j + lane;
      const int v = vv[j];
      bool valid = v >= 0 && v < NL;
      int key = valid ? v : -1 - lane;
      unsigned peers = __match_any_sync(0xFFFFFFFFu, key);
      unsigned below = peers & lanemask_lt();
      if (valid) sorted_rows[mycnt[v] + __popc(below)] = (int32_t)i;
      __syncwarp();
      if (valid && below == 0) mycnt[v] += __popc(peers);
      __syncwarp();
    }
  }
  // padding inside each expert's span (experts split over the CTAs), the tail and block_expert (strided)
  for (int e = crank + csize * tid; e < NL; e += csize * AL_THREADS) {
    int padded = (tot[e] + bm - 1) / bm * bm;
    for (int p = pend[e] - padded + tot[e]; p < pend[e]; ++p) sorted_rows[p] = (int32_t)R;
  }
  const int total = pend[NL - 1];
  const int64_t gt = (int64_t)crank * AL_THREADS + tid, gstride = (int64_t)csize * AL_THREADS;
  for (int64_t p = total + gt; p < P; p += gstride) sorted_rows[p] = (int32_t)R;
  const int64_t nb = P / bm;
  for (int64_t b = gt; b < nb; b += gstride) {
    const int64_t pos = b * bm;
    int l = 0, h = NL;
    while (l < h) {
      int mid = (l + h) >> 1;
      if (pend[mid] <= pos) l = mid + 1; else h = mid;
    }
    block_expert[b] = l < NL ? l : -1;
  }
  if (crank == 0 && tid == 0) num_padded[0] = total;
}

int align_cluster_size() {   // 16 CTAs when the device runs such clusters, else 8; 0: no cluster launch
  static int cl = -1;
  if (cl < 0) {
    cl = 0;
    if (cudaFuncSetAttribute(k_moe_align_cluster, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess ||
        cudaFuncSetAttribute(k_moe_align_cluster, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) !=
            cudaSuccess)
      (void)cudaGetLastError();
    for (int want : {16, 8}) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(want);
      cfg.blockDim = dim3(AL_THREADS);
      cfg.dynamicSmemBytes = (size_t)(AL_WARPS * 513 + 3 * 513) * sizeof(int);
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = want;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, k_moe_align_cluster, &cfg) == cudaSuccess && n >= 1) {
        cl = want;
        break;
      }
      (void)cudaGetLastError();
    }
  }
  return cl;
}

}  // namespace

extern "C" int ssb_moe_align(const int32_t* row_expert, int64_t rows, const int32_t* expert_map, int32_t map_len,
                             int32_t num_local, int32_t block_m, int32_t* sorted_rows, int32_t* block_expert,
                             int32_t* num_padded, void* stream) {
  SSB_CHECK_ARG(sorted_rows && block_expert && num_padded && rows >= 0 && (rows == 0 || row_expert));
  SSB_CHECK_ARG(num_local >= 1 && block_m >= 1 && rows < 2147483647LL);
  SSB_CHECK_ARG(!expert_map || map_len >= 0);
  if (num_local > AL_MAX_LOCAL) return SSB_EUNSUPPORTED;
  int64_t n = rows + (int64_t)num_local * (block_m - 1);
  int64_t P = (n + block_m - 1) / block_m * block_m;
  SSB_CHECK_ARG(P < 2147483647LL);
  if (rows >= AL_CLUSTER_MIN_ROWS) {
    const int cl = align_cluster_size();
    const size_t csmem = (size_t)(AL_WARPS * num_local + 3 * num_local) * sizeof(int);
    if (cl > 0 && csmem <= 200 * 1024) {
      ssb_note_smem("moe_align", k_moe_align_cluster, csmem);
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(cl);
      cfg.blockDim = dim3(AL_THREADS);
      cfg.dynamicSmemBytes = csmem;
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
      cudaError_t e = cudaLaunchKernelEx(&cfg, k_moe_align_cluster, row_expert, rows, expert_map, map_len, num_local,
                                         block_m, P, sorted_rows, block_expert, num_padded);
      if (e == cudaSuccess) return SSB_OK;
      (void)cudaGetLastError();   // fall back to the single-CTA kernel
    }
  }
  size_t smem = (size_t)(AL_WARPS * num_local + 2 * num_local) * sizeof(int);
  ssb_note_smem("moe_align", k_moe_align, smem);
  if (smem > 48 * 1024) cudaFuncSetAttribute(k_moe_align, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  return ssb_launch(k_moe_align, dim3(1), dim3(AL_THREADS), smem, (cudaStream_t)stream, true, row_expert, rows,
                    expert_map, map_len, num_local, block_m, P, sorted_rows, block_expert, num_padded);
}
