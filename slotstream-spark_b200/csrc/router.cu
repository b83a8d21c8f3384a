// Router: logits GEMV, fused softmax + stable top-k + renormalise (warp per token), and the generic
// stable top-k of the reference's topk_stable API.
//
// Selection rule (slotstream_spark/kernels/topk_stable.py:1-13): scores map to order-preserving uint32
// keys (positive: flip the sign bit; negative: bitwise not; NaN: 0, the lowest), larger keys first,
// ties to the lower index. Here each candidate becomes the 64-bit composite (key << 32) | ~index, so
// "largest composite first" is exactly that order and every composite is distinct.
#include <atomic>

#include <cub/block/block_scan.cuh>

#include "affine.cuh"
#include "registry.h"
#include "select.cuh"

namespace {

// ------------------------------------------------------------------ logits
// Warp per weight row, the row held in registers (lane l owns 16-byte chunks l, l+32, ...); a CTA covers
// 4 rows and a tile of up to TT tokens staged in shared memory. The sum order of one logit is fixed by
// (hidden) alone: lane-sequential over its chunks, then a butterfly -- the same for any token count.
constexpr int RL_WARPS = 4;
constexpr int RL_TT = 8;
constexpr int RL_MAXC = 16;  // chunks of 8 bf16 per lane: hidden <= 4096

__global__ void __launch_bounds__(RL_WARPS * 32) k_router_logits(const uint16_t* __restrict__ x,
                                                                  const uint16_t* __restrict__ w,
                                                                  const uint16_t* __restrict__ w_extra, int64_t tokens,
                                                                  int hidden, int n_rows, int ld,
                                                                  float* __restrict__ logits) {
  extern __shared__ __align__(16) uint4 xs[];  // [RL_TT][hidden / 8]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n_total = n_rows + (w_extra ? 1 : 0);
  const int row = blockIdx.x * RL_WARPS + warp;
  const int nch = hidden >> 3;       // 16-byte chunks per row
  const int cpl = nch >> 5;          // chunks per lane (hidden % 256 == 0)
  const int64_t t0 = (int64_t)blockIdx.y * RL_TT;
  const int tt = (int)(tokens - t0 < RL_TT ? tokens - t0 : RL_TT);

  uint4 wr[RL_MAXC];
  const uint16_t* wrow = nullptr;
  if (row < n_total) wrow = (row < n_rows) ? w + (int64_t)row * hidden : w_extra;
  // weights are static: prefetch them before waiting for the producer of x
#pragma unroll
  for (int i = 0; i < RL_MAXC; ++i)
    if (i < cpl && wrow) wr[i] = ld_stream_u4(wrow + (size_t)(lane + 32 * i) * 8);
  pdl_wait();
  for (int c = threadIdx.x; c < tt * nch; c += blockDim.x) {
    int t = c / nch, j = c - t * nch;
    xs[t * nch + j] = *reinterpret_cast<const uint4*>(x + (t0 + t) * hidden + (int64_t)j * 8);
  }
  __syncthreads();
  pdl_trigger();
  if (!wrow) return;
  for (int t = 0; t < tt; ++t) {
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < RL_MAXC; ++i) {
      if (i < cpl) {
        uint4 xv = xs[t * nch + lane + 32 * i];
        uint4 wv = wr[i];
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
    if (lane == 0) logits[(t0 + t) * ld + row] = acc;
  }
}

// One weight row (the shared-expert gate of a prefill chunk): a warp per token, x read straight from global
// memory with all of a lane's chunks in flight at once; the same per-lane order and butterfly as above.
constexpr int RL1_WARPS = 8;
constexpr int RL1_TPW = 4;   // tokens per warp

__global__ void __launch_bounds__(RL1_WARPS * 32) k_router_logits_row(const uint16_t* __restrict__ x,
                                                                      const uint16_t* __restrict__ w, int64_t tokens,
                                                                      int hidden, int ld, float* __restrict__ logits) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int cpl = (hidden >> 3) >> 5;
  uint4 wr[RL_MAXC];
#pragma unroll
  for (int i = 0; i < RL_MAXC; ++i)
    if (i < cpl) wr[i] = ld_stream_u4(w + (size_t)(lane + 32 * i) * 8);
  pdl_wait();
  pdl_trigger();
  const int64_t t0 = ((int64_t)blockIdx.x * RL1_WARPS + warp) * RL1_TPW;
  for (int tt = 0; tt < RL1_TPW; ++tt) {
    const int64_t t = t0 + tt;
    if (t >= tokens) break;
    uint4 xv[RL_MAXC];
#pragma unroll
    for (int i = 0; i < RL_MAXC; ++i)
      if (i < cpl) xv[i] = __ldg(reinterpret_cast<const uint4*>(x + t * hidden) + lane + 32 * i);
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < RL_MAXC; ++i) {
      if (i < cpl) {
        const uint4 a = xv[i], b = wr[i];
        acc = fmaf(bf16_lo(b.x), bf16_lo(a.x), acc);
        acc = fmaf(bf16_hi(b.x), bf16_hi(a.x), acc);
        acc = fmaf(bf16_lo(b.y), bf16_lo(a.y), acc);
        acc = fmaf(bf16_hi(b.y), bf16_hi(a.y), acc);
        acc = fmaf(bf16_lo(b.z), bf16_lo(a.z), acc);
        acc = fmaf(bf16_hi(b.z), bf16_hi(a.z), acc);
        acc = fmaf(bf16_lo(b.w), bf16_lo(a.w), acc);
        acc = fmaf(bf16_hi(b.w), bf16_hi(a.w), acc);
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) logits[t * ld] = acc;
  }
}

// ------------------------------------------------------------------ select (softmax + top-k + renorm)
constexpr int RS_WARPS = 4;
// warps (tokens) per select CTA: the per-warp scratch of 1024 experts allows two within 48 KB
constexpr int rs_warps(int epl) { return epl > 16 ? 2 : RS_WARPS; }
constexpr int RS_MAXE = 32;  // experts per lane: experts <= 1024

struct SelectArgs {
  const float* logits;
  int ld;
  int64_t tokens;
  int experts, k;
  const float* bias;
  int flags;
  int32_t* out_idx;
  float* out_w;
  float* out_probs;
  float* out_sh_gate;
  // optional: resolve the chosen experts through the slot tables and prefetch their records into L2
  int layer;
  const int32_t* map;
  int64_t map_len;
  const int64_t* slot_ptr;
  int64_t n_slots;
  int64_t* out_base;
  uint32_t prefetch_bytes;
  int32_t* err;
};

// Lane `lane` (< k) holds the rank-`lane` composite; write ids and renormalised weights, then the optional
// expert resolution / L2 prefetch and the shared-expert gate.
SSB_DEV void select_tail(const SelectArgs& a, int64_t t, int lane, unsigned long long mine, float my_p, float sum,
                         const float* lrow) {
  const int k = a.k;
  if (lane < k) {
    const int e = (int)(0xFFFFFFFFu - (uint32_t)(mine & 0xFFFFFFFFull));
    a.out_idx[t * k + lane] = e;
    a.out_w[t * k + lane] = my_p / sum;
    if (a.out_base) {
      const uint8_t* base = resolve_expert(e, a.layer, a.map, a.map_len, a.slot_ptr, a.n_slots, a.err);
      a.out_base[t * k + lane] = (int64_t)base;
      if (base && a.prefetch_bytes) {
        for (uint32_t off = 0; off < a.prefetch_bytes; off += 65536u) {
          const uint32_t n = a.prefetch_bytes - off < 65536u ? a.prefetch_bytes - off : 65536u;
          prefetch_l2(base + off, n);
        }
      }
    }
  }
  if ((a.flags & SSB_ROUTER_SHARED_GATE) && lane == 0) {
    // sigmoid(lin(x, shared_expert_gate)) with lin's bf16 output and a bf16 sigmoid (model/layers.py:401)
    const float gl = round_bf16(__ldcg(lrow + a.experts));
    a.out_sh_gate[t] = round_bf16(1.f / (1.f + expf(-gl)));
  }
}

template <int EPL>
__global__ void __launch_bounds__(RS_WARPS * 32) k_router_select(SelectArgs a) {
  __shared__ SelectScratch<EPL> s_sel[rs_warps(EPL)];
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t t = (int64_t)blockIdx.x * rs_warps(EPL) + warp;
  if (t >= a.tokens) return;
  const float* lrow = a.logits + t * a.ld;
  unsigned long long mine;
  float my_p, sum;
  warp_select<EPL>(lrow, a.experts, a.k, a.bias, a.flags, a.out_probs ? a.out_probs + t * a.experts : nullptr,
                   s_sel[warp], lane, mine, my_p, sum);
  select_tail(a, t, lane, mine, my_p, sum, lrow);
}

// ------------------------------------------------------------------ generic stable top-k
constexpr int TK_THREADS = 512;
constexpr int TK_ITEMS = 4;

__global__ void __launch_bounds__(TK_THREADS) k_topk_stable(const float* __restrict__ scores,
                                                             const int32_t* __restrict__ n_valid, int n, int k,
                                                             int32_t* __restrict__ out_idx,
                                                             float* __restrict__ out_val) {
  using Scan = cub::BlockScan<int, TK_THREADS>;
  __shared__ typename Scan::TempStorage scan_tmp;
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_digit, s_kleft;
  __shared__ int s_base_sel, s_base_eq;
  __shared__ unsigned long long cand[16];
  pdl_wait();
  pdl_trigger();
  const int64_t row = blockIdx.x;
  const float* x = scores + row * n;
  int nv = n;
  if (n_valid) nv = max(0, min(n_valid[row], n));
  const int tid = threadIdx.x;
  const bool take_all = nv <= k;

  uint32_t prefix = 0, pmask = 0, kleft = (uint32_t)k;
  if (!take_all) {
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      if (tid < 256) hist[tid] = 0;
      __syncthreads();
      for (int i = tid; i < nv; i += TK_THREADS) {
        uint32_t key = order_key(x[i]);
        if ((key & pmask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (tid == 0) {
        uint32_t cum = 0, d = 0, kl = kleft;
        for (int b = 255; b >= 0; --b) {
          uint32_t h = hist[b];
          if (cum + h >= kl) {
            d = (uint32_t)b;
            kl -= cum;
            break;
          }
          cum += h;
        }
        s_digit = d;
        s_kleft = kl;
      }
      __syncthreads();
      prefix |= s_digit << shift;
      pmask |= 255u << shift;
      kleft = s_kleft;
      __syncthreads();
    }
  }
  const uint32_t thr = prefix;   // the k-th largest key; `kleft` entries equal to it are taken, lowest index first
  if (tid == 0) {
    s_base_sel = 0;
    s_base_eq = 0;
  }
  __syncthreads();
  for (int base = 0; base < nv; base += TK_THREADS * TK_ITEMS) {
    int gt[TK_ITEMS], eq[TK_ITEMS];
    int n_eq = 0;
#pragma unroll
    for (int it = 0; it < TK_ITEMS; ++it) {
      int i = base + tid * TK_ITEMS + it;
      gt[it] = eq[it] = 0;
      if (i < nv) {
        if (take_all) {
          gt[it] = 1;
        } else {
          uint32_t key = order_key(x[i]);
          gt[it] = key > thr;
          eq[it] = key == thr;
        }
      }
      n_eq += eq[it];
    }
    int eq_before, eq_total;
    Scan(scan_tmp).ExclusiveSum(n_eq, eq_before, eq_total);
    __syncthreads();
    int eq_run = s_base_eq + eq_before;
    int sel[TK_ITEMS], n_sel = 0;
#pragma unroll
    for (int it = 0; it < TK_ITEMS; ++it) {
      sel[it] = gt[it];
      if (eq[it]) {
        sel[it] = eq_run < (int)kleft;
        ++eq_run;
      }
      n_sel += sel[it];
    }
    int sel_before, sel_total;
    Scan(scan_tmp).ExclusiveSum(n_sel, sel_before, sel_total);
    int pos = s_base_sel + sel_before;
#pragma unroll
    for (int it = 0; it < TK_ITEMS; ++it) {
      if (!sel[it]) continue;
      int i = base + tid * TK_ITEMS + it;
      if (k <= 16) {
        cand[pos] = composite(order_key(x[i]), (uint32_t)i);
      } else {
        out_idx[row * k + pos] = i;
        if (out_val) out_val[row * k + pos] = x[i];
      }
      ++pos;
    }
    __syncthreads();
    if (tid == 0) {
      s_base_sel += sel_total;
      s_base_eq += eq_total;
    }
    __syncthreads();
  }
  const int count = s_base_sel;
  if (k <= 16) {
    if (tid == 0) {
      for (int a = 1; a < count; ++a) {  // insertion sort, descending composite
        unsigned long long v = cand[a];
        int b = a - 1;
        while (b >= 0 && cand[b] < v) {
          cand[b + 1] = cand[b];
          --b;
        }
        cand[b + 1] = v;
      }
      for (int j = 0; j < count; ++j) {
        int i = (int)(0xFFFFFFFFu - (uint32_t)(cand[j] & 0xFFFFFFFFull));
        out_idx[row * k + j] = i;
        if (out_val) out_val[row * k + j] = x[i];
      }
    }
  }
  for (int j = count + tid; j < k; j += TK_THREADS) {
    out_idx[row * k + j] = -1;
    if (out_val) out_val[row * k + j] = -INFINITY;
  }
}

int launch_select(SelectArgs a, void* stream);

}  // namespace

extern "C" int ssb_router_logits(const uint16_t* x, const uint16_t* w, const uint16_t* w_extra, int64_t tokens,
                                 int32_t hidden, int32_t n_rows, int32_t ld, float* logits, void* stream) {
  SSB_CHECK_ARG(tokens >= 0 && n_rows >= 1);
  if (hidden % 256 || hidden <= 0 || hidden > 4096) return SSB_EUNSUPPORTED;
  SSB_CHECK_ARG(ld >= n_rows + (w_extra ? 1 : 0));
  if (tokens == 0) return SSB_OK;   // empty tensors may come with null pointers
  SSB_CHECK_ARG(x && w && logits);
  const int n_total = n_rows + (w_extra ? 1 : 0);
  if (n_total == 1 && tokens >= 1024) {   // one row over many tokens: no staging of x, a warp per token
    const int64_t per_cta = (int64_t)RL1_WARPS * RL1_TPW;
    ssb_note_smem("router_logits", k_router_logits_row, 0);
    return ssb_launch(k_router_logits_row, dim3((unsigned)((tokens + per_cta - 1) / per_cta)), dim3(RL1_WARPS * 32), 0,
                      (cudaStream_t)stream, true, x, w_extra ? w_extra : w, tokens, hidden, ld, logits);
  }
  dim3 grid((n_total + RL_WARPS - 1) / RL_WARPS, (unsigned)((tokens + RL_TT - 1) / RL_TT));
  SSB_CHECK_ARG(grid.y <= 65535u);
  size_t smem = (size_t)RL_TT * hidden * 2;
  ssb_note_smem("router_logits", k_router_logits, smem);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(k_router_logits, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  return ssb_launch(k_router_logits, grid, dim3(RL_WARPS * 32), smem, (cudaStream_t)stream, true, x, w, w_extra,
                    tokens, hidden, n_rows, ld, logits);
}

extern "C" int ssb_topk_stable(const float* scores, const int32_t* n_valid, int64_t rows, int32_t n, int32_t k,
                               int32_t* out_idx, float* out_val, void* stream) {
  SSB_CHECK_ARG(rows >= 0 && n >= 1 && n <= 65536 && k >= 1 && k <= n);
  if (rows == 0) return SSB_OK;   // empty tensors may come with null pointers
  SSB_CHECK_ARG(scores && out_idx);
  SSB_CHECK_ARG(rows <= 2147483647LL);
  ssb_note_smem("topk_stable", k_topk_stable, 0);
  return ssb_launch(k_topk_stable, dim3((unsigned)rows), dim3(TK_THREADS), 0, (cudaStream_t)stream, true, scores,
                    n_valid, n, k, out_idx, out_val);
}

namespace {

int launch_select(SelectArgs a, void* stream) {
  SSB_CHECK_ARG(a.tokens >= 0);
  SSB_CHECK_ARG(a.experts >= 1 && a.experts <= 32 * RS_MAXE && a.k >= 1 && a.k <= 32 && a.k <= a.experts);
  SSB_CHECK_ARG(a.ld >= a.experts + ((a.flags & SSB_ROUTER_SHARED_GATE) ? 1 : 0));
  SSB_CHECK_ARG(a.prefetch_bytes % 16 == 0);
  if (a.tokens == 0) return SSB_OK;   // empty tensors may come with null pointers
  SSB_CHECK_ARG(a.logits && a.out_idx && a.out_w);
  SSB_CHECK_ARG(!(a.flags & SSB_ROUTER_SHARED_GATE) || a.out_sh_gate);
  const int epl = (a.experts + 31) / 32;
  const int nw = rs_warps(epl <= 4 ? 4 : epl <= 8 ? 8 : epl <= 16 ? 16 : 32);
  dim3 grid((unsigned)((a.tokens + nw - 1) / nw));
  void (*kern)(SelectArgs) = epl <= 4 ? k_router_select<4> : epl <= 8 ? k_router_select<8>
                             : epl <= 16 ? k_router_select<16> : k_router_select<32>;
  ssb_note_smem("router_select", kern, 0);
  return ssb_launch(kern, grid, dim3(nw * 32), 0, (cudaStream_t)stream, true, a);
}

}  // namespace

extern "C" int ssb_router_select(const float* logits, int32_t ld, int64_t tokens, int32_t experts, int32_t k,
                                 const float* bias, int32_t flags, int32_t* out_idx, float* out_w, float* out_probs,
                                 float* out_sh_gate, void* stream) {
  SelectArgs a{};
  a.logits = logits;
  a.ld = ld;
  a.tokens = tokens;
  a.experts = experts;
  a.k = k;
  a.bias = bias;
  a.flags = flags;
  a.out_idx = out_idx;
  a.out_w = out_w;
  a.out_probs = out_probs;
  a.out_sh_gate = out_sh_gate;
  return launch_select(a, stream);
}

extern "C" int ssb_router_select_resolve(const float* logits, int32_t ld, int64_t tokens, int32_t experts,
                                         int32_t k, const float* bias, int32_t flags, int32_t* out_idx, float* out_w,
                                         float* out_sh_gate, int32_t layer, const int32_t* map_t, int64_t map_len,
                                         const int64_t* slot_ptr_t, int64_t n_slots, int64_t* out_base,
                                         int64_t prefetch_bytes, int32_t* err, void* stream) {
  SSB_CHECK_ARG(map_t && slot_ptr_t && out_base && layer >= 0 && prefetch_bytes >= 0 && prefetch_bytes < (1ll << 31));
  SelectArgs a{};
  a.logits = logits;
  a.ld = ld;
  a.tokens = tokens;
  a.experts = experts;
  a.k = k;
  a.bias = bias;
  a.flags = flags;
  a.out_idx = out_idx;
  a.out_w = out_w;
  a.out_sh_gate = out_sh_gate;
  a.layer = layer;
  a.map = map_t;
  a.map_len = map_len;
  a.slot_ptr = slot_ptr_t;
  a.n_slots = n_slots;
  a.out_base = out_base;
  a.prefetch_bytes = (uint32_t)prefetch_bytes;
  a.err = err;
  return launch_select(a, stream);
}

// ---------------------------------------------------------------------------------------------------------
// Router with its logits in a fixed, statically reserved device array (no workspace argument).
//
// Some callers cannot allocate device memory on their call path. A host binding without a caching
// allocator (cgo, JNI, plain C over this ABI) would have to call cudaMalloc, which synchronises the whole
// device, on every decode step; and a process whose expert slot pool reserved nearly all of HBM up front has
// no headroom left to hand out.
// For those callers the logits live in a file-scope __device__ array of ROUTER_STATIC_LOGITS floats
// (256 KiB): a call whose tokens * (experts + 1 with a shared gate, else experts) exceeds it is refused with
// SSB_ETOOBIG before anything is launched. The logits kernel writes every element the select kernel reads,
// earlier on the same stream, so nothing in the array has to start at zero. There is one array per device
// in the process: calls that overlap on one device (other streams, other host threads) overwrite each
// other's logits and race. The first call on a device looks the array's address up with
// cudaGetSymbolAddress (with that device current) and keeps it for the life of the process, so that first
// call should come before any stream capture, and resetting the device (cudaDeviceReset) while this library
// is loaded is not supported: the address kept for it would be stale.
namespace {
constexpr int64_t ROUTER_STATIC_LOGITS = 65536;
constexpr int ROUTER_STATIC_MAX_DEVICES = 64;
__device__ __align__(256) float g_router_static_logits[ROUTER_STATIC_LOGITS];
std::atomic<float*> g_router_static_addr[ROUTER_STATIC_MAX_DEVICES];
}  // namespace

extern "C" int ssb_router_topk_static(const uint16_t* x, const uint16_t* w, const uint16_t* w_shared_gate,
                                      int64_t tokens, int32_t hidden, int32_t experts, int32_t k,
                                      const float* bias, int32_t flags, int32_t* out_idx, float* out_w,
                                      float* out_sh_gate, void* stream) {
  SSB_CHECK_ARG(tokens >= 0 && experts >= 1 && k >= 1);
  SSB_CHECK_ARG(k <= 32 && k <= experts && experts <= 32 * RS_MAXE && (flags & ~SSB_ROUTER_ROUND_BF16) == 0);
  const int32_t ld = experts + (w_shared_gate ? 1 : 0);
  if (tokens > ROUTER_STATIC_LOGITS / ld) return SSB_ETOOBIG;
  if (tokens == 0) return SSB_OK;   // empty tensors may come with null pointers
  SSB_CHECK_ARG(x && w && out_idx && out_w);
  SSB_CHECK_ARG(!w_shared_gate || out_sh_gate);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= ROUTER_STATIC_MAX_DEVICES) return SSB_EUNSUPPORTED;
  float* logits = g_router_static_addr[dev].load(std::memory_order_acquire);
  if (!logits) {
    e = cudaGetSymbolAddress((void**)&logits, g_router_static_logits);
    if (e != cudaSuccess) return (int)e;
    g_router_static_addr[dev].store(logits, std::memory_order_release);
  }
  int rc = ssb_router_logits(x, w, w_shared_gate, tokens, hidden, experts, ld, logits, stream);
  if (rc != SSB_OK) return rc;
  return ssb_router_select(logits, ld, tokens, experts, k, bias,
                           flags | (w_shared_gate ? SSB_ROUTER_SHARED_GATE : 0), out_idx, out_w, nullptr,
                           out_sh_gate, stream);
}
