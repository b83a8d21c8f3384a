// Grouped affine-4-bit GEMM on the 5th-generation tensor cores (tcgen05 + TMEM) for the prefill MoE
// (slotstream_spark/kernels/fused_moe_affine.py:53-127) and the dense prefill GEMM (kernels/gemm_affine.py).
//
// One CTA computes a 128-row block (one expert's rows, from moe_align) times 256 B-rows:
//  * gate_up: the 256 B-rows are 128 gate rows + 128 up rows of the same inter columns, so one
//    M128xN256 accumulator holds both and the epilogue forms h = silu(g) * u -> bf16
//    (kernels/fused_moe_affine.py:76-81);
//  * down / plain: 256 output columns; the epilogue scales by the row's routing weight (fp32 out,
//    kernels/fused_moe_affine.py:103-108) or stores plain fp32 (kernels/gemm_affine.py:19-37).
// Warp roles (12 warps):
//  * warp 0      gathers the block's activation rows with 16-byte cp.async into 128B-swizzled K-major tiles;
//  * warp 1      owns TMEM (256 columns) and issues tcgen05.mma (M128 N256 K16, four per 64-wide k-block);
//  * warps 4..11 stage their weight row's packed nibbles and bf16 scale/bias with cp.async, dequantise
//                q*s + b in fp32 (two roundings, as kernels/affine_ref.py:22-31) -> bf16 (the reference's
//                _wtile rounding, kernels/fused_moe_affine.py:38-50) into the swizzled B tile, then run
//                the epilogue from TMEM.
// Stages are handed over with mbarriers (full_a / full_b / empty); every wait gives up after a bounded time
// and sets SSB_ERR_TIMEOUT instead of hanging. A row's result depends only on that row and that expert's
// bytes: the k order is fixed, so any row count or group composition gives the same bits.
#include "registry.h"
#include "tc_common.cuh"

namespace {

constexpr int BM = 128, BK = 64, BN = 256;
constexpr int STAGES = 3;        // A/B operand stages
constexpr int PD = 3;            // weight staging depth of each producer thread
constexpr int THREADS = 384;
constexpr int A_WARP = 0, MMA_WARP = 1, PROD_WARP0 = 4, N_PROD = 256;
constexpr uint32_t A_STAGE = BM * 128;           // 16 KB
constexpr uint32_t B_STAGE = BN * 128;           // 32 KB
constexpr uint32_t W_STG = N_PROD * 32;          // packed nibbles of one k-block, 32 B per B-row
constexpr uint32_t SB_STG = N_PROD * 4;          // 4-byte words holding the scale (or bias) of the k-block
constexpr uint32_t STG = W_STG + 2 * SB_STG;
constexpr uint32_t TMEM_COLS = 256;

enum { EPI_SWIGLU = 0, EPI_SCALE = 1, EPI_PLAIN = 2 };

struct GemmArgs {
  const uint16_t* a;          // bf16 activation rows, `lda` elements apart
  int64_t lda;
  const int32_t* row_token;   // nullable: the A row of row r is r
  const int32_t* sorted_rows; // nullable: identity (rows m < R)
  const int32_t* block_expert;
  const int32_t* num_padded;
  int64_t R;                  // rows; sorted_rows entries >= R are padding
  const int64_t* group_base;  // record (or weight) base address per local expert; nullable: base0
  const uint8_t* base0;
  int n_groups;
  int64_t off_w[2], off_s[2], off_b[2];   // byte offsets of weight piece 0 (and 1 for gate_up) from the base
  int K, gs;
  int dense_b;                // B rows are plain bf16 (ldb elements apart) instead of affine 4-bit pieces
  int64_t ldb;
  int shared_local;           // local index of the shared expert (bf16 rounding between its ops), -1: none
  const float* row_weight;
  void* out;
  int64_t ldo;
  int32_t* err;
};

struct Smem {
  uint8_t* a;
  uint8_t* b;
  uint8_t* stg;
  uint64_t* full_a;
  uint64_t* full_b;
  uint64_t* empty;
  uint64_t* acc_full;
  uint32_t* tmem;
  int64_t* arow;
  int32_t* orow;
};

constexpr size_t SMEM_BYTES = 1024 + STAGES * (A_STAGE + B_STAGE) + PD * STG + 8 * (3 * STAGES + 1) + 16 +
                              BM * 8 + BM * 4;

SSB_DEV Smem carve(uint8_t* raw) {
  Smem s;
  uint8_t* p = (uint8_t*)(((uintptr_t)raw + 1023) & ~(uintptr_t)1023);
  s.a = p;
  p += STAGES * A_STAGE;
  s.b = p;
  p += STAGES * B_STAGE;
  s.stg = p;
  p += PD * STG;
  s.full_a = (uint64_t*)p;
  s.full_b = s.full_a + STAGES;
  s.empty = s.full_b + STAGES;
  s.acc_full = s.empty + STAGES;
  p += 8 * (3 * STAGES + 1);
  s.tmem = (uint32_t*)p;
  p += 16;
  s.arow = (int64_t*)p;
  p += BM * 8;
  s.orow = (int32_t*)p;
  return s;
}

SSB_DEV uint32_t pack_bf16x2(float lo, float hi) {
  return (uint32_t)f32_to_bf16(lo) | ((uint32_t)f32_to_bf16(hi) << 16);
}

// fl(fl(q*s) + b) for the 8 nibbles of w; sc[j] = s * 16^-j' matches the magic-number scale of nibble j
SSB_DEV void dequant_word(uint32_t w, const float* sc, float b, float* o) {
  const uint32_t M = 0x4B000000u;
  const uint32_t w5 = w >> 12;
  const float m = 8388608.f;
  float f[8];
  f[0] = __uint_as_float((w & 0xFu) | M) - m;
  f[1] = __uint_as_float((w & 0xF0u) | M) - m;
  f[2] = __uint_as_float((w & 0xF00u) | M) - m;
  f[3] = __uint_as_float((w & 0xF000u) | M) - m;
  f[4] = __uint_as_float((w & 0xF0000u) | M) - m;
  f[5] = __uint_as_float((w5 & 0xF00u) | M) - m;
  f[6] = __uint_as_float((w5 & 0xF000u) | M) - m;
  f[7] = __uint_as_float((w5 & 0xF0000u) | M) - m;
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = __fadd_rn(__fmul_rn(f[j], sc[j]), b);
}

SSB_DEV void scales_for(float s, float* sc) {
  sc[0] = s;
  sc[1] = s * 0.0625f;
  sc[2] = s * 0.00390625f;
  sc[3] = s * 0.000244140625f;
  sc[4] = s * 1.52587890625e-05f;
  sc[5] = sc[2];
  sc[6] = sc[3];
  sc[7] = sc[4];
}

template <int EPI>
__global__ void __launch_bounds__(THREADS, 1) k_moe_gemm(GemmArgs a) {
  extern __shared__ uint8_t smraw[];
  Smem S = carve(smraw);
  __shared__ int s_fail;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int mb = blockIdx.y, nb = blockIdx.x;
  pdl_wait();
  pdl_trigger();
  if (a.num_padded && (int64_t)mb * BM >= (int64_t)__ldcg(a.num_padded)) return;
  const int e = a.block_expert ? __ldcg(a.block_expert + mb) : 0;
  if (e < 0 || e >= a.n_groups) return;
  const uint8_t* base = a.group_base ? (const uint8_t*)a.group_base[e] : a.base0;
  if (((uintptr_t)base & 15) || base == nullptr) {
    if (tid == 0) set_err(a.err, SSB_ERR_MISALIGNED);
    return;
  }
  if (tid < BM) {
    const int64_t m = (int64_t)mb * BM + tid;
    const int64_t row = a.sorted_rows ? (int64_t)__ldcg(a.sorted_rows + m) : m;
    const bool ok = row >= 0 && row < a.R;
    S.orow[tid] = ok ? (int32_t)row : -1;
    S.arow[tid] = ok ? (a.row_token ? (int64_t)__ldcg(a.row_token + row) : row) * a.lda : -1;
  }
  if (tid == 0) {
    s_fail = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&S.full_a[s], 32);
      mbar_init(&S.full_b[s], N_PROD);
      mbar_init(&S.empty[s], 1);
    }
    mbar_init(S.acc_full, 1);
    fence_mbar_init();
  }
  if (warp == MMA_WARP) tmem_alloc(S.tmem, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *S.tmem;
  const int KB = a.K / BK;

  if (warp == A_WARP) {
    // ---------------- activation gather: 1024 16-byte chunks per k-block, 32 per lane
    const int c = lane & 7;
    for (int kb = 0; kb < KB; ++kb) {
      const int s = kb % STAGES, r = kb / STAGES;
      if (!mbar_wait_ns(&S.empty[s], (r & 1) ^ 1, SSB_WAIT_NS)) {
        s_fail = 1;
        break;
      }
      const uint32_t dst = smem_u32(S.a + s * A_STAGE);
#pragma unroll 8
      for (int i = 0; i < 32; ++i) {
        const int row = (lane >> 3) + 4 * i;
        const int64_t off = S.arow[row];
        const uint16_t* src = a.a + (off >= 0 ? off : 0) + kb * BK + c * 8;
        cp_async16(dst + swz128(row, c), src, off >= 0 ? 16u : 0u);
      }
      cp_async_arrive(&S.full_a[s]);
    }
    cp_async_wait_all();
  } else if (warp == MMA_WARP) {
    // ---------------- single-thread MMA issue
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(BM, BN);
      for (int kb = 0; kb < KB; ++kb) {
        const int s = kb % STAGES, r = kb / STAGES;
        if (!mbar_wait_ns(&S.full_a[s], r & 1, SSB_WAIT_NS) || !mbar_wait_ns(&S.full_b[s], r & 1, SSB_WAIT_NS)) {
          s_fail = 1;
          break;
        }
        fence_proxy_async_smem();
        tc_fence_after();
        const uint64_t da = umma_desc_sw128(smem_u32(S.a + s * A_STAGE));
        const uint64_t db = umma_desc_sw128(smem_u32(S.b + s * B_STAGE));
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
          umma_bf16(tmem, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc, (kb | k) != 0);
        umma_commit(&S.empty[s]);
      }
      umma_commit(S.acc_full);
    }
    __syncwarp();
  } else if (warp >= PROD_WARP0) {
    // ---------------- weight producers: one B-row per thread
    const int p = tid - PROD_WARP0 * 32;
    int piece, nrow;
    if (EPI == EPI_SWIGLU) {
      piece = p >> 7;
      nrow = nb * (BN / 2) + (p & 127);
    } else {
      piece = 0;
      nrow = nb * BN + p;
    }
    if (a.dense_b) {
      // plain bf16 weight rows: 16-byte cp.async straight into the swizzled tile, no dequantisation
      const uint16_t* drow = (const uint16_t*)base + (int64_t)nrow * a.ldb;
      for (int kb = 0; kb < KB; ++kb) {
        const int s = kb % STAGES, r = kb / STAGES;
        if (!mbar_wait_ns(&S.empty[s], (r & 1) ^ 1, SSB_WAIT_NS)) {
          s_fail = 1;
          break;
        }
        const uint32_t bt = smem_u32(S.b + s * B_STAGE);
#pragma unroll
        for (int c = 0; c < 8; ++c) cp_async16(bt + swz128(p, c), drow + kb * BK + c * 8, 16);
        cp_async_arrive(&S.full_b[s]);
      }
    }
    const int ng = a.K / a.gs;
    const uint8_t* wrow = base + a.off_w[piece] + (int64_t)nrow * (a.K / 2);
    const uint16_t* srow = (const uint16_t*)(base + a.off_s[piece]) + (int64_t)nrow * ng;
    const uint16_t* brow = (const uint16_t*)(base + a.off_b[piece]) + (int64_t)nrow * ng;
    auto issue = [&](int kb) {
      uint8_t* st = S.stg + (kb % PD) * STG;
      const uint32_t dw = smem_u32(st + p * 32);
      cp_async16(dw, wrow + kb * 32, 16);
      cp_async16(dw + 16, wrow + kb * 32 + 16, 16);
      // the 4-byte-aligned word that holds the k-block's scale (bias): group kb (gs 64) or 2kb, 2kb+1 (gs 32)
      const int g0 = a.gs == 64 ? kb : 2 * kb;
      asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(st + W_STG + p * 4)),
                   "l"(srow + (g0 & ~1)) : "memory");
      asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(st + W_STG + SB_STG + p * 4)),
                   "l"(brow + (g0 & ~1)) : "memory");
    };
    for (int kb = 0; kb < PD - 1 && kb < KB && !a.dense_b; ++kb) {
      issue(kb);
      asm volatile("cp.async.commit_group;" ::: "memory");
    }
    for (int kb = 0; kb < KB && !a.dense_b; ++kb) {
      if (kb + PD - 1 < KB) issue(kb + PD - 1);
      asm volatile("cp.async.commit_group;" ::: "memory");
      asm volatile("cp.async.wait_group %0;" ::"n"(PD - 1) : "memory");
      const uint8_t* st = S.stg + (kb % PD) * STG;
      const uint4 w0 = *reinterpret_cast<const uint4*>(st + p * 32);
      const uint4 w1 = *reinterpret_cast<const uint4*>(st + p * 32 + 16);
      const uint32_t sw = *reinterpret_cast<const uint32_t*>(st + W_STG + p * 4);
      const uint32_t bw = *reinterpret_cast<const uint32_t*>(st + W_STG + SB_STG + p * 4);
      float s0, b0, s1, b1;
      if (a.gs == 64) {
        s0 = s1 = (kb & 1) ? bf16_hi(sw) : bf16_lo(sw);
        b0 = b1 = (kb & 1) ? bf16_hi(bw) : bf16_lo(bw);
      } else {
        s0 = bf16_lo(sw);
        s1 = bf16_hi(sw);
        b0 = bf16_lo(bw);
        b1 = bf16_hi(bw);
      }
      float sc0[8], sc1[8];
      scales_for(s0, sc0);
      scales_for(s1, sc1);
      const int s = kb % STAGES, r = kb / STAGES;
      if (!mbar_wait_ns(&S.empty[s], (r & 1) ^ 1, SSB_WAIT_NS)) {
        s_fail = 1;
        break;
      }
      uint8_t* bt = S.b + s * B_STAGE;
      const uint32_t ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int c = 0; c < 8; ++c) {     // chunk c = elements 8c..8c+7 = word c
        float v[8];
        dequant_word(ws[c], c < 4 ? sc0 : sc1, c < 4 ? b0 : b1, v);
        uint4 o;
        o.x = pack_bf16x2(v[0], v[1]);
        o.y = pack_bf16x2(v[2], v[3]);
        o.z = pack_bf16x2(v[4], v[5]);
        o.w = pack_bf16x2(v[6], v[7]);
        *reinterpret_cast<uint4*>(bt + swz128(p, c)) = o;
      }
      fence_proxy_async_smem();
      mbar_arrive(&S.full_b[s]);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");

    // ---------------- epilogue from TMEM
    const bool ok = mbar_wait_ns(S.acc_full, 0, SSB_WAIT_NS);
    tc_fence_after();
    const int q = (warp - PROD_WARP0) & 3, half = (warp - PROD_WARP0) >> 2;
    const int orow = S.orow[32 * q + lane];
    const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16);
    // the shared expert follows the reference's bf16 rounding between ops (model/moe_sweep.py:37-43)
    const bool shared_e = e == a.shared_local;
    if (!ok) {
      s_fail = 1;
    } else if (EPI == EPI_SWIGLU && shared_e) {
      uint16_t* out = (uint16_t*)a.out;
#pragma unroll 1
      for (int cc = 0; cc < 2; ++cc) {
        const int col = 64 * half + 32 * cc;
        float g[32], u[32];
        tmem_ld32(taddr + col, g);
        tmem_ld32(taddr + 128 + col, u);
        if (orow >= 0) {
          uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)orow * a.ldo + nb * (BN / 2) + col);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float h[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) {
              const float gb = round_bf16(g[8 * j + t]), ub = round_bf16(u[8 * j + t]);
              h[t] = round_bf16(gb / (1.f + expf(-gb))) * ub;   // bf16(silu(bf16 g)) * bf16 u -> bf16 below
            }
            dst[j] = make_uint4(pack_bf16x2(h[0], h[1]), pack_bf16x2(h[2], h[3]), pack_bf16x2(h[4], h[5]),
                                pack_bf16x2(h[6], h[7]));
          }
        }
      }
    } else if (EPI == EPI_SWIGLU) {
      uint16_t* out = (uint16_t*)a.out;
#pragma unroll 1
      for (int cc = 0; cc < 2; ++cc) {
        const int col = 64 * half + 32 * cc;
        float g[32], u[32];
        tmem_ld32(taddr + col, g);
        tmem_ld32(taddr + 128 + col, u);
        if (orow >= 0) {
          uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)orow * a.ldo + nb * (BN / 2) + col);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float h[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) {
              const float gg = g[8 * j + t];
              h[t] = gg / (1.f + expf(-gg)) * u[8 * j + t];   // silu(g) * u, kernels/fused_moe_affine.py:80
            }
            dst[j] = make_uint4(pack_bf16x2(h[0], h[1]), pack_bf16x2(h[2], h[3]), pack_bf16x2(h[4], h[5]),
                                pack_bf16x2(h[6], h[7]));
          }
        }
      }
    } else {
      float* out = (float*)a.out;
      const float wt = (EPI == EPI_SCALE && orow >= 0) ? a.row_weight[orow] : 1.f;
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        const int col = 128 * half + 32 * cc;
        float v[32];
        tmem_ld32(taddr + col, v);
        if (orow >= 0) {
          float4* dst = reinterpret_cast<float4*>(out + (int64_t)orow * a.ldo + nb * BN + col);
#pragma unroll
          if (EPI == EPI_SCALE && shared_e) {   // bf16(sigmoid gate * bf16(D h))
#pragma unroll
            for (int j = 0; j < 8; ++j)
              dst[j] = make_float4(round_bf16(wt * round_bf16(v[4 * j])), round_bf16(wt * round_bf16(v[4 * j + 1])),
                                   round_bf16(wt * round_bf16(v[4 * j + 2])),
                                   round_bf16(wt * round_bf16(v[4 * j + 3])));
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              float4 o;
              o.x = EPI == EPI_SCALE ? v[4 * j] * wt : v[4 * j];
              o.y = EPI == EPI_SCALE ? v[4 * j + 1] * wt : v[4 * j + 1];
              o.z = EPI == EPI_SCALE ? v[4 * j + 2] * wt : v[4 * j + 2];
              o.w = EPI == EPI_SCALE ? v[4 * j + 3] * wt : v[4 * j + 3];
              dst[j] = o;
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    if (s_fail) {   // let every issued MMA finish before the accumulator is released
      if (lane == 0) mbar_wait_ns(S.acc_full, 0, SSB_WAIT_NS);
      __syncwarp();
    }
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
  if (tid == 0 && s_fail) set_err(a.err, SSB_ERR_TIMEOUT);
}

int launch(int epi, const GemmArgs& a, int64_t n_mblocks, int n_nblocks, cudaStream_t st) {
  void (*k)(GemmArgs) = epi == EPI_SWIGLU ? k_moe_gemm<EPI_SWIGLU> : epi == EPI_SCALE ? k_moe_gemm<EPI_SCALE>
                                                                                      : k_moe_gemm<EPI_PLAIN>;
  if (n_mblocks <= 0) return SSB_OK;
  if (n_mblocks > 65535 * 16) return SSB_EUNSUPPORTED;
  static bool attr_set[3] = {false, false, false};
  if (!attr_set[epi]) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
    if (e != cudaSuccess) return (int)e;
    attr_set[epi] = true;
  }
  ssb_note_smem(epi == EPI_SWIGLU ? "fused_moe_gate_up" : epi == EPI_SCALE ? "fused_moe_down" : "gemm_affine4", k,
                SMEM_BYTES);
  if (n_mblocks > 65535) return SSB_EUNSUPPORTED;
  return ssb_launch(k, dim3(n_nblocks, (unsigned)n_mblocks), dim3(THREADS), SMEM_BYTES, st, true, a);
}

void set_record_offsets(GemmArgs& g, int hidden, int inter, bool gate_up) {
  RecOffs o = rec_offsets(hidden, inter, 64);
  if (gate_up) {
    g.off_w[0] = o.gw;
    g.off_s[0] = o.gsc;
    g.off_b[0] = o.gb;
    g.off_w[1] = o.uw;
    g.off_s[1] = o.usc;
    g.off_b[1] = o.ub;
  } else {
    g.off_w[0] = g.off_w[1] = o.dw;
    g.off_s[0] = g.off_s[1] = o.dsc;
    g.off_b[0] = g.off_b[1] = o.db;
  }
}

int gate_up_impl(const uint16_t* x, int32_t hidden, int32_t inter, const int32_t* row_token, int64_t rows,
                 const int32_t* sorted_rows, const int32_t* block_expert, const int32_t* num_padded,
                 int64_t padded_len, const int64_t* group_ptr, int32_t n_groups, int32_t shared_local,
                 uint16_t* h_buf, int32_t* err, void* stream) {
  SSB_CHECK_ARG(rows >= 0 && padded_len >= 0 && n_groups >= 1);
  if (hidden % BK || hidden <= 0 || inter % (BN / 2) || inter <= 0 || (hidden / 64) % 2) return SSB_EUNSUPPORTED;
  if (padded_len == 0 || rows == 0) return SSB_OK;
  SSB_CHECK_ARG(x && row_token && sorted_rows && block_expert && num_padded && group_ptr && h_buf);
  SSB_CHECK_ARG(padded_len % BM == 0);
  GemmArgs g{};
  g.a = x;
  g.lda = hidden;
  g.row_token = row_token;
  g.sorted_rows = sorted_rows;
  g.block_expert = block_expert;
  g.num_padded = num_padded;
  g.R = rows;
  g.group_base = group_ptr;
  g.n_groups = n_groups;
  set_record_offsets(g, hidden, inter, true);
  g.K = hidden;
  g.gs = 64;
  g.shared_local = shared_local;
  g.out = h_buf;
  g.ldo = inter;
  g.err = err;
  return launch(EPI_SWIGLU, g, padded_len / BM, inter / (BN / 2), (cudaStream_t)stream);
}

int down_impl(const uint16_t* h_buf, int64_t rows, int32_t hidden, int32_t inter, const float* row_weight,
              const int32_t* sorted_rows, const int32_t* block_expert, const int32_t* num_padded, int64_t padded_len,
              const int64_t* group_ptr, int32_t n_groups, int32_t shared_local, float* out_rows, int32_t* err,
              void* stream) {
  SSB_CHECK_ARG(rows >= 0 && padded_len >= 0 && n_groups >= 1);
  if (inter % BK || inter <= 0 || hidden % BN || hidden <= 0 || (inter / 64) % 2) return SSB_EUNSUPPORTED;
  if (padded_len == 0 || rows == 0) return SSB_OK;
  SSB_CHECK_ARG(h_buf && row_weight && sorted_rows && block_expert && num_padded && group_ptr && out_rows);
  SSB_CHECK_ARG(padded_len % BM == 0);
  GemmArgs g{};
  g.a = h_buf;
  g.lda = inter;
  g.sorted_rows = sorted_rows;
  g.block_expert = block_expert;
  g.num_padded = num_padded;
  g.R = rows;
  g.group_base = group_ptr;
  g.n_groups = n_groups;
  set_record_offsets(g, hidden, inter, false);
  g.K = inter;
  g.gs = 64;
  g.shared_local = shared_local;
  g.row_weight = row_weight;
  g.out = out_rows;
  g.ldo = hidden;
  g.err = err;
  return launch(EPI_SCALE, g, padded_len / BM, hidden / BN, (cudaStream_t)stream);
}

}  // namespace

extern "C" int ssb_fused_moe_gate_up(const uint16_t* x, int64_t tokens, int32_t hidden, int32_t inter,
                                     const int32_t* row_token, int64_t rows, const int32_t* sorted_rows,
                                     const int32_t* block_expert, const int32_t* num_padded, int64_t padded_len,
                                     const int64_t* group_ptr, int32_t n_groups, uint16_t* h_buf, int32_t* err,
                                     void* stream) {
  SSB_CHECK_ARG(tokens >= 0);
  return gate_up_impl(x, hidden, inter, row_token, rows, sorted_rows, block_expert, num_padded, padded_len, group_ptr,
                      n_groups, -1, h_buf, err, stream);
}

extern "C" int ssb_fused_moe_down(const uint16_t* h_buf, int64_t rows, int32_t hidden, int32_t inter,
                                  const float* row_weight, const int32_t* sorted_rows, const int32_t* block_expert,
                                  const int32_t* num_padded, int64_t padded_len, const int64_t* group_ptr,
                                  int32_t n_groups, float* out_rows, int32_t* err, void* stream) {
  return down_impl(h_buf, rows, hidden, inter, row_weight, sorted_rows, block_expert, num_padded, padded_len,
                   group_ptr, n_groups, -1, out_rows, err, stream);
}

extern "C" int ssb_prefill_experts(const uint16_t* x, int32_t hidden, int32_t inter, const int32_t* row_token,
                                   const float* row_weight, int64_t rows, const int32_t* sorted_rows,
                                   const int32_t* block_expert, const int32_t* num_padded, int64_t padded_len,
                                   const int64_t* group_ptr, int32_t n_groups, int32_t shared_local, uint16_t* h_buf,
                                   float* out_rows, int32_t* err, void* stream) {
  int rc = gate_up_impl(x, hidden, inter, row_token, rows, sorted_rows, block_expert, num_padded, padded_len,
                        group_ptr, n_groups, shared_local, h_buf, err, stream);
  if (rc) return rc;
  return down_impl(h_buf, rows, hidden, inter, row_weight, sorted_rows, block_expert, num_padded, padded_len,
                   group_ptr, n_groups, shared_local, out_rows, err, stream);
}

extern "C" int ssb_gemm_affine4(const uint16_t* x, int64_t m, int32_t k, const int32_t* q, const uint16_t* s,
                                const uint16_t* b, int32_t n, int32_t gs, float* out, void* stream) {
  SSB_CHECK_ARG(m >= 0 && k >= 1 && n >= 1 && (gs == 32 || gs == 64));
  if (k % BK || n % BN || (k / gs) % 2) return SSB_EUNSUPPORTED;
  if (m == 0) return SSB_OK;
  SSB_CHECK_ARG(x && q && s && b && out);
  SSB_CHECK_ARG((((uintptr_t)q | (uintptr_t)s | (uintptr_t)b) & 3) == 0 && ((uintptr_t)q & 15) == 0);
  // one "expert" whose base is q; scale and bias are addressed relative to it
  GemmArgs g{};
  g.a = x;
  g.lda = k;
  g.R = m;
  g.base0 = (const uint8_t*)q;
  g.n_groups = 1;
  g.K = k;
  g.gs = gs;
  g.shared_local = -1;
  g.out = out;
  g.ldo = n;
  g.off_w[0] = g.off_w[1] = 0;
  g.off_s[0] = g.off_s[1] = (int64_t)((const uint8_t*)s - (const uint8_t*)q);
  g.off_b[0] = g.off_b[1] = (int64_t)((const uint8_t*)b - (const uint8_t*)q);
  g.err = nullptr;
  return launch(EPI_PLAIN, g, (m + BM - 1) / BM, n / BN, (cudaStream_t)stream);
}

extern "C" int ssb_gemm_dense(const uint16_t* x, int64_t m, int32_t k, const uint16_t* w, int32_t n, float* out,
                              int64_t ldo, void* stream) {
  SSB_CHECK_ARG(m >= 0 && k >= 1 && n >= 1 && ldo >= n && ldo % 4 == 0);
  if (k % BK || n % BN || k % 8) return SSB_EUNSUPPORTED;
  if (m == 0) return SSB_OK;
  SSB_CHECK_ARG(x && w && out && ((uintptr_t)w & 15) == 0 && ((uintptr_t)x & 15) == 0);
  GemmArgs g{};
  g.a = x;
  g.lda = k;
  g.R = m;
  g.base0 = (const uint8_t*)w;
  g.n_groups = 1;
  g.K = k;
  g.gs = 64;
  g.dense_b = 1;
  g.ldb = k;
  g.shared_local = -1;
  g.out = out;
  g.ldo = ldo;
  g.err = nullptr;
  return launch(EPI_PLAIN, g, (m + BM - 1) / BM, n / BN, (cudaStream_t)stream);
}
