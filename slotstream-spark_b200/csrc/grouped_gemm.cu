// Grouped affine-4-bit GEMM on the 5th-generation tensor cores (tcgen05 + TMEM) for the prefill MoE
// (slotstream_spark/kernels/fused_moe_affine.py:53-127) and the dense prefill GEMMs (kernels/gemm_affine.py).
//
// Tiles are 256 rows (two 128-row halves of one expert's rows; moe_align pads each expert to 256) x 128 B-rows.
// Every k-block's dequantised B tile feeds two M128xN128 MMAs, one per half, so the weight producers -- the
// bottleneck of a fused-dequant GEMM -- do half the work per FLOP of a 128-row tile:
//  * gate_up: the 128 B-rows are 64 gate rows + 64 up rows of the same inter columns, so each accumulator
//    holds both and the epilogue forms h = silu(g) * u -> bf16 (kernels/fused_moe_affine.py:76-81);
//  * down / plain: 128 output columns; the epilogue scales by the row's routing weight (fp32 out,
//    kernels/fused_moe_affine.py:103-108) or stores plain fp32 (kernels/gemm_affine.py:19-37).
// The kernel is persistent: one CTA per SM walks tiles t = blockIdx.x, blockIdx.x + gridDim.x, ... (m-block
// major, so concurrent CTAs share activation rows and expert weights in L2). TMEM holds two accumulator pairs,
// so the epilogue of tile i overlaps the MMAs of tile i+1, and the operand pipelines run across tile borders.
// Warp roles (16 warps):
//  * warp 0      loads the tile's activation rows with TMA: one 2-D box of 256 rows (128 when the second half
//                holds only padding rows) when the rows are contiguous (permuted into expert order beforehand),
//                else lane l gathers rows 4l..4l+3 and 128+4l.. with two tile::gather4 copies; the tensor map
//                applies the 128-byte swizzle. A second half of only padding rows is skipped by every role (not
//                loaded on the box path, not multiplied, not stored);
//  * warp 1      owns TMEM (512 columns) and issues tcgen05.mma (M128 N128 K16, eight per 64-wide k-block);
//  * warps 4..7  epilogue: TMEM -> registers -> global, one accumulator row per thread;
//  * warps 8..15 weight producers, two threads per B-row (one half of the k-block each): stage the packed
//                nibbles and the bf16 scale/bias with cp.async,
//                dequantise q*s + b -> bf16 (the reference kernel's _wtile, kernels/fused_moe_affine.py:38-50,
//                whose q * sc + bi compiles to a fused multiply-add) into the swizzled B tile; or, for bf16
//                weights, cp.async the row straight into the tile.
// Stages are handed over with mbarriers; every wait gives up after a bounded time and sets SSB_ERR_TIMEOUT
// instead of hanging. A row's result depends only on that row and that expert's bytes: the k order is fixed,
// so any row count or group composition gives the same bits.
#include "registry.h"
#include "tc_common.cuh"

namespace {

constexpr int BM = 128, MT = 2, TM = BM * MT, BK = 64, BN = 128;
constexpr int STAGES = 3;        // A/B operand stages
constexpr int SS = 4;            // k-blocks of one weight super-step (one coalesced load of the codes): 4, or 2
                                 // when the k-block count is not a multiple of 4
constexpr int THREADS = 512;
constexpr int A_WARP = 0, MMA_WARP = 1, EPI_WARP0 = 4, PROD_WARP0 = 8, N_PROD = 256;
constexpr uint32_t A_STAGE = TM * 128;           // 32 KB: two 128-row halves
constexpr uint32_t A_HALF = BM * 128;
constexpr uint32_t B_STAGE = BN * 128;           // 16 KB
constexpr uint32_t W_STG = BN * SS * 32;         // codes of a super-step: 128 rows x 128 B, 16-byte pieces swizzled
constexpr uint32_t SB_STG = N_PROD * 32;         // per producer thread: its row's scales (16 B) and biases (16 B)
constexpr uint32_t STG = W_STG + SB_STG;         // one staging slot; two slots alternate
constexpr int EPI_LD = 36;                        // fp32 epilogue transpose buffer: 32 rows of 32 (+4) floats
constexpr uint32_t EPI_BYTES = 4 * 32 * EPI_LD * 4;   // one buffer per epilogue warp
constexpr uint32_t TMEM_COLS = 512;              // 2 buffers x 2 halves of M128 x N128 fp32 accumulators

enum { EPI_SWIGLU = 0, EPI_SCALE = 1, EPI_PLAIN = 2 };

struct GemmArgs {
  const uint16_t* a;          // bf16 activation rows, `lda` elements apart (read through the A tensor map)
  int64_t lda;
  int64_t a_rows;             // rows of the activation matrix (extent of the tensor map)
  int a_box_rows;             // rows per A copy: 1 (tile::gather4 of four rows) or TM (one 2-D box, identity rows)
  int out_sorted;             // SwiGLU epilogue: h row at the sorted position m instead of at row sorted_rows[m]
  int kperm;                  // operands in the K order (0,4,1,5,2,6,3,7) inside every group of 8 (sorted path):
                              // B is dequantised in bf16x2 pairs, A and the h written here follow that order
  const int32_t* row_token;   // nullable: the A row of row r is r
  const int32_t* sorted_rows; // nullable: identity (rows m < R)
  const int32_t* block_expert;
  const int32_t* num_padded;  // nullable: n_mblocks blocks
  int64_t n_mblocks;
  int n_nblocks;
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
  int64_t n_valid;            // plain epilogue: output columns (B rows) that exist; the last n-block is partial
  int out_vec;                // plain epilogue: out and ldo allow 16-byte stores
  int32_t* err;
};

struct Smem {
  uint8_t* a;
  uint8_t* b;
  uint8_t* stg;
  float* epi;
  uint64_t* full_a;
  uint64_t* full_b;
  uint64_t* empty;
  uint64_t* tmem_full;    // [2]
  uint64_t* tmem_empty;   // [2]
  uint32_t* tmem;
};

constexpr size_t SMEM_BYTES = 1024 + STAGES * (A_STAGE + B_STAGE) + 2 * STG + EPI_BYTES + 8 * (3 * STAGES + 4) + 16;

SSB_DEV Smem carve(uint8_t* raw) {
  Smem s;
  uint8_t* p = (uint8_t*)(((uintptr_t)raw + 1023) & ~(uintptr_t)1023);
  s.a = p;
  p += STAGES * A_STAGE;
  s.b = p;
  p += STAGES * B_STAGE;
  s.stg = p;
  p += 2 * STG;
  s.epi = (float*)p;
  p += EPI_BYTES;
  s.full_a = (uint64_t*)p;
  s.full_b = s.full_a + STAGES;
  s.empty = s.full_b + STAGES;
  s.tmem_full = s.empty + STAGES;
  s.tmem_empty = s.tmem_full + 2;
  p += 8 * (3 * STAGES + 4);
  s.tmem = (uint32_t*)p;
  return s;
}

// Hardware round-to-nearest-even of two floats into packed bf16 (lo in the low half).
SSB_DEV uint32_t cvt_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// 8 nibbles of w -> 8 bf16 values fma(q, s, b) in one uint4. The magic-number floats are q * 16^j' exactly;
// sc2 holds s * 16^-j' for the matching lanes, so each product is formed exactly before the fused add.
SSB_DEV uint4 dequant8(uint32_t w, const float2* sc2, float2 b2) {
  const uint32_t M = 0x4B000000u;
  const uint32_t w5 = w >> 12;
  const float2 m2 = make_float2(-8388608.f, -8388608.f);
  float2 f0 = make_float2(__uint_as_float((w & 0xFu) | M), __uint_as_float((w & 0xF0u) | M));
  float2 f1 = make_float2(__uint_as_float((w & 0xF00u) | M), __uint_as_float((w & 0xF000u) | M));
  float2 f2 = make_float2(__uint_as_float((w & 0xF0000u) | M), __uint_as_float((w5 & 0xF00u) | M));
  float2 f3 = make_float2(__uint_as_float((w5 & 0xF000u) | M), __uint_as_float((w5 & 0xF0000u) | M));
  f0 = __ffma2_rn(__fadd2_rn(f0, m2), sc2[0], b2);
  f1 = __ffma2_rn(__fadd2_rn(f1, m2), sc2[1], b2);
  f2 = __ffma2_rn(__fadd2_rn(f2, m2), sc2[2], b2);
  f3 = __ffma2_rn(__fadd2_rn(f3, m2), sc2[3], b2);
  return make_uint4(cvt_bf16x2(f0.x, f0.y), cvt_bf16x2(f1.x, f1.y), cvt_bf16x2(f2.x, f2.y), cvt_bf16x2(f3.x, f3.y));
}

// 8 nibbles of w -> bf16 q*s + b in the K order (0,4,1,5,2,6,3,7): (w >> 4j) & 0x000F000F | 0x43004300 is the bf16
// pair (128 + q_j, 128 + q_{j+4}); one bf16x2 FMA removes the 128 exactly, a second forms q*s + b with a single
// rounding to bf16 (the value the reference's fp32 q*s + b rounds to whenever that sum is exact in fp32, as it
// is for these 4-bit codes and bf16 scales and biases of similar size).
SSB_DEV uint32_t hfma2_bf16(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
SSB_DEV uint4 dequant8_perm(uint32_t w, uint32_t s2, uint32_t b2) {
  const uint32_t MAG = 0x43004300u, ONE = 0x3F803F80u, M128 = 0xC300C300u;
  const uint32_t p0 = (w & 0x000F000Fu) | MAG, p1 = ((w >> 4) & 0x000F000Fu) | MAG;
  const uint32_t p2 = ((w >> 8) & 0x000F000Fu) | MAG, p3 = ((w >> 12) & 0x000F000Fu) | MAG;
  return make_uint4(hfma2_bf16(hfma2_bf16(p0, ONE, M128), s2, b2), hfma2_bf16(hfma2_bf16(p1, ONE, M128), s2, b2),
                    hfma2_bf16(hfma2_bf16(p2, ONE, M128), s2, b2), hfma2_bf16(hfma2_bf16(p3, ONE, M128), s2, b2));
}
// bf16 pairs (lo, hi) of 8 consecutive values -> the same 8 values in the K order (0,4,1,5,2,6,3,7)
SSB_DEV uint4 kperm8(uint4 v) {
  return make_uint4(__byte_perm(v.x, v.z, 0x5410), __byte_perm(v.x, v.z, 0x7632), __byte_perm(v.y, v.w, 0x5410),
                    __byte_perm(v.y, v.w, 0x7632));
}

SSB_DEV void scales2(float s, float2* sc2) {
  const float s1 = s * 0.0625f, s2 = s * 0.00390625f, s3 = s * 0.000244140625f, s4 = s * 1.52587890625e-05f;
  sc2[0] = make_float2(s, s1);
  sc2[1] = make_float2(s2, s3);
  sc2[2] = make_float2(s4, s2);
  sc2[3] = make_float2(s3, s4);
}

SSB_DEV float silu_fast(float g) { return __fdividef(g, 1.f + __expf(-g)); }

// h = silu(g) * u for 32 accumulator columns -> 32 bf16 in four uint4, in the K order (0,4,1,5,2,6,3,7) of every
// 8 (KPERM) or in column order. SHARED: the shared expert's chain bf16(silu(bf16 g)) * bf16 u (model/moe_sweep.py:
// 37-43); routed rows: accg / (1 + exp(-accg)) * accu (kernels/fused_moe_affine.py:80). The two are separate
// instantiations so that a routed tile carries none of the shared chain's instructions (an exact expf and an IEEE
// division per element, which a per-element select would otherwise execute for every tile).
template <bool SHARED>
SSB_DEV void swiglu32(const float* g, const float* u, bool kperm, uint4* out4) {
  float hv[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    if (SHARED) {
      const float gb = round_bf16(g[i]);
      hv[i] = round_bf16(gb / (1.f + expf(-gb))) * round_bf16(u[i]);
    } else {
      hv[i] = silu_fast(g[i]) * u[i];
    }
  }
#pragma unroll
  for (int jj = 0; jj < 4; ++jj) {
    const float* v = hv + 8 * jj;
    out4[jj] = kperm ? make_uint4(cvt_bf16x2(v[0], v[4]), cvt_bf16x2(v[1], v[5]), cvt_bf16x2(v[2], v[6]),
                                  cvt_bf16x2(v[3], v[7]))
                     : make_uint4(cvt_bf16x2(v[0], v[1]), cvt_bf16x2(v[2], v[3]), cvt_bf16x2(v[4], v[5]),
                                  cvt_bf16x2(v[6], v[7]));
  }
}

SSB_DEV bool gather_path(const GemmArgs& a) { return a.a_box_rows != TM; }

template <int EPI>
__global__ void __launch_bounds__(THREADS, 1) k_moe_gemm(const __grid_constant__ CUtensorMap tm_a,
                                                          const __grid_constant__ CUtensorMap tm_h, GemmArgs a) {
  extern __shared__ uint8_t smraw[];
  Smem S = carve(smraw);
  __shared__ int s_fail;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_wait();
  pdl_trigger();
  const int NB = a.n_nblocks;
  const int64_t n_mb = a.num_padded ? (int64_t)__ldcg(a.num_padded) / TM : a.n_mblocks;
  const int64_t n_tiles = n_mb * NB;
  if ((int64_t)blockIdx.x >= n_tiles) return;
  const int my_tiles = (int)((n_tiles - blockIdx.x + gridDim.x - 1) / gridDim.x);
  const int KB = a.K / BK;
  const int64_t steps = (int64_t)my_tiles * KB;
  auto tile_of = [&](int i) -> int64_t { return (int64_t)blockIdx.x + (int64_t)i * gridDim.x; };
  // local expert and weight base of 256-row block mb (nullptr: unusable, its B tile is zero)
  auto expert_of = [&](int64_t mb) -> int { return a.block_expert ? __ldcg(a.block_expert + mb) : 0; };
  auto base_of = [&](int e) -> const uint8_t* {
    if (e < 0 || e >= a.n_groups) return nullptr;
    const uint8_t* b = a.group_base ? (const uint8_t*)__ldg(a.group_base + e) : a.base0;
    return ((uintptr_t)b & 15) ? nullptr : b;
  };
  // does the second 128-row half of 256-row block mb hold any row? moe_align puts an expert's rows first and its
  // padding after them, so the half is all padding when its first row is (identity rows: when it is past R); such a
  // half is neither loaded (box path), multiplied nor stored
  // (the single MMA thread fetches the next tile's answer a tile ahead as a raw row id and tests it only when that
  // tile starts, so the load's latency never stalls the issue of MMAs)
  auto half1_row = [&](int64_t mb) -> int64_t {
    const int64_t m1 = mb * TM + BM;
    return a.sorted_rows ? (int64_t)__ldcg(a.sorted_rows + m1) : m1;
  };
  auto half1_ok = [&](int64_t r) -> bool { return r >= 0 && r < a.R; };
  auto half1_of = [&](int64_t mb) -> bool { return half1_ok(half1_row(mb)); };

  if (tid == 0) {
    s_fail = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&S.full_a[s], 1);
      mbar_init(&S.full_b[s], N_PROD);
      mbar_init(&S.empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.tmem_full[i], 1);
      mbar_init(&S.tmem_empty[i], 4);
    }
    fence_mbar_init();
  }
  if (warp == MMA_WARP) tmem_alloc(S.tmem, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *S.tmem;

  if (warp == A_WARP) {
    // ---------------- activation rows: one 2-D box (identity rows) or 64 tile::gather4 copies per k-block
    // Gathered rows: tile rows 4*lane .. +3 and 128 + 4*lane .. +3 come from sorted_rows, then row_token; the
    // next tile's lookups start during the current tile (sorted_rows at its first k-block, row_token at its
    // second) so the two dependent loads do not stall the copies at tile borders. Padding rows read row 0.
    int32_t rc[8], nrc[8], nsr[8];
    auto load_rows = [&](int i) {
      const int64_t mb = tile_of(i) / NB;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int64_t m = mb * TM + (q >> 2) * BM + 4 * lane + (q & 3);
        nsr[q] = a.sorted_rows ? __ldcg(a.sorted_rows + m) : (int32_t)m;
      }
    };
    auto to_coords = [&]() {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const bool ok = nsr[q] >= 0 && nsr[q] < a.R;
        nrc[q] = ok ? (a.row_token ? __ldcg(a.row_token + nsr[q]) : nsr[q]) : 0;
      }
    };
    int64_t issued = 0;
    if (lane == 0) {
      prefetch_tensormap(&tm_a);
      if (!gather_path(a)) prefetch_tensormap(&tm_h);
    }
    const bool gather = a.a_box_rows != TM;
    int64_t h_tile = -1;
    bool two = true;                    // box path: the second half of this tile is loaded
    int64_t r_next = 0;                 // first row of the next tile's second half
    if (gather) {
      load_rows(0);
      to_coords();
    }
    int kb = 0, i = 0;   // k-block and tile of step j, kept incrementally (no 64-bit division per step)
    int32_t r0 = 0;
    for (int64_t j = 0; j < steps; ++j) {
      if (kb == 0) r0 = (int32_t)((tile_of(i) / NB) * TM);
      if (!gather) {
      } else if (kb == 0) {
#pragma unroll
        for (int q = 0; q < 8; ++q) rc[q] = nrc[q];
        if (i + 1 < my_tiles) {
          load_rows(i + 1);
          if (KB == 1) to_coords();
        }
      } else if (kb == 1 && i + 1 < my_tiles) {
        to_coords();
      }
      const int s = (int)(j % STAGES);
      const uint32_t ph = (uint32_t)((j / STAGES) & 1);
      bool ok = lane == 0 ? mbar_wait_ns(&S.empty[s], ph ^ 1, SSB_WAIT_NS) : true;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        s_fail = 1;
        break;
      }
      if (!gather && i != h_tile && lane == 0) {   // the next tile's answer is fetched a tile ahead
        h_tile = i;
        two = i == 0 ? half1_of(tile_of(0) / NB) : half1_ok(r_next);
        if (i + 1 < my_tiles) r_next = half1_row(tile_of(i + 1) / NB);
      }
      if (lane == 0) mbar_expect_tx(&S.full_a[s], gather || two ? A_STAGE : A_HALF);
      __syncwarp();
      if (!gather) {   // rows tile*256 .. +255 (or +127) of the activation matrix, one 128-row box per half
        if (lane == 0) {
          // both halves in one 256-row box (measurably faster than two 128-row boxes), else the first half alone
          tma_load_2d(smem_u32(S.a + s * A_STAGE), two ? &tm_a : &tm_h, kb * BK, r0, &S.full_a[s]);
        }
      } else {
        tma_gather4(smem_u32(S.a + s * A_STAGE + lane * 512), &tm_a, kb * BK, rc[0], rc[1], rc[2], rc[3],
                    &S.full_a[s]);
        tma_gather4(smem_u32(S.a + s * A_STAGE + A_HALF + lane * 512), &tm_a, kb * BK, rc[4], rc[5], rc[6], rc[7],
                    &S.full_a[s]);
      }
      ++issued;
      if (++kb == KB) {
        kb = 0;
        ++i;
      }
    }
    // no copy may still be writing shared memory when the CTA exits: wait for the last stages to land
    if (lane == 0)
      for (int64_t j = issued > STAGES ? issued - STAGES : 0; j < issued; ++j)
        mbar_wait_ns(&S.full_a[j % STAGES], (uint32_t)((j / STAGES) & 1), SSB_WAIT_NS);
    __syncwarp();
  } else if (warp == MMA_WARP) {
    // ---------------- single-thread MMA issue, double-buffered accumulators
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(BM, BN);
      int64_t j = 0;
      int64_t r_next = half1_row(tile_of(0) / NB);
      for (int i = 0; i < my_tiles && !s_fail; ++i) {
        const int nh = half1_ok(r_next) ? MT : 1;   // halves of this tile (its row fetched a tile ahead)
        if (i + 1 < my_tiles) r_next = half1_row(tile_of(i + 1) / NB);
        const int acc = i & 1;
        if (!mbar_wait_ns(&S.tmem_empty[acc], ((i >> 1) & 1) ^ 1, SSB_WAIT_NS)) {
          s_fail = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d0 = tmem + (uint32_t)(acc * MT) * BN;   // accumulators of the two halves: d0, d0 + BN
        bool ok = true;
        for (int kb = 0; kb < KB; ++kb, ++j) {
          const int s = (int)(j % STAGES);
          const uint32_t ph = (uint32_t)((j / STAGES) & 1);
          if (!mbar_wait_ns(&S.full_a[s], ph, SSB_WAIT_NS) || !mbar_wait_ns(&S.full_b[s], ph, SSB_WAIT_NS)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t db = umma_desc_sw128(smem_u32(S.b + s * B_STAGE));
#pragma unroll
          for (int h = 0; h < MT; ++h) {
            if (h >= nh) break;
            const uint64_t da = umma_desc_sw128(smem_u32(S.a + s * A_STAGE + h * A_HALF));
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              umma_bf16(d0 + h * BN, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc, (kb | k) != 0);
          }
          umma_commit(&S.empty[s]);
        }
        umma_commit(&S.tmem_full[acc]);
        if (!ok) {
          s_fail = 1;
          break;
        }
      }
    }
    __syncwarp();
  } else if (warp >= EPI_WARP0 && warp < EPI_WARP0 + 4) {
    // ---------------- epilogue: one accumulator row per thread, both halves of the tile
    const int q = warp & 3;
    for (int i = 0; i < my_tiles; ++i) {
      const int acc = i & 1;
      const int64_t t = tile_of(i), mb = t / NB;
      const int nb = (int)(t % NB);
      const bool shared_e = a.shared_local >= 0 && expert_of(mb) == a.shared_local;
      const int nh = half1_of(mb) ? MT : 1;
      int64_t rows[MT];
      float wts[MT];
#pragma unroll
      for (int h = 0; h < MT; ++h) {
        const int64_t m = mb * TM + h * BM + 32 * q + lane;
        rows[h] = a.sorted_rows ? (int64_t)__ldcg(a.sorted_rows + m) : m;
        const bool valid = rows[h] >= 0 && rows[h] < a.R;
        wts[h] = (EPI == EPI_SCALE && valid) ? __ldcg(a.row_weight + rows[h]) : 1.f;
      }
      const bool ok = mbar_wait_ns(&S.tmem_full[acc], (i >> 1) & 1, SSB_WAIT_NS);
      tc_fence_after();
      if (!ok) {
        s_fail = 1;
        break;
      }
#pragma unroll 1
      for (int h = 0; h < nh; ++h) {
        const int64_t m = mb * TM + h * BM + 32 * q + lane;
        const int64_t row = rows[h];
        const bool valid = row >= 0 && row < a.R;
        const float wt = wts[h];
        const uint32_t taddr = tmem + (uint32_t)(acc * MT + h) * BN + ((uint32_t)(32 * q) << 16);
        if (EPI == EPI_SWIGLU) {
          uint16_t* out = (uint16_t*)a.out;
#pragma unroll 1
          for (int cc = 0; cc < BN / 64; ++cc) {
            const int col = 32 * cc;
            float g[32], u[32];
            tmem_ld32(taddr + col, g);
            tmem_ld32(taddr + BN / 2 + col, u);
            if (valid) {
              uint4* dst =
                  reinterpret_cast<uint4*>(out + (a.out_sorted ? m : row) * a.ldo + (int64_t)nb * (BN / 2) + col);
              uint4 pk[4];
              if (shared_e) swiglu32<true>(g, u, a.kperm, pk);
              else swiglu32<false>(g, u, a.kperm, pk);
#pragma unroll
              for (int jj = 0; jj < 4; ++jj) dst[jj] = pk[jj];
            }
          }
        } else {
          // fp32 rows: each 32-row x 32-column chunk goes through this warp's transpose buffer so that eight
          // lanes store one row's 128 contiguous bytes (four rows per store instruction) instead of every lane
          // storing 16 bytes of its own row
          float* out = (float*)a.out;
          float* tb = S.epi + q * (32 * EPI_LD);
#pragma unroll 1
          for (int cc = 0; cc < BN / 32; ++cc) {
            const int col = 32 * cc;
            float v[32];
            tmem_ld32(taddr + col, v);
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
              float4 o;
              if (EPI == EPI_SCALE && shared_e) {   // bf16(sigmoid gate * bf16(h D^T))
                o = make_float4(round_bf16(wt * round_bf16(v[4 * jj])), round_bf16(wt * round_bf16(v[4 * jj + 1])),
                                round_bf16(wt * round_bf16(v[4 * jj + 2])), round_bf16(wt * round_bf16(v[4 * jj + 3])));
              } else if (EPI == EPI_SCALE) {
                o = make_float4(v[4 * jj] * wt, v[4 * jj + 1] * wt, v[4 * jj + 2] * wt, v[4 * jj + 3] * wt);
              } else {
                o = make_float4(v[4 * jj], v[4 * jj + 1], v[4 * jj + 2], v[4 * jj + 3]);
              }
              *reinterpret_cast<float4*>(tb + lane * EPI_LD + 4 * jj) = o;
            }
            __syncwarp();
#pragma unroll
            for (int it = 0; it < 8; ++it) {
              const int rr = 4 * it + (lane >> 3), c4 = 4 * (lane & 7);
              const int64_t rrow = __shfl_sync(0xFFFFFFFFu, row, rr);
              const float4 o = *reinterpret_cast<const float4*>(tb + rr * EPI_LD + c4);
              const int64_t c0 = (int64_t)nb * BN + col + c4;
              if (rrow >= 0 && rrow < a.R) {
                if (EPI != EPI_PLAIN || (a.out_vec && c0 + 4 <= a.n_valid)) {
                  *reinterpret_cast<float4*>(out + rrow * a.ldo + c0) = o;
                } else {   // a partial last n-block, or rows that 16-byte stores cannot address
                  const float ov[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
                  for (int e = 0; e < 4; ++e)
                    if (c0 + e < a.n_valid) out[rrow * a.ldo + c0 + e] = ov[e];
                }
              }
            }
            __syncwarp();
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.tmem_empty[acc]);   // the accumulator pair may be overwritten now
    }
  } else if (warp >= PROD_WARP0) {
    // ---------------- weight producers: B-row br = p / 2, half hf = p % 2 (elements 32hf .. 32hf+31 of the k-block)
    const int p = tid - PROD_WARP0 * 32;
    const int br = p >> 1, hf = p & 1;
    const int piece = (EPI == EPI_SWIGLU) ? (br >> 6) : 0;
    const int ng = a.K / a.gs;
    // weight base and B-row of this thread for the tile of step j, resolved once per tile (two dependent
    // L2 loads: block_expert, then the group's base); base nullptr: zero row
    int64_t t_tile = -1, t_nrow = 0;
    const uint8_t* t_base = nullptr;
    auto tile_info = [&](int64_t j) {
      const int64_t i = j / KB;
      if (i != t_tile) {
        t_tile = i;
        const int64_t t = tile_of((int)i);
        const int64_t mb = t / NB;
        const int nb = (int)(t % NB);
        t_base = base_of(expert_of(mb));
        t_nrow = (EPI == EPI_SWIGLU) ? (int64_t)nb * (BN / 2) + (br & (BN / 2 - 1)) : (int64_t)nb * BN + br;
      }
    };
    if (a.dense_b) {
      // bf16 weights: cp.async straight into the swizzled tile, DB steps in flight; a step is handed to the MMA
      // only after this thread's copies landed and were made visible to the tensor core's (async) proxy
      constexpr int DB = STAGES - 1;
      bool fail = false;
      for (int64_t j = 0; j < steps + DB; ++j) {
        if (j < steps) {
          const int kb = (int)(j % KB);
          tile_info(j);
          const int s = (int)(j % STAGES);
          const uint32_t ph = (uint32_t)((j / STAGES) & 1);
          if (!mbar_wait_ns(&S.empty[s], ph ^ 1, SSB_WAIT_NS)) {
            s_fail = 1;
            fail = true;
          } else {
            const uint32_t bt = smem_u32(S.b + s * B_STAGE);
            const bool row_ok = t_base && (EPI != EPI_PLAIN || t_nrow < a.n_valid);   // rows past n read zeros
            const uint16_t* drow =
                row_ok ? (const uint16_t*)t_base + t_nrow * a.ldb + kb * BK : (const uint16_t*)a.base0;
#pragma unroll
            for (int c = 4 * hf; c < 4 * hf + 4; ++c) cp_async16(bt + swz128(br, c), drow + c * 8, row_ok ? 16u : 0u);
          }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        if (fail) break;
        if (j >= DB) {
          asm volatile("cp.async.wait_group %0;" ::"n"(DB) : "memory");
          fence_proxy_async_smem();
          mbar_arrive(&S.full_b[(j - DB) % STAGES]);
        }
      }
      asm volatile("cp.async.wait_all;" ::: "memory");
    } else {
      // Affine 4-bit weights, one super-step of SS k-blocks at a time. The 256 producers copy the tile's codes for
      // the super-step with coalesced 16-byte pieces (thread t: pieces t + 256i of the 128 rows x 128 B; a warp
      // covers four whole lines) into a staging slot whose pieces are XOR-swizzled by row, and each thread its
      // row's SS scales and biases. Named barriers over the producers order the two slots; every producer passes
      // every barrier, and a failed wait only raises this thread's flag, OR-reduced by the barrier that starts the
      // next super-step, so all producers leave together.
      const int ss = KB % SS == 0 ? SS : 2;   // k-blocks per super-step (KB is even)
      const int n_ss = (int)(steps / ss);
      const int gsb = (a.gs == 64 ? 2 : 4) * ss;   // bytes of scales (or biases) of a super-step per row
      const void* dummy = a.a;                // valid address for zero-byte copies (rows of an unusable expert)
      uint32_t slot_ok = 0;                   // bit (n & 1): super-step n's expert has a usable record
      int my_fail = 0;
      // The super-steps are issued in order; their tile, k-block and n-block follow from 32-bit counters, and the
      // next tile's record base is fetched ahead (its expert when a tile's first super-step is issued, its base in
      // the middle of the tile), so no issue waits on a division or on the dependent block_expert -> base chain.
      const int SPT = KB / ss, MID = SPT / 2;
      int is_T = 0, is_sub = -1, is_nb = 0, nb_nxt = 0;
      int32_t e_nxt = -1;
      const uint8_t* base_nxt = nullptr;
      auto nb_at = [&](int i) -> int { return (int)(((uint32_t)blockIdx.x + (uint32_t)i * gridDim.x) % (uint32_t)NB); };
      auto base_raw = [&](int e) -> const uint8_t* {
        if (e < 0 || e >= a.n_groups) return nullptr;
        return a.group_base ? (const uint8_t*)__ldg(a.group_base + e) : a.base0;
      };
      auto usable = [](const uint8_t* b) -> const uint8_t* { return ((uintptr_t)b & 15) ? nullptr : b; };
      auto advance = [&]() {
        if (++is_sub == SPT || is_sub == 0) {
          if (is_sub == SPT) ++is_T;
          is_sub = 0;
          t_base = is_T == 0 ? usable(base_raw(expert_of(tile_of(0) / NB))) : usable(base_nxt);
          is_nb = is_T == 0 ? nb_at(0) : nb_nxt;
          t_nrow = (EPI == EPI_SWIGLU) ? (int64_t)is_nb * (BN / 2) + (br & (BN / 2 - 1)) : (int64_t)is_nb * BN + br;
          if (is_T + 1 < my_tiles) {
            e_nxt = expert_of(tile_of(is_T + 1) / NB);
            nb_nxt = nb_at(is_T + 1);
          }
        }
        if (is_sub == MID && is_T + 1 < my_tiles) base_nxt = base_raw(e_nxt);
      };
      auto issue_ss = [&](int n) {
        advance();
        const int kb0 = is_sub * ss;
        uint8_t* st = S.stg + (n & 1) * STG;
        const int nb = is_nb;
#pragma unroll
        for (int i = 0; i < SS; ++i) {
          if (i >= ss) break;
          const int pc = p + N_PROD * i, row = pc / (2 * ss), c16 = pc - row * (2 * ss);
          const int pce = (EPI == EPI_SWIGLU) ? (row >> 6) : 0;
          const int64_t nr = (EPI == EPI_SWIGLU) ? (int64_t)nb * (BN / 2) + (row & (BN / 2 - 1)) : (int64_t)nb * BN + row;
          const bool row_ok = t_base && (EPI != EPI_PLAIN || nr < a.n_valid);   // rows past n read zero codes
          const void* src = row_ok ? (const void*)(t_base + a.off_w[pce] + nr * (a.K / 2) + kb0 * 32 + c16 * 16) : dummy;
          cp_async16(smem_u32(st + row * 128 + ((c16 ^ (row & 7)) << 4)), src, row_ok ? 16u : 0u);
        }
        const int g0 = a.gs == 64 ? kb0 : 2 * kb0;   // first group of the super-step (gsb-byte aligned)
        const bool sb_ok = t_base && (EPI != EPI_PLAIN || t_nrow < a.n_valid);   // rows past n: zero scale and bias
        const uint16_t* sr = sb_ok ? (const uint16_t*)(t_base + a.off_s[piece]) + t_nrow * ng + g0 : nullptr;
        const uint16_t* bsrc = sb_ok ? (const uint16_t*)(t_base + a.off_b[piece]) + t_nrow * ng + g0 : nullptr;
        const uint32_t ds = smem_u32(st + W_STG + p * 32);
        if (gsb == 4) {
          asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(ds), "l"(sr ? (const void*)sr : dummy),
                       "r"(sr ? 4 : 0) : "memory");
          asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(ds + 16),
                       "l"(bsrc ? (const void*)bsrc : dummy), "r"(bsrc ? 4 : 0) : "memory");
        } else if (gsb == 8) {
          asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(ds), "l"(sr ? (const void*)sr : dummy),
                       "r"(sr ? 8 : 0) : "memory");
          asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(ds + 16),
                       "l"(bsrc ? (const void*)bsrc : dummy), "r"(bsrc ? 8 : 0) : "memory");
        } else {
          cp_async16(ds, sr ? (const void*)sr : dummy, sr ? 16u : 0u);
          cp_async16(ds + 16, bsrc ? (const void*)bsrc : dummy, bsrc ? 16u : 0u);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        const uint32_t bit = 1u << (n & 1);
        slot_ok = t_base ? (slot_ok | bit) : (slot_ok & ~bit);
      };
      auto prod_sync = [&]() { asm volatile("bar.sync 1, %0;" ::"n"(N_PROD) : "memory"); };
      // barrier over the producers that also ORs every producer's failure flag (the same answer for all)
      auto prod_sync_any = [&](int flag) -> bool {
        uint32_t r;
        asm volatile(
            "{\n .reg .pred p;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred p, 1, %2, p;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(r)
            : "r"(flag), "n"(N_PROD)
            : "memory");
        return r != 0;
      };
      if (n_ss > 0) issue_ss(0);
      for (int n = 0; n < n_ss; ++n) {
        // every producer is done reading slot (n + 1) & 1 (super-step n - 1); stop together after any failure
        if (prod_sync_any(my_fail)) break;
        if (n + 1 < n_ss) {
          issue_ss(n + 1);
          asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
          asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        prod_sync();   // every producer's copies of super-step n have landed
        const uint8_t* st = S.stg + (n & 1) * STG;
        const int64_t j0 = (int64_t)n * ss;
        const bool ok_row = (slot_ok >> (n & 1)) & 1u;
        if (!ok_row && p == 0) set_err(a.err, SSB_ERR_MISALIGNED);
        const uint4 sbq = *reinterpret_cast<const uint4*>(st + W_STG + p * 32);        // scales
        const uint4 bbq = *reinterpret_cast<const uint4*>(st + W_STG + p * 32 + 16);   // biases
        const uint32_t sq[4] = {sbq.x, sbq.y, sbq.z, sbq.w}, bq[4] = {bbq.x, bbq.y, bbq.z, bbq.w};
#pragma unroll
        for (int u = 0; u < SS; ++u) {
          if (u >= ss) break;
          const int64_t j = j0 + u;
          const uint4 w = ok_row ? *reinterpret_cast<const uint4*>(st + br * 128 + (((2 * u + hf) ^ (br & 7)) << 4))
                                 : make_uint4(0, 0, 0, 0);
          // the scale / bias of this thread's 32 elements: group u of the super-step (gs 64), or 2u + hf (gs 32)
          const int gi = a.gs == 64 ? u : 2 * u + hf;
          const uint32_t sw = sq[gi >> 1], bw = bq[gi >> 1];
          const bool hi = gi & 1;
          const int s = (int)(j % STAGES);
          const uint32_t ph = (uint32_t)((j / STAGES) & 1);
          if (my_fail || !mbar_wait_ns(&S.empty[s], ph ^ 1, SSB_WAIT_NS)) {
            my_fail = 1;   // keep passing the producer barriers; the loop ends at the next super-step
            s_fail = 1;
            continue;
          }
          uint8_t* bt = S.b + s * B_STAGE;
          const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
          if (a.kperm) {
            const uint32_t s2 = ok_row ? __byte_perm(sw, 0, hi ? 0x3232 : 0x1010) : 0u;
            const uint32_t b2 = ok_row ? __byte_perm(bw, 0, hi ? 0x3232 : 0x1010) : 0u;
#pragma unroll
            for (int c = 0; c < 4; ++c)   // 16-byte chunk 4hf + c = elements 8(4hf + c) .. +7 = word c of this half
              *reinterpret_cast<uint4*>(bt + swz128(br, 4 * hf + c)) = dequant8_perm(ws[c], s2, b2);
          } else {
            float2 sc[4];
            scales2(ok_row ? (hi ? bf16_hi(sw) : bf16_lo(sw)) : 0.f, sc);
            const float bv = ok_row ? (hi ? bf16_hi(bw) : bf16_lo(bw)) : 0.f;
            const float2 bb = make_float2(bv, bv);
#pragma unroll
            for (int c = 0; c < 4; ++c)
              *reinterpret_cast<uint4*>(bt + swz128(br, 4 * hf + c)) = dequant8(ws[c], sc, bb);
          }
          fence_proxy_async_smem();
          mbar_arrive(&S.full_b[s]);
        }
      }
      asm volatile("cp.async.wait_all;" ::: "memory");
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    if (s_fail) {   // every committed MMA group finishes before the accumulators are released
      if (lane == 0) {
        mbar_wait_ns(&S.tmem_full[0], 0, SSB_WAIT_NS);
        if (my_tiles > 1) mbar_wait_ns(&S.tmem_full[1], 0, SSB_WAIT_NS);
      }
      __syncwarp();
    }
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
  if (tid == 0 && s_fail) set_err(a.err, SSB_ERR_TIMEOUT);
}

#include "gate_up_wide.cuh"

// x_sorted[m, :] = x[row_token[sorted_rows[m]], :] for m < num_padded (zero rows for padding), one warp per row:
// the activation rows in expert order, so the grouped GEMM reads its A tiles as whole 2-D boxes, with every group
// of 8 columns in the K order (0,4,1,5,2,6,3,7) in which the sorted GEMMs dequantise their weights.
constexpr int PERM_UNR = 8;   // 16-byte chunks per lane in flight in k_permute_rows

__global__ void __launch_bounds__(256) k_permute_rows(const uint4* __restrict__ x, int64_t x_rows, int64_t row_vecs,
                                                      const int32_t* __restrict__ row_token,
                                                      const int32_t* __restrict__ sorted_rows,
                                                      const int32_t* __restrict__ num_padded, int64_t R,
                                                      int64_t padded_len, uint4* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int64_t np = __ldcg(num_padded);
  const int64_t n = np < padded_len ? np : padded_len;
  const int64_t step = ((int64_t)gridDim.x * blockDim.x) >> 5;
  // the source token of a sorted row (-1: padding or a bad row)
  auto token_of = [&](int64_t m) -> int64_t {
    if (m >= n) return -1;
    const int64_t r = __ldcg(sorted_rows + m);
    const int64_t t = (r >= 0 && r < R) ? (int64_t)__ldcg(row_token + r) : -1;
    return t < x_rows ? t : -1;
  };
  int64_t m = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int64_t t = token_of(m);
  for (; m < n; m += step) {
    const int64_t t_next = token_of(m + step);   // the next row's index loads overlap this row's copy
    // each 16-byte chunk in the K order of the sorted GEMMs; eight chunks per lane in flight at once
    for (int64_t c0 = 0; c0 < row_vecs; c0 += 32 * PERM_UNR) {
      uint4 v[PERM_UNR];
#pragma unroll
      for (int j = 0; j < PERM_UNR; ++j) {
        const int64_t c = c0 + lane + 32 * j;
        v[j] = (t >= 0 && c < row_vecs) ? __ldg(x + t * row_vecs + c) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int j = 0; j < PERM_UNR; ++j) {
        const int64_t c = c0 + lane + 32 * j;
        if (c < row_vecs) out[m * row_vecs + c] = t >= 0 ? kperm8(v[j]) : make_uint4(0, 0, 0, 0);
      }
    }
    t = t_next;
  }
}

// Row-order variant used inside ssb_prefill_experts: pos[r] = sorted position of row r (-1: dropped), then one
// warp per row r in row order copies x[row_token[r]] to x_sorted[pos[r]]. Rows of one token are neighbours in
// row order, so each activation row comes from DRAM about once instead of once per expert; padding rows of
// x_sorted are not written (the GEMMs never store the results of padding rows).
__global__ void __launch_bounds__(256) k_row_pos(const int32_t* __restrict__ sorted_rows,
                                                 const int32_t* __restrict__ num_padded, int64_t R,
                                                 int64_t padded_len, int32_t* __restrict__ pos) {
  pdl_wait();
  pdl_trigger();
  const int64_t np = __ldcg(num_padded);
  const int64_t n = np < padded_len ? np : padded_len;
  for (int64_t m = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; m < n; m += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = __ldcg(sorted_rows + m);
    if (r >= 0 && r < R) pos[r] = (int32_t)m;
  }
}

__global__ void __launch_bounds__(256) k_permute_by_row(const uint4* __restrict__ x, int64_t x_rows, int64_t row_vecs,
                                                        const int32_t* __restrict__ row_token,
                                                        const int32_t* __restrict__ pos, int64_t R,
                                                        uint4* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int64_t step = ((int64_t)gridDim.x * blockDim.x) >> 5;
  auto dest_of = [&](int64_t r, int64_t& t) -> int64_t {
    if (r >= R) return -1;
    const int64_t m = __ldcg(pos + r);
    t = __ldg(row_token + r);
    return (m >= 0 && t >= 0 && t < x_rows) ? m : -1;
  };
  int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int64_t t = -1, m = dest_of(r, t);
  for (; r < R; r += step) {
    int64_t t_next = -1;
    const int64_t m_next = dest_of(r + step, t_next);   // the next row's index loads overlap this row's copy
    if (m >= 0) {
      for (int64_t c0 = 0; c0 < row_vecs; c0 += 32 * PERM_UNR) {
        uint4 v[PERM_UNR];
#pragma unroll
        for (int j = 0; j < PERM_UNR; ++j) {
          const int64_t c = c0 + lane + 32 * j;
          if (c < row_vecs) v[j] = __ldg(x + t * row_vecs + c);
        }
#pragma unroll
        for (int j = 0; j < PERM_UNR; ++j) {
          const int64_t c = c0 + lane + 32 * j;
          if (c < row_vecs) out[m * row_vecs + c] = kperm8(v[j]);
        }
      }
    }
    m = m_next;
    t = t_next;
  }
}

// SMs the persistent GEMM leaves free for kernels that run beside it (collectives on another stream); set by
// ssb_set_gemm_sm_reserve, read at each launch.
int g_sm_reserve = 0;
int g_gate_up_tile = 256;   // B-rows per tile of the sorted gate_up: 256 (k_gate_up_wide) or 128 (k_moe_gemm)

int num_sms() {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
  }
  return sms;
}

// The driver's tensor-map encoder, looked up through the runtime so the library needs no link-time libcuda.
using EncodeTiledFn = decltype(&cuTensorMapEncodeTiled);
EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// 2-D tensor map over the activation rows: K elements x a_rows rows, box 64 x box_rows, 128-byte swizzle: box_rows 1
// (gathered rows), TM (a 256-row block) or BM (its first half alone, when the second holds only padding).
int encode_a_map(CUtensorMap* map, const GemmArgs& a, int box_rows) {
  if (((uintptr_t)a.a & 15) || (a.lda * 2) % 16 || a.a_rows < 1 || a.a_rows > 0x7fffffffLL) return SSB_EINVAL;
  if (a.a_box_rows != 1 && a.a_box_rows != TM) return SSB_EINVAL;
  EncodeTiledFn encode = encode_tiled_fn();
  if (!encode) return SSB_ENODEVICE;
  cuuint64_t dims[2] = {(cuuint64_t)a.K, (cuuint64_t)a.a_rows};
  cuuint64_t strides[1] = {(cuuint64_t)a.lda * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void*)a.a, dims, strides, box, estr,
                                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SSB_OK : SSB_EINVAL;
}

int launch(int epi, GemmArgs a, int64_t n_mblocks, int n_nblocks, cudaStream_t st) {
  void (*k)(CUtensorMap, CUtensorMap, GemmArgs) = epi == EPI_SWIGLU ? k_moe_gemm<EPI_SWIGLU>
                                     : epi == EPI_SCALE ? k_moe_gemm<EPI_SCALE>
                                                        : k_moe_gemm<EPI_PLAIN>;
  if (n_mblocks <= 0) return SSB_OK;
  CUtensorMap tm, tmh;
  int rc = encode_a_map(&tm, a, a.a_box_rows);
  if (!rc) rc = encode_a_map(&tmh, a, a.a_box_rows == TM ? BM : 1);
  if (rc) return rc;
  static bool attr_set[3] = {false, false, false};
  if (!attr_set[epi]) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
    if (e != cudaSuccess) return (int)e;
    attr_set[epi] = true;
  }
  ssb_note_smem(epi == EPI_SWIGLU ? "fused_moe_gate_up" : epi == EPI_SCALE ? "fused_moe_down" : "gemm_tc", k,
                SMEM_BYTES);
  a.n_mblocks = n_mblocks;
  a.n_nblocks = n_nblocks;
  const int64_t tiles = n_mblocks * n_nblocks;
  int ctas = num_sms() - g_sm_reserve;
  if (ctas < 1) ctas = 1;
  const int grid = (int)(tiles < ctas ? tiles : ctas);
  return ssb_launch(k, dim3(grid), dim3(THREADS), SMEM_BYTES, st, true, tm, tmh, a);
}

// k_gate_up_wide over the sorted rows (x permuted into expert order, gs 64): tiles of 256 rows x 128 h columns.
int launch_gate_up_wide(GemmArgs a, int64_t n_mblocks, int n_nblocks, cudaStream_t st) {
  if (n_mblocks <= 0) return SSB_OK;
  if (a.gs != 64 || !a.kperm || !a.out_sorted || a.a_box_rows != TM || !a.sorted_rows || !a.num_padded ||
      !a.block_expert || !a.group_base)
    return SSB_EINVAL;
  CUtensorMap tm, tmh;
  int rc = encode_a_map(&tm, a, TM);
  if (!rc) rc = encode_a_map(&tmh, a, BM);
  if (rc) return rc;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(k_gate_up_wide, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)WG_SMEM_BYTES);
    if (e != cudaSuccess) return (int)e;
    attr_set = true;
  }
  ssb_note_smem("fused_moe_gate_up_wide", k_gate_up_wide, WG_SMEM_BYTES);
  a.n_mblocks = n_mblocks;
  a.n_nblocks = n_nblocks;
  const int64_t tiles = n_mblocks * n_nblocks;
  int ctas = num_sms() - g_sm_reserve;
  if (ctas < 1) ctas = 1;
  const int grid = (int)(tiles < ctas ? tiles : ctas);
  return ssb_launch(k_gate_up_wide, dim3(grid), dim3(THREADS), WG_SMEM_BYTES, st, true, tm, tmh, a);
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

int gate_up_impl(const uint16_t* x, int64_t tokens, int32_t hidden, int32_t inter, const int32_t* row_token,
                 int64_t rows,
                 const int32_t* sorted_rows, const int32_t* block_expert, const int32_t* num_padded,
                 int64_t padded_len, const int64_t* group_ptr, int32_t n_groups, int32_t shared_local,
                 uint16_t* h_buf, int32_t* err, void* stream, bool sorted = false) {
  SSB_CHECK_ARG(rows >= 0 && padded_len >= 0 && n_groups >= 1);
  if (hidden % (2 * BK) || hidden <= 0 || inter % (BN / 2) || inter <= 0) return SSB_EUNSUPPORTED;
  if (padded_len == 0 || rows == 0) return SSB_OK;
  SSB_CHECK_ARG(x && row_token && sorted_rows && block_expert && num_padded && group_ptr && h_buf);
  SSB_CHECK_ARG(padded_len % TM == 0);
  GemmArgs g{};
  g.a = x;
  g.lda = hidden;
  g.a_rows = sorted ? padded_len : tokens;   // sorted: x is the permuted [padded_len, hidden] matrix
  g.a_box_rows = sorted ? TM : 1;
  g.out_sorted = sorted;
  g.kperm = sorted;
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
  if (sorted && g_gate_up_tile == WG_BN && hidden % (WG_SS * BK) == 0 && inter % 128 == 0)
    return launch_gate_up_wide(g, padded_len / TM, inter / 128, (cudaStream_t)stream);
  return launch(EPI_SWIGLU, g, padded_len / TM, inter / (BN / 2), (cudaStream_t)stream);
}

int down_impl(const uint16_t* h_buf, int64_t rows, int32_t hidden, int32_t inter, const float* row_weight,
              const int32_t* sorted_rows, const int32_t* block_expert, const int32_t* num_padded, int64_t padded_len,
              const int64_t* group_ptr, int32_t n_groups, int32_t shared_local, float* out_rows, int32_t* err,
              void* stream, bool sorted = false) {
  SSB_CHECK_ARG(rows >= 0 && padded_len >= 0 && n_groups >= 1);
  if (inter % (2 * BK) || inter <= 0 || hidden % BN || hidden <= 0) return SSB_EUNSUPPORTED;
  if (padded_len == 0 || rows == 0) return SSB_OK;
  SSB_CHECK_ARG(h_buf && row_weight && sorted_rows && block_expert && num_padded && group_ptr && out_rows);
  SSB_CHECK_ARG(padded_len % TM == 0);
  GemmArgs g{};
  g.a = h_buf;
  g.lda = inter;
  g.a_rows = sorted ? padded_len : rows;     // sorted: h rows at their sorted positions
  g.a_box_rows = sorted ? TM : 1;
  g.kperm = sorted;
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
  return launch(EPI_SCALE, g, padded_len / TM, hidden / BN, (cudaStream_t)stream);
}

}  // namespace

extern "C" int ssb_fused_moe_gate_up(const uint16_t* x, int64_t tokens, int32_t hidden, int32_t inter,
                                     const int32_t* row_token, int64_t rows, const int32_t* sorted_rows,
                                     const int32_t* block_expert, const int32_t* num_padded, int64_t padded_len,
                                     const int64_t* group_ptr, int32_t n_groups, uint16_t* h_buf, int32_t* err,
                                     void* stream) {
  SSB_CHECK_ARG(tokens >= 0);
  return gate_up_impl(x, tokens, hidden, inter, row_token, rows, sorted_rows, block_expert, num_padded, padded_len, group_ptr,
                      n_groups, -1, h_buf, err, stream);
}

extern "C" int ssb_fused_moe_down(const uint16_t* h_buf, int64_t rows, int32_t hidden, int32_t inter,
                                  const float* row_weight, const int32_t* sorted_rows, const int32_t* block_expert,
                                  const int32_t* num_padded, int64_t padded_len, const int64_t* group_ptr,
                                  int32_t n_groups, float* out_rows, int32_t* err, void* stream) {
  return down_impl(h_buf, rows, hidden, inter, row_weight, sorted_rows, block_expert, num_padded, padded_len,
                   group_ptr, n_groups, -1, out_rows, err, stream);
}

int permute_impl(const uint16_t* x, int64_t tokens, int32_t hidden, const int32_t* row_token, int64_t rows,
                 const int32_t* sorted_rows, const int32_t* num_padded, int64_t padded_len, uint16_t* x_sorted,
                 cudaStream_t st) {
  SSB_CHECK_ARG(tokens >= 0 && rows >= 0 && padded_len >= 0 && hidden > 0 && hidden % 8 == 0);
  if (padded_len == 0) return SSB_OK;
  SSB_CHECK_ARG(x && row_token && sorted_rows && num_padded && x_sorted);
  SSB_CHECK_ARG((((uintptr_t)x | (uintptr_t)x_sorted) & 15) == 0);
  const int64_t blocks = (padded_len + 7) / 8;
  return ssb_launch(k_permute_rows, dim3((unsigned)(blocks < 148 * 8 ? blocks : 148 * 8)), dim3(256), 0, st, true,
                    (const uint4*)x, tokens, (int64_t)hidden / 8, row_token, sorted_rows, num_padded, rows, padded_len,
                    (uint4*)x_sorted);
}

// x_sorted through the row-order path; pos_ws (int32 [rows]) is scratch
int permute_by_row_impl(const uint16_t* x, int64_t tokens, int32_t hidden, const int32_t* row_token, int64_t rows,
                        const int32_t* sorted_rows, const int32_t* num_padded, int64_t padded_len, uint16_t* x_sorted,
                        int32_t* pos_ws, cudaStream_t st) {
  SSB_CHECK_ARG(tokens >= 0 && rows >= 0 && padded_len >= 0 && hidden > 0 && hidden % 8 == 0);
  if (padded_len == 0 || rows == 0) return SSB_OK;
  SSB_CHECK_ARG(x && row_token && sorted_rows && num_padded && x_sorted && pos_ws);
  SSB_CHECK_ARG((((uintptr_t)x | (uintptr_t)x_sorted) & 15) == 0);
  cudaError_t e = cudaMemsetAsync(pos_ws, 0xFF, (size_t)rows * 4, st);
  if (e != cudaSuccess) return (int)e;
  const int64_t pb = (padded_len + 255) / 256;
  int rc = ssb_launch(k_row_pos, dim3((unsigned)(pb < 148 * 8 ? pb : 148 * 8)), dim3(256), 0, st, false, sorted_rows,
                      num_padded, rows, padded_len, pos_ws);
  if (rc) return rc;
  const int64_t blocks = (rows + 7) / 8;
  return ssb_launch(k_permute_by_row, dim3((unsigned)(blocks < 148 * 8 ? blocks : 148 * 8)), dim3(256), 0, st, true,
                    (const uint4*)x, tokens, (int64_t)hidden / 8, row_token, (const int32_t*)pos_ws, rows,
                    (uint4*)x_sorted);
}

extern "C" int ssb_permute_rows(const uint16_t* x, int64_t tokens, int32_t hidden, const int32_t* row_token,
                                int64_t rows, const int32_t* sorted_rows, const int32_t* num_padded,
                                int64_t padded_len, uint16_t* x_sorted, void* stream) {
  return permute_impl(x, tokens, hidden, row_token, rows, sorted_rows, num_padded, padded_len, x_sorted,
                      (cudaStream_t)stream);
}

extern "C" int ssb_sorted_gate_up(const uint16_t* x_sorted, int32_t hidden, int32_t inter, const int32_t* row_token,
                                  int64_t rows, const int32_t* sorted_rows, const int32_t* block_expert,
                                  const int32_t* num_padded, int64_t padded_len, const int64_t* group_ptr,
                                  int32_t n_groups, int32_t shared_local, uint16_t* h_sorted, int32_t* err,
                                  void* stream) {
  return gate_up_impl(x_sorted, padded_len, hidden, inter, row_token, rows, sorted_rows, block_expert, num_padded,
                      padded_len, group_ptr, n_groups, shared_local, h_sorted, err, stream, true);
}

extern "C" int ssb_sorted_down(const uint16_t* h_sorted, int64_t rows, int32_t hidden, int32_t inter,
                               const float* row_weight, const int32_t* sorted_rows, const int32_t* block_expert,
                               const int32_t* num_padded, int64_t padded_len, const int64_t* group_ptr,
                               int32_t n_groups, int32_t shared_local, float* out_rows, int32_t* err, void* stream) {
  return down_impl(h_sorted, rows, hidden, inter, row_weight, sorted_rows, block_expert, num_padded, padded_len,
                   group_ptr, n_groups, shared_local, out_rows, err, stream, true);
}

extern "C" int ssb_prefill_experts(const uint16_t* x, int64_t tokens, int32_t hidden, int32_t inter,
                                   const int32_t* row_token, const float* row_weight, int64_t rows,
                                   const int32_t* sorted_rows, const int32_t* block_expert, const int32_t* num_padded,
                                   int64_t padded_len, const int64_t* group_ptr, int32_t n_groups,
                                   int32_t shared_local, uint16_t* x_sorted, uint16_t* h_sorted, float* out_rows,
                                   int32_t* err, void* stream) {
  SSB_CHECK_ARG(tokens >= 0);
  SSB_CHECK_ARG((int64_t)padded_len * inter * 2 >= rows * 4);
  // h_sorted is written by gate_up only after the permute: until then it holds the rows' sorted positions
  int rc = permute_by_row_impl(x, tokens, hidden, row_token, rows, sorted_rows, num_padded, padded_len, x_sorted,
                               reinterpret_cast<int32_t*>(h_sorted), (cudaStream_t)stream);
  if (rc) return rc;
  rc = ssb_sorted_gate_up(x_sorted, hidden, inter, row_token, rows, sorted_rows, block_expert, num_padded, padded_len,
                          group_ptr, n_groups, shared_local, h_sorted, err, stream);
  if (rc) return rc;
  return ssb_sorted_down(h_sorted, rows, hidden, inter, row_weight, sorted_rows, block_expert, num_padded, padded_len,
                         group_ptr, n_groups, shared_local, out_rows, err, stream);
}

extern "C" int ssb_gemm_affine4(const uint16_t* x, int64_t m, int32_t k, const int32_t* q, const uint16_t* s,
                                const uint16_t* b, int32_t n, int32_t gs, float* out, void* stream) {
  SSB_CHECK_ARG(m >= 0 && k >= 1 && n >= 1 && (gs == 32 || gs == 64));
  if (k % (2 * BK)) return SSB_EUNSUPPORTED;
  if (m == 0) return SSB_OK;
  SSB_CHECK_ARG(x && q && s && b && out);
  SSB_CHECK_ARG((((uintptr_t)q | (uintptr_t)s | (uintptr_t)b) & 3) == 0 && ((uintptr_t)q & 15) == 0);
  // one "expert" whose base is q; scale and bias are addressed relative to it
  GemmArgs g{};
  g.a = x;
  g.lda = k;
  g.a_rows = m;
  g.a_box_rows = TM;   // identity rows: one 2-D box per k-block (the tail past m reads zeros)
  g.R = m;
  g.base0 = (const uint8_t*)q;
  g.n_groups = 1;
  g.K = k;
  g.gs = gs;
  g.shared_local = -1;
  g.out = out;
  g.ldo = n;
  g.n_valid = n;
  g.out_vec = (n % 4 == 0) && ((uintptr_t)out & 15) == 0;
  g.off_w[0] = g.off_w[1] = 0;
  g.off_s[0] = g.off_s[1] = (int64_t)((const uint8_t*)s - (const uint8_t*)q);
  g.off_b[0] = g.off_b[1] = (int64_t)((const uint8_t*)b - (const uint8_t*)q);
  g.err = nullptr;
  return launch(EPI_PLAIN, g, (m + TM - 1) / TM, (n + BN - 1) / BN, (cudaStream_t)stream);
}

extern "C" int ssb_gemm_dense(const uint16_t* x, int64_t m, int32_t k, const uint16_t* w, int32_t n, float* out,
                              int64_t ldo, void* stream) {
  SSB_CHECK_ARG(m >= 0 && k >= 1 && n >= 1 && ldo >= n);
  if (k % BK) return SSB_EUNSUPPORTED;
  if (m == 0) return SSB_OK;
  SSB_CHECK_ARG(x && w && out && ((uintptr_t)w & 15) == 0 && ((uintptr_t)x & 15) == 0);
  GemmArgs g{};
  g.a = x;
  g.lda = k;
  g.a_rows = m;
  g.a_box_rows = TM;   // identity rows: one 2-D box per k-block (the tail past m reads zeros)
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
  g.n_valid = n;
  g.out_vec = (ldo % 4 == 0) && ((uintptr_t)out & 15) == 0;
  g.err = nullptr;
  return launch(EPI_PLAIN, g, (m + TM - 1) / TM, (n + BN - 1) / BN, (cudaStream_t)stream);
}

extern "C" int ssb_set_gate_up_tile(int32_t b_rows) {
  SSB_CHECK_ARG(b_rows == 128 || b_rows == 256);
  g_gate_up_tile = b_rows;
  return SSB_OK;
}

extern "C" int ssb_set_gemm_sm_reserve(int32_t sms) {
  SSB_CHECK_ARG(sms >= 0 && sms < 1024);
  g_sm_reserve = sms;
  return SSB_OK;
}
