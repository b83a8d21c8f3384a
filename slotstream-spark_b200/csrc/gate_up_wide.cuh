// Wide-tile gate_up GEMM of the sorted prefill path (included by grouped_gemm.cu inside its namespace; uses its
// dequant8_perm / cvt_bf16x2 / silu_fast helpers and GemmArgs).
//
// The 256 x 128 tile of k_moe_gemm issues M128 x N128 MMAs, and an N128 tcgen05.mma occupies the tensor pipe as
// long as an N256 one, so that kernel cannot pass half of the tensor peak. This kernel's tile is 256 activation
// rows x 256 B-rows -- the gate rows and the up rows of the same 128 intermediate columns -- and every k-block
// issues M128 x N256 x K16 MMAs for each 128-row half, so the dequantised B tile still feeds both halves and
// the tensor pipe runs at its full per-instruction width.
//
// The two halves' accumulators (2 x 256 fp32 columns) fill the 512 TMEM columns, so there is one accumulator
// set: the epilogue drains half 0, hands it back (tmem_empty[0]), then drains half 1 (tmem_empty[1]); the next
// tile's first MMAs into half 0 wait only for the first hand-back, so they overlap the drain of half 1.
//
// Warp roles (16 warps):
//  * warp 0      activation rows: one 2-D TMA box of 256 rows from the permuted rows (x_sorted), or of the
//                first 128 when the second half holds only padding rows (then neither loaded, multiplied nor stored);
//  * warp 1      owns TMEM (512 columns) and issues tcgen05.mma from one thread;
//  * warps 4..7  epilogue: TMEM -> registers, h = silu(g) * u -> bf16 rows of h_sorted (one row per thread);
//  * warps 8..15 weight producers, one thread per B-row: the row's codes, scales and biases of four k-blocks
//                are loaded into registers one super-step ahead (and the super-step after that is prefetched
//                into L2), then dequantised q*s + b -> bf16 in the K order (0,4,1,5,2,6,3,7) into the 128-byte
//                swizzled B tile.
// Every wait is bounded and ends with SSB_ERR_TIMEOUT; a row's result depends only on the row and its
// expert's bytes (fixed k order), as in k_moe_gemm.

constexpr int WG_BN = 256;                            // B-rows per tile: 128 gate + 128 up
constexpr int WG_A_STAGES = 3;                        // activation stages
constexpr int WG_B_STAGES = 4;                        // dequantised weight stages (3: 2% slower, fewer: slower still)
constexpr int WG_SS = 4;                              // k-blocks per producer super-step
constexpr uint32_t WG_A_STAGE = TM * 128;             // 32 KB: two 128-row halves
constexpr uint32_t WG_B_STAGE = WG_BN * 128;          // 32 KB
constexpr uint32_t WG_TMEM_COLS = 512;                // half h's accumulator at column 256 h
constexpr size_t WG_SMEM_BYTES =
    1024 + WG_A_STAGES * WG_A_STAGE + WG_B_STAGES * WG_B_STAGE + 8 * (2 * WG_A_STAGES + 2 * WG_B_STAGES + 3) + 16;

__global__ void __launch_bounds__(THREADS, 1) k_gate_up_wide(const __grid_constant__ CUtensorMap tm_a,
                                                              const __grid_constant__ CUtensorMap tm_h, GemmArgs a) {
  extern __shared__ uint8_t smraw[];
  __shared__ int s_fail;
  uint8_t* base = (uint8_t*)(((uintptr_t)smraw + 1023) & ~(uintptr_t)1023);
  uint8_t* sa = base;
  uint8_t* sb = sa + WG_A_STAGES * WG_A_STAGE;
  uint64_t* full_a = (uint64_t*)(sb + WG_B_STAGES * WG_B_STAGE);
  uint64_t* empty_a = full_a + WG_A_STAGES;
  uint64_t* full_b = empty_a + WG_A_STAGES;
  uint64_t* empty_b = full_b + WG_B_STAGES;
  uint64_t* tmem_full = empty_b + WG_B_STAGES;   // [1]
  uint64_t* tmem_empty = tmem_full + 1;      // [2]: one per half
  uint32_t* tmem_slot = (uint32_t*)(tmem_empty + 2);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_wait();
  pdl_trigger();
  const int NB = a.n_nblocks;   // inter / 128
  const int64_t n_mb = (int64_t)__ldcg(a.num_padded) / TM;
  const int64_t n_tiles = n_mb * NB;
  if ((int64_t)blockIdx.x >= n_tiles) return;
  const int my_tiles = (int)((n_tiles - blockIdx.x + gridDim.x - 1) / gridDim.x);
  const int KB = a.K / BK;
  const int64_t steps = (int64_t)my_tiles * KB;
  auto tile_of = [&](int i) -> int64_t { return (int64_t)blockIdx.x + (int64_t)i * gridDim.x; };
  // the A and MMA threads fetch the next tile's answer a tile ahead as a raw row id and test it when that tile
  // starts, so the load's latency never stalls them
  auto half1_row = [&](int64_t mb) -> int32_t { return __ldcg(a.sorted_rows + mb * TM + BM); };
  auto half1_ok = [&](int32_t r) -> bool { return r >= 0 && r < a.R; };
  auto half1_of = [&](int64_t mb) -> bool { return half1_ok(half1_row(mb)); };

  if (tid == 0) {
    s_fail = 0;
    for (int s = 0; s < WG_A_STAGES; ++s) {
      mbar_init(&full_a[s], 1);
      mbar_init(&empty_a[s], 1);
    }
    for (int s = 0; s < WG_B_STAGES; ++s) {
      mbar_init(&full_b[s], N_PROD);
      mbar_init(&empty_b[s], 1);
    }
    mbar_init(tmem_full, 1);
    mbar_init(&tmem_empty[0], 4);
    mbar_init(&tmem_empty[1], 4);
    fence_mbar_init();
  }
  if (warp == MMA_WARP) tmem_alloc(tmem_slot, WG_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  int commits = 0;   // MMA thread: tmem_full commits issued

  if (warp == A_WARP) {
    if (lane == 0) {
      prefetch_tensormap(&tm_a);
      prefetch_tensormap(&tm_h);
      // step counters kept incrementally (no 64-bit division on the issue path)
      int64_t issued = 0;
      bool two = half1_of(tile_of(0) / NB);
      int32_t r_next = 0;
      int kb = 0, i = 0, s = 0;
      uint32_t ph = 0;
      int32_t r0 = (int32_t)((tile_of(0) / NB) * TM);
      for (int64_t j = 0; j < steps; ++j) {
        if (kb == 0) {
          if (i > 0) {
            two = half1_ok(r_next);
            r0 = (int32_t)((tile_of(i) / NB) * TM);
          }
          if (i + 1 < my_tiles) r_next = half1_row(tile_of(i + 1) / NB);
        }
        if (!mbar_wait_ns(&empty_a[s], ph ^ 1, SSB_WAIT_NS)) {
          s_fail = 1;
          break;
        }
        mbar_expect_tx(&full_a[s], two ? WG_A_STAGE : A_HALF);
        tma_load_2d(smem_u32(sa + s * WG_A_STAGE), two ? &tm_a : &tm_h, kb * BK, r0, &full_a[s]);   // 256 or 128 rows
        ++issued;
        if (++s == WG_A_STAGES) {
          s = 0;
          ph ^= 1;
        }
        if (++kb == KB) {
          kb = 0;
          ++i;
        }
      }
      // no copy may still be writing shared memory when the CTA exits
      for (int64_t j = issued > WG_A_STAGES ? issued - WG_A_STAGES : 0; j < issued; ++j)
        mbar_wait_ns(&full_a[j % WG_A_STAGES], (uint32_t)((j / WG_A_STAGES) & 1), SSB_WAIT_NS);
    }
    __syncwarp();
  } else if (warp == MMA_WARP) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(BM, WG_BN);
      int64_t j = 0;
      int32_t r_next = half1_row(tile_of(0) / NB);
      for (int i = 0; i < my_tiles && !s_fail; ++i) {
        const int nh = half1_ok(r_next) ? MT : 1;
        if (i + 1 < my_tiles) r_next = half1_row(tile_of(i + 1) / NB);
        bool ok = true;
        for (int kb = 0; kb < KB; ++kb, ++j) {
          const int s = (int)(j % WG_A_STAGES), t = (int)(j % WG_B_STAGES);
          if (!mbar_wait_ns(&full_a[s], (uint32_t)((j / WG_A_STAGES) & 1), SSB_WAIT_NS) ||
              !mbar_wait_ns(&full_b[t], (uint32_t)((j / WG_B_STAGES) & 1), SSB_WAIT_NS)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t db = umma_desc_sw128(smem_u32(sb + t * WG_B_STAGE));
#pragma unroll
          for (int h = 0; h < MT; ++h) {
            if (h >= nh) break;
            if (kb == 0) {   // the epilogue has drained this half of the previous tile
              if (!mbar_wait_ns(&tmem_empty[h], (uint32_t)(i & 1) ^ 1, SSB_WAIT_NS)) {
                ok = false;
                break;
              }
              tc_fence_after();
            }
            const uint64_t da = umma_desc_sw128(smem_u32(sa + s * WG_A_STAGE + h * A_HALF));
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              umma_bf16(tmem + (uint32_t)(h * WG_BN), da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc,
                        (kb | k) != 0);
          }
          umma_commit(&empty_a[s]);
          umma_commit(&empty_b[t]);
          if (!ok) break;
        }
        umma_commit(tmem_full);
        ++commits;
        if (!ok) {
          s_fail = 1;
          break;
        }
      }
    }
    __syncwarp();
  } else if (warp >= EPI_WARP0 && warp < EPI_WARP0 + 4) {
    const int q = warp & 3;
    uint16_t* out = (uint16_t*)a.out;
    for (int i = 0; i < my_tiles; ++i) {
      const int64_t t = tile_of(i), mb = t / NB;
      const int nb = (int)(t % NB);
      const bool shared_e = a.shared_local >= 0 && __ldcg(a.block_expert + mb) == a.shared_local;
      const int nh = half1_of(mb) ? MT : 1;
      bool valid[MT];
#pragma unroll
      for (int h = 0; h < MT; ++h) {
        const int32_t r = __ldcg(a.sorted_rows + mb * TM + h * BM + 32 * q + lane);
        valid[h] = r >= 0 && r < a.R;
      }
      const bool ok = mbar_wait_ns(tmem_full, (uint32_t)(i & 1), SSB_WAIT_NS);
      tc_fence_after();
      if (!ok) {
        s_fail = 1;
        break;
      }
#pragma unroll 1
      for (int h = 0; h < MT; ++h) {
        if (h < nh) {
          const int64_t m = mb * TM + h * BM + 32 * q + lane;
          const uint32_t taddr = tmem + (uint32_t)(h * WG_BN) + ((uint32_t)(32 * q) << 16);
#pragma unroll 1
          for (int cc = 0; cc < 4; ++cc) {
            float g[32], u[32];
            tmem_ld32(taddr + 32 * cc, g);
            tmem_ld32(taddr + 128 + 32 * cc, u);
            if (valid[h]) {
              uint4* dst = reinterpret_cast<uint4*>(out + m * a.ldo + (int64_t)nb * 128 + 32 * cc);
              uint4 pk[4];
              if (shared_e) swiglu32<true>(g, u, true, pk);
              else swiglu32<false>(g, u, true, pk);
#pragma unroll
              for (int jj = 0; jj < 4; ++jj) dst[jj] = pk[jj];
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tmem_empty[h]);   // this half may be overwritten by the next tile now
      }
    }
  } else if (warp >= PROD_WARP0) {
    // ---------------- weight producers: thread p owns B-row p (p < 128: gate row, else up row of column p % 128)
    const int p = tid - PROD_WARP0 * 32;
    const int piece = p >> 7;
    const int ng = a.K / a.gs;
    const int n_ss = (int)(steps / WG_SS);
    int my_fail = 0;
    // the row's codes (4 k-blocks x 32 B), scales and biases (4 bf16 each) of super-step n; zeros for an unusable
    // record (its error bit is set once per tile)
    struct Rows {
      uint4 w[WG_SS][2];
      uint2 s, b;
    };
    // Record base per tile, fetched ahead so that no load of a super-step waits on a dependent chain: the expert
    // of tile T+1 is read when tile T's loads start, its base in the middle of tile T, and it is checked when
    // tile T+1 starts. The loader walks super-steps in order with 32-bit counters (a tile is SPT consecutive
    // super-steps; KB is a multiple of WG_SS), so no division runs per super-step.
    const int SPT = KB / WG_SS, MID = SPT / 2;
    auto expert_at = [&](int i) -> int32_t { return __ldcg(a.block_expert + tile_of(i) / NB); };
    auto base_raw = [&](int32_t e) -> const uint8_t* {
      return (e >= 0 && e < a.n_groups) ? (const uint8_t*)__ldg(a.group_base + e) : nullptr;
    };
    auto usable = [](const uint8_t* rb) -> const uint8_t* { return ((uintptr_t)rb & 15) ? nullptr : rb; };
    auto nb_at = [&](int i) -> int { return (int)(((uint32_t)blockIdx.x + (uint32_t)i * gridDim.x) % (uint32_t)NB); };
    const uint8_t* base_cur = nullptr;   // checked base of the tile being loaded
    const uint8_t* base_nxt = nullptr;   // raw base of the next tile (from the middle of the current one)
    int32_t e_nxt = -1;
    int ld_T = 0, ld_sub = -1, nb_cur = 0, nb_nxt = 0;
    const int64_t piece_w = a.off_w[piece], piece_s = a.off_s[piece], piece_b = a.off_b[piece];
    auto row_src = [&](const uint8_t* rb, int nb, int sub, const uint8_t*& codes, const uint16_t*& sc,
                       const uint16_t*& bi) {
      const int nrow = nb * 128 + (p & 127);
      const int kb0 = sub * WG_SS;
      codes = rb + piece_w + (int64_t)nrow * (a.K / 2) + kb0 * 32;
      sc = (const uint16_t*)(rb + piece_s) + (int64_t)nrow * ng + kb0;
      bi = (const uint16_t*)(rb + piece_b) + (int64_t)nrow * ng + kb0;
    };
    auto load = [&](Rows& r) -> bool {   // the next super-step in order
      if (++ld_sub == SPT || ld_sub == 0) {
        if (ld_sub == SPT) ++ld_T;
        ld_sub = 0;
        base_cur = ld_T == 0 ? usable(base_raw(expert_at(0))) : usable(base_nxt);
        nb_cur = ld_T == 0 ? nb_at(0) : nb_nxt;
        if (ld_T + 1 < my_tiles) {
          e_nxt = expert_at(ld_T + 1);
          nb_nxt = nb_at(ld_T + 1);
        }
      }
      if (ld_sub == MID && ld_T + 1 < my_tiles) base_nxt = base_raw(e_nxt);
      if (!base_cur) {
#pragma unroll
        for (int u = 0; u < WG_SS; ++u) r.w[u][0] = r.w[u][1] = make_uint4(0, 0, 0, 0);
        r.s = r.b = make_uint2(0, 0);
        return false;
      }
      const uint8_t* c;
      const uint16_t *sc, *bi;
      row_src(base_cur, nb_cur, ld_sub, c, sc, bi);
#pragma unroll
      for (int u = 0; u < WG_SS; ++u) {
        r.w[u][0] = __ldg(reinterpret_cast<const uint4*>(c + 32 * u));
        r.w[u][1] = __ldg(reinterpret_cast<const uint4*>(c + 32 * u + 16));
      }
      r.s = __ldg(reinterpret_cast<const uint2*>(sc));
      r.b = __ldg(reinterpret_cast<const uint2*>(bi));
      return true;
    };
    // L2 prefetch of the super-step after the one just loaded: in the same tile with that tile's base, in the
    // next tile with the next base once it has had a super-step to arrive
    auto prefetch = [&]() {
      const uint8_t* rb;
      int nb, sub;
      if (ld_sub + 1 < SPT) {
        rb = base_cur, nb = nb_cur, sub = ld_sub + 1;
      } else {
        if (ld_T + 1 >= my_tiles || ld_sub <= MID) return;
        rb = usable(base_nxt), nb = nb_nxt, sub = 0;
      }
      if (!rb) return;
      const uint8_t* c;
      const uint16_t *sc, *bi;
      row_src(rb, nb, sub, c, sc, bi);
      prefetch_line_l2(c);
    };
    Rows cur, nxt;
    bool cur_ok = n_ss > 0 ? load(cur) : true;
    if (n_ss > 1) prefetch();
    int bs = 0;            // B stage of the next k-block, and its phase
    uint32_t bph = 0;
    for (int n = 0; n < n_ss; ++n) {
      bool nxt_ok = true;
      if (n + 1 < n_ss) {
        nxt_ok = load(nxt);
        if (n + 2 < n_ss) prefetch();
      }
      if (!cur_ok && p == 0 && n % SPT == 0) set_err(a.err, SSB_ERR_MISALIGNED);
#pragma unroll
      for (int u = 0; u < WG_SS; ++u) {
        const int s = bs;
        const uint32_t cur_ph = bph;
        if (++bs == WG_B_STAGES) {
          bs = 0;
          bph ^= 1;
        }
        if (my_fail || !mbar_wait_ns(&empty_b[s], cur_ph ^ 1, SSB_WAIT_NS)) {
          my_fail = 1;
          s_fail = 1;
          continue;
        }
        const uint32_t sw = (u >> 1) ? cur.s.y : cur.s.x, bw = (u >> 1) ? cur.b.y : cur.b.x;
        const uint32_t s2 = __byte_perm(sw, 0, (u & 1) ? 0x3232 : 0x1010);
        const uint32_t b2 = __byte_perm(bw, 0, (u & 1) ? 0x3232 : 0x1010);
        uint8_t* bt = sb + s * WG_B_STAGE;
        const uint32_t ws[8] = {cur.w[u][0].x, cur.w[u][0].y, cur.w[u][0].z, cur.w[u][0].w,
                                cur.w[u][1].x, cur.w[u][1].y, cur.w[u][1].z, cur.w[u][1].w};
#pragma unroll
        for (int c = 0; c < 8; ++c)   // 16-byte chunk c = elements 8c .. 8c+7 of the k-block = code word c
          *reinterpret_cast<uint4*>(bt + swz128(p, c)) = dequant8_perm(ws[c], s2, b2);
        fence_proxy_async_smem();
        mbar_arrive(&full_b[s]);
      }
      if (my_fail) break;
      cur = nxt;
      cur_ok = nxt_ok;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    if (s_fail) {   // every committed MMA group finishes before TMEM is released (the last commit's phase)
      if (lane == 0 && commits > 0) mbar_wait_ns(tmem_full, (uint32_t)((commits - 1) & 1), SSB_WAIT_NS);
      __syncwarp();
    }
    tc_fence_after();
    tmem_dealloc(tmem, WG_TMEM_COLS);
  }
  if (tid == 0 && s_fail) set_err(a.err, SSB_ERR_TIMEOUT);
}
