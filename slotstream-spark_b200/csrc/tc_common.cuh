// tcgen05 / TMEM / UMMA-descriptor helpers for the sm_100a tensor-core kernels.
//
// Shared-memory operand tiles are K-major with the 128-byte swizzle: a tile row holds 64 bf16 (128 B) of
// one M (or N) index, rows are packed at 128 B, 8-row groups at 1024 B, and 16-byte chunk c of row r sits
// at chunk position c ^ (r % 8). Tile bases are 1024-byte aligned. The UMMA shared-memory descriptor of such
// a tile has start address >> 4, LBO 1 (unused for swizzled K-major), SBO 1024 >> 4, version 1, layout
// SWIZZLE_128B (2); the K step of 16 elements inside the 64-element row advances the start address by 32 B.
#pragma once
#include <cuda.h>

#include "affine.cuh"

SSB_DEV uint32_t swz128(uint32_t row, uint32_t chunk) { return row * 128u + (((chunk ^ (row & 7u)) & 7u) << 4); }

SSB_DEV uint64_t umma_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;                 // leading byte offset (16 B)
  d |= (uint64_t)(1024u >> 4) << 32;       // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1u << 46;                 // descriptor version (sm_100)
  d |= (uint64_t)2u << 61;                 // SWIZZLE_128B
  return d;
}

// Instruction descriptor of tcgen05.mma kind::f16: bf16 A and B (both K-major), fp32 accumulator, M x N.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int m, int n) {
  return (1u << 4)                         // D format: f32
         | (1u << 7)                       // A format: bf16
         | (1u << 10)                      // B format: bf16
         | ((uint32_t)(n >> 3) << 17)      // N >> 3
         | ((uint32_t)(m >> 4) << 24);     // M >> 4
}

SSB_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
SSB_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Warp-collective TMEM allocation: writes the base address to *dst_smem.
SSB_DEV void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
SSB_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
SSB_DEV void umma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive (once) on `bar` when every tcgen05 operation this thread issued so far has completed.
SSB_DEV void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 consecutive fp32 columns of this warp's 32 TMEM lanes (thread t gets lane base + t).
SSB_DEV void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// ---------------------------------------------------------------- cp.async (16-byte, zero-fill when src_bytes = 0)
SSB_DEV void cp_async16(uint32_t dst_smem, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst_smem), "l"(src), "r"(src_bytes) : "memory");
}
// Arrive on `bar` (without changing its expected count) once this thread's earlier cp.async copies landed.
SSB_DEV void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
SSB_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// ---------------------------------------------------------------- TMA row gather
// Four rows (r0..r3) of a 2-D bf16 tensor map whose box is 64 elements x 1 row, starting at element column
// `col` (a multiple of 64, so the 16-byte rule on the inner coordinate holds), land as four consecutive
// 128-byte rows at dst with the map's 128-byte swizzle; completion is counted in bytes on `bar`.
SSB_DEV void tma_gather4(uint32_t dst, const CUtensorMap* map, int32_t col, int32_t r0, int32_t r1, int32_t r2,
                         int32_t r3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(dst),
      "l"((uint64_t)map), "r"(col), "r"(r0), "r"(r1), "r"(r2), "r"(r3), "r"(smem_u32(bar))
      : "memory");
}
// One cache line into L2 through the load/store path (no register result, nothing to wait for).
SSB_DEV void prefetch_line_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }
// One 2-D box of the tensor map at (col, row) into dst (the map's box size and swizzle), bytes counted on `bar`.
SSB_DEV void tma_load_2d(uint32_t dst, const CUtensorMap* map, int32_t col, int32_t row, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"((uint64_t)map), "r"(col), "r"(row), "r"(smem_u32(bar))
      : "memory");
}
SSB_DEV void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)map) : "memory");
}

// ---------------------------------------------------------------- bounded waits on the global timer
SSB_DEV uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Wait for phase `parity` of `bar`; false after `ns` nanoseconds without completion. Each try_wait carries a
// suspend-time hint, so a waiting warp sleeps until the phase completes (or the hint expires) instead of
// spinning and taking issue slots from the warps that do the work.
SSB_DEV bool mbar_wait_ns(uint64_t* bar, uint32_t parity, uint64_t ns) {
  const uint32_t a = smem_u32(bar);
  uint64_t t0 = 0;
  for (uint32_t i = 0;; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(parity), "r"(1000000u)
        : "memory");
    if (done) return true;
    if ((i & 7u) == 0u) {
      uint64_t t = globaltimer_ns();
      if (t0 == 0) t0 = t;
      else if (t - t0 > ns) return false;
    }
  }
}
constexpr uint64_t SSB_WAIT_NS = 250ull * 1000 * 1000;   // 250 ms: far above any stage time

// As mbar_wait_ns, polling with test_wait (no suspension): for one-shot waits on a latency-critical path, where
// a suspended thread's wake-up would add to the critical path.
SSB_DEV bool mbar_wait_spin(uint64_t* bar, uint32_t parity, uint64_t ns) {
  const uint32_t a = smem_u32(bar);
  uint64_t t0 = 0;
  for (uint32_t i = 0;; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 1023u) == 0u) {
      uint64_t t = globaltimer_ns();
      if (t0 == 0) t0 = t;
      else if (t - t0 > ns) return false;
    }
  }
}
