// Per-kernel shared-memory bookkeeping behind ssb_kernel_smem (the reference's SHARED_BYTES), and the process-wide
// bound of the cooperative kernels' grid-barrier waits (ssb_set_wait_limit_ns).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

void ssb_note_smem_bytes(const char* name, int bytes);
uint64_t ssb_barrier_wait_ns();

template <typename K>
static inline void ssb_note_smem(const char* name, K kern, size_t dyn) {
  cudaFuncAttributes a;
  if (cudaFuncGetAttributes(&a, (const void*)kern) == cudaSuccess)
    ssb_note_smem_bytes(name, (int)(a.sharedSizeBytes + dyn));
  else
    (void)cudaGetLastError();
}
