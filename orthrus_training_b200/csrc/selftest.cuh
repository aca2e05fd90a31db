// Self-test of the bounded-wait protocol that every tcgen05 / TMA kernel of the library follows,
// run on the GPU without faulting it: a wait that nothing satisfies must run out after its limit,
// record ORTHRUS_ERR_TIMEOUT in the device error word, and the kernel must then drain the copy it
// issued (a bounded wait again), free its tensor memory and return, leaving the context usable.
#pragma once

#include "sm100.cuh"

namespace orthrus {

// One CTA of 64 threads. Thread 0 issues one TMA load of a 64 x 64 bf16 tile (8 KB) on the
// `loaded` barrier, then waits on `never`, which no thread or copy ever arrives on, for limit_ns;
// then drains `loaded`. Warp 1 holds 32 TMEM columns for the whole kernel and frees them at the
// end. status bits: 1 the never-satisfied wait timed out, 2 the issued copy was drained,
// 4 the TMEM columns were freed (the kernel reached its end).
__global__ void __launch_bounds__(64, 1)
    bounded_wait_selftest_kernel(const __grid_constant__ CUtensorMap tm, uint64_t limit_ns,
                                 unsigned int* __restrict__ status) {
  __shared__ __align__(1024) uint8_t tile[64 * 128];
  __shared__ __align__(8) uint64_t loaded, never;
  __shared__ uint32_t tmem_slot;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    mbar_init(&loaded, 1);
    mbar_init(&never, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&tmem_slot, 32);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  if (threadIdx.x == 0) {
    unsigned int st = 0;
    mbar_arrive_expect_tx(&loaded, sizeof(tile));
    tma_load_2d(tile, &tm, &loaded, 0, 0);
    if (!mbar_wait_limit(&never, 0, limit_ns)) st |= 1u;  // records ORTHRUS_ERR_TIMEOUT
    if (mbar_wait(&loaded, 0)) st |= 2u;                    // drain the copy in flight
    atomicOr(status, st);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_free(tmem, 32);
    if (threadIdx.x == 32) atomicOr(status, 4u);
  }
}

}  // namespace orthrus
