// skv_kernels.cuh -- host-side launchers of the funnel kernels.
#pragma once
#include <cuda_runtime.h>

#include "skv_device.cuh"

namespace skv {

// Enqueue one decode step for every cell of `w` on `st`.
cudaError_t launch_funnel(const Work &w, cudaStream_t st, cudaEvent_t *ev = nullptr);
// Name of kernel i of one step (for per-kernel timing reports).
const char *funnel_kernel_name(int i);
// Number of kernels launch_funnel enqueues.
int funnel_kernel_count();
// One-time kernel attributes (dynamic shared memory opt-in).
cudaError_t prepare_funnel_attributes();
// Key code planes, per-dimension scales and FP8 [K|V] records of one slot
// from device BF16 K, V [4][T][256].
cudaError_t launch_key_codec(const uint16_t *k, const uint16_t *v, int T, uint32_t *smax,
                             float *const scale[G], uint8_t *const p2[G], uint8_t *const r2[G],
                             uint8_t *const r4[G], uint8_t *const kv8[G], cudaStream_t st);

}  // namespace skv
