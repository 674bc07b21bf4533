// skv_fused.cuh -- host-side launcher of the fused (one cluster per cell) funnel.
#pragma once
#include <cuda_runtime.h>

#include "skv_device.cuh"

namespace skv {

// Whether the fused kernel covers this workspace: nc <= 32768 centroids and
// a Stage-1.5 capacity <= 16384 (both multiples of 32).
bool fused_supported(const Work &w);
// One-time kernel attributes (dynamic shared memory, 16-CTA clusters).
cudaError_t prepare_fused_attributes();
// Enqueue one decode step for every cell of `w` on `st`: one kernel launch,
// carrying the L2 access-policy window `win` when it is not null.
cudaError_t launch_fused(const Work &w, cudaStream_t st, const cudaAccessPolicyWindow *win = nullptr);
// Name of a profiling mark tag written to Work::phase_ts.
const char *fused_mark_name(int tag);

}  // namespace skv
