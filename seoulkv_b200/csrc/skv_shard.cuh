// skv_shard.cuh -- host-side launchers of the sequence-sharded merge,
// partial attention and combine kernels.
#pragma once
#include <cuda_runtime.h>

#include "skv_device.cuh"

namespace skv {

// keys/ids [n_shards][n_cells][4][100], begin [n_shards] -> out [n_cells][4][100] global ids.
cudaError_t launch_shard_merge(const uint32_t *keys, const int32_t *ids, const int32_t *begin, int n_shards,
                               int n_cells, int32_t *out, cudaStream_t st);
// This shard's partials [n_cells][4][PART] over its dense zones and its winners in `gids`.
cudaError_t launch_shard_attention(const Work &w, const int32_t *gids, int token_begin, float *partials,
                                   cudaStream_t st);
// partials [n_shards][n_cells][4][PART] -> out [n_slots][16][256] BF16.
cudaError_t launch_shard_combine(const float *partials, int n_shards, int n_cells, uint16_t *out, cudaStream_t st);
// Largest n_shards the merge handles.
int shard_max_shards();

}  // namespace skv
