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

size_t shard_region_bytes();
// Merge (after pushing this shard's lists), attention, combine (after pushing
// the partials) and the epoch bump, on `st`, for a connected group.
// Bumps the group's step counter (after a step's exchanges).
cudaError_t launch_shard_epoch(const ShardLinkDev *dlink, cudaStream_t st);
cudaError_t launch_link_grow(ShardLinkDev *dlink, int m, int total_max, cudaStream_t st);
cudaError_t launch_shard_p2p_step(const Work &w, const ShardLinkDev &L, int32_t *gids, float *part,
                                  int32_t *status, cudaStream_t st);

}  // namespace skv
