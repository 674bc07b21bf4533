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

// ---- peer-memory exchange (one slot of 4 cells per shard)
constexpr int SHARD_MAX = 8;    // shards of a peer-memory group
constexpr int SHARD_CELLS = 4;  // one slot: 4 KV heads

// The exchange region every shard owns and every peer writes into.
struct ShardRegion {
  uint32_t keys[SHARD_MAX][SHARD_CELLS * G][TOPK];        // [source shard][cell*4+head][rank]
  int32_t ids[SHARD_MAX][SHARD_CELLS * G][TOPK];
  float part[SHARD_MAX][SHARD_CELLS][G][PART];            // [source shard][cell][head][m, l, 0, 0, o]
  uint32_t flag_lists[SHARD_MAX][SHARD_CELLS * G];        // epoch of each source's list
  uint32_t flag_parts[SHARD_MAX][SHARD_CELLS];            // epoch of each source's partials
};

// Kernel-side view of a connected group (passed by value).
struct ShardLinkDev {
  void *peer[SHARD_MAX];          // every shard's region as mapped here (own one included)
  int32_t begin[SHARD_MAX];       // first global token of each shard
  int32_t rank, n_shards, token_begin;
  uint32_t *epoch;                // steps completed (device counter)
};

size_t shard_region_bytes();
// Merge (after pushing this shard's lists), attention, combine (after pushing
// the partials) and the epoch bump, on `st`, for a connected group.
cudaError_t launch_shard_p2p_step(const Work &w, const ShardLinkDev &L, int32_t *gids, float *part,
                                  int32_t *status, cudaStream_t st);

}  // namespace skv
