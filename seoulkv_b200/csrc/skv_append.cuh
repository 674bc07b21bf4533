// skv_append.cuh -- cache append: device state and launchers.
//
// The reference serves a static cache (its README lists appends as out of
// scope).  Here a cache may grow by whole tokens after the index is built:
// every new token gets its key planes and FP8 [K | V] record, and the two
// lists of its spill-2 posting (the two best stored centroids for its key);
// a token enters the inverted lists when it leaves the local window, which
// is when the reference's zones stop attending to it densely.  The centroids,
// the key-code scales and the zones' sizes stay those of the build.
#pragma once
#include <cuda_runtime.h>

#include "skv_device.cuh"

namespace skv {

constexpr int APPEND_MAX = 512;    // tokens per append launch sequence
constexpr int ASSIGN_SPLIT = 128;  // centroid partitions per cell in the assignment (at most)
constexpr int REBUILD_PER_THREAD = 4;  // CSR elements per thread of the rebuild
constexpr uint32_t APPEND_FULL = 1u;       // append status: a device-side append would have passed the capacity
constexpr uint32_t APPEND_NONFINITE = 2u;  // append status: an appended key had a non-finite element

// Append state of one cell (device memory).
struct AppendCellDev {
  int32_t *offsets[2], *values[2], *mates[2];  // two CSR buffer sets; set `cur` is live
  int32_t *labels;                             // [tmax][2] the two lists of tokens from the first local window on
  uint8_t *prefix2, *residual2, *residual4;    // [tmax][64], [tmax][64], [tmax][128]
  uint8_t *kv8;                                // [tmax][512]
  const float *key_scale;                      // [256] the build's per-dimension max |k|
  int32_t cur, n_postings;
};

// Spill-2 assignment of `m` key rows per cell (rows j of cell cell0 + y at
// k + y * k_cell_stride + j * 256); results go to labels[base + j] with base
// = (use_tlen ? *tlen : 0) + lab_base.  With guard > 0 nothing runs when
// *tlen + guard > tmax (an append that does not fit).  A non-finite key
// element counts as 0 (and raises APPEND_NONFINITE in *status, if given), so
// every token gets two valid lists.  `split` partitions of the centroids'
// 16-row tiles per cell (at most ASSIGN_SPLIT).
struct AssignArgs {
  const CellDev *cells;
  AppendCellDev *acells;
  const int32_t *tlen;
  const uint16_t *k;
  long long k_cell_stride;
  int cell0, n_cells, m, nc, split, lab_base, use_tlen, guard, tmax;
  uint32_t *status;  // append status word, or null
  double *part_s;   // [cell][APPEND_MAX][ASSIGN_SPLIT][2] partial top-2 scores
  int32_t *part_i;  // same layout, centroid ids
};

// One append of `m` tokens to every cell (rows [n_cells][m][256] of k and v).
struct AppendArgs {
  CellDev *cells;
  AppendCellDev *acells;
  int32_t *tlen;
  uint32_t *status;
  const uint16_t *k, *v;
  int n_cells, m, nc, local, tmax;
  int32_t *newlist, *newtok, *newmate;  // [cell][2 * APPEND_MAX] postings entering the lists, sorted
  int32_t *newins;                      // [cell][2 * APPEND_MAX] old CSR position each one is inserted at
  uint32_t *done;                       // rebuild CTAs finished (zero between appends)
  uint32_t *assign_done;                // [cell] assignment CTAs finished (zero between appends)
  int rebuild_ctas;                     // rebuild CTAs per cell
};

cudaError_t launch_assign(const AssignArgs &a, cudaStream_t st);
cudaError_t launch_append(const AppendArgs &a, const AssignArgs &assign, cudaStream_t st);

}  // namespace skv
