// skv_shard.cu -- sequence-sharded decode: exact global top-100 merge, the
// per-shard partial attention over the winners it owns, and the
// log-sum-exp combine of the shards' partials.
//
// A long context is split into contiguous token ranges, one per GPU; every
// GPU runs the funnel on its own range (its own index, key planes and FP8
// records) and keeps, per query head, its local top-100 with the Stage-II
// keys [ordered BF16 score | 0xffff - union position].  After the host
// gathers every shard's lists (an all-gather), every GPU merges them into
// the same global top-100 per head:
//   ordered score descending, then local rank ascending, then global token
//   id ascending (a total order, so every GPU gets the same list);
// attends over the winners inside its own range plus its dense zones (the
// sink lives on the first shard, the local window on the last); and after a
// second all-gather of the (m, l, o) partials every GPU combines them into
// the same BF16 output.
#include <cuda_fp8.h>

#include "skv_device.cuh"
#include "skv_shard.cuh"

namespace skv {
namespace {

constexpr int MERGE_THREADS = 1024;  // candidates per head: shards * 100

// One CTA per (cell, query head).  keys/ids: [n_shards][n_cells][4][100]
// (ids local to the shard), begin: [n_shards] first token of each shard;
// out: [n_cells][4][100] global token ids in rank order, -1 past the end.
__global__ void __launch_bounds__(MERGE_THREADS) k_shard_merge(const uint32_t *keys, const int32_t *ids,
                                                               const int32_t *begin, int n_shards, int n_cells,
                                                               int32_t *out) {
  const int ch = blockIdx.x, tid = threadIdx.x, n = n_shards * TOPK;
  __shared__ unsigned long long sk[MERGE_THREADS];
  unsigned long long kv = 0ull;
  int gid = -1;
  if (tid < n) {
    const int s = tid / TOPK, r = tid - s * TOPK;
    const size_t at = ((size_t)s * n_cells * G + ch) * TOPK + r;
    const uint32_t key = keys[at];
    if (key) {
      gid = begin[s] + ids[at];
      kv = ((unsigned long long)(key >> 16) << 48) | ((unsigned long long)(0xffffu - (uint32_t)r) << 32) |
           (unsigned long long)(0xffffffffu - (uint32_t)gid);
    }
  }
  sk[tid] = kv;
  const int valid = __syncthreads_count(kv != 0ull);
  int32_t *dst = out + (size_t)ch * TOPK;
  if (kv) {
    int rank = 0;
    for (int j = 0; j < n; ++j) rank += sk[j] > kv;
    if (rank < TOPK) dst[rank] = gid;
  }
  if (tid < TOPK && tid >= valid) dst[tid] = -1;
}

__device__ __forceinline__ void fp8x8(uint2 v, float *o) {
  const uint32_t ws[2] = {v.x, v.y};
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const __half2_raw a = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(ws[k] & 0xffffu), __NV_E4M3);
    const __half2_raw b = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(ws[k] >> 16), __NV_E4M3);
    const float2 fa = __half22float2(*reinterpret_cast<const __half2 *>(&a));
    const float2 fb = __half22float2(*reinterpret_cast<const __half2 *>(&b));
    o[4 * k + 0] = fa.x; o[4 * k + 1] = fa.y; o[4 * k + 2] = fb.x; o[4 * k + 3] = fb.y;
  }
}

// Partition `split` of one cell: items are this shard's dense keys (one FP8
// record scored for all four heads) then, per head, the global winners
// inside [token_begin, token_begin + T).  Writes per-split partials to the
// workspace; the last partition of the cell merges them into the cell's
// un-normalised partial (m, l, 0, 0, o[256]) per head (log2 domain).
__global__ void __launch_bounds__(256) k_shard_attn(Work w, const int32_t *gids, int token_begin, float *partials) {
  const int split = blockIdx.x, cell = blockIdx.y, slot = cell >> 2, g = cell & 3;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const CellDev &c = w.cells[cell];
  const int sink = w.sink, local = w.local, T = context_of(w), dense = sink + local;
  const int nitems = dense + G * TOPK;
  const float qscale = 0.0625f * 1.4426950408889634f;  // 1/sqrt(256), log2(e)
  __shared__ float s_m[G][8], s_l[G][8];
  __shared__ float s_o[8][D];
  __shared__ int s_last;
  float qv[G][8];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    const uint4 raw = *reinterpret_cast<const uint4 *>(w.q + ((size_t)slot * 16 + g * 4 + h) * D + 8 * lane);
    const uint32_t rw[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      qv[h][2 * j] = bf16f(rw[j] & 0xffffu) * qscale;
      qv[h][2 * j + 1] = bf16f(rw[j] >> 16) * qscale;
    }
  }
  float m[G], l[G], o[G][8];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; ++e) o[h][e] = 0.0f;
  }
  for (int it = split * 8 + warp; it < nitems; it += ATTN_SPLIT * 8) {
    int tok, head = -1;
    if (it < sink) {
      tok = it;
    } else if (it < dense) {
      tok = T - local + (it - sink);
    } else {
      const int r = it - dense;
      head = r / TOPK;
      const int gid = gids[((size_t)cell * G + head) * TOPK + r % TOPK];
      tok = gid - token_begin;
      if (gid < 0 || tok < 0 || tok >= T) continue;  // not this shard's (warp-uniform)
    }
    const uint8_t *rec = c.kv8 + (size_t)tok * REC;
    float kf[8], vf[8];
    fp8x8(*reinterpret_cast<const uint2 *>(rec + 8 * lane), kf);
    fp8x8(*reinterpret_cast<const uint2 *>(rec + 256 + 8 * lane), vf);
    float dot[G];
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float a = 0.0f;
#pragma unroll
      for (int e = 0; e < 8; ++e) a = fmaf(qv[h][e], kf[e], a);
      dot[h] = a;
    }
#pragma unroll
    for (int o2 = 16; o2 > 0; o2 >>= 1)
#pragma unroll
      for (int h = 0; h < G; ++h) dot[h] += __shfl_xor_sync(0xffffffffu, dot[h], o2);
#pragma unroll
    for (int h = 0; h < G; ++h) {
      if (head >= 0 && head != h) continue;
      const float mn = fmaxf(m[h], dot[h]);
      const float scale = exp2f(m[h] - mn);
      const float p = exp2f(dot[h] - mn);
      l[h] = l[h] * scale + p;
#pragma unroll
      for (int e = 0; e < 8; ++e) o[h][e] = fmaf(o[h][e], scale, p * vf[e]);
      m[h] = mn;
    }
  }
  float *part = w.attn_part + (size_t)cell * G * ATTN_SPLIT * PART;
  for (int h = 0; h < G; ++h) {
    if (lane == 0) { s_m[h][warp] = m[h]; s_l[h][warp] = l[h]; }
#pragma unroll
    for (int e = 0; e < 8; ++e) s_o[warp][8 * lane + e] = o[h][e];
    __syncthreads();
    float M = -INFINITY;
#pragma unroll
    for (int k = 0; k < 8; ++k) M = fmaxf(M, s_m[h][k]);
    float L = 0.0f, O = 0.0f;
    if (M != -INFINITY) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (s_m[h][k] == -INFINITY) continue;
        const float e = exp2f(s_m[h][k] - M);
        L += s_l[h][k] * e;
        O += s_o[k][tid] * e;
      }
    }
    float *dst = part + ((size_t)h * ATTN_SPLIT + split) * PART;
    if (tid == 0) { dst[0] = M; dst[1] = L; }
    dst[4 + tid] = O;
    __syncthreads();
  }
  // the last partition of this cell merges them (no waiting: whoever arrives last)
  __threadfence();
  if (tid == 0) s_last = atomicAdd(&w.arrive[cell], 1u) == ATTN_SPLIT - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  {
    const int h = tid >> 6, q4 = tid & 63;
    const float *ph = part + (size_t)h * ATTN_SPLIT * PART;
    float M = -INFINITY;
    for (int sp = 0; sp < ATTN_SPLIT; ++sp) M = fmaxf(M, __ldcg(ph + sp * PART));
    float L = 0.0f;
    float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
    if (M != -INFINITY)
      for (int sp = 0; sp < ATTN_SPLIT; ++sp) {
        const float ms = __ldcg(ph + sp * PART);
        if (ms == -INFINITY) continue;
        const float e = exp2f(ms - M);
        L += __ldcg(ph + sp * PART + 1) * e;
        const float4 os = __ldcg(reinterpret_cast<const float4 *>(ph + sp * PART + 4) + q4);
        O.x += os.x * e; O.y += os.y * e; O.z += os.z * e; O.w += os.w * e;
      }
    float *dst = partials + ((size_t)cell * G + h) * PART;
    if (q4 == 0) { dst[0] = M; dst[1] = L; dst[2] = 0.0f; dst[3] = 0.0f; }
    reinterpret_cast<float4 *>(dst + 4)[q4] = O;
  }
  if (tid == 0) w.arrive[cell] = 0;
}

// One CTA per cell: out = sum_s o_s 2^(m_s - M) / sum_s l_s 2^(m_s - M).
__global__ void __launch_bounds__(256) k_shard_combine(const float *partials, int n_shards, int n_cells,
                                                       uint16_t *out) {
  const int cell = blockIdx.x, slot = cell >> 2, g = cell & 3, d = threadIdx.x;
  for (int h = 0; h < G; ++h) {
    float M = -INFINITY;
    for (int s = 0; s < n_shards; ++s) M = fmaxf(M, partials[(((size_t)s * n_cells + cell) * G + h) * PART]);
    float L = 0.0f, O = 0.0f;
    for (int s = 0; s < n_shards; ++s) {
      const float *p = partials + (((size_t)s * n_cells + cell) * G + h) * PART;
      if (p[0] == -INFINITY) continue;
      const float e = exp2f(p[0] - M);
      L += p[1] * e;
      O += p[4 + d] * e;
    }
    out[((size_t)slot * 16 + g * 4 + h) * D + d] = bf16_rne(O / L);
  }
}

// ------------------------------------------------ peer-memory exchange
//
// Without a collective library: every shard owns an exchange region in its
// own memory that the other shards write into over NVLink (CUDA IPC
// mappings), and per-step epoch flags say when a peer's part has landed.
// Each (cell, head) CTA pushes its own list to every peer and then waits for
// every peer's list of the same (cell, head); each cell CTA does the same
// with the attention partials.  No CTA waits for another CTA of its own GPU.
// Waits are bounded: after SHARD_WAIT_POLLS polls the step's status word gets
// ST_TIMEOUT and the kernel carries on with whatever arrived.

// One CTA per (cell, head): push this shard's list to every peer's slot
// `rank`, signal, wait for every shard's list of this (cell, head), merge.
__global__ void __launch_bounds__(MERGE_THREADS) k_shard_merge_p2p(ShardLinkDev L, const uint32_t *keys,
                                                                   const int32_t *ids, int32_t *out,
                                                                   int32_t *status) {
  const int ch = blockIdx.x, tid = threadIdx.x, n = L.n_shards;
  const uint32_t epoch = *L.epoch + 1;
  __shared__ unsigned long long sk[MERGE_THREADS];
  __shared__ int s_ok;
  if (tid < TOPK) {
    const uint32_t kv = keys[(size_t)ch * TOPK + tid];
    const int32_t iv = ids[(size_t)ch * TOPK + tid];
    for (int p = 0; p < n; ++p) {
      ShardRegion *R = reinterpret_cast<ShardRegion *>(L.peer[p]);
      R->keys[L.rank][ch][tid] = kv;
      R->ids[L.rank][ch][tid] = iv;
    }
  }
  __syncthreads();
  if (tid == 0) {
    // one release fence (cumulative over the CTA's pushes, which the barrier
    // above ordered before it), then the flags as relaxed stores: a fence per
    // flag (release stores) or a sequentially consistent fence costs several
    // microseconds more per exchange
    fence_acq_rel_sys();
    for (int p = 0; p < n; ++p) st_relaxed_sys(&reinterpret_cast<ShardRegion *>(L.peer[p])->flag_lists[L.rank][ch], epoch);
    const ShardRegion *mine = reinterpret_cast<const ShardRegion *>(L.peer[L.rank]);
    s_ok = wait_flags(&mine->flag_lists[0][ch], SHARD_CELLS * G, n, epoch);
    if (!s_ok) atomicOr(reinterpret_cast<unsigned *>(status), ST_TIMEOUT);
  }
  __syncthreads();
  const ShardRegion *R = reinterpret_cast<const ShardRegion *>(L.peer[L.rank]);
  unsigned long long kv = 0ull;
  int gid = -1;
  if (tid < n * TOPK) {
    const int s = tid / TOPK, r = tid - s * TOPK;
    const uint32_t key = __ldcv(&R->keys[s][ch][r]);
    if (key) {
      gid = L.begin[s] + __ldcv(&R->ids[s][ch][r]);
      kv = ((unsigned long long)(key >> 16) << 48) | ((unsigned long long)(0xffffu - (uint32_t)r) << 32) |
           (unsigned long long)(0xffffffffu - (uint32_t)gid);
    }
  }
  sk[tid] = kv;
  const int valid = __syncthreads_count(kv != 0ull);
  int32_t *dst = out + (size_t)ch * TOPK;
  if (kv) {
    int rank = 0;
    for (int j = 0; j < n * TOPK; ++j) rank += sk[j] > kv;
    if (rank < TOPK) dst[rank] = gid;
  }
  if (tid < TOPK && tid >= valid) dst[tid] = -1;
}

// One CTA per cell: push this shard's partials of the cell to every peer,
// signal, wait for every shard's partials of the cell, combine into BF16.
__global__ void __launch_bounds__(256) k_shard_combine_p2p(ShardLinkDev L, const float *part, uint16_t *out,
                                                          int32_t *status) {
  const int cell = blockIdx.x, g = cell & 3, d = threadIdx.x, n = L.n_shards;
  const uint32_t epoch = *L.epoch + 1;
  __shared__ int s_ok;
  for (int p = 0; p < n; ++p) {
    ShardRegion *R = reinterpret_cast<ShardRegion *>(L.peer[p]);
    for (int i = d; i < G * PART; i += 256) R->part[L.rank][cell][i / PART][i % PART] = part[(size_t)cell * G * PART + i];
  }
  __syncthreads();
  if (d == 0) {
    fence_acq_rel_sys();  // one release fence, cumulative over the CTA's pushes
    for (int p = 0; p < n; ++p) st_relaxed_sys(&reinterpret_cast<ShardRegion *>(L.peer[p])->flag_parts[L.rank][cell], epoch);
    const ShardRegion *mine = reinterpret_cast<const ShardRegion *>(L.peer[L.rank]);
    s_ok = wait_flags(&mine->flag_parts[0][cell], SHARD_CELLS, n, epoch);
    if (!s_ok) atomicOr(reinterpret_cast<unsigned *>(status), ST_TIMEOUT);
  }
  __syncthreads();
  const ShardRegion *R = reinterpret_cast<const ShardRegion *>(L.peer[L.rank]);
  for (int h = 0; h < G; ++h) {
    float M = -INFINITY;
    for (int s = 0; s < n; ++s) M = fmaxf(M, __ldcv(&R->part[s][cell][h][0]));
    float Lsum = 0.0f, O = 0.0f;
    for (int s = 0; s < n; ++s) {
      const float m = __ldcv(&R->part[s][cell][h][0]);
      if (m == -INFINITY) continue;
      const float e = exp2f(m - M);
      Lsum += __ldcv(&R->part[s][cell][h][1]) * e;
      O += __ldcv(&R->part[s][cell][h][4 + d]) * e;
    }
    out[((size_t)(cell >> 2) * 16 + g * 4 + h) * D + d] = bf16_rne(O / Lsum);
  }
}

__global__ void k_shard_epoch(const ShardLinkDev *L) { *L->epoch += 1; }

}  // namespace

cudaError_t launch_shard_merge(const uint32_t *keys, const int32_t *ids, const int32_t *begin, int n_shards,
                               int n_cells, int32_t *out, cudaStream_t st) {
  k_shard_merge<<<n_cells * G, MERGE_THREADS, 0, st>>>(keys, ids, begin, n_shards, n_cells, out);
  return cudaGetLastError();
}

cudaError_t launch_shard_attention(const Work &w, const int32_t *gids, int token_begin, float *partials,
                                   cudaStream_t st) {
  k_shard_attn<<<dim3(ATTN_SPLIT, w.n_cells), 256, 0, st>>>(w, gids, token_begin, partials);
  return cudaGetLastError();
}

cudaError_t launch_shard_combine(const float *partials, int n_shards, int n_cells, uint16_t *out, cudaStream_t st) {
  k_shard_combine<<<n_cells, 256, 0, st>>>(partials, n_shards, n_cells, out);
  return cudaGetLastError();
}

int shard_max_shards() { return MERGE_THREADS / TOPK; }

size_t shard_region_bytes() { return sizeof(ShardRegion); }

cudaError_t launch_shard_p2p_step(const Work &w, const ShardLinkDev &L, int32_t *gids, float *part,
                                  int32_t *status, cudaStream_t st) {
  k_shard_merge_p2p<<<SHARD_CELLS * G, MERGE_THREADS, 0, st>>>(L, w.final_keys, w.final_ids, gids, status);
  k_shard_attn<<<dim3(ATTN_SPLIT, SHARD_CELLS), 256, 0, st>>>(w, gids, L.token_begin, part);
  k_shard_combine_p2p<<<SHARD_CELLS, 256, 0, st>>>(L, part, w.out, status);
  return cudaGetLastError();
}

// The layer grows by m tokens (they joined the last shard): every shard's
// kernel reads the layer's length from its device copy of the group.  An
// append past the group's capacity is skipped, as the last shard skips it.
__global__ void k_link_grow(ShardLinkDev *L, int m, int total_max) {
  if (L->total + m <= total_max) L->total += m;
}

cudaError_t launch_link_grow(ShardLinkDev *dlink, int m, int total_max, cudaStream_t st) {
  k_link_grow<<<1, 1, 0, st>>>(dlink, m, total_max);
  return cudaGetLastError();
}

cudaError_t launch_shard_epoch(const ShardLinkDev *dlink, cudaStream_t st) {
  k_shard_epoch<<<1, 1, 0, st>>>(dlink);
  return cudaGetLastError();
}

}  // namespace skv
