// skv_device.cuh -- shared device helpers and the engine's device layout.
//
// Arithmetic conventions (identical in the CPU oracle):
//   * scoring dot products are exact sums of (operand x small integer) in
//     FP64 on operand rows flushed below 2^(E-24) (E = top exponent of the
//     row), rounded once to FP32;
//   * FP32 post-operations use __f*_rn intrinsics so nothing is contracted;
//   * FP32 -> BF16 rounds to nearest even.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace skv {

constexpr int D = 256;          // head dimension
constexpr int G = 4;            // KV heads per slot == query heads per KV head
constexpr int TOPK = 100;       // final retrieval keys per query head
constexpr int UNION15 = 1600;   // Stage-1.5 frontier entering the union
constexpr int M16 = 256;        // Stage-1.6 survivors per query head
constexpr int M15_MIN = 2048;   // smallest legal Stage-1.5 pool
constexpr int U15_MAX = G * UNION15;
constexpr int CAND_MAX = G * M16;
constexpr int SEL_MAX = G * 512;   // Fine union bound (nprobe <= 512)
constexpr int ATTN_SPLIT = 16;     // attention partitions per KV head
constexpr int REC = 512;           // FP8 [K | V] record bytes
constexpr int NCOUNT = 8;          // per-cell counters

// Per-cell counters (Work::counts[cell][*]).
enum Count { C_TAGS = 0, C_SEL = 1, C_POOL = 2, C_U15 = 3, C_CAND = 4, C_STATUS = 5, C_POSTINGS = 6 };
// Threshold slots (Work::thr[cell][stage][head]).
enum Stage { T_COARSE = 0, T_FINE = 1, T_S15 = 2, T_S16 = 3 };

constexpr uint32_t ST_POOL_OVER = 1u, ST_POOL_UNDER = 2u, ST_FINE_SHORT = 4u;

struct CellDev {
  const uint8_t *upper, *lower;      // [nc][64]
  const float *coarse_scale4;        // [nc/32]
  const float *fine_scale;           // [nc/32]
  const uint16_t *resid;             // [nc] BF16
  const int32_t *offsets;            // [nc+1]
  const int32_t *values;             // [postings]
  const int32_t *mates;              // [postings]
  const uint8_t *prefix2;            // [T][64]
  const uint8_t *residual2;          // [T][64]
  const uint8_t *residual4;          // [T][128]
  const float *key_scale;            // [256]
  const uint8_t *kv8;                // [T][512] FP8 e4m3 [K | V]
  int32_t nc, nprobe;
  float lam;
  int32_t pad;
};

// Workspace: one base pointer per buffer, indexed by cell inside kernels.
struct Work {
  int n_cells, n_slots, T, sink, local, nc, cap;
  const CellDev *cells;
  const uint16_t *q;        // [n_slots][16][256] BF16
  double *ops;              // [cell][3][256][4]  A=q, B=16*q15, Dq=qs (d-major)
  float *qscal;             // [cell][8]  qn[4], 3*sum(q)[4]
  uint16_t *lo, *hi;        // [cell][4][nc] ordered BF16 coarse bounds
  uint32_t *chist;          // [cell][4][256]
  uint32_t *thr;            // [cell][4 stages][4 heads]
  uint32_t *tags;           // [cell][nc]
  uint32_t *fkeys;          // [cell][4][nc]
  int32_t *sel;             // [cell][SEL_MAX]
  uint32_t *selbits;        // [cell][nc/32]
  int32_t *pool;            // [cell][cap]
  uint32_t *k15;            // [cell][4][cap]
  int32_t *u15pos;          // [cell][U15_MAX]
  int32_t *u15tok;          // [cell][U15_MAX]
  uint32_t *k16;            // [cell][4][U15_MAX]
  int32_t *cand;            // [cell][CAND_MAX]
  int32_t *final_pos;       // [cell][4][TOPK]
  int32_t *final_ids;       // [cell][4][TOPK]
  int32_t *counts;          // [cell][NCOUNT]
  float *attn_part;         // [cell][4][ATTN_SPLIT][260]
  uint16_t *out;            // [n_slots][16][256] BF16
};

__device__ __forceinline__ uint16_t bf16_rne(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

__device__ __forceinline__ float bf16f(uint32_t b) { return __uint_as_float(b << 16); }

// Total order of BF16 patterns (reference coarse_select.py:31-36).
__device__ __forceinline__ uint32_t ord16(uint32_t b) {
  return (b ^ (0x8000u | (0u - (b >> 15)))) & 0xffffu;
}

// IEEE order of the Fine key [bf16 score | u16 position] as an unsigned key.
__device__ __forceinline__ uint32_t ord_fused(uint32_t score, uint32_t pos) {
  uint32_t x = (score << 16) | (pos & 0xffffu);
  return (x & 0x80000000u) ? ~x : (x | 0x80000000u);
}

// Exact conversion of a small signed integer to double without I2F.
__device__ __forceinline__ double small2d(int v) {
  return __hiloint2double(0x43300000, v ^ (int)0x80000000) - 4503601774854144.0;
}

// ------------------------------------------------------------ block scans

// Exclusive prefix sum over the block (blockDim.x a multiple of 32, <= 1024).
// Returns this thread's exclusive prefix; *total receives the block sum.
__device__ __forceinline__ int block_exclusive_scan(int v, int *total) {
  __shared__ int s_warp[32];
  __shared__ int s_total;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nwarps ? s_warp[lane] : 0;
    int t = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    if (lane < nwarps) s_warp[lane] = t - w;
    if (lane == 31) s_total = t;
  }
  __syncthreads();
  const int r = s_warp[warp] + x - v;
  *total = s_total;
  __syncthreads();
  return r;
}

// Given a 256-bin histogram in shared memory, find the bin holding the k-th
// largest element (1-based k) scanning from bin 255 down.  Executed by warp 0;
// results are written to *bin and *above (count strictly above that bin).
__device__ __forceinline__ void find_bin_desc(const uint32_t *hist, uint32_t k, int *bin,
                                              uint32_t *above) {
  const int lane = threadIdx.x & 31;
  // lane l owns bins [255-8l-7, 255-8l], i.e. the l-th block from the top
  uint32_t c[8];
  uint32_t s = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) { c[j] = hist[255 - 8 * lane - j]; s += c[j]; }
  uint32_t incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  const uint32_t excl = incl - s;
  if (excl < k && k <= incl) {
    uint32_t acc = excl;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (acc + c[j] >= k) { *bin = 255 - 8 * lane - j; *above = acc; break; }
      acc += c[j];
    }
  }
}

}  // namespace skv
