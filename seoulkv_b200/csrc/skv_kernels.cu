// skv_kernels.cu -- the sparse-decode funnel as sm_100a CUDA kernels.
//
// One step decodes one query token for every cell (slot x KV head).  Cells
// index blockIdx.y (or blockIdx.x for one-CTA-per-cell kernels), so a batch
// of requests or a stack of layers runs as one launch per stage.
//
//   k_qprep          exact operand digits (int8 fragments), lambda*|q|, 3*sum(q)
//   k_coarse         2-bit centroid intervals [lo, hi] on int8 tensor cores
//   k_coarse_thresh  P-th largest lower bound per head (16-bit radix select)
//   k_surv_count     survivor head masks + survivors per 1024-centroid chunk
//   k_fine           survivor tags + 4-bit rescoring -> fused IEEE keys
//   k_select_fine    top-nprobe threshold per head, selected-cluster bitmap
//   k_pool_count     kept postings per selected cluster (spill-2 mate rule)
//   k_pool_write     first-occurrence pool, ordered by (cluster, posting)
//   k_s15            2-bit key scores of the pool
//   k_select_s15     top-1600 threshold per head, union bitmap
//   k_s16            union compaction + 4-bit rescoring
//   k_select_s16     top-256 threshold per head, candidate bitmap
//   k_s2             candidates, 8-bit scores, exact top-100 per head
//   k_attn           FP8 sink + local + top-100 online softmax, LSE combine
#include <cuda_fp8.h>

#include "skv_codec.cuh"
#include "skv_device.cuh"
#include "skv_kernels.cuh"
#include "skv_select.cuh"

namespace skv {

// ------------------------------------------------------------------ qprep

// One CTA per (operand row, query head, cell); thread d = dimension.  Writes
// the int8 digit fragments of the row (q, 16*bf16(q*s/64) or bf16(q*s/256)),
// its scale, and for the q row lambda*|q| and 3*sum(q).
__global__ void __launch_bounds__(256) k_qprep(Work w) {
  const int r = blockIdx.x >> 2, h = blockIdx.x & 3, cell = blockIdx.y, slot = cell >> 2, g = cell & 3;
  const int d = threadIdx.x, lane = d & 31, warp = d >> 5;
  __shared__ int sE[8];
  __shared__ float sx[D];
  const float xa = bf16f(w.q[((size_t)slot * 16 + g * 4 + h) * D + d]);
  float x = xa;
  if (r != R_Q) {
    const float prod = __fmul_rn(xa, w.cells[cell].key_scale[d]);
    x = r == R_Q15 ? __fmul_rn(bf16f(bf16_rne(__fmul_rn(prod, 0.015625f))), 16.0f)
                   : bf16f(bf16_rne(__fmul_rn(prod, 0.00390625f)));
  }
  int e = x != 0.0f ? ilogbf(x) : INT_MIN;
  e = __reduce_max_sync(0xffffffffu, e);
  if (lane == 0) sE[warp] = e;
  sx[d] = xa;
  __syncthreads();
  int E = INT_MIN;
#pragma unroll
  for (int k = 0; k < 8; ++k) E = max(E, sE[k]);
  int X = 0;
  if (E != INT_MIN) {
    const double v = (double)x;
    // kept elements are integers on the 2^(E-29) grid, |X| < 2^30
    if (!(fabs(v) < ldexp(1.0, E - 22))) X = __double2int_rn(ldexp(v, 29 - E));
  }
  // four signed base-256 digits, X = d0 + 2^8 d1 + 2^16 d2 + 2^24 d3
  int dg[4];
  dg[0] = (int)(int8_t)(X & 0xff);
  int rest = (X - dg[0]) >> 8;
  dg[1] = (int)(int8_t)(rest & 0xff);
  rest = (rest - dg[1]) >> 8;
  dg[2] = (int)(int8_t)(rest & 0xff);
  dg[3] = (rest - dg[2]) >> 8;
  // fragment byte of dimension d: k-step, register, byte, thread-in-quad
  const int ks = d >> 5, reg = (d >> 4) & 1, byte = (d >> 2) & 3, tq = d & 3, nt = h >> 1;
  uint8_t *frag = reinterpret_cast<uint8_t *>(w.frag + ((size_t)cell * 3 + r) * FRAG_ROW);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int lane_b = 4 * (4 * (h & 1) + j) + tq;
    frag[(((ks * 2 + nt) * 32 + lane_b) * 2 + reg) * 4 + byte] = (uint8_t)(int8_t)dg[j];
  }
  if (d == 0) w.shift[(cell * 3 + r) * G + h] = E == INT_MIN ? 0 : E - 29;
  if (r == R_Q && warp == 0) {
    // pairwise (recursive halving) FP64 sums in dimension order
    double v[8], sq[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) { v[j] = (double)sx[8 * lane + j]; sq[j] = v[j] * v[j]; }
    double a = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
    double b = ((sq[0] + sq[1]) + (sq[2] + sq[3])) + ((sq[4] + sq[5]) + (sq[6] + sq[7]));
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      a = a + __shfl_xor_sync(0xffffffffu, a, o);
      b = b + __shfl_xor_sync(0xffffffffu, b, o);
    }
    if (lane == 0) {
      const float norm = __double2float_rn(__dsqrt_rn(b));
      w.qscal[cell * 8 + h] = __fmul_rn(norm, w.cells[cell].lam);
      w.qscal[cell * 8 + 4 + h] = __fmul_rn(3.0f, __double2float_rn(a));
    }
  }
  if (r == 0 && h == 0 && d < NCOUNT) w.counts[cell * NCOUNT + d] = 0;
}

// ----------------------------------------------------------------- coarse

__device__ __forceinline__ void load_row64(const uint8_t *base, int row, uint4 (&r)[4]) {
  const uint4 *p = reinterpret_cast<const uint4 *>(base + (size_t)row * 64);
#pragma unroll
  for (int k = 0; k < 4; ++k) r[k] = p[k];
}

__global__ void __launch_bounds__(256) k_coarse(Work w) {
  const int cell = blockIdx.y, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const CellDev &c = w.cells[cell];
  const int nc = w.nc;
  BFrag F;
  load_bfrag(w, cell, R_Q, lane, F);
  const int hA = t >> 1, hB = 2 + hA;
  const Pow2 scA = pow2s(w.shift[(cell * 3 + R_Q) * G + hA]);
  const Pow2 scB = pow2s(w.shift[(cell * 3 + R_Q) * G + hB]);
  const float qnA = w.qscal[cell * 8 + hA], qnB = w.qscal[cell * 8 + hB];
  const float c3A = w.qscal[cell * 8 + 4 + hA], c3B = w.qscal[cell * 8 + 4 + hB];
  const int tiles = nc >> 4, stride = gridDim.x * 8;
  int tile = blockIdx.x * 8 + warp;
  uint4 x[4], y[4], nx[4], ny[4];
  if (tile < tiles) { load_row64(c.upper, tile * 16 + g, x); load_row64(c.upper, tile * 16 + g + 8, y); }
  for (; tile < tiles; tile += stride) {
    const int next = tile + stride;
    if (next < tiles) { load_row64(c.upper, next * 16 + g, nx); load_row64(c.upper, next * 16 + g + 8, ny); }
    int acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const uint32_t a0 = w2(word_of(x, 2 * ks), t), a1 = w2(word_of(y, 2 * ks), t);
      const uint32_t a2 = w2(word_of(x, 2 * ks + 1), t), a3 = w2(word_of(y, 2 * ks + 1), t);
      mma_s8(acc[0], a0, a1, a2, a3, F.b[ks][0][0], F.b[ks][0][1]);
      mma_s8(acc[1], a0, a1, a2, a3, F.b[ks][1][0], F.b[ks][1][1]);
    }
    long long dsum[2];
    combine_digits(acc, t, dsum);
    const int row = tile * 16 + g + ((t & 1) << 3);
    const float sc4 = c.coarse_scale4[row >> 5];
    const float r = bf16f(c.resid[row]);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int h = k ? hB : hA;
      const float dot = exact_to_float(dsum[k], k ? scB : scA);
      const float centered = __fsub_rn(__fmul_rn(2.0f, dot), k ? c3B : c3A);
      const float v = __fmul_rn(centered, sc4);
      const float margin = __fmul_rn(k ? qnB : qnA, r);
      const uint32_t lo = ord16(bf16_score(__fsub_rn(v, margin)));
      const uint32_t hi = ord16(bf16_score(__fadd_rn(v, margin)));
      w.lo[((size_t)cell * G + h) * nc + row] = (uint16_t)lo;
      w.hi[((size_t)cell * G + h) * nc + row] = (uint16_t)hi;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) { x[k] = nx[k]; y[k] = ny[k]; }
  }
}

// P-th largest lower bound per (cell, head): a 12-bit histogram pass and a
// 4-bit pass restricted to the boundary bin, both over the L2-resident bounds.
__global__ void __launch_bounds__(1024) k_coarse_thresh(Work w) {
  const int h = blockIdx.x, cell = blockIdx.y, tid = threadIdx.x;
  const int nc = w.nc;
  const uint32_t P = (uint32_t)w.cells[cell].nprobe;
  __shared__ uint32_t hist[4096];
  for (int i = tid; i < 4096; i += 1024) hist[i] = 0;
  __syncthreads();
  const uint4 *lo4 = reinterpret_cast<const uint4 *>(w.lo + ((size_t)cell * G + h) * nc);
#pragma unroll 4
  for (int i = tid; i < (nc >> 3); i += 1024) {
    const uint4 v = lo4[i];
    const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      atomicAdd(&hist[(wv[j] & 0xffffu) >> 4], 1u);
      atomicAdd(&hist[wv[j] >> 20], 1u);
    }
  }
  __syncthreads();
  int top;
  uint32_t above;
  block_find_bin(hist, 4096, P, &top, &above);
  if (tid < 16) hist[tid] = 0;
  __syncthreads();
  const uint4 *lo = reinterpret_cast<const uint4 *>(w.lo + ((size_t)cell * G + h) * nc);
  const int n8 = nc >> 3;
#pragma unroll 4
  for (int i = tid; i < n8; i += 1024) {
    const uint4 v = lo[i];
    const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t k0 = wv[j] & 0xffffu, k1 = wv[j] >> 16;
      if ((int)(k0 >> 4) == top) atomicAdd(&hist[k0 & 15u], 1u);
      if ((int)(k1 >> 4) == top) atomicAdd(&hist[k1 & 15u], 1u);
    }
  }
  __syncthreads();
  if (tid == 0) {
    uint32_t acc = above, low = 0;
    for (int b = 15; b >= 0; --b) {
      if (acc + hist[b] >= P) { low = (uint32_t)b; break; }
      acc += hist[b];
    }
    w.thr[(size_t)cell * 16 + T_COARSE * G + h] = ((uint32_t)top << 4) | low;
  }
}

// Survivor masks (bit h: hi_h >= threshold_h) and survivors per chunk.
__global__ void __launch_bounds__(256) k_surv_count(Work w) {
  const int chunk = blockIdx.x, cell = blockIdx.y, nc = w.nc;
  const uint32_t *thr = w.thr + (size_t)cell * 16 + T_COARSE * G;
  const int i = chunk * CHUNK + 4 * threadIdx.x;
  int cnt = 0;
  if (i < nc) {
    uint32_t m[4] = {0, 0, 0, 0};
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const uint2 v = *reinterpret_cast<const uint2 *>(w.hi + ((size_t)cell * G + h) * nc + i);
      const uint32_t th = thr[h];
      m[0] |= (uint32_t)((v.x & 0xffffu) >= th) << h;
      m[1] |= (uint32_t)((v.x >> 16) >= th) << h;
      m[2] |= (uint32_t)((v.y & 0xffffu) >= th) << h;
      m[3] |= (uint32_t)((v.y >> 16) >= th) << h;
    }
    *reinterpret_cast<uchar4 *>(w.smask + (size_t)cell * nc + i) =
        make_uchar4((uint8_t)m[0], (uint8_t)m[1], (uint8_t)m[2], (uint8_t)m[3]);
    cnt = (m[0] != 0) + (m[1] != 0) + (m[2] != 0) + (m[3] != 0);
  }
  int total;
  block_exclusive_scan(cnt, &total);
  if (threadIdx.x == 0) w.chunk_cnt[(size_t)cell * w.chunks_nc + chunk] = total;
}

// ------------------------------------------------------------------- fine

__global__ void __launch_bounds__(256) k_fine(Work w) {
  const int chunk = blockIdx.x, cell = blockIdx.y, nc = w.nc;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
  const CellDev &c = w.cells[cell];
  __shared__ int s_cid[CHUNK];
  __shared__ uint8_t s_mask[CHUNK];
  const int base = block_sum_prefix(w.chunk_cnt + (size_t)cell * w.chunks_nc, chunk);
  const int i = chunk * CHUNK + 4 * tid;
  uint32_t m[4] = {0, 0, 0, 0};
  if (i < nc) {
    const uchar4 v = *reinterpret_cast<const uchar4 *>(w.smask + (size_t)cell * nc + i);
    m[0] = v.x; m[1] = v.y; m[2] = v.z; m[3] = v.w;
  }
  int total;
  int r = block_exclusive_scan((m[0] != 0) + (m[1] != 0) + (m[2] != 0) + (m[3] != 0), &total);
#pragma unroll
  for (int k = 0; k < 4; ++k)
    if (m[k]) {
      s_cid[r] = i + k;
      s_mask[r] = (uint8_t)m[k];
      w.tags[(size_t)cell * nc + base + r] = (uint32_t)(i + k) | (m[k] << 28);
      ++r;
    }
  if (chunk == gridDim.x - 1 && tid == 0) w.counts[cell * NCOUNT + C_TAGS] = base + total;
  __syncthreads();
  BFrag F;
  load_bfrag(w, cell, R_Q, lane, F);
  const int hA = t >> 1, hB = 2 + hA;
  const Pow2 scA = pow2s(w.shift[(cell * 3 + R_Q) * G + hA]);
  const Pow2 scB = pow2s(w.shift[(cell * 3 + R_Q) * G + hB]);
  for (int tile = warp; tile * 16 < total; tile += 8) {
    const int rg = tile * 16 + g, r8 = rg + 8;
    const int cg = rg < total ? s_cid[rg] : 0, c8 = r8 < total ? s_cid[r8] : 0;
    uint4 ug[4], lg[4], u8[4], l8[4];
    load_row64(c.upper, cg, ug);
    load_row64(c.lower, cg, lg);
    load_row64(c.upper, c8, u8);
    load_row64(c.lower, c8, l8);
    int acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const uint32_t a0 = w_odd4(w2(word_of(ug, 2 * ks), t), w2(word_of(lg, 2 * ks), t));
      const uint32_t a1 = w_odd4(w2(word_of(u8, 2 * ks), t), w2(word_of(l8, 2 * ks), t));
      const uint32_t a2 = w_odd4(w2(word_of(ug, 2 * ks + 1), t), w2(word_of(lg, 2 * ks + 1), t));
      const uint32_t a3 = w_odd4(w2(word_of(u8, 2 * ks + 1), t), w2(word_of(l8, 2 * ks + 1), t));
      mma_s8(acc[0], a0, a1, a2, a3, F.b[ks][0][0], F.b[ks][0][1]);
      mma_s8(acc[1], a0, a1, a2, a3, F.b[ks][1][0], F.b[ks][1][1]);
    }
    long long dsum[2];
    combine_digits(acc, t, dsum);
    const int row = (t & 1) ? r8 : rg;
    if (row < total) {
      const int cid = s_cid[row], mk = s_mask[row], pos = base + row;
      const float fs = c.fine_scale[cid >> 5];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int h = k ? hB : hA;
        uint32_t key = 0;
        if ((mk >> h) & 1) {
          key = ord_fused(bf16_score(__fmul_rn(exact_to_float(dsum[k], k ? scB : scA), fs)), (uint32_t)pos);
        }
        w.fkeys[((size_t)cell * G + h) * nc + pos] = key;
      }
    }
  }
}

// ----------------------------------------------------------------- select

constexpr int SELECT_SMEM_KEYS = 40960;

// Copy n keys into shared memory with many loads in flight.
__device__ __forceinline__ void stage_keys(uint32_t *dst, const uint32_t *src, int n) {
  const int nb = blockDim.x;
#pragma unroll 8
  for (int i = threadIdx.x; i < n; i += nb) dst[i] = src[i];
}

// Threshold of the top-K of one (cell, head) and the union bitmap update.
// kind: 0 = Fine (K = nprobe, keys indexed by survivor position),
//       1 = Stage-1.5 (K = min(1600, n)), 2 = Stage-1.6 (K = min(256, n)).
__global__ void __launch_bounds__(1024) k_select(Work w, int kind) {
  extern __shared__ uint32_t skeys[];
  const int h = blockIdx.x, cell = blockIdx.y;
  const uint32_t *src;
  uint32_t *bits;
  int n, stage;
  uint32_t K;
  if (kind == 0) {
    n = w.counts[cell * NCOUNT + C_TAGS];
    K = (uint32_t)w.cells[cell].nprobe;
    src = w.fkeys + ((size_t)cell * G + h) * w.nc;
    bits = w.selbits + (size_t)cell * (w.nc >> 5);
    stage = T_FINE;
  } else if (kind == 1) {
    n = min(w.counts[cell * NCOUNT + C_POOL], w.cap);
    K = (uint32_t)min(UNION15, n);
    src = w.k15 + ((size_t)cell * G + h) * w.cap;
    bits = w.u15bits + (size_t)cell * (w.cap >> 5);
    stage = T_S15;
  } else {
    n = w.counts[cell * NCOUNT + C_U15];
    K = (uint32_t)min(M16, n);
    src = w.k16 + ((size_t)cell * G + h) * U15_MAX;
    bits = w.candbits + (size_t)cell * (U15_MAX >> 5);
    stage = T_S16;
  }
  __shared__ SelectScratch sc;
  const bool in_smem = n <= SELECT_SMEM_KEYS;
  const uint32_t *p = in_smem ? skeys : src;
  for (int i = threadIdx.x; i < SEL_BINS; i += blockDim.x) sc.hist[i] = 0;
  if (threadIdx.x == 0) sc.n_list = 0;
  __syncthreads();
  // pass 1: stage the keys (vector loads) and histogram their top 12 bits
  const int n4 = n >> 2;
  const uint4 *src4 = reinterpret_cast<const uint4 *>(src);
#pragma unroll 4
  for (int i = threadIdx.x; i < n4 + 1; i += blockDim.x) {
    uint32_t v[4];
    int cnt = 4;
    if (i < n4) {
      const uint4 x = src4[i];
      v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
    } else {
      cnt = n - 4 * n4;
      for (int j = 0; j < cnt; ++j) v[j] = src[4 * n4 + j];
    }
    for (int j = 0; j < cnt; ++j) {
      if (in_smem) skeys[4 * i + j] = v[j];
      atomicAdd(&sc.hist[v[j] >> 20], 1u);
    }
  }
  __syncthreads();
  int top;
  uint32_t above;
  block_find_bin(sc.hist, SEL_BINS, K, &top, &above);  // (synchronises)
  // pass 2: collect the boundary bin
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const uint32_t v = p[i];
    if ((int)(v >> 20) == top) {
      const int slot = atomicAdd(&sc.n_list, 1);
      if (slot < SEL_LIST) sc.list[slot] = v;
    }
  }
  __syncthreads();
  uint32_t th;
  if (K == 0) {
    th = 0xffffffffu;
  } else if (top < 0 || (int)K > n) {
    th = 0u;  // K-th largest not found: fewer than K keys
  } else {
    const int m = sc.n_list;
    __syncthreads();
    if (m <= SEL_LIST) th = radix_refine(sc.list, m, (uint32_t)top << 20, 0xfff00000u, 20, K - above, sc);
    else th = radix_refine(p, n, (uint32_t)top << 20, 0xfff00000u, 20, K - above, sc);
  }
  if (th == 0) th = 0xffffffffu;  // fewer than K eligible keys: select nothing
  if (threadIdx.x == 0) {
    w.thr[(size_t)cell * 16 + stage * G + h] = th;
    if (kind == 0 && th == 0xffffffffu)
      atomicOr(reinterpret_cast<unsigned *>(&w.counts[cell * NCOUNT + C_STATUS]), ST_FINE_SHORT);
  }
  const uint32_t *tags = w.tags + (size_t)cell * w.nc;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    if (p[i] < th) continue;
    const uint32_t b = kind == 0 ? (tags[i] & 0x0fffffffu) : (uint32_t)i;
    atomicOr(&bits[b >> 5], 1u << (b & 31));
  }
}

// ------------------------------------------------------------------- pool

// For every survivor of this chunk: whether its cluster is selected and how
// many of its postings are first occurrences.  A posting is a duplicate
// exactly when its token's other list (its mate) is selected and comes
// earlier in ascending cluster order.
__global__ void __launch_bounds__(SCHUNK) k_pool_count(Work w) {
  const int chunk = blockIdx.x, cell = blockIdx.y, tid = threadIdx.x;
  const int ntags = w.counts[cell * NCOUNT + C_TAGS];
  if (chunk * SCHUNK >= ntags) return;
  const CellDev &c = w.cells[cell];
  const uint32_t *bits = w.selbits + (size_t)cell * (w.nc >> 5);
  const int i = chunk * SCHUNK + tid;
  int kept = 0, sel = 0, post = 0;
  if (i < ntags) {
    const int cid = (int)(w.tags[(size_t)cell * w.nc + i] & 0x0fffffffu);
    const uint32_t own = bits[cid >> 5];
    const int b = c.offsets[cid], e = c.offsets[cid + 1];
    if ((own >> (cid & 31)) & 1u) {
      sel = 1;
      post = e - b;
      unsigned long long mk = 0;
      for (int j0 = b; j0 < e; j0 += 16) {
        int m[16];
        uint32_t mw[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) m[u] = j0 + u < e ? c.mates[j0 + u] : -1;
#pragma unroll
        for (int u = 0; u < 16; ++u) mw[u] = (m[u] >= 0 && m[u] < cid) ? bits[m[u] >> 5] : 0u;
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const bool keep = j0 + u < e && !(m[u] >= 0 && m[u] < cid && ((mw[u] >> (m[u] & 31)) & 1u));
          if (keep) {
            ++kept;
            if (j0 + u - b < 64) mk |= 1ull << (j0 + u - b);
          }
        }
      }
      w.keptmask[(size_t)cell * w.nc + i] = mk;
    }
    w.kept[(size_t)cell * w.nc + i] = (uint16_t)kept;
  }
  __shared__ int s3[3][SCHUNK / 32];
  int v[3] = {kept, sel, post};
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    int x = v[k];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    if ((tid & 31) == 0) s3[k][tid >> 5] = x;
  }
  __syncthreads();
  if (tid < 3) {
    int x = 0;
    for (int k = 0; k < SCHUNK / 32; ++k) x += s3[tid][k];
    int32_t *dst = tid == 0 ? w.chunk_kept : tid == 1 ? w.chunk_sel : w.chunk_post;
    dst[(size_t)cell * w.chunks_surv + chunk] = x;
  }
}

constexpr int POOL_LIST = 2048;  // pool entries of one chunk scored from shared memory

// Chunk of 256 survivors: write its first-occurrence postings to the pool at
// their global positions (ascending cluster, then CSR order) and score them
// with 2-bit key codes for the four query heads.
__global__ void __launch_bounds__(SCHUNK) k_pool_s15(Work w) {
  const int chunk = blockIdx.x, cell = blockIdx.y, tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
  const int ntags = w.counts[cell * NCOUNT + C_TAGS];
  const int used = (ntags + SCHUNK - 1) / SCHUNK;
  const bool last = chunk == used - 1 || (used == 0 && chunk == 0);
  if (chunk >= used && !last) return;
  const CellDev &c = w.cells[cell];
  __shared__ int s_tok[POOL_LIST];
  const int32_t *ck = w.chunk_kept + (size_t)cell * w.chunks_surv;
  const int32_t *cs = w.chunk_sel + (size_t)cell * w.chunks_surv;
  int pk = 0, ps = 0;
  for (int k = tid; k < chunk; k += SCHUNK) { pk += ck[k]; ps += cs[k]; }
  int base_kept, base_sel;
  block_exclusive_scan(pk, &base_kept);
  block_exclusive_scan(ps, &base_sel);
  const uint32_t *bits = w.selbits + (size_t)cell * (w.nc >> 5);
  const int i = chunk * SCHUNK + tid;
  int kept = 0, sel = 0, cid = 0;
  if (i < ntags) {
    cid = (int)(w.tags[(size_t)cell * w.nc + i] & 0x0fffffffu);
    sel = (bits[cid >> 5] >> (cid & 31)) & 1u;
    if (sel) kept = w.kept[(size_t)cell * w.nc + i];
  }
  int tot_kept, tot_sel;
  const int r0 = block_exclusive_scan(kept, &tot_kept);
  const int rs = base_sel + block_exclusive_scan(sel, &tot_sel);
  int32_t *pool = w.pool + (size_t)cell * w.cap;
  if (sel) {
    if (rs < SEL_MAX) w.sel[(size_t)cell * SEL_MAX + rs] = cid;
    const int b = c.offsets[cid], e = c.offsets[cid + 1];
    const unsigned long long mk = w.keptmask[(size_t)cell * w.nc + i];
    int r = r0;
#pragma unroll 4
    for (int j = b; j < e; ++j) {
      bool keep;
      if (j - b < 64) {
        keep = (mk >> (j - b)) & 1ull;
      } else {
        const int m = c.mates[j];
        keep = m < 0 || m > cid || !((bits[m >> 5] >> (m & 31)) & 1u);
      }
      if (keep) {
        const int tok = c.values[j];
        if (base_kept + r < w.cap) pool[base_kept + r] = tok;
        if (r < POOL_LIST) s_tok[r] = tok;
        ++r;
      }
    }
  }
  int posts = 0;
  if (last) {
    int pp = 0;
    for (int k = tid; k < used; k += SCHUNK) pp += w.chunk_post[(size_t)cell * w.chunks_surv + k];
    block_exclusive_scan(pp, &posts);
  }
  if (last && tid == 0) {
    int *cnt = w.counts + cell * NCOUNT;
    const int npool = base_kept + tot_kept;
    cnt[C_POOL] = npool;
    cnt[C_SEL] = min(base_sel + tot_sel, SEL_MAX);
    cnt[C_POSTINGS] = posts;
    uint32_t st = 0;
    if (npool > w.cap) st |= ST_POOL_OVER;
    if (npool < M15_MIN) st |= ST_POOL_UNDER;
    if (st) atomicOr(reinterpret_cast<unsigned *>(&cnt[C_STATUS]), st);
  }
  __syncthreads();
  // score this chunk's pool entries [base_kept, base_kept + nloc)
  const int nloc = min(tot_kept, w.cap - base_kept);
  if (nloc <= 0) return;
  BFrag F;
  load_bfrag(w, cell, R_Q15, lane, F);
  const int hA = t >> 1, hB = 2 + hA;
  const Pow2 scA = pow2s(w.shift[(cell * 3 + R_Q15) * G + hA]);
  const Pow2 scB = pow2s(w.shift[(cell * 3 + R_Q15) * G + hB]);
  for (int tile = warp; tile * 16 < nloc; tile += SCHUNK / 32) {
    const int rg = tile * 16 + g, r8 = rg + 8;
    const int tg = rg < nloc ? (rg < POOL_LIST ? s_tok[rg] : pool[base_kept + rg]) : 0;
    const int t8 = r8 < nloc ? (r8 < POOL_LIST ? s_tok[r8] : pool[base_kept + r8]) : 0;
    uint4 pg[4], p8[4];
    load_row64(c.prefix2, tg, pg);
    load_row64(c.prefix2, t8, p8);
    int acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const uint32_t a0 = w_odd2(w2(word_of(pg, 2 * ks), t)), a1 = w_odd2(w2(word_of(p8, 2 * ks), t));
      const uint32_t a2 = w_odd2(w2(word_of(pg, 2 * ks + 1), t)), a3 = w_odd2(w2(word_of(p8, 2 * ks + 1), t));
      mma_s8(acc[0], a0, a1, a2, a3, F.b[ks][0][0], F.b[ks][0][1]);
      mma_s8(acc[1], a0, a1, a2, a3, F.b[ks][1][0], F.b[ks][1][1]);
    }
    long long dsum[2];
    combine_digits(acc, t, dsum);
    const int row = (t & 1) ? r8 : rg;
    if (row < nloc) {
      const uint32_t pos = (uint32_t)(base_kept + row);
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const uint32_t sc = ord16(bf16_score(exact_to_float(dsum[k], k ? scB : scA)));
        const uint32_t key = (sc << 16) | (0xffffu - pos);
        w.k15[((size_t)cell * G + (k ? hB : hA)) * w.cap + pos] = key;
      }
    }
  }
}

// ------------------------------------------------------------ stage 1.6

constexpr int S16_CHUNK = 256;  // pool positions per k_s16 CTA (one per thread)

// Chunk of 256 pool positions: rank the union members (ascending pool
// position), record them, and score them with 4-bit codes.
__global__ void __launch_bounds__(256) k_s16(Work w) {
  const int chunk = blockIdx.x, cell = blockIdx.y, tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
  const int n = min(w.counts[cell * NCOUNT + C_POOL], w.cap);
  if (chunk * S16_CHUNK >= n && chunk != gridDim.x - 1) return;
  const CellDev &c = w.cells[cell];
  const uint32_t *bits = w.u15bits + (size_t)cell * (w.cap >> 5);
  __shared__ int s_tok[S16_CHUNK];
  __shared__ int s_u[S16_CHUNK];
  // union members before this chunk
  int before = 0;
  for (int k = tid; k < chunk * (S16_CHUNK / 32); k += 256) before += __popc(bits[k]);
  int base;
  block_exclusive_scan(before, &base);
  const int p0 = chunk * S16_CHUNK + tid;
  const int mine = p0 < n ? (int)((bits[p0 >> 5] >> (p0 & 31)) & 1u) : 0;
  int total;
  const int r = block_exclusive_scan(mine, &total);
  const int32_t *pool = w.pool + (size_t)cell * w.cap;
  if (mine) {
    const int u = base + r;
    const int tok = pool[p0];
    s_tok[r] = tok;
    s_u[r] = u;
    if (u < U15_MAX) {
      w.u15pos[(size_t)cell * U15_MAX + u] = p0;
      w.u15tok[(size_t)cell * U15_MAX + u] = tok;
    }
  }
  if (chunk == gridDim.x - 1 && tid == 0) w.counts[cell * NCOUNT + C_U15] = min(base + total, U15_MAX);
  __syncthreads();
  BFrag F;
  load_bfrag(w, cell, R_QS, lane, F);
  const int hA = t >> 1, hB = 2 + hA;
  const Pow2 scA = pow2s(w.shift[(cell * 3 + R_QS) * G + hA] + 4);
  const Pow2 scB = pow2s(w.shift[(cell * 3 + R_QS) * G + hB] + 4);
  for (int tile = warp; tile * 16 < total; tile += 8) {
    const int rg = tile * 16 + g, r8 = rg + 8;
    const int tg = rg < total ? s_tok[rg] : 0, t8 = r8 < total ? s_tok[r8] : 0;
    uint4 pg[4], qg[4], p8[4], q8[4];
    load_row64(c.prefix2, tg, pg);
    load_row64(c.residual2, tg, qg);
    load_row64(c.prefix2, t8, p8);
    load_row64(c.residual2, t8, q8);
    int acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const uint32_t a0 = w_odd4(w2(word_of(pg, 2 * ks), t), w2(word_of(qg, 2 * ks), t));
      const uint32_t a1 = w_odd4(w2(word_of(p8, 2 * ks), t), w2(word_of(q8, 2 * ks), t));
      const uint32_t a2 = w_odd4(w2(word_of(pg, 2 * ks + 1), t), w2(word_of(qg, 2 * ks + 1), t));
      const uint32_t a3 = w_odd4(w2(word_of(p8, 2 * ks + 1), t), w2(word_of(q8, 2 * ks + 1), t));
      mma_s8(acc[0], a0, a1, a2, a3, F.b[ks][0][0], F.b[ks][0][1]);
      mma_s8(acc[1], a0, a1, a2, a3, F.b[ks][1][0], F.b[ks][1][1]);
    }
    long long dsum[2];
    combine_digits(acc, t, dsum);
    const int row = (t & 1) ? r8 : rg;
    if (row < total) {
      const int u = s_u[row];
      if (u < U15_MAX) {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const int h = k ? hB : hA;
          // operand 16*qs: the same digits with the scale raised by 2^4
          const uint32_t s = ord16(bf16_score(exact_to_float(dsum[k], k ? scB : scA)));
          const uint32_t key = (s << 16) | (0xffffu - (uint32_t)u);
          w.k16[((size_t)cell * G + h) * U15_MAX + u] = key;
        }
      }
    }
  }
}

// ------------------------------------------------------------- stage II

__device__ __forceinline__ void load_row128(const uint8_t *base, int row, uint4 (&r)[8]) {
  const uint4 *p = reinterpret_cast<const uint4 *>(base + (size_t)row * 128);
#pragma unroll
  for (int k = 0; k < 8; ++k) r[k] = p[k];
}

__device__ __forceinline__ uint32_t word8_of(const uint4 (&r)[8], int i) {
  const uint4 v = r[i >> 2];
  return (i & 3) == 0 ? v.x : (i & 3) == 1 ? v.y : (i & 3) == 2 ? v.z : v.w;
}

constexpr int S2_ROWS = 128;  // candidates scored per k_s2_score CTA (8 warps x 16)

// Candidates (set bits of the Stage-1.6 union bitmap, ascending) ranked
// [128*part, 128*part + 128): 8-bit scores for all four heads.
__global__ void __launch_bounds__(256) k_s2_score(Work w) {
  const int part = blockIdx.x, cell = blockIdx.y, tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
  const CellDev &c = w.cells[cell];
  __shared__ int32_t s_cand[S2_ROWS];
  __shared__ int32_t s_tok[S2_ROWS];
  const int nu = w.counts[cell * NCOUNT + C_U15];
  const uint32_t word = tid < (U15_MAX >> 5) ? w.candbits[(size_t)cell * (U15_MAX >> 5) + tid] : 0u;
  int total;
  int r = block_exclusive_scan(__popc(word), &total);
  const int ncand = min(total, CAND_MAX);
  const int lo_rank = part * S2_ROWS;
  for (uint32_t m = word; m; m &= m - 1) {
    const int u = tid * 32 + __ffs(m) - 1;
    if (r >= lo_rank && r < lo_rank + S2_ROWS && r < CAND_MAX) {
      s_cand[r - lo_rank] = u;
      s_tok[r - lo_rank] = u < nu ? w.u15tok[(size_t)cell * U15_MAX + u] : 0;
      w.cand[(size_t)cell * CAND_MAX + r] = u;
    }
    ++r;
  }
  if (part == 0 && tid == 0) w.counts[cell * NCOUNT + C_CAND] = ncand;
  __syncthreads();
  const int nloc = min(S2_ROWS, ncand - lo_rank);
  if (nloc <= 0 || warp * 16 >= nloc) return;
  BFrag F;
  load_bfrag(w, cell, R_QS, lane, F);
  const int hA = t >> 1, hB = 2 + hA;
  const Pow2 scA = pow2s(w.shift[(cell * 3 + R_QS) * G + hA]);
  const Pow2 scB = pow2s(w.shift[(cell * 3 + R_QS) * G + hB]);
  const int rg = warp * 16 + g, r8 = rg + 8;
  const int tg = rg < nloc ? s_tok[rg] : 0, t8 = r8 < nloc ? s_tok[r8] : 0;
  const uint2 *pg = reinterpret_cast<const uint2 *>(c.prefix2 + (size_t)tg * 64);
  const uint2 *qg = reinterpret_cast<const uint2 *>(c.residual2 + (size_t)tg * 64);
  const uint4 *ng = reinterpret_cast<const uint4 *>(c.residual4 + (size_t)tg * 128);
  const uint2 *p8 = reinterpret_cast<const uint2 *>(c.prefix2 + (size_t)t8 * 64);
  const uint2 *q8 = reinterpret_cast<const uint2 *>(c.residual2 + (size_t)t8 * 64);
  const uint4 *n8 = reinterpret_cast<const uint4 *>(c.residual4 + (size_t)t8 * 128);
  int hi[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}}, lo[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const uint2 vpg = pg[ks], vqg = qg[ks], vp8 = p8[ks], vq8 = q8[ks];
    const uint4 vng = ng[ks], vn8 = n8[ks];
    const uint32_t a0 = w_odd4(w2(vpg.x, t), w2(vqg.x, t));
    const uint32_t a1 = w_odd4(w2(vp8.x, t), w2(vq8.x, t));
    const uint32_t a2 = w_odd4(w2(vpg.y, t), w2(vqg.y, t));
    const uint32_t a3 = w_odd4(w2(vp8.y, t), w2(vq8.y, t));
    mma_s8(hi[0], a0, a1, a2, a3, F.b[ks][0][0], F.b[ks][0][1]);
    mma_s8(hi[1], a0, a1, a2, a3, F.b[ks][1][0], F.b[ks][1][1]);
    const uint32_t b0 = w_nib(vng.x, vng.y, t), b1 = w_nib(vn8.x, vn8.y, t);
    const uint32_t b2 = w_nib(vng.z, vng.w, t), b3 = w_nib(vn8.z, vn8.w, t);
    mma_s8(lo[0], b0, b1, b2, b3, F.b[ks][0][0], F.b[ks][0][1]);
    mma_s8(lo[1], b0, b1, b2, b3, F.b[ks][1][0], F.b[ks][1][1]);
  }
  long long dh[2], dl[2];
  combine_digits(hi, t, dh);
  combine_digits(lo, t, dl);
  const int row = (t & 1) ? r8 : rg;
  if (row < nloc) {
    const uint32_t u = (uint32_t)s_cand[row];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      // 2*code8 - 255 = 16*(2*c4 - 15) + (2*r4 - 15)
      const long long dsum = 16LL * dh[k] + dl[k];
      const uint32_t s = ord16(bf16_score(exact_to_float(dsum, k ? scB : scA)));
      w.k2[((size_t)cell * G + (k ? hB : hA)) * CAND_MAX + lo_rank + row] = (s << 16) | (0xffffu - u);
    }
  }
}

// Exact top-100 of one (cell, head) in rank order.
__global__ void __launch_bounds__(1024) k_s2_select(Work w) {
  const int h = blockIdx.x, cell = blockIdx.y, tid = threadIdx.x;
  __shared__ uint32_t s_key[CAND_MAX];
  __shared__ uint32_t s_win[TOPK];
  __shared__ int s_n;
  __shared__ SelectScratch sc;
  const int n = w.counts[cell * NCOUNT + C_CAND];
  const int nu = w.counts[cell * NCOUNT + C_U15];
  const int K = min(TOPK, n);
  if (tid < n) s_key[tid] = w.k2[((size_t)cell * G + h) * CAND_MAX + tid];
  if (tid == 0) s_n = 0;
  __syncthreads();
  const uint32_t th = select_kth(s_key, n, K, sc);
  if (tid < n && s_key[tid] >= th) {
    const int slot = atomicAdd(&s_n, 1);
    if (slot < TOPK) s_win[slot] = s_key[tid];
  }
  __syncthreads();
  const int m = min(s_n, TOPK);
  int32_t *fpos = w.final_pos + ((size_t)cell * G + h) * TOPK;
  int32_t *fids = w.final_ids + ((size_t)cell * G + h) * TOPK;
  uint32_t *fkeys = w.final_keys + ((size_t)cell * G + h) * TOPK;
  if (tid < m) {
    const uint32_t key = s_win[tid];
    int rank = 0;
    for (int j = 0; j < m; ++j) rank += s_win[j] > key;
    const int u = (int)(0xffffu - (key & 0xffffu));
    const bool live = u < nu;
    fpos[rank] = live ? u : -1;
    fids[rank] = live ? w.u15tok[(size_t)cell * U15_MAX + u] : 0;
    fkeys[rank] = live ? key : 0u;
  } else if (tid < TOPK) {
    // fewer than 100 candidates: a failed step that the status word reports;
    // keep the attention gather in bounds
    fpos[tid] = -1;
    fids[tid] = 0;
    fkeys[tid] = 0u;
  }
}

// -------------------------------------------------------------- attention

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

// Clears this cell's per-step bitmaps and histograms for the next step.
__device__ void clear_step_state(const Work &w, int cell) {
  for (int i = threadIdx.x; i < (w.nc >> 5); i += blockDim.x) w.selbits[(size_t)cell * (w.nc >> 5) + i] = 0;
  for (int i = threadIdx.x; i < (w.cap >> 5); i += blockDim.x) w.u15bits[(size_t)cell * (w.cap >> 5) + i] = 0;
  for (int i = threadIdx.x; i < (U15_MAX >> 5); i += blockDim.x)
    w.candbits[(size_t)cell * (U15_MAX >> 5) + i] = 0;
}

constexpr int ATTN_ITEMS = 4;  // work items per warp per pass

// Partition `split` of one cell.  Work items are the shared dense keys (sink,
// then local; one FP8 record scored against all four query heads) followed
// by each head's top-100 (rank order).  Warp w of the CTA takes items
// split*8 + w + j*ATTN_SPLIT*8 and keeps one online softmax per head (log2
// domain); the CTA writes one (m, l, o) partial per head and the last CTA of
// the cell combines them.
__global__ void __launch_bounds__(256) k_attn(Work w) {
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
    m[h] = -INFINITY; l[h] = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) o[h][j] = 0.0f;
  }
  const int step = ATTN_SPLIT * 8;
  for (int k0 = split * 8 + warp; k0 < nitems; k0 += step * ATTN_ITEMS) {
    int tok[ATTN_ITEMS], head[ATTN_ITEMS];
#pragma unroll
    for (int j = 0; j < ATTN_ITEMS; ++j) {
      const int it = k0 + j * step;
      head[j] = -1;  // -1: dense key for all heads
      if (it >= nitems) { tok[j] = -1; continue; }
      if (it < sink) { tok[j] = it; continue; }
      if (it < dense) { tok[j] = T - local + (it - sink); continue; }
      const int r = it - dense;
      head[j] = r / TOPK;
      tok[j] = w.final_ids[((size_t)cell * G + head[j]) * TOPK + r % TOPK];
    }
    uint2 kb[ATTN_ITEMS], vb[ATTN_ITEMS];
#pragma unroll
    for (int j = 0; j < ATTN_ITEMS; ++j) {
      const uint8_t *rec = c.kv8 + (size_t)(tok[j] < 0 ? 0 : tok[j]) * REC;
      kb[j] = *reinterpret_cast<const uint2 *>(rec + 8 * lane);
      vb[j] = *reinterpret_cast<const uint2 *>(rec + 256 + 8 * lane);
    }
#pragma unroll
    for (int j = 0; j < ATTN_ITEMS; ++j) {
      if (tok[j] < 0) continue;
      float kf[8], vf[8];
      fp8x8(kb[j], kf);
      fp8x8(vb[j], vf);
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
        if (head[j] >= 0 && head[j] != h) continue;
        const float mn = fmaxf(m[h], dot[h]);
        const float scale = exp2f(m[h] - mn);
        const float p = exp2f(dot[h] - mn);
        l[h] = l[h] * scale + p;
#pragma unroll
        for (int e = 0; e < 8; ++e) o[h][e] = fmaf(o[h][e], scale, p * vf[e]);
        m[h] = mn;
      }
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
  // the last partition of this cell combines (no waiting: whoever arrives last)
  __threadfence();
  if (tid == 0) s_last = atomicAdd(&w.arrive[cell], 1u) == ATTN_SPLIT - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  {
    // thread (head, quarter): output dims 4*q .. 4*q+3 of one head; all
    // partials of that head are read at once (independent loads)
    const int h = tid >> 6, q4 = tid & 63;
    const float *ph = part + (size_t)h * ATTN_SPLIT * PART;
    float ms[ATTN_SPLIT], ls[ATTN_SPLIT];
    float4 os[ATTN_SPLIT];
#pragma unroll
    for (int sp = 0; sp < ATTN_SPLIT; ++sp) {
      ms[sp] = __ldcg(ph + sp * PART);
      ls[sp] = __ldcg(ph + sp * PART + 1);
      os[sp] = __ldcg(reinterpret_cast<const float4 *>(ph + sp * PART + 4) + q4);
    }
    float M = -INFINITY;
#pragma unroll
    for (int sp = 0; sp < ATTN_SPLIT; ++sp) M = fmaxf(M, ms[sp]);
    float L = 0.0f;
    float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int sp = 0; sp < ATTN_SPLIT; ++sp) {
      if (ms[sp] == -INFINITY) continue;
      const float e = exp2f(ms[sp] - M);
      L += ls[sp] * e;
      O.x += os[sp].x * e; O.y += os[sp].y * e; O.z += os[sp].z * e; O.w += os[sp].w * e;
    }
    uint16_t *dst = w.out + ((size_t)slot * 16 + g * 4 + h) * D + 4 * q4;
    dst[0] = bf16_rne(O.x / L);
    dst[1] = bf16_rne(O.y / L);
    dst[2] = bf16_rne(O.z / L);
    dst[3] = bf16_rne(O.w / L);
  }
  if (tid == 0) w.arrive[cell] = 0;
  clear_step_state(w, cell);
}

// ---------------------------------------------------------- upload-time

// Per-(head, dim) max |k| over all tokens (atomicMax on the FP32 bit pattern,
// which orders non-negative floats).
__global__ void __launch_bounds__(256) k_absmax(const uint16_t *k, int T, uint32_t *smax) {
  const int g = blockIdx.y, d = threadIdx.x;
  const int t0 = blockIdx.x * 256, t1 = min(T, t0 + 256);
  float mx = 0.0f;
  for (int t = t0; t < t1; ++t) mx = fmaxf(mx, fabsf(bf16f(k[((size_t)g * T + t) * D + d])));
  atomicMax(&smax[g * D + d], __float_as_uint(mx));
}

// Key code planes of every token (encode_key_quad), the scales being the
// per-dimension maxima k_absmax gathered.
__global__ void __launch_bounds__(256) k_planes(const uint16_t *k, int T, const uint32_t *smax,
                                                float *scale_out, uint8_t *p2, uint8_t *r2,
                                                uint8_t *r4, int g) {
  const int tid = threadIdx.x, tok = blockIdx.x * 4 + (tid >> 6), q = tid & 63;
  __shared__ float s_scale[D];
  s_scale[tid] = fmaxf(__uint_as_float(smax[g * D + tid]), 1e-9f);
  __syncthreads();
  if (blockIdx.x == 0) scale_out[tid] = s_scale[tid];
  if (tok >= T) return;
  encode_key_quad(k + ((size_t)g * T + tok) * D, s_scale, q, p2 + (size_t)tok * 64, r2 + (size_t)tok * 64,
                  r4 + (size_t)tok * 128);
}

__global__ void __launch_bounds__(256) k_fp8(const uint16_t *k, const uint16_t *v, int T, uint8_t *kv8, int g) {
  const size_t i = (size_t)blockIdx.x * 256 + threadIdx.x;  // element of [T][256]
  if (i >= (size_t)T * D) return;
  const size_t tok = i / D, d = i % D;
  const size_t src = (size_t)g * T * D + i;
  kv8[tok * REC + d] = to_e4m3(bf16f(k[src]));
  kv8[tok * REC + 256 + d] = to_e4m3(bf16f(v[src]));
}

// ------------------------------------------------------------- launchers

const char *const kFunnelKernels[] = {
    "k_qprep", "k_coarse", "k_coarse_thresh", "k_surv_count", "k_fine", "k_select(fine)",
    "k_pool_count", "k_pool_s15", "k_select(s15)", "k_s16", "k_select(s16)", "k_s2_score",
    "k_s2_select", "k_attn"};
constexpr int kNumKernels = sizeof(kFunnelKernels) / sizeof(kFunnelKernels[0]);

// Enqueue one decode step.  With `ev` non-null, event ev[i] is recorded
// before kernel i and ev[kNumKernels] after the last, for per-kernel timing.
cudaError_t launch_funnel(const Work &w, cudaStream_t st, cudaEvent_t *ev) {
  const int cells = w.n_cells;
  int k = 0;
  auto mark = [&]() { if (ev) cudaEventRecord(ev[k++], st); };
  const size_t smem = SELECT_SMEM_KEYS * sizeof(uint32_t);
  const int coarse_ctas = min(64, (w.nc / 16 + 31) / 32);
  mark();
  k_qprep<<<dim3(3 * G, cells), 256, 0, st>>>(w); mark();
  k_coarse<<<dim3(coarse_ctas, cells), 256, 0, st>>>(w); mark();
  k_coarse_thresh<<<dim3(G, cells), 1024, 0, st>>>(w); mark();
  k_surv_count<<<dim3(w.chunks_nc, cells), 256, 0, st>>>(w); mark();
  k_fine<<<dim3(w.chunks_nc, cells), 256, 0, st>>>(w); mark();
  k_select<<<dim3(G, cells), 1024, smem, st>>>(w, 0); mark();
  k_pool_count<<<dim3(w.chunks_surv, cells), SCHUNK, 0, st>>>(w); mark();
  k_pool_s15<<<dim3(w.chunks_surv, cells), SCHUNK, 0, st>>>(w); mark();
  k_select<<<dim3(G, cells), 1024, smem, st>>>(w, 1); mark();
  k_s16<<<dim3((w.cap + S16_CHUNK - 1) / S16_CHUNK, cells), 256, 0, st>>>(w); mark();
  k_select<<<dim3(G, cells), 1024, smem, st>>>(w, 2); mark();
  k_s2_score<<<dim3(CAND_MAX / S2_ROWS, cells), 256, 0, st>>>(w); mark();
  k_s2_select<<<dim3(G, cells), 1024, 0, st>>>(w); mark();
  k_attn<<<dim3(ATTN_SPLIT, cells), 256, 0, st>>>(w); mark();
  return cudaGetLastError();
}

const char *funnel_kernel_name(int i) { return (i >= 0 && i < kNumKernels) ? kFunnelKernels[i] : ""; }

int funnel_kernel_count() { return kNumKernels; }

cudaError_t prepare_funnel_attributes() {
  return cudaFuncSetAttribute(k_select, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              SELECT_SMEM_KEYS * (int)sizeof(uint32_t));
}

cudaError_t launch_key_codec(const uint16_t *k, const uint16_t *v, int T, uint32_t *smax, float *const scale[G],
                             uint8_t *const p2[G], uint8_t *const r2[G], uint8_t *const r4[G],
                             uint8_t *const kv8[G], cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(smax, 0, G * D * sizeof(uint32_t), st);
  if (e != cudaSuccess) return e;
  k_absmax<<<dim3((T + 255) / 256, G), 256, 0, st>>>(k, T, smax);
  for (int g = 0; g < G; ++g) {
    k_planes<<<(T + 3) / 4, 256, 0, st>>>(k, T, smax, scale[g], p2[g], r2[g], r4[g], g);
    k_fp8<<<(unsigned)(((size_t)T * D + 255) / 256), 256, 0, st>>>(k, v, T, kv8[g], g);
  }
  return cudaGetLastError();
}

}  // namespace skv
