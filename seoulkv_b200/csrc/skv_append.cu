// skv_append.cu -- cache-append kernels.
//
// An append of m tokens to every cell of the engine is two stream-ordered
// launches that read the current context from device memory, so the same
// launches replayed from a graph append at successive positions:
//
//   k_assign         spill-2 assignment of the new keys, and (partition 0)
//                    their key planes (the build's scales) and FP8 records
//                    at positions T .. T+m-1.  The score of key k against
//                    stored centroid c is
//                        S(k, c) = fl64( X(k, c) * fs_c ),
//                        X(k, c) = sum_d x_d * (2 code_cd - 15)   (exact)
//                    where x is the key on the decode's operand grid (with E
//                    its top exponent, elements below 2^(E-22) flushed, the
//                    rest integers on the 2^(E-29) grid; a non-finite element
//                    counts as 0 and is reported) and fs_c the FP16 group
//                    fine scale of c's 32-centroid group.  This is the Fine
//                    stage's centroid score with the key as the query,
//                    computed the way the decode computes it (int8 digit
//                    fragments on the tensor cores, int64 recombination) and
//                    rounded once.  Each CTA keeps a top-2 per key over a
//                    partition of the centroids; the last CTA of each cell
//                    then takes the top-2 over the partitions (ties to the
//                    lower centroid id): the new tokens' two lists; and
//                    sorts the 2m postings of the tokens leaving the local
//                    window, T-local .. T-local+m-1, by list then token,
//                    each with its mate (the other list) and its insertion
//                    point
//   k_post_rebuild   the next CSR set: every old list followed by its new
//                    postings, so each list stays in ascending token order
//                    exactly as a CSR built over all tokens would be; its
//                    last CTA to finish flips the live CSR sets and
//                    advances the context
//
// The score puts a token where the funnel looks for its nearest neighbours.
#include <cuda_runtime.h>

#include <cfloat>

#include "skv_append.cuh"
#include "skv_codec.cuh"

namespace skv {

namespace {

struct Top2 {
  double s1, s2;
  int i1, i2;
};

__device__ __forceinline__ bool better(double s, int i, double bs, int bi) { return s > bs || (s == bs && i < bi); }

__device__ __forceinline__ void top2_insert(Top2 &t, double s, int i) {
  if (better(s, i, t.s1, t.i1)) {
    t.s2 = t.s1;
    t.i2 = t.i1;
    t.s1 = s;
    t.i1 = i;
  } else if (better(s, i, t.s2, t.i2)) {
    t.s2 = s;
    t.i2 = i;
  }
}

// Merge of two top-2 lists with distinct ids.
__device__ __forceinline__ Top2 top2_merge(const Top2 &a, const Top2 &b) {
  Top2 r;
  if (better(b.s1, b.i1, a.s1, a.i1)) {
    r.s1 = b.s1;
    r.i1 = b.i1;
    const bool a1 = better(a.s1, a.i1, b.s2, b.i2);
    r.s2 = a1 ? a.s1 : b.s2;
    r.i2 = a1 ? a.i1 : b.i2;
  } else {
    r.s1 = a.s1;
    r.i1 = a.i1;
    const bool b1 = better(b.s1, b.i1, a.s2, a.i2);
    r.s2 = b1 ? b.s1 : a.s2;
    r.i2 = b1 ? b.i1 : a.i2;
  }
  return r;
}

__device__ __forceinline__ Top2 top2_empty() { return Top2{-DBL_MAX, -DBL_MAX, INT_MAX, INT_MAX}; }

__device__ __forceinline__ Top2 shfl_top2(const Top2 &t, int o) {
  Top2 u;
  u.s1 = __shfl_xor_sync(0xffffffffu, t.s1, o);
  u.s2 = __shfl_xor_sync(0xffffffffu, t.s2, o);
  u.i1 = __shfl_xor_sync(0xffffffffu, t.i1, o);
  u.i2 = __shfl_xor_sync(0xffffffffu, t.i2, o);
  return u;
}

__device__ __forceinline__ Top2 warp_top2(Top2 t) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t = top2_merge(t, shfl_top2(t, o));
  return t;
}

__device__ __forceinline__ bool append_fits(const int32_t *tlen, int m, int tmax) { return *tlen + m <= tmax; }

__device__ __forceinline__ int lower_bound_i32(const int32_t *a, int n, int x) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (a[mid] < x) lo = mid + 1; else hi = mid;
  }
  return lo;
}

__device__ __forceinline__ void prefetch_l2(const void *p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

__device__ __forceinline__ void load_plane_row(const uint8_t *base, int row, uint4 (&r)[4]) {
  const uint4 *p = reinterpret_cast<const uint4 *>(base + (size_t)row * 64);
#pragma unroll
  for (int k = 0; k < 4; ++k) r[k] = p[k];
}

// ------------------------------------------------------------------ assign

// Top-2 of key j over its partitions (a warp; split <= ASSIGN_SPLIT).
__device__ __forceinline__ Top2 reduce_parts(const AssignArgs &a, int cell, int j, int lane) {
  Top2 t = top2_empty();
  for (int s = lane; s < a.split; s += 32) {
    const size_t o = (((size_t)cell * APPEND_MAX + j) * ASSIGN_SPLIT + s) * 2;
    t = top2_merge(t, Top2{a.part_s[o], a.part_s[o + 1], a.part_i[o], a.part_i[o + 1]});
  }
  return warp_top2(t);
}

// One cell's lists step of an append (a whole CTA): the new keys' lists
// (top-2 over the partitions, ties to the lower centroid id), then the 2m
// postings of the tokens leaving the local window sorted by (list, token),
// each with its mate and its insertion point (the old CSR position where its
// list ends).
__device__ void cell_lists(const AppendArgs &a, const AssignArgs &s, int cell) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int T = *a.tlen;
  int32_t *lab = a.acells[cell].labels;
  for (int j = warp; j < a.m; j += nwarps) {
    const Top2 t = reduce_parts(s, cell, j, lane);
    if (lane == 0) {
      lab[2 * (size_t)(T + j)] = t.i1;
      lab[2 * (size_t)(T + j) + 1] = t.i2;
    }
  }
  __threadfence_block();
  __syncthreads();
  const int r1 = T - a.local;  // first token leaving the local window
  const int n = 2 * a.m;
  int np = 1;
  while (np < n) np <<= 1;
  __shared__ unsigned long long key[2 * APPEND_MAX];
  for (int i = tid; i < np; i += blockDim.x) {
    const int tk = r1 + (i >> 1);
    key[i] = i < n ? ((unsigned long long)(uint32_t)lab[2 * (size_t)tk + (i & 1)] << 32) | (uint32_t)tk : ~0ull;
  }
  __syncthreads();
  for (int k = 2; k <= np; k <<= 1)
    for (int jj = k >> 1; jj > 0; jj >>= 1) {
      for (int i = tid; i < np; i += blockDim.x) {
        const int ixj = i ^ jj;
        if (ixj > i) {
          const unsigned long long u = key[i], v = key[ixj];
          if ((u > v) == ((i & k) == 0)) {
            key[i] = v;
            key[ixj] = u;
          }
        }
      }
      __syncthreads();
    }
  const AppendCellDev &A = a.acells[cell];
  const int32_t *off = A.offsets[A.cur];
  const size_t o = (size_t)cell * 2 * APPEND_MAX;
  for (int i = tid; i < n; i += blockDim.x) {
    const int c = (int)(key[i] >> 32), tk = (int)(uint32_t)key[i];
    const int l0 = lab[2 * (size_t)tk], l1 = lab[2 * (size_t)tk + 1];
    a.newlist[o + i] = c;
    a.newtok[o + i] = tk;
    a.newmate[o + i] = l0 == c ? l1 : l0;
    a.newins[o + i] = off[c + 1];
  }
}

// One CTA per (centroid partition, cell, group of 4 keys).  The keys are the
// B operand of the decode's exact int8 dot (in the four query heads' place);
// every warp scores 16-centroid tiles with the 4-bit codes c (0..15) as the A
// operand, X = 2 sum_d c_d x_d - 15 sum_d x_d, and keeps a top-2 per key.
// With `codec` (an append), partition 0 also writes the group's key planes
// and FP8 records, and the last CTA of each cell to finish runs the cell's
// lists step.
__global__ void __launch_bounds__(256) k_assign(AssignArgs a, AppendArgs app, int codec) {
  const int split = blockIdx.x, y = blockIdx.y, cell = a.cell0 + y, j0 = blockIdx.z * 4;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
  if (a.guard > 0 && !append_fits(a.tlen, a.guard, a.tmax)) return;
  const CellDev &c = a.cells[cell];
  const uint8_t *const upper = c.upper, *const lower = c.lower;  // loaded before the prologue
  const float *const fine_scale = c.fine_scale;
  __shared__ uint32_t s_frag[FRAG_ROW];
  __shared__ int s_e[4][8];
  __shared__ long long s_sx[4][8];
  __shared__ Top2 s_t[8][4];
  __shared__ float s_scale[D];
  __shared__ bool s_last;
  float x[4];
  int ex[4];  // ilogb of each element (INT_MIN for 0)
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    float v = 0.0f;
    if (j0 + r < a.m) {
      v = bf16f(a.k[y * a.k_cell_stride + (long long)(j0 + r) * D + tid]);
      if (!isfinite(v)) {
        v = 0.0f;
        if (a.status && split == 0) atomicOr(a.status, APPEND_NONFINITE);
      }
    }
    x[r] = v;
    ex[r] = v != 0.0f ? ilogbf(v) : INT_MIN;
    const int e = __reduce_max_sync(0xffffffffu, ex[r]);
    if (lane == 0) s_e[r][warp] = e;
  }
  if (codec && split == 0) s_scale[tid] = app.acells[cell].key_scale[tid];
  __syncthreads();
  // digit fragments: the decode's operand encoding (elements below 2^(E-22)
  // flushed, the rest integers X on the 2^(E-29) grid, |X| < 2^30, as four
  // signed base-256 digits); key r of the group in query head r's columns;
  // and each key's sum of X (for the -15 of the weights)
  uint8_t *fb = reinterpret_cast<uint8_t *>(s_frag);
  const int ks = tid >> 5, reg = (tid >> 4) & 1, byte = (tid >> 2) & 3, tq = tid & 3;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    int E = INT_MIN;
#pragma unroll
    for (int k = 0; k < 8; ++k) E = max(E, s_e[r][k]);
    int X = 0;
    // kept: ilogb >= E - 22; x * 2^(29-E) is then an integer (8 significant bits), exact in FP64
    if (E != INT_MIN && ex[r] >= E - 22) X = __double2int_rn((double)x[r] * pow2d(29 - E));
    long long sx = X;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sx += __shfl_xor_sync(0xffffffffu, sx, o);
    if (lane == 0) s_sx[r][warp] = sx;
    int dg[4];
    dg[0] = (int)(int8_t)(X & 0xff);
    int rest = (X - dg[0]) >> 8;
    dg[1] = (int)(int8_t)(rest & 0xff);
    rest = (rest - dg[1]) >> 8;
    dg[2] = (int)(int8_t)(rest & 0xff);
    dg[3] = (rest - dg[2]) >> 8;
    const int nt = r >> 1;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int lane_b = 4 * (4 * (r & 1) + j) + tq;
      fb[(((ks * 2 + nt) * 32 + lane_b) * 2 + reg) * 4 + byte] = (uint8_t)(int8_t)dg[j];
    }
  }
  if (codec && split == 0) {  // the group's planes and records
    const AppendCellDev &A = app.acells[cell];
    const int T = *app.tlen;
    for (int r = 0; r < 4 && j0 + r < a.m; ++r) {
      const size_t tok = (size_t)T + j0 + r;
      const uint16_t *krow = app.k + ((size_t)cell * app.m + j0 + r) * D;
      const uint16_t *vrow = app.v + ((size_t)cell * app.m + j0 + r) * D;
      A.kv8[tok * REC + tid] = to_e4m3(bf16f(krow[tid]));
      A.kv8[tok * REC + 256 + tid] = to_e4m3(bf16f(vrow[tid]));
      if (tid < 64)
        encode_key_quad(krow, s_scale, tid, A.prefix2 + tok * 64, A.residual2 + tok * 64, A.residual4 + tok * 128);
    }
  }
  __syncthreads();
  BFrag F;
#pragma unroll
  for (int k = 0; k < 8; ++k)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      F.b[k][nt][0] = s_frag[((k * 2 + nt) * 32 + lane) * 2];
      F.b[k][nt][1] = s_frag[((k * 2 + nt) * 32 + lane) * 2 + 1];
    }
  long long sx15[2];  // 15 sum(X) of keys t/2 and 2 + t/2
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    long long v = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) v += s_sx[2 * k + (t >> 1)][w];
    sx15[k] = 15 * v;
  }
  Top2 best[2] = {top2_empty(), top2_empty()};  // keys t/2 and 2 + t/2
  const int tiles = a.nc >> 4;
  for (int tile = split * 8 + warp; tile < tiles; tile += a.split * 8) {
    const int rg = tile * 16 + g;
    const int nxt = tile + a.split * 8;
    if (nxt < tiles && t < 2) {  // the next tile's rows into L2 while this one computes
      const int rn = nxt * 16 + g + 8 * t;
      prefetch_l2(upper + (size_t)rn * 64);
      prefetch_l2(lower + (size_t)rn * 64);
    }
    uint4 ug[4], lg[4], u8[4], l8[4];
    load_plane_row(upper, rg, ug);
    load_plane_row(lower, rg, lg);
    load_plane_row(upper, rg + 8, u8);
    load_plane_row(lower, rg + 8, l8);
    int acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
#pragma unroll
    for (int k = 0; k < 8; ++k) {  // A bytes: the codes 4u + l of 4 dimensions
      const uint32_t a0 = (w2(word_of(ug, 2 * k), t) << 2) | w2(word_of(lg, 2 * k), t);
      const uint32_t a1 = (w2(word_of(u8, 2 * k), t) << 2) | w2(word_of(l8, 2 * k), t);
      const uint32_t a2 = (w2(word_of(ug, 2 * k + 1), t) << 2) | w2(word_of(lg, 2 * k + 1), t);
      const uint32_t a3 = (w2(word_of(u8, 2 * k + 1), t) << 2) | w2(word_of(l8, 2 * k + 1), t);
      mma_s8(acc[0], a0, a1, a2, a3, F.b[k][0][0], F.b[k][0][1]);
      mma_s8(acc[1], a0, a1, a2, a3, F.b[k][1][0], F.b[k][1][1]);
    }
    long long dsum[2];
    combine_digits(acc, t, dsum);
    const int row = rg + ((t & 1) << 3);
    const double fs = (double)fine_scale[row >> 5];
    // |X| < 2^42: exact as a double, then one rounding
    top2_insert(best[0], (double)(2 * dsum[0] - sx15[0]) * fs, row);
    top2_insert(best[1], (double)(2 * dsum[1] - sx15[1]) * fs, row);
  }
  // lanes with equal t >> 1 hold the same two keys
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    best[k] = top2_merge(best[k], shfl_top2(best[k], 1));
    best[k] = top2_merge(best[k], shfl_top2(best[k], 4));
    best[k] = top2_merge(best[k], shfl_top2(best[k], 8));
    best[k] = top2_merge(best[k], shfl_top2(best[k], 16));
  }
  if (lane == 0 || lane == 2) {
    s_t[warp][lane >> 1] = best[0];
    s_t[warp][2 + (lane >> 1)] = best[1];
  }
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const Top2 v = warp_top2(lane < 8 ? s_t[lane][r] : top2_empty());
      if (lane == 0 && j0 + r < a.m) {
        const size_t o = (((size_t)cell * APPEND_MAX + (j0 + r)) * ASSIGN_SPLIT + split) * 2;
        a.part_s[o] = v.s1;
        a.part_s[o + 1] = v.s2;
        a.part_i[o] = v.i1;
        a.part_i[o + 1] = v.i2;
      }
    }
  }
  if (!codec) return;
  // the cell's last CTA runs its lists step (partials of the others are
  // visible after their fence and counter increment)
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    s_last = atomicAdd(&app.assign_done[cell], 1u) == gridDim.x * gridDim.z - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  cell_lists(app, a, cell);
  if (tid == 0) app.assign_done[cell] = 0;
}

__global__ void __launch_bounds__(1024) k_assign_reduce(AssignArgs a) {
  const int cell = a.cell0 + blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int base = (a.use_tlen ? *a.tlen : 0) + a.lab_base;
  int32_t *lab = a.acells[cell].labels;
  for (int j = warp; j < a.m; j += 32) {
    const Top2 t = reduce_parts(a, cell, j, lane);
    if (lane == 0) {
      lab[2 * (size_t)(base + j)] = t.i1;
      lab[2 * (size_t)(base + j) + 1] = t.i2;
    }
  }
}

// ------------------------------------------------------------------ append

// The next CSR set, one thread per element: old posting p moves up by the
// new postings inserted at or before it (#{j : ins_j <= p}); new posting j
// lands at ins_j + j; offset c grows by the new postings of lists below c.
// The last CTA to finish (over all cells) commits: the live CSR sets flip
// and the context advances.
__global__ void __launch_bounds__(256) k_post_rebuild(AppendArgs a) {
  const int cell = blockIdx.y, tid = threadIdx.x;
  const int T = *a.tlen;
  if (T + a.m > a.tmax) {
    if (blockIdx.x == 0 && cell == 0 && tid == 0) atomicOr(a.status, APPEND_FULL);
    return;
  }
  const int n = 2 * a.m;
  __shared__ int32_t s_nl[2 * APPEND_MAX], s_ins[2 * APPEND_MAX];
  __shared__ bool s_last;
  const size_t o = (size_t)cell * 2 * APPEND_MAX;
  for (int i = tid; i < n; i += blockDim.x) {
    s_nl[i] = a.newlist[o + i];
    s_ins[i] = a.newins[o + i];
  }
  __syncthreads();
  {
    const AppendCellDev &A = a.acells[cell];
    const int cur = A.cur, n_old = A.n_postings;
    const int32_t *__restrict__ off = A.offsets[cur];
    const int32_t *__restrict__ val = A.values[cur];
    const int32_t *__restrict__ mat = A.mates[cur];
    int32_t *__restrict__ off2 = A.offsets[cur ^ 1];
    int32_t *__restrict__ val2 = A.values[cur ^ 1];
    int32_t *__restrict__ mat2 = A.mates[cur ^ 1];
    const int total = n_old + n + a.nc + 1;
    constexpr int U = REBUILD_PER_THREAD;
    for (int base = blockIdx.x * blockDim.x * U + tid; base < total; base += gridDim.x * blockDim.x * U) {
      int v[U], mt[U];  // this thread's old postings, all loaded before any store
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = base + u * blockDim.x;
        if (i < n_old) {
          v[u] = val[i];
          mt[u] = mat[i];
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = base + u * blockDim.x;
        if (i < n_old) {
          const int sft = lower_bound_i32(s_ins, n, i + 1);  // insertion points <= i
          val2[i + sft] = v[u];
          mat2[i + sft] = mt[u];
        } else if (i < n_old + n) {
          const int j = i - n_old;
          val2[s_ins[j] + j] = a.newtok[o + j];
          mat2[s_ins[j] + j] = a.newmate[o + j];
        } else if (i < total) {
          const int c = i - n_old - n;
          off2[c] = off[c] + lower_bound_i32(s_nl, n, c);
        }
      }
    }
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    s_last = atomicAdd(a.done, 1u) == gridDim.x * gridDim.y - 1;
  }
  __syncthreads();
  if (!s_last) return;
  for (int c = tid; c < a.n_cells; c += blockDim.x) {
    AppendCellDev &A = a.acells[c];
    const int nxt = A.cur ^ 1;
    A.cur = nxt;
    A.n_postings += n;
    CellDev &cd = a.cells[c];
    cd.offsets = A.offsets[nxt];
    cd.values = A.values[nxt];
    cd.mates = A.mates[nxt];
  }
  __syncthreads();
  if (tid == 0) {
    *a.done = 0;
    *a.tlen = T + a.m;
  }
}

}  // namespace

cudaError_t launch_assign(const AssignArgs &a, cudaStream_t st) {
  if (a.m < 1 || a.m > APPEND_MAX || a.split < 1 || a.split > ASSIGN_SPLIT) return cudaErrorInvalidValue;
  k_assign<<<dim3(a.split, a.n_cells, (a.m + 3) / 4), 256, 0, st>>>(a, AppendArgs{}, 0);
  k_assign_reduce<<<a.n_cells, 1024, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_append(const AppendArgs &a, const AssignArgs &assign, cudaStream_t st) {
  if (a.m < 1 || a.m > APPEND_MAX || assign.split < 1 || assign.split > ASSIGN_SPLIT) return cudaErrorInvalidValue;
  k_assign<<<dim3(assign.split, a.n_cells, (a.m + 3) / 4), 256, 0, st>>>(assign, a, 1);
  k_post_rebuild<<<dim3(a.rebuild_ctas, a.n_cells), 256, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace skv
