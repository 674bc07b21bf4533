// skv_append.cu -- cache-append kernels.
//
// An append of m tokens to every cell of the engine is six stream-ordered
// launches that read the current context from device memory, so the same
// launches replayed from a graph append at successive positions:
//
//   k_append_codec   key planes (the build's scales) and FP8 records of the
//                    new tokens at positions T .. T+m-1
//   k_assign<TG>     spill-2 assignment of the new keys: score of key k
//                    against stored centroid c is
//                        S(k, c) = fl64( fl64sum_{d=0..255}( k_d * (2 code_cd - 15) ) * fs_c )
//                    with the sum taken in dimension order in FP64 (every
//                    product is exact: an 8-bit significand times a 5-bit
//                    integer) and fs_c the FP16 group fine scale of c's
//                    32-centroid group (a non-finite key element counts as
//                    0 and is reported); each block keeps a top-2 over a
//                    share of the centroids
//   k_assign_reduce  top-2 over the shares (ties to the lower centroid id):
//                    the token's two lists
//   k_post_prepare   the tokens leaving the local window, T-local ..
//                    T-local+m-1, as 2m (list, token) postings sorted by
//                    list then token, each with its mate (the other list)
//   k_post_rebuild   the next CSR set: every old list followed by its new
//                    postings, so each list stays in ascending token order
//                    exactly as a CSR built over all tokens would be
//   k_append_commit  the live CSR set flips and the context advances
//
// The score is the Fine stage's centroid score of the key used as a query
// (the decode path scores centroids with the same 4-bit codes and scales),
// so a token is posted where the funnel looks for its nearest neighbours.
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

__device__ __forceinline__ Top2 warp_top2(Top2 t) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Top2 u;
    u.s1 = __shfl_xor_sync(0xffffffffu, t.s1, o);
    u.s2 = __shfl_xor_sync(0xffffffffu, t.s2, o);
    u.i1 = __shfl_xor_sync(0xffffffffu, t.i1, o);
    u.i2 = __shfl_xor_sync(0xffffffffu, t.i2, o);
    t = top2_merge(t, u);
  }
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

// 2 code - 15 as an FP64 value without a conversion instruction:
// 2^52 + 2 code is built from its bits and 2^52 + 15 subtracted (exact).
__device__ __forceinline__ double code_weight(uint32_t code) {
  return __hiloint2double(0x43300000, (int)(code << 1)) - 4503599627370511.0;
}

// ------------------------------------------------------------------ assign

template <int TG>
__global__ void __launch_bounds__(256) k_assign(AssignArgs a, int j_begin) {
  const int split = blockIdx.x, y = blockIdx.y, cell = a.cell0 + y, tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  if (a.guard > 0 && !append_fits(a.tlen, a.guard, a.tmax)) return;
  const int j0 = j_begin + blockIdx.z * TG;
  __shared__ double s_k[TG][D];
  __shared__ Top2 s_t[8][TG];
#pragma unroll
  for (int t = 0; t < TG; ++t) {
    float x = bf16f(a.k[y * a.k_cell_stride + (long long)(j0 + t) * D + tid]);
    if (!isfinite(x)) {
      x = 0.0f;
      if (a.status && split == 0) atomicOr(a.status, APPEND_NONFINITE);
    }
    s_k[t][tid] = (double)x;
  }
  __syncthreads();
  const CellDev &c = a.cells[cell];
  Top2 best[TG];
#pragma unroll
  for (int t = 0; t < TG; ++t) best[t] = top2_empty();
  for (int chunk = split; chunk * 256 < a.nc; chunk += a.split) {
    const int ci = chunk * 256 + tid;
    if (ci >= a.nc) continue;
    const uint4 *up = reinterpret_cast<const uint4 *>(c.upper + (size_t)ci * 64);
    const uint4 *lo = reinterpret_cast<const uint4 *>(c.lower + (size_t)ci * 64);
    double acc[TG];
#pragma unroll
    for (int t = 0; t < TG; ++t) acc[t] = 0.0;
#pragma unroll 1
    for (int qd = 0; qd < 4; ++qd) {  // 64 dimensions per 16-byte quarter of each plane
      const uint4 U = up[qd], L = lo[qd];
      const uint32_t uw[4] = {U.x, U.y, U.z, U.w}, lw[4] = {L.x, L.y, L.z, L.w};
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int d = qd * 64 + r * 16 + i;
          const uint32_t code = (((uw[r] >> (2 * i)) & 3u) << 2) | ((lw[r] >> (2 * i)) & 3u);
          const double wv = code_weight(code);
#pragma unroll
          for (int t = 0; t < TG; ++t) acc[t] = fma(s_k[t][d], wv, acc[t]);
        }
    }
    const double fs = (double)c.fine_scale[ci >> 5];
#pragma unroll
    for (int t = 0; t < TG; ++t) top2_insert(best[t], acc[t] * fs, ci);
  }
#pragma unroll
  for (int t = 0; t < TG; ++t) {
    const Top2 r = warp_top2(best[t]);
    if (lane == 0) s_t[warp][t] = r;
  }
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int t = 0; t < TG; ++t) {
      Top2 r = lane < 8 ? s_t[lane][t] : top2_empty();
      r = warp_top2(r);
      if (lane == 0) {
        const size_t o = (((size_t)cell * APPEND_MAX + (j0 + t)) * ASSIGN_SPLIT + split) * 2;
        a.part_s[o] = r.s1;
        a.part_s[o + 1] = r.s2;
        a.part_i[o] = r.i1;
        a.part_i[o + 1] = r.i2;
      }
    }
  }
}

__global__ void __launch_bounds__(1024) k_assign_reduce(AssignArgs a) {
  const int cell = a.cell0 + blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (a.guard > 0 && !append_fits(a.tlen, a.guard, a.tmax)) return;
  const int base = (a.use_tlen ? *a.tlen : 0) + a.lab_base;
  int32_t *lab = a.acells[cell].labels;
  for (int j = warp; j < a.m; j += 32) {
    Top2 t = top2_empty();
    if (lane < a.split) {
      const size_t o = (((size_t)cell * APPEND_MAX + j) * ASSIGN_SPLIT + lane) * 2;
      t = Top2{a.part_s[o], a.part_s[o + 1], a.part_i[o], a.part_i[o + 1]};
    }
    t = warp_top2(t);
    if (lane == 0) {
      lab[2 * (size_t)(base + j)] = t.i1;
      lab[2 * (size_t)(base + j) + 1] = t.i2;
    }
  }
}

// ------------------------------------------------------------------ append

__global__ void __launch_bounds__(256) k_append_codec(AppendArgs a) {
  const int j = blockIdx.x, cell = blockIdx.y, tid = threadIdx.x;
  if (!append_fits(a.tlen, a.m, a.tmax)) return;
  const size_t tok = (size_t)*a.tlen + j;
  const AppendCellDev &A = a.acells[cell];
  const uint16_t *krow = a.k + ((size_t)cell * a.m + j) * D;
  const uint16_t *vrow = a.v + ((size_t)cell * a.m + j) * D;
  __shared__ float s_scale[D];
  s_scale[tid] = A.key_scale[tid];
  __syncthreads();
  A.kv8[tok * REC + tid] = to_e4m3(bf16f(krow[tid]));
  A.kv8[tok * REC + 256 + tid] = to_e4m3(bf16f(vrow[tid]));
  if (tid < 64) encode_key_quad(krow, s_scale, tid, A.prefix2 + tok * 64, A.residual2 + tok * 64, A.residual4 + tok * 128);
}

__global__ void __launch_bounds__(1024) k_post_prepare(AppendArgs a) {
  const int cell = blockIdx.x, tid = threadIdx.x;
  if (!append_fits(a.tlen, a.m, a.tmax)) return;
  const int r1 = *a.tlen - a.local;  // first token leaving the local window
  const int n = 2 * a.m;
  int np = 1;
  while (np < n) np <<= 1;
  __shared__ unsigned long long key[2 * APPEND_MAX];
  const int32_t *lab = a.acells[cell].labels;
  for (int i = tid; i < np; i += blockDim.x) {
    const int t = r1 + (i >> 1);
    key[i] = i < n ? ((unsigned long long)(uint32_t)lab[2 * (size_t)t + (i & 1)] << 32) | (uint32_t)t : ~0ull;
  }
  __syncthreads();
  for (int k = 2; k <= np; k <<= 1)
    for (int jj = k >> 1; jj > 0; jj >>= 1) {
      for (int i = tid; i < np; i += blockDim.x) {
        const int ixj = i ^ jj;
        if (ixj > i) {
          const unsigned long long x = key[i], y = key[ixj];
          if ((x > y) == ((i & k) == 0)) {
            key[i] = y;
            key[ixj] = x;
          }
        }
      }
      __syncthreads();
    }
  const size_t o = (size_t)cell * 2 * APPEND_MAX;
  for (int i = tid; i < n; i += blockDim.x) {
    const int c = (int)(key[i] >> 32), t = (int)(uint32_t)key[i];
    const int l0 = lab[2 * (size_t)t], l1 = lab[2 * (size_t)t + 1];
    a.newlist[o + i] = c;
    a.newtok[o + i] = t;
    a.newmate[o + i] = l0 == c ? l1 : l0;
  }
}

__global__ void __launch_bounds__(256) k_post_rebuild(AppendArgs a) {
  const int cell = blockIdx.y, tid = threadIdx.x;
  if (!append_fits(a.tlen, a.m, a.tmax)) return;
  const int n = 2 * a.m;
  __shared__ int32_t nl[2 * APPEND_MAX];
  const size_t o = (size_t)cell * 2 * APPEND_MAX;
  for (int i = tid; i < n; i += blockDim.x) nl[i] = a.newlist[o + i];
  __syncthreads();
  const AppendCellDev &A = a.acells[cell];
  const int cur = A.cur;
  const int32_t *off = A.offsets[cur], *val = A.values[cur], *mat = A.mates[cur];
  int32_t *off2 = A.offsets[cur ^ 1], *val2 = A.values[cur ^ 1], *mat2 = A.mates[cur ^ 1];
  const int c = blockIdx.x * 256 + tid;
  if (c > a.nc) return;
  const int s = lower_bound_i32(nl, n, c);  // new postings in lists below c
  off2[c] = off[c] + s;
  if (c == a.nc) return;
  const int b = off[c], e = off[c + 1];
  for (int p = b; p < e; ++p) {
    val2[p + s] = val[p];
    mat2[p + s] = mat[p];
  }
  const int s1 = lower_bound_i32(nl, n, c + 1);
  for (int j = s; j < s1; ++j) {  // list c's new postings, after its old ones
    val2[e + j] = a.newtok[o + j];
    mat2[e + j] = a.newmate[o + j];
  }
}

__global__ void __launch_bounds__(256) k_append_commit(AppendArgs a) {
  const int tid = threadIdx.x;
  const int T = *a.tlen;
  const bool ok = T + a.m <= a.tmax;
  if (ok)
    for (int cell = tid; cell < a.n_cells; cell += blockDim.x) {
      AppendCellDev &A = a.acells[cell];
      const int nxt = A.cur ^ 1;
      A.cur = nxt;
      A.n_postings += 2 * a.m;
      CellDev &c = a.cells[cell];
      c.offsets = A.offsets[nxt];
      c.values = A.values[nxt];
      c.mates = A.mates[nxt];
    }
  __syncthreads();  // every thread has read the context before it moves
  if (tid == 0) {
    if (ok) *a.tlen = T + a.m;
    else atomicOr(a.status, APPEND_FULL);
  }
}

}  // namespace

cudaError_t launch_assign(const AssignArgs &a, cudaStream_t st) {
  if (a.m < 1 || a.m > APPEND_MAX || a.split < 1 || a.split > ASSIGN_SPLIT) return cudaErrorInvalidValue;
  const int full = a.m / 4, rest = a.m % 4;
  if (full) k_assign<4><<<dim3(a.split, a.n_cells, full), 256, 0, st>>>(a, 0);
  if (rest) k_assign<1><<<dim3(a.split, a.n_cells, rest), 256, 0, st>>>(a, 4 * full);
  k_assign_reduce<<<a.n_cells, 1024, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_append(const AppendArgs &a, const AssignArgs &assign, cudaStream_t st) {
  if (a.m < 1 || a.m > APPEND_MAX) return cudaErrorInvalidValue;
  k_append_codec<<<dim3(a.m, a.n_cells), 256, 0, st>>>(a);
  cudaError_t e = launch_assign(assign, st);
  if (e != cudaSuccess) return e;
  k_post_prepare<<<a.n_cells, 1024, 0, st>>>(a);
  k_post_rebuild<<<dim3(a.nc / 256 + 1, a.n_cells), 256, 0, st>>>(a);
  k_append_commit<<<1, 256, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace skv
