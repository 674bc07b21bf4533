// skv_select.cuh -- block-level K-th largest selection over 32-bit keys
// (the staged kernels' selections).
#pragma once
#include "skv_device.cuh"

namespace skv {

// Bin holding the k-th largest element of a `nbins`-bin histogram in shared
// memory (bins scanned from the top); every thread gets (bin, count above).
static __device__ void block_find_bin(const uint32_t *hist, int nbins, uint32_t k, int *bin, uint32_t *above) {
  __shared__ int s_bin;
  __shared__ uint32_t s_above;
  const int nt = blockDim.x, per = (nbins + nt - 1) / nt, tid = threadIdx.x;
  if (tid == 0) { s_bin = -1; s_above = 0; }
  uint32_t cnt = 0;
  for (int j = 0; j < per; ++j) {
    const int b = nbins - 1 - tid * per - j;
    if (b >= 0) cnt += hist[b];
  }
  int tot;
  const uint32_t excl = (uint32_t)block_exclusive_scan((int)cnt, &tot);
  if (excl < k && k <= excl + cnt) {
    uint32_t acc = excl;
    for (int j = 0; j < per; ++j) {
      const int b = nbins - 1 - tid * per - j;
      if (b < 0) break;
      if (acc + hist[b] >= k) { s_bin = b; s_above = acc; break; }
      acc += hist[b];
    }
  }
  __syncthreads();
  *bin = s_bin;
  *above = s_above;
  __syncthreads();
}

constexpr int SEL_BINS = 4096;   // first-pass histogram: top 12 key bits
constexpr int SEL_LIST = 4096;   // members of the boundary bin kept for refinement

struct SelectScratch {
  uint32_t hist[SEL_BINS];
  uint32_t list[SEL_LIST];
  int n_list, bin;
  uint32_t above;
};

// Radix refinement over `src` (n keys): keys are filtered by
// (v & mask) == prefix; digits of `bits` bits starting at `shift` downwards.
static __device__ uint32_t radix_refine(const uint32_t *src, int n, uint32_t prefix, uint32_t mask, int shift,
                                 uint32_t k, SelectScratch &sc) {
  const int tid = threadIdx.x;
  while (shift > 0) {
    const int bits = shift >= 8 ? 8 : shift;
    const int sh = shift - bits;
    const uint32_t dmask = (1u << bits) - 1u;
    for (int i = tid; i < 256; i += blockDim.x) sc.hist[i] = 0;
    if (tid == 0) { sc.bin = 0; sc.above = 0; }
    __syncthreads();
    for (int i = tid; i < n; i += blockDim.x) {
      const uint32_t v = src[i];
      if ((v & mask) == prefix) atomicAdd(&sc.hist[(v >> sh) & dmask], 1u);
    }
    __syncthreads();
    if (tid < 32) find_bin_desc(sc.hist, k, &sc.bin, &sc.above);
    __syncthreads();
    prefix |= (uint32_t)sc.bin << sh;
    mask |= dmask << sh;
    k -= sc.above;
    shift = sh;
    __syncthreads();
  }
  return prefix;
}

// K-th largest (1-based) of the n keys in shared memory `keys`.  Returns
// 0xffffffff when K == 0 and 0 when fewer than K keys exist.  Duplicates are
// allowed (the result is the K-th largest value).
static __device__ uint32_t select_kth(const uint32_t *keys, int n, int K, SelectScratch &sc) {
  const int tid = threadIdx.x, nt = blockDim.x;
  if (K <= 0) return 0xffffffffu;
  if (n < K) return 0u;
  for (int i = tid; i < SEL_BINS; i += nt) sc.hist[i] = 0;
  if (tid == 0) { sc.n_list = 0; sc.bin = 0; sc.above = 0; }
  __syncthreads();
  for (int i = tid; i < n; i += nt) atomicAdd(&sc.hist[keys[i] >> 20], 1u);
  __syncthreads();
  // thread t owns the t-th group of (SEL_BINS / nt) bins counted from the top
  const int per = SEL_BINS / nt;
  uint32_t cnt = 0;
  for (int j = 0; j < per; ++j) cnt += sc.hist[SEL_BINS - 1 - tid * per - j];
  int tot;
  const uint32_t excl = (uint32_t)block_exclusive_scan((int)cnt, &tot);
  if (excl < (uint32_t)K && (uint32_t)K <= excl + cnt) {
    uint32_t acc = excl;
    for (int j = 0; j < per; ++j) {
      const int b = SEL_BINS - 1 - tid * per - j;
      if (acc + sc.hist[b] >= (uint32_t)K) { sc.bin = b; sc.above = acc; break; }
      acc += sc.hist[b];
    }
  }
  __syncthreads();
  const uint32_t top = (uint32_t)sc.bin, above = sc.above;
  for (int i = tid; i < n; i += nt) {
    const uint32_t v = keys[i];
    if ((v >> 20) == top) {
      const int slot = atomicAdd(&sc.n_list, 1);
      if (slot < SEL_LIST) sc.list[slot] = v;
    }
  }
  __syncthreads();
  const int m = sc.n_list;
  const uint32_t k = (uint32_t)K - above;
  __syncthreads();
  if (m <= SEL_LIST) return radix_refine(sc.list, m, top << 20, 0xfff00000u, 20, k, sc);
  return radix_refine(keys, n, top << 20, 0xfff00000u, 20, k, sc);
}

}  // namespace skv
