// skv_device.cuh -- shared device helpers and the engine's device layout.
//
// Arithmetic conventions (identical in the CPU oracle):
//   * a scoring dot product is the EXACT sum of (query operand x small
//     integer code weight), rounded once to FP32.  Each operand row is first
//     flushed below 2^(E-22) (E = top exponent of the row), which puts every
//     kept element on the integer grid 2^(E-29) with |X| < 2^30.  X is split
//     into four signed base-256 digits and the code weights are int8, so the
//     sum runs on int8 tensor cores (mma.sync m16n8k32, int32 accumulate)
//     without any rounding, and the digit sums recombine exactly in int64;
//   * FP32 post-operations use __f*_rn intrinsics so nothing is contracted;
//   * FP32 -> BF16 rounds to nearest even.
#pragma once
#include <climits>
#include <cstdint>
#include <cuda_bf16.h>
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
constexpr int ATTN_SPLIT = 32;     // attention partitions per KV head
constexpr int REC = 512;           // FP8 [K | V] record bytes
constexpr int NCOUNT = 8;          // per-cell counters
constexpr int CHUNK = 1024;        // centroid / pool positions per chunk CTA
constexpr int SCHUNK = 256;        // survivors per pool-kernel CTA
constexpr int FRAG_ROW = 8 * 2 * 32 * 2;  // u32 per operand row set (ks, n-tile, lane, reg)
constexpr int PART = 260;          // floats per attention partial (m, l, pad, pad, o[256])

constexpr int FUSED_MARKS = 96;  // (tag, clock) profiling marks of the fused kernel

// Per-cell counters (Work::counts[cell][*]).
enum Count { C_TAGS = 0, C_SEL = 1, C_POOL = 2, C_U15 = 3, C_CAND = 4, C_STATUS = 5, C_POSTINGS = 6 };
// Threshold slots (Work::thr[cell][stage][head]).
enum Stage { T_COARSE = 0, T_FINE = 1, T_S15 = 2, T_S16 = 3 };
// Operand rows (Work::frag / Work::shift).
enum Row { R_Q = 0, R_Q15 = 1, R_QS = 2 };

constexpr uint32_t ST_POOL_OVER = 1u, ST_POOL_UNDER = 2u, ST_FINE_SHORT = 4u, ST_TIMEOUT = 8u;

// ---- sequence-sharded group over peer memory (one slot of 4 cells per shard)
constexpr int SHARD_MAX = 8;    // shards of a peer-memory group
constexpr int SHARD_CELLS = 4;  // one slot: 4 KV heads

// The exchange region every shard owns and every peer writes into.
struct ShardRegion {
  uint32_t keys[SHARD_MAX][SHARD_CELLS * G][TOPK];        // [source shard][cell*4+head][rank]
  int32_t ids[SHARD_MAX][SHARD_CELLS * G][TOPK];
  float part[SHARD_MAX][SHARD_CELLS][G][PART];            // [source shard][cell][head][m, l, 0, 0, o]
  uint32_t flag_lists[SHARD_MAX][SHARD_CELLS * G];        // epoch of each source's (cell, head) list
  uint32_t flag_parts[SHARD_MAX][SHARD_CELLS];            // epoch of each source's cell partials
  // the fused kernel's lists: one 8-byte entry per rank carrying its own
  // step tag, [tag 8 | score 16 | 0 8 | shard-local id 32], so a reader
  // needs no flag and the writer no fence; double-buffered by step parity
  unsigned long long ll[2][SHARD_MAX][SHARD_CELLS * G][TOPK];
};

// Kernel-side view of a connected group.
struct ShardLinkDev {
  void *peer[SHARD_MAX];          // every shard's region as mapped here (own one included)
  const uint8_t *kv8[SHARD_MAX][SHARD_CELLS];  // every shard's FP8 [K|V] records as mapped here
  int32_t begin[SHARD_MAX];       // first global token of each shard
  int32_t rank, n_shards, token_begin;
  int32_t total, sink, local;     // the whole layer's context and dense zones
  uint32_t *epoch;                // steps completed (device counter)
  uint32_t *exits;                // clusters of the current fused step that have finished
};

// Cross-GPU flags: release/acquire at system scope; bounded polls.
constexpr long long SHARD_WAIT_POLLS = 1 << 24;  // ~1.7 s at ~100 ns per poll

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
// Waits until flag[s * stride] >= epoch for every shard s; false on timeout.
__device__ __forceinline__ bool wait_flags(const uint32_t *flag, int stride, int n_shards, uint32_t epoch) {
  for (int s = 0; s < n_shards; ++s) {
    long long polls = 0;
    while (ld_acquire_sys(flag + (size_t)s * stride) < epoch) {
      if (++polls > SHARD_WAIT_POLLS) return false;
      __nanosleep(100);
    }
  }
  return true;
}

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
  const uint16_t *q;                 // the lead cell's own query [4][256] (null: the slot's query)
  int32_t nc, nprobe;
  float lam;
  int32_t context;                   // the lead cell's own context (0: the engine's)
};

// Workspace: one base pointer per buffer, indexed by cell inside kernels.
// Buffers marked (step) must be zero when a step starts; the last kernel of
// a step clears them again for the next one.
struct Work {
  int n_cells, n_slots, T, sink, local, nc, cap;
  int lead;                 // 1: the fused launch carries the lead cluster (cell n_cells, launched first)
  int trace;                // 1: the fused kernel writes every stage's intermediates (SKV_FLAG_TRACE)
  int chunks_nc;            // ceil(nc / CHUNK)
  int chunks_surv;          // ceil(nc / SCHUNK)
  int chunks_pool;          // ceil(cap / CHUNK)
  const CellDev *cells;
  const uint16_t *q;        // [n_slots][16][256] BF16
  uint32_t *frag;           // [cell][3][FRAG_ROW] int8 digit fragments of the operand rows
  int32_t *shift;           // [cell][3][4] value = digits-sum * 2^shift
  float *qscal;             // [cell][8]  lambda*|q| [4], 3*sum(q) [4]
  uint16_t *lo, *hi;        // [cell][4][nc] ordered BF16 coarse bounds
  uint32_t *thr;            // [cell][4 stages][4 heads]
  uint8_t *smask;           // [cell][nc] coarse head masks
  int32_t *chunk_cnt;       // [cell][chunks_nc] survivors per centroid chunk
  uint32_t *tags;           // [cell][nc]
  uint32_t *fkeys;          // [cell][4][nc]
  uint32_t *selbits;        // [cell][nc/32] selected clusters (step)
  uint16_t *kept;           // [cell][nc] kept postings per survivor
  unsigned long long *keptmask;  // [cell][nc] kept postings of lists <= 64 long
  int32_t *chunk_kept;      // [cell][chunks_surv]
  int32_t *chunk_sel;       // [cell][chunks_surv]
  int32_t *chunk_post;      // [cell][chunks_surv]
  int32_t *sel;             // [cell][SEL_MAX]
  int32_t *pool;            // [cell][cap]
  uint32_t *k15;            // [cell][4][cap]
  uint32_t *u15bits;        // [cell][cap/32] (step)
  int32_t *u15pos;          // [cell][U15_MAX]
  int32_t *u15tok;          // [cell][U15_MAX]
  uint32_t *k16;            // [cell][4][U15_MAX]
  uint32_t *candbits;       // [cell][U15_MAX/32] (step)
  int32_t *cand;            // [cell][CAND_MAX]
  uint32_t *k2;             // [cell][4][CAND_MAX] Stage-II keys
  int32_t *final_pos;       // [cell][4][TOPK]
  int32_t *final_ids;       // [cell][4][TOPK]
  uint32_t *final_keys;     // [cell][4][TOPK] Stage-II keys [ordered bf16 score | 0xffff - u], 0 = none
  int32_t *counts;          // [cell][NCOUNT]
  float *attn_part;         // [cell][4][ATTN_SPLIT][PART]
  uint32_t *arrive;         // [cell] attention partitions finished (step)
  uint32_t *hist;           // [cell][4 stages][4 heads][4096] first-pass histograms (step)
  uint16_t *out;            // [n_slots][16][256] BF16
  uint16_t *out_host;       // fused host-I/O step: the output also goes straight to mapped pinned memory (or null)
  int32_t *counts_host;     // ... and each cell's counters after its last barrier (or null)
  uint16_t *q_store;        // ... and the query, read from mapped memory, is mirrored here for later kernels (or null)
  long long *phase_ts;      // [FUSED_MARKS][2] (tag, SM clock) marks of cell 0, or null
  long long *cta_ts;        // [cell][16][2] global timer (ns) at CTA entry and exit, then [16][FUSED_MARKS][2]
                            // (tag, ns) phase marks of cell 0's CTAs (fused), or null
  const ShardLinkDev *link; // sequence-sharded group (device copy), or null
  int32_t *shard_gids;      // [4][4][TOPK] the group's global winners (with link)
  const int32_t *tlen;      // the slots' current context (grows with cache appends), or null: T
};

// Current context of the engine's slots: cache appends advance it on the
// device, so a step replayed from a graph sees the appended tokens.
__device__ __forceinline__ int context_of(const Work &w) { return w.tlen ? *w.tlen : w.T; }

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

// First-pass histogram (top 12 key bits) of one selection.
__device__ __forceinline__ uint32_t *hist_of(const Work &w, int cell, int stage, int head) {
  return w.hist + (((size_t)cell * 4 + stage) * G + head) * 4096;
}

// 2^e as a double, e in the normal range.
__device__ __forceinline__ double pow2d(int e) { return __hiloint2double((e + 1023) << 20, 0); }

// Scale 2^e of an exact digit sum, in the two forms exact_to_float uses.
struct Pow2 {
  double d;
  float f;
  bool fast;  // 2^e is a normal FP32 number and no 64-bit sum scaled by it overflows
};
__device__ __forceinline__ Pow2 pow2s(int e) {
  Pow2 p;
  p.d = pow2d(e);
  p.fast = e >= -126 && e <= 64;
  p.f = p.fast ? __int_as_float((e + 127) << 23) : 0.0f;
  return p;
}

// Exact digit sum -> FP32 score input, rounded once to nearest even.
// dsum * 2^e is exact in double (|dsum| < 2^53); when 2^e is a normal FP32
// number every non-zero result is normal (|dsum| >= 1) and finite
// (|dsum| < 2^63, e <= 64), and rounding dsum to FP32 first and scaling by
// 2^e afterwards is the same single rounding: one 64-bit integer conversion
// instead of three double-precision operations.
__device__ __forceinline__ float exact_to_float(long long dsum, const Pow2 &s) {
  return s.fast ? __fmul_rn(__ll2float_rn(dsum), s.f) : __double2float_rn(__ll2double_rn(dsum) * s.d);
}

// BF16 round-to-nearest-even of a finite score by the conversion
// instruction; equal to bf16_rne for every non-NaN input (scores computed from
// exact digit sums are never NaN).
__device__ __forceinline__ uint16_t bf16_score(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }

// ------------------------------------------------------ tensor-core dots

// B operand fragments of one operand row set: 8 k-steps x 2 n-tiles x 2 regs.
// Column n of n-tile nt is (head 2*nt + n/4, digit n%4).  Within k-step ks,
// register reg, byte b of lane-in-quad tq holds dimension
// 32*ks + 16*reg + 4*b + tq: the order in which w2()/w_nib() place the
// weights of a plane word into the bytes of an A register.
struct BFrag {
  uint32_t b[8][2][2];
};

__device__ __forceinline__ void load_bfrag(const Work &w, int cell, int row, int lane, BFrag &f) {
  const uint2 *p = reinterpret_cast<const uint2 *>(w.frag + ((size_t)cell * 3 + row) * FRAG_ROW);
#pragma unroll
  for (int ks = 0; ks < 8; ++ks)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const uint2 v = p[(ks * 2 + nt) * 32 + lane];
      f.b[ks][nt][0] = v.x;
      f.b[ks][nt][1] = v.y;
    }
}

__device__ __forceinline__ void mma_s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                       uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Recombine the four digit accumulators.  Thread t of a quad ends with the
// exact sum for row (t odd ? g + 8 : g) and heads t/2 (d[0]) and 2 + t/2 (d[1]).
__device__ __forceinline__ void combine_digits(const int (&acc)[2][4], int t, long long (&d)[2]) {
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    // this lane's digit pair for rows g and g + 8 (|acc| < 2^19, so the pair
    // sums fit 32 bits); even lanes hold digits 0-1 (weights 1, 256), odd
    // lanes digits 2-3 (65536, 2^24); the even lane finishes row g, the odd
    // lane row g + 8, each with one 32-bit value from its partner
    const int pg = acc[nt][0] + 256 * acc[nt][1];
    const int p8 = acc[nt][2] + 256 * acc[nt][3];
    const int x = __shfl_xor_sync(0xffffffffu, (t & 1) ? pg : p8, 1);
    d[nt] = (t & 1) ? (long long)p8 * 65536LL + x : (long long)pg + (long long)x * 65536LL;
  }
}

// Weight unpacking: byte i of the result is the weight of dimension
// 16*word + 4*i + t for a 2-bit-per-dimension plane word.
__device__ __forceinline__ uint32_t w2(uint32_t word, int t) { return (word >> (2 * t)) & 0x03030303u; }
// 2p - 3 for p in 0..3 (Stage-1.5 prefix codes).
__device__ __forceinline__ uint32_t w_odd2(uint32_t p) { return __vsub4(p << 1, 0x03030303u); }
// 2(4u + l) - 15 for the 4-bit code (u, l) (Fine centroid codes, Stage-1.6 keys).
__device__ __forceinline__ uint32_t w_odd4(uint32_t u, uint32_t l) {
  return __vsub4((u << 3) | (l << 1), 0x0f0f0f0fu);
}
// 2n - 15 for the residual4 nibbles of dimensions 16*word + 4*i + t, from the
// two residual4 words covering those 16 dimensions.
__device__ __forceinline__ uint32_t w_nib(uint32_t lo_word, uint32_t hi_word, int t) {
  const uint32_t x = (lo_word >> (4 * t)) & 0x000f000fu, y = (hi_word >> (4 * t)) & 0x000f000fu;
  return __vsub4(__byte_perm(x, y, 0x6420) << 1, 0x0f0f0f0fu);
}

__device__ __forceinline__ uint32_t word_of(const uint4 (&r)[4], int i) {
  const uint4 v = r[i >> 2];
  return (i & 3) == 0 ? v.x : (i & 3) == 1 ? v.y : (i & 3) == 2 ? v.z : v.w;
}

// --------------------------------------------------- warp-aggregated atomics

// hist[bin] += 1 for every lane whose bin != 0xffffffff.  The lanes that
// share lane 0's bin are added with one atomic (selection keys crowd into a
// few bins, where per-lane atomics on one address serialise); the others
// add individually.  All 32 lanes of the warp must call it.
__device__ __forceinline__ void hist_add_warp(uint32_t *hist, uint32_t bin) {
  const uint32_t b0 = __shfl_sync(0xffffffffu, bin, 0);
  const unsigned same = __ballot_sync(0xffffffffu, bin == b0);
  if ((threadIdx.x & 31) == 0) {
    if (b0 != 0xffffffffu) atomicAdd(&hist[b0], (uint32_t)__popc(same));
  } else if (bin != b0 && bin != 0xffffffffu) {
    atomicAdd(&hist[bin], 1u);
  }
}

// One slot of *counter for every lane with `want` (one atomic per warp);
// returns the lane's slot, or -1.  All 32 lanes of the warp must call it.
__device__ __forceinline__ int warp_claim(int *counter, bool want) {
  const unsigned m = __ballot_sync(0xffffffffu, want);
  if (!m) return -1;
  const int lane = threadIdx.x & 31, leader = __ffs(m) - 1;
  int base = 0;
  if (lane == leader) base = atomicAdd(counter, __popc(m));
  base = __shfl_sync(0xffffffffu, base, leader);
  return want ? base + __popc(m & ((1u << lane) - 1u)) : -1;
}

// ------------------------------------------------------------ block scans

// Exclusive prefix sum over the block (blockDim.x a multiple of 32, <= 1024).
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
    int wv = lane < nwarps ? s_warp[lane] : 0;
    int t = wv;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    if (lane < nwarps) s_warp[lane] = t - wv;
    if (lane == 31) s_total = t;
  }
  __syncthreads();
  const int r = s_warp[warp] + x - v;
  *total = s_total;
  __syncthreads();
  return r;
}

// Sum of src[0..n) computed by the whole block (result in every thread).
__device__ __forceinline__ int block_sum_prefix(const int32_t *src, int n) {
  int s = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += src[i];
  int total;
  block_exclusive_scan(s, &total);
  return total;
}

// Given a 256-bin histogram in shared memory, find the bin holding the k-th
// largest element (1-based k) scanning from bin 255 down.  Executed by warp 0;
// results are written to *bin and *above (count strictly above that bin).
__device__ __forceinline__ void find_bin_desc(const uint32_t *hist, uint32_t k, int *bin,
                                              uint32_t *above) {
  const int lane = threadIdx.x & 31;
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
