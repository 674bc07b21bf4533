// skv_fused.cu -- the whole decode funnel of one cell as ONE thread-block
// cluster.
//
// A cell (slot x KV head) is decoded by a cluster of CL = 16 CTAs, one CTA
// per SM; one launch covers every cell of the step.  The stages of the
// staged path (skv_kernels.cu) become phases of a single kernel, and what a
// phase hands to the next stays in shared memory or is pushed into the
// shared memory of the CTA that consumes it:
//
//   P0  query operands: every CTA derives the 12 operand rows itself
//   P1  coarse: the CTA's contiguous slice of the upper plane arrives by TMA
//       bulk copies (8 KB each, one mbarrier each) and is scored on int8
//       tensor cores; lo/hi stay in shared memory, and the coarse
//       selection's first-round histogram is built on the way
//   P2  coarse threshold: cluster radix select, two 8-bit rounds
//   P3  survivors: head masks, exchange -> global positions; every CTA
//       pushes its survivors into equal shares of the global order
//   P4  fine: upper+lower rows of this CTA's share gathered with cp.async
//   P5  fine top-nprobe per head (cluster select), selected bitmap
//   P6  pool: postings of the selected clusters, spill-2 mate rule,
//       exchange -> pool positions; kept tokens pushed into P7's shares
//   P7  Stage-1.5 and 1.6 scores over a balanced share of the pool
//   P8  top-1600 per head, ascending union (exchange)
//   P10 top-256 per head, candidates (exchange)
//   P11 Stage-II scores of this CTA's candidates (small gather), pushed to
//       CTA h for head h
//   P12 exact top-100 per head (CTA h), rank order, pushed to every CTA
//   P13 attention: CTAs 4-15 fold the sink and local zones during P12, then
//       every warp folds its share of the top-100; each CTA's partials for
//       a share of the output dimensions go to the CTA finishing them
//
// Communication inside the cluster is by asynchronous stores into the
// receiver's shared memory (st.async ... mbarrier::complete_tx), each
// completing a transaction count on the receiver's mbarrier, which the
// receiver waits on with acquire at cluster scope; the expected byte counts
// follow from counts every CTA knows at that point (exchanged four-int
// records, or fixed shapes).  Cluster selection (P2, P5, P8, P10): every CTA
// histograms its keys, pushes its counts of head h into CTA h's per-source
// table; CTA h sums them, finds the boundary bin and pushes the round's
// result (and, in the last round of a 32-bit selection, each CTA's share of
// the tied keys) back; see cluster_select.
//
// With Work::trace, every intermediate the staged path exposes (lo/hi,
// survivor tags, selected clusters, pool, unions) is also written to the same
// Work buffers in the same format, so both paths are checked by the same
// stage-by-stage parity tests; thresholds, final ranks and ids and the
// counters are always written.
//
// The lead cluster (Work::lead): the launch carries one more cluster,
// blockIdx.y 0, that decodes the engine's small synthetic cell (index
// n_cells) through the same phases.  Its work is a few percent of a real
// cell's, so it runs ahead and its instruction fetches bring the kernel's
// code into L2 before the real cells execute it; its outputs are never read.
//
// Waits: every wait on another CTA is a bounded poll of an mbarrier phase
// (XWAIT_POLLS) that records ST_TIMEOUT in the cell's status and returns
// instead of waiting on; the coarse-slice copies likewise (WAIT_POLLS); the
// sequence-sharded list entries and, in a linked cell, the merged winners
// are bounded on the global timer (SHARD_LIST_NS, WIN_WAIT_NS).  The cluster
// barriers left (the start and the end, where no CTA may leave while its
// shared memory can still be read) are reached by all threads of all CTAs:
// control flow is uniform by construction.
#include <cuda_fp8.h>

#include "skv_device.cuh"
#include "skv_fused.cuh"

namespace skv {
namespace {

constexpr int CL = 16;                            // CTAs per cluster (per cell)
constexpr int FT = 512;                           // threads per CTA
constexpr int FW = FT / 32;                       // warps per CTA
constexpr int PER_MAX = 2048;                     // centroid rows per CTA
constexpr int SLICE_CHUNK = 128;                  // rows per bulk copy (8 KB)
constexpr int NCHUNK = PER_MAX / SLICE_CHUNK;     // mbarriers
constexpr int POS_MAX = 1024;                     // pool positions per CTA
constexpr int BIG = PER_MAX * 64;                 // staging area (128 KB)
constexpr long long WAIT_POLLS = 1 << 20;         // mbarrier polls before giving up (slice copies)
constexpr long long XWAIT_POLLS = 1 << 16;        // polls before giving up on other CTAs' pushes
// Timed bounds (global timer) of the sequence-sharded step: an owner CTA
// waits at most SHARD_LIST_NS for the other shards' lists, and every CTA of a
// linked cell waits for the merged winners up to WIN_WAIT_NS from the start of
// its own wait, longer than any owner can take; so a late or missing shard
// ends the step with ST_TIMEOUT, and every push a CTA is sent still lands
// before that CTA stops waiting for it.
constexpr unsigned long long SHARD_LIST_NS = 2000000000ull;
constexpr unsigned long long WIN_WAIT_NS = 3000000000ull;

// Row strides (bytes) of gathered rows in the staging area: 16 bytes of
// padding keep the 8-byte fragment loads of a warp on distinct banks.
constexpr int STRIDE_FINE = 144;   // upper | lower
constexpr int STRIDE_S2 = 272;     // prefix2 | residual2 | residual4
constexpr int BATCH_FINE = (BIG / STRIDE_FINE) & ~15;
constexpr int BATCH_S2 = (BIG / STRIDE_S2) & ~15;
// kept pool tokens a CTA stages (P6): only pool positions below the capacity
// (<= CL * POS_MAX) are used, so a CTA keeps at most that many
constexpr int KMAX = CL * POS_MAX;
static_assert(KMAX * 4 <= BIG, "kept tokens fit the staging area");

struct SelCtl {
  uint32_t prefix[4], mask[4], krem[4], th[4];
  int done[4];
  int own[4];    // this CTA holds the cluster's K-th largest key (its threshold is the global one)
};

// A selection round's outcome for one head, pushed by the head's owner to
// every CTA: the resolved prefix and remaining count, this CTA's threshold
// and flags (bit 0 done, bit 1 this CTA holds the K-th largest key, bits
// 8-19 the tied key to pick, 1-based in local order, 0 for none).
struct SelRes {
  uint32_t pf, kr, th, flags;
};

// Profiling marks of one CTA (thread 0): buffer, count, time base.
struct MarkState {
  long long *ts;  // null unless this CTA records
  int n;
  int global;     // global-timer ns (comparable across SMs) instead of SM clocks
};

struct FusedSmem {
  uint32_t frag[3 * FRAG_ROW];     // int8 digit fragments of the three operand rows
  uint32_t hist[4 * 256];          // selection histogram: word 128 h + b / 2 holds bins b, b + 1 of head h as
                                   // 16-bit counts (the cluster selections); 256 plain bins (P12)
  alignas(16) uint32_t tab[CL][128];  // CTA h < 4: each source CTA's counts of head h's bins (16-bit pairs)
  uint32_t sum[256];               // CTA h < 4: head h's bins summed over the cluster
  alignas(16) SelRes res[4];       // the owners' results of the latest selection round
  alignas(16) int xin[2][CL][4];   // exchange slots (consecutive exchanges alternate)
  unsigned long long mbar[NCHUNK];
  unsigned long long mb_in, mb_res, mb_x[2];  // selection inputs (owners), results, exchanges
  unsigned long long mb_sh;        // the survivor share (once per step)
  unsigned long long mb_pool, mb_s2, mb_win, mb_attn;  // pool share, Stage-II keys, winners, attention partials
  alignas(16) int win[G][TOPK];    // the step's top-100 tokens per head (pushed by CTA h)
  int ph_in, ph_res, ph_x, ph_pend; // phases of mb_in / mb_res / exchanges started so far; the pending exchange
  int all[CL][4];                  // the cluster's values of the latest exchange
  SelCtl ctl;
  int shift[3][4];
  float qscal[8];
  long long sxsum[3][4];           // sum over d of X_d per operand row and head
  int round, status, n_win, pad_;
  MarkState ms;                    // profiling marks (thread 0)
  CellDev cell;                    // this cell's descriptor (read once from global)
  alignas(16) union {
    struct { uint16_t lo[4][PER_MAX]; uint16_t hi[4][PER_MAX]; } c;   // P1-P3
    uint32_t fkey[4][PER_MAX];                                        // P4-P5
    struct { uint16_t slist[PER_MAX]; int soff[PER_MAX]; int ppre[PER_MAX + 1]; } s;  // P5-P6
    struct {
      uint16_t sc15[4][POS_MAX], sc16[4][POS_MAX];   // ordered BF16 scores
      int tok[POS_MAX];
      uint16_t urank[POS_MAX];     // rank among this CTA's union members
      uint16_t clist[POS_MAX];     // candidates (local positions)
      uint8_t flag[POS_MAX];       // union member
    } p;                                                              // P7-P11
  } b;
  float sx[4 * D];                 // the cell's four query rows (FP32 of BF16)
  float kscale[D];                 // per-dimension key scales
  int offs[PER_MAX + 1];           // CSR start of each Fine share survivor's list (P4 -> P5)
  uint16_t resid[PER_MAX];         // residual norms of the slice (BF16)
  float scale4[PER_MAX / 32];
  float fsc[CL * PER_MAX / 32];    // the cell's Fine scales (one per 32 centroids)
  uint16_t sidx[PER_MAX];          // survivors: slice row
  uint8_t smask[PER_MAX];          // survivors: head mask (bits 0-3), selected (bit 4)
  uint32_t shin[PER_MAX];          // this CTA's share of the survivors: global row | head mask << 16 | selected << 24
  alignas(128) uint8_t big[BIG];
};

constexpr size_t kSmemBytes = sizeof(FusedSmem) + 128;
static_assert(kSmemBytes <= 227 * 1024, "fused shared memory exceeds 227 KB");

// Profiling marks: (tag, SM clock) pairs written by one thread when
// Work::phase_ts is set; each tag names the segment that ends at it.
enum MarkTag {
  M_START, M_ISSUE, M_QEXP, M_QPREP, M_STARTED, M_SLICE, M_COARSE, M_HIST, M_SYNC, M_READ, M_CSEL,
  M_SURV, M_FGATHER, M_FINE, M_FSEL, M_SELLIST, M_SELX, M_KEEP, M_POOL, M_S15G, M_S15, M_S15SEL,
  M_U15, M_S16, M_S16SEL, M_CAND, M_S2, M_S2SEL, M_ATTN_ITEMS, M_ATTN_CTA, M_ATTN, M_XLIST, M_NTAGS
};

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// The mark buffer and count live in shared memory (FusedSmem::ms, set by
// thread 0 at entry) and only thread 0 records, so an unprofiled step pays one
// branch on the thread index per mark and nothing is held in registers or
// local memory across the phases.  (A marker object passed by reference to
// the out-of-line phases lived in local memory, and every thread read it back
// at every mark: ~4 us per step at 128K.)
struct Marker {
  MarkState *st;
  __device__ __forceinline__ void operator()(int tag) const {
    if (threadIdx.x == 0 && st->ts) {
      const int k = st->n;
      if (k < FUSED_MARKS) {
        st->ts[2 * k] = tag;
        st->ts[2 * k + 1] = st->global ? (long long)global_ns() : clock64();
        st->n = k + 1;
      }
    }
  }
};

// ------------------------------------------------------------ primitives

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Cluster-wide barrier that orders all prior memory operations of every
// thread (shared, distributed shared and global) before all later ones: the
// CTA barrier gathers the CTA's operations behind thread 0, whose cluster-
// scope fence releases them; the arrive itself is relaxed and the wait
// acquires.  (One fence per CTA instead of one per thread.)
__device__ __forceinline__ void cluster_sync() {
  __syncthreads();
  if (threadIdx.x == 0) asm volatile("fence.acq_rel.cluster;" ::: "memory");
  asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The two halves of cluster_sync(), for overlapping independent work.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Warm L2 with data a later phase gathers (no effect on results).
__device__ __forceinline__ void prefetch_l2(const void *p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}
__device__ __forceinline__ uint32_t remote(const void *p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_init(void *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(void *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
// Contiguous global -> own shared memory copy on the TMA engine (no multicast).
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, void *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ bool mbar_try(void *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait on an mbarrier phase: false after WAIT_POLLS polls.
__device__ __noinline__ bool mbar_wait(void *bar, uint32_t parity) {
  for (long long i = 0; i < WAIT_POLLS; ++i)
    if (mbar_try(bar, parity)) return true;
  return false;
}
// As mbar_try for a phase that other CTAs' asynchronous stores complete: the
// acquire at cluster scope makes their data visible to this thread.
__device__ __forceinline__ bool mbar_try_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait of every thread of the CTA for such a phase; a wait that runs
// out records ST_TIMEOUT in the CTA's status and returns.
__device__ __noinline__ void mbar_wait_cluster(void *bar, uint32_t parity, int *status) {
  const uint32_t a = smem_addr(bar);
  for (long long i = 0; i < XWAIT_POLLS; ++i)
    if (mbar_try_cluster(a, parity)) return;
  atomicOr(reinterpret_cast<unsigned *>(status), ST_TIMEOUT);
}
// As mbar_wait_cluster, bounded by the global timer (and, should the timer
// stall, by 2^32 polls) instead of XWAIT_POLLS polls.
__device__ __noinline__ void mbar_wait_cluster_until(void *bar, uint32_t parity, int *status,
                                                     unsigned long long deadline) {
  const uint32_t a = smem_addr(bar);
  for (long long it = 0; it < (1ll << 26); ++it) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_cluster(a, parity)) return;
    if (global_ns() > deadline) break;
  }
  atomicOr(reinterpret_cast<unsigned *>(status), ST_TIMEOUT);
}
// Asynchronous 16-byte store into a CTA's shared memory (dst, from remote());
// its arrival completes 16 bytes of the transaction count of that CTA's
// mbarrier `bar` (also from remote()), with release semantics at cluster
// scope, so that a wait on the phase sees the data.
__device__ __forceinline__ void st_async_b32(uint32_t dst, uint32_t bar, uint32_t v) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(dst), "r"(v),
               "r"(bar)
               : "memory");
}
__device__ __forceinline__ void st_async_v4(uint32_t dst, uint32_t bar, uint4 v) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                   dst),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w), "r"(bar)
               : "memory");
}
// Orders this thread's earlier generic shared-memory accesses before later
// async-proxy (bulk copy) writes to the same memory.
__device__ __forceinline__ void cp16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ void load_frag(const FusedSmem &S, int row, int lane, BFrag &f) {
  const uint2 *p = reinterpret_cast<const uint2 *>(S.frag + row * FRAG_ROW);
#pragma unroll
  for (int ks = 0; ks < 8; ++ks)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const uint2 v = p[(ks * 2 + nt) * 32 + lane];
      f.b[ks][nt][0] = v.x;
      f.b[ks][nt][1] = v.y;
    }
}

// Every CTA publishes four ints (uniform over its threads); afterwards
// S.all[r][k] holds CTA r's values in every CTA.  Threads 0-15 push the
// CTA's 16 bytes into every CTA's exchange slot with asynchronous stores that
// complete the receiver's mbarrier; every CTA then waits (bounded) for the 16
// arrivals.  Consecutive exchanges alternate slots and mbarriers: a CTA can
// only start exchange k + 2 after every CTA has sent exchange k + 1, which
// each does after its wait for exchange k.
__device__ __noinline__ void exchange_send(FusedSmem &S, int v0, int v1, int v2, int v3) {
  const int tid = threadIdx.x;
  const int k = S.ph_x, b = k & 1;
  const uint32_t rank = cluster_rank();
  __syncthreads();  // every thread has read ph_x
  if (tid == 0) {
    S.ph_x = k + 1;
    S.ph_pend = k;
  }
  if (tid < CL)
    st_async_v4(remote(&S.xin[b][rank][0], (uint32_t)tid), remote(&S.mb_x[b], (uint32_t)tid),
                make_uint4((uint32_t)v0, (uint32_t)v1, (uint32_t)v2, (uint32_t)v3));
  if (tid == 0) mbar_expect_tx(&S.mb_x[b], CL * 16);
}
// The second half of exchange(): independent work may run between the two.
__device__ __noinline__ void exchange_wait(FusedSmem &S) {
  const int tid = threadIdx.x;
  __syncthreads();  // ph_pend is set
  const int k = S.ph_pend, b = k & 1;
  mbar_wait_cluster(&S.mb_x[b], (uint32_t)(k >> 1) & 1u, &S.status);
  if (tid < CL * 4) S.all[tid >> 2][tid & 3] = S.xin[b][tid >> 2][tid & 3];
  __syncthreads();
}
__device__ __forceinline__ void exchange(FusedSmem &S, int v0, int v1, int v2, int v3) {
  exchange_send(S, v0, v1, v2, v3);
  exchange_wait(S);
}
__device__ __forceinline__ int before(const FusedSmem &S, int k, int rank) {
  int s = 0;
  for (int r = 0; r < rank; ++r) s += S.all[r][k];
  return s;
}
__device__ __forceinline__ int total(const FusedSmem &S, int k) { return before(S, k, CL); }

// Warp-level: bin of the k-th largest element of a 256-bin histogram
// (bins counted from the top) and the count strictly above it.
__device__ __forceinline__ bool warp_find_desc(const uint32_t *hist, uint32_t k, int lane, int &bin,
                                               uint32_t &above) {
  uint32_t c[8], s = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) { c[j] = hist[255 - 8 * lane - j]; s += c[j]; }
  uint32_t incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  const uint32_t excl = incl - s;
  const bool mine = excl < k && k <= incl;
  const unsigned bal = __ballot_sync(0xffffffffu, mine);
  int b = 0;
  uint32_t ab = 0;
  if (mine) {
    uint32_t acc = excl;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (acc + c[j] >= k) { b = 255 - 8 * lane - j; ab = acc; break; }
      acc += c[j];
    }
  }
  const int src = bal ? __ffs(bal) - 1 : 0;
  bin = __shfl_sync(0xffffffffu, b, src);
  above = __shfl_sync(0xffffffffu, ab, src);
  return bal != 0;
}

enum KeyKind { KEY_COARSE = 0, KEY_FINE = 1, KEY_S15 = 2, KEY_S16 = 3 };

// This CTA's selection key i of head h.
//   KEY_COARSE: ordered BF16 lower bound (top 16 bits)
//   KEY_FINE:   fused IEEE key [bf16 score | u16 survivor position]
//   KEY_S15:    [ordered score | 0xffff - pool position]
//   KEY_S16:    as KEY_S15 for union members, 0 for the others
__device__ __forceinline__ uint32_t select_key(const FusedSmem &S, int kind, int h, int i, int q0) {
  switch (kind) {
    case KEY_COARSE: return (uint32_t)S.b.c.lo[h][i] << 16;
    case KEY_FINE: return S.b.fkey[h][i];
    case KEY_S15: return ((uint32_t)S.b.p.sc15[h][i] << 16) | (0xffffu - (uint32_t)(q0 + i));
    default:
      return S.b.p.flag[i] ? ((uint32_t)S.b.p.sc16[h][i] << 16) | (0xffffu - (uint32_t)(q0 + i)) : 0u;
  }
}

// One count in bin b (0..255) of head h of a selection histogram: bins b and
// b + 1 (b even) share a word as 16-bit counts (a CTA holds at most 2048 keys
// per head), the layout the histogram is pushed in.
__device__ __forceinline__ void hist_add(uint32_t *hist, int h, uint32_t b) {
  atomicAdd(&hist[h * 128 + (b >> 1)], 1u << ((b & 1u) << 4));
}

// One radix-histogram pass over this CTA's keys of `KIND`: keys with
// (key & mk[h]) == pf[h] add one to bin digit (bits sh..sh+7) of head h.
// Zero keys (a survivor position without head h, a pool position outside
// the union) are not counted: they lie below every real key, so the K-th
// largest key is the same whenever K real keys exist, and otherwise no bin
// is found and the threshold is 0 either way (the step's failure status);
// counting them only piled atomics onto bin 0.
// One shared-memory atomic per key: measured on B200 with BF16-like keys
// crowded into a few bins, this is faster than run-length counting in
// registers or per-warp aggregation (the atomic unit combines lanes of one
// instruction that hit the same address).
template <int KIND>
__device__ __forceinline__ void hist_pass(uint32_t *hist, const FusedSmem &S, int nloc, int q0,
                                          const uint32_t (&pf)[4], const uint32_t (&mk)[4], int sh) {
  if constexpr (KIND == KEY_COARSE) {
    // two 16-bit keys per 32-bit load (nloc is even: a slice is whole 16-row tiles)
#pragma unroll 1
    for (int i = 2 * threadIdx.x; i < nloc; i += 2 * FT) {
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const uint32_t two = *reinterpret_cast<const uint32_t *>(&S.b.c.lo[h][i]);
        const uint32_t v0 = two << 16, v1 = two & 0xffff0000u;
        if ((v0 & mk[h]) == pf[h]) hist_add(hist, h, (v0 >> sh) & 255u);
        if ((v1 & mk[h]) == pf[h]) hist_add(hist, h, (v1 >> sh) & 255u);
      }
    }
  } else {
    // two keys per load (i even; the second one counts only below nloc)
#pragma unroll 1
    for (int i = 2 * threadIdx.x; i < nloc; i += 2 * FT) {
      const bool two = i + 1 < nloc;
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        uint32_t v0, v1;
        if constexpr (KIND == KEY_FINE) {
          const uint2 k = *reinterpret_cast<const uint2 *>(&S.b.fkey[h][i]);
          v0 = k.x;
          v1 = k.y;
        } else if constexpr (KIND == KEY_S15) {
          const uint32_t sc = *reinterpret_cast<const uint32_t *>(&S.b.p.sc15[h][i]);
          v0 = (sc << 16) | (0xffffu - (uint32_t)(q0 + i));
          v1 = (sc & 0xffff0000u) | (0xffffu - (uint32_t)(q0 + i + 1));
        } else {
          const uint32_t sc = *reinterpret_cast<const uint32_t *>(&S.b.p.sc16[h][i]);
          const uint32_t fl = *reinterpret_cast<const uint16_t *>(&S.b.p.flag[i]);
          v0 = (fl & 0xffu) ? (sc << 16) | (0xffffu - (uint32_t)(q0 + i)) : 0u;
          v1 = (fl >> 8) ? (sc & 0xffff0000u) | (0xffffu - (uint32_t)(q0 + i + 1)) : 0u;
        }
        if (v0 && (v0 & mk[h]) == pf[h]) hist_add(hist, h, (v0 >> sh) & 255u);
        if (two && v1 && (v1 & mk[h]) == pf[h]) hist_add(hist, h, (v1 >> sh) & 255u);
      }
    }
  }
}

// warp_find_desc over bins held in registers: lane l holds c[j] = bin
// 255 - 8l - j.  Also returns the count in the found bin.
__device__ __forceinline__ bool warp_find_regs(const uint32_t (&c)[8], uint32_t k, int lane, int &bin,
                                               uint32_t &above, uint32_t &cnt) {
  uint32_t s = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) s += c[j];
  uint32_t incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  const uint32_t excl = incl - s;
  const bool mine = excl < k && k <= incl;
  const unsigned bal = __ballot_sync(0xffffffffu, mine);
  int b = 0;
  uint32_t ab = 0, cn = 0;
  if (mine) {
    uint32_t acc = excl;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (acc + c[j] >= k) { b = 255 - 8 * lane - j; ab = acc; cn = c[j]; break; }
      acc += c[j];
    }
  }
  const int src = bal ? __ffs(bal) - 1 : 0;
  bin = __shfl_sync(0xffffffffu, b, src);
  above = __shfl_sync(0xffffffffu, ab, src);
  cnt = __shfl_sync(0xffffffffu, cn, src);
  return bal != 0;
}

// K-th largest of the cluster's keys (select_key of `kind`) for each of the
// four heads; nbits (16 or 32) top bits of the 32-bit keys are significant.
// With `pre`, S.hist already holds this CTA's first-round histogram (its
// non-zero keys, counted while the keys were computed).
// On return S.ctl.th[h] holds a threshold: the keys >= it, over the whole
// cluster, are
//   exact (16 bits):  those >= the K-th largest key;
//   !exact (32 bits): exactly the K largest keys (keys are distinct), and
//                     th is 0 when K exceeds the number of keys or the K-th
//                     largest key is 0, 0xffffffff when K == 0.
// Two 8-bit radix rounds resolve the top 16 bits (for 32-bit keys the BF16
// score).  A round: every CTA histograms its own keys, pushes its 256 counts
// of each live head h (16-bit pairs, 512 bytes) into CTA h's per-source
// table with asynchronous stores that complete CTA h's input mbarrier; CTA h
// (the head's owner) waits for the 16 tables, sums them, finds the boundary
// bin and pushes a 16-byte result to every CTA, which waits for the results
// of its live heads.  No cluster barrier: a CTA sends round n + 1 only after
// it has every owner's result of round n, which each owner pushes after it
// has read its table, so one table, one input and one result mbarrier per
// CTA suffice.
// Keys of 32 bits that share the boundary score are resolved by position in
// the second round instead of by two more rounds: their low 16 bits order
// them by position (KEY_FINE: ascending for a positive score, descending for
// a negative one; KEY_S15 and KEY_S16: descending), and positions ascend with
// the CTA rank, so the krem largest tied keys are the first krem tied keys
// counted from the favoured end of the rank order.  The owner has every
// source's count of the boundary bin, gives each CTA its quota, and the
// CTA's threshold is the quota-th largest of its own tied keys (a ballot
// scan in local order).  The thresholds then differ between CTAs but select
// the keys a global K-th largest key would; S.ctl.own[h] marks the CTA whose
// threshold is the cluster's K-th largest key.
__device__ __noinline__ void cluster_select(FusedSmem &S, int nloc, uint32_t K, int nbits, bool exact, int kind,
                                            int q0, bool pre = false) {
  const Marker mark{&S.ms};
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int rank = (int)cluster_rank();
  int ph_in = S.ph_in, ph_res = S.ph_res;  // (read by every thread before the barrier below)
  if (tid < 4) {
    S.ctl.prefix[tid] = 0;
    S.ctl.mask[tid] = 0;
    S.ctl.krem[tid] = K;
    S.ctl.done[tid] = K == 0;
    S.ctl.th[tid] = K == 0 ? 0xffffffffu : 0u;
    S.ctl.own[tid] = rank == 0;
  }
  if (!pre)
    for (int e = tid; e < 4 * 128; e += FT) S.hist[e] = 0;
  __syncthreads();
  for (int sh = 24; sh >= 16; sh -= 8) {
    int live[4], nlive = 0;
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      live[h] = !S.ctl.done[h];
      nlive += live[h];
    }
    if (nlive == 0) break;
    const bool ties = !exact && nbits == 32 && sh == 16;
    // the four heads in one pass; a finished head matches no key
    uint32_t pf[4], mk[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      pf[h] = live[h] ? S.ctl.prefix[h] : 1u;
      mk[h] = live[h] ? S.ctl.mask[h] : 0u;
    }
    if (!(pre && sh == 24)) switch (kind) {
      case KEY_COARSE: hist_pass<KEY_COARSE>(S.hist, S, nloc, q0, pf, mk, sh); break;
      case KEY_FINE: hist_pass<KEY_FINE>(S.hist, S, nloc, q0, pf, mk, sh); break;
      case KEY_S15: hist_pass<KEY_S15>(S.hist, S, nloc, q0, pf, mk, sh); break;
      default: hist_pass<KEY_S16>(S.hist, S, nloc, q0, pf, mk, sh); break;
    }
    __syncthreads();
    mark(M_HIST);
    // this CTA's counts of each live head (16-bit pairs, as counted) to the
    // head's owner; each word is read and then cleared for the next round by
    // the one thread that pushes it
    const int sh_h = tid >> 5, sj = tid & 31;
    if (tid < 128 && live[sh_h]) {
      uint4 *hp = reinterpret_cast<uint4 *>(S.hist + sh_h * 128 + 4 * sj);
      const uint4 pk = *hp;
      st_async_v4(remote(&S.tab[rank][4 * sj], (uint32_t)sh_h), remote(&S.mb_in, (uint32_t)sh_h), pk);
      *hp = make_uint4(0u, 0u, 0u, 0u);
    }
    if (rank < 4 && live[rank]) {
      // owner of head h = rank
      const int h = rank;
      if (tid == 0) mbar_expect_tx(&S.mb_in, CL * 512);
      mbar_wait_cluster(&S.mb_in, (uint32_t)ph_in & 1u, &S.status);
      ++ph_in;
      if (tid < 128) {
        // word w holds bins 2w, 2w+1 as 16-bit counts; a bin's total over the
        // cluster is at most 16 * 2048 < 2^16, so the pairs add as one word
        uint32_t c = 0;
#pragma unroll
        for (int q = 0; q < CL; ++q) c += S.tab[q][tid];
        S.sum[2 * tid] = c & 0xffffu;
        S.sum[2 * tid + 1] = c >> 16;
      }
      __syncthreads();
      if (warp == 0) {
        uint32_t c[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) c[j] = S.sum[255 - 8 * lane - j];
        int bin;
        uint32_t above, cnt;
        const uint32_t krem = S.ctl.krem[h];
        const bool found = warp_find_regs(c, krem, lane, bin, above, cnt);
        const uint32_t pfx = S.ctl.prefix[h] | ((uint32_t)bin << sh);
        const uint32_t kr = krem - above;
        // result for destination CTA d = lane (lanes < 16)
        uint32_t th = 0u, flags = lane == 0 ? 2u : 0u;
        if (!found) {
          flags |= 1u;  // K exceeds the number of keys: th = 0
        } else if (sh == 32 - nbits || (!exact && cnt == kr && pfx != 0u)) {
          flags |= 1u;
          th = pfx;
        } else if (ties) {
          flags |= 1u;
          if (pfx != 0u) {
            const uint32_t B = pfx >> 16;
            const bool up = kind == KEY_FINE && (B & 0x8000u);  // low 16 bits ascend with the position
            const uint32_t cq = lane < CL ? (S.tab[lane][bin >> 1] >> (16 * (bin & 1))) & 0xffffu : 0u;
            uint32_t incl = cq;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
              const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
              if (lane >= o) incl += y;
            }
            const uint32_t all = __shfl_sync(0xffffffffu, incl, 31);
            const uint32_t pre = up ? all - incl : incl - cq;  // tied keys on the favoured side
            const uint32_t quota = kr > pre ? min(kr - pre, cq) : 0u;
            th = quota == 0 ? (B + 1u) << 16 : B << 16;  // none / all of the tied keys
            const uint32_t pick = (quota > 0 && quota < cq) ? (up ? cq - quota + 1 : quota) : 0u;
            flags = 1u | ((pre < kr && kr <= pre + cq) ? 2u : 0u) | (pick << 8);
          }
        }
        if (lane < CL)
          st_async_v4(remote(&S.res[h], (uint32_t)lane), remote(&S.mb_res, (uint32_t)lane),
                      make_uint4(pfx, kr, th, flags));
      }
    }
    mark(M_SYNC);
    if (tid == 0) mbar_expect_tx(&S.mb_res, 16u * (uint32_t)nlive);
    mbar_wait_cluster(&S.mb_res, (uint32_t)ph_res & 1u, &S.status);
    ++ph_res;
    if (warp < 4 && live[warp]) {
      const int h = warp;
      const SelRes r = S.res[h];
      uint32_t th = r.th;
      const uint32_t pick = (r.flags >> 8) & 0xfffu;
      if (pick) {
        // the pick-th tied key of this CTA in local order
        const uint32_t B = r.pf >> 16;
        uint32_t seen = 0;
        for (int base = 0; base < nloc; base += 32) {
          const int i = base + lane;
          const uint32_t v = i < nloc ? select_key(S, kind, h, i, q0) : 0u;
          const bool f = i < nloc && (v >> 16) == B;
          const unsigned bal = __ballot_sync(0xffffffffu, f);
          const bool me = f && seen + (uint32_t)__popc(bal & ((1u << lane) - 1u)) + 1u == pick;
          const unsigned hit = __ballot_sync(0xffffffffu, me);
          if (hit) {
            th = __shfl_sync(0xffffffffu, v, __ffs(hit) - 1);
            break;
          }
          seen += (uint32_t)__popc(bal);
        }
      }
      if (lane == 0) {
        S.ctl.prefix[h] = r.pf;
        S.ctl.mask[h] |= 255u << sh;
        S.ctl.krem[h] = r.kr;
        S.ctl.done[h] = (int)(r.flags & 1u);
        S.ctl.th[h] = th;
        S.ctl.own[h] = (int)((r.flags >> 1) & 1u);
      }
    }
    __syncthreads();
    mark(M_READ);
  }
  if (tid == 0) {
    S.ph_in = ph_in;
    S.ph_res = ph_res;
  }
  // a clear histogram for the next selection's first round, which the next
  // scoring phase may build on the way (heads done before any round still
  // hold a prebuilt first round)
  for (int e = tid; e < 4 * 128; e += FT) S.hist[e] = 0u;
  __syncthreads();
}

// ----------------------------------------------------- tensor-core dots

// Exact digit sums of 16 rows x 4 heads on int8 tensor cores; rows g and
// g+8 of the tile are given as shared-memory row pointers.  The weights are
// the raw codes; the odd-integer weights of the scores (2c - (2^b - 1)) are
// applied afterwards as 2 * dot - (2^b - 1) * sum(X), exactly, in int64.
//   KIND 0: 2-bit codes (0..3) of one 64-byte plane (coarse u, Stage-1.5 p)
//   KIND 1: 4-bit codes 4u + l from two 64-byte planes at +0, +64
template <int KIND>
__device__ __forceinline__ void tile_dots(const uint8_t *rg, const uint8_t *r8, int t, const BFrag &F,
                                          long long (&d)[2]) {
  int acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
  if (KIND == 0) {
    const uint4 *pg = reinterpret_cast<const uint4 *>(rg), *p8 = reinterpret_cast<const uint4 *>(r8);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 x = pg[q], y = p8[q];
      const uint32_t xs[4] = {x.x, x.y, x.z, x.w}, ys[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const int ks = 2 * q + h2;
        const uint32_t a0 = w2(xs[2 * h2], t), a1 = w2(ys[2 * h2], t);
        const uint32_t a2 = w2(xs[2 * h2 + 1], t), a3 = w2(ys[2 * h2 + 1], t);
        mma_s8(acc[0], a0, a1, a2, a3, F.b[ks][0][0], F.b[ks][0][1]);
        mma_s8(acc[1], a0, a1, a2, a3, F.b[ks][1][0], F.b[ks][1][1]);
      }
    }
    combine_digits(acc, t, d);
  } else {
    const uint2 *ug = reinterpret_cast<const uint2 *>(rg), *lg = reinterpret_cast<const uint2 *>(rg + 64);
    const uint2 *u8 = reinterpret_cast<const uint2 *>(r8), *l8 = reinterpret_cast<const uint2 *>(r8 + 64);
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const uint2 a = ug[ks], b = lg[ks], e = u8[ks], f = l8[ks];
      const uint32_t a0 = (w2(a.x, t) << 2) | w2(b.x, t), a1 = (w2(e.x, t) << 2) | w2(f.x, t);
      const uint32_t a2 = (w2(a.y, t) << 2) | w2(b.y, t), a3 = (w2(e.y, t) << 2) | w2(f.y, t);
      mma_s8(acc[0], a0, a1, a2, a3, F.b[ks][0][0], F.b[ks][0][1]);
      mma_s8(acc[1], a0, a1, a2, a3, F.b[ks][1][0], F.b[ks][1][1]);
    }
    combine_digits(acc, t, d);
  }
}

// Residual4 nibbles of dimensions 16*word + 4*i + t (bytes i) from the two
// residual4 words covering those 16 dimensions.
__device__ __forceinline__ uint32_t nib(uint32_t lo_word, uint32_t hi_word, int t) {
  return __byte_perm((lo_word >> (4 * t)) & 0x000f000fu, (hi_word >> (4 * t)) & 0x000f000fu, 0x6420);
}

// The Stage-1.6 and Stage-II raw-code sums of one tile at once: dh over the
// 4-bit codes c4 (prefix2 | residual2 at +0, +64), dl over the residual4
// nibbles r4 (+128).
__device__ __forceinline__ void tile_dots_8bit(const uint8_t *rg, const uint8_t *r8, int t, const BFrag &F,
                                               long long (&dh)[2], long long (&dl)[2]) {
  int hi[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}}, lo[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
  const uint2 *pg = reinterpret_cast<const uint2 *>(rg), *qg = reinterpret_cast<const uint2 *>(rg + 64);
  const uint4 *ng = reinterpret_cast<const uint4 *>(rg + 128);
  const uint2 *p8 = reinterpret_cast<const uint2 *>(r8), *q8 = reinterpret_cast<const uint2 *>(r8 + 64);
  const uint4 *n8 = reinterpret_cast<const uint4 *>(r8 + 128);
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const uint2 vpg = pg[ks], vqg = qg[ks], vp8 = p8[ks], vq8 = q8[ks];
    const uint4 vng = ng[ks], vn8 = n8[ks];
    const uint32_t a0 = (w2(vpg.x, t) << 2) | w2(vqg.x, t), a1 = (w2(vp8.x, t) << 2) | w2(vq8.x, t);
    const uint32_t a2 = (w2(vpg.y, t) << 2) | w2(vqg.y, t), a3 = (w2(vp8.y, t) << 2) | w2(vq8.y, t);
    mma_s8(hi[0], a0, a1, a2, a3, F.b[ks][0][0], F.b[ks][0][1]);
    mma_s8(hi[1], a0, a1, a2, a3, F.b[ks][1][0], F.b[ks][1][1]);
    const uint32_t b0 = nib(vng.x, vng.y, t), b1 = nib(vn8.x, vn8.y, t);
    const uint32_t b2 = nib(vng.z, vng.w, t), b3 = nib(vn8.z, vn8.w, t);
    mma_s8(lo[0], b0, b1, b2, b3, F.b[ks][0][0], F.b[ks][0][1]);
    mma_s8(lo[1], b0, b1, b2, b3, F.b[ks][1][0], F.b[ks][1][1]);
  }
  combine_digits(hi, t, dh);
  combine_digits(lo, t, dl);
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

// ------------------------------------------- sequence-sharded exchanges
//
// With Work::link (a connected group of shards, one per GPU), CTA h of a
// cell's cluster writes its head's top-100 (keys, shard-local ids) into every
// peer's exchange region over NVLink, raises its per-step flag there, waits
// (bounded) for every shard's list of the same (cell, head) in its own
// region, and merges: every shard's list is sorted by the 64-bit key
// [score | 0xffff - rank | ~global id], so a candidate's global rank is its
// own rank plus, per other list, a binary search for the entries above it.
// The merged global winners go to Work::shard_gids.

__device__ __forceinline__ unsigned long long merge_key(uint32_t key, int r, int gid) {
  return ((unsigned long long)(key >> 16) << 48) | ((unsigned long long)(0xffffu - (uint32_t)r) << 32) |
         (unsigned long long)(0xffffffffu - (uint32_t)gid);
}

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long *p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// The exchange and merge of head h's list (CTA h of the cell's cluster).
// Each entry travels as one naturally aligned 8-byte store (single-copy
// atomic, over NVLink too) that carries the step's tag, so a reader polls the
// entries themselves: no flag, no system-scope fence, one one-way trip.  The
// tag is the step counter's low byte and the buffer alternates with the
// step's parity; a shard can only overwrite a buffer after the whole group
// finished the step before (each shard's step ends after its own merge,
// which read every shard's entries).  The merged winners go to every CTA's
// S.win[h] by asynchronous stores (and to Work::shard_gids for the caller).
__device__ __noinline__ void shard_lists(const Work &w, FusedSmem &S, int cell, int h, const uint32_t *fkeys,
                                         const int32_t *fids) {
  const Marker mark{&S.ms};
  const ShardLinkDev &L = *w.link;
  const int tid = threadIdx.x, n = L.n_shards, ch = cell * G + h;
  const uint32_t epoch = *L.epoch + 1;
  const unsigned long long tag = (unsigned long long)(epoch & 0xffu) << 56;
  const int par = (int)(epoch & 1u);
  __syncthreads();  // this head's keys and ids are written
  for (int i = tid; i < TOPK; i += FT) {
    const unsigned long long v = tag | ((unsigned long long)(fkeys[i] >> 16) << 40) | (uint32_t)fids[i];
    for (int p = 0; p < n; ++p)
      st_relaxed_sys_u64(&reinterpret_cast<ShardRegion *>(L.peer[p])->ll[par][L.rank][ch][i], v);
  }
  // every shard's list of this (cell, head) into shared memory as 64-bit
  // merge keys, each entry polled (bounded) until it carries this step's tag;
  // the binary searches below then touch shared memory only
  const ShardRegion *R = reinterpret_cast<const ShardRegion *>(L.peer[L.rank]);
  unsigned long long *mk = reinterpret_cast<unsigned long long *>(S.big + 4096);  // [n][TOPK]
  static_assert(4096 + SHARD_MAX * TOPK * 8 <= BIG, "merge keys fit the staging area");
  // (bounded by SHARD_LIST_NS on the global timer, checked every 64 polls,
  // and by SHARD_WAIT_POLLS polls; once late, a thread stops polling)
  const unsigned long long deadline = global_ns() + SHARD_LIST_NS;
  bool late = false;
  for (int c = tid; c < n * TOPK; c += FT) {
    const int s = c / TOPK, r = c - s * TOPK;
    const unsigned long long *src = &R->ll[par][s][ch][r];
    unsigned long long v = ld_relaxed_sys_u64(src);
    for (long long polls = 0; (v & 0xff00000000000000ull) != tag; ++polls) {
      if (late || polls > SHARD_WAIT_POLLS || ((polls & 63) == 63 && global_ns() > deadline)) {
        late = true;
        break;
      }
      __nanosleep(64);
      v = ld_relaxed_sys_u64(src);
    }
    const uint32_t score = (uint32_t)(v >> 40) & 0xffffu;
    mk[c] = score ? merge_key(score << 16, r, L.begin[s] + (int32_t)(uint32_t)v) : 0ull;
  }
  if (late) atomicOr(reinterpret_cast<unsigned *>(&S.status), ST_TIMEOUT);
  __syncthreads();
  mark(M_XLIST);
  int32_t *gout = w.shard_gids + (size_t)ch * TOPK;
  int valid = 0;
  for (int c = tid; c < n * TOPK; c += FT) {
    const int s = c / TOPK, r = c - s * TOPK;
    const unsigned long long kv = mk[c];
    if (!kv) continue;
    const int gid = (int)(0xffffffffu - (uint32_t)(kv & 0xffffffffull));
    int rank = r;
    for (int s2 = 0; s2 < n; ++s2) {
      if (s2 == s) continue;
      const unsigned long long *l2 = mk + s2 * TOPK;
      int lo = 0, hi = TOPK;  // first entry of list s2 not above kv (zero keys end a list)
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (l2[mid] > kv) lo = mid + 1; else hi = mid;
      }
      rank += lo;
    }
    if (rank < TOPK) {
      gout[rank] = gid;
      for (int d = 0; d < CL; ++d)
        st_async_b32(remote(&S.win[h][rank], (uint32_t)d), remote(&S.mb_win, (uint32_t)d), (uint32_t)gid);
    }
    ++valid;
  }
  int total;
  block_exclusive_scan(valid, &total);
  // fewer than 100 candidates in the group: the remaining ranks are -1
  for (int i = total + tid; i < TOPK; i += FT) {
    gout[i] = -1;
    for (int d = 0; d < CL; ++d)
      st_async_b32(remote(&S.win[h][i], (uint32_t)d), remote(&S.mb_win, (uint32_t)d), 0xffffffffu);
  }
}

// ------------------------------------------------------------ the kernel

__global__ void __launch_bounds__(FT, 1) k_funnel(Work w) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  FusedSmem &S = *reinterpret_cast<FusedSmem *>(smem_raw + ((128u - (smem_addr(smem_raw) & 127u)) & 127u));
  const unsigned long long t_entry = global_ns();  // (CTA entry stamp of skv_profile_ctas)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, gq = lane >> 2, t = lane & 3;
  const int hA = t >> 1, hB = 2 + hA;
  const int rank = (int)cluster_rank();
  // the lead cluster (launched first: blockIdx.y 0) decodes the engine's
  // small synthetic cell n_cells; its outputs are never read
  const int cell = w.lead ? (blockIdx.y == 0 ? w.n_cells : (int)blockIdx.y - 1) : (int)blockIdx.y;
  const bool lead = cell == w.n_cells, timed = w.cta_ts && !lead;
  const int slot = cell >> 2, g = cell & 3;
  if (tid < (int)(sizeof(CellDev) / 4))
    reinterpret_cast<uint32_t *>(&S.cell)[tid] = reinterpret_cast<const uint32_t *>(w.cells + cell)[tid];
  __syncthreads();
  const CellDev &c = S.cell;
  // nc bounds this cell's loops (the lead cell's is small); ncs is the
  // workspace's per-cell stride
  const int nc = c.nc, ncs = w.nc, cap = w.cap;
  const int per = ((nc + CL * 32 - 1) / (CL * 32)) * 32;
  const int r0 = min(nc, rank * per), r1 = min(nc, r0 + per), nrows = r1 - r0;
  const uint32_t P = (uint32_t)c.nprobe;
  if (timed && tid == 0) w.cta_ts[2 * (cell * CL + rank)] = (long long)t_entry;
  // marks: SM clocks of CTA 0 of cell 0 (Work::phase_ts), or global-timer
  // marks of every CTA of cell 0 after the entry/exit stamps (Work::cta_ts)
  long long *mts = nullptr;
  if (tid == 0 && cell == 0) {
    if (w.phase_ts) mts = rank == 0 ? w.phase_ts : nullptr;
    else if (w.cta_ts) mts = w.cta_ts + 2 * (size_t)w.n_cells * CL + (size_t)rank * 2 * FUSED_MARKS;
  }
  if (tid == 0) S.ms = MarkState{mts, 0, !w.phase_ts};  // (read and written by thread 0 only)
  const Marker mark{&S.ms};
  int *counts = w.counts + cell * NCOUNT;
  mark(M_START);

  // ---------------------------------------------------------------- P0
  // the small inputs first, so that they do not queue behind the slice; all
  // loads are issued before any shared-memory store (the stores could alias
  // the generic source pointers and would otherwise serialise the loads)
  {
    static_assert(PER_MAX == 4 * FT && 4 * D == 2 * FT && PER_MAX / 32 <= FT && D <= FT, "load shapes");
    const uint16_t *qsrc = c.q ? c.q : w.q + ((size_t)slot * 16 + g * 4) * D;
    uint16_t qv[2], rv[4];
    float ks = 0.0f, s4 = 0.0f, fs[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) qv[k] = qsrc[tid + k * FT];
    if (w.q_store && rank == 0 && !lead)  // (host-I/O step: kernels after this one read the device copy)
#pragma unroll
      for (int k = 0; k < 2; ++k) w.q_store[((size_t)slot * 16 + g * 4) * D + tid + k * FT] = qv[k];
    if (tid < D) ks = c.key_scale[tid];
#pragma unroll
    for (int k = 0; k < 4; ++k) rv[k] = tid + k * FT < nrows ? c.resid[r0 + tid + k * FT] : (uint16_t)0;
    if (tid < (nrows >> 5)) s4 = c.coarse_scale4[(r0 >> 5) + tid];
#pragma unroll
    for (int k = 0; k < 2; ++k) fs[k] = tid + k * FT < (nc >> 5) ? c.fine_scale[tid + k * FT] : 0.0f;
    if (tid == 0) {
      // the coarse slice goes out right behind the small loads (the stores
      // below wait for those), with every mbarrier of the step initialised
      for (int k = 0; k < NCHUNK; ++k) mbar_init(&S.mbar[k], 1);
      mbar_init(&S.mb_in, 1);
      mbar_init(&S.mb_res, 1);
      mbar_init(&S.mb_x[0], 1);
      mbar_init(&S.mb_x[1], 1);
      mbar_init(&S.mb_sh, 1);
      mbar_init(&S.mb_pool, 1);
      mbar_init(&S.mb_s2, 1);
      mbar_init(&S.mb_win, 1);
      mbar_init(&S.mb_attn, 1);
      S.ph_in = S.ph_res = S.ph_x = 0;
      S.status = 0;
      mbar_fence_init();
      for (int k = 0; k * SLICE_CHUNK < nrows; ++k) {
        const int rows = min(SLICE_CHUNK, nrows - k * SLICE_CHUNK);
        mbar_expect_tx(&S.mbar[k], (uint32_t)rows * 64u);
        bulk_g2s(S.big + k * SLICE_CHUNK * 64, c.upper + (size_t)(r0 + k * SLICE_CHUNK) * 64, (uint32_t)rows * 64u,
                 &S.mbar[k]);
      }
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) S.sx[tid + k * FT] = bf16f(qv[k]);
    if (tid < D) S.kscale[tid] = ks;
#pragma unroll
    for (int k = 0; k < 4; ++k) S.resid[tid + k * FT] = rv[k];
    if (tid < PER_MAX / 32) S.scale4[tid] = s4;
#pragma unroll
    for (int k = 0; k < 2; ++k) S.fsc[tid + k * FT] = fs[k];
    // the slice's selected-cluster bits, set by whichever CTA scores a survivor (P5)
    if (tid < (nrows >> 5)) w.selbits[(size_t)cell * (ncs >> 5) + (r0 >> 5) + tid] = 0u;
  }
  for (int e = tid; e < 4 * 128; e += FT) S.hist[e] = 0u;  // (P1 adds the coarse first round)
  __syncthreads();
  mark(M_ISSUE);
  static_assert(FW == 16, "12 operand-row warps + 4 norm warps");
  if (warp < 12) {
    // operand row r = warp / 4 of head h = warp % 4, one warp per row; lane l
    // takes dimensions l + 32k (k = 0..7): the row's exponent and its exact
    // digit sum are warp reductions
    const int r = warp >> 2, h = warp & 3;
    float x[8];
    int e = INT_MIN;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int d = lane + 32 * k;
      const float xa = S.sx[h * D + d];
      float v = xa;
      if (r != R_Q) {
        const float prod = __fmul_rn(xa, S.kscale[d]);
        v = r == R_Q15 ? __fmul_rn(bf16f(bf16_rne(__fmul_rn(prod, 0.015625f))), 16.0f)
                       : bf16f(bf16_rne(__fmul_rn(prod, 0.00390625f)));
      }
      x[k] = v;
      e = max(e, v != 0.0f ? ilogbf(v) : INT_MIN);
    }
    const int E = __reduce_max_sync(0xffffffffu, e);
    uint8_t *fb = reinterpret_cast<uint8_t *>(S.frag) + r * FRAG_ROW * 4;
    long long xsum = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int d = lane + 32 * k;
      int X = 0;
      if (E != INT_MIN) {
        const double v = (double)x[k];
        // kept elements are integers on the 2^(E-29) grid, |X| < 2^30
        if (!(fabs(v) < pow2d(E - 22))) X = __double2int_rn(v * pow2d(29 - E));
      }
      xsum += X;
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
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int lane_b = 4 * (4 * (h & 1) + j) + tq;
        fb[(((ks * 2 + nt) * 32 + lane_b) * 2 + reg) * 4 + byte] = (uint8_t)(int8_t)dg[j];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) xsum += __shfl_xor_sync(0xffffffffu, xsum, o);
    if (lane == 0) {
      S.shift[r][h] = E == INT_MIN ? 0 : E - 29;
      S.sxsum[r][h] = xsum;
    }
  } else {
    // lambda*|q| and 3*sum(q) of head warp - 12: pairwise FP64 sums in
    // dimension order
    const int h = warp - 12;
    double v[8], sq[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) { v[j] = (double)S.sx[h * D + 8 * lane + j]; sq[j] = v[j] * v[j]; }
    double a = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
    double b = ((sq[0] + sq[1]) + (sq[2] + sq[3])) + ((sq[4] + sq[5]) + (sq[6] + sq[7]));
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      a = a + __shfl_xor_sync(0xffffffffu, a, o);
      b = b + __shfl_xor_sync(0xffffffffu, b, o);
    }
    if (lane == 0) {
      S.qscal[h] = __fmul_rn(__double2float_rn(__dsqrt_rn(b)), c.lam);
      S.qscal[4 + h] = __fmul_rn(3.0f, __double2float_rn(a));
    }
  }
  __syncthreads();
  mark(M_QEXP);
  mark(M_QPREP);
  // this CTA has started and its mbarriers are initialised (made visible by
  // fence.mbarrier_init above, so the arrive can be relaxed); the matching
  // wait precedes the first push into another CTA (P2)
  cluster_arrive_relaxed();
  __syncthreads();
  mark(M_STARTED);

  // ---------------------------------------------------------------- P1
  {
    BFrag F;
    load_frag(S, R_Q, lane, F);
    const Pow2 scA = pow2s(S.shift[R_Q][hA]), scB = pow2s(S.shift[R_Q][hB]);
    const float qnA = S.qscal[hA], qnB = S.qscal[hB], c3A = S.qscal[4 + hA], c3B = S.qscal[4 + hB];
    const int tiles = nrows >> 4;
    if (tid == 0 && S.ms.ts && tiles > 0) {
      mbar_wait(&S.mbar[(tiles * 16 - 1) / SLICE_CHUNK], 0);
      mark(M_SLICE);
    }
    uint16_t *glo = w.lo + (size_t)cell * G * ncs, *ghi = w.hi + (size_t)cell * G * ncs;
    for (int tile = warp; tile < tiles; tile += FW) {
      if (!mbar_wait(&S.mbar[(tile * 16) / SLICE_CHUNK], 0)) atomicOr(reinterpret_cast<unsigned *>(&S.status), ST_TIMEOUT);
      long long dsum[2];
      tile_dots<0>(S.big + (tile * 16 + gq) * 64, S.big + (tile * 16 + gq + 8) * 64, t, F, dsum);
      const int lr = tile * 16 + gq + ((t & 1) << 3), row = r0 + lr;
      const float sc4 = S.scale4[lr >> 5];
      const float rr = bf16f(S.resid[lr]);
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int h = k ? hB : hA;
        const float dot = exact_to_float(dsum[k], k ? scB : scA);
        const float centered = __fsub_rn(__fmul_rn(2.0f, dot), k ? c3B : c3A);
        const float v = __fmul_rn(centered, sc4);
        const float margin = __fmul_rn(k ? qnB : qnA, rr);
        const uint16_t lo = (uint16_t)ord16(bf16_score(__fsub_rn(v, margin)));
        const uint16_t hi = (uint16_t)ord16(bf16_score(__fadd_rn(v, margin)));
        S.b.c.lo[h][lr] = lo;
        hist_add(S.hist, h, lo >> 8u);  // the coarse selection's first round
        S.b.c.hi[h][lr] = hi;
        if (w.trace) {
          glo[(size_t)h * ncs + row] = lo;
          ghi[(size_t)h * ncs + row] = hi;
        }
      }
    }
  }
  __syncthreads();
  mark(M_COARSE);

  // ---------------------------------------------------------------- P2
  cluster_wait();
  {
    cluster_select(S, nrows, P, 16, true, KEY_COARSE, 0, true);
  }
  uint32_t tco[4];
#pragma unroll
  for (int h = 0; h < 4; ++h) tco[h] = S.ctl.th[h] >> 16;
  if (rank == 0 && tid < 4) w.thr[(size_t)cell * 16 + T_COARSE * G + tid] = S.ctl.th[tid] >> 16;
  mark(M_CSEL);

  // ---------------------------------------------------------------- P3
  int nsurv;
  {
    const int i0 = tid * 4;
    uint32_t m[4];
    int cnt = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = i0 + j;
      m[j] = 0;
      if (i < nrows) {
#pragma unroll
        for (int h = 0; h < 4; ++h) m[j] |= (uint32_t)(S.b.c.hi[h][i] >= tco[h]) << h;
      }
      cnt += m[j] != 0;
    }
    int r = block_exclusive_scan(cnt, &nsurv);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (m[j]) {
        S.sidx[r] = (uint16_t)(i0 + j);
        S.smask[r] = (uint8_t)m[j];
        ++r;
      }
  }
  exchange_send(S, nsurv, 0, 0, 0);
  exchange_wait(S);
  const int surv_base = before(S, 0, rank), nsurv_all = total(S, 0);
  // The Fine work is balanced over the cluster: CTA r scores the survivors at
  // global positions [r L, r L + L), L = ceil(survivors / 16) (positions stay
  // ascending with the rank, as the selection's tie rule needs); every CTA
  // pushes each of its survivors into the slot of the CTA that scores it.
  const int L = max(1, (nsurv_all + CL - 1) / CL);
  const int s0 = min(nsurv_all, rank * L), nsh = min(nsurv_all, s0 + L) - s0;
  for (int k = tid; k < nsurv; k += FT) {
    const int lr = S.sidx[k], p = surv_base + k, d = p / L;
    const uint32_t m = S.smask[k];
    if (w.trace) w.tags[(size_t)cell * ncs + p] = (uint32_t)(r0 + lr) | (m << 28);
    st_async_b32(remote(&S.shin[p - d * L], (uint32_t)d), remote(&S.mb_sh, (uint32_t)d), (uint32_t)(r0 + lr) | (m << 16));
  }
  if (tid == 0) mbar_expect_tx(&S.mb_sh, (uint32_t)nsh * 4u);
  mbar_wait_cluster(&S.mb_sh, 0u, &S.status);
  if (rank == 0 && tid == 0) counts[C_TAGS] = nsurv_all;
  mark(M_SURV);

  // ---------------------------------------------------------------- P4
  {
    BFrag F;
    load_frag(S, R_Q, lane, F);
    const Pow2 scA = pow2s(S.shift[R_Q][hA]), scB = pow2s(S.shift[R_Q][hB]);
    for (int b0 = 0; b0 < nsh; b0 += BATCH_FINE) {
      const int nb = min(BATCH_FINE, nsh - b0);
      __syncthreads();
      for (int q = tid; q < nb * 8; q += FT) {
        const int rr = q >> 3, part = q & 7, cid = (int)(S.shin[b0 + rr] & 0xffffu);
        const uint8_t *src = (part < 4 ? c.upper : c.lower) + (size_t)cid * 64 + (part & 3) * 16;
        cp16(S.big + rr * STRIDE_FINE + part * 16, src);
      }
      // the share's CSR ranges travel with the rows (P5 lists the selected
      // clusters from them without a dependent global load): start into
      // S.offs, length into S.resid (free since P1; a length that does not
      // fit 16 bits is marked 0xffff and read again in P5)
      static_assert(BATCH_FINE <= 2 * FT, "two share survivors per thread");
      int cb[2] = {0, 0}, ce[2] = {0, 0};
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int k = tid + j * FT;
        if (k < nb) {
          const int cid = (int)(S.shin[b0 + k] & 0xffffu);
          cb[j] = __ldg(c.offsets + cid);
          ce[j] = __ldg(c.offsets + cid + 1);
        }
      }
      cp_wait_all();
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int k = tid + j * FT;
        if (k < nb) {
          S.offs[b0 + k] = cb[j];
          S.resid[b0 + k] = (uint16_t)min(ce[j] - cb[j], 0xffff);
        }
      }
      __syncthreads();
      if (b0 == 0) mark(M_FGATHER);
      const int tiles = (nb + 15) >> 4;
      for (int tile = warp; tile < tiles; tile += FW) {
        const int rg = tile * 16 + gq, r8 = rg + 8;
        long long dsum[2];
        tile_dots<1>(S.big + min(rg, nb - 1) * STRIDE_FINE, S.big + min(r8, nb - 1) * STRIDE_FINE, t, F, dsum);
        dsum[0] = 2 * dsum[0] - 15 * S.sxsum[R_Q][hA];  // weights 2*c4 - 15
        dsum[1] = 2 * dsum[1] - 15 * S.sxsum[R_Q][hB];
        const int row = (t & 1) ? r8 : rg;
        if (row < nb) {
          const int k = b0 + row, sv = (int)S.shin[k], cid = sv & 0xffff, mk = (sv >> 16) & 15, pos = s0 + k;
          const float fs = S.fsc[cid >> 5];
#pragma unroll
          for (int kk = 0; kk < 2; ++kk) {
            const int h = kk ? hB : hA;
            uint32_t key = 0;
            if ((mk >> h) & 1)
              key = ord_fused(bf16_score(__fmul_rn(exact_to_float(dsum[kk], kk ? scB : scA), fs)), (uint32_t)pos);
            S.b.fkey[h][k] = key;
            if (key) hist_add(S.hist, h, key >> 24);  // the Fine selection's first round
          }
        }
      }
      __syncthreads();
    }
  }
  mark(M_FINE);

  // ---------------------------------------------------------------- P5
  {
    cluster_select(S, nsh, P, 32, false, KEY_FINE, 0, true);
  }
  mark(M_FSEL);
  uint32_t st = 0;
  {
    uint32_t tf[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      tf[h] = S.ctl.th[h];
      if (tf[h] == 0u) { tf[h] = 0xffffffffu; st |= ST_FINE_SHORT; }
    }
    if (tid < 4 && S.ctl.own[tid])
      w.thr[(size_t)cell * 16 + T_FINE * G + tid] = S.ctl.th[tid] ? S.ctl.th[tid] : 0xffffffffu;
    uint32_t *selbits = w.selbits + (size_t)cell * (ncs >> 5);
    for (int k = tid; k < nsh; k += FT) {
      bool s = false;
#pragma unroll
      for (int h = 0; h < 4; ++h) s |= S.b.fkey[h][k] >= tf[h];
      if (s) {
        const uint32_t cid = S.shin[k] & 0xffffu;
        S.shin[k] |= 1u << 24;
        atomicOr(selbits + (cid >> 5), 1u << (cid & 31));
        // the cluster's postings and mates into L2 for P6 (only selected
        // clusters: prefetching every survivor's lists read ~2 MB per step
        // that no stage used)
        const int b = S.offs[k], n = S.resid[k];
        if (n > 0) {
          prefetch_l2(c.values + b);
          prefetch_l2(c.mates + b);
          if (((b * 4) >> 7) != (((b + n - 1) * 4) >> 7)) {
            prefetch_l2(c.values + b + n - 1);
            prefetch_l2(c.mates + b + n - 1);
          }
        }
      }
    }
    __syncthreads();  // selected flags complete
  }
  // selected clusters in ascending order with their posting ranges
  int nsel, npost;
  {
    const int i0 = tid * 4;
    int f[4], cnt = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      f[j] = (i0 + j < nsh) && ((S.shin[i0 + j] >> 24) & 1u);
      cnt += f[j];
    }
    int r = block_exclusive_scan(cnt, &nsel);  // (all reads of fkey precede this barrier)
    int len[4], psum = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      len[j] = 0;
      if (f[j]) {
        const int cid = (int)(S.shin[i0 + j] & 0xffffu);
        const int b = S.offs[i0 + j];  // (P4)
        len[j] = S.resid[i0 + j] < 0xffffu ? (int)S.resid[i0 + j] : __ldg(c.offsets + cid + 1) - b;
        S.b.s.slist[r] = (uint16_t)cid;
        S.b.s.soff[r] = b;
        psum += len[j];
        ++r;
      }
    }
    int pr = block_exclusive_scan(psum, &npost);
    r -= cnt;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (f[j]) { S.b.s.ppre[r++] = pr; pr += len[j]; }
    if (tid == 0) S.b.s.ppre[nsel] = npost;
  }
  mark(M_SELLIST);
  exchange_send(S, nsel, npost, 0, 0);  // (also orders the selected bits before the mate rule reads them)
  // this CTA's postings (their clusters, mates and tokens) load while the
  // counts travel; the mate rule, which reads every CTA's selected bits, runs
  // after the wait (one pass covers up to 4 * FT postings)
  auto posting = [&](int p, int &jj, int &cid) {
    jj = -1;
    cid = 0;
    if (p < npost) {
      int lo = 0, hi = nsel - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (S.b.s.ppre[mid] <= p) lo = mid; else hi = mid - 1;
      }
      cid = S.b.s.slist[lo];
      jj = S.b.s.soff[lo] + (p - S.b.s.ppre[lo]);
    }
  };
  int pj[4], pc_[4], pm[4], pt[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    posting(tid * 4 + j, pj[j], pc_[j]);
    pm[j] = pj[j] >= 0 ? c.mates[pj[j]] : -1;
    pt[j] = pj[j] >= 0 ? c.values[pj[j]] : 0;
  }
  exchange_wait(S);
  const int sel_base = before(S, 0, rank), nsel_all = total(S, 0), npost_all = total(S, 1);
  if (w.trace)
    for (int k = tid; k < nsel; k += FT)
      if (sel_base + k < SEL_MAX) w.sel[(size_t)cell * SEL_MAX + sel_base + k] = S.b.s.slist[k];
  mark(M_SELX);

  // ---------------------------------------------------------------- P6
  int nkept = 0;
  {
    int *klist = reinterpret_cast<int *>(S.big);
    const uint32_t *selbits = w.selbits + (size_t)cell * (ncs >> 5);
    for (int p0 = 0; p0 < npost; p0 += FT * 4) {
      int jj[4], cid[4], mate[4], tok[4], keep[4];
      if (p0 == 0) {
#pragma unroll
        for (int j = 0; j < 4; ++j) { jj[j] = pj[j]; cid[j] = pc_[j]; mate[j] = pm[j]; tok[j] = pt[j]; }
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          posting(p0 + tid * 4 + j, jj[j], cid[j]);
          mate[j] = jj[j] >= 0 ? c.mates[jj[j]] : -1;
          tok[j] = jj[j] >= 0 ? c.values[jj[j]] : 0;
        }
      }
      int cnt = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const bool dup = mate[j] >= 0 && mate[j] < cid[j] && ((__ldcg(selbits + (mate[j] >> 5)) >> (mate[j] & 31)) & 1u);
        keep[j] = jj[j] >= 0 && !dup;
        cnt += keep[j];
      }
      int tot;
      int r = nkept + block_exclusive_scan(cnt, &tot);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (keep[j]) {
          if (r < KMAX) klist[r] = tok[j];
          ++r;
        }
      nkept += tot;
    }
  }
  mark(M_KEEP);
  exchange(S, nkept, 0, 0, 0);
  const int kept_base = before(S, 0, rank), npool = total(S, 0);
  // P7's balanced shares of the pool positions: every kept token goes into
  // the Stage-1.5 token slot of the CTA that scores its position
  const int n15 = min(npool, cap);
  const int pc = ((n15 + CL * 32 - 1) / (CL * 32)) * 32;
  const int q0 = min(n15, rank * pc), m15 = min(n15, q0 + pc) - q0;
  {
    const int *klist = reinterpret_cast<const int *>(S.big);
    int32_t *pool = w.pool + (size_t)cell * cap;
    for (int k = tid; k < nkept && k < KMAX; k += FT) {
      const int p = kept_base + k;
      if (w.trace && p < cap) pool[p] = klist[k];
      if (p < n15) {
        const int d = p / pc;
        st_async_b32(remote(&S.b.p.tok[p - d * pc], (uint32_t)d), remote(&S.mb_pool, (uint32_t)d), (uint32_t)klist[k]);
      }
    }
  }
  if (npool > cap) st |= ST_POOL_OVER;
  if (npool < M15_MIN) st |= ST_POOL_UNDER;
  if (rank == 0 && tid == 0) {
    counts[C_POOL] = npool;
    counts[C_SEL] = min(nsel_all, SEL_MAX);
    counts[C_POSTINGS] = npost_all;
    counts[C_STATUS] = (int)st;
  }
  if (tid == 0) mbar_expect_tx(&S.mb_pool, (uint32_t)m15 * 4u);
  mbar_wait_cluster(&S.mb_pool, 0u, &S.status);
  mark(M_POOL);

  // ---------------------------------------------------------------- P7
  // Stage-1.5 and 1.6 scores of a balanced share of the pool positions,
  // from one gather of their prefix2 | residual2 rows.  The 1.6 selection
  // breaks ties by the lower union position, which orders members like
  // their pool position does, so its keys carry the pool position and the
  // rows need no second gather.
  {
    static_assert(POS_MAX == 2 * FT, "two pool positions per thread");
    for (int b0 = 0; b0 < m15; b0 += BATCH_FINE) {
      const int nb = min(BATCH_FINE, m15 - b0);
      __syncthreads();
      for (int q = tid; q < nb * 8; q += FT) {
        const int rr = q >> 3, part = q & 7;
        const int tok = S.b.p.tok[b0 + rr];
        cp16(S.big + rr * STRIDE_FINE + part * 16, (part < 4 ? c.prefix2 : c.residual2) + (size_t)tok * 64 + (part & 3) * 16);
      }
      cp_wait_all();
      __syncthreads();
      if (b0 == 0) mark(M_S15G);
      const int tiles = (nb + 15) >> 4;
      {
        BFrag F;
        load_frag(S, R_Q15, lane, F);
        const Pow2 scA = pow2s(S.shift[R_Q15][hA]), scB = pow2s(S.shift[R_Q15][hB]);
        for (int tile = warp; tile < tiles; tile += FW) {
          const int rg = tile * 16 + gq, r8 = rg + 8;
          long long dsum[2];
          tile_dots<0>(S.big + min(rg, nb - 1) * STRIDE_FINE, S.big + min(r8, nb - 1) * STRIDE_FINE, t, F, dsum);
          dsum[0] = 2 * dsum[0] - 3 * S.sxsum[R_Q15][hA];  // weights 2p - 3
          dsum[1] = 2 * dsum[1] - 3 * S.sxsum[R_Q15][hB];
          const int row = (t & 1) ? r8 : rg;
          if (row < nb) {
#pragma unroll
            for (int k = 0; k < 2; ++k) {
              const uint32_t sc = ord16(bf16_score(exact_to_float(dsum[k], k ? scB : scA)));
              S.b.p.sc15[k ? hB : hA][b0 + row] = (uint16_t)sc;
              hist_add(S.hist, k ? hB : hA, sc >> 8);  // the Stage-1.5 selection's first round
            }
          }
        }
      }
      if (m15 > BATCH_FINE) {
        // the share spans several staging batches: Stage-1.6 scores of every
        // position now (a single batch keeps its rows, and P8 scores only
        // the union members)
        BFrag F;
        load_frag(S, R_QS, lane, F);
        const Pow2 s16A = pow2s(S.shift[R_QS][hA] + 4), s16B = pow2s(S.shift[R_QS][hB] + 4);
        for (int tile = warp; tile < tiles; tile += FW) {
          const int rg = tile * 16 + gq, r8 = rg + 8;
          long long dh[2];
          tile_dots<1>(S.big + min(rg, nb - 1) * STRIDE_FINE, S.big + min(r8, nb - 1) * STRIDE_FINE, t, F, dh);
          const int row = (t & 1) ? r8 : rg;
          if (row < nb) {
#pragma unroll
            for (int k = 0; k < 2; ++k) {
              const int h = k ? hB : hA;
              // operand 16*qs, weights 2*c4 - 15: the same digits, scale 2^4 higher
              S.b.p.sc16[h][b0 + row] = (uint16_t)ord16(
                  bf16_score(exact_to_float(2 * dh[k] - 15 * S.sxsum[R_QS][h], k ? s16B : s16A)));
            }
          }
        }
      }
      __syncthreads();
    }
  }
  mark(M_S15);

  // ---------------------------------------------------------------- P8
  {
    cluster_select(S, m15, (uint32_t)min(UNION15, n15), 32, false, KEY_S15, q0, true);
  }
  mark(M_S15SEL);
  int nu;
  {
    uint32_t tu[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) tu[h] = S.ctl.th[h] ? S.ctl.th[h] : 0xffffffffu;
    if (tid < 4 && S.ctl.own[tid])
      w.thr[(size_t)cell * 16 + T_S15 * G + tid] = S.ctl.th[tid] ? S.ctl.th[tid] : 0xffffffffu;
    const int i0 = tid * 2;
    int f[2], cnt = 0;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int i = i0 + j;
      f[j] = 0;
      if (i < m15) {
        const uint32_t lowk = 0xffffu - (uint32_t)(q0 + i);
#pragma unroll
        for (int h = 0; h < 4; ++h) f[j] |= (((uint32_t)S.b.p.sc15[h][i] << 16) | lowk) >= tu[h];
      }
      cnt += f[j];
    }
    int r = block_exclusive_scan(cnt, &nu);
#pragma unroll
    for (int j = 0; j < 2; ++j)
      if (i0 + j < m15) {
        S.b.p.flag[i0 + j] = (uint8_t)f[j];
        S.b.p.urank[i0 + j] = (uint16_t)r;
        r += f[j];
      }
  }
  exchange_send(S, nu, 0, 0, 0);
  if (m15 <= BATCH_FINE && nu > 0) {
    // Stage-1.6 scores of this CTA's union members only, from the rows P7
    // left in the staging area (row i at i * STRIDE_FINE), while the union
    // counts travel; members listed in union order in clist (free until P10)
    for (int i = tid; i < m15; i += FT)
      if (S.b.p.flag[i]) S.b.p.clist[S.b.p.urank[i]] = (uint16_t)i;
    __syncthreads();
    BFrag F;
    load_frag(S, R_QS, lane, F);
    const Pow2 s16A = pow2s(S.shift[R_QS][hA] + 4), s16B = pow2s(S.shift[R_QS][hB] + 4);
    const int tiles = (nu + 15) >> 4;
    for (int tile = warp; tile < tiles; tile += FW) {
      const int rg = tile * 16 + gq, r8 = rg + 8;
      long long dh[2];
      tile_dots<1>(S.big + S.b.p.clist[min(rg, nu - 1)] * STRIDE_FINE,
                   S.big + S.b.p.clist[min(r8, nu - 1)] * STRIDE_FINE, t, F, dh);
      const int row = (t & 1) ? r8 : rg;
      if (row < nu) {
        const int i = S.b.p.clist[row];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const int h = k ? hB : hA;
          // operand 16*qs, weights 2*c4 - 15: the same digits, scale 2^4 higher
          S.b.p.sc16[h][i] = (uint16_t)ord16(
              bf16_score(exact_to_float(2 * dh[k] - 15 * S.sxsum[R_QS][h], k ? s16B : s16A)));
        }
      }
    }
  }
  exchange_wait(S);
  const int u_base = before(S, 0, rank), nu_all = min(total(S, 0), U15_MAX);
  for (int i = tid; i < m15 && w.trace; i += FT) {
    if (!S.b.p.flag[i]) continue;
    const int u = u_base + S.b.p.urank[i];
    if (u < U15_MAX) {
      w.u15pos[(size_t)cell * U15_MAX + u] = q0 + i;
      w.u15tok[(size_t)cell * U15_MAX + u] = S.b.p.tok[i];
    }
  }
  if (rank == 0 && tid == 0) counts[C_U15] = nu_all;
  mark(M_U15);

  // ---------------------------------------------------------------- P9
  {
    cluster_select(S, m15, (uint32_t)min(M16, nu_all), 32, false, KEY_S16, q0);
  }
  mark(M_S16SEL);
  int ncl;
  {
    uint32_t tc[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) tc[h] = S.ctl.th[h] ? S.ctl.th[h] : 0xffffffffu;
    if (tid < 4 && S.ctl.own[tid])
      w.thr[(size_t)cell * 16 + T_S16 * G + tid] = S.ctl.th[tid] ? S.ctl.th[tid] : 0xffffffffu;
    const int i0 = tid * 2;
    int f[2], cnt = 0;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int i = i0 + j;
      f[j] = 0;
      if (i < m15 && S.b.p.flag[i]) {
        const uint32_t lowk = 0xffffu - (uint32_t)(q0 + i);
#pragma unroll
        for (int h = 0; h < 4; ++h) f[j] |= (((uint32_t)S.b.p.sc16[h][i] << 16) | lowk) >= tc[h];
      }
      cnt += f[j];
    }
    int r = block_exclusive_scan(cnt, &ncl);
#pragma unroll
    for (int j = 0; j < 2; ++j)
      if (f[j]) S.b.p.clist[r++] = (uint16_t)(i0 + j);
  }
  exchange_send(S, ncl, 0, 0, 0);
  // the first batch of the candidates' Stage-II rows goes out while the
  // candidate counts travel
  auto s2_gather = [&](int b0, int nb) {
    for (int q = tid; q < nb * 16; q += FT) {
      const int rr = q >> 4, part = q & 15;
      const int tok = S.b.p.tok[S.b.p.clist[b0 + rr]];
      const uint8_t *src = part < 4   ? c.prefix2 + (size_t)tok * 64 + part * 16
                           : part < 8 ? c.residual2 + (size_t)tok * 64 + (part - 4) * 16
                                      : c.residual4 + (size_t)tok * 128 + (part - 8) * 16;
      cp16(S.big + rr * STRIDE_S2 + part * 16, src);
    }
  };
  s2_gather(0, min(BATCH_S2, ncl));
  exchange_wait(S);
  const int c_base = before(S, 0, rank), ncand = min(total(S, 0), CAND_MAX);
  if (rank == 0 && tid == 0) counts[C_CAND] = ncand;
  // candidates: their union position; their Stage-II keys (8-bit scores of
  // a small gather) and tokens for head h are pushed to CTA h (slot =
  // candidate rank, asynchronous stores completing CTA h's mb_s2), into the
  // Stage-1.5 score area, which every CTA is done with once the candidate
  // exchange has completed
  uint32_t *k2 = reinterpret_cast<uint32_t *>(&S.b.p.sc15[0][0]);
  int *t2 = reinterpret_cast<int *>(&S.b.p.sc15[0][0]) + CAND_MAX;
  for (int k = tid; k < ncl; k += FT) {
    const int cr = c_base + k;
    if (cr >= CAND_MAX) break;
    const int i = S.b.p.clist[k];
    if (w.trace) w.cand[(size_t)cell * CAND_MAX + cr] = u_base + S.b.p.urank[i];
  }
  {
    BFrag F;
    load_frag(S, R_QS, lane, F);
    const Pow2 s2A = pow2s(S.shift[R_QS][hA]), s2B = pow2s(S.shift[R_QS][hB]);
    for (int b0 = 0; b0 < ncl; b0 += BATCH_S2) {
      const int nb = min(BATCH_S2, ncl - b0);
      if (b0 > 0) {
        __syncthreads();
        s2_gather(b0, nb);
      }
      cp_wait_all();
      __syncthreads();
      const int tiles = (nb + 15) >> 4;
      for (int tile = warp; tile < tiles; tile += FW) {
        const int rg = tile * 16 + gq, r8 = rg + 8;
        long long dh[2], dl[2];
        tile_dots_8bit(S.big + min(rg, nb - 1) * STRIDE_S2, S.big + min(r8, nb - 1) * STRIDE_S2, t, F, dh, dl);
        const int row = (t & 1) ? r8 : rg, cr = c_base + b0 + row;
        if (row < nb && cr < CAND_MAX) {
          const int i = S.b.p.clist[b0 + row];
          const uint32_t u = (uint32_t)(u_base + S.b.p.urank[i]);
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const int h = k ? hB : hA;
            // weights 2*code8 - 255 = 16*(2*c4 - 15) + (2*r4 - 15)
            const long long dsum = 32 * dh[k] + 2 * dl[k] - 255 * S.sxsum[R_QS][h];
            const uint32_t key = (ord16(bf16_score(exact_to_float(dsum, k ? s2B : s2A))) << 16) | (0xffffu - u);
            st_async_b32(remote(k2 + cr, (uint32_t)h), remote(&S.mb_s2, (uint32_t)h), key);
            st_async_b32(remote(t2 + cr, (uint32_t)h), remote(&S.mb_s2, (uint32_t)h), (uint32_t)S.b.p.tok[i]);
          }
        }
      }
    }
  }
  mark(M_S2);

  // --------------------------------------------------------------- P12
  if (rank < G) {
    // exact top-100 of head h in rank order: block radix select over the
    // (at most 1024) candidate keys held two per thread, then ranks
    const int h = rank;
    uint32_t *wkey = reinterpret_cast<uint32_t *>(S.big);
    int *widx = reinterpret_cast<int *>(S.big) + TOPK;
    int *wtok = reinterpret_cast<int *>(S.big) + 2 * TOPK;
    if (tid == 0) mbar_expect_tx(&S.mb_s2, (uint32_t)ncand * 8u);
    mbar_wait_cluster(&S.mb_s2, 0u, &S.status);
    const uint32_t v[2] = {tid < ncand ? k2[tid] : 0u, tid + FT < ncand ? k2[tid + FT] : 0u};
    const uint32_t K = (uint32_t)min(TOPK, ncand);
    uint32_t prefix = 0, mask = 0, krem = K;
    if (tid == 0) { S.n_win = 0; S.ctl.done[0] = K == 0; }
    for (int sh = 24; sh >= 0; sh -= 8) {
      __syncthreads();
      if (S.ctl.done[0]) break;
      for (int e = tid; e < 256; e += FT) S.hist[e] = 0;
      __syncthreads();
#pragma unroll
      for (int r = 0; r < 2; ++r)
        if (v[r] != 0u && (v[r] & mask) == prefix) atomicAdd(&S.hist[(v[r] >> sh) & 255u], 1u);
      __syncthreads();
      if (warp == 0) {
        int bin;
        uint32_t above;
        warp_find_desc(S.hist, krem, lane, bin, above);
        if (lane == 0) {
          S.ctl.prefix[0] = prefix | ((uint32_t)bin << sh);
          S.ctl.krem[0] = krem - above;
          S.ctl.done[0] = sh == 0 || S.hist[bin] == krem - above;
        }
      }
      __syncthreads();
      prefix = S.ctl.prefix[0];
      krem = S.ctl.krem[0];
      mask |= 255u << sh;
    }
    // keys are distinct and non-zero: exactly K of them are >= prefix
    const uint32_t th = K ? prefix : 0xffffffffu;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int slot = warp_claim(&S.n_win, v[r] != 0u && v[r] >= th);
      if (slot >= 0 && slot < TOPK) { wkey[slot] = v[r]; widx[slot] = tid + r * FT; }
    }
    __syncthreads();
    const int m = min(S.n_win, TOPK);
    int32_t *fpos = w.final_pos + ((size_t)cell * G + h) * TOPK;
    int32_t *fids = w.final_ids + ((size_t)cell * G + h) * TOPK;
    uint32_t *fkeys = w.final_keys + ((size_t)cell * G + h) * TOPK;
    if (tid < m) {
      const uint32_t key = wkey[tid];
      int rk = 0;
      for (int j = 0; j < m; ++j) rk += wkey[j] > key;
      fpos[rk] = (int)(0xffffu - (key & 0xffffu));
      fids[rk] = t2[widx[tid]];
      fkeys[rk] = key;
      wtok[rk] = t2[widx[tid]];
    } else if (tid < TOPK) {
      // fewer than 100 candidates: a failed step the status word reports
      fpos[tid] = -1;
      fids[tid] = 0;
      fkeys[tid] = 0u;
      wtok[tid] = 0;
    }
    if (w.link && !lead) {
      shard_lists(w, S, cell, h, fkeys, fids);
    } else {
      // head h's winners, in rank order, into every CTA's S.win[h]
      __syncthreads();
      if (tid < CL * (TOPK / 4)) {
        const int d = tid / (TOPK / 4), q = tid - d * (TOPK / 4);
        const uint4 v = make_uint4((uint32_t)wtok[4 * q], (uint32_t)wtok[4 * q + 1], (uint32_t)wtok[4 * q + 2],
                                   (uint32_t)wtok[4 * q + 3]);
        st_async_v4(remote(&S.win[h][4 * q], (uint32_t)d), remote(&S.mb_win, (uint32_t)d), v);
      }
    }
  }
  // --------------------------------------------------------------- P13
  // (the block closes after the combine below)
  const ShardLinkDev *Lk = lead ? nullptr : w.link;
  const int sink = Lk ? Lk->sink : w.sink, local = Lk ? Lk->local : w.local;
  const int T = Lk ? Lk->total : (c.context ? c.context : context_of(w));
  const int dense = sink + local;
  const float qscale = 0.0625f * 1.4426950408889634f;  // 1/sqrt(256), log2(e)
  float qv[G][8];
#pragma unroll
  for (int h = 0; h < G; ++h)
#pragma unroll
    for (int e = 0; e < 8; ++e) qv[h][e] = S.sx[h * D + 8 * lane + e] * qscale;
  float m[G], l[G], o[G][8];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; ++e) o[h][e] = 0.0f;
  }
  // the records of up to SB of a warp's items are copied into its staging
  // slots together (cp.async, one memory latency per batch rather than one per
  // item) and folded in order; lane j names item j (token, head: -1 for a
  // dense key shared by the four heads, -2 for none)
  constexpr int SB = 4;
  static_assert(88 * 1024 + FW * SB * REC <= BIG, "attention staging fits the staging area");
  uint8_t *stg = S.big + 88 * 1024 + warp * SB * REC;  // clear of ao/am/al, part and pin
  auto fold = [&](int nmine, int my_tok, int my_head) {
#pragma unroll 1
    for (int j0 = 0; j0 < nmine; j0 += SB) {
      const int nb = min(SB, nmine - j0);
#pragma unroll 1
      for (int u = 0; u < nb; ++u) {
        const int tok = __shfl_sync(0xffffffffu, my_tok, j0 + u);
        const uint8_t *rec;
        if (Lk) {
          // sharded: the record lives in the owning shard's memory (plain
          // loads over NVLink)
          int s = 0;
          while (s + 1 < Lk->n_shards && Lk->begin[s + 1] <= tok) ++s;
          rec = Lk->kv8[s][cell] + (size_t)(tok - Lk->begin[s]) * REC;
        } else {
          rec = c.kv8 + (size_t)tok * REC;
        }
        cp16(stg + u * REC + 16 * lane, rec + 16 * lane);
      }
      cp_wait_all();
      __syncwarp();
#pragma unroll 1
      for (int u = 0; u < nb; ++u) {
        const int head = __shfl_sync(0xffffffffu, my_head, j0 + u);
        if (head == -2) continue;  // (warp-uniform)
        const uint2 kb = *reinterpret_cast<const uint2 *>(stg + u * REC + 8 * lane);
        const uint2 vb = *reinterpret_cast<const uint2 *>(stg + u * REC + 256 + 8 * lane);
        float kf[8], vf[8];
        fp8x8(kb, kf);
        fp8x8(vb, vf);
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
      __syncwarp();  // the slots are read before the next batch lands
    }
  };
  auto dense_tok = [&](int it) { return it < sink ? it : T - local + (it - sink); };
  // the dense zones (sink and local window) need no winners: CTAs G.. fold
  // them while CTAs 0..G-1 select the top-100 (when the zones are small
  // enough for that split to be balanced); a warp's items go 32 at a time
  const int nwa = (CL - G) * FW;
  const bool early = dense <= nwa * 32;
  __syncthreads();  // every warp is done with its Stage-II rows in the staging area (stg lies above them)
  if (early && rank >= G) {
    const int gwa = (rank - G) * FW + warp;
    const int na = gwa < dense ? (dense - gwa + nwa - 1) / nwa : 0;
    for (int c0 = 0; c0 < na; c0 += 32) {
      const int nb = min(32, na - c0);
      fold(nb, lane < nb ? dense_tok(gwa + (c0 + lane) * nwa) : 0, -1);
    }
  }
  // the step's winners (the group's merged ones when sequence-sharded) in S.win
  if (tid == 0) mbar_expect_tx(&S.mb_win, G * TOPK * 4);
  if (Lk)
    mbar_wait_cluster_until(&S.mb_win, 0u, &S.status, global_ns() + WIN_WAIT_NS);
  else
    mbar_wait_cluster(&S.mb_win, 0u, &S.status);
  mark(M_S2SEL);
  {
    // the winners over all warps (and the dense zones too when they were
    // not folded early): items gw, gw + nw, ...
    const int nw = CL * FW, gw = rank * FW + warp;
    const int first = early ? dense : 0;
    const int nitems = dense + G * TOPK - first;
    const int nmine = gw < nitems ? (nitems - gw + nw - 1) / nw : 0;
    for (int c0 = 0; c0 < nmine; c0 += 32) {
      const int nb = min(32, nmine - c0);
      int my_tok = 0, my_head = -1;
      if (lane < nb) {
        const int it = first + gw + (c0 + lane) * nw;
        if (it < dense) {
          my_tok = dense_tok(it);
        } else {
          const int r = it - dense;
          my_head = r / TOPK;
          my_tok = S.win[r / TOPK][r - (r / TOPK) * TOPK];
          // -1: fewer than 100 in the group (sharded); any other value outside
          // the layer only after a wait for the winners ran out (ST_TIMEOUT,
          // S.win not written this step): no record is read for either
          if ((unsigned)my_tok >= (unsigned)T) { my_tok = 0; my_head = -2; }
        }
      }
      fold(nb, my_tok, my_head);
    }
    mark(M_ATTN_ITEMS);
    // warps -> CTA partial per head
    float *ao = reinterpret_cast<float *>(S.big);   // [FW][G][D]
    float *am = ao + FW * G * D;                     // [G][FW]
    float *al = am + G * FW;                         // [G][FW]
    float *part = reinterpret_cast<float *>(S.big + 72 * 1024);  // [G][PART]: m, l, -, -, o[D]
#pragma unroll
    for (int h = 0; h < G; ++h) {
      if (lane == 0) { am[h * FW + warp] = m[h]; al[h * FW + warp] = l[h]; }
#pragma unroll
      for (int e = 0; e < 8; ++e) ao[(warp * G + h) * D + 8 * lane + e] = o[h][e];
    }
    __syncthreads();
    {
      const int h = tid >> 7, d2 = (tid & 127) * 2;
      float M = -INFINITY;
      for (int k = 0; k < FW; ++k) M = fmaxf(M, am[h * FW + k]);
      float L = 0.0f, O0 = 0.0f, O1 = 0.0f;
      if (M != -INFINITY)
        for (int k = 0; k < FW; ++k) {
          const float mk = am[h * FW + k];
          if (mk == -INFINITY) continue;
          const float e = exp2f(mk - M);
          L += al[h * FW + k] * e;
          O0 += ao[(k * G + h) * D + d2] * e;
          O1 += ao[(k * G + h) * D + d2 + 1] * e;
        }
      part[h * PART + 4 + d2] = O0;
      part[h * PART + 4 + d2 + 1] = O1;
      if ((tid & 127) == 0) { part[h * PART] = M; part[h * PART + 1] = L; }
    }
    __syncthreads();
    // this CTA's (m, l) and 16 output dimensions of each head to the CTA that
    // finishes those dimensions (320 bytes each, asynchronous stores into its
    // staging area, which every CTA is done gathering into by now)
    float *pin = reinterpret_cast<float *>(S.big + 80 * 1024);  // [source CTA][head][20]: m, l, -, -, o[16]
    if (tid < CL * G * 5) {
      const int d = tid / (G * 5), hh = (tid / 5) % G, ch = tid % 5;
      const float *src = ch == 0 ? part + hh * PART : part + hh * PART + 4 + 16 * d + 4 * (ch - 1);
      const uint4 v = make_uint4(__float_as_uint(src[0]), __float_as_uint(src[1]), ch ? __float_as_uint(src[2]) : 0u,
                                 ch ? __float_as_uint(src[3]) : 0u);
      st_async_v4(remote(pin + (rank * G + hh) * 20 + 4 * ch, (uint32_t)d), remote(&S.mb_attn, (uint32_t)d), v);
    }
    if (tid == 0) mbar_expect_tx(&S.mb_attn, CL * G * 5 * 16);
    mbar_wait_cluster(&S.mb_attn, 0u, &S.status);
    mark(M_ATTN_CTA);
    // CTA `rank` finishes output dimensions [16 rank, 16 rank + 16) of the four heads
    float M = -INFINITY, L = 0.0f, O = 0.0f;
    if (tid < G * 16) {
      const int h = tid >> 4, d = 16 * rank + (tid & 15);
      // the 16 CTA partials, then the log-sum-exp merge (log2 domain)
      float ms[CL], ls[CL], os[CL];
#pragma unroll
      for (int r = 0; r < CL; ++r) {
        ms[r] = pin[(r * G + h) * 20];
        ls[r] = pin[(r * G + h) * 20 + 1];
        os[r] = pin[(r * G + h) * 20 + 4 + (d - 16 * rank)];
      }
#pragma unroll
      for (int r = 0; r < CL; ++r) M = fmaxf(M, ms[r]);
#pragma unroll
      for (int r = 0; r < CL; ++r) {
        if (ms[r] == -INFINITY) continue;
        const float e = exp2f(ms[r] - M);
        L += ls[r] * e;
        O += os[r] * e;
      }
      if (!lead) {
        // (a host-I/O step also writes the mapped pinned copy; the device
        // output stays current for borrowed device views)
        const size_t o = ((size_t)slot * 16 + g * 4 + h) * D + d;
        const uint16_t y = bf16_rne(O / L);
        w.out[o] = y;
        if (w.out_host) w.out_host[o] = y;
      }
    }
  }
  mark(M_ATTN);
  if (tid == 0 && S.status) atomicOr(reinterpret_cast<unsigned *>(counts + C_STATUS), (unsigned)S.status);
  cluster_sync();  // no CTA leaves while its shared memory may still be read
  // host-I/O step: the cell's counters (every CTA's status is in by now) to
  // mapped pinned memory, plain stores
  if (w.counts_host && !lead && rank == 0 && tid < NCOUNT)
    w.counts_host[(size_t)cell * NCOUNT + tid] = __ldcg(counts + tid);
  if (w.link && !lead && rank == 0 && tid == 0) {
    // the last cluster of the step to finish advances the group's step
    // counter (every cluster read it in P12, before this barrier)
    const ShardLinkDev *Lk = w.link;
    if (atomicAdd(Lk->exits, 1u) == (uint32_t)w.n_cells - 1u) {
      *Lk->exits = 0u;
      *Lk->epoch += 1u;
    }
  }
  if (timed && tid == 0) w.cta_ts[2 * (cell * CL + rank) + 1] = (long long)global_ns();
}

const char *const kMarkNames[M_NTAGS] = {
    "start", "issue", "qprep_exponents", "qprep", "cluster_start", "slice_landed", "coarse",
    "select_histogram", "select_reduce", "select_result", "coarse_select", "survivors",
    "fine_gather", "fine", "fine_select", "selected_list", "selected_exchange", "pool_keep", "pool",
    "s15_gather", "s15_score", "s15_select", "u15_union", "s16_score", "s16_select", "candidates",
    "s2_score", "s2_select", "attn_items", "attn_cta", "attention", "shard_list_exchange"};

}  // namespace

bool fused_supported(const Work &w) {
  return w.nc % 32 == 0 && w.nc <= CL * PER_MAX && w.cap <= CL * POS_MAX && w.cap % 32 == 0;
}

cudaError_t prepare_fused_attributes() {
  cudaError_t e = cudaFuncSetAttribute(k_funnel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(k_funnel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
}

cudaError_t launch_fused(const Work &w, cudaStream_t st, const cudaAccessPolicyWindow *win) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(CL, w.n_cells + w.lead, 1);
  cfg.blockDim = dim3(FT, 1, 1);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (win && win->num_bytes) {
    // the centroid planes stay in the persisting part of L2 across steps
    attr[1].id = cudaLaunchAttributeAccessPolicyWindow;
    attr[1].val.accessPolicyWindow = *win;
    cfg.numAttrs = 2;
  }
  return cudaLaunchKernelEx(&cfg, k_funnel, w);
}

const char *fused_mark_name(int tag) { return (tag >= 0 && tag < M_NTAGS) ? kMarkNames[tag] : ""; }

}  // namespace skv
