// skv_engine.cu -- the C ABI of include/seoulkv_b200.h.
//
// The engine owns every device buffer it uses (allocated in skv_create and
// the upload calls, never in skv_run).  The decode step is captured once into
// a CUDA graph and replayed on the caller's stream by skv_run.
#include <cuda_runtime.h>

#include <cstdio>
#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <type_traits>
#include <vector>

#include "../../include/seoulkv_b200.h"
#include "skv_append.cuh"
#include "skv_device.cuh"
#include "skv_fused.cuh"
#include "skv_kernels.cuh"
#include "skv_shard.cuh"

using namespace skv;

namespace {

thread_local std::string g_error;

int fail(int code, const std::string &msg) {
  g_error = msg;
  return code;
}

#define CK(call)                                                                          \
  do {                                                                                    \
    cudaError_t e_ = (call);                                                              \
    if (e_ != cudaSuccess)                                                                \
      return fail(SKV_E_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_));       \
  } while (0)

struct CellBufs {
  uint8_t *upper = nullptr, *lower = nullptr;
  float *coarse_scale4 = nullptr, *fine_scale = nullptr;
  uint16_t *resid = nullptr;
  int32_t *offsets = nullptr, *values = nullptr, *mates = nullptr;
  uint8_t *prefix2 = nullptr, *residual2 = nullptr, *residual4 = nullptr, *kv8 = nullptr;
  float *key_scale = nullptr;
  int32_t n_postings = 0;
  // cache append: the second CSR set and every token's two lists
  int32_t *offsets2 = nullptr, *values2 = nullptr, *mates2 = nullptr, *labels = nullptr;
};

struct Engine {
  SkvDesc desc{};
  int n_cells = 0;
  cudaStream_t stream = nullptr;  // internal stream (uploads, capture)
  std::vector<CellBufs> bufs;
  std::vector<CellDev> hcells;
  std::vector<int> index_ok, kv_ok;
  CellDev *dcells = nullptr;
  Work work{};
  std::vector<void *> allocs;     // workspace allocations
  uint16_t *q_pinned = nullptr;
  cudaEvent_t q_copied = nullptr, done = nullptr;
  bool q_pending = false, ran = false;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  // host-I/O steps: a query bound from host memory is copied in by the step
  // graph itself, which also copies the output and the counters back into
  // pinned host memory, so that a step costs one launch and one wait
  uint8_t *io_pinned = nullptr;    // output then counters (one copy back per host-I/O step)
  uint16_t *q_pinned_dev = nullptr;  // device views of the mapped pinned buffers (fused host-I/O steps)
  uint8_t *io_pinned_dev = nullptr;
  uint16_t *out_pinned = nullptr;  // views into io_pinned
  int32_t *counts_pinned = nullptr;
  size_t io_bytes = 0;
  cudaGraph_t graph_host = nullptr;
  cudaGraphExec_t exec_host = nullptr;
  bool q_host = false;   // the bound query is in q_pinned
  const uint16_t *q_bound = nullptr;  // fused path: the caller's device query, read in place by the kernel
  bool host_io = false;  // the last launch was a host-I/O step (its output and counters are in pinned memory)
  bool fused = false;             // one cluster kernel per step (else the staged kernels)
  // the centroid planes of every cell in one arena: cell c's upper plane at
  // c * nc * 128, its lower plane right after it (what an L2 access-policy
  // window covers, skv_set_l2_residency)
  uint8_t *planes = nullptr;
  size_t planes_bytes = 0;
  cudaAccessPolicyWindow l2win{};  // num_bytes 0: no window
  bool l2_resident = false;
  long long *phase_ts = nullptr;  // fused phase timestamps (skv_profile_phases)
  long long *cta_ts = nullptr;    // per-CTA entry/exit times (skv_profile_ctas)
  // sequence-sharded group over peer memory (skv_shard_setup / skv_shard_connect)
  struct {
    bool active = false;
    int rank = -1, n = 0;
    int32_t begin[SHARD_MAX] = {};
    void *region = nullptr;              // this shard's exchange region
    void *opened[SHARD_MAX] = {};        // peers' regions mapped here (IPC)
    void *kv8[SHARD_MAX][SHARD_CELLS] = {};  // peers' FP8 records mapped here (IPC)
    int32_t total = 0, sink = 0, local = 0;
    int32_t total_max = 0;               // the layer's length with every allowed append
    uint32_t *epoch = nullptr;
    int32_t *gids = nullptr;             // [4][4][100] global winners
    float *part = nullptr;               // [4][4][PART] this shard's partials
    ShardLinkDev *dev = nullptr;         // device copy of the group (Work::link)
  } link;
  // cache append (SkvDesc.max_context above the context)
  int32_t tmax = 0;                    // largest context of the slots
  int32_t t_host = 0;                  // context after the appends enqueued outside a capture
  bool appended = false;               // an append was enqueued (uploads are closed)
  bool append_captured = false;        // an append went into a caller's graph (t_host unknown)
  int32_t *tlen = nullptr;             // device context (Work::tlen)
  uint32_t *append_status = nullptr;   // APPEND_FULL when a replayed append did not fit
  AppendCellDev *dacells = nullptr;
  std::vector<AppendCellDev> hacells;
  std::vector<uint16_t *> wkeys;       // per slot: BF16 keys of the first local window [4][local][256]
  std::vector<int> labeled;            // per slot: the first window's lists are computed
  double *part_s = nullptr;
  int32_t *part_i = nullptr;
  int32_t *newlist = nullptr, *newtok = nullptr, *newmate = nullptr, *newins = nullptr;
  uint32_t *rebuild_done = nullptr;    // CTAs of the running CSR rebuild that finished
  uint32_t *assign_done = nullptr;     // [cell] CTAs of the running assignment that finished
  size_t post_cap = 0;                 // postings a CSR set holds (largest over cells)
  uint16_t *kv_stage = nullptr;        // host-input staging [2][n_cells][APPEND_MAX][256]
  bool appends() const { return tmax > desc.context; }
};

ShardLinkDev link_view(const Engine *e) {
  ShardLinkDev L{};
  for (int p = 0; p < e->link.n; ++p) L.peer[p] = p == e->link.rank ? e->link.region : e->link.opened[p];
  for (int p = 0; p < e->link.n; ++p) L.begin[p] = e->link.begin[p];
  for (int p = 0; p < e->link.n; ++p)
    for (int c = 0; c < SHARD_CELLS; ++c)
      L.kv8[p][c] = static_cast<const uint8_t *>(p == e->link.rank ? (void *)e->bufs[c].kv8 : e->link.kv8[p][c]);
  L.total = e->link.total;
  L.sink = e->link.sink;
  L.local = e->link.local;
  L.rank = e->link.rank;
  L.n_shards = e->link.n;
  L.token_begin = e->link.begin[e->link.rank];
  L.epoch = e->link.epoch;
  L.exits = e->link.epoch + 1;
  return L;
}

// The engine's Work as a launch sees it: on the fused path a device-resident
// query is read where the caller keeps it (no copy into the engine).
Work view_work(const Engine *e) {
  Work w = e->work;
  if (e->q_bound) w.q = e->q_bound;
  return w;
}

// The access-policy window the fused launches carry (null: none).
const cudaAccessPolicyWindow *window_of(const Engine *e) {
  return e->l2_resident && e->l2win.num_bytes ? &e->l2win : nullptr;
}

// Engines of this process holding an L2 window, per device: how many, the
// plane bytes they hold, and the persisting set-aside the process had before
// the first of them raised it (restored when the last one lets go).  The
// set-aside is state of this process's CUDA context: it ends with the process
// and changes no setting of the GPU.
std::mutex g_l2_lock;
constexpr int kL2Devices = 64;
int g_l2_users[kL2Devices] = {};
size_t g_l2_bytes[kL2Devices] = {};
size_t g_l2_prev[kL2Devices] = {};

void l2_release(Engine *e) {
  std::lock_guard<std::mutex> lock(g_l2_lock);
  const int dev = e->desc.device;
  const size_t bytes = e->l2win.num_bytes;
  e->l2_resident = false;
  e->l2win = cudaAccessPolicyWindow{};
  if (dev < 0 || dev >= kL2Devices || g_l2_users[dev] == 0) return;
  --g_l2_users[dev];
  g_l2_bytes[dev] -= std::min(bytes, g_l2_bytes[dev]);
  cudaCtxResetPersistingL2Cache();  // lines marked persisting become normal (others re-mark on access)
  cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, g_l2_users[dev] ? g_l2_bytes[dev] : g_l2_prev[dev]);
}

// Hold the engine's centroid planes in the persisting part of L2; false when
// the device offers no window or set-aside large enough for them.
int l2_acquire(Engine *e, bool *ok) {
  *ok = false;
  const int dev = e->desc.device;
  if (dev < 0 || dev >= kL2Devices) return SKV_OK;
  int max_persist = 0, max_win = 0;
  CK(cudaDeviceGetAttribute(&max_persist, cudaDevAttrMaxPersistingL2CacheSize, dev));
  CK(cudaDeviceGetAttribute(&max_win, cudaDevAttrMaxAccessPolicyWindowSize, dev));
  const size_t bytes = e->planes_bytes;
  std::lock_guard<std::mutex> lock(g_l2_lock);
  if (max_persist <= 0 || max_win <= 0 || bytes > (size_t)max_win || g_l2_bytes[dev] + bytes > (size_t)max_persist)
    return SKV_OK;
  if (g_l2_users[dev] == 0) CK(cudaDeviceGetLimit(&g_l2_prev[dev], cudaLimitPersistingL2CacheSize));
  CK(cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, g_l2_bytes[dev] + bytes));
  ++g_l2_users[dev];
  g_l2_bytes[dev] += bytes;
  e->l2win.base_ptr = e->planes;
  e->l2win.num_bytes = bytes;
  e->l2win.hitRatio = 1.0f;
  e->l2win.hitProp = cudaAccessPropertyPersisting;
  e->l2win.missProp = cudaAccessPropertyStreaming;
  e->l2_resident = true;
  *ok = true;
  return SKV_OK;
}

// Enqueue one decode step of the engine's path; for a connected shard group
// the global merge, attention and combine over peer memory follow.
cudaError_t launch_step(const Engine *e, const Work &w, cudaStream_t st) {
  cudaError_t r = e->fused ? launch_fused(w, st, window_of(e)) : launch_funnel(w, st);
  if (r != cudaSuccess || !e->link.active) return r;
  // the fused kernel exchanges inside itself (Work::link); the staged path
  // runs the exchange kernels after its funnel
  if (e->fused) return r;  // the fused kernel advances the step counter itself
  r = launch_shard_p2p_step(w, link_view(e), e->link.gids, e->link.part, w.counts + C_STATUS, st);
  return r == cudaSuccess ? launch_shard_epoch(e->link.dev, st) : r;
}

template <class T>
int dalloc(Engine *e, T **p, size_t count) {
  CK(cudaMalloc(reinterpret_cast<void **>(p), count * sizeof(T) + 16));
  CK(cudaMemset(*p, 0, count * sizeof(T) + 16));
  e->allocs.push_back(*p);
  return SKV_OK;
}

void free_cell(CellBufs &b, bool index, bool kv) {
  if (index) {
    // (the upper and lower planes live in the engine's plane arena)
    for (void *p : {(void *)b.coarse_scale4, (void *)b.fine_scale,
                    (void *)b.resid, (void *)b.offsets, (void *)b.values, (void *)b.mates, (void *)b.offsets2,
                    (void *)b.values2, (void *)b.mates2})
      if (p) cudaFree(p);
    b.upper = b.lower = nullptr;
    b.coarse_scale4 = b.fine_scale = nullptr;
    b.resid = nullptr;
    b.offsets = b.values = b.mates = nullptr;
    b.offsets2 = b.values2 = b.mates2 = nullptr;
  }
  if (kv) {
    for (void *p : {(void *)b.prefix2, (void *)b.residual2, (void *)b.residual4, (void *)b.kv8,
                    (void *)b.key_scale, (void *)b.labels})
      if (p) cudaFree(p);
    b.prefix2 = b.residual2 = b.residual4 = b.kv8 = nullptr;
    b.key_scale = nullptr;
    b.labels = nullptr;
  }
}

template <class T>
int upload(T **dst, const T *src, size_t count) {
  CK(cudaMalloc(reinterpret_cast<void **>(dst), count * sizeof(T) + 16));
  CK(cudaMemcpy(*dst, src, count * sizeof(T), cudaMemcpyHostToDevice));
  return SKV_OK;
}

// Upload `count` elements into a buffer of `cap` >= count elements.
template <class T>
int upload_cap(T **dst, const T *src, size_t count, size_t cap) {
  CK(cudaMalloc(reinterpret_cast<void **>(dst), cap * sizeof(T) + 16));
  if (count) CK(cudaMemcpy(*dst, src, count * sizeof(T), cudaMemcpyHostToDevice));
  return SKV_OK;
}

Engine *as_engine(void *h) { return static_cast<Engine *>(h); }

int ready(Engine *e) {
  for (int i = 0; i < e->n_cells; ++i)
    if (!e->index_ok[i] || !e->kv_ok[i])
      return fail(SKV_E_STATE, "cell " + std::to_string(i) + " has no index or K/V uploaded");
  return SKV_OK;
}

int sync_done(Engine *e) {
  CK(cudaSetDevice(e->desc.device));
  if (e->ran) CK(cudaEventSynchronize(e->done));
  CK(cudaStreamSynchronize(e->stream));
  return SKV_OK;
}

int read_counts(Engine *e, std::vector<int32_t> &c) {
  c.assign((size_t)e->n_cells * NCOUNT, 0);
  if (e->host_io) {
    std::memcpy(c.data(), e->counts_pinned, c.size() * sizeof(int32_t));
    return SKV_OK;
  }
  CK(cudaMemcpy(c.data(), e->work.counts, c.size() * sizeof(int32_t), cudaMemcpyDeviceToHost));
  return SKV_OK;
}

// The error a status with flags set turns into (skv_sync, skv_finish).
int status_error(const Engine *e, const SkvStatus &s) {
  char msg[320];
  if (s.flags & SKV_STATUS_APPEND_FULL) {
    std::snprintf(msg, sizeof msg, "a device-side append would have passed max_context %d (status 0x%x)",
                  e->tmax, s.flags);
    return fail(SKV_E_CAPACITY, msg);
  }
  if (s.flags & SKV_STATUS_APPEND_NONFINITE) {
    std::snprintf(msg, sizeof msg,
                  "an appended key had a non-finite element (assigned as 0; its FP8 record keeps it) (status 0x%x)",
                  s.flags);
    return fail(SKV_E_INVALID, msg);
  }
  std::snprintf(msg, sizeof msg,
                "live count out of range at cell %d (status 0x%x: %s%s%s); pool range [%d, %d], capacity %d",
                s.first_bad_cell, s.flags, (s.flags & SKV_STATUS_POOL_OVER) ? "pool above capacity " : "",
                (s.flags & SKV_STATUS_POOL_UNDER) ? "pool below 2048 " : "",
                (s.flags & SKV_STATUS_FINE_SHORT) ? "fewer than nprobe survivors" : "", s.pool_min, s.pool_max,
                e->desc.stage15_capacity);
  return fail(SKV_E_CAPACITY, msg);
}

// The device context (after every enqueued append has run).
int device_context(Engine *e, int32_t *t) {
  CK(cudaMemcpy(t, e->tlen, sizeof(int32_t), cudaMemcpyDeviceToHost));
  return SKV_OK;
}

void drop_graphs(Engine *e) {
  if (e->exec) { cudaGraphExecDestroy(e->exec); e->exec = nullptr; }
  if (e->graph) { cudaGraphDestroy(e->graph); e->graph = nullptr; }
  if (e->exec_host) { cudaGraphExecDestroy(e->exec_host); e->exec_host = nullptr; }
  if (e->graph_host) { cudaGraphDestroy(e->graph_host); e->graph_host = nullptr; }
}

}  // namespace

namespace skv {
// Lets other translation units of the library report through skv_last_error.
void set_last_error(const std::string &msg) { g_error = msg; }
}  // namespace skv

extern "C" {

const char *skv_last_error(void) { return g_error.c_str(); }

const char *skv_version(void) { return "seoulkv_b200 0.1 (sm_100a)"; }

// The lead cell: a small synthetic cell (512 centroids, 128 probes, a
// retrieval zone of 8192 tokens between the engine's sink and local zones)
// that the fused launch decodes in one extra cluster, scheduled first.  Its
// work is a few percent of a real cell's, so it runs through the kernel's
// phases ahead of the real cells and the instructions it fetches are in L2
// when they get there (the kernel's code is ~200 KB and runs about once per
// step, so a cold start fetches most of it from HBM).  Its data are random
// but valid: codes and planes of any bytes, a spill-2 CSR with each token in
// two distinct lists, finite FP8 records and a finite query.  Its outputs go
// to the workspace's last cell and are never read; results of the real cells
// do not depend on it.
static int build_lead_cell(Engine *e) {
  constexpr int LNC = 512, LP = 128, LR = 8192;
  const int sink = e->desc.sink, local = e->desc.local, T = sink + LR + local;
  uint64_t x = 0x9e3779b97f4a7c15ull;
  auto rnd = [&x]() {  // xorshift64*
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    return (uint32_t)((x * 0x2545f4914f6cdd1dull) >> 32);
  };
  auto bytes = [&](size_t n, uint8_t mask) {
    std::vector<uint8_t> v(n);
    for (auto &b : v) b = (uint8_t)(rnd() & mask);
    return v;
  };
  // spill-2 lists: token t in lists a != b, each list in token order
  std::vector<int> la(LR), lb(LR), cnt(LNC + 1, 0);
  for (int i = 0; i < LR; ++i) {
    la[i] = (int)(rnd() % LNC);
    lb[i] = (la[i] + 1 + (int)(rnd() % (LNC - 1))) % LNC;
    ++cnt[la[i] + 1];
    ++cnt[lb[i] + 1];
  }
  std::vector<int32_t> off(LNC + 1, 0), val(2 * LR), mate(2 * LR);
  for (int c = 0; c < LNC; ++c) off[c + 1] = off[c] + cnt[c + 1];
  std::vector<int> fill(off.begin(), off.end() - 1);
  for (int i = 0; i < LR; ++i) {
    const int t = sink + i;
    val[fill[la[i]]] = t;
    mate[fill[la[i]]++] = lb[i];
    val[fill[lb[i]]] = t;
    mate[fill[lb[i]]++] = la[i];
  }
  std::vector<float> s4(LNC / 32), fs(LNC / 32), ks(D);
  for (auto &v : s4) v = 0.02f + (rnd() % 1000) * 1e-5f;
  for (auto &v : fs) v = 0.01f + (rnd() % 1000) * 1e-5f;
  for (auto &v : ks) v = 1.0f + (rnd() % 1000) * 1e-3f;
  std::vector<uint16_t> resid(LNC), q(G * D);
  for (auto &v : resid) v = 0x3dcc;  // BF16 0.1
  for (auto &v : q) v = (uint16_t)(0x3c00 | (rnd() & 0x83ff));  // finite BF16, magnitude in [2^-7, 2)
  const auto up = bytes((size_t)LNC * 64, 0xff), lo = bytes((size_t)LNC * 64, 0xff);
  const auto p2 = bytes((size_t)T * 64, 0xff), r2 = bytes((size_t)T * 64, 0xff), r4 = bytes((size_t)T * 128, 0xff);
  const auto kv = bytes((size_t)T * REC, 0x77);  // FP8 e4m3 of magnitude < 2: no NaN
  CellDev c{};
  auto put = [e](auto **dst, const auto &src) {
    using T_ = std::remove_const_t<std::remove_reference_t<decltype(src[0])>>;
    T_ *d = nullptr;
    int rc = dalloc(e, &d, src.size());
    if (rc) return rc;
    CK(cudaMemcpy(d, src.data(), src.size() * sizeof(T_), cudaMemcpyHostToDevice));
    *dst = d;
    return SKV_OK;
  };
  int rc = SKV_OK;
  if (!rc) rc = put(&c.upper, up);
  if (!rc) rc = put(&c.lower, lo);
  if (!rc) rc = put(&c.coarse_scale4, s4);
  if (!rc) rc = put(&c.fine_scale, fs);
  if (!rc) rc = put(&c.resid, resid);
  if (!rc) rc = put(&c.offsets, off);
  if (!rc) rc = put(&c.values, val);
  if (!rc) rc = put(&c.mates, mate);
  if (!rc) rc = put(&c.prefix2, p2);
  if (!rc) rc = put(&c.residual2, r2);
  if (!rc) rc = put(&c.residual4, r4);
  if (!rc) rc = put(&c.key_scale, ks);
  if (!rc) rc = put(&c.kv8, kv);
  if (!rc) rc = put(&c.q, q);
  if (rc) return rc;
  c.nc = LNC;
  c.nprobe = LP;
  c.lam = 0.0625f;
  c.context = T;
  CK(cudaMemcpy(e->dcells + e->n_cells, &c, sizeof(CellDev), cudaMemcpyHostToDevice));
  e->work.lead = 1;
  return SKV_OK;
}

int skv_create(const SkvDesc *d, void **handle) {
  if (!d || !handle) return fail(SKV_E_INVALID, "null descriptor or handle");
  *handle = nullptr;
  if (d->n_slots < 1 || d->n_slots > 4096) return fail(SKV_E_INVALID, "n_slots must be in [1, 4096]");
  if (d->context < 1 || d->context > (1 << 20)) return fail(SKV_E_INVALID, "context must be in [1, 2^20]");
  if (d->sink < 0 || d->local < 0 || d->sink + d->local > d->context)
    return fail(SKV_E_INVALID, "sink/local must be disjoint and inside the context");
  if (d->nc < 32 || d->nc % 32 || d->nc > 65536)
    return fail(SKV_E_INVALID, "nc must be a multiple of 32 in [32, 65536]");
  if (d->stage15_capacity < M15_MIN || d->stage15_capacity > 65536 || d->stage15_capacity % 32)
    return fail(SKV_E_INVALID, "stage15_capacity must be a multiple of 32 in [2048, 65536]");
  if (d->max_context != 0 && (d->max_context < d->context || d->max_context > (1 << 20)))
    return fail(SKV_E_INVALID, "max_context must be 0 or in [context, 2^20]");
  auto *e = new Engine();
  e->desc = *d;
  e->n_cells = d->n_slots * G;
  int rc;
#define TRY(x)             \
  do {                     \
    rc = (x);              \
    if (rc) {              \
      skv_destroy(e);      \
      return rc;           \
    }                      \
  } while (0)
  {
    cudaError_t ce = cudaSetDevice(d->device);
    if (ce != cudaSuccess) {
      delete e;
      return fail(SKV_E_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(ce));
    }
  }
  TRY(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) ? fail(SKV_E_CUDA, "stream") : 0);
  TRY(cudaEventCreateWithFlags(&e->q_copied, cudaEventDisableTiming) ? fail(SKV_E_CUDA, "event") : 0);
  TRY(cudaEventCreateWithFlags(&e->done, cudaEventDisableTiming) ? fail(SKV_E_CUDA, "event") : 0);
  TRY(cudaHostAlloc(reinterpret_cast<void **>(&e->q_pinned), (size_t)d->n_slots * 16 * D * 2,
                    cudaHostAllocMapped) ? fail(SKV_E_CUDA, "pinned query buffer") : 0);
  TRY(cudaHostGetDevicePointer(reinterpret_cast<void **>(&e->q_pinned_dev), e->q_pinned, 0)
          ? fail(SKV_E_CUDA, "mapped query buffer") : 0);
  // the output and the counters live in one device block (and one pinned
  // mirror), so that a host-I/O step copies them back in one transfer
  const size_t out_bytes = (size_t)d->n_slots * 16 * D * 2;
  e->io_bytes = out_bytes + (size_t)d->n_slots * G * NCOUNT * 4;
  TRY(cudaHostAlloc(reinterpret_cast<void **>(&e->io_pinned), e->io_bytes, cudaHostAllocMapped)
          ? fail(SKV_E_CUDA, "pinned output buffer")
          : 0);
  TRY(cudaHostGetDevicePointer(reinterpret_cast<void **>(&e->io_pinned_dev), e->io_pinned, 0)
          ? fail(SKV_E_CUDA, "mapped output buffer") : 0);
  e->out_pinned = reinterpret_cast<uint16_t *>(e->io_pinned);
  e->counts_pinned = reinterpret_cast<int32_t *>(e->io_pinned + out_bytes);
  TRY(prepare_funnel_attributes() ? fail(SKV_E_CUDA, "kernel attributes") : 0);
  e->bufs.resize(e->n_cells);
  e->hcells.assign(e->n_cells, CellDev{});
  e->index_ok.assign(e->n_cells, 0);
  e->kv_ok.assign(e->n_cells, 0);
  Work &w = e->work;
  // per-cell workspace for n_cells + 1 cells: the fused path's lead cell
  // (see build_lead_cell) decodes into the last one
  const size_t C = e->n_cells + 1, nc = d->nc, cap = d->stage15_capacity;
  w.n_cells = e->n_cells;
  w.n_slots = d->n_slots;
  w.T = d->context;
  w.sink = d->sink;
  w.local = d->local;
  w.nc = d->nc;
  w.cap = d->stage15_capacity;
  e->planes_bytes = (size_t)e->n_cells * d->nc * 128;
  TRY(cudaMalloc(reinterpret_cast<void **>(&e->planes), e->planes_bytes + 16) ? fail(SKV_E_CUDA, "plane arena") : 0);
  TRY(dalloc(e, &e->dcells, C));
  w.cells = e->dcells;
  uint16_t *q = nullptr;
  TRY(dalloc(e, &q, (size_t)d->n_slots * 16 * D));
  w.q = q;
  w.chunks_nc = (d->nc + CHUNK - 1) / CHUNK;
  w.chunks_surv = (d->nc + SCHUNK - 1) / SCHUNK;
  w.chunks_pool = (d->stage15_capacity + CHUNK - 1) / CHUNK;
  TRY(dalloc(e, &w.frag, C * 3 * FRAG_ROW));
  TRY(dalloc(e, &w.shift, C * 3 * G));
  TRY(dalloc(e, &w.qscal, C * 8));
  TRY(dalloc(e, &w.lo, C * G * nc));
  TRY(dalloc(e, &w.hi, C * G * nc));
  TRY(dalloc(e, &w.thr, C * 16));
  TRY(dalloc(e, &w.smask, C * nc));
  TRY(dalloc(e, &w.chunk_cnt, C * w.chunks_nc));
  TRY(dalloc(e, &w.tags, C * nc));
  TRY(dalloc(e, &w.fkeys, C * G * nc));
  TRY(dalloc(e, &w.selbits, C * (nc / 32)));
  TRY(dalloc(e, &w.kept, C * nc));
  TRY(dalloc(e, &w.keptmask, C * nc));
  TRY(dalloc(e, &w.chunk_kept, C * w.chunks_surv));
  TRY(dalloc(e, &w.chunk_sel, C * w.chunks_surv));
  TRY(dalloc(e, &w.chunk_post, C * w.chunks_surv));
  TRY(dalloc(e, &w.sel, C * SEL_MAX));
  TRY(dalloc(e, &w.pool, C * cap));
  TRY(dalloc(e, &w.k15, C * G * cap));
  TRY(dalloc(e, &w.u15bits, C * (cap / 32)));
  TRY(dalloc(e, &w.u15pos, C * U15_MAX));
  TRY(dalloc(e, &w.u15tok, C * U15_MAX));
  TRY(dalloc(e, &w.k16, C * G * U15_MAX));
  TRY(dalloc(e, &w.candbits, C * (U15_MAX / 32)));
  TRY(dalloc(e, &w.cand, C * CAND_MAX));
  TRY(dalloc(e, &w.k2, C * G * CAND_MAX));
  TRY(dalloc(e, &w.final_pos, C * G * TOPK));
  TRY(dalloc(e, &w.final_ids, C * G * TOPK));
  TRY(dalloc(e, &w.final_keys, C * G * TOPK));
  {
    uint8_t *io = nullptr;
    TRY(dalloc(e, &io, e->io_bytes + NCOUNT * sizeof(int32_t)));  // (+ the lead cell's counters)
    w.out = reinterpret_cast<uint16_t *>(io);
    w.counts = reinterpret_cast<int32_t *>(io + out_bytes);
  }
  TRY(dalloc(e, &w.attn_part, C * G * ATTN_SPLIT * PART));
  TRY(dalloc(e, &w.arrive, C));
  TRY(dalloc(e, &w.hist, C * 4 * G * 4096));
  TRY(dalloc(e, &e->phase_ts, 2 * FUSED_MARKS));
  e->tmax = d->max_context ? d->max_context : d->context;
  e->t_host = d->context;
  {
    int32_t *tl = nullptr;
    TRY(dalloc(e, &tl, 1));
    TRY(cudaMemcpy(tl, &d->context, sizeof(int32_t), cudaMemcpyHostToDevice) ? fail(SKV_E_CUDA, "context word") : 0);
    e->tlen = tl;
    w.tlen = tl;
  }
  e->wkeys.assign(d->n_slots, nullptr);
  e->labeled.assign(d->n_slots, 0);
  if (e->appends()) {
    e->hacells.assign(e->n_cells, AppendCellDev{});
    TRY(dalloc(e, &e->dacells, e->n_cells));
    TRY(dalloc(e, &e->append_status, 1));
    TRY(dalloc(e, &e->part_s, C * APPEND_MAX * ASSIGN_SPLIT * 2));
    TRY(dalloc(e, &e->part_i, C * APPEND_MAX * ASSIGN_SPLIT * 2));
    TRY(dalloc(e, &e->newlist, C * 2 * APPEND_MAX));
    TRY(dalloc(e, &e->newtok, C * 2 * APPEND_MAX));
    TRY(dalloc(e, &e->newmate, C * 2 * APPEND_MAX));
    TRY(dalloc(e, &e->newins, C * 2 * APPEND_MAX));
    TRY(dalloc(e, &e->rebuild_done, 1));
    TRY(dalloc(e, &e->assign_done, C));
  }
  w.phase_ts = nullptr;
  w.cta_ts = nullptr;
  e->fused = !(d->flags & SKV_FLAG_STAGED) && fused_supported(w);
  w.trace = (d->flags & SKV_FLAG_TRACE) ? 1 : 0;
  if (e->fused) TRY(prepare_fused_attributes() ? fail(SKV_E_CUDA, "fused kernel attributes") : 0);
  // (the lead cell's buffers use the workspace's per-cell strides: nc >= 512)
  if (e->fused && !(d->flags & SKV_FLAG_NO_LEAD) && d->nc >= 512) TRY(build_lead_cell(e));
#undef TRY
  *handle = e;
  return SKV_OK;
}

void skv_destroy(void *handle) {
  Engine *e = as_engine(handle);
  if (!e) return;
  cudaSetDevice(e->desc.device);
  if (e->stream) cudaStreamSynchronize(e->stream);
  if (e->ran && e->done) cudaEventSynchronize(e->done);
  for (void *p : e->link.opened)
    if (p) cudaIpcCloseMemHandle(p);
  for (auto &row : e->link.kv8)
    for (void *p : row)
      if (p) cudaIpcCloseMemHandle(p);
  if (e->link.region) cudaFree(e->link.region);
  drop_graphs(e);
  if (e->l2_resident) l2_release(e);
  for (auto &b : e->bufs) free_cell(b, true, true);
  if (e->planes) cudaFree(e->planes);
  for (void *p : e->wkeys)
    if (p) cudaFree(p);
  if (e->kv_stage) cudaFree(e->kv_stage);
  for (void *p : e->allocs) cudaFree(p);
  if (e->q_pinned) cudaFreeHost(e->q_pinned);
  if (e->io_pinned) cudaFreeHost(e->io_pinned);
  if (e->q_copied) cudaEventDestroy(e->q_copied);
  if (e->done) cudaEventDestroy(e->done);
  if (e->stream) cudaStreamDestroy(e->stream);
  delete e;
}

static int refresh_cells(Engine *e) {
  CK(cudaMemcpy(e->dcells, e->hcells.data(), e->hcells.size() * sizeof(CellDev), cudaMemcpyHostToDevice));
  if (e->appends())
    CK(cudaMemcpy(e->dacells, e->hacells.data(), e->hacells.size() * sizeof(AppendCellDev),
                  cudaMemcpyHostToDevice));
  return SKV_OK;
}

// Centroid partitions of the assignment: one resident wave (2 CTAs per SM)
// over all cells and key groups, but at least 16 (many key groups), and at
// least one 16-row tile per warp.
static int assign_split(int nc, int m, int n_cells) {
  const int groups = (m + 3) / 4, fill = std::max(16, (296 + n_cells * groups - 1) / (n_cells * groups));
  return std::max(1, std::min({ASSIGN_SPLIT, (nc / 16 + 7) / 8, fill}));
}

// The two lists of every token in a slot's first local window, from the
// window's BF16 keys, once both the slot's index and its K/V are uploaded.
static int label_window(Engine *e, int slot) {
  e->labeled[slot] = 0;
  if (!e->appends()) return SKV_OK;
  for (int g = 0; g < G; ++g)
    if (!e->index_ok[slot * G + g] || !e->kv_ok[slot * G + g]) return SKV_OK;
  const int T0 = e->desc.context, local = e->desc.local;
  for (int j0 = 0; j0 < local; j0 += APPEND_MAX) {
    AssignArgs a{};
    a.cells = e->dcells;
    a.acells = e->dacells;
    a.tlen = e->tlen;
    a.k = e->wkeys[slot] + (size_t)j0 * D;
    a.k_cell_stride = (long long)local * D;
    a.cell0 = slot * G;
    a.n_cells = G;
    a.m = std::min(APPEND_MAX, local - j0);
    a.nc = e->desc.nc;
    a.split = assign_split(e->desc.nc, a.m, G);
    a.lab_base = T0 - local + j0;
    a.tmax = e->tmax;
    a.part_s = e->part_s;
    a.part_i = e->part_i;
    CK(launch_assign(a, e->stream));
  }
  CK(cudaStreamSynchronize(e->stream));
  e->labeled[slot] = 1;
  return SKV_OK;
}

int skv_upload_index(void *handle, int32_t slot, const SkvCellView *cells) {
  Engine *e = as_engine(handle);
  if (!e || !cells) return fail(SKV_E_INVALID, "null engine or cells");
  if (slot < 0 || slot >= e->desc.n_slots) return fail(SKV_E_INVALID, "slot out of range");
  if (e->appended) return fail(SKV_E_STATE, "the cache has grown by appends; uploads are closed");
  CK(cudaSetDevice(e->desc.device));
  CK(cudaStreamSynchronize(e->stream));
  const int nc = e->desc.nc, T = e->desc.context;
  for (int g = 0; g < G; ++g) {
    const SkvCellView &v = cells[g];
    if (v.nc != nc) return fail(SKV_E_INVALID, "cell nc differs from the engine's nc");
    if (v.nprobe < 16 || v.nprobe > 512 || v.nprobe % 16 || v.nprobe > nc)
      return fail(SKV_E_INVALID, "nprobe must be a multiple of 16 in [16, min(512, nc)]");
    if (!(v.lam >= 0.0f) || v.lam > 3.0e38f) return fail(SKV_E_INVALID, "lam must be finite and >= 0");
    if (!v.upper || !v.lower || !v.coarse_scale4 || !v.fine_scale || !v.resid_bf16 || !v.offsets ||
        !v.values || !v.mates)
      return fail(SKV_E_INVALID, "null index array");
    if (v.offsets[0] != 0 || v.offsets[nc] != v.n_postings || v.n_postings < 0)
      return fail(SKV_E_INVALID, "CSR offsets must start at 0 and end at n_postings");
    for (int i = 0; i < nc; ++i)
      if (v.offsets[i + 1] < v.offsets[i]) return fail(SKV_E_INVALID, "CSR offsets must be non-decreasing");
    for (int j = 0; j < v.n_postings; ++j) {
      if (v.values[j] < 0 || v.values[j] >= T) return fail(SKV_E_INVALID, "CSR token id out of range");
      if (v.mates[j] < -1 || v.mates[j] >= nc) return fail(SKV_E_INVALID, "posting mate out of range");
    }
  }
  for (int g = 0; g < G; ++g) {
    const SkvCellView &v = cells[g];
    const int cell = slot * G + g;
    CellBufs &b = e->bufs[cell];
    free_cell(b, true, false);
    int rc;
    b.upper = e->planes + (size_t)cell * nc * 128;
    b.lower = b.upper + (size_t)nc * 64;
    CK(cudaMemcpy(b.upper, v.upper, (size_t)nc * 64, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(b.lower, v.lower, (size_t)nc * 64, cudaMemcpyHostToDevice));
    if ((rc = upload(&b.coarse_scale4, v.coarse_scale4, (size_t)nc / 32))) return rc;
    if ((rc = upload(&b.fine_scale, v.fine_scale, (size_t)nc / 32))) return rc;
    if ((rc = upload(&b.resid, v.resid_bf16, (size_t)nc))) return rc;
    // with appends, both CSR sets hold the postings of a full-grown cache
    const size_t post_cap = (size_t)std::max(v.n_postings, 1) + 2 * (size_t)(e->tmax - T);
    if ((rc = upload(&b.offsets, v.offsets, (size_t)nc + 1))) return rc;
    if ((rc = upload_cap(&b.values, v.values, (size_t)v.n_postings, post_cap))) return rc;
    if ((rc = upload_cap(&b.mates, v.mates, (size_t)v.n_postings, post_cap))) return rc;
    b.n_postings = v.n_postings;
    e->post_cap = std::max(e->post_cap, post_cap);
    if (e->appends()) {
      CK(cudaMalloc(reinterpret_cast<void **>(&b.offsets2), ((size_t)nc + 1) * sizeof(int32_t)));
      CK(cudaMalloc(reinterpret_cast<void **>(&b.values2), post_cap * sizeof(int32_t)));
      CK(cudaMalloc(reinterpret_cast<void **>(&b.mates2), post_cap * sizeof(int32_t)));
      AppendCellDev &a = e->hacells[cell];
      a.offsets[0] = b.offsets;
      a.values[0] = b.values;
      a.mates[0] = b.mates;
      a.offsets[1] = b.offsets2;
      a.values[1] = b.values2;
      a.mates[1] = b.mates2;
      a.cur = 0;
      a.n_postings = v.n_postings;
    }
    CellDev &c = e->hcells[cell];
    c.upper = b.upper;
    c.lower = b.lower;
    c.coarse_scale4 = b.coarse_scale4;
    c.fine_scale = b.fine_scale;
    c.resid = b.resid;
    c.offsets = b.offsets;
    c.values = b.values;
    c.mates = b.mates;
    c.nc = nc;
    c.nprobe = v.nprobe;
    c.lam = v.lam;
    e->index_ok[cell] = 1;
  }
  int rc = refresh_cells(e);
  return rc ? rc : label_window(e, slot);
}

int skv_upload_kv(void *handle, int32_t slot, const uint16_t *k, const uint16_t *v, int32_t on_device) {
  Engine *e = as_engine(handle);
  if (!e || !k || !v) return fail(SKV_E_INVALID, "null engine or K/V");
  if (slot < 0 || slot >= e->desc.n_slots) return fail(SKV_E_INVALID, "slot out of range");
  if (e->appended) return fail(SKV_E_STATE, "the cache has grown by appends; uploads are closed");
  CK(cudaSetDevice(e->desc.device));
  CK(cudaStreamSynchronize(e->stream));
  const size_t T = e->desc.context, elems = (size_t)G * T * D;
  const size_t rows = e->tmax;  // planes and records of a full-grown cache
  const uint16_t *dk = k, *dv = v;
  uint16_t *stage = nullptr;
  if (!on_device) {
    CK(cudaMalloc(reinterpret_cast<void **>(&stage), 2 * elems * sizeof(uint16_t)));
    cudaError_t c1 = cudaMemcpy(stage, k, elems * 2, cudaMemcpyHostToDevice);
    cudaError_t c2 = c1 == cudaSuccess ? cudaMemcpy(stage + elems, v, elems * 2, cudaMemcpyHostToDevice) : c1;
    if (c2 != cudaSuccess) {
      cudaFree(stage);
      return fail(SKV_E_CUDA, std::string("K/V upload: ") + cudaGetErrorString(c2));
    }
    dk = stage;
    dv = stage + elems;
  }
  float *scale[G];
  uint8_t *p2[G], *r2[G], *r4[G], *kv8[G];
  uint32_t *smax = nullptr;
  int rc = SKV_OK;
  for (int g = 0; g < G && rc == SKV_OK; ++g) {
    CellBufs &b = e->bufs[slot * G + g];
    free_cell(b, false, true);
    if (cudaMalloc(reinterpret_cast<void **>(&b.prefix2), rows * 64) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void **>(&b.residual2), rows * 64) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void **>(&b.residual4), rows * 128) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void **>(&b.kv8), rows * REC) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void **>(&b.key_scale), D * sizeof(float)) != cudaSuccess ||
        (e->appends() && cudaMalloc(reinterpret_cast<void **>(&b.labels), rows * 2 * sizeof(int32_t)) != cudaSuccess))
      rc = fail(SKV_E_CUDA, "out of device memory for key planes / FP8 records");
    scale[g] = b.key_scale;
    p2[g] = b.prefix2;
    r2[g] = b.residual2;
    r4[g] = b.residual4;
    kv8[g] = b.kv8;
  }
  if (rc == SKV_OK && cudaMalloc(reinterpret_cast<void **>(&smax), G * D * sizeof(uint32_t)) != cudaSuccess)
    rc = fail(SKV_E_CUDA, "out of device memory");
  if (rc == SKV_OK) {
    cudaError_t ce = launch_key_codec(dk, dv, (int)T, smax, scale, p2, r2, r4, kv8, e->stream);
    // with appends, the first local window's keys stay for its spill-2 lists
    const size_t local = e->desc.local;
    if (ce == cudaSuccess && e->appends() && local > 0) {
      if (!e->wkeys[slot]) ce = cudaMalloc(reinterpret_cast<void **>(&e->wkeys[slot]), G * local * D * 2);
      for (int g = 0; g < G && ce == cudaSuccess; ++g)
        ce = cudaMemcpyAsync(e->wkeys[slot] + (size_t)g * local * D, dk + ((size_t)g * T + T - local) * D,
                             local * D * 2, cudaMemcpyDeviceToDevice, e->stream);
    }
    for (int g = 0; g < G && ce == cudaSuccess && e->appends(); ++g)
      ce = cudaMemsetAsync(e->bufs[slot * G + g].labels, 0xff, rows * 2 * sizeof(int32_t), e->stream);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(e->stream);
    if (ce != cudaSuccess) rc = fail(SKV_E_CUDA, std::string("key codec: ") + cudaGetErrorString(ce));
  }
  if (smax) cudaFree(smax);
  if (stage) cudaFree(stage);
  if (rc) return rc;
  for (int g = 0; g < G; ++g) {
    const int cell = slot * G + g;
    CellDev &c = e->hcells[cell];
    c.prefix2 = p2[g];
    c.residual2 = r2[g];
    c.residual4 = r4[g];
    c.kv8 = kv8[g];
    c.key_scale = scale[g];
    if (e->appends()) {
      AppendCellDev &a = e->hacells[cell];
      a.prefix2 = p2[g];
      a.residual2 = r2[g];
      a.residual4 = r4[g];
      a.kv8 = kv8[g];
      a.key_scale = scale[g];
      a.labels = e->bufs[cell].labels;
    }
    e->kv_ok[cell] = 1;
  }
  rc = refresh_cells(e);
  return rc ? rc : label_window(e, slot);
}

int skv_bind_query(void *handle, const uint16_t *q, int32_t on_device, void *stream) {
  Engine *e = as_engine(handle);
  if (!e || !q) return fail(SKV_E_INVALID, "null engine or query");
  CK(cudaSetDevice(e->desc.device));
  cudaStream_t st = static_cast<cudaStream_t>(stream);  // NULL: legacy default stream
  const size_t bytes = (size_t)e->desc.n_slots * 16 * D * sizeof(uint16_t);
  uint16_t *dq = const_cast<uint16_t *>(e->work.q);
  if (on_device) {
    // the fused kernel reads the caller's query in place, in stream order
    // (the caller keeps the buffer unchanged until the run has executed, as
    // for any stream-ordered input); the staged kernels take a copy
    if (e->fused) {
      e->q_bound = q;
    } else {
      CK(cudaMemcpyAsync(dq, q, bytes, cudaMemcpyDeviceToDevice, st));
      e->q_bound = nullptr;
    }
    e->q_host = false;
    return SKV_OK;
  }
  e->q_bound = nullptr;
  // the pinned staging buffer may still feed the previous host-I/O step;
  // the next skv_run copies it in as the first node of its graph
  if (e->q_pending) CK(cudaEventSynchronize(e->q_copied));
  e->q_pending = false;
  std::memcpy(e->q_pinned, q, bytes);
  e->q_host = true;
  return SKV_OK;
}

int skv_run(void *handle, void *stream) {
  Engine *e = as_engine(handle);
  if (!e) return fail(SKV_E_INVALID, "null engine");
  int rc = ready(e);
  if (rc) return rc;
  CK(cudaSetDevice(e->desc.device));
  cudaStream_t st = static_cast<cudaStream_t>(stream);  // NULL: legacy default stream
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  CK(cudaStreamIsCapturing(st, &cap));
  if (cap != cudaStreamCaptureStatusNone) {
    // the caller is capturing its own graph (e.g. a model's decode step):
    // the step's kernels go into that graph directly; the query must already
    // be on the device (a host query's pinned staging copy is not capturable
    // as a step of the caller's graph)
    if (e->q_host) return fail(SKV_E_STATE, "a captured run needs a device-resident query");
    Work w = view_work(e);
    if (e->link.active) {
      w.link = e->link.dev;
      w.shard_gids = e->link.gids;
    }
    CK(launch_step(e, w, st));
    e->host_io = false;
    return SKV_OK;
  }
  const bool host = e->q_host;
  if (!host && e->q_bound) {
    // fused path, device query: one kernel launch, reading the query in place
    Work w = view_work(e);
    if (e->link.active) {
      w.link = e->link.dev;
      w.shard_gids = e->link.gids;
    }
    CK(launch_step(e, w, st));
    e->host_io = false;
    CK(cudaEventRecord(e->done, st));
    e->ran = true;
    return SKV_OK;
  }
  if (host && e->fused) {
    // fused path, host query: one kernel launch that reads the query from
    // the mapped pinned buffer and writes the output and counters back into
    // mapped pinned memory (no copy nodes around it)
    Work w = e->work;
    w.q = e->q_pinned_dev;
    w.out_host = reinterpret_cast<uint16_t *>(e->io_pinned_dev);
    w.counts_host = reinterpret_cast<int32_t *>(e->io_pinned_dev + (size_t)e->desc.n_slots * 16 * D * 2);
    w.q_store = const_cast<uint16_t *>(e->work.q);
    if (e->link.active) {
      w.link = e->link.dev;
      w.shard_gids = e->link.gids;
    }
    CK(launch_step(e, w, st));
    CK(cudaEventRecord(e->q_copied, st));
    e->q_pending = true;
    e->host_io = true;
    CK(cudaEventRecord(e->done, st));
    e->ran = true;
    return SKV_OK;
  }
  cudaGraphExec_t &exec = host ? e->exec_host : e->exec;
  if (!exec) {
    CK(cudaStreamSynchronize(e->stream));
    CK(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
    // only the step graph carries the group; profiling launches run the funnel alone
    Work w = e->work;
    if (e->link.active) {
      w.link = e->link.dev;
      w.shard_gids = e->link.gids;
    }
    const size_t qbytes = (size_t)e->desc.n_slots * 16 * D * sizeof(uint16_t);
    cudaError_t le = cudaSuccess;
    if (host) le = cudaMemcpyAsync(const_cast<uint16_t *>(w.q), e->q_pinned, qbytes, cudaMemcpyHostToDevice, e->stream);
    if (le == cudaSuccess) le = launch_step(e, w, e->stream);
    if (host && le == cudaSuccess)  // output and counters: one contiguous block
      le = cudaMemcpyAsync(e->io_pinned, w.out, e->io_bytes, cudaMemcpyDeviceToHost, e->stream);
    cudaGraph_t g = nullptr;
    cudaError_t ce = cudaStreamEndCapture(e->stream, &g);
    if (le != cudaSuccess) {
      if (g) cudaGraphDestroy(g);
      return fail(SKV_E_CUDA, std::string("funnel launch: ") + cudaGetErrorString(le));
    }
    if (ce != cudaSuccess) return fail(SKV_E_CUDA, std::string("graph capture: ") + cudaGetErrorString(ce));
    (host ? e->graph_host : e->graph) = g;
    CK(cudaGraphInstantiate(&exec, g, 0));
  }
  CK(cudaGraphLaunch(exec, st));
  if (host) {
    CK(cudaEventRecord(e->q_copied, st));
    e->q_pending = true;
  }
  e->host_io = host;
  CK(cudaEventRecord(e->done, st));
  e->ran = true;
  return SKV_OK;
}

int skv_set_l2_residency(void *handle, int32_t enable, size_t *resident_bytes) {
  Engine *e = as_engine(handle);
  if (!e) return fail(SKV_E_INVALID, "null engine");
  if (resident_bytes) *resident_bytes = 0;
  int rc = sync_done(e);
  if (rc) return rc;
  if (!enable) {
    if (e->l2_resident) {
      l2_release(e);
      drop_graphs(e);  // the step graphs are captured again without the window
    }
    return SKV_OK;
  }
  if (!e->l2_resident && e->fused) {
    bool ok = false;
    if ((rc = l2_acquire(e, &ok))) return rc;
    if (ok) drop_graphs(e);  // captured again with the window on the funnel's launch
  }
  if (resident_bytes) *resident_bytes = e->l2_resident ? e->l2win.num_bytes : 0;
  return SKV_OK;
}

int skv_step(void *handle, const uint16_t *q, int32_t on_device, void *stream) {
  int rc = skv_bind_query(handle, q, on_device, stream);
  return rc ? rc : skv_run(handle, stream);
}

int skv_append(void *handle, const uint16_t *k, const uint16_t *v, int32_t n_tokens, int32_t on_device,
               void *stream) {
  Engine *e = as_engine(handle);
  if (!e || !k || !v) return fail(SKV_E_INVALID, "null engine or K/V");
  if (!e->appends()) return fail(SKV_E_STATE, "appends need an engine created with max_context above the context");
  if (e->link.region && !e->link.active) return fail(SKV_E_STATE, "connect the shard group before appending");
  // in a connected group the tokens join the last shard (it holds the local
  // window); every shard's kernel learns the layer's new length
  const bool linked = e->link.active, last = !linked || e->link.rank == e->link.n - 1;
  if (n_tokens < 1 || n_tokens > APPEND_MAX)
    return fail(SKV_E_INVALID, "n_tokens must be in [1, " + std::to_string(APPEND_MAX) + "]");
  int rc = ready(e);
  if (rc) return rc;
  for (int s = 0; s < e->desc.n_slots; ++s)
    if (!e->labeled[s]) return fail(SKV_E_STATE, "slot " + std::to_string(s) + " has no window lists");
  CK(cudaSetDevice(e->desc.device));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  CK(cudaStreamIsCapturing(st, &cap));
  const bool captured = cap != cudaStreamCaptureStatusNone;
  if (captured && !on_device) return fail(SKV_E_STATE, "a captured append needs device-resident K/V");
  if (!captured) {
    int32_t t = e->t_host;
    if (e->append_captured && last) {  // graph replays may have appended: ask the device
      CK(cudaStreamSynchronize(st));
      if ((rc = sync_done(e)) || (rc = device_context(e, &t))) return rc;
    }
    if (t + n_tokens > e->tmax)
      return fail(SKV_E_CAPACITY, "append of " + std::to_string(n_tokens) + " tokens to context " +
                                      std::to_string(t) + " passes max_context " + std::to_string(e->tmax));
  }
  if (!last) {  // a shard before the last: only the layer's length grows
    CK(launch_link_grow(e->link.dev, n_tokens, e->link.total_max, st));
    e->appended = true;
    if (captured) {
      e->append_captured = true;
    } else {
      e->t_host += n_tokens;
      CK(cudaEventRecord(e->done, st));
      e->ran = true;
    }
    return SKV_OK;
  }
  const size_t rows = (size_t)e->n_cells * n_tokens * D;
  const uint16_t *dk = k, *dv = v;
  if (!on_device) {
    if (!e->kv_stage)
      CK(cudaMalloc(reinterpret_cast<void **>(&e->kv_stage), 2 * (size_t)e->n_cells * APPEND_MAX * D * 2));
    uint16_t *sk = e->kv_stage, *sv = e->kv_stage + (size_t)e->n_cells * APPEND_MAX * D;
    CK(cudaMemcpyAsync(sk, k, rows * 2, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(sv, v, rows * 2, cudaMemcpyHostToDevice, st));
    dk = sk;
    dv = sv;
  }
  AppendArgs a{};
  a.cells = e->dcells;
  a.acells = e->dacells;
  a.tlen = e->tlen;
  a.status = e->append_status;
  a.k = dk;
  a.v = dv;
  a.n_cells = e->n_cells;
  a.m = n_tokens;
  a.nc = e->desc.nc;
  a.local = e->desc.local;
  a.tmax = e->tmax;
  a.newlist = e->newlist;
  a.newtok = e->newtok;
  a.newmate = e->newmate;
  a.newins = e->newins;
  a.done = e->rebuild_done;
  a.assign_done = e->assign_done;
  a.rebuild_ctas = (int)((e->post_cap + e->desc.nc + 1 + 2 * APPEND_MAX + 256 * REBUILD_PER_THREAD - 1) /
                         (256 * REBUILD_PER_THREAD));
  AssignArgs s{};
  s.cells = e->dcells;
  s.acells = e->dacells;
  s.tlen = e->tlen;
  s.k = dk;
  s.k_cell_stride = (long long)n_tokens * D;
  s.cell0 = 0;
  s.n_cells = e->n_cells;
  s.m = n_tokens;
  s.nc = e->desc.nc;
  s.split = assign_split(e->desc.nc, n_tokens, e->n_cells);
  s.use_tlen = 1;
  s.guard = n_tokens;
  s.tmax = e->tmax;
  s.status = e->append_status;
  s.part_s = e->part_s;
  s.part_i = e->part_i;
  CK(launch_append(a, s, st));
  if (linked) CK(launch_link_grow(e->link.dev, n_tokens, e->link.total_max, st));
  e->appended = true;
  if (captured) e->append_captured = true;
  else e->t_host += n_tokens;
  if (!captured) {
    CK(cudaEventRecord(e->done, st));
    e->ran = true;
  }
  return SKV_OK;
}

int skv_context(void *handle, int32_t *context) {
  Engine *e = as_engine(handle);
  if (!e || !context) return fail(SKV_E_INVALID, "null engine or output");
  int rc = sync_done(e);
  return rc ? rc : device_context(e, context);
}

int skv_finish(void *handle, uint16_t *out, SkvStatus *status) {
  Engine *e = as_engine(handle);
  if (!e) return fail(SKV_E_INVALID, "null engine");
  SkvStatus s{};
  int rc = skv_status(handle, &s);
  if (rc) return rc;
  if (status) *status = s;
  if (out) {
    if (e->host_io) {
      std::memcpy(out, e->out_pinned, (size_t)e->desc.n_slots * 16 * D * 2);
    } else {
      CK(cudaMemcpy(out, e->work.out, (size_t)e->desc.n_slots * 16 * D * 2, cudaMemcpyDeviceToHost));
    }
  }
  if (s.flags) return status_error(e, s);
  return SKV_OK;
}

int skv_status(void *handle, SkvStatus *out) {
  Engine *e = as_engine(handle);
  if (!e || !out) return fail(SKV_E_INVALID, "null engine or output");
  int rc = sync_done(e);
  if (rc) return rc;
  std::vector<int32_t> c;
  if ((rc = read_counts(e, c))) return rc;
  SkvStatus s{};
  s.first_bad_cell = -1;
  s.pool_min = 1 << 30;
  for (int i = 0; i < e->n_cells; ++i) {
    const int32_t *k = &c[(size_t)i * NCOUNT];
    const uint32_t st = (uint32_t)k[C_STATUS];
    if (st && s.first_bad_cell < 0) s.first_bad_cell = i;
    s.flags |= st;
    s.survivors_max = std::max(s.survivors_max, k[C_TAGS]);
    s.pool_max = std::max(s.pool_max, k[C_POOL]);
    s.pool_min = std::min(s.pool_min, k[C_POOL]);
    s.union15_max = std::max(s.union15_max, k[C_U15]);
    s.union16_max = std::max(s.union16_max, k[C_CAND]);
  }
  if (e->append_status) {
    uint32_t as = 0;
    CK(cudaMemcpy(&as, e->append_status, sizeof as, cudaMemcpyDeviceToHost));
    if (as & APPEND_FULL) s.flags |= SKV_STATUS_APPEND_FULL;
    if (as & APPEND_NONFINITE) s.flags |= SKV_STATUS_APPEND_NONFINITE;
  }
  *out = s;
  return SKV_OK;
}

int skv_sync(void *handle) {
  Engine *e = as_engine(handle);
  if (!e) return fail(SKV_E_INVALID, "null engine");
  if (!e->ran) return sync_done(e);
  SkvStatus s;
  int rc = skv_status(handle, &s);
  if (rc) return rc;
  if (s.flags) return status_error(e, s);
  return SKV_OK;
}

int skv_output(void *handle, void *out, int32_t to_host) {
  Engine *e = as_engine(handle);
  if (!e || !out) return fail(SKV_E_INVALID, "null engine or output");
  if (!to_host) {
    *static_cast<void **>(out) = e->work.out;
    return SKV_OK;
  }
  int rc = sync_done(e);
  if (rc) return rc;
  if (e->host_io) {
    std::memcpy(out, e->out_pinned, (size_t)e->desc.n_slots * 16 * D * 2);
    return SKV_OK;
  }
  CK(cudaMemcpy(out, e->work.out, (size_t)e->desc.n_slots * 16 * D * 2, cudaMemcpyDeviceToHost));
  return SKV_OK;
}

int skv_debug_ids(void *handle, int32_t *out) {
  Engine *e = as_engine(handle);
  if (!e || !out) return fail(SKV_E_INVALID, "null engine or output");
  int rc = sync_done(e);
  if (rc) return rc;
  CK(cudaMemcpy(out, e->work.final_ids, (size_t)e->n_cells * G * TOPK * sizeof(int32_t),
                cudaMemcpyDeviceToHost));
  return SKV_OK;
}

int skv_read_stage(void *handle, int32_t slot, int32_t which, void *dst, size_t bytes, size_t *written) {
  Engine *e = as_engine(handle);
  if (!e || !dst) return fail(SKV_E_INVALID, "null engine or destination");
  if (slot < 0 || slot >= e->desc.n_slots) return fail(SKV_E_INVALID, "slot out of range");
  int rc = sync_done(e);
  if (rc) return rc;
  const size_t nc = e->desc.nc, cap = e->desc.stage15_capacity, c0 = (size_t)slot * G;
  const Work &w = e->work;
  const void *src = nullptr;
  size_t n = 0;
  if (e->fused && !w.trace &&
      (which == SKV_STAGE_LOHI || which == SKV_STAGE_TAGS || which == SKV_STAGE_SELECTED ||
       which == SKV_STAGE_POOL || which == SKV_STAGE_U15 || which == SKV_STAGE_CAND))
    return fail(SKV_E_STATE, "this stage's intermediates need an engine created with SKV_FLAG_TRACE");
  switch (which) {
    case SKV_STAGE_COUNTS: src = w.counts + c0 * NCOUNT; n = G * NCOUNT * 4; break;
    case SKV_STAGE_LEAD_COUNTS:
      if (!w.lead) return fail(SKV_E_STATE, "the engine has no lead cluster");
      src = w.counts + (size_t)e->n_cells * NCOUNT;
      n = NCOUNT * 4;
      break;
    case SKV_STAGE_THRESH: {
      std::vector<uint32_t> t((size_t)G * 16);
      CK(cudaMemcpy(t.data(), w.thr + c0 * 16, t.size() * 4, cudaMemcpyDeviceToHost));
      std::vector<uint16_t> o(G * G);
      for (int g = 0; g < G; ++g)
        for (int h = 0; h < G; ++h) {
          const uint32_t ordv = t[(size_t)g * 16 + T_COARSE * G + h];
          o[g * G + h] = (uint16_t)((ordv & 0x8000u) ? (ordv ^ 0x8000u) : (~ordv & 0xffffu));
        }
      n = std::min(bytes, o.size() * 2);
      std::memcpy(dst, o.data(), n);
      if (written) *written = n;
      return SKV_OK;
    }
    case SKV_STAGE_TAGS: src = w.tags + c0 * nc; n = G * nc * 4; break;
    case SKV_STAGE_SELECTED: src = w.sel + c0 * SEL_MAX; n = (size_t)G * SEL_MAX * 4; break;
    case SKV_STAGE_POOL: src = w.pool + c0 * cap; n = G * cap * 4; break;
    case SKV_STAGE_U15: src = w.u15pos + c0 * U15_MAX; n = (size_t)G * U15_MAX * 4; break;
    case SKV_STAGE_CAND: src = w.cand + c0 * CAND_MAX; n = (size_t)G * CAND_MAX * 4; break;
    case SKV_STAGE_FINAL_POS: src = w.final_pos + c0 * G * TOPK; n = (size_t)G * G * TOPK * 4; break;
    case SKV_STAGE_FINAL_KEYS: src = w.final_keys + c0 * G * TOPK; n = (size_t)G * G * TOPK * 4; break;
    case SKV_STAGE_LOHI: {
      // ordered keys back to BF16 patterns, [cell][lo/hi][head][nc]
      std::vector<uint16_t> lo(G * G * nc), hi(G * G * nc);
      CK(cudaMemcpy(lo.data(), w.lo + c0 * G * nc, lo.size() * 2, cudaMemcpyDeviceToHost));
      CK(cudaMemcpy(hi.data(), w.hi + c0 * G * nc, hi.size() * 2, cudaMemcpyDeviceToHost));
      std::vector<uint16_t> o(2 * lo.size());
      auto un = [](uint16_t v) -> uint16_t { return (v & 0x8000u) ? (v ^ 0x8000u) : (uint16_t)~v; };
      for (int g = 0; g < G; ++g)
        for (size_t i = 0; i < G * nc; ++i) {
          o[((size_t)g * 2 + 0) * G * nc + i] = un(lo[(size_t)g * G * nc + i]);
          o[((size_t)g * 2 + 1) * G * nc + i] = un(hi[(size_t)g * G * nc + i]);
        }
      n = std::min(bytes, o.size() * 2);
      std::memcpy(dst, o.data(), n);
      if (written) *written = n;
      return SKV_OK;
    }
    case SKV_STAGE_OFFSETS:
    case SKV_STAGE_VALUES:
    case SKV_STAGE_MATES: {
      // the live CSR set of each cell (appends flip it on the device)
      std::vector<CellDev> cd(G);
      CK(cudaMemcpy(cd.data(), e->dcells + c0, G * sizeof(CellDev), cudaMemcpyDeviceToHost));
      size_t done = 0;
      for (int g = 0; g < G && done < bytes; ++g) {
        if (!cd[g].offsets) return fail(SKV_E_STATE, "index not uploaded for this slot");
        int32_t np = 0;
        CK(cudaMemcpy(&np, cd[g].offsets + nc, sizeof np, cudaMemcpyDeviceToHost));
        const void *p = which == SKV_STAGE_OFFSETS ? (const void *)cd[g].offsets
                      : which == SKV_STAGE_VALUES ? (const void *)cd[g].values : (const void *)cd[g].mates;
        const size_t per = (which == SKV_STAGE_OFFSETS ? nc + 1 : (size_t)np) * sizeof(int32_t);
        const size_t m = std::min(per, bytes - done);
        if (m) CK(cudaMemcpy(static_cast<char *>(dst) + done, p, m, cudaMemcpyDeviceToHost));
        done += m;
      }
      if (written) *written = done;
      return SKV_OK;
    }
    case SKV_STAGE_PREFIX2:
    case SKV_STAGE_RESIDUAL2:
    case SKV_STAGE_RESIDUAL4:
    case SKV_STAGE_KV8:
    case SKV_STAGE_KEY_SCALE:
    case SKV_STAGE_LABELS: {
      if (which == SKV_STAGE_LABELS && !e->appends()) return fail(SKV_E_STATE, "the engine takes no appends");
      int32_t tcur = 0;
      if ((rc = device_context(e, &tcur))) return rc;
      const size_t T = tcur;
      const size_t row = which == SKV_STAGE_RESIDUAL4 ? 128 : which == SKV_STAGE_KV8 ? REC
                       : which == SKV_STAGE_LABELS ? 2 * sizeof(int32_t)
                       : which == SKV_STAGE_KEY_SCALE ? 0 : 64;
      const size_t per = which == SKV_STAGE_KEY_SCALE ? D * sizeof(float) : T * row;
      size_t done = 0;
      for (int g = 0; g < G && done < bytes; ++g) {
        const CellBufs &b = e->bufs[c0 + g];
        const void *p = which == SKV_STAGE_PREFIX2 ? (const void *)b.prefix2
                      : which == SKV_STAGE_RESIDUAL2 ? (const void *)b.residual2
                      : which == SKV_STAGE_RESIDUAL4 ? (const void *)b.residual4
                      : which == SKV_STAGE_KV8 ? (const void *)b.kv8
                      : which == SKV_STAGE_LABELS ? (const void *)b.labels : (const void *)b.key_scale;
        if (!p) return fail(SKV_E_STATE, "K/V not uploaded for this slot");
        const size_t m = std::min(per, bytes - done);
        CK(cudaMemcpy(static_cast<char *>(dst) + done, p, m, cudaMemcpyDeviceToHost));
        done += m;
      }
      if (written) *written = done;
      return SKV_OK;
    }
    default: return fail(SKV_E_INVALID, "unknown stage selector");
  }
  n = std::min(n, bytes);
  CK(cudaMemcpy(dst, src, n, cudaMemcpyDeviceToHost));
  if (written) *written = n;
  return SKV_OK;
}

// ------------------------------------------------------- sharded decode

namespace {
// Makes the device that owns `p` current (the shard kernels run where their data is).
int use_device_of(const void *p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess || a.type != cudaMemoryTypeDevice)
    return fail(SKV_E_INVALID, "expected a device pointer");
  CK(cudaSetDevice(a.device));
  return SKV_OK;
}
}  // namespace

int skv_shard_outputs(void *handle, int32_t slot, const uint32_t **keys, const int32_t **ids) {
  Engine *e = as_engine(handle);
  if (!e || !keys || !ids) return fail(SKV_E_INVALID, "null engine or output");
  if (slot < 0 || slot >= e->desc.n_slots) return fail(SKV_E_INVALID, "slot out of range");
  *keys = e->work.final_keys + (size_t)slot * G * G * TOPK;
  *ids = e->work.final_ids + (size_t)slot * G * G * TOPK;
  return SKV_OK;
}

int skv_shard_merge(const uint32_t *keys, const int32_t *ids, const int32_t *begin, int32_t n_shards,
                    int32_t n_cells, int32_t *out_gids, void *stream) {
  if (!keys || !ids || !begin || !out_gids) return fail(SKV_E_INVALID, "null buffer");
  if (n_shards < 1 || n_shards > shard_max_shards()) return fail(SKV_E_INVALID, "n_shards out of range");
  if (n_cells < 1 || n_cells % G) return fail(SKV_E_INVALID, "n_cells must be a positive multiple of 4");
  int rc = use_device_of(keys);
  if (rc) return rc;
  CK(launch_shard_merge(keys, ids, begin, n_shards, n_cells, out_gids, static_cast<cudaStream_t>(stream)));
  return SKV_OK;
}

int skv_shard_attention(void *handle, const int32_t *gids, int32_t token_begin, float *partials, void *stream) {
  Engine *e = as_engine(handle);
  if (!e || !gids || !partials) return fail(SKV_E_INVALID, "null engine or buffer");
  if (token_begin < 0) return fail(SKV_E_INVALID, "negative token_begin");
  int rc = ready(e);
  if (rc) return rc;
  CK(cudaSetDevice(e->desc.device));
  CK(launch_shard_attention(view_work(e), gids, token_begin, partials, static_cast<cudaStream_t>(stream)));
  e->host_io = false;
  return SKV_OK;
}

int skv_shard_setup(void *handle, int32_t rank, int32_t n_shards, const int32_t *begin, int32_t total, int32_t sink,
                    int32_t local, void *ipc_handles) {
  Engine *e = as_engine(handle);
  if (!e || !begin || !ipc_handles) return fail(SKV_E_INVALID, "null engine or buffer");
  if (n_shards < 1 || n_shards > SHARD_MAX || rank < 0 || rank >= n_shards)
    return fail(SKV_E_INVALID, "rank / n_shards out of range (at most 8 shards)");
  if (e->n_cells != SHARD_CELLS) return fail(SKV_E_INVALID, "a shard engine holds one slot");
  if (e->link.region) return fail(SKV_E_STATE, "shard group already set up");
  for (int c = 0; c < SHARD_CELLS; ++c)
    if (!e->kv_ok[c]) return fail(SKV_E_STATE, "upload K/V before skv_shard_setup");
  if (sink < 0 || local < 0 || sink + local > total || begin[0] != 0)
    return fail(SKV_E_INVALID, "inconsistent layer context / zones");
  CK(cudaSetDevice(e->desc.device));
  for (int p = 0; p < n_shards; ++p) e->link.begin[p] = begin[p];
  e->link.total = total;
  e->link.total_max = total + (e->tmax - e->desc.context);
  e->link.sink = sink;
  e->link.local = local;
  e->link.rank = rank;
  e->link.n = n_shards;
  CK(cudaMalloc(&e->link.region, shard_region_bytes()));
  CK(cudaMemset(e->link.region, 0, shard_region_bytes()));
  int rc = dalloc(e, &e->link.epoch, 2);  // [0] steps completed, [1] the fused step's finished clusters
  if (!rc) rc = dalloc(e, &e->link.gids, (size_t)SHARD_CELLS * G * TOPK);
  if (!rc) rc = dalloc(e, &e->link.part, (size_t)SHARD_CELLS * G * PART);
  if (rc) return rc;
  // the exchange region, then the four FP8 record buffers
  cudaIpcMemHandle_t h;
  char *out = static_cast<char *>(ipc_handles);
  CK(cudaIpcGetMemHandle(&h, e->link.region));
  std::memcpy(out, &h, sizeof(h));
  for (int c = 0; c < SHARD_CELLS; ++c) {
    CK(cudaIpcGetMemHandle(&h, e->bufs[c].kv8));
    std::memcpy(out + (size_t)(1 + c) * sizeof(h), &h, sizeof(h));
  }
  return SKV_OK;
}

int skv_shard_connect(void *handle, const void *ipc_handles) {
  Engine *e = as_engine(handle);
  if (!e || !ipc_handles) return fail(SKV_E_INVALID, "null engine or handles");
  if (!e->link.region) return fail(SKV_E_STATE, "skv_shard_setup first");
  if (e->link.active) return fail(SKV_E_STATE, "shard group already connected");
  CK(cudaSetDevice(e->desc.device));
  for (int p = 0; p < e->link.n; ++p) {
    if (p == e->link.rank) continue;
    cudaIpcMemHandle_t h;
    const char *in = static_cast<const char *>(ipc_handles) + (size_t)p * (1 + SHARD_CELLS) * sizeof(h);
    std::memcpy(&h, in, sizeof(h));
    CK(cudaIpcOpenMemHandle(&e->link.opened[p], h, cudaIpcMemLazyEnablePeerAccess));
    for (int c = 0; c < SHARD_CELLS; ++c) {
      std::memcpy(&h, in + (size_t)(1 + c) * sizeof(h), sizeof(h));
      CK(cudaIpcOpenMemHandle(&e->link.kv8[p][c], h, cudaIpcMemLazyEnablePeerAccess));
    }
  }
  CK(cudaDeviceSynchronize());
  if (!e->link.dev) {
    int rc = dalloc(e, &e->link.dev, 1);
    if (rc) return rc;
  }
  const ShardLinkDev view = link_view(e);
  CK(cudaMemcpy(e->link.dev, &view, sizeof(view), cudaMemcpyHostToDevice));
  e->link.active = true;
  // the step graphs are captured again with the group's exchanges
  drop_graphs(e);
  return SKV_OK;
}

int32_t skv_shard_ipc_handle_bytes(void) { return (int32_t)((1 + SHARD_CELLS) * sizeof(cudaIpcMemHandle_t)); }

int skv_shard_gids(void *handle, const int32_t **gids) {
  Engine *e = as_engine(handle);
  if (!e || !gids) return fail(SKV_E_INVALID, "null engine or output");
  if (!e->link.gids) return fail(SKV_E_STATE, "skv_shard_setup first");
  *gids = e->link.gids;
  return SKV_OK;
}

int skv_shard_combine(const float *partials, int32_t n_shards, int32_t n_cells, uint16_t *out, void *stream) {
  if (!partials || !out) return fail(SKV_E_INVALID, "null buffer");
  if (n_shards < 1) return fail(SKV_E_INVALID, "n_shards out of range");
  if (n_cells < 1 || n_cells % G) return fail(SKV_E_INVALID, "n_cells must be a positive multiple of 4");
  int rc = use_device_of(partials);
  if (rc) return rc;
  CK(launch_shard_combine(partials, n_shards, n_cells, out, static_cast<cudaStream_t>(stream)));
  return SKV_OK;
}

int skv_traffic(void *handle, SkvTraffic *out) {
  Engine *e = as_engine(handle);
  if (!e || !out) return fail(SKV_E_INVALID, "null engine or output");
  int rc = sync_done(e);
  if (rc) return rc;
  std::vector<int32_t> c;
  if ((rc = read_counts(e, c))) return rc;
  const double nc = e->desc.nc;
  SkvTraffic t{};
  for (int i = 0; i < e->n_cells; ++i) {
    const int32_t *k = &c[(size_t)i * NCOUNT];
    t.coarse += nc * 64 + nc * 2 + nc / 32 * 4;           // upper plane, residual norm, scales
    t.fine += (double)k[C_TAGS] * (64 + 64 + 4);          // upper + lower rows of survivors, tags
    t.stage15 += (double)k[C_POSTINGS] * 8 + (double)std::min(k[C_POOL], e->desc.stage15_capacity) * 64 +
                 (double)k[C_SEL] * 8;                    // ids + mates, prefixes, offsets
    t.stage16 += (double)k[C_U15] * (64 + 64);            // prefix2 + residual2
    t.stage2 += (double)k[C_CAND] * (64 + 64 + 128);      // + residual4
    t.attention += (double)(e->desc.sink + e->desc.local + G * TOPK) * REC + G * D * 2;
  }
  t.total = t.coarse + t.fine + t.stage15 + t.stage16 + t.stage2 + t.attention;
  *out = t;
  return SKV_OK;
}

int skv_profile_step(void *handle, void *stream, float *kernel_ms, int32_t max_kernels, int32_t *n_kernels) {
  Engine *e = as_engine(handle);
  if (!e || !kernel_ms || !n_kernels) return fail(SKV_E_INVALID, "null engine or output");
  int rc = ready(e);
  if (rc) return rc;
  CK(cudaSetDevice(e->desc.device));
  cudaStream_t st = static_cast<cudaStream_t>(stream);  // NULL: legacy default stream
  const int nk = e->fused ? 1 : funnel_kernel_count();
  std::vector<cudaEvent_t> ev(nk + 1, nullptr);
  for (auto &x : ev) CK(cudaEventCreate(&x));
  cudaError_t le;
  e->host_io = false;
  if (e->fused) {
    cudaEventRecord(ev[0], st);
    le = launch_fused(view_work(e), st, window_of(e));
    cudaEventRecord(ev[1], st);
  } else {
    le = launch_funnel(view_work(e), st, ev.data());
  }
  cudaError_t se = le == cudaSuccess ? cudaEventSynchronize(ev[nk]) : le;
  const int n = std::min<int>(nk, max_kernels);
  for (int i = 0; i < n && se == cudaSuccess; ++i) se = cudaEventElapsedTime(&kernel_ms[i], ev[i], ev[i + 1]);
  for (auto &x : ev) cudaEventDestroy(x);
  if (se != cudaSuccess) return fail(SKV_E_CUDA, std::string("profile step: ") + cudaGetErrorString(se));
  CK(cudaEventRecord(e->done, st));
  e->ran = true;
  *n_kernels = n;
  return SKV_OK;
}

const char *skv_step_kernel_name(void *handle, int32_t i) {
  Engine *e = as_engine(handle);
  if (!e) return "";
  if (e->fused) return i == 0 ? "k_funnel" : "";
  return funnel_kernel_name(i);
}

int skv_profile_phases(void *handle, void *stream, int32_t *tags, double *cycles, int32_t max_marks,
                       int32_t *n_marks) {
  Engine *e = as_engine(handle);
  if (!e || !tags || !cycles || !n_marks) return fail(SKV_E_INVALID, "null engine or output");
  if (!e->fused) return fail(SKV_E_STATE, "phase timing needs the fused path");
  int rc = ready(e);
  if (rc) return rc;
  CK(cudaSetDevice(e->desc.device));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  std::vector<long long> ts(2 * FUSED_MARKS, -1);
  CK(cudaMemcpyAsync(e->phase_ts, ts.data(), ts.size() * sizeof(long long), cudaMemcpyHostToDevice, st));
  Work w = view_work(e);
  w.phase_ts = e->phase_ts;
  if (e->link.active) {  // a connected shard group: every shard must profile this step together
    w.link = e->link.dev;
    w.shard_gids = e->link.gids;
  }
  e->host_io = false;
  CK(launch_fused(w, st, window_of(e)));  // (with a connected group, the kernel advances the step counter)
  CK(cudaMemcpyAsync(ts.data(), e->phase_ts, ts.size() * sizeof(long long), cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  CK(cudaEventRecord(e->done, st));
  e->ran = true;
  int n = 0;
  for (int i = 1; i < FUSED_MARKS && n < max_marks; ++i) {
    if (ts[2 * i] < 0) break;
    tags[n] = (int32_t)ts[2 * i];
    cycles[n] = (double)(ts[2 * i + 1] - ts[2 * i - 1]);
    ++n;
  }
  *n_marks = n;
  return SKV_OK;
}

int skv_profile_ctas(void *handle, void *stream, int64_t *start_ns, int64_t *end_ns, int32_t max_ctas,
                     int32_t *n_ctas, float *kernel_ms, int64_t *marks, int32_t max_marks) {
  Engine *e = as_engine(handle);
  if (!e || !start_ns || !end_ns || !n_ctas || !kernel_ms) return fail(SKV_E_INVALID, "null engine or output");
  if (!e->fused) return fail(SKV_E_STATE, "CTA timing needs the fused path");
  if (e->link.active) return fail(SKV_E_STATE, "CTA timing of a connected shard group is not supported");
  int rc = ready(e);
  if (rc) return rc;
  CK(cudaSetDevice(e->desc.device));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int nct = e->n_cells * 16;
  const size_t nts = 2 * (size_t)nct + 16 * 2 * (size_t)FUSED_MARKS;
  if (!e->cta_ts) {
    rc = dalloc(e, &e->cta_ts, nts);
    if (rc) return rc;
  }
  CK(cudaMemsetAsync(e->cta_ts, 0xff, nts * sizeof(long long), st));  // unused marks read as tag -1
  Work w = view_work(e);
  w.cta_ts = e->cta_ts;
  cudaEvent_t ev[2];
  CK(cudaEventCreate(&ev[0]));
  CK(cudaEventCreate(&ev[1]));
  e->host_io = false;
  cudaEventRecord(ev[0], st);
  cudaError_t le = launch_fused(w, st, window_of(e));
  cudaEventRecord(ev[1], st);
  std::vector<long long> ts(nts, 0);
  cudaError_t se = le == cudaSuccess ? cudaEventSynchronize(ev[1]) : le;
  if (se == cudaSuccess) se = cudaEventElapsedTime(kernel_ms, ev[0], ev[1]);
  if (se == cudaSuccess) se = cudaMemcpy(ts.data(), e->cta_ts, nts * sizeof(long long), cudaMemcpyDeviceToHost);
  cudaEventDestroy(ev[0]);
  cudaEventDestroy(ev[1]);
  if (se != cudaSuccess) return fail(SKV_E_CUDA, std::string("profile ctas: ") + cudaGetErrorString(se));
  CK(cudaEventRecord(e->done, st));
  e->ran = true;
  const int n = std::min<int>(nct, max_ctas);
  for (int i = 0; i < n; ++i) {
    start_ns[i] = ts[2 * i];
    end_ns[i] = ts[2 * i + 1];
  }
  *n_ctas = n;
  if (marks && max_marks > 0) {
    for (int r = 0; r < 16; ++r)
      for (int j = 0; j < max_marks; ++j)
        for (int k = 0; k < 2; ++k)
          marks[((size_t)r * max_marks + j) * 2 + k] =
              j < FUSED_MARKS ? ts[2 * (size_t)nct + ((size_t)r * FUSED_MARKS + j) * 2 + k] : -1;
  }
  return SKV_OK;
}

const char *skv_phase_name(int32_t tag) { return fused_mark_name(tag); }

const char *skv_kernel_name(int32_t i) { return funnel_kernel_name(i); }

int32_t skv_kernels_per_step(void) { return funnel_kernel_count(); }

}  // extern "C"
