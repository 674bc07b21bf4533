/*
 * seoulkv_b200.h -- C ABI of the B200 SeoulKV4 sparse-decode engine.
 *
 * Plain C types only: device and host buffers are raw pointers with sizes,
 * streams are `void*` (a cudaStream_t; NULL is CUDA's legacy default stream).
 * Every function returns 0 on success and a negative SKV_E_* code on error;
 * skv_last_error() then describes the failure (thread-local).
 *
 * One engine instance serves `n_slots` independent cache snapshots (a slot
 * is one request, or one layer of a stack).  Each slot has four KV heads
 * ("cells") with their own index.  One skv_run() decodes one query token for
 * every slot.
 *
 * Counterparts in the reference (daniel-geon-park/SeoulKV, src/seoulkv4):
 *   skv_create        SeoulKV4.__init__                       api.py:16-55
 *   skv_upload_index  index upload inside _runtime.initialize   _runtime.py:36-47
 *   skv_upload_kv     key planes + FP8 [V|K] record upload       _runtime.py:48-92
 *   skv_bind_query    SeoulKV4._bind_query / query_prepare.bind api.py:70-73,
 *                                                            _kernels/query_prepare/host.py:309-319
 *   skv_run           _runtime.enqueue (4 programs, no sync)     _runtime.py:189-194
 *   skv_sync          SeoulKV4.synchronize                     api.py:104-107
 *   skv_status        capacity / live-count checks              _kernels/stage1_fine/seoulkv4_stage1_live.py:72-77,
 *                                                            _kernels/stage15/seoulkv4_stage15_ingest.py:38-42
 *   skv_debug_ids     SeoulKV4.debug_snapshot                  api.py:119-126
 *   skv_output        DecodeResult.to_torch / device_tensors   result.py:25-38
 *   skv_destroy       SeoulKV4.close                           api.py:128-137
 */
#ifndef SEOULKV_B200_H
#define SEOULKV_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SKV_OK 0
#define SKV_E_INVALID (-1)    /* bad argument, shape or state            */
#define SKV_E_CUDA (-2)       /* a CUDA runtime call failed              */
#define SKV_E_CAPACITY (-3)   /* a live count left its allowed range     */
#define SKV_E_STATE (-4)      /* wrong lifecycle order (e.g. run before upload) */

/* Status word bits reported per cell by the device (skv_status). */
#define SKV_STATUS_POOL_OVER 1u   /* Stage-1.5 pool larger than capacity  */
#define SKV_STATUS_POOL_UNDER 2u  /* Stage-1.5 pool smaller than 2048     */
#define SKV_STATUS_FINE_SHORT 4u  /* a head had fewer than nprobe survivors */
#define SKV_STATUS_TIMEOUT 8u     /* a bounded device wait gave up (results invalid) */
#define SKV_STATUS_APPEND_FULL 16u /* an append replayed from a graph did not fit max_context (skipped) */
#define SKV_STATUS_APPEND_NONFINITE 32u /* an appended key had a non-finite element (assigned as 0) */

/* SkvDesc.flags */
#define SKV_FLAG_STAGED 1         /* run the 14-kernel staged path even where the
                                     single-kernel cluster path applies      */
#define SKV_FLAG_TRACE 4          /* the fused path writes every stage's intermediates
                                     (coarse bounds, survivor tags, selected clusters,
                                     pool, unions) for skv_read_stage; without it
                                     only the counters, thresholds and final ranks
                                     are written (the staged path always writes them) */
#define SKV_FLAG_NO_LEAD 2        /* fused path without its lead cluster: one
                                     extra 16-CTA cluster in every launch that
                                     decodes a small built-in synthetic cell,
                                     runs ahead of the real cells and so brings
                                     the kernel's instructions into L2 before
                                     they need them (results do not depend on
                                     it; off only to measure it)             */

typedef struct SkvDesc {
    int32_t n_slots;          /* independent caches decoded per run        */
    int32_t context;          /* T, tokens per cache                       */
    int32_t sink;             /* dense prefix tokens                       */
    int32_t local;            /* dense suffix tokens                       */
    int32_t nc;               /* centroids per KV head (multiple of 32)    */
    int32_t stage15_capacity; /* pool slots per KV head                    */
    int32_t device;           /* CUDA device ordinal                       */
    int32_t flags;            /* SKV_FLAG_* (0: fused path where it applies) */
    int32_t max_context;      /* capacity for skv_append (0: context, no appends) */
} SkvDesc;

/* One KV head's index in the engine layout (host memory). */
typedef struct SkvCellView {
    int32_t nc;
    int32_t nprobe;               /* multiple of 16 in [16, min(512, nc)] */
    float lam;                    /* interval lambda                      */
    int32_t n_postings;           /* offsets[nc]                          */
    const uint8_t *upper;         /* [nc][64]  code >> 2, 4 codes/byte LE */
    const uint8_t *lower;         /* [nc][64]  code & 3                   */
    const float *coarse_scale4;   /* [nc/32]   group scale / 4            */
    const float *fine_scale;      /* [nc/32]   FP16 group fine scale      */
    const uint16_t *resid_bf16;   /* [nc]      BF16 residual norm         */
    const int32_t *offsets;       /* [nc+1]    CSR offsets                */
    const int32_t *values;        /* [n_postings] token ids               */
    const int32_t *mates;         /* [n_postings] other list of the token, or -1 */
} SkvCellView;

typedef struct SkvStatus {
    uint32_t flags;               /* OR of SKV_STATUS_* over all cells    */
    int32_t first_bad_cell;       /* -1 when flags == 0                   */
    int32_t survivors_max;        /* largest coarse survivor count        */
    int32_t pool_max;             /* largest Stage-1.5 pool               */
    int32_t pool_min;             /* smallest Stage-1.5 pool              */
    int32_t union15_max;          /* largest Stage-1.5 union              */
    int32_t union16_max;          /* largest Stage-II candidate set       */
    int32_t reserved;
} SkvStatus;

const char *skv_last_error(void);
const char *skv_version(void);

int skv_create(const SkvDesc *desc, void **handle);
void skv_destroy(void *handle);

/* cells[4] for one slot.  Copies everything; the caller keeps ownership. */
int skv_upload_index(void *handle, int32_t slot, const SkvCellView *cells);

/* K and V: BF16 bit patterns [4][T][256] for one slot, host or device memory.
 * Builds the key code planes and the FP8-e4m3 [K|V] records on the GPU. */
int skv_upload_kv(void *handle, int32_t slot, const uint16_t *k, const uint16_t *v,
                  int32_t on_device);

/* Q: BF16 bit patterns [n_slots][16][256], host or device memory.  Device
 * memory is copied on `stream` now.  Host memory is copied into a pinned
 * staging buffer now and reaches the device inside the next skv_run's step
 * graph, which then also copies the output and the counters back into pinned
 * host memory (skv_output to host and skv_status read them from there): a
 * host-I/O step costs one graph launch and one wait. */
int skv_bind_query(void *handle, const uint16_t *q, int32_t on_device, void *stream);

/* Enqueue the whole funnel for every slot on `stream` (no host sync), as a
 * replay of the engine's own step graph.  While `stream` is capturing (the
 * caller records its own CUDA graph, e.g. a model's decode step), the step's
 * kernels are captured into the caller's graph instead; the query must then
 * be device-resident (SKV_E_STATE otherwise). */
int skv_run(void *handle, void *stream);

/* Keep the centroid planes (upper and lower, nc * 128 bytes per cell, all
 * cells in one arena) resident in L2 across steps: the counterpart of the
 * reference uploading its coarse centroid plane into on-chip SRAM
 * (_upload(..., dram=False) in
 * src/seoulkv4/_kernels/stage1_coarse/seoulkv4_coarse_score.py:120,195).
 * enable != 0 puts an access-policy window (hits persisting) over the arena
 * on the fused funnel's launch and raises this process's persisting-L2
 * set-aside by the arena's size; enable == 0 removes the window and, when no
 * engine of the process holds one any more, restores the set-aside the
 * process had.  The set-aside is state of the calling process's CUDA
 * context (it ends with the process).  *resident_bytes (if not NULL) gets
 * the bytes now held resident: 0 on the staged path, or when the device's
 * largest window or set-aside cannot hold the arena (then nothing changes).
 * Waits for the engine's work; the step graphs are captured again. */
int skv_set_l2_residency(void *handle, int32_t enable, size_t *resident_bytes);

/* skv_bind_query + skv_run in one call (one host crossing per step). */
int skv_step(void *handle, const uint16_t *q, int32_t on_device, void *stream);

/* Wait for the last step, fill *status (if not NULL) and copy the output
 * [n_slots][16][256] BF16 into host memory `out` (if not NULL); returns
 * SKV_E_CAPACITY, after filling both, when a cell reported a live count out
 * of range.  skv_sync + skv_status + skv_output in one call. */
int skv_finish(void *handle, uint16_t *out, SkvStatus *status);

/* Wait for all work of this engine, then check the device status words:
 * returns SKV_E_CAPACITY if any cell reported a live count out of range. */
int skv_sync(void *handle);
int skv_status(void *handle, SkvStatus *out);

/* Output BF16 bit patterns [n_slots][16][256].  to_host=1 copies to `out`
 * (synchronising), to_host=0 writes the device pointer into *(void**)out. */
int skv_output(void *handle, void *out, int32_t to_host);

/* Selected token ids of the last run: int32 [n_slots][4][4][100] (KV head,
 * query head, rank).  Synchronises. */
int skv_debug_ids(void *handle, int32_t *out);

/* Cache append (no counterpart in the reference, whose cache is static: its
 * README.md:68-69 lists appends as out of scope; the build path this extends
 * is src/seoulkv4/_index_build.py:22-59 and _codecs/keys.py:16-44).  Appends n_tokens
 * tokens to every slot: k and v are BF16 [n_slots][4][n_tokens][256]
 * (host memory, or device memory with on_device != 0).  Each new token gets
 * its key planes (with the build's per-dimension scales, codes clamped to
 * 0..255) and FP8 record at positions T..T+n-1, and its two spill-2 lists:
 * the top-2 stored centroids by
 *     S(k, c) = fl64(X(k, c) * fine_scale_c),  X(k, c) = sum_d x_d (2 code_cd - 15)
 * with x the key on the decode's operand grid (elements below 2^(E-22) of
 * its top exponent E flushed, the rest integers on the 2^(E-29) grid), X
 * exact, ties to the lower centroid: the Fine score with the key as the
 * query.  The tokens leaving
 * the local window (T-local .. T-local+n-1) join their two lists after the
 * lists' current postings.  The context then advances by n on the device,
 * so decode steps replayed from graphs, and appends captured in one, see
 * it.  Needs SkvDesc.max_context above the context; n_tokens in [1, 512];
 * stream-ordered (no host wait for device input); uploads are closed
 * afterwards.  SKV_E_CAPACITY when the append would pass max_context (a
 * replayed append that does not fit is skipped and raises
 * SKV_STATUS_APPEND_FULL instead).  Keys are checked on the device: a
 * non-finite element counts as 0 in the assignment and raises
 * SKV_STATUS_APPEND_NONFINITE.  Both bits stay set for the engine's life
 * (skv_sync and skv_finish then fail).  In a connected shard group every
 * shard calls it with the same n_tokens (each engine created with the same
 * room to grow): the last shard, which holds the local window, appends the
 * tokens as above; every shard's device copy of the layer's length grows by
 * n, so the in-kernel merge and attention see the grown layer. */
int skv_append(void *handle, const uint16_t *k, const uint16_t *v, int32_t n_tokens, int32_t on_device,
               void *stream);
/* The slots' current context, after every enqueued append (waits). */
int skv_context(void *handle, int32_t *context);

/* Intermediate buffers of the last run, for diagnostics and parity tests.
 * `which` selects one of SKV_STAGE_*; copies at most `bytes` bytes of the
 * given slot's four cells (cell-major) and returns the byte count in *written.
 * On the fused path TAGS, SELECTED, POOL, U15, CAND and LOHI are written only
 * by an engine created with SKV_FLAG_TRACE (SKV_E_STATE otherwise). */
#define SKV_STAGE_COUNTS 0      /* int32 [4][8]: ntags,nsel,npool,nu15,ncand,status,0,0 */
#define SKV_STAGE_THRESH 1      /* uint16 [4][4] coarse thresholds (BF16 bits) */
#define SKV_STAGE_TAGS 2        /* uint32 [4][nc] survivor tags                */
#define SKV_STAGE_SELECTED 3    /* int32 [4][2048] Fine cluster ids            */
#define SKV_STAGE_POOL 4        /* int32 [4][capacity] pool token ids          */
#define SKV_STAGE_U15 5         /* int32 [4][6400] pool positions              */
#define SKV_STAGE_CAND 6        /* int32 [4][1024] Stage-1.5 union positions   */
#define SKV_STAGE_FINAL_POS 7   /* int32 [4][4][100] Stage-1.5 union positions */
#define SKV_STAGE_LOHI 8        /* uint16 [4][2][4][nc] coarse lo, hi (BF16)   */
#define SKV_STAGE_PREFIX2 9     /* uint8 [4][T][64]  key codes >> 6            */
#define SKV_STAGE_RESIDUAL2 10  /* uint8 [4][T][64]  (key codes >> 4) & 3      */
#define SKV_STAGE_RESIDUAL4 11  /* uint8 [4][T][128] key codes & 15            */
#define SKV_STAGE_KV8 12        /* uint8 [4][T][512] FP8-e4m3 [K | V] records  */
#define SKV_STAGE_KEY_SCALE 13  /* float [4][256] per-dimension max |k|        */
#define SKV_STAGE_FINAL_KEYS 14 /* uint32 [4][4][100] Stage-II keys of the ranks (0: none) */
#define SKV_STAGE_OFFSETS 15    /* int32 [4][nc+1] live CSR offsets              */
#define SKV_STAGE_VALUES 16     /* int32 per cell offsets[nc] token ids, cell after cell */
#define SKV_STAGE_MATES 17      /* int32 per cell offsets[nc] mates, cell after cell     */
#define SKV_STAGE_LABELS 18     /* int32 [4][T][2] spill-2 lists of tokens from the first local window on
                                   (engines with appends; -1 below the window)     */
#define SKV_STAGE_LEAD_COUNTS 19 /* int32 [8] counters of the lead cluster's synthetic cell
                                   (see SKV_FLAG_NO_LEAD), in the order of SKV_STAGE_COUNTS:
                                   ntags, nsel, npool, nu15, ncand, status, postings, 0;
                                   slot is ignored (must be valid) */
int skv_read_stage(void *handle, int32_t slot, int32_t which, void *dst, size_t bytes,
                   size_t *written);

/* Bytes the funnel read on the last run (from the live counts): the
 * algorithmic traffic used for roofline reporting, per stage, summed over slots. */
typedef struct SkvTraffic {
    double coarse, fine, stage15, stage16, stage2, attention, total;
} SkvTraffic;
int skv_traffic(void *handle, SkvTraffic *out);

/* One decode step launched kernel by kernel (no graph) with a CUDA event
 * between kernels; writes each kernel's device time in milliseconds to
 * kernel_ms[0..n) (n = min(max_kernels, kernels per step)) and n to
 * *n_kernels.  Synchronises.  For profiling; results equal skv_run's. */
int skv_profile_step(void *handle, void *stream, float *kernel_ms, int32_t max_kernels,
                     int32_t *n_kernels);
/* Name of kernel i of the STAGED path (static string; "" when out of range). */
const char *skv_kernel_name(int32_t i);
/* Kernels one step of the STAGED path enqueues. */
int32_t skv_kernels_per_step(void);
/* Name of kernel i of this engine's step: "k_funnel" (one kernel) on the
 * fused path, the staged names otherwise. */
const char *skv_step_kernel_name(void *handle, int32_t i);
/* One fused step with SM-clock marks between its phases (CTA 0 of cell 0):
 * segment i ends at mark tags[i] and took cycles[i] SM cycles; n =
 * min(max_marks, marks).  Synchronises.  SKV_E_STATE on the staged path.
 * In a connected shard group this is a whole group step: every shard must
 * call it together. */
int skv_profile_phases(void *handle, void *stream, int32_t *tags, double *cycles, int32_t max_marks,
                       int32_t *n_marks);
/* Name of a phase mark tag (static string). */
const char *skv_phase_name(int32_t tag);

/* One launch of the fused kernel with every CTA's global-timer stamps (ns)
 * at entry and at exit: start_ns[i] / end_ns[i] for CTA i = cell * 16 +
 * cluster rank (n_ctas = cells * 16, at most max_ctas), and the launch's
 * event-timed duration in *kernel_ms.  With marks != NULL, also the phase
 * marks of the 16 CTAs of cell 0: marks[(r * max_marks + j) * 2 + {0, 1}] =
 * (tag, global-timer ns) of mark j of CTA r, tag -1 past the last (tags as
 * skv_phase_name).  Launch skew, the tail of the slowest cell and the CTA on
 * the critical path of each phase are read from it.  Fused path, unconnected
 * engine only.  No counterpart in the reference (profiling of this build). */
int skv_profile_ctas(void *handle, void *stream, int64_t *start_ns, int64_t *end_ns, int32_t max_ctas,
                     int32_t *n_ctas, float *kernel_ms, int64_t *marks, int32_t max_marks);

/* Sequence-sharded decode -- no counterpart in the reference (its decode is
 * single-device).  A long context is split into contiguous token ranges,
 * one engine per GPU (sink zone on the first shard, local window on the
 * last, sink = local = 0 on the others); after skv_run each shard's local
 * top-100 per head is merged into the same global top-100 on every GPU,
 * every shard attends over the winners it owns plus its dense zones, and the
 * shards' partials are combined.  The host moves the lists and partials
 * between GPUs (an all-gather each); every pointer below is device memory
 * and every call is ordered on `stream`.
 *
 * skv_shard_outputs: this engine's per-rank Stage-II keys and shard-local
 *   token ids of slot `slot`, [4][4][100] each (key 0: rank unused).  Valid
 *   after the step that wrote them completes; overwritten by the next run. */
int skv_shard_outputs(void *handle, int32_t slot, const uint32_t **keys, const int32_t **ids);
/* Exact global top-100 per (cell, head): candidates ordered by Stage-II score
 * (descending), then local rank, then global token id (ascending).
 *   keys, ids  [n_shards][n_cells][4][100] as skv_shard_outputs gives them
 *   begin      [n_shards] first global token of each shard
 *   out_gids   [n_cells][4][100] global token ids, -1 past the winners
 * n_shards <= 10. */
int skv_shard_merge(const uint32_t *keys, const int32_t *ids, const int32_t *begin, int32_t n_shards,
                    int32_t n_cells, int32_t *out_gids, void *stream);
/* This shard's partial attention for every cell of the engine over its
 * dense zones and the winners of `gids` ([n_cells][4][100] global ids) in
 * [token_begin, token_begin + context): partials [n_cells][4][260] floats =
 * (m, l, 0, 0, o[256]) with scores in the log2 domain, o not normalised.
 * Uses the query of the last skv_bind_query. */
int skv_shard_attention(void *handle, const int32_t *gids, int32_t token_begin, float *partials, void *stream);
/* Log-sum-exp combine: partials [n_shards][n_cells][4][260] -> out BF16
 * [n_cells / 4][16][256]. */
int skv_shard_combine(const float *partials, int32_t n_shards, int32_t n_cells, uint16_t *out, void *stream);

/* Sequence-sharded group over peer memory (NVLink), without a collective
 * library.  skv_shard_setup (after skv_upload_kv; one slot, n_shards <= 8;
 * begin = host array of every shard's first global token; total / sink /
 * local = the whole layer's context and dense zones) allocates this shard's
 * exchange region and writes skv_shard_ipc_handle_bytes() bytes of CUDA IPC
 * handles (the region and the four FP8 record buffers) to ipc_handles; after
 * the caller has moved every shard's handles to every shard,
 * skv_shard_connect (n_shards x that many bytes, in shard order) maps the
 * peers' memory.  From then on every skv_run is the whole layer step: the
 * funnel; every shard writes its top-100 lists straight into every peer's
 * region and waits (bounded; SKV_STATUS_TIMEOUT on expiry) for the others';
 * the merged global winners and the dense zones are attended with their
 * records read from the owning shard's memory, so skv_output gives the
 * layer's BF16 output on every shard.  All shards must call skv_run once per
 * step. */
int skv_shard_setup(void *handle, int32_t rank, int32_t n_shards, const int32_t *begin, int32_t total,
                    int32_t sink, int32_t local, void *ipc_handles);
int skv_shard_connect(void *handle, const void *ipc_handles);
int32_t skv_shard_ipc_handle_bytes(void);
/* Device address of the connected group's global winners [4][4][100]
 * (global token ids, -1 past the end) of the last step. */
int skv_shard_gids(void *handle, const int32_t **gids);

/* Sparse attention that allocates nothing -- no counterpart in the reference.
 *
 * For callers that cannot allocate device memory while running (for example
 * a server that commits its whole HBM budget at start-up and treats a later
 * cudaMalloc as a failure, since cudaMalloc also synchronises the device).
 * Computes what the last stage of skv_run computes, from caller buffers:
 *   q    device BF16 [n_slots][16][256]
 *   kv8  host array of n_slots*4 device pointers, each FP8-e4m3 records
 *        [context][512] = K (256 B) | V (256 B) of one KV head
 *   ids  device int32 [n_slots][4][4][100] selected token ids (KV head,
 *        query head, rank); ids outside [0, context) are skipped
 *   out  device BF16 [n_slots][16][256]; a query head left with no key at
 *        all (sink = local = 0 and every one of its ids skipped) gets zeros
 * Scratch is a fixed file-scope device array sized for SKV_NOALLOC_MAX_SLOTS
 * slots (about 1 MiB, held by every GPU that loads the library until the
 * process exits); larger n_slots is rejected with SKV_E_INVALID.  The first
 * call on a device looks up the scratch address (make that first call before
 * any stream capture).  All calls share the scratch: calls that overlap on the
 * GPU (e.g. on two streams) race and must be serialised by the caller. */
#define SKV_NOALLOC_MAX_SLOTS 2
int skv_attention_noalloc(int32_t n_slots, const uint16_t *q, const uint8_t *const *kv8, const int32_t *ids,
                          int32_t context, int32_t sink, int32_t local, uint16_t *out, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* SEOULKV_B200_H */
