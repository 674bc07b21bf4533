// skv_noalloc.cu -- sparse attention entry point that performs no allocation.
//
// Some callers cannot allocate device memory once they are running: a
// serving process that reserves its whole HBM budget at start-up treats any
// later cudaMalloc as a failure (the budget is already committed, and
// cudaMalloc synchronises the device, stalling every other stream on it).
// skv_attention_noalloc serves them: the caller passes every input and output
// buffer, and the only scratch (the per-partition softmax partials and the
// arrival counters) lives in the fixed-size file-scope arrays below, which
// each GPU that loads this library keeps until the process exits.
//
// It computes the same attention as the last stage of skv_run: for every
// query head, softmax(q . k / 16) v over the sink tokens, the local tokens
// and the head's 100 selected tokens (FP8-e4m3 [K | V] records), combined
// across partitions with a log-sum-exp merge and rounded to BF16.
#include <cuda_fp8.h>

#include <mutex>
#include <string>

#include "../../include/seoulkv_b200.h"
#include "skv_device.cuh"

namespace skv {
void set_last_error(const std::string &msg);  // defined with skv_last_error
}

namespace {

using namespace skv;

constexpr int NA_SPLIT = 32;       // partitions per KV head
constexpr int NA_PART = 260;       // floats per partial: m, l, 2 pad, o[256]
constexpr int NA_MAX_SLOTS = SKV_NOALLOC_MAX_SLOTS;
constexpr int NA_ITEMS = 4;

// Scratch shared by every call on a device: partials and arrival counters.
static __device__ __align__(256) float g_part[NA_MAX_SLOTS * G * G * NA_SPLIT * NA_PART];
static __device__ __align__(256) unsigned g_arrive[NA_MAX_SLOTS * G];

struct KvPtrs {
  const uint8_t *p[NA_MAX_SLOTS * G];
};

__device__ __forceinline__ void na_fp8x8(uint2 v, float *o) {
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

__global__ void __launch_bounds__(256) k_attn_noalloc(const uint16_t *q, KvPtrs kv, const int32_t *ids, int T,
                                                      int sink, int local, uint16_t *out, float *part_all,
                                                      unsigned *arrive) {
  const int split = blockIdx.x, cell = blockIdx.y, slot = cell >> 2, g = cell & 3;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint8_t *kv8 = kv.p[cell];
  const int dense = sink + local, nitems = dense + G * TOPK;
  const float qscale = 0.0625f * 1.4426950408889634f;
  __shared__ float s_m[G][8], s_l[G][8];
  __shared__ float s_o[8][D];
  __shared__ int s_last;
  __shared__ __align__(16) float s_part[NA_SPLIT][NA_PART];
  float qv[G][8];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    const uint4 raw = *reinterpret_cast<const uint4 *>(q + ((size_t)slot * 16 + g * 4 + h) * D + 8 * lane);
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
  const int step = NA_SPLIT * 8;
  for (int k0 = split * 8 + warp; k0 < nitems; k0 += step * NA_ITEMS) {
    int tok[NA_ITEMS], head[NA_ITEMS];
#pragma unroll
    for (int j = 0; j < NA_ITEMS; ++j) {
      const int it = k0 + j * step;
      head[j] = -1;
      if (it >= nitems) { tok[j] = -1; continue; }
      if (it < sink) { tok[j] = it; continue; }
      if (it < dense) { tok[j] = T - local + (it - sink); continue; }
      const int r = it - dense;
      head[j] = r / TOPK;
      const int t = ids[((size_t)cell * G + head[j]) * TOPK + r % TOPK];
      tok[j] = (t >= 0 && t < T) ? t : -1;
    }
    uint2 kb[NA_ITEMS], vb[NA_ITEMS];
#pragma unroll
    for (int j = 0; j < NA_ITEMS; ++j) {
      const uint8_t *rec = kv8 + (size_t)(tok[j] < 0 ? 0 : tok[j]) * REC;
      kb[j] = *reinterpret_cast<const uint2 *>(rec + 8 * lane);
      vb[j] = *reinterpret_cast<const uint2 *>(rec + 256 + 8 * lane);
    }
#pragma unroll
    for (int j = 0; j < NA_ITEMS; ++j) {
      if (tok[j] < 0) continue;
      float kf[8], vf[8];
      na_fp8x8(kb[j], kf);
      na_fp8x8(vb[j], vf);
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
  float *part = part_all + (size_t)cell * G * NA_SPLIT * NA_PART;
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
    float *dst = part + ((size_t)h * NA_SPLIT + split) * NA_PART;
    if (tid == 0) { dst[0] = M; dst[1] = L; }
    dst[4 + tid] = O;
    __syncthreads();
  }
  // whichever partition of this cell finishes last merges the partials
  __threadfence();
  if (tid == 0) s_last = atomicAdd(&arrive[cell], 1u) == NA_SPLIT - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int h = 0; h < G; ++h) {
    const float4 *ph = reinterpret_cast<const float4 *>(part + (size_t)h * NA_SPLIT * NA_PART);
    float4 *dst = reinterpret_cast<float4 *>(&s_part[0][0]);
    for (int i = tid; i < NA_SPLIT * NA_PART / 4; i += 256) dst[i] = __ldcg(ph + i);
    __syncthreads();
    float M = -INFINITY;
#pragma unroll
    for (int sp = 0; sp < NA_SPLIT; ++sp) M = fmaxf(M, s_part[sp][0]);
    float L = 0.0f, O = 0.0f;
#pragma unroll
    for (int sp = 0; sp < NA_SPLIT; ++sp) {
      const float ms = s_part[sp][0];
      if (ms == -INFINITY) continue;
      const float e = exp2f(ms - M);
      L += s_part[sp][1] * e;
      O += s_part[sp][4 + tid] * e;
    }
    // a head with no key to attend (no dense zones and no selected id inside
    // the context) gets zeros rather than 0/0
    out[((size_t)slot * 16 + g * 4 + h) * D + tid] = L > 0.0f ? bf16_rne(O / L) : (uint16_t)0;
    __syncthreads();
  }
  if (tid == 0) arrive[cell] = 0;
}

// Device addresses of the scratch arrays, looked up once per device.
struct ScratchAddr {
  bool ready = false;
  float *part = nullptr;
  unsigned *arrive = nullptr;
};
constexpr int kMaxDevices = 64;
ScratchAddr g_addr[kMaxDevices];
std::mutex g_addr_lock;
int na_fail(int code, const char *msg, cudaError_t e = cudaSuccess) {
  std::string m = msg;
  if (e != cudaSuccess) m += std::string(": ") + cudaGetErrorString(e);
  skv::set_last_error(m);  // reported by skv_last_error()
  return code;
}

}  // namespace

extern "C" {

int skv_attention_noalloc(int32_t n_slots, const uint16_t *q, const uint8_t *const *kv8, const int32_t *ids,
                          int32_t context, int32_t sink, int32_t local, uint16_t *out, void *stream) {
  if (n_slots < 1 || n_slots > NA_MAX_SLOTS)
    return na_fail(SKV_E_INVALID, "n_slots outside [1, SKV_NOALLOC_MAX_SLOTS]: the fixed scratch holds "
                                  "partials for at most SKV_NOALLOC_MAX_SLOTS slots");
  if (!q || !kv8 || !ids || !out) return na_fail(SKV_E_INVALID, "null input or output pointer");
  if (context < 1 || sink < 0 || local < 0 || sink + local > context)
    return na_fail(SKV_E_INVALID, "sink/local must be disjoint and inside the context");
  KvPtrs kv{};
  for (int i = 0; i < n_slots * G; ++i) {
    if (!kv8[i]) return na_fail(SKV_E_INVALID, "null FP8 record pointer");
    kv.p[i] = kv8[i];
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return na_fail(SKV_E_CUDA, "cudaGetDevice", e);
  if (dev < 0 || dev >= kMaxDevices) return na_fail(SKV_E_INVALID, "device ordinal out of range");
  ScratchAddr addr;
  {
    // first call on this device: resolve the scratch arrays' device addresses
    std::lock_guard<std::mutex> lock(g_addr_lock);
    if (!g_addr[dev].ready) {
      void *p = nullptr;
      e = cudaGetSymbolAddress(&p, g_part);
      if (e != cudaSuccess) return na_fail(SKV_E_CUDA, "cudaGetSymbolAddress(partials)", e);
      g_addr[dev].part = static_cast<float *>(p);
      e = cudaGetSymbolAddress(&p, g_arrive);
      if (e != cudaSuccess) return na_fail(SKV_E_CUDA, "cudaGetSymbolAddress(counters)", e);
      g_addr[dev].arrive = static_cast<unsigned *>(p);
      g_addr[dev].ready = true;
    }
    addr = g_addr[dev];
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // arrival counters must start at zero (a previous call may have been cut short)
  e = cudaMemsetAsync(addr.arrive, 0, sizeof(unsigned) * n_slots * G, st);
  if (e != cudaSuccess) return na_fail(SKV_E_CUDA, "clearing the arrival counters", e);
  k_attn_noalloc<<<dim3(NA_SPLIT, n_slots * G), 256, 0, st>>>(q, kv, ids, context, sink, local, out, addr.part,
                                                              addr.arrive);
  e = cudaGetLastError();
  if (e != cudaSuccess) return na_fail(SKV_E_CUDA, "k_attn_noalloc launch", e);
  return SKV_OK;
}

}  // extern "C"
