// Allocation-free entry point for paged split-K decode attention.
//
// This entry point has no counterpart in the reference; it is an addition of this library.
//
// Who needs it: callers that cannot allocate device memory at the moment they run attention, for example
// code that runs inside a memory-allocator callback or an out-of-memory handler (allocating there would
// recurse into the allocator), hosts that embed the kernels in a runtime whose device memory is fully
// reserved up front and handed out only as fixed input/output buffers, and plain C/C++ or FFI callers
// that have no PyTorch caching allocator to borrow temporary buffers from. The regular
// `decode_attention` op needs the caller to pass split-K scratch buffers; this variant instead keeps
// that scratch in a fixed-size array that lives inside the loaded library, so a call needs nothing but
// the caller's inputs and outputs and performs no allocation of any kind.
//
// Contract:
//  * Scratch is the file-scope device array `g_noalloc_scratch` below: kNoAllocScratchFloats fp32 values
//    (4 MiB). Every GPU that loads this library holds those 4 MiB until the process exits.
//  * A call needs batch * num_q_heads * num_splits * (head_dim + 1) fp32 values of scratch; larger requests
//    are rejected with SNB_NOALLOC_ERR_TOO_LARGE before anything is launched.
//  * Host code cannot use the array's name as a device address. The first call made on a device (with that
//    device current) looks the address up with cudaGetSymbolAddress and caches it together with the
//    device's current context; a call that finds a different context (after cudaDeviceReset, which reloads
//    the module) looks it up again. Make the first call on a device outside any CUDA stream capture.
//  * A CUDA error already pending on the calling thread is reported (SNB_NOALLOC_ERR_PRIOR) and left
//    pending for its owner; the call then launches nothing.
//  * All calls share the one array and it keeps whatever the previous call left in it. Nothing in it has to
//    start at zero: each split writes every value the merge step later reads. Calls whose executions overlap
//    on the GPU (different streams, or different host threads without ordering) race on the array and must
//    be serialised by the caller.
//  * No cudaMalloc, cudaFree or allocating library routine is called.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "../common.cuh"
#include "../snb_noalloc.h"

namespace {

constexpr int kNoAllocScratchFloats = 1 << 20;  // 4 MiB of fp32 partial results
constexpr int kMaxDevices = 64;
constexpr float kLog2eNA = 1.4426950408889634f;
constexpr int kTileNA = 64;
constexpr int kThreadsNA = 128;

}  // namespace

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

namespace {

// Split partial pass: grid (splits, Hkv, B). Writes o (normalised per split) and lse (log2 domain) for
// every split, including empty ones (o = 0, lse = -inf), so the merge never reads stale values.
template <int D, int G, typename CacheT>
__global__ void __launch_bounds__(kThreadsNA) noalloc_split_kernel(
    const __nv_bfloat16* __restrict__ q, int q_stride, const CacheT* __restrict__ kc, const CacheT* __restrict__ vc,
    const int32_t* __restrict__ bt, int bt_stride, const int32_t* __restrict__ seq_lens, int page_size, int Hkv,
    int window, float scale_log2, float* __restrict__ o_part, float* __restrict__ lse_part, int S) {
  constexpr int RS = D + 8;
  __shared__ __align__(16) __nv_bfloat16 ks[kTileNA * RS];
  __shared__ __align__(16) __nv_bfloat16 vs[kTileNA * RS];
  __shared__ float qs[G * D];
  __shared__ float ps[G * kTileNA];
  __shared__ float ms[G], ls[G], al[G];
  const int split = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ctx = seq_lens[b];
  const int start = (window > 0 && ctx > window) ? ctx - window : 0;
  const int per = ((ctx - start + S - 1) / S + kTileNA - 1) / kTileNA * kTileNA;
  const int s0 = start + split * per;
  const int s1 = min(ctx, s0 + per);
  for (int i = tid; i < G * D; i += kThreadsNA)
    qs[i] = (float)q[(size_t)b * q_stride + (size_t)(hk * G + i / D) * D + i % D] * scale_log2;
  if (tid < G) {
    ms[tid] = -INFINITY;
    ls[tid] = 0.f;
  }
  constexpr int OUT = (G * D + kThreadsNA - 1) / kThreadsNA;
  float acc[OUT];
#pragma unroll
  for (int j = 0; j < OUT; ++j) acc[j] = 0.f;
  __syncthreads();
  const int32_t* row = bt + (size_t)b * bt_stride;
  for (int t0 = s0; t0 < s1; t0 += kTileNA) {
    {
      const int r = tid >> 1, sub = tid & 1, tok = t0 + r;
      __nv_bfloat16* kd = ks + r * RS;
      __nv_bfloat16* vd = vs + r * RS;
      if (tok < s1) {
        const size_t off = (((size_t)row[tok / page_size] * Hkv + hk) * page_size + tok % page_size) * D;
        for (int e = sub; e < D; e += 2) {
          if constexpr (sizeof(CacheT) == 1) {
            kd[e] = __float2bfloat16(snb::fp8e4m3_to_f(kc[off + e]));
            vd[e] = __float2bfloat16(snb::fp8e4m3_to_f(vc[off + e]));
          } else {
            kd[e] = kc[off + e];
            vd[e] = vc[off + e];
          }
        }
      } else {
        for (int e = sub; e < D; e += 2) {
          kd[e] = __float2bfloat16(0.f);
          vd[e] = __float2bfloat16(0.f);
        }
      }
    }
    __syncthreads();
    for (int p = tid; p < G * kTileNA; p += kThreadsNA) {
      const int g = p / kTileNA, t = p % kTileNA;
      float s = -INFINITY;
      if (t0 + t < s1) {
        s = 0.f;
        for (int e = 0; e < D; ++e) s += qs[g * D + e] * __bfloat162float(ks[t * RS + e]);
      }
      ps[p] = s;
    }
    __syncthreads();
    for (int g = warp; g < G; g += kThreadsNA / 32) {
      const float a0 = ps[g * kTileNA + lane], a1 = ps[g * kTileNA + lane + 32];
      const float mx = fmaxf(ms[g], snb::warp_max(fmaxf(a0, a1)));
      const float e0 = a0 == -INFINITY ? 0.f : exp2f(a0 - mx), e1 = a1 == -INFINITY ? 0.f : exp2f(a1 - mx);
      ps[g * kTileNA + lane] = e0;
      ps[g * kTileNA + lane + 32] = e1;
      const float sum = snb::warp_sum(e0 + e1);
      if (lane == 0) {
        const float a = ms[g] == -INFINITY ? 0.f : exp2f(ms[g] - mx);
        al[g] = a;
        ls[g] = ls[g] * a + sum;
        ms[g] = mx;
      }
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < OUT; ++j) {
      const int o = tid + j * kThreadsNA;
      if (o < G * D) {
        const int g = o / D, d = o % D;
        float a = acc[j] * al[g];
        for (int t = 0; t < kTileNA; ++t) a += ps[g * kTileNA + t] * __bfloat162float(vs[t * RS + d]);
        acc[j] = a;
      }
    }
    __syncthreads();
  }
  const int Hq = Hkv * G;
#pragma unroll
  for (int j = 0; j < OUT; ++j) {
    const int o = tid + j * kThreadsNA;
    if (o < G * D) {
      const int g = o / D, d = o % D;
      const size_t idx = ((size_t)b * Hq + hk * G + g) * S + split;
      o_part[idx * D + d] = ls[g] > 0.f ? acc[j] / ls[g] : 0.f;
    }
  }
  if (tid < G) {
    const size_t idx = ((size_t)b * Hq + hk * G + tid) * S + split;
    lse_part[idx] = ls[tid] > 0.f ? ms[tid] + log2f(ls[tid]) : -INFINITY;
  }
}

__global__ void noalloc_merge_kernel(const float* __restrict__ o_part, const float* __restrict__ lse_part,
                                     const float* __restrict__ sinks, __nv_bfloat16* __restrict__ out, int out_stride,
                                     int Hq, int D, int S, float v_scale) {
  const int bh = blockIdx.x, b = bh / Hq, h = bh % Hq;
  const float* lse = lse_part + (size_t)bh * S;
  float M = -INFINITY;
  for (int s = 0; s < S; ++s) M = fmaxf(M, lse[s]);
  const float sk = sinks != nullptr ? sinks[h] * kLog2eNA : -INFINITY;
  const float Mx = fmaxf(M, sk);
  float tot = sk == -INFINITY ? 0.f : exp2f(sk - Mx);
  for (int s = 0; s < S; ++s) tot += lse[s] == -INFINITY ? 0.f : exp2f(lse[s] - Mx);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float a = 0.f;
    for (int s = 0; s < S; ++s)
      if (lse[s] != -INFINITY) a += exp2f(lse[s] - Mx) * o_part[((size_t)bh * S + s) * D + d];
    out[(size_t)b * out_stride + (size_t)h * D + d] =
        __float2bfloat16((M == -INFINITY || tot <= 0.f) ? 0.f : a / tot * v_scale);
  }
}

std::mutex g_setup_mutex;
float* g_scratch_ptr[kMaxDevices] = {nullptr};
CUcontext g_scratch_ctx[kMaxDevices] = {nullptr};

// The calling thread's current context, through the runtime's driver entry point (no libcuda link needed).
CUcontext current_context() {
  using Fn = CUresult (*)(CUcontext*);
  static Fn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (Fn) nullptr;
    return reinterpret_cast<Fn>(p);
  }();
  CUcontext c = nullptr;
  if (fn == nullptr || fn(&c) != CUDA_SUCCESS) return nullptr;
  return c;
}

template <int D, typename CacheT>
int launch_na(int G, dim3 grid, cudaStream_t st, const __nv_bfloat16* q, int qs, const void* kc, const void* vc,
              const int32_t* bt, int bts, const int32_t* sl, int ps, int Hkv, int win, float scale, float* op,
              float* lp, int S) {
  const CacheT* k = static_cast<const CacheT*>(kc);
  const CacheT* v = static_cast<const CacheT*>(vc);
#define SNB_NA(GG) noalloc_split_kernel<D, GG, CacheT><<<grid, kThreadsNA, 0, st>>>(q, qs, k, v, bt, bts, sl, ps, Hkv, win, scale, op, lp, S)
  switch (G) {
    case 1: SNB_NA(1); break;
    case 2: SNB_NA(2); break;
    case 4: SNB_NA(4); break;
    case 8: SNB_NA(8); break;
    case 16: SNB_NA(16); break;
    default: return -1;
  }
#undef SNB_NA
  return 0;
}

}  // namespace

// Largest scratch request accepted, in fp32 values (batch * num_q_heads * num_splits * (head_dim + 1)).
extern "C" __attribute__((visibility("default"))) long long snb_decode_attention_noalloc_scratch_capacity(void) {
  return kNoAllocScratchFloats;
}

// Paged decode attention that allocates nothing. Same math as the `decode_attention` op: one new query per
// request over its paged context, GQA, optional sliding window and per-head sinks, bf16 or fp8-e4m3 KV with
// scales. Pointers are device pointers; `stream` may be 0. Returns 0 on success or a negative code:
// -1 bad arguments, -2 scratch request above the fixed capacity, -3 device address lookup failed, -4 a
// kernel launch failed.
extern "C" __attribute__((visibility("default"))) int snb_decode_attention_noalloc(
    void* out, int out_stride, const void* q, int q_stride, const void* k_cache, const void* v_cache, int kv_fp8,
    const int32_t* block_table, int block_table_stride, const int32_t* seq_lens, int batch, int num_q_heads,
    int num_kv_heads, int head_dim, int page_size, int window, float sm_scale, float k_scale, float v_scale,
    const float* sinks, int num_splits, cudaStream_t stream) {
  if (out == nullptr || q == nullptr || k_cache == nullptr || v_cache == nullptr || block_table == nullptr ||
      seq_lens == nullptr || batch < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || page_size <= 0 ||
      num_splits <= 0 || num_q_heads % num_kv_heads != 0 || (head_dim != 64 && head_dim != 128))
    return SNB_NOALLOC_ERR_ARGS;
  if (batch == 0) return SNB_NOALLOC_OK;
  const long long need = (long long)batch * num_q_heads * num_splits * (head_dim + 1);
  if (need > kNoAllocScratchFloats) return SNB_NOALLOC_ERR_TOO_LARGE;
  // an error left pending by earlier work belongs to its owner: report it and launch nothing, so the
  // launch checks below see only this call's launches
  if (cudaPeekAtLastError() != cudaSuccess) return SNB_NOALLOC_ERR_PRIOR;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return SNB_NOALLOC_ERR_SYMBOL;
  float* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    const CUcontext ctx = current_context();
    if (g_scratch_ptr[dev] == nullptr || ctx == nullptr || ctx != g_scratch_ctx[dev]) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return SNB_NOALLOC_ERR_SYMBOL;
      g_scratch_ptr[dev] = static_cast<float*>(p);
      g_scratch_ctx[dev] = ctx;
    }
    base = g_scratch_ptr[dev];
  }
  const int G = num_q_heads / num_kv_heads;
  float* o_part = base;
  float* lse_part = base + (size_t)batch * num_q_heads * num_splits * head_dim;
  const float scale = sm_scale * k_scale * kLog2eNA;
  dim3 grid(num_splits, num_kv_heads, batch);
  const __nv_bfloat16* qp = static_cast<const __nv_bfloat16*>(q);
  int rc;
  if (head_dim == 64) {
    rc = kv_fp8 ? launch_na<64, uint8_t>(G, grid, stream, qp, q_stride, k_cache, v_cache, block_table,
                                         block_table_stride, seq_lens, page_size, num_kv_heads, window, scale, o_part,
                                         lse_part, num_splits)
                : launch_na<64, __nv_bfloat16>(G, grid, stream, qp, q_stride, k_cache, v_cache, block_table,
                                               block_table_stride, seq_lens, page_size, num_kv_heads, window, scale,
                                               o_part, lse_part, num_splits);
  } else {
    rc = kv_fp8 ? launch_na<128, uint8_t>(G, grid, stream, qp, q_stride, k_cache, v_cache, block_table,
                                          block_table_stride, seq_lens, page_size, num_kv_heads, window, scale, o_part,
                                          lse_part, num_splits)
                : launch_na<128, __nv_bfloat16>(G, grid, stream, qp, q_stride, k_cache, v_cache, block_table,
                                                block_table_stride, seq_lens, page_size, num_kv_heads, window, scale,
                                                o_part, lse_part, num_splits);
  }
  if (rc != 0) return SNB_NOALLOC_ERR_ARGS;
  if (cudaGetLastError() != cudaSuccess) return SNB_NOALLOC_ERR_LAUNCH;
  noalloc_merge_kernel<<<batch * num_q_heads, 64, 0, stream>>>(o_part, lse_part, sinks,
                                                               static_cast<__nv_bfloat16*>(out), out_stride,
                                                               num_q_heads, head_dim, num_splits, v_scale);
  if (cudaGetLastError() != cudaSuccess) return SNB_NOALLOC_ERR_LAUNCH;
  return SNB_NOALLOC_OK;
}
