// Fused QK-RMSNorm (optional) + rotary embedding + paged K/V cache write.
//
// Parity: the reference's dense prefill op `qkv_paged` (sglang_neuron/ops/attention/qkv_paged.py:18-41)
// applies per-head RMSNorm to Q and K, RoPE, and writes K/V into the paged pool at `slot_mapping`.
// Here the QKV GEMM stays a separate launch (it is a plain GEMM) and everything after it is one
// memory-bound kernel: one warp per (token, head) row, the row staged in shared memory so any
// rotary pairing (NeoX halves, interleaved pairs, partial rotary) reads its partner directly.
//
// Paged cache layout: [num_pages, num_kv_heads, page_size, head_dim] (head-major within a page),
// bf16 or fp8-e4m3 (stored value = x / scale). A negative slot skips the write (padding rows).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "../common.cuh"

namespace {

constexpr int kWarps = 8;

template <typename T, typename CacheT>
__global__ void rope_kv_kernel(T* __restrict__ q, T* __restrict__ k, const T* __restrict__ v,
                               int stride_q, int stride_k, int stride_v, int Hq, int Hkv, int D,
                               int rot_dim, bool neox, const int64_t* __restrict__ positions,
                               const float* __restrict__ cos_sin, const T* __restrict__ q_norm_w,
                               const T* __restrict__ k_norm_w, float norm_eps,
                               CacheT* __restrict__ k_cache, CacheT* __restrict__ v_cache,
                               const int64_t* __restrict__ slots, int page_size, float inv_k_scale,
                               float inv_v_scale, int T_tokens, int64_t num_pages, int* status) {
  snb::pdl_wait();
  snb::pdl_trigger();
  __shared__ float rowbuf[kWarps][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kWarps + warp;
  const int heads_per_tok = Hq + 2 * Hkv;
  if (row >= T_tokens * heads_per_tok) return;
  const int t = row / heads_per_tok;
  const int h = row % heads_per_tok;
  const int per = D / 32;
  float vals[8];
  int64_t slot = slots != nullptr ? slots[t] : -1;
  if (slot >= 0 && slot / page_size >= num_pages) {
    // a slot past the pool: recorded (SNB_ERR_BOUNDS, the slot in status[1]) and not written
    if (status != nullptr && (threadIdx.x & 31) == 0 && atomicCAS(status, 0, SNB_ERR_BOUNDS) == 0)
      status[1] = (int)(slot & 0x7fffffff);
    slot = -1;
  }

  if (h >= Hq + Hkv) {  // V row: copy into the cache only
    if (slot < 0 || v_cache == nullptr) return;
    const int hv = h - Hq - Hkv;
    const T* src = v + (size_t)t * stride_v + (size_t)hv * D;
    const int64_t page = slot / page_size, off = slot % page_size;
    CacheT* dst = v_cache + (((size_t)page * Hkv + hv) * page_size + off) * D;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i < per) {
        float f = (float)src[lane + 32 * i];
        if constexpr (sizeof(CacheT) == 1) {
          dst[lane + 32 * i] = snb::f_to_fp8e4m3(f * inv_v_scale);
        } else {
          dst[lane + 32 * i] = (CacheT)f;
        }
      }
    }
    return;
  }

  const bool is_q = h < Hq;
  T* base = is_q ? q + (size_t)t * stride_q + (size_t)h * D
                 : k + (size_t)t * stride_k + (size_t)(h - Hq) * D;
  const T* nw = is_q ? q_norm_w : k_norm_w;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (i < per) {
      vals[i] = (float)base[lane + 32 * i];
      ss += vals[i] * vals[i];
    }
  }
  if (nw != nullptr) {
    ss = snb::warp_sum(ss);
    const float inv = rsqrtf(ss / (float)D + norm_eps);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < per) vals[i] = vals[i] * inv * (float)nw[lane + 32 * i];
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (i < per) rowbuf[warp][lane + 32 * i] = vals[i];
  __syncwarp();
  const int64_t pos = positions[t];
  const int half = rot_dim / 2;
  const float* cs = cos_sin + (size_t)pos * rot_dim;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (i < per) {
      const int e = lane + 32 * i;
      if (e < rot_dim) {
        int partner, f;
        bool first;
        if (neox) {
          first = e < half;
          partner = first ? e + half : e - half;
          f = first ? e : e - half;
        } else {
          first = (e & 1) == 0;
          partner = e ^ 1;
          f = e >> 1;
        }
        const float c = cs[f], s = cs[half + f];
        const float xp = rowbuf[warp][partner];
        vals[i] = first ? vals[i] * c - xp * s : vals[i] * c + xp * s;
      }
      base[e] = (T)vals[i];
    }
  }
  if (!is_q && slot >= 0 && k_cache != nullptr) {
    const int hk = h - Hq;
    const int64_t page = slot / page_size, off = slot % page_size;
    CacheT* dst = k_cache + (((size_t)page * Hkv + hk) * page_size + off) * D;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i < per) {
        if constexpr (sizeof(CacheT) == 1) {
          dst[lane + 32 * i] = snb::f_to_fp8e4m3(vals[i] * inv_k_scale);
        } else {
          dst[lane + 32 * i] = (CacheT)vals[i];
        }
      }
    }
  }
}

}  // namespace

// q: [T, Hq*D] view, k/v: [T, Hkv*D] views (row strides arbitrary, unit inner stride).
// k_cache/v_cache: [pages, Hkv, page_size, D] bf16 or float8_e4m3fn, or empty tensors to skip the write.
// A slot whose page is past the pool is not written; it is recorded in `status` (SNB_ERR_BOUNDS, slot in [1]).
void rope_qk_norm_kv_write(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor positions,
                           torch::Tensor cos_sin, int64_t num_q_heads, int64_t num_kv_heads,
                           int64_t head_dim, int64_t rot_dim, bool neox,
                           c10::optional<torch::Tensor> q_norm_w, c10::optional<torch::Tensor> k_norm_w,
                           double norm_eps, torch::Tensor k_cache, torch::Tensor v_cache,
                           torch::Tensor slots, int64_t page_size, double k_scale, double v_scale,
                           c10::optional<torch::Tensor> status) {
  const int T = q.size(0);
  if (T == 0) return;
  TORCH_CHECK(q.stride(-1) == 1 && k.stride(-1) == 1 && v.stride(-1) == 1, "rope_kv: inner stride");
  TORCH_CHECK(head_dim % 32 == 0 && head_dim <= 256, "rope_kv: head_dim ", head_dim);
  TORCH_CHECK(positions.scalar_type() == at::kLong && slots.scalar_type() == at::kLong, "rope_kv: int64 indices");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.size(1) == rot_dim, "rope_kv: cos_sin cache");
  const int rows = T * (num_q_heads + 2 * num_kv_heads);
  auto stream = at::cuda::getCurrentCUDAStream();
  const bool write = k_cache.numel() > 0;
  const float iks = (float)(1.0 / k_scale), ivs = (float)(1.0 / v_scale);
  const int blocks = (rows + kWarps - 1) / kWarps;
#define SNB_ROPE_LAUNCH(T_, C_)                                                                      \
  snb::launch_pdl(rope_kv_kernel<T_, C_>, blocks, kWarps * 32, 0, stream,                                         \
      (T_*)q.data_ptr(), (T_*)k.data_ptr(), (const T_*)v.data_ptr(), q.stride(0), k.stride(0),       \
      v.stride(0), num_q_heads, num_kv_heads, head_dim, rot_dim, neox, positions.data_ptr<int64_t>(), \
      cos_sin.data_ptr<float>(), q_norm_w ? (const T_*)q_norm_w->data_ptr() : nullptr,              \
      k_norm_w ? (const T_*)k_norm_w->data_ptr() : nullptr, (float)norm_eps,                        \
      write ? (C_*)k_cache.data_ptr() : nullptr, write ? (C_*)v_cache.data_ptr() : nullptr,         \
      slots.data_ptr<int64_t>(), page_size, iks, ivs, T, write ? (int64_t)k_cache.size(0) : (int64_t)0,  \
      status ? status->data_ptr<int>() : nullptr)
  if (q.scalar_type() == at::kBFloat16) {
    if (!write || k_cache.scalar_type() == at::kBFloat16) {
      SNB_ROPE_LAUNCH(__nv_bfloat16, __nv_bfloat16);
    } else {
      TORCH_CHECK(k_cache.scalar_type() == at::kFloat8_e4m3fn, "rope_kv: cache dtype");
      SNB_ROPE_LAUNCH(__nv_bfloat16, uint8_t);
    }
  } else {
    TORCH_CHECK(q.scalar_type() == at::kFloat, "rope_kv: q dtype");
    TORCH_CHECK(!write || k_cache.scalar_type() == at::kFloat, "rope_kv: fp32 q needs fp32 cache");
    SNB_ROPE_LAUNCH(float, float);
  }
#undef SNB_ROPE_LAUNCH
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
