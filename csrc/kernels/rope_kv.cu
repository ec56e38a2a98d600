// Fused QK-RMSNorm (optional) + rotary embedding + paged K/V cache write.
//
// Parity: the reference's dense prefill op `qkv_paged` (sglang_neuron/ops/attention/qkv_paged.py:18-41)
// applies per-head RMSNorm to Q and K, RoPE, and writes K/V into the paged pool at `slot_mapping`.
// Here the QKV GEMM stays a separate launch (it is a plain GEMM) and everything after it is one
// memory-bound kernel: one warp per (token, head) row, each lane moving a contiguous run of the row as one
// vector, the row staged in shared memory so any rotary pairing (NeoX halves, interleaved pairs, partial
// rotary) reads its partner directly.
//
// Paged cache layout: [num_pages, num_kv_heads, page_size, head_dim] (head-major within a page),
// bf16 or fp8-e4m3 (stored value = x / scale). A negative slot skips the write (padding rows).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "../common.cuh"

namespace {

constexpr int kWarps = 8;

// A lane's run of `per` consecutive elements (per = D / 32) as one vector access where the width allows.
template <typename T>
SNB_DEVICE void load_run(const T* p, int per, float (&f)[8]) {
  if constexpr (sizeof(T) == 2) {
    if (per == 2) {
      const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(p);
      f[0] = __bfloat162float(v.x), f[1] = __bfloat162float(v.y);
      return;
    }
    if (per == 4 || per == 8) {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        if (c * 4 < per) {
          const uint2 u = reinterpret_cast<const uint2*>(p)[c];
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
          f[c * 4 + 0] = __bfloat162float(h[0].x), f[c * 4 + 1] = __bfloat162float(h[0].y);
          f[c * 4 + 2] = __bfloat162float(h[1].x), f[c * 4 + 3] = __bfloat162float(h[1].y);
        }
      }
      return;
    }
  } else {
    if (per == 2 || per == 4 || per == 8) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (c * 2 < per) {
          const float2 u = reinterpret_cast<const float2*>(p)[c];
          f[c * 2] = u.x, f[c * 2 + 1] = u.y;
        }
      }
      return;
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (i < per) f[i] = (float)p[i];
}

template <typename T>
SNB_DEVICE void store_run(T* p, int per, const float (&f)[8]) {
  if constexpr (sizeof(T) == 2) {
    if (per == 2) {
      *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(f[0], f[1]);
      return;
    }
    if (per == 4 || per == 8) {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        if (c * 4 < per) {
          uint2 u;
          __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
          h[0] = __floats2bfloat162_rn(f[c * 4], f[c * 4 + 1]);
          h[1] = __floats2bfloat162_rn(f[c * 4 + 2], f[c * 4 + 3]);
          reinterpret_cast<uint2*>(p)[c] = u;
        }
      }
      return;
    }
  } else if constexpr (sizeof(T) == 4) {
    if (per == 2 || per == 4 || per == 8) {
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (c * 2 < per) reinterpret_cast<float2*>(p)[c] = make_float2(f[c * 2], f[c * 2 + 1]);
      return;
    }
  } else {  // fp8 e4m3 bytes
    if (per == 2 || per == 4 || per == 8) {
      uint8_t b[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (i < per) b[i] = snb::f_to_fp8e4m3(f[i]);
      if (per == 2) {
        *reinterpret_cast<uint16_t*>(p) = (uint16_t)(b[0] | (b[1] << 8));
      } else {
#pragma unroll
        for (int c = 0; c < 2; ++c)
          if (c * 4 < per)
            reinterpret_cast<uint32_t*>(p)[c] = (uint32_t)b[c * 4] | ((uint32_t)b[c * 4 + 1] << 8) |
                                                ((uint32_t)b[c * 4 + 2] << 16) | ((uint32_t)b[c * 4 + 3] << 24);
      }
      return;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < per) reinterpret_cast<uint8_t*>(p)[i] = snb::f_to_fp8e4m3(f[i]);
    return;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (i < per) p[i] = (T)f[i];
}

// One warp per (token, head) row; lane l owns elements [l * per, (l + 1) * per), read and written as one vector
// each, so a warp moves a whole row per access.
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
  const int e0 = lane * per;
  float vals[8];
  int64_t slot = slots != nullptr ? slots[t] : -1;
  if (slot >= 0 && slot / page_size >= num_pages) {
    // a slot past the pool: recorded (SNB_ERR_BOUNDS, the slot in status[1]) and not written
    if (status != nullptr && lane == 0 && atomicCAS(status, 0, SNB_ERR_BOUNDS) == 0)
      status[1] = (int)(slot & 0x7fffffff);
    slot = -1;
  }

  if (h >= Hq + Hkv) {  // V row: copy into the cache only
    if (slot < 0 || v_cache == nullptr) return;
    const int hv = h - Hq - Hkv;
    load_run(v + (size_t)t * stride_v + (size_t)hv * D + e0, per, vals);
#pragma unroll
    for (int i = 0; i < 8; ++i) vals[i] *= (sizeof(CacheT) == 1 ? inv_v_scale : 1.f);
    const int64_t page = slot / page_size, off = slot % page_size;
    store_run(v_cache + (((size_t)page * Hkv + hv) * page_size + off) * D + e0, per, vals);
    return;
  }

  const bool is_q = h < Hq;
  T* base = is_q ? q + (size_t)t * stride_q + (size_t)h * D
                 : k + (size_t)t * stride_k + (size_t)(h - Hq) * D;
  const T* nw = is_q ? q_norm_w : k_norm_w;
  load_run(base + e0, per, vals);
  if (nw != nullptr) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < per) ss += vals[i] * vals[i];
    ss = snb::warp_sum(ss);
    const float inv = rsqrtf(ss / (float)D + norm_eps);
    float w[8];
    load_run(nw + e0, per, w);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < per) vals[i] = vals[i] * inv * w[i];
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (i < per) rowbuf[warp][e0 + i] = vals[i];
  __syncwarp();
  const int64_t pos = positions[t];
  const int half = rot_dim / 2;
  const float* cs = cos_sin + (size_t)pos * rot_dim;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int e = e0 + i;
    if (i < per && e < rot_dim) {
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
  }
  store_run(base + e0, per, vals);
  if (!is_q && slot >= 0 && k_cache != nullptr) {
    const int hk = h - Hq;
    const int64_t page = slot / page_size, off = slot % page_size;
    if constexpr (sizeof(CacheT) == 1) {
#pragma unroll
      for (int i = 0; i < 8; ++i) vals[i] *= inv_k_scale;
    }
    store_run(k_cache + (((size_t)page * Hkv + hk) * page_size + off) * D + e0, per, vals);
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
