// Paged GQA attention over the KV pool: decode (split-K + LSE merge) and extend/prefill.
//
// Parity:
//  * decode: the reference's `attention_decode` / `attention_decode_paged` ops
//    (sglang_neuron/ops/attention/attention_decode.py:28-205, attention_decode_paged.py:64-127) attend one
//    new token per request over the paged prior, with learned per-head sinks, a sliding window and FP8 K/V
//    whose scales fold into the softmax scale (K) and the output (V).
//  * extend: `segmented_attention` (sglang_neuron/ops/attention/attention_segmented_cte.py:21) attends a
//    chunk of new tokens over the paged prior plus the causal chunk itself.
//
// B200 design: both kernels read K/V straight from the paged pool ([pages, kv_heads, page, D],
// bf16 or fp8-e4m3), convert to bf16 in shared memory, and keep softmax state in fp32 with exp2.
// Decode splits the context over CTAs (flash-decoding) so small batches still fill 148 SMs; a merge
// kernel folds the partial (o, lse) pairs and the sink term. GQA heads of one KV head share each
// K/V tile load.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "../common.cuh"

namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kTile = 64;      // tokens per K/V smem tile
constexpr int kThreads = 128;

template <typename CacheT>
SNB_DEVICE void load_row_to_bf16(__nv_bfloat16* dst, const CacheT* src, int D, int lane_in_row,
                                 int threads_per_row) {
  // Copies one D-element K or V row into bf16 shared memory using 16-byte global loads.
  if constexpr (sizeof(CacheT) == 2) {
    for (int c = lane_in_row; c < D / 8; c += threads_per_row)
      reinterpret_cast<uint4*>(dst)[c] = reinterpret_cast<const uint4*>(src)[c];
  } else {
    for (int c = lane_in_row; c < D / 16; c += threads_per_row) {
      uint4 raw = reinterpret_cast<const uint4*>(src)[c];
      const uint8_t* b = reinterpret_cast<const uint8_t*>(&raw);
      float f[8];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] = snb::fp8e4m3_to_f(b[h * 8 + i]);
        reinterpret_cast<uint4*>(dst)[2 * c + h] = snb::pack_bf16x8(f);
      }
    }
  }
}

template <typename CacheT>
SNB_DEVICE void zero_row(__nv_bfloat16* dst, int D, int lane_in_row, int threads_per_row) {
  for (int c = lane_in_row; c < D / 8; c += threads_per_row)
    reinterpret_cast<uint4*>(dst)[c] = make_uint4(0, 0, 0, 0);
}

// ---------------------------------------------------------------------------------------------
// Decode: grid (splits, Hkv, B), 128 threads. Each CTA: one request, one KV head, G query heads,
// a contiguous page range of the (windowed) context.
// ---------------------------------------------------------------------------------------------
template <int D, int G, typename CacheT>
__global__ void __launch_bounds__(kThreads) decode_attn_kernel(
    const __nv_bfloat16* __restrict__ q, int q_stride_tok, const CacheT* __restrict__ k_cache,
    const CacheT* __restrict__ v_cache, const int32_t* __restrict__ block_table, int bt_stride,
    const int32_t* __restrict__ seq_lens, int page_size, int Hkv, int window, float qk_scale_log2,
    float v_scale, const float* __restrict__ sinks, __nv_bfloat16* __restrict__ out, int out_stride_tok,
    float* __restrict__ o_part, float* __restrict__ lse_part, int num_splits) {
  snb::pdl_wait();
  snb::pdl_trigger();
  constexpr int RS = D + 8;  // padded smem row (bf16 elements) -> conflict-free 16B row reads
  __shared__ __align__(16) __nv_bfloat16 k_s[kTile * RS];
  __shared__ __align__(16) __nv_bfloat16 v_s[kTile * RS];
  __shared__ float q_s[G * D];
  __shared__ float p_s[G * kTile];
  __shared__ float m_s[G], l_s[G], alpha_s[G];

  const int split = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ctx = seq_lens[b];
  const int start = (window > 0 && ctx > window) ? ctx - window : 0;
  const int span = ctx - start;
  const int per_split = (span + num_splits - 1) / num_splits;
  // Round the split length up to whole tiles so splits align with tiles.
  const int per_split_t = ((per_split + kTile - 1) / kTile) * kTile;
  const int s_begin = start + split * per_split_t;
  const int s_end = min(ctx, s_begin + per_split_t);

  for (int i = tid; i < G * D; i += kThreads) {
    const int g = i / D, d = i % D;
    q_s[i] = (float)q[(size_t)b * q_stride_tok + (size_t)(hk * G + g) * D + d] * qk_scale_log2;
  }
  if (tid < G) {
    m_s[tid] = -INFINITY;
    l_s[tid] = 0.f;
  }
  constexpr int OUT_PER = (G * D + kThreads - 1) / kThreads;
  float acc[OUT_PER];
#pragma unroll
  for (int j = 0; j < OUT_PER; ++j) acc[j] = 0.f;
  __syncthreads();

  const int32_t* bt = block_table + (size_t)b * bt_stride;
  for (int t0 = s_begin; t0 < s_end; t0 += kTile) {
    // Load the K/V tile: 2 threads per token row.
    {
      const int row = tid >> 1, sub = tid & 1;
      const int tok = t0 + row;
      if (tok < s_end) {
        const int page = bt[tok / page_size];
        const size_t off = (((size_t)page * Hkv + hk) * page_size + (tok % page_size)) * D;
        load_row_to_bf16<CacheT>(k_s + row * RS, k_cache + off, D, sub, 2);
        load_row_to_bf16<CacheT>(v_s + row * RS, v_cache + off, D, sub, 2);
      } else {
        zero_row<CacheT>(k_s + row * RS, D, sub, 2);
        zero_row<CacheT>(v_s + row * RS, D, sub, 2);
      }
    }
    __syncthreads();
    // Scores for all (g, token) pairs of the tile.
    for (int p = tid; p < G * kTile; p += kThreads) {
      const int g = p / kTile, t = p % kTile;
      float s = -INFINITY;
      if (t0 + t < s_end) {
        s = 0.f;
        const __nv_bfloat16* kr = k_s + t * RS;
        const float* qr = q_s + g * D;
#pragma unroll
        for (int c = 0; c < D / 8; ++c) {
          float kf[8];
          snb::unpack_bf16x8(reinterpret_cast<const uint4*>(kr)[c], kf);
#pragma unroll
          for (int i = 0; i < 8; ++i) s += qr[c * 8 + i] * kf[i];
        }
      }
      p_s[p] = s;
    }
    __syncthreads();
    // Online softmax bookkeeping: one warp per head.
    for (int g = warp; g < G; g += kThreads / 32) {
      const float s0 = p_s[g * kTile + lane], s1 = p_s[g * kTile + lane + 32];
      const float tmax = snb::warp_max(fmaxf(s0, s1));
      const float m_old = m_s[g];
      const float m_new = fmaxf(m_old, tmax);
      const float e0 = (s0 == -INFINITY) ? 0.f : exp2f(s0 - m_new);
      const float e1 = (s1 == -INFINITY) ? 0.f : exp2f(s1 - m_new);
      p_s[g * kTile + lane] = e0;
      p_s[g * kTile + lane + 32] = e1;
      const float sum = snb::warp_sum(e0 + e1);
      if (lane == 0) {
        const float a = (m_old == -INFINITY) ? 0.f : exp2f(m_old - m_new);
        alpha_s[g] = a;
        l_s[g] = l_s[g] * a + sum;
        m_s[g] = m_new;
      }
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < OUT_PER; ++j) {
      const int o = tid + j * kThreads;
      if (o < G * D) {
        const int g = o / D, d = o % D;
        float a = acc[j] * alpha_s[g];
        const float* pr = p_s + g * kTile;
#pragma unroll 8
        for (int t = 0; t < kTile; ++t) a += pr[t] * __bfloat162float(v_s[t * RS + d]);
        acc[j] = a;
      }
    }
    __syncthreads();
  }

  if (num_splits == 1) {
#pragma unroll
    for (int j = 0; j < OUT_PER; ++j) {
      const int o = tid + j * kThreads;
      if (o < G * D) {
        const int g = o / D, d = o % D;
        float denom = l_s[g];
        if (sinks != nullptr) {
          const float sk = sinks[hk * G + g] * kLog2e;
          const float m = m_s[g];
          denom = (m == -INFINITY) ? 1.f : denom + exp2f(sk - m);
        }
        const float r = denom > 0.f ? acc[j] / denom * v_scale : 0.f;
        out[(size_t)b * out_stride_tok + (size_t)(hk * G + g) * D + d] = __float2bfloat16(r);
      }
    }
  } else {
    const int Hq = Hkv * G;
#pragma unroll
    for (int j = 0; j < OUT_PER; ++j) {
      const int o = tid + j * kThreads;
      if (o < G * D) {
        const int g = o / D, d = o % D;
        const float l = l_s[g];
        const size_t idx = (((size_t)b * Hq + hk * G + g) * num_splits + split);
        o_part[idx * D + d] = l > 0.f ? acc[j] / l : 0.f;
      }
    }
    if (tid < G) {
      const float l = l_s[tid];
      const size_t idx = (((size_t)b * Hq + hk * G + tid) * num_splits + split);
      lse_part[idx] = l > 0.f ? m_s[tid] + log2f(l) : -INFINITY;
    }
  }
}

// Merge split partials: out = sum_s w_s o_s / (sum_s w_s + sink), w_s = 2^(lse_s - M).
__global__ void decode_merge_kernel(const float* __restrict__ o_part, const float* __restrict__ lse_part,
                                    const float* __restrict__ sinks, __nv_bfloat16* __restrict__ out,
                                    int out_stride_tok, int Hq, int D, int S, float v_scale) {
  snb::pdl_wait();
  snb::pdl_trigger();
  const int bh = blockIdx.x;  // b * Hq + h
  const int b = bh / Hq, h = bh % Hq;
  const float* lse = lse_part + (size_t)bh * S;
  float M = -INFINITY;
  for (int s = 0; s < S; ++s) M = fmaxf(M, lse[s]);
  const float sk = sinks != nullptr ? sinks[h] * kLog2e : -INFINITY;
  const float Mx = fmaxf(M, sk);
  float total = (sk == -INFINITY) ? 0.f : exp2f(sk - Mx);
  for (int s = 0; s < S; ++s) total += (lse[s] == -INFINITY) ? 0.f : exp2f(lse[s] - Mx);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float a = 0.f;
    for (int s = 0; s < S; ++s) {
      if (lse[s] != -INFINITY) a += exp2f(lse[s] - Mx) * o_part[((size_t)bh * S + s) * D + d];
    }
    const float r = (M == -INFINITY || total <= 0.f) ? 0.f : a / total * v_scale;
    out[(size_t)b * out_stride_tok + (size_t)h * D + d] = __float2bfloat16(r);
  }
}

// ---------------------------------------------------------------------------------------------
// Extend (prefill with paged prior): grid (q_tiles, B, Hkv), 128 threads, one (query, head) row
// per thread (D == 64) or per thread pair (D == 128, each thread holding half the row).
// Queries of request b are q[qo_indptr[b] .. qo_indptr[b+1]); their positions are
// kv_len[b] - extend_len + i, and K/V for every position already sits in the paged pool.
// ---------------------------------------------------------------------------------------------
template <int D, int G, int TPR, typename CacheT>
__global__ void __launch_bounds__(kThreads) extend_attn_kernel(
    const __nv_bfloat16* __restrict__ q, int q_stride_tok, const CacheT* __restrict__ k_cache,
    const CacheT* __restrict__ v_cache, const int32_t* __restrict__ block_table, int bt_stride,
    const int32_t* __restrict__ qo_indptr, const int32_t* __restrict__ kv_lens, int page_size, int Hkv,
    int window, float qk_scale_log2, float v_scale, const float* __restrict__ sinks,
    __nv_bfloat16* __restrict__ out, int out_stride_tok) {
  snb::pdl_wait();
  snb::pdl_trigger();
  constexpr int RS = D + 8;
  constexpr int DH = D / TPR;                   // row elements held by one thread
  constexpr int ROWS = kThreads / TPR;          // (query, head) rows per CTA
  constexpr int QT = ROWS / G;                  // queries per CTA
  __shared__ __align__(16) __nv_bfloat16 k_s[kTile * RS];
  __shared__ __align__(16) __nv_bfloat16 v_s[kTile * RS];

  const int b = blockIdx.y, hk = blockIdx.z;
  const int q_begin = qo_indptr[b], q_end = qo_indptr[b + 1];
  const int ext = q_end - q_begin;
  const int qi0 = blockIdx.x * QT;
  if (qi0 >= ext) return;
  const int kv_len = kv_lens[b];
  const int prefix = kv_len - ext;

  const int tid = threadIdx.x;
  const int row = tid / TPR, part = tid % TPR;
  const int qi = qi0 + row / G;       // query index within the request
  const int g = row % G;
  const int h = hk * G + g;
  const bool valid = qi < ext;
  const int pos = prefix + (valid ? qi : 0);

  float qr[DH], acc[DH];
#pragma unroll
  for (int i = 0; i < DH; ++i) {
    qr[i] = valid ? (float)q[(size_t)(q_begin + qi) * q_stride_tok + (size_t)h * D + part * DH + i] *
                        qk_scale_log2
                  : 0.f;
    acc[i] = 0.f;
  }
  float m = -INFINITY, l = 0.f;

  // Token range this CTA needs: union over its queries.
  const int last_q = min(ext, qi0 + QT) - 1;
  const int hi = prefix + last_q + 1;  // exclusive
  int lo = 0;
  if (window > 0) lo = max(0, prefix + qi0 - window + 1);
  lo = (lo / kTile) * kTile;
  const int32_t* bt = block_table + (size_t)b * bt_stride;

  for (int t0 = lo; t0 < hi; t0 += kTile) {
    {
      const int r = tid >> 1, sub = tid & 1;
      const int tok = t0 + r;
      if (tok < hi) {
        const int page = bt[tok / page_size];
        const size_t off = (((size_t)page * Hkv + hk) * page_size + (tok % page_size)) * D;
        load_row_to_bf16<CacheT>(k_s + r * RS, k_cache + off, D, sub, 2);
        load_row_to_bf16<CacheT>(v_s + r * RS, v_cache + off, D, sub, 2);
      } else {
        zero_row<CacheT>(k_s + r * RS, D, sub, 2);
        zero_row<CacheT>(v_s + r * RS, D, sub, 2);
      }
    }
    __syncthreads();
    const int t_lim = min(kTile, hi - t0);
    for (int t = 0; t < t_lim; ++t) {
      const int kp = t0 + t;
      const bool allowed = valid && kp <= pos && (window <= 0 || pos - kp < window);
      const __nv_bfloat16* kr = k_s + t * RS + part * DH;
      float s = 0.f;
#pragma unroll
      for (int c = 0; c < DH / 8; ++c) {
        float kf[8];
        snb::unpack_bf16x8(reinterpret_cast<const uint4*>(kr)[c], kf);
#pragma unroll
        for (int i = 0; i < 8; ++i) s += qr[c * 8 + i] * kf[i];
      }
      if (TPR == 2) s += __shfl_xor_sync(0xffffffffu, s, 1);
      if (!allowed) continue;  // uniform within a thread pair
      const float m_new = fmaxf(m, s);
      const float a = (m == -INFINITY) ? 0.f : exp2f(m - m_new);
      const float p = exp2f(s - m_new);
      l = l * a + p;
      m = m_new;
      const __nv_bfloat16* vr = v_s + t * RS + part * DH;
#pragma unroll
      for (int c = 0; c < DH / 8; ++c) {
        float vf[8];
        snb::unpack_bf16x8(reinterpret_cast<const uint4*>(vr)[c], vf);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[c * 8 + i] = acc[c * 8 + i] * a + p * vf[i];
      }
    }
    __syncthreads();
  }
  if (!valid) return;
  float denom = l;
  if (sinks != nullptr) {
    const float sk = sinks[h] * kLog2e;
    denom = (m == -INFINITY) ? 1.f : denom + exp2f(sk - m);
  }
  const float inv = denom > 0.f ? v_scale / denom : 0.f;
  __nv_bfloat16* o = out + (size_t)(q_begin + qi) * out_stride_tok + (size_t)h * D + part * DH;
#pragma unroll
  for (int c = 0; c < DH / 8; ++c) {
    float f[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = acc[c * 8 + i] * inv;
    reinterpret_cast<uint4*>(o)[c] = snb::pack_bf16x8(f);
  }
}

template <int D, typename CacheT>
void launch_decode_g(int G, dim3 grid, cudaStream_t st, const __nv_bfloat16* q, int qs, const CacheT* kc,
                     const CacheT* vc, const int32_t* bt, int bts, const int32_t* sl, int ps, int Hkv, int win,
                     float scale, float vs, const float* sinks, __nv_bfloat16* out, int os, float* op,
                     float* lp, int S) {
#define SNB_DEC(GG)                                                                                   \
  snb::launch_pdl(decode_attn_kernel<D, GG, CacheT>, grid, kThreads, 0, st, q, qs, kc, vc, bt, bts, sl, ps, Hkv, win, \
                                                                scale, vs, sinks, out, os, op, lp, S)
  switch (G) {
    case 1: SNB_DEC(1); break;
    case 2: SNB_DEC(2); break;
    case 4: SNB_DEC(4); break;
    case 8: SNB_DEC(8); break;
    case 16: SNB_DEC(16); break;
    default: TORCH_CHECK(false, "decode_attention: unsupported GQA group ", G);
  }
#undef SNB_DEC
}

template <int D, int TPR, typename CacheT>
void launch_extend_g(int G, int max_ext, int B, int Hkv, cudaStream_t st, const __nv_bfloat16* q, int qs,
                     const CacheT* kc, const CacheT* vc, const int32_t* bt, int bts, const int32_t* qo,
                     const int32_t* kvl, int ps, int win, float scale, float vs, const float* sinks,
                     __nv_bfloat16* out, int os) {
#define SNB_EXT(GG)                                                                                 \
  {                                                                                                 \
    constexpr int QT = (kThreads / TPR) / GG;                                                       \
    dim3 grid((max_ext + QT - 1) / QT, B, Hkv);                                                     \
    snb::launch_pdl(extend_attn_kernel<D, GG, TPR, CacheT>, grid, kThreads, 0, st, q, qs, kc, vc, bt, bts, qo, kvl, \
                                                                       ps, Hkv, win, scale, vs, sinks, \
                                                                       out, os);                   \
  }
  switch (G) {
    case 1: SNB_EXT(1); break;
    case 2: SNB_EXT(2); break;
    case 4: SNB_EXT(4); break;
    case 8: SNB_EXT(8); break;
    case 16: SNB_EXT(16); break;
    default: TORCH_CHECK(false, "extend_attention: unsupported GQA group ", G);
  }
#undef SNB_EXT
}

}  // namespace

bool decode_attention_mma(torch::Tensor out, torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                          torch::Tensor block_table, torch::Tensor seq_lens, int64_t num_q_heads, int64_t num_kv_heads,
                          int64_t head_dim, int64_t page_size, int64_t window, float scale_log2, float v_scale_final,
                          const float* sinks, int64_t num_splits, float* o_part, float* lse_part);

bool decode_attention_pipelined(torch::Tensor out, torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                                torch::Tensor block_table, torch::Tensor seq_lens, int64_t num_q_heads,
                                int64_t num_kv_heads, int64_t head_dim, int64_t page_size, int64_t window,
                                float scale_log2, float v_scale_final, const float* sinks, int64_t num_splits,
                                float* o_part, float* lse_part, int* status, int* merge_cnt, float v_scale_out);

bool extend_attention_mma(torch::Tensor out, torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                          torch::Tensor block_table, torch::Tensor qo_indptr, torch::Tensor kv_lens, int64_t max_extend,
                          int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim, int64_t page_size, int64_t window,
                          float scale_log2, float v_scale, const float* sinks);

// q: [B, Hq*D] bf16 (row stride arbitrary). Caches: [pages, Hkv, page_size, D].
// block_table: [B, max_pages] int32; seq_lens: [B] int32 (tokens including the new one).
// o_part/lse_part: fp32 scratch of at least B*Hq*num_splits*D and B*Hq*num_splits elements.
void decode_attention(torch::Tensor out, torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                      torch::Tensor block_table, torch::Tensor seq_lens, int64_t num_q_heads,
                      int64_t num_kv_heads, int64_t head_dim, int64_t page_size, int64_t window,
                      double sm_scale, double k_scale, double v_scale, c10::optional<torch::Tensor> sinks,
                      int64_t num_splits, torch::Tensor o_part, torch::Tensor lse_part,
                      c10::optional<torch::Tensor> status, c10::optional<torch::Tensor> merge_counters) {
  const int B = q.size(0);
  if (B == 0) return;
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16, "decode_attention: bf16 q/out");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt, "decode_attention: int32 tables");
  TORCH_CHECK(num_q_heads % num_kv_heads == 0, "decode_attention: heads");
  const int G = num_q_heads / num_kv_heads;
  const int S = (int)num_splits;
  TORCH_CHECK(S >= 1, "decode_attention: splits");
  if (S > 1) {
    TORCH_CHECK(o_part.numel() >= (int64_t)B * num_q_heads * S * head_dim && lse_part.numel() >= (int64_t)B * num_q_heads * S,
                "decode_attention: scratch too small");
  }
  const float scale = (float)(sm_scale * k_scale) * kLog2e;
  const float* sk = sinks ? sinks->data_ptr<float>() : nullptr;
  if (sinks) TORCH_CHECK(sinks->scalar_type() == at::kFloat, "decode_attention: fp32 sinks");
  auto st = at::cuda::getCurrentCUDAStream();
  dim3 grid(S, num_kv_heads, B);
  float* op = S > 1 ? o_part.data_ptr<float>() : nullptr;
  float* lp = S > 1 ? lse_part.data_ptr<float>() : nullptr;
  const float vs = S > 1 ? 1.f : (float)v_scale;
  auto qp = (const __nv_bfloat16*)q.data_ptr();
  auto outp = (__nv_bfloat16*)out.data_ptr();
  const bool fp8 = k_cache.scalar_type() == at::kFloat8_e4m3fn;
  TORCH_CHECK(fp8 || k_cache.scalar_type() == at::kBFloat16, "decode_attention: cache dtype");
  // the bulk-async pipelined tensor-core kernels (token-major for e4m3 and bf16 caches, head-major for e4m3),
  // else the register-prefetch tensor-core kernel for every GQA group up to 16 heads; the CUDA-core kernel
  // below covers the rest
  int* stp = status ? status->data_ptr<int>() : nullptr;
  int* mcnt = nullptr;
  if (merge_counters && S > 1) {
    TORCH_CHECK(merge_counters->scalar_type() == at::kInt && merge_counters->numel() >= (int64_t)B * num_kv_heads,
                "decode_attention: merge counters");
    mcnt = merge_counters->data_ptr<int>();
  }
  const bool fp8_done = stp != nullptr && decode_attention_pipelined(out, q, k_cache, v_cache, block_table, seq_lens,
                                                                     num_q_heads, num_kv_heads, head_dim, page_size,
                                                                     window, scale, vs, sk, S, op, lp, stp, mcnt,
                                                                     (float)v_scale);
  const bool merged = fp8_done && mcnt != nullptr;
  const bool mma_done = fp8_done ||
      decode_attention_mma(out, q, k_cache, v_cache, block_table, seq_lens, num_q_heads, num_kv_heads, head_dim,
                           page_size, window, scale, vs, sk, S, op, lp);
  if (!mma_done) {
#define SNB_DEC_D(DD)                                                                                      \
  if (fp8)                                                                                                 \
    launch_decode_g<DD, uint8_t>(G, grid, st, qp, q.stride(0), (const uint8_t*)k_cache.data_ptr(),         \
                                 (const uint8_t*)v_cache.data_ptr(), block_table.data_ptr<int32_t>(),      \
                                 block_table.stride(0), seq_lens.data_ptr<int32_t>(), page_size,           \
                                 num_kv_heads, window, scale, vs, sk, outp, out.stride(0), op, lp, S);     \
  else                                                                                                     \
    launch_decode_g<DD, __nv_bfloat16>(G, grid, st, qp, q.stride(0), (const __nv_bfloat16*)k_cache.data_ptr(), \
                                       (const __nv_bfloat16*)v_cache.data_ptr(), block_table.data_ptr<int32_t>(), \
                                       block_table.stride(0), seq_lens.data_ptr<int32_t>(), page_size,     \
                                       num_kv_heads, window, scale, vs, sk, outp, out.stride(0), op, lp, S);
  if (head_dim == 64) {
    SNB_DEC_D(64)
  } else if (head_dim == 128) {
    SNB_DEC_D(128)
  } else {
    TORCH_CHECK(false, "decode_attention: head_dim ", head_dim);
  }
#undef SNB_DEC_D
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  if (S > 1 && !merged) {
    snb::launch_pdl(decode_merge_kernel, B * num_q_heads, 64, 0, st, op, lp, sk, outp, out.stride(0), num_q_heads, head_dim, S,
                                                        (float)v_scale);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

// q: [Tq, Hq*D] bf16 packed by request (qo_indptr [B+1] int32); kv_lens [B] int32 = prefix + extend.
void extend_attention(torch::Tensor out, torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                      torch::Tensor block_table, torch::Tensor qo_indptr, torch::Tensor kv_lens,
                      int64_t max_extend, int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
                      int64_t page_size, int64_t window, double sm_scale, double k_scale, double v_scale,
                      c10::optional<torch::Tensor> sinks) {
  const int B = kv_lens.size(0);
  if (B == 0 || max_extend == 0) return;
  TORCH_CHECK(q.scalar_type() == at::kBFloat16, "extend_attention: bf16 q");
  const int G = num_q_heads / num_kv_heads;
  const float scale = (float)(sm_scale * k_scale) * kLog2e;
  const float* sk = sinks ? sinks->data_ptr<float>() : nullptr;
  auto st = at::cuda::getCurrentCUDAStream();
  auto qp = (const __nv_bfloat16*)q.data_ptr();
  auto outp = (__nv_bfloat16*)out.data_ptr();
  const bool fp8 = k_cache.scalar_type() == at::kFloat8_e4m3fn;
  if (extend_attention_mma(out, q, k_cache, v_cache, block_table, qo_indptr, kv_lens, max_extend, num_q_heads,
                           num_kv_heads, head_dim, page_size, window, scale, (float)v_scale, sk))
    return;
#define SNB_EXT_D(DD, TPR)                                                                                 \
  if (fp8)                                                                                                 \
    launch_extend_g<DD, TPR, uint8_t>(G, max_extend, B, num_kv_heads, st, qp, q.stride(0),                 \
                                      (const uint8_t*)k_cache.data_ptr(), (const uint8_t*)v_cache.data_ptr(), \
                                      block_table.data_ptr<int32_t>(), block_table.stride(0),              \
                                      qo_indptr.data_ptr<int32_t>(), kv_lens.data_ptr<int32_t>(), page_size, \
                                      window, scale, (float)v_scale, sk, outp, out.stride(0));            \
  else                                                                                                     \
    launch_extend_g<DD, TPR, __nv_bfloat16>(G, max_extend, B, num_kv_heads, st, qp, q.stride(0),           \
                                            (const __nv_bfloat16*)k_cache.data_ptr(),                      \
                                            (const __nv_bfloat16*)v_cache.data_ptr(),                      \
                                            block_table.data_ptr<int32_t>(), block_table.stride(0),        \
                                            qo_indptr.data_ptr<int32_t>(), kv_lens.data_ptr<int32_t>(),    \
                                            page_size, window, scale, (float)v_scale, sk, outp, out.stride(0));
  if (head_dim == 64) {
    SNB_EXT_D(64, 1)
  } else if (head_dim == 128) {
    SNB_EXT_D(128, 2)
  } else {
    TORCH_CHECK(false, "extend_attention: head_dim ", head_dim);
  }
#undef SNB_EXT_D
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
