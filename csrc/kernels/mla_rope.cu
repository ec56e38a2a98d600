// DeepSeek-V2 latent-row construction in one kernel: the kv_a projection's compressed part is RMS-normalised
// (kv_a_layernorm), its rotary part rotated, and the latent row [norm(c) || rope(k_pe)] written into the
// paged latent pool at the token's slot; the query's rotary part rope(q_pe) of every head lands in the
// attention query rows [T, H, r + rope] next to the absorbed q_nope . W_UK block (written by the grouped
// GEMM). One CTA per token.
//
// Parity: the reference's latent projection and rope before absorbed MLA (sglang_neuron/models/deepseek_v2/
// model.py:101 `_project`).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "../common.cuh"

namespace {

constexpr int kThreadsMR = 256;

SNB_DEVICE float rot(const float* x, int e, int half, bool neox, const float* cs) {
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
  return first ? x[e] * c - x[partner] * s : x[e] * c + x[partner] * s;
}

__global__ void __launch_bounds__(kThreadsMR) mla_rope_latent_kernel(
    const __nv_bfloat16* __restrict__ kv_a, int kv_stride, const __nv_bfloat16* __restrict__ q, int q_stride,
    int H, int nope, int r, int rope, const __nv_bfloat16* __restrict__ norm_w, float eps,
    const int64_t* __restrict__ positions, const float* __restrict__ cos_sin, int neox,
    __nv_bfloat16* __restrict__ cache, const int64_t* __restrict__ slots, int page_size,
    __nv_bfloat16* __restrict__ qf, int qf_stride) {
  snb::pdl_wait();
  snb::pdl_trigger();
  extern __shared__ float sm[];  // [r + rope] latent row, then [H * rope] q_pe
  __shared__ float red[kThreadsMR / 32];
  const int t = blockIdx.x, tid = threadIdx.x;
  const __nv_bfloat16* a = kv_a + (size_t)t * kv_stride;
  float* lat = sm;
  float* qp = sm + r + rope;
  float ss = 0.f;
  for (int e = tid; e < r + rope; e += kThreadsMR) {
    const float v = __bfloat162float(a[e]);
    lat[e] = v;
    if (e < r) ss += v * v;
  }
  const __nv_bfloat16* qt = q + (size_t)t * q_stride;
  for (int i = tid; i < H * rope; i += kThreadsMR) {
    const int h = i / rope, e = i % rope;
    qp[i] = __bfloat162float(qt[(size_t)h * (nope + rope) + nope + e]);
  }
  ss = snb::warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kThreadsMR / 32; ++w) tot += red[w];
  const float inv = rsqrtf(tot / (float)r + eps);
  const float* cs = cos_sin + (size_t)positions[t] * rope;
  const int half = rope / 2;
  const int64_t slot = slots[t];
  if (slot >= 0) {
    __nv_bfloat16* row = cache + ((size_t)(slot / page_size) * page_size + slot % page_size) * (r + rope);
    for (int e = tid; e < r + rope; e += kThreadsMR) {
      const float v = e < r ? __bfloat162float(__float2bfloat16(lat[e] * inv * __bfloat162float(norm_w[e])))
                            : __bfloat162float(__float2bfloat16(rot(lat + r, e - r, half, neox != 0, cs)));
      row[e] = __float2bfloat16(v);
    }
  }
  __nv_bfloat16* qo = qf + (size_t)t * qf_stride;
  for (int i = tid; i < H * rope; i += kThreadsMR) {
    const int h = i / rope, e = i % rope;
    qo[(size_t)h * (r + rope) + r + e] = __float2bfloat16(rot(qp + h * rope, e, half, neox != 0, cs));
  }
}

}  // namespace

// kv_a: [T, r + rope] bf16; q: [T, H * (nope + rope)] bf16; cache: latent pool [pages, 1, page, r + rope] bf16;
// slots [T] int64 (< 0: no write); qf: [T, H * (r + rope)] bf16 (the rope columns of every head are written).
void mla_rope_latent(torch::Tensor kv_a, torch::Tensor q, int64_t H, int64_t nope, int64_t r, int64_t rope,
                     torch::Tensor norm_w, double eps, torch::Tensor positions, torch::Tensor cos_sin, bool neox,
                     torch::Tensor cache, torch::Tensor slots, int64_t page_size, torch::Tensor qf) {
  const int T = kv_a.size(0);
  if (T == 0) return;
  TORCH_CHECK(kv_a.scalar_type() == at::kBFloat16 && q.scalar_type() == at::kBFloat16 &&
                  cache.scalar_type() == at::kBFloat16 && qf.scalar_type() == at::kBFloat16,
              "mla_rope_latent: bf16 tensors and a bf16 latent pool");
  TORCH_CHECK(kv_a.stride(1) == 1 && q.stride(1) == 1 && qf.stride(1) == 1 && cache.is_contiguous(),
              "mla_rope_latent: layouts");
  TORCH_CHECK(kv_a.size(1) >= r + rope && q.size(1) >= H * (nope + rope) && qf.size(1) >= H * (r + rope) &&
                  cache.size(-1) == r + rope && rope % 2 == 0 && cos_sin.size(1) == rope,
              "mla_rope_latent: shapes");
  const size_t smem = (size_t)(r + rope + H * rope) * sizeof(float);
  TORCH_CHECK(smem <= 48 * 1024, "mla_rope_latent: too many heads");
  C10_CUDA_CHECK(snb::launch_pdl(mla_rope_latent_kernel, T, kThreadsMR, smem, at::cuda::getCurrentCUDAStream(),
                                 (const __nv_bfloat16*)kv_a.data_ptr(), (int)kv_a.stride(0),
                                 (const __nv_bfloat16*)q.data_ptr(), (int)q.stride(0), (int)H, (int)nope, (int)r,
                                 (int)rope, (const __nv_bfloat16*)norm_w.data_ptr(), (float)eps,
                                 positions.data_ptr<int64_t>(), cos_sin.data_ptr<float>(), (int)neox,
                                 (__nv_bfloat16*)cache.data_ptr(), slots.data_ptr<int64_t>(), (int)page_size,
                                 (__nv_bfloat16*)qf.data_ptr(), (int)qf.stride(0)));
}
