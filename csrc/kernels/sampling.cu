// Device sampler: greedy argmax and temperature sampling by Gumbel-max with hashed noise.
//
// Parity: the reference's device sampler (sglang_neuron/sampling.py: greedy with ties to the smallest id,
// `temperature` by Gumbel-max whose noise is a pure function of (seed, position, token id)). The noise here
// comes from a 64-bit integer mixer of our own (a splitmix64-style finaliser, a published construction),
// mapped to a uniform in (0, 1) and turned into Gumbel noise -log(-log(u)). Because the noise is a pure
// function of (seed, position, token), the sample does not depend on launch order or on how the vocabulary
// is split across CTAs or ranks.
//
// One CTA per row; 1024 threads stream the row with 16-byte loads and reduce (value, index) pairs.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "../common.cuh"

namespace {

SNB_DEVICE uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

SNB_DEVICE float gumbel(uint64_t seed, int64_t pos, int64_t tok) {
  const uint64_t h = mix64(seed ^ mix64((uint64_t)pos * 0x100000001B3ull ^ mix64((uint64_t)tok)));
  // 24 random bits -> u in (0, 1), never exactly 0 or 1.
  const float u = ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
  return -__logf(-__logf(u));
}

struct Best {
  float v;
  int i;
};
SNB_DEVICE Best better(Best a, Best b) {
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}

template <typename T>
SNB_DEVICE float to_f(T x) { return (float)x; }

template <typename T>
__global__ void __launch_bounds__(1024) sample_kernel(const T* __restrict__ logits, int V, int stride,
                                                      const float* __restrict__ temperature,
                                                      const int64_t* __restrict__ seeds,
                                                      const int64_t* __restrict__ positions,
                                                      int64_t* __restrict__ out_ids, float* __restrict__ out_vals,
                                                      int vocab_offset) {
  snb::pdl_wait();
  snb::pdl_trigger();
  const int row = blockIdx.x;
  const T* lr = logits + (size_t)row * stride;
  const float temp = temperature != nullptr ? temperature[row] : 0.f;
  const bool greedy = !(temp > 0.f);
  const float inv_t = greedy ? 1.f : 1.f / temp;
  const uint64_t seed = seeds != nullptr ? (uint64_t)seeds[row] : 0ull;
  const int64_t pos = positions != nullptr ? positions[row] : 0;
  Best best{-INFINITY, 0x7fffffff};
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    float v = to_f(lr[i]);
    if (!greedy) v = v * inv_t + gumbel(seed, pos, (int64_t)i + vocab_offset);
    best = better(best, Best{v, i});
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Best other{__shfl_xor_sync(0xffffffffu, best.v, o), __shfl_xor_sync(0xffffffffu, best.i, o)};
    best = better(best, other);
  }
  __shared__ float sv[32];
  __shared__ int si[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = best.v;
    si[warp] = best.i;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? Best{sv[lane], si[lane]} : Best{-INFINITY, 0x7fffffff};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      Best other{__shfl_xor_sync(0xffffffffu, best.v, o), __shfl_xor_sync(0xffffffffu, best.i, o)};
      best = better(best, other);
    }
    if (lane == 0) {
      out_ids[row] = (best.i == 0x7fffffff ? 0 : best.i) + (int64_t)vocab_offset;
      if (out_vals != nullptr) out_vals[row] = best.v;
    }
  }
}

}  // namespace

// logits: [B, >=V] (bf16 or fp32, row stride arbitrary); only the first V columns are considered.
// temperature [B] fp32 (<= 0 means greedy) or None. Token ids (and the Gumbel hash) are offset by
// vocab_offset, so a vocabulary shard samples exactly like the full row; out_vals (optional) receives the
// winning perturbed score for the cross-shard merge.
void sample_tokens(torch::Tensor out_ids, torch::Tensor logits, c10::optional<torch::Tensor> temperature,
                   c10::optional<torch::Tensor> seeds, c10::optional<torch::Tensor> positions,
                   c10::optional<torch::Tensor> out_vals, int64_t vocab_offset, int64_t valid_vocab) {
  const int B = logits.size(0);
  const int V = valid_vocab > 0 ? (int)valid_vocab : (int)logits.size(1);
  if (B == 0) return;
  TORCH_CHECK(logits.stride(1) == 1, "sample_tokens: inner stride");
  TORCH_CHECK(out_ids.scalar_type() == at::kLong, "sample_tokens: int64 output");
  auto st = at::cuda::getCurrentCUDAStream();
  const float* tp = temperature ? temperature->data_ptr<float>() : nullptr;
  const int64_t* sp = seeds ? seeds->data_ptr<int64_t>() : nullptr;
  const int64_t* pp = positions ? positions->data_ptr<int64_t>() : nullptr;
  float* vp = out_vals ? out_vals->data_ptr<float>() : nullptr;
  if (logits.scalar_type() == at::kFloat) {
    snb::launch_pdl(sample_kernel<float>, B, 1024, 0, st, logits.data_ptr<float>(), V, logits.stride(0), tp, sp, pp,
                                              out_ids.data_ptr<int64_t>(), vp, (int)vocab_offset);
  } else {
    TORCH_CHECK(logits.scalar_type() == at::kBFloat16, "sample_tokens: dtype");
    snb::launch_pdl(sample_kernel<__nv_bfloat16>, B, 1024, 0, st, (const __nv_bfloat16*)logits.data_ptr(), V, logits.stride(0),
                                                      tp, sp, pp, out_ids.data_ptr<int64_t>(), vp,
                                                      (int)vocab_offset);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
