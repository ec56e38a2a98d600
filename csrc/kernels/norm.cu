// RMSNorm kernels (plain and fused residual-add), bf16/fp32 activations, fp32 math.
//
// Parity: the reference's `rmsnorm_residual_prefill` op (sglang_neuron/ops/rmsnorm_residual_prefill.py:16)
// returns (norm(x + r), x + r); `fused_add_rmsnorm` here computes the same pair in place:
// residual <- x + residual, x <- rmsnorm(residual) * w.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "../common.cuh"

namespace {

template <typename T>
struct Vec8;
template <>
struct Vec8<__nv_bfloat16> {
  static constexpr int N = 8;
  static SNB_DEVICE void load(const __nv_bfloat16* p, float (&f)[8]) {
    snb::unpack_bf16x8(*reinterpret_cast<const uint4*>(p), f);
  }
  static SNB_DEVICE void store(__nv_bfloat16* p, const float (&f)[8]) {
    *reinterpret_cast<uint4*>(p) = snb::pack_bf16x8(f);
  }
};
template <>
struct Vec8<float> {
  static constexpr int N = 8;
  static SNB_DEVICE void load(const float* p, float (&f)[8]) {
    float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  }
  static SNB_DEVICE void store(float* p, const float (&f)[8]) {
    reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
  }
};

constexpr int kMaxVecPerThread = 4;  // up to 8 * 4 * 256 = 8192 columns with 256 threads

// One CTA per row. Keeps the row in registers (H <= 8192), two passes over registers only.
template <typename T, typename W, bool kResidual>
__global__ void rmsnorm_kernel(T* __restrict__ out, T* __restrict__ x, T* __restrict__ residual,
                               const W* __restrict__ weight, int H, int stride_x, int stride_out,
                               int stride_res, float eps, bool weight_plus_one) {
  snb::pdl_wait();
  snb::pdl_trigger();
  const int row = blockIdx.x;
  const int nvec = H / 8;
  T* xr = x + (size_t)row * stride_x;
  T* rr = kResidual ? residual + (size_t)row * stride_res : nullptr;
  float v[kMaxVecPerThread][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVecPerThread; ++i) {
    int vi = threadIdx.x + i * blockDim.x;
    if (vi < nvec) {
      Vec8<T>::load(xr + vi * 8, v[i]);
      if (kResidual) {
        float r[8];
        Vec8<T>::load(rr + vi * 8, r);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] += r[j];
        Vec8<T>::store(rr + vi * 8, v[i]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
  }
  __shared__ float red[32];
  ss = snb::warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = snb::warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / (float)H + eps);
  T* orow = out + (size_t)row * stride_out;
#pragma unroll
  for (int i = 0; i < kMaxVecPerThread; ++i) {
    int vi = threadIdx.x + i * blockDim.x;
    if (vi < nvec) {
      float w[8];
      Vec8<W>::load(weight + vi * 8, w);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = v[i][j] * inv * (weight_plus_one ? (w[j] + 1.f) : w[j]);
      Vec8<T>::store(orow + vi * 8, v[i]);
    }
  }
}

// Per-head RMSNorm over the last dim of a [T, heads, D] view (QK-norm). One warp per head row.
template <typename T, typename W>
__global__ void head_rmsnorm_kernel(T* __restrict__ x, const W* __restrict__ weight, int rows, int D,
                                    int heads, int stride_tok, float eps) {
  snb::pdl_wait();
  snb::pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const int t = warp / heads, h = warp % heads;
  T* p = x + (size_t)t * stride_tok + (size_t)h * D;
  float vals[8];
  float ss = 0.f;
  const int per = D / 32;  // D in {64, 128, 256}
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (i < per) {
      float f = (float)p[lane + 32 * i];
      vals[i] = f;
      ss += f * f;
    }
  }
  ss = snb::warp_sum(ss);
  const float inv = rsqrtf(ss / (float)D + eps);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (i < per) p[lane + 32 * i] = (T)(vals[i] * inv * (float)weight[lane + 32 * i]);
  }
}

}  // namespace

void rmsnorm_out(torch::Tensor out, torch::Tensor x, torch::Tensor weight, double eps,
                 bool weight_plus_one) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.stride(1) == 1, "rmsnorm: x must be a 2D CUDA row-major view");
  const int T = x.size(0), H = x.size(1);
  TORCH_CHECK(H % 8 == 0 && H <= 8 * kMaxVecPerThread * 256, "rmsnorm: unsupported hidden size ", H);
  if (T == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  const int threads = 256;
  if (x.scalar_type() == at::kBFloat16) {
    TORCH_CHECK(weight.scalar_type() == at::kBFloat16, "rmsnorm: bf16 x needs bf16 weight");
    snb::launch_pdl(rmsnorm_kernel<__nv_bfloat16, __nv_bfloat16, false>, T, threads, 0, stream,
        (__nv_bfloat16*)out.data_ptr(), (__nv_bfloat16*)x.data_ptr(), nullptr,
        (const __nv_bfloat16*)weight.data_ptr(), H, x.stride(0), out.stride(0), 0, (float)eps,
        weight_plus_one);
  } else {
    TORCH_CHECK(x.scalar_type() == at::kFloat && weight.scalar_type() == at::kFloat, "rmsnorm: dtype");
    snb::launch_pdl(rmsnorm_kernel<float, float, false>, T, threads, 0, stream,
        out.data_ptr<float>(), x.data_ptr<float>(), nullptr, weight.data_ptr<float>(), H, x.stride(0),
        out.stride(0), 0, (float)eps, weight_plus_one);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void fused_add_rmsnorm(torch::Tensor x, torch::Tensor residual, torch::Tensor weight, double eps,
                       bool weight_plus_one) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && residual.sizes() == x.sizes(), "fused_add_rmsnorm: shapes");
  const int T = x.size(0), H = x.size(1);
  TORCH_CHECK(H % 8 == 0 && H <= 8 * kMaxVecPerThread * 256, "fused_add_rmsnorm: hidden size ", H);
  if (T == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  if (x.scalar_type() == at::kBFloat16) {
    snb::launch_pdl(rmsnorm_kernel<__nv_bfloat16, __nv_bfloat16, true>, T, 256, 0, stream,
        (__nv_bfloat16*)x.data_ptr(), (__nv_bfloat16*)x.data_ptr(), (__nv_bfloat16*)residual.data_ptr(),
        (const __nv_bfloat16*)weight.data_ptr(), H, x.stride(0), x.stride(0), residual.stride(0),
        (float)eps, weight_plus_one);
  } else {
    snb::launch_pdl(rmsnorm_kernel<float, float, true>, T, 256, 0, stream,
        x.data_ptr<float>(), x.data_ptr<float>(), residual.data_ptr<float>(), weight.data_ptr<float>(),
        H, x.stride(0), x.stride(0), residual.stride(0), (float)eps, weight_plus_one);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void head_rmsnorm_(torch::Tensor x, torch::Tensor weight, int64_t heads, double eps) {
  // x: [T, heads * D] (row stride arbitrary), normalised per head in place.
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.stride(1) == 1, "head_rmsnorm: x layout");
  const int T = x.size(0);
  const int D = weight.size(0);
  TORCH_CHECK(D % 32 == 0 && D <= 256, "head_rmsnorm: head dim ", D);
  const int rows = T * heads;
  if (rows == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  const int threads = 256, blocks = (rows * 32 + threads - 1) / threads;
  if (x.scalar_type() == at::kBFloat16) {
    snb::launch_pdl(head_rmsnorm_kernel<__nv_bfloat16, __nv_bfloat16>, blocks, threads, 0, stream,
        (__nv_bfloat16*)x.data_ptr(), (const __nv_bfloat16*)weight.data_ptr(), rows, D, heads,
        x.stride(0), (float)eps);
  } else {
    snb::launch_pdl(head_rmsnorm_kernel<float, float>, blocks, threads, 0, stream,
        x.data_ptr<float>(), weight.data_ptr<float>(), rows, D, heads, x.stride(0), (float)eps);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
