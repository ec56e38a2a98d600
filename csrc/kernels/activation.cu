// Gated activations of the dense MLP: out[t, j] = act(x[t, j]) * x[t, I + j] over a [T, 2I] gate|up row.
// Parity: the reference's dense MLP computes SiLU(gate) * up between its fused gate_up and down projections
// (sglang_neuron/models/transformer/model.py:156-173). bf16 in/out, fp32 math, 16-byte accesses.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "../common.cuh"

namespace {

__global__ void silu_and_mul_kernel(const __nv_bfloat16* __restrict__ x, int xs, __nv_bfloat16* __restrict__ out,
                                    int os, int I) {
  snb::pdl_wait();
  snb::pdl_trigger();
  const int t = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;  // 8-element chunk
  if (c * 8 >= I) return;
  float g[8], u[8], r[8];
  snb::unpack_bf16x8(*reinterpret_cast<const uint4*>(x + (size_t)t * xs + c * 8), g);
  snb::unpack_bf16x8(*reinterpret_cast<const uint4*>(x + (size_t)t * xs + I + c * 8), u);
#pragma unroll
  for (int i = 0; i < 8; ++i) r[i] = g[i] / (1.f + __expf(-g[i])) * u[i];
  *reinterpret_cast<uint4*>(out + (size_t)t * os + c * 8) = snb::pack_bf16x8(r);
}

}  // namespace

void silu_and_mul(torch::Tensor out, torch::Tensor x) {
  const int T = x.size(0), I = x.size(1) / 2;
  if (T == 0) return;
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && I % 8 == 0 && x.stride(1) == 1, "silu_and_mul: layout");
  dim3 grid((I / 8 + 127) / 128, T);
  snb::launch_pdl(silu_and_mul_kernel, grid, 128, 0, at::cuda::getCurrentCUDAStream(),
      (const __nv_bfloat16*)x.data_ptr(), x.stride(0), (__nv_bfloat16*)out.data_ptr(), out.stride(0), I);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
