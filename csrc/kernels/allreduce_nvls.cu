// Tensor-parallel all-reduce through NVSwitch multicast (NVLS): multimem.ld_reduce / multimem.st.
//
// Every rank owns one symmetric buffer (same offsets on every rank) that is also bound to an NVLink
// multicast object, so an address in the multicast range names that offset on every rank at once:
// `multimem.ld_reduce` returns the sum over all ranks (the switch reduces), `multimem.st` writes every
// rank's copy, `multimem.red` increments every rank's copy of a flag.
//
// One kernel per call, CTA b owns chunk b of the message on every rank:
//   1. produce chunk b into this rank's buffer: a plain copy of the input, the MoE combine (weighted sum of
//      this rank's expert rows per token) or the split-K partial sum of a row-parallel GEMM (+ bias);
//   2. barrier A (flag b): multimem.red +1 on every rank, wait until this rank's copy reaches epoch * world;
//   3. the rank reduces its 1/world share of chunk b through the switch and multicasts the sum back;
//   4. barrier B (flag b), then copy chunk b of the result out of the buffer.
// NVLink traffic per rank is about 2/world of the message instead of (world - 1) x the message of a
// push-to-every-peer all-reduce. Waits are bounded (SNB_WAIT_NS): a timeout records a status code.
//
// Buffer layout: [capacity bytes of data][flags A: kMaxCtas u32][flags B: kMaxCtas u32][uses: kMaxCtas u32].
// Flag b only grows, by world per call that runs a CTA b; uses[b] (local, never multicast) counts those calls
// on this rank, so the target of a barrier is (uses[b] + 1) * world whatever grid sizes earlier calls had
// (every rank runs the same sequence of calls, so every rank's uses[b] agree).
// Parity: the reference's traced all-reduce (sglang_neuron/parallel/collectives.py:22-55) and the MoE partial
// all-reduce (models/qwen3_moe/moe.py:77, models/gpt_oss/mxfp4/common.py:356).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <algorithm>
#include "../common.cuh"

namespace {

constexpr int kMaxCtasNv = 1024;
constexpr int kThreadsNv = 256;

enum NvMode { NV_COPY = 0, NV_COMBINE = 1, NV_SPLITK = 2 };

struct NvArgs {
  uint8_t* uc;  // this rank's buffer
  uint8_t* mc;  // multicast address of the same buffer
  size_t capacity;
  int rank, world;
};

SNB_DEVICE uint32_t* flags_a(uint8_t* base, size_t cap) { return reinterpret_cast<uint32_t*>(base + cap); }
SNB_DEVICE uint32_t* flags_b(uint8_t* base, size_t cap) { return flags_a(base, cap) + kMaxCtasNv; }
SNB_DEVICE uint32_t* uses_ptr(uint8_t* base, size_t cap) { return flags_b(base, cap) + kMaxCtasNv; }

SNB_DEVICE void mm_red_add_release(uint32_t* mc_addr, uint32_t v) {
  asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(mc_addr), "r"(v) : "memory");
}
SNB_DEVICE uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
SNB_DEVICE uint4 mm_ld_reduce_bf16x8(const void* mc_addr) {
  uint4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(mc_addr)
               : "memory");
  return r;
}
SNB_DEVICE void mm_st_bf16x8(void* mc_addr, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(mc_addr), "r"(v.x),
               "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Barrier over the ranks for CTA b: every rank's CTA b has passed the same point of this call.
SNB_DEVICE bool nv_barrier(const NvArgs& a, uint32_t* flag_uc, uint32_t* flag_mc, uint32_t target, int* status) {
  __shared__ int ok_s;
  __syncthreads();
  if (threadIdx.x == 0) {
    ok_s = 1;
    __threadfence_system();
    mm_red_add_release(flag_mc, 1u);
    const uint64_t t0 = snb::globaltimer_ns();
    while (ld_acquire_sys_u32(flag_uc) < target) {
      if (snb::globaltimer_ns() - t0 > SNB_WAIT_NS) {
        snb::record_status(status, SNB_ERR_TIMEOUT_PEER);
        ok_s = 0;
        break;
      }
    }
  }
  __syncthreads();
  return ok_s != 0;
}

template <int MODE>
__global__ void __launch_bounds__(kThreadsNv) nvls_allreduce_kernel(
    NvArgs a, const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ y, int ys,
    const int32_t* __restrict__ inv_map, const float* __restrict__ w, int K, const float* __restrict__ partial,
    int splits, const __nv_bfloat16* __restrict__ bias, int rows, int cols, __nv_bfloat16* __restrict__ out,
    int* status) {
  snb::pdl_wait();
  snb::pdl_trigger();
  uint32_t* uses = uses_ptr(a.uc, a.capacity) + blockIdx.x;
  const uint32_t e = *reinterpret_cast<volatile uint32_t*>(uses) + 1;
  const uint32_t target = e * (uint32_t)a.world;
  const int64_t nvec = (int64_t)rows * cols / 8;
  const int64_t per = (nvec + gridDim.x - 1) / gridDim.x;
  const int64_t v0 = blockIdx.x * per, v1 = min(nvec, v0 + per);
  uint4* data = reinterpret_cast<uint4*>(a.uc);
  const int cv = cols / 8;
  // 1. produce this rank's contribution to chunk b
  for (int64_t v = v0 + threadIdx.x; v < v1; v += blockDim.x) {
    uint4 packed;
    if constexpr (MODE == NV_COPY) {
      packed = reinterpret_cast<const uint4*>(x)[v];
    } else if constexpr (MODE == NV_COMBINE) {
      const int t = (int)(v / cv), c = (int)(v % cv);
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int j = 0; j < K; ++j) {
        const int r = inv_map[t * K + j];
        if (r < 0) continue;
        const float wj = w[t * K + j];
        float f[8];
        snb::unpack_bf16x8(reinterpret_cast<const uint4*>(y + (size_t)r * ys)[c], f);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] += wj * f[i];
      }
      packed = snb::pack_bf16x8(acc);
    } else {
      const int c8 = (int)(v % cv) * 8;
      float acc[8];
      if (bias != nullptr) {
        snb::unpack_bf16x8(*reinterpret_cast<const uint4*>(bias + c8), acc);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.f;
      }
      for (int z = 0; z < splits; ++z) {
        const float4* pz = reinterpret_cast<const float4*>(partial + (size_t)z * rows * cols + v * 8);
        const float4 p0 = pz[0], p1 = pz[1];
        acc[0] += p0.x; acc[1] += p0.y; acc[2] += p0.z; acc[3] += p0.w;
        acc[4] += p1.x; acc[5] += p1.y; acc[6] += p1.z; acc[7] += p1.w;
      }
      packed = snb::pack_bf16x8(acc);
    }
    data[v] = packed;
  }
  // 2. every rank's chunk b is in place
  bool ok = nv_barrier(a, flags_a(a.uc, a.capacity) + blockIdx.x, flags_a(a.mc, a.capacity) + blockIdx.x, target,
                       status);
  // 3. reduce this rank's share of chunk b through the switch, multicast the sum
  if (ok) {
    const int64_t share = (v1 - v0 + a.world - 1) / a.world;
    const int64_t s0 = v0 + a.rank * share, s1 = min(v1, s0 + share);
    uint4* mdata = reinterpret_cast<uint4*>(a.mc);
    for (int64_t v = s0 + threadIdx.x; v < s1; v += blockDim.x) mm_st_bf16x8(mdata + v, mm_ld_reduce_bf16x8(mdata + v));
  }
  // 4. every share of chunk b is written everywhere; copy it out
  ok = nv_barrier(a, flags_b(a.uc, a.capacity) + blockIdx.x, flags_b(a.mc, a.capacity) + blockIdx.x, target,
                  status) && ok;
  if (ok) {
    uint4* o = reinterpret_cast<uint4*>(out);
    for (int64_t v = v0 + threadIdx.x; v < v1; v += blockDim.x) o[v] = data[v];
  }
  __syncthreads();
  if (threadIdx.x == 0) *uses = e;
}

NvArgs make_args(int64_t uc, int64_t mc, int64_t capacity, int64_t rank, int64_t world) {
  NvArgs a;
  a.uc = reinterpret_cast<uint8_t*>(uc);
  a.mc = reinterpret_cast<uint8_t*>(mc);
  a.capacity = (size_t)capacity;
  a.rank = (int)rank;
  a.world = (int)world;
  return a;
}

int pick_ctas(int64_t nvec, int64_t max_ctas) {
  // about 2 KB of every rank's share per CTA, so the switch sees many requests in flight
  return (int)std::max<int64_t>(1, std::min<int64_t>({max_ctas, (int64_t)kMaxCtasNv, (nvec + 127) / 128}));
}

}  // namespace

// Bytes past `capacity` that the flag area needs (the buffer must be capacity + this, zeroed once).
int64_t nvls_flag_bytes() { return 3 * kMaxCtasNv * 4; }

// out = sum over ranks of x; x, out: contiguous bf16 with numel % 8 == 0 and numel * 2 <= capacity.
void nvls_allreduce(torch::Tensor out, torch::Tensor x, int64_t uc, int64_t mc, int64_t capacity, int64_t rank,
                    int64_t world, int64_t max_ctas, torch::Tensor status) {
  TORCH_CHECK(x.is_contiguous() && out.is_contiguous() && x.numel() % 8 == 0, "nvls_allreduce: layout");
  TORCH_CHECK(x.numel() * 2 <= capacity, "nvls_allreduce: over capacity");
  const int64_t nvec = x.numel() / 8;
  if (nvec == 0) return;
  C10_CUDA_CHECK(snb::launch_pdl(nvls_allreduce_kernel<NV_COPY>, pick_ctas(nvec, max_ctas), kThreadsNv, 0,
                                 at::cuda::getCurrentCUDAStream(), make_args(uc, mc, capacity, rank, world),
                                 (const __nv_bfloat16*)x.data_ptr(), nullptr, 0, nullptr, nullptr, 0, nullptr, 0,
                                 nullptr, 1, (int)x.numel(), (__nv_bfloat16*)out.data_ptr(), status.data_ptr<int>()));
}

// MoE combine (out[t] = sum_j w[t,j] * y[inv_map[t,j]]) fused with the all-reduce.
void nvls_combine_allreduce(torch::Tensor out, torch::Tensor y, torch::Tensor inv_map, torch::Tensor w, int64_t uc,
                            int64_t mc, int64_t capacity, int64_t rank, int64_t world, int64_t max_ctas,
                            torch::Tensor status) {
  const int T = out.size(0), H = out.size(1);
  const int K = inv_map.numel() / std::max(T, 1);
  TORCH_CHECK(H % 8 == 0 && out.is_contiguous() && y.stride(1) == 1, "nvls_combine_allreduce: layout");
  TORCH_CHECK((int64_t)T * H * 2 <= capacity, "nvls_combine_allreduce: over capacity");
  if (T == 0) return;
  C10_CUDA_CHECK(snb::launch_pdl(nvls_allreduce_kernel<NV_COMBINE>, pick_ctas((int64_t)T * H / 8, max_ctas),
                                 kThreadsNv, 0, at::cuda::getCurrentCUDAStream(),
                                 make_args(uc, mc, capacity, rank, world), nullptr,
                                 (const __nv_bfloat16*)y.data_ptr(), (int)y.stride(0), inv_map.data_ptr<int32_t>(),
                                 w.data_ptr<float>(), K, nullptr, 0, nullptr, T, H, (__nv_bfloat16*)out.data_ptr(),
                                 status.data_ptr<int>()));
}

// Split-K partial sum (+ bias) of a row-parallel GEMM fused with the all-reduce; partial: fp32 [splits, T, F].
void nvls_splitk_allreduce(torch::Tensor out, torch::Tensor partial, int64_t splits,
                           c10::optional<torch::Tensor> bias, int64_t uc, int64_t mc, int64_t capacity, int64_t rank,
                           int64_t world, int64_t max_ctas, torch::Tensor status) {
  const int T = out.size(0), F = out.size(1);
  TORCH_CHECK(F % 8 == 0 && out.is_contiguous() && partial.scalar_type() == at::kFloat, "nvls_splitk: layout");
  TORCH_CHECK(partial.numel() >= splits * T * F && (int64_t)T * F * 2 <= capacity, "nvls_splitk: sizes");
  if (T == 0) return;
  C10_CUDA_CHECK(snb::launch_pdl(nvls_allreduce_kernel<NV_SPLITK>, pick_ctas((int64_t)T * F / 8, max_ctas),
                                 kThreadsNv, 0, at::cuda::getCurrentCUDAStream(),
                                 make_args(uc, mc, capacity, rank, world), nullptr, nullptr, 0, nullptr, nullptr, 0,
                                 partial.data_ptr<float>(), (int)splits,
                                 bias ? (const __nv_bfloat16*)bias->data_ptr() : nullptr, T, F,
                                 (__nv_bfloat16*)out.data_ptr(), status.data_ptr<int>()));
}
