// One-shot all-reduce over NVLink peer memory (CUDA IPC mappings), for the tensor-parallel collectives of
// the decode path, plus the IPC plumbing that maps every rank's buffer into every other rank.
//
// Each rank owns one device buffer laid out as [2 halves][world slots][capacity bytes] followed by per-CTA
// flags [world][max CTAs], a call counter and a completion ticket. Every CTA of a call reads the same epoch
// e = counter + 1 (the last CTA to finish stores it), and the call uses half (e & 1):
//   1. CTA c stores its chunk of the local input into every peer's buffer, slot = my rank (P2P stores),
//   2. then publishes flag[peer][my rank][c] = e with a system-scope release store,
//   3. waits (bounded, acquire loads) until flag[me][q][c] >= e for every rank q,
//   4. sums the chunk over the world slots of its own buffer and writes the output.
// Chunk c of every rank is handled by CTA c on every rank, so no grid-wide barrier is needed. Two halves
// suffice: a rank can only start call e+2 after receiving every peer's data of call e+1, which each peer
// sends only after its own call e (including the reads of half e & 1) has finished.
//
// Parity: the reference's traced all-reduce of the TP group (sglang_neuron/parallel/collectives.py:22-55).
// NCCL stays available as the baseline; this path removes NCCL's launch and protocol latency for the
// few-hundred-KB messages of decode steps.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <cuda_runtime.h>
#include "../common.cuh"
#include "../ar_common.cuh"

using namespace snb_ar;

namespace {

constexpr int kThreadsAR = 512;

// kNorm: the reduce step also adds the residual and applies RMSNorm (ar_reduce_norm_store); chunks are rows.
template <bool kNorm>
__global__ void __launch_bounds__(kThreadsAR) one_shot_allreduce_kernel(
    ARPeers peers, int rank, int world, size_t capacity, const __nv_bfloat16* __restrict__ in,
    __nv_bfloat16* __restrict__ out, int64_t n, ARNorm nm, int* status) {
  snb::pdl_wait();
  snb::pdl_trigger();
  const ARBuf b = ar_layout(peers, rank, world, capacity);
  const uint32_t e = *reinterpret_cast<volatile uint32_t*>(b.counter) + 1;
  const int half = e & 1;
  int64_t v0, v1;
  int r0, r1;
  ar_chunk(n / 8, kNorm ? nm.H / 8 : 1, kNorm, v0, v1, r0, r1);
  for (int p = 0; p < world; ++p) {
    uint4* dst = reinterpret_cast<uint4*>(ar_slot(peers, p, half, rank, world, capacity));
    const uint4* src = reinterpret_cast<const uint4*>(in);
    for (int64_t v = v0 + threadIdx.x; v < v1; v += blockDim.x) dst[v] = src[v];
  }
  if (ar_exchange(peers, b, rank, world, capacity, e, status)) {
    if constexpr (kNorm) ar_reduce_norm_store(peers, half, world, capacity, rank, out, nm, r0, r1);
    else ar_reduce_store(peers, half, world, capacity, rank, out, v0, v1);
  }
  ar_finish(b, e);
}

// MoE combine fused with the expert-parallel all-reduce: each rank forms its partial
// sum_j w[t,j] * y[inv_map[t*K+j]] over the experts it owns, stores it straight into every peer's slot,
// and reduces the world's partials for its chunk of tokens. One launch replaces combine + all-reduce.
template <bool kNorm>
__global__ void __launch_bounds__(kThreadsAR) moe_combine_allreduce_kernel(
    ARPeers peers, int rank, int world, size_t capacity, const __nv_bfloat16* __restrict__ y, int ys,
    const int32_t* __restrict__ inv_map, const float* __restrict__ w, int K, int T, int H,
    __nv_bfloat16* __restrict__ out, ARNorm nm, int* status) {
  snb::pdl_wait();
  snb::pdl_trigger();
  const ARBuf b = ar_layout(peers, rank, world, capacity);
  const uint32_t e = *reinterpret_cast<volatile uint32_t*>(b.counter) + 1;
  const int half = e & 1;
  const int hv = H / 8;
  int64_t v0, v1;
  int r0, r1;
  ar_chunk((int64_t)T * hv, hv, kNorm, v0, v1, r0, r1);
  for (int64_t v = v0 + threadIdx.x; v < v1; v += blockDim.x) {
    const int t = (int)(v / hv), c = (int)(v % hv);
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
    const uint4 packed = snb::pack_bf16x8(acc);
    for (int p = 0; p < world; ++p) reinterpret_cast<uint4*>(ar_slot(peers, p, half, rank, world, capacity))[v] = packed;
  }
  if (ar_exchange(peers, b, rank, world, capacity, e, status)) {
    if constexpr (kNorm) ar_reduce_norm_store(peers, half, world, capacity, rank, out, nm, r0, r1);
    else ar_reduce_store(peers, half, world, capacity, rank, out, v0, v1);
  }
  ar_finish(b, e);
}

// Split-K GEMM epilogue fused with the all-reduce: sum the S fp32 partial tiles of this rank (+ bias),
// push the bf16 result into every peer's slot, and reduce the world's copies. Together with the split-K
// tcgen05 GEMM this makes a row-parallel projection + all-reduce two launches with every SM busy.
template <bool kNorm>
__global__ void __launch_bounds__(kThreadsAR) splitk_allreduce_kernel(
    ARPeers peers, int rank, int world, size_t capacity, const float* __restrict__ partial, int splits,
    const __nv_bfloat16* __restrict__ bias, int T, int F, __nv_bfloat16* __restrict__ out, ARNorm nm,
    int* status) {
  snb::pdl_wait();
  snb::pdl_trigger();
  const ARBuf b = ar_layout(peers, rank, world, capacity);
  const uint32_t e = *reinterpret_cast<volatile uint32_t*>(b.counter) + 1;
  const int half = e & 1;
  const int fv = F / 8;
  int64_t v0, v1;
  int r0, r1;
  ar_chunk((int64_t)T * fv, fv, kNorm, v0, v1, r0, r1);
  for (int64_t v = v0 + threadIdx.x; v < v1; v += blockDim.x) {
    const int f8 = (int)(v % fv) * 8;
    float acc[8];
    if (bias != nullptr) {
      snb::unpack_bf16x8(*reinterpret_cast<const uint4*>(bias + f8), acc);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    }
    for (int z = 0; z < splits; ++z) {
      const float4* pz = reinterpret_cast<const float4*>(partial + (size_t)z * T * F + v * 8);
      const float4 a0 = pz[0], a1 = pz[1];
      acc[0] += a0.x; acc[1] += a0.y; acc[2] += a0.z; acc[3] += a0.w;
      acc[4] += a1.x; acc[5] += a1.y; acc[6] += a1.z; acc[7] += a1.w;
    }
    const uint4 packed = snb::pack_bf16x8(acc);
    for (int p = 0; p < world; ++p) reinterpret_cast<uint4*>(ar_slot(peers, p, half, rank, world, capacity))[v] = packed;
  }
  if (ar_exchange(peers, b, rank, world, capacity, e, status)) {
    if constexpr (kNorm) ar_reduce_norm_store(peers, half, world, capacity, rank, out, nm, r0, r1);
    else ar_reduce_store(peers, half, world, capacity, rank, out, v0, v1);
  }
  ar_finish(b, e);
}

// Sequence-parallel all-gather over NVLink: rank r's block [n8 vectors] goes into slot r of every rank's
// buffer (peer stores, CTA c owns chunk c of the block), then each rank copies every slot's chunk c into the
// rank-major output. One launch, no NCCL; the bytes each rank sends are the block times the world.
__global__ void __launch_bounds__(kThreadsAR) sp_allgather_kernel(ARPeers peers, int rank, int world, size_t capacity,
                                                                 const __nv_bfloat16* __restrict__ in,
                                                                 __nv_bfloat16* __restrict__ out, int64_t n8,
                                                                 int* status) {
  snb::pdl_wait();
  snb::pdl_trigger();
  const ARBuf b = ar_layout(peers, rank, world, capacity);
  const uint32_t e = *reinterpret_cast<volatile uint32_t*>(b.counter) + 1;
  const int half = e & 1;
  int64_t v0, v1;
  int r0, r1;
  ar_chunk(n8, 1, false, v0, v1, r0, r1);
  const uint4* src = reinterpret_cast<const uint4*>(in);
  for (int p = 0; p < world; ++p) {
    uint4* dst = reinterpret_cast<uint4*>(ar_slot(peers, p, half, rank, world, capacity));
    for (int64_t v = v0 + threadIdx.x; v < v1; v += blockDim.x) dst[v] = src[v];
  }
  if (ar_exchange(peers, b, rank, world, capacity, e, status)) {
    for (int q = 0; q < world; ++q) {
      const uint4* s = reinterpret_cast<const uint4*>(ar_slot(peers, rank, half, q, world, capacity));
      uint4* o = reinterpret_cast<uint4*>(out) + (int64_t)q * n8;
      for (int64_t v = v0 + threadIdx.x; v < v1; v += blockDim.x) o[v] = s[v];
    }
  }
  ar_finish(b, e);
}

// Sequence-parallel reduce-scatter over NVLink: `in` holds world blocks of n8 vectors (partial sums of every
// row); block j goes into slot `rank` of rank j's buffer, then each rank sums the world slots of its own
// block (fp32, rank order) into out. The bytes each rank sends are (world - 1) / world of its partials.
__global__ void __launch_bounds__(kThreadsAR) sp_reducescatter_kernel(ARPeers peers, int rank, int world,
                                                                     size_t capacity,
                                                                     const __nv_bfloat16* __restrict__ in,
                                                                     __nv_bfloat16* __restrict__ out, int64_t n8,
                                                                     int* status) {
  snb::pdl_wait();
  snb::pdl_trigger();
  const ARBuf b = ar_layout(peers, rank, world, capacity);
  const uint32_t e = *reinterpret_cast<volatile uint32_t*>(b.counter) + 1;
  const int half = e & 1;
  int64_t v0, v1;
  int r0, r1;
  ar_chunk(n8, 1, false, v0, v1, r0, r1);
  for (int j = 0; j < world; ++j) {
    const uint4* src = reinterpret_cast<const uint4*>(in) + (int64_t)j * n8;
    uint4* dst = reinterpret_cast<uint4*>(ar_slot(peers, j, half, rank, world, capacity));
    for (int64_t v = v0 + threadIdx.x; v < v1; v += blockDim.x) dst[v] = src[v];
  }
  if (ar_exchange(peers, b, rank, world, capacity, e, status))
    ar_reduce_store(peers, half, world, capacity, rank, out, v0, v1);
  ar_finish(b, e);
}

}  // namespace

void sp_allgather(torch::Tensor out, torch::Tensor in, std::vector<int64_t> bufs, int64_t rank, int64_t capacity,
                  int64_t num_ctas, torch::Tensor status, int64_t wait_ns) {
  const int world = (int)bufs.size();
  TORCH_CHECK(world >= 1 && world <= kMaxRanks, "sp_allgather: world size");
  TORCH_CHECK(in.scalar_type() == at::kBFloat16 && in.is_contiguous() && out.is_contiguous(), "sp_allgather: bf16");
  const int64_t n = in.numel();
  TORCH_CHECK(n % 8 == 0 && out.numel() == n * world && (size_t)n * 2 <= (size_t)capacity, "sp_allgather: sizes");
  TORCH_CHECK(num_ctas >= 1 && num_ctas <= kMaxCtas, "sp_allgather: CTA count");
  if (n == 0) return;
  const ARPeers peers = make_peers(bufs, wait_ns);
  C10_CUDA_CHECK(snb::launch_pdl(sp_allgather_kernel, num_ctas, kThreadsAR, 0, at::cuda::getCurrentCUDAStream(),
                                 peers, (int)rank, world, (size_t)capacity, (const __nv_bfloat16*)in.data_ptr(),
                                 (__nv_bfloat16*)out.data_ptr(), n / 8, status.data_ptr<int>()));
}

void sp_reducescatter(torch::Tensor out, torch::Tensor in, std::vector<int64_t> bufs, int64_t rank, int64_t capacity,
                      int64_t num_ctas, torch::Tensor status, int64_t wait_ns) {
  const int world = (int)bufs.size();
  TORCH_CHECK(world >= 1 && world <= kMaxRanks, "sp_reducescatter: world size");
  TORCH_CHECK(in.scalar_type() == at::kBFloat16 && in.is_contiguous() && out.is_contiguous(),
              "sp_reducescatter: bf16");
  const int64_t n = out.numel();
  TORCH_CHECK(n % 8 == 0 && in.numel() == n * world && (size_t)n * 2 <= (size_t)capacity, "sp_reducescatter: sizes");
  TORCH_CHECK(num_ctas >= 1 && num_ctas <= kMaxCtas, "sp_reducescatter: CTA count");
  if (n == 0) return;
  const ARPeers peers = make_peers(bufs, wait_ns);
  C10_CUDA_CHECK(snb::launch_pdl(sp_reducescatter_kernel, num_ctas, kThreadsAR, 0,
                                 at::cuda::getCurrentCUDAStream(), peers, (int)rank, world, (size_t)capacity,
                                 (const __nv_bfloat16*)in.data_ptr(), (__nv_bfloat16*)out.data_ptr(), n / 8,
                                 status.data_ptr<int>()));
}

// --- IPC plumbing -----------------------------------------------------------------------------------
// Allocate the communicator buffer (cudaMalloc: IPC needs whole allocations, not caching-allocator blocks)
// and return (device pointer, IPC handle bytes).
std::tuple<int64_t, py::bytes> symm_alloc(int64_t capacity, int64_t world) {
  TORCH_CHECK(world >= 1 && world <= kMaxRanks, "symm_alloc: world size");
  const size_t bytes = 2 * (size_t)world * capacity + (kMaxRanks * kMaxCtas + 2) * sizeof(uint32_t);
  void* p = nullptr;
  TORCH_CHECK(cudaMalloc(&p, bytes) == cudaSuccess, "symm_alloc: cudaMalloc failed");
  TORCH_CHECK(cudaMemset(p, 0, bytes) == cudaSuccess, "symm_alloc: memset failed");
  cudaIpcMemHandle_t h;
  TORCH_CHECK(cudaIpcGetMemHandle(&h, p) == cudaSuccess, "symm_alloc: cudaIpcGetMemHandle failed");
  return {reinterpret_cast<int64_t>(p), py::bytes(reinterpret_cast<const char*>(&h), sizeof(h))};
}

int64_t symm_open(py::bytes handle) {
  std::string s = handle;
  TORCH_CHECK(s.size() == sizeof(cudaIpcMemHandle_t), "symm_open: bad handle");
  cudaIpcMemHandle_t h;
  memcpy(&h, s.data(), sizeof(h));
  void* p = nullptr;
  TORCH_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess,
              "symm_open: cudaIpcOpenMemHandle failed");
  return reinterpret_cast<int64_t>(p);
}

void symm_close(int64_t ptr, bool owned) {
  if (owned) cudaFree(reinterpret_cast<void*>(ptr));
  else cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr));
}

// Optional fused residual add + RMSNorm of a [T, H] call (H = weight size): `out` receives the normalised
// rows and `residual` is updated in place; the CTA count is then capped at T (one or more rows per CTA).
static ARNorm make_norm(const c10::optional<torch::Tensor>& residual, const c10::optional<torch::Tensor>& weight,
                        double eps, int64_t n, int64_t& num_ctas) {
  ARNorm nm{nullptr, nullptr, (float)eps, 0};
  if (!residual) return nm;
  TORCH_CHECK(weight && weight->scalar_type() == at::kBFloat16 && residual->scalar_type() == at::kBFloat16 &&
              residual->is_contiguous() && weight->is_contiguous(), "fused norm: bf16 contiguous residual/weight");
  const int64_t H = weight->numel();
  TORCH_CHECK(H % 8 == 0 && H <= kNormVecs * 8 * kThreadsAR && n % H == 0 && residual->numel() == n,
              "fused norm: hidden size ", H);
  nm.residual = (__nv_bfloat16*)residual->data_ptr();
  nm.weight = (const __nv_bfloat16*)weight->data_ptr();
  nm.H = (int)H;
  num_ctas = std::max<int64_t>(1, std::min<int64_t>(num_ctas, n / H));
  return nm;
}

void one_shot_allreduce(torch::Tensor out, torch::Tensor in, std::vector<int64_t> bufs, int64_t rank,
                        int64_t capacity, int64_t num_ctas, torch::Tensor status,
                        c10::optional<torch::Tensor> residual, c10::optional<torch::Tensor> weight, double eps,
                        int64_t wait_ns) {
  const int world = (int)bufs.size();
  TORCH_CHECK(world >= 1 && world <= kMaxRanks, "one_shot_allreduce: world size");
  TORCH_CHECK(in.scalar_type() == at::kBFloat16 && in.is_contiguous() && out.is_contiguous(), "one_shot_allreduce: bf16");
  const int64_t n = in.numel();
  TORCH_CHECK(n % 8 == 0 && (size_t)n * 2 <= (size_t)capacity, "one_shot_allreduce: size ", n, " over capacity");
  TORCH_CHECK(num_ctas >= 1 && num_ctas <= kMaxCtas, "one_shot_allreduce: CTA count");
  const ARNorm nm = make_norm(residual, weight, eps, n, num_ctas);
  const ARPeers peers = make_peers(bufs, wait_ns);
  auto kern = residual ? one_shot_allreduce_kernel<true> : one_shot_allreduce_kernel<false>;
  snb::launch_pdl(kern, num_ctas, kThreadsAR, 0, at::cuda::getCurrentCUDAStream(),
      peers, rank, world, capacity, (const __nv_bfloat16*)in.data_ptr(), (__nv_bfloat16*)out.data_ptr(), n, nm,
      status.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void moe_combine_allreduce(torch::Tensor out, torch::Tensor y, torch::Tensor inv_map, torch::Tensor w,
                           std::vector<int64_t> bufs, int64_t rank, int64_t capacity, int64_t num_ctas,
                           torch::Tensor status, c10::optional<torch::Tensor> residual,
                           c10::optional<torch::Tensor> weight, double eps, int64_t wait_ns) {
  const int world = (int)bufs.size();
  const int T = out.size(0), H = out.size(1), K = w.size(1);
  TORCH_CHECK(world >= 1 && world <= kMaxRanks && H % 8 == 0, "moe_combine_allreduce: shape");
  TORCH_CHECK((size_t)T * H * 2 <= (size_t)capacity, "moe_combine_allreduce: over capacity");
  TORCH_CHECK(num_ctas >= 1 && num_ctas <= kMaxCtas, "moe_combine_allreduce: CTA count");
  if (T == 0) return;
  const ARNorm nm = make_norm(residual, weight, eps, (int64_t)T * H, num_ctas);
  TORCH_CHECK(!residual || nm.H == H, "moe_combine_allreduce: norm size");
  const ARPeers peers = make_peers(bufs, wait_ns);
  auto kern = residual ? moe_combine_allreduce_kernel<true> : moe_combine_allreduce_kernel<false>;
  snb::launch_pdl(kern, num_ctas, kThreadsAR, 0, at::cuda::getCurrentCUDAStream(),
      peers, rank, world, capacity, (const __nv_bfloat16*)y.data_ptr(), y.stride(0), inv_map.data_ptr<int32_t>(),
      w.data_ptr<float>(), K, T, H, (__nv_bfloat16*)out.data_ptr(), nm, status.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void splitk_allreduce(torch::Tensor out, torch::Tensor partial, int64_t splits, c10::optional<torch::Tensor> bias,
                      std::vector<int64_t> bufs, int64_t rank, int64_t capacity, int64_t num_ctas, torch::Tensor status,
                      c10::optional<torch::Tensor> residual, c10::optional<torch::Tensor> weight, double eps,
                      int64_t wait_ns) {
  const int world = (int)bufs.size();
  const int T = out.size(0), F = out.size(1);
  TORCH_CHECK(F % 8 == 0 && out.is_contiguous() && partial.scalar_type() == at::kFloat, "splitk_allreduce: layout");
  TORCH_CHECK(partial.numel() >= (int64_t)splits * T * F, "splitk_allreduce: partial size");
  TORCH_CHECK((size_t)T * F * 2 <= (size_t)capacity, "splitk_allreduce: over capacity");
  TORCH_CHECK(num_ctas >= 1 && num_ctas <= kMaxCtas, "splitk_allreduce: CTA count");
  if (T == 0) return;
  const ARNorm nm = make_norm(residual, weight, eps, (int64_t)T * F, num_ctas);
  TORCH_CHECK(!residual || nm.H == F, "splitk_allreduce: norm size");
  const ARPeers peers = make_peers(bufs, wait_ns);
  auto kern = residual ? splitk_allreduce_kernel<true> : splitk_allreduce_kernel<false>;
  snb::launch_pdl(kern, num_ctas, kThreadsAR, 0, at::cuda::getCurrentCUDAStream(),
      peers, rank, world, capacity, partial.data_ptr<float>(), splits,
      bias ? (const __nv_bfloat16*)bias->data_ptr() : nullptr, T, F, (__nv_bfloat16*)out.data_ptr(), nm,
      status.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
