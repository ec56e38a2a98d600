// One-shot all-reduce over NVLink peer memory (CUDA IPC mappings), for the tensor-parallel collectives of
// the decode path, plus the IPC plumbing that maps every rank's buffer into every other rank.
//
// Each rank owns one device buffer laid out as [2 halves][world slots][capacity bytes] followed by per-CTA
// flags [world][max CTAs] and per-CTA epochs. A call with epoch e uses half (e & 1):
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

namespace {

constexpr int kMaxRanks = 8;
constexpr int kMaxCtas = 64;
constexpr int kThreadsAR = 512;

struct ARPeers {
  uint8_t* buf[kMaxRanks];  // mapped base of every rank's buffer (mine included)
};

SNB_DEVICE void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
SNB_DEVICE uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kThreadsAR) one_shot_allreduce_kernel(
    ARPeers peers, int rank, int world, size_t capacity, const __nv_bfloat16* __restrict__ in,
    __nv_bfloat16* __restrict__ out, int64_t n, int* status) {
  const int c = blockIdx.x;
  uint8_t* mine = peers.buf[rank];
  const size_t data_bytes = 2 * (size_t)world * capacity;
  uint32_t* flags_mine = reinterpret_cast<uint32_t*>(mine + data_bytes);   // [world][kMaxCtas]
  uint32_t* epochs = flags_mine + kMaxRanks * kMaxCtas;                     // [kMaxCtas], local only
  __shared__ uint32_t e_s;
  if (threadIdx.x == 0) e_s = epochs[c] + 1;
  __syncthreads();
  const uint32_t e = e_s;
  const int half = e & 1;
  // chunk of this CTA, in 16-byte vectors
  const int64_t nvec = n / 8;
  const int64_t per = (nvec + gridDim.x - 1) / gridDim.x;
  const int64_t v0 = c * per, v1 = min(nvec, v0 + per);
  // 1. push my chunk into every peer's slot `rank`
  for (int p = 0; p < world; ++p) {
    uint4* dst = reinterpret_cast<uint4*>(peers.buf[p] + ((size_t)half * world + rank) * capacity);
    const uint4* src = reinterpret_cast<const uint4*>(in);
    for (int64_t v = v0 + threadIdx.x; v < v1; v += blockDim.x) dst[v] = src[v];
  }
  __syncthreads();
  // 2. publish (release orders the stores above for the peers' acquire loads)
  if (threadIdx.x < world) {
    const int p = threadIdx.x;
    uint32_t* fp = reinterpret_cast<uint32_t*>(peers.buf[p] + data_bytes);
    __threadfence_system();
    st_release_sys(fp + rank * kMaxCtas + c, e);
  }
  // 3. wait for every rank's chunk (bounded)
  __shared__ int ok_s;
  if (threadIdx.x == 0) ok_s = 1;
  __syncthreads();
  if (threadIdx.x < world) {
    const uint32_t* fp = flags_mine + threadIdx.x * kMaxCtas + c;
    const uint64_t t0 = snb::globaltimer_ns();
    while (ld_acquire_sys(fp) < e) {
      if (snb::globaltimer_ns() - t0 > SNB_WAIT_NS) {
        snb::record_status(status, SNB_ERR_TIMEOUT_PEER);
        ok_s = 0;
        break;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) epochs[c] = e;
  if (!ok_s) return;
  // 4. reduce over the world slots of my buffer
  for (int64_t v = v0 + threadIdx.x; v < v1; v += blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int q = 0; q < world; ++q) {
      const uint4 u = reinterpret_cast<const uint4*>(mine + ((size_t)half * world + q) * capacity)[v];
      float f[8];
      snb::unpack_bf16x8(u, f);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += f[i];
    }
    reinterpret_cast<uint4*>(out)[v] = snb::pack_bf16x8(acc);
  }
}

}  // namespace

// --- IPC plumbing -----------------------------------------------------------------------------------
// Allocate the communicator buffer (cudaMalloc: IPC needs whole allocations, not caching-allocator blocks)
// and return (device pointer, IPC handle bytes).
std::tuple<int64_t, py::bytes> symm_alloc(int64_t capacity, int64_t world) {
  TORCH_CHECK(world >= 1 && world <= kMaxRanks, "symm_alloc: world size");
  const size_t bytes = 2 * (size_t)world * capacity + (kMaxRanks * kMaxCtas + kMaxCtas) * sizeof(uint32_t);
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

void one_shot_allreduce(torch::Tensor out, torch::Tensor in, std::vector<int64_t> bufs, int64_t rank,
                        int64_t capacity, int64_t num_ctas, torch::Tensor status) {
  const int world = (int)bufs.size();
  TORCH_CHECK(world >= 1 && world <= kMaxRanks, "one_shot_allreduce: world size");
  TORCH_CHECK(in.scalar_type() == at::kBFloat16 && in.is_contiguous() && out.is_contiguous(), "one_shot_allreduce: bf16");
  const int64_t n = in.numel();
  TORCH_CHECK(n % 8 == 0 && (size_t)n * 2 <= (size_t)capacity, "one_shot_allreduce: size ", n, " over capacity");
  TORCH_CHECK(num_ctas >= 1 && num_ctas <= kMaxCtas, "one_shot_allreduce: CTA count");
  ARPeers peers;
  for (int i = 0; i < kMaxRanks; ++i) peers.buf[i] = i < world ? reinterpret_cast<uint8_t*>(bufs[i]) : nullptr;
  one_shot_allreduce_kernel<<<num_ctas, kThreadsAR, 0, at::cuda::getCurrentCUDAStream()>>>(
      peers, rank, world, capacity, (const __nv_bfloat16*)in.data_ptr(), (__nv_bfloat16*)out.data_ptr(), n,
      status.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
