// Page copies between KV pools: device <-> pinned host (HiCache tier) or device <-> device, for every layer
// buffer in one launch. Pinned host memory is addressed directly through unified virtual addressing, so
// the SMs stream the pages over the host link with 16-byte loads/stores: one launch per batch of pages
// instead of (layers x pages x K/V) copy calls.
//
// Parity: the reference's HiCache host pool moves pages with batched runtime DMA on store/load threads
// (sglang_neuron/mem_cache/host_pool.py:233 TransferEngine).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "../common.cuh"

namespace {

constexpr int kThreadsCopy = 256;

// grid: (pages, buffers). Buffer b of src/dst: base pointers with identical page size in bytes.
__global__ void __launch_bounds__(kThreadsCopy) kv_page_copy_kernel(
    const int64_t* __restrict__ src_bases, const int64_t* __restrict__ dst_bases,
    const int32_t* __restrict__ src_pages, const int32_t* __restrict__ dst_pages, int64_t page_bytes) {
  snb::pdl_wait();
  snb::pdl_trigger();
  const int i = blockIdx.x, b = blockIdx.y;
  const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(src_bases[b]) +
                                                    (int64_t)src_pages[i] * page_bytes);
  uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(dst_bases[b]) + (int64_t)dst_pages[i] * page_bytes);
  const int64_t n = page_bytes / 16;
  for (int64_t v = threadIdx.x; v < n; v += blockDim.x) dst[v] = src[v];
}

// Page-slice copy between pools of different layouts (disaggregated prefill/decode over NVLink): pair i copies
// `nbytes` from byte `src_off` of src page src_pages[i] (pages of src_page_bytes) to byte `dst_off` of dst page
// dst_pages[i] (pages of dst_page_bytes), for every buffer b. The destination is another GPU's pool mapped
// over CUDA IPC: plain 16-byte stores cross NVLink, so the KV of a head shard lands straight in its final
// pages with no staging copy on either side.
__global__ void __launch_bounds__(kThreadsCopy) kv_page_slice_copy_kernel(
    const int64_t* __restrict__ src_bases, const int64_t* __restrict__ dst_bases,
    const int32_t* __restrict__ src_pages, const int32_t* __restrict__ dst_pages, int64_t src_page_bytes,
    int64_t dst_page_bytes, int64_t src_off, int64_t dst_off, int64_t nbytes) {
  snb::pdl_wait();
  snb::pdl_trigger();
  const int i = blockIdx.x, b = blockIdx.y;
  const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(src_bases[b]) +
                                                    (int64_t)src_pages[i] * src_page_bytes + src_off);
  uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(dst_bases[b]) +
                                        (int64_t)dst_pages[i] * dst_page_bytes + dst_off);
  const int64_t n = nbytes / 16;
  for (int64_t v = threadIdx.x; v < n; v += blockDim.x) dst[v] = src[v];
}

}  // namespace

void kv_page_slice_copy(torch::Tensor src_bases, torch::Tensor dst_bases, torch::Tensor src_pages,
                        torch::Tensor dst_pages, int64_t src_page_bytes, int64_t dst_page_bytes, int64_t src_off,
                        int64_t dst_off, int64_t nbytes) {
  TORCH_CHECK(nbytes % 16 == 0 && src_off % 16 == 0 && dst_off % 16 == 0 && src_page_bytes % 16 == 0 &&
                  dst_page_bytes % 16 == 0, "kv_page_slice_copy: 16-byte aligned slices");
  TORCH_CHECK(src_off + nbytes <= src_page_bytes && dst_off + nbytes <= dst_page_bytes, "kv_page_slice_copy: bounds");
  TORCH_CHECK(src_bases.numel() == dst_bases.numel() && src_pages.numel() == dst_pages.numel(), "kv_page_slice_copy");
  const int n = src_pages.numel(), nb = src_bases.numel();
  if (n == 0 || nb == 0 || nbytes == 0) return;
  C10_CUDA_CHECK(snb::launch_pdl(kv_page_slice_copy_kernel, dim3(n, nb), kThreadsCopy, 0,
                                 at::cuda::getCurrentCUDAStream(), (const int64_t*)src_bases.data_ptr<int64_t>(),
                                 (const int64_t*)dst_bases.data_ptr<int64_t>(), src_pages.data_ptr<int32_t>(),
                                 dst_pages.data_ptr<int32_t>(), src_page_bytes, dst_page_bytes, src_off, dst_off,
                                 nbytes));
}

// src_bases / dst_bases: int64 device tensors of buffer base addresses (device or pinned host); src_pages /
// dst_pages: int32 device tensors of page indices. page_bytes must be a multiple of 16.
void kv_page_copy(torch::Tensor src_bases, torch::Tensor dst_bases, torch::Tensor src_pages, torch::Tensor dst_pages,
                  int64_t page_bytes) {
  TORCH_CHECK(page_bytes % 16 == 0, "kv_page_copy: page size must be a multiple of 16 bytes");
  TORCH_CHECK(src_bases.numel() == dst_bases.numel() && src_pages.numel() == dst_pages.numel(), "kv_page_copy");
  const int n = src_pages.numel(), nb = src_bases.numel();
  if (n == 0 || nb == 0) return;
  C10_CUDA_CHECK(snb::launch_pdl(kv_page_copy_kernel, dim3(n, nb), kThreadsCopy, 0, at::cuda::getCurrentCUDAStream(),
                                 (const int64_t*)src_bases.data_ptr<int64_t>(),
                                 (const int64_t*)dst_bases.data_ptr<int64_t>(), src_pages.data_ptr<int32_t>(),
                                 dst_pages.data_ptr<int32_t>(), page_bytes));
}
