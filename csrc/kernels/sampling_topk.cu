// Top-K candidate pool of each logits row (K <= 256) for filtered (top-k / top-p) sampling, by radix select.
//
// One CTA of 1024 threads per row. Logits map to order-preserving 32-bit keys (larger float -> larger key;
// NaN maps below every number). Three histogram passes over 11, 11 and 10 key bits find the exact key of the
// K-th largest element; two passes in index order (each warp owns a contiguous segment and walks it 32
// elements at a time, ballots giving in-order positions) collect every element above that key and the
// lowest-index elements equal to it; a bitonic sort of the pool then orders it by (value descending, index
// ascending), the same order as a stable descending sort. The row is read five times (from L2 after the
// first pass); nothing is written but the pool.
//
// Parity: the reference's per-shard top-k candidate selection for filtered sampling
// (sglang_neuron/sampling_topk.py:35, sampling.py:337 sample_filtered_sharded_logits).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "../common.cuh"

namespace {

constexpr int kThreadsTK = 1024;
constexpr int kWarpsTK = kThreadsTK / 32;
constexpr int kPool = 256;

template <typename T>
SNB_DEVICE uint32_t okey(T x) {
  const float f = (float)x;
  if (f != f) return 0u;  // NaN below everything
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

SNB_DEVICE float key_to_float(uint32_t k) {
  const uint32_t b = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(b);
}

template <typename T>
__global__ void __launch_bounds__(kThreadsTK) topk_pool_kernel(const T* __restrict__ logits, int64_t ld, int V, int K,
                                                               int64_t vocab_offset, float* __restrict__ vals_out,
                                                               int64_t* __restrict__ ids_out) {
  snb::pdl_wait();
  snb::pdl_trigger();
  __shared__ uint32_t hist[2048];
  __shared__ uint32_t sel_s, krem_s;
  __shared__ int cnt_gt[kWarpsTK], cnt_eq[kWarpsTK];
  __shared__ unsigned long long pool[kPool];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const T* row = logits + (size_t)blockIdx.x * ld;
  uint32_t prefix = 0, pmask = 0;
  uint32_t krem = (uint32_t)K;
  const int shifts[3] = {21, 10, 0};
  const int nbits[3] = {11, 11, 10};
#pragma unroll 1
  for (int pass = 0; pass < 3; ++pass) {
    const int sh = shifts[pass], nb = 1 << nbits[pass];
    for (int i = tid; i < nb; i += kThreadsTK) hist[i] = 0;
    __syncthreads();
    // the leading bins of a logits row hold most of its values: lanes of a warp that hit the same bin add
    // together (one shared atomic per distinct bin per warp step)
    for (int b = warp * 32; b < V; b += kThreadsTK) {
      const int i = b + lane;
      const uint32_t k = i < V ? okey(row[i]) : 0u;
      const bool hit = i < V && (k & pmask) == prefix;
      const uint32_t hits = __ballot_sync(0xffffffffu, hit);
      if (hit) {
        const uint32_t bin = (k >> sh) & (nb - 1);
        const uint32_t same = __match_any_sync(hits, bin);
        if ((same & ((1u << lane) - 1u)) == 0u) atomicAdd(&hist[bin], (uint32_t)__popc(same));
      }
    }
    __syncthreads();
    if (warp == 0) {
      // lane l owns bins [l*per, (l+1)*per); suffix counts from the top bin find the digit of the K-th largest
      const int per = nb / 32;
      uint32_t s = 0;
      for (int b = 0; b < per; ++b) s += hist[lane * per + b];
      uint32_t suf = s;  // inclusive suffix sum over lanes >= this one
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_down_sync(0xffffffffu, suf, o);
        if (lane + o < 32) suf += v;
      }
      const uint32_t above = suf - s;  // elements in higher lanes' bins
      const bool mine = above < krem && suf >= krem;
      const uint32_t who = __ballot_sync(0xffffffffu, mine);
      if (mine) {
        uint32_t c = above;
        int d = lane * per + per - 1;
        for (; d > lane * per; --d) {
          if (c + hist[d] >= krem) break;
          c += hist[d];
        }
        sel_s = (uint32_t)d;
        krem_s = krem - c;
      }
      if (who == 0 && lane == 0) {  // fewer than K candidates match (K > V): take the whole row
        sel_s = 0xffffffffu;
      }
    }
    __syncthreads();
    if (sel_s == 0xffffffffu) break;
    prefix |= sel_s << sh;
    pmask |= (uint32_t)(nb - 1) << sh;
    krem = krem_s;
    __syncthreads();
  }
  const bool all = sel_s == 0xffffffffu;
  const uint32_t kth = prefix;
  // ordered collection: warp w owns indices [w*seg, (w+1)*seg)
  const int seg = (V + kWarpsTK - 1) / kWarpsTK;
  const int i0 = warp * seg, i1 = min(V, i0 + seg);
  int gt = 0, eq = 0;
  for (int b = i0; b < i1; b += 32) {
    const int i = b + lane;
    const uint32_t k = i < i1 ? okey(row[i]) : 0u;
    const bool valid = i < i1;
    gt += __popc(__ballot_sync(0xffffffffu, valid && (all || k > kth)));
    eq += __popc(__ballot_sync(0xffffffffu, valid && !all && k == kth));
  }
  if (lane == 0) {
    cnt_gt[warp] = gt;
    cnt_eq[warp] = eq;
  }
  for (int i = tid; i < kPool; i += kThreadsTK) pool[i] = 0ull;
  __syncthreads();
  int gt_off = 0, eq_off = 0, G = 0;
  for (int w = 0; w < kWarpsTK; ++w) {
    if (w < warp) {
      gt_off += cnt_gt[w];
      eq_off += cnt_eq[w];
    }
    G += cnt_gt[w];
  }
  const int take = all ? 0 : (int)krem;
  const int n = all ? min(G, K) : K;
  for (int b = i0; b < i1; b += 32) {
    const int i = b + lane;
    const bool valid = i < i1;
    const uint32_t k = valid ? okey(row[i]) : 0u;
    const bool is_gt = valid && (all || k > kth), is_eq = valid && !all && k == kth;
    const uint32_t bg = __ballot_sync(0xffffffffu, is_gt), be = __ballot_sync(0xffffffffu, is_eq);
    const uint32_t below = (1u << lane) - 1u;
    if (is_gt) {
      const int p = gt_off + __popc(bg & below);
      if (p < kPool) pool[p] = ((unsigned long long)k << 32) | (0xffffffffu - (uint32_t)i);
    }
    if (is_eq) {
      const int p = eq_off + __popc(be & below);
      if (p < take) pool[G + p] = ((unsigned long long)k << 32) | (0xffffffffu - (uint32_t)i);
    }
    gt_off += __popc(bg);
    eq_off += __popc(be);
  }
  __syncthreads();
  // bitonic sort of the pool, descending (value desc, then index asc through the complemented index)
  for (int size = 2; size <= kPool; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      if (tid < kPool) {
        const int j = tid ^ stride;
        if (j > tid) {
          const bool desc = (tid & size) == 0;
          const unsigned long long a = pool[tid], b = pool[j];
          if ((a < b) == desc) {
            pool[tid] = b;
            pool[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  if (tid < K) {
    const unsigned long long p = pool[tid];
    const bool ok = tid < n;
    vals_out[(size_t)blockIdx.x * K + tid] = ok ? key_to_float((uint32_t)(p >> 32)) : -INFINITY;
    ids_out[(size_t)blockIdx.x * K + tid] = ok ? (int64_t)(0xffffffffu - (uint32_t)(p & 0xffffffffu)) + vocab_offset
                                               : vocab_offset;
  }
}

}  // namespace

// logits: [B, >= V] (bf16 or fp32, row stride arbitrary); vals [B, K] fp32, ids [B, K] int64 (+ vocab_offset).
void topk_pool(torch::Tensor logits, int64_t V, int64_t K, int64_t vocab_offset, torch::Tensor vals, torch::Tensor ids) {
  const int B = logits.size(0);
  TORCH_CHECK(K >= 1 && K <= kPool, "topk_pool: K must be in [1, 256]");
  TORCH_CHECK(V >= 1 && V <= logits.size(1) && logits.stride(1) == 1, "topk_pool: logits layout");
  TORCH_CHECK(vals.scalar_type() == at::kFloat && ids.scalar_type() == at::kLong && vals.numel() >= (int64_t)B * K &&
                  ids.numel() >= (int64_t)B * K, "topk_pool: outputs");
  if (B == 0) return;
  auto st = at::cuda::getCurrentCUDAStream();
  if (logits.scalar_type() == at::kBFloat16) {
    C10_CUDA_CHECK(snb::launch_pdl(topk_pool_kernel<__nv_bfloat16>, B, kThreadsTK, 0, st,
                                   (const __nv_bfloat16*)logits.data_ptr(), logits.stride(0), (int)V, (int)K,
                                   vocab_offset, vals.data_ptr<float>(), ids.data_ptr<int64_t>()));
  } else {
    TORCH_CHECK(logits.scalar_type() == at::kFloat, "topk_pool: bf16 or fp32 logits");
    C10_CUDA_CHECK(snb::launch_pdl(topk_pool_kernel<float>, B, kThreadsTK, 0, st, logits.data_ptr<float>(),
                                   logits.stride(0), (int)V, (int)K, vocab_offset, vals.data_ptr<float>(),
                                   ids.data_ptr<int64_t>()));
  }
}
