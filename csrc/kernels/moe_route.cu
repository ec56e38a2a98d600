// MoE routing: top-k gating, counting-sort permutation into padded expert segments, MXFP8 gather-quantise
// of the permuted rows, and the weighted combine.
//
// Parity: the reference routes in its fused MoE kernels (`moe_block_tkg`, sglang_neuron/ops/moe/moe_block_tkg.py:19-128,
// router softmax + top-k) and builds a token->block mapping for prefill (`build_blockwise_mapping`,
// sglang_neuron/ops/moe/moe_blockwise.py:24-130). Here the mapping is a device counting sort whose output
// sizes have a static upper bound (T*K + E*(BN-1) rows), so the whole MoE path is CUDA-graph capturable.
//
// Activation quantisation follows the OCP MX format: blocks of 32 values share an e8m0 power-of-two scale
// 2^X with X = ceil(log2(amax / 448)), values are e4m3 (max 448). Scales of a permuted row r are written in
// the tensor-memory scale-factor atom order consumed by tcgen05.cp (32x128b.warpx4): within a chunk of one
// BN-row tile and one 128-wide K block, the byte for (row i, 32-block kk) sits at (i%32)*16 + (i/32)*4 + kk.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "../common.cuh"

namespace {

// One warp per token. mode 0: softmax over the k selected logits (renormalised top-k);
// mode 1: softmax over all E logits, then the top-k probabilities (times `scale`).
template <typename T>
__global__ void topk_route_kernel(const T* __restrict__ logits, int T_tok, int E, int K, int mode, float scale,
                                  float* __restrict__ w_out, int32_t* __restrict__ id_out) {
  snb::pdl_wait();
  snb::pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= T_tok) return;
  const T* lr = logits + (size_t)warp * E;
  float v[8];
  const int per = (E + 31) / 32;
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int e = lane + 32 * i;
    v[i] = (i < per && e < E) ? (float)lr[e] : -INFINITY;
    mx = fmaxf(mx, v[i]);
  }
  mx = snb::warp_max(mx);
  float denom_all = 0.f;
  if (mode == 1) {
#pragma unroll
    for (int i = 0; i < 8; ++i) denom_all += (v[i] == -INFINITY) ? 0.f : __expf(v[i] - mx);
    denom_all = snb::warp_sum(denom_all);
  }
  float sel_v[16];
  int sel_i[16];
  for (int j = 0; j < K; ++j) {
    // warp argmax (ties -> smallest expert id)
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = lane + 32 * i;
      if (v[i] > bv || (v[i] == bv && e < bi)) {
        bv = v[i];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    sel_v[j] = bv;
    sel_i[j] = bi;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (lane + 32 * i == bi) v[i] = -INFINITY;
  }
  if (lane == 0) {
    if (mode == 0) {
      float s = 0.f;
      for (int j = 0; j < K; ++j) s += __expf(sel_v[j] - sel_v[0]);
      for (int j = 0; j < K; ++j) {
        w_out[(size_t)warp * K + j] = __expf(sel_v[j] - sel_v[0]) / s * scale;
        id_out[(size_t)warp * K + j] = sel_i[j];
      }
    } else {
      for (int j = 0; j < K; ++j) {
        w_out[(size_t)warp * K + j] = __expf(sel_v[j] - mx) / denom_all * scale;
        id_out[(size_t)warp * K + j] = sel_i[j];
      }
    }
  }
}

// Single-CTA counting sort of (token, slot) entries by expert into BN-padded segments.
// Entries whose expert is outside [e_lo, e_lo + E_local) are dropped (expert parallelism: another rank owns them).
__global__ void __launch_bounds__(1024) moe_align_kernel(const int32_t* __restrict__ ids, int N_entries, int K,
                                                         int e_lo, int E_local, int BN,
                                                         int32_t* __restrict__ seg_offsets,   // [E_local+1]
                                                         int32_t* __restrict__ tile_offsets,  // [E_local+1]
                                                         int32_t* __restrict__ sorted_src,    // [R_max]
                                                         int32_t* __restrict__ inv_map,       // [N_entries]
                                                         int R_max) {
  snb::pdl_wait();
  snb::pdl_trigger();
  extern __shared__ int32_t sm[];
  int32_t* cnt = sm;                 // E_local
  int32_t* off = sm + E_local;       // E_local + 1
  int32_t* cur = off + E_local + 1;  // E_local
  for (int e = threadIdx.x; e < E_local; e += blockDim.x) {
    cnt[e] = 0;
    cur[e] = 0;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < N_entries; i += blockDim.x) {
    const int e = ids[i] - e_lo;
    if (e >= 0 && e < E_local) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  // Exclusive scan of the BN-padded segment sizes by warp 0 (E_local <= 256: 8 experts per lane).
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const int per = (E_local + 31) / 32;
    int local_rows = 0, local_tiles = 0;
    for (int j = 0; j < per; ++j) {
      const int e = lane * per + j;
      if (e < E_local) {
        const int padded = ((cnt[e] + BN - 1) / BN) * BN;
        local_rows += padded;
        local_tiles += padded / BN;
      }
    }
    int inc_rows = local_rows, inc_tiles = local_tiles;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int r = __shfl_up_sync(0xffffffffu, inc_rows, o);
      const int t = __shfl_up_sync(0xffffffffu, inc_tiles, o);
      if (lane >= o) {
        inc_rows += r;
        inc_tiles += t;
      }
    }
    int acc = inc_rows - local_rows, tiles = inc_tiles - local_tiles;
    for (int j = 0; j < per; ++j) {
      const int e = lane * per + j;
      if (e < E_local) {
        off[e] = acc;
        seg_offsets[e] = acc;
        tile_offsets[e] = tiles;
        const int padded = ((cnt[e] + BN - 1) / BN) * BN;
        acc += padded;
        tiles += padded / BN;
      }
    }
    if (lane == 31) {
      off[E_local] = inc_rows;
      seg_offsets[E_local] = inc_rows;
      tile_offsets[E_local] = inc_tiles;
    }
  }
  __syncthreads();
  const int total = off[E_local];
  for (int r = threadIdx.x; r < R_max; r += blockDim.x) sorted_src[r] = -1;
  __syncthreads();
  for (int i = threadIdx.x; i < N_entries; i += blockDim.x) {
    const int e = ids[i] - e_lo;
    if (e >= 0 && e < E_local) {
      const int p = off[e] + atomicAdd(&cur[e], 1);
      sorted_src[p] = i / K;
      inv_map[i] = p;
    } else {
      inv_map[i] = -1;
    }
  }
  (void)total;
}

// One thread per (permuted row, 32-element block): consecutive threads take consecutive blocks of a row, so a
// row's loads and stores coalesce and every block of a decode batch is in flight at once.
// x: [T, H] bf16 (row stride xs). Output q: [R, Kp] e4m3 (Kp = padded row pitch), scales in atom order.
// `used` (optional, device): the number of rows the expert segments actually occupy (seg_offsets[E_local]);
// rows past it belong to no tile the grouped GEMM runs, so they are skipped. The grid stays sized for the
// static capacity R (graph capture), but the work follows the routed row count, which shrinks with EP.
__global__ void gather_quant_mxfp8_kernel(const __nv_bfloat16* __restrict__ x, int xs, const int32_t* __restrict__ src,
                                          int R, int H, int Kp, int BN, uint8_t* __restrict__ q,
                                          uint8_t* __restrict__ sf, const int32_t* __restrict__ used,
                                          const int32_t* __restrict__ skip) {
  snb::pdl_wait();
  snb::pdl_trigger();
  const int KB = (Kp + 127) / 128;           // 128-wide K blocks
  const int nblk = KB * 4;                    // 32-wide scale blocks incl. padding
  const int64_t item = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int r = (int)(item / nblk), blk = (int)(item % nblk);
  if (r >= R || (used != nullptr && r >= *used)) return;
  if (skip != nullptr && skip[r] < 0) return;  // a padding row of the permutation (see below)
  const int s = src != nullptr ? src[r] : r;
  // Padding rows of a segment (src < 0) are left as they are: row n of a tile's output depends only on
  // activation row n and its scales, and the combine never reads a padding row, so whatever they hold only
  // ever reaches outputs nobody reads. (At decode most rows are padding: 16-row tiles for 1-3 tokens.)
  if (s < 0) return;
  const int chunk_bytes = min(BN, 32) * 16;
  const int tile = r / BN, i = r % BN;
  uint8_t* qrow = q + (size_t)r * Kp;
  const int k0 = blk * 32;
  uint8_t e8 = 127;
  if (k0 < H) {
    const __nv_bfloat16* xr = x + (size_t)s * xs + k0;
    uint4 raw[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) raw[c] = reinterpret_cast<const uint4*>(xr)[c];
    float f[32];
    float amax = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float t8[8];
      snb::unpack_bf16x8(raw[c], t8);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        f[c * 8 + j] = t8[j];
        amax = fmaxf(amax, fabsf(t8[j]));
      }
    }
    int X = 0;
    if (amax > 0.f) {
      X = (int)ceilf(log2f(amax / 448.f));
      X = max(-127, min(127, X));
    }
    e8 = (uint8_t)(X + 127);
    const float inv = exp2f((float)-X);
    uint8_t ob[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) ob[j] = snb::f_to_fp8e4m3(f[j] * inv);
    reinterpret_cast<uint4*>(qrow + k0)[0] = *reinterpret_cast<uint4*>(ob);
    reinterpret_cast<uint4*>(qrow + k0)[1] = *reinterpret_cast<uint4*>(ob + 16);
  } else if (k0 < Kp) {
    reinterpret_cast<uint4*>(qrow + k0)[0] = make_uint4(0, 0, 0, 0);
    reinterpret_cast<uint4*>(qrow + k0)[1] = make_uint4(0, 0, 0, 0);
  }
  const int kb = blk >> 2, kk = blk & 3;
  sf[((size_t)tile * KB + kb) * chunk_bytes + (i % 32) * 16 + (i / 32) * 4 + kk] = e8;
}

// out[t] = sum_j w[t, j] * y[inv_map[t*K + j]]  (+ out[t] if accumulate). One CTA per token, one 8-element chunk
// per thread: the token's K row ids and weights are staged in shared memory first, then every row's chunk is
// requested before any is summed (independent loads, one round trip instead of 2K).
constexpr int kMaxCombineK = 16;

__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ y, int ys, const int32_t* __restrict__ inv_map,
                                   const float* __restrict__ w, int K, int H, __nv_bfloat16* __restrict__ out,
                                   int os, bool accumulate) {
  snb::pdl_wait();
  snb::pdl_trigger();
  __shared__ int rows[kMaxCombineK];
  __shared__ float wts[kMaxCombineK];
  const int t = blockIdx.x;
  if (threadIdx.x < K) {
    rows[threadIdx.x] = inv_map[t * K + threadIdx.x];
    wts[threadIdx.x] = w[t * K + threadIdx.x];
  }
  __syncthreads();
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) {
    float acc[8];
    if (accumulate) {
      snb::unpack_bf16x8(reinterpret_cast<const uint4*>(out + (size_t)t * os)[c], acc);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    }
    for (int j0 = 0; j0 < K; j0 += 4) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j = j0 + u;
        const int r = j < K ? rows[j] : -1;
        v[u] = r >= 0 ? reinterpret_cast<const uint4*>(y + (size_t)r * ys)[c] : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j = j0 + u;
        if (j >= K || rows[j] < 0) continue;
        float f[8];
        snb::unpack_bf16x8(v[u], f);
        const float wj = wts[j];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] += wj * f[i];
      }
    }
    reinterpret_cast<uint4*>(out + (size_t)t * os)[c] = snb::pack_bf16x8(acc);
  }
}

}  // namespace

void topk_route(torch::Tensor weights, torch::Tensor ids, torch::Tensor logits, int64_t k, int64_t mode,
                double scale) {
  const int T = logits.size(0), E = logits.size(1);
  if (T == 0) return;
  TORCH_CHECK(E <= 256 && k <= 16 && k <= E, "topk_route: E<=256, k<=16");
  TORCH_CHECK(logits.is_contiguous(), "topk_route: contiguous logits");
  auto st = at::cuda::getCurrentCUDAStream();
  const int threads = 256, blocks = (T * 32 + threads - 1) / threads;
  if (logits.scalar_type() == at::kFloat) {
    snb::launch_pdl(topk_route_kernel<float>, blocks, threads, 0, st, logits.data_ptr<float>(), T, E, k, mode, scale,
                                                         weights.data_ptr<float>(), ids.data_ptr<int32_t>());
  } else {
    snb::launch_pdl(topk_route_kernel<__nv_bfloat16>, blocks, threads, 0, st, (const __nv_bfloat16*)logits.data_ptr(), T, E, k,
                                                                 mode, scale, weights.data_ptr<float>(),
                                                                 ids.data_ptr<int32_t>());
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void moe_align(torch::Tensor ids, int64_t e_lo, int64_t e_local, int64_t bn, torch::Tensor seg_offsets,
               torch::Tensor tile_offsets, torch::Tensor sorted_src, torch::Tensor inv_map) {
  const int N = ids.numel();
  const int K = ids.dim() == 2 ? ids.size(1) : 1;
  auto st = at::cuda::getCurrentCUDAStream();
  const int R_max = sorted_src.numel();
  TORCH_CHECK(R_max >= N + e_local * (bn - 1), "moe_align: sorted_src capacity too small");
  const size_t smem = (3 * e_local + 1) * sizeof(int32_t);
  snb::launch_pdl(moe_align_kernel, 1, 1024, smem, st, ids.data_ptr<int32_t>(), N, K, e_lo, e_local, bn,
                                          seg_offsets.data_ptr<int32_t>(), tile_offsets.data_ptr<int32_t>(),
                                          sorted_src.data_ptr<int32_t>(), inv_map.data_ptr<int32_t>(), R_max);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gather_quant_mxfp8(torch::Tensor q, torch::Tensor sf, torch::Tensor x, c10::optional<torch::Tensor> src,
                        int64_t bn, c10::optional<torch::Tensor> used, c10::optional<torch::Tensor> skip) {
  const int R = q.size(0), Kp = q.size(1), H = x.size(1);
  if (R == 0) return;
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.stride(1) == 1 && H % 32 == 0, "gather_quant: x");
  TORCH_CHECK(Kp >= H && Kp % 16 == 0, "gather_quant: pitch");
  TORCH_CHECK(R % bn == 0, "gather_quant: rows must be a multiple of bn");
  const int KB = (Kp + 127) / 128;
  TORCH_CHECK(sf.numel() >= (int64_t)(R / bn) * KB * std::min<int64_t>(bn, 32) * 16, "gather_quant: sf capacity");
  auto st = at::cuda::getCurrentCUDAStream();
  const int64_t items = (int64_t)R * KB * 4;
  const int threads = 128, blocks = (int)((items + threads - 1) / threads);
  snb::launch_pdl(gather_quant_mxfp8_kernel, blocks, threads, 0, st, (const __nv_bfloat16*)x.data_ptr(), x.stride(0),
                                                       src ? src->data_ptr<int32_t>() : nullptr, R, H, Kp, bn,
                                                       (uint8_t*)q.data_ptr(), (uint8_t*)sf.data_ptr(),
                                                       used ? used->data_ptr<int32_t>() : nullptr,
                                                       skip ? skip->data_ptr<int32_t>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void moe_combine(torch::Tensor out, torch::Tensor y, torch::Tensor inv_map, torch::Tensor w, bool accumulate) {
  const int T = out.size(0), H = out.size(1);
  if (T == 0) return;
  const int K = w.size(1);
  TORCH_CHECK(H % 8 == 0, "moe_combine: H");
  TORCH_CHECK(K <= kMaxCombineK, "moe_combine: at most 16 experts per token");
  auto st = at::cuda::getCurrentCUDAStream();
  const int threads = std::min(1024, (H / 8 + 31) / 32 * 32);
  snb::launch_pdl(moe_combine_kernel, T, threads, 0, st, (const __nv_bfloat16*)y.data_ptr(), y.stride(0), inv_map.data_ptr<int32_t>(),
                                        w.data_ptr<float>(), K, H, (__nv_bfloat16*)out.data_ptr(), out.stride(0),
                                        accumulate);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
