// Decode-sized MoE routing in one launch: router GEMM -> top-k -> counting sort into BN-padded expert
// segments -> MXFP8 gather-quantise of the routed rows.
//
// The separate path takes four launches per MoE layer (router GEMM, top-k, alignment, quantise); at a few
// dozen tokens each of them is a few microseconds of launch and tail latency around well under a microsecond
// of work. Here one grid of co-resident CTAs does all of it, with two grid-wide barriers:
//   phase 1, every CTA: a [T x 16-expert] block of router logits over one K chunk, on tensor cores
//            (mma.sync m16n8k16 bf16 -> fp32; the router weight is read in the GEMM's tiled layout), written
//            as an fp32 partial;
//   phase 2, one warp per token: the K-chunk partials of its logits summed (all loads in flight at once),
//            bias added, rounded to bf16 (the logits the separate router GEMM produces), top-k selected;
//   phase 3, every CTA: the same deterministic, stable counting sort of the (token, slot) entries of the
//            experts owned here (CTA 0 publishes it for the GEMM and the combine), then its share of the routed
//            rows quantised to MXFP8 (e4m3, e8m0 scale per 32, scales in the tcgen05 atom order).
// Every phase spreads over the whole grid: an earlier design that ran the reduction, top-k and sort in the
// last CTA alone measured 110 us against 21 us for the four launches (timestamps per phase: the single-CTA
// part took 92 us). Each CTA triggers the dependent launch only after the first barrier, i.e. once every CTA
// of the grid is resident, so a programmatically launched successor never takes the SMs a late CTA needs.
// Every barrier wait is bounded (SNB_WAIT_NS); a timeout records SNB_ERR_TIMEOUT_PEER and the CTA returns.
//
// Parity: the reference's router + top-k inside its decode MoE kernel (sglang_neuron/ops/moe/moe_block_tkg.py:
// 19-128) and its token -> block mapping (ops/moe/moe_blockwise.py:24-130).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "../common.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kEGroup = 16;        // experts per CTA (two n8 tiles)
constexpr int kMaxLogits = 16384;  // T * E of a decode-sized call (partials [k_chunks, T, E])
constexpr int kMaxK = 16;

struct RouteArgs {
  const __nv_bfloat16* x;  // [T, H] rows of stride xs
  int xs, T, H;
  const __nv_bfloat16* w;  // router weight, tiled: tile (f/128, k/64) is a contiguous [128][64] block
  int nk;                  // 64-wide K tiles per 128-row F tile
  const __nv_bfloat16* bias;  // [E] or null
  int E, K, mode;
  float scale;
  int e_lo, E_local, BN, k_chunks, kc_len;  // kc_len: K elements per chunk (multiple of 64)
  float* partial;          // [k_chunks][T][E]
  float* w_out;            // [T, K]
  int32_t* id_out;         // [T, K]
  int32_t* seg_offsets;    // [E_local + 1]
  int32_t* tile_offsets;   // [E_local + 1]
  int32_t* sorted_src;     // [R_max]
  int32_t* inv_map;        // [T * K]
  int R_max;
  uint8_t* q;              // [R_max, Kp] e4m3
  uint8_t* sf;             // scale atoms
  int Kp;
  uint32_t* sync;          // grid barrier: [0] arrival counter, [1] generation
  int* status;
};

SNB_DEVICE void mma_bf16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

SNB_DEVICE uint32_t ld_u32(const __nv_bfloat16* p) { return *reinterpret_cast<const uint32_t*>(p); }

// element (f, k) of the tiled router weight
SNB_DEVICE const __nv_bfloat16* w_at(const RouteArgs& a, int f, int k) {
  return a.w + ((size_t)((f >> 7) * a.nk + (k >> 6)) * 128 + (f & 127)) * 64 + (k & 63);
}

SNB_DEVICE void phase1(const RouteArgs& a, int eg, int kc) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q2 = (lane & 3) * 2;
  const int k0 = kc * a.kc_len, k1 = min(a.H, k0 + a.kc_len);
  const int mtiles = (a.T + 15) / 16;
  float* part = a.partial + (size_t)kc * a.T * a.E;
  for (int item = warp; item < mtiles * 2; item += kWarps) {
    const int mt = item >> 1, nt = item & 1;
    const int r0 = mt * 16 + g, r1 = r0 + 8;
    const int n = eg * kEGroup + nt * 8 + g;  // this thread's B column (expert)
    const bool v0 = r0 < a.T, v1 = r1 < a.T, vn = n < a.E;
    const __nv_bfloat16* x0 = a.x + (size_t)(v0 ? r0 : 0) * a.xs;
    const __nv_bfloat16* x1 = a.x + (size_t)(v1 ? r1 : 0) * a.xs;
    float c[4] = {0.f, 0.f, 0.f, 0.f};
    // four k16 steps per iteration, every fragment load issued before the MMAs (the loop is latency-bound:
    // L2 round trips, not math)
    for (int kb = k0; kb < k1; kb += 64) {
      uint32_t fa[4][4], fb[4][2];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int k = kb + 16 * u;
        const bool vk = k < k1;
        fa[u][0] = (v0 && vk) ? ld_u32(x0 + k + q2) : 0u;
        fa[u][1] = (v1 && vk) ? ld_u32(x1 + k + q2) : 0u;
        fa[u][2] = (v0 && vk) ? ld_u32(x0 + k + q2 + 8) : 0u;
        fa[u][3] = (v1 && vk) ? ld_u32(x1 + k + q2 + 8) : 0u;
        fb[u][0] = (vn && vk) ? ld_u32(w_at(a, n, k + q2)) : 0u;
        fb[u][1] = (vn && vk) ? ld_u32(w_at(a, n, k + q2 + 8)) : 0u;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) mma_bf16_16816(c, fa[u][0], fa[u][1], fa[u][2], fa[u][3], fb[u][0], fb[u][1]);
    }
    // C fragment: c0,c1 -> (row g, cols 2*(lane%4) +0/1), c2,c3 -> (row g+8, same cols)
    const int col = eg * kEGroup + nt * 8 + q2;
    if (v0 && col < a.E) part[(size_t)r0 * a.E + col] = c[0];
    if (v0 && col + 1 < a.E) part[(size_t)r0 * a.E + col + 1] = c[1];
    if (v1 && col < a.E) part[(size_t)r1 * a.E + col] = c[2];
    if (v1 && col + 1 < a.E) part[(size_t)r1 * a.E + col + 1] = c[3];
  }
}

// Grid-wide barrier over the co-resident CTAs of this launch: arrival counter sync[0], generation sync[1]
// (the last CTA to arrive resets the counter and advances the generation). Bounded: on timeout the CTA records
// SNB_ERR_TIMEOUT_PEER and the caller returns.
SNB_DEVICE bool grid_barrier(uint32_t* sync, int* status) {
  __shared__ int ok_s;
  __syncthreads();
  if (threadIdx.x == 0) {
    ok_s = 1;
    __threadfence();
    const uint32_t gen = *reinterpret_cast<volatile uint32_t*>(&sync[1]);
    if (atomicAdd(&sync[0], 1u) == gridDim.x - 1) {
      sync[0] = 0;
      __threadfence();
      asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(&sync[1]), "r"(gen + 1u) : "memory");
    } else {
      const uint64_t t0 = snb::globaltimer_ns();
      for (;;) {
        uint32_t v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(&sync[1]) : "memory");
        if (v != gen) break;
        if (snb::globaltimer_ns() - t0 > SNB_WAIT_NS) {
          snb::record_status(status, SNB_ERR_TIMEOUT_PEER);
          ok_s = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  return ok_s != 0;
}

// Phase 2, one warp per token: lane l holds experts l, l+32, l+64, l+96 (E <= 128 here) or 8 per lane for
// E <= 256; the K-chunk partials of all of them are loaded together, summed with the bias and rounded to bf16
// (the logits the separate router GEMM produces), then the top-k selection runs on registers.
SNB_DEVICE void phase2_token(const RouteArgs& a, int t, int lane) {
  const int TE = a.T * a.E;
  float v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = 0.f;
  for (int kc = 0; kc < a.k_chunks; ++kc) {
    const float* p = a.partial + (size_t)kc * TE + (size_t)t * a.E;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = lane + 32 * i;
      if (e < a.E) v[i] += __ldcg(p + e);
    }
  }
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int e = lane + 32 * i;
    if (e < a.E) {
      float s = v[i];
      if (a.bias != nullptr) s += __bfloat162float(a.bias[e]);
      v[i] = __bfloat162float(__float2bfloat16(s));
    } else {
      v[i] = -INFINITY;
    }
    mx = fmaxf(mx, v[i]);
  }
  mx = snb::warp_max(mx);
  float denom_all = 0.f;
  if (a.mode == 1) {
#pragma unroll
    for (int i = 0; i < 8; ++i) denom_all += (v[i] == -INFINITY) ? 0.f : __expf(v[i] - mx);
    denom_all = snb::warp_sum(denom_all);
  }
  // top-k by repeated warp argmax (ties -> smallest expert id); lane j keeps the j-th pick
  float my_v = -INFINITY, first = -INFINITY;
  int my_i = 0;
  for (int j = 0; j < a.K; ++j) {
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
    if (j == 0) first = bv;
    if (lane == j) {
      my_v = bv;
      my_i = bi;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (lane + 32 * i == bi) v[i] = -INFINITY;
  }
  float s = 0.f;
  if (a.mode == 0) s = snb::warp_sum(lane < a.K ? __expf(my_v - first) : 0.f);
  if (lane < a.K) {
    const float wj = a.mode == 0 ? __expf(my_v - first) / s * a.scale : __expf(my_v - mx) / denom_all * a.scale;
    a.w_out[(size_t)t * a.K + lane] = wj;
    a.id_out[(size_t)t * a.K + lane] = my_i;
  }
}

// Phase 3, every CTA: the same deterministic counting sort of the (token, slot) entries of the experts owned
// here (stable: entries of one expert in flat-index order), in shared memory. CTA 0 publishes it for the
// grouped GEMM and the combine; every CTA then quantises its share of the rows from its own copy.
SNB_DEVICE void phase3_sort(const RouteArgs& a, int32_t* sid, int32_t* spos, int32_t* cnt, int32_t* off) {
  const int tid = threadIdx.x;
  const int N = a.T * a.K, El = a.E_local;
  for (int i = tid; i < N; i += kThreads) sid[i] = __ldcg(a.id_out + i) - a.e_lo;
  for (int e = tid; e < El; e += kThreads) cnt[e] = 0;
  __syncthreads();
  for (int i = tid; i < N; i += kThreads) {
    const int e = sid[i];
    if (e >= 0 && e < El) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (tid < 32) {  // exclusive scan of the BN-padded segment sizes (warp 0)
    const int per = (El + 31) / 32;
    int rows = 0;
    for (int j = 0; j < per; ++j) {
      const int e = tid * per + j;
      if (e < El) rows += (cnt[e] + a.BN - 1) / a.BN * a.BN;
    }
    int inc = rows;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int r = __shfl_up_sync(0xffffffffu, inc, o);
      if (tid >= o) inc += r;
    }
    int acc = inc - rows;
    for (int j = 0; j < per; ++j) {
      const int e = tid * per + j;
      if (e < El) {
        off[e] = acc;
        acc += (cnt[e] + a.BN - 1) / a.BN * a.BN;
      }
    }
    if (tid == 31) off[El] = inc;
  }
  __syncthreads();
  // stable position: the entry's segment start + earlier entries (flat index) of the same expert
  for (int i = tid; i < N; i += kThreads) {
    const int e = sid[i];
    int p = -1;
    if (e >= 0 && e < El) {
      int r = 0;
      for (int i2 = 0; i2 < i; ++i2) r += sid[i2] == e;
      p = off[e] + r;
    }
    spos[i] = p;
  }
  __syncthreads();
}

// MXFP8 quantise of permuted row r (one warp; each lane whole 32-element blocks), as gather_quant_mxfp8.
SNB_DEVICE void quant_row(const RouteArgs& a, int r, int s, int lane) {
  const int KB = (a.Kp + 127) / 128;
  const int nblk = KB * 4;
  const int chunk_bytes = min(a.BN, 32) * 16;
  const int tile = r / a.BN, i = r % a.BN;
  uint8_t* qrow = a.q + (size_t)r * a.Kp;
  for (int blk = lane; blk < nblk; blk += 32) {
    const int k0 = blk * 32;
    uint8_t e8 = 127;
    if (s >= 0 && k0 < a.H) {
      float f[32];
      const __nv_bfloat16* xr = a.x + (size_t)s * a.xs + k0;
      float amax = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float t8[8];
        snb::unpack_bf16x8(reinterpret_cast<const uint4*>(xr)[c], t8);
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
    } else if (k0 < a.Kp) {
      reinterpret_cast<uint4*>(qrow + k0)[0] = make_uint4(0, 0, 0, 0);
      reinterpret_cast<uint4*>(qrow + k0)[1] = make_uint4(0, 0, 0, 0);
    }
    const int kb = blk >> 2, kk = blk & 3;
    a.sf[((size_t)tile * KB + kb) * chunk_bytes + (i % 32) * 16 + (i / 32) * 4 + kk] = e8;
  }
}

__global__ void __launch_bounds__(kThreads) moe_route_fused_kernel(const RouteArgs a) {
  extern __shared__ __align__(16) int32_t smem_i[];
  const int eg_count = (a.E + kEGroup - 1) / kEGroup;
  const int eg = blockIdx.x % eg_count, kc = blockIdx.x / eg_count;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  snb::pdl_wait();  // x is the previous kernel's output
  phase1(a, eg, kc);
  if (!grid_barrier(a.sync, a.status)) return;
  // every CTA is resident (it passed the barrier) before any of them lets the next kernel launch
  snb::pdl_trigger();
  for (int t = blockIdx.x * kWarps + warp; t < a.T; t += gridDim.x * kWarps) phase2_token(a, t, lane);
  if (!grid_barrier(a.sync, a.status)) return;
  const int N = a.T * a.K, El = a.E_local;
  int32_t* sid = smem_i;
  int32_t* spos = sid + N;
  int32_t* cnt = spos + N;
  int32_t* off = cnt + El;
  int32_t* src = off + El + 1;  // sorted_src of the used rows
  phase3_sort(a, sid, spos, cnt, off);
  const int used = off[El];
  for (int r = threadIdx.x; r < used; r += kThreads) src[r] = -1;
  __syncthreads();
  for (int i = threadIdx.x; i < N; i += kThreads)
    if (spos[i] >= 0) src[spos[i]] = i / a.K;
  __syncthreads();
  if (blockIdx.x == 0) {
    for (int e = threadIdx.x; e <= El; e += kThreads) {
      a.seg_offsets[e] = off[e];
      a.tile_offsets[e] = off[e] / a.BN;
    }
    for (int r = threadIdx.x; r < used; r += kThreads) a.sorted_src[r] = src[r];
    for (int i = threadIdx.x; i < N; i += kThreads) a.inv_map[i] = spos[i];
  }
  // padding rows (src < 0) are skipped: the grouped GEMM's output rows for them are never read
  for (int r = blockIdx.x * kWarps + warp; r < used; r += gridDim.x * kWarps)
    if (src[r] >= 0) quant_row(a, r, src[r], lane);
}

}  // namespace

// x: [T, H] bf16; w_tiled: the router weight in the GEMM's tiled layout (ops/gemm.TiledWeight.data);
// outputs as topk_route + moe_align + gather_quant_mxfp8 (with `used`) would produce them.
void moe_route_fused(torch::Tensor x, torch::Tensor w_tiled, int64_t E, c10::optional<torch::Tensor> bias,
                     int64_t k, int64_t mode, double scale, int64_t e_lo, int64_t e_local, int64_t bn,
                     torch::Tensor partial, torch::Tensor w_out, torch::Tensor id_out, torch::Tensor seg_offsets,
                     torch::Tensor tile_offsets, torch::Tensor sorted_src, torch::Tensor inv_map, torch::Tensor q,
                     torch::Tensor sf, torch::Tensor sync, torch::Tensor status, int64_t k_chunks) {
  const int T = x.size(0), H = x.size(1);
  if (T == 0) return;
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.stride(1) == 1 && H % 64 == 0, "moe_route_fused: x");
  TORCH_CHECK((x.stride(0) * 2) % 16 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
              "moe_route_fused: x rows must be 16-byte aligned");
  TORCH_CHECK(E <= 256 && k <= kMaxK && k <= 32 && k <= E && T * E <= kMaxLogits, "moe_route_fused: T*E or k too large");
  const int nk = (H + 63) / 64;
  TORCH_CHECK(w_tiled.scalar_type() == at::kBFloat16 && w_tiled.numel() == ((E + 127) / 128) * nk * 128 * 64,
              "moe_route_fused: tiled router weight shape");
  TORCH_CHECK(partial.numel() >= k_chunks * T * E && partial.scalar_type() == at::kFloat, "moe_route_fused: partial");
  const int R_max = sorted_src.numel();
  TORCH_CHECK(R_max >= T * k + e_local * (bn - 1) && R_max % bn == 0 && q.size(0) == R_max, "moe_route_fused: rows");
  const int Kp = q.size(1);
  RouteArgs a;
  a.x = (const __nv_bfloat16*)x.data_ptr();
  a.xs = x.stride(0);
  a.T = T;
  a.H = H;
  a.w = (const __nv_bfloat16*)w_tiled.data_ptr();
  a.nk = nk;
  a.bias = bias ? (const __nv_bfloat16*)bias->data_ptr() : nullptr;
  a.E = E;
  a.K = k;
  a.mode = mode;
  a.scale = (float)scale;
  a.e_lo = e_lo;
  a.E_local = e_local;
  a.BN = bn;
  a.k_chunks = k_chunks;
  a.kc_len = ((H + k_chunks - 1) / k_chunks + 63) / 64 * 64;  // whole 64-wide blocks (four k16 steps)
  a.partial = partial.data_ptr<float>();
  a.w_out = w_out.data_ptr<float>();
  a.id_out = id_out.data_ptr<int32_t>();
  a.seg_offsets = seg_offsets.data_ptr<int32_t>();
  a.tile_offsets = tile_offsets.data_ptr<int32_t>();
  a.sorted_src = sorted_src.data_ptr<int32_t>();
  a.inv_map = inv_map.data_ptr<int32_t>();
  a.R_max = R_max;
  a.q = (uint8_t*)q.data_ptr();
  a.sf = (uint8_t*)sf.data_ptr();
  a.Kp = Kp;
  a.sync = reinterpret_cast<uint32_t*>(sync.data_ptr<int32_t>());
  a.status = status.data_ptr<int>();
  const int grid = (int)((E + kEGroup - 1) / kEGroup * k_chunks);
  // shared memory: ids and stable positions of the T*k entries, counts and offsets, the used rows' sources
  const size_t smem = ((size_t)2 * T * k + 2 * e_local + 1 + (size_t)T * k + (size_t)e_local * bn) * 4;
  TORCH_CHECK(smem <= 48 * 1024, "moe_route_fused: shared memory");
  snb::launch_pdl(moe_route_fused_kernel, grid, kThreads, smem, at::cuda::getCurrentCUDAStream(), a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
