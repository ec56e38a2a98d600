// Decode-sized MoE routing in one launch: router GEMM -> top-k -> counting sort into BN-padded expert
// segments -> MXFP8 gather-quantise of the routed rows.
//
// The separate path takes four launches per MoE layer (router GEMM, top-k, alignment, quantise); at a few
// dozen tokens each of them is a few microseconds of launch and tail latency around well under a microsecond
// of work. Here one grid does all of it:
//   phase 1, every CTA: a [T x 16-expert] block of router logits over one K chunk, on tensor cores
//            (mma.sync m16n8k16 bf16 -> fp32; the router weight is read in the GEMM's tiled layout), written
//            as an fp32 partial;
//   phase 2, the last CTA to finish phase 1 (arrival ticket): sums the K-chunk partials, adds the bias and
//            rounds to bf16 (the logits the separate router GEMM would produce), selects the top-k experts of
//            every token, and sorts the (token, slot) entries of the experts owned here by expert into
//            BN-padded segments (sorted_src, inv_map, seg_offsets, tile_offsets);
//   phase 3, every CTA, once the last CTA published phase 2 (epoch flag): quantises the routed rows to MXFP8
//            (e4m3 values, e8m0 scale per 32, scales in the tcgen05 scale-atom order), zero rows for padding.
// Each CTA triggers the dependent launch only after it has passed the arrival ticket, i.e. once every CTA of
// the grid is resident, so a programmatically launched successor can never take the SMs a late CTA needs.
// Every wait is bounded (SNB_WAIT_NS); a timeout records SNB_ERR_TIMEOUT_PEER and the CTA returns.
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
constexpr int kMaxLogits = 16384;  // T * E staged in shared memory by the last CTA (64 KB)
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
  uint32_t* sync;          // [0] arrival ticket, [1] epoch
  int* status;
  unsigned long long* dbg;  // DEBUG timestamps
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

// Last CTA: logits, top-k, counting sort. Shared memory: logits [T*E] fp32, then ids [T*K], then counters.
SNB_DEVICE void phase2(const RouteArgs& a, float* lg, int32_t* sid, int32_t* cnt) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int TE = a.T * a.E;
  {
    // sum of the K-chunk partials: each thread keeps its (up to 64) logits in registers and issues one K
    // chunk's loads for all of them at once, so the reduction costs k_chunks L2 round trips, not T*E/256 x that
    constexpr int kJ = kMaxLogits / kThreads;
    float acc[kJ];
#pragma unroll
    for (int j = 0; j < kJ; ++j) acc[j] = 0.f;
    for (int kc = 0; kc < a.k_chunks; ++kc) {
      const float* p = a.partial + (size_t)kc * TE + tid;
#pragma unroll
      for (int j = 0; j < kJ; ++j)
        if (tid + j * kThreads < TE) acc[j] += __ldcg(p + j * kThreads);
    }
#pragma unroll
    for (int j = 0; j < kJ; ++j) {
      const int i = tid + j * kThreads;
      if (i < TE) {
        float s = acc[j];
        if (a.bias != nullptr) s += __bfloat162float(a.bias[i % a.E]);
        lg[i] = __bfloat162float(__float2bfloat16(s));  // the bf16 logits of the separate router GEMM
      }
    }
  }
  __syncthreads();
  if (a.dbg && tid == 0) a.dbg[gridDim.x * 4 + 1] = snb::globaltimer_ns();
  // top-k: one warp per token (ties -> smallest expert id)
  for (int t = warp; t < a.T; t += kWarps) {
    const float* row = lg + (size_t)t * a.E;
    float v[8];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = lane + 32 * i;
      v[i] = e < a.E ? row[e] : -INFINITY;
      mx = fmaxf(mx, v[i]);
    }
    mx = snb::warp_max(mx);
    float denom_all = 0.f;
    if (a.mode == 1) {
#pragma unroll
      for (int i = 0; i < 8; ++i) denom_all += (v[i] == -INFINITY) ? 0.f : __expf(v[i] - mx);
      denom_all = snb::warp_sum(denom_all);
    }
    float sel_v[kMaxK];
    int sel_i[kMaxK];
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
      sel_v[j] = bv;
      sel_i[j] = bi;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (lane + 32 * i == bi) v[i] = -INFINITY;
    }
    if (lane == 0) {
      float s = 0.f;
      if (a.mode == 0)
        for (int j = 0; j < a.K; ++j) s += __expf(sel_v[j] - sel_v[0]);
      for (int j = 0; j < a.K; ++j) {
        const float wj = a.mode == 0 ? __expf(sel_v[j] - sel_v[0]) / s * a.scale
                                     : __expf(sel_v[j] - mx) / denom_all * a.scale;
        a.w_out[(size_t)t * a.K + j] = wj;
        a.id_out[(size_t)t * a.K + j] = sel_i[j];
        sid[t * a.K + j] = sel_i[j];
      }
    }
  }
  __syncthreads();
  if (a.dbg && tid == 0) a.dbg[gridDim.x * 4 + 2] = snb::globaltimer_ns();
  // counting sort of the entries owned here into BN-padded segments
  const int N = a.T * a.K, El = a.E_local;
  int32_t* off = cnt + El;
  int32_t* cur = off + El + 1;
  for (int e = tid; e < El; e += kThreads) cnt[e] = cur[e] = 0;
  __syncthreads();
  for (int i = tid; i < N; i += kThreads) {
    const int e = sid[i] - a.e_lo;
    if (e >= 0 && e < El) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (tid == 0) {
    int rows = 0, tiles = 0;
    for (int e = 0; e < El; ++e) {
      off[e] = rows;
      a.seg_offsets[e] = rows;
      a.tile_offsets[e] = tiles;
      const int padded = (cnt[e] + a.BN - 1) / a.BN * a.BN;
      rows += padded;
      tiles += padded / a.BN;
    }
    off[El] = rows;
    a.seg_offsets[El] = rows;
    a.tile_offsets[El] = tiles;
  }
  __syncthreads();
  for (int r = tid; r < off[El]; r += kThreads) a.sorted_src[r] = -1;
  __syncthreads();
  for (int i = tid; i < N; i += kThreads) {
    const int e = sid[i] - a.e_lo;
    if (e >= 0 && e < El) {
      const int p = off[e] + atomicAdd(&cur[e], 1);
      a.sorted_src[p] = i / a.K;
      a.inv_map[i] = p;
    } else {
      a.inv_map[i] = -1;
    }
  }
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
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ int last_s;
  __shared__ uint32_t epoch_s;
  const int eg_count = (a.E + kEGroup - 1) / kEGroup;
  const int eg = blockIdx.x % eg_count, kc = blockIdx.x / eg_count;
  snb::pdl_wait();  // x is the previous kernel's output; the previous call's epoch store is complete
  if (threadIdx.x == 0) epoch_s = *reinterpret_cast<volatile uint32_t*>(&a.sync[1]) + 1;
  if (a.dbg && threadIdx.x == 0) a.dbg[blockIdx.x * 4 + 0] = snb::globaltimer_ns();
  phase1(a, eg, kc);
  __syncthreads();
  if (a.dbg && threadIdx.x == 0) a.dbg[blockIdx.x * 4 + 1] = snb::globaltimer_ns();
  if (threadIdx.x == 0) {
    __threadfence();
    last_s = atomicAdd(&a.sync[0], 1u) == gridDim.x - 1;
  }
  __syncthreads();
  // every CTA has arrived at the ticket (hence is resident) before any of them lets the next kernel launch
  snb::pdl_trigger();
  const uint32_t e = epoch_s;
  if (last_s) {
    __threadfence();
    float* lg = reinterpret_cast<float*>(smem);
    int32_t* sid = reinterpret_cast<int32_t*>(lg + a.T * a.E);
    int32_t* cnt = sid + a.T * a.K;
    phase2(a, lg, sid, cnt);
    __syncthreads();
    if (a.dbg && threadIdx.x == 0) a.dbg[gridDim.x * 4 + 0] = snb::globaltimer_ns();
    if (threadIdx.x == 0) {
      a.sync[0] = 0;
      __threadfence();
      asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(&a.sync[1]), "r"(e) : "memory");
    }
  } else if (threadIdx.x == 0) {
    const uint64_t t0 = snb::globaltimer_ns();
    for (;;) {
      uint32_t v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(&a.sync[1]) : "memory");
      if ((int32_t)(v - e) >= 0) break;
      if (snb::globaltimer_ns() - t0 > SNB_WAIT_NS) {
        snb::record_status(a.status, SNB_ERR_TIMEOUT_PEER);
        last_s = -1;
        break;
      }
    }
  }
  __syncthreads();
  if (a.dbg && threadIdx.x == 0) a.dbg[blockIdx.x * 4 + 2] = snb::globaltimer_ns();
  if (last_s < 0) return;
  const int used = *reinterpret_cast<volatile int32_t*>(&a.seg_offsets[a.E_local]);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int r = blockIdx.x * kWarps + warp; r < used; r += gridDim.x * kWarps) {
    const int s = reinterpret_cast<volatile int32_t*>(a.sorted_src)[r];
    quant_row(a, r, s, lane);
  }
  __syncthreads();
  if (a.dbg && threadIdx.x == 0) a.dbg[blockIdx.x * 4 + 3] = snb::globaltimer_ns();
}

}  // namespace

// x: [T, H] bf16; w_tiled: the router weight in the GEMM's tiled layout (ops/gemm.TiledWeight.data);
// outputs as topk_route + moe_align + gather_quant_mxfp8 (with `used`) would produce them.
void moe_route_fused(torch::Tensor x, torch::Tensor w_tiled, int64_t E, c10::optional<torch::Tensor> bias,
                     int64_t k, int64_t mode, double scale, int64_t e_lo, int64_t e_local, int64_t bn,
                     torch::Tensor partial, torch::Tensor w_out, torch::Tensor id_out, torch::Tensor seg_offsets,
                     torch::Tensor tile_offsets, torch::Tensor sorted_src, torch::Tensor inv_map, torch::Tensor q,
                     torch::Tensor sf, torch::Tensor sync, torch::Tensor status, int64_t k_chunks,
                     c10::optional<torch::Tensor> dbg) {
  const int T = x.size(0), H = x.size(1);
  if (T == 0) return;
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.stride(1) == 1 && H % 64 == 0, "moe_route_fused: x");
  TORCH_CHECK((x.stride(0) * 2) % 16 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
              "moe_route_fused: x rows must be 16-byte aligned");
  TORCH_CHECK(E <= 256 && k <= kMaxK && k <= E && T * E <= kMaxLogits, "moe_route_fused: T*E or k too large");
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
  a.dbg = dbg ? reinterpret_cast<unsigned long long*>(dbg->data_ptr<int64_t>()) : nullptr;
  const int grid = (int)((E + kEGroup - 1) / kEGroup * k_chunks);
  const size_t smem = (size_t)T * E * 4 + (size_t)T * k * 4 + (3 * e_local + 1) * 4;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(moe_route_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
    attr_set = true;
  }
  TORCH_CHECK(smem <= 96 * 1024, "moe_route_fused: shared memory");
  snb::launch_pdl(moe_route_fused_kernel, grid, kThreads, smem, at::cuda::getCurrentCUDAStream(), a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
