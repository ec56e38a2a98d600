// Paged GQA decode attention over an FP8 (e4m3) KV cache, with the KV stream pipelined through shared
// memory by bulk async copies.
//
// CTA = one (split, KV head, request): warps 0-3 compute, warp 4 is the producer. The producer copies whole
// page segments of K and V (`cp.async.bulk`, 1 KB per 16-token page at D = 64) into a 4-stage ring of
// 64-token tiles and signals an mbarrier per stage; the compute warps release a stage through a second
// mbarrier once its bytes are in registers. Tens of KB per CTA are in flight, which is what an HBM-bound
// decode step needs (the previous design prefetched one 8 KB tile through registers).
//
// Math on mma.sync m16n8k16 with f16 operands: e4m3 converts to f16 exactly (cvt.rn.f16x2.e4m3x2, two
// values per instruction), Q converts from bf16 with satfinite, probabilities in [0, 1] keep 10 mantissa
// bits. The G query heads of the KV head are the M rows (zero rows above G). Two index permutations make
// every operand fetch a conflict-free 8/16-byte shared load with no transpose pass:
//   * the contraction index of Q K^T (head dim) is permuted so a thread's K fragments are D/4 contiguous
//     bytes of one token row (Q is gathered with the same permutation);
//   * the token order inside a warp's 16 tokens is permuted (column j of n-tile nt is token
//     (j >> 1) + 4 * (2 nt + (j & 1))), so the P fragment a thread owns covers tokens qd, qd+4, qd+8, qd+12
//     and its V fragments are D/8 contiguous bytes of four token rows; the output column c of n-tile n is
//     head-dim c * (D / 8) + n.
// Tokens outside [window start, split end) are masked in S and their V bytes are zeroed in registers (pages
// may hold stale bytes of other requests).
//
// Parity: the reference's attention_decode / attention_decode_paged (sglang_neuron/ops/attention/
// attention_decode.py:28-205) with learned sinks, sliding window and FP8 KV.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <cuda_fp8.h>
#include "../common.cuh"

namespace {

constexpr float kL2e = 1.4426950408889634f;
constexpr int kTile = 64;     // tokens per stage
constexpr int kCWarps = 4;    // compute warps, 16 tokens each per tile
constexpr int kThreads = (kCWarps + 1) * 32;
constexpr int kMaxSplitPages = 1024;  // block-table entries of one split staged in shared memory

template <int D>
struct Fp8Cfg {
  static constexpr int NST = D == 64 ? 4 : 3;           // ring stages
  static constexpr int STAGE = 2 * kTile * D;           // K tile then V tile, fp8
  static constexpr int MERGE = kCWarps * 16 * D * 4;    // fp32 [warp][16 rows][D], reuses the ring
  static constexpr int RING = NST * STAGE > MERGE ? NST * STAGE : MERGE;
  static constexpr int SMEM = RING + 2 * NST * 8 + kCWarps * 16 * 2 * 4 + 64 + kMaxSplitPages * 4;
};

SNB_DEVICE void mma_f16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// two e4m3 bytes (low byte -> low half) -> f16x2
SNB_DEVICE uint32_t e4m3x2_to_f16x2(uint32_t two_bytes) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(two_bytes & 0xffffu), __NV_E4M3);
  return static_cast<uint32_t>(h.x) | (static_cast<uint32_t>(h.y) << 16);
}

SNB_DEVICE uint32_t f32x2_to_f16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

SNB_DEVICE void bulk_load_nohint(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

template <int D>
__global__ void __launch_bounds__(kThreads) decode_attn_fp8_kernel(
    const __nv_bfloat16* __restrict__ q, int q_stride, const uint8_t* __restrict__ kc, const uint8_t* __restrict__ vc,
    const int32_t* __restrict__ block_table, int bt_stride, const int32_t* __restrict__ seq_lens, int page_size,
    int Hkv, int G, int window, float scale_log2, float v_scale, const float* __restrict__ sinks,
    __nv_bfloat16* __restrict__ out, int out_stride, float* __restrict__ o_part, float* __restrict__ lse_part,
    int num_splits, int* status, int* __restrict__ merge_cnt, float v_scale_out) {
  using C = Fp8Cfg<D>;
  constexpr int NT = D / 8;      // n8 tiles of the output (head dim)
  constexpr int KB = D / 4;      // K bytes per thread per token row
  constexpr int VB = D / 8;      // V bytes per thread per token row
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::RING);
  uint64_t* empty = full + C::NST;
  float* red_m = reinterpret_cast<float*>(empty + C::NST);  // [warp][16]
  float* red_l = red_m + kCWarps * 16;
  int* sh = reinterpret_cast<int*>(red_l + kCWarps * 16);   // [0] issued, [1] consumed, [2] error
  int32_t* sbt = sh + 16;                                    // this split's block-table entries

  const int split = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < C::NST; ++s) {
      snb::mbar_init(&full[s], 1);
      snb::mbar_init(&empty[s], kCWarps);
    }
    sh[0] = sh[1] = sh[2] = 0;
    snb::fence_mbar_init();
  }
  __syncthreads();
  snb::pdl_wait();
  snb::pdl_trigger();

  const int ctx = seq_lens[b];
  const int lo = (window > 0 && ctx > window) ? ctx - window : 0;  // first attended token
  const int base = (lo / kTile) * kTile;
  const int per = ((ctx - base + num_splits - 1) / num_splits + kTile - 1) / kTile * kTile;
  const int s0 = base + split * per;
  const int s1 = min(ctx, s0 + per);
  const int ntiles = s0 < s1 ? (s1 - s0 + kTile - 1) / kTile : 0;
  const int32_t* bt = block_table + (size_t)b * bt_stride;
  const int seg = page_size < kTile ? page_size : kTile;  // tokens per bulk copy
  // stage the split's page ids once (coalesced) so the producer never waits on a dependent global load
  const int pg0 = s0 / page_size;
  const int npg = s0 < s1 ? (s1 - 1) / page_size - pg0 + 1 : 0;
  for (int i = tid; i < min(npg, kMaxSplitPages); i += kThreads) sbt[i] = bt[pg0 + i];
  __syncthreads();

  if (warp == kCWarps) {
    // ---------------- producer
    if (lane == 0) {
      int k = 0;
      for (; k < ntiles; ++k) {
        const int s = k % C::NST;
        if (k >= C::NST &&
            !snb::mbar_wait_bounded(&empty[s], ((k / C::NST) & 1) ^ 1, status, SNB_ERR_TIMEOUT_TMA)) {
          break;
        }
        const int t0 = s0 + k * kTile;
        uint32_t bytes = 0;
        for (int i = 0; i < kTile / seg; ++i) {
          const int ta = t0 + i * seg;
          if (ta + seg > lo && ta < s1) bytes += 2u * seg * D;
        }
        snb::mbar_arrive_expect_tx(&full[s], bytes);
        const uint32_t kd = snb::smem_u32(ring + s * C::STAGE), vd = kd + kTile * D;
        for (int i = 0; i < kTile / seg; ++i) {
          const int ta = t0 + i * seg;
          if (!(ta + seg > lo && ta < s1)) continue;
          const int pi = ta / page_size - pg0;
          const int32_t page = pi < kMaxSplitPages ? sbt[pi] : bt[ta / page_size];
          const size_t off = (((size_t)page * Hkv + hk) * page_size + ta % page_size) * D;
          bulk_load_nohint(kd + i * seg * D, kc + off, seg * D, snb::smem_u32(&full[s]));
          bulk_load_nohint(vd + i * seg * D, vc + off, seg * D, snb::smem_u32(&full[s]));
        }
      }
      sh[0] = k;
    }
  } else {
    // ---------------- compute warps
    const int gq = lane >> 2, qd = lane & 3;
    // Q fragments (A operand), f16, contraction index permuted: logical (ks, h, e) -> d = qd*KB + ks*4 + h*2 + e
    uint32_t qa[D / 16][4];
    {
      const __nv_bfloat16* qb = q + (size_t)b * q_stride + (size_t)hk * G * D;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int row = gq + (r & 1) * 8;
          const int d = qd * KB + ks * 4 + (r >> 1) * 2;
          if (row < G) {
            const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(qb + (size_t)row * D + d);
            qa[ks][r] = f32x2_to_f16x2(__bfloat162float(v.x), __bfloat162float(v.y));
          } else {
            qa[ks][r] = 0u;
          }
        }
      }
    }
    float o[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
    // this thread's token rows: K rows for n-tiles 0/1, V rows i = 0..3 (token qd + 4 i)
    const int krow0 = (gq >> 1) + 4 * (gq & 1), krow1 = krow0 + 8;
    int k = 0;
    for (; k < ntiles; ++k) {
      const int s = k % C::NST;
      if (!snb::mbar_wait_bounded(&full[s], (k / C::NST) & 1, status, SNB_ERR_TIMEOUT_MMA)) {
        sh[2] = 1;
        break;
      }
      const uint8_t* kt = ring + s * C::STAGE + warp * 16 * D;
      const uint8_t* vt = kt + kTile * D;
      const int tw = s0 + k * kTile + warp * 16;  // first token of this warp's 16
      // ---- S = Q K^T (two n8 tiles)
      uint32_t kw[2][KB / 4];
#pragma unroll
      for (int i = 0; i < KB / 16; ++i) {
        const uint4 a = *reinterpret_cast<const uint4*>(kt + krow0 * D + qd * KB + i * 16);
        const uint4 c = *reinterpret_cast<const uint4*>(kt + krow1 * D + qd * KB + i * 16);
        kw[0][i * 4] = a.x; kw[0][i * 4 + 1] = a.y; kw[0][i * 4 + 2] = a.z; kw[0][i * 4 + 3] = a.w;
        kw[1][i * 4] = c.x; kw[1][i * 4 + 1] = c.y; kw[1][i * 4 + 2] = c.z; kw[1][i * 4 + 3] = c.w;
      }
      // ---- V rows (token qd + 4 i), D/8 bytes each at offset gq * VB
      uint32_t vw[4][VB / 4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint8_t* src = vt + (qd + 4 * i) * D + gq * VB;
        const int tok = tw + qd + 4 * i;
        const bool ok = tok >= lo && tok < s1;
        if constexpr (VB == 8) {
          const uint2 v = *reinterpret_cast<const uint2*>(src);
          vw[i][0] = ok ? v.x : 0u;
          vw[i][1] = ok ? v.y : 0u;
        } else {
          const uint4 v = *reinterpret_cast<const uint4*>(src);
          vw[i][0] = ok ? v.x : 0u;
          vw[i][1] = ok ? v.y : 0u;
          vw[i][2] = ok ? v.z : 0u;
          vw[i][3] = ok ? v.w : 0u;
        }
      }
      __syncwarp();
      if (lane == 0) snb::mbar_arrive(&empty[s]);  // this warp's bytes of the stage are in registers
      float sc[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t w4 = kw[nt][ks];
          mma_f16_16816(sc[nt], qa[ks], e4m3x2_to_f16x2(w4), e4m3x2_to_f16x2(w4 >> 16));
        }
      }
      // ---- online softmax over rows gq / gq + 8; column j of n-tile nt is token (j>>1) + 4*(2nt + (j&1))
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int tok = tw + qd + 4 * (2 * nt + (j & 1));
          const float v = (tok >= lo && tok < s1) ? sc[nt][j] * scale_log2 : -INFINITY;
          sc[nt][j] = v;
          mx[j >> 1] = fmaxf(mx[j >> 1], v);
        }
      }
      float alpha[2], rs[2] = {0.f, 0.f};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
        const float mn = fmaxf(m_r[h], mx[h]);
        alpha[h] = (m_r[h] == -INFINITY) ? (mn == -INFINITY ? 1.f : 0.f) : exp2f(m_r[h] - mn);
        m_r[h] = mn;
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float p = (sc[nt][j] == -INFINITY) ? 0.f : exp2f(sc[nt][j] - m_r[j >> 1]);
          sc[nt][j] = p;
          rs[j >> 1] += p;
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 1);
        rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 2);
        l_r[h] = l_r[h] * alpha[h] + rs[h];
      }
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        o[n][0] *= alpha[0];
        o[n][1] *= alpha[0];
        o[n][2] *= alpha[1];
        o[n][3] *= alpha[1];
      }
      // ---- O += P V: P is the A operand (k = the warp's 16 tokens in the permuted order)
      uint32_t pa[4];
      pa[0] = f32x2_to_f16x2(sc[0][0], sc[0][1]);
      pa[1] = f32x2_to_f16x2(sc[0][2], sc[0][3]);
      pa[2] = f32x2_to_f16x2(sc[1][0], sc[1][1]);
      pa[3] = f32x2_to_f16x2(sc[1][2], sc[1][3]);
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        // byte n of this thread's V slice (head dim gq*VB + n) for tokens (qd, qd+4) and (qd+8, qd+12)
        const int w = n >> 2, sel = n & 3;
        const uint32_t b0 = e4m3x2_to_f16x2(__byte_perm(vw[0][w], vw[1][w], sel | ((4 + sel) << 4)));
        const uint32_t b1 = e4m3x2_to_f16x2(__byte_perm(vw[2][w], vw[3][w], sel | ((4 + sel) << 4)));
        mma_f16_16816(o[n], pa, b0, b1);
      }
    }
    if (warp == 0 && lane == 0) sh[1] = k;
    // ---- per-warp state to shared memory for the merge (after every warp left the ring: barrier below)
    __syncwarp();
    asm volatile("bar.sync 1, %0;" ::"n"(kCWarps * 32) : "memory");
    float* obuf = reinterpret_cast<float*>(ring);
    if (qd == 0) {
      red_m[warp * 16 + gq] = m_r[0];
      red_m[warp * 16 + gq + 8] = m_r[1];
      red_l[warp * 16 + gq] = l_r[0];
      red_l[warp * 16 + gq + 8] = l_r[1];
    }
#pragma unroll
    for (int n = 0; n < NT; ++n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int d = (qd * 2 + e) * VB + n;
        obuf[(warp * 16 + gq) * D + d] = o[n][e];
        obuf[(warp * 16 + gq + 8) * D + d] = o[n][2 + e];
      }
    }
  }
  __syncthreads();
  if (warp < kCWarps) {
    const int Hq = Hkv * G;
    const float* obuf = reinterpret_cast<const float*>(ring);
    for (int idx = tid; idx < G * D; idx += kCWarps * 32) {
      const int g = idx / D, d = idx % D;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kCWarps; ++w) M = fmaxf(M, red_m[w * 16 + g]);
      float L = 0.f, acc = 0.f;
#pragma unroll
      for (int w = 0; w < kCWarps; ++w) {
        if (red_m[w * 16 + g] == -INFINITY) continue;
        const float f = exp2f(red_m[w * 16 + g] - M);
        L += red_l[w * 16 + g] * f;
        acc += obuf[(w * 16 + g) * D + d] * f;
      }
      const int h = hk * G + g;
      if (num_splits == 1) {
        float denom = L;
        if (sinks != nullptr) denom = (M == -INFINITY) ? 1.f : L + exp2f(sinks[h] * kL2e - M);
        out[(size_t)b * out_stride + (size_t)h * D + d] =
            __float2bfloat16(denom > 0.f ? acc / denom * v_scale : 0.f);
      } else {
        const size_t pidx = ((size_t)b * Hq + h) * num_splits + split;
        o_part[pidx * D + d] = L > 0.f ? acc / L : 0.f;
        if (d == 0) lse_part[pidx] = L > 0.f ? M + log2f(L) : -INFINITY;
      }
    }
  } else if (lane == 0) {
    // a CTA that stopped early still waits (bounded) for the copies it issued before its memory goes away
    for (int i = sh[1]; i < sh[0]; ++i)
      if (!snb::mbar_wait_bounded(&full[i % C::NST], (i / C::NST) & 1, status, SNB_ERR_TIMEOUT_TMA)) break;
  }
  if (num_splits > 1 && merge_cnt != nullptr) {
    // Split merge in this launch: the last split CTA of (request, KV head) to finish combines every split's
    // normalised partial (log2-sum-exp weights, sinks in the denominator) and writes the output rows; it
    // then re-arms the counter for the next call. Partials are read past L1 (written by other CTAs).
    __threadfence();
    __syncthreads();
    int* cnt = merge_cnt + (size_t)b * Hkv + hk;
    if (tid == 0) sh[3] = atomicAdd(cnt, 1) == num_splits - 1;
    __syncthreads();
    if (sh[3]) {
      __threadfence();
      const int Hq = Hkv * G;
      for (int idx = tid; idx < G * D; idx += kThreads) {
        const int g = idx / D, d = idx % D, h = hk * G + g;
        const size_t base = ((size_t)b * Hq + h) * num_splits;
        float M = -INFINITY;
        for (int s = 0; s < num_splits; ++s) M = fmaxf(M, __ldcg(lse_part + base + s));
        const float sk = sinks != nullptr ? sinks[h] * kL2e : -INFINITY;
        const float Mx = fmaxf(M, sk);
        float total = (sk == -INFINITY) ? 0.f : exp2f(sk - Mx), acc = 0.f;
        for (int s = 0; s < num_splits; ++s) {
          const float l = __ldcg(lse_part + base + s);
          if (l == -INFINITY) continue;
          const float f = exp2f(l - Mx);
          total += f;
          acc += f * __ldcg(o_part + (base + s) * D + d);
        }
        const float r = (M == -INFINITY || total <= 0.f) ? 0.f : acc / total * v_scale_out;
        out[(size_t)b * out_stride + (size_t)h * D + d] = __float2bfloat16(r);
      }
      if (tid == 0) *cnt = 0;
    }
  }
}

}  // namespace

// Same contract as decode_attention_mma() for an fp8 cache; false when not covered (head_dim not 64/128, G > 16,
// or a page size that is neither a divisor nor a multiple of the 64-token tile). With merge_cnt (zeroed int32
// per (request, KV head)) and more than one split, the split merge runs inside this launch (v_scale_out is
// applied there) and no merge kernel follows.
bool decode_attention_fp8(torch::Tensor out, torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                          torch::Tensor block_table, torch::Tensor seq_lens, int64_t num_q_heads, int64_t num_kv_heads,
                          int64_t head_dim, int64_t page_size, int64_t window, float scale_log2, float v_scale_final,
                          const float* sinks, int64_t num_splits, float* o_part, float* lse_part, int* status,
                          int* merge_cnt, float v_scale_out) {
  const int G = num_q_heads / num_kv_heads;
  if (k_cache.scalar_type() != at::kFloat8_e4m3fn || G > 16 || (head_dim != 64 && head_dim != 128)) return false;
  if (!((page_size >= 16 && kTile % page_size == 0) || (page_size >= kTile && page_size % kTile == 0))) return false;
  if (k_cache.data_ptr() == nullptr || reinterpret_cast<uintptr_t>(k_cache.data_ptr()) % 16 ||
      reinterpret_cast<uintptr_t>(v_cache.data_ptr()) % 16 || !k_cache.is_contiguous() || !v_cache.is_contiguous())
    return false;
  const int B = q.size(0);
  auto st = at::cuda::getCurrentCUDAStream();
  dim3 grid(num_splits, num_kv_heads, B);
#define SNB_FP8(DD)                                                                                              \
  {                                                                                                              \
    using C = Fp8Cfg<DD>;                                                                                        \
    static bool attr = false;                                                                                    \
    if (!attr) {                                                                                                 \
      C10_CUDA_CHECK(cudaFuncSetAttribute(decode_attn_fp8_kernel<DD>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                          C::SMEM));                                                             \
      attr = true;                                                                                               \
    }                                                                                                            \
    C10_CUDA_CHECK(snb::launch_pdl(decode_attn_fp8_kernel<DD>, grid, kThreads, C::SMEM, st,                      \
                                   (const __nv_bfloat16*)q.data_ptr(), (int)q.stride(0),                         \
                                   (const uint8_t*)k_cache.data_ptr(), (const uint8_t*)v_cache.data_ptr(),       \
                                   block_table.data_ptr<int32_t>(), (int)block_table.stride(0),                 \
                                   seq_lens.data_ptr<int32_t>(), (int)page_size, (int)num_kv_heads, G,           \
                                   (int)window, scale_log2, v_scale_final, sinks, (__nv_bfloat16*)out.data_ptr(), \
                                   (int)out.stride(0), o_part, lse_part, (int)num_splits, status, merge_cnt,     \
                                   v_scale_out));                                                                \
  }
  if (head_dim == 64) SNB_FP8(64) else SNB_FP8(128)
#undef SNB_FP8
  return true;
}
