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

// e4m3 byte pairs -> f16x2 (lower byte -> lower half): bytes 0-1 or bytes 2-3 of a 32-bit word, one cvt each
SNB_DEVICE uint32_t e4m3x2_to_f16x2(uint32_t w) {
  uint32_t r;
  asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, l;\n\t}" : "=r"(r) : "r"(w));
  return r;
}

SNB_DEVICE uint32_t e4m3x2_hi_to_f16x2(uint32_t w) {
  uint32_t r;
  asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, h;\n\t}" : "=r"(r) : "r"(w));
  return r;
}

// 2^x on the special-function unit (inputs here are <= 0 or -inf; -inf gives +0)
SNB_DEVICE float ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// 16-byte global -> shared copy (L2 only), and an arrival on `bar` once this thread's copies have landed
SNB_DEVICE void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

SNB_DEVICE void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(snb::smem_u32(bar)) : "memory");
}

SNB_DEVICE void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

SNB_DEVICE uint32_t f32x2_to_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
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

// CTA epilogue shared by both FP8 kernels: combine the compute warps' (max, sum, O) over shared memory and write
// the output rows (one split) or this split's normalised partial and log2-sum-exp; the producer lane waits
// (bounded) for copies a stopped CTA still has in flight; with merge counters the last split CTA of a
// (request, KV head) merges every split. red_m / red_l are [warp][16 heads], obuf is fp32 [warp][16 heads][D].
template <int D>
SNB_DEVICE void decode_fp8_finish(int warp, int tid, int lane, int b, int hk, int split, int Hkv, int G,
                                  int num_splits, const float* __restrict__ sinks, float v_scale,
                                  __nv_bfloat16* __restrict__ out, int out_stride, float* __restrict__ o_part,
                                  float* __restrict__ lse_part, const float* red_m, const float* red_l,
                                  const float* obuf, int* sh, uint64_t* full, int nst, int* status,
                                  int* __restrict__ merge_cnt, float v_scale_out) {
  if (warp < kCWarps) {
    const int Hq = Hkv * G;
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
      if (!snb::mbar_wait_bounded(&full[i % nst], (i / nst) & 1, status, SNB_ERR_TIMEOUT_TMA)) break;
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
          mma_f16_16816(sc[nt], qa[ks], e4m3x2_to_f16x2(w4), e4m3x2_hi_to_f16x2(w4));
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
  decode_fp8_finish<D>(warp, tid, lane, b, hk, split, Hkv, G, num_splits, sinks, v_scale, out, out_stride, o_part,
                       lse_part, red_m, red_l, reinterpret_cast<const float*>(ring), sh, full, C::NST, status,
                       merge_cnt, v_scale_out);
}

// ---------------------------------------------------------------------------------------------------------------
// Token-major variant: S^T = K Q^T and O^T = V^T P^T, so the MMA's M dimension is tokens (S^T) and head dims
// (O^T) and its N dimension is the G query heads (8 per n-tile, NG n-tiles). No MMA row is padding for
// G = 8, a thread holds four scores of two heads per 16 tokens (the row-sum stays a per-thread partial until the
// end), the scale is folded into Q, and O is rescaled only when some running max moved. P^T leaves the
// accumulator layout as the B operand of the second MMA through one `movmatrix.trans` per 8x8 block.
// CTA = one (split, KV head, request); 4 compute warps take 32 tokens each of a 128-token stage (e4m3 cache,
// f16 MMAs after one cvt per byte pair) or 16 tokens each of a 64-token stage (bf16 cache, bf16 MMAs on the
// cached values as they are, scores scaled after the MMA).
//
// Index maps (all bijections, chosen so every shared-memory fetch is a contiguous 8/16-byte load):
//   * contraction index of S^T (head dim): step ks, column kk = 2qq + e + 8h -> dim qq*(D/4) + 4ks + 2h + e;
//   * row r = r3 r2 r1 r0 (bits) of a 16-token block -> token 8r3 + 4r0 + 2r2 + r1, so the k-rows a thread
//     owns in O^T = V^T P^T (2qd, 2qd+1, 2qd+8, 2qd+9) are tokens qd, qd+4, qd+8, qd+12;
//   * O^T row (m-tile mt, row 8h + g) -> head dim g*(D/8) + 2mt + h.
template <int D, int NG, typename CT>
struct TokCfg {
  static constexpr int ES = (int)sizeof(CT);            // bytes per cached element (e4m3: 1, bf16: 2)
  static constexpr int TPW = ES == 1 ? 32 : 16;         // tokens per compute warp per stage
  static constexpr int U = TPW / 16;                    // 16-token blocks per warp
  static constexpr int TILE = kCWarps * TPW;            // tokens per stage
  static constexpr int NST = ES == 1 ? (D == 64 ? 3 : 2) : (D == 64 ? 4 : 3);  // ring stages
  static constexpr int STAGE = 2 * TILE * D * ES;       // K tile then V tile
  static constexpr int MERGE = kCWarps * 16 * D * 4;    // fp32 [warp][16 heads][D], reuses the ring
  static constexpr int RING = NST * STAGE > MERGE ? NST * STAGE : MERGE;
  static constexpr int SMEM = RING + 2 * NST * 8 + kCWarps * 16 * 2 * 4 + 64 + kMaxSplitPages * 4;
};

SNB_DEVICE uint32_t movmatrix_trans(uint32_t x) {
  uint32_t r;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(r) : "r"(x));
  return r;
}

SNB_DEVICE int tok_of_row(int r) {  // row r of a 16-token block -> token offset
  return ((r >> 3) & 1) * 8 + (r & 1) * 4 + ((r >> 2) & 1) * 2 + ((r >> 1) & 1);
}

template <int D, int NG, bool BULK, typename CT>
__global__ void __launch_bounds__(kThreads) decode_attn_tok_kernel(
    const __nv_bfloat16* __restrict__ q, int q_stride, const CT* __restrict__ kc, const CT* __restrict__ vc,
    const int32_t* __restrict__ block_table, int bt_stride, const int32_t* __restrict__ seq_lens, int page_size,
    int Hkv, int G, int window, float scale_log2, float v_scale, const float* __restrict__ sinks,
    __nv_bfloat16* __restrict__ out, int out_stride, float* __restrict__ o_part, float* __restrict__ lse_part,
    int num_splits, int* status, int* __restrict__ merge_cnt, float v_scale_out) {
  using C = TokCfg<D, NG, CT>;
  constexpr int TILE = C::TILE, ES = C::ES, TPW = C::TPW, U = C::U;
  constexpr int KS = D / 16;     // contraction steps of S^T = m-tiles of O^T
  constexpr int KB = D / 4;      // K elements per thread per token row
  constexpr int VB = D / 8;      // V elements per thread per token row
  constexpr int RB = D * ES;     // bytes per cached token row
  constexpr int KBB = KB * ES, VBB = VB * ES;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::RING);
  uint64_t* empty = full + C::NST;
  float* red_m = reinterpret_cast<float*>(empty + C::NST);  // [warp][16 heads]
  float* red_l = red_m + kCWarps * 16;
  int* sh = reinterpret_cast<int*>(red_l + kCWarps * 16);   // [0] issued, [1] consumed, [3] merge flag
  int32_t* sbt = sh + 16;                                    // this split's block-table entries

  const int split = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < C::NST; ++s) {
      snb::mbar_init(&full[s], BULK ? 1 : 32);  // bulk: one expect-tx arrival; cp.async: one per producer lane
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
  const int base = (lo / TILE) * TILE;
  const int per = ((ctx - base + num_splits - 1) / num_splits + TILE - 1) / TILE * TILE;
  const int s0 = base + split * per;
  const int s1 = min(ctx, s0 + per);
  const int ntiles = s0 < s1 ? (s1 - s0 + TILE - 1) / TILE : 0;
  const int32_t* bt = block_table + (size_t)b * bt_stride;
  const int seg = page_size < TILE ? page_size : TILE;  // tokens per bulk copy
  const int pg0 = s0 / page_size;
  const int npg = s0 < s1 ? (s1 - 1) / page_size - pg0 + 1 : 0;
  for (int i = tid; i < min(npg, kMaxSplitPages); i += kThreads) sbt[i] = bt[pg0 + i];
  __syncthreads();

  if (warp == kCWarps) {
    // ---------------- producer: whole page segments of K and V into the ring, either as bulk copies (one
    // segment per lane, completion counted in bytes on the stage barrier) or as 16-byte cp.async by all 32
    // lanes (each lane arrives on the stage barrier once its copies have landed). Addressing is division-free
    // for pages of at most one stage: s0 is a multiple of the stage and the stage a multiple of the page.
    const int nseg = TILE / seg;
    const size_t pstride = (size_t)Hkv * page_size * D, hoff = (size_t)hk * page_size * D;
    auto seg_offset = [&](int k, int i) -> size_t {  // element offset of segment i of stage k in the cache
      int pi, inpage = 0;
      if (page_size <= TILE) {
        pi = k * nseg + i;
      } else {
        const int ta = s0 + k * TILE;
        pi = ta / page_size - pg0;
        inpage = ta - (pg0 + pi) * page_size;
      }
      const int32_t page = pi < kMaxSplitPages ? sbt[pi] : bt[pg0 + pi];
      return (size_t)page * pstride + hoff + (size_t)inpage * D;
    };
    int k = 0;
    for (; k < ntiles; ++k) {
      const int s = k % C::NST;
      bool ok = true;
      if (k >= C::NST) {
        if (lane == 0) ok = snb::mbar_wait_bounded(&empty[s], ((k / C::NST) & 1) ^ 1, status, SNB_ERR_TIMEOUT_TMA);
        ok = __shfl_sync(0xffffffffu, ok, 0);
      }
      if (!ok) break;
      const int t0 = s0 + k * TILE;
      const uint32_t kd = snb::smem_u32(ring + s * C::STAGE), vd = kd + TILE * RB;
      if constexpr (BULK) {
        const int ta = t0 + lane * seg;
        const bool valid = lane < nseg && ta + seg > lo && ta < s1;
        const uint32_t nvalid = __popc(__ballot_sync(0xffffffffu, valid));
        if (lane == 0) snb::mbar_arrive_expect_tx(&full[s], nvalid * 2u * seg * RB);
        __syncwarp();
        if (valid) {
          const size_t off = seg_offset(k, lane);
          bulk_load_nohint(kd + lane * seg * RB, kc + off, seg * RB, snb::smem_u32(&full[s]));
          bulk_load_nohint(vd + lane * seg * RB, vc + off, seg * RB, snb::smem_u32(&full[s]));
        }
      } else {
        for (int i = 0; i < nseg; ++i) {
          const int ta = t0 + i * seg;
          if (!(ta + seg > lo && ta < s1)) continue;
          const size_t off = seg_offset(k, i);
          const uint8_t* ksrc = reinterpret_cast<const uint8_t*>(kc + off);
          const uint8_t* vsrc = reinterpret_cast<const uint8_t*>(vc + off);
          for (int c = lane * 16; c < seg * RB; c += 32 * 16) {
            cp_async16(kd + i * seg * RB + c, ksrc + c);
            cp_async16(vd + i * seg * RB + c, vsrc + c);
          }
        }
        cp_async_arrive_noinc(&full[s]);
      }
    }
    if (lane == 0) sh[0] = k;
    if constexpr (!BULK) asm volatile("cp.async.wait_all;" ::: "memory");
  } else {
    // ---------------- compute warps
    const int gq = lane >> 2, qd = lane & 3;
    // Q^T fragments (B operand of S^T): head ng*8 + gq, dims qd*KB + 4ks + {0,1} and {2,3}. For an e4m3 cache
    // (f16 MMAs) Q is pre-scaled by scale * log2(e): f16 keeps 11 mantissa bits, more than the bf16 input has;
    // for a bf16 cache (bf16 MMAs) Q stays as it is and the scores are scaled.
    uint32_t qb[NG][KS][2];
    {
      const __nv_bfloat16* qh = q + (size_t)b * q_stride + (size_t)hk * G * D;
#pragma unroll
      for (int ng = 0; ng < NG; ++ng) {
        const int h = ng * 8 + gq;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            if (h < G) {
              // dim of contraction column (ks, 2qd + 8e): e4m3 -> qd*KB + 4ks + 2e (contiguous per thread);
              // bf16 -> (4 (ks / 2) + qd) * 8 + 4 (ks % 2) + 2e (interleaved 16-byte chunks, as K is read)
              const int dq = ES == 1 ? qd * KB + ks * 4 + e * 2 : ((ks >> 1) * 4 + qd) * 8 + (ks & 1) * 4 + e * 2;
              const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(qh + (size_t)h * D + dq);
              if constexpr (ES == 1) {
                qb[ng][ks][e] =
                    f32x2_to_f16x2(__bfloat162float(v.x) * scale_log2, __bfloat162float(v.y) * scale_log2);
              } else {
                qb[ng][ks][e] = *reinterpret_cast<const uint32_t*>(&v);
              }
            } else {
              qb[ng][ks][e] = 0u;
            }
          }
        }
      }
    }
    float o[KS][NG][4];
#pragma unroll
    for (int mt = 0; mt < KS; ++mt)
#pragma unroll
      for (int ng = 0; ng < NG; ++ng) o[mt][ng][0] = o[mt][ng][1] = o[mt][ng][2] = o[mt][ng][3] = 0.f;
    // running max per head column (2qd, 2qd+1 of each n-tile; equal across the 8 lanes of a column) and the
    // thread's partial row sums (reduced over those lanes at the end)
    float m_r[NG][2], l_r[NG][2];
#pragma unroll
    for (int ng = 0; ng < NG; ++ng) m_r[ng][0] = m_r[ng][1] = -INFINITY, l_r[ng][0] = l_r[ng][1] = 0.f;
    const int krow0 = tok_of_row(gq), krow1 = krow0 + 8;  // tokens of S^T rows gq, gq + 8
    int k = 0;
    for (; k < ntiles; ++k) {
      const int s = k % C::NST;
      if (!snb::mbar_wait_bounded(&full[s], (k / C::NST) & 1, status, SNB_ERR_TIMEOUT_MMA)) {
        sh[2] = 1;
        break;
      }
      const uint8_t* kt = ring + s * C::STAGE + warp * TPW * RB;
      const uint8_t* vt = ring + s * C::STAGE + TILE * RB + warp * TPW * RB;
      const int tw = s0 + k * TILE + warp * TPW;  // first token of this warp's TPW
      const bool whole = tw >= lo && tw + TPW <= s1;
      // K rows krow0 / krow1 of each 16-token block. e4m3: KBB contiguous bytes at qd*KBB. bf16: the thread's
      // 16-byte chunks c sit at (4c + qd) * 16 (interleaved with the other lanes of its row), and lanes of odd
      // gq fetch them in XOR-1 order, then swap back with selects: the two rows a quarter-warp reads land in
      // different banks (256-byte rows all start at bank 0).
      constexpr int NKC = KBB / 16;
      uint32_t kw[U][2][KBB / 4];
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const uint8_t* krow = kt + (u * 16 + (r ? krow1 : krow0)) * RB;
          if constexpr (ES == 1) {
#pragma unroll
            for (int i = 0; i < NKC; ++i) {
              const uint4 a = *reinterpret_cast<const uint4*>(krow + qd * KBB + i * 16);
              kw[u][r][i * 4] = a.x;
              kw[u][r][i * 4 + 1] = a.y;
              kw[u][r][i * 4 + 2] = a.z;
              kw[u][r][i * 4 + 3] = a.w;
            }
          } else {
            const int rot = NKC > 1 ? (gq & 1) : 0;
            uint4 t[NKC];
#pragma unroll
            for (int i = 0; i < NKC; ++i)
              t[i] = *reinterpret_cast<const uint4*>(krow + (((NKC > 1 ? (i ^ rot) : i) * 4 + qd) * 16));
#pragma unroll
            for (int i = 0; i < NKC; ++i) {
              const uint4 a = rot ? t[NKC > 1 ? (i ^ 1) : i] : t[i];
              kw[u][r][i * 4] = a.x;
              kw[u][r][i * 4 + 1] = a.y;
              kw[u][r][i * 4 + 2] = a.z;
              kw[u][r][i * 4 + 3] = a.w;
            }
          }
        }
      // V rows qd + 4i of each block: VBB bytes at gq*VBB; tokens outside [lo, s1) zeroed (stale page bytes)
      uint32_t vw[U][4][VBB / 4];
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = u * 16 + qd + 4 * i;
          const uint8_t* src = vt + row * RB + gq * VBB;
          const bool ok = whole || (tw + row >= lo && tw + row < s1);
          if constexpr (VBB == 8) {
            const uint2 v = *reinterpret_cast<const uint2*>(src);
            vw[u][i][0] = ok ? v.x : 0u;
            vw[u][i][1] = ok ? v.y : 0u;
          } else {
            // two or more chunks: lanes of odd qd fetch them in XOR-1 order (the four rows of a quarter-warp share
            // bank offsets) and swap back with selects
            constexpr int NVC = VBB / 16;
            const int rot = NVC > 1 ? (qd & 1) : 0;
            uint4 t[NVC];
#pragma unroll
            for (int c = 0; c < NVC; ++c) t[c] = reinterpret_cast<const uint4*>(src)[NVC > 1 ? (c ^ rot) : c];
#pragma unroll
            for (int c = 0; c < NVC; ++c) {
              const uint4 v = rot ? t[NVC > 1 ? (c ^ 1) : c] : t[c];
              vw[u][i][c * 4] = ok ? v.x : 0u;
              vw[u][i][c * 4 + 1] = ok ? v.y : 0u;
              vw[u][i][c * 4 + 2] = ok ? v.z : 0u;
              vw[u][i][c * 4 + 3] = ok ? v.w : 0u;
            }
          }
        }
      __syncwarp();
      if (lane == 0) snb::mbar_arrive(&empty[s]);  // this warp's bytes of the stage are in registers
      // ---- S^T = K Q^T: sc[u][ng] rows (krow0, krow1) x heads (2qd, 2qd+1), in log2 units
      float sc[U][NG][4];
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int ng = 0; ng < NG; ++ng) {
          sc[u][ng][0] = sc[u][ng][1] = sc[u][ng][2] = sc[u][ng][3] = 0.f;
#pragma unroll
          for (int ks = 0; ks < KS; ++ks) {
            if constexpr (ES == 1) {
              const uint32_t w0 = kw[u][0][ks], w1 = kw[u][1][ks];
              const uint32_t a[4] = {e4m3x2_to_f16x2(w0), e4m3x2_to_f16x2(w1), e4m3x2_hi_to_f16x2(w0),
                                     e4m3x2_hi_to_f16x2(w1)};
              mma_f16_16816(sc[u][ng], a, qb[ng][ks][0], qb[ng][ks][1]);
            } else {
              const uint32_t a[4] = {kw[u][0][2 * ks], kw[u][1][2 * ks], kw[u][0][2 * ks + 1], kw[u][1][2 * ks + 1]};
              mma_bf16_16816(sc[u][ng], a, qb[ng][ks][0], qb[ng][ks][1]);
            }
          }
          if constexpr (ES == 2) {
#pragma unroll
            for (int j = 0; j < 4; ++j) sc[u][ng][j] *= scale_log2;
          }
        }
      if (!whole) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int t0 = tw + u * 16 + krow0, t1 = t0 + 8;
          const bool ok0 = t0 >= lo && t0 < s1, ok1 = t1 >= lo && t1 < s1;
#pragma unroll
          for (int ng = 0; ng < NG; ++ng) {
            if (!ok0) sc[u][ng][0] = sc[u][ng][1] = -INFINITY;
            if (!ok1) sc[u][ng][2] = sc[u][ng][3] = -INFINITY;
          }
        }
      }
      // ---- online softmax per head column over the warp's TPW tokens
      bool moved = false;
      float alpha[NG][2];
#pragma unroll
      for (int ng = 0; ng < NG; ++ng)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          float mx = -INFINITY;
#pragma unroll
          for (int u = 0; u < U; ++u) mx = fmaxf(mx, fmaxf(sc[u][ng][j], sc[u][ng][2 + j]));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
          const float mn = fmaxf(m_r[ng][j], mx);
          alpha[ng][j] = (mn == m_r[ng][j]) ? 1.f : ex2_approx(m_r[ng][j] - mn);
          moved |= mn != m_r[ng][j];
          m_r[ng][j] = mn;
          l_r[ng][j] *= alpha[ng][j];
        }
      // P^T as the B operand of O^T = V^T P^T: pack a row's two head columns, transpose each 8x8 block
      uint32_t pb[U][NG][2];
#pragma unroll
      for (int ng = 0; ng < NG; ++ng) {
        const float r0 = m_r[ng][0] == -INFINITY ? 0.f : m_r[ng][0];
        const float r1 = m_r[ng][1] == -INFINITY ? 0.f : m_r[ng][1];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const float p0 = ex2_approx(sc[u][ng][0] - r0), p1 = ex2_approx(sc[u][ng][1] - r1);
          const float p2 = ex2_approx(sc[u][ng][2] - r0), p3 = ex2_approx(sc[u][ng][3] - r1);
          l_r[ng][0] += p0 + p2;
          l_r[ng][1] += p1 + p3;
          if constexpr (ES == 1) {
            pb[u][ng][0] = movmatrix_trans(f32x2_to_f16x2(p0, p1));
            pb[u][ng][1] = movmatrix_trans(f32x2_to_f16x2(p2, p3));
          } else {
            pb[u][ng][0] = movmatrix_trans(f32x2_to_bf16x2(p0, p1));
            pb[u][ng][1] = movmatrix_trans(f32x2_to_bf16x2(p2, p3));
          }
        }
      }
      if (__any_sync(0xffffffffu, moved)) {
#pragma unroll
        for (int mt = 0; mt < KS; ++mt)
#pragma unroll
          for (int ng = 0; ng < NG; ++ng) {
            o[mt][ng][0] *= alpha[ng][0];
            o[mt][ng][1] *= alpha[ng][1];
            o[mt][ng][2] *= alpha[ng][0];
            o[mt][ng][3] *= alpha[ng][1];
          }
      }
      // ---- O^T += V^T P^T: A rows are head dims (element 2mt + h of the thread's V slice), k = tokens
      // qd, qd+4 | qd+8, qd+12 of each 16-token block; one permute gathers both dims of a token pair
#pragma unroll
      for (int mt = 0; mt < KS; ++mt) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
          if constexpr (ES == 1) {
            const int w = mt >> 1;
            const uint32_t sel = (mt & 1) ? 0x7362u : 0x5140u;
            const uint32_t p01 = __byte_perm(vw[u][0][w], vw[u][1][w], sel);
            const uint32_t p23 = __byte_perm(vw[u][2][w], vw[u][3][w], sel);
            const uint32_t a[4] = {e4m3x2_to_f16x2(p01), e4m3x2_hi_to_f16x2(p01), e4m3x2_to_f16x2(p23),
                                   e4m3x2_hi_to_f16x2(p23)};
#pragma unroll
            for (int ng = 0; ng < NG; ++ng) mma_f16_16816(o[mt][ng], a, pb[u][ng][0], pb[u][ng][1]);
          } else {
            // bf16: word mt of the slice holds dims 2mt (low half) and 2mt + 1 (high half)
            const uint32_t x0 = vw[u][0][mt], x1 = vw[u][1][mt], x2 = vw[u][2][mt], x3 = vw[u][3][mt];
            const uint32_t a[4] = {__byte_perm(x0, x1, 0x5410u), __byte_perm(x0, x1, 0x7632u),
                                   __byte_perm(x2, x3, 0x5410u), __byte_perm(x2, x3, 0x7632u)};
#pragma unroll
            for (int ng = 0; ng < NG; ++ng) mma_bf16_16816(o[mt][ng], a, pb[u][ng][0], pb[u][ng][1]);
          }
        }
      }
    }
    if (warp == 0 && lane == 0) sh[1] = k;
#pragma unroll
    for (int ng = 0; ng < NG; ++ng)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        l_r[ng][j] += __shfl_xor_sync(0xffffffffu, l_r[ng][j], 4);
        l_r[ng][j] += __shfl_xor_sync(0xffffffffu, l_r[ng][j], 8);
        l_r[ng][j] += __shfl_xor_sync(0xffffffffu, l_r[ng][j], 16);
      }
    // ---- per-warp state to shared memory for the merge (after every compute warp left the ring)
    __syncwarp();
    asm volatile("bar.sync 1, %0;" ::"n"(kCWarps * 32) : "memory");
    float* obuf = reinterpret_cast<float*>(ring);
    if (gq == 0) {
#pragma unroll
      for (int ng = 0; ng < NG; ++ng)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          red_m[warp * 16 + ng * 8 + 2 * qd + j] = m_r[ng][j];
          red_l[warp * 16 + ng * 8 + 2 * qd + j] = l_r[ng][j];
        }
    }
#pragma unroll
    for (int mt = 0; mt < KS; ++mt)
#pragma unroll
      for (int ng = 0; ng < NG; ++ng)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int h = ng * 8 + 2 * qd + (e & 1), d = gq * VB + 2 * mt + (e >> 1);
          obuf[(warp * 16 + h) * D + d] = o[mt][ng][e];
        }
  }
  __syncthreads();
  decode_fp8_finish<D>(warp, tid, lane, b, hk, split, Hkv, G, num_splits, sinks, v_scale, out, out_stride, o_part,
                       lse_part, red_m, red_l, reinterpret_cast<const float*>(ring), sh, full, C::NST, status,
                       merge_cnt, v_scale_out);
}

}  // namespace

// Opt a kernel into its dynamic shared memory once (one static per kernel) and return the size.
template <typename Cfg, auto Kern>
static int fp8_smem_attr() {
  static bool done = false;
  if (!done) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    done = true;
  }
  return Cfg::SMEM;
}

// Which kernel serves a call: 1 (default) the token-major kernel fed by bulk copies, 2 the token-major kernel
// fed by 16-byte cp.async, 0 the head-major kernel for an e4m3 cache and the register-prefetch kernel
// (attention_decode_mma.cu) for a bf16 cache. Page sizes that do not tile the token-major stage fall back the
// same way. Tests and the attention microbenchmark compare them.
static int g_fp8_decode_variant = 1;

void set_decode_fp8_variant(int64_t v) {
  TORCH_CHECK(v >= 0 && v <= 2, "set_decode_fp8_variant: 0 (head-major), 1 or 2 (token-major)");
  g_fp8_decode_variant = (int)v;
}

template <int D, int NG, typename CT>
static bool tok_tiles(int64_t page_size) {
  constexpr int T = TokCfg<D, NG, CT>::TILE;
  return (page_size >= 16 && T % page_size == 0) || (page_size >= T && page_size % T == 0);
}

// Same contract as decode_attention_mma() for an e4m3 or bf16 cache, served by the pipelined tensor-core
// kernels of this file; false when not covered (head_dim not 64/128, G > 16, a page size that tiles neither
// stage, or a bf16 cache with the token-major kernel switched off). With merge_cnt (zeroed int32 per
// (request, KV head)) and more than one split, the split merge runs inside this launch (v_scale_out is applied
// there) and no merge kernel follows.
bool decode_attention_pipelined(torch::Tensor out, torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                                torch::Tensor block_table, torch::Tensor seq_lens, int64_t num_q_heads,
                                int64_t num_kv_heads, int64_t head_dim, int64_t page_size, int64_t window,
                                float scale_log2, float v_scale_final, const float* sinks, int64_t num_splits,
                                float* o_part, float* lse_part, int* status, int* merge_cnt, float v_scale_out) {
  const int G = num_q_heads / num_kv_heads;
  const bool fp8 = k_cache.scalar_type() == at::kFloat8_e4m3fn;
  const bool bf16 = k_cache.scalar_type() == at::kBFloat16;
  if (!(fp8 || bf16) || G > 16 || (head_dim != 64 && head_dim != 128)) return false;
  if (k_cache.data_ptr() == nullptr || reinterpret_cast<uintptr_t>(k_cache.data_ptr()) % 16 ||
      reinterpret_cast<uintptr_t>(v_cache.data_ptr()) % 16 || !k_cache.is_contiguous() || !v_cache.is_contiguous())
    return false;
  const bool head_major_ok =
      fp8 && ((page_size >= 16 && kTile % page_size == 0) || (page_size >= kTile && page_size % kTile == 0));
  const bool tok = g_fp8_decode_variant != 0 &&
                   (fp8 ? tok_tiles<64, 1, uint8_t>(page_size) : tok_tiles<64, 1, __nv_bfloat16>(page_size));
  if (!tok && !head_major_ok) return false;
  const int B = q.size(0);
  auto st = at::cuda::getCurrentCUDAStream();
  dim3 grid(num_splits, num_kv_heads, B);
  auto launch = [&](auto kernel, int smem, auto* elem) {
    using E = std::remove_pointer_t<decltype(elem)>;
    C10_CUDA_CHECK(snb::launch_pdl(kernel, grid, kThreads, smem, st, (const __nv_bfloat16*)q.data_ptr(),
                                   (int)q.stride(0), (const E*)k_cache.data_ptr(), (const E*)v_cache.data_ptr(),
                                   block_table.data_ptr<int32_t>(), (int)block_table.stride(0),
                                   seq_lens.data_ptr<int32_t>(), (int)page_size, (int)num_kv_heads, G, (int)window,
                                   scale_log2, v_scale_final, sinks, (__nv_bfloat16*)out.data_ptr(),
                                   (int)out.stride(0), o_part, lse_part, (int)num_splits, status, merge_cnt,
                                   v_scale_out));
  };
  const bool bulk = g_fp8_decode_variant == 1;
#define SNB_TOK(DD, NGG, BB, CT) launch(decode_attn_tok_kernel<DD, NGG, BB, CT>,                              \
                                        fp8_smem_attr<TokCfg<DD, NGG, CT>, decode_attn_tok_kernel<DD, NGG, BB, CT>>(), \
                                        (CT*)nullptr)
#define SNB_TOK_D(DD, CT)                                                                                   \
  {                                                                                                         \
    if (G <= 8) { if (bulk) SNB_TOK(DD, 1, true, CT); else SNB_TOK(DD, 1, false, CT); }                     \
    else { if (bulk) SNB_TOK(DD, 2, true, CT); else SNB_TOK(DD, 2, false, CT); }                            \
  }
  if (tok) {
    if (fp8) {
      if (head_dim == 64) SNB_TOK_D(64, uint8_t) else SNB_TOK_D(128, uint8_t)
    } else {
      if (head_dim == 64) SNB_TOK_D(64, __nv_bfloat16) else SNB_TOK_D(128, __nv_bfloat16)
    }
  } else if (head_dim == 64) {
    launch(decode_attn_fp8_kernel<64>, fp8_smem_attr<Fp8Cfg<64>, decode_attn_fp8_kernel<64>>(), (uint8_t*)nullptr);
  } else {
    launch(decode_attn_fp8_kernel<128>, fp8_smem_attr<Fp8Cfg<128>, decode_attn_fp8_kernel<128>>(), (uint8_t*)nullptr);
  }
#undef SNB_TOK_D
#undef SNB_TOK
  return true;
}
