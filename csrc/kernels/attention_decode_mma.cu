// Paged GQA decode attention on tensor cores (mma.sync m16n8k16, bf16 in, fp32 accumulate).
//
// The G query heads that share one KV head form the M=16 rows of the MMA (zero rows above G), the
// context tokens form N (scores) and K (probabilities x values). Per CTA: one request, one KV head, one
// split of the (windowed) context; 4 warps each own 16 tokens of every 64-token tile and keep their own
// online-softmax state, merged through shared memory at the end. K/V tiles are read straight from the
// paged pool (fp8-e4m3 or bf16), the next tile's raw bytes are fetched into registers while the current
// tile is being multiplied, converted to bf16 and staged as K[token][d] and V^T[d][token] so every MMA
// operand is one 32-bit shared load. Decode has only G <= 16 query rows per KV head, which is below the
// 64/128-row minimum of tcgen05 tiles; the warp-level MMA keeps the kernel bound by KV bytes instead.
//
// Parity: the reference's attention_decode / attention_decode_paged ops (sglang_neuron/ops/attention/
// attention_decode.py:28-205) with learned sinks, sliding window and FP8 KV.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "../common.cuh"

namespace {

constexpr float kL2e = 1.4426950408889634f;
constexpr int kT = 64;        // tokens per CTA tile
constexpr int kWarps = 4;     // 16 tokens per warp per tile
constexpr int kThr = kWarps * 32;

SNB_DEVICE void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

SNB_DEVICE uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Raw bytes of one half row (D/2 values) of K and of V for one token.
template <int D, typename CacheT>
struct RowRegs {
  static constexpr int BYTES = (D / 2) * (int)sizeof(CacheT);
  static constexpr int VEC = BYTES / 16;
  uint4 k[VEC];
  uint4 v[VEC];
};

template <int D, typename CacheT>
SNB_DEVICE void fetch_half_row(RowRegs<D, CacheT>& r, const CacheT* kc, const CacheT* vc, const int32_t* bt,
                               int tok, int end, int page_size, int Hkv, int hk, int half) {
  if (tok < end) {
    const size_t off = (((size_t)bt[tok / page_size] * Hkv + hk) * page_size + tok % page_size) * D + half * (D / 2);
    const uint4* kp = reinterpret_cast<const uint4*>(kc + off);
    const uint4* vp = reinterpret_cast<const uint4*>(vc + off);
#pragma unroll
    for (int i = 0; i < RowRegs<D, CacheT>::VEC; ++i) {
      r.k[i] = kp[i];
      r.v[i] = vp[i];
    }
  } else {
#pragma unroll
    for (int i = 0; i < RowRegs<D, CacheT>::VEC; ++i) r.k[i] = r.v[i] = make_uint4(0, 0, 0, 0);
  }
}

// Convert the fetched half row to bf16 and stage it: K as [token][d], V transposed as [d][token].
template <int D, typename CacheT>
SNB_DEVICE void stage_half_row(const RowRegs<D, CacheT>& r, __nv_bfloat16* ks, __nv_bfloat16* vts, int row,
                               int half) {
  constexpr int KS = D + 8, VS = kT + 8;
  __nv_bfloat16* kd = ks + row * KS + half * (D / 2);
  if constexpr (sizeof(CacheT) == 2) {
#pragma unroll
    for (int i = 0; i < RowRegs<D, CacheT>::VEC; ++i) reinterpret_cast<uint4*>(kd)[i] = r.k[i];
#pragma unroll
    for (int i = 0; i < RowRegs<D, CacheT>::VEC; ++i) {
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&r.v[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) vts[(half * (D / 2) + i * 8 + j) * VS + row] = e[j];
    }
  } else {
#pragma unroll
    for (int i = 0; i < RowRegs<D, CacheT>::VEC; ++i) {
      const uint8_t* kb = reinterpret_cast<const uint8_t*>(&r.k[i]);
      const uint8_t* vb = reinterpret_cast<const uint8_t*>(&r.v[i]);
      float f[8];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] = snb::fp8e4m3_to_f(kb[h * 8 + j]);
        reinterpret_cast<uint4*>(kd)[i * 2 + h] = snb::pack_bf16x8(f);
      }
#pragma unroll
      for (int j = 0; j < 16; ++j)
        vts[(half * (D / 2) + i * 16 + j) * VS + row] = __float2bfloat16(snb::fp8e4m3_to_f(vb[j]));
    }
  }
}

template <int D, typename CacheT>
__global__ void __launch_bounds__(kThr) decode_attn_mma_kernel(
    const __nv_bfloat16* __restrict__ q, int q_stride, const CacheT* __restrict__ kc, const CacheT* __restrict__ vc,
    const int32_t* __restrict__ block_table, int bt_stride, const int32_t* __restrict__ seq_lens, int page_size,
    int Hkv, int G, int window, float scale_log2, float v_scale, const float* __restrict__ sinks,
    __nv_bfloat16* __restrict__ out, int out_stride, float* __restrict__ o_part, float* __restrict__ lse_part,
    int num_splits) {
  snb::pdl_wait();
  snb::pdl_trigger();
  constexpr int KS = D + 8, VS = kT + 8;
  constexpr int NT = D / 8;  // n8 tiles of the output
  // one buffer: K tile [kT][KS] then V^T tile [D][VS]; reused as the fp32 merge area after the loop
  constexpr int KV_ELEMS = kT * KS + D * VS;
  static_assert(kWarps * 16 * D * 4 <= KV_ELEMS * 2, "merge buffer does not fit in the staging area");
  __shared__ __align__(16) __nv_bfloat16 kv_smem[KV_ELEMS];
  __nv_bfloat16* ks = kv_smem;
  __nv_bfloat16* vts = kv_smem + kT * KS;
  __shared__ float red_m[kWarps][16], red_l[kWarps][16];

  const int split = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, qd = lane & 3;
  const int ctx = seq_lens[b];
  const int start = (window > 0 && ctx > window) ? ctx - window : 0;
  const int per = ((ctx - start + num_splits - 1) / num_splits + kT - 1) / kT * kT;
  const int s0 = start + split * per;
  const int s1 = min(ctx, s0 + per);
  const int32_t* bt = block_table + (size_t)b * bt_stride;

  // Q fragments (A operand) for all D/16 k-steps; rows >= G are zero.
  uint32_t qa[D / 16][4];
  {
    const __nv_bfloat16* qb = q + (size_t)b * q_stride + (size_t)hk * G * D;
#pragma unroll
    for (int ks_ = 0; ks_ < D / 16; ++ks_) {
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int row = gq + (r & 1) * 8;
        const int col = ks_ * 16 + qd * 2 + (r >> 1) * 8;
        qa[ks_][r] = row < G ? *reinterpret_cast<const uint32_t*>(qb + (size_t)row * D + col) : 0u;
      }
    }
  }
  float o[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};

  // staging assignment: thread -> (token row, half of D)
  const int srow = tid >> 1, shalf = tid & 1;
  RowRegs<D, CacheT> regs;
  if (s0 < s1) {
    fetch_half_row<D, CacheT>(regs, kc, vc, bt, s0 + srow, s1, page_size, Hkv, hk, shalf);
    stage_half_row<D, CacheT>(regs, ks, vts, srow, shalf);
  }
  __syncthreads();
  for (int t0 = s0; t0 < s1; t0 += kT) {
    const bool more = t0 + kT < s1;
    if (more) fetch_half_row<D, CacheT>(regs, kc, vc, bt, t0 + kT + srow, s1, page_size, Hkv, hk, shalf);
    // ---- S = Q K^T for this warp's 16 tokens (two n8 tiles)
    float s[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
      const int tok = warp * 16 + nt * 8 + gq;
#pragma unroll
      for (int ks_ = 0; ks_ < D / 16; ++ks_) {
        const __nv_bfloat16* kr = ks + tok * KS + ks_ * 16 + qd * 2;
        mma_bf16_16816(s[nt], qa[ks_], *reinterpret_cast<const uint32_t*>(kr),
                       *reinterpret_cast<const uint32_t*>(kr + 8));
      }
    }
    // ---- online softmax (rows gq and gq + 8), masking tokens past the split end
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int tok = t0 + warp * 16 + nt * 8 + qd * 2 + (j & 1);
        float v = s[nt][j] * scale_log2;
        if (tok >= s1) v = -INFINITY;
        s[nt][j] = v;
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
        const float mref = m_r[j >> 1];
        const float p = (s[nt][j] == -INFINITY) ? 0.f : exp2f(s[nt][j] - mref);
        s[nt][j] = p;
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
    // ---- O += P V: P (16 rows x this warp's 16 tokens) is the A operand of one k16 step
    uint32_t pa[4];
    pa[0] = pack_bf16x2(s[0][0], s[0][1]);
    pa[1] = pack_bf16x2(s[0][2], s[0][3]);
    pa[2] = pack_bf16x2(s[1][0], s[1][1]);
    pa[3] = pack_bf16x2(s[1][2], s[1][3]);
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const __nv_bfloat16* vr = vts + (n * 8 + gq) * VS + warp * 16 + qd * 2;
      mma_bf16_16816(o[n], pa, *reinterpret_cast<const uint32_t*>(vr), *reinterpret_cast<const uint32_t*>(vr + 8));
    }
    __syncthreads();
    if (more) {
      stage_half_row<D, CacheT>(regs, ks, vts, srow, shalf);
      __syncthreads();
    }
  }

  // ---- merge the 4 warps' partial states through shared memory (reusing the K/V staging area)
  float* obuf = reinterpret_cast<float*>(kv_smem);  // [warps][16][D]
  __syncthreads();
  if (qd == 0) {
    red_m[warp][gq] = m_r[0];
    red_m[warp][gq + 8] = m_r[1];
    red_l[warp][gq] = l_r[0];
    red_l[warp][gq + 8] = l_r[1];
  }
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    const int col = n * 8 + qd * 2;
    obuf[(warp * 16 + gq) * D + col] = o[n][0];
    obuf[(warp * 16 + gq) * D + col + 1] = o[n][1];
    obuf[(warp * 16 + gq + 8) * D + col] = o[n][2];
    obuf[(warp * 16 + gq + 8) * D + col + 1] = o[n][3];
  }
  __syncthreads();
  const int Hq = Hkv * G;
  for (int idx = tid; idx < G * D; idx += kThr) {
    const int g = idx / D, d = idx % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, red_m[w][g]);
    float L = 0.f, acc = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      if (red_m[w][g] == -INFINITY) continue;
      const float f = exp2f(red_m[w][g] - M);
      L += red_l[w][g] * f;
      acc += obuf[(w * 16 + g) * D + d] * f;
    }
    const int h = hk * G + g;
    if (num_splits == 1) {
      float denom = L;
      if (sinks != nullptr) denom = (M == -INFINITY) ? 1.f : L + exp2f(sinks[h] * kL2e - M);
      out[(size_t)b * out_stride + (size_t)h * D + d] = __float2bfloat16(denom > 0.f ? acc / denom * v_scale : 0.f);
    } else {
      const size_t pidx = ((size_t)b * Hq + h) * num_splits + split;
      o_part[pidx * D + d] = L > 0.f ? acc / L : 0.f;
      if (d == 0) lse_part[pidx] = L > 0.f ? M + log2f(L) : -INFINITY;
    }
  }
}

// ---------------------------------------------------------------------------------------------------
// Extend (prefill over a paged prior) on tensor cores. Grid (ceil(max_extend / 64), B, Hq), 128 threads:
// each warp owns 16 query rows of one query head; K/V tiles of 64 tokens are staged as in decode (the
// G heads of a KV head re-read the same tile through L2). Causal + sliding-window masks come from the
// query and key positions; sinks join the final normaliser.
// ---------------------------------------------------------------------------------------------------
template <int D, typename CacheT>
__global__ void __launch_bounds__(kThr) extend_attn_mma_kernel(
    const __nv_bfloat16* __restrict__ q, int q_stride, const CacheT* __restrict__ kc, const CacheT* __restrict__ vc,
    const int32_t* __restrict__ block_table, int bt_stride, const int32_t* __restrict__ qo_indptr,
    const int32_t* __restrict__ kv_lens, int page_size, int Hkv, int G, int window, float scale_log2, float v_scale,
    const float* __restrict__ sinks, __nv_bfloat16* __restrict__ out, int out_stride) {
  snb::pdl_wait();
  snb::pdl_trigger();
  constexpr int KS = D + 8, VS = kT + 8;
  constexpr int NT = D / 8;
  constexpr int KV_ELEMS = kT * KS + D * VS;
  __shared__ __align__(16) __nv_bfloat16 kv_smem[KV_ELEMS];
  __nv_bfloat16* ks = kv_smem;
  __nv_bfloat16* vts = kv_smem + kT * KS;

  const int b = blockIdx.y, h = blockIdx.z, hk = h / G;
  const int q_begin = qo_indptr[b], ext = qo_indptr[b + 1] - q_begin;
  const int qi0 = blockIdx.x * (kWarps * 16);
  if (qi0 >= ext) return;
  const int kv_len = kv_lens[b];
  const int prefix = kv_len - ext;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, qd = lane & 3;
  const int row0 = qi0 + warp * 16;  // first query index of this warp
  // positions of this thread's two rows
  const int qa_i = row0 + gq, qb_i = row0 + gq + 8;
  const int pos_a = prefix + qa_i, pos_b = prefix + qb_i;
  const bool va = qa_i < ext, vb = qb_i < ext;

  uint32_t qf[D / 16][4];
#pragma unroll
  for (int ks_ = 0; ks_ < D / 16; ++ks_) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int qi = row0 + gq + (r & 1) * 8;
      const int col = ks_ * 16 + qd * 2 + (r >> 1) * 8;
      qf[ks_][r] = qi < ext ? *reinterpret_cast<const uint32_t*>(q + (size_t)(q_begin + qi) * q_stride +
                                                                   (size_t)h * D + col)
                            : 0u;
    }
  }
  float o[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};

  // key range needed by the CTA's queries
  const int last_q = min(ext, qi0 + kWarps * 16) - 1;
  const int hi = prefix + last_q + 1;
  int lo = 0;
  if (window > 0) lo = max(0, prefix + qi0 - window + 1);
  lo = (lo / kT) * kT;
  const int32_t* bt = block_table + (size_t)b * bt_stride;
  const int srow = tid >> 1, shalf = tid & 1;
  RowRegs<D, CacheT> regs;
  fetch_half_row<D, CacheT>(regs, kc, vc, bt, lo + srow, hi, page_size, Hkv, hk, shalf);
  stage_half_row<D, CacheT>(regs, ks, vts, srow, shalf);
  __syncthreads();
  for (int t0 = lo; t0 < hi; t0 += kT) {
    const bool more = t0 + kT < hi;
    if (more) fetch_half_row<D, CacheT>(regs, kc, vc, bt, t0 + kT + srow, hi, page_size, Hkv, hk, shalf);
    // S = Q K^T over the 64 tile tokens: 8 n8 tiles
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
      for (int ks_ = 0; ks_ < D / 16; ++ks_) {
        const __nv_bfloat16* kr = ks + (nt * 8 + gq) * KS + ks_ * 16 + qd * 2;
        mma_bf16_16816(s[nt], qf[ks_], *reinterpret_cast<const uint32_t*>(kr),
                       *reinterpret_cast<const uint32_t*>(kr + 8));
      }
    }
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int kp = t0 + nt * 8 + qd * 2 + (j & 1);
        const int pos = (j >> 1) ? pos_b : pos_a;
        const bool valid = (j >> 1) ? vb : va;
        bool ok = valid && kp < hi && kp <= pos;
        if (window > 0) ok = ok && (pos - kp < window);
        const float v = ok ? s[nt][j] * scale_log2 : -INFINITY;
        s[nt][j] = v;
        mx[j >> 1] = fmaxf(mx[j >> 1], v);
      }
    }
    float alpha[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      mx[hh] = fmaxf(mx[hh], __shfl_xor_sync(0xffffffffu, mx[hh], 1));
      mx[hh] = fmaxf(mx[hh], __shfl_xor_sync(0xffffffffu, mx[hh], 2));
      const float mn = fmaxf(m_r[hh], mx[hh]);
      alpha[hh] = (m_r[hh] == -INFINITY) ? (mn == -INFINITY ? 1.f : 0.f) : exp2f(m_r[hh] - mn);
      m_r[hh] = mn;
    }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float p = (s[nt][j] == -INFINITY) ? 0.f : exp2f(s[nt][j] - m_r[j >> 1]);
        s[nt][j] = p;
        rs[j >> 1] += p;
      }
    }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      rs[hh] += __shfl_xor_sync(0xffffffffu, rs[hh], 1);
      rs[hh] += __shfl_xor_sync(0xffffffffu, rs[hh], 2);
      l_r[hh] = l_r[hh] * alpha[hh] + rs[hh];
    }
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      o[n][0] *= alpha[0];
      o[n][1] *= alpha[0];
      o[n][2] *= alpha[1];
      o[n][3] *= alpha[1];
    }
    // O += P V over 4 k16 steps of 16 tokens
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const __nv_bfloat16* vr = vts + (n * 8 + gq) * VS + kk * 16 + qd * 2;
        mma_bf16_16816(o[n], pa, *reinterpret_cast<const uint32_t*>(vr), *reinterpret_cast<const uint32_t*>(vr + 8));
      }
    }
    __syncthreads();
    if (more) {
      stage_half_row<D, CacheT>(regs, ks, vts, srow, shalf);
      __syncthreads();
    }
  }
  // finalise the two rows of this thread
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int qi = hh ? qb_i : qa_i;
    if (qi >= ext) continue;
    float denom = l_r[hh];
    if (sinks != nullptr) denom = (m_r[hh] == -INFINITY) ? 1.f : denom + exp2f(sinks[h] * kL2e - m_r[hh]);
    const float inv = denom > 0.f ? v_scale / denom : 0.f;
    __nv_bfloat16* orow = out + (size_t)(q_begin + qi) * out_stride + (size_t)h * D;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const int col = n * 8 + qd * 2;
      *reinterpret_cast<uint32_t*>(orow + col) = pack_bf16x2(o[n][hh * 2] * inv, o[n][hh * 2 + 1] * inv);
    }
  }
}

}  // namespace

// Same contract as decode_attention() in attention.cu; returns false when the shape is not covered
// (G > 16 or head_dim not in {64, 128}) so the caller can use the CUDA-core kernel.
bool decode_attention_mma(torch::Tensor out, torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                          torch::Tensor block_table, torch::Tensor seq_lens, int64_t num_q_heads, int64_t num_kv_heads,
                          int64_t head_dim, int64_t page_size, int64_t window, float scale_log2, float v_scale_final,
                          const float* sinks, int64_t num_splits, float* o_part, float* lse_part) {
  const int G = num_q_heads / num_kv_heads;
  if (G > 16 || (head_dim != 64 && head_dim != 128)) return false;
  const int B = q.size(0);
  auto st = at::cuda::getCurrentCUDAStream();
  dim3 grid(num_splits, num_kv_heads, B);
  const bool fp8 = k_cache.scalar_type() == at::kFloat8_e4m3fn;
#define SNB_MMA(DD, CT)                                                                                          \
  snb::launch_pdl(decode_attn_mma_kernel<DD, CT>, grid, kThr, 0, st,                                                          \
      (const __nv_bfloat16*)q.data_ptr(), q.stride(0), (const CT*)k_cache.data_ptr(), (const CT*)v_cache.data_ptr(), \
      block_table.data_ptr<int32_t>(), block_table.stride(0), seq_lens.data_ptr<int32_t>(), page_size,          \
      num_kv_heads, G, window, scale_log2, v_scale_final, sinks, (__nv_bfloat16*)out.data_ptr(), out.stride(0),   \
      o_part, lse_part, num_splits)
  if (head_dim == 64) {
    if (fp8) SNB_MMA(64, uint8_t); else SNB_MMA(64, __nv_bfloat16);
  } else {
    if (fp8) SNB_MMA(128, uint8_t); else SNB_MMA(128, __nv_bfloat16);
  }
#undef SNB_MMA
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return true;
}

// Extend attention on tensor cores; false when the shape is not covered (head_dim not 64/128).
bool extend_attention_mma(torch::Tensor out, torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                          torch::Tensor block_table, torch::Tensor qo_indptr, torch::Tensor kv_lens, int64_t max_extend,
                          int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim, int64_t page_size, int64_t window,
                          float scale_log2, float v_scale, const float* sinks) {
  if (head_dim != 64 && head_dim != 128) return false;
  const int B = kv_lens.size(0);
  const int G = num_q_heads / num_kv_heads;
  auto st = at::cuda::getCurrentCUDAStream();
  dim3 grid((max_extend + kWarps * 16 - 1) / (kWarps * 16), B, num_q_heads);
  const bool fp8 = k_cache.scalar_type() == at::kFloat8_e4m3fn;
#define SNB_EXT_MMA(DD, CT)                                                                                       \
  snb::launch_pdl(extend_attn_mma_kernel<DD, CT>, grid, kThr, 0, st,                                                          \
      (const __nv_bfloat16*)q.data_ptr(), q.stride(0), (const CT*)k_cache.data_ptr(), (const CT*)v_cache.data_ptr(), \
      block_table.data_ptr<int32_t>(), block_table.stride(0), qo_indptr.data_ptr<int32_t>(),                     \
      kv_lens.data_ptr<int32_t>(), page_size, num_kv_heads, G, window, scale_log2, v_scale, sinks,               \
      (__nv_bfloat16*)out.data_ptr(), out.stride(0))
  if (head_dim == 64) {
    if (fp8) SNB_EXT_MMA(64, uint8_t); else SNB_EXT_MMA(64, __nv_bfloat16);
  } else {
    if (fp8) SNB_EXT_MMA(128, uint8_t); else SNB_EXT_MMA(128, __nv_bfloat16);
  }
#undef SNB_EXT_MMA
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return true;
}
