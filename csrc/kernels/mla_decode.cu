// Absorbed multi-head latent attention (MLA) decode over the paged latent pool, on tensor cores.
//
// Every head of a request attends the same latent rows: row = [kv_lora (512) || rope key (64)] bf16, score =
// q_row . row (576 wide, q = [q_nope W_UK || rope(q_pe)]), value = the first 512 values of the row. CTA = one
// (context split, group of up to 16 heads, request); the heads are the 16 M rows of mma.sync m16n8k16.
// Tiles of 32 tokens are copied with cp.async into padded shared-memory rows (576 + 8 bf16: the B-fragment
// loads of 8 rows hit 32 different banks) two tiles ahead; page ids of the split are staged first.
// Per tile: the 4 warps split the 576-wide contraction (9 k16 steps each) over the tile's 4 n8 tiles and
// sum their partial scores through shared memory; 128 threads run the online softmax (8 per head row,
// shuffle reductions) and publish P (bf16) and the rescale factor; each warp then owns 128 of the 512 value
// columns and accumulates P V. Splits write normalised partials + log-sum-exp, merged by a second kernel.
//
// Extend (prefill / chunked prefill, `qo_indptr` given): the 16 M rows of a CTA are 16 consecutive
// (query token, head) pairs of one request (token-major), each with its own causal limit prefix + t + 1;
// the CTA walks the context up to its last row's limit. One query token per request with all its heads is
// the decode case, so both share the tile pipeline. Extend CTAs run two such groups of 16 rows (8 warps) over
// one latent-tile pipeline, so each tile is read once for 32 rows.
//
// Decode context parallelism (dcp_size D > 1): logical page j of a request lives on DCP rank j % D, and the
// block table given here lists only this rank's pages (local page i = logical page i * D + dcp_rank). Keys
// are walked in that local order; causal limits are compared against each key's logical position. With
// `lse_out` the kernel also writes each row's log2-sum-exp, so the D ranks' partials can be merged.
//
// Parity: the reference's `paged_absorbed_mla` decode (sglang_neuron/nki/deepseek_mla_decode.py:510:
// 128-token tiles, online softmax, direct slot addressing) and its torch twin (ops/attention/mla.py:32).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "../common.cuh"

namespace {

constexpr int DK = 576, DV = 512;
constexpr int TT = 32;              // tokens per tile
constexpr int RSK = DK + 8;         // padded shared row (bf16)
constexpr int RSP = TT + 8;         // padded P row (bf16)
constexpr int kThr = 128;
constexpr int kMaxSplitPages = 1024;
constexpr float kLog2e = 1.4426950408889634f;
constexpr int SMEM_K = 2 * TT * RSK * 2;           // two stages
constexpr int SMEM_SP = 4 * 16 * TT * 4;           // partial scores per warp
constexpr int SMEM_P = 16 * RSP * 2;
// MT row groups of 16 per CTA (4 warps each) share one latent-tile pipeline: decode uses one group (the heads
// of a token), extend two (each latent tile is read once for 32 (token, head) rows)
template <int MT>
struct MlaCfg {
  static constexpr int THR = kThr * MT;
  static constexpr int SMEM = SMEM_K + MT * (SMEM_SP + SMEM_P + 4 * 16 * 4) + kMaxSplitPages * 4;
};

SNB_DEVICE void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

SNB_DEVICE void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
SNB_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// four 8x8 b16 matrices, each transposed: with row-major [k][n] tiles in shared memory the results are the
// col-major B fragments of mma.m16n8k16 (matrix i from the row addresses of lanes 8i .. 8i+7)
SNB_DEVICE void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}
template <int N>
SNB_DEVICE void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int MT>
__global__ void __launch_bounds__(kThr * MT) mla_decode_kernel(
    const __nv_bfloat16* __restrict__ q, int q_stride, const __nv_bfloat16* __restrict__ cache,
    const int32_t* __restrict__ block_table, int bt_stride, const int32_t* __restrict__ seq_lens, int page_size,
    int H, float scale_log2, __nv_bfloat16* __restrict__ out, int out_stride, float* __restrict__ o_part,
    float* __restrict__ lse_part, int num_splits, const int32_t* __restrict__ qo_indptr, int dcp_size, int dcp_rank,
    float* __restrict__ lse_out) {
  snb::pdl_wait();
  snb::pdl_trigger();
  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16* ks = reinterpret_cast<__nv_bfloat16*>(smem);                   // [2][TT][RSK]
  constexpr int THR = kThr * MT, R = 16 * MT;  // threads, rows per CTA
  float* sp = reinterpret_cast<float*>(smem + SMEM_K);                               // [MT][4][16][TT]
  __nv_bfloat16* ps = reinterpret_cast<__nv_bfloat16*>(smem + SMEM_K + MT * SMEM_SP);  // [MT][16][RSP]
  float* alpha_s = reinterpret_cast<float*>(smem + SMEM_K + MT * (SMEM_SP + SMEM_P));  // [R]
  float* m_s = alpha_s + R;
  float* l_s = m_s + R;
  int32_t* lim_s = reinterpret_cast<int32_t*>(l_s + R);  // per-row key limit (0: row unused)
  int32_t* sbt = lim_s + R;

  const int split = blockIdx.x, hg = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gq = lane >> 2, qd = lane & 3;
  const int grp = warp >> 2, wq = warp & 3;  // row group of this warp, its quarter within the group
  const int h0 = hg * R;
  // rows of this CTA: decode -> heads h0.. of request b's token; extend -> (token, head) pairs h0..
  const bool ext = qo_indptr != nullptr;
  const int q0 = ext ? qo_indptr[b] : b;
  const int nq = ext ? qo_indptr[b + 1] - q0 : 1;
  const int nrows = ext ? nq * H - h0 : min(R, H - h0);
  if (nrows <= 0) return;  // extend: this request has fewer rows than the grid's row groups
  const int hn = min(R, nrows);
  const int kv_len = seq_lens[b];
  const int prefix = kv_len - nq;
  auto row_tok = [&](int row) { return ext ? q0 + (h0 + row) / H : b; };
  auto row_head = [&](int row) { return ext ? (h0 + row) % H : h0 + row; };
  auto row_lim = [&](int row) { return row >= hn ? 0 : (ext ? prefix + (h0 + row) / H + 1 : kv_len); };
  // keys of this DCP rank among logical positions [0, lim): whole local pages + the partial last page
  auto local_count = [&](int lim) {
    if (dcp_size == 1) return lim;
    const int full = lim / page_size, rem = lim % page_size;
    const int nfull = full > dcp_rank ? (full - dcp_rank + dcp_size - 1) / dcp_size : 0;
    return nfull * page_size + ((rem > 0 && full % dcp_size == dcp_rank) ? rem : 0);
  };
  auto logical = [&](int v) {
    return dcp_size == 1 ? v : ((v / page_size) * dcp_size + dcp_rank) * page_size + v % page_size;
  };
  const int ctx = local_count(row_lim(hn - 1));  // the last row sees the most keys
  const int per = ((ctx + num_splits - 1) / num_splits + TT - 1) / TT * TT;
  const int s0 = split * per, s1 = min(ctx, s0 + per);
  const int ntiles = s0 < s1 ? (s1 - s0 + TT - 1) / TT : 0;
  const int32_t* bt = block_table + (size_t)b * bt_stride;
  const int pg0 = s0 / page_size;
  const int npg = s0 < s1 ? (s1 - 1) / page_size - pg0 + 1 : 0;
  for (int i = tid; i < min(npg, kMaxSplitPages); i += THR) sbt[i] = bt[pg0 + i];
  if (tid < R) {
    m_s[tid] = -INFINITY;
    l_s[tid] = 0.f;
    lim_s[tid] = row_lim(tid);
  }
  __syncthreads();

  // page arithmetic without divisions for power-of-two page sizes (the usual case)
  const bool pow2 = (page_size & (page_size - 1)) == 0;
  const int pshift = __ffs(page_size) - 1;
  auto page_idx = [&](int tok) { return pow2 ? tok >> pshift : tok / page_size; };
  auto page_off = [&](int tok) { return pow2 ? tok & (page_size - 1) : tok % page_size; };
  auto page_of = [&](int tok) -> int {
    const int pi = page_idx(tok) - pg0;
    return pi < kMaxSplitPages ? sbt[pi] : bt[page_idx(tok)];
  };
  // tile k -> stage k & 1; rows past the split end are zero-filled (src size 0)
  auto load_tile = [&](int k) {
    const int t0 = s0 + k * TT;
    __nv_bfloat16* dst = ks + (k & 1) * TT * RSK;
    for (int c = tid; c < TT * (DK / 8); c += THR) {
      const int row = c / (DK / 8), col = (c % (DK / 8)) * 8;
      const int tok = t0 + row;
      const bool ok = tok < s1;
      const __nv_bfloat16* src =
          cache + ((size_t)(ok ? page_of(tok) : 0) * page_size + (ok ? page_off(tok) : 0)) * DK + col;
      cp_async16(snb::smem_u32(dst + row * RSK + col), src, ok ? 16 : 0);
    }
    cp_async_commit();
  };

  // Q fragments of this warp's 9 k16 steps (rows gq, gq + 8)
  uint32_t qa[9][4];
  {
    const __nv_bfloat16* qr[2];
#pragma unroll
    for (int rh = 0; rh < 2; ++rh) {
      const int row = grp * 16 + gq + rh * 8;
      qr[rh] = row < hn ? q + (size_t)row_tok(row) * q_stride + (size_t)row_head(row) * DK : nullptr;
    }
#pragma unroll
    for (int kk = 0; kk < 9; ++kk) {
      const int k0 = (wq * 9 + kk) * 16;
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int col = k0 + qd * 2 + (r >> 1) * 8;
        const __nv_bfloat16* p = qr[r & 1];
        qa[kk][r] = p != nullptr ? *reinterpret_cast<const uint32_t*>(p + col) : 0u;
      }
    }
  }
  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;

  if (ntiles > 0) load_tile(0);
  if (ntiles > 1) load_tile(1);
  for (int k = 0; k < ntiles; ++k) {
    if (k + 1 < ntiles) cp_async_wait<1>(); else cp_async_wait<0>();
    __syncthreads();
    const __nv_bfloat16* kt = ks + (k & 1) * TT * RSK;
    const int t0 = s0 + k * TT;
    // 1. partial scores over this warp's quarter of the 576-wide contraction (its group's 16 rows)
    float* spg = sp + grp * 4 * 16 * TT;
    float sc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 9; ++kk) {
        const __nv_bfloat16* kr = kt + (nt * 8 + gq) * RSK + (wq * 9 + kk) * 16 + qd * 2;
        mma_bf16_16816(sc[nt], qa[kk], *reinterpret_cast<const uint32_t*>(kr),
                       *reinterpret_cast<const uint32_t*>(kr + 8));
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) spg[(wq * 16 + gq + (j >> 1) * 8) * TT + nt * 8 + qd * 2 + (j & 1)] = sc[nt][j];
    }
    __syncthreads();
    // 2. online softmax: thread -> (group tid / 128, row (tid % 128) / 8, tokens 4 * (tid % 8) .. + 3)
    {
      const int g2 = tid >> 7, lrow = (tid & 127) >> 3, row = g2 * 16 + lrow, c4 = (tid & 7) * 4;
      const float* spr = sp + g2 * 4 * 16 * TT;
      __nv_bfloat16* psr = ps + g2 * 16 * RSP;
      float s[4], mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int col = c4 + j;
        float v = spr[lrow * TT + col] + spr[(16 + lrow) * TT + col] + spr[(32 + lrow) * TT + col] +
                  spr[(48 + lrow) * TT + col];
        v = (t0 + col < s1 && logical(t0 + col) < lim_s[row]) ? v * scale_log2 : -INFINITY;
        s[j] = v;
        mx = fmaxf(mx, v);
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      const float m_old = m_s[row];
      const float m_new = fmaxf(m_old, mx);
      const float alpha = (m_old == -INFINITY) ? (m_new == -INFINITY ? 1.f : 0.f) : exp2f(m_old - m_new);
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float p = s[j] == -INFINITY ? 0.f : exp2f(s[j] - m_new);
        rs += p;
        psr[lrow * RSP + c4 + j] = __float2bfloat16(p);
      }
      rs += __shfl_xor_sync(0xffffffffu, rs, 1);
      rs += __shfl_xor_sync(0xffffffffu, rs, 2);
      rs += __shfl_xor_sync(0xffffffffu, rs, 4);
      __syncwarp();
      if ((tid & 7) == 0) {
        alpha_s[row] = alpha;
        m_s[row] = m_new;
        l_s[row] = l_s[row] * alpha + rs;
      }
    }
    __syncthreads();
    // 3. O = alpha O + P V over this warp's 128 value columns of its group's rows
    {
      const float a0 = alpha_s[grp * 16 + gq], a1 = alpha_s[grp * 16 + gq + 8];
      const __nv_bfloat16* psg = ps + grp * 16 * RSP;
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        o[n][0] *= a0;
        o[n][1] *= a0;
        o[n][2] *= a1;
        o[n][3] *= a1;
      }
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        uint32_t pa[4];
        pa[0] = *reinterpret_cast<const uint32_t*>(psg + gq * RSP + kk * 16 + qd * 2);
        pa[1] = *reinterpret_cast<const uint32_t*>(psg + (gq + 8) * RSP + kk * 16 + qd * 2);
        pa[2] = *reinterpret_cast<const uint32_t*>(psg + gq * RSP + kk * 16 + 8 + qd * 2);
        pa[3] = *reinterpret_cast<const uint32_t*>(psg + (gq + 8) * RSP + kk * 16 + 8 + qd * 2);
        // V fragments by transposing loads: lane l addresses token kk*16 + 8 ((l >> 3) & 1) + (l & 7) of the
        // n-tile pair member l >> 4, giving b0 / b1 of two n8 tiles per instruction
        const uint32_t vrow = snb::smem_u32(kt + (kk * 16 + ((lane >> 3) & 1) * 8 + (lane & 7)) * RSK + wq * 128 +
                                            (lane >> 4) * 8);
#pragma unroll
        for (int n = 0; n < 16; n += 2) {
          uint32_t b[4];
          ldmatrix_x4_trans(b, vrow + n * 8 * 2);
          mma_bf16_16816(o[n], pa, b[0], b[1]);
          mma_bf16_16816(o[n + 1], pa, b[2], b[3]);
        }
      }
    }
    __syncthreads();  // the stage and P are reused by the next tile
    if (k + 2 < ntiles) load_tile(k + 2);
  }
  // write: rows gq / gq + 8 of the warp's group, columns wq * 128 + n * 8 + qd * 2 + {0, 1}
#pragma unroll
  for (int rh = 0; rh < 2; ++rh) {
    const int row = grp * 16 + gq + rh * 8;
    if (row >= hn) continue;
    const float L = l_s[row], M = m_s[row];
    const float inv = L > 0.f ? 1.f / L : 0.f;
    const int h = row_head(row);
    const int tok = row_tok(row);
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      const int col = wq * 128 + n * 8 + qd * 2;
      const float x0 = o[n][rh * 2] * inv, x1 = o[n][rh * 2 + 1] * inv;
      if (num_splits == 1) {
        *reinterpret_cast<__nv_bfloat162*>(out + (size_t)tok * out_stride + (size_t)h * DV + col) =
            __floats2bfloat162_rn(x0, x1);
        if (lse_out != nullptr && wq == 0 && n == 0 && qd == 0)
          lse_out[(size_t)tok * H + h] = L > 0.f ? M + log2f(L) : -INFINITY;
      } else {
        const size_t pidx = ((size_t)b * H + h) * num_splits + split;
        o_part[pidx * DV + col] = x0;
        o_part[pidx * DV + col + 1] = x1;
        if (wq == 0 && n == 0 && qd == 0) lse_part[pidx] = L > 0.f ? M + log2f(L) : -INFINITY;
      }
    }
  }
}

__global__ void mla_merge_kernel(const float* __restrict__ o_part, const float* __restrict__ lse_part,
                                 __nv_bfloat16* __restrict__ out, int out_stride, int H, int S) {
  snb::pdl_wait();
  snb::pdl_trigger();
  const int bh = blockIdx.x, b = bh / H, h = bh % H;
  const float* lse = lse_part + (size_t)bh * S;
  float M = -INFINITY;
  for (int s = 0; s < S; ++s) M = fmaxf(M, lse[s]);
  float total = 0.f;
  for (int s = 0; s < S; ++s) total += lse[s] == -INFINITY ? 0.f : exp2f(lse[s] - M);
  for (int d = threadIdx.x; d < DV; d += blockDim.x) {
    float a = 0.f;
    for (int s = 0; s < S; ++s)
      if (lse[s] != -INFINITY) a += exp2f(lse[s] - M) * o_part[((size_t)bh * S + s) * DV + d];
    out[(size_t)b * out_stride + (size_t)h * DV + d] = __float2bfloat16(total > 0.f ? a / total : 0.f);
  }
}

}  // namespace

// q: [B, H, 576] bf16 (row stride q.stride(0)); cache: [pages, 1, page, 576] bf16; out: [B, H, 512] bf16.
// o_part / lse_part: fp32 scratch of B*H*splits*512 and B*H*splits (used when splits > 1).
void mla_decode(torch::Tensor out, torch::Tensor q, torch::Tensor cache, torch::Tensor block_table,
                torch::Tensor seq_lens, int64_t page_size, double sm_scale, int64_t num_splits, torch::Tensor o_part,
                torch::Tensor lse_part) {
  const int B = q.size(0), H = q.size(1);
  if (B == 0) return;
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && cache.scalar_type() == at::kBFloat16, "mla_decode: bf16");
  TORCH_CHECK(q.size(2) == DK && cache.size(-1) == DK && q.stride(2) == 1 && q.stride(1) == DK, "mla_decode: q");
  TORCH_CHECK(out.size(2) == DV && out.stride(1) == DV && out.stride(2) == 1, "mla_decode: out");
  TORCH_CHECK(cache.is_contiguous() && (reinterpret_cast<uintptr_t>(cache.data_ptr()) % 16) == 0, "mla_decode: cache");
  const int S = std::max<int64_t>(1, num_splits);
  if (S > 1)
    TORCH_CHECK(o_part.numel() >= (int64_t)B * H * S * DV && lse_part.numel() >= (int64_t)B * H * S,
                "mla_decode: scratch");
  auto st = at::cuda::getCurrentCUDAStream();
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(mla_decode_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        MlaCfg<1>::SMEM));
    attr = true;
  }
  dim3 grid(S, (H + 15) / 16, B);
  float* op = S > 1 ? o_part.data_ptr<float>() : nullptr;
  float* lp = S > 1 ? lse_part.data_ptr<float>() : nullptr;
  C10_CUDA_CHECK(snb::launch_pdl(mla_decode_kernel<1>, grid, MlaCfg<1>::THR, MlaCfg<1>::SMEM, st,
                                 (const __nv_bfloat16*)q.data_ptr(),
                                 (int)q.stride(0), (const __nv_bfloat16*)cache.data_ptr(),
                                 block_table.data_ptr<int32_t>(), (int)block_table.stride(0),
                                 seq_lens.data_ptr<int32_t>(), (int)page_size, H, (float)sm_scale * kLog2e,
                                 (__nv_bfloat16*)out.data_ptr(), (int)out.stride(0), op, lp, S,
                                 (const int32_t*)nullptr, 1, 0, (float*)nullptr));
  if (S > 1)
    C10_CUDA_CHECK(snb::launch_pdl(mla_merge_kernel, B * H, 128, 0, st, (const float*)op, (const float*)lp,
                                   (__nv_bfloat16*)out.data_ptr(), (int)out.stride(0), H, S));
}

// Extend: q [T, H, 576] for the new tokens of B requests (rows qo_indptr[b] .. qo_indptr[b+1]), whose latent
// rows are already in the cache; seq_lens[b] = prefix + new tokens. out: [T, H, 512].
// dcp_size > 1: block_table holds this rank's pages only (see the kernel); lse_out [T, H] fp32 receives the
// rows' log2-sum-exp of the scaled scores (-inf for rows with no local key).
void mla_extend(torch::Tensor out, torch::Tensor q, torch::Tensor cache, torch::Tensor block_table,
                torch::Tensor seq_lens, torch::Tensor qo_indptr, int64_t max_extend, int64_t page_size,
                double sm_scale, int64_t dcp_size, int64_t dcp_rank, c10::optional<torch::Tensor> lse_out) {
  const int T = q.size(0), H = q.size(1), B = seq_lens.size(0);
  if (T == 0 || B == 0) return;
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && cache.scalar_type() == at::kBFloat16, "mla_extend: bf16");
  TORCH_CHECK(q.size(2) == DK && cache.size(-1) == DK && q.stride(2) == 1 && q.stride(1) == DK, "mla_extend: q");
  TORCH_CHECK(out.size(2) == DV && out.stride(1) == DV && out.stride(2) == 1, "mla_extend: out");
  TORCH_CHECK(cache.is_contiguous() && (reinterpret_cast<uintptr_t>(cache.data_ptr()) % 16) == 0, "mla_extend: cache");
  TORCH_CHECK(qo_indptr.scalar_type() == at::kInt && qo_indptr.numel() >= B + 1, "mla_extend: qo_indptr");
  TORCH_CHECK(seq_lens.scalar_type() == at::kInt && block_table.scalar_type() == at::kInt, "mla_extend: int32 tables");
  auto st = at::cuda::getCurrentCUDAStream();
  constexpr int kExtMT = 2;
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(mla_decode_kernel<kExtMT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        MlaCfg<kExtMT>::SMEM));
    attr = true;
  }
  TORCH_CHECK(dcp_size >= 1 && dcp_rank >= 0 && dcp_rank < dcp_size, "mla_extend: dcp rank");
  if (lse_out)
    TORCH_CHECK(lse_out->scalar_type() == at::kFloat && lse_out->is_contiguous() && lse_out->numel() >= (int64_t)T * H,
                "mla_extend: lse_out");
  const int64_t groups = (std::max<int64_t>(1, max_extend) * H + 16 * kExtMT - 1) / (16 * kExtMT);
  TORCH_CHECK(groups <= 65535, "mla_extend: too many rows per request");
  dim3 grid(1, (unsigned)groups, B);
  C10_CUDA_CHECK(snb::launch_pdl(mla_decode_kernel<kExtMT>, grid, MlaCfg<kExtMT>::THR, MlaCfg<kExtMT>::SMEM, st,
                                 (const __nv_bfloat16*)q.data_ptr(),
                                 (int)q.stride(0), (const __nv_bfloat16*)cache.data_ptr(),
                                 block_table.data_ptr<int32_t>(), (int)block_table.stride(0),
                                 seq_lens.data_ptr<int32_t>(), (int)page_size, H, (float)sm_scale * kLog2e,
                                 (__nv_bfloat16*)out.data_ptr(), (int)out.stride(0), (float*)nullptr,
                                 (float*)nullptr, 1, qo_indptr.data_ptr<int32_t>(), (int)dcp_size, (int)dcp_rank,
                                 lse_out ? lse_out->data_ptr<float>() : (float*)nullptr));
}
