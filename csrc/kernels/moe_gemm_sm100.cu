// Block-scaled grouped expert GEMM for MoE on the 5th-generation tensor cores (sm_100a).
//
//   D[f, r] = sum_k W[e][f, k] * X[r, k]     for every permuted row r of expert e's padded segment
//
// W: MXFP4 (e2m1, two per byte) or MXFP8 (e4m3) expert weights with one e8m0 scale per 32 K-values;
// X: MXFP8 activations produced by gather_quant_mxfp8 (rows grouped by expert, segments padded to BN).
// One tcgen05.mma.kind::mxf8f6f4.block_scale instruction multiplies a 128 x BN x 32 block; the scale
// factors live in tensor memory (copied from shared memory with tcgen05.cp 32x128b.warpx4) and the fp32
// accumulator lives in tensor memory, double-buffered so the epilogue of one tile overlaps the MMAs of
// the next.
//
// Parity: the reference's expert kernels `moe_block_tkg` (decode) and `moe_cte` (prefill)
// (sglang_neuron/ops/moe/moe_block_tkg.py:19-128, moe_cte.py:29-103) run MXFP4 experts with clamped
// SwiGLU (alpha 1.702, limit 7) over MX-FP8 activations (rmsnorm_mx_prefill.py:41). Here the same math is
// one persistent kernel per projection:
//   EPI_SWIGLU_CLAMP / EPI_SILU: gate/up projection, weights rows pre-arranged per 128-row tile as
//       [64 gate rows | 64 matching up rows]; the epilogue adds the bias and writes act[r, j] (bf16).
//   EPI_BIAS: down projection; the epilogue adds the bias and writes y[r, f] (bf16).
//
// Warp roles (192 threads, one CTA per SM, persistent over tiles):
//   warp 0: TMA producer (A tile via a 3D map [E, F, K], B tile via a 2D map [R, K], scale chunks via
//           cp.async.bulk), warp 1: TMEM owner + single-thread MMA issuer, warps 2-5: epilogue.
// Every wait is bounded; on timeout the kernel records a status code, stops issuing work and still
// frees its tensor memory.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "../common.cuh"
#include "../tma_host.h"

namespace {

constexpr int BM = 128;
constexpr int BK = 128;           // K elements per pipeline stage (4 MMAs of K=32)
constexpr int A_SMEM = BM * BK;   // 16 KB: one byte per element in shared memory for fp8 and unpacked fp4
constexpr int SF_SMEM = 512;      // one 32x128-bit scale atom
constexpr int MAX_EXPERTS = 256;

enum Epi : int { EPI_SWIGLU_CLAMP = 0, EPI_SILU = 1, EPI_BIAS = 2 };

// Small-N tiles (decode: a few tokens per expert) run two CTAs per SM so two independent TMA pipelines
// stream weights per SM; each then owns 128 TMEM columns (2 accumulators + per-stage scale factors).
template <int BN>
struct MoeCfg {
  static constexpr int CTAS_PER_SM = BN <= 32 ? 2 : 1;
  static constexpr int B_SMEM = BN * BK;
  static constexpr int STAGE = A_SMEM + B_SMEM + 2 * SF_SMEM;
  static constexpr int BUDGET = CTAS_PER_SM == 2 ? 96 * 1024 : 176 * 1024;
  static constexpr int STAGES = BUDGET / STAGE > 8 ? 8 : BUDGET / STAGE;
  static constexpr int ACC_BUFS = BN <= 128 ? 2 : 1;
  static constexpr int SF_COL0 = ACC_BUFS * BN;  // scale-factor columns start after the accumulators
  static constexpr int TMEM_COLS = CTAS_PER_SM == 2 ? 128 : 512;
  static_assert(SF_COL0 + 8 * STAGES <= TMEM_COLS, "TMEM plan overflows the allocation");
  static constexpr int XBUF = 64 * 32 * 4;       // epilogue exchange buffer (64 rows x 32 cols fp32)
  static constexpr int SMEM = STAGES * STAGE + XBUF + 1024 + 2048;
};

struct MoeParams {
  const int32_t* seg_offsets;   // [E_local + 1]
  const int32_t* tile_offsets;  // [E_local + 1] prefix of BN-tiles per expert
  const uint8_t* sfa;           // [E][MT][KB][512]
  const uint8_t* sfb;           // [R/BN][KB][chunk]
  const __nv_bfloat16* bias;    // [E][F] (arranged like the weight rows) or null
  __nv_bfloat16* out;           // [R, ldo]
  int ldo;
  int num_experts;
  int F;                        // weight rows (output features, or 2*I for gated)
  int K;
  int MT;                       // ceil(F / 128)
  int KB;                       // ceil(K / 128)
  float alpha, limit;           // clamped SwiGLU parameters
  int* status;
  // Gated epilogues only: write the activation straight as MXFP8 (the down projection's B operand) instead
  // of bf16: e4m3 values [R, q_ld] and e8m0 scales in the chunk-atom order (null: bf16 to `out`).
  uint8_t* qout;
  uint8_t* sfout;
  int q_ld, q_KB, q_chunk, q_bn;
};

SNB_DEVICE void bar_epi() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

SNB_DEVICE float sigmoidf_(float x) { return 1.f / (1.f + __expf(-x)); }

// Locate tile t: returns expert e and the first permuted row r0 of its n-tile.
SNB_DEVICE void locate(const int32_t* tile_off_s, const int32_t* seg_off_s, int E, int MT, int BN, int t,
                       int& e, int& mt, int& r0) {
  const int nt = t / MT;
  mt = t % MT;
  int lo = 0, hi = E;  // find e with tile_off[e] <= nt < tile_off[e+1]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (tile_off_s[mid] <= nt) lo = mid; else hi = mid;
  }
  e = lo;
  r0 = seg_off_s[e] + (nt - tile_off_s[e]) * BN;
}

template <int BN, bool A_FP4, int EPI>
__global__ void __launch_bounds__(192, MoeCfg<BN>::CTAS_PER_SM)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                    const MoeParams p) {
  snb::pdl_wait();
  snb::pdl_trigger();
  using C = MoeCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;                                   // STAGES x 16 KB (1024-aligned)
  uint8_t* sB = sA + C::STAGES * A_SMEM;                // STAGES x BN*128 (1024-aligned: BN*128 % 1024 == 0)
  uint8_t* sSF = sB + C::STAGES * C::B_SMEM;            // STAGES x (SFA 512 | SFB 512)
  float* xbuf = reinterpret_cast<float*>(sSF + C::STAGES * 2 * SF_SMEM);
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(xbuf) + C::XBUF);
  uint64_t* empty = full + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int32_t* tile_off_s = reinterpret_cast<int32_t*>(tmem_slot + 4);
  int32_t* seg_off_s = tile_off_s + MAX_EXPERTS + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = p.num_experts;
  for (int i = threadIdx.x; i <= E; i += blockDim.x) {
    tile_off_s[i] = p.tile_offsets[i];
    seg_off_s[i] = p.seg_offsets[i];
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      snb::mbar_init(&full[s], 1);
      snb::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      snb::mbar_init(&acc_full[b], 1);
      snb::mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
    }
    snb::mbar_init(drain, 1);
    *abort_flag = 0;
    snb::fence_mbar_init();
    snb::prefetch_tmap(&tmap_a);
    snb::prefetch_tmap(&tmap_b);
  }
  if (warp == 1) {
    snb::tmem_alloc(tmem_slot, C::TMEM_COLS);
    snb::tmem_relinquish();
  }
  snb::tc_fence_before();
  __syncthreads();
  snb::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int n_tiles = tile_off_s[E] * p.MT;
  const int chunk = (BN < 32 ? BN : 32) * 16;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      const uint64_t stream_once = snb::l2_policy_evict_first();
      for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
        int e, mt, r0;
        locate(tile_off_s, seg_off_s, E, p.MT, BN, t, e, mt, r0);
        for (int kb = 0; kb < p.KB; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!snb::mbar_wait_bounded(&empty[s], ph ^ 1, p.status, SNB_ERR_TIMEOUT_TMA)) {
            ok = false;
            break;
          }
          const uint32_t a_bytes = A_FP4 ? A_SMEM / 2 : A_SMEM;
          snb::mbar_arrive_expect_tx(&full[s], a_bytes + C::B_SMEM + SF_SMEM + chunk);
          // weights are pre-tiled [E][MT][KB][128 rows]: every stage reads one contiguous block
          snb::tma_load_2d_hint(sA + s * A_SMEM, &tmap_a, &full[s], 0, ((e * p.MT + mt) * p.KB + kb) * BM,
                                stream_once);
          snb::tma_load_2d(sB + s * C::B_SMEM, &tmap_b, &full[s], kb * BK, r0);
          snb::bulk_load(sSF + s * 2 * SF_SMEM, p.sfa + ((size_t)(e * p.MT + mt) * p.KB + kb) * SF_SMEM, SF_SMEM,
                         &full[s]);
          snb::bulk_load(sSF + s * 2 * SF_SMEM + SF_SMEM, p.sfb + ((size_t)(r0 / BN) * p.KB + kb) * chunk, chunk,
                         &full[s]);
        }
      }
      // Never leave a bulk copy in flight into shared memory: wait (bounded) for the last issued stages.
      for (int j = it - 1; j >= 0 && j >= it - C::STAGES; --j)
        snb::mbar_wait_bounded(&full[j % C::STAGES], (j / C::STAGES) & 1, p.status, SNB_ERR_TIMEOUT_TMA);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int it = 0, tile_i = 0;
      bool ok = true;
      const uint32_t a_fmt = A_FP4 ? 5u : 0u;  // e2m1 or e4m3
      const uint32_t idesc0 = snb::idesc_mx(BM, BN, a_fmt, 0u);
      for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x, ++tile_i) {
        const int buf = C::ACC_BUFS == 2 ? (tile_i & 1) : 0;
        const uint32_t use = C::ACC_BUFS == 2 ? (tile_i >> 1) : tile_i;
        if (!snb::mbar_wait_bounded(&acc_empty[buf], (use & 1) ^ 1, p.status, SNB_ERR_TIMEOUT_MMA)) break;
        snb::tc_fence_after();
        const uint32_t d_tmem = tmem + buf * BN;
        for (int kb = 0; kb < p.KB; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!snb::mbar_wait_bounded(&full[s], ph, p.status, SNB_ERR_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          snb::tc_fence_after();
          const uint32_t sf_col = C::SF_COL0 + s * 8;
          const uint32_t sfa_t = tmem + sf_col, sfb_t = tmem + sf_col + 4;
          const uint32_t sf_s = snb::smem_u32(sSF + s * 2 * SF_SMEM);
          snb::tmem_cp_32x128b_warpx4(sfa_t, snb::smem_desc_plain(sf_s, 128, 128));
          snb::tmem_cp_32x128b_warpx4(sfb_t, snb::smem_desc_plain(sf_s + SF_SMEM, 128, 128));
          const uint32_t a_base = snb::smem_u32(sA + s * A_SMEM);
          const uint32_t b_base = snb::smem_u32(sB + s * C::B_SMEM);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t idesc = idesc0 | ((uint32_t)kk << 4) | ((uint32_t)kk << 29);
            snb::mma_mxf8f6f4_ss(d_tmem, snb::smem_desc_sw128(a_base + kk * 32), snb::smem_desc_sw128(b_base + kk * 32),
                                 idesc, sfa_t, sfb_t, (kb | kk) != 0 ? 1u : 0u);
          }
          snb::mma_commit(&empty[s]);
        }
        if (!ok) break;
        snb::mma_commit(&acc_full[buf]);
      }
      // Wait (bounded) until every tcgen05 op issued here has completed before TMEM is released.
      snb::mma_commit(drain);
      snb::mbar_wait_bounded(drain, 0, p.status, SNB_ERR_TIMEOUT_MMA);
    }
  } else {
    // Epilogue warps 2..5 -> TMEM lane quarter q = warp % 4 (rows 32q .. 32q+31 of the tile).
    const int q = warp & 3;
    int tile_i = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++tile_i) {
      int e, mt, r0;
      locate(tile_off_s, seg_off_s, E, p.MT, BN, t, e, mt, r0);
      const int buf = C::ACC_BUFS == 2 ? (tile_i & 1) : 0;
      const uint32_t use = C::ACC_BUFS == 2 ? (tile_i >> 1) : tile_i;
      // The four epilogue warps stay in lockstep on the named barrier; a timed-out warp skips the work
      // but keeps hitting the barriers, and all warps leave together through the shared abort flag.
      const bool ok = snb::mbar_wait_bounded(&acc_full[buf], use & 1, p.status, SNB_ERR_TIMEOUT_EPI);
      if (!ok) *abort_flag = 1;
      snb::tc_fence_after();
      const uint32_t d_tmem = tmem + buf * BN + ((uint32_t)(q * 32) << 16);
      const int row = q * 32 + lane;          // row within the 128-row weight tile
      const int frow = mt * BM + row;         // weight row (arranged order)
      const float b = (p.bias != nullptr && frow < p.F) ? __bfloat162float(p.bias[(size_t)e * p.F + frow]) : 0.f;
      constexpr int NCH = BN >= 32 ? BN / 32 : 1;
      constexpr int CW = BN >= 32 ? 32 : BN;
#pragma unroll 1
      for (int c = 0; c < NCH; ++c) {
        float v[32];
        if (ok) {
          uint32_t r[32];
          if constexpr (CW == 32) {
            snb::tmem_ld_32x32b_x32(d_tmem + c * 32, r);
          } else {
            uint32_t r8[8];
#pragma unroll
            for (int h = 0; h < CW / 8; ++h) {
              snb::tmem_ld_32x32b_x8(d_tmem + h * 8, r8);
#pragma unroll
              for (int j = 0; j < 8; ++j) r[h * 8 + j] = r8[j];
            }
          }
          snb::tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < CW; ++j) v[j] = __uint_as_float(r[j]) + b;
        }
        if constexpr (EPI == EPI_BIAS) {
          if (ok && frow < p.F) {
#pragma unroll
            for (int j = 0; j < CW; ++j) p.out[(size_t)(r0 + c * 32 + j) * p.ldo + frow] = __float2bfloat16(v[j]);
          }
        } else {
          // Rows 64..127 hold the "up" half: hand them to the warps holding the matching "gate" rows.
          if (ok && q >= 2) {
#pragma unroll
            for (int j = 0; j < CW; ++j) xbuf[(row - 64) * 32 + ((j + row) & 31)] = v[j];
          }
          bar_epi();
          const bool ok_w = __all_sync(0xffffffffu, ok);  // warp-uniform for the shuffles below
          if (ok_w && q < 2) {
            const int jcol = mt * 64 + row;  // activation column; warp q holds MX block 2 mt + q
            const bool colok = jcol < p.F / 2;
#pragma unroll
            for (int j = 0; j < CW; ++j) {
              float g = v[j];
              float u = xbuf[row * 32 + ((j + row + 64) & 31)];
              float a;
              if constexpr (EPI == EPI_SWIGLU_CLAMP) {
                g = fminf(g, p.limit);
                u = fminf(fmaxf(u, -p.limit), p.limit);
                a = (u + 1.f) * (g * sigmoidf_(g * p.alpha));
              } else {
                a = g * sigmoidf_(g) * u;
              }
              const int rr = r0 + c * 32 + j;
              if (p.qout == nullptr) {
                if (colok) p.out[(size_t)rr * p.ldo + jcol] = __float2bfloat16(a);
              } else {
                // MXFP8 of the bf16-rounded activation: one e8m0 scale per 32 columns (this warp's lanes)
                a = colok ? __bfloat162float(__float2bfloat16(a)) : 0.f;
                float amax = fabsf(a);
#pragma unroll
                for (int sh = 16; sh > 0; sh >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, sh));
                int X = 0;
                if (amax > 0.f) X = max(-127, min(127, (int)ceilf(log2f(amax / 448.f))));
                if (colok) p.qout[(size_t)rr * p.q_ld + jcol] = snb::f_to_fp8e4m3(a * exp2f((float)-X));
                const int tile = rr / p.q_bn, i = rr % p.q_bn;
                uint8_t* sfrow = p.sfout + (size_t)tile * p.q_KB * p.q_chunk + (i % 32) * 16 + (i / 32) * 4;
                if (lane == 0) {
                  const int blk = 2 * mt + q;
                  sfrow[(blk >> 2) * p.q_chunk + (blk & 3)] = (uint8_t)(X + 127);
                }
                if (mt == p.MT - 1 && q == 0 && lane < 4 * p.q_KB - 2 * p.MT) {
                  const int blk = 2 * p.MT + lane;  // padding blocks past the last column: scale 1
                  sfrow[(blk >> 2) * p.q_chunk + (blk & 3)] = 127;
                }
              }
            }
          }
          bar_epi();
        }
      }
      snb::tc_fence_before();
      if (lane == 0) snb::mbar_arrive(&acc_empty[buf]);
      bar_epi();
      if (*abort_flag) break;
    }
  }
  snb::tc_fence_before();
  __syncthreads();
  if (warp == 1) snb::tmem_dealloc(tmem, C::TMEM_COLS);
}

template <int BN, bool A_FP4, int EPI>
void launch_moe(const CUtensorMap& ta, const CUtensorMap& tb, const MoeParams& p, int grid, cudaStream_t st) {
  using C = MoeCfg<BN>;
  static bool attr = false;
  if (!attr) {
    TORCH_CHECK(cudaFuncSetAttribute(moe_gemm_kernel<BN, A_FP4, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     C::SMEM) == cudaSuccess,
                "moe_gemm: smem attribute");
    attr = true;
  }
  snb::launch_pdl(moe_gemm_kernel<BN, A_FP4, EPI>, grid, 192, C::SMEM, st, ta, tb, p);
}

template <bool A_FP4, int EPI>
void dispatch_bn(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const MoeParams& p, int grid, cudaStream_t st) {
  switch (bn) {
    case 16: launch_moe<16, A_FP4, EPI>(ta, tb, p, grid, st); break;
    case 32: launch_moe<32, A_FP4, EPI>(ta, tb, p, grid, st); break;
    case 64: launch_moe<64, A_FP4, EPI>(ta, tb, p, grid, st); break;
    case 128: launch_moe<128, A_FP4, EPI>(ta, tb, p, grid, st); break;
    default: TORCH_CHECK(false, "moe_gemm: bn must be 16/32/64/128");
  }
}

}  // namespace

// w: [E, F, K/2] uint8 (fp4) or [E, F, K] float8_e4m3fn; sfa: [E, MT, KB, 512] uint8 atoms;
// xq: [R, K] float8_e4m3fn permuted activations; sfb: chunk-atom scales from gather_quant_mxfp8;
// out: [R, ldo] bf16. epi: 0 clamped SwiGLU, 1 SiLU-gated, 2 bias only.
void moe_gemm(torch::Tensor out, torch::Tensor xq, torch::Tensor sfb, torch::Tensor w, torch::Tensor sfa,
              c10::optional<torch::Tensor> bias, torch::Tensor seg_offsets, torch::Tensor tile_offsets,
              int64_t bn, int64_t epi, double alpha, double limit, int64_t num_sms, torch::Tensor status,
              int64_t F, c10::optional<torch::Tensor> qout, c10::optional<torch::Tensor> sfout) {
  // w: tiled weights [E, MT, KB, 128, bpr] (bpr = 64 bytes of packed fp4 or 128 bytes of fp8 per row of a
  // 128-wide K block), zero-padded past F rows and K columns.
  TORCH_CHECK(w.dim() == 5 && w.size(3) == BM, "moe_gemm: weights must be tiled [E, MT, KB, 128, bytes]");
  const bool fp4 = w.scalar_type() == at::kByte;
  const int E = w.size(0), MT = w.size(1), KBw = w.size(2);
  const int bpr = w.size(4);
  const int K = xq.size(1);
  TORCH_CHECK(E <= MAX_EXPERTS, "moe_gemm: at most 256 local experts");
  TORCH_CHECK(bpr == (fp4 ? 64 : 128), "moe_gemm: tile row bytes");
  TORCH_CHECK(KBw == (K + BK - 1) / BK && MT == (F + BM - 1) / BM, "moe_gemm: tile grid does not match K/F");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(w.data_ptr()) & 127) == 0, "moe_gemm: weights must be 128-byte aligned");
  TORCH_CHECK(xq.scalar_type() == at::kFloat8_e4m3fn && xq.is_contiguous(), "moe_gemm: xq");
  TORCH_CHECK(K % 32 == 0, "moe_gemm: K must be a multiple of 32");
  TORCH_CHECK(w.is_contiguous() && sfa.is_contiguous() && sfb.is_contiguous(), "moe_gemm: contiguity");
  if (epi != 2) TORCH_CHECK(F % 128 == 0, "moe_gemm: gated projections need F % 128 == 0");
  const int R = xq.size(0);
  TORCH_CHECK(R % bn == 0, "moe_gemm: rows must be a multiple of bn");
  MoeParams p;
  p.seg_offsets = seg_offsets.data_ptr<int32_t>();
  p.tile_offsets = tile_offsets.data_ptr<int32_t>();
  p.sfa = sfa.data_ptr<uint8_t>();
  p.sfb = sfb.data_ptr<uint8_t>();
  p.bias = bias ? (const __nv_bfloat16*)bias->data_ptr() : nullptr;
  p.out = (__nv_bfloat16*)out.data_ptr();
  p.ldo = out.stride(0);
  p.num_experts = E;
  p.F = F;
  p.K = K;
  p.MT = MT;
  p.KB = KBw;
  p.alpha = (float)alpha;
  p.limit = (float)limit;
  p.status = status.data_ptr<int>();
  p.qout = nullptr;
  p.sfout = nullptr;
  p.q_ld = p.q_KB = p.q_chunk = p.q_bn = 0;
  if (qout.has_value()) {
    TORCH_CHECK(epi != 2 && sfout.has_value(), "moe_gemm: MXFP8 output is for the gated projections");
    TORCH_CHECK(qout->scalar_type() == at::kFloat8_e4m3fn && qout->is_contiguous() && qout->size(0) == R &&
                    qout->size(1) == F / 2, "moe_gemm: qout must be [R, F/2] e4m3");
    p.qout = reinterpret_cast<uint8_t*>(qout->data_ptr());
    p.sfout = sfout->data_ptr<uint8_t>();
    p.q_ld = F / 2;
    p.q_KB = (F / 2 + BK - 1) / BK;
    p.q_chunk = (int)std::min<int64_t>(bn, 32) * 16;
    p.q_bn = bn;
    TORCH_CHECK(sfout->numel() >= (int64_t)(R / bn) * p.q_KB * p.q_chunk, "moe_gemm: sfout size");
  }
  TORCH_CHECK(sfa.numel() >= (int64_t)E * p.MT * p.KB * SF_SMEM, "moe_gemm: sfa size");
  // One 2D view over all tiles: rows = E*MT*KB*128, each row one 128-value K slice of one weight row.
  CUtensorMap ta = snb_host::make_tmap_2d(w.data_ptr(),
                                          fp4 ? CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B : CU_TENSOR_MAP_DATA_TYPE_UINT8,
                                          BK, (uint64_t)E * MT * KBw * BM, bpr, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tb = snb_host::make_tmap_2d(xq.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, K, R, K, BK, bn,
                                          CU_TENSOR_MAP_SWIZZLE_128B);
  auto st = at::cuda::getCurrentCUDAStream();
  const int grid = (int)num_sms * (bn <= 32 ? 2 : 1);
#define SNB_MOE(FP4, EP) dispatch_bn<FP4, EP>(bn, ta, tb, p, grid, st)
  if (fp4) {
    if (epi == 0) SNB_MOE(true, EPI_SWIGLU_CLAMP);
    else if (epi == 1) SNB_MOE(true, EPI_SILU);
    else SNB_MOE(true, EPI_BIAS);
  } else {
    TORCH_CHECK(w.scalar_type() == at::kFloat8_e4m3fn, "moe_gemm: weight dtype");
    if (epi == 0) SNB_MOE(false, EPI_SWIGLU_CLAMP);
    else if (epi == 1) SNB_MOE(false, EPI_SILU);
    else SNB_MOE(false, EPI_BIAS);
  }
#undef SNB_MOE
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
