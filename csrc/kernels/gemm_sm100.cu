// Dense bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
//   out[t, f] = sum_k x[t, k] * w[f, k] (+ bias[f])        x: [T, K], w: [F, K] (nn.Linear layout)
//
// The MMA computes the transposed product D[f, t] so the weight matrix is the M=128 operand and the
// (often small) token count is the N operand (16..256): decode batches of a few tokens still use full
// 128-row tensor-core tiles, and prefill uses N=256 tiles.
//
// CTA = 6 warps: warp 0 issues TMA loads into a STAGES-deep shared-memory ring, warp 1 allocates TMEM
// and a single elected thread issues tcgen05.mma (128 x BN x 16 per instruction, 4 per 64-wide K block)
// and tcgen05.commit to free ring slots, warps 2-5 drain the fp32 accumulator from TMEM with tcgen05.ld
// and write bf16. Every mbarrier wait is bounded; a timeout records a status code and the CTA still
// releases its tensor memory before returning.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "../common.cuh"
#include "../tma_host.h"
#include "../ar_common.cuh"

namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // bf16 elements per 128-byte swizzled row

template <int BN>
struct GemmCfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (200 * 1024) / STAGE_BYTES > 8 ? 8 : (200 * 1024) / STAGE_BYTES;
  static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

// Split-K: blockIdx.z selects a contiguous range of K blocks; with more than one split every CTA writes its
// fp32 partial tile to `partial` [splits, T, F] and splitk_reduce_kernel sums them (plus the bias) to bf16.
// Decode-sized GEMMs (few tokens, F/128 CTAs) use it to put every SM to work on the weight stream.
// AR = true: the epilogue all-reduces its output tile over the tensor-parallel group inside this kernel:
// the bf16 tile is stored straight into every peer's symmetric buffer (slot = my rank, NVLink P2P stores),
// the tile's flag is released to every peer, the CTA waits (bounded) for the same tile from every rank and
// writes the sum. Communication of a finished tile overlaps the MMAs of the tiles still running.
struct GemmAR {
  snb_ar::ARPeers peers;
  int rank, world;
  size_t capacity;
};

SNB_DEVICE void bar_epilogue() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

template <int BN, bool AR>
__global__ void __launch_bounds__(192, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                     __nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ bias, int F, int T,
                     int K, int ldo, int* status, float* __restrict__ partial, const GemmAR ar) {
  using C = GemmCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + C::STAGES * C::B_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* accum = empty + C::STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int f0 = blockIdx.x * BM, t0 = blockIdx.y * BN;
  const int nk_all = (K + BK - 1) / BK;
  const int per_split = (nk_all + gridDim.z - 1) / gridDim.z;
  const int kb0 = blockIdx.z * per_split;
  const int nk = max(0, min(nk_all, kb0 + per_split) - kb0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      snb::mbar_init(&full[s], 1);
      snb::mbar_init(&empty[s], 1);
    }
    snb::mbar_init(accum, 1);
    snb::fence_mbar_init();
    snb::prefetch_tmap(&tmap_w);
    snb::prefetch_tmap(&tmap_x);
  }
  if (warp == 1) {
    snb::tmem_alloc(tmem_slot, C::TMEM_COLS);
    snb::tmem_relinquish();
  }
  snb::tc_fence_before();
  __syncthreads();
  snb::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % C::STAGES;
        const uint32_t ph = (kb / C::STAGES) & 1;
        if (!snb::mbar_wait_bounded(&empty[s], ph ^ 1, status, SNB_ERR_TIMEOUT_TMA)) break;
        snb::mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
        snb::tma_load_2d(sA + s * C::A_BYTES, &tmap_w, &full[s], (kb0 + kb) * BK, f0);
        snb::tma_load_2d(sB + s * C::B_BYTES, &tmap_x, &full[s], (kb0 + kb) * BK, t0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = snb::idesc_bf16_f32(BM, BN);
      bool ok = true;
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % C::STAGES;
        const uint32_t ph = (kb / C::STAGES) & 1;
        if (!snb::mbar_wait_bounded(&full[s], ph, status, SNB_ERR_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        snb::tc_fence_after();
        const uint32_t a_base = snb::smem_u32(sA + s * C::A_BYTES);
        const uint32_t b_base = snb::smem_u32(sB + s * C::B_BYTES);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {
          snb::mma_bf16_ss(tmem, snb::smem_desc_sw128(a_base + k * 32), snb::smem_desc_sw128(b_base + k * 32),
                           idesc, (kb | k) != 0 ? 1u : 0u);
        }
        snb::mma_commit(&empty[s]);
      }
      if (ok) snb::mma_commit(accum);
    }
  } else {
    // Epilogue warps 2..5: warp w reads TMEM lanes 32*(w%4) .. +31.
    const int q = warp & 3;
    const bool ok = nk > 0 && snb::mbar_wait_bounded(accum, 0, status, SNB_ERR_TIMEOUT_EPI);
    snb::tc_fence_after();
    if (nk == 0 && partial != nullptr) {
      // empty split (K range past the end): contribute zeros
      const int f = f0 + q * 32 + lane;
      if (f < F)
        for (int t = t0; t < min(T, t0 + BN); ++t) partial[((size_t)blockIdx.z * T + t) * F + f] = 0.f;
    }
    uint32_t ar_epoch = 0;
    int ar_half = 0;
    snb_ar::ARBuf arb;
    if constexpr (AR) {
      arb = snb_ar::ar_layout(ar.peers, ar.rank, ar.world, ar.capacity);
      ar_epoch = *reinterpret_cast<volatile uint32_t*>(arb.counter) + 1;
      ar_half = ar_epoch & 1;
    }
    if (ok) {
      const int f = f0 + q * 32 + lane;
      const float bf = (bias != nullptr && f < F) ? __bfloat162float(bias[f]) : 0.f;
#pragma unroll 1
      for (int c = 0; c < BN / 32 + (BN % 32 ? 1 : 0); ++c) {
        uint32_t r[32];
        if constexpr (BN >= 32) {
          snb::tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + c * 32, r);
          snb::tmem_ld_wait();
        } else {
          uint32_t r8[8];
#pragma unroll
          for (int h = 0; h < BN / 8; ++h) {
            snb::tmem_ld_32x32b_x8(tmem + ((uint32_t)(q * 32) << 16) + h * 8, r8);
            snb::tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 8; ++j) r[h * 8 + j] = r8[j];
          }
        }
        if (f < F) {
          const int ncol = BN >= 32 ? 32 : BN;
          if constexpr (AR) {
#pragma unroll
            for (int j = 0; j < ncol; ++j) {
              const int t = t0 + c * 32 + j;
              if (t < T) {
                const __nv_bfloat16 v = __float2bfloat16(__uint_as_float(r[j]) + bf);
                for (int p = 0; p < ar.world; ++p)
                  reinterpret_cast<__nv_bfloat16*>(
                      snb_ar::ar_slot(ar.peers, p, ar_half, ar.rank, ar.world, ar.capacity))[(size_t)t * F + f] = v;
              }
            }
          } else if (partial != nullptr) {
            float* pz = partial + (size_t)blockIdx.z * T * F;
#pragma unroll
            for (int j = 0; j < ncol; ++j) {
              const int t = t0 + c * 32 + j;
              if (t < T) pz[(size_t)t * F + f] = __uint_as_float(r[j]);
            }
          } else {
#pragma unroll
            for (int j = 0; j < ncol; ++j) {
              const int t = t0 + c * 32 + j;
              if (t < T) out[(size_t)t * ldo + f] = __float2bfloat16(__uint_as_float(r[j]) + bf);
            }
          }
        }
      }
    }
    if constexpr (AR) {
      // publish this tile, wait for it from every rank, reduce (epilogue warps only: named barrier 1)
      __shared__ int ar_ok;
      const int tile = blockIdx.x + blockIdx.y * gridDim.x;
      bar_epilogue();
      if (warp == 2 && lane == 0) ar_ok = ok ? 1 : 0;
      if (warp == 2 && lane < ar.world) {
        uint32_t* fp = reinterpret_cast<uint32_t*>(ar.peers.buf[lane] + 2 * (size_t)ar.world * ar.capacity);
        __threadfence_system();
        snb_ar::st_release_sys(fp + ar.rank * snb_ar::kMaxCtas + tile, ar_epoch);
      }
      bar_epilogue();
      if (warp == 2 && lane < ar.world) {
        const uint32_t* fp = arb.flags + lane * snb_ar::kMaxCtas + tile;
        const uint64_t tw = snb::globaltimer_ns();
        while (snb_ar::ld_acquire_sys(fp) < ar_epoch) {
          if (snb::globaltimer_ns() - tw > SNB_WAIT_NS) {
            snb::record_status(status, SNB_ERR_TIMEOUT_PEER);
            ar_ok = 0;
            break;
          }
        }
      }
      bar_epilogue();
      const int f = f0 + q * 32 + lane;
      if (ar_ok && f < F) {
        for (int t = t0; t < min(T, t0 + BN); ++t) {
          float acc = 0.f;
          for (int p = 0; p < ar.world; ++p)
            acc += __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(
                snb_ar::ar_slot(ar.peers, ar.rank, ar_half, p, ar.world, ar.capacity))[(size_t)t * F + f]);
          out[(size_t)t * ldo + f] = __float2bfloat16(acc);
        }
      }
      bar_epilogue();
      if (warp == 2 && lane == 0) {
        __threadfence();
        const uint32_t tk = atomicAdd(arb.ticket, 1u);
        if (tk == gridDim.x * gridDim.y - 1) {
          *arb.counter = ar_epoch;
          *arb.ticket = 0;
          __threadfence();
        }
      }
    }
  }
  snb::tc_fence_before();
  __syncthreads();
  if (warp == 1) snb::tmem_dealloc(tmem, C::TMEM_COLS);
}

__global__ void splitk_reduce_kernel(const float* __restrict__ partial, const __nv_bfloat16* __restrict__ bias,
                                     __nv_bfloat16* __restrict__ out, int T, int F, int ldo, int splits) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * F) return;
  const int t = i / F, f = i % F;
  float a = bias != nullptr ? __bfloat162float(bias[f]) : 0.f;
  for (int z = 0; z < splits; ++z) a += partial[(size_t)z * T * F + i];
  out[(size_t)t * ldo + f] = __float2bfloat16(a);
}

template <int BN, bool AR = false>
void launch_gemm(const torch::Tensor& out, const torch::Tensor& x, const torch::Tensor& w,
                 const __nv_bfloat16* bias, int* status, cudaStream_t st, int splits, float* partial,
                 const GemmAR& ar = GemmAR{}) {
  using C = GemmCfg<BN>;
  const int T = x.size(0), K = x.size(1), F = w.size(0);
  CUtensorMap tw = snb_host::make_tmap_2d(w.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, K, F, w.stride(0) * 2, BK,
                                          BM, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tx = snb_host::make_tmap_2d(x.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, K, T, x.stride(0) * 2, BK,
                                          BN, CU_TENSOR_MAP_SWIZZLE_128B);
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(gemm_bf16_kernel<BN, AR>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    attr_set = true;
  }
  dim3 grid((F + BM - 1) / BM, (T + BN - 1) / BN, splits);
  gemm_bf16_kernel<BN, AR><<<grid, 192, C::SMEM, st>>>(tw, tx, (__nv_bfloat16*)out.data_ptr(), bias, F, T, K,
                                                       out.stride(0), status, splits > 1 ? partial : nullptr, ar);
  if (splits > 1) {
    const int n = T * F;
    splitk_reduce_kernel<<<(n + 255) / 256, 256, 0, st>>>(partial, bias, (__nv_bfloat16*)out.data_ptr(), T, F,
                                                          out.stride(0), splits);
  }
}

}  // namespace

// out: [T, F] bf16 (row stride arbitrary, multiple of 8), x: [T, K] bf16, w: [F, K] bf16, bias [F] or None.
// status: int32 CUDA tensor (>= 1 element) that receives a non-zero code if a bounded wait timed out.
void gemm_bf16(torch::Tensor out, torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias,
               torch::Tensor status, int64_t bn, int64_t splits, c10::optional<torch::Tensor> workspace) {
  const int T = x.size(0);
  if (T == 0) return;
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "gemm_bf16: bf16 inputs");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1 && out.stride(1) == 1, "gemm_bf16: inner stride");
  TORCH_CHECK(x.size(1) == w.size(1), "gemm_bf16: K mismatch");
  TORCH_CHECK(x.size(1) % 8 == 0, "gemm_bf16: K must be a multiple of 8");
  auto st = at::cuda::getCurrentCUDAStream();
  const __nv_bfloat16* bp = bias ? (const __nv_bfloat16*)bias->data_ptr() : nullptr;
  int* sp = status.data_ptr<int>();
  if (bn <= 0) bn = T <= 16 ? 16 : T <= 32 ? 32 : T <= 64 ? 64 : T <= 128 ? 128 : 256;
  if (splits < 1) splits = 1;
  float* part = nullptr;
  if (splits > 1) {
    TORCH_CHECK(workspace && workspace->scalar_type() == at::kFloat &&
                    workspace->numel() >= (int64_t)splits * T * w.size(0),
                "gemm_bf16: split-K needs a fp32 workspace of splits*T*F");
    part = workspace->data_ptr<float>();
  }
  switch (bn) {
    case 16: launch_gemm<16>(out, x, w, bp, sp, st, splits, part); break;
    case 32: launch_gemm<32>(out, x, w, bp, sp, st, splits, part); break;
    case 64: launch_gemm<64>(out, x, w, bp, sp, st, splits, part); break;
    case 128: launch_gemm<128>(out, x, w, bp, sp, st, splits, part); break;
    case 256: launch_gemm<256>(out, x, w, bp, sp, st, splits, part); break;
    default: TORCH_CHECK(false, "gemm_bf16: bn must be 16/32/64/128/256");
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// GEMM whose epilogue all-reduces the output over the TP group through the symmetric peer buffers
// (see gemm_bf16_kernel, AR = true). Requires one wave of CTAs (every tile co-resident) and T*F*2 bytes of
// buffer capacity; out: [T, F] contiguous.
void gemm_bf16_allreduce(torch::Tensor out, torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias,
                         torch::Tensor status, std::vector<int64_t> bufs, int64_t rank, int64_t capacity,
                         int64_t num_sms) {
  const int T = x.size(0), F = w.size(0);
  if (T == 0) return;
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "gemm_bf16_allreduce: bf16");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1 && out.is_contiguous(), "gemm_bf16_allreduce: layout");
  const int bn = T <= 16 ? 16 : T <= 32 ? 32 : T <= 64 ? 64 : T <= 128 ? 128 : 256;
  const int tiles = ((F + BM - 1) / BM) * ((T + bn - 1) / bn);
  TORCH_CHECK(tiles <= num_sms && tiles <= snb_ar::kMaxCtas, "gemm_bf16_allreduce: more tiles than one wave");
  TORCH_CHECK((size_t)T * F * 2 <= (size_t)capacity, "gemm_bf16_allreduce: over buffer capacity");
  GemmAR ar;
  ar.rank = rank;
  ar.world = (int)bufs.size();
  ar.capacity = capacity;
  TORCH_CHECK(ar.world >= 1 && ar.world <= snb_ar::kMaxRanks, "gemm_bf16_allreduce: world size");
  for (int i = 0; i < snb_ar::kMaxRanks; ++i)
    ar.peers.buf[i] = i < ar.world ? reinterpret_cast<uint8_t*>(bufs[i]) : nullptr;
  auto st = at::cuda::getCurrentCUDAStream();
  const __nv_bfloat16* bp = bias ? (const __nv_bfloat16*)bias->data_ptr() : nullptr;
  int* sp = status.data_ptr<int>();
  switch (bn) {
    case 16: launch_gemm<16, true>(out, x, w, bp, sp, st, 1, nullptr, ar); break;
    case 32: launch_gemm<32, true>(out, x, w, bp, sp, st, 1, nullptr, ar); break;
    case 64: launch_gemm<64, true>(out, x, w, bp, sp, st, 1, nullptr, ar); break;
    case 128: launch_gemm<128, true>(out, x, w, bp, sp, st, 1, nullptr, ar); break;
    default: launch_gemm<256, true>(out, x, w, bp, sp, st, 1, nullptr, ar); break;
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
