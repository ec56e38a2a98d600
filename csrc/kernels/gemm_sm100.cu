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
#include <algorithm>
#include <cstdlib>

namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // bf16 elements per 128-byte swizzled row

// OCC = CTAs per SM: 1 (a ~200 KB ring) or 2 (two ~100 KB rings: decode-sized GEMMs split K over up to
// twice as many CTAs, so more SMs stream the weights at once).
template <int BN, int OCC = 1>
struct GemmCfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int BUDGET = OCC == 2 ? 100 * 1024 : 200 * 1024;
  static constexpr int STAGES = BUDGET / STAGE_BYTES > 8 ? 8 : BUDGET / STAGE_BYTES;
  static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

// Split-K: blockIdx.z selects a contiguous range of K blocks. Decode-sized GEMMs (few tokens, F/128 tiles)
// split K so every SM works on the weight stream. Default (cluster_reduce): the S splits of a tile form one
// (1, 1, S) thread-block cluster and are summed through distributed shared memory in the same kernel.
// Explicit split counts instead write fp32 partial tiles to `partial` [splits, T, F], summed by
// splitk_reduce_kernel or by a fused consumer (the tensor-parallel all-reduce).
// Programmatic dependent launch: the producer issues the weight loads of the first ring slots before
// griddepcontrol.wait, so the weight stream starts while the previous kernel is still running.
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

// Grouped (per-head) mode: output rows f of group g = f / x_rows contract over x columns
// [g * x_stride, g * x_stride + K) (each head multiplies its own slice of x), and output column f lands at
// (f / o_rows) * o_stride + f % o_rows of `out` (a head's block inside a wider row). x_rows = 0: plain GEMM.
// DeepSeek-V2's absorbed attention uses it: q_nope . W_UK and o_latent . W_UV for every head in one launch.
struct GemmGroup {
  int x_rows, x_stride, o_rows, o_stride;
};

SNB_DEVICE int group_col(const GemmGroup& g, int f) {
  return g.o_rows ? (f / g.o_rows) * g.o_stride + f % g.o_rows : f;
}

template <int BN, bool AR, int OCC = 1>
__global__ void __launch_bounds__(192, OCC)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                     __nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ bias, int F, int T,
                     int K, int ldo, int* status, float* __restrict__ partial, const GemmAR ar, int cluster_reduce,
                     int w_tiled, const GemmGroup grp) {
  using C = GemmCfg<BN, OCC>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + C::STAGES * C::B_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* accum = empty + C::STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  int* loads = reinterpret_cast<int*>(tmem_slot + 1);  // [0] issued, [1] consumed

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int f0 = blockIdx.x * BM, t0 = blockIdx.y * BN;
  const int nk_all = (K + BK - 1) / BK;
  const int S = gridDim.z;
  const int kb0 = (int)((long long)blockIdx.z * nk_all / S);
  const int nk = (int)((long long)(blockIdx.z + 1) * nk_all / S) - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      snb::mbar_init(&full[s], 1);
      snb::mbar_init(&empty[s], 1);
    }
    snb::mbar_init(accum, 1);
    loads[0] = loads[1] = 0;
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
  snb::pdl_trigger();
  bool ep_ok = false;

  if (warp == 0) {
    if (lane == 0) {
      // Weight tile (kb, f0): row-major [F, K] weights, or pre-tiled ones where each 128 x 64 tile is one
      // contiguous 16 KB block ([F/128][K/64][128][64]) so every load is a single DRAM stream.
      // Decode grids (one token tile) read each weight byte once: evict-first keeps L2 for activations.
      const uint64_t pol = snb::l2_policy_evict_first();
      const bool once = gridDim.y == 1;
      auto load_w = [&](int s, int kb) {
        const int c0 = w_tiled ? 0 : (kb0 + kb) * BK;
        const int c1 = w_tiled ? (blockIdx.x * nk_all + kb0 + kb) * BM : f0;
        if (once) snb::tma_load_2d_hint(sA + s * C::A_BYTES, &tmap_w, &full[s], c0, c1, pol);
        else snb::tma_load_2d(sA + s * C::A_BYTES, &tmap_w, &full[s], c0, c1);
      };
      // The weights are constant: the first ring slots are filled before waiting for the previous kernel.
      const int npre = min(nk, C::STAGES);
      for (int kb = 0; kb < npre; ++kb) {
        snb::mbar_arrive_expect_tx(&full[kb], C::STAGE_BYTES);
        load_w(kb, kb);
      }
      snb::pdl_wait();
      const int xoff = grp.x_rows ? (f0 / grp.x_rows) * grp.x_stride : 0;
      int issued = npre;
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % C::STAGES;
        const uint32_t ph = (kb / C::STAGES) & 1;
        if (kb >= npre) {
          if (!snb::mbar_wait_bounded(&empty[s], ph ^ 1, status, SNB_ERR_TIMEOUT_TMA)) break;
          snb::mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
          load_w(s, kb);
          issued = kb + 1;
        }
        snb::tma_load_2d(sB + s * C::B_BYTES, &tmap_x, &full[s], (kb0 + kb) * BK + xoff, t0);
      }
      loads[0] = issued;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = snb::idesc_bf16_f32(BM, BN);
      bool ok = true;
      int kb = 0;
      for (; kb < nk; ++kb) {
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
      loads[1] = kb;
      // with ok, the epilogue waits on `accum`; otherwise this commit lets in-flight MMAs be waited for below
      snb::mma_commit(accum);
      if (!ok) snb::mbar_wait_bounded(accum, 0, status, SNB_ERR_TIMEOUT_MMA);
    }
  } else {
    snb::pdl_wait();
    // Epilogue warps 2..5: warp w reads TMEM lanes 32*(w%4) .. +31.
    const int q = warp & 3;
    const bool ok = nk > 0 && snb::mbar_wait_bounded(accum, 0, status, SNB_ERR_TIMEOUT_EPI);
    ep_ok = ok;
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
    if (ok && !cluster_reduce) {
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
              if (t < T) out[(size_t)t * ldo + group_col(grp, f)] = __float2bfloat16(__uint_as_float(r[j]) + bf);
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
          if (snb::globaltimer_ns() - tw > ar.peers.wait_ns) {
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
  if (cluster_reduce) {
    // Split-K inside a (1, 1, S) cluster, reduced by a reduce-scatter over distributed shared memory: the
    // tile's BN columns are cut into S contiguous ranges of 4-column groups, CTA r owns range r. After the
    // first cluster barrier every CTA's MMAs are done (its ring is free); each CTA stores every 4-column
    // group of its TMEM tile into the owner's ring, slot = its own rank ([src][128 rows][RS] fp32, 16-byte
    // stores, odd 16-byte row stride: conflict-free). After the second barrier each CTA sums its groups over
    // the S slots in rank order (deterministic), adds the bias and writes bf16. Every SM moves about
    // (S - 1)/S of one tile instead of one SM receiving S - 1 tiles.
    constexpr int NG = BN / 4;
    constexpr int CH = BN >= 32 ? 32 : BN;
    const int maxg = (NG + S - 1) / S;
    const int rs = 4 * (maxg + ((maxg & 1) ? 2 : 1));  // floats per row: odd number of 16-byte units
    __syncwarp();
    snb::tc_fence_before();
    snb::cluster_sync();
    snb::tc_fence_after();
    const int rank = (int)snb::cluster_ctarank();
    const int q = warp & 3, fl = q * 32 + lane;
    if (warp >= 2 && ep_ok) {
      const uint32_t my_slot = snb::smem_u32(smem) + (uint32_t)((rank * BM + fl) * rs) * 4u;
      int owner = 0;
#pragma unroll 1
      for (int c = 0; c < BN / CH; ++c) {
        uint32_t r[CH];
        if constexpr (CH == 32) {
          snb::tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + c * CH, r);
          snb::tmem_ld_wait();
        } else {
          uint32_t r8[8];
#pragma unroll
          for (int h = 0; h < CH / 8; ++h) {
            snb::tmem_ld_32x32b_x8(tmem + ((uint32_t)(q * 32) << 16) + c * CH + h * 8, r8);
            snb::tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 8; ++j) r[h * 8 + j] = r8[j];
          }
        }
#pragma unroll
        for (int j = 0; j < CH / 4; ++j) {
          const int g = c * (CH / 4) + j;
          while (owner + 1 < S && (owner + 1) * NG / S <= g) ++owner;
          const int gl = g - owner * NG / S;
          const uint32_t dst = snb::mapa_shared(my_slot + (uint32_t)(gl * 16), (uint32_t)owner);
          snb::st_cluster_v4(dst, __uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                             __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
        }
      }
    }
    __syncwarp();
    snb::cluster_sync();
    if (warp >= 2 && ep_ok) {
      const int f = f0 + fl;
      const float bf = (bias != nullptr && f < F) ? __bfloat162float(bias[f]) : 0.f;
      const int g0 = rank * NG / S, g1 = (rank + 1) * NG / S;
      const float* rows = reinterpret_cast<const float*>(smem) + fl * rs;
      for (int g = g0; g < g1; ++g) {
        float4 acc = make_float4(bf, bf, bf, bf);
        for (int src = 0; src < S; ++src) {
          const float4 v = *reinterpret_cast<const float4*>(rows + (size_t)src * BM * rs + (g - g0) * 4);
          acc.x += v.x;
          acc.y += v.y;
          acc.z += v.z;
          acc.w += v.w;
        }
        if (f < F) {
          const int t = t0 + g * 4, oc = group_col(grp, f);
          if (t < T) out[(size_t)t * ldo + oc] = __float2bfloat16(acc.x);
          if (t + 1 < T) out[(size_t)(t + 1) * ldo + oc] = __float2bfloat16(acc.y);
          if (t + 2 < T) out[(size_t)(t + 2) * ldo + oc] = __float2bfloat16(acc.z);
          if (t + 3 < T) out[(size_t)(t + 3) * ldo + oc] = __float2bfloat16(acc.w);
        }
      }
    }
  }
  snb::tc_fence_before();
  __syncthreads();
  if (warp == 0 && lane == 0) {
    // a CTA that stopped early still waits (bounded) for the loads it issued before its memory goes away
    for (int i = loads[1]; i < loads[0]; ++i)
      if (!snb::mbar_wait_bounded(&full[i % C::STAGES], (i / C::STAGES) & 1, status, SNB_ERR_TIMEOUT_TMA)) break;
  }
  if (warp == 1) snb::tmem_dealloc(tmem, C::TMEM_COLS);
}

__global__ void splitk_reduce_kernel(const float* __restrict__ partial, const __nv_bfloat16* __restrict__ bias,
                                     __nv_bfloat16* __restrict__ out, int T, int F, int ldo, int splits) {
  snb::pdl_wait();
  snb::pdl_trigger();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * F) return;
  const int t = i / F, f = i % F;
  float a = bias != nullptr ? __bfloat162float(bias[f]) : 0.f;
  for (int z = 0; z < splits; ++z) a += partial[(size_t)z * T * F + i];
  out[(size_t)t * ldo + f] = __float2bfloat16(a);
}

// Largest split count (<= 8, the portable cluster size) whose reduce-scatter slots
// (S x 128 rows x rs floats) fit in the ring.
template <int BN, int OCC = 1>
int max_cluster_splits() {
  using C = GemmCfg<BN, OCC>;
  int best = 1;
  for (int S = 2; S <= 8; ++S) {
    const int ng = BN / 4, maxg = (ng + S - 1) / S;
    const int rs = 4 * (maxg + ((maxg & 1) ? 2 : 1));
    if (S * BM * rs * 4 <= C::STAGES * C::STAGE_BYTES) best = S;
  }
  return best;
}

// Split count for the in-cluster reduction: as many K splits as keep every tile's cluster co-resident in
// one wave (checked with the occupancy calculator once per shape class).
template <int BN, int OCC = 1>
int pick_cluster_splits(int tiles, int nk, int num_sms) {
  using C = GemmCfg<BN, OCC>;
  if (tiles * 2 > num_sms * OCC) return 1;
  int S = std::min({max_cluster_splits<BN, OCC>(), num_sms * OCC / tiles, nk});
  static int max_clusters[9] = {0};
  while (S > 1) {
    if (max_clusters[S] == 0) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(1, 1, S);
      cfg.blockDim = dim3(192);
      cfg.dynamicSmemBytes = C::SMEM;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 1;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = S;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, gemm_bf16_kernel<BN, false, OCC>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        n = -1;
      }
      max_clusters[S] = n;
    }
    if (max_clusters[S] >= tiles) break;
    --S;
  }
  return S;
}

template <int BN, bool AR = false>
void launch_gemm(const torch::Tensor& out, const torch::Tensor& x, const torch::Tensor& w,
                 const __nv_bfloat16* bias, int* status, cudaStream_t st, int splits, float* partial,
                 const GemmAR& ar = GemmAR{}, bool reduce_partials = true, int num_sms = 148, int tiled_f = 0,
                 const GemmGroup grp = GemmGroup{0, 0, 0, 0}, int group_k = 0) {
  using C = GemmCfg<BN>;
  const int T = x.size(0), K = grp.x_rows ? group_k : (int)x.size(1), F = tiled_f ? tiled_f : w.size(0);
  const int wt = tiled_f ? 1 : 0;
  CUtensorMap tw = tiled_f ? snb_host::make_tmap_2d(w.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, BK, w.size(0),
                                                    BK * 2, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B)
                           : snb_host::make_tmap_2d(w.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, K, F,
                                                    w.stride(0) * 2, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tx = snb_host::make_tmap_2d(x.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x.size(1), T,
                                          x.stride(0) * 2, BK, BN, CU_TENSOR_MAP_SWIZZLE_128B);
  static bool attr_set = false;
  if (!attr_set) {
    C10_CUDA_CHECK(
        cudaFuncSetAttribute(gemm_bf16_kernel<BN, AR>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    attr_set = true;
  }
  const int tiles_f = (F + BM - 1) / BM, tiles_t = (T + BN - 1) / BN;
  __nv_bfloat16* op = (__nv_bfloat16*)out.data_ptr();
  const int ldo = out.stride(0);
  if (splits <= 0) {
    // default: split K inside a thread-block cluster when the tiles alone leave SMs idle
    int S = 1;
    if constexpr (!AR) S = pick_cluster_splits<BN>(tiles_f * tiles_t, (K + BK - 1) / BK, num_sms);
    if constexpr (!AR && BN <= 64) {
      // two CTAs per SM when that splits K over more SMs than one CTA per SM can
      using C2 = GemmCfg<BN, 2>;
      static const bool use2 = [] {
        const char* e = std::getenv("SGLANG_B200_GEMM_2CTA");
        return !(e != nullptr && e[0] == '0');
      }();
      static bool attr2 = false;
      if (use2 && !attr2) {  // before the occupancy query, which needs the shared-memory size allowed
        C10_CUDA_CHECK(cudaFuncSetAttribute(gemm_bf16_kernel<BN, false, 2>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, C2::SMEM));
        attr2 = true;
      }
      const int S2 = use2 ? pick_cluster_splits<BN, 2>(tiles_f * tiles_t, (K + BK - 1) / BK, num_sms) : 1;
      if (use2 && S2 > S) {
        C10_CUDA_CHECK(snb::launch_pdl_cluster(gemm_bf16_kernel<BN, false, 2>, dim3(tiles_f, tiles_t, S2), 192,
                                               C2::SMEM, st, S2, tw, tx, op, bias, F, T, K, ldo, status, nullptr, ar,
                                               1, wt, grp));
        return;
      }
    }
    if (S > 1) {
      C10_CUDA_CHECK(snb::launch_pdl_cluster(gemm_bf16_kernel<BN, AR>, dim3(tiles_f, tiles_t, S), 192, C::SMEM, st,
                                             S, tw, tx, op, bias, F, T, K, ldo, status, nullptr, ar, 1, wt, grp));
    } else {
      C10_CUDA_CHECK(snb::launch_pdl(gemm_bf16_kernel<BN, AR>, dim3(tiles_f, tiles_t, 1), 192, C::SMEM, st, tw, tx,
                                     op, bias, F, T, K, ldo, status, nullptr, ar, 0, wt, grp));
    }
    return;
  }
  C10_CUDA_CHECK(snb::launch_pdl(gemm_bf16_kernel<BN, AR>, dim3(tiles_f, tiles_t, splits), 192, C::SMEM, st, tw, tx,
                                 op, bias, F, T, K, ldo, status, splits > 1 ? partial : nullptr, ar, 0, wt, grp));
  if (splits > 1 && reduce_partials) {
    const int n = T * F;
    C10_CUDA_CHECK(snb::launch_pdl(splitk_reduce_kernel, (n + 255) / 256, 256, 0, st, partial, bias, op, T, F, ldo,
                                   splits));
  }
}

}  // namespace

// out: [T, F] bf16 (row stride arbitrary, multiple of 8), x: [T, K] bf16, w: [F, K] bf16, bias [F] or None.
// status: int32 CUDA tensor (>= 1 element) that receives a non-zero code if a bounded wait timed out.
// splits <= 0: automatic (K split inside a thread-block cluster for decode-sized GEMMs, one launch);
// splits == 1: one CTA per tile; splits > 1: fp32 partials [splits, T, F] in `workspace`, summed by a second
// launch when reduce_partials (else left for a fused consumer).
static void check_weight(const torch::Tensor& x, const torch::Tensor& w, int64_t tiled_f, const char* who) {
  if (tiled_f > 0) {
    const int64_t nk = (x.size(1) + BK - 1) / BK, ntf = (tiled_f + BM - 1) / BM;
    TORCH_CHECK(w.dim() == 2 && w.size(1) == BK && w.size(0) == ntf * nk * BM && w.is_contiguous(), who,
                ": tiled weight must be [ceil(F/128) * ceil(K/64) * 128, 64]");
  } else {
    TORCH_CHECK(x.size(1) == w.size(1), who, ": K mismatch");
  }
}

// tiled_f > 0: `w` is the pre-tiled layout of a [tiled_f, K] weight (see tile_weight_bf16 in ops/gemm.py).
void gemm_bf16(torch::Tensor out, torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias,
               torch::Tensor status, int64_t bn, int64_t splits, c10::optional<torch::Tensor> workspace,
               bool reduce_partials, int64_t tiled_f) {
  const int T = x.size(0);
  if (T == 0) return;
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "gemm_bf16: bf16 inputs");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1 && out.stride(1) == 1, "gemm_bf16: inner stride");
  check_weight(x, w, tiled_f, "gemm_bf16");
  TORCH_CHECK(x.size(1) % 8 == 0, "gemm_bf16: K must be a multiple of 8");
  auto st = at::cuda::getCurrentCUDAStream();
  const __nv_bfloat16* bp = bias ? (const __nv_bfloat16*)bias->data_ptr() : nullptr;
  int* sp = status.data_ptr<int>();
  if (bn <= 0) bn = T <= 16 ? 16 : T <= 32 ? 32 : T <= 64 ? 64 : T <= 128 ? 128 : 256;
  const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  float* part = nullptr;
  if (splits > 1) {
    TORCH_CHECK(workspace && workspace->scalar_type() == at::kFloat &&
                    workspace->numel() >= (int64_t)splits * T * (tiled_f ? tiled_f : w.size(0)),
                "gemm_bf16: split-K needs a fp32 workspace of splits*T*F");
    part = workspace->data_ptr<float>();
  }
  switch (bn) {
    case 16: launch_gemm<16>(out, x, w, bp, sp, st, splits, part, GemmAR{}, reduce_partials, sms, tiled_f); break;
    case 32: launch_gemm<32>(out, x, w, bp, sp, st, splits, part, GemmAR{}, reduce_partials, sms, tiled_f); break;
    case 64: launch_gemm<64>(out, x, w, bp, sp, st, splits, part, GemmAR{}, reduce_partials, sms, tiled_f); break;
    case 128: launch_gemm<128>(out, x, w, bp, sp, st, splits, part, GemmAR{}, reduce_partials, sms, tiled_f); break;
    case 256: launch_gemm<256>(out, x, w, bp, sp, st, splits, part, GemmAR{}, reduce_partials, sms, tiled_f); break;
    default: TORCH_CHECK(false, "gemm_bf16: bn must be 16/32/64/128/256");
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Grouped (per-head) GEMM, see GemmGroup: out[t, oc(f)] = sum_k x[t, (f / x_rows) * x_stride + k] * w[f, k]
// for k < group_k. w: tiled [tiled_f, group_k] weight; x_rows and o_rows multiples of 128, group_k of 64.
void gemm_bf16_grouped(torch::Tensor out, torch::Tensor x, torch::Tensor w, int64_t tiled_f, torch::Tensor status,
                       int64_t group_k, int64_t x_rows, int64_t x_stride, int64_t o_rows, int64_t o_stride) {
  const int T = x.size(0);
  if (T == 0) return;
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16,
              "gemm_bf16_grouped: bf16");
  TORCH_CHECK(x.stride(1) == 1 && out.stride(1) == 1 && w.is_contiguous(), "gemm_bf16_grouped: inner stride");
  TORCH_CHECK(group_k % BK == 0 && x_rows % BM == 0 && x_rows > 0 && (o_rows == 0 || o_rows % BM == 0) &&
                  tiled_f % x_rows == 0 && x_stride % 8 == 0, "gemm_bf16_grouped: group shape");
  TORCH_CHECK((tiled_f / x_rows - 1) * x_stride + group_k <= x.size(1), "gemm_bf16_grouped: x too narrow");
  const int64_t ntf = (tiled_f + BM - 1) / BM, nk = group_k / BK;
  TORCH_CHECK(w.dim() == 2 && w.size(1) == BK && w.size(0) == ntf * nk * BM, "gemm_bf16_grouped: tiled weight");
  const GemmGroup grp{(int)x_rows, (int)x_stride, (int)o_rows, (int)o_stride};
  auto st = at::cuda::getCurrentCUDAStream();
  int* sp = status.data_ptr<int>();
  const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  const int bn = T <= 16 ? 16 : T <= 32 ? 32 : T <= 64 ? 64 : T <= 128 ? 128 : 256;
  switch (bn) {
    case 16: launch_gemm<16>(out, x, w, nullptr, sp, st, 0, nullptr, GemmAR{}, true, sms, tiled_f, grp, group_k); break;
    case 32: launch_gemm<32>(out, x, w, nullptr, sp, st, 0, nullptr, GemmAR{}, true, sms, tiled_f, grp, group_k); break;
    case 64: launch_gemm<64>(out, x, w, nullptr, sp, st, 0, nullptr, GemmAR{}, true, sms, tiled_f, grp, group_k); break;
    case 128: launch_gemm<128>(out, x, w, nullptr, sp, st, 0, nullptr, GemmAR{}, true, sms, tiled_f, grp, group_k); break;
    default: launch_gemm<256>(out, x, w, nullptr, sp, st, 0, nullptr, GemmAR{}, true, sms, tiled_f, grp, group_k); break;
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// GEMM whose epilogue all-reduces the output over the TP group through the symmetric peer buffers
// (see gemm_bf16_kernel, AR = true). Requires one wave of CTAs (every tile co-resident) and T*F*2 bytes of
// buffer capacity; out: [T, F] contiguous.
void gemm_bf16_allreduce(torch::Tensor out, torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias,
                         torch::Tensor status, std::vector<int64_t> bufs, int64_t rank, int64_t capacity,
                         int64_t num_sms, int64_t tiled_f) {
  const int T = x.size(0), F = tiled_f ? tiled_f : w.size(0);
  if (T == 0) return;
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "gemm_bf16_allreduce: bf16");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1 && out.is_contiguous(), "gemm_bf16_allreduce: layout");
  check_weight(x, w, tiled_f, "gemm_bf16_allreduce");
  const int bn = T <= 16 ? 16 : T <= 32 ? 32 : T <= 64 ? 64 : T <= 128 ? 128 : 256;
  const int tiles = ((F + BM - 1) / BM) * ((T + bn - 1) / bn);
  TORCH_CHECK(tiles <= num_sms && tiles <= snb_ar::kMaxCtas, "gemm_bf16_allreduce: more tiles than one wave");
  TORCH_CHECK((size_t)T * F * 2 <= (size_t)capacity, "gemm_bf16_allreduce: over buffer capacity");
  GemmAR ar;
  ar.rank = rank;
  ar.world = (int)bufs.size();
  ar.capacity = capacity;
  TORCH_CHECK(ar.world >= 1 && ar.world <= snb_ar::kMaxRanks, "gemm_bf16_allreduce: world size");
  ar.peers = snb_ar::make_peers(bufs, 0);
  auto st = at::cuda::getCurrentCUDAStream();
  const __nv_bfloat16* bp = bias ? (const __nv_bfloat16*)bias->data_ptr() : nullptr;
  int* sp = status.data_ptr<int>();
  switch (bn) {
    case 16: launch_gemm<16, true>(out, x, w, bp, sp, st, 1, nullptr, ar, true, num_sms, tiled_f); break;
    case 32: launch_gemm<32, true>(out, x, w, bp, sp, st, 1, nullptr, ar, true, num_sms, tiled_f); break;
    case 64: launch_gemm<64, true>(out, x, w, bp, sp, st, 1, nullptr, ar, true, num_sms, tiled_f); break;
    case 128: launch_gemm<128, true>(out, x, w, bp, sp, st, 1, nullptr, ar, true, num_sms, tiled_f); break;
    default: launch_gemm<256, true>(out, x, w, bp, sp, st, 1, nullptr, ar, true, num_sms, tiled_f); break;
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
