// Device side of the NVLink peer-memory collectives: the symmetric buffer layout and the publish / wait /
// reduce steps shared by the one-shot all-reduce, the fused MoE combine + all-reduce and the GEMM whose
// epilogue all-reduces its output tiles.
//
// Buffer of every rank: [2 halves][world slots][capacity bytes], then flags [kMaxRanks][kMaxCtas] (uint32),
// then the call epoch counter and a completion ticket. A call reads e = counter + 1 in every CTA, uses half
// (e & 1), and its last CTA to finish stores the counter.
#pragma once
#include <vector>
#include "common.cuh"

namespace snb_ar {

constexpr int kMaxRanks = 8;
constexpr int kMaxCtas = 1024;  // flag slots per rank (CTAs or output tiles of one call)

struct ARPeers {
  uint8_t* buf[kMaxRanks];  // mapped base of every rank's buffer (mine included)
  unsigned long long wait_ns;  // budget of each peer-flag wait (a runtime argument: tests make it short)
};

// Host: the peer table of a call; wait_ns <= 0 takes the default budget SNB_WAIT_NS.
inline ARPeers make_peers(const std::vector<int64_t>& bufs, int64_t wait_ns) {
  ARPeers p;
  for (int i = 0; i < kMaxRanks; ++i) p.buf[i] = i < (int)bufs.size() ? reinterpret_cast<uint8_t*>(bufs[i]) : nullptr;
  p.wait_ns = wait_ns > 0 ? (unsigned long long)wait_ns : (unsigned long long)SNB_WAIT_NS;
  return p;
}

SNB_DEVICE void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
SNB_DEVICE uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct ARBuf {
  uint8_t* mine;
  uint32_t* flags;    // [kMaxRanks][kMaxCtas] on my buffer
  uint32_t* counter;  // call epoch
  uint32_t* ticket;   // CTAs finished in the current call
};

SNB_DEVICE ARBuf ar_layout(const ARPeers& peers, int rank, int world, size_t capacity) {
  ARBuf b;
  b.mine = peers.buf[rank];
  b.flags = reinterpret_cast<uint32_t*>(b.mine + 2 * (size_t)world * capacity);
  b.counter = b.flags + kMaxRanks * kMaxCtas;
  b.ticket = b.counter + 1;
  return b;
}

SNB_DEVICE uint8_t* ar_slot(const ARPeers& peers, int peer, int half, int slot, int world, size_t capacity) {
  return peers.buf[peer] + ((size_t)half * world + slot) * capacity;
}

// After this CTA stored its chunk into every peer: publish, then wait (bounded) for every rank's chunk.
SNB_DEVICE bool ar_exchange(const ARPeers& peers, const ARBuf& b, int rank, int world, size_t capacity, uint32_t e,
                            int* status) {
  __shared__ int ok_s;
  __syncthreads();
  if (threadIdx.x == 0) ok_s = 1;
  if (threadIdx.x < world) {
    uint32_t* fp = reinterpret_cast<uint32_t*>(peers.buf[threadIdx.x] + 2 * (size_t)world * capacity);
    __threadfence_system();
    st_release_sys(fp + rank * kMaxCtas + blockIdx.x, e);
  }
  __syncthreads();
  if (threadIdx.x < world) {
    const uint32_t* fp = b.flags + threadIdx.x * kMaxCtas + blockIdx.x;
    const uint64_t t0 = snb::globaltimer_ns();
    while (ld_acquire_sys(fp) < e) {
      if (snb::globaltimer_ns() - t0 > peers.wait_ns) {
        snb::record_status(status, SNB_ERR_TIMEOUT_PEER);
        ok_s = 0;
        break;
      }
    }
  }
  __syncthreads();
  return ok_s != 0;
}

// The last CTA of the call advances the epoch (no CTA of the next call can start before this kernel ends).
SNB_DEVICE void ar_finish(const ARBuf& b, uint32_t e) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t t = atomicAdd(b.ticket, 1u);
    if (t == gridDim.x - 1) {
      *b.counter = e;
      *b.ticket = 0;
      __threadfence();
    }
  }
}

SNB_DEVICE void ar_reduce_store(const ARPeers& peers, int half, int world, size_t capacity, int rank,
                                __nv_bfloat16* __restrict__ out, int64_t v0, int64_t v1) {
  for (int64_t v = v0 + threadIdx.x; v < v1; v += blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int q = 0; q < world; ++q) {
      const uint4 u = reinterpret_cast<const uint4*>(ar_slot(peers, rank, half, q, world, capacity))[v];
      float f[8];
      snb::unpack_bf16x8(u, f);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += f[i];
    }
    reinterpret_cast<uint4*>(out)[v] = snb::pack_bf16x8(acc);
  }
}

// Residual add + RMSNorm fused into the reduce step: the CTA owns whole rows [r0, r1) of a [T, H] call.
// For each row: x = sum of the world's slots (fp32), residual <- x + residual (stored as bf16), and
// out <- (x + residual) * rsqrt(mean((x + residual)^2) + eps) * weight, from the fp32 sum. This is the
// add + norm that follows the all-reduce in a decoder layer (the output is the next block's input).
struct ARNorm {
  __nv_bfloat16* residual;      // [T, H], updated in place
  const __nv_bfloat16* weight;  // [H]
  float eps;
  int H;
};
constexpr int kNormVecs = 2;  // 8-wide vectors per thread per row: H <= kNormVecs * 8 * blockDim.x

SNB_DEVICE void ar_reduce_norm_store(const ARPeers& peers, int half, int world, size_t capacity, int rank,
                                     __nv_bfloat16* __restrict__ out, const ARNorm& nm, int r0, int r1) {
  __shared__ float red[32];
  const int hv = nm.H / 8;
  for (int t = r0; t < r1; ++t) {
    float acc[kNormVecs][8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kNormVecs; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      if (c >= hv) continue;
      const int64_t v = (int64_t)t * hv + c;
      float r[8];
      snb::unpack_bf16x8(reinterpret_cast<const uint4*>(nm.residual)[v], r);
      for (int q = 0; q < world; ++q) {
        const uint4 u = reinterpret_cast<const uint4*>(ar_slot(peers, rank, half, q, world, capacity))[v];
        float f[8];
        snb::unpack_bf16x8(u, f);
#pragma unroll
        for (int j = 0; j < 8; ++j) r[j] += f[j];
      }
      reinterpret_cast<uint4*>(nm.residual)[v] = snb::pack_bf16x8(r);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        acc[i][j] = r[j];
        ss += r[j] * r[j];
      }
    }
    ss = snb::warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
      float s2 = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
      s2 = snb::warp_sum(s2);
      if (threadIdx.x == 0) red[0] = s2;
    }
    __syncthreads();
    const float inv = rsqrtf(red[0] / (float)nm.H + nm.eps);
    __syncthreads();  // red[0] is rewritten by the next row
#pragma unroll
    for (int i = 0; i < kNormVecs; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      if (c >= hv) continue;
      float w[8];
      snb::unpack_bf16x8(reinterpret_cast<const uint4*>(nm.weight)[c], w);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] *= inv * w[j];
      reinterpret_cast<uint4*>(out)[(int64_t)t * hv + c] = snb::pack_bf16x8(acc[i]);
    }
  }
}

// Chunk of a call: vectors [v0, v1) of n8 = T * H / 8; with a fused norm the chunk is whole rows.
SNB_DEVICE void ar_chunk(int64_t nvec, int hv, bool rows, int64_t& v0, int64_t& v1, int& r0, int& r1) {
  if (rows) {
    const int T = (int)(nvec / hv);
    const int per = (T + gridDim.x - 1) / gridDim.x;
    r0 = min(T, (int)blockIdx.x * per);
    r1 = min(T, r0 + per);
    v0 = (int64_t)r0 * hv;
    v1 = (int64_t)r1 * hv;
  } else {
    const int64_t per = (nvec + gridDim.x - 1) / gridDim.x;
    v0 = min(nvec, (int64_t)blockIdx.x * per);
    v1 = min(nvec, v0 + per);
    r0 = r1 = 0;
  }
}

}  // namespace snb_ar
