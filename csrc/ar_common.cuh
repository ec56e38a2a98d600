// Device side of the NVLink peer-memory collectives: the symmetric buffer layout and the publish / wait /
// reduce steps shared by the one-shot all-reduce, the fused MoE combine + all-reduce and the GEMM whose
// epilogue all-reduces its output tiles.
//
// Buffer of every rank: [2 halves][world slots][capacity bytes], then flags [kMaxRanks][kMaxCtas] (uint32),
// then the call epoch counter and a completion ticket. A call reads e = counter + 1 in every CTA, uses half
// (e & 1), and its last CTA to finish stores the counter.
#pragma once
#include "common.cuh"

namespace snb_ar {

constexpr int kMaxRanks = 8;
constexpr int kMaxCtas = 1024;  // flag slots per rank (CTAs or output tiles of one call)

struct ARPeers {
  uint8_t* buf[kMaxRanks];  // mapped base of every rank's buffer (mine included)
};

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
      if (snb::globaltimer_ns() - t0 > SNB_WAIT_NS) {
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


}  // namespace snb_ar
