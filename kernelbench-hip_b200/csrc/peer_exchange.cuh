// peer_exchange.cuh — the cross-GPU step of a sharded reduction, done by one
// CTA at the end of the kernel that computed this rank's partial.
//
// The sharded MSE, Frobenius and BatchNorm kernels reduce their shard to a
// handful of fp64 values (16 B, 8 B, 16 C + 8 B).  Instead of a separate
// collective launch, the CTA that finishes last (an arrival counter in the
// caller's workspace) folds the per-CTA partials in a fixed order and then
// exchanges the folded values over the communicator's peer buffers — the
// same buffers, slot/flag protocol and fault word as the standalone peer
// all-reduce in p2p.cu:
//   push   the values into slot (epoch & 1), part `rank`, of every rank's
//          buffer (posted stores over NVLink), then a system-scope fence;
//   flag   a release (one acq_rel fence per lane, then relaxed system-scope
//          stores, one peer per lane) of `epoch` into flags[slot][rank] of
//          every rank;
//   wait   (bounded by %globaltimer) until this rank's flags[slot][p] ==
//          epoch for every p;
//   sum    over p = 0 .. world-1 of part p, in rank order: bit-identical on
//          every rank.
// The slot of epoch e is written again only at epoch e + 2 (see p2p.cu for
// the argument), so the kernels can interleave with the standalone peer
// all-reduce on one communicator as long as every rank makes the same calls
// in the same order.  An expired wait records (phase << 8 | peer) in the
// fault word and yields NaN values.
#pragma once

#include "kb_common.cuh"

namespace kb {

constexpr size_t kPeerHeaderBytes = 4096;  // must match p2p.cu's header
constexpr int kPeerMaxRanks = 64;
// A fused sharded entry's workspace starts with its arrival counter: zero
// before the first call, and every call leaves it zero.
constexpr size_t kShardedCounterBytes = 256;

struct PeerHeader {
  unsigned flags[2][kPeerMaxRanks];
  unsigned bar_count;
  unsigned bar_gen;
};

// One rank's view of a communicator for one call.
struct PeerCtx {
  char* const* bufs;   // device array [world]: base of every rank's buffer
  int rank, world;
  size_t cap;          // bytes per rank part of a slot
  unsigned epoch;
  uint64_t timeout_ns;
  int* fault;          // device address of p2p.cu's fault word
};

// Device address of the peer fault word on the current device (p2p.cu).
int p2p_fault_address(int** out);
// Bytes per rank part of a slot of a peer buffer of buf_bytes (p2p.cu).
size_t p2p_part_cap(size_t buf_bytes, int world);

__device__ __forceinline__ uint64_t peer_now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// A fence.acq_rel.sys followed by relaxed system-scope stores is a release
// pattern for each of those stores (PTX memory model), so one fence per lane
// covers all of a lane's flag stores, and the lanes of a warp store their
// flags to different peers at the same time instead of one st.release
// (one fence) after another.
__device__ __forceinline__ void peer_fence_acq_rel() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void peer_store_relaxed(unsigned* p, unsigned v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned peer_load_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ size_t peer_part_off(unsigned slot, int p, int world, size_t cap) {
  return kPeerHeaderBytes + ((size_t)slot * world + p) * cap;
}

// Spin (one thread) until flags[slot][p] == epoch; false after timeout_ns or
// once the fault word is set.
__device__ inline bool peer_wait_flag(const PeerCtx& c, const unsigned* flag, int code) {
  if (peer_load_acquire(flag) == c.epoch) return true;
  const uint64_t t0 = peer_now_ns();
  for (unsigned it = 1;; ++it) {
    if (peer_load_acquire(flag) == c.epoch) return true;
    if ((it & 63) == 0) {
      if (*reinterpret_cast<volatile int*>(c.fault)) return false;
      if (peer_now_ns() - t0 > c.timeout_ns) {
        atomicCAS(c.fault, 0, code);
        return false;
      }
    }
  }
}

// All threads of one CTA: out[j] = sum over ranks of vals[j], j < n (vals
// and out may alias; n * 8 bytes <= c.cap, checked on the host).  Returns
// false (out = NaN) when a wait expired.
__device__ inline bool block_peer_allreduce(const PeerCtx& c, const double* vals, double* out, int n) {
  __shared__ int s_ok;
  const unsigned slot = c.epoch & 1u;
  const size_t mine = peer_part_off(slot, c.rank, c.world, c.cap);
  for (int i = threadIdx.x; i < n * c.world; i += blockDim.x) {
    const int p = i / n, j = i - p * n;
    reinterpret_cast<double*>(c.bufs[p] + mine)[j] = vals[j];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < 32) {
    // warp 0: the pushes of every thread are ordered before this point (their
    // system fence and the barrier); each lane releases the flag of peers
    // lane, lane + 32, ...
    peer_fence_acq_rel();
    for (int p = threadIdx.x; p < c.world; p += 32)
      peer_store_relaxed(&reinterpret_cast<PeerHeader*>(c.bufs[p])->flags[slot][c.rank], c.epoch);
    if (threadIdx.x == 0) {
      const PeerHeader* own = reinterpret_cast<const PeerHeader*>(c.bufs[c.rank]);
      bool ok = true;
      for (int p = 0; ok && p < c.world; ++p) ok = peer_wait_flag(c, &own->flags[slot][p], (2 << 8) | p);
      s_ok = ok ? 1 : 0;
    }
  }
  __syncthreads();
  if (!s_ok) {
    for (int j = threadIdx.x; j < n; j += blockDim.x) out[j] = NAN;
    __syncthreads();
    return false;
  }
  __threadfence_system();
  const char* own = c.bufs[c.rank];
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    double acc = 0.0;
    for (int p = 0; p < c.world; ++p)
      acc += __ldcv(reinterpret_cast<const double*>(own + peer_part_off(slot, p, c.world, c.cap)) + j);
    out[j] = acc;
  }
  __syncthreads();
  return true;
}

// The arrival counter of a sharded kernel: every CTA calls this once after
// its partial is written (thread 0 does the atomic); true in the CTA that
// arrived last, which then sees every other CTA's partial.  The last CTA
// resets the counter to zero for the next launch.
__device__ inline bool last_cta_arrives(unsigned* counter) {
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned total = gridDim.x * gridDim.y * gridDim.z;
    const unsigned old = atomicAdd(counter, 1u);
    s_last = (old == total - 1) ? 1 : 0;
    if (s_last) *counter = 0;
  }
  __syncthreads();
  if (s_last) __threadfence();
  return s_last != 0;
}

}  // namespace kb
