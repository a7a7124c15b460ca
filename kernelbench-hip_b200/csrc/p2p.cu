// p2p.cu — all-reduce over peer GPU memory for the sharded ops, one kernel
// per call, fused with the local finishing step (for split-K: the reduction
// of this rank's own K splits).
//
// Each rank owns one symmetric buffer (same size on every rank, cudaMalloc'd
// here, zeroed once), opened by the peers through CUDA IPC (peer access over
// NVLink; no multicast objects, no NVLS).  Layout, with cap bytes per rank:
//   [0, 4 KiB)                 header: flags[2][kMaxRanks] (flags[s][p] = the
//                              epoch at which rank p's data for slot s
//                              arrived here, written by p), grid-barrier
//                              count and generation
//   [4 KiB + (s * world + p) * cap, + cap)   slot s, data pushed by rank p
// A call with epoch e uses slot s = e & 1 and runs as one kernel
// (cooperative when it has more than one CTA, so all CTAs are co-resident):
//   1. push: this rank's contribution (for split-K: the fixed-order sum of
//      its K-split partial tiles) is stored into slot s, part `rank`, of
//      every rank's buffer — posted writes over NVLink;
//   2. system-scope fence, then a grid barrier (bounded wait);
//   3. CTA 0 publishes: a release of e into flags[s][rank] of every rank
//      (one acq_rel fence per lane of warp 0, then relaxed system-scope
//      stores, the lanes covering different ranks at the same time);
//   4. every CTA waits (bounded) until its own flags[s][p] == e for every p;
//   5. dst[i] = sum over p = 0 .. world-1 of part p of its own slot s, in
//      rank order (local reads): every rank computes bit-identical results.
// Slot reuse is safe: rank q writes part q of slot e & 1 again only in call
// e + 2, after its call e + 1 saw every rank's signal, which each rank sends
// only after its call e (and so its reads of slot e & 1) completed.
// Every wait is bounded by %globaltimer; on expiry the kernel records a
// fault word (kb_p2p_read_fault), fills dst with NaN (an in-place call would
// otherwise leave this rank's own partial there, a plausible wrong answer),
// and the buffer set must be discarded (its barrier state is no longer
// consistent).
#include <string.h>

#include "kb_common.cuh"
#include "peer_exchange.cuh"

namespace kb {

__device__ int g_p2p_fault = 0;  // (phase << 8) | peer of the first expired wait, 0 = none

namespace {

constexpr int kMaxRanks = 64;
constexpr size_t kHeaderBytes = 4096;
constexpr int kP2PThreads = 256;

struct Header {
  unsigned flags[2][kMaxRanks];
  unsigned bar_count;
  unsigned bar_gen;
};
static_assert(sizeof(Header) <= kHeaderBytes, "header");

struct P2PArgs {
  char* const* bufs;   // device array [world]: base of every rank's buffer (own at [rank])
  int rank, world;
  size_t cap;          // bytes per rank part of a slot
  int64_t n;           // elements
  const void* src;     // mode 0: n elements; mode 1: `splits` fp32 partials of n, stride n
  int splits;
  void* dst;
  unsigned epoch;
  uint64_t timeout_ns;
};

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned load_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned load_volatile(const unsigned* p) {
  return *reinterpret_cast<const volatile unsigned*>(p);
}

// Spin until `ready()`; false (and the fault word set) after timeout_ns or
// once another CTA has recorded a fault.
template <class Ready>
__device__ bool bounded_wait(Ready ready, uint64_t timeout_ns, int code) {
  if (ready()) return true;
  const uint64_t t0 = now_ns();
  for (unsigned it = 1;; ++it) {
    if (ready()) return true;
    if ((it & 63) == 0) {
      if (*reinterpret_cast<volatile int*>(&g_p2p_fault)) return false;
      if (now_ns() - t0 > timeout_ns) {
        atomicCAS(&g_p2p_fault, 0, code);
        return false;
      }
    }
  }
}

template <class T>
__device__ __forceinline__ T load_cv(const T* p) {
  return __ldcv(p);
}

// offset of part p of slot s
__device__ __forceinline__ size_t part_off(unsigned s, int p, int world, size_t cap) {
  return kHeaderBytes + ((size_t)s * world + p) * cap;
}

template <class T, int MODE>
__global__ void __launch_bounds__(kP2PThreads) p2p_allreduce_kernel(P2PArgs a) {
  __shared__ int s_ok;
  const unsigned slot = a.epoch & 1u;
  Header* mine_h = reinterpret_cast<Header*>(a.bufs[a.rank]);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t my_part = part_off(slot, a.rank, a.world, a.cap);

  // 1. push this rank's contribution into part `rank` of every rank's slot
  for (int64_t i = i0; i < a.n; i += stride) {
    T v;
    if (MODE == 0) {
      v = static_cast<const T*>(a.src)[i];
    } else {
      const float* part = static_cast<const float*>(a.src);
      float s = 0.f;
#pragma unroll 8
      for (int z = 0; z < a.splits; ++z) s += part[(int64_t)z * a.n + i];  // split order; loads run ahead
      v = s;
    }
    for (int p = 0; p < a.world; ++p) reinterpret_cast<T*>(a.bufs[p] + my_part)[i] = v;
  }

  // 2. the pushes are visible system-wide, then a grid barrier
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < 32) {
    bool ok = true;
    if (threadIdx.x == 0 && gridDim.x > 1) {
      const unsigned old = atomicAdd(&mine_h->bar_count, 1u);
      if (old == gridDim.x - 1) {
        mine_h->bar_count = 0;
        __threadfence();
        atomicExch(&mine_h->bar_gen, a.epoch);
      } else {
        ok = bounded_wait([&] { return load_volatile(&mine_h->bar_gen) == a.epoch; }, a.timeout_ns,
                          (1 << 8) | a.rank);
      }
    }
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    __syncwarp();  // orders lane 0's view of the grid barrier before every lane's fence
    // 3. tell every rank that this rank's part has arrived: one acq_rel
    //    fence per lane, then relaxed system-scope flag stores (a release
    //    pattern), lane p signalling peers p, p + 32, ... in parallel
    if (ok && blockIdx.x == 0) {
      __threadfence_system();
      asm volatile("fence.acq_rel.sys;" ::: "memory");
      for (int p = threadIdx.x; p < a.world; p += 32) {
        Header* h = reinterpret_cast<Header*>(a.bufs[p]);
        asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(&h->flags[slot][a.rank]), "r"(a.epoch)
                     : "memory");
      }
    }
    // 4. wait for every rank's slot
    if (threadIdx.x == 0) {
      for (int p = 0; ok && p < a.world; ++p)
        ok = bounded_wait([&] { return load_acquire_sys(&mine_h->flags[slot][p]) == a.epoch; },
                          a.timeout_ns, (2 << 8) | p);
      s_ok = ok ? 1 : 0;
    }
  }
  __syncthreads();
  T* dst = static_cast<T*>(a.dst);
  if (!s_ok) {  // an expired wait: NaN, so a failed exchange cannot pass for a local result
    for (int64_t i = i0; i < a.n; i += stride) dst[i] = T(NAN);
    return;
  }
  __threadfence_system();

  // 5. rank-ordered sum of the parts that arrived in this rank's slot
  const char* own = a.bufs[a.rank];
  for (int64_t i = i0; i < a.n; i += stride) {
    T acc = T(0);
    for (int p = 0; p < a.world; ++p)
      acc += load_cv(reinterpret_cast<const T*>(own + part_off(slot, p, a.world, a.cap)) + i);
    dst[i] = acc;
  }
}

template <class T, int MODE>
int launch_p2p(const char* name, P2PArgs a, cudaStream_t s) {
  KB_REQUIRE(a.bufs && a.world >= 1 && a.world <= kMaxRanks && a.rank >= 0 && a.rank < a.world,
             KB_ERR_INVALID_ARG, "%s: bad communicator (rank %d of %d)", name, a.rank, a.world);
  KB_REQUIRE(a.n >= 0 && (a.n == 0 || (a.src && a.dst)), KB_ERR_INVALID_ARG, "%s: bad buffers", name);
  KB_REQUIRE((size_t)a.n * sizeof(T) <= a.cap, KB_ERR_WORKSPACE,
             "%s: %lld elements exceed the %zu-byte slot", name, (long long)a.n, a.cap);
  auto kern = p2p_allreduce_kernel<T, MODE>;
  static int per_sm = 0;
  if (per_sm == 0) {
    int b = 0;
    KB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kern, kP2PThreads, 0));
    per_sm = b > 0 ? b : 1;
  }
  // one element per thread (the split-K form reads `splits` partials for
  // each), capped at what is co-resident
  const int64_t want = std::max<int64_t>(1, ceil_div(a.n, (int64_t)kP2PThreads));
  const int grid = (int)std::min<int64_t>(want, (int64_t)sm_count() * per_sm);
  if (grid == 1) {  // one CTA: no grid barrier, an ordinary launch
    kern<<<1, kP2PThreads, 0, s>>>(a);
    return check_launch(name);
  }
  void* args[] = {&a};
  KB_CUDA(cudaLaunchCooperativeKernel((const void*)kern, dim3(grid), dim3(kP2PThreads), args, 0, s));
  return KB_OK;
}

// bytes per rank part of a slot of a buffer of buf_bytes
size_t part_cap(size_t buf_bytes, int world) {
  return buf_bytes > kHeaderBytes && world > 0 ? ((buf_bytes - kHeaderBytes) / 2 / world) & ~(size_t)255 : 0;
}

}  // namespace

// For the fused sharded kernels (peer_exchange.cuh): they share this file's
// fault word, read through its device address, and its slot layout.
int p2p_fault_address(int** out) {
  void* p = nullptr;
  KB_CUDA(cudaGetSymbolAddress(&p, g_p2p_fault));
  *out = static_cast<int*>(p);
  return KB_OK;
}

size_t p2p_part_cap(size_t buf_bytes, int world) { return part_cap(buf_bytes, world); }

static_assert(kHeaderBytes == kPeerHeaderBytes && kMaxRanks == kPeerMaxRanks && sizeof(Header) == sizeof(PeerHeader),
              "peer_exchange.cuh and p2p.cu must agree on the buffer layout");

}  // namespace kb

extern "C" {

size_t kb_p2p_header_bytes(void) { return kb::kHeaderBytes; }

size_t kb_p2p_buffer_bytes(size_t payload_bytes, int world) {
  return kb::kHeaderBytes + 2 * (size_t)(world > 0 ? world : 1) * ((payload_bytes + 255) & ~(size_t)255);
}

int kb_p2p_buffer_alloc(size_t bytes, void** ptr) {
  KB_REQUIRE(ptr && bytes > kb::kHeaderBytes, KB_ERR_INVALID_ARG, "kb_p2p_buffer_alloc: bad arguments");
  void* p = nullptr;
  KB_CUDA(cudaMalloc(&p, bytes));
  const cudaError_t e = cudaMemset(p, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(p);
    return kb::set_error(KB_ERR_CUDA, "kb_p2p_buffer_alloc: %s", cudaGetErrorString(e));
  }
  KB_CUDA(cudaDeviceSynchronize());
  *ptr = p;
  return KB_OK;
}

int kb_p2p_buffer_free(void* ptr) {
  if (ptr) KB_CUDA(cudaFree(ptr));
  return KB_OK;
}

int kb_p2p_ipc_handle(void* ptr, void* handle) {
  KB_REQUIRE(ptr && handle, KB_ERR_INVALID_ARG, "kb_p2p_ipc_handle: null pointer");
  cudaIpcMemHandle_t h;
  KB_CUDA(cudaIpcGetMemHandle(&h, ptr));
  memcpy(handle, &h, sizeof(h));
  return KB_OK;
}

int kb_p2p_ipc_open(const void* handle, void** peer_ptr) {
  KB_REQUIRE(handle && peer_ptr, KB_ERR_INVALID_ARG, "kb_p2p_ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  KB_CUDA(cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return KB_OK;
}

int kb_p2p_ipc_close(void* peer_ptr) {
  if (peer_ptr) KB_CUDA(cudaIpcCloseMemHandle(peer_ptr));
  return KB_OK;
}

int kb_p2p_read_fault(int clear, int* value) {
  KB_REQUIRE(value, KB_ERR_INVALID_ARG, "kb_p2p_read_fault: null pointer");
  KB_CUDA(cudaMemcpyFromSymbol(value, kb::g_p2p_fault, sizeof(int)));
  if (clear) {
    const int zero = 0;
    KB_CUDA(cudaMemcpyToSymbol(kb::g_p2p_fault, &zero, sizeof(int)));
  }
  return KB_OK;
}

int kb_p2p_allreduce_f64(void* const* bufs, int rank, int world, size_t buf_bytes, const double* src,
                         double* dst, int64_t n, unsigned epoch, uint64_t timeout_ns, kbStream stream) {
  kb::P2PArgs a{reinterpret_cast<char* const*>(bufs), rank, world, kb::part_cap(buf_bytes, world), n, src, 0, dst,
                epoch, timeout_ns};
  return kb::launch_p2p<double, 0>("kb_p2p_allreduce_f64", a, stream);
}

int kb_p2p_allreduce_f32(void* const* bufs, int rank, int world, size_t buf_bytes, const float* src,
                         float* dst, int64_t n, unsigned epoch, uint64_t timeout_ns, kbStream stream) {
  kb::P2PArgs a{reinterpret_cast<char* const*>(bufs), rank, world, kb::part_cap(buf_bytes, world), n, src, 0, dst,
                epoch, timeout_ns};
  return kb::launch_p2p<float, 0>("kb_p2p_allreduce_f32", a, stream);
}

int kb_p2p_splitk_allreduce_f32(void* const* bufs, int rank, int world, size_t buf_bytes, const float* partials,
                                int splits, float* dst, int64_t n, unsigned epoch, uint64_t timeout_ns,
                                kbStream stream) {
  KB_REQUIRE(splits >= 1, KB_ERR_INVALID_ARG, "kb_p2p_splitk_allreduce_f32: splits < 1");
  kb::P2PArgs a{reinterpret_cast<char* const*>(bufs), rank, world, kb::part_cap(buf_bytes, world), n, partials,
                splits, dst, epoch, timeout_ns};
  return kb::launch_p2p<float, 1>("kb_p2p_splitk_allreduce_f32", a, stream);
}

}  // extern "C"
