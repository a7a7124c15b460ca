// reduce.cu — global reductions to a scalar: MSE loss and Frobenius
// normalisation, single-GPU and sharded (partial -> collective -> finish).
//
// Stage 1 is a persistent grid (SMs x 4 CTAs) that streams the input with
// 128-bit loads and writes one fp64 partial per CTA into the caller's
// workspace; stage 2 adds the partials in a fixed order.  No atomics: the
// result is bit-reproducible run to run (the reference used one fp32 atomicAdd
// per block, candidates/94_MSELoss/v1.py:27 and candidates/37_FrobeniusNorm_/
// v1.py:33).  Per-thread sums run in fp32 over 16-element tiles and are then
// promoted to fp64.
//
// Frobenius needs the global norm before any output can be written and the
// input (1 GiB) does not fit on chip, so x is read twice: the sum pass, a
// one-CTA finish that writes the fp64 total, and the scale pass (one
// 4096-float tile per CTA, 256-bit accesses), which walks the tensor from the
// end backwards so that its first tiles are the ones the sum pass touched
// last, still resident in the 126 MB L2.
#include "kb_common.cuh"
#include "peer_exchange.cuh"

namespace kb {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;
constexpr int kMaxPartials = 2048;

int reduce_grid(int64_t nvec) {
  const int64_t want = ceil_div(std::max<int64_t>(nvec, 1), (int64_t)kThreads * kUnroll);
  return (int)std::max<int64_t>(1, std::min<int64_t>({want, (int64_t)sm_count() * 4, (int64_t)kMaxPartials}));
}

// This thread's share of sum over i of f(a[i], b[i]) (f = (a - b)^2 or a^2)
// over a grid-stride walk of 1024-float4 tiles.
template <bool DIFF>
__device__ __forceinline__ double sq_thread_sum(const float* __restrict__ a, const float* __restrict__ b,
                                                int64_t n, bool vec) {
  double dacc = 0.0;
  int64_t scalar_begin = 0;
  if (vec) {
    const int64_t nvec = n / 4;
    const float4* a4 = reinterpret_cast<const float4*>(a);
    const float4* b4 = reinterpret_cast<const float4*>(b);
    const int64_t tile = (int64_t)kThreads * kUnroll;
    const int64_t ntiles = nvec / tile;
    for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
      const int64_t base = t * tile + threadIdx.x;
      float4 va[kUnroll], vb[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        if constexpr (DIFF) {
          va[u] = ld_stream(a4 + base + u * kThreads);
          vb[u] = ld_stream(b4 + base + u * kThreads);
        } else {
          va[u] = __ldg(a4 + base + u * kThreads);  // keep in L2 for the scale pass
        }
      }
      float s = 0.0f;
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        float4 d = va[u];
        if constexpr (DIFF) {
          d.x -= vb[u].x; d.y -= vb[u].y; d.z -= vb[u].z; d.w -= vb[u].w;
        }
        s += (d.x * d.x + d.y * d.y) + (d.z * d.z + d.w * d.w);
      }
      dacc += (double)s;
    }
    for (int64_t i = ntiles * tile + (int64_t)blockIdx.x * kThreads + threadIdx.x; i < nvec;
         i += (int64_t)gridDim.x * kThreads) {
      float4 d = DIFF ? ld_stream(a4 + i) : __ldg(a4 + i);
      if constexpr (DIFF) {
        const float4 e = ld_stream(b4 + i);
        d.x -= e.x; d.y -= e.y; d.z -= e.z; d.w -= e.w;
      }
      dacc += (double)((d.x * d.x + d.y * d.y) + (d.z * d.z + d.w * d.w));
    }
    scalar_begin = nvec * 4;
  }
  for (int64_t i = scalar_begin + (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * kThreads) {
    float d = a[i];
    if constexpr (DIFF) d -= b[i];
    dacc += (double)(d * d);
  }
  return dacc;
}

// sum over i of f(a[i], b[i]) -> partials[blockIdx.x]
template <bool DIFF>
__global__ void __launch_bounds__(kThreads)
sq_partial_kernel(const float* __restrict__ a, const float* __restrict__ b, int64_t n,
                  bool vec, double* __restrict__ partials) {
  __shared__ double red[32];
  const double tot = block_sum<kThreads>(sq_thread_sum<DIFF>(a, b, n, vec), red);
  if (threadIdx.x == 0) partials[blockIdx.x] = tot;
}

// Sharded form, one launch: the partials of this rank's shard; the CTA that
// arrives last folds them in a fixed order and exchanges the fold with every
// rank over the peer buffers (peer_exchange.cuh).  MSE (DIFF): the exchange
// carries (sum, element count) and out_f[0] = global sum / global count;
// sum of squares: out_d[0] = the global sum.
template <bool DIFF>
__global__ void __launch_bounds__(kThreads)
sq_sharded_kernel(const float* __restrict__ a, const float* __restrict__ b, int64_t n, bool vec,
                  double* __restrict__ partials, unsigned* counter, PeerCtx peer, float* out_f,
                  double* out_d) {
  __shared__ double red[32];
  __shared__ double vals[2];
  const double tot = block_sum<kThreads>(sq_thread_sum<DIFF>(a, b, n, vec), red);
  if (threadIdx.x == 0) partials[blockIdx.x] = tot;
  if (!last_cta_arrives(counter)) return;
  double v = 0.0;
  for (int i = threadIdx.x; i < (int)gridDim.x; i += kThreads) v += __ldcg(partials + i);
  v = block_sum<kThreads>(v, red);
  if (threadIdx.x == 0) {
    vals[0] = v;
    vals[1] = (double)n;
  }
  __syncthreads();
  block_peer_allreduce(peer, vals, vals, DIFF ? 2 : 1);
  if (threadIdx.x == 0) {
    if (out_f) out_f[0] = (float)(vals[0] / vals[1]);
    if (out_d) out_d[0] = vals[0];
  }
}

// Fixed-order sum of `count` fp64 partials by one CTA (identical in every
// CTA that calls it).
__device__ __forceinline__ double sum_partials(const double* __restrict__ p, int count, double* red) {
  double v = 0.0;
  for (int i = threadIdx.x; i < count; i += kThreads) v += p[i];
  return block_sum<kThreads>(v, red);
}

// mode 0: out_f = sum / denom (fp32); mode 1: out_d[0] = sum (fp64), and
// out_d[1] = elems when elems >= 0
__global__ void __launch_bounds__(kThreads)
finish_kernel(const double* __restrict__ partials, int count, double denom, float* out_f,
              double* out_d, double elems = -1.0) {
  __shared__ double red[32];
  const double s = sum_partials(partials, count, red);
  if (threadIdx.x == 0) {
    if (out_f) out_f[0] = (float)(s / denom);
    if (out_d) {
      out_d[0] = s;
      if (elems >= 0.0) out_d[1] = elems;
    }
  }
}

// denom <= 0: the element count summed with the partials, total[1]
__global__ void mse_finalize_kernel(const double* __restrict__ total, float* out, double denom) {
  out[0] = (float)(total[0] / (denom > 0.0 ? denom : total[1]));
}

// y = x / sqrt(sumsq) with sumsq one fp64 total.  One 4096-float tile per
// CTA, all of a thread's loads issued before its stores, tiles taken from
// the end of the tensor backwards (CTAs start in blockIdx order, so the
// first tiles are the ones the sum pass read last, still in L2).
constexpr int kScaleTile = 4096;

__device__ __forceinline__ float inv_norm_source(const double* sumsq) { return (float)sqrt(*sumsq); }

template <int W>
__global__ void __launch_bounds__(kThreads)
scale_tile_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t tiles,
                  const double* __restrict__ sumsq) {
  constexpr int U = kScaleTile / (kThreads * W);
  const float norm = inv_norm_source(sumsq);
  const int64_t base = (tiles - 1 - (int64_t)blockIdx.x) * kScaleTile + threadIdx.x * W;
  f32x8 v[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    if (W == 8) {
      v[u] = ld_stream8(x + base + u * kThreads * W);
    } else {
      const float4 q = ld_stream(reinterpret_cast<const float4*>(x + base + u * kThreads * W));
      v[u].v[0] = q.x;
      v[u].v[1] = q.y;
      v[u].v[2] = q.z;
      v[u].v[3] = q.w;
    }
  }
#pragma unroll
  for (int u = 0; u < U; ++u) {
#pragma unroll
    for (int k = 0; k < W; ++k) v[u].v[k] = v[u].v[k] / norm;
    if (W == 8)
      st_stream8(y + base + u * kThreads * W, v[u]);
    else
      st_stream(reinterpret_cast<float4*>(y + base + u * kThreads * W),
                make_float4(v[u].v[0], v[u].v[1], v[u].v[2], v[u].v[3]));
  }
}

__global__ void __launch_bounds__(kThreads)
scale_scalar_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t begin, int64_t n,
                    const double* __restrict__ sumsq) {
  const float norm = inv_norm_source(sumsq);
  for (int64_t i = begin + (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * kThreads)
    y[i] = x[i] / norm;
}

int launch_scale(const char* name, const float* x, float* y, int64_t n, const double* sumsq, cudaStream_t s) {
  const int64_t tiles = n / kScaleTile;
  KB_REQUIRE(tiles <= 0x7fffffff, KB_ERR_UNSUPPORTED, "%s: too large", name);
  int64_t done = 0;
  if (tiles > 0 && aligned32(x) && aligned32(y)) {
    scale_tile_kernel<8><<<(unsigned)tiles, kThreads, 0, s>>>(x, y, tiles, sumsq);
    done = tiles * kScaleTile;
  } else if (tiles > 0 && aligned16(x) && aligned16(y)) {
    scale_tile_kernel<4><<<(unsigned)tiles, kThreads, 0, s>>>(x, y, tiles, sumsq);
    done = tiles * kScaleTile;
  }
  if (done < n) {
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(n - done, kThreads), (int64_t)sm_count() * 8));
    scale_scalar_kernel<<<grid, kThreads, 0, s>>>(x, y, done, n, sumsq);
  }
  return check_launch(name);
}

int check_ws(const char* name, void* ws, size_t bytes, size_t need) {
  KB_REQUIRE(ws != nullptr && bytes >= need, KB_ERR_WORKSPACE,
             "%s: workspace of %zu bytes needed, %zu given", name, need, bytes);
  KB_REQUIRE((reinterpret_cast<uintptr_t>(ws) & 7) == 0, KB_ERR_INVALID_ARG,
             "%s: workspace must be 8-byte aligned", name);
  return KB_OK;
}

// stage 1 for both ops; returns the number of partials written
int launch_partials(const char* name, const float* a, const float* b, int64_t n, double* parts,
                    cudaStream_t s, int* count) {
  const bool vec = aligned16(a) && (!b || aligned16(b));
  const int grid = reduce_grid(vec ? n / 4 : n);
  if (b) sq_partial_kernel<true><<<grid, kThreads, 0, s>>>(a, b, n, vec, parts);
  else sq_partial_kernel<false><<<grid, kThreads, 0, s>>>(a, nullptr, n, vec, parts);
  *count = grid;
  return check_launch(name);
}

// the peer view of one call of a fused sharded entry; checks the payload fits a slot
int make_peer(const char* name, void* const* bufs, int rank, int world, size_t buf_bytes, unsigned epoch,
              uint64_t timeout_ns, size_t payload_bytes, PeerCtx* out) {
  KB_REQUIRE(bufs && world >= 1 && world <= kPeerMaxRanks && rank >= 0 && rank < world, KB_ERR_INVALID_ARG,
             "%s: bad communicator (rank %d of %d)", name, rank, world);
  KB_REQUIRE(epoch != 0, KB_ERR_INVALID_ARG, "%s: epoch 0 is reserved", name);
  const size_t cap = p2p_part_cap(buf_bytes, world);
  KB_REQUIRE(payload_bytes <= cap, KB_ERR_WORKSPACE, "%s: %zu-byte exchange exceeds the %zu-byte slot", name,
             payload_bytes, cap);
  int* fault = nullptr;
  if (int st = p2p_fault_address(&fault)) return st;
  *out = PeerCtx{reinterpret_cast<char* const*>(bufs), rank, world, cap, epoch, timeout_ns, fault};
  return KB_OK;
}

// a sharded entry's workspace: the arrival counter (first 256 bytes), then
// the per-CTA partials
constexpr size_t kShardedWorkspace = kShardedCounterBytes + kMaxPartials * sizeof(double);

// diff: MSE of (a, b); otherwise the sum of squares of a.  Explicit, because
// an empty shard may come with null data pointers.
int launch_sharded(const char* name, bool diff, const float* a, const float* b, int64_t n, void* ws,
                   size_t ws_bytes, const PeerCtx& peer, float* out_f, double* out_d, cudaStream_t s) {
  if (int st = check_ws(name, ws, ws_bytes, kShardedWorkspace)) return st;
  unsigned* counter = static_cast<unsigned*>(ws);
  double* parts = reinterpret_cast<double*>(static_cast<char*>(ws) + kShardedCounterBytes);
  const bool vec = n > 0 && aligned16(a) && (!b || aligned16(b));
  const int grid = n > 0 ? reduce_grid(vec ? n / 4 : n) : 1;
  if (diff) sq_sharded_kernel<true><<<grid, kThreads, 0, s>>>(a, b, n, vec, parts, counter, peer, out_f, out_d);
  else sq_sharded_kernel<false><<<grid, kThreads, 0, s>>>(a, nullptr, n, vec, parts, counter, peer, out_f, out_d);
  return check_launch(name);
}

}  // namespace
}  // namespace kb

extern "C" {

size_t kb_sharded_workspace_size(void) { return kb::kShardedWorkspace; }

int kb_mse_sharded_f32(const float* a, const float* b, float* out, int64_t n, void* workspace,
                       size_t workspace_bytes, void* const* bufs, int rank, int world, size_t buf_bytes,
                       unsigned epoch, uint64_t timeout_ns, kbStream stream) {
  const char* name = "kb_mse_sharded_f32";
  KB_REQUIRE(n >= 0, KB_ERR_INVALID_ARG, "%s: negative n", name);
  KB_REQUIRE(out && (n == 0 || (a && b)), KB_ERR_INVALID_ARG, "%s: null pointer", name);
  kb::PeerCtx peer;
  if (int st = kb::make_peer(name, bufs, rank, world, buf_bytes, epoch, timeout_ns, 2 * sizeof(double), &peer))
    return st;
  return kb::launch_sharded(name, true, a, b, n, workspace, workspace_bytes, peer, out, nullptr, stream);
}

int kb_sumsq_sharded_f64(const float* x, double* total, int64_t n, void* workspace, size_t workspace_bytes,
                         void* const* bufs, int rank, int world, size_t buf_bytes, unsigned epoch,
                         uint64_t timeout_ns, kbStream stream) {
  const char* name = "kb_sumsq_sharded_f64";
  KB_REQUIRE(n >= 0, KB_ERR_INVALID_ARG, "%s: negative n", name);
  KB_REQUIRE(total && (n == 0 || x), KB_ERR_INVALID_ARG, "%s: null pointer", name);
  kb::PeerCtx peer;
  if (int st = kb::make_peer(name, bufs, rank, world, buf_bytes, epoch, timeout_ns, sizeof(double), &peer))
    return st;
  return kb::launch_sharded(name, false, x, nullptr, n, workspace, workspace_bytes, peer, nullptr, total, stream);
}

size_t kb_mse_workspace_size(int64_t) { return kb::kMaxPartials * sizeof(double); }

int kb_mse_f32(const float* a, const float* b, float* out, int64_t n, void* workspace,
               size_t workspace_bytes, kbStream stream) {
  const char* name = "kb_mse_f32";
  KB_REQUIRE(n >= 0, KB_ERR_INVALID_ARG, "%s: negative n", name);
  KB_REQUIRE(out && (n == 0 || (a && b)), KB_ERR_INVALID_ARG, "%s: null pointer", name);
  if (int st = kb::check_ws(name, workspace, workspace_bytes, kb_mse_workspace_size(n))) return st;
  double* parts = static_cast<double*>(workspace);
  int count = 0;
  if (n > 0) {
    if (int st = kb::launch_partials(name, a, b, n, parts, stream, &count)) return st;
  }
  // n == 0: mean of nothing is NaN (0 / 0), as torch.mean of an empty tensor
  kb::finish_kernel<<<1, kb::kThreads, 0, stream>>>(parts, count, (double)n, out, nullptr);
  return kb::check_launch(name);
}

int kb_mse_partial_f64(const float* a, const float* b, double* partial, int64_t n,
                       void* workspace, size_t workspace_bytes, kbStream stream) {
  const char* name = "kb_mse_partial_f64";
  KB_REQUIRE(n >= 0, KB_ERR_INVALID_ARG, "%s: negative n", name);
  KB_REQUIRE(partial && (n == 0 || (a && b)), KB_ERR_INVALID_ARG, "%s: null pointer", name);
  if (int st = kb::check_ws(name, workspace, workspace_bytes, kb_mse_workspace_size(n))) return st;
  double* parts = static_cast<double*>(workspace);
  int count = 0;
  if (n > 0) {
    if (int st = kb::launch_partials(name, a, b, n, parts, stream, &count)) return st;
  }
  kb::finish_kernel<<<1, kb::kThreads, 0, stream>>>(parts, count, 1.0, nullptr, partial, (double)n);
  return kb::check_launch(name);
}

int kb_mse_finalize_f32(const double* total, float* out, int64_t total_n, kbStream stream) {
  // total_n 0: divide by total[1], the shards' element counts summed with the partials
  KB_REQUIRE(total && out && total_n >= 0, KB_ERR_INVALID_ARG, "kb_mse_finalize_f32: bad argument");
  kb::mse_finalize_kernel<<<1, 1, 0, stream>>>(total, out, (double)total_n);
  return kb::check_launch("kb_mse_finalize_f32");
}

// the partials, then the fp64 total
size_t kb_frobenius_workspace_size(int64_t) { return (kb::kMaxPartials + 2) * sizeof(double); }

int kb_frobenius_normalize_f32(const float* x, float* y, int64_t n, void* workspace,
                               size_t workspace_bytes, kbStream stream) {
  const char* name = "kb_frobenius_normalize_f32";
  KB_REQUIRE(n >= 0, KB_ERR_INVALID_ARG, "%s: negative n", name);
  if (n == 0) return KB_OK;
  KB_REQUIRE(x && y, KB_ERR_INVALID_ARG, "%s: null pointer", name);
  if (int st = kb::check_ws(name, workspace, workspace_bytes, kb_frobenius_workspace_size(n))) return st;
  double* parts = static_cast<double*>(workspace);
  double* total = parts + kb::kMaxPartials;
  int count = 0;
  if (int st = kb::launch_partials(name, x, nullptr, n, parts, stream, &count)) return st;
  kb::finish_kernel<<<1, kb::kThreads, 0, stream>>>(parts, count, 1.0, nullptr, total);
  if (int st = kb::check_launch(name)) return st;
  return kb::launch_scale(name, x, y, n, total, stream);
}

int kb_sumsq_partial_f64(const float* x, double* sumsq, int64_t n, void* workspace,
                         size_t workspace_bytes, kbStream stream) {
  const char* name = "kb_sumsq_partial_f64";
  KB_REQUIRE(n >= 0, KB_ERR_INVALID_ARG, "%s: negative n", name);
  KB_REQUIRE(sumsq && (n == 0 || x), KB_ERR_INVALID_ARG, "%s: null pointer", name);
  if (int st = kb::check_ws(name, workspace, workspace_bytes, kb_frobenius_workspace_size(n))) return st;
  double* parts = static_cast<double*>(workspace);
  int count = 0;
  if (n > 0) {
    if (int st = kb::launch_partials(name, x, nullptr, n, parts, stream, &count)) return st;
  }
  kb::finish_kernel<<<1, kb::kThreads, 0, stream>>>(parts, count, 1.0, nullptr, sumsq);
  return kb::check_launch(name);
}

int kb_scale_by_inv_norm_f32(const float* x, float* y, int64_t n, const double* total_sumsq,
                             kbStream stream) {
  const char* name = "kb_scale_by_inv_norm_f32";
  KB_REQUIRE(n >= 0, KB_ERR_INVALID_ARG, "%s: negative n", name);
  if (n == 0) return KB_OK;
  KB_REQUIRE(x && y && total_sumsq, KB_ERR_INVALID_ARG, "%s: null pointer", name);
  return kb::launch_scale(name, x, y, n, total_sumsq, stream);
}

}  // extern "C"
