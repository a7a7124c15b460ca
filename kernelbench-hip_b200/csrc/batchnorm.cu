// batchnorm.cu — training-mode BatchNorm2d over NCHW fp32 (batch statistics,
// biased variance for normalisation, optional running-statistics update).
//
// Pass 1 (stats): grid (C, S).  CTA (c, s) streams the (n, c) planes of its
// batch slice — each plane is HW contiguous floats — and writes one fp64
// (sum, sum of squares) pair to the workspace.  No atomics (the reference's
// per-256-element atomics ran at 41 GB/s, candidates/33_BatchNorm/v1.py:36-40).
// Pass 2 (apply): one CTA per (n, c) plane folds the S partials of its channel
// in a fixed order (or reads fp64 totals produced by a cross-GPU collective),
// derives mean / inv-std in fp64 and writes y = (x - mean) * (inv_std * gamma)
// + beta.  x is read twice (2 GiB does not fit on chip); planes are applied in
// reverse order so the first ones still sit in L2 from the end of pass 1.

#include "kb_common.cuh"
#include "peer_exchange.cuh"

namespace kb {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

struct BnShape {
  int64_t N, C, HW;
};

int bn_splits(int64_t N, int64_t C) {
  const int64_t want = ceil_div((int64_t)sm_count() * 4, std::max<int64_t>(C, 1));
  return (int)std::max<int64_t>(1, std::min<int64_t>(N, want));
}

// per-thread fp32 sums over one plane, promoted to fp64 per 16-element tile
__device__ __forceinline__ void plane_sums(const float* __restrict__ p, int64_t HW, bool vec,
                                           double& s1, double& s2) {
  int64_t scalar_begin = 0;
  if (vec) {
    const float4* p4 = reinterpret_cast<const float4*>(p);
    const int64_t nvec = HW / 4;
    const int64_t tile = (int64_t)kThreads * kUnroll;
    int64_t i = threadIdx.x;
    for (; i + (kUnroll - 1) * kThreads < nvec; i += tile) {
      float4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) v[u] = __ldg(p4 + i + u * kThreads);
      float a = 0.f, q = 0.f;
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        a += (v[u].x + v[u].y) + (v[u].z + v[u].w);
        q += (v[u].x * v[u].x + v[u].y * v[u].y) + (v[u].z * v[u].z + v[u].w * v[u].w);
      }
      s1 += (double)a;
      s2 += (double)q;
    }
    for (; i < nvec; i += kThreads) {
      const float4 v = __ldg(p4 + i);
      s1 += (double)((v.x + v.y) + (v.z + v.w));
      s2 += (double)((v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w));
    }
    scalar_begin = nvec * 4;
  }
  for (int64_t i = scalar_begin + threadIdx.x; i < HW; i += kThreads) {
    const float v = p[i];
    s1 += (double)v;
    s2 += (double)(v * v);
  }
}

__global__ void __launch_bounds__(kThreads)
bn_stats_kernel(const float* __restrict__ x, BnShape sh, int S, bool vec,
                double2* __restrict__ partials) {
  __shared__ double red[32];
  const int64_t c = blockIdx.x;
  const int s = blockIdx.y;
  const int64_t n0 = sh.N * s / S, n1 = sh.N * (s + 1) / S;
  double s1 = 0.0, s2 = 0.0;
  for (int64_t n = n0; n < n1; ++n) plane_sums(x + (n * sh.C + c) * sh.HW, sh.HW, vec, s1, s2);
  s1 = block_sum<kThreads>(s1, red);
  s2 = block_sum<kThreads>(s2, red);
  if (threadIdx.x == 0) partials[c * S + s] = make_double2(s1, s2);
}

// Sharded form of the statistics pass: the grid and partials of
// bn_stats_kernel; the CTA that arrives last folds every channel's S
// partials in split order into stats = [sum (C) | sum of squares (C) |
// elements per channel], then exchanges those 2C + 1 values with every rank
// over the peer buffers (peer_exchange.cuh): stats ends as the global totals.
__global__ void __launch_bounds__(kThreads)
bn_stats_sharded_kernel(const float* __restrict__ x, BnShape sh, int S, bool vec, double2* __restrict__ partials,
                        unsigned* counter, PeerCtx peer, double* __restrict__ stats) {
  __shared__ double red[32];
  const int64_t c = blockIdx.x;
  const int s = blockIdx.y;
  const int64_t n0 = sh.N * s / S, n1 = sh.N * (s + 1) / S;
  double s1 = 0.0, s2 = 0.0;
  for (int64_t n = n0; n < n1; ++n) plane_sums(x + (n * sh.C + c) * sh.HW, sh.HW, vec, s1, s2);
  s1 = block_sum<kThreads>(s1, red);
  s2 = block_sum<kThreads>(s2, red);
  if (threadIdx.x == 0) partials[c * S + s] = make_double2(s1, s2);
  if (!last_cta_arrives(counter)) return;
  for (int64_t ch = threadIdx.x; ch < sh.C; ch += kThreads) {
    double t1 = 0.0, t2 = 0.0;
    for (int z = 0; z < S; ++z) {
      const double2 p = __ldcg(partials + ch * S + z);
      t1 += p.x;
      t2 += p.y;
    }
    stats[ch] = t1;
    stats[sh.C + ch] = t2;
  }
  if (threadIdx.x == 0) stats[2 * sh.C] = (double)(sh.N * sh.HW);
  __syncthreads();
  block_peer_allreduce(peer, stats, stats, (int)(2 * sh.C + 1));
}

// totals: stats[c] = sum, stats[C + c] = sum of squares (fp64)
// stats = [sum (C) | sum of squares (C) | elements per channel]
__global__ void bn_fold_kernel(const double2* __restrict__ partials, int64_t C, int S,
                               double* __restrict__ stats, double elems) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c == 0) stats[2 * C] = elems;
  if (c >= C) return;
  double s1 = 0.0, s2 = 0.0;
  for (int s = 0; s < S; ++s) {
    const double2 p = partials[c * S + s];
    s1 += p.x;
    s2 += p.y;
  }
  stats[c] = s1;
  stats[C + c] = s2;
}

// running = (1 - momentum) * running + momentum * batch value (unbiased variance)
__device__ __forceinline__ void bn_update_running(int64_t c, float mean, double var_d, double count,
                                                  float momentum, float* running_mean, float* running_var) {
  const double unbiased = count > 1.0 ? var_d * count / (count - 1.0) : var_d;
  running_mean[c] = (1.0f - momentum) * running_mean[c] + momentum * mean;
  running_var[c] = (1.0f - momentum) * running_var[c] + momentum * (float)unbiased;
}

// Running statistics only (a rank whose batch shard is empty still applies
// the global batch's statistics to its copy).  count 0: stats[2C].
__global__ void bn_running_kernel(const double* __restrict__ stats, int64_t C, int64_t count,
                                  float momentum, float* running_mean, float* running_var) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const double cnt = count > 0 ? (double)count : stats[2 * C];
  const double mean_d = stats[c] / cnt;
  const double var_d = fmax(stats[C + c] / cnt - mean_d * mean_d, 0.0);
  bn_update_running(c, (float)mean_d, var_d, cnt, momentum, running_mean, running_var);
}

// One CTA per (n, c) plane, planes visited in reverse order.  Channel totals
// come from `partials` (S > 0, fixed-order fold) or from `stats` (S == 0;
// count 0: the element count stats[2C]).
__global__ void __launch_bounds__(kThreads)
bn_apply_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                const float* __restrict__ beta, float* __restrict__ y, BnShape sh,
                const double2* __restrict__ partials, int S, const double* __restrict__ stats,
                int64_t count, float eps, float momentum, float* running_mean,
                float* running_var, bool vec) {
  const int64_t plane = sh.N * sh.C - 1 - (int64_t)blockIdx.x;
  const int64_t n = plane / sh.C, c = plane - n * sh.C;
  double s1 = 0.0, s2 = 0.0;
  if (S > 0) {
    for (int s = 0; s < S; ++s) {
      const double2 p = partials[c * S + s];
      s1 += p.x;
      s2 += p.y;
    }
  } else {
    s1 = stats[c];
    s2 = stats[sh.C + c];
  }
  const double cnt = count > 0 ? (double)count : stats[2 * sh.C];
  const double mean_d = s1 / cnt;
  const double var_d = fmax(s2 / cnt - mean_d * mean_d, 0.0);
  const float mean = (float)mean_d;
  const float inv_std = (float)(1.0 / sqrt(var_d + (double)eps));
  const float scale = inv_std * (gamma ? gamma[c] : 1.0f);
  const float shift = beta ? beta[c] : 0.0f;
  if (n == 0 && threadIdx.x == 0 && running_mean && running_var)
    bn_update_running(c, mean, var_d, cnt, momentum, running_mean, running_var);
  const float* xp = x + plane * sh.HW;
  float* yp = y + plane * sh.HW;
  int64_t scalar_begin = 0;
  if (vec) {
    const float4* x4 = reinterpret_cast<const float4*>(xp);
    float4* y4 = reinterpret_cast<float4*>(yp);
    const int64_t nvec = sh.HW / 4;
    const int64_t tile = (int64_t)kThreads * kUnroll;
    int64_t i = threadIdx.x;
    for (; i + (kUnroll - 1) * kThreads < nvec; i += tile) {
      float4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) v[u] = ld_stream(x4 + i + u * kThreads);
#pragma unroll
      for (int u = 0; u < kUnroll; ++u)
        st_stream(y4 + i + u * kThreads,
                  make_float4((v[u].x - mean) * scale + shift, (v[u].y - mean) * scale + shift,
                              (v[u].z - mean) * scale + shift, (v[u].w - mean) * scale + shift));
    }
    for (; i < nvec; i += kThreads) {
      const float4 v = ld_stream(x4 + i);
      st_stream(y4 + i, make_float4((v.x - mean) * scale + shift, (v.y - mean) * scale + shift,
                                    (v.z - mean) * scale + shift, (v.w - mean) * scale + shift));
    }
    scalar_begin = nvec * 4;
  }
  for (int64_t i = scalar_begin + threadIdx.x; i < sh.HW; i += kThreads)
    yp[i] = (xp[i] - mean) * scale + shift;
}

// ---------------------------------------------------------------------------
// Allocation-free variant: the per-channel partials live in this file-scope
// device array instead of caller workspace.  Every device that loads the
// library holds it until exit.  Host code must not pass the symbol itself to a
// kernel (on the host it is only a stand-in, not a device address): each call
// looks the device address up on the current device with cudaGetSymbolAddress
// (cheap next to the two launches), so the address stays right when the
// module is loaded again after a cudaDeviceReset.  The first call on a device
// loads the module there and should come before any stream capture.
// ---------------------------------------------------------------------------
constexpr int kNoAllocPartials = 8192;  // (sum, sum of squares) pairs: 128 KiB
static __device__ __align__(256) double2 g_bn_noalloc_partials[kNoAllocPartials];

// Device address of g_bn_noalloc_partials on the current device.
int noalloc_partials(double2** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_bn_noalloc_partials);
  if (e != cudaSuccess || p == nullptr)
    return set_error(KB_ERR_CUDA, "cudaGetSymbolAddress(batchnorm scratch): %s", cudaGetErrorString(e));
  *out = static_cast<double2*>(p);
  return KB_OK;
}

int bn_check(const char* name, const float* x, int64_t N, int64_t C, int64_t HW) {
  KB_REQUIRE(N >= 0 && C >= 0 && HW >= 0, KB_ERR_INVALID_ARG, "%s: negative size", name);
  KB_REQUIRE(x || N * C * HW == 0, KB_ERR_INVALID_ARG, "%s: null input", name);
  KB_REQUIRE(C <= 0x7fffffff && N * C <= 0x7fffffff, KB_ERR_UNSUPPORTED, "%s: too many planes", name);
  return KB_OK;
}

}  // namespace
}  // namespace kb

extern "C" {

size_t kb_batchnorm_workspace_size(int64_t N, int64_t C, int64_t) {
  // worst case S = min(N, SMs * 4 / C) with SMs <= 160
  const int64_t S = std::max<int64_t>(1, std::min<int64_t>(N, kb::ceil_div(160 * 4, std::max<int64_t>(C, 1))));
  return (size_t)(C * S) * sizeof(double2) + 256;
}

int kb_batchnorm_train_f32(const float* x, const float* gamma, const float* beta, float* y,
                           int64_t N, int64_t C, int64_t HW, float eps, float momentum,
                           float* running_mean, float* running_var, void* workspace,
                           size_t workspace_bytes, kbStream stream) {
  const char* name = "kb_batchnorm_train_f32";
  if (int st = kb::bn_check(name, x, N, C, HW)) return st;
  if (N * C * HW == 0) return KB_OK;
  KB_REQUIRE(y, KB_ERR_INVALID_ARG, "%s: null output", name);
  KB_REQUIRE(workspace && workspace_bytes >= kb_batchnorm_workspace_size(N, C, HW),
             KB_ERR_WORKSPACE, "%s: workspace of %zu bytes needed", name,
             kb_batchnorm_workspace_size(N, C, HW));
  KB_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 15) == 0, KB_ERR_INVALID_ARG,
             "%s: workspace must be 16-byte aligned", name);
  const int S = kb::bn_splits(N, C);
  const bool vec = HW % 4 == 0 && kb::aligned16(x) && kb::aligned16(y);
  double2* parts = static_cast<double2*>(workspace);
  kb::BnShape sh{N, C, HW};
  kb::bn_stats_kernel<<<dim3((unsigned)C, (unsigned)S), kb::kThreads, 0, stream>>>(x, sh, S, vec, parts);
  if (int st = kb::check_launch(name)) return st;
  kb::bn_apply_kernel<<<(unsigned)(N * C), kb::kThreads, 0, stream>>>(
      x, gamma, beta, y, sh, parts, S, nullptr, N * HW, eps, momentum, running_mean, running_var, vec);
  return kb::check_launch(name);
}

int kb_batchnorm_train_f32_noalloc(const float* x, const float* gamma, const float* beta, float* y,
                                   int64_t N, int64_t C, int64_t HW, float eps, float momentum,
                                   float* running_mean, float* running_var, kbStream stream) {
  const char* name = "kb_batchnorm_train_f32_noalloc";
  if (int st = kb::bn_check(name, x, N, C, HW)) return st;
  if (N * C * HW == 0) return KB_OK;
  KB_REQUIRE(y, KB_ERR_INVALID_ARG, "%s: null output", name);
  const int S = kb::bn_splits(N, C);
  KB_REQUIRE(C * S <= kb::kNoAllocPartials, KB_ERR_UNSUPPORTED,
             "%s: %lld channels x %d batch splits need %lld partial slots; the built-in scratch "
             "holds %d (use kb_batchnorm_train_f32 with caller workspace)",
             name, (long long)C, S, (long long)(C * S), kb::kNoAllocPartials);
  double2* parts = nullptr;
  if (int st = kb::noalloc_partials(&parts)) return st;
  const bool vec = HW % 4 == 0 && kb::aligned16(x) && kb::aligned16(y);
  kb::BnShape sh{N, C, HW};
  // every used slot is overwritten by the stats kernel: nothing to clear
  kb::bn_stats_kernel<<<dim3((unsigned)C, (unsigned)S), kb::kThreads, 0, stream>>>(x, sh, S, vec, parts);
  if (int st = kb::check_launch(name)) return st;
  kb::bn_apply_kernel<<<(unsigned)(N * C), kb::kThreads, 0, stream>>>(
      x, gamma, beta, y, sh, parts, S, nullptr, N * HW, eps, momentum, running_mean, running_var, vec);
  return kb::check_launch(name);
}

int kb_batchnorm_stats_f64(const float* x, double* stats, int64_t N, int64_t C, int64_t HW,
                           void* workspace, size_t workspace_bytes, kbStream stream) {
  const char* name = "kb_batchnorm_stats_f64";
  if (int st = kb::bn_check(name, x, N, C, HW)) return st;
  KB_REQUIRE(stats || C == 0, KB_ERR_INVALID_ARG, "%s: null stats", name);
  if (C == 0) return KB_OK;
  KB_REQUIRE(workspace && workspace_bytes >= kb_batchnorm_workspace_size(N, C, HW),
             KB_ERR_WORKSPACE, "%s: workspace of %zu bytes needed", name,
             kb_batchnorm_workspace_size(N, C, HW));
  KB_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 15) == 0, KB_ERR_INVALID_ARG,
             "%s: workspace must be 16-byte aligned", name);
  const int S = kb::bn_splits(N, C);
  const bool vec = HW % 4 == 0 && kb::aligned16(x);
  double2* parts = static_cast<double2*>(workspace);
  kb::BnShape sh{N, C, HW};
  if (N > 0) {
    kb::bn_stats_kernel<<<dim3((unsigned)C, (unsigned)S), kb::kThreads, 0, stream>>>(x, sh, S, vec, parts);
    if (int st = kb::check_launch(name)) return st;
    kb::bn_fold_kernel<<<(unsigned)kb::ceil_div(C, 128), 128, 0, stream>>>(parts, C, S, stats,
                                                                            (double)(N * HW));
  } else {  // an empty shard: zero sums, zero elements
    KB_CUDA(cudaMemsetAsync(stats, 0, sizeof(double) * (2 * C + 1), stream));
  }
  return kb::check_launch(name);
}

size_t kb_batchnorm_sharded_workspace_size(int64_t N, int64_t C, int64_t HW) {
  return kb::kShardedCounterBytes + kb_batchnorm_workspace_size(N, C, HW);
}

int kb_batchnorm_stats_sharded_f64(const float* x, double* stats, int64_t N, int64_t C, int64_t HW,
                                   void* workspace, size_t workspace_bytes, void* const* bufs, int rank,
                                   int world, size_t buf_bytes, unsigned epoch, uint64_t timeout_ns,
                                   kbStream stream) {
  const char* name = "kb_batchnorm_stats_sharded_f64";
  if (int st = kb::bn_check(name, x, N, C, HW)) return st;
  KB_REQUIRE(C > 0 && stats, KB_ERR_INVALID_ARG, "%s: no channels or null stats", name);
  KB_REQUIRE(C <= 65535, KB_ERR_UNSUPPORTED, "%s: more than 65535 channels", name);
  KB_REQUIRE(workspace && workspace_bytes >= kb_batchnorm_sharded_workspace_size(N, C, HW), KB_ERR_WORKSPACE,
             "%s: workspace of %zu bytes needed", name, kb_batchnorm_sharded_workspace_size(N, C, HW));
  KB_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0, KB_ERR_INVALID_ARG,
             "%s: workspace must be 256-byte aligned", name);
  KB_REQUIRE(bufs && world >= 1 && world <= kb::kPeerMaxRanks && rank >= 0 && rank < world && epoch != 0,
             KB_ERR_INVALID_ARG, "%s: bad communicator (rank %d of %d, epoch %u)", name, rank, world, epoch);
  const size_t cap = kb::p2p_part_cap(buf_bytes, world);
  KB_REQUIRE((size_t)(2 * C + 1) * sizeof(double) <= cap, KB_ERR_WORKSPACE,
             "%s: %lld-value exchange exceeds the %zu-byte slot", name, (long long)(2 * C + 1), cap);
  int* fault = nullptr;
  if (int st = kb::p2p_fault_address(&fault)) return st;
  const kb::PeerCtx peer{reinterpret_cast<char* const*>(bufs), rank, world, cap, epoch, timeout_ns, fault};
  const int S = kb::bn_splits(N, C);
  const bool vec = HW % 4 == 0 && kb::aligned16(x);
  unsigned* counter = static_cast<unsigned*>(workspace);
  double2* parts = reinterpret_cast<double2*>(static_cast<char*>(workspace) + kb::kShardedCounterBytes);
  kb::BnShape sh{N, C, HW};
  kb::bn_stats_sharded_kernel<<<dim3((unsigned)C, (unsigned)S), kb::kThreads, 0, stream>>>(x, sh, S, vec, parts,
                                                                                          counter, peer, stats);
  return kb::check_launch(name);
}

int kb_batchnorm_apply_f32(const float* x, const float* gamma, const float* beta, float* y,
                           const double* stats, int64_t N, int64_t C, int64_t HW,
                           int64_t total_count, float eps, float momentum, float* running_mean,
                           float* running_var, kbStream stream) {
  const char* name = "kb_batchnorm_apply_f32";
  if (int st = kb::bn_check(name, x, N, C, HW)) return st;
  KB_REQUIRE(total_count >= 0 && (stats || C == 0), KB_ERR_INVALID_ARG, "%s: bad argument", name);
  if (N * C * HW == 0) {
    // nothing to normalise here; the running statistics still move with the global batch
    if (C > 0 && running_mean && running_var) {
      kb::bn_running_kernel<<<(unsigned)kb::ceil_div(C, 128), 128, 0, stream>>>(stats, C, total_count, momentum,
                                                                                running_mean, running_var);
      return kb::check_launch(name);
    }
    return KB_OK;
  }
  KB_REQUIRE(y, KB_ERR_INVALID_ARG, "%s: null output", name);
  const bool vec = HW % 4 == 0 && kb::aligned16(x) && kb::aligned16(y);
  kb::BnShape sh{N, C, HW};
  kb::bn_apply_kernel<<<(unsigned)(N * C), kb::kThreads, 0, stream>>>(
      x, gamma, beta, y, sh, nullptr, 0, stats, total_count, eps, momentum, running_mean,
      running_var, vec);
  return kb::check_launch(name);
}

}  // extern "C"
