// colreduce.cu — sum / mean / argmax over dim 1 of a contiguous x[B, I, J].
//
// The reduced dimension is strided (rows of length J), so the kernel keeps
// the coalesced direction across j: a CTA owns a strip of 32 * VW columns of
// one batch item and 8 warps split the I rows into 8 contiguous chunks.  Each
// warp reads full 512-byte row segments (VW = 4: one float4 per lane) with 8
// loads in flight per thread, then the 8 per-warp partials are combined in
// chunk order through shared memory, so the result is deterministic and
// argmax keeps the lowest index on ties (candidates/51_Argmax_over_a_
// dimension/v1.py:22).  Every element of x is read from HBM exactly once.
#include "kb_common.cuh"

namespace kb {
namespace {

enum ColOp { kSum = 0, kMean = 1, kArgmax = 2 };

constexpr int kWarps = 8;
constexpr int kUnrollI = 8;

template <int VW> struct Vec;
template <> struct Vec<4> { using T = float4; };
template <> struct Vec<1> { using T = float; };

__device__ __forceinline__ float comp(const float4& v, int c) {
  return c == 0 ? v.x : c == 1 ? v.y : c == 2 ? v.z : v.w;
}
__device__ __forceinline__ float comp(const float& v, int) { return v; }

// torch.argmax order: NaN is larger than everything; among equal values the
// earlier index wins (strict comparison, callers visit indices in order).
__device__ __forceinline__ bool argmax_better(float v, float best) {
  return v > best || (v != v && best == best);
}

template <ColOp OP, int VW>
__global__ void __launch_bounds__(32 * kWarps)
colreduce_kernel(const float* __restrict__ x, void* __restrict__ out, int64_t I, int64_t J) {
  using V = typename Vec<VW>::T;
  __shared__ float s_val[kWarps][32 * VW];
  __shared__ int64_t s_idx[OP == kArgmax ? kWarps : 1][OP == kArgmax ? 32 * VW : 1];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t b = blockIdx.y;
  const int64_t j0 = (int64_t)blockIdx.x * (32 * VW) + (int64_t)lane * VW;  // first column
  const bool active = j0 < J;  // J % VW == 0 for VW == 4, so a vector is all-in or all-out
  const int64_t chunk = ceil_div(I, kWarps);
  const int64_t i_begin = std::min<int64_t>((int64_t)warp * chunk, I);
  const int64_t i_end = std::min<int64_t>(i_begin + chunk, I);
  const float* xb = x + b * I * J + j0;

  float acc[VW];
  int64_t idx[VW];
#pragma unroll
  for (int c = 0; c < VW; ++c) {
    acc[c] = (OP == kArgmax) ? -INFINITY : 0.0f;
    idx[c] = i_begin;
  }

  if (active) {
    int64_t i = i_begin;
    for (; i + kUnrollI <= i_end; i += kUnrollI) {
      V v[kUnrollI];
#pragma unroll
      for (int u = 0; u < kUnrollI; ++u)
        v[u] = ld_stream(reinterpret_cast<const V*>(xb + (i + u) * J));
#pragma unroll
      for (int u = 0; u < kUnrollI; ++u)
#pragma unroll
        for (int c = 0; c < VW; ++c) {
          const float e = comp(v[u], c);
          if constexpr (OP == kArgmax) {
            if (argmax_better(e, acc[c])) { acc[c] = e; idx[c] = i + u; }
          } else {
            acc[c] += e;
          }
        }
    }
    for (; i < i_end; ++i) {
      const V v = ld_stream(reinterpret_cast<const V*>(xb + i * J));
#pragma unroll
      for (int c = 0; c < VW; ++c) {
        const float e = comp(v, c);
        if constexpr (OP == kArgmax) {
          if (argmax_better(e, acc[c])) { acc[c] = e; idx[c] = i; }
        } else {
          acc[c] += e;
        }
      }
    }
  }

#pragma unroll
  for (int c = 0; c < VW; ++c) {
    s_val[warp][lane * VW + c] = acc[c];
    if constexpr (OP == kArgmax) s_idx[warp][lane * VW + c] = idx[c];
  }
  __syncthreads();
  // combine the 8 chunk partials in chunk order (warp 0 handles the strip)
  if (warp == 0 && active) {
#pragma unroll
    for (int c = 0; c < VW; ++c) {
      const int col = lane * VW + c;
      if constexpr (OP == kArgmax) {
        float best = s_val[0][col];
        int64_t bi = s_idx[0][col];
        for (int w = 1; w < kWarps; ++w)
          if (argmax_better(s_val[w][col], best)) { best = s_val[w][col]; bi = s_idx[w][col]; }
        static_cast<int64_t*>(out)[b * J + j0 + c] = bi;
      } else {
        float s = 0.0f;
        for (int w = 0; w < kWarps; ++w) s += s_val[w][col];
        if constexpr (OP == kMean) s = s / (float)I;
        static_cast<float*>(out)[b * J + j0 + c] = s;
      }
    }
  }
}

template <ColOp OP>
int launch_colreduce(const char* name, const float* x, void* out, int64_t B, int64_t I,
                     int64_t J, cudaStream_t s) {
  KB_REQUIRE(B >= 0 && I >= 0 && J >= 0, KB_ERR_INVALID_ARG, "%s: negative size", name);
  if (B == 0 || J == 0) return KB_OK;
  KB_REQUIRE(OP != kArgmax || I > 0, KB_ERR_INVALID_ARG, "%s: argmax over an empty dimension", name);
  KB_REQUIRE(out && (x || I == 0), KB_ERR_INVALID_ARG, "%s: null pointer", name);
  KB_REQUIRE(B <= 65535, KB_ERR_UNSUPPORTED, "%s: B > 65535", name);
  const bool vec = (J % 4 == 0) && aligned16(x) && (OP == kArgmax ? ((reinterpret_cast<uintptr_t>(out) & 7) == 0) : aligned16(out));
  if (vec) {
    dim3 grid((unsigned)ceil_div(J, 128), (unsigned)B);
    colreduce_kernel<OP, 4><<<grid, 32 * kWarps, 0, s>>>(x, out, I, J);
  } else {
    dim3 grid((unsigned)ceil_div(J, 32), (unsigned)B);
    colreduce_kernel<OP, 1><<<grid, 32 * kWarps, 0, s>>>(x, out, I, J);
  }
  return check_launch(name);
}

}  // namespace
}  // namespace kb

extern "C" {

int kb_sum_dim1_f32(const float* x, float* out, int64_t B, int64_t I, int64_t J, kbStream stream) {
  return kb::launch_colreduce<kb::kSum>("kb_sum_dim1_f32", x, out, B, I, J, stream);
}
int kb_mean_dim1_f32(const float* x, float* out, int64_t B, int64_t I, int64_t J, kbStream stream) {
  return kb::launch_colreduce<kb::kMean>("kb_mean_dim1_f32", x, out, B, I, J, stream);
}
int kb_argmax_dim1_f32(const float* x, int64_t* out, int64_t B, int64_t I, int64_t J,
                       kbStream stream) {
  return kb::launch_colreduce<kb::kArgmax>("kb_argmax_dim1_f32", x, out, B, I, J, stream);
}

}  // extern "C"
