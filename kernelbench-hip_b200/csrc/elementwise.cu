// elementwise.cu — streaming activation kernels (tanh-GELU, erf-GELU, Swish,
// ReLU).
//
// Each CTA owns one 4096-float tile: its 256 threads issue two 256-bit
// streaming loads each (128-bit when the views are only 16-byte aligned)
// before any math, so the whole tile is in flight at once.  A scalar kernel
// covers the n % 4096 tail and unaligned views.
#include "kb_common.cuh"

namespace kb {
namespace {

// Activation functors.  Each mirrors the arithmetic order of the torch
// expression it replaces so that fp32 rounding matches closely.
struct GeluTanh {
  // 0.5 * x * (1 + tanh(sqrt(2/pi) * (x + 0.044715 * x^3)))
  // (candidates/88_MinGPTNewGelu/v1.py:16-17)
  __device__ __forceinline__ float operator()(float x) const {
    const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
    const float k1 = 0.044715f;
    float inner = k0 * (x + k1 * (x * x * x));
    return (0.5f * x) * (1.0f + tanhf(inner));
  }
};
struct GeluErf {
  // x * 0.5 * (1 + erf(x / sqrt(2)))   (candidates/26_GELU_/v1.py:14)
  __device__ __forceinline__ float operator()(float x) const {
    return (x * 0.5f) * (1.0f + erff(x * 0.70710678118654752440f));
  }
};
struct Swish {
  // x * sigmoid(x)   (candidates/25_Swish/v1.py:14)
  __device__ __forceinline__ float operator()(float x) const {
    return x * (1.0f / (1.0f + expf(-x)));
  }
};
struct Relu {
  // max(x, 0) as torch.relu: NaN and -0.0 pass through unchanged
  // (candidates/19_ReLU/v1.py:12 used fmaxf, which maps NaN to 0)
  __device__ __forceinline__ float operator()(float x) const {
    return x < 0.0f ? 0.0f : x;
  }
};

constexpr int kThreads = 256;
constexpr int kTile = 4096;  // floats per CTA: 16 per thread

// W-float vector access (W = 8: one 256-bit instruction; W = 4: 128-bit).
template <int W>
struct Vec;
template <>
struct Vec<8> {
  static __device__ __forceinline__ f32x8 ld(const float* p) { return ld_stream8(p); }
  static __device__ __forceinline__ void st(float* p, const f32x8& v) { st_stream8(p, v); }
};
template <>
struct Vec<4> {
  static __device__ __forceinline__ f32x8 ld(const float* p) {
    const float4 a = ld_stream(reinterpret_cast<const float4*>(p));
    f32x8 r;
    r.v[0] = a.x;
    r.v[1] = a.y;
    r.v[2] = a.z;
    r.v[3] = a.w;
    return r;
  }
  static __device__ __forceinline__ void st(float* p, const f32x8& v) {
    st_stream(reinterpret_cast<float4*>(p), make_float4(v.v[0], v.v[1], v.v[2], v.v[3]));
  }
};

// One kTile-float tile per CTA, all of a thread's loads issued before any
// math.  A grid of n / kTile short-lived CTAs streams HBM faster on B200 than a
// persistent grid-stride loop over the same tiles (86-87 us against 94-100 us
// for 2 x 256 MiB at 4096 x 16384).  Held to 32 registers (8 CTAs per SM):
// erf-GELU otherwise took 40 and ran at 6 CTAs per SM, 4 % slower in the
// power-capped bench step; the other functions fit in 32 anyway.
template <class F, int W>
__global__ void __launch_bounds__(kThreads, 8)
elementwise_tile_kernel(const float* __restrict__ x, float* __restrict__ y, F f) {
  constexpr int U = kTile / (kThreads * W);
  const int64_t base = (int64_t)blockIdx.x * kTile + threadIdx.x * W;
  f32x8 v[U];
#pragma unroll
  for (int u = 0; u < U; ++u) v[u] = Vec<W>::ld(x + base + u * kThreads * W);
#pragma unroll
  for (int u = 0; u < U; ++u) {
#pragma unroll
    for (int k = 0; k < W; ++k) v[u].v[k] = f(v[u].v[k]);
    Vec<W>::st(y + base + u * kThreads * W, v[u]);
  }
}

template <class F>
__global__ void __launch_bounds__(kThreads)
elementwise_scalar_kernel(const float* __restrict__ x, float* __restrict__ y,
                          int64_t begin, int64_t n, F f) {
  for (int64_t i = begin + (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * kThreads)
    y[i] = f(x[i]);
}

template <class F>
int launch_elementwise(const char* name, const float* x, float* y, int64_t n, cudaStream_t s) {
  KB_REQUIRE(n >= 0, KB_ERR_INVALID_ARG, "%s: negative n", name);
  if (n == 0) return KB_OK;
  KB_REQUIRE(x && y, KB_ERR_INVALID_ARG, "%s: null pointer", name);
  const int64_t tiles = n / kTile;
  KB_REQUIRE(tiles <= 0x7fffffff, KB_ERR_UNSUPPORTED, "%s: n too large", name);
  int64_t done = 0;
  if (tiles > 0 && aligned32(x) && aligned32(y)) {
    elementwise_tile_kernel<F, 8><<<(unsigned)tiles, kThreads, 0, s>>>(x, y, F{});
    done = tiles * kTile;
  } else if (tiles > 0 && aligned16(x) && aligned16(y)) {
    elementwise_tile_kernel<F, 4><<<(unsigned)tiles, kThreads, 0, s>>>(x, y, F{});
    done = tiles * kTile;
  }
  if (done < n) {
    const int64_t rem = n - done;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(rem, kThreads), (int64_t)sm_count() * 8));
    elementwise_scalar_kernel<F><<<grid, kThreads, 0, s>>>(x, y, done, n, F{});
  }
  return check_launch(name);
}

// y[i, j] = a[i] * b[i, j]: diag(a) @ B without the N x N matrix
// (candidates/12_Matmul_with_diagonal_matrices_/v1.py:10-17).  One kTile tile
// per CTA as above; cols % W == 0 keeps every vector inside one row, and
// a[row] comes from L1/L2.
template <int W>
__global__ void __launch_bounds__(kThreads)
row_scale_tile_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ y,
                      int64_t cols) {
  constexpr int U = kTile / (kThreads * W);
  const int64_t base = (int64_t)blockIdx.x * kTile + threadIdx.x * W;
  f32x8 v[U];
  float sc[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    v[u] = Vec<W>::ld(b + base + u * kThreads * W);
    sc[u] = __ldg(a + (base + u * kThreads * W) / cols);
  }
#pragma unroll
  for (int u = 0; u < U; ++u) {
#pragma unroll
    for (int k = 0; k < W; ++k) v[u].v[k] *= sc[u];
    Vec<W>::st(y + base + u * kThreads * W, v[u]);
  }
}

__global__ void __launch_bounds__(kThreads)
row_scale_scalar_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ y,
                        int64_t begin, int64_t n, int64_t cols) {
  for (int64_t i = begin + (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * kThreads)
    y[i] = a[i / cols] * b[i];
}

}  // namespace
}  // namespace kb

extern "C" {

int kb_diag_matmul_f32(const float* a, const float* b, float* y, int64_t rows, int64_t cols,
                       kbStream stream) {
  const char* name = "kb_diag_matmul_f32";
  KB_REQUIRE(rows >= 0 && cols >= 0, KB_ERR_INVALID_ARG, "%s: negative size", name);
  if (rows == 0 || cols == 0) return KB_OK;
  KB_REQUIRE(a && b && y, KB_ERR_INVALID_ARG, "%s: null pointer", name);
  const int64_t n = rows * cols;
  const int64_t tiles = n / kb::kTile;
  KB_REQUIRE(tiles <= 0x7fffffff, KB_ERR_UNSUPPORTED, "%s: too large", name);
  int64_t done = 0;
  if (tiles > 0 && cols % 8 == 0 && kb::aligned32(b) && kb::aligned32(y)) {
    kb::row_scale_tile_kernel<8><<<(unsigned)tiles, kb::kThreads, 0, stream>>>(a, b, y, cols);
    done = tiles * kb::kTile;
  } else if (tiles > 0 && cols % 4 == 0 && kb::aligned16(b) && kb::aligned16(y)) {
    kb::row_scale_tile_kernel<4><<<(unsigned)tiles, kb::kThreads, 0, stream>>>(a, b, y, cols);
    done = tiles * kb::kTile;
  }
  if (done < n) {
    const int grid = (int)std::max<int64_t>(
        1, std::min<int64_t>(kb::ceil_div(n - done, kb::kThreads), (int64_t)kb::sm_count() * 8));
    kb::row_scale_scalar_kernel<<<grid, kb::kThreads, 0, stream>>>(a, b, y, done, n, cols);
  }
  return kb::check_launch(name);
}

int kb_gelu_tanh_f32(const float* x, float* y, int64_t n, kbStream stream) {
  return kb::launch_elementwise<kb::GeluTanh>("kb_gelu_tanh_f32", x, y, n, stream);
}
int kb_gelu_erf_f32(const float* x, float* y, int64_t n, kbStream stream) {
  return kb::launch_elementwise<kb::GeluErf>("kb_gelu_erf_f32", x, y, n, stream);
}
int kb_swish_f32(const float* x, float* y, int64_t n, kbStream stream) {
  return kb::launch_elementwise<kb::Swish>("kb_swish_f32", x, y, n, stream);
}
int kb_relu_f32(const float* x, float* y, int64_t n, kbStream stream) {
  return kb::launch_elementwise<kb::Relu>("kb_relu_f32", x, y, n, stream);
}

}  // extern "C"
