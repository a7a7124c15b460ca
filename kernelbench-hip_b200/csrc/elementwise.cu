// elementwise.cu — streaming activation kernels (tanh-GELU, erf-GELU, Swish,
// ReLU).
//
// One persistent grid (SMs x resident CTAs) walks the tensor in tiles of
// NT x UNROLL float4 vectors: every thread issues UNROLL independent 128-bit
// streaming loads before it computes, so each SM keeps ~100 KB of reads in
// flight, which is what HBM3e needs to stay saturated.  A scalar path covers
// the n % 4 tail and unaligned views.
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
constexpr int kUnroll = 4;

template <class F>
__global__ void __launch_bounds__(kThreads)
elementwise_vec4_kernel(const float4* __restrict__ x, float4* __restrict__ y,
                        int64_t nvec, F f) {
  const int64_t tile = (int64_t)kThreads * kUnroll;
  const int64_t ntiles = nvec / tile;
  for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
    const int64_t base = t * tile + threadIdx.x;
    float4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) v[u] = ld_stream(x + base + u * kThreads);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      float4 r;
      r.x = f(v[u].x);
      r.y = f(v[u].y);
      r.z = f(v[u].z);
      r.w = f(v[u].w);
      st_stream(y + base + u * kThreads, r);
    }
  }
  // leftover whole vectors (fewer than one tile): spread over the grid
  for (int64_t i = ntiles * tile + (int64_t)blockIdx.x * kThreads + threadIdx.x; i < nvec;
       i += (int64_t)gridDim.x * kThreads) {
    float4 v = ld_stream(x + i), r;
    r.x = f(v.x);
    r.y = f(v.y);
    r.z = f(v.z);
    r.w = f(v.w);
    st_stream(y + i, r);
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
  static int blocks_per_sm = 0;
  if (blocks_per_sm == 0) {
    int b = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, elementwise_vec4_kernel<F>, kThreads, 0);
    blocks_per_sm = b > 0 ? b : 4;
  }
  const int sms = sm_count();
  int64_t done = 0;
  if (aligned16(x) && aligned16(y) && n >= 4) {
    const int64_t nvec = n / 4;
    const int64_t want = ceil_div(nvec, (int64_t)kThreads * kUnroll);
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)sms * blocks_per_sm));
    elementwise_vec4_kernel<F><<<grid, kThreads, 0, s>>>(
        reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(y), nvec, F{});
    done = nvec * 4;
  }
  if (done < n) {
    const int64_t rem = n - done;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(rem, kThreads), (int64_t)sms * 8));
    elementwise_scalar_kernel<F><<<grid, kThreads, 0, s>>>(x, y, done, n, F{});
  }
  return check_launch(name);
}

// y[i, j] = a[i] * b[i, j]: diag(a) @ B without the N x N matrix
// (candidates/12_Matmul_with_diagonal_matrices_/v1.py:10-17).  cols % 4 == 0
// and aligned pointers: each float4 lies in one row, a[row] comes from L1/L2.
__global__ void __launch_bounds__(kThreads)
row_scale_vec4_kernel(const float* __restrict__ a, const float4* __restrict__ b, float4* __restrict__ y,
                      int64_t nvec, int64_t cols4) {
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < nvec;
       i += (int64_t)gridDim.x * kThreads) {
    const float s = __ldg(a + i / cols4);
    const float4 v = ld_stream(b + i);
    st_stream(y + i, make_float4(s * v.x, s * v.y, s * v.z, s * v.w));
  }
}

__global__ void __launch_bounds__(kThreads)
row_scale_scalar_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ y,
                        int64_t n, int64_t cols) {
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kThreads)
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
  const int grid_cap = kb::sm_count() * 8;
  if (cols % 4 == 0 && kb::aligned16(b) && kb::aligned16(y)) {
    const int64_t nvec = n / 4;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(kb::ceil_div(nvec, kb::kThreads), grid_cap));
    kb::row_scale_vec4_kernel<<<grid, kb::kThreads, 0, stream>>>(
        a, reinterpret_cast<const float4*>(b), reinterpret_cast<float4*>(y), nvec, cols / 4);
  } else {
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(kb::ceil_div(n, kb::kThreads), grid_cap));
    kb::row_scale_scalar_kernel<<<grid, kb::kThreads, 0, stream>>>(a, b, y, n, cols);
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
