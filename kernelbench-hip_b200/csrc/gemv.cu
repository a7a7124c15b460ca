// gemv.cu — y[M] = A[M, K] x[K], fp32, HBM-bound (0.5 FLOP/byte).
//
// 256-thread CTAs stream A once with 128-bit evict-first loads, 8 float4 of
// each row in flight per thread; x (4 MB at K = 2^20) stays resident in the
// 126 MB L2 and is shared by every CTA.  Each CTA takes two rows, so every x
// vector fetched from L2 serves two rows of A: the SM-side load traffic is
// 1.5x the HBM bytes instead of 2x, which took the [4096, 2^20] launch from
// 2.60 to 2.30 ms (7.4 TB/s of A).  Below 2 rows per SM, one row per CTA
// keeps more CTAs in flight.  The row sum is a fixed shuffle tree, so y is
// deterministic and independent of the rows per CTA (the reference split
// rows into 32K chunks and combined them with fp32 atomics,
// candidates/4_Matrix_vector_multiplication_/v1.py:16-33).
#include "kb_common.cuh"

namespace kb {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 8;

// R rows per CTA: each x vector loaded from L2 serves R rows of A, so the
// SM-side load traffic is (1 + 1/R)x the HBM bytes.  Per row, thread t sums
// float4 columns t + u*256 + k*256*U into accumulator u, and the row total
// goes through one fixed tree, so the results do not depend on R.  A CTA
// whose last rows lie beyond M re-reads row M-1 for them and discards the
// sums.
template <int R, int U>
__global__ void __launch_bounds__(kThreads, 2)
gemv_rows_kernel(const float* __restrict__ A, const float* __restrict__ x, float* __restrict__ y,
                 int64_t M, int64_t K) {
  constexpr int NW = kThreads / 32;
  __shared__ float red[R][NW];
  const int64_t row0 = (int64_t)blockIdx.x * R;
  const int64_t nvec = K / 4;
  const float4* x4 = reinterpret_cast<const float4*>(x);
  const float4* a4[R];
#pragma unroll
  for (int r = 0; r < R; ++r) a4[r] = reinterpret_cast<const float4*>(A + min(row0 + r, M - 1) * K);
  float acc[R][U];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int u = 0; u < U; ++u) acc[r][u] = 0.f;
  int64_t i = threadIdx.x;
  const int64_t step = (int64_t)kThreads * U;
  for (; i + (U - 1) * kThreads < nvec; i += step) {
    float4 b[U], a[R][U];
#pragma unroll
    for (int u = 0; u < U; ++u) b[u] = __ldg(x4 + i + u * kThreads);
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int u = 0; u < U; ++u) a[r][u] = ld_stream(a4[r] + i + u * kThreads);
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int u = 0; u < U; ++u)
        acc[r][u] = fmaf(a[r][u].x, b[u].x,
                         fmaf(a[r][u].y, b[u].y, fmaf(a[r][u].z, b[u].z, fmaf(a[r][u].w, b[u].w, acc[r][u]))));
  }
  for (; i < nvec; i += kThreads) {
    const float4 b = __ldg(x4 + i);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float4 a = ld_stream(a4[r] + i);
      acc[r][0] = fmaf(a.x, b.x, fmaf(a.y, b.y, fmaf(a.z, b.z, fmaf(a.w, b.w, acc[r][0]))));
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float s[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    s[r] = 0.f;
#pragma unroll
    for (int u = 0; u < U; ++u) s[r] += acc[r][u];
    const float* ar = reinterpret_cast<const float*>(a4[r]);
    for (int64_t j = nvec * 4 + threadIdx.x; j < K; j += kThreads) s[r] = fmaf(ar[j], x[j], s[r]);
    s[r] = warp_sum(s[r]);
    if (lane == 0) red[r][warp] = s[r];
  }
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float t = lane < NW ? red[r][lane] : 0.f;
      t = warp_sum(t);
      if (lane == 0 && row0 + r < M) y[row0 + r] = t;
    }
  }
}

__global__ void __launch_bounds__(kThreads)
gemv_scalar_kernel(const float* __restrict__ A, const float* __restrict__ x,
                   float* __restrict__ y, int64_t K) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  float s = 0.f;
  for (int64_t j = threadIdx.x; j < K; j += kThreads) s = fmaf(A[row * K + j], x[j], s);
  s = block_sum<kThreads>(s, red);
  if (threadIdx.x == 0) y[row] = s;
}

}  // namespace
}  // namespace kb

extern "C" {

int kb_gemv_f32(const float* A, const float* x, float* y, int64_t M, int64_t K, kbStream stream) {
  const char* name = "kb_gemv_f32";
  KB_REQUIRE(M >= 0 && K >= 0, KB_ERR_INVALID_ARG, "%s: negative size", name);
  if (M == 0) return KB_OK;
  KB_REQUIRE(y && (K == 0 || (A && x)), KB_ERR_INVALID_ARG, "%s: null pointer", name);
  KB_REQUIRE(M <= 0x7fffffff, KB_ERR_UNSUPPORTED, "%s: M too large", name);
  if (K % 4 == 0 && kb::aligned16(A) && kb::aligned16(x)) {
    if (M >= 2 * kb::sm_count())
      kb::gemv_rows_kernel<2, kb::kUnroll><<<(unsigned)((M + 1) / 2), kb::kThreads, 0, stream>>>(A, x, y, M, K);
    else
      kb::gemv_rows_kernel<1, kb::kUnroll><<<(unsigned)M, kb::kThreads, 0, stream>>>(A, x, y, M, K);
  } else
    kb::gemv_scalar_kernel<<<(unsigned)M, kb::kThreads, 0, stream>>>(A, x, y, K);
  return kb::check_launch(name);
}

}  // extern "C"
