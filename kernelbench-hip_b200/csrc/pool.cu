// pool.cu — 2D max pooling over NCHW fp32 with stride, padding and dilation
// honoured (the reference kernel dropped stride and dilation,
// candidates/42_Max_Pooling_2D/v1.py:24-27).
//
// Fast path, kernel 3 / stride 2 / pad 1 / dilation 1 with W % 4 == 0: a CTA
// of W/4 threads owns a 64-output-row strip of one (n, c) plane.  Thread t
// reads input columns 4t..4t+3 as one float4 (column 4t-1 comes from the
// neighbouring lane by shuffle, across warps through shared memory),
// produces output columns 2t and 2t+1, and
// walks down the strip four output rows (eight input rows, loaded together)
// at a time, carrying the shared input row between consecutive output rows,
// so every input element is read from HBM once (plus one halo row per strip).
// Generic path: one thread per output element.
#include "kb_common.cuh"

namespace kb {
namespace {

// torch.max_pool2d order: a NaN anywhere in the window wins.
__device__ __forceinline__ float nanmax(float m, float v) { return (v > m || v != v) ? v : m; }

constexpr int kStripRows = 64;
constexpr int kRowsPerIter = 4;  // output rows per iteration: 8 input rows in flight

// 3-wide horizontal maxima of one input row for output columns 2t, 2t+1,
// given column 4t-1 (`left`).
__device__ __forceinline__ void hmax_row(const float4 v, float left, float& h0, float& h1) {
  h0 = nanmax(nanmax(left, v.x), v.y);
  h1 = nanmax(nanmax(v.y, v.z), v.w);
}

constexpr int kMaxWarps = 32;

__global__ void maxpool_k3s2p1_kernel(const float* __restrict__ x, float* __restrict__ y,
                                      int64_t H, int64_t W, int64_t OH, int64_t OW) {
  // column 4t-1 of thread t: lanes 1..31 take it from the neighbouring lane,
  // lane 0 from the previous warp's lane 31 through shared memory
  __shared__ float s_edge[2][kMaxWarps][2 * kRowsPerIter];
  const int64_t plane = blockIdx.y;
  const int t = threadIdx.x;                 // float4 column group
  const int lane = t & 31, warp = t >> 5;
  const float* xp = x + plane * H * W;
  float* yp = y + plane * OH * OW;
  const int64_t oh0 = (int64_t)blockIdx.x * kStripRows;
  const int64_t oh1 = std::min<int64_t>(oh0 + kStripRows, OH);
  const bool two = 2 * t + 1 < OW, one = 2 * t < OW;

  // carried maxima of input row 2*oh - 1 (padding above the first row)
  float c0 = -INFINITY, c1 = -INFINITY;
  if (oh0 > 0) {
    const float4 v = ld_stream(reinterpret_cast<const float4*>(xp + (2 * oh0 - 1) * W) + t);
    if (lane == 31) s_edge[1][warp][0] = v.w;
    __syncthreads();
    float left = __shfl_up_sync(0xffffffffu, v.w, 1);
    if (lane == 0) left = warp > 0 ? s_edge[1][warp - 1][0] : -INFINITY;
    hmax_row(v, left, c0, c1);
  }
  int buf = 0;
  for (int64_t oh = oh0; oh < oh1; oh += kRowsPerIter, buf ^= 1) {
    // input rows 2*oh .. 2*oh + 7, loaded together (rows past H are padding)
    float4 v[2 * kRowsPerIter];
#pragma unroll
    for (int j = 0; j < 2 * kRowsPerIter; ++j) {
      const int64_t r = 2 * oh + j;
      v[j] = (r < H && oh + j / 2 < oh1)
                 ? ld_stream(reinterpret_cast<const float4*>(xp + r * W) + t)
                 : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    }
    if (lane == 31) {
#pragma unroll
      for (int j = 0; j < 2 * kRowsPerIter; ++j) s_edge[buf][warp][j] = v[j].w;
    }
    __syncthreads();  // double-buffered s_edge: one barrier per iteration suffices
    float left[2 * kRowsPerIter];
#pragma unroll
    for (int j = 0; j < 2 * kRowsPerIter; ++j) {
      left[j] = __shfl_up_sync(0xffffffffu, v[j].w, 1);
      if (lane == 0) left[j] = warp > 0 ? s_edge[buf][warp - 1][j] : -INFINITY;
    }
#pragma unroll
    for (int i = 0; i < kRowsPerIter; ++i) {
      if (oh + i >= oh1) break;  // uniform across the CTA
      float a0, a1, b0, b1;
      hmax_row(v[2 * i], left[2 * i], a0, a1);
      hmax_row(v[2 * i + 1], left[2 * i + 1], b0, b1);  // a padding row is all -inf
      const float o0 = nanmax(nanmax(c0, a0), b0);
      const float o1 = nanmax(nanmax(c1, a1), b1);
      float* orow = yp + (oh + i) * OW;
      if (two) {
        st_stream(reinterpret_cast<float2*>(orow) + t, make_float2(o0, o1));
      } else if (one) {
        orow[2 * t] = o0;
      }
      c0 = b0;
      c1 = b1;
    }
  }
}

__global__ void maxpool_generic_kernel(const float* __restrict__ x, float* __restrict__ y,
                                       int64_t NC, int64_t H, int64_t W, int64_t OH, int64_t OW,
                                       int k, int stride, int pad, int dil) {
  const int64_t total = NC * OH * OW;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t ow = idx % OW;
    const int64_t oh = (idx / OW) % OH;
    const int64_t p = idx / (OW * OH);
    const float* xp = x + p * H * W;
    float m = -INFINITY;
    for (int u = 0; u < k; ++u) {
      const int64_t ih = oh * stride - pad + (int64_t)u * dil;
      if (ih < 0 || ih >= H) continue;
      for (int v = 0; v < k; ++v) {
        const int64_t iw = ow * stride - pad + (int64_t)v * dil;
        if (iw < 0 || iw >= W) continue;
        m = nanmax(m, xp[ih * W + iw]);
      }
    }
    y[idx] = m;
  }
}

}  // namespace
}  // namespace kb

extern "C" {

int kb_maxpool2d_f32(const float* x, float* y, int64_t N, int64_t C, int64_t H, int64_t W,
                     int64_t OH, int64_t OW, int kernel, int stride, int pad, int dilation,
                     kbStream stream) {
  const char* name = "kb_maxpool2d_f32";
  KB_REQUIRE(N >= 0 && C >= 0 && H >= 0 && W >= 0 && OH >= 0 && OW >= 0, KB_ERR_INVALID_ARG,
             "%s: negative size", name);
  KB_REQUIRE(kernel >= 1 && stride >= 1 && dilation >= 1 && pad >= 0 && 2 * pad <= kernel,
             KB_ERR_INVALID_ARG, "%s: bad window (k=%d s=%d p=%d d=%d)", name, kernel, stride,
             pad, dilation);
  // output extent as torch (floor mode)
  const int64_t eh = (H + 2 * pad - (int64_t)dilation * (kernel - 1) - 1);
  const int64_t ew = (W + 2 * pad - (int64_t)dilation * (kernel - 1) - 1);
  KB_REQUIRE(eh >= 0 && ew >= 0 && OH == eh / stride + 1 && OW == ew / stride + 1,
             KB_ERR_INVALID_ARG, "%s: output %lldx%lld does not match the window", name,
             (long long)OH, (long long)OW);
  const int64_t NC = N * C;
  if (NC == 0 || OH == 0 || OW == 0) return KB_OK;
  KB_REQUIRE(x && y, KB_ERR_INVALID_ARG, "%s: null pointer", name);
  const bool fast = kernel == 3 && stride == 2 && pad == 1 && dilation == 1 && W % 4 == 0 &&
                    W / 4 <= 1024 && W >= 4 && kb::aligned16(x) && kb::aligned16(y) &&
                    OW % 2 == 0 && NC <= 65535;
  if (fast) {
    const int threads = (int)(W / 4);
    dim3 grid((unsigned)kb::ceil_div(OH, kb::kStripRows), (unsigned)NC);
    // the shuffle assumes whole warps: pad the CTA to a multiple of 32
    if (threads % 32 == 0) {
      kb::maxpool_k3s2p1_kernel<<<grid, threads, 0, stream>>>(x, y, H, W, OH, OW);
      return kb::check_launch(name);
    }
  }
  const int64_t total = NC * OH * OW;
  const int grid = (int)std::min<int64_t>(kb::ceil_div(total, 256), (int64_t)kb::sm_count() * 16);
  kb::maxpool_generic_kernel<<<grid, 256, 0, stream>>>(x, y, NC, H, W, OH, OW, kernel, stride,
                                                         pad, dilation);
  return kb::check_launch(name);
}

}  // extern "C"
