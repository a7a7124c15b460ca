// pool.cu — 2D max and average pooling over NCHW fp32 with stride, padding
// and dilation honoured (the reference max-pool kernel dropped stride and
// dilation, candidates/42_Max_Pooling_2D/v1.py:24-27; average pooling has no
// reference candidate and follows torch.nn.functional.avg_pool2d: floor mode,
// count_include_pad, divisor_override).
//
// Fast path, kernel 3 / stride 2 / pad 1 / dilation 1 with W % 4 == 0 (for
// average pooling also count_include_pad or no padded window, i.e. every
// divisor 9, and no divisor override): a CTA
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

// Window reductions of the strip kernel.  Padding is the identity of the
// combine; finish() turns the combined 3x3 window into the output.
struct MaxOp {
  static constexpr float kPad = -INFINITY;
  static __device__ __forceinline__ float combine(float a, float b) { return nanmax(a, b); }
  static __device__ __forceinline__ float finish(float v) { return v; }
};
struct AvgOp {  // sum of the 3x3 window (padding counts as 0) / 9
  static constexpr float kPad = 0.0f;
  static __device__ __forceinline__ float combine(float a, float b) { return a + b; }
  static __device__ __forceinline__ float finish(float v) { return v / 9.0f; }
};

constexpr int kStripRows = 64;
constexpr int kRowsPerIter = 4;  // output rows per iteration: 8 input rows in flight

// 3-wide horizontal reductions of one input row for output columns 2t, 2t+1,
// given column 4t-1 (`left`).
template <class P>
__device__ __forceinline__ void hred_row(const float4 v, float left, float& h0, float& h1) {
  h0 = P::combine(P::combine(left, v.x), v.y);
  h1 = P::combine(P::combine(v.y, v.z), v.w);
}

constexpr int kMaxWarps = 32;

template <class P>
__global__ void pool_k3s2p1_kernel(const float* __restrict__ x, float* __restrict__ y,
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

  // carried reductions of input row 2*oh - 1 (padding above the first row)
  float c0 = P::kPad, c1 = P::kPad;
  if (oh0 > 0) {
    const float4 v = ld_stream(reinterpret_cast<const float4*>(xp + (2 * oh0 - 1) * W) + t);
    if (lane == 31) s_edge[1][warp][0] = v.w;
    __syncthreads();
    float left = __shfl_up_sync(0xffffffffu, v.w, 1);
    if (lane == 0) left = warp > 0 ? s_edge[1][warp - 1][0] : P::kPad;
    hred_row<P>(v, left, c0, c1);
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
                 : make_float4(P::kPad, P::kPad, P::kPad, P::kPad);
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
      if (lane == 0) left[j] = warp > 0 ? s_edge[buf][warp - 1][j] : P::kPad;
    }
#pragma unroll
    for (int i = 0; i < kRowsPerIter; ++i) {
      if (oh + i >= oh1) break;  // uniform across the CTA
      float a0, a1, b0, b1;
      hred_row<P>(v[2 * i], left[2 * i], a0, a1);
      hred_row<P>(v[2 * i + 1], left[2 * i + 1], b0, b1);  // a padding row is all kPad
      const float o0 = P::finish(P::combine(P::combine(c0, a0), b0));
      const float o1 = P::finish(P::combine(P::combine(c1, a1), b1));
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

// torch avg_pool2d: the window is clipped to the padded input for the
// divisor (count_include_pad) and to the real input for the sum; a nonzero
// divisor_override replaces the divisor.  Sum in window order (rows, then
// columns), then one division.
__global__ void avgpool_generic_kernel(const float* __restrict__ x, float* __restrict__ y,
                                       int64_t NC, int64_t H, int64_t W, int64_t OH, int64_t OW,
                                       int k, int stride, int pad, int count_include_pad,
                                       int divisor_override) {
  const int64_t total = NC * OH * OW;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t ow = idx % OW;
    const int64_t oh = (idx / OW) % OH;
    const int64_t p = idx / (OW * OH);
    int64_t hs = oh * stride - pad, ws = ow * stride - pad;
    int64_t he = hs + k < H + pad ? hs + k : H + pad;
    int64_t we = ws + k < W + pad ? ws + k : W + pad;
    const int64_t pool_size = (he - hs) * (we - ws);
    hs = hs > 0 ? hs : 0;
    ws = ws > 0 ? ws : 0;
    he = he < H ? he : H;
    we = we < W ? we : W;
    const float* xp = x + p * H * W;
    float s = 0.0f;
    for (int64_t ih = hs; ih < he; ++ih)
      for (int64_t iw = ws; iw < we; ++iw) s += xp[ih * W + iw];
    int64_t div;
    if (divisor_override)
      div = divisor_override;
    else
      div = count_include_pad ? pool_size : (he - hs) * (we - ws);
    y[idx] = s / (float)div;  // windows always overlap the input: div >= 1
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
      kb::pool_k3s2p1_kernel<kb::MaxOp><<<grid, threads, 0, stream>>>(x, y, H, W, OH, OW);
      return kb::check_launch(name);
    }
  }
  const int64_t total = NC * OH * OW;
  const int grid = (int)std::min<int64_t>(kb::ceil_div(total, 256), (int64_t)kb::sm_count() * 16);
  kb::maxpool_generic_kernel<<<grid, 256, 0, stream>>>(x, y, NC, H, W, OH, OW, kernel, stride,
                                                         pad, dilation);
  return kb::check_launch(name);
}

int kb_avgpool2d_f32(const float* x, float* y, int64_t N, int64_t C, int64_t H, int64_t W,
                     int64_t OH, int64_t OW, int kernel, int stride, int pad, int count_include_pad,
                     int divisor_override, kbStream stream) {
  const char* name = "kb_avgpool2d_f32";
  KB_REQUIRE(N >= 0 && C >= 0 && H >= 0 && W >= 0 && OH >= 0 && OW >= 0, KB_ERR_INVALID_ARG,
             "%s: negative size", name);
  KB_REQUIRE(kernel >= 1 && stride >= 1 && pad >= 0 && 2 * pad <= kernel && divisor_override >= 0,
             KB_ERR_INVALID_ARG, "%s: bad window (k=%d s=%d p=%d divisor %d)", name, kernel, stride,
             pad, divisor_override);
  const int64_t eh = H + 2 * pad - kernel, ew = W + 2 * pad - kernel;
  KB_REQUIRE(eh >= 0 && ew >= 0 && OH == eh / stride + 1 && OW == ew / stride + 1,
             KB_ERR_INVALID_ARG, "%s: output %lldx%lld does not match the window", name,
             (long long)OH, (long long)OW);
  const int64_t NC = N * C;
  if (NC == 0 || OH == 0 || OW == 0) return KB_OK;
  KB_REQUIRE(x && y, KB_ERR_INVALID_ARG, "%s: null pointer", name);
  // every window of k3 s2 p1 in floor mode lies inside the padded input, so
  // with count_include_pad (or an override of 9) each divisor is 9
  const bool fast = kernel == 3 && stride == 2 && pad == 1 && W % 4 == 0 && W / 4 <= 1024 &&
                    W >= 4 && kb::aligned16(x) && kb::aligned16(y) && OW % 2 == 0 && NC <= 65535 &&
                    (divisor_override == 0 ? count_include_pad != 0 : divisor_override == 9) &&
                    (W / 4) % 32 == 0;
  if (fast) {
    dim3 grid((unsigned)kb::ceil_div(OH, kb::kStripRows), (unsigned)NC);
    kb::pool_k3s2p1_kernel<kb::AvgOp><<<grid, (unsigned)(W / 4), 0, stream>>>(x, y, H, W, OH, OW);
    return kb::check_launch(name);
  }
  const int64_t total = NC * OH * OW;
  const int grid = (int)std::min<int64_t>(kb::ceil_div(total, 256), (int64_t)kb::sm_count() * 16);
  kb::avgpool_generic_kernel<<<grid, 256, 0, stream>>>(x, y, NC, H, W, OH, OW, kernel, stride, pad,
                                                        count_include_pad, divisor_override);
  return kb::check_launch(name);
}

}  // extern "C"
