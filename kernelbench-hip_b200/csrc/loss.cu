// loss.cu — cross-entropy loss over class logits, mean reduction
// (torch.nn.functional.cross_entropy(logits [rows, classes], targets int64
// [rows]) with weight None, ignore_index, no label smoothing).  The
// reference has no candidate for it (its problem list names
// 95_CrossEntropyLoss as not attempted).
//
//   loss_i = logsumexp(x_i) - x_i[t_i]   for t_i != ignore_index
//   out    = sum_i loss_i / #{i : t_i != ignore_index}
//
// Row kernel: persistent CTAs walk the rows.  Rows of up to NT * 4 * VPT
// classes are held in registers (128-bit evict-first loads), so the max and
// the sum of exp(x - max) come from one read; longer or unaligned rows take
// a one-pass online (max, sum-exp) kernel (one CTA per row).  The next row
// (and its target index) is loaded while the current row is reduced, and
// the thread that holds the target's logit publishes it through shared
// memory, so a row ends without a dependent global load.  Each CTA adds its
// rows' losses, in row order, into one (sum, count) workspace slot (double),
// and a one-CTA finish sums the slots in a fixed order: the result is
// bit-identical run to run on a device (no atomics).  A target outside
// [0, classes) that is not ignore_index makes its row loss, and so the mean,
// NaN.
#include "kb_common.cuh"

namespace kb {
namespace {

constexpr float kLog2e = 1.4426950408889634f;

// exp(x - m) is evaluated as 2^(x log2(e) - m log2(e)): one FMA and the
// hardware's ex2.approx.ftz instruction per logit (PTX ISA).  A term below
// 2^-126 becomes 0 instead of subnormal, far below the fp32 resolution of
// the row's sum; 1.3 % faster than exp2f at [32768, 4096] with the same loss.
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
struct MaxSumE {
  float m, s;
};
__device__ __forceinline__ float rescale(float m, float M) {
  return m == M ? 1.0f : exp2f((m - M) * kLog2e);  // also covers m == M == -inf
}
__device__ __forceinline__ MaxSumE combine(MaxSumE a, MaxSumE b) {
  const float M = fmaxf(a.m, b.m);
  return {M, a.s * rescale(a.m, M) + b.s * rescale(b.m, M)};
}

template <int NT>
__device__ __forceinline__ MaxSumE block_maxsum(MaxSumE v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    v = combine(v, MaxSumE{__shfl_xor_sync(0xffffffffu, v.m, o), __shfl_xor_sync(0xffffffffu, v.s, o)});
  constexpr int NW = NT / 32;
  if (NW == 1) return v;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    red[warp] = v.m;
    red[32 + warp] = v.s;
  }
  __syncthreads();
  MaxSumE r = lane < NW ? MaxSumE{red[lane], red[32 + lane]} : MaxSumE{-INFINITY, 0.0f};
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    r = combine(r, MaxSumE{__shfl_xor_sync(0xffffffffu, r.m, o), __shfl_xor_sync(0xffffffffu, r.s, o)});
  return r;
}

// One-barrier block reductions for the row kernel: every thread gets the
// result; `red` (32 floats) may be rewritten only after the next barrier.
template <int NT>
__device__ __forceinline__ float block_max_1b(float v, float* red) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_max(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  return warp_max(lane < NW ? red[lane] : -INFINITY);
}
template <int NT>
__device__ __forceinline__ float block_sum_1b(float v, float* red) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  return warp_sum(lane < NW ? red[lane] : 0.0f);
}

// Adds one row's loss, from its logsumexp pieces and the target's logit
// (published in shared memory by the thread that loaded it), to a running
// (sum, count); thread 0 only.
__device__ __forceinline__ void add_row(int64_t classes, int64_t target, int64_t ignore_index, float M,
                                        float S, float picked, double& sum, double& count) {
  if (target == ignore_index) return;
  count += 1.0;
  if (target < 0 || target >= classes)
    sum += __longlong_as_double(0x7ff8000000000000ll);  // NaN
  else
    sum += (double)(M + logf(S)) - (double)picked;
}

__device__ __forceinline__ float component(const float4 v, int c) {
  return c == 0 ? v.x : c == 1 ? v.y : c == 2 ? v.z : v.w;
}

template <int NT, int VPT>
__global__ void __launch_bounds__(NT)
ce_row_kernel(const float* __restrict__ x, const int64_t* __restrict__ targets, int64_t rows,
              int64_t classes, int64_t ignore_index, double* __restrict__ part_sum,
              double* __restrict__ part_count) {
  // persistent: rows blockIdx.x, + gridDim.x, ...; the next row's loads are
  // issued before this row is reduced.  Per row: block max, then the sum of
  // exp(x - max) against that max, then one plain block sum (two one-barrier
  // reductions; a (max, sum-exp) pair combine would cost two exponentials
  // per shuffle step in every thread).  Shared buffers alternate by row
  // parity: a buffer is rewritten two rows later, after every thread has
  // passed the barriers of the row in between.
  __shared__ float red[2][64];
  __shared__ float s_pick[2];
  const int64_t nvec = classes / 4;
  auto load = [&](int64_t r, float4 (&dst)[VPT], int64_t& tgt) {
    tgt = __ldg(targets + r);  // one address: a broadcast
    const float4* x4 = reinterpret_cast<const float4*>(x + r * classes);
#pragma unroll
    for (int u = 0; u < VPT; ++u) {
      const int64_t i = threadIdx.x + (int64_t)u * NT;
      dst[u] = i < nvec ? ld_stream(x4 + i) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    }
  };
  float4 nv[VPT];
  int64_t ntarget = 0;
  int64_t row = blockIdx.x;
  __shared__ double s_acc[2];  // thread 0: (sum, count) of this CTA's rows, in row order
  if (threadIdx.x == 0) s_acc[0] = s_acc[1] = 0.0;
  if (row < rows) load(row, nv, ntarget);
  for (int buf = 0; row < rows; row += gridDim.x, buf ^= 1) {
    float4 v[VPT];
#pragma unroll
    for (int u = 0; u < VPT; ++u) v[u] = nv[u];
    const int64_t target = ntarget;
    if (row + gridDim.x < rows) load(row + gridDim.x, nv, ntarget);
    float m = -INFINITY;
    // vector slot of the target relative to this thread (-1: none here)
    const int tslot = (target >= 0 && target < classes) ? (int)(target >> 2) - (int)threadIdx.x : -1;
#pragma unroll
    for (int u = 0; u < VPT; ++u) {
      m = fmaxf(m, fmaxf(fmaxf(v[u].x, v[u].y), fmaxf(v[u].z, v[u].w)));
      if (tslot == u * NT) s_pick[buf] = component(v[u], (int)(target & 3));  // publish the target logit
    }
    const float M = block_max_1b<NT>(m, red[buf]);
    float s = 0.0f;
    if (M != -INFINITY) {
      const float ml = -M * kLog2e;
#pragma unroll
      for (int u = 0; u < VPT; ++u)
        s += (ex2_ftz(fmaf(v[u].x, kLog2e, ml)) + ex2_ftz(fmaf(v[u].y, kLog2e, ml))) +
             (ex2_ftz(fmaf(v[u].z, kLog2e, ml)) + ex2_ftz(fmaf(v[u].w, kLog2e, ml)));
    }
    // a NaN logit: fmaxf drops it from the max but its exponential makes the sum NaN
    const float S = block_sum_1b<NT>(s, red[buf] + 32);
    if (threadIdx.x == 0) add_row(classes, target, ignore_index, M, S, s_pick[buf], s_acc[0], s_acc[1]);
  }
  if (threadIdx.x == 0) {
    part_sum[blockIdx.x] = s_acc[0];
    part_count[blockIdx.x] = s_acc[1];
  }
}

template <int NT>
__global__ void __launch_bounds__(NT)
ce_online_kernel(const float* __restrict__ x, const int64_t* __restrict__ targets, int64_t classes,
                 int64_t ignore_index, double* __restrict__ part_sum, double* __restrict__ part_count) {
  __shared__ float red[64];
  __shared__ float s_pick;
  const int64_t row = blockIdx.x;
  const int64_t target = __ldg(targets + row);
  const float* xr = x + row * classes;
  MaxSumE p{-INFINITY, 0.0f};
  for (int64_t i = threadIdx.x; i < classes; i += NT) {
    const float xi = xr[i];
    if (i == target) s_pick = xi;
    if (xi > p.m) {
      p.s = p.s * rescale(p.m, xi) + 1.0f;
      p.m = xi;
    } else {
      p.s += exp2f((xi - p.m) * kLog2e);  // NaN (or -inf - -inf) lands here and propagates
    }
  }
  const MaxSumE r = block_maxsum<NT>(p, red);
  if (threadIdx.x == 0) {
    double sum = 0.0, count = 0.0;
    add_row(classes, target, ignore_index, r.m, r.s, s_pick, sum, count);
    part_sum[row] = sum;
    part_count[row] = count;
  }
}

constexpr int kFinishThreads = 1024;

constexpr int kFinishUnroll = 8;

// out = sum(part_sum) / sum(part_count) over n partials, in a fixed order;
// with `total` set, the two sums are written there instead (sharded form)
__global__ void __launch_bounds__(kFinishThreads)
ce_finish_kernel(const double* __restrict__ part_sum, const double* __restrict__ part_count, int64_t n,
                 float* __restrict__ out, double* __restrict__ total = nullptr) {
  __shared__ double red[32];
  // kFinishUnroll independent slots per thread in flight; partial sums are
  // combined in a fixed order, so the result does not depend on timing
  double ps[kFinishUnroll], pc[kFinishUnroll];
#pragma unroll
  for (int u = 0; u < kFinishUnroll; ++u) ps[u] = pc[u] = 0.0;
  const int64_t step = (int64_t)kFinishThreads * kFinishUnroll;
  for (int64_t i0 = threadIdx.x; i0 < n; i0 += step) {
#pragma unroll
    for (int u = 0; u < kFinishUnroll; ++u) {
      const int64_t i = i0 + (int64_t)u * kFinishThreads;
      if (i < n) {
        ps[u] += part_sum[i];
        pc[u] += part_count[i];
      }
    }
  }
  double s = 0.0, c = 0.0;
#pragma unroll
  for (int u = 0; u < kFinishUnroll; ++u) {
    s += ps[u];
    c += pc[u];
  }
  s = block_sum<kFinishThreads>(s, red);
  c = block_sum<kFinishThreads>(c, red);
  if (threadIdx.x == 0) {
    if (total) {
      total[0] = s;
      total[1] = c;
    } else {
      *out = (float)(s / c);  // all rows ignored: 0 / 0 = NaN, as torch
    }
  }
}

template <int NT, int VPT>
int64_t launch_rows(const float* logits, const int64_t* targets, int64_t rows, int64_t classes,
                    int64_t ignore_index, double* part_sum, double* part_count, cudaStream_t stream) {
  static int per_sm = 0;
  if (per_sm == 0) {
    int b = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, ce_row_kernel<NT, VPT>, NT, 0);
    per_sm = b > 0 ? b : 1;
  }
  const int64_t grid = std::min<int64_t>(rows, (int64_t)sm_count() * per_sm);
  ce_row_kernel<NT, VPT><<<(unsigned)grid, NT, 0, stream>>>(logits, targets, rows, classes, ignore_index,
                                                            part_sum, part_count);
  return grid;
}

// partial (sum, count) slots: one per CTA, at most one per row
size_t ce_ws_bytes(int64_t rows) { return 2 * (size_t)rows * sizeof(double); }

}  // namespace
}  // namespace kb

extern "C" {

size_t kb_cross_entropy_workspace_size(int64_t rows) { return rows > 0 ? kb::ce_ws_bytes(rows) : 0; }

static int cross_entropy_impl(const char* name, const float* logits, const int64_t* targets, float* out,
                              double* total, int64_t rows, int64_t classes, int64_t ignore_index,
                              void* workspace, size_t workspace_bytes, kbStream stream);

int kb_cross_entropy_f32(const float* logits, const int64_t* targets, float* out, int64_t rows,
                         int64_t classes, int64_t ignore_index, void* workspace, size_t workspace_bytes,
                         kbStream stream) {
  KB_REQUIRE(out, KB_ERR_INVALID_ARG, "kb_cross_entropy_f32: null output");
  return cross_entropy_impl("kb_cross_entropy_f32", logits, targets, out, nullptr, rows, classes,
                            ignore_index, workspace, workspace_bytes, stream);
}

int kb_cross_entropy_partial_f64(const float* logits, const int64_t* targets, double* total, int64_t rows,
                                 int64_t classes, int64_t ignore_index, void* workspace,
                                 size_t workspace_bytes, kbStream stream) {
  KB_REQUIRE(total, KB_ERR_INVALID_ARG, "kb_cross_entropy_partial_f64: null output");
  return cross_entropy_impl("kb_cross_entropy_partial_f64", logits, targets, nullptr, total, rows, classes,
                            ignore_index, workspace, workspace_bytes, stream);
}

int kb_cross_entropy_finalize_f32(const double* total, float* out, kbStream stream) {
  KB_REQUIRE(total && out, KB_ERR_INVALID_ARG, "kb_cross_entropy_finalize_f32: null pointer");
  kb::ce_finish_kernel<<<1, kb::kFinishThreads, 0, stream>>>(total, total + 1, 1, out, nullptr);
  return kb::check_launch("kb_cross_entropy_finalize_f32");
}

static int cross_entropy_impl(const char* name, const float* logits, const int64_t* targets, float* out,
                              double* total, int64_t rows, int64_t classes, int64_t ignore_index,
                              void* workspace, size_t workspace_bytes, kbStream stream) {
  KB_REQUIRE(rows >= 0 && classes >= 0, KB_ERR_INVALID_ARG, "%s: negative size", name);
  if (rows == 0) {  // mean over nothing: 0 / 0 = NaN (sharded form: sum 0, count 0)
    kb::ce_finish_kernel<<<1, kb::kFinishThreads, 0, stream>>>(nullptr, nullptr, 0, out, total);
    return kb::check_launch(name);
  }
  KB_REQUIRE(classes >= 1, KB_ERR_INVALID_ARG, "%s: no classes", name);
  KB_REQUIRE(logits && targets, KB_ERR_INVALID_ARG, "%s: null pointer", name);
  KB_REQUIRE(rows <= 0x7fffffff, KB_ERR_UNSUPPORTED, "%s: too many rows", name);
  const size_t need = kb::ce_ws_bytes(rows);
  KB_REQUIRE(workspace && workspace_bytes >= need, KB_ERR_WORKSPACE,
             "%s: workspace of %zu bytes needed, %zu given", name, need, workspace_bytes);
  KB_REQUIRE(kb::aligned16(workspace), KB_ERR_INVALID_ARG, "%s: workspace must be 16-byte aligned", name);
  double* part_sum = static_cast<double*>(workspace);
  double* part_count = part_sum + rows;
  const bool vec = classes % 4 == 0 && kb::aligned16(logits);
  int64_t parts;
  if (vec && classes <= 128 * 4 * 2)
    parts = kb::launch_rows<128, 2>(logits, targets, rows, classes, ignore_index, part_sum, part_count, stream);
  else if (vec && classes <= 128 * 4 * 8)  // 32 logits per thread: the block reductions amortise over more
    parts = kb::launch_rows<128, 8>(logits, targets, rows, classes, ignore_index, part_sum, part_count, stream);
  else if (vec && classes <= 512 * 4 * 8)
    parts = kb::launch_rows<512, 8>(logits, targets, rows, classes, ignore_index, part_sum, part_count, stream);
  else {
    kb::ce_online_kernel<256><<<(unsigned)rows, 256, 0, stream>>>(logits, targets, classes, ignore_index,
                                                                  part_sum, part_count);
    parts = rows;
  }
  if (int st = kb::check_launch(name)) return st;
  kb::ce_finish_kernel<<<1, kb::kFinishThreads, 0, stream>>>(part_sum, part_count, parts, out, total);
  return kb::check_launch(name);
}

}  // extern "C"
