// rownorm.cu — single-read row kernels: LayerNorm, RMSNorm, softmax and
// log-softmax over the last dimension, plus the channel-dim RMSNorm form.
//
// Design (B200): a row is read from HBM exactly once into registers
// (VPT float4 per thread, 128-bit loads), reduced on chip, and written once.
//   <= 1K floats   one warp per row, shuffle-only reductions;
//   <= 16K floats  one CTA per row, several CTAs per SM overlapping their
//                  load / reduce / store phases;
//   <= 128K floats a persistent kernel: one 1024-thread CTA per SM (or a
//                  2/4-CTA cluster per row beyond 32K floats, partial
//                  statistics exchanged through DSMEM) holds the current row
//                  in registers while the next row streams into shared
//                  memory through a cp.async.bulk copy, so HBM keeps busy
//                  during the reductions (a 128 KB softmax row is too large
//                  for several rows per SM to overlap otherwise).
// Other shapes (cols % 4 != 0, unaligned views, > 128K columns) take a
// generic multi-pass kernel.
//
// Two-pass statistics are done on the register copy: LayerNorm computes the
// mean, then sum((x - mean)^2) — never E[x^2] - mean^2 (the cancellation-prone
// form of candidates/40_LayerNorm/v1.py:44-46).
#include <cooperative_groups.h>

#include "kb_common.cuh"

namespace cg = cooperative_groups;

namespace kb {
namespace {

enum RowOp { kLayerNorm = 0, kRmsNorm = 1, kSoftmax = 2, kLogSoftmax = 3 };

constexpr float kLog2e = 1.4426950408889634f;  // log2(e)

struct RowArgs {
  const float* x;
  const float* gamma;
  const float* beta;
  float* y;
  int64_t rows;
  int cols;
  float eps;
};

// ---------------------------------------------------------------------------
// reducers: warp-only, block, and block + cluster (DSMEM)
// ---------------------------------------------------------------------------
// Partial softmax statistics: max m and sum of exp(x - m).  Two partials
// combine as (M, s1 e^(m1 - M) + s2 e^(m2 - M)), M = max(m1, m2); the
// combination is commutative, so butterfly shuffles leave every lane with
// the same bits.  A NaN element makes its sum NaN, which then propagates.
struct MaxSum {
  float m, s;
};
__device__ __forceinline__ float ms_rescale(float m, float M) {
  return m == M ? 1.0f : exp2f((m - M) * kLog2e);  // also covers m == M == -inf
}
__device__ __forceinline__ MaxSum ms_combine(MaxSum a, MaxSum b) {
  const float M = fmaxf(a.m, b.m);
  return {M, a.s * ms_rescale(a.m, M) + b.s * ms_rescale(b.m, M)};
}
// Warp combine in three steps: a max butterfly, one rescale of each lane's
// sum to the warp max, a sum butterfly.  One exponential per lane instead of
// two per butterfly round: with every warp of a CTA combining at once, the
// per-round exponentials kept the special-function pipe busy for hundreds
// of cycles per row.  Both butterflies leave every lane with the same bits.
__device__ __forceinline__ MaxSum warp_ms(MaxSum v) {
  const float M = warp_max(v.m);
  return {M, warp_sum(v.s * ms_rescale(v.m, M))};
}
// Block-wide combine; `red` holds >= 64 floats.
template <int NT>
__device__ __forceinline__ MaxSum block_ms(MaxSum v, float* red) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_ms(v);
  if (NW == 1) return v;
  if (lane == 0) {
    red[warp] = v.m;
    red[32 + warp] = v.s;
  }
  __syncthreads();
  MaxSum r = (lane < NW) ? MaxSum{red[lane], red[32 + lane]} : MaxSum{-INFINITY, 0.0f};
  r = warp_ms(r);
  __syncthreads();
  return r;
}

struct WarpReducer {
  __device__ __forceinline__ float sum(float v, int) const { return warp_sum(v); }
  __device__ __forceinline__ float max(float v, int) const { return warp_max(v); }
  __device__ __forceinline__ MaxSum maxsum(MaxSum v, int) const { return warp_ms(v); }
};

template <int NT, int CL>
struct ClusterReducer {
  float* red;    // >= 64 floats of shared memory
  float* slots;  // >= 4 floats of shared memory: reduction stages 0 and 1
  __device__ __forceinline__ float combine_sum(float part, int slot) const {
    if constexpr (CL == 1) {
      return part;
    } else {
      cg::cluster_group cluster = cg::this_cluster();
      if (threadIdx.x == 0) slots[slot] = part;
      cluster.sync();
      float tot = 0.0f;
#pragma unroll
      for (int r = 0; r < CL; ++r) tot += *cluster.map_shared_rank(slots + slot, r);
      return tot;
    }
  }
  __device__ __forceinline__ float combine_max(float part, int slot) const {
    if constexpr (CL == 1) {
      return part;
    } else {
      cg::cluster_group cluster = cg::this_cluster();
      if (threadIdx.x == 0) slots[slot] = part;
      cluster.sync();
      float m = -INFINITY;
#pragma unroll
      for (int r = 0; r < CL; ++r) m = fmaxf(m, *cluster.map_shared_rank(slots + slot, r));
      return m;
    }
  }
  __device__ __forceinline__ float sum(float v, int slot) const {
    return combine_sum(block_sum<NT>(v, red), slot);
  }
  __device__ __forceinline__ float max(float v, int slot) const {
    return combine_max(block_max<NT>(v, red), slot);
  }
  __device__ __forceinline__ MaxSum maxsum(MaxSum v, int slot) const {
    MaxSum part = block_ms<NT>(v, red);
    if constexpr (CL == 1) {
      return part;
    } else {
      cg::cluster_group cluster = cg::this_cluster();
      if (threadIdx.x == 0) {
        slots[2 * slot] = part.m;
        slots[2 * slot + 1] = part.s;
      }
      cluster.sync();
      MaxSum tot{-INFINITY, 0.0f};
#pragma unroll
      for (int r = 0; r < CL; ++r) {
        const float* rs = cluster.map_shared_rank(slots + 2 * slot, r);
        tot = ms_combine(tot, MaxSum{rs[0], rs[1]});
      }
      return tot;
    }
  }
};

// ---------------------------------------------------------------------------
// the per-row math on a register-resident segment
//   v[k] holds float4 number (k * stride + lane) of this thread's segment;
//   col4_base + k * stride + lane is its float4 index within the full row.
// ---------------------------------------------------------------------------
// Float4 slot of a thread's k-th vector within its row segment.  PAIRED
// puts vectors 2i and 2i+1 next to each other, so a thread's results leave
// as one 256-bit store (fewer store instructions in flight per byte);
// otherwise consecutive threads hold consecutive float4s.
template <bool PAIRED>
__device__ __forceinline__ int64_t vec_slot(int k, int lane, int stride) {
  return PAIRED ? (int64_t)(k >> 1) * 2 * stride + 2 * lane + (k & 1) : (int64_t)k * stride + lane;
}

// writes the VPT result vectors of one thread (ok[k]: inside the row)
template <int VPT, bool PAIRED>
__device__ __forceinline__ void store_row(float4* yrow, const float4 (&v)[VPT], const bool (&ok)[VPT],
                                          int lane, int stride) {
  if constexpr (PAIRED) {
    static_assert(VPT % 2 == 0, "paired vectors");
#pragma unroll
    for (int k = 0; k < VPT; k += 2) {
      float4* dst = yrow + vec_slot<true>(k, lane, stride);
      if (ok[k + 1]) {  // both halves inside the row (slot k+1 = slot k + 1)
        f32x8 w;
        w.v[0] = v[k].x; w.v[1] = v[k].y; w.v[2] = v[k].z; w.v[3] = v[k].w;
        w.v[4] = v[k + 1].x; w.v[5] = v[k + 1].y; w.v[6] = v[k + 1].z; w.v[7] = v[k + 1].w;
        st_stream8(reinterpret_cast<float*>(dst), w);
      } else if (ok[k]) {
        st_stream(dst, v[k]);
      }
    }
  } else {
#pragma unroll
    for (int k = 0; k < VPT; ++k)
      if (ok[k]) st_stream(yrow + vec_slot<false>(k, lane, stride), v[k]);
  }
}

// 2^x by the hardware's ex2.approx.ftz instruction (PTX ISA); results below
// 2^-126 become 0 instead of subnormal.  For the per-element softmax
// exponentials such terms are below fp32 resolution after the division by
// the row sum (or in the log of the sum); 1 % faster at 8192 x 32768 than
// exp2f, identical outputs on N(0, 4) rows.
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <RowOp OP, int VPT, bool PAIRED = false, bool EMIT = true, class R>
__device__ __forceinline__ void row_math(float4 (&v)[VPT], const bool (&ok)[VPT],
                                         const RowArgs& a, float4* yrow, int64_t col4_base,
                                         int stride, int lane, const R& red, bool store = true) {
  const float inv_cols = 1.0f / (float)a.cols;
  if constexpr (OP == kLayerNorm) {
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < VPT; ++k)
      if (ok[k]) s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
    const float mean = red.sum(s, 0) * inv_cols;
    float q = 0.0f;
#pragma unroll
    for (int k = 0; k < VPT; ++k)
      if (ok[k]) {
        float dx = v[k].x - mean, dy = v[k].y - mean, dz = v[k].z - mean, dw = v[k].w - mean;
        q += (dx * dx + dy * dy) + (dz * dz + dw * dw);
      }
    const float var = red.sum(q, 1) * inv_cols;
    const float rstd = 1.0f / sqrtf(var + a.eps);
    const float4* g4 = reinterpret_cast<const float4*>(a.gamma);
    const float4* b4 = reinterpret_cast<const float4*>(a.beta);
#pragma unroll
    for (int k = 0; k < VPT; ++k)
      if (ok[k] && store) {
        const int64_t c4 = col4_base + vec_slot<PAIRED>(k, lane, stride);
        float4 r;
        r.x = (v[k].x - mean) * rstd;
        r.y = (v[k].y - mean) * rstd;
        r.z = (v[k].z - mean) * rstd;
        r.w = (v[k].w - mean) * rstd;
        if (g4) {
          const float4 g = __ldg(g4 + c4);
          r.x *= g.x; r.y *= g.y; r.z *= g.z; r.w *= g.w;
        }
        if (b4) {
          const float4 b = __ldg(b4 + c4);
          r.x += b.x; r.y += b.y; r.z += b.z; r.w += b.w;
        }
        v[k] = r;
      }
  } else if constexpr (OP == kRmsNorm) {
    float q = 0.0f;
#pragma unroll
    for (int k = 0; k < VPT; ++k)
      if (ok[k]) q += (v[k].x * v[k].x + v[k].y * v[k].y) + (v[k].z * v[k].z + v[k].w * v[k].w);
    const float ms = red.sum(q, 0) * inv_cols;
    const float inv = 1.0f / sqrtf(ms + a.eps);
    const float4* g4 = reinterpret_cast<const float4*>(a.gamma);
#pragma unroll
    for (int k = 0; k < VPT; ++k)
      if (ok[k] && store) {
        const int64_t c4 = col4_base + vec_slot<PAIRED>(k, lane, stride);
        float4 r;
        r.x = v[k].x * inv;
        r.y = v[k].y * inv;
        r.z = v[k].z * inv;
        r.w = v[k].w * inv;
        if (g4) {
          const float4 g = __ldg(g4 + c4);
          r.x *= g.x; r.y *= g.y; r.z *= g.z; r.w *= g.w;
        }
        v[k] = r;
      }
  } else {
    // one pass: this thread's max and sum of exp(x - max), then a single
    // block (cluster) combine of the (max, sum) pairs
    float mt = -INFINITY;
#pragma unroll
    for (int k = 0; k < VPT; ++k)
      if (ok[k]) mt = fmaxf(mt, fmaxf(fmaxf(v[k].x, v[k].y), fmaxf(v[k].z, v[k].w)));
    // exp(x - mt) = 2^(x log2(e) - mt log2(e)): one FMA and exp2f per element
    const float mtl = (mt == -INFINITY) ? 0.0f : mt * kLog2e;
    float st = 0.0f;
    if constexpr (OP == kSoftmax) {
      // keep exp(x - mt) in registers: exp is evaluated once per element
#pragma unroll
      for (int k = 0; k < VPT; ++k)
        if (ok[k]) {
          v[k].x = ex2_ftz(fmaf(v[k].x, kLog2e, -mtl));
          v[k].y = ex2_ftz(fmaf(v[k].y, kLog2e, -mtl));
          v[k].z = ex2_ftz(fmaf(v[k].z, kLog2e, -mtl));
          v[k].w = ex2_ftz(fmaf(v[k].w, kLog2e, -mtl));
          st += (v[k].x + v[k].y) + (v[k].z + v[k].w);
        }
      const MaxSum tot = red.maxsum(MaxSum{mt, st}, 0);
      const float scale = ms_rescale(mt, tot.m) / tot.s;
#pragma unroll
      for (int k = 0; k < VPT; ++k)
        v[k] = make_float4(v[k].x * scale, v[k].y * scale, v[k].z * scale, v[k].w * scale);
    } else {
#pragma unroll
      for (int k = 0; k < VPT; ++k)
        if (ok[k])
          st += (ex2_ftz(fmaf(v[k].x, kLog2e, -mtl)) + ex2_ftz(fmaf(v[k].y, kLog2e, -mtl))) +
                (ex2_ftz(fmaf(v[k].z, kLog2e, -mtl)) + ex2_ftz(fmaf(v[k].w, kLog2e, -mtl)));
      const MaxSum tot = red.maxsum(MaxSum{mt, st}, 0);
      // (x - max) - log sum, in this order: x - (max + log sum) is 2 % faster
      // but rounds max + log sum at max's magnitude (|max| ~ 1e4 gave errors
      // of 1.7e-4 where this order stays exact to an ulp of the result)
      const float m = tot.m, lse = logf(tot.s);
#pragma unroll
      for (int k = 0; k < VPT; ++k)
        v[k] = make_float4((v[k].x - m) - lse, (v[k].y - m) - lse, (v[k].z - m) - lse, (v[k].w - m) - lse);
    }
  }
  if (EMIT && store) store_row<VPT, PAIRED>(yrow, v, ok, lane, stride);
}

// One CTA (or one CL-CTA cluster) per row; NT threads x VPT float4 each.
// 256-thread CTAs are held to 48 registers so that five fit on an SM (40
// warps, five 32 KB rows in flight) instead of four: outputs are unchanged,
// LayerNorm at 8192 columns runs 8 % faster in the power-capped bench step.
template <RowOp OP, int NT, int VPT, int CL>
__global__ void __launch_bounds__(NT, (NT == 256 ? 5 : 1)) row_block_kernel(RowArgs a) {
  __shared__ float red[64];
  __shared__ float slots[4];
  const int64_t row = blockIdx.x / CL;
  int rank = 0;
  if constexpr (CL > 1) rank = (int)cg::this_cluster().block_rank();
  const int seg4 = a.cols / 4 / CL;  // float4s owned by this CTA
  const int64_t col4_base = (int64_t)rank * seg4;
  const float4* xs = reinterpret_cast<const float4*>(a.x + row * (int64_t)a.cols) + col4_base;
  float4* ys = reinterpret_cast<float4*>(a.y + row * (int64_t)a.cols) + col4_base;
  float4 v[VPT];
  bool ok[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int i = k * NT + threadIdx.x;
    ok[k] = i < seg4;
    v[k] = ok[k] ? ld_stream(xs + i) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  ClusterReducer<NT, CL> r{red, slots};
  row_math<OP, VPT>(v, ok, a, ys, col4_base, NT, threadIdx.x, r);
  // Peers may still read `slots` through DSMEM: wait for the whole cluster
  // before this CTA's shared memory goes away.  Relaxed arrive — the row's
  // global stores need no cluster-scope release, and a releasing barrier
  // would stall on them.
  if constexpr (CL > 1)
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Persistent variant with a bulk-copy prefetch.  A cluster of CL CTAs walks
// rows cluster_id, cluster_id + nclusters, ...; CTA `rank` owns one
// contiguous segment of each row.  The segment of the next row is fetched
// into shared memory by cp.async.bulk (one 1-D bulk copy, completion counted
// on an mbarrier) as soon as the current row has been moved into registers,
// so HBM keeps streaming while the row is reduced, exchanged across the
// cluster and written back.
// Abort handling stays cluster-uniform: a CTA whose bounded wait expires
// raises the fault word, stops copying and storing, but keeps executing the
// per-row cluster barriers so its peers never wait on a CTA that left.
// ---------------------------------------------------------------------------
__device__ int g_row_fault = 0;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ bool mbar_try_wait_parity(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait_parity(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t n = 1;; ++n) {
    if (mbar_try_wait_parity(bar, parity)) return true;
    if ((n & 63) == 0 && global_ns() - t0 > 2000000000ull) return false;
  }
}
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// Moves this thread's vectors k0 .. k1-1 (k0, k1 even) of a row segment from
// shared memory into registers; ok[k] tells whether vector k lies inside the
// segment.  With PAIRED slots, lane l owns float4s 2l and 2l+1 of each pair
// group, so reading "the even float4 of every lane" is a 32-byte-strided
// access: each quarter-warp of a 128-bit shared load touches only 16 of the
// 32 banks twice and needs two wavefronts.  Lanes with bit 2 set therefore
// read the odd float4 of their pair first: every quarter-warp then covers all
// 32 banks once per load, and the pair is put back in order in registers, so
// the values (and every result computed from them) are unchanged.
template <bool PAIRED, int VPT>
__device__ __forceinline__ void read_segment(float4 (&v)[VPT], bool (&ok)[VPT], const float4* buf, int k0,
                                             int k1, int lane, int stride, int seg4, bool live) {
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  if constexpr (PAIRED) {
    const int sw = (lane >> 2) & 1;
#pragma unroll
    for (int k = 0; k < VPT; k += 2) {
      if (k < k0 || k >= k1) continue;
      const int64_t j0 = vec_slot<true>(k, lane, stride);  // even float4 of the pair
      const int64_t ja = j0 + sw, jb = j0 + (sw ^ 1);
      const float4 fa = (live && ja < seg4) ? buf[ja] : zero;
      const float4 fb = (live && jb < seg4) ? buf[jb] : zero;
      v[k] = sw ? fb : fa;
      v[k + 1] = sw ? fa : fb;
      ok[k] = j0 < seg4;
      ok[k + 1] = j0 + 1 < seg4;
    }
  } else {
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      if (k < k0 || k >= k1) continue;
      const int64_t j = vec_slot<false>(k, lane, stride);
      ok[k] = j < seg4;
      v[k] = (live && ok[k]) ? buf[j] : zero;
    }
  }
}

template <RowOp OP, int NT, int VPT, int CL, int DEPTH, bool PAIRED>
__global__ void __launch_bounds__(NT) row_persist_kernel(RowArgs a) {
  extern __shared__ float4 seg_buf[];  // DEPTH segment buffers
  __shared__ float red[64];
  __shared__ float slots[8];  // two sets, alternating by row
  __shared__ __align__(8) uint64_t bars[DEPTH];
  int rank = 0;
  if constexpr (CL > 1) rank = (int)cg::this_cluster().block_rank();
  const int64_t cluster_id = blockIdx.x / CL, nclusters = gridDim.x / CL;
  const int seg4 = a.cols / 4 / CL;
  const uint32_t seg_bytes = (uint32_t)seg4 * 16u;
  const int64_t col4_base = (int64_t)rank * seg4;
  const float* xseg = a.x + col4_base * 4;
  if (threadIdx.x == 0) {
    for (int d = 0; d < DEPTH; ++d)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&bars[d])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if constexpr (CL > 1) cg::this_cluster().sync();  // peers' shared memory exists from here on
  // prologue: the first DEPTH rows of this cluster in flight
  if (threadIdx.x == 0)
    for (int d = 0; d < DEPTH; ++d) {
      const int64_t rr = cluster_id + (int64_t)d * nclusters;
      if (rr < a.rows)
        bulk_load(smem_addr(seg_buf + (size_t)d * seg4), xseg + rr * (int64_t)a.cols, seg_bytes,
                  smem_addr(&bars[d]));
    }
  bool alive = true;
  ClusterReducer<NT, CL> r{red, slots};
  int64_t i = 0;
  for (int64_t row = cluster_id; row < a.rows; row += nclusters, ++i) {
    // alternate slot sets: a peer may still read this CTA's set of the
    // previous row until it reaches this row's cluster barrier
    r.slots = slots + 4 * (int)(i & 1);
    const int slot = (int)(i % DEPTH);
    const uint32_t parity = (uint32_t)((i / DEPTH) & 1);
    const float4* buf = seg_buf + (size_t)slot * seg4;
    bool got = alive ? wait_bounded(smem_addr(&bars[slot]), parity) : true;
    float4 v[VPT];
    bool ok[VPT];
    read_segment<PAIRED>(v, ok, buf, 0, VPT, threadIdx.x, NT, seg4, alive && got);
    // everyone has read the buffer (and agrees whether the copy landed)
    got = __syncthreads_and(got) != 0;
    if (!got && alive) {
      alive = false;
      if (threadIdx.x == 0) atomicExch(&g_row_fault, 1);
    }
    const int64_t next = row + (int64_t)DEPTH * nclusters;
    if (threadIdx.x == 0 && alive && next < a.rows)
      bulk_load(smem_addr(buf), xseg + next * (int64_t)a.cols, seg_bytes, smem_addr(&bars[slot]));
    float4* ys = reinterpret_cast<float4*>(a.y + row * (int64_t)a.cols) + col4_base;
    row_math<OP, VPT, PAIRED>(v, ok, a, ys, col4_base, NT, threadIdx.x, r, alive);
  }
  if constexpr (CL > 1)
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
}

// Row results through shared memory and bulk (TMA) stores: pair group c of
// the paired layout (float4 slots c*2*NT .. c*2*NT + 2*NT - 1 of the segment,
// 32 KB for NT = 1024) is written into one of two staging buffers and leaves
// as one cp.async.bulk store issued by thread 0.  The registers are free as
// soon as the shared-memory writes are done, and the stores no longer queue
// in the SM's load/store unit behind the next row's read-out.  Thread 0 owns
// every bulk group, so its wait_group.read 1 before a buffer is reused (the
// store two groups back read that buffer) covers them all.  Lanes with bit 2
// set write the odd float4 of their pair first (no bank conflicts).
__device__ __forceinline__ void bulk_store_wait_read1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
__device__ __forceinline__ void bulk_store_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
template <int NT, int VPT>
__device__ __forceinline__ void staged_store_row(float4* ys, const float4 (&v)[VPT], int seg4, float4* stage,
                                                 bool live) {
  const int lane = threadIdx.x;
  const int sw = (lane >> 2) & 1;
#pragma unroll
  for (int c = 0; c < VPT / 2; ++c) {
    const int g0 = c * 2 * NT;
    if (g0 >= seg4) break;  // uniform over the CTA
    float4* buf = stage + (c & 1) * 2 * NT;
    if (threadIdx.x == 0) bulk_store_wait_read1();
    __syncthreads();
    if (live) {
      buf[2 * lane + sw] = sw ? v[2 * c + 1] : v[2 * c];
      buf[2 * lane + (sw ^ 1)] = sw ? v[2 * c] : v[2 * c + 1];
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    __syncthreads();
    if (threadIdx.x == 0 && live) {
      const uint32_t bytes = (uint32_t)min(2 * NT, seg4 - g0) * 16u;
      asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(ys + g0),
                   "r"(smem_addr(buf)), "r"(bytes)
                   : "memory");
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
  }
}

// The same persistent walk with the prefetch in two halves.  With one
// buffer for the whole row segment, the next row's copy can start only after
// every thread has moved the whole current row into registers, so each SM's
// read stream pauses for that copy-out and barrier once per row — a pause
// measured in SM cycles, which made these kernels slow down with the SM
// clock under the power cap.  Here the segment buffer is two halves with a
// barrier each: as soon as the first half has been read out, the next row's
// first half is already being fetched while the second half is read out.
// Each thread's first VPT/2 vectors lie in the first half (vec_slot), so the
// register layout and the math are unchanged.
template <RowOp OP, int NT, int VPT, int CL, bool PAIRED, bool TST>
__global__ void __launch_bounds__(NT) row_persist_halves_kernel(RowArgs a) {
  // one row segment: [first half | second half], then with TST two 2*NT-float4
  // staging buffers for the bulk result stores
  extern __shared__ float4 seg_buf[];
  static_assert(!TST || (PAIRED && CL == 1), "staged stores: paired layout, one CTA per row");
  __shared__ float red[64];
  __shared__ float slots[8];  // two sets, alternating by row
  __shared__ __align__(8) uint64_t bars[2];
  constexpr int H = VPT / 2;
  static_assert(!PAIRED || H % 2 == 0, "pairs must not straddle the two halves");
  int rank = 0;
  if constexpr (CL > 1) rank = (int)cg::this_cluster().block_rank();
  const int64_t cluster_id = blockIdx.x / CL, nclusters = gridDim.x / CL;
  const int seg4 = a.cols / 4 / CL;
  const int half4 = min(seg4, H * NT);  // float4s in the first half
  const int rest4 = seg4 - half4;       // in the second (0: one half only)
  const int64_t col4_base = (int64_t)rank * seg4;
  const float* xseg = a.x + col4_base * 4;
  if (threadIdx.x == 0) {
    for (int d = 0; d < 2; ++d)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&bars[d])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if constexpr (CL > 1) cg::this_cluster().sync();  // peers' shared memory exists from here on
  if (threadIdx.x == 0 && cluster_id < a.rows) {
    const float* src = xseg + cluster_id * (int64_t)a.cols;
    bulk_load(smem_addr(seg_buf), src, (uint32_t)half4 * 16u, smem_addr(&bars[0]));
    if (rest4 > 0) bulk_load(smem_addr(seg_buf + half4), src + (int64_t)half4 * 4, (uint32_t)rest4 * 16u,
                             smem_addr(&bars[1]));
  }
  bool alive = true;
  ClusterReducer<NT, CL> r{red, slots};
  int64_t i = 0;
  for (int64_t row = cluster_id; row < a.rows; row += nclusters, ++i) {
    // alternate slot sets: a peer may still read this CTA's set of the
    // previous row until it reaches this row's cluster barrier
    r.slots = slots + 4 * (int)(i & 1);
    const uint32_t parity = (uint32_t)(i & 1);
    const int64_t next = row + nclusters;
    const float* nsrc = xseg + next * (int64_t)a.cols;
    float4 v[VPT];
    bool ok[VPT];
    // first half: read out, then refill it with the next row's first half
    bool got = alive ? wait_bounded(smem_addr(&bars[0]), parity) : true;
    read_segment<PAIRED>(v, ok, seg_buf, 0, H, threadIdx.x, NT, seg4, alive && got);
    bool all = __syncthreads_and(got) != 0;
    if (threadIdx.x == 0 && alive && all && next < a.rows)
      bulk_load(smem_addr(seg_buf), nsrc, (uint32_t)half4 * 16u, smem_addr(&bars[0]));
    // second half
    got = (alive && all && rest4 > 0) ? wait_bounded(smem_addr(&bars[1]), parity) : true;
    read_segment<PAIRED>(v, ok, seg_buf, H, VPT, threadIdx.x, NT, seg4, alive && all && got);
    all = (__syncthreads_and(got) != 0) && all;
    if (threadIdx.x == 0 && alive && all && rest4 > 0 && next < a.rows)
      bulk_load(smem_addr(seg_buf + half4), nsrc + (int64_t)half4 * 4, (uint32_t)rest4 * 16u,
                smem_addr(&bars[1]));
    if (!all && alive) {
      alive = false;
      if (threadIdx.x == 0) atomicExch(&g_row_fault, 1);
    }
    float4* ys = reinterpret_cast<float4*>(a.y + row * (int64_t)a.cols) + col4_base;
    row_math<OP, VPT, PAIRED, !TST>(v, ok, a, ys, col4_base, NT, threadIdx.x, r, alive);
    if constexpr (TST) staged_store_row<NT, VPT>(ys, v, seg4, seg_buf + seg4, alive);
  }
  if constexpr (TST) {
    if (threadIdx.x == 0) bulk_store_wait_all();  // stores done before the CTA's shared memory goes
  }
  if constexpr (CL > 1)
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
}

template <RowOp OP, int NT, int VPT, int CL, bool PAIRED, bool TST>
cudaError_t launch_halves_impl(const RowArgs& a, cudaStream_t s) {
  auto kern = row_persist_halves_kernel<OP, NT, VPT, CL, PAIRED, TST>;
  const int smem = a.cols / CL * 4 + (TST ? 2 * 2 * NT * 16 : 0);
  static uint64_t attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !(attr_set >> dev & 1)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    attr_set |= 1ull << dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int nclusters = 0;
  cfg.gridDim = dim3(CL * 148);
  cudaError_t e = cudaOccupancyMaxActiveClusters(&nclusters, kern, &cfg);
  if (e != cudaSuccess || nclusters <= 0) nclusters = sm_count() / CL;
  nclusters = (int)std::max<int64_t>(1, std::min<int64_t>(nclusters, a.rows));
  cfg.gridDim = dim3((unsigned)(nclusters * CL));
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <RowOp OP, int NT, int VPT, int CL, bool TST = false>
cudaError_t launch_halves(const RowArgs& a, cudaStream_t s) {
  if (aligned32(a.x) && aligned32(a.y) && a.cols % (8 * CL) == 0)
    return launch_halves_impl<OP, NT, VPT, CL, true, TST>(a, s);
  return launch_halves_impl<OP, NT, VPT, CL, false, false>(a, s);
}

template <RowOp OP, int NT, int VPT, int CL, int DEPTH, bool PAIRED>
cudaError_t launch_persist_impl(const RowArgs& a, cudaStream_t s) {
  auto kern = row_persist_kernel<OP, NT, VPT, CL, DEPTH, PAIRED>;
  const int smem = a.cols / CL * 4 * DEPTH;
  static uint64_t attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !(attr_set >> dev & 1)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    attr_set |= 1ull << dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // resident clusters on the whole GPU, times CL CTAs each
  int nclusters = 0;
  cfg.gridDim = dim3(CL * 148);
  cudaError_t e = cudaOccupancyMaxActiveClusters(&nclusters, kern, &cfg);
  if (e != cudaSuccess || nclusters <= 0) nclusters = sm_count() / CL;
  nclusters = (int)std::max<int64_t>(1, std::min<int64_t>(nclusters, a.rows));
  cfg.gridDim = dim3((unsigned)(nclusters * CL));
  return cudaLaunchKernelEx(&cfg, kern, a);
}

// 256-bit result stores when every row segment starts on 32 bytes
template <RowOp OP, int NT, int VPT, int CL, int DEPTH>
cudaError_t launch_persist(const RowArgs& a, cudaStream_t s) {
  if (aligned32(a.x) && aligned32(a.y) && a.cols % (8 * CL) == 0)
    return launch_persist_impl<OP, NT, VPT, CL, DEPTH, true>(a, s);
  return launch_persist_impl<OP, NT, VPT, CL, DEPTH, false>(a, s);
}

// One warp per row (rows of at most 32 * VPT * 4 floats); 4 warps per CTA.
template <RowOp OP, int VPT>
__global__ void __launch_bounds__(128) row_warp_kernel(RowArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  if (row >= a.rows) return;
  const int n4 = a.cols / 4;
  const float4* xs = reinterpret_cast<const float4*>(a.x + row * (int64_t)a.cols);
  float4* ys = reinterpret_cast<float4*>(a.y + row * (int64_t)a.cols);
  float4 v[VPT];
  bool ok[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int i = k * 32 + lane;
    ok[k] = i < n4;
    v[k] = ok[k] ? ld_stream(xs + i) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  row_math<OP, VPT>(v, ok, a, ys, 0, 32, lane, WarpReducer{});
}

// Generic fallback: any cols, any alignment.  One 512-thread CTA per row,
// the row is streamed from global memory once per pass (2-3 passes; later
// passes mostly hit L2).
template <RowOp OP>
__global__ void __launch_bounds__(512) row_generic_kernel(RowArgs a) {
  constexpr int NT = 512;
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const float* xr = a.x + row * (int64_t)a.cols;
  float* yr = a.y + row * (int64_t)a.cols;
  const int n = a.cols;
  const float inv_cols = 1.0f / (float)n;
  if constexpr (OP == kLayerNorm) {
    float s = 0.f;
    for (int i = threadIdx.x; i < n; i += NT) s += xr[i];
    const float mean = block_sum<NT>(s, red) * inv_cols;
    float q = 0.f;
    for (int i = threadIdx.x; i < n; i += NT) {
      float d = xr[i] - mean;
      q += d * d;
    }
    const float rstd = 1.0f / sqrtf(block_sum<NT>(q, red) * inv_cols + a.eps);
    for (int i = threadIdx.x; i < n; i += NT) {
      float r = (xr[i] - mean) * rstd;
      if (a.gamma) r *= a.gamma[i];
      if (a.beta) r += a.beta[i];
      yr[i] = r;
    }
  } else if constexpr (OP == kRmsNorm) {
    float q = 0.f;
    for (int i = threadIdx.x; i < n; i += NT) q += xr[i] * xr[i];
    const float inv = 1.0f / sqrtf(block_sum<NT>(q, red) * inv_cols + a.eps);
    for (int i = threadIdx.x; i < n; i += NT) {
      float r = xr[i] * inv;
      if (a.gamma) r *= a.gamma[i];
      yr[i] = r;
    }
  } else {
    float m = -INFINITY;
    for (int i = threadIdx.x; i < n; i += NT) m = fmaxf(m, xr[i]);
    m = block_max<NT>(m, red);
    float s = 0.f;
    for (int i = threadIdx.x; i < n; i += NT) s += expf(xr[i] - m);
    s = block_sum<NT>(s, red);
    if constexpr (OP == kSoftmax) {
      const float inv = 1.0f / s;
      for (int i = threadIdx.x; i < n; i += NT) yr[i] = expf(xr[i] - m) * inv;
    } else {
      const float lse = logf(s);
      for (int i = threadIdx.x; i < n; i += NT) yr[i] = (xr[i] - m) - lse;
    }
  }
}

template <RowOp OP, int NT, int VPT, int CL>
cudaError_t launch_block(const RowArgs& a, cudaStream_t s) {
  auto kern = row_block_kernel<OP, NT, VPT, CL>;
  if constexpr (CL == 1) {
    kern<<<(unsigned)a.rows, NT, 0, s>>>(a);
    return cudaGetLastError();
  } else {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(a.rows * CL));
    cfg.blockDim = dim3(NT);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CL;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a);
  }
}

template <RowOp OP>
int launch_rows(const char* name, const RowArgs& a, cudaStream_t s) {
  KB_REQUIRE(a.rows >= 0 && a.cols >= 0, KB_ERR_INVALID_ARG, "%s: negative size", name);
  if (a.rows == 0 || a.cols == 0) return KB_OK;
  KB_REQUIRE(a.x && a.y, KB_ERR_INVALID_ARG, "%s: null pointer", name);
  KB_REQUIRE(a.rows <= 0x7fffffffLL / 8, KB_ERR_UNSUPPORTED, "%s: too many rows", name);
  const bool vec = (a.cols % 4 == 0) && aligned16(a.x) && aligned16(a.y) &&
                   (!a.gamma || aligned16(a.gamma)) && (!a.beta || aligned16(a.beta));
  const int c = a.cols;
  cudaError_t e = cudaSuccess;
  if (!vec || c > 131072) {
    row_generic_kernel<OP><<<(unsigned)a.rows, 512, 0, s>>>(a);
    e = cudaGetLastError();
  } else if (c <= 1024) {
    const unsigned grid = (unsigned)ceil_div(a.rows, 4);
    if (c <= 128) row_warp_kernel<OP, 1><<<grid, 128, 0, s>>>(a);
    else if (c <= 256) row_warp_kernel<OP, 2><<<grid, 128, 0, s>>>(a);
    else if (c <= 512) row_warp_kernel<OP, 4><<<grid, 128, 0, s>>>(a);
    else row_warp_kernel<OP, 8><<<grid, 128, 0, s>>>(a);
    e = cudaGetLastError();
  } else if (c <= 2048) {
    e = launch_block<OP, 128, 4, 1>(a, s);
  } else if (c <= 4096) {
    e = launch_block<OP, 256, 4, 1>(a, s);
  } else if (c <= 8192) {
    e = launch_block<OP, 256, 8, 1>(a, s);
  } else if (c <= 16384) {
    e = launch_block<OP, 512, 8, 1>(a, s);
  } else if (c <= 32768) {
    // one persistent 1024-thread CTA per SM: the row in registers, the next
    // row streaming into shared memory in two halves, results leaving through
    // shared memory as bulk stores
    e = launch_halves<OP, 1024, 8, 1, true>(a, s);
  } else if (c <= 65536 && c % 8 == 0) {
    e = launch_persist<OP, 1024, 8, 2, 1>(a, s);
  } else if (c % 16 == 0) {
    e = launch_persist<OP, 1024, 8, 4, 1>(a, s);
  } else {
    row_generic_kernel<OP><<<(unsigned)a.rows, 512, 0, s>>>(a);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return set_error(KB_ERR_CUDA, "%s launch: %s", name, cudaGetErrorString(e));
  return KB_OK;
}

// ---------------------------------------------------------------------------
// RMSNorm over dim 1 of [outer, F, inner] (inner > 1): thread per (outer,
// inner) position, coalesced across inner; features walked twice (the second
// walk re-reads the CTA's 64-feature x 256-position window from L2).
// Follows the fixed addressing of candidates/36_RMSNorm_/v3.py:17-19.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
rms_channel_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                   float* __restrict__ y, int64_t outer, int64_t F, int64_t inner, float eps) {
  const int64_t p = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (p >= outer * inner) return;
  const int64_t o = p / inner, i = p - o * inner;
  const float* xp = x + o * F * inner + i;
  float* yp = y + o * F * inner + i;
  float q = 0.f;
  for (int64_t f = 0; f < F; ++f) {
    const float v = xp[f * inner];
    q += v * v;
  }
  const float inv = 1.0f / sqrtf(q / (float)F + eps);
  for (int64_t f = 0; f < F; ++f) {
    float r = xp[f * inner] * inv;
    if (gamma) r *= gamma[f];
    yp[f * inner] = r;
  }
}

}  // namespace
}  // namespace kb

extern "C" {

int kb_layernorm_f32(const float* x, const float* gamma, const float* beta, float* y,
                     int64_t rows, int64_t cols, float eps, kbStream stream) {
  KB_REQUIRE(cols <= 0x7fffffff, KB_ERR_UNSUPPORTED, "kb_layernorm_f32: cols too large");
  kb::RowArgs a{x, gamma, beta, y, rows, (int)cols, eps};
  return kb::launch_rows<kb::kLayerNorm>("kb_layernorm_f32", a, stream);
}

int kb_rmsnorm_f32(const float* x, const float* gamma, float* y, int64_t outer,
                   int64_t features, int64_t inner, float eps, kbStream stream) {
  KB_REQUIRE(outer >= 0 && features >= 0 && inner >= 1, KB_ERR_INVALID_ARG,
             "kb_rmsnorm_f32: bad shape");
  if (outer == 0 || features == 0) return KB_OK;
  if (inner == 1) {
    KB_REQUIRE(features <= 0x7fffffff, KB_ERR_UNSUPPORTED, "kb_rmsnorm_f32: features too large");
    kb::RowArgs a{x, gamma, nullptr, y, outer, (int)features, eps};
    return kb::launch_rows<kb::kRmsNorm>("kb_rmsnorm_f32", a, stream);
  }
  KB_REQUIRE(x && y, KB_ERR_INVALID_ARG, "kb_rmsnorm_f32: null pointer");
  const int64_t pos = outer * inner;
  kb::rms_channel_kernel<<<(unsigned)kb::ceil_div(pos, 256), 256, 0, stream>>>(
      x, gamma, y, outer, features, inner, eps);
  return kb::check_launch("kb_rmsnorm_f32");
}

int kb_softmax_f32(const float* x, float* y, int64_t rows, int64_t cols, kbStream stream) {
  KB_REQUIRE(cols <= 0x7fffffff, KB_ERR_UNSUPPORTED, "kb_softmax_f32: cols too large");
  kb::RowArgs a{x, nullptr, nullptr, y, rows, (int)cols, 0.f};
  return kb::launch_rows<kb::kSoftmax>("kb_softmax_f32", a, stream);
}

int kb_logsoftmax_f32(const float* x, float* y, int64_t rows, int64_t cols, kbStream stream) {
  KB_REQUIRE(cols <= 0x7fffffff, KB_ERR_UNSUPPORTED, "kb_logsoftmax_f32: cols too large");
  kb::RowArgs a{x, nullptr, nullptr, y, rows, (int)cols, 0.f};
  return kb::launch_rows<kb::kLogSoftmax>("kb_logsoftmax_f32", a, stream);
}

}  // extern "C"
