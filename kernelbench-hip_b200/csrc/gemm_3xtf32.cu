// gemm_3xtf32.cu — fp32 GEMM on the 5th-generation tensor cores (tcgen05)
// with the 3xTF32 split, for square, batched and split-K shapes.
//
// fp32 accuracy from TF32 tensor cores.  Every operand element x is split as
// hi = x with its low 13 mantissa bits cleared (TF32 keeps 10 explicit bits)
// and lo = x - hi (exact in fp32, same sign as x), and
//     C = sum over K of  A_lo * B_hi + A_hi * B_lo + A_hi * B_hi
// (A_lo * B_lo is below fp32 resolution).  The tensor core itself truncates
// an fp32 operand to TF32, i.e. reads x as hi (verified bitwise on the B200),
// so the raw tiles serve as the hi operands and only the lo tiles are
// written.  An infinite operand meets b_hi and b_lo of one sign and yields
// +-inf as plain fp32 does; non-finite x gets lo = 0.
//
// The tensor core's fp32 accumulation is not round-to-nearest: its error
// grows with the number of MMAs chained into one accumulator.  So K is cut
// into chunks of kChunkK; each chunk is accumulated in one of two TMEM
// buffers (ping-pong), and eight promotion warps add every finished chunk
// into fp32 register totals with ordinary round-to-nearest adds.  The
// error then scales with the magnitude of one chunk, not of the whole sum,
// and stays at the level of an fp32 CUDA-core GEMM.
//
// Persistent CTAs, one per SM, walk the 128 x BN output tiles in order
// (tile id = blockIdx.x, + gridDim.x, ...).  Every role keeps running
// counters across tiles, so the stage ring and the two TMEM chunk buffers
// simply continue: while the promotion warps store tile t, the MMA warp is
// already accumulating tile t + 1 into the other buffer.
// CTA = 512 threads in 4 warpgroups:
//   warp 0       TMA producer: cp.async.bulk.tensor loads of the A tile
//                (128 x 16, K-major, 64B swizzle) and B tile (16 x BN,
//                N-major, 32-column boxes, 128B swizzle with 32-byte atoms)
//                into a 4-stage ring; mbarrier transaction counts.
//   warp 1       allocates TMEM (2 x BN columns) and one lane issues
//                6 tcgen05.mma.kind::tf32 per stage (2 K-steps x 3 products);
//                tcgen05.commit frees the stage and publishes finished chunks.
//   warps 2-7    lo converters: write A_lo, B_lo for each landed stage
//                (element-wise, so the swizzled layout carries over), fence
//                generic -> async proxy, arrive on conv[s].
//   warps 8-15   promotion + epilogue: tcgen05.ld each finished chunk, add
//                into 128-lane x BN fp32 register totals (each warp owns one
//                TMEM lane quarter and half the columns); at the end of a
//                tile each warp stages its 32-row x 32-column boxes in its
//                own 4 KB buffer (128B swizzle) and stores them with TMA
//                tensor stores (direct stores when C's strides do not allow
//                a tensor map).
// setmaxnreg moves registers from warpgroups 0-1 (64 each) to the promotion
// warpgroups (192 each); the sum equals the 512 x 128 the CTA launches with.
// Every mbarrier wait is bounded (%globaltimer); on expiry the CTA raises a
// shared abort flag and a device fault word, all roles leave their loops,
// outstanding TMA loads are drained (bounded) and TMEM is freed.
//
// Small K (at most kResKB 16-deep K blocks, e.g. [32768, 64] x [64, 32768]):
// a tile is only a few K blocks deep, so reloading and re-splitting the B
// tile for every output tile dominates.  The B-resident form (RES) keeps one
// tile column's whole B panel, raw and lo, in shared memory (128 KB) and
// streams only A through the ring.  Every tile column is cut into runs of
// p.run m-tiles; run r (segment-major: all columns' first segments, then
// the second ones, ...) goes to CTA r mod gridDim.x, which walks its runs in
// order.  So a CTA stays on one panel for a whole run, and the CTAs working
// at the same time hold horizontally adjacent tiles of one row band, as in
// the streaming form (an order that scattered concurrent tiles over C wrote
// 5-10 % slower).  At each run start the producer waits until the MMAs of
// the previous run are done (panel_empty, a tcgen05.commit), loads the new
// panel, the converters split it (panel_full -> panel_conv) and the MMA warp
// waits for panel_conv.  A run in a column's last segment ends at the last
// m-tile.  MMA order, chunking and the epilogue are those of the streaming
// form, so results are bitwise identical.
//
// Shapes the TMA path cannot describe (row strides not multiples of 16 bytes,
// unaligned bases) take a CUDA-core fp32 kernel.
#include <cuda.h>
#include <string.h>

#include "kb_common.cuh"

namespace kb {

__device__ int g_gemm_fault = 0;  // nonzero after a CTA gave up waiting

namespace gemm {

constexpr int BM = 128;
constexpr int BK = 16;                 // fp32 K per stage: one 64-byte K-major row
constexpr int kStages = 4;
constexpr int kChunkK = 128;           // K elements per TMEM accumulation chunk
constexpr int kChunkBlocks = kChunkK / BK;
constexpr int kThreads = 512;
constexpr int kConvWarp0 = 2, kConvWarps = 6;
constexpr int kConvThreads = kConvWarps * 32;
constexpr int kPromoWarp0 = 8, kPromoWarps = 8;
constexpr int kPromoThreads = kPromoWarps * 32;
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr int kBoxRows = 32, kBoxCols = 32;      // C store box: 32 rows x 128 B
constexpr int kBoxBytes = kBoxRows * kBoxCols * 4;

constexpr int kResKB = 4;  // B-resident form: K blocks the shared-memory B panel holds

template <int BN, bool RES = false>
struct Cfg {
  static constexpr int A_BYTES = BM * BK * 4;                  // 8 KB
  static constexpr int B_BYTES = BN * BK * 4;                  // 16 KB (BN 256)
  // ring stage: raw + lo of A and B (streaming form) or of A only (B resident)
  static constexpr int STAGE_BYTES = RES ? 2 * A_BYTES : 2 * (A_BYTES + B_BYTES);
  static constexpr int PANEL_BYTES = RES ? kResKB * 2 * B_BYTES : 0;  // [kb][raw | lo]
  static constexpr int STAGING_BYTES = kPromoWarps * kBoxBytes;  // one C box per promotion warp
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM_BYTES =
      kStages * STAGE_BYTES + PANEL_BYTES + STAGING_BYTES + BAR_BYTES + 1024;  // + alignment slack
  static constexpr int TMEM_COLS = 2 * BN;                     // two chunk accumulators
  static constexpr int COLS_PER_WARP = BN / 2;                 // promotion warps split columns
};
static_assert(Cfg<256, true>::SMEM_BYTES <= 232448, "B-resident form exceeds shared memory");
static_assert(Cfg<256, false>::SMEM_BYTES <= 232448, "streaming form exceeds shared memory");

// ------------------------------------------------------------------ PTX wrappers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
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
// Bounded wait: false once the CTA (or any CTA of the launch) has aborted, or
// after kWaitLimitNs without progress.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t n = 1;; ++n) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((n & 63) == 0) {
      if (*abort_flag || *(volatile int*)&g_gemm_fault) {
        *abort_flag = 1;
        return false;
      }
      if (globaltimer() - t0 > kWaitLimitNs) {
        *abort_flag = 1;
        atomicExch(&g_gemm_fault, 1);
        return false;
      }
    }
  }
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* tm, uint32_t bar, int c0,
                                            int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* tm, uint32_t src, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(tm)),
      "r"(src), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// UMMA shared-memory descriptors (version 1).  TF32 operands come in two
// canonical layouts, matching how TMA writes them:
//   K-major  (A as stored [M, K]): 64-byte swizzle (layout type 4); 64-byte
//            rows, 8-row groups 512 B apart (SBO), LBO unused.  The second
//            K step of 8 tf32 starts 32 B into each row.
//   MN-major (B [K, N], and A stored [K, M]): TF32 accepts only the 128-byte
//            swizzle with 32-byte atoms (layout type 1): 128-byte rows in
//            4-row groups 512 B apart (SBO), 32-element column blocks 2048 B
//            apart (LBO, one 16-row TMA box each).  A K step of 8 rows
//            advances the start by 1024 B.
constexpr uint32_t kLayoutSw64 = 4;
constexpr uint32_t kLayoutSw128Atom32 = 1;
__device__ __forceinline__ uint64_t make_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for tcgen05
  d |= (uint64_t)layout << 61;
  return d;
}
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t saddr) {
  return make_desc(saddr, 16, 512, kLayoutSw64);
}
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t saddr) {
  return make_desc(saddr, 2048, 512, kLayoutSw128Atom32);
}

// Instruction descriptor: D f32, A/B tf32, A K-major or MN-major, B MN-major.
__host__ __device__ constexpr uint32_t make_idesc(int M, int N, bool a_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((a_mn ? 1u : 0u) << 15) | (1u << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ float lo_part(float x) {
  const float l = x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
  return isfinite(l) ? l : 0.0f;
}

// lo[i] = x[i] - tf32_trunc(x[i]) for the float4s t, t + stride, ...
__device__ __forceinline__ void lo_buffer(const float4* __restrict__ src, float4* __restrict__ dst, int n4,
                                          int t) {
#pragma unroll 4
  for (int i = t; i < n4; i += kConvThreads) {
    const float4 v = src[i];
    dst[i] = make_float4(lo_part(v.x), lo_part(v.y), lo_part(v.z), lo_part(v.w));
  }
}

__device__ __forceinline__ void setmaxnreg_dec64() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 64;" ::: "memory");
}
__device__ __forceinline__ void setmaxnreg_inc192() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 192;" ::: "memory");
}

struct Params {
  float* C;          // output (mode 0) or partial tiles [Z][M][N] (mode 1)
  int M, N, K;
  int64_t ldc;
  int64_t batch_stride_c;
  int kb_per_split;  // mode 1: k-blocks per split
  int mode;          // 0: z = batch index, 1: z = split index (write partials)
  int tma_store;     // 1: epilogue through shared memory + TMA tensor stores (tmC)
  int tiles_n, tiles_m, tiles_z;  // output tile grid
  int run, runs;     // B-resident form: m-tiles per run, runs in all (tiles_z x tiles_n x segments);
                     // streaming form (run 0): tiles blockIdx.x + i * gridDim.x, n fastest
  int segs;          // B-resident form: runs per tile column
  int group;         // streaming form: m-tiles per tile group (1: row-band order)
};

// One output tile: its corner, batch / split index and k-block range.
struct Tile {
  int n0, m0, z, batch, kb_begin, nk;
};
// A run: tiles (z, n0, m-tiles mt0 .. mt0 + len - 1).  B-resident form: run
// r of all p.runs, segment-major; streaming form: tile id r (n fastest), len 1.
struct Run {
  int z, n0, mt0, len;
};
template <bool RES>
__device__ __forceinline__ Run run_at(const Params& p, int r, int bn) {
  Run R;
  if (RES) {
    const int per_z = p.tiles_n * p.segs;
    R.z = r / per_z;
    const int rest = r - R.z * per_z;
    const int seg = rest / p.tiles_n;
    R.n0 = (rest - seg * p.tiles_n) * bn;
    R.mt0 = seg * p.run;
    R.len = min(p.run, p.tiles_m - R.mt0);
  } else {
    const int per_z = p.tiles_n * p.tiles_m;
    R.z = r / per_z;
    const int rest = r - R.z * per_z;
    if (p.group > 1) {
      // groups of `group` m-tiles; inside a group m runs fastest, then n
      const int grp = rest / (p.group * p.tiles_n);
      const int m0 = grp * p.group;
      const int gm = min(p.group, p.tiles_m - m0);
      const int within = rest - grp * p.group * p.tiles_n;
      R.n0 = (within / gm) * bn;
      R.mt0 = m0 + within % gm;
    } else {
      R.n0 = (rest % p.tiles_n) * bn;
      R.mt0 = rest / p.tiles_n;
    }
    R.len = 1;
  }
  return R;
}
template <bool RES>
__device__ __forceinline__ int run_count(const Params& p, int ntiles) {
  return RES ? p.runs : ntiles;
}
// The run's length, and its jt-th tile; both recompute the run from r, so
// that only r and jt stay live in the loops (the promotion warps hold 128
// accumulators each).
template <bool RES>
__device__ __forceinline__ int run_len(const Params& p, int r, int bn) {
  return RES ? run_at<RES>(p, r, bn).len : 1;
}
// Step (r, jt) to this CTA's next tile.
template <bool RES>
__device__ __forceinline__ void next_in_walk(const Params& p, int& r, int& jt, int bn) {
  if (++jt >= run_len<RES>(p, r, bn)) {
    jt = 0;
    r += (int)gridDim.x;
  }
}
__device__ __forceinline__ Tile tile_in(const Params& p, const Run& R, int j, int nk_total) {
  Tile T;
  T.n0 = R.n0;
  T.m0 = (R.mt0 + j) * BM;
  T.z = R.z;
  T.batch = T.z;
  T.kb_begin = 0;
  int kb_end = nk_total;
  if (p.mode == 1) {  // z is the split index
    T.kb_begin = T.z * p.kb_per_split;
    kb_end = min(nk_total, T.kb_begin + p.kb_per_split);
    T.batch = 0;
  }
  T.nk = max(kb_end - T.kb_begin, 0);
  return T;
}

template <int BN, bool TRANS_A, bool RES>
__global__ void __launch_bounds__(kThreads, 1)
gemm3x_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const __grid_constant__ CUtensorMap tmC, Params p) {
  using CF = Cfg<BN, RES>;
  constexpr int S = kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* panel = smem + S * CF::STAGE_BYTES;    // B panel (B-resident form), 1024-aligned
  uint8_t* staging = panel + CF::PANEL_BYTES;     // 1024-aligned: all sizes above are multiples of 1 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(staging + CF::STAGING_BYTES);
  // bars: [0,S) full, [S,2S) conv, [2S,3S) empty, [3S,3S+2) chunk_full, [3S+2,3S+4) chunk_empty,
  //       3S+4 panel_full, 3S+5 panel_conv, 3S+6 panel_empty
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * S + 7);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk_total = (p.K + BK - 1) / BK;
  const int ntiles = p.tiles_n * p.tiles_m * p.tiles_z;

  auto full = [&](int s) { return smem_u32(bars + s); };
  auto conv = [&](int s) { return smem_u32(bars + S + s); };
  auto empty = [&](int s) { return smem_u32(bars + 2 * S + s); };
  auto chunk_full = [&](int b) { return smem_u32(bars + 3 * S + b); };
  auto chunk_empty = [&](int b) { return smem_u32(bars + 3 * S + 2 + b); };
  const uint32_t panel_full = smem_u32(bars + 3 * S + 4);
  const uint32_t panel_conv = smem_u32(bars + 3 * S + 5);
  const uint32_t panel_empty = smem_u32(bars + 3 * S + 6);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full(s), 1);
      mbar_init(conv(s), kConvThreads);
      mbar_init(empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(chunk_full(b), 1);
      mbar_init(chunk_empty(b), kPromoThreads);
    }
    mbar_init(panel_full, 1);
    mbar_init(panel_conv, kConvThreads);
    mbar_init(panel_empty, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), CF::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto stage_ptr = [&](int s) { return smem + s * CF::STAGE_BYTES; };

  // Every role walks the same tiles; g counts k-blocks (stage ring slots)
  // and gc TMEM chunks over all tiles of this CTA.
  if (warp < kPromoWarp0) {
    setmaxnreg_dec64();
    if (warp == 0) {
      // ---------------- TMA producer
      if (lane == 0) {
        int g = 0, np = 0;
        bool alive = true;
        for (int r = blockIdx.x; r < run_count<RES>(p, ntiles) && alive; r += gridDim.x) {
          if (RES) {
            const Run R = run_at<RES>(p, r, BN);
            // the previous panel's MMAs must be done before it is overwritten
            if (!mbar_wait(panel_empty, (np & 1) ^ 1, abort_flag)) break;
            mbar_expect_tx(panel_full, nk_total * CF::B_BYTES);
            for (int kb = 0; kb < nk_total; ++kb)
#pragma unroll
              for (int j = 0; j < BN / 32; ++j)
                tma_load_3d(smem_u32(panel + kb * 2 * CF::B_BYTES + j * 2048), &tmB, panel_full, R.n0 + 32 * j,
                            kb * BK, R.z);
            ++np;
          }
          for (int jt = 0; jt < run_len<RES>(p, r, BN) && alive; ++jt) {
            const Tile T = tile_in(p, run_at<RES>(p, r, BN), jt, nk_total);
            for (int it = 0; it < T.nk; ++it) {
              const int s = g % S;
              if (!mbar_wait(empty(s), ((g / S) & 1) ^ 1, abort_flag)) {
                alive = false;
                break;
              }
              uint8_t* st = stage_ptr(s);
              const int k0 = (T.kb_begin + it) * BK;
              mbar_expect_tx(full(s), RES ? CF::A_BYTES : CF::A_BYTES + CF::B_BYTES);
              if (TRANS_A) {
#pragma unroll
                for (int j = 0; j < BM / 32; ++j)
                  tma_load_3d(smem_u32(st + j * 2048), &tmA, full(s), T.m0 + 32 * j, k0, T.batch);
              } else {
                tma_load_3d(smem_u32(st), &tmA, full(s), k0, T.m0, T.batch);
              }
              if (!RES) {
#pragma unroll
                for (int j = 0; j < BN / 32; ++j)
                  tma_load_3d(smem_u32(st + CF::A_BYTES + j * 2048), &tmB, full(s), T.n0 + 32 * j, k0, T.batch);
              }
              ++g;
            }
          }
        }
        // drain: every issued load must land before the CTA may exit
        for (int gi = max(g - S, 0); gi < g; ++gi) {
          const int s = gi % S;
          const uint64_t t0 = globaltimer();
          while (!mbar_try_wait(full(s), (gi / S) & 1)) {
            if (globaltimer() - t0 > kWaitLimitNs) break;
          }
        }
        if (np > 0) {
          const uint64_t t0 = globaltimer();
          while (!mbar_try_wait(panel_full, (np - 1) & 1)) {
            if (globaltimer() - t0 > kWaitLimitNs) break;
          }
        }
      }
    } else if (warp == 1) {
      // ---------------- MMA issuer
      if (lane == 0) {
        constexpr uint32_t idesc = make_idesc(BM, BN, TRANS_A);
        int g = 0, gc = 0, np = 0;
        bool alive = true;
        for (int r = blockIdx.x; r < run_count<RES>(p, ntiles) && alive; r += gridDim.x) {
          if (RES) {
            if (!mbar_wait(panel_conv, np & 1, abort_flag)) break;
            ++np;
          }
          for (int jt = 0; jt < run_len<RES>(p, r, BN) && alive; ++jt) {
            const Tile T = tile_in(p, run_at<RES>(p, r, BN), jt, nk_total);
            for (int it = 0; it < T.nk; ++it, ++g) {
              const int s = g % S;
              const int b = gc & 1;
              const bool chunk_first = (it % kChunkBlocks) == 0;
              const bool chunk_last = (it % kChunkBlocks) == kChunkBlocks - 1 || it == T.nk - 1;
              if (chunk_first && !mbar_wait(chunk_empty(b), ((gc >> 1) & 1) ^ 1, abort_flag)) {
                alive = false;
                break;
              }
              if (!mbar_wait(conv(s), (g / S) & 1, abort_flag)) {
                alive = false;
                break;
              }
              tc_fence_after();
              uint8_t* st = stage_ptr(s);
              uint32_t a_hi, a_lo, b_hi, b_lo;
              if (RES) {
                a_hi = smem_u32(st);
                a_lo = a_hi + CF::A_BYTES;
                b_hi = smem_u32(panel + it * 2 * CF::B_BYTES);
                b_lo = b_hi + CF::B_BYTES;
              } else {
                a_hi = smem_u32(st);
                b_hi = a_hi + CF::A_BYTES;
                a_lo = b_hi + CF::B_BYTES;
                b_lo = a_lo + CF::A_BYTES;
              }
              const uint32_t d = tmem + (uint32_t)(b * BN);
#pragma unroll
              for (int kk = 0; kk < BK / 8; ++kk) {
                const uint32_t aoff = TRANS_A ? kk * 1024 : kk * 32;
                const uint32_t boff = kk * 1024;
                const uint64_t dah = TRANS_A ? desc_mnmajor(a_hi + aoff) : desc_kmajor(a_hi + aoff);
                const uint64_t dal = TRANS_A ? desc_mnmajor(a_lo + aoff) : desc_kmajor(a_lo + aoff);
                const uint64_t dbh = desc_mnmajor(b_hi + boff);
                const uint64_t dbl = desc_mnmajor(b_lo + boff);
                mma_tf32(d, dal, dbh, idesc, (chunk_first && kk == 0) ? 0u : 1u);
                mma_tf32(d, dah, dbl, idesc, 1u);
                mma_tf32(d, dah, dbh, idesc, 1u);
              }
              mma_commit(empty(s));
              if (chunk_last) {
                mma_commit(chunk_full(b));
                ++gc;
              }
            }
          }
          // end of a run: release the panel once its MMAs complete
          if (RES && alive) mma_commit(panel_empty);
        }
      }
    } else {
      // ---------------- lo converters (warps 2..7)
      const int t0 = threadIdx.x - kConvWarp0 * 32;
      int g = 0, np = 0;
      bool alive = true;
      for (int r = blockIdx.x; r < run_count<RES>(p, ntiles) && alive; r += gridDim.x) {
        if (RES) {
          if (!mbar_wait(panel_full, np & 1, abort_flag)) break;
          for (int kb = 0; kb < nk_total; ++kb)
            lo_buffer(reinterpret_cast<const float4*>(panel + kb * 2 * CF::B_BYTES),
                      reinterpret_cast<float4*>(panel + kb * 2 * CF::B_BYTES + CF::B_BYTES), CF::B_BYTES / 16, t0);
          fence_proxy_async();
          mbar_arrive(panel_conv);
          ++np;
        }
        for (int jt = 0; jt < run_len<RES>(p, r, BN) && alive; ++jt) {
          const Tile T = tile_in(p, run_at<RES>(p, r, BN), jt, nk_total);
          for (int it = 0; it < T.nk; ++it, ++g) {
            const int s = g % S;
            if (!mbar_wait(full(s), (g / S) & 1, abort_flag)) {
              alive = false;
              break;
            }
            uint8_t* st = stage_ptr(s);
            if (RES) {
              lo_buffer(reinterpret_cast<const float4*>(st), reinterpret_cast<float4*>(st + CF::A_BYTES),
                        CF::A_BYTES / 16, t0);
            } else {
              lo_buffer(reinterpret_cast<const float4*>(st),
                        reinterpret_cast<float4*>(st + CF::A_BYTES + CF::B_BYTES), CF::A_BYTES / 16, t0);
              lo_buffer(reinterpret_cast<const float4*>(st + CF::A_BYTES),
                        reinterpret_cast<float4*>(st + 2 * CF::A_BYTES + CF::B_BYTES), CF::B_BYTES / 16, t0);
            }
            fence_proxy_async();
            mbar_arrive(conv(s));
          }
        }
      }
    }
  } else {
    setmaxnreg_inc192();
    // ---------------- promotion + epilogue (warps 8..15)
    const int pw = warp - kPromoWarp0;
    const int q = warp & 3;                         // TMEM lane quarter this warp may access
    const int col_base = (pw >> 2) * CF::COLS_PER_WARP;
    constexpr int NCOL = CF::COLS_PER_WARP;
    uint8_t* box = staging + pw * kBoxBytes;        // this warp's 32 x 32 C box
    int gc = 0;
    bool ok = true;
    // one flat loop over this CTA's tiles (run r, position jt): nested loops
    // here cost the accumulators registers
    for (int r = blockIdx.x, jt = 0; r < run_count<RES>(p, ntiles) && ok; next_in_walk<RES>(p, r, jt, BN)) {
      const Tile T = tile_in(p, run_at<RES>(p, r, BN), jt, nk_total);
      const int nchunks = (T.nk + kChunkBlocks - 1) / kChunkBlocks;
      float tot[NCOL];
#pragma unroll
      for (int j = 0; j < NCOL; ++j) tot[j] = 0.0f;
      for (int c = 0; c < nchunks; ++c, ++gc) {
        const int b = gc & 1;
        ok = __all_sync(0xffffffffu, mbar_wait(chunk_full(b), (gc >> 1) & 1, abort_flag));
        if (!ok) break;
        tc_fence_after();
        const uint32_t base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * BN + col_base);
#pragma unroll
        for (int j = 0; j < NCOL / 32; ++j) {
          uint32_t r[32];
          tmem_ld32(base + j * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) tot[j * 32 + i] += __uint_as_float(r[i]);
        }
        tc_fence_before();
        mbar_arrive(chunk_empty(b));
      }
      if (!ok) break;
      if (p.tma_store) {
        // Rows q*32 + lane of the tile, 32 columns per box, 128B swizzle
        // (conflict-free writes).  The box buffer is reused once the previous
        // store from it has been read; rows >= M / cols >= N are clipped.
        const int zc = p.mode == 1 ? T.z : T.batch;
#pragma unroll
        for (int bx = 0; bx < NCOL / 32; ++bx) {
          if (lane == 0) bulk_wait_read_all();
          __syncwarp();
#pragma unroll
          for (int c4 = 0; c4 < 8; ++c4)
            *reinterpret_cast<float4*>(box + lane * 128 + ((c4 ^ (lane & 7)) * 16)) =
                make_float4(tot[bx * 32 + c4 * 4], tot[bx * 32 + c4 * 4 + 1], tot[bx * 32 + c4 * 4 + 2],
                            tot[bx * 32 + c4 * 4 + 3]);
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&tmC, smem_u32(box), T.n0 + col_base + 32 * bx, T.m0 + q * 32, zc);
            bulk_commit();
          }
        }
      } else {
        const int row = T.m0 + q * 32 + lane;
        float* out = p.C + (int64_t)T.batch * p.batch_stride_c;
        int64_t ldo = p.ldc;
        if (p.mode == 1) {
          out = p.C + (int64_t)T.z * p.M * p.N;
          ldo = p.N;
        }
        if (row < p.M) {
          float* orow = out + (int64_t)row * ldo;
          const int col0 = T.n0 + col_base;
          const bool vec = ((ldo & 3) == 0) && ((reinterpret_cast<uintptr_t>(out) & 15) == 0);
          if (vec && col0 + NCOL <= p.N) {
#pragma unroll
            for (int j = 0; j < NCOL; j += 4)
              *reinterpret_cast<float4*>(orow + col0 + j) = make_float4(tot[j], tot[j + 1], tot[j + 2], tot[j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < NCOL; ++j)
              if (col0 + j < p.N) orow[col0 + j] = tot[j];
          }
        }
      }
    }
    if (lane == 0) bulk_wait_all();  // stores complete before the CTA exits
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, CF::TMEM_COLS);
  }
}

// deterministic split-K reduction: C[m, n] = sum_z partial[z][m][n], z in order
__global__ void splitk_reduce_kernel(const float* __restrict__ part, float* __restrict__ C, int M, int N,
                                     int64_t ldc, int Z) {
  const int64_t total = (int64_t)M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int zz = 0; zz < Z; ++zz) s += part[(int64_t)zz * total + i];
    const int64_t m = i / N, n = i - m * N;
    C[m * ldc + n] = s;
  }
}

// CUDA-core fp32 GEMM for shapes the TMA path cannot describe.
__global__ void __launch_bounds__(256)
gemm_simt_kernel(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ C, int M,
                 int N, int K, int64_t lda, int64_t ldb, int64_t ldc, int64_t sA, int64_t sB, int64_t sC,
                 int trans_a) {
  __shared__ float As[16][17], Bs[16][17];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int b = blockIdx.z;
  A += b * sA;
  B += b * sB;
  C += b * sC;
  const int row = blockIdx.y * 16 + ty, col = blockIdx.x * 16 + tx;
  float acc = 0.f;
  for (int k0 = 0; k0 < K; k0 += 16) {
    const int ka = k0 + tx, kb = k0 + ty;
    As[ty][tx] = (row < M && ka < K) ? (trans_a ? A[(int64_t)ka * lda + row] : A[(int64_t)row * lda + ka]) : 0.f;
    Bs[ty][tx] = (kb < K && col < N) ? B[(int64_t)kb * ldb + col] : 0.f;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 16; ++k) acc = fmaf(As[ty][k], Bs[k][tx], acc);
    __syncthreads();
  }
  if (row < M && col < N) C[(int64_t)row * ldc + col] = acc;
}

// ------------------------------------------------------------------ host side
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  }
  return fn;
}

// 3-D fp32 tensor map {inner, outer, batch}, box {box_inner, box_outer, 1}.
// K-major operands (box_inner 16 = 64 B) use the 64B swizzle; MN-major
// operands (box_inner 32 = 128 B) the 128B swizzle with 32-byte atoms, the
// only MN-major layout TF32 UMMA reads.
int make_map(CUtensorMap* tm, const float* base, int64_t inner, int64_t outer, int64_t batch,
             int64_t row_stride_elems, int64_t batch_stride_elems, int box_outer, bool mn_major) {
  EncodeFn enc = encode_fn();
  KB_REQUIRE(enc != nullptr, KB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)outer, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)row_stride_elems * 4, (cuuint64_t)batch_stride_elems * 4};
  cuuint32_t box[3] = {mn_major ? 32u : (cuuint32_t)BK, (cuuint32_t)box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE,
                   mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_64B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  KB_REQUIRE(r == CUDA_SUCCESS, KB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return KB_OK;
}

// 3-D fp32 tensor map for the C tile store: {N, M, Z} with box {32, 32, 1},
// 128B swizzle (matches the staging layout of the epilogue).
int make_store_map(CUtensorMap* tm, float* base, int64_t N, int64_t M, int64_t Z, int64_t row_stride,
                   int64_t z_stride) {
  EncodeFn enc = encode_fn();
  KB_REQUIRE(enc != nullptr, KB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)N, (cuuint64_t)M, (cuuint64_t)Z};
  cuuint64_t strides[2] = {(cuuint64_t)row_stride * 4, (cuuint64_t)z_stride * 4};
  cuuint32_t box[3] = {(cuuint32_t)kBoxCols, (cuuint32_t)kBoxRows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  KB_REQUIRE(r == CUDA_SUCCESS, KB_ERR_CUDA, "cuTensorMapEncodeTiled (C) failed (%d)", (int)r);
  return KB_OK;
}

template <int BN, bool TA, bool RES = false>
int launch_tc(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const Params& p, dim3 grid,
              cudaStream_t s) {
  auto kern = gemm3x_kernel<BN, TA, RES>;
  constexpr int smem = Cfg<BN, RES>::SMEM_BYTES;
  static uint64_t attr_set = 0;  // one bit per device ordinal
  int dev = 0;
  KB_CUDA(cudaGetDevice(&dev));
  if (dev < 64 && !(attr_set >> dev & 1)) {
    KB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr_set |= 1ull << dev;
  }
  kern<<<grid, kThreads, smem, s>>>(ta, tb, tc, p);
  return check_launch("gemm3x_kernel");
}

// B-resident form: pick the run length.  Cost of a choice, in tile times:
// the runs the busiest CTA walks x (run length + kSwitchTiles for the panel
// reload between runs).  Taken when it is within 20 % of the streaming form's
// tiles per CTA: a B-resident tile is that much cheaper at 48-64 deep K
// (measured on the B200 over 32768^2, 16384^2, 32768x8192, 8192x32768,
// 65536x4096 and a 3x38400x1792 batch: 0.83-0.90 of the streaming time at
// K = 64, 0.92-0.99 at K = 48, bitwise-identical output).  At K <= 32 the
// streaming form is already near the output-write bound and the gain
// turned into losses of up to 15 %, so it keeps those.
constexpr int kResMinKB = 3;
constexpr int kSwitchTiles = 2;
struct ResPlan {
  int run = 0, segs = 0, runs = 0;
};
bool plan_runs(int64_t tm, int64_t tn, int64_t tz, int sms, ResPlan* out) {
  const int64_t ntiles = tm * tn * tz;
  if (ntiles < 2 * (int64_t)sms || ntiles > 0x7fffffff) return false;
  int64_t best_cost = -1;
  for (int64_t segs = 1; segs <= std::min<int64_t>(tm, 1024); ++segs) {
    const int64_t run = ceil_div(tm, segs);
    if (ceil_div(tm, run) != segs) continue;  // the same run length as a smaller segs
    const int64_t runs = tz * tn * segs;
    if (runs > 0x7fffffff) break;
    const int64_t per_cta = ceil_div(runs, (int64_t)sms);
    const int64_t cost = per_cta * (run + kSwitchTiles);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      out->run = (int)run;
      out->segs = (int)segs;
      out->runs = (int)runs;
    }
  }
  const int64_t stream_cost = ceil_div(ntiles, (int64_t)sms);
  return best_cost > 0 && best_cost * 5 <= stream_cost * 6;
}

struct GemmArgs {
  const float* A;
  const float* B;
  float* C;
  int64_t batch, M, N, K, lda, ldb, ldc, sA, sB, sC;
  bool trans_a;
};

bool tma_ok(const GemmArgs& g) {
  auto a16 = [](int64_t v) { return (v * 4) % 16 == 0; };
  return aligned16(g.A) && aligned16(g.B) && a16(g.lda) && a16(g.ldb) && a16(g.sA) && a16(g.sB) &&
         g.M < (1LL << 31) && g.N < (1LL << 31) && g.K < (1LL << 31) && g.K > 0 && g.batch <= 65535 &&
         (g.trans_a ? g.M : g.K) >= 4 && g.N >= 4;
}

int run_simt(const GemmArgs& g, cudaStream_t s) {
  KB_REQUIRE(g.batch <= 65535, KB_ERR_UNSUPPORTED, "batch > 65535");
  dim3 grid((unsigned)ceil_div(g.N, 16), (unsigned)ceil_div(g.M, 16), (unsigned)g.batch);
  gemm_simt_kernel<<<grid, 256, 0, s>>>(g.A, g.B, g.C, (int)g.M, (int)g.N, (int)g.K, g.lda, g.ldb, g.ldc,
                                        g.sA, g.sB, g.sC, g.trans_a ? 1 : 0);
  return check_launch("gemm_simt_kernel");
}

// Order of the streaming tile walk.  The persistent CTAs work on about
// sm_count consecutive tiles at a time and move through K at similar speed,
// so what one K slab of those tiles reads from L2 and DRAM is their distinct
// A row blocks and B column blocks.  In row-band order (n fastest) a wave of
// 148 tiles of an 8192^3 GEMM spans 4.6 row bands and all 32 column blocks,
// so every wave streams the whole of B (256 MB) from DRAM: 4.7 GB of DRAM
// reads per launch against 0.5 GB of operands (ncu).  Groups of G m-tiles
// walked m-fastest make a wave ~G x 148/G tiles; the A + B bytes of a wave,
// G * BM + (148 / G) * BN rows of K, are smallest near G = sqrt(148 BN / BM)
// = 17.  Only long-K walks with many row bands are regrouped; the B-resident
// small-K form has its own run order.
int tile_group(int tiles_m, int tiles_n, int nk, int bn) {
  constexpr int G = 16;
  if (nk < 64 || tiles_m <= G || tiles_n <= 2) return 1;
  (void)bn;
  return G;
}

// splits > 1: partial tiles go to `ws` and are reduced into C afterwards.
// reduce_into_c false (single-matrix GEMMs only): the partial tiles
// [splits][M][N] stay in `ws` (one split: C itself goes to ws) and no
// reduction runs; *splits_out reports how many there are.
int run_gemm(const GemmArgs& g, int splits, float* ws, cudaStream_t s, bool reduce_into_c = true,
             int* splits_out = nullptr) {
  if (splits_out) *splits_out = 1;
  if (g.M == 0 || g.N == 0 || g.batch == 0) return KB_OK;
  if (!tma_ok(g)) {
    if (reduce_into_c) return run_simt(g, s);
    GemmArgs w = g;
    w.C = ws;
    w.ldc = g.N;
    w.sC = g.M * g.N;
    return run_simt(w, s);
  }
  const bool bn256 = g.N > 128;
  const int BN = bn256 ? 256 : 128;
  CUtensorMap ta, tb;
  if (g.trans_a) {
    if (int st = make_map(&ta, g.A, g.M, g.K, g.batch, g.lda, g.sA, BK, true)) return st;
  } else {
    if (int st = make_map(&ta, g.A, g.K, g.M, g.batch, g.lda, g.sA, BM, false)) return st;
  }
  if (int st = make_map(&tb, g.B, g.N, g.K, g.batch, g.ldb, g.sB, BK, true)) return st;
  const int nk = (int)ceil_div(g.K, BK);
  Params p{};
  p.M = (int)g.M;
  p.N = (int)g.N;
  p.K = (int)g.K;
  dim3 grid((unsigned)ceil_div(g.N, BN), (unsigned)ceil_div(g.M, BM), 1);
  if (splits > 1 || !reduce_into_c) {
    const int kbps = (int)ceil_div(nk, splits);
    splits = (int)ceil_div(nk, kbps);  // no empty split
    if (splits_out) *splits_out = splits;
    p.C = ws;
    p.ldc = g.N;
    p.mode = 1;
    p.kb_per_split = kbps;
    grid.z = splits;
  } else {
    p.C = g.C;
    p.ldc = g.ldc;
    p.batch_stride_c = g.sC;
    p.mode = 0;
    grid.z = (unsigned)g.batch;
  }
  // TMA-store epilogue when C (or the partial buffer) is describable:
  // 16-byte aligned base and row / batch strides that are multiples of 16 B
  CUtensorMap tc;
  memset(&tc, 0, sizeof(tc));
  p.tma_store = 0;
  if (p.mode == 1) {
    if (aligned16(ws) && g.N % 4 == 0 &&
        make_store_map(&tc, ws, g.N, g.M, grid.z, g.N, g.M * g.N) == KB_OK)
      p.tma_store = 1;
  } else if (aligned16(g.C) && g.ldc % 4 == 0 && (g.batch == 1 || g.sC % 4 == 0)) {
    if (make_store_map(&tc, g.C, g.N, g.M, g.batch, g.ldc, g.batch > 1 ? g.sC : g.ldc * g.M) == KB_OK)
      p.tma_store = 1;
  }
  p.tiles_n = (int)grid.x;
  p.tiles_m = (int)grid.y;
  p.tiles_z = (int)grid.z;
  p.group = tile_group(p.tiles_m, p.tiles_n, nk, BN);
  // persistent: one CTA per SM (the shared memory and TMEM footprints allow no more)
  const int64_t ntiles = (int64_t)grid.x * grid.y * grid.z;
  KB_REQUIRE(ntiles <= 0x7fffffff, KB_ERR_UNSUPPORTED, "gemm: too many tiles");
  dim3 pgrid((unsigned)std::min<int64_t>(ntiles, sm_count()), 1, 1);
  ResPlan rp;
  const bool res = bn256 && !g.trans_a && p.mode == 0 && nk <= kResKB && nk >= kResMinKB &&
                   plan_runs(p.tiles_m, p.tiles_n, p.tiles_z, sm_count(), &rp);
  int st;
  if (res) {
    p.run = rp.run;
    p.segs = rp.segs;
    p.runs = rp.runs;
    pgrid.x = (unsigned)std::min(rp.runs, sm_count());
    st = launch_tc<256, false, true>(ta, tb, tc, p, pgrid, s);
  } else if (bn256)
    st = g.trans_a ? launch_tc<256, true>(ta, tb, tc, p, pgrid, s) : launch_tc<256, false>(ta, tb, tc, p, pgrid, s);
  else
    st = g.trans_a ? launch_tc<128, true>(ta, tb, tc, p, pgrid, s) : launch_tc<128, false>(ta, tb, tc, p, pgrid, s);
  if (st) return st;
  if (splits > 1 && reduce_into_c) {
    const int64_t total = g.M * g.N;
    const int blocks = (int)std::min<int64_t>(ceil_div(total, 256), (int64_t)sm_count() * 8);
    splitk_reduce_kernel<<<blocks, 256, 0, s>>>(ws, g.C, (int)g.M, (int)g.N, g.ldc, splits);
    return check_launch("splitk_reduce_kernel");
  }
  return KB_OK;
}

constexpr int kMaxSms = 160;

int splitk_count(int64_t M, int64_t N, int64_t K, int sms) {
  const int64_t tiles = ceil_div(M, BM) * ceil_div(N, N > 128 ? 256 : 128);
  const int64_t nk = ceil_div(K, BK);
  int64_t sp = std::max<int64_t>(1, sms / std::max<int64_t>(tiles, 1));
  sp = std::min<int64_t>(sp, std::max<int64_t>(nk / 4, 1));  // at least 4 k-blocks per split
  return (int)sp;
}

// K splits for a plain GEMM whose tiles leave most of the persistent grid
// idle: fewer output tiles than SMs (a 256-row strip of an 8192-wide,
// 8192-deep GEMM has 64 tiles for 148 SMs).  Cutting K into s splits gives
// s x tiles shorter work units; it costs one partial tile per split in
// memory, a deterministic reduction pass (s + 1 reads and writes of C's
// size) and a per-unit pipeline fill.  Model, per SM: a 16-deep K block
// takes t_kb (0.68 us measured at 8192^3 in steady state), a work unit t_unit
// more; the reduction runs at HBM speed.  The split is taken when the model
// saves at least 3 %.  Grids of a wave or more are never split: measured on
// a 1024 x 8192 x 8192 row shard (256 tiles, 1.73 waves), the split into 4
// was 2.7 % slower than the unsplit walk (0.651 vs 0.634 ms) — the SMs of
// a partial last wave run faster than the model assumes (the chip is power-
// and L2-limited, and fewer busy SMs share both), and at 256 rows
// (0.43 waves) the split into 2 was 1.75x faster (0.210 vs 0.367 ms).
int wave_splits(int64_t M, int64_t N, int64_t K, int sms) {
  constexpr double t_kb = 0.68e-6, t_unit = 2.0e-6, t_launch = 5.0e-6, hbm = 6.4e12;
  const int64_t tiles = ceil_div(M, BM) * ceil_div(N, N > 128 ? 256 : 128);
  const int64_t nk = ceil_div(K, BK);
  if (tiles >= sms) return 1;
  auto model = [&](int sp) {
    const int64_t kbps = ceil_div(nk, sp);
    const int64_t units = tiles * ceil_div(nk, kbps);
    double t = (double)ceil_div(units, (int64_t)sms) * ((double)kbps * t_kb + t_unit);
    if (sp > 1) t += (double)(sp + 1) * (double)M * (double)N * 4.0 / hbm + t_launch;
    return t;
  };
  int best = 1;
  double best_t = model(1);
  for (int sp = 2; sp <= 8; ++sp) {
    if (nk / sp < 8) break;  // at least 8 K blocks (128 of K) per split
    const double t = model(sp);
    if (t < best_t * 0.97) {
      best = sp;
      best_t = t;
    }
  }
  return best;
}

}  // namespace gemm
}  // namespace kb

extern "C" {

size_t kb_sgemm_workspace_size(int64_t M, int64_t N, int64_t K, int trans_a) {
  if (M <= 0 || N <= 0 || K <= 0 || trans_a) return 0;
  const int sp = kb::gemm::wave_splits(M, N, K, kb::sm_count());
  return sp > 1 ? (size_t)sp * M * N * sizeof(float) : 0;
}

int kb_sgemm_3xtf32_ws(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                       int64_t ldb, int64_t ldc, int trans_a, void* workspace, size_t workspace_bytes,
                       kbStream stream) {
  const char* name = "kb_sgemm_3xtf32_ws";
  KB_REQUIRE(M >= 0 && N >= 0 && K >= 0, KB_ERR_INVALID_ARG, "%s: negative size", name);
  if (M == 0 || N == 0) return KB_OK;
  KB_REQUIRE(A && B && C, KB_ERR_INVALID_ARG, "%s: null pointer", name);
  KB_REQUIRE(lda >= (trans_a ? M : K) && ldb >= N && ldc >= N, KB_ERR_INVALID_ARG,
             "%s: leading dimension too small", name);
  kb::gemm::GemmArgs g{A, B, C, 1, M, N, K, lda, ldb, ldc, 0, 0, 0, trans_a != 0};
  g.sA = lda * (trans_a ? K : M);
  g.sB = ldb * K;
  g.sC = ldc * M;
  int sp = trans_a ? 1 : kb::gemm::wave_splits(M, N, K, kb::sm_count());
  // a workspace too small for the split (or misaligned, or an operand layout
  // the TMA path cannot describe) runs the GEMM unsplit: same result class
  if (sp > 1 && (!workspace || workspace_bytes < (size_t)sp * M * N * sizeof(float) ||
                 !kb::aligned16(workspace) || !kb::gemm::tma_ok(g)))
    sp = 1;
  return kb::gemm::run_gemm(g, sp, static_cast<float*>(workspace), stream);
}

int kb_read_fault(int clear, int* value) {
  KB_REQUIRE(value, KB_ERR_INVALID_ARG, "kb_read_fault: null pointer");
  KB_CUDA(cudaMemcpyFromSymbol(value, kb::g_gemm_fault, sizeof(int)));
  if (clear) {
    const int zero = 0;
    KB_CUDA(cudaMemcpyToSymbol(kb::g_gemm_fault, &zero, sizeof(int)));
  }
  return KB_OK;
}

int kb_sgemm_3xtf32(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
                    int64_t lda, int64_t ldb, int64_t ldc, int trans_a, kbStream stream) {
  KB_REQUIRE(M >= 0 && N >= 0 && K >= 0, KB_ERR_INVALID_ARG, "kb_sgemm_3xtf32: negative size");
  if (M == 0 || N == 0) return KB_OK;
  KB_REQUIRE(A && B && C, KB_ERR_INVALID_ARG, "kb_sgemm_3xtf32: null pointer");
  KB_REQUIRE(lda >= (trans_a ? M : K) && ldb >= N && ldc >= N, KB_ERR_INVALID_ARG,
             "kb_sgemm_3xtf32: leading dimension too small");
  kb::gemm::GemmArgs g{A, B, C, 1, M, N, K, lda, ldb, ldc, 0, 0, 0, trans_a != 0};
  g.sA = lda * (trans_a ? K : M);
  g.sB = ldb * K;
  g.sC = ldc * M;
  return kb::gemm::run_gemm(g, 1, nullptr, stream);
}

int kb_bgemm_3xtf32(const float* A, const float* B, float* C, int64_t batch, int64_t M, int64_t N,
                    int64_t K, kbStream stream) {
  KB_REQUIRE(batch >= 0 && M >= 0 && N >= 0 && K >= 0, KB_ERR_INVALID_ARG, "kb_bgemm_3xtf32: negative size");
  if (batch == 0 || M == 0 || N == 0) return KB_OK;
  KB_REQUIRE(A && B && C, KB_ERR_INVALID_ARG, "kb_bgemm_3xtf32: null pointer");
  KB_REQUIRE(batch <= 65535, KB_ERR_UNSUPPORTED, "kb_bgemm_3xtf32: batch > 65535");
  kb::gemm::GemmArgs g{A, B, C, batch, M, N, K, K, N, N, M * K, K * N, M * N, false};
  return kb::gemm::run_gemm(g, 1, nullptr, stream);
}

size_t kb_gemm_splitk_workspace_size(int64_t M, int64_t N, int64_t K) {
  const int sp = kb::gemm::splitk_count(M, N, K, kb::gemm::kMaxSms);
  return sp > 1 ? (size_t)sp * M * N * sizeof(float) : 0;
}

int kb_gemm_splitk_3xtf32(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
                          void* workspace, size_t workspace_bytes, kbStream stream) {
  const char* name = "kb_gemm_splitk_3xtf32";
  KB_REQUIRE(M >= 0 && N >= 0 && K >= 0, KB_ERR_INVALID_ARG, "%s: negative size", name);
  if (M == 0 || N == 0) return KB_OK;
  KB_REQUIRE(A && B && C, KB_ERR_INVALID_ARG, "%s: null pointer", name);
  kb::gemm::GemmArgs g{A, B, C, 1, M, N, K, K, N, N, M * K, K * N, M * N, false};
  int sp = kb::gemm::splitk_count(M, N, K, kb::sm_count());
  if (sp > 1) {
    const size_t need = (size_t)sp * M * N * sizeof(float);
    KB_REQUIRE(workspace && workspace_bytes >= need, KB_ERR_WORKSPACE,
               "%s: workspace of %zu bytes needed, %zu given", name, need, workspace_bytes);
    KB_REQUIRE(kb::aligned16(workspace), KB_ERR_INVALID_ARG, "%s: workspace must be 16-byte aligned", name);
    if (!kb::gemm::tma_ok(g)) sp = 1;
  }
  return kb::gemm::run_gemm(g, sp, static_cast<float*>(workspace), stream);
}

/* K-split partial tiles only, for a caller that fuses their reduction with
 * a cross-GPU one: ws[z][M][N] for z < *splits. */
size_t kb_gemm_splitk_partials_workspace_size(int64_t M, int64_t N, int64_t K) {
  const int sp = kb::gemm::splitk_count(M, N, K, kb::gemm::kMaxSms);
  return (size_t)std::max(sp, 1) * M * N * sizeof(float);
}

int kb_gemm_splitk_partials_3xtf32(const float* A, const float* B, int64_t M, int64_t N, int64_t K,
                                   void* workspace, size_t workspace_bytes, int* splits, kbStream stream) {
  const char* name = "kb_gemm_splitk_partials_3xtf32";
  KB_REQUIRE(M >= 0 && N >= 0 && K >= 0 && splits, KB_ERR_INVALID_ARG, "%s: bad arguments", name);
  *splits = 1;
  if (M == 0 || N == 0) return KB_OK;
  KB_REQUIRE(A && B, KB_ERR_INVALID_ARG, "%s: null pointer", name);
  kb::gemm::GemmArgs g{A, B, nullptr, 1, M, N, K, K, N, N, M * K, K * N, M * N, false};
  int sp = kb::gemm::splitk_count(M, N, K, kb::sm_count());
  if (!kb::gemm::tma_ok(g)) sp = 1;
  const size_t need = (size_t)sp * M * N * sizeof(float);
  KB_REQUIRE(workspace && workspace_bytes >= need, KB_ERR_WORKSPACE,
             "%s: workspace of %zu bytes needed, %zu given", name, need, workspace_bytes);
  KB_REQUIRE(kb::aligned16(workspace), KB_ERR_INVALID_ARG, "%s: workspace must be 16-byte aligned", name);
  return kb::gemm::run_gemm(g, sp, static_cast<float*>(workspace), stream, false, splits);
}

}  // extern "C"
