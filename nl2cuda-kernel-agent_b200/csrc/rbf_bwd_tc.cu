// rbf_bwd_tc.cu -- the fused RBF backward on the sm_100a tensor cores.
//
//   W = G o K,  c = -2 gamma
//   dX[i,:] = c * ( rowsum_j(W)[i] * x_i - sum_j W[i,j] y_j )
//   dY[j,:] = c * ( colsum_i(W)[j] * y_j - sum_i W[i,j] x_i )
//
// Tiles of 128 (i) x 128 (j).  G and K are read from HBM once, as four column strips per tile
// (128 i x 32 j: one 32x128 TMA box each, 128-byte swizzle) through a 4-deep ring -- strip s of
// every tile uses stage s, so one whole tile is in flight.  Both products are 3xTF32
// (hi*hi + hi*lo + lo*hi, fp32 accumulation in TMEM) with A in TMEM:
//   R-warps (thread <-> row i): per strip W[i, 32 j] -> TF32 hi/lo -> TMEM lanes i, the A
//     operand of  D_dX[i,:] += W[i,j] Y[j,:]  (B = the strip's Y rows); rowsum_i.  Streamed:
//     two W buffers, one dX MMA batch per strip.
//   C-warp q (thread <-> column j of quadrant q): from strip q, W^T[j, all 128 i] -> TMEM lanes
//     j, the A operand of  D_dY[j,:] += W^T[j,i] X[i,:]  (B = X rows, four 32-row chunks);
//     colsum_j.  The W^T tile (256 columns) is resident for one tile; the dY batch runs once
//     all four quadrants are written.
// The B operands (X, Y rows, features contiguous) are MN-major and use the 128-byte-swizzle /
// 32-byte-atom layout (descriptor layout type 1, TMA CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B): the
// only shared-memory layout the tensor core accepts for MN-major tf32.
//
// Work split: tiles are ordered (feature slice, j-group, i-block, j-block within the group) and
// the CTAs are split into `group` interleaved sub-grids, one per j-block of a group, so
// neighbouring CTAs read neighbouring column blocks of the same rows at the same time.  Each CTA
// first walks a contiguous static range of i-blocks of one j-block -- a "segment", over which
// the dY accumulator stays in TMEM and is flushed once at the end (red.add of
// c*(colsum*y - acc)) -- then claims tail tiles one at a time from a global counter, so CTAs
// that run fast take more of the tail.  The strip producer decides the sequence and hands it to
// the other roles through a 4-entry ring in shared memory.  The dX
// accumulator is flushed once per tile: -c*acc is staged in shared memory and added into dX by
// a TMA reduce-add, rowsum is added into a per-row vector, and a finalize pass adds
// c*rowsum*x once per row.  The outputs are zeroed first; the fp32 summation order of dX / dY
// varies between runs.  Features are processed in slices of DS (32 or 64); D > 64 runs one
// slice per segment (G and K are re-read per slice).  D % 4 != 0 flushes dX with red.add too.
//
// The DOT instantiation (cosine similarity, on the normalised rows of the split pass) streams
// only G (W = G, half the strip bytes), keeps no row / column sums and uses c = -1, so that
// dX = G Y and dY = G^T X; the per-row normalisation terms are added by cos_finalize_kernel.
//
// TMEM (512 columns): dY acc, two halves (B = [X_hi | X_lo] stacked along N) | dX acc | W
// buffer(s) (hi 32 + lo 32) | [256,384) W^T hi (128 columns of i) | [384,512) W^T lo; the column
// plan by DS is TmemPlan below.
// Shared memory (DS = 64): strip ring 4 x 32 KiB, X ring 2 x 16 KiB, Y ring 2 x 16 KiB, dX
// staging 4 x 8 KiB.  (Build option RBF_BWD_XSTAGES=4: X ring 4 x 16 KiB, no staging; measured
// slower.)
// Warps: 0 TMA producer of strips + Y rows, 1 TMA producer of X rows, 2 dY MMA issuer, 3 dX MMA
// issuer, 4-7 C-warps, 8-11 R-warps (warp w reaches TMEM lanes 32*(w%4)..+31).  Independent
// pipelines sit in different warps: a lane blocked in mbarrier.try_wait holds back its whole
// warp.  Every mbarrier wait is bounded; a timeout is recorded in the workspace status word.
#include <cuda.h>

#include <algorithm>
#include <cstdlib>

#include "rbf_common.cuh"
#include "rbf_kernels.cuh"
#include "rbf_ptx.cuh"

namespace rbf {
namespace {

constexpr int BT = 128;        // tile edge (rows of i and columns of j)
constexpr int SR = 32;         // strip width
constexpr int STAGES = 4;      // strip ring: one stage per strip of a tile
#ifndef RBF_BWD_XSTAGES
#define RBF_BWD_XSTAGES 2
#endif
// X-row ring.  At 4 stages the dX flush staging gives up its shared memory (dX is then flushed
// with red.add from registers, c * rowsum * x included, and no finalize pass runs).
constexpr int XSTAGES = RBF_BWD_XSTAGES;
constexpr bool kStageDx = XSTAGES <= 2;
constexpr int YSTAGES = 2;     // Y-row ring
constexpr int THREADS = 384;
constexpr uint32_t BOX = 32 * 32 * 4;       // 32x32 fp32, 4 KiB
constexpr uint32_t STRIP = 128 * 32 * 4;    // one column strip of G (or K), 16 KiB
// TMEM: [0, 2 DS) the dY accumulator in two halves, W.X_hi (with W_lo.X_hi) | W_hi.X_lo: the dY
// MMAs take B = [X_hi | X_lo] stacked along N, one MMA of N = 2 DS where two of N = DS would be
// needed | dX | the W buffers (hi 32 | lo 32 each) | [256,512) W^T hi | lo.  DS = 64: dX at
// 128, one W buffer at 192 (the stacked accumulator takes the second); DS = 32 (not stacked):
// dY at 0, dX at 64, two W buffers at 128.
constexpr uint32_t COL_DY = 0, COL_WT = 256;
// Stacked dY MMAs at DS = 64 only: at DS = 32 two N = 32 MMAs cost no more than one of N = 64,
// and the stacked form measured 3-5% slower there.
template <int DS> constexpr bool kStackDy = DS == 64;
template <int DS> struct TmemPlan {
  static constexpr uint32_t DX = DS == 64 ? 128 : 64;
  static constexpr uint32_t W = DS == 64 ? 192 : 128;
  static constexpr int WBUFS = DS == 64 ? 1 : 2;
};
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t MN_SBO = 512;       // one K group (4 rows x 128 B) of the 32B-atom layout
constexpr uint32_t MN_LAYOUT = 1;      // descriptor layout type: 128B swizzle, 32B atom

template <int DS>
struct Cfg {
  static constexpr uint32_t X_BYTES = (DS / 32) * BOX;   // 32 rows x DS features, hi or lo
  static constexpr uint32_t STAGING = X_BYTES;           // one R-warp's dX flush: 32 x DS
  static constexpr size_t SMEM = 1024 + STAGES * 2 * STRIP + XSTAGES * 2 * X_BYTES +
                                 YSTAGES * 2 * X_BYTES + (kStageDx ? 4 : 0) * STAGING + 512;
};
static_assert(Cfg<64>::SMEM <= 232448, "backward shared memory over the sm_100 limit");

struct BwdArgs {
  const float* X;
  const float* Y;
  float* dX;
  float* dY;
  float* rowsum;  // [N] sum_j W[i,j], accumulated here when the dX flush goes through TMA
  int64_t N, M, D;
  int tiles_i, tiles_j, num_slices;
  int64_t total_tiles;
  float c;  // -2 gamma
  int* status;
  unsigned long long timeout_ns;
  int debug_skip_first_load;
  int tma_flush;  // dX partials are added by TMA reduce (needs D % 4 == 0)
  int group;             // neighbouring j-blocks walked together (divides tiles_j and the grid)
  int64_t static_rows;   // group rows [0, static_rows) are split into contiguous per-CTA ranges;
  int* counter;          // tiles from static_rows * group on are claimed from this counter
  DyRoute route;  // world > 0: dY partials go to this rank's slot of the routed buffers
  int det;        // deterministic mode: every tile stores its partials into its own slot
  float* dxp;     // [tiles_j][Npad][D]   -c * (W Y) partial of tile (ib, jb), rows ib*128..
  float* rsp;     // [tiles_j][Npad]      rowsum partial of tile (ib, jb)
  float* dyp;     // [tiles_i][M][D]      -c * (W^T X) partial of tile (ib, jb), rows jb*128..
  float* csp;     // [tiles_i][M]         colsum partial of tile (ib, jb)
  int64_t Npad;   // N rounded up to the tile edge
  int ablate;     // development builds only (RBF_TRACE): 1 skip dX reduce, 2 skip rowsum add,
                  // 4 C-warps skip W^T, 8 R-warps skip W, 16 no MMAs, 32 skip dY flush
};

struct TileCoord {
  int slice, jb, ib;
};

#ifdef RBF_TRACE
// Development timeline of CTA 0 (built only with -DRBF_TRACE): per role, events packed as
// (code << 56 | globaltimer).  Read back with rbf_debug_trace().
__device__ unsigned long long g_trace[8][1024];
__device__ int g_trace_n[8];
// Per CTA: [0] start (after setup), [1] end | smid << 48, [2] released by the previous kernel,
// [3] last strip issued | tiles << 48.
__device__ unsigned long long g_cta_span[1024][4];
__device__ __forceinline__ void trace(int role, int code) {
  if (blockIdx.x != 0) return;
  const int n = g_trace_n[role];
  if (n < 1024) {
    g_trace[role][n] = ((unsigned long long)code << 56) | (ptx::globaltimer() & ((1ull << 56) - 1));
    g_trace_n[role] = n + 1;
  }
}
#define TRACE(role, code) trace(role, code)
#else
#define TRACE(role, code) ((void)0)
#endif

// Tile index u -> (feature slice, j-block, i-block).  Order: jsub (the j-block within a group
// of `group` neighbours) fastest, then i-block, then j-group, then slice.  CTAs b with the same
// b / group walk the same i-blocks of `group` neighbouring j-blocks at the same time, so the
// row segments of G and K they read are contiguous over group x 512 bytes in DRAM.
__device__ __forceinline__ TileCoord tile_of(int64_t u, const BwdArgs& a) {
  TileCoord c;
#ifdef RBF_TRACE
  if (a.ablate & 128) {  // row-raster order: j-blocks fastest
    c.jb = (int)(u % a.tiles_j);
    c.ib = (int)((u / a.tiles_j) % a.tiles_i);
    c.slice = (int)(u / ((int64_t)a.tiles_j * a.tiles_i));
    return c;
  }
#endif
  const int jsub = (int)(u % a.group);
  const int64_t r = u / a.group;
  c.ib = (int)(r % a.tiles_i);
  const int64_t r2 = r / a.tiles_i;
  const int jgroups = a.tiles_j / a.group;
  c.jb = (int)(r2 % jgroups) * a.group + jsub;
  c.slice = (int)(r2 / jgroups);
  return c;
}

// Consecutive tiles of one dY segment share the dY accumulator.  Deterministic mode: every
// tile is a segment of its own (its dY partial goes to its own slot).
__device__ __forceinline__ bool same_segment(const TileCoord& p, const TileCoord& q, bool det) {
  return !det && p.slice == q.slice && p.jb == q.jb;
}

// The CTA's tile sequence (its static range, then tiles claimed from the global counter) is
// decided by the strip producer and handed to every other role through a small ring in shared
// memory: entry = tile index (-1 = no more work) + whether the dY segment ends with that tile.
constexpr int SQ = 4;
constexpr int SQ_CONSUMERS = 11;  // warps 1..11
struct SchedRing {
  volatile long long* tile;
  volatile int* seg_end;
  uint64_t* full;
  uint64_t* empty;
  int slot;
  uint32_t ph;
};

__device__ __forceinline__ bool sched_pop(SchedRing& r, bool whole_warp, const BwdArgs& a,
                                          int64_t& t, bool& seg_end) {
  if (!ptx::mbar_wait_bounded(&r.full[r.slot], r.ph, a.status, a.timeout_ns)) return false;
  t = r.tile[r.slot];
  seg_end = r.seg_end[r.slot] != 0;
  if (whole_warp) __syncwarp();
  if (!whole_warp || (threadIdx.x & 31) == 0) ptx::mbar_arrive(&r.empty[r.slot]);
  if (++r.slot == SQ) {
    r.slot = 0;
    r.ph ^= 1;
  }
  return true;
}

// Per-buffer mbarrier parities packed into one register (bit k = buffer k), so that indexing by
// a run-time buffer number does not put a small array in local memory.
__device__ __forceinline__ uint32_t bit_of(uint32_t bits, int k) { return (bits >> k) & 1u; }

__device__ __forceinline__ void red_add4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

__device__ __forceinline__ void red_add1(float* p, float a) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(a) : "memory");
}

// out[r, d0 + e] += c * (s * src[r, d0 + e] - acc[e]) for e < DS, d0 + e < D.
// out[r, d0..] += c * (s * src[r, d0..] - acc); SUM = false: out += -c * acc (src not read).
template <int DS, bool SUM = true>
__device__ __forceinline__ void flush_row(float* out, const float* src, int64_t r, int64_t D,
                                          int d0, float c, float s, const uint32_t* acc) {
  float* o = out + r * D + d0;
  const float* x = src + r * D + d0;
  const int n = (D - d0) < DS ? (int)(D - d0) : DS;
  if (!SUM) {
    if (n == DS && (D & 3) == 0) {
#pragma unroll
      for (int e = 0; e < DS; e += 4)
        red_add4(o + e, -c * __uint_as_float(acc[e]), -c * __uint_as_float(acc[e + 1]),
                 -c * __uint_as_float(acc[e + 2]), -c * __uint_as_float(acc[e + 3]));
    } else {
#pragma unroll
      for (int e = 0; e < DS; ++e)
        if (e < n) red_add1(o + e, -c * __uint_as_float(acc[e]));
    }
    return;
  }
  if (n == DS && (D & 3) == 0) {
#pragma unroll
    for (int e = 0; e < DS; e += 4) {
      const float4 xv = __ldg(reinterpret_cast<const float4*>(x + e));
      red_add4(o + e, c * fmaf(s, xv.x, -__uint_as_float(acc[e])),
               c * fmaf(s, xv.y, -__uint_as_float(acc[e + 1])),
               c * fmaf(s, xv.z, -__uint_as_float(acc[e + 2])),
               c * fmaf(s, xv.w, -__uint_as_float(acc[e + 3])));
    }
  } else {
#pragma unroll
    for (int e = 0; e < DS; ++e)
      if (e < n) red_add1(o + e, c * fmaf(s, __ldg(x + e), -__uint_as_float(acc[e])));
  }
}

// Deterministic mode: out[r, d0 + e] = scale * acc[e] for e < DS, d0 + e < D (plain stores).
template <int DS>
__device__ __forceinline__ void store_row(float* out, int64_t r, int64_t D, int d0, float scale,
                                          const uint32_t* acc) {
  float* o = out + r * D + d0;
  const int n = (D - d0) < DS ? (int)(D - d0) : DS;
  if (n == DS && (D & 3) == 0) {
#pragma unroll
    for (int e = 0; e < DS; e += 4)
      *reinterpret_cast<float4*>(o + e) =
          make_float4(scale * __uint_as_float(acc[e]), scale * __uint_as_float(acc[e + 1]),
                      scale * __uint_as_float(acc[e + 2]), scale * __uint_as_float(acc[e + 3]));
  } else {
#pragma unroll
    for (int e = 0; e < DS; ++e)
      if (e < n) o[e] = scale * __uint_as_float(acc[e]);
  }
}

// Load DS accumulator columns of this thread's TMEM lane.
template <int DS>
__device__ __forceinline__ void tmem_load_row(uint32_t taddr, uint32_t (&v)[64]) {
  uint32_t (&v0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&v[0]);
  ptx::tmem_ld32(taddr, v0);
  if (DS == 64) {
    uint32_t (&v1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&v[32]);
    ptx::tmem_ld32(taddr + 32, v1);
  }
  ptx::tmem_wait_ld();
}

// Store N (8, 16 or 32) consecutive TMEM columns of this thread's lane.
template <int N>
__device__ __forceinline__ void tmem_st_n(uint32_t taddr, const uint32_t* r) {
  if (N == 8) ptx::tmem_st8(taddr, r);
  else if (N == 16) ptx::tmem_st16(taddr, r);
  else ptx::tmem_st32(taddr, *reinterpret_cast<const uint32_t(*)[32]>(r));
}

#ifndef RBF_CB
#define RBF_CB 8
#endif
constexpr int CB = RBF_CB;  // rows of W^T a C-warp converts per TMEM store (code size vs. batching)

template <int DS, bool DOT = false, bool DET = false>
__global__ void __launch_bounds__(THREADS, 1)
    rbf_bwd_tc_kernel(const __grid_constant__ CUtensorMap tm_g,
                      const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_xhi,
                      const __grid_constant__ CUtensorMap tm_xlo,
                      const __grid_constant__ CUtensorMap tm_yhi,
                      const __grid_constant__ CUtensorMap tm_ylo,
                      const __grid_constant__ CUtensorMap tm_dx, const BwdArgs a) {
  using C = Cfg<DS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* ring = smem;                                 // [STAGES][G strip | K strip]
  uint8_t* xring = ring + STAGES * 2 * STRIP;           // [XSTAGES][X hi | X lo]
  uint8_t* yring = xring + XSTAGES * 2 * C::X_BYTES;    // [YSTAGES][Y hi | Y lo]
  uint8_t* staging = yring + YSTAGES * 2 * C::X_BYTES;  // [4 R-warps][32 rows x DS]
  uint64_t* bar = reinterpret_cast<uint64_t*>(staging + (kStageDx ? 4 : 0) * C::STAGING);
  uint64_t* full = bar;              // [4] strip landed            TMA -> R-warps, C-warp
  uint64_t* empty = full + 4;        // [4] strip consumed          R-warps, C-warp -> TMA
  uint64_t* xfull = empty + 4;       // [XSTAGES] X rows landed     TMA -> dY issuer
  uint64_t* xempty = xfull + XSTAGES;  // [XSTAGES] X rows consumed dY issuer -> TMA
  uint64_t* yfull = xempty + XSTAGES;  // [2] Y rows landed         TMA -> dX issuer
  uint64_t* yempty = yfull + 2;      // [2] Y rows consumed         dX issuer -> TMA
  uint64_t* w_full = yempty + 2;     // [2] W buffer written        R-warps -> dX issuer
  uint64_t* w_empty = w_full + 2;    // [2] W buffer read           dX issuer -> R-warps
  uint64_t* wt_full = w_empty + 2;   // [2] W^T half written        C-warps -> dY issuer
  uint64_t* wt_empty = wt_full + 2;  // [2] W^T half read           dY issuer -> C-warps
  uint64_t* dx_full = wt_empty + 2;  // dX accumulator complete     dX issuer -> R-warps
  uint64_t* dx_empty = dx_full + 1;  // dX accumulator drained      R-warps -> dX issuer
  uint64_t* dy_full = dx_empty + 1;  // dY accumulator complete     dY issuer -> C-warps
  uint64_t* dy_empty = dy_full + 1;  // dY accumulator drained      C-warps -> dY issuer
  uint64_t* drain = dy_empty + 1;    // teardown of both issuers
  uint64_t* sq_full = drain + 1;     // [SQ] tile entry written   producer -> every role
  uint64_t* sq_empty = sq_full + SQ; // [SQ] tile entry read      every role -> producer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sq_empty + SQ);
  long long* sq_tile = reinterpret_cast<long long*>(sq_empty + SQ + 1);
  int* sq_seg_end = reinterpret_cast<int*>(sq_tile + SQ);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < 4; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 5);  // 4 R-warps + the C-warp of this quadrant
    }
    for (int s = 0; s < XSTAGES; ++s) {
      ptx::mbar_init(&xfull[s], 1);
      ptx::mbar_init(&xempty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      ptx::mbar_init(&yfull[s], 1);
      ptx::mbar_init(&yempty[s], 1);
      ptx::mbar_init(&w_full[s], 4);
      ptx::mbar_init(&w_empty[s], 1);
      ptx::mbar_init(&wt_full[s], 4);
      ptx::mbar_init(&wt_empty[s], 1);
    }
    ptx::mbar_init(dx_full, 1);
    ptx::mbar_init(dx_empty, 4);
    ptx::mbar_init(dy_full, 1);
    ptx::mbar_init(dy_empty, 4);
    ptx::mbar_init(drain, 2);  // one commit per MMA issuer
    for (int s = 0; s < SQ; ++s) {
      ptx::mbar_init(&sq_full[s], 1);
      ptx::mbar_init(&sq_empty[s], SQ_CONSUMERS);
    }
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tensormap(&tm_g);
    if (!DOT) ptx::prefetch_tensormap(&tm_k);
    ptx::prefetch_tensormap(&tm_yhi);
    ptx::prefetch_tensormap(&tm_ylo);
    if (a.tma_flush) ptx::prefetch_tensormap(&tm_dx);
  }
  if (warp == 1 && lane == 0) {
    ptx::prefetch_tensormap(&tm_xhi);
    ptx::prefetch_tensormap(&tm_xlo);
  }
  if (warp == 2) {
    ptx::tmem_alloc(tmem_slot, TMEM_COLS);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
#ifdef RBF_TRACE
  if (threadIdx.x == 0 && blockIdx.x < 1024) g_cta_span[blockIdx.x][0] = ptx::globaltimer() & ((1ull << 48) - 1);
#endif
  ptx::griddep_wait();  // outputs zeroed and the workspace written by the previous kernels
#ifdef RBF_TRACE
  if (threadIdx.x == 0 && blockIdx.x < 1024) g_cta_span[blockIdx.x][2] = ptx::globaltimer() & ((1ull << 48) - 1);
#endif

  SchedRing sq = {sq_tile, sq_seg_end, sq_full, sq_empty, 0, 0};

  if (warp == 0) {
    if (lane == 0) {
      // ============================================================ strips of G, K + Y rows
      const uint64_t stream = ptx::policy_evict_first();
      const uint64_t keep = ptx::policy_evict_last();
      uint32_t ph = 0;  // strip stage parity: flips once per tile
      int yst = 0;
      uint32_t yph = 0;
      uint32_t issued = 0, last = 0;  // strip stages with a load in flight and their parities
      uint32_t yissued = 0, ylast = 0;
      bool ok = true, skipped = false;
      // Tile sequence: a contiguous static range (the dY accumulator stays in TMEM across a
      // segment), then tiles claimed one at a time, so CTAs that run fast take more of the tail.
      const int64_t jsub = blockIdx.x % a.group, sub = blockIdx.x / a.group;
      const int64_t subs = gridDim.x / a.group;
      int64_t s_next = a.static_rows * sub / subs;
      const int64_t s_end = a.static_rows * (sub + 1) / subs;
      const int64_t dyn_base = a.static_rows * a.group;
      bool exhausted = false;
      auto fetch = [&]() -> int64_t {
        if (s_next < s_end) return (s_next++) * a.group + jsub;
        if (exhausted || dyn_base >= a.total_tiles) return -1;
        const int64_t t = dyn_base + (int64_t)atomicAdd(a.counter, 1);
        if (t >= a.total_tiles) {
          exhausted = true;
          return -1;
        }
        return t;
      };
      int pslot = 0;
      uint32_t pph = 0;
      auto publish = [&](int64_t t, bool seg_end) -> bool {
        if (!ptx::mbar_wait_bounded(&sq_empty[pslot], pph ^ 1, a.status, a.timeout_ns)) return false;
        sq_tile[pslot] = t;
        sq_seg_end[pslot] = seg_end ? 1 : 0;
        ptx::mbar_arrive(&sq_full[pslot]);
        if (++pslot == SQ) {
          pslot = 0;
          pph ^= 1;
        }
        return true;
      };
      // Two cursors, each issued as soon as its own ring has room: the G/K strips (stage s of
      // every tile, freed by the R-warps and C-warp s) and the Y rows of each strip (2-deep
      // ring, freed by the dX MMAs).  Issuing them in one blocking sequence would hold strip
      // s+2 of a tile behind the dX MMAs of strip s.  Tile k's coordinates sit in slot k & 1;
      // the Y cursor lags the strip cursor by at most one tile.
      TileCoord slot0 = {0, 0, 0}, slot1 = {0, 0, 0};
      uint32_t n_strips = 0, n_ys = 0;  // strips / Y loads issued so far
      int ss = 4;                       // next strip of the current tile (4 = start a new tile)
      int64_t t = fetch(), nxt = -1;
      bool strips_done = t < 0;
      int i0 = 0, j0 = 0;
      uint64_t idle_since = ptx::globaltimer();
      while (ok) {
        bool progressed = false;
        if (!strips_done && ss == 4 && n_ys + 4 >= n_strips) {
          const TileCoord tc = tile_of(t, a);
          nxt = fetch();
          if (!publish(t, nxt < 0 || !same_segment(tile_of(nxt, a), tc, DET))) { ok = false; break; }
          if ((n_strips >> 2) & 1u) slot1 = tc; else slot0 = tc;
          i0 = tc.ib * BT;
          j0 = tc.jb * BT;
          ss = 0;
        }
        if (!strips_done && ss < 4 && ptx::mbar_test_wait(&empty[ss], ph ^ 1)) {
          TRACE(0, 10 + ss);
          if (a.debug_skip_first_load && !skipped && blockIdx.x == 0) {
            skipped = true;  // test hook: this strip never arrives, its consumers time out
          } else {
            uint8_t* sm = ring + ss * 2 * STRIP;
            ptx::mbar_arrive_expect_tx(&full[ss], DOT ? STRIP : 2 * STRIP);
            ptx::tma_load_2d_hint(sm, &tm_g, j0 + SR * ss, i0, &full[ss], stream);
            if (!DOT) ptx::tma_load_2d_hint(sm + STRIP, &tm_k, j0 + SR * ss, i0, &full[ss], stream);
            issued |= 1u << ss;
            last = (last & ~(1u << ss)) | (ph << ss);
          }
          ++n_strips;
          if (++ss == 4) {
            ph ^= 1;
            t = nxt;
            strips_done = t < 0;
          }
          progressed = true;
        }
        if (n_ys < n_strips && ptx::mbar_test_wait(&yempty[yst], yph ^ 1)) {
          const TileCoord ty = ((n_ys >> 2) & 1u) ? slot1 : slot0;
          const int sy = (int)(n_ys & 3u);
          uint8_t* ym = yring + yst * 2 * C::X_BYTES;
#ifdef RBF_TRACE
          if (a.ablate & 64) {
            ptx::mbar_arrive(&yfull[yst]);
          } else
#endif
          {
            ptx::mbar_arrive_expect_tx(&yfull[yst], 2 * C::X_BYTES);
#pragma unroll
            for (int b = 0; b < DS / 32; ++b) {
              ptx::tma_load_2d_hint(ym + b * BOX, &tm_yhi, ty.slice * DS + 32 * b,
                                    ty.jb * BT + SR * sy, &yfull[yst], keep);
              ptx::tma_load_2d_hint(ym + C::X_BYTES + b * BOX, &tm_ylo, ty.slice * DS + 32 * b,
                                    ty.jb * BT + SR * sy, &yfull[yst], keep);
            }
            yissued |= 1u << yst;
            ylast = (ylast & ~(1u << yst)) | (yph << yst);
          }
          if (++yst == YSTAGES) { yst = 0; yph ^= 1; }
          ++n_ys;
          progressed = true;
        }
        if (strips_done && n_ys == n_strips) break;
        if (progressed) {
          idle_since = ptx::globaltimer();
        } else {
          if (ptx::globaltimer() - idle_since > a.timeout_ns) {
            atomicExch(a.status, RBF_ERR_TIMEOUT);
            ok = false;
            break;
          }
          __nanosleep(32);  // neither ring has room: leave the issue slots to the other warps
        }
      }
#ifdef RBF_TRACE
      if (blockIdx.x < 1024)
        g_cta_span[blockIdx.x][3] = (ptx::globaltimer() & ((1ull << 48) - 1)) | ((unsigned long long)(n_strips / 4) << 48);
#endif
      if (ok && !publish(-1, true)) ok = false;
      if (!ok) {  // let every copy this thread issued land before the CTA exits
        for (int s = 0; s < 4; ++s)
          if (issued >> s & 1u) ptx::mbar_wait_bounded(&full[s], bit_of(last, s), a.status, a.timeout_ns);
        for (int s = 0; s < 2; ++s)
          if (yissued >> s & 1u) ptx::mbar_wait_bounded(&yfull[s], bit_of(ylast, s), a.status, a.timeout_ns);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ============================================================ X rows, four chunks per tile
      const uint64_t keep = ptx::policy_evict_last();
      int xst = 0;
      uint32_t xph = 0;
      uint32_t xissued = 0, xlast = 0;
      bool ok = true;
      while (ok) {
        int64_t t;
        bool seg_end;
        if (!sched_pop(sq, false, a, t, seg_end)) { ok = false; break; }
        if (t < 0) break;
        const TileCoord tc = tile_of(t, a);
        const int i0 = tc.ib * BT, d0 = tc.slice * DS;
        for (int s = 0; s < 4; ++s) {
          if (!ptx::mbar_wait_bounded(&xempty[xst], xph ^ 1, a.status, a.timeout_ns)) { ok = false; break; }
          uint8_t* xm = xring + xst * 2 * C::X_BYTES;
#ifdef RBF_TRACE
          if (a.ablate & 64) {
            ptx::mbar_arrive(&xfull[xst]);
            if (++xst == XSTAGES) { xst = 0; xph ^= 1; }
            continue;
          }
#endif
          ptx::mbar_arrive_expect_tx(&xfull[xst], 2 * C::X_BYTES);
#pragma unroll
          for (int b = 0; b < DS / 32; ++b) {
            ptx::tma_load_2d_hint(xm + b * BOX, &tm_xhi, d0 + 32 * b, i0 + SR * s, &xfull[xst], keep);
            ptx::tma_load_2d_hint(xm + C::X_BYTES + b * BOX, &tm_xlo, d0 + 32 * b, i0 + SR * s,
                                  &xfull[xst], keep);
          }
          xissued |= 1u << xst;
          xlast = (xlast & ~(1u << xst)) | (xph << xst);
          if (++xst == XSTAGES) { xst = 0; xph ^= 1; }
        }
      }
      if (!ok)
        for (int s = 0; s < XSTAGES; ++s)
          if (xissued >> s & 1u) ptx::mbar_wait_bounded(&xfull[s], bit_of(xlast, s), a.status, a.timeout_ns);
    }
  } else if (warp == 2 || warp == 3) {
    // ================================================================ MMA issuers
    constexpr uint32_t idesc = ptx::idesc_tf32(128, DS, 0, 1);
    constexpr uint32_t idesc2 = ptx::idesc_tf32(128, 2 * DS, 0, 1);  // B = [X_hi | X_lo]
    if (warp == 2 && lane == 0) {
      // ---- dY: once per tile, A = W^T (TMEM lanes j, K = 128 rows i), B = X rows in 4 chunks.
      int xs = 0;
      uint32_t xph = 0, dye_ph = 0;
      uint32_t wt_ph = 0;  // parity bits of wt_full[0..1]
      bool ok = true, dy_first = true;
      TileCoord cur = {-1, -1, -1};
      while (ok) {
        int64_t t;
        bool seg_end;
        if (!sched_pop(sq, false, a, t, seg_end)) { ok = false; break; }
        if (t < 0) break;
        const TileCoord tc = tile_of(t, a);
        if (!same_segment(tc, cur, DET)) {
          cur = tc;
          // The C-warps drained the dY accumulator of the previous segment.
          if (!ptx::mbar_wait_bounded(dy_empty, dye_ph ^ 1, a.status, a.timeout_ns)) { ok = false; break; }
          dye_ph ^= 1;
          dy_first = true;
        }
        for (int s = 0; s < 4 && ok; ++s) {
          const int h = s >> 1;  // W^T half: rows 64h .. 64h+63
          if ((s & 1) == 0) {
            if (!ptx::mbar_wait_bounded(&wt_full[h], bit_of(wt_ph, h), a.status, a.timeout_ns)) { ok = false; break; }
            TRACE(2, 10 + h);
            wt_ph ^= 1u << h;
          }
          if (!ptx::mbar_wait_bounded(&xfull[xs], xph, a.status, a.timeout_ns)) { ok = false; break; }
          TRACE(2, 20 + s);
          ptx::tc_fence_after();
          const uint32_t xb = ptx::smem_u32(xring + xs * 2 * C::X_BYTES);
          const uint32_t at = tmem + COL_WT + SR * s;
#pragma unroll
          for (int k = 0; k < SR / 8; ++k) {
            const uint64_t bh = ptx::smem_desc(xb + 1024 * k, BOX, MN_SBO, MN_LAYOUT);
#ifdef RBF_TRACE
            if (a.ablate & 16) continue;
#endif
            if constexpr (kStackDy<DS>) {
              // W^T_hi . [X_hi | X_lo] (N = 2 DS: the ring entry holds hi then lo at a uniform
              // atom stride), then W^T_lo . X_hi into the first half.
              ptx::mma_tf32_ts(tmem + COL_DY, at + 8 * k, bh, idesc2, dy_first ? 0u : 1u);
              ptx::mma_tf32_ts(tmem + COL_DY, at + 128 + 8 * k, bh, idesc, 1);
            } else {
              const uint64_t bl = ptx::smem_desc(xb + C::X_BYTES + 1024 * k, BOX, MN_SBO, MN_LAYOUT);
              ptx::mma_tf32_ts(tmem + COL_DY, at + 8 * k, bh, idesc, dy_first ? 0u : 1u);
              ptx::mma_tf32_ts(tmem + COL_DY, at + 8 * k, bl, idesc, 1);
              ptx::mma_tf32_ts(tmem + COL_DY, at + 128 + 8 * k, bh, idesc, 1);
            }
            dy_first = false;
          }
          ptx::mma_commit(&xempty[xs]);
          if (s & 1) ptx::mma_commit(&wt_empty[h]);
          if (++xs == XSTAGES) { xs = 0; xph ^= 1; }
        }
        if (!ok) break;
        if (seg_end) ptx::mma_commit(dy_full);
      }
      ptx::mma_commit(drain);  // every MMA this thread issued must finish before TMEM is freed
      ptx::mbar_wait_bounded(drain, 0, a.status, a.timeout_ns);
    } else if (warp == 3 && lane == 0) {
      // ---- dX: per strip, A = W (TMEM lanes i, K = 32 columns j), B = the strip's Y rows.
      int ys = 0, wb = 0;
      uint32_t yph = 0, dxe_ph = 0;
      uint32_t w_ph = 0;  // parity bits of w_full[0..1]
      bool ok = true;
      while (ok) {
        int64_t t;
        bool seg_end;
        if (!sched_pop(sq, false, a, t, seg_end)) { ok = false; break; }
        if (t < 0) break;
        // The R-warps drained the accumulator of the previous tile.
        if (!ptx::mbar_wait_bounded(dx_empty, dxe_ph ^ 1, a.status, a.timeout_ns)) { ok = false; break; }
        dxe_ph ^= 1;
        for (int s = 0; s < 4 && ok; ++s) {
          if (!ptx::mbar_wait_bounded(&w_full[wb], bit_of(w_ph, wb), a.status, a.timeout_ns) ||
              !ptx::mbar_wait_bounded(&yfull[ys], yph, a.status, a.timeout_ns)) { ok = false; break; }
          w_ph ^= 1u << wb;
          TRACE(3, 20 + s);
          ptx::tc_fence_after();
          const uint32_t aw = tmem + TmemPlan<DS>::W + 64 * wb;
          const uint32_t yb = ptx::smem_u32(yring + ys * 2 * C::X_BYTES);
#pragma unroll
          for (int k = 0; k < SR / 8; ++k) {
            const uint64_t bh = ptx::smem_desc(yb + 1024 * k, BOX, MN_SBO, MN_LAYOUT);
            const uint64_t bl = ptx::smem_desc(yb + C::X_BYTES + 1024 * k, BOX, MN_SBO, MN_LAYOUT);
#ifdef RBF_TRACE
            if (a.ablate & 16) continue;
#endif
            ptx::mma_tf32_ts(tmem + TmemPlan<DS>::DX, aw + 8 * k, bh, idesc, (s | k) != 0 ? 1u : 0u);
            ptx::mma_tf32_ts(tmem + TmemPlan<DS>::DX, aw + 8 * k, bl, idesc, 1);
            ptx::mma_tf32_ts(tmem + TmemPlan<DS>::DX, aw + 32 + 8 * k, bh, idesc, 1);
          }
          ptx::mma_commit(&w_empty[wb]);
          ptx::mma_commit(&yempty[ys]);
          if (++wb == TmemPlan<DS>::WBUFS) wb = 0;
          if (++ys == YSTAGES) { ys = 0; yph ^= 1; }
        }
        if (!ok) break;
        ptx::mma_commit(dx_full);
      }
      ptx::mma_commit(drain);
      ptx::mbar_wait_bounded(drain, 0, a.status, a.timeout_ns);
    }
  } else if (warp < 8) {
    // ================================================================ C-warps (column j)
    // C-warp q reads strip q (its 32 columns, all 128 rows) and writes W^T for them, in two
    // halves of 64 rows so that one half is refilled while the dY MMAs read the other.
    const int q = warp & 3;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    uint32_t ph = 0, dyf_ph = 0;
    uint32_t wte_ph = 0;  // parity bits of wt_empty[0..1]
    float colsum = 0.f;
    TileCoord cur = {-1, -1, -1};
    bool ok = true;
    // This step's slot of the routed dY buffer (fixed for the launch), picked with constant
    // indices so that the pointer array stays out of local memory.
    float* route_dst = nullptr;
    if (a.route.world > 0) {
      route_dst = a.route.bufs[0];
#pragma unroll
      for (int r = 1; r < kMaxRanks; ++r)
        if (a.route.rank == r) route_dst = a.route.bufs[r];
      route_dst += (int64_t)((*a.route.ctr) % kDySlots) * a.M * a.D;
    }
    // Byte offset of this lane's column inside a 128-byte swizzled row, for row % 8 = r.
    uint32_t coff[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) coff[r] = (((lane >> 2) ^ r) << 4) + (lane & 3) * 4;
    for (; ok; ph ^= 1) {
      int64_t t;
      bool seg_end;
      if (!sched_pop(sq, true, a, t, seg_end)) { ok = false; break; }
      if (t < 0) break;
      const TileCoord tc = tile_of(t, a);
      if (!same_segment(tc, cur, DET)) {
        cur = tc;
        colsum = 0.f;
      }
      if (!ptx::mbar_wait_bounded(&full[q], ph, a.status, a.timeout_ns)) { ok = false; break; }
      if (lane == 0 && (q == 0 || q == 3)) TRACE(q == 0 ? 4 : 6, 10);
      const uint8_t* gb = ring + q * 2 * STRIP;
      const uint8_t* kb = gb + STRIP;
#pragma unroll 1
      for (int h = 0; h < 2 && ok; ++h) {
        // This half of the W^T tile was read by the previous tile's dY MMAs.
        if (!ptx::mbar_wait_bounded(&wt_empty[h], bit_of(wte_ph, h) ^ 1, a.status, a.timeout_ns)) { ok = false; break; }
        wte_ph ^= 1u << h;
        if (lane == 0 && q == 0) TRACE(4, 20 + h);
        ptx::tc_fence_after();
#pragma unroll 1
        for (int r0 = 64 * h; r0 < 64 * h + 64; r0 += CB) {
#ifdef RBF_TRACE
          if (a.ablate & 4) break;
#endif
          uint32_t hi[CB], lo[CB];
#pragma unroll
          for (int r = 0; r < CB; ++r) {
            const uint32_t off = (uint32_t)(r0 + r) * 128 + coff[r & 7];
            float w = *reinterpret_cast<const float*>(gb + off);
            if (!DOT) {
              w *= *reinterpret_cast<const float*>(kb + off);
              colsum += w;
            }
            float hh, ll;
            tf32_split(w, hh, ll);
            hi[r] = __float_as_uint(hh);
            lo[r] = __float_as_uint(ll);
          }
          tmem_st_n<CB>(tmem + lane_base + COL_WT + r0, hi);
          tmem_st_n<CB>(tmem + lane_base + COL_WT + 128 + r0, lo);
        }
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&wt_full[h]);
        if (lane == 0 && q == 0) TRACE(4, 30 + h);
      }
      if (!ok) break;
      // The stage is refilled by TMA (async proxy) after this release; the warp's reads of it
      // (generic proxy) must be ordered before that write by a proxy fence, or the refill can
      // overwrite data a lane has not read yet (measured: wrong dX tiles, a few in 100 runs).
      ptx::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&empty[q]);
      if (lane == 0 && (q == 0 || q == 3)) TRACE(q == 0 ? 4 : 6, 40);
      if (seg_end) {
        if (!ptx::mbar_wait_bounded(dy_full, dyf_ph, a.status, a.timeout_ns)) { ok = false; break; }
        dyf_ph ^= 1;
        ptx::tc_fence_after();
        uint32_t accv[64];
        tmem_load_row<DS>(tmem + lane_base + COL_DY, accv);
#pragma unroll
        for (int c = 0; c < (kStackDy<DS> ? DS / 32 : 0); ++c) {  // + the W_hi.X_lo half
          uint32_t lo_part[32];
          ptx::tmem_ld32(tmem + lane_base + COL_DY + DS + 32 * c, lo_part);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e)
            accv[32 * c + e] = __float_as_uint(__uint_as_float(accv[32 * c + e]) +
                                               __uint_as_float(lo_part[e]));
        }
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(dy_empty);
        const int64_t j = (int64_t)tc.jb * BT + q * 32 + lane;
#ifdef RBF_TRACE
        if (a.ablate & 32) continue;
#endif
        if constexpr (DET) {
          if (j < a.M) {
            const int64_t slot = (int64_t)tc.ib * a.M + j;
            store_row<DS>(a.dyp, slot, a.D, tc.slice * DS, -a.c, accv);
            if (!DOT && tc.slice == 0) a.csp[slot] = colsum;
          }
        } else {
          float* dst = a.route.world > 0 ? route_dst : a.dY;
          if (j < a.M) flush_row<DS, !DOT>(dst, a.Y, j, a.D, tc.slice * DS, a.c, colsum, accv);
        }
        if (lane == 0 && q == 0) TRACE(4, 50);
      }
    }
  } else {
    // ================================================================ R-warps (row i)
    // Tile t's dX accumulator is drained and flushed right after the first strip of tile t+1
    // is handed over, so the flush never stalls the conversion -> MMA chain for long.
    const int q = warp & 3;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    int wb = 0;
    uint32_t ph = 0, dxf_ph = 0;
    uint32_t we_ph = 0;  // parity bits of w_empty[0..1]
    bool ok = true, pending = false;
    float prev_rowsum = 0.f;
    int64_t prev_i = 0;
    int prev_d0 = 0, prev_jb = 0;
    auto flush_prev = [&]() -> bool {
      if (!ptx::mbar_wait_bounded(dx_full, dxf_ph, a.status, a.timeout_ns)) return false;
      dxf_ph ^= 1;
      ptx::tc_fence_after();
      uint32_t accv[64];
      tmem_load_row<DS>(tmem + lane_base + TmemPlan<DS>::DX, accv);
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(dx_empty);
      // Deterministic mode: this tile's partial goes to row slot_row of its j-block's slot.
      const int64_t slot_row = DET ? (int64_t)prev_jb * a.Npad + prev_i : 0;
      if constexpr (DET) {
        if (!DOT && prev_i < a.N && prev_d0 == 0) a.rsp[slot_row] = prev_rowsum;
        if (!a.tma_flush) {
          if (prev_i < a.N) store_row<DS>(a.dxp, slot_row, a.D, prev_d0, -a.c, accv);
          return true;
        }
      }
      if (!DET && !a.tma_flush) {
        if (prev_i < a.N) flush_row<DS, !DOT>(a.dX, a.X, prev_i, a.D, prev_d0, a.c, prev_rowsum, accv);
        return true;
      }
      // -c * acc goes through shared memory to a TMA reduce-add (32 rows x DS, coalesced in L2);
      // c * rowsum * x is added once per row by the finalize pass from the rowsum vector.
      if (!DET && !DOT && prev_i < a.N && prev_d0 == 0 && !(a.ablate & 2))
        red_add1(a.rowsum + prev_i, prev_rowsum);
      uint8_t* stg = staging + q * C::STAGING;
      if (lane == 0) ptx::bulk_wait_read<0>();  // the previous reduce has read the buffer
      __syncwarp();
#pragma unroll
      for (int bx = 0; bx < DS / 32; ++bx) {
        uint8_t* row = stg + bx * BOX + lane * 128;
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4) {
          const uint32_t* v = accv + 32 * bx + 4 * c4;
          *reinterpret_cast<float4*>(row + ((c4 ^ (lane & 7)) << 4)) =
              make_float4(-a.c * __uint_as_float(v[0]), -a.c * __uint_as_float(v[1]),
                          -a.c * __uint_as_float(v[2]), -a.c * __uint_as_float(v[3]));
        }
      }
      ptx::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && !(a.ablate & 1)) {
#pragma unroll
        for (int bx = 0; bx < DS / 32; ++bx) {
          if constexpr (DET)
            ptx::tma_store_2d(&tm_dx, stg + bx * BOX, prev_d0 + 32 * bx, (int)slot_row);
          else
            ptx::tma_reduce_add_2d(&tm_dx, stg + bx * BOX, prev_d0 + 32 * bx, (int)prev_i);
        }
        ptx::bulk_commit();
      }
      return true;
    };
    for (; ok; ph ^= 1) {
      int64_t t;
      bool seg_end;
      if (!sched_pop(sq, true, a, t, seg_end)) { ok = false; break; }
      if (t < 0) break;
      const TileCoord tc = tile_of(t, a);
      float rowsum = 0.f;
      for (int s = 0; s < 4; ++s) {
        if (!ptx::mbar_wait_bounded(&full[s], ph, a.status, a.timeout_ns)) { ok = false; break; }
        if (lane == 0 && (q == 0 || q == 3)) TRACE(q == 0 ? 5 : 7, 10 + s);
        // Row (32q + lane) of strip s: its 32 columns in 128 swizzled bytes.
        const uint8_t* gb = ring + s * 2 * STRIP + (q * 32 + lane) * 128;
        const uint8_t* kb = gb + STRIP;
        uint32_t hi[32], lo[32];
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4) {
#ifdef RBF_TRACE
          if (a.ablate & 8) { hi[4 * c4] = hi[4 * c4 + 1] = hi[4 * c4 + 2] = hi[4 * c4 + 3] = 0u; lo[4 * c4] = lo[4 * c4 + 1] = lo[4 * c4 + 2] = lo[4 * c4 + 3] = 0u; continue; }
#endif
          const int off = (c4 ^ (lane & 7)) << 4;
          const float4 g = *reinterpret_cast<const float4*>(gb + off);
          float w[4] = {g.x, g.y, g.z, g.w};
          if (!DOT) {
            const float4 k = *reinterpret_cast<const float4*>(kb + off);
            w[0] *= k.x; w[1] *= k.y; w[2] *= k.z; w[3] *= k.w;
          }
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            if (!DOT) rowsum += w[e];
            float h, l;
            tf32_split(w[e], h, l);
            hi[4 * c4 + e] = __float_as_uint(h);
            lo[4 * c4 + e] = __float_as_uint(l);
          }
        }
        ptx::fence_proxy_async_smem();  // generic reads before the TMA refill (see C-warps)
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&empty[s]);
        if (!ptx::mbar_wait_bounded(&w_empty[wb], bit_of(we_ph, wb) ^ 1, a.status, a.timeout_ns)) { ok = false; break; }
        we_ph ^= 1u << wb;
        if (lane == 0 && q == 0) TRACE(5, 20 + s);
        ptx::tc_fence_after();
#ifdef RBF_TRACE
        if (!(a.ablate & 8)) {
#endif
        ptx::tmem_st32(tmem + lane_base + TmemPlan<DS>::W + 64 * wb, hi);
        ptx::tmem_st32(tmem + lane_base + TmemPlan<DS>::W + 64 * wb + 32, lo);
        ptx::tmem_wait_st();
#ifdef RBF_TRACE
        }
#endif
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&w_full[wb]);
        if (lane == 0 && q == 0) TRACE(5, 30 + s);
        if (++wb == TmemPlan<DS>::WBUFS) wb = 0;
        if (s == 0 && pending) {
          if (!flush_prev()) { ok = false; break; }
          pending = false;
          if (lane == 0 && q == 0) TRACE(5, 40);
        }
      }
      if (!ok) break;
      pending = true;
      prev_rowsum = rowsum;
      prev_i = (int64_t)tc.ib * BT + q * 32 + lane;
      prev_d0 = tc.slice * DS;
      prev_jb = tc.jb;
    }
    if (ok && pending) flush_prev();
    if (lane == 0) ptx::bulk_wait<0>();  // reduces complete before the CTA exits
  }

  ptx::griddep_launch_dependents();
  ptx::tc_fence_before();
  __syncthreads();
#ifdef RBF_TRACE
  if (threadIdx.x == 0 && blockIdx.x < 1024) {
    uint32_t smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    g_cta_span[blockIdx.x][1] = (ptx::globaltimer() & ((1ull << 48) - 1)) | ((unsigned long long)smid << 48);
  }
#endif
  if (warp == 2) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, TMEM_COLS);
  }
}

// dX[i,:] += c * rowsum[i] * X[i,:]: the part of every tile's dX flush that the TMA reduce
// leaves out (one pass over dX instead of one per tile).  One thread per 4 features.
__global__ void __launch_bounds__(256) rbf_bwd_finalize_kernel(const float* __restrict__ X,
                                                               const float* __restrict__ rowsum,
                                                               float* __restrict__ dX, int64_t N,
                                                               int64_t D, float c) {
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  const int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // float4 index
  const int64_t per_row = D / 4;
  if (q >= N * per_row) return;
  const int64_t i = q / per_row;
  const float s = c * rowsum[i];
  const float4 x = __ldg(reinterpret_cast<const float4*>(X) + q);
  float4 v = reinterpret_cast<float4*>(dX)[q];
  v.x = fmaf(s, x.x, v.x);
  v.y = fmaf(s, x.y, v.y);
  v.z = fmaf(s, x.z, v.z);
  v.w = fmaf(s, x.w, v.w);
  reinterpret_cast<float4*>(dX)[q] = v;
}

// Zeroes the three accumulation targets of the backward (dX, dY, the rowsum vector) in one
// launch, so the stream stays a chain of kernels that programmatic dependent launch can overlap.
__global__ void __launch_bounds__(256) rbf_bwd_zero_kernel(float* __restrict__ a, int64_t na,
                                                           float* __restrict__ b, int64_t nb,
                                                           float* __restrict__ c, int64_t nc,
                                                           const int* __restrict__ slot_ctr) {
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  // Routed dY: b is slot 0 of this rank's buffer and the step counter picks the slot.
  if (slot_ctr != nullptr) b += (int64_t)(*slot_ctr % kDySlots) * nb;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < na + nb + nc; k += stride) {
    if (k < na) a[k] = 0.f;
    else if (k < na + nb) b[k - na] = 0.f;
    else c[k - na - nb] = 0.f;
  }
}

// Deterministic mode: dX[i,:] = the tiles' -c * (W Y) partials summed over j-blocks in order,
// + c * (their row sums, in order) * x_i; dY likewise over i-blocks.  One thread per output
// element, so every sum has one fixed order.  sums = 0 (cosine case): the partials only.
__global__ void __launch_bounds__(256) rbf_bwd_det_finalize_kernel(
    const float* __restrict__ X, const float* __restrict__ Y, const float* __restrict__ dxp,
    const float* __restrict__ rsp, const float* __restrict__ dyp, const float* __restrict__ csp,
    float* __restrict__ dX, float* __restrict__ dY, int64_t N, int64_t M, int64_t D, int64_t Npad,
    int tiles_j, int tiles_i, float c, int sums) {
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < (N + M) * D; k += stride) {
    if (k < N * D) {
      const int64_t i = k / D, d = k - i * D;
      float acc = 0.f, rs = 0.f;
      for (int jb = 0; jb < tiles_j; ++jb) {
        acc += dxp[((int64_t)jb * Npad + i) * D + d];
        if (sums) rs += rsp[(int64_t)jb * Npad + i];
      }
      dX[k] = sums ? fmaf(c * rs, X[k], acc) : acc;
    } else {
      const int64_t k2 = k - N * D, j = k2 / D, d = k2 - j * D;
      float acc = 0.f, cs = 0.f;
      for (int ib = 0; ib < tiles_i; ++ib) {
        acc += dyp[((int64_t)ib * M + j) * D + d];
        if (sums) cs += csp[(int64_t)ib * M + j];
      }
      dY[k2] = sums ? fmaf(c * cs, Y[k2], acc) : acc;
    }
  }
}

}  // namespace

// Scratch after the split-pass layout: the rowsum vector [N] and the tile counter; in
// deterministic mode, then the per-tile partial slots.
static int64_t rowsum_bytes(int64_t N) { return round_up((int64_t)sizeof(float) * N, (int64_t)kAlign); }

struct DetLayout {
  size_t dxp, rsp, dyp, csp, end;  // byte offsets after the split-pass layout
  int64_t Npad;
};

static DetLayout det_layout(int64_t N, int64_t M, int64_t D) {
  DetLayout d;
  const int64_t tj = ceil_div(M, BT), ti = ceil_div(N, BT);
  d.Npad = round_up(N, (int64_t)BT);
  size_t off = (size_t)(rowsum_bytes(N) + kAlign);
  auto take = [&](int64_t bytes) {
    const size_t o = off;
    off = (size_t)round_up((int64_t)off + bytes, (int64_t)kAlign);
    return o;
  };
  d.dxp = take(4 * tj * d.Npad * D);
  d.rsp = take(4 * tj * d.Npad);
  d.dyp = take(4 * ti * M * D);
  d.csp = take(4 * ti * M);
  d.end = off;
  return d;
}

size_t backward_scratch_bytes(int64_t N, int64_t M, int64_t D) {
  if (deterministic_backward() && N > 0 && M > 0 && D > 0 && (M % 4) == 0)
    return det_layout(N, M, D).end;
  return (size_t)(rowsum_bytes(N) + kAlign);
}

ZeroSpec backward_zero_spec(int64_t N, int64_t M, int64_t D, void* ws, float* dX, float* dY,
                            const WaitConfig& wc) {
  ZeroSpec z;
  const PrepLayout L = prep_layout(N, M, D);
  const bool work = N > 0 && M > 0 && D > 0;
  const bool tma_flush = kStageDx && (D % 4) == 0;
  float* rowsum = ws_at<float>(ws, L.end);
  float* counter = ws_at<float>(ws, L.end + rowsum_bytes(N));
  if (wc.deterministic && work) {  // every partial is stored, not added: only the counter
    z.p[0] = counter;
    z.n[0] = 1;
    return z;
  }
  z.p[0] = dX;
  z.n[0] = N * D;
  z.p[1] = dY;
  z.n[1] = M * D;
  z.p[2] = (work && tma_flush) ? rowsum : counter;  // rowsum and the counter are adjacent
  z.n[2] = (work && tma_flush) ? rowsum_bytes(N) / 4 + 1 : (work ? 1 : 0);
  return z;
}

bool backward_tc_supported(int64_t N, int64_t M, int64_t D) {
  (void)N; (void)D;
  return (M % 4) == 0;  // G and K rows must be 16-byte pitched for TMA
}

cudaError_t launch_backward_tc(const float* X, const float* Y, const float* G, const float* K,
                               float* dX, float* dY, int64_t N, int64_t M, int64_t D,
                               float gamma, void* ws, const WaitConfig& wc, cudaStream_t stream,
                               const DyRoute* route, Epi epi, bool pre_zeroed) {
  cudaError_t e;
  const bool dot = epi == Epi::kDot;
  const bool routed = route != nullptr && route->world > 0;
  const PrepLayout L = prep_layout(N, M, D);
  const bool tma_flush = kStageDx && (D % 4) == 0;  // dX rows 16-byte pitched, staging present
  float* rowsum = ws_at<float>(ws, L.end);
  int* counter = ws_at<int>(ws, L.end + rowsum_bytes(N));
  const bool work = N > 0 && M > 0 && D > 0;
  // Deterministic mode (not with a routed dY, whose partials already sit in per-rank slots):
  // nothing is accumulated in place, so only the tile counter is zeroed.
  const bool det = wc.deterministic && !routed && work;
  const DetLayout DL = det ? det_layout(N, M, D) : DetLayout{};
  if (pre_zeroed) {
    // backward_zero_spec's ranges were zeroed by the split pass of this forward + backward.
  } else if (det) {
    if ((e = launch_kernel(rbf_bwd_zero_kernel, dim3(1), dim3(256), 0, stream, dX, (int64_t)0,
                           dY, (int64_t)0, reinterpret_cast<float*>(counter), (int64_t)1,
                           (const int*)nullptr)) != cudaSuccess)
      return e;
    note_launches(1);
  } else {
    // rowsum and the counter are adjacent: one range covers both (or just the counter).
    float* zc = (work && tma_flush) ? rowsum : reinterpret_cast<float*>(counter);
    const int64_t nz = (work && tma_flush) ? rowsum_bytes(N) / 4 + 1 : (work ? 1 : 0);
    // Routed: this rank's slot of the dY buffer instead of the caller's dY.
    float* zy = dY;
    const int* zctr = nullptr;
    if (routed) {
      zy = route->bufs[route->rank];
      zctr = route->ctr;
    }
    const int64_t ny = M * D;
    const int64_t total = N * D + ny + nz;
    if (total > 0) {
      const int64_t blocks = std::min<int64_t>(ceil_div(total, 256), 4 * device_sm_count());
      if ((e = launch_kernel(rbf_bwd_zero_kernel, dim3((unsigned)blocks), dim3(256), 0, stream, dX,
                             N * D, zy, ny, zc, nz, zctr)) != cudaSuccess)
        return e;
      note_launches(1);
    }
  }
  if (!work) return cudaGetLastError();
  const int DS = (D <= 32) ? 32 : 64;
  const int mn = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
  CUtensorMap tg, tk, txh, txl, tyh, tyl, tdx;
  if (!make_tmap_2d(&tg, G, N, M, M, 32, 128) ||
      !make_tmap_2d(&tk, dot ? G : K, N, M, M, 32, 128) ||  // DOT: not read
      !make_tmap_2d(&txh, ws_at<float>(ws, L.xhi), N, L.Dp, L.Dp, 32, 32, mn) ||
      !make_tmap_2d(&txl, ws_at<float>(ws, L.xlo), N, L.Dp, L.Dp, 32, 32, mn) ||
      !make_tmap_2d(&tyh, ws_at<float>(ws, L.yhi), M, L.Dp, L.Dp, 32, 32, mn) ||
      !make_tmap_2d(&tyl, ws_at<float>(ws, L.ylo), M, L.Dp, L.Dp, 32, 32, mn))
    return cudaErrorInvalidValue;
  if (tma_flush) {
    // Deterministic mode: the dX tile partials are stored into their slots, [tiles_j * Npad] rows.
    if (!(det ? make_tmap_2d(&tdx, ws_at<float>(ws, L.end + DL.dxp), ceil_div(M, BT) * DL.Npad, D,
                             D, 32, 32)
              : make_tmap_2d(&tdx, dX, N, D, D, 32, 32)))
      return cudaErrorInvalidValue;
  } else {
    tdx = tg;  // unused
  }
  BwdArgs a;
  a.X = X;
  a.Y = Y;
  a.dX = dX;
  a.dY = dY;
  a.rowsum = rowsum;
  a.tma_flush = tma_flush ? 1 : 0;
  a.N = N;
  a.M = M;
  a.D = D;
  a.tiles_i = (int)ceil_div(N, BT);
  a.tiles_j = (int)ceil_div(M, BT);
  a.num_slices = (int)ceil_div(L.Dp, DS);
  a.total_tiles = (int64_t)a.tiles_i * a.tiles_j * a.num_slices;
  a.counter = counter;
  a.route = routed ? *route : DyRoute{};
  if (!routed) a.route.world = 0;
  a.det = det ? 1 : 0;
  a.Npad = DL.Npad;
  a.dxp = det ? ws_at<float>(ws, L.end + DL.dxp) : nullptr;
  a.rsp = det ? ws_at<float>(ws, L.end + DL.rsp) : nullptr;
  a.dyp = det ? ws_at<float>(ws, L.end + DL.dyp) : nullptr;
  a.csp = det ? ws_at<float>(ws, L.end + DL.csp) : nullptr;
  const int grid = (int)std::min<int64_t>(a.total_tiles, device_sm_count());
  {
    // Group width (RBF_BWD_GROUP, default 4) and the share of tiles handed out dynamically
    // (RBF_BWD_DYN_PCT, default 15).
    int group = 4, pct = 15;
    if (const char* s = std::getenv("RBF_BWD_GROUP")) group = std::max(1, std::atoi(s));
    if (const char* s = std::getenv("RBF_BWD_DYN_PCT")) pct = std::max(0, std::min(100, std::atoi(s)));
    if (a.tiles_j % group != 0 || grid % group != 0 || grid < group) group = 1;
    a.group = group;
    const int64_t rows = a.total_tiles / group;
    a.static_rows = rows - rows * pct / 100;
  }
  a.c = dot ? -1.f : -2.f * gamma;
  a.status = ws_at<int>(ws, L.status);
  a.timeout_ns = wc.timeout_ns;
  a.debug_skip_first_load = wc.debug_skip_first_load;
  a.ablate = 0;
#ifdef RBF_TRACE
  if (const char* ab = std::getenv("RBF_ABLATE")) a.ablate = std::atoi(ab);
#endif
  auto launch = [&](auto kernel, size_t smem) -> cudaError_t {
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)smem);
    if (err != cudaSuccess) return err;
    return launch_kernel(kernel, dim3(grid), dim3(THREADS), smem, stream, tg, tk, txh, txl, tyh,
                         tyl, tdx, a);
  };
  if (det) {
    if (DS == 32)
      e = dot ? launch(rbf_bwd_tc_kernel<32, true, true>, Cfg<32>::SMEM)
              : launch(rbf_bwd_tc_kernel<32, false, true>, Cfg<32>::SMEM);
    else
      e = dot ? launch(rbf_bwd_tc_kernel<64, true, true>, Cfg<64>::SMEM)
              : launch(rbf_bwd_tc_kernel<64, false, true>, Cfg<64>::SMEM);
  } else if (DS == 32) {
    e = dot ? launch(rbf_bwd_tc_kernel<32, true>, Cfg<32>::SMEM)
            : launch(rbf_bwd_tc_kernel<32, false>, Cfg<32>::SMEM);
  } else {
    e = dot ? launch(rbf_bwd_tc_kernel<64, true>, Cfg<64>::SMEM)
            : launch(rbf_bwd_tc_kernel<64, false>, Cfg<64>::SMEM);
  }
  if (e != cudaSuccess) return e;
  note_launches(1);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  if (det) {
    const int64_t total = (N + M) * D;
    const int64_t blocks = std::min<int64_t>(ceil_div(total, 256), 8 * device_sm_count());
    if ((e = launch_kernel(rbf_bwd_det_finalize_kernel, dim3((unsigned)blocks), dim3(256), 0,
                           stream, X, Y, (const float*)a.dxp, (const float*)a.rsp,
                           (const float*)a.dyp, (const float*)a.csp, dX, dY, N, M, D, DL.Npad,
                           a.tiles_j, a.tiles_i, a.c, dot ? 0 : 1)) != cudaSuccess)
      return e;
    note_launches(1);
    return cudaGetLastError();
  }
  if (tma_flush && !dot) {
    const int64_t n4 = N * (D / 4);
    if ((e = launch_kernel(rbf_bwd_finalize_kernel, dim3((unsigned)ceil_div(n4, 256)), dim3(256), 0,
                           stream, X, rowsum, dX, N, D, a.c)) != cudaSuccess)
      return e;
    note_launches(1);
  }
  return cudaGetLastError();
}

}  // namespace rbf

#ifdef RBF_TRACE
extern "C" __attribute__((visibility("default"))) int rbf_debug_trace(unsigned long long* out,
                                                                      int* n) {
  cudaMemcpyFromSymbol(out, rbf::g_trace, sizeof(rbf::g_trace));
  cudaMemcpyFromSymbol(n, rbf::g_trace_n, sizeof(rbf::g_trace_n));
  int z[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  return (int)cudaMemcpyToSymbol(rbf::g_trace_n, z, sizeof(z));
}

extern "C" __attribute__((visibility("default"))) int rbf_debug_spans(unsigned long long* out) {
  return (int)cudaMemcpyFromSymbol(out, rbf::g_cta_span, sizeof(rbf::g_cta_span));
}
#endif
