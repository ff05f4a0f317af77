// rbf_bwd_tc.cu -- the fused RBF backward on the sm_100a tensor cores.
//
//   W = G o K,  c = -2 gamma
//   dX[i,:] = c * ( rowsum_j(W)[i] * x_i - sum_j W[i,j] y_j )
//   dY[j,:] = c * ( colsum_i(W)[j] * y_j - sum_i W[i,j] x_i )
//
// G and K are read from HBM exactly once, in tiles of 128 (i) x 128 (j) that arrive as four
// strips of 32 rows (TMA, 128-byte swizzle).  W is formed on the CUDA cores in two mappings:
//   C-warps (thread <-> column j): per strip, W^T[j, 32 rows] -> TF32 hi/lo -> TMEM lanes j,
//     the A operand of the dY product  D_dY[j,d] += W^T[j,i] X[i,d]  (tcgen05.mma, A in TMEM,
//     B = the strip's X rows in shared memory, MN-major).  colsum_j accumulates in a register.
//   R-warps (thread <-> row i): W[i, 128 columns] -> hi/lo -> TMEM lanes i, the A operand of
//     D_dX[i,d] += W[i,j] Y[j,d] (B = the CTA's resident Y tile).  rowsum_i in a register.
// Both products are 3xTF32 (hi*hi + hi*lo + lo*hi), fp32 accumulation in TMEM.
// MN-major tf32 operands must use the "128-byte swizzle, 32-byte atom" shared-memory layout
// (descriptor layout type 1; 4-row K groups); the X and Y tensor maps load them that way
// (CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B).
//
// Work split: tiles are ordered (feature slice, j-block, i-block) and every CTA takes a
// contiguous range, so within a j-block segment the dY accumulator stays in TMEM across all its
// i-blocks.  The dX accumulator covers one tile (128 columns) and is flushed after every tile;
// flushes and segment ends add c*(sum * x - acc) into dX / dY with vector red.global.add (the
// outputs are zeroed first), so no partial buffers exist.  Features are processed in slices of
// DS (32 or 64) columns; D > 64 runs one slice per segment (G and K are re-read per slice).
//
// TMEM (512 columns): [0,64) dY acc | [64,128) dX acc | [128,256) two W^T buffers (hi,lo x 32)
//                     | [256,384) W hi (128 cols) | [384,512) W lo.
// Shared memory: a 3-deep ring of strips (G 16 KiB + K 16 KiB + X hi/lo rows) and the resident
// Y hi/lo tile of the current j-block.
// Warps: 0 TMA producer, 1 MMA issuer, 2-5 C-warps, 6-9 R-warps (warp w owns TMEM lanes
// 32*(w%4)..+31).  Every mbarrier wait is bounded; a timeout is recorded in the status word.
#include <cuda.h>

#include <algorithm>

#include "rbf_common.cuh"
#include "rbf_kernels.cuh"
#include "rbf_ptx.cuh"

namespace rbf {
namespace {

constexpr int BT = 128;        // tile edge (rows of i and columns of j)
constexpr int SR = 32;         // strip rows
constexpr int STAGES = 3;
constexpr int THREADS = 320;
constexpr uint32_t BOX = 32 * 32 * 4;  // one 32x32 fp32 TMA box, 4 KiB
constexpr uint32_t COL_DY = 0, COL_DX = 64, COL_WT = 128, COL_W = 256;
constexpr uint32_t MN_SBO = 512;       // 4 K-rows x 128 B: one K group of the 32B-atom layout
constexpr uint32_t MN_LAYOUT = 1;      // descriptor layout type: 128B swizzle, 32B atom

template <int DS>
struct Cfg {
  static constexpr uint32_t G_BYTES = 4 * BOX;                  // strip of G: 32 x 128
  static constexpr uint32_t X_BYTES = (DS / 32) * BOX;          // strip of X (hi or lo)
  static constexpr uint32_t STAGE_BYTES = 2 * G_BYTES + 2 * X_BYTES;
  static constexpr uint32_t YBOX = 128 * 32 * 4;                // 128 j rows x 32 features
  static constexpr uint32_t Y_BYTES = (DS / 32) * YBOX;         // Y tile (hi or lo)
  static constexpr size_t SMEM = 1024 + STAGES * STAGE_BYTES + 2 * Y_BYTES + 512;
};
static_assert(Cfg<64>::SMEM <= 232448, "backward shared memory over the sm_100 limit");

struct BwdArgs {
  const float* X;
  const float* Y;
  float* dX;
  float* dY;
  int64_t N, M, D;
  int tiles_i, tiles_j, num_slices;
  int64_t total_tiles;
  float c;  // -2 gamma
  int* status;
  unsigned long long timeout_ns;
  int debug_skip_first_load;
};

struct TileCoord {
  int slice, jb, ib;
};

__device__ __forceinline__ TileCoord tile_of(int64_t t, const BwdArgs& a) {
  TileCoord c;
  c.ib = (int)(t % a.tiles_i);
  const int64_t r = t / a.tiles_i;
  c.jb = (int)(r % a.tiles_j);
  c.slice = (int)(r / a.tiles_j);
  return c;
}

__device__ __forceinline__ bool segment_ends(int64_t t, int64_t t_end, const TileCoord& tc,
                                             const BwdArgs& a) {
  if (t + 1 == t_end) return true;
  const TileCoord n = tile_of(t + 1, a);
  return n.slice != tc.slice || n.jb != tc.jb;
}

__device__ __forceinline__ void red_add4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

__device__ __forceinline__ void red_add1(float* p, float a) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(a) : "memory");
}

// out[r, d0 + e] += c * (s * src[r, d0 + e] - acc[e]) for e < DS, d0 + e < D.
template <int DS>
__device__ __forceinline__ void flush_row(float* out, const float* src, int64_t r, int64_t D,
                                          int d0, float c, float s, const uint32_t* acc) {
  float* o = out + r * D + d0;
  const float* x = src + r * D + d0;
  const int n = (D - d0) < DS ? (int)(D - d0) : DS;
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

template <int DS>
__global__ void __launch_bounds__(THREADS, 1)
    rbf_bwd_tc_kernel(const __grid_constant__ CUtensorMap tm_g,
                      const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_xhi,
                      const __grid_constant__ CUtensorMap tm_xlo,
                      const __grid_constant__ CUtensorMap tm_yhi,
                      const __grid_constant__ CUtensorMap tm_ylo, const BwdArgs a) {
  using C = Cfg<DS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint8_t* ytile = smem + STAGES * C::STAGE_BYTES;  // [Y hi | Y lo]
  uint64_t* bars = reinterpret_cast<uint64_t*>(ytile + 2 * C::Y_BYTES);
  uint64_t* full = bars;                 // [STAGES] TMA -> consumers
  uint64_t* empty = full + STAGES;       // [STAGES] consumers -> TMA
  uint64_t* wt_full = empty + STAGES;    // [2]      C-warps -> MMA
  uint64_t* wt_empty = wt_full + 2;      // [2]      MMA -> C-warps
  uint64_t* w_full = wt_empty + 2;       // R-warps -> MMA
  uint64_t* dx_full = w_full + 1;        // MMA -> R-warps
  uint64_t* dx_empty = dx_full + 1;      // R-warps -> MMA
  uint64_t* dy_full = dx_empty + 1;      // MMA -> C-warps
  uint64_t* dy_empty = dy_full + 1;      // C-warps -> MMA
  uint64_t* y_full = dy_empty + 1;       // TMA -> MMA
  uint64_t* y_empty = y_full + 1;        // MMA -> TMA
  uint64_t* drain = y_empty + 1;         // MMA teardown
  uint64_t* r_full = drain + 1;          // [4] C-warps -> R-warp s: strip s of a tile landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(r_full + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 6);  // 4 C-warps + 1 R-warp + 1 MMA commit
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(&wt_full[b], 4);
      ptx::mbar_init(&wt_empty[b], 1);
    }
    ptx::mbar_init(w_full, 4);
    ptx::mbar_init(dx_full, 1);
    ptx::mbar_init(dx_empty, 4);
    ptx::mbar_init(dy_full, 1);
    ptx::mbar_init(dy_empty, 4);
    ptx::mbar_init(y_full, 1);
    ptx::mbar_init(y_empty, 1);
    ptx::mbar_init(drain, 1);
    for (int s = 0; s < 4; ++s) ptx::mbar_init(&r_full[s], 1);
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tensormap(&tm_g);
    ptx::prefetch_tensormap(&tm_k);
    ptx::prefetch_tensormap(&tm_xhi);
    ptx::prefetch_tensormap(&tm_xlo);
    ptx::prefetch_tensormap(&tm_yhi);
    ptx::prefetch_tensormap(&tm_ylo);
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, 512);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Contiguous, balanced range of tiles for this CTA.
  const int64_t t_begin = a.total_tiles * blockIdx.x / gridDim.x;
  const int64_t t_end = a.total_tiles * (blockIdx.x + 1) / gridDim.x;

  if (warp == 0) {
    // ================================================================ TMA producer
    if (lane == 0) {
      const uint64_t stream_policy = ptx::policy_evict_first();
      const uint64_t keep_policy = ptx::policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      uint32_t y_phase = 0;
      int last_parity[STAGES];
      for (int s = 0; s < STAGES; ++s) last_parity[s] = -1;
      int y_issued = -1;
      bool ok = true, skipped = false;
      int cur_slice = -1, cur_jb = -1;
      for (int64_t t = t_begin; t < t_end && ok; ++t) {
        const TileCoord tc = tile_of(t, a);
        const int i0 = tc.ib * BT, j0 = tc.jb * BT, d0 = tc.slice * DS;
        if (tc.slice != cur_slice || tc.jb != cur_jb) {
          cur_slice = tc.slice;
          cur_jb = tc.jb;
          // The previous Y tile must be released by the MMAs that read it.
          if (!ptx::mbar_wait_bounded(y_empty, y_phase ^ 1, a.status, a.timeout_ns)) { ok = false; break; }
          ptx::mbar_arrive_expect_tx(y_full, 2 * C::Y_BYTES);
#pragma unroll
          for (int b = 0; b < DS / 32; ++b) {
            ptx::tma_load_2d_hint(ytile + b * C::YBOX, &tm_yhi, d0 + 32 * b, j0, y_full, keep_policy);
            ptx::tma_load_2d_hint(ytile + C::Y_BYTES + b * C::YBOX, &tm_ylo, d0 + 32 * b, j0,
                                  y_full, keep_policy);
          }
          y_issued = (int)y_phase;
          y_phase ^= 1;
        }
        for (int s = 0; s < 4; ++s) {
          if (!ptx::mbar_wait_bounded(&empty[stage], phase ^ 1, a.status, a.timeout_ns)) { ok = false; break; }
          if (a.debug_skip_first_load && !skipped && blockIdx.x == 0) {
            skipped = true;  // test hook: the first strip never arrives
          } else {
            uint8_t* sm = ring + stage * C::STAGE_BYTES;
            uint64_t* fb = &full[stage];
            ptx::mbar_arrive_expect_tx(fb, C::STAGE_BYTES);
            const int ir = i0 + SR * s;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              ptx::tma_load_2d_hint(sm + b * BOX, &tm_g, j0 + 32 * b, ir, fb, stream_policy);
              ptx::tma_load_2d_hint(sm + C::G_BYTES + b * BOX, &tm_k, j0 + 32 * b, ir, fb,
                                    stream_policy);
            }
#pragma unroll
            for (int b = 0; b < DS / 32; ++b) {
              ptx::tma_load_2d_hint(sm + 2 * C::G_BYTES + b * BOX, &tm_xhi, d0 + 32 * b, ir, fb,
                                    keep_policy);
              ptx::tma_load_2d_hint(sm + 2 * C::G_BYTES + C::X_BYTES + b * BOX, &tm_xlo,
                                    d0 + 32 * b, ir, fb, keep_policy);
            }
            last_parity[stage] = (int)phase;
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) {
        for (int s = 0; s < STAGES; ++s)
          if (last_parity[s] >= 0)
            ptx::mbar_wait_bounded(&full[s], (uint32_t)last_parity[s], a.status, a.timeout_ns);
        if (y_issued >= 0) ptx::mbar_wait_bounded(y_full, (uint32_t)y_issued, a.status, a.timeout_ns);
      }
    }
  } else if (warp == 1) {
    // ================================================================ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = ptx::idesc_tf32(128, DS, 0, 1);
      int stage = 0;
      uint32_t phase = 0;
      int wb = 0;
      uint32_t wt_phase[2] = {0, 0};
      uint32_t w_phase = 0, dxe_phase = 0, dye_phase = 0, y_phase = 0;
      bool ok = true;
      int cur_slice = -1, cur_jb = -1;
      bool dy_first = true;
      for (int64_t t = t_begin; t < t_end && ok; ++t) {
        const TileCoord tc = tile_of(t, a);
        if (tc.slice != cur_slice || tc.jb != cur_jb) {
          cur_slice = tc.slice;
          cur_jb = tc.jb;
          // dY accumulator drained by the C-warps (flush of the previous segment).
          if (!ptx::mbar_wait_bounded(dy_empty, dye_phase ^ 1, a.status, a.timeout_ns)) { ok = false; break; }
          dye_phase ^= 1;
          if (!ptx::mbar_wait_bounded(y_full, y_phase, a.status, a.timeout_ns)) { ok = false; break; }
          y_phase ^= 1;
          dy_first = true;
        }
        const bool seg_end = segment_ends(t, t_end, tc, a);
        // ---- dY: one 32-row strip at a time, A = W^T (TMEM lanes j), B = X strip rows.
        for (int s = 0; s < 4 && ok; ++s) {
          if (!ptx::mbar_wait_bounded(&wt_full[wb], wt_phase[wb], a.status, a.timeout_ns) ||
              !ptx::mbar_wait_bounded(&full[stage], phase, a.status, a.timeout_ns)) {
            ok = false;
            break;
          }
          wt_phase[wb] ^= 1;
          ptx::tc_fence_after();
          const uint32_t xb = ptx::smem_u32(ring + stage * C::STAGE_BYTES + 2 * C::G_BYTES);
          const uint32_t a_hi = tmem + COL_WT + 64 * wb;
#pragma unroll
          for (int k = 0; k < SR / 8; ++k) {
            const uint64_t bh = ptx::smem_desc(xb + 1024 * k, BOX, MN_SBO, MN_LAYOUT);
            const uint64_t bl = ptx::smem_desc(xb + C::X_BYTES + 1024 * k, BOX, MN_SBO, MN_LAYOUT);
            ptx::mma_tf32_ts(tmem + COL_DY, a_hi + 8 * k, bh, idesc, dy_first ? 0u : 1u);
            ptx::mma_tf32_ts(tmem + COL_DY, a_hi + 8 * k, bl, idesc, 1);
            ptx::mma_tf32_ts(tmem + COL_DY, a_hi + 32 + 8 * k, bh, idesc, 1);
            dy_first = false;
          }
          ptx::mma_commit(&wt_empty[wb]);
          ptx::mma_commit(&empty[stage]);
          wb ^= 1;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        // ---- dX: A = W (TMEM lanes i, 128 columns of K), B = resident Y tile.
        if (!ptx::mbar_wait_bounded(w_full, w_phase, a.status, a.timeout_ns) ||
            !ptx::mbar_wait_bounded(dx_empty, dxe_phase ^ 1, a.status, a.timeout_ns)) {
          ok = false;
          break;
        }
        w_phase ^= 1;
        dxe_phase ^= 1;
        ptx::tc_fence_after();
        const uint32_t yb = ptx::smem_u32(ytile);
#pragma unroll 4
        for (int k = 0; k < BT / 8; ++k) {
          const uint64_t bh = ptx::smem_desc(yb + 1024 * k, C::YBOX, MN_SBO, MN_LAYOUT);
          const uint64_t bl = ptx::smem_desc(yb + C::Y_BYTES + 1024 * k, C::YBOX, MN_SBO, MN_LAYOUT);
          ptx::mma_tf32_ts(tmem + COL_DX, tmem + COL_W + 8 * k, bh, idesc, k > 0 ? 1u : 0u);
          ptx::mma_tf32_ts(tmem + COL_DX, tmem + COL_W + 8 * k, bl, idesc, 1);
          ptx::mma_tf32_ts(tmem + COL_DX, tmem + COL_W + 128 + 8 * k, bh, idesc, 1);
        }
        ptx::mma_commit(dx_full);
        if (seg_end) {
          ptx::mma_commit(dy_full);
          ptx::mma_commit(y_empty);
        }
      }
      ptx::mma_commit(drain);
      ptx::mbar_wait_bounded(drain, 0, a.status, a.timeout_ns);
    }
  } else if (warp < 6) {
    // ================================================================ C-warps (column j)
    const int q = warp & 3;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    int stage = 0;
    uint32_t phase = 0;
    int wb = 0;
    uint32_t wte_phase[2] = {0, 0};
    uint32_t dyf_phase = 0;
    float colsum = 0.f;
    int cur_slice = -1, cur_jb = -1;
    bool ok = true;
    for (int64_t t = t_begin; t < t_end && ok; ++t) {
      const TileCoord tc = tile_of(t, a);
      if (tc.slice != cur_slice || tc.jb != cur_jb) {
        cur_slice = tc.slice;
        cur_jb = tc.jb;
        colsum = 0.f;
      }
      const bool seg_end = segment_ends(t, t_end, tc, a);
      for (int s = 0; s < 4; ++s) {
        if (!ptx::mbar_wait_bounded(&full[stage], phase, a.status, a.timeout_ns)) { ok = false; break; }
        // Hand strip s to R-warp s.  The R-warps cannot wait on full[] themselves: strip 3 sits
        // in a stage one phase ahead of strips 0-2, and a parity wait cannot tell the phases
        // apart.  r_full[s] advances exactly once per tile, so its parity is unambiguous.
        if (q == 0 && lane == 0) ptx::mbar_arrive(&r_full[s]);
        const uint8_t* sm = ring + stage * C::STAGE_BYTES;
        const uint8_t* gb = sm + q * BOX;
        const uint8_t* kb = sm + C::G_BYTES + q * BOX;
        uint32_t hi[32], lo[32];
        const int ch = lane >> 2, wi = (lane & 3) * 4;
#pragma unroll
        for (int r = 0; r < 32; ++r) {
          const int off = r * 128 + ((ch ^ (r & 7)) << 4) + wi;
          const float w = *reinterpret_cast<const float*>(gb + off) *
                          *reinterpret_cast<const float*>(kb + off);
          colsum += w;
          float h, l;
          tf32_split(w, h, l);
          hi[r] = __float_as_uint(h);
          lo[r] = __float_as_uint(l);
        }
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&empty[stage]);
        if (!ptx::mbar_wait_bounded(&wt_empty[wb], wte_phase[wb] ^ 1, a.status, a.timeout_ns)) { ok = false; break; }
        wte_phase[wb] ^= 1;
        ptx::tc_fence_after();
        ptx::tmem_st32(tmem + lane_base + COL_WT + 64 * wb, hi);
        ptx::tmem_st32(tmem + lane_base + COL_WT + 64 * wb + 32, lo);
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&wt_full[wb]);
        wb ^= 1;
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
      if (seg_end) {
        if (!ptx::mbar_wait_bounded(dy_full, dyf_phase, a.status, a.timeout_ns)) { ok = false; break; }
        dyf_phase ^= 1;
        ptx::tc_fence_after();
        uint32_t acc[64];
        tmem_load_row<DS>(tmem + lane_base + COL_DY, acc);
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(dy_empty);
        const int64_t j = (int64_t)tc.jb * BT + q * 32 + lane;
        if (j < a.M) flush_row<DS>(a.dY, a.Y, j, a.D, tc.slice * DS, a.c, colsum, acc);
      }
    }
  } else {
    // ================================================================ R-warps (row i)
    const int q = warp & 3;  // this warp's strip within the tile and its TMEM lane quadrant
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    int64_t strip_count = 0;  // strips consumed by this CTA so far (ring position)
    uint32_t dxf_phase = 0, rf_phase = 0;
    bool ok = true;
    for (int64_t t = t_begin; t < t_end && ok; ++t, strip_count += 4) {
      const TileCoord tc = tile_of(t, a);
      const int64_t pos = strip_count + q;
      const int stage = (int)(pos % STAGES);
      if (!ptx::mbar_wait_bounded(&r_full[q], rf_phase, a.status, a.timeout_ns)) { ok = false; break; }
      rf_phase ^= 1;
      const uint8_t* sm = ring + stage * C::STAGE_BYTES;
      float rowsum = 0.f;
      // The W buffer is free: this warp waited for the previous tile's dX MMAs (dx_full).
      ptx::tc_fence_after();
#pragma unroll 1
      for (int b = 0; b < 4; ++b) {
        const uint8_t* gb = sm + b * BOX + lane * 128;
        const uint8_t* kb = sm + C::G_BYTES + b * BOX + lane * 128;
        uint32_t hi[32], lo[32];
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4) {
          const int off = (c4 ^ (lane & 7)) << 4;
          const float4 g = *reinterpret_cast<const float4*>(gb + off);
          const float4 k = *reinterpret_cast<const float4*>(kb + off);
          const float w[4] = {g.x * k.x, g.y * k.y, g.z * k.z, g.w * k.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            rowsum += w[e];
            float h, l;
            tf32_split(w[e], h, l);
            hi[4 * c4 + e] = __float_as_uint(h);
            lo[4 * c4 + e] = __float_as_uint(l);
          }
        }
        ptx::tmem_st32(tmem + lane_base + COL_W + 32 * b, hi);
        ptx::tmem_st32(tmem + lane_base + COL_W + 128 + 32 * b, lo);
      }
      ptx::tmem_wait_st();
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        ptx::mbar_arrive(&empty[stage]);
        ptx::mbar_arrive(w_full);
      }
      // dX of this tile: wait for the MMAs, drain the accumulator, flush.
      if (!ptx::mbar_wait_bounded(dx_full, dxf_phase, a.status, a.timeout_ns)) { ok = false; break; }
      dxf_phase ^= 1;
      ptx::tc_fence_after();
      uint32_t acc[64];
      tmem_load_row<DS>(tmem + lane_base + COL_DX, acc);
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(dx_empty);
      const int64_t i = (int64_t)tc.ib * BT + q * 32 + lane;
      if (i < a.N) flush_row<DS>(a.dX, a.X, i, a.D, tc.slice * DS, a.c, rowsum, acc);
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, 512);
  }
}

}  // namespace

bool backward_tc_supported(int64_t N, int64_t M, int64_t D) {
  (void)N; (void)D;
  return (M % 4) == 0;  // G and K rows must be 16-byte pitched for TMA
}

cudaError_t launch_backward_tc(const float* X, const float* Y, const float* G, const float* K,
                               float* dX, float* dY, int64_t N, int64_t M, int64_t D,
                               float gamma, void* ws, const WaitConfig& wc, cudaStream_t stream) {
  cudaError_t e;
  if (N * D > 0 && (e = cudaMemsetAsync(dX, 0, sizeof(float) * (size_t)(N * D), stream)) != cudaSuccess) return e;
  if (M * D > 0 && (e = cudaMemsetAsync(dY, 0, sizeof(float) * (size_t)(M * D), stream)) != cudaSuccess) return e;
  if (N == 0 || M == 0 || D == 0) return cudaSuccess;
  const PrepLayout L = prep_layout(N, M, D);
  const int DS = (D <= 32) ? 32 : 64;
  const int mn = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
  CUtensorMap tg, tk, txh, txl, tyh, tyl;
  if (!make_tmap_2d(&tg, G, N, M, M, 32, 32) || !make_tmap_2d(&tk, K, N, M, M, 32, 32) ||
      !make_tmap_2d(&txh, ws_at<float>(ws, L.xhi), N, L.Dp, L.Dp, 32, 32, mn) ||
      !make_tmap_2d(&txl, ws_at<float>(ws, L.xlo), N, L.Dp, L.Dp, 32, 32, mn) ||
      !make_tmap_2d(&tyh, ws_at<float>(ws, L.yhi), M, L.Dp, L.Dp, 32, 128, mn) ||
      !make_tmap_2d(&tyl, ws_at<float>(ws, L.ylo), M, L.Dp, L.Dp, 32, 128, mn))
    return cudaErrorInvalidValue;
  BwdArgs a;
  a.X = X;
  a.Y = Y;
  a.dX = dX;
  a.dY = dY;
  a.N = N;
  a.M = M;
  a.D = D;
  a.tiles_i = (int)ceil_div(N, BT);
  a.tiles_j = (int)ceil_div(M, BT);
  a.num_slices = (int)ceil_div(L.Dp, DS);
  a.total_tiles = (int64_t)a.tiles_i * a.tiles_j * a.num_slices;
  a.c = -2.f * gamma;
  a.status = ws_at<int>(ws, L.status);
  a.timeout_ns = wc.timeout_ns;
  a.debug_skip_first_load = wc.debug_skip_first_load;
  const int grid = (int)std::min<int64_t>(a.total_tiles, device_sm_count());
  if (DS == 32) {
    if ((e = cudaFuncSetAttribute(rbf_bwd_tc_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)Cfg<32>::SMEM)) != cudaSuccess)
      return e;
    rbf_bwd_tc_kernel<32><<<grid, THREADS, Cfg<32>::SMEM, stream>>>(tg, tk, txh, txl, tyh, tyl, a);
  } else {
    if ((e = cudaFuncSetAttribute(rbf_bwd_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)Cfg<64>::SMEM)) != cudaSuccess)
      return e;
    rbf_bwd_tc_kernel<64><<<grid, THREADS, Cfg<64>::SMEM, stream>>>(tg, tk, txh, txl, tyh, tyl, a);
  }
  note_launches(1);
  return cudaGetLastError();
}

}  // namespace rbf
