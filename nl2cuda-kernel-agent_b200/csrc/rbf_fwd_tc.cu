// rbf_fwd_tc.cu -- the RBF forward on the sm_100a tensor cores.
//
//   K[i,j] = exp(-gamma * max(||x_i||^2 + ||y_j||^2 - 2 x_i.y_j, 0))
//
// x_i.y_j is a dense contraction over D; it runs on tcgen05 tensor cores in 3xTF32:
//   x.y ~= xhi.yhi + xhi.ylo + xlo.yhi
// where hi is the TF32-exact top of each fp32 value and lo the fp32 remainder (both written by
// the split pass, rbf_prep.cu).  The dropped lo.lo term and the TF32 rounding of lo are below
// 2^-20 relative, so the product has fp32-level accuracy.
//
// Kernel organisation (one persistent CTA per SM, 320 threads):
//   warp 0    TMA producer: per stage one 32-feature slice of Xhi, Xlo (128 rows each) and of
//             Yhi, Ylo (128 rows each), 128-byte swizzled, into a 2-deep ring (64 KiB/stage).
//   warp 1    MMA issuer (one thread): 3 x tcgen05.mma.kind::tf32 (M=128, N=128, K=8) per 8
//             features into one of two TMEM accumulators (2 x 128 columns), so the epilogue of
//             tile t overlaps the MMAs of tile t+1.  With X resident (D <= 64) the thread
//             copies X hi|lo from shared memory into TMEM (tcgen05.cp, columns 256..383) once
//             per row block and the MMAs take A from TMEM, so only Y is read from shared memory.
//   warps 2.. epilogue: warp w reads TMEM lanes 32*(w%4).. (its row quadrant) and one column group of
//             the columns, adds the norms, clamps, exponentiates (MUFU ex2), stages 32x32 fp32
//             blocks in swizzled shared memory (two per warp, so a chunk never waits for the
//             previous store to drain) and writes them with TMA stores (no multicast).
// Every mbarrier wait is bounded (globaltimer); on expiry the kernel records RBF_ERR_TIMEOUT in
// the workspace status word, waits (bounded) for its own copies in flight, frees TMEM and
// returns.
//
// HBM roofline per launch: K write 4*N*M bytes + X/Y split reads; tensor work 3 * 2*N*M*Dp.
//
// The DOT instantiation stores x_i.y_j itself (no norms, no exp): with rows the split pass
// normalised, that is the cosine-similarity matrix S[i,j] = a_i.b_j / (|a_i| |b_j|).
#include <cuda.h>

#include <algorithm>

#include "rbf_common.cuh"
#include "rbf_kernels.cuh"
#include "rbf_ptx.cuh"

namespace rbf {
namespace {

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int BK = 32;
#ifndef RBF_EPI_BUFS
#define RBF_EPI_BUFS 1
#endif
#ifndef RBF_EPI_WARPS
#define RBF_EPI_WARPS 8
#endif
constexpr int STAGES = (RBF_EPI_BUFS == 1 && RBF_EPI_WARPS == 8) ? 3 : 2;
// Epilogue warps: 4 per TMEM lane quadrant, each converting one 32-column chunk per tile (more
// warps per scheduler hide the latency of the exp (MUFU) and shuffle chains).
constexpr int EPI_WARPS = RBF_EPI_WARPS;
constexpr int CPW = 16 / EPI_WARPS;  // 32-column chunks per epilogue warp per tile
constexpr int THREADS = 32 * (2 + EPI_WARPS);
constexpr uint32_t TILE_BYTES = 128 * BK * 4;  // 16 KiB: 128 rows x 128 bytes
constexpr uint32_t STAGE_BYTES = 4 * TILE_BYTES;
constexpr int EPI_BUFS = RBF_EPI_BUFS;                      // 32x32 fp32 staging blocks per warp
constexpr uint32_t EPI_BYTES = EPI_BUFS * 32 * 32 * 4;
constexpr uint32_t TMEM_COLS = 2 * BN;
// X-in-TMEM variant (resident X, single CTA): the MMA's A operand (X hi | X lo, 64 columns each)
// sits in TMEM after the two accumulators, so the MMAs read only Y from shared memory.
#ifndef RBF_FWD_ATMEM
#define RBF_FWD_ATMEM 1
#endif
constexpr uint32_t XCOL = 2 * BN;
constexpr uint32_t TMEM_COLS_AT = 512;
constexpr size_t SMEM_BYTES = 1024 + (size_t)STAGES * STAGE_BYTES + EPI_WARPS * EPI_BYTES + 256;
static_assert(SMEM_BYTES <= 232448, "forward shared memory over the sm_100 limit");
// Resident-X variant (D <= 64, at most two 32-feature chunks): the CTA walks its tiles along j,
// so the X hi/lo slices of one row block stay in shared memory and only Y is streamed.
constexpr int RA_CHUNKS = 2;
constexpr int RB_STAGES = (EPI_BUFS == 1 && EPI_WARPS == 8) ? 4 : 3;
constexpr uint32_t CHUNK_BYTES = 2 * TILE_BYTES;  // hi + lo of one 32-feature slice, 128 rows
// Pair variant (two-CTA clusters, tcgen05.mma.cta_group::2, M = 256): each CTA keeps its own 128
// X rows resident and streams only 64 of the tile's 128 Y rows, so Y traffic per SM halves.
constexpr int PB_STAGES = 2 * RB_STAGES;  // the same bytes as the single-CTA Y ring
constexpr uint32_t PCHUNK_BYTES = CHUNK_BYTES / 2;  // hi + lo of one slice, 64 rows
constexpr int PAIR_ROWS = 64;
constexpr size_t SMEM_BYTES_RA =
    1024 + (size_t)RA_CHUNKS * CHUNK_BYTES + RB_STAGES * CHUNK_BYTES + EPI_WARPS * EPI_BYTES + 256;
static_assert(SMEM_BYTES_RA <= 232448, "forward shared memory over the sm_100 limit");

struct FwdArgs {
  const float* xn;
  const float* yn;
  float* K;  // direct-store epilogue only
  int64_t N, M;
  int tiles_m, tiles_n, num_kc;
  float scale;  // -gamma * log2(e)
  int* status;
  unsigned long long timeout_ns;
  int debug_skip_first_load;
  int ablate;  // development builds only (RBF_TRACE): 1 no MMA, 2 no epilogue math/store, 3 no store, 4 = 1+2
};

#ifdef RBF_TRACE
__device__ unsigned long long g_fwd_span[1024][3];
// Development timeline of CTA 0 (trace builds only): per role, (code << 56 | globaltimer).
__device__ unsigned long long g_ftrace[4][512];
__device__ int g_ftrace_n[4];
__device__ __forceinline__ void ftrace(int role, int code) {
  if (blockIdx.x != 0) return;
  const int n = g_ftrace_n[role];
  if (n < 512) {
    g_ftrace[role][n] = ((unsigned long long)code << 56) | (ptx::globaltimer() & ((1ull << 56) - 1));
    g_ftrace_n[role] = n + 1;
  }
}
#define FTRACE(role, code) ftrace(role, code)
#else
#define FTRACE(role, code) ((void)0)
#endif

template <bool TMA_STORE, bool RES_A, bool PAIR, bool DOT = false>
__global__ void __launch_bounds__(THREADS, 1)
    rbf_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_xhi,
                      const __grid_constant__ CUtensorMap tm_xlo,
                      const __grid_constant__ CUtensorMap tm_yhi,
                      const __grid_constant__ CUtensorMap tm_ylo,
                      const __grid_constant__ CUtensorMap tm_k, const FwdArgs a) {
#ifdef RBF_TRACE
  if (threadIdx.x == 0 && blockIdx.x < 1024) g_fwd_span[blockIdx.x][2] = ptx::globaltimer();
#endif
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  // Streamed variant: [STAGES][X hi | X lo | Y hi | Y lo].  Resident-X variant:
  // [RA_CHUNKS][X hi | X lo] then [RB_STAGES][Y hi | Y lo].
  uint8_t* stage_mem = smem;
  uint8_t* epi_mem = smem + (RES_A ? (RA_CHUNKS + RB_STAGES) * CHUNK_BYTES : STAGES * STAGE_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(epi_mem + EPI_WARPS * EPI_BYTES);
  uint64_t* full = bars;                  // [8]  TMA -> MMA (operand stage)
  uint64_t* empty = bars + 8;             // [8]  MMA -> TMA
  uint64_t* a_full = bars + 16;           // resident X landed   TMA -> MMA
  uint64_t* a_empty = bars + 17;          // resident X released MMA -> TMA
  uint64_t* acc_full = bars + 18;         // [2]       MMA -> epilogue
  uint64_t* acc_empty = acc_full + 2;     // [2]       epilogue -> MMA
  uint64_t* drain = acc_empty + 2;        // [1]       MMA teardown
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Pair variant: rank 0 of the cluster issues the MMAs and owns the barriers that count both
  // CTAs' operand bytes (full, a_full) and both CTAs' epilogue releases (acc_empty).
  const uint32_t rank = PAIR ? ptx::cluster_ctarank() : 0;
  const bool leader = rank == 0;
  constexpr bool A_TMEM = RES_A && !PAIR && RBF_FWD_ATMEM;
  constexpr uint32_t TCOLS = A_TMEM ? TMEM_COLS_AT : TMEM_COLS;
  if (threadIdx.x == 0) {
    for (int s = 0; s < 8; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    ptx::mbar_init(a_full, 1);
    ptx::mbar_init(a_empty, 1);
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(&acc_full[b], 1);
      ptx::mbar_init(&acc_empty[b], PAIR ? 2 * EPI_WARPS : EPI_WARPS);
    }
    ptx::mbar_init(drain, 1);
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tensormap(&tm_xhi);
    ptx::prefetch_tensormap(&tm_xlo);
    ptx::prefetch_tensormap(&tm_yhi);
    ptx::prefetch_tensormap(&tm_ylo);
    if (TMA_STORE) ptx::prefetch_tensormap(&tm_k);
  }
  if (PAIR) ptx::cluster_sync();  // the peer's barriers exist before any remote arrive
  if (warp == 1) {
    if (PAIR) {
      ptx::tmem_alloc_pair(tmem_slot, TCOLS);
      ptx::tmem_relinquish_pair();
    } else {
      ptx::tmem_alloc(tmem_slot, TCOLS);
      ptx::tmem_relinquish();
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
#ifdef RBF_TRACE
  if (threadIdx.x == 0 && blockIdx.x < 1024) g_fwd_span[blockIdx.x][0] = ptx::globaltimer();
#endif
  ptx::griddep_wait();  // the split pass (previous kernel) has written the workspace
  // Contiguous, balanced tile range per CTA; tiles run along j (t -> ib = t / tiles_n).
  // Pair variant: the unit is the cluster and a tile is 256 rows (128 per CTA) x 128 columns.
  const int64_t num_tiles = (int64_t)a.tiles_m * a.tiles_n;
  const int64_t unit = PAIR ? (blockIdx.x >> 1) : blockIdx.x;
  const int64_t units = PAIR ? (gridDim.x >> 1) : gridDim.x;
  const int64_t t_begin = num_tiles * unit / units;
  const int64_t t_end = num_tiles * (unit + 1) / units;
  constexpr int TILE_ROWS = PAIR ? 2 * BM : BM;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && RES_A) {
      constexpr int NS = PAIR ? PB_STAGES : RB_STAGES;
      constexpr uint32_t BSTAGE = PAIR ? PCHUNK_BYTES : CHUNK_BYTES;
      constexpr uint32_t PEERS = PAIR ? 2 : 1;
      uint8_t* bring = stage_mem + RA_CHUNKS * CHUNK_BYTES;
      const uint32_t a_full_c = PAIR ? ptx::map_to_rank(a_full, 0) : 0;
      int stage = 0;
      uint32_t phase = 0, a_phase = 0;
      // Stages with a load in flight and their parities, as bit masks (no local-memory array).
      uint32_t issued = 0, last = 0;
      int a_issued = -1;
      bool ok = true, skipped = false;
      int cur_ib = -1;
      for (int64_t t = t_begin; t < t_end && ok; ++t) {
        const int ib = (int)(t / a.tiles_n);
        const int i0 = ib * TILE_ROWS + (int)rank * BM;
        const int j0 = (int)(t % a.tiles_n) * BN + (PAIR ? (int)rank * PAIR_ROWS : 0);
        if (ib != cur_ib) {
          cur_ib = ib;
          if (!ptx::mbar_wait_bounded(a_empty, a_phase ^ 1, a.status, a.timeout_ns)) { ok = false; break; }
          if (leader) ptx::mbar_arrive_expect_tx(a_full, PEERS * (uint32_t)a.num_kc * CHUNK_BYTES);
          for (int kc = 0; kc < a.num_kc; ++kc) {
            uint8_t* am = stage_mem + kc * CHUNK_BYTES;
            if (PAIR) {
              ptx::tma_load_2d_pair(am, &tm_xhi, kc * BK, i0, a_full_c);
              ptx::tma_load_2d_pair(am + TILE_BYTES, &tm_xlo, kc * BK, i0, a_full_c);
            } else {
              ptx::tma_load_2d(am, &tm_xhi, kc * BK, i0, a_full);
              ptx::tma_load_2d(am + TILE_BYTES, &tm_xlo, kc * BK, i0, a_full);
            }
          }
          if (leader) a_issued = (int)a_phase;
          a_phase ^= 1;
        }
        for (int kc = 0; kc < a.num_kc; ++kc) {
          if (!ptx::mbar_wait_bounded(&empty[stage], phase ^ 1, a.status, a.timeout_ns)) { ok = false; break; }
          FTRACE(0, 10 + kc);
          if (a.debug_skip_first_load && !skipped && blockIdx.x == 0) {
            skipped = true;  // test hook: this stage never fills, so its consumer times out
          } else {
            uint8_t* bm = bring + stage * BSTAGE;
            if (leader) ptx::mbar_arrive_expect_tx(&full[stage], PEERS * BSTAGE);
            if (PAIR) {
              const uint32_t fc = ptx::map_to_rank(&full[stage], 0);
              ptx::tma_load_2d_pair(bm, &tm_yhi, kc * BK, j0, fc);
              ptx::tma_load_2d_pair(bm + BSTAGE / 2, &tm_ylo, kc * BK, j0, fc);
            } else {
              ptx::tma_load_2d(bm, &tm_yhi, kc * BK, j0, &full[stage]);
              ptx::tma_load_2d(bm + BSTAGE / 2, &tm_ylo, kc * BK, j0, &full[stage]);
            }
            if (leader) {
              issued |= 1u << stage;
              last = (last & ~(1u << stage)) | (phase << stage);
            }
          }
          if (++stage == NS) { stage = 0; phase ^= 1; }
        }
      }
      // Let every load issued land before the CTA exits (in the pair variant the leader's
      // barriers count both CTAs' bytes, and the final cluster barrier holds the peer until then).
      if (!ok) {
        for (int s = 0; s < NS; ++s)
          if (issued >> s & 1u)
            ptx::mbar_wait_bounded(&full[s], (last >> s) & 1u, a.status, a.timeout_ns);
        if (a_issued >= 0) ptx::mbar_wait_bounded(a_full, (uint32_t)a_issued, a.status, a.timeout_ns);
      }
    } else if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0, last = 0;
      bool ok = true;
      bool skipped = false;
      for (int64_t t = t_begin; t < t_end && ok; ++t) {
        const int i0 = (int)(t / a.tiles_n) * BM;
        const int j0 = (int)(t % a.tiles_n) * BN;
        for (int kc = 0; kc < a.num_kc; ++kc) {
          if (!ptx::mbar_wait_bounded(&empty[stage], phase ^ 1, a.status, a.timeout_ns)) {
            ok = false;
            break;
          }
          if (a.debug_skip_first_load && !skipped && blockIdx.x == 0) {
            skipped = true;  // test hook: this stage never fills, so its consumer times out
          } else {
            uint8_t* sm = stage_mem + stage * STAGE_BYTES;
            ptx::mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
            ptx::tma_load_2d(sm, &tm_xhi, kc * BK, i0, &full[stage]);
            ptx::tma_load_2d(sm + TILE_BYTES, &tm_xlo, kc * BK, i0, &full[stage]);
            ptx::tma_load_2d(sm + 2 * TILE_BYTES, &tm_yhi, kc * BK, j0, &full[stage]);
            ptx::tma_load_2d(sm + 3 * TILE_BYTES, &tm_ylo, kc * BK, j0, &full[stage]);
            issued |= 1u << stage;
            last = (last & ~(1u << stage)) | (phase << stage);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // Error path: let every load this thread issued land before the CTA exits.
        for (int s = 0; s < STAGES; ++s)
          if (issued >> s & 1u)
            ptx::mbar_wait_bounded(&full[s], (last >> s) & 1u, a.status, a.timeout_ns);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = ptx::idesc_tf32(PAIR ? 2 * BM : BM, BN, 0, 0);
      constexpr int NS = PAIR ? PB_STAGES : (RES_A ? RB_STAGES : STAGES);
      constexpr uint32_t BSTAGE = PAIR ? PCHUNK_BYTES : CHUNK_BYTES;
      // Pair variant: the commit arrives on the same barrier in both CTAs.
      auto commit = [](uint64_t* bar) {
        if (PAIR) ptx::mma_commit_pair(bar);
        else ptx::mma_commit(bar);
      };
      int stage = 0;
      uint32_t phase = 0, a_phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      int cur_ib = -1;
      for (int64_t t = t_begin; t < t_end && ok; ++t) {
        const int ib = (int)(t / a.tiles_n);
        if (RES_A && ib != cur_ib) {
          cur_ib = ib;
          // X in TMEM: the previous row block's MMAs must be done before its X is overwritten.
          if (A_TMEM && !ptx::mbar_wait_bounded(a_empty, a_phase ^ 1, a.status, a.timeout_ns)) { ok = false; break; }
          if (!ptx::mbar_wait_bounded(a_full, a_phase, a.status, a.timeout_ns)) { ok = false; break; }
          a_phase ^= 1;
          if (A_TMEM) {
            ptx::tc_fence_after();
            for (int kc = 0; kc < a.num_kc; ++kc) {
              const uint32_t xb = ptx::smem_u32(stage_mem + kc * CHUNK_BYTES);
#pragma unroll
              for (int k = 0; k < BK / 8; ++k) {
                const uint32_t col = (uint32_t)(kc * (BK / 8) + k) * 8;
                ptx::tmem_cp_128x256b(tmem + XCOL + col, ptx::smem_desc(xb + 32 * k, 16, 1024, 2));
                ptx::tmem_cp_128x256b(tmem + XCOL + 64 + col,
                                      ptx::smem_desc(xb + TILE_BYTES + 32 * k, 16, 1024, 2));
              }
            }
          }
        }
        if (!ptx::mbar_wait_bounded(&acc_empty[acc], acc_phase ^ 1, a.status, a.timeout_ns)) {
          ok = false;
          break;
        }
        FTRACE(1, 10);
        ptx::tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * BN);
        for (int kc = 0; kc < a.num_kc; ++kc) {
          if (!ptx::mbar_wait_bounded(&full[stage], phase, a.status, a.timeout_ns)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          // Operand bases: A = X hi|lo, B = Y hi|lo of this K chunk.
          const uint32_t abase = RES_A ? ptx::smem_u32(stage_mem + kc * CHUNK_BYTES)
                                       : ptx::smem_u32(stage_mem + stage * STAGE_BYTES);
          const uint32_t bbase =
              RES_A ? ptx::smem_u32(stage_mem + RA_CHUNKS * CHUNK_BYTES + stage * BSTAGE)
                    : abase + 2 * TILE_BYTES;
          const uint32_t blo_off = RES_A ? BSTAGE / 2 : TILE_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 8; ++k) {
            const uint32_t off = (uint32_t)k * 32;  // 8 tf32 = 32 bytes along the swizzled row
            const uint64_t ahi = ptx::smem_desc(abase + off, 16, 1024, 2);
            const uint64_t alo = ptx::smem_desc(abase + TILE_BYTES + off, 16, 1024, 2);
            const uint64_t bhi = ptx::smem_desc(bbase + off, 16, 1024, 2);
            const uint64_t blo = ptx::smem_desc(bbase + blo_off + off, 16, 1024, 2);
#ifdef RBF_TRACE
            if (a.ablate == 1 || a.ablate == 4) continue;
#endif
            if (A_TMEM) {
              const uint32_t xa = tmem + XCOL + (uint32_t)(kc * (BK / 8) + k) * 8;
              ptx::mma_tf32_ts(d, xa, bhi, idesc, (kc | k) != 0);
              ptx::mma_tf32_ts(d, xa, blo, idesc, 1);
              ptx::mma_tf32_ts(d, xa + 64, bhi, idesc, 1);
            } else if (PAIR) {
              ptx::mma_tf32_ss_pair(d, ahi, bhi, idesc, (kc | k) != 0);
              ptx::mma_tf32_ss_pair(d, ahi, blo, idesc, 1);
              ptx::mma_tf32_ss_pair(d, alo, bhi, idesc, 1);
            } else {
              ptx::mma_tf32_ss(d, ahi, bhi, idesc, (kc | k) != 0);
              ptx::mma_tf32_ss(d, ahi, blo, idesc, 1);
              ptx::mma_tf32_ss(d, alo, bhi, idesc, 1);
            }
          }
          commit(&empty[stage]);
          if (++stage == NS) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        commit(&acc_full[acc]);
        FTRACE(1, 20);
        // Last tile of this row block: the resident X may be replaced once these MMAs finish.
        if (RES_A && (t + 1 == t_end || (int)((t + 1) / a.tiles_n) != ib)) commit(a_empty);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      // Teardown: every MMA issued so far must finish before TMEM is freed.
      commit(drain);
      ptx::mbar_wait_bounded(drain, 0, a.status, a.timeout_ns);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;              // TMEM lane quadrant this warp may access
    const int h = (warp - 2) >> 2;       // column group of the tile (32 * CPW columns)
    uint8_t* buf = epi_mem + (warp - 2) * EPI_BYTES;
    int acc = 0;
    uint32_t acc_phase = 0;
    // The norms of the next tile are loaded one whole tile ahead (the first touch of a column
    // block after an L2 flush misses to DRAM): each lane holds ||y||^2 of its own column in the
    // two 32-column chunks and the chunk's 32 values are broadcast with warp shuffles.
    // (The dot-product epilogue uses no norms.)
    auto load_yn = [&](int64_t t, int c) {
      const int64_t j = (t % a.tiles_n) * BN + h * (32 * CPW) + c * 32 + lane;
      return !DOT && j < a.M ? __ldg(a.yn + j) : 0.f;
    };
    auto load_xn = [&](int64_t t) {
      const int64_t i = (t / a.tiles_n) * TILE_ROWS + rank * BM + q * 32 + lane;
      return !DOT && i < a.N ? __ldg(a.xn + i) : 0.f;
    };
    float xnext = 0.f, ynext[CPW];
#pragma unroll
    for (int c = 0; c < CPW; ++c) ynext[c] = 0.f;
    if (t_begin < t_end) {
      xnext = load_xn(t_begin);
#pragma unroll
      for (int c = 0; c < CPW; ++c) ynext[c] = load_yn(t_begin, c);
    }
    for (int64_t t = t_begin; t < t_end; ++t) {
      const int64_t i0 = (t / a.tiles_n) * TILE_ROWS + rank * BM;
      const int64_t j0 = (t % a.tiles_n) * BN;
      if (!ptx::mbar_wait_bounded(&acc_full[acc], acc_phase, a.status, a.timeout_ns)) break;
      if (lane == 0 && (warp == 2 || warp == 9)) FTRACE(warp == 2 ? 2 : 3, 30);
      ptx::tc_fence_after();
      const int64_t i = i0 + q * 32 + lane;
      const float xi = xnext;
      float ylane[CPW];
#pragma unroll
      for (int c = 0; c < CPW; ++c) ylane[c] = ynext[c];
      if (t + 1 < t_end) {
        xnext = load_xn(t + 1);
#pragma unroll
        for (int c = 0; c < CPW; ++c) ynext[c] = load_yn(t + 1, c);
      }
      // All of this warp's accumulator columns are read at once (one TMEM round trip) and the
      // accumulator goes back to the MMA issuer before the math.
      uint32_t vall[CPW][32];
#pragma unroll
      for (int c = 0; c < CPW; ++c)
        ptx::tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + h * (32 * CPW) + c * 32),
                       vall[c]);
      ptx::tmem_wait_ld();
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR) ptx::mbar_arrive_cluster(ptx::map_to_rank(&acc_empty[acc], 0));
        else ptx::mbar_arrive(&acc_empty[acc]);
        if (warp == 2 || warp == 9) FTRACE(warp == 2 ? 2 : 3, 50);
      }
#pragma unroll
      for (int c = 0; c < CPW; ++c) {
        const int col0 = h * (32 * CPW) + c * 32;
        const uint32_t (&v)[32] = vall[c];
        const int64_t j = j0 + col0;
#ifdef RBF_TRACE
        if (a.ablate == 2 || a.ablate == 4) continue;
#endif
        float out[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          if (DOT) {
            out[e] = __uint_as_float(v[e]);
          } else {
            const float yj = __shfl_sync(0xffffffffu, ylane[c], e);
            const float d2 = fmaxf(fmaf(-2.f, __uint_as_float(v[e]), xi + yj), 0.f);
            out[e] = exp2_approx(d2 * a.scale);
          }
        }
#ifdef RBF_TRACE
        if (lane == 0 && warp == 2) FTRACE(2, 70 + c);
        if (a.ablate == 3) { if (out[lane] == 12345.f) a.K[0] = 1.f; continue; }
#endif
#ifdef RBF_FWD_DIRECT
        if (TMA_STORE && i < a.N) {
          float4* krow = reinterpret_cast<float4*>(a.K + i * a.M + j);
#pragma unroll
          for (int c4 = 0; c4 < 8; ++c4)
            krow[c4] = make_float4(out[4 * c4], out[4 * c4 + 1], out[4 * c4 + 2], out[4 * c4 + 3]);
          if (warp == 2 || warp == 9) FTRACE(warp == 2 ? 2 : 3, 40 + c);
        } else
#endif
        if (TMA_STORE) {
          // EPI_BUFS staging blocks per warp, reused once the store that last read them is done.
          uint8_t* blk = buf + (c % EPI_BUFS) * (32 * 32 * 4);
          if (lane == 0) ptx::bulk_wait_read<EPI_BUFS - 1>();
          if (lane == 0 && warp == 2) FTRACE(2, 80 + c);
          __syncwarp();
          uint8_t* row = blk + lane * 128;
#pragma unroll
          for (int c4 = 0; c4 < 8; ++c4) {
            *reinterpret_cast<float4*>(row + ((c4 ^ (lane & 7)) << 4)) =
                make_float4(out[4 * c4], out[4 * c4 + 1], out[4 * c4 + 2], out[4 * c4 + 3]);
          }
          ptx::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            ptx::tma_store_2d(&tm_k, blk, (int32_t)j, (int32_t)(i0 + q * 32));
            if (warp == 2 || warp == 9) FTRACE(warp == 2 ? 2 : 3, 40 + c);
            ptx::bulk_commit();
          }
        } else if (i < a.N) {
          float* krow = a.K + i * a.M;
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (j + e < a.M) krow[j + e] = out[e];
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if (TMA_STORE && lane == 0) ptx::bulk_wait<0>();
  }

  ptx::griddep_launch_dependents();
  ptx::tc_fence_before();
  __syncthreads();
  // Pair variant: the leader's MMAs read the peer's shared memory and write its TMEM, and the
  // peer arrives on the leader's barriers; neither CTA leaves (or frees TMEM) before both are done.
  if (PAIR) ptx::cluster_sync();
#ifdef RBF_TRACE
  if (threadIdx.x == 0 && blockIdx.x < 1024) g_fwd_span[blockIdx.x][1] = ptx::globaltimer();
#endif
  if (warp == 1) {
    ptx::tc_fence_after();
    if (PAIR) ptx::tmem_dealloc_pair(tmem, TCOLS);
    else ptx::tmem_dealloc(tmem, TCOLS);
  }
}

// ----------------------------------------------------------------------- host side

}  // namespace

// 2-D fp32 tensor map: `rows` x `cols` row-major with row pitch `pitch_elems`, box
// box_cols x box_rows, zero fill out of bounds.  `swizzle` is CU_TENSOR_MAP_SWIZZLE_128B for
// K-major MMA operands and staging tiles, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B for MN-major
// tf32 operands (the only shared-memory layout the tensor core accepts for those).
// cuTensorMapEncodeTiled is reached through the runtime's driver entry-point table, so the
// library loads (and its host-side checks run) on machines without a CUDA driver.
using EncodeTiledFn = decltype(&cuTensorMapEncodeTiled);

static EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

bool make_tmap_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                  uint64_t pitch_elems, uint32_t box_cols, uint32_t box_rows, int swizzle) {
  const EncodeTiledFn enc = encode_tiled();
  if (enc == nullptr) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {pitch_elems * sizeof(float)};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, (CUtensorMapSwizzle)swizzle,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int device_sm_count() {
  int dev = 0, n = kSmCount;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : kSmCount;
}

// How many two-CTA clusters of the pair forward fit on the device at once (0 = do not use the
// pair variant: fewer than half the SMs could take part).  Cached per device.
static cudaError_t pair_capacity(int* clusters) {
  static int cached[64];
  static bool known[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 64 && known[dev]) {
    *clusters = cached[dev];
    return cudaSuccess;
  }
  auto kernel = rbf_fwd_tc_kernel<true, true, true>;
  if ((e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)SMEM_BYTES_RA)) != cudaSuccess)
    return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * (unsigned)device_sm_count());
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = SMEM_BYTES_RA;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if ((e = cudaOccupancyMaxActiveClusters(&n, kernel, &cfg)) != cudaSuccess) return e;
  if (2 * n < device_sm_count() / 2) n = 0;
  if (dev < 64) {
    cached[dev] = n;
    known[dev] = true;
  }
  *clusters = n;
  return cudaSuccess;
}

cudaError_t launch_forward_tc(const float* X, const float* Y, float* K, int64_t N, int64_t M,
                              int64_t D, float gamma, void* ws, const WaitConfig& wc,
                              cudaStream_t stream, Epi epi) {
  (void)X; (void)Y;
  if (N == 0 || M == 0) return cudaSuccess;
  const PrepLayout L = prep_layout(N, M, D);
  CUtensorMap txh, txl, tyh, tyl, tk;
  if (!make_tmap_2d(&txh, ws_at<float>(ws, L.xhi), N, L.Dp, L.Dp, BK, 128) ||
      !make_tmap_2d(&txl, ws_at<float>(ws, L.xlo), N, L.Dp, L.Dp, BK, 128) ||
      !make_tmap_2d(&tyh, ws_at<float>(ws, L.yhi), M, L.Dp, L.Dp, BK, 128) ||
      !make_tmap_2d(&tyl, ws_at<float>(ws, L.ylo), M, L.Dp, L.Dp, BK, 128))
    return cudaErrorInvalidValue;
  const bool tma_store = (M % 4) == 0;
  if (tma_store) {
    if (!make_tmap_2d(&tk, K, N, M, M, 32, 32)) return cudaErrorInvalidValue;
  } else {
    tk = txh;  // unused by the direct-store epilogue
  }
  FwdArgs a;
  a.xn = ws_at<float>(ws, L.xn);
  a.yn = ws_at<float>(ws, L.yn);
  a.K = K;
  a.N = N;
  a.M = M;
  a.tiles_m = (int)ceil_div(N, BM);
  a.tiles_n = (int)ceil_div(M, BN);
  a.num_kc = (int)(L.Dp / BK);
  a.scale = (float)(-(double)gamma * 1.4426950408889634);
  a.status = ws_at<int>(ws, L.status);
  a.timeout_ns = wc.timeout_ns;
  a.debug_skip_first_load = wc.debug_skip_first_load;
  a.ablate = 0;
#ifdef RBF_TRACE
  if (const char* ab = std::getenv("RBF_ABLATE")) a.ablate = std::atoi(ab);
#endif
  cudaError_t e;
  const bool res_a = a.num_kc <= RA_CHUNKS;
  // Pair variant: D <= 64, TMA-stored K, and enough two-CTA clusters resident at once.
  int pair_clusters = 0;
  if (res_a && tma_store && wc.fwd_pair && epi == Epi::kRbf) {
    if ((e = pair_capacity(&pair_clusters)) != cudaSuccess) return e;
  }
  if (pair_clusters > 0) {
    CUtensorMap tyh2, tyl2;  // 64-row Y boxes: each CTA of the pair loads half of a Y tile
    if (!make_tmap_2d(&tyh2, ws_at<float>(ws, L.yhi), M, L.Dp, L.Dp, BK, PAIR_ROWS) ||
        !make_tmap_2d(&tyl2, ws_at<float>(ws, L.ylo), M, L.Dp, L.Dp, BK, PAIR_ROWS))
      return cudaErrorInvalidValue;
    a.tiles_m = (int)ceil_div(N, 2 * BM);
    const int64_t tiles = (int64_t)a.tiles_m * a.tiles_n;
    const int clusters = (int)std::min<int64_t>(tiles, pair_clusters);
    auto kernel = rbf_fwd_tc_kernel<true, true, true>;
    if ((e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)SMEM_BYTES_RA)) != cudaSuccess)
      return e;
    e = launch_kernel_cluster(kernel, dim3(2 * clusters), dim3(THREADS), SMEM_BYTES_RA, 2, stream,
                              txh, txl, tyh2, tyl2, tk, a);
  } else {
    const int64_t tiles = (int64_t)a.tiles_m * a.tiles_n;
    const int grid = (int)std::min<int64_t>(tiles, device_sm_count());
    auto launch = [&](auto kernel, size_t smem) -> cudaError_t {
      cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
      if (err != cudaSuccess) return err;
      return launch_kernel(kernel, dim3(grid), dim3(THREADS), smem, stream, txh, txl, tyh, tyl,
                           tk, a);
    };
    if (epi == Epi::kDot) {
      if (tma_store)
        e = res_a ? launch(rbf_fwd_tc_kernel<true, true, false, true>, SMEM_BYTES_RA)
                  : launch(rbf_fwd_tc_kernel<true, false, false, true>, SMEM_BYTES);
      else
        e = res_a ? launch(rbf_fwd_tc_kernel<false, true, false, true>, SMEM_BYTES_RA)
                  : launch(rbf_fwd_tc_kernel<false, false, false, true>, SMEM_BYTES);
    } else if (tma_store) {
      e = res_a ? launch(rbf_fwd_tc_kernel<true, true, false>, SMEM_BYTES_RA)
                : launch(rbf_fwd_tc_kernel<true, false, false>, SMEM_BYTES);
    } else {
      e = res_a ? launch(rbf_fwd_tc_kernel<false, true, false>, SMEM_BYTES_RA)
                : launch(rbf_fwd_tc_kernel<false, false, false>, SMEM_BYTES);
    }
  }
  if (e != cudaSuccess) return e;
  note_launches(1);
  return cudaGetLastError();
}

}  // namespace rbf

#ifdef RBF_TRACE
extern "C" __attribute__((visibility("default"))) int rbf_debug_fwd_spans(unsigned long long* out) {
  return (int)cudaMemcpyFromSymbol(out, rbf::g_fwd_span, sizeof(rbf::g_fwd_span));
}
extern "C" __attribute__((visibility("default"))) int rbf_debug_fwd_spans_clear() {
  static unsigned long long z[1024][3];
  return (int)cudaMemcpyToSymbol(rbf::g_fwd_span, z, sizeof(z));
}
#endif

#ifdef RBF_TRACE
extern "C" __attribute__((visibility("default"))) int rbf_debug_fwd_trace(unsigned long long* out,
                                                                          int* n) {
  cudaMemcpyFromSymbol(out, rbf::g_ftrace, sizeof(rbf::g_ftrace));
  cudaMemcpyFromSymbol(n, rbf::g_ftrace_n, sizeof(rbf::g_ftrace_n));
  int z[4] = {0, 0, 0, 0};
  return (int)cudaMemcpyToSymbol(rbf::g_ftrace_n, z, sizeof(z));
}
#endif
