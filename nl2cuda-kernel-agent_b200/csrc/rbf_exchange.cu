// rbf_exchange.cu -- completes a row-sharded backward whose dY partial each rank accumulated
// into its own peer-visible buffer: the all-reduce of dY done by this library over NVLink /
// NVSwitch peer memory, with no library collective on the data path.
//
// Per step, with slot s = ctr % kDySlots of every rank's buffer (its dY partial, M x D, zeroed by
// the backward's zeroing pass before the backward added into it):
//   1. barrier A: store epoch 2*ctr + 1 into flags[r][rank] of every rank r (release, system
//      scope), wait until this rank's flags[rank][r] >= 2*ctr + 1 for every r -- every partial
//      is complete;
//   one-phase (default up to 8 ranks):
//   2'. every rank sums slot s over all ranks (peer loads) straight into its dY;
//   two-phase (less NVLink traffic per rank, one more barrier):
//   2. for the 128-row j-blocks this rank owns (jb % world == rank), sum slot s over all ranks
//      and write the sum back into this rank's slot, in place;
//   3. barrier B (epoch 2*ctr + 2), released by the last block to finish step 2;
//   4. gather: every row of dY from its owner's slot;
//   5. the last block to finish advances ctr.
// A barrier that runs out (a peer that never arrives) is sticky: the block sets tickets[2], the
// counter is not advanced, and every later exchange on these buffers skips its work and
// reports RBF_ERR_TIMEOUT until the caller rebuilds the buffers (zeroed flags and counters).
// Two slots suffice: slot s is next zeroed (and added into, by its own rank only) two steps
// later, after every rank has passed barrier A of the step in between, which each rank enters
// only after its gather of this step.  No host synchronisation, and a captured CUDA graph of the
// step can be replayed because the slot comes from device memory.  The waits are the only
// cross-GPU spins; they are bounded, record RBF_ERR_TIMEOUT in the status word and skip the rest
// on expiry.  Plain peer loads and stores only (no multimem, no TMA).
#include <algorithm>

#include "rbf_common.cuh"
#include "rbf_kernels.cuh"
#include "rbf_ptx.cuh"

namespace rbf {
namespace {

constexpr int kBlockRows = 128;  // j-block height of the backward's tiles (dY ownership unit)
constexpr int kThreads = 256;
constexpr int kChunkRows = 16;        // unit of work: 16 rows of dY (one float4 per thread at D = 64)

#ifdef RBF_TRACE
__device__ unsigned long long g_xchg_trace[8];
#define XT(k) do { if (blockIdx.x == 0 && threadIdx.x == 0) g_xchg_trace[k] = ptx::globaltimer(); } while (0)
#else
#define XT(k) ((void)0)
#endif

template <typename T>
__device__ __forceinline__ T* pick(T* const (&arr)[kMaxRanks], int r) {
  T* p = arr[0];
#pragma unroll
  for (int k = 1; k < kMaxRanks; ++k)
    if (r == k) p = arr[k];
  return p;
}

__device__ __forceinline__ void store_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int load_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Thread 0 of the block: wait until every rank's flag reached `epoch` (bounded).
__device__ bool wait_all(const ExchangeArgs& a, int epoch) {
  const int* own = pick(a.flags, a.route.rank);
  const uint64_t start = ptx::globaltimer();
  for (int r = 0; r < a.route.world; ++r) {
    while (load_acquire_sys(own + r) < epoch) {
      if (ptx::globaltimer() - start > a.timeout_ns) {
        atomicExch(a.status, RBF_ERR_TIMEOUT);
        return false;
      }
    }
  }
  return true;
}

// Release store of `epoch` into every rank's flag slot of this rank.  Release is cumulative:
// every write this thread has observed (the previous kernel's, and this grid's through the
// ticket below) is visible to a rank that acquires the flag.
__device__ void signal_all(const ExchangeArgs& a, int epoch) {
  for (int r = 0; r < a.route.world; ++r) store_release_sys(pick(a.flags, r) + a.route.rank, epoch);
}

// The float4 range [k0, k1) of 16-row chunk `c` of dY.
__device__ __forceinline__ void chunk_range(int64_t c, const ExchangeArgs& a, int64_t& k0,
                                            int64_t& k1) {
  const int64_t D4 = a.D / 4;
  const int64_t r0 = c * kChunkRows;
  k0 = r0 * D4;
  k1 = min(r0 + kChunkRows, a.M) * D4;
}

// out[k] = sum over ranks r of slot_r[k] for k in [k0, k1): every peer's load issued together.
__device__ __forceinline__ void sum_ranks(const ExchangeArgs& a, int64_t slot, int64_t k0,
                                          int64_t k1, float4* out) {
  for (int64_t k = k0 + threadIdx.x; k < k1; k += kThreads) {
    float4 v[kMaxRanks];
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < a.route.world) v[r] = reinterpret_cast<const float4*>(pick(a.route.bufs, r) + slot)[k];
    float4 s = v[0];
#pragma unroll
    for (int r = 1; r < kMaxRanks; ++r)
      if (r < a.route.world) {
        s.x += v[r].x; s.y += v[r].y; s.z += v[r].z; s.w += v[r].w;
      }
    out[k] = s;
  }
}

__global__ void __launch_bounds__(kThreads) rbf_dy_exchange_kernel(const ExchangeArgs a) {
  XT(0);
  ptx::griddep_wait();  // this rank's backward (its partial) is complete
  XT(1);
  __shared__ int s_ctr, s_ok;
  if (threadIdx.x == 0) {
    s_ctr = *reinterpret_cast<volatile int*>(a.ctr);
    // An earlier exchange on these buffers timed out: the ranks' epochs no longer agree.
    s_ok = reinterpret_cast<volatile unsigned*>(a.tickets)[2] == 0u;
    if (!s_ok) atomicExch(a.status, RBF_ERR_TIMEOUT);
  }
  __syncthreads();
  const bool usable = s_ok != 0;
  const int ctr = s_ctr;
  const int world = a.route.world, rank = a.route.rank;
  const int64_t slot = (int64_t)(ctr % kDySlots) * a.M * a.D;
  const int64_t chunks = (a.M + kChunkRows - 1) / kChunkRows;
  const int per_block = kBlockRows / kChunkRows;  // chunks per 128-row j-block
  const bool two_phase = world > a.one_phase_max;

  // 1. Barrier A: every rank's partial is complete.
  if (threadIdx.x == 0 && usable) {
    if (blockIdx.x == 0) signal_all(a, 2 * ctr + 1);
    XT(2);
    s_ok = wait_all(a, 2 * ctr + 1);
    if (!s_ok) atomicExch(&a.tickets[2], 1u);
    XT(3);
  }
  __syncthreads();
  bool ok = s_ok != 0;

  if (!two_phase) {
    // 2'. Every rank sums every rank's partial for all rows (one barrier; (world - 1) x M x D
    //     floats cross NVLink per rank).
    if (ok)
      for (int64_t c = blockIdx.x; c < chunks; c += gridDim.x) {
        int64_t k0, k1;
        chunk_range(c, a, k0, k1);
        sum_ranks(a, slot, k0, k1, reinterpret_cast<float4*>(a.dY));
      }
    XT(4);
  } else {
    // 2. The owner of each j-block (jb % world) sums it over all ranks, in place in its slot.
    if (ok) {
      float4* mine = reinterpret_cast<float4*>(pick(a.route.bufs, rank) + slot);
      const int64_t jblocks = (a.M + kBlockRows - 1) / kBlockRows;
      const int64_t owned = jblocks > rank ? (jblocks - rank + world - 1) / world : 0;
      for (int64_t u = blockIdx.x; u < owned * per_block; u += gridDim.x) {
        const int64_t c = (rank + (u / per_block) * world) * per_block + u % per_block;
        if (c >= chunks) continue;
        int64_t k0, k1;
        chunk_range(c, a, k0, k1);
        sum_ranks(a, slot, k0, k1, mine);
      }
    }
    __syncthreads();
    XT(4);
    // 3. Barrier B, released by the last block to finish its reduction.
    if (threadIdx.x == 0) {
      if (ok) {
        __threadfence();
        const unsigned t = atomicAdd(&a.tickets[0], 1u);
        if (t == gridDim.x - 1) {
          a.tickets[0] = 0u;
          __threadfence();
          signal_all(a, 2 * ctr + 2);
        }
        s_ok = wait_all(a, 2 * ctr + 2);
        if (!s_ok) atomicExch(&a.tickets[2], 1u);
        XT(5);
      }
    }
    __syncthreads();
    ok = ok && s_ok != 0;
    // 4. Gather every row of dY from its owner's slot.
    if (ok) {
      float4* out = reinterpret_cast<float4*>(a.dY);
      for (int64_t c = blockIdx.x; c < chunks; c += gridDim.x) {
        const float4* src = reinterpret_cast<const float4*>(
            pick(a.route.bufs, (int)((c / per_block) % world)) + slot);
        int64_t k0, k1;
        chunk_range(c, a, k0, k1);
        for (int64_t k = k0 + threadIdx.x; k < k1; k += kThreads) out[k] = src[k];
      }
    }
  }
  __syncthreads();
  XT(6);

  // 5. Advance the step counter once every block has read it and finished, unless a barrier
  //    ran out (then the counter stays, and the sticky flag stops later exchanges).
  if (threadIdx.x == 0) {
    __threadfence();  // this block's sticky-flag write before its ticket
    const unsigned t = atomicAdd(&a.tickets[1], 1u);
    if (t == gridDim.x - 1) {
      a.tickets[1] = 0u;
      __threadfence();
      if (reinterpret_cast<volatile unsigned*>(a.tickets)[2] == 0u) *a.ctr = ctr + 1;
    }
  }
}

}  // namespace

cudaError_t launch_dy_exchange(const ExchangeArgs& a, cudaStream_t stream) {
  if (a.route.world <= 0 || a.route.world > kMaxRanks || a.D % 4 != 0) return cudaErrorInvalidValue;
  // Every block waits on barriers that other blocks release, so all blocks must be resident at
  // once: at most one block per SM (the kernel holds no shared memory to speak of).
  const int64_t chunks = (a.M + kChunkRows - 1) / kChunkRows;
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(chunks, device_sm_count()));
  cudaError_t e = launch_kernel(rbf_dy_exchange_kernel, dim3(blocks), dim3(kThreads), 0, stream, a);
  if (e != cudaSuccess) return e;
  note_launches(1);
  return cudaGetLastError();
}

}  // namespace rbf

#ifdef RBF_TRACE
extern "C" __attribute__((visibility("default"))) int rbf_debug_xchg_trace(unsigned long long* out) {
  return (int)cudaMemcpyFromSymbol(out, rbf::g_xchg_trace, sizeof(rbf::g_xchg_trace));
}
#endif
