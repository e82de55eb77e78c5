// Fused all-reduce of the row-parallel decode projections at TP > 1, shared by the
// staged (gemv_async.cu) and dynamic (gemv_dynamic.cu) GEMV kernels.
#pragma once

#include "pim_common.cuh"
#include "pim_kernels.h"

namespace pim {

constexpr unsigned long long kAllReduceWaitNs = 1000000000ull;  // bound of the peer wait

__device__ __forceinline__ unsigned long long ar_gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- fused all-reduce (row-parallel projections at TP > 1) --------------------------
// The partial y_rank = x . W_rank^T (rounded to T, as the reference's linear output) is
// stored into row `rank` of slot epoch & 1 of every rank's exchange buffer (layout of
// p2p.cu).  The last CTA of this rank to finish (ticket 0) raises this rank's flag in
// every buffer; every CTA then waits (bounded) for all ranks' flags and, for its own
// output columns, adds the ranks' partials in rank order (rounded after every add, the
// sequential sum of comm/lowering.py:137-150), then y = residual + sum (the following
// `add` node) and, when asked, the sum itself.  All CTAs of the grid are resident at
// once (the launchers size the grid by the occupancy API), so the grid-wide wait cannot
// starve.  The last CTA
// out (ticket 1) resets the tickets and advances the epoch -- also after a wait gave up
// (error word raised, sum skipped), so that the tickets never stay dirty and every rank
// consumes the epoch of every call.
//
// The kernel is launched with programmatic dependent launch (its weight prologue
// overlaps the previous kernel) but lets its dependents start only at its very end.
// With the trigger at the start, as in the other kernels, replays of a captured TP=2
// decode graph lost one call in four to the bounded wait while eager runs were clean;
// with the trigger at the end, or no programmatic launch at all, every call completed.

__device__ __forceinline__ void ar_st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int ar_ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <typename T>
__device__ __forceinline__ void ar_push(const P2PDev* pd, int slot, size_t idx, float v) {
  const T pv = from_f<T>(v);
  const size_t off = kP2PHeaderBytes + ((size_t)slot * pd->size + pd->rank) * pd->capacity_bytes + idx * sizeof(T);
  for (int q = 0; q < pd->size; ++q) *reinterpret_cast<T*>(static_cast<char*>(pd->bufs[q]) + off) = pv;
}

template <typename T>
__device__ void ar_reduce(const FusedArgs& a, const P2PDev* pd, int t_lo, int nt, int epoch, int slot) {
  __shared__ int s_ok;
  __threadfence_system();  // this thread's partial stores, before this CTA's ticket
  __syncthreads();
  if (threadIdx.x == 0) {
    s_ok = 1;
    if (atomicAdd(&pd->tickets[0], 1) == (int)gridDim.x - 1) {  // every partial of this rank is out
      __threadfence_system();
      for (int q = 0; q < pd->size; ++q)
        ar_st_release_sys(static_cast<int*>(pd->bufs[q]) + slot * kP2PMaxRanks + pd->rank, epoch);
    }
  }
  __syncthreads();
  if (threadIdx.x < pd->size) {
    const int* flag = static_cast<const int*>(pd->bufs[pd->rank]) + slot * kP2PMaxRanks + threadIdx.x;
    if (ar_ld_acquire_sys(flag) != epoch) {
      const unsigned long long t0 = ar_gtime();
      while (ar_ld_acquire_sys(flag) != epoch)
        if (ar_gtime() - t0 > kAllReduceWaitNs) {
          s_ok = 0;
          if (pd->err) atomicExch(pd->err, 1);
          break;
        }
    }
  }
  __syncthreads();
  const char* rows = static_cast<const char*>(pd->bufs[pd->rank]) + kP2PHeaderBytes +
                     (size_t)slot * pd->size * pd->capacity_bytes;
  const T* res = static_cast<const T*>(a.residual);
  for (int i = threadIdx.x; s_ok && i < nt * a.rows; i += blockDim.x) {
    const int tl = i / a.rows, r = i % a.rows;
    const size_t idx = (size_t)r * a.ncols + t_lo + tl;
    float acc = 0.f;
    for (int q = 0; q < pd->size; ++q)
      acc = rnd<T>(acc + to_f(__ldcg(reinterpret_cast<const T*>(rows + (size_t)q * pd->capacity_bytes) + idx)));
    if (a.ar_out) static_cast<T*>(a.ar_out)[idx] = from_f<T>(acc);
    static_cast<T*>(a.y)[idx] = from_f<T>(res ? to_f(__ldcg(res + idx)) + acc : acc);
  }
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(&pd->tickets[1], 1) == (int)gridDim.x - 1) {
    pd->tickets[0] = 0;
    pd->tickets[1] = 0;
    *pd->counter = epoch;
  }
}

}  // namespace pim
