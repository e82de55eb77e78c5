// One-shot all-reduce over NVLink peer memory for one process per GPU, and the CUDA
// IPC plumbing that maps the ranks' exchange buffers into each other's address space.
//
// Exchange buffer of every rank (the same layout everywhere):
//   [flags: 2 slots x kP2PMaxRanks ints][pad to 1 KB][data: 2 slots x size rows x capacity bytes]
// A call with epoch e (this rank's call counter + 1, kept in device memory so that a
// replayed CUDA graph advances it) uses slot e & 1:
//   1. every thread stores its share of my partial into row `rank` of the slot in every
//      rank's buffer (peer stores over NVLink; my own buffer included), then fences at
//      system scope;
//   2. after a CTA barrier, thread p release-stores e into flag[slot][rank] of rank p;
//   3. thread p waits (bounded) until flag[slot][p] of my buffer reads e;
//   4. the partials are added in rank order 0..size-1, fp32 add then round to the element
//      type after every add (the sequential sum of comm/lowering.py:137-150), and written
//      to every destination.
// A rank reaches epoch e + 2 (which reuses slot e & 1) only after every rank has raised
// its e + 1 flag, i.e. after every rank finished reading epoch e: two slots suffice.
// The wait gives up after 1 s of %globaltimer and raises *err; the sum is skipped but
// the counter still advances, so every rank consumes the epoch of every call.
// With a residual, the kernel also writes y = residual + sum (the fp32 add of the rounded
// sum, rounded once: the bits of pim_ordered_sum_add), replacing the `add` launch that
// follows the all_reduce.  The kernel is one CTA launched with programmatic dependent
// launch: it becomes resident while the projection before it runs and starts pushing as
// soon as that grid's results are visible (griddepcontrol.wait); its dependents wait for
// its completion the same way.

#include <cudaTypedefs.h>

#include <mutex>

#include "pim_common.cuh"
#include "pim_kernels.h"

namespace pim {

constexpr int kP2PThreads = 512;
constexpr unsigned long long kP2PWaitNs = 1000000000ull;

__device__ __forceinline__ unsigned long long p2p_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <typename T>
__global__ void __launch_bounds__(kP2PThreads) allreduce_p2p_kernel(P2PArgs a) {
  __shared__ int s_epoch, s_ok;
  pdl_trigger();
  pdl_wait();  // the partial, the counter and the destinations are the previous grids' business
  if (threadIdx.x == 0) {
    s_epoch = *reinterpret_cast<volatile int*>(a.counter) + 1;
    s_ok = 1;
  }
  __syncthreads();
  const int epoch = s_epoch, slot = epoch & 1;
  const int nvec = (int)(a.numel * sizeof(T) / 16);  // numel * sizeof(T) is a multiple of 16
  const size_t row_bytes = (size_t)a.capacity_bytes;
  const size_t data_off = kP2PHeaderBytes + (size_t)slot * a.size * row_bytes;

  // 1. push my partial into row `rank` of every rank's buffer
  const int4* src = static_cast<const int4*>(a.src);
  for (int p = 0; p < a.size; ++p) {
    int4* dst = reinterpret_cast<int4*>(static_cast<char*>(a.bufs[p]) + data_off + (size_t)a.rank * row_bytes);
    for (int i = threadIdx.x; i < nvec; i += blockDim.x) dst[i] = src[i];
  }
  __threadfence_system();
  __syncthreads();
  // 2. raise my flag in every buffer;  3. wait for every rank's flag in mine
  if (threadIdx.x < a.size) {
    int* peer_flags = static_cast<int*>(a.bufs[threadIdx.x]);
    st_release_sys(peer_flags + slot * kP2PMaxRanks + a.rank, epoch);
    const int* mine = static_cast<const int*>(a.bufs[a.rank]) + slot * kP2PMaxRanks + threadIdx.x;
    if (ld_acquire_sys(mine) != epoch) {
      const unsigned long long t0 = p2p_now();
      while (ld_acquire_sys(mine) != epoch) {
        if (p2p_now() - t0 > kP2PWaitNs) {
          s_ok = 0;
          if (a.err) atomicExch(a.err, 1);
          break;
        }
      }
    }
  }
  __syncthreads();
  // 4. rank-order sum, rounded after every add, written to every destination (skipped
  //    when a wait gave up; the epoch is consumed either way so the ranks stay in step)
  const char* rows = static_cast<const char*>(a.bufs[a.rank]) + data_off;
  for (int64_t i = threadIdx.x; s_ok && i < a.numel; i += blockDim.x) {
    float acc = 0.f;
    for (int r = 0; r < a.size; ++r) {
      // through L2: peers wrote these rows, and this SM may hold lines of an older epoch
      const T v = __ldcg(reinterpret_cast<const T*>(rows + (size_t)r * row_bytes) + i);
      acc = rnd<T>(acc + to_f(v));
    }
    const T out = from_f<T>(acc);
    for (int d = 0; d < a.ndst; ++d) static_cast<T*>(a.dst[d])[i] = out;
    if (a.residual)
      static_cast<T*>(a.y)[i] = from_f<T>(__fadd_rn(to_f(static_cast<const T*>(a.residual)[i]), acc));
  }
  __syncthreads();
  if (threadIdx.x == 0) *a.counter = epoch;
}

// ---- low-latency (LL) protocol ----------------------------------------------------------
// The same rank-order sum, with no fence and no flag of its own: every 32-bit word of a
// partial travels as one 64-bit store (low half the data word, high half the call's
// epoch) into row `rank` of slot epoch & 1 of every rank's exchange buffer.  A 64-bit
// aligned store is seen whole or not at all, so a reader that finds the current epoch in
// the high half holds that word's data; it polls each word of each rank (bounded by
// %globaltimer) and adds the ranks in order 0..size-1.  Slot reuse is safe for the same
// reason as above: a rank writes epoch e + 2 into slot e & 1 of my buffer only after it
// read my epoch e + 1 words, which I push after finishing my reads of epoch e.  Epochs
// start at 1 on zero-filled buffers.  A group runs either this protocol or the flag one
// on its buffers, never both (stale words of the other protocol are not epoch-tagged).

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

template <typename T>
__global__ void __launch_bounds__(kP2PThreads) allreduce_ll_kernel(P2PArgs a) {
  __shared__ int s_ok;
  pdl_trigger();
  pdl_wait();  // the partial, the counter and the destinations are the previous grids' business
  const unsigned epoch = (unsigned)(*reinterpret_cast<volatile int*>(a.counter) + 1);
  const int slot = epoch & 1;
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  const int nw = (int)(a.numel * sizeof(T) / 4);  // 32-bit data words
  const size_t row_bytes = (size_t)a.capacity_bytes;
  const size_t slot_off = kP2PHeaderBytes + (size_t)slot * a.size * row_bytes;
  const uint32_t* src = static_cast<const uint32_t*>(a.src);
  const unsigned long long tag = (unsigned long long)epoch << 32;
  // 1. push every word of my partial, tagged with the epoch, into every rank's row `rank`
  for (int i = threadIdx.x; i < nw; i += blockDim.x) {
    const unsigned long long v = tag | src[i];
    for (int p = 0; p < a.size; ++p) {
      auto* dst = reinterpret_cast<unsigned long long*>(static_cast<char*>(a.bufs[p]) + slot_off +
                                                        (size_t)a.rank * row_bytes);
      st_relaxed_sys_u64(dst + i, v);
    }
  }
  // 2. for each of my words: wait for every rank's word of this epoch, add in rank order
  constexpr int E = 4 / sizeof(T);  // elements per word
  const char* mine = static_cast<const char*>(a.bufs[a.rank]) + slot_off;
  for (int i = threadIdx.x; i < nw; i += blockDim.x) {
    float acc[E];
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] = 0.f;
    for (int q = 0; q < a.size && s_ok; ++q) {
      const auto* w = reinterpret_cast<const unsigned long long*>(mine + (size_t)q * row_bytes) + i;
      unsigned long long v = ld_relaxed_sys_u64(w);
      if ((unsigned)(v >> 32) != epoch) {
        const unsigned long long t0 = p2p_now();
        while ((unsigned)((v = ld_relaxed_sys_u64(w)) >> 32) != epoch) {
          if (!*reinterpret_cast<volatile int*>(&s_ok)) break;  // another thread gave up already
          if (p2p_now() - t0 > kP2PWaitNs) {
            s_ok = 0;
            if (a.err) atomicExch(a.err, 1);
            break;
          }
        }
        if ((unsigned)(v >> 32) != epoch) break;
      }
      const uint32_t d = (uint32_t)v;
      const T* el = reinterpret_cast<const T*>(&d);
#pragma unroll
      for (int e = 0; e < E; ++e) acc[e] = rnd<T>(acc[e] + to_f(el[e]));
    }
    if (!s_ok) continue;
    T outv[E];
#pragma unroll
    for (int e = 0; e < E; ++e) outv[e] = from_f<T>(acc[e]);
    const uint32_t ow = *reinterpret_cast<const uint32_t*>(outv);
    for (int d = 0; d < a.ndst; ++d) static_cast<uint32_t*>(a.dst[d])[i] = ow;
    if (a.residual) {
      const uint32_t rw = static_cast<const uint32_t*>(a.residual)[i];
      const T* r = reinterpret_cast<const T*>(&rw);
      T yv[E];
#pragma unroll
      for (int e = 0; e < E; ++e) yv[e] = from_f<T>(__fadd_rn(to_f(r[e]), acc[e]));
      static_cast<uint32_t*>(a.y)[i] = *reinterpret_cast<const uint32_t*>(yv);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) *a.counter = (int)epoch;
}

cudaError_t allreduce_ll(const P2PArgs& a, int dtype, cudaStream_t st) {
  if (a.size < 1 || a.size > kP2PMaxRanks || a.rank < 0 || a.rank >= a.size || a.ndst < 0 || a.ndst > kP2PMaxDst)
    return cudaErrorInvalidValue;
  const size_t es = dtype == BF16 ? 2 : 4;
  // 8 bytes of buffer per 4 bytes of data
  if ((a.numel * es) % 16 || (int64_t)(2 * a.numel * es) > a.capacity_bytes) return cudaErrorInvalidValue;
  if (a.residual && !a.y) return cudaErrorInvalidValue;
  if (dtype == BF16) return launch_pdl(allreduce_ll_kernel<__nv_bfloat16>, 1, kP2PThreads, 0, st, a);
  return launch_pdl(allreduce_ll_kernel<float>, 1, kP2PThreads, 0, st, a);
}

cudaError_t allreduce_p2p(const P2PArgs& a, int dtype, cudaStream_t st) {
  if (a.size < 1 || a.size > kP2PMaxRanks || a.rank < 0 || a.rank >= a.size || a.ndst < 0 || a.ndst > kP2PMaxDst)
    return cudaErrorInvalidValue;
  const size_t es = dtype == BF16 ? 2 : 4;
  if ((a.numel * es) % 16 || (int64_t)(a.numel * es) > a.capacity_bytes) return cudaErrorInvalidValue;
  if (a.residual && !a.y) return cudaErrorInvalidValue;
  if (dtype == BF16) return launch_pdl(allreduce_p2p_kernel<__nv_bfloat16>, 1, kP2PThreads, 0, st, a);
  return launch_pdl(allreduce_p2p_kernel<float>, 1, kP2PThreads, 0, st, a);
}

// ---- CUDA IPC ---------------------------------------------------------------------------

static PFN_cuMemGetAddressRange_v3020 address_range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &p, 3020, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
  });
  return fn;
}

cudaError_t ipc_export(const void* ptr, cudaIpcMemHandle_t* handle, int64_t* offset) {
  auto fn = address_range_fn();
  if (!fn) return cudaErrorNotSupported;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (fn(&base, &size, (CUdeviceptr)ptr) != CUDA_SUCCESS) return cudaErrorInvalidValue;
  const cudaError_t e = cudaIpcGetMemHandle(handle, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return e;
  *offset = (int64_t)((CUdeviceptr)ptr - base);
  return cudaSuccess;
}

}  // namespace pim
