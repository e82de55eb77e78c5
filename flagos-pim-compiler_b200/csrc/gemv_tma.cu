// Decode projections streamed through shared memory with the bulk-copy (TMA) engine.
//
// One persistent CTA per SM owns a contiguous, balanced range of tasks (a task is
// one weight row for PLAIN and two adjacent rows -- the pair-interleaved layout --
// for ROPE and SILU).  Each task is cut along K into SP pieces of at most ~12 KB;
// piece p of task t is "stage" i = (t - t_lo) * SP + p.  A producer thread issues
// the stages in order with cp.async.bulk into a ring of S shared-memory slots
// (mbarrier complete_tx), starting before griddepcontrol.wait so that, with
// programmatic dependent launch, the weight stream of this kernel overlaps the
// end of the previous one.  Task t belongs to consumer warp (t - t_lo) % 16, which
// walks its tasks' pieces in order, accumulates in registers, releases each slot
// as soon as it has read it, and runs the task's epilogue (plain / residual /
// RoPE + KV append / SiLU*up, the rounding of the register kernel in gemv.cu).
// Warps never wait for one another, and the producer stays up to S stages ahead
// of the slowest warp.  (No deadlock: the smallest unconsumed stage is always
// issued and its warp has consumed every earlier stage it owns.)
//
// A warp can be more than one ring lap ahead of the producer on its slot (with 16
// warps and 2 pieces per task, a warp's stages are 32 apart while the ring may hold
// 24), and an mbarrier parity wait cannot tell phase n from phase n-2.  So the
// producer publishes, per slot, the stage it last issued there (release store after
// the expect_tx), and a consumer first waits until its slot carries its own stage:
// by then the slot's previous phase is complete and the parity wait is exact.
//
// Every wait is bounded (1 s of %globaltimer): on expiry the kernel
// raises *a.err (when given) and the waiting thread stops working; consumers keep
// no CTA-wide barrier inside the stage loop, so no other thread can block on it.

#include <stdlib.h>

#include "gemv_epilogue.cuh"
#include "pim_common.cuh"
#include "pim_kernels.h"
#include "sm100.cuh"

namespace pim {

constexpr int kTmaWarps = 16;                      // consumer warps
constexpr int kTmaThreads = (kTmaWarps + 1) * 32;  // + one producer warp
constexpr int kPieceBytes = 12 * 1024;

struct TmaGeom {
  int sp;          // pieces per task
  int kp;          // K elements per piece (multiple of the 16-byte vector)
  int slots;       // ring depth
  int slot_bytes;  // bytes of one slot (UPR rows x kp elements)
  int x_bytes;     // bytes reserved for the activation rows (128-aligned)
};

__device__ __forceinline__ void st_release(int* p, int v) {
  asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
  return v;
}

// Bounded wait until the slot's published stage is `stage`; false after kWaitLimitNs.
__device__ __forceinline__ bool seq_wait(const int* seq, int stage) {
  if (ld_acquire(seq) == stage) return true;
  const unsigned long long t0 = gtime_ns();
  while (ld_acquire(seq) != stage)
    if (gtime_ns() - t0 > kWaitLimitNs) return false;
  return true;
}

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kTmaWarps * 32) : "memory"); }

template <typename T, int MODE, int RMAX, bool NORM>
__global__ void __launch_bounds__(kTmaThreads, 1) gemv_tma_kernel(FusedArgs a, TmaGeom g) {
  constexpr int UPR = (MODE == MODE_PLAIN) ? 1 : 2;  // weight rows per task
  constexpr int V = VecW<T>::n;
  int* err = a.err;
  extern __shared__ __align__(128) unsigned char smem[];
  T* xs = reinterpret_cast<T*>(smem);
  unsigned char* ring = smem + g.x_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + (size_t)g.slots * g.slot_bytes);
  uint64_t* empty = full + g.slots;
  int* seq = reinterpret_cast<int*>(empty + g.slots);  // stage last issued per slot
  __shared__ float rinv[RMAX];
  __shared__ float nred[kTmaWarps][RMAX];

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int K = a.K;
  const size_t row_bytes = (size_t)K * sizeof(T);
  const int ntasks = projection_tasks(a, MODE);
  const int t_lo = (int)(((long long)blockIdx.x * ntasks) / gridDim.x);
  const int t_hi = (int)(((long long)(blockIdx.x + 1) * ntasks) / gridDim.x);
  const int nst = (t_hi - t_lo) * g.sp;

  if (threadIdx.x == 0) {
    for (int s = 0; s < g.slots; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      seq[s] = -1;
    }
    mbar_fence_init();
  }
  __syncthreads();
  pdl_trigger();

  if (warp == kTmaWarps) {
    // ---- producer: stream this CTA's weight pieces (independent of the predecessor)
    if (lane == 0) {
      for (int i = 0; i < nst; ++i) {
        const int slot = i % g.slots;
        if (i >= g.slots && !mbar_wait(&empty[slot], ((i / g.slots) - 1) & 1)) {
          if (err) atomicExch(err, 1);
          break;
        }
        const int t = t_lo + i / g.sp, p = i % g.sp;
        const int k0 = p * g.kp;
        const int kn = min(g.kp, K - k0);
        const uint32_t piece = (uint32_t)(kn * sizeof(T));
        mbar_expect_tx(&full[slot], piece * UPR);
        st_release(&seq[slot], i);
        const char* src = static_cast<const char*>(a.w) + (size_t)t * UPR * row_bytes + (size_t)k0 * sizeof(T);
        unsigned char* dst = ring + (size_t)slot * g.slot_bytes;
#pragma unroll
        for (int q = 0; q < UPR; ++q) bulk_g2s(dst + (size_t)q * g.kp * sizeof(T), src + q * row_bytes, piece, &full[slot]);
      }
    }
    return;
  }

  // ---- consumers ---------------------------------------------------------------
  pdl_wait();
  const T* __restrict__ x = static_cast<const T*>(a.x);
  const int rows = a.rows;
  if (NORM) {
    const T* __restrict__ lw = static_cast<const T*>(a.ln_w);
#pragma unroll
    for (int r = 0; r < RMAX; ++r) {
      float ss = 0.f;
      if (r < rows)
        for (int k = threadIdx.x; k < K; k += kTmaWarps * 32) {
          const float xv = to_f(x[(size_t)r * K + k]);
          ss = fmaf(xv, xv, ss);
        }
      ss = warp_sum(ss);
      if (lane == 0) nred[warp][r] = ss;
    }
    consumer_sync();
    if (threadIdx.x < RMAX) {
      float s = 0.f;
      for (int i = 0; i < kTmaWarps; ++i) s += nred[i][threadIdx.x];
      rinv[threadIdx.x] = rsqrtf(s / (float)K + a.eps);
    }
    consumer_sync();
    for (int r = 0; r < rows; ++r)
      for (int k = threadIdx.x; k < K; k += kTmaWarps * 32) {
        const float y = rnd<T>(to_f(x[(size_t)r * K + k]) * rinv[r]);
        xs[(size_t)r * K + k] = from_f<T>(y * to_f(lw[k]));
      }
  } else {
    for (int r = 0; r < rows; ++r)
      for (int k = threadIdx.x; k < K; k += kTmaWarps * 32) xs[(size_t)r * K + k] = x[(size_t)r * K + k];
  }
  consumer_sync();  // last CTA-wide barrier: the stage loop below has none

  for (int t = t_lo + warp; t < t_hi; t += kTmaWarps) {
    float acc[2][RMAX];
#pragma unroll
    for (int r = 0; r < RMAX; ++r) acc[0][r] = acc[1][r] = 0.f;
    bool ok = true;
    for (int p = 0; p < g.sp; ++p) {
      const int i = (t - t_lo) * g.sp + p;
      const int slot = i % g.slots;
      if (!seq_wait(&seq[slot], i) || !mbar_wait(&full[slot], (i / g.slots) & 1)) {
        if (err && lane == 0) atomicExch(err, 2);
        ok = false;
        break;
      }
      const int k0 = p * g.kp;
      const int nvec = min(g.kp, K - k0) / V;
      const T* st = reinterpret_cast<const T*>(ring + (size_t)slot * g.slot_bytes);
      // ILP: issue the shared-memory loads of UI vectors before using any of them.
      constexpr int UI = RMAX <= 2 ? 4 : (RMAX == 4 ? 2 : 1);
      for (int v0 = lane; v0 < nvec; v0 += 32 * UI) {
        int4 wv[UI][UPR], xv[UI][RMAX];
#pragma unroll
        for (int u = 0; u < UI; ++u) {
          const int v = v0 + 32 * u;
          if (v < nvec) {
#pragma unroll
            for (int q = 0; q < UPR; ++q)
              wv[u][q] = *reinterpret_cast<const int4*>(st + (size_t)q * g.kp + (size_t)v * V);
#pragma unroll
            for (int r = 0; r < RMAX; ++r)
              if (r < rows) xv[u][r] = *reinterpret_cast<const int4*>(xs + (size_t)r * K + k0 + (size_t)v * V);
          }
        }
#pragma unroll
        for (int u = 0; u < UI; ++u) {
          if (v0 + 32 * u < nvec) {
            float wf[UPR][V];
#pragma unroll
            for (int q = 0; q < UPR; ++q) unpack(wv[u][q], wf[q], T());
#pragma unroll
            for (int r = 0; r < RMAX; ++r) {
              if (r < rows) {
                float xf[V];
                unpack(xv[u][r], xf, T());
#pragma unroll
                for (int q = 0; q < UPR; ++q)
#pragma unroll
                  for (int e = 0; e < V; ++e) acc[q][r] = fmaf(wf[q][e], xf[e], acc[q][r]);
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);  // slot free for the producer
    }
    if (!ok) return;  // a wait expired: stop this warp (no CTA barrier follows)
#pragma unroll
    for (int r = 0; r < RMAX; ++r) {
      acc[0][r] = warp_sum(acc[0][r]);
      if (UPR == 2) acc[1][r] = warp_sum(acc[1][r]);
    }
#pragma unroll
    for (int r = 0; r < RMAX; ++r)
      if (lane == r && r < rows) row_epilogue<T, MODE>(a, t, r, acc[0][r], acc[1][r]);
  }
}

static int tma_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// Chooses the piece size and ring depth; false when the shape does not fit the kernel.
static bool tma_geometry(const FusedArgs& a, int mode, size_t es, TmaGeom* g) {
  const int upr = mode == MODE_PLAIN ? 1 : 2;
  const size_t row_bytes = (size_t)a.K * es;
  if (row_bytes % 16 || (uintptr_t)a.w % 16) return false;
  const int vec = (int)(16 / es);
  const size_t task_bytes = upr * row_bytes;
  int sp = (int)((task_bytes + kPieceBytes - 1) / kPieceBytes);
  int kp = (a.K + sp - 1) / sp;
  kp = (kp + vec - 1) / vec * vec;
  sp = (a.K + kp - 1) / kp;
  const size_t slot_bytes = (size_t)upr * kp * es;
  const size_t x_bytes = ((size_t)a.rows * row_bytes + 127) / 128 * 128;
  const size_t budget = 216 * 1024;
  if (x_bytes + 8 * (slot_bytes + 20) > budget) return false;
  int slots = (int)((budget - x_bytes) / (slot_bytes + 20));
  if (slots > 32) slots = 32;
  g->sp = sp;
  g->kp = kp;
  g->slots = slots;
  g->slot_bytes = (int)slot_bytes;
  g->x_bytes = (int)x_bytes;
  return true;
}

template <typename T, int MODE, int RMAX, bool NORM>
static cudaError_t launch_tma_t(const FusedArgs& a, const TmaGeom& g, cudaStream_t st) {
  auto kern = gemv_tma_kernel<T, MODE, RMAX, NORM>;
  const size_t smem = (size_t)g.x_bytes + (size_t)g.slots * g.slot_bytes + 2 * g.slots * sizeof(uint64_t) +
                      g.slots * sizeof(int);
  // The opt-in limit counts static shared memory too, so the attribute is raised to
  // exactly the dynamic size a launch needs (cached per device, grown when needed).
  static size_t attr_bytes[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return cudaErrorInvalidDevice;
  if (attr_bytes[dev] < smem) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr_bytes[dev] = smem;
  }
  const int ntasks = projection_tasks(a, MODE);
  int grid = tma_sms();
  if (grid > ntasks) grid = ntasks;
  return launch_pdl(kern, dim3(grid), dim3(kTmaThreads), smem, st, a, g);
}

template <typename T, int MODE, bool NORM>
static cudaError_t launch_tma_rows(const FusedArgs& a, const TmaGeom& g, cudaStream_t st) {
  if (a.rows <= 1) return launch_tma_t<T, MODE, 1, NORM>(a, g, st);
  if (a.rows <= 2) return launch_tma_t<T, MODE, 2, NORM>(a, g, st);
  if (a.rows <= 4) return launch_tma_t<T, MODE, 4, NORM>(a, g, st);
  return launch_tma_t<T, MODE, 8, NORM>(a, g, st);
}

// Streams a decode projection when the shape allows it; *handled is
// false otherwise (the caller then uses the register kernel).
cudaError_t fused_projection_tma(const FusedArgs& a, int dtype, int mode, bool norm, cudaStream_t st,
                                 bool* handled) {
  *handled = false;
  if (a.rows > kGemvMaxRows) return cudaSuccess;
  TmaGeom g;
  if (!tma_geometry(a, mode, dtype == BF16 ? 2 : 4, &g)) return cudaSuccess;
  *handled = true;
#define PIM_TMA(T)                                                                                        \
  if (mode == MODE_PLAIN)                                                                                 \
    return norm ? launch_tma_rows<T, MODE_PLAIN, true>(a, g, st) : launch_tma_rows<T, MODE_PLAIN, false>(a, g, st); \
  if (mode == MODE_ROPE)                                                                                  \
    return norm ? launch_tma_rows<T, MODE_ROPE, true>(a, g, st) : launch_tma_rows<T, MODE_ROPE, false>(a, g, st);   \
  return norm ? launch_tma_rows<T, MODE_SILU, true>(a, g, st) : launch_tma_rows<T, MODE_SILU, false>(a, g, st);
  if (dtype == BF16) {
    PIM_TMA(__nv_bfloat16)
  }
  PIM_TMA(float)
#undef PIM_TMA
}

}  // namespace pim
