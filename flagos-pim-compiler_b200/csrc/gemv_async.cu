// Decode projections with per-lane asynchronous staging (cp.async) and exact work
// balance.
//
// The weight stream is cut into stages: one stage is 32 * U consecutive 16-byte
// chunks of every weight row of one task (a task is one row for PLAIN, the row pair
// (2t, 2t + 1) of the pair-interleaved layout for ROPE and SILU).  A CTA owns a
// contiguous, balanced range of tasks; the CTA's stages are split into 8 contiguous
// ranges of equal length (+-1 stage), one per warp, so a task may be shared by two or
// more warps and every warp streams the same number of bytes.
//
// Each lane copies its own chunks with cp.async into a private ring of S slots in
// shared memory, keeping S - 1 stages in flight while it multiplies the oldest one.
// A lane only ever reads back what it copied itself, so the ring needs no barrier,
// no mbarrier and no wait other than cp.async.wait_group.  The first S - 1 stages are
// issued before griddepcontrol.wait: with programmatic dependent launch the weight
// stream overlaps the end of the previous kernel (weights never depend on it).
//
// When its range moves to the next task, a warp reduces its fp32 partial dot products
// with shuffles and stores them per (task, warp) in shared memory; after one CTA
// barrier, one thread per (task, activation row) adds the warps' partials in warp
// order (a fixed order: results do not depend on timing) and runs the epilogue of the
// register kernel (gemv_epilogue.cuh).

#include <stdlib.h>

#include "gemv_epilogue.cuh"
#include "pim_common.cuh"
#include "pim_kernels.h"

namespace pim {

constexpr int kAsyncWarps = 8;
constexpr int kAsyncThreads = kAsyncWarps * kWarp;
constexpr int kAsyncU = 2;                                 // chunks per lane, stage and weight row
constexpr int kAsyncStageChunks = kWarp * kAsyncU;         // chunks per weight row in one stage
constexpr size_t kAsyncSmemTwoCtas = 112 * 1024;           // per-CTA budget for 2 CTAs per SM
constexpr size_t kAsyncSmemOneCta = 220 * 1024;            // per-CTA budget for 1 CTA per SM

struct AsyncGeom {
  int ms;       // stages per task: ceil(chunks per row / kAsyncStageChunks)
  int x_bytes;  // shared-memory bytes of the staged activation rows (16-aligned)
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int MODE>
constexpr int async_ring_depth() {
  return MODE == MODE_PLAIN ? 8 : 5;
}

template <typename T, int MODE, int RMAX, bool NORM>
__global__ void __launch_bounds__(kAsyncThreads, 2) gemv_async_kernel(FusedArgs a, AsyncGeom g) {
  constexpr int NW = (MODE == MODE_PLAIN) ? 1 : 2;  // weight rows per task
  constexpr int U = kAsyncU;
  constexpr int S = async_ring_depth<MODE>();
  constexpr int V = VecW<T>::n;
  extern __shared__ __align__(16) unsigned char smem[];
  T* xs = reinterpret_cast<T*>(smem);
  int4* ring = reinterpret_cast<int4*>(smem + g.x_bytes);  // [warp][slot][u][q][lane]
  float* part = reinterpret_cast<float*>(ring + (size_t)kAsyncWarps * S * U * NW * kWarp);  // [task][warp][q][r]
  __shared__ float red[kAsyncWarps][RMAX];
  __shared__ float rinv[RMAX];

  const int K = a.K, rows = a.rows, nch = K / V, ms = g.ms;
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int ntasks = projection_tasks(a, MODE);
  const int t_lo = (int)(((long long)blockIdx.x * ntasks) / gridDim.x);
  const int t_hi = (int)(((long long)(blockIdx.x + 1) * ntasks) / gridDim.x);
  const int nt = t_hi - t_lo;
  const int nstages = nt * ms;
  const int s_lo = (int)(((long long)warp * nstages) / kAsyncWarps);
  const int s_hi = (int)(((long long)(warp + 1) * nstages) / kAsyncWarps);
  const T* __restrict__ w = static_cast<const T*>(a.w);
  int4* my = ring + (size_t)warp * S * U * NW * kWarp + lane;

  // Copies this lane's chunks of CTA-local stage s into ring slot `slot`.
  auto issue = [&](int s, int slot) {
    const int tl = s / ms;
    const int kc0 = (s - tl * ms) * kAsyncStageChunks + lane;
    const size_t row0 = (size_t)(t_lo + tl) * NW;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int kc = kc0 + u * kWarp;
      if (kc < nch) {
#pragma unroll
        for (int q = 0; q < NW; ++q)
          cp_async16(my + ((slot * U + u) * NW + q) * kWarp, w + (row0 + q) * K + (size_t)kc * V);
      }
    }
  };

  pdl_trigger();
#pragma unroll
  for (int j = 0; j < S - 1; ++j) {
    if (s_lo + j < s_hi) issue(s_lo + j, j);
    cp_async_commit();
  }
  pdl_wait();

  // ---- stage (normalised) activation rows; clear the partials --------------------
  const T* __restrict__ x = static_cast<const T*>(a.x);
  if (NORM) {
    const T* __restrict__ lw = static_cast<const T*>(a.ln_w);
#pragma unroll
    for (int r = 0; r < RMAX; ++r) {
      float ss = 0.f;
      if (r < rows)
        for (int k = threadIdx.x; k < K; k += kAsyncThreads) {
          const float xv = to_f(x[(size_t)r * K + k]);
          ss = fmaf(xv, xv, ss);
        }
      ss = warp_sum(ss);
      if (lane == 0) red[warp][r] = ss;
    }
    __syncthreads();
    if (threadIdx.x < RMAX) {
      float s = 0.f;
      for (int i = 0; i < kAsyncWarps; ++i) s += red[i][threadIdx.x];
      rinv[threadIdx.x] = rsqrtf(s / (float)K + a.eps);
    }
    __syncthreads();
    for (int r = 0; r < rows; ++r)
      for (int k = threadIdx.x; k < K; k += kAsyncThreads) {
        const float y = rnd<T>(to_f(x[(size_t)r * K + k]) * rinv[r]);
        xs[(size_t)r * K + k] = from_f<T>(y * to_f(lw[k]));
      }
  } else {
    for (int r = 0; r < rows; ++r)
      for (int k = threadIdx.x; k < K; k += kAsyncThreads) xs[(size_t)r * K + k] = x[(size_t)r * K + k];
  }
  for (int i = threadIdx.x; i < nt * kAsyncWarps * NW * RMAX; i += kAsyncThreads) part[i] = 0.f;
  __syncthreads();

  // ---- stream this warp's stages ----------------------------------------------------
  float acc[NW][RMAX];
#pragma unroll
  for (int q = 0; q < NW; ++q)
#pragma unroll
    for (int r = 0; r < RMAX; ++r) acc[q][r] = 0.f;

  auto flush = [&](int tl) {
#pragma unroll
    for (int q = 0; q < NW; ++q)
#pragma unroll
      for (int r = 0; r < RMAX; ++r) {
        const float v = warp_sum(acc[q][r]);
        if (lane == 0) part[((tl * kAsyncWarps + warp) * NW + q) * RMAX + r] = v;
        acc[q][r] = 0.f;
      }
  };

  int cur = s_lo / ms;
  for (int s = s_lo; s < s_hi; ++s) {
    const int j = s - s_lo;
    if (s + S - 1 < s_hi) issue(s + S - 1, (j + S - 1) % S);  // the slot read at step j - 1
    cp_async_commit();
    cp_async_wait<S - 1>();  // this lane's copies of stage s have landed
    const int tl = s / ms;
    if (tl != cur) {  // warp-uniform: the range moved to the next task
      flush(cur);
      cur = tl;
    }
    const int slot = j % S;
    const int kc0 = (s - tl * ms) * kAsyncStageChunks + lane;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int kc = kc0 + u * kWarp;
      if (kc < nch) {
        float wf[NW][V];
#pragma unroll
        for (int q = 0; q < NW; ++q) unpack(my[((slot * U + u) * NW + q) * kWarp], wf[q], T());
#pragma unroll
        for (int r = 0; r < RMAX; ++r) {
          if (r < rows) {
            float xf[V];
            unpack(*reinterpret_cast<const int4*>(xs + (size_t)r * K + (size_t)kc * V), xf, T());
#pragma unroll
            for (int q = 0; q < NW; ++q)
#pragma unroll
              for (int e = 0; e < V; ++e) acc[q][r] = fmaf(wf[q][e], xf[e], acc[q][r]);
          }
        }
      }
    }
  }
  if (s_lo < s_hi) flush(cur);
  cp_async_wait<0>();
  __syncthreads();

  // ---- epilogue: one thread per (task, activation row) ------------------------------
  for (int i = threadIdx.x; i < nt * rows; i += kAsyncThreads) {
    const int tl = i / rows, r = i % rows;
    float v[2] = {0.f, 0.f};
#pragma unroll
    for (int q = 0; q < NW; ++q)
      for (int wp = 0; wp < kAsyncWarps; ++wp) v[q] += part[((tl * kAsyncWarps + wp) * NW + q) * RMAX + r];
    row_epilogue<T, MODE>(a, t_lo + tl, r, v[0], v[1]);
  }
}

static int async_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <typename T, int MODE, int RMAX, bool NORM>
static cudaError_t launch_async_t(const FusedArgs& a, cudaStream_t st, bool* handled) {
  constexpr int NW = (MODE == MODE_PLAIN) ? 1 : 2;
  constexpr int S = async_ring_depth<MODE>();
  const int ntasks = projection_tasks(a, MODE);
  const int nch = a.K / VecW<T>::n;
  AsyncGeom g;
  g.ms = (nch + kAsyncStageChunks - 1) / kAsyncStageChunks;
  g.x_bytes = (int)(((size_t)a.rows * a.K * sizeof(T) + 15) / 16 * 16);
  const size_t ring = (size_t)kAsyncWarps * S * kAsyncU * NW * kWarp * 16;
  // Two CTAs per SM when the shared memory allows it, else one.
  int grid = 0;
  size_t smem = 0;
  for (int occ = 2; occ >= 1 && grid == 0; --occ) {
    const int gr = ntasks < async_sms() * occ ? ntasks : async_sms() * occ;
    const size_t tmax = ((size_t)ntasks + gr - 1) / gr;
    const size_t need = g.x_bytes + ring + tmax * kAsyncWarps * NW * RMAX * sizeof(float);
    if (need <= (occ == 2 ? kAsyncSmemTwoCtas : kAsyncSmemOneCta)) {
      grid = gr;
      smem = need;
    }
  }
  if (grid == 0) return cudaSuccess;  // not handled: the caller takes the register kernel
  *handled = true;
  auto kern = gemv_async_kernel<T, MODE, RMAX, NORM>;
  // The attribute is raised once per device to the largest size seen, so launches
  // inside a stream capture make no attribute calls after the first eager run.
  static size_t attr_bytes[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return cudaErrorInvalidDevice;
  if (attr_bytes[dev] < smem) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr_bytes[dev] = smem;
  }
  return launch_pdl(kern, dim3(grid), dim3(kAsyncThreads), smem, st, a, g);
}

template <typename T, int MODE, bool NORM>
static cudaError_t launch_async_rows(const FusedArgs& a, cudaStream_t st, bool* handled) {
  if (a.rows <= 1) return launch_async_t<T, MODE, 1, NORM>(a, st, handled);
  if (a.rows <= 2) return launch_async_t<T, MODE, 2, NORM>(a, st, handled);
  if (a.rows <= 4) return launch_async_t<T, MODE, 4, NORM>(a, st, handled);
  return launch_async_t<T, MODE, 8, NORM>(a, st, handled);
}

// Runs a decode projection (rows <= kGemvMaxRows) with the staged kernel; *handled is
// false when the shape does not suit it (unaligned rows, or shared memory too small),
// and the caller then uses the register kernel.
cudaError_t fused_projection_async(const FusedArgs& a, int dtype, int mode, bool norm, cudaStream_t st,
                                   bool* handled) {
  *handled = false;
  const size_t es = dtype == BF16 ? 2 : 4;
  if (a.rows < 1 || a.rows > kGemvMaxRows || ((size_t)a.K * es) % 16 || (uintptr_t)a.w % 16) return cudaSuccess;
#define PIM_ASYNC(T)                                                                                      \
  if (mode == MODE_PLAIN)                                                                                 \
    return norm ? launch_async_rows<T, MODE_PLAIN, true>(a, st, handled)                                  \
                : launch_async_rows<T, MODE_PLAIN, false>(a, st, handled);                                \
  if (mode == MODE_ROPE)                                                                                  \
    return norm ? launch_async_rows<T, MODE_ROPE, true>(a, st, handled)                                   \
                : launch_async_rows<T, MODE_ROPE, false>(a, st, handled);                                 \
  return norm ? launch_async_rows<T, MODE_SILU, true>(a, st, handled)                                     \
              : launch_async_rows<T, MODE_SILU, false>(a, st, handled);
  if (dtype == BF16) {
    PIM_ASYNC(__nv_bfloat16)
  }
  PIM_ASYNC(float)
#undef PIM_ASYNC
}

}  // namespace pim
