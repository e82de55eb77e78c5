// Decode projections streamed through shared memory with the bulk-copy (TMA) engine.
//
// One persistent CTA per SM owns a contiguous, balanced range of tasks (a task is
// one weight row for PLAIN and two adjacent rows -- the pair-interleaved layout --
// for ROPE and SILU), so the CTA's weights are one contiguous byte range.  A
// producer thread streams that range stage by stage with cp.async.bulk into a ring
// of shared-memory stages (mbarrier complete_tx), starting before
// griddepcontrol.wait: with programmatic dependent launch the weight stream of
// this kernel overlaps the end of the previous kernel.  Eight consumer warps stage
// the (normalised) activation rows once, then turn each stage into dot products:
// a stage holds UPS tasks; WPU = 8 / UPS warps split a task's K range when UPS < 8
// and combine their partial sums in shared memory; with UPS >= 8 each warp owns
// whole tasks.  The epilogues (plain / residual / RoPE + KV append / SiLU*up) are
// the ones of the register kernel in gemv.cu.
//
// Every mbarrier wait is bounded (2 s of %globaltimer): on expiry the kernel
// raises *a.err (when given) and stops instead of spinning forever.

#include <stdlib.h>

#include "pim_common.cuh"
#include "pim_kernels.h"

namespace pim {

constexpr int kTmaWarps = 8;                     // consumer warps
constexpr int kTmaThreads = (kTmaWarps + 1) * 32;  // + one producer warp
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

struct TmaGeom {
  int ups;          // tasks per stage
  int wpu;          // warps per task (ups < 8) or 1
  int stages;       // ring depth
  int stage_bytes;  // bytes of one stage
  int x_bytes;      // bytes reserved for the activation rows (128-aligned)
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long gtime_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity; false after kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = gtime_ns();
  while (!mbar_try_wait(bar, parity))
    if (gtime_ns() - t0 > kWaitLimitNs) return false;
  return true;
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kTmaWarps * 32) : "memory"); }

template <int MODE>
__device__ __forceinline__ int tma_ntasks(const FusedArgs& a) {
  if (MODE == MODE_PLAIN) return a.ncols;
  if (MODE == MODE_ROPE) return (a.hq + 2 * a.hkv) * (a.hd / 2);
  return a.inter;
}

// Epilogue of one task (same rounding as the register kernel); lane r finishes row r.
template <typename T, int MODE, int RMAX>
__device__ __forceinline__ void tma_epilogue(const FusedArgs& a, int t, int lane, const float (&acc)[2][RMAX]) {
  const int half = a.hd / 2;
#pragma unroll
  for (int r = 0; r < RMAX; ++r) {
    if (lane != r || r >= a.rows) continue;
    if (MODE == MODE_PLAIN) {
      float y = acc[0][r];
      if (a.residual) y = rnd<T>(y) + to_f(static_cast<const T*>(a.residual)[(size_t)r * a.ncols + t]);
      static_cast<T*>(a.y)[(size_t)r * a.ncols + t] = from_f<T>(y);
    } else if (MODE == MODE_SILU) {
      const float g = rnd<T>(acc[0][r]), u = rnd<T>(acc[1][r]);
      const float act = rnd<T>(g / (1.f + expf(-g)));
      static_cast<T*>(a.y)[(size_t)r * a.inter + t] = from_f<T>(act * u);
    } else {
      const int hidx = t / half, j = t % half;
      const int b = r / a.seq, s = r % a.seq;
      const int p = a.positions[b] + s;
      if (p < 0 || p >= a.max_seq) continue;  // positions are validated on the host
      const float v1 = rnd<T>(acc[0][r]), v2 = rnd<T>(acc[1][r]);
      float o1 = v1, o2 = v2;
      if (hidx < a.hq + a.hkv) {
        const float c = a.cos[(size_t)p * half + j], sn = a.sin[(size_t)p * half + j];
        o1 = rnd<T>(rnd<T>(v1 * c) + rnd<T>(-v2 * sn));
        o2 = rnd<T>(rnd<T>(v2 * c) + rnd<T>(v1 * sn));
      }
      T* dst;
      if (hidx < a.hq) {
        dst = static_cast<T*>(a.y) + (size_t)r * a.hq * a.hd + (size_t)hidx * a.hd;
      } else {
        const int kvh = hidx < a.hq + a.hkv ? hidx - a.hq : hidx - a.hq - a.hkv;
        const int which = hidx < a.hq + a.hkv ? 0 : 1;
        dst = static_cast<T*>(a.kv_base) + (2 * kvh + which) * a.block_stride + b * a.seq_stride + (size_t)p * a.hd;
      }
      dst[j] = from_f<T>(o1);
      dst[j + half] = from_f<T>(o2);
    }
  }
}

template <typename T, int MODE, int RMAX, bool NORM>
__global__ void __launch_bounds__(kTmaThreads, 1) gemv_tma_kernel(FusedArgs a, TmaGeom g) {
  int* err = a.err;
  constexpr int UPR = (MODE == MODE_PLAIN) ? 1 : 2;  // weight rows per task
  constexpr int V = VecW<T>::n;
  extern __shared__ __align__(128) unsigned char smem[];
  T* xs = reinterpret_cast<T*>(smem);
  unsigned char* ring = smem + g.x_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + (size_t)g.stages * g.stage_bytes);
  uint64_t* empty = full + g.stages;
  float* red = reinterpret_cast<float*>(empty + g.stages);  // [2][kTmaWarps][2][RMAX]
  __shared__ float rinv[RMAX];
  __shared__ float nred[kTmaWarps][RMAX];

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int K = a.K;
  const size_t task_bytes = (size_t)UPR * K * sizeof(T);
  const int ntasks = tma_ntasks<MODE>(a);
  const int t_lo = (int)(((long long)blockIdx.x * ntasks) / gridDim.x);
  const int t_hi = (int)(((long long)(blockIdx.x + 1) * ntasks) / gridDim.x);
  const int nst = (t_hi - t_lo + g.ups - 1) / g.ups;

  if (threadIdx.x == 0) {
    for (int s = 0; s < g.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kTmaWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_trigger();

  if (warp == kTmaWarps) {
    // ---- producer: stream this CTA's weight bytes (independent of the predecessor)
    if (lane == 0) {
      const char* wbase = static_cast<const char*>(a.w) + (size_t)t_lo * task_bytes;
      for (int i = 0; i < nst; ++i) {
        const int slot = i % g.stages;
        if (i >= g.stages && !mbar_wait(&empty[slot], ((i / g.stages) - 1) & 1)) {
          if (err) atomicExch(err, 1);
          break;
        }
        const int nt = min(g.ups, t_hi - (t_lo + i * g.ups));
        const uint32_t bytes = (uint32_t)(nt * task_bytes);
        mbar_expect_tx(&full[slot], bytes);
        bulk_g2s(ring + (size_t)slot * g.stage_bytes, wbase + (size_t)i * g.ups * task_bytes, bytes, &full[slot]);
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
  consumer_sync();

  const int kw = K / g.wpu;      // K range of one warp when tasks are split
  const int nvec = kw / V;
  // A warp whose wait expires raises *err and stops computing, but keeps taking
  // part in the consumer barriers so that no other warp blocks on it.
  bool dead = false;
  for (int i = 0; i < nst; ++i) {
    const int slot = i % g.stages;
    if (!dead && !mbar_wait(&full[slot], (i / g.stages) & 1)) {
      if (err && lane == 0) atomicExch(err, 2);
      dead = true;
    }
    const T* st = reinterpret_cast<const T*>(ring + (size_t)slot * g.stage_bytes);
    const int t0 = t_lo + i * g.ups;
    const int nt = min(g.ups, t_hi - t0);
    float* rb = red + (size_t)(i & 1) * kTmaWarps * 2 * RMAX;
    const int step = kTmaWarps / g.wpu;  // tasks processed concurrently
    for (int u = dead ? nt : warp / g.wpu; u < nt; u += step) {
      const int slice = warp % g.wpu;
      float acc[2][RMAX];
#pragma unroll
      for (int r = 0; r < RMAX; ++r) acc[0][r] = acc[1][r] = 0.f;
      const T* w0 = st + (size_t)u * UPR * K + (size_t)slice * kw;
      for (int v = lane; v < nvec; v += 32) {
        float wf[UPR][V];
#pragma unroll
        for (int q = 0; q < UPR; ++q)
          unpack(*reinterpret_cast<const int4*>(w0 + (size_t)q * K + (size_t)v * V), wf[q], T());
#pragma unroll
        for (int r = 0; r < RMAX; ++r) {
          if (r < rows) {
            float xf[V];
            unpack(*reinterpret_cast<const int4*>(xs + (size_t)r * K + (size_t)slice * kw + (size_t)v * V), xf, T());
#pragma unroll
            for (int q = 0; q < UPR; ++q)
#pragma unroll
              for (int e = 0; e < V; ++e) acc[q][r] = fmaf(wf[q][e], xf[e], acc[q][r]);
          }
        }
      }
#pragma unroll
      for (int r = 0; r < RMAX; ++r) {
        acc[0][r] = warp_sum(acc[0][r]);
        if (UPR == 2) acc[1][r] = warp_sum(acc[1][r]);
      }
      if (g.wpu == 1) {
        tma_epilogue<T, MODE, RMAX>(a, t0 + u, lane, acc);
      } else if (lane == 0) {
#pragma unroll
        for (int r = 0; r < RMAX; ++r) {
          rb[(warp * 2 + 0) * RMAX + r] = acc[0][r];
          rb[(warp * 2 + 1) * RMAX + r] = acc[1][r];
        }
      }
    }
    __syncwarp();
    if (lane == 0 && !dead) mbar_arrive(&empty[slot]);  // this warp is done reading the stage
    if (g.wpu > 1) {
      consumer_sync();
      if (warp < nt && !dead) {
        float acc[2][RMAX];
#pragma unroll
        for (int r = 0; r < RMAX; ++r) {
          acc[0][r] = acc[1][r] = 0.f;
          for (int s = 0; s < g.wpu; ++s) {
            acc[0][r] += rb[((warp * g.wpu + s) * 2 + 0) * RMAX + r];
            acc[1][r] += rb[((warp * g.wpu + s) * 2 + 1) * RMAX + r];
          }
        }
        tma_epilogue<T, MODE, RMAX>(a, t0 + warp, lane, acc);
      }
    }
  }
}

static bool tma_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("PIM_GEMV");
    on = (e && e[0] == 'r') ? 0 : 1;  // PIM_GEMV=reg selects the register-streaming kernel
  }
  return on == 1;
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

// Chooses the stage geometry; false when the shape does not fit the streamed kernel.
static bool tma_geometry(const FusedArgs& a, int mode, size_t es, TmaGeom* g) {
  const int upr = mode == MODE_PLAIN ? 1 : 2;
  const size_t row_bytes = (size_t)a.K * es;
  const size_t task_bytes = upr * row_bytes;
  if (row_bytes % 16 || (uintptr_t)a.w % 16) return false;
  const int vec = (int)(16 / es);
  long tasks_target = (long)(32768 / task_bytes);
  if (tasks_target < 1) tasks_target = 1;
  int ups;
  if (tasks_target >= 8) {
    ups = (int)(tasks_target / 8 * 8);
  } else {
    ups = 1;
    while (ups * 2 <= tasks_target) ups *= 2;
  }
  const int wpu = ups >= kTmaWarps ? 1 : kTmaWarps / ups;
  if (a.K % (wpu * vec)) return false;
  const size_t x_bytes = ((size_t)a.rows * row_bytes + 127) / 128 * 128;
  const size_t stage_bytes = (size_t)ups * task_bytes;
  const size_t budget = 220 * 1024;
  const size_t extras = 2 * 8 * 16 + 2 * kTmaWarps * 2 * 8 * sizeof(float);
  if (x_bytes + extras + 2 * stage_bytes > budget) return false;
  int stages = (int)((budget - x_bytes - extras) / stage_bytes);
  if (stages > 8) stages = 8;
  g->ups = ups;
  g->wpu = wpu;
  g->stages = stages;
  g->stage_bytes = (int)stage_bytes;
  g->x_bytes = (int)x_bytes;
  return true;
}

template <typename T, int MODE, int RMAX, bool NORM>
static cudaError_t launch_tma_t(const FusedArgs& a, const TmaGeom& g, cudaStream_t st) {
  auto kern = gemv_tma_kernel<T, MODE, RMAX, NORM>;
  const size_t smem = (size_t)g.x_bytes + (size_t)g.stages * g.stage_bytes + 2 * g.stages * sizeof(uint64_t) +
                      2 * kTmaWarps * 2 * RMAX * sizeof(float);
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
  const int ntasks = MODE == MODE_PLAIN ? a.ncols : (MODE == MODE_ROPE ? (a.hq + 2 * a.hkv) * (a.hd / 2) : a.inter);
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

// Streams a decode projection when the shape allows it; *handled is false otherwise
// (the caller then uses the register kernel).
cudaError_t fused_projection_tma(const FusedArgs& a, int dtype, int mode, bool norm, cudaStream_t st,
                                 bool* handled) {
  *handled = false;
  if (!tma_enabled() || a.rows > kGemvMaxRows) return cudaSuccess;
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
