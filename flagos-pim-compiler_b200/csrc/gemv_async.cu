// Decode projections with per-lane asynchronous staging (cp.async) and exact work
// balance.
//
// A task is one weight row for PLAIN and the row pair (2t, 2t + 1) of the
// pair-interleaved layout for ROPE and SILU.  The weight stream is cut into stages: one
// stage is the same 32 * U consecutive 16-byte chunks of each of the task's rows (the
// two rows of a pair share the activation chunk they multiply).  A CTA owns a
// contiguous, balanced range of tasks; the CTA's stages are split into 8 contiguous
// ranges of equal length (+-1 stage), one per warp, so every warp streams the same
// number of bytes.
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

#include "gemv_allreduce.cuh"
#include "gemv_attention.cuh"
#include "gemv_epilogue.cuh"
#include "pim_common.cuh"
#include "pim_kernels.h"

namespace pim {

constexpr int kAsyncWarps = 8;
constexpr int kAsyncThreads = kAsyncWarps * kWarp;
constexpr int kAsyncU = 2;                          // 16-byte chunks per lane, stage and weight row
constexpr int kAsyncStageChunks = kWarp * kAsyncU;  // chunks of each weight row per stage

// Ring depth S (S - 1 stages in flight per lane): 64 KB of ring per CTA for single rows,
// 80 KB for row pairs (two CTAs per SM).
template <int NW>
constexpr int async_slots() {
  return NW == 1 ? 8 : 5;
}
constexpr int kXc = 4;  // activation chunks per thread and row loaded together (norm weight in registers)
// Dynamic shared memory a CTA may use so that 1, 2 or 3 CTAs fit on an SM (228 KB,
// 1 KB reserved per CTA, a few hundred bytes of static shared memory).
constexpr size_t kAsyncSmemPerCta[3] = {220 * 1024, 112 * 1024, 74 * 1024};

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

template <typename T, int MODE, int RMAX, bool NORM, bool AR, bool ATTN = false>
__global__ void __launch_bounds__(kAsyncThreads, 3) gemv_async_kernel(FusedArgs a, AsyncGeom g) {
  constexpr int NW = (MODE == MODE_PLAIN) ? 1 : 2;  // weight rows per task
  constexpr int U = kAsyncU;
  constexpr int S = async_slots<NW>();
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

  // Copies this lane's chunks of stage (task tl, piece sub) into ring slot `slot`.
  auto issue = [&](int tl, int sub, int slot) {
    const int c0 = sub * kAsyncStageChunks + lane;
    const T* src = w + (size_t)(t_lo + tl) * NW * K;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + u * kWarp;
      if (c < nch) {
#pragma unroll
        for (int q = 0; q < NW; ++q)
          cp_async16(my + ((slot * U + u) * NW + q) * kWarp, src + (size_t)q * K + (size_t)c * V);
      }
    }
  };

  // Stages are walked as (task, piece) counters: one division at the start only.
  const int tl0 = s_lo / ms, sub0 = s_lo - tl0 * ms;
  int itl = tl0, isub = sub0, islot = 0, left = s_hi - s_lo;  // next stage to issue
  auto issue_next = [&]() {
    if (left > 0) {
      issue(itl, isub, islot);
      if (++isub == ms) {
        isub = 0;
        ++itl;
      }
      --left;
    }
    if (++islot == S) islot = 0;
    cp_async_commit();
  };

  // The norm weight is a weight (independent of the predecessor): this thread's first
  // kXc chunks of it are loaded before the wait, with the weight prologue.
  const int4* lw4 = static_cast<const int4*>(a.ln_w);
  int4 lwr[kXc];
  if (NORM) {
#pragma unroll
    for (int i = 0; i < kXc; ++i) {
      const int c = threadIdx.x + i * kAsyncThreads;
      if (c < nch) lwr[i] = ld_stream(lw4 + c);
    }
  }

  if constexpr (!AR) pdl_trigger();  // the fused all-reduce lets dependents start only at its end
#pragma unroll
  for (int j = 0; j < S - 1; ++j) issue_next();
  pdl_wait();

  // ---- stage the (normalised) activation rows; clear the partials -----------------
  // One pass of 16-byte loads through L2 (x was written by the predecessor grid, which
  // may have run on this SM while this grid started): raw rows to shared memory and
  // the sums of squares; then, for rmsnorm, the rows are normalised in place.
  const int4* x4 = static_cast<const int4*>(a.x);
  int4* xs4 = reinterpret_cast<int4*>(xs);
#pragma unroll
  for (int r = 0; r < RMAX; ++r) {
    float ss = 0.f;
    if (r < rows)
      for (int c0 = threadIdx.x; c0 < nch; c0 += kXc * kAsyncThreads) {
        int4 v[kXc];
#pragma unroll
        for (int i = 0; i < kXc; ++i)
          if (c0 + i * kAsyncThreads < nch) v[i] = ld_l2(x4 + (size_t)r * nch + c0 + i * kAsyncThreads);
#pragma unroll
        for (int i = 0; i < kXc; ++i) {
          const int c = c0 + i * kAsyncThreads;
          if (c < nch) {
            xs4[(size_t)r * nch + c] = v[i];
            if (NORM) {
              float f[V];
              unpack(v[i], f, T());
#pragma unroll
              for (int e = 0; e < V; ++e) ss = fmaf(f[e], f[e], ss);
            }
          }
        }
      }
    if (NORM) {
      ss = warp_sum(ss);
      if (lane == 0) red[warp][r] = ss;
    }
  }
  if (NORM) {
    __syncthreads();
    if (threadIdx.x < RMAX) {
      float s = 0.f;
      for (int i = 0; i < kAsyncWarps; ++i) s += red[i][threadIdx.x];
      rinv[threadIdx.x] = rsqrtf(s / (float)K + a.eps);
    }
    __syncthreads();
    for (int r = 0; r < rows; ++r)
      for (int c0 = threadIdx.x; c0 < nch; c0 += kXc * kAsyncThreads) {
#pragma unroll
        for (int i = 0; i < kXc; ++i) {
          const int c = c0 + i * kAsyncThreads;
          if (c < nch) {
            const int4 lv = c0 == (int)threadIdx.x ? lwr[i] : ld_stream(lw4 + c);
            float f[V], lf[V];
            unpack(xs4[(size_t)r * nch + c], f, T());
            unpack(lv, lf, T());
#pragma unroll
            for (int e = 0; e < V; ++e) f[e] = rnd<T>(rnd<T>(f[e] * rinv[r]) * lf[e]);
            xs4[(size_t)r * nch + c] = pack(f, T());
          }
        }
      }
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

  int cur = tl0, sub = sub0, slot = 0;
  for (int j = s_hi - s_lo; j > 0; --j) {
    issue_next();            // into the slot read one step earlier
    cp_async_wait<S - 1>();  // this lane's copies of the current stage have landed
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = sub * kAsyncStageChunks + u * kWarp + lane;
      if (c < nch) {
        int4 wv[NW];
#pragma unroll
        for (int q = 0; q < NW; ++q) wv[q] = my[((slot * U + u) * NW + q) * kWarp];
#pragma unroll
        for (int r = 0; r < RMAX; ++r) {
          if (r < rows) {
            const int4 xv = xs4[(size_t)r * nch + c];
            if constexpr (kIsBf16<T>) {  // bf16 products straight from the packed words
#pragma unroll
              for (int q = 0; q < NW; ++q) acc[q][r] = fma8_bf16(wv[q], xv, acc[q][r]);
            } else {
              float xf[V];
              unpack(xv, xf, T());
#pragma unroll
              for (int q = 0; q < NW; ++q) {
                float wf[V];
                unpack(wv[q], wf, T());
#pragma unroll
                for (int e = 0; e < V; ++e) acc[q][r] = fmaf(wf[e], xf[e], acc[q][r]);
              }
            }
          }
        }
      }
    }
    if (++slot == S) slot = 0;
    if (++sub == ms && j > 1) {  // warp-uniform: the range moves to the next task
      flush(cur);
      sub = 0;
      ++cur;
    }
  }
  if (s_lo < s_hi) flush(cur);
  cp_async_wait<0>();
  __syncthreads();

  // ---- epilogue: one thread per (task, activation row) ------------------------------
  const P2PDev* pd = static_cast<const P2PDev*>(a.p2p);
  int epoch = 0;
  if constexpr (AR) epoch = *reinterpret_cast<volatile const int*>(pd->counter) + 1;
  for (int i = threadIdx.x; i < nt * rows; i += kAsyncThreads) {
    const int tl = i / rows, r = i % rows;
    float v[2] = {0.f, 0.f};
#pragma unroll
    for (int q = 0; q < NW; ++q)
      for (int wp = 0; wp < kAsyncWarps; ++wp) v[q] += part[((tl * kAsyncWarps + wp) * NW + q) * RMAX + r];
    if constexpr (AR)
      ar_push<T>(pd, epoch & 1, (size_t)r * a.ncols + t_lo + tl, v[0]);
    else
      row_epilogue<T, MODE>(a, t_lo + tl, r, v[0], v[1]);
  }
  if constexpr (AR) {
    ar_reduce<T>(a, pd, t_lo, nt, epoch, epoch & 1);
    pdl_trigger();
  }
  // the weight ring is idle now: it holds the attention's merge buffers
  if constexpr (ATTN) fa_tail<T>(a, t_lo, t_hi, reinterpret_cast<float*>(ring));
}

// Most CTAs of the staged kernel per SM (3 by default; PIM_GEMV_MAX_CTAS=1 or 2 leaves
// room on every SM for the next kernel's CTAs to start their weight prologue early).
static int async_max_ctas() {
  static int n = 0;
  if (n == 0) {
    const char* e = getenv("PIM_GEMV_MAX_CTAS");
    n = (e && e[0] >= '1' && e[0] <= '3' && e[1] == 0) ? e[0] - '0' : 3;
  }
  return n;
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

template <typename T, int MODE, int RMAX, bool NORM, bool AR = false, bool ATTN = false>
static cudaError_t launch_async_t(const FusedArgs& a, cudaStream_t st, bool* handled) {
  constexpr int NW = (MODE == MODE_PLAIN) ? 1 : 2;
  const int ntasks = projection_tasks(a, MODE);
  const int nch = a.K / VecW<T>::n;
  AsyncGeom g;
  g.ms = (nch + kAsyncStageChunks - 1) / kAsyncStageChunks;
  g.x_bytes = (int)(((size_t)a.rows * a.K * sizeof(T) + 15) / 16 * 16);
  const size_t ring = (size_t)kAsyncWarps * async_slots<NW>() * kAsyncU * NW * kWarp * 16;
  // As many CTAs per SM (3, 2 or 1) as the shared memory allows -- and as the SM really
  // holds at once (occupancy API): the fused all-reduce variant's grid-wide wait needs
  // every CTA of the grid resident together, and a grid larger than one wave would give
  // any variant a second-wave tail.
  auto kern = gemv_async_kernel<T, MODE, RMAX, NORM, AR, ATTN>;
  static ResidentCache cache;
  int grid = 0;
  size_t smem = 0;
  for (int occ = async_max_ctas(); occ >= 1 && grid == 0; --occ) {
    const int gr = ntasks < async_sms() * occ ? ntasks : async_sms() * occ;
    const size_t tmax = ((size_t)ntasks + gr - 1) / gr;
    const size_t need = g.x_bytes + ring + tmax * kAsyncWarps * NW * RMAX * sizeof(float);
    if (need > kAsyncSmemPerCta[occ - 1]) continue;
    cudaError_t e;
    const int fits = resident_ctas(kern, kAsyncThreads, need, cache, &e);
    if (fits < 0) return e;
    if (fits < occ) continue;  // an SM holds fewer of these CTAs than planned
    grid = gr;
    smem = need;
  }
  if (grid == 0) return cudaSuccess;  // not handled: the caller takes the register kernel
  *handled = true;
  // The all-reduce variant's CTAs wait for one another (and for the peers): cooperative.
  if (AR) return launch_coop(kern, dim3(grid), dim3(kAsyncThreads), smem, st, a, g);
  return launch_pdl(kern, dim3(grid), dim3(kAsyncThreads), smem, st, a, g);
}

template <typename T, int MODE, bool NORM>
static cudaError_t launch_async_rows(const FusedArgs& a, cudaStream_t st, bool* handled) {
  if (a.rows <= 1) return launch_async_t<T, MODE, 1, NORM>(a, st, handled);
  if (a.rows <= 2) return launch_async_t<T, MODE, 2, NORM>(a, st, handled);
  if (a.rows <= 4) return launch_async_t<T, MODE, 4, NORM>(a, st, handled);
  return launch_async_t<T, MODE, 8, NORM>(a, st, handled);
}

template <typename T>
static cudaError_t launch_async_ar(const FusedArgs& a, cudaStream_t st, bool* handled) {
  if (a.rows <= 1) return launch_async_t<T, MODE_PLAIN, 1, false, true>(a, st, handled);
  if (a.rows <= 2) return launch_async_t<T, MODE_PLAIN, 2, false, true>(a, st, handled);
  if (a.rows <= 4) return launch_async_t<T, MODE_PLAIN, 4, false, true>(a, st, handled);
  return launch_async_t<T, MODE_PLAIN, 8, false, true>(a, st, handled);
}

// Row-parallel projection + all-reduce + residual add in one kernel (a.p2p set; PLAIN,
// no rmsnorm, rows <= kGemvMaxRows).  Shapes the staged kernel cannot take are an error:
// no other kernel implements the fused all-reduce.
cudaError_t fused_projection_allreduce(const FusedArgs& a, int dtype, cudaStream_t st) {
  const size_t es = dtype == BF16 ? 2 : 4;
  if (a.rows < 1 || a.rows > kGemvMaxRows || ((size_t)a.K * es) % 16 || (uintptr_t)a.w % 16 || a.ln_w)
    return cudaErrorNotSupported;
  bool handled = false;
  const cudaError_t e =
      dtype == BF16 ? launch_async_ar<__nv_bfloat16>(a, st, &handled) : launch_async_ar<float>(a, st, &handled);
  return handled ? e : cudaErrorNotSupported;
}

template <typename T, bool NORM>
static cudaError_t launch_async_attn(const FusedArgs& a, cudaStream_t st, bool* handled) {
  if (a.rows <= 1) return launch_async_t<T, MODE_ROPE, 1, NORM, false, true>(a, st, handled);
  if (a.rows <= 2) return launch_async_t<T, MODE_ROPE, 2, NORM, false, true>(a, st, handled);
  if (a.rows <= 4) return launch_async_t<T, MODE_ROPE, 4, NORM, false, true>(a, st, handled);
  return launch_async_t<T, MODE_ROPE, 8, NORM, false, true>(a, st, handled);
}

// q/k/v projection + RoPE + KV append with the layer's decode attention at the end of
// the same launch (a.attn_out set; staged kernel only).  Shapes it cannot take are an
// error: the caller asked for the attention and no other kernel computes it here.
cudaError_t fused_projection_attention(const FusedArgs& a, int dtype, bool norm, cudaStream_t st) {
  const size_t es = dtype == BF16 ? 2 : 4;
  if (!a.attn_out || !a.attn_cnt || a.rows < 1 || a.rows > kGemvMaxRows || ((size_t)a.K * es) % 16 ||
      (uintptr_t)a.w % 16 || (a.hd != 64 && a.hd != 128) || a.hq < 1 || a.hq > kFusedAttnMaxHeads ||
      a.hkv < 1 || a.hq % a.hkv)
    return cudaErrorNotSupported;
  bool handled = false;
  cudaError_t e;
  if (dtype == BF16)
    e = norm ? launch_async_attn<__nv_bfloat16, true>(a, st, &handled)
             : launch_async_attn<__nv_bfloat16, false>(a, st, &handled);
  else
    e = norm ? launch_async_attn<float, true>(a, st, &handled) : launch_async_attn<float, false>(a, st, &handled);
  return handled ? e : cudaErrorNotSupported;
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
