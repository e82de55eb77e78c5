// Decode projections (rows <= 8) with dynamic work assignment: the staged GEMV of
// gemv_async.cu, except that a CTA takes its work in units of a few tasks from a
// counter, so CTAs that stream faster take more units and the launch ends when the
// last unit does (per-CTA timing of the static kernel showed CTA end times spread over
// 24-40 us in a 40 us launch although every CTA streamed the same bytes).
//
// * Unit u = tasks [u*UT, min((u+1)*UT, ntasks)).  A CTA's first unit is blockIdx.x
//   (static: its weight prologue is issued before griddepcontrol.wait, as in the static
//   kernel); later units come from atomicAdd on ctr[0] (+ gridDim.x), which is only
//   touched after griddepcontrol.wait.  Unit ids are known one unit ahead (a 3-entry ring
//   in shared memory), so each warp's cp.async stream runs on from one unit into the next.
// * Within a unit, the unit's stages (task, 32*U-chunk piece) are split evenly over the 8
//   warps, partial sums per (task, warp) go to a per-unit buffer (two buffers, by unit
//   parity), and after a CTA barrier one thread per (task, row) adds the warps' partials
//   in warp order and runs the node's epilogue (gemv_epilogue.cuh).
// * cp.async groups are committed only for issued stages; before consuming a stage a
//   lane waits until at most the number of groups committed after that stage's group are
//   pending, which stays exact when a stage is issued late (its unit id not yet known).
//   A ring slot is reissued only after the stage that used it was consumed.
// * The last CTA to finish resets ctr[0] and ctr[1] to zero for the next launch.
//
// With AR the units' partials go to the exchange buffers and the grid ends with the
// fused all-reduce + residual add of gemv_allreduce.cuh (row-parallel projections at
// TP > 1), each CTA reducing a static range of columns.
//
// Selected by pim_set_projection_kernel(PIM_PROJ_KERNEL_DYNAMIC) when the call has the
// counter scratch (pim_projection_scratch_bytes asks for it while this kernel is
// selected); otherwise the static staged kernel runs.

#include <stdlib.h>

#include "gemv_allreduce.cuh"
#include "gemv_epilogue.cuh"
#include "pim_common.cuh"
#include "pim_kernels.h"

namespace pim {

constexpr int kDynWarps = 8;
constexpr int kDynThreads = kDynWarps * kWarp;
constexpr int kDynU = 2;                         // 16-byte chunks per lane, stage and weight row
constexpr int kDynStageChunks = kWarp * kDynU;   // chunks of each weight row per stage
constexpr int kDynXc = 4;                        // activation chunks per thread loaded together
constexpr size_t kDynSmemPerCta[3] = {220 * 1024, 112 * 1024, 74 * 1024};

template <int NW>
constexpr int dyn_slots() {
  return NW == 1 ? 8 : 5;
}

struct DynGeom {
  int ms;          // stages per task
  int unit_tasks;  // UT
  int n_units;
  int x_bytes;
};

__device__ __forceinline__ void dyn_cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void dyn_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

// Waits until at most n of this thread's cp.async groups are pending (n clamped to 7).
__device__ __forceinline__ void dyn_wait_pending(int n) {
  switch (n <= 0 ? 0 : (n >= 7 ? 7 : n)) {
    case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
    case 3: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
    case 4: asm volatile("cp.async.wait_group 4;" ::: "memory"); break;
    case 5: asm volatile("cp.async.wait_group 5;" ::: "memory"); break;
    case 6: asm volatile("cp.async.wait_group 6;" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 7;" ::: "memory"); break;
  }
}

// Stage range [lo, hi) of warp w in a unit of `n` stages.
__device__ __forceinline__ void dyn_share(int n, int w, int* lo, int* hi) {
  *lo = (int)(((long long)w * n) / kDynWarps);
  *hi = (int)(((long long)(w + 1) * n) / kDynWarps);
}

template <typename T, int MODE, int RMAX, bool NORM, bool AR>
__global__ void __launch_bounds__(kDynThreads, 3) gemv_dynamic_kernel(FusedArgs a, DynGeom g, int* ctr) {
  constexpr int NW = (MODE == MODE_PLAIN) ? 1 : 2;
  constexpr int U = kDynU;
  constexpr int S = dyn_slots<NW>();
  constexpr int V = VecW<T>::n;
  extern __shared__ __align__(16) unsigned char smem[];
  T* xs = reinterpret_cast<T*>(smem);
  int4* ring = reinterpret_cast<int4*>(smem + g.x_bytes);  // [warp][slot][u][q][lane]
  float* part = reinterpret_cast<float*>(ring + (size_t)kDynWarps * S * U * NW * kWarp);  // [2][UT][warp][q][r]
  __shared__ float red[kDynWarps][RMAX];
  __shared__ float rinv[RMAX];
  __shared__ int s_unit[3];

  const int K = a.K, rows = a.rows, nch = K / V, ms = g.ms, UT = g.unit_tasks;
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int ntasks = projection_tasks(a, MODE);
  const T* __restrict__ w = static_cast<const T*>(a.w);
  int4* my = ring + (size_t)warp * S * U * NW * kWarp + lane;
  const size_t part_unit = (size_t)UT * kDynWarps * NW * RMAX;

  auto unit_tasks = [&](int u) { return min(UT, ntasks - u * UT); };
  // Next unit id, or -1 when none is left (or the counter holds anything but a count
  // of this launch's fetches, so that no unit outside [gridDim.x, n_units) is read).
  auto fetch = [&]() -> int {
    const int v = atomicAdd(&ctr[0], 1);
    return v >= 0 && v < g.n_units - (int)gridDim.x ? v + (int)gridDim.x : -1;
  };

  // ---- issue side: (unit index ik, stage in this warp's share is / ihi) ----
  int ik = 0, iu = blockIdx.x, is = 0, ihi = 0, issued = 0;
  dyn_share(unit_tasks(iu) * ms, warp, &is, &ihi);
  auto issue_stage = [&](int u, int st, int slot) {
    const int tl = st / ms;
    const int c0 = (st - tl * ms) * kDynStageChunks + lane;
    const T* src = w + (size_t)(u * UT + tl) * NW * K;
#pragma unroll
    for (int uu = 0; uu < U; ++uu) {
      const int c = c0 + uu * kWarp;
      if (c < nch) {
#pragma unroll
        for (int q = 0; q < NW; ++q)
          dyn_cp16(my + ((slot * U + uu) * NW + q) * kWarp, src + (size_t)q * K + (size_t)c * V);
      }
    }
  };
  // Issues stages while fewer than S stages are issued and not consumed (the new stage
  // reuses the slot of a consumed one) and the next stage's unit is known (known_k:
  // highest unit index whose id is in s_unit).
  auto issue_more = [&](int consumed, int known_k) {
    while (issued - consumed < S && iu >= 0) {
      if (is == ihi) {  // this warp's share of unit ik is issued: move to the next unit
        if (ik + 1 > known_k) break;
        ++ik;
        iu = s_unit[ik % 3];
        if (iu < 0) break;
        dyn_share(unit_tasks(iu) * ms, warp, &is, &ihi);
        continue;
      }
      issue_stage(iu, is, issued % S);
      dyn_commit();
      ++is;
      ++issued;
    }
  };

  // Norm weight chunks before the wait (a weight), as in the static kernel.
  const int4* lw4 = static_cast<const int4*>(a.ln_w);
  int4 lwr[kDynXc];
  if (NORM) {
#pragma unroll
    for (int i = 0; i < kDynXc; ++i) {
      const int c = threadIdx.x + i * kDynThreads;
      if (c < nch) lwr[i] = ld_stream(lw4 + c);
    }
  }

  if constexpr (!AR) pdl_trigger();  // the fused all-reduce lets dependents start only at its end
  if (threadIdx.x == 0) s_unit[0] = blockIdx.x;
  issue_more(0, 0);  // the static first unit's stages (up to S) before the wait
  pdl_wait();
  const P2PDev* pd = static_cast<const P2PDev*>(a.p2p);
  int epoch = 0;
  if constexpr (AR) epoch = *reinterpret_cast<volatile const int*>(pd->counter) + 1;

  // ---- activation rows (one pass of 16-byte loads through L2) ----
  const int4* x4 = static_cast<const int4*>(a.x);
  int4* xs4 = reinterpret_cast<int4*>(xs);
#pragma unroll
  for (int r = 0; r < RMAX; ++r) {
    float ss = 0.f;
    if (r < rows)
      for (int c0 = threadIdx.x; c0 < nch; c0 += kDynXc * kDynThreads) {
        int4 v[kDynXc];
#pragma unroll
        for (int i = 0; i < kDynXc; ++i)
          if (c0 + i * kDynThreads < nch) v[i] = ld_l2(x4 + (size_t)r * nch + c0 + i * kDynThreads);
#pragma unroll
        for (int i = 0; i < kDynXc; ++i) {
          const int c = c0 + i * kDynThreads;
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
      for (int i = 0; i < kDynWarps; ++i) s += red[i][threadIdx.x];
      rinv[threadIdx.x] = rsqrtf(s / (float)K + a.eps);
    }
    __syncthreads();
    for (int r = 0; r < rows; ++r)
      for (int c0 = threadIdx.x; c0 < nch; c0 += kDynXc * kDynThreads) {
#pragma unroll
        for (int i = 0; i < kDynXc; ++i) {
          const int c = c0 + i * kDynThreads;
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
  for (int i = threadIdx.x; i < 2 * (int)part_unit; i += kDynThreads) part[i] = 0.f;
  if (threadIdx.x == 0) s_unit[1] = fetch();
  __syncthreads();

  // ---- units ----
  float acc[NW][RMAX];
#pragma unroll
  for (int q = 0; q < NW; ++q)
#pragma unroll
    for (int r = 0; r < RMAX; ++r) acc[q][r] = 0.f;
  int consumed = 0;
  for (int k = 0;; ++k) {
    const int u = s_unit[k % 3];
    if (u < 0) break;
    float* pu = part + (size_t)(k & 1) * part_unit;
    int lo, hi;
    dyn_share(unit_tasks(u) * ms, warp, &lo, &hi);
    if (ik < k) {  // this warp's issue pointer stopped in an earlier unit: all of it is consumed
      ik = k;
      iu = u;
      is = lo;
      ihi = hi;
    }
    int cur = lo < hi ? lo / ms : 0;
    auto flush = [&](int tl) {
#pragma unroll
      for (int q = 0; q < NW; ++q)
#pragma unroll
        for (int r = 0; r < RMAX; ++r) {
          const float v = warp_sum(acc[q][r]);
          if (lane == 0) pu[((tl * kDynWarps + warp) * NW + q) * RMAX + r] = v;
          acc[q][r] = 0.f;
        }
    };
    for (int st = lo; st < hi; ++st) {
      issue_more(consumed, k + 1);
      dyn_wait_pending(issued - 1 - consumed);  // groups committed after this stage's
      const int tl = st / ms;
      if (tl != cur) {  // warp-uniform: next task of the unit
        flush(cur);
        cur = tl;
      }
      const int slot = consumed % S;
      const int c0 = (st - tl * ms) * kDynStageChunks + lane;
#pragma unroll
      for (int uu = 0; uu < U; ++uu) {
        const int c = c0 + uu * kWarp;
        if (c < nch) {
          int4 wv[NW];
#pragma unroll
          for (int q = 0; q < NW; ++q) wv[q] = my[((slot * U + uu) * NW + q) * kWarp];
#pragma unroll
          for (int r = 0; r < RMAX; ++r) {
            if (r < rows) {
              const int4 xv = xs4[(size_t)r * nch + c];
              if constexpr (kIsBf16<T>) {
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
      ++consumed;
    }
    if (lo < hi) flush(cur);
    __syncthreads();  // every warp's partials of unit u are in pu; s_unit[(k + 2) % 3] is free
    if (threadIdx.x == 0) s_unit[(k + 2) % 3] = s_unit[(k + 1) % 3] < 0 ? -1 : fetch();
    const int nt = unit_tasks(u);
    for (int i = threadIdx.x; i < nt * rows; i += kDynThreads) {
      const int tl = i / rows, r = i % rows;
      float v[2] = {0.f, 0.f};
#pragma unroll
      for (int q = 0; q < NW; ++q)
        for (int wp = 0; wp < kDynWarps; ++wp) {
          float* slot = pu + ((tl * kDynWarps + wp) * NW + q) * RMAX + r;
          v[q] += *slot;
          *slot = 0.f;  // clear for unit k + 2, which reuses this buffer
        }
      if constexpr (AR)
        ar_push<T>(pd, epoch & 1, (size_t)r * a.ncols + u * UT + tl, v[0]);
      else
        row_epilogue<T, MODE>(a, u * UT + tl, r, v[0], v[1]);
    }
    __syncthreads();  // s_unit[(k + 2) % 3] visible; pu cleared before unit k + 2
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  if (threadIdx.x == 0) __threadfence();  // this CTA's fetches precede its arrival
  if (threadIdx.x == 0 && atomicAdd(&ctr[1], 1) == (int)gridDim.x - 1) {
    ctr[0] = 0;  // every CTA is past its last fetch: ready for the next launch
    ctr[1] = 0;
  }
  if constexpr (AR) {
    const int t_lo = (int)(((long long)blockIdx.x * ntasks) / gridDim.x);
    const int t_hi = (int)(((long long)(blockIdx.x + 1) * ntasks) / gridDim.x);
    ar_reduce<T>(a, pd, t_lo, t_hi - t_lo, epoch, epoch & 1);
    pdl_trigger();
  }
}

static int dyn_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <typename T, int MODE, int RMAX, bool NORM, bool AR = false>
static cudaError_t launch_dyn_t(const FusedArgs& a, int* ctr, cudaStream_t st, bool* handled) {
  constexpr int NW = (MODE == MODE_PLAIN) ? 1 : 2;
  const int ntasks = projection_tasks(a, MODE);
  const int nch = a.K / VecW<T>::n;
  DynGeom g;
  g.ms = (nch + kDynStageChunks - 1) / kDynStageChunks;
  g.x_bytes = (int)(((size_t)a.rows * a.K * sizeof(T) + 15) / 16 * 16);
  const size_t ring = (size_t)kDynWarps * dyn_slots<NW>() * kDynU * NW * kWarp * 16;
  auto kern = gemv_dynamic_kernel<T, MODE, RMAX, NORM, AR>;
  static ResidentCache cache;
  int grid = 0;
  size_t smem = 0;
  for (int occ = 3; occ >= 1 && grid == 0; --occ) {
    int gr = ntasks < dyn_sms() * occ ? ntasks : dyn_sms() * occ;
    // about four units per CTA, and at least one stage per warp in a full unit
    int ut = ntasks / (gr * 4);
    const int min_ut = (kDynWarps + g.ms - 1) / g.ms;
    if (ut < min_ut) ut = min_ut;
    const int n_units = (ntasks + ut - 1) / ut;
    if (gr > n_units) gr = n_units;
    const size_t need = g.x_bytes + ring + 2 * (size_t)ut * kDynWarps * NW * RMAX * sizeof(float);
    if (need > kDynSmemPerCta[occ - 1]) continue;
    cudaError_t e;
    const int fits = resident_ctas(kern, kDynThreads, need, cache, &e);
    if (fits < 0) return e;
    if (fits < occ) continue;  // an SM holds fewer of these CTAs than planned
    grid = gr;
    smem = need;
    g.unit_tasks = ut;
    g.n_units = n_units;
  }
  if (grid == 0) return cudaSuccess;  // not handled
  *handled = true;
  // The all-reduce variant's CTAs wait for one another (and for the peers): cooperative.
  if (AR) return launch_coop(kern, dim3(grid), dim3(kDynThreads), smem, st, a, g, ctr);
  return launch_pdl(kern, dim3(grid), dim3(kDynThreads), smem, st, a, g, ctr);
}

template <typename T, int MODE, bool NORM>
static cudaError_t launch_dyn_rows(const FusedArgs& a, int* ctr, cudaStream_t st, bool* handled) {
  if (a.rows <= 1) return launch_dyn_t<T, MODE, 1, NORM>(a, ctr, st, handled);
  if (a.rows <= 2) return launch_dyn_t<T, MODE, 2, NORM>(a, ctr, st, handled);
  if (a.rows <= 4) return launch_dyn_t<T, MODE, 4, NORM>(a, ctr, st, handled);
  return launch_dyn_t<T, MODE, 8, NORM>(a, ctr, st, handled);
}

template <typename T>
static cudaError_t launch_dyn_ar(const FusedArgs& a, int* ctr, cudaStream_t st, bool* handled) {
  if (a.rows <= 1) return launch_dyn_t<T, MODE_PLAIN, 1, false, true>(a, ctr, st, handled);
  if (a.rows <= 2) return launch_dyn_t<T, MODE_PLAIN, 2, false, true>(a, ctr, st, handled);
  if (a.rows <= 4) return launch_dyn_t<T, MODE_PLAIN, 4, false, true>(a, ctr, st, handled);
  return launch_dyn_t<T, MODE_PLAIN, 8, false, true>(a, ctr, st, handled);
}

// Row-parallel projection + all-reduce + residual add (a.p2p set; PLAIN, no rmsnorm)
// with dynamic work assignment; *handled is false when the shape does not suit it.
cudaError_t fused_projection_dynamic_allreduce(const FusedArgs& a, int dtype, int* ctr, cudaStream_t st,
                                               bool* handled) {
  *handled = false;
  const size_t es = dtype == BF16 ? 2 : 4;
  if (!ctr || !a.p2p || a.ln_w || a.rows < 1 || a.rows > kGemvMaxRows || ((size_t)a.K * es) % 16 ||
      (uintptr_t)a.w % 16)
    return cudaSuccess;
  return dtype == BF16 ? launch_dyn_ar<__nv_bfloat16>(a, ctr, st, handled) : launch_dyn_ar<float>(a, ctr, st, handled);
}

cudaError_t fused_projection_dynamic(const FusedArgs& a, int dtype, int mode, bool norm, int* ctr, cudaStream_t st,
                                     bool* handled) {
  *handled = false;
  const size_t es = dtype == BF16 ? 2 : 4;
  if (!ctr || a.rows < 1 || a.rows > kGemvMaxRows || ((size_t)a.K * es) % 16 || (uintptr_t)a.w % 16)
    return cudaSuccess;
#define PIM_DYN(T)                                                                                          \
  if (mode == MODE_PLAIN)                                                                                   \
    return norm ? launch_dyn_rows<T, MODE_PLAIN, true>(a, ctr, st, handled)                                 \
                : launch_dyn_rows<T, MODE_PLAIN, false>(a, ctr, st, handled);                               \
  if (mode == MODE_ROPE)                                                                                    \
    return norm ? launch_dyn_rows<T, MODE_ROPE, true>(a, ctr, st, handled)                                  \
                : launch_dyn_rows<T, MODE_ROPE, false>(a, ctr, st, handled);                                \
  return norm ? launch_dyn_rows<T, MODE_SILU, true>(a, ctr, st, handled)                                    \
              : launch_dyn_rows<T, MODE_SILU, false>(a, ctr, st, handled);
  if (dtype == BF16) {
    PIM_DYN(__nv_bfloat16)
  }
  PIM_DYN(float)
#undef PIM_DYN
}

}  // namespace pim
