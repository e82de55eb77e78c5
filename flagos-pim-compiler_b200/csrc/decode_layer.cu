// One decoder layer of a batch-1 decode step in one launch (opt-in): attn_in with the
// decode attention, o_proj + residual, mlp_in, down + residual -- the five kernels of a
// layer as four phases of one grid, separated by grid-wide barriers.
//
// Each phase is the staged GEMV of gemv_async.cu (per-lane cp.async rings, exact
// per-warp stage balance, partial dot products summed per (task, warp) in warp order, the
// same epilogues) over a static partition of its tasks, restated here for one activation
// row as a prologue / body pair (DlPhase) rather than shared with gemv_async.cu, whose
// kernel stays as measured.  What the single launch adds:
//   * the next phase's first S - 1 weight stages are issued before the grid barrier that
//     separates the phases (weights never depend on the previous phase), so the weight
//     stream does not stop at phase boundaries and no CTA drains or refills between them;
//   * the attention is the tail of the first phase (gemv_attention.cuh: the CTA that
//     writes a head's last q / k / v value computes the head), finished before barrier 1.
// The grid is at most the CTAs an SM holds at once (occupancy API) times the SMs, so every
// CTA is resident when the barriers are waited on.  The kernel is launched with
// programmatic dependent launch: the next layer's CTAs start their weight prologue as this
// grid's CTAs leave, and wait for it to complete before reading its output.
//
// Barrier: arrival count and generation in global memory (zero before the first call, the
// count back at zero after every barrier).  Each CTA fences, reads the generation, arrives;
// the last arrival resets the count and advances the generation; the others wait for the
// new generation, at most kDlWaitNs, after which they raise *err and go on (the layer's
// output is then wrong, and the error word says so).
//
// At TP > 1 (one process per GPU, AR form): o_proj and down are row-parallel, and each
// ends in the fused all-reduce of gemv_allreduce.cuh -- every CTA pushes its rounded
// partials into every rank's exchange buffer, the rank's last CTA raises its flags, every
// CTA waits for all ranks and writes residual + the rank-order sum of its own columns.
// One launch makes two consecutive all-reduce calls (epochs counter + 1 and counter + 2,
// read once after griddepcontrol.wait); the grid barrier after the first one separates
// its ticket reset from the second one's tickets.  The mlp weights' first stages are
// issued before the first peer wait.  As in the fused projection kernel, the AR form lets
// its dependents start only at its end.

#include <stdlib.h>

#include <vector>

#include "gemv_allreduce.cuh"
#include "gemv_attention.cuh"
#include "gemv_epilogue.cuh"
#include "pim_common.cuh"
#include "pim_kernels.h"

namespace pim {

constexpr int kDlWarps = 8;
constexpr int kDlThreads = kDlWarps * kWarp;
constexpr int kDlU = 2;                          // 16-byte chunks per lane, stage and weight row
constexpr int kDlStageChunks = kWarp * kDlU;
constexpr unsigned long long kDlWaitNs = 1000000000ull;
constexpr size_t kDlRingBytes = (size_t)kDlWarps * 5 * kDlU * 2 * kWarp * 16;  // 80 KB: the largest ring (row pairs)

template <int NW>
constexpr int dl_slots() {
  return NW == 1 ? 8 : 5;
}

struct DecodeLayerArgs {
  FusedArgs qkv, o, mlp, down;  // one activation row each; qkv carries attn_out / attn_cnt
  unsigned* bar;                // [2]: arrival count, generation
  int* err;
  const P2PDev* pd;             // AR form: the rank's P2P group (o and down all-reduced)
  int x_bytes;                  // shared bytes of the staged activation row (largest K)
};

__device__ __forceinline__ void dl_cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void dl_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void dl_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ unsigned long long dl_time() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Grid-wide barrier (all CTAs resident).  `err0` is *err as this CTA found it at the
// start of the launch: once a wait of this launch has given up (raising *err), the
// later waits of every CTA give up at once instead of running out their time too.
__device__ void dl_grid_barrier(unsigned* bar, int* err, int err0) {
  __threadfence();  // this thread's writes of the phase, device-wide, before the arrival
  __syncthreads();
  if (threadIdx.x == 0) {
    volatile unsigned* gen = bar + 1;
    const unsigned g = *gen;
    __threadfence();  // the generation is read before this CTA arrives
    if (atomicAdd(&bar[0], 1u) == gridDim.x - 1) {
      atomicExch(&bar[0], 0u);  // before the generation moves: no CTA arrives at the next barrier earlier
      __threadfence();
      atomicExch(&bar[1], g + 1);
    } else {
      const unsigned long long t0 = dl_time();
      while (*gen == g) {
        if (dl_time() - t0 > kDlWaitNs || (err && *(volatile int*)err != err0)) {
          if (err) atomicExch(err, 1);
          break;
        }
        __nanosleep(64);
      }
      __threadfence();  // acquire: the generation seen, then the phase's data
    }
  }
  __syncthreads();
  __threadfence();  // the other CTAs' writes, seen through the barrier, before this CTA reads them
}

// The projection epilogue of gemv_epilogue.cuh for activation row 0, except that a
// residual is read through L2: it was written earlier in this launch by other CTAs.
template <typename T, int MODE>
__device__ __forceinline__ void dl_epilogue(const FusedArgs& a, int t, float v1, float v2) {
  if (MODE == MODE_PLAIN && a.residual) {
    const T r = __ldcg(static_cast<const T*>(a.residual) + t);
    static_cast<T*>(a.y)[t] = from_f<T>(rnd<T>(v1) + to_f(r));
  } else {
    row_epilogue<T, MODE>(a, t, 0, v1, v2);
  }
}

// One staged-GEMV phase over tasks [t_lo, t_hi) of projection `a` (one activation row).
template <typename T, int MODE, bool NORM>
struct DlPhase {
  static constexpr int NW = (MODE == MODE_PLAIN) ? 1 : 2;
  static constexpr int U = kDlU;
  static constexpr int S = dl_slots<NW>();
  static constexpr int V = VecW<T>::n;

  const FusedArgs* pa;  // kernel parameters or a table in device memory
  int K, nch, ms, t_lo, t_hi, nt, s_lo, s_hi;
  int itl, isub, islot, left;
  int4* my;
  const T* w;

  __device__ DlPhase(const FusedArgs& args, int4* ring) : pa(&args) {
    const FusedArgs& a = *pa;
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    K = a.K;
    nch = K / V;
    ms = (nch + kDlStageChunks - 1) / kDlStageChunks;
    if (ms < 1) ms = 1;  // an empty phase (the step kernel's absent head): no tasks, no stages
    const int ntasks = projection_tasks(a, MODE);
    t_lo = (int)(((long long)blockIdx.x * ntasks) / gridDim.x);
    t_hi = (int)(((long long)(blockIdx.x + 1) * ntasks) / gridDim.x);
    nt = t_hi - t_lo;
    const int nstages = nt * ms;
    s_lo = (int)(((long long)warp * nstages) / kDlWarps);
    s_hi = (int)(((long long)(warp + 1) * nstages) / kDlWarps);
    itl = s_lo / ms;
    isub = s_lo - itl * ms;
    islot = 0;
    left = s_hi - s_lo;
    my = ring + (size_t)warp * S * U * NW * kWarp + lane;
    w = static_cast<const T*>(a.w);
  }

  __device__ void issue_next() {
    const int lane = threadIdx.x % kWarp;
    if (left > 0) {
      const int c0 = isub * kDlStageChunks + lane;
      const T* src = w + (size_t)(t_lo + itl) * NW * K;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + u * kWarp;
        if (c < nch) {
#pragma unroll
          for (int q = 0; q < NW; ++q)
            dl_cp16(my + ((islot * U + u) * NW + q) * kWarp, src + (size_t)q * K + (size_t)c * V);
        }
      }
      if (++isub == ms) {
        isub = 0;
        ++itl;
      }
      --left;
    }
    if (++islot == S) islot = 0;
    dl_commit();
  }

  // The weight prologue: independent of every earlier phase.
  __device__ void prologue() {
#pragma unroll
    for (int j = 0; j < S - 1; ++j) issue_next();
  }

  // Everything after the prologue: the (normalised) activation row, the weight stream,
  // the epilogue.  `xs` holds the row; `part` the per-(task, warp) partial sums.
  // PUSH: the epilogue stores the rounded partial of each task into every rank's
  // exchange row of `ar_slot` (ar_push) instead of writing the output.
  template <bool PUSH = false>
  __device__ void body(unsigned char* xsm, float* part, const P2PDev* pd = nullptr, int ar_slot = 0) {
    const FusedArgs& a = *pa;
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    __shared__ float red[kDlWarps];
    __shared__ float rinv;
    const int4* x4 = static_cast<const int4*>(a.x);
    int4* xs4 = reinterpret_cast<int4*>(xsm);
    float ss = 0.f;
    for (int c = threadIdx.x; c < nch; c += kDlThreads) {
      const int4 v = ld_l2(x4 + c);  // written by other CTAs of this grid (or the previous launch)
      xs4[c] = v;
      if (NORM) {
        float f[V];
        unpack(v, f, T());
#pragma unroll
        for (int e = 0; e < V; ++e) ss = fmaf(f[e], f[e], ss);
      }
    }
    if (NORM) {
      ss = warp_sum(ss);
      if (lane == 0) red[warp] = ss;
      __syncthreads();
      if (threadIdx.x == 0) {
        float s = 0.f;
        for (int i = 0; i < kDlWarps; ++i) s += red[i];
        rinv = rsqrtf(s / (float)a.K + a.eps);
      }
      __syncthreads();
      const int4* lw4 = static_cast<const int4*>(a.ln_w);
      for (int c = threadIdx.x; c < nch; c += kDlThreads) {
        float f[V], lf[V];
        unpack(xs4[c], f, T());
        unpack(ld_stream(lw4 + c), lf, T());
#pragma unroll
        for (int e = 0; e < V; ++e) f[e] = rnd<T>(rnd<T>(f[e] * rinv) * lf[e]);
        xs4[c] = pack(f, T());
      }
    }
    for (int i = threadIdx.x; i < nt * kDlWarps * NW; i += kDlThreads) part[i] = 0.f;
    __syncthreads();

    float acc[NW];
#pragma unroll
    for (int q = 0; q < NW; ++q) acc[q] = 0.f;
    auto flush = [&](int tl) {
#pragma unroll
      for (int q = 0; q < NW; ++q) {
        const float v = warp_sum(acc[q]);
        if (lane == 0) part[(tl * kDlWarps + warp) * NW + q] = v;
        acc[q] = 0.f;
      }
    };
    const int tl0 = s_lo / ms;
    int cur = tl0, sub = s_lo - tl0 * ms, slot = 0;
    for (int j = s_hi - s_lo; j > 0; --j) {
      issue_next();
      dl_wait<S - 1>();  // this lane's copies of the current stage have landed
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = sub * kDlStageChunks + u * kWarp + lane;
        if (c < nch) {
          const int4 xv = xs4[c];
#pragma unroll
          for (int q = 0; q < NW; ++q) {
            const int4 wv = my[((slot * U + u) * NW + q) * kWarp];
            if constexpr (kIsBf16<T>) {
              acc[q] = fma8_bf16(wv, xv, acc[q]);
            } else {
              float xf[V], wf[V];
              unpack(xv, xf, T());
              unpack(wv, wf, T());
#pragma unroll
              for (int e = 0; e < V; ++e) acc[q] = fmaf(wf[e], xf[e], acc[q]);
            }
          }
        }
      }
      if (++slot == S) slot = 0;
      if (++sub == ms && j > 1) {
        flush(cur);
        sub = 0;
        ++cur;
      }
    }
    if (s_lo < s_hi) flush(cur);
    dl_wait<0>();
    __syncthreads();
    for (int tl = threadIdx.x; tl < nt; tl += kDlThreads) {
      float v[2] = {0.f, 0.f};
#pragma unroll
      for (int q = 0; q < NW; ++q)
        for (int wp = 0; wp < kDlWarps; ++wp) v[q] += part[(tl * kDlWarps + wp) * NW + q];
      if constexpr (PUSH)
        ar_push<T>(pd, ar_slot, (size_t)(t_lo + tl), v[0]);
      else
        dl_epilogue<T, MODE>(a, t_lo + tl, v[0], v[1]);
    }
  }
};

// Phases 1-4 of one layer.  On entry `p1` (the layer's q/k/v phase) has its weight
// prologue issued and the layer's input is complete.  `next()` runs once the down phase's
// outputs (or, AR, its partials) are written and before its all-reduce: it issues the
// prologue of whatever phase follows, so those weights stream during the peer wait and
// across the barrier after it.  `s_err0` and `s_epoch` are the kernel's shared words,
// written by thread 0 after griddepcontrol.wait and read here only after a CTA barrier;
// the layer's first all-reduce (AR) has epoch *s_epoch + e_off.
template <typename T, bool AR, typename Next>
__device__ __forceinline__ void dl_layer_phases(const DecodeLayerArgs& L, DlPhase<T, MODE_ROPE, true>& p1,
                                                unsigned char* xs, int4* ring, float* part, unsigned* bar,
                                                int* err, const int* s_err0, const P2PDev* pd,
                                                const int* s_epoch, int e_off, Next next) {
  p1.body(xs, part);
  DlPhase<T, MODE_PLAIN, false> p2(L.o, ring);
  p2.prologue();  // o_proj weights stream while the attention runs and the grid meets
  fa_tail<T>(L.qkv, p1.t_lo, p1.t_hi, reinterpret_cast<float*>(xs));
  dl_grid_barrier(bar, err, *s_err0);
  DlPhase<T, MODE_SILU, true> p3(L.mlp, ring);
  const int e1 = AR ? *s_epoch + e_off : 0;
  if constexpr (AR) {
    p2.template body<true>(xs, part, pd, e1 & 1);
    p3.prologue();  // gate/up weights stream during the wait for the peers
    ar_reduce<T>(L.o, pd, p2.t_lo, p2.nt, e1, e1 & 1);
  } else {
    p2.body(xs, part);
    p3.prologue();
  }
  dl_grid_barrier(bar, err, *s_err0);
  p3.body(xs, part);
  DlPhase<T, MODE_PLAIN, false> p4(L.down, ring);
  p4.prologue();
  dl_grid_barrier(bar, err, *s_err0);
  if constexpr (AR) {
    const int e2 = e1 + 1;
    p4.template body<true>(xs, part, pd, e2 & 1);
    next();
    ar_reduce<T>(L.down, pd, p4.t_lo, p4.nt, e2, e2 & 1);
  } else {
    p4.body(xs, part);
    next();
  }
}

template <typename T, bool AR>
__global__ void __launch_bounds__(kDlThreads, 2) decode_layer_kernel(DecodeLayerArgs L) {
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned char* xs = smem;
  int4* ring = reinterpret_cast<int4*>(smem + L.x_bytes);
  float* part = reinterpret_cast<float*>(smem + L.x_bytes + kDlRingBytes);

  __shared__ int s_err0, s_epoch;
  if constexpr (!AR) pdl_trigger();
  DlPhase<T, MODE_ROPE, true> p1(L.qkv, ring);
  p1.prologue();
  pdl_wait();  // the previous layer's output (this layer's input) is complete
  if (threadIdx.x == 0) {  // read by thread 0; s_epoch is read by all after later CTA barriers
    s_err0 = L.err ? *(volatile int*)L.err : 0;
    if constexpr (AR) s_epoch = *(volatile int*)L.pd->counter + 1;
  }
  dl_layer_phases<T, AR>(L, p1, xs, ring, part, L.bar, L.err, &s_err0, L.pd, &s_epoch, 0, [] {});
  if constexpr (AR) pdl_trigger();
}

// A whole decode step: the layers of a table in device memory, each as above, with a
// grid barrier (instead of a kernel boundary) between consecutive layers -- the next
// layer's q/k/v weights in flight across it -- then the lm_head_in phase (final rmsnorm
// and the vocabulary GEMV) when `head.w` is set.  AR: two all-reduce epochs per layer.
struct DecodeStepArgs {
  const DecodeLayerArgs* layers;  // device table (qkv / o / mlp / down of each layer)
  int nlayers;
  FusedArgs head;                 // PLAIN with rmsnorm; head.w == nullptr: no head phase
  unsigned* bar;
  int* err;
  const P2PDev* pd;
  int x_bytes;
};

template <typename T, bool AR>
__global__ void __launch_bounds__(kDlThreads, 2) decode_step_kernel(DecodeStepArgs S) {
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned char* xs = smem;
  int4* ring = reinterpret_cast<int4*>(smem + S.x_bytes);
  float* part = reinterpret_cast<float*>(smem + S.x_bytes + kDlRingBytes);

  __shared__ int s_err0, s_epoch;
  if constexpr (!AR) pdl_trigger();
  DlPhase<T, MODE_ROPE, true> p1(S.layers[0].qkv, ring);
  p1.prologue();
  pdl_wait();  // the step's input (the embedding row) is complete
  if (threadIdx.x == 0) {
    s_err0 = S.err ? *(volatile int*)S.err : 0;
    if constexpr (AR) s_epoch = *(volatile int*)S.pd->counter + 1;
  }
  DlPhase<T, MODE_PLAIN, true> ph(S.head, ring);
  const bool head = S.head.w != nullptr;
  for (int l = 0; l < S.nlayers; ++l) {
    const bool last = l + 1 == S.nlayers;
    dl_layer_phases<T, AR>(S.layers[l], p1, xs, ring, part, S.bar, S.err, &s_err0, S.pd, &s_epoch, 2 * l,
                           [&] {
                             if (!last) {
                               p1 = DlPhase<T, MODE_ROPE, true>(S.layers[l + 1].qkv, ring);
                               p1.prologue();
                             } else if (head) {
                               ph.prologue();
                             }
                           });
    if (!last || head) dl_grid_barrier(S.bar, S.err, s_err0);  // thread 0 reads its own write
  }
  if (head) ph.body(xs, part);
  if constexpr (AR) pdl_trigger();
}

static int dl_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// Shared bytes of the activation row (the largest K of any phase) -- at least the attention
// tail's merge buffers: fa_head_row's G = warps * (32 / lanes per key) groups of (max,
// sum, hd accumulators).
static size_t dl_x_bytes(int kmax, int hd, size_t es) {
  size_t x_bytes = ((size_t)kmax * es + 15) / 16 * 16;
  const int groups = kDlWarps * (kWarp / (hd / (16 / (int)es)));
  const size_t attn_scratch = (size_t)groups * (hd + 2) * sizeof(float);
  return x_bytes < attn_scratch ? (attn_scratch + 15) / 16 * 16 : x_bytes;
}

// Per-CTA partial sums: the most (task, weight row) pairs any phase gives one CTA.
static int dl_tmax(const FusedArgs* const* ph, const int* modes, int n, int grid) {
  int tmax = 0;
  for (int i = 0; i < n; ++i) {
    const int nw = modes[i] == MODE_PLAIN ? 1 : 2;
    const int t = (projection_tasks(*ph[i], modes[i]) + grid - 1) / grid * nw;
    if (t > tmax) tmax = t;
  }
  return tmax;
}

// Grid and dynamic shared memory of a layer or step kernel: two CTAs per SM when they fit
// in 112 KB each and the SM holds them (occupancy API), else one; every CTA must be
// resident for the grid barriers.  Returns cudaErrorNotSupported when neither fits.
template <typename Kern>
static cudaError_t dl_geometry(Kern kern, ResidentCache& cache, size_t x_bytes, const FusedArgs* const* ph,
                               const int* modes, int n, int* grid_out, size_t* smem_out) {
  for (int occ = 2; occ >= 1; --occ) {
    const int grid = dl_sms() * occ;
    const size_t smem = x_bytes + kDlRingBytes + (size_t)dl_tmax(ph, modes, n, grid) * kDlWarps * sizeof(float);
    if (smem > (occ == 2 ? 112 * 1024 : 220 * 1024)) continue;
    cudaError_t e;
    const int fits = resident_ctas(kern, kDlThreads, smem, cache, &e);
    if (fits < 0) return e;
    if (fits < occ) continue;
    *grid_out = grid;
    *smem_out = smem;
    return cudaSuccess;
  }
  return cudaErrorNotSupported;
}

template <typename T, bool AR>
static cudaError_t launch_decode_layer(DecodeLayerArgs L, cudaStream_t st) {
  int kmax = L.qkv.K;
  if (L.o.K > kmax) kmax = L.o.K;
  if (L.mlp.K > kmax) kmax = L.mlp.K;
  if (L.down.K > kmax) kmax = L.down.K;
  L.x_bytes = (int)dl_x_bytes(kmax, L.qkv.hd, sizeof(T));
  const FusedArgs* ph[4] = {&L.qkv, &L.o, &L.mlp, &L.down};
  const int modes[4] = {MODE_ROPE, MODE_PLAIN, MODE_SILU, MODE_PLAIN};
  static ResidentCache cache;
  int grid = 0;
  size_t smem = 0;
  const cudaError_t e = dl_geometry(decode_layer_kernel<T, AR>, cache, L.x_bytes, ph, modes, 4, &grid, &smem);
  if (e != cudaSuccess) return e;
  return launch_coop(decode_layer_kernel<T, AR>, dim3(grid), dim3(kDlThreads), smem, st, L);
}

cudaError_t decode_layer(const FusedArgs& qkv, const FusedArgs& o, const FusedArgs& mlp, const FusedArgs& down,
                         unsigned* bar, int* err, int dtype, cudaStream_t st) {
  DecodeLayerArgs L;
  L.qkv = qkv;
  L.o = o;
  L.mlp = mlp;
  L.down = down;
  L.bar = bar;
  L.err = err;
  L.pd = static_cast<const P2PDev*>(o.p2p);  // both row-parallel phases, or neither
  L.x_bytes = 0;
  if (L.pd)
    return dtype == BF16 ? launch_decode_layer<__nv_bfloat16, true>(L, st) : launch_decode_layer<float, true>(L, st);
  return dtype == BF16 ? launch_decode_layer<__nv_bfloat16, false>(L, st) : launch_decode_layer<float, false>(L, st);
}

// ---- the whole-step kernel: host side ----------------------------------------------

size_t decode_step_table_bytes(int nlayers) { return (size_t)nlayers * sizeof(DecodeLayerArgs); }

}  // namespace pim

struct pim_decode_step_plan {
  pim::DecodeStepArgs args;  // bar / err set at each launch
  int dtype;
  bool ar;
  int grid;
  size_t smem;
};

namespace pim {

template <typename T, bool AR>
static cudaError_t size_step(pim_decode_step_plan* p, const std::vector<DecodeLayerArgs>& layers) {
  std::vector<const FusedArgs*> ph;
  std::vector<int> modes;
  int kmax = 0, hd = 0;
  for (const DecodeLayerArgs& L : layers) {
    const FusedArgs* f[4] = {&L.qkv, &L.o, &L.mlp, &L.down};
    const int m[4] = {MODE_ROPE, MODE_PLAIN, MODE_SILU, MODE_PLAIN};
    for (int i = 0; i < 4; ++i) {
      ph.push_back(f[i]);
      modes.push_back(m[i]);
      if (f[i]->K > kmax) kmax = f[i]->K;
    }
    if (L.qkv.hd > hd) hd = L.qkv.hd;
  }
  if (p->args.head.w) {
    ph.push_back(&p->args.head);
    modes.push_back(MODE_PLAIN);
    if (p->args.head.K > kmax) kmax = p->args.head.K;
  }
  p->args.x_bytes = (int)dl_x_bytes(kmax, hd, sizeof(T));
  static ResidentCache cache;
  return dl_geometry(decode_step_kernel<T, AR>, cache, p->args.x_bytes, ph.data(), modes.data(), (int)ph.size(),
                     &p->grid, &p->smem);
}

cudaError_t decode_step_prepare(const FusedArgs* phases, int nlayers, const FusedArgs* head, int dtype, void* table,
                                size_t table_bytes, pim_decode_step_plan** out) {
  if (nlayers <= 0 || table_bytes < decode_step_table_bytes(nlayers)) return cudaErrorInvalidValue;
  std::vector<DecodeLayerArgs> layers((size_t)nlayers);
  for (int l = 0; l < nlayers; ++l) {
    DecodeLayerArgs& L = layers[l];
    L.qkv = phases[4 * l];
    L.o = phases[4 * l + 1];
    L.mlp = phases[4 * l + 2];
    L.down = phases[4 * l + 3];
    L.bar = nullptr;
    L.err = nullptr;
    L.pd = static_cast<const P2PDev*>(L.o.p2p);
    L.x_bytes = 0;
  }
  pim_decode_step_plan* p = new pim_decode_step_plan{};
  p->args.layers = static_cast<const DecodeLayerArgs*>(table);
  p->args.nlayers = nlayers;
  p->args.head = head ? *head : FusedArgs{};
  p->args.pd = layers[0].pd;
  p->dtype = dtype;
  p->ar = p->args.pd != nullptr;
  cudaError_t e;
  if (dtype == BF16)
    e = p->ar ? size_step<__nv_bfloat16, true>(p, layers) : size_step<__nv_bfloat16, false>(p, layers);
  else
    e = p->ar ? size_step<float, true>(p, layers) : size_step<float, false>(p, layers);
  if (e == cudaSuccess)
    e = cudaMemcpy(table, layers.data(), decode_step_table_bytes(nlayers), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    delete p;
    return e;
  }
  *out = p;
  return cudaSuccess;
}

cudaError_t decode_step(const pim_decode_step_plan* p, unsigned* bar, int* err, cudaStream_t st) {
  DecodeStepArgs a = p->args;
  a.bar = bar;
  a.err = err;
  const dim3 grid(p->grid), block(kDlThreads);
  if (p->dtype == BF16)
    return p->ar ? launch_coop(decode_step_kernel<__nv_bfloat16, true>, grid, block, p->smem, st, a)
                 : launch_coop(decode_step_kernel<__nv_bfloat16, false>, grid, block, p->smem, st, a);
  return p->ar ? launch_coop(decode_step_kernel<float, true>, grid, block, p->smem, st, a)
               : launch_coop(decode_step_kernel<float, false>, grid, block, p->smem, st, a);
}

void decode_step_free(pim_decode_step_plan* p) { delete p; }

}  // namespace pim
