// Decode-path projection kernels: one warp per weight row (or row pair), 16-byte
// streaming loads of the weight, the activation rows staged once per CTA in shared
// memory, fp32 accumulation and a warp-shuffle reduction.
//
// Fused variants (the nodes of the step graph):
//   PLAIN  y[r, n]            = x[r] . W[n]
//   ROPE   (attn_in)          rmsnorm(x) . W_qkv, RoPE on the q/k column pairs
//                             (j, j + hd/2), q written out, k/v appended to the KV
//                             blocks at the row's position
//   SILU   (mlp_in)           rmsnorm(x) . [gate_j ; up_j] -> silu(gate) * up
// The optional rmsnorm prologue is recomputed by every CTA from x (a few KB out of
// L2), so no separate normalisation pass or buffer exists on the decode path.
//
// Rounding follows the HF bf16 model: every tensor HF materialises in bf16 is
// rounded here at the same point (rnd<T>), accumulation stays fp32.

#include <stdlib.h>

#include <atomic>

#include "gemv_epilogue.cuh"
#include "pim_common.cuh"
#include "pim_kernels.h"

namespace pim {

// Loads one batch (U 16-byte chunks per weight row, NW rows) of a warp's current task.
template <typename T, int NW, int U>
__device__ __forceinline__ void load_batch(int4 (&v)[NW][U], const T* __restrict__ w0, const T* __restrict__ w1,
                                           int c0, int nch) {
  const int4* p0 = reinterpret_cast<const int4*>(w0);
  const int4* p1 = reinterpret_cast<const int4*>(w1);
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int c = c0 + u * kWarp;
    if (c < nch) {
      v[0][u] = ld_stream(p0 + c);
      if (NW == 2) v[NW - 1][u] = ld_stream(p1 + c);
    }
  }
}

template <typename T, int NW, int U, int RMAX>
__device__ __forceinline__ void fma_batch(const int4 (&v)[NW][U], const T* __restrict__ xs, int K, int rows,
                                          int c0, int nch, float (&acc)[2][RMAX]) {
  constexpr int V = VecW<T>::n;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int c = c0 + u * kWarp;
    if (c < nch) {
      float wf[NW][V];
#pragma unroll
      for (int i = 0; i < NW; ++i) unpack(v[i][u], wf[i], T());
#pragma unroll
      for (int r = 0; r < RMAX; ++r) {
        if (r < rows) {
          const int4 xv = *reinterpret_cast<const int4*>(xs + (size_t)r * K + (size_t)c * V);
          float xf[V];
          unpack(xv, xf, T());
#pragma unroll
          for (int i = 0; i < NW; ++i)
#pragma unroll
            for (int e = 0; e < V; ++e) acc[i][r] = fmaf(wf[i][e], xf[e], acc[i][r]);
        }
      }
    }
  }
}

// Scalar dot for shapes whose rows are not 16-byte aligned.
template <typename T, int NW, int RMAX>
__device__ __forceinline__ void dot_scalar(const T* __restrict__ w0, const T* __restrict__ w1,
                                           const T* __restrict__ xs, int K, int rows, int lane,
                                           float (&acc)[2][RMAX]) {
  for (int k = lane; k < K; k += kWarp) {
    const float a0 = to_f(w0[k]);
    const float a1 = NW == 2 ? to_f(w1[k]) : 0.f;
#pragma unroll
    for (int r = 0; r < RMAX; ++r) {
      if (r < rows) {
        const float xv = to_f(xs[(size_t)r * K + k]);
        acc[0][r] = fmaf(a0, xv, acc[0][r]);
        if (NW == 2) acc[1][r] = fmaf(a1, xv, acc[1][r]);
      }
    }
  }
}

// Weight rows of task t.  PLAIN: row t.  The two-row modes use the pair-interleaved
// weight layout, so task t is always rows (2t, 2t + 1): ROPE the columns (j, j + hd/2)
// of head block t / (hd/2) with j = t % (hd/2); SILU the gate row and the up row of
// output column t.
template <int MODE>
__device__ __forceinline__ void task_rows(int t, int& n1, int& n2) {
  n1 = MODE == MODE_PLAIN ? t : 2 * t;
  n2 = MODE == MODE_PLAIN ? t : 2 * t + 1;
}

// Lane r finishes activation row r of task t.
template <typename T, int MODE, int RMAX>
__device__ __forceinline__ void task_epilogue(const FusedArgs& a, int t, int lane, float (&acc)[2][RMAX]) {
#pragma unroll
  for (int r = 0; r < RMAX; ++r)
    if (lane == r && r < a.rows) row_epilogue<T, MODE>(a, t, r, acc[0][r], acc[1][r]);
}

// Each CTA owns a contiguous, balanced range of tasks; its warps take the range's
// tasks in turn.  A warp's weight loads run one batch ahead of its arithmetic: the
// next batch (possibly the next task's first) is issued before the finished task's
// reduction and epilogue.  The first batch is issued before pdl_wait(), so with
// programmatic dependent launch the weight stream of this kernel overlaps the tail
// of the previous kernel (weights never depend on it; x does).
template <typename T, int MODE, int RMAX, bool NORM, bool VEC>
__global__ void __launch_bounds__(256, 2) fused_gemv_kernel(FusedArgs a) {
  constexpr int NW = (MODE == MODE_PLAIN) ? 1 : 2;
  constexpr int U = (NW == 1) ? 16 : 8;
  constexpr int V = VecW<T>::n;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* xs = reinterpret_cast<T*>(smem_raw);
  __shared__ float red[8][RMAX];
  __shared__ float rinv[RMAX];
  const T* __restrict__ x = static_cast<const T*>(a.x);
  const T* __restrict__ w = static_cast<const T*>(a.w);
  const int K = a.K, rows = a.rows;
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int wpb = blockDim.x / kWarp;
  const int nch = K / V;
  const int ntasks = projection_tasks(a, MODE);
  const int t_lo = (int)(((long long)blockIdx.x * ntasks) / gridDim.x);
  const int t_hi = (int)(((long long)(blockIdx.x + 1) * ntasks) / gridDim.x);

  pdl_trigger();
  int t = t_lo + warp, c0 = lane, n1 = 0, n2 = 0;
  int4 v[NW][U];
  if (VEC && t < t_hi) {
    task_rows<MODE>(t, n1, n2);
    load_batch<T, NW, U>(v, w + (size_t)n1 * K, w + (size_t)n2 * K, c0, nch);
  }
  pdl_wait();

  // ---- stage (normalised) activation rows in shared memory -------------------
  if (NORM) {
    const T* __restrict__ lw = static_cast<const T*>(a.ln_w);
#pragma unroll
    for (int r = 0; r < RMAX; ++r) {
      float ss = 0.f;
      if (r < rows)
        for (int k = threadIdx.x; k < K; k += blockDim.x) {
          const float xv = to_f(x[(size_t)r * K + k]);
          ss = fmaf(xv, xv, ss);
        }
      ss = warp_sum(ss);
      if (lane == 0) red[warp][r] = ss;
    }
    __syncthreads();
    if (threadIdx.x < RMAX) {
      float s = 0.f;
      for (int i = 0; i < wpb; ++i) s += red[i][threadIdx.x];
      rinv[threadIdx.x] = rsqrtf(s / (float)K + a.eps);
    }
    __syncthreads();
    for (int r = 0; r < rows; ++r)
      for (int k = threadIdx.x; k < K; k += blockDim.x) {
        const float y = rnd<T>(to_f(x[(size_t)r * K + k]) * rinv[r]);
        xs[(size_t)r * K + k] = from_f<T>(y * to_f(lw[k]));
      }
  } else {
    for (int r = 0; r < rows; ++r)
      for (int k = threadIdx.x; k < K; k += blockDim.x) xs[(size_t)r * K + k] = x[(size_t)r * K + k];
  }
  __syncthreads();

  float acc[2][RMAX];
#pragma unroll
  for (int r = 0; r < RMAX; ++r) acc[0][r] = acc[1][r] = 0.f;
  if constexpr (!VEC) {
    for (; t < t_hi; t += wpb) {
      task_rows<MODE>(t, n1, n2);
#pragma unroll
      for (int r = 0; r < RMAX; ++r) acc[0][r] = acc[1][r] = 0.f;
      dot_scalar<T, NW, RMAX>(w + (size_t)n1 * K, w + (size_t)n2 * K, xs, K, rows, lane, acc);
#pragma unroll
      for (int r = 0; r < RMAX; ++r) {
        acc[0][r] = warp_sum(acc[0][r]);
        if (NW == 2) acc[1][r] = warp_sum(acc[1][r]);
      }
      task_epilogue<T, MODE, RMAX>(a, t, lane, acc);
    }
  } else {
    while (t < t_hi) {
      fma_batch<T, NW, U, RMAX>(v, xs, K, rows, c0, nch, acc);
      int nt = t, nc0 = c0 + kWarp * U;
      const bool done = nc0 >= nch;
      if (done) {
        nt = t + wpb;
        nc0 = lane;
      }
      if (nt < t_hi) {
        if (done) task_rows<MODE>(nt, n1, n2);
        load_batch<T, NW, U>(v, w + (size_t)n1 * K, w + (size_t)n2 * K, nc0, nch);
      }
      if (done) {
#pragma unroll
        for (int r = 0; r < RMAX; ++r) {
          acc[0][r] = warp_sum(acc[0][r]);
          if (NW == 2) acc[1][r] = warp_sum(acc[1][r]);
        }
        task_epilogue<T, MODE, RMAX>(a, t, lane, acc);
#pragma unroll
        for (int r = 0; r < RMAX; ++r) acc[0][r] = acc[1][r] = 0.f;
      }
      t = nt;
      c0 = nc0;
    }
  }
}

// ---------------------------------------------------------------------------------
// Row-batched path (prefill, batched decode): rmsnorm -> GEMM -> epilogue.
// ---------------------------------------------------------------------------------

template <typename T>
__global__ void rmsnorm_rows_kernel(const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ y,
                                    int K, float eps) {
  const int r = blockIdx.x;
  __shared__ float red[32];
  float ss = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const float v = to_f(x[(size_t)r * K + k]);
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  if (threadIdx.x % kWarp == 0) red[threadIdx.x / kWarp] = ss;
  __syncthreads();
  if (threadIdx.x < kWarp) {
    float s = threadIdx.x < blockDim.x / kWarp ? red[threadIdx.x] : 0.f;
    s = warp_sum(s);
    if (threadIdx.x == 0) red[0] = rsqrtf(s / (float)K + eps);
  }
  __syncthreads();
  const float ri = red[0];
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const float v = rnd<T>(to_f(x[(size_t)r * K + k]) * ri);
    y[(size_t)r * K + k] = from_f<T>(v * to_f(w[k]));
  }
}

// The same with 16-byte loads and stores, for rows whose bytes are a multiple of 16 (and
// at most 48 KB): the row goes to shared memory in one pass, each thread then adds its
// squares in the order of rmsnorm_rows_kernel (elements t, t + 256, ...), so the norm and
// every output are bit-identical to it; x is read once instead of twice.
template <typename T>
__global__ void rmsnorm_rows_vec_kernel(const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ y,
                                        int K, float eps) {
  constexpr int V = VecW<T>::n;
  extern __shared__ __align__(16) unsigned char rn_smem[];
  int4* row = reinterpret_cast<int4*>(rn_smem);
  const T* rs = reinterpret_cast<const T*>(rn_smem);
  const int r = blockIdx.x;
  const int nch = K / V;
  const int4* x4 = reinterpret_cast<const int4*>(x + (size_t)r * K);
  for (int c = threadIdx.x; c < nch; c += blockDim.x) row[c] = ld_stream(x4 + c);
  __syncthreads();
  __shared__ float red[32];
  float ss = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const float v = to_f(rs[k]);
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  if (threadIdx.x % kWarp == 0) red[threadIdx.x / kWarp] = ss;
  __syncthreads();
  if (threadIdx.x < kWarp) {
    float sum = threadIdx.x < blockDim.x / kWarp ? red[threadIdx.x] : 0.f;
    sum = warp_sum(sum);
    if (threadIdx.x == 0) red[0] = rsqrtf(sum / (float)K + eps);
  }
  __syncthreads();
  const float ri = red[0];
  const int4* w4 = reinterpret_cast<const int4*>(w);
  int4* y4 = reinterpret_cast<int4*>(y + (size_t)r * K);
  for (int c = threadIdx.x; c < nch; c += blockDim.x) {
    float f[V], wf[V];
    unpack(row[c], f, T());
    unpack(ld_stream(w4 + c), wf, T());
#pragma unroll
    for (int e = 0; e < V; ++e) f[e] = rnd<T>(rnd<T>(f[e] * ri) * wf[e]);
    y4[c] = pack(f, T());
  }
}

// Tiled CUDA-core GEMM  C[M,N] = A[M,K] . B[N,K]^T  with fp32 accumulation.
// 64x64 tile, 16-deep K slices, 256 threads each owning a 4x4 block.
template <typename T, typename OutT>
__global__ void __launch_bounds__(256) gemm_tn_kernel(const T* __restrict__ A, const T* __restrict__ B,
                                                      OutT* __restrict__ C, int M, int N, int K) {
  __shared__ float As[16][64 + 4];
  __shared__ float Bs[16][64 + 4];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int i = threadIdx.x; i < 64 * 16; i += 256) {
      const int rr = i / 16, kk = i % 16;
      const int gm = m0 + rr, gn = n0 + rr, gk = k0 + kk;
      As[kk][rr] = (gm < M && gk < K) ? to_f(A[(size_t)gm * K + gk]) : 0.f;
      Bs[kk][rr] = (gn < N && gk < K) ? to_f(B[(size_t)gn * K + gk]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        av[i] = As[kk][ty * 4 + i];
        bv[i] = Bs[kk][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) acc[i][jj] = fmaf(av[i], bv[jj], acc[i][jj]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int gm = m0 + ty * 4 + i, gn = n0 + tx * 4 + jj;
      if (gm < M && gn < N) C[(size_t)gm * N + gn] = from_f<OutT>(acc[i][jj]);
    }
}

// RoPE + KV append epilogue over a fp32 GEMM result tmp[rows, (hq+2hkv)*hd]; one CTA per row.
template <typename T>
__global__ void rope_kv_epilogue_kernel(const float* __restrict__ tmp, FusedArgs a) {
  const int r = blockIdx.x;
  const int ntasks = projection_tasks(a, MODE_ROPE);
  const float* row = tmp + (size_t)r * 2 * ntasks;
  for (int t = threadIdx.x; t < ntasks; t += blockDim.x)  // pair-interleaved columns (2t, 2t + 1)
    row_epilogue<T, MODE_ROPE>(a, t, r, row[2 * t], row[2 * t + 1]);
}

template <typename T>
__global__ void residual_epilogue_kernel(const float* __restrict__ tmp, const T* __restrict__ res, T* __restrict__ y,
                                         int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = from_f<T>(rnd<T>(tmp[i]) + to_f(res[i]));
}

template <typename T>
__global__ void silu_pair_epilogue_kernel(const float* __restrict__ tmp, T* __restrict__ y, int rows, int inter) {
  const int64_t total = (int64_t)rows * inter;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / inter, t = i % inter;
    const float g = rnd<T>(tmp[r * 2 * inter + 2 * t]), u = rnd<T>(tmp[r * 2 * inter + 2 * t + 1]);
    const float act = rnd<T>(g / (1.f + expf(-g)));
    y[i] = from_f<T>(act * u);
  }
}

// ---------------------------------------------------------------------------------
// host-side dispatch
// ---------------------------------------------------------------------------------

bool pdl_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("PIM_PDL");
    on = (e && e[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

// Decode projection kernel (rows <= kGemvMaxRows): by default the cp.async-staged
// kernel (gemv_async.cu); PIM_GEMV="reg" selects the register kernel above and "dyn" the
// staged kernel with dynamic work assignment (gemv_dynamic.cu) at the first call, and
// set_gemv_variant() at any time.
// Shapes a variant cannot take run on the register kernel.
static std::atomic<int> g_gemv_variant{-1};

int gemv_variant() {
  int v = g_gemv_variant.load(std::memory_order_relaxed);
  if (v < 0) {
    const char* e = getenv("PIM_GEMV");
    v = kGemvStaged;
    if (e && e[0] == 'r') v = kGemvRegister;
    if (e && e[0] == 'd') v = kGemvDynamic;
    int expected = -1;
    if (!g_gemv_variant.compare_exchange_strong(expected, v)) v = expected;
  }
  return v;
}

void set_gemv_variant(int v) { g_gemv_variant.store(v, std::memory_order_relaxed); }

static int g_num_sms = 0;

static int num_sms() {
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  return g_num_sms;
}

template <typename T, int MODE, int RMAX, bool NORM>
static cudaError_t launch_fused_rmax(const FusedArgs& a, cudaStream_t st) {
  const size_t smem = (size_t)a.rows * a.K * sizeof(T);
  const bool vec = (a.K % VecW<T>::n == 0) && ((uintptr_t)a.w % 16 == 0);
  const int ntasks = projection_tasks(a, MODE);
  const int threads = 256, wpb = threads / kWarp;
  auto kern = vec ? fused_gemv_kernel<T, MODE, RMAX, NORM, true> : fused_gemv_kernel<T, MODE, RMAX, NORM, false>;
  // Opt-in shared memory and occupancy are queried once per (kernel, smem size) and cached,
  // so launches inside a CUDA-graph capture make no attribute calls.
  static size_t cached_smem[2] = {0, 0};
  static int cached_occ[2] = {0, 0};
  const int slot = vec ? 1 : 0;
  if (cached_smem[slot] < smem || cached_occ[slot] == 0) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    int o = 1;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, kern, threads, smem);
    cached_smem[slot] = smem;
    cached_occ[slot] = o < 1 ? 1 : o;
  }
  const int occ = cached_occ[slot];
  int grid = ceil_div(ntasks, wpb);
  const int cap = num_sms() * occ;
  if (grid > cap) grid = cap;
  return launch_pdl(kern, dim3(grid), dim3(threads), smem, st, a);
}

template <typename T, int MODE, bool NORM>
static cudaError_t launch_fused_t(const FusedArgs& a, cudaStream_t st) {
  if (a.rows <= 1) return launch_fused_rmax<T, MODE, 1, NORM>(a, st);
  if (a.rows <= 2) return launch_fused_rmax<T, MODE, 2, NORM>(a, st);
  if (a.rows <= 4) return launch_fused_rmax<T, MODE, 4, NORM>(a, st);
  return launch_fused_rmax<T, MODE, 8, NORM>(a, st);
}

template <typename T>
static cudaError_t launch_gemm(const T* A, const T* B, void* C, bool out_f32, int M, int N, int K,
                               cudaStream_t st) {
  dim3 grid(ceil_div(N, 64), ceil_div(M, 64));
  if (out_f32)
    launch_plain(gemm_tn_kernel<T, float>, grid, 256, 0, st, A, B, static_cast<float*>(C), M, N, K);
  else
    launch_plain(gemm_tn_kernel<T, T>, grid, 256, 0, st, A, B, static_cast<T*>(C), M, N, K);
  return cudaGetLastError();
}

// Row-batched projection: rmsnorm rows (when normalising) -> GEMM -> epilogue.  bf16
// with K % 8 == 0 runs on the tensor cores with the epilogue fused (gemm_tc.cu); other
// shapes and fp32 take the CUDA-core GEMM and a separate epilogue over an fp32 result.
template <typename T>
static cudaError_t fused_rows_t(const FusedArgs& a, int mode, bool norm, void* scratch, cudaStream_t st) {
  // scratch layout: [xn: rows*K*sizeof(T), 256-aligned][tmp: rows*width*4, CUDA-core path only]
  const T* xin = static_cast<const T*>(a.x);
  char* sp = static_cast<char*>(scratch);
  T* xn = reinterpret_cast<T*>(sp);
  size_t xn_bytes = ((size_t)a.rows * a.K * sizeof(T) + 255) / 256 * 256;
  float* tmp = reinterpret_cast<float*>(sp + xn_bytes);
  if (norm) {
    const size_t row_bytes = (size_t)a.K * sizeof(T);
    if (row_bytes % 16 == 0 && row_bytes <= 48 * 1024 && (((uintptr_t)xin | (uintptr_t)a.ln_w | (uintptr_t)xn) & 15) == 0)
      launch_plain(rmsnorm_rows_vec_kernel<T>, a.rows, 256, row_bytes, st, xin, static_cast<const T*>(a.ln_w), xn,
                   a.K, a.eps);
    else
      launch_plain(rmsnorm_rows_kernel<T>, a.rows, 256, 0, st, xin, static_cast<const T*>(a.ln_w), xn, a.K, a.eps);
    xin = xn;
  }
  if constexpr (kIsBf16<T>) {
    if (gemm_tc_supported(a.K)) return gemm_tc(a, mode, xin, st);
  }
  const T* w = static_cast<const T*>(a.w);
  cudaError_t e;
  if (mode == MODE_PLAIN && a.residual) {
    e = launch_gemm<T>(xin, w, tmp, true, a.rows, a.ncols, a.K, st);
    if (e == cudaSuccess) {
      int grid = ceil_div((int64_t)a.rows * a.ncols, 256);
      if (grid > 4096) grid = 4096;
      launch_plain(residual_epilogue_kernel<T>, grid, 256, 0, st, tmp, static_cast<const T*>(a.residual),
                   static_cast<T*>(a.y), (int64_t)a.rows * a.ncols);
      e = cudaGetLastError();
    }
  } else if (mode == MODE_PLAIN) {
    e = launch_gemm<T>(xin, w, a.y, false, a.rows, a.ncols, a.K, st);
  } else if (mode == MODE_ROPE) {
    const int width = (a.hq + 2 * a.hkv) * a.hd;
    e = launch_gemm<T>(xin, w, tmp, true, a.rows, width, a.K, st);
    if (e == cudaSuccess) {
      launch_plain(rope_kv_epilogue_kernel<T>, a.rows, 256, 0, st, tmp, a);
      e = cudaGetLastError();
    }
  } else {
    e = launch_gemm<T>(xin, w, tmp, true, a.rows, 2 * a.inter, a.K, st);
    if (e == cudaSuccess) {
      int grid = ceil_div((int64_t)a.rows * a.inter, 256);
      if (grid > 4096) grid = 4096;
      launch_plain(silu_pair_epilogue_kernel<T>, grid, 256, 0, st, tmp, static_cast<T*>(a.y), a.rows,
                   a.inter);
      e = cudaGetLastError();
    }
  }
  return e;
}

size_t fused_scratch_bytes(const FusedArgs& a, int dtype, int mode) {
  if (a.rows <= kGemvMaxRows) return gemv_variant() == kGemvDynamic ? kGemvCounterBytes : 0;
  const size_t es = dtype == BF16 ? 2 : 4;
  const size_t xn = ((size_t)a.rows * a.K * es + 255) / 256 * 256;
  if (dtype == BF16 && gemm_tc_supported(a.K)) return xn;  // tensor-core path: epilogue fused
  size_t width = 0;
  if (mode == MODE_PLAIN && a.residual) width = (size_t)a.ncols;
  if (mode == MODE_ROPE) width = (size_t)(a.hq + 2 * a.hkv) * a.hd;
  else if (mode == MODE_SILU) width = 2 * (size_t)a.inter;
  return xn + (size_t)a.rows * width * 4;
}

cudaError_t fused_projection(const FusedArgs& a, int dtype, int mode, bool norm, void* scratch, cudaStream_t st) {
  if (a.p2p) {  // row-parallel projection with its all-reduce and residual add fused
    if (mode != MODE_PLAIN || norm || a.rows > kGemvMaxRows) return cudaErrorNotSupported;
    if (gemv_variant() == kGemvDynamic && scratch) {
      bool handled = false;
      const cudaError_t e = fused_projection_dynamic_allreduce(a, dtype, static_cast<int*>(scratch), st, &handled);
      if (handled) return e;
    }
    return fused_projection_allreduce(a, dtype, st);
  }
  if (a.attn_out) {  // attn_in with the decode attention fused (staged kernel)
    if (mode != MODE_ROPE || a.rows > kGemvMaxRows) return cudaErrorNotSupported;
    return fused_projection_attention(a, dtype, norm, st);
  }
  if (a.rows > kGemvMaxRows) {
    if (dtype == BF16) return fused_rows_t<__nv_bfloat16>(a, mode, norm, scratch, st);
    return fused_rows_t<float>(a, mode, norm, scratch, st);
  }
  bool handled = false;
  int variant = gemv_variant();
  cudaError_t te = cudaSuccess;
  if (variant == kGemvDynamic) {
    // `scratch` is the zeroed work counter, or nullptr (the call was prepared without
    // it): then the static staged kernel runs.
    te = fused_projection_dynamic(a, dtype, mode, norm, static_cast<int*>(scratch), st, &handled);
    if (!handled) variant = kGemvStaged;
  }
  if (!handled && variant == kGemvStaged) te = fused_projection_async(a, dtype, mode, norm, st, &handled);
  if (handled) return te;
#define PIM_DISPATCH(T)                                                                       \
  if (mode == MODE_PLAIN)                                                                     \
    return norm ? launch_fused_t<T, MODE_PLAIN, true>(a, st) : launch_fused_t<T, MODE_PLAIN, false>(a, st); \
  if (mode == MODE_ROPE)                                                                      \
    return norm ? launch_fused_t<T, MODE_ROPE, true>(a, st) : launch_fused_t<T, MODE_ROPE, false>(a, st);   \
  return norm ? launch_fused_t<T, MODE_SILU, true>(a, st) : launch_fused_t<T, MODE_SILU, false>(a, st);
  if (dtype == BF16) {
    PIM_DISPATCH(__nv_bfloat16)
  }
  PIM_DISPATCH(float)
#undef PIM_DISPATCH
}

}  // namespace pim
