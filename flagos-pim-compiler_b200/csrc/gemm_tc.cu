// Row-batched projections (prefill, rows > 8) in bf16 on the 5th-generation tensor
// cores, with the node's epilogue fused.
//
// C[M, N] = A[M, K] . B[N, K]^T: A the (normalised) activation rows, B the weight rows,
// both bf16 and K-major; fp32 accumulation in TMEM.  One CTA computes one 128 x 256
// output tile with 192 threads:
//   warp 4 (one thread)  producer: TMA loads of 64-wide K blocks of A (128 x 64) and B
//                        (256 x 64), 128-byte swizzle, into a 4-stage ring of 48 KB;
//   warp 5 (one thread)  MMA issuer: four tcgen05.mma (K = 16 each) per stage into a
//                        128 x 256 fp32 accumulator (256 TMEM columns); tcgen05.commit
//                        frees each stage and finally marks the accumulator complete;
//   warps 0-3            epilogue: warp w reads TMEM lanes 32w..32w+31 (the tile's rows)
//                        32 columns at a time and writes the node's outputs, 32 or 64
//                        contiguous bytes per thread and store.
// Tiles are issued in groups of 16 row blocks that sweep the column blocks, so the CTAs
// resident at one time share A and B tiles in L2.
//
// Epilogues (pair-interleaved weights put the pair (2t, 2t + 1) in one thread):
//   PLAIN  y = acc, or round(acc) + residual
//   SILU   y[t] = round(silu(round(acc[2t]))) * round(acc[2t + 1])
//   ROPE   RoPE on the column pair at the row's position, q -> y, k / v -> KV blocks
// with the rounding of the GEMV kernels (gemv_epilogue.cuh).
//
// Warp 0 allocates and frees the TMEM.  Every mbarrier wait is bounded: on expiry the
// kernel raises *a.err, the role that waited stops, the producer still waits (bounded)
// for the copies it issued, and every thread reaches the final barrier, after which
// the TMEM is freed.

#include <cudaTypedefs.h>

#include <mutex>

#include "gemv_epilogue.cuh"
#include "pim_common.cuh"
#include "pim_kernels.h"
#include "sm100.cuh"

namespace pim {

constexpr int kTcBM = 128, kTcBN = 256, kTcBK = 64, kTcStages = 4;
constexpr int kTcThreads = 192;
constexpr int kTcABytes = kTcBM * kTcBK * 2;  // 16 KB
constexpr int kTcBBytes = kTcBN * kTcBK * 2;  // 32 KB
constexpr int kTcStageBytes = kTcABytes + kTcBBytes;
constexpr int kTcGroupM = 16;  // row blocks per raster group
constexpr size_t kTcSmem = 1024 + (size_t)kTcStages * kTcStageBytes + 256;

// Stores n consecutive outputs (16-byte vectors when the address allows it).
__device__ __forceinline__ void store_run(__nv_bfloat16* dst, const float* v, int n) {
  if (n % 8 == 0 && ((uintptr_t)dst & 15) == 0) {
    for (int i = 0; i < n; i += 8) {
      float f[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = v[i + e];
      *reinterpret_cast<int4*>(dst + i) = pack(f, __nv_bfloat16());
    }
  } else {
    for (int i = 0; i < n; ++i) dst[i] = __float2bfloat16_rn(v[i]);
  }
}

// Epilogue of 32 accumulator columns [n, n + 32) of row m.
template <int MODE>
__device__ __forceinline__ void tc_epilogue(const FusedArgs& a, int m, int n, int N, const float (&v)[32]) {
  using T = __nv_bfloat16;
  if (MODE == MODE_PLAIN) {
    const int cnt = N - n < 32 ? N - n : 32;
    float o[32];
    const T* res = static_cast<const T*>(a.residual);
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] = v[i];
    if (res)
      for (int i = 0; i < cnt; ++i) o[i] = rnd<T>(v[i]) + to_f(res[(size_t)m * N + n + i]);
    store_run(static_cast<T*>(a.y) + (size_t)m * N + n, o, cnt);
  } else if (MODE == MODE_SILU) {
    const int t0 = n / 2;
    const int cnt = a.inter - t0 < 16 ? a.inter - t0 : 16;
    float o[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float g = rnd<T>(v[2 * i]), u = rnd<T>(v[2 * i + 1]);
      o[i] = rnd<T>(g / (1.f + expf(-g))) * u;
    }
    store_run(static_cast<T*>(a.y) + (size_t)m * a.inter + t0, o, cnt);
  } else {
    const int half = a.hd / 2;
    const int t0 = n / 2;
    if (half % 16 != 0) {  // pairs of this run may span two heads: one pair at a time
      const int ntasks = projection_tasks(a, MODE_ROPE);
      for (int i = 0; i < 16 && t0 + i < ntasks; ++i) row_epilogue<T, MODE_ROPE>(a, t0 + i, m, v[2 * i], v[2 * i + 1]);
      return;
    }
    const int hidx = t0 / half, j0 = t0 % half;
    if (hidx >= a.hq + 2 * a.hkv) return;
    const int b = m / a.seq, s = m % a.seq;
    const int p = a.positions[b] + s;
    if (p < 0 || p >= a.max_seq) return;  // positions are validated on the host
    float o1[16], o2[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float x1 = rnd<T>(v[2 * i]), x2 = rnd<T>(v[2 * i + 1]);
      o1[i] = x1;
      o2[i] = x2;
    }
    if (hidx < a.hq + a.hkv) {
      const float* cs = a.cos + (size_t)p * half + j0;
      const float* sn = a.sin + (size_t)p * half + j0;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float x1 = o1[i], x2 = o2[i], c = cs[i], sv = sn[i];
        o1[i] = rnd<T>(rnd<T>(x1 * c) + rnd<T>(-x2 * sv));
        o2[i] = rnd<T>(rnd<T>(x2 * c) + rnd<T>(x1 * sv));
      }
    }
    T* dst;
    if (hidx < a.hq) {
      dst = static_cast<T*>(a.y) + (size_t)m * a.hq * a.hd + (size_t)hidx * a.hd;
    } else {
      const int kvh = hidx < a.hq + a.hkv ? hidx - a.hq : hidx - a.hq - a.hkv;
      const int which = hidx < a.hq + a.hkv ? 0 : 1;
      dst = static_cast<T*>(a.kv_base) + (2 * kvh + which) * a.block_stride + b * a.seq_stride + (size_t)p * a.hd;
    }
    store_run(dst + j0, o1, 16);
    store_run(dst + j0 + half, o2, 16);
  }
}

template <int MODE>
__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                   FusedArgs a, int M, int N, int K) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_u = smem_u32(smem_raw);
  unsigned char* smem = smem_raw + (((raw_u + 1023u) & ~1023u) - raw_u);  // swizzled tiles: 1024-aligned
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kTcStages * kTcStageBytes);
  uint64_t* empty = full + kTcStages;
  uint64_t* acc_bar = empty + kTcStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_bar + 1);
  int* failed = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  // Raster: groups of kTcGroupM row blocks; inside a group the row block varies fastest.
  const int n_mt = (M + kTcBM - 1) / kTcBM, n_nt = (N + kTcBN - 1) / kTcBN;
  const int id = blockIdx.x;
  const int group = id / (kTcGroupM * n_nt);
  const int first_mt = group * kTcGroupM;
  const int gsize = n_mt - first_mt < kTcGroupM ? n_mt - first_mt : kTcGroupM;
  const int in_group = id - group * kTcGroupM * n_nt;
  const int m0 = (first_mt + in_group % gsize) * kTcBM;
  const int n0 = (in_group / gsize) * kTcBN;
  const int nkb = (K + kTcBK - 1) / kTcBK;
  int* err = a.err;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_bar, 1);
    *failed = 0;
    mbar_fence_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, kTcBN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    if (lane == 0) {
      tma_prefetch_map(&tma_a);
      tma_prefetch_map(&tma_b);
      int issued = 0;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % kTcStages;
        if (kb >= kTcStages && !mbar_wait(&empty[s], ((kb / kTcStages) - 1) & 1)) {
          if (err) atomicExch(err, 3);
          break;
        }
        unsigned char* st = smem + s * kTcStageBytes;
        mbar_expect_tx(&full[s], kTcStageBytes);
        tma_load_2d(st, &tma_a, kb * kTcBK, m0, &full[s]);
        tma_load_2d(st + kTcABytes, &tma_b, kb * kTcBK, n0, &full[s]);
        issued = kb + 1;
      }
      // Every copy issued has landed before the CTA can exit (immediate on the normal path).
      for (int kb = issued - kTcStages < 0 ? 0 : issued - kTcStages; kb < issued; ++kb)
        if (!mbar_wait(&full[kb % kTcStages], (kb / kTcStages) & 1) && err) atomicExch(err, 3);
    }
  } else if (warp == 5) {
    if (lane == 0) {
      constexpr uint32_t idesc = mma_idesc_bf16(kTcBM, kTcBN);
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % kTcStages;
        if (!mbar_wait(&full[s], (kb / kTcStages) & 1)) {
          if (err) atomicExch(err, 4);
          *failed = 1;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + s * kTcStageBytes), sb = sa + kTcABytes;
#pragma unroll
        for (int k = 0; k < kTcBK / 16; ++k)
          mma_bf16(tmem, sw128_desc(sa + k * 32), sw128_desc(sb + k * 32), idesc, (kb | k) != 0 ? 1u : 0u);
        mma_commit(&empty[s]);
      }
      mma_commit(acc_bar);  // also on failure: the epilogue then waits for issued MMAs only
    }
  } else {
    // ---- epilogue warps 0-3 ----
    // tcgen05.ld is warp-collective: every lane takes the same branch.
    const bool done = __all_sync(0xffffffffu, mbar_wait(acc_bar, 0));
    if (!done && err && lane == 0) atomicExch(err, 5);
    tc_fence_after();
    if (__all_sync(0xffffffffu, done && !*reinterpret_cast<volatile int*>(failed))) {
      const int m = m0 + warp * 32 + lane;
      const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
      for (int cc = 0; cc < kTcBN / 32; ++cc) {
        const int n = n0 + cc * 32;
        if (n >= N) break;  // uniform across the warp
        float v[32];
        tmem_ld32(trow + cc * 32, v);
        if (m < M) tc_epilogue<MODE>(a, m, n, N, v);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTcBN);
  }
}

// ---- host side ------------------------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 encode_tiled() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Tensor map of a row-major bf16 [rows, k] matrix read in boxes of box_rows x 64.
static bool bf16_rows_map(CUtensorMap* map, const void* ptr, int rows, int k, int box_rows) {
  auto fn = encode_tiled();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)k * 2};
  cuuint32_t box[2] = {(cuuint32_t)kTcBK, (cuuint32_t)box_rows};
  cuuint32_t elem[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, elem,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool gemm_tc_supported(int K) { return K > 0 && K % 8 == 0; }

template <int MODE>
static cudaError_t launch_tc(const CUtensorMap& ma, const CUtensorMap& mb, const FusedArgs& a, int M, int N,
                             cudaStream_t st) {
  auto kern = gemm_tc_kernel<MODE>;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const int tiles = ((M + kTcBM - 1) / kTcBM) * ((N + kTcBN - 1) / kTcBN);
  return launch_plain(kern, dim3(tiles), dim3(kTcThreads), kTcSmem, st, ma, mb, a, M, N, a.K);
}

// C = xin . W^T with the node's epilogue, for bf16 rows > kGemvMaxRows.  `xin` is the
// activation (or its rmsnorm) as [rows, K] bf16.
cudaError_t gemm_tc(const FusedArgs& a, int mode, const void* xin, cudaStream_t st) {
  if (!gemm_tc_supported(a.K) || ((uintptr_t)xin & 15) || ((uintptr_t)a.w & 15)) return cudaErrorInvalidValue;
  const int M = a.rows;
  const int N = mode == MODE_PLAIN ? a.ncols : 2 * projection_tasks(a, mode);
  CUtensorMap ma, mb;
  if (!bf16_rows_map(&ma, xin, M, a.K, kTcBM) || !bf16_rows_map(&mb, a.w, N, a.K, kTcBN))
    return cudaErrorInvalidValue;
  if (mode == MODE_PLAIN) return launch_tc<MODE_PLAIN>(ma, mb, a, M, N, st);
  if (mode == MODE_ROPE) return launch_tc<MODE_ROPE>(ma, mb, a, M, N, st);
  return launch_tc<MODE_SILU>(ma, mb, a, M, N, st);
}

}  // namespace pim
