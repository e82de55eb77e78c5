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

#include <stdlib.h>

#include <atomic>
#include <mutex>

#include "gemm_tc.cuh"

namespace pim {

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
  int m0, n0;
  tc_tile_origin(blockIdx.x, M, N, &m0, &n0);
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

PFN_cuTensorMapEncodeTiled_v12000 encode_tiled() {
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

// Row-batch GEMM kernel: the persistent kernel of gemm_tc_persistent.cu (the default:
// 8 x 2048 LLaMA2-7B prefill 239 ms against 282 ms with one tile per CTA on a B200, same
// bits) or the one-tile-per-CTA kernel below, chosen by PIM_GEMM=tile at the first call
// and by set_gemm_kernel() at any time.  The tile kernel stays as the bit-exact reference
// the persistent kernel is tested against.
static std::atomic<int> g_gemm_kernel{-1};

int gemm_kernel() {
  int v = g_gemm_kernel.load(std::memory_order_relaxed);
  if (v < 0) {
    const char* e = getenv("PIM_GEMM");
    v = (e && e[0] == 't') ? kGemmTile : kGemmPersistent;
    int expected = -1;
    if (!g_gemm_kernel.compare_exchange_strong(expected, v)) v = expected;
  }
  return v;
}

void set_gemm_kernel(int v) { g_gemm_kernel.store(v, std::memory_order_relaxed); }

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
  if (gemm_kernel() == kGemmPersistent) return gemm_tc_persistent(ma, mb, a, mode, M, N, st);
  if (mode == MODE_PLAIN) return launch_tc<MODE_PLAIN>(ma, mb, a, M, N, st);
  if (mode == MODE_ROPE) return launch_tc<MODE_ROPE>(ma, mb, a, M, N, st);
  return launch_tc<MODE_SILU>(ma, mb, a, M, N, st);
}

}  // namespace pim
