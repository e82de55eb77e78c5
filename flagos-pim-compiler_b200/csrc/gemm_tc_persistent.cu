// Persistent variant of the tcgen05 row-batch GEMM (gemm_tc.cu): one CTA per SM walks
// the tile raster (tiles blockIdx.x, blockIdx.x + gridDim.x, ...) and the epilogue of a
// tile overlaps the MMAs of the next one.
//
// Same roles and tiles as gemm_tc.cu (128 x 256 tiles, 64-wide K blocks, 4-stage TMA
// ring, one MMA thread, four epilogue warps), plus:
//   * the producer's k-block counter runs across tile boundaries, so the ring never
//     drains between tiles;
//   * two 256-column TMEM accumulators (all 512 columns): tile i uses accumulator i & 1;
//     the MMA thread waits for acc_empty[i & 1] (the epilogue of tile i - 2 is done)
//     before the first MMA of tile i and commits acc_full[i & 1] after its last;
//   * the epilogue warps wait for acc_full[i & 1], read TMEM, write the outputs and arrive
//     on acc_empty[i & 1] (one arrival per warp).
// Phase k of acc_full[b] / acc_empty[b] belongs to the k-th tile using accumulator b, so
// the parity waited for is (i / 2) & 1 (and ((i / 2) - 1) & 1 for acc_empty); neither side
// can run more than one use ahead of the other.
//
// Every wait is bounded (kWaitLimitNs): a role whose wait expires raises *a.err and stops;
// the other roles' waits then expire in turn, the producer waits (bounded) for the copies
// it issued, the MMA thread waits (bounded) for its own last MMAs, and the TMEM is freed
// after the final barrier.
//
// Selected with PIM_GEMM=persistent; the one-tile-per-CTA kernel stays the default until
// this one has been measured.

#include "gemm_tc.cuh"

namespace pim {

template <int MODE>
__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_tc_persistent_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                              FusedArgs a, int M, int N, int K) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_u = smem_u32(smem_raw);
  unsigned char* smem = smem_raw + (((raw_u + 1023u) & ~1023u) - raw_u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kTcStages * kTcStageBytes);
  uint64_t* empty = full + kTcStages;
  uint64_t* acc_full = empty + kTcStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;      // [2]
  uint64_t* mma_done = acc_empty + 2;      // every MMA of this CTA has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* stop = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int tiles = ((M + kTcBM - 1) / kTcBM) * ((N + kTcBN - 1) / kTcBN);
  const int nkb = (K + kTcBK - 1) / kTcBK;
  int* err = a.err;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
    }
    mbar_init(mma_done, 1);
    *stop = 0;
    mbar_fence_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, 2 * kTcBN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    if (lane == 0) {
      tma_prefetch_map(&tma_a);
      tma_prefetch_map(&tma_b);
      int g = 0;  // k blocks issued by this CTA so far
      for (int tile = blockIdx.x; tile < tiles && !*stop; tile += gridDim.x) {
        int m0, n0;
        tc_tile_origin(tile, M, N, &m0, &n0);
        for (int kb = 0; kb < nkb; ++kb, ++g) {
          const int s = g % kTcStages;
          if (g >= kTcStages && !mbar_wait(&empty[s], ((g / kTcStages) - 1) & 1)) {
            if (err) atomicExch(err, 3);
            *stop = 1;
            break;
          }
          unsigned char* st = smem + s * kTcStageBytes;
          mbar_expect_tx(&full[s], kTcStageBytes);
          tma_load_2d(st, &tma_a, kb * kTcBK, m0, &full[s]);
          tma_load_2d(st + kTcABytes, &tma_b, kb * kTcBK, n0, &full[s]);
        }
      }
      // every copy issued has landed before the CTA exits (immediate on the normal path)
      for (int j = g - kTcStages < 0 ? 0 : g - kTcStages; j < g; ++j)
        if (!mbar_wait(&full[j % kTcStages], (j / kTcStages) & 1) && err) atomicExch(err, 3);
    }
  } else if (warp == 5) {
    if (lane == 0) {
      constexpr uint32_t idesc = mma_idesc_bf16(kTcBM, kTcBN);
      int g = 0, i = 0;
      for (int tile = blockIdx.x; tile < tiles && !*stop; tile += gridDim.x, ++i) {
        const int b = i & 1;
        if (i >= 2 && !mbar_wait(&acc_empty[b], ((i / 2) - 1) & 1)) {
          if (err) atomicExch(err, 4);
          *stop = 1;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(b * kTcBN);
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb, ++g) {
          const int s = g % kTcStages;
          if (!mbar_wait(&full[s], (g / kTcStages) & 1)) {
            if (err) atomicExch(err, 4);
            *stop = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * kTcStageBytes), sb = sa + kTcABytes;
#pragma unroll
          for (int k = 0; k < kTcBK / 16; ++k)
            mma_bf16(acc, sw128_desc(sa + k * 32), sw128_desc(sb + k * 32), idesc, (kb | k) != 0 ? 1u : 0u);
          mma_commit(&empty[s]);
        }
        mma_commit(&acc_full[b]);  // also after a failure: the epilogue then sees only issued MMAs
        if (!ok) break;
      }
      // No MMA may still be writing TMEM when it is freed (the epilogue may have stopped early).
      mma_commit(mma_done);
      if (!mbar_wait(mma_done, 0) && err) atomicExch(err, 4);
    }
  } else {
    // ---- epilogue warps 0-3 ----
    int i = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++i) {
      const int b = i & 1;
      // tcgen05.ld is warp-collective: every lane takes the same branch
      const bool ready = __all_sync(0xffffffffu, mbar_wait(&acc_full[b], (i / 2) & 1));
      if (!ready || __any_sync(0xffffffffu, *stop != 0)) {
        if (!ready && err && lane == 0) atomicExch(err, 5);
        break;
      }
      tc_fence_after();
      int m0, n0;
      tc_tile_origin(tile, M, N, &m0, &n0);
      const int m = m0 + warp * 32 + lane;
      const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(b * kTcBN);
      for (int cc = 0; cc < kTcBN / 32; ++cc) {
        const int n = n0 + cc * 32;
        if (n >= N) break;  // uniform across the warp
        float v[32];
        tmem_ld32(trow + cc * 32, v);
        if (m < M) tc_epilogue<MODE>(a, m, n, N, v);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);  // accumulator b free for tile i + 2
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * kTcBN);
  }
}

static int persistent_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <int MODE>
static cudaError_t launch_persistent(const CUtensorMap& ma, const CUtensorMap& mb, const FusedArgs& a, int M, int N,
                                     cudaStream_t st) {
  auto kern = gemm_tc_persistent_kernel<MODE>;
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
  const int grid = tiles < persistent_sms() ? tiles : persistent_sms();
  return launch_plain(kern, dim3(grid), dim3(kTcThreads), kTcSmem, st, ma, mb, a, M, N, a.K);
}

cudaError_t gemm_tc_persistent(const CUtensorMap& ma, const CUtensorMap& mb, const FusedArgs& a, int mode, int M,
                               int N, cudaStream_t st) {
  if (mode == MODE_PLAIN) return launch_persistent<MODE_PLAIN>(ma, mb, a, M, N, st);
  if (mode == MODE_ROPE) return launch_persistent<MODE_ROPE>(ma, mb, a, M, N, st);
  return launch_persistent<MODE_SILU>(ma, mb, a, M, N, st);
}

}  // namespace pim
