// Tile geometry and the fused epilogue of the tcgen05 row-batch GEMMs (gemm_tc.cu,
// gemm_tc_persistent.cu).
#pragma once

#include <cudaTypedefs.h>

#include "gemv_epilogue.cuh"
#include "pim_common.cuh"
#include "pim_kernels.h"
#include "sm100.cuh"

namespace pim {

// cuTensorMapEncodeTiled from the driver (nullptr when the driver lacks it).
PFN_cuTensorMapEncodeTiled_v12000 encode_tiled();

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

// Tile `id` of the raster: groups of kTcGroupM row blocks; inside a group the row block
// varies fastest, so the CTAs resident at one time share A and B tiles in L2.
__device__ __forceinline__ void tc_tile_origin(int id, int M, int N, int* m0, int* n0) {
  const int n_mt = (M + kTcBM - 1) / kTcBM, n_nt = (N + kTcBN - 1) / kTcBN;
  const int group = id / (kTcGroupM * n_nt);
  const int first_mt = group * kTcGroupM;
  const int gsize = n_mt - first_mt < kTcGroupM ? n_mt - first_mt : kTcGroupM;
  const int in_group = id - group * kTcGroupM * n_nt;
  *m0 = (first_mt + in_group % gsize) * kTcBM;
  *n0 = (in_group / gsize) * kTcBN;
}

// The persistent variant (gemm_tc_persistent.cu): same tiles and epilogues.
cudaError_t gemm_tc_persistent(const CUtensorMap& ma, const CUtensorMap& mb, const FusedArgs& a, int mode, int M,
                               int N, cudaStream_t st);

}  // namespace pim
