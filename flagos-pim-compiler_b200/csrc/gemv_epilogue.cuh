// Epilogue of one output row of a fused decode projection, shared by the projection
// kernels so that all of them round identically.
//
// Task t, activation row r, with v1 / v2 the fp32 dot products of the task's weight
// rows (v2 unused for PLAIN):
//   PLAIN  y[r, t] = v1, or round(v1) + residual[r, t] when a residual is given
//   SILU   y[r, t] = round(silu(round(gate))) * round(up)      (gate = v1, up = v2)
//   ROPE   the column pair (j, j + hd/2) of head block t / (hd/2): RoPE at the row's
//          position for q and k blocks, then q -> y, k / v -> the KV blocks
// Rounding follows the HF bf16 model: every tensor HF materialises in bf16 is rounded
// at the same point (rnd<T>).
#pragma once

#include "pim_common.cuh"
#include "pim_kernels.h"

namespace pim {

template <typename T, int MODE>
__device__ __forceinline__ void row_epilogue(const FusedArgs& a, int t, int r, float v1, float v2) {
  if (MODE == MODE_PLAIN) {
    float y = v1;
    if (a.residual) y = rnd<T>(y) + to_f(static_cast<const T*>(a.residual)[(size_t)r * a.ncols + t]);
    static_cast<T*>(a.y)[(size_t)r * a.ncols + t] = from_f<T>(y);
  } else if (MODE == MODE_SILU) {
    const float g = rnd<T>(v1), u = rnd<T>(v2);
    const float act = rnd<T>(g / (1.f + expf(-g)));
    static_cast<T*>(a.y)[(size_t)r * a.inter + t] = from_f<T>(act * u);
  } else {
    const int half = a.hd / 2;
    const int hidx = t / half, j = t % half;
    const int b = r / a.seq, s = r % a.seq;
    const int p = a.positions[b] + s;
    if (p < 0 || p >= a.max_seq) return;  // positions are validated on the host
    const float x1 = rnd<T>(v1), x2 = rnd<T>(v2);
    float o1 = x1, o2 = x2;
    if (hidx < a.hq + a.hkv) {
      const float c = a.cos[(size_t)p * half + j], sn = a.sin[(size_t)p * half + j];
      o1 = rnd<T>(rnd<T>(x1 * c) + rnd<T>(-x2 * sn));
      o2 = rnd<T>(rnd<T>(x2 * c) + rnd<T>(x1 * sn));
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

// Number of tasks of a projection: weight rows (PLAIN) or row pairs (ROPE, SILU).
__host__ __device__ __forceinline__ int projection_tasks(const FusedArgs& a, int mode) {
  if (mode == MODE_PLAIN) return a.ncols;
  if (mode == MODE_ROPE) return (a.hq + 2 * a.hkv) * (a.hd / 2);
  return a.inter;
}

}  // namespace pim
