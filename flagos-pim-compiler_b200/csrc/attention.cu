// Attention over the per-rank KV blocks of memory/kv_layout: one contiguous
// [max_seq, head_dim] K block and V block per (layer, kv head, sequence).
//
// Split-K ("flash-decoding"): the grid is (query rows) x (key splits); each CTA
// walks its key range with an online softmax, a group of LPK lanes owning one key
// (16 bytes of the K/V row per lane, one coalesced 256-byte row per group), and
// writes a partial (max, sum, acc[hd]) that a second kernel merges.  The key range
// of a query is [0, pos + s] (causal); splits past the context exit early, so the
// grid depends only on max_seq and stays valid inside a captured CUDA graph.

#include <math.h>

#include "pim_common.cuh"
#include "pim_kernels.h"

namespace pim {

constexpr int kAttnWarps = 4;

template <typename T, int HD>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_split_kernel(AttnArgs a, int splits, int chunk,
                                                                      float* __restrict__ part) {
  constexpr int V = VecW<T>::n;          // elements per 16-byte vector
  constexpr int LPK = HD / V;            // lanes per key
  constexpr int KPW = 32 / LPK;          // keys per warp per step
  static_assert(LPK >= 1 && LPK <= 32 && 32 % LPK == 0, "head_dim not supported");
  const int row = blockIdx.x;            // ((b * seq) + s) * hq + h
  const int split = blockIdx.y;
  const int h = row % a.hq;
  const int bs = row / a.hq;
  const int b = bs / a.seq, s = bs % a.seq;
  const int group = a.hq / a.hkv;
  const int kvh = h / group;
  const int qpos = a.positions[b] + s;
  const int ctx = min(qpos + 1, a.max_seq);
  const int k_lo = split * chunk;
  const int k_hi = min(ctx, k_lo + chunk);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int sub = lane / LPK, sl = lane % LPK;

  __shared__ float sm_m[kAttnWarps * KPW], sm_l[kAttnWarps * KPW];
  __shared__ float sm_acc[kAttnWarps * KPW][HD];

  float m = -INFINITY, l = 0.f, acc[V];
#pragma unroll
  for (int e = 0; e < V; ++e) acc[e] = 0.f;

  if (k_lo < k_hi) {
    float qv[V];
    const T* qrow = static_cast<const T*>(a.q) + ((size_t)bs * a.hq + h) * HD;
    unpack(*reinterpret_cast<const int4*>(qrow + sl * V), qv, T());
#pragma unroll
    for (int e = 0; e < V; ++e) qv[e] *= a.scale;
    const T* kb = static_cast<const T*>(a.kv_base) + (2 * kvh) * a.block_stride + b * a.seq_stride;
    const T* vb = kb + a.block_stride;
    // Every lane of a warp runs the same number of iterations (the shuffle below
    // names the full warp); lanes whose key is past the range compute on zeros and
    // leave their state unchanged.
    for (int base = k_lo + warp * KPW; base < k_hi; base += kAttnWarps * KPW) {
      const int key = base + sub;
      const bool valid = key < k_hi;
      float kf[V], vf[V];
      if (valid) {
        unpack(*reinterpret_cast<const int4*>(kb + (size_t)key * HD + sl * V), kf, T());
        unpack(*reinterpret_cast<const int4*>(vb + (size_t)key * HD + sl * V), vf, T());
      } else {
#pragma unroll
        for (int e = 0; e < V; ++e) kf[e] = vf[e] = 0.f;
      }
      float d = 0.f;
#pragma unroll
      for (int e = 0; e < V; ++e) d = fmaf(qv[e], kf[e], d);
#pragma unroll
      for (int o = LPK / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
      if (valid) {
        const float mn = fmaxf(m, d);
        const float alpha = expf(m - mn);
        const float p = expf(d - mn);
#pragma unroll
        for (int e = 0; e < V; ++e) acc[e] = fmaf(p, vf[e], acc[e] * alpha);
        l = l * alpha + p;
        m = mn;
      }
    }
  }
  const int slot = warp * KPW + sub;
  if (sl == 0) {
    sm_m[slot] = m;
    sm_l[slot] = l;
  }
#pragma unroll
  for (int e = 0; e < V; ++e) sm_acc[slot][sl * V + e] = acc[e];
  __syncthreads();
  // merge the kAttnWarps*KPW key groups of this CTA
  for (int d = threadIdx.x; d < HD; d += blockDim.x) {
    float M = -INFINITY;
    for (int i = 0; i < kAttnWarps * KPW; ++i) M = fmaxf(M, sm_m[i]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY)
      for (int i = 0; i < kAttnWarps * KPW; ++i) {
        const float w = sm_m[i] == -INFINITY ? 0.f : expf(sm_m[i] - M);
        L += sm_l[i] * w;
        A += sm_acc[i][d] * w;
      }
    float* pp = part + ((size_t)row * splits + split) * (HD + 2);
    pp[2 + d] = A;
    if (d == 0) {
      pp[0] = M;
      pp[1] = L;
    }
  }
}

template <typename T, int HD>
__global__ void attn_merge_kernel(AttnArgs a, int splits, const float* __restrict__ part, int rows) {
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;
  const float* pr = part + (size_t)row * splits * (HD + 2);
  float M = -INFINITY;
  for (int i = 0; i < splits; ++i) M = fmaxf(M, pr[(size_t)i * (HD + 2)]);
  float L = 0.f;
  for (int i = 0; i < splits; ++i) {
    const float mi = pr[(size_t)i * (HD + 2)];
    if (mi != -INFINITY) L += pr[(size_t)i * (HD + 2) + 1] * expf(mi - M);
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  T* out = static_cast<T*>(a.out) + (size_t)row * HD;
  for (int d = lane; d < HD; d += 32) {
    float A = 0.f;
    for (int i = 0; i < splits; ++i) {
      const float mi = pr[(size_t)i * (HD + 2)];
      if (mi != -INFINITY) A += pr[(size_t)i * (HD + 2) + 2 + d] * expf(mi - M);
    }
    out[d] = from_f<T>(A * inv);
  }
}

static void attn_geometry(const AttnArgs& a, int* splits, int* chunk) {
  const int rows = a.batch * a.seq * a.hq;
  int target = 4 * 148;
  int s = target / (rows > 0 ? rows : 1);
  const int max_s = (a.max_seq + 31) / 32;
  if (s < 1) s = 1;
  if (s > max_s) s = max_s;
  int c = (a.max_seq + s - 1) / s;
  c = (c + 31) / 32 * 32;
  *splits = (a.max_seq + c - 1) / c;
  *chunk = c;
}

size_t attention_workspace_bytes(const AttnArgs& a) {
  int splits, chunk;
  attn_geometry(a, &splits, &chunk);
  return (size_t)a.batch * a.seq * a.hq * splits * (a.hd + 2) * sizeof(float);
}

template <typename T, int HD>
static cudaError_t attn_t(const AttnArgs& a, void* ws, cudaStream_t st) {
  int splits, chunk;
  attn_geometry(a, &splits, &chunk);
  const int rows = a.batch * a.seq * a.hq;
  float* part = static_cast<float*>(ws);
  attn_split_kernel<T, HD><<<dim3(rows, splits), kAttnWarps * 32, 0, st>>>(a, splits, chunk, part);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  attn_merge_kernel<T, HD><<<(rows + 7) / 8, 256, 0, st>>>(a, splits, part, rows);
  return cudaGetLastError();
}

cudaError_t attention(const AttnArgs& a, int dtype, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (ws_bytes < attention_workspace_bytes(a)) return cudaErrorInvalidValue;
  if (dtype == BF16) {
    if (a.hd == 128) return attn_t<__nv_bfloat16, 128>(a, ws, st);
    if (a.hd == 64) return attn_t<__nv_bfloat16, 64>(a, ws, st);
  } else {
    if (a.hd == 128) return attn_t<float, 128>(a, ws, st);
    if (a.hd == 64) return attn_t<float, 64>(a, ws, st);
  }
  return cudaErrorNotSupported;
}

}  // namespace pim
