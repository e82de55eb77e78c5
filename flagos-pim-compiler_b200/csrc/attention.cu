// Attention over the per-rank KV blocks of memory/kv_layout: one contiguous
// [max_seq, head_dim] K block and V block per (layer, kv head, sequence).
//
// Split-K: the grid is (query rows) x (key splits).  Each CTA (8 warps) walks its
// key range with an online softmax; a group of LPK lanes owns one key (16 bytes of
// the K/V row per lane: one coalesced row per group) and each lane keeps UK keys'
// K and V loads in flight.  A CTA's partial (max, sum, acc[hd]) goes to the
// workspace; the last CTA of a row to finish (an atomic ticket per row) merges the
// splits and writes the output, then resets the ticket to zero for the next call.
// With one split the CTA writes the output directly.  The key range of a query is
// [0, pos + s] (causal); a split past the context stores an empty partial (max -inf,
// sum 0) that the merge skips, so the grid depends only on max_seq and stays valid
// inside a captured CUDA graph.
//
// Workspace layout: [partials: rows * splits * (hd + 2) floats][tickets: rows ints].
// The tickets must be zero before the first call (the caller zero-fills the
// workspace once and lets nothing else write it); every call leaves them zero.
//
// bf16 row batches (seq >= 16) with head_dim 128 take the tensor-core kernel of
// attention_prefill.cu instead (or, with PIM_ATTN=tc, the tcgen05 kernel of
// attention_tc.cu).

#include <math.h>

#include "pim_common.cuh"
#include "pim_kernels.h"

namespace pim {

constexpr int kAttnWarps = 8;
constexpr int kUK = 4;  // keys per lane group in flight (the same key order per group as one at a time)

template <typename T, int HD>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_kernel(AttnArgs a, int splits, int chunk,
                                                                 float* __restrict__ part, int* __restrict__ tickets) {
  constexpr int V = VecW<T>::n;  // elements per 16-byte vector
  constexpr int LPK = HD / V;    // lanes per key
  constexpr int KPW = 32 / LPK;  // key groups per warp
  constexpr int G = kAttnWarps * KPW;
  static_assert(LPK >= 1 && LPK <= 32 && 32 % LPK == 0, "head_dim not supported");
  const int row = blockIdx.x;  // ((b * seq) + s) * hq + h
  const int split = blockIdx.y;
  const int h = row % a.hq;
  const int bs = row / a.hq;
  const int b = bs / a.seq, s = bs % a.seq;
  const int kvh = h / (a.hq / a.hkv);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int sub = lane / LPK, sl = lane % LPK;
  const int grp = warp * KPW + sub;

  __shared__ float sm_m[G], sm_l[G];
  __shared__ float sm_acc[G][HD];
  __shared__ int sm_last;

  pdl_trigger();
  pdl_wait();
  const int qpos = a.positions[b] + s;
  const int ctx = min(qpos + 1, a.max_seq);
  const int k_lo = split * chunk;
  const int k_hi = min(ctx, k_lo + chunk);

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
    // Every lane of a warp runs the same number of iterations (the shuffles name the
    // full warp); lanes whose key is past the range compute on zeros and keep state.
    for (int wb = k_lo + warp * KPW; wb < k_hi; wb += G * kUK) {  // wb is uniform across the warp
      const int base = wb + sub;
      int4 kr[kUK], vr[kUK];
#pragma unroll
      for (int u = 0; u < kUK; ++u) {
        const int key = base + u * G;
        if (key < k_hi) {
          kr[u] = *reinterpret_cast<const int4*>(kb + (size_t)key * HD + sl * V);
          vr[u] = *reinterpret_cast<const int4*>(vb + (size_t)key * HD + sl * V);
        } else {
          kr[u] = vr[u] = make_int4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int u = 0; u < kUK; ++u) {
        const int key = base + u * G;
        float kf[V], vf[V];
        unpack(kr[u], kf, T());
        float d = 0.f;
#pragma unroll
        for (int e = 0; e < V; ++e) d = fmaf(qv[e], kf[e], d);
#pragma unroll
        for (int o = LPK / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        if (key < k_hi) {
          unpack(vr[u], vf, T());
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
  }
  if (sl == 0) {
    sm_m[grp] = m;
    sm_l[grp] = l;
  }
#pragma unroll
  for (int e = 0; e < V; ++e) sm_acc[grp][sl * V + e] = acc[e];
  __syncthreads();
  // merge the key groups of this CTA
  float* pp = part + ((size_t)row * splits + split) * (HD + 2);
  for (int d = threadIdx.x; d < HD; d += blockDim.x) {
    float M = -INFINITY;
    for (int i = 0; i < G; ++i) M = fmaxf(M, sm_m[i]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY)
      for (int i = 0; i < G; ++i) {
        const float w = sm_m[i] == -INFINITY ? 0.f : expf(sm_m[i] - M);
        L += sm_l[i] * w;
        A += sm_acc[i][d] * w;
      }
    if (splits == 1) {
      static_cast<T*>(a.out)[(size_t)row * HD + d] = from_f<T>(L > 0.f ? A / L : 0.f);
    } else {
      pp[2 + d] = A;
      if (d == 0) {
        pp[0] = M;
        pp[1] = L;
      }
    }
  }
  if (splits == 1) return;
  // the last CTA of this row merges every split
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) sm_last = (atomicAdd(&tickets[row], 1) == splits - 1);
  __syncthreads();
  if (!sm_last) return;
  __threadfence();
  const float* pr = part + (size_t)row * splits * (HD + 2);
  for (int d = threadIdx.x; d < HD; d += blockDim.x) {
    float M = -INFINITY;
    for (int i = 0; i < splits; ++i) M = fmaxf(M, __ldcg(pr + (size_t)i * (HD + 2)));
    float L = 0.f, A = 0.f;
    if (M != -INFINITY)
      for (int i = 0; i < splits; ++i) {
        const float mi = __ldcg(pr + (size_t)i * (HD + 2));
        if (mi == -INFINITY) continue;
        const float w = expf(mi - M);
        L += __ldcg(pr + (size_t)i * (HD + 2) + 1) * w;
        A += __ldcg(pr + (size_t)i * (HD + 2) + 2 + d) * w;
      }
    static_cast<T*>(a.out)[(size_t)row * HD + d] = from_f<T>(L > 0.f ? A / L : 0.f);
  }
  if (threadIdx.x == 0) tickets[row] = 0;
}

// Key splits: enough CTAs to cover the SMs twice, at least 64 keys per split.
static void attn_geometry(const AttnArgs& a, int* splits, int* chunk) {
  const int rows = a.batch * a.seq * a.hq;
  int s = (2 * 148 + rows - 1) / (rows > 0 ? rows : 1);
  const int max_s = (a.max_seq + 63) / 64;
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
  const size_t rows = (size_t)a.batch * a.seq * a.hq;
  const size_t part = (rows * splits * (a.hd + 2) * sizeof(float) + 255) / 256 * 256;
  return part + rows * sizeof(int);
}

template <typename T, int HD>
static cudaError_t attn_t(const AttnArgs& a, void* ws, cudaStream_t st) {
  int splits, chunk;
  attn_geometry(a, &splits, &chunk);
  const size_t rows = (size_t)a.batch * a.seq * a.hq;
  const size_t part_bytes = (rows * splits * (a.hd + 2) * sizeof(float) + 255) / 256 * 256;
  float* part = static_cast<float*>(ws);
  int* tickets = reinterpret_cast<int*>(static_cast<char*>(ws) + part_bytes);
  return launch_pdl(attn_kernel<T, HD>, dim3((unsigned)rows, splits), dim3(kAttnWarps * 32), 0, st, a, splits, chunk,
                    part, tickets);
}

bool attention_uses_workspace(const AttnArgs& a, int dtype) {
  return !attention_tc_supported(a, dtype) && !attention_prefill_supported(a, dtype);
}

cudaError_t attention(const AttnArgs& a, int dtype, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (attention_tc_supported(a, dtype)) return attention_tc(a, st);  // tcgen05 (opt-in); no workspace
  if (attention_prefill_supported(a, dtype)) return attention_prefill(a, st);  // tensor cores; no workspace
  if (ws_bytes < attention_workspace_bytes(a)) return cudaErrorInvalidValue;  // the split-K kernel's
  if (dtype == BF16) {
    if (a.hd == 128) return attn_t<__nv_bfloat16, 128>(a, ws, st);
    if (a.hd == 64) return attn_t<__nv_bfloat16, 64>(a, ws, st);
    if (a.hd == 32) return attn_t<__nv_bfloat16, 32>(a, ws, st);
  } else {
    if (a.hd == 128) return attn_t<float, 128>(a, ws, st);
    if (a.hd == 64) return attn_t<float, 64>(a, ws, st);
    if (a.hd == 32) return attn_t<float, 32>(a, ws, st);
  }
  return cudaErrorNotSupported;
}

}  // namespace pim
