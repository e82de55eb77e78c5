// Decode attention folded into the end of the q/k/v projection (attn_in, decode rows).
//
// The staged GEMV kernel writes q (after RoPE) to its output and k, v at the step's
// positions into the KV blocks.  With attention fused, each CTA, once its epilogue
// writes are out, adds to a per-query-head counter how many of the tasks it just
// finished feed that head (the head's q pairs and its kv head's k and v pairs: 3 * hd/2
// tasks in all; with grouped-query attention a kv head's k / v tasks count for every
// query head of its group).  The add that completes a head's count tells this CTA that
// every q, k and v value of the head is in memory: it computes the head's attention for
// every activation row and resets the counter for the next call.  No CTA ever waits for
// another; the last contributor does the work.
//
// The attention of one head and row: keys 0..p (p = positions[b] + s, the query's own
// position included), scores q . k / sqrt(hd) with an online softmax, as the split-K
// attention kernel computes with one split.  Groups of hd / 8 (bf16) or hd / 4 (fp32)
// lanes own one key (16 bytes of its row per lane); each group keeps kFaUK keys' K and
// V loads in flight; the groups' partial (max, sum, acc) meet in shared memory (the
// CTA's weight ring, idle by then) and are merged in group order.  Loads of q, K and V
// go through L2 (ld.global.cg): other CTAs of the same grid wrote them.
#pragma once

#include <math.h>

#include "pim_common.cuh"
#include "pim_kernels.h"

namespace pim {

constexpr int kFaUK = 4;  // keys per lane group in flight

// Number of tasks in [lo, hi) that feed query head h (q pairs of h, k and v pairs of its
// kv head) in the ROPE task order: q heads, then k heads, then v heads, hd/2 pairs each.
__device__ __forceinline__ int fa_tasks_for_head(const FusedArgs& a, int h, int lo, int hi) {
  const int half = a.hd / 2;
  const int kvh = h / (a.hq / a.hkv);
  auto overlap = [&](int b0) { return max(0, min(hi, b0 + half) - max(lo, b0)); };
  return overlap(h * half) + overlap((a.hq + kvh) * half) + overlap((a.hq + a.hkv + kvh) * half);
}

// Attention of query head h for activation row r into a.attn_out; all threads of the CTA
// call it; `scratch` holds at least (kWarp / (HD / VecW<T>::n) * 8) * (HD + 2) floats.
template <typename T, int HD>
__device__ void fa_head_row(const FusedArgs& a, int h, int r, float* scratch) {
  constexpr int V = VecW<T>::n;  // elements per 16-byte vector
  constexpr int LPK = HD / V;    // lanes per key
  constexpr int KPW = kWarp / LPK;
  const int nwarps = blockDim.x / kWarp;
  const int G = nwarps * KPW;
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int sub = lane / LPK, sl = lane % LPK;
  const int grp = warp * KPW + sub;
  float* sm_m = scratch;
  float* sm_l = scratch + G;
  float* sm_acc = scratch + 2 * G;  // [G][HD]

  const int b = r / a.seq, s = r % a.seq;
  const int qpos = a.positions[b] + s;
  const int ctx = min(qpos + 1, a.max_seq);
  const int kvh = h / (a.hq / a.hkv);
  const float scale = rsqrtf((float)HD);
  float qv[V];
  const T* qrow = static_cast<const T*>(a.y) + ((size_t)r * a.hq + h) * HD;
  unpack(__ldcg(reinterpret_cast<const int4*>(qrow + sl * V)), qv, T());
#pragma unroll
  for (int e = 0; e < V; ++e) qv[e] *= scale;
  const T* kb = static_cast<const T*>(a.kv_base) + (2 * kvh) * a.block_stride + b * a.seq_stride;
  const T* vb = kb + a.block_stride;

  float m = -INFINITY, l = 0.f, acc[V];
#pragma unroll
  for (int e = 0; e < V; ++e) acc[e] = 0.f;
  // every lane of a warp runs the same number of iterations (the shuffles name the full warp)
  for (int wb = warp * KPW; wb < ctx; wb += G * kFaUK) {
    const int base = wb + sub;
    int4 kr[kFaUK], vr[kFaUK];
#pragma unroll
    for (int u = 0; u < kFaUK; ++u) {
      const int key = base + u * G;
      if (key < ctx) {
        kr[u] = __ldcg(reinterpret_cast<const int4*>(kb + (size_t)key * HD + sl * V));
        vr[u] = __ldcg(reinterpret_cast<const int4*>(vb + (size_t)key * HD + sl * V));
      } else {
        kr[u] = vr[u] = make_int4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int u = 0; u < kFaUK; ++u) {
      const int key = base + u * G;
      float kf[V], vf[V];
      unpack(kr[u], kf, T());
      float d = 0.f;
#pragma unroll
      for (int e = 0; e < V; ++e) d = fmaf(qv[e], kf[e], d);
#pragma unroll
      for (int o = LPK / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
      if (key < ctx) {
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
  if (sl == 0) {
    sm_m[grp] = m;
    sm_l[grp] = l;
  }
#pragma unroll
  for (int e = 0; e < V; ++e) sm_acc[grp * HD + sl * V + e] = acc[e];
  __syncthreads();
  T* out = static_cast<T*>(a.attn_out) + ((size_t)r * a.hq + h) * HD;
  for (int d = threadIdx.x; d < HD; d += blockDim.x) {
    float M = -INFINITY;
    for (int i = 0; i < G; ++i) M = fmaxf(M, sm_m[i]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY)
      for (int i = 0; i < G; ++i) {
        const float w = sm_m[i] == -INFINITY ? 0.f : expf(sm_m[i] - M);
        L += sm_l[i] * w;
        A += sm_acc[i * HD + d] * w;
      }
    out[d] = from_f<T>(L > 0.f ? A / L : 0.f);
  }
  __syncthreads();  // the scratch is reused by the next head or row
}

// The tail of an attn_in launch with attention fused: count this CTA's finished tasks
// [t_lo, t_hi) per query head and compute every head this CTA completed.  All threads of
// the CTA call it after the projection epilogue; `scratch` is shared memory the CTA no
// longer needs (see fa_head_row for its size).
template <typename T>
__device__ void fa_tail(const FusedArgs& a, int t_lo, int t_hi, float* scratch) {
  __shared__ int s_n;
  __shared__ short s_heads[64];
  __threadfence();  // this thread's epilogue writes are visible device-wide ...
  __syncthreads();  // ... for every thread of the CTA, before the counts that announce them
  if (threadIdx.x == 0) {
    int n = 0;
    const int full = 3 * (a.hd / 2);
    for (int h = 0; h < a.hq; ++h) {
      const int c = fa_tasks_for_head(a, h, t_lo, t_hi);
      if (c > 0 && atomicAdd(&a.attn_cnt[h], c) + c == full) {
        a.attn_cnt[h] = 0;  // every contribution is in: ready for the next call
        if (n < 64) s_heads[n] = (short)h;
        ++n;
      }
    }
    s_n = n < 64 ? n : 64;
  }
  __syncthreads();
  __threadfence();  // the other CTAs' q, k and v, seen through their counts, before the reads
  for (int i = 0; i < s_n; ++i)
    for (int r = 0; r < a.rows; ++r) {
      if (a.hd == 128)
        fa_head_row<T, 128>(a, s_heads[i], r, scratch);
      else
        fa_head_row<T, 64>(a, s_heads[i], r, scratch);
    }
}

}  // namespace pim
