// Causal attention for row batches (prefill) on the 5th-generation tensor cores: bf16,
// head_dim 128, S = Q K^T and O = P V as tcgen05.mma with fp32 accumulators in TMEM.
// Opt-in (PIM_ATTN=tc); attention_prefill.cu (warp-level mma.sync) is the default.
//
// One CTA = 128 query rows of one (sequence, head); 192 threads:
//   warp 4 (one thread)  producer: TMA loads of the Q tile (once) and of 128-key K and V
//                        tiles into a 2-stage ring (128-byte swizzle, 64-column halves);
//   warp 5 (one thread)  MMA issuer: S(j) = Q K(j)^T into one of two 128-column TMEM
//                        buffers, then O += P(j) V(j) into a third (the output
//                        accumulator, fp32 in TMEM across all key tiles); V is the
//                        MN-major B operand (its rows are keys, the MMA's K dimension);
//   warps 0-3            softmax: thread r owns query row r (TMEM lane r).  Per key tile:
//                        row max of the masked, scaled scores (pass 1); once the previous
//                        P V is done, O *= exp2(old max - new max) in TMEM (skipped by a
//                        warp whose 32 rows kept their max); then P = exp2(S - max) as bf16
//                        into shared memory in the 128-byte-swizzled K-major layout of an
//                        A operand (pass 2) and the running sum; at the end O / sum.
// Barriers (mbarrier, one producer each): Q loaded; per stage K/V loaded and freed (MMA
// commit after the stage's P V); per S buffer full (commit) and free (4 softmax warps);
// P written (4 warps); P V done (commit) and O rescaled (4 warps).  S(j + 1) is computed
// while the softmax warps work on tile j, and P(j) V(j) while they take the next max.
//
// The query at position p sees keys 0..p (positions[b] + row); keys past each row's
// position or past the tile's key range get probability 0.  Rows past `seq` (the last
// tile's padding) compute with a clamped position and are not stored.
//
// Every mbarrier wait is bounded: on expiry the role raises the library's device error
// word (attention_tc_errors), stops, and every thread still reaches the final barrier,
// after which the TMEM is freed; the output of that CTA is then undefined.

#include <cudaTypedefs.h>
#include <math.h>
#include <stdlib.h>

#include <atomic>

#include "gemm_tc.cuh"
#include "pim_kernels.h"
#include "sm100.cuh"

namespace pim {

constexpr int kAtRows = 128;                      // query rows per CTA (MMA M)
constexpr int kAtKeys = 128;                      // keys per tile (MMA N of S, K of P V)
constexpr int kAtHd = 128;                        // head_dim
constexpr int kAtThreads = 192;
constexpr uint32_t kAtHalf = 128 * 64 * 2;        // 16 KB: 128 rows x one 64-element half
constexpr uint32_t kAtTile = 2 * kAtHalf;         // 32 KB
constexpr uint32_t kAtQ = 0, kAtP = kAtTile, kAtKV = 2 * kAtTile;  // K(s) = KV + 2s tiles, V(s) = K(s) + tile
constexpr uint32_t kAtBar = kAtKV + 4 * kAtTile;  // 192 KB
constexpr size_t kAtSmem = 1024 + kAtBar + 256;

__device__ int g_attn_tc_err;

__device__ __forceinline__ void at_fail() { atomicExch(&g_attn_tc_err, 1); }

__global__ void __launch_bounds__(kAtThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tkv, AttnArgs a) {
  extern __shared__ unsigned char at_raw[];
  const uint32_t raw_u = smem_u32(at_raw);
  unsigned char* sm = at_raw + (((raw_u + 1023u) & ~1023u) - raw_u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kAtBar);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* s_free = bars + 7;    // [2]
  uint64_t* p_full = bars + 9;
  uint64_t* o_full = bars + 10;
  uint64_t* o_free = bars + 11;
  uint64_t* mma_done = bars + 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  volatile int* stop = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int nqb = (a.seq + kAtRows - 1) / kAtRows;
  const int qb = nqb - 1 - (int)blockIdx.x;  // heavy tiles first
  const int h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (a.hq / a.hkv);
  const int q0 = qb * kAtRows;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(o_full, 1);
    mbar_init(o_free, 4);
    mbar_init(mma_done, 1);
    *stop = 0;
    mbar_fence_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, 512);  // S0 [0,128) S1 [128,256) O_j [256,384)
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  pdl_trigger();
  pdl_wait();
  const int pos0 = a.positions[b];
  const int last_row = min(q0 + kAtRows, a.seq) - 1;
  const int kv_len = min(pos0 + last_row + 1, a.max_seq);
  const int n = (kv_len + kAtKeys - 1) / kAtKeys;

  if (warp == 4) {
    // ---------------- producer ----------------
    if (lane == 0) {
      tma_prefetch_map(&tq);
      tma_prefetch_map(&tkv);
      mbar_expect_tx(q_full, kAtTile);
      for (int hh = 0; hh < 2; ++hh)
        tma_load_2d(sm + kAtQ + hh * kAtHalf, &tq, h * kAtHd + hh * 64, b * a.seq + q0, q_full);
      int issued = 0;
      for (int j = 0; j < n && !*stop; ++j) {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&kv_empty[s], ((j >> 1) - 1) & 1)) {
          at_fail();
          *stop = 1;
          break;
        }
        unsigned char* kt = sm + kAtKV + s * 2 * kAtTile;
        mbar_expect_tx(&kv_full[s], 2 * kAtTile);
        for (int hh = 0; hh < 2; ++hh) {
          tma_load_4d(kt + hh * kAtHalf, &tkv, hh * 64, j * kAtKeys, 2 * kvh, b, &kv_full[s]);
          tma_load_4d(kt + kAtTile + hh * kAtHalf, &tkv, hh * 64, j * kAtKeys, 2 * kvh + 1, b, &kv_full[s]);
        }
        issued = j + 1;
      }
      // every copy issued has landed before the CTA exits (immediate on the normal path)
      if (!mbar_wait(q_full, 0)) at_fail();
      for (int j = issued - 2 < 0 ? 0 : issued - 2; j < issued; ++j)
        if (!mbar_wait(&kv_full[j & 1], (j >> 1) & 1)) at_fail();
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t id_s = mma_idesc_bf16(kAtRows, kAtKeys);
      constexpr uint32_t id_pv = mma_idesc_bf16_bmn(kAtRows, kAtHd);
      const uint32_t sq = smem_u32(sm + kAtQ), sp = smem_u32(sm + kAtP);
      bool ok = mbar_wait(q_full, 0);
      for (int j = 0; ok && j <= n && !*stop; ++j) {
        if (j < n) {  // S(j) = Q K(j)^T
          const int s = j & 1;
          ok = mbar_wait(&kv_full[s], (j >> 1) & 1) && (j < 2 || mbar_wait(&s_free[s], ((j >> 1) - 1) & 1));
          if (!ok) break;
          tc_fence_after();
          const uint32_t sk = smem_u32(sm + kAtKV + s * 2 * kAtTile);
#pragma unroll
          for (int kk = 0; kk < kAtHd / 16; ++kk) {
            const uint32_t off = (kk / 4) * kAtHalf + (kk % 4) * 32;
            mma_bf16(tmem + s * kAtKeys, sw128_desc(sq + off), sw128_desc(sk + off), id_s, kk > 0 ? 1u : 0u);
          }
          mma_commit(&s_full[s]);
        }
        if (j >= 1) {  // O_i = P(i) V(i), i = j - 1
          const int i = j - 1, s = i & 1;
          ok = mbar_wait(p_full, i & 1) && (i < 1 || mbar_wait(o_free, (i - 1) & 1));
          if (!ok) break;
          tc_fence_after();
          const uint32_t sv = smem_u32(sm + kAtKV + s * 2 * kAtTile + kAtTile);
#pragma unroll
          for (int kk = 0; kk < kAtKeys / 16; ++kk)
            mma_bf16(tmem + 2 * kAtKeys, sw128_desc(sp + (kk / 4) * kAtHalf + (kk % 4) * 32),
                     sw128_mn_desc(sv + kk * 2048, kAtHalf, 1024), id_pv, (i > 0 || kk > 0) ? 1u : 0u);
          mma_commit(o_full);
          mma_commit(&kv_empty[s]);
        }
      }
      if (!ok) {
        at_fail();
        *stop = 1;
      }
      // no MMA may still be writing TMEM when it is freed
      mma_commit(mma_done);
      if (!mbar_wait(mma_done, 0)) at_fail();
    }
  } else {
    // ---------------- softmax warps 0-3: row r = TMEM lane r ----------------
    const int r = warp * 32 + lane;
    // last key row r sees: its position, clamped to the tile's key range
    const int lim = min(pos0 + min(q0 + r, a.seq - 1), kv_len - 1);
    const float sl2 = a.scale * 1.4426950408889634f;  // scores in log2 units
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
    const uint32_t to = lane_base + 2 * kAtKeys;  // the output accumulator
    unsigned char* prow = sm + kAtP;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      const int s = j & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[s], (j >> 1) & 1) && !*stop);  // warp-uniform
      if (!ok) break;
      tc_fence_after();
      const uint32_t ts = lane_base + s * kAtKeys;
      const int k0 = j * kAtKeys;
      // pass 1: row max
      float mx = m;
#pragma unroll
      for (int c = 0; c < kAtKeys / 16; ++c) {
        float v[16];
        tmem_ld16(ts + c * 16, v);
#pragma unroll
        for (int e = 0; e < 16; ++e)
          if (k0 + c * 16 + e <= lim) mx = fmaxf(mx, v[e] * sl2);
      }
      const float alpha = exp2f(m - mx);  // 0 for the first tile (m = -inf, mx finite)
      if (j >= 1) {
        // P(j - 1) V(j - 1) is done: O is relative to the previous max; rescale it
        ok = __all_sync(0xffffffffu, mbar_wait(o_full, (j - 1) & 1));
        if (!ok) break;
        tc_fence_after();
        if (!__all_sync(0xffffffffu, alpha == 1.f)) {
#pragma unroll 1
          for (int c = 0; c < kAtHd / 16; ++c) {
            float v[16];
            tmem_ld16(to + c * 16, v);
#pragma unroll
            for (int e = 0; e < 16; ++e) v[e] *= alpha;
            tmem_st16(to + c * 16, v);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(o_free);
      }
      // pass 2: P = exp2(S - max) as bf16 into the A-operand layout, running sum
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < kAtKeys / 16; ++c) {
        float v[16];
        tmem_ld16(ts + c * 16, v);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          v[e] = k0 + c * 16 + e <= lim ? exp2f(v[e] * sl2 - mx) : 0.f;
          sum += v[e];
        }
        // keys c*16 .. c*16+15: half c / 4, 16-byte chunks 2 * (c % 4) and + 1
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          float f[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] = v[q * 8 + e];
          const int chunk = 2 * (c % 4) + q;
          *reinterpret_cast<int4*>(prow + (c / 4) * kAtHalf + r * 128 + ((chunk ^ (r & 7)) << 4)) =
              pack(f, __nv_bfloat16());
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();  // P is read by the tensor cores (async proxy)
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&s_free[s]);
        mbar_arrive(p_full);
      }
      l = l * alpha + sum;
      m = mx;
    }
    if (ok && n > 0) ok = __all_sync(0xffffffffu, mbar_wait(o_full, (n - 1) & 1));
    if (!ok) {
      if (lane == 0) at_fail();
      *stop = 1;
    } else {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* out =
          static_cast<__nv_bfloat16*>(a.out) + (((size_t)b * a.seq + q0 + r) * a.hq + h) * kAtHd;
#pragma unroll 1
      for (int c = 0; c < kAtHd / 16; ++c) {
        float v[16];
        tmem_ld16(to + c * 16, v);  // every lane loads (warp-collective), valid rows store
        if (q0 + r < a.seq) {
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = v[q * 8 + e] * inv;
            *reinterpret_cast<int4*>(out + c * 16 + q * 8) = pack(f, __nv_bfloat16());
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---- host side ------------------------------------------------------------------------

// Prefill attention kernel: warp-level MMA (attention_prefill.cu, the default) or this
// one, chosen by PIM_ATTN=tc at the first call and by set_prefill_attention_kernel().
static std::atomic<int> g_prefill_attn{-1};

int prefill_attention_kernel() {
  int v = g_prefill_attn.load(std::memory_order_relaxed);
  if (v < 0) {
    const char* e = getenv("PIM_ATTN");
    v = (e && e[0] == 't') ? 1 : 0;
    int expected = -1;
    if (!g_prefill_attn.compare_exchange_strong(expected, v)) v = expected;
  }
  return v;
}

void set_prefill_attention_kernel(int v) { g_prefill_attn.store(v, std::memory_order_relaxed); }

static bool attention_tc_enabled() { return prefill_attention_kernel() == 1; }

bool attention_tc_supported(const AttnArgs& a, int dtype) {
  return attention_tc_enabled() && dtype == BF16 && a.hd == kAtHd && a.seq >= 16 && a.hkv > 0 &&
         a.hq % a.hkv == 0 && ((uintptr_t)a.q & 15) == 0 && ((uintptr_t)a.kv_base & 15) == 0 &&
         (a.block_stride * 2) % 16 == 0 && (a.seq_stride * 2) % 16 == 0 && a.block_stride >= (long long)a.max_seq * kAtHd;
}

cudaError_t attention_tc(const AttnArgs& a, cudaStream_t st) {
  auto fn = encode_tiled();
  if (!fn) return cudaErrorNotSupported;
  CUtensorMap tq, tkv;
  {  // Q: [batch * seq rows, hq * hd] bf16, boxes of 128 rows x 64 columns
    cuuint64_t dims[2] = {(cuuint64_t)a.hq * kAtHd, (cuuint64_t)a.batch * a.seq};
    cuuint64_t strides[1] = {(cuuint64_t)a.hq * kAtHd * 2};
    cuuint32_t box[2] = {64, kAtRows};
    cuuint32_t elem[2] = {1, 1};
    if (fn(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(a.q), dims, strides, box, elem,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  {  // K / V blocks: (head dim, position, block = 2 * kv head + k|v, sequence)
    cuuint64_t dims[4] = {(cuuint64_t)kAtHd, (cuuint64_t)a.max_seq, (cuuint64_t)2 * a.hkv, (cuuint64_t)a.batch};
    cuuint64_t strides[3] = {(cuuint64_t)kAtHd * 2, (cuuint64_t)a.block_stride * 2, (cuuint64_t)a.seq_stride * 2};
    cuuint32_t box[4] = {64, kAtKeys, 1, 1};
    cuuint32_t elem[4] = {1, 1, 1, 1};
    if (a.batch == 1) strides[2] = strides[1] * 2 * a.hkv;  // unused dimension: any valid stride
    if (fn(&tkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(a.kv_base), dims, strides, box, elem,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    const cudaError_t e =
        cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAtSmem);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const dim3 grid((a.seq + kAtRows - 1) / kAtRows, a.hq, a.batch);
  return launch_pdl(attn_tc_kernel, grid, dim3(kAtThreads), kAtSmem, st, tq, tkv, a);
}

int attention_tc_errors(bool reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_attn_tc_err, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_attn_tc_err, &zero, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

}  // namespace pim
