// Causal attention for row batches (prefill), bf16, head_dim 128, on the tensor cores
// (warp-level mma.sync m16n8k16, fp32 accumulation), online softmax over 64-key blocks.
//
// One CTA = 64 query rows of one (sequence, head), 4 warps of 16 rows each.  The Q tile
// is loaded once; K and V blocks of 64 keys are double-buffered in shared memory with
// cp.async (16-byte chunks XOR-swizzled by row so that ldmatrix reads are conflict-free).
// Per block a warp computes S = Q K^T (16 x 64), masks keys past each row's position,
// updates the running max / sum, rescales its O accumulator (16 x 128) and adds P V with
// P taken straight from the S accumulators as bf16 A fragments.  Heavy query blocks
// (late rows see more keys) are scheduled first.
//
// Keys are read from the KV blocks of the layer ([pos][head_dim] per (kv head, k|v,
// sequence)); the query at position p sees keys 0..p, as the split-K decode kernel.

#include "pim_common.cuh"
#include "pim_kernels.h"

namespace pim {

constexpr int kFaRows = 64;   // query rows per CTA
constexpr int kFaKeys = 64;   // keys per block
constexpr int kFaHd = 128;    // head_dim
constexpr int kFaThreads = 128;
constexpr int kFaTileBytes = 64 * kFaHd * 2;  // 16 KB: 64 rows of 256 bytes
constexpr size_t kFaSmem = 5 * (size_t)kFaTileBytes;  // Q + 2 x (K, V)

// Byte offset of 16-byte chunk c (0..15) of row r in a swizzled 64 x 128 bf16 tile.
__device__ __forceinline__ uint32_t fa_off(int r, int c) { return (uint32_t)(r * 256 + ((c ^ (r & 7)) << 4)); }

__device__ __forceinline__ void fa_cp16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// D (16x8 fp32) += A (16x16 bf16, row) . B (16x8 bf16, col)
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(lo)) |
         ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(hi)) << 16);
}

// Copies rows [r0, r0 + 64) of a [rows_valid, 128] bf16 matrix (row stride `ld`
// elements) into a swizzled tile; rows past rows_valid are zero-filled.
__device__ __forceinline__ void fa_load_tile(uint32_t tile, const __nv_bfloat16* base, size_t ld, int r0,
                                             int rows_valid) {
#pragma unroll
  for (int i = 0; i < (64 * 16) / kFaThreads; ++i) {
    const int idx = threadIdx.x + i * kFaThreads;
    const int r = idx / 16, c = idx % 16;
    const bool ok = r0 + r < rows_valid;
    const __nv_bfloat16* src = base + (size_t)(ok ? r0 + r : 0) * ld + c * 8;
    fa_cp16(tile + fa_off(r, c), src, ok);
  }
}

__global__ void __launch_bounds__(kFaThreads, 2) attn_prefill_kernel(AttnArgs a) {
  extern __shared__ __align__(128) unsigned char fa_smem[];
  const uint32_t sq = smem_u32(fa_smem);
  const uint32_t sk[2] = {sq + kFaTileBytes, sq + 3 * kFaTileBytes};
  const uint32_t sv[2] = {sq + 2 * kFaTileBytes, sq + 4 * kFaTileBytes};

  const int nqb = (a.seq + kFaRows - 1) / kFaRows;
  const int qb = nqb - 1 - (int)blockIdx.x;  // heavy blocks first
  const int h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (a.hq / a.hkv);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int g = lane / 4, t = lane % 4;
  const int q0 = qb * kFaRows;

  pdl_trigger();
  pdl_wait();
  const int pos0 = a.positions[b];
  // keys needed by this tile: 0 .. position of its last valid row (within max_seq)
  const int last_row = min(q0 + kFaRows, a.seq) - 1;
  const int kv_len = min(pos0 + last_row + 1, a.max_seq);
  const int nkb = (kv_len + kFaKeys - 1) / kFaKeys;

  const __nv_bfloat16* q = static_cast<const __nv_bfloat16*>(a.q) + ((size_t)b * a.seq * a.hq + h) * kFaHd;
  const size_t q_ld = (size_t)a.hq * kFaHd;
  const __nv_bfloat16* kbase =
      static_cast<const __nv_bfloat16*>(a.kv_base) + (2 * kvh) * a.block_stride + b * a.seq_stride;
  const __nv_bfloat16* vbase = kbase + a.block_stride;

  fa_load_tile(sq, q, q_ld, q0, a.seq);
  fa_load_tile(sk[0], kbase, kFaHd, 0, kv_len);
  fa_load_tile(sv[0], vbase, kFaHd, 0, kv_len);
  asm volatile("cp.async.commit_group;" ::: "memory");

  // Rows of this thread: r_lo = warp * 16 + g and r_lo + 8 (tile-relative).
  const int r_lo = warp * 16 + g;
  const int p_lo = pos0 + min(q0 + r_lo, a.seq - 1);
  const int p_hi = pos0 + min(q0 + r_lo + 8, a.seq - 1);
  const float sl2 = a.scale * 1.4426950408889634f;  // scores in log2 units

  uint32_t qf[8][4];
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;

  for (int kb = 0; kb < nkb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < nkb) {
      fa_load_tile(sk[buf ^ 1], kbase, kFaHd, (kb + 1) * kFaKeys, kv_len);
      fa_load_tile(sv[buf ^ 1], vbase, kFaHd, (kb + 1) * kFaKeys, kv_len);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 1;" ::: "memory");
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int r = warp * 16 + (lane % 8) + 8 * ((lane / 8) % 2);
        ldsm_x4(sq + fa_off(r, 2 * ks + lane / 16), qf[ks]);
      }
    }
    // ---- S = Q K^T for 64 keys: 8 n-tiles of 8 keys ----
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {  // pairs of n-tiles
        uint32_t kf[4];
        const int key = jp * 16 + (lane % 8) + 8 * (lane / 16);
        ldsm_x4(sk[buf] + fa_off(key, 2 * ks + (lane / 8) % 2), kf);
        mma16816(s[2 * jp], qf[ks], kf[0], kf[1]);
        mma16816(s[2 * jp + 1], qf[ks], kf[2], kf[3]);
      }
    }
    // ---- mask, online softmax ----
    const int k0 = kb * kFaKeys;
    float mx_lo = m_lo, mx_hi = m_hi;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = k0 + 8 * j + 2 * t + e;
        s[j][e] = key <= p_lo && key < kv_len ? s[j][e] * sl2 : -INFINITY;
        s[j][2 + e] = key <= p_hi && key < kv_len ? s[j][2 + e] * sl2 : -INFINITY;
        mx_lo = fmaxf(mx_lo, s[j][e]);
        mx_hi = fmaxf(mx_hi, s[j][2 + e]);
      }
    }
    mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 1));
    mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 2));
    mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 1));
    mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 2));
    const float base_lo = mx_lo == -INFINITY ? 0.f : mx_lo;
    const float base_hi = mx_hi == -INFINITY ? 0.f : mx_hi;
    const float al_lo = exp2f(m_lo - base_lo), al_hi = exp2f(m_hi - base_hi);
    m_lo = mx_lo;
    m_hi = mx_hi;
    float sum_lo = 0.f, sum_hi = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        s[j][e] = exp2f(s[j][e] - base_lo);
        s[j][2 + e] = exp2f(s[j][2 + e] - base_hi);
        sum_lo += s[j][e];
        sum_hi += s[j][2 + e];
      }
    }
    l_lo = l_lo * al_lo + sum_lo;
    l_hi = l_hi * al_hi + sum_hi;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      o[i][0] *= al_lo;
      o[i][1] *= al_lo;
      o[i][2] *= al_hi;
      o[i][3] *= al_hi;
    }
    // ---- O += P V: 4 key steps of 16, 16 n-tiles of 8 head dims ----
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {  // pairs of d n-tiles (16 head dims)
        uint32_t vf[4];
        const int key = kk * 16 + (lane % 8) + 8 * ((lane / 8) % 2);
        ldsm_x4_t(sv[buf] + fa_off(key, 2 * dp + lane / 16), vf);
        mma16816(o[2 * dp], pa, vf[0], vf[1]);
        mma16816(o[2 * dp + 1], pa, vf[2], vf[3]);
      }
    }
    __syncthreads();  // this buffer is refilled by the next iteration's prefetch
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");

  // ---- normalise and store ----
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);
  const float inv_lo = l_lo > 0.f ? 1.f / l_lo : 0.f, inv_hi = l_hi > 0.f ? 1.f / l_hi : 0.f;
  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out) + ((size_t)b * a.seq * a.hq + h) * kFaHd;
  const int row_lo = q0 + r_lo, row_hi = q0 + r_lo + 8;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int d = 8 * i + 2 * t;
    if (row_lo < a.seq)
      *reinterpret_cast<uint32_t*>(out + (size_t)row_lo * q_ld + d) = pack_bf16x2(o[i][0] * inv_lo, o[i][1] * inv_lo);
    if (row_hi < a.seq)
      *reinterpret_cast<uint32_t*>(out + (size_t)row_hi * q_ld + d) = pack_bf16x2(o[i][2] * inv_hi, o[i][3] * inv_hi);
  }
}

bool attention_prefill_supported(const AttnArgs& a, int dtype) {
  return dtype == BF16 && a.hd == kFaHd && a.seq >= 16 && a.hq % a.hkv == 0;
}

cudaError_t attention_prefill(const AttnArgs& a, cudaStream_t st) {
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    const cudaError_t e =
        cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kFaSmem);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const dim3 grid((a.seq + kFaRows - 1) / kFaRows, a.hq, a.batch);
  return launch_pdl(attn_prefill_kernel, grid, dim3(kFaThreads), kFaSmem, st, a);
}

}  // namespace pim
