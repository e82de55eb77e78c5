// Redistribute kernels: the device form of the host-star combine steps.
//
// ordered_sum  Partial -> Replicate.  out = (((0 + p0) + p1) + ... ) with the sum
//              rounded to the element type after every partial, in rank order,
//              then an optional division by the partial count (mean).  For bf16
//              each step is an fp32 add followed by round-to-nearest-even to bf16,
//              which is exactly how the host-star all_reduce accumulates in its
//              dtype, so the result is bit-identical to it.  Writes every
//              destination (one per receiving rank).
//              Launched with programmatic dependent launch, so that the kernel after
//              it (the residual add) can start while it runs.
// batched_copy A table of (src, dst, nbytes) runs executed by one launch: the
//              collect/writeback segments of all_gather, all_to_all and scatter.

#include "pim_common.cuh"

namespace pim {

constexpr int kMaxRanks = 8;

struct PtrSet {
  const void* src[kMaxRanks];
  void* dst[kMaxRanks];
};

template <typename T>
__global__ void ordered_sum_kernel(PtrSet p, int nsrc, int ndst, int64_t n, int mean) {
  pdl_trigger();
  pdl_wait();  // the partials come from the previous kernel
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float acc = 0.f;
#pragma unroll 1
    for (int s = 0; s < nsrc; ++s) acc = rnd<T>(__fadd_rn(acc, to_f(static_cast<const T*>(p.src[s])[i])));
    if (mean) acc = rnd<T>(__fdiv_rn(acc, (float)nsrc));
    const T v = from_f<T>(acc);
#pragma unroll 1
    for (int d = 0; d < ndst; ++d) static_cast<T*>(p.dst[d])[i] = v;
  }
}

// Vectorised variant for bf16 when every pointer is 16-byte aligned and n % 8 == 0.
__global__ void ordered_sum_bf16x8_kernel(PtrSet p, int nsrc, int ndst, int64_t nvec, int mean) {
  pdl_trigger();
  pdl_wait();  // the partials come from the previous kernel
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nvec; i += (int64_t)gridDim.x * blockDim.x) {
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll 1
    for (int s = 0; s < nsrc; ++s) {
      const int4 v = reinterpret_cast<const int4*>(p.src[s])[i];
      float f[8];
      unpack(v, f, __nv_bfloat16());
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = rnd<__nv_bfloat16>(__fadd_rn(acc[e], f[e]));
    }
    if (mean)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = rnd<__nv_bfloat16>(__fdiv_rn(acc[e], (float)nsrc));
    int4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(acc[2 * e]));
      const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(acc[2 * e + 1]));
      ow[e] = lo | (hi << 16);
    }
#pragma unroll 1
    for (int d = 0; d < ndst; ++d) reinterpret_cast<int4*>(p.dst[d])[i] = o;
  }
}

// ordered_sum followed by the plan's residual `add`: y = residual + S, S the rank-order
// sum rounded to T after every partial (as ordered_sum), the add rounded once more (as
// the add kernel); S itself also goes to sum_out when another command reads it.
template <typename T>
__global__ void ordered_sum_add_kernel(PtrSet p, int nsrc, const T* __restrict__ res, T* __restrict__ y,
                                       T* __restrict__ sum_out, int64_t n) {
  pdl_trigger();
  pdl_wait();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float acc = 0.f;
#pragma unroll 1
    for (int s = 0; s < nsrc; ++s) acc = rnd<T>(__fadd_rn(acc, to_f(static_cast<const T*>(p.src[s])[i])));
    if (sum_out) sum_out[i] = from_f<T>(acc);
    y[i] = from_f<T>(__fadd_rn(to_f(res[i]), acc));
  }
}

// Vectorised bf16 form (every pointer 16-byte aligned, n % 8 == 0).
__global__ void ordered_sum_add_bf16x8_kernel(PtrSet p, int nsrc, const int4* __restrict__ res, int4* __restrict__ y,
                                              int4* __restrict__ sum_out, int64_t nvec) {
  pdl_trigger();
  pdl_wait();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nvec; i += (int64_t)gridDim.x * blockDim.x) {
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll 1
    for (int s = 0; s < nsrc; ++s) {
      float f[8];
      unpack(reinterpret_cast<const int4*>(p.src[s])[i], f, __nv_bfloat16());
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = rnd<__nv_bfloat16>(__fadd_rn(acc[e], f[e]));
    }
    if (sum_out) sum_out[i] = pack(acc, __nv_bfloat16());
    float r[8];
    unpack(res[i], r, __nv_bfloat16());
#pragma unroll
    for (int e = 0; e < 8; ++e) r[e] = __fadd_rn(r[e], acc[e]);
    y[i] = pack(r, __nv_bfloat16());
  }
}

struct CopyDesc {
  const char* src;
  char* dst;
  int64_t nbytes;
};

// blockIdx.x: descriptor; blockIdx.y: slice of a long run.
__global__ void batched_copy_kernel(const CopyDesc* __restrict__ desc, int count, int64_t slice) {
  const int di = blockIdx.x;
  if (di >= count) return;
  const CopyDesc d = desc[di];
  const int64_t lo = (int64_t)blockIdx.y * slice;
  if (lo >= d.nbytes) return;
  const int64_t hi = min(d.nbytes, lo + slice);
  const bool vec = (((uintptr_t)(d.src + lo) | (uintptr_t)(d.dst + lo)) % 16 == 0);
  if (vec) {
    const int64_t nv = (hi - lo) / 16;
    const int4* s = reinterpret_cast<const int4*>(d.src + lo);
    int4* t = reinterpret_cast<int4*>(d.dst + lo);
    for (int64_t i = threadIdx.x; i < nv; i += blockDim.x) t[i] = s[i];
    for (int64_t i = lo + nv * 16 + threadIdx.x; i < hi; i += blockDim.x) d.dst[i] = d.src[i];
  } else {
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) d.dst[i] = d.src[i];
  }
}

static int clamp_grid(int64_t work) {
  int64_t g = (work + 255) / 256;
  if (g > 148 * 8) g = 148 * 8;
  return g < 1 ? 1 : (int)g;
}

cudaError_t ordered_sum(const void* const* src, int nsrc, void* const* dst, int ndst, int64_t n, int dtype, int mean,
                        cudaStream_t st) {
  if (nsrc < 1 || nsrc > kMaxRanks || ndst < 0 || ndst > kMaxRanks) return cudaErrorInvalidValue;
  if (ndst == 0 || n == 0) return cudaSuccess;
  PtrSet p{};
  uintptr_t align = 0;
  for (int i = 0; i < nsrc; ++i) {
    p.src[i] = src[i];
    align |= (uintptr_t)src[i];
  }
  for (int i = 0; i < ndst; ++i) {
    p.dst[i] = dst[i];
    align |= (uintptr_t)dst[i];
  }
  if (dtype == BF16 && n % 8 == 0 && align % 16 == 0) {
    launch_pdl(ordered_sum_bf16x8_kernel, clamp_grid(n / 8), 256, 0, st, p, nsrc, ndst, n / 8, mean);
  } else if (dtype == BF16) {
    launch_pdl(ordered_sum_kernel<__nv_bfloat16>, clamp_grid(n), 256, 0, st, p, nsrc, ndst, n, mean);
  } else {
    launch_pdl(ordered_sum_kernel<float>, clamp_grid(n), 256, 0, st, p, nsrc, ndst, n, mean);
  }
  return cudaGetLastError();
}

cudaError_t ordered_sum_add(const void* const* src, int nsrc, const void* res, void* y, void* sum_out, int64_t n,
                            int dtype, cudaStream_t st) {
  if (nsrc < 1 || nsrc > kMaxRanks || !res || !y) return cudaErrorInvalidValue;
  if (n == 0) return cudaSuccess;
  PtrSet p{};
  uintptr_t align = (uintptr_t)res | (uintptr_t)y | (uintptr_t)sum_out;
  for (int i = 0; i < nsrc; ++i) {
    p.src[i] = src[i];
    align |= (uintptr_t)src[i];
  }
  if (dtype == BF16 && n % 8 == 0 && align % 16 == 0) {
    launch_pdl(ordered_sum_add_bf16x8_kernel, clamp_grid(n / 8), 256, 0, st, p, nsrc,
                 static_cast<const int4*>(res), static_cast<int4*>(y), static_cast<int4*>(sum_out), n / 8);
  } else if (dtype == BF16) {
    launch_pdl(ordered_sum_add_kernel<__nv_bfloat16>, clamp_grid(n), 256, 0, st, p, nsrc,
                 static_cast<const __nv_bfloat16*>(res), static_cast<__nv_bfloat16*>(y),
                 static_cast<__nv_bfloat16*>(sum_out), n);
  } else {
    launch_pdl(ordered_sum_add_kernel<float>, clamp_grid(n), 256, 0, st, p, nsrc, static_cast<const float*>(res),
                 static_cast<float*>(y), static_cast<float*>(sum_out), n);
  }
  return cudaGetLastError();
}

cudaError_t batched_copy(const void* desc_dev, int count, int64_t max_nbytes, cudaStream_t st) {
  if (count <= 0) return cudaSuccess;
  int64_t slice = 256 * 1024;
  int64_t ys = (max_nbytes + slice - 1) / slice;
  if (ys > 1024) {
    slice = (max_nbytes + 1023) / 1024;
    slice = (slice + 15) / 16 * 16;
    ys = (max_nbytes + slice - 1) / slice;
  }
  if (ys < 1) ys = 1;
  launch_plain(batched_copy_kernel, dim3(count, (unsigned)ys), 256, 0, st, static_cast<const CopyDesc*>(desc_dev),
               count, slice);
  return cudaGetLastError();
}

}  // namespace pim
