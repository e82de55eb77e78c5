// Bandwidth-bound helpers of the step graph: embedding gather, residual add,
// row selection, greedy argmax, plain copies and the seeded normal initialiser.

#include <math.h>

#include "pim_common.cuh"

namespace pim {

// out[i, :] = table[ids[i], :]; out-of-range ids produce a zero row and raise *err.
template <typename T>
__global__ void embedding_kernel(const int* __restrict__ ids, const T* __restrict__ table, T* __restrict__ out,
                                 int n_ids, int hidden, int vocab, int* err) {
  const int i = blockIdx.x;
  if (i >= n_ids) return;
  const int id = ids[i];
  const bool ok = id >= 0 && id < vocab;
  if (!ok && threadIdx.x == 0 && err) atomicExch(err, 1);
  for (int k = threadIdx.x; k < hidden; k += blockDim.x)
    out[(size_t)i * hidden + k] = ok ? table[(size_t)id * hidden + k] : from_f<T>(0.f);
}

template <typename T>
__global__ void add_kernel(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ y, int64_t n) {
  pdl_trigger();
  pdl_wait();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = from_f<T>(to_f(a[i]) + to_f(b[i]));
}

// out[b, 0, :] = x[b, index, :]
__global__ void select_rows_kernel(const char* __restrict__ x, char* __restrict__ out, int seq, int64_t row_bytes,
                                   int index) {
  const int b = blockIdx.x;
  const char* src = x + ((int64_t)b * seq + index) * row_bytes;
  char* dst = out + (int64_t)b * row_bytes;
  for (int64_t i = threadIdx.x; i < row_bytes; i += blockDim.x) dst[i] = src[i];
}

// First index of the maximum of each row (numpy.argmax tie rule).
template <typename T>
__global__ void argmax_kernel(const T* __restrict__ x, int* __restrict__ out, int n) {
  constexpr int V = VecW<T>::n;
  const int r = blockIdx.x;
  const T* row = x + (size_t)r * n;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  pdl_trigger();
  pdl_wait();
  // 16-byte vectors when the row allows it, scalars for the rest
  const bool vec = ((uintptr_t)row % 16 == 0);
  const int nv = vec ? n / V : 0;
  for (int c = threadIdx.x; c < nv; c += blockDim.x) {
    float f[V];
    unpack(*reinterpret_cast<const int4*>(row + (size_t)c * V), f, T());
#pragma unroll
    for (int e = 0; e < V; ++e) {
      const int i = c * V + e;
      if (f[e] > best || (f[e] == best && i < bi)) {
        best = f[e];
        bi = i;
      }
    }
  }
  for (int i = nv * V + threadIdx.x; i < n; i += blockDim.x) {
    const float v = to_f(row[i]);
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < blockDim.x / 32; ++w)
      if (sv[w] > best || (sv[w] == best && si[w] < bi)) {
        best = sv[w];
        bi = si[w];
      }
    out[r] = bi == 0x7fffffff ? 0 : bi;
  }
}

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

// Seeded N(0, std^2) values: counter-based splitmix64 -> two uniforms -> Box-Muller.
template <typename T>
__global__ void fill_normal_kernel(T* __restrict__ out, int64_t n, uint64_t seed, float std) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t r = splitmix64(seed * 0x100000001b3ull + (uint64_t)i);
    const float u1 = ((float)(r >> 40) + 1.f) * (1.f / 16777217.f);
    const float u2 = (float)((r >> 16) & 0xffffff) * (1.f / 16777216.f);
    const float z = sqrtf(-2.f * logf(u1)) * cospif(2.f * u2);
    out[i] = from_f<T>(z * std);
  }
}

template <typename T>
__global__ void fill_const_kernel(T* __restrict__ out, int64_t n, float v) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = from_f<T>(v);
}

static int grid_for(int64_t n, int threads = 256) {
  int64_t g = (n + threads - 1) / threads;
  if (g > 148 * 16) g = 148 * 16;
  return (int)(g < 1 ? 1 : g);
}

cudaError_t embedding(const int* ids, const void* table, void* out, int n_ids, int hidden, int vocab, int dtype,
                      int* err, cudaStream_t st) {
  if (dtype == BF16)
    launch_plain(embedding_kernel<__nv_bfloat16>, n_ids, 256, 0, st, ids, static_cast<const __nv_bfloat16*>(table),
                 static_cast<__nv_bfloat16*>(out), n_ids, hidden, vocab, err);
  else
    launch_plain(embedding_kernel<float>, n_ids, 256, 0, st, ids, static_cast<const float*>(table),
                 static_cast<float*>(out), n_ids, hidden, vocab, err);
  return cudaGetLastError();
}

cudaError_t add(const void* a, const void* b, void* y, int64_t n, int dtype, cudaStream_t st) {
  if (dtype == BF16)
    return launch_pdl(add_kernel<__nv_bfloat16>, dim3(grid_for(n)), dim3(256), 0, st,
                      static_cast<const __nv_bfloat16*>(a), static_cast<const __nv_bfloat16*>(b),
                      static_cast<__nv_bfloat16*>(y), n);
  return launch_pdl(add_kernel<float>, dim3(grid_for(n)), dim3(256), 0, st, static_cast<const float*>(a),
                    static_cast<const float*>(b), static_cast<float*>(y), n);
}

cudaError_t select_rows(const void* x, void* out, int batch, int seq, int64_t row_bytes, int index, cudaStream_t st) {
  launch_plain(select_rows_kernel, batch, 256, 0, st, static_cast<const char*>(x), static_cast<char*>(out), seq,
               row_bytes, index);
  return cudaGetLastError();
}

cudaError_t argmax(const void* x, int* out, int rows, int n, int dtype, cudaStream_t st) {
  if (dtype == BF16)
    return launch_pdl(argmax_kernel<__nv_bfloat16>, dim3(rows), dim3(1024), 0, st,
                      static_cast<const __nv_bfloat16*>(x), out, n);
  return launch_pdl(argmax_kernel<float>, dim3(rows), dim3(1024), 0, st, static_cast<const float*>(x), out, n);
}

cudaError_t fill_normal(void* out, int64_t n, int dtype, uint64_t seed, float std, cudaStream_t st) {
  if (dtype == BF16)
    launch_plain(fill_normal_kernel<__nv_bfloat16>, grid_for(n), 256, 0, st, static_cast<__nv_bfloat16*>(out), n,
                 seed, std);
  else
    launch_plain(fill_normal_kernel<float>, grid_for(n), 256, 0, st, static_cast<float*>(out), n, seed, std);
  return cudaGetLastError();
}

cudaError_t fill_const(void* out, int64_t n, int dtype, float v, cudaStream_t st) {
  if (dtype == BF16)
    launch_plain(fill_const_kernel<__nv_bfloat16>, grid_for(n), 256, 0, st, static_cast<__nv_bfloat16*>(out), n, v);
  else
    launch_plain(fill_const_kernel<float>, grid_for(n), 256, 0, st, static_cast<float*>(out), n, v);
  return cudaGetLastError();
}

}  // namespace pim
