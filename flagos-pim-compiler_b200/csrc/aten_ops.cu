// Generic tensor operations for graphs compiled at aten granularity by the reference's
// own passes (graph/partition.py: linear / add / mul / tanh on the DPUs, the rest --
// embedding, RMSNorm's pow / mean / rsqrt, views, transposes, slices, cat, dtype casts,
// the rotary embedding's matmul / cos / sin, scaled_dot_product_attention, silu -- as
// host nodes).  On the B200 every one of them runs on the device: DPU nodes on their
// rank's arena, host nodes on the plan's device-resident host buffer.
//
// Every operand is a strided view (pim_tensor_view): base pointer, element offset,
// shape and element strides, so views, transposes, slices, expands and the broadcasting
// of elementwise operands need no copies of their own; a stride of 0 broadcasts.  The
// outputs the plans give these kernels are contiguous buffers.  These kernels serve the
// aten-level path (tiny models, correctness); the LLaMA step graphs of this runtime run
// on the fused kernels instead.

#include <math.h>
#include <stdint.h>

#include "pim_b200.h"
#include "pim_common.cuh"

namespace pim {

constexpr int kAtenMaxDims = PIM_MAX_DIMS;

struct View {
  char* data;
  int dtype;
  int ndim;
  long long offset;
  long long shape[kAtenMaxDims];
  long long stride[kAtenMaxDims];
};

static View to_view(const pim_tensor_view& v) {
  View o;
  o.data = static_cast<char*>(v.data);
  o.dtype = v.dtype;
  o.ndim = v.ndim;
  o.offset = v.offset;
  for (int i = 0; i < kAtenMaxDims; ++i) {
    o.shape[i] = i < v.ndim ? v.shape[i] : 1;
    o.stride[i] = i < v.ndim ? v.stride[i] : 0;
  }
  return o;
}

__device__ __forceinline__ double ld(const View& v, long long off) {
  switch (v.dtype) {
    case PIM_F32: return reinterpret_cast<const float*>(v.data)[off];
    case PIM_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(v.data)[off]);
    case PIM_I32: return reinterpret_cast<const int32_t*>(v.data)[off];
    default: return (double)reinterpret_cast<const long long*>(v.data)[off];
  }
}

__device__ __forceinline__ void st(const View& v, long long off, double x) {
  switch (v.dtype) {
    case PIM_F32: reinterpret_cast<float*>(v.data)[off] = (float)x; break;
    case PIM_BF16: reinterpret_cast<__nv_bfloat16*>(v.data)[off] = __float2bfloat16_rn((float)x); break;
    case PIM_I32: reinterpret_cast<int32_t*>(v.data)[off] = (int32_t)x; break;
    default: reinterpret_cast<long long*>(v.data)[off] = (long long)x; break;
  }
}

// Element offset in `v` of the element whose index in the iteration `shape` (ndim dims,
// the last fastest) has linear number i; `v` must have the same ndim (its shape may be 1
// with stride 0 where it broadcasts).
__device__ __forceinline__ long long offset_of(const View& v, const long long* shape, int ndim, long long i) {
  long long off = v.offset;
  for (int d = ndim - 1; d >= 0; --d) {
    const long long idx = i % shape[d];
    i /= shape[d];
    off += idx * v.stride[d];
  }
  return off;
}

static long long numel(const View& v) {
  long long n = 1;
  for (int i = 0; i < v.ndim; ++i) n *= v.shape[i];
  return n;
}

static unsigned grid_for(long long n) {
  long long g = (n + 255) / 256;
  if (g > 148LL * 16) g = 148LL * 16;
  return (unsigned)(g < 1 ? 1 : g);
}

__global__ void copy_kernel(View dst, View src, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    st(dst, offset_of(dst, dst.shape, dst.ndim, i), ld(src, offset_of(src, dst.shape, dst.ndim, i)));
}

__device__ __forceinline__ float unary(int op, float x, float s) {
  switch (op) {
    case PIM_ATEN_NEG: return -x;
    case PIM_ATEN_RSQRT: return rsqrtf(x);
    case PIM_ATEN_SQRT: return sqrtf(x);
    case PIM_ATEN_SILU: return x / (1.f + expf(-x));
    case PIM_ATEN_COS: return cosf(x);
    case PIM_ATEN_SIN: return sinf(x);
    case PIM_ATEN_TANH: return tanhf(x);
    case PIM_ATEN_EXP: return expf(x);
    case PIM_ATEN_RECIPROCAL: return 1.f / x;
    case PIM_ATEN_POW_SCALAR: return s == 2.f ? x * x : powf(x, s);
    case PIM_ATEN_ADD_SCALAR: return x + s;
    case PIM_ATEN_MUL_SCALAR: return x * s;
    case PIM_ATEN_SUB_SCALAR: return x - s;
    case PIM_ATEN_DIV_SCALAR: return x / s;
    default: return x;
  }
}

__global__ void unary_kernel(int op, View dst, View src, float s, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float x = (float)ld(src, offset_of(src, dst.shape, dst.ndim, i));
    st(dst, offset_of(dst, dst.shape, dst.ndim, i), unary(op, x, s));
  }
}

__global__ void binary_kernel(int op, View dst, View a, View b, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float x = (float)ld(a, offset_of(a, dst.shape, dst.ndim, i));
    const float y = (float)ld(b, offset_of(b, dst.shape, dst.ndim, i));
    float r;
    switch (op) {
      case PIM_ATEN_ADD: r = x + y; break;
      case PIM_ATEN_SUB: r = x - y; break;
      case PIM_ATEN_MUL: r = x * y; break;
      default: r = x / y; break;
    }
    st(dst, offset_of(dst, dst.shape, dst.ndim, i), r);
  }
}

// Mean over the last dimension, one warp per output element (rows of `src` in the
// iteration order of dst's shape, which is src's with the last dimension 1).
__global__ void mean_last_kernel(View dst, View src, long long rows) {
  const long long row = blockIdx.x * (long long)(blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;
  const int last = src.ndim - 1;
  const long long n = src.shape[last];
  const long long base = offset_of(src, src.shape, last, row);  // index over the leading dims
  float acc = 0.f;
  for (long long j = lane; j < n; j += 32) acc += (float)ld(src, base + j * src.stride[last]);
  acc = warp_sum(acc);
  if (lane == 0) st(dst, offset_of(dst, dst.shape, dst.ndim, row), acc / (float)n);
}

__global__ void arange_kernel(View dst, double start, double step, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    st(dst, offset_of(dst, dst.shape, dst.ndim, i), start + step * (double)i);
}

// dst[..., m, n] = sum_k a[..., m, k] * b[..., k, n] (fp32 accumulation, k in order).
__global__ void matmul_kernel(View dst, View a, View b, long long n) {
  const int nd = dst.ndim;
  const long long K = a.shape[nd - 1];
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    // index of dst, then of the a row and b column it needs
    long long rem = i, idx[kAtenMaxDims];
    for (int d = nd - 1; d >= 0; --d) {
      idx[d] = rem % dst.shape[d];
      rem /= dst.shape[d];
    }
    long long ao = a.offset, bo = b.offset, dof = dst.offset;
    for (int d = 0; d < nd - 2; ++d) {
      ao += (a.shape[d] == 1 ? 0 : idx[d]) * a.stride[d];
      bo += (b.shape[d] == 1 ? 0 : idx[d]) * b.stride[d];
      dof += idx[d] * dst.stride[d];
    }
    ao += idx[nd - 2] * a.stride[nd - 2];
    bo += idx[nd - 1] * b.stride[nd - 1];
    dof += idx[nd - 2] * dst.stride[nd - 2] + idx[nd - 1] * dst.stride[nd - 1];
    float acc = 0.f;
    for (long long k = 0; k < K; ++k)
      acc = fmaf((float)ld(a, ao + k * a.stride[nd - 1]), (float)ld(b, bo + k * b.stride[nd - 2]), acc);
    st(dst, dof, acc);
  }
}

// Scaled dot-product attention of one query row per CTA: q [B, H, S, D], k / v [B, Hk, L,
// D], an additive mask broadcastable to [B, H, S, L] (or none), optional causal masking
// (key j > query s excluded, torch's is_causal);
// fp32 scores and softmax, output [B, H, S, D].  Scores live in shared memory.
constexpr int kSdpaThreads = 128;
constexpr int kSdpaMaxKeys = 8192;

__global__ void __launch_bounds__(kSdpaThreads) sdpa_kernel(View out, View q, View k, View v, View mask,
                                                               int has_mask, float scale, int causal) {
  __shared__ float sc[kSdpaMaxKeys];
  __shared__ float red[kSdpaThreads / 32];
  const long long S = q.shape[2], D = q.shape[3], L = k.shape[2];
  const long long H = q.shape[1], Hk = k.shape[1];
  const long long row = blockIdx.x;  // (b * H + h) * S + s
  const long long s = row % S, h = (row / S) % H, b = row / (S * H);
  const long long hk = h / (H / Hk);
  const long long qo = q.offset + b * q.stride[0] + h * q.stride[1] + s * q.stride[2];
  const long long ko = k.offset + b * k.stride[0] + hk * k.stride[1];
  const long long vo = v.offset + b * v.stride[0] + hk * v.stride[1];
  float mx = -INFINITY;
  for (long long j = threadIdx.x; j < L; j += blockDim.x) {
    float d = 0.f;
    for (long long e = 0; e < D; ++e)
      d = fmaf((float)ld(q, qo + e * q.stride[3]), (float)ld(k, ko + j * k.stride[2] + e * k.stride[3]), d);
    d *= scale;
    if (has_mask) {
      const long long mo = mask.offset + (mask.shape[0] == 1 ? 0 : b) * mask.stride[0] +
                           (mask.shape[1] == 1 ? 0 : h) * mask.stride[1] + (mask.shape[2] == 1 ? 0 : s) * mask.stride[2] +
                           j * mask.stride[3];
      d += (float)ld(mask, mo);
    }
    if (causal && j > s) d = -INFINITY;  // torch's is_causal: lower-triangular from the top left
    sc[j] = d;
    mx = fmaxf(mx, d);
  }
  mx = warp_max(mx);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = mx;
  __syncthreads();
  mx = red[0];
  for (int w = 1; w < kSdpaThreads / 32; ++w) mx = fmaxf(mx, red[w]);
  __syncthreads();
  float sum = 0.f;
  for (long long j = threadIdx.x; j < L; j += blockDim.x) {
    const float p = mx == -INFINITY ? 0.f : expf(sc[j] - mx);
    sc[j] = p;
    sum += p;
  }
  sum = warp_sum(sum);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = sum;
  __syncthreads();
  sum = 0.f;
  for (int w = 0; w < kSdpaThreads / 32; ++w) sum += red[w];
  const float inv = sum > 0.f ? 1.f / sum : 0.f;
  const long long oo = out.offset + b * out.stride[0] + h * out.stride[1] + s * out.stride[2];
  for (long long e = threadIdx.x; e < D; e += blockDim.x) {
    float acc = 0.f;
    for (long long j = 0; j < L; ++j) acc = fmaf(sc[j], (float)ld(v, vo + j * v.stride[2] + e * v.stride[3]), acc);
    st(out, oo + e * out.stride[3], acc * inv);
  }
}

// out[i, :] = table[ids[i], :] for ids of any integer type; ids outside the table give a
// zero row and raise *err.
__global__ void gather_rows_kernel(View out, View table, View ids, long long n_ids, int* err) {
  const long long rows = table.shape[0], width = table.shape[1];
  for (long long i = blockIdx.x; i < n_ids; i += gridDim.x) {
    const long long id = (long long)ld(ids, offset_of(ids, ids.shape, ids.ndim, i));
    const bool ok = id >= 0 && id < rows;
    if (!ok && threadIdx.x == 0 && err) atomicExch(err, 1);
    for (long long e = threadIdx.x; e < width; e += blockDim.x)
      st(out, out.offset + i * width + e, ok ? ld(table, table.offset + id * table.stride[0] + e * table.stride[1]) : 0.0);
  }
}

}  // namespace pim

// ---------------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------------

namespace pim {
int report_status(int code, const char* msg);
int report_cuda(cudaError_t e, const char* what);
}  // namespace pim

static bool valid(const pim_tensor_view* v) {
  if (!v || !v->data || v->ndim < 0 || v->ndim > PIM_MAX_DIMS) return false;
  if (v->dtype != PIM_F32 && v->dtype != PIM_BF16 && v->dtype != PIM_I32 && v->dtype != PIM_I64) return false;
  for (int i = 0; i < v->ndim; ++i)
    if (v->shape[i] < 0) return false;
  return v->offset >= 0;
}

// Operand views must use the output's rank (shape entries of 1 with stride 0 broadcast).
static bool same_rank_broadcast(const pim_tensor_view* dst, const pim_tensor_view* x) {
  if (x->ndim != dst->ndim) return false;
  for (int i = 0; i < dst->ndim; ++i)
    if (x->shape[i] != dst->shape[i] && !(x->shape[i] == 1 && x->stride[i] == 0)) return false;
  return true;
}

extern "C" {

int pim_aten_copy(const pim_tensor_view* dst, const pim_tensor_view* src, void* stream) {
  if (!valid(dst) || !valid(src) || !same_rank_broadcast(dst, src))
    return pim::report_status(PIM_EINVAL, "pim_aten_copy: bad views");
  const pim::View d = pim::to_view(*dst), s = pim::to_view(*src);
  const long long n = pim::numel(d);
  if (n == 0) return PIM_OK;
  pim::launch_plain(pim::copy_kernel, dim3(pim::grid_for(n)), dim3(256), 0, (cudaStream_t)stream, d, s, n);
  return pim::report_cuda(cudaGetLastError(), "pim_aten_copy");
}

int pim_aten_unary(int32_t op, const pim_tensor_view* dst, const pim_tensor_view* src, double scalar, void* stream) {
  if (op < PIM_ATEN_NEG || op > PIM_ATEN_DIV_SCALAR) return pim::report_status(PIM_EINVAL, "pim_aten_unary: bad op");
  if (!valid(dst) || !valid(src) || !same_rank_broadcast(dst, src))
    return pim::report_status(PIM_EINVAL, "pim_aten_unary: bad views");
  const pim::View d = pim::to_view(*dst), s = pim::to_view(*src);
  const long long n = pim::numel(d);
  if (n == 0) return PIM_OK;
  pim::launch_plain(pim::unary_kernel, dim3(pim::grid_for(n)), dim3(256), 0, (cudaStream_t)stream, (int)op, d, s,
                    (float)scalar, n);
  return pim::report_cuda(cudaGetLastError(), "pim_aten_unary");
}

int pim_aten_binary(int32_t op, const pim_tensor_view* dst, const pim_tensor_view* a, const pim_tensor_view* b,
                    void* stream) {
  if (op < PIM_ATEN_ADD || op > PIM_ATEN_DIV) return pim::report_status(PIM_EINVAL, "pim_aten_binary: bad op");
  if (!valid(dst) || !valid(a) || !valid(b) || !same_rank_broadcast(dst, a) || !same_rank_broadcast(dst, b))
    return pim::report_status(PIM_EINVAL, "pim_aten_binary: bad views");
  const pim::View d = pim::to_view(*dst), x = pim::to_view(*a), y = pim::to_view(*b);
  const long long n = pim::numel(d);
  if (n == 0) return PIM_OK;
  pim::launch_plain(pim::binary_kernel, dim3(pim::grid_for(n)), dim3(256), 0, (cudaStream_t)stream, (int)op, d, x, y,
                    n);
  return pim::report_cuda(cudaGetLastError(), "pim_aten_binary");
}

int pim_aten_mean_last(const pim_tensor_view* dst, const pim_tensor_view* src, void* stream) {
  if (!valid(dst) || !valid(src) || src->ndim < 1 || dst->ndim != src->ndim || dst->shape[dst->ndim - 1] != 1)
    return pim::report_status(PIM_EINVAL, "pim_aten_mean_last: bad views");
  for (int i = 0; i + 1 < src->ndim; ++i)
    if (dst->shape[i] != src->shape[i]) return pim::report_status(PIM_EINVAL, "pim_aten_mean_last: shapes");
  const pim::View d = pim::to_view(*dst), s = pim::to_view(*src);
  const long long rows = pim::numel(d);
  if (rows == 0) return PIM_OK;
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  pim::launch_plain(pim::mean_last_kernel, dim3(blocks), dim3(256), 0, (cudaStream_t)stream, d, s, rows);
  return pim::report_cuda(cudaGetLastError(), "pim_aten_mean_last");
}

int pim_aten_arange(const pim_tensor_view* dst, double start, double step, void* stream) {
  if (!valid(dst)) return pim::report_status(PIM_EINVAL, "pim_aten_arange: bad view");
  const pim::View d = pim::to_view(*dst);
  const long long n = pim::numel(d);
  if (n == 0) return PIM_OK;
  pim::launch_plain(pim::arange_kernel, dim3(pim::grid_for(n)), dim3(256), 0, (cudaStream_t)stream, d, start, step, n);
  return pim::report_cuda(cudaGetLastError(), "pim_aten_arange");
}

int pim_aten_matmul(const pim_tensor_view* dst, const pim_tensor_view* a, const pim_tensor_view* b, void* stream) {
  if (!valid(dst) || !valid(a) || !valid(b) || dst->ndim < 2 || a->ndim != dst->ndim || b->ndim != dst->ndim)
    return pim::report_status(PIM_EINVAL, "pim_aten_matmul: bad views");
  const int nd = dst->ndim;
  if (a->shape[nd - 2] != dst->shape[nd - 2] || b->shape[nd - 1] != dst->shape[nd - 1] ||
      a->shape[nd - 1] != b->shape[nd - 2])
    return pim::report_status(PIM_EINVAL, "pim_aten_matmul: shapes");
  for (int i = 0; i < nd - 2; ++i)
    if ((a->shape[i] != dst->shape[i] && a->shape[i] != 1) || (b->shape[i] != dst->shape[i] && b->shape[i] != 1))
      return pim::report_status(PIM_EINVAL, "pim_aten_matmul: batch dims");
  const pim::View d = pim::to_view(*dst), x = pim::to_view(*a), y = pim::to_view(*b);
  const long long n = pim::numel(d);
  if (n == 0) return PIM_OK;
  pim::launch_plain(pim::matmul_kernel, dim3(pim::grid_for(n)), dim3(256), 0, (cudaStream_t)stream, d, x, y, n);
  return pim::report_cuda(cudaGetLastError(), "pim_aten_matmul");
}

int pim_aten_sdpa(const pim_tensor_view* out, const pim_tensor_view* q, const pim_tensor_view* k,
                  const pim_tensor_view* v, const pim_tensor_view* mask, double scale, int32_t causal, void* stream) {
  if (!valid(out) || !valid(q) || !valid(k) || !valid(v) || q->ndim != 4 || k->ndim != 4 || v->ndim != 4 ||
      out->ndim != 4)
    return pim::report_status(PIM_EINVAL, "pim_aten_sdpa: q, k, v and out must be 4-d views");
  if (k->shape[2] > pim::kSdpaMaxKeys || k->shape[1] <= 0 || q->shape[1] % k->shape[1] ||
      k->shape[3] != q->shape[3] || v->shape[2] != k->shape[2] || q->shape[2] > k->shape[2])
    return pim::report_status(PIM_EINVAL, "pim_aten_sdpa: shapes (at most 8192 keys)");
  const bool has_mask = mask != nullptr && mask->data != nullptr;
  if (has_mask && (!valid(mask) || mask->ndim != 4))
    return pim::report_status(PIM_EINVAL, "pim_aten_sdpa: the mask must be a 4-d view");
  pim::View mv{};
  if (has_mask) mv = pim::to_view(*mask);
  const pim::View o = pim::to_view(*out), qv = pim::to_view(*q), kv = pim::to_view(*k), vv = pim::to_view(*v);
  const long long rows = q->shape[0] * q->shape[1] * q->shape[2];
  if (rows == 0) return PIM_OK;
  pim::launch_plain(pim::sdpa_kernel, dim3((unsigned)rows), dim3(pim::kSdpaThreads), 0, (cudaStream_t)stream, o, qv,
                    kv, vv, mv, has_mask ? 1 : 0, (float)scale, (int)causal);
  return pim::report_cuda(cudaGetLastError(), "pim_aten_sdpa");
}

int pim_aten_embedding(const pim_tensor_view* out, const pim_tensor_view* table, const pim_tensor_view* ids,
                       int32_t* err_flag, void* stream) {
  if (!valid(out) || !valid(table) || !valid(ids) || table->ndim != 2 || ids->dtype == PIM_F32 ||
      ids->dtype == PIM_BF16)
    return pim::report_status(PIM_EINVAL, "pim_aten_embedding: bad views");
  const pim::View o = pim::to_view(*out), t = pim::to_view(*table), i = pim::to_view(*ids);
  const long long n = pim::numel(i);
  if (n == 0) return PIM_OK;
  pim::launch_plain(pim::gather_rows_kernel, dim3((unsigned)(n < 148 * 8 ? n : 148 * 8)), dim3(256), 0,
                    (cudaStream_t)stream, o, t, i, n, err_flag);
  return pim::report_cuda(cudaGetLastError(), "pim_aten_embedding");
}

}  // extern "C"
