// Shared device helpers for the B200 ExecutionPlan kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

namespace pim {

enum DType : int { F32 = 0, BF16 = 1, I32 = 2 };

constexpr int kWarp = 32;

__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ float from_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// Round an fp32 value to the storage precision of T and back (identity for fp32).
template <typename T>
__device__ __forceinline__ float rnd(float x) { return to_f(from_f<T>(x)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// 16-byte streaming load that bypasses L1 allocation: weights are read once per step.
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte load cached in L2 only: for data another grid wrote while this one may
// already have been running (programmatic dependent launch), read after pdl_wait().
__device__ __forceinline__ int4 ld_l2(const int4* p) {
  int4 r;
  asm volatile("ld.global.cg.v4.s32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

__device__ __forceinline__ int4 ld_stream(const int4* p) {
  int4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Elements of T per 16-byte vector.
template <typename T>
struct VecW {
  static constexpr int n = 16 / sizeof(T);
};

// Unpack a 16-byte vector into fp32 values.
__device__ __forceinline__ void unpack(const int4& v, float (&f)[4], float) {
  f[0] = __int_as_float(v.x);
  f[1] = __int_as_float(v.y);
  f[2] = __int_as_float(v.z);
  f[3] = __int_as_float(v.w);
}

__device__ __forceinline__ void unpack(const int4& v, float (&f)[8], __nv_bfloat16) {
  const uint32_t w[4] = {(uint32_t)v.x, (uint32_t)v.y, (uint32_t)v.z, (uint32_t)v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// Pack fp32 values (already representable in the element type) into a 16-byte vector.
__device__ __forceinline__ int4 pack(const float (&f)[4], float) {
  return make_int4(__float_as_int(f[0]), __float_as_int(f[1]), __float_as_int(f[2]), __float_as_int(f[3]));
}

__device__ __forceinline__ int4 pack(const float (&f)[8], __nv_bfloat16) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    w[i] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(f[2 * i])) |
           ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(f[2 * i + 1])) << 16);
  return make_int4((int)w[0], (int)w[1], (int)w[2], (int)w[3]);
}

template <typename T>
constexpr bool kIsBf16 = false;
template <>
constexpr bool kIsBf16<__nv_bfloat16> = true;

// acc + sum of the 8 bf16 products w[e] * x[e], accumulated in element order (low then
// high half of each 32-bit word).  Each step is one mixed-precision fma.rn.f32.bf16:
// the product of two bf16 values is exact in fp32 and the sum is rounded once, so the
// result equals fmaf(float(w[e]), float(x[e]), acc) step by step, without unpacking.
__device__ __forceinline__ float fma8_bf16(const int4& w, const int4& x, float acc) {
  asm("{\n"
      " .reg .b16 w0, w1, w2, w3, w4, w5, w6, w7, x0, x1, x2, x3, x4, x5, x6, x7;\n"
      " mov.b32 {w0, w1}, %1;\n mov.b32 {w2, w3}, %2;\n mov.b32 {w4, w5}, %3;\n mov.b32 {w6, w7}, %4;\n"
      " mov.b32 {x0, x1}, %5;\n mov.b32 {x2, x3}, %6;\n mov.b32 {x4, x5}, %7;\n mov.b32 {x6, x7}, %8;\n"
      " fma.rn.f32.bf16 %0, w0, x0, %0;\n fma.rn.f32.bf16 %0, w1, x1, %0;\n"
      " fma.rn.f32.bf16 %0, w2, x2, %0;\n fma.rn.f32.bf16 %0, w3, x3, %0;\n"
      " fma.rn.f32.bf16 %0, w4, x4, %0;\n fma.rn.f32.bf16 %0, w5, x5, %0;\n"
      " fma.rn.f32.bf16 %0, w6, x6, %0;\n fma.rn.f32.bf16 %0, w7, x7, %0;\n"
      "}"
      : "+f"(acc)
      : "r"(w.x), "r"(w.y), "r"(w.z), "r"(w.w), "r"(x.x), "r"(x.y), "r"(x.z), "r"(x.w));
  return acc;
}

inline int ceil_div(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

// Programmatic dependent launch.  A kernel launched with launch_pdl() may start
// while its predecessor in the stream is still running: it must call pdl_wait()
// before reading the predecessor's outputs or writing anything the predecessor
// reads.  pdl_trigger() lets the successor launch once every CTA of this grid
// has started.  Both are no-ops for an ordinary launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// PDL is on unless PIM_PDL=0 is set in the environment.
bool pdl_enabled();

// How many CTAs of `kern` (`threads` threads, `smem` bytes of dynamic shared memory) an
// SM holds at once, as the launch will see it: first (once per device) the kernel asks
// for the largest shared-memory carveout and its dynamic shared-memory limit is raised
// to the largest size seen -- so that launches recorded in a stream capture make no
// attribute calls after the first eager run -- then the occupancy API answers (the last
// 16 sizes are cached, more than any plan uses per kernel, so a capture that follows an
// eager run of its plan queries nothing).  Returns -1 with the CUDA error in *err on failure.
struct ResidentCache {
  size_t attr_bytes[64] = {};
  bool carveout[64] = {};
  size_t smem[64][16] = {};
  int ctas[64][16] = {};
  int next[64] = {};
};

template <typename Kern>
int resident_ctas(Kern kern, int threads, size_t smem, ResidentCache& c, cudaError_t* err) {
  int dev = 0;
  *err = cudaGetDevice(&dev);
  if (*err != cudaSuccess) return -1;
  if (dev >= 64) {
    *err = cudaErrorInvalidDevice;
    return -1;
  }
  if (!c.carveout[dev]) {
    *err = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                (int)cudaSharedmemCarveoutMaxShared);
    if (*err != cudaSuccess) return -1;
    c.carveout[dev] = true;
  }
  if (c.attr_bytes[dev] < smem) {
    *err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (*err != cudaSuccess) return -1;
    c.attr_bytes[dev] = smem;
  }
  for (int i = 0; i < 16; ++i)
    if (c.smem[dev][i] == smem && c.ctas[dev][i] > 0) return c.ctas[dev][i];
  int n = 0;
  *err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, threads, smem);
  if (*err != cudaSuccess) return -1;
  const int slot = c.next[dev]++ & 15;
  c.smem[dev][slot] = smem;
  c.ctas[dev][slot] = n;
  return n;
}

// Counts one kernel launch of this library (process-wide, every device and stream);
// every launch goes through launch_pdl() or launch_plain(), which call it.
void count_launch();
uint64_t launches_so_far();

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e == cudaSuccess) count_launch();
  return e;
}

// Whether this device accepts a cooperative launch that also carries programmatic
// stream serialization: 1 yes, 0 no, -1 not known yet.  Settled by the first cooperative
// launch on the device made outside a stream capture (a refused launch inside a capture
// could invalidate it, so captures use the plain cooperative form until then).
int coop_pdl_state(int dev);
void set_coop_pdl_state(int dev, int ok);

// A launch whose CTAs wait on one another (grid-wide barriers, a grid-wide wait for peer
// flags): cooperative, so the driver either makes every CTA of the grid resident at
// once or refuses the launch (cudaErrorCooperativeLaunchTooLarge) -- a grid that cannot
// be co-resident fails loudly instead of spinning out its bounded waits.  It also asks
// for programmatic dependent launch where the device accepts the two together.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_coop(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                               Args&&... args) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  e = cudaStreamIsCapturing(st, &cap);
  if (e != cudaSuccess) return e;
  const int state = coop_pdl_state(dev);
  const bool try_pdl = pdl_enabled() && (state == 1 || (state < 0 && cap == cudaStreamCaptureStatusNone));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = try_pdl ? 2 : 1;
  e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (try_pdl && state < 0) {
    set_coop_pdl_state(dev, e == cudaSuccess ? 1 : 0);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();  // the refused combination; retry as a plain cooperative launch
      cfg.numAttrs = 1;
      e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
    }
  }
  if (e == cudaSuccess) count_launch();
  return e;
}

// An ordinary launch (no programmatic dependent launch).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_plain(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e == cudaSuccess) count_launch();
  return e;
}

}  // namespace pim
