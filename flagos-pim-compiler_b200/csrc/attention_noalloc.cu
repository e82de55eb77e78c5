// pim_attention_noalloc: the attention entry point for callers that cannot allocate.
//
// pim_attention asks its caller for a workspace.  Some callers have no way to
// provide one: a plugin loaded into a host program whose device memory belongs to
// that program's own pool allocator (it must not call cudaMalloc behind the pool's
// back), or code on a latency-critical path where a cudaMalloc would synchronize the
// device.  This variant allocates nothing: its workspace is the fixed array below.
//
// * The array is a file-scope __device__ variable of PIM_ATTENTION_NOALLOC_SCRATCH_BYTES
//   (4 MiB).  Every GPU that loads the library holds it until the process exits.
// * Host code cannot use the array's name as a device address (on the host it names
//   a host-side stand-in), so the first call on each device, with that device
//   current, asks cudaGetSymbolAddress for the real address and caches it together
//   with the CUDA context that was current.  A call made under another context (a
//   non-primary context of the same device) asks again.  That first call should
//   come before any stream capture.  A device reset (cudaDeviceReset) after the first
//   call is not supported: the recreated context can carry the same handle, and the
//   cached address would then be stale.
// * Only the split-K kernel uses a workspace.  Shapes that run on it and need more
//   than the array are rejected with PIM_EINVAL; shapes that run on the tensor-core
//   row-batch kernels (bf16, head_dim 128, 16 or more query rows per sequence) use no
//   workspace and are accepted at any size.
// * Every call shares the array and it keeps the last call's contents: the per-row
//   tickets the split-K kernel counts with are cleared (cudaMemsetAsync on the call's
//   stream) before each launch.  Calls that overlap on the GPU -- on different
//   streams, or from different threads on one device -- race on the array.

#include <math.h>
#include <stdio.h>

#include <mutex>

#include "pim_b200.h"
#include "pim_common.cuh"
#include "pim_kernels.h"

namespace pim {
int report_status(int code, const char* msg);
int report_cuda(cudaError_t e, const char* what);
}  // namespace pim

namespace {

static __device__ __align__(256) unsigned char g_attention_scratch[PIM_ATTENTION_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
struct ScratchSlot {
  void* ctx;   // the CUDA context current when the address was taken
  void* addr;  // device address of g_attention_scratch in that context
};
ScratchSlot g_scratch[kMaxDevices] = {};

// cuCtxGetCurrent through the runtime's driver entry point (the library links only
// libcudart); null when the driver does not provide it.
typedef int (*CtxGetCurrentFn)(void**);
CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 4000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<CtxGetCurrentFn>(p);
    return static_cast<CtxGetCurrentFn>(nullptr);
  }();
  return fn;
}

}  // namespace

extern "C" int pim_attention_noalloc(const void* q, const int32_t* positions, const void* kv_base,
                                     int64_t kv_block_stride, int64_t kv_seq_stride, void* out, int32_t batch,
                                     int32_t seq, int32_t q_heads, int32_t kv_heads, int32_t head_dim,
                                     int32_t max_seq, int32_t dtype, void* stream) {
  if (!q || !positions || !kv_base || !out)
    return pim::report_status(PIM_EINVAL, "pim_attention_noalloc: null pointer");
  if (dtype != PIM_F32 && dtype != PIM_BF16) return pim::report_status(PIM_EINVAL, "pim_attention_noalloc: bad dtype");
  if (batch <= 0 || seq <= 0 || q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads || max_seq <= 0)
    return pim::report_status(PIM_EINVAL, "pim_attention_noalloc: bad geometry");
  if (head_dim != 32 && head_dim != 64 && head_dim != 128)
    return pim::report_status(PIM_EUNSUPPORTED, "pim_attention_noalloc: head_dim must be 32, 64 or 128");
  pim::AttnArgs a{};
  a.q = q;
  a.positions = positions;
  a.kv_base = kv_base;
  a.block_stride = kv_block_stride;
  a.seq_stride = kv_seq_stride;
  a.out = out;
  a.batch = batch;
  a.seq = seq;
  a.hq = q_heads;
  a.hkv = kv_heads;
  a.hd = head_dim;
  a.max_seq = max_seq;
  a.scale = (float)(1.0 / sqrt((double)head_dim));
  const bool uses_ws = pim::attention_uses_workspace(a, dtype);
  const size_t need = pim::attention_workspace_bytes(a);
  if (uses_ws && need > (size_t)PIM_ATTENTION_NOALLOC_SCRATCH_BYTES)
    return pim::report_status(PIM_EINVAL,
                              "pim_attention_noalloc: this shape needs more workspace than the fixed 4 MiB "
                              "scratch; use pim_attention with a caller workspace");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return pim::report_cuda(e, "pim_attention_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return pim::report_status(PIM_EUNSUPPORTED, "pim_attention_noalloc: device id");
  void* ctx = nullptr;
  if (CtxGetCurrentFn fn = ctx_get_current()) {
    if (fn(&ctx) != 0) return pim::report_status(PIM_ECUDA, "pim_attention_noalloc: cuCtxGetCurrent failed");
  }
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch[dev].addr || g_scratch[dev].ctx != ctx) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_attention_scratch);
      if (e != cudaSuccess) return pim::report_cuda(e, "pim_attention_noalloc: cudaGetSymbolAddress");
      // the lookup made the runtime's context current if none was: key the cache on that one
      if (CtxGetCurrentFn fn = ctx_get_current()) {
        if (fn(&ctx) != 0) return pim::report_status(PIM_ECUDA, "pim_attention_noalloc: cuCtxGetCurrent failed");
      }
      g_scratch[dev] = ScratchSlot{ctx, p};
    }
    scratch = g_scratch[dev].addr;
  }
  if (uses_ws) {
    // The workspace ends with one ticket (int) per query row; they must start at zero.
    const size_t rows = (size_t)batch * seq * q_heads;
    e = cudaMemsetAsync(static_cast<char*>(scratch) + need - rows * sizeof(int), 0, rows * sizeof(int),
                        (cudaStream_t)stream);
    if (e != cudaSuccess) return pim::report_cuda(e, "pim_attention_noalloc: clearing tickets");
  }
  return pim::report_cuda(pim::attention(a, dtype, scratch, (size_t)PIM_ATTENTION_NOALLOC_SCRATCH_BYTES,
                                         (cudaStream_t)stream),
                          "pim_attention_noalloc");
}
