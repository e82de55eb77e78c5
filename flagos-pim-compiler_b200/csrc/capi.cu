// extern "C" entry points declared in include/pim_b200.h: argument checks, then the
// launches of the kernels in gemv.cu / attention.cu / elementwise.cu / comm.cu.

#include <math.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <vector>

#include "pim_b200.h"
#include "pim_common.cuh"
#include "pim_kernels.h"

namespace pim {
cudaError_t embedding(const int* ids, const void* table, void* out, int n_ids, int hidden, int vocab, int dtype,
                      int* err, cudaStream_t st);
cudaError_t add(const void* a, const void* b, void* y, int64_t n, int dtype, cudaStream_t st);
cudaError_t select_rows(const void* x, void* out, int batch, int seq, int64_t row_bytes, int index, cudaStream_t st);
cudaError_t argmax(const void* x, int* out, int rows, int n, int dtype, cudaStream_t st);
cudaError_t fill_normal(void* out, int64_t n, int dtype, uint64_t seed, float std, cudaStream_t st);
cudaError_t fill_const(void* out, int64_t n, int dtype, float v, cudaStream_t st);
cudaError_t ordered_sum(const void* const* src, int nsrc, void* const* dst, int ndst, int64_t n, int dtype, int mean,
                        cudaStream_t st);
cudaError_t ordered_sum_add(const void* const* src, int nsrc, const void* res, void* y, void* sum_out, int64_t n,
                            int dtype, cudaStream_t st);
cudaError_t batched_copy(const void* desc_dev, int count, int64_t max_nbytes, cudaStream_t st);

static std::atomic<uint64_t> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
uint64_t launches_so_far() { return g_launches.load(std::memory_order_relaxed); }

// Per device: whether a cooperative launch may also carry programmatic stream
// serialization (-1 not known yet, 0 no, 1 yes).
static std::atomic<int>* coop_pdl_table() {
  static std::atomic<int> t[64];
  static const bool init = [] {
    for (auto& v : t) v.store(-1, std::memory_order_relaxed);
    return true;
  }();
  (void)init;
  return t;
}
int coop_pdl_state(int dev) { return (dev < 0 || dev >= 64) ? 0 : coop_pdl_table()[dev].load(std::memory_order_relaxed); }
void set_coop_pdl_state(int dev, int ok) {
  if (dev >= 0 && dev < 64) coop_pdl_table()[dev].store(ok, std::memory_order_relaxed);
}
}  // namespace pim

static thread_local char g_err[512];

static int fail(int code, const char* msg) {
  snprintf(g_err, sizeof(g_err), "%s", msg);
  return code;
}

static int check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return PIM_OK;
  snprintf(g_err, sizeof(g_err), "%s: %s", what, cudaGetErrorString(e));
  return e == cudaErrorNotSupported ? PIM_EUNSUPPORTED : PIM_ECUDA;
}

static bool dtype_ok(int32_t d) { return d == PIM_F32 || d == PIM_BF16; }

namespace pim {
// Status reporting for entry points defined in other .cu files (same pim_last_error()).
int report_status(int code, const char* msg) { return fail(code, msg); }
int report_cuda(cudaError_t e, const char* what) { return check(e, what); }
}  // namespace pim

static pim::FusedArgs to_fused(const pim_projection_args* a) {
  pim::FusedArgs f{};
  f.x = a->x;
  f.ln_w = a->norm_weight;
  f.w = a->weight;
  f.y = a->out;
  f.rows = (int)a->rows;
  f.K = (int)a->k;
  f.ncols = (int)a->ncols;
  f.eps = a->eps;
  f.cos = a->rope_cos;
  f.sin = a->rope_sin;
  f.positions = a->positions;
  f.seq = a->seq;
  f.hq = a->q_heads;
  f.hkv = a->kv_heads;
  f.hd = a->head_dim;
  f.kv_base = a->kv_base;
  f.block_stride = a->kv_block_stride;
  f.seq_stride = a->kv_seq_stride;
  f.max_seq = a->max_seq;
  f.inter = a->inter;
  f.residual = a->residual;
  f.err = a->err_flag;
  f.p2p = a->p2p_desc;
  f.ar_out = a->allreduce_out;
  f.attn_out = a->attn_out;
  f.attn_cnt = a->attn_counters;
  return f;
}

extern "C" {

int pim_abi_version(void) { return PIM_ABI_VERSION; }

uint64_t pim_kernel_launches(void) { return pim::launches_so_far(); }

int pim_cooperative_pdl(int32_t device) { return pim::coop_pdl_state(device); }

const char* pim_last_error(void) { return g_err; }

int pim_enable_peer_access(int32_t device, int32_t peer) {
  int can = 0;
  cudaError_t e = cudaDeviceCanAccessPeer(&can, device, peer);
  if (e != cudaSuccess) return check(e, "cudaDeviceCanAccessPeer");
  if (!can) return fail(PIM_EUNSUPPORTED, "device cannot access peer");
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  e = cudaDeviceEnablePeerAccess(peer, 0);
  cudaSetDevice(prev);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    return PIM_OK;
  }
  return check(e, "cudaDeviceEnablePeerAccess");
}

int64_t pim_projection_scratch_bytes(const pim_projection_args* a, int32_t dtype, int32_t mode) {
  if (!a) return -1;
  return (int64_t)pim::fused_scratch_bytes(to_fused(a), dtype, mode);
}

int pim_set_projection_kernel(int32_t kernel) {
  if (kernel != PIM_PROJ_KERNEL_REGISTER && kernel != PIM_PROJ_KERNEL_STAGED && kernel != PIM_PROJ_KERNEL_DYNAMIC)
    return fail(PIM_EINVAL, "pim_set_projection_kernel: unknown kernel");
  pim::set_gemv_variant(kernel);
  return PIM_OK;
}

int32_t pim_projection_kernel(void) { return pim::gemv_variant(); }

int pim_set_row_batch_kernel(int32_t kernel) {
  if (kernel != PIM_ROW_BATCH_KERNEL_TILE && kernel != PIM_ROW_BATCH_KERNEL_PERSISTENT)
    return fail(PIM_EINVAL, "pim_set_row_batch_kernel: unknown kernel");
  pim::set_gemm_kernel(kernel);
  return PIM_OK;
}

int32_t pim_row_batch_kernel(void) { return pim::gemm_kernel(); }

int pim_projection(const pim_projection_args* a, int32_t dtype, int32_t mode, void* scratch, int64_t scratch_bytes,
                   void* stream) {
  if (!a || !a->x || !a->weight || !a->out) return fail(PIM_EINVAL, "pim_projection: null pointer");
  if (!dtype_ok(dtype)) return fail(PIM_EINVAL, "pim_projection: bad dtype");
  if (mode < 0 || mode > 2) return fail(PIM_EINVAL, "pim_projection: bad mode");
  if (a->rows <= 0 || a->k <= 0 || a->rows > (1 << 30) || a->k > (1 << 30))
    return fail(PIM_EINVAL, "pim_projection: bad rows/k");
  if (mode == PIM_PROJ_PLAIN && a->ncols <= 0) return fail(PIM_EINVAL, "pim_projection: bad ncols");
  if (mode == PIM_PROJ_ROPE_KV) {
    if (!a->rope_cos || !a->rope_sin || !a->positions || !a->kv_base)
      return fail(PIM_EINVAL, "pim_projection: ROPE_KV needs cos/sin/positions/kv_base");
    if (a->head_dim <= 0 || a->head_dim % 2 || a->q_heads <= 0 || a->kv_heads <= 0 || a->seq <= 0 ||
        a->rows % a->seq || a->max_seq <= 0)
      return fail(PIM_EINVAL, "pim_projection: bad head geometry");
  }
  if (mode == PIM_PROJ_SILU_MUL && a->inter <= 0) return fail(PIM_EINVAL, "pim_projection: bad inter");
  if (a->residual && mode != PIM_PROJ_PLAIN) return fail(PIM_EINVAL, "pim_projection: residual needs mode PLAIN");
  if (a->p2p_desc && (mode != PIM_PROJ_PLAIN || a->norm_weight || a->rows > 8))
    return fail(PIM_EINVAL, "pim_projection: the fused all-reduce needs mode PLAIN, no norm, rows <= 8");
  if (a->attn_out && (mode != PIM_PROJ_ROPE_KV || a->rows > 8 || !a->attn_counters || a->q_heads > 64 ||
                      (a->head_dim != 64 && a->head_dim != 128) || a->q_heads % a->kv_heads))
    return fail(PIM_EINVAL,
                "pim_projection: fused attention needs mode ROPE_KV, rows <= 8, attn_counters, q_heads <= 64, "
                "head_dim 64 or 128");
  const pim::FusedArgs f = to_fused(a);
  const size_t need = pim::fused_scratch_bytes(f, dtype, mode);
  if (a->rows > pim::kGemvMaxRows && need > 0 && (!scratch || scratch_bytes < (int64_t)need))
    return fail(PIM_EINVAL, "pim_projection: scratch too small");
  // Decode rows: the scratch is optional (the dynamic kernel's work counter).
  if (a->rows <= pim::kGemvMaxRows && (!scratch || scratch_bytes < (int64_t)pim::kGemvCounterBytes ||
                                       (uintptr_t)scratch % 16))
    scratch = nullptr;
  if (a->rows <= pim::kGemvMaxRows && (size_t)a->rows * a->k * (dtype == PIM_BF16 ? 2 : 4) > 200 * 1024)
    return fail(PIM_EUNSUPPORTED, "pim_projection: activation rows exceed shared memory");
  return check(pim::fused_projection(f, dtype, mode, a->norm_weight != nullptr, scratch, (cudaStream_t)stream),
               "pim_projection");
}

}  // extern "C"

// Checks of one decode layer's four projections for the layer kernel (pim_decode_layer,
// pim_decode_step_prepare); `who` prefixes the message.
static int layer_status(const pim_projection_args* const ph[4], int64_t es, const char* who) {
  char msg[256];
  auto bad = [&](const char* what) {
    snprintf(msg, sizeof(msg), "%s: %s", who, what);
    return fail(PIM_EINVAL, msg);
  };
  for (int i = 0; i < 4; ++i)
    if (!ph[i]) return bad("null pointer");
  for (int i = 0; i < 4; ++i) {
    const pim_projection_args* a = ph[i];
    if (!a->x || !a->weight || !a->out) return bad("null x/weight/out");
    if (a->rows != 1) return bad("one activation row per phase");
    if (a->k <= 0 || (a->k * es) % 16 || a->k > (1 << 20)) return bad("bad k");
    if ((uintptr_t)a->x % 16 || (uintptr_t)a->weight % 16 || (uintptr_t)a->norm_weight % 16)
      return bad("x, weight and norm_weight must be 16-byte aligned");
    if ((i == 0 || i == 2) && (a->p2p_desc || a->allreduce_out)) return bad("only o_proj and down take a p2p_desc");
    if (a->allreduce_out && !a->p2p_desc) return bad("allreduce_out needs p2p_desc");
    if ((i == 0 || i == 2) != (a->norm_weight != nullptr))
      return bad("attn_in and mlp_in take a norm_weight, o_proj and down none");
    if ((i == 0 || i == 2) && a->residual) return bad("residual needs mode PLAIN");
    if (i != 0 && a->attn_out) return bad("attn_out belongs to attn_in");
  }
  const pim_projection_args *a = ph[0], *o_proj = ph[1], *mlp_in = ph[2], *down = ph[3];
  if (!a->rope_cos || !a->rope_sin || !a->positions || !a->kv_base || !a->attn_out || !a->attn_counters)
    return bad("attn_in needs cos/sin/positions/kv_base/attn_out/attn_counters");
  if ((a->head_dim != 64 && a->head_dim != 128) || a->q_heads <= 0 || a->kv_heads <= 0 ||
      a->q_heads > pim::kFusedAttnMaxHeads || a->q_heads % a->kv_heads || a->seq != 1 || a->max_seq <= 0)
    return bad("bad head geometry (head_dim 64/128, q_heads <= 64, seq 1)");
  const int64_t qw = (int64_t)a->q_heads * a->head_dim;
  if (o_proj->x != a->attn_out || o_proj->k != qw) return bad("o_proj must read attn_in's attention output");
  if (o_proj->ncols <= 0 || mlp_in->x != o_proj->out || mlp_in->k != o_proj->ncols)
    return bad("mlp_in must read o_proj's output");
  if (mlp_in->inter <= 0 || down->x != mlp_in->out || down->k != mlp_in->inter)
    return bad("down must read mlp_in's output");
  if (down->ncols <= 0) return bad("bad ncols");
  if (o_proj->p2p_desc != down->p2p_desc) return bad("o_proj and down take the same p2p_desc, or none");
  return PIM_OK;
}

extern "C" {

int pim_decode_layer(const pim_projection_args* attn_in, const pim_projection_args* o_proj,
                     const pim_projection_args* mlp_in, const pim_projection_args* down, void* barrier,
                     int32_t* err_flag, int32_t dtype, void* stream) {
  const pim_projection_args* const ph[4] = {attn_in, o_proj, mlp_in, down};
  if (!dtype_ok(dtype)) return fail(PIM_EINVAL, "pim_decode_layer: bad dtype");
  const int rc = layer_status(ph, dtype == PIM_BF16 ? 2 : 4, "pim_decode_layer");
  if (rc != PIM_OK) return rc;
  if (!barrier) return fail(PIM_EINVAL, "pim_decode_layer: null barrier");
  if ((uintptr_t)barrier % 16) return fail(PIM_EINVAL, "pim_decode_layer: barrier must be 16-byte aligned");
  return check(pim::decode_layer(to_fused(attn_in), to_fused(o_proj), to_fused(mlp_in), to_fused(down),
                                 static_cast<unsigned*>(barrier), err_flag, dtype, (cudaStream_t)stream),
               "pim_decode_layer");
}

int64_t pim_decode_step_table_bytes(int32_t nlayers) {
  return nlayers > 0 ? (int64_t)pim::decode_step_table_bytes(nlayers) : -1;
}

int pim_decode_step_prepare(const pim_projection_args* const* layers, int32_t nlayers,
                            const pim_projection_args* head, int32_t dtype, void* table, int64_t table_bytes,
                            pim_decode_step_plan** plan) {
  if (!layers || !plan || nlayers <= 0 || nlayers > 4096)
    return fail(PIM_EINVAL, "pim_decode_step_prepare: bad arguments");
  *plan = nullptr;
  if (!dtype_ok(dtype)) return fail(PIM_EINVAL, "pim_decode_step_prepare: bad dtype");
  const int64_t es = dtype == PIM_BF16 ? 2 : 4;
  for (int l = 0; l < nlayers; ++l) {
    const int rc = layer_status(layers + 4 * l, es, "pim_decode_step_prepare");
    if (rc != PIM_OK) return rc;
    if (l > 0 && layers[4 * l]->x != layers[4 * l - 1]->out)
      return fail(PIM_EINVAL, "pim_decode_step_prepare: a layer must read the previous layer's output");
    if (layers[4 * l + 1]->p2p_desc != layers[1]->p2p_desc)
      return fail(PIM_EINVAL, "pim_decode_step_prepare: every layer takes the same p2p_desc, or none");
  }
  const pim_projection_args* last = layers[4 * nlayers - 1];
  if (head) {
    if (!head->x || !head->weight || !head->out || !head->norm_weight || head->rows != 1 || head->ncols <= 0 ||
        head->k != last->ncols || head->x != last->out)
      return fail(PIM_EINVAL, "pim_decode_step_prepare: the head takes the last layer's output, a norm_weight, "
                              "one row, ncols > 0");
    if (head->residual || head->p2p_desc || head->attn_out || (head->k * es) % 16 || (uintptr_t)head->x % 16 ||
        (uintptr_t)head->weight % 16 || (uintptr_t)head->norm_weight % 16)
      return fail(PIM_EINVAL, "pim_decode_step_prepare: the head is a plain aligned projection");
  }
  if (!table || (uintptr_t)table % 16 || table_bytes < (int64_t)pim::decode_step_table_bytes(nlayers))
    return fail(PIM_EINVAL, "pim_decode_step_prepare: table too small or not 16-byte aligned");
  std::vector<pim::FusedArgs> f(4 * (size_t)nlayers);
  for (int i = 0; i < 4 * nlayers; ++i) f[i] = to_fused(layers[i]);
  const pim::FusedArgs hf = head ? to_fused(head) : pim::FusedArgs{};
  return check(pim::decode_step_prepare(f.data(), nlayers, head ? &hf : nullptr, dtype, table, (size_t)table_bytes,
                                        plan),
               "pim_decode_step_prepare");
}

int pim_decode_step(const pim_decode_step_plan* plan, void* barrier, int32_t* err_flag, void* stream) {
  if (!plan || !barrier || (uintptr_t)barrier % 16) return fail(PIM_EINVAL, "pim_decode_step: bad arguments");
  return check(pim::decode_step(plan, static_cast<unsigned*>(barrier), err_flag, (cudaStream_t)stream),
               "pim_decode_step");
}

void pim_decode_step_free(pim_decode_step_plan* plan) { pim::decode_step_free(plan); }

int64_t pim_attention_workspace_bytes(int32_t batch, int32_t seq, int32_t q_heads, int32_t head_dim,
                                      int32_t max_seq) {
  pim::AttnArgs a{};
  a.batch = batch;
  a.seq = seq;
  a.hq = q_heads;
  a.hd = head_dim;
  a.max_seq = max_seq;
  return (int64_t)pim::attention_workspace_bytes(a);
}

int pim_attention(const void* q, const int32_t* positions, const void* kv_base, int64_t kv_block_stride,
                  int64_t kv_seq_stride, void* out, int32_t batch, int32_t seq, int32_t q_heads, int32_t kv_heads,
                  int32_t head_dim, int32_t max_seq, int32_t dtype, void* workspace, int64_t workspace_bytes,
                  void* stream) {
  if (!q || !positions || !kv_base || !out || !workspace) return fail(PIM_EINVAL, "pim_attention: null pointer");
  if (!dtype_ok(dtype)) return fail(PIM_EINVAL, "pim_attention: bad dtype");
  if (batch <= 0 || seq <= 0 || q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads || max_seq <= 0)
    return fail(PIM_EINVAL, "pim_attention: bad geometry");
  if (head_dim != 32 && head_dim != 64 && head_dim != 128)
    return fail(PIM_EUNSUPPORTED, "pim_attention: head_dim must be 32, 64 or 128");
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
  if ((int64_t)pim::attention_workspace_bytes(a) > workspace_bytes)
    return fail(PIM_EINVAL, "pim_attention: workspace too small");
  return check(pim::attention(a, dtype, workspace, (size_t)workspace_bytes, (cudaStream_t)stream), "pim_attention");
}

int32_t pim_attention_errors(int32_t reset) { return pim::attention_tc_errors(reset != 0); }

int pim_set_prefill_attention_kernel(int32_t kernel) {
  if (kernel != PIM_PREFILL_ATTENTION_MMA && kernel != PIM_PREFILL_ATTENTION_TCGEN05)
    return fail(PIM_EINVAL, "pim_set_prefill_attention_kernel: unknown kernel");
  pim::set_prefill_attention_kernel(kernel);
  return PIM_OK;
}

int32_t pim_prefill_attention_kernel(void) { return pim::prefill_attention_kernel(); }

int pim_embedding(const int32_t* ids, const void* table, void* out, int64_t n_ids, int64_t hidden, int64_t vocab,
                  int32_t dtype, int32_t* err_flag, void* stream) {
  if (!ids || !table || !out || n_ids <= 0 || hidden <= 0 || vocab <= 0 || !dtype_ok(dtype))
    return fail(PIM_EINVAL, "pim_embedding: bad arguments");
  return check(pim::embedding(ids, table, out, (int)n_ids, (int)hidden, (int)vocab, dtype, err_flag,
                              (cudaStream_t)stream),
               "pim_embedding");
}

int pim_add(const void* a, const void* b, void* out, int64_t n, int32_t dtype, void* stream) {
  if (!a || !b || !out || n < 0 || !dtype_ok(dtype)) return fail(PIM_EINVAL, "pim_add: bad arguments");
  if (n == 0) return PIM_OK;
  return check(pim::add(a, b, out, n, dtype, (cudaStream_t)stream), "pim_add");
}

int pim_select_rows(const void* x, void* out, int32_t batch, int32_t seq, int64_t row_bytes, int32_t index,
                    void* stream) {
  if (!x || !out || batch <= 0 || seq <= 0 || index < 0 || index >= seq || row_bytes <= 0)
    return fail(PIM_EINVAL, "pim_select_rows: bad arguments");
  return check(pim::select_rows(x, out, batch, seq, row_bytes, index, (cudaStream_t)stream), "pim_select_rows");
}

int pim_argmax(const void* x, int32_t* out, int32_t rows, int64_t n, int32_t dtype, void* stream) {
  if (!x || !out || rows <= 0 || n <= 0 || n > (1ll << 31) - 1 || !dtype_ok(dtype))
    return fail(PIM_EINVAL, "pim_argmax: bad arguments");
  return check(pim::argmax(x, out, rows, (int)n, dtype, (cudaStream_t)stream), "pim_argmax");
}

int pim_copy(void* dst, const void* src, int64_t nbytes, void* stream) {
  if (nbytes < 0 || ((!dst || !src) && nbytes > 0)) return fail(PIM_EINVAL, "pim_copy: bad arguments");
  if (nbytes == 0) return PIM_OK;
  return check(cudaMemcpyAsync(dst, src, (size_t)nbytes, cudaMemcpyDefault, (cudaStream_t)stream), "pim_copy");
}

int pim_ordered_sum(const void* const* src, int32_t nsrc, void* const* dst, int32_t ndst, int64_t n, int32_t dtype,
                    int32_t mean, void* stream) {
  if (!src || !dst || nsrc < 1 || nsrc > 8 || ndst < 0 || ndst > 8 || n < 0 || !dtype_ok(dtype))
    return fail(PIM_EINVAL, "pim_ordered_sum: bad arguments");
  for (int i = 0; i < nsrc; ++i)
    if (!src[i]) return fail(PIM_EINVAL, "pim_ordered_sum: null source");
  for (int i = 0; i < ndst; ++i)
    if (!dst[i]) return fail(PIM_EINVAL, "pim_ordered_sum: null destination");
  return check(pim::ordered_sum(src, nsrc, dst, ndst, n, dtype, mean, (cudaStream_t)stream), "pim_ordered_sum");
}

int pim_ordered_sum_add(const void* const* src, int32_t nsrc, const void* residual, void* out, void* sum_out,
                        int64_t n, int32_t dtype, void* stream) {
  if (!src || nsrc < 1 || nsrc > 8 || !residual || !out || n < 0 || !dtype_ok(dtype))
    return fail(PIM_EINVAL, "pim_ordered_sum_add: bad arguments");
  for (int i = 0; i < nsrc; ++i)
    if (!src[i]) return fail(PIM_EINVAL, "pim_ordered_sum_add: null source");
  return check(pim::ordered_sum_add(src, nsrc, residual, out, sum_out, n, dtype, (cudaStream_t)stream),
               "pim_ordered_sum_add");
}

static int p2p_args(const char* who, const void* src, void* const* dsts, int32_t ndst, int64_t numel, int32_t dtype,
                    int32_t rank, int32_t size, void* const* bufs, int64_t capacity_bytes, int32_t* counter,
                    int32_t* err_flag, pim::P2PArgs* a) {
  char msg[160];
  if (!src || !bufs || !counter || (ndst > 0 && !dsts) || ndst < 0 || ndst > pim::kP2PMaxDst || size < 1 ||
      size > PIM_P2P_MAX_RANKS || rank < 0 || rank >= size || numel < 0 || capacity_bytes <= 0 || !dtype_ok(dtype)) {
    snprintf(msg, sizeof(msg), "%s: bad arguments", who);
    return fail(PIM_EINVAL, msg);
  }
  *a = pim::P2PArgs{};
  a->src = src;
  a->ndst = ndst;
  for (int i = 0; i < ndst; ++i) {
    if (!dsts[i]) {
      snprintf(msg, sizeof(msg), "%s: null destination", who);
      return fail(PIM_EINVAL, msg);
    }
    a->dst[i] = dsts[i];
  }
  for (int i = 0; i < size; ++i) {
    if (!bufs[i]) {
      snprintf(msg, sizeof(msg), "%s: null exchange buffer", who);
      return fail(PIM_EINVAL, msg);
    }
    a->bufs[i] = bufs[i];
  }
  a->numel = numel;
  a->rank = rank;
  a->size = size;
  a->capacity_bytes = capacity_bytes;
  a->counter = counter;
  a->err = err_flag;
  const int64_t es = dtype == PIM_BF16 ? 2 : 4;
  if ((numel * es) % 16 || numel * es > capacity_bytes) {
    snprintf(msg, sizeof(msg), "%s: numel * element size must be a multiple of 16 within capacity", who);
    return fail(PIM_EINVAL, msg);
  }
  return PIM_OK;
}

int pim_allreduce_p2p(const void* src, void* const* dsts, int32_t ndst, int64_t numel, int32_t dtype,
                      int32_t rank, int32_t size, void* const* bufs, int64_t capacity_bytes, int32_t* counter,
                      int32_t* err_flag, void* stream) {
  pim::P2PArgs a;
  const int rc = p2p_args("pim_allreduce_p2p", src, dsts, ndst, numel, dtype, rank, size, bufs, capacity_bytes,
                          counter, err_flag, &a);
  if (rc != PIM_OK || numel == 0) return rc;
  return check(pim::allreduce_p2p(a, dtype, (cudaStream_t)stream), "pim_allreduce_p2p");
}

int pim_allreduce_p2p_add(const void* src, const void* residual, void* y, void* sum_out, int64_t numel, int32_t dtype,
                          int32_t rank, int32_t size, void* const* bufs, int64_t capacity_bytes, int32_t* counter,
                          int32_t* err_flag, void* stream) {
  if (!residual || !y) return fail(PIM_EINVAL, "pim_allreduce_p2p_add: residual and y are required");
  void* dsts[1] = {sum_out};
  pim::P2PArgs a;
  const int rc = p2p_args("pim_allreduce_p2p_add", src, dsts, sum_out ? 1 : 0, numel, dtype, rank, size, bufs,
                          capacity_bytes, counter, err_flag, &a);
  if (rc != PIM_OK || numel == 0) return rc;
  a.residual = residual;
  a.y = y;
  return check(pim::allreduce_p2p(a, dtype, (cudaStream_t)stream), "pim_allreduce_p2p_add");
}

int pim_allreduce_p2p_ll(const void* src, const void* residual, void* y, void* sum_out, int64_t numel, int32_t dtype,
                         int32_t rank, int32_t size, void* const* bufs, int64_t capacity_bytes, int32_t* counter,
                         int32_t* err_flag, void* stream) {
  if ((residual == nullptr) != (y == nullptr))
    return fail(PIM_EINVAL, "pim_allreduce_p2p_ll: residual and y go together");
  if (!sum_out && !y) return fail(PIM_EINVAL, "pim_allreduce_p2p_ll: no output");
  void* dsts[1] = {sum_out};
  pim::P2PArgs a;
  const int rc = p2p_args("pim_allreduce_p2p_ll", src, dsts, sum_out ? 1 : 0, numel, dtype, rank, size, bufs,
                          capacity_bytes, counter, err_flag, &a);
  if (rc != PIM_OK || numel == 0) return rc;
  const int64_t es = dtype == PIM_BF16 ? 2 : 4;
  if (2 * numel * es > capacity_bytes)
    return fail(PIM_EINVAL, "pim_allreduce_p2p_ll: 2 * numel * element size must fit the row capacity");
  a.residual = residual;
  a.y = y;
  return check(pim::allreduce_ll(a, dtype, (cudaStream_t)stream), "pim_allreduce_p2p_ll");
}

int64_t pim_p2p_desc_bytes(void) { return (int64_t)sizeof(pim::P2PDev); }

int pim_p2p_desc_init(void* desc, int32_t rank, int32_t size, void* const* bufs, int64_t capacity_bytes,
                      int32_t* counter, int32_t* tickets, int32_t* err_flag) {
  if (!desc || !bufs || !counter || !tickets || size < 1 || size > PIM_P2P_MAX_RANKS || rank < 0 || rank >= size ||
      capacity_bytes <= 0 || capacity_bytes % 16)
    return fail(PIM_EINVAL, "pim_p2p_desc_init: bad arguments");
  pim::P2PDev d = {};
  d.rank = rank;
  d.size = size;
  d.capacity_bytes = capacity_bytes;
  d.counter = counter;
  d.tickets = tickets;
  d.err = err_flag;
  for (int i = 0; i < size; ++i) {
    if (!bufs[i]) return fail(PIM_EINVAL, "pim_p2p_desc_init: null exchange buffer");
    d.bufs[i] = bufs[i];
  }
  return check(cudaMemcpy(desc, &d, sizeof(d), cudaMemcpyHostToDevice), "pim_p2p_desc_init");
}

int pim_ipc_export(const void* ptr, void* handle64, int64_t* offset) {
  if (!ptr || !handle64 || !offset) return fail(PIM_EINVAL, "pim_ipc_export: null argument");
  cudaIpcMemHandle_t h;
  const int rc = check(pim::ipc_export(ptr, &h, offset), "pim_ipc_export");
  if (rc == PIM_OK) memcpy(handle64, &h, sizeof(h));
  return rc;
}

int pim_ipc_open(const void* handle64, void** base) {
  if (!handle64 || !base) return fail(PIM_EINVAL, "pim_ipc_open: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  return check(cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess), "pim_ipc_open");
}

int pim_ipc_close(void* base) {
  if (!base) return fail(PIM_EINVAL, "pim_ipc_close: null argument");
  return check(cudaIpcCloseMemHandle(base), "pim_ipc_close");
}

int pim_batched_copy(const void* desc_dev, int32_t count, int64_t max_nbytes, void* stream) {
  if (count < 0 || (count > 0 && !desc_dev) || max_nbytes < 0)
    return fail(PIM_EINVAL, "pim_batched_copy: bad arguments");
  return check(pim::batched_copy(desc_dev, count, max_nbytes, (cudaStream_t)stream), "pim_batched_copy");
}

int pim_fill_normal(void* out, int64_t n, int32_t dtype, uint64_t seed, float std, void* stream) {
  if (!out || n < 0 || !dtype_ok(dtype)) return fail(PIM_EINVAL, "pim_fill_normal: bad arguments");
  if (n == 0) return PIM_OK;
  return check(pim::fill_normal(out, n, dtype, seed, std, (cudaStream_t)stream), "pim_fill_normal");
}

int pim_fill_const(void* out, int64_t n, int32_t dtype, float value, void* stream) {
  if (!out || n < 0 || !dtype_ok(dtype)) return fail(PIM_EINVAL, "pim_fill_const: bad arguments");
  if (n == 0) return PIM_OK;
  return check(pim::fill_const(out, n, dtype, value, (cudaStream_t)stream), "pim_fill_const");
}

}  // extern "C"
