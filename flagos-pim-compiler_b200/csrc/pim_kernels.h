// Internal launch interfaces shared by the .cu files (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

struct pim_decode_step_plan;  // opaque to the C ABI (decode_layer.cu)

namespace pim {

enum FusedMode : int { MODE_PLAIN = 0, MODE_ROPE = 1, MODE_SILU = 2 };

// Rows up to this count take the GEMV path; more rows take rmsnorm -> GEMM -> epilogue.
constexpr int kGemvMaxRows = 8;

struct FusedArgs {
  const void* x;      // [rows, K] activations
  const void* ln_w;   // [K] rmsnorm weight (nullptr: no normalisation)
  const void* w;      // [ncols, K] weight rows of this rank
  void* y;            // output
  int rows, K, ncols;
  float eps;
  // ROPE (attn_in): q/k/v column blocks, rotary tables and the KV blocks of one layer
  const float* cos;
  const float* sin;
  const int* positions;  // [batch] start position of each sequence
  int seq;               // tokens per sequence (rows = batch * seq)
  int hq, hkv, hd;
  void* kv_base;              // K block of the layer's first local kv head
  long long block_stride;     // elements between consecutive (head, k|v) blocks
  long long seq_stride;       // elements between sequences
  int max_seq;
  // SILU (mlp_in)
  int inter;
  // PLAIN only: y = residual + x . W (the residual add fused into the epilogue), or nullptr
  const void* residual;
  // Device int raised when a bounded wait expires (may be nullptr)
  int* err;
  // PLAIN at TP > 1 (decode rows): a device P2PDev; the partial goes to every rank's
  // exchange buffer, the kernel adds the ranks' partials in rank order and writes
  // y = residual + sum (and the sum itself to ar_out when given).  nullptr: no all-reduce.
  const void* p2p;
  void* ar_out;
  // ROPE at decode rows, opt-in: the layer's decode attention computed at the end of the
  // same launch (gemv_attention.cuh) into attn_out [rows, hq * hd]; attn_cnt: hq ints,
  // zero between launches.  nullptr: no attention.
  void* attn_out;
  int* attn_cnt;
};

// Decode projection kernels (gemv_variant() picks one per process; see gemv.cu).
// (2 was a bulk-copy streamed kernel, removed after it measured slower than the staged one.)
enum GemvVariant : int { kGemvRegister = 0, kGemvStaged = 1, kGemvDynamic = 3 };
int gemv_variant();
void set_gemv_variant(int v);
cudaError_t fused_projection_async(const FusedArgs& a, int dtype, int mode, bool norm, cudaStream_t st,
                                   bool* handled);
// attn_in (ROPE, rows <= kGemvMaxRows) with the decode attention fused (a.attn_out set).
cudaError_t fused_projection_attention(const FusedArgs& a, int dtype, bool norm, cudaStream_t st);
constexpr int kFusedAttnMaxHeads = 64;
// Work counter of the dynamic kernel (two ints, zero between launches) in the scratch of
// a decode projection; without it the staged kernel runs.
constexpr size_t kGemvCounterBytes = 256;
cudaError_t fused_projection_dynamic(const FusedArgs& a, int dtype, int mode, bool norm, int* ctr, cudaStream_t st,
                                     bool* handled);
cudaError_t fused_projection_dynamic_allreduce(const FusedArgs& a, int dtype, int* ctr, cudaStream_t st,
                                               bool* handled);

cudaError_t fused_projection(const FusedArgs& a, int dtype, int mode, bool norm, void* scratch, cudaStream_t st);
// One decode layer (one activation row): attn_in (ROPE, norm, attention fused) -> o_proj
// (PLAIN) -> mlp_in (SILU, norm) -> down (PLAIN) in one launch (decode_layer.cu).
// bar: two zero unsigned words; err: raised when a grid barrier wait gives up.
cudaError_t decode_layer(const FusedArgs& qkv, const FusedArgs& o, const FusedArgs& mlp, const FusedArgs& down,
                         unsigned* bar, int* err, int dtype, cudaStream_t st);
// A whole decode step in one launch: `phases` holds attn_in, o_proj, mlp_in, down of each
// of `nlayers` layers; prepare writes their table into `table` (synchronous copy) and
// sizes the grid; head (nullable): lm_head_in (PLAIN with rmsnorm).
size_t decode_step_table_bytes(int nlayers);
cudaError_t decode_step_prepare(const FusedArgs* phases, int nlayers, const FusedArgs* head, int dtype, void* table,
                                size_t table_bytes, pim_decode_step_plan** out);
cudaError_t decode_step(const pim_decode_step_plan* plan, unsigned* bar, int* err, cudaStream_t st);
void decode_step_free(pim_decode_step_plan* plan);
// Tensor-core GEMM with the node's epilogue for bf16 row batches (gemm_tc.cu).
enum GemmKernel : int { kGemmTile = 0, kGemmPersistent = 1 };
int gemm_kernel();
void set_gemm_kernel(int v);
bool gemm_tc_supported(int K);
cudaError_t gemm_tc(const FusedArgs& a, int mode, const void* xin, cudaStream_t st);
size_t fused_scratch_bytes(const FusedArgs& a, int dtype, int mode);

struct AttnArgs {
  const void* q;        // [batch, seq, hq*hd]
  const int* positions; // [batch]
  const void* kv_base;  // K block of the layer's first local kv head
  long long block_stride, seq_stride;
  void* out;            // [batch, seq, hq*hd]
  int batch, seq, hq, hkv, hd, max_seq;
  float scale;
};

cudaError_t attention(const AttnArgs& a, int dtype, void* workspace, size_t workspace_bytes, cudaStream_t st);
// Row batches (seq >= 16), bf16, head_dim 128: flash-style tensor-core kernel (attention_prefill.cu).
bool attention_prefill_supported(const AttnArgs& a, int dtype);
cudaError_t attention_prefill(const AttnArgs& a, cudaStream_t st);
// The same on tcgen05 (attention_tc.cu), opt-in with PIM_ATTN=tc; errors() reads (and
// with reset clears) its device error word, raised when one of its waits gave up.
bool attention_tc_supported(const AttnArgs& a, int dtype);
cudaError_t attention_tc(const AttnArgs& a, cudaStream_t st);
int attention_tc_errors(bool reset);
int prefill_attention_kernel();  // 0 warp-level MMA, 1 tcgen05
void set_prefill_attention_kernel(int v);
size_t attention_workspace_bytes(const AttnArgs& a);
// Whether attention() runs `a` on the split-K kernel, the only one that uses the workspace
// (the tensor-core row-batch kernels take none).
bool attention_uses_workspace(const AttnArgs& a, int dtype);

// One-shot all-reduce over peer memory (p2p.cu).
constexpr int kP2PMaxRanks = 64;
constexpr int kP2PMaxDst = 4;
constexpr int64_t kP2PHeaderBytes = 1024;  // 2 slots x kP2PMaxRanks flags, padded

// Device-resident description of a P2P group, read by fused projection + all-reduce
// kernels (written once by pim_p2p_desc_init).
struct P2PDev {
  int rank, size;
  int64_t capacity_bytes;
  int* counter;  // this rank's call counter (shared with pim_allreduce_p2p)
  int* tickets;  // two ints, zero between calls
  int* err;      // raised when a wait for a peer gives up
  void* bufs[kP2PMaxRanks];
};

struct P2PArgs {
  const void* src;             // this rank's partial [numel]
  void* dst[kP2PMaxDst];       // destinations of the sum
  int ndst;
  int64_t numel;
  int rank, size;
  void* bufs[kP2PMaxRanks];    // every rank's exchange buffer, as mapped in this process
  int64_t capacity_bytes;      // bytes of one row of a slot
  int* counter;                // this rank's call counter (device, starts at 0)
  int* err;                    // raised when the wait for a peer gives up
  const void* residual;        // optional: y = residual + sum (the residual add after the all_reduce)
  void* y;
};

cudaError_t allreduce_p2p(const P2PArgs& a, int dtype, cudaStream_t st);
cudaError_t allreduce_ll(const P2PArgs& a, int dtype, cudaStream_t st);  // epoch-tagged words, no fences
cudaError_t fused_projection_allreduce(const FusedArgs& a, int dtype, cudaStream_t st);
cudaError_t ipc_export(const void* ptr, cudaIpcMemHandle_t* handle, int64_t* offset);

}  // namespace pim
