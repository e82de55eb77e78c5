/*
 * pim_b200.h -- C ABI of the B200 execution backend for the flagos-pim-compiler
 * ExecutionPlan runtime.
 *
 * The reference runtime has no native boundary: its HAL (backend/hal_numpy.py) runs
 * kernel stubs as Python callables and its communication library
 * (comm/lowering.py) reduces in NumPy on the host.  Each entry point below is the
 * device implementation of one of those Python-level operations; the comment on
 * each cites the reference interface it replaces.  The B200 HAL
 * (backend/hal_cuda.py) binds them with ctypes.
 *
 * Conventions
 *   - every pointer is a device address (the rank's arena + a planner offset), except
 *     where noted; no function allocates or frees memory;
 *   - `stream` is a cudaStream_t passed as void*; work is enqueued, never synchronised;
 *   - dtype codes: PIM_F32 = 0, PIM_BF16 = 1;
 *   - return 0 on success, a PIM_E* code otherwise; pim_last_error() describes the
 *     last failure on the calling thread.
 */
#ifndef PIM_B200_H
#define PIM_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PIM_ABI_VERSION 13

enum pim_dtype { PIM_F32 = 0, PIM_BF16 = 1, PIM_I32 = 2, PIM_I64 = 3 };
enum pim_status { PIM_OK = 0, PIM_EINVAL = 1, PIM_ECUDA = 2, PIM_EUNSUPPORTED = 3 };
enum pim_projection_mode { PIM_PROJ_PLAIN = 0, PIM_PROJ_ROPE_KV = 1, PIM_PROJ_SILU_MUL = 2 };

/* Version of this ABI (PIM_ABI_VERSION). */
int pim_abi_version(void);

/* Number of kernels this library has launched in this process (every device and stream),
 * counting launches recorded into a CUDA graph once at capture (graph replays launch
 * them again without calling the library).  No counterpart in the reference. */
uint64_t pim_kernel_launches(void);

/* Message for the last non-zero status returned on this thread. */
const char* pim_last_error(void);

/* Whether kernels whose CTAs wait on one another (the decode layer / step kernels, the
 * fused projection + all-reduce) were launched on `device` as cooperative launches that
 * also carry programmatic dependent launch: 1 yes, 0 the driver refused the combination
 * (they run as plain cooperative launches), -1 no such launch was made yet.  Every such
 * launch is cooperative: a grid that cannot be resident at once is refused with a CUDA
 * error instead of waiting.  No counterpart in the reference. */
int pim_cooperative_pdl(int32_t device);

/* Lets kernels running on `device` dereference arena pointers of `peer` (one process
 * driving several GPUs).  Replaces nothing: the reference forbids device-to-device
 * copies (backend/hal_numpy.py:56-57); peers are read only inside redistribute kernels. */
int pim_enable_peer_access(int32_t device, int32_t peer);

typedef struct pim_projection_args {
  const void* x;            /* [rows, k] activations of the rank                      */
  const void* norm_weight;  /* [k] RMSNorm weight, or NULL for no normalisation        */
  const void* weight;       /* [ncols, k] weight rows of the rank (HF [out, in] layout) */
  void* out;                /* PLAIN: [rows, ncols]; ROPE_KV: q [rows, q_heads*head_dim];
                               SILU_MUL: [rows, inter]                                 */
  int64_t rows, k, ncols;
  float eps;
  /* ROPE_KV only */
  const float* rope_cos;    /* [max_seq, head_dim/2] */
  const float* rope_sin;
  const int32_t* positions; /* [rows/seq] start position of each sequence */
  int32_t seq, q_heads, kv_heads, head_dim, max_seq;
  void* kv_base;            /* K block of the layer's first local kv head              */
  int64_t kv_block_stride;  /* elements between (head, k|v) blocks                     */
  int64_t kv_seq_stride;    /* elements between sequences                              */
  /* SILU_MUL only */
  int32_t inter;
  /* PLAIN only: out = residual + x . weight^T (the residual add fused), or NULL */
  const void* residual;
  /* device int32 set to non-zero if a bounded internal wait expires (may be NULL) */
  int32_t* err_flag;
  /* PLAIN at TP > 1, rows <= 8, one process per GPU: a device descriptor written by
   * pim_p2p_desc_init.  The partial x . weight^T of this rank goes to every rank's
   * exchange buffer over NVLink and the kernel writes out = residual + (rank-order sum
   * of the partials), i.e. the linear node, its Partial -> Replicate all_reduce
   * (comm/lowering.py:137-150) and the following add node in one launch; the sum alone
   * also goes to allreduce_out when non-NULL.  NULL: no all-reduce. */
  const void* p2p_desc;
  void* allreduce_out;
  /* ROPE_KV at rows <= 8 (decode), optional: the layer's causal decode attention (the
   * `attention` node after attn_in; the tiled KV reads of PIMStaticKVCache.read_tile,
   * memory/kv_layout.py:207-230, masked as decode_mask, :239-252) computed at the end of
   * the same launch, for every q head and row, into attn_out [rows, q_heads*head_dim]:
   * the CTA that writes the last q / k / v value a head needs computes that head.
   * attn_counters: q_heads device int32, zero-filled before the first call, left zero by
   * every call and written by nothing else.  q_heads <= 64, head_dim 64 or 128; the
   * staged kernel runs whatever pim_set_projection_kernel chose.  NULL: no attention. */
  void* attn_out;
  int32_t* attn_counters;
} pim_projection_args;

/* One projection launch of a rank.  Replaces the DPU `aten.linear` kernel stub that
 * NumpyBackend.submit runs for a "launch" command (backend/hal_numpy.py:251-256; rule
 * graph/spec_prop.py:236-256) together with the host glue that surrounds it in the
 * exported graph: RMSNorm (pow/mean/rsqrt + mul), RoPE (slice/neg/cat + mul/add) and
 * the KV append of PIMStaticKVCache.update (memory/kv_layout.py:187-205) in mode
 * ROPE_KV; silu + mul in mode SILU_MUL.  rows <= 8 run as a GEMV; larger row counts
 * need `scratch` of pim_projection_scratch_bytes() bytes.  For rows <= 8 the scratch is
 * optional: while PIM_PROJ_KERNEL_DYNAMIC is selected, pim_projection_scratch_bytes()
 * asks for a work counter that must be zero-filled before the first call and not be
 * written by anything else (the kernel leaves it zero); a call without it runs the
 * staged kernel. */
int pim_projection(const pim_projection_args* a, int32_t dtype, int32_t mode, void* scratch,
                   int64_t scratch_bytes, void* stream);
int64_t pim_projection_scratch_bytes(const pim_projection_args* a, int32_t dtype, int32_t mode);

/* Kernel that runs decode projections (rows <= 8) from now on, for the whole process:
 * PIM_PROJ_KERNEL_REGISTER (weights streamed through registers), PIM_PROJ_KERNEL_STAGED
 * (cp.async-staged, every warp streams the same bytes) or PIM_PROJ_KERNEL_DYNAMIC
 * (staged, CTAs take units of work from a counter); any other value (2 included: it
 * was a bulk-copy kernel, removed) is refused with PIM_EINVAL.  All give results within
 * fp32 summation-order differences of one another; shapes a kernel cannot take run on
 * the register kernel.  The initial choice is the staged kernel unless the environment
 * variable PIM_GEMV says "reg" or "dyn".
 * Launches already recorded in a CUDA graph keep their kernel.  No counterpart in the
 * reference. */
#define PIM_PROJ_KERNEL_REGISTER 0
#define PIM_PROJ_KERNEL_STAGED 1
#define PIM_PROJ_KERNEL_DYNAMIC 3
int pim_set_projection_kernel(int32_t kernel);
int32_t pim_projection_kernel(void);

/* Bytes of the zero-filled barrier word pair that pim_decode_layer takes. */
#define PIM_DECODE_LAYER_BARRIER_BYTES 256

/* One decoder layer of a decode step with one activation row (batch 1) in ONE
 * launch: the four projections attn_in (mode ROPE_KV, with attn_out / attn_counters:
 * the layer's decode attention), o_proj (PLAIN, residual optional), mlp_in (SILU_MUL)
 * and down (PLAIN, residual optional) -- the five launch commands a layer of the decode
 * plan lowers to (pim_projection x 4 + the attention), run by one grid of at most as many
 * CTAs as the GPU holds at once, with a grid-wide barrier between phases.  Each phase
 * computes what pim_projection computes (the staged kernel's arithmetic; results equal
 * pim_projection's up to fp32 summation order).  The chain is checked: o_proj.x ==
 * attn_in.attn_out, mlp_in.x == o_proj.out, down.x == mlp_in.out, and the k of each
 * phase equals the width of the previous phase's output; attn_in and mlp_in take a
 * norm_weight, o_proj and down none.  At TP > 1 (one process per GPU) o_proj and down
 * carry the same p2p_desc (and optionally allreduce_out): each is then the row-parallel
 * projection + rank-order all-reduce + residual add of pim_projection's p2p_desc, two
 * all-reduce calls per launch on the descriptor's group (exchange rows of at least
 * ncols x element bytes).  `barrier`: PIM_DECODE_LAYER_BARRIER_BYTES
 * of device memory, zero-filled before the first call and written by nothing else (every
 * call leaves the count zero); calls on one barrier must not overlap on the GPU.
 * `err_flag` (device int32, may be NULL) is raised when a barrier wait gives up (one
 * second): the layer's output is then not valid.  PIM_EUNSUPPORTED when the shapes do not
 * fit the kernel's shared memory or the GPU cannot hold its grid.  Replaces the five
 * `launch` commands of a decode layer; no single counterpart in the reference. */
int pim_decode_layer(const pim_projection_args* attn_in, const pim_projection_args* o_proj,
                     const pim_projection_args* mlp_in, const pim_projection_args* down, void* barrier,
                     int32_t* err_flag, int32_t dtype, void* stream);

/* A whole decode step with one activation row in ONE launch: every layer as in
 * pim_decode_layer, with a grid-wide barrier in place of the kernel boundary between
 * consecutive layers (the next layer's q/k/v weights streaming across it), then, when
 * `head` is given, the lm_head_in projection (PLAIN with norm_weight: the final RMSNorm
 * and the vocabulary GEMV of the decode plan).  Replaces the 5 x nlayers + 1 launch
 * commands of a decode step between the embedding and the logits; no single counterpart
 * in the reference.
 *
 * pim_decode_step_prepare checks `layers` (4 * nlayers pointers: attn_in, o_proj, mlp_in,
 * down of each layer, each layer as pim_decode_layer checks it, layer l + 1 reading layer
 * l's output, the same p2p_desc in every layer or none) and `head` (NULL, or reading the
 * last layer's output), writes the layers' argument table into `table` (device memory of
 * pim_decode_step_table_bytes(nlayers) bytes, 16-byte aligned; a synchronous copy: not
 * during a stream capture), sizes the grid (PIM_EUNSUPPORTED when no grid fits) and returns
 * a host-side plan.  The table must stay untouched while the plan is used.
 * pim_decode_step launches it; `barrier` and `err_flag` as in pim_decode_layer (calls on
 * one barrier must not overlap on the GPU).  pim_decode_step_free releases the plan (host
 * memory only). */
typedef struct pim_decode_step_plan pim_decode_step_plan;
int64_t pim_decode_step_table_bytes(int32_t nlayers);
int pim_decode_step_prepare(const pim_projection_args* const* layers, int32_t nlayers,
                            const pim_projection_args* head, int32_t dtype, void* table, int64_t table_bytes,
                            pim_decode_step_plan** plan);
int pim_decode_step(const pim_decode_step_plan* plan, void* barrier, int32_t* err_flag, void* stream);
void pim_decode_step_free(pim_decode_step_plan* plan);

/* Kernel that runs bf16 row-batch projections (rows > 8, the tcgen05 GEMM) from now on,
 * for the whole process: PIM_ROW_BATCH_KERNEL_TILE (one 128 x 256 output tile per CTA)
 * or PIM_ROW_BATCH_KERNEL_PERSISTENT (one CTA per SM looping over the tiles, the epilogue
 * of one tile overlapping the MMAs of the next).  Both accumulate every output in the
 * same order (fp32 over K blocks in order), so results are identical.  The initial
 * choice is the persistent kernel (the faster on B200) unless the environment variable
 * PIM_GEMM says "tile".
 * Launches already recorded in a CUDA graph keep their kernel.  No counterpart in the
 * reference. */
#define PIM_ROW_BATCH_KERNEL_TILE 0
#define PIM_ROW_BATCH_KERNEL_PERSISTENT 1
int pim_set_row_batch_kernel(int32_t kernel);
int32_t pim_row_batch_kernel(void);

/* Attention of one layer over the rank's KV blocks (causal; the query at position p
 * sees keys 0..p).  Replaces the host `aten.scaled_dot_product_attention` node and
 * the tiled KV reads of PIMStaticKVCache.read_tile (memory/kv_layout.py:207-230),
 * masked as decode_mask / prefill_mask (memory/kv_layout.py:233-252).  head_dim 32,
 * 64 or 128.  Needs a caller-provided `workspace` of pim_attention_workspace_bytes()
 * bytes, used by the split-K kernel (bf16 head_dim-128 row batches of 16 or more query
 * rows per sequence run on the tensor-core kernels and leave it untouched). */
int pim_attention(const void* q, const int32_t* positions, const void* kv_base, int64_t kv_block_stride,
                  int64_t kv_seq_stride, void* out, int32_t batch, int32_t seq, int32_t q_heads,
                  int32_t kv_heads, int32_t head_dim, int32_t max_seq, int32_t dtype, void* workspace,
                  int64_t workspace_bytes, void* stream);

/* Row batches (seq >= 16) of bf16 with head_dim 128 run on the tensor cores: warp-level
 * MMA (PIM_PREFILL_ATTENTION_MMA, the default) or tcgen05 with TMEM accumulators and
 * TMA-loaded tiles (PIM_PREFILL_ATTENTION_TCGEN05), for the whole process from the call
 * on; the initial choice is tcgen05 when the environment variable PIM_ATTN says "tc".
 * Launches already recorded in a CUDA graph keep their kernel.  The tcgen05 kernel has
 * no error argument: a wait of it that gives up raises a library-wide device word, which
 * pim_attention_errors returns (1 raised, 0 clear, -1 when it cannot be read) and clears
 * when `reset` != 0 (synchronous; not during a stream capture).  No counterpart in the
 * reference. */
#define PIM_PREFILL_ATTENTION_MMA 0
#define PIM_PREFILL_ATTENTION_TCGEN05 1
int pim_set_prefill_attention_kernel(int32_t kernel);
int32_t pim_prefill_attention_kernel(void);
int32_t pim_attention_errors(int32_t reset);
int64_t pim_attention_workspace_bytes(int32_t batch, int32_t seq, int32_t q_heads, int32_t head_dim,
                                      int32_t max_seq);

/* Size of the fixed scratch behind pim_attention_noalloc (4 MiB on every GPU that loads
 * the library, held until the process exits). */
#define PIM_ATTENTION_NOALLOC_SCRATCH_BYTES (4u << 20)

/* pim_attention without a caller workspace, for callers that cannot allocate device
 * memory -- for example a plugin whose host program owns all device memory through its
 * own pool allocator, or code on a latency-critical path where cudaMalloc would
 * synchronize the device.  No counterpart in the reference (its attention runs on the
 * host).  Allocates nothing: the workspace is a file-scope device array of
 * PIM_ATTENTION_NOALLOC_SCRATCH_BYTES.  Only the split-K kernel uses it: shapes that run
 * there and whose workspace (pim_attention_workspace_bytes) is larger are rejected with
 * PIM_EINVAL; bf16 head_dim-128 row batches (16 or more query rows per sequence) run on
 * the tensor-core kernels, need no workspace and are accepted at any size.  The first
 * call on each device (and under each CUDA context) looks the array up
 * (cudaGetSymbolAddress) with that device current; make that first call before any
 * stream capture.  A cudaDeviceReset after the first call is not supported (the cached
 * address can go stale).  All calls share the array: calls that overlap on the GPU race;
 * each call clears the counters it needs zeroed. */
int pim_attention_noalloc(const void* q, const int32_t* positions, const void* kv_base, int64_t kv_block_stride,
                          int64_t kv_seq_stride, void* out, int32_t batch, int32_t seq, int32_t q_heads,
                          int32_t kv_heads, int32_t head_dim, int32_t max_seq, int32_t dtype, void* stream);

/* Embedding row gather.  Replaces the host `aten.embedding` node of the exported graph
 * (the reference keeps the table Replicate@host, docs/spec.md:1994). Out-of-range ids
 * give a zero row and set *err_flag (device int32, may be NULL). */
int pim_embedding(const int32_t* ids, const void* table, void* out, int64_t n_ids, int64_t hidden,
                  int64_t vocab, int32_t dtype, int32_t* err_flag, void* stream);

/* out = a + b (rounded to dtype).  Replaces the DPU `aten.add.Tensor` stub for the
 * residual adds (graph/spec_prop.py:265-305). */
int pim_add(const void* a, const void* b, void* out, int64_t n, int32_t dtype, void* stream);

/* out[b] = x[b, index] for b < batch (rows of row_bytes bytes).  Replaces taking the
 * prefill logits at position P-1 (docs/spec.md:1552-1553). */
int pim_select_rows(const void* x, void* out, int32_t batch, int32_t seq, int64_t row_bytes, int32_t index,
                    void* stream);

/* Greedy sampling: first index of each row's maximum.  Replaces the host argmax of
 * the decode loop (docs/spec.md:1552-1556). */
int pim_argmax(const void* x, int32_t* out, int32_t rows, int64_t n, int32_t dtype, void* stream);

/* Device copy (same device or peer).  Replaces dpu_copy_to / dpu_copy_from byte
 * moves of one segment (backend/dpu_sdk.py:139-157). */
int pim_copy(void* dst, const void* src, int64_t nbytes, void* stream);

/* Partial -> Replicate combine: dst[d][i] = ((0 + src[0][i]) + src[1][i]) + ..., rounded to
 * dtype after every add, in the given (rank) order; divided by nsrc when mean != 0.
 * Bit-identical to the host accumulation of comm/lowering.py:137-150.  src/dst are
 * HOST arrays of up to 8 device pointers each. */
int pim_ordered_sum(const void* const* src, int32_t nsrc, void* const* dst, int32_t ndst, int64_t n,
                    int32_t dtype, int32_t mean, void* stream);

/* The Partial -> Replicate combine followed by the residual add that consumes it (the
 * `add` node after o_proj / down_proj, graph/spec_prop.py:265-305):
 * out[i] = residual[i] + S[i], S the rank-order sum of pim_ordered_sum (rounded to dtype
 * after every partial) and the add rounded to dtype once more, exactly as the combine
 * followed by the add; S itself is also written to sum_out unless it is NULL.  src is a
 * HOST array of up to 8 device pointers; dtype PIM_F32 or PIM_BF16. */
int pim_ordered_sum_add(const void* const* src, int32_t nsrc, const void* residual, void* out, void* sum_out,
                        int64_t n, int32_t dtype, void* stream);

/* One process per GPU: the Partial -> Replicate combine over NVLink peer memory, one
 * kernel per call.  Every rank calls it in the same order with its partial `src`
 * (numel elements, numel * element size a multiple of 16 and at most capacity_bytes);
 * `bufs` is a HOST array of `size` device pointers: every rank's exchange buffer of
 * PIM_P2P_HEADER_BYTES + 2 * size * capacity_bytes bytes (zero-filled before the first
 * call) as mapped in this process (pim_ipc_open), this rank's own at bufs[rank].  The
 * result is the rank-order sum of pim_ordered_sum (bit-identical to comm/lowering.py:
 * 137-150), written to the `ndst` (<= 4) device pointers of the HOST array `dsts`.
 * `counter` is a device int32 of this rank, zero before the first call.  A rank that
 * waits more than 1 s for a peer raises *err_flag (when given) and returns.  Replaces
 * the host-star all_reduce of comm/lowering.py:137-150 at TP > 1; no kernel in the
 * reference. */
#define PIM_P2P_HEADER_BYTES 1024
#define PIM_P2P_MAX_RANKS 64

/* Size of the device descriptor of a P2P group, and its initialisation (synchronous):
 * the group's exchange buffers as mapped here (HOST array of `size` device pointers), the
 * row capacity, this rank's call counter (shared with pim_allreduce_p2p), two device
 * int32 tickets (zero) and the error word raised when a wait for a peer gives up. */
int64_t pim_p2p_desc_bytes(void);
int pim_p2p_desc_init(void* desc, int32_t rank, int32_t size, void* const* bufs, int64_t capacity_bytes,
                      int32_t* counter, int32_t* tickets, int32_t* err_flag);
int pim_allreduce_p2p(const void* src, void* const* dsts, int32_t ndst, int64_t numel, int32_t dtype,
                      int32_t rank, int32_t size, void* const* bufs, int64_t capacity_bytes, int32_t* counter,
                      int32_t* err_flag, void* stream);
/* pim_allreduce_p2p followed by the residual add that consumes the sum, in the same
 * kernel: y = residual + sum (the fp32 add of the rounded sum, rounded once -- the bits of
 * pim_ordered_sum_add, i.e. of the reference's all_reduce then aten.add), and the sum itself
 * into `sum_out` when it is not NULL.  Replaces the host-star all_reduce of
 * comm/lowering.py:137-150 together with the DPU `add` node after it. */
int pim_allreduce_p2p_add(const void* src, const void* residual, void* y, void* sum_out, int64_t numel,
                          int32_t dtype, int32_t rank, int32_t size, void* const* bufs, int64_t capacity_bytes,
                          int32_t* counter, int32_t* err_flag, void* stream);

/* The same bit-exact rank-order all-reduce over the same exchange buffers with the
 * low-latency protocol: every 32-bit word of the partial is stored to the peers as one
 * 64-bit word whose high half is the call's epoch, and readers poll the words themselves
 * (no system-scope fence, no separate flag).  Writes the sum to `sum_out` and/or, when
 * `residual` and `y` are given, y = residual + sum (the bits of pim_ordered_sum_add).
 * 2 * numel * element size must fit `capacity_bytes`.  A group of exchange buffers is used
 * with this protocol or with pim_allreduce_p2p / the fused projection, not both.  Replaces
 * the host-star all_reduce of comm/lowering.py:137-150 (and the add node after it). */
int pim_allreduce_p2p_ll(const void* src, const void* residual, void* y, void* sum_out, int64_t numel,
                         int32_t dtype, int32_t rank, int32_t size, void* const* bufs, int64_t capacity_bytes,
                         int32_t* counter, int32_t* err_flag, void* stream);

/* CUDA IPC for the exchange buffers: the 64-byte handle of the allocation holding `ptr`
 * and ptr's byte offset in it; opening a peer's handle maps that allocation here
 * (*base; add the peer's offset); closing unmaps it.  No reference counterpart. */
int pim_ipc_export(const void* ptr, void* handle64, int64_t* offset);
int pim_ipc_open(const void* handle64, void** base);
int pim_ipc_close(void* base);

/* Executes `count` (src, dst, nbytes) runs stored at desc_dev (device memory, 24 bytes
 * each: two pointers and an int64).  Replaces the collect / writeback transfer
 * sequences of dma_sequence (comm/plan.py:330-347) as executed by DmaEngine
 * (comm/lowering.py:55-97) for all_gather, all_to_all, scatter and broadcast. */
int pim_batched_copy(const void* desc_dev, int32_t count, int64_t max_nbytes, void* stream);

/* Seeded N(0, std^2) fill (counter-based; same seed -> same values).  Used for
 * random-init weights; no reference counterpart (HF initialises on the host). */
int pim_fill_normal(void* out, int64_t n, int32_t dtype, uint64_t seed, float std, void* stream);

/* Constant fill (e.g. RMSNorm weights = 1).  No reference counterpart. */
int pim_fill_const(void* out, int64_t n, int32_t dtype, float value, void* stream);


/* ---- aten-level operations -------------------------------------------------------
 * For graphs compiled at aten granularity by the reference's own passes (torch.export,
 * graph/partition.py:36-81, graph/spec_prop.py:411-451): the DPU nodes (aten.linear,
 * aten.add / mul.Tensor, aten.tanh; the reference's kernel stubs) run on their rank's
 * arena and the host nodes (the torch callables the reference runs on the CPU:
 * embedding, pow / mean / rsqrt, view / reshape / transpose / slice / cat / expand,
 * to.dtype, matmul, cos / sin, scaled_dot_product_attention, silu, neg, alias) run on the
 * plan's device-resident host buffer.  Operands are strided views: element offset,
 * shape and element strides (a stride of 0 broadcasts); operand views have the output's
 * rank.  Dtypes PIM_F32, PIM_BF16, PIM_I32, PIM_I64; arithmetic in fp32 (copies convert
 * exactly between the integer types and fp32 where the value allows). */
#define PIM_MAX_DIMS 8
typedef struct pim_tensor_view {
  void* data;                    /* base pointer (device) */
  int32_t dtype;                 /* pim_dtype */
  int32_t ndim;                  /* 0..PIM_MAX_DIMS */
  int64_t offset;                /* elements from data to element [0, ..., 0] */
  int64_t shape[PIM_MAX_DIMS];
  int64_t stride[PIM_MAX_DIMS];  /* elements; 0 broadcasts */
} pim_tensor_view;

enum pim_aten_op {
  /* unary (pim_aten_unary; `scalar` is the second operand of the *_SCALAR ops and the
   * exponent of POW_SCALAR) */
  PIM_ATEN_NEG = 0, PIM_ATEN_RSQRT = 1, PIM_ATEN_SQRT = 2, PIM_ATEN_SILU = 3, PIM_ATEN_COS = 4,
  PIM_ATEN_SIN = 5, PIM_ATEN_TANH = 6, PIM_ATEN_EXP = 7, PIM_ATEN_RECIPROCAL = 8, PIM_ATEN_POW_SCALAR = 9,
  PIM_ATEN_ADD_SCALAR = 10, PIM_ATEN_MUL_SCALAR = 11, PIM_ATEN_SUB_SCALAR = 12, PIM_ATEN_DIV_SCALAR = 13,
  /* binary (pim_aten_binary) */
  PIM_ATEN_ADD = 20, PIM_ATEN_SUB = 21, PIM_ATEN_MUL = 22, PIM_ATEN_DIV = 23
};

/* dst[i] = src[i] over dst's shape, converting the element type: aten view / reshape /
 * unsqueeze / alias / transpose / slice / expand / to.dtype, and one input of aten.cat
 * (dst a view into the output).  Replaces the host FX callables of those nodes. */
int pim_aten_copy(const pim_tensor_view* dst, const pim_tensor_view* src, void* stream);
/* dst = op(src[, scalar]): aten.neg / rsqrt / silu / cos / sin / tanh / pow.Tensor_Scalar
 * and add / mul / sub / div with a scalar operand (the reference's DPU aten.add / mul stub
 * when one operand is a Python number, graph/spec_prop.py:265-305). */
int pim_aten_unary(int32_t op, const pim_tensor_view* dst, const pim_tensor_view* src, double scalar,
                   void* stream);
/* dst = a op b with broadcasting: the DPU aten.add / mul.Tensor stubs
 * (graph/spec_prop.py:265-305) and their host counterparts. */
int pim_aten_binary(int32_t op, const pim_tensor_view* dst, const pim_tensor_view* a, const pim_tensor_view* b,
                    void* stream);
/* aten.mean.dim over the last dimension with keepdim (RMSNorm's variance). */
int pim_aten_mean_last(const pim_tensor_view* dst, const pim_tensor_view* src, void* stream);
/* aten.arange: dst[i] = start + i * step (the positions of the exported model). */
int pim_aten_arange(const pim_tensor_view* dst, double start, double step, void* stream);
/* aten.matmul of batched matrices [..., M, K] x [..., K, N] (batch dims broadcast). */
int pim_aten_matmul(const pim_tensor_view* dst, const pim_tensor_view* a, const pim_tensor_view* b, void* stream);
/* aten.scaled_dot_product_attention: q [B, H, S, D], k / v [B, Hk, L, D] (H a multiple of
 * Hk), an additive mask broadcastable to [B, H, S, L] (mask->data NULL or mask NULL for
 * none), causal != 0 for is_causal; at most 8192 keys. */
int pim_aten_sdpa(const pim_tensor_view* out, const pim_tensor_view* q, const pim_tensor_view* k,
                  const pim_tensor_view* v, const pim_tensor_view* mask, double scale, int32_t causal,
                  void* stream);
/* aten.embedding with integer ids of any width; an id outside the table gives a zero
 * row and sets *err_flag (device int32, may be NULL). */
int pim_aten_embedding(const pim_tensor_view* out, const pim_tensor_view* table, const pim_tensor_view* ids,
                       int32_t* err_flag, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PIM_B200_H */
