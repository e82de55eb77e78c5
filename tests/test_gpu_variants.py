"""Kernel variants and extra shapes on the B200 HAL (GPU).

* the dynamic-assignment decode GEMV (``PIM_PROJ_KERNEL_DYNAMIC``): results within the
  GEMV tolerance, identical across calls (units are fixed, only their CTA varies), and
  the work counter back at zero after every launch; the 7B-architecture model vs the
  oracle with it selected;
* the persistent tcgen05 GEMM (``PIM_ROW_BATCH_KERNEL_PERSISTENT``, the default row-batch
  kernel): bit-identical to the one-tile-per-CTA kernel (same MMA order per tile),
  including grids with more tiles than SMs (both TMEM accumulators reused) and ragged
  M / N / K edges;
* ``pim_ordered_sum_add`` (the all_reduce combine with its residual add folded in):
  bit-identical to ``pim_ordered_sum`` followed by ``pim_add``;
* the tcgen05 prefill attention (``PIM_PREFILL_ATTENTION_TCGEN05``): against NumPy and
  the warp-level MMA kernel (causal, GQA, ragged tiles, offsets, several key tiles), with
  no bounded wait giving up, and in the 7B-architecture 200-token prefill vs the oracle;
* the decode attention computed at the end of attn_in (``attn_out`` / ``fuse_attention``):
  equal to attn_in followed by ``pim_attention`` (MHA and GQA, several sequences, two
  calls in a row, counters left at zero), and in the 7B-architecture and tiny models;
* the tiny configuration with grouped-query attention (8 query heads on 2 kv heads,
  head_dim 32) on the B200 HAL vs HF, at TP=1 and 2, and several sequences decoded
  together (tiny at batch 3 vs HF; 7B-architecture at batch 4 and 16 vs the oracle, fed
  the oracle's tokens);
* an HF safetensors checkpoint streamed into the arenas by ``LlamaRunner.load_checkpoint``;
* one launch per decode layer (``pim_decode_layer`` / ``decode_layer``): equal to the five
  launches it replaces (MHA and GQA, head_dim 64 and 128, fp32 and bf16, two calls in a
  row, barrier words, counters and error word checked), and in the 7B-architecture and
  tiny models at TP=1; a barrier wait that runs out;
* one launch per decode step (``pim_decode_step`` / ``decode_step``): the 7B-architecture
  model vs the oracle, the tiny model vs HF, graph replays equal to eager steps.

The tests select the variants explicitly; only the persistent GEMM is a default.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from helpers import cuda_hal, oracle_hal, projection_kernel

pytestmark = pytest.mark.gpu


def _t():
    import torch

    return torch


def _np_dtype(dt):
    from comm.plan import np_dtype

    return np_dtype(dt)


def _dev(a):
    torch = _t()
    if a.dtype.name == "bfloat16":
        return torch.from_numpy(a.view(np.uint16).astype(np.int16)).view(torch.bfloat16).cuda()
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _host(t):
    torch = _t()
    torch.cuda.synchronize()
    if t.dtype == torch.bfloat16:
        import ml_dtypes

        return t.view(torch.int16).cpu().numpy().view(np.uint16).view(ml_dtypes.bfloat16).astype(np.float32)
    return t.cpu().numpy()


def _rnd(x, dt):
    from oracle.kernels import _r

    return _r(x, dt)


def _check(got, ref, tol):
    scale = np.abs(ref).max()
    assert np.abs(got - ref).max() <= tol * scale, (np.abs(got - ref).max(), scale)


# ---- dynamic-assignment GEMV ------------------------------------------------------


def _dynamic_call(a, code, mode):
    """Two launches of the dynamic kernel with its zeroed counter; returns the counter bytes."""
    from backend import _native as nat

    torch = _t()
    need = nat.lib.pim_projection_scratch_bytes(ctypes.byref(a), code, mode)
    assert need >= 8
    ctr = torch.zeros(need, dtype=torch.uint8, device="cuda")
    for _ in range(2):
        nat.check(nat.lib.pim_projection(ctypes.byref(a), code, mode, ctr.data_ptr(), need,
                                         torch.cuda.current_stream().cuda_stream), "dynamic projection")
    torch.cuda.synchronize()
    return ctr


@pytest.mark.parametrize("dt", ["float32", "bfloat16"])
@pytest.mark.parametrize("rows,k,n", [(1, 4096, 4096), (1, 11008, 512), (1, 512, 4096), (4, 256, 688),
                                      (3, 11008, 300), (8, 1000, 40), (1, 64, 7)])
def test_dynamic_projection_plain(dt, rows, k, n):
    from backend import _native as nat

    torch = _t()
    rng = np.random.default_rng(0)
    x = rng.standard_normal((rows, k), dtype=np.float32).astype(_np_dtype(dt))
    w = (rng.standard_normal((n, k), dtype=np.float32) * 0.02).astype(_np_dtype(dt))
    dx, dw = _dev(x), _dev(w)
    code = nat.DTYPE_CODE[dt]
    outs = []
    with projection_kernel("dynamic"):
        for _ in range(2):
            dy = torch.full((rows, n), float("nan"), dtype=dx.dtype, device="cuda")
            a = nat.ProjectionArgs(x=dx.data_ptr(), weight=dw.data_ptr(), out=dy.data_ptr(), rows=rows, k=k,
                                   ncols=n)
            ctr = _dynamic_call(a, code, nat.PROJ_PLAIN)
            assert int(ctr[:8].count_nonzero()) == 0  # the last CTA reset the counter
            outs.append(_host(dy))
    assert np.array_equal(outs[0], outs[1])  # fixed units: the same sums whatever CTA ran them
    ref = _rnd(x.astype(np.float32) @ w.astype(np.float32).T, dt)
    _check(outs[0], ref, 1e-4 if dt == "float32" else 2e-2)


@pytest.mark.parametrize("dt", ["float32", "bfloat16"])
@pytest.mark.parametrize("rows", [1, 5])
def test_dynamic_projection_norm_silu_mul(dt, rows):
    from backend import _native as nat
    from oracle.kernels import rmsnorm

    torch = _t()
    rng = np.random.default_rng(1)
    k, inter = 4096, 1376
    x = rng.standard_normal((rows, k), dtype=np.float32).astype(_np_dtype(dt))
    lw = (1 + 0.1 * rng.standard_normal(k, dtype=np.float32)).astype(_np_dtype(dt))
    w = (rng.standard_normal((2 * inter, k), dtype=np.float32) * 0.02).astype(_np_dtype(dt))
    dx, dl, dw = _dev(x), _dev(lw), _dev(w)
    dy = torch.empty((rows, inter), dtype=dx.dtype, device="cuda")
    a = nat.ProjectionArgs(x=dx.data_ptr(), norm_weight=dl.data_ptr(), weight=dw.data_ptr(), out=dy.data_ptr(),
                           rows=rows, k=k, ncols=2 * inter, eps=1e-5, inter=inter)
    with projection_kernel("dynamic"):
        ctr = _dynamic_call(a, nat.DTYPE_CODE[dt], nat.PROJ_SILU_MUL)
    assert int(ctr[:8].count_nonzero()) == 0
    xn = rmsnorm(x.astype(np.float32), lw.astype(np.float32), 1e-5, dt)
    gu = xn @ w.astype(np.float32).T
    g, u = _rnd(gu[:, 0::2], dt), _rnd(gu[:, 1::2], dt)
    ref = _rnd(_rnd(g / (1 + np.exp(-g)), dt) * u, dt)
    _check(_host(dy), ref, 1e-4 if dt == "float32" else 2e-2)


@pytest.mark.parametrize("tp", [1, 2])
def test_dynamic_kernel_in_the_7b_arch_model_matches_oracle(tp):
    """The plan lowering gives the dynamic kernel its own counter pool: prefill + 3 steps vs the oracle."""
    from graph.llama import ModelConfig
    from runtime.executor import greedy_generate
    from runtime.program import compile_llama, fused_weights, load_weights
    from test_gpu_model import _l7b_weights

    cfg = ModelConfig.llama2_7b(max_seq=32, num_layers=2)
    prog = compile_llama(cfg, tp, batch=1, prompt_len=16)
    w = fused_weights(cfg, _l7b_weights(cfg), tp)
    prompt = np.random.default_rng(1).integers(0, cfg.vocab_size, (1, 16))
    runs = []
    with projection_kernel("dynamic"):
        hal = cuda_hal(prog)
    for h in (hal, oracle_hal(prog)):
        load_weights(prog, h, w)
        runs.append(greedy_generate(prog.plans["prefill"], prog.plans["decode"], h, prompt, 4))
    rc, ro = runs
    assert rc.tokens.tolist() == ro.tokens.tolist()
    for a, b in zip([rc.prefill_logits] + rc.step_logits, [ro.prefill_logits] + ro.step_logits):
        a, b = a.astype(np.float32), b.astype(np.float32)
        assert np.abs(a - b).max() <= 2e-2 * np.abs(b).max()
    assert all(v == 0 for v in hal.read_error_flags().values())


# ---- persistent tcgen05 GEMM -------------------------------------------------------


class _row_batch_kernel:
    def __init__(self, code: int) -> None:
        self.code = code

    def __enter__(self):
        from backend import _native as nat

        self.prev = nat.lib.pim_row_batch_kernel()
        nat.check(nat.lib.pim_set_row_batch_kernel(self.code), "pim_set_row_batch_kernel")

    def __exit__(self, *exc):
        from backend import _native as nat

        nat.lib.pim_set_row_batch_kernel(self.prev)


@pytest.mark.parametrize("rows,k,n,residual", [(300, 520, 1000, False), (256, 4096, 512, True),
                                               (129, 64, 264, True), (2048, 4096, 4096, False),
                                               (4096, 1024, 11008, True)])
def test_persistent_gemm_is_bit_identical_to_the_tile_kernel(rows, k, n, residual):
    from backend import _native as nat

    torch = _t()
    rng = np.random.default_rng(7)
    bf = _np_dtype("bfloat16")
    x = rng.standard_normal((rows, k), dtype=np.float32).astype(bf)
    w = (rng.standard_normal((n, k), dtype=np.float32) * 0.05).astype(bf)
    res = rng.standard_normal((rows, n), dtype=np.float32).astype(bf)
    dx, dw, dr = _dev(x), _dev(w), _dev(res)
    code = nat.DTYPE_CODE["bfloat16"]
    outs = []
    for kernel in (nat.ROW_BATCH_KERNEL_TILE, nat.ROW_BATCH_KERNEL_PERSISTENT):
        dy = torch.full((rows, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        a = nat.ProjectionArgs(x=dx.data_ptr(), weight=dw.data_ptr(), out=dy.data_ptr(), rows=rows, k=k, ncols=n,
                               residual=dr.data_ptr() if residual else None)
        need = nat.lib.pim_projection_scratch_bytes(ctypes.byref(a), code, nat.PROJ_PLAIN)
        scratch = torch.empty(max(need, 1), dtype=torch.uint8, device="cuda")
        with _row_batch_kernel(kernel):
            nat.check(nat.lib.pim_projection(ctypes.byref(a), code, nat.PROJ_PLAIN, scratch.data_ptr(), need,
                                             torch.cuda.current_stream().cuda_stream), "projection")
        outs.append(dy.view(torch.int16).cpu().numpy())
    assert np.array_equal(outs[0], outs[1])
    if rows * n <= 1 << 20:  # and within tolerance of the fp32 product (small cases)
        acc = x.astype(np.float32) @ w.astype(np.float32).T
        ref = _rnd(_rnd(acc, "bfloat16") + res.astype(np.float32), "bfloat16") if residual else _rnd(acc, "bfloat16")
        _check(_host(torch.from_numpy(outs[1]).view(torch.bfloat16)), ref, 2e-2)


def test_persistent_gemm_in_the_7b_arch_long_prefill_matches_oracle():
    from graph.llama import ModelConfig
    from runtime.executor import greedy_generate
    from runtime.program import compile_llama, fused_weights, load_weights
    from test_gpu_model import _l7b_weights

    from backend import _native as nat

    cfg = ModelConfig.llama2_7b(max_seq=256, num_layers=2)
    prog = compile_llama(cfg, 1, batch=1, prompt_len=200)
    w = fused_weights(cfg, _l7b_weights(ModelConfig.llama2_7b(max_seq=32, num_layers=2)), 1)
    prompt = np.random.default_rng(2).integers(0, cfg.vocab_size, (1, 200))
    runs = []
    for h in (cuda_hal(prog), oracle_hal(prog)):
        load_weights(prog, h, w)
        with _row_batch_kernel(nat.ROW_BATCH_KERNEL_PERSISTENT):
            runs.append(greedy_generate(prog.plans["prefill"], prog.plans["decode"], h, prompt, 2))
    rc, ro = runs
    assert rc.tokens.tolist() == ro.tokens.tolist()
    for a, b in zip([rc.prefill_logits] + rc.step_logits, [ro.prefill_logits] + ro.step_logits):
        a, b = a.astype(np.float32), b.astype(np.float32)
        assert np.abs(a - b).max() <= 2e-2 * np.abs(b).max()


# ---- ordered sum + residual add ------------------------------------------------------


@pytest.mark.parametrize("dt", ["float32", "bfloat16"])
@pytest.mark.parametrize("n,nsrc,with_sum", [(4096, 2, False), (4096 * 16, 8, True), (1000, 3, True)])
def test_ordered_sum_add_equals_the_sum_then_the_add(dt, n, nsrc, with_sum):
    from backend import _native as nat

    torch = _t()
    rng = np.random.default_rng(n + nsrc)
    parts = [rng.standard_normal(n, dtype=np.float32).astype(_np_dtype(dt)) for _ in range(nsrc)]
    res = rng.standard_normal(n, dtype=np.float32).astype(_np_dtype(dt))
    dp, dr = [_dev(p) for p in parts], _dev(res)
    code = nat.DTYPE_CODE[dt]
    st = torch.cuda.current_stream().cuda_stream
    s_ref, y_ref = torch.empty_like(dr), torch.empty_like(dr)
    nat.check(nat.lib.pim_ordered_sum(nat.ptr_array([p.data_ptr() for p in dp]), nsrc,
                                      nat.ptr_array([s_ref.data_ptr()]), 1, n, code, 0, st), "sum")
    nat.check(nat.lib.pim_add(s_ref.data_ptr(), dr.data_ptr(), y_ref.data_ptr(), n, code, st), "add")
    y, s = torch.full_like(dr, float("nan")), torch.full_like(dr, float("nan"))
    nat.check(nat.lib.pim_ordered_sum_add(nat.ptr_array([p.data_ptr() for p in dp]), nsrc, dr.data_ptr(),
                                          y.data_ptr(), s.data_ptr() if with_sum else None, n, code, st), "fused")
    torch.cuda.synchronize()
    bits = torch.int16 if dt == "bfloat16" else torch.int32
    assert torch.equal(y.view(bits), y_ref.view(bits))
    if with_sum:
        assert torch.equal(s.view(bits), s_ref.view(bits))


# ---- grouped-query attention, end to end -------------------------------------------


@pytest.mark.parametrize("tp", [1, 2])
def test_tiny_gqa_llama_on_the_b200_hal_matches_hf(tp):
    from graph.llama import ModelConfig
    from helpers import hf_greedy, tiny_gqa_hf_model
    from runtime.executor import greedy_generate
    from runtime.program import compile_llama, fused_weights, hf_state_dict, load_weights

    model = tiny_gqa_hf_model()
    prompt = np.random.default_rng(0).integers(0, 1024, (1, 16))
    toks, logits = hf_greedy(model, prompt, 5)
    cfg = ModelConfig.from_hf(model.config, 32, "float32")
    prog = compile_llama(cfg, tp, batch=1, prompt_len=16)
    hal = cuda_hal(prog)
    load_weights(prog, hal, fused_weights(cfg, hf_state_dict(model, "float32"), tp))
    res = greedy_generate(prog.plans["prefill"], prog.plans["decode"], hal, prompt, 5)
    assert res.tokens[0].tolist() == toks[:len(res.tokens[0])]
    for got, ref in zip([res.prefill_logits] + res.step_logits, logits):
        ref = ref.reshape(-1)
        assert np.abs(got.reshape(-1) - ref).max() <= 1e-4 * np.abs(ref).max()
    assert all(v == 0 for v in hal.read_error_flags().values())


# ---- several sequences at once -------------------------------------------------------


@pytest.mark.parametrize("tp", [1, 2])
def test_tiny_llama_batch_of_three_on_the_b200_hal_matches_hf(tp):
    from helpers import hf_greedy, tiny_hf_model, tiny_program, tiny_weights
    from runtime.executor import greedy_generate
    from runtime.program import load_weights

    model = tiny_hf_model()
    prompts = np.random.default_rng(7).integers(0, 1024, (3, 8))
    prog = tiny_program(tp, batch=3, prompt_len=8)
    hal = cuda_hal(prog)
    load_weights(prog, hal, tiny_weights(prog, model))
    res = greedy_generate(prog.plans["prefill"], prog.plans["decode"], hal, prompts, 4)
    steps = [np.asarray(res.prefill_logits).reshape(3, -1)] + [np.asarray(x).reshape(3, -1) for x in res.step_logits]
    for b in range(3):
        toks, logits = hf_greedy(model, prompts[b:b + 1], 4)
        assert res.tokens[b].tolist() == toks[:len(res.tokens[b])]
        for got, ref in zip(steps, logits):
            assert np.abs(got[b] - ref).max() <= 1e-4 * np.abs(ref).max()


@pytest.mark.parametrize("batch", [4, 16])
def test_7b_arch_batched_decode_matches_oracle(batch):
    """Batched decode as in the batched bench (rows = batch: GEMV at 4, tensor-core GEMMs at 16).

    The oracle decodes greedily; the B200 HAL is fed the oracle's tokens (teacher forcing), so
    each step compares logits computed from the same inputs: within 2e-2, and greedy ids equal
    except where the oracle's two candidates tie at that tolerance."""
    from assert_node_matches_ref import argmax_within_tolerance
    from graph.llama import ModelConfig
    from helpers import forced_generate
    from runtime.executor import greedy_generate
    from runtime.program import compile_llama, fused_weights, load_weights
    from test_gpu_model import _l7b_weights

    cfg = ModelConfig.llama2_7b(max_seq=32, num_layers=2)
    prog = compile_llama(cfg, 1, batch=batch, prompt_len=16)
    w = fused_weights(cfg, _l7b_weights(cfg), 1)
    prompts = np.random.default_rng(5).integers(0, cfg.vocab_size, (batch, 16))
    ho, hc = oracle_hal(prog), cuda_hal(prog)
    for h in (ho, hc):
        load_weights(prog, h, w)
    ro = greedy_generate(prog.plans["prefill"], prog.plans["decode"], ho, prompts, 3)
    got = forced_generate(prog, hc, prompts, ro.tokens[:, :2])
    ties = 0
    for a, b in zip(got, [ro.prefill_logits] + ro.step_logits):
        a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
        assert np.abs(a - b).max() <= 2e-2 * np.abs(b).max()
        gi, ri, tied = argmax_within_tolerance(a, b, 2e-2)
        assert all(g == r or i in tied for i, (g, r) in enumerate(zip(gi, ri))), (gi, ri, tied)
        ties += len(tied)
    assert ties <= batch * 3 // 4  # ties are rare but legitimate; garbage logits fail the bound above


# ---- tcgen05 prefill attention -------------------------------------------------------


class _prefill_attention_kernel:
    def __init__(self, code: int) -> None:
        self.code = code

    def __enter__(self):
        from backend import _native as nat

        self.prev = nat.lib.pim_prefill_attention_kernel()
        nat.check(nat.lib.pim_set_prefill_attention_kernel(self.code), "pim_set_prefill_attention_kernel")

    def __exit__(self, *exc):
        from backend import _native as nat

        nat.lib.pim_set_prefill_attention_kernel(self.prev)


def _prefill_attention(kernel, q, kv, pos, batch, seq, hq, hkv, max_seq):
    from backend import _native as nat

    torch = _t()
    hd = 128
    dq, dkv, dpos = _dev(q), _dev(kv), _dev(pos)
    out = torch.full((batch, seq, hq * hd), float("nan"), dtype=dq.dtype, device="cuda")
    ws_bytes = nat.lib.pim_attention_workspace_bytes(batch, seq, hq, hd, max_seq)
    ws = torch.zeros(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
    with _prefill_attention_kernel(kernel):
        nat.check(nat.lib.pim_attention(dq.data_ptr(), dpos.data_ptr(), dkv.data_ptr(), max_seq * hd,
                                        hkv * 2 * max_seq * hd, out.data_ptr(), batch, seq, hq, hkv, hd, max_seq,
                                        nat.DTYPE_CODE["bfloat16"], ws.data_ptr(), ws_bytes,
                                        torch.cuda.current_stream().cuda_stream))
    return _host(out).reshape(batch, seq, hq, hd)


@pytest.mark.parametrize("batch,seq,hq,hkv,max_seq,pos", [(2, 100, 4, 2, 300, (0, 37)), (1, 64, 2, 2, 64, (0,)),
                                                          (1, 130, 3, 1, 200, (5,)), (3, 16, 2, 2, 40, (24, 0, 9)),
                                                          (2, 512, 4, 4, 600, (0, 50)), (1, 384, 2, 1, 384, (0,))])
def test_tcgen05_prefill_attention_matches_numpy_and_the_mma_kernel(batch, seq, hq, hkv, max_seq, pos):
    """Causal, GQA, ragged query and key tiles, position offsets, several key tiles per row."""
    from backend import _native as nat

    hd, dt = 128, "bfloat16"
    rng = np.random.default_rng(3)
    pos = np.array(pos, dtype=np.int32)
    q = rng.standard_normal((batch, seq, hq * hd), dtype=np.float32).astype(_np_dtype(dt))
    kv = rng.standard_normal((batch, hkv, 2, max_seq, hd), dtype=np.float32).astype(_np_dtype(dt))
    assert nat.lib.pim_attention_errors(1) == 0
    got = _prefill_attention(nat.PREFILL_ATTENTION_TCGEN05, q, kv, pos, batch, seq, hq, hkv, max_seq)
    assert nat.lib.pim_attention_errors(1) == 0  # no wait gave up
    mma = _prefill_attention(nat.PREFILL_ATTENTION_MMA, q, kv, pos, batch, seq, hq, hkv, max_seq)
    assert not np.isnan(got).any()
    qf, kvf = q.astype(np.float32).reshape(batch, seq, hq, hd), kv.astype(np.float32)
    for b in range(batch):
        for h in range(hq):
            kh = h // (hq // hkv)
            ctx = min(pos[b] + seq, max_seq)
            sc = qf[b, :, h] @ kvf[b, kh, 0, :ctx].T / np.sqrt(hd)  # [seq, ctx]
            sc = np.where(np.arange(ctx)[None, :] <= pos[b] + np.arange(seq)[:, None], sc, -np.inf)
            p = np.exp(sc - sc.max(-1, keepdims=True))
            ref = _rnd((p / p.sum(-1, keepdims=True)) @ kvf[b, kh, 1, :ctx], dt)
            for s in range(seq):
                _check(got[b, s, h], ref[s], 2e-2)
                _check(got[b, s, h], mma[b, s, h], 2e-2)


def test_tcgen05_prefill_attention_in_the_7b_arch_long_prefill_matches_oracle():
    from graph.llama import ModelConfig
    from runtime.executor import greedy_generate
    from runtime.program import compile_llama, fused_weights, load_weights
    from test_gpu_model import _l7b_weights

    from backend import _native as nat

    cfg = ModelConfig.llama2_7b(max_seq=256, num_layers=2)
    prog = compile_llama(cfg, 1, batch=1, prompt_len=200)
    w = fused_weights(cfg, _l7b_weights(ModelConfig.llama2_7b(max_seq=32, num_layers=2)), 1)
    prompt = np.random.default_rng(2).integers(0, cfg.vocab_size, (1, 200))
    runs = []
    for h in (cuda_hal(prog), oracle_hal(prog)):
        load_weights(prog, h, w)
        with _prefill_attention_kernel(nat.PREFILL_ATTENTION_TCGEN05):
            runs.append(greedy_generate(prog.plans["prefill"], prog.plans["decode"], h, prompt, 2))
    rc, ro = runs
    assert nat.lib.pim_attention_errors(1) == 0
    assert rc.tokens.tolist() == ro.tokens.tolist()
    for a, b in zip([rc.prefill_logits] + rc.step_logits, [ro.prefill_logits] + ro.step_logits):
        a, b = a.astype(np.float32), b.astype(np.float32)
        assert np.abs(a - b).max() <= 2e-2 * np.abs(b).max()


# ---- decode attention fused into attn_in ----------------------------------------------


@pytest.mark.parametrize("dt", ["float32", "bfloat16"])
@pytest.mark.parametrize("batch,hq,hkv,hd,pos", [(1, 32, 32, 128, (191,)), (3, 8, 2, 64, (5, 0, 40)),
                                                 (2, 4, 1, 128, (63, 17))])
def test_fused_decode_attention_equals_the_attention_kernel(dt, batch, hq, hkv, hd, pos):
    """attn_in with attn_out set == attn_in then pim_attention on what it wrote, twice in a row."""
    from backend import _native as nat

    torch = _t()
    rng = np.random.default_rng(11)
    k, max_seq, code = 512, 96 if max(pos) < 90 else 256, nat.DTYPE_CODE[dt]
    width = (hq + 2 * hkv) * hd
    x = rng.standard_normal((batch, k), dtype=np.float32).astype(_np_dtype(dt))
    lw = np.ones(k, np.float32).astype(_np_dtype(dt))
    w = (rng.standard_normal((width, k), dtype=np.float32) * 0.05).astype(_np_dtype(dt))
    half = hd // 2
    ang = np.arange(max_seq)[:, None] / (10000.0 ** (np.arange(half)[None, :] / half))
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    kv = rng.standard_normal((batch, hkv, 2, max_seq, hd), dtype=np.float32).astype(_np_dtype(dt))
    dx, dl, dw, dc, ds = _dev(x), _dev(lw), _dev(w), _dev(cos), _dev(sin)
    dpos = _dev(np.array(pos, np.int32))
    block, seqs = max_seq * hd, hkv * 2 * max_seq * hd
    outs = []
    for fused in (False, True, True):
        dkv = _dev(kv)
        q = torch.zeros((batch, hq * hd), dtype=dx.dtype, device="cuda")
        att = torch.full((batch, hq * hd), float("nan"), dtype=dx.dtype, device="cuda")
        cnt = torch.zeros(hq, dtype=torch.int32, device="cuda")
        a = nat.ProjectionArgs(x=dx.data_ptr(), norm_weight=dl.data_ptr(), weight=dw.data_ptr(), out=q.data_ptr(),
                               rows=batch, k=k, ncols=width, eps=1e-5, rope_cos=dc.data_ptr(), rope_sin=ds.data_ptr(),
                               positions=dpos.data_ptr(), seq=1, q_heads=hq, kv_heads=hkv, head_dim=hd,
                               max_seq=max_seq, kv_base=dkv.data_ptr(), kv_block_stride=block, kv_seq_stride=seqs,
                               attn_out=att.data_ptr() if fused else None,
                               attn_counters=cnt.data_ptr() if fused else None)
        st = torch.cuda.current_stream().cuda_stream
        calls = 2 if fused else 1  # a second call finds the counters it left at zero
        for _ in range(calls):
            nat.check(nat.lib.pim_projection(ctypes.byref(a), code, nat.PROJ_ROPE_KV, None, 0, st), "attn_in")
        if not fused:
            ws_bytes = nat.lib.pim_attention_workspace_bytes(batch, 1, hq, hd, max_seq)
            ws = torch.zeros(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
            nat.check(nat.lib.pim_attention(q.data_ptr(), dpos.data_ptr(), dkv.data_ptr(), block, seqs, att.data_ptr(),
                                            batch, 1, hq, hkv, hd, max_seq, code, ws.data_ptr(), ws_bytes, st),
                      "attention")
        torch.cuda.synchronize()
        assert int(cnt.count_nonzero()) == 0
        outs.append(_host(att))
    tol = 1e-4 if dt == "float32" else 2e-2
    _check(outs[1], outs[0], tol)
    _check(outs[2], outs[0], tol)


@pytest.mark.parametrize("tp", [1, 2])
def test_fused_decode_attention_in_the_7b_arch_model_matches_oracle(tp):
    from graph.llama import ModelConfig
    from runtime.executor import greedy_generate
    from runtime.program import compile_llama, fused_weights, load_weights
    from test_gpu_model import _l7b_weights

    cfg = ModelConfig.llama2_7b(max_seq=64, num_layers=2)
    prog = compile_llama(cfg, tp, batch=1, prompt_len=16)
    w = fused_weights(cfg, _l7b_weights(ModelConfig.llama2_7b(max_seq=32, num_layers=2)), tp)
    prompt = np.random.default_rng(1).integers(0, cfg.vocab_size, (1, 16))
    hal = cuda_hal(prog, fuse_attention=True)
    assert hal.fused_attentions == 2 * tp  # decode: one per layer and rank
    runs = []
    for h in (hal, oracle_hal(prog)):
        load_weights(prog, h, w)
        runs.append(greedy_generate(prog.plans["prefill"], prog.plans["decode"], h, prompt, 6))
    rc, ro = runs
    assert rc.tokens.tolist() == ro.tokens.tolist()
    for a, b in zip([rc.prefill_logits] + rc.step_logits, [ro.prefill_logits] + ro.step_logits):
        a, b = a.astype(np.float32), b.astype(np.float32)
        assert np.abs(a - b).max() <= 2e-2 * np.abs(b).max()


def test_fused_decode_attention_tiny_llama_matches_hf():
    from helpers import tiny_golden, tiny_hf_model, tiny_program, tiny_weights
    from runtime.executor import greedy_generate
    from runtime.program import load_weights

    gold = tiny_golden()
    prog = tiny_program(2)
    hal = cuda_hal(prog, fuse_attention=True)
    load_weights(prog, hal, tiny_weights(prog, tiny_hf_model()))
    res = greedy_generate(prog.plans["prefill"], prog.plans["decode"], hal, gold["prompt"][None], 8)
    assert res.tokens[0].tolist() == gold["tokens"].tolist()
    for got, ref in zip([res.prefill_logits] + res.step_logits, gold["step_logits"]):
        assert np.abs(got.reshape(-1) - ref).max() <= 1e-4 * np.abs(ref).max()


# ---- HF checkpoint streamed into the device arenas ------------------------------------


def test_runner_load_checkpoint_reproduces_the_hf_golden(tmp_path):
    """save_pretrained -> LlamaRunner.load_checkpoint (memory-mapped, layer by layer) -> HF's tokens."""
    from helpers import tiny_golden, tiny_hf_model, tiny_program
    from runtime.executor import greedy_generate

    gold = tiny_golden()
    tiny_hf_model().save_pretrained(str(tmp_path / "m"), safe_serialization=True)
    prog = tiny_program(1)
    hal = cuda_hal(prog)
    from runtime.session import LlamaRunner

    runner = LlamaRunner(prog, hal)
    runner.load_checkpoint(tmp_path / "m")
    res = greedy_generate(prog.plans["prefill"], prog.plans["decode"], hal, gold["prompt"][None], 8)
    assert res.tokens[0].tolist() == gold["tokens"].tolist()
    for got, ref in zip([res.prefill_logits] + res.step_logits, gold["step_logits"]):
        assert np.abs(got.reshape(-1) - ref).max() <= 1e-4 * np.abs(ref).max()


# ---- one launch per decode layer ------------------------------------------------------


@pytest.mark.parametrize("dt", ["float32", "bfloat16"])
@pytest.mark.parametrize("hq,hkv,hd,pos", [(4, 4, 128, 40), (8, 2, 64, 0), (32, 32, 128, 191)])
def test_decode_layer_equals_the_five_launches(dt, hq, hkv, hd, pos):
    """pim_decode_layer == attn_in, pim_attention, o_proj + residual, mlp_in, down + residual
    launched one by one (same weights), twice in a row; barrier words, counters and the error
    word back where they started."""
    _layer_case(dt, hq, hkv, hd, pos)


def test_a_layer_barrier_wait_that_runs_out_raises_the_error_word_and_the_context_lives_on():
    """A barrier whose arrival count starts far above the grid (no arrival is ever the last)
    makes every wait of the first launch give up: the first after its one-second bound, the
    others at once once the error word is up.  The launch ends, the word reads 1, and the
    same context then runs the layer correctly on fresh barrier words."""
    _layer_case("bfloat16", 8, 2, 128, 40, stuck=True)


def _layer_case(dt, hq, hkv, hd, pos, stuck=False):
    from backend import _native as nat

    torch = _t()
    rng = np.random.default_rng(5)
    hidden, inter, max_seq, code = 512, 688, 256, nat.DTYPE_CODE[dt]
    nd = _np_dtype(dt)
    width = (hq + 2 * hkv) * hd

    def w(n, k):
        return _dev((rng.standard_normal((n, k), dtype=np.float32) * 0.05).astype(nd))

    x = _dev(rng.standard_normal((1, hidden), dtype=np.float32).astype(nd))
    ln1, ln2 = (_dev((1 + 0.1 * rng.standard_normal(hidden, dtype=np.float32)).astype(nd)) for _ in range(2))
    wqkv, wo, wgu, wd = w(width, hidden), w(hidden, hq * hd), w(2 * inter, hidden), w(hidden, inter)
    half = hd // 2
    ang = np.arange(max_seq)[:, None] / (10000.0 ** (np.arange(half)[None, :] / half))
    dc, ds = _dev(np.cos(ang).astype(np.float32)), _dev(np.sin(ang).astype(np.float32))
    dpos = _dev(np.array([pos], np.int32))
    kv0 = rng.standard_normal((hkv, 2, max_seq, hd), dtype=np.float32).astype(nd)
    block, seqs = max_seq * hd, hkv * 2 * max_seq * hd
    st = torch.cuda.current_stream().cuda_stream
    outs = []
    for fused in (False, True):
        dkv = _dev(kv0)
        q = torch.zeros((1, hq * hd), dtype=x.dtype, device="cuda")
        att = torch.zeros((1, hq * hd), dtype=x.dtype, device="cuda")
        h = torch.zeros((1, hidden), dtype=x.dtype, device="cuda")
        act = torch.zeros((1, inter), dtype=x.dtype, device="cuda")
        y = torch.full((1, hidden), float("nan"), dtype=x.dtype, device="cuda")
        cnt = torch.zeros(hq, dtype=torch.int32, device="cuda")
        bar = torch.zeros(nat.DECODE_LAYER_BARRIER_BYTES // 4, dtype=torch.int32, device="cuda")
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        a_in = nat.ProjectionArgs(x=x.data_ptr(), norm_weight=ln1.data_ptr(), weight=wqkv.data_ptr(),
                                  out=q.data_ptr(), rows=1, k=hidden, ncols=width, eps=1e-5, rope_cos=dc.data_ptr(),
                                  rope_sin=ds.data_ptr(), positions=dpos.data_ptr(), seq=1, q_heads=hq, kv_heads=hkv,
                                  head_dim=hd, max_seq=max_seq, kv_base=dkv.data_ptr(), kv_block_stride=block,
                                  kv_seq_stride=seqs, attn_out=att.data_ptr() if fused else None,
                                  attn_counters=cnt.data_ptr() if fused else None)
        a_o = nat.ProjectionArgs(x=att.data_ptr(), weight=wo.data_ptr(), out=h.data_ptr(), rows=1, k=hq * hd,
                                 ncols=hidden, residual=x.data_ptr())
        a_mlp = nat.ProjectionArgs(x=h.data_ptr(), norm_weight=ln2.data_ptr(), weight=wgu.data_ptr(),
                                   out=act.data_ptr(), rows=1, k=hidden, ncols=2 * inter, inter=inter, eps=1e-5)
        a_d = nat.ProjectionArgs(x=act.data_ptr(), weight=wd.data_ptr(), out=y.data_ptr(), rows=1, k=inter,
                                 ncols=hidden, residual=h.data_ptr())
        if fused:
            refs = [ctypes.byref(a) for a in (a_in, a_o, a_mlp, a_d)]
            if stuck:
                bar[0] = 1 << 20
                nat.check(nat.lib.pim_decode_layer(*refs, bar.data_ptr(), err.data_ptr(), code, st), "stuck layer")
                torch.cuda.synchronize()
                assert int(err[0]) == 1
                bar.zero_(), err.zero_(), cnt.zero_()
                dkv.copy_(_dev(kv0))
            for _ in range(2):  # the second call finds the barrier and counters as the first left them
                nat.check(nat.lib.pim_decode_layer(*refs, bar.data_ptr(), err.data_ptr(), code, st), "decode layer")
            torch.cuda.synchronize()
            assert bar[:2].tolist() == [0, 6] and int(err[0]) == 0
            assert int(cnt.count_nonzero()) == 0
        else:
            ws_bytes = nat.lib.pim_attention_workspace_bytes(1, 1, hq, hd, max_seq)
            ws = torch.zeros(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
            nat.check(nat.lib.pim_projection(ctypes.byref(a_in), code, nat.PROJ_ROPE_KV, None, 0, st), "attn_in")
            nat.check(nat.lib.pim_attention(q.data_ptr(), dpos.data_ptr(), dkv.data_ptr(), block, seqs,
                                            att.data_ptr(), 1, 1, hq, hkv, hd, max_seq, code, ws.data_ptr(),
                                            ws_bytes, st), "attention")
            for a, mode in ((a_o, nat.PROJ_PLAIN), (a_mlp, nat.PROJ_SILU_MUL), (a_d, nat.PROJ_PLAIN)):
                nat.check(nat.lib.pim_projection(ctypes.byref(a), code, mode, None, 0, st), "projection")
        outs.append([_host(t) for t in (q, att, h, act, y, dkv)])
    tol = 1e-4 if dt == "float32" else 2e-2
    for got, ref in zip(outs[1], outs[0]):
        _check(got, ref, tol)


def test_decode_layer_in_the_7b_arch_model_matches_oracle():
    from graph.llama import ModelConfig
    from runtime.executor import greedy_generate
    from runtime.program import compile_llama, fused_weights, load_weights
    from test_gpu_model import _l7b_weights

    cfg = ModelConfig.llama2_7b(max_seq=64, num_layers=2)
    prog = compile_llama(cfg, 1, batch=1, prompt_len=16)
    w = fused_weights(cfg, _l7b_weights(ModelConfig.llama2_7b(max_seq=32, num_layers=2)), 1)
    prompt = np.random.default_rng(1).integers(0, cfg.vocab_size, (1, 16))
    hal = cuda_hal(prog, decode_layer=True)
    assert hal.decode_layers == 2
    runs = []
    for h in (hal, oracle_hal(prog)):
        load_weights(prog, h, w)
        runs.append(greedy_generate(prog.plans["prefill"], prog.plans["decode"], h, prompt, 6))
    assert hal.read_error_flags() == {0: 0}
    rc, ro = runs
    assert rc.tokens.tolist() == ro.tokens.tolist()
    for a, b in zip([rc.prefill_logits] + rc.step_logits, [ro.prefill_logits] + ro.step_logits):
        a, b = a.astype(np.float32), b.astype(np.float32)
        assert np.abs(a - b).max() <= 2e-2 * np.abs(b).max()


def test_decode_layer_tiny_llama_matches_hf():
    from helpers import tiny_golden, tiny_hf_model, tiny_program, tiny_weights
    from runtime.executor import greedy_generate
    from runtime.program import load_weights

    gold = tiny_golden()
    prog = tiny_program(1)
    hal = cuda_hal(prog, decode_layer=True)
    assert hal.decode_layers == 2
    load_weights(prog, hal, tiny_weights(prog, tiny_hf_model()))
    res = greedy_generate(prog.plans["prefill"], prog.plans["decode"], hal, gold["prompt"][None], 8)
    assert res.tokens[0].tolist() == gold["tokens"].tolist()
    for got, ref in zip([res.prefill_logits] + res.step_logits, gold["step_logits"]):
        assert np.abs(got.reshape(-1) - ref).max() <= 1e-4 * np.abs(ref).max()


# ---- one launch per decode step --------------------------------------------------------


def test_decode_step_in_the_7b_arch_model_matches_oracle():
    from graph.llama import ModelConfig
    from runtime.executor import greedy_generate
    from runtime.program import compile_llama, fused_weights, load_weights
    from test_gpu_model import _l7b_weights

    cfg = ModelConfig.llama2_7b(max_seq=64, num_layers=2)
    prog = compile_llama(cfg, 1, batch=1, prompt_len=16)
    w = fused_weights(cfg, _l7b_weights(ModelConfig.llama2_7b(max_seq=32, num_layers=2)), 1)
    prompt = np.random.default_rng(1).integers(0, cfg.vocab_size, (1, 16))
    hal = cuda_hal(prog, decode_layer=True, decode_step=True)
    assert hal.decode_steps == 1 and hal.decode_layers == 2
    runs = []
    for h in (hal, oracle_hal(prog)):
        load_weights(prog, h, w)
        runs.append(greedy_generate(prog.plans["prefill"], prog.plans["decode"], h, prompt, 6))
    assert hal.read_error_flags() == {0: 0}
    rc, ro = runs
    assert rc.tokens.tolist() == ro.tokens.tolist()
    for a, b in zip([rc.prefill_logits] + rc.step_logits, [ro.prefill_logits] + ro.step_logits):
        a, b = a.astype(np.float32), b.astype(np.float32)
        assert np.abs(a - b).max() <= 2e-2 * np.abs(b).max()


def test_decode_step_tiny_llama_matches_hf_and_its_graph_replays_equal_eager():
    from helpers import tiny_golden, tiny_hf_model, tiny_program, tiny_weights
    from runtime.executor import bind_inputs, execute_plan, greedy_generate, read_logits, read_tokens
    from runtime.program import load_weights

    gold = tiny_golden()
    prog = tiny_program(1)
    w = tiny_weights(prog, tiny_hf_model())
    hal = cuda_hal(prog, decode_layer=True, decode_step=True)
    assert hal.decode_steps == 1
    load_weights(prog, hal, w)
    res = greedy_generate(prog.plans["prefill"], prog.plans["decode"], hal, gold["prompt"][None], 8)
    assert res.tokens[0].tolist() == gold["tokens"].tolist()
    for got, ref in zip([res.prefill_logits] + res.step_logits, gold["step_logits"]):
        assert np.abs(got.reshape(-1) - ref).max() <= 1e-4 * np.abs(ref).max()
    # the same steps again, eager and as replays of a captured graph (one kernel per step)
    dec = prog.plans["decode"]
    outs = {}
    for name in ("eager", "graph"):
        execute_plan(prog.plans["prefill"], hal, tokens=gold["prompt"][None], pos=np.zeros(1, np.int32))
        tok = read_tokens(prog.plans["prefill"], hal)
        logits = []
        if name == "graph":
            bind_inputs(dec, hal, tokens=tok.reshape(1, 1), pos=np.full(1, 16, np.int32))
            cap = hal.capture(dec)
            logits.append(read_logits(dec, hal))
            for pos in range(17, 20):
                bind_inputs(dec, hal, pos=np.full(1, pos, np.int32))
                cap.replay()
                logits.append(read_logits(dec, hal))
        else:
            for pos in range(16, 20):
                execute_plan(dec, hal, tokens=tok.reshape(1, 1), pos=np.full(1, pos, np.int32))
                logits.append(read_logits(dec, hal))
                tok = read_tokens(dec, hal)
        outs[name] = logits
    for a, b in zip(outs["eager"], outs["graph"]):
        assert np.array_equal(a, b)
    assert hal.read_error_flags() == {0: 0}
