"""Each C-ABI kernel against a NumPy statement of the same op (GPU).

Projection and attention shapes include LLaMA2-7B ranks at TP=1 and TP=8 and
the row-batched (prefill) path.  fp32 results must agree to 1e-4 relative;
bf16 results to 2e-2 relative (one bf16 rounding of the output plus fp32
accumulation-order differences).
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from helpers import PROJECTION_KERNELS, projection_kernel

pytestmark = pytest.mark.gpu


def _t():
    import torch

    return torch


def _dev(a):
    torch = _t()
    if a.dtype.name == "bfloat16":
        return torch.from_numpy(a.view(np.uint16).astype(np.int16)).view(torch.bfloat16).cuda()
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _host(t, bf16=False):
    torch = _t()
    torch.cuda.synchronize()
    if bf16:
        import ml_dtypes

        return t.view(torch.int16).cpu().numpy().view(np.uint16).view(ml_dtypes.bfloat16).astype(np.float32)
    return t.cpu().numpy()


def _rnd(x, dt):
    from oracle.kernels import _r

    return _r(x, dt)


def _check(got, ref, tol):
    scale = np.abs(ref).max()
    assert np.abs(got - ref).max() <= tol * scale, (np.abs(got - ref).max(), scale)


def _np_dtype(dt):
    from comm.plan import np_dtype

    return np_dtype(dt)


@pytest.mark.parametrize("kernel", PROJECTION_KERNELS)
@pytest.mark.parametrize("dt", ["float32", "bfloat16"])
@pytest.mark.parametrize("rows,k,n", [(1, 4096, 4096), (1, 11008, 512), (1, 512, 4096), (4, 256, 688),
                                      (3, 11008, 300), (8, 1000, 40), (32, 256, 1024)])
def test_projection_plain(kernel, dt, rows, k, n):
    from backend import _native as nat

    torch = _t()
    rng = np.random.default_rng(0)
    x = (rng.standard_normal((rows, k), dtype=np.float32)).astype(_np_dtype(dt))
    w = (rng.standard_normal((n, k), dtype=np.float32) * 0.02).astype(_np_dtype(dt))
    dx, dw = _dev(x), _dev(w)
    dy = torch.empty((rows, n), dtype=dx.dtype, device="cuda")
    a = nat.ProjectionArgs(x=dx.data_ptr(), weight=dw.data_ptr(), out=dy.data_ptr(), rows=rows, k=k, ncols=n)
    code = nat.DTYPE_CODE[dt]
    need = nat.lib.pim_projection_scratch_bytes(ctypes.byref(a), code, nat.PROJ_PLAIN)
    scratch = torch.empty(max(need, 1), dtype=torch.uint8, device="cuda")
    with projection_kernel(kernel):
        nat.check(nat.lib.pim_projection(ctypes.byref(a), code, nat.PROJ_PLAIN, scratch.data_ptr(), need,
                                         torch.cuda.current_stream().cuda_stream))
    ref = _rnd(x.astype(np.float32) @ w.astype(np.float32).T, dt)
    _check(_host(dy, dt == "bfloat16"), ref, 1e-4 if dt == "float32" else 2e-2)


@pytest.mark.parametrize("rows,k,n,residual", [(300, 520, 1000, False), (256, 4096, 512, True), (129, 64, 264, True),
                                               (1024, 1024, 768, False)])
def test_row_batch_tensor_core_gemm(rows, k, n, residual):
    """bf16 row batches (rows > 8) run on the tcgen05 GEMM: tile edges in M, N and K, fused residual."""
    from backend import _native as nat

    torch = _t()
    rng = np.random.default_rng(7)
    bf = _np_dtype("bfloat16")
    x = rng.standard_normal((rows, k), dtype=np.float32).astype(bf)
    w = (rng.standard_normal((n, k), dtype=np.float32) * 0.05).astype(bf)
    res = rng.standard_normal((rows, n), dtype=np.float32).astype(bf)
    dx, dw, dr = _dev(x), _dev(w), _dev(res)
    dy = torch.empty((rows, n), dtype=torch.bfloat16, device="cuda")
    a = nat.ProjectionArgs(x=dx.data_ptr(), weight=dw.data_ptr(), out=dy.data_ptr(), rows=rows, k=k, ncols=n,
                           residual=dr.data_ptr() if residual else None)
    code = nat.DTYPE_CODE["bfloat16"]
    need = nat.lib.pim_projection_scratch_bytes(ctypes.byref(a), code, nat.PROJ_PLAIN)
    scratch = torch.empty(max(need, 1), dtype=torch.uint8, device="cuda")
    n0 = nat.lib.pim_kernel_launches()
    nat.check(nat.lib.pim_projection(ctypes.byref(a), code, nat.PROJ_PLAIN, scratch.data_ptr(), need,
                                     torch.cuda.current_stream().cuda_stream))
    assert nat.lib.pim_kernel_launches() - n0 == 1  # one fused kernel, no separate epilogue
    acc = x.astype(np.float32) @ w.astype(np.float32).T
    ref = _rnd(_rnd(acc, "bfloat16") + res.astype(np.float32), "bfloat16") if residual else _rnd(acc, "bfloat16")
    _check(_host(dy, True), ref, 2e-2)


@pytest.mark.parametrize("kernel", PROJECTION_KERNELS)
@pytest.mark.parametrize("rows", [1, 3])
def test_bf16_products_are_exact(kernel, rows):
    """Each bf16 product enters the fp32 sum unrounded.

    Pairs of products (1+2^-7)^2 and -(1+2^-6) leave 2^-14 each; every partial sum is an
    exact multiple of 2^-14 in fp32 whatever the summation order, so the dot product of
    4096 elements is exactly 0.125.  Rounding a product to bf16 would give 0.
    """
    import ml_dtypes

    from backend import _native as nat

    torch = _t()
    k, n = 4096, 300
    bf = ml_dtypes.bfloat16
    w = np.tile(np.array([1 + 2 ** -7, -1.0], np.float32), k // 2).astype(bf)
    x = np.tile(np.array([1 + 2 ** -7, 1 + 2 ** -6], np.float32), k // 2).astype(bf)
    dx, dw = _dev(np.tile(x, (rows, 1))), _dev(np.tile(w, (n, 1)))
    dy = torch.empty((rows, n), dtype=torch.bfloat16, device="cuda")
    a = nat.ProjectionArgs(x=dx.data_ptr(), weight=dw.data_ptr(), out=dy.data_ptr(), rows=rows, k=k, ncols=n)
    with projection_kernel(kernel):
        nat.check(nat.lib.pim_projection(ctypes.byref(a), nat.DTYPE_CODE["bfloat16"], nat.PROJ_PLAIN, None, 0,
                                         torch.cuda.current_stream().cuda_stream))
    assert np.all(_host(dy, True) == 0.125)


@pytest.mark.parametrize("kernel", PROJECTION_KERNELS)
@pytest.mark.parametrize("dt", ["float32", "bfloat16"])
@pytest.mark.parametrize("rows", [1, 5, 16])
def test_projection_norm_silu_mul(kernel, dt, rows):
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
    code = nat.DTYPE_CODE[dt]
    need = nat.lib.pim_projection_scratch_bytes(ctypes.byref(a), code, nat.PROJ_SILU_MUL)
    scratch = torch.empty(max(need, 1), dtype=torch.uint8, device="cuda")
    with projection_kernel(kernel):
        nat.check(nat.lib.pim_projection(ctypes.byref(a), code, nat.PROJ_SILU_MUL, scratch.data_ptr(), need,
                                         torch.cuda.current_stream().cuda_stream))
    xn = rmsnorm(x.astype(np.float32), lw.astype(np.float32), 1e-5, dt)
    gu = xn @ w.astype(np.float32).T
    g, u = _rnd(gu[:, 0::2], dt), _rnd(gu[:, 1::2], dt)  # rows interleaved gate_j, up_j
    ref = _rnd(_rnd(g / (1 + np.exp(-g)), dt) * u, dt)
    _check(_host(dy, dt == "bfloat16"), ref, 1e-4 if dt == "float32" else 2e-2)


@pytest.mark.parametrize("dt", ["float32", "bfloat16"])
@pytest.mark.parametrize("batch,seq,hd,hq,hkv", [(1, 1, 128, 4, 4), (2, 1, 64, 4, 2), (1, 5, 64, 2, 2),
                                                 (1, 12, 128, 2, 2)])
@pytest.mark.parametrize("max_seq", [48, 300])  # one key split / several splits merged by the last CTA
def test_attention_over_kv_blocks(dt, batch, seq, hd, hq, hkv, max_seq):
    from backend import _native as nat

    torch = _t()
    rng = np.random.default_rng(2)
    top = max_seq - 18
    pos = np.array([top - seq + 1 - b * 3 for b in range(batch)], dtype=np.int32)
    q = rng.standard_normal((batch, seq, hq * hd), dtype=np.float32).astype(_np_dtype(dt))
    # layout: [seq b][kv head][k|v][max_seq][hd]
    kv = rng.standard_normal((batch, hkv, 2, max_seq, hd), dtype=np.float32).astype(_np_dtype(dt))
    dq, dkv, dpos = _dev(q), _dev(kv), _dev(pos)
    out = torch.empty((batch, seq, hq * hd), dtype=dq.dtype, device="cuda")
    ws_bytes = nat.lib.pim_attention_workspace_bytes(batch, seq, hq, hd, max_seq)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")  # the row tickets start at zero
    outs = []
    for _ in range(2):  # the second call reuses the workspace: the row tickets must have been reset
        nat.check(nat.lib.pim_attention(dq.data_ptr(), dpos.data_ptr(), dkv.data_ptr(), max_seq * hd,
                                        hkv * 2 * max_seq * hd, out.data_ptr(), batch, seq, hq, hkv, hd, max_seq,
                                        nat.DTYPE_CODE[dt], ws.data_ptr(), ws_bytes,
                                        torch.cuda.current_stream().cuda_stream))
        outs.append(_host(out, dt == "bfloat16"))
        out.zero_()
    assert np.array_equal(outs[0], outs[1])
    got = outs[0].reshape(batch, seq, hq, hd)
    qf, kvf = q.astype(np.float32).reshape(batch, seq, hq, hd), kv.astype(np.float32)
    for b in range(batch):
        for s in range(seq):
            ctx = pos[b] + s + 1
            for h in range(hq):
                kh = h // (hq // hkv)
                sc = kvf[b, kh, 0, :ctx] @ qf[b, s, h] / np.sqrt(hd)
                p = np.exp(sc - sc.max())
                ref = _rnd((p / p.sum()) @ kvf[b, kh, 1, :ctx], dt)
                _check(got[b, s, h], ref, 1e-4 if dt == "float32" else 2e-2)


@pytest.mark.parametrize("batch,seq,hq,hkv,max_seq,pos", [(2, 100, 4, 2, 300, (0, 37)), (1, 64, 2, 2, 64, (0,)),
                                                          (1, 130, 3, 1, 200, (5,)), (3, 16, 2, 2, 40, (24, 0, 9))])
def test_prefill_attention_tensor_cores(batch, seq, hq, hkv, max_seq, pos):
    """bf16 row batches with head_dim 128 (flash-style mma.sync kernel): causal, GQA, ragged tiles, offsets."""
    from backend import _native as nat

    torch = _t()
    hd, dt = 128, "bfloat16"
    rng = np.random.default_rng(3)
    pos = np.array(pos, dtype=np.int32)
    q = rng.standard_normal((batch, seq, hq * hd), dtype=np.float32).astype(_np_dtype(dt))
    kv = rng.standard_normal((batch, hkv, 2, max_seq, hd), dtype=np.float32).astype(_np_dtype(dt))
    dq, dkv, dpos = _dev(q), _dev(kv), _dev(pos)
    out = torch.zeros((batch, seq, hq * hd), dtype=dq.dtype, device="cuda")
    ws_bytes = nat.lib.pim_attention_workspace_bytes(batch, seq, hq, hd, max_seq)
    ws = torch.zeros(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
    nat.check(nat.lib.pim_attention(dq.data_ptr(), dpos.data_ptr(), dkv.data_ptr(), max_seq * hd,
                                    hkv * 2 * max_seq * hd, out.data_ptr(), batch, seq, hq, hkv, hd, max_seq,
                                    nat.DTYPE_CODE[dt], ws.data_ptr(), ws_bytes,
                                    torch.cuda.current_stream().cuda_stream))
    got = _host(out, True).reshape(batch, seq, hq, hd)
    qf, kvf = q.astype(np.float32).reshape(batch, seq, hq, hd), kv.astype(np.float32)
    for b in range(batch):
        for h in range(hq):
            kh = h // (hq // hkv)
            ctx = pos[b] + seq
            sc = qf[b, :, h] @ kvf[b, kh, 0, :ctx].T / np.sqrt(hd)  # [seq, ctx]
            sc = np.where(np.arange(ctx)[None, :] <= pos[b] + np.arange(seq)[:, None], sc, -np.inf)
            p = np.exp(sc - sc.max(-1, keepdims=True))
            ref = _rnd((p / p.sum(-1, keepdims=True)) @ kvf[b, kh, 1, :ctx], dt)
            for s in range(seq):
                _check(got[b, s, h], ref[s], 2e-2)


def test_ordered_sum_is_sequential_bf16_rne():
    import ml_dtypes

    from backend import _native as nat

    torch = _t()
    rng = np.random.default_rng(3)
    parts = [rng.standard_normal(1 << 16, dtype=np.float32).astype(ml_dtypes.bfloat16) for _ in range(8)]
    dev = [_dev(p) for p in parts]
    out = torch.empty(1 << 16, dtype=torch.bfloat16, device="cuda")
    nat.check(nat.lib.pim_ordered_sum(nat.ptr_array([d.data_ptr() for d in dev]), 8, nat.ptr_array([out.data_ptr()]),
                                      1, 1 << 16, nat.BF16, 0, torch.cuda.current_stream().cuda_stream))
    acc = np.zeros(1 << 16, ml_dtypes.bfloat16)
    for p in parts:
        acc += p
    torch.cuda.synchronize()
    assert np.array_equal(out.view(torch.int16).cpu().numpy().view(np.uint16), acc.view(np.uint16))


def test_argmax_embedding_add_select():
    from backend import _native as nat

    torch = _t()
    st = torch.cuda.current_stream().cuda_stream
    x = torch.randn(3, 32000, device="cuda")
    x[1, 7] = 100.0
    x[1, 9] = 100.0  # tie: the first index wins, as numpy.argmax
    idx = torch.empty(3, dtype=torch.int32, device="cuda")
    nat.check(nat.lib.pim_argmax(x.data_ptr(), idx.data_ptr(), 3, 32000, nat.F32, st))
    assert idx.cpu().tolist() == np.argmax(x.cpu().numpy(), axis=1).tolist()
    table = torch.randn(10, 16, device="cuda")
    ids = torch.tensor([3, 0, 11, 9], dtype=torch.int32, device="cuda")
    out = torch.empty(4, 16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    nat.check(nat.lib.pim_embedding(ids.data_ptr(), table.data_ptr(), out.data_ptr(), 4, 16, 10, nat.F32,
                                    err.data_ptr(), st))
    torch.cuda.synchronize()
    assert torch.equal(out[[0, 1, 3]], table[[3, 0, 9]]) and torch.all(out[2] == 0) and err.item() == 1
    a, b = torch.randn(1000, device="cuda"), torch.randn(1000, device="cuda")
    y = torch.empty_like(a)
    nat.check(nat.lib.pim_add(a.data_ptr(), b.data_ptr(), y.data_ptr(), 1000, nat.F32, st))
    h = torch.randn(2, 5, 8, device="cuda")
    sel = torch.empty(2, 8, device="cuda")
    nat.check(nat.lib.pim_select_rows(h.data_ptr(), sel.data_ptr(), 2, 5, 32, 4, st))
    torch.cuda.synchronize()
    assert torch.equal(y, a + b) and torch.equal(sel, h[:, 4])


def test_p2p_allreduce_wait_for_a_missing_peer_times_out_with_an_error_word():
    """A peer that never raises its flag: the bounded wait gives up (~1 s), raises the error
    word, skips the sum, consumes the epoch (the counter still advances, keeping ranks in
    step), and the context keeps working."""
    import time

    from backend import _native as nat

    torch = _t()
    numel, cap = 4096, 256 << 10
    me = torch.zeros(1024 + 2 * 2 * cap, dtype=torch.uint8, device="cuda")
    ghost = torch.zeros_like(me)  # "rank 1": local memory nobody writes a flag into
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    src = torch.ones(numel, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros_like(src)
    t0 = time.time()
    nat.check(nat.lib.pim_allreduce_p2p(src.data_ptr(), nat.ptr_array([out.data_ptr()]), 1, numel,
                                        nat.DTYPE_CODE["bfloat16"], 0, 2, nat.ptr_array([me.data_ptr(), ghost.data_ptr()]),
                                        cap, counter.data_ptr(), err.data_ptr(),
                                        torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert time.time() - t0 < 30
    assert int(err.item()) == 1 and int(counter.item()) == 1 and int(out.abs().sum().item()) == 0
    assert torch.equal(src + src, torch.full_like(src, 2.0))  # the context still runs kernels


def test_p2p_ll_allreduce_wait_for_a_missing_peer_times_out_with_an_error_word():
    """The low-latency protocol with a peer whose tagged words never arrive: every poll
    gives up together (~1 s, not 1 s per word), the error word is raised, nothing is
    written, the epoch is consumed and the context keeps working."""
    import time

    from backend import _native as nat

    torch = _t()
    numel, cap = 16384, 256 << 10  # 32 KB of bf16: 16 words per thread of the 512
    me = torch.zeros(1024 + 2 * 2 * cap, dtype=torch.uint8, device="cuda")
    ghost = torch.zeros_like(me)  # "rank 1": local memory nobody writes a word into
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    src = torch.ones(numel, dtype=torch.bfloat16, device="cuda")
    resid = torch.ones_like(src)
    out, y = torch.zeros_like(src), torch.zeros_like(src)
    t0 = time.time()
    nat.check(nat.lib.pim_allreduce_p2p_ll(src.data_ptr(), resid.data_ptr(), y.data_ptr(), out.data_ptr(), numel,
                                           nat.DTYPE_CODE["bfloat16"], 0, 2,
                                           nat.ptr_array([me.data_ptr(), ghost.data_ptr()]), cap,
                                           counter.data_ptr(), err.data_ptr(),
                                           torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert time.time() - t0 < 10
    assert int(err.item()) == 1 and int(counter.item()) == 1
    assert int(out.abs().sum().item()) == 0 and int(y.abs().sum().item()) == 0
    assert torch.equal(src + src, torch.full_like(src, 2.0))  # the context still runs kernels
