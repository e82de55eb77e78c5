"""pim_attention_noalloc: attention for callers that cannot allocate device memory (GPU).

Some callers cannot hand pim_attention a workspace -- a plugin whose host program
owns every device allocation through its own pool, or code where a cudaMalloc would
synchronize the device.  pim_attention_noalloc runs the same kernels on a fixed
device array compiled into the library instead.  These tests call it through the C
ABI and compare each result with pim_attention given a fresh caller workspace and
with a NumPy statement of the attention (fp32 scores and softmax over keys 0..pos,
output rounded to the storage type), with the tolerances of the other attention tests:

* twice in a row on the same shape (the second call reuses the array and must not see
  the first call's leftovers);
* a large shape and then a small one, so that the small call's row tickets lie inside
  the large call's partial results (the case the per-call ticket clearing is for);
* a bf16 row batch that the tensor-core kernel runs without any workspace, accepted
  although the split-K workspace of its shape would exceed the 4 MiB array.

This file is collected last on purpose (and runs alone as well): a failure here
leaves every other test already run.
"""

from __future__ import annotations


import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = {"float32": 1e-4, "bfloat16": 2e-2}


def _host(t):
    import torch

    torch.cuda.synchronize()
    if t.dtype == torch.bfloat16:
        return t.float().cpu().numpy()
    return t.cpu().numpy()


def _reference(q, kv, pos, hq, hkv, hd, dt):
    """NumPy attention over the [batch][kv head][k|v][max_seq][hd] blocks, causal within a row batch."""
    from comm.plan import np_dtype

    batch, seq = q.shape[0], q.shape[1]
    qf, kvf = q.astype(np.float32).reshape(batch, seq, hq, hd), kv.astype(np.float32)
    out = np.zeros((batch, seq, hq, hd), np.float32)
    for b in range(batch):
        for h in range(hq):
            kh = h // (hq // hkv)
            ctx = int(pos[b]) + seq
            sc = qf[b, :, h] @ kvf[b, kh, 0, :ctx].T / np.sqrt(hd)
            sc = np.where(np.arange(ctx)[None, :] <= int(pos[b]) + np.arange(seq)[:, None], sc, -np.inf)
            p = np.exp(sc - sc.max(-1, keepdims=True))
            out[b, :, h] = (p / p.sum(-1, keepdims=True)) @ kvf[b, kh, 1, :ctx]
    return out.astype(np_dtype(dt)).astype(np.float32).reshape(batch, seq, hq * hd)


def _case(dt, batch, seq, hd, hq, hkv, max_seq, seed=11):
    import torch

    from comm.plan import np_dtype

    rng = np.random.default_rng(seed)
    top = max_seq - 7
    pos = np.array([max(top - seq + 1 - 3 * b, 0) for b in range(batch)], dtype=np.int32)
    q = rng.standard_normal((batch, seq, hq * hd), dtype=np.float32).astype(np_dtype(dt))
    kv = rng.standard_normal((batch, hkv, 2, max_seq, hd), dtype=np.float32).astype(np_dtype(dt))

    def dev(a):
        if a.dtype.name == "bfloat16":
            return torch.from_numpy(a.view(np.uint16).astype(np.int16)).view(torch.bfloat16).cuda()
        return torch.from_numpy(np.ascontiguousarray(a)).cuda()

    return (q, kv, pos), (dev(q), dev(kv), dev(pos))


def _call(fn_name, dt, dq, dkv, dpos, batch, seq, hd, hq, hkv, max_seq, ws=None):
    """One attention call through the C ABI; returns the output on the host (fp32)."""
    import torch

    from backend import _native as nat

    st = torch.cuda.current_stream().cuda_stream
    out = torch.full_like(dq, float("nan"))
    common = (dq.data_ptr(), dpos.data_ptr(), dkv.data_ptr(), max_seq * hd, hkv * 2 * max_seq * hd, out.data_ptr(),
              batch, seq, hq, hkv, hd, max_seq, nat.DTYPE_CODE[dt])
    if fn_name == "pim_attention":
        ws_bytes = nat.lib.pim_attention_workspace_bytes(batch, seq, hq, hd, max_seq)
        ws = torch.zeros(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")  # fresh: tickets at zero
        nat.check(nat.lib.pim_attention(*common, ws.data_ptr(), ws_bytes, st), fn_name)
    else:
        nat.check(nat.lib.pim_attention_noalloc(*common, st), fn_name)
    return _host(out)


def _check_against_both(got, want_ws, want_np, dt):
    assert np.isfinite(got).all()
    scale = np.abs(want_np).max()
    assert np.abs(got - want_ws).max() <= TOL[dt] * scale
    assert np.abs(got - want_np).max() <= TOL[dt] * scale


@pytest.mark.parametrize("dt", ["float32", "bfloat16"])
@pytest.mark.parametrize("batch,seq,hd,hq,hkv,max_seq", [(1, 1, 128, 32, 32, 256), (2, 1, 64, 4, 2, 300),
                                                         (1, 6, 128, 4, 4, 64)])
def test_noalloc_attention_matches_workspace_attention_twice(dt, batch, seq, hd, hq, hkv, max_seq):
    host, dev = _case(dt, batch, seq, hd, hq, hkv, max_seq)
    geom = (batch, seq, hd, hq, hkv, max_seq)
    want_ws = _call("pim_attention", dt, *dev, *geom)
    want_np = _reference(*host, hq, hkv, hd, dt)
    for _ in range(2):
        _check_against_both(_call("pim_attention_noalloc", dt, *dev, *geom), want_ws, want_np, dt)


@pytest.mark.parametrize("dt", ["float32", "bfloat16"])
def test_noalloc_attention_large_then_small_shape(dt):
    """The small call's tickets sit where the large call left partial results: they must be cleared."""
    big = (1, 1, 128, 32, 32, 256)
    small = (2, 1, 64, 4, 2, 300)
    host_b, dev_b = _case(dt, *big, seed=21)
    host_s, dev_s = _case(dt, *small, seed=22)
    _check_against_both(_call("pim_attention_noalloc", dt, *dev_b, *big), _call("pim_attention", dt, *dev_b, *big),
                        _reference(*host_b, big[3], big[4], big[2], dt), dt)
    want_ws = _call("pim_attention", dt, *dev_s, *small)
    want_np = _reference(*host_s, small[3], small[4], small[2], dt)
    for _ in range(2):
        _check_against_both(_call("pim_attention_noalloc", dt, *dev_s, *small), want_ws, want_np, dt)


def test_noalloc_attention_runs_workspace_free_row_batches_of_any_size():
    """bf16, head_dim 128, 128 query rows per sequence: the tensor-core kernel, no scratch used."""
    from backend import _native as nat

    geom = (4, 128, 128, 32, 32, 512)  # batch, seq, hd, hq, hkv, max_seq
    assert nat.lib.pim_attention_workspace_bytes(4, 128, 32, 128, 512) > 4 * 2**20
    host, dev = _case("bfloat16", *geom, seed=23)
    want_ws = _call("pim_attention", "bfloat16", *dev, *geom)
    want_np = _reference(*host, 32, 32, 128, "bfloat16")
    _check_against_both(_call("pim_attention_noalloc", "bfloat16", *dev, *geom), want_ws, want_np, "bfloat16")


def test_noalloc_attention_rejects_shapes_beyond_its_scratch():
    import torch

    from backend import _native as nat

    _, (dq, dkv, dpos) = _case("float32", 1, 1, 64, 2, 2, 16)
    need = nat.lib.pim_attention_workspace_bytes(64, 2048, 32, 128, 4096)
    assert need > 4 * 2**20
    out = torch.empty_like(dq)
    rc = nat.lib.pim_attention_noalloc(dq.data_ptr(), dpos.data_ptr(), dkv.data_ptr(), 16 * 64, 2 * 2 * 16 * 64,
                                       out.data_ptr(), 64, 2048, 32, 32, 128, 4096, nat.F32,
                                       torch.cuda.current_stream().cuda_stream)
    assert rc == 1
    assert b"4 MiB" in nat.lib.pim_last_error()
