"""pim_attention_noalloc: attention for callers that cannot allocate device memory (GPU).

Some callers cannot hand pim_attention a workspace -- a plugin whose host program
owns every device allocation through its own pool, or code where a cudaMalloc would
synchronize the device.  pim_attention_noalloc runs the same kernel on a fixed
device array compiled into the library instead.  These tests call it through the C
ABI, twice in a row on the same shape (the second call reuses the array and must
not see the first call's leftovers), and compare each result with pim_attention
given a fresh caller workspace, with the tolerances of the other attention tests.

This file is collected last on purpose (and runs alone as well): a failure here
leaves every other test already run.
"""

from __future__ import annotations


import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = {"float32": 1e-4, "bfloat16": 2e-2}


def _setup(dt, batch, seq, hd, hq, hkv, max_seq):
    import torch

    from comm.plan import np_dtype

    rng = np.random.default_rng(11)
    top = max_seq - 7
    pos = np.array([top - seq + 1 - 3 * b for b in range(batch)], dtype=np.int32)
    q = rng.standard_normal((batch, seq, hq * hd), dtype=np.float32).astype(np_dtype(dt))
    kv = rng.standard_normal((batch, hkv, 2, max_seq, hd), dtype=np.float32).astype(np_dtype(dt))

    def dev(a):
        if a.dtype.name == "bfloat16":
            return torch.from_numpy(a.view(np.uint16).astype(np.int16)).view(torch.bfloat16).cuda()
        return torch.from_numpy(np.ascontiguousarray(a)).cuda()

    return dev(q), dev(kv), dev(pos)


def _host(t):
    import torch

    torch.cuda.synchronize()
    if t.dtype == torch.bfloat16:
        return t.float().cpu().numpy()
    return t.cpu().numpy()


@pytest.mark.parametrize("dt", ["float32", "bfloat16"])
@pytest.mark.parametrize("batch,seq,hd,hq,hkv,max_seq", [(1, 1, 128, 32, 32, 256), (2, 1, 64, 4, 2, 300),
                                                         (1, 6, 128, 4, 4, 64)])
def test_noalloc_attention_matches_workspace_attention_twice(dt, batch, seq, hd, hq, hkv, max_seq):
    import torch

    from backend import _native as nat

    dq, dkv, dpos = _setup(dt, batch, seq, hd, hq, hkv, max_seq)
    st = torch.cuda.current_stream().cuda_stream
    code = nat.DTYPE_CODE[dt]
    common = (dq.data_ptr(), dpos.data_ptr(), dkv.data_ptr(), max_seq * hd, hkv * 2 * max_seq * hd)
    geom = (batch, seq, hq, hkv, hd, max_seq, code)
    ref = torch.empty_like(dq)
    ws_bytes = nat.lib.pim_attention_workspace_bytes(batch, seq, hq, hd, max_seq)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    nat.check(nat.lib.pim_attention(*common, ref.data_ptr(), *geom, ws.data_ptr(), ws_bytes, st), "pim_attention")
    want = _host(ref)
    scale = np.abs(want).max()
    for _ in range(2):
        out = torch.full_like(dq, float("nan"))
        nat.check(nat.lib.pim_attention_noalloc(*common, out.data_ptr(), *geom, st), "pim_attention_noalloc")
        got = _host(out)
        assert np.isfinite(got).all()
        assert np.abs(got - want).max() <= TOL[dt] * scale


def test_noalloc_attention_rejects_shapes_beyond_its_scratch():
    import torch

    from backend import _native as nat

    dq, dkv, dpos = _setup("float32", 1, 1, 64, 2, 2, 16)
    need = nat.lib.pim_attention_workspace_bytes(64, 2048, 32, 128, 4096)
    assert need > 4 * 2**20
    out = torch.empty_like(dq)
    rc = nat.lib.pim_attention_noalloc(dq.data_ptr(), dpos.data_ptr(), dkv.data_ptr(), 16 * 64, 2 * 2 * 16 * 64,
                                       out.data_ptr(), 64, 2048, 32, 32, 128, 4096, nat.F32,
                                       torch.cuda.current_stream().cuda_stream)
    assert rc == 1
    assert b"4 MiB" in nat.lib.pim_last_error()
