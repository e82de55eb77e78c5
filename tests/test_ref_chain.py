"""The reference's own compile chain feeding this runtime (CPU; the B200 run is marked gpu).

``tests/golden/ref_chain_tiny_tp4.json`` is the tiny LLaMA (``helpers.tiny_hf_model``)
exported with ``torch.export`` (strict) and annotated by the reference's
``partition_graph`` and ``propagate_specs`` at TP=4 (tests/golden/make_ref_chain.py).
``graph.fx_import.decode_graph`` reads it unchanged, ``runtime.fx_program.compile_fx``
runs this runtime's planner, comm plan and plan generator on it, and:

* the fixture is the reference's output (regenerated here when the reference is
  importable, skipped otherwise);
* the oracle HAL runs the plan and reproduces HF's logits for all 16 positions (1e-4)
  and the HF golden's last-position logits;
* the B200 lowering of every aten node is checked on the CPU: each command is lowered
  by ``backend.cuda_aten.lower_aten`` against a fake address space holding the oracle's
  bytes, every view it builds stays inside its buffer, and the C-ABI calls, emulated in
  NumPy, reproduce the oracle's output of the node (no GPU involved);
* on a B200 (``-m gpu``): the plan on ``CudaBackend`` (4 ranks, one GPU) matches HF at
  1e-4 and the oracle node by node (``lockstep_compare``).
"""

from __future__ import annotations

import ctypes
import json
from pathlib import Path

import numpy as np
import pytest

from helpers import tiny_golden, tiny_hf_model

FIXTURE = Path(__file__).resolve().parent / "golden" / "ref_chain_tiny_tp4.json"
REFERENCE = Path("/root/reference")
FP32_TOL = 1e-4


def _graph():
    from graph.fx_import import decode_graph

    return decode_graph(json.loads(FIXTURE.read_text()), name="tiny_tp4")


def _weights():
    model = tiny_hf_model()
    named = list(model.named_parameters()) + list(model.named_buffers())
    return model, {"model." + k: v.detach().numpy() for k, v in named}


def _inputs():
    ids = tiny_golden()["prompt"][None].astype(np.int64)
    s = ids.shape[1]
    mask = np.zeros((1, 1, s, s), np.float32)
    mask[0, 0][np.triu(np.ones((s, s), bool), 1)] = np.finfo(np.float32).min
    return {"input_ids": ids, "causal_mask": mask}


def _hf_logits(model, ids):
    import torch

    with torch.no_grad():
        return model(torch.tensor(ids)).logits.numpy()


def _oracle(prog):
    from oracle.hal_numpy import NumpyBackend, NumpyBackendConfig

    hal = NumpyBackend(NumpyBackendConfig(prog.tp, prog.arena_bytes))
    hal.register_plan(prog.plan)
    return hal


@pytest.mark.skipif(not (REFERENCE / "graph" / "spec_prop.py").exists(), reason="the reference is not importable here")
def test_fixture_is_what_the_reference_passes_produce():
    import subprocess
    import sys

    code = ("import json,sys; sys.path.insert(0, 'tests/golden'); import make_ref_chain as m; "
            "print(json.dumps(m.build()['nodes']))")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600,
                         cwd=FIXTURE.parent.parent.parent)
    assert out.returncode == 0, out.stderr[-2000:]
    fresh = json.loads(out.stdout.strip().splitlines()[-1])
    assert fresh == json.loads(FIXTURE.read_text())["nodes"]


def test_reference_placements_are_kept():
    from graph.fx_import import graph_edges
    from graph.llama import SPEC_META_KEY

    g = _graph()
    edges = graph_edges(g)
    kinds = {k: sum(e.type == k for e in edges) for k in ("scatter", "all_gather", "all_reduce")}
    assert kinds == {"scatter": 46, "all_gather": 29, "all_reduce": 4}  # tests/test_spec_prop.py:328-376 shapes
    dpu_ops = {n.op for n in g.nodes if n.op != "weight" and n.meta[SPEC_META_KEY] is not None
               and n.meta[SPEC_META_KEY].device == "dpu"}
    assert dpu_ops == {"aten.linear", "aten.add.Tensor", "aten.mul.Tensor"}  # graph/partition.py:13-21
    # o_proj / down_proj are row-parallel: Partial outputs, each consumed through an all_reduce
    partial = [n for n in g.nodes if n.meta.get(SPEC_META_KEY) is not None
               and n.meta[SPEC_META_KEY].placement.kind == "Partial"]
    assert len(partial) == 4


def test_oracle_runs_the_reference_compiled_plan_and_matches_hf():
    from runtime.fx_program import compile_fx, load_fx_weights, run_fx

    prog = compile_fx(_graph())
    assert prog.tp == 4
    model, w = _weights()
    hal = _oracle(prog)
    load_fx_weights(prog, hal, w)
    ins = _inputs()
    (logits,) = run_fx(prog, hal, ins).values()
    ref = _hf_logits(model, ins["input_ids"])
    assert np.abs(logits - ref).max() <= FP32_TOL * np.abs(ref).max()
    gold = tiny_golden()["step_logits"][0]
    assert np.abs(logits[0, -1] - gold).max() <= FP32_TOL * np.abs(gold).max()
    assert int(logits[0, -1].argmax()) == int(tiny_golden()["tokens"][0])


# ---------------------------------------------------------------------------------------
# the B200 lowering, emulated on the CPU
# ---------------------------------------------------------------------------------------


class _Memory:
    """Fake device address space: one region per rank arena and one for the host buffer."""

    def __init__(self) -> None:
        self.regions = []  # (base, uint8 array)

    def add(self, base: int, data: np.ndarray) -> int:
        self.regions.append((base, data))
        return base

    def locate(self, addr: int):
        for base, data in self.regions:
            if base <= addr < base + max(len(data), 1):
                return data, addr - base
        raise AssertionError(f"address {addr:#x} outside every buffer")


_DT = {0: np.float32, 2: np.int32, 3: np.int64}


def _array(mem: _Memory, v) -> np.ndarray:
    """The strided NumPy view a pim_tensor_view describes; checks it lies inside its buffer."""
    dt = np.dtype(_DT[v.dtype])
    shape = [int(v.shape[i]) for i in range(v.ndim)]
    strides = [int(v.stride[i]) for i in range(v.ndim)]
    assert v.offset >= 0 and all(s >= 0 for s in strides)
    hi = v.offset + sum((n - 1) * s for n, s in zip(shape, strides)) if all(shape) else 0
    assert hi < v.buffer_elems, (shape, strides, v.offset, v.buffer_elems)
    buf, off = _memory_slice(mem, v.data, v.buffer_elems * dt.itemsize)
    typed = buf[off:off + v.buffer_elems * dt.itemsize].view(dt)
    return np.lib.stride_tricks.as_strided(typed[v.offset:], shape, [s * dt.itemsize for s in strides])


def _memory_slice(mem, addr, nbytes):
    buf, off = mem.locate(addr)
    assert off + nbytes <= len(buf), "buffer runs past its region"
    return buf, off


def _emulate(mem: _Memory, fn, args) -> None:
    name = fn.__name__
    v = [a._obj if isinstance(a, type(ctypes.byref(ctypes.c_int()))) else a for a in args]
    f32 = np.float32
    if name == "pim_aten_copy":
        d, s = _array(mem, v[0]), _array(mem, v[1])
        d[...] = s.astype(d.dtype)
    elif name == "pim_aten_unary":
        op, d, s, sc = v[0], _array(mem, v[1]), _array(mem, v[2]).astype(f32), f32(v[3])
        fns = {0: lambda x: -x, 1: lambda x: f32(1) / np.sqrt(x), 2: np.sqrt, 3: lambda x: x / (f32(1) + np.exp(-x)),
               4: np.cos, 5: np.sin, 6: np.tanh, 7: np.exp, 8: lambda x: f32(1) / x, 9: lambda x: x ** sc,
               10: lambda x: x + sc, 11: lambda x: x * sc, 12: lambda x: x - sc, 13: lambda x: x / sc}
        d[...] = fns[op](s).astype(d.dtype)
    elif name == "pim_aten_binary":
        op, d, a, b = v[0], _array(mem, v[1]), _array(mem, v[2]).astype(f32), _array(mem, v[3]).astype(f32)
        d[...] = {20: np.add, 21: np.subtract, 22: np.multiply, 23: np.divide}[op](a, b).astype(d.dtype)
    elif name == "pim_aten_mean_last":
        d, s = _array(mem, v[0]), _array(mem, v[1]).astype(f32)
        d[...] = s.mean(-1, keepdims=True, dtype=f32).astype(d.dtype)
    elif name == "pim_aten_arange":
        d = _array(mem, v[0])
        d[...] = (v[1] + v[2] * np.arange(d.size)).reshape(d.shape).astype(d.dtype)
    elif name == "pim_aten_matmul":
        d, a, b = _array(mem, v[0]), _array(mem, v[1]).astype(f32), _array(mem, v[2]).astype(f32)
        d[...] = np.matmul(a, b).astype(d.dtype)
    elif name == "pim_aten_sdpa":
        o, q, k, vv = (_array(mem, x).astype(f32) if i else _array(mem, x) for i, x in enumerate(v[:4]))
        s = np.matmul(q, np.swapaxes(np.repeat(k, q.shape[1] // k.shape[1], 1), -1, -2)) * f32(v[5])
        if v[4] is not None:
            s = s + _array(mem, v[4]).astype(f32)
        if v[6]:
            s = np.where(np.tril(np.ones(s.shape[-2:], bool)), s, -np.inf)
        e = np.exp(s - s.max(-1, keepdims=True))
        o[...] = np.matmul(e / e.sum(-1, keepdims=True), np.repeat(vv, q.shape[1] // vv.shape[1], 1))
    elif name == "pim_aten_embedding":
        o, t, ids = _array(mem, v[0]), _array(mem, v[1]), _array(mem, v[2])
        o[...] = t[ids.reshape(-1).astype(np.int64)]
    elif name == "pim_projection":  # PLAIN mode, no norm: y = x . W^T (fp32 here)
        a = v[0]
        rows, k, n = int(a.rows), int(a.k), int(a.ncols)
        (xb, xo), (wb, wo), (yb, yo) = (_memory_slice(mem, p, b) for p, b in
                                        ((a.x, rows * k * 4), (a.weight, n * k * 4), (a.out, rows * n * 4)))
        X = xb[xo:xo + rows * k * 4].view(np.float32).reshape(rows, k)
        W = wb[wo:wo + n * k * 4].view(np.float32).reshape(n, k)
        yb[yo:yo + rows * n * 4].view(np.float32)[...] = (X @ W.T).reshape(-1)
    else:
        raise AssertionError(f"no emulation of {name}")


class _FakeHal:
    local = [0]

    def __init__(self, mem: _Memory) -> None:
        self.mem = mem
        self.scratch_base = mem.add(1 << 46, np.zeros(1 << 22, np.uint8))

    def error_flag_ptr(self, rank):
        return self.scratch_base

    def scratch(self, rank, nbytes, pool=None):
        return self.scratch_base + 4096, nbytes


def test_b200_lowering_of_every_aten_node_emulated_on_cpu():
    """Each aten command of the plan, lowered for the B200 and emulated in NumPy against the
    oracle's bytes (reuse=False keeps every value), reproduces the oracle's output."""
    from backend.cuda_aten import lower_aten
    from runtime.fx_program import compile_fx, load_fx_weights, run_fx

    prog = compile_fx(_graph(), reuse=False)
    _, w = _weights()
    hal = _oracle(prog)
    load_fx_weights(prog, hal, w)
    run_fx(prog, hal, _inputs())
    plan = prog.plan
    arenas = {r: hal.copy_from_dpu(r, 0, (prog.arena_bytes,), np.uint8) for r in range(prog.tp)}
    host = hal.host_arena(plan).copy()
    checked = 0
    for cmd in plan.commands:
        kind = str(cmd.payload.get("kernel", ""))
        if not kind.startswith("aten."):
            continue
        mem = _Memory()
        fake = _FakeHal(mem)
        if cmd.op == "launch":
            base = mem.add(1 << 40, arenas[cmd.dpu_id].copy())
            out_buf = mem.regions[-1][1]
            want = arenas[cmd.dpu_id]
        else:
            base = mem.add(1 << 44, host.copy())
            out_buf = mem.regions[-1][1]
            want = host
        off, shape, dt = cmd.payload["output"]
        nbytes = int(np.prod(shape)) * np.dtype(dt).itemsize
        out_buf[off:off + nbytes] = 0xFF  # every output element must be written
        run = lower_aten(fake, base, 0, cmd.payload, cmd.dpu_id)
        for fn, args in run.calls:
            _emulate(mem, fn, args)
        got = out_buf[off:off + nbytes].view(np.dtype(dt))
        ref = want[off:off + nbytes].view(np.dtype(dt))
        if np.dtype(dt).kind == "f":
            scale = max(float(np.abs(ref).max()), 1e-30)
            assert np.abs(got.astype(np.float64) - ref).max() <= 1e-5 * scale, cmd.payload.get("node")
        else:
            assert np.array_equal(got, ref), cmd.payload.get("node")
        checked += 1
    aten_cmds = [c for c in plan.commands if str(c.payload.get("kernel", "")).startswith("aten.")]
    assert checked == len(aten_cmds) > 250  # DPU nodes on all 4 ranks, and every host node


@pytest.mark.gpu
def test_b200_runs_the_reference_compiled_plan():
    """CudaBackend (TP=4 on one GPU) runs the reference-compiled plan: HF at 1e-4, and node by
    node against the oracle from identical state."""
    from assert_node_matches_ref import lockstep_compare
    from backend import _native as nat
    from backend.hal_cuda import CudaBackend, CudaBackendConfig
    from runtime.fx_program import bind_fx_inputs, compile_fx, load_fx_weights, run_fx

    prog = compile_fx(_graph())
    model, w = _weights()
    hal = CudaBackend(CudaBackendConfig(prog.tp, prog.arena_bytes))
    hal.register_plan(prog.plan)
    load_fx_weights(prog, hal, w)
    ins = _inputs()
    n0 = nat.lib.pim_kernel_launches()
    (logits,) = run_fx(prog, hal, ins).values()
    assert nat.lib.pim_kernel_launches() - n0 > 100  # every node is a device kernel
    ref = _hf_logits(model, ins["input_ids"])
    assert np.abs(logits - ref).max() <= FP32_TOL * np.abs(ref).max()
    # node by node: a second compile for the oracle (it attaches host callables to its plan)
    prog2 = compile_fx(_graph())
    ora = _oracle(prog2)
    load_fx_weights(prog2, ora, w)
    load_fx_weights(prog, hal, w)
    for h, p in ((hal, prog), (ora, prog2)):
        bind_fx_inputs(p, h, ins)
    res = lockstep_compare(prog.plan, hal, ora, ref_plan=prog2.plan)
    bad = [(n, k, v) for n, k, v in res if (k == "rel" and v > FP32_TOL) or (k == "mismatches" and v)]
    assert len(res) > 100 and not bad, bad[:10]
    assert all(v == 0 for v in hal.read_error_flags().values())
    hal.close()
