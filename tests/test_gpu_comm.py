"""Redistribute microbench parity (config 5) on the B200 HAL (GPU).

Ranks are simulated as arenas of one process; the device collectives must be
bit-identical to the reference's host-star lowering (golden hashes) and to the
oracle at every size of the microbench, T in {1, 16, 256, 2048}.
"""

from __future__ import annotations

import json

import numpy as np
import pytest

from helpers import GOLDEN, comm_inputs, redistribute_entry, sha

pytestmark = pytest.mark.gpu

COMM = json.loads((GOLDEN / "comm_golden.json").read_text())


def _hal(n, nbytes):
    from backend.hal_cuda import CudaBackend, CudaBackendConfig

    return CudaBackend(CudaBackendConfig(n, 4 * nbytes))


def _load(kind, hal, entry, n, t, data):
    if kind == "all_reduce":
        for d, p in enumerate(data):
            hal.copy_to_dpu(d, 0, p.reshape(-1))
    elif kind == "all_gather":
        w = 4096 // n
        for d in range(n):
            hal.copy_to_dpu(d, 0, np.ascontiguousarray(data[:, d * w:(d + 1) * w]).reshape(-1))
    else:
        r = t // n
        for d in range(n):
            hal.copy_to_dpu(d, 0, np.ascontiguousarray(data[d * r:(d + 1) * r, :]).reshape(-1))


@pytest.mark.parametrize("case", COMM["cases"], ids=[c["key"] for c in COMM["cases"]])
def test_device_redistribute_matches_reference_bit_exact(case):
    from backend import cuda_collectives as cc

    n, t, kind = case["n"], case["tokens"], case["type"]
    entry, nbytes = redistribute_entry(kind, n, (t, 4096))
    hal = _hal(n, nbytes)
    data = comm_inputs(kind, n, t)
    _load(kind, hal, entry, n, t, data)
    out = getattr(cc, kind)(entry, cc.CudaDmaEngine(hal))
    assert sha(out) == case["out_sha"]
    if kind == "all_reduce":
        for d in range(n):
            assert sha(hal.read_local(d, nbytes, (t * 4096,), entry.dtype)) == case["out_sha"]
    if kind == "all_to_all":
        for d in range(n):
            assert sha(hal.read_local(d, nbytes, (t * 4096 // n,), entry.dtype)) == case["dst_local_sha"][d]


@pytest.mark.parametrize("n", [2, 4, 8])
@pytest.mark.parametrize("t", [1, 2048])
@pytest.mark.parametrize("kind", ["all_reduce", "all_gather", "all_to_all"])
def test_device_redistribute_matches_oracle_at_microbench_sizes(kind, t, n):
    from backend import cuda_collectives as cc
    from oracle import lowering
    from oracle.hal_numpy import NumpyBackend, NumpyBackendConfig

    if kind == "all_to_all" and t % n:
        pytest.skip("Shard(0) of T=1 over N>1 ranks is undefined in the reference (dim not divisible)")
    entry, nbytes = redistribute_entry(kind, n, (t, 4096))
    data = comm_inputs(kind, n, t, seed=5)
    hal = _hal(n, nbytes)
    ora = lowering.DmaEngine(NumpyBackend(NumpyBackendConfig(n, 4 * nbytes)))
    _load(kind, hal, entry, n, t, data)
    _load(kind, ora.hal, entry, n, t, data)
    got = getattr(cc, kind)(entry, cc.CudaDmaEngine(hal))
    ref = getattr(lowering, kind)(entry, ora)
    assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))
    for d in range(n):
        if entry.writeback_segments:
            size = sum(s.nbytes for s in entry.writeback_segments if s.dst_dpu == d) // 2
            a = hal.read_local(d, nbytes, (size,), entry.dtype)
            b = ora.hal.read_local(d, nbytes, (size,), entry.dtype)
            assert np.array_equal(a.view(np.uint16), b.view(np.uint16))


def test_scatter_and_broadcast_deliver_host_slices():
    from backend import cuda_collectives as cc

    entry, nbytes = redistribute_entry("scatter", 4, (8, 64), dtype="float32")
    hal = _hal(4, nbytes)
    g = np.arange(8 * 64, dtype=np.float32).reshape(8, 64)
    cc.scatter(entry, cc.CudaDmaEngine(hal), g)
    for d in range(4):
        assert np.array_equal(hal.read_local(d, nbytes, (2, 64), np.float32), g[2 * d:2 * d + 2])


def test_primitive_rejects_mismatched_entry_type():
    from backend import cuda_collectives as cc

    entry, nbytes = redistribute_entry("all_gather", 2, (4, 8), dtype="float32")
    with pytest.raises(ValueError, match="all_reduce received"):
        cc.all_reduce(entry, cc.CudaDmaEngine(_hal(2, nbytes)))


def test_plans_built_and_dropped_in_turn_each_match_the_reference():
    """The redistribute microbench's loop on one B200 HAL: each case a new single-edge plan,
    the previous one dropped (half of them released, half only unreferenced).  Lowered
    commands are keyed by id(cmd); the HAL holds every registered plan, so a new plan never
    runs a dropped plan's lowering."""
    import gc

    from runtime.exec_plan_gen import redistribute_edge, redistribute_plan
    from runtime.executor import execute_plan

    cases = [c for c in COMM["cases"] if c["n"] == 2] * 2
    nbytes = max(c["tokens"] for c in cases) * 4096 * 2
    hal = _hal(2, nbytes)
    for i, case in enumerate(cases):
        t, kind = case["tokens"], case["type"]
        edge, entry = redistribute_edge(kind, 2, (t, 4096))
        plan = redistribute_plan(edge, entry)
        hal.register_plan(plan)
        _load(kind, hal, entry, 2, t, comm_inputs(kind, 2, t))
        execute_plan(plan, hal)
        size = t * 4096 // (2 if kind == "all_to_all" else 1)
        for d in range(2):
            got = sha(hal.read_local(d, t * 4096 * 2, (size,), entry.dtype))
            assert got == (case["dst_local_sha"][d] if kind == "all_to_all" else case["out_sha"]), (i, kind, t, d)
        if i % 2:
            hal.release_plan(plan)
        del plan
        gc.collect()
    hal.close()
