"""One redistribute edge as its own ExecutionPlan (the redistribute microbench's plan), on the oracle (CPU).

``redistribute_plan`` emits the fixed template of the edge type (collect transfers ->
one combine -> writeback transfers, scatter: host slice -> writebacks); run on the
oracle HAL it must leave every rank's destination bit-identical to the reference's
outputs (golden hashes) at the golden sizes, and the scatter must land each rank's
rows of the host tensor.
"""

from __future__ import annotations

import json
from math import prod

import numpy as np
import pytest

from helpers import GOLDEN, comm_inputs, sha

COMM = json.loads((GOLDEN / "comm_golden.json").read_text())


def _oracle(n, nbytes, plan):
    from oracle.hal_numpy import NumpyBackend, NumpyBackendConfig

    hal = NumpyBackend(NumpyBackendConfig(n, 4 * nbytes))
    hal.register_plan(plan)
    return hal


@pytest.mark.parametrize("case", COMM["cases"], ids=[c["key"] for c in COMM["cases"]])
def test_single_edge_plan_reproduces_the_reference(case):
    from runtime.exec_plan_gen import redistribute_edge, redistribute_plan
    from runtime.executor import execute_plan
    from runtime.validate import plan_hazards

    n, t, kind = case["n"], case["tokens"], case["type"]
    edge, entry = redistribute_edge(kind, n, (t, 4096))
    plan = redistribute_plan(edge, entry)
    assert plan_hazards(plan) == []
    roles = [c.payload.get("role") for c in plan.commands]
    assert roles.count("combine") == 1
    assert roles.count("collect") == len(entry.collect_segments)
    assert roles.count("writeback") == len(entry.writeback_segments)
    nbytes = prod((t, 4096)) * 2
    hal = _oracle(n, nbytes, plan)
    data = comm_inputs(kind, n, t)
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
    execute_plan(plan, hal)
    for d in range(n):
        if kind == "all_to_all":
            got = hal.read_local(d, nbytes, (t * 4096 // n,), entry.dtype)
            assert sha(got) == case["dst_local_sha"][d]
        else:
            assert sha(hal.read_local(d, nbytes, (t * 4096,), entry.dtype)) == case["out_sha"]
    hal.close()


@pytest.mark.parametrize("n", [2, 4])
def test_single_edge_scatter_plan_lands_each_ranks_rows(n):
    from runtime.exec_plan_gen import redistribute_edge, redistribute_plan
    from runtime.executor import execute_plan

    t = 16
    edge, entry = redistribute_edge("scatter", n, (t, 4096))
    plan = redistribute_plan(edge, entry)
    src = next(c for c in plan.commands if c.payload.get("role") == "combine").payload["src_host"]
    nbytes = t * 4096 * 2
    hal = _oracle(n, nbytes, plan)
    data = comm_inputs("all_gather", n, t, seed=3)
    hal.write_host(plan, src, data.reshape(-1))
    execute_plan(plan, hal)
    r = t // n
    for d in range(n):
        got = hal.read_local(d, nbytes, (r * 4096,), entry.dtype)
        assert np.array_equal(got.view(np.uint16), data[d * r:(d + 1) * r].reshape(-1).view(np.uint16))
    hal.close()


def test_unknown_kind_is_refused():
    from runtime.exec_plan_gen import redistribute_edge

    with pytest.raises(ValueError):
        redistribute_edge("reduce_scatter", 2, (16, 4096))


def test_registered_plan_stays_alive_until_released():
    """The HALs key per-plan state by id(plan) and id(cmd): a registered plan is held until
    ``release_plan``, so a plan built later can never reuse those ids (a reused id once made
    one rank of the redistribute microbench replay the previous case's lowering)."""
    import gc
    import weakref

    from runtime.exec_plan_gen import redistribute_edge, redistribute_plan

    edge, entry = redistribute_edge("all_gather", 2, (16, 4096))
    plan = redistribute_plan(edge, entry)
    hal = _oracle(2, 16 * 4096 * 2, plan)
    ref = weakref.ref(plan)
    del plan
    gc.collect()
    assert ref() is not None  # still registered
    hal.release_plan(ref())
    gc.collect()
    assert ref() is None
    hal.close()


def test_plans_built_and_dropped_in_turn_each_reproduce_the_reference():
    """The microbench's loop on one HAL: every case a new plan, the previous one dropped."""
    import gc

    from runtime.exec_plan_gen import redistribute_edge, redistribute_plan
    from runtime.executor import execute_plan

    from oracle.hal_numpy import NumpyBackend, NumpyBackendConfig

    cases = [c for c in COMM["cases"] if c["n"] == 2]
    nbytes = max(c["tokens"] for c in cases) * 4096 * 2
    hal = NumpyBackend(NumpyBackendConfig(2, 4 * nbytes))
    for case in cases:
        t, kind = case["tokens"], case["type"]
        edge, entry = redistribute_edge(kind, 2, (t, 4096))
        plan = redistribute_plan(edge, entry)
        hal.register_plan(plan)
        data = comm_inputs(kind, 2, t)
        if kind == "all_reduce":
            for d, p in enumerate(data):
                hal.copy_to_dpu(d, 0, p.reshape(-1))
        elif kind == "all_gather":
            for d in range(2):
                hal.copy_to_dpu(d, 0, np.ascontiguousarray(data[:, d * 2048:(d + 1) * 2048]).reshape(-1))
        else:
            for d in range(2):
                hal.copy_to_dpu(d, 0, np.ascontiguousarray(data[d * t // 2:(d + 1) * t // 2, :]).reshape(-1))
        execute_plan(plan, hal)
        size = t * 4096 // (2 if kind == "all_to_all" else 1)
        for d in range(2):
            got = sha(hal.read_local(d, t * 4096 * 2, (size,), entry.dtype))
            assert got == (case["dst_local_sha"][d] if kind == "all_to_all" else case["out_sha"]), (kind, t, d)
        hal.release_plan(plan)
        del plan
        gc.collect()
    hal.close()
