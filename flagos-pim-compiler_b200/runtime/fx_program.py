"""Programs compiled from graphs annotated by the reference's own passes.

``compile_fx`` takes an ``OpGraph`` from ``graph.fx_import.decode_graph`` -- placements
and redistribute edges exactly as the reference's ``propagate_specs`` left them -- and
runs this runtime's half of the chain the reference specifies: the three-zone memory
plan per rank (``plan_dpu``, docs/spec.md:2033-2069; no KV zone, the exported forward
has no cache), the comm plan of every edge (``build_comm_plan``, comm/plan.py:294-301)
and one ExecutionPlan (``build_execution_plan``, docs/spec.md:1435-1529).  The plan runs
unchanged on the oracle HAL and on the B200 HAL (``execute_plan``).

Weights: ``load_fx_weights`` puts each DPU weight's shard (its ``TensorShardDetail``
slice) into every rank's arena and each host-resident weight (the embedding table, the
rotary ``inv_freq`` buffer) into the plan's host location.  Values are looked up by the
attribute path the graph read them from (``model.model.layers.0.self_attn.q_proj.weight``).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from comm.plan import CommPlanEntry, build_comm_plan, np_dtype
from contracts.exec_plan import ExecutionPlan
from graph.fx_import import graph_edges
from graph.llama import SPEC_META_KEY, OpGraph
from memory.mem_planner import DPUPlan, HardwareSpec, backfill_offsets, plan_dpu
from runtime.exec_plan_gen import HostLayout, build_execution_plan


@dataclass
class FxProgram:
    graph: OpGraph
    tp: int
    dpu_plans: dict[int, DPUPlan]
    entries: list[CommPlanEntry]
    plan: ExecutionPlan

    @property
    def arena_bytes(self) -> int:
        return max(max(p.total for p in self.dpu_plans.values()), 256)


def compile_fx(g: OpGraph, *, align: int = 256, reuse: bool = True, mram_budget: int = 1 << 62) -> FxProgram:
    ranks = sorted({r for n in g.nodes for r in (n.meta.get(SPEC_META_KEY).shard_map
                                                 if n.meta.get(SPEC_META_KEY) is not None else {})})
    if not ranks:
        raise ValueError("the graph places nothing on a DPU")
    hw = HardwareSpec(mram_budget=mram_budget, align=align)
    plans = {r: plan_dpu([g], r, None, hw, reuse) for r in ranks}
    backfill_offsets([g], plans)
    entries = build_comm_plan(graph_edges(g))
    plan = build_execution_plan(g, entries, plans, {}, HostLayout())
    plan.meta["program"] = "fx"
    return FxProgram(g, len(ranks), plans, entries, plan)


def _shard(value: np.ndarray, det) -> np.ndarray:
    if det.shard_dim < 0:
        return value
    idx = [slice(None)] * value.ndim
    idx[det.shard_dim] = slice(det.start_idx, det.end_idx)
    return value[tuple(idx)]


def load_fx_weights(prog: FxProgram, hal, values: dict[str, np.ndarray]) -> None:
    """Every weight of the graph from ``values`` (keyed by attribute path, or by node name)."""
    plan = prog.plan
    for n in prog.graph.nodes:
        if n.op != "weight":
            continue
        key = n.attrs.get("target") or n.name
        v = values.get(key, values.get(n.name))
        if v is None:
            raise KeyError(f"no value for weight {key}")
        v = np.ascontiguousarray(np.asarray(v).astype(np_dtype(n.dtype), copy=False))
        if tuple(v.shape) != tuple(n.shape):
            raise ValueError(f"{key}: shape {v.shape} != {n.shape}")
        spec = n.meta[SPEC_META_KEY]
        if spec.device == "host":
            hal.write_host(plan, plan.meta["host_weights"][n.name].offset, v)
            continue
        for r, det in spec.shard_map.items():
            hal.copy_to_dpu(r, det.mram_offset, np.ascontiguousarray(_shard(v, det)))


def bind_fx_inputs(prog: FxProgram, hal, inputs: dict[str, np.ndarray]) -> None:
    plan = prog.plan
    for name, ref in plan.meta["inputs"].items():
        if name not in inputs:
            raise KeyError(f"input {name!r} not given")
        v = np.ascontiguousarray(np.asarray(inputs[name]).astype(np_dtype(ref.dtype), copy=False))
        if tuple(v.shape) != tuple(ref.shape):
            raise ValueError(f"input {name}: shape {v.shape} != {ref.shape}")
        hal.write_host(plan, ref.offset, v)


def read_fx_outputs(prog: FxProgram, hal) -> dict[str, np.ndarray]:
    plan = prog.plan
    return {name: hal.read_host(plan, ref.offset, tuple(ref.shape), np_dtype(ref.dtype))
            for name, ref in plan.meta["outputs"].items()}


def run_fx(prog: FxProgram, hal, inputs: dict[str, np.ndarray], timeout: float | None = 300.0) -> dict:
    """One execution of the program's plan: bind ``inputs``, run, return the outputs."""
    from runtime.executor import execute_plan

    bind_fx_inputs(prog, hal, inputs)
    execute_plan(prog.plan, hal, timeout=timeout)
    return read_fx_outputs(prog, hal)
