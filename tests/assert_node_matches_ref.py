"""Node-by-node comparator (the reference leaves tests/assert_node_matches_ref.py empty).

Follows docs/spec.md:1649-1656: a tensor spread over ranks is reassembled by
its placement -- Shard(d) -> concatenation along d in shard order, Partial ->
sum, Replicate -> one copy (all copies must agree) -- and compared elementwise
with the reference environment.  Any HAL with ``read_local`` works (the oracle
NumPy HAL, the B200 HAL); compile the program with ``reuse=False`` so every
node's bytes survive the run.
"""

from __future__ import annotations

import numpy as np

from graph.llama import SPEC_META_KEY, OpGraph


def _np(dtype: str):
    from comm.plan import np_dtype

    return np_dtype(dtype)


class NodeEnv:
    """Resolves node names to full tensors on one HAL after a plan ran."""

    def __init__(self, hal, graph: OpGraph) -> None:
        self.hal, self.graph = hal, graph

    def __getitem__(self, name: str) -> np.ndarray:
        return gather_by_placement(self.hal, self.graph, name)


def gather_by_placement(hal, graph: OpGraph, name: str) -> np.ndarray:
    node = graph.node(name)
    spec = node.meta[SPEC_META_KEY]
    if spec.device != "dpu":
        raise ValueError(f"{name} is a host tensor")
    dt = _np(node.dtype)
    parts = sorted(((det.start_idx, hal.read_local(r, det.mram_offset, tuple(det.local_shape), dt))
                    for r, det in spec.shard_map.items()), key=lambda x: x[0])
    arrays = [p for _, p in parts]
    kind = spec.placement.kind
    if kind == "Shard":
        return np.concatenate(arrays, axis=spec.placement.dim)
    if kind == "Partial":
        return np.sum([a.astype(np.float32) for a in arrays], axis=0)
    first = arrays[0]
    for other in arrays[1:]:
        assert np.array_equal(first.view(np.uint8), other.view(np.uint8)), f"{name}: Replicate copies differ"
    return first


def assert_node_matches_ref(node: str, env, ref_env, *, rtol: float, atol: float) -> None:
    got = np.asarray(env[node], dtype=np.float32)
    ref = np.asarray(ref_env[node], dtype=np.float32)
    assert got.shape == ref.shape, f"{node}: shape {got.shape} != {ref.shape}"
    scale = max(float(np.abs(ref).max()), 1e-30)
    err = float(np.abs(got - ref).max())
    assert err <= atol * scale + rtol * scale, f"{node}: max |diff| {err:.3e} > tolerance (max |ref| {scale:.3e})"


def compare_all_nodes(graph: OpGraph, env, ref_env, *, rtol: float, atol: float) -> list[str]:
    """Compare every device node in graph order; returns the names compared."""
    names = [n.name for n in graph.nodes
             if n.meta.get(SPEC_META_KEY) is not None and n.meta[SPEC_META_KEY].device == "dpu"
             and n.op not in ("weight",)]
    for name in names:
        assert_node_matches_ref(name, env, ref_env, rtol=rtol, atol=atol)
    return names


def _read_access(hal, plan, acc) -> np.ndarray:
    if acc.loc[0] == "dpu":
        return hal.copy_from_dpu(int(acc.loc[1]), acc.offset, (acc.length,), np.uint8)
    return hal.read_host(plan, acc.offset, (acc.length,), np.uint8)


def _write_access(hal, plan, acc, data: np.ndarray) -> None:
    if acc.loc[0] == "dpu":
        hal.copy_to_dpu(int(acc.loc[1]), acc.offset, data)
    else:
        hal.write_host(plan, acc.offset, data)


def lockstep_compare(plan, hal, ref_hal, *, tokens=None, pos=None, timeout: float = 900.0,
                     ref_plan=None) -> list[tuple]:
    """Node-by-node comparison on identical inputs, command by command (docs/spec.md:1649-1656).

    Both HALs hold the same arena bytes when called.  Every command of ``plan`` runs on
    ``hal`` and then on ``ref_hal``; each interval the command leaves final is read back
    from both and compared, then ``hal``'s bytes are copied into ``ref_hal``, so every later
    command reads exactly the inputs ``hal`` produced.  Errors therefore do not accumulate
    along the plan: each entry measures one command alone.

    Which intervals are final: everything a launch or a host op writes; for a redistribute
    edge, the destinations its writebacks fill (compared at each writeback, the point where
    both HALs have them whichever command moved the bytes) and a host destination its
    combine fills.  Virtual host staging (offsets from VIRTUAL_HOST_BASE) exists only on
    HALs that move bytes through the host and is never compared.

    Returns ``(node, kind, value)`` per compared interval: ``"rel"`` with the largest
    ``|got - ref|`` over the largest ``|ref|`` for floating-point data, ``"mismatches"``
    with the count of differing elements for integer data (token ids, positions).

    ``ref_plan``: the same plan compiled a second time, for ``ref_hal`` (two oracle HALs
    cannot share one plan object: the oracle attaches its host callables to the plan's
    commands).  By default both HALs run ``plan``.
    """
    from runtime.exec_plan_gen import VIRTUAL_HOST_BASE
    from runtime.executor import PlanRun, bind_inputs

    ref_plan = plan if ref_plan is None else ref_plan
    assert len(ref_plan.commands) == len(plan.commands)
    runs = {}
    for h, pl in ((hal, plan), (ref_hal, ref_plan)):
        h.begin_run(pl)
        runs[id(h)] = PlanRun(pl, h)
        pl.meta["run"] = runs[id(h)]
        bind_inputs(pl, h, tokens, pos)
    out = []
    for cmd, ref_cmd in zip(plan.commands, ref_plan.commands):
        for h, pl, c in ((hal, plan, cmd), (ref_hal, ref_plan, ref_cmd)):
            pl.meta["run"] = runs[id(h)]  # the oracle's host combine reads its own collects
            ev = h.submit(c)
            runs[id(h)].events[c.id] = ev
            h.wait(ev, timeout=timeout)
        p = cmd.payload
        role = p.get("role")
        if cmd.op == "dma_out" or role == "collect":
            continue
        if role == "combine":
            accs = [a for a in cmd.writes if a.loc[0] == "host" and a.offset < VIRTUAL_HOST_BASE]
            dt = np.dtype(p["entry"].dtype)
        elif role == "writeback":
            accs = list(cmd.writes)
            dt = _np(str(p["dtype"])) if not isinstance(p["dtype"], np.dtype) else p["dtype"]
        else:
            accs = [a for a in cmd.writes if not (a.loc[0] == "host" and a.offset >= VIRTUAL_HOST_BASE)]
            o = p.get("output")
            dt = _np(o[2]) if isinstance(o, (tuple, list)) and len(o) == 3 else np.dtype(np.uint8)
        node = p.get("node", p.get("kernel", f"{cmd.op}#{cmd.id}"))
        for acc in accs:
            got, ref = _read_access(hal, plan, acc), _read_access(ref_hal, ref_plan, acc)
            if dt.kind == "f" or dt.name == "bfloat16":
                g = got.view(dt).astype(np.float32)
                r = ref.view(dt).astype(np.float32)
                err = float(np.abs(g - r).max() / max(float(np.abs(r).max()), 1e-30)) if r.size else 0.0
                out.append((node, "rel", err))
            else:
                item = dt.itemsize if dt.itemsize in (1, 2, 4, 8) and got.size % dt.itemsize == 0 else 1
                out.append((node, "mismatches", int(np.count_nonzero(got.view(f"u{item}") != ref.view(f"u{item}")))))
            _write_access(ref_hal, ref_plan, acc, got)
    return out


def argmax_within_tolerance(got_logits, ref_logits, tol: float) -> tuple[list[int], list[int], list[int]]:
    """Greedy ids of two logit sets ``[..., vocab]`` row by row: (got ids, ref ids, tied rows).

    A row counts as tied when the ids differ but the reference logit at ``got``'s id is
    within ``tol`` x max |ref| of the reference maximum, i.e. the two candidates are equal
    at the comparison's tolerance; any other difference is a mismatch the caller rejects.
    """
    g = np.asarray(got_logits, np.float32).reshape(-1, np.shape(got_logits)[-1])
    r = np.asarray(ref_logits, np.float32).reshape(-1, np.shape(ref_logits)[-1])
    gi, ri = g.argmax(-1), r.argmax(-1)
    scale = np.abs(r).max(-1)
    tied = [i for i in range(len(gi)) if gi[i] != ri[i] and r[i, gi[i]] >= r[i, ri[i]] - tol * scale[i]]
    return gi.tolist(), ri.tolist(), tied
