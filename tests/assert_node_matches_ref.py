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
