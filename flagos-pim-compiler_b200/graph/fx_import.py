"""Graphs annotated by the reference's own compile passes, as plans for this runtime.

The reference compiles a model by ``torch.export`` (strict), ``partition_graph``
(graph/partition.py:36-81: ``aten.linear / addmm / add / mul / tanh`` on the DPUs,
everything else on the host) and ``propagate_specs`` (graph/spec_prop.py:411-451:
a ``PIMTensorSpec`` on every tensor node and ``RedistributeEdge`` lists on the
consumers, under the ``"device"``, ``"spec"`` and ``"redistribute"`` meta keys of
contracts/graph_meta.py).  This module takes such a graph unchanged and turns it
into this runtime's ``OpGraph`` at aten granularity, so the memory planner, the comm
plan and the ExecutionPlan generator run on exactly the placements the reference
chose:

* ``encode_fx(gm)`` reads an annotated ``GraphModule`` into a plain, JSON-serialisable
  dict (node names, aten targets, operands with node references, shapes, dtypes,
  specs and edges).  Higher-order host wrappers (``wrap_with_set_grad_enabled``, the
  rotary-embedding subgraph of HF LLaMA) are inlined: their inner nodes become host
  nodes named ``<wrapper>.<inner>`` and each ``getitem`` of the wrapper an alias of the
  inner output.  ``_assert_tensor_metadata`` checks and export guards carry no data and
  are dropped.
* ``decode_graph(d)`` builds the ``OpGraph`` from that dict with this runtime's contract
  records (same fields as the reference's, contracts/pim_tensor_spec.py:5-96).

Every node keeps its full operand list in ``attrs["args"]`` / ``attrs["kwargs"]``
(tensor operands as ``{"node": name}``), which is what the aten kernels of both HALs
read; ``OpNode.args`` lists the tensor operands for liveness and dependencies.
"""

from __future__ import annotations

from math import prod

from contracts.pim_tensor_spec import Placement, PIMTensorSpec, RedistributeEdge, TensorShardDetail
from graph.llama import DEVICE_META_KEY, REDISTRIBUTE_META_KEY, SPEC_META_KEY, OpGraph, OpNode

FORMAT = "pim-fx-graph/1"
_DROPPED = ("aten._assert_tensor_metadata.default", "aten._assert_scalar.default")
_WRAPPERS = ("wrap_with_set_grad_enabled", "wrap_with_autocast")


# ---------------------------------------------------------------------------
# encoding (needs torch; reads the reference passes' annotations)
# ---------------------------------------------------------------------------


def _dtype_name(dt) -> str:
    return str(dt).replace("torch.", "")


def _enc_value(v, rename):
    import torch
    from torch.fx import Node

    if isinstance(v, Node):
        return {"node": rename(v)}
    if isinstance(v, (list, tuple)):
        return [_enc_value(x, rename) for x in v]
    if isinstance(v, dict):
        return {"dict": {str(k): _enc_value(x, rename) for k, x in v.items()}}
    if isinstance(v, torch.dtype):
        return {"dtype": _dtype_name(v)}
    if isinstance(v, torch.device):
        return {"device": str(v)}
    if isinstance(v, torch.memory_format):
        return {"memory_format": str(v)}
    if isinstance(v, torch.layout):
        return {"layout": str(v)}
    if v is None or isinstance(v, (bool, int, float, str)):
        return v
    raise TypeError(f"cannot encode operand {v!r} of type {type(v).__name__}")


def _enc_spec(s) -> dict | None:
    if s is None:
        return None
    return {"device": s.device, "placement": [s.placement.kind, s.placement.dim, s.placement.reduce_type],
            "residency": s.residency, "pinned_dpu_id": s.pinned_dpu_id, "reduce_type": s.reduce_type,
            "shard_map": {str(r): [d.dpu_id, d.shard_dim, d.start_idx, d.end_idx, list(d.local_shape), d.mram_offset]
                          for r, d in s.shard_map.items()}}


def _enc_edge(e) -> dict:
    return {"edge_id": e.edge_id, "src": e.src, "dst": e.dst,
            "from_placement": [e.from_placement.kind, e.from_placement.dim, e.from_placement.reduce_type],
            "to_placement": [e.to_placement.kind, e.to_placement.dim, e.to_placement.reduce_type],
            "src_spec": _enc_spec(e.src_spec), "dst_spec": _enc_spec(e.dst_spec), "type": e.type,
            "src_loc": e.src_loc, "dst_loc": e.dst_loc, "nbytes": e.nbytes, "reduce_type": e.reduce_type,
            "shape": list(e.shape), "dtype": str(e.dtype).replace("torch.", "")}


def _val(node):
    import torch

    v = node.meta.get("val")
    if isinstance(v, torch.Tensor):
        return list(v.shape), _dtype_name(v.dtype)
    return None, None


def _host_spec_dict() -> dict:
    return {"device": "host", "placement": ["Replicate", None, None], "residency": "transient",
            "pinned_dpu_id": None, "reduce_type": None, "shard_map": {}}


def encode_fx(gm) -> dict:
    """A reference-annotated GraphModule as a JSON-serialisable dict (see the module docstring)."""
    out = []
    alias: dict[str, str] = {}  # dropped / inlined names -> the node that carries their value

    def rename(n) -> str:
        return alias.get(n.name, n.name)

    def emit(name, op, target, args, kwargs, node_for_val, device, spec, edges):
        shape, dtype = _val(node_for_val)
        out.append({"name": name, "op": op, "target": target, "args": args, "kwargs": kwargs,
                    "shape": shape, "dtype": dtype, "device": device, "spec": spec, "redistribute": edges})

    def inline(wrapper, sub_gm, operands):
        inner = {}
        placeholders = [n for n in sub_gm.graph.nodes if n.op == "placeholder"]
        for p, v in zip(placeholders, operands):
            inner[p.name] = rename(v) if hasattr(v, "name") else v
        result = []
        for n in sub_gm.graph.nodes:
            if n.op == "placeholder":
                continue
            if n.op == "output":
                result = [inner[a.name] for a in n.args[0]]
                continue
            tgt = str(n.target)
            if tgt in _DROPPED:
                continue
            name = f"{wrapper.name}.{n.name}"

            def sub_rename(x, _inner=inner):
                return _inner[x.name]

            emit(name, n.op, tgt, _enc_value(list(n.args), sub_rename), _enc_value(dict(n.kwargs), sub_rename),
                 n, "host", _host_spec_dict(), [])
            inner[n.name] = name
        return result

    wrapper_outputs: dict[str, list[str]] = {}
    for n in gm.graph.nodes:
        spec = n.meta.get(SPEC_META_KEY)
        device = n.meta.get(DEVICE_META_KEY, "host")
        edges = [_enc_edge(e) for e in n.meta.get(REDISTRIBUTE_META_KEY, [])]
        if n.op == "placeholder":
            emit(n.name, "placeholder", None, [], {}, n, "host", _enc_spec(spec), edges)
        elif n.op == "get_attr":
            shape, _ = _val(n)
            if shape is None:
                continue  # a subgraph, inlined at its wrapper
            emit(n.name, "get_attr", str(n.target), [], {}, n, spec.device if spec else device, _enc_spec(spec),
                 edges)
        elif n.op == "call_module":
            continue  # export guards
        elif n.op == "output":
            out.append({"name": "output", "op": "output", "target": None,
                        "args": _enc_value(list(n.args), rename), "kwargs": {}, "shape": None, "dtype": None,
                        "device": "host", "spec": None, "redistribute": edges})
        else:
            tgt = str(n.target)
            if tgt in _DROPPED:
                continue
            if getattr(n.target, "__name__", "") in _WRAPPERS or tgt in _WRAPPERS:
                sub = next(a for a in n.args if hasattr(a, "op") and a.op == "get_attr")
                sub_gm = getattr(gm, sub.target)
                operands = [a for a in n.args[n.args.index(sub) + 1:]]
                wrapper_outputs[n.name] = inline(n, sub_gm, operands)
                continue
            if getattr(n.target, "__name__", "") == "getitem" and n.args and hasattr(n.args[0], "name") \
                    and n.args[0].name in wrapper_outputs:
                src = wrapper_outputs[n.args[0].name][n.args[1]]
                emit(n.name, "call_function", "aten.alias.default", [{"node": src}], {}, n, "host",
                     _enc_spec(spec) or _host_spec_dict(), edges)
                continue
            emit(n.name, "call_function", tgt, _enc_value(list(n.args), rename), _enc_value(dict(n.kwargs), rename),
                 n, device, _enc_spec(spec), edges)
    return {"format": FORMAT, "nodes": out}


# ---------------------------------------------------------------------------
# decoding (no torch needed)
# ---------------------------------------------------------------------------


def _placement(p) -> Placement:
    return Placement(p[0], p[1], p[2])


def spec_from_dict(d: dict | None) -> PIMTensorSpec | None:
    if d is None:
        return None
    sm = {int(r): TensorShardDetail(v[0], v[1], v[2], v[3], tuple(v[4]), v[5]) for r, v in d["shard_map"].items()}
    return PIMTensorSpec(d["device"], _placement(d["placement"]), d["residency"], d["pinned_dpu_id"], sm,
                         d["reduce_type"])


def edge_from_dict(d: dict) -> RedistributeEdge:
    return RedistributeEdge(d["edge_id"], d["src"], d["dst"], _placement(d["from_placement"]),
                            _placement(d["to_placement"]), spec_from_dict(d["src_spec"]),
                            spec_from_dict(d["dst_spec"]), d["type"], d["src_loc"], d["dst_loc"], d["nbytes"],
                            d["reduce_type"], tuple(d["shape"]), d["dtype"])


def tensor_operands(v) -> list[str]:
    """Names of the nodes referenced in an encoded operand tree, in order (duplicates kept once)."""
    found: list[str] = []

    def walk(x):
        if isinstance(x, dict):
            if "node" in x and len(x) == 1:
                if x["node"] not in found:
                    found.append(x["node"])
            elif "dict" in x:
                for y in x["dict"].values():
                    walk(y)
        elif isinstance(x, list):
            for y in x:
                walk(y)

    walk(v)
    return found


def aten_name(target: str) -> str:
    """``aten.linear.default`` -> ``aten.linear``; ``aten.add.Tensor`` -> ``aten.add.Tensor`` is kept
    whole except for the ``.default`` overload, so overloads that differ stay apart."""
    return target[:-len(".default")] if target.endswith(".default") else target


def decode_graph(d: dict, name: str = "fx", phase: str = "prefill") -> OpGraph:
    """This runtime's OpGraph for an encoded, reference-annotated graph.

    Node ops: ``input`` (placeholders), ``weight`` (tensor attributes), the aten target
    for calls (``aten.linear``, ``aten.add.Tensor``, ...), ``output``.
    """
    if d.get("format") != FORMAT:
        raise ValueError(f"not a {FORMAT} graph")
    nodes = []
    for e in d["nodes"]:
        if e["op"] == "output":
            args = tuple(tensor_operands(e["args"]))
            n = OpNode("output", "output", args, (), "float32", "host",
                       {"args": e["args"], "kwargs": {}})
        else:
            op = {"placeholder": "input", "get_attr": "weight"}.get(e["op"]) or aten_name(e["target"])
            args = tuple(tensor_operands([e["args"], e["kwargs"]]))
            shape = tuple(e["shape"] or ())
            n = OpNode(e["name"], op, args, shape, e["dtype"] or "float32", e["device"],
                       {"args": e["args"], "kwargs": e["kwargs"], "target": e["target"]})
        spec = spec_from_dict(e["spec"])
        n.meta[SPEC_META_KEY] = spec
        n.meta[DEVICE_META_KEY] = e["device"]
        n.meta[REDISTRIBUTE_META_KEY] = [edge_from_dict(x) for x in e["redistribute"]]
        nodes.append(n)
    # An edge's source spec is its producer's spec (graph/spec_prop.py:371-409 builds the edge
    # from it): share the object, so the offsets the memory planner writes into the producer's
    # shards are the ones the comm plan collects from.
    by_name = {n.name: n for n in nodes}
    for n in nodes:
        edges = []
        for e in n.meta[REDISTRIBUTE_META_KEY]:
            src = by_name.get(e.src)
            spec = src.meta.get(SPEC_META_KEY) if src is not None else None
            if spec is not None and spec.placement == e.src_spec.placement and spec.device == e.src_spec.device:
                from dataclasses import replace

                e = replace(e, src_spec=spec)
            edges.append(e)
        n.meta[REDISTRIBUTE_META_KEY] = edges
    batch = 1
    seq = 1
    for n in nodes:
        if n.op == "input" and len(n.shape) == 2:
            batch, seq = n.shape
            break
    return OpGraph(name, phase, None, batch, seq, nodes)


def graph_edges(g: OpGraph) -> list[RedistributeEdge]:
    """Every redistribute edge of the graph, in edge-id order."""
    return sorted((e for n in g.nodes for e in n.meta.get(REDISTRIBUTE_META_KEY, [])), key=lambda e: e.edge_id)


def numel(shape) -> int:
    return prod(shape) if shape else 1
