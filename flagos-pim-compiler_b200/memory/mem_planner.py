"""Per-rank three-zone static memory plan (``DPU_k.plan``).

Implements the planner the reference specifies but leaves empty
(memory/mem_planner.py is 0 bytes; design in docs/spec.md:2033-2082):

    | weights (pinned, both graphs) | KV (kv_base, build_kv_layout) | activations |

* weights: the union of both graphs' weights on this rank, sorted by name,
  each aligned (docs/spec.md:2041-2045); ``mram_offset`` is back-filled into
  the weight's ``PIMTensorSpec.shard_map`` so the comm plan, the generator and
  the HAL share one source of addresses;
* KV: ``kv_base`` is the next aligned offset and ``kv_allocated_bytes`` from
  ``build_kv_layout`` advances the cursor (docs/spec.md:2046-2052);
* activations: prefill and decode are a mutually exclusive overlay at one
  ``act_base``; inside each graph a liveness + greedy-by-size packing lets
  tensors with disjoint lifetimes share addresses (docs/spec.md:2053-2062).
  Every transient tensor is counted: node outputs on the rank *and* the
  destination buffers that redistribute edges materialize, with the
  collect-side reads of those edges counted as reads of the source tensor
  (docs/spec.md:1984-1990).
* ``pending_readers``: for every placed tensor, the readers of every earlier
  tensor that shares its bytes; the generator turns them into WAR waits
  (docs/spec.md:2067-2069, 1977-1983).  Reader ids are node names for kernel
  reads and ``"edge<id>"`` for collect reads of a redistribute edge.

On the B200 the whole plan is one device allocation per rank (the arena);
offsets are arena-relative, aligned to 256 B so every buffer starts on a
TMA/128-bit-load boundary.
"""

from __future__ import annotations

from dataclasses import dataclass, field, replace
from math import prod

from contracts.exec_plan import Access
from graph.llama import DEVICE_META_KEY, REDISTRIBUTE_META_KEY, SPEC_META_KEY, OpGraph, dtype_bytes
from memory.kv_layout import KVRegionSpec, align_up, build_kv_layout

DEFAULT_ALIGN = 256


@dataclass
class HardwareSpec:
    mram_budget: int
    align: int = DEFAULT_ALIGN
    sys_reserve: int = 0


@dataclass
class TensorLife:
    """One transient buffer on one rank: its size, lifetime and readers."""

    key: str  # node name, or "edge<id>" for a materialized redistribute destination
    nbytes: int
    start: int
    end: int
    readers: list[str] = field(default_factory=list)
    offset: int = -1


@dataclass
class DPUPlan:
    dpu_id: int
    weight: dict[str, int] = field(default_factory=dict)
    kv_base: int = 0
    kv_spec: KVRegionSpec | None = None
    act_base: int = 0
    act: dict[str, dict[str, int]] = field(default_factory=dict)  # graph name -> key -> offset
    pending_readers: dict[str, dict[tuple, list[str]]] = field(default_factory=dict)
    lifetimes: dict[str, list[TensorLife]] = field(default_factory=dict)
    total: int = 0

    def act_offset(self, graph: str, key: str) -> int:
        return self.act[graph][key]


def weights_on(graphs: list[OpGraph], rank: int):
    seen = {}
    for g in graphs:
        for n in g.nodes:
            if n.op == "weight" and n.meta.get(DEVICE_META_KEY) == "dpu":
                spec = n.meta[SPEC_META_KEY]
                if rank in spec.shard_map:
                    seen.setdefault(n.name, n)
    return [seen[k] for k in sorted(seen)]


def local_nbytes(node, spec, rank: int) -> int:
    return prod(spec.shard_map[rank].local_shape) * dtype_bytes(node.dtype)


def transient_tensors(g: OpGraph, rank: int) -> list[TensorLife]:
    """Activation buffers of ``g`` on ``rank`` with [def, last use] on a 2i/2i+1 clock.

    Node ``i`` runs at time ``2i+1``; the redistribute edges it consumes are
    materialized at ``2i`` (after their sources, before the node).
    """
    lives: dict[str, TensorLife] = {}
    order = {n.name: i for i, n in enumerate(g.nodes)}
    for i, n in enumerate(g.nodes):
        spec = n.meta.get(SPEC_META_KEY)
        if n.op in ("weight", "input") or spec is None or spec.device != "dpu":
            continue
        if rank in spec.shard_map:
            lives[n.name] = TensorLife(n.name, local_nbytes(n, spec, rank), 2 * i + 1, 2 * i + 1)
    for i, n in enumerate(g.nodes):
        redirected = {}
        for e in n.meta.get(REDISTRIBUTE_META_KEY, []):
            src = lives.get(e.src)
            if src is not None and e.src_spec.device == "dpu" and rank in e.src_spec.shard_map:
                src.end = max(src.end, 2 * i)
                src.readers.append(f"edge{e.edge_id}")
            if e.dst_spec.device == "dpu" and rank in e.dst_spec.shard_map and e.type != "local_slice":
                key = f"edge{e.edge_id}"
                nb = prod(e.dst_spec.shard_map[rank].local_shape) * dtype_bytes(e.dtype)
                lives[key] = TensorLife(key, nb, 2 * i, 2 * i + 1, [n.name])
                redirected[e.src] = key
        for a in n.args:
            if a in redirected:
                continue
            life = lives.get(a)
            if life is not None:
                life.end = max(life.end, 2 * i + 1)
                life.readers.append(n.name)
    del order
    return list(lives.values())


def greedy_reuse(tensors: list[TensorLife], base: int, align: int, reuse: bool = True) -> tuple[dict[str, int], int]:
    """Largest-first placement at the lowest offset free over the tensor's lifetime.

    ``reuse=False`` gives every tensor its own bytes (a debug layout in which
    every node's value survives the whole run, for node-by-node comparison).
    """
    placed: list[TensorLife] = []
    end = base
    for t in sorted(tensors, key=lambda t: (-t.nbytes, t.start, t.key)):
        if not reuse:
            t.offset = end
            placed.append(t)
            end += align_up(max(t.nbytes, 1), align)
            continue
        size = align_up(max(t.nbytes, 1), align)
        busy = sorted((p.offset, p.offset + align_up(max(p.nbytes, 1), align)) for p in placed
                      if not (p.end < t.start or t.end < p.start))
        cur = base
        for lo, hi in busy:
            if cur + size <= lo:
                break
            cur = max(cur, hi)
        t.offset = cur
        placed.append(t)
        end = max(end, cur + size)
    return {t.key: t.offset for t in tensors}, end


def pending_readers_of_reused(tensors: list[TensorLife], rank: int, align: int) -> dict[tuple, list[str]]:
    """``{(("dpu", rank), offset): [reader ids]}`` for every tensor that reuses bytes."""
    out: dict[tuple, list[str]] = {}
    for t in tensors:
        a = Access(("dpu", rank), t.offset, align_up(max(t.nbytes, 1), align))
        readers: list[str] = []
        for p in tensors:
            if p is t or p.end >= t.start:
                continue
            b = Access(("dpu", rank), p.offset, align_up(max(p.nbytes, 1), align))
            if a.overlaps(b):
                readers += [r for r in p.readers if r not in readers]
        if readers:
            out[(("dpu", rank), t.offset)] = readers
    return out


def plan_dpu(graphs: list[OpGraph], rank: int, kv_spec: KVRegionSpec | None, hw: HardwareSpec,
             reuse: bool = True) -> DPUPlan:
    """Plan one rank for all ``graphs`` (prefill and decode share weights and KV)."""
    plan = DPUPlan(rank)
    off = 0
    for w in weights_on(graphs, rank):
        spec = w.meta[SPEC_META_KEY]
        plan.weight[w.name] = off
        off += align_up(local_nbytes(w, spec, rank), hw.align)
    off = align_up(off, hw.align)
    plan.kv_base = off
    if kv_spec is not None:
        kv_spec.kv_base = off
        build_kv_layout(kv_spec, hw.align)
        plan.kv_spec = kv_spec
        off += kv_spec.kv_allocated_bytes
    off = align_up(off, hw.align)
    plan.act_base = off
    total = off
    for g in graphs:
        lives = transient_tensors(g, rank)
        table, end = greedy_reuse(lives, off, hw.align, reuse)
        plan.act[g.name] = table
        plan.lifetimes[g.name] = lives
        plan.pending_readers[g.name] = pending_readers_of_reused(lives, rank, hw.align)
        total = max(total, end)
    plan.total = total
    if plan.total > hw.mram_budget - hw.sys_reserve:
        raise ValueError(f"dpu{rank}: plan needs {plan.total} bytes > budget {hw.mram_budget - hw.sys_reserve}")
    return plan


def backfill_offsets(graphs: list[OpGraph], plans: dict[int, DPUPlan]) -> None:
    """Write each rank's offsets into the specs (weights, node outputs, edge destinations)."""
    for g in graphs:
        for n in g.nodes:
            spec = n.meta.get(SPEC_META_KEY)
            if spec is None or spec.device != "dpu":
                continue
            for rank in list(spec.shard_map):
                p = plans[rank]
                if n.op == "weight":
                    off = p.weight[n.name]
                else:
                    off = p.act[g.name].get(n.name)
                    if off is None:
                        continue
                spec.shard_map[rank] = replace(spec.shard_map[rank], mram_offset=off)
            for e in n.meta.get(REDISTRIBUTE_META_KEY, []):
                if e.dst_spec.device == "dpu":
                    for rank in list(e.dst_spec.shard_map):
                        off = plans[rank].act[g.name].get(f"edge{e.edge_id}")
                        if off is not None:
                            e.dst_spec.shard_map[rank] = replace(e.dst_spec.shard_map[rank], mram_offset=off)
