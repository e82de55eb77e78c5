"""Comm plan: expand each RedistributeEdge into flat-coordinate segments.

Restates the reference's compile-time comm plan (comm/plan.py:33-347) so the
GPU runtime can build it without the reference checkout.  The segment algebra
has to be identical -- segment tables are the contract between the plan
compiler and every redistribute executor -- so the rules are kept, in this
module's own code:

* every coordinate is an element index into the row-major flattened global
  tensor; a Shard(d) slice is ``prod(shape[:d])`` contiguous runs
  (comm/plan.py:90-108);
* Replicate / Partial sources contribute one full-range run; a Replicate
  source is collected from one rank only (comm/plan.py:187-188);
* writeback segments exist only when the destination is a dpu set
  (comm/plan.py:198-199);
* all_to_all rows are the pairwise intersections of source and destination
  runs (comm/plan.py:216-237);
* a coverage check rejects gaps/overlaps (comm/plan.py:240-254);
* ``dma_sequence`` batches same-address transfers into push/broadcast ops
  (comm/plan.py:330-347).

``src_addr``/``dst_addr`` are absolute arena byte addresses
(``mram_offset + local element offset * itemsize``).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from math import prod
from typing import Iterator, Literal

import numpy as np

from contracts.pim_tensor_spec import PIMTensorSpec, RedistributeEdge, TensorShardDetail

CommType = Literal["all_reduce", "all_gather", "all_to_all", "scatter", "local_slice"]


def np_dtype(name) -> np.dtype:
    """numpy dtype for a torch dtype name; bfloat16 comes from ml_dtypes."""
    if isinstance(name, np.dtype):
        return name
    if str(name) == "bfloat16":
        import ml_dtypes

        return np.dtype(ml_dtypes.bfloat16)
    return np.dtype(str(name))


@dataclass(frozen=True)
class CommSegment:
    edge_id: int
    type: CommType
    src_dpu: int | None
    src_local_range: tuple[int, int]
    global_range: tuple[int, int]
    dst_dpu: int | None
    dst_local_offset: int
    nbytes: int
    reduce: str | None = None
    src_addr: int = 0
    dst_addr: int = 0
    dst_ready_after: tuple = ()


@dataclass
class CommPlanEntry:
    edge_id: int
    type: CommType
    reduce: str | None
    shape: tuple[int, ...]
    dtype: np.dtype
    dst_loc: dict
    wait_for: tuple[int, ...]
    segments: list[CommSegment] = field(default_factory=list)

    @property
    def numel(self) -> int:
        return prod(self.shape)

    @property
    def collect_segments(self) -> list[CommSegment]:
        return [s for s in self.segments if s.src_dpu is not None]

    @property
    def writeback_segments(self) -> list[CommSegment]:
        return [s for s in self.segments if s.dst_dpu is not None]


# ---------------------------------------------------------------------------
# shard -> runs in flat coordinates
# ---------------------------------------------------------------------------


def shard_runs(
    shape: tuple[int, ...], kind: str, dim: int, detail: TensorShardDetail
) -> list[tuple[int, int, int]]:
    """``[(global_start, local_start, length)]`` for one rank's slice."""
    if kind != "Shard":
        return [(0, 0, prod(shape))]
    inner = prod(shape[dim + 1:])
    span = shape[dim] * inner
    width = (detail.end_idx - detail.start_idx) * inner
    first = detail.start_idx * inner
    return [(row * span + first, row * width, width) for row in range(prod(shape[:dim]))]


def global_shape_of(spec: PIMTensorSpec) -> tuple[int, ...]:
    details = list(spec.shard_map.values())
    local = details[0].local_shape
    if spec.placement.kind != "Shard":
        return tuple(local)
    d = spec.placement.dim
    total = sum(x.end_idx - x.start_idx for x in details)
    return tuple(local[:d]) + (total,) + tuple(local[d + 1:])


def spec_runs(spec: PIMTensorSpec) -> Iterator[tuple[int, TensorShardDetail, int, int, int]]:
    if not spec.shard_map:
        return
    shape = global_shape_of(spec)
    kind, dim = spec.placement.kind, spec.placement.dim or 0
    for rank, detail in spec.shard_map.items():
        for g, loc, n in shard_runs(shape, kind, dim, detail):
            yield rank, detail, g, loc, n


# ---------------------------------------------------------------------------
# edge -> entry
# ---------------------------------------------------------------------------


def _seg(edge, itemsize, src_dpu, src_lo, src_base, g_lo, n, dst_dpu, dst_lo, dst_base) -> CommSegment:
    return CommSegment(
        edge_id=edge.edge_id,
        type=edge.type,
        src_dpu=src_dpu,
        src_local_range=(src_lo, src_lo + n),
        global_range=(g_lo, g_lo + n),
        dst_dpu=dst_dpu,
        dst_local_offset=dst_lo,
        nbytes=n * itemsize,
        reduce=edge.reduce_type if edge.type == "all_reduce" else None,
        src_addr=src_base + src_lo * itemsize,
        dst_addr=dst_base + dst_lo * itemsize,
    )


def _collect(edge: RedistributeEdge, itemsize: int) -> list[CommSegment]:
    out = []
    for rank, detail, g, loc, n in spec_runs(edge.src_spec):
        out.append(_seg(edge, itemsize, rank, loc, detail.mram_offset, g, n, None, g, 0))
        if edge.src_spec.placement.kind == "Replicate":
            break
    return out


def _writeback(edge: RedistributeEdge, itemsize: int) -> list[CommSegment]:
    if edge.dst_loc["device"] == "host":
        return []
    return [
        _seg(edge, itemsize, None, g, 0, g, n, rank, loc, detail.mram_offset)
        for rank, detail, g, loc, n in spec_runs(edge.dst_spec)
    ]


def _exchange(edge: RedistributeEdge, itemsize: int) -> list[CommSegment]:
    out = []
    dst_runs = list(spec_runs(edge.dst_spec))
    for s_rank, s_det, s_g, s_loc, s_n in spec_runs(edge.src_spec):
        for d_rank, d_det, d_g, d_loc, d_n in dst_runs:
            lo, hi = max(s_g, d_g), min(s_g + s_n, d_g + d_n)
            if lo < hi:
                out.append(_seg(edge, itemsize, s_rank, s_loc + lo - s_g, s_det.mram_offset, lo, hi - lo,
                                d_rank, d_loc + lo - d_g, d_det.mram_offset))
    return out


def _check_coverage(segs: list[CommSegment], full: bool, numel: int, label: str) -> None:
    if full:
        for s in segs:
            if s.global_range != (0, numel):
                raise ValueError(f"{label}: segment {s.global_range} is not the full range [0, {numel})")
        return
    cursor = 0
    for lo, hi in sorted(s.global_range for s in segs):
        if lo != cursor:
            raise ValueError(f"{label}: global ranges break or overlap at [{cursor}, {lo})")
        cursor = hi
    if cursor != numel:
        raise ValueError(f"{label}: segments cover [0, {cursor}) != [0, {numel})")


def entry_of_edge(edge: RedistributeEdge) -> CommPlanEntry:
    try:
        dtype = np_dtype(edge.dtype)
    except TypeError:
        raise ValueError(f"edge {edge.edge_id}: dtype {edge.dtype!r} has no numpy equivalent") from None
    numel = prod(edge.shape)
    if numel * dtype.itemsize != edge.nbytes:
        raise ValueError(f"edge {edge.edge_id}: shape/dtype disagree with nbytes={edge.nbytes}")
    entry = CommPlanEntry(
        edge_id=edge.edge_id,
        type=edge.type,
        reduce=edge.reduce_type if edge.type == "all_reduce" else None,
        shape=tuple(edge.shape),
        dtype=dtype,
        dst_loc=edge.dst_loc,
        wait_for=tuple(edge.src_loc["dpus"]) if edge.src_loc["device"] == "dpu" else (),
    )
    if edge.type == "local_slice":
        return entry
    if edge.type == "all_to_all":
        entry.segments = _exchange(edge, dtype.itemsize)
        _check_coverage(entry.segments, False, numel, f"edge {edge.edge_id} all_to_all")
        return entry
    collect, wb = _collect(edge, dtype.itemsize), _writeback(edge, dtype.itemsize)
    entry.segments = collect + wb
    if collect:
        _check_coverage(collect, edge.src_spec.placement.kind != "Shard", numel, f"edge {edge.edge_id} collect")
    if wb:
        _check_coverage(wb, edge.dst_spec.placement.kind != "Shard", numel, f"edge {edge.edge_id} writeback")
    return entry


def build_comm_plan(edges: list[RedistributeEdge]) -> list[CommPlanEntry]:
    """One entry per edge, in edge order; local_slice keeps an empty placeholder."""
    return [entry_of_edge(e) for e in edges]


# ---------------------------------------------------------------------------
# transfer batching (host-star SDK calls) and cost
# ---------------------------------------------------------------------------


@dataclass(frozen=True)
class DmaOp:
    kind: Literal["copy_from", "copy_to", "push_from", "push_to", "broadcast_to"]
    segments: tuple[CommSegment, ...]


def _groups(segs: list[CommSegment], key) -> list[list[CommSegment]]:
    table: dict = {}
    for s in segs:
        table.setdefault(key(s), []).append(s)
    return list(table.values())


def dma_sequence(entry: CommPlanEntry) -> list[DmaOp]:
    ops = [DmaOp("push_from" if len(g) > 1 else "copy_from", tuple(g))
           for g in _groups(entry.collect_segments, lambda s: (s.src_addr, s.nbytes))]
    wb = entry.writeback_segments
    if wb and len({(s.global_range, s.dst_addr) for s in wb}) == 1:
        ops.append(DmaOp("broadcast_to", tuple(wb)))
    else:
        ops += [DmaOp("push_to" if len(g) > 1 else "copy_to", tuple(g))
                for g in _groups(wb, lambda s: (s.dst_addr, s.nbytes))]
    return ops


@dataclass(frozen=True)
class HostStarCostModel:
    """Per-call setup + host-bandwidth model of the reference (comm/plan.py:355-365)."""

    dma_setup_s: float = 1e-5
    host_bytes_per_s: float = 25e9
    topology: str = "host_star"


@dataclass(frozen=True)
class NvlinkCostModel:
    """Measured-collective model for NVLink 5 / NVSwitch ranks.

    ``latency_s`` is a per-collective launch+sync floor and ``bus_bytes_per_s``
    the bus bandwidth; all_reduce moves 2(N-1)/N of the payload per rank,
    all_gather (N-1)/N, all_to_all (N-1)/N^2 (NCCL bus-bytes convention).
    """

    latency_s: float = 8e-6
    bus_bytes_per_s: float = 725e9
    topology: str = "nvswitch"


@dataclass(frozen=True)
class CommCost:
    transfers: int
    nbytes: int
    seconds: float


@dataclass(frozen=True)
class MeasuredCostModel:
    """Per-collective costs fitted to measured edges: ``latency + bus_bytes / bandwidth``.

    ``fit`` takes the cases of the redistribute microbench (``{"kind", "bus_bytes_per_rank",
    "us"}`` per measured edge, as ``bench.py --redistribute`` prints them) and fits one
    latency and one bus bandwidth per collective kind by least squares (latency >= 0);
    kinds without measurements use ``fallback``.  This is the measured per-edge comm cost
    the reference's plan_cost consumer expects from a real topology (comm/plan.py:355-384
    models a host star instead).
    """

    fits: tuple = ()  # ((kind, latency_s, bus_bytes_per_s), ...)
    fallback: NvlinkCostModel = NvlinkCostModel()
    topology: str = "nvswitch-measured"

    def params(self, kind: str) -> tuple[float, float]:
        for k, lat, bw in self.fits:
            if k == kind:
                return lat, bw
        return self.fallback.latency_s, self.fallback.bus_bytes_per_s

    @classmethod
    def fit(cls, cases, fallback: NvlinkCostModel | None = None) -> "MeasuredCostModel":
        fallback = fallback or NvlinkCostModel()
        by_kind: dict[str, list[tuple[float, float]]] = {}
        for c in cases:
            if "us" in c and c.get("bus_bytes_per_rank", 0) > 0:
                by_kind.setdefault(c["kind"], []).append((float(c["bus_bytes_per_rank"]), c["us"] * 1e-6))
        fits = []
        for kind, pts in sorted(by_kind.items()):
            x = np.array([p[0] for p in pts])
            t = np.array([p[1] for p in pts])
            if len(set(x.tolist())) >= 2:
                slope, lat = np.polyfit(x, t, 1)
                if lat < 0:  # through the origin
                    lat, slope = 0.0, float((x * t).sum() / (x * x).sum())
            else:
                lat = min(fallback.latency_s, float(t.min()))
                slope = float(((t - lat) / x).mean())
            if slope <= 0:
                continue
            fits.append((kind, float(lat), float(1.0 / slope)))
        return cls(tuple(fits), fallback)

    @classmethod
    def from_bench_line(cls, line: str | dict) -> "MeasuredCostModel":
        """From one JSON line of ``bench.py --redistribute``."""
        import json

        d = json.loads(line) if isinstance(line, str) else line
        return cls.fit(d["cases"])


def bus_bytes(entry: CommPlanEntry) -> int:
    """Bytes one rank moves for ``entry`` by the NCCL bus-bytes convention."""
    n = max(1, len({s.src_dpu for s in entry.collect_segments} | {s.dst_dpu for s in entry.writeback_segments}))
    size = entry.numel * entry.dtype.itemsize
    factor = {"all_reduce": 2 * (n - 1) / n, "all_gather": (n - 1) / n,
              "all_to_all": (n - 1) / (n * n)}.get(entry.type, 1.0)
    return int(size * factor)


def plan_cost(entry: CommPlanEntry, model=None) -> CommCost:
    model = model or HostStarCostModel()
    if isinstance(model, (NvlinkCostModel, MeasuredCostModel)):
        bus = bus_bytes(entry)
        if isinstance(model, NvlinkCostModel):
            lat, bw = model.latency_s, model.bus_bytes_per_s
        else:
            lat, bw = model.params(entry.type)
        return CommCost(1 if entry.segments else 0, bus, (lat if entry.segments else 0.0) + bus / bw)
    ops = dma_sequence(entry)
    nbytes = sum(s.nbytes for op in ops for s in op.segments)
    return CommCost(len(ops), nbytes, len(ops) * model.dma_setup_s + nbytes / model.host_bytes_per_s)


def format_comm_plan(entries: list[CommPlanEntry], *, max_segments: int | None = None) -> str:
    lines = [f"== comm plan ({len(entries)} entries) =="]
    counts: dict[str, int] = {}
    for e in entries:
        counts[e.type] = counts.get(e.type, 0) + 1
        lines.append(f"e{e.edge_id}: {e.type} shape={e.shape} dtype={e.dtype} wait_for={list(e.wait_for)}"
                     f" dst_loc={e.dst_loc} segments={len(e.segments)}")
        shown = e.segments if max_segments is None else e.segments[:max_segments]
        for s in shown:
            lines.append(f"    src_dpu={s.src_dpu} src_local={s.src_local_range} global={s.global_range}"
                         f" dst_dpu={s.dst_dpu} dst_off={s.dst_local_offset} nbytes={s.nbytes}"
                         f" src_addr={s.src_addr} dst_addr={s.dst_addr}" + (f" reduce={s.reduce}" if s.reduce else ""))
        if len(shown) < len(e.segments):
            lines.append(f"    ... {len(e.segments) - len(shown)} more")
    lines.append(f"== by type == {dict(sorted(counts.items()))}")
    return "\n".join(lines)
