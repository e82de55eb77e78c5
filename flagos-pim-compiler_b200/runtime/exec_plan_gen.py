"""Compile an annotated step graph into an ExecutionPlan (command DAG).

Implements the generator the reference specifies but leaves empty
(runtime/exec_plan_gen.py is 0 bytes; algorithm in docs/spec.md:1397-1529):

* one ``launch`` per (dpu node, rank) with the byte intervals it reads and
  writes (inputs, weights, output, and -- docs/spec.md:1529 -- the KV blocks
  the kernel touches);
* waits from an interval ``writers`` table (read-after-write, plus
  write-after-write) and from the planner's ``pending_readers`` translated
  through ``reader_cmds`` (write-after-read), docs/spec.md:1427-1466;
* every redistribute edge expands into the fixed template of its type
  (docs/spec.md:1471-1506): collect transfers -> one host combine command ->
  writeback transfers; scatter is host_slice -> writebacks;
* host nodes become one ``host_op`` each (docs/spec.md:1512-1525).

Transfer direction follows the HAL contract, not the spec's prose
(backend/hal_numpy.py:114-139): ``dma_out`` moves DPU -> host (collect) and
``dma_in`` moves host -> DPU (writeback).

Payloads are declarative (offsets, shapes, dtypes, the comm entry), so the
same plan runs on the CPU oracle HAL and on the B200 HAL; each HAL binds its
own implementation of every kernel and host command.

Edges with one source rank whose destination is that same rank
(all_reduce / all_gather at TP=1) are identities and emit no commands: the
consumer reads the producer's bytes in place.  (A sum over one partial equals
the partial; the only observable difference from an explicit ``0 + x`` is
that a stored -0.0 stays -0.0.)
"""

from __future__ import annotations

from dataclasses import dataclass, field
from math import prod

from comm.plan import CommPlanEntry
from contracts.exec_plan import Access, Command, ExecutionPlan
from contracts.pim_tensor_spec import RedistributeEdge
from graph.llama import REDISTRIBUTE_META_KEY, SPEC_META_KEY, OpGraph, OpNode, dtype_bytes
from memory.kv_layout import KVRegionSpec, kv_layer_access
from memory.mem_planner import DPUPlan, align_up

HOST = ("host", None)
VIRTUAL_HOST_BASE = 1 << 48  # host staging that no host node reads: dependency tracking only

HOST_COMBINE = {"all_reduce": "host_reduce", "all_gather": "host_concat", "all_to_all": "host_permute"}


def is_identity_edge(e: RedistributeEdge) -> bool:
    if e.type not in ("all_reduce", "all_gather"):
        return False
    if e.src_spec.device != "dpu" or e.dst_spec.device != "dpu":
        return False
    ranks = set(e.src_spec.shard_map)
    return len(ranks) == 1 and ranks == set(e.dst_spec.shard_map)


@dataclass
class HostLayout:
    """Byte layout of host-resident tensors (the "host" location)."""

    offsets: dict[str, int] = field(default_factory=dict)
    sizes: dict[str, int] = field(default_factory=dict)
    total: int = 0
    virtual_next: int = VIRTUAL_HOST_BASE

    def alloc(self, key: str, nbytes: int, virtual: bool = False) -> int:
        if key in self.offsets:
            return self.offsets[key]
        if virtual:
            off = self.virtual_next
            self.virtual_next += align_up(max(nbytes, 1), 256)
        else:
            off = self.total
            self.total += align_up(max(nbytes, 1), 256)
        self.offsets[key] = off
        self.sizes[key] = nbytes
        return off


@dataclass
class TensorRef:
    """Where one rank (or the host) finds a tensor: byte offset, local shape, dtype."""

    loc: tuple
    offset: int
    shape: tuple[int, ...]
    dtype: str

    @property
    def nbytes(self) -> int:
        return prod(self.shape) * dtype_bytes(self.dtype)

    @property
    def access(self) -> Access:
        return Access(self.loc, self.offset, self.nbytes)

    def as_tuple(self) -> tuple:
        return (self.offset, tuple(self.shape), self.dtype)


class _Gen:
    def __init__(self, g: OpGraph, entries: dict[int, CommPlanEntry], plans: dict[int, DPUPlan],
                 kv_specs: dict[int, KVRegionSpec], host: HostLayout) -> None:
        self.g, self.entries, self.plans, self.kv, self.host = g, entries, plans, kv_specs, host
        self.plan = ExecutionPlan(commands=[])
        self.writers: dict[tuple, list[tuple[Access, int]]] = {}
        self.reader_cmds: dict[tuple[str, object], list[int]] = {}
        self.pending = {r: p.pending_readers.get(g.name, {}) for r, p in plans.items()}
        self.edge_host: dict[int, int] = {}
        self.consumer_view: dict[tuple[str, str], RedistributeEdge] = {}
        self.host_readers: list[tuple[Access, int]] = []

    # -- bookkeeping -------------------------------------------------------
    def append(self, op, dpu_id, payload, reads=(), writes=(), extra_waits=()) -> Command:
        waits = []
        for a in list(reads) + list(writes):
            for wa, cid in self.writers.get(a.loc, []):
                if a.overlaps(wa) and cid not in waits:
                    waits.append(cid)
        for w in writes:
            if w.loc[0] == "dpu":
                for rid in self.pending.get(w.loc[1], {}).get((w.loc, w.offset), []):
                    for cid in self.reader_cmds.get((rid, w.loc[1]), []):
                        if cid not in waits:
                            waits.append(cid)
            else:
                # Host buffers are not reused by the planner; a host write that
                # overlaps an earlier host read (the decode plan overwriting its
                # own input tokens) waits for that reader directly.
                for ra, cid in self.host_readers:
                    if w.overlaps(ra) and cid not in waits:
                        waits.append(cid)
        for cid in extra_waits:
            if cid not in waits:
                waits.append(cid)
        cmd = Command(len(self.plan.commands), op, dpu_id, payload, list(reads), list(writes), sorted(waits))
        self.plan.commands.append(cmd)
        for w in writes:
            self.writers.setdefault(w.loc, []).append((w, cmd.id))
        for r in reads:
            if r.loc == HOST:
                self.host_readers.append((r, cmd.id))
        return cmd

    def note_reader(self, reader_id: str, rank, cid: int) -> None:
        self.reader_cmds.setdefault((reader_id, rank), []).append(cid)

    # -- tensor locations --------------------------------------------------
    def dpu_ref(self, name: str, rank: int) -> TensorRef:
        node = self.g.node(name)
        spec = node.meta[SPEC_META_KEY]
        det = spec.shard_map[rank]
        return TensorRef(("dpu", rank), det.mram_offset, tuple(det.local_shape), node.dtype)

    def host_ref(self, name: str) -> TensorRef:
        node = self.g.node(name)
        return TensorRef(HOST, self.host.offsets[name], tuple(node.shape), node.dtype)

    def input_ref(self, consumer: OpNode, arg: str, rank) -> TensorRef:
        e = self.consumer_view.get((consumer.name, arg))
        if e is not None and not is_identity_edge(e) and e.type != "local_slice":
            if e.dst_spec.device == "host":
                return TensorRef(HOST, self.edge_host[e.edge_id], tuple(e.shape), e.dtype)
            det = e.dst_spec.shard_map[rank]
            return TensorRef(("dpu", rank), det.mram_offset, tuple(det.local_shape), e.dtype)
        src = self.g.node(arg)
        if src.meta[SPEC_META_KEY].device == "host":
            return self.host_ref(arg)
        return self.dpu_ref(arg, rank)

    # -- emitters ----------------------------------------------------------
    def emit_redistribute(self, consumer: OpNode, e: RedistributeEdge) -> None:
        self.consumer_view[(consumer.name, e.src)] = e
        if is_identity_edge(e) or e.type == "local_slice":
            return
        entry = self.entries[e.edge_id]
        itemsize = entry.dtype.itemsize
        host_is_consumer = e.dst_spec.device == "host"
        hb = self.host.alloc(f"edge{e.edge_id}", entry.numel * itemsize, virtual=not host_is_consumer)
        self.edge_host[e.edge_id] = hb
        host_acc = Access(HOST, hb, entry.numel * itemsize)
        reader_id = f"edge{e.edge_id}"
        # A HAL may perform the whole edge inside the combine command (the B200 HAL
        # reads the sources and writes every destination there), so the combine
        # declares those intervals too: it then waits for the destinations' earlier
        # readers (WAR) and later writers of a source wait for it.  For a HAL that
        # moves bytes in the transfers these extra waits are merely conservative.
        wb_writes = [Access(("dpu", s.dst_dpu), s.dst_addr, s.nbytes) for s in entry.writeback_segments]
        if e.type == "scatter":
            src = self.host_ref(e.src)
            combine = self.append("host_slice", None,
                                  {"edge": e.edge_id, "entry": entry, "role": "combine", "kind": "scatter",
                                   "src_host": src.offset, "host_offset": hb},
                                  reads=[src.access], writes=[host_acc] + wb_writes)
        else:
            collect = []
            src_reads = []
            for i, s in enumerate(entry.collect_segments):
                r = Access(("dpu", s.src_dpu), s.src_addr, s.nbytes)
                src_reads.append(r)
                cmd = self.append("dma_out", s.src_dpu,
                                  {"offset": s.src_addr, "shape": (s.nbytes // itemsize,), "dtype": entry.dtype,
                                   "edge": e.edge_id, "segment": i, "role": "collect"},
                                  reads=[r])
                self.note_reader(reader_id, s.src_dpu, cmd.id)
                collect.append(cmd.id)
            combine = self.append(HOST_COMBINE[e.type], None,
                                  {"edge": e.edge_id, "entry": entry, "role": "combine", "kind": e.type,
                                   "collect": collect, "host_offset": hb},
                                  reads=src_reads, writes=[host_acc] + wb_writes, extra_waits=collect)
            for s in entry.collect_segments:
                self.note_reader(reader_id, s.src_dpu, combine.id)
        for i, s in enumerate(entry.writeback_segments):
            src_acc = Access(HOST, hb + s.global_range[0] * itemsize, s.nbytes)
            dst_acc = Access(("dpu", s.dst_dpu), s.dst_addr, s.nbytes)
            self.append("dma_in", s.dst_dpu,
                        {"offset": s.dst_addr, "host_offset": src_acc.offset, "nbytes": s.nbytes,
                         "dtype": entry.dtype, "edge": e.edge_id, "segment": i, "role": "writeback",
                         "data": None},
                        reads=[src_acc], writes=[dst_acc], extra_waits=[combine.id])

    def kv_info(self, rank: int, layer: int) -> dict:
        s = self.kv[rank]
        return {"layer_base": s.kv_off[(layer, s.kv_heads[0], "k")],
                "block_stride": (s.kv_off[(layer, s.kv_heads[0], "v")] - s.kv_off[(layer, s.kv_heads[0], "k")]),
                "seq_stride": s.seq_stride, "max_seq": s.max_seq, "head_dim": s.head_dim,
                "kv_heads": list(s.kv_heads), "num_seqs": s.num_seqs, "dtype": s.dtype_name}

    def emit_launch(self, n: OpNode) -> None:
        spec = n.meta[SPEC_META_KEY]
        for rank in sorted(spec.shard_map):
            ins = [self.input_ref(n, a, rank) for a in n.args]
            out = self.dpu_ref(n.name, rank)
            reads = [r.access for r in ins]
            writes = [out.access]
            payload = {"kernel": n.op, "node": n.name, "graph": self.g.name, "rank": rank,
                       "inputs": [r.as_tuple() for r in ins], "output": out.as_tuple(), "attrs": dict(n.attrs),
                       "tp": len(spec.shard_map)}
            if n.op in ("attn_in", "attention"):
                layer = n.attrs["layer"]
                payload["kv"] = self.kv_info(rank, layer)
                acc = kv_layer_access(self.kv[rank], layer)
                (writes if n.op == "attn_in" else reads).append(acc)
            cmd = self.append("launch", rank, payload, reads=reads, writes=writes)
            for a in n.args:
                e = self.consumer_view.get((n.name, a))
                rid = n.name
                if e is not None and not is_identity_edge(e) and e.type != "local_slice":
                    rid = n.name  # the consumer reads the materialized copy, registered under its own name
                self.note_reader(rid, rank, cmd.id)

    def emit_host_op(self, n: OpNode) -> None:
        ins = [self.input_ref(n, a, None) for a in n.args]
        out = None
        writes = []
        if n.op != "output":
            out_name = n.attrs.get("target", n.name) if n.op == "feed_next" else n.name
            out = self.host_ref(out_name)
            writes.append(out.access)
        self.append("host_op", None,
                    {"kernel": n.op, "node": n.name, "graph": self.g.name,
                     "inputs": [r.as_tuple() for r in ins], "output": out.as_tuple() if out else None,
                     "attrs": dict(n.attrs)},
                    reads=[r.access for r in ins], writes=writes)

    def run(self) -> ExecutionPlan:
        g = self.g
        for n in g.nodes:
            host_weight = n.op == "weight" and n.meta[SPEC_META_KEY].device == "host"
            if n.op == "input" or host_weight or (n.device == "host" and n.op not in ("weight", "output")):
                if n.op != "feed_next":
                    self.host.alloc(n.name, n.nbytes)
        for n in g.nodes:
            if n.op in ("weight", "input"):
                continue
            for e in n.meta.get(REDISTRIBUTE_META_KEY, []):
                self.emit_redistribute(n, e)
            spec = n.meta.get(SPEC_META_KEY)
            if spec is not None and spec.device == "dpu":
                self.emit_launch(n)
            else:
                self.emit_host_op(n)
        names = {n.name for n in g.nodes}
        if {"input_ids", "positions", "next_token"} <= names:  # a LLaMA step graph of graph/llama.py
            inputs = {k: self.host_ref(k) for k in ("input_ids", "positions")}
            outputs = {"logits": self._logits_ref(), "token": self.host_ref("next_token")}
        else:  # an exported graph: its placeholders, and the operands of its output node
            inputs = {n.name: self.host_ref(n.name) for n in g.nodes if n.op == "input"}
            out = next((n for n in g.nodes if n.op == "output"), None)
            outputs = {a: self.input_ref(out, a, None) for a in out.args} if out is not None else {}
        self.plan.meta.update({"graph": g.name, "phase": g.phase, "batch": g.batch, "seq": g.seq,
                               "host_layout": self.host, "inputs": inputs, "outputs": outputs,
                               "host_weights": {n.name: self.host_ref(n.name) for n in g.nodes
                                                if n.op == "weight" and n.meta[SPEC_META_KEY].device == "host"}})
        return self.plan

    def _logits_ref(self) -> TensorRef:
        return self.input_ref(self.g.node("next_token"), "logits", None)


def build_execution_plan(g: OpGraph, entries: list[CommPlanEntry], plans: dict[int, DPUPlan],
                         kv_specs: dict[int, KVRegionSpec], host: HostLayout | None = None) -> ExecutionPlan:
    """ExecutionPlan for one graph; ``host`` may be shared between the prefill and decode plans."""
    return _Gen(g, {e.edge_id: e for e in entries}, plans, kv_specs, host or HostLayout()).run()


# ---------------------------------------------------------------------------
# one redistribute edge on its own (the redistribute microbench)
# ---------------------------------------------------------------------------


def redistribute_edge(kind: str, n: int, shape: tuple[int, ...], dtype: str = "bfloat16"):
    """``(edge, entry)``: one redistribute of a ``shape`` tensor over ranks 0..n-1.

    all_reduce is Partial -> Replicate, all_gather Shard(last) -> Replicate, all_to_all
    Shard(0) -> Shard(1) and scatter host -> Shard(0) (the four placements of the
    reference's comm tests, tests/test_comm_lowering.py:34-185).  Every rank's source
    sits at arena offset 0 and its destination right after the whole tensor's bytes.
    """
    from dataclasses import replace

    from comm.plan import build_comm_plan
    from contracts.pim_tensor_spec import PARTIAL_SUM, REPLICATE, Placement
    from graph.llama import dpu_spec, host_spec

    dpus = tuple(range(n))
    nbytes = prod(shape) * dtype_bytes(dtype)
    if kind == "all_reduce":
        src, dst = dpu_spec(PARTIAL_SUM, shape, dpus), dpu_spec(REPLICATE, shape, dpus)
    elif kind == "all_gather":
        src, dst = dpu_spec(Placement("Shard", len(shape) - 1), shape, dpus), dpu_spec(REPLICATE, shape, dpus)
    elif kind == "all_to_all":
        src, dst = dpu_spec(Placement("Shard", 0), shape, dpus), dpu_spec(Placement("Shard", 1), shape, dpus)
    elif kind == "scatter":
        src, dst = host_spec(), dpu_spec(Placement("Shard", 0), shape, dpus)
    else:
        raise ValueError(f"unknown redistribute kind {kind!r}")
    dst.shard_map = {r: replace(d, mram_offset=nbytes) for r, d in dst.shard_map.items()}
    edge = RedistributeEdge(0, "producer", "consumer", src.placement, dst.placement, src, dst, kind,
                            {"device": "host"} if src.device == "host" else {"device": "dpu", "dpus": list(dpus)},
                            {"device": "dpu", "dpus": list(dpus)}, nbytes,
                            "sum" if kind == "all_reduce" else None, tuple(shape), dtype)
    (entry,) = build_comm_plan([edge])
    return edge, entry


class _EdgeGen(_Gen):
    """Generator state for a plan holding one edge and nothing else."""

    def __init__(self, edge: RedistributeEdge, entry: CommPlanEntry) -> None:
        g = OpGraph("redistribute", "redistribute", None, 1, 1, [])
        super().__init__(g, {entry.edge_id: entry}, {}, {}, HostLayout())
        self.edge = edge

    def host_ref(self, name: str) -> TensorRef:  # the scatter's host source: the whole tensor
        return TensorRef(HOST, self.host.offsets[name], tuple(self.edge.shape), self.edge.dtype)


def redistribute_plan(edge: RedistributeEdge, entry: CommPlanEntry) -> ExecutionPlan:
    """ExecutionPlan of one edge: the fixed template of its type (docs/spec.md:1471-1506)."""
    gen = _EdgeGen(edge, entry)
    if edge.type == "scatter":
        gen.host.alloc(edge.src, entry.numel * entry.dtype.itemsize)
    consumer = OpNode(edge.dst, "output", (edge.src,), tuple(edge.shape), edge.dtype)
    gen.emit_redistribute(consumer, edge)
    gen.plan.meta.update({"graph": "redistribute", "phase": "redistribute", "host_layout": gen.host,
                          "edge": edge.edge_id, "kind": edge.type, "inputs": {}, "outputs": {}})
    return gen.plan
