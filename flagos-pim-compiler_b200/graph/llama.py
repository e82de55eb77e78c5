"""LLaMA step graphs at the granularity of the B200 kernels.

A prefill graph processes ``batch x seq`` prompt tokens; a decode graph
processes one new token per sequence.  Both are plain topologically ordered
node lists (the role the exported FX graph plays for the reference, whose
passes annotate ``node.meta["device"]``, ``["spec"]`` and
``["redistribute"]`` -- graph/partition.py:36-81, graph/spec_prop.py:411-451).
This module keeps those three annotation keys on every node so the comm plan,
the memory planner and the ExecutionPlan generator consume the same
information the reference passes produce.

Node granularity follows the fused kernels, not single aten ops.  The
correspondence to the HF ``LlamaForCausalLM`` graph the reference exports:

=================  ========================================================
node op            HF ops covered
=================  ========================================================
``embedding``      ``embed_tokens``
``attn_in``        ``input_layernorm`` + ``q/k/v_proj`` + RoPE on q, k +
                   the KV append of k, v at the step's positions
``attention``      ``scaled_dot_product_attention`` (causal / decode) over
                   the layer's KV blocks
``linear``         ``o_proj`` / ``down_proj`` (row-sharded, Partial output)
``add``            residual adds
``mlp_in``         ``post_attention_layernorm`` + ``gate/up_proj`` +
                   ``silu(gate) * up``
``lm_head_in``     final ``norm`` + ``lm_head``
``select_last``    taking the last prompt position (prefill only)
``argmax``         greedy sampling (host)
``feed_next``      the sampled token becomes the next step's input (host)
=================  ========================================================

The shard layout is Megatron column/row exactly as ``llama_shard_config``
(graph/spec_prop.py:77-120): q/k/v/gate/up/lm_head Shard(0),
o/down Shard(1).  Two fused weights exist only as a memory layout:
``qkv_proj.weight`` is the rank-major concatenation ``[q_d; k_d; v_d]`` for
d = 0..N-1, and ``gate_up_proj.weight`` is ``[gate_d; up_d]``; Shard(0) of
each gives every rank exactly its own column blocks.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from math import prod

from contracts.pim_tensor_spec import (
    PARTIAL_SUM,
    REPLICATE,
    PIMTensorSpec,
    Placement,
    RedistributeEdge,
    TensorShardDetail,
)

DEVICE_META_KEY = "device"
SPEC_META_KEY = "spec"
REDISTRIBUTE_META_KEY = "redistribute"

_DTYPE_BYTES = {"float32": 4, "bfloat16": 2, "float16": 2, "int32": 4, "int64": 8, "uint8": 1}


def dtype_bytes(name: str) -> int:
    return _DTYPE_BYTES[name]


@dataclass(frozen=True)
class ModelConfig:
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    rms_eps: float
    rope_theta: float
    dtype: str  # weight / activation dtype: "float32" or "bfloat16"
    max_seq: int  # KV reservation per sequence

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads

    @classmethod
    def tiny(cls, max_seq: int = 32) -> "ModelConfig":
        """2 layers, hidden 256, 4x64 MHA, MLP 688, vocab 1024, fp32 (the CPU-runnable case)."""
        return cls(1024, 256, 688, 2, 4, 4, 1e-6, 10000.0, "float32", max_seq)

    @classmethod
    def llama2_7b(cls, max_seq: int = 256, num_layers: int = 32, dtype: str = "bfloat16") -> "ModelConfig":
        return cls(32000, 4096, 11008, num_layers, 32, 32, 1e-5, 10000.0, dtype, max_seq)

    @classmethod
    def from_hf(cls, cfg, max_seq: int, dtype: str) -> "ModelConfig":
        return cls(cfg.vocab_size, cfg.hidden_size, cfg.intermediate_size, cfg.num_hidden_layers,
                   cfg.num_attention_heads, cfg.num_key_value_heads, float(cfg.rms_norm_eps),
                   float(getattr(cfg, "rope_theta", 10000.0)), dtype, max_seq)

    def weight_bytes(self) -> int:
        """Bytes of every weight read by one decode step (embedding rows excluded)."""
        h, i, v, hd = self.hidden_size, self.intermediate_size, self.vocab_size, self.head_dim
        per_layer = (h * h + 2 * self.num_kv_heads * hd * h + h * h + 3 * h * i + 2 * h)
        return (self.num_layers * per_layer + v * h + h) * dtype_bytes(self.dtype)


@dataclass
class OpNode:
    name: str
    op: str
    args: tuple[str, ...]
    shape: tuple[int, ...]
    dtype: str
    device: str = "dpu"
    attrs: dict = field(default_factory=dict)
    meta: dict = field(default_factory=dict)

    @property
    def nbytes(self) -> int:
        return prod(self.shape) * dtype_bytes(self.dtype)


@dataclass
class OpGraph:
    name: str
    phase: str  # "prefill" | "decode"
    model: ModelConfig
    batch: int
    seq: int
    nodes: list[OpNode]

    def node(self, name: str) -> OpNode:
        return self._index()[name]

    def _index(self) -> dict[str, OpNode]:
        if getattr(self, "_idx", None) is None or len(self._idx) != len(self.nodes):
            self._idx = {n.name: n for n in self.nodes}
        return self._idx

    def users(self, name: str) -> list[OpNode]:
        return [n for n in self.nodes if name in n.args]


# ---------------------------------------------------------------------------
# graph construction
# ---------------------------------------------------------------------------


def weight_names(cfg: ModelConfig) -> list[str]:
    names = ["model.embed_tokens.weight", "model.rotary.cos", "model.rotary.sin"]
    for l in range(cfg.num_layers):
        p = f"model.layers.{l}."
        names += [p + "input_layernorm.weight", p + "self_attn.qkv_proj.weight", p + "self_attn.o_proj.weight",
                  p + "post_attention_layernorm.weight", p + "mlp.gate_up_proj.weight", p + "mlp.down_proj.weight"]
    names += ["model.norm.weight", "lm_head.weight"]
    return names


def weight_shape(cfg: ModelConfig, name: str) -> tuple[tuple[int, ...], str]:
    h, i, v, hd = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size, cfg.head_dim
    if name.endswith("embed_tokens.weight"):
        return (v, h), cfg.dtype
    if name.startswith("model.rotary."):
        return (cfg.max_seq, hd // 2), "float32"
    if name.endswith("layernorm.weight") or name == "model.norm.weight":
        return (h,), cfg.dtype
    if name.endswith("qkv_proj.weight"):
        return ((cfg.num_heads + 2 * cfg.num_kv_heads) * hd, h), cfg.dtype
    if name.endswith("o_proj.weight"):
        return (h, cfg.num_heads * hd), cfg.dtype
    if name.endswith("gate_up_proj.weight"):
        return (2 * i, h), cfg.dtype
    if name.endswith("down_proj.weight"):
        return (h, i), cfg.dtype
    if name == "lm_head.weight":
        return (v, h), cfg.dtype
    raise KeyError(name)


def build_llama_graph(cfg: ModelConfig, phase: str, batch: int, seq: int, fuse_residual: bool = False) -> OpGraph:
    """Fused-op graph for one prefill pass (``seq`` prompt tokens) or one decode step (seq=1).

    ``fuse_residual`` replaces each o_proj/down_proj ``linear`` + residual ``add``
    pair by one ``linear_add`` node (the add done in the projection's epilogue).
    It is only valid on one rank, where the Partial -> Replicate exchange between
    the two is an identity.
    """
    if phase == "decode" and seq != 1:
        raise ValueError("a decode step processes exactly one token per sequence")
    if phase not in ("prefill", "decode"):
        raise ValueError(phase)
    h, hd, dt = cfg.hidden_size, cfg.head_dim, cfg.dtype
    B, S = batch, seq
    nodes: list[OpNode] = []

    def add(name, op, args, shape, dtype=dt, device="dpu", **attrs):
        nodes.append(OpNode(name, op, tuple(args), tuple(shape), dtype, device, attrs))
        return name

    for w in weight_names(cfg):
        shape, wdt = weight_shape(cfg, w)
        add(w, "weight", (), shape, wdt, "host")
    ids = add("input_ids", "input", (), (B, S), "int32", "host")
    pos = add("positions", "input", (), (B,), "int32", "host")
    pos_d = add("positions_dev", "materialize", (pos,), (B,), "int32")
    ids_d = add("input_ids_dev", "materialize", (ids,), (B, S), "int32")
    x = add("embedding", "embedding", (ids_d, "model.embed_tokens.weight"), (B, S, h))
    q_dim = cfg.num_heads * hd
    for l in range(cfg.num_layers):
        p = f"model.layers.{l}."
        q = add(f"l{l}.q_rot", "attn_in", (x, p + "input_layernorm.weight", p + "self_attn.qkv_proj.weight",
                                           "model.rotary.cos", "model.rotary.sin", pos_d),
                (B, S, q_dim), layer=l, eps=cfg.rms_eps)
        a = add(f"l{l}.attn", "attention", (q, pos_d), (B, S, q_dim), layer=l, causal=(phase == "prefill"))
        if fuse_residual:
            x = add(f"l{l}.resid_attn", "linear_add", (a, p + "self_attn.o_proj.weight", x), (B, S, h))
        else:
            o = add(f"l{l}.o_proj", "linear", (a, p + "self_attn.o_proj.weight"), (B, S, h))
            x = add(f"l{l}.resid_attn", "add", (x, o), (B, S, h))
        m = add(f"l{l}.mlp_act", "mlp_in", (x, p + "post_attention_layernorm.weight", p + "mlp.gate_up_proj.weight"),
                (B, S, cfg.intermediate_size), layer=l, eps=cfg.rms_eps)
        if fuse_residual:
            x = add(f"l{l}.resid_mlp", "linear_add", (m, p + "mlp.down_proj.weight", x), (B, S, h))
        else:
            d = add(f"l{l}.down_proj", "linear", (m, p + "mlp.down_proj.weight"), (B, S, h))
            x = add(f"l{l}.resid_mlp", "add", (x, d), (B, S, h))
    if phase == "prefill":
        x = add("last_hidden", "select_last", (x,), (B, 1, h), index=S - 1)
    logits = add("logits", "lm_head_in", (x, "model.norm.weight", "lm_head.weight"), (B, 1, cfg.vocab_size),
                 eps=cfg.rms_eps)
    tok = add("next_token", "argmax", (logits,), (B,), "int32", "host")
    if phase == "decode":
        add("feed_next", "feed_next", (tok,), (B,), "int32", "host", target="input_ids")
    # The gathered logits are read through argmax's input (one gather per step).
    add("output", "output", (tok,), (), "float32", "host")
    return OpGraph(f"llama_{phase}_b{B}_s{S}", phase, cfg, B, S, nodes)


# ---------------------------------------------------------------------------
# placement propagation (the role of graph/spec_prop.py)
# ---------------------------------------------------------------------------


@dataclass(frozen=True)
class ShardConfig:
    """Megatron column/row split for ``num_dpus`` ranks (graph/spec_prop.py:49-120)."""

    num_dpus: int
    dpu_ids: tuple[int, ...] | None = None

    def __post_init__(self) -> None:
        if self.num_dpus <= 0:
            raise ValueError("num_dpus must be positive")
        if self.num_dpus & (self.num_dpus - 1):
            raise ValueError(f"num_dpus={self.num_dpus} is not a power of two")
        ids = tuple(range(self.num_dpus)) if self.dpu_ids is None else tuple(self.dpu_ids)
        if len(ids) != self.num_dpus or len(set(ids)) != len(ids) or min(ids) < 0:
            raise ValueError("dpu_ids must be unique non-negative ids, one per dpu")
        object.__setattr__(self, "dpu_ids", ids)

    def check_model(self, cfg: ModelConfig) -> None:
        for name, n in (("num_heads", cfg.num_heads), ("num_kv_heads", cfg.num_kv_heads),
                        ("intermediate_size", cfg.intermediate_size), ("vocab_size", cfg.vocab_size)):
            if n % self.num_dpus:
                raise ValueError(f"{name}={n} is not divisible by num_dpus={self.num_dpus}")

    @staticmethod
    def weight_rule(name: str) -> str | None:
        for pattern, mode in (("qkv_proj.weight", "col"), ("o_proj.weight", "row"), ("gate_up_proj.weight", "col"),
                              ("down_proj.weight", "row"), ("lm_head.weight", "col")):
            if pattern in name:
                return mode
        return None


def host_spec() -> PIMTensorSpec:
    return PIMTensorSpec("host", REPLICATE, "transient", None, {}, None)


def dpu_spec(placement: Placement, shape: tuple[int, ...], dpus: tuple[int, ...],
             residency: str = "transient") -> PIMTensorSpec:
    if placement.kind == "Shard":
        d = placement.dim
        if d >= len(shape):
            raise ValueError(f"shape={shape} has no dim {d}")
        if shape[d] % len(dpus):
            raise ValueError(f"dim {d} of {shape} is not divisible by {len(dpus)} dpus")
        w = shape[d] // len(dpus)
        smap = {r: TensorShardDetail(r, d, i * w, (i + 1) * w, shape[:d] + (w,) + shape[d + 1:])
                for i, r in enumerate(dpus)}
    else:
        n = prod(shape)
        smap = {r: TensorShardDetail(r, -1, 0, n, tuple(shape)) for r in dpus}
    spec = PIMTensorSpec("dpu", placement, residency, None, smap, placement.reduce_type)
    spec.validate()
    return spec


def _shard_last(node: OpNode) -> Placement:
    return Placement("Shard", len(node.shape) - 1)


# Consumer requirements per op: list of (arg index, placement) for tensor inputs
# that are activations; weights are pinned and checked separately.
def _rule(node: OpNode, specs: dict[str, PIMTensorSpec], g: OpGraph, sc: ShardConfig):
    op = node.op
    if op == "materialize":
        return [(0, REPLICATE)], REPLICATE
    if op == "embedding":
        return [(0, REPLICATE)], REPLICATE
    if op == "attn_in":
        return [(0, REPLICATE), (5, REPLICATE)], _shard_last(node)
    if op == "mlp_in":
        return [(0, REPLICATE)], _shard_last(node)
    if op == "attention":
        return [(0, _shard_last(node)), (1, REPLICATE)], _shard_last(node)
    if op == "linear":
        w = specs[node.args[1]].placement
        if w == Placement("Shard", 0):
            return [(0, REPLICATE)], _shard_last(node)
        if w == Placement("Shard", 1):
            return [(0, _shard_last(node))], PARTIAL_SUM
        raise NotImplementedError(f"{node.name}: unsupported weight placement {w}")
    if op == "add":
        a, b = (specs[x].placement for x in node.args)
        kinds = {a.kind, b.kind}
        if a.kind == b.kind == "Shard":
            if a.dim != b.dim:
                raise NotImplementedError(f"{node.name}: Shard dims differ (needs all_to_all)")
            return [(0, a), (1, a)], a
        if kinds == {"Shard", "Replicate"}:
            out = a if a.kind == "Shard" else b
            return [(0, out), (1, out)], out
        if a.kind == b.kind == "Partial":
            if a.reduce_type != b.reduce_type:
                raise ValueError(f"{node.name}: Partial reduce types differ")
            return [(0, a), (1, a)], a
        if kinds <= {"Partial", "Replicate"}:
            return [(0, REPLICATE), (1, REPLICATE)], REPLICATE
        raise NotImplementedError(f"{node.name}: unsupported layouts {a}, {b}")
    if op == "linear_add":
        if sc.num_dpus != 1:
            raise ValueError(f"{node.name}: linear_add fuses a Partial sum and is only valid on one rank")
        return [(0, _shard_last(node)), (2, REPLICATE)], REPLICATE
    if op == "select_last":
        return [(0, REPLICATE)], REPLICATE
    if op == "lm_head_in":
        return [(0, REPLICATE)], _shard_last(node)
    raise ValueError(f"no placement rule for op {op!r}")


def _edge_type(actual: PIMTensorSpec, want_device: str, want: Placement, name: str) -> str:
    a = actual.placement
    if not (a == want or (a.kind == "Partial" and want.kind == "Replicate")
            or (a.kind == "Shard" and want.kind == "Replicate") or (a.kind == "Replicate" and want.kind == "Shard")
            or (a.kind == "Shard" and want.kind == "Shard")):
        raise ValueError(f"{name}: unsupported layout change {a}@{actual.device} -> {want}@{want_device}")
    if a == want:
        return "scatter" if actual.device == "host" else "all_gather"
    if a.kind == "Partial":
        return "all_reduce"
    if a.kind == "Shard" and want.kind == "Replicate":
        return "all_gather"
    if a.kind == "Shard" and want.kind == "Shard":
        return "all_to_all"
    return "scatter" if actual.device == "host" else "local_slice"


def propagate_specs(g: OpGraph, sc: ShardConfig) -> list[RedistributeEdge]:
    """Annotate every node with device/spec and emit the redistribute edges.

    Weights get their pinned Megatron placement; activations follow the rule
    table above; any producer/consumer mismatch becomes a RedistributeEdge on
    the consumer (``node.meta["redistribute"]``), numbered in discovery order.
    """
    sc.check_model(g.model)
    dpus = sc.dpu_ids
    specs: dict[str, PIMTensorSpec] = {}
    edges: list[RedistributeEdge] = []
    for n in g.nodes:
        n.meta[REDISTRIBUTE_META_KEY] = []
        n.meta[DEVICE_META_KEY] = n.device

    def need(consumer: OpNode, src: str, device: str, placement: Placement) -> None:
        actual = specs[src]
        if actual.device == device and actual.placement == placement:
            return
        if actual.residency == "pinned":
            raise ValueError(f"pinned tensor {src} cannot be redistributed ({actual.placement} -> {placement})")
        node = g.node(src)
        dst = host_spec() if device == "host" else dpu_spec(placement, node.shape, dpus)
        e = RedistributeEdge(
            edge_id=len(edges), src=src, dst=consumer.name, from_placement=actual.placement,
            to_placement=placement, src_spec=actual, dst_spec=dst,
            type=_edge_type(actual, device, placement, consumer.name),
            src_loc={"device": "host"} if actual.device == "host" else {"device": "dpu", "dpus": sorted(actual.shard_map)},
            dst_loc={"device": "host"} if device == "host" else {"device": "dpu", "dpus": sorted(dst.shard_map)},
            nbytes=node.nbytes, reduce_type=actual.reduce_type, shape=node.shape, dtype=node.dtype)
        edges.append(e)
        consumer.meta[REDISTRIBUTE_META_KEY].append(e)

    for n in g.nodes:
        if n.op == "weight":
            users = [u for u in g.nodes if n.name in u.args]
            if any(u.device == "dpu" for u in users):
                mode = ShardConfig.weight_rule(n.name)
                pl = REPLICATE if mode is None else Placement("Shard", 0 if mode == "col" else 1)
                specs[n.name] = dpu_spec(pl, n.shape, dpus, residency="pinned")
                n.device = "dpu"
                n.meta[DEVICE_META_KEY] = "dpu"
            else:
                specs[n.name] = host_spec()
        elif n.op == "input":
            specs[n.name] = host_spec()
        elif n.device == "host":
            for a in n.args:
                need(n, a, "host", REPLICATE)
            specs[n.name] = host_spec()
        else:
            reqs, out = _rule(n, specs, g, sc)
            for idx, pl in reqs:
                need(n, n.args[idx], "dpu", pl)
            specs[n.name] = dpu_spec(out, n.shape, dpus)
        n.meta[SPEC_META_KEY] = specs[n.name]
    return edges


def format_spec_report(g: OpGraph, edges: list[RedistributeEdge]) -> str:
    def fp(p: Placement) -> str:
        return f"Shard({p.dim})" if p.kind == "Shard" else (f"Partial({p.reduce_type})" if p.kind == "Partial" else "Replicate")

    lines = [f"== {g.name}: {len(g.nodes)} nodes =="]
    for n in g.nodes:
        s = n.meta.get(SPEC_META_KEY)
        lines.append(f"  {n.name} [{n.meta.get(DEVICE_META_KEY)}] -> {fp(s.placement)}@{s.device}" if s else f"  {n.name}")
        for e in n.meta.get(REDISTRIBUTE_META_KEY, []):
            lines.append(f"    in e{e.edge_id}: {e.src} {fp(e.from_placement)} -> {fp(e.to_placement)} = {e.type}")
    counts: dict[str, int] = {}
    for e in edges:
        counts[e.type] = counts.get(e.type, 0) + 1
    lines.append(f"== edges by type == {dict(sorted(counts.items()))}")
    return "\n".join(lines)
