"""Compile-time driver: graph -> placements -> comm plan -> memory plan -> ExecutionPlans.

Chains the passes in the order the reference describes for its compile chain
(graph/partition.py, graph/spec_prop.py:411-451, comm/plan.py:294-301,
memory/kv_layout.py:102-145, then the planner and generator of
docs/spec.md:2033-2069 and 1435-1466): both plans of a program share one
weight zone and one KV zone per rank; their activations overlay.

Also packs model weights into per-rank shards that match the memory plan:
HF ``[out, in]`` weights are split Megatron style (q/k/v/gate/up/lm_head by
rows, o/down by columns) and the fused ``qkv_proj`` / ``gate_up_proj``
weights are assembled rank-major.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from comm.plan import CommPlanEntry, build_comm_plan, np_dtype
from contracts.exec_plan import ExecutionPlan
from contracts.pim_tensor_spec import Placement
from graph.llama import (
    SPEC_META_KEY,
    ModelConfig,
    OpGraph,
    ShardConfig,
    build_llama_graph,
    dpu_spec,
    propagate_specs,
    weight_names,
    weight_shape,
)
from memory.kv_layout import KVRegionSpec, kv_specs_from_placement
from memory.mem_planner import DPUPlan, HardwareSpec, backfill_offsets, plan_dpu
from runtime.exec_plan_gen import HostLayout, build_execution_plan


@dataclass
class LlamaProgram:
    cfg: ModelConfig
    shard: ShardConfig
    batch: int
    prompt_len: int
    graphs: dict[str, OpGraph]
    entries: dict[str, list[CommPlanEntry]]
    kv_specs: dict[int, KVRegionSpec]
    dpu_plans: dict[int, DPUPlan]
    plans: dict[str, ExecutionPlan]
    hw: HardwareSpec
    extra: dict = field(default_factory=dict)

    @property
    def arena_bytes(self) -> int:
        return max(p.total for p in self.dpu_plans.values())

    @property
    def tp(self) -> int:
        return self.shard.num_dpus


def compile_llama(cfg: ModelConfig, tp: int, batch: int = 1, prompt_len: int = 16, *,
                  phases=("prefill", "decode"), align: int = 256, mram_budget: int = 1 << 62,
                  reuse: bool = True, fuse_residual: bool | None = None) -> LlamaProgram:
    """Compile prefill/decode ExecutionPlans for ``tp`` ranks.

    ``reuse=False`` gives the debug layout (no activation sharing);
    ``fuse_residual`` (default: on for one rank) folds the residual adds into
    the o_proj / down_proj epilogues.
    """
    sc = ShardConfig(tp)
    sc.check_model(cfg)
    if prompt_len + 1 > cfg.max_seq and "decode" in phases:
        raise ValueError(f"max_seq={cfg.max_seq} leaves no room to decode after a {prompt_len}-token prompt")
    if fuse_residual is None:
        fuse_residual = tp == 1
    graphs, edges, entries = {}, {}, {}
    for ph in phases:
        g = build_llama_graph(cfg, ph, batch, prompt_len if ph == "prefill" else 1, fuse_residual=fuse_residual)
        edges[ph] = propagate_specs(g, sc)
        graphs[ph] = g
    hd = cfg.head_dim
    kproj = dpu_spec(Placement("Shard", 0), (cfg.num_kv_heads * hd, cfg.hidden_size), sc.dpu_ids)
    kv_dtype = cfg.dtype
    kv_specs = kv_specs_from_placement(kproj, num_layers=cfg.num_layers, num_kv_heads=cfg.num_kv_heads,
                                       num_q_heads=cfg.num_heads, head_dim=hd, max_seq=cfg.max_seq,
                                       dtype_bytes=np_dtype(kv_dtype).itemsize, kv_base=0, num_seqs=batch,
                                       dtype=kv_dtype)
    hw = HardwareSpec(mram_budget=mram_budget, align=align)
    glist = list(graphs.values())
    dplans = {r: plan_dpu(glist, r, kv_specs[r], hw, reuse) for r in sc.dpu_ids}
    backfill_offsets(glist, dplans)
    for ph, g in graphs.items():
        entries[ph] = build_comm_plan(edges[ph])
    plans = {ph: build_execution_plan(graphs[ph], entries[ph], dplans, kv_specs, HostLayout()) for ph in graphs}
    for ph, p in plans.items():
        p.meta["program"] = ph
    return LlamaProgram(cfg, sc, batch, prompt_len, graphs, entries, kv_specs, dplans, plans, hw)


# ---------------------------------------------------------------------------
# weights
# ---------------------------------------------------------------------------


def rotary_tables(cfg: ModelConfig) -> tuple[np.ndarray, np.ndarray]:
    """``cos, sin`` of shape ``[max_seq, head_dim/2]`` in fp32, HF LlamaRotaryEmbedding formula.

    For a bf16 model the values are rounded to bf16 first, because HF casts
    cos/sin to the activation dtype before applying them.
    """
    import torch

    hd = cfg.head_dim
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, hd, 2, dtype=torch.int64).float() / hd))
    pos = torch.arange(cfg.max_seq, dtype=torch.float32)
    freqs = pos[:, None] @ inv[None, :]
    cos, sin = freqs.cos(), freqs.sin()
    if cfg.dtype == "bfloat16":
        cos, sin = cos.to(torch.bfloat16).float(), sin.to(torch.bfloat16).float()
    return cos.numpy().astype(np.float32), sin.numpy().astype(np.float32)


def interleave_head_pairs(w: np.ndarray, head_dim: int) -> np.ndarray:
    """Rows of each head block reordered to (j, j + hd/2) pairs: [r0, r0+h, r1, r1+h, ...].

    RoPE mixes exactly those two rows, so a kernel task is two adjacent rows.
    """
    n, k = w.shape
    half = head_dim // 2
    return np.ascontiguousarray(w.reshape(n // head_dim, 2, half, k).transpose(0, 2, 1, 3).reshape(n, k))


def fused_weights(cfg: ModelConfig, sd: dict, tp: int) -> dict[str, np.ndarray]:
    """Logical (global) weights of the step graph from an HF-named state dict of numpy arrays.

    Memory layout of the fused weights (rank-major blocks, then pair-interleaved
    rows so that every two-row task of a kernel reads one contiguous range):

    * ``qkv_proj.weight``: for rank d the q, k and v rows of d's heads, each head
      block in RoPE pair order (``interleave_head_pairs``);
    * ``gate_up_proj.weight``: for rank d the rows gate_0, up_0, gate_1, up_1, ...
    """
    out = fused_globals(cfg, sd)
    for l in range(cfg.num_layers):
        out.update(fused_layer(cfg, sd, tp, l))
    return out


def fused_globals(cfg: ModelConfig, sd) -> dict[str, np.ndarray]:
    """The weights outside the decoder layers (embedding, final norm, lm_head, rotary tables)."""
    out = {"model.embed_tokens.weight": sd["model.embed_tokens.weight"],
           "model.norm.weight": sd["model.norm.weight"], "lm_head.weight": sd["lm_head.weight"]}
    out["model.rotary.cos"], out["model.rotary.sin"] = rotary_tables(cfg)
    return out


def fused_layer(cfg: ModelConfig, sd, tp: int, l: int) -> dict[str, np.ndarray]:
    """Fused weights of decoder layer ``l`` (layout of ``fused_weights``)."""
    hd = cfg.head_dim
    hq, hkv = cfg.num_heads // tp, cfg.num_kv_heads // tp
    i_l = cfg.intermediate_size // tp
    p = f"model.layers.{l}."
    out = {}
    q, k, v = (sd[p + f"self_attn.{n}_proj.weight"] for n in "qkv")
    blocks = []
    for d in range(tp):
        blocks += [interleave_head_pairs(q[d * hq * hd:(d + 1) * hq * hd], hd),
                   interleave_head_pairs(k[d * hkv * hd:(d + 1) * hkv * hd], hd),
                   interleave_head_pairs(v[d * hkv * hd:(d + 1) * hkv * hd], hd)]
    out[p + "self_attn.qkv_proj.weight"] = np.concatenate(blocks, 0)
    gate, up = sd[p + "mlp.gate_proj.weight"], sd[p + "mlp.up_proj.weight"]
    blocks = []
    for d in range(tp):
        g, u = gate[d * i_l:(d + 1) * i_l], up[d * i_l:(d + 1) * i_l]
        blocks.append(np.stack([g, u], axis=1).reshape(2 * i_l, -1))
    out[p + "mlp.gate_up_proj.weight"] = np.concatenate(blocks, 0)
    for n in ("self_attn.o_proj.weight", "mlp.down_proj.weight", "input_layernorm.weight",
              "post_attention_layernorm.weight"):
        out[p + n] = sd[p + n]
    return out


def rank_shards(prog: LlamaProgram, logical: dict[str, np.ndarray]) -> dict[int, list[tuple[int, np.ndarray]]]:
    """``{rank: [(arena offset, contiguous local array)]}`` for every weight on every rank."""
    out: dict[int, list] = {r: [] for r in prog.shard.dpu_ids}
    for name in weight_names(prog.cfg):
        for r, off, local in _name_shards(prog, name, logical[name]):
            out[r].append((off, local))
    return out


def _name_shards(prog: LlamaProgram, name: str, w) -> list[tuple[int, int, np.ndarray]]:
    """``[(rank, arena offset, contiguous local array)]`` of one logical weight."""
    spec = next(iter(prog.graphs.values())).node(name).meta[SPEC_META_KEY]
    shape, dt = weight_shape(prog.cfg, name)
    if tuple(w.shape) != tuple(shape):
        raise ValueError(f"{name}: expected {shape}, got {w.shape}")
    w = np.asarray(w).astype(np_dtype(dt), copy=False)
    out = []
    for r, det in spec.shard_map.items():
        if spec.placement.kind == "Shard":
            sl = [slice(None)] * w.ndim
            sl[det.shard_dim] = slice(det.start_idx, det.end_idx)
            local = np.ascontiguousarray(w[tuple(sl)])
        else:
            local = np.ascontiguousarray(w)
        out.append((r, prog.dpu_plans[r].weight[name], local))
    return out


def hf_state_dict(model, dtype: str) -> dict[str, np.ndarray]:
    """numpy copy of an HF LlamaForCausalLM state dict in ``dtype`` (float32 / bfloat16)."""
    import torch

    out = {}
    for k, v in model.state_dict().items():
        out[k] = v.detach().to(torch.float32).numpy().astype(np_dtype(dtype))
    if "lm_head.weight" not in out:
        out["lm_head.weight"] = out["model.embed_tokens.weight"]
    return out


def load_weights(prog: LlamaProgram, hal, logical: dict[str, np.ndarray]) -> None:
    """Copy every rank's weight shards into its arena (done once, before any plan runs).

    A HAL that owns only some ranks (one process per GPU: ``hal.local``) gets its own.
    """
    local = getattr(hal, "local", None)
    for r, items in rank_shards(prog, logical).items():
        if local is not None and r not in local:
            continue
        for off, arr in items:
            hal.copy_to_dpu(r, off, arr)


def load_state_dict(prog: LlamaProgram, hal, sd) -> None:
    """``load_weights`` from an HF-named state dict (any mapping of numpy arrays, e.g.
    a memory-mapped checkpoint), one decoder layer at a time: host memory holds one
    layer's fused weights, not the model's."""
    local = getattr(hal, "local", None)

    def put(fused: dict) -> None:
        for name, w in fused.items():
            for r, off, arr in _name_shards(prog, name, w):
                if local is None or r in local:
                    hal.copy_to_dpu(r, off, arr)

    put(fused_globals(prog.cfg, sd))
    for l in range(prog.cfg.num_layers):
        put(fused_layer(prog.cfg, sd, prog.tp, l))
