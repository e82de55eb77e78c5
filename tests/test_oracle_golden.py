"""Pins the oracle and the plan compiler to vectors produced by the reference itself.

Fixtures come from tests/golden/make_golden.py, which ran the reference's
comm/plan.py, comm/lowering.py, memory/kv_layout.py and graph passes, and HF
LlamaForCausalLM, on seeded inputs.
"""

from __future__ import annotations

import json
from math import prod

import numpy as np
import pytest

from helpers import GOLDEN, comm_inputs, oracle_hal, redistribute_entry, sha, tiny_golden, tiny_hf_model, \
    tiny_program, tiny_weights, weights_sha

COMM = json.loads((GOLDEN / "comm_golden.json").read_text())


def _engine(n, nbytes):
    from oracle.hal_numpy import NumpyBackend, NumpyBackendConfig
    from oracle.lowering import DmaEngine

    return DmaEngine(NumpyBackend(NumpyBackendConfig(n, 4 * nbytes)))


@pytest.mark.parametrize("case", COMM["cases"], ids=[c["key"] for c in COMM["cases"]])
def test_oracle_lowering_bit_exact_vs_reference(case):
    """Package comm plan + oracle host-star lowering reproduce the reference outputs bit for bit."""
    from oracle import lowering

    n, t, kind = case["n"], case["tokens"], case["type"]
    shape = (t, 4096)
    entry, nbytes = redistribute_entry(kind, n, shape)
    assert len(entry.segments) == case["n_segments"]
    eng = _engine(n, nbytes)
    if kind == "all_reduce":
        parts = comm_inputs(kind, n, t)
        assert [sha(p) for p in parts] == case["inputs_sha"]
        for d, p in enumerate(parts):
            eng.copy_to_dpu(d, 0, p.reshape(-1))
        out = lowering.all_reduce(entry, eng)
        for d in range(n):
            assert sha(eng.hal.read_local(d, nbytes, (prod(shape),), entry.dtype)) == case["out_sha"]
    elif kind == "all_gather":
        g = comm_inputs(kind, n, t)
        assert sha(g) == case["inputs_sha"][0]
        w = 4096 // n
        for d in range(n):
            eng.copy_to_dpu(d, 0, np.ascontiguousarray(g[:, d * w:(d + 1) * w]).reshape(-1))
        out = lowering.all_gather(entry, eng)
        assert np.array_equal(out.view(np.uint16), g.view(np.uint16))
    else:
        g = comm_inputs(kind, n, t)
        r = t // n
        for d in range(n):
            eng.copy_to_dpu(d, 0, np.ascontiguousarray(g[d * r:(d + 1) * r, :]).reshape(-1))
        out = lowering.all_to_all(entry, eng)
        w = 4096 // n
        for d in range(n):
            assert sha(eng.hal.read_local(d, nbytes, (t * w,), entry.dtype)) == case["dst_local_sha"][d]
    assert sha(out) == case["out_sha"]


def test_bf16_all_reduce_is_sequential_rne_not_fp32_accumulate():
    """The reference's bf16 sum rounds after every partial; an fp32 accumulate differs."""
    import ml_dtypes

    from oracle import lowering

    entry, nbytes = redistribute_entry("all_reduce", 8, (16, 4096))
    parts = comm_inputs("all_reduce", 8, 16)
    eng = _engine(8, nbytes)
    for d, p in enumerate(parts):
        eng.copy_to_dpu(d, 0, p.reshape(-1))
    out = lowering.all_reduce(entry, eng)
    gold = np.load(GOLDEN / "comm_golden.npz")["all_reduce_n8_t16"]
    assert np.array_equal(out.view(np.uint16), gold)
    f32 = sum(p.astype(np.float32) for p in parts).astype(ml_dtypes.bfloat16)
    assert not np.array_equal(f32.view(np.uint16), gold)


def _ref_style_spec(kind, shape, dpus, dim=None, permuted=False, mram_offset=0, reduce=None):
    """Hand-built specs with the semantics of the reference test helper (chunk order reversible)."""
    from contracts.pim_tensor_spec import PIMTensorSpec, Placement, TensorShardDetail

    if kind == "host":
        return PIMTensorSpec("host", Placement("Replicate"), "transient", None, {}, None)
    pl = Placement(kind, dim, reduce)
    if kind == "Shard":
        w = shape[dim] // len(dpus)
        smap = {}
        for i, d in enumerate(dpus):
            c = len(dpus) - 1 - i if permuted else i
            smap[d] = TensorShardDetail(d, dim, c * w, (c + 1) * w, shape[:dim] + (w,) + shape[dim + 1:], mram_offset)
    else:
        smap = {d: TensorShardDetail(d, -1, 0, prod(shape), shape, mram_offset) for d in dpus}
    return PIMTensorSpec("dpu", pl, "transient", None, smap, reduce)


TABLE_SPECS = {
    "gather_permuted": ("all_gather", ("Shard", (6,), (0, 1), 0, True, 0), ("Replicate", (6,), (0, 1), None, False, 0)),
    "gather_shard2_host": ("all_gather", ("Shard", (1, 4, 8), (0, 1), 2, False, 0), ("host",)),
    "gather_replicate_src": ("all_gather", ("Replicate", (4, 4), (0, 1, 2, 3), None, False, 0), ("host",)),
    "reduce_mean_host": ("all_reduce", ("Partial", (4,), (0, 1), None, False, 0, "mean"), ("host",)),
    "a2a_4x6": ("all_to_all", ("Shard", (4, 6), (0, 1), 0, False, 0), ("Shard", (4, 6), (0, 1), 1, False, 128)),
    "scatter_shard0": ("scatter", ("host",), ("Shard", (4, 6), (0, 1), 0, False, 32)),
    "scatter_bcast": ("scatter", ("host",), ("Replicate", (4,), (0, 1, 2), None, False, 0)),
    "reduce_bf16_8": ("all_reduce", ("Partial", (2, 8), tuple(range(8)), None, False, 0, "sum"),
                      ("Replicate", (2, 8), tuple(range(8)), None, False, 64)),
}


def _spec_from(t):
    if t[0] == "host":
        return _ref_style_spec("host", None, None)
    return _ref_style_spec(t[0], t[1], t[2], t[3], t[4], t[5], t[6] if len(t) > 6 else None)


@pytest.mark.parametrize("table", COMM["tables"], ids=[t["name"] for t in COMM["tables"]])
def test_comm_plan_segments_match_reference(table):
    from comm.plan import build_comm_plan, dma_sequence
    from contracts.pim_tensor_spec import RedistributeEdge

    typ, s, d = TABLE_SPECS[table["name"]]
    src, dst = _spec_from(s), _spec_from(d)
    shape = tuple(table["shape"])
    itemsize = 2 if table["dtype"] == "bfloat16" else 4
    loc = lambda sp: {"device": "host"} if sp.device == "host" else {"device": "dpu", "dpus": sorted(sp.shard_map)}
    e = RedistributeEdge(7, "producer", "consumer", src.placement, dst.placement, src, dst, typ, loc(src), loc(dst),
                         prod(shape) * itemsize, table["reduce"], shape, table["dtype"])
    (entry,) = build_comm_plan([e])
    got = [{"src_dpu": x.src_dpu, "src_local_range": list(x.src_local_range), "global_range": list(x.global_range),
            "dst_dpu": x.dst_dpu, "dst_local_offset": x.dst_local_offset, "nbytes": x.nbytes, "reduce": x.reduce,
            "src_addr": x.src_addr, "dst_addr": x.dst_addr} for x in entry.segments]
    assert got == table["segments"]
    ops = [[op.kind, [entry.segments.index(x) for x in op.segments]] for op in dma_sequence(entry)]
    assert ops == table["dma"]


def test_small_fp32_lowering_numerics_match_reference():
    from oracle import lowering

    g = np.load(GOLDEN / "comm_golden.npz")
    entry, nb = redistribute_entry("all_reduce", 3, (8,), dtype="float32")
    eng = _engine(3, 256)
    for d in range(3):
        eng.copy_to_dpu(d, 0, g["reduce3_in"][d])
    assert np.array_equal(lowering.all_reduce(entry, eng).reshape(-1), g["reduce3_out"])


@pytest.mark.parametrize("row", json.loads((GOLDEN / "kv_golden.json").read_text()), ids=lambda r: r["name"])
def test_kv_layout_matches_reference(row):
    from contracts.pim_tensor_spec import Placement
    from graph.llama import dpu_spec
    from memory.kv_layout import build_kv_layout, kv_access, kv_specs_from_placement

    cfg = {"tiny_tp4": (2, 4, 64, 4, 24, 4, 4096, 64), "l7b_tp8_bf16": (32, 32, 128, 8, 256, 2, 1 << 20, 256),
           "l7b_tp1_bf16": (32, 32, 128, 1, 256, 2, 0, 256)}[row["name"]]
    layers, heads, hd, tp, max_seq, db, base, align = cfg
    kspec = dpu_spec(Placement("Shard", 0), (heads * hd, heads * hd), tuple(range(tp)))
    specs = kv_specs_from_placement(kspec, num_layers=layers, num_kv_heads=heads, num_q_heads=heads, head_dim=hd,
                                    max_seq=max_seq, dtype_bytes=db, kv_base=base)
    s = build_kv_layout(specs[row["rank"]], align)
    assert s.kv_heads == row["kv_heads"]
    assert s.kv_allocated_bytes == row["kv_allocated_bytes"]
    offs = [[l, h, w, o] for (l, h, w), o in sorted(s.kv_off.items())]
    assert offs[:12] == row["kv_off"] and offs[-2:] == row["kv_off_last"]
    acc = kv_access(s, layers - 1, s.kv_heads[-1], "v", 3, max_seq)
    assert [acc.loc[1], acc.offset, acc.length] == row["access"]


def test_partial_to_replicate_exchanges_match_reference_graph():
    """The reference's graph passes find 4 all_reduce edges on the tiny TP=4 graph; so does ours."""
    rows = json.loads((GOLDEN / "spec_prop_tiny_golden.json").read_text())
    ref = sum(r["type"] == "all_reduce" for r in rows)
    prog = tiny_program(4)
    ours = sum(e.type == "all_reduce" for e in prog.entries["prefill"])
    assert ref == ours == 4


@pytest.mark.parametrize("tp", [1, 2, 4])
def test_tiny_llama_oracle_matches_hf(tp):
    """Config 1: prefill + 8 greedy steps on the oracle HAL == HF single-card logits and tokens."""
    from runtime.executor import greedy_generate
    from runtime.program import load_weights

    model = tiny_hf_model()
    gold = tiny_golden()
    assert weights_sha(model) == str(gold["weights_sha"][0])
    prog = tiny_program(tp)
    hal = oracle_hal(prog)
    load_weights(prog, hal, tiny_weights(prog, model))
    res = greedy_generate(prog.plans["prefill"], prog.plans["decode"], hal, gold["prompt"][None], 8)
    assert res.tokens[0].tolist() == gold["tokens"].tolist()
    logits = [res.prefill_logits.reshape(-1)] + [x.reshape(-1) for x in res.step_logits]
    for got, ref in zip(logits, gold["step_logits"]):
        np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-4 * np.abs(ref).max())


@pytest.mark.parametrize("tp", [1, 2])
def test_tiny_gqa_llama_oracle_matches_hf(tp):
    """Grouped-query attention (8 query heads on 2 kv heads, split over TP ranks): HF's tokens and logits."""
    from graph.llama import ModelConfig
    from helpers import hf_greedy, tiny_gqa_hf_model
    from runtime.executor import greedy_generate
    from runtime.program import compile_llama, fused_weights, hf_state_dict, load_weights

    model = tiny_gqa_hf_model()
    prompt = np.random.default_rng(0).integers(0, 1024, (1, 16))
    toks, logits = hf_greedy(model, prompt, 5)
    cfg = ModelConfig.from_hf(model.config, 32, "float32")
    prog = compile_llama(cfg, tp, batch=1, prompt_len=16)
    hal = oracle_hal(prog)
    load_weights(prog, hal, fused_weights(cfg, hf_state_dict(model, "float32"), tp))
    res = greedy_generate(prog.plans["prefill"], prog.plans["decode"], hal, prompt, 5)
    assert res.tokens[0].tolist() == toks[:len(res.tokens[0])]
    for got, ref in zip([res.prefill_logits] + res.step_logits, logits):
        ref = ref.reshape(-1)
        np.testing.assert_allclose(got.reshape(-1), ref, rtol=1e-4, atol=1e-4 * np.abs(ref).max())
    hal.close()


@pytest.mark.parametrize("tp", [1, 2])
def test_tiny_llama_batch_of_three_oracle_matches_hf(tp):
    """Three sequences decoded together (rows = batch; KV regions per sequence) == HF one by one."""
    from helpers import hf_greedy, tiny_program, tiny_weights
    from runtime.executor import greedy_generate
    from runtime.program import load_weights

    model = tiny_hf_model()
    prompts = np.random.default_rng(7).integers(0, 1024, (3, 8))
    prog = tiny_program(tp, batch=3, prompt_len=8)
    hal = oracle_hal(prog)
    load_weights(prog, hal, tiny_weights(prog, model))
    res = greedy_generate(prog.plans["prefill"], prog.plans["decode"], hal, prompts, 4)
    steps = [np.asarray(res.prefill_logits).reshape(3, -1)] + [np.asarray(x).reshape(3, -1) for x in res.step_logits]
    for b in range(3):
        toks, logits = hf_greedy(model, prompts[b:b + 1], 4)
        assert res.tokens[b].tolist() == toks[:len(res.tokens[b])]
        for got, ref in zip(steps, logits):
            np.testing.assert_allclose(got[b], ref, rtol=1e-4, atol=1e-4 * np.abs(ref).max())
    hal.close()
