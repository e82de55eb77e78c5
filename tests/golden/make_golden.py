"""Generate the golden fixtures that pin the oracle and the plan compiler.

Run in a container where the reference checkout is readable:

    python tests/golden/make_golden.py /root/reference

It imports the reference's own modules (comm/plan.py, comm/lowering.py,
backend/dpu_sdk.py, memory/kv_layout.py, graph/*) and records what they
produce on seeded inputs.  The fixtures are small JSON / NPZ files; the GPU box
never needs the reference checkout.  HuggingFace ``LlamaForCausalLM`` (the
model math the reference exports, tests/test_partition.py:128-167) supplies the
end-to-end logits and greedy tokens for the tiny configuration.
"""

from __future__ import annotations

import hashlib
import json
import sys
from math import prod
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).view(np.uint8).tobytes()).hexdigest()


def _seg_dict(s) -> dict:
    return {
        "src_dpu": s.src_dpu, "src_local_range": list(s.src_local_range),
        "global_range": list(s.global_range), "dst_dpu": s.dst_dpu,
        "dst_local_offset": s.dst_local_offset, "nbytes": s.nbytes, "reduce": s.reduce,
        "src_addr": s.src_addr, "dst_addr": s.dst_addr,
    }


def comm_inputs(kind: str, n: int, tokens: int, hidden: int = 4096, seed: int = 0):
    """Seeded bf16 inputs for the redistribute microbench (N(0,1) values).

    all_reduce: n partial tensors [tokens, hidden];  all_gather / all_to_all:
    one global tensor [tokens, hidden].  Shared with the tests (same recipe).
    """
    import ml_dtypes

    rng = np.random.default_rng(seed + 1000 * n + tokens)
    if kind == "all_reduce":
        return [rng.standard_normal((tokens, hidden), dtype=np.float32).astype(ml_dtypes.bfloat16)
                for _ in range(n)]
    return rng.standard_normal((tokens, hidden), dtype=np.float32).astype(ml_dtypes.bfloat16)


def make_comm(ref: Path) -> None:
    import ml_dtypes  # noqa: F401  (registers np.dtype("bfloat16") for comm/plan.py)
    from backend.dpu_sdk import dpu_alloc
    from comm.lowering import DmaEngine, all_gather, all_reduce, all_to_all, scatter
    from comm.plan import build_comm_plan, dma_sequence
    from contracts.pim_tensor_spec import Placement
    from tests.test_comm_plan import PARTIAL_SUM, REPLICATE, _dpu_spec, _edge, _host_spec

    cases = []
    arrays = {}
    for n in (2, 4, 8):
        for tokens in (16, 256):
            shape = (tokens, 4096)
            nbytes = prod(shape) * 2
            dpus = tuple(range(n))
            mram = 4 * nbytes
            # Partial(sum) -> Replicate@dpu  (all_reduce, writeback to every rank)
            src = _dpu_spec(PARTIAL_SUM, shape, dpus)
            dst = _dpu_spec(REPLICATE, shape, dpus, mram_offset=nbytes)
            (entry,) = build_comm_plan([_edge(0, "all_reduce", src, dst, shape, dtype="bfloat16", reduce_type="sum")])
            eng = DmaEngine(dpu_alloc(n, mram_bytes=mram))
            parts = comm_inputs("all_reduce", n, tokens)
            for d, p in enumerate(parts):
                eng.copy_to_dpu(d, 0, p.reshape(-1))
            out = all_reduce(entry, eng)
            wb = [eng.copy_from_dpu(d, nbytes, prod(shape), np.dtype("bfloat16")) for d in dpus]
            assert all(np.array_equal(w.view(np.uint16), out.reshape(-1).view(np.uint16)) for w in wb)
            key = f"all_reduce_n{n}_t{tokens}"
            cases.append({"key": key, "type": "all_reduce", "n": n, "tokens": tokens,
                          "inputs_sha": [_sha(p) for p in parts], "out_sha": _sha(out),
                          "n_segments": len(entry.segments),
                          "dma_kinds": [op.kind for op in dma_sequence(entry)]})
            if tokens == 16:
                arrays[key] = out.view(np.uint16)
            # Shard(1) -> Replicate@dpu  (all_gather)
            src = _dpu_spec(Placement("Shard", 1), shape, dpus)
            dst = _dpu_spec(REPLICATE, shape, dpus, mram_offset=nbytes)
            (entry,) = build_comm_plan([_edge(1, "all_gather", src, dst, shape, dtype="bfloat16")])
            eng = DmaEngine(dpu_alloc(n, mram_bytes=mram))
            g = comm_inputs("all_gather", n, tokens)
            w = 4096 // n
            for d in dpus:
                eng.copy_to_dpu(d, 0, np.ascontiguousarray(g[:, d * w:(d + 1) * w]).reshape(-1))
            out = all_gather(entry, eng)
            key = f"all_gather_n{n}_t{tokens}"
            cases.append({"key": key, "type": "all_gather", "n": n, "tokens": tokens,
                          "inputs_sha": [_sha(g)], "out_sha": _sha(out),
                          "n_segments": len(entry.segments),
                          "dma_kinds": [op.kind for op in dma_sequence(entry)],
                          "segments_head": [_seg_dict(s) for s in entry.segments[:4]]})
            # Shard(0) -> Shard(1)  (all_to_all)
            src = _dpu_spec(Placement("Shard", 0), shape, dpus)
            dst = _dpu_spec(Placement("Shard", 1), shape, dpus, mram_offset=nbytes)
            (entry,) = build_comm_plan([_edge(2, "all_to_all", src, dst, shape, dtype="bfloat16")])
            eng = DmaEngine(dpu_alloc(n, mram_bytes=mram))
            g = comm_inputs("all_to_all", n, tokens)
            r = tokens // n
            for d in dpus:
                eng.copy_to_dpu(d, 0, np.ascontiguousarray(g[d * r:(d + 1) * r, :]).reshape(-1))
            staging = all_to_all(entry, eng)
            locals_ = [eng.copy_from_dpu(d, nbytes, tokens * w, np.dtype("bfloat16")) for d in dpus]
            key = f"all_to_all_n{n}_t{tokens}"
            cases.append({"key": key, "type": "all_to_all", "n": n, "tokens": tokens,
                          "inputs_sha": [_sha(g)], "out_sha": _sha(staging),
                          "dst_local_sha": [_sha(x) for x in locals_],
                          "n_segments": len(entry.segments),
                          "segments_head": [_seg_dict(s) for s in entry.segments[:4]]})
    # Hand-built segment tables (Appendix-B style), including a permuted shard order,
    # a Shard(2) multi-row gather, a Replicate source and a scatter/broadcast.
    tables = []
    specs = [
        ("gather_permuted", "all_gather", (_dpu_spec(Placement("Shard", 0), (6,), (0, 1), permuted=True),
                                           _dpu_spec(REPLICATE, (6,), (0, 1))), (6,), "float32", None),
        ("gather_shard2_host", "all_gather", (_dpu_spec(Placement("Shard", 2), (1, 4, 8), (0, 1)), _host_spec()),
         (1, 4, 8), "float32", None),
        ("gather_replicate_src", "all_gather", (_dpu_spec(REPLICATE, (4, 4), (0, 1, 2, 3)), _host_spec()),
         (4, 4), "float32", None),
        ("reduce_mean_host", "all_reduce", (_dpu_spec(Placement("Partial", reduce_type="mean"), (4,), (0, 1)),
                                            _host_spec()), (4,), "float32", "mean"),
        ("a2a_4x6", "all_to_all", (_dpu_spec(Placement("Shard", 0), (4, 6), (0, 1)),
                                   _dpu_spec(Placement("Shard", 1), (4, 6), (0, 1), mram_offset=128)),
         (4, 6), "float32", None),
        ("scatter_shard0", "scatter", (_host_spec(), _dpu_spec(Placement("Shard", 0), (4, 6), (0, 1), mram_offset=32)),
         (4, 6), "float32", None),
        ("scatter_bcast", "scatter", (_host_spec(), _dpu_spec(REPLICATE, (4,), (0, 1, 2))), (4,), "float32", None),
        ("reduce_bf16_8", "all_reduce", (_dpu_spec(PARTIAL_SUM, (2, 8), tuple(range(8))),
                                         _dpu_spec(REPLICATE, (2, 8), tuple(range(8)), mram_offset=64)),
         (2, 8), "bfloat16", "sum"),
    ]
    for name, typ, (s, d), shape, dtype, red in specs:
        (entry,) = build_comm_plan([_edge(7, typ, s, d, shape, dtype=dtype, reduce_type=red)])
        tables.append({"name": name, "type": typ, "shape": list(shape), "dtype": dtype, "reduce": red,
                       "segments": [_seg_dict(x) for x in entry.segments],
                       "dma": [[op.kind, [entry.segments.index(x) for x in op.segments]]
                               for op in dma_sequence(entry)]})
    # Small numeric cases kept in full (fp32, exact) for the lowering restatement.
    rng = np.random.default_rng(7)
    small = {}
    shape = (8,)
    src = _dpu_spec(PARTIAL_SUM, shape, (0, 1, 2))
    (entry,) = build_comm_plan([_edge(0, "all_reduce", src, _host_spec(), shape, reduce_type="sum")])
    eng = DmaEngine(dpu_alloc(3, mram_bytes=256))
    parts = [rng.standard_normal(8).astype(np.float32) for _ in range(3)]
    for d, p in enumerate(parts):
        eng.copy_to_dpu(d, 0, p)
    small["reduce3_in"] = np.stack(parts)
    small["reduce3_out"] = all_reduce(entry, eng)
    h = rng.standard_normal((4, 6)).astype(np.float32)
    dst = _dpu_spec(Placement("Shard", 1), (4, 6), (0, 1), mram_offset=32)
    (entry,) = build_comm_plan([_edge(0, "scatter", _host_spec(), dst, (4, 6))])
    eng = DmaEngine(dpu_alloc(2, mram_bytes=256))
    scatter(entry, eng, h)
    small["scatter_in"] = h
    small["scatter_d0"] = eng.copy_from_dpu(0, 32, 12, np.dtype(np.float32))
    small["scatter_d1"] = eng.copy_from_dpu(1, 32, 12, np.dtype(np.float32))

    (HERE / "comm_golden.json").write_text(json.dumps({"cases": cases, "tables": tables}, indent=1))
    np.savez_compressed(HERE / "comm_golden.npz", **arrays, **small)


def make_kv(ref: Path) -> None:
    from contracts.pim_tensor_spec import Placement
    from memory.kv_layout import build_kv_layout, kv_access, kv_specs_from_placement
    from tests.test_comm_plan import _dpu_spec

    out = []
    for name, layers, heads, hd, tp, max_seq, dbytes, base, align in (
        ("tiny_tp4", 2, 4, 64, 4, 24, 4, 4096, 64),
        ("l7b_tp8_bf16", 32, 32, 128, 8, 256, 2, 1 << 20, 256),
        ("l7b_tp1_bf16", 32, 32, 128, 1, 256, 2, 0, 256),
    ):
        kspec = _dpu_spec(Placement("Shard", 0), (heads * hd, heads * hd), tuple(range(tp)))
        specs = kv_specs_from_placement(kspec, num_layers=layers, num_kv_heads=heads, num_q_heads=heads,
                                        head_dim=hd, max_seq=max_seq, dtype_bytes=dbytes, kv_base=base)
        for d, s in specs.items():
            build_kv_layout(s, align)
        rank = max(specs)
        s = specs[rank]
        acc = kv_access(s, layers - 1, s.kv_heads[-1], "v", 3, max_seq)
        out.append({"name": name, "tp": tp, "rank": rank, "kv_heads": s.kv_heads,
                    "kv_allocated_bytes": s.kv_allocated_bytes,
                    "kv_off": [[l, h, w, o] for (l, h, w), o in sorted(s.kv_off.items())][:12],
                    "kv_off_last": [[l, h, w, o] for (l, h, w), o in sorted(s.kv_off.items())][-2:],
                    "access": [acc.loc[1], acc.offset, acc.length]})
    (HERE / "kv_golden.json").write_text(json.dumps(out, indent=1))


def make_tiny_model() -> None:
    """HF LlamaForCausalLM on CPU for the tiny configuration: 16-token prompt, 8 greedy steps."""
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=1024, hidden_size=256, intermediate_size=688, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=4, rms_norm_eps=1e-6, rope_theta=10000.0,
                      max_position_embeddings=64, bos_token_id=1, eos_token_id=2, pad_token_id=0,
                      initializer_range=0.02)
    model = LlamaForCausalLM(cfg).eval()
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    rng = np.random.default_rng(0)
    prompt = rng.integers(0, 1024, size=16).astype(np.int64)
    ids = torch.tensor(prompt).unsqueeze(0)
    toks, steps_logits = [], []
    with torch.no_grad():
        for _ in range(9):  # prefill + 8 decode steps, full recompute (no cache)
            logits = model(input_ids=ids, use_cache=False).logits[0, -1].float()
            steps_logits.append(logits.numpy().copy())
            nxt = int(torch.argmax(logits))
            toks.append(nxt)
            ids = torch.cat([ids, torch.tensor([[nxt]])], dim=1)
    np.savez_compressed(HERE / "tiny_llama_golden.npz", prompt=prompt, tokens=np.array(toks[:8]),
                        step_logits=np.stack(steps_logits[:8]),
                        weights_sha=np.array([hashlib.sha256(b"".join(sd[k].numpy().tobytes()
                                                                      for k in sorted(sd))).hexdigest()]))


def make_spec_prop(ref: Path) -> None:
    """Edge list that the reference's graph passes produce for the tiny exported graph (TP=4)."""
    import ml_dtypes  # noqa: F401
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM
    from graph.partition import partition_graph
    from graph.spec_prop import llama_shard_config, propagate_specs
    from comm.plan import build_comm_plan
    from tests.test_partition import _FixedMaskLlama

    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=1024, hidden_size=256, intermediate_size=688, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=4, rms_norm_eps=1e-6, rope_theta=10000.0,
                      max_position_embeddings=64, bos_token_id=1, eos_token_id=2, pad_token_id=0)
    model = LlamaForCausalLM(cfg).eval()
    S = 16
    ids = torch.arange(S).unsqueeze(0)
    blocked = torch.triu(torch.ones(S, S, dtype=torch.bool), diagonal=1)
    mask = torch.zeros((1, 1, S, S)).masked_fill_(blocked, torch.finfo(torch.float32).min)
    gm = torch.export.export(_FixedMaskLlama(model), (ids, mask), strict=True).module()
    partition_graph(gm)
    edges = propagate_specs(gm, llama_shard_config(4, num_heads=4, num_kv_heads=4,
                                                   intermediate_size=688, vocab_size=1024))
    entries = build_comm_plan(edges)
    rows = []
    for e, ent in zip(edges, entries):
        rows.append({"edge_id": e.edge_id, "type": e.type, "src": e.src, "dst": e.dst,
                     "from": [e.from_placement.kind, e.from_placement.dim, e.from_placement.reduce_type],
                     "to": [e.to_placement.kind, e.to_placement.dim, e.to_placement.reduce_type],
                     "shape": list(e.shape), "dtype": e.dtype, "nbytes": e.nbytes,
                     "n_segments": len(ent.segments)})
    (HERE / "spec_prop_tiny_golden.json").write_text(json.dumps(rows, indent=1))


# Small static-KV-cache case: 2 layers, 2 ranks with kv heads (0, 1) / (2, 3), head_dim 8,
# max_seq 16, fp32, 64-byte block alignment, tiles of 6 positions (16 is not a multiple).
KVC_LAYERS, KVC_HD, KVC_MAX, KVC_TILE = 2, 8, 16, 6


def kv_cache_steps(seed: int = 5):
    """Seeded K/V rows written by the cache test: [(layer, pos, {rank: {head: (k, v)}})]."""
    rng = np.random.default_rng(seed)
    steps = []
    for layer in range(KVC_LAYERS):
        for pos in range(7):
            by = {}
            for rank, heads in ((0, (0, 1)), (1, (2, 3))):
                by[rank] = {h: (rng.standard_normal(KVC_HD).astype(np.float32),
                                rng.standard_normal(KVC_HD).astype(np.float32)) for h in heads}
            steps.append((layer, pos, by))
    return steps


def kv_cache_attention(cache, read_tile, layer, q_by_head, valid_len, decode_mask):
    """Decode attention over tiles read back from the cache (scores per tile, softmax with
    the decode mask, weights @ V per tile), the restated form of the reference's test."""
    mask = decode_mask(valid_len, KVC_MAX)
    out = {}
    for rank, heads in ((0, (0, 1)), (1, (2, 3))):
        for h in heads:
            scores = np.concatenate([read_tile(layer, rank, h, s, min(s + KVC_TILE, KVC_MAX))[0] @ q_by_head[h]
                                     / np.sqrt(KVC_HD) for s in range(0, KVC_MAX, KVC_TILE)])
            x = scores + mask
            e = np.exp(x - x.max())
            wts = e / e.sum()
            acc = np.zeros(KVC_HD, np.float32)
            for s in range(0, KVC_MAX, KVC_TILE):
                v = read_tile(layer, rank, h, s, min(s + KVC_TILE, KVC_MAX))[1]
                acc += wts[s:s + v.shape[0]] @ v
            out[h] = acc
    return out


def make_kv_cache(ref: Path) -> None:
    """The reference's PIMStaticKVCache on its NumpyBackend: arena bytes, tiles, masks, attention."""
    from backend.hal_numpy import NumpyBackend, NumpyBackendConfig
    from memory.kv_layout import KVRegionSpec, PIMStaticKVCache, build_kv_layout, decode_mask, prefill_mask

    def spec(rank, heads):
        return build_kv_layout(KVRegionSpec(dpu_id=rank, layers=list(range(KVC_LAYERS)), kv_heads=list(heads),
                                            q_heads_by_kv={h: [h] for h in heads}, max_seq=KVC_MAX,
                                            head_dim=KVC_HD, dtype_bytes=4, kv_base=0), align=64)

    specs = {0: spec(0, (0, 1)), 1: spec(1, (2, 3))}
    hal = NumpyBackend(NumpyBackendConfig(num_dpus=2, mram_bytes_per_dpu=1 << 16))
    cache = PIMStaticKVCache(hal, specs, wram_budget_bytes=KVC_TILE * KVC_HD * 4)
    for layer, pos, by in kv_cache_steps():
        cache.update(layer, pos, {r: {h: kv[0] for h, kv in d.items()} for r, d in by.items()},
                     {r: {h: kv[1] for h, kv in d.items()} for r, d in by.items()})
    arena_bytes = max(s.kv_allocated_bytes for s in specs.values())
    tiles = {}
    for layer in range(KVC_LAYERS):
        for rank, heads in ((0, (0, 1)), (1, (2, 3))):
            for h in heads:
                for s0 in range(0, KVC_MAX, KVC_TILE):
                    k, v = cache.read_tile(layer, rank, h, s0, min(s0 + KVC_TILE, KVC_MAX))
                    tiles[f"{layer}/{rank}/{h}/{s0}"] = [_sha(k), _sha(v)]
    rng = np.random.default_rng(6)
    q = {h: rng.standard_normal(KVC_HD).astype(np.float32) for h in range(4)}
    attn = kv_cache_attention(cache, cache.read_tile, 1, q, 6, decode_mask)
    out = {"kv_off": {str(r): [[l, h, w, o] for (l, h, w), o in sorted(s.kv_off.items())] for r, s in specs.items()},
           "kv_allocated_bytes": arena_bytes,
           "arena_sha": [_sha(hal.read_local(r, 0, (arena_bytes,), np.uint8)) for r in (0, 1)],
           "tiles": tiles,
           "prefill_mask_sha": {f"{p}/{m}": _sha(prefill_mask(p, m)) for p, m in ((5, 16), (16, 16), (1, 24))},
           "decode_mask_sha": {f"{v}/{m}": _sha(decode_mask(v, m)) for v, m in ((6, 16), (0, 16), (23, 24))},
           "attention_q_seed": 6, "attention_valid_len": 6,
           "attention": {str(h): attn[h].tolist() for h in sorted(attn)}}
    (HERE / "kv_cache_golden.json").write_text(json.dumps(out, indent=1))


def main() -> None:
    ref = Path(sys.argv[1] if len(sys.argv) > 1 else "/root/reference").resolve()
    sys.path.insert(0, str(ref))
    only = sys.argv[2:]  # e.g. "kv_cache": regenerate just that fixture
    makers = {"comm": lambda: make_comm(ref), "kv": lambda: make_kv(ref), "spec_prop": lambda: make_spec_prop(ref),
              "tiny_model": make_tiny_model, "kv_cache": lambda: make_kv_cache(ref)}
    for name, fn in makers.items():
        if not only or name in only:
            fn()
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
