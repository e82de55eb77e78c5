"""Fixture: the tiny LLaMA compiled by the reference's own passes, for the aten-level tests.

    python tests/golden/make_ref_chain.py [path-to-reference]   (default /root/reference)

Runs the reference's compile chain exactly as its tests do (tests/test_partition.py:148-168):
HF ``LlamaForCausalLM`` of the tiny configuration (the model ``helpers.tiny_hf_model``
builds: vocab 1024, hidden 256, 4 x 64 MHA, MLP 688, 2 layers, fp32, seed 0) wrapped to
take ``(input_ids, causal_mask)``, ``torch.export.export(strict=True).module()``, then
``graph.partition.partition_graph`` and ``graph.spec_prop.propagate_specs`` with
``llama_shard_config(4, ...)`` -- TP=4.  The annotated graph is written with
``graph.fx_import.encode_fx`` to ``ref_chain_tiny_tp4.json`` next to this script.  The
B200 tests read only that file; the reference itself is needed only to regenerate it.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
SEQ, TP = 16, 4


def build(ref_root: str = "/root/reference") -> dict:
    import torch

    sys.path.insert(0, str(ROOT / "flagos-pim-compiler_b200"))
    sys.path.insert(0, str(ROOT / "tests"))
    from graph.fx_import import encode_fx
    from helpers import tiny_hf_model

    sys.path.insert(0, ref_root)
    # the reference's own modules (its graph/ and contracts/ packages, not this repo's)
    import importlib

    for mod in [m for m in list(sys.modules) if m == "graph" or m.startswith(("graph.", "contracts."))
                or m == "contracts"]:
        if "fx_import" not in mod:
            sys.modules.pop(mod)
    saved = sys.path[:]
    sys.path[:] = [ref_root] + [p for p in sys.path if "flagos-pim-compiler_b200" not in p]
    partition = importlib.import_module("graph.partition")
    spec_prop = importlib.import_module("graph.spec_prop")
    sys.path[:] = saved

    class FixedMaskLlama(torch.nn.Module):
        def __init__(self, model):
            super().__init__()
            self.model = model

        def forward(self, input_ids, causal_mask):
            return self.model(input_ids=input_ids, attention_mask=causal_mask, use_cache=False,
                              return_dict=True).logits

    model = tiny_hf_model()
    ids = torch.arange(SEQ, dtype=torch.long).unsqueeze(0)
    blocked = torch.triu(torch.ones(SEQ, SEQ, dtype=torch.bool), diagonal=1)
    mask = torch.zeros((1, 1, SEQ, SEQ), dtype=torch.float32)
    mask.masked_fill_(blocked, torch.finfo(mask.dtype).min)
    gm = torch.export.export(FixedMaskLlama(model), (ids, mask), strict=True).module()
    partition.partition_graph(gm)
    edges = spec_prop.propagate_specs(gm, spec_prop.llama_shard_config(
        TP, num_heads=4, num_kv_heads=4, intermediate_size=688, vocab_size=1024))
    d = encode_fx(gm)
    d["meta"] = {"model": "tiny LLaMA (helpers.tiny_hf_model)", "tp": TP, "seq": SEQ,
                 "inputs": ["input_ids int64 [1, 16]", "causal_mask float32 [1, 1, 16, 16] (0 / finfo.min)"],
                 "edges": len(edges), "edge_types": sorted({e.type for e in edges}),
                 "torch": torch.__version__}
    return d


if __name__ == "__main__":
    d = build(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
    out = HERE / "ref_chain_tiny_tp4.json"
    out.write_text(json.dumps(d, separators=(",", ":")))
    print(f"wrote {out} ({out.stat().st_size} bytes, {len(d['nodes'])} nodes, {d['meta']['edges']} edges)")
