"""HF safetensors checkpoints: read lazily, converted like torch, streamed into the arenas (CPU).

The checkpoints are written by transformers' own ``save_pretrained`` from the tiny
LLaMA configuration (single file, sharded with an index, bf16, tied embeddings);
the weights read back must equal the model's state dict bit for bit, and the
oracle run on them must reproduce the HF golden tokens.
"""

from __future__ import annotations

import json

import numpy as np
import pytest

from helpers import oracle_hal, tiny_golden, tiny_hf_model, tiny_program


def _save(model, path, **kw):
    model.save_pretrained(str(path), safe_serialization=True, **kw)
    return path


def _assert_same(got, ref):
    assert got.dtype == ref.dtype and got.shape == ref.shape
    assert np.array_equal(got.view(np.uint8), np.ascontiguousarray(ref).view(np.uint8))


def test_single_file_fp32_reads_back_bit_exact(tmp_path):
    from runtime.checkpoint import Checkpoint

    model = tiny_hf_model()
    ck = Checkpoint(_save(model, tmp_path / "m"))
    sd = model.state_dict()
    assert set(ck) == {k for k in sd if k != "lm_head.weight" or not model.config.tie_word_embeddings}
    for k in ck:
        _assert_same(ck[k], sd[k].numpy())
        assert not ck[k].flags.writeable  # a view of the read-only map, no copy


def test_sharded_bf16_checkpoint_and_the_index(tmp_path):
    import torch

    from runtime.checkpoint import state_dict
    from runtime.program import hf_state_dict

    model = tiny_hf_model().to(torch.bfloat16)
    path = _save(model, tmp_path / "m", max_shard_size="300KB")
    index = json.loads((path / "model.safetensors.index.json").read_text())
    assert len(set(index["weight_map"].values())) > 1
    got, ref = state_dict(path, "bfloat16"), hf_state_dict(model, "bfloat16")
    assert set(got) == set(ref)
    for k in ref:
        _assert_same(got[k], ref[k])


def test_conversion_on_read_rounds_like_torch(tmp_path):
    from runtime.checkpoint import state_dict
    from runtime.program import hf_state_dict

    model = tiny_hf_model()
    got, ref = state_dict(_save(model, tmp_path / "m"), "bfloat16"), hf_state_dict(model, "bfloat16")
    for k in ref:
        _assert_same(got[k], ref[k])


def test_tied_embeddings_serve_lm_head(tmp_path):
    import torch
    from transformers import LlamaForCausalLM

    from runtime.checkpoint import state_dict

    base = tiny_hf_model()
    cfg = base.config
    cfg.tie_word_embeddings = True
    torch.manual_seed(1)
    model = LlamaForCausalLM(cfg).eval()
    sd = state_dict(_save(model, tmp_path / "m"), "float32")
    assert "lm_head.weight" in sd
    _assert_same(sd["lm_head.weight"], model.model.embed_tokens.weight.detach().numpy())


def test_model_config_from_config_json(tmp_path):
    from graph.llama import ModelConfig
    from runtime.checkpoint import model_config

    model = tiny_hf_model()
    path = _save(model, tmp_path / "m")
    assert model_config(path, 32) == ModelConfig.from_hf(model.config, 32, "float32")
    assert model_config(path, 32, "bfloat16").dtype == "bfloat16"
    cfg = json.loads((path / "config.json").read_text())
    for key, value in (("rope_scaling", {"rope_type": "linear", "factor": 2.0}), ("attention_bias", True),
                       ("head_dim", 32), ("model_type", "mistral")):
        bad = dict(cfg, **{key: value})
        (path / "config.json").write_text(json.dumps(bad))
        with pytest.raises(ValueError):
            model_config(path, 32)


def test_malformed_files_are_refused(tmp_path):
    from runtime.checkpoint import Checkpoint, SafetensorsFile

    model = tiny_hf_model()
    path = _save(model, tmp_path / "m")
    raw = (path / "model.safetensors").read_bytes()
    (tmp_path / "short.safetensors").write_bytes(raw[:4])
    (tmp_path / "trunc.safetensors").write_bytes(raw[:len(raw) // 2])
    for name in ("short.safetensors", "trunc.safetensors"):
        with pytest.raises(ValueError):
            SafetensorsFile(tmp_path / name)
    with pytest.raises(FileNotFoundError):
        Checkpoint(tmp_path / "nothing_here")


@pytest.mark.parametrize("tp", [1, 2])
def test_streamed_checkpoint_reproduces_the_hf_golden_on_the_oracle(tmp_path, tp):
    """load_state_dict (layer by layer from the memory map) == the in-memory load: HF's tokens."""
    from runtime.checkpoint import state_dict
    from runtime.executor import greedy_generate
    from runtime.program import load_state_dict

    gold = tiny_golden()
    prog = tiny_program(tp)
    hal = oracle_hal(prog)
    load_state_dict(prog, hal, state_dict(_save(tiny_hf_model(), tmp_path / "m"), prog.cfg.dtype))
    res = greedy_generate(prog.plans["prefill"], prog.plans["decode"], hal, gold["prompt"][None], 8)
    assert res.tokens[0].tolist() == gold["tokens"].tolist()
    logits = [res.prefill_logits.reshape(-1)] + [x.reshape(-1) for x in res.step_logits]
    for got, ref in zip(logits, gold["step_logits"]):
        np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-4 * np.abs(ref).max())
