"""LLaMA prefill + greedy decode on the B200 HAL vs the oracle HAL and HF (GPU).

Tolerances (north star): fp32 max-abs <= 1e-4 relative to the largest
magnitude; bf16 <= 2e-2 relative, with identical greedy token ids.
"""

from __future__ import annotations

import numpy as np
import pytest

from assert_node_matches_ref import NodeEnv, compare_all_nodes
from helpers import (PROJECTION_KERNELS, cuda_hal, oracle_hal, projection_kernel, tiny_golden, tiny_hf_model,
                     tiny_program, tiny_weights)

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-4
BF16_TOL = 2e-2


def _run(prog, hal, weights, prompt, steps):
    from runtime.executor import greedy_generate
    from runtime.program import load_weights

    load_weights(prog, hal, weights)
    return greedy_generate(prog.plans["prefill"], prog.plans["decode"], hal, prompt, steps)


@pytest.mark.parametrize("kernel", PROJECTION_KERNELS)
@pytest.mark.parametrize("tp", [1, 2, 4])
def test_tiny_llama_matches_hf(tp, kernel):
    model, gold = tiny_hf_model(), tiny_golden()
    prog = tiny_program(tp)
    hal = cuda_hal(prog)
    with projection_kernel(kernel):
        res = _run(prog, hal, tiny_weights(prog, model), gold["prompt"][None], 8)
    assert res.tokens[0].tolist() == gold["tokens"].tolist()
    for got, ref in zip([res.prefill_logits] + res.step_logits, gold["step_logits"]):
        got = got.reshape(-1)
        assert np.abs(got - ref).max() <= FP32_TOL * np.abs(ref).max()
    assert all(v == 0 for v in hal.read_error_flags().values())


@pytest.mark.parametrize("tp", [1, 4])
def test_tiny_node_by_node_vs_oracle(tp):
    """Every device node of the prefill and of one decode step equals the oracle's."""
    from runtime.executor import execute_plan
    from runtime.program import load_weights

    model, gold = tiny_hf_model(), tiny_golden()
    prog = tiny_program(tp)
    from graph.llama import ModelConfig
    from runtime.program import compile_llama

    prog = compile_llama(ModelConfig.tiny(max_seq=32), tp, batch=1, prompt_len=16, reuse=False)
    w = tiny_weights(prog, model)
    halc, halo = cuda_hal(prog), oracle_hal(prog)
    for hal in (halc, halo):
        load_weights(prog, hal, w)
        execute_plan(prog.plans["prefill"], hal, tokens=gold["prompt"][None], pos=np.zeros(1, np.int32))
    names = compare_all_nodes(prog.graphs["prefill"], NodeEnv(halc, prog.graphs["prefill"]),
                              NodeEnv(halo, prog.graphs["prefill"]), rtol=FP32_TOL, atol=0)
    assert len(names) > 10
    for hal in (halc, halo):
        execute_plan(prog.plans["decode"], hal, tokens=gold["tokens"][:1].reshape(1, 1), pos=np.full(1, 16, np.int32))
    compare_all_nodes(prog.graphs["decode"], NodeEnv(halc, prog.graphs["decode"]),
                      NodeEnv(halo, prog.graphs["decode"]), rtol=FP32_TOL, atol=0)


def _l7b_weights(cfg, seed=0):
    """Random-init 7B-architecture weights (bf16 N(0, 0.02), norm weights 1) as an HF-named state dict."""
    import ml_dtypes

    rng = np.random.default_rng(seed)
    bf = ml_dtypes.bfloat16
    h, i, v = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size

    def w(*shape):
        return (rng.standard_normal(shape, dtype=np.float32) * 0.02).astype(bf)

    sd = {"model.embed_tokens.weight": w(v, h), "lm_head.weight": w(v, h), "model.norm.weight": np.ones(h, bf)}
    for l in range(cfg.num_layers):
        p = f"model.layers.{l}."
        for n in ("q", "k", "v", "o"):
            sd[p + f"self_attn.{n}_proj.weight"] = w(h, h)
        sd[p + "mlp.gate_proj.weight"], sd[p + "mlp.up_proj.weight"] = w(i, h), w(i, h)
        sd[p + "mlp.down_proj.weight"] = w(h, i)
        sd[p + "input_layernorm.weight"] = np.ones(h, bf)
        sd[p + "post_attention_layernorm.weight"] = np.ones(h, bf)
    return sd


@pytest.fixture(scope="module")
def l7b_2layer():
    from graph.llama import ModelConfig

    cfg = ModelConfig.llama2_7b(max_seq=32, num_layers=2)
    return cfg, _l7b_weights(cfg), {}


@pytest.mark.parametrize("kernel", PROJECTION_KERNELS)
@pytest.mark.parametrize("tp", [1, 2])
def test_llama2_7b_arch_bf16_matches_oracle(l7b_2layer, tp, kernel):
    """7B-width bf16 (2 layers): logits within 2e-2 and identical greedy tokens, prefill + 3 steps."""
    from runtime.program import compile_llama, fused_weights

    cfg, sd, oracle_runs = l7b_2layer
    prog = compile_llama(cfg, tp, batch=1, prompt_len=16)
    w = fused_weights(cfg, sd, tp)
    prompt = np.random.default_rng(1).integers(0, cfg.vocab_size, (1, 16))
    with projection_kernel(kernel):
        rc = _run(prog, cuda_hal(prog), w, prompt, 4)
    if tp not in oracle_runs:
        oracle_runs[tp] = _run(prog, oracle_hal(prog), w, prompt, 4)
    ro = oracle_runs[tp]
    assert rc.tokens.tolist() == ro.tokens.tolist()
    for a, b in zip([rc.prefill_logits] + rc.step_logits, [ro.prefill_logits] + ro.step_logits):
        a, b = a.astype(np.float32), b.astype(np.float32)
        assert np.abs(a - b).max() <= BF16_TOL * np.abs(b).max()


@pytest.mark.parametrize("tp", [1, 2])
def test_llama2_7b_arch_bf16_long_prefill_matches_oracle(l7b_2layer, tp):
    """A 200-token prefill (tensor-core GEMMs with a partial last row tile) and 2 steps vs the oracle."""
    from graph.llama import ModelConfig
    from runtime.program import compile_llama, fused_weights

    _, sd, _ = l7b_2layer
    cfg = ModelConfig.llama2_7b(max_seq=256, num_layers=2)
    prog = compile_llama(cfg, tp, batch=1, prompt_len=200)
    w = fused_weights(cfg, sd, tp)
    prompt = np.random.default_rng(2).integers(0, cfg.vocab_size, (1, 200))
    rc = _run(prog, cuda_hal(prog), w, prompt, 2)
    ro = _run(prog, oracle_hal(prog), w, prompt, 2)
    assert rc.tokens.tolist() == ro.tokens.tolist()
    for a, b in zip([rc.prefill_logits] + rc.step_logits, [ro.prefill_logits] + ro.step_logits):
        a, b = a.astype(np.float32), b.astype(np.float32)
        assert np.abs(a - b).max() <= BF16_TOL * np.abs(b).max()


def test_captured_decode_graph_replays_equal_eager_steps():
    """A CUDA-graph replay of the decode plan produces exactly the eager plan's logits."""
    from runtime.executor import bind_inputs, execute_plan, read_logits, read_tokens
    from runtime.program import load_weights

    model, gold = tiny_hf_model(), tiny_golden()
    prog = tiny_program(2)
    w = tiny_weights(prog, model)
    eager, graphed = cuda_hal(prog), cuda_hal(prog)
    outs = {}
    for name, hal in (("eager", eager), ("graph", graphed)):
        load_weights(prog, hal, w)
        execute_plan(prog.plans["prefill"], hal, tokens=gold["prompt"][None], pos=np.zeros(1, np.int32))
        tok = read_tokens(prog.plans["prefill"], hal)
        dec = prog.plans["decode"]
        logits = []
        if name == "graph":
            bind_inputs(dec, hal, tokens=tok.reshape(1, 1), pos=np.full(1, 16, np.int32))
            cap = hal.capture(dec)  # the warm-up inside capture() runs step pos=16
            logits.append(read_logits(dec, hal))
            for pos in range(17, 20):
                # feed_next already moved the sampled token into the inputs on device
                bind_inputs(dec, hal, pos=np.full(1, pos, np.int32))
                cap.replay()
                logits.append(read_logits(dec, hal))
        else:
            for pos in range(16, 20):
                execute_plan(dec, hal, tokens=tok.reshape(1, 1), pos=np.full(1, pos, np.int32))
                logits.append(read_logits(dec, hal))
                tok = read_tokens(dec, hal)
        outs[name] = logits
    for a, b in zip(outs["eager"], outs["graph"]):
        assert np.array_equal(a, b)
