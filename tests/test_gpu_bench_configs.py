"""Parity at the benchmarked workloads themselves (GPU), B200 HAL vs the oracle HAL.

The weights (and for batched decode the pre-filled KV blocks) are generated on the
device by the same calls ``bench.py`` uses (``LlamaRunner.load_random_weights``,
``pim_fill_normal``) and the oracle receives exactly those arena bytes, so both sides
start from identical state:

* LLaMA2-7B architecture decode, all 32 layers, TP=1: a 128-token uniform-random prompt
  and 4 greedy decode steps at max_seq 256 -- the shape ``bench.py`` times.  Node by node
  (every command of the prefill and of 4 decode steps run on both HALs from identical
  inputs, ``lockstep_compare``) within 2e-2, and the free-running greedy tokens identical;
* prefill of 8 x 2048 uniform-random ids (2 layers, TP=1 and TP=2): the last-position
  logits of every sequence and the whole KV zone (every layer, head and position);
* batched decode of 64 sequences whose KV blocks hold N(0, 1) values, decoding at
  positions 4096 and 4097 (2 layers, TP=1): node by node at the first step, then a
  free-running step.

Tolerances (docs/spec.md:1649-1656 and the north-star bar): bf16 values within 2e-2 of
the largest reference magnitude, identical greedy token ids.  A greedy id may differ
only where the reference's two candidates are equal at that tolerance (a tie at the
comparison's resolution: with random N(0, 0.02) weights the top logits of 32000 are
often closer than bf16 rounding), and the test counts such ties.  End to end through
32 layers the free-running bf16 logits of the two HALs drift apart by several percent
(rounding differences compound layer by layer); the per-node comparison is the bound.
"""

from __future__ import annotations

import numpy as np
import pytest

from assert_node_matches_ref import argmax_within_tolerance, lockstep_compare
from helpers import max_rel_err, mirror_arena, mirror_zone

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2


def _pair(prog, seed, **kw):
    """A B200 HAL with device-initialised random weights and an oracle HAL holding the same bytes."""
    from oracle.hal_numpy import NumpyBackend, NumpyBackendConfig
    from backend.hal_cuda import CudaBackend, CudaBackendConfig
    from runtime.session import LlamaRunner

    hal = CudaBackend(CudaBackendConfig(prog.tp, prog.arena_bytes, **kw))
    runner = LlamaRunner(prog, hal)
    runner.load_random_weights(seed=seed)
    ora = NumpyBackend(NumpyBackendConfig(prog.tp, prog.arena_bytes))
    for p in prog.plans.values():
        ora.register_plan(p)
    mirror_zone(prog, hal, ora, "weight")
    return hal, ora


def _kv_layers(prog, hal, rank):
    """The rank's KV zone as [layers, sequences * rest] fp32.  The zone holds one region set
    per sequence (seq_stride apart), each in build_kv_layout's order (layer, kv head, k|v)."""
    import ml_dtypes

    spec = prog.kv_specs[rank]
    dp = prog.dpu_plans[rank]
    n = spec.kv_allocated_bytes // 2
    kv = hal.copy_from_dpu(rank, dp.kv_base, (n,), ml_dtypes.bfloat16).astype(np.float32)
    kv = kv.reshape(spec.num_seqs, prog.cfg.num_layers, -1)
    return kv.transpose(1, 0, 2).reshape(prog.cfg.num_layers, -1)


def _assert_nodes(results, what):
    assert results, what
    bad = [(n, k, v) for n, k, v in results if (k == "rel" and v > BF16_TOL) or (k == "mismatches" and v)]
    assert not bad, (what, bad[:10])


def test_llama2_7b_arch_32_layers_prompt_128_decode_matches_oracle():
    """The decode benchmark's model and prompt: every node within 2e-2, greedy tokens identical."""
    from graph.llama import ModelConfig
    from runtime.executor import greedy_generate, read_tokens
    from runtime.program import compile_llama

    cfg = ModelConfig.llama2_7b(max_seq=256, num_layers=32)
    prog = compile_llama(cfg, 1, batch=1, prompt_len=128)
    hal, ora = _pair(prog, seed=0)
    prompt = np.random.default_rng(0).integers(0, cfg.vocab_size, (1, 128))
    # free-running greedy decode on both HALs: the same 5 tokens
    got, ref = [greedy_generate(prog.plans["prefill"], prog.plans["decode"], h, prompt, 5) for h in (hal, ora)]
    assert got.tokens.tolist() == ref.tokens.tolist()
    # node by node from identical state: the prefill, then 4 decode steps
    mirror_arena(prog, hal, ora)
    res = lockstep_compare(prog.plans["prefill"], hal, ora, tokens=prompt, pos=np.zeros(1, np.int32))
    _assert_nodes(res, "prefill")
    tok = read_tokens(prog.plans["prefill"], hal)
    for i in range(4):
        res = lockstep_compare(prog.plans["decode"], hal, ora, tokens=tok.reshape(1, 1),
                               pos=np.full(1, 128 + i, np.int32))
        _assert_nodes(res, f"decode step {i}")
        assert sum(1 for n, _, _ in res if str(n).endswith("mlp_act")) == 32
        tok = read_tokens(prog.plans["decode"], hal)
    assert all(v == 0 for v in hal.read_error_flags().values())
    hal.close()
    ora.close()


@pytest.mark.parametrize("tp", [1, 2])
def test_prefill_8x2048_last_logits_and_kv_match_oracle(tp):
    """The prefill benchmark's batch (8 x 2048, causal), 2 layers: last-position logits and KV."""
    from graph.llama import ModelConfig
    from runtime.executor import execute_plan, read_logits, read_tokens
    from runtime.program import compile_llama

    cfg = ModelConfig.llama2_7b(max_seq=2048, num_layers=2)
    prog = compile_llama(cfg, tp, batch=8, prompt_len=2048, phases=("prefill",))
    hal, ora = _pair(prog, seed=1)
    ids = np.random.default_rng(1).integers(0, cfg.vocab_size, (8, 2048))
    pf = prog.plans["prefill"]
    out = {}
    for name, h in (("b200", hal), ("oracle", ora)):
        execute_plan(pf, h, tokens=ids, pos=np.zeros(8, np.int32), timeout=600.0)
        out[name] = (read_logits(pf, h), read_tokens(pf, h))
    (lg, tg), (lr, tr) = out["b200"], out["oracle"]
    assert lg.shape[0] == 8
    assert max_rel_err(lg, lr) <= BF16_TOL
    assert tg.tolist() == tr.tolist()
    for r in range(tp):
        kg, kr = _kv_layers(prog, hal, r), _kv_layers(prog, ora, r)
        assert np.count_nonzero(kr) > 0.9 * kr.size  # every position of every sequence was written
        for layer in range(cfg.num_layers):
            assert max_rel_err(kg[layer], kr[layer]) <= BF16_TOL, (r, layer)
    assert all(v == 0 for v in hal.read_error_flags().values())
    hal.close()
    ora.close()


def test_batched_decode_64_sequences_at_context_4096_matches_oracle():
    """The batched-decode benchmark's shape (64 sequences, every KV block pre-filled with
    N(0, 1) values, decoding at positions 4096 and 4097), 2 layers: node by node at the first
    step, then a free-running step (logits within 2e-2, greedy ids equal up to ties)."""
    from backend import _native as nat
    from graph.llama import ModelConfig
    from runtime.executor import execute_plan, read_logits, read_tokens
    from runtime.program import compile_llama

    ctx, seqs = 4096, 64
    cfg = ModelConfig.llama2_7b(max_seq=ctx + 16, num_layers=2)
    prog = compile_llama(cfg, 1, batch=seqs, prompt_len=16, phases=("decode",))
    hal, ora = _pair(prog, seed=3)
    dp = prog.dpu_plans[0]
    nat.check(nat.lib.pim_fill_normal(hal.arena_ptr(0) + dp.kv_base, (dp.act_base - dp.kv_base) // 2, nat.BF16,
                                      1234, 1.0, hal.stream_handle(0)), "fill kv")
    hal.synchronize()
    mirror_arena(prog, hal, ora)
    dec = prog.plans["decode"]
    tokens = np.random.default_rng(3).integers(0, cfg.vocab_size, seqs).astype(np.int32)
    res = lockstep_compare(dec, hal, ora, tokens=tokens.reshape(seqs, 1), pos=np.full(seqs, ctx, np.int32))
    _assert_nodes(res, "batched decode step at 4096")
    tokens = read_tokens(dec, hal).reshape(-1)
    out = {}
    for n, h in (("b", hal), ("o", ora)):
        execute_plan(dec, h, tokens=tokens.reshape(seqs, 1), pos=np.full(seqs, ctx + 1, np.int32), timeout=900.0)
        out[n] = read_logits(dec, h)
    assert max_rel_err(out["b"], out["o"]) <= BF16_TOL
    gi, ri, tied = argmax_within_tolerance(out["b"], out["o"], BF16_TOL)
    assert all(g == r or i in tied for i, (g, r) in enumerate(zip(gi, ri))), (gi, ri, tied)
    assert len(tied) <= seqs // 4, tied
    assert read_tokens(dec, hal).reshape(-1).tolist() == gi
    assert all(v == 0 for v in hal.read_error_flags().values())
    hal.close()
    ora.close()
