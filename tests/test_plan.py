"""Compile-time checks: memory plan disjointness, plan hazard freedom, plan shapes."""

from __future__ import annotations

import pytest

from helpers import tiny_program


def _programs():
    from graph.llama import ModelConfig
    from runtime.program import compile_llama

    yield "tiny_tp1", tiny_program(1)
    yield "tiny_tp2", tiny_program(2)
    yield "tiny_tp4", tiny_program(4)
    yield "tiny_tp4_b2", tiny_program(4, batch=2, prompt_len=8)
    yield "l7b_2layer_tp8", compile_llama(ModelConfig.llama2_7b(max_seq=64, num_layers=2), 8, batch=1,
                                          prompt_len=16)


@pytest.mark.parametrize("name,prog", list(_programs()), ids=lambda x: x if isinstance(x, str) else "")
def test_plans_are_hazard_free(name, prog):
    from runtime.validate import plan_hazards

    for phase, plan in prog.plans.items():
        assert plan_hazards(plan) == [], f"{name}/{phase}"


@pytest.mark.parametrize("name,prog", list(_programs()), ids=lambda x: x if isinstance(x, str) else "")
def test_arenas_disjoint_and_within_budget(name, prog):
    from runtime.validate import arena_overlaps

    for r, p in prog.dpu_plans.items():
        assert arena_overlaps(p) == [], f"{name}/dpu{r}"
        assert p.total <= prog.arena_bytes
        weights = sorted(p.weight.values())
        assert weights == sorted(set(weights))
        assert max(weights) < p.kv_base <= p.act_base


def test_activation_reuse_emits_pending_readers():
    prog = tiny_program(2)
    pr = prog.dpu_plans[0].pending_readers["llama_decode_b1_s1"]
    assert pr, "greedy reuse must share at least one address in a 2-layer decode step"
    assert all(loc == ("dpu", 0) for loc, _ in pr)


def test_collectives_per_decode_step():
    """Per layer exactly two Partial->Replicate all_reduces (o_proj, down_proj) plus the logits gather."""
    prog = tiny_program(4)
    types = [e.type for e in prog.entries["decode"]]
    assert types.count("all_reduce") == 2 * prog.cfg.num_layers
    assert types.count("all_gather") == 1
    assert set(types) == {"all_reduce", "all_gather", "scatter"}


def test_tp1_elides_identity_collectives():
    prog = tiny_program(1)
    ops = {c.op for c in prog.plans["decode"].commands}
    assert "host_reduce" not in ops  # a sum over one partial is the partial itself


def test_plan_rejects_bad_shard_config():
    from graph.llama import ModelConfig
    from runtime.program import compile_llama

    with pytest.raises(ValueError):
        compile_llama(ModelConfig.tiny(), 3)
    with pytest.raises(ValueError):
        compile_llama(ModelConfig.tiny(), 8)  # 4 heads do not split over 8 ranks
    with pytest.raises(ValueError):
        compile_llama(ModelConfig.tiny(max_seq=16), 1, prompt_len=16)


def test_grouped_query_attention_needs_a_kv_head_per_rank():
    """GQA shards whole kv heads: 2 kv heads split over 2 ranks, not over 4."""
    from dataclasses import replace

    from graph.llama import ModelConfig
    from runtime.program import compile_llama

    gqa = replace(ModelConfig.tiny(max_seq=32), num_heads=8, num_kv_heads=2)
    assert compile_llama(gqa, 2, batch=1, prompt_len=16).arena_bytes > 0
    with pytest.raises(ValueError, match="num_kv_heads=2 is not divisible by num_dpus=4"):
        compile_llama(gqa, 4, batch=1, prompt_len=16)


def test_capacity_check_raises():
    from graph.llama import ModelConfig
    from runtime.program import compile_llama

    with pytest.raises(ValueError, match="budget"):
        compile_llama(ModelConfig.tiny(), 1, mram_budget=1 << 20)
