"""One process per GPU (NCCL), the way bench.py runs under torchrun (GPU; needs 2 GPUs).

Each process owns one rank of a TP=2 program; combines run as NCCL all_gathers plus
the rank-ordered sum.  The tiny fp32 model must reproduce HF's greedy tokens and
logits; the 7B-architecture bf16 model (2 layers) must match the oracle at TP=2.
"""

from __future__ import annotations

import os
import socket
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir, model):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from backend.hal_cuda import CudaBackend, CudaBackendConfig
    from helpers import tiny_golden, tiny_hf_model, tiny_program, tiny_weights
    from runtime.executor import greedy_generate
    from runtime.program import compile_llama, fused_weights, load_weights

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        if model == "tiny":
            prog = tiny_program(world)
            w = tiny_weights(prog, tiny_hf_model())
            prompt, steps = tiny_golden()["prompt"][None], 8
        else:
            from graph.llama import ModelConfig
            from test_gpu_model import _l7b_weights

            cfg = ModelConfig.llama2_7b(max_seq=256, num_layers=2)
            prog = compile_llama(cfg, world, batch=1, prompt_len=64)
            w = fused_weights(cfg, _l7b_weights(ModelConfig.llama2_7b(max_seq=32, num_layers=2)), world)
            prompt, steps = np.random.default_rng(4).integers(0, cfg.vocab_size, (1, 64)), 3
        hal = CudaBackend(CudaBackendConfig(world, prog.arena_bytes, rank=rank))
        for p in prog.plans.values():
            hal.register_plan(p)
        load_weights(prog, hal, w)
        res = greedy_generate(prog.plans["prefill"], prog.plans["decode"], hal, prompt, steps)
        np.savez(Path(out_dir) / f"rank{rank}.npz", tokens=res.tokens,
                 logits=np.stack([l.astype(np.float32).reshape(-1) for l in [res.prefill_logits] + res.step_logits]))
        assert all(v == 0 for v in hal.read_error_flags().values())
    finally:
        dist.destroy_process_group()


def _spawn(model, tmp_path):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs (one process per GPU)")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path), model), nprocs=2, join=True)
    return [np.load(tmp_path / f"rank{r}.npz") for r in range(2)]


def test_tiny_llama_tp2_one_process_per_gpu_matches_hf(tmp_path):
    from helpers import tiny_golden

    gold = tiny_golden()
    for r in _spawn("tiny", tmp_path):
        assert r["tokens"][0].tolist() == gold["tokens"].tolist()
        for got, ref in zip(r["logits"], gold["step_logits"]):
            assert np.abs(got - ref.reshape(-1)).max() <= 1e-4 * np.abs(ref).max()


def test_llama2_7b_arch_tp2_one_process_per_gpu_matches_oracle(tmp_path):
    from graph.llama import ModelConfig
    from helpers import oracle_hal
    from runtime.executor import greedy_generate
    from runtime.program import compile_llama, fused_weights, load_weights
    from test_gpu_model import _l7b_weights

    ranks = _spawn("7b", tmp_path)
    cfg = ModelConfig.llama2_7b(max_seq=256, num_layers=2)
    prog = compile_llama(cfg, 2, batch=1, prompt_len=64)
    hal = oracle_hal(prog)
    load_weights(prog, hal, fused_weights(cfg, _l7b_weights(ModelConfig.llama2_7b(max_seq=32, num_layers=2)), 2))
    ref = greedy_generate(prog.plans["prefill"], prog.plans["decode"], hal,
                          np.random.default_rng(4).integers(0, cfg.vocab_size, (1, 64)), 3)
    ref_logits = [l.astype(np.float32).reshape(-1) for l in [ref.prefill_logits] + ref.step_logits]
    for r in ranks:
        assert r["tokens"].tolist() == ref.tokens.tolist()
        for got, want in zip(r["logits"], ref_logits):
            assert np.abs(got - want).max() <= 2e-2 * np.abs(want).max()
