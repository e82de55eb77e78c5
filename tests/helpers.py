"""Shared builders for the tests (tiny HF model, programs, HALs)."""

from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def tiny_hf_model():
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=1024, hidden_size=256, intermediate_size=688, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=4, rms_norm_eps=1e-6, rope_theta=10000.0,
                      max_position_embeddings=64, bos_token_id=1, eos_token_id=2, pad_token_id=0,
                      initializer_range=0.02)
    return LlamaForCausalLM(cfg).eval()


def tiny_gqa_hf_model():
    """The tiny configuration with grouped-query attention: 8 query heads share 2 kv heads."""
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=1024, hidden_size=256, intermediate_size=688, num_hidden_layers=2,
                      num_attention_heads=8, num_key_value_heads=2, rms_norm_eps=1e-6, rope_theta=10000.0,
                      max_position_embeddings=64, initializer_range=0.02)
    return LlamaForCausalLM(cfg).eval()


def hf_greedy(model, prompt, steps):
    """HF single-card greedy decode: (tokens, [logits of the prompt's last position and of each step])."""
    import torch

    ids = torch.tensor(np.asarray(prompt))
    toks, logits = [], []
    with torch.no_grad():
        for _ in range(steps + 1):
            out = model(ids).logits[0, -1].float().numpy()
            logits.append(out)
            t = int(out.argmax())
            toks.append(t)
            ids = torch.cat([ids, torch.tensor([[t]])], 1)
    return toks, logits


def tiny_golden():
    return np.load(GOLDEN / "tiny_llama_golden.npz")


def weights_sha(model) -> str:
    sd = model.state_dict()
    return hashlib.sha256(b"".join(sd[k].numpy().tobytes() for k in sorted(sd))).hexdigest()


def tiny_program(tp: int, max_seq: int = 32, batch: int = 1, prompt_len: int = 16):
    from graph.llama import ModelConfig
    from runtime.program import compile_llama

    return compile_llama(ModelConfig.tiny(max_seq=max_seq), tp, batch=batch, prompt_len=prompt_len)


def tiny_weights(prog, model):
    from runtime.program import fused_weights, hf_state_dict

    return fused_weights(prog.cfg, hf_state_dict(model, prog.cfg.dtype), prog.tp)


def oracle_hal(prog):
    from oracle.hal_numpy import NumpyBackend, NumpyBackendConfig

    hal = NumpyBackend(NumpyBackendConfig(prog.tp, prog.arena_bytes))
    for p in prog.plans.values():
        hal.register_plan(p)
    return hal


def cuda_hal(prog, **kw):
    from backend.hal_cuda import CudaBackend, CudaBackendConfig

    hal = CudaBackend(CudaBackendConfig(prog.tp, prog.arena_bytes, **kw))
    for p in prog.plans.values():
        hal.register_plan(p)
    return hal


def comm_inputs(kind: str, n: int, tokens: int, hidden: int = 4096, seed: int = 0):
    """Same recipe as tests/golden/make_golden.py:comm_inputs."""
    import ml_dtypes

    rng = np.random.default_rng(seed + 1000 * n + tokens)
    if kind == "all_reduce":
        return [rng.standard_normal((tokens, hidden), dtype=np.float32).astype(ml_dtypes.bfloat16)
                for _ in range(n)]
    return rng.standard_normal((tokens, hidden), dtype=np.float32).astype(ml_dtypes.bfloat16)


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).view(np.uint8).tobytes()).hexdigest()


def redistribute_entry(kind: str, n: int, shape, dtype: str = "bfloat16"):
    """One comm-plan entry for the redistribute microbench (src at offset 0, dst after it)."""
    from math import prod

    from runtime.exec_plan_gen import redistribute_edge

    _, entry = redistribute_edge(kind, n, tuple(shape), dtype)
    return entry, prod(shape) * (2 if dtype == "bfloat16" else 4)


PROJECTION_KERNELS = ("register", "staged")
# Selectable by name too; not in PROJECTION_KERNELS (the GPU parametrisation) yet.
PROJECTION_KERNEL_CODES = {"register": 0, "staged": 1, "dynamic": 3}


class projection_kernel:
    """Context manager: run decode projections on one of the library's GEMV kernels."""

    def __init__(self, name: str) -> None:
        self.code = PROJECTION_KERNEL_CODES[name]

    def __enter__(self):
        from backend import _native as nat

        self.prev = nat.lib.pim_projection_kernel()
        nat.check(nat.lib.pim_set_projection_kernel(self.code), "pim_set_projection_kernel")
        return self

    def __exit__(self, *exc):
        from backend import _native as nat

        nat.lib.pim_set_projection_kernel(self.prev)


def mirror_zone(prog, src_hal, dst_hal, lo_attr: str = "weight", chunk: int = 1 << 30) -> None:
    """Copy one zone of every rank's arena from ``src_hal`` to ``dst_hal`` (same program, so the
    same offsets): ``"weight"`` is [0, kv_base), ``"kv"`` is [kv_base, act_base).  Used to give
    the oracle exactly the bytes a device-side initialisation wrote."""
    for r, dp in prog.dpu_plans.items():
        lo, hi = (0, dp.kv_base) if lo_attr == "weight" else (dp.kv_base, dp.act_base)
        for off in range(lo, hi, chunk):
            n = min(chunk, hi - off)
            dst_hal.copy_to_dpu(r, off, src_hal.copy_from_dpu(r, off, (n,), np.uint8))


def max_rel_err(got, ref) -> float:
    """max |got - ref| / max |ref| over fp32 views of two arrays of one shape."""
    a, b = np.asarray(got, np.float32), np.asarray(ref, np.float32)
    assert a.shape == b.shape, (a.shape, b.shape)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def forced_generate(prog, hal, prompt, tokens):
    """Prefill ``prompt`` ([batch, P]), then one decode step per column of ``tokens``
    ([batch, n]) fed as that step's input whatever this HAL would have sampled (teacher
    forcing): returns [prefill logits, logits of each step].  Two HALs given the same
    tokens see the same inputs at every step, so a near-tie that flips one greedy id
    cannot send them down different sequences."""
    from runtime.executor import execute_plan, read_logits

    prompt = np.asarray(prompt, np.int32)
    b, p = prompt.shape
    execute_plan(prog.plans["prefill"], hal, tokens=prompt, pos=np.zeros(b, np.int32), timeout=900.0)
    logits = [read_logits(prog.plans["prefill"], hal)]
    tokens = np.asarray(tokens, np.int32).reshape(b, -1)
    for i in range(tokens.shape[1]):
        execute_plan(prog.plans["decode"], hal, tokens=tokens[:, i:i + 1], pos=np.full(b, p + i, np.int32),
                     timeout=900.0)
        logits.append(read_logits(prog.plans["decode"], hal))
    return logits


def mirror_arena(prog, src_hal, dst_hal, chunk: int = 1 << 30) -> None:
    """Copy every rank's whole arena (weights, KV, activations) from ``src_hal`` to ``dst_hal``."""
    for r in prog.dpu_plans:
        total = prog.arena_bytes
        for off in range(0, total, chunk):
            n = min(chunk, total - off)
            dst_hal.copy_to_dpu(r, off, src_hal.copy_from_dpu(r, off, (n,), np.uint8))
