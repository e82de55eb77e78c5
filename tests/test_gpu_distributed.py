"""One process per GPU (NCCL), the way bench.py runs under torchrun (GPU; needs 2+ GPUs).

Each process owns one rank of a TP=N program, N = the GPUs of the box (2, 4 or 8; the
tiny model, with 4 heads, runs on at most 4); combines run as NCCL collectives plus the
rank-ordered sum (or the P2P / fused all-reduce).  The tiny fp32 model must reproduce
HF's greedy tokens and logits; the 7B-architecture bf16 model (2 layers) must match the
oracle at the same TP: the oracle decodes greedily first and every rank is fed its
tokens (teacher forcing), so each step's logits are compared from identical inputs
(within 2e-2, greedy ids equal except at ties within that tolerance).
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


def _p2p_inputs(rank, t, call, dt):
    import ml_dtypes

    rng = np.random.default_rng(100 * t + 10 * call + rank)
    x = rng.standard_normal((t, 4096), dtype=np.float32)
    return x.astype(ml_dtypes.bfloat16) if dt == "bfloat16" else x


def _p2p_residual(t, call, dt):
    import ml_dtypes

    x = np.random.default_rng(7 * t + call).standard_normal((t, 4096), dtype=np.float32)
    return x.astype(ml_dtypes.bfloat16) if dt == "bfloat16" else x


def _p2p_worker(rank, world, out_dir):
    import torch

    from backend import _native as nat
    from backend.p2p import P2PGroup

    dev = torch.cuda.current_device()
    g = P2PGroup.create(rank, world, dev)
    assert g is not None, "peer mapping failed"
    err = torch.zeros(4, dtype=torch.int32, device=dev)
    res = {}
    for dt in ("bfloat16", "float32"):
        for t in (1, 16):
            for call in range(3):  # consecutive calls alternate the two slots
                x = _p2p_inputs(rank, t, call, dt)
                src = torch.from_numpy(x.view(np.uint16).astype(np.int16) if dt == "bfloat16" else x).cuda()
                out = torch.zeros_like(src)
                host_copy = torch.zeros_like(src)
                dsts = nat.ptr_array([out.data_ptr(), host_copy.data_ptr()])
                nat.check(nat.lib.pim_allreduce_p2p(src.data_ptr(), dsts, 2, x.size, nat.DTYPE_CODE[dt], rank, world,
                                                    g.ptrs, g.capacity, g.counter.data_ptr(), err.data_ptr(),
                                                    torch.cuda.current_stream().cuda_stream), "p2p")
                torch.cuda.synchronize()
                assert torch.equal(out, host_copy)
                res[f"{dt}_{t}_{call}"] = out.cpu().numpy()
                # the same all-reduce with the residual add folded in: y = residual + sum
                r_host = _p2p_residual(t, call, dt)
                resid = torch.from_numpy(r_host.view(np.uint16).astype(np.int16) if dt == "bfloat16" else r_host).cuda()
                y = torch.zeros_like(src)
                sum_out = torch.zeros_like(src)
                nat.check(nat.lib.pim_allreduce_p2p_add(src.data_ptr(), resid.data_ptr(), y.data_ptr(),
                                                        sum_out.data_ptr(), x.size, nat.DTYPE_CODE[dt], rank, world,
                                                        g.ptrs, g.capacity, g.counter.data_ptr(), err.data_ptr(),
                                                        torch.cuda.current_stream().cuda_stream), "p2p + add")
                torch.cuda.synchronize()
                assert torch.equal(sum_out, out)
                res[f"add_{dt}_{t}_{call}"] = y.cpu().numpy()
    # the low-latency protocol, on a group of its own (a group runs one protocol only); each
    # 8-byte word carries 4 payload bytes, so a row holds twice the payload: 16 x 4096 fp32
    # needs 512 KB
    g2 = P2PGroup.create(rank, world, dev, capacity=2 * 16 * 4096 * 4)
    assert g2 is not None, "peer mapping failed"
    for dt in ("bfloat16", "float32"):
        for t in (1, 16):
            for call in range(3):
                x = _p2p_inputs(rank, t, call, dt)
                src = torch.from_numpy(x.view(np.uint16).astype(np.int16) if dt == "bfloat16" else x).cuda()
                r_host = _p2p_residual(t, call, dt)
                resid = torch.from_numpy(r_host.view(np.uint16).astype(np.int16) if dt == "bfloat16" else r_host).cuda()
                out, y = torch.zeros_like(src), torch.zeros_like(src)
                code = nat.DTYPE_CODE[dt]
                st = torch.cuda.current_stream().cuda_stream
                nat.check(nat.lib.pim_allreduce_p2p_ll(src.data_ptr(), None, None, out.data_ptr(), x.size, code, rank,
                                                       world, g2.ptrs, g2.capacity, g2.counter.data_ptr(),
                                                       err.data_ptr(), st), "p2p ll")
                nat.check(nat.lib.pim_allreduce_p2p_ll(src.data_ptr(), resid.data_ptr(), y.data_ptr(), None, x.size,
                                                       code, rank, world, g2.ptrs, g2.capacity,
                                                       g2.counter.data_ptr(), err.data_ptr(), st), "p2p ll + add")
                torch.cuda.synchronize()
                res[f"ll_{dt}_{t}_{call}"] = out.cpu().numpy()
                res[f"lladd_{dt}_{t}_{call}"] = y.cpu().numpy()
    assert int(err.abs().sum()) == 0
    np.savez(Path(out_dir) / f"rank{rank}.npz", **res)
    g.close()
    g2.close()


def _redist_worker(rank, world, out_dir, allreduce, extra):
    """Every golden redistribute edge of this world size as its own single-edge plan, this
    process running rank ``rank``: load the rank's share of the golden inputs, execute, hash
    the rank's destination."""
    import json

    from backend.hal_cuda import CudaBackend, CudaBackendConfig
    from helpers import GOLDEN, comm_inputs, sha
    from runtime.exec_plan_gen import redistribute_edge, redistribute_plan
    from runtime.executor import execute_plan

    cases = [c for c in json.loads((GOLDEN / "comm_golden.json").read_text())["cases"] if c["n"] == world]
    nbytes = max(c["tokens"] for c in cases) * 4096 * 2
    hal = CudaBackend(CudaBackendConfig(world, 2 * nbytes + 4096, rank=rank, allreduce=allreduce, **(extra or {})))
    res = {}
    for c in cases:
        t, kind = c["tokens"], c["type"]
        edge, entry = redistribute_edge(kind, world, (t, 4096))
        plan = redistribute_plan(edge, entry)
        hal.register_plan(plan)
        data = comm_inputs(kind, world, t)
        if kind == "all_reduce":
            mine = data[rank]
        elif kind == "all_gather":  # Shard(last): this rank's columns
            w = 4096 // world
            mine = data[:, rank * w:(rank + 1) * w]
        else:  # all_to_all from Shard(0): this rank's rows
            r = t // world
            mine = data[rank * r:(rank + 1) * r, :]
        hal.copy_to_dpu(rank, 0, np.ascontiguousarray(mine).reshape(-1))
        execute_plan(plan, hal)
        size = t * 4096 // (world if kind == "all_to_all" else 1)
        res[c["key"]] = np.array(sha(hal.read_local(rank, t * 4096 * 2, (size,), entry.dtype)))
        hal.release_plan(plan)
    assert all(v == 0 for v in hal.read_error_flags().values())
    np.savez(Path(out_dir) / f"rank{rank}.npz", **res)
    hal.close()


def _worker(rank, world, port, out_dir, model, allreduce="ordered", extra=None):
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
        if model == "p2p":
            _p2p_worker(rank, world, out_dir)
            return
        if model == "redistribute":
            _redist_worker(rank, world, out_dir, allreduce, extra)
            return
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
            prompt, steps = _7B_PROMPT(cfg), 3
        extra = dict(extra or {})
        kernel = extra.pop("projection_kernel", None)
        if kernel is not None:  # a decode GEMV other than the default, in this process
            from backend import _native as nat

            nat.check(nat.lib.pim_set_projection_kernel(kernel), "pim_set_projection_kernel")
        hal = CudaBackend(CudaBackendConfig(world, prog.arena_bytes, rank=rank, allreduce=allreduce, **extra))
        for p in prog.plans.values():
            hal.register_plan(p)
        load_weights(prog, hal, w)
        forced = Path(out_dir) / "forced_tokens.npy"
        if model == "7b" and forced.exists():  # teacher forcing with the oracle's tokens
            from helpers import forced_generate

            logits = forced_generate(prog, hal, prompt, np.load(forced)[:, :steps - 1])
            tokens = np.stack([np.asarray(l, np.float32).reshape(1, -1).argmax(-1) for l in logits], 1)
        else:
            res = greedy_generate(prog.plans["prefill"], prog.plans["decode"], hal, prompt, steps)
            tokens, logits = res.tokens, [res.prefill_logits] + res.step_logits
        if allreduce == "fused":  # decode's o_proj and down_proj chains run as one kernel each
            assert hal.fused_allreduces == 2 * 2, hal.fused_allreduces
        if extra.get("combine_add"):  # every all_reduce of both plans folds its add
            assert hal.combine_adds == 2 * 2 * 2, hal.combine_adds
        if extra.get("decode_layer"):  # both decode layers, each with its two all-reduces, as one launch
            assert hal.decode_layers == 2, hal.decode_layers
        if extra.get("decode_step"):  # and the whole decode step as one launch
            assert hal.decode_steps == 1, hal.decode_steps
        np.savez(Path(out_dir) / f"rank{rank}.npz", tokens=tokens,
                 logits=np.stack([np.asarray(l, np.float32).reshape(-1) for l in logits]))
        assert all(v == 0 for v in hal.read_error_flags().values())
    finally:
        dist.destroy_process_group()


def _7B_PROMPT(cfg):
    return np.random.default_rng(4).integers(0, cfg.vocab_size, (1, 64))


def _world(model: str) -> int:
    """Ranks of a run: every GPU of the box (2, 4 or 8), at most 4 for the 4-head tiny model."""
    import torch

    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs (one process per GPU)")
    n = 8 if n >= 8 else (4 if n >= 4 else 2)
    return min(n, 4) if model == "tiny" else n


def _spawn(model, tmp_path, allreduce="ordered", extra=None, forced_tokens=None):
    import torch.multiprocessing as mp

    world = _world(model)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    Path(tmp_path).mkdir(parents=True, exist_ok=True)
    if forced_tokens is not None:
        np.save(Path(tmp_path) / "forced_tokens.npy", np.asarray(forced_tokens))
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path), model, allreduce, extra), nprocs=world, join=True)
    return [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]


def test_p2p_allreduce_is_the_rank_order_sum_bit_exact(tmp_path):
    """pim_allreduce_p2p (flag protocol) and pim_allreduce_p2p_ll (epoch-tagged words) over NVLink
    equal the sequential sum of comm/lowering.py bit for bit, alone and with the residual add."""
    import ml_dtypes

    ranks = _spawn("p2p", tmp_path)
    for dt in ("bfloat16", "float32"):
        for t in (1, 16):
            for call in range(3):
                acc = np.zeros((t, 4096), np.float32)
                for r in range(len(ranks)):  # fp32 add, then round to the element type after every add
                    acc = acc + _p2p_inputs(r, t, call, dt).astype(np.float32)
                    if dt == "bfloat16":
                        acc = acc.astype(ml_dtypes.bfloat16).astype(np.float32)
                want = acc.astype(ml_dtypes.bfloat16).view(np.uint16) if dt == "bfloat16" else acc.view(np.uint32)
                # y = residual + sum: the fp32 add of the rounded sum, rounded once (pim_ordered_sum_add)
                y = _p2p_residual(t, call, dt).astype(np.float32) + acc
                want_y = y.astype(ml_dtypes.bfloat16).view(np.uint16) if dt == "bfloat16" else y.view(np.uint32)
                for r in ranks:
                    got = r[f"{dt}_{t}_{call}"]
                    got = got.view(np.uint16) if dt == "bfloat16" else got.view(np.uint32)
                    assert np.array_equal(got.reshape(want.shape), want), (dt, t, call)
                    for key, w in ((f"add_{dt}_{t}_{call}", want_y), (f"ll_{dt}_{t}_{call}", want),
                                   (f"lladd_{dt}_{t}_{call}", want_y)):
                        got_y = r[key]
                        got_y = got_y.view(np.uint16) if dt == "bfloat16" else got_y.view(np.uint32)
                        assert np.array_equal(got_y.reshape(w.shape), w), key


@pytest.mark.parametrize("allreduce,extra", [("ordered", {}), ("p2p", {}), ("ordered", {"allreduce_split_bytes": 65536})],
                         ids=["ordered", "p2p", "split"])
def test_redistribute_edges_one_process_per_gpu_match_the_reference(tmp_path, allreduce, extra):
    """The redistribute microbench's edges with one rank per GPU (NCCL all_gather + rank-order
    sum, the low-latency P2P all-reduce for edges that fit its rows, the split all-reduce,
    the NCCL all_gather and per-peer all_to_all): every rank's destination bit-identical to
    the reference's lowering (golden hashes of comm/lowering.py's outputs, N = the box's GPUs)."""
    import json

    from helpers import GOLDEN

    ranks = _spawn("redistribute", tmp_path, allreduce, extra)
    cases = [c for c in json.loads((GOLDEN / "comm_golden.json").read_text())["cases"] if c["n"] == len(ranks)]
    assert cases
    for r, res in enumerate(ranks):
        for c in cases:
            want = c["dst_local_sha"][r] if c["type"] == "all_to_all" else c["out_sha"]
            assert str(res[c["key"]]) == want, (allreduce, extra, r, c["key"])


def test_tiny_llama_one_process_per_gpu_matches_hf(tmp_path):
    from helpers import tiny_golden

    gold = tiny_golden()
    for r in _spawn("tiny", tmp_path):
        assert r["tokens"][0].tolist() == gold["tokens"].tolist()
        for got, ref in zip(r["logits"], gold["step_logits"]):
            assert np.abs(got - ref.reshape(-1)).max() <= 1e-4 * np.abs(ref).max()


def _check_7b_vs_oracle(tmp_path, allreduce="ordered", extra=None):
    """The 7B-architecture 2-layer model at TP = the box's GPU count against the oracle at the
    same TP: the oracle decodes greedily, the ranks are fed its tokens, and every step's
    logits must agree within 2e-2 with greedy ids equal up to ties at that tolerance."""
    from assert_node_matches_ref import argmax_within_tolerance
    from graph.llama import ModelConfig
    from helpers import oracle_hal
    from runtime.executor import greedy_generate
    from runtime.program import compile_llama, fused_weights, load_weights
    from test_gpu_model import _l7b_weights

    world = _world("7b")
    cfg = ModelConfig.llama2_7b(max_seq=256, num_layers=2)
    prog = compile_llama(cfg, world, batch=1, prompt_len=64)
    hal = oracle_hal(prog)
    load_weights(prog, hal, fused_weights(cfg, _l7b_weights(ModelConfig.llama2_7b(max_seq=32, num_layers=2)), world))
    ref = greedy_generate(prog.plans["prefill"], prog.plans["decode"], hal, _7B_PROMPT(cfg), 3)
    hal.close()
    ranks = _spawn("7b", tmp_path, allreduce, extra, forced_tokens=ref.tokens)
    ref_logits = [l.astype(np.float32).reshape(-1) for l in [ref.prefill_logits] + ref.step_logits]
    for r in ranks:
        assert len(r["logits"]) == len(ref_logits)
        for got, want in zip(r["logits"], ref_logits):
            assert np.abs(got - want).max() <= 2e-2 * np.abs(want).max()
            gi, ri, tied = argmax_within_tolerance(got[None], want[None], 2e-2)
            assert gi == ri or tied == [0], (gi, ri)
    # every rank holds the same gathered logits
    for r in ranks[1:]:
        assert np.array_equal(r["logits"].view(np.uint32), ranks[0]["logits"].view(np.uint32))


@pytest.mark.parametrize("allreduce", ["ordered", "p2p", "fused"])
def test_llama2_7b_arch_one_process_per_gpu_matches_oracle(tmp_path, allreduce):
    _check_7b_vs_oracle(tmp_path, allreduce)


@pytest.mark.skipif(os.environ.get("PIM_TEST_OPT_IN") != "1", reason="opt-in paths: set PIM_TEST_OPT_IN=1")
@pytest.mark.parametrize("mode,extra", [("ordered", {"combine_add": True}), ("ordered", {"allreduce_split_bytes": 1}),
                                        ("ordered", {"allreduce_split_bytes": 1 << 20, "combine_add": True}),
                                        ("p2p", {}), ("p2p", {"combine_add": True})],
                         ids=["combine_add", "split", "split_large_and_combine_add", "p2p", "p2p_combine_add"])
def test_opt_in_ordered_paths_give_the_default_bits(tmp_path, mode, extra):
    """The fold of the add into the combine (NCCL or P2P sum), the split all_reduce and the P2P
    all-reduce keep every bit of the default path."""
    base = _spawn("7b", tmp_path / "base")
    ranks = _spawn("7b", tmp_path / "opt", mode, extra)
    for got, want in zip(ranks, base):
        assert got["tokens"].tolist() == want["tokens"].tolist()
        assert np.array_equal(got["logits"].view(np.uint32), want["logits"].view(np.uint32))


@pytest.mark.skipif(os.environ.get("PIM_TEST_OPT_IN") != "1", reason="opt-in paths: set PIM_TEST_OPT_IN=1")
@pytest.mark.parametrize("allreduce", ["ordered", "fused"])
def test_dynamic_gemv_one_process_per_gpu_matches_oracle(tmp_path, allreduce):
    """The dynamic-assignment GEMV one process per GPU, alone and in its fused all-reduce form."""
    _check_7b_vs_oracle(tmp_path, allreduce, {"projection_kernel": 3})


@pytest.mark.skipif(os.environ.get("PIM_TEST_OPT_IN") != "1", reason="opt-in paths: set PIM_TEST_OPT_IN=1")
def test_decode_layer_fused_one_process_per_gpu_matches_oracle(tmp_path):
    """One launch per decode layer with its two fused all-reduces (pim_decode_layer, AR form)."""
    _check_7b_vs_oracle(tmp_path, "fused", {"decode_layer": True})


@pytest.mark.skipif(os.environ.get("PIM_TEST_OPT_IN") != "1", reason="opt-in paths: set PIM_TEST_OPT_IN=1")
def test_decode_layer_tiny_llama_one_process_per_gpu_matches_hf(tmp_path):
    from helpers import tiny_golden

    gold = tiny_golden()
    for r in _spawn("tiny", tmp_path, "fused", {"decode_layer": True}):
        assert r["tokens"][0].tolist() == gold["tokens"].tolist()
        for got, ref in zip(r["logits"], gold["step_logits"]):
            assert np.abs(got - ref.reshape(-1)).max() <= 1e-4 * np.abs(ref).max()


@pytest.mark.skipif(os.environ.get("PIM_TEST_OPT_IN") != "1", reason="opt-in paths: set PIM_TEST_OPT_IN=1")
def test_decode_step_fused_one_process_per_gpu_matches_oracle(tmp_path):
    """The whole decode step as one launch per rank, every layer's all-reduces inside it."""
    _check_7b_vs_oracle(tmp_path, "fused", {"decode_layer": True, "decode_step": True})
