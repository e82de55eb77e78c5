"""LLaMA2-7B-architecture decode throughput on B200 (tokens/s), the ExecutionPlan hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload (one "step" = one greedy decode step): LLaMA2-7B architecture
(32 layers, hidden 4096, 32x128 heads, MLP 11008, vocab 32000), bf16
random-init weights N(0, 0.02), batch 1, a 128-token random prompt prefilled
first, then decode steps at positions 128.. (max_seq 256), TP = N ranks.
With N > 1 the driver launches one process per GPU (torchrun); the two per-layer
all_reduces of decode go over NVLink peer memory (the low-latency protocol, with the
residual add in the same kernel), larger edges and the logits gather over NCCL.

``value`` is device-timed (CUDA events on the host stream, barrier +
synchronize around, max over ranks) with every input resident in HBM: each
step is one replay of the captured decode plan, the sampled token fed back on
the device.  ``e2e`` is the same metric through ``LlamaRunner.step`` -- the
token and position copied from pinned host memory and the next token read
back, every step.  The weights (13.5 GB) exceed L2 (126 MB), so no flush is
needed between steps.

``prefill`` (an extra object on the same line) is the other half of the metric:
8 x 2048 uniform random ids, causal, TP = N, the whole prefill plan timed with CUDA
events (max over ranks), with the tensor-core roofline of the layer-0 projections.

``--batched`` measures batched decode instead (64 sequences, KV pre-filled with
N(0, 1) at context 4096, 32 steps) and prints its own line; ``--redistribute`` the
redistribute microbench (bf16 [T, 4096] edges at N >= 2 ranks, bus bandwidth against
NVLink); ``--ab`` times the default kernels against each opt-in decode and prefill
variant in one process (one GPU); ``--allreduce`` picks the Partial->Replicate path at
N > 1 (default p2p; ``ordered``: NCCL all_gather + rank-order sum for every edge).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for p in (str(ROOT / "flagos-pim-compiler_b200"), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

PROMPT = 128
MAX_SEQ = 256
METRIC = "LLaMA2-7B decode tokens/s (TP=N, batch 1, bf16)"
SPLIT_BYTES_DEFAULT = 8 << 20  # prefill's [8 x 2048, 4096] bf16 edges (134 MB); decode edges are 8-512 KB


def _peaks() -> dict:
    """Roofline denominators: the measured HBM copy bandwidth and cuBLAS bf16 throughput, as a
    burst (kernels timed alone) and sustained (inside a long step)."""
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d["bf16_tflops_sustained"], "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


_REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
            ("sw_power_cap", 0x4))


class ClockSampler:
    """SM clocks and throttle reasons of this process's GPU sampled DURING the timed region.

    NVML is polled from a thread every ``period_s`` (read-only queries: SM clock, max SM
    clock, clock-event reasons), so even a timed region of a few tens of milliseconds gets
    samples; ``__enter__`` returns once the first sample is in.  Without NVML it falls back
    to ``nvidia-smi -lms 50``.
    """

    def __init__(self, gpu: int, period_s: float = 0.005) -> None:
        self.gpu, self.period, self.rows, self.proc, self.nvml = gpu, period_s, [], None, None
        self._stop = threading.Event()
        self.max_mhz = None

    def _nvml_handle(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        uuid = "GPU-" + str(torch.cuda.get_device_properties(self.gpu).uuid)
        for i in range(pynvml.nvmlDeviceGetCount()):
            h = pynvml.nvmlDeviceGetHandleByIndex(i)
            u = pynvml.nvmlDeviceGetUUID(h)
            if (u.decode() if isinstance(u, bytes) else u) == uuid:
                return pynvml, h
        raise RuntimeError("this GPU is not in NVML's list")

    def __enter__(self):
        try:
            self.nvml, self.h = self._nvml_handle()
            self.max_mhz = float(self.nvml.nvmlDeviceGetMaxClockInfo(self.h, self.nvml.NVML_CLOCK_SM))
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
            t0 = time.perf_counter()
            while not self.rows and time.perf_counter() - t0 < 2.0:
                time.sleep(0.001)
            return self
        except Exception:  # noqa: BLE001 -- no NVML: sample with nvidia-smi instead
            self.nvml = None
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _poll(self):
        nv, h = self.nvml, self.h
        while not self._stop.is_set():
            try:
                sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                mask = int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))
            except Exception:  # noqa: BLE001 -- a failed query ends the sampling
                return
            self.rows.append((sm, self.max_mhz, [n for n, bit in _REASONS if mask & bit]))
            self._stop.wait(self.period)

    def _read(self):
        names = [n for n, _ in _REASONS]
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) == 7 and parts[0].replace(".", "").isdigit():
                mx = float(parts[1]) if parts[1].replace(".", "").isdigit() else None
                self.rows.append((float(parts[0]), mx, [names[i] for i in range(4) if parts[3 + i].lower() == "active"]))

    def __exit__(self, *exc):
        self._stop.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(2)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.nvml is not None:
            self.t.join(1.0)

    def summary(self) -> dict:
        sm = [r[0] for r in self.rows]
        mx = [r[1] for r in self.rows if r[1] is not None]
        reasons = sorted({n for r in self.rows for n in r[2]})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows), "source": "nvml" if self.nvml else "nvidia-smi"}


# ncu summary of the roofline kernel (the layer-0 mlp_in projection at TP=1); its
# "traffic_bytes_per_launch:" line is dram__bytes_read.sum + dram__bytes_write.sum of one launch.
ROOFLINE_PROFILE = ROOT / "profiles" / "gemv_staged_llama2_7b_decode_layer0.md"


def _profiled_traffic(tp: int):
    """DRAM bytes of one launch of the roofline kernel, from its committed ncu summary (TP=1 only)."""
    if tp != 1 or not ROOFLINE_PROFILE.exists():
        return None
    for line in ROOFLINE_PROFILE.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            return int(line.split(":", 1)[1].strip())
    return None


def _dist_setup(n: int, timeout_s: int = 120):
    """One process per GPU: NCCL process group with a bounded collective timeout."""
    import torch
    import torch.distributed as dist

    if n == 1:
        return 0, None
    rank = int(os.environ["RANK"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    from datetime import timedelta

    dist.init_process_group("nccl", timeout=timedelta(seconds=timeout_s))
    return rank, dist


def cpu_baseline(tp: int, budget_s: float = 30.0, layers: int = 32, max_steps: int = 8) -> dict:
    """The oracle (NumPy HAL restating the reference runtime) timing whole decode steps of the
    benchmarked model: LLaMA2-7B architecture, all ``layers`` layers, TP = ``tp`` simulated
    ranks, batch 1, positions 128, 129, ... (max_seq 256).

    One untimed step first (it touches every page of the arenas), then whole steps until
    ``budget_s`` is spent (at least one, at most ``max_steps``); the value is steps / seconds.  The
    weights are random bf16 (a repeated N(0, 0.02) block: the oracle's time does not depend
    on the values), the NumPy BLAS and the HAL's per-rank threads use every host core.
    """
    import ml_dtypes
    import numpy as np

    from graph.llama import ModelConfig
    from oracle.hal_numpy import NumpyBackend, NumpyBackendConfig
    from runtime.executor import execute_plan
    from runtime.program import compile_llama

    block = (np.random.default_rng(0).standard_normal(1 << 20, dtype=np.float32) * 0.02).astype(ml_dtypes.bfloat16)
    cfg = ModelConfig.llama2_7b(max_seq=MAX_SEQ, num_layers=layers)
    prog = compile_llama(cfg, tp, batch=1, prompt_len=PROMPT, phases=("decode",))
    hal = NumpyBackend(NumpyBackendConfig(tp, prog.arena_bytes))
    hal.register_plan(prog.plans["decode"])
    for r in range(tp):
        for name, off in prog.dpu_plans[r].weight.items():
            det = prog.graphs["decode"].node(name).meta["spec"].shard_map[r]
            n = int(np.prod(det.local_shape))
            if name.startswith("model.rotary"):
                arr = np.zeros(n, np.float32)
            elif "norm" in name:
                arr = np.ones(n, ml_dtypes.bfloat16)
            else:
                arr = np.resize(block, n)
            hal.copy_to_dpu(r, off, arr)
    dec = prog.plans["decode"]
    execute_plan(dec, hal, tokens=np.array([[1]]), pos=np.array([PROMPT]), timeout=None)
    steps, t0 = 0, time.perf_counter()
    while steps < max_steps and (steps == 0 or time.perf_counter() - t0 < budget_s):
        execute_plan(dec, hal, tokens=np.array([[1]]), pos=np.array([PROMPT + 1 + steps]), timeout=None)
        steps += 1
    sec = (time.perf_counter() - t0) / steps
    hal.close()
    return {"value": round(1.0 / sec, 4), "unit": "tokens/s", "cores": len(os.sched_getaffinity(0)),
            "kind": "port", "steps": steps, "seconds_per_step": round(sec, 3),
            "sample": f"oracle NumPy HAL, {steps} whole decode steps of the {layers}-layer 7B-arch model at "
                      f"TP={tp} (batch 1, positions {PROMPT + 1}..{PROMPT + steps}), {sec:.2f} s per step, "
                      f"after one untimed step"}


def bench_config(n: int, layers: int = 32, allreduce: str = "ordered", combine_add: bool = False,
                 fuse_attention: bool = False, decode_layer: bool = False, decode_step: bool = False) -> dict:
    out = {"workload": "llama2-7b-arch decode, batch 1, prompt 128, positions 128..255 cycled, max_seq 256",
           "tp": n, "layers": layers, "l2": "weights 13.5 GB > L2 (126 MB); no flush needed",
           "parallelism": f"tp{n}", "allreduce": allreduce}
    if combine_add:
        out["combine_add"] = True
    if fuse_attention:
        out["fuse_attention"] = True
    if decode_layer:
        out["decode_layer"] = True
    if decode_step:
        out["decode_step"] = True
    return out


PARITY_LAYERS, PARITY_TOKENS, PARITY_TOL = 2, 8, 2e-2


def _argmax_ties(got, ref, tol):
    """Greedy ids of two logit rows and whether they differ only by a tie at ``tol``
    (the reference logit at ``got``'s id within tol x max |ref| of the reference maximum)."""
    import numpy as np

    g, r = np.asarray(got, np.float32).reshape(-1), np.asarray(ref, np.float32).reshape(-1)
    gi, ri = int(g.argmax()), int(r.argmax())
    return gi, ri, gi != ri and r[gi] >= r[ri] - tol * float(np.abs(r).max())


def bench_parity(n: int, rank: int, dist, hal_kw: dict) -> dict | None:
    """Parity of the timed path at this TP: a 2-layer slice of the benchmarked model (same
    widths, prompt 128, max_seq 256) on a B200 HAL with the bench's own options, decoded the
    way the bench times it (eager prefill, then the captured decode graph replayed through
    ``LlamaRunner``), against the oracle HAL holding byte-identical weights (generated on
    rank 0's GPU by the same per-rank seeds and copied over).

    The oracle decodes greedily first; its 8 tokens are then fed to the B200 path step by
    step (teacher forcing), so both compute every step from the same input.  Returns, on
    rank 0: both sides' greedy ids per step, the relative logit error per step (bound
    2e-2), and the steps whose ids differ only by a tie at that bound; None elsewhere.
    """
    import numpy as np
    import torch

    from backend.hal_cuda import CudaBackend, CudaBackendConfig
    from graph.llama import ModelConfig
    from oracle.hal_numpy import NumpyBackend, NumpyBackendConfig
    from runtime.executor import greedy_generate, read_logits
    from runtime.program import compile_llama
    from runtime.session import LlamaRunner

    cfg = ModelConfig.llama2_7b(max_seq=MAX_SEQ, num_layers=PARITY_LAYERS)
    prog = compile_llama(cfg, n, batch=1, prompt_len=PROMPT)
    prompt = np.random.default_rng(5).integers(0, cfg.vocab_size, (1, PROMPT))
    dec = prog.plans["decode"]
    ref_toks = torch.zeros(PARITY_TOKENS, dtype=torch.int64, device="cuda")
    ref = None
    if rank == 0:
        # the oracle: the same program and per-rank weight bytes, every rank in this process
        src = CudaBackend(CudaBackendConfig(n, prog.arena_bytes))
        LlamaRunner(prog, src).load_random_weights(seed=5)
        ora = NumpyBackend(NumpyBackendConfig(n, prog.arena_bytes))
        for p in prog.plans.values():
            ora.register_plan(p)
        for r, dp in prog.dpu_plans.items():
            ora.copy_to_dpu(r, 0, src.copy_from_dpu(r, 0, (dp.kv_base,), np.uint8))
        src.close()
        ref = greedy_generate(prog.plans["prefill"], dec, ora, prompt, PARITY_TOKENS)
        ora.close()
        ref_toks.copy_(torch.as_tensor(ref.tokens.reshape(-1).astype(np.int64)))
    if dist is not None:
        dist.broadcast(ref_toks, 0)
    fed = [int(t) for t in ref_toks.cpu()]
    # the B200 path, fed the oracle's tokens: prefill, then the step at position 128 (run
    # once while the decode graph is captured), then graph replays through LlamaRunner.step
    hal = CudaBackend(CudaBackendConfig(n, prog.arena_bytes, rank=(rank if n > 1 else None), **hal_kw))
    runner = LlamaRunner(prog, hal)
    runner.load_random_weights(seed=5)
    runner.prefill(prompt)
    logits = [read_logits(prog.plans["prefill"], hal)]
    runner.capture(np.array([fed[0]], np.int32))
    logits.append(read_logits(dec, hal))
    for t in fed[1:PARITY_TOKENS - 1]:
        runner.step(np.array([t], np.int32))
        logits.append(read_logits(dec, hal))
    errors = hal.read_error_flags()
    runner.graph = None
    hal.close()
    out = None
    if rank == 0:
        refs = [ref.prefill_logits] + ref.step_logits
        errs, got_ids, ref_ids, ties = [], [], [], []
        for i, (a, b) in enumerate(zip(logits, refs)):
            a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
            errs.append(round(float(np.abs(a - b).max() / np.abs(b).max()), 6))
            gi, ri, tie = _argmax_ties(a, b, PARITY_TOL)
            got_ids.append(gi)
            ref_ids.append(ri)
            if tie:
                ties.append(i)
        mism = [i for i in range(len(got_ids)) if got_ids[i] != ref_ids[i] and i not in ties]
        out = {"layers": PARITY_LAYERS, "tp": n, "prompt": PROMPT, "tokens": got_ids, "oracle_tokens": ref_ids,
               "tokens_match": got_ids == ref_ids, "tied_steps": ties, "mismatched_steps": mism,
               # a differing id counts as a mismatch unless the oracle's top two logits are equal
               # within `tol` of the largest magnitude there (a tie at the comparison's resolution)
               "tokens_match_outside_ties": not mism,
               "rel_logit_err_per_step": errs, "max_rel_logit_err": max(errs), "tol": PARITY_TOL,
               "within_tol": max(errs) <= PARITY_TOL and not mism,
               "error_words": {str(k): v for k, v in errors.items()},
               "path": "eager prefill + captured decode graph replays (the timed path), bench HAL options; "
                       "the oracle's greedy tokens fed at every step"}
    if dist is not None:
        dist.barrier()
    return out


PREFILL_BATCH, PREFILL_LEN = 8, 2048


def measure_prefill(n: int, rank: int, dist, layers: int, reps: int = 3, allreduce: str = "ordered",
                    split_bytes: int = 0) -> dict:
    """Prefill of 8 x 2048 random ids (causal) at TP=n: tokens/s and the GEMMs' tensor-core roofline.

    The whole prefill plan is timed with CUDA events on the rank stream (max over ranks);
    the GEMM figure times the four projections of layer 0 (qkv + RoPE/KV, o, gate/up +
    SiLU, down), each launched alone, against the burst bf16 peak of MEASURED_PEAKS.json
    (the sustained figure is reported beside it).
    """
    import numpy as np
    import torch

    from backend.hal_cuda import CudaBackend, CudaBackendConfig
    from graph.llama import ModelConfig
    from runtime.executor import execute_plan
    from runtime.program import compile_llama
    from runtime.session import LlamaRunner

    cfg = ModelConfig.llama2_7b(max_seq=PREFILL_LEN, num_layers=layers)
    prog = compile_llama(cfg, n, batch=PREFILL_BATCH, prompt_len=PREFILL_LEN, phases=("prefill",))
    hal = CudaBackend(CudaBackendConfig(n, prog.arena_bytes, rank=(rank if n > 1 else None), allreduce=allreduce,
                                        allreduce_split_bytes=split_bytes))
    runner = LlamaRunner(prog, hal)
    runner.load_random_weights(seed=1)
    ids = np.random.default_rng(1).integers(0, cfg.vocab_size, (PREFILL_BATCH, PREFILL_LEN))
    pf = prog.plans["prefill"]
    zero = np.zeros(PREFILL_BATCH, np.int32)
    st = hal.stream(hal.local[0])
    execute_plan(pf, hal, tokens=ids, pos=zero)  # warm-up
    hal.synchronize()
    if dist is not None:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("prefill_timed")
    e0.record(st)
    for _ in range(reps):
        execute_plan(pf, hal, tokens=ids, pos=zero, sync=False)
    hal.end_run()
    e1.record(st)
    hal.synchronize()
    torch.cuda.nvtx.range_pop()
    ms = e0.elapsed_time(e1) / reps
    if dist is not None:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    # the layer-0 projections, each timed alone (5 launches)
    me = hal.local[0]
    tokens = PREFILL_BATCH * PREFILL_LEN
    h, i = cfg.hidden_size, cfg.intermediate_size
    flops = {"q_rot": 2 * tokens * h * (3 * h) // n, "resid_attn": 2 * tokens * h * h // n,
             "mlp_act": 2 * tokens * h * (2 * i) // n, "resid_mlp": 2 * tokens * i * h // n}
    gemm_ms, gemm_flops, attn_ms = 0.0, 0, None
    for c in pf.commands:
        node = c.payload.get("node", "") if c.op == "launch" else ""
        if c.dpu_id != me or not node.startswith("l0."):
            continue
        fn = hal._lowered[id(c)]
        fn()
        k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        k0.record(st)
        for _ in range(5):
            fn()
        k1.record(st)
        torch.cuda.synchronize()
        t_ms = k0.elapsed_time(k1) / 5
        key = node.split(".", 1)[1]
        if key in flops:
            gemm_ms += t_ms
            gemm_flops += flops[key]
        elif key == "attn":
            attn_ms = t_ms
    peak = _peaks()  # each projection is timed alone: the burst peak applies
    tflops = gemm_flops / (gemm_ms * 1e-3) / 1e12
    runner.graph = None
    hal.close()
    return {"value": round(tokens / (ms * 1e-3), 1), "unit": "tokens/s", "ms_per_step": round(ms, 3),
            "config": {"workload": "llama2-7b-arch prefill, batch 8 x 2048 uniform random ids, causal",
                       "tp": n, "layers": layers, "allreduce": allreduce, "allreduce_split_bytes": split_bytes},
            "gemm": {"bound": "tensor", "achieved": round(tflops, 1), "peak": peak["bf16_tflops"],
                     "peak_kind": f"burst ({peak['src']})", "unit": "TFLOP/s",
                     "frac": round(tflops / peak["bf16_tflops"], 4),
                     "frac_of_sustained": round(tflops / peak["bf16_tflops_sustained"], 4),
                     "kernel": "tcgen05 GEMM + fused epilogue, 4 projections of layer 0, each timed alone",
                     "ms": round(gemm_ms, 3)},
            "attention_ms_per_layer": round(attn_ms, 3) if attn_ms is not None else None}


BATCH_SEQS, BATCH_CTX = 64, 4096
BATCHED_METRIC = "LLaMA2-7B batched decode tokens/s (batch 64, context 4096, TP=N, bf16)"


def run_batched(args) -> None:
    """Batched decode: 64 sequences whose KV blocks hold 4096 N(0, 1) positions, then
    ``--steps`` greedy steps (32 by default) at positions 4096.. -- graph replays timed with
    CUDA events, max over ranks.  Prints its own JSON line (HBM roofline of the step:
    weights + every sequence's keys and values, per rank)."""
    import numpy as np
    import torch

    from backend import _native as nat
    from backend.hal_cuda import CudaBackend, CudaBackendConfig
    from graph.llama import ModelConfig
    from runtime.program import compile_llama
    from runtime.session import LlamaRunner

    n = args.gpus
    rank, dist = _dist_setup(n)
    if n == 1:
        torch.cuda.set_device(0)
    steps, warmup = args.steps, args.warmup
    cfg = ModelConfig.llama2_7b(max_seq=BATCH_CTX + warmup + steps + 8, num_layers=args.layers)
    prog = compile_llama(cfg, n, batch=BATCH_SEQS, prompt_len=16, phases=("decode",))
    hal = CudaBackend(CudaBackendConfig(n, prog.arena_bytes, rank=(rank if n > 1 else None),
                                        allreduce=args.allreduce, allreduce_split_bytes=args.allreduce_split_bytes,
                                        combine_add=args.combine_add, fuse_attention=args.fuse_attention))
    runner = LlamaRunner(prog, hal)
    runner.load_random_weights(seed=3)
    for r in hal.local:  # every KV block of every sequence: N(0, 1) bf16
        dp = prog.dpu_plans[r]
        nat.check(nat.lib.pim_fill_normal(hal.arena_ptr(r) + dp.kv_base, (dp.act_base - dp.kv_base) // 2,
                                          nat.BF16, 1234 + r, 1.0, hal.stream_handle(r)), "fill kv")
    hal.synchronize()
    runner.state.valid_len = BATCH_CTX
    runner.capture(np.random.default_rng(3).integers(0, cfg.vocab_size, BATCH_SEQS).astype(np.int32))
    first = runner.state.valid_len
    positions = (first + torch.arange(warmup + steps, dtype=torch.int32)).repeat_interleave(BATCH_SEQS)
    positions = positions.to(hal.host_device)
    st = hal.capture_stream()
    runner.device_steps(positions, 0, warmup)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        e0.record(st)
        runner.device_steps(positions, warmup, steps)
        e1.record(st)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / steps
    ctx = first + warmup + (steps + 1) / 2.0  # mean keys read per sequence in the timed steps
    step_bytes = cfg.weight_bytes() / n + BATCH_SEQS * 2 * cfg.num_layers * (cfg.num_heads // n) * cfg.head_dim * 2 * ctx
    peaks = _peaks()
    if rank == 0:
        gbs = step_bytes / (ms_step * 1e-3) / 1e9
        print(json.dumps({
            "metric": BATCHED_METRIC, "value": round(BATCH_SEQS * 1000.0 / ms_step, 1), "unit": "tokens/s",
            "n_gpus": n, "steps": steps, "warmup": warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init weights, KV blocks N(0,1), random token ids)",
            "config": {"workload": f"llama2-7b-arch decode, {BATCH_SEQS} sequences at context {BATCH_CTX}",
                       "tp": n, "layers": cfg.num_layers, "allreduce": args.allreduce},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(gbs / peaks["hbm_gbs"], 4), "bytes_per_step_per_rank": int(step_bytes)},
            "gpu_launches": runner.graph.kernels * steps, "clocks": clocks.summary()}), flush=True)
    if dist is not None:
        runner.graph = None
        dist.barrier()
        dist.destroy_process_group()


REDIST_KINDS = ("all_reduce", "all_gather", "all_to_all")
REDIST_TOKENS = (1, 16, 256, 2048)
REDIST_HIDDEN = 4096
REDIST_METRIC = "redistribute bus bandwidth, bf16 [2048, 4096] all_reduce over N ranks (NCCL busbw convention)"
NVLINK_PEER_GBS = 770.0  # measured peer copy per direction on this GPU type (nominal 900)


def redistribute_bus_bytes(entry) -> int:
    """Bus bytes of one edge per rank: all_reduce 2(N-1)/N S, all_gather (N-1)/N S, all_to_all (N-1)/N^2 S."""
    from comm.plan import bus_bytes

    return bus_bytes(entry)


def redistribute_cpu_baseline(n: int, tokens: int = 2048, kind: str = "all_reduce", budget_s: float = 10.0) -> dict:
    """The oracle (host-star lowering of the reference, N ranks simulated in one process) on one edge."""
    import numpy as np

    from oracle.hal_numpy import NumpyBackend, NumpyBackendConfig
    from runtime.exec_plan_gen import redistribute_edge, redistribute_plan
    from runtime.executor import execute_plan

    edge, entry = redistribute_edge(kind, n, (tokens, REDIST_HIDDEN))
    plan = redistribute_plan(edge, entry)
    size = tokens * REDIST_HIDDEN * 2
    hal = NumpyBackend(NumpyBackendConfig(n, 2 * size + 4096))
    hal.register_plan(plan)
    src = np.random.default_rng(0).standard_normal(tokens * REDIST_HIDDEN, dtype=np.float32)
    import ml_dtypes

    src = src.astype(ml_dtypes.bfloat16)
    for s in entry.collect_segments:
        hal.copy_to_dpu(s.src_dpu, s.src_addr, src[:s.nbytes // 2])
    reps, t0 = 0, time.perf_counter()
    while reps < 3 or (time.perf_counter() - t0 < budget_s and reps < 50):
        execute_plan(plan, hal)
        reps += 1
    sec = (time.perf_counter() - t0) / reps
    hal.close()
    return {"value": round(redistribute_bus_bytes(entry) / sec / 1e9, 4), "unit": "GB/s",
            "cores": len(os.sched_getaffinity(0)), "kind": "port",
            "sample": f"oracle NumPy HAL, {kind} of bf16 [{tokens}, {REDIST_HIDDEN}] over {n} simulated ranks, "
                      f"{reps} runs, {sec * 1e3:.2f} ms per edge"}


def _merge_runs(runs):
    """(offset, nbytes) ranges sorted and merged where one ends at the next one's start."""
    out = []
    for a, nb in sorted(runs):
        if out and out[-1][0] + out[-1][1] == a:
            out[-1] = (out[-1][0], out[-1][1] + nb)
        else:
            out.append((a, nb))
    return out


def run_redistribute(args) -> None:
    """Config 5: every redistribute edge of the microbench, each one plan captured in a CUDA
    graph and replayed; per replay a 256 MB buffer is written first (L2 flush) and the replay
    is bracketed by CUDA events on the capture stream (max over ranks).  ``e2e`` adds, every
    step, the copy of the rank's source rows from pinned host memory and the read-back of its
    destination."""
    import numpy as np
    import torch

    from backend import _native as nat
    from backend.hal_cuda import CudaBackend, CudaBackendConfig
    from comm.plan import NvlinkCostModel, plan_cost
    from runtime.exec_plan_gen import redistribute_edge, redistribute_plan

    n = args.gpus
    if n < 2:
        print(json.dumps({"metric": REDIST_METRIC, "impl": "b200",
                          "unavailable": "the redistribute microbench needs N >= 2 ranks, one per GPU"}), flush=True)
        return
    rank, dist = _dist_setup(n, timeout_s=600)  # captured graphs hold NCCL work for the whole run
    steps, warmup = args.steps, max(args.warmup, 3)
    size_max = max(REDIST_TOKENS) * REDIST_HIDDEN * 2
    hal = CudaBackend(CudaBackendConfig(n, 2 * size_max + 4096, rank=rank, allreduce=args.allreduce,
                                        allreduce_split_bytes=args.allreduce_split_bytes))
    me = hal.local[0]
    st = hal.capture_stream()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=hal.host_device)
    arena = hal.arena(me)
    cases, head = [], None
    with ClockSampler(torch.cuda.current_device()) as clocks:
        for kind in REDIST_KINDS:
            for t in REDIST_TOKENS:
                if kind == "all_to_all" and t % n:
                    cases.append({"kind": kind, "tokens": t, "n/a": f"Shard(0) of T={t} over {n} ranks is "
                                                                     "undefined in the reference (not divisible)"})
                    continue
                torch.cuda.synchronize()
                dist.barrier()  # every rank enters each case together
                print(f"[rank {rank}] redistribute case {kind} T={t}", file=sys.stderr, flush=True)
                edge, entry = redistribute_edge(kind, n, (t, REDIST_HIDDEN))
                plan = redistribute_plan(edge, entry)
                hal.register_plan(plan)
                src = [s for s in entry.collect_segments if s.src_dpu == me]
                dst = [s for s in entry.writeback_segments if s.dst_dpu == me]
                src_bytes, dst_bytes = sum(s.nbytes for s in src), sum(s.nbytes for s in dst)
                for s in src:
                    nat.check(nat.lib.pim_fill_normal(hal.arena_ptr(me) + s.src_addr, s.nbytes // 2, nat.BF16,
                                                      17 + me, 1.0, hal.stream_handle(me)), "fill")
                # the host copies of e2e: one per run of adjacent arena bytes (a Shard(last) source
                # is T segments of one row each, back to back in the arena)
                src_runs = _merge_runs([(s.src_addr, s.nbytes) for s in src])
                dst_runs = _merge_runs([(s.dst_addr, s.nbytes) for s in dst])
                hal.synchronize()
                dist.barrier()
                g = hal.capture(plan)
                torch.cuda.synchronize()
                pin_src = torch.empty(src_bytes, dtype=torch.uint8, pin_memory=True)
                pin_dst = torch.empty(dst_bytes, dtype=torch.uint8, pin_memory=True)
                off = 0
                for a, nb in src_runs:
                    pin_src[off:off + nb].copy_(arena[a:a + nb])
                    off += nb

                def timed(e2e: bool) -> float:
                    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                          for _ in range(steps)]
                    for i in range(warmup + steps):
                        with torch.cuda.stream(st):
                            flush.zero_()
                            if i >= warmup:
                                ev[i - warmup][0].record(st)
                            if e2e:
                                off = 0
                                for a, nb in src_runs:
                                    arena[a:a + nb].copy_(pin_src[off:off + nb], non_blocking=True)
                                    off += nb
                            g.replay()  # on the capture stream, between the events
                            if e2e:
                                off = 0
                                for a, nb in dst_runs:
                                    pin_dst[off:off + nb].copy_(arena[a:a + nb], non_blocking=True)
                                    off += nb
                            if i >= warmup:
                                ev[i - warmup][1].record(st)
                    torch.cuda.synchronize()
                    ms = sum(a.elapsed_time(b) for a, b in ev) / steps
                    tt = torch.tensor([ms], device="cuda")
                    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
                    return float(tt.item())

                dist.barrier()
                ms = timed(False)
                ms_e2e = timed(True)
                bus = redistribute_bus_bytes(entry)
                case = {"kind": kind, "tokens": t, "bytes": t * REDIST_HIDDEN * 2, "bus_bytes_per_rank": bus,
                        "us": round(ms * 1e3, 2), "busbw_gbs": round(bus / (ms * 1e-3) / 1e9, 2),
                        "e2e_us": round(ms_e2e * 1e3, 2), "h2d_bytes_per_step": src_bytes,
                        "d2h_bytes_per_step": dst_bytes, "launches_per_step": g.kernels,
                        "host_copies_per_step": len(src_runs) + len(dst_runs),
                        "model_us": round(plan_cost(entry, NvlinkCostModel()).seconds * 1e6, 2)}
                cases.append(case)
                if rank == 0:  # each case as soon as it is measured (the summary line follows at the end)
                    print(json.dumps({"redistribute_case": case, "n_gpus": n}), file=sys.stderr, flush=True)
                if kind == "all_reduce" and t == max(REDIST_TOKENS):
                    head = case
                del g
                torch.cuda.synchronize()
                hal.release_plan(plan)
    peaks_bw = NVLINK_PEER_GBS
    if rank == 0:
        line = {
            "metric": REDIST_METRIC, "value": head["busbw_gbs"], "unit": "GB/s", "n_gpus": n, "steps": steps,
            "warmup": warmup, "ms_per_step": round(head["us"] / 1e3, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (N(0,1) bf16 sources)",
            "config": {"workload": f"redistribute microbench: {', '.join(REDIST_KINDS)} of bf16 [T, {REDIST_HIDDEN}], "
                                   f"T in {list(REDIST_TOKENS)}", "ranks": n, "allreduce": args.allreduce,
                       "allreduce_split_bytes": args.allreduce_split_bytes,
                       "l2": "256 MB written between timed replays"},
            "e2e": {"value": round(head["bus_bytes_per_rank"] / (head["e2e_us"] * 1e-6) / 1e9, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": head["h2d_bytes_per_step"],
                    "d2h_bytes_per_step": head["d2h_bytes_per_step"]},
            "roofline": {"bound": "nvlink", "achieved": head["busbw_gbs"], "peak": peaks_bw, "unit": "GB/s",
                         "frac": round(head["busbw_gbs"] / peaks_bw, 4), "traffic": None,
                         "peak_src": "measured peer copy per direction"},
            "gpu_launches": head["launches_per_step"] * steps, "cases": cases, "clocks": clocks.summary()}
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = redistribute_cpu_baseline(n)
        print(json.dumps(line), flush=True)
    dist.barrier()
    hal.close()
    dist.destroy_process_group()


AB_DECODE = {"default": {}, "dynamic_gemv": {"projection_kernel": 3}, "fuse_attention": {"fuse_attention": True},
             "dynamic_gemv+fuse_attention": {"projection_kernel": 3, "fuse_attention": True},
             "decode_layer": {"decode_layer": True}, "decode_step": {"decode_layer": True, "decode_step": True}}
AB_PREFILL = {"default": {}, "persistent_gemm": {"row_batch_kernel": 1}, "tcgen05_attention": {"prefill_attention": 1},
              "persistent_gemm+tcgen05_attention": {"row_batch_kernel": 1, "prefill_attention": 1}}


def run_ab(args) -> None:
    """One GPU: the default kernels and each opt-in variant back to back in one process --
    decode ms per step (graph replays, CUDA events) and the 8 x 2048 prefill time, plus
    whether each variant's greedy tokens equal the default's.  Prints one JSON line."""
    import numpy as np
    import torch

    from backend import _native as nat
    from backend.hal_cuda import CudaBackend, CudaBackendConfig
    from graph.llama import ModelConfig
    from runtime.executor import execute_plan, read_tokens
    from runtime.program import compile_llama
    from runtime.session import LlamaRunner

    torch.cuda.set_device(0)
    lib = nat.lib
    saved = (lib.pim_projection_kernel(), lib.pim_row_batch_kernel(), lib.pim_prefill_attention_kernel())

    def select(v):
        nat.check(lib.pim_set_projection_kernel(v.get("projection_kernel", saved[0])), "projection kernel")
        nat.check(lib.pim_set_row_batch_kernel(v.get("row_batch_kernel", saved[1])), "row-batch kernel")
        nat.check(lib.pim_set_prefill_attention_kernel(v.get("prefill_attention", saved[2])), "attention kernel")

    cfg = ModelConfig.llama2_7b(max_seq=MAX_SEQ, num_layers=args.layers)
    prog = compile_llama(cfg, 1, batch=1, prompt_len=PROMPT, phases=("prefill", "decode"))
    prompt = np.random.default_rng(0).integers(0, cfg.vocab_size, (1, PROMPT))
    out = {"decode": {}, "prefill": {}}
    ref_tokens = None

    def guarded(section, name, fn):
        """One variant; an error is recorded in its entry and the next variant runs."""
        try:
            fn()
        except Exception as e:  # noqa: BLE001 -- reported in the JSON line
            out[section][name] = {"error": f"{type(e).__name__}: {e}"[:400]}
        finally:
            torch.cuda.empty_cache()

    def decode_variant(name, v):
        select(v)
        hal = CudaBackend(CudaBackendConfig(1, prog.arena_bytes, fuse_attention=v.get("fuse_attention", False),
                                            decode_layer=v.get("decode_layer", False),
                                            decode_step=v.get("decode_step", False)))
        try:
            decode_run(name, hal)
        finally:
            hal.close()

    def decode_run(name, hal):
        nonlocal ref_tokens
        runner = LlamaRunner(prog, hal)
        runner.load_random_weights(seed=0)
        tok = runner.prefill(prompt)
        runner.capture(tok)
        start = runner.state.valid_len
        total = args.warmup + args.steps
        positions = (start + torch.arange(total, dtype=torch.int32) % (MAX_SEQ - start)).to(hal.host_device)
        runner.device_steps(positions, 0, args.warmup)
        torch.cuda.synchronize()
        st = hal.capture_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        runner.device_steps(positions, args.warmup, args.steps)
        e1.record(st)
        torch.cuda.synchronize()
        # greedy tokens of 8 steps from the prompt, for the comparison with the default
        runner.state.valid_len = start
        toks = [int(tok[0])]
        t = np.asarray(tok, np.int32)
        for _ in range(8):
            t = runner.step(t)
            toks.append(int(t[0]))
        if ref_tokens is None:
            ref_tokens = toks
        out["decode"][name] = {"ms_per_step": round(e0.elapsed_time(e1) / args.steps, 4),
                               "kernels_per_step": runner.graph.kernels, "tokens_match_default": toks == ref_tokens,
                               "errors": hal.read_error_flags()}
        runner.graph = None

    for name, v in AB_DECODE.items():
        guarded("decode", name, lambda: decode_variant(name, v))
    pcfg = ModelConfig.llama2_7b(max_seq=PREFILL_LEN, num_layers=args.layers)
    pprog = compile_llama(pcfg, 1, batch=PREFILL_BATCH, prompt_len=PREFILL_LEN, phases=("prefill",))
    ids = np.random.default_rng(1).integers(0, pcfg.vocab_size, (PREFILL_BATCH, PREFILL_LEN))
    zero = np.zeros(PREFILL_BATCH, np.int32)
    ref_tokens = None

    def prefill_variant(name, v):
        select(v)
        hal = CudaBackend(CudaBackendConfig(1, pprog.arena_bytes))
        try:
            prefill_run(name, hal)
        finally:
            hal.close()

    def prefill_run(name, hal):
        nonlocal ref_tokens
        runner = LlamaRunner(pprog, hal)
        runner.load_random_weights(seed=1)
        pf = pprog.plans["prefill"]
        execute_plan(pf, hal, tokens=ids, pos=zero)
        toks = read_tokens(pf, hal).reshape(-1).tolist()
        st = hal.stream(0)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(3):
            execute_plan(pf, hal, tokens=ids, pos=zero, sync=False)
        hal.end_run()
        e1.record(st)
        hal.synchronize()
        if ref_tokens is None:
            ref_tokens = toks
        ms = e0.elapsed_time(e1) / 3
        out["prefill"][name] = {"ms": round(ms, 3), "tokens_per_s": round(PREFILL_BATCH * PREFILL_LEN / (ms * 1e-3), 1),
                                "tokens_match_default": toks == ref_tokens,
                                "attention_errors": int(lib.pim_attention_errors(1))}

    for name, v in AB_PREFILL.items():
        guarded("prefill", name, lambda: prefill_variant(name, v))
    select({})
    print(json.dumps({"metric": "opt-in kernel A/B (LLaMA2-7B arch, TP=1)", "n_gpus": 1, "steps": args.steps,
                      "warmup": args.warmup, "layers": args.layers, "ab": out}), flush=True)


def run_reference(args) -> None:
    """The reference arm: the oracle's restatement of the reference runtime (NumpyBackend over the
    ExecutionPlan, NumPy kernels; the reference's own runtime files are empty) on this host's
    cores, timing whole 32-layer decode steps of the same workload at TP = N simulated ranks.
    One untimed step, then up to ``--steps`` steps within about a minute; ``steps`` on the line
    is the number actually timed.  Under torchrun only rank 0 runs it."""
    n = args.gpus
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cb = cpu_baseline(n, budget_s=60.0, layers=args.layers, max_steps=max(1, args.steps))
    tok_s = cb["value"]
    line = {"metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": n, "steps": cb["steps"],
            "steps_requested": args.steps, "warmup": 1, "ms_per_step": round(1000.0 / tok_s, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic", "config": bench_config(n, args.layers), "impl": "reference", "cpu_baseline": cb,
            "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="skip the 8 x 2048 prefill measurement")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the parity check of the timed path (2-layer slice vs the oracle)")
    ap.add_argument("--allreduce", default="p2p", choices=["ordered", "p2p", "fused", "nccl"],
                    help="Partial->Replicate path at N > 1 (CudaBackendConfig.allreduce); default p2p, the "
                         "low-latency NVLink protocol for edges that fit its rows, NCCL + rank-order sum above")
    ap.add_argument("--allreduce-split-bytes", type=int, default=None,
                    help="all_reduce edges of at least this size as all_to_all + slice sums + all_gather "
                         "(CudaBackendConfig.allreduce_split_bytes; 0: never; default 8 MiB at N >= 4, where "
                         "it moves 2(N-1)/N of a prefill edge per rank instead of N-1 partials, else 0)")
    ap.add_argument("--combine-add", action=argparse.BooleanOptionalAction, default=True,
                    help="fold the residual add into each ordered / p2p all_reduce combine "
                         "(CudaBackendConfig.combine_add; default on)")
    ap.add_argument("--ab", action="store_true",
                    help="one GPU: default kernels vs each opt-in variant, decode and prefill, one JSON line")
    ap.add_argument("--fuse-attention", action="store_true",
                    help="decode attention inside each attn_in launch (CudaBackendConfig.fuse_attention)")
    ap.add_argument("--decode-layer", action="store_true",
                    help="each decode layer as one launch (CudaBackendConfig.decode_layer): at N=1, or at N>1 "
                         "with --allreduce fused")
    ap.add_argument("--decode-step", action="store_true",
                    help="the whole decode step as one launch (CudaBackendConfig.decode_step; implies --decode-layer)")
    ap.add_argument("--batched", action="store_true",
                    help=f"batched decode instead: {BATCH_SEQS} sequences at context {BATCH_CTX}, 32 steps by default")
    ap.add_argument("--redistribute", action="store_true",
                    help="the redistribute microbench instead (all_reduce / all_gather / all_to_all of bf16 "
                         "[T, 4096], T in 1, 16, 256, 2048; N >= 2), 100 steps by default")
    args = ap.parse_args()
    if args.allreduce_split_bytes is None:
        args.allreduce_split_bytes = SPLIT_BYTES_DEFAULT if args.gpus >= 4 else 0
    if args.impl == "reference":
        return run_reference(args)
    if args.redistribute:
        if "--steps" not in sys.argv:
            args.steps = 100
        return run_redistribute(args)
    if args.ab:
        if "--steps" not in sys.argv:
            args.steps = 128
        return run_ab(args)
    if args.batched:
        if "--steps" not in sys.argv:
            args.steps = 32
        return run_batched(args)

    import numpy as np
    import torch

    from backend import _native as nat
    from backend.hal_cuda import CudaBackend, CudaBackendConfig
    from graph.llama import ModelConfig
    from runtime.program import compile_llama
    from runtime.session import LlamaRunner

    n = args.gpus
    rank, dist = _dist_setup(n)
    if n == 1:
        torch.cuda.set_device(0)
    cfg = ModelConfig.llama2_7b(max_seq=MAX_SEQ, num_layers=args.layers)
    prog = compile_llama(cfg, n, batch=1, prompt_len=PROMPT)
    hal_kw = dict(allreduce=args.allreduce, allreduce_split_bytes=args.allreduce_split_bytes,
                  combine_add=args.combine_add, fuse_attention=args.fuse_attention,
                  decode_layer=args.decode_layer or args.decode_step, decode_step=args.decode_step)
    hal = CudaBackend(CudaBackendConfig(n, prog.arena_bytes, rank=(rank if n > 1 else None), **hal_kw))
    runner = LlamaRunner(prog, hal)
    runner.load_random_weights(seed=0)
    prompt = np.random.default_rng(0).integers(0, cfg.vocab_size, (1, PROMPT))
    tok = runner.prefill(prompt)
    runner.capture(tok)  # executes the step at position 128 once while capturing
    total = args.warmup + args.steps
    start_pos = runner.state.valid_len
    span = MAX_SEQ - start_pos  # steps cycle through positions start_pos .. MAX_SEQ - 1
    positions = (start_pos + torch.arange(total, dtype=torch.int32) % span).to(hal.host_device)
    st = hal.capture_stream()  # graph replays run on the first rank's stream

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    runner.device_steps(positions, 0, args.warmup)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        torch.cuda.nvtx.range_push("decode_timed")
        e0.record(st)
        runner.device_steps(positions, args.warmup, args.steps)
        e1.record(st)
        barrier()
        torch.cuda.nvtx.range_pop()
    ms = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    launches_per_step = runner.graph.kernels  # library kernels recorded in the decode graph

    # e2e: the public runner API with host I/O every step
    runner.state.valid_len = start_pos  # positions are rewritten before they are read again
    tok = np.zeros(1, np.int32)
    e2e_steps = args.steps
    barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        if runner.state.valid_len >= MAX_SEQ:
            runner.state.valid_len = start_pos
        tok = runner.step(tok)
    barrier()
    e2e_s = (time.perf_counter() - t0) / max(e2e_steps, 1)
    if dist is not None:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())

    # roofline of the dominant kernel: the gate/up projection (rmsnorm + GEMV + SiLU*up),
    # launched for layers 0, 1, ..., L-1 in turn so that no launch finds its weights in L2
    # (per-rank gate/up weights are 22-180 MB at TP 8-1; all layers' together >= 720 MB)
    me = hal.local[0]
    cmds = [c for c in prog.plans["decode"].commands
            if c.op == "launch" and c.dpu_id == me and str(c.payload.get("node", "")).endswith(".mlp_act")]
    roof_kernel = "fused rmsnorm+gate/up GEMV+SiLU*up, every layer in turn"
    if args.decode_layer or args.decode_step:  # the step runs it inside the layer kernel: time it alone
        from backend.cuda_kernels import lower_launch

        fns = [lower_launch(hal, me, c) for c in cmds]
        roof_kernel += ", launched alone (the timed steps run it inside the layer kernel)"
    else:
        fns = [hal._lowered[id(c)] for c in cmds]
    w_bytes = int(np.prod(cmds[0].payload["inputs"][2][1])) * 2
    act_bytes = cfg.hidden_size * 2 * 2 + cfg.intermediate_size // n * 2
    ks = hal.stream(me)
    for f in fns:
        f()
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cycles = max(1, 64 // len(fns))
    k0.record(ks)
    for _ in range(cycles):
        for f in fns:
            f()
    k1.record(ks)
    torch.cuda.synchronize()
    kern_ms = k0.elapsed_time(k1) / (cycles * len(fns))
    peaks = _peaks()
    achieved = (w_bytes + act_bytes) / (kern_ms * 1e-3) / 1e9
    kv_len = float((positions[args.warmup:].double() + 1).mean())  # mean keys read per timed step
    step_bytes = cfg.weight_bytes() // n + cfg.hidden_size * 2 + 2 * cfg.num_layers * kv_len * \
        cfg.num_heads // n * cfg.head_dim * 2

    prefill = None if args.no_prefill else measure_prefill(n, rank, dist, args.layers, allreduce=args.allreduce,
                                                           split_bytes=args.allreduce_split_bytes)
    parity = None if args.no_parity else bench_parity(n, rank, dist, hal_kw)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(1000.0 / ms_step, 3), "unit": "tokens/s", "n_gpus": n,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init bf16 N(0,0.02) weights, uniform random prompt ids)",
            "config": bench_config(n, cfg.num_layers, args.allreduce, args.combine_add, args.fuse_attention,
                                   args.decode_layer or args.decode_step, args.decode_step),
            "e2e": {"value": round(1.0 / e2e_s, 3), "unit": "tokens/s", "h2d_bytes_per_step": 8,
                    "d2h_bytes_per_step": 4},
            "roofline": {"bound": "hbm", "kernel": roof_kernel,
                         "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": _profiled_traffic(n),
                         "peak_src": peaks["src"], "kernel_ms": round(kern_ms, 4),
                         "algorithmic_bytes_per_launch": w_bytes + act_bytes,
                         "l2": f"{len(fns)} layers' weights cycled ({len(fns) * w_bytes / 1e6:.0f} MB "
                               f"{'>' if len(fns) * w_bytes > 126e6 else '<'} L2 126 MB)",
                         "step_achieved_gbs": round(step_bytes / (ms_step * 1e-3) / 1e9, 1),
                         "step_frac": round(step_bytes / (ms_step * 1e-3) / 1e9 / peaks["hbm_gbs"], 4)},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks.summary(),
        }
        coop = nat.lib.pim_cooperative_pdl(torch.cuda.current_device())
        if coop >= 0:  # kernels with grid-wide waits ran: whether their cooperative launch kept PDL
            line["config"]["cooperative_launch_with_pdl"] = bool(coop)
        if prefill is not None:
            line["prefill"] = prefill
        if parity is not None:
            line["parity"] = parity
        if not args.no_cpu_baseline and n == 1:  # the CPU baseline is taken at N=1 only
            line["cpu_baseline"] = cpu_baseline(n)
        print(json.dumps(line), flush=True)
    if dist is not None:
        runner.graph = None
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
