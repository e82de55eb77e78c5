"""Serving-style front end over compiled plans: prefill once, then graph-replayed decode steps.

``LlamaRunner`` is the public entry a user calls: it owns the program, the
HAL, the weights and the captured decode graph, and follows the spec's decode
loop (docs/spec.md:1549-1563) with ``DecodeState.valid_len`` as the position:

    runner = LlamaRunner(prog, hal)
    runner.load_random_weights(seed)        # or runner.load_checkpoint(hf_dir)
    tok = runner.prefill(prompt)            # writes KV[0..P-1], returns argmax at P-1
    for _ in range(n):
        tok = runner.step(tok)              # writes KV[pos], returns the next token

Each ``step`` copies the step's token and position from pinned host memory,
replays the captured decode plan, and reads the sampled token back.
``device_steps`` runs steps entirely on the device (the sampled token feeds the
next step on device; positions come from a device array), for timing.
"""

from __future__ import annotations

import hashlib

import numpy as np

from graph.llama import SPEC_META_KEY, weight_names, weight_shape
from runtime.executor import DecodeState, execute_plan, read_tokens
from runtime.program import LlamaProgram, rotary_tables


class LlamaRunner:
    def __init__(self, prog: LlamaProgram, hal) -> None:
        import torch

        self.prog, self.hal, self.torch = prog, hal, torch
        for p in prog.plans.values():
            hal.register_plan(p)
        self.state = DecodeState(0)
        self.graph = None
        if "decode" not in prog.plans:  # a prefill-only program: no step I/O buffers
            return
        dec = prog.plans["decode"]
        b = prog.batch
        self._pin_tok = torch.zeros(b, dtype=torch.int32, pin_memory=True)
        self._pin_pos = torch.zeros(b, dtype=torch.int32, pin_memory=True)
        self._pin_out = torch.zeros(b, dtype=torch.int32, pin_memory=True)
        host = hal.host_tensor(dec)
        ins, outs = dec.meta["inputs"], dec.meta["outputs"]
        self._ids = host[ins["input_ids"].offset:ins["input_ids"].offset + 4 * b].view(torch.int32)
        self._pos = host[ins["positions"].offset:ins["positions"].offset + 4 * b].view(torch.int32)
        self._tok = host[outs["token"].offset:outs["token"].offset + 4 * b].view(torch.int32)

    # -- weights --------------------------------------------------------------
    def load_random_weights(self, seed: int = 0, std: float = 0.02) -> None:
        """Random-init weights generated on the device: N(0, std^2) matrices, unit norms, HF rotary tables."""
        from backend import _native as nat

        prog, hal = self.prog, self.hal
        cos, sin = rotary_tables(prog.cfg)
        g = next(iter(prog.graphs.values()))
        for name in weight_names(prog.cfg):
            spec = g.node(name).meta[SPEC_META_KEY]
            _, dt = weight_shape(prog.cfg, name)
            for r, det in spec.shard_map.items():
                if r not in hal.local:
                    continue
                off = prog.dpu_plans[r].weight[name]
                n = int(np.prod(det.local_shape))
                if name.startswith("model.rotary."):
                    hal.copy_to_dpu(r, off, cos if name.endswith("cos") else sin)
                    continue
                ptr, st = hal.arena_ptr(r) + off, hal.stream_handle(r)
                if name.endswith("norm.weight"):
                    nat.check(nat.lib.pim_fill_const(ptr, n, nat.DTYPE_CODE[dt], 1.0, st), "fill")
                else:
                    h = int.from_bytes(hashlib.sha256(f"{seed}/{name}/{r}".encode()).digest()[:8], "little")
                    nat.check(nat.lib.pim_fill_normal(ptr, n, nat.DTYPE_CODE[dt], h, std, st), "fill")
        hal.synchronize()

    def load_checkpoint(self, path) -> None:
        """Weights of an HF LLaMA safetensors checkpoint (directory or file), streamed
        into the arenas one decoder layer at a time."""
        from runtime.checkpoint import state_dict
        from runtime.program import load_state_dict

        load_state_dict(self.prog, self.hal, state_dict(path, self.prog.cfg.dtype))
        self.hal.synchronize()

    # -- steps ------------------------------------------------------------------
    def prefill(self, prompt) -> np.ndarray:
        prompt = np.asarray(prompt, dtype=np.int32).reshape(self.prog.batch, -1)
        pf = self.prog.plans["prefill"]
        execute_plan(pf, self.hal, tokens=prompt, pos=np.zeros(self.prog.batch, np.int32))
        self.state.valid_len = prompt.shape[1]
        return read_tokens(pf, self.hal)

    def capture(self, token) -> None:
        """Capture the decode plan (its warm-up executes the step at the current position)."""
        from runtime.executor import bind_inputs

        dec = self.prog.plans["decode"]
        bind_inputs(dec, self.hal, tokens=np.asarray(token).reshape(self.prog.batch, 1),
                    pos=np.full(self.prog.batch, self.state.valid_len, np.int32))
        self.graph = self.hal.capture(dec)
        self.state.commit_one_position()

    def step(self, token) -> np.ndarray:
        """One decode step through pinned host I/O: H2D token+position, replay, D2H next token."""
        torch = self.torch
        if self.state.valid_len >= self.prog.cfg.max_seq:
            raise ValueError(f"position {self.state.valid_len} is past max_seq={self.prog.cfg.max_seq}")
        st = self.hal.capture_stream()  # the stream graph replays run on
        self._pin_tok.copy_(torch.as_tensor(np.asarray(token, dtype=np.int32).reshape(-1)))
        self._pin_pos.fill_(self.state.valid_len)
        with torch.cuda.stream(st):
            self._ids.copy_(self._pin_tok, non_blocking=True)
            self._pos.copy_(self._pin_pos, non_blocking=True)
            self.graph.replay()
            self._pin_out.copy_(self._tok, non_blocking=True)
        st.synchronize()
        self.state.commit_one_position()
        return self._pin_out.numpy().copy()

    def device_steps(self, positions_dev, start: int, count: int) -> None:
        """Enqueue ``count`` decode steps with positions taken from a device int32 array."""
        torch = self.torch
        st = self.hal.capture_stream()  # the stream graph replays run on
        b = self.prog.batch
        with torch.cuda.stream(st):
            for k in range(start, start + count):
                self._pos.copy_(positions_dev[k * b:(k + 1) * b], non_blocking=True)
                self.graph.replay()
