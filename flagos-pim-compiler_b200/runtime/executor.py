"""Runtime interpreter for ExecutionPlans and the greedy decode loop.

Implements the runtime the reference specifies but leaves empty
(runtime/executor.py is 0 bytes; design in docs/spec.md:1537-1597):

* ``execute_plan`` submits commands in plan order.  Dependencies are the
  commands' ``waits``.  A HAL that resolves waits on the device (the B200 HAL
  turns them into stream-event waits) is given the commands back to back; a
  HAL that snapshots host payloads at submit time (the NumPy HAL's ``dma_in``,
  backend/hal_numpy.py:115) first gets a host-side ``wait`` on every
  predecessor, exactly as in docs/spec.md:1540-1544;
* ``DecodeState.valid_len`` is the single source of truth for the position
  (docs/spec.md:1381, 1549-1563): prefill writes KV[0..P-1], logits are taken
  at P-1, then each decode step writes KV[pos] and advances by one;
* waits carry a timeout and raise ``HALTimeout`` naming the command
  (docs/spec.md:1578-1597).
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field

import numpy as np

from contracts.exec_plan import ExecutionPlan


class HALTimeout(RuntimeError):
    """A wait ran out; the message names the command (rank, kernel, addresses)."""


def describe(cmd) -> str:
    p = cmd.payload
    what = p.get("kernel") or p.get("kind") or p.get("role") or cmd.op
    where = f"dpu{cmd.dpu_id}" if cmd.dpu_id is not None else "host"
    extra = ""
    if cmd.op in ("dma_in", "dma_out"):
        extra = f" offset={p.get('offset')} edge={p.get('edge')}"
    return f"command {cmd.id} ({cmd.op} {what} on {where}{extra})"


@dataclass
class PlanRun:
    plan: ExecutionPlan
    hal: object
    events: dict[int, object] = field(default_factory=dict)

    def result(self, cmd_id: int, timeout: float | None = None):
        return self.hal.wait(self.events[cmd_id], timeout=timeout)

    def wait_all(self, timeout: float | None = None) -> None:
        by_id = {c.id: c for c in self.plan.commands}
        sync = getattr(self.hal, "synchronize", None)
        if callable(sync):
            sync()  # one device-wide wait; the per-event waits below then only surface errors
        for cid, ev in self.events.items():
            try:
                self.hal.wait(ev, timeout=timeout)
            except TimeoutError as exc:
                raise HALTimeout(describe(by_id[cid])) from exc


def bind_inputs(plan: ExecutionPlan, hal, tokens=None, pos=None) -> None:
    ins = plan.meta["inputs"]
    if tokens is not None:
        ref = ins["input_ids"]
        arr = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32).reshape(ref.shape))
        hal.write_host(plan, ref.offset, arr)
    if pos is not None:
        ref = ins["positions"]
        arr = np.ascontiguousarray(np.broadcast_to(np.asarray(pos, dtype=np.int32), ref.shape))
        hal.write_host(plan, ref.offset, arr)


def execute_plan(plan: ExecutionPlan, hal, *, tokens=None, pos=None, timeout: float | None = 60.0,
                 sync: bool = True) -> PlanRun:
    """Run ``plan`` once on ``hal``; ``tokens``/``pos`` are bound to the plan's host inputs."""
    hal.begin_run(plan)
    run = PlanRun(plan, hal)
    plan.meta["run"] = run
    bind_inputs(plan, hal, tokens, pos)
    device_waits = bool(getattr(hal, "device_side_waits", False))
    for cmd in plan.commands:
        if not device_waits:
            for w in cmd.waits:
                try:
                    hal.wait(run.events[w], timeout=timeout)
                except TimeoutError as exc:
                    raise HALTimeout(describe(plan.commands[w])) from exc
        run.events[cmd.id] = hal.submit(cmd)
    if sync:
        run.wait_all(timeout)
    return run


def read_logits(plan: ExecutionPlan, hal) -> np.ndarray:
    ref = plan.meta["outputs"]["logits"]
    return hal.read_host(plan, ref.offset, ref.shape, ref.dtype)


def read_tokens(plan: ExecutionPlan, hal) -> np.ndarray:
    ref = plan.meta["outputs"]["token"]
    return hal.read_host(plan, ref.offset, ref.shape, "int32")


@dataclass
class DecodeState:
    valid_len: int = 0

    def commit_one_position(self) -> None:
        self.valid_len += 1


@dataclass
class GenerateResult:
    tokens: np.ndarray  # [batch, steps]
    prefill_logits: np.ndarray
    step_logits: list[np.ndarray]
    seconds: float


def greedy_generate(prefill_plan: ExecutionPlan, decode_plan: ExecutionPlan, hal, prompt, steps: int,
                    eos: int | None = None, keep_logits: bool = True) -> GenerateResult:
    """Prefill ``prompt`` ([batch, P] ids), then ``steps`` greedy decode steps.

    The prefill plan's argmax gives the first generated token; every decode
    step writes KV at ``state.valid_len`` and samples the next token.
    """
    prompt = np.asarray(prompt, dtype=np.int32)
    if prompt.ndim == 1:
        prompt = prompt[None]
    b, p = prompt.shape
    state = DecodeState(0)
    t0 = time.perf_counter()
    execute_plan(prefill_plan, hal, tokens=prompt, pos=np.zeros(b, np.int32))
    state.valid_len = p
    prefill_logits = read_logits(prefill_plan, hal)
    token = read_tokens(prefill_plan, hal)
    out = [token.copy()]
    step_logits = []
    for _ in range(steps - 1 if steps > 0 else 0):
        execute_plan(decode_plan, hal, tokens=token.reshape(b, 1), pos=np.full(b, state.valid_len, np.int32))
        state.commit_one_position()
        if keep_logits:
            step_logits.append(read_logits(decode_plan, hal))
        token = read_tokens(decode_plan, hal)
        out.append(token.copy())
        if eos is not None and np.all(token == eos):
            break
    return GenerateResult(np.stack(out, axis=1), prefill_logits, step_logits, time.perf_counter() - t0)
