"""NumPy HAL (oracle): restatement of the reference NumpyBackend.

Follows backend/hal_numpy.py:12-189 and the byte model of
backend/dpu_sdk.py:44-191:

* each DPU owns an isolated zero-initialised byte array (its MRAM);
* ``submit`` runs commands on a thread pool; commands of one DPU form a serial
  stream (tail future, hal_numpy.py:156-175); ``waits`` are futures that must
  resolve first (hal_numpy.py:147-154);
* ``launch`` calls the registered kernel ``fn(hal, dpu_id, cmd)``;
  ``dma_in`` copies host -> DPU and snapshots its data at submit time;
  ``dma_out`` copies DPU -> host and returns the array; host commands run
  ``payload["fn"](cmd)`` (hal_numpy.py:104-145, 177-183);
* out-of-range accesses raise ``ValueError("invalid MRAM range ...")``;
  duplicate / unknown command ids raise ``ValueError``; errors surface at
  ``wait``; device-to-device copies are refused.

Additions needed to run whole plans repeatedly (not in the reference class):
``register_plan`` binds the oracle implementation of every host command of a
compiled plan and gives the plan a host byte arena (``write_host`` /
``read_host``); ``begin_run`` drains outstanding work and clears the command-id
table so the same plan can execute again; ``dma_in`` / ``dma_out`` commands
that carry ``host_offset`` move bytes between a DPU and the plan's host arena.
"""

from __future__ import annotations

from concurrent.futures import Future, ThreadPoolExecutor
from dataclasses import dataclass
from threading import Lock
from typing import Callable, Literal

import numpy as np


def np_dtype(name) -> np.dtype:
    if isinstance(name, np.dtype):
        return name
    if str(name) == "bfloat16":
        import ml_dtypes

        return np.dtype(ml_dtypes.bfloat16)
    return np.dtype(name)


@dataclass
class NumpyBackendConfig:
    num_dpus: int
    mram_bytes_per_dpu: int
    allow_device_to_device: bool = False


@dataclass
class Event:
    kind: Literal["dpu", "dma", "host"]
    future: Future


class NumpyBackend:
    device_side_waits = False

    def __init__(self, config: NumpyBackendConfig) -> None:
        if config.allow_device_to_device:
            raise ValueError("device-to-device copies are not supported in Phase 1")
        if config.num_dpus <= 0:
            raise ValueError("num_dpus must be positive")
        self.config = config
        self._kernels: dict[str, Callable] = {}
        self._pool = ThreadPoolExecutor(max_workers=config.num_dpus + 1)
        self._locks = {d: Lock() for d in range(config.num_dpus)}
        self._tails: dict[int, Future] = {}
        self._events: dict[int, Event] = {}
        self._mram = [np.zeros(config.mram_bytes_per_dpu, dtype=np.uint8) for _ in range(config.num_dpus)]
        self._host: dict[int, np.ndarray] = {}
        self._plans: dict[int, object] = {}  # keeps every registered plan alive, so ids stay unique
        self._staging: dict[int, dict] = {}

    # -- memory ------------------------------------------------------------
    def _check(self, offset: int, nbytes: int) -> None:
        cap = self.config.mram_bytes_per_dpu
        if offset < 0 or nbytes < 0 or offset + nbytes > cap:
            raise ValueError(f"invalid MRAM range offset={offset} nbytes={nbytes} capacity={cap}")

    def _mem(self, dpu_id: int) -> np.ndarray:
        if not 0 <= int(dpu_id) < self.config.num_dpus:
            raise ValueError(f"dpu_id {dpu_id} out of range")
        return self._mram[int(dpu_id)]

    def copy_to_dpu(self, dpu_id: int, offset: int, data: np.ndarray) -> None:
        blob = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        self._check(offset, blob.nbytes)
        self._mem(dpu_id)[offset:offset + blob.nbytes] = blob

    def copy_from_dpu(self, dpu_id: int, offset: int, shape, dtype) -> np.ndarray:
        dt = np_dtype(dtype)
        size = int(np.prod(shape)) * dt.itemsize
        self._check(offset, size)
        return self._mem(dpu_id)[offset:offset + size].copy().view(dt).reshape(shape)

    def write_local(self, dpu_id: int, offset: int, data: np.ndarray) -> None:
        self.copy_to_dpu(dpu_id, offset, data)

    def read_local(self, dpu_id: int, offset: int, shape, dtype) -> np.ndarray:
        return self.copy_from_dpu(dpu_id, offset, shape, dtype)

    def push_xfer(self, transfers: list[tuple[int, int, np.ndarray]]) -> None:
        for dpu_id, offset, data in transfers:
            self.copy_to_dpu(dpu_id, offset, data)

    # -- plans ------------------------------------------------------------
    def register_kernel(self, name: str, fn: Callable) -> None:
        self._kernels[name] = fn

    def register_plan(self, plan) -> None:
        from oracle import kernels

        self._plans[id(plan)] = plan
        layout = plan.meta.get("host_layout")
        self._host[id(plan)] = np.zeros(max(layout.total if layout else 0, 1), dtype=np.uint8)
        self._staging[id(plan)] = {}
        kernels.bind(self, plan)
        self._plan = plan

    def release_plan(self, plan) -> None:
        """Drop a registered plan's host arena and staging buffers."""
        if self._plans.pop(id(plan), None) is not None:
            self._host.pop(id(plan), None)
            self._staging.pop(id(plan), None)
            if self._plan is plan:
                self._plan = None

    def host_arena(self, plan) -> np.ndarray:
        return self._host[id(plan)]

    def staging(self, plan) -> dict:
        return self._staging[id(plan)]

    def write_host(self, plan, offset: int, data: np.ndarray) -> None:
        blob = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        self._host[id(plan)][offset:offset + blob.nbytes] = blob

    def read_host(self, plan, offset: int, shape, dtype) -> np.ndarray:
        dt = np_dtype(dtype)
        n = int(np.prod(shape)) * dt.itemsize
        return self._host[id(plan)][offset:offset + n].copy().view(dt).reshape(shape)

    def begin_run(self, plan=None) -> None:
        for ev in list(self._events.values()):
            try:
                ev.future.result()
            except Exception:
                pass
        self._events.clear()
        self._tails.clear()
        if plan is not None:
            self._plan = plan

    # -- async core --------------------------------------------------------
    def submit(self, cmd) -> Event:
        if cmd.id in self._events:
            raise ValueError(f"duplicate command id {cmd.id}")
        deps = []
        for w in cmd.waits:
            ev = self._events.get(w)
            if ev is None:
                raise ValueError(f"unknown dependency command id {w}")
            deps.append(ev.future)
        p = cmd.payload
        if cmd.op == "launch":
            kernel = self._kernels[str(p["kernel"])]
            ev = Event("dpu", self._on_dpu(int(cmd.dpu_id), deps, kernel, self, int(cmd.dpu_id), cmd))
        elif cmd.op == "dma_in":
            if p.get("data") is None and "host_offset" in p:
                arena = self._host_for(cmd)
                data = arena[p["host_offset"]:p["host_offset"] + p["nbytes"]].copy()
            else:
                data = np.ascontiguousarray(np.asarray(p["data"])).copy()
            ev = Event("dma", self._on_dpu(int(cmd.dpu_id), deps, self.copy_to_dpu, int(cmd.dpu_id),
                                           int(p["offset"]), data))
        elif cmd.op == "dma_out":
            ev = Event("dma", self._on_dpu(int(cmd.dpu_id), deps, self.copy_from_dpu, int(cmd.dpu_id),
                                           int(p["offset"]), tuple(p["shape"]), np_dtype(p["dtype"])))
        elif cmd.dpu_id is None:
            ev = Event("host", self._pool.submit(self._run_host, cmd, deps))
        else:
            raise ValueError(f"unsupported command op {cmd.op!r}")
        self._events[cmd.id] = ev
        return ev

    def _host_for(self, cmd) -> np.ndarray:
        return self._host[id(self._plan)]

    def _on_dpu(self, dpu_id: int, deps, fn, *args) -> Future:
        with self._locks[dpu_id]:
            prev = self._tails.get(dpu_id)

            def run():
                if prev is not None:
                    prev.result()
                for d in deps:
                    d.result()
                return fn(*args)

            fut = self._pool.submit(run)
            self._tails[dpu_id] = fut
            return fut

    @staticmethod
    def _run_host(cmd, deps):
        for d in deps:
            d.result()
        fn = cmd.payload.get("fn")
        if callable(fn):
            return fn(cmd)
        return None

    def wait(self, event: Event, timeout: float | None = None):
        return event.future.result(timeout=timeout)

    def query(self, event: Event) -> bool:
        return event.future.done()

    def close(self) -> None:
        self._pool.shutdown(wait=True)
