"""Host-star redistribute primitives (oracle): restatement of comm/lowering.py.

Every primitive takes a ``CommPlanEntry`` and an engine over per-DPU byte
arrays (comm/lowering.py:38-97) and runs collect -> host combine -> writeback:

* ``all_reduce`` (comm/lowering.py:137-150): ``acc = zeros(numel, dtype)``, then
  ``acc[global_range] += buf`` for every collect segment in order, *in the
  entry's dtype* (for bf16 that is an fp32 add rounded to bf16 after every
  partial -- the rounding the B200 ordered-sum kernel reproduces); ``mean``
  divides by the number of collect segments;
* ``all_gather`` / ``all_to_all`` (comm/lowering.py:153-173): place each
  collected run at its global range, ordered by ``global_range[0]`` -- never
  by rank id (comm/lowering.py:121-129);
* ``scatter`` / ``broadcast`` (comm/lowering.py:176-194): writeback only.

``combine`` is the shared host step; the oracle HAL's host commands call it
with the arrays the plan's collect transfers returned.
"""

from __future__ import annotations

import numpy as np

from oracle.hal_numpy import NumpyBackend


class DmaEngine:
    def __init__(self, hal: NumpyBackend) -> None:
        self.hal = hal

    def copy_from_dpu(self, dpu_id: int, addr: int, length: int, dtype) -> np.ndarray:
        return self.hal.copy_from_dpu(dpu_id, addr, (length,), dtype)

    def copy_to_dpu(self, dpu_id: int, addr: int, data: np.ndarray) -> None:
        self.hal.copy_to_dpu(dpu_id, addr, np.ascontiguousarray(data).reshape(-1))


def combine(entry, collected: list[tuple[object, np.ndarray]]) -> np.ndarray:
    """The host step between collect and writeback; returns the flat global buffer."""
    if entry.type == "all_reduce":
        acc = np.zeros(entry.numel, dtype=entry.dtype)
        for seg, buf in collected:
            acc[seg.global_range[0]:seg.global_range[1]] += buf
        if entry.reduce == "mean":
            acc /= len(entry.collect_segments)
        return acc
    merged = np.zeros(entry.numel, dtype=entry.dtype)
    for seg, buf in sorted(collected, key=lambda item: item[0].global_range[0]):
        merged[seg.global_range[0]:seg.global_range[1]] = buf
    return merged


def _check(entry, expect: str) -> None:
    if entry.type != expect:
        raise ValueError(f"{expect} received an entry of type {entry.type} (edge {entry.edge_id})")


def _collect(entry, engine: DmaEngine):
    return [(s, engine.copy_from_dpu(s.src_dpu, s.src_addr, s.nbytes // entry.dtype.itemsize, entry.dtype))
            for s in entry.collect_segments]


def _writeback(entry, engine: DmaEngine, flat: np.ndarray) -> None:
    for s in entry.writeback_segments:
        engine.copy_to_dpu(s.dst_dpu, s.dst_addr, flat[s.global_range[0]:s.global_range[1]])


def all_reduce(entry, engine: DmaEngine) -> np.ndarray:
    _check(entry, "all_reduce")
    acc = combine(entry, _collect(entry, engine))
    _writeback(entry, engine, acc)
    return acc.reshape(entry.shape)


def all_gather(entry, engine: DmaEngine) -> np.ndarray:
    _check(entry, "all_gather")
    merged = combine(entry, _collect(entry, engine))
    _writeback(entry, engine, merged)
    return merged.reshape(entry.shape)


def all_to_all(entry, engine: DmaEngine) -> np.ndarray:
    _check(entry, "all_to_all")
    staging = combine(entry, _collect(entry, engine))
    _writeback(entry, engine, staging)
    return staging.reshape(entry.shape)


def scatter(entry, engine: DmaEngine, host_buf: np.ndarray) -> None:
    _check(entry, "scatter")
    flat = np.ascontiguousarray(host_buf, dtype=entry.dtype).reshape(-1)
    if flat.size != entry.numel:
        raise ValueError(f"scatter host_buf has {flat.size} elements, entry has {entry.numel}")
    _writeback(entry, engine, flat)


def broadcast(entry, engine: DmaEngine, host_buf: np.ndarray) -> None:
    flat = np.ascontiguousarray(host_buf, dtype=entry.dtype).reshape(-1)
    if flat.size != entry.numel:
        raise ValueError(f"broadcast host_buf has {flat.size} elements, entry has {entry.numel}")
    _writeback(entry, engine, flat)
