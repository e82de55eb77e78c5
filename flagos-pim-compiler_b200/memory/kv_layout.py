"""Static KV-cache layout, per-rank append/read, and attention masks.

Restates the reference's KV module (memory/kv_layout.py:28-266).  The layout
is a contract between the planner, the K/V-writing kernels and the attention
kernels, so its order is kept exactly:

    kv_off[(layer, head, "k"|"v")] = kv_base + i * align_up(max_seq*head_dim*dtype_bytes, align)

with ``i`` counting layer-major, then kv head, then k before v
(memory/kv_layout.py:81-99).  Each block is a contiguous ``[max_seq, head_dim]``
row-major matrix that never leaves its rank.

Two additions the B200 runtime needs, both off by default so the reference
layout is reproduced byte for byte:

* ``num_seqs`` -- batched decode keeps one complete region set per sequence,
  sequence ``s`` starting at ``kv_base + s * seq_stride``; ``seq_stride`` is the
  single-sequence ``kv_allocated_bytes``;
* ``dtype`` -- the element type name read back by ``read_tile`` (the reference
  maps 2-byte KV to float16 only, memory/kv_layout.py:25; bf16 caches pass
  ``dtype="bfloat16"``).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Literal

import numpy as np

from contracts.exec_plan import Access
from contracts.pim_tensor_spec import PIMTensorSpec

_DEFAULT_DTYPE = {2: "float16", 4: "float32"}


def align_up(n: int, align: int) -> int:
    if align <= 0:
        raise ValueError(f"align must be positive, got {align}")
    return -(-n // align) * align


def _np(name: str) -> np.dtype:
    if name == "bfloat16":
        import ml_dtypes

        return np.dtype(ml_dtypes.bfloat16)
    return np.dtype(name)


@dataclass
class KVRegionSpec:
    dpu_id: int
    layers: list[int]
    kv_heads: list[int]
    q_heads_by_kv: dict[int, list[int]]
    max_seq: int
    head_dim: int
    dtype_bytes: int
    kv_base: int
    kv_off: dict[tuple[int, int, str], int] = field(default_factory=dict)
    kv_allocated_bytes: int = 0
    num_seqs: int = 1
    dtype: str | None = None
    seq_stride: int = 0

    @property
    def dtype_name(self) -> str:
        return self.dtype or _DEFAULT_DTYPE[self.dtype_bytes]

    @property
    def block_bytes(self) -> int:
        return self.max_seq * self.head_dim * self.dtype_bytes

    def validate(self) -> None:
        if self.dpu_id < 0:
            raise ValueError("dpu_id must be non-negative")
        if not self.layers or not self.kv_heads:
            raise ValueError("layers / kv_heads must not be empty")
        if self.max_seq <= 0 or self.head_dim <= 0:
            raise ValueError("max_seq / head_dim must be positive")
        if self.dtype_bytes not in _DEFAULT_DTYPE:
            raise ValueError(f"unsupported dtype_bytes {self.dtype_bytes}")
        if self.dtype is not None and _np(self.dtype).itemsize != self.dtype_bytes:
            raise ValueError(f"dtype {self.dtype} does not have {self.dtype_bytes} bytes")
        if self.kv_base < 0:
            raise ValueError("kv_base must be non-negative")
        if self.num_seqs <= 0:
            raise ValueError("num_seqs must be positive")
        missing = [h for h in self.kv_heads if h not in self.q_heads_by_kv]
        if missing:
            raise ValueError(f"q_heads_by_kv lacks kv heads {missing}")

    def offset(self, layer: int, head: int, which: str, seq: int = 0) -> int:
        return self.kv_off[(layer, head, which)] + seq * self.seq_stride


def kv_bytes(spec: KVRegionSpec) -> int:
    """Unaligned lower bound (capacity estimate only; not an allocation size)."""
    return 2 * len(spec.layers) * spec.max_seq * len(spec.kv_heads) * spec.head_dim * spec.dtype_bytes * spec.num_seqs


def build_kv_layout(spec: KVRegionSpec, align: int) -> KVRegionSpec:
    """Fill ``kv_off`` and ``kv_allocated_bytes`` (alignment padding included)."""
    spec.validate()
    step = align_up(spec.block_bytes, align)
    table = {}
    i = 0
    for layer in spec.layers:
        for head in spec.kv_heads:
            for which in ("k", "v"):
                table[(layer, head, which)] = spec.kv_base + i * step
                i += 1
    spec.kv_off = table
    spec.seq_stride = i * step
    spec.kv_allocated_bytes = i * step * spec.num_seqs
    return spec


def kv_specs_from_placement(
    k_proj_spec: PIMTensorSpec,
    *,
    num_layers: int,
    num_kv_heads: int,
    num_q_heads: int,
    head_dim: int,
    max_seq: int,
    dtype_bytes: int,
    kv_base: int,
    num_seqs: int = 1,
    dtype: str | None = None,
) -> dict[int, KVRegionSpec]:
    """KV follows the k_proj head split: rank d keeps the heads of its Shard(0) rows."""
    if k_proj_spec.placement.kind != "Shard" or k_proj_spec.placement.dim != 0:
        raise ValueError(f"KV head sharding needs k_proj Shard(0), got {k_proj_spec.placement}")
    if num_q_heads % num_kv_heads:
        raise ValueError(f"num_q_heads={num_q_heads} is not a multiple of num_kv_heads={num_kv_heads}")
    group = num_q_heads // num_kv_heads
    out = {}
    for rank, det in sorted(k_proj_spec.shard_map.items()):
        if det.start_idx % head_dim or det.end_idx % head_dim:
            raise ValueError(f"dpu{rank} k_proj rows [{det.start_idx},{det.end_idx}) not aligned to head_dim={head_dim}")
        heads = list(range(det.start_idx // head_dim, det.end_idx // head_dim))
        out[rank] = KVRegionSpec(
            dpu_id=rank,
            layers=list(range(num_layers)),
            kv_heads=heads,
            q_heads_by_kv={h: list(range(h * group, (h + 1) * group)) for h in heads},
            max_seq=max_seq,
            head_dim=head_dim,
            dtype_bytes=dtype_bytes,
            kv_base=kv_base,
            num_seqs=num_seqs,
            dtype=dtype,
        )
    return out


def kv_access(
    spec: KVRegionSpec, layer: int, head: int, which: Literal["k", "v"], pos_start: int, pos_end: int,
    seq: int = 0,
) -> Access:
    """Byte interval of rows ``[pos_start, pos_end)`` of one KV block (absolute arena address)."""
    if not (0 <= pos_start < pos_end <= spec.max_seq):
        raise ValueError(f"range [{pos_start},{pos_end}) outside [0,{spec.max_seq})")
    row = spec.head_dim * spec.dtype_bytes
    return Access(("dpu", spec.dpu_id), spec.offset(layer, head, which, seq) + pos_start * row,
                  (pos_end - pos_start) * row)


def kv_layer_access(spec: KVRegionSpec, layer: int) -> Access:
    """One interval covering every block of ``layer`` for sequence 0..num_seqs-1.

    Blocks of a layer are adjacent (layer-major order), so a layer is one span
    per sequence; with several sequences the span repeats every ``seq_stride``
    and this returns the hull, which is what the plan's dependency table needs.
    """
    first = spec.kv_off[(layer, spec.kv_heads[0], "k")]
    last = spec.kv_off[(layer, spec.kv_heads[-1], "v")] + spec.block_bytes
    end = last + (spec.num_seqs - 1) * spec.seq_stride
    return Access(("dpu", spec.dpu_id), first, end - first)


class PIMStaticKVCache:
    """Per-rank static KV cache with no internal position pointer.

    Writes and reads go through the HAL's ``write_local`` / ``read_local`` on
    the owning rank only (memory/kv_layout.py:167-230); the position is always
    passed in by the caller (``DecodeState.valid_len``).  The object holds no
    data: dropping and rebuilding it reads back the same values.
    """

    def __init__(self, backend, specs: dict[int, KVRegionSpec], wram_budget_bytes: int) -> None:
        self.backend = backend
        self.specs = specs
        self.wram_budget_bytes = wram_budget_bytes
        for spec in specs.values():
            spec.validate()
            if not spec.kv_off:
                raise ValueError(f"dpu{spec.dpu_id}: KVRegionSpec has not been through build_kv_layout")

    def update(self, layer: int, pos: int, k_by_dpu: dict, v_by_dpu: dict, seq: int = 0) -> None:
        for rank, spec in self.specs.items():
            assert 0 <= pos < spec.max_seq, f"pos={pos} outside [0,{spec.max_seq})"
            row = spec.head_dim * spec.dtype_bytes
            for head in spec.kv_heads:
                for which, by_dpu in (("k", k_by_dpu), ("v", v_by_dpu)):
                    vec = np.asarray(by_dpu[rank][head])
                    if vec.size != spec.head_dim or vec.dtype.itemsize != spec.dtype_bytes:
                        raise ValueError(
                            f"dpu{rank} layer{layer} head{head} {which}: expected [{spec.head_dim}]x"
                            f"{spec.dtype_bytes}B, got shape={vec.shape} dtype={vec.dtype}")
                    self.backend.write_local(rank, spec.offset(layer, head, which, seq) + pos * row, vec)

    def read_tile(self, layer: int, dpu_id: int, head: int, tile_start: int, tile_end: int,
                  seq: int = 0) -> tuple[np.ndarray, np.ndarray]:
        spec = self.specs[dpu_id]
        if head not in spec.kv_heads:
            raise KeyError(f"head {head} is not among dpu{dpu_id} kv_heads {spec.kv_heads}")
        if not (0 <= tile_start < tile_end <= spec.max_seq):
            raise ValueError(f"tile [{tile_start},{tile_end}) outside [0,{spec.max_seq})")
        row = spec.head_dim * spec.dtype_bytes
        if (tile_end - tile_start) * row > self.wram_budget_bytes:
            raise ValueError("tile exceeds the staging budget; use a smaller tile")
        shape = (tile_end - tile_start, spec.head_dim)
        dt = _np(spec.dtype_name)
        k = self.backend.read_local(dpu_id, spec.offset(layer, head, "k", seq) + tile_start * row, shape, dt)
        v = self.backend.read_local(dpu_id, spec.offset(layer, head, "v", seq) + tile_start * row, shape, dt)
        return k, v


def prefill_mask(prompt_len: int, max_seq: int) -> np.ndarray:
    """``[max_seq, max_seq]`` additive mask: 0 where key j <= query i and j < prompt_len."""
    i = np.arange(max_seq)[:, None]
    j = np.arange(max_seq)[None, :]
    return np.where((j <= i) & (j < prompt_len), 0.0, -np.inf).astype(np.float32)


def decode_mask(valid_len: int, max_seq: int) -> np.ndarray:
    """``[max_seq]`` additive mask: 0 on ``[0, valid_len]`` (the new token included)."""
    j = np.arange(max_seq)
    return np.where(j <= valid_len, 0.0, -np.inf).astype(np.float32)


def format_kv_layout(specs: dict[int, KVRegionSpec]) -> str:
    lines = []
    for rank, s in sorted(specs.items()):
        lines.append(
            f"dpu{rank}: layers={len(s.layers)} kv_heads=[{s.kv_heads[0]}..{s.kv_heads[-1]}] seqs={s.num_seqs}"
            f" max_seq={s.max_seq} head_dim={s.head_dim} kv_base={s.kv_base}"
            f" kv_allocated_bytes={s.kv_allocated_bytes} (kv_bytes lower bound={kv_bytes(s)}) blocks={len(s.kv_off)}")
    return "KV layout:\n" + "\n".join(lines)
