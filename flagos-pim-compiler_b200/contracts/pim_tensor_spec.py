"""Tensor placement contract shared by the compile passes and the runtime.

Same records as the reference (contracts/pim_tensor_spec.py:5-96):
``Placement`` is Shard(dim) / Replicate / Partial(sum|mean);
``TensorShardDetail`` is one rank's slice and its arena byte offset;
``PIMTensorSpec`` bundles them; ``RedistributeEdge`` marks a producer/consumer
placement mismatch that the comm plan expands into segments.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Literal


@dataclass(frozen=True)
class Placement:
    kind: Literal["Shard", "Replicate", "Partial"]
    dim: int | None = None
    reduce_type: str | None = None

    def validate(self) -> None:
        if self.kind == "Shard":
            ok = self.dim is not None and self.dim >= 0 and self.reduce_type is None
            if not ok:
                raise ValueError("Shard placement requires a non-negative dim and no reduce_type")
        elif self.kind == "Replicate":
            if self.dim is not None or self.reduce_type is not None:
                raise ValueError("Replicate placement requires no dim or reduce_type")
        elif self.kind == "Partial":
            if self.dim is not None or self.reduce_type not in ("sum", "mean"):
                raise ValueError("Partial placement requires reduce_type 'sum' or 'mean' and no dim")
        else:
            raise ValueError(f"unsupported placement kind: {self.kind}")


REPLICATE = Placement("Replicate")
PARTIAL_SUM = Placement("Partial", reduce_type="sum")


@dataclass(frozen=True)
class TensorShardDetail:
    dpu_id: int
    shard_dim: int
    start_idx: int
    end_idx: int
    local_shape: tuple[int, ...]
    mram_offset: int = 0

    def validate(self) -> None:
        if self.dpu_id < 0:
            raise ValueError("dpu_id must be non-negative")
        if self.start_idx < 0 or self.end_idx < self.start_idx:
            raise ValueError("shard range must be non-negative and ordered")
        if self.mram_offset < 0:
            raise ValueError("mram_offset must be non-negative")
        if any(d < 0 for d in self.local_shape):
            raise ValueError("local_shape dimensions must be non-negative")


@dataclass
class PIMTensorSpec:
    device: Literal["host", "dpu"]
    placement: Placement
    residency: Literal["transient", "pinned"]
    pinned_dpu_id: int | None
    shard_map: dict[int, TensorShardDetail]
    reduce_type: str | None

    def validate(self) -> None:
        self.placement.validate()
        if self.reduce_type != self.placement.reduce_type:
            raise ValueError("spec reduce_type must match placement reduce_type")
        if self.device == "host":
            if self.shard_map:
                raise ValueError("host spec must have an empty shard_map")
            return
        if not self.shard_map:
            raise ValueError("dpu spec must have a non-empty shard_map")
        for rank, detail in self.shard_map.items():
            if rank != detail.dpu_id:
                raise ValueError("shard_map key must match TensorShardDetail.dpu_id")
            detail.validate()
            want = self.placement.dim if self.placement.kind == "Shard" else -1
            if detail.shard_dim != want:
                raise ValueError("shard detail shard_dim does not match the placement")


@dataclass(frozen=True)
class RedistributeEdge:
    """One placement mismatch on a producer -> consumer edge.

    ``type`` is all_reduce (Partial->Replicate), all_gather (Shard->Replicate or
    dpu->host), all_to_all (Shard(i)->Shard(j)), scatter (host->dpu) or
    local_slice (Replicate@dpu -> Shard@dpu, no data motion).
    """

    edge_id: int
    src: str
    dst: str
    from_placement: Placement
    to_placement: Placement
    src_spec: PIMTensorSpec
    dst_spec: PIMTensorSpec
    type: Literal["all_reduce", "all_gather", "all_to_all", "scatter", "local_slice"]
    src_loc: dict
    dst_loc: dict
    nbytes: int
    reduce_type: str | None = None
    shape: tuple[int, ...] = ()
    dtype: str = ""
