"""ExecutionPlan contract: the command DAG the runtime interprets.

Field-for-field the same record layout as the reference contract
(contracts/exec_plan.py:5-34) because every pass and both HALs exchange these
objects; the docs/spec.md:1397-1420 definition is the source of truth.

``Access.loc`` is ``("dpu", rank)`` or ``("host", None)``; ``offset``/``length``
are byte positions inside that location's arena.  ``Command.waits`` lists the
ids of earlier commands that must complete first.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Literal

CommandOp = Literal[
    "launch",
    "dma_in",
    "dma_out",
    "host_reduce",
    "host_concat",
    "host_permute",
    "host_slice",
    "host_op",
]

HOST_OPS = ("host_reduce", "host_concat", "host_permute", "host_slice", "host_op")


@dataclass(frozen=True)
class Access:
    loc: tuple[str, int | None]
    offset: int
    length: int

    def overlaps(self, other: "Access") -> bool:
        """Half-open byte-interval intersection on the same location (docs/spec.md:1432-1433)."""
        return (
            self.loc == other.loc
            and self.offset < other.offset + other.length
            and other.offset < self.offset + self.length
        )


@dataclass
class Command:
    id: int
    op: CommandOp
    dpu_id: int | None
    payload: dict[str, object]
    reads: list[Access] = field(default_factory=list)
    writes: list[Access] = field(default_factory=list)
    waits: list[int] = field(default_factory=list)


@dataclass
class ExecutionPlan:
    commands: list[Command]
    # Free-form description the generator attaches (graph name, phase, buffers);
    # interpreters ignore it.  Not part of the reference record.
    meta: dict[str, object] = field(default_factory=dict)
