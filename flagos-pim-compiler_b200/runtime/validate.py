"""Static checks of compiled plans (debug aid and test oracle for the generator).

``plan_hazards`` proves that every pair of conflicting accesses in an
ExecutionPlan is ordered: for commands ``a`` before ``b`` whose byte intervals
overlap on one location and at least one of which writes, ``b`` must reach
``a`` through ``waits`` (transitively) or both must run on the same rank's
serial stream.  This is the correctness condition docs/spec.md:1421-1466 asks
of the writers / pending_readers algorithm; an empty result means the plan can
run with full cross-stream concurrency without races.

``arena_overlaps`` checks a DPUPlan: weights, KV and every pair of activation
buffers whose lifetimes intersect occupy disjoint bytes.
"""

from __future__ import annotations

from contracts.exec_plan import ExecutionPlan
from memory.mem_planner import DPUPlan, align_up


def _ancestors(plan: ExecutionPlan) -> list[set[int]]:
    anc: list[set[int]] = []
    by_id = {c.id: i for i, c in enumerate(plan.commands)}
    last_on_stream: dict[int, int] = {}
    for i, c in enumerate(plan.commands):
        s: set[int] = set()
        preds = [by_id[w] for w in c.waits]
        if c.dpu_id is not None and c.dpu_id in last_on_stream:
            preds.append(last_on_stream[c.dpu_id])
        for p in preds:
            s.add(p)
            s |= anc[p]
        anc.append(s)
        if c.dpu_id is not None:
            last_on_stream[c.dpu_id] = i
    return anc


def plan_hazards(plan: ExecutionPlan, limit: int = 20) -> list[str]:
    anc = _ancestors(plan)
    out = []
    cmds = plan.commands
    for j, b in enumerate(cmds):
        for i in range(j):
            a = cmds[i]
            if i in anc[j]:
                continue
            conflict = None
            for wa in a.writes:
                for x in b.reads + b.writes:
                    if wa.overlaps(x):
                        conflict = ("RAW/WAW", wa, x)
                        break
                if conflict:
                    break
            if not conflict:
                for ra in a.reads:
                    for wb in b.writes:
                        if ra.overlaps(wb):
                            conflict = ("WAR", ra, wb)
                            break
                    if conflict:
                        break
            if conflict:
                out.append(f"{conflict[0]}: cmd {a.id} ({a.op} {a.payload.get('node') or a.payload.get('role')}) "
                           f"and cmd {b.id} ({b.op} {b.payload.get('node') or b.payload.get('role')}) "
                           f"on {conflict[1].loc} are unordered")
                if len(out) >= limit:
                    return out
    return out


def arena_overlaps(plan: DPUPlan, align: int = 256) -> list[str]:
    out = []
    for g, lives in plan.lifetimes.items():
        for i, a in enumerate(lives):
            if a.offset < plan.act_base:
                out.append(f"{g}: {a.key} below act_base")
            a_hi = a.offset + align_up(max(a.nbytes, 1), align)
            for b in lives[i + 1:]:
                if a.end < b.start or b.end < a.start:
                    continue
                b_hi = b.offset + align_up(max(b.nbytes, 1), align)
                if a.offset < b_hi and b.offset < a_hi:
                    out.append(f"{g}: {a.key} and {b.key} overlap while both live")
    if plan.kv_spec is not None and plan.kv_base + plan.kv_spec.kv_allocated_bytes > plan.act_base:
        out.append("KV zone runs into the activation zone")
    return out
