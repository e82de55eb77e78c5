"""The lockstep node comparator on the CPU: oracle against oracle (CPU).

``lockstep_compare`` runs a plan command by command on two HALs, compares every interval
each command writes and then copies the first HAL's bytes into the second.  Two oracle
HALs must agree exactly on every command of the tiny prefill and decode plans; a mistake
planted in one oracle kernel (a scaled RMSNorm weight inside ``mlp_in`` of layer 1) must
show up at that node and only there, because the copy-back keeps it from reaching the
nodes after it.
"""

from __future__ import annotations

import numpy as np

from assert_node_matches_ref import argmax_within_tolerance, lockstep_compare
from helpers import oracle_hal, tiny_golden, tiny_hf_model, tiny_program, tiny_weights


def _pair():
    """Two oracle HALs with the tiny weights, each with its own compile of the same program."""
    from runtime.program import load_weights

    progs = [tiny_program(1), tiny_program(1)]
    w = tiny_weights(progs[0], tiny_hf_model())
    hals = [oracle_hal(p) for p in progs]
    for p, h in zip(progs, hals):
        load_weights(p, h, w)
    return progs, hals


def test_two_oracles_agree_on_every_command():
    (pa, pb), (a, b) = _pair()
    gold = tiny_golden()
    res = lockstep_compare(pa.plans["prefill"], a, b, tokens=gold["prompt"][None], pos=np.zeros(1, np.int32),
                           ref_plan=pb.plans["prefill"])
    assert len(res) > 10 and all(v == 0 for _, _, v in res)
    assert {"logits", "l1.mlp_act", "next_token"} <= {n for n, _, _ in res}
    res = lockstep_compare(pa.plans["decode"], a, b, tokens=gold["tokens"][:1].reshape(1, 1),
                           pos=np.full(1, 16, np.int32), ref_plan=pb.plans["decode"])
    assert all(v == 0 for _, _, v in res)


def test_a_planted_mistake_shows_at_its_node_only():
    import oracle.kernels as ok

    (pa, pb), (a, b) = _pair()
    gold = tiny_golden()
    orig = ok.KERNELS["mlp_in"]

    def wrong_mlp_in(hal, rank, cmd):
        orig(hal, rank, cmd)
        if cmd.payload.get("node") == "l1.mlp_act":
            off, shape, dt = cmd.payload["output"]
            y = hal.read_local(rank, off, shape, np.dtype(dt))
            hal.write_local(rank, off, (y * np.float32(1.05)).astype(np.dtype(dt)))

    b.register_kernel("mlp_in", wrong_mlp_in)
    res = lockstep_compare(pa.plans["prefill"], a, b, tokens=gold["prompt"][None], pos=np.zeros(1, np.int32),
                           ref_plan=pb.plans["prefill"])
    bad = {n for n, _, v in res if v}
    assert bad == {"l1.mlp_act"}, bad


def test_greedy_ids_differ_only_at_ties():
    ref = np.array([[0.0, 1.0, 0.999, -1.0], [0.0, 1.0, 0.5, -1.0]], np.float32)
    got = np.array([[0.0, 0.998, 1.0, -1.0], [0.0, 0.6, 1.0, -1.0]], np.float32)
    gi, ri, tied = argmax_within_tolerance(got, ref, 2e-2)
    assert gi == [2, 2] and ri == [1, 1] and tied == [0]  # row 1 is a real mismatch
