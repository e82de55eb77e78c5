"""Shared-memory geometry of the layer kernel (csrc/decode_layer.cu), checked on the CPU.

A restatement of launch_decode_layer's sizing (activation row, attention merge buffers,
weight ring, per-(task, warp) partials; 2 CTAs per SM when that fits in 112 KB, else 1)
and of DlPhase's partition (tasks by CTA, stages by warp, ring slots by lane), walked for
every CTA and warp at the shapes the kernel takes: each shared-memory index must stay
inside its buffer, every task must belong to exactly one CTA and every stage to exactly
one warp.
"""

from __future__ import annotations

import pytest

WARPS, WARP, U = 8, 32, 2
STAGE_CHUNKS = WARP * U
RING_BYTES = WARPS * 5 * U * 2 * WARP * 16


def slots(nw):
    return 8 if nw == 1 else 5


def tasks(phase):
    mode, p = phase["mode"], phase
    if mode == "plain":
        return p["ncols"]
    if mode == "rope":
        return (p["hq"] + 2 * p["hkv"]) * (p["hd"] // 2)
    return p["inter"]


def sizing(phases, es, hd, sms=148):
    kmax = max(p["k"] for p in phases)
    x_bytes = (kmax * es + 15) // 16 * 16
    groups = WARPS * (WARP // (hd // (16 // es)))
    attn = groups * (hd + 2) * 4
    if x_bytes < attn:
        x_bytes = (attn + 15) // 16 * 16
    for occ in (2, 1):
        grid = sms * occ
        tmax = max((tasks(p) + grid - 1) // grid * (1 if p["mode"] == "plain" else 2) for p in phases)
        smem = x_bytes + RING_BYTES + tmax * WARPS * 4
        if smem <= (112 if occ == 2 else 220) * 1024:
            return grid, x_bytes, tmax, smem
    return None


def walk(phase, es, grid, x_bytes, tmax):
    nw = 1 if phase["mode"] == "plain" else 2
    S, V = slots(nw), 16 // es
    nch = phase["k"] // V
    ms = (nch + STAGE_CHUNKS - 1) // STAGE_CHUNKS
    nt_all = tasks(phase)
    assert nch * 16 <= x_bytes  # the staged activation row
    seen = []
    for b in range(grid):
        t_lo, t_hi = b * nt_all // grid, (b + 1) * nt_all // grid
        nt = t_hi - t_lo
        seen += range(t_lo, t_hi)
        nst = nt * ms
        covered = []
        for w in range(WARPS):
            s_lo, s_hi = w * nst // WARPS, (w + 1) * nst // WARPS
            covered += range(s_lo, s_hi)
            if s_lo < s_hi:
                tl_first, tl_last = s_lo // ms, (s_hi - 1) // ms
                assert 0 <= tl_first <= tl_last < nt
                # partial sums of (task, warp): the highest index this warp writes
                assert ((tl_last * WARPS + w) * nw + nw - 1) < tmax * WARPS
                # weight rows it reads stay inside the projection
                assert (t_lo + tl_last) * nw + nw - 1 < nt_all * nw
            # ring: the highest int4 a lane of this warp touches
            top = w * S * U * nw * WARP + ((S - 1) * U + U - 1) * nw * WARP + (nw - 1) * WARP + WARP - 1
            assert (top + 1) * 16 <= RING_BYTES
        assert covered == list(range(nst))
        # the epilogue's reads of the partials of every task of the CTA
        assert nt == 0 or ((nt - 1) * WARPS + WARPS - 1) * nw + nw - 1 < tmax * WARPS
    assert seen == list(range(nt_all))


def layer(hidden, inter, hq, hkv, hd):
    return [dict(mode="rope", k=hidden, hq=hq, hkv=hkv, hd=hd), dict(mode="plain", k=hq * hd, ncols=hidden),
            dict(mode="silu", k=hidden, inter=inter), dict(mode="plain", k=inter, ncols=hidden)]


CASES = {
    "7b_tp1_bf16": (layer(4096, 11008, 32, 32, 128), 2),
    "7b_tp2_bf16": (layer(4096, 5504, 16, 16, 128), 2),
    "7b_tp4_bf16": (layer(4096, 2752, 8, 8, 128), 2),
    "7b_tp8_bf16": (layer(4096, 1376, 4, 4, 128), 2),
    "7b_tp1_fp32": (layer(4096, 11008, 32, 32, 128), 4),
    "gqa_hd64_bf16": (layer(512, 688, 8, 2, 64), 2),
    "tiny_tp1_fp32": (layer(256, 688, 4, 4, 64), 4),
    "tiny_tp2_fp32": (layer(256, 344, 2, 2, 64), 4),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_every_shared_memory_index_of_the_layer_kernel_stays_in_its_buffer(name):
    phases, es = CASES[name]
    hd = phases[0]["hd"]
    got = sizing(phases, es, hd)
    assert got is not None, "no grid fits"
    grid, x_bytes, tmax, smem = got
    assert smem <= 227 * 1024
    for p in phases:
        walk(p, es, grid, x_bytes, tmax)


def test_7b_bf16_layers_run_two_ctas_per_sm():
    for name in ("7b_tp1_bf16", "7b_tp2_bf16", "7b_tp4_bf16", "7b_tp8_bf16"):
        phases, es = CASES[name]
        grid, x_bytes, tmax, smem = sizing(phases, es, 128)
        assert grid == 296 and smem <= 112 * 1024, (name, smem)


@pytest.mark.parametrize("tp", [1, 2, 4, 8])
def test_the_step_kernel_with_its_lm_head_phase_fits_two_ctas_per_sm_at_7b(tp):
    """The whole-step kernel sizes its grid over every layer's phases and the lm_head_in
    phase (final rmsnorm + vocabulary GEMV over this rank's 32000 / TP rows)."""
    phases, es = CASES[f"7b_tp{tp}_bf16"]
    head = dict(mode="plain", k=4096, ncols=32000 // tp)
    grid, x_bytes, tmax, smem = sizing(phases * 32 + [head], es, 128)
    assert grid == 296 and smem <= 112 * 1024
    walk(head, es, grid, x_bytes, tmax)
