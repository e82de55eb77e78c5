"""Comm cost models for plan_cost: host star, NVLink constants, and costs fitted to measured edges (CPU)."""

from __future__ import annotations

import json

import pytest

from helpers import redistribute_entry


def _cases(lat_us, gbs, kind, n, tokens=(1, 16, 256, 2048)):
    from comm.plan import bus_bytes

    out = []
    for t in tokens:
        entry, _ = redistribute_entry(kind, n, (t, 4096))
        b = bus_bytes(entry)
        out.append({"kind": kind, "tokens": t, "bus_bytes_per_rank": b, "us": lat_us + b / (gbs * 1e3)})
    return out


def test_bus_bytes_follow_the_nccl_convention():
    from comm.plan import bus_bytes

    s = 2048 * 4096 * 2
    for n in (2, 4, 8):
        assert bus_bytes(redistribute_entry("all_reduce", n, (2048, 4096))[0]) == int(s * 2 * (n - 1) / n)
        assert bus_bytes(redistribute_entry("all_gather", n, (2048, 4096))[0]) == int(s * (n - 1) / n)
        assert bus_bytes(redistribute_entry("all_to_all", n, (2048, 4096))[0]) == int(s * (n - 1) / n ** 2)


def test_fit_recovers_latency_and_bandwidth_per_kind():
    from comm.plan import MeasuredCostModel, plan_cost

    cases = _cases(9.0, 600.0, "all_reduce", 8) + _cases(5.0, 700.0, "all_gather", 8)
    m = MeasuredCostModel.fit(cases)
    lat, bw = m.params("all_reduce")
    assert lat == pytest.approx(9e-6, rel=1e-6) and bw == pytest.approx(600e9, rel=1e-6)
    lat, bw = m.params("all_gather")
    assert lat == pytest.approx(5e-6, rel=1e-6) and bw == pytest.approx(700e9, rel=1e-6)
    assert m.params("all_to_all") == (m.fallback.latency_s, m.fallback.bus_bytes_per_s)  # no data: fallback
    entry, _ = redistribute_entry("all_reduce", 8, (512, 4096))
    c = plan_cost(entry, m)
    assert c.transfers == 1 and c.seconds == pytest.approx(9e-6 + c.nbytes / 600e9, rel=1e-6)


def test_fit_clamps_a_negative_intercept_and_reads_a_bench_line():
    from comm.plan import MeasuredCostModel

    cases = [{"kind": "all_reduce", "bus_bytes_per_rank": 1e6, "us": 1.0},
             {"kind": "all_reduce", "bus_bytes_per_rank": 2e6, "us": 3.0},
             {"kind": "all_to_all", "tokens": 1, "n/a": "undefined"}]
    line = json.dumps({"metric": "redistribute", "cases": cases})
    m = MeasuredCostModel.from_bench_line(line)
    lat, bw = m.params("all_reduce")
    assert lat == 0.0 and bw == pytest.approx(1e6 / ((1e6 * 1e-6 + 2e6 * 3e-6) / 5e6), rel=1e-9)


def test_host_star_and_nvlink_models_still_price_every_edge():
    from comm.plan import HostStarCostModel, NvlinkCostModel, plan_cost

    entry, _ = redistribute_entry("all_gather", 4, (16, 4096))
    host = plan_cost(entry, HostStarCostModel())
    nv = plan_cost(entry, NvlinkCostModel())
    assert host.transfers > 1 and host.seconds > nv.seconds > 0


def test_fit_to_the_measured_b200_edges_predicts_each_edge():
    """Costs fitted to the redistribute microbench measured on 4 B200 GPUs (the committed
    bench line): the large edges within 5 %, the latency-bound ones within a factor 1.5."""
    from comm.plan import MeasuredCostModel, NvlinkCostModel, plan_cost

    from helpers import GOLDEN

    line = json.loads((GOLDEN / "redistribute_b200_n4.json").read_text())["line"]
    m = MeasuredCostModel.from_bench_line(line)
    assert {k for k, _, _ in m.fits} == {"all_reduce", "all_gather", "all_to_all"}
    for c in line["cases"]:
        if "us" not in c:
            continue
        entry, _ = redistribute_entry(c["kind"], line["n_gpus"], (c["tokens"], 4096))
        got = plan_cost(entry, m)
        assert got.nbytes == c["bus_bytes_per_rank"]
        ratio = got.seconds / (c["us"] * 1e-6)
        assert (0.95 <= ratio <= 1.05) if c["tokens"] == 2048 else (1 / 1.5 <= ratio <= 1.5), (c, ratio)
    # the measured floor per collective (a graph replay of pack + NCCL + placement) is far
    # above the constant model's 8 us; its bandwidth is below the all-reduce bus figure
    assert all(lat > NvlinkCostModel().latency_s for _, lat, _ in m.fits)
    assert all(bw < NvlinkCostModel().bus_bytes_per_s for _, _, bw in m.fits)
