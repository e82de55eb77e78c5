"""The HAL contract of backend/hal_numpy.py, checked on the oracle HAL (CPU) and on CudaBackend (GPU).

Restates tests/test_hal_numpy.py of the reference: isolation, round trips,
submit/wait/query, same-rank ordering, errors surfacing at wait, payload
snapshot at submit, cross-rank waits, no device-to-device API, read copies,
push_xfer fan-out and a LLaMA-shaped payload.  The threading-gated variants
(kernel stubs that block on host events) apply to the thread-pool oracle only:
a B200 kernel function enqueues device work and never blocks.
"""

from __future__ import annotations

import threading

import numpy as np
import pytest

from contracts.exec_plan import Access, Command, ExecutionPlan

BACKENDS = ["oracle", pytest.param("cuda", marks=pytest.mark.gpu)]


def make(kind, num_dpus, mram, **kw):
    if kind == "oracle":
        from oracle.hal_numpy import NumpyBackend, NumpyBackendConfig

        return NumpyBackend(NumpyBackendConfig(num_dpus, mram, **kw))
    from backend.hal_cuda import CudaBackend, CudaBackendConfig

    return CudaBackend(CudaBackendConfig(num_dpus, mram, **kw))


def _write_kernel(kind):
    """A kernel stub that writes payload['value'] (int32) at payload['offset'] on its rank."""
    if kind == "oracle":
        def fill(hal, dpu_id, cmd):
            hal.write_local(dpu_id, cmd.payload["offset"], np.asarray(cmd.payload["value"], dtype=np.int32))
        return fill

    import torch

    def fill_dev(hal, dpu_id, cmd):
        vals = torch.tensor(cmd.payload["value"], dtype=torch.int32).to(hal.device_of(dpu_id))
        off = cmd.payload["offset"]
        hal.arena(dpu_id)[off:off + 4 * vals.numel()].copy_(vals.view(torch.uint8), non_blocking=True)
    return fill_dev


def test_runtime_contracts_have_the_expected_fields():
    from contracts.pim_tensor_spec import PIMTensorSpec, Placement, TensorShardDetail

    shard = TensorShardDetail(dpu_id=0, shard_dim=1, start_idx=0, end_idx=4, local_shape=(2, 2))
    spec = PIMTensorSpec(device="dpu", placement=Placement(kind="Shard", dim=1), residency="pinned",
                         pinned_dpu_id=0, shard_map={0: shard}, reduce_type=None)
    spec.validate()
    plan = ExecutionPlan(commands=[Command(id=0, op="launch", dpu_id=0, payload={"kernel": "noop"}, reads=[],
                                           writes=[Access(("dpu", 0), 0, 16)], waits=[])])
    assert spec.shard_map[0].local_shape == (2, 2)
    assert plan.commands[0].writes[0].offset == 0


@pytest.mark.parametrize("kind", BACKENDS)
def test_dpu_isolation_and_copy_round_trip(kind):
    hal = make(kind, 2, 64)
    payload = np.arange(8, dtype=np.int32)
    hal.copy_to_dpu(0, 0, payload)
    assert np.array_equal(hal.copy_from_dpu(0, 0, payload.shape, payload.dtype), payload)
    assert np.array_equal(hal.copy_from_dpu(1, 0, payload.shape, payload.dtype), np.zeros_like(payload))


@pytest.mark.parametrize("kind", BACKENDS)
def test_submit_wait_query_and_kernel_stub(kind):
    hal = make(kind, 1, 64)
    hal.register_kernel("fill", _write_kernel(kind))
    ev = hal.submit(Command(1, "launch", 0, {"kernel": "fill", "offset": 0, "value": [1, 2, 3, 4]},
                            writes=[Access(("dpu", 0), 0, 16)]))
    hal.wait(ev)
    assert hal.query(ev)
    assert hal.read_local(0, 0, (4,), np.int32).tolist() == [1, 2, 3, 4]


@pytest.mark.parametrize("kind", BACKENDS)
def test_same_dpu_commands_run_in_submission_order(kind):
    hal = make(kind, 1, 64)
    hal.register_kernel("w", _write_kernel(kind))
    for i in range(1, 6):
        last = hal.submit(Command(i, "launch", 0, {"kernel": "w", "offset": 0, "value": [i]}))
    hal.wait(last)
    assert hal.read_local(0, 0, (1,), np.int32)[0] == 5


@pytest.mark.parametrize("kind", BACKENDS)
def test_dma_and_host_paths_return_results_and_propagate_errors(kind):
    hal = make(kind, 1, 32)
    payload = np.arange(4, dtype=np.int32)
    hal.wait(hal.submit(Command(1, "dma_in", 0, {"offset": 0, "data": payload})))
    out = hal.submit(Command(2, "dma_out", 0, {"offset": 0, "shape": payload.shape, "dtype": payload.dtype}))
    assert np.array_equal(hal.wait(out), payload)
    host = hal.submit(Command(3, "host_op", None, {"fn": lambda cmd: cmd.id + 10}))
    assert hal.wait(host) == 13

    def fail_host(cmd):
        raise RuntimeError(f"host failure in cmd {cmd.id}")

    failed = hal.submit(Command(4, "host_op", None, {"fn": fail_host}))
    with pytest.raises(RuntimeError, match="host failure in cmd 4"):
        hal.wait(failed)
    bad = hal.submit(Command(5, "dma_in", 0, {"offset": 24, "data": payload}))
    with pytest.raises(ValueError, match="invalid MRAM range"):
        hal.wait(bad)


@pytest.mark.parametrize("kind", BACKENDS)
def test_duplicate_and_unknown_ids_raise_at_submit(kind):
    hal = make(kind, 1, 32)
    hal.submit(Command(1, "host_op", None, {"fn": lambda c: None}))
    with pytest.raises(ValueError, match="duplicate command id"):
        hal.submit(Command(1, "host_op", None, {"fn": lambda c: None}))
    with pytest.raises(ValueError, match="unknown dependency"):
        hal.submit(Command(2, "host_op", None, {"fn": lambda c: None}, waits=[99]))


@pytest.mark.parametrize("kind", BACKENDS)
def test_dma_in_snapshots_payload_at_submit(kind):
    hal = make(kind, 1, 32)
    payload = np.asarray([1, 2, 3, 4], dtype=np.int32)
    ev = hal.submit(Command(1, "dma_in", 0, {"offset": 0, "data": payload}))
    payload[:] = 99
    hal.wait(ev)
    assert hal.read_local(0, 0, (4,), np.int32).tolist() == [1, 2, 3, 4]


@pytest.mark.parametrize("kind", BACKENDS)
def test_cross_dpu_waits_order_a_consumer_after_its_producer(kind):
    """A dma_out of rank 1 waits for rank 0's producer through its host relay.

    Producer (rank 0, 16 MiB write) -> dma_out rank 0 -> host fn -> dma_in rank 1.
    """
    hal = make(kind, 2, 1 << 25)
    n = 1 << 22
    big = np.arange(n, dtype=np.int32)
    hal.register_kernel("w", _write_kernel(kind))
    e1 = hal.submit(Command(1, "launch", 0, {"kernel": "w", "offset": 0, "value": big.tolist()[:1024]}))
    e2 = hal.submit(Command(2, "dma_out", 0, {"offset": 0, "shape": (1024,), "dtype": np.int32}, waits=[1]))
    got = hal.wait(e2)
    assert np.array_equal(got, big[:1024])
    e3 = hal.submit(Command(3, "dma_in", 1, {"offset": 0, "data": got}, waits=[2]))
    hal.wait(e3)
    assert np.array_equal(hal.read_local(1, 0, (1024,), np.int32), big[:1024])
    assert hal.query(e1)


@pytest.mark.parametrize("kind", BACKENDS)
def test_device_to_device_direct_copy_has_no_api(kind):
    hal = make(kind, 2, 32)
    assert hal.config.allow_device_to_device is False
    assert not hasattr(hal, "copy_dpu_to_dpu")
    with pytest.raises(ValueError, match="device-to-device copies are not supported"):
        make(kind, 2, 32, allow_device_to_device=True)


@pytest.mark.parametrize("kind", BACKENDS)
def test_read_local_returns_a_copy_and_push_xfer_fans_out(kind):
    hal = make(kind, 2, 64)
    payload = np.arange(4, dtype=np.float32)
    hal.push_xfer([(0, 0, payload), (1, 16, payload)])
    host_copy = hal.read_local(0, 0, payload.shape, payload.dtype)
    host_copy[0] = -1
    assert hal.read_local(0, 0, payload.shape, payload.dtype)[0] != -1
    assert np.array_equal(hal.read_local(1, 16, payload.shape, payload.dtype), payload)


@pytest.mark.parametrize("kind", BACKENDS)
def test_llama2_shaped_payload_round_trip(kind):
    act = np.arange(128 * 4096, dtype=np.float16).reshape(1, 128, 4096)
    hal = make(kind, 1, act.nbytes * 2)
    hal.copy_to_dpu(0, 0, act)
    assert np.array_equal(hal.copy_from_dpu(0, 0, act.shape, act.dtype), act)


# --- thread-pool semantics of the oracle HAL (blocking stubs) -------------------------


def test_oracle_submit_is_asynchronous_and_serialises_one_dpu():
    hal = make("oracle", 1, 64)
    started, release = threading.Event(), threading.Event()

    def slow(h, d, cmd):
        started.set()
        release.wait()
        h.write_local(d, 0, np.asarray([1], dtype=np.int32))

    hal.register_kernel("slow", slow)
    hal.register_kernel("w", _write_kernel("oracle"))
    first = hal.submit(Command(1, "launch", 0, {"kernel": "slow"}))
    assert started.wait(1.0)
    second = hal.submit(Command(2, "launch", 0, {"kernel": "w", "offset": 0, "value": [2]}))
    assert not hal.query(first)
    release.set()
    hal.wait(second)
    assert hal.read_local(0, 0, (1,), np.int32)[0] == 2


def test_oracle_waits_block_a_consumer_on_another_dpu():
    hal = make("oracle", 2, 32)
    started, release, ran = threading.Event(), threading.Event(), threading.Event()

    def one(h, d, cmd):
        started.set()
        release.wait()

    def two(h, d, cmd):
        ran.set()

    hal.register_kernel("one", one)
    hal.register_kernel("two", two)
    hal.submit(Command(1, "launch", 0, {"kernel": "one"}))
    assert started.wait(1.0)
    second = hal.submit(Command(2, "launch", 1, {"kernel": "two"}, waits=[1]))
    assert not ran.wait(0.05)
    release.set()
    hal.wait(second)
    assert ran.is_set()
