"""One process per rank (world size 2 and 4, gloo on CPU): the host logic of the
distributed redistribute path.

In ``torchrun`` mode each process owns one rank; ``backend.cuda_collectives``
lowers a combine edge into: pack my collect segments into a send chunk
(``distributed_layout``), all_gather the chunks, then place the gathered segments
into my writeback segments (``intersections``), or, for all_reduce, add the ranks'
partials in plan order with an RNE rounding after every add; all_to_all packs the
pieces each peer holds (``all_to_all_layout``), exchanges them with one
all_to_all and places what each sender sent.  Here the same
functions run over CPU byte buffers with a gloo all_gather, and every rank's
destination bytes must equal the oracle's host-star lowering (comm/lowering.py).
"""

from __future__ import annotations

import os
import socket
from pathlib import Path

import numpy as np
import pytest

from helpers import comm_inputs, redistribute_entry

HIDDEN = 512


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _load(kind, n, t, data, nbytes):
    """Per-rank source bytes at arena offset 0 (the layout redistribute_entry builds)."""
    arenas = [np.zeros(4 * nbytes, np.uint8) for _ in range(n)]
    for d in range(n):
        if kind == "all_reduce":
            src = data[d]
        elif kind == "all_gather":
            w = HIDDEN // n
            src = data[:, d * w:(d + 1) * w]
        else:
            r = t // n
            src = data[d * r:(d + 1) * r, :]
        b = np.ascontiguousarray(src).reshape(-1).view(np.uint8)
        arenas[d][:b.size] = b
    return arenas


def _rank_main(rank, world, kind, t, port, out_dir):
    import ml_dtypes
    import torch
    import torch.distributed as dist

    from backend.cuda_collectives import all_to_all_layout, distributed_layout, intersections

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        entry, nbytes = redistribute_entry(kind, world, (t, HIDDEN))
        arena = _load(kind, world, t, comm_inputs(kind, world, t, hidden=HIDDEN, seed=3), nbytes)[rank]
        item = entry.dtype.itemsize
        if kind == "all_to_all":  # pack per peer, one all_to_all, place per sender
            send_l, recv_l, local_l = all_to_all_layout(entry, rank)
            send = np.concatenate([arena[sa:sa + nb] for q in range(world) for sa, nb in send_l.get(q, [])]
                                  or [np.zeros(0, np.uint8)])
            in_split = [sum(nb for _, nb in send_l.get(q, [])) for q in range(world)]
            out_split = [sum(nb for _, nb in recv_l.get(r, [])) for r in range(world)]
            recv = torch.zeros(sum(out_split), dtype=torch.uint8)
            dist.all_to_all_single(recv, torch.from_numpy(send), out_split, in_split)
            recv = recv.numpy()
            for sa, da, nb in local_l:
                arena[da:da + nb] = arena[sa:sa + nb]
            off = 0
            for r in range(world):
                for da, nb in recv_l.get(r, []):
                    arena[da:da + nb] = recv[off:off + nb]
                    off += nb
            np.save(Path(out_dir) / f"rank{rank}.npy", arena)
            return
        mine, chunk, order, placed = distributed_layout(entry, rank)
        send = np.zeros(chunk, np.uint8)
        for s, off in mine:
            send[off:off + s.nbytes] = arena[s.src_addr:s.src_addr + s.nbytes]
        parts = [torch.zeros(chunk, dtype=torch.uint8) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(send))
        recv = np.concatenate([p.numpy() for p in parts])
        my_wb = [s for s in entry.writeback_segments if s.dst_dpu == rank]
        if kind == "all_reduce":
            n = entry.numel
            acc = np.zeros(n, ml_dtypes.bfloat16)
            for r in order:  # plan order, fp32 add then round to bf16 after every add
                part = recv[r * chunk:r * chunk + n * item].view(ml_dtypes.bfloat16)
                acc = (acc.astype(np.float32) + part.astype(np.float32)).astype(ml_dtypes.bfloat16)
            for s in my_wb:
                arena[s.dst_addr:s.dst_addr + s.nbytes] = acc.view(np.uint8)[:s.nbytes]
        else:
            # virtual addresses: recv at 1 << 40, the arena at 0
            vrecv = 1 << 40
            src_runs = [(s.global_range[0], s.global_range[1], vrecv + r * chunk + off)
                        for r, lst in placed.items() for s, off in lst]
            dst_runs = [(s.global_range[0], s.global_range[1], s.dst_addr) for s in my_wb]
            for sa, da, nb in intersections(src_runs, dst_runs, item):
                arena[da:da + nb] = recv[sa - vrecv:sa - vrecv + nb]
        np.save(Path(out_dir) / f"rank{rank}.npy", arena)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("kind,world,t", [("all_gather", 2, 16), ("all_reduce", 2, 16), ("all_reduce", 4, 1),
                                          ("all_to_all", 2, 16), ("all_to_all", 4, 16)])
def test_distributed_combine_host_logic_matches_oracle(kind, world, t, tmp_path):
    import torch.multiprocessing as mp

    from oracle import lowering
    from oracle.hal_numpy import NumpyBackend, NumpyBackendConfig

    mp.spawn(_rank_main, args=(world, kind, t, _free_port(), str(tmp_path)), nprocs=world, join=True)

    entry, nbytes = redistribute_entry(kind, world, (t, HIDDEN))
    data = comm_inputs(kind, world, t, hidden=HIDDEN, seed=3)
    ora = lowering.DmaEngine(NumpyBackend(NumpyBackendConfig(world, 4 * nbytes)))
    for d, arena in enumerate(_load(kind, world, t, data, nbytes)):
        ora.hal.copy_to_dpu(d, 0, arena[:nbytes])
    getattr(lowering, kind)(entry, ora)
    for d in range(world):
        got = np.load(tmp_path / f"rank{d}.npy")
        for s in (s for s in entry.writeback_segments if s.dst_dpu == d):
            ref = ora.hal.read_local(d, s.dst_addr, (s.nbytes,), np.uint8)
            assert np.array_equal(got[s.dst_addr:s.dst_addr + s.nbytes], ref), (kind, d)
    ora.hal.close()


@pytest.mark.parametrize("world,t", [(2, 16), (4, 256), (8, 2048)])
def test_all_to_all_layout_moves_only_what_each_peer_holds(world, t):
    """Senders and receivers agree piece by piece, and each rank sends (N-1)/N^2 of the tensor."""
    from backend.cuda_collectives import all_to_all_layout

    entry, nbytes = redistribute_entry("all_to_all", world, (t, HIDDEN))
    lay = {r: all_to_all_layout(entry, r) for r in range(world)}
    for r in range(world):
        send, _, local = lay[r]
        assert sum(nb for q in send for _, nb in send[q]) == nbytes * (world - 1) // world ** 2
        assert sum(nb for _, _, nb in local) == nbytes // world ** 2
        for q in range(world):
            if q != r:
                assert [nb for _, nb in send[q]] == [nb for _, nb in lay[q][1][r]]


def _split_rank_main(rank, world, t, port, out_dir):
    """The split all_reduce's host logic: all_to_all of slices, rank-order sum, all_gather."""
    import ml_dtypes
    import torch
    import torch.distributed as dist

    from backend.cuda_collectives import split_allreduce_layout

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        entry, nbytes = redistribute_entry("all_reduce", world, (t, HIDDEN))
        arena = _load("all_reduce", world, t, comm_inputs("all_reduce", world, t, hidden=HIDDEN, seed=3), nbytes)[rank]
        width, lengths, order = split_allreduce_layout(entry, world)
        item = 2
        (mine,) = [s for s in entry.collect_segments if s.src_dpu == rank]
        src = torch.from_numpy(arena[mine.src_addr:mine.src_addr + entry.numel * item].copy())
        recv = torch.zeros(world * lengths[rank] * item, dtype=torch.uint8)
        dist.all_to_all_single(recv, src, [lengths[rank] * item] * world, [ln * item for ln in lengths])
        blocks = recv.numpy().view(ml_dtypes.bfloat16).reshape(world, lengths[rank])
        acc = np.zeros(lengths[rank], ml_dtypes.bfloat16)
        for r in order:  # plan order, fp32 add then round to bf16 after every add
            acc = (acc.astype(np.float32) + blocks[r].astype(np.float32)).astype(ml_dtypes.bfloat16)
        part = np.zeros(width, ml_dtypes.bfloat16)
        part[:lengths[rank]] = acc
        parts = [torch.zeros(width * item, dtype=torch.uint8) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(part.view(np.uint8).copy()))
        full = np.concatenate([p.numpy() for p in parts])[:entry.numel * item]
        for s in (s for s in entry.writeback_segments if s.dst_dpu == rank):
            arena[s.dst_addr:s.dst_addr + s.nbytes] = full[:s.nbytes]
        np.save(Path(out_dir) / f"rank{rank}.npy", arena)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,t", [(2, 16), (4, 3)])
def test_split_allreduce_host_logic_is_bit_exact(world, t, tmp_path):
    """Slice-wise rank-order sums + all_gather == the oracle's whole-tensor sequential sum."""
    import torch.multiprocessing as mp

    from oracle import lowering
    from oracle.hal_numpy import NumpyBackend, NumpyBackendConfig

    mp.spawn(_split_rank_main, args=(world, t, _free_port(), str(tmp_path)), nprocs=world, join=True)
    entry, nbytes = redistribute_entry("all_reduce", world, (t, HIDDEN))
    data = comm_inputs("all_reduce", world, t, hidden=HIDDEN, seed=3)
    ora = lowering.DmaEngine(NumpyBackend(NumpyBackendConfig(world, 4 * nbytes)))
    for d, arena in enumerate(_load("all_reduce", world, t, data, nbytes)):
        ora.hal.copy_to_dpu(d, 0, arena[:nbytes])
    lowering.all_reduce(entry, ora)
    for d in range(world):
        got = np.load(tmp_path / f"rank{d}.npy")
        for s in (s for s in entry.writeback_segments if s.dst_dpu == d):
            ref = ora.hal.read_local(d, s.dst_addr, (s.nbytes,), np.uint8)
            assert np.array_equal(got[s.dst_addr:s.dst_addr + s.nbytes], ref), d
    ora.hal.close()


def test_split_allreduce_layout_slices():
    from backend.cuda_collectives import split_allreduce_layout

    entry, _ = redistribute_entry("all_reduce", 8, (1, 4096))
    width, lengths, order = split_allreduce_layout(entry, 8)
    assert width == 512 and lengths == [512] * 8 and order == list(range(8))
    entry, _ = redistribute_entry("all_reduce", 4, (3, HIDDEN))  # 1536 elements: 384 each
    assert split_allreduce_layout(entry, 4)[1] == [384] * 4
    entry, _ = redistribute_entry("all_reduce", 4, (1, 40))  # 40 elements: widths of 16 leave rank 3 empty
    assert split_allreduce_layout(entry, 4) is None
    entry, _ = redistribute_entry("all_gather", 2, (4, HIDDEN))  # not whole partials
    assert split_allreduce_layout(entry, 2) is None
