"""Device collectives for redistribute edges (B200 replacement of comm/lowering.py).

``lower_combine`` compiles the combine command of one redistribute edge into
one device operation that performs the whole edge (collect + combine +
writeback), enqueued on the host stream:

* all_reduce (Partial -> Replicate): ``pim_ordered_sum`` over the collect
  segments in plan order, writing every writeback segment (and the host copy
  when a host node consumes it).  Bit-identical to the sequential in-dtype
  accumulation of comm/lowering.py:137-150;
* all_gather / all_to_all / scatter: one ``pim_batched_copy`` over the run
  intersections of source and destination segments (the segment algebra of
  comm/plan.py; placement is by global range, never by rank id,
  comm/lowering.py:121-129).

With one process per GPU (``torch.distributed``) the same edge becomes an NCCL
all_gather of every rank's collect bytes into a staging buffer followed by the
same ordered sum / placement copies, or -- for all_reduce with
``allreduce="nccl"`` -- a plain NCCL all_reduce (faster, not bit-identical to
the host-star sum), or with ``"p2p"`` one peer-memory kernel; all_to_all is one
NCCL all_to_all of exactly the pieces each peer holds (``all_to_all_layout``).

The redistribute primitives with the reference's ``(entry, engine)``
signatures (``all_reduce``, ``all_gather``, ``all_to_all``, ``scatter``,
``broadcast``) run one edge immediately on a ``CudaBackend`` and return the
host-visible result like comm/lowering.py does.
"""

from __future__ import annotations

import numpy as np
import torch

from backend import _native as nat

_CODE = {"bfloat16": nat.BF16, "float32": nat.F32}


def _dtype_code(entry) -> int:
    name = entry.dtype.name if hasattr(entry.dtype, "name") else str(entry.dtype)
    if name not in _CODE:
        raise NotImplementedError(f"redistribute of dtype {name} has no device kernel")
    return _CODE[name]


def intersections(src_runs, dst_runs, item):
    """``[(src_addr, dst_addr, nbytes)]`` for every overlap of ``(g0, g1, addr)`` runs.

    ``g0, g1`` are flat element ranges of the global tensor; addresses are byte
    addresses of each run's first element.
    """
    out = []
    for dg0, dg1, dad in dst_runs:
        for sg0, sg1, sad in src_runs:
            lo, hi = max(dg0, sg0), min(dg1, sg1)
            if lo < hi:
                out.append((sad + (lo - sg0) * item, dad + (lo - dg0) * item, (hi - lo) * item))
    return out


class CopyTable:
    """A device-resident (src, dst, nbytes) table executed by one batched copy."""

    def __init__(self, device, runs) -> None:
        self.count = len(runs)
        self.max_nbytes = max((r[2] for r in runs), default=0)
        arr = np.zeros((max(self.count, 1), 3), dtype=np.int64)
        for i, (s, d, n) in enumerate(runs):
            arr[i] = (s, d, n)
        self.dev = torch.from_numpy(arr.reshape(-1)).to(device)

    def run(self, stream_handle: int) -> None:
        if self.count:
            nat.check(nat.lib.pim_batched_copy(self.dev.data_ptr(), self.count, self.max_nbytes, stream_handle),
                      "batched copy")


def ordered_sum(srcs, dsts, n, code, mean, st) -> None:
    for i in range(0, len(dsts), 8):
        chunk = dsts[i:i + 8]
        nat.check(nat.lib.pim_ordered_sum(nat.ptr_array(srcs), len(srcs), nat.ptr_array(chunk), len(chunk), n,
                                          code, mean, st), "ordered sum")


def lower_combine(hal, plan, cmd, add_fusion=None):
    p = cmd.payload
    entry = p["entry"]
    kind = p["kind"]
    item = entry.dtype.itemsize
    host_off = p["host_offset"]
    host_buf = hal.host_tensor(plan)
    host_real = host_off < host_buf.numel()
    hb = hal.host_ptr(plan)
    if hal.distributed:
        return _lower_distributed(hal, plan, cmd, entry, kind, item, host_real, hb + host_off, add_fusion)
    if add_fusion is not None:
        raise ValueError("combine_add fusion needs one process per GPU")
    st = hal.host_stream_handle()
    if kind == "all_reduce":
        srcs = [hal.arena_ptr(s.src_dpu) + s.src_addr for s in entry.collect_segments]
        dsts = [hal.arena_ptr(s.dst_dpu) + s.dst_addr for s in entry.writeback_segments]
        if host_real:
            dsts.append(hb + host_off)
        code, mean, n = _dtype_code(entry), int(entry.reduce == "mean"), entry.numel

        def run():
            ordered_sum(srcs, dsts, n, code, mean, st)

        return run
    if kind == "scatter":
        src_runs = [(0, entry.numel, hb + p["src_host"])]
    else:
        src_runs = [(s.global_range[0], s.global_range[1], hal.arena_ptr(s.src_dpu) + s.src_addr)
                    for s in entry.collect_segments]
    dst_runs = [(s.global_range[0], s.global_range[1], hal.arena_ptr(s.dst_dpu) + s.dst_addr)
                for s in entry.writeback_segments]
    if host_real and kind != "scatter":
        dst_runs.append((0, entry.numel, hb + host_off))
    table = CopyTable(hal.host_device, intersections(src_runs, dst_runs, item))

    def run():
        table.run(st)

    run.keep = table
    return run


def distributed_layout(entry, me: int):
    """Static layout of one edge for the process owning rank ``me``.

    Returns ``(pack, chunk, order, per_rank)``: ``pack`` lists my collect
    segments with their byte offset in my send buffer; ``chunk`` is the send
    size of every rank (the largest rank's share); ``order`` is the rank of each
    collect segment in plan order (the all_reduce summation order);
    ``per_rank[r]`` lists rank r's collect segments with their offsets in r's
    slot of the gathered buffer.
    """
    per_rank: dict[int, list] = {}
    for s in entry.collect_segments:
        per_rank.setdefault(s.src_dpu, []).append(s)
    placed = {}
    for r, segs in per_rank.items():
        cur, lst = 0, []
        for s in segs:
            lst.append((s, cur))
            cur += s.nbytes
        placed[r] = lst
    chunk = max(sum(s.nbytes for s in v) for v in per_rank.values())
    order = [s.src_dpu for s in entry.collect_segments]
    return placed.get(me, []), chunk, order, placed


def all_to_all_layout(entry, me: int):
    """Static layout of an all_to_all edge for the process owning rank ``me``.

    Returns ``(send, recv, local)``: ``send[q]`` lists the ``(src_addr, nbytes)`` pieces of
    my collect segments that rank q's writeback segments hold, ``recv[r]`` the
    ``(dst_addr, nbytes)`` pieces of my writeback segments that rank r's collect segments
    hold, and ``local`` the ``(src_addr, dst_addr, nbytes)`` pieces that stay on this rank.
    Pieces of one (sender, receiver) pair are in global element order on both sides, so
    the sender packs them and the receiver places them in the same order.
    """
    item = entry.dtype.itemsize
    by_src: dict[int, list] = {}
    by_dst: dict[int, list] = {}
    for s in entry.collect_segments:
        by_src.setdefault(s.src_dpu, []).append((s.global_range[0], s.global_range[1], s.src_addr))
    for w in entry.writeback_segments:
        by_dst.setdefault(w.dst_dpu, []).append((w.global_range[0], w.global_range[1], w.dst_addr))
    for runs in (*by_src.values(), *by_dst.values()):
        runs.sort()
        if any(runs[i][1] > runs[i + 1][0] for i in range(len(runs) - 1)):
            raise ValueError(f"all_to_all edge {entry.edge_id}: one rank's segments overlap")

    def pieces(r, q):  # merge of two sorted lists of disjoint runs, in global order
        a, b = by_src.get(r, []), by_dst.get(q, [])
        out, i, j = [], 0, 0
        while i < len(a) and j < len(b):
            (s0, s1, sa), (d0, d1, da) = a[i], b[j]
            lo, hi = max(s0, d0), min(s1, d1)
            if lo < hi:
                out.append((sa + (lo - s0) * item, da + (lo - d0) * item, (hi - lo) * item))
            if s1 <= d1:
                i += 1
            else:
                j += 1
        return out

    ranks = sorted(by_src.keys() | by_dst.keys())
    send = {q: [(sa, nb) for sa, _, nb in pieces(me, q)] for q in ranks if q != me}
    recv = {r: [(da, nb) for _, da, nb in pieces(r, me)] for r in ranks if r != me}
    return send, recv, pieces(me, me)


def split_allreduce_layout(entry, n_ranks: int):
    """Slices of the bit-exact split all_reduce, or None when the edge does not take it.

    Every rank r holds a whole partial (one collect segment of the whole tensor); the
    flat element range is cut into ``n_ranks`` slices of ``width`` elements (a multiple of
    8, so every slice starts 16-byte aligned; the last one is shorter).  Rank q receives
    slice q of every partial (one all_to_all), adds them in plan order -- per element the
    same rounded additions as the whole-tensor sum -- and an all_gather of the ``width``-
    element sums assembles the result.  Returns ``(width, lengths, order)``: ``lengths[q]``
    is slice q's element count, ``order`` the ranks in summation order.
    """
    n = entry.numel
    order = [s.src_dpu for s in entry.collect_segments]
    whole = all(s.nbytes == n * entry.dtype.itemsize for s in entry.collect_segments)
    if not whole or sorted(order) != list(range(n_ranks)):
        return None
    width = -(-n // n_ranks)
    width = -(-width // 8) * 8
    lengths = [max(0, min(width, n - q * width)) for q in range(n_ranks)]
    if min(lengths) == 0:
        return None
    return width, lengths, order


def _lower_split_allreduce(hal, entry, me, n_ranks, st_obj, dsts, layout):
    """Bit-exact all_reduce as all_to_all of slices + rank-order slice sum + all_gather."""
    import torch.distributed as dist

    st = st_obj.cuda_stream
    width, lengths, order = layout
    item = entry.dtype.itemsize
    n = entry.numel
    (mine,) = [s for s in entry.collect_segments if s.src_dpu == me]
    src = hal.arena(me)[mine.src_addr:mine.src_addr + n * item]
    mine_len = lengths[me]
    recv = torch.empty(n_ranks * mine_len * item, dtype=torch.uint8, device=hal.host_device)
    part = torch.zeros(width * item, dtype=torch.uint8, device=hal.host_device)
    gathered = torch.empty(n_ranks * width * item, dtype=torch.uint8, device=hal.host_device)
    in_split = [ln * item for ln in lengths]
    out_split = [mine_len * item] * n_ranks
    srcs = [recv.data_ptr() + r * mine_len * item for r in order]
    code, mean = _dtype_code(entry), int(entry.reduce == "mean")

    def run_split():
        with torch.cuda.stream(st_obj):
            dist.all_to_all_single(recv, src, out_split, in_split)
        ordered_sum(srcs, [part.data_ptr()], mine_len, code, mean, st)
        with torch.cuda.stream(st_obj):
            dist.all_gather_into_tensor(gathered, part)
        for d in dsts:
            nat.check(nat.lib.pim_copy(d, gathered.data_ptr(), n * item, st), "copy")

    run_split.keep = (recv, part, gathered, src)
    return run_split


def _lower_all_to_all(hal, entry, me, n_ranks, st_obj):
    """Shard(i) -> Shard(j) with one NCCL all_to_all: each rank sends every peer only the
    pieces that peer holds ((N-1)/N^2 of the tensor per rank, not the all_gather's (N-1)/N)."""
    import torch.distributed as dist

    st = st_obj.cuda_stream
    base = hal.arena_ptr(me)
    send_l, recv_l, local_l = all_to_all_layout(entry, me)
    in_split = [sum(nb for _, nb in send_l.get(q, [])) for q in range(n_ranks)]
    out_split = [sum(nb for _, nb in recv_l.get(r, [])) for r in range(n_ranks)]
    send = torch.empty(max(sum(in_split), 16), dtype=torch.uint8, device=hal.host_device)
    recv = torch.empty(max(sum(out_split), 16), dtype=torch.uint8, device=hal.host_device)
    pack, off = [], 0
    for q in range(n_ranks):
        for sa, nb in send_l.get(q, []):
            pack.append((base + sa, send.data_ptr() + off, nb))
            off += nb
    place, off = [], 0
    for r in range(n_ranks):
        for da, nb in recv_l.get(r, []):
            place.append((recv.data_ptr() + off, base + da, nb))
            off += nb
    pack_t = CopyTable(hal.host_device, pack + [(base + sa, base + da, nb) for sa, da, nb in local_l])
    place_t = CopyTable(hal.host_device, place)
    s_in, s_out = send[:sum(in_split)], recv[:sum(out_split)]

    def run_all_to_all():
        pack_t.run(st)
        with torch.cuda.stream(st_obj):
            dist.all_to_all_single(s_out, s_in, out_split, in_split)
        place_t.run(st)

    run_all_to_all.keep = (send, recv, pack_t, place_t)
    return run_all_to_all


def _lower_distributed(hal, plan, cmd, entry, kind, item, host_real, host_addr, add_fusion=None):
    import torch.distributed as dist

    me = hal.local[0]
    n_ranks = hal.config.num_dpus
    st_obj = hal.host_stream()
    st = st_obj.cuda_stream
    base = hal.arena_ptr(me)
    my_wb = [s for s in entry.writeback_segments if s.dst_dpu == me]
    dst_runs = [(s.global_range[0], s.global_range[1], base + s.dst_addr) for s in my_wb]
    if host_real and kind != "scatter":
        dst_runs.append((0, entry.numel, host_addr))
    if kind == "scatter":
        src_runs = [(0, entry.numel, hal.host_ptr(plan) + cmd.payload["src_host"])]
        table = CopyTable(hal.host_device, intersections(src_runs, dst_runs, item))
        return lambda: table.run(st)
    if kind == "all_to_all" and not host_real:
        return _lower_all_to_all(hal, entry, me, n_ranks, st_obj)
    mine, chunk, order, placed = distributed_layout(entry, me)
    send = torch.empty(chunk, dtype=torch.uint8, device=hal.host_device)
    recv = torch.empty(chunk * n_ranks, dtype=torch.uint8, device=hal.host_device)
    pack_t = CopyTable(hal.host_device, [(base + s.src_addr, send.data_ptr() + off, s.nbytes) for s, off in mine])
    # A rank whose collect bytes are one contiguous run of the exchanged size (every
    # decode all_reduce: the linear's whole partial) sends them from the arena itself.
    direct = len(mine) == 1 and mine[0][0].nbytes == chunk
    gsrc = hal.arena(me)[mine[0][0].src_addr:mine[0][0].src_addr + chunk] if direct else send
    if kind == "all_reduce":
        srcs = [recv.data_ptr() + r * chunk for r in order]
        dsts = [d for _, _, d in dst_runs]
        code, mean, n = _dtype_code(entry), int(entry.reduce == "mean"), entry.numel
        g = hal._p2p
        ll = hal.config.allreduce == "p2p"  # P2P mode: the low-latency protocol (8 buffer bytes per 4 data bytes)
        if (g is not None and not mean and order == list(range(n_ranks)) and g.fits((2 if ll else 1) * n * item)
                and 1 <= len(dsts) <= 4):
            # one kernel: partials straight into every rank's exchange buffer over NVLink,
            # then the rank-order sum (same bits as the all_gather + ordered sum below)
            single = len(mine) == 1 and mine[0][0].nbytes == n * item
            src = base + mine[0][0].src_addr if single else send.data_ptr()
            dst_arr = nat.ptr_array(dsts)
            err = hal.error_flag_ptr(me) + 8
            counter = g.counter.data_ptr()
            if ll:
                if add_fusion is not None:  # the residual add that reads the sum, in the same kernel
                    _, res_off, y_off, sum_off = add_fusion
                    res_p, y_p = base + res_off, base + y_off
                    sum_p = base + sum_off if sum_off is not None else None
                else:
                    res_p = y_p = None
                    sum_p = dsts[0]
                extra = list(dsts[1:]) if add_fusion is None else []

                def run_ll():
                    if not single:
                        pack_t.run(st)
                    nat.check(nat.lib.pim_allreduce_p2p_ll(src, res_p, y_p, sum_p, n, code, g.rank, g.size, g.ptrs,
                                                           g.capacity, counter, err, st), "allreduce_p2p_ll")
                    for d in extra:  # further destinations of the sum (the host copy of the logits)
                        nat.check(nat.lib.pim_copy(d, sum_p, n * item, st), "copy")

                run_ll.keep = (send, pack_t)
                return run_ll
            if add_fusion is not None:  # the residual add that reads the sum, in the same kernel
                _, res_off, y_off, sum_off = add_fusion
                res_p, y_p = base + res_off, base + y_off
                sum_p = base + sum_off if sum_off is not None else None

                def run_p2p_add():
                    if not single:
                        pack_t.run(st)
                    nat.check(nat.lib.pim_allreduce_p2p_add(src, res_p, y_p, sum_p, n, code, g.rank, g.size, g.ptrs,
                                                            g.capacity, counter, err, st), "allreduce_p2p + add")

                run_p2p_add.keep = (send, pack_t)
                return run_p2p_add

            def run_p2p():
                if not single:
                    pack_t.run(st)
                nat.check(nat.lib.pim_allreduce_p2p(src, dst_arr, len(dsts), n, code, g.rank, g.size, g.ptrs,
                                                    g.capacity, counter, err, st), "allreduce_p2p")

            run_p2p.keep = (send, pack_t, dst_arr)
            return run_p2p
        split = hal.config.allreduce_split_bytes
        if hal.config.allreduce != "nccl" and split and n * item >= split:
            layout = split_allreduce_layout(entry, n_ranks)
            if layout is not None:
                return _lower_split_allreduce(hal, entry, me, n_ranks, st_obj, dsts, layout)
        if hal.config.allreduce == "nccl":
            tdt = torch.bfloat16 if code == nat.BF16 else torch.float32

            def run_nccl():
                pack_t.run(st)
                with torch.cuda.stream(st_obj):
                    t = send.view(tdt)
                    dist.all_reduce(t)
                    if mean:
                        t.div_(len(order))
                for d in dsts:
                    nat.check(nat.lib.pim_copy(d, send.data_ptr(), n * item, st), "copy")

            run_nccl.keep = (send, recv, pack_t)
            return run_nccl

        if add_fusion is not None:  # the residual add that reads the sum, in the same kernel
            _, res_off, y_off, sum_off = add_fusion
            src_arr = nat.ptr_array(srcs)
            res_p, y_p = base + res_off, base + y_off
            sum_p = base + sum_off if sum_off is not None else None

            def run_ordered_add():
                if not direct:
                    pack_t.run(st)
                with torch.cuda.stream(st_obj):
                    dist.all_gather_into_tensor(recv, gsrc)
                nat.check(nat.lib.pim_ordered_sum_add(src_arr, len(srcs), res_p, y_p, sum_p, n, code, st),
                          "ordered sum + add")

            run_ordered_add.keep = (send, recv, pack_t, gsrc, src_arr)
            return run_ordered_add

        def run_ordered():
            if not direct:
                pack_t.run(st)
            with torch.cuda.stream(st_obj):
                dist.all_gather_into_tensor(recv, gsrc)
            ordered_sum(srcs, dsts, n, code, mean, st)

        run_ordered.keep = (send, recv, pack_t, gsrc)
        return run_ordered
    src_runs = [(s.global_range[0], s.global_range[1], recv.data_ptr() + r * chunk + off)
                for r, lst in placed.items() for s, off in lst]
    place = CopyTable(hal.host_device, intersections(src_runs, dst_runs, item))

    def run_gather():
        if not direct:
            pack_t.run(st)
        with torch.cuda.stream(st_obj):
            dist.all_gather_into_tensor(recv, gsrc)
        place.run(st)

    run_gather.keep = (send, recv, pack_t, place, gsrc)
    return run_gather


# ---------------------------------------------------------------------------
# (entry, engine) primitives with the signatures of comm/lowering.py:137-194
# ---------------------------------------------------------------------------


class CudaDmaEngine:
    """Engine argument of the primitives: wraps a single-process CudaBackend."""

    def __init__(self, hal) -> None:
        if hal.distributed:
            raise ValueError("the immediate primitives need every rank in this process")
        self.hal = hal


def _run_edge(entry, engine, kind, host_buf=None) -> np.ndarray:
    hal = engine.hal if isinstance(engine, CudaDmaEngine) else engine
    item = entry.dtype.itemsize
    size = entry.numel * item
    host = torch.zeros(max(size, 16), dtype=torch.uint8, device=hal.host_device)
    hb = host.data_ptr()
    st = hal.host_stream_handle()
    hal.synchronize()
    torch.cuda.synchronize(hal.host_device)  # the zero fill above ran on the default stream
    if kind == "all_reduce":
        srcs = [hal.arena_ptr(s.src_dpu) + s.src_addr for s in entry.collect_segments]
        dsts = [hal.arena_ptr(s.dst_dpu) + s.dst_addr for s in entry.writeback_segments] + [hb]
        ordered_sum(srcs, dsts, entry.numel, _dtype_code(entry), int(entry.reduce == "mean"), st)
    else:
        if host_buf is not None:
            flat = np.ascontiguousarray(host_buf, dtype=entry.dtype).reshape(-1)
            if flat.size != entry.numel:
                raise ValueError(f"{entry.type} host_buf has {flat.size} elements, entry has {entry.numel}")
            host[:size].copy_(torch.from_numpy(flat.view(np.uint8).copy()).to(hal.host_device))
            torch.cuda.synchronize(hal.host_device)
            src_runs = [(0, entry.numel, hb)]
        else:
            src_runs = [(s.global_range[0], s.global_range[1], hal.arena_ptr(s.src_dpu) + s.src_addr)
                        for s in entry.collect_segments]
        dst_runs = [(s.global_range[0], s.global_range[1], hal.arena_ptr(s.dst_dpu) + s.dst_addr)
                    for s in entry.writeback_segments]
        if host_buf is None:
            dst_runs.append((0, entry.numel, hb))
        table = CopyTable(hal.host_device, intersections(src_runs, dst_runs, item))
        torch.cuda.synchronize(hal.host_device)  # the descriptor upload ran on the default stream
        table.run(st)
    hal.host_stream().synchronize()
    return host[:size].cpu().numpy().view(entry.dtype).reshape(entry.shape)


def _check(entry, expect):
    if entry.type != expect:
        raise ValueError(f"{expect} received an entry of type {entry.type} (edge {entry.edge_id})")


def all_reduce(entry, engine) -> np.ndarray:
    _check(entry, "all_reduce")
    return _run_edge(entry, engine, "all_reduce")


def all_gather(entry, engine) -> np.ndarray:
    _check(entry, "all_gather")
    return _run_edge(entry, engine, "all_gather")


def all_to_all(entry, engine) -> np.ndarray:
    _check(entry, "all_to_all")
    return _run_edge(entry, engine, "all_to_all")


def scatter(entry, engine, host_buf) -> None:
    _check(entry, "scatter")
    _run_edge(entry, engine, "scatter", host_buf)


def broadcast(entry, engine, host_buf) -> None:
    _run_edge(entry, engine, "scatter", host_buf)
