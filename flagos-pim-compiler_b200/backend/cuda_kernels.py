"""Lowering of ExecutionPlan commands to C-ABI launches (B200 HAL side).

``lower_launch`` turns one ``launch`` command of a rank into a zero-argument
callable that enqueues the matching libpim_b200 entry point on the rank's
stream; ``lower_host_op`` does the same for the plan's host nodes, whose
buffers live in the plan's device-resident host arena.  Argument structs are
built once here (at ``register_plan``), so executing a command is one ctypes
call.  Every op of the step graph has a native implementation; an unknown op
raises instead of falling back.
"""

from __future__ import annotations

import ctypes

from backend import _native as nat

_ITEM = {"float32": 4, "bfloat16": 2, "int32": 4}


def _dt(name: str) -> int:
    if name not in nat.DTYPE_CODE:
        raise NotImplementedError(f"dtype {name} has no B200 kernel")
    return nat.DTYPE_CODE[name]


def _numel(shape) -> int:
    n = 1
    for s in shape:
        n *= int(s)
    return n


def _allreduce_args(hal, rank: int, lin, add, sum_in_add: int, sum_offset: int | None):
    """``pim_projection_args`` of a ``linear`` -> Partial->Replicate all_reduce -> ``add``
    chain at TP > 1: the linear command's x and weight, the add's other input (not
    ``sum_in_add``, where the add reads the sum) as the residual and the add's output as
    the output; the all-reduced sum also goes to ``sum_offset`` (the combine's writeback)
    when another command reads it.  See pim_projection_args.p2p_desc."""
    base = hal.arena_ptr(rank)
    x, w = lin.payload["inputs"][:2]
    lin_out = lin.payload["output"]
    res = next(r for r in add.payload["inputs"] if r[0] != sum_in_add)
    out_off, out_shape, out_dt = add.payload["output"]
    a = nat.ProjectionArgs()
    a.x, a.weight, a.out = base + x[0], base + w[0], base + out_off
    a.rows, a.k, a.ncols = _numel(x[1][:-1]), x[1][-1], w[1][0]
    a.residual = base + res[0]
    a.err_flag = hal.error_flag_ptr(rank) + 4
    a.p2p_desc = hal._p2p.descriptor(hal.error_flag_ptr(rank) + 8)
    a.allreduce_out = base + sum_offset if sum_offset is not None else None
    if _numel(lin_out[1]) != _numel(out_shape) or lin_out[2] != out_dt:
        raise ValueError(f"{lin.payload.get('node')}: linear and add outputs differ")
    return a


def lower_linear_allreduce(hal, rank: int, lin, add, sum_in_add: int, sum_offset: int | None):
    """One launch for ``linear`` -> Partial->Replicate all_reduce -> ``add`` at TP > 1
    (``_allreduce_args``)."""
    st = hal.stream_handle(rank)
    a = _allreduce_args(hal, rank, lin, add, sum_in_add, sum_offset)
    ref, code = ctypes.byref(a), _dt(add.payload["output"][2])
    node = f"{lin.payload.get('node')}+all_reduce+{add.payload.get('node')}"
    # the dynamic-assignment kernel's work counter, when that kernel is selected
    need = nat.lib.pim_projection_scratch_bytes(ref, code, nat.PROJ_PLAIN)
    scratch, sbytes = hal.scratch(rank, need, pool="gemv_counter")

    def run():
        nat.check(nat.lib.pim_projection(ref, code, nat.PROJ_PLAIN, scratch, sbytes, st), node)

    run.keep = a
    return run


_PROJECTIONS = ("attn_in", "mlp_in", "lm_head_in", "linear", "linear_add")


def projection_args(hal, rank: int, cmd, attn_fusion=None):
    """The ``pim_projection_args`` of a projection command: (args, mode, dtype code).

    ``attn_fusion``: the decode ``attention`` command that this ``attn_in`` computes too.
    """
    p = cmd.payload
    op = p["kernel"]
    base = hal.arena_ptr(rank)
    ins = p["inputs"]
    out_off, out_shape, out_dt = p["output"]

    def addr(ref):
        return base + ref[0]

    x = ins[0]
    a = nat.ProjectionArgs()
    a.x, a.out, a.rows, a.k = addr(x), base + out_off, _numel(x[1][:-1]), x[1][-1]
    a.err_flag = hal.error_flag_ptr(rank) + 4  # slot 1 of the rank's error flags
    if op in ("linear", "linear_add"):
        w = ins[1]
        a.norm_weight, a.weight, a.ncols, mode = None, addr(w), w[1][0], nat.PROJ_PLAIN
        if op == "linear_add":
            a.residual = addr(ins[2])
    else:
        a.norm_weight, a.weight, a.eps = addr(ins[1]), addr(ins[2]), float(p["attrs"]["eps"])
        if op == "lm_head_in":
            a.ncols, mode = ins[2][1][0], nat.PROJ_PLAIN
        elif op == "mlp_in":
            a.inter, a.ncols, mode = out_shape[-1], ins[2][1][0], nat.PROJ_SILU_MUL
        else:
            kv = p["kv"]
            item = _ITEM[kv["dtype"]]
            hd = kv["head_dim"]
            a.rope_cos, a.rope_sin, a.positions = addr(ins[3]), addr(ins[4]), addr(ins[5])
            a.seq = x[1][1]
            a.q_heads = out_shape[-1] // hd
            a.kv_heads = len(kv["kv_heads"])
            a.head_dim, a.max_seq = hd, kv["max_seq"]
            a.kv_base = base + kv["layer_base"]
            a.kv_block_stride = kv["block_stride"] // item
            a.kv_seq_stride = kv["seq_stride"] // item
            a.ncols = ins[2][1][0]
            mode = nat.PROJ_ROPE_KV
            if attn_fusion is not None:  # the layer's decode attention at the end of the launch
                a.attn_out = base + attn_fusion.payload["output"][0]
                a.attn_counters = hal.scratch(rank, 4 * a.q_heads, pool="attn_heads")[0]
    return a, mode, _dt(x[2])


def _layer_args(hal, rank: int, chain, allreduces):
    """The four ``pim_projection_args`` of a fused decode layer (``lower_decode_layer``)."""
    attn_in, attention, o_proj, mlp_in, down = chain
    if allreduces is None:
        o_args, d_args = (projection_args(hal, rank, c)[0] for c in (o_proj, down))
    else:
        (_, _, o_add, o_in, o_sum), (_, _, d_add, d_in, d_sum) = allreduces
        o_args = _allreduce_args(hal, rank, o_proj, o_add, o_in, o_sum)
        d_args = _allreduce_args(hal, rank, down, d_add, d_in, d_sum)
    return [projection_args(hal, rank, attn_in, attention)[0], o_args, projection_args(hal, rank, mlp_in)[0], d_args]


class _StepPlan:
    """Owns a ``pim_decode_step_plan`` (host memory of the library) and its table."""

    def __init__(self, ptr: int, keep) -> None:
        self.ptr, self.keep = ptr, keep

    def __del__(self):
        if self.ptr and nat is not None and nat.lib is not None:
            nat.lib.pim_decode_step_free(self.ptr)
        self.ptr = 0


def lower_decode_step(hal, rank: int, run, head):
    """One launch for a whole decode step: the fused layers of ``run`` ([(chain,
    all-reduces)], as ``lower_decode_layer`` takes them) and the ``lm_head_in`` command
    ``head``: ``pim_decode_step_prepare`` (now, outside any capture) + ``pim_decode_step``."""
    args = [a for chain, ar in run for a in _layer_args(hal, rank, chain, ar)]
    head_args = projection_args(hal, rank, head)[0]
    code = _dt(run[0][0][0].payload["inputs"][0][2])
    ptrs = (ctypes.POINTER(nat.ProjectionArgs) * len(args))(*[ctypes.pointer(a) for a in args])
    n = len(run)
    need = nat.lib.pim_decode_step_table_bytes(n)
    table, tbytes = hal.scratch(rank, need, pool=("decode_step_table", id(run[0][0][0])))
    handle = ctypes.c_void_p()
    node = f"{run[0][0][0].payload.get('node')}..{head.payload.get('node')}"
    nat.check(nat.lib.pim_decode_step_prepare(ptrs, n, ctypes.byref(head_args), code, table, tbytes,
                                              ctypes.byref(handle)), node)
    plan = _StepPlan(handle.value, (args, head_args, ptrs))
    bar = hal.scratch(rank, nat.DECODE_LAYER_BARRIER_BYTES, pool="decode_layer_barrier")[0]
    err = hal.error_flag_ptr(rank) + 12  # slot 3 of the rank's error flags
    st = hal.stream_handle(rank)

    def run_step():
        nat.check(nat.lib.pim_decode_step(plan.ptr, bar, err, st), node)

    run_step.keep = plan
    return run_step


def lower_decode_layer(hal, rank: int, chain, allreduces=None):
    """One launch for a decode layer's five commands at one activation row:
    ``pim_decode_layer``.  ``chain``: attn_in, attention, o_proj, mlp_in, down_proj;
    ``allreduces`` (TP > 1): the fused all-reduce chains (linear, combine, add, sum
    offset read by the add, sum offset to write) that o_proj and down_proj head."""
    attn_in, down = chain[0], chain[4]
    args = _layer_args(hal, rank, chain, allreduces)
    code = _dt(attn_in.payload["inputs"][0][2])
    refs = [ctypes.byref(a) for a in args]
    bar = hal.scratch(rank, nat.DECODE_LAYER_BARRIER_BYTES, pool="decode_layer_barrier")[0]
    err = hal.error_flag_ptr(rank) + 12  # slot 3 of the rank's error flags
    st = hal.stream_handle(rank)
    node = f"{attn_in.payload.get('node')}..{down.payload.get('node')}"

    def run():
        nat.check(nat.lib.pim_decode_layer(*refs, bar, err, code, st), node)

    run.keep = args
    return run


def lower_launch(hal, rank: int, cmd, attn_fusion=None):
    """``attn_fusion``: the decode ``attention`` command that this ``attn_in`` computes too."""
    p = cmd.payload
    op = p["kernel"]
    base = hal.arena_ptr(rank)
    st = hal.stream_handle(rank)
    ins = p["inputs"]
    out_off, out_shape, out_dt = p["output"]
    node = p.get("node", op)
    lib = nat.lib

    def addr(ref):
        return base + ref[0]

    if op.startswith("aten."):  # a node of a graph exported and annotated by the reference's passes
        from backend.cuda_aten import lower_aten

        return lower_aten(hal, base, st, p, rank)

    if op in _PROJECTIONS:
        a, mode, code = projection_args(hal, rank, cmd, attn_fusion)
        ref = ctypes.byref(a)
        need = lib.pim_projection_scratch_bytes(ref, code, mode)
        # Decode rows get a scratch only for the dynamic kernel's work counter, which
        # must stay zero between launches: a pool of its own, never the row-batch one.
        rows = int(a.rows)
        scratch, sbytes = hal.scratch(rank, need, pool="gemv_counter" if rows <= nat.GEMV_MAX_ROWS else None)

        def run():
            nat.check(lib.pim_projection(ref, code, mode, scratch, sbytes, st), node)

        run.keep = a
        return run

    if op == "attention":
        q, pos = ins
        kv = p["kv"]
        item = _ITEM[kv["dtype"]]
        b, s, width = q[1]
        hd = kv["head_dim"]
        hq, hkv = width // hd, len(kv["kv_heads"])
        need = lib.pim_attention_workspace_bytes(b, s, hq, hd, kv["max_seq"])
        ws, wbytes = hal.scratch(rank, need, pool=("attention", b, s, hq, hd, kv["max_seq"]))
        args = (addr(q), addr(pos), base + kv["layer_base"], kv["block_stride"] // item, kv["seq_stride"] // item,
                base + out_off, b, s, hq, hkv, hd, kv["max_seq"], _dt(q[2]), ws, wbytes, st)

        def run():
            nat.check(lib.pim_attention(*args), node)

        return run

    if op == "embedding":
        ids, tab = ins
        args = (addr(ids), addr(tab), base + out_off, _numel(ids[1]), tab[1][1], tab[1][0], _dt(tab[2]),
                hal.error_flag_ptr(rank), st)

        def run():
            nat.check(lib.pim_embedding(*args), node)

        return run

    if op == "add":
        a0, a1 = ins
        args = (addr(a0), addr(a1), base + out_off, _numel(out_shape), _dt(out_dt), st)

        def run():
            nat.check(lib.pim_add(*args), node)

        return run

    if op == "materialize":
        src = ins[0]
        args = (base + out_off, addr(src), _numel(out_shape) * _ITEM[out_dt], st)

        def run():
            nat.check(lib.pim_copy(*args), node)

        return run

    if op == "select_last":
        x = ins[0]
        b, s, h = x[1]
        args = (addr(x), base + out_off, b, s, h * _ITEM[x[2]], int(p["attrs"]["index"]), st)

        def run():
            nat.check(lib.pim_select_rows(*args), node)

        return run

    raise NotImplementedError(f"no B200 kernel for launch op {op!r}")


def lower_host_op(hal, plan, cmd):
    """Host nodes run on the host stream against the plan's device-resident host arena."""
    p = cmd.payload
    kind = p["kernel"]
    hb = hal.host_ptr(plan)
    st = hal.host_stream_handle()
    lib = nat.lib
    if kind == "argmax":
        (off, shape, dt), = p["inputs"]
        rows = int(shape[0])
        n = _numel(shape) // rows
        args = (hb + off, hb + p["output"][0], rows, n, _dt(dt), st)

        def run():
            nat.check(lib.pim_argmax(*args), "argmax")

        return run
    if kind == "feed_next":
        (off, shape, dt), = p["inputs"]
        args = (hb + p["output"][0], hb + off, _numel(shape) * 4, st)

        def run():
            nat.check(lib.pim_copy(*args), "feed_next")

        return run
    if kind == "output":
        return lambda: None
    if kind.startswith("aten."):  # a host node of an exported graph: runs on the device-resident host buffer
        from backend.cuda_aten import lower_aten

        return lower_aten(hal, hb, st, p, None)
    raise NotImplementedError(f"no B200 implementation for host op {kind!r}")
