"""B200 lowering of aten-level nodes (graphs compiled by the reference's own passes).

A node compiled from an exported graph (``graph.fx_import``) carries its aten target as
the command's ``kernel`` (``aten.linear``, ``aten.transpose.int``, ...), its tensor
operands as ``inputs`` (byte offset, local shape, dtype, in operand order) and the full
operand tree in ``attrs["args"] / attrs["kwargs"]``.  ``lower_aten`` turns one such
command into a closure of C-ABI calls on strided views (``pim_tensor_view``): the DPU
nodes of the reference's whitelist (aten.linear / addmm / add / mul / tanh,
graph/partition.py:13-21) on their rank's arena, every host node on the plan's
device-resident host buffer.  Nothing runs on the CPU: an op without a device
implementation raises ``NotImplementedError`` at ``register_plan``.

Every buffer a plan gives a node is contiguous, so each view below starts from the
contiguous strides of its operand's local shape.
"""

from __future__ import annotations

import ctypes
from math import prod, sqrt

from backend import _native as nat
from graph.fx_import import tensor_operands

INT64_MAX = 9223372036854775807
_ITEM = {"float32": 4, "bfloat16": 2, "int32": 4, "int64": 8}


def contiguous_strides(shape) -> list[int]:
    st, acc = [], 1
    for d in reversed(list(shape)):
        st.append(acc)
        acc *= int(d)
    return list(reversed(st))


def make_view(base: int, ref, shape=None, strides=None, offset: int = 0) -> nat.TensorView:
    """A view of buffer ``ref`` = (byte offset, shape, dtype) at ``base``; by default contiguous."""
    off, rshape, dt = ref
    shape = list(rshape if shape is None else shape)
    strides = contiguous_strides(shape) if strides is None else list(strides)
    if len(shape) > nat.MAX_DIMS:
        raise NotImplementedError(f"views of rank {len(shape)} > {nat.MAX_DIMS}")
    item = _ITEM[dt]
    if off % item:
        raise ValueError(f"buffer offset {off} is not aligned to {dt}")
    v = nat.TensorView()
    v.data, v.dtype, v.ndim, v.offset = base + off, nat.DTYPE_CODE[dt], len(shape), int(offset)
    for i, (s, t) in enumerate(zip(shape, strides)):
        v.shape[i], v.stride[i] = int(s), int(t)
    v.buffer_elems = prod(rshape)  # extent of the buffer the view reads or writes (checked by tests)
    return v


def broadcast_view(base: int, ref, out_shape) -> nat.TensorView:
    """``ref`` broadcast to ``out_shape`` (numpy rules: leading 1s, stride 0 where size 1)."""
    shape = list(ref[1])
    st = contiguous_strides(shape)
    pad = len(out_shape) - len(shape)
    if pad < 0:
        raise ValueError(f"cannot broadcast {shape} to {list(out_shape)}")
    shape, st = [1] * pad + shape, [0] * pad + st
    out_st = []
    for s, t, o in zip(shape, st, out_shape):
        if s == o:
            out_st.append(t)
        elif s == 1:
            out_st.append(0)
        else:
            raise ValueError(f"cannot broadcast {list(ref[1])} to {list(out_shape)}")
    return make_view(base, ref, shape=list(out_shape), strides=out_st)


def _dim(d: int, rank: int) -> int:
    return d + rank if d < 0 else d


class Operands:
    """Resolves a node's encoded operand tree: tensors to their buffer refs, the rest as is."""

    def __init__(self, payload) -> None:
        attrs = payload["attrs"]
        self.args, self.kwargs = attrs.get("args", []), attrs.get("kwargs", {})
        names = tensor_operands([self.args, self.kwargs])
        self.refs = dict(zip(names, payload["inputs"]))

    def value(self, v):
        if isinstance(v, dict):
            if "node" in v:
                return self.refs[v["node"]]
            if "dtype" in v:
                return v["dtype"]
            if "dict" in v:
                return {k: self.value(x) for k, x in v["dict"].items()}
            return v
        if isinstance(v, list):
            return [self.value(x) for x in v]
        return v

    def arg(self, i: int, name: str | None = None, default=None):
        if i < len(self.args):
            return self.value(self.args[i])
        kw = self.kwargs.get("dict", self.kwargs) if isinstance(self.kwargs, dict) else {}
        if name is not None and name in kw:
            return self.value(kw[name])
        return default


def _is_ref(x) -> bool:
    return isinstance(x, (tuple, list)) and len(x) == 3 and isinstance(x[1], (tuple, list)) and isinstance(x[2], str)


_UNARY = {"aten.neg": "neg", "aten.rsqrt": "rsqrt", "aten.sqrt": "sqrt", "aten.silu": "silu", "aten.cos": "cos",
          "aten.sin": "sin", "aten.tanh": "tanh", "aten.exp": "exp", "aten.reciprocal": "reciprocal"}
_BINARY = {"aten.add.Tensor": "add", "aten.sub.Tensor": "sub", "aten.mul.Tensor": "mul", "aten.div.Tensor": "div"}
_COPIES = ("aten.view", "aten.reshape", "aten._unsafe_view", "aten.alias", "aten.unsqueeze", "aten.squeeze.dim",
           "aten.squeeze", "aten.to.dtype", "aten.to.dtype_layout", "aten._to_copy", "aten.contiguous",
           "aten.clone", "aten.flatten.using_ints", "aten.lift_fresh_copy")


def lower_aten(hal, base: int, stream: int, payload, rank=None):
    """Closure running one aten node: ``base`` is the arena (DPU node) or the host buffer
    (host node) the command's offsets refer to, ``stream`` the CUDA stream handle."""
    op = payload["kernel"]
    node = payload.get("node", op)
    out = payload["output"]
    ops = Operands(payload)
    lib = nat.lib
    calls = []  # (fn, args) pairs, run in order
    keep = []

    def call(fn, *args):
        calls.append((fn, args))

    def ptr(v):
        keep.append(v)
        return ctypes.byref(v)

    oshape = list(out[1])
    dst = make_view(base, out)

    if op in _COPIES:
        src = ops.arg(0, "self")
        if prod(src[1]) != prod(oshape):
            raise ValueError(f"{node}: {op} changes the element count")
        call(lib.pim_aten_copy, ptr(dst), ptr(make_view(base, src, shape=oshape, strides=contiguous_strides(oshape))))
    elif op == "aten.expand":
        call(lib.pim_aten_copy, ptr(dst), ptr(broadcast_view(base, ops.arg(0, "self"), oshape)))
    elif op in ("aten.transpose.int", "aten.permute"):
        src = ops.arg(0, "self")
        r = len(src[1])
        st = contiguous_strides(src[1])
        if op == "aten.transpose.int":
            d0, d1 = _dim(ops.arg(1, "dim0"), r), _dim(ops.arg(2, "dim1"), r)
            perm = list(range(r))
            perm[d0], perm[d1] = perm[d1], perm[d0]
        else:
            perm = [_dim(d, r) for d in ops.arg(1, "dims")]
        call(lib.pim_aten_copy, ptr(dst), ptr(make_view(base, src, shape=oshape, strides=[st[p] for p in perm])))
    elif op == "aten.slice.Tensor":
        src = ops.arg(0, "self")
        r = len(src[1])
        d = _dim(ops.arg(1, "dim", 0), r)
        size = src[1][d]
        start = ops.arg(2, "start", 0) or 0
        end = ops.arg(3, "end", INT64_MAX)
        end = size if end is None or end > size else end
        step = ops.arg(4, "step", 1)
        start = start + size if start < 0 else start
        end = end + size if end < 0 else end
        st = contiguous_strides(src[1])
        off = start * st[d]
        st[d] *= step
        call(lib.pim_aten_copy, ptr(dst), ptr(make_view(base, src, shape=oshape, strides=st, offset=off)))
    elif op == "aten.select.int":
        src = ops.arg(0, "self")
        r = len(src[1])
        d = _dim(ops.arg(1, "dim"), r)
        idx = ops.arg(2, "index")
        idx = idx + src[1][d] if idx < 0 else idx
        st = contiguous_strides(src[1])
        off = idx * st[d]
        st.pop(d)
        call(lib.pim_aten_copy, ptr(dst), ptr(make_view(base, src, shape=oshape, strides=st, offset=off)))
    elif op == "aten.cat":
        tensors = ops.arg(0, "tensors")
        d = _dim(ops.arg(1, "dim", 0) or 0, len(oshape))
        ost = contiguous_strides(oshape)
        pos = 0
        for t in tensors:
            piece = make_view(base, out, shape=list(t[1]), strides=ost, offset=pos * ost[d])
            call(lib.pim_aten_copy, ptr(piece), ptr(make_view(base, t)))
            pos += t[1][d]
    elif op in _UNARY:
        call(lib.pim_aten_unary, nat.ATEN_UNARY[_UNARY[op]], ptr(dst), ptr(broadcast_view(base, ops.arg(0), oshape)),
             0.0)
    elif op == "aten.pow.Tensor_Scalar":
        call(lib.pim_aten_unary, nat.ATEN_UNARY["pow_scalar"], ptr(dst),
             ptr(broadcast_view(base, ops.arg(0, "self"), oshape)), float(ops.arg(1, "exponent")))
    elif op in _BINARY:
        a, b = ops.arg(0, "self"), ops.arg(1, "other")
        alpha = ops.arg(2, "alpha", 1)
        if alpha not in (1, 1.0, None):
            raise NotImplementedError(f"{node}: {op} with alpha={alpha}")
        kind = _BINARY[op]
        if _is_ref(a) and _is_ref(b):
            call(lib.pim_aten_binary, nat.ATEN_BINARY[kind], ptr(dst), ptr(broadcast_view(base, a, oshape)),
                 ptr(broadcast_view(base, b, oshape)))
        elif _is_ref(a):
            call(lib.pim_aten_unary, nat.ATEN_UNARY[kind + "_scalar"], ptr(dst), ptr(broadcast_view(base, a, oshape)),
                 float(b))
        elif _is_ref(b) and kind in ("add", "mul"):
            call(lib.pim_aten_unary, nat.ATEN_UNARY[kind + "_scalar"], ptr(dst), ptr(broadcast_view(base, b, oshape)),
                 float(a))
        else:
            raise NotImplementedError(f"{node}: {op} with operands {type(a).__name__}, {type(b).__name__}")
    elif op == "aten.mean.dim":
        src = ops.arg(0, "self")
        dims = ops.arg(1, "dim")
        dims = [dims] if isinstance(dims, int) else list(dims or [])
        r = len(src[1])
        if [_dim(d, r) for d in dims] != [r - 1]:
            raise NotImplementedError(f"{node}: mean over dims {dims} (only the last)")
        keep_shape = list(src[1][:-1]) + [1]
        call(lib.pim_aten_mean_last, ptr(make_view(base, out, shape=keep_shape)), ptr(make_view(base, src)))
    elif op == "aten.arange" or op == "aten.arange.start" or op == "aten.arange.start_step":
        if op == "aten.arange":
            start, step = 0.0, 1.0
        else:
            start, step = float(ops.arg(0, "start")), float(ops.arg(2, "step", 1) or 1)
        call(lib.pim_aten_arange, ptr(dst), start, step)
    elif op == "aten.embedding":
        table, ids = ops.arg(0, "weight"), ops.arg(1, "indices")
        err = hal.error_flag_ptr(rank) if rank is not None else hal.error_flag_ptr(hal.local[0])
        call(lib.pim_aten_embedding, ptr(make_view(base, out, shape=[prod(ids[1]), table[1][1]])),
             ptr(make_view(base, table)), ptr(make_view(base, ids)), err)
    elif op == "aten.matmul" or op == "aten.bmm" or op == "aten.mm":
        a, b = ops.arg(0, "self"), ops.arg(1, "other" if op == "aten.matmul" else "mat2")
        r = len(oshape)
        if len(a[1]) != r or len(b[1]) != r:
            raise NotImplementedError(f"{node}: matmul of ranks {len(a[1])}, {len(b[1])} -> {r}")
        call(lib.pim_aten_matmul, ptr(dst), ptr(make_view(base, a)), ptr(make_view(base, b)))
    elif op == "aten.scaled_dot_product_attention":
        q, k, v = ops.arg(0, "query"), ops.arg(1, "key"), ops.arg(2, "value")
        mask = ops.arg(3, "attn_mask")
        dropout = ops.arg(4, "dropout_p", 0.0) or 0.0
        causal = bool(ops.arg(5, "is_causal", False))
        scale = ops.arg(6, "scale")
        if dropout:
            raise NotImplementedError(f"{node}: dropout in inference")
        scale = 1.0 / sqrt(q[1][-1]) if scale is None else float(scale)
        mview = None
        if mask is not None:
            mview = broadcast_view(base, mask, [q[1][0], q[1][1], q[1][2], k[1][2]])
        call(lib.pim_aten_sdpa, ptr(dst), ptr(make_view(base, q)), ptr(make_view(base, k)), ptr(make_view(base, v)),
             ptr(mview) if mview is not None else None, scale, int(causal))
    elif op in ("aten.linear", "aten.addmm"):
        if op == "aten.linear":
            x, w, bias = ops.arg(0, "input"), ops.arg(1, "weight"), ops.arg(2, "bias")
        else:
            bias, x, wt = ops.arg(0, "self"), ops.arg(1, "mat1"), ops.arg(2, "mat2")
            w = None
        if op == "aten.linear" and x[2] == w[2] and x[2] in ("float32", "bfloat16") and x[0] % 16 == 0 \
                and w[0] % 16 == 0 and out[0] % 16 == 0:
            # the projection kernels: y = x . W^T with W in HF [out, in] layout
            a = nat.ProjectionArgs(x=base + x[0], weight=base + w[0], out=base + out[0], rows=prod(x[1][:-1]),
                                   k=x[1][-1], ncols=w[1][0])
            code = nat.DTYPE_CODE[x[2]]
            need = lib.pim_projection_scratch_bytes(ctypes.byref(a), code, nat.PROJ_PLAIN)
            scratch, sbytes = (hal.scratch(rank if rank is not None else hal.local[0], need)
                               if need > 0 else (0, 0))
            call(lib.pim_projection, ptr(a), code, nat.PROJ_PLAIN, scratch, sbytes)
        else:
            # general form: out = x @ W^T (or mat1 @ mat2) through the batched matmul
            r = len(oshape)
            xs = list(x[1])
            if op == "aten.linear":
                wv = make_view(base, w, shape=[1] * (r - 2) + [w[1][1], w[1][0]],
                               strides=[0] * (r - 2) + [1, w[1][1]])
            else:
                wv = make_view(base, wt, shape=[1] * (r - 2) + list(wt[1]),
                               strides=[0] * (r - 2) + contiguous_strides(wt[1]))
            xv = make_view(base, x, shape=[1] * (r - len(xs)) + xs,
                           strides=[0] * (r - len(xs)) + contiguous_strides(xs))
            call(lib.pim_aten_matmul, ptr(dst), ptr(xv), ptr(wv))
        if bias is not None:
            call(lib.pim_aten_binary, nat.ATEN_BINARY["add"], ptr(dst), ptr(make_view(base, out)),
                 ptr(broadcast_view(base, bias, oshape)))
    else:
        raise NotImplementedError(f"no B200 kernel for {op} (node {node})")

    def run():
        for fn, args in calls:
            nat.check(fn(*args, stream), node)

    run.keep = keep
    run.calls = calls  # the C-ABI calls in order, for inspection
    return run
