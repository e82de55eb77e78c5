"""NumPy restatement of the aten ops of an exported graph (oracle; test infrastructure).

The reference executes a graph compiled by its own passes with the DPU nodes as kernel
stubs and every host node as the node's torch callable on the CPU
(backend/hal_numpy.py:104-189 runs ``payload["fn"]``; docs/spec.md:1512-1525).  This
module states the same ops on NumPy arrays with torch's semantics (fp32 arithmetic,
numpy broadcasting, torch's argument conventions), so the oracle HAL can run a plan
compiled from the reference's annotated graph without torch.  Only tests, the smoke
check and the bench's CPU legs use the oracle.

``aten_eval(payload, read)`` computes one node: ``payload`` is a command payload of
``runtime.exec_plan_gen`` (kernel = aten target, inputs = operand buffer refs in
operand order, attrs = the encoded operand tree) and ``read(ref)`` returns the array a
ref holds.
"""

from __future__ import annotations

import numpy as np

from graph.fx_import import tensor_operands

INT64_MAX = 9223372036854775807

_NP = {"float32": np.float32, "int64": np.int64, "int32": np.int32, "bool": np.bool_, "float64": np.float64}


class _Ops:
    def __init__(self, payload, read) -> None:
        attrs = payload["attrs"]
        self.args, self.kwargs = attrs.get("args", []), attrs.get("kwargs", {})
        names = tensor_operands([self.args, self.kwargs])
        self.refs = dict(zip(names, payload["inputs"]))
        self.read = read

    def value(self, v):
        if isinstance(v, dict):
            if "node" in v:
                return self.read(self.refs[v["node"]])
            if "dtype" in v:
                return v["dtype"]
            if "dict" in v:
                return {k: self.value(x) for k, x in v["dict"].items()}
            return v
        if isinstance(v, list):
            return [self.value(x) for x in v]
        return v

    def arg(self, i, name=None, default=None):
        if i < len(self.args):
            return self.value(self.args[i])
        kw = self.kwargs.get("dict", self.kwargs) if isinstance(self.kwargs, dict) else {}
        if name is not None and name in kw:
            return self.value(kw[name])
        return default


def _f32(x):
    return np.asarray(x, dtype=np.float32)


def _shape(shape, numel):
    shape = list(shape)
    if -1 in shape:
        i = shape.index(-1)
        rest = int(np.prod([s for j, s in enumerate(shape) if j != i]))
        shape[i] = numel // rest
    return shape


def aten_eval(payload, read) -> np.ndarray:
    op = payload["kernel"]
    out_shape, out_dt = tuple(payload["output"][1]), payload["output"][2]
    o = _Ops(payload, read)
    if op in ("aten.view", "aten.reshape", "aten._unsafe_view"):
        x = o.arg(0)
        r = x.reshape(_shape(o.arg(1, "shape", out_shape), x.size))
    elif op in ("aten.alias", "aten.contiguous", "aten.clone", "aten.lift_fresh_copy"):
        r = o.arg(0).copy()
    elif op == "aten.unsqueeze":
        x = o.arg(0)
        d = o.arg(1, "dim")
        r = np.expand_dims(x, d if d >= 0 else d + x.ndim + 1)
    elif op in ("aten.squeeze.dim", "aten.squeeze"):
        r = o.arg(0).reshape(out_shape)
    elif op in ("aten.to.dtype", "aten.to.dtype_layout", "aten._to_copy"):
        r = o.arg(0).astype(_NP[out_dt])
    elif op == "aten.expand":
        x = o.arg(0)
        shape = [x.shape[i - (len(out_shape) - x.ndim)] if s == -1 else s for i, s in enumerate(o.arg(1, "size"))]
        r = np.broadcast_to(x, shape).copy()
    elif op == "aten.transpose.int":
        r = np.swapaxes(o.arg(0), o.arg(1, "dim0"), o.arg(2, "dim1")).copy()
    elif op == "aten.permute":
        r = np.transpose(o.arg(0), o.arg(1, "dims")).copy()
    elif op == "aten.slice.Tensor":
        x = o.arg(0)
        d = o.arg(1, "dim", 0)
        start, end, step = o.arg(2, "start", 0) or 0, o.arg(3, "end", INT64_MAX), o.arg(4, "step", 1)
        end = x.shape[d] if end is None or end > x.shape[d] else end
        idx = [slice(None)] * x.ndim
        idx[d] = slice(start, end, step)
        r = x[tuple(idx)].copy()
    elif op == "aten.select.int":
        r = np.take(o.arg(0), o.arg(2, "index"), axis=o.arg(1, "dim")).copy()
    elif op == "aten.cat":
        r = np.concatenate(o.arg(0, "tensors"), axis=o.arg(1, "dim", 0) or 0)
    elif op == "aten.neg":
        r = -_f32(o.arg(0))
    elif op == "aten.rsqrt":
        r = np.float32(1.0) / np.sqrt(_f32(o.arg(0)))
    elif op == "aten.sqrt":
        r = np.sqrt(_f32(o.arg(0)))
    elif op == "aten.silu":
        x = _f32(o.arg(0))
        r = x / (np.float32(1.0) + np.exp(-x))
    elif op in ("aten.cos", "aten.sin", "aten.tanh", "aten.exp"):
        r = getattr(np, op.split(".")[1])(_f32(o.arg(0)))
    elif op == "aten.reciprocal":
        r = np.float32(1.0) / _f32(o.arg(0))
    elif op == "aten.pow.Tensor_Scalar":
        r = _f32(o.arg(0)) ** np.float32(o.arg(1, "exponent"))
    elif op in ("aten.add.Tensor", "aten.sub.Tensor", "aten.mul.Tensor", "aten.div.Tensor"):
        a, b = o.arg(0), o.arg(1)
        a = _f32(a) if isinstance(a, np.ndarray) else np.float32(a)
        b = _f32(b) if isinstance(b, np.ndarray) else np.float32(b)
        r = {"add": np.add, "sub": np.subtract, "mul": np.multiply, "div": np.divide}[op.split(".")[1]](a, b)
    elif op == "aten.mean.dim":
        x = _f32(o.arg(0))
        dims = o.arg(1, "dim")
        keep = bool(o.arg(2, "keepdim", False))
        r = np.mean(x, axis=tuple(dims) if isinstance(dims, list) else dims, keepdims=keep, dtype=np.float32)
    elif op in ("aten.arange", "aten.arange.start", "aten.arange.start_step"):
        if op == "aten.arange":
            r = np.arange(o.arg(0, "end"))
        else:
            r = np.arange(o.arg(0, "start"), o.arg(1, "end"), o.arg(2, "step", 1) or 1)
    elif op == "aten.embedding":
        table, ids = o.arg(0, "weight"), o.arg(1, "indices")
        r = table[ids.astype(np.int64)]
    elif op in ("aten.matmul", "aten.bmm", "aten.mm"):
        r = np.matmul(_f32(o.arg(0)), _f32(o.arg(1)))
    elif op == "aten.scaled_dot_product_attention":
        q, k, v = _f32(o.arg(0, "query")), _f32(o.arg(1, "key")), _f32(o.arg(2, "value"))
        mask = o.arg(3, "attn_mask")
        causal = bool(o.arg(5, "is_causal", False))
        scale = o.arg(6, "scale")
        scale = np.float32(1.0 / np.sqrt(q.shape[-1]) if scale is None else scale)
        if k.shape[1] != q.shape[1]:  # grouped heads
            k = np.repeat(k, q.shape[1] // k.shape[1], axis=1)
            v = np.repeat(v, q.shape[1] // v.shape[1], axis=1)
        s = np.matmul(q, np.swapaxes(k, -1, -2)) * scale
        if mask is not None:
            s = s + _f32(mask)
        if causal:
            L, S = s.shape[-2], s.shape[-1]
            s = np.where(np.tril(np.ones((L, S), bool)), s, -np.inf)
        s = s - s.max(-1, keepdims=True)
        e = np.exp(s)
        r = np.matmul(e / e.sum(-1, keepdims=True), v)
    elif op == "aten.linear":
        x, w, bias = _f32(o.arg(0)), _f32(o.arg(1)), o.arg(2, "bias")
        r = np.matmul(x, w.T)
        if bias is not None:
            r = r + _f32(bias)
    elif op == "aten.addmm":
        r = _f32(o.arg(0)) + np.matmul(_f32(o.arg(1)), _f32(o.arg(2)))
    else:
        raise NotImplementedError(f"oracle: no restatement of {op}")
    r = np.asarray(r).astype(_NP.get(out_dt, np.float32), copy=False)
    if tuple(r.shape) != out_shape:
        r = r.reshape(out_shape)
    return r


# DPU ops of the reference's whitelist (graph/partition.py:13-21) registered as kernels;
# every other aten op of a plan is a host command.
DPU_OPS = ("aten.linear", "aten.addmm", "aten.add.Tensor", "aten.mul.Tensor", "aten.tanh")
