"""NumPy kernel stubs and host commands for the step graph (oracle).

Each launch reads and writes the rank's MRAM bytes only (``read_local`` /
``write_local``), the contract of the reference's kernel stubs
(tests/test_hal_numpy.py:66-70, docs/spec.md:1529).  Arithmetic follows HF
``LlamaForCausalLM`` with its rounding points made explicit for bf16 models
(``_r`` rounds fp32 -> bf16 -> fp32; for fp32 models it is the identity):

* RMSNorm: ``w * round(x * rsqrt(mean(x^2) + eps))`` rounded;
* linear: fp32 accumulation, rounded once;
* RoPE: ``round(round(q*cos) + round(rotate_half(q)*sin))`` with bf16 cos/sin;
* SiLU*up: ``round(round(silu(gate)) * up)``;
* attention: fp32 scores/softmax over keys 0..pos, output rounded.

Host commands implement the comm combine (oracle.lowering.combine), argmax
and the decode feedback.
"""

from __future__ import annotations

import numpy as np

from oracle.hal_numpy import np_dtype
from oracle.lowering import combine


def _r(x: np.ndarray, dt: str) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    if dt == "bfloat16":
        return x.astype(np_dtype("bfloat16")).astype(np.float32)
    if dt == "float16":
        return x.astype(np.float16).astype(np.float32)
    return x


def _read(hal, rank, ref, as_f32=True):
    off, shape, dt = ref
    a = hal.read_local(rank, off, shape, np_dtype(dt))
    return a.astype(np.float32) if as_f32 and dt not in ("int32", "int64") else a


def _write(hal, rank, ref, value) -> None:
    off, shape, dt = ref
    hal.write_local(rank, off, np.ascontiguousarray(np.asarray(value).astype(np_dtype(dt)).reshape(shape)))


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float, dt: str) -> np.ndarray:
    var = np.mean(x.astype(np.float32) ** 2, axis=-1, keepdims=True)
    y = _r(x / np.sqrt(var + np.float32(eps)), dt)
    return _r(y * w, dt)


def rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, dt: str) -> np.ndarray:
    """x: [..., heads, hd]; cos/sin broadcast to [..., 1, hd/2]."""
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    c = np.concatenate([cos, cos], -1)
    s = np.concatenate([sin, sin], -1)
    rot = np.concatenate([-x2, x1], -1)
    return _r(_r(x * c, dt) + _r(rot * s, dt), dt)


def _kv_addr(kv: dict, head_local: int, which: int, seq: int) -> int:
    return kv["layer_base"] + (2 * head_local + which) * kv["block_stride"] + seq * kv["seq_stride"]


def k_attn_in(hal, rank, cmd):
    p = cmd.payload
    x_ref, lnw_ref, w_ref, cos_ref, sin_ref, pos_ref = p["inputs"]
    dt = x_ref[2]
    x = _read(hal, rank, x_ref)
    b, s, h = x.shape
    w = _read(hal, rank, w_ref)
    lnw = _read(hal, rank, lnw_ref)
    cos, sin = _read(hal, rank, cos_ref), _read(hal, rank, sin_ref)
    pos = _read(hal, rank, pos_ref).astype(np.int64)
    kv = p["kv"]
    hd = kv["head_dim"]
    hkv = len(kv["kv_heads"])
    out_ref = p["output"]
    hq = out_ref[1][-1] // hd
    xn = rmsnorm(x, lnw, p["attrs"]["eps"], dt)
    qkv = _r(xn.reshape(b * s, h) @ w.T, dt).reshape(b, s, -1)
    # weight rows of each head come in RoPE pair order (j, j + hd/2); undo it per head
    qkv = qkv.reshape(b, s, -1, hd // 2, 2).transpose(0, 1, 2, 4, 3).reshape(b, s, -1)
    q = qkv[..., :hq * hd].reshape(b, s, hq, hd)
    k = qkv[..., hq * hd:(hq + hkv) * hd].reshape(b, s, hkv, hd)
    v = qkv[..., (hq + hkv) * hd:].reshape(b, s, hkv, hd)
    positions = pos[:, None] + np.arange(s)[None, :]  # [b, s]
    c = cos[positions][:, :, None, :]
    sn = sin[positions][:, :, None, :]
    q = rope(q, c, sn, dt)
    k = rope(k, c, sn, dt)
    kdt = np_dtype(kv["dtype"])
    row = hd * kdt.itemsize
    for bi in range(b):
        for j in range(hkv):
            base_k = _kv_addr(kv, j, 0, bi) + int(positions[bi, 0]) * row
            base_v = _kv_addr(kv, j, 1, bi) + int(positions[bi, 0]) * row
            hal.write_local(rank, base_k, np.ascontiguousarray(k[bi, :, j, :].astype(kdt)))
            hal.write_local(rank, base_v, np.ascontiguousarray(v[bi, :, j, :].astype(kdt)))
    _write(hal, rank, out_ref, q.reshape(b, s, hq * hd))


def k_attention(hal, rank, cmd):
    p = cmd.payload
    q_ref, pos_ref = p["inputs"]
    dt = q_ref[2]
    q = _read(hal, rank, q_ref)
    pos = _read(hal, rank, pos_ref).astype(np.int64)
    kv = p["kv"]
    hd = kv["head_dim"]
    hkv = len(kv["kv_heads"])
    b, s, _ = q.shape
    hq = q.shape[-1] // hd
    group = hq // hkv
    kdt = np_dtype(kv["dtype"])
    out = np.zeros((b, s, hq, hd), np.float32)
    scale = np.float32(1.0 / np.sqrt(hd))
    qh = q.reshape(b, s, hq, hd)
    for bi in range(b):
        ctx = int(pos[bi]) + s
        for j in range(hkv):
            K = hal.read_local(rank, _kv_addr(kv, j, 0, bi), (ctx, hd), kdt).astype(np.float32)
            V = hal.read_local(rank, _kv_addr(kv, j, 1, bi), (ctx, hd), kdt).astype(np.float32)
            for gq in range(group):
                hi = j * group + gq
                sc = (qh[bi, :, hi, :] @ K.T) * scale  # [s, ctx]
                qpos = int(pos[bi]) + np.arange(s)[:, None]
                sc = np.where(np.arange(ctx)[None, :] <= qpos, sc, -np.inf)
                sc = sc - sc.max(-1, keepdims=True)
                e = np.exp(sc)
                out[bi, :, hi, :] = (e / e.sum(-1, keepdims=True)) @ V
    _write(hal, rank, p["output"], _r(out, dt).reshape(b, s, hq * hd))


def k_linear(hal, rank, cmd):
    p = cmd.payload
    x_ref, w_ref = p["inputs"]
    x = _read(hal, rank, x_ref)
    w = _read(hal, rank, w_ref)
    lead = x.shape[:-1]
    y = x.reshape(-1, x.shape[-1]) @ w.T
    _write(hal, rank, p["output"], _r(y, p["output"][2]).reshape(*lead, -1))


def k_linear_add(hal, rank, cmd):
    """o_proj / down_proj with the residual add: ``round(round(x @ W.T) + residual)``."""
    p = cmd.payload
    x_ref, w_ref, r_ref = p["inputs"]
    x = _read(hal, rank, x_ref)
    w = _read(hal, rank, w_ref)
    res = _read(hal, rank, r_ref)
    dt = p["output"][2]
    y = _r(x.reshape(-1, x.shape[-1]) @ w.T, dt).reshape(*x.shape[:-1], -1)
    _write(hal, rank, p["output"], _r(y + res, dt))


def k_add(hal, rank, cmd):
    p = cmd.payload
    a, b = (_read(hal, rank, r) for r in p["inputs"])
    _write(hal, rank, p["output"], _r(a + b, p["output"][2]))


def k_mlp_in(hal, rank, cmd):
    p = cmd.payload
    x_ref, lnw_ref, w_ref = p["inputs"]
    dt = x_ref[2]
    x = _read(hal, rank, x_ref)
    xn = rmsnorm(x, _read(hal, rank, lnw_ref), p["attrs"]["eps"], dt)
    w = _read(hal, rank, w_ref)
    i_l = w.shape[0] // 2
    gu = xn.reshape(-1, x.shape[-1]) @ w.T
    gate, up = _r(gu[:, 0::2], dt), _r(gu[:, 1::2], dt)  # rows interleaved gate_j, up_j
    act = _r(gate / (1.0 + np.exp(-gate)), dt)
    _write(hal, rank, p["output"], _r(act * up, dt).reshape(*x.shape[:-1], i_l))


def k_lm_head_in(hal, rank, cmd):
    p = cmd.payload
    x_ref, nw_ref, w_ref = p["inputs"]
    dt = x_ref[2]
    x = _read(hal, rank, x_ref)
    xn = rmsnorm(x, _read(hal, rank, nw_ref), p["attrs"]["eps"], dt)
    w = _read(hal, rank, w_ref)
    y = xn.reshape(-1, x.shape[-1]) @ w.T
    _write(hal, rank, p["output"], _r(y, p["output"][2]).reshape(*x.shape[:-1], -1))


def k_embedding(hal, rank, cmd):
    p = cmd.payload
    ids_ref, tab_ref = p["inputs"]
    ids = _read(hal, rank, ids_ref).astype(np.int64)
    off, (v, h), dt = tab_ref
    rows = np.stack([hal.read_local(rank, off + int(i) * h * np_dtype(dt).itemsize, (h,), np_dtype(dt))
                     for i in ids.reshape(-1)])
    _write(hal, rank, p["output"], rows.reshape(*ids.shape, h))


def k_select_last(hal, rank, cmd):
    p = cmd.payload
    x = _read(hal, rank, p["inputs"][0], as_f32=False)
    idx = p["attrs"]["index"]
    _write(hal, rank, p["output"], x[:, idx:idx + 1, :])


def k_materialize(hal, rank, cmd):
    p = cmd.payload
    _write(hal, rank, p["output"], _read(hal, rank, p["inputs"][0], as_f32=False))


def k_aten(hal, rank, cmd):
    """A DPU node of an exported graph (the reference's aten.linear / add / mul / tanh stubs)."""
    from oracle.aten import aten_eval

    def read(ref):
        off, shape, dt = ref
        return hal.read_local(rank, off, tuple(shape), np_dtype(dt))

    _write(hal, rank, cmd.payload["output"], aten_eval(cmd.payload, read))


KERNELS = {
    "attn_in": k_attn_in, "attention": k_attention, "linear": k_linear, "linear_add": k_linear_add, "add": k_add,
    "mlp_in": k_mlp_in,
    "lm_head_in": k_lm_head_in, "embedding": k_embedding, "select_last": k_select_last,
    "materialize": k_materialize,
}
KERNELS.update({name: k_aten for name in ("aten.linear", "aten.addmm", "aten.add.Tensor", "aten.mul.Tensor",
                                          "aten.tanh", "aten.sub.Tensor", "aten.div.Tensor")})


# ---------------------------------------------------------------------------
# host commands
# ---------------------------------------------------------------------------


def _host_read(hal, plan, ref):
    off, shape, dt = ref
    return hal.read_host(plan, off, shape, np_dtype(dt))


def _make_combine(hal, plan):
    def fn(cmd):
        p = cmd.payload
        entry = p["entry"]
        run = plan.meta["run"]
        itemsize = entry.dtype.itemsize
        if p["kind"] == "scatter":
            src = hal.host_arena(plan)[p["src_host"]:p["src_host"] + entry.numel * itemsize]
            flat = src.copy().view(entry.dtype)
        else:
            collected = [(entry.collect_segments[i], np.asarray(run.result(cid)).reshape(-1))
                         for i, cid in enumerate(p["collect"])]
            flat = combine(entry, collected)
        hb = p["host_offset"]
        if hb < hal.host_arena(plan).size:
            hal.write_host(plan, hb, flat)
        else:
            hal.staging(plan)[hb] = flat
        return flat
    return fn


def _make_host_op(hal, plan):
    def fn(cmd):
        p = cmd.payload
        kind = p["kernel"]
        if kind == "argmax":
            logits = _host_read(hal, plan, p["inputs"][0]).astype(np.float32)
            tok = np.argmax(logits.reshape(logits.shape[0], -1), axis=-1).astype(np.int32)
            hal.write_host(plan, p["output"][0], tok)
            return tok
        if kind == "feed_next":
            tok = _host_read(hal, plan, p["inputs"][0])
            hal.write_host(plan, p["output"][0], tok.astype(np.int32))
            return tok
        if kind == "output":
            return None
        if kind.startswith("aten."):  # a host node of an exported graph: its torch callable, restated
            from oracle.aten import aten_eval

            val = aten_eval(p, lambda ref: hal.read_host(plan, ref[0], tuple(ref[1]), np_dtype(ref[2])))
            hal.write_host(plan, p["output"][0], np.ascontiguousarray(val))
            return val
        raise ValueError(f"no oracle host implementation for {kind!r}")
    return fn


def bind(hal, plan) -> None:
    """Register every kernel stub and attach host implementations to ``plan``'s host commands.

    Writeback transfers whose host buffer is staging (not in the host arena)
    read it through ``data``, resolved when the transfer is submitted.
    """
    for name, fn in KERNELS.items():
        hal.register_kernel(name, fn)
    comb, hop = _make_combine(hal, plan), _make_host_op(hal, plan)
    staging = hal.staging(plan)
    arena_size = hal.host_arena(plan).size
    for cmd in plan.commands:
        if cmd.op in ("host_reduce", "host_concat", "host_permute", "host_slice"):
            cmd.payload["fn"] = comb
        elif cmd.op == "host_op":
            cmd.payload["fn"] = hop
        elif cmd.op == "dma_in" and cmd.payload.get("role") == "writeback":
            hb_seg = cmd.payload["host_offset"]
            if hb_seg >= arena_size:
                cmd.payload["data"] = _StagingView(staging, plan, cmd)


class _StagingView:
    """Lazy ``data`` for a writeback whose source is virtual host staging."""

    def __init__(self, staging: dict, plan, cmd) -> None:
        self.staging, self.plan, self.cmd = staging, plan, cmd

    def __array__(self, dtype=None, copy=None):
        p = self.cmd.payload
        entry = next(c.payload["entry"] for c in self.plan.commands
                     if c.payload.get("role") == "combine" and c.payload.get("edge") == p["edge"])
        base = next(c.payload["host_offset"] for c in self.plan.commands
                    if c.payload.get("role") == "combine" and c.payload.get("edge") == p["edge"])
        flat = self.staging[base]
        itemsize = entry.dtype.itemsize
        lo = (p["host_offset"] - base) // itemsize
        arr = np.ascontiguousarray(flat[lo:lo + p["nbytes"] // itemsize])
        return arr if dtype is None else arr.astype(dtype)
