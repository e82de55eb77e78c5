"""ctypes binding of libpim_b200.so (the C ABI declared in include/pim_b200.h).

There is no fallback: if the library is missing or was built for another ABI
version, importing this module raises, and so does every HAL that needs it.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent.parent / "csrc" / "libpim_b200.so"
ABI_VERSION = 13

F32, BF16, I32, I64 = 0, 1, 2, 3
PROJ_PLAIN, PROJ_ROPE_KV, PROJ_SILU_MUL = 0, 1, 2
PROJ_KERNEL_REGISTER, PROJ_KERNEL_STAGED, PROJ_KERNEL_DYNAMIC = 0, 1, 3
ROW_BATCH_KERNEL_TILE, ROW_BATCH_KERNEL_PERSISTENT = 0, 1
PREFILL_ATTENTION_MMA, PREFILL_ATTENTION_TCGEN05 = 0, 1
GEMV_MAX_ROWS = 8  # decode projections up to this many rows run as a GEMV
DECODE_LAYER_BARRIER_BYTES = 256

DTYPE_CODE = {"float32": F32, "bfloat16": BF16, "int32": I32, "int64": I64}
MAX_DIMS = 8
# pim_aten_op
ATEN_UNARY = {"neg": 0, "rsqrt": 1, "sqrt": 2, "silu": 3, "cos": 4, "sin": 5, "tanh": 6, "exp": 7,
              "reciprocal": 8, "pow_scalar": 9, "add_scalar": 10, "mul_scalar": 11, "sub_scalar": 12,
              "div_scalar": 13}
ATEN_BINARY = {"add": 20, "sub": 21, "mul": 22, "div": 23}

c_vp = ctypes.c_void_p
c_i32 = ctypes.c_int32
c_i64 = ctypes.c_int64
c_f32 = ctypes.c_float


class ProjectionArgs(ctypes.Structure):
    """Mirror of ``pim_projection_args``."""

    _fields_ = [
        ("x", c_vp), ("norm_weight", c_vp), ("weight", c_vp), ("out", c_vp),
        ("rows", c_i64), ("k", c_i64), ("ncols", c_i64),
        ("eps", c_f32),
        ("rope_cos", c_vp), ("rope_sin", c_vp), ("positions", c_vp),
        ("seq", c_i32), ("q_heads", c_i32), ("kv_heads", c_i32), ("head_dim", c_i32), ("max_seq", c_i32),
        ("kv_base", c_vp), ("kv_block_stride", c_i64), ("kv_seq_stride", c_i64),
        ("inter", c_i32), ("residual", c_vp), ("err_flag", c_vp), ("p2p_desc", c_vp), ("allreduce_out", c_vp),
        ("attn_out", c_vp), ("attn_counters", c_vp),
    ]


EXPORTS = {
    "pim_abi_version": ([], c_i32),
    "pim_kernel_launches": ([], ctypes.c_uint64),
    "pim_last_error": ([], ctypes.c_char_p),
    "pim_cooperative_pdl": ([c_i32], c_i32),
    "pim_enable_peer_access": ([c_i32, c_i32], c_i32),
    "pim_projection": ([ctypes.POINTER(ProjectionArgs), c_i32, c_i32, c_vp, c_i64, c_vp], c_i32),
    "pim_projection_scratch_bytes": ([ctypes.POINTER(ProjectionArgs), c_i32, c_i32], c_i64),
    "pim_set_projection_kernel": ([c_i32], c_i32),
    "pim_projection_kernel": ([], c_i32),
    "pim_decode_layer": ([ctypes.POINTER(ProjectionArgs)] * 4 + [c_vp, c_vp, c_i32, c_vp], c_i32),
    "pim_decode_step_table_bytes": ([c_i32], c_i64),
    "pim_decode_step_prepare": ([ctypes.POINTER(ctypes.POINTER(ProjectionArgs)), c_i32,
                                 ctypes.POINTER(ProjectionArgs), c_i32, c_vp, c_i64, ctypes.POINTER(c_vp)], c_i32),
    "pim_decode_step": ([c_vp, c_vp, c_vp, c_vp], c_i32),
    "pim_decode_step_free": ([c_vp], None),
    "pim_set_row_batch_kernel": ([c_i32], c_i32),
    "pim_attention_errors": ([c_i32], c_i32),
    "pim_set_prefill_attention_kernel": ([c_i32], c_i32),
    "pim_prefill_attention_kernel": ([], c_i32),
    "pim_row_batch_kernel": ([], c_i32),
    "pim_attention": ([c_vp, c_vp, c_vp, c_i64, c_i64, c_vp, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32,
                       c_vp, c_i64, c_vp], c_i32),
    "pim_attention_workspace_bytes": ([c_i32, c_i32, c_i32, c_i32, c_i32], c_i64),
    "pim_attention_noalloc": ([c_vp, c_vp, c_vp, c_i64, c_i64, c_vp, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32,
                               c_vp], c_i32),
    "pim_embedding": ([c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i32, c_vp, c_vp], c_i32),
    "pim_add": ([c_vp, c_vp, c_vp, c_i64, c_i32, c_vp], c_i32),
    "pim_select_rows": ([c_vp, c_vp, c_i32, c_i32, c_i64, c_i32, c_vp], c_i32),
    "pim_argmax": ([c_vp, c_vp, c_i32, c_i64, c_i32, c_vp], c_i32),
    "pim_copy": ([c_vp, c_vp, c_i64, c_vp], c_i32),
    "pim_ordered_sum": ([ctypes.POINTER(c_vp), c_i32, ctypes.POINTER(c_vp), c_i32, c_i64, c_i32, c_i32, c_vp], c_i32),
    "pim_ordered_sum_add": ([ctypes.POINTER(c_vp), c_i32, c_vp, c_vp, c_vp, c_i64, c_i32, c_vp], c_i32),
    "pim_batched_copy": ([c_vp, c_i32, c_i64, c_vp], c_i32),
    "pim_allreduce_p2p": ([c_vp, ctypes.POINTER(c_vp), c_i32, c_i64, c_i32, c_i32, c_i32, ctypes.POINTER(c_vp), c_i64,
                           c_vp, c_vp, c_vp], c_i32),
    "pim_allreduce_p2p_add": ([c_vp, c_vp, c_vp, c_vp, c_i64, c_i32, c_i32, c_i32, ctypes.POINTER(c_vp), c_i64,
                               c_vp, c_vp, c_vp], c_i32),
    "pim_allreduce_p2p_ll": ([c_vp, c_vp, c_vp, c_vp, c_i64, c_i32, c_i32, c_i32, ctypes.POINTER(c_vp), c_i64,
                              c_vp, c_vp, c_vp], c_i32),
    "pim_ipc_export": ([c_vp, c_vp, ctypes.POINTER(c_i64)], c_i32),
    "pim_p2p_desc_bytes": ([], c_i64),
    "pim_p2p_desc_init": ([c_vp, c_i32, c_i32, ctypes.POINTER(c_vp), c_i64, c_vp, c_vp, c_vp], c_i32),
    "pim_ipc_open": ([c_vp, ctypes.POINTER(c_vp)], c_i32),
    "pim_ipc_close": ([c_vp], c_i32),
    "pim_fill_normal": ([c_vp, c_i64, c_i32, ctypes.c_uint64, c_f32, c_vp], c_i32),
    "pim_fill_const": ([c_vp, c_i64, c_i32, c_f32, c_vp], c_i32),
}


class TensorView(ctypes.Structure):
    """pim_tensor_view: a strided view (element offset, shape, element strides)."""

    _fields_ = [("data", c_vp), ("dtype", c_i32), ("ndim", c_i32), ("offset", c_i64),
                ("shape", c_i64 * MAX_DIMS), ("stride", c_i64 * MAX_DIMS)]


_PV = ctypes.POINTER(TensorView)
EXPORTS.update({
    "pim_aten_copy": ([_PV, _PV, c_vp], c_i32),
    "pim_aten_unary": ([c_i32, _PV, _PV, ctypes.c_double, c_vp], c_i32),
    "pim_aten_binary": ([c_i32, _PV, _PV, _PV, c_vp], c_i32),
    "pim_aten_mean_last": ([_PV, _PV, c_vp], c_i32),
    "pim_aten_arange": ([_PV, ctypes.c_double, ctypes.c_double, c_vp], c_i32),
    "pim_aten_matmul": ([_PV, _PV, _PV, c_vp], c_i32),
    "pim_aten_sdpa": ([_PV, _PV, _PV, _PV, _PV, ctypes.c_double, c_i32, c_vp], c_i32),
    "pim_aten_embedding": ([_PV, _PV, _PV, c_vp, c_vp], c_i32),
})


class NativeError(RuntimeError):
    pass


def _load() -> ctypes.CDLL:
    path = Path(os.environ.get("PIM_B200_LIB", _LIB_PATH))
    if not path.exists():
        raise NativeError(f"{path} is missing: build it with `python flagos-pim-compiler_b200/csrc/build.py` "
                          "(the B200 backend has no CPU fallback)")
    lib = ctypes.CDLL(str(path))
    for name, (argtypes, restype) in EXPORTS.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = restype
    ver = lib.pim_abi_version()
    if ver != ABI_VERSION:
        raise NativeError(f"{path}: ABI version {ver}, expected {ABI_VERSION}")
    return lib


lib = _load()
LIB_PATH = _LIB_PATH


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        msg = lib.pim_last_error().decode(errors="replace")
        kind = {1: ValueError, 3: NotImplementedError}.get(rc, NativeError)
        raise kind(f"{what or 'pim call'} failed (status {rc}): {msg}")


def ptr_array(ptrs) -> ctypes.Array:
    arr = (c_vp * len(ptrs))()
    for i, p in enumerate(ptrs):
        arr[i] = p
    return arr
