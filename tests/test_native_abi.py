"""The C-ABI library loads and exports every symbol include/pim_b200.h declares (no GPU needed)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "pim_b200.h"


def declared_symbols() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(pim_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_abi():
    syms = declared_symbols()
    assert "pim_projection" in syms and "pim_ordered_sum" in syms and "pim_attention" in syms
    assert len(syms) >= 15


def test_library_exports_every_declared_symbol():
    from backend import _native as nat

    lib = ctypes.CDLL(str(nat.LIB_PATH))
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert missing == []
    assert lib.pim_abi_version() == nat.ABI_VERSION


def test_binding_covers_every_declared_symbol():
    from backend import _native as nat

    assert sorted(nat.EXPORTS) == declared_symbols()


def test_bad_arguments_are_rejected_without_touching_the_gpu():
    """Argument validation runs before any CUDA call, so it works on a CPU-only machine."""
    from backend import _native as nat

    a = nat.ProjectionArgs()
    rc = nat.lib.pim_projection(ctypes.byref(a), 0, 0, None, 0, None)
    assert rc == 1 and b"null pointer" in nat.lib.pim_last_error()
    assert nat.lib.pim_ordered_sum(None, 0, None, 0, 0, 0, 0, None) == 1
    assert nat.lib.pim_attention(None, None, None, 0, 0, None, 1, 1, 1, 1, 64, 8, 0, None, 0, None) == 1


def test_noalloc_attention_refusals_happen_before_any_cuda_call():
    """pim_attention_noalloc checks its pointers, dtype, geometry and the 4 MiB limit of its
    fixed array before touching the GPU (dummy non-null pointers are never dereferenced)."""
    from backend import _native as nat

    lib = nat.lib
    p = 1 << 20  # a non-null dummy address

    def call(q=p, dtype=nat.F32, batch=1, seq=1, hq=4, hkv=4, hd=64, max_seq=64):
        return lib.pim_attention_noalloc(q, p, p, max_seq * hd, hkv * 2 * max_seq * hd, p, batch, seq, hq, hkv, hd,
                                         max_seq, dtype, None)

    assert call(q=None) == 1 and b"null pointer" in lib.pim_last_error()
    assert call(dtype=7) == 1 and b"bad dtype" in lib.pim_last_error()
    assert call(hq=3, hkv=2) == 1 and b"bad geometry" in lib.pim_last_error()
    assert call(hd=96) == 3 and b"head_dim" in lib.pim_last_error()
    # split-K shapes whose workspace exceeds the array are refused ...
    assert lib.pim_attention_workspace_bytes(64, 2048, 32, 128, 4096) > 4 * 2**20
    assert call(batch=64, seq=2048, hq=32, hkv=32, hd=128, max_seq=4096) == 1
    assert b"4 MiB" in lib.pim_last_error()
    # ... fp32 and short bf16 row batches run there; bf16 head_dim 128 with 16+ rows does not
    assert call(batch=64, seq=8, hq=32, hkv=32, hd=128, max_seq=4096, dtype=nat.BF16) == 1


def test_decode_scratch_is_the_dynamic_kernels_counter_only():
    """Decode rows need no scratch except the work counter of PIM_PROJ_KERNEL_DYNAMIC (also
    in its fused all-reduce form);
    row batches size theirs by rows x k whatever kernel is selected (no CUDA call)."""
    from backend import _native as nat

    def need(rows, dtype="bfloat16", p2p=None):
        a = nat.ProjectionArgs(x=16, weight=16, out=16, rows=rows, k=4096, ncols=4096, p2p_desc=p2p)
        return nat.lib.pim_projection_scratch_bytes(ctypes.byref(a), nat.DTYPE_CODE[dtype], nat.PROJ_PLAIN)

    prev = nat.lib.pim_projection_kernel()
    try:
        for kernel in (nat.PROJ_KERNEL_REGISTER, nat.PROJ_KERNEL_STAGED):
            assert nat.lib.pim_set_projection_kernel(kernel) == 0
            assert need(1) == 0 and need(8) == 0
        assert nat.lib.pim_set_projection_kernel(nat.PROJ_KERNEL_DYNAMIC) == 0
        assert nat.lib.pim_projection_kernel() == nat.PROJ_KERNEL_DYNAMIC
        assert need(1) == need(8) == 256
        assert need(1, p2p=16) == 256  # its fused all-reduce form takes the same counter
        assert need(16) == 16 * 4096 * 2  # normalised rows of a tensor-core row batch
        assert nat.lib.pim_set_projection_kernel(4) == 1  # no such kernel
        assert nat.lib.pim_set_projection_kernel(2) == 1  # the removed bulk-copy kernel
    finally:
        nat.lib.pim_set_projection_kernel(prev)


def _layer_args():
    """Four chained pim_projection_args of a decode layer (fake, 256-aligned addresses:
    the checks below return before any device access)."""
    from backend import _native as nat

    base = 1 << 20
    x, q, att, h, act, y = (base + i * 65536 for i in range(6))
    w, ln = base + (64 << 20), base + (32 << 20)
    a_in = nat.ProjectionArgs(x=x, norm_weight=ln, weight=w, out=q, rows=1, k=512, ncols=1536, eps=1e-5,
                              rope_cos=base, rope_sin=base, positions=base, seq=1, q_heads=4, kv_heads=4,
                              head_dim=128, max_seq=64, kv_base=base, kv_block_stride=8192, kv_seq_stride=65536,
                              attn_out=att, attn_counters=base)
    a_o = nat.ProjectionArgs(x=att, weight=w, out=h, rows=1, k=512, ncols=512, residual=x)
    a_mlp = nat.ProjectionArgs(x=h, norm_weight=ln, weight=w, out=act, rows=1, k=512, ncols=1376, inter=688, eps=1e-5)
    a_d = nat.ProjectionArgs(x=act, weight=w, out=y, rows=1, k=688, ncols=512, residual=h)
    return [a_in, a_o, a_mlp, a_d]


@pytest.mark.parametrize("breakage,message", [
    (lambda a: setattr(a[1], "x", a[1].x + 256), b"o_proj must read attn_in's attention output"),
    (lambda a: setattr(a[2], "x", a[0].x), b"mlp_in must read o_proj's output"),
    (lambda a: setattr(a[3], "k", 680), b"down must read mlp_in's output"),
    (lambda a: setattr(a[0], "rows", 2), b"one activation row"),
    (lambda a: setattr(a[0], "attn_out", None), b"attn_in needs"),
    (lambda a: setattr(a[0], "head_dim", 96), b"bad head geometry"),
    (lambda a: setattr(a[0], "q_heads", 65), b"bad head geometry"),
    (lambda a: setattr(a[1], "norm_weight", a[0].norm_weight), b"take a norm_weight"),
    (lambda a: setattr(a[2], "residual", a[0].x), b"residual needs mode PLAIN"),
    (lambda a: setattr(a[3], "x", a[3].x + 8), b"16-byte aligned"),
    (lambda a: setattr(a[1], "p2p_desc", 4096), b"the same p2p_desc"),
    (lambda a: setattr(a[0], "p2p_desc", 4096), b"only o_proj and down"),
    (lambda a: setattr(a[3], "allreduce_out", 4096), b"allreduce_out needs p2p_desc"),
    (lambda a: setattr(a[3], "k", 7), b"bad k"),
])
def test_decode_layer_chain_is_checked_without_touching_the_gpu(breakage, message):
    from backend import _native as nat

    args = _layer_args()
    breakage(args)
    rc = nat.lib.pim_decode_layer(*[ctypes.byref(a) for a in args], 1 << 20, None, nat.BF16, None)
    assert rc == 1 and message in nat.lib.pim_last_error(), nat.lib.pim_last_error()


def test_decode_layer_refuses_a_missing_or_unaligned_barrier():
    from backend import _native as nat

    refs = [ctypes.byref(a) for a in _layer_args()]
    assert nat.lib.pim_decode_layer(*refs, None, None, nat.BF16, None) == 1
    assert b"null barrier" in nat.lib.pim_last_error()
    assert nat.lib.pim_decode_layer(*refs, (1 << 20) + 4, None, nat.BF16, None) == 1
    assert b"aligned" in nat.lib.pim_last_error()
    assert nat.lib.pim_decode_layer(*refs, 1 << 20, None, 7, None) == 1  # dtype


def test_decode_step_prepare_checks_layers_chain_and_head_without_touching_the_gpu():
    from backend import _native as nat

    one, two = _layer_args(), _layer_args()
    two[0].x = one[3].out + 256  # layer 2 does not read layer 1's output
    ptrs = (ctypes.POINTER(nat.ProjectionArgs) * 8)(*[ctypes.pointer(a) for a in one + two])
    plan = ctypes.c_void_p()
    table = 1 << 24
    assert nat.lib.pim_decode_step_table_bytes(2) > 0
    rc = nat.lib.pim_decode_step_prepare(ptrs, 2, None, nat.BF16, table, 1 << 20, ctypes.byref(plan))
    assert rc == 1 and b"previous layer's output" in nat.lib.pim_last_error() and not plan.value
    rc = nat.lib.pim_decode_step_prepare(ptrs, 1, None, nat.BF16, table, 8, ctypes.byref(plan))
    assert rc == 1 and b"table too small" in nat.lib.pim_last_error()
    head = nat.ProjectionArgs(x=one[3].out + 64, norm_weight=one[0].norm_weight, weight=one[0].weight,
                              out=one[0].out, rows=1, k=512, ncols=1024)
    rc = nat.lib.pim_decode_step_prepare(ptrs, 1, ctypes.byref(head), nat.BF16, table, 1 << 20, ctypes.byref(plan))
    assert rc == 1 and b"the head takes the last layer's output" in nat.lib.pim_last_error()
    one[1].k = 256  # a broken layer is named as pim_decode_layer names it
    rc = nat.lib.pim_decode_step_prepare(ptrs, 1, None, nat.BF16, table, 1 << 20, ctypes.byref(plan))
    assert rc == 1 and b"o_proj must read attn_in's attention output" in nat.lib.pim_last_error()
    assert nat.lib.pim_decode_step(None, 1 << 20, None, None) == 1
