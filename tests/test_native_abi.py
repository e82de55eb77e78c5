"""The C-ABI library loads and exports every symbol include/pim_b200.h declares (no GPU needed)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

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
        for kernel in (nat.PROJ_KERNEL_REGISTER, nat.PROJ_KERNEL_STAGED, nat.PROJ_KERNEL_STREAMED):
            assert nat.lib.pim_set_projection_kernel(kernel) == 0
            assert need(1) == 0 and need(8) == 0
        assert nat.lib.pim_set_projection_kernel(nat.PROJ_KERNEL_DYNAMIC) == 0
        assert nat.lib.pim_projection_kernel() == nat.PROJ_KERNEL_DYNAMIC
        assert need(1) == need(8) == 256
        assert need(1, p2p=16) == 256  # its fused all-reduce form takes the same counter
        assert need(16) == 16 * 4096 * 2  # normalised rows of a tensor-core row batch
        assert nat.lib.pim_set_projection_kernel(4) == 1  # no such kernel
    finally:
        nat.lib.pim_set_projection_kernel(prev)
