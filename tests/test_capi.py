"""The C-ABI library loads on a machine without a GPU, exports every function the
public header declares, and rejects bad requests before touching the device."""
import ctypes
import os
import re

from pto_fuser import native as nv

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = []
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            txt = open(os.path.join(ROOT, "include", fn)).read()
            names += re.findall(r"PTOF_API\s+[\w\s\*]+?\b(ptof_\w+)\s*\(", txt)
    return names


def test_exports_every_declared_symbol():
    lib = ctypes.CDLL(nv.LIB_PATH)
    names = _declared()
    assert len(names) >= 10
    for n in names:
        assert hasattr(lib, n), n


def test_setup_rejects_bad_chunk_length():
    p = nv.GdnParams(1, 1, 128, 32, 128, 128, nv.BF16, nv.BF16, nv.BF16, nv.GATE_RAW,
                     nv.LAYOUT_BHTD, 0.1)
    assert not nv.lib().ptof_gdn_fwd_setup(ctypes.byref(p))
    assert "chunk length" in nv.last_error()


def test_setup_rejects_ragged_T():
    p = nv.GdnParams(1, 1, 100, 64, 128, 128, nv.BF16, nv.BF16, nv.BF16, nv.GATE_RAW,
                     nv.LAYOUT_BHTD, 0.1)
    assert not nv.lib().ptof_gdn_fwd_setup(ctypes.byref(p))
    assert "multiple" in nv.last_error()


def test_compat_execs_validate_before_launch():
    L = nv.lib()
    assert L.ptof_tri_inv_exec(None, None, nv.F16, None, 4, 256, None) == nv.EINVAL
    assert L.ptof_qkv_flash_exec(None, None, None, None, None, None, 1, 64, 64, 64, nv.F16, None) == nv.EINVAL
    assert L.ptof_gated_qk_exec(None, None, None, None, None, None, 1, 64, 64, 7, nv.F16, 0, None) == nv.EINVAL
