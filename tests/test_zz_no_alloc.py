"""The allocation-free GDN forward entry point, ptof_gdn_fwd_exec_noalloc.

Some callers of this library cannot allocate device memory: code running inside a
device-memory allocator or an arena that owns all of the GPU's memory, or code that
replays a fixed memory plan, must not call cudaMalloc, so it cannot create the
workspace that ptof_gdn_fwd_setup allocates. The no-alloc entry point keeps its
per-chunk scratch in a fixed array inside the library instead. These tests call it
through the C ABI, twice in a row on different inputs (the array keeps the previous
call's contents), and require each result to be bit-identical to the workspace entry
point's (ptof_gdn_fwd_exec): both run the same kernels on the same coefficient
records, so any difference would mean a stale or partially written record. They also check that
a problem larger than the array is refused.

This file is collected last so that a run stopping at the first failure has run
every other test first.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

def _rel_l2(a, b):
    a, b = a.float(), b.float()
    return (torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b).clamp_min(1e-30)).item()


def _params(nv, B, H, T, D, dtype):
    return nv.GdnParams(B, H, T, 64, D, D, nv.dtype_code(dtype), nv.dtype_code(dtype),
                        nv.dtype_code(dtype), nv.GATE_RAW, nv.LAYOUT_BHTD, D ** -0.5)


def _noalloc(nv, inp, B, H, T, D, dtype):
    p = _params(nv, B, H, T, D, dtype)
    o = torch.empty(B, H, T, D, device="cuda", dtype=dtype)
    S = torch.empty(B, H, D, D, device="cuda", dtype=torch.float32)
    rc = nv.lib().ptof_gdn_fwd_exec_noalloc(
        ctypes.byref(p), inp["q"].data_ptr(), inp["k"].data_ptr(), inp["v"].data_ptr(),
        inp["beta"].data_ptr(), inp["g"].data_ptr(), None, o.data_ptr(), S.data_ptr(),
        nv.stream_handle())
    nv.check(rc)
    return o, S


@pytest.mark.parametrize("D", [128, 64])
def test_noalloc_matches_workspace_entry_twice(D):
    from pto_fuser import GDNChunkForward, make_gdn_inputs, native as nv
    B, H, T = 2, 8, 2048                     # 512 chunks, within the fixed maximum
    runner = GDNChunkForward(B, H, T, D, D, in_dtype=torch.bfloat16)
    for seed in (1, 2):                      # two calls in a row, different inputs
        inp = make_gdn_inputs(B, H, T, D, dtype=torch.bfloat16, device="cuda", seed=seed)
        o, S = _noalloc(nv, inp, B, H, T, D, torch.bfloat16)
        ref_o, ref_S = runner(inp["q"], inp["k"], inp["v"], inp["beta"], inp["g"])
        torch.cuda.synchronize()
        runner.check_status()
        # the entry's own status word: no bounded wait gave up
        nv.check(nv.lib().ptof_gdn_fwd_noalloc_status(nv.stream_handle()))
        assert torch.isfinite(o.float()).all() and torch.isfinite(S).all()
        assert torch.equal(o, ref_o) and torch.equal(S, ref_S), (
            seed, _rel_l2(o, ref_o), _rel_l2(S, ref_S))
    runner.close()


def test_noalloc_rejects_sizes_beyond_its_array():
    from pto_fuser import native as nv
    p = _params(nv, 1, 64, 8192, 128, torch.bfloat16)   # 8192 chunks > 4096
    dummy = torch.empty(16, device="cuda", dtype=torch.bfloat16)
    ptr = dummy.data_ptr()
    rc = nv.lib().ptof_gdn_fwd_exec_noalloc(ctypes.byref(p), ptr, ptr, ptr, ptr, ptr, None,
                                            ptr, None, nv.stream_handle())
    assert rc == nv.EINVAL
    assert "fixed maximum" in nv.last_error()
