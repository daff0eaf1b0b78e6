"""GPU self-tests of the sm_100a primitives the kernels are built from: UMMA
descriptors and operand majors, TMEM accumulator lane maps (M=64 / M=128), the
TMEM A operand, negated A, and the TMA 128-byte swizzle."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _umma(M, N, K, mode):
    from pto_fuser import native as nv
    torch.manual_seed(M * 7 + N * 3 + K + mode)
    A = torch.randn(M, K, device="cuda")
    B = torch.randn(N, K, device="cuda")
    D = torch.full((M, N), float("nan"), device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    nv.check(nv.lib().ptof_selftest_umma(A.data_ptr(), B.data_ptr(), D.data_ptr(), M, N, K,
                                         mode, st.data_ptr(), nv.stream_handle()))
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    ref = A.bfloat16().float() @ B.bfloat16().float().T
    if mode & 8:
        ref = -ref
    return D, ref


@pytest.mark.parametrize("M,N,K,mode", [
    (128, 64, 128, 0), (128, 128, 64, 0), (64, 64, 128, 0), (64, 128, 64, 0),
    (128, 64, 64, 1), (128, 128, 128, 1),          # A MN-major
    (128, 64, 128, 2), (64, 128, 64, 2), (128, 192, 64, 2),   # B MN-major
    (128, 64, 64, 3), (64, 64, 64, 3),             # both MN-major
    (128, 64, 128, 4), (128, 128, 64, 4),          # A from TMEM
    (128, 64, 128, 8), (128, 64, 128, 12),         # negated A (smem / TMEM)
    (128, 256, 64, 0),
])
def test_umma(M, N, K, mode):
    D, ref = _umma(M, N, K, mode)
    err = (D - ref).abs().max().item()
    assert err < 1e-3 * max(1.0, ref.abs().max().item()), (err, mode)


def test_tma_swizzle_matches_software_layout():
    from pto_fuser import native as nv
    rows, cols = 256, 192
    src = torch.randn(rows, cols, device="cuda").bfloat16()
    out = torch.empty(64, 64, device="cuda", dtype=torch.bfloat16)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    for x0, y0 in [(0, 0), (64, 64), (128, 192)]:
        nv.check(nv.lib().ptof_selftest_tma(src.data_ptr(), rows, cols, x0, y0, out.data_ptr(),
                                            st.data_ptr(), nv.stream_handle()))
        torch.cuda.synchronize()
        assert int(st.item()) == 0
        assert torch.equal(out, src[y0:y0 + 64, x0:x0 + 64])
