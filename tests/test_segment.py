"""Chunk-segment scan on CPU: the affine segment algebra against the serial oracle,
and the GDNSegmentScan orchestration (sub-segments, composition, all-gather, prefix)
in one process and as gloo world 2 / 3, with oracle backends standing in for the
CUDA forward, ptof_seg_scan_exec and ptof_seg_fix_exec (those are covered by the
-m gpu tests).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import gdn_oracle as orc
from pto_fuser import make_gdn_inputs
from pto_fuser.segment import GDNSegmentScan, split_tokens

P, T, D = 2, 768, 32       # 12 chunks per pair
SCALE = D ** -0.5


def _inputs(seed=5):
    inp = make_gdn_inputs(1, P, T, D, dtype=torch.float32, seed=seed)
    S0 = torch.randn(1, P, D, D, generator=torch.Generator().manual_seed(seed)) * 0.1
    return {n: t[0] for n, t in inp.items()}, S0[0]


def _serial(inp, S0):
    n = lambda k: inp[k].unsqueeze(0).numpy()
    o, S = orc.gdn_forward(n("q"), n("k"), n("v"), n("beta"), n("g"), SCALE, S0=S0[None].numpy())
    return o[0], S[0]


def oracle_forward(which, q4, k4, v4, b3, g3, S0, o, S_out):
    npy = lambda t: None if t is None else t.double().numpy()
    o_np, S_np = orc.gdn_forward(npy(q4), npy(k4), npy(v4), npy(b3), npy(g3), SCALE, S0=npy(S0))
    o.copy_(torch.from_numpy(o_np))
    S_out.copy_(torch.from_numpy(S_np))


def oracle_scan(A, B, X0, Xout, Xf, heads, nseg, D_, Dv):
    X0n = np.zeros((heads, D_, Dv)) if X0 is None else X0.double().numpy()
    entries, X = orc.segment_scan(A.numpy(), None if B is None else B.numpy(), X0n)
    if Xout is not None:
        Xout.copy_(torch.from_numpy(entries))
    if Xf is not None:
        Xf.copy_(torch.from_numpy(X))


def oracle_fix(o, oa, X, units, Tseg, D_):
    """o += oa @ X per unit (the checker of ptof_seg_fix_exec)."""
    prod = torch.bmm(oa.reshape(units, Tseg, D_).double(), X.reshape(units, D_, D_).double())
    o.view(units, Tseg, D_).add_(prod.to(o.dtype))


def test_split_tokens():
    assert split_tokens(768, 1) == (768,)
    assert split_tokens(768, 5) == (192, 192, 128, 128, 128)
    assert sum(split_tokens(131072, 8)) == 131072
    with pytest.raises(ValueError):
        split_tokens(100, 2)


def test_affine_segment_maps_equal_serial():
    """Segment maps from the oracle forward (A: S0 = I, v = 0; B: S0 = 0), combined by
    segment_scan, give every segment's true entry state and the serial final state."""
    inp, S0 = _inputs()
    o_ref, S_ref = _serial(inp, S0)
    nseg, Ts = 4, T // 4
    seg = lambda k, j: inp[k][:, j * Ts:(j + 1) * Ts].unsqueeze(0).numpy()
    A = np.empty((P, nseg, D, D)); B = np.empty((P, nseg, D, D))
    for j in range(nseg):
        _, A[:, j] = (x[0] for x in orc.gdn_forward(seg("q", j), seg("k", j),
                                                     np.zeros_like(seg("v", j)), seg("beta", j),
                                                     seg("g", j), SCALE,
                                                     S0=np.broadcast_to(np.eye(D), (1, P, D, D))))
        _, B[:, j] = (x[0] for x in orc.gdn_forward(seg("q", j), seg("k", j), seg("v", j),
                                                     seg("beta", j), seg("g", j), SCALE))
    entries, S_fin = orc.segment_scan(A, B, S0.numpy())
    assert np.allclose(S_fin, S_ref, rtol=1e-9, atol=1e-11)
    for j in range(nseg):
        o_j, _ = orc.gdn_forward(seg("q", j), seg("k", j), seg("v", j), seg("beta", j),
                                 seg("g", j), SCALE, S0=entries[None, :, j])
        assert np.allclose(o_j[0], o_ref[:, j * Ts:(j + 1) * Ts], rtol=1e-9, atol=1e-11)


@pytest.mark.parametrize("segments", [1, 3])
def test_segment_scan_single_process(segments):
    inp, S0 = _inputs(seed=7)
    o_ref, S_ref = _serial(inp, S0)
    run = GDNSegmentScan(P, T, D, segments=segments, in_dtype=torch.float64, out_dtype=torch.float64,
                         scale=SCALE, forward=oracle_forward, scan=oracle_scan, fix=oracle_fix)
    d = lambda k: inp[k].double()
    o, S = run(d("q"), d("k"), d("v"), d("beta"), d("g"), S0.double())
    assert np.allclose(o.numpy(), o_ref, rtol=1e-5, atol=1e-6)   # states are fp32
    assert np.allclose(S.numpy(), S_ref, rtol=1e-5, atol=1e-6)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "pto-fuser_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from tests.test_segment import _inputs, oracle_fix, oracle_forward, oracle_scan
        from pto_fuser.segment import GDNSegmentScan as Seg, split_tokens as split
        inp, S0 = _inputs(seed=11)
        sizes = split(T, world)
        a = sum(sizes[:rank])
        loc = lambda k: inp[k][:, a:a + sizes[rank]].double().contiguous()
        run = Seg(P, sizes[rank], D, segments=2 if sizes[rank] % 256 == 0 else 1,
                  group=dist.group.WORLD, in_dtype=torch.float64, out_dtype=torch.float64,
                  scale=SCALE, forward=oracle_forward, scan=oracle_scan, fix=oracle_fix)
        o, S = run(loc("q"), loc("k"), loc("v"), loc("beta"), loc("g"), S0.double())
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), o=o.numpy(), S=S.numpy(), a=a)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_segment_scan_matches_serial(tmp_path, world):
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    inp, S0 = _inputs(seed=11)
    o_ref, S_ref = _serial(inp, S0)
    sizes = split_tokens(T, world)
    for r in range(world):
        res = np.load(tmp_path / f"r{r}.npz")
        a = int(res["a"])
        assert np.allclose(res["o"], o_ref[:, a:a + sizes[r]], rtol=1e-5, atol=1e-6)
    assert np.allclose(res["S"], S_ref, rtol=1e-5, atol=1e-6)   # last rank: final state


def test_local_split_planner():
    """The head/tail planner: no split when the pairs fill the SMs, a split that tiles
    T (whole 128-token tail tiles) when they do not."""
    from pto_fuser.segment import plan_local_split
    assert plan_local_split(148, 16384, 148) is None
    assert plan_local_split(128, 16384, 148) is None
    assert plan_local_split(64, 16384, 148) is None   # measured: no split beats serial
    for P in (32, 16, 8):
        L0, s, Ls = plan_local_split(P, 16384, 148)
        assert L0 + s * Ls == 16384 and Ls % 128 == 0 and L0 % 64 == 0
        assert s >= 1 and L0 < 16384
