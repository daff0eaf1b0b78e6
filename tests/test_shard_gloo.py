"""Host-side multi-process path on CPU: world_size 2 over gloo.

Each rank takes its contiguous block of (b, h) pairs (pto_fuser.shard), runs the
forward on it (here the CPU oracle: the GPU kernel is covered by the -m gpu tests,
and a gloo rank has no GPU), and rank 0 gathers the blocks; the result must equal
the unsharded forward. Also checks the max-over-ranks step time and the partition.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from pto_fuser.shard import gather_pairs, max_over_ranks, shard_heads, shard_pairs

B, H, T, D = 1, 5, 128, 32   # 5 pairs over 2 ranks: blocks of 3 and 2


def test_shard_pairs_partition():
    for n in (1, 5, 128):
        for world in (1, 2, 3, 8):
            seen = []
            for r in range(world):
                a, b = shard_pairs(n, world, r)
                assert 0 <= a <= b <= n
                seen.extend(range(a, b))
            assert seen == list(range(n))
    with pytest.raises(ValueError):
        shard_pairs(4, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "pto-fuser_b200")]
    from oracle import gdn_oracle as orc
    from pto_fuser import make_gdn_inputs
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        inp = make_gdn_inputs(B, H, T, D, dtype=torch.float32, seed=3)   # same on every rank
        f = lambda n: shard_heads(inp[n], world, rank).unsqueeze(0).numpy()
        o, S = orc.gdn_forward(f("q"), f("k"), f("v"), f("beta"), f("g"), D ** -0.5)
        o_all = gather_pairs(torch.from_numpy(o[0]), B * H)
        S_all = gather_pairs(torch.from_numpy(S[0]), B * H)
        t = max_over_ranks(1.0 + rank)
        if rank == 0:
            np.savez(os.path.join(out_dir, "res.npz"), o=o_all.numpy(), S=S_all.numpy(), t=t)
    finally:
        dist.destroy_process_group()


def test_gloo_world2_sharded_forward_matches_unsharded(tmp_path):
    from oracle import gdn_oracle as orc
    from pto_fuser import make_gdn_inputs
    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    res = np.load(tmp_path / "res.npz")
    inp = make_gdn_inputs(B, H, T, D, dtype=torch.float32, seed=3)
    n = lambda k: inp[k].numpy()
    o, S = orc.gdn_forward(n("q"), n("k"), n("v"), n("beta"), n("g"), D ** -0.5)
    assert np.allclose(res["o"], o.reshape(B * H, T, D), rtol=1e-10, atol=1e-12)
    assert np.allclose(res["S"], S.reshape(B * H, D, D), rtol=1e-10, atol=1e-12)
    assert float(res["t"]) == 2.0   # the slower rank's time
