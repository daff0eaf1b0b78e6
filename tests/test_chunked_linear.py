"""The chunked linear-attention family (vanilla LA, RetNet, Mamba-2, GLA) on the IR:
the canonical program (pto_fuser.forwards.chunked) against the token-recurrent
oracle on CPU, and the batch-chunk-intra-score transform's rewrite."""
import numpy as np
import pytest
import torch

from oracle import gdn_oracle as orc
from pto_fuser import FusedNode, StagedExecutor
from pto_fuser.forwards import build_chunked_linear_program, prepare_chunked_inputs
from pto_fuser.transforms import BatchChunkIntraScore

N, NC, C, DK, DV = 3, 4, 16, 32, 24


def _qkv(seed=0):
    g = torch.Generator().manual_seed(seed)
    mk = lambda *s: torch.randn(*s, generator=g) * 0.2
    q = torch.nn.functional.normalize(mk(N, NC, C, DK), dim=-1)
    k = torch.nn.functional.normalize(mk(N, NC, C, DK), dim=-1)
    return q, k, mk(N, NC, C, DV), g


def _gates(kind, g):
    shape = (N, NC, C, DK)
    if kind == "vanilla":
        return torch.ones(shape)
    if kind == "retnet":       # one constant per head
        return torch.tensor([0.97, 0.95, 0.99]).view(N, 1, 1, 1).expand(shape).clone()
    if kind == "mamba2":       # one scalar per token
        return (0.95 + 0.05 * torch.rand(N, NC, C, 1, generator=g)).expand(shape).clone()
    return 0.95 + 0.05 * torch.rand(shape, generator=g)          # gla: per channel


@pytest.mark.parametrize("kind", ["vanilla", "retnet", "mamba2", "gla"])
def test_canonical_program_matches_recurrence(kind):
    q, k, v, g = _qkv()
    gates = _gates(kind, g)
    binds = prepare_chunked_inputs(q, k, v, gates, work=torch.float32)
    prog = build_chunked_linear_program(N, NC, C, DK, DV, work=torch.float32)
    o = StagedExecutor().run(prog, binds)["o"]
    flat = lambda t: t.reshape(N, NC * C, -1).numpy()
    ref = orc.linear_attention_recurrent(flat(q), flat(k), flat(v), flat(gates))
    assert orc.rel_l2(o.reshape(N, NC * C, DV).numpy(), ref) < 1e-5


@pytest.mark.parametrize("per_dim,C_,kernel", [(False, 16, "gated_qk_native_v2"),
                                               (True, 16, "qk_prologue"),
                                               (True, 128, "qk_prologue_v2")])
def test_batch_chunk_intra_score_rewrite(per_dim, C_, kernel):
    prog = build_chunked_linear_program(N, NC, C_, DK, DV)
    t = BatchChunkIntraScore(N, NC, C_, DK, DV, per_dim_gate=per_dim)
    assert t.match(prog) == 1
    res = t.apply(prog)
    assert res.changed
    fused = [n for n in res.program.nodes if isinstance(n, FusedNode)]
    assert len(fused) == 1 and fused[0].kernel == kernel and len(fused[0].subsumes) == NC
    eq = lambda p: sum(1 for n in p.nodes if getattr(n, "equation", "") == "nid,njd->nij")
    assert eq(prog) == NC and eq(res.program) == 0
    assert t.match(res.program) == 0          # idempotent
