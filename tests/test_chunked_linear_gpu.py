"""The chunked linear family with the batched intra score on CUDA: the transformed
program (one fused qk_prologue / gated_qk_native_v2 launch for all chunks) against
the token-recurrent oracle, at the reference's own gate (rel-L2 2e-2, fp16 work)."""
import pytest
import torch

from oracle import gdn_oracle as orc

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind", ["retnet", "mamba2", "gla"])
def test_transformed_program_on_gpu(kind):
    from pto_fuser import StagedExecutor
    from pto_fuser.forwards import build_chunked_linear_program, prepare_chunked_inputs
    from pto_fuser.transforms import BatchChunkIntraScore
    N, NC, C, DK, DV = 4, 8, 64, 64, 64
    g = torch.Generator().manual_seed(1)
    mk = lambda *s: torch.randn(*s, generator=g) * 0.2
    q = torch.nn.functional.normalize(mk(N, NC, C, DK), dim=-1)
    k = torch.nn.functional.normalize(mk(N, NC, C, DK), dim=-1)
    v = mk(N, NC, C, DV)
    shape = (N, NC, C, DK)
    if kind == "retnet":
        gates = torch.full(shape, 0.985)
    elif kind == "mamba2":
        gates = (0.97 + 0.03 * torch.rand(N, NC, C, 1, generator=g)).expand(shape).clone()
    else:
        gates = 0.97 + 0.03 * torch.rand(shape, generator=g)
    binds = {n: t.cuda() for n, t in prepare_chunked_inputs(q, k, v, gates).items()}
    prog = build_chunked_linear_program(N, NC, C, DK, DV)
    fused = BatchChunkIntraScore(N, NC, C, DK, DV, per_dim_gate=(kind == "gla")).apply(prog)
    assert fused.changed
    o = StagedExecutor().run(fused.program, binds)["o"]
    torch.cuda.synchronize()
    flat = lambda t: t.reshape(N, NC * C, -1).numpy()
    ref = orc.linear_attention_recurrent(flat(q), flat(k), flat(v), flat(gates))
    assert orc.rel_l2(o.float().reshape(N, NC * C, DV).cpu().numpy(), ref) < 2e-2
