"""Seeded synthetic GDN inputs with the benchmark distributions.

q, k ~ N(0,1) with each token's head vector L2-normalised; v ~ N(0,1);
beta = sigmoid(N(0,1)); per-token log decay g = logsigmoid(N(mu,1)); optional
initial state S0 ~ N(0, s0_std^2) in fp32. Generated on the CPU in fp32 with a
private generator (so results do not depend on the device), then cast and moved.
The reference's own helper (examples/attention/_gdn_full.py:37-50) draws
beta ~ U(0,1) and g = logsigmoid(N(0,1)); ``mu=0, beta_uniform=True`` reproduces it.
"""
from __future__ import annotations

from typing import Dict, Optional

import torch


def make_gdn_inputs(B: int, H: int, T: int, Dk: int, Dv: Optional[int] = None, *,
                    dtype=torch.bfloat16, device="cpu", mu: float = 2.0, seed: int = 0,
                    layout: str = "bhtd", s0_std: Optional[float] = None,
                    gated: bool = True, beta_uniform: bool = False) -> Dict[str, torch.Tensor]:
    Dv = Dk if Dv is None else Dv
    gen = torch.Generator().manual_seed(seed)
    nrm = torch.nn.functional.normalize
    q = nrm(torch.randn(B, H, T, Dk, generator=gen), dim=-1)
    k = nrm(torch.randn(B, H, T, Dk, generator=gen), dim=-1)
    v = torch.randn(B, H, T, Dv, generator=gen)
    if beta_uniform:
        beta = torch.rand(B, H, T, generator=gen)
    else:
        beta = torch.sigmoid(torch.randn(B, H, T, generator=gen))
    g = torch.nn.functional.logsigmoid(torch.randn(B, H, T, generator=gen) + mu)
    if not gated:
        g = torch.zeros_like(g)
    out = dict(q=q, k=k, v=v, beta=beta, g=g)
    if s0_std is not None:
        out["S0"] = torch.randn(B, H, Dk, Dv, generator=gen) * s0_std
    if layout == "bthd":
        out = {n: (t.transpose(1, 2) if n != "S0" else t) for n, t in out.items()}
    res = {}
    for n, t in out.items():
        dt = torch.float32 if n in ("g", "S0") else dtype
        res[n] = t.contiguous().to(device=device, dtype=dt)
    return res
