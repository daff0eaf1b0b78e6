"""Generate the golden vectors that pin the CPU oracle to the reference.

Runs the reference's own fp32 torch implementations (vloncar/pto-fuser, read-only
checkout given by --ref) on small seeded inputs and stores inputs + outputs as
.npz files next to this script:

  gdn_d64.npz, gdn_d128.npz  examples/attention/_gdn_full.py:57-97  gdn_reference
  deltanet_d64.npz           src/pto_fuser/forwards/deltanet.py:114-143 deltanet_reference
  kkt_c128.npz               src/pto_fuser/forwards/fused_stages.py:140-156 kkt_reference
  scan_c128.npz              src/pto_fuser/forwards/fused_stages.py:46-62 scan_reference
  kda_d32.npz                examples/attention/_kda_full.py:38-77 kda_reference
  linear_gla.npz             examples/attention/_chunked.py:194-208 chunked_linear_reference

Inputs follow the build's benchmark distributions (q,k L2-normalised N(0,1), v N(0,1),
beta = sigmoid(N(0,1)), g = logsigmoid(N(2,1))) except where the reference helper fixes
its own (kkt/scan use make_kkt_inputs / make_scan_inputs shapes with fixed seeds).

Usage (in a container that has the reference checkout):
    python tests/golden/make_golden.py --ref /path/to/pto-fuser
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _gdn_inputs(B, H, nc, C, D, mu, seed):
    g = torch.Generator().manual_seed(seed)
    nrm = torch.nn.functional.normalize
    q = nrm(torch.randn(B, H, nc, C, D, generator=g), dim=-1)
    k = nrm(torch.randn(B, H, nc, C, D, generator=g), dim=-1)
    v = torch.randn(B, H, nc, C, D, generator=g)
    beta = torch.sigmoid(torch.randn(B, H, nc, C, generator=g))
    g_in = torch.nn.functional.logsigmoid(torch.randn(B, H, nc, C, generator=g) + mu)
    return q, k, v, beta, g_in


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="reference checkout root")
    args = ap.parse_args()
    sys.path.insert(0, os.path.join(args.ref, "src"))
    sys.path.insert(0, os.path.join(args.ref, "examples"))
    from attention._gdn_full import gdn_reference            # noqa: E402
    from pto_fuser.forwards.deltanet import deltanet_reference  # noqa: E402
    from pto_fuser.forwards import fused_stages as fs        # noqa: E402

    torch.set_num_threads(4)
    for name, (B, H, nc, C, D, seed) in {"gdn_d64": (1, 2, 2, 64, 64, 11),
                                         "gdn_d128": (1, 1, 2, 64, 128, 12)}.items():
        q, k, v, beta, g_in = _gdn_inputs(B, H, nc, C, D, 2.0, seed)
        scale = D ** -0.5
        o = gdn_reference(q, k, v, beta, g_in, scale)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"),
                            q=q.numpy(), k=k.numpy(), v=v.numpy(), beta=beta.numpy(),
                            g_in=g_in.numpy(), scale=np.float32(scale), o=o.numpy())

    B, H, nc, C, D = 1, 1, 2, 64, 64
    q, k, v, beta, _ = _gdn_inputs(B, H, nc, C, D, 2.0, 13)
    scale = D ** -0.5
    ref = deltanet_reference(q, k, v, beta, B, H, nc, C, D, scale)
    np.savez_compressed(os.path.join(HERE, "deltanet_d64.npz"),
                        q=q.numpy(), k=k.numpy(), v=v.numpy(), beta=beta.numpy(),
                        scale=np.float32(scale),
                        **{n: ref[n].numpy() for n in ("A", "T", "W", "U", "v_new",
                                                       "h_state", "o")})

    torch.manual_seed(14)
    kin = fs.make_kkt_inputs(2, 2, device="cpu")
    L = fs.kkt_reference(kin, 2, 2)["L"]
    np.savez_compressed(os.path.join(HERE, "kkt_c128.npz"),
                        k=kin["k"].float().numpy(), g_sum=kin["g_sum"].numpy(),
                        beta=kin["beta"].float().numpy(), L=L.float().numpy())

    torch.manual_seed(15)
    sin = fs.make_scan_inputs(1, 2, 2, device="cpu")
    sref = fs.scan_reference(sin, 1, 2, 2)
    np.savez_compressed(os.path.join(HERE, "scan_c128.npz"),
                        w=sin["w"].float().numpy(), u=sin["u"].float().numpy(),
                        k=sin["k"].float().numpy(), decay=sin["decay"].numpy(),
                        h_out=sref["h_out"].numpy(), final=sref["final"].numpy())
    from attention._kda_full import kda_reference, make_kda_inputs  # noqa: E402
    torch.manual_seed(16)
    kin = make_kda_inputs(1, 2, 3, 16, 32, device="cpu", dtype=torch.float32)
    ko = kda_reference(kin["q"], kin["k"], kin["v"], kin["beta"], kin["g_in"], 32 ** -0.5)
    np.savez_compressed(os.path.join(HERE, "kda_d32.npz"),
                        **{n: t.numpy() for n, t in kin.items()}, o=ko.numpy())

    from attention._chunked import chunked_linear_reference  # noqa: E402
    g = torch.Generator().manual_seed(17)
    N, nc, C, dk, dv = 2, 3, 16, 16, 8
    q = torch.nn.functional.normalize(torch.randn(N, nc, C, dk, generator=g), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(N, nc, C, dk, generator=g), dim=-1)
    v = torch.randn(N, nc, C, dv, generator=g)
    gates = 0.95 + 0.05 * torch.rand(N, nc, C, dk, generator=g)
    lo = chunked_linear_reference(q, k, v, gates, 1, N, nc, C)["o"]
    np.savez_compressed(os.path.join(HERE, "linear_gla.npz"), q=q.numpy(), k=k.numpy(),
                        v=v.numpy(), gates=gates.numpy(), o=lo.numpy())
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
