"""KDA's resident-state scan lowering: the unrolled per-chunk scan of
``build_kda_program`` becomes one ``chunk_h_scan`` FusedNode with a per-key-dimension
decay ([B, H, nc, D]) plus the all-chunk ``v_new = U - W h`` recompute; the per-channel
counterpart of ``LowerResidentScan`` (contract of the reference's
transforms/kda.py:19-70: its name, the nodes it matches and the key it emits)."""
from __future__ import annotations

from .gdn import _ResidentScanRewrite


class LowerPerDimScan(_ResidentScanRewrite):
    name = "lower-perdim-scan"
    summary = "unrolled KDA scan -> chunk_h_scan FusedNode (resident S, per-dim decay)"
    key_coef = "coef_krest"
    chunk_names = ("Wc{c}_s", "Wc{c}", "WS{c}", "Uc{c}", "vn{c}", "kc{c}_s", "kc{c}", "krc{c}",
                   "krest{c}", "dS{c}", "sc{c}", "Sd{c}", "S{c1}")
    perdim = True
