"""Structural transforms of the GDN forward: the resident-state scan lowering
(reference: src/pto_fuser/transforms/gdn.py) and the B200 whole-forward fusion."""
from .gdn import FuseGDNForward, LowerResidentScan

__all__ = ["LowerResidentScan", "FuseGDNForward"]
