"""Structural transforms: the GDN forward's resident-state scan lowering (reference:
src/pto_fuser/transforms/gdn.py), the B200 whole-forward fusion, and the batched
intra-chunk scores of the chunked linear family (reference: transforms/chunked.py)."""
from .chunked import BatchChunkIntraScore, select_prologue_kernel
from .gdn import FuseGDNForward, LowerResidentScan
from .kda import LowerPerDimScan

__all__ = ["LowerResidentScan", "FuseGDNForward", "BatchChunkIntraScore",
           "select_prologue_kernel", "LowerPerDimScan"]
