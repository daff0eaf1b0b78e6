"""pto_fuser on B200 — the chunked Gated DeltaNet forward of vloncar/pto-fuser,
rebuilt for sm_100a (hand-written tcgen05/TMA CUDA kernels behind a C ABI)."""
from .gdn import GDNChunkForward, chunk_gdn_forward
from .inputs import make_gdn_inputs
