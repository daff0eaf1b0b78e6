"""pto_fuser on B200 — the chunked Gated DeltaNet forward of vloncar/pto-fuser,
rebuilt for sm_100a behind the same Python API.

The IR (EinsumNode / OpaqueNode / VecGlueNode / FusedNode / TensorOp / Program),
the staged and CUDA-graph backends, the opaque and fused-kernel registries, the
correctness gates and the transform / cost-model / policy / verifier stack keep the
reference's names. Underneath, the kernels are hand-written sm_100a CUDA in one
prebuilt library (``pto_fuser.native``), and ``fuse-gdn-forward`` lowers the whole
canonical GDN program to one tcgen05 kernel (``chunk_gdn_forward``).
"""
from .ir import (EinsumNode, FusedNode, Node, OpaqueNode, Program, TensorOp, TensorRef,
                 VecGlueNode)
from .executor import StagedExecutor, library_modes
from .registry import OpaqueContract, OpaqueRegistry, capture_mode, default_registry
from .fused import (FusedContract, FusedKernel, FusedKernelRegistry, default_fused_registry,
                    shared_fused_registry)
from .gate import GateResult, frob_rel, gate_determinism, gate_frob_rel, gate_outputs
from .graph import CaptureExecutor, GraphReplayExecutor
from .transform import (EnableDirectReads, EnableFusedStore, Transform, TransformResult,
                        canonicalize)
from .cost import CostModel, Features, Prediction
from .policy import PlannedTransform, Policy
from .report import CompilationReport, TransformRecord
from .compile import CompileResult, compile_program
from .template import (EpilogueUnit, FuseChunkOFlash, FuseContractionEpilogue,
                       FusePerDimChunkOFlash, Template, default_templates, epilogue_report,
                       extract_epilogue_unit)
from .transforms import FuseGDNForward, LowerResidentScan
from .gdn import GDNChunkForward, GDNChunkForwardVarlen, KDAChunkForward, chunk_gdn_forward
from .inputs import make_gdn_inputs

__all__ = [
    "TensorRef", "Node", "EinsumNode", "OpaqueNode", "VecGlueNode", "TensorOp", "FusedNode",
    "Program", "StagedExecutor", "library_modes", "OpaqueRegistry", "OpaqueContract",
    "default_registry", "capture_mode", "GateResult", "FusedContract", "FusedKernel",
    "FusedKernelRegistry", "default_fused_registry", "shared_fused_registry", "frob_rel",
    "gate_frob_rel", "gate_outputs", "gate_determinism", "CaptureExecutor",
    "GraphReplayExecutor", "Transform", "TransformResult", "canonicalize", "EnableDirectReads",
    "EnableFusedStore", "CostModel", "Features", "Prediction", "Policy", "PlannedTransform",
    "CompilationReport", "TransformRecord", "CompileResult", "compile_program", "EpilogueUnit",
    "extract_epilogue_unit", "Template", "default_templates", "FuseContractionEpilogue",
    "FuseChunkOFlash", "FusePerDimChunkOFlash", "epilogue_report", "LowerResidentScan",
    "FuseGDNForward", "GDNChunkForward", "GDNChunkForwardVarlen", "KDAChunkForward", "chunk_gdn_forward", "make_gdn_inputs",
]
