"""Reference chunk-attention forwards built on the IR (program builders + fp32
torch references)."""
from .chunked import build_chunked_linear_program, prepare_chunked_inputs
from .kda import build_kda_program, make_kda_inputs, prepare_kda_bindings
from .deltanet import build_deltanet_program, deltanet_reference, make_inputs
from .fused_stages import (build_kkt_fused_program, build_scan_fused_program,
                           build_scan_staged_program, kkt_reference, make_kkt_inputs,
                           make_scan_inputs, scan_reference)
from .gdn import (build_gdn_program, gdn_contraction_stages, gdn_reference, make_gdn_inputs,
                  prepare_gdn_bindings)

__all__ = ["build_kda_program", "make_kda_inputs", "prepare_kda_bindings",
           "build_chunked_linear_program", "prepare_chunked_inputs", "build_deltanet_program", "deltanet_reference", "make_inputs",
           "gdn_contraction_stages", "build_gdn_program", "gdn_reference", "make_gdn_inputs",
           "prepare_gdn_bindings", "make_scan_inputs", "scan_reference",
           "build_scan_staged_program", "build_scan_fused_program", "make_kkt_inputs",
           "kkt_reference", "build_kkt_fused_program"]
