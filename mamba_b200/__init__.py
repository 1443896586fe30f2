"""mamba_b200 — a B200-native (sm_100a) selective-scan engine.

Public operators (all CUDA-only, backed by libmamba_b200_ss.so):
  selective_scan_fn, SelectiveScanFn   forward / backward scan with optional SiLU(z) gate
  selective_state_update               single-token decode step
  selective_scan_ext                   drop-in for the reference's native `selective_scan`
  mamba_inner_fn, MambaInnerFn         the whole Mamba block from the input projection's output
                                       (conv + SiLU, projections, scan + gate, output projection)
  mamba_simple_forward                 a MambaSimple module's forward through mamba_inner_fn
  rms_norm_fn, rms_norm                residual add + RMSNorm in one kernel (forward / backward)
  causal_lm_forward                    a CausalLM's forward through the fused block and norm
  generate, Decoder                    prefill + cached single-token decode (CUDA-graph step)
  check_device_status                  raise if a kernel's bounded wait gave up since the last check
  set_status_check                     check after every scan call (debugging; synchronises)
"""
from ._lib import check_device_status, set_status_check
from .decode import Decoder, generate
from .inner import MambaInnerFn, mamba_inner_fn, mamba_simple_forward
from .lm import causal_lm_forward
from .norm import rms_norm, rms_norm_fn
from .selective_scan_interface import SelectiveScanFn, selective_scan_fn, selective_state_update

__all__ = ["SelectiveScanFn", "selective_scan_fn", "selective_state_update", "MambaInnerFn", "mamba_inner_fn",
           "mamba_simple_forward", "rms_norm_fn", "rms_norm", "causal_lm_forward", "generate", "Decoder",
           "check_device_status", "set_status_check"]
__version__ = "0.1.0"
