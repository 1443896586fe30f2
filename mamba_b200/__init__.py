"""mamba_b200 — a B200-native (sm_100a) selective-scan engine.

Public operators (all CUDA-only, backed by libmamba_b200_ss.so):
  selective_scan_fn, SelectiveScanFn   forward / backward scan with optional SiLU(z) gate
  selective_state_update               single-token decode step
  selective_scan_ext                   drop-in for the reference's native `selective_scan`
"""
from .selective_scan_interface import SelectiveScanFn, selective_scan_fn, selective_state_update

__all__ = ["SelectiveScanFn", "selective_scan_fn", "selective_state_update"]
__version__ = "0.1.0"
