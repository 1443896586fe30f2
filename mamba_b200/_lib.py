"""ctypes binding of libmamba_b200_ss.so (declared in include/mamba_b200_ss.h).

The library is the product's only compute path: there is no CPU or PyTorch fallback.
Loading fails loudly if the library was not built, and every call checks that its
tensors are CUDA tensors on one device.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libmamba_b200_ss.so")

SS_F32, SS_BF16, SS_F16 = 0, 1, 2
SS_LAYOUT_BDL, SS_LAYOUT_BLD = 0, 1
SS_OK, SS_ERR_INVALID, SS_ERR_UNSUPPORTED, SS_ERR_CUDA = 0, 1, 2, 3
SS_MAX_DSTATE = 256
TILE = 16  # time steps between checkpoints (kTile in csrc/ss_common.cuh)

_DTYPES = {torch.float32: SS_F32, torch.bfloat16: SS_BF16, torch.float16: SS_F16}

c_int, c_i64, c_vp = ctypes.c_int, ctypes.c_int64, ctypes.c_void_p


class FwdArgs(ctypes.Structure):
    _fields_ = [
        ("batch", c_int), ("dim", c_int), ("seqlen", c_int), ("dstate", c_int), ("ngroups", c_int),
        ("var_B", c_int), ("var_C", c_int), ("delta_softplus", c_int), ("io_dtype", c_int),
        ("bc_dtype", c_int),
        ("u", c_vp), ("u_batch_stride", c_i64), ("u_dim_stride", c_i64),
        ("delta", c_vp), ("delta_batch_stride", c_i64), ("delta_dim_stride", c_i64),
        ("A", c_vp), ("B", c_vp), ("C", c_vp), ("D", c_vp),
        ("z", c_vp), ("z_batch_stride", c_i64), ("z_dim_stride", c_i64),
        ("delta_bias", c_vp),
        ("out", c_vp), ("out_batch_stride", c_i64), ("out_dim_stride", c_i64),
        ("ckpt", c_vp), ("last_state", c_vp),
        ("out_y", c_vp), ("out_y_batch_stride", c_i64), ("out_y_dim_stride", c_i64),
        ("work", c_vp),
        ("layout", c_int),
    ]


class BwdArgs(ctypes.Structure):
    _fields_ = [
        ("f", FwdArgs),
        ("dout", c_vp), ("dout_batch_stride", c_i64), ("dout_dim_stride", c_i64),
        ("du", c_vp), ("du_batch_stride", c_i64), ("du_dim_stride", c_i64),
        ("ddelta", c_vp), ("ddelta_batch_stride", c_i64), ("ddelta_dim_stride", c_i64),
        ("dz", c_vp), ("dz_batch_stride", c_i64), ("dz_dim_stride", c_i64),
        ("y", c_vp), ("y_batch_stride", c_i64), ("y_dim_stride", c_i64),
        ("dA", c_vp), ("dB", c_vp), ("dC", c_vp), ("dD", c_vp), ("ddelta_bias", c_vp),
    ]


class StepArgs(ctypes.Structure):
    _fields_ = [
        ("batch", c_int), ("dim", c_int), ("dstate", c_int), ("ngroups", c_int),
        ("dt_softplus", c_int), ("io_dtype", c_int), ("bc_dtype", c_int),
        ("state", c_vp), ("state_batch_stride", c_i64),
        ("x", c_vp), ("x_batch_stride", c_i64),
        ("dt", c_vp), ("dt_batch_stride", c_i64),
        ("A", c_vp), ("B", c_vp), ("B_batch_stride", c_i64), ("C", c_vp), ("C_batch_stride", c_i64),
        ("D", c_vp),
        ("z", c_vp), ("z_batch_stride", c_i64),
        ("dt_bias", c_vp),
        ("out", c_vp), ("out_batch_stride", c_i64),
        ("dt_proj", c_vp), ("dt_rank", c_int),
    ]


class ConvArgs(ctypes.Structure):
    _fields_ = [
        ("batch", c_int), ("dim", c_int), ("seqlen", c_int), ("width", c_int), ("silu", c_int),
        ("io_dtype", c_int),
        ("x", c_vp), ("x_batch_stride", c_i64), ("x_seq_stride", c_i64),
        ("weight", c_vp), ("bias", c_vp), ("state_in", c_vp), ("state_out", c_vp),
        ("u", c_vp), ("u_batch_stride", c_i64), ("u_dim_stride", c_i64),
        ("z", c_vp), ("z_batch_stride", c_i64), ("z_seq_stride", c_i64),
        ("zt", c_vp), ("zt_batch_stride", c_i64), ("zt_dim_stride", c_i64),
    ]


class ConvBwdArgs(ctypes.Structure):
    _fields_ = [
        ("f", ConvArgs),
        ("du", c_vp), ("du_batch_stride", c_i64), ("du_dim_stride", c_i64),
        ("dx", c_vp), ("dx_batch_stride", c_i64), ("dx_seq_stride", c_i64),
        ("dzt", c_vp), ("dzt_batch_stride", c_i64), ("dzt_dim_stride", c_i64),
        ("dz", c_vp), ("dz_batch_stride", c_i64), ("dz_seq_stride", c_i64),
        ("dweight", c_vp), ("dbias", c_vp),
    ]


class ConvStepArgs(ctypes.Structure):
    _fields_ = [
        ("batch", c_int), ("dim", c_int), ("width", c_int), ("silu", c_int), ("io_dtype", c_int),
        ("state", c_vp), ("state_batch_stride", c_i64),
        ("x", c_vp), ("x_batch_stride", c_i64),
        ("weight", c_vp), ("bias", c_vp),
        ("u", c_vp), ("u_batch_stride", c_i64),
    ]


class RmsNormArgs(ctypes.Structure):
    _fields_ = [
        ("rows", c_int), ("dim", c_int), ("io_dtype", c_int), ("unit_offset", c_int), ("eps", ctypes.c_float),
        ("x", c_vp), ("x_row_stride", c_i64),
        ("residual", c_vp), ("residual_row_stride", c_i64),
        ("weight", c_vp),
        ("y", c_vp), ("y_row_stride", c_i64),
        ("residual_out", c_vp), ("residual_out_row_stride", c_i64),
        ("rstd", c_vp),
    ]


class RmsNormBwdArgs(ctypes.Structure):
    _fields_ = [
        ("rows", c_int), ("dim", c_int), ("io_dtype", c_int), ("unit_offset", c_int),
        ("h", c_vp), ("h_row_stride", c_i64),
        ("weight", c_vp), ("rstd", c_vp),
        ("dy", c_vp), ("dy_row_stride", c_i64),
        ("dh_in", c_vp), ("dh_in_row_stride", c_i64),
        ("dh", c_vp), ("dh_row_stride", c_i64),
        ("dweight", c_vp),
    ]


class MambaStepArgs(ctypes.Structure):
    _fields_ = [
        ("batch", c_int), ("dim", c_int), ("dstate", c_int), ("width", c_int), ("dt_rank", c_int),
        ("io_dtype", c_int), ("dt_softplus", c_int),
        ("xz", c_vp), ("xz_batch_stride", c_i64),
        ("conv_state", c_vp), ("conv_weight", c_vp), ("conv_bias", c_vp),
        ("x_proj", c_vp), ("dt_proj", c_vp), ("dt_bias", c_vp), ("A", c_vp), ("D", c_vp),
        ("ssm_state", c_vp),
        ("y", c_vp), ("y_batch_stride", c_i64),
    ]


# ss_struct_size index order
STRUCTS = (FwdArgs, BwdArgs, StepArgs, ConvArgs, ConvBwdArgs, ConvStepArgs, RmsNormArgs, RmsNormBwdArgs,
           MambaStepArgs)
ABI_VERSION = 8
MAX_CONV_WIDTH = 4

EXPORTS = ("ss_fwd", "ss_bwd", "ss_step", "ss_ckpt_elems", "ss_work_elems", "ss_status_string",
           "ss_last_cuda_error", "ss_abi_version", "ss_struct_size", "ss_device_status",
           "ss_bwd_noalloc", "ss_conv_fwd", "ss_conv_bwd", "ss_conv_step", "ss_rmsnorm_fwd", "ss_rmsnorm_bwd",
           "ss_mamba_step", "ss_set_wait_limit", "ss_set_time_chunks")
NOALLOC_MAX_CKPT_ELEMS = 4194304  # SS_NOALLOC_MAX_CKPT_ELEMS

_lib = None
_lock = threading.Lock()


def lib():
    """Load the library once.  Raises if it is missing (no fallback exists)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"{LIB_PATH} is not built; run `python -m mamba_b200.build` "
                        "(mamba_b200 has no CPU fallback)")
                L = ctypes.CDLL(LIB_PATH)
                L.ss_fwd.argtypes = [ctypes.POINTER(FwdArgs), c_vp]
                L.ss_bwd.argtypes = [ctypes.POINTER(BwdArgs), c_vp]
                L.ss_bwd_noalloc.argtypes = [ctypes.POINTER(BwdArgs), c_vp]
                L.ss_bwd_noalloc.restype = c_int
                L.ss_step.argtypes = [ctypes.POINTER(StepArgs), c_vp]
                L.ss_conv_fwd.argtypes = [ctypes.POINTER(ConvArgs), c_vp]
                L.ss_conv_bwd.argtypes = [ctypes.POINTER(ConvBwdArgs), c_vp]
                L.ss_conv_step.argtypes = [ctypes.POINTER(ConvStepArgs), c_vp]
                L.ss_rmsnorm_fwd.argtypes = [ctypes.POINTER(RmsNormArgs), c_vp]
                L.ss_rmsnorm_bwd.argtypes = [ctypes.POINTER(RmsNormBwdArgs), c_vp]
                L.ss_mamba_step.argtypes = [ctypes.POINTER(MambaStepArgs), c_vp]
                for f in ("ss_fwd", "ss_bwd", "ss_step", "ss_last_cuda_error", "ss_abi_version",
                          "ss_conv_fwd", "ss_conv_bwd", "ss_conv_step", "ss_rmsnorm_fwd", "ss_rmsnorm_bwd",
                          "ss_mamba_step", "ss_set_wait_limit", "ss_set_time_chunks"):
                    getattr(L, f).restype = c_int
                L.ss_ckpt_elems.argtypes = [c_int, c_int, c_int, c_int]
                L.ss_ckpt_elems.restype = ctypes.c_size_t
                L.ss_work_elems.argtypes = [c_int, c_int, c_int, c_int]
                L.ss_work_elems.restype = ctypes.c_size_t
                L.ss_status_string.argtypes = [c_int]
                L.ss_status_string.restype = ctypes.c_char_p
                L.ss_device_status.argtypes = [c_int, c_vp]
                L.ss_device_status.restype = c_int
                L.ss_set_time_chunks.argtypes = [c_int]
                L.ss_set_time_chunks.restype = c_int
                L.ss_set_wait_limit.argtypes = [ctypes.c_longlong]
                L.ss_set_wait_limit.restype = ctypes.c_longlong
                L.ss_struct_size.argtypes = [c_int]
                L.ss_struct_size.restype = ctypes.c_size_t
                if L.ss_abi_version() != ABI_VERSION:
                    raise RuntimeError(f"{LIB_PATH}: ABI version {L.ss_abi_version()} != {ABI_VERSION}; rebuild it")
                for i, st in enumerate(STRUCTS):
                    if L.ss_struct_size(i) != ctypes.sizeof(st):
                        raise RuntimeError(f"{LIB_PATH}: struct {st.__name__} layout mismatch "
                                           f"({L.ss_struct_size(i)} != {ctypes.sizeof(st)} bytes)")
                _lib = L
    return _lib


def check(rc: int, what: str) -> None:
    if rc == SS_OK:
        return
    L = lib()
    msg = L.ss_status_string(rc).decode()
    if rc == SS_ERR_CUDA:
        msg += f" (cudaError {L.ss_last_cuda_error()})"
    if rc == SS_ERR_UNSUPPORTED:
        raise NotImplementedError(f"{what}: {msg}")
    if rc == SS_ERR_INVALID:
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what}: {msg}")


def dtype_code(t: torch.dtype) -> int:
    try:
        return _DTYPES[t]
    except KeyError:
        raise NotImplementedError(f"dtype {t} is not supported (float32, bfloat16, float16)") from None


def ptr(t):
    return None if t is None else t.data_ptr()


# the current stream's handle without building a torch.cuda.Stream object per call
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_of(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    return _raw_stream(idx) if _raw_stream is not None else torch.cuda.current_stream(device).cuda_stream


def device_status(device, reset: bool = True) -> int:
    """Error bits raised by kernels on `device` (1 = a bounded TMA wait timed out)."""
    import torch

    with torch.cuda.device(device):
        return int(lib().ss_device_status(int(reset), stream_of(torch.device(device))))


STATUS_BITS = {1: "a bounded wait for a TMA tile gave up (the CTA ended early; its outputs are incomplete)"}


def check_device_status(device=None, what: str = "mamba_b200") -> None:
    """Raise RuntimeError if any kernel on `device` (default: the current one) raised an error bit
    since the last check; clears the bits.  Synchronises the current stream."""
    import torch

    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    bits = device_status(dev, reset=True)
    if bits < 0:
        raise RuntimeError(f"{what}: the device status word of {dev} could not be read")
    if bits:
        why = "; ".join(v for k, v in STATUS_BITS.items() if bits & k) or "unknown bits"
        raise RuntimeError(f"{what}: kernel error status 0x{bits:x} on {dev}: {why}")


# Per-call status checks: off by default (each check synchronises the stream); on with
# set_status_check(True) or MAMBA_B200_CHECK_STATUS=1 in the environment.
_status_check = os.environ.get("MAMBA_B200_CHECK_STATUS", "0") not in ("", "0")


def set_status_check(enabled: bool) -> bool:
    """Check the device status word after every scan call (raising on an error bit); returns the
    previous setting.  Each check synchronises the stream, so it is a debugging aid."""
    global _status_check
    prev, _status_check = _status_check, bool(enabled)
    return prev


def maybe_check_status(device, what: str) -> None:
    if _status_check:
        check_device_status(device, what)


def set_wait_limit(cycles: int) -> int:
    """Limit (SM clock cycles) of the scan kernels' bounded waits for a TMA tile, for the launches
    that follow; returns the previous one.  cycles < 0 restores the default (~2 s)."""
    return int(lib().ss_set_wait_limit(int(cycles)))


def set_time_chunks(chunks: int) -> int:
    """Time chunks per scan pass for the calls that follow (0: chosen from the shape; k >= 1:
    forced, 1 = never split).  Returns the previous setting."""
    return int(lib().ss_set_time_chunks(int(chunks)))


def ckpt_elems(batch, dim, seqlen, dstate) -> int:
    return int(lib().ss_ckpt_elems(batch, dim, seqlen, dstate))


def work_elems(batch, dim, seqlen, dstate) -> int:
    """fp32 scratch of a scan call: the state groups' sums (dstate > 16) or the time chunks'
    summaries (dstate <= 16 when the sequence is split; 0 otherwise)."""
    return int(lib().ss_work_elems(batch, dim, seqlen, dstate))
