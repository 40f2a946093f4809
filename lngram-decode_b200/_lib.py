"""ctypes binding of the C ABI (``include/lngram_b200.h``) and its status -> exception mapping.

The library is the in-tree ``liblngram_b200.so``; there is no CPU fallback: importing works
anywhere (for the symbol checks), but every compute entry point raises unless the library is
built and a CUDA device of compute capability 10.x is present.
"""

from __future__ import annotations

import contextlib
import ctypes as C
from pathlib import Path

import torch

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "liblngram_b200.so"

F32, BF16, F16, U8, I32, I64, BOOL = range(7)
MAX_ORDERS = 4
OK, ERR_ARGUMENT, ERR_CUDA, ERR_UNSUPPORTED, ERR_DEVICE, ERR_STATE = range(6)

_TORCH_DT = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16, torch.uint8: U8, torch.int32: I32,
             torch.int64: I64, torch.bool: BOOL}


def dtype_code(t: torch.dtype) -> int:
    try:
        return _TORCH_DT[t]
    except KeyError:
        raise ValueError(f"unsupported dtype {t}") from None


class Tables(C.Structure):
    _fields_ = [("n_orders", C.c_int32), ("orders", C.c_int32 * MAX_ORDERS), ("tables", C.c_void_p * MAX_ORDERS),
                ("table_dtype", C.c_int32), ("bits", C.c_int32), ("num_routes", C.c_int64),
                ("memory_dim", C.c_int64), ("row_ss", C.c_void_p * MAX_ORDERS)]


class Readout(C.Structure):
    _fields_ = [("hidden", C.c_int64), ("num_heads", C.c_int32), ("num_kv_heads", C.c_int32),
                ("head_dim", C.c_int32), ("eps", C.c_float), ("sink_logit", C.c_float), ("conv_kernel", C.c_int32),
                ("conv_dilation", C.c_int32), ("act_dtype", C.c_int32), ("w_qk", C.c_void_p), ("w_vo", C.c_void_p),
                ("conv_norm", C.c_void_p), ("conv_weight", C.c_void_p), ("conv_bias", C.c_void_p),
                ("router_w", C.c_void_p), ("router_in_dim", C.c_int64), ("router_w_split", C.c_void_p)]


class Array(C.Structure):
    _fields_ = [("name", C.c_char_p), ("data_host", C.c_void_p), ("dtype", C.c_int32), ("ndim", C.c_int32),
                ("shape", C.c_int64 * 4)]


class DrafterNumbers(C.Structure):
    _fields_ = [("d_model", C.c_int64), ("vocab", C.c_int64), ("routes", C.c_int64), ("bits", C.c_int64),
                ("mem_dim", C.c_int64), ("kv_heads", C.c_int64), ("head_dim", C.c_int64), ("q_heads", C.c_int64),
                ("ssm_dim", C.c_int64), ("sketch_k", C.c_int64), ("shortlist_cap", C.c_int64),
                ("router_eps", C.c_double), ("draft_eps", C.c_double), ("mem_eps", C.c_double),
                ("ssm_eps", C.c_double), ("softmax_scale", C.c_double), ("sink_logit", C.c_double),
                ("router_ssm", C.c_int32), ("query_ssm", C.c_int32), ("n_orders", C.c_int32),
                ("orders", C.c_int32 * MAX_ORDERS)]


P = C.c_void_p
i32, i64, f32, sz = C.c_int32, C.c_int64, C.c_float, C.c_size_t
PT, PR = C.POINTER(Tables), C.POINTER(Readout)

# name -> (restype, argtypes); mirrors include/lngram_b200.h
SIGNATURES = {
    "lng_abi_version": (C.c_int, []),
    "lng_last_error": (C.c_char_p, []),
    "lng_device_ok": (C.c_int, []),
    "lng_device_error": (C.c_int, [C.c_int]),
    "lng_quantize_route_logits": (C.c_int, [P, i64, i64, i32, P, i32, P]),
    "lng_route_codes": (C.c_int, [P, i32, i64, i64, i64, P, i64, i32, P, i32, P, P]),
    "lng_router_prepare": (C.c_int, [P, i64, i64, P, P]),
    "lng_route_codes_split": (C.c_int, [P, i64, i64, i64, P, i64, i32, P, P]),
    "lng_embed2_features": (C.c_int, [P, P, i64, P, i32, i64, i64, P, P, P, f32, P, P]),
    "lng_table_row_ss": (C.c_int, [PT, C.POINTER(C.c_void_p), P]),
    "lng_lookup_route_chunk": (C.c_int, [PT, P, i32, i64, i64, i64, i64, P, P, i64, P, i32, P]),
    "lng_lookup_backward": (C.c_int, [PT, P, i32, i64, i64, i64, i64, P, P, P, i32, P, i64, f32, f32, i32, P,
                                      C.POINTER(C.c_void_p), P]),
    "lng_lookup_windows": (C.c_int, [PT, P, i32, i64, i64, P, P, i32, P]),
    "lng_lookup_serving_rows": (C.c_int, [PT, P, i32, i64, i64, i64, P, P]),
    "lng_serving_permute": (C.c_int, [P, P, i32, i64, i32, i32, i64, P]),
    "lng_host_map": (C.c_int, [P, sz, C.POINTER(P)]),
    "lng_host_unmap": (C.c_int, [P]),
    "lng_packed_suffix": (C.c_int, [P, i32, i64, i64, i64, i32, i32, P, P, P, P]),
    "lng_fold_readout": (C.c_int, [i64, i64, i32, i32, i32, P, P, P, P, P, P, P, i32, P]),
    "lng_route_attend": (C.c_int, [PT, P, i32, i64, i64, i64, P, P, P, i64, i64, i64, i32, f32, f32, P, P, P, i32, i32,
                                   P, P, P]),
    "lng_route_attend_rows": (C.c_int, [P, i32, i64, i64, i64, i32, f32, f32, P, P, P, i32, P]),
    "lng_sink_gqa": (C.c_int, [P, P, P, i32, i64, i32, i32, i64, i32, f32, P, P]),
    "lng_gemm": (C.c_int, [P, i32, i64, P, i32, i64, P, i32, i64, i64, i64, i64, P, i32, P]),
    "lng_rms_rows": (C.c_int, [P, i32, i64, i64, f32, P, P]),
    "lng_rms_norm_model": (C.c_int, [P, i32, i64, i64, P, i32, f32, P, i32, P]),
    "lng_rms_norm": (C.c_int, [P, i32, i64, i64, P, f32, P, i32, P]),
    "lng_conv_finish": (C.c_int, [PR, P, i64, i64, P, P, P, P, P]),
    "lng_conv_window": (C.c_int, [PR, P, i64, P, P, P, P, P]),
    "lng_memory_workspace_bytes": (sz, [PT, PR, i64]),
    "lng_memory_forward": (C.c_int, [PT, PR, i64, i64, P, P, i32, P, i32, P, P, P, P, P, sz, P]),
    "lng_attend_rescale": (C.c_int, [P, P, P, P, i64, i32, i64, P]),
    "lng_attend_normalize": (C.c_int, [P, P, i64, i32, i64, P, i32, P]),
    "lng_attend_pack": (C.c_int, [P, P, P, P, i64, i32, i32, P, i32, P]),
    "lng_attend_unpack": (C.c_int, [P, i32, i64, i32, i32, P, i32, P]),
    "lng_attend_pack_rescale": (C.c_int, [P, P, i64, i32, i32, P, i32, P]),
    "lng_logits_topk": (C.c_int, [P, i64, i64, P, i32, i64, i32, P, P, P, P, sz, P]),
    "lng_logits_topk_scratch_bytes": (sz, [i64, i64, i64, i32]),
    "lng_logits_topk_static": (C.c_int, [P, i64, i64, P, i32, i64, i32, P, P, P, P]),
    "lng_drafter_create": (C.c_int, [C.POINTER(DrafterNumbers), C.POINTER(Array), i32, i32, C.POINTER(P)]),
    "lng_drafter_destroy": (None, [P]),
    "lng_drafter_reset": (C.c_int, [P]),
    "lng_drafter_length": (i64, [P]),
    "lng_drafter_truncate": (C.c_int, [P, i64]),
    "lng_drafter_committed_codes": (C.c_int, [P, P]),
    "lng_drafter_commit": (C.c_int, [P, P, i64, P]),
    "lng_drafter_draft": (C.c_int, [P, i64, P, i64, i32, i32, P, P, P, P]),
    "lng_drafter_trace": (C.c_int, [P, P, i64, P, i32, i64, P, P, P]),
    "lng_drafter_draft_batch": (C.c_int, [P, P, i64, i64, i64, P, P]),
    "lng_tree_workspace_bytes": (C.c_size_t, [PT, PR, i64, i64, i64]),
    "lng_tree_memory_block": (C.c_int, [PT, PR, i64, i64, i64, i64, i64, i64, P, P, P, P, P, P, P, P, P, P, P,
                                        C.c_size_t, P]),
    "lng_online_counts_mix": (C.c_int, [P, i64, i64, P, i32, i32, P, P, P, i64, i64, P, P, i64, f32, P, P]),
}

_LIB = None


def library(require_device: bool = True):
    """The loaded C library (raises if it is missing, or, with ``require_device``, if no B200 is usable)."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH.name} is not built: run __graft_entry__.build() "
                               f"(python lngram-decode_b200/csrc/build.py)")
        lib = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = lib
    if require_device:
        dev = torch.cuda.current_device() if torch.cuda.is_available() else None
        if dev not in _DEVICE_OK:
            if dev is None:
                raise RuntimeError("lngram_b200 needs a CUDA device (sm_100a); there is no CPU fallback")
            if not _LIB.lng_device_ok():
                raise RuntimeError("lngram_b200 needs a compute-capability 10.x (B200) device")
            _DEVICE_OK.add(dev)
    return _LIB


_DEVICE_OK: set = set()  # devices already checked (the check queries device properties)


def check(status: int, what: str = "") -> None:
    if status == OK:
        return
    msg = (_LIB.lng_last_error() or b"").decode(errors="replace") if _LIB is not None else ""
    text = f"{what}: {msg}" if what else msg
    if status in (ERR_ARGUMENT,):
        raise ValueError(text)
    raise RuntimeError(f"[lngram_b200 status {status}] {text}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)
_cur_device = getattr(torch._C, "_cuda_getDevice", None)


def on_device(device):
    """``torch.cuda.device(device)`` unless ``device`` is current already (then a no-op context): the
    guard's own device lookups cost microseconds of host time on every library call."""
    idx = device.index if isinstance(device, torch.device) else device
    if idx is None or (_cur_device is not None and torch.cuda.is_initialized() and _cur_device() == idx):
        return contextlib.nullcontext()
    return torch.cuda.device(device)


def stream_ptr(stream: torch.cuda.Stream | None = None) -> int:
    """The cudaStream_t (as an int) of ``stream``, or of the current device's current stream: read
    straight from torch's C layer when it offers the call (a Stream object per call costs ~10 us of
    host time, which the short decode / tree steps would otherwise spend once per launch)."""
    if stream is not None:
        return stream.cuda_stream
    if _raw_stream is not None and _cur_device is not None and torch.cuda.is_initialized():
        return int(_raw_stream(_cur_device()))
    return torch.cuda.current_stream().cuda_stream


def device_error(clear: bool = True) -> int:
    return int(library().lng_device_error(1 if clear else 0))
