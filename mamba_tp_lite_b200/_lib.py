"""ctypes binding of libmtp.so (the C ABI in include/mtp.h).

The library is the only compute path: if it is missing or a call fails, an
exception is raised -- there is no CPU or eager-PyTorch fallback.
"""
from __future__ import annotations

import ctypes as C
import os

import torch

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libmtp.so")

MTP_OK, MTP_ERR_ARG, MTP_ERR_CUDA, MTP_ERR_TIMEOUT, MTP_ERR_UNSUPPORTED = 0, 1, 2, 3, 4
F32, BF16, F16 = 0, 1, 2
RED_FP32, RED_FP16, RED_INT8TOK, RED_INT8TENSOR, RED_INT8SUM, RED_INT8LEGACY = 0, 1, 2, 3, 4, 5
EPI_STORE, EPI_BIAS_SOFTPLUS, EPI_BIAS = 0, 1, 2
GEMM_AUTO, GEMM_TCGEN05, GEMM_SIMT, GEMM_GEMV = 0, 1, 2, 3

_vp, _i, _f, _d, _u64 = C.c_void_p, C.c_int, C.c_float, C.c_double, C.c_uint64

# name -> argtypes (all return int unless listed in _RESTYPES)
_SIGS = {
    "mtp_version": [],
    "mtp_last_error": [],
    "mtp_launch_count": [],
    "mtp_gemm": [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _vp, _i, _vp],
    "mtp_gemm_ex": [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _vp, _i, _i, _vp],
    "mtp_conv1d_silu": [_vp, _i, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp],
    "mtp_scan_prefill": [_vp, _i, _vp, _i, _i, _vp, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _vp, _vp,
                         _i, _i, _i, _i, _i, _i, _vp],
    "mtp_scan_prefill_fused": [_vp, _i, _vp, _i, _vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _vp,
                               _vp, _i, _i, _i, _i, _i, _i, _vp],
    "mtp_scan_prefill_xc": [_vp, _i, _vp, _i, _vp, _i, _i, _vp, _i, _vp, _vp, _vp, _vp, _vp, _i, _vp, _vp,
                            _i, _i, _i, _i, _i, _i, _vp],
    "mtp_exp2_fma": [_vp, _vp, _i, _vp],
    "mtp_scan_status": [C.POINTER(_i)],
    "mtp_step": [_vp, _i, _vp, _i, _vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i,
                 _i, _i, _i, _i, _i, _i, _vp],
    "mtp_embedding": [_vp, _i, _vp, _i, _i, _vp, _vp],
    "mtp_rmsnorm": [_vp, _i, _i, _vp, _i, _f, _vp, _i, _vp],
    "mtp_argmax_rows": [_vp, _i, _i, _i, _i, _vp, _vp],
    "mtp_quantize_rows_int8": [_vp, _i, _i, _i, _vp, _vp, _vp],
    "mtp_dequant_sum": [_vp, _i, _i, _i, _vp, _vp],
    "mtp_comm_create": [_i, _i, _i, _i, _i, _d, C.POINTER(_vp)],
    "mtp_comm_ipc_handle": [_vp, _vp],
    "mtp_comm_open_peers": [_vp, _vp],
    "mtp_comm_destroy": [_vp],
    "mtp_comm_status": [_vp, C.POINTER(_i)],
    "mtp_comm_reset_status": [_vp],
    "mtp_comm_reset_state": [_vp],
    "mtp_comm_set_max_ctas": [_vp, _i],
    "mtp_comm_set_sequence_parallel": [_vp, _i],
    "mtp_comm_set_trace": [_vp, _i],
    "mtp_comm_read_trace": [_vp, C.POINTER(_u64), _i, C.POINTER(_i)],
    "mtp_comm_sent_bytes": [_vp, _i, _i, _i, _i, C.POINTER(_d)],
    "mtp_reduce_xproj": [_vp, _i, _vp, _i, _i, _i, _vp, _i, _vp, _vp],
    "mtp_reduce_outproj": [_vp, _i, _vp, _i, _i, _vp, _vp, _vp, _f, _vp, _i, _vp],
    "mtp_allreduce": [_vp, _i, _i, _vp, _vp, _i, _i, _vp],
    "mtp_xproj_fused": [_vp, _i, _vp, _i, _vp, _i, _i, _i, _i, _i, _i, _vp, _vp, _i, _vp, _vp],
    "mtp_allreduce_noalloc": [_i, _vp, _vp, _i, _i, _vp],
    "mtp_vocab_shard": [_i, _i, _i, C.POINTER(_i), C.POINTER(_i)],
    "mtp_lm_head_vocab_parallel": [_vp, _vp, _i, _i, _i, _vp, _i, _i, _i, _vp, _i, _vp],
    "mtp_decode_plan_create": [_vp, _i, _vp, _vp, _i, _i, _i, _i, _i, _f, _i, _i, _vp, C.POINTER(_vp)],
    "mtp_decode_bind_cache": [_vp, _vp, _vp, _i, C.POINTER(_vp)],
    "mtp_decode_step": [_vp, _vp, _vp, _vp, _vp],
    "mtp_decode_status": [_vp, C.POINTER(_i)],
    "mtp_decode_reset": [_vp],
    "mtp_decode_set_trace": [_vp, _i],
    "mtp_decode_read_trace": [_vp, C.POINTER(_u64), _i, C.POINTER(_i)],
    "mtp_decode_cache_destroy": [_vp],
    "mtp_decode_plan_destroy": [_vp],
}
_RESTYPES = {"mtp_version": C.c_char_p, "mtp_last_error": C.c_char_p, "mtp_launch_count": _u64,
             "mtp_decode_cache_destroy": None, "mtp_decode_plan_destroy": None}


class DecodeLayer(C.Structure):
    """mtp_decode_layer of include/mtp.h."""
    _fields_ = [(n, C.c_void_p) for n in ("norm_w", "in_w", "in_b", "conv_w", "conv_b", "x_w", "dt_w", "dt_b",
                                           "A_log", "Dp", "out_w", "out_b")] + [("mode_x", C.c_int),
                                                                                ("mode_out", C.c_int)]

_lib = None


class MTPError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"libmtp error {code}: {msg}")
        self.code = code


def load(path: str = LIB_PATH) -> C.CDLL:
    """Loads the library (once) and declares every entry point of include/mtp.h."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(f"{path} is missing: build it with `python -m mamba_tp_lite_b200.build`")
    lib = C.CDLL(path)
    for name, args in _SIGS.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RESTYPES.get(name, _i)
    _lib = lib
    return lib


def exported_names() -> list[str]:
    return list(_SIGS)


def check(rc: int) -> None:
    if rc != MTP_OK:
        raise MTPError(rc, load().mtp_last_error().decode())


def call(name: str, *args) -> None:
    rc = getattr(load(), name)(*args)
    if _RESTYPES.get(name, _i) is _i:
        check(rc)


def launch_count() -> int:
    return int(load().mtp_launch_count())


def comm_sent_bytes(comm, mode: int, rows: int, cols: int, rdt: int) -> float:
    """Bytes one rank sends to its peers for a reduction call (0 at world size 1)."""
    out = C.c_double(0.0)
    call("mtp_comm_sent_bytes", comm, mode, rows, cols, rdt, C.byref(out))
    return out.value


def vocab_shard(V: int, ws: int, rank: int) -> tuple[int, int]:
    """(first column, columns) of ``rank``'s logits in the vocabulary-parallel lm_head."""
    c0, n = C.c_int(0), C.c_int(0)
    call("mtp_vocab_shard", V, ws, rank, C.byref(c0), C.byref(n))
    return c0.value, n.value


def stream_ptr(stream=None) -> int:
    s = torch.cuda.current_stream() if stream is None else stream
    return s.cuda_stream


def ptr(t) -> int | None:
    """Device pointer of a tensor, or None for a missing optional argument."""
    if t is None:
        return None
    return t.data_ptr()


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return F32
    if dt == torch.bfloat16:
        return BF16
    if dt == torch.float16:
        return F16
    raise TypeError(f"unsupported dtype {dt}")


def require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{what}: the mamba_tp_lite_b200 kernels need CUDA tensors (no CPU path)")
