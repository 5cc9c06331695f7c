"""Projections around attention on the GPU: QKV + bias (src/model/forward.rs:
275-294) and wo + residual (:345-350), over the reference's quantised
weights (GGUF Q4_K / Q6_K / Q4_0 / Q8_0 / F16, src/kernels.rs).

Weights are dequantised once into bf16 in HBM (dequantize); every
projection is then one bf16 GEMM with fp32 accumulation and the bias and
residual in its epilogue (linear). embed() gathers and dequantises token
embedding rows (embed_tokens, forward.rs:175-246)."""
from __future__ import annotations

import ctypes

from . import CaError, _ptr, _stream, lib

F16, Q4_0, Q8_0, Q4_K, Q6_K = 1, 2, 8, 12, 14
_UNIT = {F16: (8, 2), Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}


class CaLinearArgs(ctypes.Structure):
    _fields_ = [("act", ctypes.c_void_p), ("act_stride", ctypes.c_int64),
                ("w", ctypes.c_void_p), ("bias", ctypes.c_void_p),
                ("residual", ctypes.c_void_p), ("out", ctypes.c_void_p),
                ("out_f32", ctypes.c_int32), ("n", ctypes.c_int64), ("rows", ctypes.c_int64),
                ("cols", ctypes.c_int64)]


lib.ca_dequantize.argtypes = [ctypes.c_int32, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                              ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int32,
                              ctypes.c_int64, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p]
lib.ca_dequantize.restype = ctypes.c_int
lib.ca_linear.argtypes = [ctypes.POINTER(CaLinearArgs), ctypes.c_void_p]
lib.ca_linear.restype = ctypes.c_int


def row_bytes(qtype: int, cols: int) -> int:
    unit, nbytes = _UNIT[qtype]
    return cols // unit * nbytes


def dequantize(qtype, src, rows, cols, dst, *, row_ids=None, n_out=None, dst_f32=False,
               dst_stride=0, scale=1.0, status=None, stream=None) -> None:
    """ca_dequantize on device buffers (src: uint8 bytes of `rows` rows)."""
    n = rows if n_out is None else n_out
    rc = lib.ca_dequantize(int(qtype), _ptr(src), int(rows), int(cols), _ptr(row_ids), int(n),
                           _ptr(dst), 1 if dst_f32 else 0, int(dst_stride), float(scale),
                           _ptr(status), _stream(stream))
    if rc != 0:
        raise CaError(rc, "ca_dequantize")


def embed(qtype, table, n_vocab, cols, tokens, dst, *, dst_f32=True, scale=1.0, status=None,
          stream=None) -> None:
    """embed_tokens: rows `tokens` (device int32) of the quantised table."""
    dequantize(qtype, table, n_vocab, cols, dst, row_ids=tokens, n_out=int(tokens.numel()),
               dst_f32=dst_f32, scale=scale, status=status, stream=stream)


def linear(act, w, out, *, n, rows, cols, bias=None, residual=None, act_stride=0,
           stream=None) -> None:
    """out = act . w^T (+ bias) (+ residual): bf16 act [n, cols] and w
    [rows, cols]; out bf16 or fp32 [n, rows] (fp32 when out is float32)."""
    import torch
    a = CaLinearArgs(_ptr(act), int(act_stride), _ptr(w), _ptr(bias), _ptr(residual), _ptr(out),
                     1 if out.dtype == torch.float32 else 0, int(n), int(rows), int(cols))
    rc = lib.ca_linear(ctypes.byref(a), _stream(stream))
    if rc != 0:
        raise CaError(rc, "ca_linear")
