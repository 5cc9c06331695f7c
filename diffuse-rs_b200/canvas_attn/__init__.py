"""Python host mirror of diffuse-rs's attention interface over libcanvas_attn.so.

The names and argument meanings follow the reference:
  AttnShape          src/model/attention.rs:10-27
  Rows               src/model/attention.rs:65-77
  attention()        src/model/attention.rs:106 (host fp32 in/out, in place)
  build_rope_cache   src/model/ops.rs:392-416
Everything computes on the GPU through the C ABI in include/canvas_attn.h;
there is no CPU fallback: if the shared library is missing, importing this
package raises.

Device-resident entry points (`attention_dev`, `attention_block_dev`) take
anything with a ``data_ptr()`` method (e.g. torch CUDA tensors) or raw ints.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("CANVAS_ATTN_LIB") or os.path.join(_HERE, "libcanvas_attn.so")

CA_OK = 0
CA_ERR_INVALID = -1
CA_ERR_UNSUPPORTED = -2
CA_ERR_CUDA = -3
CA_ERR_TIMEOUT = -4
CA_ERR_NOMEM = -5
CA_ERR_SCRATCH = -6
NOALLOC_SCRATCH_BYTES = 16 * 1024 * 1024

# Every symbol include/canvas_attn.h declares.
EXPORTED_SYMBOLS = (
    "ca_attention_host_f32",
    "ca_attention_dev",
    "ca_attention_block_dev",
    "ca_attention_block_dev_noalloc",
    "ca_build_rope_table",
    "ca_dequantize",
    "ca_linear",
    "ca_candidate_stats",
    "ca_tokens_to_unmask",
    "ca_ipc_export",
    "ca_ipc_import",
    "ca_ipc_close",
    "ca_device_status",
    "ca_selftest_wait_timeout",
    "ca_selftest_wait_timeout_status",
    "ca_status_string",
    "ca_version",
    "ca_round_bf16_host",
)


class CaError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {status_string(status)} ({status})")


class CaShape(ctypes.Structure):
    _fields_ = [("nq", ctypes.c_int64), ("nk", ctypes.c_int64), ("n_head", ctypes.c_int64),
                ("n_head_kv", ctypes.c_int64), ("head_dim", ctypes.c_int64),
                ("sliding_window", ctypes.c_int64), ("causal_prefix", ctypes.c_int64),
                ("scale", ctypes.c_float), ("softcap", ctypes.c_float)]


class CaRows(ctypes.Structure):
    _fields_ = [("pos", ctypes.c_void_p), ("seq", ctypes.c_void_p), ("n_seq", ctypes.c_size_t),
                ("prefix", ctypes.c_void_p), ("n_prefix", ctypes.c_size_t)]


class CaDevArgs(ctypes.Structure):
    _fields_ = [("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
                ("out", ctypes.c_void_p), ("out_f32", ctypes.c_int32),
                ("q_row_stride", ctypes.c_int64), ("kv_row_stride", ctypes.c_int64),
                ("out_row_stride", ctypes.c_int64), ("batch", ctypes.c_int32),
                ("sq", ctypes.c_int32), ("sk", ctypes.c_int32), ("cu_q", ctypes.c_void_p),
                ("cu_k", ctypes.c_void_p), ("max_sq", ctypes.c_int32),
                ("total_q", ctypes.c_int64), ("total_k", ctypes.c_int64),
                ("n_head", ctypes.c_int32), ("n_head_kv", ctypes.c_int32),
                ("head_dim", ctypes.c_int32), ("q_pos", ctypes.c_void_p),
                ("k_pos", ctypes.c_void_p), ("q_seq", ctypes.c_void_p),
                ("k_seq", ctypes.c_void_p), ("q_prefix", ctypes.c_void_p),
                ("sliding_window", ctypes.c_int64), ("causal_prefix", ctypes.c_int64),
                ("scale", ctypes.c_float), ("softcap", ctypes.c_float),
                ("precise", ctypes.c_int32), ("status", ctypes.c_void_p),
                ("peer_out", ctypes.c_void_p), ("n_peer_out", ctypes.c_int32),
                ("seq_prefix", ctypes.c_void_p), ("out_multicast", ctypes.c_void_p)]


class CaBlockArgs(ctypes.Structure):
    _fields_ = [("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
                ("batch", ctypes.c_int32), ("n_active", ctypes.c_int32),
                ("active_pos", ctypes.c_void_p), ("q_norm_w", ctypes.c_void_p),
                ("k_norm_w", ctypes.c_void_p), ("v_norm", ctypes.c_int32),
                ("rms_eps", ctypes.c_float), ("rope", ctypes.c_void_p),
                ("rope_len", ctypes.c_int32), ("rope_dim", ctypes.c_int32),
                ("cache_k", ctypes.c_void_p), ("cache_v", ctypes.c_void_p),
                ("n_total", ctypes.c_int32), ("q_work", ctypes.c_void_p),
                ("out", ctypes.c_void_p), ("out_f32", ctypes.c_int32),
                ("n_head", ctypes.c_int32), ("n_head_kv", ctypes.c_int32),
                ("head_dim", ctypes.c_int32), ("sliding_window", ctypes.c_int64),
                ("causal_prefix", ctypes.c_int64), ("scale", ctypes.c_float),
                ("softcap", ctypes.c_float), ("precise", ctypes.c_int32),
                ("status", ctypes.c_void_p), ("out_row_stride", ctypes.c_int64),
                ("peer_out", ctypes.c_void_p), ("n_peer_out", ctypes.c_int32),
                ("cu_active", ctypes.c_void_p), ("cu_total", ctypes.c_void_p),
                ("max_active", ctypes.c_int32), ("total_active", ctypes.c_int64),
                ("total_cache", ctypes.c_int64), ("seq_prefix", ctypes.c_void_p),
                ("out_multicast", ctypes.c_void_p)]


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"libcanvas_attn.so not built at {LIB_PATH}; run `make -C diffuse-rs_b200` "
            "(there is no CPU fallback)")
    L = ctypes.CDLL(LIB_PATH)
    L.ca_attention_host_f32.argtypes = [ctypes.c_void_p] * 4 + [
        ctypes.POINTER(CaShape), ctypes.POINTER(CaRows), ctypes.POINTER(CaRows)]
    L.ca_attention_host_f32.restype = ctypes.c_int
    L.ca_attention_dev.argtypes = [ctypes.POINTER(CaDevArgs), ctypes.c_void_p]
    L.ca_attention_dev.restype = ctypes.c_int
    L.ca_attention_block_dev.argtypes = [ctypes.POINTER(CaBlockArgs), ctypes.c_void_p]
    L.ca_attention_block_dev.restype = ctypes.c_int
    L.ca_attention_block_dev_noalloc.argtypes = [ctypes.POINTER(CaBlockArgs), ctypes.c_void_p]
    L.ca_attention_block_dev_noalloc.restype = ctypes.c_int
    L.ca_build_rope_table.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                      ctypes.c_float, ctypes.c_void_p]
    L.ca_build_rope_table.restype = ctypes.c_int
    L.ca_round_bf16_host.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64]
    L.ca_round_bf16_host.restype = ctypes.c_int
    L.ca_device_status.argtypes = [ctypes.c_void_p]
    L.ca_device_status.restype = ctypes.c_int
    L.ca_selftest_wait_timeout.argtypes = [ctypes.c_int64, ctypes.c_void_p]
    L.ca_selftest_wait_timeout.restype = ctypes.c_int
    L.ca_selftest_wait_timeout_status.argtypes = [ctypes.c_int64, ctypes.c_void_p,
                                                  ctypes.c_void_p]
    L.ca_selftest_wait_timeout_status.restype = ctypes.c_int
    L.ca_ipc_export.argtypes = [ctypes.c_void_p, ctypes.c_void_p,
                                ctypes.POINTER(ctypes.c_uint64)]
    L.ca_ipc_export.restype = ctypes.c_int
    L.ca_ipc_import.argtypes = [ctypes.c_void_p, ctypes.c_uint64,
                                ctypes.POINTER(ctypes.c_void_p)]
    L.ca_ipc_import.restype = ctypes.c_int
    L.ca_ipc_close.argtypes = [ctypes.c_void_p]
    L.ca_ipc_close.restype = ctypes.c_int
    L.ca_status_string.argtypes = [ctypes.c_int]
    L.ca_status_string.restype = ctypes.c_char_p
    L.ca_version.restype = ctypes.c_char_p
    return L


lib = _load()


def status_string(status: int) -> str:
    return lib.ca_status_string(int(status)).decode()


def version() -> str:
    return lib.ca_version().decode()


def _check(rc: int, what: str) -> None:
    if rc != CA_OK:
        raise CaError(rc, what)


@dataclass
class AttnShape:
    """AttnShape (src/model/attention.rs:10-27). None = the reference's None."""
    nq: int
    nk: int
    n_head: int
    n_head_kv: int
    head_dim: int
    sliding_window: Optional[int] = None
    causal_prefix: Optional[int] = None
    scale: float = 1.0
    softcap: float = 0.0  # extension: 0 = off

    def to_c(self) -> CaShape:
        return CaShape(self.nq, self.nk, self.n_head, self.n_head_kv, self.head_dim,
                       -1 if self.sliding_window is None else int(self.sliding_window),
                       -1 if self.causal_prefix is None else int(self.causal_prefix),
                       float(self.scale), float(self.softcap))


@dataclass
class Rows:
    """Rows (src/model/attention.rs:65-77): positions, optional seq ids and
    per-row causal prefixes (empty = the reference's &[] default)."""
    pos: Sequence[int]
    seq: Sequence[int] = field(default_factory=list)
    prefix: Sequence[int] = field(default_factory=list)

    def to_c(self):
        keep = []

        def arr(x):
            if x is None or len(x) == 0:
                return None, 0
            a = np.ascontiguousarray(np.asarray(x, dtype=np.int64))
            keep.append(a)
            return a.ctypes.data, len(a)

        p, _ = arr(self.pos)
        s, ns = arr(self.seq)
        f, nf = arr(self.prefix)
        return CaRows(p, s, ns, f, nf), keep


def attention(out: np.ndarray, q: np.ndarray, k: np.ndarray, v: np.ndarray,
              s: AttnShape, qr: Rows, kr: Rows) -> None:
    """attention(out, q, k, v, s, qr, kr) -- src/model/attention.rs:106.

    Host fp32 buffers; `out` ([nq * n_head * head_dim] fp32, C-contiguous) is
    written in place. Computes on the GPU (bf16 operands, fp32 accumulation).
    """
    for name, a in (("out", out), ("q", q), ("k", k), ("v", v)):
        if a.dtype != np.float32 or not a.flags.c_contiguous:
            raise ValueError(f"{name} must be a C-contiguous float32 array")
    if out.size != s.nq * s.n_head * s.head_dim:
        raise ValueError("out has the wrong length")
    if q.size != s.nq * s.n_head * s.head_dim or k.size != s.nk * s.n_head_kv * s.head_dim \
            or v.size != k.size:
        raise ValueError("q/k/v lengths disagree with the shape")
    if len(qr.pos) != s.nq or len(kr.pos) != s.nk:
        raise ValueError("row metadata lengths disagree with the shape")
    cs = s.to_c()
    cq, kq = qr.to_c()
    ck, kk = kr.to_c()
    rc = lib.ca_attention_host_f32(out.ctypes.data, q.ctypes.data, k.ctypes.data, v.ctypes.data,
                                   ctypes.byref(cs), ctypes.byref(cq), ctypes.byref(ck))
    _check(rc, "ca_attention_host_f32")


def _ptr(x) -> Optional[int]:
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return int(x.data_ptr())


def _peer_array(peer_out):
    """peer_out: device pointers (ints or tensors) of other GPUs' buffers ->
    (ctypes array or None, count)."""
    if not peer_out:
        return None, 0
    ptrs = [_ptr(x) for x in peer_out]
    return (ctypes.c_void_p * len(ptrs))(*ptrs), len(ptrs)


IPC_HANDLE_BYTES = 64


def ipc_export(x):
    """(handle bytes, byte offset) of device buffer x within its allocation,
    for another process's ipc_import."""
    h = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    off = ctypes.c_uint64(0)
    _check(lib.ca_ipc_export(_ptr(x), h, ctypes.byref(off)), "ca_ipc_export")
    return bytes(h.raw), int(off.value)


def ipc_import(handle: bytes, offset: int) -> int:
    """Maps another process's buffer (ipc_export's output) on the current
    device; returns its device address (an int)."""
    p = ctypes.c_void_p()
    _check(lib.ca_ipc_import(handle, int(offset), ctypes.byref(p)), "ca_ipc_import")
    return int(p.value)


def ipc_close(ptr: int) -> None:
    _check(lib.ca_ipc_close(int(ptr)), "ca_ipc_close")


def _stream(stream) -> Optional[int]:
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream
    return int(getattr(stream, "cuda_stream", stream))


def make_dev_args(q, k, v, out, *, batch, sq, sk, n_head, n_head_kv, head_dim,
                  out_f32=False, cu_q=None, cu_k=None, max_sq=0, total_q=0, total_k=0,
                  q_pos=None, k_pos=None, q_seq=None, k_seq=None, q_prefix=None,
                  sliding_window=None, causal_prefix=None, scale=1.0, softcap=0.0,
                  q_row_stride=0, kv_row_stride=0, out_row_stride=0,
                  precise=False, status=None, peer_out=None, seq_prefix=None,
                  out_multicast=None) -> CaDevArgs:
    peers, n_peers = _peer_array(peer_out)
    a = CaDevArgs(_ptr(q), _ptr(k), _ptr(v), _ptr(out), 1 if out_f32 else 0,
                     q_row_stride, kv_row_stride, out_row_stride, batch, sq, sk,
                     _ptr(cu_q), _ptr(cu_k), max_sq, total_q, total_k,
                     n_head, n_head_kv, head_dim, _ptr(q_pos), _ptr(k_pos), _ptr(q_seq),
                     _ptr(k_seq), _ptr(q_prefix),
                     -1 if sliding_window is None else int(sliding_window),
                     -1 if causal_prefix is None else int(causal_prefix),
                     float(scale), float(softcap), 1 if precise else 0, _ptr(status),
                     ctypes.cast(peers, ctypes.c_void_p) if peers is not None else None, n_peers,
                     _ptr(seq_prefix), out_multicast)
    a._keep = peers
    return a


def attention_dev(q, k, v, out, *, stream=None, **kw) -> None:
    """ca_attention_dev: device-resident bf16 attention (see make_dev_args)."""
    a = make_dev_args(q, k, v, out, **kw)
    _check(lib.ca_attention_dev(ctypes.byref(a), _stream(stream)), "ca_attention_dev")


def attention_dev_args(a: CaDevArgs, stream=None) -> None:
    _check(lib.ca_attention_dev(ctypes.byref(a), _stream(stream)), "ca_attention_dev")


def make_block_args(q, k, v, *, batch, n_active, active_pos, rope, rope_len, rope_dim,
                    cache_k, cache_v, n_total, q_work, out, n_head, n_head_kv, head_dim,
                    q_norm_w=None, k_norm_w=None, v_norm=False, rms_eps=1e-6,
                    out_f32=False, sliding_window=None, causal_prefix=None, scale=1.0,
                    softcap=0.0, precise=False, status=None, out_row_stride=0,
                    peer_out=None, cu_active=None, cu_total=None, max_active=0,
                    total_active=0, total_cache=0, seq_prefix=None,
                    out_multicast=None) -> CaBlockArgs:
    peers, n_peers = _peer_array(peer_out)
    a = CaBlockArgs(_ptr(q), _ptr(k), _ptr(v), batch, n_active, _ptr(active_pos),
                       _ptr(q_norm_w), _ptr(k_norm_w), 1 if v_norm else 0, float(rms_eps),
                       _ptr(rope), rope_len, rope_dim, _ptr(cache_k), _ptr(cache_v), n_total,
                       _ptr(q_work), _ptr(out), 1 if out_f32 else 0, n_head, n_head_kv,
                       head_dim, -1 if sliding_window is None else int(sliding_window),
                       -1 if causal_prefix is None else int(causal_prefix), float(scale),
                       float(softcap), 1 if precise else 0, _ptr(status), int(out_row_stride),
                       ctypes.cast(peers, ctypes.c_void_p) if peers is not None else None,
                       n_peers, _ptr(cu_active), _ptr(cu_total), int(max_active),
                       int(total_active), int(total_cache), _ptr(seq_prefix), out_multicast)
    a._keep = peers
    return a


def attention_block_dev(*args, stream=None, **kw) -> None:
    """ca_attention_block_dev: QK-norm -> RoPE -> cache store -> attention."""
    a = make_block_args(*args, **kw)
    _check(lib.ca_attention_block_dev(ctypes.byref(a), _stream(stream)),
           "ca_attention_block_dev")


def attention_block_dev_noalloc(*args, stream=None, **kw) -> None:
    """ca_attention_block_dev_noalloc: the fused block for callers that cannot
    allocate device memory; pass q_work=None (the library's fixed 16 MiB
    scratch holds the rotated queries). Overlapping calls race on that
    scratch; the first call on a device should precede any stream capture."""
    kw.setdefault("q_work", None)
    a = make_block_args(*args, **kw)
    _check(lib.ca_attention_block_dev_noalloc(ctypes.byref(a), _stream(stream)),
           "ca_attention_block_dev_noalloc")


def build_rope_cache(max_seq_len: int, rope_dim: int, theta: float,
                     freq_factors: Optional[np.ndarray] = None) -> np.ndarray:
    """build_rope_cache_ff (src/model/ops.rs:398-416): fp32 [len, rope_dim/2, 2]
    of (sin, cos)."""
    out = np.zeros(max_seq_len * (rope_dim // 2) * 2, dtype=np.float32)
    ff = None
    if freq_factors is not None:
        ff = np.ascontiguousarray(freq_factors, dtype=np.float32)
    rc = lib.ca_build_rope_table(out.ctypes.data, max_seq_len, rope_dim, float(theta),
                                 None if ff is None else ff.ctypes.data)
    _check(rc, "ca_build_rope_table")
    return out


def device_status(stream=None) -> int:
    """Synchronises `stream`, then reads and clears the device-wide error word
    (the word of launches that were given no status word of their own)."""
    return int(lib.ca_device_status(_stream(stream)))


def selftest_wait_timeout(limit_ns: int, stream=None) -> None:
    """Launches the failure-detection self-test: a wait on an mbarrier that
    nothing arrives on, bounded by `limit_ns`. Returns once launched; the
    expiry shows up in the next device_status() as CA_ERR_TIMEOUT."""
    _check(lib.ca_selftest_wait_timeout(int(limit_ns), _stream(stream)),
           "ca_selftest_wait_timeout")


def selftest_wait_timeout_status(limit_ns: int, status, stream=None) -> None:
    """The same self-test, reporting to the caller's device int32 `status`
    (a per-call status word as in make_dev_args(status=...)) instead of the
    device-wide word."""
    _check(lib.ca_selftest_wait_timeout_status(int(limit_ns), _ptr(status), _stream(stream)),
           "ca_selftest_wait_timeout_status")


def round_bf16_host(x):
    """ca_round_bf16_host: numpy float32 array -> numpy uint16 bf16 bit
    patterns, rounded on the host as the host-buffer entry point does."""
    import numpy as np
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    _check(lib.ca_round_bf16_host(x.ctypes.data, out.ctypes.data, x.size), "ca_round_bf16_host")
    return out
