"""project_willamette_b200 -- the BitLinear hot path of project-willamette on B200.

A Python mirror of the reference crate's call surface (Rust crate
``project_willamette`` v0.14.0) over the C ABI in ``include/willamette_b200.h``:

=======================================  ==========================================
this module                              reference
=======================================  ==========================================
``TensorView``                           ``gguf::tensor::TensorView`` (tensor.rs:21)
``GgmlType``                             ``gguf::types::GgmlType`` (types.rs:66-99)
``WillametteError``                      ``error::WillametteError`` (error.rs:9)
``bitlinear_i2s_matvec_f32(w, x, y)``    ``model::bitlinear`` (bitlinear.rs:67)
``linear_matvec_f32(w, x, y)``           ``model::linear`` (linear.rs:11)
``compute_logits(h, w, n_embd, vocab)``  ``model::lm_head`` (lm_head.rs:29)
``argmax(logits)``                       ``model::lm_head`` (lm_head.rs:161)
``lm_head_greedy(h, w, n_embd, vocab)``  compute_logits + argmax (sampler.rs:133)
=======================================  ==========================================

Every call runs the CUDA library; there is no CPU fallback.  Without the built
library the import fails; without a B200 the calls raise WillametteError.

Weights are uploaded to the GPU on first use and cached by (address, length,
type, shape).  The reference's weights are an immutable mmap for the life of
the process; to keep that contract this module holds a reference to every
uploaded array until ``release_weights()``.
"""
from __future__ import annotations

import ctypes as C
import enum
import os
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

from . import _abi
from ._abi import LIB_PATH, WLStatus

__all__ = [
    "GgmlType", "TensorView", "WillametteError", "bitlinear_i2s_matvec_f32",
    "bitlinear_i2s_matvec_f32_dbg", "bitlinear_i2s_gemm_f32", "linear_matvec_f32",
    "compute_logits", "argmax", "lm_head_greedy", "release_weights", "init", "LIB_PATH",
    "lib", "i2s_expected_byte_len", "q6k_expected_byte_len", "q8_0_expected_byte_len",
]


class GgmlType(enum.IntEnum):
    """Raw GGML type ids (src/gguf/types.rs:66-99) on the hot path."""
    F32 = 0
    F16 = 1
    Q4_0 = 2
    Q8_0 = 8
    Q4K = 12
    Q6K = 14
    BitNetI2S = 36


class WillametteError(Exception):
    """Error from the library; ``status`` names the WillametteError variant
    (UnsupportedTensorType / GgufParse / NotImplemented) or a device failure."""

    def __init__(self, status: int, message: str, raw_type: Optional[int] = None):
        self.status = WLStatus(status)
        self.raw_type = raw_type
        self.message = message
        super().__init__(f"{self.status.name}: {message}")


@dataclass
class TensorView:
    """Zero-copy weight view (src/gguf/tensor.rs:21-54).

    ``shape`` is GGUF order, innermost first: ``[in_dim, out_dim]``.  For
    I2_S, ``data`` is the packed-codes area and ``scale_data`` the 32-byte
    trailing block whose first 4 bytes are the f32 per-tensor scale."""
    name: str
    shape: Sequence[int]
    ggml_type: int
    data: np.ndarray
    scale_data: Optional[np.ndarray] = None

    def __post_init__(self):
        self.data = np.ascontiguousarray(np.frombuffer(self.data, np.uint8)
                                         if isinstance(self.data, (bytes, bytearray))
                                         else self.data).view(np.uint8).reshape(-1)
        if self.scale_data is not None:
            sd = self.scale_data
            if isinstance(sd, (bytes, bytearray)):
                sd = np.frombuffer(sd, np.uint8)
            self.scale_data = np.ascontiguousarray(sd).view(np.uint8).reshape(-1)

    def __getstate__(self):
        # the cached C struct (see _view) holds ctypes pointers: rebuilt on use
        state = dict(self.__dict__)
        state.pop("_cview", None)
        return state

    @staticmethod
    def i2s(name: str, in_dim: int, out_dim: int, packed, scale: float) -> "TensorView":
        block = np.zeros(32, np.uint8)
        block[:4] = np.frombuffer(np.float32(scale).tobytes(), np.uint8)
        return TensorView(name, [in_dim, out_dim], GgmlType.BitNetI2S, packed, block)


def lib() -> C.CDLL:
    return _abi.lib()


_keepalive: dict = {}


def _view(t: TensorView):
    """The C struct for ``t``; returns (struct, objects to keep alive).  Built
    once per TensorView and reused while its data, scale, shape, type and name
    are unchanged (a per-call rebuild cost ~10 us, a quarter of a small
    host-buffer matvec)."""
    c = t.__dict__.get("_cview")
    if (c is not None and c[0] is t.data and c[1] is t.scale_data and c[2] == tuple(t.shape)
            and c[3] == t.ggml_type and c[4] == t.name):
        if c[7] not in _keepalive:
            _keepalive[c[7]] = t.data
        return c[5], c[6]
    v, keep, key = _build_view(t)
    t.__dict__["_cview"] = (t.data, t.scale_data, tuple(t.shape), t.ggml_type, t.name, v, keep,
                            key)
    return v, keep


def _build_view(t: TensorView):
    shape = (C.c_uint64 * len(t.shape))(*[int(s) for s in t.shape])
    name = t.name.encode()
    v = _abi.WlTensorView()
    v.name = name
    v.shape = shape
    v.n_dims = len(t.shape)
    v.ggml_type = int(t.ggml_type)
    v.data = t.data.ctypes.data_as(C.POINTER(C.c_uint8))
    v.data_len = t.data.size
    if t.scale_data is not None:
        v.scale_data = t.scale_data.ctypes.data_as(C.POINTER(C.c_uint8))
        v.scale_len = t.scale_data.size
    key = (t.data.ctypes.data, t.data.size, int(t.ggml_type), tuple(int(s) for s in t.shape))
    _keepalive[key] = t.data
    return v, (shape, name), key


def _check(rc: int) -> None:
    if rc != WLStatus.OK:
        L = lib()
        msg = L.wl_last_error().decode(errors="replace")
        raw = int(L.wl_last_error_tensor_type()) if rc == WLStatus.UNSUPPORTED_TENSOR_TYPE else None
        raise WillametteError(rc, msg, raw)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _out(a: np.ndarray, name: str) -> np.ndarray:
    if not (isinstance(a, np.ndarray) and a.dtype == np.float32 and a.flags.c_contiguous):
        raise TypeError(f"{name} must be a C-contiguous float32 numpy array (written in place)")
    return a


_fp = C.POINTER(C.c_float)


def init(device: int = 0) -> None:
    _check(lib().wl_init(device))


def release_weights() -> None:
    _check(lib().wl_release_weights())
    _keepalive.clear()


_matvec_fn = None


def _matvec_entry():
    """wl_bitlinear_i2s_matvec_f32 declared with address-sized arguments, so
    a call passes the arrays' addresses as integers instead of building two
    ctypes pointer objects (a few microseconds of a small call)."""
    global _matvec_fn
    if _matvec_fn is None:
        L = lib()
        f = type(L.wl_bitlinear_i2s_matvec_f32)(("wl_bitlinear_i2s_matvec_f32", L))
        f.argtypes = [C.POINTER(_abi.WlTensorView), C.c_void_p, C.c_size_t, C.c_void_p,
                      C.c_size_t]
        f.restype = C.c_int
        _matvec_fn = f
    return _matvec_fn


def bitlinear_i2s_matvec_f32(weight: TensorView, input, output: np.ndarray,
                             kernel: Optional[int] = None) -> None:
    """output = i2_scale * (W_ternary . input) via int8 activations
    (bitlinear.rs:67 -> bitlinear_sse2.rs:313).  Writes ``output`` in place.

    ``kernel`` (an ``_abi.I2sKernel``) picks the kernel the reference's
    dispatch would run instead of the x86 default: SCALAR, SCALAR_LUT and
    SSE2_F32 are its f32-activation kernels, reproduced bit for bit; NEON
    raises WillametteError(NOT_IMPLEMENTED)."""
    x = _f32(input)
    y = _out(output, "output")
    v, keep = _view(weight)
    if kernel is None:
        _check(_matvec_entry()(C.byref(v), x.ctypes.data, x.size, y.ctypes.data, y.size))
    else:
        _check(lib().wl_bitlinear_i2s_matvec_f32_kernel(
            C.byref(v), x.ctypes.data_as(C.POINTER(C.c_float)), x.size,
            y.ctypes.data_as(C.POINTER(C.c_float)), y.size, int(kernel)))


def bitlinear_i2s_matvec_f32_dbg(weight: TensorView, input):
    """Returns (y f32[out], acc i32[out], act_scale, act_q i8[in])."""
    x = _f32(input)
    in_dim, out_dim = int(weight.shape[0]), int(weight.shape[1]) if len(weight.shape) > 1 else 0
    y = np.zeros(out_dim, np.float32)
    acc = np.zeros(out_dim, np.int32)
    q = np.zeros(max(in_dim, 1), np.int8)
    s = C.c_float(0.0)
    v, keep = _view(weight)
    _check(lib().wl_bitlinear_i2s_matvec_f32_dbg(
        C.byref(v), x.ctypes.data_as(_fp), x.size, y.ctypes.data_as(_fp), y.size,
        acc.ctypes.data_as(C.POINTER(C.c_int32)), C.byref(s),
        q.ctypes.data_as(C.POINTER(C.c_int8))))
    return y, acc, float(s.value), q[:in_dim]


def bitlinear_i2s_gemm_f32(weight: TensorView, X, with_acc: bool = False):
    """Y[m, out] for m tokens (per-token absmax quantisation, as the reference
    prefills one token at a time)."""
    X = _f32(X)
    m = X.shape[0]
    out_dim = int(weight.shape[1])
    Y = np.zeros((m, out_dim), np.float32)
    acc = np.zeros((m, out_dim), np.int32) if with_acc else None
    v, keep = _view(weight)
    _check(lib().wl_bitlinear_i2s_gemm_f32(
        C.byref(v), X.ctypes.data_as(_fp), m, Y.ctypes.data_as(_fp),
        acc.ctypes.data_as(C.POINTER(C.c_int32)) if acc is not None else None))
    return (Y, acc) if with_acc else Y


def linear_matvec_f32(weight: TensorView, input, output: np.ndarray) -> None:
    """linear.rs:11 -- I2_S, Q8_0 and Q6_K arms on the GPU."""
    x = _f32(input)
    y = _out(output, "output")
    v, keep = _view(weight)
    _check(lib().wl_linear_matvec_f32(C.byref(v), x.ctypes.data_as(_fp), x.size,
                                      y.ctypes.data_as(_fp), y.size))


def compute_logits(final_hidden, token_embd: TensorView, embedding_length: int,
                   vocab_size: int) -> np.ndarray:
    """lm_head.rs:29 -- full logit vector (bit-identical to the x86 row dot)."""
    h = _f32(final_hidden)
    logits = np.zeros(vocab_size, np.float32)
    v, keep = _view(token_embd)
    _check(lib().wl_compute_logits(h.ctypes.data_as(_fp), h.size, C.byref(v), embedding_length,
                                   vocab_size, logits.ctypes.data_as(_fp), logits.size))
    return logits


def argmax(logits) -> Optional[int]:
    """lm_head.rs:161 -- None for an empty slice."""
    l = _f32(logits)
    out = C.c_int64(0)
    _check(lib().wl_argmax(l.ctypes.data_as(_fp), l.size, C.byref(out)))
    return None if out.value < 0 else int(out.value)


def lm_head_greedy(hidden, token_embd: TensorView, embedding_length: int, vocab_size: int,
                   return_logits: bool = False):
    """Greedy next-token ids for a batch of hidden rows (compute_logits + argmax)."""
    H = _f32(hidden).reshape(-1, embedding_length) if embedding_length else _f32(hidden)
    batch = H.shape[0]
    ids = np.zeros(batch, np.uint32)
    logits = np.zeros((batch, vocab_size), np.float32) if return_logits else None
    v, keep = _view(token_embd)
    _check(lib().wl_lm_head_greedy(
        H.ctypes.data_as(_fp), batch, C.byref(v), embedding_length, vocab_size,
        ids.ctypes.data_as(C.POINTER(C.c_uint32)),
        logits.ctypes.data_as(_fp) if logits is not None else None))
    return (ids, logits) if return_logits else ids


# Layout helpers (src/gguf/tensor.rs:120-249).
def i2s_expected_byte_len(shape: Sequence[int]) -> int:
    n = int(np.prod(shape, dtype=np.int64))
    if n % 128:
        raise WillametteError(WLStatus.GGUF_PARSE, f"I2_S shape product {n} not a multiple of 128")
    return n // 4


def _block_len(shape, per, nbytes, name) -> int:
    if not shape:
        raise WillametteError(WLStatus.GGUF_PARSE, f"{name} tensor has no dimensions")
    row = int(shape[0])
    if row == 0:
        return 0
    if row % per:
        raise WillametteError(WLStatus.GGUF_PARSE, f"{name} row length {row} not a multiple of {per}")
    rows = int(np.prod([int(s) for s in shape[1:]], dtype=np.int64)) if len(shape) > 1 else 1
    return row // per * nbytes * rows


def q6k_expected_byte_len(shape: Sequence[int]) -> int:
    return _block_len(shape, 256, 210, "Q6_K")


def q8_0_expected_byte_len(shape: Sequence[int]) -> int:
    return _block_len(shape, 32, 34, "Q8_0")
