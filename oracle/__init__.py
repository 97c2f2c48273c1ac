"""ctypes binding for the CPU oracle (test infrastructure only).

The oracle is a C restatement of project-willamette's x86 BitLinear /
lm-head path (see ``willamette_oracle.h``).  It is the parity checker for
the CUDA library and the timed CPU baseline.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline and
``--impl reference`` legs import this module; the product package never
does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libwillamette_oracle.so")

_u8p = C.POINTER(C.c_uint8)
_i8p = C.POINTER(C.c_int8)
_i32p = C.POINTER(C.c_int32)
_f32p = C.POINTER(C.c_float)
_sz = C.c_size_t
_u32 = C.c_uint32


def build() -> str:
    """Compile the oracle with its Makefile (no-op when up to date)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return LIB_PATH


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        L.or_f16_to_f32.argtypes = [C.c_uint16]
        L.or_f16_to_f32.restype = C.c_float
        L.or_f32_to_f16.argtypes = [C.c_float]
        L.or_f32_to_f16.restype = C.c_uint16
        L.or_ternary_from_code.argtypes = [C.c_uint8]
        L.or_ternary_from_code.restype = C.c_int8
        L.or_i2s_matvec_scalar.argtypes = [_u8p, _sz, C.c_float, _u32, _u32, _f32p, _f32p]
        L.or_quantize_absmax_i8.argtypes = [_f32p, _sz, _i8p]
        L.or_quantize_absmax_i8.restype = C.c_float
        L.or_i2s_matvec_sse2_i8.argtypes = [_u8p, _sz, C.c_float, _u32, _u32, _f32p, _f32p,
                                            _i32p, _f32p, _i8p]
        L.or_i2s_gemm_rows.argtypes = [_u8p, _sz, C.c_float, _u32, _u32, _u32, _f32p, _f32p,
                                       _i32p, _f32p, C.c_int]
        L.or_i2s_matvec_sse2_f32.argtypes = [_u8p, _sz, C.c_float, _u32, _u32, _f32p, _f32p]
        L.or_i2s_matvec_lut.argtypes = [_u8p, _sz, C.c_float, _u32, _u32, _f32p, _f32p]
        L.or_i2s_unpack_row.argtypes = [_u8p, _sz, _u32, _u32, _u32, _i8p]
        for name in ("or_q6k_dot_row_scalar", "or_q6k_dot_row_sse2", "or_q8_0_dot_row_scalar",
                     "or_q8_0_dot_row_avx2", "or_q8_0_dot_row_sse2"):
            getattr(L, name).argtypes = [_u8p, _sz, _f32p, _sz, _f32p]
        L.or_q6k_dequantize_row.argtypes = [_u8p, _sz, _f32p, _sz]
        L.or_q8_0_dequantize_row.argtypes = [_u8p, _sz, _f32p, _sz]
        L.or_q6k_quantize_row.argtypes = [_f32p, _sz, _u8p, _sz]
        L.or_q8_0_matvec.argtypes = [_u8p, _sz, _u32, _u32, _f32p, _f32p, C.c_int]
        L.or_compute_logits.argtypes = [_f32p, _u32, _u8p, _sz, _u32, _u32, _f32p, C.c_int]
        L.or_argmax.argtypes = [_f32p, _sz]
        L.or_argmax.restype = C.c_int64
        _lib = L
    return _lib


class OracleError(RuntimeError):
    """The reference would have returned Err(..) for these inputs."""


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t)


def _u8(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint8)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise OracleError(f"{what}: reference rejects these inputs (rc={rc})")


def f16_to_f32(bits: int) -> float:
    return float(lib().or_f16_to_f32(bits))


def f32_to_f16(value: float) -> int:
    return int(lib().or_f32_to_f16(value))


def ternary_from_code(code: int) -> int:
    return int(lib().or_ternary_from_code(code))


def quantize_absmax_i8(x) -> tuple[np.ndarray, float]:
    x = _f32(x)
    q = np.zeros(x.size, np.int8)
    s = lib().or_quantize_absmax_i8(_p(x, _f32p), x.size, _p(q, _i8p))
    return q, float(s)


def i2s_matvec_scalar(packed, scale: float, in_dim: int, out_dim: int, x) -> np.ndarray:
    packed, x = _u8(packed), _f32(x)
    y = np.zeros(out_dim, np.float32)
    _check(lib().or_i2s_matvec_scalar(_p(packed, _u8p), packed.size, scale, in_dim, out_dim,
                                      _p(x, _f32p), _p(y, _f32p)), "i2s_matvec_scalar")
    return y


def i2s_matvec_sse2_i8(packed, scale: float, in_dim: int, out_dim: int, x):
    """Returns (y f32[out_dim], acc i32[out_dim], act_scale, act_q i8[in_dim])."""
    packed, x = _u8(packed), _f32(x)
    y = np.zeros(out_dim, np.float32)
    acc = np.zeros(out_dim, np.int32)
    q = np.zeros(in_dim, np.int8)
    s = C.c_float(0.0)
    _check(lib().or_i2s_matvec_sse2_i8(_p(packed, _u8p), packed.size, scale, in_dim, out_dim,
                                       _p(x, _f32p), _p(y, _f32p), _p(acc, _i32p), C.byref(s),
                                       _p(q, _i8p)), "i2s_matvec_sse2_i8")
    return y, acc, float(s.value), q


def i2s_gemm_rows(packed, scale: float, in_dim: int, out_dim: int, X, n_threads: int = 1):
    """Per-token SSE2-i8 matvec over the rows of X (how the reference prefills)."""
    packed, X = _u8(packed), _f32(X)
    m = X.shape[0]
    Y = np.zeros((m, out_dim), np.float32)
    acc = np.zeros((m, out_dim), np.int32)
    sc = np.zeros(m, np.float32)
    _check(lib().or_i2s_gemm_rows(_p(packed, _u8p), packed.size, scale, in_dim, out_dim, m,
                                  _p(X, _f32p), _p(Y, _f32p), _p(acc, _i32p), _p(sc, _f32p),
                                  n_threads), "i2s_gemm_rows")
    return Y, acc, sc


def i2s_matvec_sse2_f32(packed, scale: float, in_dim: int, out_dim: int, x) -> np.ndarray:
    packed, x = _u8(packed), _f32(x)
    y = np.zeros(out_dim, np.float32)
    _check(lib().or_i2s_matvec_sse2_f32(_p(packed, _u8p), packed.size, scale, in_dim, out_dim,
                                        _p(x, _f32p), _p(y, _f32p)), "i2s_matvec_sse2_f32")
    return y


def i2s_matvec_lut(packed, scale: float, in_dim: int, out_dim: int, x) -> np.ndarray:
    packed, x = _u8(packed), _f32(x)
    y = np.zeros(out_dim, np.float32)
    _check(lib().or_i2s_matvec_lut(_p(packed, _u8p), packed.size, scale, in_dim, out_dim,
                                   _p(x, _f32p), _p(y, _f32p)), "i2s_matvec_lut")
    return y


def i2s_unpack_row(packed, in_dim: int, out_dim: int, row: int) -> np.ndarray:
    packed = _u8(packed)
    out = np.zeros(in_dim, np.int8)
    _check(lib().or_i2s_unpack_row(_p(packed, _u8p), packed.size, in_dim, out_dim, row,
                                   _p(out, _i8p)), "i2s_unpack_row")
    return out


def _row_fn(name: str, row, x) -> float:
    row, x = _u8(row), _f32(x)
    out = C.c_float(0.0)
    _check(getattr(lib(), name)(_p(row, _u8p), row.size, _p(x, _f32p), x.size, C.byref(out)), name)
    return float(out.value)


def q6k_dot_row_scalar(row, x) -> float:
    return _row_fn("or_q6k_dot_row_scalar", row, x)


def q6k_dot_row_sse2(row, x) -> float:
    return _row_fn("or_q6k_dot_row_sse2", row, x)


def q8_0_dot_row_scalar(row, x) -> float:
    return _row_fn("or_q8_0_dot_row_scalar", row, x)


def q8_0_dot_row_avx2(row, x) -> float:
    return _row_fn("or_q8_0_dot_row_avx2", row, x)


def q8_0_dot_row_sse2(row, x) -> float:
    return _row_fn("or_q8_0_dot_row_sse2", row, x)


def q6k_dequantize_row(row, n: int) -> np.ndarray:
    row = _u8(row)
    out = np.zeros(n, np.float32)
    _check(lib().or_q6k_dequantize_row(_p(row, _u8p), row.size, _p(out, _f32p), n),
           "q6k_dequantize_row")
    return out


def q8_0_dequantize_row(row, n: int) -> np.ndarray:
    row = _u8(row)
    out = np.zeros(n, np.float32)
    _check(lib().or_q8_0_dequantize_row(_p(row, _u8p), row.size, _p(out, _f32p), n),
           "q8_0_dequantize_row")
    return out


def q6k_quantize_row(x) -> np.ndarray:
    x = _f32(x)
    out = np.zeros(x.size // 256 * 210, np.uint8)
    _check(lib().or_q6k_quantize_row(_p(x, _f32p), x.size, _p(out, _u8p), out.size),
           "q6k_quantize_row")
    return out


def q8_0_matvec(w, in_dim: int, out_dim: int, x, n_threads: int = 0) -> np.ndarray:
    w, x = _u8(w), _f32(x)
    y = np.zeros(out_dim, np.float32)
    _check(lib().or_q8_0_matvec(_p(w, _u8p), w.size, in_dim, out_dim, _p(x, _f32p),
                                _p(y, _f32p), n_threads), "q8_0_matvec")
    return y


def compute_logits(hidden, w, ggml_type: int, n_embd: int, vocab: int,
                   n_threads: int = 0) -> np.ndarray:
    hidden, w = _f32(hidden), _u8(w)
    logits = np.zeros(vocab, np.float32)
    _check(lib().or_compute_logits(_p(hidden, _f32p), n_embd, _p(w, _u8p), w.size, ggml_type,
                                   vocab, _p(logits, _f32p), n_threads), "compute_logits")
    return logits


def argmax(logits):
    logits = _f32(logits)
    r = lib().or_argmax(_p(logits, _f32p), logits.size)
    return None if r < 0 else int(r)


# ------------------------------------------------------------ decode step
class OrBitnetConfig(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("n_layers", "n_embd", "n_heads", "n_kv_heads",
                                          "head_dim", "n_ff", "vocab", "n_rot", "max_seq")] + \
               [("eps", C.c_float), ("freq_base", C.c_float), ("variant", _u32),
                ("linear_type", _u32), ("embd_type", _u32), ("kv_f16", _u32)]


class OrBitnetWeights(C.Structure):
    _fields_ = [("w", C.POINTER(_u8p)), ("w_scale", _f32p), ("norms", _f32p),
                ("output_norm", _f32p), ("token_embd", _u8p)]


class OrKvCache(C.Structure):
    _fields_ = [("k_q", _i8p), ("v_q", _i8p), ("k_s", _f32p), ("v_s", _f32p), ("pos", _u32)]


def _bitnet_prototypes(L):
    L.or_bitnet_forward.argtypes = [C.POINTER(OrBitnetConfig), C.POINTER(OrBitnetWeights),
                                    C.POINTER(OrKvCache), _u32, _u32, _f32p, C.c_int]
    L.or_bitnet_generate.argtypes = [C.POINTER(OrBitnetConfig), C.POINTER(OrBitnetWeights),
                                     C.POINTER(OrKvCache), C.POINTER(_u32), _u32, _u32,
                                     C.POINTER(_u32), _f32p, C.c_int]
    L.or_rms_norm.argtypes = [_f32p, _f32p, C.c_float, _f32p, _u32]
    L.or_rope_neox.argtypes = [_f32p, _u32, _u32, C.c_float]
    L.or_rope_norm.argtypes = [_f32p, _u32, _u32, C.c_float]
    L.or_silu_inplace.argtypes = [_f32p, _u32]
    L.or_softmax_inplace.argtypes = [_f32p, _u32]
    L.or_kv_quantise.argtypes = [_f32p, _u32, _i8p, _f32p]
    for n in ("or_rms_norm", "or_rope_neox", "or_rope_norm", "or_silu_inplace",
              "or_softmax_inplace", "or_kv_quantise"):
        getattr(L, n).restype = None


def _blib():
    L = lib()
    if not getattr(L, "_bitnet_ready", False):
        _bitnet_prototypes(L)
        L._bitnet_ready = True
    return L


def rms_norm(x, w, eps: float) -> np.ndarray:
    x, w = _f32(x), _f32(w)
    out = np.zeros(x.size, np.float32)
    _blib().or_rms_norm(_p(x, _f32p), _p(w, _f32p), eps, _p(out, _f32p), x.size)
    return out


def rope_neox(x, n_rot: int, position: int, freq_base: float) -> np.ndarray:
    x = _f32(x).copy()
    _blib().or_rope_neox(_p(x, _f32p), n_rot, position, freq_base)
    return x


def rope_norm(x, n_rot: int, position: int, freq_base: float) -> np.ndarray:
    x = _f32(x).copy()
    _blib().or_rope_norm(_p(x, _f32p), n_rot, position, freq_base)
    return x


def silu(x) -> np.ndarray:
    x = _f32(x).copy()
    _blib().or_silu_inplace(_p(x, _f32p), x.size)
    return x


def softmax(x) -> np.ndarray:
    x = _f32(x).copy()
    _blib().or_softmax_inplace(_p(x, _f32p), x.size)
    return x


def kv_quantise(x) -> tuple[np.ndarray, float]:
    x = _f32(x)
    q = np.zeros(x.size, np.int8)
    s = C.c_float(0.0)
    _blib().or_kv_quantise(_p(x, _f32p), x.size, _p(q, _i8p), C.byref(s))
    return q, float(s.value)


class BitnetOracle:
    """The reference's cached forward + greedy generation on a model dict
    (see project_willamette_b200.synth.bitnet_model)."""

    def __init__(self, model: dict, kv_f16: bool = False):
        """kv_f16: binary16 KV rows instead of the reference's int8 ones (the
        checker of the library's kv_f16 option; not a reference layout)."""
        self.m = model
        c = model["config"]
        self.cfg = OrBitnetConfig(**{k: c[k] for k in (
            "n_layers", "n_embd", "n_heads", "n_kv_heads", "head_dim", "n_ff", "vocab", "n_rot",
            "max_seq", "eps", "freq_base")}, variant=c.get("variant", 0),
            linear_type=c.get("linear_type", 0), embd_type=c.get("embd_type", 14),
            kv_f16=int(kv_f16))
        ws = model["w"]
        self._wp = (_u8p * len(ws))(*[_p(a, _u8p) for a in ws])
        self.weights = OrBitnetWeights(self._wp, _p(model["w_scale"], _f32p),
                                       _p(model["norms"], _f32p), _p(model["output_norm"], _f32p),
                                       _p(model["token_embd"], _u8p))
        kv = c["n_kv_heads"] * c["head_dim"]
        n = c["n_layers"] * c["max_seq"]
        esz = 2 if kv_f16 else 1
        self.kq = np.zeros(n * kv * esz, np.int8)
        self.vq = np.zeros(n * kv * esz, np.int8)
        self.ks = np.zeros(n, np.float32)
        self.vs = np.zeros(n, np.float32)
        self.kv = OrKvCache(_p(self.kq, _i8p), _p(self.vq, _i8p), _p(self.ks, _f32p),
                            _p(self.vs, _f32p), 0)

    def reset(self):
        self.kv.pos = 0

    def forward(self, token: int, position: int, n_threads: int = 0) -> np.ndarray:
        out = np.zeros(self.cfg.n_embd, np.float32)
        _check(_blib().or_bitnet_forward(C.byref(self.cfg), C.byref(self.weights),
                                         C.byref(self.kv), token, position, _p(out, _f32p),
                                         n_threads or os.cpu_count()), "bitnet_forward")
        return out

    def generate(self, prompt, n_new: int, n_threads: int = 0, hiddens: bool = False):
        self.reset()
        pr = np.ascontiguousarray(prompt, dtype=np.uint32)
        ids = np.zeros(max(n_new, 1), np.uint32)
        hs = np.zeros((max(n_new, 1), self.cfg.n_embd), np.float32) if hiddens else None
        _check(_blib().or_bitnet_generate(
            C.byref(self.cfg), C.byref(self.weights), C.byref(self.kv),
            pr.ctypes.data_as(C.POINTER(_u32)), pr.size, n_new,
            ids.ctypes.data_as(C.POINTER(_u32)), _p(hs, _f32p) if hs is not None else None,
            n_threads or os.cpu_count()), "bitnet_generate")
        return (ids[:n_new], hs[:n_new]) if hiddens else ids[:n_new]
