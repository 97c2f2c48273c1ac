"""Device-resident BitNet b1.58 decode: the reference's cached single-token
forward and greedy generation, on the GPU.

Mirrors ``forward_with_cache`` (src/model/cached_forward.rs:131-149) and
``greedy_generate_with_cache`` (src/model/generate.rs:111-190): the same
argument meaning and ordering rules (position must equal the cache position;
an empty prompt or a token outside the vocabulary is a GgufParse error).  The
model is a dict of host arrays (``synth.bitnet_model`` builds a random one
with the 2B shapes); the weights are copied to the device once.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import numpy as np

from . import WillametteError
from ._abi import WlBitnetConfig, WlBitnetWeights, lib

_CFG_KEYS = ("n_layers", "n_embd", "n_heads", "n_kv_heads", "head_dim", "n_ff", "vocab", "n_rot",
             "max_seq", "eps", "freq_base")


def _check(rc: int):
    if rc != 0:
        L = lib()
        raise WillametteError(rc, L.wl_last_error().decode(errors="replace"),
                              L.wl_last_error_tensor_type())


def _fp(a: Optional[np.ndarray]):
    return a.ctypes.data_as(C.POINTER(C.c_float)) if a is not None else None


class BitNet:
    def __init__(self, model: dict, device: int = 0, exact: bool = False,
                 persistent: bool = False, tp=None, kv_f16: bool = False):
        """tp: a connected ``tp.TPGroup`` (one per rank) for the tensor-parallel
        engine; its symmetric region must hold ``BitNet.tp_sym_bytes(model)``.
        kv_f16: binary16 KV cache rows (benchmark config 2's layout) instead
        of the reference's per-token absmax int8 rows."""
        L = lib()
        if tp is None:
            _check(L.wl_init(device))
        c = model["config"]
        self.cfg = WlBitnetConfig(**{k: c[k] for k in _CFG_KEYS}, exact=int(exact),
                                  persistent=int(persistent), kv_f16=int(kv_f16))
        self.n_embd = c["n_embd"]
        ws = [np.ascontiguousarray(a, np.uint8) for a in model["w"]]
        self._keep = [ws, np.ascontiguousarray(model["w_scale"], np.float32),
                      np.ascontiguousarray(model["norms"], np.float32),
                      np.ascontiguousarray(model["output_norm"], np.float32),
                      np.ascontiguousarray(model["token_embd"], np.uint8)]
        ptrs = (C.c_void_p * len(ws))(*[a.ctypes.data for a in ws])
        w = WlBitnetWeights(ptrs, _fp(self._keep[1]), _fp(self._keep[2]), _fp(self._keep[3]),
                            self._keep[4].ctypes.data)
        self._h = C.c_void_p()
        if tp is None:
            _check(L.wl_bitnet_create(C.byref(self.cfg), C.byref(w), C.byref(self._h)))
        else:
            _check(L.wl_bitnet_create_tp(C.byref(self.cfg), C.byref(w), tp._g, C.byref(self._h)))
        self._tp = tp  # the engine's gathered vectors live in the group's block
        self._keep = None  # the library holds device copies

    @classmethod
    def from_gguf(cls, gguf_file, max_seq: int = 0, exact: bool = False,
                  persistent: bool = False, device: int = 0) -> "BitNet":
        """The engine straight from a parsed BitNet-family GGUF
        (``gguf.GgufFile``): ModelGraph::from_gguf, src/model/graph.rs:95-240.
        max_seq 0 = the file's context_length."""
        L = lib()
        _check(L.wl_init(device))
        self = cls.__new__(cls)
        cfg, _ = gguf_file.model_config()
        self.cfg = WlBitnetConfig(**cfg, exact=int(exact), persistent=int(persistent))
        self.n_embd = cfg["n_embd"]
        self._tp = None
        self._h = C.c_void_p()
        _check(L.wl_bitnet_create_from_gguf(gguf_file._g, max_seq, int(exact), int(persistent),
                                            C.byref(self._h)))
        return self

    @staticmethod
    def tp_sym_bytes(model: dict) -> int:
        """Symmetric-region bytes the tensor-parallel engine needs."""
        c = model["config"]
        cfg = WlBitnetConfig(**{k: c[k] for k in _CFG_KEYS}, exact=0, persistent=0)
        return int(lib().wl_bitnet_tp_sym_bytes(C.byref(cfg)))

    @property
    def persistent(self) -> bool:
        return bool(lib().wl_bitnet_uses_persistent_kernel(self._h))

    @property
    def position(self) -> int:
        return int(lib().wl_bitnet_position(self._h))

    def reset(self):
        _check(lib().wl_bitnet_reset(self._h))

    def forward(self, token: int, position: int) -> np.ndarray:
        out = np.zeros(self.n_embd, np.float32)
        _check(lib().wl_bitnet_forward(self._h, token, position, _fp(out)))
        return out

    def prefill(self, tokens):
        t = np.ascontiguousarray(tokens, np.uint32)
        _check(lib().wl_bitnet_prefill(self._h, t.ctypes.data_as(C.POINTER(C.c_uint32)), t.size))

    def decode(self, n_new: int, hiddens: bool = False, timed: bool = False):
        ids = np.zeros(max(n_new, 1), np.uint32)
        hs = np.zeros((max(n_new, 1), self.n_embd), np.float32) if hiddens else None
        ms = C.c_float(0.0)
        _check(lib().wl_bitnet_decode(self._h, n_new, ids.ctypes.data_as(C.POINTER(C.c_uint32)),
                                      _fp(hs), C.byref(ms) if timed else None))
        out = [ids[:n_new]]
        if hiddens:
            out.append(hs[:n_new])
        if timed:
            out.append(float(ms.value))
        return out[0] if len(out) == 1 else tuple(out)

    def generate(self, prompt, n_new: int, hiddens: bool = False):
        p = np.ascontiguousarray(prompt, np.uint32)
        ids = np.zeros(max(n_new, 1), np.uint32)
        hs = np.zeros((max(n_new, 1), self.n_embd), np.float32) if hiddens else None
        _check(lib().wl_bitnet_generate(self._h, p.ctypes.data_as(C.POINTER(C.c_uint32)), p.size,
                                        n_new, ids.ctypes.data_as(C.POINTER(C.c_uint32)),
                                        _fp(hs)))
        return (ids[:n_new], hs[:n_new]) if hiddens else ids[:n_new]

    def close(self):
        if self._h:
            lib().wl_bitnet_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
