"""Batched greedy decode of independent sequences with the reference's
VanillaLlama forward and Q8_0 weights (the SmolLM shapes), on the GPU.

Per sequence this is ``greedy_generate_with_cache``
(src/model/generate.rs:111-190) over ``forward_with_cache``
(src/model/cached_forward.rs:206-504, VanillaLlama branches: no sub-norms,
silu(gate) * up, Norm RoPE) with Q8_0 linears (``q8_0_matvec_f32``,
src/model/linear.rs:171-224) and the tied Q8_0 lm-head; the engine runs all
sequences in lock step, one token each per step, every sequence with its own
KV cache and position.  Errors follow the reference's rules (an empty prompt,
a token outside the vocabulary or a full cache is a GgufParse error).  The
model is a dict of host arrays (``synth.llama_q8_model``).
"""
from __future__ import annotations

import ctypes as C
from typing import Sequence

import numpy as np

from ._abi import WlBitnetConfig, WlLlamaWeights, lib
from .bitnet import _CFG_KEYS, _check, _fp

_U32P = C.POINTER(C.c_uint32)


def _u32p(a: np.ndarray):
    return a.ctypes.data_as(_U32P)


def _prompts(prompts: Sequence) -> tuple[np.ndarray, np.ndarray]:
    lens = [len(p) for p in prompts]
    offsets = np.zeros(len(prompts) + 1, np.uint32)
    offsets[1:] = np.cumsum(lens)
    flat = np.concatenate([np.asarray(p, np.uint32).reshape(-1) for p in prompts]) \
        if sum(lens) else np.zeros(1, np.uint32)
    return np.ascontiguousarray(flat, np.uint32), offsets


class LlamaBatch:
    def __init__(self, model: dict, n_seqs: int, device: int = 0, exact: bool = False):
        L = lib()
        _check(L.wl_init(device))
        c = model["config"]
        if c.get("variant", 1) != 1 or c.get("linear_type", 8) != 8 or c.get("embd_type", 8) != 8:
            raise ValueError("LlamaBatch runs the VanillaLlama variant with Q8_0 weights")
        self.cfg = WlBitnetConfig(**{k: c[k] for k in _CFG_KEYS}, exact=int(exact), persistent=0)
        self.n_embd, self.n_seqs = c["n_embd"], n_seqs
        E, F, nl = c["n_embd"], c["n_ff"], c["n_layers"]
        per = np.asarray(model["norms"], np.float32).reshape(nl, 3 * E + F)
        ws = [np.ascontiguousarray(a, np.uint8) for a in model["w"]]
        keep = [ws, np.ascontiguousarray(per[:, :E]), np.ascontiguousarray(per[:, 2 * E:3 * E]),
                np.ascontiguousarray(model["output_norm"], np.float32),
                np.ascontiguousarray(model["token_embd"], np.uint8)]
        ptrs = (C.c_void_p * len(ws))(*[a.ctypes.data for a in ws])
        w = WlLlamaWeights(ptrs, _fp(keep[1]), _fp(keep[2]), _fp(keep[3]), keep[4].ctypes.data)
        self._h = C.c_void_p()
        _check(L.wl_llama_batch_create(C.byref(self.cfg), C.byref(w), n_seqs, C.byref(self._h)))

    @classmethod
    def from_gguf(cls, gguf_file, n_seqs: int, max_seq: int = 0, exact: bool = False,
                  device: int = 0) -> "LlamaBatch":
        """The engine straight from a parsed llama GGUF (``gguf.GgufFile``,
        Q8_0 linears and tied Q8_0 embedding).  max_seq 0 = context_length."""
        L = lib()
        _check(L.wl_init(device))
        self = cls.__new__(cls)
        cfg, _ = gguf_file.model_config()
        self.cfg = WlBitnetConfig(**cfg, exact=int(exact), persistent=0)
        self.n_embd, self.n_seqs = cfg["n_embd"], n_seqs
        self._h = C.c_void_p()
        _check(L.wl_llama_batch_create_from_gguf(gguf_file._g, n_seqs, max_seq, int(exact),
                                                 C.byref(self._h)))
        return self

    def position(self, seq: int) -> int:
        return int(lib().wl_llama_batch_position(self._h, seq))

    @property
    def attention_splits(self) -> int:
        return int(lib().wl_llama_batch_attention_splits(self._h))

    def set_tokens_per_cta(self, tg: int):
        """1, 4, 8 or 32 tokens per CTA of the linears; 0: chosen per launch."""
        _check(lib().wl_llama_batch_set_tokens_per_cta(self._h, tg))

    def reset(self):
        _check(lib().wl_llama_batch_reset(self._h))

    def prefill(self, prompts: Sequence):
        flat, off = _prompts(prompts)
        if len(off) != self.n_seqs + 1:
            raise ValueError(f"{len(off) - 1} prompts for {self.n_seqs} sequences")
        _check(lib().wl_llama_batch_prefill(self._h, _u32p(flat), _u32p(off)))

    def decode(self, n_new: int, hiddens: bool = False, timed: bool = False):
        """ids [n_new, n_seqs] (and hiddens [n_new, n_seqs, n_embd], device ms)."""
        S = self.n_seqs
        ids = np.zeros((max(n_new, 1), S), np.uint32)
        hs = np.zeros((max(n_new, 1), S, self.n_embd), np.float32) if hiddens else None
        ms = C.c_float(0.0)
        _check(lib().wl_llama_batch_decode(self._h, n_new, _u32p(ids), _fp(hs),
                                           C.byref(ms) if timed else None))
        out = [ids[:n_new]]
        if hiddens:
            out.append(hs[:n_new])
        if timed:
            out.append(float(ms.value))
        return out[0] if len(out) == 1 else tuple(out)

    def generate(self, prompts: Sequence, n_new: int, hiddens: bool = False):
        flat, off = _prompts(prompts)
        if len(off) != self.n_seqs + 1:
            raise ValueError(f"{len(off) - 1} prompts for {self.n_seqs} sequences")
        S = self.n_seqs
        ids = np.zeros((max(n_new, 1), S), np.uint32)
        hs = np.zeros((max(n_new, 1), S, self.n_embd), np.float32) if hiddens else None
        _check(lib().wl_llama_batch_generate(self._h, _u32p(flat), _u32p(off), n_new, _u32p(ids),
                                             _fp(hs)))
        return (ids[:n_new], hs[:n_new]) if hiddens else ids[:n_new]

    def close(self):
        if self._h:
            lib().wl_llama_batch_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
