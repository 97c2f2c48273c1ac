"""GGUF files: a writer for synthetic models and a reader over the library's
parser (``wl_gguf_*``, the reference's ``GgufFile::parse``,
src/gguf/reader.rs:120-415).

The writer produces GGUF v3 with the reference's layout conventions: tensor
data aligned to ``general.alignment`` (default 32), I2_S tensors followed by
their 32-byte trailing block (little-endian f32 scale + 28 zero bytes,
src/gguf/reader.rs:360-395).  ``bitnet_gguf`` / ``llama_gguf`` turn the
``synth`` model dicts into files the engines load with
``BitNet.from_gguf`` / ``LlamaBatch.from_gguf``.
"""
from __future__ import annotations

import ctypes as C
import struct
from typing import Iterable, Sequence

import numpy as np

from ._abi import WlBitnetConfig, WlTensorView, lib
from .bitnet import _check

# metadata value types (src/gguf/types.rs:221-236)
U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
_PACK = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f",
         BOOL: "<B", U64: "<Q", I64: "<q", F64: "<d"}
GGML_F32, GGML_F16, GGML_Q8_0, GGML_Q6_K, GGML_I2_S = 0, 1, 8, 14, 36


def _s(x: str) -> bytes:
    b = x.encode()
    return struct.pack("<Q", len(b)) + b


def _value(t: int, v) -> bytes:
    if t == STR:
        return _s(v)
    if t == ARR:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(_value(et, x) for x in items)
    return struct.pack(_PACK[t], v)


def _typed(v):
    if isinstance(v, tuple) and len(v) == 2 and isinstance(v[0], int):
        return v
    if isinstance(v, bool):
        return BOOL, int(v)
    if isinstance(v, int):
        return (U32, v) if 0 <= v < 2 ** 32 else (U64, v)
    if isinstance(v, float):
        return F32, v
    if isinstance(v, str):
        return STR, v
    if isinstance(v, (list, tuple)) and all(isinstance(x, str) for x in v):
        return ARR, (STR, list(v))
    raise TypeError(f"cannot infer a GGUF type for {v!r}")


def write_gguf(metadata: dict, tensors: Sequence[tuple], alignment: int = 32,
               version: int = 3) -> bytes:
    """metadata: key -> value (int / float / str / bool / list of str, or an
    explicit (type, value)); tensors: (name, shape (GGUF order), ggml_type,
    data bytes[, i2s_scale]) in file order."""
    meta = dict(metadata)
    if alignment != 32:
        meta.setdefault("general.alignment", (U32, alignment))
    head = struct.pack("<IIQQ", 0x46554747, version, len(tensors), len(meta))
    for k, v in meta.items():
        t, val = _typed(v)
        head += _s(k) + struct.pack("<I", t) + _value(t, val)
    blobs, off = [], 0
    infos = b""
    for item in tensors:
        name, shape, gtype, data = item[:4]
        data = bytes(np.ascontiguousarray(data).view(np.uint8).reshape(-1)) \
            if isinstance(data, np.ndarray) else bytes(data)
        if gtype == GGML_I2_S:
            scale = item[4]
            data = data + struct.pack("<f", float(scale)) + bytes(28)
        infos += _s(name) + struct.pack("<I", len(shape)) + \
            b"".join(struct.pack("<Q", d) for d in shape) + struct.pack("<IQ", gtype, off)
        blobs.append((off, data))
        off = (off + len(data) + alignment - 1) // alignment * alignment
    out = bytearray(head + infos)
    out += bytes((-len(out)) % alignment)
    base = len(out)
    out += bytes(off)
    for o, d in blobs:
        out[base + o: base + o + len(d)] = d
    return bytes(out)


def bitnet_gguf(model: dict, arch: str = "bitnet-b1.58") -> bytes:
    """A BitNet-family file from a ``synth.bitnet_model`` dict (Q6_K tied
    embedding: the reference's embedding-q6-k artifact layout)."""
    c = model["config"]
    E, F, nl = c["n_embd"], c["n_ff"], c["n_layers"]
    KV = c["n_kv_heads"] * c["head_dim"]
    p = arch + "."
    meta = {"general.architecture": arch, p + "block_count": nl, p + "embedding_length": E,
            p + "feed_forward_length": F, p + "context_length": c["max_seq"],
            p + "attention.head_count": c["n_heads"], p + "attention.head_count_kv": c["n_kv_heads"],
            p + "attention.layer_norm_rms_epsilon": float(c["eps"]),
            p + "rope.dimension_count": c["n_rot"], p + "rope.freq_base": float(c["freq_base"]),
            p + "vocab_size": c["vocab"]}
    tensors = [("token_embd.weight", (E, c["vocab"]), GGML_Q6_K, model["token_embd"]),
               ("output_norm.weight", (E,), GGML_F32, np.asarray(model["output_norm"], np.float32))]
    shapes = [(E, E), (E, KV), (E, KV), (E, E), (E, F), (E, F), (F, E)]
    roles = ["attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"]
    norms = np.asarray(model["norms"], np.float32).reshape(nl, 3 * E + F)
    for l in range(nl):
        b = f"blk.{l}."
        n = norms[l]
        tensors += [(b + "attn_norm.weight", (E,), GGML_F32, n[:E]),
                    (b + "attn_sub_norm.weight", (E,), GGML_F32, n[E:2 * E]),
                    (b + "ffn_norm.weight", (E,), GGML_F32, n[2 * E:3 * E]),
                    (b + "ffn_sub_norm.weight", (F,), GGML_F32, n[3 * E:])]
        for k in range(7):
            tensors.append((b + roles[k] + ".weight", shapes[k], GGML_I2_S, model["w"][l * 7 + k],
                            float(model["w_scale"][l * 7 + k])))
    return write_gguf(meta, tensors)


def llama_gguf(model: dict) -> bytes:
    """A llama file from a ``synth.llama_q8_model`` dict (Q8_0 linears, tied
    Q8_0 embedding; the vocabulary size is the tokenizer's token count)."""
    c = model["config"]
    E, F, nl = c["n_embd"], c["n_ff"], c["n_layers"]
    KV = c["n_kv_heads"] * c["head_dim"]
    meta = {"general.architecture": "llama", "llama.block_count": nl, "llama.embedding_length": E,
            "llama.feed_forward_length": F, "llama.context_length": c["max_seq"],
            "llama.attention.head_count": c["n_heads"],
            "llama.attention.head_count_kv": c["n_kv_heads"],
            "llama.attention.layer_norm_rms_epsilon": float(c["eps"]),
            "llama.rope.freq_base": float(c["freq_base"]),
            "tokenizer.ggml.tokens": [f"<t{i}>" for i in range(c["vocab"])]}
    tensors = [("token_embd.weight", (E, c["vocab"]), GGML_Q8_0, model["token_embd"]),
               ("output_norm.weight", (E,), GGML_F32, np.asarray(model["output_norm"], np.float32))]
    shapes = [(E, E), (E, KV), (E, KV), (E, E), (E, F), (E, F), (F, E)]
    roles = ["attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"]
    norms = np.asarray(model["norms"], np.float32).reshape(nl, 3 * E + F)
    for l in range(nl):
        b = f"blk.{l}."
        tensors += [(b + "attn_norm.weight", (E,), GGML_F32, norms[l, :E]),
                    (b + "ffn_norm.weight", (E,), GGML_F32, norms[l, 2 * E:3 * E])]
        for k in range(7):
            tensors.append((b + roles[k] + ".weight", shapes[k], GGML_Q8_0, model["w"][l * 7 + k]))
    return write_gguf(meta, tensors)


class GgufFile:
    """The library's parse of a GGUF image (bytes, bytearray or mmap), kept
    alive with the image: tensor views point into it."""

    def __init__(self, data):
        self._buf = data
        mv = memoryview(data)
        self._arr = (C.c_uint8 * len(mv)).from_buffer_copy(mv) if mv.readonly else \
            (C.c_uint8 * len(mv)).from_buffer(data)
        self._g = C.c_void_p()
        _check(lib().wl_gguf_open(self._arr, len(mv), C.byref(self._g)))

    @property
    def version(self) -> int:
        return int(lib().wl_gguf_version(self._g))

    @property
    def alignment(self) -> int:
        return int(lib().wl_gguf_alignment(self._g))

    def __len__(self) -> int:
        return int(lib().wl_gguf_tensor_count(self._g))

    @staticmethod
    def _view(v: WlTensorView) -> dict:
        shape = tuple(v.shape[i] for i in range(v.n_dims))
        data = np.ctypeslib.as_array(v.data, (v.data_len,)).copy() if v.data_len else \
            np.zeros(0, np.uint8)
        out = {"name": v.name.decode(), "shape": shape, "type": int(v.ggml_type), "data": data}
        if v.scale_len:
            out["scale_block"] = np.ctypeslib.as_array(v.scale_data, (v.scale_len,)).copy()
        return out

    def tensor(self, key) -> dict:
        v = WlTensorView()
        if isinstance(key, int):
            _check(lib().wl_gguf_tensor(self._g, key, C.byref(v)))
        else:
            _check(lib().wl_gguf_find_tensor(self._g, key.encode(), C.byref(v)))
        return self._view(v)

    def tensors(self) -> Iterable[dict]:
        return (self.tensor(i) for i in range(len(self)))

    def u64(self, key: str) -> int:
        out = C.c_uint64()
        _check(lib().wl_gguf_get_u64(self._g, key.encode(), C.byref(out)))
        return int(out.value)

    def f32(self, key: str) -> float:
        out = C.c_float()
        _check(lib().wl_gguf_get_f32(self._g, key.encode(), C.byref(out)))
        return float(out.value)

    def str(self, key: str) -> str:
        out = C.c_char_p()
        _check(lib().wl_gguf_get_str(self._g, key.encode(), C.byref(out)))
        return out.value.decode()

    def array_len(self, key: str) -> int:
        return int(lib().wl_gguf_array_len(self._g, key.encode()))

    def model_config(self) -> tuple[dict, int]:
        """ModelConfig::from_gguf_metadata: (config dict, variant)."""
        cfg, var = WlBitnetConfig(), C.c_uint32()
        _check(lib().wl_gguf_model_config(self._g, C.byref(cfg), C.byref(var)))
        keys = ("n_layers", "n_embd", "n_heads", "n_kv_heads", "head_dim", "n_ff", "vocab",
                "n_rot", "max_seq", "eps", "freq_base")
        return {k: getattr(cfg, k) for k in keys}, int(var.value)

    def close(self):
        if self._g:
            lib().wl_gguf_close(self._g)
            self._g = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
