"""Seeded synthetic weights and activations with the benchmark configs' distributions.

The reference builds synthetic GGUFs in src/synth.rs (xorshift codes, scale
1.0).  The benchmark configurations ask for other distributions, generated
here (numpy, seeded):

* I2_S: codes i.i.d. with P(01 -> 0) = 0.5 and P(00 -> -1) = P(10 -> +1) =
  0.25, packed in the reference layout (4 codes per byte, element gp +
  32k of a 128-block at bits 7-2k:6-2k); one f32 scale ~ U[0.01, 0.1].
  Because the codes are i.i.d., drawing each byte's four codes independently
  is the same distribution as drawing per element and packing.
* Q6_K: 6-bit values uniform in [-32, 31] (stored as value + 32 across the ql
  nibble and 2 qh bits, q6_k.rs:195-214, so uniform random ql/qh bytes are
  exactly that distribution), int8 sub-block scales uniform in [-128, 127],
  d = f16(|N(0, 0.002)|).
* Q8_0: int8 quants uniform in [-127, 127], d = f16(|N(0, 0.01)|).
* Activations: f32 N(0, 1).
"""
from __future__ import annotations

import numpy as np

# uniform 2-bit draw -> I2_S code: 00 -> 00 (-1), 01 -> 10 (+1), 10/11 -> 01 (0)
_CODE_OF_DRAW = np.array([0, 2, 1, 1], np.uint8)
_BYTE_LUT = np.array([(_CODE_OF_DRAW[(b >> 6) & 3] << 6) | (_CODE_OF_DRAW[(b >> 4) & 3] << 4)
                      | (_CODE_OF_DRAW[(b >> 2) & 3] << 2) | _CODE_OF_DRAW[b & 3]
                      for b in range(256)], np.uint8)


def i2s_packed(rng: np.random.Generator, in_dim: int, out_dim: int,
               code3_fraction: float = 0.0) -> np.ndarray:
    """Packed I2_S codes, out_dim x in_dim/4 bytes (flat)."""
    raw = rng.integers(0, 256, size=out_dim * in_dim // 4, dtype=np.uint8)
    packed = _BYTE_LUT[raw]
    if code3_fraction > 0:
        n = packed.size
        k = max(1, int(n * code3_fraction))
        idx = rng.choice(n, size=k, replace=False)
        shift = rng.integers(0, 4, size=k).astype(np.uint8) * 2
        packed[idx] |= (np.uint8(3) << shift).astype(np.uint8)
    return packed


def i2s_scale(rng: np.random.Generator) -> float:
    return float(np.float32(rng.uniform(0.01, 0.1)))


def activations(rng: np.random.Generator, *shape) -> np.ndarray:
    return rng.standard_normal(shape, dtype=np.float32)


def q6k_rows(rng: np.random.Generator, n_embd: int, vocab: int) -> np.ndarray:
    """GGUF Q6_K rows: vocab x (n_embd/256) x 210 bytes (flat)."""
    nb = n_embd // 256
    blocks = rng.integers(0, 256, size=(vocab * nb, 210), dtype=np.uint8)
    d = np.abs(rng.normal(0.0, 0.002, size=vocab * nb)).astype(np.float16)
    blocks[:, 208:210] = d.view(np.uint8).reshape(-1, 2)
    return blocks.reshape(-1)


def q8_0_rows(rng: np.random.Generator, in_dim: int, out_dim: int) -> np.ndarray:
    """GGUF Q8_0 rows: out_dim x (in_dim/32) x 34 bytes (flat)."""
    nb = in_dim // 32
    blocks = np.empty((out_dim * nb, 34), np.uint8)
    blocks[:, 2:] = rng.integers(-127, 128, size=(out_dim * nb, 32), dtype=np.int8).view(np.uint8)
    d = np.abs(rng.normal(0.0, 0.01, size=out_dim * nb)).astype(np.float16)
    blocks[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
    return blocks.reshape(-1)


# BitNet-b1.58-2B shapes (benchmark config 2): (name, in_dim, out_dim) per layer.
BITNET_2B_LAYER = [
    ("attn_q", 2560, 2560), ("attn_k", 2560, 640), ("attn_v", 2560, 640),
    ("attn_output", 2560, 2560), ("ffn_gate", 2560, 6912), ("ffn_up", 2560, 6912),
    ("ffn_down", 6912, 2560),
]
BITNET_2B_LAYERS = 30
BITNET_2B_VOCAB = 128256
BITNET_2B_EMBD = 2560


def bitnet_model(rng: np.random.Generator, n_layers: int = 30, n_embd: int = 2560,
                 n_heads: int = 20, n_kv_heads: int = 5, head_dim: int = 128, n_ff: int = 6912,
                 vocab: int = 128256, max_seq: int = 1024, eps: float = 1e-5,
                 freq_base: float = 500000.0) -> dict:
    """A random BitNet-b1.58-shaped model (benchmark config 2 distributions):
    every linear I2_S with P(0)=0.5 and a U[0.01, 0.1] scale, norm weights
    U[0.5, 1.5], tied Q6_K embedding / lm-head (config 4 distributions).
    Defaults are the 2B shapes."""
    kv = n_kv_heads * head_dim
    shapes = [(n_embd, n_embd), (n_embd, kv), (n_embd, kv), (n_embd, n_embd), (n_embd, n_ff),
              (n_embd, n_ff), (n_ff, n_embd)]
    w, sc = [], []
    for _ in range(n_layers):
        for k, n in shapes:
            w.append(i2s_packed(rng, k, n))
            sc.append(i2s_scale(rng))
    norms = rng.uniform(0.5, 1.5, size=n_layers * (3 * n_embd + n_ff)).astype(np.float32)
    return {
        "config": dict(n_layers=n_layers, n_embd=n_embd, n_heads=n_heads, n_kv_heads=n_kv_heads,
                       head_dim=head_dim, n_ff=n_ff, vocab=vocab, n_rot=head_dim,
                       max_seq=max_seq, eps=eps, freq_base=freq_base),
        "w": w,
        "w_scale": np.asarray(sc, np.float32),
        "norms": norms,
        "output_norm": rng.uniform(0.5, 1.5, size=n_embd).astype(np.float32),
        "token_embd": q6k_rows(rng, n_embd, vocab),
    }


def llama_q8_model(rng: np.random.Generator, n_layers: int = 30, n_embd: int = 576,
                   n_heads: int = 9, n_kv_heads: int = 3, head_dim: int = 64, n_ff: int = 1536,
                   vocab: int = 49152, max_seq: int = 1088, eps: float = 1e-5,
                   freq_base: float = 10000.0) -> dict:
    """A random SmolLM-135M-shaped Llama model (benchmark config 5): every
    linear and the tied embedding / lm-head Q8_0 (int8 quants U[-127, 127],
    f16 scale |N(0, 0.01)|), norm weights U[0.5, 1.5].  Defaults are the 135M
    shapes.  The norms array keeps the per-layer layout of ``bitnet_model``
    (attn_norm, attn_sub_norm, ffn_norm, ffn_sub_norm); the Llama forward
    reads only attn_norm and ffn_norm."""
    kv = n_kv_heads * head_dim
    shapes = [(n_embd, n_embd), (n_embd, kv), (n_embd, kv), (n_embd, n_embd), (n_embd, n_ff),
              (n_embd, n_ff), (n_ff, n_embd)]
    w = [q8_0_rows(rng, k, n) for _ in range(n_layers) for k, n in shapes]
    norms = rng.uniform(0.5, 1.5, size=n_layers * (3 * n_embd + n_ff)).astype(np.float32)
    return {
        "config": dict(n_layers=n_layers, n_embd=n_embd, n_heads=n_heads, n_kv_heads=n_kv_heads,
                       head_dim=head_dim, n_ff=n_ff, vocab=vocab, n_rot=head_dim,
                       max_seq=max_seq, eps=eps, freq_base=freq_base, variant=1,
                       linear_type=8, embd_type=8),
        "w": w,
        "w_scale": np.ones(len(w), np.float32),
        "norms": norms,
        "output_norm": rng.uniform(0.5, 1.5, size=n_embd).astype(np.float32),
        "token_embd": q8_0_rows(rng, n_embd, vocab),
    }
