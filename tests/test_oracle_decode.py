"""The decode-step oracle (oracle/bitnet_forward.c) pinned by the reference's
own unit tests of the primitives it restates, plus the forward's validation
rules and determinism.  CPU only.

The reference's primitive tests assert properties with tolerances (not
golden bit patterns); they are restated here with the same inputs and
bounds, each citing its source.
"""
import math

import numpy as np
import pytest

import oracle
from project_willamette_b200 import synth


def test_rms_norm_unit_weight():
    # primitives.rs:485-502
    x = np.array([1.0, 2.0, 3.0, 4.0], np.float32)
    out = oracle.rms_norm(x, np.ones(4, np.float32), 1e-5)
    denom = np.float32(math.sqrt(np.float32(7.5) + np.float32(1e-5)))
    assert np.all(np.abs(out - x / denom) < 1e-6)


def test_rope_position_zero_is_identity():
    # primitives.rs:513-526, attention.rs:368-380
    x = np.array([0.1, 0.2, 0.3, 0.4], np.float32)
    assert np.all(np.abs(oracle.rope_neox(x, 4, 0, 10000.0) - x) < 1e-6)
    q = np.full(128, 0.5, np.float32)
    assert np.all(np.abs(oracle.rope_neox(q, 128, 0, 500000.0) - q) < 1e-6)


def test_rope_preserves_neox_pair_norms():
    # primitives.rs:527-547
    x = np.array([0.4, 0.7, 0.1, -0.5, 0.2, 0.3, -0.6, 0.05], np.float32)
    y = oracle.rope_neox(x, 8, 3, 500000.0)
    for j in range(4):
        pre = x[j] ** 2 + x[j + 4] ** 2
        post = y[j] ** 2 + y[j + 4] ** 2
        assert abs(pre - post) < 1e-5
    # a zero head stays zero (attention.rs:382-395)
    assert np.all(oracle.rope_neox(np.zeros(128, np.float32), 128, 7, 500000.0) == 0.0)


def test_softmax_reference_cases():
    # attention.rs:321-366
    assert oracle.softmax([1.25]).tolist() == [1.0]
    u = oracle.softmax([0.0] * 4)
    assert np.all(np.abs(u - 0.25) < 1e-6) and abs(u.sum() - 1.0) < 1e-6
    m = oracle.softmax([-np.inf, 0.0])
    assert m[0] == 0.0 and abs(m[1] - 1.0) < 1e-6
    t = oracle.softmax([1.0, 2.0, 3.0, 4.0, 5.0])
    assert abs(t.sum() - 1.0) < 1e-6 and np.all(np.diff(t) > 0)
    assert np.all(oracle.softmax([-np.inf] * 4) == 0.0)
    # NaN or +inf present: the max is not finite -> zeros (attention.rs:55-61)
    assert np.all(oracle.softmax([1.0, np.inf]) == 0.0)


def test_kv_quantise_round_trip():
    # kv_cache.rs:290-318
    k = np.array([0.1, -0.2, 0.3, -0.4], np.float32)
    v = np.array([10.0, -20.0, 30.0, -40.0], np.float32)
    for x, tol in ((k, 0.4 / 200.0), (v, 40.0 / 200.0)):
        q, s = oracle.kv_quantise(x)
        assert np.all(np.abs(q.astype(np.float32) * np.float32(s) - x) <= tol)
    q, s = oracle.kv_quantise(np.zeros(4, np.float32))
    assert s == 0.0 and np.all(q == 0)
    q, s = oracle.kv_quantise(np.array([1.0, np.inf], np.float32))
    assert s == 0.0 and np.all(q == 0)  # non-finite absmax stores zeros


def _small(seed=5, **kw):
    args = dict(n_layers=2, n_embd=256, n_heads=2, n_kv_heads=1, n_ff=512, vocab=300,
                max_seq=32)
    args.update(kw)
    return synth.bitnet_model(np.random.default_rng(seed), **args)


def test_forward_validation_and_thread_independence():
    m = _small()
    o = oracle.BitnetOracle(m)
    with pytest.raises(oracle.OracleError):
        o.forward(1, 1)  # position must equal the cache position
    with pytest.raises(oracle.OracleError):
        o.forward(300, 0)  # token outside the vocabulary
    h1 = o.forward(7, 0, n_threads=1)
    o2 = oracle.BitnetOracle(m)
    h8 = o2.forward(7, 0, n_threads=8)
    assert np.array_equal(h1.view(np.uint32), h8.view(np.uint32))
    with pytest.raises(oracle.OracleError):
        o.generate([], 3)  # generate.rs:121-125


def test_generate_matches_step_by_step_forward():
    m = _small(seed=9)
    o = oracle.BitnetOracle(m)
    prompt = [3, 141, 59, 26]
    ids, hs = o.generate(prompt, 5, hiddens=True)
    o2 = oracle.BitnetOracle(m)
    for i, t in enumerate(prompt):
        h = o2.forward(t, i)
    assert np.array_equal(h, hs[0])
    logits = oracle.compute_logits(h, m["token_embd"], 14, 256, 300)
    assert ids[0] == oracle.argmax(logits)


def test_silu_known_values():
    # ffn.rs:157-164
    v = oracle.silu([-1.0, 0.0, 1.0])
    assert abs(v[0] + 0.26894143) < 1e-6 and v[1] == 0.0 and abs(v[2] - 0.7310586) < 1e-6


def test_rope_norm_pairs_and_differs_from_neox():
    # primitives.rs:549-566 and tests/primitives.rs:233-251
    a = oracle.rope_norm([1.0, 0.0, 0.0, 0.0], 4, 1, 10000.0)
    b = oracle.rope_neox([1.0, 0.0, 0.0, 0.0], 4, 1, 10000.0)
    assert np.max(np.abs(a - b)) > 1e-6
    x = (np.arange(128) * 0.01).astype(np.float32)
    y = oracle.rope_norm(x, 128, 5, 500000.0)
    assert np.max(np.abs(y - oracle.rope_neox(x, 128, 5, 500000.0))) > 1e-3
    for j in range(64):  # the (2j, 2j+1) pair norms are kept
        assert abs(x[2 * j] ** 2 + x[2 * j + 1] ** 2 - y[2 * j] ** 2 - y[2 * j + 1] ** 2) < 1e-5
    assert np.all(np.abs(oracle.rope_norm(x, 128, 0, 10000.0) - x) < 1e-6)


def _small_llama(seed=5, **kw):
    args = dict(n_layers=2, n_embd=128, n_heads=2, n_kv_heads=1, n_ff=256, vocab=300,
                max_seq=32)
    args.update(kw)
    return synth.llama_q8_model(np.random.default_rng(seed), **args)


def test_llama_q8_forward_follows_its_primitives():
    """The VanillaLlama variant with Q8_0 linears, checked against a numpy
    composition of the pinned primitives (one layer, position 0, where the
    attention output is V itself: softmax over one key is exactly 1), down to
    the final output norm the forward returns."""
    m = _small_llama(n_layers=1)
    c = m["config"]
    E, KV, F = c["n_embd"], c["n_kv_heads"] * c["head_dim"], c["n_ff"]
    tok = 17
    emb = oracle.q8_0_dequantize_row(m["token_embd"][tok * (E // 32) * 34:][:(E // 32) * 34], E)
    nrm = m["norms"]
    attn_norm, ffn_norm = nrm[:E], nrm[2 * E:3 * E]  # layer layout: attn, attn_sub, ffn, ffn_sub
    w = m["w"]

    def lin(i, x, n):
        return oracle.q8_0_matvec(w[i], x.size, n, x)

    xn = oracle.rms_norm(emb, attn_norm, c["eps"])
    v = lin(2, xn, KV)
    vq, vs = oracle.kv_quantise(v)
    att = np.tile(vq.astype(np.float32) * np.float32(vs), c["n_heads"] // c["n_kv_heads"])
    h = emb + lin(3, att, E)
    xn = oracle.rms_norm(h, ffn_norm, c["eps"])
    fused = oracle.silu(lin(4, xn, F)) * lin(5, xn, F)
    h = h + lin(6, fused, E)
    want = oracle.rms_norm(h, m["output_norm"], c["eps"])  # cached_forward.rs:248-257
    got = oracle.BitnetOracle(m).forward(tok, 0)
    assert np.array_equal(got, want)


def test_f16_kv_variant_stores_rounded_rows():
    """The oracle's binary16-KV variant (the checker of the library's kv_f16
    option): each cached row is the f32 row rounded to nearest even, the
    first forward (one position: softmax weight 1) equals the i8 variant's
    except through the cached values, and generation stays finite."""
    m = _small(seed=5)
    o16 = oracle.BitnetOracle(m, kv_f16=True)
    o8 = oracle.BitnetOracle(m)
    h16 = o16.forward(7, 0)
    h8 = o8.forward(7, 0)
    c = m["config"]
    kv = c["n_kv_heads"] * c["head_dim"]
    row = o16.kq.view(np.uint16)[:kv]
    # every stored value is a finite half, and re-rounding it is the identity
    vals = row.view(np.float16).astype(np.float32)
    assert np.all(np.isfinite(vals))
    assert np.array_equal(vals.astype(np.float16).view(np.uint16), row)
    # the i8 variant's cache for the same forward quantises differently
    assert not np.array_equal(h16, h8)
    assert np.max(np.abs(h16 - h8)) / np.max(np.abs(h8)) < 0.5
    ids = o16.generate([3, 141, 59], 4)
    assert len(ids) == 4
