"""Device-resident BitNet decode step against the oracle of the reference's
cached forward and greedy generation (oracle/bitnet_forward.c).

Two modes.  Exact mode is the reference's arithmetic -- its sequential sums
in its order and its exp (glibc's expf, restated in csrc/glibc_expf.cuh): hidden states must agree within EXACT_RTOL (1e-5, the
north-star f32 bound, stated here although the arithmetic is the
reference's own) and greedy ids must be identical.  Fast mode sums RMSNorm,
softmax and the weighted V as parallel trees: rounding-level differences, which the int8 re-quantisation at every
BitLinear occasionally turns into a one-step flip of one activation (about
1 % of a hidden vector), so it is held to greedy-id identity plus a
rounding-level median and a flip-level maximum on small models.
"""
import numpy as np
import pytest

import oracle
from project_willamette_b200 import WillametteError, synth
from project_willamette_b200._abi import WLStatus

pytestmark = pytest.mark.gpu

EXACT_RTOL = 1e-5    # exact mode, every step
DECODE_RTOL = 1e-4   # fast mode, median over steps: rounding-level agreement
FLIP_RTOL = 5e-2     # fast mode, worst step: a few int8 re-quantisation flips


def _rel(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def _check_errs(errs, what):
    errs = np.asarray(errs)
    msg = f"{what}: per-step max-norm rel err {np.array2string(errs, precision=2)}"
    assert np.median(errs) <= DECODE_RTOL, msg
    assert errs.max() <= FLIP_RTOL, msg


def _check_exact(errs, what):
    errs = np.asarray(errs)
    assert errs.max() <= EXACT_RTOL, \
        f"{what}: per-step max-norm rel err {np.array2string(errs, precision=2)}"


def _model(seed, **kw):
    return synth.bitnet_model(np.random.default_rng(seed), **kw)


CASES = {
    "tiny_mha": dict(n_layers=2, n_embd=256, n_heads=2, n_kv_heads=1, n_ff=512, vocab=300,
                     max_seq=32),
    "gqa": dict(n_layers=3, n_embd=512, n_heads=4, n_kv_heads=2, n_ff=768, vocab=1000,
                max_seq=48),
    "head64": dict(n_layers=2, n_embd=256, n_heads=4, n_kv_heads=2, head_dim=64, n_ff=384,
                   vocab=500, max_seq=24),
}


@pytest.mark.parametrize("persistent", [False, True])
@pytest.mark.parametrize("exact", [False, True])
@pytest.mark.parametrize("name", list(CASES))
def test_decode_matches_oracle(name, exact, persistent):
    """Both engines: the per-op chain and the persistent whole-forward kernel."""
    from project_willamette_b200.bitnet import BitNet
    m = _model(100 + list(CASES).index(name), **CASES[name])
    rng = np.random.default_rng(1)
    n_prompt = m["config"]["max_seq"] // 2
    prompt = rng.integers(0, m["config"]["vocab"], n_prompt)
    o = oracle.BitnetOracle(m)
    g = BitNet(m, exact=exact, persistent=persistent)
    assert g.persistent == persistent
    check = _check_exact if exact else _check_errs
    try:
        errs = []
        for i, t in enumerate(prompt):  # forward_with_cache, token by token
            want = o.forward(int(t), i)
            got = g.forward(int(t), i)
            errs.append(_rel(got, want))
        check(errs, "prefill")
        n_new = m["config"]["max_seq"] - n_prompt
        want_ids, want_h = o.generate(prompt, n_new, hiddens=True)
        got_ids, got_h = g.generate(prompt, n_new, hiddens=True)
        assert got_ids.tolist() == want_ids.tolist()
        check([_rel(a, b) for a, b in zip(got_h, want_h)], "decode")
        assert g.position == n_prompt + n_new - 1
    finally:
        g.close()


def test_decode_errors_follow_the_reference():
    from project_willamette_b200.bitnet import BitNet
    m = _model(3, **CASES["tiny_mha"])
    g = BitNet(m)
    try:
        for bad in (lambda: g.forward(1, 5), lambda: g.forward(300, 0),
                    lambda: g.generate([], 3), lambda: g.generate([1] * 30, 5)):
            with pytest.raises(WillametteError) as e:
                bad()
            assert e.value.status == WLStatus.GGUF_PARSE
        # a non-finite hidden after a layer is an error (cached_forward.rs:507-517)
        m2 = dict(m)
        m2["w_scale"] = m["w_scale"].copy()
        m2["w_scale"][6] = 3e38  # layer 0's down projection overflows to inf
        g2 = BitNet(m2)
        try:
            with pytest.raises(WillametteError) as e:
                g2.forward(1, 0)
            assert e.value.status == WLStatus.GGUF_PARSE
        finally:
            g2.close()
        with pytest.raises(oracle.OracleError):
            oracle.BitnetOracle(m2).forward(1, 0)
    finally:
        g.close()


@pytest.fixture(scope="module")
def bitnet2b():
    m = _model(0x5EED + 2, max_seq=16)
    prompt = [11, 2024, 77777, 5, 128255, 42]
    ids, hs = oracle.BitnetOracle(m).generate(prompt, 6, hiddens=True)
    return m, prompt, ids, hs


@pytest.mark.parametrize("exact", [True, False])
@pytest.mark.parametrize("persistent", [False, True])
def test_decode_bitnet2b_shapes(bitnet2b, exact, persistent):
    """Benchmark config 2 shapes (30 layers, 2560, 20/5 heads, 6912, vocab
    128256), a short prompt and a few greedy tokens.  Fast mode at 30 layers
    accumulates re-quantisation flips in the hidden state (see the module
    docstring), so only its ids are held to the reference there."""
    from project_willamette_b200.bitnet import BitNet
    m, prompt, want_ids, want_h = bitnet2b
    g = BitNet(m, exact=exact, persistent=persistent)
    assert g.persistent == persistent
    try:
        got_ids, got_h = g.generate(prompt, 6, hiddens=True)
        assert got_ids.tolist() == want_ids.tolist()
        if exact:
            _check_exact([_rel(a, b) for a, b in zip(got_h, want_h)], "decode")
    finally:
        g.close()


@pytest.mark.parametrize("exact", [False, True])
@pytest.mark.parametrize("name", list(CASES))
def test_decode_f16_kv_matches_oracle_f16_variant(name, exact):
    """kv_f16: binary16 KV rows (benchmark config 2's cache layout).  The
    reference has no such cache, so the checker is the oracle's f16 variant
    (the same forward with the rows rounded to binary16 and read back):
    exact mode to EXACT_RTOL with identical ids.  Fast mode: identical ids
    and every step within FLIP_RTOL -- not the rounding-level median, since
    one re-quantisation flip during the prefill changes the cached rows of
    every later position (with the int8 cache too; at these seeds the int8
    runs happen to have none).  The persistent flag is ignored with this
    layout (per-operation engine)."""
    from project_willamette_b200.bitnet import BitNet
    m = _model(200 + list(CASES).index(name), **CASES[name])
    rng = np.random.default_rng(2)
    n_prompt = m["config"]["max_seq"] // 2
    prompt = rng.integers(0, m["config"]["vocab"], n_prompt)
    n_new = m["config"]["max_seq"] - n_prompt
    o = oracle.BitnetOracle(m, kv_f16=True)
    want_ids, want_h = o.generate(prompt, n_new, hiddens=True)
    g = BitNet(m, exact=exact, persistent=True, kv_f16=True)
    assert not g.persistent
    try:
        got_ids, got_h = g.generate(prompt, n_new, hiddens=True)
        assert got_ids.tolist() == want_ids.tolist()
        errs = [_rel(a, b) for a, b in zip(got_h, want_h)]
        if exact:
            _check_exact(errs, "decode")
        else:
            assert max(errs) <= FLIP_RTOL, f"decode: per-step rel err {np.round(errs, 4)}"
    finally:
        g.close()


@pytest.mark.parametrize("exact", [True, False])
def test_decode_f16_kv_bitnet2b_shapes(bitnet2b, exact):
    """kv_f16 at benchmark config 2 shapes against the oracle's f16 variant
    (ids; exact mode also the hidden states)."""
    from project_willamette_b200.bitnet import BitNet
    m, prompt, _, _ = bitnet2b
    want_ids, want_h = oracle.BitnetOracle(m, kv_f16=True).generate(prompt, 6, hiddens=True)
    g = BitNet(m, exact=exact, kv_f16=True)
    try:
        got_ids, got_h = g.generate(prompt, 6, hiddens=True)
        assert got_ids.tolist() == want_ids.tolist()
        if exact:
            _check_exact([_rel(a, b) for a, b in zip(got_h, want_h)], "decode")
    finally:
        g.close()
