"""Device-resident BitNet decode step against the oracle of the reference's
cached forward and greedy generation (oracle/bitnet_forward.c).

Bar: greedy token ids identical; final hidden states within DECODE_RTOL
(max-norm relative).  The per-element arithmetic is the reference's, but the
norms' and the attention's sums run as parallel trees on the GPU (and exp
is rounded from double), so hidden states agree to rounding level rather
than bit for bit; the BitLinears re-quantise to int8 at every layer, where a
rounding-level difference can flip one activation by one step, which is why
the bound is on the whole vector.
"""
import numpy as np
import pytest

import oracle
from project_willamette_b200 import WillametteError, synth
from project_willamette_b200._abi import WLStatus

pytestmark = pytest.mark.gpu

DECODE_RTOL = 1e-4


def _rel(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


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


@pytest.mark.parametrize("name", list(CASES))
def test_decode_matches_oracle(name):
    from project_willamette_b200.bitnet import BitNet
    m = _model(100 + list(CASES).index(name), **CASES[name])
    rng = np.random.default_rng(1)
    n_prompt = m["config"]["max_seq"] // 2
    prompt = rng.integers(0, m["config"]["vocab"], n_prompt)
    o = oracle.BitnetOracle(m)
    g = BitNet(m)
    try:
        worst = 0.0
        for i, t in enumerate(prompt):  # forward_with_cache, token by token
            want = o.forward(int(t), i)
            got = g.forward(int(t), i)
            worst = max(worst, _rel(got, want))
        assert worst <= DECODE_RTOL, f"prefill hidden rel err {worst:.3g}"
        n_new = m["config"]["max_seq"] - n_prompt
        want_ids, want_h = o.generate(prompt, n_new, hiddens=True)
        got_ids, got_h = g.generate(prompt, n_new, hiddens=True)
        assert got_ids.tolist() == want_ids.tolist()
        err = max(_rel(a, b) for a, b in zip(got_h, want_h))
        assert err <= DECODE_RTOL, f"decode hidden rel err {err:.3g}"
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


def test_decode_bitnet2b_shapes():
    """BASELINE config 2 shapes (30 layers, 2560, 20/5 heads, 6912, vocab
    128256), a short prompt and a few greedy tokens."""
    from project_willamette_b200.bitnet import BitNet
    m = _model(0x5EED + 2, max_seq=16)
    prompt = [11, 2024, 77777, 5, 128255, 42]
    o = oracle.BitnetOracle(m)
    want_ids, want_h = o.generate(prompt, 6, hiddens=True)
    g = BitNet(m)
    try:
        got_ids, got_h = g.generate(prompt, 6, hiddens=True)
        assert got_ids.tolist() == want_ids.tolist()
        err = max(_rel(a, b) for a, b in zip(got_h, want_h))
        assert err <= DECODE_RTOL, f"hidden rel err {err:.3g}"
    finally:
        g.close()
