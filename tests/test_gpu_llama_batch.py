"""Batched Q8_0 Llama decode (project_willamette_b200.llama.LlamaBatch)
against the oracle of the reference's per-sequence greedy generation with the
VanillaLlama forward (oracle/bitnet_forward.c, variant 1, Q8_0).

Exact mode runs the reference's arithmetic everywhere: the Q8_0 linears are
bit-exact, the norms and softmax sum in the reference's order, and exp
(softmax and SiLU) is glibc's expf restated (csrc/glibc_expf.cuh), so hidden
states are held to EXACT_RTOL (the north-star f32 bound) and greedy ids must
be identical.  Fast mode contracts the Q8_0 products into FMAs and sums norms
and softmax as trees: rounding-level differences, which the per-token int8
quantisation of K and V in the cache (kv_cache.rs:245-259) occasionally
turns into a one-step flip of one cached value, so fast mode is held to
identical ids, a rounding-level median (FAST_RTOL) and a flip-level maximum
(FLIP_RTOL).
"""
import numpy as np
import pytest

import oracle
from project_willamette_b200 import WillametteError, synth
from project_willamette_b200._abi import WLStatus

pytestmark = pytest.mark.gpu

EXACT_RTOL = 1e-5   # exact mode, every step
FAST_RTOL = 1e-4    # fast mode, median over steps and sequences
FLIP_RTOL = 5e-2    # fast mode, worst step: a few KV re-quantisation flips


def _rel(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def _check(errs, exact, what=""):
    errs = np.asarray(errs)
    msg = f"{what} per-step max-norm rel err {np.array2string(errs, precision=2)}"
    if exact:
        assert errs.max() <= EXACT_RTOL, msg
    else:
        assert np.median(errs) <= FAST_RTOL and errs.max() <= FLIP_RTOL, msg


def _model(seed, **kw):
    return synth.llama_q8_model(np.random.default_rng(seed), **kw)


CASES = {
    "mha": dict(n_layers=2, n_embd=128, n_heads=2, n_kv_heads=2, n_ff=256, vocab=300,
                max_seq=40),
    "gqa": dict(n_layers=3, n_embd=192, n_heads=3, n_kv_heads=1, n_ff=384, vocab=700,
                max_seq=48),
    "smol_head": dict(n_layers=2, n_embd=576, n_heads=9, n_kv_heads=3, n_ff=1536, vocab=1000,
                      max_seq=64),
}


def _oracle_runs(m, prompts, n_new):
    ids, hs = [], []
    for p in prompts:
        i, h = oracle.BitnetOracle(m).generate(p, n_new, hiddens=True)
        ids.append(i)
        hs.append(h)
    return np.stack(ids, 1), np.stack(hs, 1)  # [n_new, S], [n_new, S, E]


@pytest.mark.parametrize("exact", [True, False])
@pytest.mark.parametrize("n_seqs", [1, 5])
@pytest.mark.parametrize("name", list(CASES))
def test_batch_generate_matches_oracle(name, n_seqs, exact):
    from project_willamette_b200.llama import LlamaBatch
    m = _model(300 + list(CASES).index(name), **CASES[name])
    c = m["config"]
    rng = np.random.default_rng(n_seqs)
    n_new = 6
    lens = rng.integers(1, c["max_seq"] - n_new, n_seqs)
    prompts = [rng.integers(0, c["vocab"], int(n)) for n in lens]
    want_ids, want_h = _oracle_runs(m, prompts, n_new)
    g = LlamaBatch(m, n_seqs, exact=exact)
    try:
        got_ids, got_h = g.generate(prompts, n_new, hiddens=True)
        assert got_ids.tolist() == want_ids.tolist()
        _check([_rel(got_h[s, b], want_h[s, b]) for s in range(n_new) for b in range(n_seqs)],
               exact)
        for b in range(n_seqs):
            assert g.position(b) == lens[b] + n_new - 1
    finally:
        g.close()


@pytest.mark.parametrize("tg", [1, 4, 8, 32])
def test_batch_tokens_per_cta_do_not_change_results(tg):
    """Every kernel instance (tokens per CTA) gives the oracle's ids and, in
    exact mode, its hiddens; 37 sequences leave a ragged last token group."""
    from project_willamette_b200.llama import LlamaBatch
    m = _model(21, **CASES["gqa"])
    rng = np.random.default_rng(tg)
    prompts = [rng.integers(0, 700, int(n)) for n in rng.integers(1, 10, 37)]
    want_ids, want_h = _oracle_runs(m, prompts, 3)
    g = LlamaBatch(m, 37, exact=True)
    try:
        g.set_tokens_per_cta(tg)
        ids, hs = g.generate(prompts, 3, hiddens=True)
        assert ids.tolist() == want_ids.tolist()
        _check([_rel(hs[s, b], want_h[s, b]) for s in range(3) for b in range(37)], True)
    finally:
        g.close()


def test_batch_prefill_in_pieces_and_idle_sequences():
    """Prefill in two calls, one sequence idle in each (empty prompt part),
    equals one prefill of the whole prompts."""
    from project_willamette_b200.llama import LlamaBatch
    m = _model(7, **CASES["gqa"])
    rng = np.random.default_rng(3)
    prompts = [rng.integers(0, 700, n) for n in (9, 4, 13)]
    want_ids, want_h = _oracle_runs(m, prompts, 5)
    g = LlamaBatch(m, 3, exact=True)
    try:
        g.prefill([prompts[0][:5], [], prompts[2][:1]])
        assert [g.position(b) for b in range(3)] == [5, 0, 1]
        g.prefill([prompts[0][5:], prompts[1], prompts[2][1:]])
        ids, hs = g.decode(5, hiddens=True)
        assert ids.tolist() == want_ids.tolist()
        _check([_rel(hs[s, b], want_h[s, b]) for s in range(5) for b in range(3)], True)
        more = g.decode(3)  # decoding further continues every sequence from its last id
        assert more.shape == (3, 3)
    finally:
        g.close()


def test_batch_errors_follow_the_reference():
    from project_willamette_b200.llama import LlamaBatch
    m = _model(11, **CASES["mha"])
    g = LlamaBatch(m, 2)
    try:
        for bad, status in (
                (lambda: g.generate([[1, 2], []], 3), WLStatus.GGUF_PARSE),       # empty prompt
                (lambda: g.generate([[1, 300], [2]], 3), WLStatus.GGUF_PARSE),    # token >= vocab
                (lambda: g.generate([[1] * 38, [2]], 3), WLStatus.GGUF_PARSE),    # cache too small
        ):
            with pytest.raises(WillametteError) as e:
                bad()
            assert e.value.status == status
        g.reset()
        with pytest.raises(WillametteError) as e:
            g.decode(2)  # nothing prefilled
        assert e.value.status == WLStatus.INVALID_ARGUMENT
    finally:
        g.close()
    # a non-finite Q8_0 block scale is rejected (q8_0.rs:50-70)
    m2 = dict(m)
    m2["w"] = [a.copy() for a in m["w"]]
    m2["w"][4][0:2] = np.frombuffer(np.float16(np.inf).tobytes(), np.uint8)
    with pytest.raises(WillametteError) as e:
        LlamaBatch(m2, 1)
    assert e.value.status == WLStatus.GGUF_PARSE


def test_batch_nonfinite_hidden_is_an_error():
    """A layer whose hidden overflows fails the step (cached_forward.rs:
    507-517), as the oracle does."""
    from project_willamette_b200.llama import LlamaBatch
    m = _model(13, **CASES["mha"])
    m2 = dict(m)
    m2["norms"] = m["norms"].copy()
    E = m["config"]["n_embd"]
    m2["norms"][2 * E:3 * E] = 1e30  # layer 0's ffn_norm: gate * up overflows
    with pytest.raises(oracle.OracleError):
        oracle.BitnetOracle(m2).generate([1, 2, 3], 2)
    g = LlamaBatch(m2, 2)
    try:
        with pytest.raises(WillametteError) as e:
            g.generate([[1, 2, 3], [4]], 2)
        assert e.value.status == WLStatus.GGUF_PARSE
    finally:
        g.close()


@pytest.fixture(scope="module")
def smollm():
    m = _model(0x5EED + 5, max_seq=48)
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, 49152, n) for n in (7, 12, 3, 20)]
    want_ids, want_h = _oracle_runs(m, prompts, 4)
    return m, prompts, want_ids, want_h


@pytest.mark.parametrize("exact", [True, False])
def test_batch_smollm_shapes(smollm, exact):
    """Benchmark config 5 shapes (30 layers, 576, 9 / 3 heads of 64, 1536,
    vocab 49152, all Q8_0), four sequences of different lengths."""
    from project_willamette_b200.llama import LlamaBatch
    m, prompts, want_ids, want_h = smollm
    g = LlamaBatch(m, len(prompts), exact=exact)
    try:
        ids, hs = g.generate(prompts, 4, hiddens=True)
        assert ids.tolist() == want_ids.tolist()
        _check([_rel(hs[s, b], want_h[s, b]) for s in range(4) for b in range(len(prompts))],
               exact)
    finally:
        g.close()
