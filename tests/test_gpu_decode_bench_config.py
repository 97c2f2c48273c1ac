"""Greedy decode at the configurations bench.py times, against the oracle.

Benchmark config 2 (BitNet-b1.58-2B shapes, 512-token prompt, 128 greedy
tokens) and config 5 (SmolLM-135M shapes, 32 sequences with contexts
U[64, 1024], 64 greedy tokens each), on the same seeded models and prompts
as the bench.  The oracle's answers (every id, and hidden states at several
steps) were computed once by tests/golden/make_decode_fixtures.py, because
the oracle needs minutes at these sizes.

Exact mode is the reference's arithmetic (its sequential sums bit for bit,
and its exp, glibc's expf, restated): ids identical at every step and every
compared hidden state within EXACT_RTOL (1e-5, the north-star f32 bound).
Fast mode reorders sums (trees instead of sequential loops).  At the BitNet
configuration its 128 ids still equal the reference's and are held to that;
at the SmolLM configuration they do not (some sequences leave the
reference's ids after a few steps), so fast mode is benchmarked there as a
labelled non-conforming variant and not tested against these fixtures.
"""
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")
sys.path.insert(0, GOLDEN)

EXACT_RTOL = 1e-5


def _rel(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


@pytest.fixture(scope="module")
def bitnet_case():
    import make_decode_fixtures as mk
    m, prompt = mk.bitnet_inputs()
    f = np.load(os.path.join(GOLDEN, "decode_bitnet2b_512p128.npz"))
    np.testing.assert_array_equal(mk.fingerprint(m), f["fingerprint"])
    return m, prompt, f


@pytest.fixture(scope="module")
def smollm_case():
    import make_decode_fixtures as mk
    m, prompts = mk.smollm_inputs()
    f = np.load(os.path.join(GOLDEN, "decode_smollm_32x64.npz"))
    np.testing.assert_array_equal(mk.fingerprint(m), f["fingerprint"])
    return m, prompts, f


@pytest.mark.parametrize("exact", [True, False])
def test_bitnet2b_512_prompt_128_tokens(bitnet_case, exact):
    from project_willamette_b200.bitnet import BitNet
    m, prompt, f = bitnet_case
    g = BitNet(m, exact=exact)
    try:
        ids, hs = g.generate(prompt, 128, hiddens=True)
    finally:
        g.close()
    first_diff = next((i for i, (a, b) in enumerate(zip(ids, f["ids"])) if a != b), None)
    assert first_diff is None, f"ids differ from step {first_diff} of 128"
    if exact:
        errs = [_rel(hs[s], f["hiddens"][k]) for k, s in enumerate(f["steps"])]
        assert max(errs) <= EXACT_RTOL, f"hidden rel err per compared step {errs}"


def test_smollm_32_sequences_64_tokens(smollm_case):
    from project_willamette_b200.llama import LlamaBatch
    m, prompts, f = smollm_case
    exact = True
    g = LlamaBatch(m, len(prompts), exact=exact)
    try:
        ids, hs = g.generate(prompts, 64, hiddens=True)  # [64, S], [64, S, E]
    finally:
        g.close()
    diff = np.argwhere(ids != f["ids"])
    assert diff.size == 0, f"{len(diff)} ids differ, first at (step, sequence) {diff[0].tolist()}"
    if exact:
        errs = [_rel(hs[s, q], f["hiddens"][k, q]) for k, s in enumerate(f["steps"])
                for q in range(len(prompts))]
        assert max(errs) <= EXACT_RTOL, f"worst hidden rel err {max(errs):.3g}"
