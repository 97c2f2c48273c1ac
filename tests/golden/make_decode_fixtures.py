"""Golden fixtures of the two benchmarked decode configurations, made by the
oracle (oracle/bitnet_forward.c: the reference's cached forward and greedy
generation, cached_forward.rs:164-504 and generate.rs:111-190) on the same
seeded synthetic models and prompts that bench.py times:

  decode_bitnet2b_512p128.npz -- benchmark config 2: BitNet-b1.58-2B shapes,
      KV cache prefilled with a 512-token prompt, 128 greedy tokens: every id,
      and the final hidden state (after output_norm) of every 16th step.
  decode_smollm_32x64.npz -- benchmark config 5: SmolLM-135M shapes, 32
      sequences with contexts U[64, 1024], 64 greedy tokens each: every id,
      and every sequence's final hidden state at steps 0, 31 and 63.

The GPU tests (tests/test_gpu_decode_bench_config.py) rebuild the same
models from the same seeds and compare the engines with these arrays.  The
oracle needs minutes for these sizes, which is why it runs here once and
not inside the test.  Usage: python tests/golden/make_decode_fixtures.py
"""
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

SEED = 0x5EED + 2           # bench.py's seed base
BITNET_STEPS = list(range(0, 128, 16)) + [127]
SMOLLM_STEPS = [0, 31, 63]


def bitnet_inputs():
    from project_willamette_b200 import synth
    m = synth.bitnet_model(np.random.default_rng(SEED + 7), max_seq=512 + 128)
    prompt = np.random.default_rng(SEED + 8).integers(0, m["config"]["vocab"], 512)
    return m, prompt


def smollm_inputs():
    from project_willamette_b200 import synth
    m = synth.llama_q8_model(np.random.default_rng(SEED + 11))
    rng = np.random.default_rng(SEED + 12)
    ctx = rng.integers(64, 1025, 32)
    prompts = [rng.integers(0, m["config"]["vocab"], int(n)) for n in ctx]
    return m, prompts


def fingerprint(m) -> np.ndarray:
    """A few weight bytes and norms, so a changed generator is caught."""
    w = m["w"]
    return np.concatenate([np.asarray(w[0][:64], np.float64), np.asarray(w[-1][-64:], np.float64),
                           np.asarray(m["norms"][:16], np.float64),
                           np.asarray(m["w_scale"][:8], np.float64)])


def main():
    import oracle
    t0 = time.time()
    m, prompt = bitnet_inputs()
    ids, hs = oracle.BitnetOracle(m).generate(prompt, 128, hiddens=True)
    np.savez_compressed(os.path.join(HERE, "decode_bitnet2b_512p128.npz"), ids=ids,
                        steps=np.array(BITNET_STEPS), hiddens=hs[BITNET_STEPS],
                        fingerprint=fingerprint(m))
    print(f"bitnet2b 512+128: {time.time() - t0:.0f} s", flush=True)
    t0 = time.time()
    m, prompts = smollm_inputs()
    all_ids, all_h = [], []
    for p in prompts:
        i, h = oracle.BitnetOracle(m).generate(p, 64, hiddens=True)
        all_ids.append(i)
        all_h.append(h[SMOLLM_STEPS])
    np.savez_compressed(os.path.join(HERE, "decode_smollm_32x64.npz"),
                        ids=np.stack(all_ids, 1), steps=np.array(SMOLLM_STEPS),
                        hiddens=np.stack(all_h, 1), fingerprint=fingerprint(m))
    print(f"smollm 32x64: {time.time() - t0:.0f} s", flush=True)


if __name__ == "__main__":
    main()
