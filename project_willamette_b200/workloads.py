"""Named single workloads at the benchmark's shapes, for profiling one
kernel family without the rest of ``bench.py``:

    python -m project_willamette_b200.workloads smollm_decode
    python -m project_willamette_b200.workloads bitnet_decode

Each sets its model up (seeded as in ``bench.py``), prefills, and then runs
two decode steps inside a CUDA profiler range (``cudaProfilerStart`` /
``Stop``), so ``ncu --profile-from-start off`` captures only the steady
decode kernels.
"""
from __future__ import annotations

import sys

import numpy as np

SEED = 0x5EED + 2  # bench.py's seed base


def _profiled(fn):
    import torch
    torch.cuda.init()
    torch.cuda.profiler.start()
    out = fn()
    torch.cuda.profiler.stop()
    return out


def smollm_decode(steps: int = 2) -> float:
    """32 sequences prefilled to contexts U[64, 1024],
    then `steps` batched greedy steps (fast mode)."""
    from . import synth
    from .llama import LlamaBatch
    m = synth.llama_q8_model(np.random.default_rng(SEED + 11))
    rng = np.random.default_rng(SEED + 12)
    ctx = rng.integers(64, 1025, 32)
    prompts = [rng.integers(0, m["config"]["vocab"], int(n)) for n in ctx]
    g = LlamaBatch(m, 32)
    g.prefill(prompts)
    _, ms = _profiled(lambda: g.decode(steps, timed=True))
    g.close()
    return ms


def bitnet_decode(steps: int = 2) -> float:
    """BitNet-2B shapes, 512-token prompt, then `steps`
    greedy steps (fast mode, per-operation engine)."""
    from . import synth
    from .bitnet import BitNet
    m = synth.bitnet_model(np.random.default_rng(SEED + 7), max_seq=512 + 128)
    prompt = np.random.default_rng(SEED + 8).integers(0, m["config"]["vocab"], 512)
    g = BitNet(m)
    g.prefill(prompt)
    _, ms = _profiled(lambda: g.decode(steps, timed=True))
    g.close()
    return ms


WORKLOADS = {"smollm_decode": smollm_decode, "bitnet_decode": bitnet_decode}

if __name__ == "__main__":
    name = sys.argv[1] if len(sys.argv) > 1 else ""
    if name not in WORKLOADS:
        sys.exit(f"usage: python -m project_willamette_b200.workloads {{{','.join(WORKLOADS)}}}")
    print(f"{name}: {WORKLOADS[name]():.3f} ms")
