"""Named single workloads at the benchmark's shapes, for profiling one
kernel family without the rest of ``bench.py``:

    python workloads.py smollm_decode
    python workloads.py bitnet_decode
    python workloads.py bitnet_decode_exact
    python workloads.py lm_head
    python workloads.py gemm_small

Each sets its model up (seeded as in ``bench.py``), prefills, and then runs
two decode steps inside a CUDA profiler range (``cudaProfilerStart`` /
``Stop``), so ``ncu --profile-from-start off`` captures only the steady
decode kernels.  ``lm_head`` repacks a 128256 x 2560 Q6_K matrix (config 4)
and runs the greedy head at batch 1 (twice) and batch 64 (once) inside the
range.  ``gemm_small`` runs the prefill GEMM of config 3's smallest case
(M 128, K 6912, N 2560: quantisation + warp-specialised tcgen05 GEMM over
expanded int8 weights) twice inside the range.
"""
from __future__ import annotations

import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

SEED = 0x5EED + 2  # bench.py's seed base


def _profiled(fn):
    import torch
    torch.cuda.init()
    torch.cuda.profiler.start()
    out = fn()
    torch.cuda.profiler.stop()
    return out


def smollm_decode(steps: int = 2) -> float:
    """Benchmark config 5: 32 sequences prefilled to contexts U[64, 1024],
    then `steps` batched greedy steps (fast mode)."""
    from project_willamette_b200 import synth
    from project_willamette_b200.llama import LlamaBatch
    m = synth.llama_q8_model(np.random.default_rng(SEED + 11))
    rng = np.random.default_rng(SEED + 12)
    ctx = rng.integers(64, 1025, 32)
    prompts = [rng.integers(0, m["config"]["vocab"], int(n)) for n in ctx]
    g = LlamaBatch(m, 32)
    g.prefill(prompts)
    _, ms = _profiled(lambda: g.decode(steps, timed=True))
    g.close()
    return ms


def bitnet_decode(steps: int = 2, exact: bool = False) -> float:
    """Benchmark config 2: BitNet-2B shapes, 512-token prompt, then `steps`
    greedy steps (per-operation engine; fast mode, or exact mode with the
    reference's sequential sums)."""
    from project_willamette_b200 import synth
    from project_willamette_b200.bitnet import BitNet
    m = synth.bitnet_model(np.random.default_rng(SEED + 7), max_seq=512 + 128)
    prompt = np.random.default_rng(SEED + 8).integers(0, m["config"]["vocab"], 512)
    g = BitNet(m, exact=exact)
    g.prefill(prompt)
    _, ms = _profiled(lambda: g.decode(steps, timed=True))
    g.close()
    return ms


def lm_head(calls: int = 2) -> float:
    """Benchmark config 4: Q6_K tied lm-head + greedy argmax, 128256 x 2560;
    `calls` batch-1 calls and one batch-64 call, device entry points on
    device buffers.  Returns the batch-1 ms per call."""
    import torch
    from project_willamette_b200 import synth
    from project_willamette_b200._abi import lib
    L = lib()
    d_model, vocab = 2560, 128256
    dev = torch.device("cuda:0")
    raw = torch.from_numpy(synth.q6k_rows(np.random.default_rng(SEED + 4), d_model, vocab))
    raw = raw.to(dev)
    packed = torch.empty(L.wl_q6k_packed_bytes(d_model, vocab), dtype=torch.uint8, device=dev)
    s = torch.cuda.current_stream().cuda_stream
    if L.wl_dev_q6k_repack(raw.data_ptr(), d_model, vocab, packed.data_ptr(), s):
        raise RuntimeError(L.wl_last_error().decode())
    del raw
    H = torch.randn(64, d_model, device=dev, generator=torch.Generator(dev).manual_seed(SEED))
    ids = torch.zeros(64, dtype=torch.int32, device=dev)
    scratch = torch.zeros(L.wl_q6k_scratch_bytes(64), dtype=torch.uint8, device=dev)

    def head(batch):
        if L.wl_dev_q6k_lm_head(packed.data_ptr(), d_model, vocab, H.data_ptr(), batch, None,
                                ids.data_ptr(), scratch.data_ptr(), s):
            raise RuntimeError(L.wl_last_error().decode())

    head(1)
    torch.cuda.synchronize()

    def run():
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(calls):
            head(1)
        b.record()
        head(64)
        torch.cuda.synchronize()
        return a.elapsed_time(b) / calls

    return _profiled(run)


def gemm_small(calls: int = 2) -> float:
    """Benchmark config 3, M = 128 x (K 6912 -> N 2560): device entry points on
    device buffers.  Returns ms per call."""
    import torch
    from project_willamette_b200 import synth
    from project_willamette_b200._abi import lib
    L = lib()
    M, K, N = 128, 6912, 2560
    dev = torch.device("cuda:0")
    rng = np.random.default_rng(SEED + 3)
    packed = torch.from_numpy(synth.i2s_packed(rng, K, N)).to(dev)
    x = torch.randn(M, K, device=dev, generator=torch.Generator(dev).manual_seed(SEED))
    y = torch.empty(M, N, device=dev)
    ws = torch.empty(L.wl_i2s_gemm_workspace_bytes(M, K), dtype=torch.uint8, device=dev)
    tern = torch.empty(L.wl_i2s_expanded_bytes(K, N), dtype=torch.int8, device=dev)
    s = torch.cuda.current_stream().cuda_stream
    if L.wl_dev_i2s_expand(packed.data_ptr(), K, N, tern.data_ptr(), s):
        raise RuntimeError(L.wl_last_error().decode())

    def call():
        if L.wl_dev_i2s_gemm_s8_f32(tern.data_ptr(), 0.05, K, N, M, x.data_ptr(), y.data_ptr(),
                                    None, ws.data_ptr(), s):
            raise RuntimeError(L.wl_last_error().decode())

    call()
    torch.cuda.synchronize()

    def run():
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(calls):
            call()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / calls

    return _profiled(run)


def bitnet_decode_exact(steps: int = 2) -> float:
    """`bitnet_decode` in exact mode."""
    return bitnet_decode(steps, exact=True)


WORKLOADS = {"smollm_decode": smollm_decode, "bitnet_decode": bitnet_decode,
             "bitnet_decode_exact": bitnet_decode_exact,
             "lm_head": lm_head, "gemm_small": gemm_small}

if __name__ == "__main__":
    name = sys.argv[1] if len(sys.argv) > 1 else ""
    if name not in WORKLOADS:
        sys.exit(f"usage: python workloads.py {{{','.join(WORKLOADS)}}}")
    print(f"{name}: {WORKLOADS[name]():.3f} ms")
