"""Tensor-parallel BitNet decode on 2+ GPUs (one process per GPU): every
BitLinear row-split over the ranks and gathered in-kernel, attention and the
KV cache replicated, the lm-head vocab-sharded.  Each rank's greedy ids and
hidden states must equal the single-GPU engine's bit for bit (the per-row
arithmetic is unchanged by the split), and the ids the oracle's.

Needs at least two GPUs; skipped otherwise.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CASES = [
    ("gqa", dict(n_layers=3, n_embd=512, n_heads=4, n_kv_heads=2, n_ff=768, vocab=1000,
                 max_seq=40)),
    ("head64", dict(n_layers=2, n_embd=256, n_heads=4, n_kv_heads=2, head_dim=64, n_ff=384,
                    vocab=501, max_seq=24)),
]


def _n_gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    try:
        import datetime

        import torch
        import torch.distributed as dist

        import oracle
        from project_willamette_b200 import synth
        from project_willamette_b200.bitnet import BitNet
        from project_willamette_b200.tp import TPGroup

        torch.cuda.set_device(rank)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120))
        for ci, (name, kw) in enumerate(CASES):
            m = synth.bitnet_model(np.random.default_rng(700 + ci), **kw)
            c = m["config"]
            prompt = np.random.default_rng(ci).integers(0, c["vocab"], c["max_seq"] // 2)
            n_new = c["max_seq"] - len(prompt)
            g = TPGroup(rank, world, BitNet.tp_sym_bytes(m) + (1 << 20), device=rank)
            for exact in (False, True):
                eng = BitNet(m, exact=exact, tp=g)
                ids, hs = eng.generate(prompt, n_new, hiddens=True)
                ids2, hs2 = eng.generate(prompt, n_new, hiddens=True)  # graphs replayed
                eng.close()
                assert ids.tolist() == ids2.tolist() and np.array_equal(hs, hs2), f"{name} replay"
                if rank == 0:
                    ref = BitNet(m, exact=exact, device=rank)
                    want_ids, want_h = ref.generate(prompt, n_new, hiddens=True)
                    ref.close()
                    assert ids.tolist() == want_ids.tolist(), f"{name} exact={exact} ids"
                    assert np.array_equal(hs.view(np.uint32), want_h.view(np.uint32)), \
                        f"{name} exact={exact} hidden states differ from the single-GPU engine"
                    if exact:
                        o_ids = oracle.BitnetOracle(m).generate(prompt, n_new)
                        assert ids.tolist() == o_ids.tolist(), f"{name} oracle ids"
                dist.barrier()
            g.close()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc(limit=6)))


def test_tp_decode_matches_single_gpu():
    world = min(_n_gpus(), 8)
    if world < 2:
        pytest.skip("needs at least two GPUs")
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in procs:
            r, msg = q.get(timeout=600)
            results[r] = msg
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(results.get(r) == "ok" for r in range(world)), results
