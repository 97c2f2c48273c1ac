"""Tensor parallel on 2+ GPUs: one process per GPU, outputs gathered by the
library's own kernels over NVLink peer memory.

Each rank holds a row slice of every BitLinear and a vocab shard of the
Q6_K lm-head.  The gathered vectors (on every rank) and the greedy ids must
equal the single-GPU oracle bit for bit: a chain of three fused BitLinear
calls where each consumes the previous gathered output (in-kernel wait on
the arrival counters), a stream plan of row slices, and the vocab-sharded
head with ties across the shard boundary and a NaN logit at index 0.  The
whole sequence runs twice so counters and key-slot sets are reused.

Needs at least two GPUs; skipped otherwise (the host logic is covered on
CPU by test_tp_host.py).
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


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
        import ctypes
        import datetime

        import torch
        import torch.distributed as dist

        import oracle
        import project_willamette_b200 as wl
        from project_willamette_b200 import synth
        from project_willamette_b200._abi import WL_I2S_NO_CODE3, WlI2sStreamOp
        from project_willamette_b200.tp import TPGroup, shard_rows

        torch.cuda.set_device(rank)
        dev = f"cuda:{rank}"
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120))
        L = wl.lib()
        g = TPGroup(rank, world, 16 << 20, device=rank)
        stream = torch.cuda.current_stream().cuda_stream
        rng = np.random.default_rng(2024)  # identical data on every rank
        keep = []
        dummy = torch.zeros(64, dtype=torch.uint8, device=dev)

        def to_dev(a):
            t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
            keep.append(t)
            return t

        off = [0]

        def sym(n):
            v = g.view(off[0], n)
            off[0] += (n * 4 + 255) // 256 * 256
            return v

        def read(v):
            return torch.as_tensor(v, device=dev).cpu().numpy().copy()

        def slice_of(packed, K, N, align=1):
            r0, n = shard_rows(N, world, rank, align)
            rb = K // 4
            part = packed[r0 * rb:(r0 + n) * rb]
            has3 = bool(((part & (part >> 1)) & 0x55).any()) if n else False
            ptr = to_dev(part).data_ptr() if n else dummy.data_ptr()
            return r0, n, ptr, (0 if has3 else WL_I2S_NO_CODE3)

        def bitlinear(K, N, c3=0.0):
            return synth.i2s_packed(rng, K, N, c3), synth.i2s_scale(rng)

        # a decoder-layer-shaped chain: QKV (shared x) -> gate/up on Q -> down on gate
        x0 = synth.activations(rng, 2560)
        A = [bitlinear(2560, n, 0.001 if n == 640 else 0.0) for n in (2560, 640, 640)]
        B = [bitlinear(2560, 6912) for _ in range(2)]
        C_ = bitlinear(6912, 2560, 0.0005)
        yA = [sym(n) for n in (2560, 640, 640)]
        yB = [sym(6912) for _ in range(2)]
        yC = sym(2560)
        refA = [oracle.i2s_matvec_sse2_i8(p, s, 2560, n, x0)[0]
                for (p, s), n in zip(A, (2560, 640, 640))]
        refB = [oracle.i2s_matvec_sse2_i8(p, s, 2560, 6912, refA[0])[0] for p, s in B]
        refC = oracle.i2s_matvec_sse2_i8(C_[0], C_[1], 6912, 2560, refB[0])[0]
        sA = [slice_of(p, 2560, n) for (p, _), n in zip(A, (2560, 640, 640))]
        sB = [slice_of(p, 2560, 6912) for p, _ in B]
        sC = slice_of(C_[0], 6912, 2560)
        x0d = to_dev(x0)

        # stream plan over row slices (64-row units), local inputs
        x1 = synth.activations(rng, 2560)
        S = [bitlinear(2560, 2560), bitlinear(2560, 6912, 0.002), bitlinear(2560, 100)]
        yS = [sym(n) for n in (2560, 6912, 100)]
        refS = [oracle.i2s_matvec_sse2_i8(p, s, 2560, n, x1)[0]
                for (p, s), n in zip(S, (2560, 6912, 100))]
        x1d = to_dev(x1)
        ops = []
        for (p, s), n, y in zip(S, (2560, 6912, 100), yS):
            r0, cnt, ptr, fl = slice_of(p, 2560, n, 64)
            op = WlI2sStreamOp()
            op.packed, op.w_scale, op.in_dim, op.out_dim = ptr, s, 2560, cnt
            op.x, op.y, op.acc, op.flags, op.row_off = x1d.data_ptr(), y.ptr, None, fl, r0
            ops.append(op)
        plan = ctypes.c_void_p()
        arr = (WlI2sStreamOp * len(ops))(*ops)
        assert L.wl_i2s_stream_plan_create(arr, len(ops), ctypes.byref(plan)) == 0, \
            L.wl_last_error()

        # vocab-sharded lm-head: random rows, then planted ties and a NaN at 0
        n_embd, vocab, batch = 2560, 4099, 5
        RB = n_embd // 256 * 210  # Q6_K bytes per row; a row's first block at [0, 210)
        heads = []
        raw = synth.q6k_rows(rng, n_embd, vocab)
        heads.append(raw)
        tie = raw.reshape(vocab, RB).copy()
        tie[:] = tie[7]
        tie[vocab - 3, 192:208] = np.minimum(tie[vocab - 3, 192:208].astype(np.int16) + 1,
                                             127).astype(np.uint8)
        heads.append(tie.reshape(-1))          # equal rows but one, in the last shard
        tie2 = raw.reshape(vocab, RB).copy()
        tie2[:] = tie2[7]
        heads.append(tie2.reshape(-1))         # all equal: id 0
        nan0 = raw.reshape(vocab, RB).copy()
        nan0[0, 208:210] = np.frombuffer(np.float16(np.nan).tobytes(), np.uint8)
        heads.append(nan0.reshape(-1))
        H = synth.activations(rng, batch, n_embd)
        Hd = to_dev(H)
        v0, nv = shard_rows(vocab, world, rank)
        shards = []
        for hraw in heads:
            part = to_dev(hraw[v0 * RB:(v0 + nv) * RB])
            pk = torch.empty(max(L.wl_q6k_packed_bytes(n_embd, nv), 16), dtype=torch.uint8,
                             device=dev)
            keep.append(pk)
            assert L.wl_dev_q6k_repack(part.data_ptr(), n_embd, nv, pk.data_ptr(), stream) == 0
            want = []
            for b in range(batch):
                full = oracle.compute_logits(H[b], hraw, 14, n_embd, vocab, n_threads=0)
                want.append(oracle.argmax(full))
            shards.append((pk, want))
        scratch = torch.zeros(L.wl_q6k_scratch_bytes(batch) // 4 + 4, dtype=torch.int32,
                              device=dev)
        ids = torch.zeros(batch, dtype=torch.int32, device=dev)

        for it in range(2):
            g.i2s_matvec([(sA[j][2], A[j][1], sA[j][1], yA[j].ptr, sA[j][3]) for j in range(3)],
                         [sA[j][0] for j in range(3)], 2560, x0d.data_ptr(), False, stream)
            g.i2s_matvec([(sB[j][2], B[j][1], sB[j][1], yB[j].ptr, sB[j][3]) for j in range(2)],
                         [sB[j][0] for j in range(2)], 2560, yA[0].ptr, True, stream)
            g.i2s_matvec([(sC[2], C_[1], sC[1], yC.ptr, sC[3])], [sC[0]], 6912, yB[0].ptr, True,
                         stream)
            g.stream_run(plan, stream)
            g.wait(stream)
            torch.cuda.synchronize()
            for v, r, name in [(yA[0], refA[0], "qkv0"), (yA[1], refA[1], "qkv1"),
                               (yA[2], refA[2], "qkv2"), (yB[0], refB[0], "up0"),
                               (yB[1], refB[1], "up1"), (yC, refC, "down"),
                               (yS[0], refS[0], "s0"), (yS[1], refS[1], "s1"),
                               (yS[2], refS[2], "s2")]:
                got = read(v)
                assert np.array_equal(got.view(np.uint32), r.view(np.uint32)), (it, name)
            for hi, (pk, want) in enumerate(shards):
                g.lm_head_greedy(pk.data_ptr(), n_embd, nv, v0, Hd.data_ptr(), batch,
                                 ids.data_ptr(), scratch.data_ptr(), stream)
                torch.cuda.synchronize()
                assert ids.cpu().tolist() == want, (it, hi, ids.cpu().tolist(), want)
            flags = ctypes.c_uint32(0)
            assert L.wl_device_status(ctypes.byref(flags)) == 0 and flags.value == 0, flags.value

        # The same chain and head captured once in a CUDA graph and replayed
        # with fresh inputs: wait targets and key sets are read on the device,
        # so replays need no host bookkeeping.
        side = torch.cuda.Stream(device=dev)
        graph = torch.cuda.CUDAGraph()
        dist.barrier()
        with torch.cuda.stream(side):
            with torch.cuda.graph(graph, stream=side):
                h = torch.cuda.current_stream().cuda_stream
                g.i2s_matvec([(sA[j][2], A[j][1], sA[j][1], yA[j].ptr, sA[j][3])
                              for j in range(3)], [sA[j][0] for j in range(3)], 2560,
                             x0d.data_ptr(), True, h)
                g.i2s_matvec([(sB[j][2], B[j][1], sB[j][1], yB[j].ptr, sB[j][3])
                              for j in range(2)], [sB[j][0] for j in range(2)], 2560,
                             yA[0].ptr, True, h)
                g.i2s_matvec([(sC[2], C_[1], sC[1], yC.ptr, sC[3])], [sC[0]], 6912, yB[0].ptr,
                             True, h)
                g.lm_head_greedy(shards[0][0].data_ptr(), n_embd, nv, v0, Hd.data_ptr(), batch,
                                 ids.data_ptr(), scratch.data_ptr(), h)
                g.wait(h)
        grng = np.random.default_rng(555)  # same on every rank
        for rep in range(3):
            xr = synth.activations(grng, 2560)
            Hr = synth.activations(grng, batch, n_embd)
            x0d.copy_(torch.from_numpy(xr))
            Hd.copy_(torch.from_numpy(Hr))
            torch.cuda.synchronize()
            dist.barrier()  # every rank's inputs are in place before any replay
            graph.replay()
            torch.cuda.synchronize()
            ra = oracle.i2s_matvec_sse2_i8(A[0][0], A[0][1], 2560, 2560, xr)[0]
            rb = oracle.i2s_matvec_sse2_i8(B[0][0], B[0][1], 2560, 6912, ra)[0]
            rc = oracle.i2s_matvec_sse2_i8(C_[0], C_[1], 6912, 2560, rb)[0]
            assert np.array_equal(read(yC).view(np.uint32), rc.view(np.uint32)), ("graph", rep)
            want = [oracle.argmax(oracle.compute_logits(Hr[b], heads[0], 14, n_embd, vocab,
                                                        n_threads=0)) for b in range(batch)]
            assert ids.cpu().tolist() == want, ("graph ids", rep)
        flags = ctypes.c_uint32(0)
        assert L.wl_device_status(ctypes.byref(flags)) == 0 and flags.value == 0, flags.value
        del graph
        dist.barrier()
        L.wl_i2s_stream_plan_destroy(plan)
        g.close()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:
        import traceback
        q.put((rank, traceback.format_exc(limit=6)))


def test_tp_gathered_chain_stream_and_lm_head():
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
