"""Tensor-parallel host logic on CPU: world-size-2 ``gloo`` ranks.

Each rank computes its row slice of a BitLinear and its vocab shard of the
lm-head with the oracle, then the ranks exchange (all-gather of y, all-gather
of per-shard argmax keys).  The gathered results must equal the single-rank
oracle exactly: the row split is exact (rows are independent dots,
bitlinear_sse2.rs:313-342) and the key reduction reproduces the reference's
first-maximum scan with its NaN rule (lm_head.rs:161-176).
"""
import os
import socket

import numpy as np
import pytest

from project_willamette_b200 import synth
from project_willamette_b200.tp import decode_key, order_keys, reduce_keys, shard_rows


def test_shard_rows_cover_exactly():
    for n in (0, 1, 5, 63, 64, 65, 640, 2560, 6912, 128256):
        for world in (1, 2, 3, 4, 8):
            for align in (1, 64):
                covered, nxt = 0, 0
                for r in range(world):
                    b, c = shard_rows(n, world, r, align)
                    assert b == nxt and c >= 0
                    if b + c < n:
                        assert c % align == 0
                    nxt, covered = b + c, covered + c
                assert covered == n and nxt == n
    with pytest.raises(ValueError):
        shard_rows(10, 2, 2)


def test_order_keys_match_oracle_argmax(oracle):
    rng = np.random.default_rng(3)
    cases = [rng.standard_normal(1000).astype(np.float32),
             np.array([np.nan, 5.0, 7.0], np.float32),         # NaN at 0 -> 0
             np.array([1.0, np.nan, 7.0, np.nan], np.float32),  # NaN elsewhere ignored
             np.array([-0.0, 0.0, -1.0], np.float32),           # -0 ties +0 -> 0
             np.array([-1.0, -0.0, 0.0], np.float32),
             np.array([3.0, 9.0, 9.0, 1.0], np.float32),        # first max
             np.array([-np.inf, -np.inf], np.float32),
             np.array([np.inf, np.inf, 1.0], np.float32),
             np.full(7, np.nan, np.float32)]
    for v in cases:
        assert decode_key(reduce_keys(order_keys(v))) == oracle.argmax(v), v


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, q):
    try:
        import torch
        import torch.distributed as dist
        import oracle
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=__import__("datetime").timedelta(seconds=60))
        rng = np.random.default_rng(77)  # same data on every rank
        # BitLinear row split + all-gather of y
        for K, N in ((2560, 640), (512, 65), (128, 1)):
            packed = synth.i2s_packed(rng, K, N, 0.01)
            scale = synth.i2s_scale(rng)
            x = synth.activations(rng, K)
            r0, n = shard_rows(N, world, rank, 64)
            rb = K // 4
            ys = oracle.i2s_matvec_sse2_i8(packed[r0 * rb:(r0 + n) * rb].copy(), scale, K, n, x)[0]
            parts = [None] * world
            dist.all_gather_object(parts, ys.tobytes())
            y = np.frombuffer(b"".join(parts), np.float32)
            want = oracle.i2s_matvec_sse2_i8(packed, scale, K, N, x)[0]
            assert np.array_equal(y.view(np.uint32), want.view(np.uint32)), (K, N)
        # lm-head vocab shards + key reduction (all-reduce MAX on the keys)
        n_embd = 256
        for vocab, plant in ((3001, None), (1, None), (777, "tie"), (777, "nan0"), (900, "nanmid")):
            raw = synth.q6k_rows(rng, n_embd, vocab)
            if plant:
                blk = raw.reshape(vocab, 210)
                if plant == "tie":  # equal rows straddle the shard boundary
                    blk[:] = blk[5]
                elif plant == "nan0":
                    blk[0, 208:210] = np.frombuffer(np.float16(np.nan).tobytes(), np.uint8)
                else:
                    blk[450, 208:210] = np.frombuffer(np.float16(np.nan).tobytes(), np.uint8)
                raw = blk.reshape(-1)
            h = synth.activations(rng, n_embd)
            v0, nv = shard_rows(vocab, world, rank)
            key = 0
            if nv:
                part = raw[v0 * 210:(v0 + nv) * 210].copy()
                logits = oracle.compute_logits(h, part, 14, n_embd, nv, n_threads=1)
                key = reduce_keys(order_keys(logits, v0))
            # u64 keys do not fit torch's signed MAX all-reduce; gather instead
            keys = [None] * world
            dist.all_gather_object(keys, key)
            got = decode_key(reduce_keys(keys))
            full = oracle.compute_logits(h, raw, 14, n_embd, vocab, n_threads=1)
            assert got == oracle.argmax(full), (vocab, plant, got)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, repr(e)))


def test_tp_split_and_reduce_gloo_world2():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in procs:
            r, msg = q.get(timeout=240)
            results[r] = msg
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert results == {0: "ok", 1: "ok"}, results


# ---- group setup when a peer fails: the library's group calls are faked on
# the host (no GPU); the group must be destroyed before the error propagates.
class _FakeTpLib:
    """The TP entry points of the library, answering without a device."""
    GROUP = 0xB200

    def __init__(self, connect_rc=0):
        self.connect_rc, self.calls = connect_rc, []

    def wl_init(self, device):
        self.calls.append(("init", device))
        return 0

    def wl_tp_create(self, rank, world, sym_bytes, group_ref, handle):
        group_ref._obj.value = self.GROUP
        for i in range(len(handle)):
            handle[i] = rank + 1
        self.calls.append(("create", rank, world))
        return 0

    def wl_tp_connect(self, group, handles):
        self.calls.append(("connect", bytes(handles)))
        return self.connect_rc

    def wl_tp_destroy(self, group):
        self.calls.append(("destroy", group.value))
        return 0

    def wl_last_error(self):
        return b"opening rank 1's block: fake failure"

    def wl_last_error_tensor_type(self):
        return 0


@pytest.fixture
def fake_tp(monkeypatch):
    from project_willamette_b200 import tp

    def make(connect_rc=0):
        fake = _FakeTpLib(connect_rc)
        monkeypatch.setattr(tp, "lib", lambda: fake)
        return fake
    return make


def _destroys(fake):
    return [c for c in fake.calls if c[0] == "destroy"]


def test_group_freed_when_a_peer_never_joins(fake_tp):
    from project_willamette_b200.tp import TPGroup

    fake = fake_tp()

    def exchange(handle, world):
        raise TimeoutError("rank 1 never joined the handle exchange")
    with pytest.raises(TimeoutError):
        TPGroup(0, 2, 4096, device=0, exchange=exchange)
    assert _destroys(fake) == [("destroy", _FakeTpLib.GROUP)]
    assert not any(c[0] == "connect" for c in fake.calls)


def test_group_freed_on_a_malformed_exchange(fake_tp):
    from project_willamette_b200 import WillametteError
    from project_willamette_b200.tp import TPGroup

    fake = fake_tp()
    with pytest.raises(WillametteError) as e:
        TPGroup(0, 2, 4096, device=0, exchange=lambda h, w: [h])  # one handle for two ranks
    assert e.value.status == 8 and "wrong shape" in e.value.message
    assert _destroys(fake) == [("destroy", _FakeTpLib.GROUP)]


def test_group_freed_when_mapping_a_peer_fails(fake_tp):
    from project_willamette_b200 import WillametteError
    from project_willamette_b200.tp import TPGroup

    fake = fake_tp(connect_rc=8)  # WL_ERR_COMM from wl_tp_connect
    with pytest.raises(WillametteError) as e:
        TPGroup(1, 2, 4096, device=0, exchange=lambda h, w: [bytes([1]) * len(h), h])
    assert e.value.status == 8 and "fake failure" in e.value.message
    assert _destroys(fake) == [("destroy", _FakeTpLib.GROUP)]


def test_group_connects_and_closes_once(fake_tp):
    from project_willamette_b200.tp import TPGroup

    fake = fake_tp()
    g = TPGroup(1, 2, 4096, device=0, exchange=lambda h, w: [bytes([1]) * len(h), h])
    connect = [c for c in fake.calls if c[0] == "connect"]
    assert len(connect) == 1 and connect[0][1] == bytes([1]) * 64 + bytes([2]) * 64
    assert not _destroys(fake)
    g.close()
    g.close()
    assert _destroys(fake) == [("destroy", _FakeTpLib.GROUP)]


def _dead_peer_main(rank, port, q):
    """Rank 1 joins the process group and exits before the handle exchange;
    rank 0 must get an error from the exchange, not wait for good, and free
    its group."""
    try:
        import datetime

        import torch.distributed as dist
        from project_willamette_b200 import tp
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=2,
                                timeout=datetime.timedelta(seconds=10))
        if rank == 1:
            q.put((rank, "left"))
            q.close()
            q.join_thread()  # flush the message before the hard exit
            os._exit(0)  # dies between steps, with nothing in flight
        fake = _FakeTpLib()
        tp.lib = lambda: fake
        try:
            tp.TPGroup(0, 2, 4096, device=0)
            q.put((rank, "exchange returned without the peer"))
        except Exception as e:  # the exchange's own error
            ok = _destroys(fake) == [("destroy", _FakeTpLib.GROUP)]
            q.put((rank, "raised+freed" if ok else f"raised, not freed: {e!r}"))
        q.close()
        q.join_thread()
        os._exit(0)  # the group is broken; skip its teardown
    except Exception as e:
        q.put((rank, repr(e)))


def test_handle_exchange_errors_when_a_rank_leaves_gloo_world2():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dead_peer_main, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in procs:
            try:
                r, msg = q.get(timeout=90)
            except Exception:
                break  # reported below with what did arrive
            results[r] = msg
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert results == {0: "raised+freed", 1: "left"}, results
