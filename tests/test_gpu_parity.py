"""GPU parity: the CUDA library, called through its C ABI, against the oracle.

Bar (north star): int32 accumulators and greedy token ids bit-exact; f32
outputs within 1e-5 relative.  Every kernel here reproduces the reference's
own x86 arithmetic, so the f32 outputs are compared bit for bit (NaN
positions must agree; NaN payloads are not compared).
"""
import numpy as np
import pytest

import oracle
import project_willamette_b200 as wl
from project_willamette_b200 import GgmlType, TensorView, synth
from project_willamette_b200._abi import WLStatus

pytestmark = pytest.mark.gpu

RTOL = 1e-5  # the north-star tolerance for f32 outputs (bit-exact is asserted first)


def assert_bitexact(got, want, what=""):
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    assert got.shape == want.shape, what
    gn, wn = np.isnan(got), np.isnan(want)
    assert np.array_equal(gn, wn), f"{what}: NaN positions differ"
    g, w = got[~gn], want[~wn]
    if not np.array_equal(g.view(np.uint32), w.view(np.uint32)):
        bad = np.flatnonzero(g.view(np.uint32) != w.view(np.uint32))
        rel = np.max(np.abs(g[bad] - w[bad]) / np.maximum(np.abs(w[bad]), 1e-30))
        raise AssertionError(f"{what}: {bad.size} values differ (first {bad[:5]}), max rel {rel:g}"
                             f" (tolerance {RTOL})")


def _i2s_case(rng, in_dim, out_dim, code3=0.0, x=None):
    packed = synth.i2s_packed(rng, in_dim, out_dim, code3)
    scale = synth.i2s_scale(rng)
    if x is None:
        x = synth.activations(rng, in_dim)
    return TensorView.i2s(f"w{in_dim}x{out_dim}", in_dim, out_dim, packed, scale), packed, scale, x


def _check_i2s(t, packed, scale, x):
    in_dim, out_dim = t.shape
    y, acc, s, q = wl.bitlinear_i2s_matvec_f32_dbg(t, x)
    ry, racc, rs, rq = oracle.i2s_matvec_sse2_i8(packed, scale, in_dim, out_dim, x)
    assert np.array_equal(q, rq), "quantised activations differ"
    assert_bitexact([s], [rs], "activation scale")
    assert np.array_equal(acc, racc), "int32 accumulators differ"
    assert_bitexact(y, ry, "output")
    y2 = np.zeros(out_dim, np.float32)
    wl.bitlinear_i2s_matvec_f32(t, x, y2)
    assert_bitexact(y2, ry, "output (plain entry point)")


def test_i2s_config1_bit_exact():
    """Benchmark config 1: 6912 x 2560 ternary, P(0)=0.5, scale U[0.01,0.1], x N(0,1)."""
    rng = np.random.default_rng(0x5EED + 1)
    _check_i2s(*_i2s_case(rng, 2560, 6912))


@pytest.mark.parametrize("in_dim", [128, 256, 640, 1024, 2560, 4096, 6912, 12288, 20480])
@pytest.mark.parametrize("out_dim", [1, 31, 33, 640, 2560])
def test_i2s_fuzz_shapes(in_dim, out_dim):
    rng = np.random.default_rng(in_dim * 7919 + out_dim)
    _check_i2s(*_i2s_case(rng, in_dim, out_dim, code3=0.02 if out_dim % 2 else 0.0))


@pytest.mark.parametrize("kind", ["zeros", "outlier", "nan", "inf", "neg_zero", "tiny", "ties",
                                  "round_edges"])
def test_i2s_activation_edge_cases(kind):
    rng = np.random.default_rng(42)
    in_dim, out_dim = 768, 97
    x = synth.activations(rng, in_dim)
    if kind == "zeros":
        x[:] = 0
    elif kind == "outlier":
        x[17] = 1e6
    elif kind == "nan":
        x[5] = np.nan
        x[700] = np.nan
    elif kind == "inf":
        x[3] = np.inf
    elif kind == "neg_zero":
        x[:] = -0.0
        x[9] = -0.0
    elif kind == "tiny":
        x *= np.float32(1e-38)
    elif kind == "ties":  # values landing exactly on .5 after scaling
        x = (np.arange(in_dim, dtype=np.float32) % 255 - 127) / np.float32(2.0)
        x[0] = 127.0
    elif kind == "round_edges":
        # max |x| = 127 makes the scale exactly 1, so each x is rounded as is:
        # every k + 0.5 (k = 0..126) and its two float neighbours, both signs
        h = np.arange(127, dtype=np.float32) + np.float32(0.5)
        e = np.concatenate([np.nextafter(h, np.float32(0)), h, np.nextafter(h, np.float32(200))])
        x = np.zeros(in_dim, np.float32)
        x[0] = 127.0
        x[1:1 + e.size] = e
        x[1 + e.size:1 + 2 * e.size] = -e
    _check_i2s(*_i2s_case(rng, in_dim, out_dim, code3=0.01, x=x))


def test_i2s_all_codes_three():
    """Code 0b11 maps to 0 (bitlinear.rs:48): an all-0xFF tensor gives exactly 0."""
    t = TensorView.i2s("c3", 256, 5, np.full(5 * 64, 0xFF, np.uint8), 0.5)
    y, acc, _, _ = wl.bitlinear_i2s_matvec_f32_dbg(t, np.linspace(-3, 3, 256))
    assert np.all(acc == 0) and np.all(y == 0.0)


def test_i2s_kats_on_gpu(kats):
    for c in kats:
        if c["op"] not in ("i2s_matvec", "i2s_deterministic"):
            continue
        packed = np.frombuffer(bytes.fromhex(c["packed"]), np.uint8)
        t = TensorView.i2s(c["id"], c["in_dim"], c["out_dim"], packed, c["scale"])
        y, acc, s, q = wl.bitlinear_i2s_matvec_f32_dbg(t, c["x"])
        ry, racc, rs, rq = oracle.i2s_matvec_sse2_i8(packed, c["scale"], c["in_dim"],
                                                     c["out_dim"], c["x"])
        assert np.array_equal(acc, racc), c["id"]
        assert_bitexact(y, ry, c["id"])
        if c["op"] == "i2s_matvec" and c["path"] == "dispatch":
            np.testing.assert_allclose(y, c["expect"], atol=c["tol_abs"], rtol=0, err_msg=c["id"])


def test_i2s_column_stride_mapping_exact():
    """bitlinear.rs:430-465 with activations that quantise exactly (max 127):
    byte 0x86 -> +1@0, -1@32, 0@64, +1@96."""
    packed = np.full(32, 0x55, np.uint8)
    packed[0] = 0x86
    x = np.zeros(128, np.float32)
    x[0], x[32], x[64], x[96] = 1.0, 10.0, 100.0, 127.0
    t = TensorView.i2s("map", 128, 1, packed, 1.0)
    y, acc, s, q = wl.bitlinear_i2s_matvec_f32_dbg(t, x)
    assert acc[0] == 1 - 10 + 127 and y[0] == 118.0 and s == 1.0


def test_i2s_gemm_rows_match_per_token_matvec():
    rng = np.random.default_rng(3)
    in_dim, out_dim, m = 2560, 640, 7
    packed = synth.i2s_packed(rng, in_dim, out_dim)
    scale = synth.i2s_scale(rng)
    X = synth.activations(rng, m, in_dim)
    X[2] = 0.0
    t = TensorView.i2s("g", in_dim, out_dim, packed, scale)
    Y, acc = wl.bitlinear_i2s_gemm_f32(t, X, with_acc=True)
    RY, racc, _ = oracle.i2s_gemm_rows(packed, scale, in_dim, out_dim, X)
    assert np.array_equal(acc, racc)
    assert_bitexact(Y, RY, "gemm")


@pytest.mark.parametrize("in_dim,out_dim,m", [(2560, 2560, 16), (2560, 640, 33), (640, 1000, 128),
                                              (512, 64, 200), (6912, 2560, 130),
                                              (2560, 6912, 256), (128, 3, 40)])
def test_i2s_gemm_tensor_core_bit_exact(in_dim, out_dim, m):
    """Prefill (>= 16 tokens, code-3-free weights) runs as one tcgen05 GEMM;
    every token must match the reference's per-token matvec bit for bit."""
    rng = np.random.default_rng(in_dim + out_dim + m)
    packed = synth.i2s_packed(rng, in_dim, out_dim)
    scale = synth.i2s_scale(rng)
    X = synth.activations(rng, m, in_dim)
    X[1] = 0.0
    X[m // 2, 7] = 1e5
    t = TensorView.i2s("gemm", in_dim, out_dim, packed, scale)
    Y, acc = wl.bitlinear_i2s_gemm_f32(t, X, with_acc=True)
    RY, racc, _ = oracle.i2s_gemm_rows(packed, scale, in_dim, out_dim, X, n_threads=0)
    assert np.array_equal(acc, racc)
    assert_bitexact(Y, RY, "tcgen05 gemm")


def test_i2s_gemm_with_code3_falls_back_exactly():
    rng = np.random.default_rng(8)
    in_dim, out_dim, m = 1024, 300, 48
    packed = synth.i2s_packed(rng, in_dim, out_dim, code3_fraction=0.01)
    scale = synth.i2s_scale(rng)
    X = synth.activations(rng, m, in_dim)
    Y, acc = wl.bitlinear_i2s_gemm_f32(TensorView.i2s("g3", in_dim, out_dim, packed, scale), X,
                                       with_acc=True)
    RY, racc, _ = oracle.i2s_gemm_rows(packed, scale, in_dim, out_dim, X, n_threads=0)
    assert np.array_equal(acc, racc)
    assert_bitexact(Y, RY, "gemm code-3 fallback")


def test_i2s_gemm_config3_full_size_sampled():
    """Benchmark config 3 at M = 2048 for the 6912 x 2560 weight: all rows
    checked against the oracle on a sample of tokens, plus y(-X) = -y(X)."""
    rng = np.random.default_rng(0x5EED + 3)
    in_dim, out_dim, m = 2560, 6912, 2048
    packed = synth.i2s_packed(rng, in_dim, out_dim)
    scale = synth.i2s_scale(rng)
    X = synth.activations(rng, m, in_dim)
    t = TensorView.i2s("cfg3", in_dim, out_dim, packed, scale)
    Y, acc = wl.bitlinear_i2s_gemm_f32(t, X, with_acc=True)
    sample = np.array([0, 1, 127, 128, 1000, 2047])
    RY, racc, _ = oracle.i2s_gemm_rows(packed, scale, in_dim, out_dim, X[sample], n_threads=0)
    assert np.array_equal(acc[sample], racc)
    assert_bitexact(Y[sample], RY, "config 3 sample")
    Yn, accn = wl.bitlinear_i2s_gemm_f32(t, -X, with_acc=True)
    assert np.array_equal(accn, -acc)


def test_i2s_dev_fused_weights_match_separate():
    """One launch over Q/K/V-shaped weights sharing one quantised input."""
    import torch
    rng = np.random.default_rng(11)
    K = 2560
    shapes = [2560, 640, 640]
    x = synth.activations(rng, K)
    ws = [(synth.i2s_packed(rng, K, n), synth.i2s_scale(rng), n) for n in shapes]
    dev = torch.device("cuda")
    xd = torch.from_numpy(x).to(dev)
    q = torch.empty(K, dtype=torch.int8, device=dev)
    sc = torch.empty(1, dtype=torch.float32, device=dev)
    packs = [torch.from_numpy(p).to(dev) for p, _, _ in ws]
    ys = [torch.empty(n, dtype=torch.float32, device=dev) for n in shapes]
    accs = [torch.empty(n, dtype=torch.int32, device=dev) for n in shapes]
    L = wl.lib()
    stream = torch.cuda.current_stream().cuda_stream
    assert L.wl_dev_quantize_absmax_i8(xd.data_ptr(), K, 1, q.data_ptr(), sc.data_ptr(), stream) == 0
    arr = (wl._abi.WlI2sDevWeight * 3)()
    for i, ((p, s, n), pd, yd, ad) in enumerate(zip(ws, packs, ys, accs)):
        arr[i].packed, arr[i].w_scale, arr[i].out_dim = pd.data_ptr(), s, n
        arr[i].y, arr[i].acc = yd.data_ptr(), ad.data_ptr()
    assert L.wl_dev_i2s_matvec(arr, 3, K, q.data_ptr(), sc.data_ptr(), stream) == 0
    torch.cuda.synchronize()
    for (p, s, n), yd, ad in zip(ws, ys, accs):
        ry, racc, _, _ = oracle.i2s_matvec_sse2_i8(p, s, K, n, x)
        assert np.array_equal(ad.cpu().numpy(), racc)
        assert_bitexact(yd.cpu().numpy(), ry, "fused")


def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda")


def test_i2s_fused_input_and_code3_scan():
    """wl_dev_i2s_matvec_fused_f32 (in-kernel quantisation) over Q/K/V- and
    gate/up-shaped groups, with and without the no-code-3 fast path."""
    import torch
    L = wl.lib()
    rng = np.random.default_rng(12)
    stream = torch.cuda.current_stream().cuda_stream
    found = torch.zeros(1, dtype=torch.int32, device="cuda")
    for K, shapes, c3 in [(2560, [2560, 640, 640], 0.0), (2560, [6912, 6912], 0.001),
                          (6912, [2560], 0.0), (128, [3, 5], 0.05), (8192, [33], 0.0)]:
        x = synth.activations(rng, K)
        ws = [(synth.i2s_packed(rng, K, n, c3), synth.i2s_scale(rng), n) for n in shapes]
        arr = (wl._abi.WlI2sDevWeight * len(ws))()
        keep = []
        for i, (p, s, n) in enumerate(ws):
            pd = _dev(torch, p)
            assert L.wl_dev_i2s_scan_code3(pd.data_ptr(), pd.numel(), found.data_ptr(), stream) == 0
            torch.cuda.synchronize()
            has3 = bool(((p & (p >> 1)) & 0x55).any())
            assert int(found.item()) == int(has3)
            yd = torch.empty(n, dtype=torch.float32, device="cuda")
            ad = torch.empty(n, dtype=torch.int32, device="cuda")
            keep += [pd, yd, ad]
            arr[i].packed, arr[i].w_scale, arr[i].out_dim = pd.data_ptr(), s, n
            arr[i].y, arr[i].acc = yd.data_ptr(), ad.data_ptr()
            arr[i].flags = 0 if has3 else wl._abi.WL_I2S_NO_CODE3
        xd = _dev(torch, x)
        assert L.wl_dev_i2s_matvec_fused_f32(arr, len(ws), K, xd.data_ptr(), stream) == 0
        torch.cuda.synchronize()
        for i, (p, s, n) in enumerate(ws):
            ry, racc, _, _ = oracle.i2s_matvec_sse2_i8(p, s, K, n, x)
            yd, ad = keep[3 * i + 1], keep[3 * i + 2]
            assert np.array_equal(ad.cpu().numpy(), racc), (K, n)
            assert_bitexact(yd.cpu().numpy(), ry, f"fused {K}x{n}")


def test_i2s_stream_plan_block_mode_bit_exact():
    """A plan large enough that each CTA owns more than 64 row blocks, so the
    streaming kernel deals whole blocks to its warps dynamically (5, 2 and 1
    boxes per block mixed), bit-exact against the oracle, run twice."""
    import ctypes
    import torch
    L = wl.lib()
    rng = np.random.default_rng(4242)
    specs = [(512, 300000), (2560, 150000), (1024, 200003)]
    ops, keep, ref = [], [], []
    for K, N in specs:
        x = synth.activations(rng, K)
        p = synth.i2s_packed(rng, K, N)
        s = synth.i2s_scale(rng)
        pd, xd = _dev(torch, p), _dev(torch, x)
        yd = torch.full((N,), float("nan"), dtype=torch.float32, device="cuda")
        keep += [pd, xd, yd]
        op = wl._abi.WlI2sStreamOp()
        op.packed, op.w_scale, op.in_dim, op.out_dim = pd.data_ptr(), s, K, N
        op.x, op.y, op.acc, op.flags = xd.data_ptr(), yd.data_ptr(), None, 0
        ops.append(op)
        ref.append((yd, oracle.i2s_matvec_sse2_i8(p, s, K, N, x)[0]))
    blocks = sum((N + 63) // 64 for _, N in specs)
    assert blocks > 64 * 148  # block mode on a 148-SM B200
    arr = (wl._abi.WlI2sStreamOp * len(ops))(*ops)
    plan = ctypes.c_void_p()
    assert L.wl_i2s_stream_plan_create(arr, len(ops), ctypes.byref(plan)) == 0, L.wl_last_error()
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        for yd, _r in ref:
            yd.fill_(float("nan"))
        assert L.wl_dev_i2s_stream_run(plan, stream) == 0
        torch.cuda.synchronize()
        for yd, ry in ref:
            assert_bitexact(yd.cpu().numpy(), ry, "stream block mode")
    assert L.wl_i2s_stream_plan_destroy(plan) == 0


@pytest.mark.parametrize("with_code3", [False, True])
def test_i2s_stream_plan_bit_exact(with_code3):
    """Many independent matvecs (mixed in_dim, shared and distinct inputs,
    tiny and large ops) in one persistent launch, run twice."""
    import ctypes
    import torch
    L = wl.lib()
    rng = np.random.default_rng(99 + with_code3)
    specs = [(2560, 2560, 0), (2560, 640, 0), (2560, 640, 0), (6912, 2560, 1), (512, 1, 2),
             (2560, 6912, 3), (2560, 6912, 3), (640, 37, 4), (6912, 100, 5), (7168, 300, 6),
             (12288, 45, 7), (2560, 0, 0), (1024, 64, 8)]
    xs = {}
    ops, keep, ref = [], [], []
    for K, N, xi in specs:
        if xi not in xs:
            xs[xi] = synth.activations(rng, K)
        p = synth.i2s_packed(rng, K, N, 0.002 if (with_code3 and N == 37) else 0.0)
        if N == 0:
            p = np.zeros(16, np.uint8)
        s = synth.i2s_scale(rng)
        pd, xd = _dev(torch, p), _dev(torch, xs[xi])
        yd = torch.full((N,), float("nan"), dtype=torch.float32, device="cuda")
        ad = torch.empty(N, dtype=torch.int32, device="cuda")
        keep += [pd, xd, yd, ad]
        op = wl._abi.WlI2sStreamOp()
        op.packed, op.w_scale, op.in_dim, op.out_dim = pd.data_ptr(), s, K, N
        op.x, op.y, op.acc, op.flags = xd.data_ptr(), yd.data_ptr(), ad.data_ptr(), 0
        ops.append(op)
        ref.append((yd, ad) + oracle.i2s_matvec_sse2_i8(p, s, K, N, xs[xi])[:2])
    arr = (wl._abi.WlI2sStreamOp * len(ops))(*ops)
    plan = ctypes.c_void_p()
    assert L.wl_i2s_stream_plan_create(arr, len(ops), ctypes.byref(plan)) == 0, L.wl_last_error()
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        assert L.wl_dev_i2s_stream_run(plan, stream) == 0
        torch.cuda.synchronize()
        for yd, ad, ry, racc in ref:
            assert np.array_equal(ad.cpu().numpy(), racc)
            assert_bitexact(yd.cpu().numpy(), ry, "stream")
    assert L.wl_i2s_stream_plan_destroy(plan) == 0


def test_i2s_properties_full_size():
    """Size-independent properties at the BitNet-2B shapes: y(-x) = -y(x)
    (round-half-away-from-zero is odd), y(2^k x) = 2^k y(x) exactly."""
    rng = np.random.default_rng(5)
    for in_dim, out_dim in [(2560, 6912), (6912, 2560)]:
        t, packed, scale, x = _i2s_case(rng, in_dim, out_dim)
        y, acc, s, q = wl.bitlinear_i2s_matvec_f32_dbg(t, x)
        yn, accn, sn, qn = wl.bitlinear_i2s_matvec_f32_dbg(t, -x)
        assert np.array_equal(accn, -acc) and np.array_equal(qn, -q) and sn == s
        y8, acc8, s8, q8 = wl.bitlinear_i2s_matvec_f32_dbg(t, x * np.float32(8.0))
        assert np.array_equal(acc8, acc) and s8 == s * 8
        assert_bitexact(y8, y * np.float32(8.0), "power-of-two scaling")


# ----------------------------------------------------------------- Q6_K lm-head

def _q6k(rng, n_embd, vocab):
    raw = synth.q6k_rows(rng, n_embd, vocab)
    return TensorView("token_embd.weight", [n_embd, vocab], GgmlType.Q6K, raw), raw


@pytest.mark.parametrize("n_embd,vocab", [(256, 1), (512, 1000), (2560, 3001), (2560, 16032)])
def test_q6k_logits_bit_exact(n_embd, vocab):
    rng = np.random.default_rng(n_embd + vocab)
    t, raw = _q6k(rng, n_embd, vocab)
    h = synth.activations(rng, n_embd)
    got = wl.compute_logits(h, t, n_embd, vocab)
    want = oracle.compute_logits(h, raw, 14, n_embd, vocab)
    assert_bitexact(got, want, "Q6_K logits")
    ids = wl.lm_head_greedy(h, t, n_embd, vocab)
    assert ids[0] == oracle.argmax(want)


@pytest.mark.parametrize("batch", [1, 2, 4, 5, 9])
def test_q6k_greedy_batch(batch):
    rng = np.random.default_rng(100 + batch)
    n_embd, vocab = 2560, 4099
    t, raw = _q6k(rng, n_embd, vocab)
    H = synth.activations(rng, batch, n_embd)
    ids, logits = wl.lm_head_greedy(H, t, n_embd, vocab, return_logits=True)
    for b in range(batch):
        want = oracle.compute_logits(H[b], raw, 14, n_embd, vocab)
        assert_bitexact(logits[b], want, f"batch row {b}")
        assert ids[b] == oracle.argmax(want), b


def test_q6k_config4_full_vocab():
    """Benchmark config 4 at full size: 128256 x 2560 Q6_K, batch 1, and a
    batch-64 call (one launch: every hidden row against each weight chunk)
    with all 64 logit rows bit for bit and every id."""
    rng = np.random.default_rng(0x5EED + 4)
    n_embd, vocab = 2560, 128256
    t, raw = _q6k(rng, n_embd, vocab)
    h = synth.activations(rng, n_embd)
    want = oracle.compute_logits(h, raw, 14, n_embd, vocab)
    got = wl.compute_logits(h, t, n_embd, vocab)
    assert_bitexact(got, want, "full-vocab logits")
    assert int(wl.lm_head_greedy(h, t, n_embd, vocab)[0]) == oracle.argmax(want)
    H = synth.activations(rng, 64, n_embd)
    ids, logits = wl.lm_head_greedy(H, t, n_embd, vocab, return_logits=True)
    for b in range(64):
        ref = oracle.compute_logits(H[b], raw, 14, n_embd, vocab)
        assert_bitexact(logits[b], ref, f"batch-64 row {b}")
        assert ids[b] == oracle.argmax(ref), b


def test_q6k_argmax_ties_and_nan():
    """All-equal rows tie -> id 0; the strict '>' scan keeps the first max."""
    n_embd, vocab = 256, 777
    blk = np.zeros(210, np.uint8)
    blk[:128] = 0x11
    blk[128:192] = 0xAA
    blk[192:208] = 1
    blk[208:210] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)
    raw = np.tile(blk, vocab)
    t = TensorView("tied", [n_embd, vocab], GgmlType.Q6K, raw)
    h = np.ones(n_embd, np.float32)
    ids, logits = wl.lm_head_greedy(h, t, n_embd, vocab, return_logits=True)
    assert ids[0] == 0 and np.all(logits == logits[0, 0])
    raw2 = raw.copy().reshape(vocab, 210)
    raw2[500, 192:208] = 2  # one row doubles
    raw2[600, 192:208] = 2  # a later equal row must not win
    t2 = TensorView("tied2", [n_embd, vocab], GgmlType.Q6K, raw2.reshape(-1))
    assert wl.lm_head_greedy(h, t2, n_embd, vocab)[0] == 500
    raw3 = raw2.copy()
    raw3[0, 208:210] = np.frombuffer(np.float16(np.nan).tobytes(), np.uint8)
    t3 = TensorView("nan0", [n_embd, vocab], GgmlType.Q6K, raw3.reshape(-1))
    want = oracle.compute_logits(h, raw3.reshape(-1), 14, n_embd, vocab)
    assert np.isnan(want[0]) and oracle.argmax(want) == 0
    assert wl.lm_head_greedy(h, t3, n_embd, vocab)[0] == 0


def test_q6k_kat_rectangular(kats):
    for c in kats:
        if c["op"] != "q6k_matvec":
            continue
        w = np.frombuffer(bytes.fromhex(c["w"]), np.uint8)
        t = TensorView("q6_k.weight", [c["in_dim"], c["out_dim"]], GgmlType.Q6K, w)
        y = np.zeros(c["out_dim"], np.float32)
        wl.linear_matvec_f32(t, c["x"], y)
        assert list(y) == c["expect"], c["id"]


# ----------------------------------------------------------------- argmax

def test_argmax_semantics():
    nan, inf = float("nan"), float("inf")
    cases = [[0.1, 0.5, 0.3], [0.5], [1.0, 1.0], [nan, 5.0, 7.0], [1.0, nan, 0.5],
             [1.0, nan, 2.0], [-0.0, 0.0], [0.0, -0.0, 0.0], [-inf, -inf], [nan, nan],
             [-inf, nan, -inf, -3.0]]
    for c in cases:
        assert wl.argmax(c) == oracle.argmax(c), c
    rng = np.random.default_rng(9)
    for n in (1, 31, 512, 513, 100000, 128256):
        v = rng.standard_normal(n).astype(np.float32)
        v[rng.integers(0, n, 3)] = v.max()  # ties with the max
        assert wl.argmax(v) == oracle.argmax(v) == int(np.argmax(v)), n


# ----------------------------------------------------------------- Q8_0

@pytest.mark.parametrize("in_dim,out_dim", [(32, 2), (576, 1536), (1536, 576), (576, 49152),
                                            (8192, 7), (9216, 33)])
def test_q8_0_matvec_bit_exact(in_dim, out_dim):
    rng = np.random.default_rng(in_dim + 3 * out_dim)
    raw = synth.q8_0_rows(rng, in_dim, out_dim)
    t = TensorView("blk.0.ffn_up.weight", [in_dim, out_dim], GgmlType.Q8_0, raw)
    x = synth.activations(rng, in_dim)
    y = np.zeros(out_dim, np.float32)
    wl.linear_matvec_f32(t, x, y)
    assert_bitexact(y, oracle.q8_0_matvec(raw, in_dim, out_dim, x), "Q8_0 matvec")


def test_q8_0_lm_head_and_kats(kats):
    rng = np.random.default_rng(77)
    n_embd, vocab = 576, 49152
    raw = synth.q8_0_rows(rng, n_embd, vocab)
    t = TensorView("token_embd.weight", [n_embd, vocab], GgmlType.Q8_0, raw)
    h = synth.activations(rng, n_embd)
    want = oracle.compute_logits(h, raw, 8, n_embd, vocab)
    assert_bitexact(wl.compute_logits(h, t, n_embd, vocab), want, "Q8_0 logits")
    assert wl.lm_head_greedy(h, t, n_embd, vocab)[0] == oracle.argmax(want)
    for c in kats:
        if c["op"] == "q8_matvec":
            w = np.frombuffer(bytes.fromhex(c["w"]), np.uint8)
            tk = TensorView("q8.weight", [c["in_dim"], c["out_dim"]], GgmlType.Q8_0, w)
            y = np.zeros(c["out_dim"], np.float32)
            wl.linear_matvec_f32(tk, c["x"], y)
            assert list(y) == c["expect"], c["id"]
        elif c["op"] == "q8_reject":
            w = np.frombuffer(bytes.fromhex(c["row"]), np.uint8)
            tk = TensorView("nan", [32, 1], GgmlType.Q8_0, w)
            with pytest.raises(wl.WillametteError) as e:
                wl.linear_matvec_f32(tk, c["x"], np.zeros(1, np.float32))
            assert e.value.status == WLStatus.GGUF_PARSE
