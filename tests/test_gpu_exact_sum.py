"""The reference's sequential f32 sums and its exp, bit for bit, on the GPU.

rms_norm_f32's sum of squares (primitives.rs:245-248) and softmax_inplace's
denominator (attention.rs:61-65) are one-term-at-a-time f32 loops; exact mode
runs them in that order (wl_ptx.cuh seq_sum, the squares formed in
parallel first).  wl_dev_rms_norm_f32 is checked with inputs that stress f32
rounding -- exact ties (dyadic and integer squares), many binade crossings,
subnormal partial sums, zeros, a dynamic range of 10^30, NaN, inf and totals
beyond the f32 range -- against the oracle's rms_norm_f32, every output bit.

wl_dev_softmax_f32 adds the reference's exp: f32::exp is the C library's
expf (glibc 2.39 here), restated in csrc/glibc_expf.cuh.  Its cases put one
element at 0 (the maximum) so that every other element's exponential is
expf of that element itself, over a sweep of arguments from -104 to 0, the
argument where glibc corrects its polynomial, and random vectors, compared
bit for bit with the oracle's softmax_inplace.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _cases(rng):
    for n in (64, 100, 640, 2560, 6912, 8192, 16384):
        yield "normal", rng.standard_normal(n)
        yield "dyadic", rng.integers(1, 4096, n) * np.exp2(-rng.integers(0, 21, n).astype(np.float64))
        yield "small_ints", rng.integers(0, 4, n).astype(np.float64)
        yield "wide", np.power(10.0, rng.uniform(-15, 15, n)) * rng.choice([-1, 1], n)
        yield "subnormal_squares", rng.standard_normal(n) * 1e-22
        x = rng.standard_normal(n)
        x[: n // 2] *= 1e-22
        yield "subnormal_then_normal", x
        x = rng.standard_normal(n)
        x[rng.random(n) < 0.5] = 0.0
        yield "half_zeros", x
        yield "ones", np.ones(n)
        yield "powers_of_two", np.exp2(rng.integers(-15, 15, n).astype(np.float64))
    yield "all_zero", np.zeros(2560)
    x = rng.standard_normal(2560)
    x[1234] = np.nan
    yield "nan", x
    x = rng.standard_normal(2560)
    x[7] = np.inf
    yield "inf", x
    yield "near_f32_limit", rng.standard_normal(2560) * 1e18
    yield "max_n", rng.standard_normal(16384) * 3.0


def test_rms_norm_sum_is_the_sequential_sum_bit_for_bit(oracle):
    import torch
    import project_willamette_b200 as wl

    L = wl.lib()
    assert L.wl_init(0) == 0
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(0xE5)
    eps = np.float32(1e-5)
    bad = []
    n_cases = 0
    for name, x64 in _cases(rng):
        x = x64.astype(np.float32)
        n = x.size
        w = rng.uniform(0.5, 1.5, n).astype(np.float32)
        want = oracle.rms_norm(x, w, float(eps))
        dx = torch.from_numpy(x).cuda()
        dw = torch.from_numpy(w).cuda()
        out = torch.full((n,), float("nan"), device="cuda")
        rc = L.wl_dev_rms_norm_f32(dx.data_ptr(), dw.data_ptr(), n, eps, out.data_ptr(), stream)
        assert rc == 0, L.wl_last_error()
        got = out.cpu().numpy()
        n_cases += 1
        # bit for bit; a NaN only has to be a NaN (payload bits are the
        # platform's: x86 makes 0xffc00000, the GPU 0x7fffffff)
        diff = ~_same_or_both_nan(got, want)
        if diff.any():
            bad.append(f"{name}/{n}: {int(diff.sum())} elements differ")
    assert not bad, "; ".join(bad)
    assert n_cases >= 60


def _same_or_both_nan(got, want):
    return (got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))


def _softmax_cases(rng):
    # a sweep of float arguments over [-104, 0] with a stride of 1024 floats
    hi = np.float32(-104.0).view(np.uint32)
    sweep = np.arange(0x80000001, int(hi) + 1, 1024, dtype=np.uint64).astype(np.uint32).view(np.float32)
    for k in range(0, sweep.size, 16383):
        yield "sweep", np.concatenate([[0.0], sweep[k:k + 16383]]).astype(np.float32)
    # with the maximum at 0, exp(-0x1.f8cbb2p+5): one of the two arguments where
    # glibc corrects its polynomial (the other is positive, out of softmax's reach)
    h = np.float32(float.fromhex("-0x1.f8cbb2p+5"))
    yield "hard_case", np.array([0.0, h, np.nextafter(h, np.float32(0)),
                                 np.nextafter(h, np.float32(-200))], np.float32)
    for n in (1, 7, 640, 2560, 16384):
        yield "normal", rng.standard_normal(n).astype(np.float32) * 4
        yield "wide", (rng.standard_normal(n) * 60).astype(np.float32)
    x = rng.standard_normal(100).astype(np.float32)
    x[3] = np.nan
    yield "nan", x
    yield "all_neg_inf", np.full(8, -np.inf, np.float32)
    x = rng.standard_normal(50).astype(np.float32)
    x[10] = np.inf
    yield "pos_inf", x


def test_softmax_with_the_reference_expf_bit_for_bit(oracle):
    import torch
    import project_willamette_b200 as wl

    L = wl.lib()
    assert L.wl_init(0) == 0
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(0xE6)
    bad, n_cases, n_values = [], 0, 0
    for name, x in _softmax_cases(rng):
        want = oracle.softmax(x)
        d = torch.from_numpy(x.copy()).cuda()
        assert L.wl_dev_softmax_f32(d.data_ptr(), x.size, stream) == 0, L.wl_last_error()
        got = d.cpu().numpy()
        n_cases += 1
        n_values += x.size
        ok = _same_or_both_nan(got, want)
        if not ok.all():
            bad.append(f"{name}/{x.size}: {int((~ok).sum())} differ")
    assert not bad, "; ".join(bad[:10])
    assert n_values > 1_000_000


def test_rms_norm_rejects_bad_sizes():
    import project_willamette_b200 as wl
    from project_willamette_b200._abi import WLStatus

    L = wl.lib()
    assert L.wl_dev_rms_norm_f32(16, 16, 6, 1e-5, 16, None) == WLStatus.INVALID_ARGUMENT
    assert L.wl_dev_rms_norm_f32(16, 16, 16384 + 4, 1e-5, 16, None) == WLStatus.INVALID_ARGUMENT
    assert L.wl_dev_rms_norm_f32(None, None, 0, 1e-5, None, None) == 0  # empty: nothing to do
