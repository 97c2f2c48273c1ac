"""The reference's sequential f32 sums, bit for bit, from a whole CTA.

Exact mode reproduces rms_norm_f32's sum of squares (primitives.rs:245-248)
and softmax_inplace's denominator (attention.rs:61-65) with the bits of the
reference's one-term-at-a-time loop, but computes them in parallel
(csrc/exact_sum.cuh): runs of additions that stay inside one binade are
exact integer steps and are summed with a block scan, and only binade
crossings and rounding ties are added one by one.  These cases drive that
algorithm through wl_dev_rms_norm_f32 with inputs chosen to break it --
exact ties (dyadic and integer squares), many binade crossings, subnormal
partial sums, zeros, a dynamic range of 10^30, and the fallbacks (NaN, inf,
totals near the f32 limit) -- and compare every output bit with the oracle's
rms_norm_f32.
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
        if not np.array_equal(got.view(np.uint32), want.view(np.uint32)):
            bad.append(f"{name}/{n}: {int(np.sum(got.view(np.uint32) != want.view(np.uint32)))} "
                       f"elements differ")
    assert not bad, "; ".join(bad)
    assert n_cases >= 60


def test_rms_norm_rejects_bad_sizes():
    import project_willamette_b200 as wl
    from project_willamette_b200._abi import WLStatus

    L = wl.lib()
    assert L.wl_dev_rms_norm_f32(16, 16, 6, 1e-5, 16, None) == WLStatus.INVALID_ARGUMENT
    assert L.wl_dev_rms_norm_f32(16, 16, 16384 + 4, 1e-5, 16, None) == WLStatus.INVALID_ARGUMENT
    assert L.wl_dev_rms_norm_f32(None, None, 0, 1e-5, None, None) == 0  # empty: nothing to do
