"""The reference's f32-activation I2_S kernels on the GPU, bit for bit.

A caller whose dispatch (src/model/dispatch.rs:159-184) would not pick the
x86 int8 kernel -- the scalar fallback (bitlinear.rs:146-242), the scalar LUT
of SSE2-only hosts (bitlinear_lut.rs:59-131), or the SSE2 f32 kernel of a
--cfg willamette_sse2_f32 build (bitlinear_sse2.rs:89-124) -- passes that
kernel to wl_bitlinear_i2s_matvec_f32_kernel and must get that kernel's
numbers.  Each is compared with its oracle restatement on fuzz shapes with
code 0b11 present and on activation edge cases (zeros, -0.0, NaN, +-inf,
huge and tiny values).
"""
import numpy as np
import pytest

import oracle
from project_willamette_b200 import TensorView, synth
from project_willamette_b200._abi import I2sKernel

pytestmark = pytest.mark.gpu

ORACLE = {
    I2sKernel.SCALAR: oracle.i2s_matvec_scalar,
    I2sKernel.SSE2_F32: oracle.i2s_matvec_sse2_f32,
    I2sKernel.SCALAR_LUT: oracle.i2s_matvec_lut,
}


def _edge_inputs(rng, k):
    yield "normal", synth.activations(rng, k)
    yield "zeros", np.zeros(k, np.float32)
    x = synth.activations(rng, k)
    x[::7] = -0.0
    yield "neg_zero", x
    x = synth.activations(rng, k)
    x[5] = np.nan
    yield "nan", x
    x = synth.activations(rng, k)
    x[3], x[k - 1] = np.inf, -np.inf
    yield "inf", x
    yield "huge", (synth.activations(rng, k) * np.float32(1e30)).astype(np.float32)
    yield "tiny", (synth.activations(rng, k) * np.float32(1e-40)).astype(np.float32)


@pytest.mark.parametrize("kernel", list(ORACLE))
def test_f32_activation_kernels_match_the_reference_bit_for_bit(kernel):
    import project_willamette_b200 as wl
    rng = np.random.default_rng(40 + int(kernel))
    shapes = [(128, 1), (256, 31), (2560, 640), (2560, 6912), (6912, 33), (768, 257)]
    for k, n in shapes:
        packed = synth.i2s_packed(rng, k, n, code3_fraction=0.01)
        scale = synth.i2s_scale(rng)
        t = TensorView.i2s(f"w{k}x{n}", k, n, packed, scale)
        for name, x in _edge_inputs(rng, k):
            want = ORACLE[kernel](packed, scale, k, n, x)
            got = np.full(n, 123.0, np.float32)
            wl.bitlinear_i2s_matvec_f32(t, x, got, kernel=kernel)
            # bit for bit; a NaN output only has to be a NaN (payload bits are
            # the platform's: x86 makes 0xffc00000, the GPU 0x7fffffff)
            ok = (got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))
            assert ok.all(), f"{kernel.name} {k}x{n} {name}: {int((~ok).sum())} rows differ"
    wl.release_weights()


def test_default_kernel_is_the_int8_one():
    import project_willamette_b200 as wl
    rng = np.random.default_rng(7)
    k, n = 2560, 640
    packed = synth.i2s_packed(rng, k, n)
    scale = synth.i2s_scale(rng)
    x = synth.activations(rng, k)
    t = TensorView.i2s("w", k, n, packed, scale)
    a = np.empty(n, np.float32)
    b = np.empty(n, np.float32)
    wl.bitlinear_i2s_matvec_f32(t, x, a)
    wl.bitlinear_i2s_matvec_f32(t, x, b, kernel=I2sKernel.SSE2_I8)
    want = oracle.i2s_matvec_sse2_i8(packed, scale, k, n, x)[0]
    assert np.array_equal(a.view(np.uint32), want.view(np.uint32))
    assert np.array_equal(b.view(np.uint32), want.view(np.uint32))
    wl.release_weights()
