"""The no-allocation I2_S entry point gives the allocating entry point's answer.

wl_dev_i2s_matvec_f32_noalloc is for callers that cannot call cudaMalloc:
for example a serving engine that reserved the GPU's memory for its own pools
up front, or a decode loop where a cudaMalloc/cudaFree would stall it by
synchronising the device.  Its int8 activations and their scale live in a
static device array of the library instead of caller buffers.  This file runs
last (pytest collects it last) and also passes on its own in a fresh process.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL = 1e-5  # the tolerance the parity tests state; the kernels agree bit for bit


def _run(L, fn_noalloc, packed, scale, K, N, x, torch, dev, stream):
    y_ref = torch.empty(N, dtype=torch.float32, device=dev)
    y_new = torch.full((N,), float("nan"), dtype=torch.float32, device=dev)
    q = torch.empty(K, dtype=torch.int8, device=dev)
    sc = torch.empty(4, dtype=torch.float32, device=dev)
    rc = L.wl_dev_i2s_matvec_f32(packed.data_ptr(), scale, K, N, x.data_ptr(), y_ref.data_ptr(),
                                 q.data_ptr(), sc.data_ptr(), stream)
    assert rc == 0, L.wl_last_error()
    if fn_noalloc:
        rc = L.wl_dev_i2s_matvec_f32_noalloc(packed.data_ptr(), scale, K, N, x.data_ptr(),
                                             y_new.data_ptr(), stream)
        assert rc == 0, L.wl_last_error()
    torch.cuda.synchronize()
    return y_ref.cpu().numpy(), y_new.cpu().numpy()


def test_noalloc_matches_allocating_entry_point_on_consecutive_calls():
    import torch
    import project_willamette_b200 as wl
    from project_willamette_b200 import synth

    L = wl.lib()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(20261201)
    # Two calls in a row that reuse the shared scratch: the second must not
    # see anything of the first (different shape and a larger activation).
    for K, N, xscale in [(6912, 2560, 1.0), (2560, 6912, 1000.0), (2560, 6912, 0.001)]:
        packed = torch.from_numpy(synth.i2s_packed(rng, K, N, code3_fraction=0.001)).to(dev)
        scale = synth.i2s_scale(rng)
        x = torch.from_numpy(synth.activations(rng, K) * np.float32(xscale)).to(dev)
        y_ref, y_new = _run(L, True, packed, scale, K, N, x, torch, dev, stream)
        np.testing.assert_allclose(y_new, y_ref, rtol=RTOL, atol=0)
        assert np.array_equal(y_new.view(np.uint32), y_ref.view(np.uint32))


def test_noalloc_rejects_in_dim_beyond_its_scratch():
    import project_willamette_b200 as wl
    from project_willamette_b200._abi import WLStatus

    L = wl.lib()
    K = 16384 + 128
    rc = L.wl_dev_i2s_matvec_f32_noalloc(16, 0.05, K, 8, 16, 16, None)
    assert rc == WLStatus.INVALID_ARGUMENT
    assert b"WL_NOALLOC_MAX_IN_DIM" in L.wl_last_error()
