"""The no-allocation I2_S entry point gives the allocating entry point's answer.

wl_dev_i2s_matvec_f32_noalloc is for callers that cannot call cudaMalloc:
for example a serving engine that reserved the GPU's memory for its own pools
up front, or a decode loop where a cudaMalloc/cudaFree would stall it by
synchronising the device.  Its int8 activations and their scale live in a
static device array of the library instead of caller buffers.  This file runs
last (pytest collects it last) and also passes on its own in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL = 1e-5  # the tolerance the parity tests state; the kernels agree bit for bit
MAX_IN_DIM = 16384  # WL_NOALLOC_MAX_IN_DIM


def _allocating(L, packed, scale, K, N, x, torch, dev, stream):
    y = torch.empty(N, dtype=torch.float32, device=dev)
    q = torch.empty(K, dtype=torch.int8, device=dev)
    sc = torch.empty(4, dtype=torch.float32, device=dev)
    rc = L.wl_dev_i2s_matvec_f32(packed.data_ptr(), scale, K, N, x.data_ptr(), y.data_ptr(),
                                 q.data_ptr(), sc.data_ptr(), stream)
    assert rc == 0, L.wl_last_error()
    return y


def _noalloc(L, packed, scale, K, N, x, torch, dev, stream):
    y = torch.full((N,), float("nan"), dtype=torch.float32, device=dev)
    rc = L.wl_dev_i2s_matvec_f32_noalloc(packed.data_ptr(), scale, K, N, x.data_ptr(),
                                         y.data_ptr(), stream)
    assert rc == 0, L.wl_last_error()
    return y


def _same(y_new, y_ref):
    a, b = y_new.cpu().numpy(), y_ref.cpu().numpy()
    np.testing.assert_allclose(a, b, rtol=RTOL, atol=0)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def _setup():
    import torch
    import project_willamette_b200 as wl
    L = wl.lib()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    return torch, L, dev, torch.cuda.current_stream().cuda_stream


def test_noalloc_matches_allocating_entry_point_on_consecutive_calls():
    from project_willamette_b200 import synth
    torch, L, dev, stream = _setup()
    rng = np.random.default_rng(20261201)
    # Calls one after another that reuse the shared scratch: each must not see
    # anything of the one before (different shape and a larger activation).
    for K, N, xscale in [(6912, 2560, 1.0), (2560, 6912, 1000.0), (2560, 6912, 0.001)]:
        packed = torch.from_numpy(synth.i2s_packed(rng, K, N, code3_fraction=0.001)).to(dev)
        scale = synth.i2s_scale(rng)
        x = torch.from_numpy(synth.activations(rng, K) * np.float32(xscale)).to(dev)
        y_ref = _allocating(L, packed, scale, K, N, x, torch, dev, stream)
        y_new = _noalloc(L, packed, scale, K, N, x, torch, dev, stream)
        torch.cuda.synchronize()
        _same(y_new, y_ref)


def test_noalloc_back_to_back_on_one_stream_and_at_its_size_limit():
    """Several calls queued on one stream with different inputs and no host
    synchronisation between them (each call's scratch writes follow the
    previous call's reads in stream order), including in_dim at the limit."""
    from project_willamette_b200 import synth
    torch, L, dev, stream = _setup()
    rng = np.random.default_rng(20261202)
    cases = [(2560, 2560, 1.0), (MAX_IN_DIM, 640, 3.0), (6912, 2560, 0.01), (2560, 640, 50.0),
             (MAX_IN_DIM, 1024, 0.5)]
    inputs, refs, outs = [], [], []
    for K, N, xscale in cases:
        packed = torch.from_numpy(synth.i2s_packed(rng, K, N, code3_fraction=0.001)).to(dev)
        x = torch.from_numpy(synth.activations(rng, K) * np.float32(xscale)).to(dev)
        inputs.append((packed, synth.i2s_scale(rng), K, N, x))
    torch.cuda.synchronize()
    for packed, scale, K, N, x in inputs:
        refs.append(_allocating(L, packed, scale, K, N, x, torch, dev, stream))
    for packed, scale, K, N, x in inputs:
        outs.append(_noalloc(L, packed, scale, K, N, x, torch, dev, stream))
    torch.cuda.synchronize()
    for y_new, y_ref in zip(outs, refs):
        _same(y_new, y_ref)
    # the entry point's status word (in its static array) is read by
    # wl_device_status: no bounded wait ran out in these calls
    st = C.c_uint32(0xFFFFFFFF)
    assert L.wl_device_status(C.byref(st)) == 0, L.wl_last_error()
    assert st.value == 0


def test_noalloc_rejects_in_dim_beyond_its_scratch():
    import project_willamette_b200 as wl
    from project_willamette_b200._abi import WLStatus

    L = wl.lib()
    K = MAX_IN_DIM + 128
    rc = L.wl_dev_i2s_matvec_f32_noalloc(16, 0.05, K, 8, 16, 16, None)
    assert rc == WLStatus.INVALID_ARGUMENT
    assert b"WL_NOALLOC_MAX_IN_DIM" in L.wl_last_error()
