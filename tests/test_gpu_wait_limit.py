"""A bounded device wait that nothing satisfies runs out, reports
WL_ERR_DEVICE_TIMEOUT's status bit, and leaves the library usable.

Every device-side wait of the library (TMA stage waits, tensor-parallel peer
waits, grid barriers, wl_dev_wait_flag) gives up after the limit that
wl_set_wait_limit_ns sets (default 2 s).  The test shortens the limit, waits
on a flag that nothing sets, checks the status word and the elapsed time,
restores the limit, and then runs a matvec that must still be bit-exact
against the oracle.  No fault, trap or endless loop is involved.
"""
import ctypes as C
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

DEV_ERR_TIMEOUT = 1
DEFAULT_LIMIT_NS = 2_000_000_000


def test_unsatisfied_wait_times_out_and_library_stays_usable(oracle):
    import torch
    import project_willamette_b200 as wl
    from project_willamette_b200 import TensorView, synth

    L = wl.lib()
    assert L.wl_init(0) == 0, L.wl_last_error()
    torch.cuda.set_device(0)
    stream = torch.cuda.current_stream().cuda_stream
    st = C.c_uint32(0)
    assert L.wl_device_status(C.byref(st)) == 0  # start clean
    flag = torch.zeros(4, dtype=torch.int32, device="cuda:0")
    limit_ns = 20_000_000  # 20 ms
    try:
        assert L.wl_set_wait_limit_ns(limit_ns) == 0, L.wl_last_error()
        t0 = time.perf_counter()
        assert L.wl_dev_wait_flag(flag.data_ptr(), 1, stream) == 0, L.wl_last_error()
        torch.cuda.synchronize()
        waited = time.perf_counter() - t0
        assert L.wl_device_status(C.byref(st)) == 0
        assert st.value & DEV_ERR_TIMEOUT, st.value
        # it waited for the shortened limit, not for the 2 s default
        assert limit_ns * 1e-9 * 0.9 < waited < 1.5, waited
        assert L.wl_device_status(C.byref(st)) == 0 and st.value == 0  # reading cleared it
    finally:
        assert L.wl_set_wait_limit_ns(DEFAULT_LIMIT_NS) == 0, L.wl_last_error()

    # a wait whose word is already there returns at once and reports nothing
    flag.fill_(1)
    assert L.wl_dev_wait_flag(flag.data_ptr(), 1, stream) == 0
    torch.cuda.synchronize()
    assert L.wl_device_status(C.byref(st)) == 0 and st.value == 0

    # the context is intact: a BitLinear matvec is still bit-exact
    rng = np.random.default_rng(0x7157)
    K, N = 2560, 640
    packed = synth.i2s_packed(rng, K, N, code3_fraction=0.001)
    scale = synth.i2s_scale(rng)
    x = synth.activations(rng, K)
    y = np.empty(N, np.float32)
    wl.bitlinear_i2s_matvec_f32(TensorView.i2s("w", K, N, packed, scale), x, y)
    ry = oracle.i2s_matvec_sse2_i8(packed, scale, K, N, x)[0]
    assert np.array_equal(y.view(np.uint32), ry.view(np.uint32))
    wl.release_weights()
