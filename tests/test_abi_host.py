"""Host-side tests of the C ABI (no GPU needed).

The shared library must load and export every function the header
declares, and every shape/type/scale rejection the reference performs must be
reported with the matching status before anything touches a device (the
reference "never writes fake zeros on error", docs/BITLINEAR_I2S_MATVEC.md
section 7, so the output buffer must be untouched).
"""
import math

import numpy as np
import pytest

import project_willamette_b200 as wl
from project_willamette_b200 import GgmlType, TensorView, WillametteError
from project_willamette_b200._abi import WLStatus, header_functions, lib


def test_library_exports_every_header_function():
    L = lib()
    names = header_functions()
    assert len(names) >= 20
    for n in names:
        assert hasattr(L, n), n
    assert b"sm_100a" in L.wl_version()


def _i2s(in_dim=128, out_dim=1, scale=1.0, data_len=None, scale_block=True):
    n = in_dim * out_dim // 4 if data_len is None else data_len
    t = TensorView.i2s("blk.0.attn_q.weight", in_dim, out_dim, np.full(n, 0xAA, np.uint8), scale)
    if not scale_block:
        t.scale_data = None
    return t


def _expect(status, fn, *a):
    with pytest.raises(WillametteError) as e:
        fn(*a)
    assert e.value.status == status, str(e.value)
    return e.value


def test_i2s_rejections_match_reference():
    y = np.full(1, 123.0, np.float32)
    # bitlinear.rs:151-155 wrong dtype -> UnsupportedTensorType(raw)
    t = _i2s()
    t.ggml_type = GgmlType.F32
    err = _expect(WLStatus.UNSUPPORTED_TENSOR_TYPE, wl.bitlinear_i2s_matvec_f32, t, np.ones(128), y)
    assert err.raw_type == 0
    # not 2-D
    t = _i2s()
    t.shape = [128]
    _expect(WLStatus.GGUF_PARSE, wl.bitlinear_i2s_matvec_f32, t, np.ones(128), y)
    # bitlinear.rs:484-502 wrong input / output lengths
    _expect(WLStatus.GGUF_PARSE, wl.bitlinear_i2s_matvec_f32, _i2s(), np.ones(64), y)
    _expect(WLStatus.GGUF_PARSE, wl.bitlinear_i2s_matvec_f32, _i2s(), np.ones(128),
            np.zeros(2, np.float32))
    # bitlinear.rs:504-512 in_dim not a multiple of 128
    _expect(WLStatus.GGUF_PARSE, wl.bitlinear_i2s_matvec_f32, _i2s(64, 1, data_len=32),
            np.ones(64), y)
    # bitlinear_sse2.rs:167-175 packed area too short (>= is accepted)
    _expect(WLStatus.GGUF_PARSE, wl.bitlinear_i2s_matvec_f32, _i2s(data_len=31), np.ones(128), y)
    # tensor.rs:286-307 missing / short / non-finite scale
    _expect(WLStatus.GGUF_PARSE, wl.bitlinear_i2s_matvec_f32, _i2s(scale_block=False),
            np.ones(128), y)
    t = _i2s()
    t.scale_data = t.scale_data[:3]
    _expect(WLStatus.GGUF_PARSE, wl.bitlinear_i2s_matvec_f32, t, np.ones(128), y)
    for bad in (math.nan, math.inf, -math.inf):
        _expect(WLStatus.GGUF_PARSE, wl.bitlinear_i2s_matvec_f32, _i2s(scale=bad), np.ones(128), y)
    assert y[0] == 123.0  # never written on error


def test_linear_matvec_dispatch_errors():
    y = np.zeros(2, np.float32)
    for ty in (GgmlType.F16, GgmlType.Q4_0, GgmlType.Q4K):
        t = TensorView("w", [32, 2], ty, np.zeros(64, np.uint8))
        _expect(WLStatus.NOT_IMPLEMENTED, wl.linear_matvec_f32, t, np.ones(32), y)
    t = TensorView("w", [32, 2], 7, np.zeros(64, np.uint8))  # Q5_1: linear.rs:23
    err = _expect(WLStatus.UNSUPPORTED_TENSOR_TYPE, wl.linear_matvec_f32, t, np.ones(32), y)
    assert err.raw_type == 7
    # Q8_0: lengths / row multiple / data length (linear.rs:176-213)
    t = TensorView("w", [32, 2], GgmlType.Q8_0, np.zeros(68, np.uint8))
    _expect(WLStatus.GGUF_PARSE, wl.linear_matvec_f32, t, np.ones(31), y)
    t = TensorView("w", [16, 2], GgmlType.Q8_0, np.zeros(68, np.uint8))
    _expect(WLStatus.GGUF_PARSE, wl.linear_matvec_f32, t, np.ones(16), y)
    t = TensorView("w", [32, 2], GgmlType.Q8_0, np.zeros(67, np.uint8))
    _expect(WLStatus.GGUF_PARSE, wl.linear_matvec_f32, t, np.ones(32), y)
    t = TensorView("w", [128, 2], GgmlType.Q6K, np.zeros(420, np.uint8))
    _expect(WLStatus.GGUF_PARSE, wl.linear_matvec_f32, t, np.ones(128), y)


def test_compute_logits_validation():
    h = np.ones(256, np.float32)
    t = TensorView("token_embd.weight", [256, 3], GgmlType.Q6K, np.zeros(630, np.uint8))
    # lm_head.rs:35-44 type not in {F16, Q4_0, Q4_K, Q6_K, Q8_0} -> GgufParse
    bad = TensorView("token_embd.weight", [256, 3], GgmlType.F32, np.zeros(3072, np.uint8))
    _expect(WLStatus.GGUF_PARSE, wl.compute_logits, h, bad, 256, 3)
    # shape mismatch (:45-50), hidden length (:52-58), data length (:79-85)
    _expect(WLStatus.GGUF_PARSE, wl.compute_logits, h, t, 256, 4)
    _expect(WLStatus.GGUF_PARSE, wl.compute_logits, np.ones(255), t, 256, 3)
    short = TensorView("token_embd.weight", [256, 3], GgmlType.Q6K, np.zeros(629, np.uint8))
    _expect(WLStatus.GGUF_PARSE, wl.compute_logits, h, short, 256, 3)
    # F16 tables are served by the reference's CPU arm
    f16 = TensorView("token_embd.weight", [256, 3], GgmlType.F16, np.zeros(1536, np.uint8))
    _expect(WLStatus.NOT_IMPLEMENTED, wl.compute_logits, h, f16, 256, 3)


def test_empty_cases_need_no_device():
    assert wl.argmax([]) is None
    # out_dim == 0: the reference loops over nothing and returns Ok.
    t = TensorView.i2s("w", 128, 0, np.zeros(0, np.uint8), 1.0)
    wl.bitlinear_i2s_matvec_f32(t, np.ones(128), np.zeros(0, np.float32))


def test_layout_byte_counts(kats):
    fns = {"Q6_K": wl.q6k_expected_byte_len, "Q8_0": wl.q8_0_expected_byte_len,
           "I2_S": wl.i2s_expected_byte_len}
    for c in kats:
        if c["op"] != "byte_len":
            continue
        for ty, shape, want in c["cases"]:
            if want is None:
                with pytest.raises(WillametteError):
                    fns[ty](shape)
            else:
                assert fns[ty](shape) == want, (ty, shape)


def test_no_gpu_is_a_loud_error():
    """On a machine without an sm_100 device the library reports it; it never
    computes on the CPU instead."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(WillametteError) as e:
        wl.bitlinear_i2s_matvec_f32(_i2s(), np.ones(128), np.zeros(1, np.float32))
    assert e.value.status in (WLStatus.NO_DEVICE, WLStatus.CUDA)


def test_header_documents_reference_for_each_hot_entry_point():
    src = open(wl._abi.HEADER_PATH).read()
    for ref in ("bitlinear.rs:67", "bitlinear_sse2.rs:313", "linear.rs:11", "lm_head.rs:29",
                "lm_head.rs:161", "q6_k_sse2.rs:46", "q8_0_simd.rs:72"):
        assert ref in src, ref


def test_stream_plan_validation_before_any_device_work():
    """A stream plan rejects shapes it cannot stream before touching a device."""
    import ctypes
    from project_willamette_b200._abi import WlI2sStreamOp
    L = lib()
    buf = (ctypes.c_uint8 * 4096 * 4)()
    base = (ctypes.addressof(buf) + 15) // 16 * 16
    op = WlI2sStreamOp()
    op.packed, op.w_scale, op.in_dim, op.out_dim = base, 0.05, 384, 4
    op.x, op.y, op.acc, op.flags = base, base, None, 0
    plan = ctypes.c_void_p()
    assert L.wl_i2s_stream_plan_create(ctypes.byref(op), 1, ctypes.byref(plan)) == WLStatus.INVALID_ARGUMENT
    assert b"in_dim 384" in L.wl_last_error()
    op.in_dim = 512
    op.packed = base + 4  # misaligned
    assert L.wl_i2s_stream_plan_create(ctypes.byref(op), 1, ctypes.byref(plan)) == WLStatus.INVALID_ARGUMENT
    op.packed = base
    op.w_scale = float("nan")
    assert L.wl_i2s_stream_plan_create(ctypes.byref(op), 1, ctypes.byref(plan)) == WLStatus.GGUF_PARSE
    assert not plan.value


def test_tensor_view_struct_cached_and_invalidated():
    """The C struct of a TensorView is built once and rebuilt when the view
    changes (data, shape, type or name); pickling drops the cached struct."""
    import pickle
    import project_willamette_b200 as wl_pkg
    from project_willamette_b200 import synth
    t = wl_pkg.TensorView.i2s("w", 256, 8, synth.i2s_packed(np.random.default_rng(5), 256, 8), 0.5)
    v1, _ = wl_pkg._view(t)
    v2, _ = wl_pkg._view(t)
    assert v1 is v2 and v1.data_len == 256 // 4 * 8
    t.shape = [256, 8]  # equal shape: still cached
    assert wl_pkg._view(t)[0] is v1
    t.name = "renamed"
    v3, _ = wl_pkg._view(t)
    assert v3 is not v1 and v3.name == b"renamed"
    t.data = np.zeros(256 // 4 * 8, np.uint8)
    v4, _ = wl_pkg._view(t)
    assert v4 is not v3 and v4.data_len == 512
    t2 = pickle.loads(pickle.dumps(t))
    assert "_cview" not in t2.__dict__ and list(t2.shape) == [256, 8]


def test_wait_limit_and_flag_wait_validation():
    """wl_set_wait_limit_ns rejects limits outside [1 us, 600 s] and
    wl_dev_wait_flag a NULL or misaligned flag, before touching a device."""
    L = lib()
    for bad in (0, 999, 600_000_000_001):
        assert L.wl_set_wait_limit_ns(bad) == WLStatus.INVALID_ARGUMENT
        assert b"wait limit" in L.wl_last_error()
    assert L.wl_dev_wait_flag(None, 1, None) == WLStatus.INVALID_ARGUMENT
    assert L.wl_dev_wait_flag(2, 1, None) == WLStatus.INVALID_ARGUMENT


def test_f32_activation_dispatch_validation():
    """Before any device work: the NEON choice has no GPU arm (the caller keeps
    its CPU kernel), an unknown kernel is rejected, and the scalar and LUT
    kernels want the packed length exactly (bitlinear.rs:192,
    bitlinear_lut.rs:174) while the SSE2 kernels accept longer data."""
    from project_willamette_b200._abi import I2sKernel
    x = np.ones(128, np.float32)
    y = np.full(1, 7.0, np.float32)
    _expect(WLStatus.NOT_IMPLEMENTED, wl.bitlinear_i2s_matvec_f32, _i2s(), x, y, I2sKernel.NEON)
    _expect(WLStatus.INVALID_ARGUMENT, wl.bitlinear_i2s_matvec_f32, _i2s(), x, y, 9)
    for k in (I2sKernel.SCALAR, I2sKernel.SCALAR_LUT):
        e = _expect(WLStatus.GGUF_PARSE, wl.bitlinear_i2s_matvec_f32, _i2s(data_len=40), x, y, k)
        assert "expected packed" in str(e)
    assert y[0] == 7.0
