"""Pin the CPU oracle to the reference's own known-answer tests.

Each case in tests/golden/reference_kats.json is a unit test of the Rust
reference, transcribed with its file:line; here the C restatement must
reproduce the value (or meet the tolerance) the Rust test asserts.  "dispatch"
cases run the kernel the reference's x86 dispatch selects on an SSSE3+ host
(bitlinear.rs:106-129 -> bitlinear_sse2.rs:313 int8-activation kernel).
"""
import math

import numpy as np
import pytest


def _b(h):
    return np.frombuffer(bytes.fromhex(h), dtype=np.uint8)


def _i2s(oracle, c):
    fn = {"dispatch": lambda *a: oracle.i2s_matvec_sse2_i8(*a)[0],
          "scalar": oracle.i2s_matvec_scalar}[c["path"]]
    return fn(_b(c["packed"]), c["scale"], c["in_dim"], c["out_dim"], c["x"])


def test_kat_file_covers_reference_tests(kats):
    assert len(kats) >= 25
    assert all(":" in c["id"] for c in kats)


def test_i2s_kats(kats, oracle):
    n = 0
    for c in kats:
        if c["op"] == "i2s_matvec":
            y = _i2s(oracle, c)
            np.testing.assert_allclose(y, c["expect"], atol=c["tol_abs"], rtol=0, err_msg=c["id"])
            if c["tol_abs"] == 0.0:
                assert list(y) == c["expect"], c["id"]
            n += 1
        elif c["op"] == "i2s_deterministic":
            a, b = _i2s(oracle, c), _i2s(oracle, c)
            assert np.array_equal(a, b), c["id"]
            n += 1
        elif c["op"] == "i2s_reject":
            for fn in (oracle.i2s_matvec_scalar, oracle.i2s_matvec_lut,
                       oracle.i2s_matvec_sse2_f32):
                with pytest.raises(oracle.OracleError):
                    fn(_b(c["packed"]), c["scale"], c["in_dim"], c["out_dim"], c["x"])
            with pytest.raises(oracle.OracleError):
                oracle.i2s_matvec_sse2_i8(_b(c["packed"]), c["scale"], c["in_dim"],
                                          c["out_dim"], c["x"])
            n += 1
        elif c["op"] == "i2s_unpack":
            row = oracle.i2s_unpack_row(_b(c["packed"]), c["in_dim"], c["out_dim"], c["row"])
            assert list(row) == c["expect"], c["id"]
            n += 1
    assert n == 9


def test_i2s_scalar_sse2_lut_agree_on_kats(kats, oracle):
    """The f32 kernels (scalar, SSE2 mask-add, LUT) agree on every KAT input
    (tests/bitlinear_sse2.rs:30 and tests/bitlinear_lut.rs:26 use 1e-2)."""
    for c in kats:
        if c["op"] != "i2s_matvec":
            continue
        args = (_b(c["packed"]), c["scale"], c["in_dim"], c["out_dim"], c["x"])
        ref = oracle.i2s_matvec_scalar(*args)
        np.testing.assert_allclose(oracle.i2s_matvec_sse2_f32(*args), ref, atol=1e-2, rtol=0)
        np.testing.assert_allclose(oracle.i2s_matvec_lut(*args), ref, atol=1e-2, rtol=0)


def test_i2s_scale_must_be_finite(oracle):
    """tensor.rs:296-307: a non-finite scale is an error for every kernel."""
    args = (np.full(32, 0xAA, np.uint8),)
    for bad in (float("nan"), float("inf")):
        with pytest.raises(oracle.OracleError):
            oracle.i2s_matvec_sse2_i8(*args, bad, 128, 1, np.ones(128))
        with pytest.raises(oracle.OracleError):
            oracle.i2s_matvec_scalar(*args, bad, 128, 1, np.ones(128))


def test_absmax_kats(kats, oracle):
    for c in kats:
        if c["op"] != "absmax_i8":
            continue
        q, s = oracle.quantize_absmax_i8(c["x"])
        assert abs(s - c["expect_scale"]) <= c["scale_tol"], c["id"]
        for k, v in c["expect_q"].items():
            assert int(q[int(k)]) == v, c["id"]


def test_q6k_kats(kats, oracle):
    n = 0
    for c in kats:
        op = c["op"]
        if op == "q6k_dequant":
            out = oracle.q6k_dequantize_row(_b(c["row"]), c["n"])
            if "expect_all" in c:
                assert np.all(out == c["expect_all"]), c["id"]
            for k, v in c.get("expect_at", {}).items():
                assert out[int(k)] == v, c["id"]
            n += 1
        elif op == "q6k_dot":
            row = _b(c["row"])
            assert oracle.q6k_dot_row_scalar(row, c["x"]) == c["expect_scalar_exact"], c["id"]
            assert abs(oracle.q6k_dot_row_sse2(row, c["x"]) - c["expect"]) < c["tol_abs"]
            n += 1
        elif op == "q6k_quantize_dot":
            q = oracle.q6k_quantize_row(c["x"])
            assert q.size == 420
            scalar = oracle.q6k_dot_row_scalar(q, c["probe"])
            simd = oracle.q6k_dot_row_sse2(q, c["probe"])
            dec = oracle.q6k_dequantize_row(q, 512)
            sum_abs = float(np.sum(np.abs(dec.astype(np.float32) * np.float32(c["probe"]))))
            assert abs(simd - scalar) <= c["rel_tol"] * max(sum_abs, 1.0), c["id"]
            n += 1
        elif op == "q6k_roundtrip":
            q = oracle.q6k_quantize_row(c["x"])
            dec = oracle.q6k_dequantize_row(q, len(c["x"]))
            assert float(np.max(np.abs(np.float32(c["x"]) - dec))) < c["max_error"], c["id"]
            n += 1
        elif op == "q6k_matvec":
            w = _b(c["w"])
            out = oracle.compute_logits(c["x"], w, 14, c["in_dim"], c["out_dim"], n_threads=1)
            assert list(out) == c["expect"], c["id"]
            n += 1
    assert n == 6


def test_q8_kats(kats, oracle):
    n = 0
    for c in kats:
        op = c["op"]
        if op == "q8_dequant":
            out = oracle.q8_0_dequantize_row(_b(c["row"]), c["n"])
            for k, v in c["expect_at"].items():
                assert out[int(k)] == v, c["id"]
            n += 1
        elif op == "q8_dot":
            for fn in (oracle.q8_0_dot_row_avx2, oracle.q8_0_dot_row_sse2,
                       oracle.q8_0_dot_row_scalar):
                assert abs(fn(_b(c["row"]), c["x"]) - c["expect"]) < c["tol_abs"], c["id"]
            n += 1
        elif op == "q8_dot_vs_scalar":
            row = _b(c["row"])
            ref = oracle.q8_0_dot_row_scalar(row, c["x"])
            for fn in (oracle.q8_0_dot_row_avx2, oracle.q8_0_dot_row_sse2):
                assert abs(fn(row, c["x"]) - ref) < c["tol_abs"], c["id"]
            n += 1
        elif op == "q8_reject":
            for fn in (oracle.q8_0_dot_row_avx2, oracle.q8_0_dot_row_sse2,
                       oracle.q8_0_dot_row_scalar):
                with pytest.raises(oracle.OracleError):
                    fn(_b(c["row"]), c["x"])
            n += 1
        elif op == "q8_matvec":
            y = oracle.q8_0_matvec(_b(c["w"]), c["in_dim"], c["out_dim"], c["x"], n_threads=1)
            assert list(y) == c["expect"], c["id"]
            n += 1
    assert n == 5


def test_misc_kats(kats, oracle):
    for c in kats:
        if c["op"] == "argmax":
            for logits, want in c["cases"]:
                assert oracle.argmax(logits) == want, c["id"]
        elif c["op"] == "f16":
            for bits, want in c["cases"]:
                got = oracle.f16_to_f32(bits)
                if want == "nan":
                    assert math.isnan(got)
                elif want == "-0.0":
                    assert got == 0.0 and math.copysign(1.0, got) < 0
                else:
                    assert got == float(want), (c["id"], bits)
        elif c["op"] == "ternary":
            for code, want in c["cases"]:
                assert oracle.ternary_from_code(code) == want


def test_argmax_nan_semantics(oracle):
    """lm_head.rs:161-174 uses strict '>': a NaN never wins unless it is at index 0."""
    nan = float("nan")
    assert oracle.argmax([nan, 5.0, 7.0]) == 0
    assert oracle.argmax([1.0, nan, 0.5]) == 0
    assert oracle.argmax([1.0, nan, 2.0]) == 2
    assert oracle.argmax([-0.0, 0.0]) == 0
    assert oracle.argmax([float("-inf"), float("-inf")]) == 0


def test_f32_to_f16_round_trip(oracle):
    """RNE binary16 rounding used by the Q6_K quantiser matches numpy's."""
    rng = np.random.default_rng(7)
    vals = np.concatenate([rng.standard_normal(2000).astype(np.float32) * 10,
                           rng.standard_normal(200).astype(np.float32) * 1e-6,
                           np.float32([65504, 65520, 1e6, -1e6, 2 ** -25, 2 ** -24, 0.0])])
    for v in vals:
        with np.errstate(over="ignore"):  # 65520 and +-1e6 round to +-inf on purpose
            want = int(np.array([v], np.float32).astype(np.float16).view(np.uint16)[0])
        assert oracle.f32_to_f16(float(v)) == want, float(v)
