"""Write reference_kats.json: the reference's own known-answer tests.

The reference (Rust crate project-willamette v0.14.0) cannot be executed on
these machines (no Rust toolchain), so its unit tests are transcribed here
as data: each case rebuilds the exact input bytes the Rust test constructs
and records the value or tolerance the Rust test asserts, with the
file:line it comes from.  Both the CPU oracle (tests/test_oracle_kats.py)
and the CUDA library (the KAT cases of tests/test_gpu_parity.py) are checked
against this file.

Cases whose expected value the Rust test computes at run time from its own
inputs (e.g. "expected = sum of the inputs") are evaluated here with the same
f32 arithmetic, in the same order, in numpy float32.

Run:  python tests/golden/make_kats.py   (rewrites reference_kats.json)
"""
from __future__ import annotations

import json
import os
import struct

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "reference_kats.json")


def f32(v: float) -> float:
    return float(np.float32(v))


def seq_sum_f32(vals) -> float:
    acc = np.float32(0.0)
    for v in vals:
        acc = np.float32(acc + np.float32(v))
    return float(acc)


def f16_bits(v: float) -> int:
    return int(np.array([v], dtype=np.float16).view(np.uint16)[0])


def hexb(b: bytes | bytearray | list[int]) -> str:
    return bytes(bytearray(b)).hex()


def i2s_cases():
    cases = []
    x01 = [f32(np.float32(i) * np.float32(0.1)) for i in range(128)]  # (i as f32) * 0.1
    cases.append(dict(
        id="bitlinear.rs:342-360 matvec_all_plus_one_weights", op="i2s_matvec",
        path="dispatch", in_dim=128, out_dim=1, packed=hexb([0xAA] * 32), scale=1.0,
        x=x01, expect=[seq_sum_f32(x01)], tol_abs=1e-4))
    cases.append(dict(
        id="bitlinear.rs:362-380 matvec_all_minus_one_weights", op="i2s_matvec",
        path="dispatch", in_dim=128, out_dim=1, packed=hexb([0x00] * 32), scale=1.0,
        x=x01, expect=[-seq_sum_f32(x01)], tol_abs=1e-4))
    xz = [f32(np.float32(1.0) + np.float32(i) * np.float32(0.01)) for i in range(128)]
    cases.append(dict(
        id="bitlinear.rs:382-397 matvec_all_zero_weights", op="i2s_matvec",
        path="dispatch", in_dim=128, out_dim=1, packed=hexb([0x55] * 32), scale=1.0,
        x=xz, expect=[0.0], tol_abs=0.0))
    cases.append(dict(
        id="bitlinear.rs:399-411 matvec_scale_applied_at_end", op="i2s_matvec",
        path="dispatch", in_dim=128, out_dim=1, packed=hexb([0xAA] * 32), scale=3.5,
        x=[2.0] * 128, expect=[896.0], tol_abs=1e-3))
    cases.append(dict(
        id="bitlinear.rs:413-428 matvec_two_rows_different_patterns", op="i2s_matvec",
        path="dispatch", in_dim=128, out_dim=2, packed=hexb([0xAA] * 32 + [0x00] * 32),
        scale=1.0, x=[1.0] * 128, expect=[128.0, -128.0], tol_abs=1e-4))
    packed = [0x55] * 32
    packed[0] = 0x86
    xm = [0.0] * 128
    xm[0], xm[32], xm[64], xm[96] = 1.0, 10.0, 100.0, 1000.0
    cases.append(dict(
        id="bitlinear.rs:430-465 matvec_column_stride_32_mapping (scalar kernel)",
        op="i2s_matvec", path="scalar", in_dim=128, out_dim=1, packed=hexb(packed), scale=1.0,
        x=xm, expect=[991.0], tol_abs=1e-4))
    xs = [f32(np.sin(np.float32(i))) for i in range(128)]
    cases.append(dict(
        id="bitlinear.rs:514-524 matvec_is_deterministic_for_same_inputs", op="i2s_deterministic",
        path="dispatch", in_dim=128, out_dim=1, packed=hexb([0xAA] * 32), scale=1.0, x=xs))
    # Rejections (bitlinear.rs:484-512): shape errors are checked before any work.
    cases.append(dict(
        id="bitlinear.rs:504-512 matvec_rejects_in_dim_not_multiple_of_128", op="i2s_reject",
        in_dim=64, out_dim=1, packed=hexb([0xAA] * 32), scale=1.0, x=[0.0] * 64))
    unpack_expect = [0] * 128
    unpack_expect[0], unpack_expect[32], unpack_expect[64], unpack_expect[96] = 1, -1, 0, 1
    cases.append(dict(
        id="bitlinear.rs:526-548 unpack_row_matches_packing", op="i2s_unpack",
        in_dim=128, out_dim=1, packed=hexb(packed), row=0, expect=unpack_expect))
    return cases


def quant_cases():
    return [
        dict(id="bitlinear_sparse.rs:205-212 quantize_absmax_basic", op="absmax_i8",
             x=[1.0, -0.5, 0.0, 0.25], expect_scale=f32(np.float32(1.0) / np.float32(127.0)),
             scale_tol=1e-9, expect_q={"0": 127, "2": 0}),
        dict(id="bitlinear_sparse.rs:214-219 quantize_all_zero_returns_unit_scale",
             op="absmax_i8", x=[0.0, 0.0, 0.0], expect_scale=1.0, scale_tol=0.0,
             expect_q={"0": 0, "1": 0, "2": 0}),
    ]


def q6k_ones_block() -> list[int]:
    # q6_k.rs:244-250
    return [0x11] * 128 + [0xAA] * 64 + [1] * 16 + list(struct.pack("<H", 0x3C00))


def q6k_cases():
    cases = []
    cases.append(dict(id="q6_k.rs:252-257 decodes_exact_ones_block", op="q6k_dequant",
                      row=hexb(q6k_ones_block()), n=256, expect_all=1.0))
    blk = [0] * 210
    blk[0] = 0xF0
    blk[32] = 0xE1
    blk[128] = 0xE4
    for i in range(16):
        blk[192 + i] = i + 1
    blk[200] = (-2) & 0xFF
    blk[64] = 0x0F
    blk[160] = 0x03
    blk[208:210] = list(struct.pack("<H", 0x3C00))
    cases.append(dict(id="q6_k.rs:259-280 decodes_pinned_upstream_bit_and_scale_mapping",
                      op="q6k_dequant", row=hexb(blk), n=256,
                      expect_at={"0": -32.0, "32": -45.0, "64": 75.0, "96": 210.0, "128": -62.0}))
    x = [f32(np.float32(i) / np.float32(32.0) - np.float32(4.0)) for i in range(256)]
    deq = [1.0] * 256
    expected = seq_sum_f32([np.float32(a) * np.float32(b) for a, b in zip(deq, x)])
    cases.append(dict(id="q6_k.rs:282-292 direct_dot_matches_dequantized_dot", op="q6k_dot",
                      row=hexb(q6k_ones_block()), x=x, expect_scalar_exact=expected,
                      expect=expected, tol_abs=1e-3))
    xin = [f32(np.sin(np.float32(i) * np.float32(0.173)) * np.float32(5.0)
               - np.float32(i % 11) * np.float32(0.2)) for i in range(512)]
    probe = [f32(np.cos(np.float32(i) * np.float32(0.311)) * np.float32(2.0)
                 + np.float32(i % 5)) for i in range(512)]
    cases.append(dict(id="q6_k.rs:294-324 sse2_dot_matches_scalar_with_cancellation",
                      op="q6k_quantize_dot", x=xin, probe=probe, rel_tol=1e-5))
    xr = [f32(np.sin(np.float32(i) * np.float32(0.37)) * np.float32(3.0)
              + np.float32(i % 7) * np.float32(0.1)) for i in range(512)]
    cases.append(dict(id="q6_k.rs:326-341 quantize_roundtrip_has_small_error",
                      op="q6k_roundtrip", x=xr, max_error=0.15))

    def q6k_const_block(scale: int) -> list[int]:
        # linear.rs:388-394
        return [0x11] * 128 + [0xAA] * 64 + [scale] * 16 + list(struct.pack("<H", f16_bits(1.0)))
    cases.append(dict(id="linear.rs:396-411 q6_k_rectangular_matvec_matches_hand_result",
                      op="q6k_matvec", in_dim=256, out_dim=2,
                      w=hexb(q6k_const_block(1) + q6k_const_block(2)), x=[1.0] * 256,
                      expect=[256.0, 512.0], tol_abs=0.0))
    return cases


def q8_block(scale: float, values) -> list[int]:
    # q8_0.rs:111-115
    return list(struct.pack("<H", f16_bits(scale))) + [int(v) & 0xFF for v in values]


def q8_cases():
    cases = []
    cases.append(dict(id="q8_0.rs:117-125 dequantizes_signed_values_with_per_block_scale",
                      op="q8_dequant", row=hexb(q8_block(0.5, range(-16, 16))), n=32,
                      expect_at={"0": -8.0, "16": 0.0, "31": 7.5}))
    row = q8_block(0.25, [v - 16 for v in range(32)])
    x = [f32(np.float32(v) / np.float32(7.0)) for v in range(32)]
    deq = [np.float32(0.25) * np.float32(v - 16) for v in range(32)]
    expected = seq_sum_f32([np.float32(w) * np.float32(v) for w, v in zip(deq, x)])
    cases.append(dict(id="q8_0.rs:127-139 direct_dot_matches_dequantized_dot", op="q8_dot",
                      row=hexb(row), x=x, expect=expected, tol_abs=1e-5))
    data = []
    for bi in range(4):
        data += q8_block(0.125 * (bi + 1), [((v * 17 + bi * 11) % 127) - 63 for v in range(32)])
    xin = [f32((np.float32((v * 29) % 101) - np.float32(50.0)) / np.float32(13.0))
           for v in range(128)]
    cases.append(dict(id="q8_0.rs:141-156 dispatched_dot_matches_scalar_across_blocks",
                      op="q8_dot_vs_scalar", row=hexb(data), x=xin, tol_abs=1e-3))
    nan_row = list(struct.pack("<H", 0x7E00)) + [0] * 32
    cases.append(dict(id="q8_0.rs:158-163 rejects_non_finite_scale", op="q8_reject",
                      row=hexb(nan_row), x=[0.0] * 32))
    w = q8_block(0.5, [2] * 32) + q8_block(0.25, [-4] * 32)
    cases.append(dict(id="linear.rs:337-357 q8_0_rectangular_matvec_matches_hand_result",
                      op="q8_matvec", in_dim=32, out_dim=2, w=hexb(w), x=[1.0] * 32,
                      expect=[32.0, -32.0], tol_abs=0.0))
    return cases


def misc_cases():
    return [
        dict(id="lm_head.rs:220-226 argmax_returns_index_of_largest", op="argmax",
             cases=[[[0.1, 0.5, 0.3], 1], [[], None], [[0.5], 0], [[1.0, 1.0], 0]]),
        dict(id="primitives.rs:459-473 f16_known_values", op="f16",
             cases=[[0x0000, 0.0], [0x3C00, 1.0], [0xBC00, -1.0], [0x4000, 2.0],
                    [0x3800, 0.5], [0x7C00, "inf"], [0xFC00, "-inf"], [0x7E00, "nan"],
                    [0x8000, "-0.0"]]),
        dict(id="primitives.rs:475-483 f16_smallest_subnormal_is_finite_and_positive",
             op="f16", cases=[[0x0001, float(2.0 ** -24)]]),
        dict(id="bitlinear.rs:334-340 ternary_code_table", op="ternary",
             cases=[[0, -1], [1, 0], [2, 1], [3, 0]]),
        dict(id="tensor.rs:415-425,476-489 layout byte counts", op="byte_len",
             cases=[["Q6_K", [256, 1], 210], ["Q6_K", [512, 3], 1260],
                    ["Q6_K", [2560, 128256], 269337600], ["Q6_K", [128, 2], None],
                    ["Q8_0", [32, 2], 68], ["Q8_0", [64, 3], 204], ["Q8_0", [16, 2], None],
                    ["I2_S", [6912, 2560], 4423680], ["I2_S", [2560, 6912], 4423680],
                    ["I2_S", [2560, 2560], 1638400], ["I2_S", [2560, 640], 409600]]),
    ]


def main() -> None:
    cases = i2s_cases() + quant_cases() + q6k_cases() + q8_cases() + misc_cases()
    with open(OUT, "w") as f:
        json.dump({"source": "project-willamette v0.14.0 unit tests (transcribed)",
                   "cases": cases}, f, indent=1)
    print(f"wrote {len(cases)} cases to {OUT}")


if __name__ == "__main__":
    main()
