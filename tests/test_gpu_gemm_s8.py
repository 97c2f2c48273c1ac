"""Prefill GEMM over expanded int8 ternary weights (wl_dev_i2s_expand +
wl_dev_i2s_gemm_s8_f32: warp-specialised persistent tcgen05 kernel) against
the oracle of the reference's per-token matvec.  Bar: int32 accumulators and
f32 outputs bit-exact (the tensor core's int32 sums are exact in any order).
"""
import numpy as np
import pytest

import oracle
from project_willamette_b200 import synth
from project_willamette_b200._abi import lib

pytestmark = pytest.mark.gpu


def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda")


def _expand(torch, packed, in_dim, out_dim):
    L = lib()
    pd = _dev(torch, packed)
    t = torch.empty(L.wl_i2s_expanded_bytes(in_dim, out_dim), dtype=torch.int8, device="cuda")
    assert L.wl_dev_i2s_expand(pd.data_ptr(), in_dim, out_dim, t.data_ptr(),
                               torch.cuda.current_stream().cuda_stream) == 0, L.wl_last_error()
    return t


def test_expand_matches_reference_code_map():
    import torch
    rng = np.random.default_rng(5)
    for in_dim, out_dim in [(128, 3), (2560, 17), (6912, 5)]:
        packed = synth.i2s_packed(rng, in_dim, out_dim, code3_fraction=0.05)
        t = _expand(torch, packed, in_dim, out_dim).cpu().numpy().reshape(out_dim, in_dim)
        for r in range(out_dim):
            assert np.array_equal(t[r], oracle.i2s_unpack_row(packed, in_dim, out_dim, r)), r


@pytest.mark.parametrize("in_dim,out_dim,m", [(2560, 2560, 16), (2560, 640, 33), (640, 1000, 128),
                                              (512, 64, 200), (6912, 2560, 130),
                                              (2560, 6912, 256), (128, 3, 40), (1024, 300, 48)])
def test_gemm_s8_bit_exact(in_dim, out_dim, m):
    import torch
    L = lib()
    rng = np.random.default_rng(in_dim * 7 + out_dim + m)
    packed = synth.i2s_packed(rng, in_dim, out_dim, code3_fraction=0.01 if out_dim == 300 else 0.0)
    scale = synth.i2s_scale(rng)
    X = synth.activations(rng, m, in_dim)
    X[1] = 0.0
    X[m // 2, 7] = 1e5
    t = _expand(torch, packed, in_dim, out_dim)
    xd = _dev(torch, X)
    y = torch.full((m, out_dim), float("nan"), device="cuda")
    acc = torch.zeros((m, out_dim), dtype=torch.int32, device="cuda")
    ws = torch.empty(L.wl_i2s_gemm_workspace_bytes(m, in_dim), dtype=torch.uint8, device="cuda")
    assert L.wl_dev_i2s_gemm_s8_f32(t.data_ptr(), scale, in_dim, out_dim, m, xd.data_ptr(),
                                    y.data_ptr(), acc.data_ptr(), ws.data_ptr(),
                                    torch.cuda.current_stream().cuda_stream) == 0, L.wl_last_error()
    torch.cuda.synchronize()
    RY, racc, _ = oracle.i2s_gemm_rows(packed, scale, in_dim, out_dim, X, n_threads=0)
    assert np.array_equal(acc.cpu().numpy(), racc)
    got = y.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), RY.view(np.uint32))


def test_gemm_s8_config3_full_size_sampled():
    """Benchmark config 3, M = 2048 x (6912 x 2560): sampled tokens against the
    oracle, every token through y(-X) = -y(X)."""
    import torch
    L = lib()
    rng = np.random.default_rng(0x5EED + 3)
    in_dim, out_dim, m = 2560, 6912, 2048
    packed = synth.i2s_packed(rng, in_dim, out_dim)
    scale = synth.i2s_scale(rng)
    X = synth.activations(rng, m, in_dim)
    t = _expand(torch, packed, in_dim, out_dim)
    ws = torch.empty(L.wl_i2s_gemm_workspace_bytes(m, in_dim), dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    outs = []
    for sign in (1.0, -1.0):
        xd = _dev(torch, sign * X)
        y = torch.empty((m, out_dim), device="cuda")
        acc = torch.empty((m, out_dim), dtype=torch.int32, device="cuda")
        assert L.wl_dev_i2s_gemm_s8_f32(t.data_ptr(), scale, in_dim, out_dim, m, xd.data_ptr(),
                                        y.data_ptr(), acc.data_ptr(), ws.data_ptr(), s) == 0
        torch.cuda.synchronize()
        outs.append(acc.cpu().numpy())
    sample = np.array([0, 1, 127, 128, 1000, 2047])
    RY, racc, _ = oracle.i2s_gemm_rows(packed, scale, in_dim, out_dim, X[sample], n_threads=0)
    assert np.array_equal(outs[0][sample], racc)
    assert np.array_equal(outs[1], -outs[0])
