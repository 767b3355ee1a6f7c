"""The allocation-free split-K GEMM entry point (w4a8_gemm_splitk_noalloc).

Some callers cannot allocate device memory: plugins and serving runtimes
whose device memory belongs to the host application's pool or fixed budget,
where cudaMalloc can fail and cudaMalloc / cudaFree synchronise the device.
This entry point takes only inputs and outputs. Its int32 partial sums live in
a fixed device array inside the library, so two calls in a row must each clear
it. Both calls are checked bit-exact against the workspace-taking entry point
(w4a8_gemm_splitk) and the oracle. This file is collected last and must pass
on its own as well as after the other tests.
"""
import ctypes

import numpy as np
import pytest
import torch

import int4_int8_ext as ext
from oracle import oracle as orc
from tests.helpers import assert_equal, rand_i4, rand_i8, rng, to_dev

pytestmark = pytest.mark.gpu


def _noalloc(xd, wd, m, n, k, epi, out):
    return ext.lib().w4a8_gemm_splitk_noalloc(xd.data_ptr(), xd.stride(0), wd.data_ptr(), wd.stride(0), ext.W_INT4, m,
                                              n, k, ctypes.byref(epi), out.data_ptr(), out.stride(0),
                                              torch.cuda.current_stream().cuda_stream)


def _with_workspace(xd, wd, m, n, k, epi, out):
    nbytes = ext.splitk_workspace_bytes(m, n, k, ext.W_INT4)
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=xd.device)
    return ext.lib().w4a8_gemm_splitk(xd.data_ptr(), xd.stride(0), wd.data_ptr(), wd.stride(0), ext.W_INT4, m, n, k,
                                      ctypes.byref(epi), out.data_ptr(), out.stride(0), ws.data_ptr(), nbytes,
                                      torch.cuda.current_stream().cuda_stream)


def test_noalloc_two_calls_match_workspace_entry(cuda):
    m, n, k = 37, 1000, 2048  # 9..64 tokens and >= 16 k-blocks: the split-K path
    assert ext.splitk_workspace_bytes(m, n, k, ext.W_INT4) == m * n * 4
    for call in range(2):
        g = rng(4000 + call)
        x = rand_i8(g, (m, k))
        w = rand_i4(g, (n, k))
        alpha = g.uniform(1e-5, 1e-4, n).astype(np.float32)
        beta = g.normal(0, 0.1, n).astype(np.float32)
        bp = orc.pack_int4(w)
        xd, wd = to_dev(x, cuda), to_dev(bp, cuda)
        epi = ext.make_epilogue(ext.OUT_F32, alpha=to_dev(alpha, cuda), beta=to_dev(beta, cuda), relu=True)
        got = torch.full((m, n), float("nan"), dtype=torch.float32, device=cuda)
        ref = torch.full((m, n), float("nan"), dtype=torch.float32, device=cuda)
        assert _noalloc(xd, wd, m, n, k, epi, got) == 0
        assert _with_workspace(xd, wd, m, n, k, epi, ref) == 0
        torch.cuda.synchronize()
        assert torch.equal(got, ref), f"call {call}"
        assert_equal(got, orc.epilogue(orc.int4_int8_gemm(x, bp), alpha, beta, relu=True), f"oracle call {call}")
    assert ext.device_error() == 0


def test_noalloc_rejects_beyond_scratch(cuda):
    m, n, k = 64, (ext.NOALLOC_SCRATCH_BYTES // (4 * 64)) + 16, 2048  # M * N * 4 above the scratch size
    x = torch.zeros((m, k), dtype=torch.int8, device=cuda)
    w = torch.zeros((n, k // 2), dtype=torch.uint8, device=cuda)
    out = torch.empty((m, n), dtype=torch.int32, device=cuda)
    epi = ext.make_epilogue(ext.OUT_S32)
    assert _noalloc(x, w, m, n, k, epi, out) == ext.ERR_ARG


def test_noalloc_unsplit_shape_beyond_scratch_runs(cuda):
    """A shape with enough output tiles runs unsplit and never touches the
    scratch array, so M * N * 4 above its size is accepted; results equal
    w4a8_gemm."""
    m, n, k = 256, 8192, 1024
    assert m * n * 4 > ext.NOALLOC_SCRATCH_BYTES and ext.splitk_workspace_bytes(m, n, k, ext.W_INT4) == 0
    g = rng(4100)
    x = rand_i8(g, (m, k))
    bp = orc.pack_int4(rand_i4(g, (n, k)))
    xd, wd = to_dev(x, cuda), to_dev(bp, cuda)
    epi = ext.make_epilogue(ext.OUT_S32)
    got = torch.zeros((m, n), dtype=torch.int32, device=cuda)
    assert _noalloc(xd, wd, m, n, k, epi, got) == 0
    torch.cuda.synchronize()
    assert_equal(got, orc.int4_int8_gemm(x, bp), "unsplit noalloc")
