"""W4A8 / W8A8 GEMM on the tcgen05 kernel vs the CPU oracle.

Integer outputs are compared bit-exact (the reference's own known-answer
check, benchmarks/benchmark_inference.py:62-79). Float epilogues follow the
documented float32 op order and are compared bit-exact as well; the
contract tolerance for them is rel 1e-3.
"""
import ctypes

import numpy as np
import pytest
import torch

import int4_int8_ext as ext
from oracle import oracle as orc
from tests.helpers import assert_close, assert_equal, rand_i4, rand_i8, rng, to_dev

pytestmark = pytest.mark.gpu

GEMM_SHAPES = [
    (1, 64, 64), (7, 48, 96), (128, 128, 128), (130, 200, 256), (256, 1000, 512),
    (300, 520, 1040), (64, 96, 4096), (513, 257, 384), (32, 1024, 1024), (1, 4096, 4096),
]


@pytest.mark.parametrize("m,n,k", GEMM_SHAPES)
def test_int4_int8_gemm_bitexact(cuda, m, n, k):
    g = rng(m * 7919 + n * 31 + k)
    a = rand_i8(g, (m, k))
    w = rand_i4(g, (n, k))
    bp = orc.pack_int4(w)
    got = ext.int4_int8_gemm(to_dev(a, cuda), to_dev(bp, cuda))
    assert_equal(got, orc.int4_int8_gemm(a, bp), f"int4 gemm {m}x{n}x{k}")
    assert ext.device_error() == 0


@pytest.mark.parametrize("m,n,k", [(1, 64, 64), (7, 48, 80), (130, 200, 256), (256, 1000, 512), (64, 96, 4096)])
def test_int8_int8_gemm_bitexact(cuda, m, n, k):
    g = rng(m + n + k)
    a = rand_i8(g, (m, k))
    b = rand_i8(g, (n, k))
    got = ext.int8_int8_gemm(to_dev(a, cuda), to_dev(b, cuda))
    assert_equal(got, orc.gemm_s32(a, b), f"int8 gemm {m}x{n}x{k}")


def test_gemm_extremes(cuda):
    """Saturating magnitudes: every product at its extreme (|acc| up to 2^20)."""
    m, n, k = 128, 64, 8192
    a = np.full((m, k), -128, np.int8)
    a[1::2] = 127
    w = np.full((n, k), -8, np.int8)
    w[::3] = 7
    bp = orc.pack_int4(w)
    got = ext.int4_int8_gemm(to_dev(a, cuda), to_dev(bp, cuda))
    assert_equal(got, orc.int4_int8_gemm(a, bp), "extremes")


@pytest.mark.parametrize("out_kind", [ext.OUT_F32, ext.OUT_F16, ext.OUT_S8])
def test_fc_layer_epilogue(cuda, out_kind):
    """ResNet-18 classifier shape: X int8 [256,512] x W int4 [1000,512],
    per-channel s_w, s_a = 0.05, bias N(0, 0.01)."""
    g = rng(0)
    x = rand_i8(g, (256, 512))
    w = rand_i4(g, (1000, 512))
    s_w = g.uniform(1e-3, 1e-2, 1000).astype(np.float32)
    bias = g.normal(0, 0.01, 1000).astype(np.float32)
    alpha = (np.float64(0.05) * s_w.astype(np.float64)).astype(np.float32)
    bp = orc.pack_int4(w)
    acc = orc.int4_int8_gemm(x, bp)
    want = orc.epilogue(acc, alpha, bias)
    dtype = {ext.OUT_F32: torch.float32, ext.OUT_F16: torch.float16, ext.OUT_S8: torch.int8}[out_kind]
    out = torch.empty((256, 1000), dtype=dtype, device=cuda)
    alpha_t, bias_t = to_dev(alpha, cuda), to_dev(bias, cuda)
    epi = ext.make_epilogue(out_kind, alpha=alpha_t, beta=bias_t, out_scale=0.01, qn=-128, qp=127)
    ext.gemm(to_dev(x, cuda), to_dev(bp, cuda), ext.W_INT4, 512, epi, out)
    if out_kind == ext.OUT_F32:
        assert_equal(out, want, "fc f32")
    elif out_kind == ext.OUT_F16:
        assert_equal(out, want.astype(np.float16), "fc f16")
    else:
        assert_equal(out, orc.quantize(want, 0.01, -128, 127), "fc s8")


def test_epilogue_residual_relu_aux(cuda):
    g = rng(5)
    m, n, k = 200, 192, 320
    x = rand_i8(g, (m, k), 0, 127)
    w = rand_i4(g, (n, k))
    alpha = g.uniform(1e-4, 1e-3, n).astype(np.float32)
    beta = g.normal(0, 0.1, n).astype(np.float32)
    res = g.normal(0, 1.0, (m, n)).astype(np.float32)
    bp = orc.pack_int4(w)
    y = orc.epilogue(orc.int4_int8_gemm(x, bp), alpha, beta, res, relu=True)
    q = orc.quantize(y, 0.05, 0, 127)
    out = torch.empty((m, n), dtype=torch.int8, device=cuda)
    aux = torch.empty((m, n), dtype=torch.float32, device=cuda)
    epi = ext.make_epilogue(ext.OUT_S8, alpha=to_dev(alpha, cuda), beta=to_dev(beta, cuda),
                            residual=to_dev(res, cuda), res_ld=n, relu=True, out_scale=0.05, qn=0, qp=127,
                            aux=aux, aux_ld=n)
    ext.gemm(to_dev(x, cuda), to_dev(bp, cuda), ext.W_INT4, k, epi, out)
    assert_equal(aux, y, "aux")
    assert_equal(out, q, "requant")


@pytest.mark.parametrize("pad", [4, 8])
def test_epilogue_padded_float_rows(cuda, pad):
    """Residual, float side output and float32 output with row strides of
    n + pad floats: pad 4 keeps rows 16-byte but not 32-byte aligned (the
    16-byte vector path), pad 8 keeps 32-byte rows (the 32-byte path)."""
    g = rng(6 + pad)
    m, n, k = 136, 160, 256
    x = rand_i8(g, (m, k), 0, 127)
    w = rand_i4(g, (n, k))
    alpha = g.uniform(1e-4, 1e-3, n).astype(np.float32)
    beta = g.normal(0, 0.1, n).astype(np.float32)
    res = np.zeros((m, n + pad), np.float32)
    res[:, :n] = g.normal(0, 1.0, (m, n))
    bp = orc.pack_int4(w)
    y = orc.epilogue(orc.int4_int8_gemm(x, bp), alpha, beta, res[:, :n], relu=True)
    aux = torch.full((m, n + pad), float("nan"), dtype=torch.float32, device=cuda)
    out = torch.empty((m, n), dtype=torch.int8, device=cuda)
    epi = ext.make_epilogue(ext.OUT_S8, alpha=to_dev(alpha, cuda), beta=to_dev(beta, cuda),
                            residual=to_dev(res, cuda), res_ld=n + pad, relu=True, out_scale=0.05, qn=0, qp=127,
                            aux=aux, aux_ld=n + pad)
    ext.gemm(to_dev(x, cuda), to_dev(bp, cuda), ext.W_INT4, k, epi, out)
    assert_equal(aux[:, :n], y, "aux")
    assert torch.isnan(aux[:, n:]).all(), "aux padding written"
    assert_equal(out, orc.quantize(y, 0.05, 0, 127), "requant")
    yf = torch.full((m, n + pad), float("nan"), dtype=torch.float32, device=cuda)
    epi = ext.make_epilogue(ext.OUT_F32, alpha=to_dev(alpha, cuda), beta=to_dev(beta, cuda),
                            residual=to_dev(res, cuda), res_ld=n + pad, relu=True)
    ext.gemm(to_dev(x, cuda), to_dev(bp, cuda), ext.W_INT4, k, epi, yf[:, :n])
    assert_equal(yf[:, :n], y, "f32 out")
    assert torch.isnan(yf[:, n:]).all(), "out padding written"


def test_linear_op_matches_oracle(cuda):
    g = rng(11)
    m, k, o = 37, 200, 96
    x = g.normal(0, 3, (m, k)).astype(np.float32)
    w = rand_i4(g, (o, k))
    bp = orc.pack_int4(w)
    bias = g.normal(0, 0.1, o).astype(np.float32)
    for half in (False, True):
        got = ext.linear_int4_int8(to_dev(x, cuda), to_dev(bp, cuda), 0.05, 0.0123, -127, 127,
                                   to_dev(bias, cuda), half)
        want = orc.linear(x, bp, 0.05, 0.0123, -127, 127, bias, half)
        assert_equal(got, want, f"linear half={half}")
        assert_close(got, want.astype(np.float32), 1e-3, "linear tolerance")


# One or two tokens run on the TMA-fed GEMV: 16-row groups streamed through a
# shared-memory ring in k-slices of up to 1 KB per row. The cases cover a
# ragged last row group (N % 16), fewer groups than SMs, many groups per CTA,
# rows of one slice, exactly one full slice, a short tail slice (1056-byte
# rows), several slices, strided weight rows (ldw > K/2) and activations
# (lda > K), and the largest K whose activations still leave four stages.
GEMV_CASES = [
    # m, n, k, ldw pad (bytes), lda pad
    (1, 8, 64, 0, 0),
    (2, 33, 128, 0, 0),
    (1, 1000, 2048, 0, 0),
    (2, 1000, 2112, 16, 64),
    (1, 5000, 4096, 0, 0),
    (2, 4100, 8192, 48, 16),
    (1, 300, 65536, 0, 0),
    (2, 40, 65536, 0, 0),
    (1, 40000, 1024, 0, 0),  # 17 units of 16 rows per block, one 512-byte segment per row
    (2, 3000, 3072, 32, 0),
    (1, 24, 1024, 0, 0),  # fewer segments than warps
]


@pytest.mark.parametrize("m,n,k,wpad,apad", GEMV_CASES)
def test_gemv_tma_bitexact(cuda, m, n, k, wpad, apad):
    g = rng(5000 + m * 7 + n + k)
    x = rand_i8(g, (m, k))
    w = rand_i4(g, (n, k))
    bp = orc.pack_int4(w)
    want = orc.int4_int8_gemm(x, bp)
    wbuf = torch.zeros((n, k // 2 + wpad), dtype=torch.uint8, device=cuda)
    wbuf[:, : k // 2] = to_dev(bp, cuda)
    abuf = torch.zeros((m, k + apad), dtype=torch.int8, device=cuda)
    abuf[:, :k] = to_dev(x, cuda)
    out = torch.full((m, n), -7, dtype=torch.int32, device=cuda)
    epi = ext.make_epilogue(ext.OUT_S32)
    ext._check(ext.lib().w4a8_gemm(abuf.data_ptr(), abuf.stride(0), wbuf.data_ptr(), wbuf.stride(0), ext.W_INT4, m,
                                   n, k, ctypes.byref(epi), out.data_ptr(), out.stride(0),
                                   torch.cuda.current_stream().cuda_stream), "w4a8_gemm")
    torch.cuda.synchronize()
    assert_equal(out, want, f"gemv {m}x{n}x{k}")
    assert ext.device_error() == 0


@pytest.mark.parametrize("m", [1, 2, 5, 37])
def test_gemm_small_m_paths(cuda, m):
    """Small-M INT4 GEMMs: up to 8 tokens run on the CUDA-core GEMV (packed
    weights streamed into registers), 9..64 tokens split K across work units
    (int32 partial sums in a workspace, epilogue after the sum). The fused
    float epilogue with residual, ReLU and float side output, and the int8
    requantisation, must equal the oracle and the workspace-free entry point
    bit for bit."""
    g = rng(900 + m)
    n, k = 1000, 2048
    x = rand_i8(g, (m, k))
    w = rand_i4(g, (n, k))
    alpha = g.uniform(1e-5, 1e-4, n).astype(np.float32)
    beta = g.normal(0, 0.1, n).astype(np.float32)
    res = g.normal(0, 1.0, (m, n)).astype(np.float32)
    bp = orc.pack_int4(w)
    assert ext.splitk_workspace_bytes(m, n, k, ext.W_INT4) == (0 if m <= 8 else m * n * 4)
    y = orc.epilogue(orc.int4_int8_gemm(x, bp), alpha, beta, res, relu=True)
    outs = {}
    for split in (True, False):
        out = torch.empty((m, n), dtype=torch.int8, device=cuda)
        aux = torch.empty((m, n), dtype=torch.float32, device=cuda)
        epi = ext.make_epilogue(ext.OUT_S8, alpha=to_dev(alpha, cuda), beta=to_dev(beta, cuda),
                                residual=to_dev(res, cuda), res_ld=n, relu=True, out_scale=0.05, qn=0, qp=127,
                                aux=aux, aux_ld=n)
        xd, wd = to_dev(x, cuda), to_dev(bp, cuda)
        if split:
            ext.gemm(xd, wd, ext.W_INT4, k, epi, out)
        else:
            ext._check(ext.lib().w4a8_gemm(xd.data_ptr(), xd.stride(0), wd.data_ptr(), wd.stride(0), ext.W_INT4, m,
                                           n, k, ctypes.byref(epi), out.data_ptr(), out.stride(0),
                                           torch.cuda.current_stream().cuda_stream), "w4a8_gemm")
        torch.cuda.synchronize()
        assert_equal(aux, y, f"aux split={split}")
        assert_equal(out, orc.quantize(y, 0.05, 0, 127), f"requant split={split}")
        outs[split] = out
    assert torch.equal(outs[True], outs[False])
    assert ext.device_error() == 0


def test_gemm_cta_pair_ragged(cuda):
    """Large W4 GEMMs run on CTA pairs (256 x 256 tiles, each CTA holding
    half of B); ragged M, N and K exercise the follower's partial rows, a
    partial n-tile and a partial k-block. Rows sampled from every 128-row
    block (both CTAs of each pair) are checked bit-exact."""
    m, n, k = 2300, 2100, 1056
    gen = torch.Generator().manual_seed(2300)
    a = torch.randint(-128, 128, (m, k), dtype=torch.int8, generator=gen)
    w = torch.randint(-8, 8, (n, k), dtype=torch.int8, generator=gen)
    bp = orc.pack_int4(w.numpy())
    got = ext.int4_int8_gemm(a.to(cuda), to_dev(bp, cuda)).cpu().numpy()
    rows = np.unique(np.concatenate([np.arange(0, m, 128), np.arange(127, m, 128), np.arange(61, m, 128),
                                     [m - 1]]))
    want = orc.gemm_s32(a.numpy()[rows], w.numpy())
    assert np.array_equal(got[rows], want)
    assert ext.device_error() == 0


@pytest.mark.parametrize("m", [1, 32, 256, 4096])
@pytest.mark.parametrize("nk", [1024, 4096, 8192])
def test_gemm_sweep_sampled_bitexact(cuda, m, nk):
    """GEMM sweep shapes; int32 checked bit-exact on a seeded row sample."""
    gen = torch.Generator().manual_seed(m * 10 + nk)
    a = torch.randint(-128, 128, (m, nk), dtype=torch.int8, generator=gen)
    w = torch.randint(-8, 8, (nk, nk), dtype=torch.int8, generator=gen)
    bp = orc.pack_int4(w.numpy())
    got = ext.int4_int8_gemm(a.to(cuda), to_dev(bp, cuda)).cpu().numpy()
    rows = np.unique(np.linspace(0, m - 1, num=min(m, 48)).astype(np.int64))
    want = orc.gemm_s32(a.numpy()[rows], w.numpy())
    assert np.array_equal(got[rows], want)
