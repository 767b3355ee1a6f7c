"""Implicit-GEMM NHWC convolution and the reference's conv ops vs the oracle."""
import numpy as np
import pytest
import torch

import int4_int8_ext as ext
from oracle import oracle as orc
from tests.helpers import assert_close, assert_equal, rand_i4, rand_i8, rng, to_dev

pytestmark = pytest.mark.gpu


def kernel_order_weights(w_ohwi: np.ndarray) -> np.ndarray:
    """OHWI weights -> the conv kernel's [o, groups, taps, 128] order (identity for c <= 128)."""
    o, kh, kw, c = w_ohwi.shape
    if c <= 128:
        return w_ohwi.reshape(o, -1)
    g = c // 128
    return w_ohwi.reshape(o, kh * kw, g, 128).transpose(0, 2, 1, 3).reshape(o, -1)


def run_nhwc_conv(cuda, xq, w_ohwi, stride, pad, ho, wo, epi_kw, out_kind, int4=True):
    n, h, w, c = xq.shape
    o, kh, kw, _ = w_ohwi.shape
    wk = kernel_order_weights(w_ohwi)
    if int4:
        wdev = orc.pack_int4(wk)
        ld = -(-wdev.shape[1] // 16) * 16
        wpad = np.zeros((o, ld), np.uint8)
        wpad[:, : wdev.shape[1]] = wdev
        kind = ext.W_INT4
    else:
        ld = -(-wk.shape[1] // 16) * 16
        wpad = np.zeros((o, ld), np.int8)
        wpad[:, : wk.shape[1]] = wk
        kind = ext.W_INT8
    dtype = {ext.OUT_S32: torch.int32, ext.OUT_F32: torch.float32, ext.OUT_S8: torch.int8,
             ext.OUT_F16: torch.float16}[out_kind]
    out = torch.empty((n, ho, wo, o), dtype=dtype, device=cuda)
    geom = ext.ConvGeom(n, h, w, c, kh, kw, stride, pad, pad, ho, wo, o, ext.LAYOUT_NHWC, o)
    epi = ext.make_epilogue(out_kind, **epi_kw)
    ext.conv2d_nhwc(to_dev(xq, cuda), to_dev(wpad, cuda), kind, geom, epi, out)
    return out


CONV_CASES = [
    # n, h, w, c, o, k, stride, pad
    (2, 10, 10, 16, 64, 3, 1, 1),
    (2, 14, 14, 64, 64, 3, 1, 1),
    (1, 56, 56, 64, 64, 3, 1, 1),
    (2, 28, 28, 128, 128, 3, 1, 1),
    (2, 14, 14, 256, 256, 3, 1, 1),
    (2, 7, 7, 512, 512, 3, 1, 1),
    (2, 56, 56, 64, 128, 3, 2, 1),
    (2, 28, 28, 128, 256, 3, 2, 1),
    (2, 14, 14, 256, 512, 3, 2, 1),
    (2, 56, 56, 64, 128, 1, 2, 0),
    (2, 14, 14, 256, 512, 1, 2, 0),
    # two-image tiles (outputs <= 8x8): odd image count, ragged 5x6 / 3x3 outputs, stride 2 phases
    (3, 7, 7, 128, 64, 3, 1, 1),
    (3, 5, 6, 64, 128, 3, 1, 1),
    (5, 13, 11, 128, 128, 3, 2, 1),
    (3, 6, 6, 64, 64, 1, 2, 0),
    (2, 9, 13, 32, 48, 1, 1, 0),
    (2, 11, 9, 32, 80, 3, 1, 1),
    (2, 9, 9, 384, 64, 3, 2, 1),
    # odd tile counts (3 and 15 tiles): the second CTA of the last CTA pair has no tile
    (1, 16, 24, 64, 64, 3, 1, 1),
    (3, 40, 20, 64, 128, 3, 1, 1),
]


@pytest.mark.parametrize("n,h,w,c,o,k,stride,pad", CONV_CASES)
def test_conv_nhwc_s32_bitexact(cuda, n, h, w, c, o, k, stride, pad):
    g = rng(n * 1000 + h * 10 + c + o + k + stride)
    xq = rand_i8(g, (n, h, w, c), 0, 127)
    wt = rand_i4(g, (o, k, k, c))
    ho = (h + 2 * pad - k) // stride + 1
    wo = (w + 2 * pad - k) // stride + 1
    got = run_nhwc_conv(cuda, xq, wt, stride, pad, ho, wo, {}, ext.OUT_S32)
    want = orc.conv_nhwc_s32(xq, wt, stride, pad, pad, ho, wo)
    assert_equal(got, want, f"conv {n},{h},{w},{c}->{o} k{k}s{stride}")
    assert ext.device_error() == 0


@pytest.mark.parametrize("c,stride", [(48, 1), (96, 1), (16, 2)])
def test_conv_channel_rule(cuda, c, stride):
    """c = 48 or 96 is not a halo row width, c = 16 at stride 2 would split a
    32-byte K-step across stride phases: rejected on the host."""
    g = rng(9)
    xq = rand_i8(g, (1, 8, 8, c), 0, 127)
    wt = rand_i4(g, (16, 3, 3, c))
    ho = (8 + 2 - 3) // stride + 1
    with pytest.raises(RuntimeError, match="status 3"):
        run_nhwc_conv(cuda, xq, wt, stride, 1, ho, ho, {}, ext.OUT_S32)


def test_module_matches_reference_golden(cuda):
    """Int4WeightInt8ActConv2d general-path geometries vs outputs of the
    reference module itself (tests/golden/conv_paths.npz)."""
    from pathlib import Path
    from quant_pipeline.ops import Int4WeightInt8ActConv2d

    d = np.load(Path(__file__).resolve().parent / "golden" / "conv_paths.npz")
    cases = {"k3s2": (16, 32, 3, 2, 1), "k1s2": (16, 32, 1, 2, 0), "k7s2": (3, 16, 7, 2, 3), "k5s1": (3, 8, 5, 1, 2)}
    for name, (cin, cout, k, s, p) in cases.items():
        m = Int4WeightInt8ActConv2d(cin, cout, (k, k), (s, s), (p, p), (1, 1), 1, 0.0123, 0.05, -128, 127,
                                    out_dtype=torch.float32, bias=True)
        m.load_int4_weight(torch.from_numpy(d[f"{name}_w"]))
        with torch.no_grad():
            m.bias.copy_(torch.from_numpy(d[f"{name}_bias"]))
        assert np.array_equal(m.weight_packed.numpy(), d[f"{name}_packed"])
        m = m.to(cuda)
        with torch.no_grad():
            y = m(to_dev(d[f"{name}_x"], cuda))
        assert_equal(y, d[f"{name}_y"], f"module {name} vs reference")


def test_module_large_weights_stream_int8(cuda):
    """A conv whose int8 weights exceed CONV_STREAMED_W4_BYTES runs on int8
    codes expanded once from its packed int4 weights; outputs equal the
    4-bit-weight kernel path bit for bit."""
    from quant_pipeline.ops import Int4WeightInt8ActConv2d

    g = rng(43)
    cin = cout = 256
    m = Int4WeightInt8ActConv2d(cin, cout, (3, 3), (1, 1), (1, 1), (1, 1), 1, 0.0123, 0.05, -128, 127,
                                out_dtype=torch.float32, bias=True)
    m.load_int4_weight(torch.from_numpy(g.integers(-8, 8, (cout, cin, 3, 3)).astype(np.int8)))
    with torch.no_grad():
        m.bias.copy_(torch.from_numpy(g.normal(0, 0.1, cout).astype(np.float32)))
    m = m.to(cuda)
    assert cout * 9 * cin > ext.CONV_STREAMED_W4_BYTES
    w8, kind = m._conv_weight()
    assert kind == ext.W_INT8 and w8.dtype == torch.int8
    x = to_dev(g.normal(0, 2, (2, cin, 7, 9)).astype(np.float32), cuda)
    with torch.no_grad():
        y = m(x)
    w4 = ext.repack_oihw_int4(m.weight_packed.contiguous(), cin, 3, 3, cin)
    alpha_s, alpha_t = m._alpha(x.device)
    want = ext.conv_nchw(x, w4, ext.W_INT4, cin, 3, 3, 1, 1, m.a_scale_host, m.a_qn, m.a_qp, alpha_scalar=alpha_s,
                         alpha=alpha_t, bias=m.bias, out_dtype=torch.float32, pad_code_of_zero=m.is_spatial_3x3)
    torch.cuda.synchronize()
    assert torch.equal(y, want)


def test_s2d_quantize_matches_oracle(cuda):
    """fp32 NCHW images -> int8 space-to-depth codes (channel (dy*2+dx)*3+c,
    padded to 16): clamp(rint(x / s)) in IEEE float32, checked on values at
    and next to the half-integer rounding boundaries and past the clamp."""
    g = rng(31)
    n, c, h, w, s, qn, qp = 2, 3, 32, 40, 0.05, -128, 127
    x = g.normal(0, 3, (n, c, h, w)).astype(np.float32)
    half = ((np.arange(-140, 140) + 0.5) * np.float32(s)).astype(np.float32)
    edge = np.concatenate([half, np.nextafter(half, np.float32(np.inf)), np.nextafter(half, np.float32(-np.inf)),
                           np.float32([1e3, -1e3, 6.4, -6.4, 6.45, -6.45])])
    flat = x.reshape(-1)
    flat[:edge.size] = edge
    q = np.clip(np.rint(x / np.float32(s)), qn, qp).astype(np.int8)
    want = np.zeros((n, h // 2, w // 2, 16), np.int8)
    for dy in range(2):
        for dx in range(2):
            for cc in range(c):
                want[..., (dy * 2 + dx) * 3 + cc] = q[:, cc, dy::2, dx::2]
    xd = to_dev(x, cuda)
    got = torch.full((n, h // 2, w // 2, 16), 99, dtype=torch.int8, device=cuda)
    rc = ext.lib().w4a8_s2d_quantize(xd.data_ptr(), got.data_ptr(), n, c, h, w, 16, s, qn, qp,
                                     torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    assert_equal(got, want, "s2d quantize")


def test_stem_s2d_conv(cuda):
    """4x4 conv, pad 2 top/left, 16 channels: the space-to-depth stem."""
    g = rng(77)
    xq = rand_i8(g, (2, 32, 32, 16))
    wt = rand_i8(g, (64, 4, 4, 16))
    got = run_nhwc_conv(cuda, xq, wt, 1, 2, 32, 32, {}, ext.OUT_S32, int4=False)
    assert_equal(got, orc.conv_nhwc_s32(xq, wt, 1, 2, 2, 32, 32), "stem s2d")


def test_conv_fused_requant_epilogue(cuda):
    """Config-2 style layer (reduced batch): 3x3 s1 p1 64->64, per-channel
    scale, bias, ReLU, requant to int8 with scale 0.05."""
    g = rng(2)
    n, h, w, c, o = 4, 56, 56, 64, 64
    xq = rand_i8(g, (n, h, w, c), 0, 127)
    wt = rand_i4(g, (o, 3, 3, c))
    s_w = g.uniform(1e-3, 1e-2, o).astype(np.float32)
    bias = g.normal(0, 0.01, o).astype(np.float32)
    alpha = (np.float64(0.05) * s_w.astype(np.float64)).astype(np.float32)
    acc = orc.conv_nhwc_s32(xq, wt, 1, 1, 1, h, w)
    want = orc.quantize(orc.epilogue(acc, alpha, bias, relu=True), 0.05, 0, 127)
    epi = dict(alpha=to_dev(alpha, cuda), beta=to_dev(bias, cuda), relu=True, out_scale=0.05, qn=0, qp=127)
    got = run_nhwc_conv(cuda, xq, wt, 1, 1, h, w, epi, ext.OUT_S8)
    assert_equal(got, want, "requant conv")


def test_conv3x3_op_matches_oracle(cuda):
    g = rng(3)
    for (n, c, h, w, o) in [(2, 3, 10, 12, 16), (2, 16, 9, 9, 32), (1, 64, 20, 17, 64), (2, 130, 8, 8, 24)]:
        x = g.normal(0, 2, (n, c, h, w)).astype(np.float32)
        k = c * 9 + (c * 9) % 2
        wt = rand_i4(g, (o, k))
        wt[:, c * 9:] = 0
        bp = orc.pack_int4(wt)
        bias = g.normal(0, 0.1, o).astype(np.float32)
        for half in (False, True):
            got = ext.conv3x3_int4_int8_s1_p1(to_dev(x, cuda), to_dev(bp, cuda), 0.05, 0.02, -127, 127,
                                              to_dev(bias, cuda), half)
            want = orc.conv3x3_s1_p1(x, bp, 0.05, 0.02, -127, 127, bias, half)
            assert_equal(got, want, f"conv3x3 op c={c} half={half}")


def test_conv3x3_op_zero_outside_range(cuda):
    """qn > 0: the reference's lowering pads with the code of 0.0 (= qn)."""
    g = rng(4)
    x = g.normal(0, 2, (2, 16, 8, 8)).astype(np.float32)
    wt = rand_i4(g, (32, 144))
    bp = orc.pack_int4(wt)
    got = ext.conv3x3_int4_int8_s1_p1(to_dev(x, cuda), to_dev(bp, cuda), 0.05, 0.02, 3, 100, None, False)
    assert_equal(got, orc.conv3x3_s1_p1(x, bp, 0.05, 0.02, 3, 100, None, False), "qn>0 padding")


def test_conv1x1_op_matches_oracle(cuda):
    g = rng(6)
    for (n, c, h, w, o, sh, sw) in [(2, 64, 14, 14, 128, 2, 2), (2, 32, 9, 11, 16, 1, 1), (1, 16, 10, 10, 32, 3, 2)]:
        x = g.normal(0, 2, (n, c, h, w)).astype(np.float32)
        bp = orc.pack_int4(rand_i4(g, (o, c)))
        bias = g.normal(0, 0.1, o).astype(np.float32)
        got = ext.conv1x1_int4_int8(to_dev(x, cuda), to_dev(bp, cuda), 0.05, 0.02, -128, 127, sh, sw,
                                    to_dev(bias, cuda), False)
        want = orc.conv1x1(x, bp, 0.05, 0.02, -128, 127, sh, sw, bias, False)
        assert_equal(got, want, f"conv1x1 s{sh}{sw}")
        assert_close(got, want, 1e-3)


def test_lower_quantize_3x3_matches_oracle(cuda):
    g = rng(8)
    x = g.normal(0, 2, (2, 5, 7, 6)).astype(np.float32)
    got = ext.lower_quantize_3x3_s1_p1(to_dev(x, cuda), 0.05, -128, 127, 50)
    assert_equal(got, orc.lower_quantize_3x3(x, 0.05, -128, 127, 50), "lowering")
    got = ext.lower_quantize_3x3_s1_p1(to_dev(x, cuda), 0.05, 2, 127, 46)
    assert_equal(got, orc.lower_quantize_3x3(x, 0.05, 2, 127, 46), "lowering qn>0")


@pytest.mark.parametrize("h,w,n,o", [(30, 26, 2, 64), (29, 27, 2, 64), (29, 27, 40, 64), (31, 25, 23, 40)])
def test_conv_fused_maxpool(cuda, h, w, n, o):
    """Stem-style conv with the 3x3/s2/p1 max pool fused into the epilogue;
    alpha has both signs (pooling picks the max or min accumulator). Odd
    sizes put the last pooled row / column's window partly outside the image.
    Two tiles share each accumulator buffer: with 2 images every CTA gets one
    tile (a pair with its second half empty), with 40 and 23 images CTAs get
    several tiles, odd and even counts; 40 output channels leave part of
    the channel lanes idle."""
    g = rng(21 + h + n)
    c = 16
    xq = rand_i8(g, (n, h, w, c))
    wt = rand_i8(g, (o, 4, 4, c))
    alpha = g.uniform(1e-4, 1e-3, o).astype(np.float32)
    alpha[::3] *= -1
    beta = g.normal(0, 0.5, o).astype(np.float32)
    acc = orc.conv_nhwc_s32(xq, wt, 1, 2, 2, h, w)
    y = orc.epilogue(acc, alpha, beta, relu=True)
    pooled = orc.maxpool3x3s2(y)
    ph, pw = pooled.shape[1:3]
    codes = torch.empty((n, ph, pw, o), dtype=torch.int8, device=cuda)
    aux = torch.empty((n, ph, pw, o), dtype=torch.float32, device=cuda)
    wk = to_dev(np.ascontiguousarray(wt.reshape(o, -1)), cuda)
    geom = ext.ConvGeom(n, h, w, c, 4, 4, 1, 2, 2, h, w, o, ext.LAYOUT_NHWC, o, 1)
    alpha_t, beta_t = to_dev(alpha, cuda), to_dev(beta, cuda)
    epi = ext.make_epilogue(ext.OUT_S8, alpha=alpha_t, beta=beta_t, relu=True, out_scale=0.05, qn=0, qp=127,
                            aux=aux, aux_ld=o)
    ext.conv2d_nhwc(to_dev(xq, cuda), wk, ext.W_INT8, geom, epi, codes)
    assert_equal(aux, pooled, "pooled f32")
    assert_equal(codes, orc.quantize(pooled, 0.05, 0, 127), "pooled codes")


def test_maxpool_kernel(cuda):
    g = rng(22)
    x = g.normal(0, 1, (2, 17, 12, 8)).astype(np.float32)
    want = orc.maxpool3x3s2(x)
    yf = torch.empty(want.shape, dtype=torch.float32, device=cuda)
    yq = torch.empty(want.shape, dtype=torch.int8, device=cuda)
    xd = to_dev(x, cuda)
    with torch.cuda.device(cuda):
        rc = ext.lib().w4a8_maxpool3x3s2(xd.data_ptr(), yf.data_ptr(), yq.data_ptr(), 2, 17, 12, 8, want.shape[1],
                                          want.shape[2], 0.05, -128, 127, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    assert_equal(yf, want, "maxpool f32")
    assert_equal(yq, orc.quantize(want, 0.05, -128, 127), "maxpool codes")
