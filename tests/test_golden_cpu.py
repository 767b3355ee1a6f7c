"""Oracle and host-side drop-ins vs golden vectors produced by the reference's
own Python code (tests/golden/make_golden.py). CPU only."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle as orc

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name):
    return np.load(GOLDEN / name)


def test_oracle_pack_matches_reference():
    d = load("pack.npz")
    assert np.array_equal(orc.pack_int4(d["w"]), d["packed"])
    assert np.array_equal(orc.unpack_int4(d["all_bytes"]), d["unpacked_all"])
    assert np.array_equal(orc.unpack_int4(d["packed"]), d["w"])
    assert d["pair"][0, 0] == 0xA4 and orc.pack_int4(np.array([[4, -6]]))[0, 0] == 0xA4


def test_pack_module_matches_reference():
    from quant_pipeline.quantization import pack_int4_weights, unpack_int4_weights

    d = load("pack.npz")
    assert np.array_equal(pack_int4_weights(torch.from_numpy(d["w"])).numpy(), d["packed"])
    assert np.array_equal(unpack_int4_weights(torch.from_numpy(d["all_bytes"])).numpy(), d["unpacked_all"])
    with pytest.raises(ValueError):
        pack_int4_weights(torch.tensor([[8, 0]], dtype=torch.int8))
    with pytest.raises(ValueError):
        pack_int4_weights(torch.tensor([[1, 2, 3]], dtype=torch.int8))
    with pytest.raises(TypeError):
        pack_int4_weights(torch.tensor([[1.0, 2.0]]))


def test_conv_module_weight_padding_matches_reference():
    from quant_pipeline.ops import Int4WeightInt8ActConv2d

    d = load("module_pack.npz")
    for name, (cin, cout, k) in {"c3k3": (3, 8, 3), "c3k5": (3, 4, 5), "c16k3": (16, 8, 3)}.items():
        m = Int4WeightInt8ActConv2d(cin, cout, (k, k), (1, 1), (k // 2, k // 2), (1, 1), 1, 0.01, 0.05, 0, 127,
                                    out_dtype=torch.float32)
        m.load_int4_weight(torch.from_numpy(d[f"{name}_w"]))
        assert np.array_equal(m.weight_packed.numpy(), d[f"{name}_packed"]), name


def test_adapter_conversion_matches_reference():
    import sys
    sys.path.insert(0, str(GOLDEN))
    from lsq_standin import build_standin
    from quant_pipeline.integration import convert_lsq_modules

    d = load("adapter.npz")
    model = build_standin(0)
    for k, v in model.state_dict().items():
        assert np.array_equal(v.numpy(), d[f"float::{k}"]), k
    results = convert_lsq_modules(model, convert_conv=True)
    want = json.loads((GOLDEN / "adapter.json").read_text())
    got = [dict(name=r.name, module_type=r.module_type, converted=r.converted, reason=r.reason) for r in results]
    assert got == want
    sd = model.state_dict()
    ref_keys = sorted(k[len("conv::"):] for k in d.files if k.startswith("conv::"))
    assert sorted(sd.keys()) == ref_keys
    for k in ref_keys:
        assert np.array_equal(sd[k].numpy(), d[f"conv::{k}"]), k


def test_oracle_conv_paths_match_reference():
    d = load("conv_paths.npz")
    cases = {"k3s2": (2, 1), "k1s2": (2, 0), "k7s2": (2, 3), "k5s1": (1, 2)}
    for name, (s, p) in cases.items():
        y = orc.conv_unfold_path(d[f"{name}_x"], d[f"{name}_w"], 0.05, 0.0123, -128, 127, s, p,
                                 bias=d[f"{name}_bias"])
        assert np.array_equal(y, d[f"{name}_y"]), name


def test_oracle_gemm_known_answer():
    d = load("gemm.npz")
    assert np.array_equal(orc.gemm_s32(d["a"], d["b8"]), d["c8"])
    assert np.array_equal(orc.int4_int8_gemm(d["a"], d["b4_packed"]), d["c4"])


def test_oracle_lowering_equals_unfold_for_symmetric_range():
    g = np.random.default_rng(0)
    x = g.normal(0, 2, (2, 5, 6, 7)).astype(np.float32)
    w = g.integers(-8, 8, (4, 5, 3, 3)).astype(np.int8)
    flat = np.concatenate([w.reshape(4, -1), np.zeros((4, 1), np.int8)], 1)
    a = orc.conv3x3_s1_p1(x, orc.pack_int4(flat), 0.05, 0.02, -127, 127)
    b = orc.conv_unfold_path(x, w, 0.05, 0.02, -127, 127, 1, 1)
    assert np.array_equal(a, b)


def test_oracle_resnet_matches_lsq_fake_quant():
    """The integer model equals the LSQ fake-quant float model up to float
    rounding (which can move single activation codes)."""
    from oracle import resnet_oracle as ro
    from quant_pipeline.runtime.lsq_resnet import build_lsq_resnet, synthetic_images

    model = build_lsq_resnet("resnet18")
    x = synthetic_images(2, seed=3)
    got = ro.resnet_forward(model, x.numpy())
    with torch.no_grad():
        want = model(x).numpy()
    assert ro.top1_agreement(got, want) == 1.0
    assert ro.rel_err(got, want) < 2e-2
