"""Generates the golden fixtures in this directory from the REFERENCE's own
Python code (peihengzju/lsq-lowbit-optimization), imported from the
read-only checkout, whose path is the one required argument. Run where
that checkout exists:

    python tests/golden/make_golden.py <path to the reference checkout>

Fixtures (small .npz / .json files) are committed; tests never import the
reference. What each file pins:
  pack.npz         pack_int4_weights / unpack_int4_weights (int4_pack.py:9-50)
  module_pack.npz  Int4WeightInt8ActConv2d.load_int4_weight K padding (int4_conv2d.py:85-109)
  adapter.npz/json convert_lsq_modules on stand-in LSQ layers (lsq_adapter.py:107-234)
  conv_paths.npz   Int4WeightInt8ActConv2d.forward general path (int4_conv2d.py:171-201)
                   with its GEMM evaluated by the reference's own CPU check
                   formula (benchmarks/benchmark_inference.py:67-76)
  gemm.npz         that check formula on a 64x64x256 slice, int8 and int4
"""
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
if len(sys.argv) != 2 or not (Path(sys.argv[1]) / "quant_pipeline").is_dir():
    sys.exit("usage: make_golden.py <path to the reference checkout (the directory holding quant_pipeline/)>")
sys.path.insert(0, sys.argv[1])

from lsq_standin import build_standin  # noqa: E402
from quant_pipeline.integration import lsq_adapter  # noqa: E402  (reference package)
from quant_pipeline.ops import int4_conv2d as ref_conv  # noqa: E402
from quant_pipeline.ops.int4_conv2d import Int4WeightInt8ActConv2d  # noqa: E402
from quant_pipeline.quantization import pack_int4_weights, unpack_int4_weights  # noqa: E402


def ref_cpu_gemm(a_int8, b_packed):
    """benchmarks/benchmark_inference.py:67-76 pattern: int32 matmul on CPU."""
    return a_int8.to(torch.int32) @ unpack_int4_weights(b_packed).to(torch.int32).t()


def main():
    g = torch.Generator().manual_seed(2024)
    # pack / unpack
    w = torch.randint(-8, 8, (16, 64), dtype=torch.int8, generator=g)
    w[0, :16] = torch.arange(-8, 8, dtype=torch.int8)
    all_bytes = torch.arange(256, dtype=torch.int32).to(torch.uint8).reshape(1, 256)
    np.savez(HERE / "pack.npz", w=w.numpy(), packed=pack_int4_weights(w).numpy(),
             all_bytes=all_bytes.numpy(), unpacked_all=unpack_int4_weights(all_bytes).numpy(),
             pair=pack_int4_weights(torch.tensor([[4, -6]], dtype=torch.int8)).numpy())

    # module weight packing with odd flattened K
    out = {}
    for name, (cin, cout, k) in {"c3k3": (3, 8, 3), "c3k5": (3, 4, 5), "c16k3": (16, 8, 3)}.items():
        m = Int4WeightInt8ActConv2d(cin, cout, (k, k), (1, 1), (k // 2, k // 2), (1, 1), 1, 0.01, 0.05, 0, 127,
                                    out_dtype=torch.float32)
        wi = torch.randint(-8, 8, (cout, cin, k, k), dtype=torch.int8, generator=g)
        m.load_int4_weight(wi)
        out[f"{name}_w"] = wi.numpy()
        out[f"{name}_packed"] = m.weight_packed.numpy()
    np.savez(HERE / "module_pack.npz", **out)

    # adapter conversion of stand-in LSQ layers
    model = build_standin(0)
    floats = {k: v.detach().numpy() for k, v in model.state_dict().items()}
    results = lsq_adapter.convert_lsq_modules(model, convert_conv=True)
    res = [dict(name=r.name, module_type=r.module_type, converted=r.converted, reason=r.reason) for r in results]
    converted = {f"conv::{k}": v.detach().numpy() for k, v in model.state_dict().items()}
    np.savez(HERE / "adapter.npz", **{f"float::{k}": v for k, v in floats.items()}, **converted)
    (HERE / "adapter.json").write_text(json.dumps(res, indent=1))

    # general conv path of the reference module, GEMM by the reference's CPU check formula
    ref_conv.int4_int8_gemm = ref_cpu_gemm
    out = {}
    cases = {"k3s2": (16, 32, 3, 2, 1), "k1s2": (16, 32, 1, 2, 0), "k7s2": (3, 16, 7, 2, 3), "k5s1": (3, 8, 5, 1, 2)}
    for name, (cin, cout, k, s, p) in cases.items():
        m = Int4WeightInt8ActConv2d(cin, cout, (k, k), (s, s), (p, p), (1, 1), 1, 0.0123, 0.05, -128, 127,
                                    out_dtype=torch.float32, bias=True)
        wi = torch.randint(-8, 8, (cout, cin, k, k), dtype=torch.int8, generator=g)
        m.load_int4_weight(wi)
        with torch.no_grad():
            m.bias.copy_(torch.randn(cout, generator=g) * 0.1)
        x = torch.randn((2, cin, 13, 11), generator=g) * 3
        assert not (m.is_spatial_3x3 or m.is_pointwise)
        with torch.no_grad():
            y = m(x)
        out.update({f"{name}_x": x.numpy(), f"{name}_w": wi.numpy(), f"{name}_bias": m.bias.detach().numpy(),
                    f"{name}_packed": m.weight_packed.numpy(), f"{name}_y": y.numpy()})
    np.savez(HERE / "conv_paths.npz", **out)

    # the benchmark's --check known answer, on CPU data
    a = torch.randint(-127, 128, (64, 256), dtype=torch.int8, generator=g)
    b8 = torch.randint(-127, 128, (64, 256), dtype=torch.int8, generator=g)
    b4 = torch.randint(-8, 8, (64, 256), dtype=torch.int8, generator=g)
    bp = pack_int4_weights(b4)
    np.savez(HERE / "gemm.npz", a=a.numpy(), b8=b8.numpy(), b4_packed=bp.numpy(),
             c8=(a.to(torch.int32) @ b8.to(torch.int32).t()).numpy(), c4=ref_cpu_gemm(a, bp).numpy())
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
