"""Whole-network W4A8 ResNet on the GPU engine vs the CPU integer oracle.

Gates: logits within rel 1e-3 (max-abs over max-abs) and top-1 agreement
>= 99.9% (all images at these batch sizes). The engine follows the oracle's
op order, so the logits are expected to match bit for bit; that is
reported but the gate is the tolerance. The comparison with the converted
model's own module-by-module forward, at batch 256, is in
test_headline_gpu.py.
"""
import numpy as np
import pytest
import torch

from oracle import resnet_oracle as ro
from quant_pipeline.integration import convert_lsq_modules
from quant_pipeline.ops import Int4WeightInt8ActConv2d
from quant_pipeline.runtime.engine import W4A8ResNetEngine
from quant_pipeline.runtime.lsq_resnet import build_lsq_resnet, synthetic_images

pytestmark = pytest.mark.gpu


def _check(got: torch.Tensor, want: np.ndarray, what: str):
    g = got.detach().cpu().numpy()
    err = ro.rel_err(g, want)
    agree = ro.top1_agreement(g, want)
    print(f"{what}: rel_err={err:.3e} top1={agree:.4f} bit_exact={np.array_equal(g, want)}")
    assert err <= 1e-3, (what, err)
    assert agree >= 0.999, (what, agree)


@pytest.mark.parametrize("arch,batch", [("resnet18", 4), ("resnet50", 2)])
def test_engine_matches_oracle(cuda, arch, batch):
    model = build_lsq_resnet(arch)
    images = synthetic_images(batch, seed=1)
    want = ro.resnet_forward(model, images.numpy())
    eng = W4A8ResNetEngine(model, batch, device=cuda, use_graph=False)
    _check(eng.forward(images.to(cuda)), want, f"{arch} eager")
    eng_g = W4A8ResNetEngine(model, batch, device=cuda, use_graph=True)
    _check(eng_g.forward(images.to(cuda)), want, f"{arch} graph")
    _check(eng_g.forward(images.to(cuda)), want, f"{arch} graph replay")
    eng_g.release()


def test_engine_from_converted_model(cuda):
    """convert_lsq_modules (the reference's adapter flow) then the engine:
    INT4 layers come from packed weight buffers, 8-bit stem/fc are skipped
    by the adapter and read from the LSQ layers."""
    model = build_lsq_resnet("resnet18", seed=3)
    images = synthetic_images(2, seed=4)
    want = ro.resnet_forward(model, images.numpy())
    results = convert_lsq_modules(model, convert_conv=True)
    converted = [r for r in results if r.converted]
    skipped = [r.name for r in results if not r.converted]
    assert len(converted) == 19 and sorted(skipped) == ["conv1", "fc"]
    assert sum(isinstance(m, Int4WeightInt8ActConv2d) for m in model.modules()) == 19
    eng = W4A8ResNetEngine(model, 2, device=cuda, use_graph=True)
    _check(eng.forward(images.to(cuda)), want, "converted resnet18")
    eng.release()


def test_infer_host_pipeline_matches_oracle(cuda):
    """Overlapped serving loop: three host batches through the two input
    slots; every batch's logits equal the oracle's for that batch."""
    model = build_lsq_resnet("resnet18", seed=7)
    eng = W4A8ResNetEngine(model, 2, device=cuda, use_graph=True)
    batches = [synthetic_images(2, seed=s).pin_memory() for s in (10, 11, 12)]
    outs = eng.infer_host(batches)
    torch.cuda.synchronize()
    for i, (b, o) in enumerate(zip(batches, outs)):
        _check(o, ro.resnet_forward(model, b.numpy()), f"infer_host batch {i}")
    eng.release()
