"""Whole-network W4A8 inference engine for LSQ ResNets on one GPU.

Compiles a ResNet built from LSQ layers (``lsq_resnet``) — or the same model
after ``convert_lsq_modules(model, convert_conv=True)`` swapped its INT4
layers for ``Int4WeightInt8ActConv2d`` — into a fixed chain of libw4a8 calls:

  images f32 NCHW --s2d+quantise--> int8 [B,112,112,16]
    --4x4 conv (the 7x7/s2 stem re-indexed, W8) + BN + ReLU + 3x3/s2 max pool,
      one launch--> pooled f32 + codes
    --per block: conv1 -> codes, [downsample -> f32 identity],
                 conv2/conv3 (+identity, ReLU) -> codes (+ f32 when needed)
    --avgpool+quantise--> int8 [B, C] --W8 GEMM--> logits f32 [B, classes]

Activations between layers are LSQ codes (int8 NHWC), produced by the
previous layer's epilogue with the consumer's (s_a, qn, qp): exactly the
quantisation the consumer would apply to the fp32 value. Residual
identities stay float32, as in the reference's converted model where BN,
ReLU and the residual add run in float32. BatchNorm is folded into each
epilogue: alpha = f32((s_a*s_w) * gamma/sqrt(var+eps)),
beta = f32((bias-mean) * gamma/sqrt(var+eps) + beta_bn).

All buffers are allocated once for a fixed batch; ``forward`` can replay
the chain as one CUDA graph.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Tuple

import torch
import torch.nn as nn

import int4_int8_ext as ext
from quant_pipeline.ops.int4_conv2d import Int4WeightInt8ActConv2d
from quant_pipeline.quantization.int4_pack import pack_int4_weights, unpack_int4_weights

QParams = Tuple[float, int, int]  # (s_a, qn, qp)


@dataclass
class ConvSpec:
    """A conv layer reduced to integer weights and a folded epilogue."""
    w_codes: torch.Tensor      # int8 OHWI codes [o, kh, kw, c]
    w_bits: int                # 4 or 8
    stride: int
    pad: int
    qin: QParams               # input activation quantisation
    alpha: torch.Tensor        # f32 [o]
    beta: torch.Tensor         # f32 [o]
    kernel_weight: Optional[torch.Tensor] = None  # device weights in kernel order
    cin_pad: int = 0


def _fold(s_a: float, s_w, bias: Optional[torch.Tensor], bn: Optional[nn.BatchNorm2d], o: int):
    s_w64 = s_w.to(torch.float64) if isinstance(s_w, torch.Tensor) else torch.full((o,), float(s_w),
                                                                                    dtype=torch.float64)
    b = bias.detach().to(torch.float64).cpu() if bias is not None else torch.zeros(o, dtype=torch.float64)
    if bn is not None:
        mult = bn.weight.detach().cpu().to(torch.float64) / torch.sqrt(
            bn.running_var.detach().cpu().to(torch.float64) + bn.eps)
        shift = (b - bn.running_mean.detach().cpu().to(torch.float64)) * mult + bn.bias.detach().cpu().to(
            torch.float64)
    else:
        mult, shift = torch.ones(o, dtype=torch.float64), b
    alpha = ((torch.tensor(s_a, dtype=torch.float64) * s_w64.cpu()) * mult).to(torch.float32)
    return alpha, shift.to(torch.float32)


def conv_spec(layer: nn.Module, bn: Optional[nn.BatchNorm2d]) -> ConvSpec:
    """Reads an LSQ QuantConv2d (float weights + steps) or a converted
    Int4WeightInt8ActConv2d (packed weights + steps)."""
    if isinstance(layer, Int4WeightInt8ActConv2d):
        o, c = layer.out_channels, layer.in_channels
        kh, kw = layer.kernel_size
        flat = unpack_int4_weights(layer.weight_packed.detach().cpu())[:, : c * kh * kw]
        w = flat.reshape(o, c, kh, kw).permute(0, 2, 3, 1).contiguous()
        s_w = layer.w_scale_host
        qin = (layer.a_scale_host, layer.a_qn, layer.a_qp)
        stride, pad, bias, bits = layer.stride[0], layer.padding[0], layer.bias, 4
    else:
        conv = layer.conv
        s_w = float(torch.clamp(layer.w_quant.s.detach(), min=1e-8))
        s_a = float(torch.clamp(layer.a_quant.s.detach(), min=1e-8))
        w = torch.clamp(torch.round(conv.weight.detach().cpu() / s_w), layer.w_quant.qn, layer.w_quant.qp)
        w = w.to(torch.int8).permute(0, 2, 3, 1).contiguous()
        qin = (s_a, layer.a_quant.qn, layer.a_quant.qp)
        stride, pad, bias = conv.stride[0], conv.padding[0], conv.bias
        bits = 4 if (layer.w_quant.qn, layer.w_quant.qp) == (-8, 7) else 8
    alpha, beta = _fold(qin[0], s_w, bias, bn, w.shape[0])
    return ConvSpec(w, bits, stride, pad, qin, alpha, beta)


def _kernel_weights(w_ohwi: torch.Tensor, bits: int, c_pad: int, device) -> torch.Tensor:
    """OHWI codes -> device weights in the conv kernel's order (channel
    groups of 128 outermost when c_pad > 128), row stride a multiple of 16."""
    o, kh, kw, c = w_ohwi.shape
    w = torch.zeros((o, kh, kw, c_pad), dtype=torch.int8)
    w[..., :c] = w_ohwi
    if c_pad > 128:
        w = w.reshape(o, kh * kw, c_pad // 128, 128).permute(0, 2, 1, 3)
    w = w.reshape(o, -1)
    if bits == 4:
        w = pack_int4_weights(w)
    ld = -(-w.shape[1] // 16) * 16
    out = torch.zeros((o, ld), dtype=w.dtype)
    out[:, : w.shape[1]] = w
    return out.to(device)


def stem_s2d_weights(w_codes_ohwi: torch.Tensor) -> torch.Tensor:
    """7x7/s2/p3 weights over c channels -> 4x4/s1 weights over the
    space-to-depth input (channel (dy*2+dx)*c + ch), ky = 2*ty + dy - 1."""
    o, kh, kw, c = w_codes_ohwi.shape
    assert (kh, kw) == (7, 7)
    out = torch.zeros((o, 4, 4, 16), dtype=torch.int8)
    for ty in range(4):
        for tx in range(4):
            for dy in range(2):
                for dx in range(2):
                    ky, kx = 2 * ty + dy - 1, 2 * tx + dx - 1
                    if 0 <= ky < 7 and 0 <= kx < 7:
                        base = (dy * 2 + dx) * c
                        out[:, ty, tx, base:base + c] = w_codes_ohwi[:, ky, kx, :]
    return out


class Activation:
    """A layer output: f32 NHWC tensor (optional) and LSQ code tensors."""

    def __init__(self, shape):
        self.shape = shape  # (n, h, w, c)
        self.f32: Optional[torch.Tensor] = None
        self.codes: Dict[QParams, torch.Tensor] = {}


def _block_layers(block) -> dict:
    d = dict(conv1=conv_spec(block.conv1, block.bn1), conv2=conv_spec(block.conv2, block.bn2))
    if hasattr(block, "conv3"):
        d["conv3"] = conv_spec(block.conv3, block.bn3)
    d["ds"] = conv_spec(block.downsample[0], block.downsample[1]) if block.downsample is not None else None
    return d


class W4A8ResNetEngine:
    """Fixed-batch W4A8 ResNet-18/50 forward on one GPU (see module docstring).

    ``forward(images)`` takes float32 NCHW images on the engine's device
    and returns the logits buffer (float32 [batch, classes]); the buffer is
    reused by the next call.
    """

    def __init__(self, model: nn.Module, batch: int, device: Optional[torch.device] = None, image_hw: int = 224,
                 use_graph: bool = True):
        self.device = torch.device(device) if device is not None else torch.device("cuda",
                                                                                    torch.cuda.current_device())
        self.batch = int(batch)
        self.lib = ext.lib()
        self.steps: List[Callable[[int], None]] = []
        self.meta: List[dict] = []  # per launch: name, algorithmic ops and bytes
        self.launches = 0
        self._keep: list = []
        self.use_graph = use_graph
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.graphs: List[torch.cuda.CUDAGraph] = []
        with torch.cuda.device(self.device):
            self._build(model, image_hw)

    # ------------------------------------------------------------ planning
    def _buf(self, shape, dtype) -> torch.Tensor:
        t = torch.empty(shape, dtype=dtype, device=self.device)
        self._keep.append(t)
        return t

    def _add(self, fn, args: tuple, what: str, ops: float = 0.0, nbytes: float = 0.0) -> None:
        self._keep.append(args)
        self.meta.append({"name": what, "ops": float(ops), "bytes": float(nbytes)})

        def step(stream: int, fn=fn, args=args, what=what) -> None:
            rc = fn(*args, stream)
            if rc != 0:
                raise RuntimeError(f"{what} failed: libw4a8 status {rc}")

        self.steps.append(step)
        self.launches += 1

    def _add_conv(self, spec: ConvSpec, x: torch.Tensor, in_shape, out_kind: int, out: torch.Tensor,
                  relu: bool, qout: QParams = (1.0, -128, 127), residual: Optional[torch.Tensor] = None,
                  aux: Optional[torch.Tensor] = None, what: str = "conv",
                  macs_per_pixel: Optional[int] = None,
                  out_hw: Optional[Tuple[int, int]] = None, pool: bool = False) -> Tuple[int, int, int, int]:
        """``out_hw`` overrides the symmetric-padding output size (the
        space-to-depth stem pads 2 top/left and 1 bottom/right); ``pool``
        fuses the 3x3/s2/p1 max pool, so ``out``/``aux`` are pooled."""
        n, h, w, c = in_shape
        o, kh, kw, _ = spec.w_codes.shape
        if out_hw is None:
            ho = (h + 2 * spec.pad - kh) // spec.stride + 1
            wo = (w + 2 * spec.pad - kw) // spec.stride + 1
        else:
            ho, wo = out_hw
        oh_, ow_ = ((ho - 1) // 2 + 1, (wo - 1) // 2 + 1) if pool else (ho, wo)
        for name, t in (("out", out), ("residual", residual), ("aux", aux)):
            if t is not None and tuple(t.shape) != (n, oh_, ow_, o):
                raise ValueError(f"{what}: {name} buffer {tuple(t.shape)} != output {(n, oh_, ow_, o)}")
        if tuple(x.shape) != (n, h, w, c):
            raise ValueError(f"{what}: input buffer {tuple(x.shape)} != {(n, h, w, c)}")
        pix, opix = n * ho * wo, n * oh_ * ow_
        ops = 2.0 * pix * (macs_per_pixel if macs_per_pixel is not None else o * kh * kw * c)
        nbytes = n * h * w * c + opix * o * out.element_size() + o * kh * kw * c * spec.w_bits / 8
        nbytes += (opix * o * 4 if residual is not None else 0) + (opix * o * 4 if aux is not None else 0)
        # 4-bit weights whose int8 form exceeds ext.CONV_STREAMED_W4_BYTES
        # cannot stay resident in shared memory (ResNet-18: the 3x3 convs of
        # layers 3-4): the conv kernel would re-expand the same nibbles for
        # every output tile. They are expanded once here and streamed as int8
        # codes (same values, same int32 sums).
        bits = spec.w_bits
        if bits == 4 and o * kh * kw * c > ext.CONV_STREAMED_W4_BYTES:
            bits = 8
        wk = _kernel_weights(spec.w_codes, bits, c, self.device)
        alpha = spec.alpha.to(self.device)
        beta = spec.beta.to(self.device)
        kind = ext.W_INT4 if bits == 4 else ext.W_INT8
        epi = ext.make_epilogue(out_kind, alpha=alpha, beta=beta, residual=residual, res_ld=o, relu=relu,
                                out_scale=qout[0], qn=qout[1], qp=qout[2], aux=aux, aux_ld=o)
        self._keep += [wk, alpha, beta, epi]
        if kh == 1 and kw == 1 and spec.stride == 1 and spec.pad == 0:
            self._add(self.lib.w4a8_gemm, (x.data_ptr(), c, wk.data_ptr(), wk.stride(0), kind, n * h * w, o, c,
                                           ctypes.byref(epi), out.data_ptr(), o), what, ops, nbytes)
        else:
            geom = ext.ConvGeom(n, h, w, c, kh, kw, spec.stride, spec.pad, spec.pad, ho, wo, o, ext.LAYOUT_NHWC, o,
                                int(pool))
            self._keep.append(geom)
            self._add(self.lib.w4a8_conv2d, (x.data_ptr(), wk.data_ptr(), kind, wk.stride(0), ctypes.byref(geom),
                                             ctypes.byref(epi), out.data_ptr()), what, ops, nbytes)
        return n, ho, wo, o

    def _add_requant(self, src_f32: torch.Tensor, dst: torch.Tensor, q: QParams) -> None:
        rows = src_f32.numel() // src_f32.shape[-1]
        c = src_f32.shape[-1]
        self._add(self.lib.w4a8_quantize_rows, (src_f32.data_ptr(), c, dst.data_ptr(), c, rows, c, q[0], q[1], q[2]),
                  "requant")

    def _build(self, model: nn.Module, image_hw: int) -> None:
        B = self.batch
        stem = conv_spec(model.conv1, model.bn1)
        blocks = [_block_layers(b) for st in (model.layer1, model.layer2, model.layer3, model.layer4) for b in st]
        fc = model.fc

        def consumers_of(i: int):
            """Quant params and f32 need of the activation feeding block i
            (i == len(blocks): the classifier's average pool)."""
            if i == len(blocks):
                return [], True
            b = blocks[i]
            params = [b["conv1"].qin]
            if b["ds"] is not None and b["ds"].qin not in params:
                params.append(b["ds"].qin)
            return params, (b["ds"] is None) or len(params) > 1

        # Stem: s2d + quantise, then the fused conv + pool below.
        s_a, qn, qp = stem.qin
        # Two input slots: a graph is captured per slot so the next batch can
        # be uploaded into one slot while the other is being consumed.
        self.inputs = [self._buf((B, 3, image_hw, image_hw), torch.float32) for _ in range(2)]
        self.images = self.inputs[0]
        self._slot = 0
        h2 = image_hw // 2
        s2d = self._buf((B, h2, h2, 16), torch.int8)
        s2d_args = (s2d.data_ptr(), B, 3, image_hw, image_hw, 16, s_a, qn, qp)
        self._keep.append(s2d_args)

        def s2d_step(stream: int, fn=self.lib.w4a8_s2d_quantize, args=s2d_args) -> None:
            rc = fn(self.inputs[self._slot].data_ptr(), *args, stream)
            if rc != 0:
                raise RuntimeError(f"s2d failed: libw4a8 status {rc}")

        self.steps.append(s2d_step)
        self.meta.append({"name": "s2d", "ops": 0.0, "bytes": float(B * 3 * image_hw * image_hw * 4 + s2d.numel())})
        self.launches += 1
        stem4 = ConvSpec(stem_s2d_weights(stem.w_codes), stem.w_bits, 1, 2, stem.qin, stem.alpha, stem.beta)
        o = stem.w_codes.shape[0]
        kh0, kw0, c0 = stem.w_codes.shape[1:]
        hp = (h2 - 1) // 2 + 1
        params, need_f32 = consumers_of(0)
        act = Activation((B, hp, hp, o))
        act.codes[params[0]] = self._buf(act.shape, torch.int8)
        act.f32 = self._buf(act.shape, torch.float32) if (need_f32 or len(params) > 1) else None
        # Stem conv + BN + ReLU + 3x3/s2 max pool in one launch: pooled codes
        # for the first block and the pooled float32 identity.
        self._add_conv(stem4, s2d, (B, h2, h2, 16), ext.OUT_S8, act.codes[params[0]], relu=True, qout=params[0],
                       aux=act.f32, what="stem+maxpool", macs_per_pixel=o * kh0 * kw0 * c0, out_hw=(h2, h2),
                       pool=True)
        for q in params[1:]:
            act.codes[q] = self._buf(act.shape, torch.int8)
            self._add_requant(act.f32, act.codes[q], q)

        for i, b in enumerate(blocks):
            act = self._add_block(i, b, act, consumers_of(i + 1))

        # Classifier: mean pool + quantise -> W8 GEMM -> logits.
        fc_w_s = float(torch.clamp(fc.w_quant.s.detach(), min=1e-8))
        fc_a = (float(torch.clamp(fc.a_quant.s.detach(), min=1e-8)), fc.a_quant.qn, fc.a_quant.qp)
        n, h, w, c = act.shape
        ldq = -(-c // 16) * 16
        pooled = self._buf((B, ldq), torch.int8)
        pooled.zero_()
        self._add(self.lib.w4a8_avgpool_quantize, (act.f32.data_ptr(), pooled.data_ptr(), ldq, B, h * w, c,
                                                   fc_a[0], fc_a[1], fc_a[2]), "avgpool")
        wq = torch.clamp(torch.round(fc.linear.weight.detach().cpu() / fc_w_s), fc.w_quant.qn, fc.w_quant.qp)
        classes = wq.shape[0]
        bits = 4 if (fc.w_quant.qn, fc.w_quant.qp) == (-8, 7) else 8
        wk = wq.to(torch.int8)
        if bits == 4:
            wk = pack_int4_weights(wk)
        ldw = -(-wk.shape[1] // 16) * 16
        wdev = torch.zeros((classes, ldw), dtype=wk.dtype)
        wdev[:, : wk.shape[1]] = wk
        wdev = wdev.to(self.device)
        alpha, beta = _fold(fc_a[0], fc_w_s, fc.linear.bias, None, classes)
        alpha, beta = alpha.to(self.device), beta.to(self.device)
        self.logits = self._buf((B, classes), torch.float32)
        epi = ext.make_epilogue(ext.OUT_F32, alpha=alpha, beta=beta)
        self._keep += [wdev, alpha, beta, epi]
        self._add(self.lib.w4a8_gemm, (pooled.data_ptr(), ldq, wdev.data_ptr(), ldw,
                                       ext.W_INT4 if bits == 4 else ext.W_INT8, B, classes, c, ctypes.byref(epi),
                                       self.logits.data_ptr(), classes), "fc")

    def _add_block(self, i: int, b: dict, x: Activation, next_consumers) -> Activation:
        n, h, w, c = x.shape
        tag = f"block{i}"
        last = "conv3" if "conv3" in b else "conv2"
        # Inner convs: ReLU, codes for the following conv.
        inner = ["conv1", "conv2"] if last == "conv3" else ["conv1"]
        cur, cur_shape = x.codes[b["conv1"].qin], x.shape
        for j, name in enumerate(inner):
            spec = b[name]
            nxt = b[inner[j + 1]] if j + 1 < len(inner) else b[last]
            o = spec.w_codes.shape[0]
            ho = (cur_shape[1] + 2 * spec.pad - spec.w_codes.shape[1]) // spec.stride + 1
            wo = (cur_shape[2] + 2 * spec.pad - spec.w_codes.shape[2]) // spec.stride + 1
            out = self._buf((n, ho, wo, o), torch.int8)
            self._add_conv(spec, cur, cur_shape, ext.OUT_S8, out, relu=True, qout=nxt.qin, what=f"{tag}.{name}")
            cur, cur_shape = out, (n, ho, wo, o)
        # Identity: f32 block input or the folded downsample conv.
        spec = b[last]
        o = spec.w_codes.shape[0]
        ho = (cur_shape[1] + 2 * spec.pad - spec.w_codes.shape[1]) // spec.stride + 1
        wo = (cur_shape[2] + 2 * spec.pad - spec.w_codes.shape[2]) // spec.stride + 1
        if b["ds"] is not None:
            identity = self._buf((n, ho, wo, o), torch.float32)
            self._add_conv(b["ds"], x.codes[b["ds"].qin], x.shape, ext.OUT_F32, identity, relu=False,
                           what=f"{tag}.downsample")
        else:
            identity = x.f32
        params, need_f32 = next_consumers
        y = Activation((n, ho, wo, o))
        y.f32 = self._buf(y.shape, torch.float32) if need_f32 else None
        if params:
            y.codes[params[0]] = self._buf(y.shape, torch.int8)
            self._add_conv(spec, cur, cur_shape, ext.OUT_S8, y.codes[params[0]], relu=True, qout=params[0],
                           residual=identity, aux=y.f32, what=f"{tag}.{last}")
        else:
            self._add_conv(spec, cur, cur_shape, ext.OUT_F32, y.f32, relu=True, residual=identity,
                           what=f"{tag}.{last}")
        for q in params[1:]:
            y.codes[q] = self._buf(y.shape, torch.int8)
            self._add_requant(y.f32, y.codes[q], q)
        return y

    def profile_steps(self, iters: int = 5) -> List[dict]:
        """Average device time of every launch (eager, CUDA events on the
        current stream); returns meta entries extended with ``ms``."""
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream(self.device)
            self.run_steps()
            torch.cuda.synchronize(self.device)
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(self.steps) + 1)]
            tot = [0.0] * len(self.steps)
            for _ in range(iters):
                ev[0].record(stream)
                for i, step in enumerate(self.steps):
                    step(stream.cuda_stream)
                    ev[i + 1].record(stream)
                torch.cuda.synchronize(self.device)
                for i in range(len(self.steps)):
                    tot[i] += ev[i].elapsed_time(ev[i + 1])
        return [dict(m, ms=t / iters) for m, t in zip(self.meta, tot)]

    # ------------------------------------------------------------- running
    def run_steps(self, stream: Optional[int] = None) -> None:
        s = torch.cuda.current_stream(self.device).cuda_stream if stream is None else stream
        for step in self.steps:
            step(s)

    def capture(self) -> None:
        """Runs the chain once eagerly, then captures one CUDA graph per
        input slot."""
        graphs = []
        with torch.cuda.device(self.device):
            self._slot = 0
            self.run_steps()
            torch.cuda.synchronize(self.device)
            for slot in range(len(self.inputs)):
                self._slot = slot
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    self.run_steps()
                graphs.append(g)
            torch.cuda.synchronize(self.device)
        self._slot = 0
        self.graphs = graphs
        self.graph = graphs[0]

    def forward(self, images: Optional[torch.Tensor] = None, slot: int = 0) -> torch.Tensor:
        """images: float32 [batch, 3, H, W] on the engine's device, copied
        into input slot ``slot`` (None: the slot ``self.inputs[slot]`` was
        filled in place). Runs on the current stream."""
        buf = self.inputs[slot]
        if images is not None and images.data_ptr() != buf.data_ptr():
            if images.shape != buf.shape:
                raise ValueError(f"expected images {tuple(buf.shape)}, got {tuple(images.shape)}")
            buf.copy_(images, non_blocking=True)
        with torch.cuda.device(self.device):
            if self.use_graph:
                if self.graph is None:
                    self.capture()
                self.graphs[slot].replay()
            else:
                self._slot = slot
                self.run_steps()
                self._slot = 0
        return self.logits

    def infer_host(self, batches, out: Optional[List[torch.Tensor]] = None,
                   copy_stream: Optional[torch.cuda.Stream] = None,
                   post: Optional[Callable[[torch.Tensor], None]] = None) -> List[torch.Tensor]:
        """Serving loop over host batches (pinned float32 [batch, 3, H, W]):
        batch i+1 is uploaded on ``copy_stream`` into the free input slot
        while batch i runs; logits come back into ``out[i]`` (pinned host
        tensors, allocated when absent). ``post(logits)``, when given, runs
        on the compute stream after each forward (e.g. the data-parallel
        logits gather). Returns ``out``; completion is ordered on the current
        stream (synchronise before reading)."""
        batches = list(batches)
        if out is None:
            out = [torch.empty(tuple(self.logits.shape), dtype=torch.float32).pin_memory() for _ in batches]
        with torch.cuda.device(self.device):
            if self.use_graph and self.graph is None:
                self.capture()
            compute = torch.cuda.current_stream(self.device)
            copy_stream = copy_stream or torch.cuda.Stream(self.device)
            copied = [torch.cuda.Event() for _ in self.inputs]
            consumed = [torch.cuda.Event() for _ in self.inputs]
            start = torch.cuda.Event()
            start.record(compute)
            copy_stream.wait_event(start)

            def upload(i: int) -> None:
                slot = i % len(self.inputs)
                with torch.cuda.stream(copy_stream):
                    if i >= len(self.inputs):
                        copy_stream.wait_event(consumed[slot])
                    self.inputs[slot].copy_(batches[i], non_blocking=True)
                    copied[slot].record(copy_stream)

            if batches:
                upload(0)
            for i in range(len(batches)):
                slot = i % len(self.inputs)
                if i + 1 < len(batches):
                    upload(i + 1)
                compute.wait_event(copied[slot])
                self.forward(slot=slot)
                consumed[slot].record(compute)
                if post is not None:
                    post(self.logits)
                out[i].copy_(self.logits, non_blocking=True)
        return out

    __call__ = forward

    def release(self) -> None:
        """Drops the CUDA graphs (before destroying process groups / exit)."""
        self.graph = None
        self.graphs = []
