"""Host-side logic on CPU: weight re-indexing, C-ABI exports, the reference
ops' argument errors, and the data-parallel gather over gloo ranks."""
import os
import re
import socket
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as orc

ROOT = Path(__file__).resolve().parents[1]


def test_stem_space_to_depth_reindex():
    """7x7/s2/p3 conv == 4x4/s1 conv (pad 2 top/left) over the s2d input."""
    from quant_pipeline.runtime.engine import stem_s2d_weights

    g = np.random.default_rng(0)
    n, h, w, c, o = 2, 18, 14, 3, 8
    x = g.integers(-128, 128, (n, h, w, c)).astype(np.int8)
    w7 = g.integers(-128, 128, (o, 7, 7, c)).astype(np.int8)
    ho, wo = (h + 6 - 7) // 2 + 1, (w + 6 - 7) // 2 + 1
    want = orc.conv_nhwc_s32(x, w7, 2, 3, 3, ho, wo)
    xs = np.zeros((n, h // 2, w // 2, 16), np.int8)
    for dy in range(2):
        for dx in range(2):
            xs[..., (dy * 2 + dx) * c:(dy * 2 + dx + 1) * c] = x[:, dy::2, dx::2, :]
    w4 = stem_s2d_weights(torch.from_numpy(w7)).numpy()
    got = orc.conv_nhwc_s32(xs, w4, 1, 2, 2, ho, wo)
    assert np.array_equal(got, want)


def test_kernel_weight_order_groups_of_128():
    from quant_pipeline.runtime.engine import _kernel_weights

    g = np.random.default_rng(1)
    w = g.integers(-8, 8, (4, 3, 3, 256)).astype(np.int8)
    got = _kernel_weights(torch.from_numpy(w), 4, 256, "cpu").numpy()
    order = w.reshape(4, 9, 2, 128).transpose(0, 2, 1, 3).reshape(4, -1)
    assert np.array_equal(got[:, : order.shape[1] // 2], orc.pack_int4(order))
    assert got.shape[1] % 16 == 0


def test_expand_int4_rows_matches_oracle_packing():
    """Packed int4 rows -> int8 codes (the int8 form large-weight convs stream)."""
    import int4_int8_ext as ext
    g = np.random.default_rng(41)
    w = g.integers(-8, 8, (37, 96), dtype=np.int8)
    packed = torch.from_numpy(orc.pack_int4(w))
    got = ext.expand_int4_rows(packed)
    assert got.dtype == torch.int8 and tuple(got.shape) == (37, 96)
    assert np.array_equal(got.numpy(), w)


def test_c_abi_exports_every_declared_symbol():
    import build_native
    import int4_int8_ext as ext

    build_native.build()
    header = (ROOT / "include" / "w4a8.h").read_text()
    declared = set(re.findall(r"W4A8_API int (w4a8_\w+)\(", header))
    assert len(declared) >= 12
    lib = ext.lib()
    for name in sorted(declared):
        assert hasattr(lib, name), name
    assert set(ext._SIGNATURES) >= declared
    assert lib.w4a8_abi_version() == ext.ABI_VERSION


def test_reference_op_argument_errors():
    import int4_int8_ext as ext

    a = torch.zeros((4, 8), dtype=torch.int8)
    with pytest.raises(RuntimeError, match="a must be a CUDA tensor"):
        ext.int8_int8_gemm(a, a)
    with pytest.raises(RuntimeError, match="x must be a CUDA tensor"):
        ext.linear_int4_int8(torch.zeros(2, 8), torch.zeros((3, 4), dtype=torch.uint8), 0.1, 0.1, -127, 127, None,
                             False)
    with pytest.raises(RuntimeError, match="x must be a CUDA tensor"):
        ext.conv3x3_int4_int8_s1_p1(torch.zeros(1, 2, 3, 3), torch.zeros((3, 9), dtype=torch.uint8), 0.1, 0.1,
                                    -127, 127, None, False)


def test_conv_channel_padding_rule():
    import int4_int8_ext as ext

    assert ext.conv_channels_padded(3) == 16 and ext.conv_channels_padded(3, 2) == 32
    assert ext.conv_channels_padded(48) == 64 and ext.conv_channels_padded(130) == 256
    assert ext.conv_channels_padded(96) == 128 and ext.conv_channels_padded(20) == 32
    assert ext.conv_channels_padded(512) == 512


def test_shard_range_partitions():
    from quant_pipeline.runtime.dp import shard_range

    for total in (0, 1, 7, 256, 2048):
        for world in (1, 2, 3, 8):
            spans = [shard_range(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            assert max(b - a for a, b in spans) - min(b - a for a, b in spans) <= 1


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank: int, world: int, port: int, q) -> None:
    from quant_pipeline.runtime.dp import gather_logits, shard_range
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        total = 6 * world
        a, b = shard_range(total, world, rank)
        full = torch.arange(total * 5, dtype=torch.float32).reshape(total, 5)
        out = gather_logits(full[a:b].clone())
        q.put((rank, bool(torch.equal(out, full))))
    finally:
        dist.destroy_process_group()


def test_dp_gather_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    results = sorted(q.get(timeout=5) for _ in range(2))
    assert results == [(0, True), (1, True)]
