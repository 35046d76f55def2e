"""Input packing on the GPU (`ffb_pack_rgb`, `ffb_pack_rgb_batch`) and single-packet
staging (`fastforward_b200.staging.Packet`).  Bar: bit-exact against the reference's own
outputs (golden fixtures) and against the oracle on the canvas sizes the reference's
runtimes use (square 256/320/512 and the rectangles of its aspect policies)."""
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from fastforward_b200 import _lib as L
from fastforward_b200 import ops, staging
from tests._util import assert_bytes_equal

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_ops.pt"


def test_pack_matches_reference_golden():
    for c in torch.load(GOLDEN, weights_only=False)["pack_rgb"]:
        rgb = c["rgb"].to(DEV)
        got = ops.pack_rgb(rgb) if c["kind"] == "square" else ops.pack_rectangle(rgb, c["width"])
        torch.cuda.synchronize()
        assert_bytes_equal(got, c["pixels"], f"{c['kind']} {c['height']}x{c['width']}")
    assert L.device_error() == 0


# square canvases of the reference's side buckets and the rectangles of its aspect
# policies (`_family/depth_geometry.py:7-15`: 32-pixel multiples, e.g. 6x10 and 2x50 cells)
@pytest.mark.parametrize("hw", [(256, 256), (320, 320), (512, 512), (192, 320), (320, 192), (64, 1600),
                                (1600, 64), (128, 512), (32, 32)])
def test_pack_matches_oracle(hw):
    H, W = hw
    g = np.random.default_rng(H * 7919 + W)
    rgb = g.integers(0, 256, (H, W, 3), dtype=np.uint8)
    got = ops.pack_rectangle(torch.from_numpy(rgb).to(DEV))
    torch.cuda.synchronize()
    assert_bytes_equal(got, oracle.pack_rgb(rgb), f"{H}x{W}")


def test_pack_unaligned_canvas_and_batch():
    """A canvas that does not start on a 16-byte boundary takes the byte-load path; a batch
    gives each canvas's rows in order, identical to packing them one by one."""
    H, W, n = 96, 160, 3
    g = np.random.default_rng(3)
    rgb = g.integers(0, 256, (n, H, W, 3), dtype=np.uint8)
    flat = torch.zeros(rgb.size + 16, dtype=torch.uint8, device=DEV)
    off = flat[5:5 + rgb.size].view(n, H, W, 3)
    off.copy_(torch.from_numpy(rgb))
    assert off.data_ptr() % 16 != 0
    got_one = ops.pack_rectangle(off[1])
    batch = ops.pack_rectangle(torch.from_numpy(rgb).to(DEV))
    torch.cuda.synchronize()
    P = (H // 16) * (W // 16)
    assert_bytes_equal(got_one, oracle.pack_rgb(rgb[1]), "unaligned canvas")
    for i in range(n):
        assert_bytes_equal(batch[i * P:(i + 1) * P], oracle.pack_rgb(rgb[i]), f"batch canvas {i}")


def test_pack_rejects_bad_input():
    with pytest.raises(ValueError):
        ops.pack_rectangle(torch.zeros((48, 64, 3), dtype=torch.uint8, device=DEV))
    with pytest.raises(ValueError):
        ops.pack_rgb(torch.zeros((64, 64, 3), dtype=torch.uint8, device=DEV), side=32)
    with pytest.raises(ValueError):  # no CPU path
        ops.pack_rgb(torch.zeros((64, 64, 3), dtype=torch.uint8))


def _request(side, bucket, n, k, seed):
    g = np.random.default_rng(seed)
    picks = np.zeros(9, np.int64)
    picks[:k] = np.sort(g.choice(np.arange(1, n - 1), k, replace=False))
    picks[8] = n - 1
    return dict(rgb=g.integers(0, 256, (side, side, 3), dtype=np.uint8),
                ids=torch.from_numpy(g.integers(0, 150000, n, dtype=np.int64)),
                picks=torch.from_numpy(picks), k=k)


@pytest.mark.parametrize("cls", [staging.Packet, staging.SerialPacket])
def test_packet_stages_a_request_in_one_copy(cls):
    side, bucket = 256, 320
    pk = cls([(side, side, 3), (1, bucket), (9,), (1, 8)], [torch.uint8, torch.int64, torch.int64, torch.bool])
    assert all(v.data_ptr() % 256 == 0 for v in pk.device_views)
    pix = torch.empty(((side // 16) ** 2, 1536), dtype=torch.bfloat16, device=DEV)
    for i, (n, k) in enumerate([(300, 4), (170, 2), (320, 8)]):  # reused packet, shrinking and growing
        r = _request(side, bucket, n, k, seed=i)
        pk.fill(r)
        ops.pack_rgb(pk.device_views[0], side, pixels=pix)  # same stream: ordered after the copy
        torch.cuda.synchronize()
        rgb, ids, picks, mask = (v.cpu() for v in pk.device_views)
        assert np.array_equal(rgb.numpy(), r["rgb"])
        assert torch.equal(ids[0, :n], r["ids"]) and not ids[0, n:].any()
        assert torch.equal(picks, r["picks"])
        assert mask[0, :k].all() and not mask[0, k:].any()
        assert_bytes_equal(pix, oracle.pack_rgb(r["rgb"]), f"packed canvas of request {i}")


def test_packet_stage_generic_views():
    pk = staging.Packet([(5,), (2, 3)], [torch.float32, torch.int16])
    a, b = np.arange(5, dtype=np.float32), np.arange(6, dtype=np.int16).reshape(2, 3)
    pk.stage(a, b)
    torch.cuda.synchronize()
    assert np.array_equal(pk.device_views[0].cpu().numpy(), a)
    assert np.array_equal(pk.device_views[1].cpu().numpy(), b)
    with pytest.raises(ValueError):
        pk.stage(a)
