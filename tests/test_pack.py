"""Input packing and staging, host side: the oracle's `pack_rgb` against the reference's own
`pack_rgb` / `pack_rectangle` outputs (tests/golden/reference_ops.pt), the bf16 value table's
independence from the division's last bit, the packet layout of `search_transport.Packet`,
and the C entry's argument checks (no kernel launch)."""
from fractions import Fraction
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from fastforward_b200 import _lib as L
from fastforward_b200 import staging

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_ops.pt"


@pytest.fixture(scope="module")
def ref():
    return torch.load(GOLDEN, weights_only=False)


def test_oracle_pack_matches_reference(ref):
    cases = ref["pack_rgb"]
    assert {c["kind"] for c in cases} == {"square", "rectangle"}
    for c in cases:
        got = oracle.pack_rgb(c["rgb"])
        want = c["pixels"]
        assert got.shape == want.shape == ((c["height"] // 16) * (c["width"] // 16), 1536)
        n = int((got.view(torch.int16) != want.view(torch.int16)).sum())
        assert n == 0, f"{c['kind']} {c['height']}x{c['width']}: {n} elements differ from the reference"
        # every byte value occurs in the fixture
        assert torch.unique(c["rgb"]).numel() == 256


def test_pixel_values_do_not_depend_on_division_rounding():
    """(u - 127.5) / 127.5 = (2u - 255) / 255: for every byte the fp32 quotient is at least
    a few fp32 ulps away from a bf16 rounding boundary, so any fp32 division accurate to
    2 ulps (the GPU's IEEE `__fdiv_rn`, Triton's fp32 `/`, numpy) gives the same bf16."""
    for u in range(256):
        exact = Fraction(2 * u - 255, 255)
        q = np.float32(float(exact))  # nearest fp32 to the exact quotient
        neigh = [q]
        for direction in (np.float32(np.inf), np.float32(-np.inf)):
            x = q
            for _ in range(2):
                x = np.nextafter(x, direction, dtype=np.float32)
                neigh.append(x)
        bf = {torch.tensor(float(v), dtype=torch.float32).to(torch.bfloat16).view(torch.int16).item() for v in neigh}
        assert len(bf) == 1, (u, neigh)


def test_kernel_value_arithmetic_matches_ieee_division():
    """The kernel computes (u - 127.5) * fp32(2/255) (exact byte-to-float and subtraction,
    one rounded product); for all 256 bytes its bf16 equals the bf16 of the IEEE quotient
    (u - 127.5) / 127.5 that the reference and the oracle compute."""
    src = (Path(__file__).resolve().parents[1] / "fastforward_b200" / "csrc" / "pack.cu").read_text()
    assert "TWO_OVER_255 = 0x1.010102p-7f" in src
    k = np.float32(float.fromhex("0x1.010102p-7"))
    lo, hi = np.nextafter(k, np.float32(0)), np.nextafter(k, np.float32(1))
    exact = Fraction(2, 255)
    assert abs(Fraction(float(k)) - exact) <= min(abs(Fraction(float(lo)) - exact), abs(Fraction(float(hi)) - exact))
    u = np.arange(256, dtype=np.uint32)
    m = (u | np.uint32(0x4B000000)).view(np.float32)  # 2^23 + u, as the byte permute builds it
    x = (m - np.float32(8388608.0)) - np.float32(127.5)
    assert np.array_equal(x, u.astype(np.float32) - np.float32(127.5))
    got = torch.from_numpy(x * k).to(torch.bfloat16)
    want = torch.from_numpy(x / np.float32(127.5)).to(torch.bfloat16)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


def test_pack_layout_is_the_patch_merge_order():
    """Hand-checked elements of the packing: patch rows in 2x2 merge-group order, channel
    planes of 512, both temporal copies equal."""
    H, W = 64, 96
    rgb = np.zeros((H, W, 3), np.uint8)
    rgb[40, 70, 1] = 255  # merge group (row 1, column 2), its top-left patch, pixel (8, 6)
    out = oracle.pack_rgb(rgb).float()
    groups_w = W // 32
    gy, gx, my, mx, y0, x0 = 40 // 32, 70 // 32, (40 % 32) // 16, (70 % 32) // 16, 40 % 16, 70 % 16
    p = (gy * groups_w + gx) * 4 + my * 2 + mx
    hot = (out > -1).nonzero().tolist()
    assert hot == [[p, 1 * 512 + 0 * 256 + y0 * 16 + x0], [p, 1 * 512 + 1 * 256 + y0 * 16 + x0]]
    assert out[p, 512 + y0 * 16 + x0] == 1.0 and out.min() == -1.0


def test_packet_layout_of_the_reference_request():
    """The reference's packet for a 256x256 canvas and a 320-token bucket
    (`_legacy/search_runtime.py:118`): views at 256-byte multiples, packed in order."""
    shapes = [(256, 256, 3), (1, 320), (9,), (1, 8)]
    dtypes = [torch.uint8, torch.int64, torch.int64, torch.bool]
    offs, total = staging.layout(shapes, dtypes)
    assert offs == [(0, 196608), (196608, 2560), (199168, 72), (199424, 8)]
    assert total == 199432
    assert (offs, total) == oracle.packet_layout(shapes, dtypes)
    offs2, total2 = staging.layout([(3,), (5,), (1,)], [torch.uint8, torch.float32, torch.int64])
    assert offs2 == [(0, 3), (256, 20), (512, 8)] and total2 == 520


def test_pack_entry_rejects_bad_canvases():
    with pytest.raises(ValueError, match="multiples of 32"):
        L.call("ffb_pack_rgb", 16, 16, 48, 64, None)
    with pytest.raises(ValueError, match="multiples of 32"):
        L.call("ffb_pack_rgb", 16, 16, 0, 64, None)
    with pytest.raises(ValueError, match="NULL"):
        L.call("ffb_pack_rgb", None, 16, 64, 64, None)
    with pytest.raises(ValueError, match="aligned"):
        L.call("ffb_pack_rgb", 16, 18, 64, 64, None)
    with pytest.raises(ValueError, match="canvases"):
        L.call("ffb_pack_rgb_batch", 16, 16, 0, 64, 64, None)
    with pytest.raises(ValueError, match="2\\^30"):
        L.call("ffb_pack_rgb_batch", 16, 16, 1 << 12, 1024, 1024, None)
