"""CPU oracle for the input packing and staging in front of the vision tower (TEST
INFRASTRUCTURE: only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU legs use it).

`pack_rgb` restates the reference's Triton kernels `pack_rgb`
(`_legacy/sub10_runtime.py:21-29`) and `pack_rectangle` (`_family/depth_runtime.py:18-25`)
element by element with numpy: output element i of a [(H/16)(W/16), 1536] tensor takes
patch p = i // 1536 and offset d = i % 1536, channel c = d // 512, pixel row
y0 = (d % 256) // 16, column x0 = d % 16 (the two temporal copies d // 256 % 2 read the same
pixel), merge group gy = p // (4 * W/32), gx = (p // 4) % (W/32), quadrant my = (p % 4) // 2,
mx = p % 2, and pixel (gy*32 + my*16 + y0, gx*32 + mx*16 + x0); the value is
(u8 - 127.5) / 127.5 in fp32, stored as bf16 (round to nearest even, as GPU Triton's store
into a bf16 tensor).  Pinned by `tests/golden/make_golden.py`, which runs the reference's
kernels themselves.

`packet_layout` restates the byte layout of `search_transport.Packet`
(`_legacy/search_transport.py:6-16`): views in order, each starting at the next multiple
of 256 bytes.
"""
import numpy as np
import torch

__all__ = ["pack_rgb", "packet_layout", "PATCH_ROW"]

PATCH_ROW = 1536


def pack_rgb(rgb):
    """rgb [H, W, 3] uint8 (numpy or CPU tensor) -> [(H/16)(W/16), 1536] bf16 CPU tensor."""
    a = np.ascontiguousarray(rgb.numpy() if isinstance(rgb, torch.Tensor) else rgb)
    assert a.dtype == np.uint8 and a.ndim == 3 and a.shape[2] == 3
    H, W = a.shape[:2]
    n = (H // 16) * (W // 16) * PATCH_ROW
    i = np.arange(n, dtype=np.int64)
    p, d = i // PATCH_ROW, i % PATCH_ROW
    c, y0, x0 = d // 512, (d % 256) // 16, d % 16
    gw = W // 16
    gy, gx = p // (gw // 2 * 4), (p // 4) % (gw // 2)
    my, mx = (p % 4) // 2, p % 2
    y, x = gy * 32 + my * 16 + y0, gx * 32 + mx * 16 + x0
    raw = a.reshape(-1)[(y * W + x) * 3 + c].astype(np.float32)
    v = (raw - np.float32(127.5)) / np.float32(127.5)
    return torch.from_numpy(v).to(torch.bfloat16).view(-1, PATCH_ROW)


def packet_layout(shapes, dtypes):
    """[(offset, nbytes)] of each view and the total size of a staging packet."""
    out, total = [], 0
    for s, dt in zip(shapes, dtypes):
        nb = torch.empty((), dtype=dt).element_size() * int(np.prod(s, dtype=np.int64))
        total = (total + 255) // 256 * 256
        out.append((total, nb))
        total += nb
    return out, total
