"""Single-packet host->device staging of a request's raw inputs.

Mirrors `search_transport.Packet` (`_legacy/search_transport.py:5-25`) and its serial
variant `SerialPacket` (`_legacy/lower_runtime.py:13-26`): one pinned host buffer and one
device buffer of the same size hold every input of a request (RGB canvas, token ids, pick
rows, choice mask) at 256-byte aligned offsets, so staging a request is ONE
`cudaMemcpyAsync` instead of one copy per tensor.  `host_views` / `device_views` are typed
views into the two buffers (the device views are what a captured graph reads).

B200 notes: the device buffer is allocated once per packet (graph-stable addresses); the
copy is issued on the caller's current stream, so the graph replay or the `ffb_pack_rgb`
launch that follows on the same stream is ordered after it without a host wait; `done`
records the copy so the host buffer is only rewritten after the previous copy has read it.
"""
import numpy as np
import torch

ALIGN = 256


def layout(shapes, dtypes):
    """[(offset, nbytes)] of each view (each at the next multiple of 256 bytes) and the
    packet's total size in bytes (`search_transport.py:7-10`)."""
    out, total = [], 0
    for s, dt in zip(shapes, dtypes):
        nb = torch.empty((), dtype=dt).element_size() * int(np.prod(s, dtype=np.int64))
        total = (total + ALIGN - 1) // ALIGN * ALIGN
        out.append((total, nb))
        total += nb
    return out, total


class Packet:
    """Pinned host / device packet with typed views.

    shapes, dtypes: one entry per view.  `fill(g)` expects the reference's four views
    (rgb [S, S, 3] uint8, ids [1, b] int64, picks [9] int64, mask [1, 8] bool) and a
    request dict g with `rgb`, `ids`, `picks`, `k`; other layouts use `stage(*arrays)`."""

    def __init__(self, shapes, dtypes, device=None):
        if len(shapes) != len(dtypes) or not shapes:
            raise ValueError("one dtype per shape, at least one view")
        self.device_ = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        offsets, total = layout(shapes, dtypes)
        self.offsets = offsets
        self.host = torch.empty(total, dtype=torch.uint8, pin_memory=True)
        self.device = torch.empty(total, dtype=torch.uint8, device=self.device_)
        self.host.zero_()
        self.host_views = tuple(self.host[o:o + n].view(d).view(s) for (o, n), d, s in zip(offsets, dtypes, shapes))
        self.device_views = tuple(self.device[o:o + n].view(d).view(s)
                                  for (o, n), d, s in zip(offsets, dtypes, shapes))
        self.numpy_views = tuple(x.numpy() for x in self.host_views)
        self.done = torch.cuda.Event()
        self.pending = False

    def _reuse(self):
        """Waits until the previous copy out of the host buffer has completed."""
        if self.pending and not self.done.query():
            self.done.synchronize()

    def _send(self):
        self.device.copy_(self.host, non_blocking=True)
        self.done.record()
        self.pending = True

    def fill(self, g):
        """Stages one request (`search_transport.py:18-25`): the canvas, the ids zero-padded
        to the bucket, the pick rows, the first k mask entries set; then one host->device
        copy on the current stream."""
        self._reuse()
        rgb, ids, picks, mask = self.numpy_views
        n = len(g["ids"])
        if n > ids.shape[1]:
            raise ValueError(f"{n} ids exceed the packet's bucket {ids.shape[1]}")
        if not 0 <= int(g["k"]) <= mask.shape[1]:
            raise ValueError("k outside the mask")
        rgb[...] = _np(g["rgb"])
        ids.fill(0)
        ids[0, :n] = _np(g["ids"])
        picks[...] = _np(g["picks"])
        mask.fill(False)
        mask[0, :int(g["k"])] = True
        self._send()

    def stage(self, *arrays):
        """Copies one array per view (same shapes) into the host buffer, then one
        host->device copy on the current stream."""
        if len(arrays) != len(self.numpy_views):
            raise ValueError(f"{len(self.numpy_views)} arrays expected")
        self._reuse()
        for dst, a in zip(self.numpy_views, arrays):
            dst[...] = _np(a)
        self._send()


class SerialPacket(Packet):
    """The serial API's packet (`_legacy/lower_runtime.py:13-26`): the caller guarantees
    that the previous request has completed (a lock plus a blocking read of its answer), so
    `fill` does not wait on the previous copy."""

    def _reuse(self):
        pass


def _np(a):
    return a.numpy() if isinstance(a, torch.Tensor) else np.asarray(a)
