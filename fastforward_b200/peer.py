"""Peer memory for the tensor-parallel engine: the buffers through which the ranks' kernels
read each other's o_proj / down_proj partial sums and per-token activation maxima over
NVLink (CUDA IPC mappings between the one-process-per-GPU ranks; plain loads, stores and
atomics, no multicast).

Per rank: two fp32 planes [nslots, H] (the row-parallel GEMMs' partial outputs, used by
consecutive reductions in turn, so a rank never overwrites a plane that a peer may still be
reading: every reduction in between is a handshake that follows the peer's read), two
activation-maximum buffers [world, nslots], the handshake flags [world, nslots] and the
rank's own call counts [nslots].  The handles are exchanged once with the process group;
`ffb_add_rmsnorm_peers` / `ffb_quantize_fp8_peers` take the mapped pointers.
"""
import ctypes

import torch

from . import _lib as L
from ._lib import call


class PeerBuffers:
    def __init__(self, group, rank, world, nslots, hidden, device):
        import torch.distributed as dist
        if world > L.MAX_PEERS:
            raise ValueError(f"at most {L.MAX_PEERS} tensor-parallel ranks")
        self.rank, self.world, self.nslots = rank, world, nslots
        self.device = device
        self._own, self._opened = [], []
        sizes = [world * nslots * 4,                                  # flags
                 nslots * hidden * 4, nslots * hidden * 4,           # planes 0, 1
                 world * nslots * 4, world * nslots * 4]             # amax 0, 1
        handles = []
        with torch.cuda.device(device):
            for nbytes in sizes:
                p = ctypes.c_void_p()
                h = ctypes.create_string_buffer(64)
                call("ffb_peer_alloc", ctypes.c_size_t(nbytes), ctypes.byref(p), h)
                self._own.append(p.value)
                handles.append(h.raw)
            gathered = [None] * world
            dist.all_gather_object(gathered, handles, group=group)
            ptrs = []  # ptrs[r][i]: rank r's buffer i as mapped here
            for r in range(world):
                if r == rank:
                    ptrs.append(list(self._own))
                    continue
                row = []
                for h in gathered[r]:
                    p = ctypes.c_void_p()
                    call("ffb_peer_open", ctypes.create_string_buffer(h, 64), ctypes.byref(p))
                    self._opened.append(p.value)
                    row.append(p.value)
                ptrs.append(row)
            self.local = torch.zeros(nslots, dtype=torch.int32, device=device)
        flags = (ctypes.c_void_p * L.MAX_PEERS)(*[ptrs[r][0] for r in range(world)])
        self.sync = L.PeerSync(flags=flags, local=self.local.data_ptr(), rank=rank, world=world, nslots=nslots)
        self.planes = [(ctypes.c_void_p * world)(*[ptrs[r][1 + k] for r in range(world)]) for k in (0, 1)]
        self.amax = [(ctypes.c_void_p * world)(*[ptrs[r][3 + k] for r in range(world)]) for k in (0, 1)]
        self.own_plane = [self._own[1], self._own[2]]

    def close(self):
        for p in self._opened:
            call("ffb_peer_close", ctypes.c_void_p(p))
        for p in self._own:
            call("ffb_peer_free", ctypes.c_void_p(p))
        self._opened, self._own = [], []


class DevicePtr:
    """A raw device pointer where the engine's launch helpers expect a tensor."""
    is_cuda = True

    def __init__(self, p):
        self.p = p

    def data_ptr(self):
        return self.p
