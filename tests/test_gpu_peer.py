"""The tensor-parallel peer-memory kernels on ONE GPU (`ffb_add_rmsnorm_peers`,
`ffb_quantize_fp8_peers`): with world = 1 they equal the plain kernels; a second rank is
emulated by a local buffer standing in for its flags, whose handshake counts are set ahead
(no kernel ever waits for another launch), which pins the rank-order sum and the maximum
over the ranks' slices; and a handshake that nobody answers gives up after its bounded
wait with the device error word set, leaving the context usable.  The two-GPU engine is
covered by tests/test_gpu_tp.py."""
import ctypes

import pytest
import torch

from fastforward_b200 import _lib as L
from fastforward_b200._lib import call, ptr

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
BF16 = torch.bfloat16
ERR_PEER_TIMEOUT = 1 << 4


def _sync(rank, world, nslots, flags, local):
    arr = (ctypes.c_void_p * L.MAX_PEERS)(*[f.data_ptr() for f in flags])
    return L.PeerSync(flags=arr, local=local.data_ptr(), rank=rank, world=world, nslots=nslots)


def _ptrs(*ts):
    return (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])


def _case(T, H, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(T, H, generator=g).to(BF16).to(DEV)
    w = (1 + 0.1 * torch.randn(H, generator=g)).to(BF16).to(DEV)
    planes = [torch.randn(T, H, generator=g).to(DEV) for _ in range(2)]
    return a, w, planes


@pytest.mark.parametrize("T,H", [(320, 2560), (17, 5120)])
def test_add_rmsnorm_peers_world1_equals_add_rmsnorm(T, H):
    a, w, planes = _case(T, H, 1)
    flags, local = torch.zeros(T, dtype=torch.int32, device=DEV), torch.zeros(T, dtype=torch.int32, device=DEV)
    sync = _sync(0, 1, T, [flags], local)
    outs = {}
    for name in ("plain", "peer"):
        res = torch.empty_like(a)
        q8 = torch.empty(T, H, dtype=torch.uint8, device=DEV)
        qs = torch.empty(T, dtype=torch.float32, device=DEV)
        for _ in range(3):  # the handshake counts advance call after call
            if name == "plain":
                call("ffb_add_rmsnorm", ptr(a), None, ptr(planes[0]), 1, None, 0, 0, ptr(w), 1e-6, ptr(res), None,
                     L.QUANT_ROWWISE, 0.0, ptr(q8), ptr(qs), T, H, L.stream_ptr())
            else:
                pl = _ptrs(planes[0])
                call("ffb_add_rmsnorm_peers", ptr(a), ctypes.addressof(pl), ctypes.addressof(sync), None, 0, 0,
                     ptr(w), 1e-6, ptr(res), None, L.QUANT_ROWWISE, 0.0, ptr(q8), ptr(qs), T, H, L.stream_ptr())
        torch.cuda.synchronize()
        outs[name] = (res.cpu(), q8.cpu(), qs.cpu())
    for x, y in zip(outs["plain"], outs["peer"]):
        assert torch.equal(x.view(torch.uint8), y.view(torch.uint8))
    assert torch.equal(local.cpu(), torch.full((T,), 3, dtype=torch.int32))
    assert L.device_error(clear=True) == 0


def test_add_rmsnorm_peers_two_ranks_sum_in_rank_order():
    """Rank 0 of two: the partial planes are summed (p0 + p1), the split-K sum of the plain
    kernel over the same two planes; its signal lands in rank 1's (stand-in) flags."""
    T, H = 128, 4096
    a, w, planes = _case(T, H, 2)
    own, peer_flags = torch.zeros(2 * T, dtype=torch.int32, device=DEV), torch.zeros(2 * T, dtype=torch.int32,
                                                                                     device=DEV)
    own[T:] = 1  # rank 1 has signalled every slot once
    local = torch.zeros(T, dtype=torch.int32, device=DEV)
    sync = _sync(0, 2, T, [own, peer_flags], local)
    res, out = torch.empty_like(a), torch.empty_like(a)
    pl = _ptrs(*planes)
    call("ffb_add_rmsnorm_peers", ptr(a), ctypes.addressof(pl), ctypes.addressof(sync), None, 0, 0, ptr(w), 1e-6,
         ptr(res), ptr(out), L.QUANT_NONE, 0.0, None, None, T, H, L.stream_ptr())
    both = torch.stack(planes).contiguous()
    res2, out2 = torch.empty_like(a), torch.empty_like(a)
    call("ffb_add_rmsnorm", ptr(a), None, ptr(both), 2, None, 0, 0, ptr(w), 1e-6, ptr(res2), ptr(out2),
         L.QUANT_NONE, 0.0, None, None, T, H, L.stream_ptr())
    torch.cuda.synchronize()
    assert torch.equal(res.view(torch.int16), res2.view(torch.int16))
    assert torch.equal(out.view(torch.int16), out2.view(torch.int16))
    assert torch.equal(peer_flags[:T].cpu(), torch.ones(T, dtype=torch.int32)), "rank 0's signal to rank 1"
    assert L.device_error(clear=True) == 0


def test_quantize_peers_takes_the_maximum_over_ranks():
    """Rank 0 of two: the scale is the maximum over its own slice maximum and rank 1's
    published one -- the unsharded row's ROWWISE scale."""
    M, K = 200, 2048
    g = torch.Generator().manual_seed(3)
    x = torch.randn(M, K, generator=g).to(BF16).to(DEV)
    peer_max = (torch.rand(M, generator=g) * 8).to(DEV)
    amax_own = torch.zeros(2 * M, device=DEV)
    amax_peer = torch.zeros(2 * M, device=DEV)
    amax_own[M:] = peer_max  # rank 1's slice maxima, as it would have written them
    own, peer_flags = torch.zeros(2 * M, dtype=torch.int32, device=DEV), torch.zeros(2 * M, dtype=torch.int32,
                                                                                     device=DEV)
    own[M:] = 1
    local = torch.zeros(M, dtype=torch.int32, device=DEV)
    sync = _sync(0, 2, M, [own, peer_flags], local)
    q8 = torch.empty(M, K, dtype=torch.uint8, device=DEV)
    qs = torch.empty(M, device=DEV)
    am = _ptrs(amax_own, amax_peer)
    call("ffb_quantize_fp8_peers", ptr(x), ctypes.addressof(am), ctypes.addressof(sync), ptr(q8), ptr(qs), M, K,
         L.stream_ptr())
    torch.cuda.synchronize()
    own_max = x.float().abs().amax(1)
    # the IEEE fp32 quotient (float64 then rounded; torch's CUDA scalar division multiplies
    # by the reciprocal)
    want_s = (torch.maximum(own_max, peer_max).clamp(min=1e-12).double() / 448.0).float()
    assert torch.equal(qs, want_s)
    want8 = torch.empty(M, K, dtype=torch.uint8, device=DEV)
    call("ffb_quantize_fp8", ptr(x), L.QUANT_ROWSCALE, 0.0, ptr(want8), ptr(want_s), M, K, L.stream_ptr())
    torch.cuda.synchronize()
    assert torch.equal(q8, want8)
    assert torch.equal(amax_peer[:M], own_max), "rank 0's maximum published into rank 1's buffer"
    assert L.device_error(clear=True) == 0


def test_unanswered_handshake_gives_up_with_an_error():
    """A second rank that never signals: every row's wait gives up after its bounded time,
    the device error word records it, and the context keeps working."""
    T, H = 4, 1024
    a, w, planes = _case(T, H, 4)
    own, peer_flags = torch.zeros(2 * T, dtype=torch.int32, device=DEV), torch.zeros(2 * T, dtype=torch.int32,
                                                                                     device=DEV)
    local = torch.zeros(T, dtype=torch.int32, device=DEV)
    sync = _sync(0, 2, T, [own, peer_flags], local)
    res, out = torch.empty_like(a), torch.empty_like(a)
    pl = _ptrs(*planes)
    L.device_error(clear=True)
    call("ffb_add_rmsnorm_peers", ptr(a), ctypes.addressof(pl), ctypes.addressof(sync), None, 0, 0, ptr(w), 1e-6,
         ptr(res), ptr(out), L.QUANT_NONE, 0.0, None, None, T, H, L.stream_ptr())
    torch.cuda.synchronize()
    assert L.device_error(clear=True) & ERR_PEER_TIMEOUT
    assert torch.equal((torch.ones(3, device=DEV) * 2).cpu(), torch.full((3,), 2.0))  # the context still runs work
