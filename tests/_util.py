"""Comparison helpers shared by the parity tests."""
import torch


def bf16_ulp_diff(a, b):
    """Per-element distance in bf16 ulps between two bf16 tensors (same sign-magnitude order)."""
    ia = a.contiguous().view(torch.int16).to(torch.int32)
    ib = b.contiguous().view(torch.int16).to(torch.int32)
    # map sign-magnitude to a monotonic integer line
    ia = torch.where(ia < 0, -(ia & 0x7FFF), ia)
    ib = torch.where(ib < 0, -(ib & 0x7FFF), ib)
    return (ia - ib).abs()


def assert_bf16_near(got, want, max_ulp=1, max_frac=0.01, what="", atol=0.0):
    """Every element within `max_ulp` bf16 ulps of `want` or within `atol` absolute (the
    latter covers results of cancellation near zero, where one ulp of an operand is many
    ulps of the result); at most `max_frac` of the elements not bit-identical."""
    got = got.detach().cpu().to(torch.bfloat16)
    want = want.detach().cpu().to(torch.bfloat16)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    d = bf16_ulp_diff(got, want)
    frac = (d > 0).float().mean().item()
    bad = (d > max_ulp) & ((got.float() - want.float()).abs() > atol)
    assert not bad.any(), (f"{what}: {int(bad.sum())} elements beyond {max_ulp} ulp / atol {atol}; "
                           f"max ulp {d.max().item()}, max abs {(got.float() - want.float()).abs().max().item():.3g}")
    assert frac <= max_frac, f"{what}: {frac:.4%} elements differ (> {max_frac:.2%})"
    return frac


def assert_bytes_equal(got, want, what=""):
    g = got.detach().cpu().contiguous().view(torch.uint8)
    w = want.detach().cpu().contiguous().view(torch.uint8)
    assert g.shape == w.shape, (what, g.shape, w.shape)
    bad = (g != w).sum().item()
    assert bad == 0, f"{what}: {bad} of {g.numel()} bytes differ"
