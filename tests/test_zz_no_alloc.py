"""ffb_quantize_weight_fp8_noalloc (weight quantisation with the library's fixed device
scratch) against ffb_quantize_weight_fp8 (caller scratch), called through the C ABI.
Collected last so that it also runs after every other test has used the device."""
import pytest
import torch

from fastforward_b200 import _lib as L
from fastforward_b200._lib import call, ptr

MAX_N = 65536  # FFB_QW_NOALLOC_MAX_N in include/ffb200.h


def test_header_states_the_limit():
    from pathlib import Path
    text = (Path(__file__).resolve().parents[1] / "include" / "ffb200.h").read_text()
    assert f"#define FFB_QW_NOALLOC_MAX_N {MAX_N}" in text


def test_rejects_rows_beyond_the_fixed_scratch():
    # host-side check, before any CUDA call: the pointers are never touched
    with pytest.raises(ValueError, match="fixed scratch"):
        call("ffb_quantize_weight_fp8_noalloc", 16, 1, 16, 16, MAX_N + 1, 128, None)


@pytest.mark.gpu
def test_noalloc_matches_caller_scratch_on_two_calls_in_a_row():
    dev = torch.device("cuda")
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator().manual_seed(31)
    # two different weights back to back (per-channel, then per-tensor with more rows):
    # the second call must not see anything the first left in the shared scratch
    cases = [(1, 3072, 2560, 0.02), (0, 4096, 1024, 0.5)]
    for per_channel, N, K, std in cases:
        w = (torch.randn(N, K, generator=g) * std).to(torch.bfloat16).to(dev)
        n_scale = N if per_channel else 1
        w8_ref = torch.empty(N, K, dtype=torch.uint8, device=dev)
        s_ref = torch.empty(n_scale, dtype=torch.float32, device=dev)
        ws = torch.empty(N, dtype=torch.float32, device=dev)
        call("ffb_quantize_weight_fp8", ptr(w), per_channel, ptr(w8_ref), ptr(s_ref), ptr(ws), N, K, stream)
        w8 = torch.full((N, K), 0x7F, dtype=torch.uint8, device=dev)
        s = torch.full((n_scale,), -1.0, dtype=torch.float32, device=dev)
        call("ffb_quantize_weight_fp8_noalloc", ptr(w), per_channel, ptr(w8), ptr(s), N, K, stream)
        torch.cuda.synchronize()
        assert torch.equal(w8, w8_ref), f"w8 differs (per_channel={per_channel}, N={N})"
        assert torch.equal(s, s_ref), f"scales differ (per_channel={per_channel}, N={N})"
    assert L.device_error() == 0
