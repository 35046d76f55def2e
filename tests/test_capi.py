"""The C-ABI library: builds, loads without a GPU, exports every declared entry point, and
rejects bad arguments on the host (no kernel launches here)."""
import ctypes
import re
from pathlib import Path

import pytest

from fastforward_b200 import _lib as L

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "ffb200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ffb_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "ffb_fp8_gemm" in names and "ffb_attention" in names
    assert len(names) >= 18


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(L.LIB_PATH))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"symbols declared in ffb200.h but not exported: {missing}"


def test_python_binding_covers_header():
    assert set(declared_functions()) == set(L.SIGNATURES), "ctypes signature table out of sync with the header"


def test_version_string():
    assert L.lib().ffb_version().decode().startswith("ffb200")


def test_host_side_argument_errors():
    # invalid shapes are rejected before any CUDA call
    with pytest.raises(ValueError, match="multiple of 128"):
        L.call("ffb_fp8_gemm", 16, 16, 1, 16, 16, 1, L.EPI_BF16, 16, None, 1, 0, 16, 100, 128, None)
    with pytest.raises(ValueError, match="NULL"):
        L.call("ffb_attention", None, None, None, None, 0, None, 1, 1, 8, 8, 1.0, None)
    with pytest.raises(ValueError):
        L.call("ffb_readout", 16, None, None, 0, 16, 1e-6, 16, 9, 4, 16, None, 2048, None)
    with pytest.raises(ValueError, match="splits"):
        L.call("ffb_fp8_gemm", 16, 16, 1, 16, 16, 1, L.EPI_F32_PARTIAL, None, 16, 99, 0, 16, 128, 128, None)
    msg = L.last_error()
    assert "splits" in msg


def test_pdl_toggle_roundtrip():
    old = L.set_pdl(0)
    assert L.set_pdl(old) == 0


def test_fused_static_quant_entries_reject_bad_arguments():
    """The epilogue-quantising entries check their arguments on the host before any launch."""
    with pytest.raises(ValueError, match="out_inv"):
        L.call("ffb_fp8_gemm_swiglu_fp8", 16, 16, 0, 16, 16, 1, 0.0, 16, 320, 512, 2560, None)
    with pytest.raises(ValueError, match="aligned"):
        L.call("ffb_fp8_gemm_swiglu_fp8", 16, 16, 0, 16, 16, 1, 10.0, 17, 320, 512, 2560, None)
    with pytest.raises(ValueError, match="multiple of 128"):
        L.call("ffb_fp8_gemm_swiglu_fp8", 16, 16, 0, 16, 16, 1, 10.0, 16, 320, 500, 2560, None)
    with pytest.raises(ValueError, match="out_inv"):
        L.call("ffb_attention_fp8", 16, 16, 16, None, -1.0, 16, 320, 32, 8, 0.1, None)
    with pytest.raises(ValueError, match="NULL"):
        L.call("ffb_attention_fp8", None, 16, 16, None, 1.0, 16, 320, 32, 8, 0.1, None)
    with pytest.raises(ValueError, match="bad shape"):
        L.call("ffb_attention_fp8", 16, 16, 16, None, 1.0, 16, 320, 30, 8, 0.1, None)
