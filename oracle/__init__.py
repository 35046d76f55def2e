"""CPU oracle for the Qwen3-VL prefill + choice-scoring path (TEST INFRASTRUCTURE).

This package restates, on the CPU with PyTorch, the arithmetic of FastForward's
language-decoder prefill and option scoring so that the CUDA path can be checked
against it.  It is the checker only: `tests/`, `__graft_entry__.smoke()` and the
CPU legs of `bench.py` may import it; the product package `fastforward_b200`
never does, and it never runs in place of a CUDA kernel.

Pinning: `tests/golden/make_golden.py` runs the reference's own Triton kernels
(imported from the reference source tree, executed by Triton's CPU interpreter
with its float down-casts patched to round-to-nearest-even like the GPU) and
Hugging Face's Qwen3-VL rotary/position code, and stores their outputs as
fixtures; `tests/test_oracle_golden.py` checks every oracle function against
those fixtures.
"""
from .qwen_path import *  # noqa: F401,F403
from .pack import *  # noqa: F401,F403,E402
from .vision import *  # noqa: F401,F403,E402
