"""fastforward_b200: B200-native (sm_100a) Qwen3-VL prefill + choice scoring.

A from-scratch implementation of the hot path of FastForward (`fastforward_accel`):
the language-decoder prefill and option-letter scoring that follows the vision tower,
behind the same `Accelerator(bundle, backend="fast").predict(...)` surface and the same
fused-op signatures (`fastforward_b200.ops`).  Kernels live in `libffb200.so` (C ABI in
`include/ffb200.h`), built in-tree by `python -m fastforward_b200.build`.
"""
from .api import Accelerator, response, validate_request  # noqa: F401

__version__ = "0.1.0"
