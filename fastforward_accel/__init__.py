"""Drop-in import name for the reference's public surface.

Code written against FastForward imports `fastforward_accel.Accelerator(config,
backend="fast")`, `validate_request` and `response` (the reference's `api.py:17-99`).
This package gives those names, unchanged in signature, error types and messages, backed
by the sm_100a implementation in `fastforward_b200`, so such code runs without edits.
"""
from fastforward_b200.api import Accelerator, response, validate_request  # noqa: F401

__all__ = ["Accelerator", "response", "validate_request"]
