"""sa3_b200: B200-native (sm_100a) Stable Audio 3 DiT denoiser forward path.

Compute lives in ``libsa3b200.so`` (hand-written CUDA for sm_100a behind a
C ABI, see include/sa3b200.h). This package binds it with ctypes and mirrors
the reference's PyTorch operator API (flash-attn style attention calls, the
SWA plugin op, quantized nn.Linear replacements and the DiT modules).
"""
from . import build, _lib  # noqa: F401

__all__ = ["build", "_lib"]
__version__ = "0.1.0"
