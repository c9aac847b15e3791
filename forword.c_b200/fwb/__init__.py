"""Python host helpers for forword-b200: ctypes bindings of the C ABI,
model shapes, and the seeded synthetic GGUF writer used by tests and bench.py.

The compute path is the CUDA library lib/libforword_b200.so; nothing here
computes a forward pass.
"""
from . import configs, native  # noqa: F401
