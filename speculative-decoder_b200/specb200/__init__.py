"""B200-native engine behind the reference's spec/, cache/ and lm/ API.

libspecb200.so (csrc/, built in-tree by specb200.build) holds every kernel; _ffi binds its C
ABI, ops wraps single kernels, engine packs a Hugging Face model for the forward, and rounds
runs the device-resident speculative round used by spec.loop.generate.
"""
from specb200._ffi import LIB_PATH, lib  # noqa: F401
