"""hexanima_b200 — B200-native DiT block runtime (the per-block operator path of Herolias/hexanima).

The compute lives in libhxdit.so (hand-written sm_100a CUDA behind the C ABI of include/hxdit.h);
`runtime` binds it with ctypes, `packs` builds and reads the block weight packs, `pipeline` runs
whole denoise steps on top of the chain call.
"""
from . import runtime  # noqa: F401
from .runtime import Handle, HxError, lib, version  # noqa: F401
