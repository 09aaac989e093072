"""hexanima_b200 — B200-native DiT block runtime (the per-block operator path of Herolias/hexanima).

The compute lives in libhxdit.so (hand-written sm_100a CUDA behind the C ABI of include/hxdit.h);
`runtime` binds it with ctypes (handles, buffers, weight sets, the per-block call, the chain and the
samplers), `synth` makes the seeded synthetic weight sets of the benchmarks and tests, `build`
compiles the library in-tree for sm_100a, `opbench` times single operators on the device.
"""
from . import runtime  # noqa: F401
from .runtime import Handle, HxError, lib, version  # noqa: F401
