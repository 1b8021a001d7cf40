"""The tests call the engine through its C ABI with the package's ctypes
binding (ns_fps_b200/capi.py)."""
from ns_fps_b200.capi import *  # noqa: F401,F403
from ns_fps_b200 import capi as _c

_u64p, _f32p, _u32p = _c._u64p, _c._f32p, _c._u32p


def lib():
    return _c.lib()


def last_error():
    return _c.last_error()
