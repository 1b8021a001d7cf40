"""ns_fps_b200 -- B200-native farthest point sampling, a drop-in for the
sampling path of satreeby/ns_fps (``yuezu_fps.yuezu_fps_module``).

* ``ns_fps_b200.yuezu_fps_module`` -- the pybind11 module with the reference's
  surface (``fps``, ``fps_with_bbox``, ``make_range``, ``make_uniform_range``,
  ``SpaceRange``, ``MORTON_BLOCK_SIZE`` ...), computing on the GPU.
* ``ns_fps_b200.libnsfps_path()`` -- the C ABI library (``include/nsfps.h``).

Build in place with ``python -m ns_fps_b200.build``.  There is no CPU
fallback: importing the module without the built extension raises.
"""
from __future__ import annotations

import importlib
import os

_HERE = os.path.dirname(os.path.abspath(__file__))

__all__ = ["yuezu_fps_module", "libnsfps_path", "load_library"]


def libnsfps_path() -> str:
    return os.path.join(_HERE, "libnsfps.so")


def load_library():
    """ctypes handle of libnsfps.so (raises when it has not been built)."""
    import ctypes
    path = libnsfps_path()
    if not os.path.exists(path):
        raise ImportError(f"{path} is missing: build it with `python -m ns_fps_b200.build`")
    return ctypes.CDLL(path)


def __getattr__(name):
    if name == "yuezu_fps_module":
        try:
            return importlib.import_module(".yuezu_fps_module", __name__)
        except ImportError as e:
            raise ImportError(
                "ns_fps_b200.yuezu_fps_module is not built; run `python -m ns_fps_b200.build` "
                f"({e})") from e
    raise AttributeError(name)
