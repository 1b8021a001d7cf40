"""The reference's import name for its extension, served by this engine.

satreeby/ns_fps installs its pybind11 module as ``yuezu_fps.yuezu_fps_module``
(setup.py:6) and its scripts import it as
``import yuezu_fps.yuezu_fps_module as yf`` (test.py:3, example.py).  With the
repository root on ``sys.path`` that import resolves here, to the engine's
module ``ns_fps_b200.yuezu_fps_module`` itself (the same module object, so its
``SpaceRange`` is one class whichever name imported it).  Nothing in a
caller's code changes.  There is no CPU fallback: when the extension is not
built the import raises.
"""
import sys as _sys

from ns_fps_b200 import yuezu_fps_module

_sys.modules[__name__ + ".yuezu_fps_module"] = yuezu_fps_module

__all__ = ["yuezu_fps_module"]
