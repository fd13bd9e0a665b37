"""rust_katago_b200 — B200-native (sm_100a) quantized KataGo trunk forward.

The product is the C-ABI shared library ``libkatab200.so`` (CUDA kernels plus
the C++ host runtime, declared in ``include/katab200.h``).  This Python
package is a thin ctypes mirror of the reference's host interfaces, used by
the tests and the benchmark.  Importing it does not load the library; the
first call does, and fails loudly when the library was not built.
"""

from . import _capi  # noqa: F401

__all__ = ["_capi"]
