"""B200-native (sm_100a) SmoothQuant ``sample_actions`` for SmolVLA.

The compute path is ``csrc/`` (hand-written CUDA for sm_100a behind a C ABI,
``include/svla.h``).  The Python side is a thin host layer: a ctypes loader
(``_lib``), torch custom ops (``ops``), the model/weight builder (``model``)
and the ``sample_actions`` drop-in (``policy``).  There is no CPU or library
fallback: when ``libsvla.so`` is missing every entry point raises.
"""

__all__ = ["config", "synthetic"]
