"""proxima_b200: Proxima's exact-kNN and PQ-ADC hot path on NVIDIA B200.

``from proxima_b200 import FlatIndex, PqIndex, Metric`` gives the classes of
the reference's ``proxima`` package (python/proxima/__init__.py:1-3) backed
by sm_100a kernels in libproxima_b200.so, including the reference's `.sfidx`
index files (persist.py). The CPU HNSW index and the corpus tooling of the
reference are not part of this package.
"""

from ._core import FlatIndex, Metric, PqIndex, PX_MAX_K, PxError  # noqa: F401
from ._lib import device_count, launch_count, set_profiling, LIB_PATH  # noqa: F401

__all__ = ["FlatIndex", "PqIndex", "Metric", "PxError", "PX_MAX_K", "device_count",
           "launch_count", "set_profiling"]
__version__ = "0.1.0"
