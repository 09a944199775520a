"""flash_kmeans_cuda (B200 build) - batched Euclidean K-Means Lloyd iteration on sm_100a.

Same public API as OpsiClear/flash-kmeans-cuda (``flash_kmeans_cuda/__init__.py``):
``batch_kmeans_Euclid``, ``euclid_assign``, ``centroid_update_sorted``,
``centroid_finalize`` and the ``_C`` module. The kernels live in
``libfkc_b200.so`` behind the C-ABI of ``include/fkc_capi.h``; importing this
package fails if that library is missing (there is no CPU or PyTorch fallback).
Multi-GPU sharding over N or B is in ``flash_kmeans_cuda.distributed``;
host-resident x streamed through one or more GPUs is
``flash_kmeans_cuda.largen.kmeans_largeN`` (not a reference export).
"""

from ._version import __version__
from .kmeans import batch_kmeans_Euclid
from .ops import euclid_assign, centroid_update_sorted, centroid_finalize

__all__ = [
    "__version__",
    "batch_kmeans_Euclid",
    "euclid_assign",
    "centroid_update_sorted",
    "centroid_finalize",
]
