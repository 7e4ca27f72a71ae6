"""apple_b200 — B200-native RFSN compressed-KV decode path.

Drop-in for the reference's decode path (dawsonblock/apple, RFSN v10.2):
``RFSNConfig``, ``HybridQuantizerMLX`` / ``ProductQuantizerMLX`` /
``ResidualVQMLX``, ``RFSNv10KVCacheMLX``, ``RFSNHybridAttentionMLX``,
``AsyncHierarchicalRouterMLX`` and ``RFSNDecoderLayerMLX`` keep the reference
names and signatures; arrays are CUDA torch tensors instead of mx.arrays, and
every hot-path computation runs in librfsn_b200.so (hand-written sm_100a CUDA
behind the C ABI in include/rfsn_b200.h).
"""
from . import kernels  # noqa: F401
from ._lib import RFSNError, lib  # noqa: F401

__all__ = ["kernels", "lib", "RFSNError"]
