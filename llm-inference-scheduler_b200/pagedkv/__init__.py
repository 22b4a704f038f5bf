"""pagedkv -- B200-native paged KV cache for mini_engine.

The product is libpagedkv.so (hand-written sm_100a CUDA behind the C ABI in
include/pagedkv.h); this package is its host side: ctypes bindings (`_lib`),
torch-facing wrappers (`ops`) and the reference's operator surface
(`BlockManager`, `PagedKVCache`, `OutOfBlocks`) with the pools in HBM.
"""

from .block_manager import BlockManager, OutOfBlocks, PagedKVCache, StepMetadata  # noqa: F401

__all__ = ["BlockManager", "OutOfBlocks", "PagedKVCache", "StepMetadata"]
