"""Python façade over the C++ paged KV block manager (``lightbulb_b200._native``)."""
from __future__ import annotations

from typing import List, Sequence as Seq, Tuple

import torch  # noqa: F401  (loads libc10 for the native extension)

try:
    from .._native import BlockManager as _CppBlockManager  # type: ignore
    from .._native import hash_block  # type: ignore  # noqa: F401
except Exception as e:  # pragma: no cover
    _CppBlockManager = None
    _IMPORT_ERR = e
else:
    _IMPORT_ERR = None


def native_available() -> bool:
    return _CppBlockManager is not None


class BlockManager:
    """Paged allocator with refcounts, copy-on-write and a chained-hash prefix index.

    Thin wrapper: all state lives in C++; this class only adapts argument types."""

    def __init__(self, num_blocks: int, block_size: int, enable_prefix: bool = True):
        if _CppBlockManager is None:
            raise RuntimeError(f"lightbulb_b200._native is not built: {_IMPORT_ERR}")
        self._m = _CppBlockManager(int(num_blocks), int(block_size), bool(enable_prefix))
        self.block_size = block_size
        self.num_blocks = num_blocks

    def __getattr__(self, name):
        return getattr(self._m, name)

    def append_slots(self, sid: int, n: int, tokens: Seq[int] = ()) -> Tuple[List[int], List[int]]:
        return self._m.append_slots(sid, n, list(tokens))

    def match_prefix(self, sid: int, tokens: Seq[int]) -> int:
        return self._m.match_prefix(sid, list(tokens))

    def prefix_hit_rate(self) -> float:
        hit, q = self._m.prefix_stats()
        return hit / q if q else 0.0
