"""Device-aware LRU cache for shifted-window attention masks.

Same contract as the reference mask cache (torch-ext/crumpet/cache.py:1-97):
keys are (D, H, W, window_size, shift_size, dtype, device), at most
``CRUMPET_MASK_CACHE_SIZE`` entries (default 64) and
``CRUMPET_MASK_CACHE_MAX_BYTES`` bytes (default 1 GiB) are kept, a value
larger than the byte cap is returned uncached, and
``CRUMPET_DISABLE_MASK_CACHE=1`` bypasses the cache.  Not thread-safe.
"""

from __future__ import annotations

import os
from collections import OrderedDict
from typing import Callable

import torch

MaskKey = tuple[int, int, int, tuple[int, int, int], tuple[int, int, int], torch.dtype, str]

_DEFAULT_ENTRIES = 64
_DEFAULT_BYTES = 1 << 30

_entries: "OrderedDict[MaskKey, torch.Tensor]" = OrderedDict()
_total_bytes = 0


def _env_int(name: str, default: int) -> int:
    raw = os.environ.get(name)
    if raw is None:
        return default
    try:
        return int(raw)
    except ValueError:
        return default


def _limits() -> tuple[int, int]:
    return (
        _env_int("CRUMPET_MASK_CACHE_SIZE", _DEFAULT_ENTRIES),
        _env_int("CRUMPET_MASK_CACHE_MAX_BYTES", _DEFAULT_BYTES),
    )


def _device_key(device: torch.device | str) -> str:
    dev = torch.device(device)
    if dev.type != "cuda":
        return str(dev)
    index = dev.index
    if index is None and torch.cuda.is_available():
        index = torch.cuda.current_device()
    return f"cuda:{0 if index is None else index}"


def make_mask_key(
    D: int,
    H: int,
    W: int,
    window_size: tuple[int, int, int],
    shift_size: tuple[int, int, int],
    dtype: torch.dtype,
    device: torch.device | str,
) -> MaskKey:
    return (D, H, W, tuple(window_size), tuple(shift_size), dtype, _device_key(device))


def clear_mask_cache() -> None:
    global _total_bytes
    _entries.clear()
    _total_bytes = 0


def mask_cache_info() -> dict[str, int]:
    max_entries, max_bytes = _limits()
    return {
        "entries": len(_entries),
        "bytes": _total_bytes,
        "max_entries": max_entries,
        "max_bytes": max_bytes,
    }


def _nbytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()


def get_or_compute_mask(key: MaskKey, compute: Callable[[], torch.Tensor]) -> torch.Tensor:
    """Return the cached mask for ``key`` or compute, insert and return it.

    The cache is a convenience LRU, not a lifetime guarantee: callers in hot
    loops keep their own reference to the returned tensor.
    """
    global _total_bytes
    if os.environ.get("CRUMPET_DISABLE_MASK_CACHE", "0") == "1":
        return compute()
    cached = _entries.get(key)
    if cached is not None:
        _entries.move_to_end(key)
        return cached
    value = compute()
    max_entries, max_bytes = _limits()
    size = _nbytes(value)
    if max_entries <= 0 or size > max_bytes:
        return value
    _entries[key] = value
    _total_bytes += size
    while _entries and (len(_entries) > max_entries or _total_bytes > max_bytes):
        _, old = _entries.popitem(last=False)
        _total_bytes -= _nbytes(old)
    return value
