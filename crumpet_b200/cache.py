"""Per-device LRU of shifted-window attention masks.

The user-visible contract is the reference's mask cache
(torch-ext/crumpet/cache.py:1-97): an entry is keyed by
(D, H, W, window_size, shift_size, dtype, device); ``CRUMPET_MASK_CACHE_SIZE``
(default 64) bounds the number of entries and ``CRUMPET_MASK_CACHE_MAX_BYTES``
(default 1 GiB) their total size; a mask bigger than the byte bound is handed
back without being stored; the least recently used entries go first; and
``CRUMPET_DISABLE_MASK_CACHE=1`` turns caching off.  The limits are read from
the environment on every insertion, so they can change at run time.  Not
thread-safe (callers hold the GIL, as every op wrapper does).
"""

from __future__ import annotations

import os
import weakref
from collections import OrderedDict
from typing import Callable

import torch

MaskKey = tuple[int, int, int, tuple[int, int, int], tuple[int, int, int], torch.dtype, str]

_ENTRIES_VAR, _ENTRIES_DEFAULT = "CRUMPET_MASK_CACHE_SIZE", 64
_BYTES_VAR, _BYTES_DEFAULT = "CRUMPET_MASK_CACHE_MAX_BYTES", 1 << 30


def _setting(var: str, default: int) -> int:
    try:
        return int(os.environ[var])
    except (KeyError, ValueError):
        return default


class _MaskLRU:
    """Masks in least- to most-recently-used order, with their running byte total."""

    def __init__(self) -> None:
        self.items: "OrderedDict[MaskKey, torch.Tensor]" = OrderedDict()
        self.nbytes = 0

    @staticmethod
    def size_of(t: torch.Tensor) -> int:
        return t.numel() * t.element_size()

    def limits(self) -> tuple[int, int]:
        return _setting(_ENTRIES_VAR, _ENTRIES_DEFAULT), _setting(_BYTES_VAR, _BYTES_DEFAULT)

    def lookup(self, key: MaskKey) -> torch.Tensor | None:
        hit = self.items.get(key)
        if hit is not None:
            self.items.move_to_end(key)
        return hit

    def insert(self, key: MaskKey, value: torch.Tensor) -> None:
        max_entries, max_bytes = self.limits()
        size = self.size_of(value)
        if max_entries <= 0 or size > max_bytes:
            return  # too big to keep: the caller still gets the tensor
        self.items[key] = value
        self.nbytes += size
        while self.items and (len(self.items) > max_entries or self.nbytes > max_bytes):
            _, evicted = self.items.popitem(last=False)
            self.nbytes -= self.size_of(evicted)

    def clear(self) -> None:
        self.items.clear()
        self.nbytes = 0

    def live(self) -> list[torch.Tensor]:
        """The tensors held right now (a CUDA graph captured over them keeps these alive)."""
        return list(self.items.values())


_LRU = _MaskLRU()


def _device_key(device: torch.device | str) -> str:
    dev = torch.device(device)
    if dev.type == "cuda" and dev.index is None:
        # an index-less CUDA device means the current one
        index = torch.cuda.current_device() if torch.cuda.is_available() else 0
        return f"cuda:{index}"
    return str(dev)


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
    _LRU.clear()


def mask_cache_info() -> dict[str, int]:
    max_entries, max_bytes = _LRU.limits()
    return {"entries": len(_LRU.items), "bytes": _LRU.nbytes, "max_entries": max_entries,
            "max_bytes": max_bytes}


def cached_masks() -> list[torch.Tensor]:
    """Every mask the cache holds at this moment."""
    return _LRU.live()


def get_or_compute_mask(key: MaskKey, compute: Callable[[], torch.Tensor]) -> torch.Tensor:
    """The mask stored under ``key``; on a miss, ``compute()`` builds it and it is stored
    (unless it exceeds the byte bound).

    An entry can be evicted at any later insertion, so code that reuses a mask across
    many calls should hold on to the tensor it got back rather than look it up again.
    """
    if os.environ.get("CRUMPET_DISABLE_MASK_CACHE", "0") == "1":
        return compute()
    hit = _LRU.lookup(key)
    if hit is not None:
        return hit
    value = compute()
    _LRU.insert(key, value)
    return value


# Window geometry of the masks compute_attn_mask_3d built, so fused_swin_attention can add
# such a mask on chip instead of reading it: id(mask) -> (weak reference, torch version
# counter at creation, (windows per axis, window, shift)).  A mask modified in place since
# (its version counter moved on) or a copy of it is not recognised and is read as given.
_GEOMETRY: dict[int, tuple[weakref.ref, int, tuple]] = {}


def _version(t: torch.Tensor):
    # inference tensors keep no version counter: writes to them cannot be seen, so they
    # are never recognised
    try:
        return t._version
    except RuntimeError:
        return None


def remember_mask_geometry(mask: torch.Tensor, num_windows, window, shift) -> None:
    version = _version(mask)
    if version is None:
        return
    key = id(mask)

    def forget(_ref, key=key):
        entry = _GEOMETRY.get(key)
        if entry is not None and entry[0] is _ref:
            del _GEOMETRY[key]

    ref = weakref.ref(mask, forget)
    _GEOMETRY[key] = (ref, version, (tuple(num_windows), tuple(window), tuple(shift)))


def mask_geometry(mask: torch.Tensor):
    """(windows per axis, window, shift) of a mask compute_attn_mask_3d built and nobody
    has written to since, else None."""
    if torch.compiler.is_compiling():
        return None  # traced code keeps the plain mask-reading call
    entry = _GEOMETRY.get(id(mask))
    if entry is None or entry[0]() is not mask or entry[1] != _version(mask):
        return None
    return entry[2]
