"""Small helpers shared by the test modules."""

from __future__ import annotations

import ctypes
import hashlib
import re
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[1]
DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(
        t.detach().contiguous().cpu().view(-1).view(torch.uint8).numpy().tobytes()
    ).hexdigest()


def header_functions() -> list[str]:
    text = (ROOT / "include" / "crumpet_b200.h").read_text()
    return re.findall(r"CRUMPET_API\s+[\w\s\*]+?\b(crumpet_\w+)\s*\(", text)


def ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def stream_ptr() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
