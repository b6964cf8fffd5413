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


def header_prototypes() -> dict[str, tuple[str, list[str]]]:
    """name -> (return type, parameter types) of every function include/crumpet_b200.h
    declares, comments stripped and parameter names dropped."""
    text = (ROOT / "include" / "crumpet_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    text = re.sub(r"//[^\n]*", " ", text)
    protos = {}
    for ret, name, params in re.findall(
            r"CRUMPET_API\s+([\w\s\*]+?)\s*\b(crumpet_\w+)\s*\(([^)]*)\)\s*;", text):
        types = []
        for param in params.split(","):
            param = " ".join(param.split())
            if param in ("", "void"):
                continue
            # drop the parameter name: the last identifier, unless the type ends in '*'
            m = re.fullmatch(r"(.*?[\s\*])(\w+)", param)
            types.append(" ".join(m.group(1).split()) if m else param)
        protos[name] = (" ".join(ret.split()), types)
    return protos


def ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def stream_ptr() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
