"""Load and save the golden fixtures (tensors stored as raw bits in compressed .npz files).

Each case is a dict of named CPU tensors plus scalar metadata.  Tensors keep their exact
bits: bfloat16 / float16 / float8 are stored through integer views.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch

GOLDEN_DIR = Path(__file__).resolve().parent

_INT_VIEW = {
    torch.bfloat16: torch.int16,
    torch.float16: torch.int16,
    torch.float8_e4m3fn: torch.uint8,
}
_DTYPES = {str(d): d for d in (torch.float32, torch.float16, torch.bfloat16, torch.float8_e4m3fn, torch.uint8,
                               torch.bool, torch.int64, torch.int32, torch.int16)}


def save_cases(path: Path, cases: dict[str, dict]) -> None:
    arrays = {}
    meta = {}
    for case, fields in cases.items():
        meta[case] = {}
        for name, value in fields.items():
            if isinstance(value, torch.Tensor):
                t = value.detach().cpu().contiguous()
                view = t.view(_INT_VIEW[t.dtype]) if t.dtype in _INT_VIEW else t
                arrays[f"{case}/{name}"] = view.numpy()
                meta[case][name] = {"dtype": str(t.dtype), "shape": list(t.shape)}
            else:
                meta[case][name] = {"value": value}
    arrays["__meta__"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(path, **arrays)


def load_cases(path: Path) -> dict[str, dict]:
    data = np.load(path)
    meta = json.loads(bytes(data["__meta__"]).decode())
    cases: dict[str, dict] = {}
    for case, fields in meta.items():
        out = {}
        for name, info in fields.items():
            if "value" in info:
                out[name] = info["value"]
                continue
            dtype = _DTYPES[info["dtype"]]
            raw = torch.from_numpy(data[f"{case}/{name}"].copy())
            t = raw.view(dtype) if dtype in _INT_VIEW else raw.to(dtype)
            out[name] = t.reshape(info["shape"])
        cases[case] = out
    return cases
