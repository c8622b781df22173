"""Read/write helpers for the golden fixtures (``tests/golden/*.npz``).

bfloat16 arrays are stored as their uint16 bit patterns under ``<name>__bf16``; every
other array is stored as is. Loading returns CPU torch tensors with the original dtypes.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

GOLDEN_DIR = Path(__file__).resolve().parent


def to_numpy_entries(tensors: dict[str, torch.Tensor]) -> dict[str, np.ndarray]:
    out = {}
    for name, t in tensors.items():
        t = t.detach().cpu().contiguous()
        if t.dtype == torch.bfloat16:
            out[f"{name}__bf16"] = t.view(torch.int16).numpy().view(np.uint16)
        else:
            out[name] = t.numpy()
    return out


def save(case: str, tensors: dict[str, torch.Tensor], meta: dict[str, float | int | str]) -> Path:
    path = GOLDEN_DIR / f"{case}.npz"
    entries = to_numpy_entries(tensors)
    for key, value in meta.items():
        entries[f"meta__{key}"] = np.array(value)
    np.savez_compressed(path, **entries)
    return path


def load(case: str) -> tuple[dict[str, torch.Tensor], dict[str, object]]:
    path = GOLDEN_DIR / f"{case}.npz"
    tensors: dict[str, torch.Tensor] = {}
    meta: dict[str, object] = {}
    with np.load(path) as data:
        for key in data.files:
            arr = data[key]
            if key.startswith("meta__"):
                meta[key[6:]] = arr.item()
            elif key.endswith("__bf16"):
                tensors[key[:-6]] = torch.from_numpy(arr.view(np.int16).copy()).view(torch.bfloat16)
            else:
                tensors[key] = torch.from_numpy(arr.copy())
    return tensors, meta


def cases() -> list[str]:
    return sorted(p.stem for p in GOLDEN_DIR.glob("*.npz"))
