"""Read/write helpers for the golden ``.npz`` fixtures.

A fixture file holds several cases; array ``"<case>/<field>"`` holds one
tensor.  bf16 tensors are stored as uint16 bit patterns under
``"<case>/<field>@bf16"`` so that round trips are bit-exact.
"""
from __future__ import annotations

import os
from typing import Dict

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

def pack(cases: Dict[str, Dict[str, torch.Tensor]]) -> Dict[str, np.ndarray]:
    out = {}
    for case, fields in cases.items():
        for k, t in fields.items():
            t = t.detach().contiguous().cpu()
            if t.dtype == torch.bfloat16:
                out[f"{case}/{k}@bf16"] = t.view(torch.int16).numpy().view(np.uint16)
            else:
                out[f"{case}/{k}"] = t.numpy()
    return out


def load(name: str) -> Dict[str, Dict[str, torch.Tensor]]:
    """All cases of ``tests/golden/<name>.npz`` as ``{case: {field: tensor}}``."""
    z = np.load(os.path.join(HERE, f"{name}.npz"))
    cases: Dict[str, Dict[str, torch.Tensor]] = {}
    for key in z.files:
        case, field = key.split("/", 1)
        arr = z[key]
        if field.endswith("@bf16"):
            t = torch.from_numpy(arr.view(np.int16).copy()).view(torch.bfloat16)
            field = field[:-5]
        else:
            t = torch.from_numpy(arr.copy())
        cases.setdefault(case, {})[field] = t
    return cases


def load_arrays(name: str) -> Dict[str, np.ndarray]:
    z = np.load(os.path.join(HERE, f"{name}.npz"))
    return {k: z[k] for k in z.files}
