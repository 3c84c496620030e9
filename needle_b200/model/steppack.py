"""Host-side packing of a step's padded block table.

needle's scheduler hands ``ModelRunner`` one fresh Python list of block ids
per sequence every step (``needle/backend/scheduler.py:127-130``).  The
CPython extension ``_steppack`` (``needle_b200/host/steppack.c``, built with
the CUDA library) writes them as a padded int32 table straight into the
pinned staging buffer that goes to the device in one copy;
``block_table_np`` is the same table built with numpy, used when the
extension is not built and as its check.
"""
from __future__ import annotations

import importlib.util
import itertools
import os
from typing import List, Optional, Sequence

import numpy as np

_ext = None
_tried = False


def ext():
    """The loaded ``_steppack`` extension, or None if it has not been built."""
    global _ext, _tried
    if not _tried:
        _tried = True
        from ..build import host_ext_path
        path = host_ext_path()
        if os.path.exists(path):
            try:
                spec = importlib.util.spec_from_file_location("needle_b200._steppack", path)
                mod = importlib.util.module_from_spec(spec)
                spec.loader.exec_module(mod)
                _ext = mod
            except ImportError as e:  # built for another interpreter: use the numpy table
                import warnings
                warnings.warn(f"needle_b200: {path} does not load ({e}); "
                              "packing block tables with numpy")
    return _ext


def block_table_np(rows: Sequence[Sequence[int]], width: int, pad: int) -> np.ndarray:
    """Padded int32 ``[len(rows), width]`` table: one C-level pass over all
    ids (``np.fromiter`` over the chained lists), then a masked scatter."""
    B = len(rows)
    lens = np.fromiter(map(len, rows), np.int64, B)
    bt = np.full((B, width), pad, dtype=np.int32)
    if B:
        flat = np.fromiter(itertools.chain.from_iterable(rows), np.int32, int(lens.sum()))
        bt[np.arange(width)[None, :] < lens[:, None]] = flat
    return bt


def fill_block_table(rows: List[Sequence[int]], address: int, capacity: int, width: int,
                     pad: int) -> None:
    """Write the padded table at ``address`` (``capacity`` bytes available)."""
    ext().fill_block_table(rows, address, capacity, width, pad)
