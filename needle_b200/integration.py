"""Switch an existing needle installation onto the B200 kernels.

needle's ``Attention`` and ``RMSNorm`` keep their attributes (``q_proj`` ..
``o_proj``, ``num_heads``, ``num_kv_heads``, ``head_dim``, ``scale``;
``weight``, ``eps``) and their ``forward`` signatures, so swapping the two
``forward`` methods is enough for needle's own model classes, ModelRunner,
Scheduler and engine to run on this library unchanged::

    import needle
    from needle_b200.integration import patch_needle
    patch_needle()          # before building the ModelRunner

With the patch, needle's decoder layers still perform their residual adds
with torch; ``needle_b200.model`` additionally fuses each add into the next
RMSNorm.  ``unpatch_needle()`` restores the originals.
"""
from __future__ import annotations

import importlib

_saved = {}


def patch_needle() -> None:
    """Route ``needle.layers.attention.Attention.forward``,
    ``needle.layers.norm.RMSNorm.forward`` and ``needle.model.sampler.Sampler.sample``
    (same signature; CUDA logits take one ``nb_sample`` launch per step) to
    this library."""
    importlib.import_module("needle")
    importlib.import_module("needle.model")  # needle.layers.attention alone is a circular import
    attn_mod = importlib.import_module("needle.layers.attention")
    norm_mod = importlib.import_module("needle.layers.norm")
    samp_mod = importlib.import_module("needle.model.sampler")
    from .layers.attention import Attention
    from .layers.norm import RMSNorm
    from .model.sampler import Sampler
    if not _saved:
        _saved["attn"] = attn_mod.Attention.forward
        _saved["norm"] = norm_mod.RMSNorm.forward
        _saved["sample"] = samp_mod.Sampler.sample
    attn_mod.Attention.forward = Attention.forward
    norm_mod.RMSNorm.forward = RMSNorm.forward
    samp_mod.Sampler.sample = Sampler.sample


def unpatch_needle() -> None:
    if not _saved:
        return
    attn_mod = importlib.import_module("needle.layers.attention")
    norm_mod = importlib.import_module("needle.layers.norm")
    samp_mod = importlib.import_module("needle.model.sampler")
    attn_mod.Attention.forward = _saved.pop("attn")
    norm_mod.RMSNorm.forward = _saved.pop("norm")
    samp_mod.Sampler.sample = _saved.pop("sample")
