"""patch_needle() on CPU with stand-in needle classes.

The stand-ins carry exactly the attributes needle's ``Attention``
(``needle/layers/attention.py:38-50``) and ``RMSNorm``
(``needle/layers/norm.py:8-12``) have.  After the patch their ``forward``
must reach this library's ops -- which refuse CPU tensors with a
ValueError -- without touching attributes only this library's own classes
define; ``unpatch_needle()`` restores the originals.
"""
import math
import sys
import types

import pytest
import torch
import torch.nn as nn


class _NeedleAttention(nn.Module):
    def __init__(self, hidden=64, H=4, KV=2, D=16):
        super().__init__()
        self.num_heads, self.num_kv_heads, self.head_dim = H, KV, D
        self.scale = 1.0 / math.sqrt(D)
        self.q_proj = nn.Linear(hidden, H * D, bias=False)
        self.k_proj = nn.Linear(hidden, KV * D, bias=False)
        self.v_proj = nn.Linear(hidden, KV * D, bias=False)
        self.o_proj = nn.Linear(H * D, hidden, bias=False)

    def forward(self, *a):
        return "needle attention"


class _NeedleRMSNorm(nn.Module):
    def __init__(self, hidden=64, eps=1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden))
        self.eps = eps

    def forward(self, x):
        return "needle norm"


class _NeedleSampler:
    def sample(self, logits, sampling_params_list):
        return "needle sampler"


@pytest.fixture
def fake_needle(monkeypatch):
    mods = {name: types.ModuleType(name) for name in
            ("needle", "needle.model", "needle.layers", "needle.layers.attention",
             "needle.layers.norm", "needle.model.sampler")}
    mods["needle.layers.attention"].Attention = _NeedleAttention
    mods["needle.layers.norm"].RMSNorm = _NeedleRMSNorm
    mods["needle.model.sampler"].Sampler = _NeedleSampler
    for name, m in mods.items():
        monkeypatch.setitem(sys.modules, name, m)
    yield
    from needle_b200.integration import unpatch_needle
    unpatch_needle()


def test_patch_routes_needle_modules_to_the_library(fake_needle):
    from needle_b200.integration import patch_needle, unpatch_needle
    attn, norm = _NeedleAttention(), _NeedleRMSNorm()
    T = 3
    x = torch.randn(T, 64)
    cache = torch.zeros(2, 4, 2, 16, 16)
    bt = torch.zeros(T, 1, dtype=torch.int32)
    ctx = torch.zeros(T, dtype=torch.int32)
    cos = torch.ones(T, 16)
    patch_needle()
    # the ops refuse CPU tensors: reaching them proves the module attributes sufficed
    with pytest.raises(ValueError, match="CUDA"):
        attn(x, torch.arange(T), cache, bt, None, ctx, 1, False, cos, cos)
    with pytest.raises(ValueError, match="CUDA"):
        norm(x)
    with pytest.raises(ValueError, match="CUDA"):
        norm(x, x.clone())
    # the sampler takes needle's signature; on CPU logits it runs the host path
    from needle_b200.model.sequence import SamplingParams
    ids = _NeedleSampler().sample(torch.tensor([[0.1, 2.0, -1.0]]), [SamplingParams(temperature=0.0)])
    assert ids == [1]
    unpatch_needle()
    assert attn(x) == "needle attention" and norm(x) == "needle norm"
    assert _NeedleSampler().sample(None, []) == "needle sampler"
