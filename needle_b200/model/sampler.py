"""Batched on-device sampler with needle's per-row semantics.

needle's ``Sampler.sample`` (``needle/model/sampler.py:15-48``) walks the
batch row by row: ``int(argmax)`` for temperature 0, otherwise temperature
scaling, top-k masking (``logit < kth`` -> -inf), top-p masking on the
sorted, top-k-masked logits (drop a token when the probability mass before
it exceeds ``top_p``), softmax and one ``torch.multinomial`` draw, each
``int(...)`` a device-to-host sync.  Here the whole batch goes through the
same operations at once, in the logits' dtype like the reference, with one
device-to-host read of all the token ids:

* greedy rows: one batched ``argmax``;
* sampled rows: one batched divide, one ``topk`` with the largest k of the
  batch (each row reads its own k-th value), one descending ``sort`` for the
  rows with ``top_p < 1``, one ``softmax`` and one ``multinomial`` over the
  rows.

On the GPU the step runs as one kernel (``nb_sample``, see ``Sampler``); the
torch formulation below is the host path and the documented restatement the
kernel is tested against.  Every row-wise operation gives a row the same
values as the reference's per-row call, so the filtered distribution each row samples from is the
reference's (``filtered_logits`` is tested against a restatement of needle's
loop).  The draws come from one batched ``multinomial`` instead of one call
per row, so for a given seed the sampled ids differ from the reference's
while following the same distribution.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch
import torch.nn.functional as F


def filtered_logits(logits: torch.Tensor, temperature: Sequence[float], top_k: Sequence[int],
                    top_p: Sequence[float]) -> torch.Tensor:
    """Temperature, top-k and top-p applied to every row of ``logits``
    ``[n, V]`` (the reference's steps ``sampler.py:33-46``, batched).

    ``temperature`` (> 0), ``top_k`` (<= 0: off) and ``top_p`` (1: off) are
    per-row host values, so no device value is read back here.  Returns
    logits of the same dtype with the removed tokens at -inf.  Rounding as
    in the reference: ``x / t`` divides in fp32 and rounds once to the
    logits' dtype (a tensor-by-Python-scalar divide); the top-p comparison
    is made in the logits' dtype.
    """
    n, V = logits.shape
    dev, dt = logits.device, logits.dtype
    t = torch.tensor(list(temperature), dtype=torch.float32).to(dev, non_blocking=True)
    x = (logits.float() / t[:, None]).to(dt)
    ks = [min(int(k), V) if k > 0 else 0 for k in top_k]
    if any(ks):
        kmax = max(ks)
        kk = torch.tensor([max(k, 1) - 1 for k in ks]).to(dev, non_blocking=True)
        kth = x.topk(kmax, dim=-1).values.gather(1, kk[:, None])
        use_k = torch.tensor([k > 0 for k in ks]).to(dev, non_blocking=True)
        x = x.masked_fill((x < kth) & use_k[:, None], float("-inf"))
    prow = [i for i, p in enumerate(top_p) if p < 1.0]
    if prow:
        rows = torch.tensor(prow).to(dev, non_blocking=True)
        pp = torch.tensor([top_p[i] for i in prow], dtype=torch.float32).to(dev, non_blocking=True)
        xs = x[rows]
        sl, si = xs.sort(dim=-1, descending=True)
        probs = sl.softmax(dim=-1)
        cum = probs.cumsum(dim=-1)
        remove = cum - probs > pp.to(dt)[:, None]
        sl = sl.masked_fill(remove, float("-inf"))
        x = x.index_copy(0, rows, xs.scatter(1, si, sl))
    return x


def _step_params(owner, params_list, dev, generator):
    """The step's per-row (temperature, top_k, top_p, uniform) device arrays.
    An all-greedy step reuses arrays cached on ``owner`` (this library's
    Sampler, or needle's once ``patch_needle()`` bound ``Sampler.sample`` to
    it) and copies nothing; otherwise the parameters go over in one copy."""
    n = len(params_list)
    if all(p.temperature == 0.0 for p in params_list):
        g = getattr(owner, "_nb_greedy", None)
        if g is None or g[0].numel() < n or g[0].device != dev:
            m = max(n, 256)
            g = (torch.zeros(m, dtype=torch.float32, device=dev),
                 torch.zeros(m, dtype=torch.int32, device=dev),
                 torch.ones(m, dtype=torch.float32, device=dev),
                 torch.zeros(m, dtype=torch.float32, device=dev))
            owner._nb_greedy = g
        return g
    host = torch.empty(4 * n, dtype=torch.float32).pin_memory()
    host[:n] = torch.tensor([float(p.temperature) for p in params_list])
    host[n:2 * n].view(torch.int32)[:] = torch.tensor(
        [int(p.top_k) if p.top_k > 0 else 0 for p in params_list], dtype=torch.int32)
    host[2 * n:3 * n] = torch.tensor([float(p.top_p) for p in params_list])
    d = host.to(dev, non_blocking=True)
    if generator is not None and generator.device.type != "cuda":
        u = torch.rand(n, generator=generator).to(dev, non_blocking=True)
    else:
        u = torch.rand(n, device=dev, generator=generator)
    return d[:n], d[n:2 * n].view(torch.int32), d[2 * n:3 * n], u


class Sampler:
    """Drop-in for needle's ``Sampler`` (same ``sample`` signature).

    On CUDA logits the whole step is one ``nb_sample`` launch (greedy rows,
    temperature / top-k / top-p filtering and the draws) and one host read of
    the token ids; the per-row parameters go to the device in one copy (an
    all-greedy step reuses cached parameter arrays and copies nothing).  CPU
    logits (host callers and tests) take the batched torch path below.
    """

    @torch.no_grad()
    def sample(self, logits: torch.Tensor, params_list: Sequence,
               generator: Optional[torch.Generator] = None) -> List[int]:
        n = logits.shape[0]
        assert n == len(params_list)
        if n == 0:
            return []
        dev = logits.device
        if logits.is_cuda:
            from .. import ops
            t, k, p, u = _step_params(self, params_list, dev, generator)
            return ops.sample(logits, t, k, p, u).tolist()  # the step's only host read
        greedy = [p.temperature == 0.0 for p in params_list]
        ids = logits.argmax(dim=-1)
        if not all(greedy):
            rows = [i for i, g in enumerate(greedy) if not g]
            sel = torch.tensor(rows).to(dev, non_blocking=True)
            ps = [params_list[i] for i in rows]
            x = filtered_logits(logits[sel], [p.temperature for p in ps], [p.top_k for p in ps],
                                [p.top_p for p in ps])
            probs = F.softmax(x, dim=-1)
            drawn = torch.multinomial(probs, num_samples=1, generator=generator).flatten()
            ids = ids.index_copy(0, sel, drawn)
        return ids.tolist()  # the step's only device-to-host read
