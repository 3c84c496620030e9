"""Batched sampler against needle's per-row recipe (CPU).

``filtered_logits`` must give every row exactly the logits needle's loop
produces before its draw (``oracle.needle_oracle.sampler_filtered_logits``
restates ``needle/model/sampler.py:33-46``), in bf16 and fp32; greedy rows
are the row argmax; draws land only on tokens the filter kept and follow
the filtered distribution.
"""
import pytest
import torch

from needle_b200.model.sampler import Sampler, filtered_logits
from needle_b200.model.sequence import SamplingParams
from oracle import needle_oracle as no

PARAMS = [(0.7, 50, 1.0), (1.0, -1, 0.9), (1.3, 5, 0.5), (0.5, 0, 0.95), (2.0, 2000, 0.3),
          (0.9, 1, 1.0), (1.0, -1, 1.0), (0.37, 17, 0.8)]


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_filtered_logits_match_needle_rows(dt):
    g = torch.Generator().manual_seed(0)
    V = 1000
    logits = (3 * torch.randn(len(PARAMS), V, generator=g)).to(dt)
    logits[2, 10:20] = logits[2, 10]  # ties at the top-k boundary
    got = filtered_logits(logits, [p[0] for p in PARAMS], [p[1] for p in PARAMS],
                          [p[2] for p in PARAMS])
    assert got.dtype == dt
    for i, (t, k, p) in enumerate(PARAMS):
        ref = no.sampler_filtered_logits(logits[i].clone(), t, k, p)
        assert torch.equal(got[i], ref), (i, (got[i] != ref).sum())


def test_sample_greedy_rows_and_allowed_tokens():
    g = torch.Generator().manual_seed(1)
    V = 300
    params = [SamplingParams(temperature=0.0), SamplingParams(temperature=0.8, top_k=3),
              SamplingParams(temperature=0.0), SamplingParams(temperature=1.0, top_p=0.6),
              SamplingParams(temperature=1.2, top_k=1)]
    logits = torch.randn(len(params), V, generator=g).to(torch.bfloat16)
    allowed = [no.sampler_filtered_logits(logits[i].clone(), p.temperature, p.top_k, p.top_p)
               if p.temperature > 0 else None for i, p in enumerate(params)]
    s = Sampler()
    for seed in range(20):
        ids = s.sample(logits, params, generator=torch.Generator().manual_seed(seed))
        assert ids[0] == int(logits[0].argmax()) and ids[2] == int(logits[2].argmax())
        assert ids[4] == int(logits[4].argmax())  # top_k = 1
        for i in (1, 3):
            assert torch.isfinite(allowed[i][ids[i]]), (seed, i, ids[i])
    assert s.sample(logits[:0], []) == []


def test_sample_follows_the_filtered_distribution():
    V = 6
    logits = torch.tensor([[2.0, 1.0, 0.5, 0.0, -1.0, -3.0]])
    params = [SamplingParams(temperature=0.9, top_k=4, top_p=0.95)]
    probs = torch.softmax(no.sampler_filtered_logits(logits[0].clone(), 0.9, 4, 0.95), -1)
    n = 20000
    big = logits.expand(n, V).contiguous()
    ids = torch.tensor(Sampler().sample(big, params * n,
                                        generator=torch.Generator().manual_seed(3)))
    freq = torch.bincount(ids, minlength=V).double() / n
    sigma = (probs.double() * (1 - probs.double()) / n).sqrt()
    assert torch.all((freq - probs.double()).abs() <= 5 * sigma + 1e-12), (freq, probs)


@pytest.mark.parametrize("dt", ["bfloat16", "float32"])
def test_oracle_and_batched_filter_pinned_to_needle(dt):
    """Golden case made by running needle's own Sampler.sample
    (tests/golden/make_golden.py): the probabilities it handed to
    torch.multinomial for every sampled row, and its greedy ids."""
    from tests.golden import cases as C
    from tests.golden.fixtures import load
    gold = load("sampler")[f"sampler_{dt}"]
    x = C.sampler_inputs(dt)
    assert int(gold["input_crc"]) == C.crc(*x.values())
    logits = x["logits"]
    rows = [i for i, (t, _, _) in enumerate(C.SAMPLER_PARAMS) if t > 0]
    for j, i in enumerate(rows):
        t, k, p = C.SAMPLER_PARAMS[i]
        probs = torch.softmax(no.sampler_filtered_logits(logits[i].clone(), t, k, p), dim=-1)
        assert torch.equal(probs, gold["probs"][j]), (dt, i)
    ps = [C.SAMPLER_PARAMS[i] for i in rows]
    got = torch.softmax(filtered_logits(logits[rows], [p[0] for p in ps], [p[1] for p in ps],
                                        [p[2] for p in ps]), dim=-1)
    assert torch.equal(got, gold["probs"])
    greedy = gold["greedy_rows"].tolist()
    assert [int(logits[i].argmax()) for i in greedy] == gold["greedy_ids"].tolist()
    params = [SamplingParams(temperature=t, top_k=k, top_p=p) for t, k, p in C.SAMPLER_PARAMS]
    ids = Sampler().sample(logits, params, generator=torch.Generator().manual_seed(0))
    assert [ids[i] for i in greedy] == gold["greedy_ids"].tolist()
