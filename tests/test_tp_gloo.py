"""Tensor-parallel host logic on CPU with two gloo ranks.

Under TP the attention heads and MLP columns shard across ranks with no
exchange inside the attention kernels; the only collective is the
row-parallel all-reduce after o_proj and down_proj
(needle/layers/linear.py:92-98).  This test checks, with world_size 2 on
gloo: the weight sharding rule (needle/model/loader.py:116-127), that the
per-rank head counts match needle's (needle/layers/attention.py:45-46), and
that a TP=2 attention-output + MLP block (column-parallel, local compute,
row-parallel all-reduce) equals the unsharded computation.
"""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

from needle_b200.layers.linear import ColumnParallelLinear, RowParallelLinear, shard_for_rank


def _worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        g = torch.Generator().manual_seed(0)
        hid, inter, T = 64, 96, 5
        Wg = torch.randn(inter, hid, generator=g)
        Wu = torch.randn(inter, hid, generator=g)
        Wd = torch.randn(hid, inter, generator=g)
        Wo = torch.randn(hid, hid, generator=g)
        attn = torch.randn(T, hid, generator=g)  # attention output, heads concatenated
        x = torch.randn(T, hid, generator=g)
        ref = F.linear(attn, Wo) + F.linear(F.silu(F.linear(x, Wg)) * F.linear(x, Wu), Wd)

        gate = ColumnParallelLinear(hid, inter, tp_size=world, tp_rank=rank)
        up = ColumnParallelLinear(hid, inter, tp_size=world, tp_rank=rank)
        down = RowParallelLinear(inter, hid, tp_size=world, tp_rank=rank)
        o = RowParallelLinear(hid, hid, tp_size=world, tp_rank=rank)
        with torch.no_grad():
            gate.weight.copy_(shard_for_rank("mlp.gate_proj.weight", Wg, world, rank))
            up.weight.copy_(shard_for_rank("mlp.up_proj.weight", Wu, world, rank))
            down.weight.copy_(shard_for_rank("mlp.down_proj.weight", Wd, world, rank))
            o.weight.copy_(shard_for_rank("self_attn.o_proj.weight", Wo, world, rank))
            # this rank's heads: the matching column slice of the attention output
            a_local = attn.narrow(1, rank * hid // world, hid // world)
            out = o(a_local) + down(F.silu(gate(x)) * up(x))
        err = (out - ref).abs().max().item()
        q.put((rank, err))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e)))


def test_row_parallel_allreduce_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert isinstance(res[r], float), res[r]
        assert res[r] < 1e-3, res


def test_shard_rule_round_trip():
    full = {
        "model.layers.0.self_attn.q_proj.weight": torch.arange(32 * 8.).view(32, 8),
        "model.layers.0.self_attn.q_proj.bias": torch.arange(32.),
        "model.layers.0.self_attn.o_proj.weight": torch.arange(8 * 32.).view(8, 32),
        "model.layers.0.mlp.down_proj.weight": torch.arange(8 * 16.).view(8, 16),
        "model.norm.weight": torch.arange(8.),
    }
    for tp in (1, 2, 4, 8):
        for name, t in full.items():
            parts = [shard_for_rank(name, t, tp, r) for r in range(tp)]
            if name.endswith(("o_proj.weight", "down_proj.weight")):
                assert torch.equal(torch.cat(parts, 1), t)
            elif name.endswith(("q_proj.weight", "q_proj.bias")):
                assert torch.equal(torch.cat(parts, 0), t)
            else:
                assert all(torch.equal(p, t) for p in parts)


@pytest.mark.parametrize("H,KV,tp,hl,kvl", [(32, 8, 2, 16, 4), (32, 8, 8, 4, 1),
                                            (64, 8, 8, 8, 1), (14, 2, 2, 7, 1)])
def test_per_rank_head_counts_match_needle(H, KV, tp, hl, kvl):
    """needle/layers/attention.py:45-46: H // tp query heads and
    max(1, KV // tp) KV heads per rank."""
    from needle_b200.model.config import ModelConfig
    cfg = ModelConfig(hidden_size=H * 64, num_attention_heads=H, num_key_value_heads=KV)
    with torch.device("meta"):
        from needle_b200.layers.attention import Attention
        a = Attention(cfg, 0, tp_size=tp, tp_rank=0)
    assert (a.num_heads, a.num_kv_heads) == (hl, kvl)
    assert a.q_proj.weight.shape[0] == hl * 64 and a.k_proj.weight.shape[0] == kvl * 64


class _HostComm:
    """Stand-in for ``TPComm`` with the same interface, reducing with gloo on
    the CPU: checks that ``RowParallelLinear`` hands its partial sum to the
    following ``RMSNorm`` and that the norm receives the residual."""

    def __init__(self, max_tokens, hidden):
        self.partial = torch.zeros(max_tokens, hidden)
        self.residual = torch.zeros(max_tokens, hidden)
        self.max_tokens = max_tokens
        self.calls = 0

    def can_fuse(self, n):
        return 0 < n <= self.max_tokens

    def is_partial(self, x):
        return x.data_ptr() == self.partial.data_ptr()

    def allreduce_add_rmsnorm(self, T, residual, weight, eps):
        from oracle.needle_oracle import add_rms_norm
        self.calls += 1
        s = self.partial[:T].clone()
        dist.all_reduce(s)
        y, h = add_rms_norm(s, residual, weight, eps)
        self.residual[:T].copy_(h)
        return y, self.residual[:T]


def _fused_worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from needle_b200.layers.norm import RMSNorm
        from needle_b200.layers.tp_comm import attach
        from oracle.needle_oracle import add_rms_norm
        g = torch.Generator().manual_seed(0)
        hid, T = 64, 5
        Wo = torch.randn(hid, hid, generator=g)
        attn = torch.randn(T, hid, generator=g)
        res = torch.randn(T, hid, generator=g)
        nw = 1 + 0.1 * torch.randn(hid, generator=g)
        ref_y, ref_h = add_rms_norm(F.linear(attn, Wo), res, nw, 1e-6)
        blk = torch.nn.ModuleDict({"o": RowParallelLinear(hid, hid, tp_size=world, tp_rank=rank),
                                   "norm": RMSNorm(hid, eps=1e-6)})
        comm = _HostComm(16, hid)
        attach(blk, comm)
        with torch.no_grad():
            blk["o"].weight.copy_(shard_for_rank("self_attn.o_proj.weight", Wo, world, rank))
            blk["norm"].weight.copy_(nw)
            part = blk["o"](attn.narrow(1, rank * hid // world, hid // world))
            assert comm.is_partial(part)
            y, h = blk["norm"](part, res)
        attach(blk, None)
        assert blk["o"].comm is None and blk["norm"].comm is None
        q.put((rank, (comm.calls, float((y - ref_y).abs().max()), float((h - ref_h).abs().max()))))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e)))


def test_deferred_allreduce_reaches_norm_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 28500 + os.getpid() % 1000
    procs = [ctx.Process(target=_fused_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert isinstance(res[r], tuple), res[r]
        calls, ey, eh = res[r]
        assert calls == 1 and ey < 1e-4 and eh < 1e-4, res
