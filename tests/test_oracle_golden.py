"""Pin the CPU oracle to needle itself: every oracle function against the
golden vectors that ``tests/golden/make_golden.py`` produced by running
needle's own code.  Integer/byte work must match bit for bit; the floating
point ops are the same torch CPU ops as the reference and are compared
exactly too."""
import numpy as np
import pytest
import torch

from oracle import needle_oracle as no
from tests.golden import cases as C
from tests.golden.fixtures import load


def _changed(before, after):
    D = before.shape[-1]
    b = before.reshape(-1, D)
    a = after.reshape(-1, D)
    bits = torch.int16 if a.dtype == torch.bfloat16 else torch.int32
    diff = (a.view(bits) != b.view(bits)).any(dim=1).nonzero().flatten()
    return diff, C.crc(a[diff])


def _check_changed(before, after, gold):
    idx, crc = _changed(before, after)
    assert torch.equal(idx, gold["changed_idx"]), "written cache rows differ from needle's"
    assert crc == int(gold["changed_crc"]), "written cache contents differ from needle's"


def _exact(a, b):
    if a.dtype == torch.bfloat16:
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    else:
        assert torch.equal(a, b)


GOLD_KV = load("kv_write")
GOLD_DEC = load("decode")
GOLD_PRE = load("prefill")
GOLD_ROPE = load("rope")
GOLD_NORM = load("norm")


@pytest.mark.parametrize("dt", ["bfloat16", "float32"])
@pytest.mark.parametrize("kv,D", C.KV_WRITE_SHAPES)
def test_write_kv_matches_needle(dt, kv, D):
    x = C.kv_write_inputs(dt, kv, D)
    gold = GOLD_KV[f"write_kv_{dt}_kv{kv}_d{D}"]
    assert C.crc(*x.values()) == int(gold["input_crc"])
    before = x["cache"].clone()
    no.write_kv(x["k"], x["v"], x["cache"], x["block_table"], x["cu_seqlens"], x["context_lens"])
    _check_changed(before, x["cache"], gold)


@pytest.mark.parametrize("dt", ["bfloat16", "float32"])
def test_write_kv_clamp_matches_needle(dt):
    x = C.kv_write_clamp_inputs(dt)
    gold = GOLD_KV[f"write_kv_clamp_{dt}"]
    assert C.crc(*x.values()) == int(gold["input_crc"])
    before = x["cache"].clone()
    no.write_kv(x["k"], x["v"], x["cache"], x["block_table"], x["cu_seqlens"], x["context_lens"])
    _check_changed(before, x["cache"], gold)


@pytest.mark.parametrize("dt", ["bfloat16", "float32"])
@pytest.mark.parametrize("H,kv,D", C.DECODE_SHAPES)
def test_decode_matches_needle(dt, H, kv, D):
    x = C.decode_inputs(dt, H, kv, D)
    gold = GOLD_DEC[f"decode_{dt}_h{H}_kv{kv}_d{D}"]
    assert C.crc(*x.values()) == int(gold["input_crc"])
    before = x["cache"].clone()
    no.decode_write_kv(x["k"], x["v"], x["cache"], x["block_table"], x["context_lens"])
    _check_changed(before, x["cache"], gold)
    out = no.decode_attention(x["q"], x["cache"], x["block_table"], x["context_lens"],
                              no.default_scale(D), H, kv, D)
    _exact(out, gold["out"])


@pytest.mark.parametrize("dt", ["bfloat16", "float32"])
@pytest.mark.parametrize("H,kv,D", C.PREFILL_SHAPES)
def test_prefill_matches_needle(dt, H, kv, D):
    x = C.prefill_inputs(dt, H, kv, D)
    gold = GOLD_PRE[f"prefill_{dt}_h{H}_kv{kv}_d{D}"]
    assert C.crc(*[t for t in x.values() if isinstance(t, torch.Tensor)]) == int(gold["input_crc"])
    before = x["cache"].clone()
    no.write_kv(x["k"], x["v"], x["cache"], x["block_table"], x["cu_seqlens"], x["context_lens"])
    _check_changed(before, x["cache"], gold)
    out = no.prefill_attention(x["q"], x["k"], x["v"], x["cu_seqlens"], H, kv)
    _exact(out, gold["out"])


@pytest.mark.parametrize("dt", ["bfloat16", "float32"])
@pytest.mark.parametrize("H,kv,D,base", C.ROPE_SHAPES)
def test_rope_matches_needle(dt, H, kv, D, base):
    x = C.rope_inputs(dt, H, kv, D)
    gold = GOLD_ROPE[f"rope_{dt}_d{D}"]
    assert C.crc(*x.values()) == int(gold["input_crc"])
    cos, sin = no.rope_cache(D, 4096, base)
    cos = cos.to(C.DTYPES[dt])[x["positions"]]
    sin = sin.to(C.DTYPES[dt])[x["positions"]]
    _exact(cos, gold["cos"])
    _exact(sin, gold["sin"])
    qo, ko = no.apply_rope(x["q"], x["k"], cos, sin)
    _exact(qo, gold["q_out"])
    _exact(ko, gold["k_out"])


@pytest.mark.parametrize("dt", ["bfloat16", "float32"])
@pytest.mark.parametrize("hid,eps", C.NORM_SHAPES)
def test_rmsnorm_matches_needle(dt, hid, eps):
    x = C.norm_inputs(dt, hid)
    gold = GOLD_NORM[f"norm_{dt}_h{hid}"]
    assert C.crc(*x.values()) == int(gold["input_crc"])
    _exact(no.rms_norm(x["x"], x["weight"], eps), gold["y"])
    y, h = no.add_rms_norm(x["x"], x["residual"], x["weight"], eps)
    _exact(h, gold["h"])
    _exact(y, gold["y_add"])


def test_slot_mapping_integer_math():
    # two sequences, ctx 5 and 0, lengths 3 and 17, table width 2
    bt = np.array([[4, 9], [1, 2]])
    cu = np.array([0, 3, 20])
    ctx = np.array([5, 0])
    phys, off, seq = no.slot_mapping(bt, cu, ctx, 16)
    assert phys.tolist() == [4, 4, 4] + [1] * 16 + [2]
    assert off.tolist() == [5, 6, 7] + list(range(16)) + [0]
    assert seq.tolist() == [0] * 3 + [1] * 17


@pytest.mark.slow
def test_config1_greedy_tokens_match_needle():
    """Config 1 end to end (Qwen2-0.5B shape, fp32, 8 x 128 prompts, 65 tokens):
    the oracle's greedy tokens equal needle's engine output exactly."""
    from needle_b200.model.config import preset
    from needle_b200.synth import synth_state_dict
    from oracle.model_oracle import OracleModel, greedy_generate
    from tests.golden.fixtures import load_arrays
    g = load_arrays("e2e_config1")
    cfg = preset("qwen2-0.5b")
    torch.set_num_threads(max(1, torch.get_num_threads()))
    model = OracleModel(cfg, synth_state_dict(cfg, seed=0), dtype=torch.float32)
    prompts = g["prompts"].tolist()
    toks, margins = greedy_generate(model, prompts, g["tokens"].shape[1], num_gpu_blocks=256)
    assert np.array_equal(np.array(toks), g["tokens"])
    np.testing.assert_allclose(np.array(margins), g["margins"], rtol=0, atol=0)
