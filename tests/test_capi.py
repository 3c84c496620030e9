"""C-ABI checks that need no GPU: the library loads, exports every symbol the
header declares with the declared arity, and rejects invalid arguments on
the host before touching a device."""
import ctypes
import subprocess

import pytest

from needle_b200 import _lib as L


def test_header_declares_the_hot_path():
    decl = L.declared_functions()
    for name in ("nb_store_kvcache", "nb_rope", "nb_rope_store_kvcache", "nb_paged_decode",
                 "nb_paged_decode_plan", "nb_paged_decode_workspace_size",
                 "nb_prefill_attention", "nb_rmsnorm", "nb_fused_add_rmsnorm",
                 "nb_last_error", "nb_device_errors", "nb_abi_version", "nb_silu_mul",
                 "nb_swap_kv_blocks", "nb_tp_allreduce_add_rmsnorm", "nb_ipc_handle",
                 "nb_ipc_open", "nb_ipc_close", "nb_paged_decode_noalloc",
                 "nb_tp_set_wait_limit_ns", "nb_linear", "nb_sample", "nb_slot_mapping",
                 "nb_prefill_attention_paged"):
        assert name in decl, name


def test_library_exports_every_declared_symbol():
    lib = L.lib()
    out = subprocess.run(["nm", "-D", "--defined-only", L.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    for name in L.declared_functions():
        assert name in exported, f"{name} declared but not exported"
        assert getattr(lib, name) is not None
    assert lib.nb_abi_version() == 3


def test_no_torch_types_in_signatures():
    for name, (ret, params) in L.declared_functions().items():
        for typ, _ in params:
            assert "Tensor" not in typ and "at::" not in typ, (name, typ)


def _err(rc):
    return rc, L.lib().nb_last_error().decode()


def test_invalid_dtype_rejected_on_host():
    lib = L.lib()
    rc, msg = _err(lib.nb_store_kvcache(1, 64, 1, 64, 1, 4, 1, 16, 64, 1, 4, 4, None, 1, 1, 1,
                                        7, None))
    assert rc == L.NB_ERR_INVALID_ARG and "dtype" in msg


def test_store_kvcache_arg_checks():
    lib = L.lib()
    # k row stride smaller than kv_heads * head_dim
    rc, msg = _err(lib.nb_store_kvcache(16, 8, 16, 64, 16, 4, 1, 16, 64, 16, 4, 4, None, 16, 1, 1,
                                        L.NB_DTYPE_BF16, None))
    assert rc == L.NB_ERR_INVALID_ARG and "stride" in msg
    # decode form needs one token per sequence
    rc, msg = _err(lib.nb_store_kvcache(16, 64, 16, 64, 16, 4, 1, 16, 64, 16, 4, 4, None, 16, 2, 3,
                                        L.NB_DTYPE_BF16, None))
    assert rc == L.NB_ERR_INVALID_ARG and "cu_seqlens" in msg
    # block table narrower than its declared width
    rc, msg = _err(lib.nb_store_kvcache(16, 64, 16, 64, 16, 4, 1, 16, 64, 16, 2, 4, None, 16, 1, 1,
                                        L.NB_DTYPE_BF16, None))
    assert rc == L.NB_ERR_INVALID_ARG


def test_paged_decode_arg_checks():
    lib = L.lib()
    # 14 query heads over 3 KV heads is not a grouping
    rc, msg = _err(lib.nb_paged_decode(16, 14 * 64, 64, 16, 8, 3, 16, 64, 14, 16, 4, 4, 16, 1,
                                       0.125, 16, 14 * 64, 64, None, 0, 4, L.NB_DTYPE_BF16, None))
    assert rc == L.NB_ERR_INVALID_ARG and "multiple" in msg
    # split-K needs a workspace
    rc, msg = _err(lib.nb_paged_decode(16, 8 * 64, 64, 16, 8, 2, 16, 64, 8, 16, 16, 16, 16, 2,
                                       0.125, 16, 8 * 64, 64, None, 0, 4, L.NB_DTYPE_BF16, None))
    assert rc == L.NB_ERR_INVALID_ARG and "workspace" in msg


def test_decode_plan_and_workspace():
    lib = L.lib()
    pps, ms = ctypes.c_int(0), ctypes.c_int(0)
    assert lib.nb_paged_decode_plan(64, 8, 256, 16, ctypes.byref(pps), ctypes.byref(ms)) == 0
    assert 1 <= pps.value <= 128 and ms.value == -(-256 // pps.value)
    assert lib.nb_paged_decode_plan(1, 1, 1, 16, ctypes.byref(pps), ctypes.byref(ms)) == 0
    assert pps.value == 1 and ms.value == 1
    assert lib.nb_paged_decode_workspace_size(64, 32, 128, 1) == 0
    assert lib.nb_paged_decode_workspace_size(64, 32, 128, 3) == 64 * 32 * 3 * (128 * 4 + 8)
    assert lib.nb_paged_decode_plan(0, 8, 256, 16, ctypes.byref(pps), ctypes.byref(ms)) != 0


@pytest.mark.parametrize("fn", ["nb_rmsnorm"])
def test_norm_arg_checks(fn):
    lib = L.lib()
    rc, msg = _err(lib.nb_rmsnorm(16, 100, 16, 16, 128, 4, 128, 1e-6, L.NB_DTYPE_BF16, None))
    assert rc == L.NB_ERR_INVALID_ARG and "stride" in msg
    assert lib.nb_rmsnorm(16, 128, 16, 16, 128, 0, 128, 1e-6, L.NB_DTYPE_BF16, None) == 0


def test_bench_cpu_baseline_model_runs_on_a_tiny_config():
    """The extrapolated CPU leg of the model benchmarks (needle's CPU path for
    one decoder layer, x layers, + lm_head) runs and reports its sample."""
    import bench
    from needle_b200.model.config import ModelConfig
    cfg = ModelConfig(model_type="qwen2", hidden_size=64, num_hidden_layers=3,
                      num_attention_heads=4, num_key_value_heads=2, intermediate_size=96,
                      vocab_size=100, max_position_embeddings=512, rms_norm_eps=1e-6,
                      rope_theta=1e6)
    r = bench.cpu_baseline_model(cfg, [5, 40, 17], 0.5)
    assert r["extrapolated"] is True and r["kind"] == "port" and r["value"] > 0
    assert "x3 layers" in r["sample"]


def _ptrs(*vals):
    arr = (ctypes.c_void_p * len(vals))(*vals)
    return ctypes.cast(arr, ctypes.c_void_p), arr


def test_tp_allreduce_arg_checks():
    """nb_tp_allreduce_add_rmsnorm validates everything on the host."""
    lib = L.lib()
    recv, _r = _ptrs(4096, 8192)
    gath, _g = _ptrs(4096 * 3, 4096 * 5)
    ep = ctypes.cast(ctypes.c_void_p(4096 * 7), ctypes.POINTER(ctypes.c_uint))
    f = lib.nb_tp_allreduce_add_rmsnorm
    ok = dict(partial=4096, recv=recv, gather=gath, slot_rows=64, out=4096 * 9, res=4096 * 11,
              epochs=ep, rank=0, world=2, weight=4096 * 13, T=64, hidden=1024, eps=1e-6,
              dtype=L.NB_DTYPE_BF16)

    def call(**kw):
        a = dict(ok, **kw)
        return _err(f(a["partial"], a["recv"], a["gather"], a["slot_rows"], a["out"], a["res"],
                      a["epochs"], None, a["rank"], a["world"], a["weight"], a["T"],
                      a["hidden"], a["eps"], a["dtype"], None))
    assert call(dtype=L.NB_DTYPE_F32)[0] == L.NB_ERR_UNSUPPORTED
    assert call(partial=None)[0] == L.NB_ERR_INVALID_ARG
    assert call(world=9)[0] == L.NB_ERR_INVALID_ARG
    assert call(rank=2)[0] == L.NB_ERR_INVALID_ARG
    assert call(hidden=1028)[0] == L.NB_ERR_UNSUPPORTED
    assert call(hidden=16384)[0] == L.NB_ERR_UNSUPPORTED
    rc, msg = call(T=200)                          # 100 rows per rank > 64 slot rows
    assert rc == L.NB_ERR_INVALID_ARG and "slot rows" in msg
    rc, msg = call(T=2 * 1025, slot_rows=2048)     # more rows per rank than the kernel holds
    assert rc == L.NB_ERR_UNSUPPORTED
    rc, msg = call(weight=4096 + 2)
    assert rc == L.NB_ERR_INVALID_ARG and "aligned" in msg
    bad, _b = _ptrs(4096, 8192 + 8)
    rc, msg = call(recv=bad)
    assert rc == L.NB_ERR_INVALID_ARG and "aligned" in msg
    assert call(T=0)[0] == L.NB_OK                  # nothing to do, nothing launched


def test_tp_wait_limit_arg_checks():
    lib = L.lib()
    rc, msg = _err(lib.nb_tp_set_wait_limit_ns(61 * 10**9))
    assert rc == L.NB_ERR_INVALID_ARG and "60 s" in msg
    assert _err(lib.nb_tp_set_wait_limit_ns(0))[0] == L.NB_OK   # back to the default


def test_ipc_and_swap_and_silu_arg_checks():
    lib = L.lib()
    assert _err(lib.nb_ipc_handle(None, None, None))[0] == L.NB_ERR_INVALID_ARG
    assert _err(lib.nb_ipc_open(None, None))[0] == L.NB_ERR_INVALID_ARG
    src, _s = _ptrs(4096)
    dst, _d = _ptrs(8192)
    # block bytes must be a positive multiple of 16
    rc, msg = _err(lib.nb_swap_kv_blocks(src, dst, 1, 4096, 1, 10, 10, 100, None))
    assert rc == L.NB_ERR_INVALID_ARG and "multiple of 16" in msg
    rc, msg = _err(lib.nb_swap_kv_blocks(src, dst, 0, 4096, 1, 10, 10, 128, None))
    assert rc == L.NB_ERR_INVALID_ARG and "num_layers" in msg
    assert _err(lib.nb_swap_kv_blocks(src, dst, 1, 4096, 0, 10, 10, 128, None))[0] == L.NB_OK
    rc, msg = _err(lib.nb_silu_mul(4096, 100, 8192, 64, 4, 64, L.NB_DTYPE_BF16, None))
    assert rc == L.NB_ERR_INVALID_ARG and "stride" in msg
    assert _err(lib.nb_silu_mul(None, 128, 8192, 64, 4, 64, L.NB_DTYPE_BF16, None))[0] == \
        L.NB_ERR_INVALID_ARG


def test_swap_wrapper_rejects_mixed_layer_geometry():
    """Every layer is addressed with layer 0's block count and block size, so
    a layer of another shape is rejected before anything reaches the device."""
    import torch
    from needle_b200 import ops
    a = torch.zeros(2, 8, 2, 16, 64, dtype=torch.bfloat16)
    b = torch.zeros(2, 9, 2, 16, 64, dtype=torch.bfloat16)        # another block count
    d = torch.zeros(2, 8, 2, 16, 64, dtype=torch.bfloat16)
    pairs = torch.zeros(1, 2, dtype=torch.int32)
    with pytest.raises(ValueError, match="every source cache"):
        ops.swap_kv_blocks([a, b], [d, d], pairs)
    with pytest.raises(ValueError, match="every destination cache"):
        ops.swap_kv_blocks([a, a], [d, b], pairs)


def test_linear_arg_checks():
    lib = L.lib()
    # more than 256 rows: not this kernel's shape (caller keeps its GEMM)
    rc, msg = _err(lib.nb_linear(16, 64, 16, 64, None, 16, 64, 300, 64, 64, L.NB_DTYPE_BF16,
                                 None))
    assert rc == L.NB_ERR_UNSUPPORTED and "256" in msg
    rc, msg = _err(lib.nb_linear(16, 64, 16, 64, None, 16, 64, 8, 64, 64, L.NB_DTYPE_F32, None))
    assert rc == L.NB_ERR_UNSUPPORTED
    # K not a multiple of 8 (TMA rows must be 16-byte aligned)
    rc, msg = _err(lib.nb_linear(16, 68, 16, 68, None, 16, 64, 8, 64, 60, L.NB_DTYPE_BF16, None))
    assert rc == L.NB_ERR_UNSUPPORTED and "aligned" in msg
    rc, msg = _err(lib.nb_linear(16, 32, 16, 64, None, 16, 64, 8, 64, 64, L.NB_DTYPE_BF16, None))
    assert rc == L.NB_ERR_INVALID_ARG and "stride" in msg
    assert lib.nb_linear(16, 64, 16, 64, None, 16, 64, 0, 64, 64, L.NB_DTYPE_BF16, None) == 0


def test_paged_prefill_arg_checks():
    lib = L.lib()
    args = dict(q=16, qs=1024, cache=16, nblk=64, kvh=2, bt=16, bts=8, maxb=8, ctx=16, hq=8,
                d=128, cu=16, B=2, T=10, msl=5, scale=0.1, out=16, os=1024)

    def call(dtype=L.NB_DTYPE_BF16, **kw):
        a = dict(args, **kw)
        return _err(lib.nb_prefill_attention_paged(
            a["q"], a["qs"], a["cache"], a["nblk"], a["kvh"], a["bt"], a["bts"], a["maxb"],
            a["ctx"], a["hq"], a["d"], a["cu"], a["B"], a["T"], a["msl"], a["scale"], a["out"],
            a["os"], dtype, None))
    rc, msg = call(dtype=L.NB_DTYPE_F32)
    assert rc == L.NB_ERR_UNSUPPORTED
    rc, msg = call(d=96)
    assert rc == L.NB_ERR_UNSUPPORTED and "head_dim" in msg
    rc, msg = call(hq=7)
    assert rc == L.NB_ERR_INVALID_ARG and "multiple" in msg
    rc, msg = call(bts=4)
    assert rc == L.NB_ERR_INVALID_ARG
    rc, msg = call(qs=512)
    assert rc == L.NB_ERR_INVALID_ARG and "stride" in msg
    assert call(T=0)[0] == 0
