"""The C ABI without a GPU: the library loads, exports every function that
include/fastembed_b200.h declares, validates arguments before touching the device,
and its host-only helpers (batch packing, cost-balanced shard planning) are right."""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "fastembed_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fe_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_op_and_engine_api():
    names = declared_functions()
    for must in ("fe_linear_bf16", "fe_attention_varlen_bf16", "fe_embed_layernorm", "fe_layernorm_dual",
                 "fe_linear_layernorm_bf16",
                 "fe_pool_l2", "fe_sgemm_nt", "fe_mha_f32", "fe_engine_create", "fe_engine_encode_packed",
                 "fe_engine_encode_host", "fe_plan_shards", "fe_plan_shards_costs"):
        assert must in names


def test_library_exports_every_declared_symbol(fe_lib):
    from fastembed_b200 import capi
    out = subprocess.run(["nm", "-D", "--defined-only", capi.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, missing
    # and the ctypes table binds exactly what the header declares
    assert sorted(capi.exported_symbols()) == declared_functions()


def test_status_strings(fe_lib):
    assert fe_lib.fe_status_string(0) == b"ok"
    assert b"invalid" in fe_lib.fe_status_string(1)
    assert fe_lib.fe_version().startswith(b"fastembed_b200")


def test_validation_happens_before_any_device_work(fe_lib):
    from fastembed_b200.capi import EPI, DTYPE
    buf = C.c_void_p(16)  # never dereferenced: every call below must be rejected first
    L = fe_lib
    assert L.fe_linear_bf16(buf, buf, None, None, buf, 4, 8, 60, EPI["none"], DTYPE["bf16"], None) == 1
    assert L.fe_linear_bf16(buf, buf, None, None, buf, 4, 8, 64, EPI["bias_residual"], DTYPE["bf16"], None) == 1
    assert L.fe_linear_bf16(buf, buf, None, None, buf, 4, 8, 64, EPI["bias"], DTYPE["bf16"], None) == 1
    assert L.fe_attention_varlen_bf16(buf, buf, 2, 10, 4, 128, buf, 20, None) == 4  # head_dim 128 unsupported
    assert L.fe_mha_f32(buf, buf, buf, buf, buf, buf, buf, buf, 10, 100, 3, buf, 1 << 20, None) == 1  # 100 % 3
    assert b"divisible" in L.fe_last_error_message()
    assert L.fe_embed_layernorm(buf, buf, 1, 4, buf, buf, buf, buf, buf, 100, 10, 10, 1e-12, buf, buf, None) == 4
    assert L.fe_pool_l2(buf, buf, 1, 64, 9, buf, None) == 1
    size = C.c_size_t(0)
    assert L.fe_linear_layernorm_workspace_bytes(4097, 1024, C.byref(size)) == 0
    assert size.value >= 4097 * 1024 * 4 + 4097 * 4 * 8  # fp32 scratch + (mean, M2) per row and part
    assert L.fe_linear_layernorm_workspace_bytes(4, 1024, None) == 1
    assert L.fe_linear_layernorm_bf16(buf, buf, buf, buf, buf, buf, None, 4, 640, 64, 1e-12, buf, 1 << 30,
                                      None) == 4  # row width 640 unsupported
    assert L.fe_linear_layernorm_bf16(buf, buf, buf, buf, buf, buf, None, 4, 1024, 64, 1e-12, buf, 64,
                                      None) == 1  # workspace too small
    # zero-sized work is a no-op
    assert L.fe_linear_bf16(None, None, None, None, None, 0, 8, 64, EPI["none"], DTYPE["bf16"], None) == 0
    assert L.fe_set_wait_limit(0, 0) == 1  # a zero limit is refused before any device is touched


def test_deferred_rmsnorm_entry_points_validate_before_device_work(fe_lib):
    """The deferred pre-norm step and its row-scaled consumers reject bad shapes and
    arguments without touching the device; the partial count is n / 256."""
    from fastembed_b200.capi import EPI, DTYPE
    buf = C.c_void_p(16)  # never dereferenced
    L = fe_lib
    assert [L.fe_linear_rmsnorm_deferred_parts(n) for n in (256, 768, 1024, 2048, 640, 2304, 0)] == [1, 3, 4, 8, 0, 0, 0]
    # n = 640 is not a multiple of 256; k = 60 is not a multiple of 8; a null row_ss
    assert L.fe_linear_rmsnorm_deferred_bf16(buf, buf, buf, buf, buf, buf, buf, 4, 640, 64, None) == 4
    assert L.fe_linear_rmsnorm_deferred_bf16(buf, buf, buf, buf, buf, buf, buf, 4, 1024, 60, None) == 1
    assert L.fe_linear_rmsnorm_deferred_bf16(buf, buf, buf, buf, buf, buf, None, 4, 1024, 64, None) == 1
    assert L.fe_linear_rmsnorm_deferred_bf16(None, None, None, None, None, None, None, 0, 1024, 64, None) == 0
    # ss_parts outside 1..8, or no row_ss for a non-empty input
    for parts, rss in ((0, buf), (9, buf), (4, None)):
        assert L.fe_linear_row_scaled_bf16(buf, buf, None, None, buf, 4, 256, 64, EPI["none"], DTYPE["bf16"], rss,
                                           parts, 1e-6, None) == 1
        assert L.fe_linear_qk_norm_rope_scaled_bf16(buf, buf, buf, buf, buf, buf, 4, 1024, 16, 8, 128, 0, 1e-6, 1e6,
                                                    rss, parts, None) == 1
    # the row-scaled linear keeps fe_linear_bf16's own checks (k = 60)
    assert L.fe_linear_row_scaled_bf16(buf, buf, None, None, buf, 4, 256, 60, EPI["none"], DTYPE["bf16"], buf, 4, 1e-6,
                                       None) == 1
    assert b"fe_linear_row_scaled_bf16" in L.fe_last_error_message()


def test_engine_create_without_gpu_fails_cleanly(fe_lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    from fastembed_b200 import capi
    cfg = capi.EncoderConfig(21128, 1024, 24, 16, 4096, 512, 2, 1e-12, 0, 0)
    h = C.c_void_p()
    st = fe_lib.fe_engine_create(C.byref(cfg), 0, C.byref(h))
    assert st != 0 and not h.value


def test_engine_config_validation(fe_lib):
    from fastembed_b200 import capi
    h = C.c_void_p()
    bad = capi.EncoderConfig(21128, 1000, 24, 16, 4096, 512, 2, 1e-12, 0, 0)  # 1000 % 16 != 0
    assert fe_lib.fe_engine_create(C.byref(bad), 0, C.byref(h)) == 4
    bad = capi.EncoderConfig(21128, 1024, 24, 8, 4096, 512, 2, 1e-12, 0, 0)  # head_dim 128
    assert fe_lib.fe_engine_create(C.byref(bad), 0, C.byref(h)) == 4


def test_pack_batch_is_exact(fe_lib):
    from fastembed_b200 import ops
    rng = np.random.default_rng(0)
    lengths = np.array([3, 0, 7, 1, 16], np.int32)
    ids = rng.integers(0, 1000, size=(5, 16)).astype(np.int32)
    packed, cu = ops.pack(ids, lengths)
    assert cu.tolist() == [0, 3, 3, 10, 11, 27]
    assert np.array_equal(packed, np.concatenate([ids[b, :L] for b, L in enumerate(lengths)]))
    with pytest.raises(Exception):
        ops.pack(ids, np.array([3, 0, 7, 1, 17], np.int32))  # longer than the stride


@pytest.mark.parametrize("parts", [2, 4, 8])
def test_plan_shards_matches_python_and_balances(fe_lib, parts):
    from fastembed_b200 import ops, workload as W
    shape = W.SHAPES["bge-large"]
    L = np.sort(W.sample_lengths(shape, batch=256 * parts))[::-1].copy()
    cuts = ops.plan_shards(shape, L, parts)
    assert cuts == W.balanced_cuts(shape, L, parts)
    assert cuts == sorted(cuts) and 0 < cuts[0] and cuts[-1] < L.size
    bounds = [0] + cuts + [L.size]
    work = [sum(shape.shard_cost(int(x)) for x in L[a:b]) for a, b in zip(bounds, bounds[1:])]
    assert max(work) / (sum(work) / parts) < 1.02  # within 2% of a perfect split
    with pytest.raises(Exception):
        ops.plan_shards(shape, L[::-1].copy(), parts)  # ascending order is rejected


@pytest.mark.parametrize("name", ["qwen3-0.6b", "gemma-300m"])
@pytest.mark.parametrize("parts", [2, 4, 8])
def test_plan_shards_rms_shapes(fe_lib, name, parts):
    """The Qwen3 / Gemma3 shapes split by their own per-sentence FLOPs
    (fe_plan_shards_costs), as bench.py does for torchrun ranks."""
    from fastembed_b200 import ops, workload as W
    shape = W.RMS_SHAPES[name]
    L = np.sort(W.sample_rms_lengths(shape, batch=shape.batch * parts))[::-1].copy()
    cuts = ops.plan_shards(shape, L, parts)
    assert cuts == W.balanced_cuts(shape, L, parts)
    bounds = [0] + cuts + [L.size]
    assert all(a < b for a, b in zip(bounds, bounds[1:]))
    work = [sum(shape.flops_per_sentence(int(x)) for x in L[a:b]) for a, b in zip(bounds, bounds[1:])]
    assert max(work) / (sum(work) / parts) < 1.02


def test_plan_shards_costs_matches_the_bert_planner(fe_lib):
    import ctypes as C
    from fastembed_b200 import capi, ops, workload as W
    shape = W.SHAPES["bge-base"]
    L = np.sort(W.sample_lengths(shape, batch=500, seed=3))[::-1].copy()
    costs = np.array([shape.shard_cost(int(x)) for x in L], np.float64)
    for parts in (1, 3, 8):
        cuts = np.zeros(max(parts - 1, 1), np.int32)
        capi.call("fe_plan_shards_costs", costs.ctypes.data_as(C.c_void_p), L.size, parts,
                  cuts.ctypes.data_as(C.c_void_p))
        assert [int(c) for c in cuts[:parts - 1]] == ops.plan_shards(shape, L, parts)
    bad = costs.copy()
    bad[5] = -1.0
    with pytest.raises(Exception):
        capi.call("fe_plan_shards_costs", bad.ctypes.data_as(C.c_void_p), L.size, 2,
                  np.zeros(1, np.int32).ctypes.data_as(C.c_void_p))


def test_coalescer_merges_concurrent_calls():
    """fe::Coalescer, which merges concurrent SentenceTransformer calls into one device
    batch (host-only: tests/cpp/coalescer_check.cpp)."""
    here = os.path.join(ROOT, "tests", "cpp")
    subprocess.run(["make", "-s", "-C", here, os.path.join(here, "coalescer_check")], check=True)
    r = subprocess.run([os.path.join(here, "coalescer_check")], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip() == "ok", r.stdout + r.stderr
