"""Bounded device waits: a wait that runs out is reported through the status word, the
kernel returns, and the device stays usable.

fe_set_wait_limit shortens the limit of the work waits to 1 microsecond.  The linear
layer below (128 x 256 output, K = 8192: one tile, a 128-block mainloop of tens of
microseconds) runs on the one-CTA tcgen05 kernel, whose epilogue warps wait for the
whole mainloop before their accumulator is ready, so that wait cannot complete in
time.  The test asserts FE_ERR_DEVICE_TIMEOUT from fe_device_status, restores the 2 s
default, and checks that the next call gives the same bits as a call made before.
The reference has no bounded waits: its CUDA ops exit() on an error
(src/ops/cuda/cuda_matrix_ops.cu:13-19)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

DEFAULT_NS = 2_000_000_000
TIMEOUT = 5  # FE_ERR_DEVICE_TIMEOUT


def test_wait_runs_out_then_recovers(cuda_dev):
    from fastembed_b200 import capi, ops
    L = capi.lib()
    g = torch.Generator(device=cuda_dev).manual_seed(11)
    m, n, k = 128, 256, 8192
    x = (torch.randn(m, k, device=cuda_dev, generator=g) * 0.1).to(torch.bfloat16)
    w = (torch.randn(n, k, device=cuda_dev, generator=g) * 0.1).to(torch.bfloat16)
    before = ops.linear_bf16(x, w, None, None, "none", "f32")
    torch.cuda.synchronize()
    assert L.fe_device_status(0) == 0
    assert L.fe_set_wait_limit(0, 1000) == 0
    try:
        ops.linear_bf16(x, w, None, None, "none", "f32")  # launches; the kernel gives up and returns
        st = L.fe_device_status(0)  # synchronises, reads and clears the word
    finally:
        assert L.fe_set_wait_limit(0, DEFAULT_NS) == 0
    assert st == TIMEOUT, capi.STATUS.get(st, st)
    assert b"wait ran out" in L.fe_last_error_message()
    after = ops.linear_bf16(x, w, None, None, "none", "f32")
    torch.cuda.synchronize()
    assert L.fe_device_status(0) == 0
    assert torch.equal(after, before)


def test_attention_wait_runs_out_then_recovers(cuda_dev):
    """The head_dim-64 attention under a 1 microsecond wait limit: a fold warp's first wait
    for its O spans the first item's K load, S, softmax and PV, so it runs out.  Every role
    leaves its loop, the producer and the S / PV issuer drain what they started, the CTA
    releases its TMEM, and the launch's work counter is reset by its last CTA: the next
    call, with the default limit, gives the same bits as a call made before."""
    import numpy as np
    from fastembed_b200 import capi, ops
    L = capi.lib()
    lens = [96, 300, 17, 128, 512, 64] * 8
    g = torch.Generator(device=cuda_dev).manual_seed(12)
    qkv = torch.randn(sum(lens), 3 * 16 * 64, device=cuda_dev, generator=g).to(torch.bfloat16)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device=cuda_dev)
    before = ops.attention_varlen(qkv, cu, max(lens), 16)
    torch.cuda.synchronize()
    assert L.fe_device_status(0) == 0
    assert L.fe_set_wait_limit(0, 1000) == 0
    try:
        ops.attention_varlen(qkv, cu, max(lens), 16)
        st = L.fe_device_status(0)
    finally:
        assert L.fe_set_wait_limit(0, DEFAULT_NS) == 0
    assert st == TIMEOUT, capi.STATUS.get(st, st)
    after = ops.attention_varlen(qkv, cu, max(lens), 16)
    torch.cuda.synchronize()
    assert L.fe_device_status(0) == 0
    assert torch.equal(after, before)


def test_wait_limit_rejects_bad_arguments(cuda_dev):
    from fastembed_b200 import capi
    assert capi.lib().fe_set_wait_limit(0, 0) == 1  # FE_ERR_INVALID_ARGUMENT
    assert capi.lib().fe_set_wait_limit(10_000, DEFAULT_NS) == 1  # no such device
