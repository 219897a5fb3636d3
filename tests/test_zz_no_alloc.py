"""The allocation-free attention entry point, fe_mha_f32_noalloc, checked against
fe_mha_f32 (the same computation with a caller-provided workspace) through the C ABI.

It exists for callers that cannot allocate device memory on demand (hosts whose
device memory belongs to another allocator, serving loops that must not call
cudaMalloc / cudaFree mid-request): its Q/K/V scratch is a fixed array inside the
library.  Calls in a row with different shapes, a large one before a small one and
back, check that the shared scratch carries nothing from one call into the next: both
entry points run the same kernels in the same order, so their outputs must agree bit
for bit.  This file is collected last."""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

def _run(fn, tensors, L, D, H, extra=()):
    from fastembed_b200 import capi
    x, wq, wk, wv, bq, bk, bv = tensors
    out = torch.empty(L * D, dtype=torch.float32, device=x.device)
    ptrs = [C.c_void_p(t.data_ptr()) for t in (x, wq, wk, wv, bq, bk, bv, out)]
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    capi.call(fn, *ptrs, L, D, H, *extra, stream)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def _inputs(L, D, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    mk = lambda n: (torch.rand(n, device=dev, generator=g) * 2 - 1)
    return [mk(L * D), mk(D * D), mk(D * D), mk(D * D), mk(D), mk(D), mk(D)]


def test_noalloc_matches_workspace_version_twice(cuda_dev):
    from fastembed_b200 import capi
    # large, then small (the small call must not read the large call's leftovers), then the maximum
    for (L, D, H, seed) in [(200, 512, 8, 2), (10, 1024, 16, 1), (256, 1024, 16, 3)]:
        t = _inputs(L, D, seed, cuda_dev)
        nbytes = capi.lib().fe_mha_f32_workspace_bytes(L, D, H)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=cuda_dev)
        ref = _run("fe_mha_f32", t, L, D, H, extra=(C.c_void_p(ws.data_ptr()), nbytes))
        got = _run("fe_mha_f32_noalloc", t, L, D, H)
        assert np.array_equal(got, ref), float(np.abs(got - ref).max())


def test_noalloc_rejects_oversize(cuda_dev):
    from fastembed_b200 import capi
    L, D, H = 300, 1024, 16  # 307,200 elements per projection > 262,144
    t = _inputs(8, D, 3, cuda_dev)
    out = torch.empty(L * D, dtype=torch.float32, device=cuda_dev)
    ptrs = [C.c_void_p(x.data_ptr()) for x in t] + [C.c_void_p(out.data_ptr())]
    st = capi.lib().fe_mha_f32_noalloc(*ptrs, L, D, H, None)
    assert st == 4  # FE_ERR_UNSUPPORTED
    assert b"scratch" in capi.lib().fe_last_error_message()
