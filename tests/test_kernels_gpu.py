"""Parity of each CUDA kernel, called through the C ABI, on a B200.

Floating-point kernels are compared with a plain PyTorch fp32 computation on the
same (bf16-rounded, where the kernel takes bf16) inputs; the tolerance is written
beside each check.  Index work (sentence offsets, positions, pooled rows) must be
exact and is checked with equality."""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel_err(a, b):
    return float((a.float() - b.float()).abs().max() / (b.float().abs().max() + 1e-12))


# ------------------------------------------------------------ tcgen05 linear
LINEAR_SHAPES = [
    (1, 128, 64),       # single row, BN=128 tile, one k-block
    (130, 256, 64),     # ragged M tail
    (200, 384, 128),    # N = 3 x 128 -> BN=128
    (333, 1024, 1024),  # out-proj shape, ragged M
    (1000, 3072, 1024), # QKV shape
    (257, 4096, 1024),  # FFN1 shape
    (129, 1024, 4096),  # FFN2 shape (long K)
    (64, 512, 72),      # K not a multiple of 64 (TMA zero fill)
    (96, 1000, 64),     # N not a multiple of 64 (clipped store)
    (700, 1024, 4096),  # 2-CTA pair tiles, ragged last pair
    (4097, 256, 64),    # 2-CTA, many m tiles, peer half of the last tile out of range
    (520, 768, 72),     # 2-CTA with a zero-filled K tail
]


@pytest.mark.parametrize("pair", ["1", "0"])
@pytest.mark.parametrize("m,n,k", LINEAR_SHAPES)
@pytest.mark.parametrize("epi,out", [("none", "f32"), ("bias", "bf16"), ("bias_gelu", "bf16"),
                                     ("bias_swish", "bf16"), ("bias_residual", "f32")])
def test_linear_bf16(cuda_dev, monkeypatch, m, n, k, epi, out, pair):
    """Both linear kernels: the 2-CTA pair kernel (default for m >= 512 and n % 256 == 0)
    and the 1-CTA kernel (FE_LINEAR_PAIR=0)."""
    from fastembed_b200 import ops
    monkeypatch.setenv("FE_LINEAR_PAIR", pair)
    g = torch.Generator(device=cuda_dev).manual_seed(m * 7 + n + k)
    x = torch.randn(m, k, device=cuda_dev, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, device=cuda_dev, generator=g) / math.sqrt(k)).to(torch.bfloat16)
    bias = torch.randn(n, device=cuda_dev, generator=g) * 0.1
    res = torch.randn(m, n, device=cuda_dev, generator=g)
    y = ops.linear_bf16(x, w, bias if epi != "none" else None, res if epi == "bias_residual" else None, epi, out)
    ref = x.float() @ w.float().T
    if epi != "none":
        ref = ref + bias
    if epi == "bias_gelu":
        ref = 0.5 * ref * (1 + torch.tanh(math.sqrt(2 / math.pi) * (ref + 0.044715 * ref ** 3)))
    if epi == "bias_swish":
        ref = ref * torch.sigmoid(ref)
    if epi == "bias_residual":
        ref = ref + res
    torch.cuda.synchronize()
    # fp32 out: only the accumulation order differs -> 1e-4 relative to the output scale;
    # bf16 out: one bf16 rounding (2^-8 relative) plus the hardware tanh / ex2 / rcp -> 1e-2.
    tol = 1e-4 if out == "f32" else 1e-2
    assert _rel_err(y, ref) < tol
    ops.device_status(0)


def test_linear_rejects_bad_shapes(cuda_dev):
    from fastembed_b200 import ops
    from fastembed_b200.capi import FeError
    x = torch.zeros(4, 60, dtype=torch.bfloat16, device=cuda_dev)
    w = torch.zeros(8, 60, dtype=torch.bfloat16, device=cuda_dev)
    with pytest.raises(FeError):  # k % 8 != 0
        ops.linear_bf16(x, w)
    with pytest.raises(FeError):  # the residual epilogue needs a residual
        ops.linear_bf16(torch.zeros(4, 64, dtype=torch.bfloat16, device=cuda_dev),
                        torch.zeros(8, 64, dtype=torch.bfloat16, device=cuda_dev),
                        torch.zeros(8, device=cuda_dev), None, "bias_residual", "f32")


def test_linear_deterministic_and_row_independent(cuda_dev):
    """Each output row depends only on its own input row: computing a row block
    alone gives bit-identical results (the batch-invariance the engine relies on)."""
    from fastembed_b200 import ops
    g = torch.Generator(device=cuda_dev).manual_seed(3)
    x = torch.randn(700, 1024, device=cuda_dev, generator=g).to(torch.bfloat16)
    w = (torch.randn(3072, 1024, device=cuda_dev, generator=g) / 32).to(torch.bfloat16)
    b = torch.randn(3072, device=cuda_dev, generator=g)
    y1 = ops.linear_bf16(x, w, b, None, "bias", "bf16")
    y2 = ops.linear_bf16(x, w, b, None, "bias", "bf16")
    y3 = ops.linear_bf16(x[300:437].contiguous(), w, b, None, "bias", "bf16")
    assert torch.equal(y1, y2)
    assert torch.equal(y1[300:437], y3)  # 1-CTA kernel for the block, pair kernel for the batch


# ------------------------------------------------------------ varlen attention
def _attn_ref(qkv, lens, heads, hd=64):
    D = heads * hd
    out = torch.zeros(qkv.shape[0], D, device=qkv.device)
    s = 0
    for L in lens:
        q = qkv[s:s + L, :D].float().view(L, heads, hd).transpose(0, 1)
        k = qkv[s:s + L, D:2 * D].float().view(L, heads, hd).transpose(0, 1)
        v = qkv[s:s + L, 2 * D:].float().view(L, heads, hd).transpose(0, 1)
        p = torch.softmax(q @ k.transpose(1, 2) / math.sqrt(hd), dim=-1)
        out[s:s + L] = (p @ v).transpose(0, 1).reshape(L, D)
        s += L
    return out


@pytest.mark.parametrize("lens,heads", [
    ([1], 1), ([7, 1, 63], 2), ([64, 65, 127, 128, 129], 4), ([200, 255, 256, 257], 16),
    ([512, 3, 511, 300], 12), ([96] * 40, 16)])
def test_attention_varlen(cuda_dev, lens, heads):
    from fastembed_b200 import ops
    g = torch.Generator(device=cuda_dev).manual_seed(sum(lens) + heads)
    T = sum(lens)
    qkv = torch.randn(T, 3 * heads * 64, device=cuda_dev, generator=g).to(torch.bfloat16)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device=cuda_dev)
    out = ops.attention_varlen(qkv, cu, max(lens), heads)
    ref = _attn_ref(qkv, lens, heads)
    torch.cuda.synchronize()
    # P is rounded to bf16 before PV (2^-9 relative per weight) and O to bf16: 2e-2 abs on unit-scale V.
    assert float((out.float() - ref).abs().max()) < 2e-2
    ops.device_status(0)


def test_attention_many_sentences_and_repeat(cuda_dev):
    """More sentences than one launch takes (2048): the batch runs as chunks, each
    handing out its units from its own work counter; a repeat is bit-identical."""
    from fastembed_b200 import ops
    rng = np.random.default_rng(4)
    lens = rng.integers(0, 40, size=2300).tolist()
    lens[5] = 300  # one multi-tile sentence among many short and empty ones
    heads = 2
    g = torch.Generator(device=cuda_dev).manual_seed(4)
    T = sum(lens)
    qkv = torch.randn(T, 3 * heads * 64, device=cuda_dev, generator=g).to(torch.bfloat16)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device=cuda_dev)
    out1 = ops.attention_varlen(qkv, cu, max(lens), heads)
    out2 = ops.attention_varlen(qkv, cu, max(lens), heads)
    ref = _attn_ref(qkv, lens, heads)
    torch.cuda.synchronize()
    assert float((out1.float() - ref).abs().max()) < 2e-2
    assert torch.equal(out1, out2)
    ops.device_status(0)


def _attn_gqa_ref(qkv, lens, hq, hkv, hd, causal, scale):
    out = torch.zeros(qkv.shape[0], hq * hd, device=qkv.device)
    kc, vc = hq * hd, (hq + hkv) * hd
    s = 0
    for L in lens:
        if L == 0:
            continue
        q = qkv[s:s + L, :kc].float().view(L, hq, hd).transpose(0, 1)
        k = qkv[s:s + L, kc:vc].float().view(L, hkv, hd).transpose(0, 1).repeat_interleave(hq // hkv, 0)
        v = qkv[s:s + L, vc:].float().view(L, hkv, hd).transpose(0, 1).repeat_interleave(hq // hkv, 0)
        sc = q @ k.transpose(1, 2) * scale
        if causal:
            sc = sc.masked_fill(torch.ones(L, L, dtype=torch.bool, device=qkv.device).triu(1), float("-inf"))
        out[s:s + L] = (torch.softmax(sc, -1) @ v).transpose(0, 1).reshape(L, hq * hd)
        s += L
    return out


@pytest.mark.parametrize("hd,hq,hkv,causal,lens", [
    (128, 16, 8, True, [1, 7, 128, 129, 300, 64, 511]),
    (128, 4, 4, False, [200, 3, 128, 255]),
    (128, 8, 2, True, [1024, 40]),
    (256, 3, 1, False, [1, 8, 100, 256, 257, 33]),
    (256, 4, 2, True, [130, 12, 384]),
])
def test_attention_gqa(cuda_dev, hd, hq, hkv, causal, lens):
    """Grouped-query attention for head_dim 128 / 256 against fp32 torch: causal and
    bidirectional, ragged lengths, several 128-key items per unit (O rescaled in TMEM)."""
    from fastembed_b200 import ops
    g = torch.Generator(device=cuda_dev).manual_seed(sum(lens) + hd + hq)
    T = sum(lens)
    qkv = (torch.randn(T, (hq + 2 * hkv) * hd, device=cuda_dev, generator=g) * 1.5).to(torch.bfloat16)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device=cuda_dev)
    out = ops.attention_gqa(qkv, cu, max(lens), hq, hkv, hd, causal)
    ref = _attn_gqa_ref(qkv, lens, hq, hkv, hd, causal, hd ** -0.5)
    torch.cuda.synchronize()
    # P rounded to bf16 (2^-9 relative per weight), O to bf16: 3e-2 abs on unit-scale V
    assert float((out.float() - ref).abs().max()) < 3e-2
    ops.device_status(0)


def test_attention_sharp_softmax(cuda_dev):
    """Large scores (near one-hot rows) exercise the online max / rescale across key tiles."""
    from fastembed_b200 import ops
    g = torch.Generator(device=cuda_dev).manual_seed(11)
    lens = [300, 129, 17]
    T = sum(lens)
    qkv = (torch.randn(T, 3 * 2 * 64, device=cuda_dev, generator=g) * 3).to(torch.bfloat16)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device=cuda_dev)
    out = ops.attention_varlen(qkv, cu, max(lens), 2)
    ref = _attn_ref(qkv, lens, 2)
    assert float((out.float() - ref).abs().max()) < 6e-2  # |V| up to ~12: 2^-8 relative of the output scale


# ------------------------------------------------------------ row kernels
def test_embed_layernorm_exact_indexing(cuda_dev):
    from fastembed_b200 import ops
    g = torch.Generator(device=cuda_dev).manual_seed(5)
    V, P, D = 1000, 512, 1024
    word = torch.randn(V, D, device=cuda_dev, generator=g)
    pos = torch.randn(P, D, device=cuda_dev, generator=g)
    typ = torch.randn(2, D, device=cuda_dev, generator=g)
    gam = torch.rand(D, device=cuda_dev, generator=g) + 0.5
    bet = torch.randn(D, device=cuda_dev, generator=g)
    lens = [1, 5, 512, 33]
    ids = torch.randint(0, V, (sum(lens),), device=cuda_dev, generator=g, dtype=torch.int32)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device=cuda_dev)
    h32, h16 = ops.embed_layernorm(ids, cu, word, pos, typ, gam, bet, 1e-12)
    posids = torch.cat([torch.arange(L, device=cuda_dev) for L in lens])
    x = word[ids.long()] + pos[posids] + typ[0]
    mu = x.mean(-1, keepdim=True)
    var = ((x - mu) ** 2).mean(-1, keepdim=True)
    ref = (x - mu) / torch.sqrt(var + 1e-12) * gam + bet
    assert float((h32 - ref).abs().max()) < 5e-5
    assert torch.equal(h16, h32.to(torch.bfloat16))


def test_layernorm_dual(cuda_dev):
    from fastembed_b200 import ops
    g = torch.Generator(device=cuda_dev).manual_seed(6)
    for D in (512, 768, 1024, 640):
        x = torch.randn(777, D, device=cuda_dev, generator=g) * 3 + 1
        gam = torch.randn(D, device=cuda_dev, generator=g)
        bet = torch.randn(D, device=cuda_dev, generator=g)
        h32, h16 = ops.layernorm_dual(x, gam, bet, 1e-12)
        ref = torch.nn.functional.layer_norm(x, (D,), gam, bet, 1e-12)
        assert float((h32 - ref).abs().max()) < 1e-4
        assert torch.equal(h16, h32.to(torch.bfloat16))
        if D in (512, 768, 1024):  # residual form: LN(x + res), sum formed in the kernel
            res = torch.randn(777, D, device=cuda_dev, generator=g)
            h32r, h16r = ops.layernorm_dual(x, gam, bet, 1e-12, residual=res)
            refr = torch.nn.functional.layer_norm(x + res, (D,), gam, bet, 1e-12)
            assert float((h32r - refr).abs().max()) < 1e-4
            assert torch.equal(h16r, h32r.to(torch.bfloat16))


def test_embed_layernorm_xlmr_rows(cuda_dev):
    """fe_embed_layernorm_xlmr: pad tokens take position row 0, the others rows 2, 3, ... of
    their sentence, a row at or past the table row 0; against the fp32 torch composition."""
    from fastembed_b200 import ops
    g = torch.Generator(device=cuda_dev).manual_seed(5)
    D, V, P, pad = 768, 300, 40, 1
    lens = [1, 3, 38, 39, 45, 17]
    T = sum(lens)
    ids = torch.randint(0, 6, (T,), device=cuda_dev, generator=g).to(torch.int32)  # many pads
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device=cuda_dev)
    word = torch.randn(V, D, device=cuda_dev, generator=g)
    pos = torch.randn(P, D, device=cuda_dev, generator=g)
    typ = torch.randn(1, D, device=cuda_dev, generator=g)
    gam = torch.randn(D, device=cuda_dev, generator=g)
    bet = torch.randn(D, device=cuda_dev, generator=g)
    h32, h16 = ops.embed_layernorm(ids, cu, word, pos, typ, gam, bet, 1e-5, pad_id=pad)
    rows, host = [], ids.cpu().numpy()
    for s, L in zip(np.cumsum([0] + lens[:-1]), lens):
        nxt = 2
        for t in range(s, s + L):
            r = 0 if host[t] == pad else nxt
            nxt += int(host[t] != pad)
            rows.append(r if r < P else 0)
    x = word[ids.long()] + pos[torch.tensor(rows, device=cuda_dev)] + typ[0]
    ref = torch.nn.functional.layer_norm(x, (D,), gam, bet, 1e-5)
    assert float((h32 - ref).abs().max()) < 1e-4
    assert torch.equal(h16, h32.to(torch.bfloat16))
    ops.device_status(0)


# ----------------------------------------- linear + residual + LayerNorm, one launch
def _linear_ln_ref(x, w, b, res, gam, bet, eps):
    y = (x.float() @ w.float().T + b) + res
    return torch.nn.functional.layer_norm(y, (w.shape[0],), gam, bet, eps)


def _linear_ln_inputs(m, n, k, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, device=dev, generator=g) / math.sqrt(k)).to(torch.bfloat16)
    b = torch.randn(n, device=dev, generator=g) * 0.1
    res = torch.randn(m, n, device=dev, generator=g) * 2 + 0.5
    gam = torch.randn(n, device=dev, generator=g)
    bet = torch.randn(n, device=dev, generator=g)
    return x, w, b, res, gam, bet


# (m, n, k): the one-launch form (k >= 2048) with the row-statistics exchange across 4, 3,
# 1, 2 and 8 column tiles of 256, a single 256-row tile among them; and the two-launch
# form (linear, then LayerNorm) for k < 2048 and for n = 384.
LINEAR_LN_SHAPES = [(700, 1024, 4096), (4097, 768, 3072), (300, 256, 2048), (33, 512, 2048), (1000, 2048, 2048),
                    (700, 1024, 1024), (520, 384, 384)]


@pytest.mark.parametrize("pair", ["1", "0"])
@pytest.mark.parametrize("m,n,k", LINEAR_LN_SHAPES)
def test_linear_layernorm(cuda_dev, monkeypatch, m, n, k, pair):
    """h32 <- LN((x W^T + b) + h32) against the fp32 composition of the same steps;
    FE_LINEAR_PAIR=0 takes the two-launch form for every shape."""
    from fastembed_b200 import ops
    monkeypatch.setenv("FE_LINEAR_PAIR", pair)
    x, w, b, res, gam, bet = _linear_ln_inputs(m, n, k, m + n + k, cuda_dev)
    ref = _linear_ln_ref(x, w, b, res, gam, bet, 1e-12)
    h32, h16 = ops.linear_layernorm(x, w, b, gam, bet, res.clone(), 1e-12)
    torch.cuda.synchronize()
    assert float((h32 - ref).abs().max()) < 1e-4
    assert torch.equal(h16, h32.to(torch.bfloat16))
    ops.device_status(0)


# (m, n, k, mode): the cluster form (linear_ln_cluster: R = n / 256 CTAs per 128-row block,
# row statistics exchanged through distributed shared memory) at 2, 3 and 4 CTAs, one
# row, partial and exact row blocks, the bge-large out-projection shape, and K = 4096
# (FE_LN_CLUSTER=all takes it there too)
LINEAR_LN_CLUSTER_SHAPES = [(1, 1024, 1024, "1"), (129, 512, 1024, "1"), (4097, 768, 768, "1"), (256, 1024, 1024, "1"),
                            (26508, 1024, 1024, "1"), (700, 1024, 4096, "all"), (3001, 768, 3072, "all")]


@pytest.mark.parametrize("m,n,k,mode", LINEAR_LN_CLUSTER_SHAPES)
def test_linear_layernorm_cluster(cuda_dev, monkeypatch, m, n, k, mode):
    """The cluster form against the fp32 composition of the same steps; repeated calls and a
    row block computed alone are bit-identical to the batch (each row depends only on itself)."""
    from fastembed_b200 import ops
    monkeypatch.setenv("FE_LN_CLUSTER", mode)
    x, w, b, res, gam, bet = _linear_ln_inputs(m, n, k, m + n + k + 1, cuda_dev)
    ref = _linear_ln_ref(x, w, b, res, gam, bet, 1e-12)
    h32, h16 = ops.linear_layernorm(x, w, b, gam, bet, res.clone(), 1e-12)
    again, _ = ops.linear_layernorm(x, w, b, gam, bet, res.clone(), 1e-12)
    torch.cuda.synchronize()
    assert float((h32 - ref).abs().max()) < 1e-4
    assert torch.equal(h16, h32.to(torch.bfloat16))
    assert torch.equal(again, h32)
    if m > 200:
        part, _ = ops.linear_layernorm(x[37:200].contiguous(), w, b, gam, bet, res[37:200].clone(), 1e-12)
        assert torch.equal(part, h32[37:200])
    ops.device_status(0)


def test_linear_layernorm_workspace_reuse_and_determinism(cuda_dev):
    """One workspace sized for the largest m serves calls with smaller m in between
    (every call leaves its counters at zero); repeated calls are bit-identical, a row
    block computed alone equals its rows of the batch, and h16 may be omitted."""
    from fastembed_b200 import ops
    n, k = 1024, 4096
    ws = ops.linear_layernorm_workspace(4097, n, cuda_dev)
    outs = {}
    for m in (4097, 700, 4097, 137, 700):
        x, w, b, res, gam, bet = _linear_ln_inputs(m, n, k, m, cuda_dev)
        h32, h16 = ops.linear_layernorm(x, w, b, gam, bet, res.clone(), 1e-12, workspace=ws)
        torch.cuda.synchronize()
        assert float((h32 - _linear_ln_ref(x, w, b, res, gam, bet, 1e-12)).abs().max()) < 1e-4
        if m in outs:
            assert torch.equal(outs[m], h32)
        outs[m] = h32
    x, w, b, res, gam, bet = _linear_ln_inputs(700, n, k, 700, cuda_dev)
    part, none16 = ops.linear_layernorm(x[300:437].contiguous(), w, b, gam, bet, res[300:437].clone(), 1e-12,
                                        workspace=ws, want_h16=False)
    assert none16 is None
    assert torch.equal(part, outs[700][300:437])
    ops.device_status(0)


def test_linear_layernorm_rejects(cuda_dev):
    from fastembed_b200 import ops
    from fastembed_b200.capi import FeError
    x, w, b, res, gam, bet = _linear_ln_inputs(64, 640, 64, 1, cuda_dev)
    with pytest.raises(FeError):  # n = 640 is not a supported row width
        ops.linear_layernorm(x, w, b, gam, bet, res, 1e-12)
    x, w, b, res, gam, bet = _linear_ln_inputs(64, 512, 64, 1, cuda_dev)
    small = torch.zeros(16, dtype=torch.uint8, device=cuda_dev)
    with pytest.raises(FeError):  # workspace too small
        ops.linear_layernorm(x, w, b, gam, bet, res, 1e-12, workspace=small)


# (m, n, k): Qwen3-0.6B's o_proj and down_proj (one launch), a single column tile, and the
# two-launch form for k < 2048
LINEAR_RMS_SHAPES = [(700, 1024, 2048), (1500, 1024, 3072), (130, 256, 2048), (333, 1024, 1024)]


@pytest.mark.parametrize("pair", ["1", "0"])
@pytest.mark.parametrize("m,n,k", LINEAR_RMS_SHAPES)
def test_linear_rmsnorm(cuda_dev, monkeypatch, m, n, k, pair):
    """Pre-norm: h32 <- (x W^T + b) + h32 stays un-normalised, h16 <- bf16(RMSNorm(h32) * w)."""
    from fastembed_b200 import ops
    monkeypatch.setenv("FE_LINEAR_PAIR", pair)
    x, w, b, res, gam, _ = _linear_ln_inputs(m, n, k, 3 * m + n + k, cuda_dev)
    y = (x.float() @ w.float().T + b) + res
    ref16 = _rms_ref(y, gam, 1e-6, False)
    ws = ops.linear_layernorm_workspace(m, n, cuda_dev)
    for _ in range(2):  # the second call reuses the workspace (epoch-tagged statistics)
        h32, h16 = ops.linear_rmsnorm(x, w, b, gam, res.clone(), 1e-6, workspace=ws)
        torch.cuda.synchronize()
        assert float((h32 - y).abs().max()) < 1e-3
        err = (h16.float() - ref16).abs()
        assert bool((err <= ref16.abs() * 2.0 ** -7 + 1e-4).all()), float(err.max())
    h32n, none16 = ops.linear_rmsnorm(x, w, b, gam, res.clone(), 1e-6, workspace=ws, want_h16=False)
    assert none16 is None
    assert torch.equal(h32n, h32)
    ops.device_status(0)


@pytest.mark.parametrize("mode", ["cls", "mean", "last"])
def test_pool_l2_indices(cuda_dev, mode):
    from fastembed_b200 import ops
    g = torch.Generator(device=cuda_dev).manual_seed(9)
    lens = [1, 9, 128, 2]
    D = 768
    h = torch.randn(sum(lens), D, device=cuda_dev, generator=g)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device=cuda_dev)
    out = ops.pool_l2(h, cu, mode)
    starts = np.concatenate([[0], np.cumsum(lens)[:-1]])
    for b, (s, L) in enumerate(zip(starts, lens)):
        if mode == "cls":
            v = h[s]
        elif mode == "last":
            v = h[s + L - 1]
        else:
            v = h[s:s + L].mean(0)
        v = v / v.norm()
        tol = 0 if mode != "mean" else 1e-5
        assert float((out[b] - v).abs().max()) <= tol + 1e-7


@pytest.mark.parametrize("D", [256, 768, 1024, 1532, 1536, 2048, 4000, 6140, 6144, 770])
def test_pool_mean_l2_shapes(cuda_dev, D):
    """Mean pooling + L2 over the dims of each kernel form (block per sentence with 8 / 4 / 2
    warps, and the warp-per-sentence kernel for dim % 4 != 0, an unaligned base or a dim whose
    partial sums exceed 48 KB), with an
    empty sentence and sentences past 256 tokens; a sentence alone gives its row of the batch
    bit for bit.  Tolerance 1e-5 against a float64 reference of the mean."""
    from fastembed_b200 import ops
    g = torch.Generator(device=cuda_dev).manual_seed(D)
    lens = [3, 0, 300, 1, 64, 257, 17]
    h = torch.randn(sum(lens) + 1, D, device=cuda_dev, generator=g)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device=cuda_dev)
    aligned = h[:-1]
    for hh in (aligned, h.view(-1)[1:sum(lens) * D + 1].view(sum(lens), D)):  # aligned, then 4 bytes off
        out = ops.pool_l2(hh, cu, "mean")
        ref = hh.double()
        starts = np.concatenate([[0], np.cumsum(lens)[:-1]])
        for b, (s0, L) in enumerate(zip(starts, lens)):
            if L == 0:
                assert bool((out[b] == 0).all())
                continue
            v = ref[s0:s0 + L].mean(0)
            v = v / v.norm()
            assert float((out[b].double() - v).abs().max()) <= 1e-5, (D, b)
        for b in ((2, 5) if hh is aligned else ()):  # the slice below is aligned: same kernel only then
            s0, L = int(starts[b]), lens[b]
            one = ops.pool_l2(hh[s0:s0 + L].contiguous(), torch.tensor([0, L], dtype=torch.int32, device=cuda_dev),
                              "mean")
            assert torch.equal(one[0], out[b])


# ------------------------------------------------------------ fp32 op API
def test_fp32_ops_match_oracle(cuda_dev, oracle_lib):
    from fastembed_b200 import ops
    O = oracle_lib
    rng = np.random.default_rng(0)
    for (m, n, k) in [(2, 2, 2), (4, 5, 6), (16, 16, 16), (1, 1, 1), (100, 200, 300), (65, 130, 70)]:
        a = rng.uniform(-1, 1, m * n).astype(np.float32)
        b = rng.uniform(-1, 1, n * k).astype(np.float32)
        ta, tb = torch.tensor(a, device=cuda_dev), torch.tensor(b, device=cuda_dev)
        # the CPU ops' dot-product order is reproduced exactly
        assert np.array_equal(ops.sgemm_nn(ta, tb, m, n, k).cpu().numpy(), O.matmul_nn(a, b, m, n, k))
        assert np.array_equal(ops.sgemm_nt(ta, tb, m, n, k).cpu().numpy(), O.matmul_nt(a, b, m, n, k))
    x = rng.uniform(-4, 4, 100000).astype(np.float32)
    tx = torch.tensor(x, device=cuda_dev)
    for name in ("gelu", "relu", "swish"):
        assert np.abs(ops.unary(name, tx).cpu().numpy() - O.unary(name, x)).max() < 1e-6
    for D in (16, 1024, 3000):
        xs = rng.uniform(-1, 1, 10 * D).astype(np.float32)
        gm = rng.uniform(-1, 1, D).astype(np.float32)
        bt = rng.uniform(-1, 1, D).astype(np.float32)
        t = lambda v: torch.tensor(v, device=cuda_dev)
        for eps in (1e-5, 1e-10):
            assert np.abs(ops.layer_norm_f32(t(xs), t(gm), t(bt), D, eps).cpu().numpy()
                          - O.layer_norm(xs, gm, bt, D, eps)).max() < 1e-5
        assert np.abs(ops.rms_norm_f32(t(xs), t(gm), D, 1e-6).cpu().numpy() - O.rms_norm(xs, gm, D, 1e-6)).max() < 1e-5
        assert np.abs(ops.softmax_rows_f32(t(xs), D).cpu().numpy() - O.softmax_rows(xs, D)).max() < 1e-6


def test_fp32_mha_matches_oracle_reference_inputs(cuda_dev, oracle_lib):
    """tests/attention_ops_test.cpp's cases: every tensor is a fresh mt19937(42)
    U(-1,1) stream, 1e-3 absolute."""
    from fastembed_b200 import ops
    O = oracle_lib
    for (L, D, H) in [(10, 64, 4), (10, 128, 8), (10, 512, 16), (10, 1024, 16), (77, 256, 4)]:
        x = O.uniform_mt19937(L * D)
        w = O.uniform_mt19937(D * D)
        b = O.uniform_mt19937(D)
        ref = O.mha(x, w, w, w, b, b, b, H, D)
        t = lambda v: torch.tensor(v, device=cuda_dev)
        got = ops.mha_f32(t(x), t(w), t(w), t(w), t(b), t(b), t(b), H, D).cpu().numpy()
        assert np.abs(got - ref).max() < 1e-3


# ------------------------------------ RMSNorm / RoPE / gated-MLP encoders (Qwen3, Gemma3)
def _interleave32(gate, up):
    """Gate / up weights -> the gated epilogue's layout: 32 gate rows, 32 up rows, ..."""
    F, K = gate.shape
    return torch.stack([gate.view(F // 32, 32, K), up.view(F // 32, 32, K)], 1).reshape(2 * F, K).contiguous()


@pytest.mark.parametrize("pair", ["1", "0"])
@pytest.mark.parametrize("m,F,k", [(600, 3072, 1024), (77, 1152, 768), (1000, 128, 64)])
@pytest.mark.parametrize("epi", ["swiglu", "geglu"])
def test_linear_gated(cuda_dev, monkeypatch, m, F, k, epi, pair):
    from fastembed_b200 import ops
    monkeypatch.setenv("FE_LINEAR_PAIR", pair)
    g = torch.Generator(device=cuda_dev).manual_seed(m + F + k)
    x = torch.randn(m, k, device=cuda_dev, generator=g).to(torch.bfloat16)
    wg = (torch.randn(F, k, device=cuda_dev, generator=g) / math.sqrt(k)).to(torch.bfloat16)
    wu = (torch.randn(F, k, device=cuda_dev, generator=g) / math.sqrt(k)).to(torch.bfloat16)
    y = ops.linear_bf16(x, _interleave32(wg, wu), None, None, epi, "bf16")
    a = x.float() @ wg.float().T
    act = torch.nn.functional.silu(a) if epi == "swiglu" else torch.nn.functional.gelu(a, approximate="tanh")
    ref = act * (x.float() @ wu.float().T)
    torch.cuda.synchronize()
    assert y.shape == (m, F)
    assert _rel_err(y, ref) < 1e-2  # bf16 output rounding and the fast exp / tanh
    ops.device_status(0)


def _rms_ref(x, w, eps, one_plus):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * ((1 + w) if one_plus else w)


@pytest.mark.parametrize("D,one_plus", [(1024, False), (768, True), (256, True)])
def test_rms_rows_and_sandwich(cuda_dev, D, one_plus):
    from fastembed_b200 import ops
    g = torch.Generator(device=cuda_dev).manual_seed(D)
    x = torch.randn(517, D, device=cuda_dev, generator=g) * 3 + 0.5
    w = torch.randn(D, device=cuda_dev, generator=g) * 0.2 + (0 if one_plus else 1)
    o32, o16 = ops.rms_norm_rows(x, w, 1e-6, one_plus)
    ref = _rms_ref(x, w, 1e-6, one_plus)
    assert float((o32 - ref).abs().max()) < 1e-4
    assert torch.equal(o16, o32.to(torch.bfloat16))
    y = torch.randn(517, D, device=cuda_dev, generator=g) * 5
    h = torch.randn(517, D, device=cuda_dev, generator=g)
    w2 = torch.randn(D, device=cuda_dev, generator=g) * 0.2
    h_ref = h + _rms_ref(y, w, 1e-6, one_plus)
    s32, s16 = ops.rms_sandwich(y, w, h, w2, 1e-6, one_plus)
    assert float((h - h_ref).abs().max()) < 1e-4
    assert float((s32 - _rms_ref(h_ref, w2, 1e-6, one_plus)).abs().max()) < 1e-4
    assert torch.equal(s16, s32.to(torch.bfloat16))
    # y in bf16 (fe_rms_sandwich_bf16): the same step on the widened values
    y16 = y.to(torch.bfloat16)
    h2 = torch.randn(517, D, device=cuda_dev, generator=g)
    h2_ref = h2 + _rms_ref(y16.float(), w, 1e-6, one_plus)
    t32, t16 = ops.rms_sandwich(y16, w, h2, w2, 1e-6, one_plus)
    assert float((h2 - h2_ref).abs().max()) < 1e-4
    assert float((t32 - _rms_ref(h2_ref, w2, 1e-6, one_plus)).abs().max()) < 1e-4
    assert torch.equal(t16, t32.to(torch.bfloat16))


def _rope_ref(x, pos, theta):
    hd = x.shape[-1]
    inv = 1.0 / (theta ** (torch.arange(0, hd, 2, device=x.device).float() / hd))
    ang = pos[:, None].float() * inv[None]
    cos, sin = torch.cat([ang.cos(), ang.cos()], -1), torch.cat([ang.sin(), ang.sin()], -1)
    rot = torch.cat([-x[..., hd // 2:], x[..., :hd // 2]], -1)
    return x * cos[:, None] + rot * sin[:, None]


@pytest.mark.parametrize("hd,hq,hkv,theta,one_plus", [(128, 16, 8, 1e6, False), (256, 3, 1, 1e4, True)])
def test_qk_norm_rope(cuda_dev, hd, hq, hkv, theta, one_plus):
    from fastembed_b200 import ops
    g = torch.Generator(device=cuda_dev).manual_seed(hd + hq)
    lens = [1, 130, 7, 600]
    T = sum(lens)
    qkv = (torch.randn(T, (hq + 2 * hkv) * hd, device=cuda_dev, generator=g) * 2).to(torch.bfloat16)
    qw = torch.randn(hd, device=cuda_dev, generator=g) * 0.3 + (0 if one_plus else 1)
    kw = torch.randn(hd, device=cuda_dev, generator=g) * 0.3 + (0 if one_plus else 1)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device=cuda_dev)
    pos = torch.cat([torch.arange(L, device=cuda_dev) for L in lens])
    src = qkv.float()
    q = src[:, :hq * hd].view(T, hq, hd)
    k = src[:, hq * hd:(hq + hkv) * hd].view(T, hkv, hd)
    q_ref = _rope_ref(_rms_ref(q, qw, 1e-6, one_plus), pos, theta).reshape(T, -1)
    k_ref = _rope_ref(_rms_ref(k, kw, 1e-6, one_plus), pos, theta).reshape(T, -1)
    out = ops.qk_norm_rope(qkv.clone(), cu, hq, hkv, hd, qw, kw, 1e-6, theta, one_plus).float()
    torch.cuda.synchronize()
    scale = float(max(q_ref.abs().max(), k_ref.abs().max()))
    assert float((out[:, :hq * hd] - q_ref).abs().max()) < 1e-2 * scale  # bf16 output
    assert float((out[:, hq * hd:(hq + hkv) * hd] - k_ref).abs().max()) < 1e-2 * scale
    assert torch.equal(out[:, (hq + hkv) * hd:], src[:, (hq + hkv) * hd:])  # V untouched
    ops.device_status(0)


def test_embed_scale_exact(cuda_dev):
    from fastembed_b200 import ops
    g = torch.Generator(device=cuda_dev).manual_seed(9)
    word = torch.randn(5000, 768, device=cuda_dev, generator=g)
    ids = torch.randint(0, 5000, (1234,), device=cuda_dev, generator=g, dtype=torch.int32)
    h = ops.embed_scale(ids, word, 27.712812)
    assert torch.equal(h, word[ids.long()] * torch.tensor(27.712812, device=cuda_dev))


@pytest.mark.parametrize("pair", [True, False])
@pytest.mark.parametrize("hd,hq,hkv,theta,one_plus", [(128, 16, 8, 1e6, False), (128, 4, 2, 1e6, False),
                                                       (256, 3, 1, 1e4, True), (256, 3, 1, 1e6, True)])
def test_linear_qk_norm_rope(cuda_dev, monkeypatch, pair, hd, hq, hkv, theta, one_plus):
    """The QKV projection with the q/k RMSNorm and RoPE in its epilogue against a torch
    fp32 reference of the same steps (fp32 product of the bf16 inputs, per-head RMSNorm,
    rotate-half RoPE); lengths cover one token, tile edges (128 / 129 rows) and a long
    sentence; the 2-CTA kernel (m >= 512) and the 1-CTA kernel (FE_LINEAR_PAIR=0)."""
    from fastembed_b200 import ops
    if not pair:
        monkeypatch.setenv("FE_LINEAR_PAIR", "0")
    g = torch.Generator(device=cuda_dev).manual_seed(hd + hq + int(pair))
    lens = [1, 128, 129, 7, 600]
    T = sum(lens)
    D = 768 if hd == 256 else 1024
    N = (hq + 2 * hkv) * hd
    x = torch.randn(T, D, device=cuda_dev, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, D, device=cuda_dev, generator=g) * 0.05).to(torch.bfloat16)
    qw = torch.randn(hd, device=cuda_dev, generator=g) * 0.3 + (0 if one_plus else 1)
    kw = torch.randn(hd, device=cuda_dev, generator=g) * 0.3 + (0 if one_plus else 1)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device=cuda_dev)
    pos = ops.token_positions(cu)
    assert torch.equal(pos.long(), torch.cat([torch.arange(L, device=cuda_dev) for L in lens]))
    y = ops.linear_qk_norm_rope(x, w, qw, kw, pos, hq, hkv, hd, 1e-6, theta, one_plus).float()
    torch.cuda.synchronize()
    src = x.float() @ w.float().t()
    q = src[:, :hq * hd].view(T, hq, hd)
    k = src[:, hq * hd:(hq + hkv) * hd].view(T, hkv, hd)
    q_ref = _rope_ref(_rms_ref(q, qw, 1e-6, one_plus), pos.long(), theta).reshape(T, -1)
    k_ref = _rope_ref(_rms_ref(k, kw, 1e-6, one_plus), pos.long(), theta).reshape(T, -1)
    v_ref = src[:, (hq + hkv) * hd:]
    scale = float(max(q_ref.abs().max(), k_ref.abs().max()))
    # one bf16 rounding of the result (2^-8 relative) plus the fp32 accumulation order
    assert float((y[:, :hq * hd] - q_ref).abs().max()) < 1e-2 * scale
    assert float((y[:, hq * hd:(hq + hkv) * hd] - k_ref).abs().max()) < 1e-2 * scale
    assert float((y[:, (hq + hkv) * hd:] - v_ref).abs().max()) < 1e-2 * float(v_ref.abs().max())
    ops.device_status(0)


# (m, n, k): Qwen3-0.6B's o_proj (k 2048) and down_proj (k 3072), a k = 4096 shape (the
# one-slab configuration), a short k, 3 and 8 column tiles and a single ragged row tile
DEFERRED_SHAPES = [(700, 1024, 2048), (1500, 1024, 3072), (333, 1024, 4096), (600, 1024, 1024), (4097, 768, 2048),
                   (130, 2048, 2048), (1, 256, 512)]


@pytest.mark.parametrize("m,n,k", DEFERRED_SHAPES)
def test_linear_rmsnorm_deferred(cuda_dev, m, n, k):
    """Pre-norm step with the RMSNorm deferred: h32 <- (x W^T + b) + h32, h16 <- bf16(h32 * w)
    and the row sums of h32^2 per 256-column part, against fp32 torch; twice on the same
    buffers (the sums are overwritten, not accumulated)."""
    from fastembed_b200 import capi, ops
    x, w, b, res, gam, _ = _linear_ln_inputs(m, n, k, 5 * m + n + k, cuda_dev)
    y = (x.float() @ w.float().T + b) + res
    parts = capi.lib().fe_linear_rmsnorm_deferred_parts(n)
    assert parts == n // 256
    ref_ss = (y * y).view(m, parts, n // parts).sum(-1)
    ref16 = y * gam
    for _ in range(2):
        h32, h16, ss = ops.linear_rmsnorm_deferred(x, w, b, gam, res.clone())
        torch.cuda.synchronize()
        assert float((h32 - y).abs().max()) < 1e-3
        err = (h16.float() - ref16).abs()
        assert bool((err <= ref16.abs() * 2.0 ** -7 + 1e-4).all()), float(err.max())
        assert float(((ss - ref_ss).abs() / ref_ss).max()) < 1e-4
    h32n, none16, ss2 = ops.linear_rmsnorm_deferred(x, w, b, gam, res.clone(), want_h16=False)
    torch.cuda.synchronize()
    assert none16 is None
    assert torch.equal(h32n, h32) and torch.equal(ss2, ss)
    ops.device_status(0)


@pytest.mark.parametrize("epi,m,F,k", [("swiglu", 700, 3072, 1024), ("swiglu", 77, 1152, 768), ("none", 600, 512, 1024),
                                       ("none", 100, 384, 256)])
def test_linear_row_scaled(cuda_dev, monkeypatch, epi, m, F, k):
    """A projection of rows that still need their RMSNorm factor: row i of x W^T is scaled by
    1 / sqrt(sum(row_ss[i]) / k + eps) before the epilogue, against fp32 torch on the
    normalised rows; the 2-CTA and the 1-CTA kernels."""
    from fastembed_b200 import ops
    g = torch.Generator(device=cuda_dev).manual_seed(m + F + k + 1)
    h = torch.randn(m, k, device=cuda_dev, generator=g) * 3 + 0.2
    wn = torch.randn(k, device=cuda_dev, generator=g) * 0.5 + 1
    parts = max(1, k // 256)
    row_ss = (h * h).view(m, parts, k // parts).sum(-1).contiguous()
    x = (h * wn).to(torch.bfloat16)  # the producer's bf16(h * w)
    xn = h * torch.rsqrt((h * h).mean(-1, keepdim=True) + 1e-6) * wn  # the normalised rows
    if epi == "swiglu":
        wg = (torch.randn(F, k, device=cuda_dev, generator=g) / math.sqrt(k)).to(torch.bfloat16)
        wu = (torch.randn(F, k, device=cuda_dev, generator=g) / math.sqrt(k)).to(torch.bfloat16)
        wt, ref = _interleave32(wg, wu), torch.nn.functional.silu(xn @ wg.float().T) * (xn @ wu.float().T)
    else:
        wt = (torch.randn(F, k, device=cuda_dev, generator=g) / math.sqrt(k)).to(torch.bfloat16)
        ref = xn @ wt.float().T
    for pair in ("1", "0"):
        monkeypatch.setenv("FE_LINEAR_PAIR", pair)
        y = ops.linear_row_scaled(x, wt, row_ss, 1e-6, epilogue=epi)
        torch.cuda.synchronize()
        assert _rel_err(y, ref) < 1e-2  # bf16 input and output rounding, fast exp
    ops.device_status(0)


@pytest.mark.parametrize("hd,hq,hkv", [(128, 16, 8), (256, 4, 2)])
def test_linear_qk_norm_rope_scaled(cuda_dev, hd, hq, hkv):
    """The QKV projection with q/k norms and RoPE on rows that still need their RMSNorm
    factor equals (within bf16 rounding) the same projection of the normalised rows."""
    from fastembed_b200 import ops
    g = torch.Generator(device=cuda_dev).manual_seed(hd + hq + 7)
    lens = [1, 128, 129, 7, 600]
    T, D = sum(lens), 1024
    N = (hq + 2 * hkv) * hd
    h = torch.randn(T, D, device=cuda_dev, generator=g) * 2 - 0.3
    wn = torch.randn(D, device=cuda_dev, generator=g) * 0.3 + 1
    row_ss = (h * h).view(T, 4, D // 4).sum(-1).contiguous()
    x = (h * wn).to(torch.bfloat16)
    xn = (h * torch.rsqrt((h * h).mean(-1, keepdim=True) + 1e-6) * wn).to(torch.bfloat16)
    w = (torch.randn(N, D, device=cuda_dev, generator=g) * 0.05).to(torch.bfloat16)
    qw = torch.randn(hd, device=cuda_dev, generator=g) * 0.3 + 1
    kw = torch.randn(hd, device=cuda_dev, generator=g) * 0.3 + 1
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device=cuda_dev)
    pos = ops.token_positions(cu)
    y = ops.linear_qk_norm_rope_scaled(x, w, qw, kw, pos, hq, hkv, hd, 1e-6, 1e6, row_ss).float()
    ref = ops.linear_qk_norm_rope(xn, w, qw, kw, pos, hq, hkv, hd, 1e-6, 1e6).float()
    torch.cuda.synchronize()
    kc = (hq + hkv) * hd
    assert float((y[:, :kc] - ref[:, :kc]).abs().max()) < 2e-2 * float(ref[:, :kc].abs().max())
    assert float((y[:, kc:] - ref[:, kc:]).abs().max()) < 2e-2 * float(ref[:, kc:].abs().max())
    ops.device_status(0)


def test_linear_qk_norm_rope_rejects_unaligned_heads(cuda_dev):
    import ctypes as C
    from fastembed_b200 import capi
    buf = C.c_void_p(256)
    # 3 query heads of 128 columns do not fill whole 256-column tiles
    st = capi.lib().fe_linear_qk_norm_rope_bf16(buf, buf, buf, buf, buf, buf, 16, 64, 3, 1, 128, 0, 1e-6, 1e6, None)
    assert st == 4  # FE_ERR_UNSUPPORTED
