"""Per-kernel parity on a B200, through the C ABI (ctypes -> libtfx_b200.so).

Each kernel is compared with an fp32/fp64 CPU computation on the same
(fp16-rounded, where the kernel consumes fp16) inputs:

* LayerNorm / residual LayerNorm: fp32 statistics, fp16 or fp32 output;
  tolerance = one fp16 ulp of the output (rtol 2**-10) + 1e-5 absolute.
* Tensor-core linear: fp32 accumulation of fp16 products; tolerance
  rtol 2e-3 + atol 2e-3 on fp16 outputs, 1e-4 on fp32 (residual) outputs.
* Attention: fp64 softmax reference on the fp16 q/k/v; the kernel rounds P
  to fp16 before P.V, so tolerance atol 2e-3.
"""

from __future__ import annotations

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def _randn(*shape, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g) * scale


@pytest.mark.parametrize("rows,d", [(1, 128), (777, 128), (513, 1024), (64, 96), (33, 4096),
                                    (40003, 128), (19001, 256)])  # last two: rows per warp > 1
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32])
def test_layer_norm(pkg, dev, rows, d, out_dtype):
    x = _randn(rows, d, seed=rows + d) * 3 + 0.5
    w = _randn(d, seed=1) * 0.2 + 1
    b = _randn(d, seed=2) * 0.1
    ref = torch.nn.functional.layer_norm(x, (d,), w, b, 1e-5)
    got = pkg.ops.layer_norm(x.to(dev), w.to(dev), b.to(dev), 1e-5, out_dtype).float().cpu()
    tol = 2 ** -10 if out_dtype == torch.float16 else 1e-6
    assert torch.allclose(got, ref, rtol=tol, atol=1e-5 + tol), (got - ref).abs().max()


@pytest.mark.parametrize("rows,d", [(300, 128), (100, 1024), (40001, 128)])
@pytest.mark.parametrize("store", [True, False])
def test_residual_layer_norm(pkg, dev, rows, d, store):
    r = _randn(rows, d, seed=3)
    u = _randn(rows, d, seed=4).half()
    w = torch.ones(d)
    b = torch.zeros(d)
    s = r + u.float()
    ref = torch.nn.functional.layer_norm(s, (d,), w, b, 1e-5)
    r_out, n = pkg.ops.fused_residual_layer_norm(
        r.to(dev), u.to(dev), w.to(dev), b.to(dev), 1e-5, torch.float16, store_residual=store
    )
    assert torch.allclose(n.float().cpu(), ref, rtol=2 ** -10, atol=2e-3)
    if store:
        assert torch.allclose(r_out.cpu(), s, atol=1e-6)


GEMM_SHAPES = [
    # (m, n, k): c1/c2/c4 projections, c3/c5 projections, ragged edges
    (512, 384, 128),
    (512, 128, 128),
    (1000, 128, 128),
    (8192, 3072, 1024),
    (1200, 1024, 1024),
    (130, 256, 1024),
    (77, 96, 40),
    (1, 32, 8),
    (40000, 128, 128),
    # deep-K shapes with ragged M and each N-tile width
    (300, 512, 512),
    (1100, 384, 768),
    (2048, 1024, 2048),
    (512, 128, 1024),
    (4096, 1024, 1024),
]


@pytest.mark.parametrize("m,n,k", GEMM_SHAPES)
@pytest.mark.parametrize("epi", ["bias", "gelu", "residual"])
def test_linear(pkg, dev, m, n, k, epi):
    a = _randn(m, k, seed=m + k).half()
    w = (_randn(n, k, seed=n + 7) / math.sqrt(k)).half()
    bias = _randn(n, seed=5) * 0.1
    acc = a.float() @ w.float().T + bias
    if epi == "bias":
        got = pkg.ops.linear(a.to(dev), w.to(dev), bias.to(dev)).float().cpu()
        ref = acc
        tol = 2e-3
    elif epi == "gelu":
        got = pkg.ops.linear_gelu(a.to(dev), w.to(dev), bias.to(dev)).float().cpu()
        ref = torch.nn.functional.gelu(acc, approximate="none")
        tol = 2e-3
    else:
        res = _randn(m, n, seed=9)
        got = pkg.ops.linear_residual(a.to(dev), w.to(dev), bias.to(dev), res.to(dev)).cpu()
        ref = acc + res
        tol = 1e-4
    err = (got - ref).abs()
    bound = tol + tol * ref.abs()
    assert bool((err <= bound).all()), f"max err {err.max():.3g} at {int(err.argmax())}"


def _attn_ref(q, k, v, causal, valid_len=None, key_mask=None):
    """fp64 softmax(QK^T/sqrt(hd)) V on [B, S, H, hd] fp16 inputs; a query
    with no visible key gets a zero row."""
    b, s, h, hd = q.shape
    qd, kd, vd = (t.double().permute(0, 2, 1, 3) for t in (q, k, v))
    sc = (qd @ kd.transpose(-1, -2)) / math.sqrt(hd)
    if causal:
        sc = sc.masked_fill(torch.ones(s, s, dtype=torch.bool).triu(1), float("-inf"))
    if valid_len is not None:
        keymask = torch.arange(s)[None, :] >= valid_len[:, None]
        sc = sc.masked_fill(keymask[:, None, None, :], float("-inf"))
    if key_mask is not None:
        sc = sc.masked_fill(~key_mask[:, None, None, :], float("-inf"))
    p = torch.softmax(sc, dim=-1)
    p = torch.nan_to_num(p, nan=0.0)
    return (p @ vd).permute(0, 2, 1, 3).reshape(b, s, h * hd)


ATTN_CASES = [
    # (batch, seq, heads, hd, causal)
    (2, 128, 4, 32, True),
    (2, 128, 16, 8, True),
    (1, 128, 4, 256, True),
    (1, 300, 16, 64, True),
    (3, 37, 4, 32, True),
    (2, 1, 4, 32, True),
    (1, 200, 2, 128, True),
    (2, 70, 8, 16, True),
    (2, 100, 4, 32, False),
    (1, 64, 2, 256, False),
    # head_dim 64/128 run on the tcgen05 kernel: two query tiles per CTA, a
    # ragged last query block, several KV tiles, non-causal.
    (2, 384, 2, 64, True),
    (2, 257, 4, 64, False),
    (1, 513, 2, 128, False),
    (3, 129, 2, 128, True),
    # head_dim 8/16/32 with heads filling 64-column blocks run the tcgen05
    # multi-head kernel: many KV tiles (stage ring wraps), ragged blocks,
    # non-causal, several head blocks per sequence.
    (2, 1024, 4, 32, True),
    (1, 700, 8, 16, False),
    (2, 400, 16, 8, True),
    (1, 385, 16, 8, False),
    (2, 129, 8, 32, True),
    # d_model 32 (official shape 7) stays on the mma.sync kernel
    (2, 128, 4, 8, True),
]


@pytest.mark.parametrize("b,s,h,hd,causal", ATTN_CASES)
def test_attention(pkg, dev, b, s, h, hd, causal):
    qkv = _randn(b, s, 3, h, hd, seed=b * 1000 + s + hd).half()
    q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
    ref = _attn_ref(q, k, v, causal)
    g = qkv.to(dev)
    got = pkg.ops.attention(g[:, :, 0], g[:, :, 1], g[:, :, 2], is_causal=causal)
    err = (got.double().cpu() - ref).abs().max().item()
    assert err < 2e-3, err


@pytest.mark.parametrize("s,hd", [(128, 32), (300, 64), (300, 128), (300, 8), (260, 16)])
def test_attention_key_padding(pkg, dev, s, hd):
    """Keys at or past valid_len are masked; length 0 gives a zero output."""
    b, h = 4, 64 // hd if hd < 32 else 4
    qkv = _randn(b, s, 3, h, hd, seed=11 + hd).half()
    lengths = torch.tensor([s, 97, 5, 0], dtype=torch.int32)
    ref = _attn_ref(qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2], True, lengths)
    g = qkv.to(dev)
    got = pkg.ops.attention(g[:, :, 0], g[:, :, 1], g[:, :, 2], is_causal=True,
                            valid_lengths=lengths.to(dev))
    err = (got.double().cpu() - ref).abs().max().item()
    assert err < 2e-3, err


VT_CASES = [
    # (batch, seq, heads, hd, causal, lengths or None)
    (2, 384, 4, 64, True, None),
    (1, 261, 2, 64, False, None),
    (3, 300, 2, 128, True, [300, 129, 0]),
    (4, 200, 4, 64, True, [200, 97, 5, 1]),
    # head_dim 256: one query tile per CTA, one K/V stage
    (2, 128, 4, 256, True, None),
    (1, 300, 2, 256, True, [300]),
    (2, 136, 2, 256, False, [136, 57]),
]


@pytest.mark.parametrize("b,s,h,hd,causal,lengths", VT_CASES)
def test_attention_transposed_v_path(pkg, dev, b, s, h, hd, causal, lengths):
    """The forward's path for head_dim 64/128: tfx_transpose_v (exact, zero
    padded to a multiple of 8 keys) then tfx_attention_vt."""
    lib = pkg._lib.load()
    qkv = _randn(b, s, 3, h, hd, seed=s + hd + b).half()
    vl = None if lengths is None else torch.tensor(lengths, dtype=torch.int32)
    ref = _attn_ref(qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2], causal, vl)
    g = qkv.to(dev)
    ld_vt = lib.tfx_attention_vt_ld(s)
    assert ld_vt == (s + 7) // 8 * 8
    vt = torch.full((b, h * hd, ld_vt), float("nan"), dtype=torch.float16, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    base = g.data_ptr()
    row = 3 * h * hd
    pkg._lib.check(lib.tfx_transpose_v(base + 2 * h * hd * 2, row, vt.data_ptr(), b, s, h * hd,
                                       stream), "tfx_transpose_v")
    torch.cuda.synchronize()
    want = g[:, :, 2].reshape(b, s, h * hd).transpose(1, 2)
    assert torch.equal(vt[:, :, :s], want)
    assert bool((vt[:, :, s:] == 0).all())
    out = torch.empty(b, s, h * hd, dtype=torch.float16, device=dev)
    vl_dev = None if vl is None else vl.to(dev)
    pkg._lib.check(lib.tfx_attention_vt(base, base + h * hd * 2, vt.data_ptr(), row,
                                        out.data_ptr(), h * hd, b, h, s, hd, hd ** -0.5,
                                        int(causal),
                                        None if vl_dev is None else vl_dev.data_ptr(), stream),
                   "tfx_attention_vt")
    torch.cuda.synchronize()
    err = (out.double().cpu() - ref).abs().max().item()
    assert err < 2e-3, err


MASKED_CASES = [
    # (batch, seq, heads, hd, causal): every head_dim, both kernels
    (3, 128, 16, 8, True), (2, 70, 8, 16, False), (3, 200, 4, 32, True),
    (2, 300, 4, 64, False), (2, 257, 2, 128, True), (1, 130, 2, 256, True),
]


@pytest.mark.parametrize("b,s,h,hd,causal", MASKED_CASES)
def test_attention_arbitrary_key_mask(pkg, dev, b, s, h, hd, causal):
    """tfx_attention_masked: random holes in the keys (about 30 %), whole
    masked 128-key tiles and masked first keys (causal queries with no
    visible key get zero rows)."""
    qkv = _randn(b, s, 3, h, hd, seed=7 * s + hd).half()
    g = torch.Generator().manual_seed(s + hd)
    mask = torch.rand(b, s, generator=g) > 0.3
    if s > 140:
        mask[0, :130] = False  # a whole masked 128-key tile
    mask[-1, 0] = False
    ref = _attn_ref(qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2], causal, key_mask=mask)
    gq = qkv.to(dev)
    out = pkg.ops.attention(gq[:, :, 0], gq[:, :, 1], gq[:, :, 2], is_causal=causal,
                            key_mask=mask.to(dev)).cpu()
    err = (out.double() - ref).abs().max().item()
    assert err < 2e-3, err


def test_attention_long_sequence_rows(pkg, dev):
    """A long causal sequence (S=4096, hd=64): spot-check late query rows
    against the blockwise fp64 oracle."""
    from oracle.baseline import blockwise_causal_attention_fp64

    s, h, hd = 4096, 2, 64
    qkv = _randn(1, s, 3, h, hd, seed=21).half()
    g = qkv.to(dev)
    got = pkg.ops.attention(g[:, :, 0], g[:, :, 1], g[:, :, 2], is_causal=True).cpu()
    for head in range(h):
        ref = blockwise_causal_attention_fp64(
            qkv[0, :, 0, head], qkv[0, :, 1, head], qkv[0, :, 2, head], hd ** -0.5
        )
        err = (got[0, :, head * hd:(head + 1) * hd].double() - ref).abs().max().item()
        assert err < 2e-3, (head, err)


def test_no_device_timeout_recorded(pkg, dev):
    torch.cuda.synchronize()
    assert pkg._lib.read_device_error() == 0
