"""Tensor-level wrappers over the C ABI, mirroring the reference's op layer.

Same names, argument meaning and error behaviour as the reference's Python
kernels where one exists (``layer_norm`` / ``fused_residual_layer_norm`` of
triton_fused_norm.py:140-215), plus the ops the reference took from PyTorch
(``F.linear``, ``torch._addmm_activation``, ``F.scaled_dot_product_attention``;
torch_transformer_benchmark.py:741, 767-818, 875-896). All work runs on the
current CUDA stream through ``lib/libtfx_b200.so``; there is no fallback.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

from . import _lib


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(t: torch.Tensor, what: str) -> None:
    if t.device.type != "cuda":
        raise ValueError(f"{what} requires CUDA tensors")


def _dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float16:
        return _lib.TFX_DTYPE_F16
    if dtype == torch.float32:
        return _lib.TFX_DTYPE_F32
    raise ValueError(f"output dtype must be float16 or float32, got {dtype}")


def layer_norm(
    inputs: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor,
    eps: float,
    output_dtype: torch.dtype,
    apply_affine: bool = True,
) -> torch.Tensor:
    """LayerNorm whose output is stored directly in the next GEMM's dtype.

    Mirrors triton_fused_norm.py:140-170: fp32 ``inputs`` [..., D], fp32
    statistics, output in ``output_dtype`` (float16 or float32).
    """
    _require_cuda(inputs, "the fused LayerNorm kernel")
    n_cols = inputs.shape[-1]
    if n_cols != weight.numel() or weight.shape != bias.shape:
        raise ValueError("LayerNorm parameters do not match the input width")
    if inputs.dtype != torch.float32:
        raise ValueError("layer_norm expects float32 inputs")
    x = inputs.contiguous()
    w = weight.detach().float().contiguous()
    b = bias.detach().float().contiguous()
    out = torch.empty(x.shape, device=x.device, dtype=output_dtype)
    rows = x.numel() // n_cols
    _lib.check(
        _lib.load().tfx_layer_norm(
            x.data_ptr(), w.data_ptr(), b.data_ptr(), out.data_ptr(), _dtype_code(output_dtype),
            rows, n_cols, float(eps), int(apply_affine), _stream(x.device),
        ),
        "tfx_layer_norm",
    )
    return out


def fused_residual_layer_norm(
    residual: torch.Tensor,
    update: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor,
    eps: float,
    norm_dtype: torch.dtype,
    store_residual: bool = True,
    apply_affine: bool = True,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Return the fp32 residual sum and the normalised output in ``norm_dtype``.

    Mirrors triton_fused_norm.py:173-215 (``store_residual=False`` returns the
    input residual object, as the reference does).
    """
    _require_cuda(residual, "the fused LayerNorm kernel")
    if residual.shape != update.shape:
        raise ValueError("residual and update must have identical shapes")
    if residual.shape[-1] != weight.numel() or weight.shape != bias.shape:
        raise ValueError("LayerNorm parameters do not match the input width")
    if residual.dtype != torch.float32:
        raise ValueError("residual must be float32")
    n_cols = residual.shape[-1]
    r = residual.contiguous()
    u = update.to(torch.float16).contiguous()
    w = weight.detach().float().contiguous()
    b = bias.detach().float().contiguous()
    r_out = torch.empty_like(r) if store_residual else r
    out = torch.empty(r.shape, device=r.device, dtype=norm_dtype)
    rows = r.numel() // n_cols
    _lib.check(
        _lib.load().tfx_residual_layer_norm(
            r.data_ptr(), u.data_ptr(), w.data_ptr(), b.data_ptr(),
            r_out.data_ptr() if store_residual else None, out.data_ptr(),
            _dtype_code(norm_dtype), rows, n_cols, float(eps), int(apply_affine),
            _stream(r.device),
        ),
        "tfx_residual_layer_norm",
    )
    return r_out, out


def _linear(x, weight, bias, residual, epilogue, out_dtype, what):
    _require_cuda(x, what)
    if weight.ndim != 2 or bias.ndim != 1:
        raise ValueError("weight must be 2-D and bias must be 1-D")
    n, k = weight.shape
    if x.shape[-1] != k or bias.numel() != n:
        raise ValueError("weight does not match the input")
    lead = x.shape[:-1]
    a = x.reshape(-1, k).to(torch.float16).contiguous()
    w = weight.detach().to(torch.float16).contiguous()
    b = bias.detach().float().contiguous()
    m = a.shape[0]
    res_ptr = None
    if residual is not None:
        if residual.shape[:-1] != lead or residual.shape[-1] != n:
            raise ValueError("residual does not match the output shape")
        residual = residual.float().contiguous()
        res_ptr = residual.data_ptr()
    out = torch.empty((m, n), device=x.device, dtype=out_dtype)
    _lib.check(
        _lib.load().tfx_linear(
            a.data_ptr(), w.data_ptr(), b.data_ptr(), res_ptr, out.data_ptr(), m, n, k,
            epilogue, _stream(x.device),
        ),
        what,
    )
    return out.view(*lead, n)


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """fp16 tensor-core ``F.linear(x, weight, bias)`` (fp32 accumulate, fp16 out).

    ``weight`` is nn.Linear's [out, in]. Replaces the cached-fp16 ``F.linear``
    of torch_transformer_benchmark.py:675-685 / :741.
    """
    return _linear(x, weight, bias, None, _lib.TFX_EPI_BIAS, torch.float16, "tfx_linear")


def linear_gelu(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """``gelu_erf(x @ weight.T + bias)`` in one tensor-core kernel, fp16 out.

    Replaces ``triton_ffn_gelu`` (triton_fused_ffn.py:224-261), which takes the
    weight transposed ([K, N]) and applies the tanh GELU; this takes
    nn.Linear's [N, K] weight and applies the exact erf GELU the baseline
    uses (torch_transformer_benchmark.py:286).
    """
    return _linear(x, weight, bias, None, _lib.TFX_EPI_BIAS_GELU, torch.float16,
                   "tfx_linear(gelu)")


def linear_residual(
    x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, residual: torch.Tensor
) -> torch.Tensor:
    """``residual + x @ weight.T + bias`` with the add done in fp32 (fp32 out)."""
    return _linear(x, weight, bias, residual, _lib.TFX_EPI_BIAS_RESIDUAL, torch.float32,
                   "tfx_linear(residual)")


def attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    is_causal: bool = True,
    scale: Optional[float] = None,
    valid_lengths: Optional[torch.Tensor] = None,
    key_mask: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Flash attention on [B, S, H, hd] views (e.g. slices of the packed QKV).

    Key padding: ``valid_lengths`` (int [B], keys >= length masked) or
    ``key_mask`` (bool [B, S], False = masked key, any pattern), not both.

    q, k, v: fp16 tensors indexed (b, s, h, e) whose last two dims are
    contiguous and which share the same row stride (the packed projection's
    [B, S, 3, H, hd] layout qualifies). Returns ctx [B, S, H*hd] fp16.
    Replaces F.scaled_dot_product_attention in
    torch_transformer_benchmark.py:767-808 (which takes [B, H, S, hd] views of
    the same memory).
    """
    _require_cuda(q, "tfx_attention")
    if q.dtype != torch.float16 or k.dtype != torch.float16 or v.dtype != torch.float16:
        raise ValueError("q, k and v must be float16")
    if q.ndim != 4 or q.shape != k.shape or q.shape != v.shape:
        raise ValueError("q, k, v must be [B, S, H, hd] with identical shapes")
    bsz, seq, heads, hd = q.shape
    for t in (q, k, v):
        if t.stride(3) != 1 or t.stride(2) != hd or t.stride(1) != q.stride(1) or \
                t.stride(0) != seq * q.stride(1):
            raise ValueError("q, k, v must share a [B, S, *] row layout with contiguous heads")
    if scale is None:
        scale = hd ** -0.5
    out = torch.empty((bsz, seq, heads * hd), device=q.device, dtype=torch.float16)
    if key_mask is not None:
        if valid_lengths is not None:
            raise ValueError("pass valid_lengths or key_mask, not both")
        if key_mask.shape != (bsz, seq) or key_mask.dtype != torch.bool:
            raise ValueError("key_mask must be a [B, S] bool tensor")
        from .model import key_bitmask

        words = key_bitmask(key_mask.to(q.device))
        _lib.check(
            _lib.load().tfx_attention_masked(
                q.data_ptr(), k.data_ptr(), v.data_ptr(), q.stride(1), out.data_ptr(),
                heads * hd, bsz, heads, seq, hd, float(scale), int(is_causal), words.data_ptr(),
                _stream(q.device),
            ),
            "tfx_attention_masked",
        )
        return out
    vl_ptr = None
    if valid_lengths is not None:
        valid_lengths = valid_lengths.to(device=q.device, dtype=torch.int32).contiguous()
        if valid_lengths.numel() != bsz:
            raise ValueError("valid_lengths must have one entry per batch element")
        vl_ptr = valid_lengths.data_ptr()
    _lib.check(
        _lib.load().tfx_attention(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), q.stride(1), out.data_ptr(), heads * hd,
            bsz, heads, seq, hd, float(scale), int(is_causal), vl_ptr, _stream(q.device),
        ),
        "tfx_attention",
    )
    return out


def math_scale(head_dim: int) -> float:
    """Softmax scale head_dim**-0.5 (torch_transformer_benchmark.py:215)."""
    return 1.0 / math.sqrt(head_dim)
