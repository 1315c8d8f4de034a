"""FP32 CPU restatement of the reference's explicit Transformer (the oracle).

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

Every function names the reference lines it restates. The module tree and the
order in which parameters are created follow the reference exactly, because
``torch.manual_seed(seed)`` followed by construction must draw the same
``nn.Linear`` default-initialised weights (U(+-1/sqrt(fan_in))) as the
reference does (torch_transformer_benchmark.py:1724, 1731) and the state_dict
keys must be identical (torch_transformer_benchmark.py:217-220, 273-277,
297-305).
"""

from __future__ import annotations

import hashlib
import math
from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass(frozen=True)
class TransformerConfig:
    """Same fields and validation as torch_transformer_benchmark.py:47-74."""

    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    ffn_dim: int
    num_layers: int
    causal: bool

    def validate(self) -> None:
        for name in ("batch_size", "seq_len", "d_model", "num_heads"):
            if getattr(self, name) <= 0:
                raise ValueError(f"{name} must be positive")
        if self.d_model % self.num_heads != 0:
            raise ValueError(
                f"d_model ({self.d_model}) must be divisible by "
                f"num_heads ({self.num_heads})"
            )
        if self.ffn_dim <= 0:
            raise ValueError("ffn_dim must be positive")
        if self.num_layers <= 0:
            raise ValueError("num_layers must be positive")


class BaselineSelfAttention(nn.Module):
    """torch_transformer_benchmark.py:204-267: separate q/k/v/out projections,
    explicit Q.K^T scaled by head_dim**-0.5, strict-upper-triangle causal
    mask, key-padding mask, softmax in fp32, P.V, output rows of padded
    tokens zeroed."""

    def __init__(self, d_model: int, num_heads: int) -> None:
        super().__init__()
        if d_model % num_heads != 0:
            raise ValueError("d_model must be divisible by num_heads")
        self.d_model = d_model
        self.num_heads = num_heads
        self.head_dim = d_model // num_heads
        self.scale = self.head_dim ** -0.5
        # Creation order q, k, v, out fixes the RNG draws (reference :217-220).
        self.q_proj = nn.Linear(d_model, d_model, bias=True)
        self.k_proj = nn.Linear(d_model, d_model, bias=True)
        self.v_proj = nn.Linear(d_model, d_model, bias=True)
        self.out_proj = nn.Linear(d_model, d_model, bias=True)

    def _heads(self, t: torch.Tensor) -> torch.Tensor:
        b, s, _ = t.shape
        return t.reshape(b, s, self.num_heads, self.head_dim).permute(0, 2, 1, 3)

    def forward(
        self,
        x: torch.Tensor,
        valid_token_mask: Optional[torch.Tensor] = None,
        causal: bool = False,
    ) -> torch.Tensor:
        b, s, _ = x.shape
        q = self._heads(self.q_proj(x))
        k = self._heads(self.k_proj(x))
        v = self._heads(self.v_proj(x))
        scores = (q @ k.transpose(-1, -2)) * self.scale
        if causal:
            future = torch.ones(s, s, dtype=torch.bool, device=x.device).triu(1)
            scores = scores.masked_fill(future, float("-inf"))
        if valid_token_mask is not None:
            scores = scores.masked_fill(
                ~valid_token_mask[:, None, None, :], float("-inf")
            )
        probs = torch.softmax(scores.float(), dim=-1).to(x.dtype)
        ctx = (probs @ v).permute(0, 2, 1, 3).reshape(b, s, self.d_model)
        out = self.out_proj(ctx)
        if valid_token_mask is not None:
            out = out.masked_fill(~valid_token_mask[..., None], 0)
        return out


class BaselineTransformerBlock(nn.Module):
    """torch_transformer_benchmark.py:270-290: pre-norm block with exact
    (erf) GELU; padded rows zeroed after the block."""

    def __init__(self, d_model: int, num_heads: int, ffn_dim: int) -> None:
        super().__init__()
        self.norm1 = nn.LayerNorm(d_model)
        self.attention = BaselineSelfAttention(d_model, num_heads)
        self.norm2 = nn.LayerNorm(d_model)
        self.ffn_in = nn.Linear(d_model, ffn_dim)
        self.ffn_out = nn.Linear(ffn_dim, d_model)

    def forward(self, x, valid_token_mask, causal):
        x = x + self.attention(self.norm1(x), valid_token_mask, causal)
        hidden = F.gelu(self.ffn_in(self.norm2(x)), approximate="none")
        x = x + self.ffn_out(hidden)
        if valid_token_mask is not None:
            x = x.masked_fill(~valid_token_mask[..., None], 0)
        return x


class BaselineTransformer(nn.Module):
    """torch_transformer_benchmark.py:293-317: L blocks then final LayerNorm."""

    def __init__(self, config: TransformerConfig) -> None:
        super().__init__()
        self.config = config
        self.layers = nn.ModuleList(
            BaselineTransformerBlock(config.d_model, config.num_heads, config.ffn_dim)
            for _ in range(config.num_layers)
        )
        self.final_norm = nn.LayerNorm(config.d_model)

    def forward(self, x, valid_token_mask=None):
        for layer in self.layers:
            x = layer(x, valid_token_mask, self.config.causal)
        x = self.final_norm(x)
        if valid_token_mask is not None:
            x = x.masked_fill(~valid_token_mask[..., None], 0)
        return x


def make_baseline(config: TransformerConfig, seed: int) -> BaselineTransformer:
    """Seeded construction as in torch_transformer_benchmark.py:1724, 1731 and
    streamed_shape14.py:78-83 (``torch.manual_seed`` then the constructor)."""
    torch.manual_seed(seed)
    return BaselineTransformer(config).eval()


def state_dict_checksum(module: nn.Module) -> str:
    """SHA-256 over the state_dict's keys and fp32 bytes, in key order."""
    digest = hashlib.sha256()
    for key, value in module.state_dict().items():
        digest.update(key.encode())
        digest.update(value.detach().float().contiguous().numpy().tobytes())
    return digest.hexdigest()


def generate_random_case(
    config: TransformerConfig,
    seed: int,
    padding_ratio: float = 0.0,
    input_scale: float = 1.0,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """torch_transformer_benchmark.py:1182-1220 on a CPU generator.

    x ~ N(0,1)*input_scale of shape [B,S,D]; with padding, each sequence gets
    a prefix-valid length drawn uniformly from [round(S*(1-ratio)), S] and the
    padded rows of x are zeroed. The reference draws on the target device;
    CPU and CUDA generators produce different streams, so every caller of this
    oracle draws on the CPU and then moves the tensors.
    """
    gen = torch.Generator(device="cpu")
    gen.manual_seed(seed)
    x = torch.randn(
        config.batch_size, config.seq_len, config.d_model, generator=gen
    ) * input_scale
    if padding_ratio <= 0:
        return x, torch.ones(config.batch_size, config.seq_len, dtype=torch.bool)
    min_valid = max(1, int(round(config.seq_len * (1.0 - padding_ratio))))
    lengths = torch.randint(
        min_valid, config.seq_len + 1, (config.batch_size,), generator=gen
    )
    mask = torch.arange(config.seq_len)[None, :] < lengths[:, None]
    return x.masked_fill(~mask[..., None], 0), mask


@dataclass
class AccuracyResult:
    passed: bool
    total_elements: int
    failed_elements: int
    max_abs_error: float
    max_relative_error: float
    mean_abs_error: float
    failed_feature_dims: List[int]
    worst_index: Tuple[int, ...]
    reference_at_worst: float
    optimized_at_worst: float


def compare_outputs(
    reference: torch.Tensor,
    optimized: torch.Tensor,
    rtol: float = 0.02,
    atol: float = 0.002,
) -> AccuracyResult:
    """The elementwise OR rule of torch_transformer_benchmark.py:1237-1304.

    An element passes when both values are finite and
    ``|opt-ref| <= atol`` OR ``|opt-ref| <= rtol*|ref|`` (deliberately not
    torch.isclose's ``atol + rtol*|ref|``). The verdict is
    ``failed_elements == 0``.
    """
    if reference.shape != optimized.shape:
        raise AssertionError(
            f"shape mismatch: baseline={tuple(reference.shape)}, "
            f"optimized={tuple(optimized.shape)}"
        )
    ref = reference.detach().float().cpu()
    opt = optimized.detach().float().cpu()
    err = (opt - ref).abs()
    ok = torch.isfinite(ref) & torch.isfinite(opt) & (
        (err <= atol) | (err <= rtol * ref.abs())
    )
    failed = ~ok
    n_failed = int(failed.sum())
    flat = int(err.reshape(-1).argmax()) if err.numel() else 0
    worst = tuple(int(i) for i in torch.unravel_index(torch.tensor(flat), ref.shape)) if err.numel() else ()
    if ref.ndim >= 2:
        dims = torch.nonzero(failed.any(dim=tuple(range(ref.ndim - 1)))).flatten().tolist()
    else:
        dims = torch.nonzero(failed).flatten().tolist()
    rel = err / ref.abs().clamp_min(1e-12)
    return AccuracyResult(
        passed=n_failed == 0,
        total_elements=ref.numel(),
        failed_elements=n_failed,
        max_abs_error=float(err.max()) if err.numel() else 0.0,
        max_relative_error=float(rel.max()) if err.numel() else 0.0,
        mean_abs_error=float(err.mean()) if err.numel() else 0.0,
        failed_feature_dims=dims,
        worst_index=worst,
        reference_at_worst=float(ref[worst]) if err.numel() else 0.0,
        optimized_at_worst=float(opt[worst]) if err.numel() else 0.0,
    )


def blockwise_causal_attention_fp64(q, k, v, scale, block=1024):
    """Causal softmax(Q.K^T*scale).V in float64 over key blocks.

    Used only for long-sequence spot checks of the attention kernel, where the
    explicit S x S score matrix of the reference would not fit. q, k, v are
    [S, hd] for one (batch, head); returns [S, hd] float64. Mathematically the
    same softmax as torch_transformer_benchmark.py:237-253.
    """
    q = q.double()
    k = k.double()
    v = v.double()
    s = q.shape[0]
    out = torch.empty_like(q)
    for q0 in range(0, s, block):
        q1 = min(s, q0 + block)
        sc = (q[q0:q1] @ k[:q1].T) * scale
        rows = torch.arange(q0, q1)[:, None]
        cols = torch.arange(q1)[None, :]
        sc = sc.masked_fill(cols > rows, -math.inf)
        p = torch.softmax(sc, dim=-1)
        out[q0:q1] = p @ v[:q1]
    return out


def causal_attention_rows_fp64(q, k, v, rows, scale):
    """Selected query rows of causal softmax(Q.K^T*scale).V in float64.

    q, k, v are [S, hd] for one (batch, head); ``rows`` lists query positions;
    row r attends keys 0..r (torch_transformer_benchmark.py:237-253). Returns
    [len(rows), hd] float64. For spot checks of late rows of very long
    sequences, where even the blockwise full computation is too slow.
    """
    rows = torch.as_tensor(rows, dtype=torch.long)
    hi = int(rows.max()) + 1
    sc = (q[rows].double() @ k[:hi].double().T) * scale
    sc = sc.masked_fill(torch.arange(hi)[None, :] > rows[:, None], -math.inf)
    return torch.softmax(sc, dim=-1) @ v[:hi].double()
