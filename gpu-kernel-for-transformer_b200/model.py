"""Drop-in module API: ``TransformerConfig``, ``BaselineTransformer`` and
``UserOptimizedTransformer`` with the reference's constructor, parameter
names/layout, toggles and ``forward(x, valid_token_mask)`` contract
(torch_transformer_benchmark.py:47-74, 204-317, 320-1148).

``UserOptimizedTransformer.forward`` makes ONE call into the native runtime
(``tfx_forward`` in lib/libtfx_b200.so), which enqueues every kernel of the
forward on the current stream. UserOptimizedTransformer never computes on the
CPU: a CPU input raises (the reference's CPU fallback,
torch_transformer_benchmark.py:1003-1006, is deliberately not reproduced), as
does a missing library. BaselineTransformer is the explicit eager model, for
any device.
"""

from __future__ import annotations

import ctypes
import warnings
from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib


@dataclass(frozen=True)
class TransformerConfig:
    """torch_transformer_benchmark.py:47-74 (same fields, same validation)."""

    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    ffn_dim: int
    num_layers: int
    causal: bool

    def validate(self) -> None:
        if self.batch_size <= 0:
            raise ValueError("batch_size must be positive")
        if self.seq_len <= 0:
            raise ValueError("seq_len must be positive")
        if self.d_model <= 0:
            raise ValueError("d_model must be positive")
        if self.num_heads <= 0:
            raise ValueError("num_heads must be positive")
        if self.d_model % self.num_heads != 0:
            raise ValueError(
                f"d_model ({self.d_model}) must be divisible by "
                f"num_heads ({self.num_heads})"
            )
        if self.ffn_dim <= 0:
            raise ValueError("ffn_dim must be positive")
        if self.num_layers <= 0:
            raise ValueError("num_layers must be positive")


# The reference's official shape table (torch_transformer_benchmark.py:80-95);
# ids 3, 6, 8, 11 and 14 are the benchmark configs c1..c5.
OFFICIAL_BENCHMARK_SHAPES: Dict[int, TransformerConfig] = {
    1: TransformerConfig(64, 128, 128, 4, 128, 4, True),
    2: TransformerConfig(1, 128, 128, 4, 128, 4, True),
    3: TransformerConfig(4, 128, 128, 4, 128, 4, True),
    4: TransformerConfig(16, 128, 128, 4, 128, 4, True),
    5: TransformerConfig(128, 128, 128, 4, 128, 4, True),
    6: TransformerConfig(10000, 128, 128, 4, 128, 4, True),
    7: TransformerConfig(64, 128, 32, 4, 32, 4, True),
    8: TransformerConfig(64, 128, 1024, 4, 1024, 4, True),
    9: TransformerConfig(64, 128, 128, 1, 128, 4, True),
    10: TransformerConfig(64, 128, 128, 2, 128, 4, True),
    11: TransformerConfig(64, 128, 128, 16, 128, 4, True),
    12: TransformerConfig(64, 32, 128, 4, 128, 4, True),
    13: TransformerConfig(64, 1024, 128, 4, 128, 4, True),
    14: TransformerConfig(32, 100000, 1024, 16, 1024, 2, True),
}


class _SelfAttention(nn.Module):
    """Multi-head self-attention with BaselineSelfAttention's parameter names
    and creation order (torch_transformer_benchmark.py:204-220), and its
    explicit FP32 eager forward (:222-267)."""

    def __init__(self, d_model: int, num_heads: int) -> None:
        super().__init__()
        if d_model % num_heads != 0:
            raise ValueError("d_model must be divisible by num_heads")
        self.d_model = d_model
        self.num_heads = num_heads
        self.head_dim = d_model // num_heads
        self.scale = self.head_dim ** -0.5
        self.q_proj = nn.Linear(d_model, d_model, bias=True)
        self.k_proj = nn.Linear(d_model, d_model, bias=True)
        self.v_proj = nn.Linear(d_model, d_model, bias=True)
        self.out_proj = nn.Linear(d_model, d_model, bias=True)

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None,
                causal: bool = False) -> torch.Tensor:
        b, s, _ = x.shape

        def by_head(t: torch.Tensor) -> torch.Tensor:  # [B, S, D] -> [B, H, S, hd]
            return t.view(b, s, self.num_heads, self.head_dim).transpose(1, 2)

        q, k, v = by_head(self.q_proj(x)), by_head(self.k_proj(x)), by_head(self.v_proj(x))
        scores = torch.matmul(q, k.transpose(-2, -1)) * self.scale
        if causal:
            later = torch.ones(s, s, dtype=torch.bool, device=x.device).triu(1)
            scores = scores.masked_fill(later, float("-inf"))
        if valid_token_mask is not None:  # padded keys, per sequence
            scores = scores.masked_fill(~valid_token_mask[:, None, None, :], float("-inf"))
        weights = torch.softmax(scores.float(), dim=-1).to(x.dtype)
        ctx = torch.matmul(weights, v).transpose(1, 2).reshape(b, s, self.d_model)
        out = self.out_proj(ctx)
        if valid_token_mask is not None:
            out = out.masked_fill(~valid_token_mask[..., None], 0)
        return out


class _Block(nn.Module):
    """Pre-norm block with BaselineTransformerBlock's parameters
    (torch_transformer_benchmark.py:270-277) and forward (:279-290): exact
    (erf) GELU, padded rows zeroed after the block."""

    def __init__(self, d_model: int, num_heads: int, ffn_dim: int) -> None:
        super().__init__()
        self.norm1 = nn.LayerNorm(d_model)
        self.attention = _SelfAttention(d_model, num_heads)
        self.norm2 = nn.LayerNorm(d_model)
        self.ffn_in = nn.Linear(d_model, ffn_dim)
        self.ffn_out = nn.Linear(ffn_dim, d_model)

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor],
                causal: bool) -> torch.Tensor:
        x = x + self.attention(self.norm1(x), valid_token_mask, causal)
        x = x + self.ffn_out(F.gelu(self.ffn_in(self.norm2(x)), approximate="none"))
        if valid_token_mask is not None:
            x = x.masked_fill(~valid_token_mask[..., None], 0)
        return x


class BaselineTransformer(nn.Module):
    """The reference's explicit model (torch_transformer_benchmark.py:293-317).

    Constructing it under ``torch.manual_seed(s)`` draws exactly the weights
    the reference draws, and its state_dict keys are the reference's, so
    ``load_state_dict`` of a reference checkpoint works unchanged. Its forward
    is the plain eager PyTorch computation in the parameters' dtype (FP32 by
    default) on any device: the accuracy baseline the reference's harness
    compares the optimized module against, and the CPU path.
    """

    def __init__(self, config: TransformerConfig) -> None:
        super().__init__()
        self.config = config
        self.layers = nn.ModuleList(
            [
                _Block(config.d_model, config.num_heads, config.ffn_dim)
                for _ in range(config.num_layers)
            ]
        )
        self.final_norm = nn.LayerNorm(config.d_model)

    def forward(self, x: torch.Tensor,
                valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        for layer in self.layers:
            x = layer(x, valid_token_mask, self.config.causal)
        x = self.final_norm(x)
        if valid_token_mask is not None:
            x = x.masked_fill(~valid_token_mask[..., None], 0)
        return x


@dataclass(frozen=True)
class ShapeExecutionPlan:
    """Diagnostic description of the kernels a config runs
    (the reference's per-shape plan, torch_transformer_benchmark.py:98-157)."""

    official_shape_id: Optional[int]
    head_dim: int
    path: str
    gemm_tiles: str
    attention: str

    def describe(self) -> str:
        shape = (
            f"official-{self.official_shape_id}"
            if self.official_shape_id is not None
            else "general"
        )
        return (
            f"{shape}: {self.path}; gemm=tcgen05 {self.gemm_tiles}, "
            f"attention={self.attention} (head_dim {self.head_dim}), norm=fp32 LayerNorm"
        )


def _plan_for(config: TransformerConfig) -> ShapeExecutionPlan:
    """The dispatch the native runtime makes for this config (forward.cu,
    fused_block.cu, attention.cu), as text."""
    ids = {c: i for i, c in OFFICIAL_BENCHMARK_SHAPES.items()}
    d, hd, s = config.d_model, config.d_model // config.num_heads, config.seq_len
    fused = (d == 128 and config.ffn_dim == 128 and 128 % s == 0 and config.num_layers <= 5
             and hd in (8, 16, 32, 64, 128))
    if fused:
        tiles = -(-config.batch_size * s // 128)
        pairs = "one CTA per tile" if hd == 128 else (
            f"a CTA pair per tile (heads split) on GPUs with at least {2 * tiles} SMs "
            "(B200: 148), else one CTA per tile")
        return ShapeExecutionPlan(
            official_shape_id=ids.get(config), head_dim=hd,
            path=f"fused whole-forward kernel, {tiles} tiles of 128 tokens, {pairs}",
            gemm_tiles="128x128 in TMEM", attention="in-kernel tcgen05, S/P/O in TMEM")
    if hd in (64, 128, 256):
        attention = "tcgen05 flash (V transposed)" if hd != 256 else "tcgen05 flash"
    elif (config.num_heads * hd) % 64 == 0 and s > 128:
        attention = "tcgen05 flash, 64-column head blocks per CTA"
    else:
        attention = "mma.sync flash"
    widest = max(t for t in (256, 192, 128, 64, 32) if d % t == 0) if d % 32 == 0 else 0
    return ShapeExecutionPlan(
        official_shape_id=ids.get(config), head_dim=hd, path="per-op kernel chain",
        gemm_tiles=f"128x{min(widest, 256)} persistent", attention=attention)


def key_bitmask(mask: torch.Tensor) -> torch.Tensor:
    """[B, S] bool -> int32 [B, ceil(S/32)]: bit k of word w of row b is
    mask[b, 32*w + k] (the key_mask layout of tfx_forward_masked)."""
    b, s = mask.shape
    words = (s + 31) // 32
    m = torch.zeros(b, words * 32, dtype=torch.int64, device=mask.device)
    m[:, :s] = mask
    weights = torch.ones(32, dtype=torch.int64, device=mask.device) << torch.arange(
        32, dtype=torch.int64, device=mask.device)
    w = (m.view(b, words, 32) * weights).sum(dim=-1)  # in [0, 2^32)
    w = torch.where(w >= 2 ** 31, w - 2 ** 32, w)     # same bits as int32
    return w.to(torch.int32).contiguous()


def _version(t: torch.Tensor) -> Optional[int]:
    try:
        return t._version
    except RuntimeError:  # inference tensors expose no version counter
        return None


class UserOptimizedTransformer(BaselineTransformer):
    """B200 inference module; same API as the reference's
    (torch_transformer_benchmark.py:320-1148)."""

    def __init__(self, config: TransformerConfig) -> None:
        super().__init__(config)
        self._shape_execution_plan = _plan_for(config)
        self._mixed_precision_dtype: Optional[torch.dtype] = torch.float16
        self._kv_cache_enabled = False
        self._kv_cache: Optional[Tuple[torch.Tensor, torch.Tensor]] = None
        self._kv_cache_length = 0
        self._packed = None  # (key, tensors, ctypes structs)
        self._workspace: Dict[torch.device, torch.Tensor] = {}
        self._mask_cache = None
        self._path = _lib.TFX_PATH_AUTO

    # ------------------------------------------------------------ toggles
    @property
    def shape_execution_plan(self) -> ShapeExecutionPlan:
        return self._shape_execution_plan

    def enable_mixed_precision(self, dtype: Optional[torch.dtype] = torch.float16) -> None:
        """torch_transformer_benchmark.py:369-377. Tensor-core operands are
        always fp16: bf16 fails the accuracy rule on these configs, so a bf16
        request is accepted with a warning and runs fp16; None (pure FP32 GPU
        compute) is not provided by this implementation."""
        if dtype not in (None, torch.float16, torch.bfloat16):
            raise ValueError("mixed precision dtype must be float16 or bfloat16")
        if self._kv_cache_length:
            raise RuntimeError("reset the KV cache before changing precision")
        if dtype is None:
            raise NotImplementedError(
                "the B200 path computes tensor-core operands in fp16; there is no FP32 path"
            )
        if dtype == torch.bfloat16:
            warnings.warn("bfloat16 operands exceed the accuracy tolerance; using float16")
        self._mixed_precision_dtype = torch.float16

    def enable_triton_fused_norm(self, enabled: bool = True) -> None:
        """Kept for API compatibility: normalisation is always the fused
        native kernel (there is no unfused fallback)."""
        if not enabled:
            raise NotImplementedError("the native path has no unfused LayerNorm fallback")

    def enable_triton_fused_ffn(self, enabled: bool = True) -> None:
        """Kept for API compatibility: the FFN always runs the native
        tcgen05 GEMM with the fused GELU epilogue."""
        if not enabled:
            raise NotImplementedError("the native path has no unfused FFN fallback")

    def enable_fused_forward(self, enabled: bool = True) -> None:
        """Per-module choice of kernels, like the reference's per-module
        ``enable_triton_fused_*`` toggles (torch_transformer_benchmark.py
        :379-393): True (default) runs the whole forward as one fused kernel
        where it applies (d_model = ffn_dim = 128, seq_len dividing 128),
        False always runs the per-op kernel chain. Only this module changes."""
        self._path = _lib.TFX_PATH_AUTO if enabled else _lib.TFX_PATH_CHAIN
        if self._packed is not None:
            self._packed[3].path = self._path

    def enable_attention_fp16_accumulation(self, enabled: bool = True) -> None:
        """torch_transformer_benchmark.py:395-407: fp16 accumulation is never
        used (every accumulator is fp32), so only False is meaningful."""
        if enabled and self.config.causal:
            raise ValueError(
                "FP16 attention accumulation is disabled for causal models "
                "because it exceeds the accuracy tolerance"
            )

    def enable_kv_cache(self, enabled: bool = True) -> None:
        """Incremental decoding (torch_transformer_benchmark.py:409-415):
        each forward then takes the next chunk of tokens of the same
        sequences, appends its keys/values to per-layer caches of capacity
        ``config.seq_len`` and attends over everything cached so far."""
        if enabled and not self.config.causal:
            raise ValueError("KV caching requires a causal Transformer")
        if enabled and self.training:
            raise RuntimeError("call eval() before enabling the KV cache")
        self._kv_cache_enabled = enabled
        self.reset_kv_cache()

    def reset_kv_cache(self) -> None:
        """Clear cached keys and values before starting a new sequence
        (torch_transformer_benchmark.py:417-420)."""
        self._kv_cache = None
        self._kv_cache_length = 0

    @property
    def kv_cache_length(self) -> int:
        return self._kv_cache_length

    def _kv_cache_for(self, x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """fp16 [layers, B, capacity, D] key and value caches, allocated on
        first use (torch_transformer_benchmark.py:426-462)."""
        cfg = self.config
        shape = (cfg.num_layers, x.shape[0], cfg.seq_len, cfg.d_model)
        c = self._kv_cache
        if c is None:
            c = (torch.empty(shape, dtype=torch.float16, device=x.device),
                 torch.empty(shape, dtype=torch.float16, device=x.device))
            self._kv_cache = c
        elif c[0].shape != shape or c[0].device != x.device:
            raise RuntimeError(
                "KV cache does not match this input; reset it before changing "
                "batch size, device, or dtype"
            )
        return c

    def _forward_kv(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor]):
        """One incremental step: x holds the next x.shape[1] tokens."""
        if valid_token_mask is not None and not bool(valid_token_mask.all().item()):
            raise ValueError("KV-cached decoding does not support padding")
        batch, new_tokens, _ = x.shape
        start = self._kv_cache_length
        end = start + new_tokens
        if end > self.config.seq_len:
            raise ValueError(f"KV cache capacity exceeded ({end} > {self.config.seq_len})")
        k_cache, v_cache = self._kv_cache_for(x)
        _, _, _, model = self._prepare(x.device)
        lib = _lib.load()
        need = lib.tfx_forward_kv_workspace_bytes(ctypes.byref(model), batch, new_tokens)
        if need < 0:
            _lib.check(_lib.TFX_ERR_INVALID_ARGUMENT, "tfx_forward_kv_workspace_bytes")
        ws = self._workspace.get(x.device)
        if ws is None or ws.numel() < need:
            ws = torch.empty(int(need), dtype=torch.uint8, device=x.device)
            self._workspace[x.device] = ws
        y = torch.empty_like(x)
        stream = torch.cuda.current_stream(x.device).cuda_stream
        _lib.check(
            lib.tfx_forward_kv(
                ctypes.byref(model), x.data_ptr(), y.data_ptr(), batch, new_tokens, start,
                self.config.seq_len, k_cache.data_ptr(), v_cache.data_ptr(), ws.data_ptr(),
                ws.numel(), stream,
            ),
            "tfx_forward_kv",
        )
        self._kv_cache_length = end
        return y

    # ---------------------------------------------------------- packing
    def _param_key(self, device: torch.device) -> Tuple:
        """Identity of the parameters as packed: storage address, version
        counter and dtype of each. Inference tensors expose no version
        counter; for them a content fingerprint (sum and sum of squares of
        all parameters, read back once per forward) stands in, so an
        in-place update inside ``torch.inference_mode()`` still repacks and an
        unchanged model is not re-uploaded on every call. During CUDA graph
        capture (no host reads allowed) the addresses alone decide."""
        key = [device]
        versionless = []
        for p in self.parameters():
            ver = _version(p)
            key.append((p.data_ptr(), ver, p.dtype))
            if ver is None:
                versionless.append(p)
        if versionless:
            if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
                key.append("capturing")
            else:
                with torch.no_grad():
                    flat = torch.cat([p.detach().reshape(-1).double() for p in versionless])
                    fp = torch.stack((flat.sum(), flat.square().sum())).tolist()
                key.append(tuple(fp))
        return tuple(key)

    def _prepare(self, device: torch.device):
        """Pack the weights once per parameter version (the reference's
        version-checked caches, torch_transformer_benchmark.py:524-655):
        fp16 [out, in] GEMM weights (q|k|v stacked), fp32 biases and norms."""
        key = self._param_key(device)
        if self._packed is not None and (
                self._packed[0] == key
                or (key[-1] == "capturing" and self._packed[0][:-1] == key[:-1])):
            return self._packed
        keep = []

        def f32(t):
            t = t.detach().to(device=device, dtype=torch.float32).contiguous()
            keep.append(t)
            return t.data_ptr()

        def f16(t):
            t = t.detach().to(device=device, dtype=torch.float16).contiguous()
            keep.append(t)
            return t.data_ptr()

        layers = (_lib.TfxLayer * self.config.num_layers)()
        for i, blk in enumerate(self.layers):
            att = blk.attention
            L = layers[i]
            L.norm1_weight = f32(blk.norm1.weight)
            L.norm1_bias = f32(blk.norm1.bias)
            L.qkv_weight = f16(torch.cat(
                (att.q_proj.weight, att.k_proj.weight, att.v_proj.weight), dim=0))
            L.qkv_bias = f32(torch.cat((att.q_proj.bias, att.k_proj.bias, att.v_proj.bias)))
            L.out_weight = f16(att.out_proj.weight)
            L.out_bias = f32(att.out_proj.bias)
            L.norm2_weight = f32(blk.norm2.weight)
            L.norm2_bias = f32(blk.norm2.bias)
            L.ffn_in_weight = f16(blk.ffn_in.weight)
            L.ffn_in_bias = f32(blk.ffn_in.bias)
            L.ffn_out_weight = f16(blk.ffn_out.weight)
            L.ffn_out_bias = f32(blk.ffn_out.bias)
        model = _lib.TfxModel()
        model.d_model = self.config.d_model
        model.num_heads = self.config.num_heads
        model.ffn_dim = self.config.ffn_dim
        model.num_layers = self.config.num_layers
        model.causal = int(self.config.causal)
        model.eps = float(self.final_norm.eps)
        model.layers = ctypes.cast(layers, ctypes.POINTER(_lib.TfxLayer))
        model.final_norm_weight = f32(self.final_norm.weight)
        model.final_norm_bias = f32(self.final_norm.bias)
        model.path = self._path
        self._packed = (key, keep, layers, model)
        return self._packed

    def _workspace_for(self, device: torch.device, model, batch: int, seq: int) -> torch.Tensor:
        need = _lib.load().tfx_forward_workspace_bytes(ctypes.byref(model), batch, seq)
        if need < 0:
            _lib.check(_lib.TFX_ERR_INVALID_ARGUMENT, "tfx_forward_workspace_bytes")
        ws = self._workspace.get(device)
        if ws is None or ws.numel() < need:
            ws = torch.empty(int(need), dtype=torch.uint8, device=device)
            self._workspace[device] = ws
        return ws

    # ------------------------------------------------------------- masks
    def _valid_lengths(self, x: torch.Tensor, mask: Optional[torch.Tensor]):
        """The padding mask in the form the kernels take.

        All-True (or None) -> None; a prefix-valid mask (the form the
        reference's generator makes) -> int32 lengths [B]; any other mask ->
        the token bitmask int32 [B, ceil(S/32)] (bit k of word w = token
        32w+k is valid), which masks those keys in every layer and zeroes
        their output rows, as the reference does for any [B, S] bool mask
        (torch_transformer_benchmark.py:237-253, 496-510).

        Inspected once per mask object and version, like the reference's
        cached mask preparation (torch_transformer_benchmark.py:464-522),
        so graph capture sees no host synchronisation.
        """
        if mask is None:
            return None
        if mask.shape != x.shape[:2] or mask.dtype != torch.bool:
            raise ValueError("valid_token_mask must be a [B, S] bool tensor")
        ver = _version(mask)
        c = self._mask_cache
        if c is not None and ver is not None and c[0] is mask and c[1] == ver:
            return c[2]
        m = mask.to(x.device)
        if bool(m.all().item()):
            result = None
        else:
            lengths = m.sum(dim=1, dtype=torch.int32)
            prefix = torch.arange(m.shape[1], device=m.device)[None, :] < lengths[:, None]
            result = lengths.contiguous() if bool(torch.equal(prefix, m)) else key_bitmask(m)
        if ver is not None:
            self._mask_cache = (mask, ver, result)
        return result

    # ----------------------------------------------------------- forward
    def forward(
        self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None
    ) -> torch.Tensor:
        if x.device.type != "cuda":
            if self._kv_cache_enabled:
                raise RuntimeError("KV caching is implemented for CUDA inference")
            raise RuntimeError(
                "UserOptimizedTransformer runs only on CUDA (sm_100a); there is no CPU fallback"
            )
        if x.dim() != 3 or x.shape[-1] != self.config.d_model:
            raise ValueError(f"expected x of shape [B, S, {self.config.d_model}]")
        if x.dtype != torch.float32:
            raise ValueError("x must be float32 (the residual stream is fp32)")
        x = x.contiguous()
        if self._kv_cache_enabled:
            return self._forward_kv(x, valid_token_mask)
        batch, seq, _ = x.shape
        valid_len = self._valid_lengths(x, valid_token_mask)
        _, _, _, model = self._prepare(x.device)
        ws = self._workspace_for(x.device, model, batch, seq)
        y = torch.empty_like(x)
        self.run_into(x, y, valid_len, ws)
        return y

    def run_into(self, x: torch.Tensor, y: torch.Tensor,
                 valid_len: Optional[torch.Tensor] = None,
                 workspace: Optional[torch.Tensor] = None) -> None:
        """Enqueue the forward of ``x`` into the preallocated ``y`` (no
        allocation when ``workspace`` is given: safe inside graph capture).
        ``valid_len`` is what ``_valid_lengths`` returns: None, int32
        lengths [B], or the int32 token bitmask [B, ceil(S/32)]."""
        _, _, _, model = self._prepare(x.device)
        batch, seq, _ = x.shape
        if workspace is None:
            workspace = self._workspace_for(x.device, model, batch, seq)
        stream = torch.cuda.current_stream(x.device).cuda_stream
        if valid_len is not None and valid_len.dim() == 2:  # token bitmask
            _lib.check(
                _lib.load().tfx_forward_masked(
                    ctypes.byref(model), x.data_ptr(), y.data_ptr(), batch, seq,
                    valid_len.data_ptr(), workspace.data_ptr(), workspace.numel(), stream,
                ),
                "tfx_forward_masked",
            )
            return
        _lib.check(
            _lib.load().tfx_forward(
                ctypes.byref(model), x.data_ptr(), y.data_ptr(), batch, seq,
                valid_len.data_ptr() if valid_len is not None else None,
                workspace.data_ptr(), workspace.numel(), stream,
            ),
            "tfx_forward",
        )
