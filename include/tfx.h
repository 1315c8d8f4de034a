/*
 * tfx.h -- C ABI of the B200 (sm_100a) pre-norm causal Transformer forward.
 *
 * Every entry point takes caller-owned DEVICE pointers, plain sizes and a
 * CUDA stream (cudaStream_t, passed as tfx_stream_t), enqueues its kernels on
 * that stream and returns immediately: no allocation, no host
 * synchronisation, no host reads of device data, so every call can be
 * captured in a CUDA graph. Return value: TFX_OK (0) or a negative
 * tfx_status; tfx_last_error_message() gives the detail for the calling
 * thread. Argument errors are detected on the host before anything is
 * enqueued.
 *
 * Dtypes: activations entering a tensor-core op are IEEE fp16 (tfx_half);
 * the residual stream, LayerNorm parameters, biases, statistics and all
 * accumulators are fp32.
 *
 * Each declaration names the reference interface it replaces
 * (gwenlim89/GPU-kernel-for-transformer, file:line).
 */
#ifndef TFX_B200_H
#define TFX_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define TFX_API __attribute__((visibility("default")))
#else
#define TFX_API
#endif

typedef struct CUstream_st* tfx_stream_t; /* identical to cudaStream_t */
typedef uint16_t tfx_half;                /* IEEE binary16 bit pattern   */

typedef enum tfx_status {
  TFX_OK = 0,
  TFX_ERR_INVALID_ARGUMENT = -1, /* null pointer, non-positive size, bad enum     */
  TFX_ERR_UNSUPPORTED = -2,      /* shape outside what the kernels implement       */
  TFX_ERR_MISALIGNED = -3,       /* pointer / leading dimension alignment violated */
  TFX_ERR_WORKSPACE = -4,        /* workspace too small                            */
  TFX_ERR_CUDA = -5,             /* a CUDA runtime call or launch failed           */
  TFX_ERR_DEVICE = -6            /* a kernel reported a bounded-wait timeout       */
} tfx_status;

typedef enum tfx_dtype { TFX_DTYPE_F16 = 0, TFX_DTYPE_F32 = 1 } tfx_dtype;

typedef enum tfx_epilogue {
  TFX_EPI_BIAS = 0,          /* out(f16) = A.W^T + bias                          */
  TFX_EPI_BIAS_GELU = 1,     /* out(f16) = gelu_erf(A.W^T + bias)                */
  TFX_EPI_BIAS_RESIDUAL = 2  /* out(f32) = A.W^T + bias + residual(f32)          */
} tfx_epilogue;

/* Library version (major*10000 + minor*100 + patch). */
TFX_API int tfx_version(void);

/* Static description of a status code. */
TFX_API const char* tfx_status_string(int status);

/* Detail of the last failure on the calling thread ("" if none). */
TFX_API const char* tfx_last_error_message(void);

/*
 * LayerNorm over the last dimension: y = (x - mean) * rsqrt(var + eps)
 * [* gamma + beta when apply_affine], statistics in fp32, biased variance.
 * x: [rows, d] fp32; y: [rows, d] in y_dtype (TFX_DTYPE_F16 or _F32).
 * d: multiple of 4, 4..4096.
 * Replaces: triton_fused_norm.py:140-170 (layer_norm) and its kernel
 * triton_fused_norm.py:84-121.
 */
TFX_API int tfx_layer_norm(const float* x, const float* gamma, const float* beta, void* y, int y_dtype,
                   int64_t rows, int d, float eps, int apply_affine, tfx_stream_t stream);

/*
 * Fused residual add + LayerNorm: s = residual + update (fp32 math);
 * if residual_out != NULL store s there (may equal residual); y = LN(s).
 * residual: [rows, d] fp32; update: [rows, d] fp16; y in y_dtype.
 * Replaces: triton_fused_norm.py:173-215 (fused_residual_layer_norm) and
 * triton_fused_norm.py:37-81; residual_out == NULL is STORE_RESIDUAL=False.
 */
TFX_API int tfx_residual_layer_norm(const float* residual, const tfx_half* update, const float* gamma,
                            const float* beta, float* residual_out, void* y, int y_dtype,
                            int64_t rows, int d, float eps, int apply_affine,
                            tfx_stream_t stream);

/*
 * Tensor-core linear layer (tcgen05 + TMEM, fp16 operands, fp32 accumulate):
 *   acc[m, n] = sum_k a[m, k] * w[n, k]      (w is nn.Linear's [out, in])
 * followed by the epilogue (tfx_epilogue). a: [m, k] fp16 row-major;
 * w: [n, k] fp16 row-major; bias: [n] fp32; residual: [m, n] fp32 (only for
 * TFX_EPI_BIAS_RESIDUAL; may alias out). out: [m, n], fp16 or fp32 per
 * epilogue. Requirements: k % 8 == 0, n % 16 == 0, 16-byte aligned pointers.
 * Replaces: F.linear with cached fp16 weights (torch_transformer_benchmark.py
 * :675-685, :741, :818, :994) and triton_ffn_gelu / _ffn_gelu_kernel
 * (triton_fused_ffn.py:224-261, :106-221) -- with exact-erf GELU, as the
 * baseline model uses (torch_transformer_benchmark.py:286), not tanh.
 */
TFX_API int tfx_linear(const tfx_half* a, const tfx_half* w, const float* bias, const float* residual,
               void* out, int64_t m, int n, int k, int epilogue, tfx_stream_t stream);

/*
 * Flash-style multi-head self-attention, softmax(Q.K^T * scale [+ causal
 * mask] [+ key padding]) . V, never materialising the S x S matrix.
 * q/k/v: element (b, s, h, e) at ptr[(b*seq + s)*ld_qkv + h*head_dim + e]
 * (the packed [B, S, 3, H, hd] projection output is q = base,
 * k = base + H*hd, v = base + 2*H*hd, ld_qkv = 3*H*hd).
 * out: element (b, s, h, e) at out[(b*seq + s)*ld_out + h*head_dim + e].
 * valid_len: NULL, or [batch] int32 prefix lengths; keys >= valid_len[b]
 * are masked. head_dim in {8, 16, 32, 64, 128, 256}.
 * Replaces: the F.scaled_dot_product_attention call and its backend
 * dispatch in _fast_attention_impl (torch_transformer_benchmark.py:767-808).
 */
TFX_API int tfx_attention(const tfx_half* q, const tfx_half* k, const tfx_half* v, int64_t ld_qkv,
                  tfx_half* out, int64_t ld_out, int batch, int heads, int seq, int head_dim,
                  float scale, int causal, const int32_t* valid_len, tfx_stream_t stream);

/*
 * tfx_attention with key padding of any pattern instead of prefix lengths:
 * key_mask [batch][(seq + 31) / 32] uint32, bit k of word w of sequence b set
 * = key 32*w + k of that sequence may be attended (4-byte aligned). A query
 * whose visible keys are all masked gets a zero output row.
 * Replaces: SDPA with the dense attn_mask = key_mask & causal_mask that
 * _prepare_attention_args builds for padded inputs
 * (torch_transformer_benchmark.py:496-510, 767-808).
 */
TFX_API int tfx_attention_masked(const tfx_half* q, const tfx_half* k, const tfx_half* v,
                                 int64_t ld_qkv, tfx_half* out, int64_t ld_out, int batch,
                                 int heads, int seq, int head_dim, float scale, int causal,
                                 const uint32_t* key_mask, tfx_stream_t stream);

/*
 * The attention path tfx_forward takes for head_dim 64 and 128, in its two
 * steps. No counterpart in the reference: V transposed is this library's
 * internal layout (the tcgen05 P.V products then read V as a K-major operand
 * at full rate); exported so the per-kernel benchmark and the parity tests can
 * drive exactly what the forward runs.
 *
 * tfx_transpose_v: vt[b][c][s] = v[(b*seq + s)*ld_qkv + c] for c < cols
 * (cols = H*head_dim, a multiple of 64), s < seq; row pitch
 * tfx_attention_vt_ld(seq) elements (seq rounded up to 8), zero-filled pad.
 * tfx_attention_vt: as tfx_attention with V given as that vt; head_dim in
 * {64, 128, 256}, scale > 0.
 */
TFX_API int64_t tfx_attention_vt_ld(int seq);
TFX_API int tfx_transpose_v(const tfx_half* v, int64_t ld_qkv, tfx_half* vt, int batch, int seq,
                            int cols, tfx_stream_t stream);
TFX_API int tfx_attention_vt(const tfx_half* q, const tfx_half* k, const tfx_half* vt,
                             int64_t ld_qkv, tfx_half* out, int64_t ld_out, int batch, int heads,
                             int seq, int head_dim, float scale, int causal,
                             const int32_t* valid_len, tfx_stream_t stream);

/* One pre-norm block's parameters, all device pointers (see tfx_model). */
typedef struct tfx_layer {
  const float* norm1_weight;  /* [D] */
  const float* norm1_bias;    /* [D] */
  const tfx_half* qkv_weight; /* [3D, D]: rows q_proj | k_proj | v_proj */
  const float* qkv_bias;      /* [3D] */
  const tfx_half* out_weight; /* [D, D] */
  const float* out_bias;      /* [D] */
  const float* norm2_weight;  /* [D] */
  const float* norm2_bias;    /* [D] */
  const tfx_half* ffn_in_weight;  /* [F, D] */
  const float* ffn_in_bias;       /* [F] */
  const tfx_half* ffn_out_weight; /* [D, F] */
  const float* ffn_out_bias;      /* [D] */
} tfx_layer;

/* Which kernels tfx_forward runs for a model (tfx_model.path). */
typedef enum tfx_path {
  TFX_PATH_AUTO = 0,  /* fused whole-forward kernel wherever it applies (d_model =
                         ffn_dim = 128, seq_len dividing 128, head_dim in
                         {8, 16, 32, 64, 128}, <= 5 layers), else the per-op chain */
  TFX_PATH_CHAIN = 1  /* always the per-op kernel chain */
} tfx_path;

typedef struct tfx_model {
  int d_model;
  int num_heads;
  int ffn_dim;
  int num_layers;
  int causal;
  float eps;                   /* LayerNorm eps (nn.LayerNorm default 1e-5) */
  const tfx_layer* layers;     /* HOST array of num_layers entries         */
  const float* final_norm_weight;
  const float* final_norm_bias;
  /* tfx_path of this model (zero-initialised structs get TFX_PATH_AUTO).
   * A per-model setting, like the reference's per-module toggles
   * enable_triton_fused_norm / _ffn (torch_transformer_benchmark.py:379-393):
   * two models in one process never change each other's kernels. Query
   * tfx_forward_workspace_bytes again after changing it. */
  int path;
} tfx_model;

/* Bytes of device workspace tfx_forward needs for a [batch, seq] input
 * (0 when the fused whole-forward kernel applies to this model and path). */
TFX_API int64_t tfx_forward_workspace_bytes(const tfx_model* model, int batch, int seq);

/*
 * Whole forward: y = final_norm(blocks(x)), x and y [batch, seq, D] fp32,
 * 16-byte aligned (TFX_ERR_MISALIGNED otherwise; the fused kernel reads x
 * with TMA), batch * seq below 2^31 tokens
 * (the two ranges must not overlap: TFX_ERR_INVALID_ARGUMENT). valid_len: NULL or [batch] int32 prefix lengths
 * (padded rows of y are zeroed, padded keys masked). workspace: device
 * buffer of at least tfx_forward_workspace_bytes() (may be NULL when that
 * is 0).
 * Replaces: UserOptimizedTransformer.forward -> _forward_cuda ->
 * _forward_cuda_fused_norm (torch_transformer_benchmark.py:996-1020,
 * :1051-1090, :1092-1148).
 */
TFX_API int tfx_forward(const tfx_model* model, const float* x, float* y, int batch, int seq,
                const int32_t* valid_len, void* workspace, size_t workspace_bytes,
                tfx_stream_t stream);

/*
 * tfx_forward with a padding mask of any pattern: key_mask [batch]
 * [(seq + 31) / 32] uint32, bit k of word w of sequence b set = token 32*w+k
 * is valid (4-byte aligned). Padded tokens are masked as keys in every
 * layer and their output rows are zero, as in the reference's baseline
 * (torch_transformer_benchmark.py:237-253, 288-289, 314-316). Same kernels,
 * workspace and errors as tfx_forward.
 * Replaces: _prepare_attention_args for a non-prefix valid_token_mask
 * (torch_transformer_benchmark.py:464-522) and the masked forward it feeds.
 */
TFX_API int tfx_forward_masked(const tfx_model* model, const float* x, float* y, int batch,
                               int seq, const uint32_t* key_mask, void* workspace,
                               size_t workspace_bytes, tfx_stream_t stream);

/*
 * tfx_forward without a workspace argument, for callers that cannot allocate
 * device memory (plugins whose host runtime owns all GPU memory, FFI
 * bindings that can pass only the input and output buffers, serving loops
 * that must not allocate after start-up). The per-op kernel chain's
 * intermediates live in a fixed 32 MiB device array inside this library,
 * held on every GPU that loads it until the process exits; calls whose
 * tfx_forward_workspace_bytes() exceeds 32 MiB return TFX_ERR_WORKSPACE
 * before anything is enqueued. All calls on a device share that array:
 * calls that overlap on the GPU (unordered streams, several threads) race.
 * The array need not be cleared between calls. The first call on each
 * device looks up the array's device address, so make it before any stream
 * capture. No counterpart in the reference.
 */
TFX_API int tfx_forward_static(const tfx_model* model, const float* x, float* y, int batch,
                               int seq, const int32_t* valid_len, tfx_stream_t stream);

/*
 * KV-cached incremental forward of a causal model: replaces the reference's
 * enable_kv_cache path (torch_transformer_benchmark.py:409-462 cache
 * management and _append_kv_cache, 747-765 the new tokens' attention over
 * the cache, 1085-1086 the length update).
 * x, y: [batch, new_tokens, d_model] fp32, the tokens at positions
 * cache_len .. cache_len + new_tokens - 1 of each sequence.
 * k_cache, v_cache: caller-owned fp16 device arrays [num_layers][batch]
 * [capacity][d_model] (16-byte aligned). Positions < cache_len hold the
 * earlier tokens' keys / values; this call writes positions cache_len ..
 * cache_len + new_tokens - 1 of every layer and leaves the rest untouched.
 * Each new token attends every key at or before its own position.
 * Errors: TFX_ERR_UNSUPPORTED for a non-causal model, TFX_ERR_INVALID_ARGUMENT
 * when cache_len + new_tokens > capacity (the reference's "KV cache capacity
 * exceeded"), TFX_ERR_WORKSPACE when the workspace is below
 * tfx_forward_kv_workspace_bytes(model, batch, new_tokens).
 */
TFX_API int64_t tfx_forward_kv_workspace_bytes(const tfx_model* model, int batch,
                                               int new_tokens);
TFX_API int tfx_forward_kv(const tfx_model* model, const float* x, float* y, int batch,
                           int new_tokens, int cache_len, int capacity, void* k_cache,
                           void* v_cache, void* workspace, size_t workspace_bytes,
                           tfx_stream_t stream);

/*
 * Reads and clears the calling device's kernel error word (synchronises the
 * device). *code receives 0 or a timeout code; returns TFX_OK or TFX_ERR_CUDA.
 * No reference counterpart (the reference's kernels have no waits).
 */
TFX_API int tfx_read_device_error(int* code);

/*
 * Error codes a kernel writes to the device error word (first one wins).
 */
enum {
  TFX_DEV_TIMEOUT_FULL = 1,       /* gave up waiting for a loaded stage          */
  TFX_DEV_TIMEOUT_EMPTY = 2,      /* producer gave up waiting for a free stage   */
  TFX_DEV_TIMEOUT_ACCUM = 3,      /* gave up waiting for an accumulator          */
  TFX_DEV_TIMEOUT_ACCUM_FREE = 4, /* gave up waiting for a free accumulator      */
  TFX_DEV_TIMEOUT_OTHER = 5
};

/*
 * Runs the bounded-wait protocol of the pipelined kernels on a wait that
 * cannot complete: one CTA holds a TMEM allocation and a bulk copy in
 * flight while a consumer warp waits on an mbarrier nobody arrives on, for
 * at most limit_cycles SM cycles (0 < limit_cycles <= 2e9, about 1 s); it then
 * records TFX_DEV_TIMEOUT_ACCUM, drains its copy, frees TMEM and returns.
 * tfx_read_device_error afterwards reports the code and the context stays
 * usable. For tests of failure detection. No reference counterpart (the
 * reference's kernels have no waits).
 */
TFX_API int tfx_selftest_bounded_wait(int64_t limit_cycles, tfx_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* TFX_B200_H */
