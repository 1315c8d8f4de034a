// Native whole-forward runtime: y = final_norm(blocks(x)).
//
// Sequences, on the caller's stream, the same dataflow as the reference's
// fused-norm CUDA path (torch_transformer_benchmark.py:1092-1148):
//
//   h   = LN(x; layers[0].norm1)                              [fp16]
//   per layer l:
//     qkv = h . Wqkv^T + bqkv                                 [fp16, tcgen05]
//     (head_dim 64/128: V^T = transpose(V) into h's buffer)   [fp16]
//     ctx = attention(qkv)                                    [fp16]
//     r   = ctx . Wo^T + bo + (l == 0 ? x : r)                [fp32, tcgen05]
//     h   = LN(r; norm2)                                      [fp16]
//     g   = gelu(h . W1^T + b1)  (exact erf form)             [fp16, tcgen05]
//     r   = g . W2^T + b2 + r                                 [fp32, tcgen05]
//     h   = LN(r; next norm1)  or  y = LN(r; final_norm)      [fp16 / fp32]
//
// The residual stream r stays fp32 end to end and the residual add happens
// in the GEMM epilogue (in fp32, before any rounding), where the reference
// adds an fp16-rounded update inside its LayerNorm kernel.
// No allocation, no host synchronisation: graph-capturable.
#include "internal.h"
#include "ptx.cuh"

namespace tfx {
namespace {

// Rows of padded tokens -> 0 (prefix lengths or a token bitmask).
__global__ void zero_padded_rows_kernel(float* y, int seq, int d, const int32_t* valid_len,
                                        const uint32_t* key_bits, int key_words, int64_t rows) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int b = static_cast<int>(row / seq), s = static_cast<int>(row % seq);
  const bool valid = valid_len != nullptr
                         ? s < valid_len[b]
                         : ((key_bits[static_cast<int64_t>(b) * key_words + s / 32] >> (s % 32)) & 1u);
  if (valid) return;
  float4* yr = reinterpret_cast<float4*>(y + row * d);
  for (int c = threadIdx.x & 31; c < d / 4; c += 32) yr[c] = make_float4(0.f, 0.f, 0.f, 0.f);
}

// KV cache append: the K and V thirds of each new token's packed projection
// row -> its position in the layer's caches ([batch][capacity][d] each).
// A warp per token row, 16-byte accesses.
__global__ void kv_append_kernel(const __half* __restrict__ qkv, int64_t ld_qkv,
                                 __half* __restrict__ k_cache, __half* __restrict__ v_cache,
                                 int new_tokens, int d, int capacity, int cache_len,
                                 int64_t rows) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int64_t b = row / new_tokens, t = row % new_tokens;
  const int64_t dst = (b * capacity + cache_len + t) * d;
  const uint4* sk = reinterpret_cast<const uint4*>(qkv + row * ld_qkv + d);
  const uint4* sv = reinterpret_cast<const uint4*>(qkv + row * ld_qkv + 2 * d);
  uint4* dk = reinterpret_cast<uint4*>(k_cache + dst);
  uint4* dv = reinterpret_cast<uint4*>(v_cache + dst);
  for (int c = threadIdx.x & 31; c < d / 8; c += 32) {
    dk[c] = sk[c];
    dv[c] = sv[c];
  }
}

constexpr size_t kAlign = 256;

// The model's own path setting decides (tfx_model.path); nothing here is
// process-wide.
bool use_fused(const tfx_model* m, int seq) {
  return m->path == TFX_PATH_AUTO && fused_forward_supported(m, seq);
}

// [a, a + a_bytes) and [b, b + b_bytes) share at least one byte.
bool ranges_overlap(const void* a, size_t a_bytes, const void* b, size_t b_bytes) {
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(a), b0 = reinterpret_cast<uintptr_t>(b);
  return a0 < b0 + b_bytes && b0 < a0 + a_bytes;
}

size_t round_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

struct Workspace {
  __half* h;
  __half* qkv;
  __half* ctx;
  float* res;
  __half* g;
  float* part;  // KV decode steps only: split-KV attention partials
  size_t bytes;
};

// The tcgen05 attention path (head_dim 64/128) reads V transposed; the copy
// lives in h's buffer, which is dead between the QKV GEMM and LayerNorm 2.
// (head_dim 256 keeps V in place: one K/V tile per query tile at the lengths
// it is used with, where the transpose would cost more than it saves.)
bool attention_reads_vt(int hd) { return hd == 64 || hd == 128; }

Workspace plan_workspace(char* base, int batch, int seq, int d, int f, int hd,
                         bool decode_scratch = false) {
  Workspace w{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    char* p = base ? base + off : nullptr;
    off += round_up(bytes);
    return p;
  };
  const int64_t m = static_cast<int64_t>(batch) * seq;
  size_t h_bytes = sizeof(__half) * m * d;
  if (attention_reads_vt(hd)) {
    const size_t vt_bytes = sizeof(__half) * static_cast<size_t>(batch) * d * attention_vt_ld(seq);
    h_bytes = h_bytes > vt_bytes ? h_bytes : vt_bytes;
  }
  w.h = reinterpret_cast<__half*>(take(h_bytes));
  w.qkv = reinterpret_cast<__half*>(take(sizeof(__half) * m * 3 * d));
  w.ctx = reinterpret_cast<__half*>(take(sizeof(__half) * m * d));
  w.res = reinterpret_cast<float*>(take(sizeof(float) * m * d));
  w.g = reinterpret_cast<__half*>(take(sizeof(__half) * m * f));
  if (decode_scratch)
    w.part = reinterpret_cast<float*>(take(attention_decode_part_bytes(batch, d / hd, seq, hd)));
  w.bytes = off;
  return w;
}

int check_model(const tfx_model* mdl) {
  if (mdl == nullptr || mdl->layers == nullptr)
    return fail(TFX_ERR_INVALID_ARGUMENT, "tfx_forward: null model");
  if (mdl->path != TFX_PATH_AUTO && mdl->path != TFX_PATH_CHAIN)
    return fail(TFX_ERR_INVALID_ARGUMENT, "tfx_forward: model path %d is not a tfx_path",
                mdl->path);
  const int d = mdl->d_model, h = mdl->num_heads, f = mdl->ffn_dim;
  if (d <= 0 || h <= 0 || f <= 0 || mdl->num_layers <= 0)
    return fail(TFX_ERR_INVALID_ARGUMENT, "tfx_forward: model sizes must be positive");
  if (d % h != 0) return fail(TFX_ERR_INVALID_ARGUMENT, "tfx_forward: d_model %% num_heads != 0");
  const int hd = d / h;
  if (hd != 8 && hd != 16 && hd != 32 && hd != 64 && hd != 128 && hd != 256)
    return fail(TFX_ERR_UNSUPPORTED, "tfx_forward: head_dim %d not in {8,16,32,64,128,256}", hd);
  if (d % 32 != 0 || f % 32 != 0 || d > 4096)
    return fail(TFX_ERR_UNSUPPORTED,
                "tfx_forward: d_model and ffn_dim must be multiples of 32, d_model <= 4096");
  for (int l = 0; l < mdl->num_layers; ++l) {
    const tfx_layer& L = mdl->layers[l];
    if (!L.norm1_weight || !L.norm1_bias || !L.qkv_weight || !L.qkv_bias || !L.out_weight ||
        !L.out_bias || !L.norm2_weight || !L.norm2_bias || !L.ffn_in_weight || !L.ffn_in_bias ||
        !L.ffn_out_weight || !L.ffn_out_bias)
      return fail(TFX_ERR_INVALID_ARGUMENT, "tfx_forward: layer %d has a null parameter", l);
  }
  if (!mdl->final_norm_weight || !mdl->final_norm_bias)
    return fail(TFX_ERR_INVALID_ARGUMENT, "tfx_forward: null final norm");
  return TFX_OK;
}

// Caller-owned KV caches of an incremental forward: fp16 [layers][batch]
// [capacity][d] each; positions < cache_len hold earlier tokens.
struct KvCache {
  __half* k;
  __half* v;
  int capacity;
  int cache_len;
};

// The per-op chain over `seq` token rows per sequence. With `kv`, each
// layer's new K/V rows are appended to its cache, and the new tokens attend
// every cached key (positions before theirs: causal with an offset).
int run_chain(const tfx_model* model, const float* x, float* y, int batch, int seq,
              const KeyMask& km, const Workspace& ws, cudaStream_t stream, const KvCache* kv) {
  const int64_t m = static_cast<int64_t>(batch) * seq;
  const int d = model->d_model, f = model->ffn_dim, nh = model->num_heads, hd = d / nh;
  const float eps = model->eps;
  const float scale = 1.0f / sqrtf(static_cast<float>(hd));

  int st = launch_layer_norm(x, model->layers[0].norm1_weight, model->layers[0].norm1_bias, ws.h,
                             TFX_DTYPE_F16, m, d, eps, 1, stream);
  if (st != TFX_OK) return st;
  for (int l = 0; l < model->num_layers; ++l) {
    const tfx_layer& L = model->layers[l];
    const __half* wqkv = reinterpret_cast<const __half*>(L.qkv_weight);
    st = launch_linear(ws.h, d, wqkv, L.qkv_bias, nullptr, 0, ws.qkv, 3 * d, m, 3 * d, d,
                       TFX_EPI_BIAS, stream);
    if (st != TFX_OK) return st;
    if (kv != nullptr) {
      const size_t layer_elems = static_cast<size_t>(batch) * kv->capacity * d;
      __half* kc = kv->k + l * layer_elems;
      __half* vc = kv->v + l * layer_elems;
      launch_pdl(kv_append_kernel, dim3(static_cast<unsigned>((m + 7) / 8)), dim3(256), 0,
                 stream, ws.qkv, static_cast<int64_t>(3 * d), kc, vc, seq, d, kv->capacity,
                 kv->cache_len, m);
      st = check_launch("kv_append_kernel");
      if (st != TFX_OK) return st;
    }
    if (kv != nullptr && kv->cache_len > 0) {
      const AttnKv geom{d, kv->capacity, kv->cache_len + seq, kv->cache_len};
      const size_t layer_elems = static_cast<size_t>(batch) * kv->capacity * d;
      if (seq <= kDecodeMaxQueries)  // decode step: split-KV over the cache
        st = launch_attention_decode(ws.qkv, 3 * d, kv->k + l * layer_elems,
                                     kv->v + l * layer_elems, geom, ws.ctx, d, batch, nh, seq, hd,
                                     scale, ws.part, stream);
      else
        st = launch_attention_kv(ws.qkv, 3 * d, kv->k + l * layer_elems, kv->v + l * layer_elems,
                                 geom, ws.ctx, d, batch, nh, seq, hd, scale, stream);
    } else if (attention_reads_vt(hd)) {
      st = launch_transpose_v(ws.qkv + 2 * d, 3 * d, ws.h, batch, seq, d, stream);
      if (st != TFX_OK) return st;
      st = launch_attention_tc_vt(ws.qkv, ws.qkv + d, ws.h, 3 * d, ws.ctx, d, batch, nh, seq, hd,
                                  scale, model->causal, km, stream);
    } else {
      st = launch_attention(ws.qkv, ws.qkv + d, ws.qkv + 2 * d, 3 * d, ws.ctx, d, batch, nh, seq,
                            hd, scale, model->causal, km, stream);
    }
    if (st != TFX_OK) return st;
    st = launch_linear(ws.ctx, d, reinterpret_cast<const __half*>(L.out_weight), L.out_bias,
                       l == 0 ? x : ws.res, d, ws.res, d, m, d, d, TFX_EPI_BIAS_RESIDUAL, stream);
    if (st != TFX_OK) return st;
    st = launch_layer_norm(ws.res, L.norm2_weight, L.norm2_bias, ws.h, TFX_DTYPE_F16, m, d, eps, 1,
                           stream);
    if (st != TFX_OK) return st;
    st = launch_linear(ws.h, d, reinterpret_cast<const __half*>(L.ffn_in_weight), L.ffn_in_bias,
                       nullptr, 0, ws.g, f, m, f, d, TFX_EPI_BIAS_GELU, stream);
    if (st != TFX_OK) return st;
    st = launch_linear(ws.g, f, reinterpret_cast<const __half*>(L.ffn_out_weight), L.ffn_out_bias,
                       ws.res, d, ws.res, d, m, d, f, TFX_EPI_BIAS_RESIDUAL, stream);
    if (st != TFX_OK) return st;
    const bool last = l + 1 == model->num_layers;
    if (!last) {
      st = launch_layer_norm(ws.res, model->layers[l + 1].norm1_weight,
                             model->layers[l + 1].norm1_bias, ws.h, TFX_DTYPE_F16, m, d, eps, 1,
                             stream);
    } else {
      st = launch_layer_norm(ws.res, model->final_norm_weight, model->final_norm_bias, y,
                             TFX_DTYPE_F32, m, d, eps, 1, stream);
    }
    if (st != TFX_OK) return st;
  }
  if (km.any()) {
    const int64_t blocks = (m + 7) / 8;
    launch_pdl(zero_padded_rows_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream,
               y, seq, d, km.len, km.bits, key_words(seq), m);
    st = check_launch("zero_padded_rows_kernel");
  }
  return st;
}


int forward_impl(const char* fn, const tfx_model* model, const float* x, float* y, int batch,
                 int seq, const KeyMask& km, void* workspace, size_t workspace_bytes,
                 cudaStream_t stream) {
  int st = check_model(model);
  if (st != TFX_OK) return st;
  if (x == nullptr || y == nullptr) return fail(TFX_ERR_INVALID_ARGUMENT, "%s: null x or y", fn);
  if (batch <= 0 || seq <= 0)
    return fail(TFX_ERR_INVALID_ARGUMENT, "%s: batch and seq must be positive", fn);
  const size_t act_bytes = sizeof(float) * static_cast<size_t>(batch) * seq * model->d_model;
  if (ranges_overlap(x, act_bytes, y, act_bytes))
    return fail(TFX_ERR_INVALID_ARGUMENT, "%s: y must not overlap x", fn);
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(y) % 16 ||
      reinterpret_cast<uintptr_t>(workspace) % kAlign)
    return fail(TFX_ERR_MISALIGNED, "%s: x/y 16-byte and workspace 256-byte alignment", fn);
  if (use_fused(model, seq)) return launch_fused_forward(model, x, y, batch, seq, km, stream);
  if (workspace == nullptr) return fail(TFX_ERR_INVALID_ARGUMENT, "%s: null workspace", fn);
  const int d = model->d_model, f = model->ffn_dim, hd = d / model->num_heads;
  const Workspace ws = plan_workspace(static_cast<char*>(workspace), batch, seq, d, f, hd);
  if (workspace_bytes < ws.bytes)
    return fail(TFX_ERR_WORKSPACE, "%s: workspace %zu < required %zu bytes", fn, workspace_bytes,
                ws.bytes);
  return run_chain(model, x, y, batch, seq, km, ws, stream, nullptr);
}

}  // namespace
}  // namespace tfx

using namespace tfx;

extern "C" {

int64_t tfx_forward_workspace_bytes(const tfx_model* model, int batch, int seq) {
  if (check_model(model) != TFX_OK || batch <= 0 || seq <= 0) return -1;
  if (use_fused(model, seq)) return 0;
  return static_cast<int64_t>(plan_workspace(nullptr, batch, seq, model->d_model, model->ffn_dim,
                                            model->d_model / model->num_heads)
                                 .bytes);
}

int tfx_forward(const tfx_model* model, const float* x, float* y, int batch, int seq,
                const int32_t* valid_len, void* workspace, size_t workspace_bytes,
                tfx_stream_t stream_) {
  KeyMask km;
  km.len = valid_len;
  return forward_impl("tfx_forward", model, x, y, batch, seq, km, workspace, workspace_bytes,
                      reinterpret_cast<cudaStream_t>(stream_));
}

int tfx_forward_masked(const tfx_model* model, const float* x, float* y, int batch, int seq,
                       const uint32_t* key_mask, void* workspace, size_t workspace_bytes,
                       tfx_stream_t stream_) {
  if (key_mask == nullptr)
    return fail(TFX_ERR_INVALID_ARGUMENT, "tfx_forward_masked: null key_mask");
  if (reinterpret_cast<uintptr_t>(key_mask) % 4)
    return fail(TFX_ERR_MISALIGNED, "tfx_forward_masked: key_mask must be 4-byte aligned");
  KeyMask km;
  km.bits = key_mask;
  return forward_impl("tfx_forward_masked", model, x, y, batch, seq, km, workspace,
                      workspace_bytes, reinterpret_cast<cudaStream_t>(stream_));
}

int64_t tfx_forward_kv_workspace_bytes(const tfx_model* model, int batch, int new_tokens) {
  if (check_model(model) != TFX_OK || batch <= 0 || new_tokens <= 0) return -1;
  return static_cast<int64_t>(plan_workspace(nullptr, batch, new_tokens, model->d_model,
                                            model->ffn_dim, model->d_model / model->num_heads,
                                            new_tokens <= kDecodeMaxQueries)
                                 .bytes);
}

int tfx_forward_kv(const tfx_model* model, const float* x, float* y, int batch, int new_tokens,
                   int cache_len, int capacity, void* k_cache, void* v_cache, void* workspace,
                   size_t workspace_bytes, tfx_stream_t stream_) {
  int st = check_model(model);
  if (st != TFX_OK) return st;
  if (!model->causal)
    return fail(TFX_ERR_UNSUPPORTED, "tfx_forward_kv: KV caching requires a causal model");
  if (x == nullptr || y == nullptr || k_cache == nullptr || v_cache == nullptr ||
      workspace == nullptr)
    return fail(TFX_ERR_INVALID_ARGUMENT, "tfx_forward_kv: null pointer argument");
  if (batch <= 0 || new_tokens <= 0 || cache_len < 0 || capacity <= 0)
    return fail(TFX_ERR_INVALID_ARGUMENT,
                "tfx_forward_kv: batch, new_tokens and capacity must be positive, cache_len >= 0");
  if (static_cast<int64_t>(cache_len) + new_tokens > capacity)
    return fail(TFX_ERR_INVALID_ARGUMENT, "tfx_forward_kv: KV cache capacity exceeded (%lld > %d)",
                static_cast<long long>(cache_len) + new_tokens, capacity);
  const size_t act_bytes = sizeof(float) * static_cast<size_t>(batch) * new_tokens *
                           model->d_model;
  if (ranges_overlap(x, act_bytes, y, act_bytes))
    return fail(TFX_ERR_INVALID_ARGUMENT, "tfx_forward_kv: y must not overlap x");
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(y) % 16 ||
      reinterpret_cast<uintptr_t>(k_cache) % 16 || reinterpret_cast<uintptr_t>(v_cache) % 16 ||
      reinterpret_cast<uintptr_t>(workspace) % kAlign)
    return fail(TFX_ERR_MISALIGNED,
                "tfx_forward_kv: x/y/caches 16-byte and workspace 256-byte alignment");
  const int d = model->d_model, f = model->ffn_dim, hd = d / model->num_heads;
  const Workspace ws = plan_workspace(static_cast<char*>(workspace), batch, new_tokens, d, f, hd,
                                      new_tokens <= kDecodeMaxQueries);
  if (workspace_bytes < ws.bytes)
    return fail(TFX_ERR_WORKSPACE, "tfx_forward_kv: workspace %zu < required %zu bytes",
                workspace_bytes, ws.bytes);
  const KvCache kv{static_cast<__half*>(k_cache), static_cast<__half*>(v_cache), capacity,
                   cache_len};
  return run_chain(model, x, y, batch, new_tokens, KeyMask{}, ws,
                   reinterpret_cast<cudaStream_t>(stream_), &kv);
}

}  // extern "C"
