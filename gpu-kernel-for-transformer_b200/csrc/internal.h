// Internal host-side declarations shared by the .cu translation units.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/tfx.h"

namespace tfx {

// Records a human-readable detail for the calling thread and returns `status`.
int fail(int status, const char* fmt, ...);

// Checks cudaGetLastError after a launch; maps a failure to TFX_ERR_CUDA.
int check_launch(const char* what);

// Launches `kern` with programmatic stream serialization: the kernel may be
// scheduled while the previous kernel in the stream is still running, and
// waits for it inside (grid_dep_wait in ptx.cuh) after its prologue, so the
// launch latency and prologue overlap the predecessor's tail. Every kernel of
// this library calls grid_dep_wait before its first global or TMEM access;
// launches after a non-kernel operation (copy, event wait) are ordinary.
template <typename... P, typename... A>
inline cudaError_t launch_pdl(void (*kern)(P...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, A&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<A&&>(args)...);
}

// Device error word (per device) the kernels write on a bounded-wait timeout.
int* device_error_word();

int num_sms();
int current_device();

// Opt a kernel into more than 48 KB of dynamic shared memory, once per device.
int ensure_smem(const void* func, int bytes, int* done_flags /* [kMaxDevices] */);
constexpr int kMaxDevices = 64;

// cuTensorMapEncodeTiled resolved through the runtime (no -lcuda link).
// 2-D fp16/fp32 row-major matrix [rows, cols] with row pitch `ld` elements;
// box = box_cols x box_rows; swizzle as given.
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                 uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_cols, uint32_t box_rows,
                 CUtensorMapSwizzle swizzle);

// 3-D fp16 view [batch][rows][cols] (row pitch `ld`, batch pitch
// `batch_stride`, both in elements) with a box of box_cols x box_rows x 1 and
// the 128-byte swizzle. Rows past `rows` inside a batch read as zeros.
int make_tmap_3d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t batch, uint64_t cols,
                 uint64_t ld, uint64_t batch_stride, uint32_t box_cols, uint32_t box_rows);

// Which keys of each sequence attention may use, and which output rows are
// real tokens: all of them (both null), a prefix per sequence (len: [batch]
// int32 valid lengths), or any pattern (bits: [batch][key_words(seq)] uint32,
// bit k of word w set = token 32w+k is valid). At most one is set.
struct KeyMask {
  const int32_t* len = nullptr;
  const uint32_t* bits = nullptr;
  bool any() const { return len != nullptr || bits != nullptr; }
};
inline int key_words(int seq) { return (seq + 31) / 32; }

// Kernel launchers (validated by the C-ABI layer before they are called).
int launch_layer_norm(const float* x, const float* gamma, const float* beta, void* y, int y_dtype,
                      int64_t rows, int d, float eps, int apply_affine, cudaStream_t stream);
int launch_residual_layer_norm(const float* r, const __half* u, const float* gamma,
                               const float* beta, float* r_out, void* y, int y_dtype,
                               int64_t rows, int d, float eps, int apply_affine,
                               cudaStream_t stream);
int launch_linear(const __half* a, int64_t lda, const __half* w, const float* bias,
                  const float* residual, int64_t ldr, void* out, int64_t ldo, int64_t m, int n,
                  int k, int epilogue, cudaStream_t stream);
int launch_attention(const __half* q, const __half* k, const __half* v, int64_t ld_qkv,
                     __half* out, int64_t ld_out, int batch, int heads, int seq, int head_dim,
                     float scale, int causal, const KeyMask& km, cudaStream_t stream);

// Where an attention call's keys and values live relative to its queries.
// Self-attention: interleaved with the queries ({ld_qkv, seq, seq, 0}). KV
// cache: [batch][capacity][d] arrays of their own, the new tokens' queries
// at key positions q_off .. q_off + q_len - 1.
struct AttnKv {
  int64_t ld;          // K/V row pitch (elements)
  int64_t batch_rows;  // rows from one sequence's K/V to the next
  int len;             // keys per sequence
  int q_off;           // key position of query row 0 (causal: row i sees keys <= q_off + i)
};

// Decode steps (q_len <= kDecodeMaxQueries new queries per sequence over a KV
// cache): split-KV kernel + combine; `part` is scratch of
// attention_decode_part_bytes(batch, heads, q_len, head_dim) bytes.
constexpr int kDecodeMaxQueries = 16;
size_t attention_decode_part_bytes(int batch, int heads, int q_len, int head_dim);
int launch_attention_decode(const __half* q, int64_t ld_q, const __half* k, const __half* v,
                            const AttnKv& kv, __half* out, int64_t ld_out, int batch, int heads,
                            int q_len, int head_dim, float scale, float* part,
                            cudaStream_t stream);

// Causal attention of q_len new queries per sequence (row pitch ld_q,
// sequences q_len rows apart) over kv.len cached keys; every head_dim.
int launch_attention_kv(const __half* q, int64_t ld_q, const __half* k, const __half* v,
                        const AttnKv& kv, __half* out, int64_t ld_out, int batch, int heads,
                        int q_len, int head_dim, float scale, cudaStream_t stream);

// tcgen05/TMEM flash attention for head_dim 64 and 128 (scale > 0).
bool attention_tc_supported(int head_dim, float scale);
int launch_attention_tc(const __half* q, const __half* k, const __half* v, int64_t ld_qkv,
                        __half* out, int64_t ld_out, int batch, int heads, int seq, int head_dim,
                        float scale, int causal, const KeyMask& km, cudaStream_t stream);
// tcgen05/TMEM flash attention for head_dim 8, 16 and 32: one CTA per 128
// query rows and 64-column block of heads (heads * head_dim a multiple of 64).
bool attention_tc_small_supported(int head_dim, int heads, int batch, int seq, float scale);
int launch_attention_tc_small(const __half* q, const __half* k, const __half* v, int64_t ld_qkv,
                              __half* out, int64_t ld_out, int batch, int heads, int seq,
                              int head_dim, float scale, int causal, const KeyMask& km,
                              cudaStream_t stream);
// Same kernel reading V from a transposed copy vt[b][h*hd + d][s] (row pitch
// attention_vt_ld(seq) elements), written by launch_transpose_v from the
// packed projection; the P.V products then use a K-major operand.
int64_t attention_vt_ld(int seq);
int launch_transpose_v(const __half* v, int64_t ld_qkv, __half* vt, int batch, int seq, int cols,
                       cudaStream_t stream);
int launch_attention_tc_kv(const __half* q, int64_t ld_q, const __half* k, const __half* v,
                           const AttnKv& kv, __half* out, int64_t ld_out, int batch, int heads,
                           int q_len, int head_dim, float scale, cudaStream_t stream);
int launch_attention_tc_vt(const __half* q, const __half* k, const __half* vt, int64_t ld_qkv,
                           __half* out, int64_t ld_out, int batch, int heads, int seq,
                           int head_dim, float scale, int causal, const KeyMask& km,
                           cudaStream_t stream);

// Whole-forward fused kernel (d_model = ffn_dim = 128, seq | 128).
bool fused_forward_supported(const tfx_model* m, int seq);
int launch_fused_forward(const tfx_model* m, const float* x, float* y, int batch, int seq,
                         const KeyMask& km, cudaStream_t stream);

}  // namespace tfx
