// C ABI (include/tfx.h): host-side validation, error reporting, and the
// native whole-forward runtime that sequences the kernels of one
// pre-norm causal Transformer forward on the caller's stream.
#include <cstdarg>
#include <cstring>
#include <mutex>

#include "internal.h"

namespace tfx {

namespace {
thread_local char g_msg[512] = {0};

__device__ int g_device_error[1];

struct DeviceProps {
  int sms = 0;
};
DeviceProps g_props[kMaxDevices];
std::mutex g_mu;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
}  // namespace

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return status;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(TFX_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return TFX_OK;
}

int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

int num_sms() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return 148;
  if (g_props[dev].sms == 0) {
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    g_props[dev].sms = sms > 0 ? sms : 148;
  }
  return g_props[dev].sms;
}

int* device_error_word() {
  static int* ptrs[kMaxDevices] = {nullptr};
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  if (ptrs[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    ptrs[dev] = static_cast<int*>(p);
  }
  return ptrs[dev];
}

int ensure_smem(const void* func, int bytes, int* done_flags) {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return fail(TFX_ERR_CUDA, "device index out of range");
  if (done_flags[dev]) return TFX_OK;
  const cudaError_t e =
      cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess)
    return fail(TFX_ERR_CUDA, "cudaFuncSetAttribute(%d B smem): %s", bytes, cudaGetErrorString(e));
  done_flags[dev] = 1;
  return TFX_OK;
}

// cuTensorMapEncodeTiled, looked up once through the runtime.
static int resolve_encode() {
  if (g_encode == nullptr) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_encode == nullptr) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      const cudaError_t e =
          cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
      if (e != cudaSuccess || fn == nullptr || q != cudaDriverEntryPointSuccess)
        return fail(TFX_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
  }
  return TFX_OK;
}

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                 uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_cols, uint32_t box_rows,
                 CUtensorMapSwizzle swizzle) {
  if (int st = resolve_encode()) return st;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld * static_cast<uint64_t>(elem_bytes)};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = g_encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(TFX_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d): rows=%llu cols=%llu ld=%llu",
                static_cast<int>(r), (unsigned long long)rows, (unsigned long long)cols,
                (unsigned long long)ld);
  return TFX_OK;
}

int make_tmap_3d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t batch, uint64_t cols,
                 uint64_t ld, uint64_t batch_stride, uint32_t box_cols, uint32_t box_rows) {
  if (int st = resolve_encode()) return st;
  const cuuint64_t dims[3] = {cols, rows, batch};
  const cuuint64_t strides[2] = {ld * 2, batch_stride * 2};
  const cuuint32_t box[3] = {box_cols, box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base),
                              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(TFX_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed (%d): rows=%llu batch=%llu",
                static_cast<int>(r), (unsigned long long)rows, (unsigned long long)batch);
  return TFX_OK;
}

namespace {

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int check_ln_args(const char* fn, const void* x, const float* gamma, const float* beta,
                  const void* y, int y_dtype, int64_t rows, int d, int affine) {
  if (x == nullptr || y == nullptr) return fail(TFX_ERR_INVALID_ARGUMENT, "%s: null tensor", fn);
  if (affine && (gamma == nullptr || beta == nullptr))
    return fail(TFX_ERR_INVALID_ARGUMENT, "%s: affine LayerNorm needs gamma and beta", fn);
  if (rows <= 0 || d <= 0)
    return fail(TFX_ERR_INVALID_ARGUMENT, "%s: rows and d must be positive", fn);
  if (y_dtype != TFX_DTYPE_F16 && y_dtype != TFX_DTYPE_F32)
    return fail(TFX_ERR_INVALID_ARGUMENT, "%s: y_dtype must be F16 or F32", fn);
  if (d % 4 != 0 || d > 4096)
    return fail(TFX_ERR_UNSUPPORTED, "%s: d=%d must be a multiple of 4 and <= 4096", fn, d);
  if (!aligned(x, 16) || !aligned(y, 16) || (affine && (!aligned(gamma, 16) || !aligned(beta, 16))))
    return fail(TFX_ERR_MISALIGNED, "%s: pointers must be 16-byte aligned", fn);
  return TFX_OK;
}

int attention_checked(const char* fn, const tfx_half* q, const tfx_half* k, const tfx_half* v,
                      int64_t ld_qkv, tfx_half* out, int64_t ld_out, int batch, int heads, int seq,
                      int head_dim, float scale, int causal, const KeyMask& km,
                      cudaStream_t stream) {
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr)
    return fail(TFX_ERR_INVALID_ARGUMENT, "%s: null tensor", fn);
  if (batch <= 0 || heads <= 0 || seq <= 0 || head_dim <= 0)
    return fail(TFX_ERR_INVALID_ARGUMENT, "%s: sizes must be positive", fn);
  if (heads > 65535 || batch > 65535)
    return fail(TFX_ERR_UNSUPPORTED, "%s: batch and heads must be <= 65535", fn);
  if (ld_qkv < static_cast<int64_t>(heads) * head_dim ||
      ld_out < static_cast<int64_t>(heads) * head_dim)
    return fail(TFX_ERR_INVALID_ARGUMENT, "%s: leading dimension smaller than H*hd", fn);
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(out, 16) ||
      ld_qkv % 8 != 0 || ld_out % 8 != 0)
    return fail(TFX_ERR_MISALIGNED,
                "%s: pointers 16-byte aligned and leading dims multiples of 8 needed", fn);
  return launch_attention(reinterpret_cast<const __half*>(q), reinterpret_cast<const __half*>(k),
                          reinterpret_cast<const __half*>(v), ld_qkv,
                          reinterpret_cast<__half*>(out), ld_out, batch, heads, seq, head_dim,
                          scale, causal, km, stream);
}

}  // namespace
}  // namespace tfx

using namespace tfx;

extern "C" {

int tfx_version(void) { return 100; }

const char* tfx_status_string(int status) {
  switch (status) {
    case TFX_OK: return "ok";
    case TFX_ERR_INVALID_ARGUMENT: return "invalid argument";
    case TFX_ERR_UNSUPPORTED: return "unsupported shape";
    case TFX_ERR_MISALIGNED: return "misaligned pointer or leading dimension";
    case TFX_ERR_WORKSPACE: return "workspace too small";
    case TFX_ERR_CUDA: return "CUDA error";
    case TFX_ERR_DEVICE: return "device-side timeout";
    default: return "unknown status";
  }
}

const char* tfx_last_error_message(void) { return g_msg; }

int tfx_layer_norm(const float* x, const float* gamma, const float* beta, void* y, int y_dtype,
                   int64_t rows, int d, float eps, int apply_affine, tfx_stream_t stream) {
  g_msg[0] = 0;
  int st = check_ln_args("tfx_layer_norm", x, gamma, beta, y, y_dtype, rows, d, apply_affine);
  if (st != TFX_OK) return st;
  return launch_layer_norm(x, gamma, beta, y, y_dtype, rows, d, eps, apply_affine,
                           reinterpret_cast<cudaStream_t>(stream));
}

int tfx_residual_layer_norm(const float* residual, const tfx_half* update, const float* gamma,
                            const float* beta, float* residual_out, void* y, int y_dtype,
                            int64_t rows, int d, float eps, int apply_affine,
                            tfx_stream_t stream) {
  g_msg[0] = 0;
  int st = check_ln_args("tfx_residual_layer_norm", residual, gamma, beta, y, y_dtype, rows, d,
                         apply_affine);
  if (st != TFX_OK) return st;
  if (update == nullptr)
    return fail(TFX_ERR_INVALID_ARGUMENT, "tfx_residual_layer_norm: null update");
  if (!aligned(update, 8) || (residual_out && !aligned(residual_out, 16)))
    return fail(TFX_ERR_MISALIGNED, "tfx_residual_layer_norm: misaligned update/residual_out");
  return launch_residual_layer_norm(residual, reinterpret_cast<const __half*>(update), gamma, beta,
                                    residual_out, y, y_dtype, rows, d, eps, apply_affine,
                                    reinterpret_cast<cudaStream_t>(stream));
}

int tfx_linear(const tfx_half* a, const tfx_half* w, const float* bias, const float* residual,
               void* out, int64_t m, int n, int k, int epilogue, tfx_stream_t stream) {
  g_msg[0] = 0;
  if (a == nullptr || w == nullptr || bias == nullptr || out == nullptr)
    return fail(TFX_ERR_INVALID_ARGUMENT, "tfx_linear: null tensor");
  if (m <= 0 || n <= 0 || k <= 0)
    return fail(TFX_ERR_INVALID_ARGUMENT, "tfx_linear: sizes must be positive");
  if (m > 0x7fffffffLL - 128)
    return fail(TFX_ERR_UNSUPPORTED, "tfx_linear: m=%lld exceeds 2^31-129 rows", (long long)m);
  if (epilogue == TFX_EPI_BIAS_RESIDUAL && residual == nullptr)
    return fail(TFX_ERR_INVALID_ARGUMENT, "tfx_linear: residual epilogue needs a residual");
  if (k % 8 != 0 || n % 32 != 0)
    return fail(TFX_ERR_UNSUPPORTED, "tfx_linear: need k %% 8 == 0 and n %% 32 == 0 (k=%d n=%d)",
                k, n);
  if (!aligned(a, 16) || !aligned(w, 16) || !aligned(bias, 16) || !aligned(out, 16) ||
      (residual && !aligned(residual, 16)))
    return fail(TFX_ERR_MISALIGNED, "tfx_linear: pointers must be 16-byte aligned");
  return launch_linear(reinterpret_cast<const __half*>(a), k,
                       reinterpret_cast<const __half*>(w), bias, residual, n, out, n, m, n, k,
                       epilogue, reinterpret_cast<cudaStream_t>(stream));
}

int tfx_attention_masked(const tfx_half* q, const tfx_half* k, const tfx_half* v,
                         int64_t ld_qkv, tfx_half* out, int64_t ld_out, int batch, int heads,
                         int seq, int head_dim, float scale, int causal, const uint32_t* key_mask,
                         tfx_stream_t stream) {
  g_msg[0] = 0;
  if (key_mask == nullptr)
    return fail(TFX_ERR_INVALID_ARGUMENT, "tfx_attention_masked: null key_mask");
  if (!aligned(key_mask, 4))
    return fail(TFX_ERR_MISALIGNED, "tfx_attention_masked: key_mask must be 4-byte aligned");
  return attention_checked("tfx_attention_masked", q, k, v, ld_qkv, out, ld_out, batch, heads,
                           seq, head_dim, scale, causal, KeyMask{nullptr, key_mask},
                           reinterpret_cast<cudaStream_t>(stream));
}

int tfx_attention(const tfx_half* q, const tfx_half* k, const tfx_half* v, int64_t ld_qkv,
                  tfx_half* out, int64_t ld_out, int batch, int heads, int seq, int head_dim,
                  float scale, int causal, const int32_t* valid_len, tfx_stream_t stream) {
  g_msg[0] = 0;
  return attention_checked("tfx_attention", q, k, v, ld_qkv, out, ld_out, batch, heads, seq,
                           head_dim, scale, causal, KeyMask{valid_len, nullptr},
                           reinterpret_cast<cudaStream_t>(stream));
}

int64_t tfx_attention_vt_ld(int seq) { return seq > 0 ? attention_vt_ld(seq) : -1; }

int tfx_transpose_v(const tfx_half* v, int64_t ld_qkv, tfx_half* vt, int batch, int seq, int cols,
                    tfx_stream_t stream) {
  g_msg[0] = 0;
  if (v == nullptr || vt == nullptr) return fail(TFX_ERR_INVALID_ARGUMENT, "tfx_transpose_v: null tensor");
  if (batch <= 0 || seq <= 0 || cols <= 0 || ld_qkv < cols)
    return fail(TFX_ERR_INVALID_ARGUMENT, "tfx_transpose_v: bad sizes");
  if (cols % 64 != 0 || batch > 65535 || (cols / 64) > 65535)
    return fail(TFX_ERR_UNSUPPORTED, "tfx_transpose_v: cols must be a multiple of 64");
  if (!aligned(v, 16) || !aligned(vt, 16) || ld_qkv % 8 != 0)
    return fail(TFX_ERR_MISALIGNED, "tfx_transpose_v: 16-byte aligned pointers, ld_qkv %% 8 == 0");
  return launch_transpose_v(reinterpret_cast<const __half*>(v), ld_qkv,
                            reinterpret_cast<__half*>(vt), batch, seq, cols,
                            reinterpret_cast<cudaStream_t>(stream));
}

int tfx_attention_vt(const tfx_half* q, const tfx_half* k, const tfx_half* vt, int64_t ld_qkv,
                     tfx_half* out, int64_t ld_out, int batch, int heads, int seq, int head_dim,
                     float scale, int causal, const int32_t* valid_len, tfx_stream_t stream) {
  g_msg[0] = 0;
  if (q == nullptr || k == nullptr || vt == nullptr || out == nullptr)
    return fail(TFX_ERR_INVALID_ARGUMENT, "tfx_attention_vt: null tensor");
  if (batch <= 0 || heads <= 0 || seq <= 0 || head_dim <= 0)
    return fail(TFX_ERR_INVALID_ARGUMENT, "tfx_attention_vt: sizes must be positive");
  if (!attention_tc_supported(head_dim, scale))
    return fail(TFX_ERR_UNSUPPORTED, "tfx_attention_vt: head_dim %d not in {64,128,256} or scale <= 0",
                head_dim);
  if (heads > 65535 || batch > 65535)
    return fail(TFX_ERR_UNSUPPORTED, "tfx_attention_vt: batch and heads must be <= 65535");
  if (ld_qkv < static_cast<int64_t>(heads) * head_dim ||
      ld_out < static_cast<int64_t>(heads) * head_dim)
    return fail(TFX_ERR_INVALID_ARGUMENT, "tfx_attention_vt: leading dimension smaller than H*hd");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(vt, 16) || !aligned(out, 16) ||
      ld_qkv % 8 != 0 || ld_out % 8 != 0)
    return fail(TFX_ERR_MISALIGNED,
                "tfx_attention_vt: pointers 16-byte aligned and leading dims multiples of 8 needed");
  return launch_attention_tc_vt(reinterpret_cast<const __half*>(q),
                                reinterpret_cast<const __half*>(k),
                                reinterpret_cast<const __half*>(vt), ld_qkv,
                                reinterpret_cast<__half*>(out), ld_out, batch, heads, seq,
                                head_dim, scale, causal, KeyMask{valid_len, nullptr},
                                reinterpret_cast<cudaStream_t>(stream));
}

int tfx_read_device_error(int* code) {
  g_msg[0] = 0;
  if (code == nullptr) return fail(TFX_ERR_INVALID_ARGUMENT, "tfx_read_device_error: null code");
  int* word = device_error_word();
  if (word == nullptr) return fail(TFX_ERR_CUDA, "device error word unavailable");
  int host = 0;
  cudaError_t e = cudaMemcpy(&host, word, sizeof(int), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemset(word, 0, sizeof(int));
  if (e != cudaSuccess) return fail(TFX_ERR_CUDA, "tfx_read_device_error: %s", cudaGetErrorString(e));
  *code = host;
  return TFX_OK;
}

}  // extern "C"
