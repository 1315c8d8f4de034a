// LayerNorm and fused residual-add + LayerNorm (HBM-bound).
//
// One warp per row. Lane l owns the float4 columns {4*(l + 32*i)}, so every
// warp-wide load/store instruction moves 512 contiguous bytes (fully
// coalesced 128-bit accesses). Mean and the centred variance are reduced
// with warp shuffles in fp32; the whole row stays in registers, so the input
// is read exactly once. Output is fp16 (feeding the next tensor-core GEMM) or
// fp32 (the model's final output).
#include "internal.h"
#include "ptx.cuh"

namespace tfx {
namespace {

constexpr int kRowsPerBlock = 8;  // 8 warps

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename OutT>
__device__ __forceinline__ void store4(OutT* y, float a, float b, float c, float d);

template <>
__device__ __forceinline__ void store4<float>(float* y, float a, float b, float c, float d) {
  *reinterpret_cast<float4*>(y) = make_float4(a, b, c, d);
}

template <>
__device__ __forceinline__ void store4<__half>(__half* y, float a, float b, float c, float d) {
  *reinterpret_cast<uint2*>(y) = make_uint2(pack_half2(a, b), pack_half2(c, d));
}

// NV = float4 chunks per lane = ceil(D / 128). HAS_UPDATE: residual variant.
template <int NV, bool HAS_UPDATE, typename OutT>
__global__ void __launch_bounds__(32 * kRowsPerBlock)
    layer_norm_kernel(const float* x, const __half* __restrict__ update,
                      const float* __restrict__ gamma, const float* __restrict__ beta,
                      float* residual_out, OutT* __restrict__ y, int64_t rows, int d, float eps,
                      int apply_affine) {
  grid_dep_wait();
  grid_dep_launch();
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kRowsPerBlock + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* xr = x + row * d;
  float4 v[NV];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int col = 4 * (lane + 32 * i);
    if (col < d) {
      v[i] = __ldcs(reinterpret_cast<const float4*>(xr + col));
      if constexpr (HAS_UPDATE) {
        const uint2 u = __ldcs(reinterpret_cast<const uint2*>(update + row * d + col));
        const float2 u01 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
        const float2 u23 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
        v[i].x += u01.x;
        v[i].y += u01.y;
        v[i].z += u23.x;
        v[i].w += u23.y;
        if (residual_out != nullptr)
          *reinterpret_cast<float4*>(residual_out + row * d + col) = v[i];
      }
    } else {
      v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  }
  const float mean = warp_sum(sum) / static_cast<float>(d);
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int col = 4 * (lane + 32 * i);
    if (col < d) {
      const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, e = v[i].w - mean;
      sq += (a * a + b * b) + (c * c + e * e);
    }
  }
  const float rstd = rsqrtf(warp_sum(sq) / static_cast<float>(d) + eps);
  OutT* yr = y + row * d;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int col = 4 * (lane + 32 * i);
    if (col < d) {
      float a = (v[i].x - mean) * rstd, b = (v[i].y - mean) * rstd;
      float c = (v[i].z - mean) * rstd, e = (v[i].w - mean) * rstd;
      if (apply_affine) {
        const float4 g = __ldg(reinterpret_cast<const float4*>(gamma + col));
        const float4 bb = __ldg(reinterpret_cast<const float4*>(beta + col));
        a = a * g.x + bb.x;
        b = b * g.y + bb.y;
        c = c * g.z + bb.z;
        e = e * g.w + bb.w;
      }
      store4<OutT>(yr + col, a, b, c, e);
    }
  }
}

template <int NV, bool HAS_UPDATE>
int launch_nv(const float* x, const __half* u, const float* gamma, const float* beta, float* r_out,
              void* y, int y_dtype, int64_t rows, int d, float eps, int affine,
              cudaStream_t stream) {
  const int64_t blocks = (rows + kRowsPerBlock - 1) / kRowsPerBlock;
  if (y_dtype == TFX_DTYPE_F16) {
    launch_pdl(layer_norm_kernel<NV, HAS_UPDATE, __half>, dim3(static_cast<unsigned>(blocks)),
               dim3(32 * kRowsPerBlock), 0, stream, x, u, gamma, beta, r_out,
               static_cast<__half*>(y), rows, d, eps, affine);
  } else {
    launch_pdl(layer_norm_kernel<NV, HAS_UPDATE, float>, dim3(static_cast<unsigned>(blocks)),
               dim3(32 * kRowsPerBlock), 0, stream, x, u, gamma, beta, r_out,
               static_cast<float*>(y), rows, d, eps, affine);
  }
  return check_launch("layer_norm_kernel");
}

template <bool HAS_UPDATE>
int dispatch(const float* x, const __half* u, const float* gamma, const float* beta, float* r_out,
             void* y, int y_dtype, int64_t rows, int d, float eps, int affine,
             cudaStream_t stream) {
  const int nv = (d + 127) / 128;
#define TFX_LN_CASE(N) \
  case N:              \
    return launch_nv<N, HAS_UPDATE>(x, u, gamma, beta, r_out, y, y_dtype, rows, d, eps, affine, stream);
  switch (nv) {
    TFX_LN_CASE(1)
    TFX_LN_CASE(2)
    TFX_LN_CASE(3)
    TFX_LN_CASE(4)
    TFX_LN_CASE(5)
    TFX_LN_CASE(6)
    TFX_LN_CASE(7)
    TFX_LN_CASE(8)
    default:
      break;
  }
#undef TFX_LN_CASE
  if (nv <= 16)
    return launch_nv<16, HAS_UPDATE>(x, u, gamma, beta, r_out, y, y_dtype, rows, d, eps, affine,
                                     stream);
  return launch_nv<32, HAS_UPDATE>(x, u, gamma, beta, r_out, y, y_dtype, rows, d, eps, affine,
                                   stream);
}

}  // namespace

int launch_layer_norm(const float* x, const float* gamma, const float* beta, void* y, int y_dtype,
                      int64_t rows, int d, float eps, int apply_affine, cudaStream_t stream) {
  return dispatch<false>(x, nullptr, gamma, beta, nullptr, y, y_dtype, rows, d, eps, apply_affine,
                         stream);
}

int launch_residual_layer_norm(const float* r, const __half* u, const float* gamma,
                               const float* beta, float* r_out, void* y, int y_dtype,
                               int64_t rows, int d, float eps, int apply_affine,
                               cudaStream_t stream) {
  return dispatch<true>(r, u, gamma, beta, r_out, y, y_dtype, rows, d, eps, apply_affine, stream);
}

}  // namespace tfx
