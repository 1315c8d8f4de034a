// LayerNorm and fused residual-add + LayerNorm (HBM-bound).
//
// One warp per row (up to four rows per warp for d <= 256, loaded together).
// Lane l owns the float4 columns {4*(l + 32*i)}, so every warp-wide
// load/store instruction moves 512 contiguous bytes (fully coalesced 128-bit
// accesses). Mean and the centred variance are reduced
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

// NV = float4 chunks per lane = ceil(D / 128); RPW rows per warp, all their
// loads issued before the first reduction (narrow rows: more bytes in flight
// per warp). HAS_UPDATE: residual variant.
template <int NV, int RPW, bool HAS_UPDATE, typename OutT>
__global__ void __launch_bounds__(32 * kRowsPerBlock)
    layer_norm_kernel(const float* x, const __half* __restrict__ update,
                      const float* __restrict__ gamma, const float* __restrict__ beta,
                      float* residual_out, OutT* __restrict__ y, int64_t rows, int d, float eps,
                      int apply_affine) {
  grid_dep_wait();
  grid_dep_launch();
  const int lane = threadIdx.x & 31;
  const int64_t row0 =
      (static_cast<int64_t>(blockIdx.x) * kRowsPerBlock + (threadIdx.x >> 5)) * RPW;
  if (row0 >= rows) return;  // warp-uniform
  float4 v[RPW][NV];
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const int64_t row = row0 + r;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int col = 4 * (lane + 32 * i);
      v[r][i] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (row < rows && col < d) {
        v[r][i] = __ldcs(reinterpret_cast<const float4*>(x + row * d + col));
        if constexpr (HAS_UPDATE) {
          const uint2 u = __ldcs(reinterpret_cast<const uint2*>(update + row * d + col));
          const float2 u01 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
          const float2 u23 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
          v[r][i].x += u01.x;
          v[r][i].y += u01.y;
          v[r][i].z += u23.x;
          v[r][i].w += u23.y;
          if (residual_out != nullptr)
            *reinterpret_cast<float4*>(residual_out + row * d + col) = v[r][i];
        }
      }
    }
  }
  float mean[RPW], rstd[RPW];
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) sum += (v[r][i].x + v[r][i].y) + (v[r][i].z + v[r][i].w);
    mean[r] = warp_sum(sum) / static_cast<float>(d);
  }
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    float sq = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int col = 4 * (lane + 32 * i);
      if (col < d) {
        const float a = v[r][i].x - mean[r], b = v[r][i].y - mean[r];
        const float c = v[r][i].z - mean[r], e = v[r][i].w - mean[r];
        sq += (a * a + b * b) + (c * c + e * e);
      }
    }
    rstd[r] = rsqrtf(warp_sum(sq) / static_cast<float>(d) + eps);
  }
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int col = 4 * (lane + 32 * i);
    if (col >= d) continue;
    float4 g = make_float4(1.f, 1.f, 1.f, 1.f), bb = make_float4(0.f, 0.f, 0.f, 0.f);
    if (apply_affine) {
      g = __ldg(reinterpret_cast<const float4*>(gamma + col));
      bb = __ldg(reinterpret_cast<const float4*>(beta + col));
    }
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      if (row0 + r >= rows) break;
      const float a = (v[r][i].x - mean[r]) * rstd[r], b = (v[r][i].y - mean[r]) * rstd[r];
      const float c = (v[r][i].z - mean[r]) * rstd[r], e = (v[r][i].w - mean[r]) * rstd[r];
      store4<OutT>(y + (row0 + r) * d + col, a * g.x + bb.x, b * g.y + bb.y, c * g.z + bb.z,
                   e * g.w + bb.w);
    }
  }
}

template <int NV, int RPW, bool HAS_UPDATE>
int launch_rpw(const float* x, const __half* u, const float* gamma, const float* beta,
               float* r_out, void* y, int y_dtype, int64_t rows, int d, float eps, int affine,
               cudaStream_t stream) {
  const int64_t per_block = static_cast<int64_t>(kRowsPerBlock) * RPW;
  const int64_t blocks = (rows + per_block - 1) / per_block;
  if (y_dtype == TFX_DTYPE_F16) {
    launch_pdl(layer_norm_kernel<NV, RPW, HAS_UPDATE, __half>, dim3(static_cast<unsigned>(blocks)),
               dim3(32 * kRowsPerBlock), 0, stream, x, u, gamma, beta, r_out,
               static_cast<__half*>(y), rows, d, eps, affine);
  } else {
    launch_pdl(layer_norm_kernel<NV, RPW, HAS_UPDATE, float>, dim3(static_cast<unsigned>(blocks)),
               dim3(32 * kRowsPerBlock), 0, stream, x, u, gamma, beta, r_out,
               static_cast<float*>(y), rows, d, eps, affine);
  }
  return check_launch("layer_norm_kernel");
}

// Rows per warp: 4 at d <= 128 and 2 at d <= 256 (16 or 32 floats in flight
// per lane) when there are enough rows to keep every SM full of warps that
// way (c2's 1.28M rows: 45.4 -> 37.3 us, 0.68 -> 0.82 of the measured HBM
// bandwidth); small inputs (8192 rows) keep one row per warp, whose 4x more
// warps cover the latency better.
template <int NV, bool HAS_UPDATE>
int launch_nv(const float* x, const __half* u, const float* gamma, const float* beta, float* r_out,
              void* y, int y_dtype, int64_t rows, int d, float eps, int affine,
              cudaStream_t stream) {
  constexpr int kMulti = NV == 1 ? 4 : (NV == 2 ? 2 : 1);
  if (kMulti > 1 && rows >= static_cast<int64_t>(num_sms()) * 64 * kMulti)
    return launch_rpw<NV, kMulti, HAS_UPDATE>(x, u, gamma, beta, r_out, y, y_dtype, rows, d, eps,
                                              affine, stream);
  return launch_rpw<NV, 1, HAS_UPDATE>(x, u, gamma, beta, r_out, y, y_dtype, rows, d, eps, affine,
                                       stream);
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
