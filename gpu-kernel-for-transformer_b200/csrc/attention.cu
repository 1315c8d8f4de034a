// Flash-style multi-head attention (causal or not, optional key padding).
//
// CTA = 4 warps = 64 query rows of one (batch, head). K/V tiles of BKV keys
// stream through a cp.async double buffer in shared memory; each warp owns
// 16 query rows and keeps its O accumulator and the online-softmax state
// (running max m, running sum l, fp32) in registers, so the S x S matrix is
// never materialised. Scores are computed in the log2 domain
// (scale * log2(e) folded in) and exponentiated with exp2f.
//
// Head dims 8 and 16 pad the QK^T reduction to the 16-wide MMA K: the pad
// columns of the Q and K tiles are zero-filled once, so they add nothing.
// Causal CTAs are launched heaviest-first (last query block first).
#include "internal.h"
#include "ptx.cuh"

namespace tfx {
namespace {

constexpr int kBQ = 64;
constexpr int kAttnThreads = 128;

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // zero-fill when the source row is out of range
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(addr));
}
// D(16x8, f32) += A(16x16, f16, row) * B(16x8, f16, col)
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int HD>
struct AttnCfg {
  static constexpr int kHDP = HD < 16 ? 16 : HD;        // QK^T reduction width
  static constexpr int kBKV = HD >= 256 ? 32 : 64;       // keys per tile
  static constexpr int kQStride = kHDP + 8;              // +16 B: conflict-free ldmatrix
  static constexpr int kKStride = kHDP + 8;
  static constexpr int kVStride = (HD < 16 ? 16 : HD) + 8;
  static constexpr int kQElems = kBQ * kQStride;
  static constexpr int kKElems = kBKV * kKStride;
  static constexpr int kVElems = kBKV * kVStride;
  static constexpr int kSmemBytes = 2 * (kQElems + 2 * kKElems + 2 * kVElems);
};

template <int HD, bool CAUSAL>
__global__ void __launch_bounds__(kAttnThreads)
    attention_mma_kernel(const __half* __restrict__ q, int64_t ld_q, const __half* __restrict__ k,
                         const __half* __restrict__ v, AttnKv kv, __half* __restrict__ out,
                         int64_t ld_out, int heads, int q_len, float scale_log2,
                         const int32_t* __restrict__ valid_len) {
  grid_dep_wait();
  grid_dep_launch();
  using C = AttnCfg<HD>;
  constexpr int HDP = C::kHDP, BKV = C::kBKV;
  constexpr int NT_S = BKV / 8;  // score n-tiles per warp
  constexpr int NT_O = HD / 8;   // output n-tiles (HD >= 8)
  extern __shared__ __align__(16) __half smem_attn[];
  __half* sQ = smem_attn;
  __half* sK = sQ + C::kQElems;      // 2 buffers
  __half* sV = sK + 2 * C::kKElems;  // 2 buffers

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nqb = (q_len + kBQ - 1) / kBQ;
  const int qb = CAUSAL ? (nqb - 1 - static_cast<int>(blockIdx.x)) : static_cast<int>(blockIdx.x);
  const int h = blockIdx.y, b = blockIdx.z;
  const int q0 = qb * kBQ;
  const int64_t row0 = static_cast<int64_t>(b) * q_len;      // queries and outputs
  const int64_t kv_row0 = static_cast<int64_t>(b) * kv.batch_rows;
  // Query row i sits at key position kv.q_off + i; causal rows see keys up to it.
  const int klen = valid_len ? min(kv.len, max(0, valid_len[b])) : kv.len;
  int kend = CAUSAL ? min(klen, kv.q_off + q0 + kBQ) : klen;
  const int nkb = (kend + BKV - 1) / BKV;

  // Zero the reduction padding columns once (HD < 16 only).
  if constexpr (HD < 16) {
    for (int i = tid; i < kBQ; i += kAttnThreads)
      *reinterpret_cast<uint4*>(sQ + i * C::kQStride + HD) = make_uint4(0, 0, 0, 0);
    for (int i = tid; i < 2 * BKV; i += kAttnThreads)
      *reinterpret_cast<uint4*>(sK + i * C::kKStride + HD) = make_uint4(0, 0, 0, 0);
  }

  constexpr int CH = HD / 8;  // 16-byte chunks per row
  // Q tile.
  for (int i = tid; i < kBQ * CH; i += kAttnThreads) {
    const int r = i / CH, c = i % CH;
    const int qi = q0 + r;
    const bool ok = qi < q_len;
    const __half* src = q + (row0 + (ok ? qi : 0)) * ld_q + h * HD + c * 8;
    cp_async16(smem_u32(sQ + r * C::kQStride + c * 8), src, ok);
  }
  auto load_kv = [&](int kb, int buf) {
    const int k0 = kb * BKV;
    for (int i = tid; i < BKV * CH; i += kAttnThreads) {
      const int r = i / CH, c = i % CH;
      const int ki = k0 + r;
      const bool ok = ki < kend;
      const int64_t off = (kv_row0 + (ok ? ki : 0)) * kv.ld + h * HD + c * 8;
      cp_async16(smem_u32(sK + buf * C::kKElems + r * C::kKStride + c * 8), k + off, ok);
      cp_async16(smem_u32(sV + buf * C::kVElems + r * C::kVStride + c * 8), v + off, ok);
    }
  };
  if (nkb > 0) load_kv(0, 0);
  cp_async_commit();

  float o[NT_O][4];
#pragma unroll
  for (int i = 0; i < NT_O; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.f, 0.f};
  const int g = lane >> 2, t = lane & 3;
  const int qrow_a = q0 + warp * 16 + g;  // rows owned: qrow_a and qrow_a + 8
  const int qpos_a = kv.q_off + qrow_a;   // their key positions

  for (int kb = 0; kb < nkb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < nkb) load_kv(kb + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();

    const __half* cK = sK + buf * C::kKElems;
    const __half* cV = sV + buf * C::kVElems;
    // ---- S = Q K^T (16 x BKV per warp)
    float s[NT_S][4];
#pragma unroll
    for (int j = 0; j < NT_S; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HDP / 16; ++kk) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4(smem_u32(sQ + (warp * 16 + (lane & 15)) * C::kQStride + kk * 16 + (lane >> 4) * 8),
              a0, a1, a2, a3);
#pragma unroll
      for (int j = 0; j < NT_S; j += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(smem_u32(cK + (j * 8 + (lane >> 4) * 8 + (lane & 7)) * C::kKStride + kk * 16 +
                         ((lane >> 3) & 1) * 8),
                b0, b1, b2, b3);
        mma16816(s[j], a0, a1, a2, a3, b0, b1);
        mma16816(s[j + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    // ---- mask + online softmax (log2 domain)
    const int k0 = kb * BKV;
    const bool need_mask =
        (k0 + BKV > kend) || (CAUSAL && k0 + BKV - 1 > kv.q_off + q0 + warp * 16);
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < NT_S; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float val = s[j][e] * scale_log2;
        if (need_mask) {
          const int key = k0 + j * 8 + 2 * t + (e & 1);
          const int qr = qpos_a + (e >> 1) * 8;
          if (key >= kend || (CAUSAL && key > qr)) val = -INFINITY;
        }
        s[j][e] = val;
        mx[e >> 1] = fmaxf(mx[e >> 1], val);
      }
    }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float m_new = fmaxf(m_run[r], mx[r]);
      // A row with every key so far masked keeps m = -inf; use 0 as the
      // reference so exp2 sees -inf - 0 = -inf (weight 0), never NaN.
      const float m_ref = (m_new == -INFINITY) ? 0.f : m_new;
      corr[r] = exp2f(m_run[r] - m_ref);
      m_run[r] = m_new;
      mx[r] = m_ref;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < NT_S; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float p = exp2f(s[j][e] - mx[e >> 1]);
        s[j][e] = p;
        rs[e >> 1] += p;
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) l_run[r] = l_run[r] * corr[r] + rs[r];
#pragma unroll
    for (int i = 0; i < NT_O; ++i) {
      o[i][0] *= corr[0];
      o[i][1] *= corr[0];
      o[i][2] *= corr[1];
      o[i][3] *= corr[1];
    }
    // ---- O += P V
#pragma unroll
    for (int kk = 0; kk < BKV / 16; ++kk) {
      const uint32_t a0 = pack_half2(s[2 * kk][0], s[2 * kk][1]);
      const uint32_t a1 = pack_half2(s[2 * kk][2], s[2 * kk][3]);
      const uint32_t a2 = pack_half2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      const uint32_t a3 = pack_half2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
      if constexpr (NT_O == 1) {
        uint32_t b0, b1;
        ldsm_x2_t(smem_u32(cV + (kk * 16 + (lane & 15)) * C::kVStride), b0, b1);
        mma16816(o[0], a0, a1, a2, a3, b0, b1);
      } else {
#pragma unroll
        for (int i = 0; i < NT_O; i += 2) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(smem_u32(cV + (kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * C::kVStride +
                             i * 8 + (lane >> 4) * 8),
                    b0, b1, b2, b3);
          mma16816(o[i], a0, a1, a2, a3, b0, b1);
          mma16816(o[i + 1], a0, a1, a2, a3, b2, b3);
        }
      }
    }
    __syncthreads();  // buffer `buf` is refilled by the next iteration's prefetch
  }
  cp_async_wait<0>();

  // ---- finalise: O / l, fp16 store
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
  }
  const float inv0 = l_run[0] > 0.f ? 1.f / l_run[0] : 0.f;
  const float inv1 = l_run[1] > 0.f ? 1.f / l_run[1] : 0.f;
#pragma unroll
  for (int i = 0; i < NT_O; ++i) {
    const int col = h * HD + i * 8 + 2 * t;
    if (qrow_a < q_len)
      *reinterpret_cast<uint32_t*>(out + (row0 + qrow_a) * ld_out + col) =
          pack_half2(o[i][0] * inv0, o[i][1] * inv0);
    if (qrow_a + 8 < q_len)
      *reinterpret_cast<uint32_t*>(out + (row0 + qrow_a + 8) * ld_out + col) =
          pack_half2(o[i][2] * inv1, o[i][3] * inv1);
  }
}

template <int HD>
int launch_hd(const __half* q, int64_t ld_q, const __half* k, const __half* v, const AttnKv& kv,
              __half* out, int64_t ld_out, int batch, int heads, int q_len, float scale,
              int causal, const int32_t* valid_len, cudaStream_t stream) {
  using C = AttnCfg<HD>;
  static int done_c[kMaxDevices] = {0};
  static int done_n[kMaxDevices] = {0};
  const float scale_log2 = scale * 1.4426950408889634f;
  dim3 grid((q_len + kBQ - 1) / kBQ, heads, batch);
  if (causal) {
    auto kern = attention_mma_kernel<HD, true>;
    int st = ensure_smem(reinterpret_cast<const void*>(kern), C::kSmemBytes, done_c);
    if (st != TFX_OK) return st;
    launch_pdl(kern, grid, dim3(kAttnThreads), C::kSmemBytes, stream, q, ld_q, k, v, kv, out,
               ld_out, heads, q_len, scale_log2, valid_len);
  } else {
    auto kern = attention_mma_kernel<HD, false>;
    int st = ensure_smem(reinterpret_cast<const void*>(kern), C::kSmemBytes, done_n);
    if (st != TFX_OK) return st;
    launch_pdl(kern, grid, dim3(kAttnThreads), C::kSmemBytes, stream, q, ld_q, k, v, kv, out,
               ld_out, heads, q_len, scale_log2, valid_len);
  }
  return check_launch("attention_mma_kernel");
}

int launch_mma(const __half* q, int64_t ld_q, const __half* k, const __half* v, const AttnKv& kv,
               __half* out, int64_t ld_out, int batch, int heads, int q_len, int head_dim,
               float scale, int causal, const int32_t* valid_len, cudaStream_t stream) {
  switch (head_dim) {
    case 8:
      return launch_hd<8>(q, ld_q, k, v, kv, out, ld_out, batch, heads, q_len, scale, causal,
                          valid_len, stream);
    case 16:
      return launch_hd<16>(q, ld_q, k, v, kv, out, ld_out, batch, heads, q_len, scale, causal,
                           valid_len, stream);
    case 32:
      return launch_hd<32>(q, ld_q, k, v, kv, out, ld_out, batch, heads, q_len, scale, causal,
                           valid_len, stream);
    case 64:
      return launch_hd<64>(q, ld_q, k, v, kv, out, ld_out, batch, heads, q_len, scale, causal,
                           valid_len, stream);
    case 128:
      return launch_hd<128>(q, ld_q, k, v, kv, out, ld_out, batch, heads, q_len, scale, causal,
                            valid_len, stream);
    case 256:
      return launch_hd<256>(q, ld_q, k, v, kv, out, ld_out, batch, heads, q_len, scale, causal,
                            valid_len, stream);
    default:
      return fail(TFX_ERR_UNSUPPORTED, "tfx_attention: head_dim %d not in {8,16,32,64,128,256}",
                  head_dim);
  }
}

}  // namespace

int launch_attention(const __half* q, const __half* k, const __half* v, int64_t ld_qkv,
                     __half* out, int64_t ld_out, int batch, int heads, int seq, int head_dim,
                     float scale, int causal, const int32_t* valid_len, cudaStream_t stream) {
  // Head dims 64, 128 and 256 run on the tcgen05 kernel (attention_tc.cu).
  if (attention_tc_supported(head_dim, scale))
    return launch_attention_tc(q, k, v, ld_qkv, out, ld_out, batch, heads, seq, head_dim, scale,
                               causal, valid_len, stream);
  return launch_mma(q, ld_qkv, k, v, AttnKv{ld_qkv, seq, seq, 0}, out, ld_out, batch, heads, seq,
                    head_dim, scale, causal, valid_len, stream);
}

int launch_attention_kv(const __half* q, int64_t ld_q, const __half* k, const __half* v,
                        const AttnKv& kv, __half* out, int64_t ld_out, int batch, int heads,
                        int q_len, int head_dim, float scale, cudaStream_t stream) {
  if (attention_tc_supported(head_dim, scale))
    return launch_attention_tc_kv(q, ld_q, k, v, kv, out, ld_out, batch, heads, q_len, head_dim,
                                  scale, stream);
  return launch_mma(q, ld_q, k, v, kv, out, ld_out, batch, heads, q_len, head_dim, scale, 1,
                    nullptr, stream);
}

}  // namespace tfx
