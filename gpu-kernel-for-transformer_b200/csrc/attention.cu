// Flash-style multi-head attention (causal or not, optional key padding).
//
// CTA = 4 warps = 64 query rows of one (batch, head). K/V tiles of BKV keys
// stream through a cp.async double buffer in shared memory; each warp owns
// 16 query rows and keeps its O accumulator and the online-softmax state
// (running max m, running sum l, fp32) in registers, so the S x S matrix is
// never materialised. Scores are computed in the log2 domain
// (scale * log2(e) folded in) and exponentiated with exp2f.
//
// Key padding: prefix lengths (valid_len) or a key bitmask of any pattern.
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
                         const int32_t* __restrict__ valid_len,
                         const uint32_t* __restrict__ key_bits, int key_words) {
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
    // Key bitmask (any padding pattern): the BKV bits of this tile, the
    // same for every row (uniform loads).
    uint32_t kw[BKV / 32];
    bool bits_full = true;
#pragma unroll
    for (int w = 0; w < BKV / 32; ++w) {
      const int wi = k0 / 32 + w;
      kw[w] = (key_bits == nullptr) ? 0xffffffffu
              : (wi < key_words ? key_bits[static_cast<int64_t>(b) * key_words + wi] : 0u);
      bits_full = bits_full && kw[w] == 0xffffffffu;
    }
    const bool need_mask = !bits_full || (k0 + BKV > kend) ||
                           (CAUSAL && k0 + BKV - 1 > kv.q_off + q0 + warp * 16);
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < NT_S; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float val = s[j][e] * scale_log2;
        if (need_mask) {
          const int kk = j * 8 + 2 * t + (e & 1);  // key within the tile
          const int key = k0 + kk;
          const int qr = qpos_a + (e >> 1) * 8;
          if (key >= kend || (CAUSAL && key > qr) || !((kw[kk >> 5] >> (kk & 31)) & 1u))
            val = -INFINITY;
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
              int causal, const KeyMask& km, cudaStream_t stream) {
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
               ld_out, heads, q_len, scale_log2, km.len, km.bits, key_words(kv.len));
  } else {
    auto kern = attention_mma_kernel<HD, false>;
    int st = ensure_smem(reinterpret_cast<const void*>(kern), C::kSmemBytes, done_n);
    if (st != TFX_OK) return st;
    launch_pdl(kern, grid, dim3(kAttnThreads), C::kSmemBytes, stream, q, ld_q, k, v, kv, out,
               ld_out, heads, q_len, scale_log2, km.len, km.bits, key_words(kv.len));
  }
  return check_launch("attention_mma_kernel");
}

int launch_mma(const __half* q, int64_t ld_q, const __half* k, const __half* v, const AttnKv& kv,
               __half* out, int64_t ld_out, int batch, int heads, int q_len, int head_dim,
               float scale, int causal, const KeyMask& km, cudaStream_t stream) {
  switch (head_dim) {
    case 8:
      return launch_hd<8>(q, ld_q, k, v, kv, out, ld_out, batch, heads, q_len, scale, causal,
                          km, stream);
    case 16:
      return launch_hd<16>(q, ld_q, k, v, kv, out, ld_out, batch, heads, q_len, scale, causal,
                           km, stream);
    case 32:
      return launch_hd<32>(q, ld_q, k, v, kv, out, ld_out, batch, heads, q_len, scale, causal,
                           km, stream);
    case 64:
      return launch_hd<64>(q, ld_q, k, v, kv, out, ld_out, batch, heads, q_len, scale, causal,
                           km, stream);
    case 128:
      return launch_hd<128>(q, ld_q, k, v, kv, out, ld_out, batch, heads, q_len, scale, causal,
                            km, stream);
    case 256:
      return launch_hd<256>(q, ld_q, k, v, kv, out, ld_out, batch, heads, q_len, scale, causal,
                            km, stream);
    default:
      return fail(TFX_ERR_UNSUPPORTED, "tfx_attention: head_dim %d not in {8,16,32,64,128,256}",
                  head_dim);
  }
}

// ------------------------------------------------------------------ decode
// Split-KV attention for decode steps: q_len <= 16 new queries per sequence
// attending a KV cache of kv.len keys (query row i at key position
// kv.q_off + i, causal). The queries fit one 16-row MMA tile, so the work is
// reading the cache: each CTA streams one contiguous range of 64-key tiles
// of one (batch, head) through a cp.async double buffer, the 4 warps each
// take 16 keys of every tile with their own online-softmax state, merge in
// shared memory at the end, and write an unnormalised partial O with its
// row max and sum. attention_decode_combine_kernel merges the splits.
// Memory-bound at M <= 16: mma.sync products are a small share of each
// tile's time next to its 64 x HD x 4 bytes of K and V.
constexpr int kDecRows = 16;   // MMA rows: queries (rows >= q_len are padding)
constexpr int kDecBKV = 64;    // keys per tile, 16 per warp
constexpr int kDecThreads = 128;
constexpr int64_t kDecMaxCtas = 4096;  // bound on (batch*heads) x splits beyond batch*heads

// Floats of the partial-O block for `rows` (batch, head, split) rows, padded
// so the (max, sum) pairs after it stay 16-byte aligned.
inline int64_t decode_part_o_floats(int64_t rows, int q_len, int hd) {
  return (rows * q_len * hd + 3) / 4 * 4;
}

template <int HD>
struct DecCfg {
  static constexpr int kHDP = HD < 16 ? 16 : HD;  // QK^T reduction width (zero padded)
  static constexpr int kQStride = kHDP + 8;       // +16 B rows: conflict-free ldmatrix
  static constexpr int kKStride = kHDP + 8;
  static constexpr int kVStride = (HD < 16 ? 16 : HD) + 8;
  static constexpr int kQElems = kDecRows * kQStride;
  static constexpr int kKElems = kDecBKV * kKStride;
  static constexpr int kVElems = kDecBKV * kVStride;
  // head_dim 256 fits one CTA per SM: a third stage keeps two tiles in flight.
  static constexpr int kStages = HD >= 256 ? 3 : 2;
  static constexpr int kStageElems = kStages * (kKElems + kVElems);  // K and V stages
  static constexpr int kMergeBytes = 4 * kDecRows * (HD + 2) * 4;
  static constexpr int kSmemBytes =
      2 * kQElems + (2 * kStageElems > kMergeBytes ? 2 * kStageElems : kMergeBytes);
};

template <int HD>
__global__ void __launch_bounds__(kDecThreads)
    attention_decode_kernel(const __half* __restrict__ q, int64_t ld_q,
                            const __half* __restrict__ k, const __half* __restrict__ v, AttnKv kv,
                            int heads, int q_len, int tiles_per_split, float scale_log2,
                            float* __restrict__ part_o, float2* __restrict__ part_ml) {
  grid_dep_wait();
  grid_dep_launch();
  using C = DecCfg<HD>;
  constexpr int HDP = C::kHDP;
  constexpr int NT_O = HD / 8;  // output n-tiles
  constexpr int CH = HD / 8;    // 16-byte chunks per row
  constexpr int NS = C::kStages;
  extern __shared__ __align__(16) __half smem_dec[];
  __half* sQ = smem_dec;
  __half* sK = sQ + C::kQElems;         // NS stages
  __half* sV = sK + NS * C::kKElems;    // NS stages

  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int splits = gridDim.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kend = kv.len;
  const int kb0 = split * tiles_per_split;
  const int kb1 = min(kb0 + tiles_per_split, (kend + kDecBKV - 1) / kDecBKV);
  const int64_t kv_row0 = static_cast<int64_t>(b) * kv.batch_rows;

  if constexpr (HD < 16) {  // zero the reduction padding columns once
    for (int i = tid; i < kDecRows; i += kDecThreads)
      *reinterpret_cast<uint4*>(sQ + i * C::kQStride + HD) = make_uint4(0, 0, 0, 0);
    for (int i = tid; i < NS * kDecBKV; i += kDecThreads)
      *reinterpret_cast<uint4*>(sK + i * C::kKStride + HD) = make_uint4(0, 0, 0, 0);
  }
  for (int i = tid; i < kDecRows * CH; i += kDecThreads) {
    const int r = i / CH, c = i % CH;
    const bool ok = r < q_len;
    const __half* src = q + (static_cast<int64_t>(b) * q_len + (ok ? r : 0)) * ld_q + h * HD + c * 8;
    cp_async16(smem_u32(sQ + r * C::kQStride + c * 8), src, ok);
  }
  auto load_kv = [&](int kb, int stage) {
    const int k0 = kb * kDecBKV;
    for (int i = tid; i < kDecBKV * CH; i += kDecThreads) {
      const int r = i / CH, c = i % CH;
      const int key = k0 + r;
      const bool ok = key < kend;
      const int64_t off = (kv_row0 + (ok ? key : 0)) * kv.ld + h * HD + c * 8;
      cp_async16(smem_u32(sK + stage * C::kKElems + r * C::kKStride + c * 8), k + off, ok);
      cp_async16(smem_u32(sV + stage * C::kVElems + r * C::kVStride + c * 8), v + off, ok);
    }
  };
#pragma unroll
  for (int p = 0; p < NS - 1; ++p) {  // the Q group rides with the first tile's
    if (kb0 + p < kb1) load_kv(kb0 + p, p);
    cp_async_commit();
  }

  float o[NT_O][4];
#pragma unroll
  for (int i = 0; i < NT_O; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.f, 0.f};
  const int g = lane >> 2, t = lane & 3;

  for (int kb = kb0; kb < kb1; ++kb) {
    const int stage = (kb - kb0) % NS;
    // Refill the stage the previous iteration consumed (freed by its
    // closing barrier) with the tile NS - 1 ahead.
    if (kb + NS - 1 < kb1) load_kv(kb + NS - 1, (kb - kb0 + NS - 1) % NS);
    cp_async_commit();
    cp_async_wait<NS - 1>();
    __syncthreads();
    const __half* cK = sK + stage * C::kKElems;
    const __half* cV = sV + stage * C::kVElems;
    // S = Q K^T for this warp's 16 keys: two 16 x 8 fragments.
    float s[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HDP / 16; ++kk) {
      uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
      ldsm_x4(smem_u32(sQ + (lane & 15) * C::kQStride + kk * 16 + (lane >> 4) * 8), a0, a1, a2,
              a3);
      ldsm_x4(smem_u32(cK + (warp * 16 + (lane >> 4) * 8 + (lane & 7)) * C::kKStride + kk * 16 +
                       ((lane >> 3) & 1) * 8),
              b0, b1, b2, b3);
      mma16816(s[0], a0, a1, a2, a3, b0, b1);
      mma16816(s[1], a0, a1, a2, a3, b2, b3);
    }
    // Mask (cache end, causal limit of each query row) + online softmax.
    const int k0 = kb * kDecBKV + warp * 16;
    const bool need_mask = (k0 + 16 > kend) || (k0 + 15 > kv.q_off);
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float val = s[j][e] * scale_log2;
        if (need_mask) {
          const int key = k0 + j * 8 + 2 * t + (e & 1);
          const int qpos = kv.q_off + g + (e >> 1) * 8;
          if (key >= kend || key > qpos) val = -INFINITY;
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
      const float m_ref = (m_new == -INFINITY) ? 0.f : m_new;  // all masked: weights 0, no NaN
      corr[r] = exp2f(m_run[r] - m_ref);
      m_run[r] = m_new;
      mx[r] = m_ref;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
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
    // O += P V over this warp's 16 keys.
    const uint32_t a0 = pack_half2(s[0][0], s[0][1]);
    const uint32_t a1 = pack_half2(s[0][2], s[0][3]);
    const uint32_t a2 = pack_half2(s[1][0], s[1][1]);
    const uint32_t a3 = pack_half2(s[1][2], s[1][3]);
    if constexpr (NT_O == 1) {
      uint32_t b0, b1;
      ldsm_x2_t(smem_u32(cV + (warp * 16 + (lane & 15)) * C::kVStride), b0, b1);
      mma16816(o[0], a0, a1, a2, a3, b0, b1);
    } else {
#pragma unroll
      for (int i = 0; i < NT_O; i += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(smem_u32(cV + (warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * C::kVStride +
                           i * 8 + (lane >> 4) * 8),
                  b0, b1, b2, b3);
        mma16816(o[i], a0, a1, a2, a3, b0, b1);
        mma16816(o[i + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();  // stage `stage` is refilled by the next iteration's prefetch
  }
  cp_async_wait<0>();
  __syncthreads();

  // Merge the four warps' states through shared memory (over the K/V stages).
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
  }
  float* mo = reinterpret_cast<float*>(sK);  // [warp][row][HD]
  float* mm = mo + 4 * kDecRows * HD;       // [warp][row] running max
  float* ml = mm + 4 * kDecRows;            // [warp][row] running sum
#pragma unroll
  for (int i = 0; i < NT_O; ++i) {
    float* r0 = mo + (warp * kDecRows + g) * HD + i * 8 + 2 * t;
    r0[0] = o[i][0];
    r0[1] = o[i][1];
    r0[8 * HD] = o[i][2];
    r0[8 * HD + 1] = o[i][3];
  }
  if (t == 0) {
    mm[warp * kDecRows + g] = m_run[0];
    mm[warp * kDecRows + g + 8] = m_run[1];
    ml[warp * kDecRows + g] = l_run[0];
    ml[warp * kDecRows + g + 8] = l_run[1];
  }
  __syncthreads();
  const int64_t prow = (static_cast<int64_t>(b) * heads + h) * splits + split;
  for (int i = tid; i < q_len * HD; i += kDecThreads) {
    const int r = i / HD, d = i % HD;
    float m = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) m = fmaxf(m, mm[w * kDecRows + r]);
    float acc = 0.f, l = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float mw = mm[w * kDecRows + r];
      const float f = mw == -INFINITY ? 0.f : exp2f(mw - m);
      acc += f * mo[(w * kDecRows + r) * HD + d];
      l += f * ml[w * kDecRows + r];
    }
    part_o[(prow * q_len + r) * HD + d] = acc;
    if (d == 0) part_ml[prow * q_len + r] = make_float2(m, l);
  }
}

// ctx[b, t, h] = sum over splits of partial O scaled to the common max, / sum.
template <int HD>
__global__ void attention_decode_combine_kernel(const float* __restrict__ part_o,
                                                const float2* __restrict__ part_ml,
                                                __half* __restrict__ out, int64_t ld_out,
                                                int heads, int q_len, int splits) {
  grid_dep_wait();
  grid_dep_launch();
  const int t = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int64_t prow0 = (static_cast<int64_t>(b) * heads + h) * splits;
  float m = -INFINITY;
  for (int s = 0; s < splits; ++s) m = fmaxf(m, part_ml[(prow0 + s) * q_len + t].x);
  float acc = 0.f, l = 0.f;
  const int d = threadIdx.x;
  for (int s = 0; s < splits; ++s) {
    const float2 st = part_ml[(prow0 + s) * q_len + t];
    const float f = st.x == -INFINITY ? 0.f : exp2f(st.x - m);
    l += f * st.y;
    if (d < HD) acc += f * part_o[((prow0 + s) * q_len + t) * HD + d];
  }
  if (d < HD)
    out[(static_cast<int64_t>(b) * q_len + t) * ld_out + h * HD + d] =
        __float2half_rn(l > 0.f ? acc / l : 0.f);
}

// Splits per (batch, head): about four waves of CTAs over the SMs, at least
// four 64-key tiles per split, and at most kDecMaxCtas CTAs in all (the
// partial buffer's bound).
int decode_splits(int64_t bh, int kv_len, int smem_bytes, int* tiles_per_split) {
  const int tiles = (kv_len + kDecBKV - 1) / kDecBKV;
  int per_sm = 227 * 1024 / smem_bytes;
  per_sm = per_sm < 1 ? 1 : (per_sm > 16 ? 16 : per_sm);
  const int64_t want = (4LL * num_sms() * per_sm + bh - 1) / bh;
  int64_t splits = want;
  const int64_t cap_tiles = tiles / 4 > 0 ? tiles / 4 : 1;
  if (splits > cap_tiles) splits = cap_tiles;
  const int64_t cap_ctas = kDecMaxCtas / bh > 0 ? kDecMaxCtas / bh : 1;
  if (splits > cap_ctas) splits = cap_ctas;
  if (splits < 1) splits = 1;
  const int tps = static_cast<int>((tiles + splits - 1) / splits);
  *tiles_per_split = tps;
  return (tiles + tps - 1) / tps;
}

template <int HD>
int launch_decode_hd(const __half* q, int64_t ld_q, const __half* k, const __half* v,
                     const AttnKv& kv, __half* out, int64_t ld_out, int batch, int heads,
                     int q_len, float scale, float* part, cudaStream_t stream) {
  using C = DecCfg<HD>;
  static int done[kMaxDevices] = {0};
  auto kern = attention_decode_kernel<HD>;
  int st = ensure_smem(reinterpret_cast<const void*>(kern), C::kSmemBytes, done);
  if (st != TFX_OK) return st;
  const int64_t bh = static_cast<int64_t>(batch) * heads;
  int tps = 1;
  const int splits = decode_splits(bh, kv.len, C::kSmemBytes, &tps);
  float* part_o = part;
  float2* part_ml = reinterpret_cast<float2*>(part + decode_part_o_floats(bh * splits, q_len, HD));
  launch_pdl(kern, dim3(splits, heads, batch), dim3(kDecThreads), C::kSmemBytes, stream, q, ld_q,
             k, v, kv, heads, q_len, tps, scale * 1.4426950408889634f, part_o, part_ml);
  st = check_launch("attention_decode_kernel");
  if (st != TFX_OK) return st;
  launch_pdl(attention_decode_combine_kernel<HD>, dim3(q_len, heads, batch),
             dim3(HD < 32 ? 32 : HD), 0, stream, static_cast<const float*>(part_o),
             static_cast<const float2*>(part_ml), out, ld_out, heads, q_len, splits);
  return check_launch("attention_decode_combine_kernel");
}

}  // namespace

int launch_attention(const __half* q, const __half* k, const __half* v, int64_t ld_qkv,
                     __half* out, int64_t ld_out, int batch, int heads, int seq, int head_dim,
                     float scale, int causal, const KeyMask& km, cudaStream_t stream) {
  // Head dims 64, 128 and 256 run on the tcgen05 kernel (attention_tc.cu);
  // 8, 16 and 32 on its multi-head variant (attention_tc_small.cu) when the
  // heads fill 64-column blocks and the sequence spans more than one
  // 128-key tile. The mma.sync kernel below takes the rest (one-tile
  // sequences, where it measured faster; d_model 32: official shape 7) and
  // KV-cache chunks.
  if (attention_tc_supported(head_dim, scale))
    return launch_attention_tc(q, k, v, ld_qkv, out, ld_out, batch, heads, seq, head_dim, scale,
                               causal, km, stream);
  if (attention_tc_small_supported(head_dim, heads, batch, seq, scale))
    return launch_attention_tc_small(q, k, v, ld_qkv, out, ld_out, batch, heads, seq, head_dim,
                                     scale, causal, km, stream);
  return launch_mma(q, ld_qkv, k, v, AttnKv{ld_qkv, seq, seq, 0}, out, ld_out, batch, heads, seq,
                    head_dim, scale, causal, km, stream);
}

size_t attention_decode_part_bytes(int batch, int heads, int q_len, int head_dim) {
  int64_t rows = static_cast<int64_t>(batch) * heads;
  if (rows < kDecMaxCtas) rows = kDecMaxCtas;
  return static_cast<size_t>(decode_part_o_floats(rows, q_len, head_dim)) * 4 +
         static_cast<size_t>(rows) * q_len * 8;
}

int launch_attention_decode(const __half* q, int64_t ld_q, const __half* k, const __half* v,
                            const AttnKv& kv, __half* out, int64_t ld_out, int batch, int heads,
                            int q_len, int head_dim, float scale, float* part,
                            cudaStream_t stream) {
  if (q_len < 1 || q_len > kDecodeMaxQueries || kv.len < 1)
    return fail(TFX_ERR_INVALID_ARGUMENT, "attention_decode: 1 <= q_len <= %d, kv.len >= 1",
                kDecodeMaxQueries);
  if (heads > 65535 || batch > 65535)
    return fail(TFX_ERR_UNSUPPORTED, "attention_decode: batch and heads must be <= 65535");
  switch (head_dim) {
    case 8:
      return launch_decode_hd<8>(q, ld_q, k, v, kv, out, ld_out, batch, heads, q_len, scale, part,
                                 stream);
    case 16:
      return launch_decode_hd<16>(q, ld_q, k, v, kv, out, ld_out, batch, heads, q_len, scale,
                                  part, stream);
    case 32:
      return launch_decode_hd<32>(q, ld_q, k, v, kv, out, ld_out, batch, heads, q_len, scale,
                                  part, stream);
    case 64:
      return launch_decode_hd<64>(q, ld_q, k, v, kv, out, ld_out, batch, heads, q_len, scale,
                                  part, stream);
    case 128:
      return launch_decode_hd<128>(q, ld_q, k, v, kv, out, ld_out, batch, heads, q_len, scale,
                                   part, stream);
    case 256:
      return launch_decode_hd<256>(q, ld_q, k, v, kv, out, ld_out, batch, heads, q_len, scale,
                                   part, stream);
    default:
      return fail(TFX_ERR_UNSUPPORTED, "attention_decode: head_dim %d not in {8,...,256}",
                  head_dim);
  }
}

int launch_attention_kv(const __half* q, int64_t ld_q, const __half* k, const __half* v,
                        const AttnKv& kv, __half* out, int64_t ld_out, int batch, int heads,
                        int q_len, int head_dim, float scale, cudaStream_t stream) {
  if (attention_tc_supported(head_dim, scale))
    return launch_attention_tc_kv(q, ld_q, k, v, kv, out, ld_out, batch, heads, q_len, head_dim,
                                  scale, stream);
  return launch_mma(q, ld_q, k, v, kv, out, ld_out, batch, heads, q_len, head_dim, scale, 1,
                    KeyMask{}, stream);
}

}  // namespace tfx

