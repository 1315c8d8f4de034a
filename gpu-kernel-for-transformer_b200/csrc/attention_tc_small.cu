// Flash attention on the 5th-generation tensor cores for head_dim 8, 16 and
// 32, where one head is too narrow for a tcgen05 tile of its own.
//
// CTA = 128 query rows of one sequence x one 64-column block of heads
// (G = 64 / head_dim heads: 8, 4 or 2), so every TMA box is a full
// 128-byte-swizzled 64-column tile and the heads of a block share each K/V
// stage. 6 warps, one CTA per SM (all 512 TMEM columns):
//   warp 0      TMA producer (one lane): the Q block once, then K_j and V_j
//               (128 keys x 64 columns each) into a ring of stages
//   warp 1      TMEM owner + MMA issuer (one lane)
//   warps 2..5  softmax: thread = query row = TMEM lane, all G heads
// TMEM columns: S double buffer [0,256), fp16 P double buffer [256,384),
// O of head g at [384 + g*N, +N) with N = max(16, head_dim).
//
// Per KV tile j and head g (flattened i = j*G + g, buffer i % 2):
//   S_i = Q_g K_g^T   SS MMA, 128 x 128 x K (K = head_dim, or 16 at head_dim
//                     8: the Q block is staged twice, each copy with the other
//                     parity's heads zeroed, so one K=16 step over a head pair
//                     adds only this head's products)
//   softmax           row max, lazy rescale of O_g, P = 2^(S*c - m) fp16
//   O_g += P_i V_g    TS MMA, P from TMEM; V_g straight from the row-major
//                     [keys x 64] tile as an MN-major operand starting at the
//                     head's column (N = 16 covers a head pair at head_dim 8;
//                     this head's half of O is kept)
// S_{i+2} is issued as soon as the softmax warps hold S_i in registers, so
// the tensor core computes one head's scores while another head's softmax
// runs.
//
// Masking as in attention_tc.cu: causal on the diagonal tile, prefix lengths
// on the ragged tile, a key bitmask on every tile whose 128 bits are not all
// set. Rows past the sequence end read as zeros (3-D tensor maps) and are
// never stored.
//
// Used for sequences longer than one 128-key tile (official shape 13 and
// longer); shorter ones run the mma.sync kernel in attention.cu, which is
// faster there (see attention_tc_small_supported). Replaces the
// reference's SDPA call (torch_transformer_benchmark.py:767-808; the
// reference forces the CUTLASS memory-efficient backend for head_dim 8,
// :145-147, 788-799).
#include "internal.h"
#include "ptx.cuh"

namespace tfx {
namespace {

constexpr int kSmThreads = 192;
constexpr int kSmTile = 128;  // query rows per CTA = keys per KV tile
constexpr int kSmStages = 3;
constexpr float kSmRescaleLog2 = 8.0f;  // lazy-rescale threshold (P <= 2^8)

template <int HD>
struct SmallAttn {
  static constexpr int G = 64 / HD;                 // heads per CTA
  static constexpr int kN = HD < 16 ? 16 : HD;      // P.V N (a head pair at HD 8)
  static constexpr int kKSteps = HD < 16 ? 1 : HD / 16;  // QK^T K-steps of 16
  static constexpr int kTileBytes = kSmTile * 128;  // 128 rows x 64 fp16 columns
  static constexpr int kQCopies = HD == 8 ? 2 : 1;
  static constexpr int kQ = 0;
  static constexpr int kK = kQCopies * kTileBytes;
  static constexpr int kV = kK + kSmStages * kTileBytes;
  static constexpr int kBar = kV + kSmStages * kTileBytes;
  static constexpr int kSmem = kBar + 256 + 1024;  // barriers + alignment slack
  static constexpr uint32_t kColS = 0;
  static constexpr uint32_t kColP = 256;
  static constexpr uint32_t kColO = 384;
  static_assert(kColO + G * kN <= 512, "TMEM budget");
  static_assert(G % 2 == 0, "buffers alternate by head parity");
  static_assert(kSmem <= 227 * 1024, "shared-memory budget");
};

// Column (fp16 elements) inside the 64-column block where head g's QK^T
// reduction and P.V operand start.
template <int HD>
__device__ __forceinline__ int head_col(int g) {
  return HD == 8 ? 16 * (g >> 1) : g * HD;
}

template <int HD, bool CAUSAL>
__global__ void __launch_bounds__(kSmThreads, 1)
    attention_tc_small_kernel(const __grid_constant__ CUtensorMap tm_q,
                              const __grid_constant__ CUtensorMap tm_k,
                              const __grid_constant__ CUtensorMap tm_v, __half* __restrict__ out,
                              int64_t ld_out, int groups, int seq, int nqb, float scale_log2,
                              const int32_t* __restrict__ valid_len,
                              const uint32_t* __restrict__ key_bits, int key_words, int* err) {
  grid_dep_wait();
  grid_dep_launch();
  using L = SmallAttn<HD>;
  constexpr int G = L::G;
  constexpr int NS = kSmStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* q_full = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* q_ready = q_full + 1;   // HD 8: zero-padded Q copies written (4 warps)
  uint64_t* k_full = q_ready + 1;   // [NS]
  uint64_t* v_full = k_full + NS;   // [NS]
  uint64_t* k_empty = v_full + NS;  // [NS] K_j no longer read (after its last S)
  uint64_t* v_empty = k_empty + NS; // [NS] V_j no longer read (after its last P.V)
  uint64_t* s_full = v_empty + NS;  // [2] S_i computed
  uint64_t* s_free = s_full + 2;    // [2] S_i in the softmax warps' registers (4 warps)
  uint64_t* p_full = s_free + 2;    // [2] P_i written, O rescaled (4 warps)
  uint64_t* o_done = p_full + 2;    // [2] P_i . V completed
  uint64_t* drain = o_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bg = static_cast<int>(blockIdx.x);
  const int b = bg / groups, hg = bg % groups;
  const int qb = CAUSAL ? nqb - 1 - static_cast<int>(blockIdx.y) : static_cast<int>(blockIdx.y);
  const int q0 = qb * kSmTile;
  const int kend = valid_len ? min(seq, max(0, valid_len[b])) : seq;
  const int lim = CAUSAL ? min(kend, q0 + kSmTile) : kend;
  const int n = (lim + kSmTile - 1) / kSmTile;  // KV tiles this query block needs
  const int total = n * G;

  if (threadIdx.x == 0) {
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
    mbar_init(q_full, 1);
    mbar_init(q_ready, 4);
    for (int s = 0; s < NS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&s_free[x], 4);
      mbar_init(&p_full[x], 4);
      mbar_init(&o_done[x], 1);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int col0 = hg * 64;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, L::kQCopies * L::kTileBytes);
#pragma unroll
      for (int c = 0; c < L::kQCopies; ++c)
        tma_load_3d(smem + L::kQ + c * L::kTileBytes, &tm_q, q_full, col0, q0, b);
      int k_issued = 0, v_issued = 0;
      for (int j = 0; j < n; ++j) {
        const int st = j % NS;
        const uint32_t par = ((j / NS) - 1) & 1;  // phase of the tile that last used st
        if (j >= NS && !mbar_wait(&k_empty[st], par, err, kDevTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&k_full[st], L::kTileBytes);
        tma_load_3d(smem + L::kK + st * L::kTileBytes, &tm_k, &k_full[st], col0, j * kSmTile, b);
        k_issued = j + 1;
        if (j >= NS && !mbar_wait(&v_empty[st], par, err, kDevTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&v_full[st], L::kTileBytes);
        tma_load_3d(smem + L::kV + st * L::kTileBytes, &tm_v, &v_full[st], col0, j * kSmTile, b);
        v_issued = j + 1;
      }
      // Our own copies land before the CTA may exit (after a timeout nobody
      // else waits for them); on the normal path these phases are complete.
      mbar_wait(q_full, 0, nullptr, 0);
      for (int j = max(0, k_issued - NS); j < k_issued; ++j)
        mbar_wait(&k_full[j % NS], (j / NS) & 1, nullptr, 0);
      for (int j = max(0, v_issued - NS); j < v_issued; ++j)
        mbar_wait(&v_full[j % NS], (j / NS) & 1, nullptr, 0);
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_qk = idesc_f16_f32(kSmTile, kSmTile);
      constexpr uint32_t id_pv = idesc_f16_f32_bmn(kSmTile, L::kN);
      // Descriptors built once; each MMA adds a byte offset (16-byte units)
      // to the address field (shared addresses < 2^18: no carry).
      const uint64_t dq0 = sdesc_k_sw128(smem_u32(smem + L::kQ));
      const uint64_t dk0 = sdesc_k_sw128(smem_u32(smem + L::kK));
      const uint64_t dv0 = sdesc_mn_sw128(smem_u32(smem + L::kV), L::kTileBytes);
      auto issue_s = [&](int i) -> bool {  // S_i = Q_g K_g^T -> S buffer i % 2
        const int j = i / G, g = i % G, st = j % NS, buf = i & 1;
        if (g == 0 && !mbar_wait(&k_full[st], (j / NS) & 1, err, kDevTimeoutFull)) return false;
        if (i >= 2 && !mbar_wait(&s_free[buf], ((i >> 1) - 1) & 1, err, kDevTimeoutOther))
          return false;
        tc_fence_after();
        const int copy = HD == 8 ? (g & 1) : 0;
        const uint64_t da = dq0 + static_cast<uint64_t>((copy * L::kTileBytes) >> 4);
        const uint64_t db = dk0 + static_cast<uint64_t>((st * L::kTileBytes) >> 4);
        const int c = head_col<HD>(g);
#pragma unroll
        for (int k = 0; k < L::kKSteps; ++k) {
          const uint64_t off = static_cast<uint64_t>((2 * c + 32 * k) >> 4);
          mma_f16_ss(tmem + L::kColS + buf * kSmTile, da + off, db + off, id_qk, k > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[buf]);
        if (g == G - 1) mma_commit(&k_empty[st]);  // K_j read by every head
        return true;
      };
      bool ok = mbar_wait(q_full, 0, err, kDevTimeoutFull);
      if (ok && HD == 8) ok = mbar_wait(q_ready, 0, err, kDevTimeoutOther);
      if (ok && total > 0) ok = issue_s(0);
      if (ok && total > 1) ok = issue_s(1);
      for (int i = 0; ok && i < total; ++i) {
        const int j = i / G, g = i % G, st = j % NS, buf = i & 1;
        if (g == 0 && !(ok = mbar_wait(&v_full[st], (j / NS) & 1, err, kDevTimeoutFull))) break;
        if (!(ok = mbar_wait(&p_full[buf], (i >> 1) & 1, err, kDevTimeoutOther))) break;
        tc_fence_after();
        // O_g (+)= P_i V_g: 16 keys (8 packed P columns, 16 V rows = 2 KB) per step.
        const uint64_t db = dv0 + static_cast<uint64_t>((st * L::kTileBytes + 2 * head_col<HD>(g)) >> 4);
#pragma unroll
        for (int k = 0; k < kSmTile / 16; ++k)
          mma_f16_ts(tmem + L::kColO + g * L::kN, tmem + L::kColP + buf * 64 + 8 * k,
                     db + static_cast<uint64_t>((k * 2048) >> 4), id_pv, (j > 0 || k > 0) ? 1u : 0u);
        mma_commit(&o_done[buf]);
        if (g == G - 1) mma_commit(&v_empty[st]);  // V_j read by every head
        if (i + 2 < total) ok = issue_s(i + 2);
      }
      // Every MMA this thread issued completes before TMEM is released.
      mma_commit(drain);
      mbar_wait(drain, 0, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, +32)
    const int row = quarter * 32 + lane;
    const int q = q0 + row;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const int lim_row = CAUSAL ? min(kend, q + 1) : kend;  // keys [0, lim_row) visible
    const int lim_tile = CAUSAL ? min(kend, q0 + 1) : kend; // smallest of the tile
    bool ok = true;
    if constexpr (HD == 8) {
      // Zero the other parity's heads in each Q copy: logical 16-byte chunk
      // c (= head c) of row r sits at physical chunk c ^ (r % 8).
      if (!__all_sync(0xffffffffu, mbar_wait(q_full, 0, err, kDevTimeoutFull))) ok = false;
      if (ok) {
#pragma unroll
        for (int copy = 0; copy < 2; ++copy) {
          const uint32_t rb = smem_u32(smem + L::kQ + copy * L::kTileBytes) + row * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c)
            if ((c & 1) != copy)
              asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(
                               rb + ((c ^ (row & 7)) << 4)),
                           "r"(0u)
                           : "memory");
        }
        fence_proxy_async_smem();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(q_ready);
    }
    float m_ref[G], l_sum[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      m_ref[g] = 0.f;
      l_sum[g] = 0.f;
    }
    const uint64_t c2 = f2_pack(scale_log2, scale_log2);
    for (int j = 0; ok && j < n; ++j) {
      // Key bitmask words of this KV tile (uniform loads).
      uint32_t kw[4] = {0xffffffffu, 0xffffffffu, 0xffffffffu, 0xffffffffu};
      bool bits_full = true;
      if (key_bits != nullptr) {
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const int wi = 4 * j + w;
          kw[w] = wi < key_words ? key_bits[static_cast<int64_t>(b) * key_words + wi] : 0u;
          bits_full = bits_full && kw[w] == 0xffffffffu;
        }
      }
      const bool edge = (j + 1) * kSmTile > lim_tile;  // diagonal or ragged tile (uniform)
      const int c0 = lim_row - j * kSmTile;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const int i = j * G + g;
        const int buf = g & 1;  // == i & 1 (G is even)
        if (!__all_sync(0xffffffffu,
                        mbar_wait(&s_full[buf], (i >> 1) & 1, err, kDevTimeoutAccum))) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t s[kSmTile];
#pragma unroll
        for (int c = 0; c < kSmTile / 32; ++c)
          tmem_ld32(tmem + lane_off + L::kColS + buf * kSmTile + 32 * c,
                    *reinterpret_cast<uint32_t(*)[32]>(s + 32 * c));
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[buf]);  // the next S may overwrite this buffer
        if (edge) {
#pragma unroll
          for (int c = 0; c < kSmTile; ++c)
            if (c >= c0) s[c] = 0xff800000u;  // -inf
        }
        if (!bits_full) {
#pragma unroll
          for (int c = 0; c < kSmTile; ++c)
            if (!((kw[c >> 5] >> (c & 31)) & 1u)) s[c] = 0xff800000u;
        }
        float mm[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) mm[t] = fmaxf(__uint_as_float(s[t]), __uint_as_float(s[t + 8]));
#pragma unroll
        for (int c = 16; c < kSmTile; c += 16)
#pragma unroll
          for (int t = 0; t < 8; ++t)
            mm[t] = fmax3(mm[t], __uint_as_float(s[c + t]), __uint_as_float(s[c + 8 + t]));
        const float mx =
            fmaxf(fmax3(mm[0], mm[1], mm[2]), fmax3(fmax3(mm[3], mm[4], mm[5]), mm[6], mm[7]));
        const float m_new = mx * scale_log2;  // -inf when every key of the row is masked
        bool rescale = false;
        float f = 1.f;
        if (j == 0) {
          m_ref[g] = mx == -INFINITY ? 0.f : m_new;
        } else if (__any_sync(0xffffffffu, m_new > m_ref[g] + kSmRescaleLog2)) {
          const float m_up = fmaxf(m_ref[g], m_new);
          f = fast_exp2(m_ref[g] - m_up);
          m_ref[g] = m_up;
          l_sum[g] *= f;
          rescale = true;
        }
        const uint64_t negm2 = f2_pack(-m_ref[g], -m_ref[g]);
        uint64_t ls0 = 0, ls1 = 0;
        const uint32_t t_p = tmem + lane_off + L::kColP + buf * 64;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t pw[32];
#pragma unroll
          for (int t = 0; t < 32; ++t) {
            const int c = 64 * half + 2 * t;
            const uint64_t arg =
                f2_fma(f2_pack(__uint_as_float(s[c]), __uint_as_float(s[c + 1])), c2, negm2);
            uint64_t e;
            if ((t & 7) < 2) {  // a quarter of the exponentials on the FMA pipe
              e = exp2_poly_f2(arg);
            } else {
              float a0, a1;
              f2_unpack(arg, a0, a1);
              e = f2_pack(fast_exp2(a0), fast_exp2(a1));
            }
            if (t & 1) ls1 = f2_add(ls1, e); else ls0 = f2_add(ls0, e);
            float e0, e1;
            f2_unpack(e, e0, e1);
            pw[t] = pack_half2(e0, e1);
          }
          if (half == 0) {
            // P buffer and O_g are read / written by P.V of i - 2 until it
            // completes (in issue order, so O_g's own last update too).
            if (i >= 2 && !__all_sync(0xffffffffu, mbar_wait(&o_done[buf], ((i >> 1) - 1) & 1,
                                                             err, kDevTimeoutAccum))) {
              ok = false;
              break;
            }
            tc_fence_after();
            if (rescale) {
              const uint32_t t_o = tmem + lane_off + L::kColO + g * L::kN;
              uint32_t o[16];
#pragma unroll
              for (int c = 0; c < L::kN; c += 16) {
                tmem_ld16(t_o + c, o);
                tmem_ld_wait();
#pragma unroll
                for (int t = 0; t < 16; ++t) o[t] = __float_as_uint(__uint_as_float(o[t]) * f);
                tmem_st16(t_o + c, o);
              }
            }
          }
          tmem_st32(t_p + 32 * half, pw);
        }
        if (!ok) break;
        float la, lb, lc, ld;
        f2_unpack(ls0, la, lb);
        f2_unpack(ls1, lc, ld);
        l_sum[g] += (la + lb) + (lc + ld);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[buf]);
      }
    }
    // The last P.V (in issue order) completes after all earlier ones.
    if (ok && total > 0)
      ok = __all_sync(0xffffffffu,
                      mbar_wait(&o_done[(total - 1) & 1], ((total - 1) >> 1) & 1, err,
                                kDevTimeoutAccum));
    // tcgen05.ld is warp-collective (.sync.aligned): the TMEM reads below run
    // on every lane of the warp (ok and total are warp-uniform); only the
    // global stores are predicated on the row being inside the sequence.
    const bool store = q < seq;
    if (ok && total == 0) {
      // No visible key at all (valid length 0): zero rows, O never computed.
      if (store) {
        uint4* d4 =
            reinterpret_cast<uint4*>(out + (static_cast<int64_t>(b) * seq + q) * ld_out + col0);
#pragma unroll
        for (int t = 0; t < 8; ++t) d4[t] = make_uint4(0u, 0u, 0u, 0u);
      }
    } else if (ok) {
      tc_fence_after();
      __half* dst = out + (static_cast<int64_t>(b) * seq + q) * ld_out + col0;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float inv = l_sum[g] > 0.f ? 1.f / l_sum[g] : 0.f;
        const uint32_t t_o = tmem + lane_off + L::kColO + g * L::kN + (HD == 8 ? 8 * (g & 1) : 0);
        uint32_t w[HD / 2];
        if constexpr (HD == 8) {
          uint32_t o[8];
          tmem_ld8(t_o, o);
          tmem_ld_wait();
#pragma unroll
          for (int t = 0; t < 4; ++t)
            w[t] = pack_half2(__uint_as_float(o[2 * t]) * inv, __uint_as_float(o[2 * t + 1]) * inv);
        } else {
#pragma unroll
          for (int c = 0; c < HD; c += 16) {
            uint32_t o[16];
            tmem_ld16(t_o + c, o);
            tmem_ld_wait();
#pragma unroll
            for (int t = 0; t < 8; ++t)
              w[c / 2 + t] =
                  pack_half2(__uint_as_float(o[2 * t]) * inv, __uint_as_float(o[2 * t + 1]) * inv);
          }
        }
        if (store) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + g * HD);
#pragma unroll
          for (int t = 0; t < HD / 8; ++t)
            d4[t] = make_uint4(w[4 * t], w[4 * t + 1], w[4 * t + 2], w[4 * t + 3]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, 512);
  }
}

template <int HD, bool CAUSAL>
int launch_small(const __half* q, const __half* k, const __half* v, int64_t ld_qkv, __half* out,
                 int64_t ld_out, int batch, int heads, int seq, float scale, const KeyMask& km,
                 cudaStream_t stream) {
  using L = SmallAttn<HD>;
  static int smem_done[kMaxDevices] = {0};
  auto kern = attention_tc_small_kernel<HD, CAUSAL>;
  int st = ensure_smem(reinterpret_cast<const void*>(kern), L::kSmem, smem_done);
  if (st != TFX_OK) return st;
  const uint64_t cols = static_cast<uint64_t>(heads) * HD;
  const uint64_t bstride = static_cast<uint64_t>(seq) * static_cast<uint64_t>(ld_qkv);
  CUtensorMap tq, tk, tv;
  st = make_tmap_3d(&tq, q, seq, batch, cols, ld_qkv, bstride, 64, kSmTile);
  if (st == TFX_OK) st = make_tmap_3d(&tk, k, seq, batch, cols, ld_qkv, bstride, 64, kSmTile);
  if (st == TFX_OK) st = make_tmap_3d(&tv, v, seq, batch, cols, ld_qkv, bstride, 64, kSmTile);
  if (st != TFX_OK) return st;
  const int groups = static_cast<int>(cols / 64);
  const int nqb = (seq + kSmTile - 1) / kSmTile;
  const dim3 grid(static_cast<unsigned>(batch) * static_cast<unsigned>(groups),
                  static_cast<unsigned>(nqb));
  launch_pdl(kern, grid, dim3(kSmThreads), L::kSmem, stream, tq, tk, tv, out, ld_out, groups, seq,
             nqb, scale * 1.4426950408889634f, km.len, km.bits, key_words(seq),
             device_error_word());
  return check_launch("attention_tc_small_kernel");
}

template <int HD>
int launch_small_c(const __half* q, const __half* k, const __half* v, int64_t ld_qkv, __half* out,
                   int64_t ld_out, int batch, int heads, int seq, float scale, int causal,
                   const KeyMask& km, cudaStream_t stream) {
  return causal ? launch_small<HD, true>(q, k, v, ld_qkv, out, ld_out, batch, heads, seq, scale,
                                         km, stream)
                : launch_small<HD, false>(q, k, v, ld_qkv, out, ld_out, batch, heads, seq, scale,
                                          km, stream);
}

}  // namespace

// Sequences of one 128-key tile stay on the mma.sync kernel: there a CTA's
// work is a few small products per head and its latency, not the tensor
// core, sets the time (one B200, per launch: B=64, S=128, H=16, head_dim 8:
// mma.sync 13.6 us, this kernel 22.1 us; head_dim 16: 9.0 / 9.9; head_dim
// 32: 7.2 / 7.0). From two tiles on this kernel is ahead (head_dim 32:
// S=1024, B=64: 138.0 / 91.3 us; S=4096, B=8: 273.6 / 136.1 us).
bool attention_tc_small_supported(int head_dim, int heads, int batch, int seq, float scale) {
  if (head_dim != 8 && head_dim != 16 && head_dim != 32) return false;
  if (seq <= kSmTile) return false;
  const int64_t cols = static_cast<int64_t>(heads) * head_dim;
  return cols % 64 == 0 && scale > 0.f &&
         static_cast<int64_t>(batch) * (cols / 64) <= 0x7fffffffLL &&
         (seq + kSmTile - 1) / kSmTile <= 65535;
}

int launch_attention_tc_small(const __half* q, const __half* k, const __half* v, int64_t ld_qkv,
                              __half* out, int64_t ld_out, int batch, int heads, int seq,
                              int head_dim, float scale, int causal, const KeyMask& km,
                              cudaStream_t stream) {
  switch (head_dim) {
    case 8:
      return launch_small_c<8>(q, k, v, ld_qkv, out, ld_out, batch, heads, seq, scale, causal, km,
                               stream);
    case 16:
      return launch_small_c<16>(q, k, v, ld_qkv, out, ld_out, batch, heads, seq, scale, causal, km,
                                stream);
    case 32:
      return launch_small_c<32>(q, k, v, ld_qkv, out, ld_out, batch, heads, seq, scale, causal, km,
                                stream);
    default:
      return fail(TFX_ERR_UNSUPPORTED, "attention_tc_small: head_dim %d not in {8,16,32}",
                  head_dim);
  }
}

}  // namespace tfx
