// Flash attention on the 5th-generation tensor cores, head_dim 64 and 128.
//
// CTA = 256 query rows of one (batch, head), split into two 128-row tiles A
// and B that share every K/V tile; 10 warps, one CTA per SM:
//   warp 0      TMA producer (one lane): Q_A and Q_B once, then K_j and V_j
//               into a ring of shared-memory stages
//   warp 1      TMEM owner (all 512 columns) + MMA issuer (one lane)
//   warps 2..5  softmax of tile A, warps 6..9 softmax of tile B; thread =
//               query row = TMEM lane, so no cross-thread reductions
// TMEM columns: S_A [0,128), S_B [128,256), O_A [256,256+HD), O_B after it.
//
// Per KV tile j and query tile X:
//   S_X  = Q_X K_j^T      SS MMA 128x128xHD, fp32 into TMEM
//   softmax warps         row max; lazy rescale of O_X; P = 2^(S*c - m) as
//                         fp16, written over the first 64 columns of S_X
//   O_X += P V_j          TS MMA: P straight from TMEM, V_j read MN-major
//                         from its row-major [keys x HD] tile
// The tensor core works on one tile's products while the other tile's
// softmax runs (A and B ping-pong), so neither unit waits for the other.
//
// Lazy rescaling: a row's reference max m only moves when its running max
// exceeds m by more than 8 (log2 units). P is then at most 2^8, fine in fp16,
// and O is rescaled in TMEM only on those (rare, warp-uniform) tiles.
// Scores are handled in the log2 domain: c = scale * log2(e) folds the
// softmax scale into the exponent's FMA.
//
// Masking: causal (key > query) and key padding (key >= valid_len[b]) apply
// only on a tile's diagonal / ragged KV tile. Rows past the sequence end are
// read as zeros by the 3-D tensor maps and never stored.
//
// Replaces the reference's attention call, F.scaled_dot_product_attention
// with is_causal=True inside _fast_attention_impl
// (torch_transformer_benchmark.py:718-818; scale hd^-0.5 at :215):
// softmax(Q K^T * scale + causal mask) V per head, fp32 statistics.
#include "internal.h"
#include "ptx.cuh"

namespace tfx {
namespace {

constexpr int kTcThreads = 320;
constexpr int kTile = 128;            // query rows per tile = keys per KV tile
constexpr float kRescaleLog2 = 8.0f;  // lazy-rescale threshold (P <= 2^8)
constexpr uint32_t kTmemCols = 512;

template <int HD>
struct TcAttn {
  static constexpr int kStages = HD == 64 ? 4 : 2;
  static constexpr int kBlocks = HD / 64;            // 128-byte column blocks per row
  static constexpr int kBlockBytes = kTile * 128;    // one 64-column block of a tile
  static constexpr int kTileBytes = kTile * HD * 2;  // one Q/K/V tile, fp16
  static constexpr int kQ = 0;                        // Q_A, Q_B
  static constexpr int kK = 2 * kTileBytes;
  static constexpr int kV = kK + kStages * kTileBytes;
  static constexpr int kBar = kV + kStages * kTileBytes;
  static constexpr int kSmem = kBar + 256 + 1024;    // barriers + alignment slack
  static constexpr uint32_t kColO = 2 * kTile;
  static_assert(kColO + 2 * HD <= kTmemCols, "TMEM budget");
  static_assert(kSmem <= 227 * 1024, "shared-memory budget");
};

template <int HD, bool CAUSAL>
__global__ void __launch_bounds__(kTcThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tm_q,
                        const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, __half* __restrict__ out,
                        int64_t ld_out, int heads, int seq, int nqb, float scale_log2,
                        const int32_t* __restrict__ valid_len, int* err) {
  using L = TcAttn<HD>;
  constexpr int S = L::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* q_full = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* k_full = q_full + 1;
  uint64_t* v_full = k_full + S;
  uint64_t* kv_empty = v_full + S;
  uint64_t* s_full = kv_empty + S;  // [2]: S_X computed
  uint64_t* p_full = s_full + 2;    // [2]: P_X written (and O_X rescaled), 4 warps arrive
  uint64_t* o_done = p_full + 2;    // [2]: O_X += P_X V completed
  uint64_t* drain = o_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int h = static_cast<int>(blockIdx.x % heads);
  const int b = static_cast<int>(blockIdx.x / heads);
  // Causal: the heaviest query blocks (the last ones) are launched first.
  const int qb = CAUSAL ? nqb - 1 - static_cast<int>(blockIdx.y) : static_cast<int>(blockIdx.y);
  const int q0 = qb * 2 * kTile;
  const int kend = valid_len ? min(seq, max(0, valid_len[b])) : seq;
  auto tiles_for = [&](int qx) {
    if (qx >= seq) return 0;
    const int lim = CAUSAL ? min(kend, qx + kTile) : kend;
    return (lim + kTile - 1) / kTile;
  };
  const int nA = tiles_for(q0);
  const int nB = tiles_for(q0 + kTile);
  const int n_iter = max(nA, nB);

  if (threadIdx.x == 0) {
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
    mbar_init(q_full, 1);
    for (int s = 0; s < S; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&p_full[x], 4);
      mbar_init(&o_done[x], 1);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      const int col0 = h * HD;
      mbar_arrive_expect_tx(q_full, 2 * L::kTileBytes);
#pragma unroll
      for (int x = 0; x < 2; ++x)
#pragma unroll
        for (int cb = 0; cb < L::kBlocks; ++cb)
          tma_load_3d(smem + L::kQ + x * L::kTileBytes + cb * L::kBlockBytes, &tm_q, q_full,
                      col0 + 64 * cb, q0 + x * kTile, b);
      int issued = 0;
      for (int j = 0; j < n_iter; ++j) {
        const int st = j % S;
        if (j >= S && !mbar_wait(&kv_empty[st], ((j / S) - 1) & 1, err, kDevTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&k_full[st], L::kTileBytes);
#pragma unroll
        for (int cb = 0; cb < L::kBlocks; ++cb)
          tma_load_3d(smem + L::kK + st * L::kTileBytes + cb * L::kBlockBytes, &tm_k, &k_full[st],
                      col0 + 64 * cb, j * kTile, b);
        mbar_arrive_expect_tx(&v_full[st], L::kTileBytes);
#pragma unroll
        for (int cb = 0; cb < L::kBlocks; ++cb)
          tma_load_3d(smem + L::kV + st * L::kTileBytes + cb * L::kBlockBytes, &tm_v, &v_full[st],
                      col0 + 64 * cb, j * kTile, b);
        issued = j + 1;
      }
      // Our own copies land before the CTA may exit (after a timeout nobody
      // else waits for them); on the normal path these phases are complete.
      mbar_wait(q_full, 0, nullptr, 0);
      for (int j = max(0, issued - S); j < issued; ++j) {
        mbar_wait(&k_full[j % S], (j / S) & 1, nullptr, 0);
        mbar_wait(&v_full[j % S], (j / S) & 1, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    // --------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_qk = idesc_f16_f32(kTile, kTile);
      constexpr uint32_t id_pv = idesc_f16_f32_bmn(kTile, HD);
      const uint32_t sq = smem_u32(smem + L::kQ);
      const uint32_t sk = smem_u32(smem + L::kK);
      const uint32_t sv = smem_u32(smem + L::kV);
      // S_x = Q_x K^T: both operands K-major; K advances 16 columns = 32 B
      // inside a 128-byte swizzled row, then to the next 64-column block.
      auto issue_qk = [&](int x, int st) {
        const uint32_t a0 = sq + x * L::kTileBytes;
        const uint32_t b0 = sk + st * L::kTileBytes;
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t off = (k >> 2) * L::kBlockBytes + (k & 3) * 32;
          mma_f16_ss(tmem + x * kTile, sdesc_k_sw128(a0 + off), sdesc_k_sw128(b0 + off), id_qk,
                     k > 0 ? 1u : 0u);
        }
      };
      // O_x += P_x V: P from TMEM (16 keys = 8 packed columns per step), V
      // MN-major (16 keys = 16 rows = 2048 B per step; 64-column blocks of
      // HD apart by one block).
      auto issue_pv = [&](int x, int st, bool accumulate) {
        const uint32_t b0 = sv + st * L::kTileBytes;
#pragma unroll
        for (int k = 0; k < kTile / 16; ++k) {
          mma_f16_ts(tmem + L::kColO + x * HD, tmem + x * kTile + 8 * k,
                     sdesc_mn_sw128(b0 + k * 2048, L::kBlockBytes), id_pv,
                     (accumulate || k > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(q_full, 0, err, kDevTimeoutFull);
      if (ok && n_iter > 0) {
        ok = mbar_wait(&k_full[0], 0, err, kDevTimeoutFull);
        if (ok) {
          tc_fence_after();
          if (nA > 0) {
            issue_qk(0, 0);
            mma_commit(&s_full[0]);
          }
          if (nB > 0) {
            issue_qk(1, 0);
            mma_commit(&s_full[1]);
          }
        }
      }
      for (int j = 0; ok && j < n_iter; ++j) {
        const int st = j % S, st1 = (j + 1) % S;
        const uint32_t par = (j / S) & 1, par1 = ((j + 1) / S) & 1;
        const uint32_t jp = j & 1;
        if (!mbar_wait(&v_full[st], par, err, kDevTimeoutFull)) break;
        bool k1 = false;
        if (j < nA) {
          if (!mbar_wait(&p_full[0], jp, err, kDevTimeoutOther)) break;
          tc_fence_after();
          issue_pv(0, st, j > 0);
          mma_commit(&o_done[0]);
          if (j + 1 < nA) {
            // S_A(j+1) overwrites P_A(j): wait for PV_A(j) to finish reading it.
            if (!mbar_wait(&k_full[st1], par1, err, kDevTimeoutFull)) break;
            k1 = true;
            if (!mbar_wait(&o_done[0], jp, err, kDevTimeoutAccum)) break;
            tc_fence_after();
            issue_qk(0, st1);
            mma_commit(&s_full[0]);
          }
        }
        if (j < nB) {
          if (!mbar_wait(&p_full[1], jp, err, kDevTimeoutOther)) break;
          tc_fence_after();
          issue_pv(1, st, j > 0);
          mma_commit(&o_done[1]);
        }
        mma_commit(&kv_empty[st]);  // K_j and V_j are free once these MMAs complete
        if (j + 1 < nB) {
          if (!k1 && !mbar_wait(&k_full[st1], par1, err, kDevTimeoutFull)) break;
          if (!mbar_wait(&o_done[1], jp, err, kDevTimeoutAccum)) break;
          tc_fence_after();
          issue_qk(1, st1);
          mma_commit(&s_full[1]);
        }
      }
      // Every MMA issued so far completes before TMEM is released.
      mma_commit(drain);
      mbar_wait(drain, 0, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int x = (warp - 2) >> 2;  // 0: tile A, 1: tile B
    const int quarter = warp & 3;   // this warp's TMEM lanes [32*quarter, +32)
    const int row = quarter * 32 + lane;
    const int qx = q0 + x * kTile;
    const int q = qx + row;
    const int nx = x == 0 ? nA : nB;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t t_s = tmem + lane_off + x * kTile;
    const uint32_t t_o = tmem + lane_off + L::kColO + x * HD;
    const int lim_row = CAUSAL ? min(kend, q + 1) : kend;    // keys [0, lim_row) visible
    const int lim_tile = CAUSAL ? min(kend, qx + 1) : kend;  // smallest lim_row of the tile
    float m_ref = 0.f;
    float l0 = 0.f, l1 = 0.f;
    bool ok = true;
    for (int j = 0; j < nx; ++j) {
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[x], j & 1, err, kDevTimeoutAccum))) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t s[kTile];
#pragma unroll
      for (int c = 0; c < kTile / 32; ++c)
        tmem_ld32(t_s + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(s + 32 * c));
      tmem_ld_wait();
      if ((j + 1) * kTile > lim_tile) {  // diagonal or ragged KV tile (warp-uniform)
        const int c0 = lim_row - j * kTile;
#pragma unroll
        for (int c = 0; c < kTile; ++c)
          if (c >= c0) s[c] = 0xff800000u;  // -inf
      }
      float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
      for (int c = 0; c < kTile; c += 4) {
        mx0 = fmaxf(mx0, __uint_as_float(s[c]));
        mx1 = fmaxf(mx1, __uint_as_float(s[c + 1]));
        mx2 = fmaxf(mx2, __uint_as_float(s[c + 2]));
        mx3 = fmaxf(mx3, __uint_as_float(s[c + 3]));
      }
      const float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
      const float m_new = mx * scale_log2;  // -inf when every key of the row is masked
      if (j == 0) {
        m_ref = mx == -INFINITY ? 0.f : m_new;
      } else if (__any_sync(0xffffffffu, m_new > m_ref + kRescaleLog2)) {
        const float m_up = fmaxf(m_ref, m_new);
        const float f = fast_exp2(m_ref - m_up);
        m_ref = m_up;
        l0 *= f;
        l1 *= f;
        // PV(j-1) completed before S(j) was issued, so O is stable here.
#pragma unroll 1
        for (int c = 0; c < HD; c += 16) {  // 16 columns at a time: S stays in registers
          uint32_t o[16];
          tmem_ld16(t_o + c, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
          tmem_st16(t_o + c, o);
        }
      }
      const float neg = -m_ref;
#pragma unroll
      for (int c = 0; c < kTile / 32; ++c) {
        uint32_t p[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float e0 = fast_exp2(fmaf(__uint_as_float(s[32 * c + 2 * i]), scale_log2, neg));
          const float e1 =
              fast_exp2(fmaf(__uint_as_float(s[32 * c + 2 * i + 1]), scale_log2, neg));
          l0 += e0;
          l1 += e1;
          p[i] = pack_half2(e0, e1);
        }
        tmem_st16(t_s + 16 * c, p);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[x]);
    }
    if (ok && nx > 0)
      ok = __all_sync(0xffffffffu, mbar_wait(&o_done[x], (nx - 1) & 1, err, kDevTimeoutAccum));
    const float l = l0 + l1;
    const float inv = l > 0.f ? 1.f / l : 0.f;
    __half* dst = out + (static_cast<int64_t>(b) * seq + q) * ld_out + h * HD;
    if (ok && nx > 0) {
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < HD; c += 32) {
        uint32_t o[32];
        tmem_ld32(t_o + c, o);
        tmem_ld_wait();
        if (q < seq) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float* f = reinterpret_cast<const float*>(o + 8 * i);
            d4[i] = make_uint4(pack_half2(f[0] * inv, f[1] * inv), pack_half2(f[2] * inv, f[3] * inv),
                               pack_half2(f[4] * inv, f[5] * inv), pack_half2(f[6] * inv, f[7] * inv));
          }
        }
      }
    } else if (ok && q < seq) {
      // No visible key (valid_len 0): the output row is zero.
      uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
      for (int i = 0; i < HD / 8; ++i) d4[i] = make_uint4(0, 0, 0, 0);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int HD, bool CAUSAL>
int launch_tc(const __half* q, const __half* k, const __half* v, int64_t ld_qkv, __half* out,
              int64_t ld_out, int batch, int heads, int seq, float scale,
              const int32_t* valid_len, cudaStream_t stream) {
  using L = TcAttn<HD>;
  static int smem_done[kMaxDevices] = {0};
  auto kern = attention_tc_kernel<HD, CAUSAL>;
  int st = ensure_smem(reinterpret_cast<const void*>(kern), L::kSmem, smem_done);
  if (st != TFX_OK) return st;
  const uint64_t cols = static_cast<uint64_t>(heads) * HD;
  const uint64_t bstride = static_cast<uint64_t>(seq) * static_cast<uint64_t>(ld_qkv);
  CUtensorMap tq, tk, tv;
  const __half* bases[3] = {q, k, v};
  CUtensorMap* maps[3] = {&tq, &tk, &tv};
  for (int i = 0; i < 3; ++i) {
    st = make_tmap_3d(maps[i], bases[i], static_cast<uint64_t>(seq), static_cast<uint64_t>(batch),
                      cols, static_cast<uint64_t>(ld_qkv), bstride, 64, kTile);
    if (st != TFX_OK) return st;
  }
  const int nqb = (seq + 2 * kTile - 1) / (2 * kTile);
  const dim3 grid(static_cast<unsigned>(batch) * static_cast<unsigned>(heads),
                  static_cast<unsigned>(nqb));
  kern<<<grid, kTcThreads, L::kSmem, stream>>>(tq, tk, tv, out, ld_out, heads, seq, nqb,
                                                scale * 1.4426950408889634f, valid_len,
                                                device_error_word());
  return check_launch("attention_tc_kernel");
}

}  // namespace

bool attention_tc_supported(int head_dim, float scale) {
  return (head_dim == 64 || head_dim == 128) && scale > 0.f;
}

int launch_attention_tc(const __half* q, const __half* k, const __half* v, int64_t ld_qkv,
                        __half* out, int64_t ld_out, int batch, int heads, int seq, int head_dim,
                        float scale, int causal, const int32_t* valid_len, cudaStream_t stream) {
  if (static_cast<int64_t>(batch) * heads > 0x7fffffff || (seq + 2 * kTile - 1) / (2 * kTile) > 65535)
    return fail(TFX_ERR_UNSUPPORTED, "tfx_attention: batch*heads or seq too large for the grid");
  if (head_dim == 64)
    return causal ? launch_tc<64, true>(q, k, v, ld_qkv, out, ld_out, batch, heads, seq, scale,
                                        valid_len, stream)
                  : launch_tc<64, false>(q, k, v, ld_qkv, out, ld_out, batch, heads, seq, scale,
                                         valid_len, stream);
  if (head_dim == 128)
    return causal ? launch_tc<128, true>(q, k, v, ld_qkv, out, ld_out, batch, heads, seq, scale,
                                         valid_len, stream)
                  : launch_tc<128, false>(q, k, v, ld_qkv, out, ld_out, batch, heads, seq, scale,
                                          valid_len, stream);
  return fail(TFX_ERR_UNSUPPORTED, "attention_tc: head_dim %d not in {64,128}", head_dim);
}

}  // namespace tfx
