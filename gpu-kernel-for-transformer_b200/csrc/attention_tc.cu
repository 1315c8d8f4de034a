// Flash attention on the 5th-generation tensor cores, head_dim 64, 128 and
// 256 (256: one query tile per CTA, one K/V stage).
//
// CTA = 256 query rows of one (batch, head), split into two 128-row tiles A
// and B that share every K/V tile; 11 warps, one CTA per SM:
//   warp 0      TMA producer (one lane): Q_A and Q_B once, then K_j and V_j
//               into a ring of shared-memory stages
//   warp 1      TMEM owner (all 512 columns) + MMA issuer of tile A (one lane)
//   warp 10     MMA issuer of tile B (one lane)
//   warps 2..5  softmax of tile A, warps 6..9 softmax of tile B; thread =
//               query row = TMEM lane, so no cross-thread reductions
// tcgen05.mma issue blocks while the tensor core's short instruction queue
// is full; with one issuer per tile, one tile's commits and barrier waits
// overlap the other tile's queued products instead of draining the queue.
// TMEM columns (512):
//   HD 64:  S_A [0,128) S_B [128,256) P_A [256,320) P_B [320,384) O_A, O_B
//   HD 128: S_A [0,128) S_B [128,256) O_A [256,384) O_B [384,512), and P_X
//           is written over the first 64 columns of S_X
//
// Per KV tile j and query tile X:
//   S_X  = Q_X K_j^T      SS MMA 128x128xHD, fp32 into TMEM
//   softmax warps         row max; lazy rescale of O_X; P = 2^(S*c - m) as
//                         fp16 into TMEM
//   O_X += P V_j          TS MMA, P straight from TMEM. V_j comes either
//                         K-major from a transposed copy V^T [b][h][d][s]
//                         (the forward path; full-rate MMAs) or MN-major
//                         from the row-major [keys x HD] tile (the plain
//                         tfx_attention call, whose MMAs run about half as
//                         fast with an MN-major operand)
// With a separate P region (HD 64) S_X(j+1) is computed as soon as the
// softmax warps hold S_X(j) in registers, so the softmax of consecutive KV
// tiles runs back to back and only the P store waits for PV_X(j-1). The two
// query tiles' softmax warps share each SM sub-partition, so one tile's
// loads and reductions hide behind the other tile's exponentials.
//
// Lazy rescaling: a row's reference max m only moves when its running max
// exceeds m by more than 8 (log2 units). P is then at most 2^8, fine in fp16,
// and O is rescaled in TMEM only on those (rare, warp-uniform) tiles.
// Scores are handled in the log2 domain: c = scale * log2(e) folds the
// softmax scale into the exponent's FMA.
//
// Masking: causal (key > query position) and prefix key padding (key >=
// valid_len[b]) apply only on a tile's diagonal / ragged KV tile; a key
// bitmask (any padding pattern: bit k of word w of sequence b = key 32w+k
// is valid) masks each KV tile whose 128 bits are not all set. Rows past
// the sequence end are read as zeros by the 3-D tensor maps and never stored.
// Queries may sit at an offset among the keys (new tokens over a KV cache:
// query row i at key position q_off + i).
//
// Grid: query blocks heaviest-first. When all K/V is well beyond L2, the
// query blocks of one (batch, head) run side by side and share its K/V in L2
// (fewer DRAM reads: under the power cap the SM clock rises); otherwise
// (batch, head) varies fastest, for a globally heaviest-first schedule.
//
// Replaces the reference's attention call, F.scaled_dot_product_attention
// with is_causal=True inside _fast_attention_impl
// (torch_transformer_benchmark.py:718-818; scale hd^-0.5 at :215):
// softmax(Q K^T * scale + causal mask) V per head, fp32 statistics.
#include "internal.h"
#include "ptx.cuh"

namespace tfx {
namespace {

constexpr int kTcThreads = 352;
constexpr int kTile = 128;            // query rows per tile = keys per KV tile
constexpr float kRescaleLog2 = 8.0f;  // lazy-rescale threshold (P <= 2^8)
// Of every 8 pairs of scores, this many take 2^x from the FMA-pipe polynomial
// (exp2_poly_f2) and the rest from the MUFU unit (16 results per clock per
// SM), which alone bounds the softmax at head_dim 64.
#ifndef TFX_ATTN_POLY_OF8
#define TFX_ATTN_POLY_OF8 2
#endif
constexpr int kPolyOf8 = TFX_ATTN_POLY_OF8;
constexpr uint32_t kTmemCols = 512;

template <int HD>
struct TcAttn {
  // Query tiles per CTA: two share each K/V tile; head_dim 256 has room
  // (TMEM: S 128 + P 64 + O 256 columns; shared memory: Q, K, V 64 KB each)
  // for one.
  static constexpr int kNT = HD == 256 ? 1 : 2;
  static constexpr int kStages = HD == 64 ? 4 : (HD == 128 ? 2 : 1);
  static constexpr int kBlocks = HD / 64;            // 128-byte column blocks per row
  static constexpr int kBlockBytes = kTile * 128;    // one 64-column block of a tile
  static constexpr int kTileBytes = kTile * HD * 2;  // one Q/K/V tile, fp16
  static constexpr int kVtBoxBytes = HD * 128;        // V^T box: HD rows x 64 keys
  static constexpr int kQ = 0;                        // Q_A (, Q_B)
  static constexpr int kK = kNT * kTileBytes;
  static constexpr int kV = kK + kStages * kTileBytes;
  static constexpr int kBar = kV + kStages * kTileBytes;
  static constexpr int kSmem = kBar + 512 + 1024;    // barriers + alignment slack
  static constexpr bool kSepP = HD != 128;                // P has its own TMEM columns
  static constexpr uint32_t kColP = kSepP ? kNT * kTile : 0;
  static constexpr uint32_t kPStride = kSepP ? kTile / 2 : kTile;
  static constexpr uint32_t kColO = kNT == 1 ? 2 * kTile : (kSepP ? 3 * kTile : 2 * kTile);
  static_assert(kColO + kNT * HD <= kTmemCols, "TMEM budget");
  static_assert(kSmem <= 227 * 1024, "shared-memory budget");
};

template <int HD, bool CAUSAL, bool VT>
__global__ void __launch_bounds__(kTcThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tm_q,
                        const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, __half* __restrict__ out,
                        int64_t ld_out, int heads, int q_len, int nqb, int kv_len, int q_off,
                        float scale_log2, const int32_t* __restrict__ valid_len,
                        const uint32_t* __restrict__ key_bits, int key_words, int bh_in_y,
                        int* err) {
  grid_dep_wait();
  grid_dep_launch();
  using L = TcAttn<HD>;
  constexpr int S = L::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* q_full = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* k_full = q_full + 1;
  uint64_t* v_full = k_full + S;
  // K and V stages are released separately (K after its QK^T, V after its
  // P.V), per query tile: with one stage the next K must load before P.V.
  uint64_t* k_empty = v_full + S;       // [2][S]
  uint64_t* v_empty = k_empty + 2 * S;  // [2][S]
  uint64_t* s_full = v_empty + 2 * S;   // [2]: S_X computed
  uint64_t* s_free = s_full + 2;    // [2]: S_X read into registers (separate P only), 4 warps
  uint64_t* p_full = s_free + 2;    // [2]: P_X written (and O_X rescaled), 4 warps arrive
  uint64_t* o_done = p_full + 2;    // [2]: O_X += P_X V completed
  uint64_t* drain = o_done + 2;     // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // bh_in_y: grid x = query block, y = batch * heads, so the CTAs running at
  // once are mostly query blocks of one (b, h) and share its K/V in L2.
  // Otherwise x = batch * heads (globally heaviest-first order).
  const int bh = static_cast<int>(bh_in_y ? blockIdx.y : blockIdx.x);
  const int qblk = static_cast<int>(bh_in_y ? blockIdx.x : blockIdx.y);
  const int h = bh % heads;
  const int b = bh / heads;
  // Causal: the heaviest query blocks (the last ones) are launched first.
  const int qb = CAUSAL ? nqb - 1 - qblk : qblk;
  const int q0 = qb * L::kNT * kTile;
  // Query row i of this sequence sits at key position q_off + i (q_off > 0:
  // new tokens attending a KV cache); causal rows see keys <= their position.
  const int kend = valid_len ? min(kv_len, max(0, valid_len[b])) : kv_len;
  auto tiles_for = [&](int qx) {
    if (qx >= q_len) return 0;
    const int lim = CAUSAL ? min(kend, q_off + qx + kTile) : kend;
    return (lim + kTile - 1) / kTile;
  };
  const int nA = tiles_for(q0);
  const int nB = L::kNT == 2 ? tiles_for(q0 + kTile) : 0;
  const int n_iter = max(nA, nB);

  if (threadIdx.x == 0) {
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
    mbar_init(q_full, 1);
    for (int s = 0; s < S; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      for (int x = 0; x < 2; ++x) {
        mbar_init(&k_empty[x * S + s], 1);
        mbar_init(&v_empty[x * S + s], 1);
      }
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&s_free[x], 4);
      mbar_init(&p_full[x], 4);
      mbar_init(&o_done[x], 1);
    }
    mbar_init(&drain[0], 1);
    mbar_init(&drain[1], 1);
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
      mbar_arrive_expect_tx(q_full, L::kNT * L::kTileBytes);
#pragma unroll
      for (int x = 0; x < L::kNT; ++x)
#pragma unroll
        for (int cb = 0; cb < L::kBlocks; ++cb)
          tma_load_3d(smem + L::kQ + x * L::kTileBytes + cb * L::kBlockBytes, &tm_q, q_full,
                      col0 + 64 * cb, q0 + x * kTile, b);
      int issued = 0, k_issued = 0;
      for (int j = 0; j < n_iter; ++j) {
        const int st = j % S;
        // Stage st last held tile j - S: wait for the query tiles that used it.
        const uint32_t par = ((j / S) - 1) & 1;
        if (j >= S) {
          if (j - S < nA && !mbar_wait(&k_empty[st], par, err, kDevTimeoutEmpty)) break;
          if (j - S < nB && !mbar_wait(&k_empty[S + st], par, err, kDevTimeoutEmpty)) break;
        }
        mbar_arrive_expect_tx(&k_full[st], L::kTileBytes);
#pragma unroll
        for (int cb = 0; cb < L::kBlocks; ++cb)
          tma_load_3d(smem + L::kK + st * L::kTileBytes + cb * L::kBlockBytes, &tm_k, &k_full[st],
                      col0 + 64 * cb, j * kTile, b);
        k_issued = j + 1;
        if (j >= S) {
          if (j - S < nA && !mbar_wait(&v_empty[st], par, err, kDevTimeoutEmpty)) break;
          if (j - S < nB && !mbar_wait(&v_empty[S + st], par, err, kDevTimeoutEmpty)) break;
        }
        mbar_arrive_expect_tx(&v_full[st], L::kTileBytes);
        if constexpr (VT) {  // V^T rows h*HD.. (+HD), keys j*128.. in two 64-key boxes
#pragma unroll
          for (int kb = 0; kb < 2; ++kb)
            tma_load_3d(smem + L::kV + st * L::kTileBytes + kb * L::kVtBoxBytes, &tm_v,
                        &v_full[st], j * kTile + 64 * kb, col0, b);
        } else {
#pragma unroll
          for (int cb = 0; cb < L::kBlocks; ++cb)
            tma_load_3d(smem + L::kV + st * L::kTileBytes + cb * L::kBlockBytes, &tm_v,
                        &v_full[st], col0 + 64 * cb, j * kTile, b);
        }
        issued = j + 1;
      }
      // Our own copies land before the CTA may exit (after a timeout nobody
      // else waits for them); on the normal path these phases are complete.
      mbar_wait(q_full, 0, nullptr, 0);
      for (int j = max(0, k_issued - S); j < k_issued; ++j)
        mbar_wait(&k_full[j % S], (j / S) & 1, nullptr, 0);
      for (int j = max(0, issued - S); j < issued; ++j)
        mbar_wait(&v_full[j % S], (j / S) & 1, nullptr, 0);
    }
  } else if (warp == 1 || warp == 10) {
    // ------------------------------------------------ MMA issuer of tile x
    if (lane == 0) {
      const int x = warp == 1 ? 0 : 1;
      const int nx = x == 0 ? nA : nB;
      uint64_t* k_free = k_empty + x * S;
      uint64_t* v_free = v_empty + x * S;
      constexpr uint32_t id_qk = idesc_f16_f32(kTile, kTile);
      constexpr uint32_t id_pv = VT ? idesc_f16_f32(kTile, HD) : idesc_f16_f32_bmn(kTile, HD);
      // Descriptors are built once; each MMA adds a constant to the 64-bit
      // value (address field in 16-byte units, bits 0-13; shared addresses
      // stay below 2^18 so the field never carries into the next one).
      const uint64_t dq0 = sdesc_k_sw128(smem_u32(smem + L::kQ));
      const uint64_t dk0 = sdesc_k_sw128(smem_u32(smem + L::kK));
      const uint64_t dv0 = VT ? sdesc_k_sw128(smem_u32(smem + L::kV))
                              : sdesc_mn_sw128(smem_u32(smem + L::kV), L::kBlockBytes);
      // S_x = Q_x K^T: both operands K-major; K advances 16 columns = 32 B
      // inside a 128-byte swizzled row, then to the next 64-column block.
      auto issue_qk = [&](int x, int st) {
        const uint64_t da = dq0 + static_cast<uint64_t>(x * (L::kTileBytes >> 4));
        const uint64_t db = dk0 + static_cast<uint64_t>(st * (L::kTileBytes >> 4));
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint64_t off = static_cast<uint64_t>(((k >> 2) * L::kBlockBytes + (k & 3) * 32) >> 4);
          mma_f16_ss(tmem + x * kTile, da + off, db + off, id_qk, k > 0 ? 1u : 0u);
        }
      };
      // O_x += P_x V: P from TMEM (16 keys = 8 packed columns per step).
      // V^T K-major: 16 keys = 32 B inside a 128-byte row, 64 keys per box.
      // V MN-major: 16 keys = 16 rows = 2048 B; 64-column blocks one block apart.
      auto issue_pv = [&](int x, int st, bool accumulate) {
        const uint64_t db = dv0 + static_cast<uint64_t>(st * (L::kTileBytes >> 4));
#pragma unroll
        for (int k = 0; k < kTile / 16; ++k) {
          const uint64_t bdesc = db + static_cast<uint64_t>(
              (VT ? (k >> 2) * L::kVtBoxBytes + (k & 3) * 32 : k * 2048) >> 4);
          mma_f16_ts(tmem + L::kColO + x * HD, tmem + L::kColP + x * L::kPStride + 8 * k, bdesc,
                     id_pv, (accumulate || k > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(q_full, 0, err, kDevTimeoutFull);
      if (ok && nx > 0) {
        ok = mbar_wait(&k_full[0], 0, err, kDevTimeoutFull);
        if (ok) {
          tc_fence_after();
          issue_qk(x, 0);
          mma_commit(&s_full[x]);
          mma_commit(&k_free[0]);
        }
      }
      for (int j = 0; ok && j < nx; ++j) {
        const int st = j % S, st1 = (j + 1) % S;
        const uint32_t par = (j / S) & 1, par1 = ((j + 1) / S) & 1;
        const uint32_t jp = j & 1;
        if constexpr (L::kSepP) {
          // S_X(j) is read early in its softmax, P_X(j) written late: the
          // next product is queued before this tile's P.V.
          if (j + 1 < nx) {
            if (!mbar_wait(&k_full[st1], par1, err, kDevTimeoutFull)) break;
            if (!mbar_wait(&s_free[x], jp, err, kDevTimeoutOther)) break;
            tc_fence_after();
            issue_qk(x, st1);
            mma_commit(&s_full[x]);
            mma_commit(&k_free[st1]);  // K_{j+1} is free for this tile
          }
          if (!mbar_wait(&v_full[st], par, err, kDevTimeoutFull)) break;
          if (!mbar_wait(&p_full[x], jp, err, kDevTimeoutOther)) break;
          tc_fence_after();
          issue_pv(x, st, j > 0);
          mma_commit(&o_done[x]);
          mma_commit(&v_free[st]);  // V_j is free for this tile
        } else {
          if (!mbar_wait(&v_full[st], par, err, kDevTimeoutFull)) break;
          if (!mbar_wait(&p_full[x], jp, err, kDevTimeoutOther)) break;
          tc_fence_after();
          issue_pv(x, st, j > 0);
          mma_commit(&o_done[x]);
          mma_commit(&v_free[st]);
          if (j + 1 < nx) {
            // S_X(j+1) overwrites P_X(j): wait for PV_X(j) to finish reading it.
            if (!mbar_wait(&k_full[st1], par1, err, kDevTimeoutFull)) break;
            if (!mbar_wait(&o_done[x], jp, err, kDevTimeoutAccum)) break;
            tc_fence_after();
            issue_qk(x, st1);
            mma_commit(&s_full[x]);
            mma_commit(&k_free[st1]);
          }
        }
      }
      // Every MMA this thread issued completes before TMEM is released.
      mma_commit(&drain[x]);
      mbar_wait(&drain[x], 0, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int x = (warp - 2) >> 2;  // 0: tile A, 1: tile B
    if (x < L::kNT) {
    const int quarter = warp & 3;   // this warp's TMEM lanes [32*quarter, +32)
    const int row = quarter * 32 + lane;
    const int qx = q0 + x * kTile;
    const int q = qx + row;
    const int nx = x == 0 ? nA : nB;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t t_s = tmem + lane_off + x * kTile;
    const uint32_t t_p = tmem + lane_off + L::kColP + x * L::kPStride;
    const uint32_t t_o = tmem + lane_off + L::kColO + x * HD;
    const int lim_row = CAUSAL ? min(kend, q_off + q + 1) : kend;  // keys [0, lim_row) visible
    const int lim_tile = CAUSAL ? min(kend, q_off + qx + 1) : kend;  // smallest of the tile
    float m_ref = 0.f;
    uint64_t lsum0 = 0, lsum1 = 0;
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
      if constexpr (L::kSepP) {  // S_X is in registers: the next S_X may be computed
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[x]);
      }
      if ((j + 1) * kTile > lim_tile) {  // diagonal or ragged KV tile (warp-uniform)
        const int c0 = lim_row - j * kTile;
#pragma unroll
        for (int c = 0; c < kTile; ++c)
          if (c >= c0) s[c] = 0xff800000u;  // -inf
      }
      if (key_bits != nullptr) {
        // Key padding of any pattern: bit k of the tile's 128-bit word is key
        // j*128 + k (same for every row: uniform loads, L1 broadcast).
        uint32_t kw[4];
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const int wi = 4 * j + w;
          kw[w] = wi < key_words ? key_bits[static_cast<int64_t>(b) * key_words + wi] : 0u;
        }
        if ((kw[0] & kw[1] & kw[2] & kw[3]) != 0xffffffffu) {
#pragma unroll
          for (int c = 0; c < kTile; ++c)
            if (!((kw[c >> 5] >> (c & 31)) & 1u)) s[c] = 0xff800000u;
        }
      }
      float mm[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mm[i] = fmaxf(__uint_as_float(s[i]), __uint_as_float(s[i + 8]));
#pragma unroll
      for (int c = 16; c < kTile; c += 16)
#pragma unroll
        for (int i = 0; i < 8; ++i) mm[i] = fmax3(mm[i], __uint_as_float(s[c + i]), __uint_as_float(s[c + 8 + i]));
      const float mx = fmaxf(fmax3(mm[0], mm[1], mm[2]), fmax3(fmax3(mm[3], mm[4], mm[5]), mm[6], mm[7]));
      const float m_new = mx * scale_log2;  // -inf when every key of the row is masked
      bool rescale = false;
      float f = 1.f;
      if (j == 0) {
        m_ref = mx == -INFINITY ? 0.f : m_new;
      } else if (__any_sync(0xffffffffu, m_new > m_ref + kRescaleLog2)) {
        const float m_up = fmaxf(m_ref, m_new);
        f = fast_exp2(m_ref - m_up);
        m_ref = m_up;
        const uint64_t f2v = f2_pack(f, f);
        lsum0 = f2_fma(lsum0, f2v, 0);
        lsum1 = f2_fma(lsum1, f2v, 0);
        rescale = true;
      }
      const uint64_t c2 = f2_pack(scale_log2, scale_log2);
      const uint64_t negm2 = f2_pack(-m_ref, -m_ref);
      // P in two halves of 64 keys (32 packed columns each), so S and P never
      // need registers at the same time.
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t p[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int c = 64 * half + 2 * i;
          const uint64_t arg = f2_fma(f2_pack(__uint_as_float(s[c]), __uint_as_float(s[c + 1])), c2, negm2);
          uint64_t e;
          if ((i & 7) < kPolyOf8) {
            e = exp2_poly_f2(arg);
          } else {
            float a0, a1;
            f2_unpack(arg, a0, a1);
            e = f2_pack(fast_exp2(a0), fast_exp2(a1));
          }
          if (i & 1) lsum1 = f2_add(lsum1, e); else lsum0 = f2_add(lsum0, e);
          float e0, e1;
          f2_unpack(e, e0, e1);
          p[i] = pack_half2(e0, e1);
        }
        if (half == 0) {
          if constexpr (L::kSepP) {
            // P_X(j-1) and O_X are read / written by PV_X(j-1) until it completes.
            if (j > 0 && !__all_sync(0xffffffffu,
                                     mbar_wait(&o_done[x], (j - 1) & 1, err, kDevTimeoutAccum))) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          // (HD 128: PV_X(j-1) completed before S_X(j) was issued.)
          if (rescale) {
#pragma unroll 1
            for (int c = 0; c < HD; c += 16) {
              uint32_t o[16];
              tmem_ld16(t_o + c, o);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
              tmem_st16(t_o + c, o);
            }
          }
        }
        tmem_st32(t_p + 32 * half, p);
      }
      if (!ok) break;
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[x]);
    }
    if (ok && nx > 0)
      ok = __all_sync(0xffffffffu, mbar_wait(&o_done[x], (nx - 1) & 1, err, kDevTimeoutAccum));
    float la, lb, lc, ld;
    f2_unpack(lsum0, la, lb);
    f2_unpack(lsum1, lc, ld);
    const float l = (la + lb) + (lc + ld);
    const float inv = l > 0.f ? 1.f / l : 0.f;
    __half* dst = out + (static_cast<int64_t>(b) * q_len + q) * ld_out + h * HD;
    if (ok && nx > 0) {
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < HD; c += 32) {
        uint32_t o[32];
        tmem_ld32(t_o + c, o);
        tmem_ld_wait();
        if (q < q_len) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float* f = reinterpret_cast<const float*>(o + 8 * i);
            d4[i] = make_uint4(pack_half2(f[0] * inv, f[1] * inv), pack_half2(f[2] * inv, f[3] * inv),
                               pack_half2(f[4] * inv, f[5] * inv), pack_half2(f[6] * inv, f[7] * inv));
          }
        }
      }
    } else if (ok && q < q_len) {
      // No visible key (valid_len 0): the output row is zero.
      uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
      for (int i = 0; i < HD / 8; ++i) d4[i] = make_uint4(0, 0, 0, 0);
    }
    }  // x < kNT
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// vt[b][c][s] = v[b * seq + s][c] for c < cols, s < seq; zero for seq <= s < ld_vt.
// Each lane transposes one 8-key x 8-column block in registers: eight 16-byte
// row loads, 32 byte permutes, eight 16-byte column stores. A warp covers 32
// keys x 64 columns (per load instruction 4 rows x 128 contiguous bytes; per
// store 8 output rows x 64 contiguous bytes); a CTA of 8 warps 128 keys x
// 128 columns. No shared memory: every lane keeps 8 loads in flight.
__global__ void __launch_bounds__(256)
    transpose_v_kernel(const __half* __restrict__ v, int64_t ld_qkv, __half* __restrict__ vt,
                       int64_t ld_vt, int seq, int cols) {
  grid_dep_wait();
  grid_dep_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z;
  const int s0 = blockIdx.x * 128 + (warp & 3) * 32 + (lane >> 3) * 8;  // first key
  const int c0 = blockIdx.y * 128 + (warp >> 2) * 64 + (lane & 7) * 8;   // first column
  if (c0 >= cols || s0 >= ld_vt) return;
  uint4 r[8];
#pragma unroll
  for (int k = 0; k < 8; ++k)
    r[k] = (s0 + k < seq) ? __ldcs(reinterpret_cast<const uint4*>(
                                v + (static_cast<int64_t>(b) * seq + s0 + k) * ld_qkv + c0))
                          : make_uint4(0u, 0u, 0u, 0u);
  // Word j of row k holds columns 2j, 2j+1; word m of output column c holds
  // keys 2m, 2m+1: low halves pair up for the even column, high for the odd.
  const uint32_t* w = reinterpret_cast<const uint32_t*>(r);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t lo[4], hi[4];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      lo[m] = __byte_perm(w[8 * m + j], w[8 * m + 4 + j], 0x5410);
      hi[m] = __byte_perm(w[8 * m + j], w[8 * m + 4 + j], 0x7632);
    }
    __half* dst = vt + (static_cast<int64_t>(b) * cols + c0 + 2 * j) * ld_vt + s0;
    __stcs(reinterpret_cast<uint4*>(dst), make_uint4(lo[0], lo[1], lo[2], lo[3]));
    __stcs(reinterpret_cast<uint4*>(dst + ld_vt), make_uint4(hi[0], hi[1], hi[2], hi[3]));
  }
}

template <int HD, bool CAUSAL, bool VT>
int launch_tc(const __half* q, int64_t ld_q, const __half* k, const __half* v, int64_t ld_vt,
              __half* out, int64_t ld_out, int batch, int heads, int q_len, const AttnKv& kv,
              float scale, const KeyMask& km, cudaStream_t stream) {
  using L = TcAttn<HD>;
  static int smem_done[kMaxDevices] = {0};
  auto kern = attention_tc_kernel<HD, CAUSAL, VT>;
  int st = ensure_smem(reinterpret_cast<const void*>(kern), L::kSmem, smem_done);
  if (st != TFX_OK) return st;
  const uint64_t cols = static_cast<uint64_t>(heads) * HD;
  const uint64_t kv_len = static_cast<uint64_t>(kv.len);
  const uint64_t kv_bstride = static_cast<uint64_t>(kv.batch_rows) * static_cast<uint64_t>(kv.ld);
  CUtensorMap tq, tk, tv;
  // K/V rows at or past kv.len read as zeros (TMA out-of-bounds fill), so a
  // partly used last tile never multiplies a masked score by stale data.
  st = make_tmap_3d(&tq, q, static_cast<uint64_t>(q_len), static_cast<uint64_t>(batch), cols,
                    static_cast<uint64_t>(ld_q),
                    static_cast<uint64_t>(q_len) * static_cast<uint64_t>(ld_q), 64, kTile);
  if (st == TFX_OK)
    st = make_tmap_3d(&tk, k, kv_len, static_cast<uint64_t>(batch), cols,
                      static_cast<uint64_t>(kv.ld), kv_bstride, 64, kTile);
  if (st == TFX_OK) {
    if (VT)  // [batch][cols][ld_vt]: keys innermost, keys >= kv.len read as zeros
      st = make_tmap_3d(&tv, v, cols, static_cast<uint64_t>(batch), kv_len,
                        static_cast<uint64_t>(ld_vt), cols * static_cast<uint64_t>(ld_vt), 64, HD);
    else
      st = make_tmap_3d(&tv, v, kv_len, static_cast<uint64_t>(batch), cols,
                        static_cast<uint64_t>(kv.ld), kv_bstride, 64, kTile);
  }
  if (st != TFX_OK) return st;
  const int nqb = (q_len + L::kNT * kTile - 1) / (L::kNT * kTile);
  // Query blocks of one (b, h) side by side when all K/V is well beyond L2
  // (long sequences): fewer DRAM reads lower the power draw, and under the
  // power cap the SM clock rises (B=4, S=100k, hd 64: 1488 -> 1739 MHz,
  // 122.6 -> 105.4 ms at equal cycles). Below that, (b, h)-fastest order keeps
  // the global heaviest-first schedule (S=32k, B=1: 5.6 % faster).
  const unsigned bh = static_cast<unsigned>(batch) * static_cast<unsigned>(heads);
  const double kv_bytes = 4.0 * static_cast<double>(bh) * static_cast<double>(kv.len) * HD;
  const int bh_in_y = (bh <= 65535u && nqb >= 4 && kv_bytes > 256.0 * (1 << 20)) ? 1 : 0;
  const dim3 grid = bh_in_y ? dim3(static_cast<unsigned>(nqb), bh) : dim3(bh, static_cast<unsigned>(nqb));
  launch_pdl(kern, grid, dim3(kTcThreads), L::kSmem, stream, tq, tk, tv, out, ld_out, heads, q_len,
             nqb, kv.len, kv.q_off, scale * 1.4426950408889634f, km.len, km.bits,
             key_words(kv.len), bh_in_y, device_error_word());
  return check_launch("attention_tc_kernel");
}

template <int HD, bool VT>
int launch_tc_c(const __half* q, int64_t ld_q, const __half* k, const __half* v, int64_t ld_vt,
                __half* out, int64_t ld_out, int batch, int heads, int q_len, const AttnKv& kv,
                float scale, int causal, const KeyMask& km, cudaStream_t stream) {
  return causal ? launch_tc<HD, true, VT>(q, ld_q, k, v, ld_vt, out, ld_out, batch, heads, q_len,
                                          kv, scale, km, stream)
                : launch_tc<HD, false, VT>(q, ld_q, k, v, ld_vt, out, ld_out, batch, heads, q_len,
                                           kv, scale, km, stream);
}

template <bool VT>
int dispatch_tc(const __half* q, int64_t ld_q, const __half* k, const __half* v, int64_t ld_vt,
                __half* out, int64_t ld_out, int batch, int heads, int q_len, const AttnKv& kv,
                int head_dim, float scale, int causal, const KeyMask& km,
                cudaStream_t stream) {
  if (static_cast<int64_t>(batch) * heads > 0x7fffffff || (q_len + kTile - 1) / kTile > 65535)
    return fail(TFX_ERR_UNSUPPORTED, "tfx_attention: batch*heads or seq too large for the grid");
  if (head_dim == 64)
    return launch_tc_c<64, VT>(q, ld_q, k, v, ld_vt, out, ld_out, batch, heads, q_len, kv, scale,
                               causal, km, stream);
  if (head_dim == 128)
    return launch_tc_c<128, VT>(q, ld_q, k, v, ld_vt, out, ld_out, batch, heads, q_len, kv, scale,
                                causal, km, stream);
  if (head_dim == 256)
    return launch_tc_c<256, VT>(q, ld_q, k, v, ld_vt, out, ld_out, batch, heads, q_len, kv, scale,
                                causal, km, stream);
  return fail(TFX_ERR_UNSUPPORTED, "attention_tc: head_dim %d not in {64,128,256}", head_dim);
}

}  // namespace

bool attention_tc_supported(int head_dim, float scale) {
  return (head_dim == 64 || head_dim == 128 || head_dim == 256) && scale > 0.f;
}

int launch_attention_tc(const __half* q, const __half* k, const __half* v, int64_t ld_qkv,
                        __half* out, int64_t ld_out, int batch, int heads, int seq, int head_dim,
                        float scale, int causal, const KeyMask& km, cudaStream_t stream) {
  return dispatch_tc<false>(q, ld_qkv, k, v, 0, out, ld_out, batch, heads, seq,
                            AttnKv{ld_qkv, seq, seq, 0}, head_dim, scale, causal, km, stream);
}

int64_t attention_vt_ld(int seq) { return (static_cast<int64_t>(seq) + 7) / 8 * 8; }

int launch_transpose_v(const __half* v, int64_t ld_qkv, __half* vt, int batch, int seq,
                       int cols, cudaStream_t stream) {
  const int64_t ld_vt = attention_vt_ld(seq);
  const dim3 grid(static_cast<unsigned>((ld_vt + 127) / 128), static_cast<unsigned>((cols + 127) / 128),
                  static_cast<unsigned>(batch));
  launch_pdl(transpose_v_kernel, grid, dim3(256), 0, stream, v, ld_qkv, vt, ld_vt, seq, cols);
  return check_launch("transpose_v_kernel");
}

int launch_attention_tc_kv(const __half* q, int64_t ld_q, const __half* k, const __half* v,
                           const AttnKv& kv, __half* out, int64_t ld_out, int batch, int heads,
                           int q_len, int head_dim, float scale, cudaStream_t stream) {
  return dispatch_tc<false>(q, ld_q, k, v, 0, out, ld_out, batch, heads, q_len, kv, head_dim,
                            scale, 1, KeyMask{}, stream);
}

int launch_attention_tc_vt(const __half* q, const __half* k, const __half* vt, int64_t ld_qkv,
                           __half* out, int64_t ld_out, int batch, int heads, int seq,
                           int head_dim, float scale, int causal, const KeyMask& km,
                           cudaStream_t stream) {
  return dispatch_tc<true>(q, ld_qkv, k, vt, attention_vt_ld(seq), out, ld_out, batch, heads, seq,
                           AttnKv{ld_qkv, seq, seq, 0}, head_dim, scale, causal, km, stream);
}

}  // namespace tfx
