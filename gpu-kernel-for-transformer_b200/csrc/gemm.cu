// Persistent, warp-specialised tcgen05 GEMM with fused epilogues.
//
//   out[m, n] = epi( sum_k A[m, k] * W[n, k] + bias[n] (, residual[m, n]) )
//
// A (activations) and W (nn.Linear weight, [out, in]) are fp16 and K-major,
// so both feed tcgen05.mma directly from 128-byte-swizzled shared memory
// written by TMA. The fp32 accumulator lives in TMEM, double-buffered so the
// epilogue of tile i overlaps the MMAs of tile i+1.
//
// CTA = 10 warps, one CTA per SM, grid = min(#tiles, #SMs):
//   warp 0      TMA producer (one lane): A and W k-blocks into a STAGES ring
//   warp 1      TMEM allocator + MMA issuer (one lane)
//   warps 2..9  epilogue, two warps per TMEM lane quarter (warp w may only
//               touch lanes [32*(w%4), +32)), each taking half of a tile's
//               columns: tcgen05.ld rows out of TMEM, then through a per-warp
//               shared-memory staging tile so that the bias / exact-erf GELU
//               (gelu_poly_f2) / residual work, the residual loads and the
//               output stores are row-contiguous and coalesced (a lane per
//               row would touch 32 rows per warp-wide access).
#include "internal.h"
#include "ptx.cuh"

namespace tfx {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;  // 64 fp16 = one 128-byte swizzle row
// Epilogue warps: two per TMEM lane quarter (SM sub-partition), each taking
// half of a tile's columns. One warp per sub-partition was latency-bound:
// a 128x256 tile's epilogue took ~10 us against ~5.4 us of MMAs.
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;

template <int BN, int STAGES>
struct GemmLayout {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOffset = STAGES * kStageBytes;
  // Epilogue staging: per epilogue warp 32 rows x 32 fp32 columns; the eight
  // 16-byte chunks of row r sit at chunk index j ^ (r & 7), so the lane-per-row
  // writes and the row-contiguous reads are both conflict-free.
  static constexpr int kStgStride = 32;
  static constexpr int kStgOffset = kBarOffset + 256;
  static constexpr int kStgBytes = kEpiWarps * 32 * kStgStride * 4;
  // Columns of a tile per epilogue warp (BN 32: one warp of each pair idles).
  static constexpr int kEpiCols = BN >= 64 ? BN / 2 : BN;
  static constexpr int kSmemBytes = kStgOffset + kStgBytes + 1024;  // + 1 KB alignment slack
  static_assert(kSmemBytes <= 227 * 1024, "shared-memory budget");
  // Two accumulator buffers; TMEM allocations are powers of two >= 32 columns.
  static constexpr uint32_t kTmemCols = 2 * BN <= 32 ? 32 : 2 * BN <= 64 ? 64 : 2 * BN <= 128 ? 128
                                      : 2 * BN <= 256 ? 256 : 512;
};

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                   const float* __restrict__ bias, const float* residual, void* out, int M, int N,
                   int K, int64_t ldr, int64_t ldo, int* err) {
  using L = GemmLayout<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Tiles in N-fastest order: the CTAs running at once share a few A row
  // blocks (read from DRAM once, then from L2) and all of W; M-fastest order
  // streamed the whole of A once per N block (c5 QKV: 2.46 GB of DRAM reads
  // for a 205 MB A).
  const int tiles_m = (M + kBM - 1) / kBM;
  const int tiles_n = N / BN;
  const int num_tiles = tiles_m * tiles_n;
  const int kblocks = (K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmW);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 32 * kEpiWarps);
    }
    fence_mbar_init();
  }
  grid_dep_wait();
  grid_dep_launch();
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------ TMA producer
    int stage = 0;
    uint32_t phase = 0;
    int issued_parity[STAGES];
    for (int s = 0; s < STAGES; ++s) issued_parity[s] = -1;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      const int m0 = (tile / tiles_n) * kBM;
      const int n0 = (tile % tiles_n) * BN;
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1, err, kDevTimeoutEmpty)) {
          ok = false;
          break;
        }
        uint8_t* sa = smem + stage * L::kStageBytes;
        mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
        tma_load_2d(sa, &tmA, &full[stage], kb * kBK, m0);
        tma_load_2d(sa + L::kABytes, &tmW, &full[stage], kb * kBK, n0);
        issued_parity[stage] = static_cast<int>(phase);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    if (!ok) {
      // Unwinding after a timeout: let our own copies land before exit.
      for (int s = 0; s < STAGES; ++s)
        if (issued_parity[s] >= 0) mbar_wait(&full[s], issued_parity[s], nullptr, 0);
    }
  } else if (warp == 1 && lane == 0) {
    // --------------------------------------------------------- MMA issuer
    constexpr uint32_t idesc = idesc_f16_f32(kBM, BN);
    // Descriptors built once; per stage and k-step a constant is added to the
    // 64-bit value (address field in 16-byte units, no carry below 2^18 B).
    const uint64_t da0 = sdesc_k_sw128(smem_u32(smem));
    const uint64_t db0 = sdesc_k_sw128(smem_u32(smem + L::kABytes));
    int stage = 0;
    uint32_t phase = 0;
    int local = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
      const int buf = local & 1;
      const uint32_t use = static_cast<uint32_t>(local >> 1);
      if (!mbar_wait(&acc_empty[buf], (use & 1) ^ 1, err, kDevTimeoutAccumFree)) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * BN);
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!mbar_wait(&full[stage], phase, err, kDevTimeoutFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t soff = static_cast<uint64_t>(stage * (L::kStageBytes >> 4));
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {
          mma_f16_ss(d_tmem, da0 + soff + 2 * k, db0 + soff + 2 * k, idesc,
                     (kb | k) != 0 ? 1u : 0u);
        }
        mma_commit(&empty[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (ok) mma_commit(&acc_full[buf]);
    }
  } else if (warp >= 2) {
    // ----------------------------------------------------------- epilogue
    const int quarter = warp & 3;
    // This warp's columns of every tile: [cbeg, cend). (BN 32: the second
    // warp of each pair has none; it still waits and arrives with the others
    // so the accumulator barriers keep their counts.)
    const int cbeg = ((warp - 2) >> 2) * L::kEpiCols;
    const int cend = cbeg + L::kEpiCols <= BN ? cbeg + L::kEpiCols : cbeg;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int buf = local & 1;
      const uint32_t use = static_cast<uint32_t>(local >> 1);
      // Warp-uniform outcome (the TMEM loads below are warp-collective).
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[buf], use & 1, err, kDevTimeoutAccum)))
        break;
      tc_fence_after();
      const int m0 = (tile / tiles_n) * kBM;
      const int n0 = (tile % tiles_n) * BN;
      const int wrow0 = m0 + quarter * 32;  // this warp's 32 rows
      const uint32_t t_row =
          tmem_base + static_cast<uint32_t>(buf * BN) + (static_cast<uint32_t>(quarter * 32) << 16);
      float* stg = reinterpret_cast<float*>(smem + L::kStgOffset) + (warp - 2) * 32 * L::kStgStride;
      // Residual chunks: 8 lanes x float4 = one row's 32 columns, 4 rows per
      // pass, 8 passes; all 8 loads are issued before the TMEM read so they
      // are in flight while the accumulator is staged.
      const int rsub = lane >> 3, rc4 = (lane & 7) * 4;
      float4 res[8], nxt[8];
      auto load_res = [&](float4 (&dst)[8], int c) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int row = wrow0 + rsub + 4 * i;
          // Read exactly once: evict-first, so the reused A/W tiles stay in L2.
          dst[i] = row < M ? __ldcs(reinterpret_cast<const float4*>(residual + row * ldr + n0 + c + rc4))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      };
      if (EPI == TFX_EPI_BIAS_RESIDUAL && cbeg < cend) load_res(nxt, cbeg);
      // The next chunk's TMEM load is in flight while this chunk is stored.
      uint32_t r[32];
      if (cbeg < cend) tmem_ld32(t_row + cbeg, r);
      const int sub = lane >> 2, c8 = (lane & 3) * 8;  // fp16 out: 4 lanes per row, 8 rows/pass
#pragma unroll 1
      for (int c = cbeg; c < cend; c += 32) {
        if constexpr (EPI == TFX_EPI_BIAS_RESIDUAL) {
          // This chunk's residual was loaded one chunk ahead; start the next.
#pragma unroll
          for (int i = 0; i < 8; ++i) res[i] = nxt[i];
          if (c + 32 < cend) load_res(nxt, c + 32);
        }
        tmem_ld_wait();
        // Lane = row: the raw accumulator into the staging tile.
        float4* srow = reinterpret_cast<float4*>(stg + lane * L::kStgStride);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          srow[j ^ (lane & 7)] =
              make_float4(__uint_as_float(r[4 * j + 0]), __uint_as_float(r[4 * j + 1]),
                          __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
        __syncwarp();
        if (c + 32 < cend) tmem_ld32(t_row + c + 32, r);
        // Row-contiguous phase: consecutive lanes take consecutive columns, so
        // each lane needs only its own columns' bias.
        if constexpr (EPI == TFX_EPI_BIAS_RESIDUAL) {
          const float4 bb = __ldg(reinterpret_cast<const float4*>(bias + n0 + c + rc4));
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int rr = rsub + 4 * i;
            const int row = wrow0 + rr;
            if (row < M) {
              const float4 v = reinterpret_cast<const float4*>(
                  stg + rr * L::kStgStride)[(rc4 >> 2) ^ (rr & 7)];
              *reinterpret_cast<float4*>(static_cast<float*>(out) + row * ldo + n0 + c + rc4) =
                  make_float4((v.x + bb.x) + res[i].x, (v.y + bb.y) + res[i].y,
                              (v.z + bb.z) + res[i].z, (v.w + bb.w) + res[i].w);
            }
          }
        } else {
          const float4 b0 = __ldg(reinterpret_cast<const float4*>(bias + n0 + c + c8));
          const float4 b1 = __ldg(reinterpret_cast<const float4*>(bias + n0 + c + c8 + 4));
#pragma unroll
          for (int rr = sub; rr < 32; rr += 8) {
            const int row = wrow0 + rr;
            if (row < M) {
              const float4* sr = reinterpret_cast<const float4*>(stg + rr * L::kStgStride);
              const float4 v0 = sr[(c8 >> 2) ^ (rr & 7)];
              const float4 v1 = sr[((c8 >> 2) + 1) ^ (rr & 7)];
              float e[8] = {v0.x + b0.x, v0.y + b0.y, v0.z + b0.z, v0.w + b0.w,
                            v1.x + b1.x, v1.y + b1.y, v1.z + b1.z, v1.w + b1.w};
              if constexpr (EPI == TFX_EPI_BIAS_GELU) {
#pragma unroll
                for (int u = 0; u < 8; u += 2)
                  f2_unpack(gelu_poly_f2(f2_pack(e[u], e[u + 1])), e[u], e[u + 1]);
              }
              *reinterpret_cast<uint4*>(static_cast<__half*>(out) + row * ldo + n0 + c + c8) =
                  make_uint4(pack_half2(e[0], e[1]), pack_half2(e[2], e[3]),
                             pack_half2(e[4], e[5]), pack_half2(e[6], e[7]));
            }
          }
        }
        __syncwarp();  // staging tile reused by the next chunk
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, L::kTmemCols);
}

template <int BN, int STAGES, int EPI>
int launch_gemm_t(const __half* a, int64_t lda, const __half* w, const float* bias,
                  const float* residual, int64_t ldr, void* out, int64_t ldo, int64_t m, int n,
                  int k, cudaStream_t stream) {
  using L = GemmLayout<BN, STAGES>;
  static int smem_done[kMaxDevices] = {0};
  auto kern = gemm_tc_kernel<BN, STAGES, EPI>;
  int st = ensure_smem(reinterpret_cast<const void*>(kern), L::kSmemBytes, smem_done);
  if (st != TFX_OK) return st;
  CUtensorMap tmA, tmW;
  st = make_tmap_2d(&tmA, a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, static_cast<uint64_t>(m),
                    static_cast<uint64_t>(k), static_cast<uint64_t>(lda), kBK, kBM,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != TFX_OK) return st;
  st = make_tmap_2d(&tmW, w, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, static_cast<uint64_t>(n),
                    static_cast<uint64_t>(k), static_cast<uint64_t>(k), kBK, BN,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != TFX_OK) return st;
  const int64_t tiles = ((m + kBM - 1) / kBM) * (n / BN);
  const int grid = static_cast<int>(tiles < num_sms() ? tiles : num_sms());
  launch_pdl(kern, dim3(grid), dim3(kThreads), L::kSmemBytes, stream, tmA, tmW, bias, residual,
             out, static_cast<int>(m), n, k, ldr, ldo, device_error_word());
  return check_launch("gemm_tc_kernel");
}

template <int EPI>
int launch_gemm_epi(const __half* a, int64_t lda, const __half* w, const float* bias,
                    const float* residual, int64_t ldr, void* out, int64_t ldo, int64_t m, int n,
                    int k, cudaStream_t stream) {
  // N tile: the tile count should fill the last wave of the persistent grid
  // (768 tiles of 256 on 148 SMs are 5.19 waves; 1024 tiles of 192 are 6.92),
  // but narrow tiles cost more per output: the mainloop is bound by shared-
  // memory bandwidth (TMA writes plus tensor-core operand reads), so a
  // 128x256 tile takes ~190 cycles per K=16 step (the measured cuBLAS rate)
  // and a 128x192 tile ~183. Score = wave efficiency x relative throughput.
  const int sms = num_sms();
  const int64_t mt = (m + kBM - 1) / kBM;
  auto score = [&](int bn, double per_tile) {
    if (n % bn != 0) return 0.0;
    const int64_t t = mt * (n / bn);
    const int64_t waves = (t + sms - 1) / sms;
    return per_tile * static_cast<double>(t) / static_cast<double>(waves * sms);
  };
  const double s256 = score(256, 1.0), s192 = score(192, 0.78), s128 = score(128, 0.70);
  if (s256 > 0 && s256 >= s192 && s256 >= s128)
    return launch_gemm_t<256, 4, EPI>(a, lda, w, bias, residual, ldr, out, ldo, m, n, k, stream);
  if (s192 > 0 && s192 >= s128)
    return launch_gemm_t<192, 4, EPI>(a, lda, w, bias, residual, ldr, out, ldo, m, n, k, stream);
  if (n % 128 == 0)
    return launch_gemm_t<128, 6, EPI>(a, lda, w, bias, residual, ldr, out, ldo, m, n, k, stream);
  if (n % 64 == 0)
    return launch_gemm_t<64, 8, EPI>(a, lda, w, bias, residual, ldr, out, ldo, m, n, k, stream);
  if (n % 32 == 0)
    return launch_gemm_t<32, 8, EPI>(a, lda, w, bias, residual, ldr, out, ldo, m, n, k, stream);
  return fail(TFX_ERR_UNSUPPORTED, "tfx_linear: n=%d must be a multiple of 32", n);
}

}  // namespace

int launch_linear(const __half* a, int64_t lda, const __half* w, const float* bias,
                  const float* residual, int64_t ldr, void* out, int64_t ldo, int64_t m, int n,
                  int k, int epilogue, cudaStream_t stream) {
  switch (epilogue) {
    case TFX_EPI_BIAS:
      return launch_gemm_epi<TFX_EPI_BIAS>(a, lda, w, bias, residual, ldr, out, ldo, m, n, k,
                                           stream);
    case TFX_EPI_BIAS_GELU:
      return launch_gemm_epi<TFX_EPI_BIAS_GELU>(a, lda, w, bias, residual, ldr, out, ldo, m, n, k,
                                                stream);
    case TFX_EPI_BIAS_RESIDUAL:
      return launch_gemm_epi<TFX_EPI_BIAS_RESIDUAL>(a, lda, w, bias, residual, ldr, out, ldo, m,
                                                    n, k, stream);
    default:
      return fail(TFX_ERR_INVALID_ARGUMENT, "tfx_linear: unknown epilogue %d", epilogue);
  }
}

}  // namespace tfx
