// K1 for large GEMMs on CTA pairs: the W8A8 matmul with 256 x BN tiles shared by the two CTAs
// of a 2-CTA cluster (tcgen05.mma.cta_group::2, M = 256).  Each CTA stages its own 128 rows of A
// and its half (BN/2 rows) of B, so per MMA instruction each SM's shared memory supplies half the
// operand bytes of a 128 x BN single-CTA tile of the same width; the even CTA issues the MMAs.
// Same arithmetic and epilogue as qgemm_sm100_kernel (qg_epilogue_chunk), so the results are
// identical bit for bit.  Persistent over tiles in bands of QG2_BAND row tiles so the A and B
// bands in flight stay in L2.
//
// Barriers (all waits bounded, like the single-CTA kernel):
//   full[s]   (even CTA)   both CTAs' loads of stage s landed: expect_tx by the even CTA's producer
//                          for both CTAs' bytes; each CTA's load counts its bytes there
//   empty[s]  (each CTA)   the MMAs reading stage s finished (one commit reaching both CTAs)
//   tfull[a]  (each CTA)   accumulator a of the tile is complete (one commit reaching both CTAs)
//   tempty[a] (even CTA)   both CTAs' epilogues read accumulator a (2 x EPI_THREADS arrivals,
//                          the odd CTA's arriving remotely)
// The CTA pair meets at a cluster barrier after barrier initialization (remote signals only reach
// initialized barriers) and before the tensor memory is freed (the odd CTA's shared memory and
// tensor memory stay valid until the even CTA's last MMA completed).
#pragma once
#include "qgemm_sm100.cuh"

namespace mira {

constexpr int QG2_BAND = 8;   // row tiles (of 256) per band of the tile order

template <int BN, int STAGES, int G>
struct Qg2Cfg {
  static constexpr int A_BYTES = QG_BM * QG_BK;           // this CTA's 128 rows
  static constexpr int B_BYTES = (BN / 2) * QG_BK;        // this CTA's half of the columns
  static constexpr int CW = 16;
  static constexpr int EPI_WARP0 = 2;
  static constexpr int EPI_WARPS = 4 * G;
  static constexpr int THREADS = 32 * (EPI_WARP0 + EPI_WARPS);
  static constexpr int EPI_THREADS = 32 * EPI_WARPS;
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static constexpr int STAGE_PITCH = 20;
  static constexpr int STAGING_BYTES = EPI_WARPS * 32 * STAGE_PITCH * 4;
  static constexpr size_t SMEM = 1024 + size_t(STAGES) * (A_BYTES + B_BYTES) + STAGING_BYTES + 256;
  static_assert(BN == 128 || BN == 256, "BN");
  static_assert(SMEM <= 232448, "shared memory budget");
};

// Pair tile t -> (row tile of 256, column tile), banded: QG2_BAND row tiles x all column tiles.
__device__ __forceinline__ void qg2_tile(int t, int m_tiles, int n_tiles, int& t_m, int& t_n) {
  const int per_band = QG2_BAND * n_tiles;
  const int band = t / per_band;
  const int first = band * QG2_BAND;
  const int rows = min(m_tiles - first, QG2_BAND);
  const int r = t - band * per_band;
  t_m = first + r % rows;
  t_n = r / rows;
}

template <int BN, int STAGES, bool ROWCOL, int G>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Qg2Cfg<BN, STAGES, G>::THREADS, 1)
    qgemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ QgParams p) {
  using Cfg = Qg2Cfg<BN, STAGES, G>;
  constexpr int A_BYTES = Cfg::A_BYTES;
  constexpr int B_BYTES = Cfg::B_BYTES;
  constexpr uint32_t IDESC = idesc_i8(2 * QG_BM, BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  float* staging = reinterpret_cast<float*>(sB + STAGES * B_BYTES);
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(staging) + Cfg::STAGING_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * Cfg::EPI_THREADS);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_holder);

  const int m_tiles = (p.M + 2 * QG_BM - 1) / (2 * QG_BM);
  const int num_tiles = m_tiles * p.n_tiles;
  const int cluster = blockIdx.x >> 1, clusters = gridDim.x >> 1;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      const uint32_t full_even = mapa_shared(smem_u32(full), 0);
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int t = cluster; t < num_tiles && ok; t += clusters) {
        int t_m, t_n;
        qg2_tile(t, m_tiles, p.n_tiles, t_m, t_n);
        const int m0 = t_m * 2 * QG_BM + int(rank) * QG_BM;
        const int n0 = t_n * BN + int(rank) * (BN / 2);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, QG_TIMEOUT_NS)) { ok = false; break; }
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * (A_BYTES + B_BYTES));
          const uint32_t fb = full_even + stage * sizeof(uint64_t);
          tma_load_2d_pair(sA + stage * A_BYTES, &tmA, kb * QG_BK, m0, fb);
          tma_load_2d_pair(sB + stage * B_BYTES, &tmB, kb * QG_BK, n0, fb);
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok && rank == 0) {
        // the even CTA's full barriers also count the odd CTA's bytes: once they complete, every
        // copy of those stages has landed in both CTAs
        for (int i = 1; i <= STAGES && i <= issued; ++i) {
          const int idx = issued - i;
          mbar_wait_drain(&full[idx % STAGES], (idx / STAGES) & 1);
        }
      }
      if (!ok && rank != 0) {
        // copies of stages the even CTA never expected cannot be tracked here: give them time to
        // land (a copy takes microseconds) before this CTA may leave
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 200000ull) {
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer (even CTA)
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      // descriptors built once, moved by their start-address field (see qgemm_sm100_kernel)
      constexpr uint32_t KU = QG_UMMA_K >> 4;
      const uint64_t a_desc0 = smem_desc_k_sw128(smem_u32(sA)), b_desc0 = smem_desc_k_sw128(smem_u32(sB));
      for (int t = cluster; t < num_tiles && ok; t += clusters, ++it) {
        const int acc = it & 1;
        if (!mbar_wait(&tempty[acc], ((it >> 1) & 1) ^ 1, abort_flag, QG_TIMEOUT_NS)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, QG_TIMEOUT_NS)) { ok = false; break; }
          tc_fence_after();
          const uint64_t a_d = a_desc0 + static_cast<uint64_t>(stage * (A_BYTES >> 4));
          const uint64_t b_d = b_desc0 + static_cast<uint64_t>(stage * (B_BYTES >> 4));
          const int rem = p.K - kb * QG_BK;
          if (rem >= QG_BK) {
#pragma unroll
            for (int kk = 0; kk < QG_BK / QG_UMMA_K; ++kk)
              mma_i8_pair(d_tmem, a_d + kk * KU, b_d + kk * KU, IDESC, (kb != 0 || kk != 0) ? 1u : 0u);
          } else {
            const int nk = (rem + QG_UMMA_K - 1) / QG_UMMA_K;
            for (int kk = 0; kk < nk; ++kk)
              mma_i8_pair(d_tmem, a_d + kk * KU, b_d + kk * KU, IDESC, (kb != 0 || kk != 0) ? 1u : 0u);
          }
          mma_commit_pair_both(&empty[stage], 0x3);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (ok) mma_commit_pair_both(&tfull[acc], 0x3);
      }
      mma_commit_pair(drain);
      mbar_wait_drain(drain, 0);
    }
  } else {
    // ------------------------------------------------ epilogue (both CTAs, their own 128 rows)
    const int ew = warp - Cfg::EPI_WARP0;
    const int quarter = warp & 3;
    const int group = ew >> 2;
    float* stage = staging + ew * 32 * Cfg::STAGE_PITCH;
    const uint32_t tempty_even = mapa_shared(smem_u32(tempty), 0);
    int it = 0;
    for (int t = cluster; t < num_tiles; t += clusters, ++it) {
      const int acc = it & 1;
      if (!mbar_wait(&tfull[acc], (it >> 1) & 1, abort_flag, QG_TIMEOUT_NS)) break;
      tc_fence_after();
      int t_m, t_n;
      qg2_tile(t, m_tiles, p.n_tiles, t_m, t_n);
      const int n0 = t_n * BN;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
      const int m_warp0 = t_m * 2 * QG_BM + int(rank) * QG_BM + quarter * 32;
      const QgRow row = qg_row<QG_A_TMA>(p, m_warp0 + lane);
#pragma unroll 1
      for (int c = group; c < BN / Cfg::CW; c += G) {
        const int nb = n0 + c * Cfg::CW;
        if (nb >= p.N) break;  // warp-uniform
        qg_epilogue_chunk<ROWCOL, Cfg::STAGE_PITCH>(p, tbase + c * Cfg::CW, row, m_warp0, nb, stage, lane,
                                                    p.out_f32);
      }
      tc_fence_before();
      if (rank == 0) mbar_arrive(&tempty[acc]);
      else mbar_arrive_remote(tempty_even + acc * sizeof(uint64_t));
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicExch(p.err, 1);
}

}  // namespace mira
