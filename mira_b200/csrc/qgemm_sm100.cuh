// K1/K2: the W8A8 matmul and implicit-GEMM convolution on tcgen05.mma kind::i8.
//
// One persistent CTA per SM walks 128 x BN output tiles.  Warp roles:
//   warp 0      TMA producer: B (weights, K-major) and, for matmuls, A tiles into a STAGES-deep
//               ring of shared-memory stages (128-byte swizzle, no multicast)
//   warp 1      allocates TMEM (2 x BN columns: two accumulators) and issues the MMAs from one
//               thread; tcgen05.commit frees a stage / publishes an accumulator
//   warps 4-7   epilogue: tcgen05.ld of their 32 TMEM lanes (one output row per thread), exact
//               dequant, the fused epilogue steps, f32 and/or requantized int8 stores
//   warps 8-11  (convolutions only) im2col gather of A from NHWC int8 with cp.async, one output
//               pixel (tile row) per thread, zero fill for padding
// The two TMEM accumulators let the epilogue of tile i overlap the main loop of tile i+1.
#pragma once
#include <cuda.h>

#include "exact_math.cuh"
#include "ptx_sm100.cuh"

namespace mira {

constexpr int QG_BM = 128;               // tile rows = TMEM lanes
constexpr int QG_BK = 128;               // K bytes per stage = one 128-byte swizzle row
constexpr int QG_UMMA_K = 32;            // K per tcgen05.mma kind::i8
constexpr uint64_t QG_TIMEOUT_NS = 2000000000ull;

enum QgAMode { QG_A_TMA = 0, QG_A_GATHER16 = 1, QG_A_GATHER4 = 2 };

struct QgConv {
  int n, h, w, cp;      // input NHWC (cp = padded channels)
  int oh, ow;
  int kh, kw, sh, sw, ph, pw, dh, dw;
};

struct QgParams {
  int M, N, K;          // K = bytes of the reduction actually used
  int num_kb;           // ceil(K / QG_BK)
  int m_tiles, n_tiles;
  const int8_t* A;      // gather modes: NHWC input
  QgConv g;
  const double* scale64;
  const float* scale_hi;
  const float* scale_lo;
  const float* row_scale;
  const float* col_scale;
  int n_steps;
  mira_epi_step steps[MIRA_EPI_MAX_STEPS];
  float* out_f32;
  int64_t ld_f32;
  int8_t* out_i8;
  int64_t ld_i8;
  float q_scale, q_rcp, q_lim;   // requant divisor, RN32(1/divisor), 256 * divisor
  int* err;
};

template <int BN, int STAGES, int AMODE>
struct QgCfg {
  static constexpr int A_BYTES = QG_BM * QG_BK;
  static constexpr int B_BYTES = BN * QG_BK;
  static constexpr int THREADS = AMODE == QG_A_TMA ? 256 : 384;
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static constexpr int GATHER_LAG = STAGES > 3 ? 3 : STAGES - 1;
  static constexpr size_t SMEM = 1024 + size_t(STAGES) * (A_BYTES + B_BYTES) + 256;
  static_assert(BN == 64 || BN == 128 || BN == 256, "BN");
};

// Bounded wait that ignores the abort flag: used only to let in-flight copies land before exit.
__device__ __forceinline__ void mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > QG_TIMEOUT_NS) return;
  }
}

// ---------------------------------------------------------------- epilogue (one 32-column chunk)

template <bool ROWCOL>
__device__ __forceinline__ void qg_dequant_chunk(const QgParams& p, const uint32_t (&r)[32], int m, int nb,
                                                 float (&v)[32]) {
  if (!ROWCOL) {
    const float4* hi4 = reinterpret_cast<const float4*>(p.scale_hi + nb);
    const float4* lo4 = reinterpret_cast<const float4*>(p.scale_lo + nb);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 h = __ldg(hi4 + q), l = __ldg(lo4 + q);
      const float hs[4] = {h.x, h.y, h.z, h.w}, ls[4] = {l.x, l.y, l.z, l.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = 4 * q + e;
        float y;
        if (!dequant_fast(static_cast<int32_t>(r[j]), hs[e], ls[e], y))
          y = __double2float_rn(static_cast<double>(static_cast<int32_t>(r[j])) * p.scale64[nb + j]);
        v[j] = y;
      }
    }
  } else {
    const float rs = p.row_scale[m];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float cs = (nb + j < p.N) ? __ldg(p.col_scale + nb + j) : 0.0f;
      float hi, lo, y;
      split_rowcol(rs, cs, hi, lo);
      if (!dequant_fast(static_cast<int32_t>(r[j]), hi, lo, y))
        y = __double2float_rn(static_cast<double>(static_cast<int32_t>(r[j])) *
                              (static_cast<double>(rs) * static_cast<double>(cs)));
      v[j] = y;
    }
  }
}

#define QG_APPLY_BINARY(EXPR)                         \
  do {                                                \
    if (st.swapped) {                                 \
      _Pragma("unroll") for (int j = 0; j < 32; ++j) { \
        const float a = o[j], b = v[j];               \
        v[j] = (EXPR);                                \
      }                                               \
    } else {                                          \
      _Pragma("unroll") for (int j = 0; j < 32; ++j) { \
        const float a = v[j], b = o[j];               \
        v[j] = (EXPR);                                \
      }                                               \
    }                                                 \
  } while (0)

__device__ __forceinline__ void qg_epilogue_steps(const QgParams& p, int m, int nb, bool full_chunk,
                                                  float (&v)[32]) {
  for (int s = 0; s < p.n_steps; ++s) {
    const mira_epi_step& st = p.steps[s];
    if (st.operand == MIRA_OPND_NONE) {
      switch (st.op) {
        case MIRA_EPI_RELU:
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = np_maximum(v[j], 0.0f);
          break;
        default:
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = apply_unary(st.op, v[j]);
          break;
      }
      continue;
    }
    float o[32];
    if (st.operand == MIRA_OPND_SCALAR) {
#pragma unroll
      for (int j = 0; j < 32; ++j) o[j] = st.scalar;
    } else if (st.operand == MIRA_OPND_CHANNEL) {
      const float4* c4 = reinterpret_cast<const float4*>(st.ptr + nb);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 t = __ldg(c4 + q);
        o[4 * q] = t.x; o[4 * q + 1] = t.y; o[4 * q + 2] = t.z; o[4 * q + 3] = t.w;
      }
    } else if (st.operand == MIRA_OPND_ROW) {
      const float t = st.ptr[m];
#pragma unroll
      for (int j = 0; j < 32; ++j) o[j] = t;
    } else {  // FULL
      const float* src = st.ptr + static_cast<int64_t>(m) * st.ld + nb;
      if (full_chunk && (st.ld % 4) == 0) {
        const float4* s4 = reinterpret_cast<const float4*>(src);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 t = __ldg(s4 + q);
          o[4 * q] = t.x; o[4 * q + 1] = t.y; o[4 * q + 2] = t.z; o[4 * q + 3] = t.w;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) o[j] = (nb + j < p.N) ? src[j] : 0.0f;
      }
    }
    switch (st.op) {
      case MIRA_EPI_ADD: QG_APPLY_BINARY(__fadd_rn(a, b)); break;
      case MIRA_EPI_SUB: QG_APPLY_BINARY(__fsub_rn(a, b)); break;
      case MIRA_EPI_MUL: QG_APPLY_BINARY(__fmul_rn(a, b)); break;
      case MIRA_EPI_DIV: QG_APPLY_BINARY(__fdiv_rn(a, b)); break;
      case MIRA_EPI_MAXIMUM: QG_APPLY_BINARY(np_maximum(a, b)); break;
      case MIRA_EPI_MINIMUM: QG_APPLY_BINARY(np_minimum(a, b)); break;
      default: break;
    }
  }
}

__device__ __forceinline__ void qg_store_chunk(const QgParams& p, int m, int nb, bool full_chunk,
                                               const float (&v)[32]) {
  if (p.out_f32 != nullptr) {
    float* dst = p.out_f32 + static_cast<int64_t>(m) * p.ld_f32 + nb;
    if (full_chunk && (p.ld_f32 % 4) == 0) {
      float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
      for (int q = 0; q < 8; ++q) d4[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (nb + j < p.N) dst[j] = v[j];
    }
  }
  if (p.out_i8 != nullptr) {
    uint32_t w[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      uint32_t b[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = 4 * q + e;
        b[e] = (nb + j < p.N) ? round_clip_i8(div_by_scale(v[j], p.q_scale, p.q_rcp, p.q_lim)) : 0u;
      }
      w[q] = pack4_i8(b[0], b[1], b[2], b[3]);
    }
    int8_t* dst = p.out_i8 + static_cast<int64_t>(m) * p.ld_i8 + nb;
    const int64_t room = p.ld_i8 - nb;  // multiple of 16
    if (room >= 16) reinterpret_cast<uint4*>(dst)[0] = make_uint4(w[0], w[1], w[2], w[3]);
    if (room >= 32) reinterpret_cast<uint4*>(dst)[1] = make_uint4(w[4], w[5], w[6], w[7]);
  }
}

// ---------------------------------------------------------------- the kernel

template <int BN, int STAGES, int AMODE, bool ROWCOL>
__global__ void __launch_bounds__(QgCfg<BN, STAGES, AMODE>::THREADS, 1)
    qgemm_sm100_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       const __grid_constant__ QgParams p) {
  using Cfg = QgCfg<BN, STAGES, AMODE>;
  constexpr int A_BYTES = Cfg::A_BYTES;
  constexpr int B_BYTES = Cfg::B_BYTES;
  constexpr uint32_t IDESC = idesc_i8(QG_BM, BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], AMODE == QG_A_TMA ? 1 : 1 + 128);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmB);
    if (AMODE == QG_A_TMA) tma_prefetch_desc(&tmA);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_holder);

  const int num_tiles = p.m_tiles * p.n_tiles;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const int m0 = (t / p.n_tiles) * QG_BM;
        const int n0 = (t % p.n_tiles) * BN;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, QG_TIMEOUT_NS)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[stage], (AMODE == QG_A_TMA ? A_BYTES : 0) + B_BYTES);
          if (AMODE == QG_A_TMA) tma_load_2d(sA + stage * A_BYTES, &tmA, kb * QG_BK, m0, &full[stage]);
          tma_load_2d(sB + stage * B_BYTES, &tmB, kb * QG_BK, n0, &full[stage]);
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) {
        // let the copies already issued land before the CTA can exit
        for (int i = 1; i <= STAGES && i <= issued; ++i) {
          const int idx = issued - i;
          mbar_wait_drain(&full[idx % STAGES], (idx / STAGES) & 1);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++it) {
        const int acc = it & 1;
        if (!mbar_wait(&tempty[acc], ((it >> 1) & 1) ^ 1, abort_flag, QG_TIMEOUT_NS)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, QG_TIMEOUT_NS)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * B_BYTES);
          const int rem = p.K - kb * QG_BK;
          const int nk = rem >= QG_BK ? QG_BK / QG_UMMA_K : (rem + QG_UMMA_K - 1) / QG_UMMA_K;
          for (int kk = 0; kk < nk; ++kk) {
            mma_i8(d_tmem, smem_desc_k_sw128(a_addr + kk * QG_UMMA_K), smem_desc_k_sw128(b_addr + kk * QG_UMMA_K),
                   IDESC, (kb | kk) != 0 ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (ok) mma_commit(&tfull[acc]);
      }
      // every MMA issued by this thread has finished once `drain` completes
      mma_commit(drain);
      mbar_wait_drain(drain, 0);
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------ epilogue
    const int ew = warp - 4;
    int it = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
      const int acc = it & 1;
      if (!mbar_wait(&tfull[acc], (it >> 1) & 1, abort_flag, QG_TIMEOUT_NS)) break;
      tc_fence_after();
      const int m0 = (t / p.n_tiles) * QG_BM;
      const int n0 = (t % p.n_tiles) * BN;
      const int m = m0 + ew * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        const int nb = n0 + c * 32;
        if (nb >= p.N) break;  // warp-uniform
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(ew * 32) << 16) + acc * BN + c * 32, r);
        tmem_ld_wait();
        if (m < p.M) {
          const bool full_chunk = nb + 32 <= p.N;
          float v[32];
          qg_dequant_chunk<ROWCOL>(p, r, m, nb, v);
          qg_epilogue_steps(p, m, nb, full_chunk, v);
          qg_store_chunk(p, m, nb, full_chunk, v);
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  } else if (AMODE != QG_A_TMA && warp >= 8) {
    // ------------------------------------------------ im2col gather of A (convolutions)
    constexpr int LAG = Cfg::GATHER_LAG;
    const int row = threadIdx.x - 256;
    const QgConv& g = p.g;
    int stage = 0;
    uint32_t phase = 0;
    int ring[LAG];
    int pending = 0, head = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
      const int m = (t / p.n_tiles) * QG_BM + row;
      const bool row_ok = m < p.M;
      int img = 0, oy = 0, ox = 0;
      if (row_ok) {
        img = m / (g.oh * g.ow);
        const int rem = m - img * g.oh * g.ow;
        oy = rem / g.ow;
        ox = rem - oy * g.ow;
      }
      const int iy0 = oy * g.sh - g.ph;
      const int ix0 = ox * g.sw - g.pw;
      const int8_t* base = p.A + static_cast<int64_t>(img) * g.h * g.w * g.cp;
      // reduction position k = (ti * kw + tj) * cp + ci, advanced incrementally
      int ti = 0, tj = 0, ci = 0;
      for (int kb = 0; kb < p.num_kb; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, QG_TIMEOUT_NS)) { ok = false; break; }
        const uint32_t dst_row = smem_u32(sA + stage * A_BYTES) + row * QG_BK;
        if (AMODE == QG_A_GATHER16) {
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const int k = kb * QG_BK + c * 16;
            const int iy = iy0 + ti * g.dh, ix = ix0 + tj * g.dw;
            const bool valid = row_ok && k < p.K && iy >= 0 && iy < g.h && ix >= 0 && ix < g.w;
            const int8_t* src = valid ? base + (static_cast<int64_t>(iy) * g.w + ix) * g.cp + ci : p.A;
            cp_async_16(dst_row + ((c ^ (row & 7)) << 4), src, valid ? 16u : 0u);
            ci += 16;
            if (ci == g.cp) {
              ci = 0;
              if (++tj == g.kw) { tj = 0; ++ti; }
            }
          }
        } else {
#pragma unroll 4
          for (int c = 0; c < 32; ++c) {
            const int k = kb * QG_BK + c * 4;
            const int iy = iy0 + ti * g.dh, ix = ix0 + tj * g.dw;
            const bool valid = row_ok && k < p.K && iy >= 0 && iy < g.h && ix >= 0 && ix < g.w;
            const int8_t* src = valid ? base + (static_cast<int64_t>(iy) * g.w + ix) * 4 : p.A;
            cp_async_4(dst_row + (((c >> 2) ^ (row & 7)) << 4) + ((c & 3) << 2), src, valid ? 4u : 0u);
            if (++tj == g.kw) { tj = 0; ++ti; }
          }
        }
        cp_async_commit();
        ring[(head + pending) % LAG] = stage;
        if (++pending == LAG) {
          cp_async_wait<LAG - 1>();
          fence_proxy_async_smem();
          mbar_arrive(&full[ring[head]]);
          head = (head + 1) % LAG;
          --pending;
        }
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
    cp_async_wait<0>();
    fence_proxy_async_smem();
    while (pending > 0) {
      mbar_arrive(&full[ring[head]]);
      head = (head + 1) % LAG;
      --pending;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicExch(p.err, 1);
}

}  // namespace mira
