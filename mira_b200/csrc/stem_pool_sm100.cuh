// A stride-2 convolution over the row-expanded int8 input (ResNet's 7x7/2 stem) fused with the
// -inf pad + 3x3/2 max pool after it: reference qconv2d (ops.py:630-634) with its epilogue, then
// pad (ops.py:469-470) and maxpool2d (ops.py:293-296).  The conv outputs never leave the SM.
//
// One persistent CTA per SM walks work units = (image, band of pooled rows).  Each conv output row
// of the band is one 128-row MMA tile (its ow <= 128 pixels; tcgen05.mma kind::i8, M = 128, N = 64,
// K = kh * 32): kernel row i of output row oy reads input row iy = 2 oy - pad + i, whose row-expanded
// entries ox and ox + 2 hold input pixels 2 ox - pad .. 2 ox - pad + 7 of output pixel ox.  So every
// input row is one contiguous bulk copy into a shared-memory plane (entry e at byte 16 e), and the
// A operand of kernel row i is that plane read as a K-major matrix without swizzle: rows 16 bytes
// apart, the second 16-byte K chunk 32 bytes (two entries) further.  The producer warp streams the
// input rows through a ring of planes in the order the conv rows need them; rows outside the image
// read a plane of zeros.  Weights stay in shared memory.
//
// Epilogue (8 warps): each conv row's int32 accumulators go to a 3-row ring in shared memory; once
// rows 2 py - 1 .. 2 py + 1 are there, pooled row py is the max over each 3 x 3 window of int32
// values, and only the pooled values are dequantized and run through the epilogue: dequant
// (positive scale), adding constants, relu and clamping are all monotone non-decreasing, so they
// commute with max (the host checks the steps) and the result is the reference's bit for bit.
// Outputs: pooled f32 NHWC and/or int8 (NHWC rows or the chunk-planar layout).
#pragma once
#include "qgemm_sm100.cuh"

namespace mira {

constexpr int SP_NIN = 24;          // input-row planes in the ring (7 in use, the rest prefetch)
constexpr int SP_PLANE = 2176;      // bytes per plane: 128 rows + the 2-entry shift, padded (136 x 16)
constexpr int SP_KH_MAX = 8;        // kernel rows (K = kh * 32 <= 256)
constexpr int SP_PITCH = 68;        // int32 per pixel in the conv-row ring (64 channels + 4)
constexpr int SP_OW_MAX = 128;
constexpr int SP_EPI_WARPS = 8;    // groups of the four TMEM lane quarters
constexpr int SP_THREADS = 32 * (2 + SP_EPI_WARPS);
constexpr int SP_ACCS = 4;

struct SpParams {
  int n, h, w;            // input images
  int oh, ow;             // conv output
  int ph, pw;             // pooled output
  int kh, pad_h;          // kernel rows, vertical padding of the conv
  int row_entries;        // entries per input row of the row-expanded layout
  int o;                  // output channels (<= 64)
  int band, bands;        // pooled rows per work unit, units per image
  const int8_t* x;
  const int8_t* wq;       // [o, ldw] row-expanded weights (k = i * 32 + j * 4 + c)
  int64_t ldw;
  const double* scale64;
  const float* scale_hi;
  const float* scale_lo;
  int epi_kind;           // QG_EPI_* program (0: the step loop)
  int n_steps;
  mira_epi_step steps[MIRA_EPI_MAX_STEPS];
  float* out_f32;
  int64_t ld_f32;
  int8_t* out_i8;
  int64_t ld_i8;
  int i8_cp, i8_guard;
  int64_t i8_chunk;
  float q_scale, q_rcp, q_c127;
  int nonneg;
  int* err;
};

struct SpSmem {
  static constexpr int B_BYTES = 2 * SP_KH_MAX * 64 * 16;          // weight chunk planes
  static constexpr int IN_BYTES = (SP_NIN + 1) * SP_PLANE;          // ring + the zero plane
  static constexpr int RING_BYTES = 3 * SP_OW_MAX * SP_PITCH * 4;   // 3 conv rows of int32
  static constexpr int BAR_BYTES = 8 * (2 * SP_NIN + 2 * SP_ACCS + 2) + 16;
  static constexpr size_t TOTAL = 1024 + B_BYTES + IN_BYTES + RING_BYTES + ((BAR_BYTES + 127) / 128) * 128;
  static_assert(TOTAL <= 232448, "shared memory budget");
};

// The range of conv rows of work unit u and the input rows they read.
struct SpUnit {
  int img, py0, py1, cr0, cr1, iy0, iy1;
};

__device__ __forceinline__ SpUnit sp_unit(const SpParams& p, int u) {
  SpUnit s;
  s.img = u / p.bands;
  const int b = u - s.img * p.bands;
  s.py0 = b * p.band;
  s.py1 = min(p.ph, s.py0 + p.band);
  s.cr0 = max(0, 2 * s.py0 - 1);
  s.cr1 = min(p.oh - 1, 2 * s.py1 - 1);
  s.iy0 = 2 * s.cr0 - p.pad_h;
  s.iy1 = 2 * s.cr1 - p.pad_h + p.kh - 1;
  return s;
}

__global__ void __launch_bounds__(SP_THREADS, 1) stem_pool_kernel(const __grid_constant__ SpParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sB = smem;
  uint8_t* sIn = sB + SpSmem::B_BYTES;                       // SP_NIN planes, then the zero plane
  uint8_t* sZero = sIn + SP_NIN * SP_PLANE;
  int32_t* ring = reinterpret_cast<int32_t*>(sIn + SpSmem::IN_BYTES);
  uint64_t* in_full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(ring) + SpSmem::RING_BYTES);
  uint64_t* in_empty = in_full + SP_NIN;
  uint64_t* tfull = in_empty + SP_NIN;
  uint64_t* tempty = tfull + SP_ACCS;
  uint64_t* drain = tempty + SP_ACCS;
  uint64_t* ep_bar = drain + 1;     // the epilogue warps meet here (bounded waits, unlike bar.sync)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(ep_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int units = p.n * p.bands;

  // weights as K-major chunk planes without swizzle: plane c (16 bytes of K) holds rows 0..63
  for (int e = threadIdx.x; e < 2 * p.kh * 64; e += SP_THREADS) {
    const int c = e >> 6, r = e & 63;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (r < p.o) v = *reinterpret_cast<const uint4*>(p.wq + static_cast<int64_t>(r) * p.ldw + c * 16);
    reinterpret_cast<uint4*>(sB)[e] = v;
  }
  for (int e = threadIdx.x; e < SP_PLANE / 16; e += SP_THREADS)
    reinterpret_cast<uint4*>(sZero)[e] = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async_smem();   // the generic-proxy writes above are read by tcgen05.mma
  if (threadIdx.x == 0) {
    for (int s = 0; s < SP_NIN; ++s) {
      mbar_init(&in_full[s], 1);
      mbar_init(&in_empty[s], 1);
    }
    for (int a = 0; a < SP_ACCS; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], SP_EPI_WARPS * 32);
    }
    mbar_init(drain, 1);
    mbar_init(ep_bar, SP_EPI_WARPS * 32);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, SP_ACCS * 64);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_holder);

  if (warp == 0) {
    // ------------------------------------------------ producer: input rows in the ring
    if (lane == 0) {
      uint32_t seq = 0;
      bool ok = true;
      const uint32_t row_bytes = static_cast<uint32_t>(p.row_entries) * 16u;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const SpUnit s = sp_unit(p, u);
        for (int iy = s.iy0; iy <= s.iy1; ++iy, ++seq) {
          const int slot = seq % SP_NIN;
          if (!mbar_wait(&in_empty[slot], ((seq / SP_NIN) & 1) ^ 1, abort_flag, QG_TIMEOUT_NS)) { ok = false; break; }
          if (iy >= 0 && iy < p.h) {
            mbar_arrive_expect_tx(&in_full[slot], row_bytes);
            bulk_load(sIn + slot * SP_PLANE, p.x + (static_cast<int64_t>(s.img) * p.h + iy) * row_bytes, row_bytes,
                      &in_full[slot]);
          } else {
            mbar_arrive(&in_full[slot]);   // outside the image: the MMAs read the zero plane
          }
        }
      }
      if (!ok) {
        for (int i = 1; i <= SP_NIN && static_cast<uint32_t>(i) <= seq; ++i) {
          const uint32_t idx = seq - i;
          mbar_wait_drain(&in_full[idx % SP_NIN], (idx / SP_NIN) & 1);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer: one conv row per accumulator
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_i8(QG_BM, 64);
      // A: a plane read as K-major without swizzle, rows 16 bytes apart, its second K chunk 2 rows
      // (32 bytes) further; B: chunk planes of 64 rows, 1 KB apart
      const uint64_t in_d0 = smem_desc_k_none(smem_u32(sIn), 32, 128);
      const uint64_t zero_d = smem_desc_k_none(smem_u32(sZero), 32, 128);
      const uint64_t b_d0 = smem_desc_k_none(smem_u32(sB), 1024, 128);
      uint32_t seq = 0;     // input rows consumed (the producer's numbering)
      int crow = 0;         // conv rows issued (accumulator rotation)
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const SpUnit s = sp_unit(p, u);
        const uint32_t seq0 = seq;
        uint32_t retired = 0;   // input rows of this unit released so far
        for (int oy = s.cr0; oy <= s.cr1 && ok; ++oy, ++crow) {
          const int acc = crow % SP_ACCS;
          if (!mbar_wait(&tempty[acc], ((crow / SP_ACCS) & 1) ^ 1, abort_flag, QG_TIMEOUT_NS)) { ok = false; break; }
          tc_fence_after();
          const int iyb = 2 * oy - p.pad_h;
          for (int i = 0; i < p.kh; ++i) {
            const uint32_t q = seq0 + static_cast<uint32_t>(iyb + i - s.iy0);
            if (!mbar_wait(&in_full[q % SP_NIN], (q / SP_NIN) & 1, abort_flag, QG_TIMEOUT_NS)) { ok = false; break; }
          }
          if (!ok) break;
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + acc * 64;
          for (int i = 0; i < p.kh; ++i) {
            const int iy = iyb + i;
            const uint32_t q = seq0 + static_cast<uint32_t>(iy - s.iy0);
            const uint64_t a_d = (iy >= 0 && iy < p.h) ? in_d0 + (q % SP_NIN) * (SP_PLANE >> 4) : zero_d;
            mma_i8(d_tmem, a_d, b_d0 + static_cast<uint64_t>(2 * i * 64), IDESC, i > 0 ? 1u : 0u);
          }
          mma_commit(&tfull[acc]);
          // input rows no later conv row of the unit reads are released when these MMAs finish
          const uint32_t keep_from = oy < s.cr1 ? static_cast<uint32_t>(2 * (oy + 1) - p.pad_h - s.iy0)
                                                : static_cast<uint32_t>(s.iy1 - s.iy0 + 1);
          for (; retired < keep_from; ++retired) mma_commit(&in_empty[(seq0 + retired) % SP_NIN]);
        }
        seq = seq0 + static_cast<uint32_t>(s.iy1 - s.iy0 + 1);
      }
      mma_commit(drain);
      mbar_wait_drain(drain, 0);
    }
  } else {
    // ------------------------------------------------ epilogue: conv rows to the ring, pooled rows out
    const int ew = warp - 2;                  // 0 .. SP_EPI_WARPS - 1
    const int quarter = warp & 3;             // TMEM lanes 32 * quarter ..
    const int group = ew >> 2;                // 16-column chunks group, group + groups, ...
    constexpr int kGroups = SP_EPI_WARPS / 4;
    const int et = threadIdx.x - 64;          // 0 .. 32 * SP_EPI_WARPS - 1
    const int pix = quarter * 32 + lane;
    int crow = 0;
    uint32_t ep_phase = 0;
    // pooling: each thread keeps one group of 4 channels and strides over the pooled pixels, so its
    // per-channel constants are loaded once
    const int c4 = p.o >> 2;
    const int pstride = (SP_EPI_WARPS * 32) / c4;
    const int cg = et % c4, px0 = et / c4;
    const bool cg_ok = px0 < pstride;
    const int ch = 4 * cg;
    const float4 hs = __ldg(reinterpret_cast<const float4*>(p.scale_hi + ch));
    const float4 ls = __ldg(reinterpret_cast<const float4*>(p.scale_lo + ch));
    double s64[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) s64[j] = p.scale64[ch + j];
    const float4 bias = (p.epi_kind & QG_EPI_BIAS) ? __ldg(reinterpret_cast<const float4*>(p.steps[0].ptr + ch))
                                                   : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const float clamp_lo = (p.epi_kind & QG_EPI_CLAMP) ? p.steps[p.n_steps - 2].scalar : 0.0f;
    const float clamp_hi = (p.epi_kind & QG_EPI_CLAMP) ? p.steps[p.n_steps - 1].scalar : 0.0f;
    const int64_t i8_ch = static_cast<int64_t>(ch >> 4) * p.i8_chunk + (ch & 15);
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      const SpUnit s = sp_unit(p, u);
      bool ok = true;
      for (int oy = s.cr0; oy <= s.cr1; ++oy, ++crow) {
        const int acc = crow % SP_ACCS;
        if (!mbar_wait(&tfull[acc], (crow / SP_ACCS) & 1, abort_flag, QG_TIMEOUT_NS)) { ok = false; break; }
        tc_fence_after();
        int32_t* rrow = ring + ((oy % 3) * SP_OW_MAX + pix) * SP_PITCH;
#pragma unroll
        for (int cc = 0; cc < 4 / kGroups; ++cc) {
          const int c = group + kGroups * cc;   // 16-column chunk
          uint32_t r[16];
          tmem_ld_32x32b_x16(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * 64 + c * 16, r);
          tmem_ld_wait();
          if (pix < p.ow) {
            uint4* d = reinterpret_cast<uint4*>(rrow + c * 16);
#pragma unroll
            for (int q = 0; q < 4; ++q) d[q] = make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
        // every conv row of the window is in the ring
        mbar_arrive(ep_bar);
        if (!mbar_wait_spin(ep_bar, ep_phase, abort_flag, QG_TIMEOUT_NS)) { ok = false; break; }
        ep_phase ^= 1;
        // pooled row py is complete once conv row min(2 py + 1, oh - 1) is in the ring
        const int py = (oy + 1) >> 1;
        const bool last = oy == s.cr1;
        int pys[2];
        int npy = 0;
        if ((oy & 1) && py - 1 >= s.py0 && py - 1 < s.py1) pys[npy++] = py - 1;   // oy = 2 (py-1) + 1
        if (last && (oy & 1) == 0 && oy / 2 >= s.py0 && oy / 2 < s.py1) pys[npy++] = oy / 2;
        for (int k = 0; k < npy; ++k) {
          const int prow = pys[k];
          // rows of the window inside the conv output (the others are the -inf padding)
          const int32_t* rows[3];
          int nrows = 0;
#pragma unroll
          for (int dy = 0; dy < 3; ++dy) {
            const int cy = 2 * prow - 1 + dy;
            if (cy >= 0 && cy < p.oh) rows[nrows++] = ring + (cy % 3) * SP_OW_MAX * SP_PITCH + 4 * cg;
          }
          for (int px = px0; px < p.pw && cg_ok; px += pstride) {
            int32_t mx[4] = {INT32_MIN, INT32_MIN, INT32_MIN, INT32_MIN};
            const int cx0 = 2 * px - 1;
            for (int r = 0; r < nrows; ++r) {
#pragma unroll
              for (int dx = 0; dx < 3; ++dx) {
                const int cx = cx0 + dx;
                if (cx < 0 || cx >= p.ow) continue;
                const int4 t = *reinterpret_cast<const int4*>(rows[r] + cx * SP_PITCH);
                mx[0] = max(mx[0], t.x); mx[1] = max(mx[1], t.y); mx[2] = max(mx[2], t.z); mx[3] = max(mx[3], t.w);
              }
            }
            float v[4];
            uint32_t slow = 0;
            dequant4_x2(reinterpret_cast<const uint32_t*>(mx), hs, ls, v, slow, 0);
            if (slow) {
#pragma unroll
              for (int j = 0; j < 4; ++j)
                if (slow & (1u << j)) v[j] = __double2float_rn(static_cast<double>(mx[j]) * s64[j]);
            }
            if (p.epi_kind != 0) {
              if (p.epi_kind & QG_EPI_BIAS) {
                v[0] = __fadd_rn(v[0], bias.x); v[1] = __fadd_rn(v[1], bias.y);
                v[2] = __fadd_rn(v[2], bias.z); v[3] = __fadd_rn(v[3], bias.w);
              }
              if (p.epi_kind & QG_EPI_RELU) {
#pragma unroll
                for (int j = 0; j < 4; ++j) v[j] = np_maximum(v[j], 0.0f);
              }
              if (p.epi_kind & QG_EPI_CLAMP) {
#pragma unroll
                for (int j = 0; j < 4; ++j) v[j] = np_minimum(np_maximum(v[j], clamp_lo), clamp_hi);
              }
            } else {
              for (int st = 0; st < p.n_steps; ++st) {
                const mira_epi_step& e = p.steps[st];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  if (e.operand == MIRA_OPND_NONE) {
                    v[j] = apply_unary(e.op, v[j]);
                  } else {
                    const float o = e.operand == MIRA_OPND_SCALAR ? e.scalar : __ldg(e.ptr + ch + j);
                    v[j] = e.swapped ? apply_binary(e.op, o, v[j]) : apply_binary(e.op, v[j], o);
                  }
                }
              }
            }
            const int64_t opix = (static_cast<int64_t>(s.img) * p.ph + prow) * p.pw + px;
            if (p.out_f32 != nullptr)
              *reinterpret_cast<float4*>(p.out_f32 + opix * p.ld_f32 + ch) = make_float4(v[0], v[1], v[2], v[3]);
            if (p.out_i8 != nullptr) {
              uint32_t b[4];
              if (p.nonneg) requant_x2<4, true>(v, p.q_scale, p.q_rcp, p.q_c127, b);
              else requant_x2<4, false>(v, p.q_scale, p.q_rcp, p.q_c127, b);
              const int64_t base =
                  p.i8_cp ? (static_cast<int64_t>(p.i8_guard) + (static_cast<int64_t>(s.img) * (p.ph + 2) + prow + 1) *
                                                                    (p.pw + 2) + px + 1) * 16 + i8_ch
                          : opix * p.ld_i8 + ch;
              *reinterpret_cast<uint32_t*>(p.out_i8 + base) = pack4_i8(b[0], b[1], b[2], b[3]);
            }
          }
        }
        // the ring slot the next conv row overwrites was read above
        mbar_arrive(ep_bar);
        if (!mbar_wait_spin(ep_bar, ep_phase, abort_flag, QG_TIMEOUT_NS)) { ok = false; break; }
        ep_phase ^= 1;
      }
      if (!ok) break;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, SP_ACCS * 64);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicExch(p.err, 1);
}

}  // namespace mira
