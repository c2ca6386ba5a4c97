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
// input rows through a ring of SP_RING rows (row r of the stream at ring row r mod SP_RING, rows
// row_entries * 16 bytes apart), filled SP_ROWS consecutive rows per bulk copy (a bulk copy costs a
// few hundred cycles of the copy engine whatever its size, so rows are moved several at a time);
// ring rows for input rows outside the image are zero-filled.  The A operand of a kernel row may
// read past its input row (pixels beyond ow), into the next ring row or the tail pad after the
// ring: those accumulator rows are never used.  Weights stay in shared memory.
//
// Epilogue (8 warps, one TMEM lane = one conv output pixel per thread, 32 of its channels): the
// vertical max of each pooled window (conv rows 2 py - 1 .. 2 py + 1) is taken in registers as the
// conv rows arrive; when the window's last row is in, the column maxima go to shared memory (one of
// two row buffers), the warps meet once, and pooled row py is the max over 3 columns of those int32
// values.  Only the pooled values are dequantized and run through the epilogue: dequant
// (positive scale), adding constants, relu and clamping are all monotone non-decreasing, so they
// commute with max (the host checks the steps) and the result is the reference's bit for bit.
// Outputs: pooled f32 NHWC and/or int8 (NHWC rows or the chunk-planar layout).
#pragma once
#include "qgemm_sm100.cuh"

namespace mira {

constexpr int SP_ROWS = 4;          // input rows per ring slot (one bulk copy)
constexpr int SP_NIN = 8;           // ring slots (up to 3 in use by a conv row, the rest prefetch)
constexpr int SP_RING = SP_ROWS * SP_NIN;   // ring rows (a power of two)
constexpr int SP_ENTRIES_MAX = 136; // entries per input row
// the ring, then room for the A operand of the last ring row to read 130 entries (128 pixels + the
// 2-entry shift of the second K chunk)
constexpr int SP_IN_BYTES = (SP_RING * SP_ENTRIES_MAX * 16 + 130 * 16 + 127) / 128 * 128;
static_assert((SP_RING & (SP_RING - 1)) == 0, "ring rows must be a power of two");
constexpr int SP_KH_MAX = 8;        // kernel rows (K = kh * 32 <= 256)
constexpr int SP_PITCH = 68;        // int32 per pixel in a column-max row (64 channels + 4)
constexpr int SP_OW_MAX = 128;
constexpr int SP_EPI_WARPS = 8;    // groups of the four TMEM lane quarters
constexpr int SP_THREADS = 32 * (2 + SP_EPI_WARPS);
constexpr int SP_ACCS = 4;
constexpr int SP_PX_ITEMS = 4;      // pooled pixels a thread works on together

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
  static constexpr int IN_BYTES = SP_IN_BYTES;                     // the input-row ring
  static constexpr int RING_BYTES = 2 * SP_OW_MAX * SP_PITCH * 4;   // 2 column-max rows of int32
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
  uint8_t* sIn = sB + SpSmem::B_BYTES;                       // the input-row ring
  int32_t* ring = reinterpret_cast<int32_t*>(sIn + SpSmem::IN_BYTES);
  uint64_t* in_full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(ring) + SpSmem::RING_BYTES);
  uint64_t* in_empty = in_full + SP_NIN;
  uint64_t* tfull = in_empty + SP_NIN;
  uint64_t* tempty = tfull + SP_ACCS;
  uint64_t* drain = tempty + SP_ACCS;
  // the epilogue warps meet here (bounded waits, unlike bar.sync; waiting warps are suspended, so
  // they leave the issue slots to the warps still working)
  uint64_t* ep_bar = drain + 1;
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
  for (int e = threadIdx.x; e < SP_IN_BYTES / 16; e += SP_THREADS)   // the tail pad is read, never written
    reinterpret_cast<uint4*>(sIn)[e] = make_uint4(0u, 0u, 0u, 0u);
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
        for (int a = s.iy0; a <= s.iy1; a += SP_ROWS, ++seq) {
          const int slot = seq % SP_NIN;
          if (!mbar_wait(&in_empty[slot], ((seq / SP_NIN) & 1) ^ 1, abort_flag, QG_TIMEOUT_NS)) { ok = false; break; }
          // rows a .. a + SP_ROWS - 1 of the unit: those inside the image in one copy, the others
          // zero-filled (the slot's previous rows were released by the MMAs that read them)
          uint8_t* dst = sIn + static_cast<uint32_t>(slot * SP_ROWS) * row_bytes;
          const int b = min(a + SP_ROWS, s.iy1 + 1);
          const int va = max(a, 0), vb = max(va, min(b, p.h));
          if (va > a || vb < b) {
            for (int r = a; r < b; ++r) {
              if (r >= va && r < vb) continue;
              uint4* z = reinterpret_cast<uint4*>(dst + static_cast<uint32_t>(r - a) * row_bytes);
              for (int e = 0; e < p.row_entries; ++e) z[e] = make_uint4(0u, 0u, 0u, 0u);
            }
            fence_proxy_async_smem();   // the zeros are read by tcgen05.mma
          }
          if (va < vb) {
            const uint32_t bytes = static_cast<uint32_t>(vb - va) * row_bytes;
            mbar_arrive_expect_tx(&in_full[slot], bytes);
            bulk_load(dst + static_cast<uint32_t>(va - a) * row_bytes,
                      p.x + (static_cast<int64_t>(s.img) * p.h + va) * row_bytes, bytes, &in_full[slot]);
          } else {
            mbar_arrive(&in_full[slot]);
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
      // A: an input row read as K-major without swizzle, rows 16 bytes apart, its second K chunk 2
      // entries (32 bytes) further; B: chunk planes of 64 rows, 1 KB apart
      const uint64_t in_d0 = smem_desc_k_none(smem_u32(sIn), 32, 128);
      const uint64_t b_d0 = smem_desc_k_none(smem_u32(sB), 1024, 128);
      const uint32_t row_units = static_cast<uint32_t>(p.row_entries);   // 16-byte units per row
      uint32_t seq = 0;     // ring slots consumed (the producer's numbering)
      int crow = 0;         // conv rows issued (accumulator rotation)
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const SpUnit s = sp_unit(p, u);
        const uint32_t seq0 = seq;
        const int nslots = (s.iy1 - s.iy0) / SP_ROWS + 1;
        int retired = 0;   // slots of this unit released so far
        for (int oy = s.cr0; oy <= s.cr1 && ok; ++oy, ++crow) {
          const int acc = crow % SP_ACCS;
          if (!mbar_wait(&tempty[acc], ((crow / SP_ACCS) & 1) ^ 1, abort_flag, QG_TIMEOUT_NS)) { ok = false; break; }
          tc_fence_after();
          const int r0 = 2 * oy - p.pad_h - s.iy0;     // the unit's row index of kernel row 0
          for (int k = r0 / SP_ROWS; k <= (r0 + p.kh - 1) / SP_ROWS; ++k) {
            const uint32_t q = seq0 + static_cast<uint32_t>(k);
            if (!mbar_wait(&in_full[q % SP_NIN], (q / SP_NIN) & 1, abort_flag, QG_TIMEOUT_NS)) { ok = false; break; }
          }
          if (!ok) break;
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + acc * 64;
          const uint32_t rb = seq0 * SP_ROWS + static_cast<uint32_t>(r0);   // stream row of kernel row 0
          if (p.kh == 7) {   // the 7 x 7 stem: straight-line issue
#pragma unroll
            for (int i = 0; i < 7; ++i)
              mma_i8(d_tmem, in_d0 + ((rb + i) & (SP_RING - 1)) * row_units, b_d0 + static_cast<uint64_t>(2 * i * 64),
                     IDESC, i > 0 ? 1u : 0u);
          } else {
            for (int i = 0; i < p.kh; ++i)
              mma_i8(d_tmem, in_d0 + ((rb + i) & (SP_RING - 1)) * row_units, b_d0 + static_cast<uint64_t>(2 * i * 64),
                     IDESC, i > 0 ? 1u : 0u);
          }
          mma_commit(&tfull[acc]);
          // slots whose rows no later conv row of the unit reads are released when these MMAs finish
          const int keep_from = oy < s.cr1 ? (r0 + 2) / SP_ROWS : nslots;
          for (; retired < keep_from; ++retired) mma_commit(&in_empty[(seq0 + retired) % SP_NIN]);
        }
        seq = seq0 + static_cast<uint32_t>(nslots);
      }
      mma_commit(drain);
      mbar_wait_drain(drain, 0);
    }
  } else {
    // ------------------------------------------------ epilogue: column maxima, pooled rows out
    constexpr int kGroups = SP_EPI_WARPS / 4;
    constexpr int kCh = 64 / kGroups;         // channels of a thread's pixel
    const int ew = warp - 2;                  // 0 .. SP_EPI_WARPS - 1
    const int quarter = warp & 3;             // TMEM lanes 32 * quarter ..
    const int c0 = (ew >> 2) * kCh;           // first channel of this warp
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
    const float4 bias = (p.epi_kind & QG_EPI_BIAS) ? __ldg(reinterpret_cast<const float4*>(p.steps[0].ptr + ch))
                                                   : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const float clamp_lo = (p.epi_kind & QG_EPI_CLAMP) ? p.steps[p.n_steps - 2].scalar : 0.0f;
    const float clamp_hi = (p.epi_kind & QG_EPI_CLAMP) ? p.steps[p.n_steps - 1].scalar : 0.0f;
    const int64_t i8_ch = static_cast<int64_t>(ch >> 4) * p.i8_chunk + (ch & 15);
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      const SpUnit s = sp_unit(p, u);
      bool ok = true;
      int pyc = s.py0;          // the pooled row whose window the next conv row belongs to
      int32_t vm[kCh];          // vertical max of window pyc so far
#pragma unroll
      for (int j = 0; j < kCh; ++j) vm[j] = INT32_MIN;
      for (int oy = s.cr0; oy <= s.cr1; ++oy, ++crow) {
        const int acc = crow % SP_ACCS;
        if (!mbar_wait(&tfull[acc], (crow / SP_ACCS) & 1, abort_flag, QG_TIMEOUT_NS)) { ok = false; break; }
        tc_fence_after();
        uint32_t r[kCh / 16][16];
#pragma unroll
        for (int cc = 0; cc < kCh / 16; ++cc)
          tmem_ld_32x32b_x16(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * 64 + c0 + cc * 16,
                             r[cc]);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
#pragma unroll
        for (int j = 0; j < kCh; ++j) vm[j] = max(vm[j], static_cast<int32_t>(r[j >> 4][j & 15]));
        // the window's last conv row: min(2 pyc + 1, oh - 1)
        if (oy != min(2 * pyc + 1, p.oh - 1)) continue;
        const int prow = pyc;
        int32_t* vrow = ring + (prow & 1) * SP_OW_MAX * SP_PITCH;
        if (pix < p.ow) {
          uint4* d = reinterpret_cast<uint4*>(vrow + pix * SP_PITCH + c0);
#pragma unroll
          for (int q = 0; q < kCh / 4; ++q)
            d[q] = make_uint4(static_cast<uint32_t>(vm[4 * q]), static_cast<uint32_t>(vm[4 * q + 1]),
                              static_cast<uint32_t>(vm[4 * q + 2]), static_cast<uint32_t>(vm[4 * q + 3]));
        }
        // an odd conv row 2 pyc + 1 is also the first row of the next window
#pragma unroll
        for (int j = 0; j < kCh; ++j) vm[j] = static_cast<int32_t>(r[j >> 4][j & 15]);
        ++pyc;
        // every column max of the pooled row is in shared memory (and the buffer written here was
        // last read two pooled rows ago, before every thread arrived at the previous meeting)
        mbar_arrive(ep_bar);
        if (!mbar_wait(ep_bar, ep_phase, abort_flag, QG_TIMEOUT_NS)) { ok = false; break; }
        ep_phase ^= 1;
        // pooled pixels px0, px0 + pstride, ... taken SP_PX_ITEMS at a time, so the chains of several
        // pixels interleave (pixels past the row recompute the last one and store nothing)
        const int32_t* col = vrow + 4 * cg;
        const int64_t orow = static_cast<int64_t>(s.img) * p.ph + prow;
        int8_t* const i8_row = p.out_i8 == nullptr ? nullptr
                               : p.i8_cp ? p.out_i8 + (static_cast<int64_t>(p.i8_guard) +
                                                       (static_cast<int64_t>(s.img) * (p.ph + 2) + prow + 1) * (p.pw + 2) + 1) *
                                                          16 + i8_ch
                                         : p.out_i8 + orow * p.pw * p.ld_i8 + ch;
        const int i8_px = p.i8_cp ? 16 : static_cast<int>(p.ld_i8);
        float* const f32_row = p.out_f32 == nullptr ? nullptr : p.out_f32 + orow * p.pw * p.ld_f32 + ch;
        for (int pxb = px0; pxb < p.pw && cg_ok; pxb += SP_PX_ITEMS * pstride) {
          int32_t mx[SP_PX_ITEMS][4];
#pragma unroll
          for (int it = 0; it < SP_PX_ITEMS; ++it) {
            const int px = min(pxb + it * pstride, p.pw - 1);
            const int cx0 = 2 * px - 1;
            int4 t = *reinterpret_cast<const int4*>(col + (2 * px) * SP_PITCH);
            mx[it][0] = t.x; mx[it][1] = t.y; mx[it][2] = t.z; mx[it][3] = t.w;
            if (cx0 >= 0) {
              t = *reinterpret_cast<const int4*>(col + cx0 * SP_PITCH);
              mx[it][0] = max(mx[it][0], t.x); mx[it][1] = max(mx[it][1], t.y);
              mx[it][2] = max(mx[it][2], t.z); mx[it][3] = max(mx[it][3], t.w);
            }
            if (cx0 + 2 < p.ow) {
              t = *reinterpret_cast<const int4*>(col + (cx0 + 2) * SP_PITCH);
              mx[it][0] = max(mx[it][0], t.x); mx[it][1] = max(mx[it][1], t.y);
              mx[it][2] = max(mx[it][2], t.z); mx[it][3] = max(mx[it][3], t.w);
            }
          }
          float v[SP_PX_ITEMS][4];
          uint32_t bad = 0, range = 0;
#pragma unroll
          for (int it = 0; it < SP_PX_ITEMS; ++it)
            dequant4_fold(reinterpret_cast<const uint32_t*>(mx[it]), hs, ls, v[it], bad, range);
          if ((bad | (range & 0xFF800000u)) != 0) {   // rare: the exact product in f64
#pragma unroll
            for (int it = 0; it < SP_PX_ITEMS; ++it)
#pragma unroll
              for (int j = 0; j < 4; ++j)
                v[it][j] = __double2float_rn(static_cast<double>(mx[it][j]) * p.scale64[ch + j]);
          }
          if (p.epi_kind != 0) {
#pragma unroll
            for (int it = 0; it < SP_PX_ITEMS; ++it) {
              if (p.epi_kind & QG_EPI_BIAS) {
                v[it][0] = __fadd_rn(v[it][0], bias.x); v[it][1] = __fadd_rn(v[it][1], bias.y);
                v[it][2] = __fadd_rn(v[it][2], bias.z); v[it][3] = __fadd_rn(v[it][3], bias.w);
              }
              if (p.epi_kind & QG_EPI_RELU) {
#pragma unroll
                for (int j = 0; j < 4; ++j) v[it][j] = np_maximum(v[it][j], 0.0f);
              }
              if (p.epi_kind & QG_EPI_CLAMP) {
#pragma unroll
                for (int j = 0; j < 4; ++j) v[it][j] = np_minimum(np_maximum(v[it][j], clamp_lo), clamp_hi);
              }
            }
          } else {
#pragma unroll
            for (int it = 0; it < SP_PX_ITEMS; ++it)
              for (int st = 0; st < p.n_steps; ++st) {
                const mira_epi_step& e = p.steps[st];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  if (e.operand == MIRA_OPND_NONE) {
                    v[it][j] = apply_unary(e.op, v[it][j]);
                  } else {
                    const float o = e.operand == MIRA_OPND_SCALAR ? e.scalar : __ldg(e.ptr + ch + j);
                    v[it][j] = e.swapped ? apply_binary(e.op, o, v[it][j]) : apply_binary(e.op, v[it][j], o);
                  }
                }
              }
          }
#pragma unroll
          for (int it = 0; it < SP_PX_ITEMS; ++it) {
            const int px = pxb + it * pstride;
            if (px >= p.pw) break;
            if (f32_row != nullptr)
              *reinterpret_cast<float4*>(f32_row + static_cast<int64_t>(px) * p.ld_f32) =
                  make_float4(v[it][0], v[it][1], v[it][2], v[it][3]);
            if (i8_row != nullptr) {
              uint32_t q[4];
              if (p.nonneg) requant_x2<4, true>(v[it], p.q_scale, p.q_rcp, p.q_c127, q);
              else requant_x2<4, false>(v[it], p.q_scale, p.q_rcp, p.q_c127, q);
              *reinterpret_cast<uint32_t*>(i8_row + static_cast<int64_t>(px) * i8_px) = pack4_i8(q[0], q[1], q[2], q[3]);
            }
          }
        }
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
