// K1/K2: the W8A8 matmul and implicit-GEMM convolution on tcgen05.mma kind::i8.
//
// One persistent CTA per SM walks 128 x BN output tiles.  Warp roles:
//   warp 0      TMA producer: B (weights, K-major) and, for matmuls, A tiles into a STAGES-deep
//               ring of shared-memory stages (128-byte swizzle, no multicast)
//   warp 1      allocates TMEM (2 x BN columns: two accumulators) and issues the MMAs from one
//               thread; tcgen05.commit frees a stage / publishes an accumulator
//   warps 2 .. 2+4G-1
//               epilogue: G groups of four warps (any four consecutive warps cover the four TMEM
//               lane quarters, warp w reads lanes 32 * (w % 4) ...).  A group owns every G-th
//               16-column chunk of a tile; one output row per thread: tcgen05.ld, exact dequant,
//               the fused epilogue steps, requantized int8 stores, and f32 stores staged through
//               shared memory so each store instruction writes whole 64-byte row segments
//   next 4 warps (convolutions only) im2col gather of A from NHWC int8 (or, for inputs of at most
//               4 channels, from the row-expanded layout: 16-byte entries holding 4 consecutive
//               pixels, so a kernel row of up to 8 taps is two copies) with cp.async, one output
//               pixel (tile row) per thread, zero fill for padding; each thread's copies arrive on
//               the stage barrier when they land (cp.async.mbarrier.arrive.noinc), so the gather
//               runs up to STAGES K-blocks ahead of the MMAs
// The two TMEM accumulators let the epilogue of tile i overlap the main loop of tile i+1.  The
// epilogue is latency-bound at few warps per scheduler, so G = 4 (16 epilogue warps) is used
// for short reductions and G = 2 with deeper operand pipelines for long ones.
#pragma once
#include <cuda.h>

#include "exact_math.cuh"
#include "ptx_sm100.cuh"

namespace mira {

constexpr int QG_BM = 128;               // tile rows = TMEM lanes
constexpr int QG_BK = 128;               // K bytes per stage = one 128-byte swizzle row
constexpr int QG_UMMA_K = 32;            // K per tcgen05.mma kind::i8
constexpr uint64_t QG_TIMEOUT_NS = 2000000000ull;

enum QgAMode { QG_A_TMA = 0, QG_A_GATHER16 = 1, QG_A_GATHER4 = 2, QG_A_ROW4 = 3, QG_A_IM2COL = 4, QG_A_PATCH = 5 };

// A operand comes from TMA (2-D tiles of a row-major matrix, or im2col tiles of an NHWC tensor)
// into the stages of the operand ring, rather than from the cp.async gather warps.
constexpr bool qg_a_by_tma(int amode) { return amode == QG_A_TMA || amode == QG_A_IM2COL; }
// A operand is a tile's whole input halo, bulk-copied once per tile from the chunk-planar layout
// (3x3 stride-1 convolutions): no gather warps, the ring stages carry weights only.
constexpr bool qg_a_patch(int amode) { return amode == QG_A_PATCH; }
constexpr bool qg_a_async(int amode) { return qg_a_by_tma(amode) || qg_a_patch(amode); }

// n / d for 0 <= n < 2^31 without a divide: q = (hi32(n * mul) + n) >> shr, with shr = ceil(log2 d)
// and mul = floor(2^32 (2^shr - d) / d) + 1 computed on the host (the round-up multiplier method).
struct QgDiv {
  uint32_t mul, shr;
};

__device__ __forceinline__ int qg_div(int n, QgDiv d) {
  return static_cast<int>((__umulhi(static_cast<uint32_t>(n), d.mul) + static_cast<uint32_t>(n)) >> d.shr);
}

struct QgConv {
  int n, h, w, cp;      // input NHWC (cp = padded channels)
  int oh, ow;
  int kh, kw, sh, sw, ph, pw, dh, dw;
  int row_entries;      // QG_A_ROW4: 16-byte entries per image row (entry e = pixels sw*e - pw .. sw*e - pw + 3)
  // QG_A_PATCH (chunk-planar input, 3x3 stride 1 pad 1): guard slots, slots per chunk plane, and
  // the slots of one tile's halo (128 + 2 (w + 3)); GEMM rows are the padded output slots
  int guard, patch_slots;
  int64_t plane;
};

struct QgParams {
  int M, N, K;          // K = bytes of the reduction actually used
  int num_kb;           // ceil(K / QG_BK)
  int m_tiles, n_tiles;
  // split-K (TMA mode): tile t covers output tile t % (m_tiles * n_tiles) and K-blocks
  // [s * kb_per_split, (s + 1) * kb_per_split) with s = t / (m_tiles * n_tiles); with raw set the
  // epilogue stores the int32 accumulators (as 4-byte words) to out_f32 + s * split_stride
  int k_splits, kb_per_split;
  int raw;
  int64_t split_stride;
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
  float q_c127;                  // RN32(127 * divisor): the clamp of the packed requantization
  // int8 output layout: rows of ld_i8 bytes (i8_cp = 0, i8_chunk = 16), or chunk-planar for a
  // convolution's output (i8_cp = 1: slot guard + c16 * plane + padded pixel, i8_chunk = plane * 16)
  int i8_cp, i8_guard;
  int64_t i8_chunk;
  // tile index math: divisors n_tiles and m_tiles * n_tiles; row mapping of convolutions: PATCH rows
  // by (oh + 2)(ow + 2) and ow + 2, chunk-planar int8 output of other convs by oh * ow and ow
  QgDiv dv_ntiles, dv_mntiles, dv_a, dv_b;
  // the epilogue's last steps leave no negative value (relu, maximum with a scalar >= 0, then at
  // most minimum with a scalar >= 0): requantization clamps from above only
  int nonneg;
  // a common step sequence run as one fused program (QG_EPI_* flags), 0: the general step loop
  int epi_kind;
  int* err;
  // fused max pooling (POOL kernels only): window pool_p, stride pool_s, padding pool_pad holding
  // pool_pad_value; a tile is pool_t x pool_t pooled pixels whose conv inputs form a
  // pool_span x pool_span block (pool_span = (pool_t - 1) * pool_s + pool_p, pool_span^2 <= 128)
  int pool_p, pool_s, pool_pad, pool_t, pool_span, ph_out, pw_out, tiles_y, tiles_x;
  float pool_pad_value;
};

// Tile row r of a POOL tile (tile index t_m over images x tiles_y x tiles_x): the conv output
// pixel it computes, and whether that pixel exists.
__device__ __forceinline__ void pool_row_pixel(const QgParams& p, int t_m, int r, int& img, int& cy, int& cx,
                                               int& ty, int& tx, bool& valid) {
  const int per_img = p.tiles_y * p.tiles_x;
  img = t_m / per_img;
  const int rem = t_m - img * per_img;
  ty = rem / p.tiles_x;
  tx = rem - ty * p.tiles_x;
  const int ry = r / p.pool_span, rx = r - ry * p.pool_span;
  cy = ty * p.pool_t * p.pool_s - p.pool_pad + ry;
  cx = tx * p.pool_t * p.pool_s - p.pool_pad + rx;
  valid = r < p.pool_span * p.pool_span && cy >= 0 && cy < p.g.oh && cx >= 0 && cx < p.g.ow;
}

// RKB > 0: the whole B operand (at most RKB K-blocks) stays in shared memory for the CTA's lifetime
// (one output column tile, loaded once); the stages then carry A only.
// PATCH > 0 (QG_A_PATCH): bytes of one of the two halo buffers that replace the A stages.
template <int BN, int STAGES, int AMODE, int G, bool POOL = false, int BK = QG_BK, int RKB = 0, int PATCH = 0>
struct QgCfg {
  static constexpr int A_BYTES = QG_BM * BK;
  static constexpr int B_BYTES = BN * BK;
  // TMEM accumulators in flight: the MMA warp can run that many tiles ahead of the epilogue (four
  // when the tile width leaves room in the 512 columns; POOL kernels pair them with two pooling
  // buffers)
  static constexpr int ACCS = (!POOL && BN <= 128) ? 4 : 2;
  static constexpr int CW = 16;                       // epilogue chunk width (columns)
  static constexpr int EPI_WARP0 = 2;
  static constexpr int EPI_WARPS = 4 * G;
  static constexpr int GATHER_WARP0 = EPI_WARP0 + EPI_WARPS;
  static constexpr int THREADS = 32 * (GATHER_WARP0 + (qg_a_async(AMODE) ? 0 : 4));
  static constexpr int EPI_THREADS = 32 * EPI_WARPS;
  static constexpr uint32_t TMEM_COLS = ACCS * BN;
  // per epilogue warp: a 32-row x 16-column f32 staging block (row pitch 20 floats)
  static constexpr int STAGE_PITCH = 20;
  // POOL kernels instead keep two 128-row x BN conv-output tiles (row pitch BN + 4 floats)
  static constexpr int POOL_PITCH = BN + 4;
  static constexpr int POOL_ROWS = 96;
  static constexpr int STAGING_BYTES = POOL ? 2 * POOL_ROWS * POOL_PITCH * 4 : EPI_WARPS * 32 * STAGE_PITCH * 4;
  static constexpr int B_REGION = RKB > 0 ? RKB * B_BYTES : STAGES * B_BYTES;
  // the barrier region after the staging: the stage, accumulator and halo barriers, drain, pool,
  // resident-B, then the TMEM address and the abort flag
  static constexpr int NBAR = 2 * STAGES + 2 * ACCS + 2 * 6 + 4;
  static constexpr int BAR_BYTES = 8 * NBAR + 8 <= 256 ? 256 : 512;
  static constexpr int FIXED_BYTES = 1024 + B_REGION + STAGING_BYTES + BAR_BYTES;
  // PATCH: halo buffers in flight (the producer fetches up to NHALO - 1 tiles ahead of the MMAs),
  // as many as shared memory leaves room for, at most 6
  static constexpr int NHALO_FIT = PATCH > 0 ? (232448 - FIXED_BYTES) / PATCH : 0;
  static constexpr int NHALO = PATCH == 0 ? 1 : (NHALO_FIT > 6 ? 6 : NHALO_FIT);
  static constexpr int A_REGION = qg_a_patch(AMODE) ? NHALO * PATCH : STAGES * A_BYTES;
  static constexpr size_t SMEM = size_t(FIXED_BYTES) + A_REGION;
  static_assert(!POOL || (AMODE != 0 && BN == 64), "fused pooling: convolutions with at most 64 channels");
  static_assert(BN == 64 || BN == 128 || BN == 256, "BN");
  static_assert(SMEM <= 232448, "shared memory budget");
  static_assert(8 * NBAR + 8 <= BAR_BYTES, "barrier region");
  static_assert(!qg_a_patch(AMODE) || NHALO >= 2, "at least two halo buffers");
  static_assert(BK == 128 || (BK == 64 && (AMODE == QG_A_IM2COL || AMODE == QG_A_PATCH)),
                "64-byte K-blocks: convolutions with 64-channel inputs only");
  static_assert(qg_a_patch(AMODE) == (PATCH > 0) && PATCH % 1024 == 0, "halo buffers: PATCH mode only");
};

// Bounded wait that ignores the abort flag: used only to let in-flight copies land before exit.
__device__ __forceinline__ void mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait_suspend(bar, parity, 1000000u)) {
    if (globaltimer_ns() - t0 > QG_TIMEOUT_NS) return;
  }
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// ---------------------------------------------------------------- epilogue (one 16-column chunk)

// Fused programs for the step sequences the networks use, in the order they run: add of a
// per-channel operand (steps[0]), add of a full operand (steps[1]), relu, or maximum then minimum
// with scalars (ReLU6, the last two steps).  The same IEEE operations in the same order as the
// general loop, without its per-step dispatch.
enum : int { QG_EPI_BIAS = 1, QG_EPI_RES = 2, QG_EPI_RELU = 4, QG_EPI_CLAMP = 8 };

// Where GEMM row m of a tile goes: the f32 row (output pixel; operands with rows are read there
// too), the byte offset of its int8 output row, and whether the row exists.  Plain GEMMs and the
// convolutions other than PATCH have row m = pixel m; PATCH convolutions compute every slot of the
// zero-padded output plane, and the padding slots are not written.
struct QgRow {
  int64_t pix;
  int64_t i8;
  bool ok;
};

template <int AMODE>
__device__ __forceinline__ QgRow qg_row(const QgParams& p, int m) {
  QgRow r;
  if (AMODE == QG_A_PATCH) {
    const int pw = p.g.ow + 2, pimg = (p.g.oh + 2) * pw;
    const int img = qg_div(m, p.dv_a), rem = m - img * pimg, yy = qg_div(rem, p.dv_b), xx = rem - yy * pw;
    r.ok = m < p.M && yy >= 1 && yy <= p.g.oh && xx >= 1 && xx <= p.g.ow;
    r.pix = r.ok ? (static_cast<int64_t>(img) * p.g.oh + yy - 1) * p.g.ow + xx - 1 : 0;
    r.i8 = p.i8_cp ? (static_cast<int64_t>(p.i8_guard) + m) * 16 : r.pix * p.ld_i8;
  } else {
    r.ok = m < p.M;
    r.pix = m;
    r.i8 = static_cast<int64_t>(m) * p.ld_i8;
    if (p.i8_cp && r.ok) {
      const int hw = p.g.oh * p.g.ow;
      const int img = qg_div(m, p.dv_a), rem = m - img * hw, y = qg_div(rem, p.dv_b), x = rem - y * p.g.ow;
      r.i8 = (static_cast<int64_t>(p.i8_guard) +
              (static_cast<int64_t>(img) * (p.g.oh + 2) + y + 1) * (p.g.ow + 2) + x + 1) * 16;
    }
  }
  return r;
}

#define QG_APPLY_BINARY(EXPR)                          \
  do {                                                 \
    if (st.swapped) {                                  \
      _Pragma("unroll") for (int j = 0; j < 16; ++j) { \
        const float a = o[j], b = v[j];                \
        v[j] = (EXPR);                                 \
      }                                                \
    } else {                                           \
      _Pragma("unroll") for (int j = 0; j < 16; ++j) { \
        const float a = v[j], b = o[j];                \
        v[j] = (EXPR);                                 \
      }                                                \
    }                                                  \
  } while (0)

__device__ __forceinline__ void ld16(const float* src, float (&o)[16]) {
  const float4* s4 = reinterpret_cast<const float4*>(src);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 t = __ldg(s4 + q);
    o[4 * q] = t.x; o[4 * q + 1] = t.y; o[4 * q + 2] = t.z; o[4 * q + 3] = t.w;
  }
}

// Loads a binary step's operand for this thread's row and chunk columns [nb, nb + 16).
__device__ __forceinline__ void qg_operand(const QgParams& p, const mira_epi_step& st, int64_t m, bool row_ok, int nb,
                                           bool full_chunk, float (&o)[16]) {
  if (st.operand == MIRA_OPND_SCALAR) {
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j] = st.scalar;
  } else if (st.operand == MIRA_OPND_CHANNEL) {
    ld16(st.ptr + nb, o);   // channel arrays are padded to a multiple of 256 entries
  } else if (st.operand == MIRA_OPND_ROW) {
    const float t = row_ok ? st.ptr[m] : 0.0f;
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j] = t;
  } else {  // FULL
    const float* src = st.ptr + m * st.ld + nb;
    if (!row_ok) {
#pragma unroll
      for (int j = 0; j < 16; ++j) o[j] = 0.0f;
    } else if (full_chunk && (st.ld % 4) == 0) {
      ld16(src, o);
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) o[j] = (nb + j < p.N) ? src[j] : 0.0f;
    }
  }
}

// Stores this thread's 16 values of a chunk: through the warp's staging block (coalesced 16-byte
// stores of whole rows) when the chunk is full and rows are 16-byte aligned, else directly.  With
// MAPPED rows the other rows' pixels come from their lanes.
template <int PITCH, bool MAPPED>
__device__ __forceinline__ void qg_store_f32(const QgParams& p, const float (&v)[16], const QgRow& row, int m_warp0,
                                             int nb, bool full_chunk, float* stage, int lane, float* out_f32) {
  if (full_chunk && (p.ld_f32 % 4) == 0) {
    float4* srow = reinterpret_cast<float4*>(stage + lane * PITCH);
#pragma unroll
    for (int q = 0; q < 4; ++q) srow[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int rr = i * 8 + (lane >> 2), qq = lane & 3;
      const float4 t = reinterpret_cast<const float4*>(stage + rr * PITCH)[qq];
      int64_t pr;
      bool okr;
      if (MAPPED) {
        // each lane left its row's pixel (-1: a padding slot) in the pad column of its staging row
        pr = reinterpret_cast<const int*>(stage)[rr * PITCH + 16];
        okr = pr >= 0;
      } else {
        pr = m_warp0 + rr;
        okr = pr < p.M;
      }
      if (okr) reinterpret_cast<float4*>(out_f32 + pr * p.ld_f32 + nb)[qq] = t;
    }
    __syncwarp();
  } else if (row.ok) {
    float* dst = out_f32 + row.pix * p.ld_f32 + nb;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (nb + j < p.N) dst[j] = v[j];
  }
}

__device__ __forceinline__ void qg_apply_step(const mira_epi_step& st, const float (&o)[16], float (&v)[16]) {
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

// A binary step on 16 values: add/sub two lanes per instruction, the others one by one.  A
// multiply stays scalar: ptxas fuses a packed mul.rn.f32x2 with a following packed add into one
// fma (measured on sm_100a), which would round a mul step and the next add step once instead of
// twice; the scalar mul.rn.f32 with its explicit rounding mode is never fused.
__device__ __forceinline__ void qg_apply_binary(const mira_epi_step& st, const float (&o)[16], float (&v)[16]) {
  if (st.op == MIRA_EPI_ADD || st.op == MIRA_EPI_SUB) {
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      const f2_t x = f2(v[j], v[j + 1]), y = f2(o[j], o[j + 1]);
      f2_t r;
      if (st.op == MIRA_EPI_ADD) r = f2_add(x, y);                // commutative: swapped gives the same
      else r = st.swapped ? f2_sub(y, x) : f2_sub(x, y);
      f2_split(r, v[j], v[j + 1]);
    }
    return;
  }
  qg_apply_step(st, o, v);
}

// The whole epilogue of one 16-column chunk of this warp's 32 rows.  Everything that does not
// depend on the accumulator (dequant scales, the first binary operand) is loaded before the TMEM
// read so the two latencies overlap.  In raw mode (split-K partial sums) the int32 accumulators
// are stored unchanged.
template <bool ROWCOL, int PITCH, bool MAPPED = false>
__device__ __forceinline__ void qg_epilogue_chunk(const QgParams& p, uint32_t taddr, const QgRow& row, int m_warp0,
                                                  int nb, float* stage, int lane, float* out_f32) {
  const bool full_chunk = nb + 16 <= p.N;
  const int64_t m = row.pix;
  const bool row_ok = row.ok;
  if (p.raw) {
    uint32_t r[16];
    tmem_ld_32x32b_x16(taddr, r);
    tmem_ld_wait();
    float v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
    qg_store_f32<PITCH, MAPPED>(p, v, row, m_warp0, nb, full_chunk, stage, lane, out_f32);
    return;
  }
  float hs[16], ls[16];
  if (!ROWCOL) {
    ld16(p.scale_hi + nb, hs);
    ld16(p.scale_lo + nb, ls);
  } else {
    const float rs = row_ok ? p.row_scale[m] : 0.0f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float cs = (nb + j < p.N) ? __ldg(p.col_scale + nb + j) : 0.0f;
      split_rowcol(rs, cs, hs[j], ls[j]);
    }
  }
  // operands that read memory are fetched before the accumulator so their latency overlaps the
  // TMEM read: for a fused program its bias and residual, for the general loop one full-tensor
  // operand (a residual in DRAM) if there is one, else the first per-channel or per-row one
  const int kind = p.epi_kind;
  int mem0 = -1;
  float o0[16], o1[16];
  if (kind != 0) {
    if (kind & QG_EPI_BIAS) ld16(p.steps[0].ptr + nb, o0);
    if (kind & QG_EPI_RES) qg_operand(p, p.steps[1], m, row_ok, nb, full_chunk, o1);
  } else {
    for (int s = 0; s < p.n_steps; ++s) {
      const int opnd = p.steps[s].operand;
      if (opnd == MIRA_OPND_FULL) {
        mem0 = s;
        break;
      }
      if (mem0 < 0 && (opnd == MIRA_OPND_CHANNEL || opnd == MIRA_OPND_ROW)) mem0 = s;
    }
    if (mem0 >= 0) qg_operand(p, p.steps[mem0], m, row_ok, nb, full_chunk, o0);
  }

  uint32_t r[16];
  tmem_ld_32x32b_x16(taddr, r);
  tmem_ld_wait();

  float v[16];
  const bool exact = dequant16_x2(r, hs, ls, v);
  if (__any_sync(0xffffffffu, !exact)) {   // rare: about 3 chunks in 10^4 have an element to redo
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (!exact) {
        const double s64 = ROWCOL ? static_cast<double>(row_ok ? p.row_scale[m] : 0.0f) *
                                        static_cast<double>((nb + j < p.N) ? p.col_scale[nb + j] : 0.0f)
                                  : p.scale64[nb + j];
        v[j] = __double2float_rn(static_cast<double>(static_cast<int32_t>(r[j])) * s64);
      }
    }
  }

  if (kind != 0) {
    if (kind & QG_EPI_BIAS) {
#pragma unroll
      for (int j = 0; j < 16; j += 2) f2_split(f2_add(f2(v[j], v[j + 1]), f2(o0[j], o0[j + 1])), v[j], v[j + 1]);
    }
    if (kind & QG_EPI_RES) {
#pragma unroll
      for (int j = 0; j < 16; j += 2) f2_split(f2_add(f2(v[j], v[j + 1]), f2(o1[j], o1[j + 1])), v[j], v[j + 1]);
    }
    if (kind & QG_EPI_RELU) {
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = np_maximum(v[j], 0.0f);
    }
    if (kind & QG_EPI_CLAMP) {
      const float lo = p.steps[p.n_steps - 2].scalar, hi = p.steps[p.n_steps - 1].scalar;
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = np_minimum(np_maximum(v[j], lo), hi);
    }
  }
  for (int s = 0; kind == 0 && s < p.n_steps; ++s) {
    const mira_epi_step& st = p.steps[s];
    if (st.operand == MIRA_OPND_NONE) {
      if (st.op == MIRA_EPI_RELU) {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = np_maximum(v[j], 0.0f);
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = apply_unary(st.op, v[j]);
      }
      continue;
    }
    if (s == mem0) {
      qg_apply_binary(st, o0, v);
    } else {
      float o[16];
      qg_operand(p, st, m, row_ok, nb, full_chunk, o);
      qg_apply_binary(st, o, v);
    }
  }

  if (out_f32 != nullptr) qg_store_f32<PITCH, MAPPED>(p, v, row, m_warp0, nb, full_chunk, stage, lane, out_f32);
  if (p.out_i8 != nullptr && row_ok && nb < p.ld_i8) {
    uint32_t b[16];
    if (p.nonneg) requant_x2<16, true>(v, p.q_scale, p.q_rcp, p.q_c127, b);
    else requant_x2<16, false>(v, p.q_scale, p.q_rcp, p.q_c127, b);
    if (!full_chunk) {
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (nb + j >= p.N) b[j] = 0u;
    }
    *reinterpret_cast<uint4*>(p.out_i8 + row.i8 + (nb >> 4) * p.i8_chunk) =
        make_uint4(pack4_i8(b[0], b[1], b[2], b[3]), pack4_i8(b[4], b[5], b[6], b[7]),
                   pack4_i8(b[8], b[9], b[10], b[11]), pack4_i8(b[12], b[13], b[14], b[15]));
  }
}

// ---------------------------------------------------------------- the kernel

template <int BN, int STAGES, int AMODE, bool ROWCOL, int G, bool POOL = false, int BK = QG_BK, int RKB = 0,
          int PATCH = 0>
__global__ void __launch_bounds__(QgCfg<BN, STAGES, AMODE, G, POOL, BK, RKB, PATCH>::THREADS, 1)
    qgemm_sm100_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       const __grid_constant__ QgParams p) {
  using Cfg = QgCfg<BN, STAGES, AMODE, G, POOL, BK, RKB, PATCH>;
  constexpr int A_BYTES = Cfg::A_BYTES;
  constexpr int B_BYTES = Cfg::B_BYTES;
  constexpr uint32_t IDESC = idesc_i8(QG_BM, BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + Cfg::A_REGION;
  float* staging = reinterpret_cast<float*>(sB + Cfg::B_REGION);
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(staging) + Cfg::STAGING_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + Cfg::ACCS;
  uint64_t* drain = tempty + Cfg::ACCS;
  uint64_t* pool_bar = drain + 1;   // [2]: all epilogue threads wrote the tile buffer
  uint64_t* bres = pool_bar + 2;    // resident B landed (RKB > 0)
  uint64_t* pfull = bres + 1;       // [NHALO]: a halo buffer landed (PATCH)
  uint64_t* pempty = pfull + 6;     // [NHALO]: the MMAs reading a halo buffer finished (PATCH)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(pempty + 6);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], qg_a_async(AMODE) ? 1 : 1 + 128);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < Cfg::ACCS; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], Cfg::EPI_THREADS);
    }
    mbar_init(drain, 1);
    mbar_init(&pool_bar[0], Cfg::EPI_THREADS);
    mbar_init(&pool_bar[1], Cfg::EPI_THREADS);
    mbar_init(bres, 1);
    for (int b = 0; b < Cfg::NHALO; ++b) {
      mbar_init(&pfull[b], 1);
      mbar_init(&pempty[b], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmB);
    if (qg_a_by_tma(AMODE)) tma_prefetch_desc(&tmA);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_holder);

  const int mn_tiles = p.m_tiles * p.n_tiles;
  const int num_tiles = mn_tiles * p.k_splits;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer (lane 0; in PATCH mode the whole
    // warp, whose lanes issue the halo planes' bulk copies together: a copy costs the issuing thread
    // several hundred cycles, copies issued by different lanes in one instruction overlap)
    if (lane == 0 || AMODE == QG_A_PATCH) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0, patches = 0;
      bool ok = true;
      if (RKB > 0 && blockIdx.x < num_tiles && lane == 0) {
        // the whole B operand (one column tile, checked by the host) once for the CTA
        mbar_arrive_expect_tx(bres, p.num_kb * B_BYTES);
        for (int kb = 0; kb < p.num_kb; ++kb) tma_load_2d(sB + kb * B_BYTES, &tmB, kb * BK, 0, bres);
      }
      for (int t = blockIdx.x, it = 0; t < num_tiles && ok; t += gridDim.x, ++it) {
        const int split = qg_div(t, p.dv_mntiles), t_mn = t - split * mn_tiles;
        const int t_m = qg_div(t_mn, p.dv_ntiles);
        const int m0 = t_m * QG_BM;
        const int n0 = (t_mn - t_m * p.n_tiles) * BN;
        const int kb0 = split * p.kb_per_split, kb1 = min(p.num_kb, kb0 + p.kb_per_split);
        if (AMODE == QG_A_PATCH) {
          // the tile's input halo: output slots m0 .. m0 + 127 read input slots m0 - (w + 3) ..
          // m0 + 127 + (w + 3) of every chunk plane (guards and padding ring are zero)
          const int pb = it % Cfg::NHALO;
          bool free_buf = true;
          if (lane == 0) free_buf = mbar_wait(&pempty[pb], ((it / Cfg::NHALO) & 1) ^ 1, abort_flag, QG_TIMEOUT_NS);
          if (!__shfl_sync(0xffffffffu, free_buf ? 1 : 0, 0)) { ok = false; break; }
          const uint32_t pbytes = static_cast<uint32_t>(p.g.patch_slots) * 16u;
          const int planes = p.g.cp >> 4;
          if (lane == 0) mbar_arrive_expect_tx(&pfull[pb], planes * pbytes);
          __syncwarp();
          const int8_t* src = p.A + (static_cast<int64_t>(p.g.guard) + m0 - (p.g.ow + 3)) * 16;
          for (int c = lane; c < planes; c += 32)
            bulk_load(sA + pb * PATCH + c * pbytes, src + c * p.g.plane * 16, pbytes, &pfull[pb]);
          ++patches;
          if (RKB > 0) continue;
        }
        if (AMODE != QG_A_PATCH || lane == 0) {   // the K-block stages: lane 0 alone
          // im2col: traversal position of the tile's first output pixel
          int iw0 = 0, ih0 = 0, img0 = 0;
          if (AMODE == QG_A_IM2COL) {
            const int hw = p.g.oh * p.g.ow;
            img0 = m0 / hw;
            const int rem = m0 - img0 * hw;
            const int oy = rem / p.g.ow;
            iw0 = (rem - oy * p.g.ow) * p.g.sw - p.g.pw;
            ih0 = oy * p.g.sh - p.g.ph;
          }
          for (int kb = kb0; kb < kb1; ++kb) {
            if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, QG_TIMEOUT_NS)) { ok = false; break; }
            mbar_arrive_expect_tx(&full[stage], (qg_a_by_tma(AMODE) ? A_BYTES : 0) + (RKB > 0 ? 0 : B_BYTES));
            if (AMODE == QG_A_TMA) tma_load_2d(sA + stage * A_BYTES, &tmA, kb * BK, m0, &full[stage]);
            if (AMODE == QG_A_IM2COL) {
              // K-block kb = channels [c0, c0 + BK) of tap (i, j): k = (i * kw + j) * cp + c
              const int kbyte = kb * BK;
              const int tap = kbyte / p.g.cp;
              const int c0 = kbyte - tap * p.g.cp;
              const int ti = tap / p.g.kw, tj = tap - ti * p.g.kw;
              tma_load_im2col_4d(sA + stage * A_BYTES, &tmA, c0, iw0, ih0, img0, static_cast<uint16_t>(tj * p.g.dw),
                                 static_cast<uint16_t>(ti * p.g.dh), &full[stage]);
            }
            if (RKB == 0) tma_load_2d(sB + stage * B_BYTES, &tmB, kb * BK, n0, &full[stage]);
            ++issued;
            if (++stage == STAGES) { stage = 0; phase ^= 1; }
          }
        }
        if (AMODE == QG_A_PATCH) ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      }
      if (!ok && lane == 0) {
        // let the copies already issued land before the CTA can exit
        for (int i = 1; i <= STAGES && i <= issued; ++i) {
          const int idx = issued - i;
          mbar_wait_drain(&full[idx % STAGES], (idx / STAGES) & 1);
        }
        for (int i = 1; i <= Cfg::NHALO && i <= patches; ++i) {
          const int idx = patches - i;
          mbar_wait_drain(&pfull[idx % Cfg::NHALO], (idx / Cfg::NHALO) & 1);
        }
      }
      if (RKB > 0 && blockIdx.x < num_tiles && lane == 0) mbar_wait_drain(bres, 0);
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      if (RKB > 0 && blockIdx.x < num_tiles && !mbar_wait(bres, 0, abort_flag, QG_TIMEOUT_NS)) ok = false;
      // PATCH mode with resident weights waits on nothing per K-block: the halo and B are in place
      constexpr bool kStaged = !(AMODE == QG_A_PATCH && RKB > 0);
      // The operand descriptors are built once: a stage, a K step or a tap shift only moves the start
      // address field (16-byte units in the low 14 bits; shared addresses stay below 256 KB, so no
      // carry leaves the field), so each MMA costs one add per operand.  A single thread issues every
      // MMA, and rebuilding both descriptors per instruction made its dependent integer chain, not the
      // tensor pipe, the limit of the main loop.
      constexpr uint32_t KU = QG_UMMA_K >> 4;   // one MMA's K step (32 bytes) in 16-byte units
      const uint64_t b_desc0 = BK == 64 ? smem_desc_k_sw64(smem_u32(sB)) : smem_desc_k_sw128(smem_u32(sB));
      const uint64_t a_desc0 =
          qg_a_patch(AMODE) ? smem_desc_k_none(smem_u32(sA), static_cast<uint32_t>(p.g.patch_slots) * 16u, 128)
                            : (BK == 64 ? smem_desc_k_sw64(smem_u32(sA)) : smem_desc_k_sw128(smem_u32(sA)));
      // PATCH: the slot shift of each tap and one halo plane, in descriptor units (16-byte slots)
      uint32_t tap_u[9];
      uint32_t plane_u = 0;
      int kbc = 1;
      if (AMODE == QG_A_PATCH) {
#pragma unroll
        for (int tp = 0; tp < 9; ++tp)
          tap_u[tp] = static_cast<uint32_t>(p.g.ow + 3 + (tp / 3 - 1) * (p.g.ow + 2) + (tp % 3 - 1));
        plane_u = static_cast<uint32_t>(p.g.patch_slots);
        kbc = p.g.cp / BK;
      }
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++it) {
        const int acc = it % Cfg::ACCS;
        if (!mbar_wait(&tempty[acc], ((it / Cfg::ACCS) & 1) ^ 1, abort_flag, QG_TIMEOUT_NS)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        if (AMODE == QG_A_PATCH) {
          // K-block (tap, cb) = channels [cb * BK, cb * BK + BK) of tap (tap / 3, tap % 3): the A rows
          // are the halo's slots shifted by the tap, each 16-channel chunk one plane of the halo
          const int hb = it % Cfg::NHALO;
          if (!mbar_wait(&pfull[hb], (it / Cfg::NHALO) & 1, abort_flag, QG_TIMEOUT_NS)) { ok = false; break; }
          tc_fence_after();
          const uint64_t halo_d = a_desc0 + static_cast<uint64_t>(hb) * (PATCH >> 4);
          uint32_t accum = 0;
          if (RKB > 0 && BK == 64) {
            // one 64-channel K-block per tap, weights resident: the tile's 18 MMAs as straight-line
            // code, each operand one add away from a per-CTA constant
#pragma unroll
            for (int tp = 0; tp < 9; ++tp) {
#pragma unroll
              for (int kk = 0; kk < BK / QG_UMMA_K; ++kk) {
                mma_i8(d_tmem, halo_d + tap_u[tp] + kk * KU * plane_u,
                       b_desc0 + static_cast<uint64_t>(tp * (B_BYTES >> 4) + kk * KU), IDESC, accum);
                accum = 1;
              }
            }
          }
#pragma unroll
          for (int tp = 0; tp < 9 && !(RKB > 0 && BK == 64); ++tp) {
            for (int cb = 0; cb < kbc && ok; ++cb) {
              const int kb = tp * kbc + cb;
              if (kStaged) {
                if (!mbar_wait(&full[stage], phase, abort_flag, QG_TIMEOUT_NS)) { ok = false; break; }
                tc_fence_after();
              }
              const uint64_t a_d = halo_d + tap_u[tp] + static_cast<uint64_t>(cb * (BK >> 4)) * plane_u;
              const uint64_t b_d = b_desc0 + static_cast<uint64_t>((RKB > 0 ? kb : stage) * (B_BYTES >> 4));
#pragma unroll
              for (int kk = 0; kk < BK / QG_UMMA_K; ++kk) {
                mma_i8(d_tmem, a_d + static_cast<uint64_t>(kk * KU) * plane_u, b_d + kk * KU, IDESC, accum);
                accum = 1;
              }
              if (kStaged) {
                mma_commit(&empty[stage]);
                if (++stage == STAGES) { stage = 0; phase ^= 1; }
              }
            }
          }
          if (ok) mma_commit(&pempty[hb]);
        } else {
          const int split = qg_div(t, p.dv_mntiles);
          const int kb0 = split * p.kb_per_split, kb1 = min(p.num_kb, kb0 + p.kb_per_split);
          for (int kb = kb0; kb < kb1; ++kb) {
            if (!mbar_wait(&full[stage], phase, abort_flag, QG_TIMEOUT_NS)) { ok = false; break; }
            if (!qg_a_async(AMODE)) fence_proxy_async_smem();  // A was written by cp.async (generic proxy)
            tc_fence_after();
            const uint64_t a_d = a_desc0 + static_cast<uint64_t>(stage * (A_BYTES >> 4));
            const uint64_t b_d = b_desc0 + static_cast<uint64_t>((RKB > 0 ? kb : stage) * (B_BYTES >> 4));
            const int rem = p.K - kb * BK;
            if (rem >= BK) {
#pragma unroll
              for (int kk = 0; kk < BK / QG_UMMA_K; ++kk)
                mma_i8(d_tmem, a_d + kk * KU, b_d + kk * KU, IDESC, (kb != kb0 || kk != 0) ? 1u : 0u);
            } else {
              const int nk = (rem + QG_UMMA_K - 1) / QG_UMMA_K;
              for (int kk = 0; kk < nk; ++kk)
                mma_i8(d_tmem, a_d + kk * KU, b_d + kk * KU, IDESC, (kb != kb0 || kk != 0) ? 1u : 0u);
            }
            mma_commit(&empty[stage]);
            if (++stage == STAGES) { stage = 0; phase ^= 1; }
          }
        }
        if (ok) mma_commit(&tfull[acc]);
      }
      // every MMA issued by this thread has finished once `drain` completes
      mma_commit(drain);
      mbar_wait_drain(drain, 0);
    }
  } else if (warp >= Cfg::EPI_WARP0 && warp < Cfg::GATHER_WARP0) {
    // ------------------------------------------------ epilogue
    const int ew = warp - Cfg::EPI_WARP0;
    const int quarter = warp & 3;
    const int group = ew >> 2;
    float* stage = staging + ew * 32 * Cfg::STAGE_PITCH;
    int it = 0;
    // a residual operand (one f32 row per output row) is read from DRAM in the epilogue; each
    // thread asks L2 for its rows of the next tile while this one is processed
    const bool prefetch_res = !POOL && !p.raw && (p.epi_kind & QG_EPI_RES) != 0 &&
                              p.steps[1].operand == MIRA_OPND_FULL;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
      const int acc = it % Cfg::ACCS;
      if (prefetch_res && t + static_cast<int>(gridDim.x) < num_tiles) {
        const int tn = t + gridDim.x;
        const int sn = qg_div(tn, p.dv_mntiles), tn_mn = tn - sn * mn_tiles;
        const int tn_m = qg_div(tn_mn, p.dv_ntiles);
        const int n0n = (tn_mn - tn_m * p.n_tiles) * BN;
        const QgRow rn = qg_row<AMODE>(p, tn_m * QG_BM + quarter * 32 + lane);
        if (rn.ok) {
          for (int c = group; c < BN / Cfg::CW; c += G) {
            const int nb = n0n + c * Cfg::CW;
            if (nb < p.N) prefetch_l2(p.steps[1].ptr + rn.pix * p.steps[1].ld + nb);
          }
        }
      }
      if (!mbar_wait(&tfull[acc], (it / Cfg::ACCS) & 1, abort_flag, QG_TIMEOUT_NS)) break;
      tc_fence_after();
      const int split = qg_div(t, p.dv_mntiles), t_mn = t - split * mn_tiles;
      const int t_m = qg_div(t_mn, p.dv_ntiles);
      const int n0 = (t_mn - t_m * p.n_tiles) * BN;
      float* out_f32 = p.out_f32 != nullptr ? p.out_f32 + split * p.split_stride : nullptr;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
      if (!POOL) {
        const int m_warp0 = t_m * QG_BM + quarter * 32;
        const QgRow row = qg_row<AMODE>(p, m_warp0 + lane);
        if (AMODE == QG_A_PATCH) reinterpret_cast<int*>(stage)[lane * Cfg::STAGE_PITCH + 16] = row.ok ? int(row.pix) : -1;
#pragma unroll 1
        for (int c = group; c < BN / Cfg::CW; c += G) {
          const int nb = n0 + c * Cfg::CW;
          if (nb >= p.N) break;  // warp-uniform
          qg_epilogue_chunk<ROWCOL, Cfg::STAGE_PITCH, AMODE == QG_A_PATCH>(p, tbase + c * Cfg::CW, row, m_warp0, nb,
                                                                         stage, lane, out_f32);
        }
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
      } else {
        // The conv epilogue (dequant, then steps that the host checked are monotone non-decreasing)
        // commutes with max, so the int32 accumulators are pooled first and the epilogue runs on the
        // pooled values only: accumulators -> shared tile (acc parity) -> window max -> epilogue.
        const int r = quarter * 32 + lane;
        int img, cy, cx, ty, tx;
        bool valid;
        pool_row_pixel(p, t_m, r, img, cy, cx, ty, tx, valid);
        int32_t* ptile = reinterpret_cast<int32_t*>(staging) + acc * Cfg::POOL_ROWS * Cfg::POOL_PITCH;
        const int span = p.pool_span;
        const bool warp_used = quarter * 32 < span * span;   // warp-uniform
#pragma unroll 1
        for (int c = group; warp_used && c < BN / Cfg::CW; c += G) {
          if (n0 + c * Cfg::CW >= p.N) break;
          uint32_t acc_r[16];
          tmem_ld_32x32b_x16(tbase + c * Cfg::CW, acc_r);
          tmem_ld_wait();
          if (r < span * span) {
            // conv pixels outside the conv output are the pool's -inf padding
            uint4* d4 = reinterpret_cast<uint4*>(ptile + r * Cfg::POOL_PITCH + c * Cfg::CW);
#pragma unroll
            for (int q = 0; q < 4; ++q)
              d4[q] = valid ? make_uint4(acc_r[4 * q], acc_r[4 * q + 1], acc_r[4 * q + 2], acc_r[4 * q + 3])
                            : make_uint4(0x80000000u, 0x80000000u, 0x80000000u, 0x80000000u);
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
        mbar_arrive(&pool_bar[acc]);
        if (!mbar_wait(&pool_bar[acc], (it >> 1) & 1, abort_flag, QG_TIMEOUT_NS)) break;
        const int et = threadIdx.x - 32 * Cfg::EPI_WARP0;
        const int T = p.pool_t, S = p.pool_s, P = p.pool_p;
        for (int o = et; o < T * T * BN; o += Cfg::EPI_THREADS) {
          const int ch = o % BN, pp = o / BN;
          const int py = pp / T, px = pp - (pp / T) * T;
          const int gy = ty * T + py, gx = tx * T + px;
          if (gy >= p.ph_out || gx >= p.pw_out) continue;
          const int64_t orow = (static_cast<int64_t>(img) * p.ph_out + gy) * p.pw_out + gx;
          const int col = n0 + ch;
          if (col >= p.N) {
            if (p.out_i8 != nullptr && col < p.ld_i8) p.out_i8[orow * p.ld_i8 + col] = 0;
            continue;
          }
          int32_t mx = INT32_MIN;
          for (int dy = 0; dy < P; ++dy) {
            const int32_t* prow = ptile + ((S * py + dy) * span + S * px) * Cfg::POOL_PITCH + ch;
            for (int dx = 0; dx < P; ++dx) mx = max(mx, prow[dx * Cfg::POOL_PITCH]);
          }
          float y;
          if (!dequant_fast(mx, __ldg(p.scale_hi + col), __ldg(p.scale_lo + col), y))
            y = __double2float_rn(static_cast<double>(mx) * p.scale64[col]);
          for (int s = 0; s < p.n_steps; ++s) {
            const mira_epi_step& st = p.steps[s];
            if (st.operand == MIRA_OPND_NONE) {
              y = apply_unary(st.op, y);
            } else {
              const float opnd = st.operand == MIRA_OPND_SCALAR ? st.scalar : __ldg(st.ptr + col);
              y = st.swapped ? apply_binary(st.op, opnd, y) : apply_binary(st.op, y, opnd);
            }
          }
          if (p.out_f32 != nullptr) p.out_f32[orow * p.ld_f32 + col] = y;
          if (p.out_i8 != nullptr)
            p.out_i8[orow * p.ld_i8 + col] =
                static_cast<int8_t>(round_clip_i8(div_by_scale(y, p.q_scale, p.q_rcp, p.q_lim)) & 0xff);
        }
      }
    }
  } else if (!qg_a_async(AMODE) && warp >= Cfg::GATHER_WARP0) {
    // ------------------------------------------------ im2col gather of A (convolutions)
    const int row = threadIdx.x - 32 * Cfg::GATHER_WARP0;
    const QgConv& g = p.g;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
      int img = 0, oy = 0, ox = 0;
      bool row_ok;
      if (POOL) {
        int ty, tx;
        pool_row_pixel(p, t / p.n_tiles, row, img, oy, ox, ty, tx, row_ok);
        if (!row_ok) img = oy = ox = 0;
      } else {
        const int m = (t / p.n_tiles) * QG_BM + row;
        row_ok = m < p.M;
        if (row_ok) {
          img = m / (g.oh * g.ow);
          const int rem = m - img * g.oh * g.ow;
          oy = rem / g.ow;
          ox = rem - oy * g.ow;
        }
      }
      const int iy0 = oy * g.sh - g.ph;
      const int ix0 = ox * g.sw - g.pw;
      const int8_t* base = p.A + static_cast<int64_t>(img) * g.h * g.w * g.cp;
      // which kernel columns land inside the image for this output pixel (kw <= 32)
      uint32_t colmask = 0;
      for (int j = 0; j < g.kw; ++j)
        colmask |= (static_cast<unsigned>(ix0 + j * g.dw) < static_cast<unsigned>(g.w)) ? (1u << j) : 0u;
      // current tap (ti, tj), channel offset ci within it, and the tap's source pixel
      int ti = 0, tj = 0, ci = 0;
      int iy = iy0;
      bool row_in = row_ok && static_cast<unsigned>(iy) < static_cast<unsigned>(g.h);
      const int64_t tap_step = static_cast<int64_t>(g.dw) * g.cp;
      const int8_t* tap_ptr = base + (static_cast<int64_t>(iy) * g.w + ix0) * g.cp;
      const int swz = row & 7;
      for (int kb = 0; kb < p.num_kb; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, QG_TIMEOUT_NS)) { ok = false; break; }
        const uint32_t dst_row = smem_u32(sA + stage * A_BYTES) + row * QG_BK;
        const int kmax = p.K - kb * QG_BK;   // reduction bytes left from this K-block on
        if (AMODE == QG_A_GATHER16) {
          int c = 0;
          while (c < 8) {   // one tap (or what is left of it) per iteration
            const bool tap_ok = row_in && ((colmask >> tj) & 1u);
            int n_here = (g.cp - ci) >> 4;
            if (n_here > 8 - c) n_here = 8 - c;
            const int8_t* src = tap_ptr + ci;
            for (int e = 0; e < n_here; ++e, ++c, src += 16) {
              const bool v = tap_ok && (c * 16 < kmax);
              cp_async_16(dst_row + ((c ^ swz) << 4), v ? src : p.A, v ? 16u : 0u);
            }
            ci += n_here * 16;
            if (ci == g.cp) {
              ci = 0;
              tap_ptr += tap_step;
              if (++tj == g.kw) {
                tj = 0;
                ++ti;
                iy += g.dh;
                row_in = row_ok && static_cast<unsigned>(iy) < static_cast<unsigned>(g.h);
                tap_ptr = base + (static_cast<int64_t>(iy) * g.w + ix0) * g.cp;
              }
            }
          }
        } else if (AMODE == QG_A_ROW4) {
          // k = i * 32 + j * 4 + c: chunk (i, half) is entry ox + (4 / sw) * half of input row iy0 + i
          // (entries are laid out at the convolution's horizontal stride)
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const int i = kb * 4 + (c >> 1);
            const int iy = iy0 + i;
            const bool v = row_ok && i < g.kh && static_cast<unsigned>(iy) < static_cast<unsigned>(g.h) &&
                           (c * 16 < kmax);
            const int8_t* src = p.A + ((static_cast<int64_t>(img) * g.h + iy) * g.row_entries +
                                       ox + (4 / g.sw) * (c & 1)) * 16;
            cp_async_16(dst_row + ((c ^ swz) << 4), v ? src : p.A, v ? 16u : 0u);
          }
        } else {
#pragma unroll 4
          for (int c = 0; c < 32; ++c) {
            const bool v = row_in && ((colmask >> tj) & 1u) && (c * 4 < kmax);
            cp_async_4(dst_row + (((c >> 2) ^ swz) << 4) + ((c & 3) << 2), v ? tap_ptr : p.A, v ? 4u : 0u);
            tap_ptr += tap_step;
            if (++tj == g.kw) {
              tj = 0;
              ++ti;
              iy += g.dh;
              row_in = row_ok && static_cast<unsigned>(iy) < static_cast<unsigned>(g.h);
              tap_ptr = base + (static_cast<int64_t>(iy) * g.w + ix0) * g.cp;
            }
          }
        }
        // the stage's barrier counts this thread's arrival when its copies have landed
        cp_async_arrive_noinc(&full[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
    // no copy may still be landing when the CTA exits
    cp_async_wait<0>();
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
