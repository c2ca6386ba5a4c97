// Prefill attention on the tensor cores, f32-accurate: o = softmax((q @ k^T) * scale + mask) @ v
// (reference _matmul_ref ops.py:217-219, _softmax_ref 310-313) for a head dimension of 64.
//
// The reference computes in float32.  Every f32 operand x is split into three bf16 pieces,
// x = x0 + x1 + x2 exactly (8 + 8 + 8 significant bits; bf16 has float32's exponent range), and a
// product x * y is the sum of the six piece products x_i * y_j with i + j <= 2, each exact in the
// tensor core's f32 accumulator; the three dropped ones are below 2^-24 of |x * y|.  So q @ k^T
// and p @ v come out of tcgen05.mma.kind::f16 (bf16 operands, f32 accumulation in TMEM) with about
// the accuracy of f32 FMA sums, in another summation order.
//
// A first kernel splits k and v into their pieces once per (batch0, batch1) entry, in the caller's
// workspace (k as [piece][key][d] rows, v transposed as [piece][d][key] rows).  Then one CTA per
// 128 query rows walks the key tiles of 64 keys as a pipeline: one thread loads the k and v piece
// tiles with TMA (128-byte swizzle; k and v in separate two-stage rings, k one tile ahead, since a k
// tile is free as soon as its score MMAs are done), one thread issues the 24 MMAs of a score tile
// S = q k^T into one of two TMEM buffers ahead of the softmax, and sixteen softmax warps (four
// threads per query row, TMEM lane i, each with 16 of the tile's columns; they swap their row
// maxima through shared memory) read their rows, apply the scale step and the mask (loaded a tile
// ahead), update the running maximum and the rescaled partial sums as the f32 kernel does, with
// e^(s - m) evaluated as 2^(s log2(e) - m log2(e)) by the ex2.approx instruction (a few ulp), and
// store the probabilities' pieces into one of two TMEM p buffers, the A operand of the 24 MMAs of
// O_tile = p v (two TMEM buffers), which they add to their f32 output rows one tile later, while
// the next tile's softmax runs.  The output rows are divided by the sums (reciprocal and one
// residual correction) and stored through shared memory as whole rows.  Key tiles whose mask is
// all strongly negative are skipped under the f32 kernel's certificate (|scale| ||q_i||_1 max|k| +
// tile_max - m_i < -110 for every row; the tiles some row cannot skip are processed at the end).
#pragma once
#include <cuda_bf16.h>
#include "qgemm_sm100.cuh"
#include "sequence_ops.cuh"

namespace mira {

constexpr int ATC_BQ = 128, ATC_BK = 64, ATC_DH = 64, ATC_PIECES = 3;
// warps 0 .. 4 ATC_CG - 1 softmax (thread t: query row t % 128 = TMEM lane, columns HC (t / 128) ..
// + HC - 1 with HC = 64 / ATC_CG), then one warp that issues the MMAs and one for the TMA loads
constexpr int ATC_CG = 4;                                   // threads (column groups) per query row
constexpr int ATC_SOFTMAX = ATC_BQ * ATC_CG, ATC_THREADS = ATC_SOFTMAX + 64;
constexpr int ATC_MMA_WARP = ATC_SOFTMAX / 32, ATC_TMA_WARP = ATC_MMA_WARP + 1;
constexpr int ATC_MAX_KB = 256;   // key tiles of a row (tk <= 16384)
// TMEM columns: S tiles at 0 and 64, O tiles at 128 and 192, the two p tiles (three bf16 pieces of
// 32 columns each, two keys per column) at ATC_PCOL and ATC_PCOL + ATC_PCOLS
constexpr uint32_t ATC_PCOL = 256, ATC_PCOLS = ATC_PIECES * ATC_BK / 2;
constexpr uint64_t ATC_TIMEOUT_NS = 2000000000ull;

struct AtcSmem {
  // 128-byte-swizzled K-major tiles (rows of 64 bf16 values), one per bf16 piece
  uint8_t q[ATC_PIECES][ATC_BQ * 128];       // [query][d]
  uint8_t k[2][ATC_PIECES][ATC_BK * 128];    // [key][d], two tiles in flight
  uint8_t vt[2][ATC_PIECES][ATC_DH * 128];   // [d][key]
  // k and v have stages of their own: a k tile is free once its score MMAs are done, a tile ahead
  // of the v tile beside it
  uint64_t k_full[2], k_empty[2], v_full[2], v_empty[2];
  uint64_t s_full[2], s_empty[2], o_full[2], o_empty[2], p_full[2], p_empty[2], drain;
  uint64_t mx_bar[2];          // the two halves of a row have swapped their maxima (per tile, double-buffered)
  float xmax[2][ATC_CG][ATC_BQ];  // [tile parity][column group][row]
  float xl[ATC_CG][ATC_BQ];       // [column group][row]: the groups' sums, combined at the end
  uint32_t tmem;
  int abort;
  float qn1[ATC_BQ];
  float kmax;                  // max |k| (the skipping certificate)
  float tmax[ATC_MAX_KB];      // the largest mask value of each key tile over the block's rows
  int16_t tiles[ATC_MAX_KB];   // the key tiles that are not skipping candidates, in order
  uint8_t cand[ATC_MAX_KB];    // 1: a skipping candidate
  uint8_t fail[ATC_MAX_KB];    // 1: a candidate that some row cannot skip
  uint8_t zmask[2][ATC_MAX_KB];  // [64-row half][key tile] 1: every mask value of the tile is +0
  int n_main;
};

// Byte offset of 16-byte chunk `chunk` of row `row` in a 128-byte-swizzled tile (8-row atoms of
// 1 KB, the chunk index XOR the row within the atom): the layout TMA's 128-byte swizzle writes.
__device__ __forceinline__ int atc_sw128(int row, int chunk) {
  return (row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4);
}

// a and b rounded to bf16 (to nearest, ties to even), a in the low half of the word
__device__ __forceinline__ uint32_t atc_bf2(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// The three pieces of 8 values as three 16-byte words: piece 0 is x rounded to bf16, piece 1 the
// remainder x - x0 (exact in f32) rounded to bf16, piece 2 the remainder after that (exact in
// bf16: at most 8 significant bits are left); two values per conversion.
__device__ __forceinline__ void atc_pack8(const float (&x)[8], uint4 (&w)[ATC_PIECES]) {
  uint32_t t[ATC_PIECES][4];
#pragma unroll
  for (int e = 0; e < 8; e += 2) {
    const uint32_t w0 = atc_bf2(x[e], x[e + 1]);
    const float ra = __fsub_rn(x[e], __uint_as_float(w0 << 16));
    const float rb = __fsub_rn(x[e + 1], __uint_as_float(w0 & 0xffff0000u));
    const uint32_t w1 = atc_bf2(ra, rb);
    const float sa = __fsub_rn(ra, __uint_as_float(w1 << 16));
    const float sb = __fsub_rn(rb, __uint_as_float(w1 & 0xffff0000u));
    t[0][e >> 1] = w0;
    t[1][e >> 1] = w1;
    t[2][e >> 1] = atc_bf2(sa, sb);
  }
#pragma unroll
  for (int pc = 0; pc < ATC_PIECES; ++pc) w[pc] = make_uint4(t[pc][0], t[pc][1], t[pc][2], t[pc][3]);
}

// Splits 8 values and stores their pieces as 16-byte chunk `chunk` of row `row` of three
// consecutive swizzled tiles of `tile_bytes` each.
__device__ __forceinline__ void atc_store8(uint8_t* base, int tile_bytes, int row, int chunk, const float (&x)[8]) {
  uint4 w[ATC_PIECES];
  atc_pack8(x, w);
  const int off = atc_sw128(row, chunk);
#pragma unroll
  for (int pc = 0; pc < ATC_PIECES; ++pc) *reinterpret_cast<uint4*>(base + pc * tile_bytes + off) = w[pc];
}

// 2^x by the ex2.approx instruction (a few ulp; subnormal results kept).  The softmax weights are
// computed as e^(s - m) = 2^(s log2(e) - m log2(e)).
__device__ __forceinline__ float atc_ex2(float x) {
  float y;
  asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr float ATC_LOG2E = 1.4426950408889634f;

// D (TMEM) (+)= A B^T with A (M = 128 rows x K = 16 bf16) in TMEM (row i in lane i, two bf16 per
// 32-bit column, the lower k in the low half) and B in shared memory.
__device__ __forceinline__ void mma_bf16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Four 32-bit columns of this thread's TMEM lane (warp-collective: lanes 32 (warp % 4) .. + 31).
__device__ __forceinline__ void tmem_st_32x32b_x4(uint32_t taddr, const uint4& v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// The 24 MMAs of O = p v over the 64 keys of a tile: p's three pieces in TMEM (ATC_BK / 2 columns
// apart), v's as K-major [d][key] tiles in shared memory.
__device__ __forceinline__ void atc_mma_ts(uint32_t d_tmem, uint32_t p_tmem, const uint8_t* b_tiles, int b_bytes) {
  constexpr uint32_t IDESC = idesc_bf16(ATC_BQ, 64);
  constexpr int PI[6] = {0, 0, 1, 0, 1, 2}, PJ[6] = {0, 1, 0, 2, 1, 0};
  bool first = true;
#pragma unroll
  for (int t = 0; t < 6; ++t) {
    const uint64_t bd = smem_desc_k_sw128(smem_u32(b_tiles + PJ[t] * b_bytes));
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      mma_bf16_tmem_a(d_tmem, p_tmem + PI[t] * (ATC_BK / 2) + 8 * ks, bd + 2 * ks, IDESC, first ? 0u : 1u);
      first = false;
    }
  }
}

// This thread's lane of TMEM columns taddr .. taddr + N - 1 (warp-collective).
__device__ __forceinline__ void atc_tmem_ld(uint32_t taddr, uint32_t (&r)[32]) { tmem_ld_32x32b_x32(taddr, r); }
__device__ __forceinline__ void atc_tmem_ld(uint32_t taddr, uint32_t (&r)[16]) { tmem_ld_32x32b_x16(taddr, r); }

// The key tiles kb < nkb with flag[kb] == want, in order, into out[]; their number into *n.  Run by
// one whole warp.
__device__ __forceinline__ void atc_list(const uint8_t* flag, uint8_t want, int nkb, int16_t* out, int* n) {
  const int lane = threadIdx.x & 31;
  int count = 0;
  for (int base = 0; base < nkb; base += 32) {
    const int kb = base + lane;
    const bool f = kb < nkb && flag[kb] == want;
    const uint32_t bal = __ballot_sync(0xffffffffu, f);
    if (f) out[count + __popc(bal & ((1u << lane) - 1u))] = static_cast<int16_t>(kb);
    count += __popc(bal);
  }
  if (lane == 0) *n = count;
}

// The 24 MMAs of D = A B^T over K = 64: six piece pairs (i + j <= 2) x four K-steps of 16.
__device__ __forceinline__ void atc_mma(uint32_t d_tmem, const uint8_t* a_tiles, int a_bytes, const uint8_t* b_tiles,
                                        int b_bytes) {
  constexpr uint32_t IDESC = idesc_bf16(ATC_BQ, 64);
  constexpr int PI[6] = {0, 0, 1, 0, 1, 2}, PJ[6] = {0, 1, 0, 2, 1, 0};
  bool first = true;
#pragma unroll
  for (int t = 0; t < 6; ++t) {
    const uint64_t ad = smem_desc_k_sw128(smem_u32(a_tiles + PI[t] * a_bytes));
    const uint64_t bd = smem_desc_k_sw128(smem_u32(b_tiles + PJ[t] * b_bytes));
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      mma_bf16(d_tmem, ad + 2 * ks, bd + 2 * ks, IDESC, first ? 0u : 1u);
      first = false;
    }
  }
}

// k and v of one key tile of one (batch0, batch1) entry into pieces: kpc[((bh * 3 + piece) * tkp +
// key) * 64 + d] and vtc[((bh * 3 + piece) * 64 + d) * tkp + key] (bf16), keys past tk 0.  Every
// thread issues all its loads before the first conversion; v goes through shared memory so that the
// transposed rows leave as whole 128-byte segments.
constexpr int ATC_PIECE_THREADS = 256;
__global__ void __launch_bounds__(ATC_PIECE_THREADS) attention_pieces_kernel(const AttnParams p, int tkp,
                                                                             uint16_t* __restrict__ kpc,
                                                                             uint16_t* __restrict__ vtc) {
  __shared__ float vs[ATC_BK][ATC_DH + 1];   // [key][d], padded against bank conflicts
  const int k0 = blockIdx.x * ATC_BK, tid = threadIdx.x;
  const int64_t b1 = blockIdx.y, b0 = blockIdx.z, bh = b0 * gridDim.y + b1;
  const float* kp = p.k + b0 * p.ks[0] + b1 * p.ks[1];
  const float* vp = p.v + b0 * p.vs[0] + b1 * p.vs[1];
  constexpr int KT = ATC_BK * 8 / ATC_PIECE_THREADS;    // k tasks per thread: (key, 8 values of d)
  constexpr int VT = ATC_BK * 16 / ATC_PIECE_THREADS;   // v loads per thread: (key, 4 values of d)
  float xk[KT][8];
  float4 xv[VT];
#pragma unroll
  for (int t = 0; t < KT; ++t) {
    const int task = tid + t * ATC_PIECE_THREADS, j = task >> 3, ch = task & 7;
    const bool live = k0 + j < p.tk;
    const float* src = kp + int64_t(k0 + j) * p.ks[2];
    if (live && p.vec) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(src + 8 * ch));
      const float4 c = __ldg(reinterpret_cast<const float4*>(src + 8 * ch + 4));
      xk[t][0] = a.x; xk[t][1] = a.y; xk[t][2] = a.z; xk[t][3] = a.w;
      xk[t][4] = c.x; xk[t][5] = c.y; xk[t][6] = c.z; xk[t][7] = c.w;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) xk[t][e] = live ? __ldg(src + int64_t(8 * ch + e) * p.ks[3]) : 0.0f;
    }
  }
#pragma unroll
  for (int t = 0; t < VT; ++t) {
    const int task = tid + t * ATC_PIECE_THREADS, j = task >> 4, c4 = task & 15;
    const bool live = k0 + j < p.tk;
    const float* src = vp + int64_t(k0 + j) * p.vs[2];
    if (live && p.vec) {
      xv[t] = __ldg(reinterpret_cast<const float4*>(src + 4 * c4));
    } else {
      xv[t].x = live ? __ldg(src + int64_t(4 * c4) * p.vs[3]) : 0.0f;
      xv[t].y = live ? __ldg(src + int64_t(4 * c4 + 1) * p.vs[3]) : 0.0f;
      xv[t].z = live ? __ldg(src + int64_t(4 * c4 + 2) * p.vs[3]) : 0.0f;
      xv[t].w = live ? __ldg(src + int64_t(4 * c4 + 3) * p.vs[3]) : 0.0f;
    }
  }
#pragma unroll
  for (int t = 0; t < VT; ++t) {
    const int task = tid + t * ATC_PIECE_THREADS, j = task >> 4, c4 = task & 15;
    vs[j][4 * c4] = xv[t].x;
    vs[j][4 * c4 + 1] = xv[t].y;
    vs[j][4 * c4 + 2] = xv[t].z;
    vs[j][4 * c4 + 3] = xv[t].w;
  }
#pragma unroll
  for (int t = 0; t < KT; ++t) {
    const int task = tid + t * ATC_PIECE_THREADS, j = task >> 3, ch = task & 7;
    uint4 w[ATC_PIECES];
    atc_pack8(xk[t], w);
#pragma unroll
    for (int pc = 0; pc < ATC_PIECES; ++pc)
      *reinterpret_cast<uint4*>(kpc + ((bh * ATC_PIECES + pc) * tkp + k0 + j) * ATC_DH + 8 * ch) = w[pc];
  }
  __syncthreads();
#pragma unroll
  for (int t = 0; t < KT; ++t) {
    const int task = tid + t * ATC_PIECE_THREADS, n = task >> 3, kc = task & 7;   // v: d n, keys 8 kc .. + 7
    float x[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = vs[8 * kc + e][n];
    uint4 w[ATC_PIECES];
    atc_pack8(x, w);
#pragma unroll
    for (int pc = 0; pc < ATC_PIECES; ++pc)
      *reinterpret_cast<uint4*>(vtc + ((bh * ATC_PIECES + pc) * ATC_DH + n) * int64_t(tkp) + k0 + 8 * kc) = w[pc];
  }
}

__global__ void __launch_bounds__(ATC_THREADS, 1) attention_tc_kernel(const __grid_constant__ CUtensorMap map_k,
                                                                      const __grid_constant__ CUtensorMap map_vt,
                                                                      const AttnParams p, int tkp) {
  extern __shared__ uint8_t atc_raw[];
  AtcSmem& sm = *reinterpret_cast<AtcSmem*>((reinterpret_cast<uintptr_t>(atc_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5;
  const int nqb = (p.tq + ATC_BQ - 1) / ATC_BQ, nkb = (p.tk + ATC_BK - 1) / ATC_BK;
  const int qb = nqb - 1 - static_cast<int>(blockIdx.x);     // the longest rows first
  const int q0 = qb * ATC_BQ;
  const int64_t b1 = blockIdx.y, b0 = blockIdx.z;
  const int64_t bh = b0 * gridDim.y + b1;
  const float* qp = p.q + b0 * p.qs[0] + b1 * p.qs[1];
  const float* mp = p.mask != nullptr ? p.mask + b0 * p.ms[0] + b1 * p.ms[1] : nullptr;
  volatile int* abort_flag = &sm.abort;

  if (tid == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.k_full[b], 1);
      mbar_init(&sm.k_empty[b], 1);
      mbar_init(&sm.v_full[b], 1);
      mbar_init(&sm.v_empty[b], 1);
      mbar_init(&sm.s_full[b], 1);
      mbar_init(&sm.s_empty[b], ATC_SOFTMAX);
      mbar_init(&sm.o_full[b], 1);
      mbar_init(&sm.o_empty[b], ATC_SOFTMAX);
    }
    mbar_init(&sm.p_full[0], ATC_SOFTMAX);
    mbar_init(&sm.p_full[1], ATC_SOFTMAX);
    mbar_init(&sm.mx_bar[0], ATC_SOFTMAX);
    mbar_init(&sm.mx_bar[1], ATC_SOFTMAX);
    mbar_init(&sm.p_empty[0], 1);
    mbar_init(&sm.p_empty[1], 1);
    mbar_init(&sm.drain, 1);
    sm.abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&map_k);
    tma_prefetch_desc(&map_vt);
  }
  if (warp == 0) {
    tmem_alloc(&sm.tmem, 512);   // S buffers in columns 0..127, O_tile 128..255, p 256..447
    tmem_relinquish();
  }
  // q rows (zero past tq) as pieces, all loads of a thread in flight at once; ||q_i||_1 for the
  // skipping certificate (the 8 chunks of a row are 8 consecutive lanes)
  {
    constexpr int QT = (ATC_BQ * 8 + ATC_THREADS - 1) / ATC_THREADS;
    const bool qvec = p.qs[3] == 1 && ((p.qs[0] | p.qs[1] | p.qs[2]) & 3) == 0 &&
                      (reinterpret_cast<uintptr_t>(qp) & 15) == 0;
    float x[QT][8];
#pragma unroll
    for (int j = 0; j < QT; ++j) {
      const int task = tid + j * ATC_THREADS, row = task >> 3, ch = task & 7;
      const bool live = task < ATC_BQ * 8 && q0 + row < p.tq;
      const float* src = qp + int64_t(q0 + row) * p.qs[2];
      if (live && qvec) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(src + 8 * ch));
        const float4 c = __ldg(reinterpret_cast<const float4*>(src + 8 * ch + 4));
        x[j][0] = a.x; x[j][1] = a.y; x[j][2] = a.z; x[j][3] = a.w;
        x[j][4] = c.x; x[j][5] = c.y; x[j][6] = c.z; x[j][7] = c.w;
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) x[j][e] = live ? __ldg(src + int64_t(8 * ch + e) * p.qs[3]) : 0.0f;
      }
    }
#pragma unroll
    for (int j = 0; j < QT; ++j) {
      const int task = tid + j * ATC_THREADS, row = task >> 3, ch = task & 7;
      float a = 0.0f;
#pragma unroll
      for (int e = 0; e < 8; ++e) a += fabsf(x[j][e]);
      a += __shfl_xor_sync(0xffffffffu, a, 1);
      a += __shfl_xor_sync(0xffffffffu, a, 2);
      a += __shfl_xor_sync(0xffffffffu, a, 4);
      if (task < ATC_BQ * 8) {
        atc_store8(&sm.q[0][0], sizeof(sm.q[0]), row, ch, x[j]);
        if (ch == 0) sm.qn1[row] = a;
      }
    }
  }
  // skipping candidates and all-zero mask tiles once, into shared memory: tile_max / tile_zero
  // describe 64 x 64 (query, key) tiles, this block holds two 64-row halves
  const bool can_skip = p.tile_max != nullptr && p.kmax != nullptr;
  const int nqb64 = (p.tq + 63) / 64;
  if (tid == 0 && can_skip) sm.kmax = __uint_as_float(__ldg(p.kmax));
  for (int kb = tid; kb < nkb; kb += ATC_THREADS) {
    float t = -INFINITY;
    if (can_skip) {
      t = __ldg(p.tile_max + int64_t(2 * qb) * nkb + kb);
      if (2 * qb + 1 < nqb64) t = fmaxf(t, __ldg(p.tile_max + int64_t(2 * qb + 1) * nkb + kb));
    }
    sm.tmax[kb] = t;
    sm.cand[kb] = can_skip && t <= -200.0f ? 1 : 0;
    sm.fail[kb] = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h)
      sm.zmask[h][kb] = p.tile_zero != nullptr && 2 * qb + h < nqb64 &&
                        __ldg(p.tile_zero + int64_t(2 * qb + h) * nkb + kb) != 0;
  }
  fence_proxy_async_smem();   // generic-proxy writes of q read by tcgen05.mma
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) atc_list(sm.cand, 0, nkb, sm.tiles, &sm.n_main);
  __syncthreads();
  const uint32_t tmem = sm.tmem;

  // softmax state of query row r = q0 + (tid & 127), columns HC * cg .. + HC - 1
  const int srow = tid & (ATC_BQ - 1), cg = (tid >> 7) % ATC_CG;
  const int r = q0 + srow;
  constexpr int HC = ATC_BK / ATC_CG;   // columns per thread (of the scores and of the output)
  static_assert(HC == 16 || HC == 32, "column group width");
  float m = -INFINITY, ml = -INFINITY, l = 0.0f;   // ml = m log2(e), rounded once
  float o[HC];
#pragma unroll
  for (int d = 0; d < HC; ++d) o[d] = 0.0f;
  uint32_t seq = 0;   // tiles through the pipeline so far (mbarrier phases); the same in every role

  // Runs key tiles list(0) .. list(count - 1) through the pipeline (every role calls it with the
  // same list).
  auto run = [&](int count, auto list) {
    if (warp == ATC_TMA_WARP) {
      // ------------------------------------------------ producer: the k and v piece tiles by TMA,
      // k one tile ahead of v (k(i + 1) is needed by the score MMAs before v(i) by the p v MMAs)
      if ((tid & 31) == 0) {
        int nk = 0, nv = 0;   // tiles issued
        auto load_k = [&](int i) {
          const uint32_t sq = seq + i, b = sq & 1;
          if (!mbar_wait(&sm.k_empty[b], ((sq >> 1) & 1) ^ 1, abort_flag, ATC_TIMEOUT_NS)) return false;
          ++nk;
          const int k0 = list(i) * ATC_BK;
          mbar_arrive_expect_tx(&sm.k_full[b], ATC_PIECES * ATC_BK * 128);
#pragma unroll
          for (int pc = 0; pc < ATC_PIECES; ++pc)
            tma_load_2d(&sm.k[b][pc][0], &map_k, 0, static_cast<int32_t>((bh * ATC_PIECES + pc) * tkp + k0),
                        &sm.k_full[b]);
          return true;
        };
        auto load_v = [&](int i) {
          const uint32_t sq = seq + i, b = sq & 1;
          if (!mbar_wait(&sm.v_empty[b], ((sq >> 1) & 1) ^ 1, abort_flag, ATC_TIMEOUT_NS)) return false;
          ++nv;
          const int k0 = list(i) * ATC_BK;
          mbar_arrive_expect_tx(&sm.v_full[b], ATC_PIECES * ATC_DH * 128);
#pragma unroll
          for (int pc = 0; pc < ATC_PIECES; ++pc)
            tma_load_2d(&sm.vt[b][pc][0], &map_vt, k0, static_cast<int32_t>((bh * ATC_PIECES + pc) * ATC_DH),
                        &sm.v_full[b]);
          return true;
        };
        bool ok = count > 0 ? load_k(0) : true;
        for (int i = 0; i < count && ok; ++i) {
          if (i + 1 < count && !load_k(i + 1)) break;
          if (!load_v(i)) break;
        }
        if (*abort_flag) {
          // let the copies still in flight land before the shared memory goes away (bounded)
          auto settle = [&](uint64_t* full, int n) {
            for (int i = n > 2 ? n - 2 : 0; i < n; ++i) {
              const uint32_t sq = seq + i;
              const uint64_t t0 = globaltimer_ns();
              while (!mbar_try_wait_suspend(&full[sq & 1], (sq >> 1) & 1, 1000000u) &&
                     globaltimer_ns() - t0 < ATC_TIMEOUT_NS) {
              }
            }
          };
          settle(sm.k_full, nk);
          settle(sm.v_full, nv);
        }
      }
    } else if (warp == ATC_MMA_WARP) {
      // ------------------------------------------------ MMA issuer: S one tile ahead of p v
      if ((tid & 31) == 0) {
        auto issue_s = [&](uint32_t sq) {
          const uint32_t b = sq & 1;
          if (!mbar_wait(&sm.k_full[b], (sq >> 1) & 1, abort_flag, ATC_TIMEOUT_NS)) return false;
          if (!mbar_wait(&sm.s_empty[b], ((sq >> 1) & 1) ^ 1, abort_flag, ATC_TIMEOUT_NS)) return false;
          tc_fence_after();
          atc_mma(tmem + 64 * b, &sm.q[0][0], sizeof(sm.q[0]), &sm.k[b][0][0], sizeof(sm.k[0][0]));
          mma_commit(&sm.s_full[b]);
          mma_commit(&sm.k_empty[b]);
          return true;
        };
        bool ok = count > 0 ? issue_s(seq) : true;
        for (int i = 0; i < count && ok; ++i) {
          const uint32_t sq = seq + i, b = sq & 1;
          if (i + 1 < count && !issue_s(sq + 1)) break;
          if (!mbar_wait(&sm.v_full[b], (sq >> 1) & 1, abort_flag, ATC_TIMEOUT_NS)) break;
          if (!mbar_wait(&sm.p_full[b], (sq >> 1) & 1, abort_flag, ATC_TIMEOUT_NS)) break;
          if (!mbar_wait(&sm.o_empty[b], ((sq >> 1) & 1) ^ 1, abort_flag, ATC_TIMEOUT_NS)) break;
          tc_fence_after();
          atc_mma_ts(tmem + 128 + 64 * b, tmem + ATC_PCOL + ATC_PCOLS * b, &sm.vt[b][0][0], sizeof(sm.vt[0][0]));
          mma_commit(&sm.o_full[b]);
          mma_commit(&sm.p_empty[b]);
          mma_commit(&sm.v_empty[b]);
        }
      }
    } else {
      // ------------------------------------------------ softmax rows
      const uint32_t lane_base = static_cast<uint32_t>(warp & 3) * 32u << 16;
      const int half = srow >> 6;   // which 64-row half of the block this row is in
      auto add_o = [&](uint32_t sq) {   // the p v tile of sq into the output row
        const uint32_t b = sq & 1;
        if (!mbar_wait(&sm.o_full[b], (sq >> 1) & 1, abort_flag, ATC_TIMEOUT_NS)) return;
        tc_fence_after();
        uint32_t raw[HC];
        atc_tmem_ld(tmem + lane_base + 128 + 64 * b + HC * cg, raw);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < HC; ++c) o[c] += __uint_as_float(raw[c]);
        tc_fence_before();
        mbar_arrive(&sm.o_empty[b]);
      };
      // the mask values of tile list(i) in this thread's columns, loaded one tile ahead (a tile of
      // +0 adds nothing: x + 0 turns -0 into +0, which leaves exp(x - m) alone)
      float mk[HC];
      bool mk_on = false;
      auto fetch_mask = [&](int i) {
        mk_on = false;
        if (mp == nullptr || i >= count || r >= p.tq) return;
        const int kb = list(i), k0 = kb * ATC_BK + HC * cg;
        if (sm.zmask[half][kb]) return;
        mk_on = true;
        const float* mrow = mp + int64_t(r) * p.ms[2];
        if (p.ms[3] == 1 && (reinterpret_cast<uintptr_t>(mrow + k0) & 15) == 0 && k0 + HC <= p.tk) {
#pragma unroll
          for (int c = 0; c < HC; c += 4) {
            const float4 t = __ldg(reinterpret_cast<const float4*>(mrow + k0 + c));
            mk[c] = t.x; mk[c + 1] = t.y; mk[c + 2] = t.z; mk[c + 3] = t.w;
          }
        } else {
#pragma unroll
          for (int c = 0; c < HC; ++c) mk[c] = k0 + c < p.tk ? __ldg(mrow + int64_t(k0 + c) * p.ms[3]) : 0.0f;
        }
      };
      fetch_mask(0);
      for (int i = 0; i < count; ++i) {
        const uint32_t sq = seq + i, b = sq & 1;
        const int kb = list(i), k0 = kb * ATC_BK + HC * cg;   // this thread's first column
        float s[HC];
        if (!mbar_wait(&sm.s_full[b], (sq >> 1) & 1, abort_flag, ATC_TIMEOUT_NS)) break;
        tc_fence_after();
        {
          uint32_t raw[HC];
          atc_tmem_ld(tmem + lane_base + 64 * b + HC * cg, raw);
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < HC; ++c) s[c] = __uint_as_float(raw[c]);
        }
        tc_fence_before();
        mbar_arrive(&sm.s_empty[b]);
        if (p.scale_op == MIRA_EPI_MUL) {
#pragma unroll
          for (int c = 0; c < HC; ++c) s[c] = __fmul_rn(s[c], p.scale);
        } else if (p.scale_op == MIRA_EPI_DIV) {
#pragma unroll
          for (int c = 0; c < HC; ++c) s[c] = __fdiv_rn(s[c], p.scale);
        }
        if (mk_on) {
#pragma unroll
          for (int c = 0; c < HC; ++c) s[c] = __fadd_rn(s[c], mk[c]);
        }
        if (kb * ATC_BK + ATC_BK > p.tk) {   // the ragged last tile: keys past tk do not exist
#pragma unroll
          for (int c = 0; c < HC; ++c)
            if (k0 + c >= p.tk) s[c] = -INFINITY;
        }
        float rmax = -INFINITY;
#pragma unroll
        for (int c = 0; c < HC; ++c) rmax = fmaxf(rmax, s[c]);
        // the row's maximum over the column groups
        sm.xmax[b][cg][srow] = rmax;
        mbar_arrive(&sm.mx_bar[b]);
        if (!mbar_wait_spin(&sm.mx_bar[b], (sq >> 1) & 1, abort_flag, ATC_TIMEOUT_NS)) break;
#pragma unroll
        for (int g = 0; g < ATC_CG; ++g) rmax = fmaxf(rmax, sm.xmax[b][g][srow]);
        const float mnew = fmaxf(m, rmax);
        const bool dead = mnew == -INFINITY;   // no key of the row so far can carry weight
        const float mlnew = __fmul_rn(mnew, ATC_LOG2E);
        const float corr = dead ? 1.0f : atc_ex2(__fsub_rn(ml, mlnew));
        m = mnew;
        ml = mlnew;
        // e^(s - m) piece by piece into this tile's p buffer in TMEM once the p v two tiles back has
        // read it: the thread's 32 keys are 16 columns of each piece (two bf16 per column)
        if (!mbar_wait(&sm.p_empty[b], ((sq >> 1) & 1) ^ 1, abort_flag, ATC_TIMEOUT_NS)) break;
        tc_fence_after();
        float rsum = 0.0f;
        const uint32_t pcol = tmem + lane_base + ATC_PCOL + ATC_PCOLS * b + (HC / 2) * cg;
#pragma unroll
        for (int ch = 0; ch < HC / 8; ++ch) {
          float x[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            x[e] = dead ? 0.0f : atc_ex2(fmaf(s[8 * ch + e], ATC_LOG2E, -mlnew));
            rsum += x[e];
          }
          uint4 w[ATC_PIECES];
          atc_pack8(x, w);
#pragma unroll
          for (int pc = 0; pc < ATC_PIECES; ++pc) tmem_st_32x32b_x4(pcol + pc * (ATC_BK / 2) + 4 * ch, w[pc]);
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&sm.p_full[b]);
        l = fmaf(l, corr, rsum);
        fetch_mask(i + 1);
        // the previous tile's p v (at the previous maximum), then this tile's rescale
        if (i > 0) add_o(sq - 1);
#pragma unroll
        for (int d = 0; d < HC; ++d) o[d] *= corr;
      }
      if (count > 0 && !*abort_flag) add_o(seq + count - 1);
    }
    seq += count;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  };

  run(sm.n_main, [&](int i) { return static_cast<int>(sm.tiles[i]); });
  if (can_skip && !*abort_flag) {
    // every candidate checked once against the row maxima of the main pass; the candidates that some
    // row cannot skip are processed (exactly), the rest skipped (the maxima only grow, so a tile
    // skippable now stays skippable)
    if (tid < ATC_SOFTMAX) {
      const float kmax = sm.kmax;
      for (int kb = 0; kb < nkb; ++kb) {
        if (!sm.cand[kb]) continue;
        bool ok = true;
        if (r < p.tq) {
          // every score of this tile is at most this bound (the factor covers the products' rounding)
          const float bound = p.scale_abs * sm.qn1[srow] * kmax * 1.001f + sm.tmax[kb];
          ok = bound - m < -110.0f;
        }
        if (!__all_sync(0xffffffffu, ok) && (tid & 31) == 0) sm.fail[kb] = 1;
      }
    }
    __syncthreads();
    if (warp == 0) atc_list(sm.fail, 1, nkb, sm.tiles, &sm.n_main);
    __syncthreads();
    if (sm.n_main > 0) run(sm.n_main, [&](int i) { return static_cast<int>(sm.tiles[i]); });
  }
  // the row's sum: the two halves' partial sums (both rescaled by the same maxima)
  if (tid < ATC_SOFTMAX) sm.xl[cg][srow] = l;
  __syncthreads();
  const bool live = !*abort_flag;
  float* obase = p.out != nullptr ? p.out + b0 * p.os[0] + b1 * p.os[1] : nullptr;
  // f32 output rows staged in shared memory and stored coalesced
  constexpr int OST = ATC_DH + 4;   // staged row stride in floats
  // (the k tiles' space: every score MMA has completed once the last p v tile has been added)
  static_assert(sizeof(AtcSmem::k) >= ATC_BQ * OST * sizeof(float), "staging space");
  float* stage = reinterpret_cast<float*>(&sm.k[0][0][0]);
  const bool ostage = obase != nullptr && p.os[3] == 1 && ((p.os[0] | p.os[1] | p.os[2]) & 3) == 0 &&
                      (reinterpret_cast<uintptr_t>(obase) & 15) == 0;
  if (tid < ATC_SOFTMAX && live) {
    if (r < p.tq) {
      // o / l: the product with the rounded reciprocal and one residual correction (Markstein)
      float lsum = sm.xl[0][srow];
#pragma unroll
      for (int g = 1; g < ATC_CG; ++g) lsum = __fadd_rn(lsum, sm.xl[g][srow]);
      const float rl = __frcp_rn(lsum);
#pragma unroll
      for (int c = 0; c < HC; ++c) {
        const float y = __fmul_rn(o[c], rl);
        o[c] = fmaf(fmaf(-lsum, y, o[c]), rl, y);
      }
    }
    if (ostage) {
#pragma unroll
      for (int c = 0; c < HC; c += 4)
        *reinterpret_cast<float4*>(stage + srow * OST + HC * cg + c) = make_float4(o[c], o[c + 1], o[c + 2], o[c + 3]);
    }
    if (r < p.tq) {
      int8_t* qrow = p.out_i8 != nullptr ? p.out_i8 + b0 * p.is[0] + b1 * p.is[1] + int64_t(r) * p.is[2] : nullptr;
      // the int8 row's HC bytes as whole 4-byte words where they are contiguous and aligned
      const bool qvec = qrow != nullptr && p.is[3] == 1 && (reinterpret_cast<uintptr_t>(qrow + HC * cg) & 3) == 0;
      if (qvec) {
#pragma unroll
        for (int c = 0; c < HC; c += 4) {
          uint32_t w = 0;
#pragma unroll
          for (int e = 0; e < 4; ++e) w |= (static_cast<uint32_t>(quant_byte(o[c + e], p.q8)) & 0xffu) << (8 * e);
          *reinterpret_cast<uint32_t*>(qrow + HC * cg + c) = w;
        }
      }
#pragma unroll
      for (int c = 0; c < HC; ++c) {
        const int d = HC * cg + c;
        if (obase != nullptr && !ostage) obase[int64_t(r) * p.os[2] + int64_t(d) * p.os[3]] = o[c];
        if (qrow != nullptr && !qvec) qrow[int64_t(d) * p.is[3]] = static_cast<int8_t>(quant_byte(o[c], p.q8) & 0xff);
      }
    }
  }
  if (ostage) {
    __syncthreads();
    if (tid < ATC_SOFTMAX && live) {
#pragma unroll
      for (int j = 0; j < ATC_BQ * (ATC_DH / 4) / ATC_SOFTMAX; ++j) {
        const int idx = tid + j * ATC_SOFTMAX, row = idx >> 4, c4 = idx & 15;
        if (q0 + row < p.tq)
          *reinterpret_cast<float4*>(obase + int64_t(q0 + row) * p.os[2] + 4 * c4) =
              *reinterpret_cast<const float4*>(stage + row * OST + 4 * c4);
      }
    }
  }
  if (tid == ATC_SOFTMAX) {
    // every MMA this thread issued has finished once `drain` completes (bounded wait)
    mma_commit(&sm.drain);
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(&sm.drain, 0) && globaltimer_ns() - t0 < ATC_TIMEOUT_NS) {
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (tid == 0 && *abort_flag) atomicExch(p.err, 2);
}

}  // namespace mira
