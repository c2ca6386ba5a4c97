// The f32 kernels between the quantized matmuls of a decoder-only transformer: embedding rows,
// layer normalization (fused with the int8 requantization of its consumers), softmax, a strided
// batched f32 matmul with the epilogue steps of the reference, and strided view copies.
//
// Row reductions reproduce NumPy's float32 pairwise summation (the order np.sum / np.mean use on
// a contiguous axis) with one warp per row: the row is cut into the same leaves as NumPy's
// recursion, each leaf's eight interleaved partial sums run on eight lanes, the leaf total is
// combined by shuffles in NumPy's ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) order, and lane 0 adds
// the leaves up along the recursion.
#pragma once
#include <cstdint>

#include "exact_math.cuh"
#include "memory_bound.cuh"
#include "ptx_sm100.cuh"

namespace mira {

constexpr int PW_MAX_LEAVES = 128;

// Leaves of NumPy's pairwise recursion for rows of n elements and the additions that combine
// them, in post order (computed on the host).  Value ids: leaves 0 .. count-1, the result of
// addition t is PW_MAX_LEAVES + t.
struct PwLeaves {
  int n;
  int count;
  int nodes;
  int start[PW_MAX_LEAVES + 1];
  uint8_t left[PW_MAX_LEAVES], right[PW_MAX_LEAVES];
};

// Combines the leaf sums in buf[0 .. count) along the recursion (one lane; buf has
// 2 * PW_MAX_LEAVES floats).
__device__ __forceinline__ float pw_tree(const PwLeaves& pw, float* buf) {
  for (int t = 0; t < pw.nodes; ++t) buf[PW_MAX_LEAVES + t] = __fadd_rn(buf[pw.left[t]], buf[pw.right[t]]);
  return pw.nodes ? buf[PW_MAX_LEAVES + pw.nodes - 1] : buf[0];
}

// Sum of elem(0) .. elem(n-1) in NumPy's float32 pairwise order; every lane returns the total.
// leaf_sum: 2 * PW_MAX_LEAVES floats of shared memory owned by this warp.
template <class F>
__device__ __forceinline__ float warp_pairwise_sum(const PwLeaves& pw, F elem, float* leaf_sum) {
  const int lane = threadIdx.x & 31;
  if (pw.n < 8) {
    float r = 0.0f;
    if (lane == 0)
      for (int i = 0; i < pw.n; ++i) r = __fadd_rn(r, elem(i));
    return __shfl_sync(0xffffffffu, r, 0);
  }
  for (int base = 0; base < pw.count; base += 4) {
    const int leaf = base + (lane >> 3), j = lane & 7;
    const bool live = leaf < pw.count;
    int s = 0, m8 = 0, m = 0;
    float r = 0.0f;
    if (live) {
      s = pw.start[leaf];
      m = pw.start[leaf + 1] - s;
      m8 = m - m % 8;
      r = elem(s + j);
      for (int i = 8 + j; i < m8; i += 8) r = __fadd_rn(r, elem(s + i));
    }
    r = __fadd_rn(r, __shfl_xor_sync(0xffffffffu, r, 1));
    r = __fadd_rn(r, __shfl_xor_sync(0xffffffffu, r, 2));
    r = __fadd_rn(r, __shfl_xor_sync(0xffffffffu, r, 4));
    if (live && j == 0) {
      for (int i = m8; i < m; ++i) r = __fadd_rn(r, elem(s + i));
      leaf_sum[leaf] = r;
    }
  }
  __syncwarp();
  float total = 0.0f;
  if (lane == 0) total = pw_tree(pw, leaf_sum);
  total = __shfl_sync(0xffffffffu, total, 0);
  __syncwarp();
  return total;
}

// ---------------------------------------------------------------- layer normalization

struct LnParams {
  const float* x;
  int64_t rows, ld_x;
  int d;
  const float* gamma;
  const float* beta;
  float eps;
  float* out;
  int64_t ld_out;
  int8_t* out_i8;
  int64_t ld_i8;
  QuantScale q;
  PwLeaves pw;
};

constexpr int ROW_WARPS = 8;

// mu = mean(x), var = mean((x - mu)^2), y = (x - mu) / sqrt(var + eps) * gamma + beta, each step
// one float32 rounding like the reference's NumPy expression.
__global__ void __launch_bounds__(ROW_WARPS * 32) layernorm_rows_kernel(const LnParams p) {
  __shared__ float leaf_sum[ROW_WARPS][2 * PW_MAX_LEAVES];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float dn = static_cast<float>(p.d);
  for (int64_t row = blockIdx.x * int64_t(ROW_WARPS) + warp; row < p.rows; row += int64_t(gridDim.x) * ROW_WARPS) {
    const float* __restrict__ xr = p.x + row * p.ld_x;
    const float mu = __fdiv_rn(warp_pairwise_sum(p.pw, [&](int i) { return __ldg(xr + i); }, leaf_sum[warp]), dn);
    const float var = __fdiv_rn(warp_pairwise_sum(p.pw, [&](int i) {
                                  const float t = __fsub_rn(__ldg(xr + i), mu);
                                  return __fmul_rn(t, t);
                                }, leaf_sum[warp]), dn);
    const float sd = __fsqrt_rn(__fadd_rn(var, p.eps));
    for (int i = lane; i < p.d; i += 32) {
      const float y = __fadd_rn(__fmul_rn(__fdiv_rn(__fsub_rn(__ldg(xr + i), mu), sd), __ldg(p.gamma + i)),
                                __ldg(p.beta + i));
      if (p.out != nullptr) p.out[row * p.ld_out + i] = y;
      if (p.out_i8 != nullptr) p.out_i8[row * p.ld_i8 + i] = static_cast<int8_t>(quant_byte(y, p.q) & 0xff);
    }
  }
}

// Rows of at most 512 * ROUNDS elements with the row held in registers: lane (leaf 4r + lane/8,
// chain lane % 8) keeps elements start + chain + 8i of its leaf, so every pairwise chain is
// lane-local, all loads of a row are issued at once, and the three passes (sum, squared
// deviations, output) read the row from DRAM once.
template <int ROUNDS>
__global__ void __launch_bounds__(ROW_WARPS * 32, ROUNDS == 1 ? 3 : (ROUNDS == 2 ? 2 : 1)) layernorm_rows_reg_kernel(const LnParams p) {
  __shared__ float leaf_sum[ROW_WARPS][2 * PW_MAX_LEAVES];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, j = lane & 7;
  const float dn = static_cast<float>(p.d);
  int start[ROUNDS], m8[ROUNDS], m[ROUNDS];
#pragma unroll
  for (int r = 0; r < ROUNDS; ++r) {
    const int leaf = 4 * r + (lane >> 3);
    const bool live = leaf < p.pw.count;
    start[r] = live ? p.pw.start[leaf] : 0;
    m[r] = live ? p.pw.start[leaf + 1] - start[r] : 0;
    m8[r] = m[r] - m[r] % 8;
  }
  for (int64_t row = blockIdx.x * int64_t(ROW_WARPS) + warp; row < p.rows; row += int64_t(gridDim.x) * ROW_WARPS) {
    const float* __restrict__ xr = p.x + row * p.ld_x;
    float v[ROUNDS][16];
#pragma unroll
    for (int r = 0; r < ROUNDS; ++r)
#pragma unroll
      for (int i = 0; i < 16; ++i) v[r][i] = (j + 8 * i < m8[r]) ? __ldg(xr + start[r] + j + 8 * i) : 0.0f;
    float mu = 0.0f;
    // pass 0: sum of x; pass 1: sum of (x - mu)^2
#pragma unroll
    for (int pass = 0; pass < 2; ++pass) {
#pragma unroll
      for (int r = 0; r < ROUNDS; ++r) {
        float acc = 0.0f;
        if (m8[r] > 0) {
          const float t0 = pass ? __fsub_rn(v[r][0], mu) : v[r][0];
          acc = pass ? __fmul_rn(t0, t0) : t0;
#pragma unroll
          for (int i = 1; i < 16; ++i) {
            if (j + 8 * i < m8[r]) {
              const float t = pass ? __fsub_rn(v[r][i], mu) : v[r][i];
              acc = __fadd_rn(acc, pass ? __fmul_rn(t, t) : t);
            }
          }
        }
        acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
        acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 2));
        acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 4));
        if (j == 0 && m[r] > 0) {
          for (int i = m8[r]; i < m[r]; ++i) {
            const float t = pass ? __fsub_rn(__ldg(xr + start[r] + i), mu) : __ldg(xr + start[r] + i);
            acc = __fadd_rn(acc, pass ? __fmul_rn(t, t) : t);
          }
          leaf_sum[warp][4 * r + (lane >> 3)] = acc;
        }
      }
      __syncwarp();
      float total = 0.0f;
      if (lane == 0) total = pw_tree(p.pw, leaf_sum[warp]);
      total = __fdiv_rn(__shfl_sync(0xffffffffu, total, 0), dn);
      __syncwarp();
      if (pass == 0) {
        mu = total;
      } else {
        const float sd = __fsqrt_rn(__fadd_rn(total, p.eps));
        const float rsd = __frcp_rn(sd);
        // no output aliases gamma or beta: the unrolled loop below may then issue every gamma and
        // beta load ahead of the stores instead of one round trip per element
        const float* __restrict__ gam = p.gamma;
        const float* __restrict__ bet = p.beta;
        float* __restrict__ yout = p.out;
        int8_t* __restrict__ qout = p.out_i8;
        auto emit = [&](int idx, float x) {
          // (x - mu) / sd correctly rounded: Markstein's correction of RN(t * RN(1/sd)), exact for
          // normal quotients (|t| / sd <= sqrt(d) here); tiny and zero t take the IEEE divide
          const float t = __fsub_rn(x, mu);
          float qt;
          if (fabsf(t) >= 0x1p-100f) {
            const float q0 = __fmul_rn(t, rsd);
            qt = __fmaf_rn(__fmaf_rn(-q0, sd, t), rsd, q0);
          } else {
            qt = __fdiv_rn(t, sd);
          }
          const float y = __fadd_rn(__fmul_rn(qt, __ldg(gam + idx)), __ldg(bet + idx));
          if (yout != nullptr) yout[row * p.ld_out + idx] = y;
          if (qout != nullptr) qout[row * p.ld_i8 + idx] = static_cast<int8_t>(quant_byte(y, p.q) & 0xff);
        };
#pragma unroll
        for (int r = 0; r < ROUNDS; ++r) {
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (j + 8 * i < m8[r]) emit(start[r] + j + 8 * i, v[r][i]);
          if (j == 0)
            for (int i = m8[r]; i < m[r]; ++i) emit(start[r] + i, __ldg(xr + start[r] + i));
        }
      }
    }
  }
}

// Rows whose NumPy pairwise recursion is a perfect binary tree: d = NL * L with NL a power of two
// (at most 16) and L a multiple of 8, L <= 128 and, when NL > 1, L > 64 (every split halves the
// range exactly and stops at leaves of L elements: d = 768 is 8 leaves of 96).  A leaf's 8 chains
// (NumPy's 8-way unrolled sum) go to 8 / CPL lanes, CPL chains each: lane q of a leaf loads
// elements CPL*q .. CPL*q + CPL - 1 of every 8 (one 16-byte load for CPL = 4, 8-byte for CPL = 2)
// and accumulates them in element order; lane sums and xor shuffles then rebuild
// ((r0 + r1) + (r2 + r3)) + ((r4 + r5) + (r6 + r7)) and add the leaves up the tree.  Same
// arithmetic as layernorm_rows_reg_kernel, with 32 / (NL * 8 / CPL) rows per warp and no per-element
// bounds or shared-memory tree.  CPL = 2 halves the registers and the serial work per lane.
constexpr int LN_TREE_THREADS = 128;

__device__ __forceinline__ float ln_divide(float t, float sd, float rsd) {
  // (x - mu) / sd correctly rounded: Markstein's correction of RN(t * RN(1/sd)), exact for normal
  // quotients (|t| / sd <= sqrt(d) here); tiny and zero t take the IEEE divide
  if (fabsf(t) >= 0x1p-100f) {
    const float q0 = __fmul_rn(t, rsd);
    return __fmaf_rn(__fmaf_rn(-q0, sd, t), rsd, q0);
  }
  return __fdiv_rn(t, sd);
}

template <int CPL>
struct LnVec;
template <>
struct LnVec<4> {
  using T = float4;
  static __device__ __forceinline__ void get(const T& v, float (&e)[4]) { e[0] = v.x; e[1] = v.y; e[2] = v.z; e[3] = v.w; }
  static __device__ __forceinline__ T make(const float (&e)[4]) { return make_float4(e[0], e[1], e[2], e[3]); }
  static __device__ __forceinline__ T zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }
};
template <>
struct LnVec<2> {
  using T = float2;
  static __device__ __forceinline__ void get(const T& v, float (&e)[2]) { e[0] = v.x; e[1] = v.y; }
  static __device__ __forceinline__ T make(const float (&e)[2]) { return make_float2(e[0], e[1]); }
  static __device__ __forceinline__ T zero() { return make_float2(0.f, 0.f); }
};

template <int L, int NL, int CPL>
__global__ void __launch_bounds__(LN_TREE_THREADS) layernorm_tree_kernel(const LnParams p) {
  using Vec = LnVec<CPL>;
  using VT = typename Vec::T;
  constexpr int LPL = 8 / CPL;        // lanes per leaf
  constexpr int LPR = NL * LPL;       // lanes per row
  static_assert(LPR <= 32, "a row fits a warp");
  constexpr int RPW = 32 / LPR;       // rows per warp
  constexpr int V = L / 8;            // vectors per lane
  const int lane = threadIdx.x & 31;
  const int sub = lane % LPR;
  const int col0 = (sub / LPL) * L + CPL * (sub % LPL);   // first element of this lane; then every 8
  const float dn = static_cast<float>(p.d);
  const VT* __restrict__ gam = reinterpret_cast<const VT*>(p.gamma + col0);
  const VT* __restrict__ bet = reinterpret_cast<const VT*>(p.beta + col0);
  constexpr int STEP = 8 / CPL;       // vectors between a lane's consecutive loads
  const int64_t warps = int64_t(gridDim.x) * (LN_TREE_THREADS / 32);
  for (int64_t w = (int64_t(blockIdx.x) * LN_TREE_THREADS + threadIdx.x) >> 5; w * RPW < p.rows; w += warps) {
    const int64_t row = w * RPW + lane / LPR;
    const bool live = row < p.rows;
    const VT* __restrict__ xr = reinterpret_cast<const VT*>(p.x + (live ? row : 0) * p.ld_x + col0);
    VT v[V];
#pragma unroll
    for (int i = 0; i < V; ++i) v[i] = live ? __ldg(xr + STEP * i) : Vec::zero();
    float mu = 0.0f, sd = 0.0f, rsd = 0.0f;
#pragma unroll
    for (int pass = 0; pass < 2; ++pass) {
      float r[CPL];
#pragma unroll
      for (int i = 0; i < V; ++i) {
        float e[CPL];
        Vec::get(v[i], e);
#pragma unroll
        for (int k = 0; k < CPL; ++k) {
          float t = e[k];
          if (pass) {
            t = __fsub_rn(t, mu);
            t = __fmul_rn(t, t);
          }
          r[k] = i == 0 ? t : __fadd_rn(r[k], t);
        }
      }
      float s;
      if constexpr (CPL == 4) s = __fadd_rn(__fadd_rn(r[0], r[1]), __fadd_rn(r[2], r[3]));
      else s = __fadd_rn(r[0], r[1]);
#pragma unroll
      for (int m = 1; m < LPR; m <<= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, m));
      const float total = __fdiv_rn(s, dn);
      if (pass == 0) {
        mu = total;
      } else {
        sd = __fsqrt_rn(__fadd_rn(total, p.eps));
        rsd = __frcp_rn(sd);
      }
    }
    if (!live) continue;
    VT* __restrict__ yout = p.out != nullptr ? reinterpret_cast<VT*>(p.out + row * p.ld_out + col0) : nullptr;
    int8_t* __restrict__ qout = p.out_i8 != nullptr ? p.out_i8 + row * p.ld_i8 + col0 : nullptr;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      float x[CPL], g[CPL], b[CPL], y[CPL];
      Vec::get(v[i], x);
      Vec::get(__ldg(gam + STEP * i), g);
      Vec::get(__ldg(bet + STEP * i), b);
      uint32_t packed = 0;
#pragma unroll
      for (int k = 0; k < CPL; ++k) {
        y[k] = __fadd_rn(__fmul_rn(ln_divide(__fsub_rn(x[k], mu), sd, rsd), g[k]), b[k]);
        packed |= (quant_byte(y[k], p.q) & 0xffu) << (8 * k);
      }
      if (yout != nullptr) yout[STEP * i] = Vec::make(y);
      if (qout != nullptr) {
        if constexpr (CPL == 4) *reinterpret_cast<uint32_t*>(qout + 8 * i) = packed;
        else *reinterpret_cast<uint16_t*>(qout + 8 * i) = static_cast<uint16_t>(packed);
      }
    }
  }
}

// ---------------------------------------------------------------- softmax

struct SoftmaxParams {
  const float* x;
  int64_t rows, ld_x;
  float* out;
  int64_t ld_out;
  PwLeaves pw;
};

__global__ void __launch_bounds__(ROW_WARPS * 32) softmax_rows_kernel(const SoftmaxParams p) {
  __shared__ float leaf_sum[ROW_WARPS][2 * PW_MAX_LEAVES];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = p.pw.n;
  for (int64_t row = blockIdx.x * int64_t(ROW_WARPS) + warp; row < p.rows; row += int64_t(gridDim.x) * ROW_WARPS) {
    const float* __restrict__ xr = p.x + row * p.ld_x;
    float m = -INFINITY;
    for (int i = lane; i < n; i += 32) m = np_maximum(m, __ldg(xr + i));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = np_maximum(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float s = warp_pairwise_sum(p.pw, [&](int i) { return expf(__fsub_rn(__ldg(xr + i), m)); }, leaf_sum[warp]);
    float* __restrict__ yr = p.out + row * p.ld_out;
    for (int i = lane; i < n; i += 32) yr[i] = __fdiv_rn(expf(__fsub_rn(__ldg(xr + i), m)), s);
  }
}

// ---------------------------------------------------------------- embedding rows

struct EmbedParams {
  const float* table;
  int64_t vocab, d;
  const int32_t* idx;
  int64_t rows;
  const float* addend;
  int64_t addend_rows;
  float* out;
  int64_t ld_out;
  int* err;
};

__global__ void embed_rows_kernel(const EmbedParams p) {
  const int64_t total = p.rows * p.d;
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < total; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = e / p.d, c = e - r * p.d;
    int64_t t = __ldg(p.idx + r);
    if (t < 0) t += p.vocab;
    float v = 0.0f;
    if (t >= 0 && t < p.vocab) {
      v = __ldg(p.table + t * p.d + c);
    } else if (c == 0) {
      atomicExch(p.err, 3);
    }
    if (p.addend != nullptr) v = __fadd_rn(v, __ldg(p.addend + (r % p.addend_rows) * p.d + c));
    p.out[r * p.ld_out + c] = v;
  }
}

// ---------------------------------------------------------------- strided copies

struct View4 {
  int64_t n[4];
  const float* src;
  int64_t ss[4];
  float* dst;
  int64_t ds[4];
};

// One warp per innermost row (the index arithmetic of the outer dimensions once per row).
__global__ void copy_view_kernel(const View4 v) {
  const int64_t rows = v.n[0] * v.n[1] * v.n[2];
  const int lane = threadIdx.x & 31;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
  for (int64_t row = blockIdx.x * int64_t(blockDim.x >> 5) + (threadIdx.x >> 5); row < rows; row += warps) {
    const int64_t i2 = row % v.n[2], i01 = row / v.n[2];
    const int64_t i1 = i01 % v.n[1], i0 = i01 / v.n[1];
    const float* src = v.src + i0 * v.ss[0] + i1 * v.ss[1] + i2 * v.ss[2];
    float* dst = v.dst + i0 * v.ds[0] + i1 * v.ds[1] + i2 * v.ds[2];
    for (int64_t i3 = lane; i3 < v.n[3]; i3 += 32) dst[i3 * v.ds[3]] = __ldg(src + i3 * v.ss[3]);
  }
}

// ---------------------------------------------------------------- standalone element-wise ops

// out = f(a) for the unary MIRA_EPI_* ops, or f(a, b) / f(b, a) (swapped) for the binary ones, b a
// view or a scalar; [n0, n1, n2, n3] through 4-D views (broadcast dims have stride 0), one warp per
// innermost row.  The arithmetic is the epilogue's (apply_unary / apply_binary): the reference's
// UNARY / BINARY ops (ops.py:99-139) with IEEE rounding for the binary ones.
struct EltParams {
  int64_t n[4];
  const float* a;
  int64_t as[4];
  const float* b;
  int64_t bs[4];
  float scalar;
  int op, unary, swapped;
  float* out;
  int64_t os[4];
};

__global__ void elementwise_f32_kernel(const EltParams p) {
  const int64_t rows = p.n[0] * p.n[1] * p.n[2];
  const int lane = threadIdx.x & 31;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
  for (int64_t row = blockIdx.x * int64_t(blockDim.x >> 5) + (threadIdx.x >> 5); row < rows; row += warps) {
    const int64_t i2 = row % p.n[2], i01 = row / p.n[2];
    const int64_t i1 = i01 % p.n[1], i0 = i01 / p.n[1];
    const float* a = p.a + i0 * p.as[0] + i1 * p.as[1] + i2 * p.as[2];
    const float* b = p.b != nullptr ? p.b + i0 * p.bs[0] + i1 * p.bs[1] + i2 * p.bs[2] : nullptr;
    float* o = p.out + i0 * p.os[0] + i1 * p.os[1] + i2 * p.os[2];
    for (int64_t i3 = lane; i3 < p.n[3]; i3 += 32) {
      const float x = __ldg(a + i3 * p.as[3]);
      float y;
      if (p.unary) {
        y = apply_unary(p.op, x);
      } else {
        const float v = b != nullptr ? __ldg(b + i3 * p.bs[3]) : p.scalar;
        y = p.swapped ? apply_binary(p.op, v, x) : apply_binary(p.op, x, v);
      }
      o[i3 * p.os[3]] = y;
    }
  }
}

// ---------------------------------------------------------------- slices at runtime positions

// The reference's dynamic_slice / dynamic_update_slice (ops.py:533-576): a window of shape n at a
// start position read from device memory (so a captured CUDA graph stays valid while the position
// changes), each start clamped to [0, dims - n] like _clamped_starts (ops.py:536-537).  The start
// vector has `rank` entries for the last `rank` of the 4 dimensions; the others start at 0.
// update == 0: dst[e] = src[start + e] (slice); update == 1: dst[start + e] = src[e] (update).
// Elements are 4 bytes (f32 or i32), copied as bits.
struct DynWindowParams {
  const uint32_t* src;
  int64_t ss[4];
  uint32_t* dst;
  int64_t ds[4];
  int64_t n[4];       // window shape
  int64_t dims[4];    // full shape of the windowed side
  const int32_t* start;
  int rank;
  int update;
};

// One warp per innermost window row.
__global__ void dyn_window_kernel(const DynWindowParams p) {
  __shared__ int64_t s[4];
  if (threadIdx.x < 4) {
    const int d = threadIdx.x, j = d - (4 - p.rank);
    int64_t v = 0;
    if (j >= 0) {
      v = __ldg(p.start + j);
      v = v < 0 ? 0 : v;
      v = v > p.dims[d] - p.n[d] ? p.dims[d] - p.n[d] : v;
    }
    s[d] = v;
  }
  __syncthreads();
  const int64_t ws0 = p.update ? 0 : s[0], ws1 = p.update ? 0 : s[1], ws2 = p.update ? 0 : s[2],
                ws3 = p.update ? 0 : s[3];
  const int64_t wd0 = p.update ? s[0] : 0, wd1 = p.update ? s[1] : 0, wd2 = p.update ? s[2] : 0,
                wd3 = p.update ? s[3] : 0;
  const int64_t rows = p.n[0] * p.n[1] * p.n[2];
  const int lane = threadIdx.x & 31;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
  for (int64_t row = blockIdx.x * int64_t(blockDim.x >> 5) + (threadIdx.x >> 5); row < rows; row += warps) {
    const int64_t i2 = row % p.n[2], i01 = row / p.n[2];
    const int64_t i1 = i01 % p.n[1], i0 = i01 / p.n[1];
    const uint32_t* src = p.src + (ws0 + i0) * p.ss[0] + (ws1 + i1) * p.ss[1] + (ws2 + i2) * p.ss[2] + ws3 * p.ss[3];
    uint32_t* dst = p.dst + (wd0 + i0) * p.ds[0] + (wd1 + i1) * p.ds[1] + (wd2 + i2) * p.ds[2] + wd3 * p.ds[3];
    for (int64_t i3 = lane; i3 < p.n[3]; i3 += 32) dst[i3 * p.ds[3]] = src[i3 * p.ss[3]];
  }
}

// ---------------------------------------------------------------- batched f32 matmul

constexpr int BMM_BM = 128, BMM_BN = 64, BMM_BK = 16, BMM_THREADS = 256;
constexpr int BMM_TM = 8, BMM_TN = 4;      // outputs per thread: 16 x 16 threads cover 128 x 64
constexpr int BMM_APAD = BMM_BM + 4, BMM_BPAD = BMM_BN + 4;

struct BmmParams {
  int64_t batches, batch1, m, n, k;
  const float* a;
  int64_t as[4];
  const float* b;
  int64_t bs[4];
  // weight-only int8 B (b == nullptr): element (k, n) is RN(f32(b_i8[k, n]) * b_scale[n]), the
  // reference's dequantize (ops.py:583-587) of a [K, N] weight with one scale per column
  const int8_t* b_i8;
  const float* b_scale;
  bool a_kfast, b_nfast;
  int n_steps;
  mira_bmm_step steps[MIRA_EPI_MAX_STEPS];
  float* out;
  int64_t os[4];
  int8_t* out_i8;
  int64_t qs[4];
  QuantScale q;
};

__device__ __forceinline__ void bmm_load_tiles(const BmmParams& p, const float* a, int64_t boff, int64_t m0,
                                               int64_t n0, int64_t k0, float (&ra)[8], float (&rb)[4]) {
  const int t = threadIdx.x;
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const int idx = t + r * BMM_THREADS;
    int mm, kk;
    if (p.a_kfast) { kk = idx % BMM_BK; mm = idx / BMM_BK; } else { mm = idx % BMM_BM; kk = idx / BMM_BM; }
    const int64_t gm = m0 + mm, gk = k0 + kk;
    ra[r] = (gm < p.m && gk < p.k) ? __ldg(a + gm * p.as[2] + gk * p.as[3]) : 0.0f;
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int idx = t + r * BMM_THREADS;
    int nn, kk;
    if (p.b_nfast) { nn = idx % BMM_BN; kk = idx / BMM_BN; } else { kk = idx % BMM_BK; nn = idx / BMM_BK; }
    const int64_t gn = n0 + nn, gk = k0 + kk;
    const int64_t off = boff + gk * p.bs[2] + gn * p.bs[3];
    if (p.b_i8 != nullptr)
      rb[r] = (gn < p.n && gk < p.k) ? __fmul_rn(static_cast<float>(__ldg(p.b_i8 + off)), __ldg(p.b_scale + gn)) : 0.0f;
    else
      rb[r] = (gn < p.n && gk < p.k) ? __ldg(p.b + off) : 0.0f;
  }
}

__device__ __forceinline__ void bmm_store_tiles(const BmmParams& p, float (*As)[BMM_APAD], float (*Bs)[BMM_BPAD],
                                                const float (&ra)[8], const float (&rb)[4]) {
  const int t = threadIdx.x;
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const int idx = t + r * BMM_THREADS;
    int mm, kk;
    if (p.a_kfast) { kk = idx % BMM_BK; mm = idx / BMM_BK; } else { mm = idx % BMM_BM; kk = idx / BMM_BM; }
    As[kk][mm] = ra[r];
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int idx = t + r * BMM_THREADS;
    int nn, kk;
    if (p.b_nfast) { nn = idx % BMM_BN; kk = idx / BMM_BN; } else { kk = idx % BMM_BK; nn = idx / BMM_BK; }
    Bs[kk][nn] = rb[r];
  }
}

// One 128 x 64 output tile per CTA; blockIdx.z strides over the batch entries.  Operand tiles go through
// registers (the next k-slice is fetched while the current one is multiplied) into shared memory.
__global__ void __launch_bounds__(BMM_THREADS, 1) bmm_f32_kernel(const BmmParams p) {
  __shared__ __align__(16) float As[2][BMM_BK][BMM_APAD];
  __shared__ __align__(16) float Bs[2][BMM_BK][BMM_BPAD];
  for (int64_t bz = blockIdx.z; bz < p.batches; bz += gridDim.z) {
  const int64_t b0 = bz / p.batch1, b1 = bz - b0 * p.batch1;
  const float* a = p.a + b0 * p.as[0] + b1 * p.as[1];
  const int64_t boff = b0 * p.bs[0] + b1 * p.bs[1];
  const int64_t m0 = int64_t(blockIdx.y) * BMM_BM, n0 = int64_t(blockIdx.x) * BMM_BN;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;

  float acc[BMM_TM][BMM_TN];
#pragma unroll
  for (int i = 0; i < BMM_TM; ++i)
#pragma unroll
    for (int j = 0; j < BMM_TN; ++j) acc[i][j] = 0.0f;

  float ra[8], rb[4];
  bmm_load_tiles(p, a, boff, m0, n0, 0, ra, rb);
  bmm_store_tiles(p, As[0], Bs[0], ra, rb);
  __syncthreads();
  const int nk = static_cast<int>((p.k + BMM_BK - 1) / BMM_BK);
  for (int kt = 0; kt < nk; ++kt) {
    const int cur = kt & 1;
    if (kt + 1 < nk) bmm_load_tiles(p, a, boff, m0, n0, int64_t(kt + 1) * BMM_BK, ra, rb);
#pragma unroll
    for (int kk = 0; kk < BMM_BK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[cur][kk][ty * BMM_TM]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[cur][kk][ty * BMM_TM + 4]);
      const float4 bv = *reinterpret_cast<const float4*>(&Bs[cur][kk][tx * BMM_TN]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
      for (int i = 0; i < BMM_TM; ++i)
#pragma unroll
        for (int j = 0; j < BMM_TN; ++j) acc[i][j] = fmaf(av[i], bw[j], acc[i][j]);
    }
    if (kt + 1 < nk) bmm_store_tiles(p, As[cur ^ 1], Bs[cur ^ 1], ra, rb);
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < BMM_TM; ++i) {
    const int64_t gm = m0 + ty * BMM_TM + i;
    if (gm >= p.m) continue;
#pragma unroll
    for (int j = 0; j < BMM_TN; ++j) {
      const int64_t gn = n0 + tx * BMM_TN + j;
      if (gn >= p.n) continue;
      float v = acc[i][j];
      for (int s = 0; s < p.n_steps; ++s) {
        const mira_bmm_step& st = p.steps[s];
        if (st.operand == MIRA_OPND_NONE) {
          v = apply_unary(st.op, v);
          continue;
        }
        float o = st.scalar;
        if (st.operand == MIRA_OPND_VIEW) {
          const float* op = static_cast<const float*>(st.view.ptr);
          o = __ldg(op + b0 * st.view.stride[0] + b1 * st.view.stride[1] + gm * st.view.stride[2] +
                    gn * st.view.stride[3]);
        }
        v = st.swapped ? apply_binary(st.op, o, v) : apply_binary(st.op, v, o);
      }
      if (p.out != nullptr) p.out[b0 * p.os[0] + b1 * p.os[1] + gm * p.os[2] + gn * p.os[3]] = v;
      if (p.out_i8 != nullptr)
        p.out_i8[b0 * p.qs[0] + b1 * p.qs[1] + gm * p.qs[2] + gn * p.qs[3]] =
            static_cast<int8_t>(quant_byte(v, p.q) & 0xff);
    }
  }
  __syncthreads();   // the next batch entry refills the shared tiles
  }
}

}  // namespace mira

namespace mira {

// ---------------------------------------------------------------- max |x| over a view

struct AbsMaxParams {
  int64_t n[4];
  const float* x;
  int64_t s[4];
  unsigned int* out;      // float bits of the maximum (non-negative floats order like integers)
};

__global__ void absmax_view_kernel(const AbsMaxParams p) {
  const int64_t rows = p.n[0] * p.n[1] * p.n[2];
  const int lane = threadIdx.x & 31;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
  float m = 0.0f;
  for (int64_t row = blockIdx.x * int64_t(blockDim.x >> 5) + (threadIdx.x >> 5); row < rows; row += warps) {
    const int64_t i2 = row % p.n[2], i01 = row / p.n[2];
    const int64_t i1 = i01 % p.n[1], i0 = i01 / p.n[1];
    const float* x = p.x + i0 * p.s[0] + i1 * p.s[1] + i2 * p.s[2];
    for (int64_t i3 = lane; i3 < p.n[3]; i3 += 32) {
      float a = fabsf(__ldg(x + i3 * p.s[3]));
      if (a != a) a = INFINITY;
      m = fmaxf(m, a);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(p.out, __float_as_uint(m));
}

// ---------------------------------------------------------------- fused attention (f32)
//
// One chain of the reference, o = softmax((q @ k^T) * scale + mask, axis=-1) @ v, per (batch0,
// batch1) and block of 64 query rows, without materializing the scores: the score tile lives in
// registers, the softmax runs online (running row maximum and sum, earlier partial outputs
// rescaled by exp(m_old - m_new)) and the probabilities go through shared memory into p @ v.
//
// Skipping key tiles.  A key tile whose mask entries are all strongly negative (tile_max from the
// host) is left out only when, for every row i of the block,
//   |scale| * ||q_i||_1 * max|k| + tile_max - m_i < -110,
// where m_i is the running row maximum: then every score of the tile is below m_i - 110 and the
// reference's exp(s - max) is exactly 0 for it, so its contribution to the sum and to p @ v is
// exactly 0 there too.  Tiles that fail the test are processed like the others.

constexpr int ATT_BQ = 64, ATT_BK = 64, ATT_THREADS = 256;

struct AttnParams {
  int tq, tk, dh;
  const float* q;
  int64_t qs[4];
  const float* k;
  int64_t ks[4];
  const float* v;
  int64_t vs[4];
  int vec;                  // k and v rows load as 16-byte chunks (cp.async, double-buffered)
  int scale_op;             // 0, MIRA_EPI_MUL or MIRA_EPI_DIV
  float scale;
  float scale_abs;          // an upper bound of |scale| (|1/scale| for DIV)
  const float* mask;        // added after the scale step; NULL: none
  int64_t ms[4];
  const float* tile_max;    // [nqb][nkb] maximum mask value per tile; NULL: no skipping
  const unsigned int* kmax; // max |k| (float bits); NULL: no skipping
  const unsigned char* tile_zero;  // [nqb][nkb] 1 where every mask entry of the tile is +0; may be NULL
  float* out;
  int64_t os[4];
  int8_t* out_i8;
  int64_t is[4];
  QuantScale q8;
  int* err;                 // kernel error record (the tensor-core kernel's bounded waits)
};

// Row-major tiles with a 4-float pad: a thread reads rows ty + 16u of q and tx + 16v of k as
// 16-byte vectors along d, which keeps every 8-thread phase of a 128-bit shared load on distinct
// banks; k and v are double-buffered.
template <int DH>
struct AttnSmem {
  float q[ATT_BQ][DH + 4];
  float k[2][ATT_BK][DH + 4];
  float v[2][ATT_BK][DH + 4];
  float p[ATT_BQ][ATT_BK + 4];
  float qn1[ATT_BQ];
};

template <int DH>
__device__ __forceinline__ void attn_load_kv(const AttnParams& p, AttnSmem<DH>& sm, const float* kp, const float* vp,
                                             int k0, int buf) {
  const int tid = threadIdx.x;
  if (p.vec) {
    constexpr int CH = DH / 4;    // 16-byte chunks per row
    for (int e = tid; e < ATT_BK * CH; e += ATT_THREADS) {
      const int c = e / CH, d = (e - c * CH) * 4;
      const bool ok = k0 + c < p.tk && d < p.dh;
      const float* ks = ok ? kp + int64_t(k0 + c) * p.ks[2] + d : kp;
      const float* vs = ok ? vp + int64_t(k0 + c) * p.vs[2] + d : vp;
      cp_async_16(static_cast<uint32_t>(__cvta_generic_to_shared(&sm.k[buf][c][d])), ks, ok ? 16u : 0u);
      cp_async_16(static_cast<uint32_t>(__cvta_generic_to_shared(&sm.v[buf][c][d])), vs, ok ? 16u : 0u);
    }
  } else {
    for (int e = tid; e < ATT_BK * DH; e += ATT_THREADS) {
      const int c = e / DH, d = e - c * DH;
      const bool ok = k0 + c < p.tk && d < p.dh;
      sm.k[buf][c][d] = ok ? __ldg(kp + int64_t(k0 + c) * p.ks[2] + int64_t(d) * p.ks[3]) : 0.0f;
      sm.v[buf][c][d] = ok ? __ldg(vp + int64_t(k0 + c) * p.vs[2] + int64_t(d) * p.vs[3]) : 0.0f;
    }
  }
}

// One key tile: scores, online-softmax update, probabilities through shared memory, p @ v.
template <int DH>
__device__ __forceinline__ void attn_compute(const AttnParams& p, AttnSmem<DH>& sm, const float* mp, int q0, int k0,
                                             int buf, float (&m)[4], float (&l)[4], float (&o)[4][DH / 16]) {
  constexpr int CN = DH / 16;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  float s[4][4];
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int v = 0; v < 4; ++v) s[u][v] = 0.0f;
#pragma unroll
  for (int d = 0; d < DH; d += 4) {
    float4 a[4], b[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) a[u] = *reinterpret_cast<const float4*>(&sm.q[ty + 16 * u][d]);
#pragma unroll
    for (int v = 0; v < 4; ++v) b[v] = *reinterpret_cast<const float4*>(&sm.k[buf][tx + 16 * v][d]);
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        float t = fmaf(a[u].x, b[v].x, s[u][v]);
        t = fmaf(a[u].y, b[v].y, t);
        t = fmaf(a[u].z, b[v].z, t);
        s[u][v] = fmaf(a[u].w, b[v].w, t);
      }
  }
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int r = q0 + ty + 16 * u;
    float rmax = -INFINITY;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const int c = k0 + tx + 16 * v;
      float x = s[u][v];
      if (p.scale_op == MIRA_EPI_MUL) x = __fmul_rn(x, p.scale);
      else if (p.scale_op == MIRA_EPI_DIV) x = __fdiv_rn(x, p.scale);
      if (mp != nullptr && r < p.tq && c < p.tk) x = __fadd_rn(x, __ldg(mp + int64_t(r) * p.ms[2] + int64_t(c) * p.ms[3]));
      if (c >= p.tk) x = -INFINITY;
      s[u][v] = x;
      rmax = fmaxf(rmax, x);
    }
#pragma unroll
    for (int off = 1; off < 16; off <<= 1) rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, off));
    const float mnew = fmaxf(m[u], rmax);
    const float corr = (mnew == -INFINITY) ? 1.0f : expf(m[u] - mnew);
    float rsum = 0.0f;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const float e = (mnew == -INFINITY) ? 0.0f : expf(s[u][v] - mnew);
      sm.p[ty + 16 * u][tx + 16 * v] = e;
      rsum += e;
    }
#pragma unroll
    for (int off = 1; off < 16; off <<= 1) rsum += __shfl_xor_sync(0xffffffffu, rsum, off);
    l[u] = fmaf(l[u], corr, rsum);
#pragma unroll
    for (int c = 0; c < CN; ++c) o[u][c] *= corr;
    m[u] = mnew;
  }
  __syncthreads();
#pragma unroll 4
  for (int j = 0; j < ATT_BK; j += 4) {
    float4 pa[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) pa[u] = *reinterpret_cast<const float4*>(&sm.p[ty + 16 * u][j]);
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      float bv[CN];
      if constexpr (CN % 4 == 0) {
#pragma unroll
        for (int c = 0; c < CN; c += 4) {
          const float4 t = *reinterpret_cast<const float4*>(&sm.v[buf][j + jj][tx * CN + c]);
          bv[c] = t.x; bv[c + 1] = t.y; bv[c + 2] = t.z; bv[c + 3] = t.w;
        }
      } else {
#pragma unroll
        for (int c = 0; c < CN; ++c) bv[c] = sm.v[buf][j + jj][tx * CN + c];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float pv = jj == 0 ? pa[u].x : (jj == 1 ? pa[u].y : (jj == 2 ? pa[u].z : pa[u].w));
#pragma unroll
        for (int c = 0; c < CN; ++c) o[u][c] = fmaf(pv, bv[c], o[u][c]);
      }
    }
  }
}

template <int DH>
__global__ void __launch_bounds__(ATT_THREADS) attention_f32_kernel(const AttnParams p) {
  extern __shared__ __align__(16) unsigned char att_smem_raw[];
  AttnSmem<DH>& sm = *reinterpret_cast<AttnSmem<DH>*>(att_smem_raw);
  constexpr int CN = DH / 16;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int nqb = (p.tq + ATT_BQ - 1) / ATT_BQ, nkb = (p.tk + ATT_BK - 1) / ATT_BK;
  const int qb = nqb - 1 - static_cast<int>(blockIdx.x);     // the longest rows first
  const int q0 = qb * ATT_BQ;
  const int64_t b1 = blockIdx.y, b0 = blockIdx.z;
  const float* qp = p.q + b0 * p.qs[0] + b1 * p.qs[1];
  const float* kp = p.k + b0 * p.ks[0] + b1 * p.ks[1];
  const float* vp = p.v + b0 * p.vs[0] + b1 * p.vs[1];
  const float* mp = p.mask != nullptr ? p.mask + b0 * p.ms[0] + b1 * p.ms[1] : nullptr;
  const bool can_skip = p.tile_max != nullptr && p.kmax != nullptr;
  const float* tmax = can_skip ? p.tile_max + int64_t(qb) * nkb : nullptr;
  auto candidate = [&](int kb) { return can_skip && __ldg(tmax + kb) <= -200.0f; };
  auto next_tile = [&](int kb) {
    while (kb < nkb && candidate(kb)) ++kb;
    return kb;
  };

  int cur = next_tile(0);
  if (cur < nkb) attn_load_kv<DH>(p, sm, kp, vp, cur * ATT_BK, 0);
  cp_async_commit();
  for (int e = tid; e < ATT_BQ * DH; e += ATT_THREADS) {
    const int r = e / DH, d = e - r * DH;
    sm.q[r][d] = (q0 + r < p.tq && d < p.dh) ? __ldg(qp + int64_t(q0 + r) * p.qs[2] + int64_t(d) * p.qs[3]) : 0.0f;
  }
  __syncthreads();
  {
    // ||q_i||_1: four threads per row
    const int r = tid >> 2, part = tid & 3;
    float a = 0.0f;
    for (int d = part; d < DH; d += 4) a += fabsf(sm.q[r][d]);
    a += __shfl_xor_sync(0xffffffffu, a, 1);
    a += __shfl_xor_sync(0xffffffffu, a, 2);
    if (part == 0) sm.qn1[r] = a;
  }
  float m[4], l[4], o[4][CN];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    m[u] = -INFINITY;
    l[u] = 0.0f;
#pragma unroll
    for (int c = 0; c < CN; ++c) o[u][c] = 0.0f;
  }
  int buf = 0;
  while (cur < nkb) {
    const int nxt = next_tile(cur + 1);
    if (nxt < nkb) {
      attn_load_kv<DH>(p, sm, kp, vp, nxt * ATT_BK, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    // a tile whose mask entries are all +0 adds nothing: x + 0 only turns -0 into +0, which
    // leaves every exp(x - m) unchanged
    const bool zero_mask = p.tile_zero != nullptr && __ldg(p.tile_zero + int64_t(qb) * nkb + cur) != 0;
    attn_compute<DH>(p, sm, zero_mask ? nullptr : mp, q0, cur * ATT_BK, buf, m, l, o);
    __syncthreads();
    cur = nxt;
    buf ^= 1;
  }
  cp_async_wait<0>();
  __syncthreads();
  if (can_skip) {
    const float kmax = __uint_as_float(__ldg(p.kmax));
    for (int kb = 0; kb < nkb; ++kb) {
      if (!candidate(kb)) continue;
      const float tm = __ldg(tmax + kb);
      bool ok = true;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int r = ty + 16 * u;
        if (q0 + r < p.tq) {
          // every score of this tile is at most this bound; the factor 1.001 and the margin
          // cover the rounding of the products
          const float bound = p.scale_abs * sm.qn1[r] * kmax * 1.001f + tm;
          ok = ok && (bound - m[u] < -110.0f);
        }
      }
      if (!__syncthreads_and(ok)) {
        attn_load_kv<DH>(p, sm, kp, vp, kb * ATT_BK, 0);
        cp_async_commit();
        cp_async_wait<0>();
        __syncthreads();
        attn_compute<DH>(p, sm, mp, q0, kb * ATT_BK, 0, m, l, o);
        __syncthreads();
      }
    }
  }
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int r = q0 + ty + 16 * u;
    if (r >= p.tq) continue;
#pragma unroll
    for (int c = 0; c < CN; ++c) {
      const int col = tx * CN + c;
      if (col >= p.dh) continue;
      const float y = __fdiv_rn(o[u][c], l[u]);
      if (p.out != nullptr) p.out[b0 * p.os[0] + b1 * p.os[1] + int64_t(r) * p.os[2] + int64_t(col) * p.os[3]] = y;
      if (p.out_i8 != nullptr)
        p.out_i8[b0 * p.is[0] + b1 * p.is[1] + int64_t(r) * p.is[2] + int64_t(col) * p.is[3]] =
            static_cast<int8_t>(quant_byte(y, p.q8) & 0xff);
    }
  }
}

// ---------------------------------------------------------------- single-query attention (decode)

constexpr int ATT1_WARPS = 8;
constexpr int ATT1_UNROLL = 4;     // keys per lane group in flight

// One query row per (batch0, batch1) entry against tk keys: the decode step, where a key/value
// cache of tk rows is read once and nothing is reused.  One CTA per entry; each warp is split into
// groups of DH/4 lanes, a group holds one key at a time (every lane 4 of its DH values, 16-byte
// loads of k and v rows), the warps stride over the keys.  Each group keeps its own online softmax
// state with the arithmetic of attn_compute (scale step, mask add, expf(s - m), rescaled sums);
// the groups are merged in shared memory at the end, then o / l (rounded division) and the
// optional int8 requantization like attention_f32_kernel.  Needs tq == 1 and vec (contiguous
// 16-byte aligned k and v rows).
template <int DH>
__global__ void __launch_bounds__(ATT1_WARPS * 32) attention_q1_kernel(const AttnParams p) {
  constexpr int G = DH / 4;              // lanes per key
  constexpr int KPW = 32 / G;            // keys per warp per round
  constexpr int NGRP = ATT1_WARPS * KPW;
  __shared__ float s_m[NGRP], s_l[NGRP];
  __shared__ __align__(16) float s_o[NGRP][DH];
  const int64_t b0 = blockIdx.y, b1 = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane % G, slot = lane / G, grp = warp * KPW + slot;
  const int d0 = 4 * sub;
  const bool dim_ok = d0 < p.dh;
  const float* qp = p.q + b0 * p.qs[0] + b1 * p.qs[1];
  float4 q4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  if (dim_ok) {
    q4.x = __ldg(qp + int64_t(d0) * p.qs[3]);
    q4.y = __ldg(qp + int64_t(d0 + 1) * p.qs[3]);
    q4.z = __ldg(qp + int64_t(d0 + 2) * p.qs[3]);
    q4.w = __ldg(qp + int64_t(d0 + 3) * p.qs[3]);
  }
  const float* kp = p.k + b0 * p.ks[0] + b1 * p.ks[1];
  const float* vp = p.v + b0 * p.vs[0] + b1 * p.vs[1];
  const float* mp = p.mask != nullptr ? p.mask + b0 * p.ms[0] + b1 * p.ms[1] : nullptr;
  float m = -INFINITY, l = 0.0f;
  float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  const int stride = NGRP * ATT1_UNROLL;
  // the loop bound is the warp's first key, the same for all 32 lanes, so every lane reaches the
  // full-mask shuffles below; keys past tk enter the softmax as -inf
  for (int jw = warp * KPW * ATT1_UNROLL; jw < p.tk; jw += stride) {
    const int j0 = jw + slot * ATT1_UNROLL;
    float4 kv[ATT1_UNROLL], vv[ATT1_UNROLL];
#pragma unroll
    for (int u = 0; u < ATT1_UNROLL; ++u) {
      const int j = j0 + u;
      const bool ok = j < p.tk && dim_ok;
      kv[u] = ok ? __ldg(reinterpret_cast<const float4*>(kp + int64_t(j) * p.ks[2] + d0)) : make_float4(0.f, 0.f, 0.f, 0.f);
      vv[u] = ok ? __ldg(reinterpret_cast<const float4*>(vp + int64_t(j) * p.vs[2] + d0)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < ATT1_UNROLL; ++u) {
      const int j = j0 + u;
      float t = fmaf(q4.x, kv[u].x, 0.0f);
      t = fmaf(q4.y, kv[u].y, t);
      t = fmaf(q4.z, kv[u].z, t);
      t = fmaf(q4.w, kv[u].w, t);
#pragma unroll
      for (int off = 1; off < G; off <<= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
      float x = t;
      if (p.scale_op == MIRA_EPI_MUL) x = __fmul_rn(x, p.scale);
      else if (p.scale_op == MIRA_EPI_DIV) x = __fdiv_rn(x, p.scale);
      if (mp != nullptr && j < p.tk) x = __fadd_rn(x, __ldg(mp + int64_t(j) * p.ms[3]));
      if (j >= p.tk) x = -INFINITY;
      const float mnew = fmaxf(m, x);
      const float corr = (mnew == -INFINITY) ? 1.0f : expf(m - mnew);
      const float e = (mnew == -INFINITY) ? 0.0f : expf(x - mnew);
      l = fmaf(l, corr, e);
      o.x = fmaf(e, vv[u].x, o.x * corr);
      o.y = fmaf(e, vv[u].y, o.y * corr);
      o.z = fmaf(e, vv[u].z, o.z * corr);
      o.w = fmaf(e, vv[u].w, o.w * corr);
      m = mnew;
    }
  }
  if (sub == 0) { s_m[grp] = m; s_l[grp] = l; }
  if (dim_ok) *reinterpret_cast<float4*>(&s_o[grp][d0]) = o;
  __syncthreads();
  for (int d = threadIdx.x; d < p.dh; d += blockDim.x) {
    float mt = -INFINITY;
    for (int g = 0; g < NGRP; ++g) mt = fmaxf(mt, s_m[g]);
    float lt = 0.0f, ot = 0.0f;
    for (int g = 0; g < NGRP; ++g) {
      if (s_m[g] == -INFINITY) continue;
      const float c = expf(s_m[g] - mt);
      lt = fmaf(s_l[g], c, lt);
      ot = fmaf(s_o[g][d], c, ot);
    }
    const float y = __fdiv_rn(ot, lt);
    if (p.out != nullptr) p.out[b0 * p.os[0] + b1 * p.os[1] + int64_t(d) * p.os[3]] = y;
    if (p.out_i8 != nullptr)
      p.out_i8[b0 * p.is[0] + b1 * p.is[1] + int64_t(d) * p.is[3]] = static_cast<int8_t>(quant_byte(y, p.q8) & 0xff);
  }
}

}  // namespace mira
