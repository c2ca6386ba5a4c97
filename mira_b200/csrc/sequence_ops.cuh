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

namespace mira {

constexpr int PW_MAX_LEAVES = 128;

// Leaves of NumPy's pairwise recursion for rows of n elements (computed on the host).
struct PwLeaves {
  int n;
  int count;
  int start[PW_MAX_LEAVES + 1];
};

__device__ float pw_tree(const float* leaf_sum, int n, int& k) {
  if (n <= 128) return leaf_sum[k++];
  int n2 = n / 2;
  n2 -= n2 % 8;
  const float a = pw_tree(leaf_sum, n2, k);
  const float b = pw_tree(leaf_sum, n - n2, k);
  return __fadd_rn(a, b);
}

// Sum of elem(0) .. elem(n-1) in NumPy's float32 pairwise order; every lane returns the total.
// leaf_sum: PW_MAX_LEAVES floats of shared memory owned by this warp.
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
  if (lane == 0) {
    int k = 0;
    total = pw_tree(leaf_sum, pw.n, k);
  }
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
  __shared__ float leaf_sum[ROW_WARPS][PW_MAX_LEAVES];
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

// ---------------------------------------------------------------- softmax

struct SoftmaxParams {
  const float* x;
  int64_t rows, ld_x;
  float* out;
  int64_t ld_out;
  PwLeaves pw;
};

__global__ void __launch_bounds__(ROW_WARPS * 32) softmax_rows_kernel(const SoftmaxParams p) {
  __shared__ float leaf_sum[ROW_WARPS][PW_MAX_LEAVES];
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
      atomicExch(p.err, 2);
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

__global__ void copy_view_kernel(const View4 v) {
  const int64_t total = v.n[0] * v.n[1] * v.n[2] * v.n[3];
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < total; e += int64_t(gridDim.x) * blockDim.x) {
    int64_t r = e;
    const int64_t i3 = r % v.n[3];
    r /= v.n[3];
    const int64_t i2 = r % v.n[2];
    r /= v.n[2];
    const int64_t i1 = r % v.n[1];
    const int64_t i0 = r / v.n[1];
    v.dst[i0 * v.ds[0] + i1 * v.ds[1] + i2 * v.ds[2] + i3 * v.ds[3]] =
        __ldg(v.src + i0 * v.ss[0] + i1 * v.ss[1] + i2 * v.ss[2] + i3 * v.ss[3]);
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
  bool a_kfast, b_nfast;
  int n_steps;
  mira_bmm_step steps[MIRA_EPI_MAX_STEPS];
  float* out;
  int64_t os[4];
  int8_t* out_i8;
  int64_t qs[4];
  QuantScale q;
};

__device__ __forceinline__ void bmm_load_tiles(const BmmParams& p, const float* a, const float* b, int64_t m0,
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
    rb[r] = (gn < p.n && gk < p.k) ? __ldg(b + gk * p.bs[2] + gn * p.bs[3]) : 0.0f;
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
  const float* b = p.b + b0 * p.bs[0] + b1 * p.bs[1];
  const int64_t m0 = int64_t(blockIdx.y) * BMM_BM, n0 = int64_t(blockIdx.x) * BMM_BN;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;

  float acc[BMM_TM][BMM_TN];
#pragma unroll
  for (int i = 0; i < BMM_TM; ++i)
#pragma unroll
    for (int j = 0; j < BMM_TN; ++j) acc[i][j] = 0.0f;

  float ra[8], rb[4];
  bmm_load_tiles(p, a, b, m0, n0, 0, ra, rb);
  bmm_store_tiles(p, As[0], Bs[0], ra, rb);
  __syncthreads();
  const int nk = static_cast<int>((p.k + BMM_BK - 1) / BMM_BK);
  for (int kt = 0; kt < nk; ++kt) {
    const int cur = kt & 1;
    if (kt + 1 < nk) bmm_load_tiles(p, a, b, m0, n0, int64_t(kt + 1) * BMM_BK, ra, rb);
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
