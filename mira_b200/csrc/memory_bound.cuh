// K3/K4/K5: the memory-bound kernels around the int8 GEMMs: activation quantization (with the
// NCHW -> NHWC layout change at graph inputs), max pooling, the global mean, the f32 depthwise
// convolution, and the f32 layout changes at graph outputs.  All are 128-bit vectorised where the
// layout allows and use the exact rounding helpers of exact_math.cuh.
#pragma once
#include <cstdint>

#include "exact_math.cuh"

namespace mira {

struct QuantScale {
  float s, rcp, lim;   // divisor, RN32(1/divisor), 256 * divisor
  float c127;          // RN32(127 * divisor): the clamp of the packed requantization (requant_x2)
};

__device__ __forceinline__ uint32_t quant_byte(float x, const QuantScale& q) {
  return round_clip_i8(div_by_scale(x, q.s, q.rcp, q.lim));
}

// ---------------------------------------------------------------- K3: quantize rows

// One thread per 16 output bytes of a row: xq[r, c0:c0+16] from x[r, c0:c0+16] (0 past `cols`).
__global__ void quantize_rows_kernel(const float* __restrict__ x, int64_t rows, int64_t cols, int64_t ld_x,
                                     QuantScale q, int8_t* __restrict__ xq, int64_t ld_q) {
  const int64_t groups = ld_q / 16;
  const int64_t total = rows * groups;
  const bool vec = (ld_x % 4) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  for (int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; idx < total;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = idx / groups;
    const int64_t c0 = (idx - r * groups) * 16;
    const float* src = x + r * ld_x + c0;
    float v[16];
    if (vec && c0 + 16 <= cols) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(src) + k);
        v[4 * k] = t.x; v[4 * k + 1] = t.y; v[4 * k + 2] = t.z; v[4 * k + 3] = t.w;
      }
    } else {
#pragma unroll
      for (int k = 0; k < 16; ++k) v[k] = (c0 + k < cols) ? src[k] : 0.0f;
    }
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t b[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) b[e] = (c0 + 4 * k + e < cols) ? quant_byte(v[4 * k + e], q) : 0u;
      w[k] = pack4_i8(b[0], b[1], b[2], b[3]);
    }
    *reinterpret_cast<uint4*>(xq + r * ld_q + c0) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// ---------------------------------------------------------------- K3: quantize NCHW -> NHWC

// One thread per (pixel, group of 4 output channels): reads are coalesced along W for each
// channel plane, writes are one 32-bit word per thread.
__global__ void quantize_nchw_nhwc_kernel(const float* __restrict__ x, int64_t n, int64_t c, int64_t hw,
                                          QuantScale q, int8_t* __restrict__ xq, int64_t cp) {
  const int64_t g4 = cp / 4;
  const int64_t total = n * hw * g4;
  for (int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; idx < total;
       idx += int64_t(gridDim.x) * blockDim.x) {
    // pixel-fastest order so neighbouring threads read neighbouring pixels
    const int64_t pix_all = n * hw;
    const int64_t grp = idx / pix_all;
    const int64_t pix = idx - grp * pix_all;
    const int64_t img = pix / hw;
    const int64_t p = pix - img * hw;
    uint32_t b[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int64_t ch = grp * 4 + e;
      b[e] = ch < c ? quant_byte(__ldg(x + (img * c + ch) * hw + p), q) : 0u;
    }
    *reinterpret_cast<uint32_t*>(xq + pix * cp + grp * 4) = pack4_i8(b[0], b[1], b[2], b[3]);
  }
}

// Quantization of an NCHW f32 image batch with at most 4 channels into the row-expanded int8
// layout read by the ROW4 convolution gather: for every image row, `entries` 16-byte entries, entry
// e holding pixels e - pad .. e - pad + 3 with 4 channels each (zero outside the image and for
// channels >= c).  One thread per entry; neighbouring threads read neighbouring pixels.
constexpr int Q4_ROWS = 4;   // image rows a thread has in flight (their loads issued before any math)

template <int S>
__global__ void quantize_nchw_row4_kernel(const float* __restrict__ x, int n, int c, int h, int w, QuantScale q,
                                          int8_t* __restrict__ xq, int entries, int pad) {
  // blockIdx.y: groups of Q4_ROWS image rows (strided over gridDim.y); each warp of the block: 32
  // entries of those rows.  Entry e holds pixels S*e - pad .. S*e - pad + 3: lane l quantizes the S
  // pixels that start its entry (lanes 0 .. 4/S - 2 also those of the entries after the warp) and
  // the entries are assembled from 4/S neighbouring lanes by shuffles.  All loads of the Q4_ROWS
  // rows are issued before the first is used, so a thread keeps several rows of reads in flight.
  constexpr int L = 4 / S;
  const int lane = threadIdx.x & 31;
  const int e0 = (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 32;
  if (e0 >= entries) return;   // warp-uniform
  const int64_t rows = int64_t(n) * h;
  const int64_t plane = int64_t(h) * w;
  const int x_own = S * (e0 + lane) - pad;
  const int x_extra = S * (e0 + 32 + lane) - pad;
  const bool has_extra = lane < L - 1;
  for (int64_t row0 = int64_t(blockIdx.y) * Q4_ROWS; row0 < rows; row0 += int64_t(gridDim.y) * Q4_ROWS) {
    float v[Q4_ROWS][4 * S], t[Q4_ROWS][4 * S];
#pragma unroll
    for (int r = 0; r < Q4_ROWS; ++r) {
      const int64_t row = row0 + r;
      const bool row_ok = row < rows;
      const int img = row_ok ? static_cast<int>(row / h) : 0;
      const int y = row_ok ? static_cast<int>(row - int64_t(img) * h) : 0;
      const float* base = x + (int64_t(img) * c * h + y) * w;
#pragma unroll
      for (int j = 0; j < S; ++j)
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          const int xo = x_own + j, xe = x_extra + j;
          v[r][4 * j + ch] = (row_ok && ch < c && xo >= 0 && xo < w) ? __ldg(base + ch * plane + xo) : 0.0f;
          t[r][4 * j + ch] =
              (row_ok && has_extra && ch < c && xe >= 0 && xe < w) ? __ldg(base + ch * plane + xe) : 0.0f;
        }
    }
#pragma unroll
    for (int r = 0; r < Q4_ROWS; ++r) {
      const int64_t row = row0 + r;
      uint32_t own[S], extra[S];
      {
        uint32_t b[4 * S], d[4 * S];
        requant_x2<4 * S>(v[r], q.s, q.rcp, q.c127, b);
        requant_x2<4 * S>(t[r], q.s, q.rcp, q.c127, d);
#pragma unroll
        for (int j = 0; j < S; ++j) {
          own[j] = pack4_i8(b[4 * j], b[4 * j + 1], b[4 * j + 2], b[4 * j + 3]);
          extra[j] = pack4_i8(d[4 * j], d[4 * j + 1], d[4 * j + 2], d[4 * j + 3]);
        }
      }
      uint32_t word[4];
#pragma unroll
      for (int k = 0; k < L; ++k) {
#pragma unroll
        for (int j = 0; j < S; ++j) {
          const uint32_t down = __shfl_down_sync(0xffffffffu, own[j], k);
          const uint32_t tail = __shfl_sync(0xffffffffu, extra[j], (lane + k - 32) & 31);
          word[k * S + j] = lane + k < 32 ? down : tail;
        }
      }
      if (row < rows && e0 + lane < entries)
        reinterpret_cast<uint4*>(xq)[row * entries + e0 + lane] = make_uint4(word[0], word[1], word[2], word[3]);
    }
  }
}

// ---------------------------------------------------------------- K5: max pooling (NHWC)

// Where an output pixel's int8 channels go: rows of `ld` bytes (cp == 0), or the chunk-planar,
// zero-padded layout (MIRA_LAYOUT_CP) of an [n, oh, ow, c] activation, `chunk` bytes apart per
// 16 channels.
struct I8Dst {
  int8_t* base;
  int64_t ld;
  int cp, guard;
  int64_t chunk;
  __device__ __forceinline__ int8_t* pixel(int img, int oy, int ox, int oh, int ow, int64_t pix) const {
    return base + (cp ? (guard + (static_cast<int64_t>(img) * (oh + 2) + oy + 1) * (ow + 2) + ox + 1) * 16 : pix * ld);
  }
  // byte offset of channel ch (a multiple of 4 stays inside one 16-byte chunk with its 3 followers)
  __device__ __forceinline__ int64_t channel(int ch) const { return static_cast<int64_t>(ch >> 4) * chunk + (ch & 15); }
};

// f32 input.  blockIdx.y: output rows (n * oh, strided over gridDim.y); threadIdx.x: groups of 4
// channels (strided over blockDim.x), threadIdx.y + blockIdx.x * blockDim.y: the output column.
// Padding pixels take `pad_value` (the reference pads with -inf before pooling).  Writes f32
// and/or the quantized int8 value.
__global__ void maxpool_f32_kernel(const float* __restrict__ x, int n, int h, int w, int c, int64_t ldc,
                                   int size, int stride, int pad, float pad_value, int oh, int ow,
                                   float* __restrict__ out, int64_t ldo, I8Dst o8, QuantScale q) {
  const int c4 = (c + 3) / 4;
  const int ox = blockIdx.x * blockDim.y + threadIdx.y;
  if (ox >= ow) return;
  const bool vec = (c % 4) == 0 && (ldc % 4) == 0;
  const int64_t rows = int64_t(n) * oh;
  for (int64_t orow = blockIdx.y; orow < rows; orow += gridDim.y) {
    const int img = static_cast<int>(orow / oh);
    const int oy = static_cast<int>(orow - int64_t(img) * oh);
    const int64_t pix = orow * ow + ox;
    for (int cg = threadIdx.x; cg < c4; cg += blockDim.x) {
      float mx[4];
      bool first = true;
      for (int i = 0; i < size; ++i) {
        const int iy = oy * stride + i - pad;
        for (int j = 0; j < size; ++j) {
          const int ix = ox * stride + j - pad;
          float v[4];
          if (iy < 0 || iy >= h || ix < 0 || ix >= w) {
            v[0] = v[1] = v[2] = v[3] = pad_value;
          } else {
            const float* src = x + (int64_t(img) * h * w + int64_t(iy) * w + ix) * ldc + cg * 4;
            if (vec) {
              const float4 t = __ldg(reinterpret_cast<const float4*>(src));
              v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
            } else {
#pragma unroll
              for (int e = 0; e < 4; ++e) v[e] = (cg * 4 + e < c) ? src[e] : 0.0f;
            }
          }
#pragma unroll
          for (int e = 0; e < 4; ++e) mx[e] = first ? v[e] : np_maximum(mx[e], v[e]);
          first = false;
        }
      }
      if (out != nullptr) {
        float* dst = out + pix * ldo + cg * 4;
        if (vec && (ldo % 4) == 0) {
          *reinterpret_cast<float4*>(dst) = make_float4(mx[0], mx[1], mx[2], mx[3]);
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (cg * 4 + e < c) dst[e] = mx[e];
        }
      }
      if (o8.base != nullptr) {
        uint32_t b[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) b[e] = (cg * 4 + e < c) ? quant_byte(mx[e], q) : 0u;
        *reinterpret_cast<uint32_t*>(o8.pixel(img, oy, ox, oh, ow, pix) + o8.channel(cg * 4)) =
            pack4_i8(b[0], b[1], b[2], b[3]);
      }
    }
  }
}

// 3x3 windows, 4 channels per thread (c % 4 == 0, 16-byte aligned rows): the same maxima as
// maxpool_f32_kernel with far fewer instructions (the general kernel spends most of its issue
// slots on per-tap 64-bit index arithmetic and checks): three row pointers computed once, no
// bounds checks for windows inside the image, the nine 16-byte loads in flight together, and
// the packed requantization.  max.NaN is commutative (NaN wins, +0 over -0), so the order of the
// maxima cannot change a result.
__global__ void maxpool3_f32_kernel(const float* __restrict__ x, int n, int h, int w, int c, int64_t ldc, int stride,
                                    int pad, float pad_value, int oh, int ow, float* __restrict__ out, int64_t ldo,
                                    I8Dst o8, QuantScale q) {
  const int c4 = c >> 2;
  const int ox = blockIdx.x * blockDim.y + threadIdx.y;
  if (ox >= ow) return;
  const int ix0 = ox * stride - pad;
  const bool cols_in = ix0 >= 0 && ix0 + 2 < w;
  const int64_t rows = int64_t(n) * oh;
  for (int64_t orow = blockIdx.y; orow < rows; orow += gridDim.y) {
    const int img = static_cast<int>(orow / oh);
    const int oy = static_cast<int>(orow - int64_t(img) * oh);
    const int iy0 = oy * stride - pad;
    const bool inside = cols_in && iy0 >= 0 && iy0 + 2 < h;
    const float* r0 = x + (int64_t(img) * h + iy0) * w * ldc + int64_t(ix0) * ldc;   // window's top-left pixel
    const int64_t rs = int64_t(w) * ldc;
    float* q0 = out != nullptr ? out + (orow * ow + ox) * ldo : nullptr;
    int8_t* q8 = o8.base != nullptr ? o8.pixel(img, oy, ox, oh, ow, orow * ow + ox) : nullptr;
    for (int cg = threadIdx.x; cg < c4; cg += blockDim.x) {
      float4 t[9];
      if (inside) {
#pragma unroll
        for (int i = 0; i < 3; ++i)
#pragma unroll
          for (int j = 0; j < 3; ++j)
            t[3 * i + j] = __ldg(reinterpret_cast<const float4*>(r0 + i * rs + j * ldc + 4 * cg));
      } else {
#pragma unroll
        for (int i = 0; i < 3; ++i)
#pragma unroll
          for (int j = 0; j < 3; ++j) {
            const bool in = iy0 + i >= 0 && iy0 + i < h && ix0 + j >= 0 && ix0 + j < w;
            t[3 * i + j] = in ? __ldg(reinterpret_cast<const float4*>(r0 + i * rs + j * ldc + 4 * cg))
                              : make_float4(pad_value, pad_value, pad_value, pad_value);
          }
      }
      float mx[4] = {t[0].x, t[0].y, t[0].z, t[0].w};
#pragma unroll
      for (int k = 1; k < 9; ++k) {
        mx[0] = np_maximum(mx[0], t[k].x);
        mx[1] = np_maximum(mx[1], t[k].y);
        mx[2] = np_maximum(mx[2], t[k].z);
        mx[3] = np_maximum(mx[3], t[k].w);
      }
      if (q0 != nullptr)
        *reinterpret_cast<float4*>(q0 + 4 * cg) = make_float4(mx[0], mx[1], mx[2], mx[3]);
      if (q8 != nullptr) {
        uint32_t b[4];
        requant_x2<4>(mx, q.s, q.rcp, q.c127, b);
        *reinterpret_cast<uint32_t*>(q8 + o8.channel(4 * cg)) = pack4_i8(b[0], b[1], b[2], b[3]);
      }
    }
  }
}

// int8 input (already quantized with the output's scale): quantize(max(x)) == max(quantize(x)),
// so pooling the int8 values gives the reference's int8 result.  One thread per 16 channels.
__global__ void maxpool_i8_kernel(const int8_t* __restrict__ x, int n, int h, int w, int64_t cp, int size,
                                  int stride, int pad, int8_t pad_q, int oh, int ow, int8_t* __restrict__ out,
                                  int64_t ldo) {
  const int64_t c16 = cp / 16;
  const int64_t total = int64_t(n) * oh * ow * c16;
  const uint32_t padw = 0x01010101u * static_cast<uint8_t>(pad_q);
  for (int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; idx < total;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int64_t cg = idx % c16;
    const int64_t pix = idx / c16;
    const int img = static_cast<int>(pix / (int64_t(oh) * ow));
    const int rem = static_cast<int>(pix - int64_t(img) * oh * ow);
    const int oy = rem / ow, ox = rem - (rem / ow) * ow;
    uint4 mx = make_uint4(0x81818181u, 0x81818181u, 0x81818181u, 0x81818181u);  // -127
    for (int i = 0; i < size; ++i) {
      const int iy = oy * stride + i - pad;
      for (int j = 0; j < size; ++j) {
        const int ix = ox * stride + j - pad;
        uint4 v;
        if (iy < 0 || iy >= h || ix < 0 || ix >= w) {
          v = make_uint4(padw, padw, padw, padw);
        } else {
          v = __ldg(reinterpret_cast<const uint4*>(x + (int64_t(img) * h * w + int64_t(iy) * w + ix) * cp) + cg);
        }
        mx.x = __vmaxs4(mx.x, v.x);
        mx.y = __vmaxs4(mx.y, v.y);
        mx.z = __vmaxs4(mx.z, v.z);
        mx.w = __vmaxs4(mx.w, v.w);
      }
    }
    reinterpret_cast<uint4*>(out + pix * ldo)[cg] = mx;
  }
}

// ---------------------------------------------------------------- K5: mean over H*W (NHWC)

// NumPy's float32 pairwise summation (numpy/_core/src/umath/loops_utils.h.src, pairwise_sum):
// below 8 elements a plain loop; up to 128 eight interleaved partial sums combined as
// ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) plus a sequential tail; above 128 a split at
// n/2 rounded down to a multiple of 8.
__device__ float pairwise_block(const float* __restrict__ x, int n, int64_t stride) {
  if (n < 8) {
    float r = 0.0f;
    for (int i = 0; i < n; ++i) r = __fadd_rn(r, x[i * stride]);
    return r;
  }
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = x[j * stride];
  int i = 8;
  for (; i < n - (n % 8); i += 8) {
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = __fadd_rn(acc[j], x[(i + j) * stride]);
  }
  float r = __fadd_rn(__fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3])),
                      __fadd_rn(__fadd_rn(acc[4], acc[5]), __fadd_rn(acc[6], acc[7])));
  for (; i < n; ++i) r = __fadd_rn(r, x[i * stride]);
  return r;
}

__device__ float pairwise_sum(const float* __restrict__ x, int n, int64_t stride) {
  if (n <= 128) return pairwise_block(x, n, stride);
  int n2 = n / 2;
  n2 -= n2 % 8;
  return __fadd_rn(pairwise_sum(x, n2, stride), pairwise_sum(x + n2 * stride, n - n2, stride));
}

__global__ void mean_hw_kernel(const float* __restrict__ x, int n, int hw, int c, int64_t ldc,
                               float* __restrict__ out, int8_t* __restrict__ out_i8, int64_t ld_i8, QuantScale q) {
  const int64_t total = int64_t(n) * c;
  const float count = static_cast<float>(hw);
  for (int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; idx < total;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int img = static_cast<int>(idx / c);
    const int ch = static_cast<int>(idx - int64_t(img) * c);
    const float s = pairwise_sum(x + int64_t(img) * hw * ldc + ch, hw, ldc);
    const float mean = __fdiv_rn(s, count);
    if (out != nullptr) out[idx] = mean;
    if (out_i8 != nullptr) out_i8[int64_t(img) * ld_i8 + ch] = static_cast<int8_t>(quant_byte(mean, q) & 0xff);
  }
}

// zero the int8 padding columns [c, ld_i8) of each row
__global__ void zero_pad_cols_kernel(int8_t* __restrict__ y, int64_t rows, int64_t c, int64_t ld) {
  const int64_t w = ld - c;
  const int64_t total = rows * w;
  for (int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; idx < total;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = idx / w;
    y[r * ld + c + (idx - r * w)] = 0;
  }
}

// ---------------------------------------------------------------- split-K finish

// Adds the int32 partial sums of a split-K GEMM (exact: the full sum fits int32) and applies the
// quantized matmul's epilogue element by element: exact dequant (f64 fallback), steps, f32 and
// int8 outputs (int8 padding columns [N, ld_i8) written as 0).
struct SplitkFinishParams {
  const int32_t* ws;
  int splits;
  int64_t slice;            // elements per partial slice (M * N)
  int M, N;
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
  QuantScale q;
};

__global__ void qgemm_splitk_finish_kernel(const SplitkFinishParams p) {
  const int width = (p.out_i8 != nullptr && p.ld_i8 > p.N) ? static_cast<int>(p.ld_i8) : p.N;
  const int64_t total = int64_t(p.M) * width;
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < total; e += int64_t(gridDim.x) * blockDim.x) {
    const int m = static_cast<int>(e / width), n = static_cast<int>(e - int64_t(m) * width);
    if (n >= p.N) {
      p.out_i8[int64_t(m) * p.ld_i8 + n] = 0;
      continue;
    }
    const int64_t idx = int64_t(m) * p.N + n;
    int32_t acc = 0;
    for (int s = 0; s < p.splits; ++s) acc += __ldg(p.ws + s * p.slice + idx);
    float y;
    if (p.scale64 != nullptr) {
      if (!dequant_fast(acc, __ldg(p.scale_hi + n), __ldg(p.scale_lo + n), y))
        y = __double2float_rn(static_cast<double>(acc) * __ldg(p.scale64 + n));
    } else {
      const float rs = __ldg(p.row_scale + m), cs = __ldg(p.col_scale + n);
      float hi, lo;
      split_rowcol(rs, cs, hi, lo);
      if (!dequant_fast(acc, hi, lo, y))
        y = __double2float_rn(static_cast<double>(acc) * (static_cast<double>(rs) * static_cast<double>(cs)));
    }
    for (int s = 0; s < p.n_steps; ++s) {
      const mira_epi_step& st = p.steps[s];
      if (st.operand == MIRA_OPND_NONE) {
        y = apply_unary(st.op, y);
        continue;
      }
      float o = st.scalar;
      if (st.operand == MIRA_OPND_CHANNEL) o = __ldg(st.ptr + n);
      else if (st.operand == MIRA_OPND_ROW) o = __ldg(st.ptr + m);
      else if (st.operand == MIRA_OPND_FULL) o = __ldg(st.ptr + int64_t(m) * st.ld + n);
      y = st.swapped ? apply_binary(st.op, o, y) : apply_binary(st.op, y, o);
    }
    if (p.out_f32 != nullptr) p.out_f32[int64_t(m) * p.ld_f32 + n] = y;
    if (p.out_i8 != nullptr) p.out_i8[int64_t(m) * p.ld_i8 + n] = static_cast<int8_t>(quant_byte(y, p.q) & 0xff);
  }
}

// ---------------------------------------------------------------- K4: depthwise f32 conv (NHWC)

struct DwParams {
  int n, h, w, c, oh, ow, kh, kw, sh, sw, ph, pw, dh, dw;
  int n_steps;
  mira_epi_step steps[MIRA_EPI_MAX_STEPS];
  float* out_f32;
  int64_t ld_f32;
  int8_t* out_i8;
  int64_t ld_i8;
  QuantScale q;
};

// One thread per (output pixel, channel): per-tap products added in (i, j) order starting from
// 0 (reference _conv2d_ref ops.py:272-275: one einsum term per tap over the zero-padded input,
// `acc +=`), then the epilogue.  Threads run channel-fastest so x and w reads coalesce.  This is the
// path for channel counts that are not a multiple of 4 and for unaligned buffers.
__global__ void dwconv_kernel(const float* __restrict__ x, const float* __restrict__ wt, const __grid_constant__ DwParams p) {
  const int64_t total = int64_t(p.n) * p.oh * p.ow * p.c;
  for (int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; idx < total;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int ch = static_cast<int>(idx % p.c);
    const int64_t pix = idx / p.c;
    const int img = static_cast<int>(pix / (int64_t(p.oh) * p.ow));
    const int rem = static_cast<int>(pix - int64_t(img) * p.oh * p.ow);
    const int oy = rem / p.ow, ox = rem - (rem / p.ow) * p.ow;
    float acc = 0.0f;
    for (int i = 0; i < p.kh; ++i) {
      const int iy = oy * p.sh - p.ph + i * p.dh;
      for (int j = 0; j < p.kw; ++j) {
        const int ix = ox * p.sw - p.pw + j * p.dw;
        // a padded tap still adds 0 * w, as the zero-padded reference does (NaN for an inf weight)
        const bool in = iy >= 0 && iy < p.h && ix >= 0 && ix < p.w;
        const float xv = in ? __ldg(x + ((int64_t(img) * p.h + iy) * p.w + ix) * p.c + ch) : 0.0f;
        acc = __fadd_rn(acc, __fmul_rn(xv, __ldg(wt + (i * p.kw + j) * p.c + ch)));
      }
    }
    float v = acc;
    for (int s = 0; s < p.n_steps; ++s) {
      const mira_epi_step& st = p.steps[s];
      if (st.operand == MIRA_OPND_NONE) {
        v = apply_unary(st.op, v);
        continue;
      }
      float o;
      if (st.operand == MIRA_OPND_SCALAR) o = st.scalar;
      else if (st.operand == MIRA_OPND_CHANNEL) o = __ldg(st.ptr + ch);
      else if (st.operand == MIRA_OPND_ROW) o = st.ptr[pix];
      else o = st.ptr[pix * st.ld + ch];
      v = st.swapped ? apply_binary(st.op, o, v) : apply_binary(st.op, v, o);
    }
    if (p.out_f32 != nullptr) p.out_f32[pix * p.ld_f32 + ch] = v;
    if (p.out_i8 != nullptr) p.out_i8[pix * p.ld_i8 + ch] = static_cast<int8_t>(quant_byte(v, p.q) & 0xff);
  }
}

// Apply `expr` (of a, the value, and b, the operand) to every value of a thread's tile, with
// the operand order of step `st` (b op a when swapped).
#define DW_BINARY(SWAP, expr)                                                             \
  _Pragma("unroll") for (int t = 0; t < T; ++t) _Pragma("unroll") for (int e = 0; e < 4; ++e) { \
    const float a = (SWAP) ? o[t][e] : v[t][e];                                           \
    const float b = (SWAP) ? v[t][e] : o[t][e];                                           \
    v[t][e] = (expr);                                                                     \
  }

// The epilogue of T adjacent output pixels (pix0 ...) x 4 channels (4 * cg ...) and the 16-byte
// f32 / 4-byte int8 stores of the first `nvalid` pixels.  Each step's operand kind and op are
// decoded once for the whole tile (they are uniform across the grid), not per value.
template <int T>
__device__ __forceinline__ void dw_epilogue_tile(const DwParams& p, int64_t pix0, int cg, int nvalid,
                                                 float (&v)[T][4]) {
  for (int s = 0; s < p.n_steps; ++s) {
    const mira_epi_step& st = p.steps[s];
    if (st.operand == MIRA_OPND_NONE) {
      if (st.op == MIRA_EPI_RELU) {
#pragma unroll
        for (int t = 0; t < T; ++t)
#pragma unroll
          for (int e = 0; e < 4; ++e) v[t][e] = np_maximum(v[t][e], 0.0f);
      } else {
#pragma unroll
        for (int t = 0; t < T; ++t)
#pragma unroll
          for (int e = 0; e < 4; ++e) v[t][e] = apply_unary(st.op, v[t][e]);
      }
      continue;
    }
    float o[T][4];
    if (st.operand == MIRA_OPND_SCALAR || st.operand == MIRA_OPND_CHANNEL) {
      float4 c4 = make_float4(st.scalar, st.scalar, st.scalar, st.scalar);
      if (st.operand == MIRA_OPND_CHANNEL) c4 = __ldg(reinterpret_cast<const float4*>(st.ptr + 4 * cg));
#pragma unroll
      for (int t = 0; t < T; ++t) { o[t][0] = c4.x; o[t][1] = c4.y; o[t][2] = c4.z; o[t][3] = c4.w; }
    } else {
#pragma unroll
      for (int t = 0; t < T; ++t) {
        const int64_t pix = pix0 + (t < nvalid ? t : 0);
        if (st.operand == MIRA_OPND_ROW) {
          o[t][0] = o[t][1] = o[t][2] = o[t][3] = st.ptr[pix];
        } else {
          const float4 f = __ldg(reinterpret_cast<const float4*>(st.ptr + pix * st.ld + 4 * cg));
          o[t][0] = f.x; o[t][1] = f.y; o[t][2] = f.z; o[t][3] = f.w;
        }
      }
    }
    // add, mul, maximum and minimum are commutative (np_maximum/np_minimum up to the sign of a
    // zero, which quantizes alike), so only sub and div look at the operand order
    const bool sw = st.swapped != 0;
    switch (st.op) {
      case MIRA_EPI_ADD: DW_BINARY(false, __fadd_rn(a, b)); break;
      case MIRA_EPI_SUB: if (sw) { DW_BINARY(true, __fsub_rn(a, b)); } else { DW_BINARY(false, __fsub_rn(a, b)); } break;
      case MIRA_EPI_MUL: DW_BINARY(false, __fmul_rn(a, b)); break;
      case MIRA_EPI_DIV: if (sw) { DW_BINARY(true, __fdiv_rn(a, b)); } else { DW_BINARY(false, __fdiv_rn(a, b)); } break;
      case MIRA_EPI_MAXIMUM: DW_BINARY(false, np_maximum(a, b)); break;
      case MIRA_EPI_MINIMUM: DW_BINARY(false, np_minimum(a, b)); break;
      default: break;
    }
  }
#pragma unroll
  for (int t = 0; t < T; ++t) {
    if (t >= nvalid) break;
    const int64_t pix = pix0 + t;
    if (p.out_f32 != nullptr)
      *reinterpret_cast<float4*>(p.out_f32 + pix * p.ld_f32 + 4 * cg) = make_float4(v[t][0], v[t][1], v[t][2], v[t][3]);
    if (p.out_i8 != nullptr) {
      uint32_t b[4];
      requant_x2<4>(v[t], p.q.s, p.q.rcp, p.q.c127, b);
      *reinterpret_cast<uint32_t*>(p.out_i8 + pix * p.ld_i8 + 4 * cg) = pack4_i8(b[0], b[1], b[2], b[3]);
    }
  }
}
#undef DW_BINARY

// Four channels per thread (c % 4 == 0): blockIdx.y walks output rows (n * oh, strided over
// gridDim.y), threadIdx.x groups of 4 channels (strided over blockDim.x), threadIdx.y +
// blockIdx.x * blockDim.y the output column.  Inputs, weights and operands move as 16-byte vectors;
// the per-tap sums run two channels per packed f32x2 add, each lane rounded like the scalar kernel
// (product, then sum, per tap in (i, j) order, padded taps as 0 * w).
__global__ void dwconv4_kernel(const float* __restrict__ x, const float* __restrict__ wt, const __grid_constant__ DwParams p) {
  const int c4 = p.c >> 2;
  const int ox = blockIdx.x * blockDim.y + threadIdx.y;
  if (ox >= p.ow) return;
  const int64_t rows = int64_t(p.n) * p.oh;
  for (int64_t orow = blockIdx.y; orow < rows; orow += gridDim.y) {
    const int img = static_cast<int>(orow / p.oh);
    const int oy = static_cast<int>(orow - int64_t(img) * p.oh);
    const int64_t pix = orow * p.ow + ox;
    for (int cg = threadIdx.x; cg < c4; cg += blockDim.x) {
      f2_t a01 = f2(0.0f, 0.0f), a23 = f2(0.0f, 0.0f);
      for (int i = 0; i < p.kh; ++i) {
        const int iy = oy * p.sh - p.ph + i * p.dh;
        const bool row_in = iy >= 0 && iy < p.h;
        const float* xrow = x + ((int64_t(img) * p.h + (row_in ? iy : 0)) * p.w) * p.c + 4 * cg;
        const float* wrow = wt + int64_t(i) * p.kw * p.c + 4 * cg;
        for (int j = 0; j < p.kw; ++j) {
          const int ix = ox * p.sw - p.pw + j * p.dw;
          const float4 xv = row_in && ix >= 0 && ix < p.w ? __ldg(reinterpret_cast<const float4*>(xrow + int64_t(ix) * p.c))
                                                          : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          const float4 wv = __ldg(reinterpret_cast<const float4*>(wrow + int64_t(j) * p.c));
          // scalar products (a packed mul.rn.f32x2 would be fused with the packed add into an fma)
          a01 = f2_add(a01, f2(__fmul_rn(xv.x, wv.x), __fmul_rn(xv.y, wv.y)));
          a23 = f2_add(a23, f2(__fmul_rn(xv.z, wv.z), __fmul_rn(xv.w, wv.w)));
        }
      }
      float v[1][4];
      f2_split(a01, v[0][0], v[0][1]);
      f2_split(a23, v[0][2], v[0][3]);
      dw_epilogue_tile<1>(p, pix, cg, 1, v);
    }
  }
}

// 3x3 depthwise, dilation 1, stride S (1 or 2), c % 4 == 0: each thread computes OXT adjacent
// output columns of one output row for 4 channels.  The taps are unrolled so one input row's
// (OXT - 1) * S + 3 16-byte loads are in flight together, and each loaded column feeds every
// output column whose window covers it.  Per output the order is the reference's: (i, j) taps
// ascending, each product rounded, then added to the running sum from 0; padded taps add 0 * w.
// Four blocks per SM (at most 64 registers, a few bytes spilled): the kernel is latency-bound, and
// the extra warps outweigh the loads the compiler can no longer hoist (measured on MobileNetV2's
// depthwise layers per batch of 256: 3.45 ms at 122 registers, 2.54 ms at 3 blocks, 2.40 ms at 4).
template <int S, int OXT>
__global__ void __launch_bounds__(256, 4) dwconv3x3_kernel(const float* __restrict__ x, const float* __restrict__ wt,
                                                        const __grid_constant__ DwParams p) {
  constexpr int NIN = (OXT - 1) * S + 3;
  const int c4 = p.c >> 2;
  const int ox0 = (blockIdx.x * blockDim.y + threadIdx.y) * OXT;
  if (ox0 >= p.ow) return;
  const int64_t rows = int64_t(p.n) * p.oh;
  for (int64_t orow = blockIdx.y; orow < rows; orow += gridDim.y) {
    const int img = static_cast<int>(orow / p.oh);
    const int oy = static_cast<int>(orow - int64_t(img) * p.oh);
    for (int cg = threadIdx.x; cg < c4; cg += blockDim.x) {
      f2_t acc[OXT][2];
#pragma unroll
      for (int t = 0; t < OXT; ++t) acc[t][0] = acc[t][1] = f2(0.0f, 0.0f);
#pragma unroll
      for (int i = 0; i < 3; ++i) {
        const int iy = oy * S - p.ph + i;
        const bool row_in = iy >= 0 && iy < p.h;
        const float* xrow = x + ((int64_t(img) * p.h + (row_in ? iy : 0)) * p.w) * p.c + 4 * cg;
        float4 xin[NIN];
#pragma unroll
        for (int u = 0; u < NIN; ++u) {
          const int ix = ox0 * S - p.pw + u;
          xin[u] = row_in && ix >= 0 && ix < p.w ? __ldg(reinterpret_cast<const float4*>(xrow + int64_t(ix) * p.c))
                                                  : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        float4 wv[3];
#pragma unroll
        for (int j = 0; j < 3; ++j) wv[j] = __ldg(reinterpret_cast<const float4*>(wt + (i * 3 + j) * p.c + 4 * cg));
#pragma unroll
        for (int t = 0; t < OXT; ++t)
#pragma unroll
          for (int j = 0; j < 3; ++j) {
            const float4 xv = xin[t * S + j];
            // scalar products (a packed mul.rn.f32x2 would be fused with the packed add into an fma)
            acc[t][0] = f2_add(acc[t][0], f2(__fmul_rn(xv.x, wv[j].x), __fmul_rn(xv.y, wv[j].y)));
            acc[t][1] = f2_add(acc[t][1], f2(__fmul_rn(xv.z, wv[j].z), __fmul_rn(xv.w, wv[j].w)));
          }
      }
      float v[OXT][4];
#pragma unroll
      for (int t = 0; t < OXT; ++t) {
        f2_split(acc[t][0], v[t][0], v[t][1]);
        f2_split(acc[t][1], v[t][2], v[t][3]);
      }
      dw_epilogue_tile<OXT>(p, orow * p.ow + ox0, cg, p.ow - ox0 < OXT ? p.ow - ox0 : OXT, v);
    }
  }
}

// ---------------------------------------------------------------- K4c: W8A8 depthwise convolution

// The opt-in int8 depthwise mode: reference _qconv2d_ref (ops.py:630-634) with groups = channels.
// Its per-tap f32 einsum sums of int8 products are exact integers (|sum| <= kh * kw * 127^2 < 2^24),
// so the device sums int32 products; then the per-channel dequant y = f32(f64(acc) * S[c]) (exact,
// as in the GEMM epilogue) and the depthwise epilogue.  Inputs: int8 NHWC pixels `ldx` bytes apart
// (channels padded with zeros), weights as int32 words [kh * kw][c / 4] (4 channels' int8 taps).

__device__ __forceinline__ int32_t sext_byte(uint32_t v, int e) {
  // byte e of v, sign-extended
  return static_cast<int32_t>(static_cast<int8_t>(static_cast<uint8_t>(v >> (8 * e))));
}

struct QdwScales {
  const float* hi;
  const float* lo;
  const double* s64;
};

template <int T>
__device__ __forceinline__ void qdw_dequant(const int32_t (&acc)[T][4], const QdwScales& sc, int cg, float (&v)[T][4]) {
  const float4 hs = __ldg(reinterpret_cast<const float4*>(sc.hi + 4 * cg));
  const float4 ls = __ldg(reinterpret_cast<const float4*>(sc.lo + 4 * cg));
  uint32_t bad = 0, range = 0;
#pragma unroll
  for (int t = 0; t < T; ++t) dequant4_fold(reinterpret_cast<const uint32_t*>(acc[t]), hs, ls, v[t], bad, range);
  if ((bad | (range & 0xFF800000u)) != 0) {   // rare: the exact product in f64
#pragma unroll
    for (int t = 0; t < T; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) v[t][e] = __double2float_rn(static_cast<double>(acc[t][e]) * sc.s64[4 * cg + e]);
  }
}

// 3 x 3, stride S, dilation 1: 4 channels x OXT output columns per thread (as dwconv3x3_kernel).
// The taps run on dp4a: per input row, the NIN pixels' words (4 channels each) are transposed into
// one byte stream per channel (x[0][c], x[1][c], ...), the three taps of output column t are the
// stream's bytes S t .. S t + 2 (a funnel shift), and the row's three weights of channel c are one
// word (w[i][0][c], w[i][1][c], w[i][2][c], 0): one dp4a adds the three products of a row exactly
// (the fourth byte is multiplied by 0).  The int32 sums are the same as tap-by-tap products.
template <int S, int OXT>
__global__ void __launch_bounds__(256, 3) qdwconv3x3_kernel(const int8_t* __restrict__ x, int64_t ldx,
                                                         const uint32_t* __restrict__ wt, const QdwScales sc,
                                                         const __grid_constant__ DwParams p) {
  constexpr int NIN = (OXT - 1) * S + 3;
  static_assert(NIN >= 5 && NIN <= 6, "pixel window of one thread");
  const int c4 = p.c >> 2;
  const int ox0 = (blockIdx.x * blockDim.y + threadIdx.y) * OXT;
  if (ox0 >= p.ow) return;
  const int64_t rows = int64_t(p.n) * p.oh;
  for (int64_t orow = blockIdx.y; orow < rows; orow += gridDim.y) {
    const int img = static_cast<int>(orow / p.oh);
    const int oy = static_cast<int>(orow - int64_t(img) * p.oh);
    for (int cg = threadIdx.x; cg < c4; cg += blockDim.x) {
      // all three input rows' words in flight at once
      uint32_t xin[3][NIN];
#pragma unroll
      for (int i = 0; i < 3; ++i) {
        const int iy = oy * S - p.ph + i;
        const bool row_in = iy >= 0 && iy < p.h;
        const int8_t* xrow = x + (int64_t(img) * p.h + (row_in ? iy : 0)) * p.w * ldx + 4 * cg;
#pragma unroll
        for (int u = 0; u < NIN; ++u) {
          const int ix = ox0 * S - p.pw + u;
          xin[i][u] = row_in && ix >= 0 && ix < p.w ? __ldg(reinterpret_cast<const uint32_t*>(xrow + int64_t(ix) * ldx)) : 0u;
        }
      }
      int32_t acc[OXT][4];
#pragma unroll
      for (int t = 0; t < OXT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0;
#pragma unroll
      for (int i = 0; i < 3; ++i) {
        // weights of row i, one word per channel: (w[i][0][c], w[i][1][c], w[i][2][c], 0)
        const uint32_t w0 = __ldg(wt + (i * 3 + 0) * c4 + cg);
        const uint32_t w1 = __ldg(wt + (i * 3 + 1) * c4 + cg);
        const uint32_t w2 = __ldg(wt + (i * 3 + 2) * c4 + cg);
        int32_t wr[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t t01 = __byte_perm(w0, w1, c | ((4 + c) << 4));
          wr[c] = static_cast<int32_t>(__byte_perm(t01, w2, 0x0010u | ((4 + c) << 8)) & 0x00ffffffu);
        }
        // channel byte streams: lo[c] = pixels 0..3 of channel c, hi[c] = pixels 4.. of channel c
        const uint32_t* xr = xin[i];
        const uint32_t a01l = __byte_perm(xr[0], xr[1], 0x5140), a01h = __byte_perm(xr[0], xr[1], 0x7362);
        const uint32_t a23l = __byte_perm(xr[2], xr[3], 0x5140), a23h = __byte_perm(xr[2], xr[3], 0x7362);
        uint32_t lo[4], hi[4];
        lo[0] = __byte_perm(a01l, a23l, 0x5410);
        lo[1] = __byte_perm(a01l, a23l, 0x7632);
        lo[2] = __byte_perm(a01h, a23h, 0x5410);
        lo[3] = __byte_perm(a01h, a23h, 0x7632);
        if constexpr (NIN == 6) {
          const uint32_t b45l = __byte_perm(xr[4], xr[5], 0x5140), b45h = __byte_perm(xr[4], xr[5], 0x7362);
          hi[0] = b45l;
          hi[1] = b45l >> 16;
          hi[2] = b45h;
          hi[3] = b45h >> 16;
        } else {
          hi[0] = xr[4];
          hi[1] = xr[4] >> 8;
          hi[2] = xr[4] >> 16;
          hi[3] = xr[4] >> 24;
        }
#pragma unroll
        for (int t = 0; t < OXT; ++t)
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint32_t taps = t == 0 ? lo[c] : __funnelshift_r(lo[c], hi[c], 8 * S * t);
            acc[t][c] = __dp4a(static_cast<int32_t>(taps), wr[c], acc[t][c]);
          }
      }
      float v[OXT][4];
      qdw_dequant<OXT>(acc, sc, cg, v);
      dw_epilogue_tile<OXT>(p, orow * p.ow + ox0, cg, p.ow - ox0 < OXT ? p.ow - ox0 : OXT, v);
    }
  }
}

// Any kernel size, stride and dilation: one (output pixel, 4 channels) per thread.
__global__ void qdwconv4_kernel(const int8_t* __restrict__ x, int64_t ldx, const uint32_t* __restrict__ wt,
                                const QdwScales sc, const __grid_constant__ DwParams p) {
  const int c4 = p.c >> 2;
  const int ox = blockIdx.x * blockDim.y + threadIdx.y;
  if (ox >= p.ow) return;
  const int64_t rows = int64_t(p.n) * p.oh;
  for (int64_t orow = blockIdx.y; orow < rows; orow += gridDim.y) {
    const int img = static_cast<int>(orow / p.oh);
    const int oy = static_cast<int>(orow - int64_t(img) * p.oh);
    for (int cg = threadIdx.x; cg < c4; cg += blockDim.x) {
      int32_t acc[1][4] = {{0, 0, 0, 0}};
      for (int i = 0; i < p.kh; ++i) {
        const int iy = oy * p.sh - p.ph + i * p.dh;
        if (iy < 0 || iy >= p.h) continue;
        for (int j = 0; j < p.kw; ++j) {
          const int ix = ox * p.sw - p.pw + j * p.dw;
          if (ix < 0 || ix >= p.w) continue;
          const uint32_t xw = __ldg(reinterpret_cast<const uint32_t*>(x + ((int64_t(img) * p.h + iy) * p.w + ix) * ldx + 4 * cg));
          const uint32_t ww = __ldg(wt + (i * p.kw + j) * c4 + cg);
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[0][e] += sext_byte(xw, e) * sext_byte(ww, e);
        }
      }
      float v[1][4];
      qdw_dequant<1>(acc, sc, cg, v);
      dw_epilogue_tile<1>(p, orow * p.ow + ox, cg, 1, v);
    }
  }
}

// ---------------------------------------------------------------- K4b: general f32 convolution

// The patch matrix of an f32 convolution over an NHWC input: row m = output pixel (img, oy, ox),
// column (i * kw + j) * c + ch = x[img, oy * sh - ph + i * dh, ox * sw - pw + j * dw, ch], 0 in the
// padding (the reference pads with zeros, ops.py:256-263).  One warp per (pixel, tap) row of c
// values; the convolution is then the f32 matmul of this matrix with the [kh * kw * c, o] weights.
__global__ void im2col_f32_kernel(const float* __restrict__ x, int n, int h, int w, int c, int64_t ldc, int kh,
                                  int kw, int sh, int sw, int ph, int pw, int dh, int dw, int oh, int ow,
                                  float* __restrict__ out, int64_t ld_out) {
  const int lane = threadIdx.x & 31;
  const int taps = kh * kw;
  const int64_t rows = int64_t(n) * oh * ow * taps;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = blockIdx.x * int64_t(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const int tap = static_cast<int>(r % taps);
    const int64_t pix = r / taps;
    const int ox = static_cast<int>(pix % ow);
    const int64_t t2 = pix / ow;
    const int oy = static_cast<int>(t2 % oh);
    const int img = static_cast<int>(t2 / oh);
    const int i = tap / kw, j = tap - (tap / kw) * kw;
    const int iy = oy * sh - ph + i * dh, ix = ox * sw - pw + j * dw;
    float* dst = out + pix * ld_out + int64_t(tap) * c;
    if (iy >= 0 && iy < h && ix >= 0 && ix < w) {
      const float* src = x + ((int64_t(img) * h + iy) * w + ix) * ldc;
      for (int ch = lane; ch < c; ch += 32) dst[ch] = __ldg(src + ch);
    } else {
      for (int ch = lane; ch < c; ch += 32) dst[ch] = 0.0f;
    }
  }
}

// ---------------------------------------------------------------- layout changes (f32)

// NCHW -> NHWC through a 32x32 shared-memory tile per (image, 32 channels, 32 pixels).
__global__ void nchw_to_nhwc_kernel(const float* __restrict__ x, int c, int hw, float* __restrict__ y, int64_t ldc) {
  __shared__ float tile[32][33];
  const int img = blockIdx.z;
  const int c0 = blockIdx.y * 32, p0 = blockIdx.x * 32;
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int ch = c0 + k, p = p0 + threadIdx.x;
    tile[k][threadIdx.x] = (ch < c && p < hw) ? x[(int64_t(img) * c + ch) * hw + p] : 0.0f;
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int p = p0 + k, ch = c0 + threadIdx.x;
    if (p < hw && ch < c) y[(int64_t(img) * hw + p) * ldc + ch] = tile[threadIdx.x][k];
  }
}

__global__ void nhwc_to_nchw_kernel(const float* __restrict__ x, int c, int hw, int64_t ldc, float* __restrict__ y) {
  __shared__ float tile[32][33];
  const int img = blockIdx.z;
  const int c0 = blockIdx.y * 32, p0 = blockIdx.x * 32;
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int p = p0 + k, ch = c0 + threadIdx.x;
    tile[k][threadIdx.x] = (p < hw && ch < c) ? x[(int64_t(img) * hw + p) * ldc + ch] : 0.0f;
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int ch = c0 + k, p = p0 + threadIdx.x;
    if (ch < c && p < hw) y[(int64_t(img) * c + ch) * hw + p] = tile[threadIdx.x][k];
  }
}

}  // namespace mira
