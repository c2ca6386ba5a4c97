// Depthwise 3x3 convolutions (stride 1 or 2) with their input staged in shared memory by TMA.
//
// The f32 depthwise conv of MobileNetV2 (reference _conv2d_ref with groups == channels,
// ops.py:265-276) and the opt-in int8 one (_qconv2d_ref, 630-634, on such a conv) read every input
// pixel up to nine times.  Reading those taps from global memory left the kernels latency-bound
// (a few 16-byte loads in flight per thread).  Here persistent CTAs (two per SM) walk work units =
// (image, band of R output rows, chunk of CC channels): one 4-D TMA tile load brings the unit's
// input window - (R - 1) * S + 3 rows x cols_in pixels x CC channels, the padding and anything past
// the image read as zeros by the TMA unit - into one of two shared-memory buffers while the CTA
// computes the previous unit from the other.  The arithmetic and the epilogue are those of the
// unstaged kernels (memory_bound.cuh): for f32 the per-tap products added in (i, j) order from 0,
// bit for bit the reference's; for int8 exact integer sums and the exact per-channel dequant.
#pragma once
#include "memory_bound.cuh"
#include "ptx_sm100.cuh"

namespace mira {

constexpr int DWS_THREADS = 256;
constexpr uint64_t DWS_TIMEOUT_NS = 2000000000ull;

__device__ __forceinline__ void dws_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait_suspend(bar, parity, 1000000u)) {
    if (globaltimer_ns() - t0 > DWS_TIMEOUT_NS) return;
  }
}

struct DwsParams {
  DwParams p;             // shapes, epilogue steps and outputs (as the unstaged kernels)
  QdwScales sc;           // int8 only: per-channel dequant
  int rows;               // R: output rows per unit
  int cc;                 // channels per unit (a multiple of 4, 16 bytes of elements at least)
  int cols_in, rows_in;   // the unit's input window
  int tiles;              // column tiles of OXT outputs per row
  int bands, chunks, units;
  int box_bytes;          // bytes of one window (the TMA box)
  int* err;
};

// Output pixels ox0 .. ox0 + OXT - 1 of output row r of the unit, channels 4 cg .. 4 cg + 3 of the
// chunk, from the staged window `win` ([rows_in][cols_in][cc] elements).
template <int S, int OXT>
__device__ __forceinline__ void dws_task(const float* win, const float* __restrict__ wt, int c_abs4, int cc, int cols_in,
                                         int r, int ox0, int lcg, float (&v)[OXT][4]) {
  constexpr int NIN = (OXT - 1) * S + 3;
  f2_t acc[OXT][2];
#pragma unroll
  for (int t = 0; t < OXT; ++t) acc[t][0] = acc[t][1] = f2(0.0f, 0.0f);
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const float* row = win + ((r * S + i) * cols_in + ox0 * S) * cc + 4 * lcg;
    float4 xin[NIN];
#pragma unroll
    for (int u = 0; u < NIN; ++u) xin[u] = *reinterpret_cast<const float4*>(row + u * cc);
    float4 wv[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) wv[j] = __ldg(reinterpret_cast<const float4*>(wt) + (i * 3 + j) * c_abs4);
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
#pragma unroll
  for (int t = 0; t < OXT; ++t) {
    f2_split(acc[t][0], v[t][0], v[t][1]);
    f2_split(acc[t][1], v[t][2], v[t][3]);
  }
}

template <int S, int OXT>
__device__ __forceinline__ void dws_task(const int8_t* win, const uint32_t* __restrict__ wt, int c_abs4, int cc,
                                         int cols_in, int r, int ox0, int lcg, int32_t (&acc)[OXT][4]) {
  constexpr int NIN = (OXT - 1) * S + 3;
#pragma unroll
  for (int t = 0; t < OXT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const int8_t* row = win + ((r * S + i) * cols_in + ox0 * S) * cc + 4 * lcg;
    int32_t wv[3][4];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const uint32_t wword = __ldg(wt + (i * 3 + j) * c_abs4);
#pragma unroll
      for (int e = 0; e < 4; ++e) wv[j][e] = sext_byte(wword, e);
    }
#pragma unroll
    for (int u = 0; u < NIN; ++u) {
      const uint32_t xw = *reinterpret_cast<const uint32_t*>(row + u * cc);
      int32_t xv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) xv[e] = sext_byte(xw, e);
#pragma unroll
      for (int t = 0; t < OXT; ++t) {
        const int j = u - t * S;
        if (j < 0 || j > 2) continue;
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[t][e] += xv[e] * wv[j][e];
      }
    }
  }
}

// T = float: wt is f32 [9][c]; T = int8_t: wt is [9][c / 4] words of 4 int8 weights.
template <typename T, int S, int OXT>
__global__ void __launch_bounds__(DWS_THREADS, 2) dw_staged_kernel(const __grid_constant__ CUtensorMap map,
                                                                   const void* __restrict__ wt_raw,
                                                                   const __grid_constant__ DwsParams q) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int buf_bytes = (q.box_bytes + 127) & ~127;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * buf_bytes);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full + 2);
  const DwParams& p = q.p;
  const int tid = threadIdx.x;
  if (tid == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&map);
  }
  __syncthreads();

  auto issue = [&](int u, int b) {
    const int chunk = u % q.chunks;
    const int rest = u / q.chunks;
    const int band = rest % q.bands, img = rest / q.bands;
    mbar_arrive_expect_tx(&full[b], static_cast<uint32_t>(q.box_bytes));
    tma_load_4d(smem + b * buf_bytes, &map, chunk * q.cc, -p.pw, band * q.rows * S - p.ph, img, &full[b]);
  };

  int k = 0;
  int issued = 0;   // copies issued by thread 0 (for the drain on an abort)
  if (tid == 0 && blockIdx.x < q.units) { issue(blockIdx.x, 0); issued = 1; }
  for (int u = blockIdx.x; u < q.units; u += gridDim.x, ++k) {
    const int b = k & 1;
    if (tid == 0 && u + static_cast<int>(gridDim.x) < q.units) { issue(u + gridDim.x, b ^ 1); ++issued; }
    if (mbar_wait(&full[b], (k >> 1) & 1, abort_flag, DWS_TIMEOUT_NS)) {
      const T* win = reinterpret_cast<const T*>(smem + b * buf_bytes);
      const int chunk = u % q.chunks;
      const int rest = u / q.chunks;
      const int band = rest % q.bands, img = rest / q.bands;
      const int oy0 = band * q.rows;
      const int nrows = min(q.rows, p.oh - oy0);
      const int c0 = chunk * q.cc;
      const int ncg = q.cc >> 2;
      const int tasks = ncg * q.tiles * nrows;
      for (int t = tid; t < tasks; t += DWS_THREADS) {
        const int lcg = t % ncg;
        const int rest2 = t / ncg;
        const int tile = rest2 % q.tiles, r = rest2 / q.tiles;
        const int cg = (c0 >> 2) + lcg;
        if (4 * cg >= p.c) continue;
        const int ox0 = tile * OXT;
        float v[OXT][4];
        if constexpr (sizeof(T) == 4) {
          dws_task<S, OXT>(win, static_cast<const float*>(wt_raw) + 4 * cg, p.c >> 2, q.cc, q.cols_in, r, ox0, lcg, v);
        } else {
          int32_t acc[OXT][4];
          dws_task<S, OXT>(win, static_cast<const uint32_t*>(wt_raw) + cg, p.c >> 2, q.cc, q.cols_in, r, ox0, lcg, acc);
          qdw_dequant<OXT>(acc, q.sc, cg, v);
        }
        const int64_t pix0 = (static_cast<int64_t>(img) * p.oh + oy0 + r) * p.ow + ox0;
        dw_epilogue_tile<OXT>(p, pix0, cg, p.ow - ox0 < OXT ? p.ow - ox0 : OXT, v);
      }
    }
    __syncthreads();   // every thread is done with buffer b (and saw the same abort flag)
    if (*abort_flag) break;
  }
  if (tid == 0 && *abort_flag) {
    // let the copies still in flight land before the shared memory goes away (bounded waits)
    for (int j = max(0, k); j < issued; ++j) dws_drain(&full[j & 1], (j >> 1) & 1);
    atomicExch(q.err, 1);
  }
}

}  // namespace mira
