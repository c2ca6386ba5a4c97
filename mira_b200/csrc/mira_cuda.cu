// libmira_cuda.so: the C ABI declared in include/mira_cuda.h.  One translation unit so that the
// kernels, the device-side error record and the host wrappers share one module.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/mira_cuda.h"
#include "memory_bound.cuh"
#include "qgemm_sm100.cuh"
#include "qgemm_pair_sm100.cuh"
#include "stem_pool_sm100.cuh"
#include "dw_staged.cuh"
#include "runtime.h"
#include "sequence_ops.cuh"
#include "attention_tc.cuh"

// Set by a kernel that gave up on a bounded wait or met an impossible index; read and cleared by
// mira_cuda_sync.  One copy per device (module global).
__device__ int g_mira_kernel_error;

// Scratch of mira_cuda_qgemm_splitk_static: the split-K partial sums of one call.  A fixed module
// array (8 MiB), so that entry point allocates nothing; every call on the device shares it.
constexpr int64_t kStaticSplitkBytes = int64_t(8) << 20;
__device__ __align__(256) int32_t g_mira_splitk_scratch[kStaticSplitkBytes / sizeof(int32_t)];

namespace mira {

namespace {

constexpr int kMaxDevices = 16;
DeviceState g_devices[kMaxDevices];
int* g_err_ptr[kMaxDevices];
int32_t* g_splitk_scratch[kMaxDevices];   // device address of g_mira_splitk_scratch, per device
std::mutex g_init_mutex;
thread_local int t_device = -1;
thread_local std::string t_last_error;
std::atomic<int64_t> g_launches{0};
PFN_cuTensorMapEncodeTiled_v12000 g_encode_tiled = nullptr;
PFN_cuTensorMapEncodeIm2col_v12000 g_encode_im2col = nullptr;

int init_device(int d) {
  std::lock_guard<std::mutex> lock(g_init_mutex);
  DeviceState& st = g_devices[d];
  if (st.ready) return MIRA_CUDA_OK;
  MIRA_CUDA_TRY(cudaSetDevice(d), "cudaSetDevice");
  cudaDeviceProp prop;
  MIRA_CUDA_TRY(cudaGetDeviceProperties(&prop, d), "cudaGetDeviceProperties");
  if (prop.major != 10) {
    return set_error(MIRA_CUDA_ENODEV, "device " + std::to_string(d) + " is sm_" + std::to_string(prop.major) +
                                           std::to_string(prop.minor) + "; this library is built for sm_100a");
  }
  st.device = d;
  st.sm_count = prop.multiProcessorCount;
  st.cc_major = prop.major;
  st.cc_minor = prop.minor;
  MIRA_CUDA_TRY(cudaStreamCreateWithFlags(&st.stream, cudaStreamNonBlocking), "cudaStreamCreate");
  MIRA_CUDA_TRY(cudaStreamCreateWithFlags(&st.copy_stream, cudaStreamNonBlocking), "cudaStreamCreate(copy)");
  void* err_ptr = nullptr;
  MIRA_CUDA_TRY(cudaGetSymbolAddress(&err_ptr, g_mira_kernel_error), "cudaGetSymbolAddress(error record)");
  g_err_ptr[d] = static_cast<int*>(err_ptr);
  void* scratch = nullptr;
  MIRA_CUDA_TRY(cudaGetSymbolAddress(&scratch, g_mira_splitk_scratch), "cudaGetSymbolAddress(split-K scratch)");
  g_splitk_scratch[d] = static_cast<int32_t*>(scratch);
  const int zero = 0;
  MIRA_CUDA_TRY(cudaMemcpyToSymbol(g_mira_kernel_error, &zero, sizeof(int)), "clear error record");
  if (g_encode_tiled == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    MIRA_CUDA_TRY(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q),
                  "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
    if (q != cudaDriverEntryPointSuccess || fn == nullptr)
      return set_error(MIRA_CUDA_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
    g_encode_tiled = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  if (g_encode_im2col == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    MIRA_CUDA_TRY(cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &fn, cudaEnableDefault, &q),
                  "cudaGetDriverEntryPoint(cuTensorMapEncodeIm2col)");
    if (q != cudaDriverEntryPointSuccess || fn == nullptr)
      return set_error(MIRA_CUDA_ECUDA, "cuTensorMapEncodeIm2col is not available from the driver");
    g_encode_im2col = reinterpret_cast<PFN_cuTensorMapEncodeIm2col_v12000>(fn);
  }
  st.ready = true;
  return MIRA_CUDA_OK;
}

}  // namespace

DeviceState* current_device() {
  if (t_device < 0) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return nullptr;
    t_device = 0;
  }
  if (!g_devices[t_device].ready) {
    if (init_device(t_device) != MIRA_CUDA_OK) return nullptr;
  }
  if (cudaSetDevice(t_device) != cudaSuccess) return nullptr;
  return &g_devices[t_device];
}

int set_error(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

int cuda_error(cudaError_t e, const char* what) {
  return set_error(MIRA_CUDA_ECUDA, std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int after_launch(const char* kernel) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, kernel);
  count_launch();
  return MIRA_CUDA_OK;
}

static int* device_err_ptr() { return g_err_ptr[t_device]; }

static QuantScale make_qscale(float s) {
  QuantScale q;
  q.s = s;
  q.rcp = 1.0f / s;          // correctly rounded (IEEE division on the host)
  q.lim = 256.0f * s;        // exact (power of two)
  q.c127 = 127.0f * s;       // correctly rounded product
  return q;
}

// clip(rint(v / s), -127, 127) on the host, for constant pad values (-inf gives -127).
static uint32_t quant_byte_host(float v, float s) {
  float z = v / s;
  if (z != z) z = 0.0f;
  z = std::fmin(std::fmax(z, -127.0f), 127.0f);
  return static_cast<uint32_t>(static_cast<int32_t>(std::nearbyint(z))) & 0xffu;
}

static int grid_for(const DeviceState* dev, int64_t work, int threads) {
  int64_t blocks = (work + threads - 1) / threads;
  const int64_t cap = int64_t(dev->sm_count) * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<int>(blocks);
}

// ---------------------------------------------------------------- tensor maps

// 2-D int8 tiles for TMA: box_inner bytes of box_rows rows, swizzled (128 or 64 bytes).
static int encode_2d_i8_sw(CUtensorMap* map, const void* base, uint64_t inner_bytes, uint64_t rows, uint64_t row_stride,
                           uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return set_error(MIRA_CUDA_EINVAL, "TMA base not 16-byte aligned");
  if (row_stride % 16 != 0) return set_error(MIRA_CUDA_EINVAL, "TMA row stride not a multiple of 16 bytes");
  const cuuint64_t dims[2] = {inner_bytes, rows};
  const cuuint64_t strides[1] = {row_stride};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = g_encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                                    estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(MIRA_CUDA_ECUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  return MIRA_CUDA_OK;
}

// im2col tiles of an NHWC int8 tensor [n, h, w, cp] for a square kernel with symmetric padding:
// each load brings `bk` channels of one tap for 128 consecutive output pixels (zeros outside the
// image), the bounding box of the traversal being [-pad, dim - 1 + pad - (k - 1) * dil] per
// spatial dimension with the convolution's strides as traversal steps.
static int encode_im2col_i8(CUtensorMap* map, const void* base, int64_t n, int64_t h, int64_t w, int64_t cp,
                            int64_t k, int64_t stride_h, int64_t stride_w, int64_t pad, int64_t dil, int bk) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return set_error(MIRA_CUDA_EINVAL, "TMA base not 16-byte aligned");
  const cuuint64_t dims[4] = {uint64_t(cp), uint64_t(w), uint64_t(h), uint64_t(n)};
  const cuuint64_t strides[3] = {uint64_t(cp), uint64_t(w * cp), uint64_t(h * w * cp)};
  const int lower[2] = {int(-pad), int(-pad)};
  const int upper[2] = {int(pad - (k - 1) * dil), int(pad - (k - 1) * dil)};
  const cuuint32_t estr[4] = {1, uint32_t(stride_w), uint32_t(stride_h), 1};
  const CUresult r = g_encode_im2col(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(base), dims, strides, lower,
                                     upper, uint32_t(bk), uint32_t(QG_BM), estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                     bk == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(MIRA_CUDA_ECUDA, "cuTensorMapEncodeIm2col failed (" + std::to_string(r) + ")");
  return MIRA_CUDA_OK;
}

static int encode_2d_i8(CUtensorMap* map, const void* base, uint64_t inner_bytes, uint64_t rows, uint64_t row_stride,
                        uint32_t box_inner, uint32_t box_rows) {
  return encode_2d_i8_sw(map, base, inner_bytes, rows, row_stride, box_inner, box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
}

// ---------------------------------------------------------------- qgemm dispatch

// The kernels' division by d (1 <= d < 2^31) for dividends below 2^31 (QgDiv).
static QgDiv make_div(int64_t d) {
  uint32_t l = 0;
  while ((int64_t(1) << l) < d) ++l;
  const uint64_t mul = ((uint64_t(1) << 32) * ((uint64_t(1) << l) - uint64_t(d))) / uint64_t(d) + 1;
  return QgDiv{static_cast<uint32_t>(mul), l};
}

template <int BN, int STAGES, int AMODE, bool ROWCOL, int G, bool POOL = false, int BK = QG_BK, int RKB = 0,
          int PATCH = 0>
static int launch_qgemm_cfg(DeviceState* dev, const CUtensorMap& tmA, const CUtensorMap& tmB, const QgParams& p_in) {
  QgParams p = p_in;
  if (p.k_splits < 1) {   // no split: one K range per output tile
    p.k_splits = 1;
    p.kb_per_split = p.num_kb;
  }
  if (RKB > 0 && (p.n_tiles != 1 || p.k_splits != 1 || p.num_kb > RKB))
    return set_error(MIRA_CUDA_EINVAL, "resident-weight kernel used for a shape it does not cover");
  p.dv_ntiles = make_div(p.n_tiles);
  p.dv_mntiles = make_div(int64_t(p.m_tiles) * p.n_tiles);
  using Cfg = QgCfg<BN, STAGES, AMODE, G, POOL, BK, RKB, PATCH>;
  auto kern = qgemm_sm100_kernel<BN, STAGES, AMODE, ROWCOL, G, POOL, BK, RKB, PATCH>;
  static bool attr_set[kMaxDevices] = {};
  if (!attr_set[dev->device]) {
    MIRA_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(Cfg::SMEM)),
                  "cudaFuncSetAttribute(qgemm smem)");
    attr_set[dev->device] = true;
  }
  const int tiles = p.m_tiles * p.n_tiles * p.k_splits;
  const int grid = tiles < dev->sm_count ? tiles : dev->sm_count;
  kern<<<grid, Cfg::THREADS, Cfg::SMEM, dev->stream>>>(tmA, tmB, p);
  return after_launch("qgemm_sm100_kernel");
}

// Tile width BN and the epilogue/pipeline split: short reductions (at most 24 K-blocks of 128)
// are epilogue-bound and get 16 epilogue warps (G = 4); long ones get 8 epilogue warps and the
// shared memory goes to deeper operand pipelines.
template <int AMODE, bool ROWCOL>
static int launch_qgemm_bn(DeviceState* dev, const CUtensorMap& tmA, const CUtensorMap& tmB, QgParams& p, int bn) {
  const bool short_k = p.num_kb <= 24;
  switch (bn) {
    case 64:
      return short_k ? launch_qgemm_cfg<64, 7, AMODE, ROWCOL, 4>(dev, tmA, tmB, p)
                     : launch_qgemm_cfg<64, 8, AMODE, ROWCOL, 2>(dev, tmA, tmB, p);
    case 128:
      return short_k ? launch_qgemm_cfg<128, 5, AMODE, ROWCOL, 4>(dev, tmA, tmB, p)
                     : launch_qgemm_cfg<128, 6, AMODE, ROWCOL, 2>(dev, tmA, tmB, p);
    default:
      return short_k ? launch_qgemm_cfg<256, 3, AMODE, ROWCOL, 4>(dev, tmA, tmB, p)
                     : launch_qgemm_cfg<256, 4, AMODE, ROWCOL, 2>(dev, tmA, tmB, p);
  }
}

static int pick_bn(int64_t N) { return N <= 64 ? 64 : (N <= 128 ? 128 : 256); }

// CTA-pair GEMM (256 x 256 tiles over two SMs): on unless MIRA_CUDA_PAIR_GEMM=0.
static bool pair_gemm_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("MIRA_CUDA_PAIR_GEMM");
    return e == nullptr || std::strcmp(e, "0") != 0;
  }();
  return on;
}

template <int BN, int STAGES, bool ROWCOL, int G>
static int launch_qgemm_pair_cfg(DeviceState* dev, const CUtensorMap& tmA, const CUtensorMap& tmB,
                                 const QgParams& p_in) {
  QgParams p = p_in;
  p.k_splits = 1;
  p.kb_per_split = p.num_kb;
  p.dv_ntiles = make_div(p.n_tiles);
  p.dv_mntiles = make_div(int64_t(p.m_tiles) * p.n_tiles);
  using Cfg = Qg2Cfg<BN, STAGES, G>;
  auto kern = qgemm_pair_kernel<BN, STAGES, ROWCOL, G>;
  static bool attr_set[kMaxDevices] = {};
  if (!attr_set[dev->device]) {
    MIRA_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(Cfg::SMEM)),
                  "cudaFuncSetAttribute(qgemm pair smem)");
    attr_set[dev->device] = true;
  }
  const int tiles = int((p.M + 2 * QG_BM - 1) / (2 * QG_BM)) * p.n_tiles;
  const int pairs = dev->sm_count / 2;
  const int grid = 2 * (tiles < pairs ? tiles : pairs);
  kern<<<grid, Cfg::THREADS, Cfg::SMEM, dev->stream>>>(tmA, tmB, p);
  return after_launch("qgemm_pair_kernel");
}

// Whether a GEMM of this shape runs on CTA pairs: wide enough for 256-column tiles, unsplit, a
// long reduction (more than 24 K-blocks of 128: with shorter ones the tile is epilogue-bound and
// the single-CTA kernel with 16 epilogue warps is faster), and at least one 256 x 256 tile per SM
// pair.
static bool use_pair_gemm(const DeviceState* dev, int64_t M, int64_t N, int64_t K, int splits) {
  if (!pair_gemm_enabled() || splits > 1 || N < 256 || (K + QG_BK - 1) / QG_BK <= 24) return false;
  const int64_t tiles = ((M + 255) / 256) * ((N + 255) / 256);
  return tiles >= dev->sm_count / 2;
}

// im2col convolutions: K-blocks of 64 bytes (64-channel inputs) or 128 bytes; the stages fill
// about 144 KB, 16 epilogue warps for short reductions, 8 for long ones.
static int launch_qgemm_im2col(DeviceState* dev, const CUtensorMap& tmA, const CUtensorMap& tmB, QgParams& p, int bn,
                               int bk) {
  const bool short_k = p.num_kb * bk <= 24 * 128;
  if (bk == 64) {
    switch (bn) {
      case 64:
        // one column tile of weights (N <= 64) of at most 16 K-blocks stays in shared memory
        if (p.n_tiles == 1 && p.num_kb <= 16 && short_k)
          return launch_qgemm_cfg<64, 12, QG_A_IM2COL, false, 4, false, 64, 16>(dev, tmA, tmB, p);
        return short_k ? launch_qgemm_cfg<64, 12, QG_A_IM2COL, false, 4, false, 64>(dev, tmA, tmB, p)
                       : launch_qgemm_cfg<64, 14, QG_A_IM2COL, false, 2, false, 64>(dev, tmA, tmB, p);
      case 128:
        return short_k ? launch_qgemm_cfg<128, 9, QG_A_IM2COL, false, 4, false, 64>(dev, tmA, tmB, p)
                       : launch_qgemm_cfg<128, 10, QG_A_IM2COL, false, 2, false, 64>(dev, tmA, tmB, p);
      default:
        return short_k ? launch_qgemm_cfg<256, 6, QG_A_IM2COL, false, 4, false, 64>(dev, tmA, tmB, p)
                       : launch_qgemm_cfg<256, 7, QG_A_IM2COL, false, 2, false, 64>(dev, tmA, tmB, p);
    }
  }
  switch (bn) {
    case 64:
      return short_k ? launch_qgemm_cfg<64, 7, QG_A_IM2COL, false, 4>(dev, tmA, tmB, p)
                     : launch_qgemm_cfg<64, 8, QG_A_IM2COL, false, 2>(dev, tmA, tmB, p);
    case 128:
      return short_k ? launch_qgemm_cfg<128, 5, QG_A_IM2COL, false, 4>(dev, tmA, tmB, p)
                     : launch_qgemm_cfg<128, 6, QG_A_IM2COL, false, 2>(dev, tmA, tmB, p);
    default:
      return short_k ? launch_qgemm_cfg<256, 3, QG_A_IM2COL, false, 4>(dev, tmA, tmB, p)
                     : launch_qgemm_cfg<256, 4, QG_A_IM2COL, false, 2>(dev, tmA, tmB, p);
  }
}

// 3x3 stride-1 convolutions over the chunk-planar layout (QG_A_PATCH): per tile one bulk copy per
// 16-channel plane brings the whole input halo (w + 3 slots either side of the tile's 128 output
// slots) into one of two shared-memory buffers, and the nine taps are views of it shifted by whole
// slots; weights stream through the ring, or stay resident for a 64 x 64 conv.  Halo buffer sizes
// per input channel count (the largest image width each serves): 64 -> 16 KB (w <= 56),
// 128 -> 24 KB (w <= 28), 256 -> 41 KB (w <= 14), 512 -> 74 KB (w <= 7).
static int patch_cap(int cp) {
  switch (cp) {
    case 64: return 16384;
    case 128: return 24576;
    case 256: return 41984;
    case 512: return 75776;
    default: return 0;
  }
}

static int launch_qgemm_patch(DeviceState* dev, const int8_t* wq, int64_t ldw, int64_t o, QgParams& p) {
  const int cp = p.g.cp;
  const int64_t halo = int64_t(p.g.patch_slots) * cp;
  MIRA_CHECK_ARG(patch_cap(cp) > 0 && halo <= patch_cap(cp),
                 "no chunk-planar conv kernel for this channel count and image width");
  const int bk = cp == 64 ? 64 : 128;
  int bn = o <= 64 ? 64 : (o <= 128 ? 128 : 256);
  if (cp >= 256 && bn == 64) bn = 128;
  if (cp == 512) bn = 128;
  p.num_kb = 9 * cp / bk;
  p.m_tiles = int((p.M + QG_BM - 1) / QG_BM);
  p.n_tiles = int((o + bn - 1) / bn);
  CUtensorMap tmA, tmB;
  std::memset(&tmA, 0, sizeof(tmA));
  int rc = encode_2d_i8_sw(&tmB, wq, uint64_t(ldw), uint64_t(o), uint64_t(ldw), uint32_t(bk), uint32_t(bn),
                           bk == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != MIRA_CUDA_OK) return rc;
  switch (cp) {
    case 64:
      // 18 warps (16 epilogue warps) cap ptxas at 96 registers and spill; without an f32 output the
      // 8-warp epilogue (10 warps, no spills) is faster, with one the 16 warps hide the f32 stores
      if (bn == 64 && p.n_tiles == 1 && p.out_f32 == nullptr)
        return launch_qgemm_cfg<64, 1, QG_A_PATCH, false, 2, false, 64, 9, 16384>(dev, tmA, tmB, p);
      if (bn == 64 && p.n_tiles == 1)
        return launch_qgemm_cfg<64, 1, QG_A_PATCH, false, 4, false, 64, 9, 16384>(dev, tmA, tmB, p);
      if (bn == 64) return launch_qgemm_cfg<64, 8, QG_A_PATCH, false, 4, false, 64, 0, 16384>(dev, tmA, tmB, p);
      if (bn == 128) return launch_qgemm_cfg<128, 8, QG_A_PATCH, false, 4, false, 64, 0, 16384>(dev, tmA, tmB, p);
      return launch_qgemm_cfg<256, 6, QG_A_PATCH, false, 4, false, 64, 0, 16384>(dev, tmA, tmB, p);
    case 128:
      if (bn == 64) return launch_qgemm_cfg<64, 8, QG_A_PATCH, false, 4, false, 128, 0, 24576>(dev, tmA, tmB, p);
      if (bn == 128) return launch_qgemm_cfg<128, 6, QG_A_PATCH, false, 4, false, 128, 0, 24576>(dev, tmA, tmB, p);
      return launch_qgemm_cfg<256, 3, QG_A_PATCH, false, 4, false, 128, 0, 24576>(dev, tmA, tmB, p);
    case 256:
      if (bn == 128) return launch_qgemm_cfg<128, 5, QG_A_PATCH, false, 4, false, 128, 0, 41984>(dev, tmA, tmB, p);
      return launch_qgemm_cfg<256, 3, QG_A_PATCH, false, 2, false, 128, 0, 41984>(dev, tmA, tmB, p);
    default:
      return launch_qgemm_cfg<128, 3, QG_A_PATCH, false, 2, false, 128, 0, 75776>(dev, tmA, tmB, p);
  }
}

static int fill_epilogue(QgParams& p, const mira_dequant* dq, const mira_epilogue* epi) {
  MIRA_CHECK_ARG(dq != nullptr && epi != nullptr, "dequant and epilogue descriptors are required");
  MIRA_CHECK_ARG(epi->n_steps >= 0 && epi->n_steps <= MIRA_EPI_MAX_STEPS, "too many epilogue steps");
  MIRA_CHECK_ARG(epi->out_f32 != nullptr || epi->out_i8 != nullptr, "epilogue has no output");
  p.scale64 = dq->scale64;
  p.scale_hi = dq->scale_hi;
  p.scale_lo = dq->scale_lo;
  p.row_scale = dq->row_scale;
  p.col_scale = dq->col_scale;
  if (dq->scale64 != nullptr) {
    MIRA_CHECK_ARG(dq->scale_hi != nullptr && dq->scale_lo != nullptr, "per-channel scales need scale_hi/scale_lo");
    MIRA_CHECK_ARG((reinterpret_cast<uintptr_t>(dq->scale_hi) & 15) == 0 &&
                       (reinterpret_cast<uintptr_t>(dq->scale_lo) & 15) == 0,
                   "scale arrays must be 16-byte aligned");
  } else {
    MIRA_CHECK_ARG(dq->row_scale != nullptr && dq->col_scale != nullptr, "no dequant scales given");
  }
  p.n_steps = epi->n_steps;
  for (int s = 0; s < epi->n_steps; ++s) {
    const mira_epi_step& st = epi->steps[s];
    MIRA_CHECK_ARG((st.op >= MIRA_EPI_RELU && st.op <= MIRA_EPI_TANH) || (st.op >= MIRA_EPI_ADD && st.op <= MIRA_EPI_MINIMUM),
                   "unknown epilogue op");
    const bool unary = st.op < MIRA_EPI_ADD;
    MIRA_CHECK_ARG(unary == (st.operand == MIRA_OPND_NONE), "epilogue operand kind does not match the op");
    if (st.operand == MIRA_OPND_CHANNEL)
      MIRA_CHECK_ARG(st.ptr != nullptr && (reinterpret_cast<uintptr_t>(st.ptr) & 15) == 0, "channel operand must be 16-byte aligned");
    if (st.operand == MIRA_OPND_FULL || st.operand == MIRA_OPND_ROW)
      MIRA_CHECK_ARG(st.ptr != nullptr, "operand pointer missing");
    if (st.operand == MIRA_OPND_FULL)
      MIRA_CHECK_ARG(st.ld % 4 != 0 || (reinterpret_cast<uintptr_t>(st.ptr) & 15) == 0, "full operand misaligned");
    p.steps[s] = st;
  }
  p.out_f32 = epi->out_f32;
  p.ld_f32 = epi->ld_f32;
  p.out_i8 = epi->out_i8;
  p.ld_i8 = epi->ld_i8;
  if (epi->out_f32 != nullptr)
    MIRA_CHECK_ARG(epi->ld_f32 % 4 != 0 || (reinterpret_cast<uintptr_t>(epi->out_f32) & 15) == 0, "f32 output misaligned");
  if (epi->out_i8 != nullptr) {
    MIRA_CHECK_ARG(epi->ld_i8 % 16 == 0 && (reinterpret_cast<uintptr_t>(epi->out_i8) & 15) == 0,
                   "int8 output needs a 16-byte aligned base and a row stride multiple of 16");
    MIRA_CHECK_ARG(epi->out_scale > 0.0f && std::isfinite(epi->out_scale), "requant scale must be positive");
  }
  MIRA_CHECK_ARG(epi->i8_layout == MIRA_LAYOUT_NHWC || epi->i8_layout == MIRA_LAYOUT_CP, "unknown int8 output layout");
  p.i8_cp = 0;
  p.i8_guard = 0;
  p.i8_chunk = 16;   // rows layout: the next 16 channels are the next 16 bytes (set_i8_layout for CP)
  // whether the steps end in values that cannot be negative (NaN aside): relu, or maximum with a
  // scalar >= 0, followed at most by minimum with a scalar >= 0 (ReLU6)
  bool nonneg = false;
  for (int s = 0; s < epi->n_steps; ++s) {
    const mira_epi_step& st = epi->steps[s];
    const bool scalar = st.operand == MIRA_OPND_SCALAR;
    if (st.op == MIRA_EPI_RELU) nonneg = true;
    else if (st.op == MIRA_EPI_MAXIMUM && scalar && st.scalar >= 0.0f) nonneg = true;
    else if (st.op == MIRA_EPI_MINIMUM && scalar && st.scalar >= 0.0f) nonneg = nonneg;
    else nonneg = false;
  }
  p.nonneg = nonneg ? 1 : 0;
  // the fused step programs: [add channel] [add full] [relu | maximum scalar, minimum scalar]
  {
    const mira_epi_step* st = epi->steps;
    const int n = epi->n_steps;
    int i = 0, kind = 0;
    if (i < n && st[i].op == MIRA_EPI_ADD && st[i].operand == MIRA_OPND_CHANNEL && i == 0) { kind |= QG_EPI_BIAS; ++i; }
    if (i < n && st[i].op == MIRA_EPI_ADD && st[i].operand == MIRA_OPND_FULL && i == 1) { kind |= QG_EPI_RES; ++i; }
    if (i < n && st[i].op == MIRA_EPI_RELU) {
      kind |= QG_EPI_RELU;
      ++i;
    } else if (i + 1 < n && st[i].op == MIRA_EPI_MAXIMUM && st[i].operand == MIRA_OPND_SCALAR &&
               st[i + 1].op == MIRA_EPI_MINIMUM && st[i + 1].operand == MIRA_OPND_SCALAR && i + 2 == n) {
      kind |= QG_EPI_CLAMP;
      i += 2;
    }
    p.epi_kind = (i == n && n > 0) ? kind : 0;
  }
  const QuantScale q = make_qscale(epi->out_i8 != nullptr ? epi->out_scale : 1.0f);
  p.q_scale = q.s;
  p.q_rcp = q.rcp;
  p.q_lim = q.lim;
  p.q_c127 = 127.0f * q.s;
  p.err = device_err_ptr();
  return MIRA_CUDA_OK;
}

// Guard slots in front of the chunk-planar layout's planes (MIRA_LAYOUT_CP) for image width w: a
// tile's halo starts w + 3 slots before its first output slot.
static int64_t cp_guard(int64_t w) { return round_up(w + 3, 8); }

// The int8 output of a convolution with output [n, oh, ow] in the chunk-planar layout when the
// epilogue asks for it.
static int set_i8_layout(QgParams& p, const mira_epilogue* epi, int64_t n, int64_t oh, int64_t ow) {
  if (epi->out_i8 == nullptr || epi->i8_layout != MIRA_LAYOUT_CP) return MIRA_CUDA_OK;
  MIRA_CHECK_ARG(n * (oh + 2) * (ow + 2) * 16 < (int64_t(1) << 40), "chunk-planar output too large");
  p.i8_cp = 1;
  p.i8_guard = int(cp_guard(ow));
  p.i8_chunk = n * (oh + 2) * (ow + 2) * 16;
  return MIRA_CUDA_OK;
}

// Diagnostic kernel: waits on an mbarrier that nothing ever completes, with the kernels' usual
// bounded wait shortened to `timeout_ns`; records error 2 when the wait gives up, as every kernel
// here does on an expired wait.
__global__ void selftest_wait_kernel(uint64_t timeout_ns, int* err) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (!mbar_wait(&bar, 0, &abort_flag, timeout_ns)) atomicExch(err, 2);
    mbar_arrive(&bar);   // complete the phase so the barrier is not left pending
  }
  __syncthreads();
}

}  // namespace mira

using namespace mira;

// ================================================================== C ABI: runtime

extern "C" int mira_cuda_abi_version(void) { return MIRA_CUDA_ABI_VERSION; }

extern "C" int mira_cuda_last_error(char* buf, size_t n) {
  if (buf == nullptr || n == 0) return MIRA_CUDA_EINVAL;
  std::snprintf(buf, n, "%s", t_last_error.c_str());
  return MIRA_CUDA_OK;
}

extern "C" int mira_cuda_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
  return n;
}

extern "C" int mira_cuda_set_device(int device) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return set_error(MIRA_CUDA_ENODEV, "no CUDA device");
  if (device < 0 || device >= n || device >= kMaxDevices) return set_error(MIRA_CUDA_EINVAL, "device index out of range");
  const int rc = init_device(device);
  if (rc != MIRA_CUDA_OK) return rc;
  t_device = device;
  MIRA_CUDA_TRY(cudaSetDevice(device), "cudaSetDevice");
  return MIRA_CUDA_OK;
}

extern "C" int mira_cuda_device_info(int* sm_count, int* cc_major, int* cc_minor) {
  MIRA_GET_DEVICE(dev);
  if (sm_count) *sm_count = dev->sm_count;
  if (cc_major) *cc_major = dev->cc_major;
  if (cc_minor) *cc_minor = dev->cc_minor;
  return MIRA_CUDA_OK;
}

extern "C" int mira_cuda_malloc(void** ptr, size_t bytes) {
  MIRA_GET_DEVICE(dev);
  MIRA_CHECK_ARG(ptr != nullptr, "null out pointer");
  *ptr = nullptr;
  MIRA_CUDA_TRY(cudaMalloc(ptr, bytes == 0 ? 16 : bytes), "cudaMalloc");
  return MIRA_CUDA_OK;
}

extern "C" int mira_cuda_free(void* ptr) {
  MIRA_GET_DEVICE(dev);
  if (ptr != nullptr) MIRA_CUDA_TRY(cudaFree(ptr), "cudaFree");
  return MIRA_CUDA_OK;
}

extern "C" int mira_cuda_host_alloc(void** ptr, size_t bytes) {
  MIRA_GET_DEVICE(dev);
  MIRA_CHECK_ARG(ptr != nullptr, "null out pointer");
  MIRA_CUDA_TRY(cudaHostAlloc(ptr, bytes == 0 ? 16 : bytes, cudaHostAllocPortable), "cudaHostAlloc");
  return MIRA_CUDA_OK;
}

extern "C" int mira_cuda_host_free(void* ptr) {
  if (ptr != nullptr) MIRA_CUDA_TRY(cudaFreeHost(ptr), "cudaFreeHost");
  return MIRA_CUDA_OK;
}

extern "C" int mira_cuda_memset(void* dst, int value, size_t bytes) {
  MIRA_GET_DEVICE(dev);
  MIRA_CUDA_TRY(cudaMemsetAsync(dst, value, bytes, dev->stream), "cudaMemsetAsync");
  return MIRA_CUDA_OK;
}

extern "C" int mira_cuda_h2d(void* dst, const void* src, size_t bytes) {
  MIRA_GET_DEVICE(dev);
  MIRA_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, dev->stream), "cudaMemcpyAsync H2D");
  return MIRA_CUDA_OK;
}

extern "C" int mira_cuda_d2h(void* dst, const void* src, size_t bytes) {
  MIRA_GET_DEVICE(dev);
  MIRA_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, dev->stream), "cudaMemcpyAsync D2H");
  return MIRA_CUDA_OK;
}

extern "C" int mira_cuda_d2d(void* dst, const void* src, size_t bytes) {
  MIRA_GET_DEVICE(dev);
  MIRA_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, dev->stream), "cudaMemcpyAsync D2D");
  return MIRA_CUDA_OK;
}

extern "C" int mira_cuda_h2d_copy_stream(void* dst, const void* src, size_t bytes) {
  MIRA_GET_DEVICE(dev);
  MIRA_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, dev->copy_stream),
                "cudaMemcpyAsync H2D (copy stream)");
  return MIRA_CUDA_OK;
}

extern "C" int mira_cuda_copy_stream_record(void* ev) {
  MIRA_GET_DEVICE(dev);
  MIRA_CUDA_TRY(cudaEventRecord(static_cast<cudaEvent_t>(ev), dev->copy_stream), "cudaEventRecord(copy stream)");
  return MIRA_CUDA_OK;
}

extern "C" int mira_cuda_copy_stream_wait(void* ev) {
  MIRA_GET_DEVICE(dev);
  MIRA_CUDA_TRY(cudaStreamWaitEvent(dev->copy_stream, static_cast<cudaEvent_t>(ev), 0), "cudaStreamWaitEvent(copy)");
  return MIRA_CUDA_OK;
}

extern "C" int mira_cuda_stream_wait(void* ev) {
  MIRA_GET_DEVICE(dev);
  MIRA_CUDA_TRY(cudaStreamWaitEvent(dev->stream, static_cast<cudaEvent_t>(ev), 0), "cudaStreamWaitEvent");
  return MIRA_CUDA_OK;
}

extern "C" int mira_cuda_event_sync(void* ev) {
  MIRA_GET_DEVICE(dev);
  MIRA_CUDA_TRY(cudaEventSynchronize(static_cast<cudaEvent_t>(ev)), "cudaEventSynchronize");
  return MIRA_CUDA_OK;
}

extern "C" int mira_cuda_sync(void) {
  MIRA_GET_DEVICE(dev);
  MIRA_CUDA_TRY(cudaStreamSynchronize(dev->copy_stream), "cudaStreamSynchronize(copy)");
  MIRA_CUDA_TRY(cudaStreamSynchronize(dev->stream), "cudaStreamSynchronize");
  int flag = 0;
  MIRA_CUDA_TRY(cudaMemcpyFromSymbol(&flag, g_mira_kernel_error, sizeof(int)), "read kernel error record");
  if (flag != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_mira_kernel_error, &zero, sizeof(int));
    if (flag == 3) return set_error(MIRA_CUDA_EKERNEL, "embedding row index out of range (error record 3)");
    return set_error(MIRA_CUDA_EKERNEL, "a kernel gave up on a bounded wait (error record " + std::to_string(flag) + ")");
  }
  return MIRA_CUDA_OK;
}

extern "C" int mira_cuda_get_stream(void** stream) {
  MIRA_GET_DEVICE(dev);
  MIRA_CHECK_ARG(stream != nullptr, "null out pointer");
  *stream = dev->stream;
  return MIRA_CUDA_OK;
}

extern "C" int mira_cuda_event_create(void** ev) {
  MIRA_GET_DEVICE(dev);
  cudaEvent_t e;
  MIRA_CUDA_TRY(cudaEventCreate(&e), "cudaEventCreate");
  *ev = e;
  return MIRA_CUDA_OK;
}

extern "C" int mira_cuda_event_record(void* ev) {
  MIRA_GET_DEVICE(dev);
  MIRA_CUDA_TRY(cudaEventRecord(static_cast<cudaEvent_t>(ev), dev->stream), "cudaEventRecord");
  return MIRA_CUDA_OK;
}

extern "C" int mira_cuda_event_elapsed(void* start, void* end, float* ms) {
  MIRA_GET_DEVICE(dev);
  MIRA_CUDA_TRY(cudaEventSynchronize(static_cast<cudaEvent_t>(end)), "cudaEventSynchronize");
  MIRA_CUDA_TRY(cudaEventElapsedTime(ms, static_cast<cudaEvent_t>(start), static_cast<cudaEvent_t>(end)),
                "cudaEventElapsedTime");
  return MIRA_CUDA_OK;
}

extern "C" int mira_cuda_event_destroy(void* ev) {
  if (ev != nullptr) MIRA_CUDA_TRY(cudaEventDestroy(static_cast<cudaEvent_t>(ev)), "cudaEventDestroy");
  return MIRA_CUDA_OK;
}

extern "C" int mira_cuda_graph_begin(void) {
  MIRA_GET_DEVICE(dev);
  MIRA_CUDA_TRY(cudaStreamBeginCapture(dev->stream, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
  return MIRA_CUDA_OK;
}

extern "C" int mira_cuda_graph_end(void** graph_exec) {
  MIRA_GET_DEVICE(dev);
  cudaGraph_t g = nullptr;
  MIRA_CUDA_TRY(cudaStreamEndCapture(dev->stream, &g), "cudaStreamEndCapture");
  cudaGraphExec_t ge = nullptr;
  const cudaError_t e = cudaGraphInstantiate(&ge, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return cuda_error(e, "cudaGraphInstantiate");
  *graph_exec = ge;
  return MIRA_CUDA_OK;
}

extern "C" int mira_cuda_graph_launch(void* graph_exec) {
  MIRA_GET_DEVICE(dev);
  MIRA_CUDA_TRY(cudaGraphLaunch(static_cast<cudaGraphExec_t>(graph_exec), dev->stream), "cudaGraphLaunch");
  return MIRA_CUDA_OK;
}

extern "C" int mira_cuda_graph_destroy(void* graph_exec) {
  if (graph_exec != nullptr) MIRA_CUDA_TRY(cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(graph_exec)), "cudaGraphExecDestroy");
  return MIRA_CUDA_OK;
}

extern "C" int64_t mira_cuda_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

extern "C" int mira_cuda_selftest_wait_timeout(int64_t timeout_us) {
  MIRA_GET_DEVICE(dev);
  MIRA_CHECK_ARG(timeout_us > 0 && timeout_us <= 1000000, "timeout must be in (0, 1 s]");
  selftest_wait_kernel<<<1, 32, 0, dev->stream>>>(uint64_t(timeout_us) * 1000u, device_err_ptr());
  return after_launch("selftest_wait_kernel");
}

// ================================================================== C ABI: kernels

extern "C" int mira_cuda_quantize_rows(const float* x, int64_t rows, int64_t cols, int64_t ld_x, float scale,
                                       int8_t* xq, int64_t ld_q) {
  MIRA_GET_DEVICE(dev);
  MIRA_CHECK_ARG(rows >= 0 && cols >= 0 && ld_x >= cols && ld_q >= cols, "bad quantize shape");
  MIRA_CHECK_ARG(ld_q % 16 == 0 && (reinterpret_cast<uintptr_t>(xq) & 15) == 0, "int8 rows must be 16-byte aligned");
  MIRA_CHECK_ARG(scale > 0.0f && std::isfinite(scale), "quantization scale must be positive");
  if (rows == 0 || ld_q == 0) return MIRA_CUDA_OK;
  const int threads = 256;
  quantize_rows_kernel<<<grid_for(dev, rows * (ld_q / 16), threads), threads, 0, dev->stream>>>(
      x, rows, cols, ld_x, make_qscale(scale), xq, ld_q);
  return after_launch("quantize_rows_kernel");
}

extern "C" int mira_cuda_quantize_nchw_to_nhwc(const float* x, int64_t n, int64_t c, int64_t h, int64_t w, float scale,
                                               int8_t* xq, int64_t cp) {
  MIRA_GET_DEVICE(dev);
  MIRA_CHECK_ARG(n >= 0 && c > 0 && h > 0 && w > 0 && cp >= c && cp % 4 == 0, "bad quantize_nchw shape");
  MIRA_CHECK_ARG((reinterpret_cast<uintptr_t>(xq) & 3) == 0, "int8 output must be 4-byte aligned");
  MIRA_CHECK_ARG(scale > 0.0f && std::isfinite(scale), "quantization scale must be positive");
  if (n == 0) return MIRA_CUDA_OK;
  const int threads = 256;
  const int64_t work = n * h * w * (cp / 4);
  quantize_nchw_nhwc_kernel<<<grid_for(dev, work, threads), threads, 0, dev->stream>>>(x, n, c, h * w,
                                                                                       make_qscale(scale), xq, cp);
  return after_launch("quantize_nchw_nhwc_kernel");
}

extern "C" int mira_cuda_quantize_nchw_to_row4(const float* x, int64_t n, int64_t c, int64_t h, int64_t w,
                                               float scale, int8_t* xq, int64_t row_entries, int64_t pad,
                                               int64_t entry_stride) {
  MIRA_GET_DEVICE(dev);
  MIRA_CHECK_ARG(n >= 0 && c > 0 && c <= 4 && h > 0 && w > 0 && row_entries > 0 && pad >= 0, "bad quantize_row4 shape");
  MIRA_CHECK_ARG((reinterpret_cast<uintptr_t>(xq) & 15) == 0, "int8 output must be 16-byte aligned");
  MIRA_CHECK_ARG(scale > 0.0f && std::isfinite(scale), "quantization scale must be positive");
  if (n == 0) return MIRA_CUDA_OK;
  MIRA_CHECK_ARG(row_entries < (int64_t(1) << 24), "rows too long");
  MIRA_CHECK_ARG(entry_stride == 1 || entry_stride == 2 || entry_stride == 4, "entry stride must be 1, 2 or 4");
  const int64_t warps = (row_entries + 31) / 32;
  const int threads = int(32 * (warps < 8 ? warps : 8));
  const int64_t groups = (n * h + Q4_ROWS - 1) / Q4_ROWS;
  const dim3 grid(unsigned((warps * 32 + threads - 1) / threads), unsigned(groups < 65535 ? groups : 65535));
  const QuantScale qs = make_qscale(scale);
  if (entry_stride == 1)
    quantize_nchw_row4_kernel<1><<<grid, threads, 0, dev->stream>>>(x, int(n), int(c), int(h), int(w), qs, xq,
                                                                    int(row_entries), int(pad));
  else if (entry_stride == 2)
    quantize_nchw_row4_kernel<2><<<grid, threads, 0, dev->stream>>>(x, int(n), int(c), int(h), int(w), qs, xq,
                                                                    int(row_entries), int(pad));
  else
    quantize_nchw_row4_kernel<4><<<grid, threads, 0, dev->stream>>>(x, int(n), int(c), int(h), int(w), qs, xq,
                                                                    int(row_entries), int(pad));
  return after_launch("quantize_nchw_row4_kernel");
}

namespace mira {

// Split-K plan for a GEMM whose output tiles cannot fill the GPU: the number of K ranges per
// output tile (1: no split) and the K-blocks per range.  A split pays off when fewer than half
// the SMs would get a tile and the reduction is long enough to cut into ranges of >= 4 blocks.
// Tile width of a GEMM.  One row tile (M <= 128: the skinny shapes of decode steps and small
// batches) takes the widest tile, no wider than N needs, whose split-K plan (below) still puts
// CTAs on three quarters of the SMs, else the width with the most CTAs: long reductions keep wide
// tiles with long K ranges, short ones (K of a few K-blocks) narrow tiles.  Otherwise by N.
static int pick_bn_gemm(int64_t M, int64_t N, int64_t K, int sm_count) {
  if (M > QG_BM) return pick_bn(N);
  const int64_t num_kb = (K + QG_BK - 1) / QG_BK;
  int best_bn = 64;
  int64_t best = -1;
  for (int bn = pick_bn(N); bn >= 64; bn /= 2) {
    const int64_t tiles = (N + bn - 1) / bn;
    int64_t s = tiles * 2 > sm_count ? 1 : sm_count / tiles;
    if (s > num_kb) s = num_kb;
    if (s > 16) s = 16;
    const int64_t ctas = tiles * (s < 1 ? 1 : s);
    if (ctas * 4 >= int64_t(sm_count) * 3) return bn;
    if (ctas > best) {
      best = ctas;
      best_bn = bn;
    }
  }
  return best_bn;
}

// Split-K for GEMMs whose output tiles cannot fill the GPU: a single row tile splits its K-blocks
// over up to sm_count / tiles CTAs per tile (one K-block each at least); taller shapes need 8
// K-blocks and keep at least 4 per split.  splits = ceil(num_kb / kb_per), so every split covers at
// least one K-block: mira_cuda_qgemm_splitk_static relies on that (it never clears its scratch).
static void splitk_plan(int64_t M, int64_t N, int64_t K, int sm_count, int& splits, int& kb_per) {
  const int bn = pick_bn_gemm(M, N, K, sm_count);
  const int64_t tiles = ((M + QG_BM - 1) / QG_BM) * ((N + bn - 1) / bn);
  const int num_kb = int((K + QG_BK - 1) / QG_BK);
  const bool one_row = M <= QG_BM;
  splits = 1;
  kb_per = num_kb;
  if (tiles * 2 > sm_count || (!one_row && num_kb < 8)) return;
  int s = int(sm_count / tiles);
  if (s > (one_row ? num_kb : num_kb / 4)) s = one_row ? num_kb : num_kb / 4;
  if (s > 16) s = 16;
  if (s < 2) return;
  kb_per = (num_kb + s - 1) / s;
  splits = (num_kb + kb_per - 1) / kb_per;
  if (splits < 2) {
    splits = 1;
    kb_per = num_kb;
  }
}

static int qgemm_check(int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb) {
  MIRA_CHECK_ARG(M >= 0 && N > 0 && K > 0, "bad qgemm shape");
  MIRA_CHECK_ARG(M < (int64_t(1) << 31) && N < (int64_t(1) << 24) && K < (int64_t(1) << 24), "qgemm shape too large");
  MIRA_CHECK_ARG(K <= 133000, "K too large for exact int32 accumulation of int8 products");
  MIRA_CHECK_ARG(lda >= round_up(K, 16) && lda % 16 == 0 && ldb >= round_up(K, 16) && ldb % 16 == 0,
                 "int8 operands need row strides >= round_up(K, 16), multiples of 16");
  return MIRA_CUDA_OK;
}

// The quantized GEMM, optionally split over K: with splits > 1 the tcgen05 kernel stores each K
// range's int32 sums to ws (splits x M x N) and qgemm_splitk_finish_kernel adds them and runs the
// epilogue.
static int qgemm_run(DeviceState* dev, int64_t M, int64_t N, int64_t K, const int8_t* A, int64_t lda, const int8_t* B,
                     int64_t ldb, const mira_dequant* dq, const mira_epilogue* epi, int splits, int kb_per,
                     int32_t* ws) {
  QgParams p;
  std::memset(&p, 0, sizeof(p));
  const int rc = fill_epilogue(p, dq, epi);
  if (rc != MIRA_CUDA_OK) return rc;
  MIRA_CHECK_ARG(epi->out_i8 == nullptr || epi->i8_layout == MIRA_LAYOUT_NHWC,
                 "the chunk-planar int8 output is for convolutions");
  const int bn = pick_bn_gemm(M, N, K, dev->sm_count);
  p.M = int(M);
  p.N = int(N);
  p.K = int(K);
  p.num_kb = int((K + QG_BK - 1) / QG_BK);
  p.m_tiles = int((M + QG_BM - 1) / QG_BM);
  p.n_tiles = int((N + bn - 1) / bn);
  SplitkFinishParams f;
  if (splits > 1) {
    std::memset(&f, 0, sizeof(f));
    f.ws = ws; f.splits = splits; f.slice = M * N; f.M = int(M); f.N = int(N);
    f.scale64 = p.scale64; f.scale_hi = p.scale_hi; f.scale_lo = p.scale_lo;
    f.row_scale = p.row_scale; f.col_scale = p.col_scale;
    f.n_steps = p.n_steps;
    for (int s = 0; s < p.n_steps; ++s) f.steps[s] = p.steps[s];
    f.out_f32 = p.out_f32; f.ld_f32 = p.ld_f32; f.out_i8 = p.out_i8; f.ld_i8 = p.ld_i8;
    f.q = make_qscale(p.out_i8 != nullptr ? epi->out_scale : 1.0f);
    p.k_splits = splits;
    p.kb_per_split = kb_per;
    p.raw = 1;
    p.split_stride = M * N;
    p.out_f32 = reinterpret_cast<float*>(ws);
    p.ld_f32 = N;
    p.out_i8 = nullptr;
    p.n_steps = 0;
  }
  CUtensorMap tmA, tmB;
  int r = encode_2d_i8(&tmA, A, uint64_t(lda), uint64_t(M), uint64_t(lda), QG_BK, QG_BM);
  if (r != MIRA_CUDA_OK) return r;
  if (use_pair_gemm(dev, M, N, K, splits)) {
    // each CTA of a pair stages 128 of the tile's 256 columns of B
    r = encode_2d_i8(&tmB, B, uint64_t(ldb), uint64_t(N), uint64_t(ldb), QG_BK, 128);
    if (r != MIRA_CUDA_OK) return r;
    p.n_tiles = int((N + 255) / 256);
    return p.scale64 != nullptr ? launch_qgemm_pair_cfg<256, 6, false, 2>(dev, tmA, tmB, p)
                                : launch_qgemm_pair_cfg<256, 6, true, 2>(dev, tmA, tmB, p);
  }
  r = encode_2d_i8(&tmB, B, uint64_t(ldb), uint64_t(N), uint64_t(ldb), QG_BK, uint32_t(bn));
  if (r != MIRA_CUDA_OK) return r;
  r = p.scale64 != nullptr ? launch_qgemm_bn<QG_A_TMA, false>(dev, tmA, tmB, p, bn)
                           : launch_qgemm_bn<QG_A_TMA, true>(dev, tmA, tmB, p, bn);
  if (r != MIRA_CUDA_OK || splits <= 1) return r;
  const int threads = 256;
  const int64_t width = (f.out_i8 != nullptr && f.ld_i8 > N) ? f.ld_i8 : N;
  qgemm_splitk_finish_kernel<<<grid_for(dev, M * width, threads), threads, 0, dev->stream>>>(f);
  return after_launch("qgemm_splitk_finish_kernel");
}

}  // namespace mira

extern "C" int mira_cuda_qgemm(int64_t M, int64_t N, int64_t K, const int8_t* A, int64_t lda, const int8_t* B,
                               int64_t ldb, const mira_dequant* dq, const mira_epilogue* epi) {
  MIRA_GET_DEVICE(dev);
  const int rc = qgemm_check(M, N, K, lda, ldb);
  if (rc != MIRA_CUDA_OK) return rc;
  if (M == 0) return MIRA_CUDA_OK;
  return qgemm_run(dev, M, N, K, A, lda, B, ldb, dq, epi, 1, 0, nullptr);
}

extern "C" int64_t mira_cuda_qgemm_workspace(int64_t M, int64_t N, int64_t K) {
  DeviceState* dev = current_device();
  if (dev == nullptr || M <= 0 || N <= 0 || K <= 0) return 0;
  int splits, kb_per;
  splitk_plan(M, N, K, dev->sm_count, splits, kb_per);
  return splits > 1 ? int64_t(splits) * M * N * int64_t(sizeof(int32_t)) : 0;
}

extern "C" int mira_cuda_qgemm_splitk(int64_t M, int64_t N, int64_t K, const int8_t* A, int64_t lda, const int8_t* B,
                                      int64_t ldb, const mira_dequant* dq, const mira_epilogue* epi, void* workspace,
                                      int64_t workspace_bytes) {
  MIRA_GET_DEVICE(dev);
  const int rc = qgemm_check(M, N, K, lda, ldb);
  if (rc != MIRA_CUDA_OK) return rc;
  if (M == 0) return MIRA_CUDA_OK;
  int splits, kb_per;
  splitk_plan(M, N, K, dev->sm_count, splits, kb_per);
  if (splits > 1) {
    const int64_t need = int64_t(splits) * M * N * int64_t(sizeof(int32_t));
    MIRA_CHECK_ARG(workspace != nullptr && workspace_bytes >= need,
                   "split-K workspace smaller than mira_cuda_qgemm_workspace() bytes");
    MIRA_CHECK_ARG((reinterpret_cast<uintptr_t>(workspace) & 15) == 0, "split-K workspace must be 16-byte aligned");
  }
  return qgemm_run(dev, M, N, K, A, lda, B, ldb, dq, epi, splits, kb_per, static_cast<int32_t*>(workspace));
}

// Shared argument checks and parameter setup of the implicit-GEMM convolutions.
static int conv_setup(int64_t n, int64_t h, int64_t w, int64_t cp, const int8_t* x, int64_t x_layout,
                      int64_t x_row_entries, int64_t o, int64_t kh, int64_t kw, int64_t ldw, int64_t stride_h,
                      int64_t stride_w, int64_t pad_h, int64_t pad_w, int64_t dil_h, int64_t dil_w,
                      const mira_dequant* dq, const mira_epilogue* epi, QgParams& p, int64_t& oh, int64_t& ow) {
  MIRA_CHECK_ARG(n >= 0 && h > 0 && w > 0 && o > 0 && kh > 0 && kw > 0, "bad qconv2d shape");
  MIRA_CHECK_ARG(cp == 4 || (cp > 0 && cp % 16 == 0), "input channels must be padded to 4 or a multiple of 16");
  MIRA_CHECK_ARG(stride_h > 0 && stride_w > 0 && dil_h > 0 && dil_w > 0 && pad_h >= 0 && pad_w >= 0, "bad conv geometry");
  MIRA_CHECK_ARG(kw <= 32, "kernel width above 32");
  MIRA_CHECK_ARG((reinterpret_cast<uintptr_t>(x) & 15) == 0, "conv input must be 16-byte aligned");
  oh = (h + 2 * pad_h - dil_h * (kh - 1) - 1) / stride_h + 1;
  ow = (w + 2 * pad_w - dil_w * (kw - 1) - 1) / stride_w + 1;
  MIRA_CHECK_ARG(oh > 0 && ow > 0, "kernel larger than the padded input");
  MIRA_CHECK_ARG(x_layout == MIRA_LAYOUT_NHWC || x_layout == MIRA_LAYOUT_ROW4 || x_layout == MIRA_LAYOUT_CP,
                 "unknown input layout");
  if (x_layout == MIRA_LAYOUT_CP)
    MIRA_CHECK_ARG(cp % 64 == 0 && kh == 3 && kw == 3 && stride_h == 1 && stride_w == 1 && pad_h == 1 && pad_w == 1 &&
                       dil_h == 1 && dil_w == 1,
                   "the chunk-planar layout feeds 3x3, stride-1, pad-1 convolutions of 64k input channels");
  if (x_layout == MIRA_LAYOUT_ROW4) {
    MIRA_CHECK_ARG(cp == 4 && kw <= 8 && dil_h == 1 && dil_w == 1,
                   "the row-expanded layout serves 4-channel inputs, kernel width <= 8, no dilation");
    MIRA_CHECK_ARG(stride_w == 1 || stride_w == 2 || stride_w == 4, "row-expanded inputs: horizontal stride 1, 2 or 4");
    MIRA_CHECK_ARG(x_row_entries >= ow + 4 / stride_w, "row-expanded input has too few entries per row");
  }
  const int64_t K = x_layout == MIRA_LAYOUT_ROW4 ? kh * 32 : kh * kw * cp;
  MIRA_CHECK_ARG(K <= 133000, "K too large for exact int32 accumulation of int8 products");
  MIRA_CHECK_ARG(ldw >= round_up(K, 16) && ldw % 16 == 0, "weight row stride must be >= round_up(K, 16)");
  const int64_t M = n * oh * ow;
  MIRA_CHECK_ARG(M < (int64_t(1) << 31) && n * h * w * cp < (int64_t(1) << 40), "conv too large");
  std::memset(&p, 0, sizeof(p));
  const int rc = fill_epilogue(p, dq, epi);
  if (rc != MIRA_CUDA_OK) return rc;
  MIRA_CHECK_ARG(p.scale64 != nullptr, "convolutions use per-channel scales");
  p.M = int(M);
  p.N = int(o);
  p.K = int(K);
  p.num_kb = int((K + QG_BK - 1) / QG_BK);
  p.A = x;
  p.g = QgConv{int(n), int(h), int(w), int(cp), int(oh), int(ow), int(kh), int(kw), int(stride_h), int(stride_w),
               int(pad_h), int(pad_w), int(dil_h), int(dil_w), int(x_row_entries), 0, 0, 0};
  if (x_layout == MIRA_LAYOUT_CP) {
    // GEMM rows = every slot of the zero-padded output plane (same geometry as the input)
    const int64_t plane = n * (h + 2) * (w + 2);
    MIRA_CHECK_ARG(plane < (int64_t(1) << 31) - 256, "conv too large for the chunk-planar layout");
    p.M = int(plane);
    p.dv_a = make_div((h + 2) * (w + 2));
    p.dv_b = make_div(w + 2);
    p.g.guard = int(cp_guard(w));
    p.g.patch_slots = int(QG_BM + 2 * (w + 3));
    p.g.plane = plane;
  } else {
    // rows are output pixels: divisors for pixel -> (image, y, x) of a chunk-planar int8 output
    p.dv_a = make_div(oh * ow);
    p.dv_b = make_div(ow);
  }
  return set_i8_layout(p, epi, n, oh, ow);
}

extern "C" int mira_cuda_qconv2d(int64_t n, int64_t h, int64_t w, int64_t cp, const int8_t* x, int64_t x_layout,
                                 int64_t x_row_entries, int64_t o, int64_t kh, int64_t kw, const int8_t* wq,
                                 int64_t ldw, int64_t stride_h, int64_t stride_w, int64_t pad_h, int64_t pad_w,
                                 int64_t dil_h, int64_t dil_w, const mira_dequant* dq, const mira_epilogue* epi) {
  MIRA_GET_DEVICE(dev);
  QgParams p;
  int64_t oh, ow;
  int rc = conv_setup(n, h, w, cp, x, x_layout, x_row_entries, o, kh, kw, ldw, stride_h, stride_w, pad_h, pad_w, dil_h,
                      dil_w, dq, epi, p, oh, ow);
  if (rc != MIRA_CUDA_OK) return rc;
  if (p.M == 0) return MIRA_CUDA_OK;
  const int bn = pick_bn(o);
  p.m_tiles = int((p.M + QG_BM - 1) / QG_BM);
  p.n_tiles = int((o + bn - 1) / bn);
  if (x_layout == MIRA_LAYOUT_CP) return launch_qgemm_patch(dev, wq, ldw, o, p);
  // a 1x1 stride-1 convolution without padding is a GEMM over the NHWC activation matrix [n*h*w, cp]
  if (x_layout == MIRA_LAYOUT_NHWC && kh == 1 && kw == 1 && stride_h == 1 && stride_w == 1 && pad_h == 0 &&
      pad_w == 0 && cp % 16 == 0 && (epi->out_i8 == nullptr || epi->i8_layout == MIRA_LAYOUT_NHWC))
    return qgemm_run(dev, p.M, o, cp, x, cp, wq, ldw, dq, epi, 1, 0, nullptr);
  CUtensorMap tmA, tmB;
  std::memset(&tmA, 0, sizeof(tmA));
  // TMA im2col for NHWC inputs of 64k channels and square, symmetric kernels
  if (x_layout == MIRA_LAYOUT_NHWC && cp % 64 == 0 && kh == kw && pad_h == pad_w && dil_h == dil_w &&
      pad_h <= 127 && (kw - 1) * dil_w - pad_w <= 128 && stride_h <= 8 && stride_w <= 8 && (kw - 1) * dil_w < 65536) {
    const int bk = cp % 128 == 0 ? 128 : 64;
    p.num_kb = int(p.K / bk);
    rc = encode_im2col_i8(&tmA, x, n, h, w, cp, kw, stride_h, stride_w, pad_w, dil_w, bk);
    if (rc != MIRA_CUDA_OK) return rc;
    rc = encode_2d_i8_sw(&tmB, wq, uint64_t(ldw), uint64_t(o), uint64_t(ldw), uint32_t(bk), uint32_t(bn),
                         bk == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != MIRA_CUDA_OK) return rc;
    return launch_qgemm_im2col(dev, tmA, tmB, p, bn, bk);
  }
  rc = encode_2d_i8(&tmB, wq, uint64_t(ldw), uint64_t(o), uint64_t(ldw), QG_BK, uint32_t(bn));
  if (rc != MIRA_CUDA_OK) return rc;
  if (x_layout == MIRA_LAYOUT_ROW4) {
    // the stem: weights resident in shared memory; 8 epilogue warps (with the 4 gather warps, 16
    // epilogue warps would cap the registers at 80 and spill)
    if (bn == 64 && p.n_tiles == 1 && p.num_kb <= 2)
      return launch_qgemm_cfg<64, 7, QG_A_ROW4, false, 2, false, QG_BK, 2>(dev, tmA, tmB, p);
    return launch_qgemm_bn<QG_A_ROW4, false>(dev, tmA, tmB, p, bn);
  }
  if (cp == 4) return launch_qgemm_bn<QG_A_GATHER4, false>(dev, tmA, tmB, p, bn);
  return launch_qgemm_bn<QG_A_GATHER16, false>(dev, tmA, tmB, p, bn);
}

// The stem + pool kernel (stem_pool_sm100.cuh).  Work units are (image, band of pooled rows); the
// band is chosen so that the units fill whole waves of CTAs with the fewest conv rows computed twice
// (each band recomputes the conv row it shares with the band above).
static int launch_stem_pool(DeviceState* dev, const QgParams& qp, int64_t n, int64_t h, int64_t w, int64_t oh,
                            int64_t ow, int64_t ph, int64_t pw, int64_t kh, int64_t pad_h, int64_t row_entries,
                            int64_t o, const int8_t* x, const int8_t* wq, int64_t ldw, const mira_epilogue* epi) {
  MIRA_CHECK_ARG(qp.out_f32 == nullptr || (qp.ld_f32 % 4 == 0 && (reinterpret_cast<uintptr_t>(qp.out_f32) & 15) == 0),
                 "pooled f32 output: rows of a multiple of 4 floats, 16-byte aligned");
  MIRA_CHECK_ARG(qp.out_i8 == nullptr || (qp.ld_i8 % 4 == 0 && qp.ld_i8 >= o), "pooled int8 output rows");
  if (n == 0) return MIRA_CUDA_OK;
  SpParams p;
  std::memset(&p, 0, sizeof(p));
  p.n = int(n); p.h = int(h); p.w = int(w);
  p.oh = int(oh); p.ow = int(ow); p.ph = int(ph); p.pw = int(pw);
  p.kh = int(kh); p.pad_h = int(pad_h); p.row_entries = int(row_entries); p.o = int(o);
  int64_t best_cost = -1;
  for (int b = 1; b <= 8; ++b) {
    const int64_t units = n * ((ph + b - 1) / b);
    const int64_t cost = ((units + dev->sm_count - 1) / dev->sm_count) * (2 * b + 1);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      p.band = b;
    }
  }
  p.bands = int((ph + p.band - 1) / p.band);
  MIRA_CHECK_ARG(n * p.bands < (int64_t(1) << 31), "too many work units");
  p.x = x; p.wq = wq; p.ldw = ldw;
  p.scale64 = qp.scale64; p.scale_hi = qp.scale_hi; p.scale_lo = qp.scale_lo;
  p.epi_kind = qp.epi_kind; p.n_steps = qp.n_steps;
  for (int s = 0; s < qp.n_steps; ++s) p.steps[s] = qp.steps[s];
  p.out_f32 = qp.out_f32; p.ld_f32 = qp.ld_f32;
  p.out_i8 = qp.out_i8; p.ld_i8 = qp.ld_i8;
  if (qp.out_i8 != nullptr && epi->i8_layout == MIRA_LAYOUT_CP) {
    MIRA_CHECK_ARG(qp.ld_i8 % 16 == 0, "chunk-planar int8 output: padded channel count a multiple of 16");
    p.i8_cp = 1;
    p.i8_guard = int(cp_guard(pw));
    p.i8_chunk = n * (ph + 2) * (pw + 2) * 16;
  }
  p.q_scale = qp.q_scale; p.q_rcp = qp.q_rcp; p.q_c127 = qp.q_c127; p.nonneg = qp.nonneg;
  p.err = qp.err;
  static bool attr_set[kMaxDevices] = {};
  if (!attr_set[dev->device]) {
    MIRA_CUDA_TRY(cudaFuncSetAttribute(stem_pool_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(SpSmem::TOTAL)),
                  "cudaFuncSetAttribute(stem_pool smem)");
    attr_set[dev->device] = true;
  }
  const int64_t units = n * p.bands;
  const int grid = int(units < dev->sm_count ? units : dev->sm_count);
  stem_pool_kernel<<<grid, SP_THREADS, SpSmem::TOTAL, dev->stream>>>(p);
  return after_launch("stem_pool_kernel");
}

extern "C" int mira_cuda_qconv2d_maxpool(int64_t n, int64_t h, int64_t w, int64_t cp, const int8_t* x,
                                         int64_t x_layout, int64_t x_row_entries, int64_t o, int64_t kh, int64_t kw,
                                         const int8_t* wq, int64_t ldw, int64_t stride_h, int64_t stride_w,
                                         int64_t pad_h, int64_t pad_w, int64_t dil_h, int64_t dil_w, int64_t pool_size,
                                         int64_t pool_stride, int64_t pool_pad, float pool_pad_value,
                                         const mira_dequant* dq, const mira_epilogue* epi) {
  MIRA_GET_DEVICE(dev);
  QgParams p;
  int64_t oh, ow;
  int rc = conv_setup(n, h, w, cp, x, x_layout, x_row_entries, o, kh, kw, ldw, stride_h, stride_w, pad_h, pad_w, dil_h,
                      dil_w, dq, epi, p, oh, ow);
  if (rc != MIRA_CUDA_OK) return rc;
  MIRA_CHECK_ARG(o <= 64, "fused pooling supports convolutions with at most 64 output channels");
  MIRA_CHECK_ARG(pool_size > 0 && pool_stride > 0 && pool_pad >= 0 && pool_pad < pool_size, "bad pool geometry");
  // the kernel pools the int32 accumulators and applies the epilogue to the pooled values, which
  // equals pooling the epilogue's outputs when every step is monotone non-decreasing in its input
  for (int s = 0; s < p.n_steps; ++s) {
    const mira_epi_step& st = p.steps[s];
    const bool monotone =
        (st.operand == MIRA_OPND_NONE && st.op == MIRA_EPI_RELU) ||
        ((st.operand == MIRA_OPND_SCALAR || st.operand == MIRA_OPND_CHANNEL) &&
         (st.op == MIRA_EPI_ADD || st.op == MIRA_EPI_MAXIMUM || st.op == MIRA_EPI_MINIMUM ||
          (st.op == MIRA_EPI_SUB && !st.swapped)));
    MIRA_CHECK_ARG(monotone, "fused pooling needs a monotone epilogue (relu, add/sub/max/min of constants)");
  }
  MIRA_CHECK_ARG(pool_pad == 0 || std::isinf(pool_pad_value) && pool_pad_value < 0,
                 "fused pooling pads with -inf only");
  const int64_t ph = (oh + 2 * pool_pad - pool_size) / pool_stride + 1;
  const int64_t pw = (ow + 2 * pool_pad - pool_size) / pool_stride + 1;
  MIRA_CHECK_ARG(ph > 0 && pw > 0, "pool window larger than the conv output");
  // the ResNet stem form (row-expanded input, stride 2, 3x3/2 pool with one pixel of padding)
  if (x_layout == MIRA_LAYOUT_ROW4 && stride_h == 2 && stride_w == 2 && kh <= SP_KH_MAX && pool_size == 3 &&
      pool_stride == 2 && pool_pad == 1 && ow <= SP_OW_MAX && x_row_entries <= SP_ENTRIES_MAX && o % 4 == 0)
    return launch_stem_pool(dev, p, n, h, w, oh, ow, ph, pw, kh, pad_h, x_row_entries, o, x, wq, ldw, epi);
  MIRA_CHECK_ARG(x_layout != MIRA_LAYOUT_CP && (epi->out_i8 == nullptr || epi->i8_layout == MIRA_LAYOUT_NHWC),
                 "fused pooling reads and writes the NHWC / row-expanded layouts");
  int T = 0;
  for (int t = 1; t <= 16; ++t) {
    const int64_t span = (t - 1) * pool_stride + pool_size;
    if (span * span <= 96) T = t;   // QgCfg<...>::POOL_ROWS
  }
  MIRA_CHECK_ARG(T > 0, "pool window too large to fuse");
  if (n == 0) return MIRA_CUDA_OK;
  p.pool_p = int(pool_size);
  p.pool_s = int(pool_stride);
  p.pool_pad = int(pool_pad);
  p.pool_t = T;
  p.pool_span = int((T - 1) * pool_stride + pool_size);
  p.ph_out = int(ph);
  p.pw_out = int(pw);
  p.tiles_y = int((ph + T - 1) / T);
  p.tiles_x = int((pw + T - 1) / T);
  p.pool_pad_value = pool_pad_value;
  p.M = 0x7fffffff;
  p.m_tiles = int(n * p.tiles_y * p.tiles_x);
  p.n_tiles = 1;
  CUtensorMap tmA, tmB;
  std::memset(&tmA, 0, sizeof(tmA));
  rc = encode_2d_i8(&tmB, wq, uint64_t(ldw), uint64_t(o), uint64_t(ldw), QG_BK, 64u);
  if (rc != MIRA_CUDA_OK) return rc;
  if (x_layout == MIRA_LAYOUT_ROW4) return launch_qgemm_cfg<64, 7, QG_A_ROW4, false, 2, true>(dev, tmA, tmB, p);
  if (cp == 4) return launch_qgemm_cfg<64, 7, QG_A_GATHER4, false, 2, true>(dev, tmA, tmB, p);
  return launch_qgemm_cfg<64, 7, QG_A_GATHER16, false, 2, true>(dev, tmA, tmB, p);
}

extern "C" int mira_cuda_maxpool2d_nhwc(const float* x_f32, const int8_t* x_i8, int64_t n, int64_t h, int64_t w,
                                        int64_t c, int64_t ldc_in, int64_t size, int64_t stride, int64_t pad,
                                        float pad_value, float* out_f32, int64_t ldc_out_f32, int8_t* out_i8,
                                        int64_t ldc_out_i8, float out_scale) {
  return mira_cuda_maxpool2d_nhwc_ex(x_f32, x_i8, n, h, w, c, ldc_in, size, stride, pad, pad_value, out_f32,
                                     ldc_out_f32, out_i8, ldc_out_i8, out_scale, MIRA_LAYOUT_NHWC);
}

extern "C" int64_t mira_cuda_cp_bytes(int64_t n, int64_t h, int64_t w, int64_t cp) {
  if (n < 0 || h <= 0 || w <= 0 || cp <= 0 || cp % 16 != 0) return 0;
  return (2 * mira::cp_guard(w) + QG_BM + (cp / 16) * n * (h + 2) * (w + 2)) * 16;
}

extern "C" int mira_cuda_maxpool2d_nhwc_ex(const float* x_f32, const int8_t* x_i8, int64_t n, int64_t h, int64_t w,
                                           int64_t c, int64_t ldc_in, int64_t size, int64_t stride, int64_t pad,
                                           float pad_value, float* out_f32, int64_t ldc_out_f32, int8_t* out_i8,
                                           int64_t ldc_out_i8, float out_scale, int64_t i8_layout) {
  MIRA_GET_DEVICE(dev);
  MIRA_CHECK_ARG(i8_layout == MIRA_LAYOUT_NHWC || (i8_layout == MIRA_LAYOUT_CP && x_i8 == nullptr && ldc_out_i8 % 16 == 0),
                 "chunk-planar int8 output: f32 input, padded channel count a multiple of 16");
  MIRA_CHECK_ARG(n >= 0 && h > 0 && w > 0 && c > 0 && size > 0 && stride > 0 && pad >= 0 && pad < size,
                 "bad maxpool geometry");
  const int64_t oh = (h + 2 * pad - size) / stride + 1, ow = (w + 2 * pad - size) / stride + 1;
  MIRA_CHECK_ARG(oh > 0 && ow > 0, "pool window larger than the input");
  if (n == 0) return MIRA_CUDA_OK;
  const int threads = 256;
  if (x_i8 != nullptr) {
    MIRA_CHECK_ARG(out_f32 == nullptr && out_i8 != nullptr, "int8 pooling produces int8 only");
    MIRA_CHECK_ARG(ldc_in % 16 == 0 && ldc_out_i8 == ldc_in, "int8 pooling keeps the padded channel stride");
    MIRA_CHECK_ARG(out_scale > 0.0f, "requant scale must be positive");
    const uint32_t pq = quant_byte_host(pad_value, out_scale);
    const int64_t work = n * oh * ow * (ldc_in / 16);
    maxpool_i8_kernel<<<grid_for(dev, work, threads), threads, 0, dev->stream>>>(
        x_i8, int(n), int(h), int(w), ldc_in, int(size), int(stride), int(pad), static_cast<int8_t>(pq & 0xff),
        int(oh), int(ow), out_i8, ldc_out_i8);
    return after_launch("maxpool_i8_kernel");
  }
  MIRA_CHECK_ARG(x_f32 != nullptr && (out_f32 != nullptr || out_i8 != nullptr), "maxpool needs an input and an output");
  if (out_i8 != nullptr) MIRA_CHECK_ARG(ldc_out_i8 % 4 == 0 && ldc_out_i8 >= c && out_scale > 0.0f, "bad int8 output");
  I8Dst o8{out_i8, ldc_out_i8, 0, 0, 16};
  if (out_i8 != nullptr && i8_layout == MIRA_LAYOUT_CP) {
    o8.cp = 1;
    o8.guard = int(cp_guard(ow));
    o8.chunk = n * (oh + 2) * (ow + 2) * 16;
  }
  const auto a16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
  if (size == 3 && c % 4 == 0 && ldc_in % 4 == 0 && a16(x_f32) &&
      (out_f32 == nullptr || (ldc_out_f32 % 4 == 0 && a16(out_f32))) &&
      (out_i8 == nullptr || (ldc_out_i8 % 4 == 0 && (reinterpret_cast<uintptr_t>(out_i8) & 3u) == 0))) {
    const int c4 = int(c / 4);
    const int tx = c4 < 64 ? c4 : 64;
    const int ty = threads / tx < 1 ? 1 : threads / tx;
    const int64_t orows = n * oh;
    const dim3 grid(unsigned((ow + ty - 1) / ty), unsigned(orows < 65535 ? orows : 65535));
    maxpool3_f32_kernel<<<grid, dim3(tx, ty), 0, dev->stream>>>(
        x_f32, int(n), int(h), int(w), int(c), ldc_in, int(stride), int(pad), pad_value, int(oh), int(ow), out_f32,
        ldc_out_f32, o8, make_qscale(out_i8 != nullptr ? out_scale : 1.0f));
    return after_launch("maxpool3_f32_kernel");
  }
  // threads: x = groups of 4 channels (at most 64), y = output columns; blocks: columns x rows
  const int c4 = int((c + 3) / 4);
  const int tx = c4 < 64 ? c4 : 64;
  const int ty = threads / tx < 1 ? 1 : threads / tx;
  const int64_t orows = n * oh;
  const dim3 grid(unsigned((ow + ty - 1) / ty), unsigned(orows < 65535 ? orows : 65535));
  maxpool_f32_kernel<<<grid, dim3(tx, ty), 0, dev->stream>>>(
      x_f32, int(n), int(h), int(w), int(c), ldc_in, int(size), int(stride), int(pad), pad_value, int(oh), int(ow),
      out_f32, ldc_out_f32, o8, make_qscale(out_i8 != nullptr ? out_scale : 1.0f));
  return after_launch("maxpool_f32_kernel");
}

extern "C" int mira_cuda_mean_hw_nhwc(const float* x, int64_t n, int64_t hw, int64_t c, int64_t ldc, float* out_f32,
                                      int8_t* out_i8, int64_t ld_i8, float out_scale) {
  MIRA_GET_DEVICE(dev);
  MIRA_CHECK_ARG(n >= 0 && hw > 0 && hw < (1 << 20) && c > 0 && ldc >= c, "bad mean shape");
  MIRA_CHECK_ARG(out_f32 != nullptr || out_i8 != nullptr, "mean has no output");
  if (out_i8 != nullptr) MIRA_CHECK_ARG(ld_i8 >= c && out_scale > 0.0f, "bad int8 output");
  if (n == 0) return MIRA_CUDA_OK;
  const int threads = 128;
  mean_hw_kernel<<<grid_for(dev, n * c, threads), threads, 0, dev->stream>>>(
      x, int(n), int(hw), int(c), ldc, out_f32, out_i8, ld_i8, make_qscale(out_i8 != nullptr ? out_scale : 1.0f));
  return after_launch("mean_hw_kernel");
}

extern "C" int mira_cuda_im2col_f32(const float* x, int64_t n, int64_t h, int64_t w, int64_t c, int64_t ldc, int64_t kh,
                                    int64_t kw, int64_t stride_h, int64_t stride_w, int64_t pad_h, int64_t pad_w,
                                    int64_t dil_h, int64_t dil_w, float* out, int64_t ld_out) {
  MIRA_GET_DEVICE(dev);
  MIRA_CHECK_ARG(n >= 0 && h > 0 && w > 0 && c > 0 && ldc >= c && kh > 0 && kw > 0, "bad im2col shape");
  MIRA_CHECK_ARG(stride_h > 0 && stride_w > 0 && dil_h > 0 && dil_w > 0 && pad_h >= 0 && pad_w >= 0, "bad im2col geometry");
  MIRA_CHECK_ARG(ld_out >= kh * kw * c, "im2col rows hold kh * kw * c values");
  MIRA_CHECK_ARG(x != nullptr && out != nullptr, "im2col needs an input and an output");
  const int64_t oh = (h + 2 * pad_h - dil_h * (kh - 1) - 1) / stride_h + 1;
  const int64_t ow = (w + 2 * pad_w - dil_w * (kw - 1) - 1) / stride_w + 1;
  MIRA_CHECK_ARG(oh > 0 && ow > 0, "kernel larger than the padded input");
  if (n == 0) return MIRA_CUDA_OK;
  const int threads = 256;
  im2col_f32_kernel<<<grid_for(dev, n * oh * ow * kh * kw * 32, threads), threads, 0, dev->stream>>>(
      x, int(n), int(h), int(w), int(c), ldc, int(kh), int(kw), int(stride_h), int(stride_w), int(pad_h), int(pad_w),
      int(dil_h), int(dil_w), int(oh), int(ow), out, ld_out);
  return after_launch("im2col_f32_kernel");
}

// The TMA-staged depthwise 3x3 kernel (dw_staged.cuh) for an NHWC input of elements T (f32 rows of
// c values, or int8 rows of ldx bytes): picks the unit shape (R output rows x cc channels) so that
// two input windows fit in shared memory, encodes the 4-D tensor map and launches one persistent
// CTA per SM (more when the windows are small).  Returns -1 when the shape does not suit it.
template <typename T>
static int launch_dw_staged(DeviceState* dev, const T* x, int64_t ldx, const DwParams& p, const void* wt,
                            const QdwScales& sc) {
  constexpr int64_t es = sizeof(T);
  const int S = p.sh;
  const int oxt = S == 1 ? 4 : 2;
  const int64_t tiles = (p.ow + oxt - 1) / oxt;
  const int64_t cols_in = (tiles * oxt - 1) * S + 3;
  if (cols_in > 256 || (ldx * es) % 16 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) != 0) return -1;
  const int64_t unit_c = 16 / es;                               // channels per 16 bytes
  const int64_t c_pad = (p.c + unit_c - 1) / unit_c * unit_c;
  const int64_t budget = 55 * 1024;                             // bytes per window buffer (2 CTAs per SM)
  // the unit shape that re-reads the fewest input rows (R / rows_in largest), with enough tasks
  // (4-channel groups x column tiles x rows) for the CTA's threads; wider channel chunks on ties
  int64_t cc = 0, rows = 0;
  double best = -1.0;
  for (int64_t c_try = c_pad < 256 ? c_pad : 256; c_try >= unit_c; c_try = c_try > unit_c ? (c_try / 2 + unit_c - 1) / unit_c * unit_c : 0) {
    for (int64_t r = 8; r >= 1; --r) {
      const int64_t r_eff = r < p.oh ? r : p.oh;
      if ((r_eff - 1) * S + 3 > 0 && ((r_eff - 1) * S + 3) * cols_in * c_try * es > budget) continue;
      const double reuse = double(r_eff) / double((r_eff - 1) * S + 3);
      const double fill = std::min(1.0, double((c_try / 4) * tiles * r_eff) / DWS_THREADS);
      const double score = reuse * fill;
      if (score > best + 1e-9) { best = score; cc = c_try; rows = r_eff; }
      break;   // the largest r that fits is the best for this chunk width
    }
    if (c_try == unit_c) break;
  }
  if (rows == 0) return -1;
  if (rows > p.oh) rows = p.oh;
  const int64_t rows_in = (rows - 1) * S + 3;
  DwsParams q;
  std::memset(&q, 0, sizeof(q));
  q.p = p;
  q.sc = sc;
  q.rows = int(rows); q.cc = int(cc); q.cols_in = int(cols_in); q.rows_in = int(rows_in); q.tiles = int(tiles);
  q.bands = int((p.oh + rows - 1) / rows);
  q.chunks = int((p.c + cc - 1) / cc);
  const int64_t units = int64_t(p.n) * q.bands * q.chunks;
  if (units >= (int64_t(1) << 31)) return -1;
  q.units = int(units);
  q.box_bytes = int(rows_in * cols_in * cc * es);
  q.err = device_err_ptr();
  CUtensorMap map;
  const cuuint64_t dims[4] = {cuuint64_t(ldx), cuuint64_t(p.w), cuuint64_t(p.h), cuuint64_t(p.n)};
  const cuuint64_t strides[3] = {cuuint64_t(ldx * es), cuuint64_t(ldx * es * p.w), cuuint64_t(ldx * es * p.w * p.h)};
  const cuuint32_t box[4] = {cuuint32_t(cc), cuuint32_t(cols_in), cuuint32_t(rows_in), 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = g_encode_tiled(&map, es == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 4,
                                    const_cast<T*>(x), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                    CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(MIRA_CUDA_ECUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  const int buf_bytes = (q.box_bytes + 127) & ~127;
  const int smem = 128 + 2 * buf_bytes + 64;
  int per_sm = 232448 / (smem + 1024);
  if (per_sm > 2) per_sm = 2;   // two CTAs of 256 threads at up to 128 registers fill an SM
  if (per_sm < 1) return -1;
  const int64_t grid64 = units < int64_t(dev->sm_count) * per_sm ? units : int64_t(dev->sm_count) * per_sm;
  auto launch = [&](auto kernel) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    kernel<<<unsigned(grid64), DWS_THREADS, smem, dev->stream>>>(map, wt, q);
  };
  if (S == 1) launch(dw_staged_kernel<T, 1, 4>);
  else launch(dw_staged_kernel<T, 2, 2>);
  return after_launch("dw_staged_kernel");
}

extern "C" int mira_cuda_dwconv2d_nhwc(const float* x, int64_t n, int64_t h, int64_t w, int64_t c, const float* wt,
                                       int64_t kh, int64_t kw, int64_t stride_h, int64_t stride_w, int64_t pad_h,
                                       int64_t pad_w, int64_t dil_h, int64_t dil_w, const mira_epilogue* epi) {
  MIRA_GET_DEVICE(dev);
  MIRA_CHECK_ARG(n >= 0 && h > 0 && w > 0 && c > 0 && kh > 0 && kw > 0, "bad dwconv shape");
  MIRA_CHECK_ARG(stride_h > 0 && stride_w > 0 && dil_h > 0 && dil_w > 0 && pad_h >= 0 && pad_w >= 0, "bad dwconv geometry");
  MIRA_CHECK_ARG(epi != nullptr && epi->n_steps >= 0 && epi->n_steps <= MIRA_EPI_MAX_STEPS, "bad epilogue");
  MIRA_CHECK_ARG(epi->out_f32 != nullptr || epi->out_i8 != nullptr, "dwconv has no output");
  const int64_t oh = (h + 2 * pad_h - dil_h * (kh - 1) - 1) / stride_h + 1;
  const int64_t ow = (w + 2 * pad_w - dil_w * (kw - 1) - 1) / stride_w + 1;
  MIRA_CHECK_ARG(oh > 0 && ow > 0, "kernel larger than the padded input");
  if (n == 0) return MIRA_CUDA_OK;
  DwParams p;
  std::memset(&p, 0, sizeof(p));
  p.n = int(n); p.h = int(h); p.w = int(w); p.c = int(c); p.oh = int(oh); p.ow = int(ow);
  p.kh = int(kh); p.kw = int(kw); p.sh = int(stride_h); p.sw = int(stride_w); p.ph = int(pad_h); p.pw = int(pad_w);
  p.dh = int(dil_h); p.dw = int(dil_w);
  p.n_steps = epi->n_steps;
  for (int s = 0; s < epi->n_steps; ++s) p.steps[s] = epi->steps[s];
  p.out_f32 = epi->out_f32; p.ld_f32 = epi->ld_f32; p.out_i8 = epi->out_i8; p.ld_i8 = epi->ld_i8;
  p.q = make_qscale(epi->out_i8 != nullptr ? epi->out_scale : 1.0f);
  const int threads = 256;
  bool vec = c % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(wt) & 15) == 0;
  if (epi->out_f32 != nullptr) vec = vec && epi->ld_f32 % 4 == 0 && (reinterpret_cast<uintptr_t>(epi->out_f32) & 15) == 0;
  if (epi->out_i8 != nullptr) vec = vec && epi->ld_i8 % 4 == 0 && (reinterpret_cast<uintptr_t>(epi->out_i8) & 3) == 0;
  for (int s = 0; s < epi->n_steps; ++s) {
    const mira_epi_step& st = epi->steps[s];
    if (st.operand == MIRA_OPND_CHANNEL || st.operand == MIRA_OPND_FULL)
      vec = vec && (reinterpret_cast<uintptr_t>(st.ptr) & 15) == 0 && (st.operand != MIRA_OPND_FULL || st.ld % 4 == 0);
  }
  if (vec && kh == 3 && kw == 3 && dil_h == 1 && dil_w == 1 && stride_h == stride_w && stride_h <= 2) {
    // the staged kernel wins on the narrower late layers (measured on MobileNetV2's: 28 x 28 and
    // smaller outputs); the early wide layers stay on the unstaged one
    if (oh <= 28) {
      const int rc = launch_dw_staged<float>(dev, x, c, p, wt, QdwScales{nullptr, nullptr, nullptr});
      if (rc >= 0) return rc;
    }
    // threadIdx.x: 4-channel groups (all of them up to 256 threads), threadIdx.y: groups of
    // output columns, so narrow late layers with many channels keep every thread busy
    const int oxt = stride_h == 1 ? 4 : 2;
    const int c4 = int(c / 4);
    const int64_t col_groups = (ow + oxt - 1) / oxt;
    const int tx = c4 < threads ? c4 : threads;
    const int ty_max = threads / tx;
    const int ty = int(col_groups < ty_max ? col_groups : ty_max);
    const int64_t orows = n * oh;
    const dim3 grid(unsigned((col_groups + ty - 1) / ty), unsigned(orows < 65535 ? orows : 65535));
    if (stride_h == 1) dwconv3x3_kernel<1, 4><<<grid, dim3(tx, ty), 0, dev->stream>>>(x, wt, p);
    else dwconv3x3_kernel<2, 2><<<grid, dim3(tx, ty), 0, dev->stream>>>(x, wt, p);
    return after_launch("dwconv3x3_kernel");
  }
  if (vec) {
    const int c4 = int(c / 4);
    const int tx = c4 < 32 ? c4 : 32;
    const int ty = threads / tx;
    const int64_t orows = n * oh;
    const dim3 grid(unsigned((ow + ty - 1) / ty), unsigned(orows < 65535 ? orows : 65535));
    dwconv4_kernel<<<grid, dim3(tx, ty), 0, dev->stream>>>(x, wt, p);
    return after_launch("dwconv4_kernel");
  }
  dwconv_kernel<<<grid_for(dev, n * oh * ow * c, threads), threads, 0, dev->stream>>>(x, wt, p);
  return after_launch("dwconv_kernel");
}

extern "C" int mira_cuda_qdwconv2d_nhwc(const int8_t* x, int64_t n, int64_t h, int64_t w, int64_t c, int64_t ldx,
                                        const int8_t* wq, int64_t kh, int64_t kw, int64_t stride_h, int64_t stride_w,
                                        int64_t pad_h, int64_t pad_w, int64_t dil_h, int64_t dil_w,
                                        const mira_dequant* dq, const mira_epilogue* epi) {
  MIRA_GET_DEVICE(dev);
  MIRA_CHECK_ARG(n >= 0 && h > 0 && w > 0 && c > 0 && c % 4 == 0 && ldx >= c && ldx % 4 == 0 && kh > 0 && kw > 0,
                 "bad int8 depthwise shape (channels must be a multiple of 4)");
  MIRA_CHECK_ARG(kh * kw * 127 * 127 < (int64_t(1) << 24), "int8 depthwise kernel too large for exact f32 sums");
  MIRA_CHECK_ARG(stride_h > 0 && stride_w > 0 && dil_h > 0 && dil_w > 0 && pad_h >= 0 && pad_w >= 0,
                 "bad int8 depthwise geometry");
  MIRA_CHECK_ARG((reinterpret_cast<uintptr_t>(x) & 3) == 0 && (reinterpret_cast<uintptr_t>(wq) & 3) == 0,
                 "int8 depthwise operands must be 4-byte aligned");
  MIRA_CHECK_ARG(dq != nullptr && dq->scale64 != nullptr && dq->scale_hi != nullptr && dq->scale_lo != nullptr &&
                     (reinterpret_cast<uintptr_t>(dq->scale_hi) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(dq->scale_lo) & 15) == 0,
                 "int8 depthwise needs per-channel dequant scales (16-byte aligned)");
  MIRA_CHECK_ARG(epi != nullptr && epi->n_steps >= 0 && epi->n_steps <= MIRA_EPI_MAX_STEPS, "bad epilogue");
  MIRA_CHECK_ARG(epi->out_f32 != nullptr || epi->out_i8 != nullptr, "int8 depthwise has no output");
  MIRA_CHECK_ARG(epi->i8_layout == MIRA_LAYOUT_NHWC, "int8 depthwise writes NHWC rows");
  if (epi->out_f32 != nullptr)
    MIRA_CHECK_ARG(epi->ld_f32 % 4 == 0 && (reinterpret_cast<uintptr_t>(epi->out_f32) & 15) == 0,
                   "f32 output must hold 16-byte aligned rows");
  if (epi->out_i8 != nullptr)
    MIRA_CHECK_ARG(epi->ld_i8 % 4 == 0 && (reinterpret_cast<uintptr_t>(epi->out_i8) & 3) == 0,
                   "int8 output must hold 4-byte aligned rows");
  for (int s = 0; s < epi->n_steps; ++s) {
    const mira_epi_step& st = epi->steps[s];
    if (st.operand == MIRA_OPND_CHANNEL || st.operand == MIRA_OPND_FULL)
      MIRA_CHECK_ARG((reinterpret_cast<uintptr_t>(st.ptr) & 15) == 0 && (st.operand != MIRA_OPND_FULL || st.ld % 4 == 0),
                     "epilogue operands must be 16-byte aligned");
  }
  const int64_t oh = (h + 2 * pad_h - dil_h * (kh - 1) - 1) / stride_h + 1;
  const int64_t ow = (w + 2 * pad_w - dil_w * (kw - 1) - 1) / stride_w + 1;
  MIRA_CHECK_ARG(oh > 0 && ow > 0, "kernel larger than the padded input");
  if (n == 0) return MIRA_CUDA_OK;
  DwParams p;
  std::memset(&p, 0, sizeof(p));
  p.n = int(n); p.h = int(h); p.w = int(w); p.c = int(c); p.oh = int(oh); p.ow = int(ow);
  p.kh = int(kh); p.kw = int(kw); p.sh = int(stride_h); p.sw = int(stride_w); p.ph = int(pad_h); p.pw = int(pad_w);
  p.dh = int(dil_h); p.dw = int(dil_w);
  p.n_steps = epi->n_steps;
  for (int s = 0; s < epi->n_steps; ++s) p.steps[s] = epi->steps[s];
  p.out_f32 = epi->out_f32; p.ld_f32 = epi->ld_f32; p.out_i8 = epi->out_i8; p.ld_i8 = epi->ld_i8;
  p.q = make_qscale(epi->out_i8 != nullptr ? epi->out_scale : 1.0f);
  const QdwScales sc{dq->scale_hi, dq->scale_lo, dq->scale64};
  const uint32_t* wt = reinterpret_cast<const uint32_t*>(wq);
  const int threads = 256;
  const int c4 = int(c / 4);
  const int64_t orows = n * oh;
  if (kh == 3 && kw == 3 && dil_h == 1 && dil_w == 1 && stride_h == stride_w && stride_h <= 2) {
    const int oxt = stride_h == 1 ? 4 : 2;
    const int64_t col_groups = (ow + oxt - 1) / oxt;
    const int tx = c4 < threads ? c4 : threads;
    const int ty_max = threads / tx;
    const int ty = int(col_groups < ty_max ? col_groups : ty_max);
    const dim3 grid(unsigned((col_groups + ty - 1) / ty), unsigned(orows < 65535 ? orows : 65535));
    if (stride_h == 1) qdwconv3x3_kernel<1, 4><<<grid, dim3(tx, ty), 0, dev->stream>>>(x, ldx, wt, sc, p);
    else qdwconv3x3_kernel<2, 2><<<grid, dim3(tx, ty), 0, dev->stream>>>(x, ldx, wt, sc, p);
    return after_launch("qdwconv3x3_kernel");
  }
  const int tx = c4 < 32 ? c4 : 32;
  const int ty = threads / tx;
  const dim3 grid(unsigned((ow + ty - 1) / ty), unsigned(orows < 65535 ? orows : 65535));
  qdwconv4_kernel<<<grid, dim3(tx, ty), 0, dev->stream>>>(x, ldx, wt, sc, p);
  return after_launch("qdwconv4_kernel");
}

extern "C" int mira_cuda_nchw_to_nhwc_f32(const float* x, int64_t n, int64_t c, int64_t h, int64_t w, float* y,
                                          int64_t ldc) {
  MIRA_GET_DEVICE(dev);
  MIRA_CHECK_ARG(n >= 0 && c > 0 && h > 0 && w > 0 && ldc >= c && n < 65536, "bad layout-change shape");
  if (n == 0) return MIRA_CUDA_OK;
  const dim3 grid(unsigned((h * w + 31) / 32), unsigned((c + 31) / 32), unsigned(n));
  nchw_to_nhwc_kernel<<<grid, dim3(32, 8), 0, dev->stream>>>(x, int(c), int(h * w), y, ldc);
  return after_launch("nchw_to_nhwc_kernel");
}

extern "C" int mira_cuda_nhwc_to_nchw_f32(const float* x, int64_t n, int64_t h, int64_t w, int64_t c, int64_t ldc,
                                          float* y) {
  MIRA_GET_DEVICE(dev);
  MIRA_CHECK_ARG(n >= 0 && c > 0 && h > 0 && w > 0 && ldc >= c && n < 65536, "bad layout-change shape");
  if (n == 0) return MIRA_CUDA_OK;
  const dim3 grid(unsigned((h * w + 31) / 32), unsigned((c + 31) / 32), unsigned(n));
  nhwc_to_nchw_kernel<<<grid, dim3(32, 8), 0, dev->stream>>>(x, int(c), int(h * w), ldc, y);
  return after_launch("nhwc_to_nchw_kernel");
}

// ---------------------------------------------------------------- sequence (transformer) ops

namespace mira {

static int pw_leaves_rec(int start, int n, PwLeaves& pw) {
  if (n <= 128) {
    pw.start[pw.count] = start;
    return pw.count++;
  }
  int n2 = n / 2;
  n2 -= n2 % 8;
  const int a = pw_leaves_rec(start, n2, pw);
  const int b = pw_leaves_rec(start + n2, n - n2, pw);
  pw.left[pw.nodes] = static_cast<uint8_t>(a);
  pw.right[pw.nodes] = static_cast<uint8_t>(b);
  return PW_MAX_LEAVES + pw.nodes++;
}

// NumPy's pairwise recursion cut into leaves of at most 128 elements (rows up to MIRA_ROW_MAX
// give at most 128 leaves of more than 64 elements each).
static void pw_leaves(int n, PwLeaves& pw) {
  std::memset(&pw, 0, sizeof(pw));
  pw.n = n;
  if (n >= 8) pw_leaves_rec(0, n, pw);
  pw.start[pw.count] = n;
}

// Whether NumPy's pairwise recursion over d elements is a perfect binary tree of NL leaves of L
// elements (layernorm_tree_kernel): NL a power of two up to 16, L a multiple of 8 of at most 128,
// and more than 64 when the range is split (halves of multiples of 8 split exactly).
static bool ln_tree_shape(int64_t d, int& L, int& NL) {
  for (int nl = 1; nl <= 16; nl *= 2) {
    if (d % nl != 0) continue;
    const int64_t l = d / nl;
    if (l % 8 == 0 && l <= 128 && (nl == 1 ? l >= 8 : l > 64)) {
      L = int(l);
      NL = nl;
      return true;
    }
  }
  return false;
}

static bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

static int row_grid(const DeviceState* dev, int64_t rows) {
  int64_t blocks = (rows + ROW_WARPS - 1) / ROW_WARPS;
  const int64_t cap = int64_t(dev->sm_count) * 8;
  return static_cast<int>(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
}

}  // namespace mira

extern "C" int mira_cuda_layernorm_rows(const float* x, int64_t rows, int64_t d, int64_t ld_x, const float* gamma,
                                        const float* beta, float eps, float* out_f32, int64_t ld_f32, int8_t* out_i8,
                                        int64_t ld_i8, float out_scale) {
  MIRA_GET_DEVICE(dev);
  MIRA_CHECK_ARG(rows >= 0 && d > 0 && d <= MIRA_ROW_MAX && ld_x >= d, "bad layernorm shape");
  MIRA_CHECK_ARG(x != nullptr && gamma != nullptr && beta != nullptr, "layernorm needs x, gamma and beta");
  MIRA_CHECK_ARG(out_f32 != nullptr || out_i8 != nullptr, "layernorm has no output");
  if (out_f32 != nullptr) MIRA_CHECK_ARG(ld_f32 >= d, "bad f32 output stride");
  if (out_i8 != nullptr) MIRA_CHECK_ARG(ld_i8 >= d && out_scale > 0.0f, "bad int8 output");
  if (rows == 0) return MIRA_CUDA_OK;
  LnParams p;
  std::memset(&p, 0, sizeof(p));
  p.x = x; p.rows = rows; p.ld_x = ld_x; p.d = int(d); p.gamma = gamma; p.beta = beta; p.eps = eps;
  p.out = out_f32; p.ld_out = ld_f32; p.out_i8 = out_i8; p.ld_i8 = ld_i8;
  p.q = make_qscale(out_i8 != nullptr ? out_scale : 1.0f);
  pw_leaves(int(d), p.pw);
  int L = 0, NL = 0;
  if (ln_tree_shape(d, L, NL) && (L == 96 || L == 128) && aligned16(x) && ld_x % 4 == 0 && aligned16(gamma) &&
      aligned16(beta) && (out_f32 == nullptr || (aligned16(out_f32) && ld_f32 % 4 == 0)) &&
      (out_i8 == nullptr || ((reinterpret_cast<uintptr_t>(out_i8) & 3u) == 0 && ld_i8 % 4 == 0))) {
    // 2 chains per lane (4 lanes per leaf) while a row fits a warp, else 4
    const int lanes_per_row = NL <= 8 ? 4 * NL : 2 * NL;
    const int64_t rows_per_block = (LN_TREE_THREADS / 32) * (32 / lanes_per_row);
    const int64_t blocks = (rows + rows_per_block - 1) / rows_per_block;
    const int64_t cap = int64_t(dev->sm_count) * 16;
    const int grid = int(blocks < cap ? blocks : cap);
    auto kern = L == 96 ? (NL == 1   ? layernorm_tree_kernel<96, 1, 2>
                           : NL == 2 ? layernorm_tree_kernel<96, 2, 2>
                           : NL == 4 ? layernorm_tree_kernel<96, 4, 2>
                           : NL == 8 ? layernorm_tree_kernel<96, 8, 2>
                                     : layernorm_tree_kernel<96, 16, 4>)
                        : (NL == 1   ? layernorm_tree_kernel<128, 1, 2>
                           : NL == 2 ? layernorm_tree_kernel<128, 2, 2>
                           : NL == 4 ? layernorm_tree_kernel<128, 4, 2>
                           : NL == 8 ? layernorm_tree_kernel<128, 8, 2>
                                     : layernorm_tree_kernel<128, 16, 4>);
    kern<<<grid, LN_TREE_THREADS, 0, dev->stream>>>(p);
    return after_launch("layernorm_tree_kernel");
  }
  if (d >= 8 && p.pw.count <= 16) {
    // leaves of at most 128 elements, 4 per round, chains of at most 16 in registers
    if (p.pw.count <= 4) layernorm_rows_reg_kernel<1><<<row_grid(dev, rows), ROW_WARPS * 32, 0, dev->stream>>>(p);
    else if (p.pw.count <= 8) layernorm_rows_reg_kernel<2><<<row_grid(dev, rows), ROW_WARPS * 32, 0, dev->stream>>>(p);
    else layernorm_rows_reg_kernel<4><<<row_grid(dev, rows), ROW_WARPS * 32, 0, dev->stream>>>(p);
    return after_launch("layernorm_rows_reg_kernel");
  }
  layernorm_rows_kernel<<<row_grid(dev, rows), ROW_WARPS * 32, 0, dev->stream>>>(p);
  return after_launch("layernorm_rows_kernel");
}

extern "C" int mira_cuda_softmax_rows(const float* x, int64_t rows, int64_t n, int64_t ld_x, float* out,
                                      int64_t ld_out) {
  MIRA_GET_DEVICE(dev);
  MIRA_CHECK_ARG(rows >= 0 && n > 0 && n <= MIRA_ROW_MAX && ld_x >= n && ld_out >= n, "bad softmax shape");
  MIRA_CHECK_ARG(x != nullptr && out != nullptr, "softmax needs an input and an output");
  if (rows == 0) return MIRA_CUDA_OK;
  SoftmaxParams p;
  std::memset(&p, 0, sizeof(p));
  p.x = x; p.rows = rows; p.ld_x = ld_x; p.out = out; p.ld_out = ld_out;
  pw_leaves(int(n), p.pw);
  softmax_rows_kernel<<<row_grid(dev, rows), ROW_WARPS * 32, 0, dev->stream>>>(p);
  return after_launch("softmax_rows_kernel");
}

extern "C" int mira_cuda_embed_rows(const float* table, int64_t vocab, int64_t d, const int32_t* idx, int64_t rows,
                                    const float* addend, int64_t addend_rows, float* out, int64_t ld_out) {
  MIRA_GET_DEVICE(dev);
  MIRA_CHECK_ARG(vocab > 0 && d > 0 && rows >= 0 && ld_out >= d, "bad embedding shape");
  MIRA_CHECK_ARG(table != nullptr && idx != nullptr && out != nullptr, "embedding needs a table, indices and an output");
  if (addend != nullptr) MIRA_CHECK_ARG(addend_rows > 0, "addend needs at least one row");
  if (rows == 0) return MIRA_CUDA_OK;
  EmbedParams p;
  p.table = table; p.vocab = vocab; p.d = d; p.idx = idx; p.rows = rows; p.addend = addend;
  p.addend_rows = addend_rows; p.out = out; p.ld_out = ld_out; p.err = device_err_ptr();
  const int threads = 256;
  embed_rows_kernel<<<grid_for(dev, rows * d, threads), threads, 0, dev->stream>>>(p);
  return after_launch("embed_rows_kernel");
}

extern "C" int mira_cuda_copy_view_f32(int64_t n0, int64_t n1, int64_t n2, int64_t n3, const mira_view4* src,
                                       const mira_view4* dst) {
  MIRA_GET_DEVICE(dev);
  MIRA_CHECK_ARG(n0 >= 0 && n1 >= 0 && n2 >= 0 && n3 >= 0, "bad view shape");
  MIRA_CHECK_ARG(src != nullptr && dst != nullptr && src->ptr != nullptr && dst->ptr != nullptr, "null view");
  const int64_t total = n0 * n1 * n2 * n3;
  if (total == 0) return MIRA_CUDA_OK;
  View4 v;
  v.n[0] = n0; v.n[1] = n1; v.n[2] = n2; v.n[3] = n3;
  v.src = static_cast<const float*>(src->ptr);
  v.dst = static_cast<float*>(dst->ptr);
  for (int i = 0; i < 4; ++i) { v.ss[i] = src->stride[i]; v.ds[i] = dst->stride[i]; }
  const int threads = 256;
  copy_view_kernel<<<grid_for(dev, (total / (n3 > 0 ? n3 : 1)) * 32, threads), threads, 0, dev->stream>>>(v);
  return after_launch("copy_view_kernel");
}

extern "C" int mira_cuda_elementwise_f32(int32_t op, int64_t n0, int64_t n1, int64_t n2, int64_t n3,
                                         const mira_view4* a, const mira_view4* b, float scalar, int32_t swapped,
                                         const mira_view4* out) {
  MIRA_GET_DEVICE(dev);
  const bool unary = op >= MIRA_EPI_RELU && op <= MIRA_EPI_TANH;
  MIRA_CHECK_ARG(unary || (op >= MIRA_EPI_ADD && op <= MIRA_EPI_MINIMUM), "unknown element-wise op");
  MIRA_CHECK_ARG(n0 >= 0 && n1 >= 0 && n2 >= 0 && n3 >= 0, "bad element-wise shape");
  MIRA_CHECK_ARG(a != nullptr && out != nullptr, "element-wise op needs an input and an output view");
  const int64_t total = n0 * n1 * n2 * n3;
  if (total == 0) return MIRA_CUDA_OK;
  MIRA_CHECK_ARG(a->ptr != nullptr && out->ptr != nullptr && (b == nullptr || b->ptr != nullptr), "null view");
  EltParams p;
  std::memset(&p, 0, sizeof(p));
  p.n[0] = n0; p.n[1] = n1; p.n[2] = n2; p.n[3] = n3;
  p.a = static_cast<const float*>(a->ptr);
  p.b = (!unary && b != nullptr) ? static_cast<const float*>(b->ptr) : nullptr;
  p.out = static_cast<float*>(out->ptr);
  for (int i = 0; i < 4; ++i) {
    p.as[i] = a->stride[i]; p.os[i] = out->stride[i]; p.bs[i] = p.b != nullptr ? b->stride[i] : 0;
  }
  p.scalar = scalar;
  p.op = op;
  p.unary = unary ? 1 : 0;
  p.swapped = swapped ? 1 : 0;
  const int threads = 256;
  elementwise_f32_kernel<<<grid_for(dev, (total / (n3 > 0 ? n3 : 1)) * 32, threads), threads, 0, dev->stream>>>(p);
  return after_launch("elementwise_f32_kernel");
}

namespace mira {

static int dyn_window(DeviceState* dev, const mira_view4* src, const mira_view4* dst, const int64_t* n,
                      const int64_t* dims, const int32_t* start, int64_t rank, int update) {
  MIRA_CHECK_ARG(src != nullptr && dst != nullptr && n != nullptr && dims != nullptr, "null argument");
  MIRA_CHECK_ARG(rank >= 0 && rank <= 4 && (rank == 0 || start != nullptr), "start vector: rank 0..4, device i32");
  int64_t total = 1;
  for (int i = 0; i < 4; ++i) {
    MIRA_CHECK_ARG(n[i] >= 0 && n[i] <= dims[i], "the window must fit in the full shape");
    MIRA_CHECK_ARG(i >= 4 - rank || n[i] == dims[i], "dimensions without a start entry are copied whole");
    total *= n[i];
  }
  if (total == 0) return MIRA_CUDA_OK;
  MIRA_CHECK_ARG(src->ptr != nullptr && dst->ptr != nullptr, "null view");
  DynWindowParams p;
  std::memset(&p, 0, sizeof(p));
  p.src = static_cast<const uint32_t*>(src->ptr);
  p.dst = static_cast<uint32_t*>(dst->ptr);
  for (int i = 0; i < 4; ++i) {
    p.ss[i] = src->stride[i]; p.ds[i] = dst->stride[i]; p.n[i] = n[i]; p.dims[i] = dims[i];
  }
  p.start = start;
  p.rank = int(rank);
  p.update = update;
  const int threads = 256;
  dyn_window_kernel<<<grid_for(dev, (total / (n[3] > 0 ? n[3] : 1)) * 32, threads), threads, 0, dev->stream>>>(p);
  return after_launch("dyn_window_kernel");
}

}  // namespace mira

extern "C" int mira_cuda_dynamic_slice(const mira_view4* x, const int64_t* x_dims, const int32_t* start, int64_t rank,
                                       const int64_t* size, const mira_view4* out) {
  MIRA_GET_DEVICE(dev);
  return dyn_window(dev, x, out, size, x_dims, start, rank, 0);
}

extern "C" int mira_cuda_dynamic_update_slice(const mira_view4* x, const int64_t* x_dims, const mira_view4* upd,
                                              const int64_t* upd_dims, const int32_t* start, int64_t rank) {
  MIRA_GET_DEVICE(dev);
  return dyn_window(dev, upd, x, upd_dims, x_dims, start, rank, 1);
}

namespace mira {

// The f32 batched matmul behind mira_cuda_bmm_f32 (b_scale == nullptr: b holds f32) and
// mira_cuda_bmm_f32_w8 (b holds int8 weights, dequantized with b_scale[n] as tiles are loaded).
static int bmm_launch(DeviceState* dev, int64_t batch0, int64_t batch1, int64_t m, int64_t n, int64_t k,
                      const mira_view4* a, const mira_view4* b, const float* b_scale, const mira_bmm_epilogue* epi) {
  MIRA_CHECK_ARG(batch0 >= 0 && batch1 > 0 && m >= 0 && n >= 0 && k >= 0, "bad bmm shape");
  MIRA_CHECK_ARG(a != nullptr && b != nullptr && epi != nullptr, "bmm needs a, b and an epilogue");
  MIRA_CHECK_ARG(k == 0 || (a->ptr != nullptr && b->ptr != nullptr), "null bmm operand");
  MIRA_CHECK_ARG(epi->n_steps >= 0 && epi->n_steps <= MIRA_EPI_MAX_STEPS, "bad epilogue");
  MIRA_CHECK_ARG(epi->out_f32.ptr != nullptr || epi->out_i8.ptr != nullptr, "bmm has no output");
  if (epi->out_i8.ptr != nullptr) MIRA_CHECK_ARG(epi->out_scale > 0.0f, "requant scale must be positive");
  for (int s = 0; s < epi->n_steps; ++s) {
    const mira_bmm_step& st = epi->steps[s];
    MIRA_CHECK_ARG(st.operand == MIRA_OPND_NONE || st.operand == MIRA_OPND_SCALAR ||
                       (st.operand == MIRA_OPND_VIEW && st.view.ptr != nullptr),
                   "bmm epilogue operands are scalars or views");
  }
  const int64_t batches = batch0 * batch1;
  if (batches == 0 || m == 0 || n == 0) return MIRA_CUDA_OK;
  BmmParams p;
  std::memset(&p, 0, sizeof(p));
  p.batches = batches; p.batch1 = batch1; p.m = m; p.n = n; p.k = k;
  p.a = static_cast<const float*>(a->ptr);
  if (b_scale != nullptr) {
    p.b_i8 = static_cast<const int8_t*>(b->ptr);
    p.b_scale = b_scale;
  } else {
    p.b = static_cast<const float*>(b->ptr);
  }
  for (int i = 0; i < 4; ++i) {
    p.as[i] = a->stride[i]; p.bs[i] = b->stride[i];
    p.os[i] = epi->out_f32.stride[i]; p.qs[i] = epi->out_i8.stride[i];
  }
  p.a_kfast = a->stride[3] == 1 || a->stride[2] != 1;
  p.b_nfast = b->stride[3] == 1 || b->stride[2] != 1;
  p.n_steps = epi->n_steps;
  for (int s = 0; s < epi->n_steps; ++s) p.steps[s] = epi->steps[s];
  p.out = static_cast<float*>(epi->out_f32.ptr);
  p.out_i8 = static_cast<int8_t*>(epi->out_i8.ptr);
  p.q = make_qscale(p.out_i8 != nullptr ? epi->out_scale : 1.0f);
  const int64_t gy = (m + BMM_BM - 1) / BMM_BM, gx = (n + BMM_BN - 1) / BMM_BN;
  MIRA_CHECK_ARG(gy <= 65535, "bmm has too many rows");
  MIRA_CHECK_ARG(gx <= int64_t(INT32_MAX), "bmm has too many columns");
  const dim3 grid(unsigned(gx), unsigned(gy), unsigned(batches < 65535 ? batches : 65535));
  bmm_f32_kernel<<<grid, BMM_THREADS, 0, dev->stream>>>(p);
  return after_launch("bmm_f32_kernel");
}

}  // namespace mira

extern "C" int mira_cuda_bmm_f32(int64_t batch0, int64_t batch1, int64_t m, int64_t n, int64_t k,
                                 const mira_view4* a, const mira_view4* b, const mira_bmm_epilogue* epi) {
  MIRA_GET_DEVICE(dev);
  return bmm_launch(dev, batch0, batch1, m, n, k, a, b, nullptr, epi);
}

extern "C" int mira_cuda_bmm_f32_w8(int64_t batch0, int64_t batch1, int64_t m, int64_t n, int64_t k,
                                    const mira_view4* a, const mira_view4* b_i8, const float* b_scale,
                                    const mira_bmm_epilogue* epi) {
  MIRA_GET_DEVICE(dev);
  MIRA_CHECK_ARG(b_scale != nullptr, "weight-only bmm needs the per-column scales");
  return bmm_launch(dev, batch0, batch1, m, n, k, a, b_i8, b_scale, epi);
}

namespace mira {

template <int DH>
static int launch_attention(DeviceState* dev, const AttnParams& p, int64_t b0, int64_t b1) {
  const int smem = static_cast<int>(sizeof(AttnSmem<DH>));
  static bool configured[64] = {};
  if (!configured[dev->device & 63]) {
    MIRA_CUDA_TRY(cudaFuncSetAttribute(attention_f32_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                  "cudaFuncSetAttribute(attention)");
    configured[dev->device & 63] = true;
  }
  const dim3 grid(unsigned((p.tq + ATT_BQ - 1) / ATT_BQ), unsigned(b1), unsigned(b0));
  attention_f32_kernel<DH><<<grid, ATT_THREADS, smem, dev->stream>>>(p);
  return after_launch("attention_f32_kernel");
}

// Whether the tensor-core kernel takes a shape, and its workspace: k and v as three bf16 pieces.
static bool attention_tc_shape(int64_t tq, int64_t tk, int64_t dh) {
  const char* choice = std::getenv("MIRA_CUDA_ATTENTION");   // "simt": the f32 FMA kernel, for comparisons
  const bool simt = choice != nullptr && std::strcmp(choice, "simt") == 0;
  return dh == ATC_DH && tq >= 64 && tk > 0 && tk <= int64_t(ATC_MAX_KB) * ATC_BK && !simt;
}

static int64_t attention_tc_bytes(int64_t b0, int64_t b1, int64_t tk) {
  const int64_t tkp = (tk + ATC_BK - 1) / ATC_BK * ATC_BK;
  // the TMA row coordinates of the piece arrays are 32-bit
  if (b0 * b1 * ATC_PIECES * tkp >= (int64_t(1) << 31)) return 0;
  return 2 * b0 * b1 * ATC_PIECES * tkp * ATC_DH * 2;
}

// The tensor-core path (attention_tc.cuh): k and v into pieces, then 128 query rows per CTA.
static int launch_attention_tc(DeviceState* dev, const AttnParams& p, int64_t b0, int64_t b1, void* ws) {
  const int smem = static_cast<int>(sizeof(AtcSmem)) + 1024;
  static bool configured[64] = {};
  if (!configured[dev->device & 63]) {
    MIRA_CUDA_TRY(cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                  "cudaFuncSetAttribute(attention_tc)");
    configured[dev->device & 63] = true;
  }
  const int64_t tkp = (p.tk + ATC_BK - 1) / ATC_BK * ATC_BK;
  const int64_t bh = b0 * b1;
  uint16_t* kpc = static_cast<uint16_t*>(ws);
  uint16_t* vtc = kpc + bh * ATC_PIECES * tkp * ATC_DH;
  attention_pieces_kernel<<<dim3(unsigned(tkp / ATC_BK), unsigned(b1), unsigned(b0)), ATC_PIECE_THREADS, 0, dev->stream>>>(
      p, int(tkp), kpc, vtc);
  const int rc = after_launch("attention_pieces_kernel");
  if (rc != MIRA_CUDA_OK) return rc;
  CUtensorMap map_k, map_vt;
  const cuuint32_t estr[2] = {1, 1};
  {
    const cuuint64_t dims[2] = {cuuint64_t(ATC_DH), cuuint64_t(bh * ATC_PIECES * tkp)};
    const cuuint64_t strides[1] = {cuuint64_t(ATC_DH * 2)};
    const cuuint32_t box[2] = {cuuint32_t(ATC_DH), cuuint32_t(ATC_BK)};
    const CUresult r = g_encode_tiled(&map_k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kpc, dims, strides, box, estr,
                                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(MIRA_CUDA_ECUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  }
  {
    const cuuint64_t dims[2] = {cuuint64_t(tkp), cuuint64_t(bh * ATC_PIECES * ATC_DH)};
    const cuuint64_t strides[1] = {cuuint64_t(tkp * 2)};
    const cuuint32_t box[2] = {cuuint32_t(ATC_BK), cuuint32_t(ATC_DH)};
    const CUresult r = g_encode_tiled(&map_vt, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, vtc, dims, strides, box, estr,
                                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(MIRA_CUDA_ECUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  }
  const dim3 grid(unsigned((p.tq + ATC_BQ - 1) / ATC_BQ), unsigned(b1), unsigned(b0));
  attention_tc_kernel<<<grid, ATC_THREADS, smem, dev->stream>>>(map_k, map_vt, p, int(tkp));
  return after_launch("attention_tc_kernel");
}

}  // namespace mira

extern "C" int mira_cuda_attention_f32(const mira_attention* a) {
  MIRA_GET_DEVICE(dev);
  MIRA_CHECK_ARG(a != nullptr, "null attention descriptor");
  MIRA_CHECK_ARG(a->batch0 >= 0 && a->batch1 >= 0 && a->tq >= 0 && a->tk > 0 && a->dh > 0 && a->dh <= 128,
                 "bad attention shape (dh <= 128, at least one key)");
  MIRA_CHECK_ARG(a->batch0 <= 65535 && a->batch1 <= 65535 && a->tq <= (int64_t(1) << 30) && a->tk <= (int64_t(1) << 30),
                 "attention batch or sequence too large");
  MIRA_CHECK_ARG(a->q.ptr != nullptr && a->k.ptr != nullptr && a->v.ptr != nullptr, "null attention operand");
  MIRA_CHECK_ARG(a->out_f32.ptr != nullptr || a->out_i8.ptr != nullptr, "attention has no output");
  MIRA_CHECK_ARG(a->scale_op == 0 || a->scale_op == MIRA_EPI_MUL || a->scale_op == MIRA_EPI_DIV, "bad scale step");
  if (a->out_i8.ptr != nullptr) MIRA_CHECK_ARG(a->out_scale > 0.0f, "requant scale must be positive");
  if (a->batch0 == 0 || a->batch1 == 0 || a->tq == 0) return MIRA_CUDA_OK;
  AttnParams p;
  std::memset(&p, 0, sizeof(p));
  p.tq = int(a->tq); p.tk = int(a->tk); p.dh = int(a->dh);
  p.q = static_cast<const float*>(a->q.ptr);
  p.k = static_cast<const float*>(a->k.ptr);
  p.v = static_cast<const float*>(a->v.ptr);
  for (int i = 0; i < 4; ++i) {
    p.qs[i] = a->q.stride[i]; p.ks[i] = a->k.stride[i]; p.vs[i] = a->v.stride[i];
    p.ms[i] = a->mask.stride[i]; p.os[i] = a->out_f32.stride[i]; p.is[i] = a->out_i8.stride[i];
  }
  const auto aligned16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
  p.vec = a->dh % 4 == 0 && a->k.stride[3] == 1 && a->v.stride[3] == 1 && aligned16(a->k.ptr) && aligned16(a->v.ptr);
  for (int i = 0; i < 3; ++i) p.vec = p.vec && a->k.stride[i] % 4 == 0 && a->v.stride[i] % 4 == 0;
  p.scale_op = a->scale_op;
  p.scale = a->scale;
  const float s_abs = a->scale_op == MIRA_EPI_MUL ? std::fabs(a->scale)
                      : (a->scale_op == MIRA_EPI_DIV ? 1.0f / std::fabs(a->scale) : 1.0f);
  p.scale_abs = std::isfinite(s_abs) ? s_abs * 1.0001f : INFINITY;
  p.mask = static_cast<const float*>(a->mask.ptr);
  p.tile_max = a->tile_max;
  p.tile_zero = a->tile_zero;
  p.kmax = reinterpret_cast<const unsigned int*>(a->kmax);
  p.out = static_cast<float*>(a->out_f32.ptr);
  p.out_i8 = static_cast<int8_t*>(a->out_i8.ptr);
  p.q8 = make_qscale(p.out_i8 != nullptr ? a->out_scale : 1.0f);
  p.err = device_err_ptr();
  if (p.tq == 1 && p.vec) {       // one query row (a decode step): stream the keys and values once
    const dim3 grid(unsigned(a->batch1), unsigned(a->batch0));
    if (a->dh <= 32) attention_q1_kernel<32><<<grid, ATT1_WARPS * 32, 0, dev->stream>>>(p);
    else if (a->dh <= 64) attention_q1_kernel<64><<<grid, ATT1_WARPS * 32, 0, dev->stream>>>(p);
    else attention_q1_kernel<128><<<grid, ATT1_WARPS * 32, 0, dev->stream>>>(p);
    return after_launch("attention_q1_kernel");
  }
  // prefill with a head dimension of 64 and a workspace: the tensor-core path
  if (attention_tc_shape(a->tq, a->tk, a->dh) && a->workspace != nullptr &&
      (reinterpret_cast<uintptr_t>(a->workspace) & 127) == 0 &&
      attention_tc_bytes(a->batch0, a->batch1, a->tk) > 0 &&
      a->workspace_bytes >= attention_tc_bytes(a->batch0, a->batch1, a->tk))
    return launch_attention_tc(dev, p, a->batch0, a->batch1, a->workspace);
  if (a->dh <= 32) return launch_attention<32>(dev, p, a->batch0, a->batch1);
  if (a->dh <= 64) return launch_attention<64>(dev, p, a->batch0, a->batch1);
  return launch_attention<128>(dev, p, a->batch0, a->batch1);
}

extern "C" int64_t mira_cuda_attention_workspace(int64_t batch0, int64_t batch1, int64_t tq, int64_t tk, int64_t dh) {
  if (batch0 <= 0 || batch1 <= 0 || !attention_tc_shape(tq, tk, dh)) return 0;
  return attention_tc_bytes(batch0, batch1, tk);
}

extern "C" int mira_cuda_absmax_f32(int64_t n0, int64_t n1, int64_t n2, int64_t n3, const mira_view4* x, float* out) {
  MIRA_GET_DEVICE(dev);
  MIRA_CHECK_ARG(n0 >= 0 && n1 >= 0 && n2 >= 0 && n3 >= 0, "bad view shape");
  MIRA_CHECK_ARG(x != nullptr && x->ptr != nullptr && out != nullptr, "null absmax operand");
  MIRA_CUDA_TRY(cudaMemsetAsync(out, 0, sizeof(float), dev->stream), "cudaMemsetAsync(absmax)");
  const int64_t total = n0 * n1 * n2 * n3;
  if (total == 0) return MIRA_CUDA_OK;
  AbsMaxParams p;
  p.n[0] = n0; p.n[1] = n1; p.n[2] = n2; p.n[3] = n3;
  p.x = static_cast<const float*>(x->ptr);
  for (int i = 0; i < 4; ++i) p.s[i] = x->stride[i];
  p.out = reinterpret_cast<unsigned int*>(out);
  const int threads = 256;
  absmax_view_kernel<<<grid_for(dev, (total / n3) * 32, threads), threads, 0, dev->stream>>>(p);
  return after_launch("absmax_view_kernel");
}

extern "C" int mira_cuda_qgemm_splitk_static(int64_t M, int64_t N, int64_t K, const int8_t* A, int64_t lda,
                                             const int8_t* B, int64_t ldb, const mira_dequant* dq,
                                             const mira_epilogue* epi) {
  MIRA_GET_DEVICE(dev);
  const int rc = qgemm_check(M, N, K, lda, ldb);
  if (rc != MIRA_CUDA_OK) return rc;
  if (M == 0) return MIRA_CUDA_OK;
  int splits, kb_per;
  splitk_plan(M, N, K, dev->sm_count, splits, kb_per);
  const int64_t need = splits > 1 ? int64_t(splits) * M * N * int64_t(sizeof(int32_t)) : 0;
  MIRA_CHECK_ARG(need <= kStaticSplitkBytes, "split-K partial sums exceed the 8 MiB static scratch");
  int32_t* scratch = g_splitk_scratch[dev->device];
  MIRA_CHECK_ARG(splits <= 1 || scratch != nullptr, "static split-K scratch not set up for this device");
  // nothing in the scratch needs clearing: every K range writes its whole M x N slice before the
  // finishing kernel reads it, which holds because no range is empty (a plan with an empty range
  // would leave the previous call's partial sums in its slice)
  const int64_t num_kb = (K + QG_BK - 1) / QG_BK;
  MIRA_CHECK_ARG(splits <= 1 || int64_t(splits - 1) * kb_per < num_kb, "split-K plan with an empty K range");
  return qgemm_run(dev, M, N, K, A, lda, B, ldb, dq, epi, splits, kb_per, scratch);
}
