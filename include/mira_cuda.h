/*
 * mira_cuda.h - C ABI of libmira_cuda.so, the B200 (sm_100a) execution library behind MIRA's
 * `cuda` target for the W8A8 path (`mira run ... -t cuda --quantize w8a8`).
 *
 * Every entry point takes plain pointers and sizes; device pointers come from mira_cuda_malloc.
 * Every entry point returns 0 on success or a non-zero MIRA_CUDA_E* status; the message of the
 * last failure on the calling thread is available through mira_cuda_last_error.  Launch entry
 * points are asynchronous on the library's stream for the current device (mira_cuda_set_device);
 * mira_cuda_sync waits for it and reports any error a kernel recorded on the device.
 *
 * The reference implements all of this in NumPy inside its op registry; each kernel entry point
 * names the reference function (path within the myramay/MIRA project, file:line) it replaces.
 *
 * Layouts.  4-D activations live on the device as NHWC ("channels last") with the channel count
 * padded to a multiple of 16 for int8 tensors (padding channels hold 0).  2-D int8 activations
 * [M, K] have a row stride of round_up(K, 16) bytes, padding bytes hold 0.  int8 weights are
 * K-major: qmatmul weights [N, Kp] (the transpose of the reference's [K, N] attr "q"), qconv2d
 * weights [O, KH, KW, Cp] flattened to [O, Kp] with Kp = round_up(KH*KW*Cp, 16).
 */
#ifndef MIRA_CUDA_H
#define MIRA_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MIRA_CUDA_ABI_VERSION 1

/* status codes */
#define MIRA_CUDA_OK 0
#define MIRA_CUDA_EINVAL 1      /* bad argument (shape, stride, alignment, unsupported case) */
#define MIRA_CUDA_ECUDA 2       /* a CUDA runtime/driver call failed */
#define MIRA_CUDA_ENODEV 3      /* no usable sm_100 device */
#define MIRA_CUDA_EKERNEL 4     /* a kernel recorded an error (bounded wait expired, bad index) */

/* epilogue step opcodes: reference ops.py:99-139 (UNARY/BINARY tables) restricted to
 * passes.py:151-152 (FUSABLE_UNARY / FUSABLE_BINARY) */
#define MIRA_EPI_RELU 1
#define MIRA_EPI_GELU 2
#define MIRA_EPI_SIGMOID 3
#define MIRA_EPI_TANH 4
#define MIRA_EPI_ADD 16
#define MIRA_EPI_SUB 17
#define MIRA_EPI_MUL 18
#define MIRA_EPI_DIV 19
#define MIRA_EPI_MAXIMUM 20
#define MIRA_EPI_MINIMUM 21

/* how a binary step's operand broadcasts against the [M, N] result (M = rows, N = channels) */
#define MIRA_OPND_NONE 0        /* unary step */
#define MIRA_OPND_SCALAR 1      /* one value: `scalar` */
#define MIRA_OPND_CHANNEL 2     /* ptr[n], padded by the caller to a multiple of 256 floats */
#define MIRA_OPND_FULL 3        /* ptr[m * ld + n] */
#define MIRA_OPND_ROW 4         /* ptr[m] */

#define MIRA_EPI_MAX_STEPS 8

/* int8 convolution input layouts */
#define MIRA_LAYOUT_NHWC 0      /* [n, h, w, cp] */
#define MIRA_LAYOUT_ROW4 1      /* row-expanded, for inputs of at most 4 channels: [n, h, entries, 16]
                                   where entry e holds pixels s*e - pad_w .. s*e - pad_w + 3, 4 channels
                                   each, 0 outside the image, s = the horizontal stride of the
                                   convolution that reads it (1, 2 or 4); weights [o, kh * 32] with
                                   k = i * 32 + j * 4 + c (taps j >= kw and channels >= c are 0) */
#define MIRA_LAYOUT_CP 2        /* chunk-planar, zero-padded: for [n, h, w, cp] with cp % 16 == 0,
                                   cp / 16 planes of n * (h + 2) * (w + 2) slots of 16 bytes; slot
                                   (c16, img, y, x) = G + c16 * plane + (img * (h + 2) + y + 1) *
                                   (w + 2) + x + 1 holds channels [16 c16, 16 c16 + 16) of pixel
                                   (img, y, x); G = round_up(w + 3, 8) guard slots come first and
                                   G + 128 after the last plane; every other slot (the padding ring
                                   of each image, the guards) is 0.  Bytes: mira_cuda_cp_bytes().
                                   Read by 3x3, stride-1, pad-1 convolutions of cp % 64 == 0 input
                                   channels, which then fetch each tile's input halo once */

typedef struct mira_epi_step {
  int32_t op;         /* MIRA_EPI_* */
  int32_t operand;    /* MIRA_OPND_* */
  int32_t swapped;    /* 1: f(operand, acc) instead of f(acc, operand) (reference ops.py:192-199) */
  float scalar;       /* MIRA_OPND_SCALAR value */
  const float* ptr;   /* device pointer for CHANNEL / FULL / ROW */
  int64_t ld;         /* row stride (elements) for FULL */
} mira_epi_step;

/* The fused epilogue of a quantized matmul/conv.  The dequantized f32 value
 * y = f32(f64(acc) * S) goes through the steps in order, then is written as f32 (out_f32) and/or
 * requantized for the next int8 op: clip(round_half_even(f32(y / out_scale)), -127, 127) (out_i8). */
typedef struct mira_epilogue {
  int32_t n_steps;
  mira_epi_step steps[MIRA_EPI_MAX_STEPS];
  float* out_f32;     /* may be NULL */
  int64_t ld_f32;     /* elements */
  int8_t* out_i8;     /* may be NULL */
  int64_t ld_i8;      /* bytes, multiple of 16; columns [N, ld_i8) are written as 0 */
  float out_scale;    /* np.float32(x_scale) of the consumer of out_i8 */
  int32_t i8_layout;  /* MIRA_LAYOUT_NHWC (rows of ld_i8 bytes), or MIRA_LAYOUT_CP for convolutions:
                         out_i8 in the chunk-planar layout of the conv output [n, oh, ow, ld_i8] */
} mira_epilogue;

/* Dequant scales.  Per-channel mode (qmatmul / qconv2d): S[n] = f64(x_scale) * f64(w_scale[n]),
 * the reference's combined scale (ops.py:619, ops.py:633).  The caller passes it as device arrays
 * padded to a multiple of 256 entries: scale64[n] = S[n] (double), scale_hi[n] = f32(S[n]) and
 * scale_lo[n] = f32(S[n] - scale_hi[n]) (round-to-nearest conversions).  Row/column mode (the
 * standalone GEMM sweep): S[m, n] = f64(row_scale[m]) * f64(col_scale[n]). */
typedef struct mira_dequant {
  const double* scale64;    /* per-channel mode when non-NULL */
  const float* scale_hi;
  const float* scale_lo;
  const float* row_scale;   /* row/column mode */
  const float* col_scale;
} mira_dequant;

/* ---------------------------------------------------------------- runtime */

int mira_cuda_abi_version(void);
/* Copies the message of the last failure on this thread into buf (always NUL-terminated). */
int mira_cuda_last_error(char* buf, size_t n);
/* Number of visible CUDA devices (0 without a GPU; never fails). */
int mira_cuda_device_count(void);
/* Selects the device for this thread and sets up its stream and helpers on first use. */
int mira_cuda_set_device(int device);
/* SM count and compute capability of the current device. */
int mira_cuda_device_info(int* sm_count, int* cc_major, int* cc_minor);
int mira_cuda_malloc(void** ptr, size_t bytes);
int mira_cuda_free(void* ptr);
int mira_cuda_host_alloc(void** ptr, size_t bytes);   /* pinned host memory */
int mira_cuda_host_free(void* ptr);
int mira_cuda_memset(void* dst, int value, size_t bytes);                 /* async */
int mira_cuda_h2d(void* dst, const void* src, size_t bytes);               /* async */
int mira_cuda_d2h(void* dst, const void* src, size_t bytes);               /* async */
int mira_cuda_d2d(void* dst, const void* src, size_t bytes);               /* async */
/* Copies that overlap the kernels: the device keeps a second stream for host<->device copies.
 * mira_cuda_h2d_copy_stream queues an H2D copy there (host memory pinned for overlap);
 * mira_cuda_copy_stream_record / mira_cuda_copy_stream_wait record an event on / make that stream
 * wait for an event; mira_cuda_stream_wait makes the kernel stream wait for an event;
 * mira_cuda_event_sync blocks the host until an event completed.  mira_cuda_sync waits for both
 * streams.  (No counterpart in the reference, which runs on the host.) */
int mira_cuda_h2d_copy_stream(void* dst, const void* src, size_t bytes);
int mira_cuda_copy_stream_record(void* event);
int mira_cuda_copy_stream_wait(void* event);
int mira_cuda_stream_wait(void* event);
int mira_cuda_event_sync(void* event);

/* Waits for the current device's streams; returns MIRA_CUDA_EKERNEL if a kernel recorded an
 * error since the last call (the record is cleared). */
int mira_cuda_sync(void);
/* The cudaStream_t of the current device, for callers that time with events on it. */
int mira_cuda_get_stream(void** stream);
/* Events on the library stream: create, record, elapsed milliseconds between two, destroy. */
int mira_cuda_event_create(void** ev);
int mira_cuda_event_record(void* ev);
int mira_cuda_event_elapsed(void* start, void* end, float* ms);
int mira_cuda_event_destroy(void* ev);
/* CUDA graph capture of the launches issued on the library stream between begin and end. */
int mira_cuda_graph_begin(void);
int mira_cuda_graph_end(void** graph_exec);
int mira_cuda_graph_launch(void* graph_exec);
int mira_cuda_graph_destroy(void* graph_exec);
/* Number of kernels this library launched (all threads, all devices). */
int64_t mira_cuda_launch_count(void);
/* Diagnostic: launches a kernel whose bounded wait on a barrier that nothing completes gives up
 * after timeout_us (at most 1 s); the following mira_cuda_sync must return MIRA_CUDA_EKERNEL and
 * leave the device usable.  No counterpart in the reference (it has no device code). */
int mira_cuda_selftest_wait_timeout(int64_t timeout_us);

/* ---------------------------------------------------------------- kernels */

/* Activation quantization, reference ops.py:602-603 (quantize_activation):
 *   xq = clip(round_half_even(f32(x) / f32(scale)), -127, 127).
 * x: f32 [rows, cols] with row stride ld_x (elements); xq: int8 [rows, ld_q], ld_q >= cols,
 * columns [cols, ld_q) written as 0. */
int mira_cuda_quantize_rows(const float* x, int64_t rows, int64_t cols, int64_t ld_x,
                            float scale, int8_t* xq, int64_t ld_q);

/* Quantization of an NCHW f32 tensor into NHWC int8 with Cp >= C channels (extra channels 0).
 * Also reference ops.py:602-603; the layout change is this library's. */
int mira_cuda_quantize_nchw_to_nhwc(const float* x, int64_t n, int64_t c, int64_t h, int64_t w,
                                    float scale, int8_t* xq, int64_t cp);

/* The same quantization into the MIRA_LAYOUT_ROW4 layout (c <= 4): `row_entries` entries per image
 * row, `pad` and `entry_stride` = the consumer convolution's horizontal padding and stride (1, 2 or
 * 4; a convolution with output width ow reads ow + 4 / entry_stride entries per row). */
int mira_cuda_quantize_nchw_to_row4(const float* x, int64_t n, int64_t c, int64_t h, int64_t w,
                                    float scale, int8_t* xq, int64_t row_entries, int64_t pad,
                                    int64_t entry_stride);

/* W8A8 matmul, reference ops.py:616-620 (_qmatmul_ref) with the epilogue of ops.py:192-199:
 *   acc[m, n] = sum_k A[m, k] * B[n, k]   (exact int32)
 *   y = epilogue(f32(f64(acc) * S))        (S from `dq`)
 * A: int8 [M, lda] (lda = round_up(K, 16)); B: int8 [N, ldb] K-major (ldb = round_up(K, 16)).
 * Runs on tcgen05.mma kind::i8 with TMEM accumulators and TMA-staged shared-memory tiles. */
int mira_cuda_qgemm(int64_t M, int64_t N, int64_t K, const int8_t* A, int64_t lda,
                    const int8_t* B, int64_t ldb, const mira_dequant* dq,
                    const mira_epilogue* epi);

/* Bytes of workspace mira_cuda_qgemm_splitk needs for an M x N x K product on the current device;
 * 0 when the output tiles already fill the GPU (then it runs like mira_cuda_qgemm). */
int64_t mira_cuda_qgemm_workspace(int64_t M, int64_t N, int64_t K);

/* mira_cuda_qgemm for shapes with few output tiles (small M, the skinny rows of the GEMM sweep and
 * of decoding): the reduction is cut into K ranges processed by different CTAs, whose int32 partial
 * sums go to `workspace` (device memory, 16-byte aligned, at least mira_cuda_qgemm_workspace()
 * bytes); a second kernel adds them (exact in int32) and applies the same dequant and epilogue, so
 * the results equal mira_cuda_qgemm's bit for bit.  Calls sharing a workspace must not overlap. */
int mira_cuda_qgemm_splitk(int64_t M, int64_t N, int64_t K, const int8_t* A, int64_t lda,
                           const int8_t* B, int64_t ldb, const mira_dequant* dq,
                           const mira_epilogue* epi, void* workspace, int64_t workspace_bytes);

/* mira_cuda_qgemm_splitk without a caller workspace and without allocating anything: the partial
 * sums go to a fixed 8 MiB scratch array inside the library (one per device; its address is looked
 * up once when the device is set up, so call mira_cuda_set_device before any stream capture).
 * Shapes whose partial sums need more than 8 MiB (mira_cuda_qgemm_workspace() > 8 MiB) return
 * MIRA_CUDA_EINVAL.  Nothing in the scratch has to start at zero.  All calls on a device share the
 * scratch: calls that overlap in time (other streams, concurrently replayed graphs) race.
 * No counterpart in the reference (it has no device memory). */
int mira_cuda_qgemm_splitk_static(int64_t M, int64_t N, int64_t K, const int8_t* A, int64_t lda,
                                  const int8_t* B, int64_t ldb, const mira_dequant* dq,
                                  const mira_epilogue* epi);

/* W8A8 convolution as an implicit GEMM over int8 activations, reference ops.py:630-634
 * (_qconv2d_ref, through _conv2d_ref ops.py:265-276 with groups = 1).
 * x: MIRA_LAYOUT_NHWC int8 [n, h, w, cp] (cp 4 or a multiple of 16) with weights int8 [o, ldw],
 * k = (i * kw + j) * cp + c, ldw = round_up(kh*kw*cp, 16); or MIRA_LAYOUT_ROW4 (x_row_entries
 * entries per row) with its weight layout; or MIRA_LAYOUT_CP (3x3, stride 1, pad 1, no dilation,
 * cp % 64 == 0) with the NHWC weight layout.  The result [n*oh*ow, o] (NHWC) goes through the same
 * epilogue as mira_cuda_qgemm; its int8 output may be MIRA_LAYOUT_CP (epi->i8_layout). */
int mira_cuda_qconv2d(int64_t n, int64_t h, int64_t w, int64_t cp, const int8_t* x,
                      int64_t x_layout, int64_t x_row_entries,
                      int64_t o, int64_t kh, int64_t kw, const int8_t* wq, int64_t ldw,
                      int64_t stride_h, int64_t stride_w, int64_t pad_h, int64_t pad_w,
                      int64_t dil_h, int64_t dil_w, const mira_dequant* dq,
                      const mira_epilogue* epi);

/* qconv2d followed by max pooling, fused: the reference's qconv2d (ops.py:630-634) with its
 * epilogue, then pad (ops.py:469-470, `pool_pad` pixels of `pool_pad_value`) and maxpool2d
 * (ops.py:293-296, window `pool_size`, stride `pool_stride`).  The conv outputs never leave the
 * SM: each tile computes the conv pixels under a block of pooled outputs and pools them in shared
 * memory; `epi`'s outputs are the pooled [n*ph*pw, o] f32 / int8 tensors.  o <= 64; the epilogue
 * must be monotone non-decreasing (relu; add, non-swapped sub, maximum, minimum of scalar or
 * per-channel constants) because the kernel pools the int32 accumulators and applies it to the
 * pooled values; pool padding must be -inf. */
int mira_cuda_qconv2d_maxpool(int64_t n, int64_t h, int64_t w, int64_t cp, const int8_t* x,
                              int64_t x_layout, int64_t x_row_entries, int64_t o,
                              int64_t kh, int64_t kw, const int8_t* wq, int64_t ldw, int64_t stride_h,
                              int64_t stride_w, int64_t pad_h, int64_t pad_w, int64_t dil_h, int64_t dil_w,
                              int64_t pool_size, int64_t pool_stride, int64_t pool_pad, float pool_pad_value,
                              const mira_dequant* dq, const mira_epilogue* epi);

/* Max pooling over NHWC, reference ops.py:293-296 (maxpool2d) preceded by an optional constant
 * pad (ops.py:469-470) of `pad` pixels holding `pad_value` (the -inf pad in front of ResNet's
 * pool).  f32 in -> f32 out (out_f32) and/or int8 out; int8 in (x_i8 non-NULL) -> int8 out,
 * which equals quantize(maxpool(x)) because quantization is monotone. */
int mira_cuda_maxpool2d_nhwc(const float* x_f32, const int8_t* x_i8, int64_t n, int64_t h,
                             int64_t w, int64_t c, int64_t ldc_in, int64_t size, int64_t stride,
                             int64_t pad, float pad_value, float* out_f32, int64_t ldc_out_f32,
                             int8_t* out_i8, int64_t ldc_out_i8, float out_scale);
/* The same with the int8 output's layout chosen: MIRA_LAYOUT_NHWC as above, or MIRA_LAYOUT_CP
 * (f32 input only; ldc_out_i8 = the padded channel count, a multiple of 16). */
int mira_cuda_maxpool2d_nhwc_ex(const float* x_f32, const int8_t* x_i8, int64_t n, int64_t h,
                                int64_t w, int64_t c, int64_t ldc_in, int64_t size, int64_t stride,
                                int64_t pad, float pad_value, float* out_f32, int64_t ldc_out_f32,
                                int8_t* out_i8, int64_t ldc_out_i8, float out_scale, int64_t i8_layout);
/* Bytes of an int8 activation [n, h, w, cp] in MIRA_LAYOUT_CP (0 for bad sizes). */
int64_t mira_cuda_cp_bytes(int64_t n, int64_t h, int64_t w, int64_t cp);

/* Mean over H and W of NHWC f32 (reference ops.py:318-343 reduce_mean over axes (2, 3)), summed
 * in NumPy's pairwise order so the f32 result is bit-identical; optional f32 and int8 outputs
 * [n, c] (int8 rows padded to ld_i8). */
int mira_cuda_mean_hw_nhwc(const float* x, int64_t n, int64_t hw, int64_t c, int64_t ldc,
                           float* out_f32, int8_t* out_i8, int64_t ld_i8, float out_scale);

/* Patch matrix of a general f32 convolution (reference _conv2d_ref with groups = 1, ops.py:265-276,
 * taps from _taps 256-263): x NHWC f32 [n, h, w, c] with pixel stride ldc; out [n * oh * ow, ld_out]
 * with row m = output pixel and column (i * kw + j) * c + ch the input value under tap (i, j), 0 in
 * the zero padding.  The convolution is the f32 matmul of out with the weights reshaped to
 * [kh * kw * c, o] (mira_cuda_bmm_f32, or mira_cuda_bmm_f32_w8 for weight-only int8 weights). */
int mira_cuda_im2col_f32(const float* x, int64_t n, int64_t h, int64_t w, int64_t c, int64_t ldc, int64_t kh,
                         int64_t kw, int64_t stride_h, int64_t stride_w, int64_t pad_h, int64_t pad_w,
                         int64_t dil_h, int64_t dil_w, float* out, int64_t ld_out);

/* Depthwise f32 convolution over NHWC (reference ops.py:265-276 _conv2d_ref with
 * groups == channels, which the reference never quantizes, quantize.py:105-106): per-tap f32
 * products summed in (i, j) order from 0, then the epilogue on [n*oh*ow, c]. weights f32
 * [kh*kw, c] (tap-major). */
int mira_cuda_dwconv2d_nhwc(const float* x, int64_t n, int64_t h, int64_t w, int64_t c,
                            const float* wt, int64_t kh, int64_t kw, int64_t stride_h,
                            int64_t stride_w, int64_t pad_h, int64_t pad_w, int64_t dil_h,
                            int64_t dil_w, const mira_epilogue* epi);

/* W8A8 depthwise convolution, the opt-in int8 depthwise mode: reference _qconv2d_ref
 * (ops.py:630-634) on a qconv2d with groups == channels (what quantize_w8a8 would produce if
 * _w8a8_weight, quantize.py:95-115, accepted depthwise weights).  x: int8 NHWC [n, h, w, ldx]
 * (quantized at the op's x_scale, channels >= c zero); wq: int8 [kh*kw, c] tap-major, 4-byte
 * aligned; dq: per-channel dequant (scale64/hi/lo of x_scale * w_scale[c]).  Integer sums over the
 * taps, the exact dequant, then the epilogue on [n*oh*ow, c] (int8 NHWC rows and/or f32).
 * c must be a multiple of 4. */
int mira_cuda_qdwconv2d_nhwc(const int8_t* x, int64_t n, int64_t h, int64_t w, int64_t c, int64_t ldx,
                             const int8_t* wq, int64_t kh, int64_t kw, int64_t stride_h, int64_t stride_w,
                             int64_t pad_h, int64_t pad_w, int64_t dil_h, int64_t dil_w,
                             const mira_dequant* dq, const mira_epilogue* epi);

/* Layout changes between the reference's NCHW f32 tensors and the device's NHWC. */
int mira_cuda_nchw_to_nhwc_f32(const float* x, int64_t n, int64_t c, int64_t h, int64_t w,
                               float* y, int64_t ldc);
int mira_cuda_nhwc_to_nchw_f32(const float* x, int64_t n, int64_t h, int64_t w, int64_t c,
                               int64_t ldc, float* y);

/* ---------------------------------------------------------------- sequence (transformer) ops
 *
 * These cover the f32 ops between the quantized matmuls of a decoder-only transformer.  Tensors
 * of rank <= 4 are addressed as views: a base pointer and element strides over four dimensions
 * (batch0, batch1, row, col), lower ranks padded with leading size-1 dimensions, broadcast
 * dimensions with stride 0.  Row kernels accept rows of at most MIRA_ROW_MAX elements. */

#define MIRA_ROW_MAX 8192
#define MIRA_OPND_VIEW 5        /* bmm epilogue operand read through a mira_view4 */

typedef struct mira_view4 {
  void* ptr;                /* device pointer (f32, or int8 for mira_bmm_epilogue.out_i8) */
  int64_t stride[4];        /* element strides over (batch0, batch1, row, col) */
} mira_view4;

typedef struct mira_bmm_step {
  int32_t op;               /* MIRA_EPI_* */
  int32_t operand;          /* MIRA_OPND_NONE, MIRA_OPND_SCALAR or MIRA_OPND_VIEW */
  int32_t swapped;          /* 1: f(operand, acc) */
  float scalar;
  mira_view4 view;          /* MIRA_OPND_VIEW operand, indexed like the output */
} mira_bmm_step;

typedef struct mira_bmm_epilogue {
  int32_t n_steps;
  mira_bmm_step steps[MIRA_EPI_MAX_STEPS];
  mira_view4 out_f32;       /* ptr may be NULL */
  mira_view4 out_i8;        /* ptr may be NULL: int8 requantized with out_scale */
  float out_scale;
} mira_bmm_epilogue;

/* Batched f32 matmul C[b0, b1] = A[b0, b1] (M x K) @ B[b0, b1] (K x N) followed by an epilogue,
 * reference ops.py:217-219 (_matmul_ref: np.matmul of f32 operands, then epilogue_ref,
 * ops.py:192-199).  Products are accumulated in f32 in k order with fused multiply-adds, so
 * results agree with the reference's BLAS matmul to f32 rounding, not bit for bit. */
int mira_cuda_bmm_f32(int64_t batch0, int64_t batch1, int64_t m, int64_t n, int64_t k,
                      const mira_view4* a, const mira_view4* b, const mira_bmm_epilogue* epi);

/* Weight-only int8 matmul (reference `quantize="int8"`: quantize.py:45-68 turns a [K, N] matmul
 * weight into a `dequantize` constant, ops.py:583-587, feeding the f32 matmul of ops.py:217-219).
 * Like mira_cuda_bmm_f32, but b_i8 views the int8 weights q (element strides) and b_scale holds
 * the f32 scale of each of the n columns; every weight is rebuilt as RN(f32(q[k, n]) * b_scale[n]),
 * the reference's own rounding, while it is staged into shared memory, so the weights stay int8 in
 * device memory. */
int mira_cuda_bmm_f32_w8(int64_t batch0, int64_t batch1, int64_t m, int64_t n, int64_t k,
                         const mira_view4* a, const mira_view4* b_i8, const float* b_scale,
                         const mira_bmm_epilogue* epi);

/* Layer normalization over the last axis of rows [rows, d] (row stride ld_x), reference
 * ops.py:356-360 (_layernorm_ref): mean and variance in NumPy's pairwise summation order and
 * float32 division by d, so the f32 result is bit-identical.  Optional outputs: f32 rows
 * (out_f32, ld_f32) and int8 rows requantized with out_scale (out_i8, ld_i8 bytes). */
int mira_cuda_layernorm_rows(const float* x, int64_t rows, int64_t d, int64_t ld_x, const float* gamma,
                             const float* beta, float eps, float* out_f32, int64_t ld_f32, int8_t* out_i8,
                             int64_t ld_i8, float out_scale);

/* Softmax over the last axis of rows [rows, n], reference ops.py:310-313 (_softmax_ref):
 * e = exp(x - max(x)), e / sum(e) with the sum in NumPy's pairwise order.  exp is CUDA's
 * expf (NumPy's own float32 exp is not correctly rounded either), so results agree to a few
 * units in the last place. */
int mira_cuda_softmax_rows(const float* x, int64_t rows, int64_t n, int64_t ld_x, float* out, int64_t ld_out);

/* Embedding rows: out[r, :] = table[idx[r], :] (+ addend[r % addend_rows, :] when addend is
 * non-NULL), reference ops.py:482-487 (_gather_ref, np.take on axis 0) followed by an f32 add.
 * Negative indices count from the end like np.take; an index outside [-vocab, vocab) writes 0
 * and makes the next mira_cuda_sync fail (the reference raises IndexError). */
int mira_cuda_embed_rows(const float* table, int64_t vocab, int64_t d, const int32_t* idx, int64_t rows,
                         const float* addend, int64_t addend_rows, float* out, int64_t ld_out);

/* Fused attention, o = softmax((q @ k^T) <scale step> (+ mask), axis=-1) @ v: the reference's
 * matmul with its fused epilogue (ops.py:217-219, 192-199), softmax (ops.py:310-313) and second
 * matmul computed in one pass per block of 64 query rows without storing the scores (online
 * softmax).  q [b0, b1, tq, dh], k [b0, b1, tk, dh] (keys as rows, i.e. the transpose of the
 * reference's k^T operand), v [b0, b1, tk, dh], mask indexed [b0, b1, q, k].  A key tile whose
 * mask entries are all <= -200 (tile_max, [ceil(tq/64)][ceil(tk/64)]) is skipped only when
 * |scale| * ||q_i||_1 * max|k| + tile_max - m_i < -110 for every row (m_i the running row maximum,
 * kmax from mira_cuda_absmax_f32), i.e. when the reference's exp gives exactly 0 on the whole
 * tile.  Results agree with the reference to f32 rounding. */
typedef struct mira_attention {
  int64_t batch0, batch1, tq, tk, dh;   /* dh <= 128 */
  mira_view4 q, k, v;
  int32_t scale_op;         /* 0, MIRA_EPI_MUL or MIRA_EPI_DIV (applied before the mask) */
  float scale;
  mira_view4 mask;          /* ptr NULL: no mask */
  const float* tile_max;    /* NULL: no skipping */
  const float* kmax;        /* device scalar; NULL: no skipping */
  const uint8_t* tile_zero; /* [ceil(tq/64)][ceil(tk/64)]: 1 where the mask tile is all +0 (its add
                               is skipped); may be NULL */
  mira_view4 out_f32;       /* ptr may be NULL */
  mira_view4 out_i8;        /* ptr may be NULL: int8 requantized with out_scale */
  float out_scale;
  void* workspace;          /* device scratch for the tensor-core path (k and v split into bf16 pieces),
                               128-byte aligned; NULL or smaller than mira_cuda_attention_workspace():
                               the f32 kernel */
  int64_t workspace_bytes;
} mira_attention;

int mira_cuda_attention_f32(const mira_attention* a);

/* Bytes of workspace the tensor-core attention path needs for these sizes (0: the shape takes the
 * f32 FMA kernel).  Prefill (tq >= 64) with dh == 64 and tk <= 16384 runs on the tensor cores:
 * q @ k^T and p @ v as sums of bf16 piece products (three pieces per f32 value, exact), f32
 * accumulation in TMEM, the f32 kernel's online softmax.  MIRA_CUDA_ATTENTION=simt in the
 * environment selects the f32 kernel for every shape. */
int64_t mira_cuda_attention_workspace(int64_t batch0, int64_t batch1, int64_t tq, int64_t tk, int64_t dh);

/* *out = max |x| over a [n0, n1, n2, n3] f32 view (NaN counts as +inf); out is device memory. */
int mira_cuda_absmax_f32(int64_t n0, int64_t n1, int64_t n2, int64_t n3, const mira_view4* x, float* out);

/* Strided copy of a [n0, n1, n2, n3] f32 view into another view (the device form of the
 * reference's transpose, ops.py:375, when a consumer needs the data in a new order). */
int mira_cuda_copy_view_f32(int64_t n0, int64_t n1, int64_t n2, int64_t n3, const mira_view4* src,
                            const mira_view4* dst);

/* A standalone f32 element-wise op (reference UNARY / BINARY, ops.py:99-139, when no matmul or
 * convolution epilogue absorbed it): op a unary MIRA_EPI_* code (out = f(a); b, scalar ignored) or a
 * binary one (out = f(a, B), or f(B, a) when swapped, with B the view b or, when b is NULL, the
 * scalar).  [n0, n1, n2, n3] through element-stride views (0 for broadcast dimensions); the same
 * arithmetic as the epilogue steps, so add/sub/mul/div/maximum/minimum match NumPy bit for bit. */
int mira_cuda_elementwise_f32(int32_t op, int64_t n0, int64_t n1, int64_t n2, int64_t n3, const mira_view4* a,
                              const mira_view4* b, float scalar, int32_t swapped, const mira_view4* out);

/* Slices at runtime positions (reference dynamic_slice / dynamic_update_slice, ops.py:533-576),
 * for 4-byte elements (f32 or i32) in views of at most 4 dimensions (shapes padded with leading 1s
 * to 4).  `start` is DEVICE memory holding `rank` int32 start entries for the last `rank`
 * dimensions (the leading ones start at 0 and must be taken whole); every entry is clamped to
 * [0, dims - window] like the reference's _clamped_starts (ops.py:536-537).  Reading the start on
 * the device keeps a captured CUDA graph valid while the position changes between steps.
 *   dynamic_slice:        out[e] = x[start + e] for e < size.
 *   dynamic_update_slice: x[start + e] = upd[e] for e < upd_dims, in place (the reference returns an
 *                         updated copy; a caller that needs the old x copies it first). */
int mira_cuda_dynamic_slice(const mira_view4* x, const int64_t* x_dims, const int32_t* start, int64_t rank,
                            const int64_t* size, const mira_view4* out);
int mira_cuda_dynamic_update_slice(const mira_view4* x, const int64_t* x_dims, const mira_view4* upd,
                                   const int64_t* upd_dims, const int32_t* start, int64_t rank);

#ifdef __cplusplus
}
#endif

#endif /* MIRA_CUDA_H */
