/*
 * gcdr_cuda.h -- C ABI of the B200 (sm_100a) CUDA backend for GCDRNet
 * document enhancement (u8 image -> GC-Net -> division correction ->
 * DR-Net -> u8 image).
 *
 * The library is the drop-in for the `GcdrBackend.Cuda` arm of the
 * reference's `GcdrEnhancer` (src/Sdcb.SimdGcdrNet/GcdrEnhancer.cs).  Two
 * levels are exported, mirroring the reference's own two levels:
 *
 *   gcdr_enhancer_*  the public, thread-safe enhancer
 *                    (GcdrEnhancer.FromBytes / Enhance / PoolStats / Dispose,
 *                    GcdrEnhancer.cs:82-100, 181-271, 67-68, 325-331):
 *                    argument validation, top/left pad to /32, a pool of
 *                    workers rented per call, retry-once on device loss.
 *   gcdr_cuda_*      one worker: a CUDA stream and a cache of shape plans
 *                    (per image shape: a device arena, the op sequence and
 *                    its CUDA graph; up to 8, least recently used evicted);
 *                    NOT thread-safe (the VkGcdrPipeline contract,
 *                    Backends/Vulkan/VkPipeline2.cs:21-379).
 *
 * Plain pointers and sizes only.  Source and destination images are HOST
 * memory in the caller's layout (any row stride, dst may alias src when the
 * strides are equal).  Pixel formats carry the values of GcdrPixelFormat
 * (GcdrPixelFormat.cs:7-17).  Every entry point returns a GCDR_* status; on
 * failure *_last_error() gives a message.
 */
#ifndef GCDR_CUDA_H
#define GCDR_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define GCDR_API __declspec(dllexport)
#else
#define GCDR_API __attribute__((visibility("default")))
#endif

/* Status codes.  The reference throws; the mapping is:
 *   GCDR_ERR_RANGE       ArgumentOutOfRangeException (width/height < 1, stride
 *                        < width*bpp, unknown pixel format; GcdrEnhancer.cs:184-188,
 *                        GcdrPixelFormat.cs:21-26)
 *   GCDR_ERR_ARG         ArgumentException (short buffers, GcdrEnhancer.cs:189-192),
 *                        ArgumentNullException (null model streams, :97-98)
 *   GCDR_ERR_UNSUPPORTED NotSupportedException (model graph not the GCDRNet
 *                        topology, GC output shape mismatch, :249-250)
 *   GCDR_ERR_DEVICE      VkDeviceLostException analogue: the CUDA context
 *                        reported an error; the enhancer retries once on a
 *                        fresh worker pool (GcdrEnhancer.cs:218-222)
 *   GCDR_ERR_TIMEOUT     a device-side bounded wait expired (the kernel gave
 *                        up and returned instead of hanging)
 *   GCDR_ERR_OOM         device or pinned host allocation failed
 *   GCDR_ERR_MODEL       the ONNX bytes could not be parsed
 */
#define GCDR_OK 0
#define GCDR_ERR_ARG 1
#define GCDR_ERR_RANGE 2
#define GCDR_ERR_UNSUPPORTED 3
#define GCDR_ERR_DEVICE 4
#define GCDR_ERR_TIMEOUT 5
#define GCDR_ERR_OOM 6
#define GCDR_ERR_MODEL 7

/* GcdrPixelFormat (GcdrPixelFormat.cs:7-17) */
#define GCDR_BGR24 0
#define GCDR_RGB24 1
#define GCDR_BGRA32 2
#define GCDR_RGBA32 3

/* precision: the tensor-core layers' operand/storage type.  The stem conv,
 * the head (UpHead) and the division glue always run in fp32. */
#define GCDR_PRECISION_FP16 0

typedef struct gcdr_model gcdr_model;       /* parsed GC-Net + DR-Net weights */
typedef struct gcdr_cuda gcdr_cuda;         /* one worker (not thread-safe)   */
typedef struct gcdr_enhancer gcdr_enhancer; /* thread-safe pooled enhancer    */

/* ---------------------------------------------------------------- models */

/* Parses both ONNX models and checks that each is the GCDRNet UNeXt
 * topology.  Replaces OnnxModel.Load (GcdrEnhancer.cs:84,91,99) plus the part
 * of GraphCompiler.Compile + the GCDR fusion passes that this backend needs
 * (Extensions/GcdrExtensions.cs:12-15: FuseShiftPass, FuseUpHeadPass,
 * UpHeadSkipRecomputePass).  The bytes are only read during the call.  No
 * GPU is touched. */
GCDR_API int gcdr_model_load(const void *gc_onnx, size_t gc_len,
                             const void *dr_onnx, size_t dr_len,
                             gcdr_model **out, char *err, size_t err_cap);
GCDR_API void gcdr_model_free(gcdr_model *m);
/* Writes a JSON description of the recognised topology (channels, shift
 * groups and offsets) into buf; returns the length needed (excluding NUL). */
GCDR_API size_t gcdr_model_describe(const gcdr_model *m, char *buf, size_t cap);

/* ---------------------------------------------------------- one worker */

/* Creates a worker on `device` (CUDA ordinal): uploads packed weights, owns
 * one stream, a grow-only device arena and pinned staging.  Mirrors
 * `new VkGcdrPipeline(backend, gc, dr)` (VkPipeline2.cs:42-64). */
GCDR_API int gcdr_cuda_create(int device, const gcdr_model *m, int precision,
                              gcdr_cuda **out);
/* Legacy convenience matching the proposed shim: parse + create in one call. */
GCDR_API int gcdr_cuda_create_from_onnx(int device, const void *gc_onnx, size_t gc_len,
                                        const void *dr_onnx, size_t dr_len,
                                        int precision, gcdr_cuda **out);
/* Enhance one image (host buffers).  Binds the worker to the image's shape
 * plan first (a cached plan, or arena plan + CUDA-graph capture for a new
 * shape), then copies the strided source in (through pinned staging, or by
 * DMA when it is page-locked), runs the graph, copies back with the
 * destination stride.  VkGcdrPipeline.Enhance (VkPipeline2.cs:296-327). */
GCDR_API int gcdr_cuda_enhance(gcdr_cuda *w, const uint8_t *src, int width, int height,
                               int src_stride, uint8_t *dst, int dst_stride,
                               int pixel_format);
/* Same, device-resident: src/dst are DEVICE pointers of tight images
 * (stride = width*bpp) and the call is asynchronous on the worker's stream
 * (or `stream` when non-null).  Used for throughput runs with inputs
 * already in HBM. */
GCDR_API int gcdr_cuda_enhance_device(gcdr_cuda *w, const uint8_t *d_src, int width, int height,
                                      uint8_t *d_dst, int pixel_format, void *stream);
/* Batched images per launch: n (1..16) images of one shape and format in ONE
 * CUDA-graph launch.  The worker's batch plan for (width, height, format, n)
 * holds n image slices in its arena (each image's buffers at the same offset
 * of its slice) and every kernel of its graph covers all n images, one launch
 * per layer: the low-resolution layers of one image occupy only part of the
 * GPU, n images fill it.  Each image gets the bytes of a single-image enhance
 * (the summation order of every layer is the one-image plan's).  Host buffers
 * as gcdr_cuda_enhance (dst[k] may alias src[k] at equal strides; page-locked
 * sources are copied by DMA directly); the _device form takes tight device
 * images and is asynchronous on `stream`.  No counterpart in the reference:
 * its README lists batching as not covered (README.md:182). */
GCDR_API int gcdr_cuda_enhance_batch(gcdr_cuda *w, const uint8_t *const *src, int n, int width, int height,
                                     int src_stride, uint8_t *const *dst, int dst_stride, int pixel_format);
GCDR_API int gcdr_cuda_enhance_batch_device(gcdr_cuda *w, const uint8_t *const *d_src, int n, int width,
                                            int height, uint8_t *const *d_dst, int pixel_format, void *stream);
/* Device bytes held by the worker (arena + staging): VkPipeline2.cs:141. */
GCDR_API int64_t gcdr_cuda_device_bytes(const gcdr_cuda *w);
/* Debug: padded NHWC fp32 intermediates of the last enhance -- the GC
 * input x [h][w][3], the shading map I_sm [h][w][3] and the DR input
 * [h][w][6] -- as VkGcdrPipeline.DebugIntermediates (VkPipeline2.cs:356-364).
 * Any pointer may be NULL.  Sizes use the padded h, w of the last call. */
GCDR_API int gcdr_cuda_debug_intermediates(gcdr_cuda *w, float *gc_in, float *gc_out, float *dr_in);
/* Debug: kernel launches per enhance in the captured graph, and the padded
 * shape the worker is bound to. */
GCDR_API int gcdr_cuda_launch_count(const gcdr_cuda *w);
/* Shape plans: a worker keeps the arena, op sequence and CUDA graph of up to 8
 * image shapes (width, height, format, debug mode), least recently used
 * evicted first and the cached arenas kept within a 12 GB budget (the
 * reference caches 8 sizes, GcdrEnhancer.cs:45-46, 128-136, within the arena
 * budget of VkPipeline2.cs:104-117).  captures: graphs captured so far (one
 * per shape seen while not cached); plans: shapes held now. */
GCDR_API int gcdr_cuda_plan_stats(const gcdr_cuda *w, int *captures, int *plans);
/* Debug mode: the heads also write the shading map I_sm and the DR output as
 * fp32 planes, returned by gcdr_cuda_debug_intermediates (gc_out) and
 * gcdr_cuda_debug_output.  Re-captures the graph on the next enhance. */
GCDR_API int gcdr_cuda_set_debug(gcdr_cuda *w, int on);
GCDR_API int gcdr_cuda_debug_output(gcdr_cuda *w, float *dr_out);
/* Per-op profile of the bound shape (the analogue of the reference's
 * GCDRNET_PROF per-op timers, bench/Sdcb.SimdGcdrNet.Benchmark/Program.cs:993-1010):
 * runs the op sequence `reps` times eagerly with CUDA events around each op and
 * fills up to `cap` entries with the mean duration and the op's algorithmic
 * FLOPs and HBM bytes.  Returns the op count, or -GCDR_ERR_* on failure. */
typedef struct {
    char name[48];
    double ms;
    double flops;
    double bytes;
    int tensor_core;
} gcdr_op_profile;
GCDR_API int gcdr_cuda_profile(gcdr_cuda *w, int reps, gcdr_op_profile *out, int cap);
GCDR_API const char *gcdr_cuda_last_error(const gcdr_cuda *w);
GCDR_API void gcdr_cuda_destroy(gcdr_cuda *w);

/* ----------------------------------------------------- pooled enhancer */

/* GcdrEnhancer.FromBytes(gc, dr, GcdrBackend.Cuda) (GcdrEnhancer.cs:89-91). */
GCDR_API int gcdr_enhancer_create(int device, const void *gc_onnx, size_t gc_len,
                                  const void *dr_onnx, size_t dr_len, int precision,
                                  gcdr_enhancer **out, char *err, size_t err_cap);
/* GcdrEnhancer.Enhance(src, width, height, srcStride, dst, dstStride, format)
 * (GcdrEnhancer.cs:181-271).  src_len/dst_len are the buffer lengths in bytes
 * (the Span lengths).  Thread-safe; dst may alias src at equal strides. */
GCDR_API int gcdr_enhancer_enhance(gcdr_enhancer *e, const uint8_t *src, size_t src_len,
                                   int width, int height, int src_stride,
                                   uint8_t *dst, size_t dst_len, int dst_stride,
                                   int pixel_format, char *err, size_t err_cap);
/* n (1..16) images of one shape and format through one pooled worker's batch
 * plan (gcdr_cuda_enhance_batch): each image is validated as by
 * gcdr_enhancer_enhance (src_len[k], dst_len[k] its buffer lengths) and gets the
 * bytes a single enhance gives it.  Thread-safe; dst[k] may alias src[k] at
 * equal strides.  No counterpart in the reference (README.md:182). */
GCDR_API int gcdr_enhancer_enhance_batch(gcdr_enhancer *e, const uint8_t *const *src, const size_t *src_len, int n,
                                         int width, int height, int src_stride, uint8_t *const *dst,
                                         const size_t *dst_len, int dst_stride, int pixel_format, char *err,
                                         size_t err_cap);
/* Concurrent gcdr_enhancer_enhance calls of one shape, format and stride pair are batched
 * opportunistically: when no batch of that shape runs, or a full batch is queued and fewer than
 * `max_running` run, a waiting caller takes the oldest queued calls (a power of two of them, at
 * most `max_batch`) and runs them as one batch-plan launch for all; a lone call runs at once,
 * alone.  Every call returns when its
 * own image is written and gets the bytes a single-image plan gives it.  Defaults 8 and 3;
 * max_batch = 1 turns the batching off.  No counterpart in the reference (every Enhance call
 * runs alone there). */
GCDR_API int gcdr_enhancer_set_batching(gcdr_enhancer *e, int max_batch, int max_running);
/* Enhance calls so far, and the worker launches that ran them (launches < calls when calls
 * were batched). */
GCDR_API void gcdr_enhancer_batch_stats(const gcdr_enhancer *e, int64_t *calls, int64_t *launches);
/* GcdrEnhancer.PoolStats (GcdrEnhancer.cs:67-68): pools created, workers
 * created, pools evicted. */
GCDR_API void gcdr_enhancer_pool_stats(const gcdr_enhancer *e, int64_t *pools,
                                       int64_t *workers, int64_t *evicted);
/* Test hook: the next `count` worker enhances report GCDR_ERR_DEVICE before
 * touching the GPU (host-side fault injection, the analogue of setting
 * Dev.Lost in VulkanDeviceLossTests.cs:14-33). */
GCDR_API void gcdr_enhancer_inject_device_loss(gcdr_enhancer *e, int count);
/* Page-locks the caller's host buffer [p, p + bytes) for every device
 * (cudaHostRegister, portable), or releases it (before the memory is freed).
 * Enhance calls whose source or destination lies wholly in page-locked memory
 * (registered here, or allocated pinned) copy it by DMA directly, in any row
 * stride, instead of through the worker's pinned staging: the host then moves
 * each image once instead of three times.  A destination apart from the
 * source is written by DMA right behind the graph; after a device error its
 * contents are unspecified (the source is untouched, so the retry is exact).
 * No counterpart in the reference (its buffers are managed Spans). */
GCDR_API int gcdr_host_register(void *p, size_t bytes);
GCDR_API int gcdr_host_unregister(void *p);
/* GcdrEnhancer.Dispose (GcdrEnhancer.cs:325-331). */
GCDR_API void gcdr_enhancer_destroy(gcdr_enhancer *e);

/* ------------------------------------------------- standalone kernels */

/* The three glue stages as separate device kernels (the fused pipeline does
 * them inside the stem and head kernels).  Pointers are DEVICE pointers,
 * launches are asynchronous on `stream` (NULL = default stream).
 *   bgr2nhwc  Shaders/bgr2nhwc.comp (u8 any format/stride -> padded NHWC fp32)
 *   div6      Shaders/div6.comp / PixelOps.DivConcatNhwc
 *   nhwc2bgr  Shaders/nhwc2bgr.comp (crop, round, R/B swap, alpha from src) */
GCDR_API int gcdr_k_bgr2nhwc(const uint8_t *src, int w, int h, int stride, int fmt,
                             float *x, int ph, int pw, void *stream);
GCDR_API int gcdr_k_div6(const float *x, const float *shadow, size_t npx, float *out6, void *stream);
GCDR_API int gcdr_k_nhwc2bgr(const float *y, int H, int W, int ph, int pw, uint8_t *dst,
                             int w, int h, int dst_stride, int fmt, const uint8_t *alpha_src,
                             int alpha_stride, void *stream);

/* One tensor-core convolution layer, for layer-level parity tests and the
 * conv microbenchmark.  All pointers are DEVICE pointers.
 *   kind 0  3x3 stride 1, reflect pad 1   input [H+2][W+2][C] (gcdr_k_to_layout kind 1)
 *   kind 1  3x3 stride 2, zero pad 1      input phase planes (gcdr_k_to_layout kind 2)
 *   kind 2  1x1 (token Gemm)              input [H][W][C]
 *   kind 3  3x3 stride 1, zero pad 1      input [H+2][W+2][C] with a zero border
 *                                         (gcdr_k_to_layout kind 3)
 * weight: fp16 [N][taps*C], k = (ky*3 + kx)*C + c (taps = 9, or 1 for kind 2).
 * epilogue: 0 bias, 1 bias + maxpool 2x2 + relu, 2 bias + relu,
 *           3 raw fp32 split-K partial sums (no bias) into out as float
 *             [ksplit][Ho*Wo][N] (the first stage of the LayerNorm layers).
 * out: fp16 [Ho][Wo][N] (epilogue 0-2).  nsplit: N slices per 128-row tile
 * (N/nsplit a multiple of 16); ksplit: k splits (epilogue 3 only; must divide
 * 9*C/BK).  0 means 1.  reference != 0 runs the SIMT reference kernels instead
 * of tcgen05 (nsplit = ksplit = 1; scratch: ceil(Ho*pitch/128)*128*N floats).
 * bias_host: optional HOST copy of the bias (N floats).  The epilogues take the
 *   bias as kernel parameters, so without it gcdr_k_conv reads the device bias
 *   back first (a blocking copy); with it (or with epilogue 3, which adds no
 *   bias) the call only enqueues work on `stream`.
 * wait_cycles: bound of every device-side wait of the tensor-core kernel in SM
 *   cycles (0: the default, about 2 s).  A wait that runs out makes the kernel
 *   give up, drain its own copies and return; gcdr_k_status then reports
 *   GCDR_ERR_TIMEOUT.
 * timeout_probe: test hook; nonzero makes the kernel issue no copies and no
 *   MMAs, so its first waits run out after wait_cycles and nothing is written. */
typedef struct {
    int kind;
    int H, W, C, N;
    const void *in;
    const void *weight;
    const float *bias;
    int epilogue;
    void *out;
    float *scratch;
    int nsplit;
    int ksplit;
    const float *bias_host;
    long long wait_cycles;
    int timeout_probe;
} gcdr_conv_desc;
/* Enqueues one layer on `stream` (see bias_host for the one blocking case).
 * Device-side waits report through the current device's layer error word,
 * read by gcdr_k_status. */
GCDR_API int gcdr_k_conv(const gcdr_conv_desc *d, int reference, void *stream);
/* Waits for `stream`, then reads and clears the current device's layer error
 * word: GCDR_ERR_TIMEOUT if a gcdr_k_conv kernel gave up on a wait since the
 * last gcdr_k_status, else GCDR_OK (GCDR_ERR_DEVICE if the stream failed). */
GCDR_API int gcdr_k_status(void *stream);
/* Repacks fp16 NHWC [H][W][C] into a layer input layout:
 *   kind 1  [H+2][W+2][C] with a reflect border
 *   kind 2  four zero-bordered phase planes [(H+2)/2][(W+2)/2][C] (H, W even)
 *   kind 3  [H+2][W+2][C] with a zero border
 * Returns the element count of the layout when dst is NULL. */
GCDR_API int64_t gcdr_k_to_layout(const void *src, int H, int W, int C, int kind, void *dst, void *stream);
/* The token-stage kernels of the shifted-MLP blocks and decoder joins, for
 * kernel-level parity tests.  DEVICE pointers, fp16 activations, fp32
 * parameters (16-byte aligned), asynchronous on `stream`.
 *
 * gcdr_act: an activation in one of the layer layouts (kind 0 tokens
 * [H][W][C]; 1, 2, 3 as gcdr_k_to_layout).  gcdr_shift: a channel shift
 * (ChannelShiftOp, Extensions/ChannelShiftOp.cs:70-188): `ngroups` (<= 5)
 * cumulative channel-group ends; group g is shifted by offs[g]
 * (out[y] = in[y + off], zero fill), channels past the last end unshifted. */
typedef struct {
    void *p;
    int H, W, C;
    int kind;
} gcdr_act;
typedef struct {
    int ngroups;
    int ends[5];
    int offs[5];
} gcdr_shift;
/* Depthwise 3x3 (zero pad 1) + bias -> exact GELU -> shift along W
 * (gc#85-95): in, out tokens [H][W][C]; wt tap-major [9][C], b [C]. */
GCDR_API int gcdr_k_dw_gelu_shift(const void *in, int H, int W, int C, const float *wt, const float *b,
                                  const gcdr_shift *shift, void *out, void *stream);
/* Decoder join (gc#236-240): out = relu(bilinear2x(d)) + skip, d tokens
 * [H/2][W/2][C].  With g != NULL (token form, gc#240-250) out must be tokens
 * and h (tokens) gets LayerNorm(out; g, b, eps) shifted along H. */
GCDR_API int gcdr_k_up_add(const void *d, const gcdr_act *skip, const gcdr_act *out, const float *g,
                           const float *b, float eps, const gcdr_shift *shift, void *h, void *stream);
/* Finishes a split-K layer: per token, the ksplit fp32 partials
 * [ksplit][H*W][N] summed in order + bias (+ res tokens), then
 * out = LayerNorm(v; g1, b1, eps1) in out's layout; with g2 != NULL also
 * out2 (tokens) = LayerNorm(out; g2, b2, eps2) shifted along H. */
GCDR_API int gcdr_k_ln_finalize(const float *partial, int ksplit, int H, int W, int N, const float *bias,
                                const void *res, const float *g1, const float *b1, float eps1,
                                const float *g2, const float *b2, float eps2, const gcdr_shift *shift,
                                const gcdr_act *out, void *out2, void *stream);
/* Scratch floats gcdr_k_conv needs with reference != 0. */
GCDR_API int64_t gcdr_k_conv_scratch(const gcdr_conv_desc *d);
/* Number of SMs the tcgen05 kernels use on the current device. */
GCDR_API int gcdr_device_sms(void);

/* gcdr_k_conv_static -- no counterpart in the reference (its CPU and Vulkan
 * engines have no layer-level entry of this kind).  Runs the layer described
 * by `d` as a k-split tensor-core convolution without allocating any device
 * memory, for callers that must not allocate: the d->ksplit fp32 partial sums
 * (and the kernels' error word) live in a static workspace compiled into the
 * library, GCDR_STATIC_WS_BYTES per device, and are summed in order with the
 * bias (epilogue 2: then relu) into d->out, fp16 [Ho][Wo][N].
 *   - epilogue must be 0 or 2 (no pool); d->scratch is ignored; nsplit as in
 *     gcdr_k_conv; ksplit (0 = 1) must divide the layer's k-blocks.
 *   - ksplit * Ho * Wo * N must not exceed GCDR_STATIC_WS_BYTES / 4 floats,
 *     else GCDR_ERR_RANGE (nothing is launched, a message goes to stderr).
 *   - The first call on a device loads the workspace's address with
 *     cudaGetSymbolAddress (the driver reserves the workspace then): make it
 *     before any stream capture.  Every call looks the address up again.
 *   - Synchronous: returns after the layer has finished on `stream`
 *     (GCDR_ERR_TIMEOUT if a device-side wait expired).  d->bias stays on the
 *     device (bias_host is not needed).
 *   - One workspace per device: calls that overlap in time race on it. */
#define GCDR_STATIC_WS_BYTES (16 * 1024 * 1024)
GCDR_API int gcdr_k_conv_static(const gcdr_conv_desc *d, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* GCDR_CUDA_H */
