/*
 * libsdxcuda -- B200 (sm_100a) CUDA execution backend for SimdOnnx's fused conv/GEMM hot path.
 *
 * C ABI: plain pointers, sizes and POD descriptor structs; no C++ exceptions cross it. Every
 * function returns an int status (SDX_OK = 0); the message of the last failure on the calling
 * thread is read with sdx_last_error. Device pointers are opaque uint64 (sdx_dptr). A context is
 * used from one host thread at a time; different devices may run on different threads.
 *
 * It is the fourth execution backend beside the reference's CPU, Vulkan and Metal ones
 * (PlanTarget, src/Sdcb.SimdOnnx/Engine/ExecPlan.cs:320). The reference's Vulkan backend lowers
 * every ExecNode to a dispatch record (VkGraphModel.Emit, src/Sdcb.SimdOnnx/Backends/Vulkan/
 * VkGraph.cs:472-1112) over one device arena whose plan offsets map 1:1 to buffer offsets
 * (VkGraph.cs:362-378) and records them into one command buffer (VkSession.cs:282-337). Here the
 * same node list is issued through the sdx_* op entry points below on device pointers
 * (arena base + BufOffset * element size) and captured once into a CUDA graph by a session.
 *
 * Paths in comments are relative to the reference project root (src/ = src/Sdcb.SimdOnnx/).
 */
#ifndef SDXCUDA_H
#define SDXCUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif
#ifdef __cplusplus
extern "C" {
#endif

#define SDX_ABI_VERSION 1

/* ---- status codes (VkDevice errors -> exceptions in the reference, src/Backends/Vulkan/VkDevice.cs:11-18) */
#define SDX_OK 0
#define SDX_ERR_INVALID 1
#define SDX_ERR_CUDA 2
#define SDX_ERR_OOM 3
#define SDX_ERR_TIMEOUT 4
#define SDX_ERR_DEVICE 5
#define SDX_ERR_INJECTED 6
#define SDX_ERR_POISONED 7
#define SDX_ERR_NOT_SUPPORTED 8

typedef uint64_t sdx_dptr;
typedef struct sdx_ctx sdx_ctx;
typedef struct sdx_session sdx_session;
typedef void* sdx_stream; /* a cudaStream_t; NULL = the context's own stream */

/* ---- enums of the reference plan (src/Engine/ExecPlan.cs:42-46) */
enum sdx_act { SDX_ACT_NONE = 0, SDX_ACT_RELU = 1, SDX_ACT_SIGMOID = 2, SDX_ACT_GELU = 3, SDX_ACT_HARDSWISH = 4, SDX_ACT_SWISH = 5 };
enum sdx_ew { SDX_EW_ADD = 0, SDX_EW_SUB = 1, SDX_EW_MUL = 2, SDX_EW_DIV = 3 };
enum sdx_dtype { SDX_F16 = 0, SDX_F32 = 1 };
enum sdx_layout { SDX_NHWC = 0, SDX_NCHW = 1 };

/* ======================================================================================
 * Runtime (replaces the Vulkan device / buffer / queue layer, src/Backends/Vulkan/VkDevice.cs,
 * src/Backends/Vulkan/Vk.cs:452 P/Invoke surface)
 * ====================================================================================== */
int sdx_abi_version(void);
int sdx_last_error(char* buf, int len);
int sdx_device_count(int* count);
/* One context per device: owns a stream and a device error word (VkBackend.Default, VkBackend.cs:26-47). */
int sdx_open(int ordinal, sdx_ctx** ctx);
int sdx_close(sdx_ctx* ctx);
int sdx_ctx_stream(sdx_ctx* ctx, sdx_stream* stream);
int sdx_device_info(sdx_ctx* ctx, char* name, int name_len, int* sm_count, int* cc_major, int* cc_minor,
                    size_t* total_mem);
/* Device memory (the whole arena is one allocation, VkSession.cs:83-143). */
int sdx_malloc(sdx_ctx* ctx, size_t bytes, sdx_dptr* out);
int sdx_free(sdx_ctx* ctx, sdx_dptr p);
int sdx_host_alloc_pinned(size_t bytes, void** out);
int sdx_host_free(void* p);
int sdx_memcpy_htod_async(sdx_ctx* ctx, sdx_dptr dst, const void* src, size_t bytes, sdx_stream s);
int sdx_memcpy_dtoh_async(sdx_ctx* ctx, void* dst, sdx_dptr src, size_t bytes, sdx_stream s);
int sdx_memcpy_dtod_async(sdx_ctx* ctx, sdx_dptr dst, sdx_dptr src, size_t bytes, sdx_stream s);
int sdx_memset_async(sdx_ctx* ctx, sdx_dptr dst, int value, size_t bytes, sdx_stream s);
/* Streams (queue submit / fence wait, VkDevice.cs:885-898). timeout_ms <= 0 waits without a deadline;
 * otherwise SDX_ERR_TIMEOUT when the stream is still busy at the deadline (host watchdog). A device
 * error word set by a kernel turns into SDX_ERR_DEVICE and poisons the context. */
int sdx_stream_create(sdx_ctx* ctx, sdx_stream* out);
int sdx_stream_destroy(sdx_ctx* ctx, sdx_stream s);
int sdx_stream_sync(sdx_ctx* ctx, sdx_stream s, int timeout_ms);
int sdx_stream_query(sdx_ctx* ctx, sdx_stream s, int* done);
int sdx_event_create(sdx_ctx* ctx, void** ev);
int sdx_event_record(sdx_ctx* ctx, void* ev, sdx_stream s);
int sdx_event_elapsed_ms(void* start, void* stop, float* ms);
int sdx_event_destroy(void* ev);
/* CUDA graphs (the pre-recorded command buffer of VkInferenceSession.Record, VkSession.cs:282-337). */
int sdx_graph_begin(sdx_ctx* ctx, sdx_stream s);
int sdx_graph_end(sdx_ctx* ctx, sdx_stream s, void** graph_exec);
int sdx_graph_launch(sdx_ctx* ctx, void* graph_exec, sdx_stream s);
int sdx_graph_destroy(void* graph_exec);
/* Device error word: first error code a kernel recorded (bounded waits), 0 = none. */
int sdx_device_error(sdx_ctx* ctx, unsigned int* code);
int sdx_clear_device_error(sdx_ctx* ctx);
/* Fault injection (host side only; no GPU fault is ever provoked): the nth (1-based) call of `kind`
 * after this call returns SDX_ERR_INJECTED. kind: 1 malloc, 2 kernel launch, 3 graph launch,
 * 4 device-to-host copy, 5 stream sync. nth = 0 clears. Mirrors the host-faked device loss of
 * tests/Sdcb.SimdOnnx.Tests/VkDeviceLossTests.cs:28-33. */
int sdx_fault_inject(int kind, int nth);
/* Number of kernels this library launched in this process (bench accounting). */
uint64_t sdx_launch_count(void);
/* Self-test of the bounded device wait: one tiny kernel spins on a flag nothing sets for at most
 * `wait_ms` and then records SDX_DEV_TEST_WAIT (0x1F0) in the error word and returns. */
int sdx_selftest_bounded_wait(sdx_ctx* ctx, int wait_ms, sdx_stream s);

/* ======================================================================================
 * Weight packing (host): the backend-private const kinds of the GPU backends
 * (ConstKind / GpuPack, src/Engine/Extensions.cs:125-245); fp16 except biases (fp32).
 * Call with out == NULL to get the size in bytes in *bytes.
 * ====================================================================================== */
/* ConvP weights w [oc][ic/group][kh][kw] for the kernel sdx_conv2d routes `d` to (Nhwc.Pack,
 * src/Kernels/Nhwc.cs:102-125). The layout depends on the shape and layout fields of `d` (batch and
 * spatial sizes, channels, kernel, strides, pads, dtypes, layouts, y_pix_stride / y_ch_off, add_up,
 * w_terms) and on whether in_scale is set, not on the pointers' values: pack with the descriptor
 * that sdx_conv2d will get (thin 1x1 convs over whole fp16 tensors without in_scale are packed for
 * pixel folding, which depends on batch * ih * iw). */
struct sdx_conv_desc;
int sdx_pack_conv(const struct sdx_conv_desc* d, const float* w, void* out, size_t* bytes);
/* ConvTP weights w [ic][oc][kh][kw] (Nhwc.PackConvT, src/Kernels/Nhwc.Det.cs:26-44). */
int sdx_pack_convt(int ic, int oc, int kh, int kw, const float* w, void* out, size_t* bytes);
/* GemmP B [K,N] (or [N,K] when trans_b) (Nhwc.PackGemm, src/Kernels/Nhwc.cs:127-138). */
int sdx_pack_gemm(int k, int n, int trans_b, const float* b, void* out, size_t* bytes);

/* ======================================================================================
 * Ops: one entry point per fused ExecNode kind, enqueued on a stream, device pointers only.
 * ====================================================================================== */

/* Fused conv node: ConvP (src/Engine/ExecPlan.cs:50-65) executed by Nhwc.Conv / ConvPool
 * (src/Kernels/Nhwc.cs:172-217, :666-727). y = act(conv(x) + bias [+ add]) [then 2x2/2 max pool].
 * Routing (like VkGraphModel's conv routing, VkGraph.cs:159-320):
 *   group == ic == oc            -> depthwise bandwidth kernel
 *   ic % 8 == 0, stride 1, fp16  -> tcgen05 implicit GEMM (1x1 pad 0: batch folded into rows)
 *   otherwise (stem: ic = 3, stride 2, fp32 / NCHW input) -> direct small-channel kernel. */
typedef struct sdx_conv_desc {
  int batch, ih, iw, ic;
  int oh, ow, oc;
  int kh, kw, sh, sw;
  int pad_t, pad_l, pad_b, pad_r;
  int group;
  int act;           /* sdx_act */
  int pool;          /* 1: fused 2x2/2 max pool epilogue (ConvP.Pool); y is then [batch, oh/2, ow/2, oc] */
  int pool_relu;     /* relu after the pool (PoolP.FuseRelu) */
  int x_dtype;       /* sdx_dtype */
  int x_layout;      /* sdx_layout (NCHW only for the direct small-channel kernel: graph inputs) */
  int y_dtype;       /* sdx_dtype */
  int add_dtype;     /* sdx_dtype of the residual */
  int add_layout;    /* sdx_layout of the residual */
  int y_layout;      /* sdx_layout of the output */
  int pad_mode;      /* PadMode: 0 constant (the only mode with a CUDA kernel), 1 reflect -> NOT_SUPPORTED */
  float pad_value;   /* constant-mode fill; only 0 has a CUDA kernel */
  int64_t y_pix_stride; /* elements between output pixels (0 = oc); > oc writes into a channel slice */
  int y_ch_off;      /* first output channel in that slice */
  sdx_dptr x, w, bias, add, y;  /* w: packed by sdx_pack_conv; bias fp32 [oc] or 0; add 0 = none */
  sdx_dptr in_scale; /* fp32 [batch, ic] per-image channel scale of x (an SE gate's output: the conv reads
                        x * s without it being stored), or 0. Depthwise: applied to the staged weights.
                        1x1 tensor-core route: the weights are scaled per image into `w_scaled` first
                        (needs sdx_conv_scaled_weights_bytes(d) > 0, no gap_sums) */
  int w_terms;       /* tensor-core routes: fp16 weight terms, 1 (w) or 2 (hi + lo, ~22-bit weights);
                        0 = default: 2 for 1x1 kernels with ic < 128 (early narrow layers, whose weight
                        rounding every later layer amplifies), 1 for 1x1 kernels with ic >= 128 and for
                        larger kernels (their MMAs' operand traffic bounds them; one fp16 term is the
                        reference GPU backends' weight type) */
  int add_up;        /* 0 or 1: the residual as given; 2: `add` is [batch, oh/2, ow/2, oc] fp16 NHWC, read
                        nearest-upsampled (an FPN top-down ResizeNearest(x, add = this conv) fused into
                        the conv: y = act(conv + up2(add))); tensor-core routes, oh and ow even */
  sdx_dptr gap_sums; /* fp32 [batch * oh * ow / 32, oc]: channel sums of y over each run of 32 pixels
                        (the global average pool of a following SE gate, fused: pass it as that gate's
                        `sums`), or 0. 1x1 tensor-core route with the fp16 TMA-store epilogue
                        (y fp16, oc 16, 32, 64 or a multiple of 128, 16-byte aligned rows);
                        (batch * oh * ow) % 32 == 0 */
  sdx_dptr w_scaled; /* device scratch of sdx_conv_scaled_weights_bytes(d) bytes for a 1x1 conv with
                        in_scale (per-image two-term weights), else unused */
} sdx_conv_desc;
int sdx_conv2d(sdx_ctx* ctx, const sdx_conv_desc* d, sdx_stream s);
/* Fused depthwise -> pointwise (no reference counterpart; equals the two ConvP nodes it replaces): a
 * depthwise 3x3 conv, stride 1, pads 1 (`dw`: group == ic == oc, fp16 NHWC, bias, act, in_scale allowed;
 * its y is not written) whose output only the 1x1 conv `pw` reads (its x is ignored; bias, act and
 * gap_sums as sdx_conv2d; fp16 output, no residual). The depthwise output is built per 32 x 4 pixel
 * tile in shared memory and fed to the tensor cores; it never reaches HBM. dw.w: sdx_pack_conv(&dw),
 * pw.w: sdx_pack_conv(&pw). sdx_dw_pw_supported: 1 when the shapes take this form (64 or 128
 * channels, dw.act none, relu or hardswish, at most 128 outputs), else 0; pw.gap_sums further needs ow a multiple of 32 and oh of 4. */
typedef struct sdx_dwpw_desc {
  sdx_conv_desc dw, pw;
} sdx_dwpw_desc;
int sdx_dw_pw_supported(const sdx_dwpw_desc* d);
int sdx_dw_pw(sdx_ctx* ctx, const sdx_dwpw_desc* d, sdx_stream s);

/* Bytes of the per-image weight scratch a 1x1 tensor-core conv with in_scale needs (batch two-term
 * copies of its packed weights), or 0 when that form does not apply to the descriptor's shape: it
 * needs fp16 NHWC x, ic % 8 == 0, oc in [8, 128] and ic <= 256. */
size_t sdx_conv_scaled_weights_bytes(const sdx_conv_desc* d);

/* Gemm node: GemmP (src/Engine/ExecPlan.cs:87-93) via Nhwc.Gemm (src/Kernels/Nhwc.Avx512.cs:241-266):
 * y[m, n] = act(a[m, k] . B + bias[n] [+ add[m, n]]), a fp16 row stride lda, y fp16/fp32. */
typedef struct sdx_gemm_desc {
  int m, k, n;
  int64_t lda;
  int act;
  int y_dtype, add_dtype;
  int64_t ldy, ldadd;
  sdx_dptr a, w, bias, add, y;
} sdx_gemm_desc;
int sdx_gemm(sdx_ctx* ctx, const sdx_gemm_desc* d, sdx_stream s);

/* Fused CTC projection + argmax (CtcProjection.ArgMax, src/Decoding/CtcProjection.cs:47-55;
 * MatMul.TryArgMax, src/Decoding/Kernels/MatMul.ArgMax.cs:29-70): for each of the m rows of the Gemm
 * `gemm` (a [m, k] fp16 x packed B [k, n] + bias; act none, no residual; y unused), the index of the
 * largest logit (ties keep the first) into indices (int32 [m]) and its softmax probability over the
 * row into probs (fp32 [m]); the [m, n] logits are never stored. The tensor-core epilogue folds each
 * 128-column tile into (max, index, online denominator) as UpdateArgMax does; a second kernel merges
 * the tiles in column order. scratch: sdx_gemm_argmax_scratch_bytes(m, n) bytes of device memory.
 * A non-finite logit records SDX_DEV_NONFINITE (0x201) in the device error word and writes index -1
 * (the reference throws InvalidDataException); sdx_stream_sync then returns SDX_ERR_DEVICE. */
typedef struct sdx_gemm_argmax_desc {
  sdx_gemm_desc gemm;
  sdx_dptr indices, probs, scratch;
} sdx_gemm_argmax_desc;
size_t sdx_gemm_argmax_scratch_bytes(int m, int n);
int sdx_gemm_argmax(sdx_ctx* ctx, const sdx_gemm_argmax_desc* d, sdx_stream s);

/* ConvTranspose node, stride == kernel, no pad (ConvTP, src/Engine/ExecPlan.cs:108-114;
 * Nhwc.ConvTranspose / ConvTDot, src/Kernels/Nhwc.Det.cs:51-131). x fp16 NHWC, y [b, ih*kh, iw*kw, oc]. */
typedef struct sdx_convt_desc {
  int batch, ih, iw, ic, oc, kh, kw;
  int act, y_dtype;
  sdx_dptr x, w, bias, y;  /* w packed by sdx_pack_convt (oc >= 8) or raw fp32 [ic][oc][kh][kw] (oc < 8) */
} sdx_convt_desc;
int sdx_convt(sdx_ctx* ctx, const sdx_convt_desc* d, sdx_stream s);

/* Two chained ConvTranspose nodes, the second reading only the first's output (the det head's
 * ConvT 2x2 -> ConvT 2x2): `first` as in sdx_convt (oc 8, 16 or 24, 2x2, packed by sdx_pack_convt; its y
 * is not written), then a 2x2 stride-2 ConvT to one channel with raw fp32 weights w2
 * [first.oc][1][2][2], bias2 [1] and act2, written to y [batch, 4 * ih, 4 * iw, 1] (y_dtype).
 * No reference counterpart (ConvTranspose nodes run one by one there); equals sdx_convt twice with
 * the intermediate kept in fp32. SDX_ERR_NOT_SUPPORTED for other shapes. */
typedef struct sdx_convt_chain_desc {
  sdx_convt_desc first;
  int oc2, kh2, kw2, act2, y_dtype;
  sdx_dptr w2, bias2, y;
} sdx_convt_chain_desc;
int sdx_convt_chain(sdx_ctx* ctx, const sdx_convt_chain_desc* d, sdx_stream s);

/* Max / average pool (PoolP, src/Engine/ExecPlan.cs:67-74; Nhwc.MaxPool src/Kernels/Nhwc.cs:730-770,
 * Nhwc.AvgPool src/Kernels/Ops.Seq.cs:180-225). fp16 NHWC. */
typedef struct sdx_pool_desc {
  int batch, ih, iw, c, oh, ow, kh, kw, sh, sw, pad_t, pad_l;
  int is_avg, relu, count_include_pad;
  sdx_dptr x, y;
  int64_t x_pix_stride; /* elements between input pixels (0 = c): x is a channel slice of a wider tensor */
  int x_ch_off;         /* first channel of that slice */
} sdx_pool_desc;
int sdx_pool(sdx_ctx* ctx, const sdx_pool_desc* d, sdx_stream s);

/* Squeeze-excitation gate (ChannelGateP, src/Engine/ExecPlan.cs:151-158; Nhwc.ChannelGate,
 * src/Kernels/Nhwc.Det.cs:287-314): s[n, c] = gate(b2 + W2 . act1(b1 + W1 . mean_hw x[n])) + offset.
 * x fp16 NHWC; w1 fp32 [r][c], w2 fp32 [c][r]; s fp32 [batch, c]. `partial` is device scratch of
 * sdx_channel_gate_scratch_bytes() bytes (per-block channel sums and the hidden layer); r <= c. */
typedef struct sdx_gate_desc {
  int batch, hw, c, r;
  int act1_relu, hard;
  float alpha, beta, offset;
  sdx_dptr x, w1, b1, w2, b2, s, partial;
  sdx_dptr sums;     /* fp32 [batch, hw / 32, c]: 32-pixel channel sums of x written by the producing
                        conv (sdx_conv_desc.gap_sums), or 0. When set, x is not read; hw % 32 == 0 */
} sdx_gate_desc;
size_t sdx_channel_gate_scratch_bytes(int batch, int hw, int c);
int sdx_channel_gate(sdx_ctx* ctx, const sdx_gate_desc* d, sdx_stream s);

/* Same gate as sdx_channel_gate, but it allocates nothing: the channel-sum scratch is a fixed
 * device array inside the library (one per device) of SDX_GATE_STATIC_MAX_SCRATCH_BYTES, and
 * d->partial is ignored. No counterpart in the reference (its CPU gate uses stack/pooled buffers).
 * For callers that cannot hand out device memory at call time: a host runtime that owns all device
 * memory and gives its plugins no allocator, or a caller that must not pay cudaMalloc/cudaFree,
 * which can wait for work already running on the device.
 * Limits and rules:
 *  - sdx_channel_gate_scratch_bytes(batch, hw, c) must be <= SDX_GATE_STATIC_MAX_SCRATCH_BYTES,
 *    else SDX_ERR_NOT_SUPPORTED (nothing enqueued); e.g. c = 512 with one pixel chunk allows
 *    1024 images.
 *  - The first call on a device looks up the array's device address (cudaGetSymbolAddress) and
 *    caches it; make that first call before beginning any stream capture on that device. The
 *    cached address belongs to the device's primary context: after cudaDeviceReset (or anything
 *    else that destroys that context) do not call this entry point again in the same process.
 *  - All calls on one device share the one array: two calls whose kernels overlap on the GPU
 *    (different streams, no ordering between them) race and give wrong gates. Order them on one
 *    stream or with events.
 *  - The array keeps the last call's partial sums; each call writes every entry it reads before
 *    reading it, so nothing needs clearing. */
#define SDX_GATE_STATIC_MAX_SCRATCH_BYTES (4 * 1024 * 1024)
int sdx_channel_gate_static(sdx_ctx* ctx, const sdx_gate_desc* d, sdx_stream s);

/* Per-image channel broadcast y[n, p, c] = x[n, p, c] op v[n, c] (+relu) (Ew.Channel via
 * Ops.Elementwise, src/Kernels/Ops.cs:388-420). x, y fp16; v fp32. */
int sdx_channel_broadcast(sdx_ctx* ctx, int batch, int64_t pixels, int c, int op, int relu, sdx_dptr x,
                          sdx_dptr v, sdx_dptr y, sdx_stream s);

/* Nearest resize, asymmetric floor, integer scale, + optional addend (ResizeNearestP +
 * FuseResizeAdd, src/Engine/GraphCompiler.cs:911-948; Nhwc.ResizeNearest, src/Kernels/Nhwc.Det.cs:167-204).
 * fp16 NHWC; y may be a channel slice (y_pix_stride, y_ch_off) of a wider tensor (fused concat). */
typedef struct sdx_resize_desc {
  int batch, ih, iw, c, oh, ow;
  int add_relu;
  int64_t y_pix_stride;
  int y_ch_off;
  sdx_dptr x, add, y;
} sdx_resize_desc;
int sdx_resize_nearest(sdx_ctx* ctx, const sdx_resize_desc* d, sdx_stream s);

/* NHWC channel concat (Nhwc.ConcatInner, src/Kernels/Nhwc.Det.cs:354-370), fp16, up to 8 inputs. An
 * input pointer of 0 means that input's producer already wrote its slice of y (its channels still
 * count for the slice offsets). */
int sdx_concat_channels(sdx_ctx* ctx, int64_t pixels, int nin, const int* counts, const sdx_dptr* ins,
                        sdx_dptr y, sdx_stream s);
/* Image-session preprocessing (the reference's Vulkan image session, src/Backends/Vulkan/
 * VkImageSession.cs; shader src/Backends/Vulkan/Shaders/img2nhwc.comp:4-37): interleaved u8 pixels
 * (bpp 3 or 4, row stride `stride` bytes, images `image_bytes` apart; 0 = packed) mapped through
 * lut[c * 256 + byte] (fp32 [3][256], tensor channel c; swap_rb = 1 takes channel 0 from byte 2),
 * replicate padding around the image placed at (pad_t, pad_l) of the [oh, ow] tensor. Output fp32
 * NCHW [batch, 3, oh, ow] (y_nhwc_f16 = 0) or fp16 NHWC [batch, oh, ow, 3]. */
typedef struct sdx_image_desc {
  int batch, ih, iw, bpp, swap_rb;
  int oh, ow, pad_t, pad_l, y_nhwc_f16;
  int64_t stride, image_bytes;
  sdx_dptr src, lut, y;
} sdx_image_desc;
int sdx_image_to_tensor(sdx_ctx* ctx, const sdx_image_desc* d, sdx_stream s);

/* The image-session preprocessing fused into the first conv of the graph: the conv `conv` reads the
 * tensor that `image` describes (conv.ih/iw = image.oh/ow, 3 channels; conv.x and image.y are not
 * used), so the fp32 tensor is never materialised. No reference counterpart (VkImageSession runs
 * img2nhwc.comp as its own pass); results equal sdx_image_to_tensor followed by sdx_conv2d.
 * SDX_ERR_NOT_SUPPORTED when the conv is not a shape the fused kernel handles (today the 3 -> 16,
 * 3x3 stride-2 stem with fp16 NHWC output); the caller then runs the two calls. */
typedef struct sdx_image_conv_desc {
  sdx_image_desc image;
  sdx_conv_desc conv;
} sdx_image_conv_desc;
int sdx_image_conv(sdx_ctx* ctx, const sdx_image_conv_desc* d, sdx_stream s);

/* Channel concat of nearest-upsampled inputs: y[n, oy, ox, off_i + c] = x_i[n, oy / s_i, ox / s_i, c]
 * (a Concat whose inputs are ResizeNearest outputs, Nhwc.ResizeNearest src/Kernels/Nhwc.Det.cs:160-200,
 * fused with Nhwc.ConcatInner). Input i is [batch, oh / s_i, ow / s_i, counts[i]] fp16 NHWC; s_i = 1
 * for a full-size input. Every output pixel is written whole. */
int sdx_concat_nearest(sdx_ctx* ctx, int batch, int oh, int ow, int nin, const int* counts, const int* scales,
                       const sdx_dptr* ins, sdx_dptr y, sdx_stream s);

/* Elementwise binary on equal shapes (Ew.Binary, src/Kernels/Ew.cs:75-84), fp16, optional relu. */
int sdx_binary(sdx_ctx* ctx, int64_t n, int op, int relu, sdx_dptr a, sdx_dptr b, sdx_dptr y, sdx_stream s);
/* Activation node (Act.Apply, src/Kernels/Act.cs:70-81), fp16. */
int sdx_act(sdx_ctx* ctx, int64_t n, int act, sdx_dptr x, sdx_dptr y, sdx_stream s);

/* Elementwise binary with numpy broadcasting (Ops.Elementwise, src/Kernels/Ops.cs:388-441):
 * y = act(a op b) over out_shape; a_shape / b_shape are right-aligned to `rank` (leading 1s for a
 * lower-rank operand) and each dim is 1 or the output's. act: the EwP activation (relu fused in the
 * reference; the others applied after, the same elementwise result). Storage per operand fp16 or
 * fp32 (sdx_dtype), arithmetic fp32; y contiguous. */
#define SDX_BCAST_MAX_RANK 6
typedef struct sdx_bcast_desc {
  int rank;
  int64_t out_shape[SDX_BCAST_MAX_RANK], a_shape[SDX_BCAST_MAX_RANK], b_shape[SDX_BCAST_MAX_RANK];
  int op, act;
  int a_dtype, b_dtype, y_dtype;
  sdx_dptr a, b, y;
} sdx_bcast_desc;
int sdx_binary_bcast(sdx_ctx* ctx, const sdx_bcast_desc* d, sdx_stream s);

/* SafeDiv fused op: y = clamp(a / max(b, eps), lo, hi) over n same-shape elements, fp32 arithmetic
 * (SafeDivOp, src/Engine/Fusions/SafeDivOp.cs:14-34; FusedKernels.SafeDiv, src/Kernels/FusedKernels.cs:32-55). */
typedef struct sdx_safediv_desc {
  int64_t n;
  float eps, lo, hi;
  int dtype;  /* storage of a, b and y (sdx_dtype) */
  sdx_dptr a, b, y;
} sdx_safediv_desc;
int sdx_safe_div(sdx_ctx* ctx, const sdx_safediv_desc* d, sdx_stream s);

/* ChannelShift fused op, NHWC (ChannelShiftOp / ShiftP, src/Engine/Fusions/ChannelShiftOp.cs:9-66;
 * FusedKernels.ChannelShift, src/Kernels/FusedKernels.cs:196-221): channel group g = [end[g-1], end[g])
 * reads y[n, y, x, ch] = x[n, y + off[g], x, ch] (axis 2) or x[n, y, x + off[g], ch] (axis 3), zero
 * outside the image; channels from the last end on are copied. Up to 8 groups. */
typedef struct sdx_shift_desc {
  int batch, h, w, c;
  int axis;  /* 2: shift along H, 3: along W (the logical NCHW axis) */
  int ngroups;
  int group_ends[8], offsets[8];
  int dtype;
  sdx_dptr x, y;
} sdx_shift_desc;
int sdx_channel_shift(sdx_ctx* ctx, const sdx_shift_desc* d, sdx_stream s);

/* UpHead fused network tail, NHWC (UpHeadOp / UpHeadP, src/Engine/Fusions/UpHeadOp.cs:9-30;
 * FusedKernels.UpHead, src/Kernels/FusedKernels.cs:71-193): y[n, oy, ox, o] = act(bias[o] +
 * sum_c w[o, c] * s[c]), s = [relu](bilinear resize of x by (scale_h, scale_w)) + [relu](skip), the
 * full-resolution resize / add tensors never stored. x [batch, ih, iw, c], skip and y at [oh, ow];
 * w fp32 [oc][c] (the 1x1 conv's weights), bias fp32 [oc] or 0; oc <= 8, c % 4 == 0, c <= 128;
 * act none, relu or sigmoid. The reference's recomputed-skip variant (UpHeadP.SkipConv) has no CUDA
 * kernel: run the skip conv, then this. */
typedef struct sdx_uphead_desc {
  int batch, ih, iw, c, oh, ow, oc;
  float scale_h, scale_w;
  int resize_relu, skip_relu, act;
  int x_dtype, skip_dtype, y_dtype;
  sdx_dptr x, skip, w, bias, y;
} sdx_uphead_desc;
int sdx_uphead(sdx_ctx* ctx, const sdx_uphead_desc* d, sdx_stream s);

/* Batched MatMul of two activations (ExecOp.MatMul, Ops.MatMul src/Kernels/Ops.Seq.cs:90-113):
 * a [.., m, k] x b [.., k, n] -> y [batch dims, m, n] with numpy broadcast over the batch dims (shapes
 * right-aligned to `rank` >= 2, leading 1s). fp32 accumulation in ascending k. */
typedef struct sdx_matmul_desc {
  int rank;
  int64_t a_shape[SDX_BCAST_MAX_RANK], b_shape[SDX_BCAST_MAX_RANK];
  int a_dtype, b_dtype, y_dtype;
  sdx_dptr a, b, y;
} sdx_matmul_desc;
int sdx_matmul(sdx_ctx* ctx, const sdx_matmul_desc* d, sdx_stream s);
/* Storage conversion / boundary relayout: fp32 <-> fp16, NCHW <-> NHWC (VkSession f32to16 / f16to32
 * staging, src/Backends/Vulkan/VkSession.cs:286-310). */
int sdx_convert(sdx_ctx* ctx, int batch, int c, int64_t hw, int x_dtype, int x_layout, int y_dtype, int y_layout,
                sdx_dptr x, sdx_dptr y, sdx_stream s);
/* The same with the channels zero-padded to c_out >= c (a 3-channel graph input widened to 8 so that
 * a tensor-core conv reads it). Session node SDX_OP_CONVERT: misc.aux[0] = c_out, or 0 for c. */
int sdx_convert_pad(sdx_ctx* ctx, int batch, int c, int c_out, int64_t hw, int x_dtype, int x_layout, int y_dtype,
                    int y_layout, sdx_dptr x, sdx_dptr y, sdx_stream s);

/* LayerNorm over the last dim (LnP, Ops.LayerNorm src/Kernels/Ops.cs:544-575), fp16 in/out, fp32 w/b. */
int sdx_layernorm(sdx_ctx* ctx, int64_t rows, int c, float eps, sdx_dptr x, sdx_dptr w, sdx_dptr b, sdx_dptr y,
                  sdx_stream s);
/* Row softmax (Ops.Softmax, src/Kernels/Ops.Seq.cs:28-75), fp16 in, fp16/fp32 out. */
int sdx_softmax(sdx_ctx* ctx, int64_t rows, int c, int y_dtype, sdx_dptr x, sdx_dptr y, sdx_stream s);
/* Fused attention (AttentionP, src/Engine/ExecPlan.cs:160-174; GPU plans fuse MatMul -> scale ->
 * Softmax -> MatMul, src/Engine/GraphCompiler.cs:614-770): qkv fp16 [batch, t, 3, heads, d] rows
 * (one fused projection), out fp16 [batch, t, heads*d]. */
int sdx_attention(sdx_ctx* ctx, int batch, int t, int heads, int d, float scale, sdx_dptr qkv, sdx_dptr y,
                  sdx_stream s);

/* ======================================================================================
 * Session: CudaGraphModel + CudaInferenceSession (the VkGraphModel / VkInferenceSession pair,
 * src/Backends/Vulkan/VkGraph.cs:44-155, src/Backends/Vulkan/VkSession.cs:63-143). Nodes are added
 * in plan order with device pointers into the session arena; sdx_session_build captures them into
 * one CUDA graph; sdx_session_run = H2D of the input + graph launch + D2H of the output + sync.
 * ====================================================================================== */
enum sdx_op_kind {
  SDX_OP_CONV = 1, SDX_OP_GEMM = 2, SDX_OP_CONVT = 3, SDX_OP_POOL = 4, SDX_OP_CHANNEL_GATE = 5,
  SDX_OP_CHANNEL_BROADCAST = 6, SDX_OP_RESIZE_NEAREST = 7, SDX_OP_CONCAT = 8, SDX_OP_BINARY = 9, SDX_OP_ACT = 10,
  SDX_OP_CONVERT = 11, SDX_OP_LAYERNORM = 12, SDX_OP_SOFTMAX = 13, SDX_OP_ATTENTION = 14,
  SDX_OP_CONCAT_NEAREST = 15, SDX_OP_IMAGE = 16, SDX_OP_IMAGE_CONV = 17, SDX_OP_CONVT_CHAIN = 18,
  SDX_OP_BINARY_BCAST = 19, SDX_OP_SAFE_DIV = 20, SDX_OP_CHANNEL_SHIFT = 21, SDX_OP_UPHEAD = 22,
  SDX_OP_MATMUL = 23, SDX_OP_GEMM_ARGMAX = 24, SDX_OP_DW_PW = 25
};
/* Generic argument block for the ops without a descriptor struct. */
typedef struct sdx_misc_desc {
  int64_t n, rows, pixels;
  int batch, c, t, heads, d, op, act, relu, x_dtype, x_layout, y_dtype, y_layout, nin;
  int counts[8];
  float eps, scale;
  sdx_dptr a, b, x, y, w, bias;
  sdx_dptr ins[8];
  int aux[8];  /* SDX_OP_CONCAT_NEAREST: per-input scale */
} sdx_misc_desc;

/* sizeof the descriptor struct sdx_session_add_node expects for op_kind (0 = unknown kind). */
size_t sdx_desc_size(int op_kind);
int sdx_session_create(sdx_ctx* ctx, size_t arena_bytes, sdx_session** out);
int sdx_session_arena(sdx_session* s, sdx_dptr* base, size_t* bytes);
int sdx_session_add_node(sdx_session* s, int op_kind, const void* desc, size_t desc_bytes);
int sdx_session_set_io(sdx_session* s, sdx_dptr in, size_t in_bytes, sdx_dptr out, size_t out_bytes);
int sdx_session_build(sdx_session* s, int use_graph);
int sdx_session_stream(sdx_session* s, sdx_stream* stream);
/* Device-resident run: replay the node list (graph) on the session stream, no copies, no sync. */
int sdx_session_enqueue(sdx_session* s);
/* End-to-end run: host input -> device, graph, device -> host output, wait (timeout_ms as sdx_stream_sync). */
int sdx_session_run(sdx_session* s, const void* host_in, void* host_out, int timeout_ms);
/* Pipelined end-to-end runs (the Submit / Wait split of VkInferenceSession, src/Backends/Vulkan/
 * VkSession.cs:543-556, with the host copies inside): submit enqueues host -> device copy of host_in, the graph and the device ->
 * host copy into host_out, and returns at once. Two device staging slots per direction and two copy
 * streams let the input copy of batch i+1 and the output copy of batch i-1 run while batch i
 * computes. host_in / host_out should be pinned (sdx_host_alloc_pinned) and must stay valid and
 * unmodified until sdx_session_wait returns; with more than two submissions in flight, alternate
 * at least two host buffer pairs. sdx_session_wait blocks until every submission finished. */
int sdx_session_submit(sdx_session* s, const void* host_in, void* host_out);
int sdx_session_wait(sdx_session* s, int timeout_ms);
int sdx_session_node_count(sdx_session* s, int* count);
/* Runs node `index` alone, eagerly, on the session stream (per-node timing, like the reference's
 * VkInferenceSession.DebugProfile, src/Backends/Vulkan/VkSession.cs:413-492). */
int sdx_session_enqueue_node(sdx_session* s, int index);
int sdx_session_destroy(sdx_session* s);

#ifdef __cplusplus
}
#endif
#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#endif /* SDXCUDA_H */
