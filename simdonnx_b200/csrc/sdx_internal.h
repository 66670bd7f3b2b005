// Internal declarations shared by the libsdxcuda translation units.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <atomic>

#include "sdx_status.h"

struct sdx_ctx {
  int device;
  cudaStream_t stream;
  unsigned int* err_word;  // device error word (one per context)
  int poisoned;
  int sm_count;
};

namespace sdx {

// thread-local last-error message; returns `code`
int set_error(int code, const char* fmt, ...);
int set_cuda_error(cudaError_t e, const char* what);
void clear_error();

typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
PFN_encodeTiled get_encode_tiled();
int num_sms(int device);
void count_launch();

// Per-kernel, per-device record of the dynamic shared-memory limit already raised with
// cudaFuncSetAttribute (the attribute belongs to the kernel on the CURRENT device: a process that
// drives several GPUs must raise it on each). Zero-initialised as a function-local static.
constexpr int SDX_MAX_DEVICES = 64;
struct SmemAttr {
  std::atomic<int> bytes[SDX_MAX_DEVICES];
};
// Raises `fn`'s dynamic shared-memory limit to at least `bytes` on the current device, once per
// device (thread-safe: concurrent first calls both set the same value, which is idempotent). The
// record is updated only after the call succeeded, so a failure (e.g. inside a stream capture) is
// retried by the next launch. Returns SDX_OK or an SDX_ERR_CUDA status naming `what`.
int raise_smem_limit(SmemAttr& rec, const void* fn, int bytes, const char* what);
// fault injection: true when the call of `kind` must fail now (see sdx_fault_inject)
bool inject_fire(int kind);
enum { FAULT_MALLOC = 1, FAULT_LAUNCH = 2, FAULT_GRAPH = 3, FAULT_D2H = 4, FAULT_SYNC = 5 };

// ---- tcgen05 implicit GEMM (conv_tc.cu)
enum { TC_ROWS = 0, TC_CONV = 1 };
struct TcProblem {
  int mode;
  // A: TC_ROWS -> [M, K] rows with stride lda (halves); TC_CONV -> NHWC [batch, H, W, C] fp16
  const __half* a;
  int64_t lda;
  int M, K;
  int batch, H, W, C, OH, OW, kh, kw, pad_t, pad_l;
  // B: packed weights (tc_pack_*)
  const __half* w;
  int N;
  int wterms;  // fp16 weight terms in w: 1, or 2 (hi, lo)
  // epilogue
  const float* bias;
  const void* res;
  int res_f32;
  int64_t res_pix_stride;
  int res_ch_off;
  int res_up;  // 2: the residual is the nearest 2x downsample grid [batch, OH/2, OW/2, N] (read upsampled)
  float* gap;  // fp32 [M / 32][N]: channel sums of the activated output over each 32-row run, or null
  // pixel folding of a 1x1 conv (rows mode): M, K, N, lda, strides are those of the folded GEMM
  // (fold pixels per row, block-diagonal weights from tc_pack_conv_fold); bias_mod = OC, the
  // bias repeats every OC columns; gap (if any) is still [pixels / 32][OC]
  int fold;
  int bias_mod;
  // fused CTC head (rows mode, no output tensor): per row and N tile the argmax state over the
  // tile's columns of act(bias + A x B) ([n_tiles][M] each; merged by ctc_argmax_merge_launch)
  float* arg_m;
  int* arg_i;
  float* arg_s;
  int arg_ld;  // entries between two N tiles' states (>= M)
  // per-image weights (rows mode, one N tile, two terms): w holds M / img_rows consecutive weight
  // sets of the packed layout, image i's GEMM rows being [i * img_rows, (i + 1) * img_rows) with
  // img_rows a multiple of 128; 0 = one weight set for every row
  int img_rows;
  // fused depthwise 3x3 stride 1 pad 1 in front of this 1x1 conv (TC_CONV mode, kh = kw = 1): `a` is the
  // depthwise input [batch, H, W, C] (fp16 NHWC, C a multiple of 64, at most 128), dw_w [9][C] and
  // dw_b [C] its weights and bias, dw_scale [batch][C] a per-image input scale or null, dw_act its
  // activation; the depthwise output is built per tile in shared memory and never stored
  const float* dw_w;
  const float* dw_b;
  const float* dw_scale;
  int dw_act;
  void* out;
  int out_f32;
  int64_t out_pix_stride;
  int out_ch_off;
  int act;
  int convt_kh, convt_kw, convt_oc, convt_H, convt_W;
  int kxn;  // 3x3 conv with its column taps as GEMM columns (tc_conv_kxn)
  // ConvT chain: a second 2x2 stride-2 ConvT with one output channel applied in the epilogue to the
  // first one's (activated, fp32) output, which is never stored; `out` is unused then
  const float* chain_w2;  // raw fp32 [convt_oc][1][2][2]
  const float* chain_b2;  // [1]
  int chain_act2;
  void* chain_y;          // [batch, 4 * convt_H, 4 * convt_W, 1]
  int chain_y_f32;
  unsigned int* err;
};
void tc_plan_n(int N, int* BN, int* n_tiles);
int tc_launch(const TcProblem& p, cudaStream_t stream);
size_t tc_weights_halves(int N, int K, int taps, int terms);
// 3x3 stride-1 SAME convs with at most 64 output channels run with the three column taps kx as
// GEMM columns (N = 3 x 32, or 3 x 64 above 32 outputs): a third of the thin MMAs; the epilogue adds
// the column-shifted parts.
bool tc_conv_kxn(int kh, int kw, int sh, int sw, int pt, int pl, int pb, int pr, int oc, int ic, int terms);
int tc_kxn_block(int oc);
size_t tc_kxn_weights_halves(int K, int OC, int terms);
void tc_pack_conv_kxn(const float* w, int OC, int IC, int terms, __half* out);
size_t tc_convt_weights_halves(int IC, int OC, int KH, int KW);
void tc_plan_n_convt(int kh, int kw, int OC, int* BN, int* n_tiles);
void tc_pack_conv(const float* w, int OC, int IC, int KH, int KW, int terms, __half* out);
// Pixel folding factor of a 1x1 conv over `pixels` rows (1, 2 or 4): F consecutive pixels per GEMM
// row when OC * F <= 128 and IC * F <= 128 (thin convs: F times the pixels per tile for the same
// per-tile cost). The caller checks the layout conditions (dense fp16 output and residual).
int tc_fold_factor(int64_t pixels, int IC, int OC);
// Per-image weights of a 1x1 conv whose input is x * s (s fp32 [batch, K], an SE gate): out[i] =
// the two-term fp16 split of (w_hi + w_lo) * s[i, k] over every K column k of the packed rows-mode
// weights w (terms 1 or 2, `rows` rows of kpad halves per term); out is [batch][2][rows][kpad].
int tc_scale_weights_launch(const __half* w, int terms, int rows, int kpad, int K, const float* s, int batch,
                            __half* out, cudaStream_t st);
int tc_kpad_of(int K);
size_t tc_fold_weights_halves(int IC, int OC, int fold, int terms);
// Block-diagonal B operand of the folded GEMM: row j*OC + o, column j*IC + c = w[o][c]
void tc_pack_conv_fold(const float* w, int OC, int IC, int fold, int terms, __half* out);
void tc_pack_convt(const float* w, int IC, int OC, int KH, int KW, __half* out);
void tc_pack_gemm(const float* b, int K, int N, int trans_b, __half* out);

// ---- bandwidth kernels (bw_kernels.cu); all return SDX_* status
struct DwArgs {
  int batch, ih, iw, c, oh, ow, kh, kw, sh, sw, pt, pl, act;
  const __half* x;
  const float* w;  // [kh*kw][c]
  const float* bias;
  const float* in_scale;  // [batch, c] or null
  const __half* add;
  __half* y;
  unsigned int* err;      // device error word (bounded waits of the TMA-fed kernel)
};
int depthwise_launch(const DwArgs& a, cudaStream_t st);
// smem-tiled variant (tiled_kernels.cu); false when the shape is not one it handles
bool depthwise_tiled_launch(const DwArgs& a, cudaStream_t st);

struct DirectArgs {
  int batch, ih, iw, ic, oh, ow, oc, kh, kw, sh, sw, pt, pl, act;
  const void* x;
  int x_f32, x_nchw;
  const float* w;  // [kh*kw][ic][oc]
  const float* bias;
  const void* add;
  int add_f32, add_nchw;
  void* y;
  int y_f32, y_nchw;
  int64_t y_pix_stride;
  int y_ch_off;
  unsigned int* err;  // device error word (bounded waits of the TMA-fed stem)
  // fused 2x2 stride-2 max pool (ConvP.Pool): y is [batch, oh / 2, ow / 2, oc] NHWC (odd last
  // rows / columns of the conv output dropped), relu after the max when pool_relu
  int pool, pool_relu;
};
int direct_conv_launch(const DirectArgs& a, cudaStream_t st);
bool stem_tiled_launch(const DirectArgs& a, cudaStream_t st);

struct ConvtDotArgs {
  int batch, ih, iw, ic, oc, kh, kw, act, y_f32;
  const __half* x;
  const float* w;  // [ic][oc][kh][kw]
  const float* bias;
  void* y;
};
int convt_dot_launch(const ConvtDotArgs& a, cudaStream_t st);

struct PoolArgs {
  int batch, ih, iw, c, oh, ow, kh, kw, sh, sw, pt, pl, is_avg, relu, incl;
  const __half* x;
  __half* y;
  int64_t x_ps;  // elements between input pixels (c, or a wider tensor's when x is a channel slice)
  int x_co;      // first channel of that slice
};
int pool_launch(const PoolArgs& a, cudaStream_t st);

struct GateArgs {
  int batch, hw, c, r, act1_relu, hard;
  float alpha, beta, offset;
  const __half* x;
  const float *w1, *b1, *w2, *b2;
  float* s;
  float* partial;
  const float* sums;  // fp32 [batch][hw / 32][c] 32-pixel channel sums (a conv's fused output), or null
};
size_t gate_scratch_bytes(int batch, int hw, int c);
int gate_launch(const GateArgs& a, cudaStream_t st);

int broadcast_launch(int batch, int64_t pixels, int c, int op, int relu, const __half* x, const float* v, __half* y,
                     cudaStream_t st);

struct ResizeArgs {
  int batch, ih, iw, c, oh, ow, add_relu;
  int64_t y_pix_stride;
  int y_ch_off;
  const __half* x;
  const __half* add;
  __half* y;
};
int resize_launch(const ResizeArgs& a, cudaStream_t st);

struct ImageArgs {
  int batch, ih, iw, bpp, swap, oh, ow, pt, pl, y_nhwc_f16;
  int64_t stride, img_bytes;  // source row stride and per-image stride, bytes
  const uint8_t* src;
  const float* lut;           // [3][256]
  void* y;
};
int image_launch(const ImageArgs& a, cudaStream_t st);
// image normalisation fused into the det stem conv (tiled_kernels.cu); false when the conv is not
// that shape (the caller then runs the two nodes separately)
bool stem_image_launch(const ImageArgs& im, const DirectArgs& a, cudaStream_t st);

struct ConcatNearestArgs {
  int batch, oh, ow, nin, ctot;
  int c[8], s[8], off[8];  // channels, upsampling scale and first output channel of input i
  const __half* x[8];
  __half* y;
};
int concat_nearest_launch(const ConcatNearestArgs& a, cudaStream_t st);
int slice_copy_launch(int64_t pixels, int c, const __half* x, int64_t y_pix_stride, int y_ch_off, __half* y,
                      cudaStream_t st);
int binary_launch(int64_t n, int op, int relu, const __half* a, const __half* b, __half* y, cudaStream_t st);
int act_launch(int64_t n, int act, const __half* x, __half* y, cudaStream_t st);
int convert_launch(int batch, int c, int c_out, int64_t hw, int x_f32, int x_nchw, int y_f32, int y_nchw,
                   const void* x, void* y, cudaStream_t st);
int layernorm_launch(int64_t rows, int c, float eps, const __half* x, const float* w, const float* b, __half* y,
                     cudaStream_t st);
int softmax_launch(int64_t rows, int c, int y_f32, const __half* x, void* y, cudaStream_t st);
int attention_launch(int batch, int t, int heads, int d, float scale, const __half* qkv, __half* y, cudaStream_t st);
int bounded_wait_selftest_launch(unsigned int* err, int wait_ms, cudaStream_t st);

// ---- ext_kernels.cu: broadcast elementwise, fused ops, batched MatMul, CTC argmax merge
constexpr int BCAST_RANK_MAX = 6;
struct BcastArgs {
  int rank;                              // output rank (1 .. BCAST_RANK_MAX)
  int64_t shape[BCAST_RANK_MAX];     // output shape (contiguous output)
  int64_t sa[BCAST_RANK_MAX], sb[BCAST_RANK_MAX];  // element strides, 0 on broadcast dims
  int64_t n;                             // output elements
  int op, act, a_f32, b_f32, y_f32;
  const void* a;
  const void* b;
  void* y;
};
int bcast_binary_launch(const BcastArgs& p, cudaStream_t st);
int safediv_launch(int64_t n, float eps, float lo, float hi, int f32, const void* a, const void* b, void* y,
                   cudaStream_t st);
struct ShiftArgs {
  int batch, h, w, c, axis, ng;
  int ends[8], offs[8];
  int f32;
  const void* x;
  void* y;
};
int channel_shift_launch(const ShiftArgs& a, cudaStream_t st);
struct UpHeadArgs {
  int batch, ih, iw, c, oh, ow, oc;
  float sy, sx;  // resize scales (output / input) of H and W
  int resize_relu, skip_relu, act;
  int x_f32, skip_f32, y_f32;
  const void* x;
  const void* skip;
  const float* w;     // [oc][c]
  const float* bias;  // [oc] or null
  void* y;
};
int uphead_launch(const UpHeadArgs& a, cudaStream_t st);
struct MatMulArgs {
  int batch, m, k, n;
  int batch_rank;                               // output batch dims (<= 6)
  int64_t bshape[6], a_bstride[6], b_bstride[6];  // batch shape and per-operand element strides (0 = broadcast)
  int a_f32, b_f32, y_f32;
  const void* a;
  const void* b;
  void* y;
};
int batched_matmul_launch(const MatMulArgs& p, cudaStream_t st);
int ctc_argmax_merge_launch(const float* pm, const int* pi, const float* ps, int rows, int ld, int tiles,
                            int* indices, float* probs, unsigned int* err, cudaStream_t st);

}  // namespace sdx
