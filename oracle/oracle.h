// CPU restatement of SimdOnnx's NHWC CPU kernels (the reference's own CPU path for the fused
// conv/GEMM hot path). TEST INFRASTRUCTURE ONLY: this library is the parity checker and the timed
// CPU baseline. The product (libsdxcuda) never links, loads or calls it.
//
// Every function names the reference file:line it restates (paths relative to the SimdOnnx
// project root, `src/` = src/Sdcb.SimdOnnx). Per output element the arithmetic follows the
// reference: bias-init, taps ascending, input channels ascending, one fused multiply-add per
// product, then the residual add, then the activation (src/Kernels/Nhwc.Avx512.cs:11-18).
//
// All tensors are fp32, NHWC, batch-major ([N, H, W, C]), contiguous.
#pragma once
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// ActivationKind (src/Engine/ExecPlan.cs:42): None, Relu, Sigmoid, Gelu, HardSwish, Swish.
enum { ORC_ACT_NONE = 0, ORC_ACT_RELU = 1, ORC_ACT_SIGMOID = 2, ORC_ACT_GELU = 3, ORC_ACT_HARDSWISH = 4, ORC_ACT_SWISH = 5 };
// PadMode (src/Engine/ExecPlan.cs:44).
enum { ORC_PAD_CONSTANT = 0, ORC_PAD_REFLECT = 1 };
// EwOp (src/Engine/ExecPlan.cs:46).
enum { ORC_EW_ADD = 0, ORC_EW_SUB = 1, ORC_EW_MUL = 2, ORC_EW_DIV = 3 };

void orc_set_threads(int threads);
int orc_get_threads(void);
// 1 when this build vectorises with AVX-512, 0 for the AVX2 build.
int orc_isa_avx512(void);

// ---- weight packing (src/Kernels/Nhwc.cs:102-138, src/Kernels/NhwcWinograd.cs:46-68, src/Kernels/Nhwc.Det.cs:26-44)
// Dense: w [oc][ic][kh][kw] -> pw [ceil(oc/16)][kh*kw][ic][16], pb [ceil(oc/16)*16].
int64_t orc_pack_conv_floats(int oc, int ic, int kh, int kw);
void orc_pack_conv(const float* w, const float* bias, int oc, int ic, int kh, int kw, float* pw, float* pb);
// Depthwise: w [c][1][kh][kw] -> pw [kh*kw][c], pb [c].
void orc_pack_depthwise(const float* w, const float* bias, int c, int kh, int kw, float* pw, float* pb);
// Winograd F(4x4,3x3): w [oc][ic][3][3] -> u [36][ceil(oc/16)][ic][16].
int64_t orc_pack_winograd_floats(int oc, int ic);
void orc_pack_winograd(const float* w, int oc, int ic, float* u);
// Gemm B ([K,N], or [N,K] when transB) -> pw [ceil(n/16)][k][16], pb [ceil(n/16)*16].
void orc_pack_gemm(const float* b, int k, int n, int trans_b, const float* bias, float* pw, float* pb);
// Winograd eligibility (src/Kernels/NhwcWinograd.cs:28-32), Vector<float>.Count = 8.
int orc_winograd_eligible(int group, int kh, int kw, int sh, int sw, int ic);

// ---- dense / depthwise conv (src/Kernels/Nhwc.cs:172-217 and the kernels it dispatches to)
// pw/pb from orc_pack_conv (dense) or orc_pack_depthwise (depthwise != 0); wino_u from
// orc_pack_winograd or NULL (direct conv). add: same-shape residual or NULL.
void orc_conv(const float* src, int batch, int ih, int iw, int ic, float* dst, int oh, int ow, int oc,
              int kh, int kw, int sh, int sw, int pt, int pl, int pad_mode, float pad_value,
              const float* pw, const float* pb, const float* wino_u, int depthwise,
              const float* add, int act);
// Dense conv + fused 2x2/2 max pool (src/Kernels/Nhwc.cs:666-727); dst [batch, oh/2, ow/2, oc].
void orc_conv_pool(const float* src, int batch, int ih, int iw, int ic, float* dst, int oh, int ow, int oc,
                   int kh, int kw, int sh, int sw, int pt, int pl, int pad_mode, float pad_value,
                   const float* pw, const float* pb, const float* wino_u, int act, int pool_relu);
// Plain fp64 direct conv (grouped), ONNX weights [oc][ic/group][kh][kw]; the independent check.
void orc_conv_ref64(const float* src, int batch, int ih, int iw, int ic, double* dst, int oh, int ow, int oc,
                    int kh, int kw, int sh, int sw, int pt, int pl, int group, int pad_mode, float pad_value,
                    const float* w, const float* bias, const float* add, int act);

// ---- Gemm (src/Kernels/Nhwc.Avx512.cs:241-266): dst[m,n] = act(a[m,k] . B + bias)
void orc_gemm(const float* a, int m, int k, float* dst, int n, const float* pw, const float* pb, int act);
// Batched MatMul of two activations (src/Kernels/Ops.Seq.cs:92-125 -> src/Kernels/Avx2Kernels.cs:504-560)
// a [batch, m, k] x b [batch, k, n] -> dst [batch, m, n].
void orc_matmul(const float* a, const float* b, float* dst, int batch, int m, int k, int n);

// ---- ConvTranspose stride == kernel (src/Kernels/Nhwc.Det.cs:26-131); w [ic][oc][kh][kw]
void orc_convt(const float* src, int batch, int ih, int iw, int ic, float* dst, int oc, int kh, int kw,
               const float* w, const float* bias, int act);

// ---- pools (src/Kernels/Nhwc.cs:730-770, src/Kernels/Ops.Seq.cs:180-225, src/Kernels/Nhwc.Det.cs:134-164)
void orc_maxpool(const float* src, int batch, int ih, int iw, int c, float* dst, int oh, int ow,
                 int kh, int kw, int sh, int sw, int pt, int pl, int relu);
void orc_avgpool(const float* src, int batch, int ih, int iw, int c, float* dst, int oh, int ow,
                 int kh, int kw, int sh, int sw, int pt, int pl, int count_include_pad);
// dst [batch, c]; chunks follow the reference's thread-dependent split (threads = orc_get_threads()).
void orc_global_avg_pool(const float* src, int batch, int hw, int c, float* dst);

// ---- SE gate (src/Kernels/Nhwc.Det.cs:287-314): s [batch, c]
void orc_channel_gate(const float* src, int batch, int hw, int c, const float* w1, const float* b1,
                      const float* w2, const float* b2, int r, int act1_relu, int hard, float alpha, float beta,
                      float offset, float* dst);
// dst[n, p, c] = full[n, p, c] op vec[n, c] (src/Kernels/Ops.cs:388-420 -> src/Kernels/Ew.cs Channel path)
void orc_channel_broadcast(const float* full, const float* vec, float* dst, int batch, int64_t rows, int c,
                           int op, int rev, int relu);
// Nearest resize (+ addend) (src/Kernels/Nhwc.Det.cs:167-204).
void orc_resize_nearest(const float* src, int batch, int ih, int iw, int c, float* dst, int oh, int ow,
                        float sy, float sx, const float* add, int add_relu);
// NHWC channel concat (src/Kernels/Nhwc.Det.cs:354-370): ins[i] has counts[i] channels per row.
void orc_concat_inner(const float* const* ins, const int* counts, int nin, int64_t outer, float* dst);

// ---- elementwise / activations (src/Kernels/Ops.cs:388-441, src/Kernels/Act.cs:70-117)
void orc_act(const float* src, float* dst, int64_t n, int act);
void orc_binary(const float* a, const float* b, float* dst, int64_t n, int op, int relu);
void orc_hardsigmoid(const float* src, float* dst, int64_t n, float alpha, float beta);

// ---- sequence ops (src/Kernels/Avx2Kernels.cs:563-600, src/Kernels/Ops.Seq.cs:28-75)
void orc_layernorm(const float* x, int64_t rows, int c, const float* w, const float* b, float* dst, float eps);
void orc_softmax(const float* src, float* dst, int64_t rows, int c);

// ---- math cores used by the fused epilogues (src/Kernels/SimdMath.cs:120-170)
float orc_exp_core(float x);
float orc_erf_core(float x);
float orc_act_scalar(float v, int act);

#ifdef __cplusplus
}
#endif
