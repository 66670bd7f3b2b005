// Bandwidth-bound kernels of the fused conv path (depthwise, small-channel direct conv, ConvT dot,
// pools, SE gate, broadcast, nearest resize, concat slices, elementwise, conversion, LayerNorm,
// softmax, attention). fp16 NHWC storage, fp32 math, 128-bit (8 x fp16) accesses along channels.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "sdx_device.cuh"
#include "sdx_internal.h"

namespace sdx {

static inline bool aligned8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; }

static inline int grid_for(int64_t n, int block) {
  int64_t g = (n + block - 1) / block;
  return (int)std::min<int64_t>(g, (int64_t)1 << 30);
}

#define SDX_LAUNCH_CHECK(what)                                  \
  do {                                                          \
    cudaError_t e_ = cudaGetLastError();                        \
    if (e_ != cudaSuccess) return set_cuda_error(e_, what);     \
    count_launch();                                             \
  } while (0)

__device__ __forceinline__ void h8_to_f(const uint4& u, float* f) {
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; i++) {
    float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 f_to_h8(const float* f) {
  uint4 u;
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; i++) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
  return u;
}

// ------------------------------------------------------------------ depthwise
// Nhwc.Depthwise (src/Kernels/Nhwc.cs:496-631): y[c] = act(b[c] + sum_tap w[tap,c] * x[tap,c] [+ add]);
// out-of-range taps read the constant 0 pad. Thread = one output pixel x 8 channels.
template <int ACT>
__global__ void depthwise_kernel(DwArgs a) {
  const int cg = a.c >> 3;
  const int64_t total = (int64_t)a.batch * a.oh * a.ow * cg;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int g = (int)(idx % cg);
    int64_t p = idx / cg;
    const int ox = (int)(p % a.ow);
    p /= a.ow;
    const int oy = (int)(p % a.oh);
    const int n = (int)(p / a.oh);
    const int c0 = g * 8;
    float acc[8];
    {
      const float4* bp = reinterpret_cast<const float4*>(a.bias + c0);
      float4 b0 = __ldg(bp), b1 = __ldg(bp + 1);
      acc[0] = b0.x; acc[1] = b0.y; acc[2] = b0.z; acc[3] = b0.w;
      acc[4] = b1.x; acc[5] = b1.y; acc[6] = b1.z; acc[7] = b1.w;
    }
    float sc[8];
    if (a.in_scale) {
      const float4* sp = reinterpret_cast<const float4*>(a.in_scale + (int64_t)n * a.c + c0);
      float4 s0 = __ldg(sp), s1 = __ldg(sp + 1);
      sc[0] = s0.x; sc[1] = s0.y; sc[2] = s0.z; sc[3] = s0.w;
      sc[4] = s1.x; sc[5] = s1.y; sc[6] = s1.z; sc[7] = s1.w;
    }
    const __half* xb = a.x + (int64_t)n * a.ih * a.iw * a.c + c0;
    for (int ky = 0; ky < a.kh; ky++) {
      const int iy = oy * a.sh + ky - a.pt;
      if ((unsigned)iy >= (unsigned)a.ih) continue;
      for (int kx = 0; kx < a.kw; kx++) {
        const int ix = ox * a.sw + kx - a.pl;
        if ((unsigned)ix >= (unsigned)a.iw) continue;
        float xv[8];
        h8_to_f(__ldg(reinterpret_cast<const uint4*>(xb + ((int64_t)iy * a.iw + ix) * a.c)), xv);
        const float4* wp = reinterpret_cast<const float4*>(a.w + (int64_t)(ky * a.kw + kx) * a.c + c0);
        float4 w0 = __ldg(wp), w1 = __ldg(wp + 1);
        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        if (a.in_scale) {
#pragma unroll
          for (int j = 0; j < 8; j++) acc[j] = fmaf(xv[j] * sc[j], wv[j], acc[j]);
        } else {
#pragma unroll
          for (int j = 0; j < 8; j++) acc[j] = fmaf(xv[j], wv[j], acc[j]);
        }
      }
    }
    const int64_t o = (((int64_t)n * a.oh + oy) * a.ow + ox) * a.c + c0;
    if (a.add) {
      float r[8];
      h8_to_f(__ldg(reinterpret_cast<const uint4*>(a.add + o)), r);
#pragma unroll
      for (int j = 0; j < 8; j++) acc[j] += r[j];
    }
#pragma unroll
    for (int j = 0; j < 8; j++) acc[j] = act_t<ACT>(acc[j]);
    *reinterpret_cast<uint4*>(a.y + o) = f_to_h8(acc);
  }
}

int depthwise_launch(const DwArgs& a, cudaStream_t st) {
  if (a.c % 8 != 0) return set_error(SDX_ERR_NOT_SUPPORTED, "depthwise: channels must be a multiple of 8");
  const int64_t total = (int64_t)a.batch * a.oh * a.ow * (a.c / 8);
  if (total == 0) return SDX_OK;
  if (depthwise_tiled_launch(a, st)) {
    SDX_LAUNCH_CHECK("depthwise_tiled");
    return SDX_OK;
  }
  SDX_ACT_DISPATCH(a.act, ACTC, depthwise_kernel<ACTC><<<grid_for(total, 256), 256, 0, st>>>(a));
  SDX_LAUNCH_CHECK("depthwise");
  return SDX_OK;
}

// ------------------------------------------------------------------ direct small-channel conv
// Stem convs (ic < 8, fp32 NCHW graph input, stride 2) and other convs the tensor-core path does
// not take: thread = one output pixel x 8 output channels; weights [tap][ic][oc] staged in smem.
__device__ __forceinline__ float load_x(const DirectArgs& a, int n, int c, int iy, int ix) {
  int64_t off = a.x_nchw ? (((int64_t)n * a.ic + c) * a.ih + iy) * a.iw + ix
                         : (((int64_t)n * a.ih + iy) * a.iw + ix) * a.ic + c;
  return a.x_f32 ? __ldg(static_cast<const float*>(a.x) + off) : __half2float(static_cast<const __half*>(a.x)[off]);
}

template <int ACT>
__global__ void direct_conv_kernel(DirectArgs a) {
  extern __shared__ float sw[];
  const int wn = a.kh * a.kw * a.ic * a.oc;
  for (int i = threadIdx.x; i < wn; i += blockDim.x) sw[i] = a.w[i];
  __syncthreads();
  const int og = (a.oc + 7) / 8;
  const int64_t total = (int64_t)a.batch * a.oh * a.ow * og;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    // pixel-fastest order: neighbouring threads read neighbouring input columns
    int64_t p = idx;
    const int ox = (int)(p % a.ow);
    p /= a.ow;
    const int oy = (int)(p % a.oh);
    p /= a.oh;
    const int n = (int)(p % a.batch);
    const int g = (int)(p / a.batch);
    const int o0 = g * 8;
    const int no = min(8, a.oc - o0);
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; j++) acc[j] = (j < no && a.bias) ? a.bias[o0 + j] : 0.0f;
    for (int ky = 0; ky < a.kh; ky++) {
      const int iy = oy * a.sh + ky - a.pt;
      if ((unsigned)iy >= (unsigned)a.ih) continue;
      for (int kx = 0; kx < a.kw; kx++) {
        const int ix = ox * a.sw + kx - a.pl;
        if ((unsigned)ix >= (unsigned)a.iw) continue;
        const float* wt = sw + ((ky * a.kw + kx) * a.ic) * a.oc + o0;
        for (int c = 0; c < a.ic; c++) {
          const float xv = load_x(a, n, c, iy, ix);
          const float* wc = wt + c * a.oc;
#pragma unroll
          for (int j = 0; j < 8; j++)
            if (j < no) acc[j] = fmaf(xv, wc[j], acc[j]);
        }
      }
    }
    for (int j = 0; j < no; j++) {
      const int o = o0 + j;
      float v = acc[j];
      if (a.add) {
        int64_t ao = a.add_nchw ? (((int64_t)n * a.oc + o) * a.oh + oy) * a.ow + ox
                                : (((int64_t)n * a.oh + oy) * a.ow + ox) * a.oc + o;
        v += a.add_f32 ? static_cast<const float*>(a.add)[ao] : __half2float(static_cast<const __half*>(a.add)[ao]);
      }
      v = act_t<ACT>(v);
      int64_t yo = a.y_nchw ? (((int64_t)n * a.oc + o) * a.oh + oy) * a.ow + ox
                            : (((int64_t)n * a.oh + oy) * a.ow + ox) * a.y_pix_stride + a.y_ch_off + o;
      if (a.y_f32) static_cast<float*>(a.y)[yo] = v;
      else static_cast<__half*>(a.y)[yo] = __float2half_rn(v);
    }
  }
}

// Conv + fused 2x2 stride-2 max pool (Nhwc.ConvPool / PoolBand, src/Kernels/Nhwc.cs:666-727; the
// GPU plans fuse it for small stems, src/Engine/GraphCompiler.cs:883-904): thread = one pooled pixel
// x 8 output channels; it computes the four conv outputs of its 2x2 window (each bias-initialised,
// taps then input channels ascending, one FMA per term, activation), takes their max in the
// reference's order max(max(max(s0, s1), s2), s3) and applies the optional relu. The full-size
// conv output is never stored.
template <int ACT>
__global__ void conv_pool_direct_kernel(DirectArgs a) {
  extern __shared__ float sw[];
  const int wn = a.kh * a.kw * a.ic * a.oc;
  for (int i = threadIdx.x; i < wn; i += blockDim.x) sw[i] = a.w[i];
  __syncthreads();
  const int ph = a.oh / 2, pw = a.ow / 2;
  const int og = (a.oc + 7) / 8;
  const int64_t total = (int64_t)a.batch * ph * pw * og;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    int64_t p = idx;
    const int px = (int)(p % pw);
    p /= pw;
    const int py = (int)(p % ph);
    p /= ph;
    const int n = (int)(p % a.batch);
    const int g = (int)(p / a.batch);
    const int o0 = g * 8;
    const int no = min(8, a.oc - o0);
    float best[8];
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const int oy = 2 * py + (q >> 1), ox = 2 * px + (q & 1);
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; j++) acc[j] = (j < no && a.bias) ? a.bias[o0 + j] : 0.0f;
      for (int ky = 0; ky < a.kh; ky++) {
        const int iy = oy * a.sh + ky - a.pt;
        if ((unsigned)iy >= (unsigned)a.ih) continue;
        for (int kx = 0; kx < a.kw; kx++) {
          const int ix = ox * a.sw + kx - a.pl;
          if ((unsigned)ix >= (unsigned)a.iw) continue;
          const float* wt = sw + ((ky * a.kw + kx) * a.ic) * a.oc + o0;
          for (int c = 0; c < a.ic; c++) {
            const float xv = load_x(a, n, c, iy, ix);
            const float* wc = wt + c * a.oc;
#pragma unroll
            for (int j = 0; j < 8; j++)
              if (j < no) acc[j] = fmaf(xv, wc[j], acc[j]);
          }
        }
      }
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const float v = act_t<ACT>(acc[j]);
        best[j] = q == 0 ? v : fmaxf(best[j], v);
      }
    }
    const int64_t yo = (((int64_t)n * ph + py) * pw + px) * a.y_pix_stride + a.y_ch_off + o0;
    for (int j = 0; j < no; j++) {
      const float v = a.pool_relu ? fmaxf(best[j], 0.0f) : best[j];
      if (a.y_f32) static_cast<float*>(a.y)[yo + j] = v;
      else static_cast<__half*>(a.y)[yo + j] = __float2half_rn(v);
    }
  }
}

// 1x1 conv to at most 8 outputs over an fp16 NHWC tensor (e.g. a network's final 32 -> 3 projection
// with the fp32 input image as residual): thread = one pixel, its ic channels read as 16-byte words,
// oc accumulators (bias first, channels ascending, one FMA each), then the residual in either layout,
// the activation and oc stores. Weights [ic][oc] and bias staged in shared memory.
template <int OC>
__global__ void __launch_bounds__(256) pw_small_kernel(DirectArgs a) {
  extern __shared__ float sw[];
  for (int i = threadIdx.x; i < a.ic * OC; i += blockDim.x) sw[i] = __ldg(a.w + i);
  if (threadIdx.x < OC) sw[a.ic * OC + threadIdx.x] = a.bias ? __ldg(a.bias + threadIdx.x) : 0.0f;
  __syncthreads();
  const int64_t hw = (int64_t)a.oh * a.ow, pixels = (int64_t)a.batch * hw;
  const int c8n = a.ic >> 3;
  for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < pixels; p += (int64_t)gridDim.x * blockDim.x) {
    float acc[OC];
#pragma unroll
    for (int o = 0; o < OC; o++) acc[o] = sw[a.ic * OC + o];
    const uint4* xp = reinterpret_cast<const uint4*>(static_cast<const __half*>(a.x) + p * a.ic);
    for (int c8 = 0; c8 < c8n; c8++) {
      const uint4 u = __ldg(xp + c8);
      const __half2* h = reinterpret_cast<const __half2*>(&u);
      const float* w0 = sw + c8 * 8 * OC;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float2 f = __half22float2(h[j]);
#pragma unroll
        for (int o = 0; o < OC; o++) acc[o] = fmaf(f.x, w0[(2 * j) * OC + o], acc[o]);
#pragma unroll
        for (int o = 0; o < OC; o++) acc[o] = fmaf(f.y, w0[(2 * j + 1) * OC + o], acc[o]);
      }
    }
    const int64_t n = p / hw, r = p - n * hw;
    if (a.add) {
#pragma unroll
      for (int o = 0; o < OC; o++) {
        const int64_t ro = a.add_nchw ? (n * OC + o) * hw + r : p * OC + o;
        acc[o] += a.add_f32 ? __ldg(static_cast<const float*>(a.add) + ro)
                            : __half2float(static_cast<const __half*>(a.add)[ro]);
      }
    }
#pragma unroll
    for (int o = 0; o < OC; o++) {
      const float v = act_apply(acc[o], a.act);
      const int64_t yo = a.y_nchw ? (n * OC + o) * hw + r : p * a.y_pix_stride + a.y_ch_off + o;
      if (a.y_f32) static_cast<float*>(a.y)[yo] = v;
      else static_cast<__half*>(a.y)[yo] = __float2half_rn(v);
    }
  }
}

static bool pw_small_ok(const DirectArgs& a) {
  return a.kh == 1 && a.kw == 1 && a.sh == 1 && a.sw == 1 && a.pt == 0 && a.pl == 0 && !a.pool && !a.x_f32 &&
         !a.x_nchw && a.ic % 8 == 0 && a.oc >= 1 && a.oc <= 8 && a.ih == a.oh && a.iw == a.ow &&
         (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 && (size_t)(a.ic + 1) * a.oc * sizeof(float) <= 48 * 1024;
}

template <int OC>
static void pw_small_run(const DirectArgs& a, int64_t pixels, cudaStream_t st) {
  pw_small_kernel<OC><<<grid_for(pixels, 256), 256, sizeof(float) * (size_t)(a.ic + 1) * OC, st>>>(a);
}

int direct_conv_launch(const DirectArgs& a, cudaStream_t st) {
  if (pw_small_ok(a)) {
    const int64_t pixels = (int64_t)a.batch * a.oh * a.ow;
    if (pixels == 0) return SDX_OK;
    switch (a.oc) {
      case 1: pw_small_run<1>(a, pixels, st); break;
      case 2: pw_small_run<2>(a, pixels, st); break;
      case 3: pw_small_run<3>(a, pixels, st); break;
      case 4: pw_small_run<4>(a, pixels, st); break;
      case 5: pw_small_run<5>(a, pixels, st); break;
      case 6: pw_small_run<6>(a, pixels, st); break;
      case 7: pw_small_run<7>(a, pixels, st); break;
      default: pw_small_run<8>(a, pixels, st); break;
    }
    SDX_LAUNCH_CHECK("pw_small");
    return SDX_OK;
  }
  const size_t wbytes = sizeof(float) * a.kh * a.kw * a.ic * a.oc;
  if (wbytes > 96 * 1024) return set_error(SDX_ERR_NOT_SUPPORTED, "direct conv: weights exceed the smem stage");
  if (a.pool) {
    if (a.add || a.y_nchw) return set_error(SDX_ERR_NOT_SUPPORTED, "conv + pool: no residual, NHWC output");
    const int64_t ptotal = (int64_t)a.batch * (a.oh / 2) * (a.ow / 2) * ((a.oc + 7) / 8);
    if (ptotal == 0) return SDX_OK;
    SDX_ACT_DISPATCH(a.act, ACTC, {
      static SmemAttr attr{};
      const int rc = raise_smem_limit(attr, (const void*)conv_pool_direct_kernel<ACTC>, 96 * 1024,
                                      "cudaFuncSetAttribute(conv_pool_direct)");
      if (rc) return rc;
      conv_pool_direct_kernel<ACTC><<<grid_for(ptotal, 256), 256, wbytes, st>>>(a);
    });
    SDX_LAUNCH_CHECK("conv_pool_direct");
    return SDX_OK;
  }
  const int64_t total = (int64_t)a.batch * a.oh * a.ow * ((a.oc + 7) / 8);
  if (total == 0) return SDX_OK;
  if (stem_tiled_launch(a, st)) {
    SDX_LAUNCH_CHECK("stem_tiled");
    return SDX_OK;
  }
  SDX_ACT_DISPATCH(a.act, ACTC, {
    static SmemAttr attr{};
    const int rc = raise_smem_limit(attr, (const void*)direct_conv_kernel<ACTC>, 96 * 1024,
                                    "cudaFuncSetAttribute(direct_conv)");
    if (rc) return rc;
    direct_conv_kernel<ACTC><<<grid_for(total, 256), 256, wbytes, st>>>(a);
  });
  SDX_LAUNCH_CHECK("direct_conv");
  return SDX_OK;
}

// ------------------------------------------------------------------ ConvT, oc < 8 (dot path)
// ConvTDot (src/Kernels/Nhwc.Det.cs:96-131): per output element one dot product over ic + bias, act.
// Fast form (kh*kw*oc in {4, 8, 12, 16}): blocks walk input rows; a thread reads its input pixel once, in
// 8-channel pieces, and keeps all kh*kw*oc sums in registers; weights [tap][o][ic] in shared memory
// (staged once per block).
// TO = kh*kw*oc is a template constant: the per-output loops then hold exactly TO accumulators
// (predicated-off copies of a wider unrolled loop would still issue).
template <int ACT, int TO>
__global__ void convt_dot_rows_kernel(ConvtDotArgs a) {
  extern __shared__ float sw[];
  const int taps = a.kh * a.kw;
  constexpr int to = TO;
  const int nw = to * a.ic;
  for (int i = threadIdx.x; i < nw; i += blockDim.x) {
    const int c = i % a.ic, k = i / a.ic;
    const int o = k % a.oc, tap = k / a.oc;
    sw[i] = a.w[((int64_t)c * a.oc + o) * taps + tap];
  }
  float* sb = sw + nw;
  for (int i = threadIdx.x; i < a.oc; i += blockDim.x) sb[i] = a.bias ? a.bias[i] : 0.0f;
  __syncthreads();
  const int ow = a.iw * a.kw, oh = a.ih * a.kh;
  const int per_row = (a.iw + blockDim.x - 1) / blockDim.x;  // jobs (row pieces) per input row
  const int jobs = a.batch * a.ih * per_row;
  for (int job = blockIdx.x; job < jobs; job += gridDim.x) {
    const int row = job / per_row;  // n * ih + y
    const int x = (job - row * per_row) * blockDim.x + threadIdx.x;
    if (x >= a.iw) continue;
    const int n = row / a.ih, y = row - n * a.ih;
    const __half* xp = a.x + ((int64_t)row * a.iw + x) * a.ic;
    float acc[TO];
#pragma unroll
    for (int k = 0; k < TO; k++) acc[k] = sb[k % a.oc];
    for (int c = 0; c < a.ic; c += 8) {
      float xv[8];
      h8_to_f(__ldg(reinterpret_cast<const uint4*>(xp + c)), xv);
#pragma unroll
      for (int k = 0; k < TO; k++) {
        const float4* wk = reinterpret_cast<const float4*>(sw + k * a.ic + c);
        const float4 w0 = wk[0], w1 = wk[1];
        float s = acc[k];
        s = fmaf(xv[0], w0.x, s); s = fmaf(xv[1], w0.y, s); s = fmaf(xv[2], w0.z, s); s = fmaf(xv[3], w0.w, s);
        s = fmaf(xv[4], w1.x, s); s = fmaf(xv[5], w1.y, s); s = fmaf(xv[6], w1.z, s); s = fmaf(xv[7], w1.w, s);
        acc[k] = s;
      }
    }
    if (a.oc == 1 && a.kw == 2 && a.y_f32) {
      // one output channel, two taps per output row: adjacent floats, one 8-byte store per row
#pragma unroll
      for (int dy = 0; dy < TO / 2; dy++) {
        if (dy < a.kh) {
          const int64_t op = ((int64_t)n * oh + y * a.kh + dy) * ow + x * 2;
          *reinterpret_cast<float2*>(static_cast<float*>(a.y) + op) =
              make_float2(act_t<ACT>(acc[2 * dy]), act_t<ACT>(acc[2 * dy + 1]));
        }
      }
    } else {
#pragma unroll
      for (int k = 0; k < TO; k++) {
        {
          const int o = k % a.oc, tap = k / a.oc;
          const int dy = tap / a.kw, dx = tap - dy * a.kw;
          const int64_t op = ((int64_t)n * oh + y * a.kh + dy) * ow + x * a.kw + dx;
          const float v = act_t<ACT>(acc[k]);
          if (a.y_f32) static_cast<float*>(a.y)[op * a.oc + o] = v;
          else static_cast<__half*>(a.y)[op * a.oc + o] = __float2half_rn(v);
        }
      }
    }
  }
}

// General form (any kh*kw*oc): one thread per input pixel, weights from global memory.
template <int ACT>
__global__ void convt_dot_kernel(ConvtDotArgs a) {
  const int taps = a.kh * a.kw;
  const int64_t total = (int64_t)a.batch * a.ih * a.iw;
  const int ow = a.iw * a.kw, oh = a.ih * a.kh;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int x = (int)(idx % a.iw);
    const int64_t t = idx / a.iw;
    const int y = (int)(t % a.ih);
    const int n = (int)(t / a.ih);
    const __half* xp = a.x + idx * a.ic;
    for (int tap = 0; tap < taps; tap++) {
      const int dy = tap / a.kw, dx = tap % a.kw;
      const int64_t op = ((int64_t)n * oh + y * a.kh + dy) * ow + x * a.kw + dx;
      for (int o = 0; o < a.oc; o++) {
        float s = a.bias ? a.bias[o] : 0.0f;
        for (int c = 0; c < a.ic; c += 8) {
          float xv[8];
          h8_to_f(__ldg(reinterpret_cast<const uint4*>(xp + c)), xv);
#pragma unroll
          for (int j = 0; j < 8; j++) s = fmaf(xv[j], __ldg(a.w + ((int64_t)(c + j) * a.oc + o) * taps + tap), s);
        }
        s = act_t<ACT>(s);
        if (a.y_f32) static_cast<float*>(a.y)[op * a.oc + o] = s;
        else static_cast<__half*>(a.y)[op * a.oc + o] = __float2half_rn(s);
      }
    }
  }
}

int convt_dot_launch(const ConvtDotArgs& a, cudaStream_t st) {
  if (a.ic % 8 != 0) return set_error(SDX_ERR_NOT_SUPPORTED, "convt dot: ic must be a multiple of 8");
  const int64_t total = (int64_t)a.batch * a.ih * a.iw;
  if (total == 0) return SDX_OK;
  const int to = a.kh * a.kw * a.oc;
  const size_t wbytes = sizeof(float) * ((size_t)to * a.ic + a.oc);
  const int64_t rows = (int64_t)a.batch * a.ih;
  if ((to == 4 || to == 8 || to == 12 || to == 16) && wbytes <= 48 * 1024 && rows * a.iw <= INT32_MAX &&
      aligned8(a.y)) {
    const int block = a.iw >= 128 ? 128 : (a.iw + 31) / 32 * 32;
    const int64_t jobs = rows * ((a.iw + block - 1) / block);
    int dev = 0;
    cudaGetDevice(&dev);
    const int grid = (int)std::min<int64_t>(jobs, (int64_t)num_sms(dev) * 16);
#define SDX_CT_TO(TOV) \
  if (to == TOV) SDX_ACT_DISPATCH(a.act, ACTC, convt_dot_rows_kernel<ACTC, TOV><<<grid, block, wbytes, st>>>(a));
    SDX_CT_TO(4) SDX_CT_TO(8) SDX_CT_TO(12) SDX_CT_TO(16)
#undef SDX_CT_TO
  } else {
    SDX_ACT_DISPATCH(a.act, ACTC, convt_dot_kernel<ACTC><<<grid_for(total, 256), 256, 0, st>>>(a));
  }
  SDX_LAUNCH_CHECK("convt_dot");
  return SDX_OK;
}

// ------------------------------------------------------------------ pools
// MaxPool (src/Kernels/Nhwc.cs:730-770): max over in-range taps, 0 when none, optional relu.
// AvgPool (src/Kernels/Ops.Seq.cs:180-225): sum of in-range taps / count (or kh*kw).
__global__ void pool_kernel(PoolArgs a) {
  const int cg = a.c >> 3;
  const int64_t total = (int64_t)a.batch * a.oh * a.ow * cg;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int g = (int)(idx % cg);
    int64_t p = idx / cg;
    const int ox = (int)(p % a.ow);
    p /= a.ow;
    const int oy = (int)(p % a.oh);
    const int n = (int)(p / a.oh);
    float acc[8];
    bool any = false;
    int cnt = 0;
    for (int j = 0; j < 8; j++) acc[j] = 0.0f;
    for (int ky = 0; ky < a.kh; ky++) {
      const int iy = oy * a.sh + ky - a.pt;
      if ((unsigned)iy >= (unsigned)a.ih) continue;
      for (int kx = 0; kx < a.kw; kx++) {
        const int ix = ox * a.sw + kx - a.pl;
        if ((unsigned)ix >= (unsigned)a.iw) continue;
        float v[8];
        h8_to_f(__ldg(reinterpret_cast<const uint4*>(a.x + (((int64_t)n * a.ih + iy) * a.iw + ix) * a.x_ps + a.x_co + g * 8)), v);
        if (a.is_avg) {
#pragma unroll
          for (int j = 0; j < 8; j++) acc[j] += v[j];
        } else if (!any) {
#pragma unroll
          for (int j = 0; j < 8; j++) acc[j] = v[j];
        } else {
#pragma unroll
          for (int j = 0; j < 8; j++) acc[j] = fmaxf(acc[j], v[j]);
        }
        any = true;
        cnt++;
      }
    }
    if (a.is_avg) {
      const float inv = 1.0f / (float)(a.incl ? a.kh * a.kw : max(cnt, 1));
#pragma unroll
      for (int j = 0; j < 8; j++) acc[j] *= inv;
    } else if (a.relu) {
#pragma unroll
      for (int j = 0; j < 8; j++) acc[j] = fmaxf(acc[j], 0.0f);
    }
    *reinterpret_cast<uint4*>(a.y + (((int64_t)n * a.oh + oy) * a.ow + ox) * a.c + g * 8) = f_to_h8(acc);
  }
}

int pool_launch(const PoolArgs& a, cudaStream_t st) {
  if (a.c % 8 != 0) return set_error(SDX_ERR_NOT_SUPPORTED, "pool: channels must be a multiple of 8");
  const int64_t total = (int64_t)a.batch * a.oh * a.ow * (a.c / 8);
  if (total == 0) return SDX_OK;
  pool_kernel<<<grid_for(total, 256), 256, 0, st>>>(a);
  SDX_LAUNCH_CHECK("pool");
  return SDX_OK;
}

// ------------------------------------------------------------------ SE gate
// Stage 1: per (image, pixel chunk) channel sums into scratch; stage 2: one CTA per image reduces
// the chunks, forms the means, runs FC1 (+relu) and FC2 and the (hard) sigmoid gate
// (Nhwc.ChannelGate, src/Kernels/Nhwc.Det.cs:287-314).
// Pixel chunks per image (about 64 KB of input each, at most 64) depend on the image's size only,
// so an image's gate (and everything after it) is bit-identical whatever batch it runs in.
static int gate_chunks(int hw, int c) {
  const int64_t bytes = (int64_t)hw * c * 2;
  return (int)std::min<int64_t>(64, std::max<int64_t>(1, std::min<int64_t>(hw, (bytes + 65535) / 65536)));
}

// Chunks over the [batch][hw / 32][c] fp32 32-pixel sums a conv wrote (about 32 KB each); never
// more than gate_chunks(hw, c), so the same scratch serves both forms. Also batch-independent.
static int gate_sum_chunks(int hw, int c) {
  const int rows = hw / 32;
  const int64_t bytes = (int64_t)rows * c * 4;
  return (int)std::min<int64_t>(gate_chunks(hw, c),
                                std::max<int64_t>(1, std::min<int64_t>(rows, (bytes + 32767) / 32768)));
}

// Scratch: per-chunk channel sums [batch][chunks][c], then the hidden layer [batch][r <= c].
size_t gate_scratch_bytes(int batch, int hw, int c) {
  return sizeof(float) * (size_t)batch * (gate_chunks(hw, c) + 1) * c;
}

// eight consecutive channels of one row as fp32
__device__ __forceinline__ void ld8f(const __half* p, float (&v)[8]) { h8_to_f(__ldg(reinterpret_cast<const uint4*>(p)), v); }
__device__ __forceinline__ void ld8f(const float* p, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p)), b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// Channel sums of rows [p0, p1) of image n's `rows` x c tile: fp16 pixels, or fp32 32-pixel sums.
template <typename T>
__global__ void gap_partial_kernel(const T* __restrict__ x, int rows, int c, int chunks, float* __restrict__ partial) {
  extern __shared__ float red[];
  const int n = blockIdx.y, chunk = blockIdx.x;
  const int cg = c >> 3;
  const int lanes_p = blockDim.x / cg;  // pixel lanes (blockDim is a multiple of cg)
  const int g = threadIdx.x % cg, lp = threadIdx.x / cg;
  const int p0 = (int)((int64_t)chunk * rows / chunks), p1 = (int)((int64_t)(chunk + 1) * rows / chunks);
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (lp < lanes_p) {
    const T* base = x + (int64_t)n * rows * c + g * 8;
    int p = p0 + lp;
    // four independent row loads in flight per thread, then the remainder
    for (; p + 3 * lanes_p < p1; p += 4 * lanes_p) {
      float v[4][8];
#pragma unroll
      for (int k = 0; k < 4; k++) ld8f(base + (int64_t)(p + k * lanes_p) * c, v[k]);
#pragma unroll
      for (int k = 0; k < 4; k++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[j] += v[k][j];
    }
    for (; p < p1; p += lanes_p) {
      float v[8];
      ld8f(base + (int64_t)p * c, v);
#pragma unroll
      for (int j = 0; j < 8; j++) acc[j] += v[j];
    }
  }
  // reduce over pixel lanes through smem: red[lp][c]
  if (lp < lanes_p)
    for (int j = 0; j < 8; j++) red[lp * c + g * 8 + j] = acc[j];
  __syncthreads();
  for (int ch = threadIdx.x; ch < c; ch += blockDim.x) {
    float s = 0.0f;
    for (int l = 0; l < lanes_p; l++) s += red[l * c + ch];
    partial[((int64_t)n * chunks + chunk) * c + ch] = s;
  }
}

// FC stages, GATE_IMG images per CTA: every weight row is read once per CTA (coalesced, one warp
// per row of W1 [r][c] and of W2 [c][r]) and applied to all of the CTA's images; the rows are spread
// over a second grid dimension (GATE_RJ hidden units / GATE_CJ output channels per CTA). Each
// image's sums run in the same order whatever images share its CTA, so the gate of an image does
// not depend on the batch it runs in. The hidden layer goes through scratch (after the partials).
constexpr int GATE_IMG = 8, GATE_RJ = 8, GATE_CJ = 32;

// Warp sum of v[0..GATE_IMG-1]; lane 0 holds the totals.
__device__ __forceinline__ void warp_sum_img(float (&v)[GATE_IMG]) {
#pragma unroll
  for (int i = 0; i < GATE_IMG; i++)
#pragma unroll
    for (int off = 16; off; off >>= 1) v[i] += __shfl_xor_sync(0xffffffffu, v[i], off);
}

__global__ void gate_fc1_kernel(GateArgs a, int chunks, float* __restrict__ hid) {
  extern __shared__ float mean[];  // [GATE_IMG][c]
  const int n0 = blockIdx.x * GATE_IMG;
  const int nimg = min(GATE_IMG, a.batch - n0);
  const float inv = 1.0f / (float)a.hw;
  for (int idx = threadIdx.x; idx < GATE_IMG * a.c; idx += blockDim.x) {
    const int i = idx / a.c, ch = idx - i * a.c;
    float s = 0.0f;
    if (i < nimg)
      for (int k = 0; k < chunks; k++) s += a.partial[((int64_t)(n0 + i) * chunks + k) * a.c + ch];
    mean[idx] = s * inv;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int j1 = min(a.r, (int)(blockIdx.y + 1) * GATE_RJ);
  for (int j = blockIdx.y * GATE_RJ + warp; j < j1; j += nw) {
    float s[GATE_IMG];
#pragma unroll
    for (int i = 0; i < GATE_IMG; i++) s[i] = 0.0f;
    const float* wr = a.w1 + (int64_t)j * a.c;
    for (int k = lane; k < a.c; k += 32) {
      const float w = __ldg(wr + k);
#pragma unroll
      for (int i = 0; i < GATE_IMG; i++) s[i] = fmaf(w, mean[i * a.c + k], s[i]);
    }
    warp_sum_img(s);
    if (lane == 0) {
      const float b = a.b1 ? a.b1[j] : 0.0f;
#pragma unroll
      for (int i = 0; i < GATE_IMG; i++) {
        const float h = s[i] + b;
        if (i < nimg) hid[(int64_t)(n0 + i) * a.r + j] = a.act1_relu ? fmaxf(h, 0.0f) : h;
      }
    }
  }
}

__global__ void gate_fc2_kernel(GateArgs a, const float* __restrict__ hid) {
  extern __shared__ float hs[];  // [GATE_IMG][r]
  const int n0 = blockIdx.x * GATE_IMG;
  const int nimg = min(GATE_IMG, a.batch - n0);
  for (int idx = threadIdx.x; idx < GATE_IMG * a.r; idx += blockDim.x) {
    const int i = idx / a.r;
    hs[idx] = i < nimg ? hid[(int64_t)n0 * a.r + idx] : 0.0f;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int c1 = min(a.c, (int)(blockIdx.y + 1) * GATE_CJ);
  for (int ch = blockIdx.y * GATE_CJ + warp; ch < c1; ch += nw) {
    float z[GATE_IMG];
#pragma unroll
    for (int i = 0; i < GATE_IMG; i++) z[i] = 0.0f;
    const float* wr = a.w2 + (int64_t)ch * a.r;
    for (int j = lane; j < a.r; j += 32) {
      const float w = __ldg(wr + j);
#pragma unroll
      for (int i = 0; i < GATE_IMG; i++) z[i] = fmaf(w, hs[i * a.r + j], z[i]);
    }
    warp_sum_img(z);
    if (lane == 0) {
      const float b = a.b2 ? a.b2[ch] : 0.0f;
#pragma unroll
      for (int i = 0; i < GATE_IMG; i++) {
        const float zz = z[i] + b;
        const float g = a.hard ? __saturatef(zz * a.alpha + a.beta) : 1.0f / (1.0f + expf(-zz));
        if (i < nimg) a.s[(int64_t)(n0 + i) * a.c + ch] = g + a.offset;
      }
    }
  }
}

// Whole gate of one image in one CTA, from the producing conv's 32-pixel sums: column sums of the
// image's hw / 32 rows (fixed lane and row order, so batch-independent), the mean, FC1 (+relu) and
// FC2 with the gate, one warp per output row of each FC. smem: [lanes][c] reduction, mean[c], hid[r].
__global__ void __launch_bounds__(256) gate_sums_kernel(GateArgs a) {
  extern __shared__ float gsm[];
  const int n = blockIdx.x, c = a.c, rows = a.hw >> 5;
  const int cg = c >> 3, lanes_p = blockDim.x / cg;
  float* red = gsm;                      // [lanes_p][c]
  float* mean = red + lanes_p * c;       // [c]
  float* hid = mean + c;                 // [r]
  const int g = threadIdx.x % cg, lp = threadIdx.x / cg;
  if (lp < lanes_p) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const float* base = a.sums + (int64_t)n * rows * c + g * 8;
    int p = lp;
    for (; p + 3 * lanes_p < rows; p += 4 * lanes_p) {
      float v[4][8];
#pragma unroll
      for (int k = 0; k < 4; k++) ld8f(base + (int64_t)(p + k * lanes_p) * c, v[k]);
#pragma unroll
      for (int k = 0; k < 4; k++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[j] += v[k][j];
    }
    for (; p < rows; p += lanes_p) {
      float v[8];
      ld8f(base + (int64_t)p * c, v);
#pragma unroll
      for (int j = 0; j < 8; j++) acc[j] += v[j];
    }
#pragma unroll
    for (int j = 0; j < 8; j++) red[lp * c + g * 8 + j] = acc[j];
  }
  __syncthreads();
  const float inv = 1.0f / (float)a.hw;
  for (int ch = threadIdx.x; ch < c; ch += blockDim.x) {
    float sum = 0.0f;
    for (int l = 0; l < lanes_p; l++) sum += red[l * c + ch];
    mean[ch] = sum * inv;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  // FC1, four hidden units per warp pass (their weight rows' loads in flight together)
  for (int j0 = warp * 4; j0 < a.r; j0 += nw * 4) {
    float sum[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 2
    for (int k = lane; k < c; k += 32) {
      const float m = mean[k];
#pragma unroll
      for (int u = 0; u < 4; u++)
        if (j0 + u < a.r) sum[u] = fmaf(__ldg(a.w1 + (int64_t)(j0 + u) * c + k), m, sum[u]);
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
#pragma unroll
      for (int off = 16; off; off >>= 1) sum[u] += __shfl_xor_sync(0xffffffffu, sum[u], off);
      if (lane == 0 && j0 + u < a.r) {
        const float h = sum[u] + (a.b1 ? a.b1[j0 + u] : 0.0f);
        hid[j0 + u] = a.act1_relu ? fmaxf(h, 0.0f) : h;
      }
    }
  }
  __syncthreads();
  // FC2 and the gate, four channels per warp pass
  for (int c0 = warp * 4; c0 < c; c0 += nw * 4) {
    float z[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 2
    for (int j = lane; j < a.r; j += 32) {
      const float h = hid[j];
#pragma unroll
      for (int u = 0; u < 4; u++)
        if (c0 + u < c) z[u] = fmaf(__ldg(a.w2 + (int64_t)(c0 + u) * a.r + j), h, z[u]);
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
#pragma unroll
      for (int off = 16; off; off >>= 1) z[u] += __shfl_xor_sync(0xffffffffu, z[u], off);
      if (lane == 0 && c0 + u < c) {
        const float zz = z[u] + (a.b2 ? a.b2[c0 + u] : 0.0f);
        const float gv = a.hard ? __saturatef(zz * a.alpha + a.beta) : 1.0f / (1.0f + expf(-zz));
        a.s[(int64_t)n * c + c0 + u] = gv + a.offset;
      }
    }
  }
}

int gate_launch(const GateArgs& a, cudaStream_t st) {
  if (a.c % 8 != 0 || a.c > 4096) return set_error(SDX_ERR_NOT_SUPPORTED, "channel gate: c must be a multiple of 8, <= 4096");
  if (a.r < 1 || a.r > a.c) return set_error(SDX_ERR_NOT_SUPPORTED, "channel gate: hidden width must be in 1..c");
  if (!a.partial) return set_error(SDX_ERR_INVALID, "channel gate: scratch buffer missing");
  if (a.sums && a.hw % 32 != 0) return set_error(SDX_ERR_NOT_SUPPORTED, "channel gate: 32-pixel sums need hw % 32 == 0");
  if (a.sums && (reinterpret_cast<uintptr_t>(a.sums) & 15))
    return set_error(SDX_ERR_INVALID, "channel gate: sums must be 16-byte aligned");
  if (a.sums && a.c <= 2048) {
    // one CTA per image: the 32-pixel sums are small enough to reduce where the FCs run
    const int lanes = 256 / (a.c / 8);
    const size_t smem = sizeof(float) * ((size_t)std::max(1, lanes) * a.c + a.c + a.r);
    if (lanes >= 1 && smem <= 48 * 1024) {
      if (a.batch > 0) gate_sums_kernel<<<a.batch, 256, smem, st>>>(a);
      SDX_LAUNCH_CHECK("gate_sums");
      return SDX_OK;
    }
  }
  const int chunks = a.sums ? gate_sum_chunks(a.hw, a.c) : gate_chunks(a.hw, a.c);
  const int cg = a.c / 8;
  int block = std::max(cg, std::min(256, (256 / cg) * cg));
  if (block > 1024) return set_error(SDX_ERR_NOT_SUPPORTED, "channel gate: too many channels");
  const int lanes_p = block / cg;
  const size_t red = sizeof(float) * lanes_p * a.c;
  if (red > 48 * 1024) return set_error(SDX_ERR_NOT_SUPPORTED, "channel gate: reduction stage too large");
  const size_t fc1_smem = sizeof(float) * GATE_IMG * a.c, fc2_smem = sizeof(float) * GATE_IMG * a.r;
  if (fc1_smem > 160 * 1024) return set_error(SDX_ERR_NOT_SUPPORTED, "channel gate: too many channels for the FC stage");
  static SmemAttr attr1{}, attr2{};
  int rc = raise_smem_limit(attr1, (const void*)gate_fc1_kernel, 160 * 1024, "cudaFuncSetAttribute(gate_fc1)");
  if (rc == SDX_OK)
    rc = raise_smem_limit(attr2, (const void*)gate_fc2_kernel, 160 * 1024, "cudaFuncSetAttribute(gate_fc2)");
  if (rc) return rc;
  float* hid = a.partial + (size_t)a.batch * chunks * a.c;  // [batch][r], r <= c
  if (a.sums) gap_partial_kernel<float><<<dim3(chunks, a.batch), block, red, st>>>(a.sums, a.hw / 32, a.c, chunks, a.partial);
  else gap_partial_kernel<__half><<<dim3(chunks, a.batch), block, red, st>>>(a.x, a.hw, a.c, chunks, a.partial);
  SDX_LAUNCH_CHECK("gap_partial");
  const int gx = (a.batch + GATE_IMG - 1) / GATE_IMG;
  gate_fc1_kernel<<<dim3(gx, (a.r + GATE_RJ - 1) / GATE_RJ), 256, fc1_smem, st>>>(a, chunks, hid);
  SDX_LAUNCH_CHECK("gate_fc1");
  gate_fc2_kernel<<<dim3(gx, (a.c + GATE_CJ - 1) / GATE_CJ), 256, fc2_smem, st>>>(a, hid);
  SDX_LAUNCH_CHECK("gate_fc2");
  return SDX_OK;
}

// ------------------------------------------------------------------ channel broadcast
__device__ __forceinline__ float ew_op(float a, float b, int op) {
  switch (op) {
    case 0: return a + b;
    case 1: return a - b;
    case 2: return a * b;
    default: return a / b;
  }
}

__global__ void broadcast_kernel(int batch, int64_t pixels, int c, int op, int relu, const __half* __restrict__ x,
                                 const float* __restrict__ v, __half* __restrict__ y) {
  // grid: (chunk blocks of one image, images); chunk index inside an image is 32-bit
  const int cg = c >> 3;
  const int n = blockIdx.y;
  const int per_img = (int)(pixels * cg);
  const uint4* xi = reinterpret_cast<const uint4*>(x) + (int64_t)n * per_img;
  uint4* yi = reinterpret_cast<uint4*>(y) + (int64_t)n * per_img;
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < per_img; idx += gridDim.x * blockDim.x) {
    const int g = idx % cg;
    float xv[8];
    h8_to_f(__ldg(xi + idx), xv);
    const float4* vp = reinterpret_cast<const float4*>(v + (int64_t)n * c + g * 8);
    float4 v0 = __ldg(vp), v1 = __ldg(vp + 1);
    const float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
    for (int j = 0; j < 8; j++) {
      float s = ew_op(xv[j], vv[j], op);
      xv[j] = relu ? fmaxf(s, 0.0f) : s;
    }
    yi[idx] = f_to_h8(xv);
  }
}

int broadcast_launch(int batch, int64_t pixels, int c, int op, int relu, const __half* x, const float* v, __half* y,
                     cudaStream_t st) {
  if (c % 8 != 0) return set_error(SDX_ERR_NOT_SUPPORTED, "broadcast: channels must be a multiple of 8");
  const int64_t per_img = pixels * (c / 8);
  if (per_img == 0 || batch == 0) return SDX_OK;
  if (per_img > INT32_MAX / 2 || batch > 65535) return set_error(SDX_ERR_NOT_SUPPORTED, "broadcast: too large");
  const int bx = (int)std::min<int64_t>((per_img + 255) / 256, 4096);
  broadcast_kernel<<<dim3(bx, batch), 256, 0, st>>>(batch, pixels, c, op, relu, x, v, y);
  SDX_LAUNCH_CHECK("broadcast");
  return SDX_OK;
}

// ------------------------------------------------------------------ image -> tensor
// Image-session preprocessing (img2nhwc.comp of the reference's Vulkan image session,
// src/Backends/Vulkan/Shaders/img2nhwc.comp:4-37): interleaved u8 pixels (3 or 4 bytes, optional
// R/B swap) mapped through a per-channel table lut[c][byte], replicate padding around an image
// placed at (pt, pl) in the tensor; here written as fp32 NCHW planes (the graph input of the det
// and UNet plans) or fp16 NHWC. One block per output row; the table sits in shared memory.
__global__ void image_kernel(ImageArgs a) {
  __shared__ float lut[3 * 256];
  for (int i = threadIdx.x; i < 3 * 256; i += blockDim.x) lut[i] = __ldg(a.lut + i);
  __syncthreads();
  const int row = blockIdx.x;  // n * oh + oy
  const int n = row / a.oh, oy = row - n * a.oh;
  const int sy = min(max(oy - a.pt, 0), a.ih - 1);
  const uint8_t* srow = a.src + (int64_t)n * a.img_bytes + (int64_t)sy * a.stride;
  const int ob = a.swap ? 2 : 0;
  for (int ox = threadIdx.x; ox < a.ow; ox += blockDim.x) {
    const int sx = min(max(ox - a.pl, 0), a.iw - 1);
    const uint8_t* px = srow + (int64_t)sx * a.bpp;
    const float v0 = lut[px[ob]], v1 = lut[256 + px[1]], v2 = lut[512 + px[2 - ob]];
    if (a.y_nhwc_f16) {
      __half* y = static_cast<__half*>(a.y) + ((int64_t)row * a.ow + ox) * 3;
      y[0] = __float2half_rn(v0);
      y[1] = __float2half_rn(v1);
      y[2] = __float2half_rn(v2);
    } else {
      float* y = static_cast<float*>(a.y);
      const int64_t plane = (int64_t)a.oh * a.ow, o = (int64_t)n * 3 * plane + (int64_t)oy * a.ow + ox;
      y[o] = v0;
      y[o + plane] = v1;
      y[o + 2 * plane] = v2;
    }
  }
}

int image_launch(const ImageArgs& a, cudaStream_t st) {
  if (a.bpp != 3 && a.bpp != 4) return set_error(SDX_ERR_INVALID, "image: 3 or 4 bytes per pixel");
  if (a.ih <= 0 || a.iw <= 0 || a.oh <= 0 || a.ow <= 0 || a.batch <= 0) return set_error(SDX_ERR_INVALID, "image: empty");
  if (a.stride < (int64_t)a.iw * a.bpp || a.img_bytes < a.stride * a.ih) return set_error(SDX_ERR_INVALID, "image: stride");
  if (!a.src || !a.lut || !a.y) return set_error(SDX_ERR_INVALID, "image: null pointer");
  const int64_t rows = (int64_t)a.batch * a.oh;
  if (rows > INT32_MAX) return set_error(SDX_ERR_NOT_SUPPORTED, "image: too large");
  image_kernel<<<(unsigned)rows, 256, 0, st>>>(a);
  SDX_LAUNCH_CHECK("image");
  return SDX_OK;
}

// ------------------------------------------------------------------ nearest resize (+ addend)
// One block per output row (n, oy); threads walk the row's 16-byte chunks, so the index math is
// 32-bit and per row. src = floor(dst / scale) (src/Kernels/Nhwc.Det.cs:173, :180).
__global__ void resize_kernel(ResizeArgs a) {
  const int cg = a.c >> 3;
  const int row = blockIdx.x;  // n * oh + oy
  const int n = row / a.oh, oy = row - n * a.oh;
  const int fy = a.oh / a.ih, fx = a.ow / a.iw;
  const int iy = min(oy / fy, a.ih - 1);
  const __half* xrow = a.x + ((int64_t)n * a.ih + iy) * a.iw * a.c;
  const int64_t op0 = (int64_t)row * a.ow;
  const int total = a.ow * cg;
  for (int t = threadIdx.x; t < total; t += blockDim.x) {
    const int ox = t / cg, g = t - ox * cg;
    const int ix = min(ox / fx, a.iw - 1);
    uint4 u = __ldg(reinterpret_cast<const uint4*>(xrow + (int64_t)ix * a.c + g * 8));
    const int64_t op = op0 + ox;
    if (a.add) {
      float v[8], r[8];
      h8_to_f(u, v);
      h8_to_f(__ldg(reinterpret_cast<const uint4*>(a.add + op * a.c + g * 8)), r);
#pragma unroll
      for (int j = 0; j < 8; j++) v[j] += a.add_relu ? fmaxf(r[j], 0.0f) : r[j];
      u = f_to_h8(v);
    }
    *reinterpret_cast<uint4*>(a.y + op * a.y_pix_stride + a.y_ch_off + g * 8) = u;
  }
}

int resize_launch(const ResizeArgs& a, cudaStream_t st) {
  if (a.c % 8 || a.y_pix_stride % 8 || a.y_ch_off % 8)
    return set_error(SDX_ERR_NOT_SUPPORTED, "resize: channels / slice must be multiples of 8");
  if (a.ih <= 0 || a.iw <= 0 || a.oh % a.ih || a.ow % a.iw)
    return set_error(SDX_ERR_NOT_SUPPORTED, "resize: integer scales only");
  const int64_t rows = (int64_t)a.batch * a.oh;
  if (rows == 0 || a.ow == 0 || a.c == 0) return SDX_OK;
  if (rows > INT32_MAX || (int64_t)a.ow * (a.c / 8) > INT32_MAX) return set_error(SDX_ERR_NOT_SUPPORTED, "resize: too large");
  resize_kernel<<<(unsigned)rows, 256, 0, st>>>(a);
  SDX_LAUNCH_CHECK("resize_nearest");
  return SDX_OK;
}

// Channel concat of nearest-upsampled inputs (a Concat whose inputs are ResizeNearest outputs or
// full-size tensors, fused): every output pixel is written whole, in 16-byte chunks, so no
// partial-sector writes reach HBM. Input i has spatial size (oh / s_i, ow / s_i).
// One block per output row (n, oy); thread (g, r) copies 16-byte channel group g of the pixels
// ox = r, r + blockDim.y, ...: the source tensor, its scale and its row (n, oy / s) are fixed per
// thread, so the loop is one shift (or division), one load and one store per 16 bytes (unrolled
// by four so that four loads are in flight).
__global__ void concat_nearest_kernel(ConcatNearestArgs a) {
  const int row = blockIdx.x;  // n * oh + oy
  const int n = row / a.oh, oy = row - n * a.oh;
  const int g = threadIdx.x, ch = g * 8;
  int i = 0;
#pragma unroll
  for (int k = 1; k < 8; k++)
    if (k < a.nin && ch >= a.off[k]) i = k;
  const int sc = a.s[i], ci = a.c[i];
  const int ih = a.oh / sc, iw = a.ow / sc;
  const int lg = (sc & (sc - 1)) == 0 ? __ffs(sc) - 1 : -1;  // log2 of a power-of-two scale
  const __half* src = a.x[i] + ((int64_t)n * ih + oy / sc) * iw * ci + (ch - a.off[i]);
  __half* dst = a.y + (int64_t)row * a.ow * a.ctot + ch;
  auto sxo = [&](int ox) { return (int64_t)(lg >= 0 ? ox >> lg : ox / sc) * ci; };
  const int by = blockDim.y;
  int ox = threadIdx.y;
  // four loads in flight per thread before their stores
  for (; ox + 3 * by < a.ow; ox += 4 * by) {
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; u++) v[u] = __ldg(reinterpret_cast<const uint4*>(src + sxo(ox + u * by)));
#pragma unroll
    for (int u = 0; u < 4; u++) *reinterpret_cast<uint4*>(dst + (int64_t)(ox + u * by) * a.ctot) = v[u];
  }
  for (; ox < a.ow; ox += by)
    *reinterpret_cast<uint4*>(dst + (int64_t)ox * a.ctot) = __ldg(reinterpret_cast<const uint4*>(src + sxo(ox)));
}

int concat_nearest_launch(const ConcatNearestArgs& a, cudaStream_t st) {
  if (a.nin <= 0 || a.nin > 8) return set_error(SDX_ERR_INVALID, "concat nearest: 1..8 inputs");
  if (a.oh <= 0 || a.ow <= 0 || a.batch < 0) return set_error(SDX_ERR_INVALID, "concat nearest: bad output size");
  for (int i = 0; i < a.nin; i++) {
    if (a.c[i] <= 0 || a.c[i] % 8) return set_error(SDX_ERR_NOT_SUPPORTED, "concat nearest: channels must be multiples of 8");
    if (a.s[i] <= 0 || a.oh % a.s[i] || a.ow % a.s[i])
      return set_error(SDX_ERR_NOT_SUPPORTED, "concat nearest: integer scales that divide the output size only");
    if (!a.x[i]) return set_error(SDX_ERR_INVALID, "concat nearest: null input");
  }
  const int64_t rows = (int64_t)a.batch * a.oh;
  if (rows == 0) return SDX_OK;
  const int cg = a.ctot / 8;
  if (rows > INT32_MAX || cg > 256 || a.ctot % 8) return set_error(SDX_ERR_NOT_SUPPORTED, "concat nearest: too large");
  const dim3 block((unsigned)cg, (unsigned)std::max(1, 256 / cg));
  concat_nearest_kernel<<<(unsigned)rows, block, 0, st>>>(a);
  SDX_LAUNCH_CHECK("concat_nearest");
  return SDX_OK;
}

__global__ void slice_copy_kernel(int64_t pixels, int c, const __half* __restrict__ x, int64_t ys, int yo,
                                  __half* __restrict__ y) {
  const int cg = c >> 3;
  const int64_t total = pixels * cg;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int g = (int)(idx % cg);
    const int64_t p = idx / cg;
    *reinterpret_cast<uint4*>(y + p * ys + yo + g * 8) = __ldg(reinterpret_cast<const uint4*>(x) + idx);
  }
}

int slice_copy_launch(int64_t pixels, int c, const __half* x, int64_t y_pix_stride, int y_ch_off, __half* y,
                      cudaStream_t st) {
  if (c % 8 || y_pix_stride % 8 || y_ch_off % 8) return set_error(SDX_ERR_NOT_SUPPORTED, "concat: multiples of 8 only");
  const int64_t total = pixels * (c / 8);
  if (total == 0) return SDX_OK;
  slice_copy_kernel<<<grid_for(total, 256), 256, 0, st>>>(pixels, c, x, y_pix_stride, y_ch_off, y);
  SDX_LAUNCH_CHECK("concat_slice");
  return SDX_OK;
}

// ------------------------------------------------------------------ elementwise
__global__ void binary_kernel(int64_t n8, int op, int relu, const uint4* __restrict__ a, const uint4* __restrict__ b,
                              uint4* __restrict__ y) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    float x[8], z[8];
    h8_to_f(__ldg(a + i), x);
    h8_to_f(__ldg(b + i), z);
#pragma unroll
    for (int j = 0; j < 8; j++) {
      float s = ew_op(x[j], z[j], op);
      x[j] = relu ? fmaxf(s, 0.0f) : s;
    }
    y[i] = f_to_h8(x);
  }
}

int binary_launch(int64_t n, int op, int relu, const __half* a, const __half* b, __half* y, cudaStream_t st) {
  if (n % 8) return set_error(SDX_ERR_NOT_SUPPORTED, "binary: element count must be a multiple of 8");
  if (n == 0) return SDX_OK;
  binary_kernel<<<grid_for(n / 8, 256), 256, 0, st>>>(n / 8, op, relu, reinterpret_cast<const uint4*>(a),
                                                      reinterpret_cast<const uint4*>(b), reinterpret_cast<uint4*>(y));
  SDX_LAUNCH_CHECK("binary");
  return SDX_OK;
}

template <int ACT>
__global__ void act_kernel(int64_t n8, const uint4* __restrict__ x, uint4* __restrict__ y) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    float v[8];
    h8_to_f(__ldg(x + i), v);
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = act_t<ACT>(v[j]);
    y[i] = f_to_h8(v);
  }
}

int act_launch(int64_t n, int act, const __half* x, __half* y, cudaStream_t st) {
  if (n % 8) return set_error(SDX_ERR_NOT_SUPPORTED, "act: element count must be a multiple of 8");
  if (n == 0) return SDX_OK;
  SDX_ACT_DISPATCH(act, ACTC,
                   act_kernel<ACTC><<<grid_for(n / 8, 256), 256, 0, st>>>(n / 8, reinterpret_cast<const uint4*>(x),
                                                                          reinterpret_cast<uint4*>(y)));
  SDX_LAUNCH_CHECK("act");
  return SDX_OK;
}

// fp32 <-> fp16 and NCHW <-> NHWC in one pass. Thread = one element of the output.
// y[n, ch, p] (layout of y) = x[n, ch, p] for ch < c, 0 for c <= ch < c_out (channel padding of a
// graph input so that a tensor-core conv can read it: channel counts there are multiples of 8).
__global__ void convert_kernel(int batch, int c, int c_out, int64_t hw, int x_f32, int x_nchw, int y_f32, int y_nchw,
                               const void* __restrict__ x, void* __restrict__ y) {
  const int64_t total = (int64_t)batch * c_out * hw;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    int64_t n, ch, p;
    if (y_nchw) {
      p = idx % hw;
      ch = (idx / hw) % c_out;
      n = idx / hw / c_out;
    } else {
      ch = idx % c_out;
      p = (idx / c_out) % hw;
      n = idx / c_out / hw;
    }
    float v = 0.0f;
    if (ch < c) {
      const int64_t xi = x_nchw ? (n * c + ch) * hw + p : (n * hw + p) * c + ch;
      v = x_f32 ? __ldg(static_cast<const float*>(x) + xi) : __half2float(static_cast<const __half*>(x)[xi]);
    }
    if (y_f32) static_cast<float*>(y)[idx] = v;
    else static_cast<__half*>(y)[idx] = __float2half_rn(v);
  }
}

// NCHW (fp32 or fp16) -> NHWC fp16 with c_out a multiple of 8: thread = one pixel's 8 output
// channels, read plane by plane (coalesced across the warp's pixels), written as one 16-byte word.
__global__ void convert_nchw_nhwc8_kernel(int batch, int c, int c_out, int64_t hw, int x_f32, const void* __restrict__ x,
                                          __half* __restrict__ y) {
  const int g8 = c_out >> 3;
  const int64_t total = (int64_t)batch * hw * g8;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int g = (int)(idx % g8);
    const int64_t q = idx / g8, n = q / hw, p = q - n * hw;
    uint4 u;
    __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
    for (int j = 0; j < 4; j++) {
      float v[2];
#pragma unroll
      for (int k = 0; k < 2; k++) {
        const int ch = g * 8 + 2 * j + k;
        const int64_t xi = (n * c + ch) * hw + p;
        v[k] = ch >= c ? 0.0f : x_f32 ? __ldg(static_cast<const float*>(x) + xi) : __half2float(static_cast<const __half*>(x)[xi]);
      }
      h[j] = __floats2half2_rn(v[0], v[1]);
    }
    reinterpret_cast<uint4*>(y)[idx] = u;
  }
}

int convert_launch(int batch, int c, int c_out, int64_t hw, int x_f32, int x_nchw, int y_f32, int y_nchw,
                   const void* x, void* y, cudaStream_t st) {
  if (c <= 0 || c_out < c) return set_error(SDX_ERR_INVALID, "convert: output channels below input channels");
  const int64_t total = (int64_t)batch * c_out * hw;
  if (total == 0) return SDX_OK;
  if (x_nchw && !y_nchw && !y_f32 && c_out % 8 == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0) {
    convert_nchw_nhwc8_kernel<<<grid_for(total / 8, 256), 256, 0, st>>>(batch, c, c_out, hw, x_f32, x,
                                                                         static_cast<__half*>(y));
    SDX_LAUNCH_CHECK("convert_nchw_nhwc8");
    return SDX_OK;
  }
  convert_kernel<<<grid_for(total, 256), 256, 0, st>>>(batch, c, c_out, hw, x_f32, x_nchw, y_f32, y_nchw, x, y);
  SDX_LAUNCH_CHECK("convert");
  return SDX_OK;
}

// ------------------------------------------------------------------ LayerNorm / softmax (warp per row)
__global__ void layernorm_kernel(int64_t rows, int c, float eps, const __half* __restrict__ x,
                                 const float* __restrict__ w, const float* __restrict__ b, __half* __restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (row >= rows) return;
  const __half* xr = x + row * c;
  float s = 0.0f, ss = 0.0f;
  for (int i = lane; i < c; i += 32) {
    float v = __half2float(xr[i]);
    s += v;
    ss = fmaf(v, v, ss);
  }
  for (int off = 16; off; off >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, off);
    ss += __shfl_xor_sync(0xffffffffu, ss, off);
  }
  const float mean = s / c;
  const float inv = rsqrtf(fmaxf(ss / c - mean * mean, 0.0f) + eps);
  for (int i = lane; i < c; i += 32)
    y[row * c + i] = __float2half_rn(fmaf(__half2float(xr[i]) - mean, inv * w[i], b[i]));
}

int layernorm_launch(int64_t rows, int c, float eps, const __half* x, const float* w, const float* b, __half* y,
                     cudaStream_t st) {
  if (rows == 0) return SDX_OK;
  layernorm_kernel<<<grid_for(rows * 32, 256), 256, 0, st>>>(rows, c, eps, x, w, b, y);
  SDX_LAUNCH_CHECK("layernorm");
  return SDX_OK;
}

__global__ void softmax_kernel(int64_t rows, int c, int y_f32, const __half* __restrict__ x, void* __restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (row >= rows) return;
  const __half* xr = x + row * c;
  float mx = -INFINITY;
  for (int i = lane; i < c; i += 32) mx = fmaxf(mx, __half2float(xr[i]));
  for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  float s = 0.0f;
  for (int i = lane; i < c; i += 32) s += expf(__half2float(xr[i]) - mx);
  for (int off = 16; off; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  const float inv = 1.0f / s;
  for (int i = lane; i < c; i += 32) {
    float v = expf(__half2float(xr[i]) - mx) * inv;
    if (y_f32) static_cast<float*>(y)[row * c + i] = v;
    else static_cast<__half*>(y)[row * c + i] = __float2half_rn(v);
  }
}

int softmax_launch(int64_t rows, int c, int y_f32, const __half* x, void* y, cudaStream_t st) {
  if (rows == 0) return SDX_OK;
  softmax_kernel<<<grid_for(rows * 32, 256), 256, 0, st>>>(rows, c, y_f32, x, y);
  SDX_LAUNCH_CHECK("softmax");
  return SDX_OK;
}

// ------------------------------------------------------------------ attention (short sequences)
// out[n, t, h*d + j] = sum_s softmax_s(scale * q[n,t,h,:] . k[n,s,h,:]) v[n,s,h,j], one CTA per (n, h);
// q/k/v rows of the fused projection [n, t, 3, h, d].
__global__ void attention_kernel(int t, int heads, int d, float scale, const __half* __restrict__ qkv,
                                 __half* __restrict__ y) {
  extern __shared__ float sm[];
  const int n = blockIdx.x / heads, h = blockIdx.x % heads;
  float* q = sm;
  float* k = q + t * d;
  float* v = k + t * d;
  float* p = v + t * d;  // [t][t]
  const int64_t row_stride = 3LL * heads * d;
  for (int i = threadIdx.x; i < t * d; i += blockDim.x) {
    const int s = i / d, j = i % d;
    const __half* r = qkv + ((int64_t)n * t + s) * row_stride + (int64_t)h * d + j;
    q[i] = __half2float(r[0]);
    k[i] = __half2float(r[(int64_t)heads * d]);
    v[i] = __half2float(r[2LL * heads * d]);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < t * t; i += blockDim.x) {
    const int a = i / t, b = i % t;
    float s = 0.0f;
    for (int j = 0; j < d; j++) s = fmaf(q[a * d + j], k[b * d + j], s);
    p[i] = s * scale;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int a = warp; a < t; a += nw) {
    float mx = -INFINITY;
    for (int b = lane; b < t; b += 32) mx = fmaxf(mx, p[a * t + b]);
    for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    float s = 0.0f;
    for (int b = lane; b < t; b += 32) {
      float e = expf(p[a * t + b] - mx);
      p[a * t + b] = e;
      s += e;
    }
    for (int off = 16; off; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    const float inv = 1.0f / s;
    __syncwarp();
    for (int b = lane; b < t; b += 32) p[a * t + b] *= inv;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < t * d; i += blockDim.x) {
    const int a = i / d, j = i % d;
    float s = 0.0f;
    for (int b = 0; b < t; b++) s = fmaf(p[a * t + b], v[b * d + j], s);
    y[((int64_t)n * t + a) * heads * d + (int64_t)h * d + j] = __float2half_rn(s);
  }
}

int attention_launch(int batch, int t, int heads, int d, float scale, const __half* qkv, __half* y, cudaStream_t st) {
  const size_t smem = sizeof(float) * ((size_t)3 * t * d + (size_t)t * t);
  if (smem > 160 * 1024) return set_error(SDX_ERR_NOT_SUPPORTED, "attention: sequence too long for the smem kernel");
  if (batch * heads == 0) return SDX_OK;
  static SmemAttr attr{};
  const int rc = raise_smem_limit(attr, (const void*)attention_kernel, 160 * 1024, "cudaFuncSetAttribute(attention)");
  if (rc) return rc;
  attention_kernel<<<batch * heads, 128, smem, st>>>(t, heads, d, scale, qkv, y);
  SDX_LAUNCH_CHECK("attention");
  return SDX_OK;
}

// ------------------------------------------------------------------ bounded-wait self test
// Spins on a shared flag that nothing sets, for at most wait_ms, then records SDX_DEV_TEST_WAIT and
// returns: the failure path of every bounded wait in this library, exercised without a fault.
__global__ void bounded_wait_kernel(unsigned int* err, uint64_t wait_ns) {
  __shared__ volatile int flag;
  if (threadIdx.x == 0) flag = 0;
  __syncthreads();
  if (threadIdx.x != 0) return;
  const uint64_t t0 = global_timer_ns();
  while (!flag) {
    if (global_timer_ns() - t0 > wait_ns) {
      record_error(err, SDX_DEV_TEST_WAIT);
      return;
    }
  }
}

int bounded_wait_selftest_launch(unsigned int* err, int wait_ms, cudaStream_t st) {
  bounded_wait_kernel<<<1, 32, 0, st>>>(err, (uint64_t)std::max(1, wait_ms) * 1000000ull);
  SDX_LAUNCH_CHECK("bounded_wait_selftest");
  return SDX_OK;
}

}  // namespace sdx
