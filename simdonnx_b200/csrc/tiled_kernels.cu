// Shared-memory tiled bandwidth kernels: depthwise conv and the small-channel stem conv.
//
// Both stage an input tile (+ halo) and the weights in shared memory once per block with coalesced
// 16-byte loads, then every output reads its taps from shared memory, so each input element
// crosses L2 -> SM about once per tile instead of once per tap. Kernel size, stride and the fused
// activation are compile-time, so the tap loops unroll completely.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "sdx_device.cuh"
#include "sdx_internal.h"

namespace sdx {

// ------------------------------------------------------------------ depthwise
// y[n, oy, ox, c] = act(b[c] + sum_{ky,kx} w[ky,kx,c] * s[n,c] * x[n, oy*S+ky-pt, ox*S+kx-pl, c] [+ add])
// (Nhwc.Depthwise, src/Kernels/Nhwc.cs:496-631; constant-0 padding). Block = TH x TW outputs of one
// image for a slab of CS channels (G = CS/8 channel groups of 8). Thread = one channel group of a
// strip of R = 4 horizontally adjacent outputs: per kernel row it reads the strip's (R-1)*S+K input
// vectors once and each tap's 8 weights once, and reuses them across the strip (register blocking).
// The squeeze-excitation scale s[n, c] of the producer is folded into the staged weights
// (sum w*(s*x) == sum (w*s)*x, one rounding either way).
constexpr int DW_R = 4;

template <int ACT, int K, int S>
__global__ void __launch_bounds__(256) dw_tiled_kernel(DwArgs a, int CS, int TH, int TW, int tiles_x) {
  extern __shared__ float4 dsm_f4[];
  float* sw = reinterpret_cast<float*>(dsm_f4);
  const int G = CS >> 3;
  const int IWt = (TW - 1) * S + K, IHt = (TH - 1) * S + K;
  uint4* stile = reinterpret_cast<uint4*>(sw + K * K * CS);  // [IHt*IWt][G] x 8 halves
  const int n = blockIdx.z, c0 = blockIdx.y * CS;
  const int ty = blockIdx.x / tiles_x, tx = blockIdx.x - ty * tiles_x;
  const int oy0 = ty * TH, ox0 = tx * TW;
  const int iy0 = oy0 * S - a.pt, ix0 = ox0 * S - a.pl;
  const int tid = threadIdx.x;

  for (int i = tid; i < K * K * CS; i += blockDim.x) {
    const int tap = i / CS, c = i - tap * CS;
    float w = __ldg(a.w + (int64_t)tap * a.c + c0 + c);
    if (a.in_scale) w *= __ldg(a.in_scale + (int64_t)n * a.c + c0 + c);
    sw[i] = w;
  }
  const __half* xb = a.x + (int64_t)n * a.ih * a.iw * a.c + c0;
  for (int i = tid; i < IHt * IWt * G; i += blockDim.x) {
    const int p = i / G, g = i - p * G;
    const int r = p / IWt, col = p - r * IWt;
    const int iy = iy0 + r, ix = ix0 + col;
    uint4 u = make_uint4(0, 0, 0, 0);
    if ((unsigned)iy < (unsigned)a.ih && (unsigned)ix < (unsigned)a.iw)
      u = __ldg(reinterpret_cast<const uint4*>(xb + ((int64_t)iy * a.iw + ix) * a.c + g * 8));
    stile[i] = u;
  }
  __syncthreads();

  const int cg = tid % G, strip = tid / G;
  const int spr = TW / DW_R;
  const int sy = strip / spr, sx = strip - sy * spr;
  if (sy >= TH) return;
  const int oy = oy0 + sy;
  if (oy >= a.oh) return;
  const int c = c0 + cg * 8;
  float acc[DW_R][8];
  {
    const float4* bp = reinterpret_cast<const float4*>(a.bias + c);
    float4 b0 = __ldg(bp), b1 = __ldg(bp + 1);
#pragma unroll
    for (int r = 0; r < DW_R; r++) {
      acc[r][0] = b0.x; acc[r][1] = b0.y; acc[r][2] = b0.z; acc[r][3] = b0.w;
      acc[r][4] = b1.x; acc[r][5] = b1.y; acc[r][6] = b1.z; acc[r][7] = b1.w;
    }
  }
  constexpr int NX = (DW_R - 1) * S + K;
  const int lx0 = sx * DW_R * S;
#pragma unroll
  for (int ky = 0; ky < K; ky++) {
    const uint4* row = stile + ((sy * S + ky) * IWt + lx0) * G + cg;
    float xv[NX][8];
#pragma unroll
    for (int j = 0; j < NX; j++) {
      const uint4 u = row[j * G];
      const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
      for (int i = 0; i < 4; i++) {
        float2 t = __half22float2(h[i]);
        xv[j][2 * i] = t.x;
        xv[j][2 * i + 1] = t.y;
      }
    }
#pragma unroll
    for (int kx = 0; kx < K; kx++) {
      const float4* wp = reinterpret_cast<const float4*>(sw + (ky * K + kx) * CS + cg * 8);
      const float4 w0 = wp[0], w1 = wp[1];
      const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int r = 0; r < DW_R; r++)
#pragma unroll
        for (int q = 0; q < 8; q++) acc[r][q] = fmaf(xv[r * S + kx][q], wv[q], acc[r][q]);
    }
  }
#pragma unroll
  for (int r = 0; r < DW_R; r++) {
    const int ox = ox0 + sx * DW_R + r;
    if (ox >= a.ow) break;
    const int64_t off = (((int64_t)n * a.oh + oy) * a.ow + ox) * a.c + c;
    if (a.add) {
      const uint4 ru = __ldg(reinterpret_cast<const uint4*>(a.add + off));
      const __half2* h = reinterpret_cast<const __half2*>(&ru);
#pragma unroll
      for (int i = 0; i < 4; i++) {
        float2 t = __half22float2(h[i]);
        acc[r][2 * i] += t.x;
        acc[r][2 * i + 1] += t.y;
      }
    }
    uint4 u;
    __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; i++) h[i] = __floats2half2_rn(act_t<ACT>(acc[r][2 * i]), act_t<ACT>(acc[r][2 * i + 1]));
    *reinterpret_cast<uint4*>(a.y + off) = u;
  }
}

template <int ACT, int K, int S>
static int dw_launch_t(const DwArgs& a, cudaStream_t st) {
  const int CS = a.c <= 64 ? a.c : 64;
  const int G = CS / 8;
  const int TW = 16, TH = (256 / G) / (TW / DW_R);
  const int IWt = (TW - 1) * S + K, IHt = (TH - 1) * S + K;
  const size_t smem = sizeof(float) * K * K * CS + (size_t)IHt * IWt * CS * 2;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(dw_tiled_kernel<ACT, K, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    attr = true;
  }
  const int tiles_x = (a.ow + TW - 1) / TW, tiles_y = (a.oh + TH - 1) / TH;
  dim3 grid(tiles_x * tiles_y, a.c / CS, a.batch);
  dw_tiled_kernel<ACT, K, S><<<grid, 256, smem, st>>>(a, CS, TH, TW, tiles_x);
  return SDX_OK;
}

template <int ACT>
static bool dw_dispatch_ks(const DwArgs& a, cudaStream_t st) {
#define SDX_DW_CASE(KK, SS)                                   \
  if (a.kh == KK && a.kw == KK && a.sh == SS && a.sw == SS) { \
    dw_launch_t<ACT, KK, SS>(a, st);                          \
    return true;                                              \
  }
  SDX_DW_CASE(3, 1)
  SDX_DW_CASE(3, 2)
  SDX_DW_CASE(5, 1)
  SDX_DW_CASE(5, 2)
#undef SDX_DW_CASE
  return false;
}

bool depthwise_tiled_launch(const DwArgs& a, cudaStream_t st) {
  // channel slabs of 16, 32 or 64 (the strip layout needs 256 / (CS/8) to be a multiple of 4)
  if (a.c % 8 != 0 || a.batch > 65535) return false;
  if (!(a.c == 16 || a.c == 32 || a.c % 64 == 0)) return false;
  switch (a.act) {
    case ACT_HARDSWISH: return dw_dispatch_ks<ACT_HARDSWISH>(a, st);
    case ACT_RELU: return dw_dispatch_ks<ACT_RELU>(a, st);
    case ACT_NONE: return dw_dispatch_ks<ACT_NONE>(a, st);
    default: return false;
  }
}

// ------------------------------------------------------------------ small-channel stem conv
// Dense k x k conv with IC <= 4 (graph-input stems: fp32 NCHW or NHWC input, fp16 NHWC output):
// the input planes of a TH x TW output tile (+ halo) and all weights in shared memory; thread = one
// output pixel, output channels in groups of 8 (16-byte stores).
template <int ACT, int K, int S>
__global__ void __launch_bounds__(256) stem_tiled_kernel(DirectArgs a, int TH, int TW, int tiles_x) {
  extern __shared__ float ssm[];
  const int IWt = (TW - 1) * S + K, IHt = (TH - 1) * S + K;
  float* sw = ssm;                                // [K*K][IC][OC]
  float* st = ssm + K * K * a.ic * a.oc;          // [IC][IHt][IWt]
  const int n = blockIdx.y;
  const int ty = blockIdx.x / tiles_x, tx = blockIdx.x - ty * tiles_x;
  const int oy0 = ty * TH, ox0 = tx * TW;
  const int iy0 = oy0 * S - a.pt, ix0 = ox0 * S - a.pl;
  const int tid = threadIdx.x;
  for (int i = tid; i < K * K * a.ic * a.oc; i += blockDim.x) sw[i] = __ldg(a.w + i);
  for (int i = tid; i < a.ic * IHt * IWt; i += blockDim.x) {
    const int c = i / (IHt * IWt), rem = i - c * IHt * IWt;
    const int r = rem / IWt, col = rem - r * IWt;
    const int iy = iy0 + r, ix = ix0 + col;
    float v = 0.0f;
    if ((unsigned)iy < (unsigned)a.ih && (unsigned)ix < (unsigned)a.iw) {
      const int64_t off = a.x_nchw ? (((int64_t)n * a.ic + c) * a.ih + iy) * a.iw + ix
                                   : (((int64_t)n * a.ih + iy) * a.iw + ix) * a.ic + c;
      v = a.x_f32 ? __ldg(static_cast<const float*>(a.x) + off) : __half2float(static_cast<const __half*>(a.x)[off]);
    }
    st[i] = v;
  }
  __syncthreads();
  const int ly = tid / TW, lx = tid - ly * TW;
  const int oy = oy0 + ly, ox = ox0 + lx;
  if (ly >= TH || oy >= a.oh || ox >= a.ow) return;
  const int64_t obase = (((int64_t)n * a.oh + oy) * a.ow + ox) * a.y_pix_stride + a.y_ch_off;
  for (int o0 = 0; o0 < a.oc; o0 += 8) {
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; j++) acc[j] = a.bias ? __ldg(a.bias + o0 + j) : 0.0f;
    for (int c = 0; c < a.ic; c++) {
      const float* tc = st + c * IHt * IWt;
#pragma unroll
      for (int ky = 0; ky < K; ky++) {
#pragma unroll
        for (int kx = 0; kx < K; kx++) {
          const float xv = tc[(ly * S + ky) * IWt + lx * S + kx];
          const float* wp = sw + ((ky * K + kx) * a.ic + c) * a.oc + o0;
#pragma unroll
          for (int j = 0; j < 8; j++) acc[j] = fmaf(xv, wp[j], acc[j]);
        }
      }
    }
    uint4 u;
    __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; i++) h[i] = __floats2half2_rn(act_t<ACT>(acc[2 * i]), act_t<ACT>(acc[2 * i + 1]));
    *reinterpret_cast<uint4*>(static_cast<__half*>(a.y) + obase + o0) = u;
  }
}

template <int ACT, int K, int S>
static void stem_launch_t(const DirectArgs& a, cudaStream_t st) {
  const int TH = 8, TW = 32;
  const int IWt = (TW - 1) * S + K, IHt = (TH - 1) * S + K;
  const size_t smem = sizeof(float) * ((size_t)K * K * a.ic * a.oc + (size_t)a.ic * IHt * IWt);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(stem_tiled_kernel<ACT, K, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
    attr = true;
  }
  const int tiles_x = (a.ow + TW - 1) / TW, tiles_y = (a.oh + TH - 1) / TH;
  dim3 grid(tiles_x * tiles_y, a.batch);
  stem_tiled_kernel<ACT, K, S><<<grid, 256, smem, st>>>(a, TH, TW, tiles_x);
}

bool stem_tiled_launch(const DirectArgs& a, cudaStream_t st) {
  if (a.ic > 4 || a.oc % 8 != 0 || a.oc > 64 || a.add || a.y_f32 || a.y_nchw || a.kh != 3 || a.kw != 3 ||
      a.sh != a.sw || (a.sh != 1 && a.sh != 2) || a.batch > 65535 || (a.y_pix_stride % 8) || (a.y_ch_off % 8))
    return false;
  const size_t smem = sizeof(float) * ((size_t)9 * a.ic * a.oc + (size_t)a.ic * (7 * a.sh + 3) * (31 * a.sh + 3));
  if (smem > 96 * 1024) return false;
  switch (a.act) {
#define SDX_STEM_CASE(ACTC)                                               \
  case ACTC:                                                              \
    if (a.sh == 1) stem_launch_t<ACTC, 3, 1>(a, st);                      \
    else stem_launch_t<ACTC, 3, 2>(a, st);                                \
    return true;
    SDX_STEM_CASE(ACT_HARDSWISH)
    SDX_STEM_CASE(ACT_RELU)
    SDX_STEM_CASE(ACT_NONE)
#undef SDX_STEM_CASE
    default: return false;
  }
}

}  // namespace sdx
