// Shared-memory tiled bandwidth kernels: depthwise conv and the small-channel stem conv.
//
// Both stage an input tile (+ halo) and the weights in shared memory once per block with coalesced
// 16-byte loads, then every output reads its taps from shared memory, so each input element
// crosses L2 -> SM about once per tile instead of once per tap. Kernel size, stride and the fused
// activation are compile-time, so the tap loops unroll completely.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <type_traits>

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
static bool dw_launch_t(const DwArgs& a, cudaStream_t st) {
  const int CS = a.c <= 64 ? a.c : 64;
  const int G = CS / 8;
  const int TW = 16, TH = (256 / G) / (TW / DW_R);
  const int IWt = (TW - 1) * S + K, IHt = (TH - 1) * S + K;
  const size_t smem = sizeof(float) * K * K * CS + (size_t)IHt * IWt * CS * 2;
  static SmemAttr attr{};
  if (raise_smem_limit(attr, (const void*)dw_tiled_kernel<ACT, K, S>, 160 * 1024, "cudaFuncSetAttribute(dw_tiled)"))
    return false;
  const int tiles_x = (a.ow + TW - 1) / TW, tiles_y = (a.oh + TH - 1) / TH;
  dim3 grid(tiles_x * tiles_y, a.c / CS, a.batch);
  dw_tiled_kernel<ACT, K, S><<<grid, 256, smem, st>>>(a, CS, TH, TW, tiles_x);
  return true;
}

// ---- persistent, TMA-fed form. Each CTA walks a contiguous range of tiles (image, channel slab,
// tile row, tile column); thread 0 prefetches the next tile's input box (+ halo, zero fill = padding)
// with one TMA load into the other of two buffers while all threads compute the current one, so
// loads overlap compute and need no per-element index math. Weights (times the image's SE scale)
// are restaged only when the image or slab changes. All waits are bounded; a failed wait ends the
// CTA through a block-uniform vote after draining its copies in flight.
template <int ACT, int K, int S, int R>
__global__ void __launch_bounds__(256) dw_tma_kernel(const __grid_constant__ CUtensorMap tmX, DwArgs a, int CS, int TH,
                                                     int TW, int tiles_x, int tiles_per_img, int slabs, int total) {
  extern __shared__ uint8_t dsm_raw[];
  uint8_t* dsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 127) & ~uintptr_t(127));
  const int G = CS >> 3;
  const int IWt = (TW - 1) * S + K, IHt = (TH - 1) * S + K;
  const uint32_t tile_bytes = (uint32_t)IHt * IWt * CS * 2;
  const uint32_t buf_bytes = (tile_bytes + 127u) & ~127u;
  const uint4* bufs = reinterpret_cast<const uint4*>(dsm);
  float* sw = reinterpret_cast<float*>(dsm + 2 * buf_bytes);                       // [K*K][CS]
  uint64_t* full = reinterpret_cast<uint64_t*>(dsm + 2 * buf_bytes + ((K * K * CS * 4 + 15) & ~15));
  __shared__ int abort_flag;
  const int tid = threadIdx.x;
  const int per = (total + gridDim.x - 1) / gridDim.x;
  const int t0 = blockIdx.x * per, t1 = min(total, t0 + per);
  if (t0 >= t1) return;
  auto decode = [&](int t, int& n, int& slab, int& oy0, int& ox0) {
    n = t / (slabs * tiles_per_img);
    const int r = t - n * slabs * tiles_per_img;
    slab = r / tiles_per_img;
    const int q = r - slab * tiles_per_img;
    const int ty = q / tiles_x;
    oy0 = ty * TH;
    ox0 = (q - ty * tiles_x) * TW;
  };
  // warp 0 issues the tile copies warp-uniformly from its elected lane
  uint32_t ld0 = 0;
  if (tid < 32) ld0 = elect_leader();
  auto issue = [&](int t, int b) {
    int n, slab, oy0, ox0;
    decode(t, n, slab, oy0, ox0);
    const uint32_t bar = smem_u32(&full[b]);
    mbar_arrive_expect_tx_p(ld0, bar, tile_bytes);
    tma_load_4d_p(ld0, smem_u32(dsm + b * buf_bytes), &tmX, bar, slab * CS, ox0 * S - a.pl, oy0 * S - a.pt, n);
  };
  uint32_t issued[2] = {0, 0};  // warp 0: copies issued into each buffer
  if (tid == 0) {
    abort_flag = 0;
    mbar_init(smem_u32(&full[0]), 1);
    mbar_init(smem_u32(&full[1]), 1);
    mbar_fence_init();
    tma_prefetch_desc(&tmX);
  }
  __syncthreads();
  if (tid < 32) {
    issue(t0, 0);
    issued[0] = 1;
  }
  const int cg = tid % G, strip = tid / G;
  const int spr = TW / R;
  const int sy = strip / spr, sx = strip - sy * spr;
  constexpr int NX = (R - 1) * S + K;
  int key = -1;
  int i = 0;
  for (int t = t0; t < t1; t++, i++) {
    const int b = i & 1;
    if (tid < 32 && t + 1 < t1) {
      // buffer b^1 was last read by tile i-1, which every thread finished before the barrier that
      // ended that iteration
      issue(t + 1, b ^ 1);
      issued[b ^ 1]++;
    }
    int n, slab, oy0, ox0;
    decode(t, n, slab, oy0, ox0);
    const int c0 = slab * CS;
    if (n * slabs + slab != key) {
      key = n * slabs + slab;
      for (int j = tid; j < K * K * CS; j += blockDim.x) {
        const int tap = j / CS, c = j - tap * CS;
        float w = __ldg(a.w + (int64_t)tap * a.c + c0 + c);
        if (a.in_scale) w *= __ldg(a.in_scale + (int64_t)n * a.c + c0 + c);
        sw[j] = w;
      }
      __syncthreads();
    }
    const bool ok = mbar_wait(smem_u32(&full[b]), (uint32_t)(i >> 1) & 1u, a.err, SDX_DEV_WAIT_FULL, &abort_flag);
    if (__syncthreads_or(!ok)) break;
    const uint4* stile = bufs + (size_t)b * (buf_bytes / 16);
    const int oy = oy0 + sy;
    if (sy < TH && oy < a.oh) {
      const int c = c0 + cg * 8;
      float acc[R][8];
      {
        const float4* bp = reinterpret_cast<const float4*>(a.bias + c);
        const float4 b0 = __ldg(bp), b1 = __ldg(bp + 1);
#pragma unroll
        for (int r = 0; r < R; r++) {
          acc[r][0] = b0.x; acc[r][1] = b0.y; acc[r][2] = b0.z; acc[r][3] = b0.w;
          acc[r][4] = b1.x; acc[r][5] = b1.y; acc[r][6] = b1.z; acc[r][7] = b1.w;
        }
      }
      const int lx0 = sx * R * S;
#pragma unroll
      for (int ky = 0; ky < K; ky++) {
        // this kernel row's weights stay in registers; input vectors stream through once each
        float wr[K][8];
#pragma unroll
        for (int kx = 0; kx < K; kx++) {
          const float4* wp = reinterpret_cast<const float4*>(sw + (ky * K + kx) * CS + cg * 8);
          const float4 w0 = wp[0], w1 = wp[1];
          wr[kx][0] = w0.x; wr[kx][1] = w0.y; wr[kx][2] = w0.z; wr[kx][3] = w0.w;
          wr[kx][4] = w1.x; wr[kx][5] = w1.y; wr[kx][6] = w1.z; wr[kx][7] = w1.w;
        }
        const uint4* row = stile + ((sy * S + ky) * IWt + lx0) * G + cg;
#pragma unroll
        for (int j = 0; j < NX; j++) {
          const uint4 u = row[j * G];
          const __half2* h = reinterpret_cast<const __half2*>(&u);
          float xv[8];
#pragma unroll
          for (int q = 0; q < 4; q++) {
            const float2 f = __half22float2(h[q]);
            xv[2 * q] = f.x;
            xv[2 * q + 1] = f.y;
          }
#pragma unroll
          for (int r = 0; r < R; r++) {
            const int kx = j - r * S;
            if (kx >= 0 && kx < K) {
#pragma unroll
              for (int q = 0; q < 8; q++) acc[r][q] = fmaf(xv[q], wr[kx][q], acc[r][q]);
            }
          }
        }
      }
#pragma unroll
      for (int r = 0; r < R; r++) {
        const int ox = ox0 + sx * R + r;
        if (ox >= a.ow) break;
        const int64_t off = (((int64_t)n * a.oh + oy) * a.ow + ox) * a.c + c;
        if (a.add) {
          const uint4 ru = __ldg(reinterpret_cast<const uint4*>(a.add + off));
          const __half2* h = reinterpret_cast<const __half2*>(&ru);
#pragma unroll
          for (int q = 0; q < 4; q++) {
            const float2 f = __half22float2(h[q]);
            acc[r][2 * q] += f.x;
            acc[r][2 * q + 1] += f.y;
          }
        }
        uint4 u;
        __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
        for (int q = 0; q < 4; q++) h[q] = __floats2half2_rn(act_t<ACT>(acc[r][2 * q]), act_t<ACT>(acc[r][2 * q + 1]));
        *reinterpret_cast<uint4*>(a.y + off) = u;
      }
    }
    __syncthreads();
  }
  // wind-down (only after an abort can a copy still be in flight): drain every issued copy
  if (tid < 32) {
    for (int b = 0; b < 2; b++)
      if (issued[b] > 0) mbar_wait_drain(smem_u32(&full[b]), (issued[b] - 1) & 1u, a.err, SDX_DEV_WAIT_DRAIN);
  }
}

template <int ACT, int K, int S, int R>
static bool dw_tma_launch_t(const DwArgs& a, cudaStream_t st) {
  if ((reinterpret_cast<uintptr_t>(a.x) & 15u) || (a.c * 2) % 16) return false;
  const int CS = a.c <= 64 ? a.c : 64;
  const int G = CS / 8;
  const int TW = 16, TH = (256 / G) / (TW / R);
  const int IWt = (TW - 1) * S + K, IHt = (TH - 1) * S + K;
  if (IWt > 256 || IHt > 256) return false;
  const size_t tile_bytes = (size_t)IHt * IWt * CS * 2;
  const size_t smem = 128 + 2 * ((tile_bytes + 127) & ~(size_t)127) + ((K * K * CS * 4 + 15) & ~15) + 16;
  if (smem > 200 * 1024) return false;
  PFN_encodeTiled enc = get_encode_tiled();
  if (!enc) return false;
  CUtensorMap map;
  const cuuint64_t dims[4] = {(cuuint64_t)a.c, (cuuint64_t)a.iw, (cuuint64_t)a.ih, (cuuint64_t)a.batch};
  const cuuint64_t strides[3] = {(cuuint64_t)a.c * 2, (cuuint64_t)a.iw * a.c * 2, (cuuint64_t)a.ih * a.iw * a.c * 2};
  const cuuint32_t box[4] = {(cuuint32_t)CS, (cuuint32_t)IWt, (cuuint32_t)IHt, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<__half*>(a.x), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  static SmemAttr attr{};
  if (raise_smem_limit(attr, (const void*)dw_tma_kernel<ACT, K, S, R>, 200 * 1024, "cudaFuncSetAttribute(dw_tma)"))
    return false;
  const int tiles_x = (a.ow + TW - 1) / TW, tiles_y = (a.oh + TH - 1) / TH;
  const int slabs = a.c / CS;
  const int64_t total = (int64_t)a.batch * slabs * tiles_x * tiles_y;
  if (total <= 0 || total > INT32_MAX) return false;
  int dev = 0, per_sm = 1;
  cudaGetDevice(&dev);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, dw_tma_kernel<ACT, K, S, R>, 256, smem);
  const int grid = (int)std::min<int64_t>(total, (int64_t)num_sms(dev) * std::max(1, per_sm));
  dw_tma_kernel<ACT, K, S, R><<<grid, 256, smem, st>>>(map, a, CS, TH, TW, tiles_x, tiles_x * tiles_y, slabs, (int)total);
  return true;
}

// ---- stride-1 sliding-window form. A thread owns CPT channels (1 or 2) of a strip of RX output
// columns and walks down the tile's rows: each input row is read from shared memory once (RX + K - 1
// pixels), turned into fp32 once, and applied to the K output rows it touches, whose accumulators
// sit in a ring of K register rows. An output row is finished, activated and stored as soon as its
// last input row has been applied. The weights of the thread's channels (times the image's SE scale)
// stay in fp32 registers. The slab width CS, the strip and the tile width are compile-time, so every
// shared-memory offset inside a row is an immediate; the tile height TH is one less than a multiple
// of K, so the row walk splits into a prologue (K - 1 rows), whole groups of K rows and a tail (K - 1
// rows) in which every ring slot and every kernel-row bound is compile-time.
// A warp reads whole pixel runs of the [IHt][IWt][CS] tile; with RX = 5 the strips that share a
// warp start 40 or 80 words apart, so the reads are conflict-free.
// Register budget (two 256-thread CTAs per SM, <= 128 each): a channel pair per thread (CPT = 2,
// one packed f32x2 FMA per tap) for K = 3 and K = 5 (K = 5 takes all 128: 50 accumulators, 50
// weights, 18 inputs).
template <int CPT>
__device__ __forceinline__ void dw_load_px(const uint8_t* p, float (&v)[CPT]) {
  if constexpr (CPT == 2) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(p));
    v[0] = f.x;
    v[1] = f.y;
  } else {
    v[0] = __half2float(*reinterpret_cast<const __half*>(p));
  }
}

// acc += x * w on a channel pair with one packed f32x2 FMA (sm_100): each lane is the same
// single-rounding fmaf, so results equal the scalar form bit for bit.
__device__ __forceinline__ void ffma2(float& a0, float& a1, float x0, float x1, float w0, float w1) {
  asm("{\n\t.reg .b64 ra, rx, rw;\n\t"
      "mov.b64 ra, {%0, %1};\n\tmov.b64 rx, {%2, %3};\n\tmov.b64 rw, {%4, %5};\n\t"
      "fma.rn.f32x2 ra, rx, rw, ra;\n\tmov.b64 {%0, %1}, ra;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(x0), "f"(x1), "f"(w0), "f"(w1));
}

// acc[q] += x[q] * w[q] over the CPT channels of a thread (packed for channel pairs)
template <int CPT>
__device__ __forceinline__ void fma_px(float (&acc)[CPT], const float (&x)[CPT], const float (&w)[CPT]) {
  if constexpr (CPT == 2) {
    ffma2(acc[0], acc[1], x[0], x[1], w[0], w[1]);
  } else {
#pragma unroll
    for (int q = 0; q < CPT; q++) acc[q] = fmaf(x[q], w[q], acc[q]);
  }
}

// Compile-time loop: f(std::integral_constant<int, I>) for I = I0 .. N-1.
template <int I0, int N, class F>
__device__ __forceinline__ void static_for(F&& f) {
  if constexpr (I0 < N) {
    f(std::integral_constant<int, I0>{});
    static_for<I0 + 1, N>(f);
  }
}

// Applies input row `rowp` (kernel rows KY0..KY1) to the ring: kernel row ky feeds ring slot
// (SL0 - ky) mod K.
template <int K, int RX, int CPT, int PXB, int KY0, int KY1, int SL0>
__device__ __forceinline__ void dw_row(const uint8_t* rowp, float (&acc)[K][RX][CPT], const float (&w)[K][K][CPT]) {
  float xf[RX + K - 1][CPT];
#pragma unroll
  for (int j = 0; j < RX + K - 1; j++) dw_load_px<CPT>(rowp + j * PXB, xf[j]);
#pragma unroll
  for (int ky = KY0; ky <= KY1; ky++) {
    const int sl = ((SL0 - ky) % K + K) % K;
#pragma unroll
    for (int r = 0; r < RX; r++)
#pragma unroll
      for (int kx = 0; kx < K; kx++) fma_px<CPT>(acc[sl][r], xf[r + kx], w[ky][kx]);
  }
}

// Finishes output row `oy` from ring slot SL: bias is already in; + residual, activation, store;
// then the slot restarts at the bias.
template <int ACT, int K, int RX, int CPT, int SL>
__device__ __forceinline__ void dw_store_row(const DwArgs& a, float (&acc)[K][RX][CPT], const float (&bias)[CPT], int oy,
                                             int64_t base, int ncols) {
  if (oy < a.oh) {
    if (ncols >= RX) {
#pragma unroll
      for (int r = 0; r < RX; r++) {
        float v[CPT];
#pragma unroll
        for (int q = 0; q < CPT; q++) v[q] = acc[SL][r][q];
        if (a.add) {
          float ad[CPT];
          dw_load_px<CPT>(reinterpret_cast<const uint8_t*>(a.add + base + (int64_t)r * a.c), ad);
#pragma unroll
          for (int q = 0; q < CPT; q++) v[q] += ad[q];
        }
        if constexpr (CPT == 2)
          *reinterpret_cast<__half2*>(a.y + base + (int64_t)r * a.c) =
              __floats2half2_rn(act_t<ACT>(v[0]), act_t<ACT>(v[1]));
        else
          a.y[base + (int64_t)r * a.c] = __float2half_rn(act_t<ACT>(v[0]));
      }
    } else {
#pragma unroll
      for (int r = 0; r < RX; r++) {
        if (r < ncols) {
          float v[CPT];
#pragma unroll
          for (int q = 0; q < CPT; q++) v[q] = acc[SL][r][q];
          if (a.add) {
            float ad[CPT];
            dw_load_px<CPT>(reinterpret_cast<const uint8_t*>(a.add + base + (int64_t)r * a.c), ad);
#pragma unroll
            for (int q = 0; q < CPT; q++) v[q] += ad[q];
          }
          if constexpr (CPT == 2)
            *reinterpret_cast<__half2*>(a.y + base + (int64_t)r * a.c) =
                __floats2half2_rn(act_t<ACT>(v[0]), act_t<ACT>(v[1]));
          else
            a.y[base + (int64_t)r * a.c] = __float2half_rn(act_t<ACT>(v[0]));
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RX; r++)
#pragma unroll
    for (int q = 0; q < CPT; q++) acc[SL][r][q] = bias[q];
}

template <int ACT, int K, int RX, int CPT, int CS>
__global__ void __launch_bounds__(256, 2) dw_slide_kernel(const __grid_constant__ CUtensorMap tmX, DwArgs a, int TH,
                                                          int tiles_x, int tiles_y, int slabs, int total) {
  constexpr int TPP = CS / CPT;          // threads per pixel
  constexpr int TW = RX * (256 / TPP);   // tile width: one strip per thread group
  constexpr int IWt = TW + K - 1;
  constexpr int PXB = CS * 2;            // bytes per pixel in the tile
  constexpr int ROWB = IWt * PXB;        // bytes per tile row
  extern __shared__ uint8_t dsm_raw[];
  uint8_t* dsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 127) & ~uintptr_t(127));
  const int IHt = TH + K - 1;
  const uint32_t tile_bytes = (uint32_t)IHt * ROWB;
  const uint32_t buf_bytes = (tile_bytes + 127u) & ~127u;
  uint64_t* full = reinterpret_cast<uint64_t*>(dsm + 2 * buf_bytes);
  __shared__ int abort_flag;
  const int tid = threadIdx.x;
  const int per = (total + gridDim.x - 1) / gridDim.x;
  const int t0 = blockIdx.x * per, t1 = min(total, t0 + per);
  if (t0 >= t1) return;
  const int tiles_per_img = tiles_x * tiles_y;
  auto decode = [&](int t, int& n, int& slab, int& oy0, int& ox0) {
    n = t / (slabs * tiles_per_img);
    const int r = t - n * slabs * tiles_per_img;
    slab = r / tiles_per_img;
    const int q = r - slab * tiles_per_img;
    const int ty = q / tiles_x;
    oy0 = ty * TH;
    ox0 = (q - ty * tiles_x) * TW;
  };
  // warp 0 issues the tile copies warp-uniformly from its elected lane
  uint32_t ld0 = 0;
  if (tid < 32) ld0 = elect_leader();
  auto issue = [&](int t, int b) {
    int n, slab, oy0, ox0;
    decode(t, n, slab, oy0, ox0);
    const uint32_t bar = smem_u32(&full[b]);
    mbar_arrive_expect_tx_p(ld0, bar, tile_bytes);
    tma_load_4d_p(ld0, smem_u32(dsm + b * buf_bytes), &tmX, bar, slab * CS, ox0 - a.pl, oy0 - a.pt, n);
  };
  uint32_t issued[2] = {0, 0};
  if (tid == 0) {
    abort_flag = 0;
    mbar_init(smem_u32(&full[0]), 1);
    mbar_init(smem_u32(&full[1]), 1);
    mbar_fence_init();
    tma_prefetch_desc(&tmX);
  }
  __syncthreads();
  if (tid < 32) {
    issue(t0, 0);
    issued[0] = 1;
  }
  const int cp = tid % TPP, strip = tid / TPP;
  const int lx0 = strip * RX;  // first output column of the strip inside the tile
  int key = -1;
  float w[K][K][CPT];
  float bias[CPT];
  int i = 0;
  for (int t = t0; t < t1; t++, i++) {
    const int b = i & 1;
    if (tid < 32 && t + 1 < t1) {
      // buffer b^1 was last read by tile i-1, finished by every thread before the closing barrier
      issue(t + 1, b ^ 1);
      issued[b ^ 1]++;
    }
    int n, slab, oy0, ox0;
    decode(t, n, slab, oy0, ox0);
    const int c = slab * CS + CPT * cp;
    if (n * slabs + slab != key) {
      key = n * slabs + slab;
#pragma unroll
      for (int q = 0; q < CPT; q++) {
        const float sc = a.in_scale ? __ldg(a.in_scale + (int64_t)n * a.c + c + q) : 1.0f;
#pragma unroll
        for (int ky = 0; ky < K; ky++)
#pragma unroll
          for (int kx = 0; kx < K; kx++) w[ky][kx][q] = __ldg(a.w + (int64_t)(ky * K + kx) * a.c + c + q) * sc;
        bias[q] = __ldg(a.bias + c + q);
      }
    }
    const bool ok = mbar_wait(smem_u32(&full[b]), (uint32_t)(i >> 1) & 1u, a.err, SDX_DEV_WAIT_FULL, &abort_flag);
    if (__syncthreads_or(!ok)) break;
    const uint8_t* sp = dsm + (size_t)b * buf_bytes + (lx0 * CS + CPT * cp) * 2;
    float acc[K][RX][CPT];
#pragma unroll
    for (int sl = 0; sl < K; sl++)
#pragma unroll
      for (int r = 0; r < RX; r++)
#pragma unroll
        for (int q = 0; q < CPT; q++) acc[sl][r][q] = bias[q];
    const int ncols = min(RX, a.ow - (ox0 + lx0));  // <= 0: strip past the right edge, nothing stored
    const int64_t row_step = (int64_t)a.ow * a.c;
    int64_t base = (((int64_t)n * a.oh + oy0) * a.ow + ox0 + lx0) * a.c + c;  // output row oy0
    // prologue: input rows 0 .. K-2 feed kernel rows 0 .. iy (output row iy - ky, slot iy - ky)
    static_for<0, K - 1>([&](auto ic) {
      constexpr int iy = decltype(ic)::value;
      dw_row<K, RX, CPT, PXB, 0, iy, iy>(sp + iy * ROWB, acc, w);
    });
    // steady state: groups of K input rows; input row K-1 + g*K + u feeds every kernel row and
    // finishes output row g*K + u (slot u)
    const int groups = (TH - K + 1) / K;
    const uint8_t* gp = sp + (K - 1) * ROWB;
    int oy = oy0;
    for (int g = 0; g < groups; g++) {
      static_for<0, K>([&](auto ic) {
        constexpr int u = decltype(ic)::value;
        dw_row<K, RX, CPT, PXB, 0, K - 1, K - 1 + u>(gp + u * ROWB, acc, w);
        dw_store_row<ACT, K, RX, CPT, u>(a, acc, bias, oy + u, base + u * row_step, ncols);
      });
      gp += K * ROWB;
      oy += K;
      base += K * row_step;
    }
    // tail: input row TH + e (e = 0 .. K-2, TH = -1 mod K) feeds kernel rows e+1 .. K-1 and
    // finishes output row TH - K + 1 + e (slot e)
    static_for<0, K - 1>([&](auto ic) {
      constexpr int e = decltype(ic)::value;
      dw_row<K, RX, CPT, PXB, e + 1, K - 1, K - 1 + e>(gp + e * ROWB, acc, w);
      dw_store_row<ACT, K, RX, CPT, e>(a, acc, bias, oy + e, base + e * row_step, ncols);
    });
    __syncthreads();
  }
  // wind-down (only after an abort can a copy still be in flight): drain every issued copy
  if (tid < 32) {
    for (int b = 0; b < 2; b++)
      if (issued[b] > 0) mbar_wait_drain(smem_u32(&full[b]), (issued[b] - 1) & 1u, a.err, SDX_DEV_WAIT_DRAIN);
  }
}

constexpr int DW_SLIDE_RX = 5;

// Sliding-window launch for stride-1 layers with 16, 32 or a multiple of 64 channels, K in {3, 5}:
// a tile is 256 / TPP strips of RX columns wide and TH rows high, TH = K*m - 1 chosen so that two
// CTAs (each double-buffered) fit on an SM and the rows loaded per column band
// (tiles x (TH + K - 1)) are fewest.
template <int ACT, int K, int CS>
static bool dw_slide_launch_cs(const DwArgs& a, cudaStream_t st) {
  constexpr int RX = DW_SLIDE_RX, CPT = 2;
  constexpr int TPP = CS / CPT, TW = RX * (256 / TPP), IWt = TW + K - 1;
  static_assert(IWt <= 256, "TMA box width");
  const size_t row_bytes = (size_t)IWt * CS * 2;
  const size_t buf_cap = 54 * 1024;  // two CTAs per SM, two buffers each
  const int ih_max = (int)std::min<size_t>(buf_cap / row_bytes, 256);
  int TH = 0, best = INT32_MAX;
  for (int th = K - 1; th + K - 1 <= ih_max; th += K) {
    const int rows = (a.oh + th - 1) / th * (th + K - 1);
    if (rows <= best) {
      best = rows;
      TH = th;
    }
  }
  if (TH < K - 1 || TH == 0) return false;
  const int IHt = TH + K - 1;
  const size_t tile_bytes = (size_t)IHt * row_bytes;
  const size_t smem = 128 + 2 * ((tile_bytes + 127) & ~(size_t)127) + 16;
  PFN_encodeTiled enc = get_encode_tiled();
  if (!enc) return false;
  CUtensorMap map;
  const cuuint64_t dims[4] = {(cuuint64_t)a.c, (cuuint64_t)a.iw, (cuuint64_t)a.ih, (cuuint64_t)a.batch};
  const cuuint64_t strides[3] = {(cuuint64_t)a.c * 2, (cuuint64_t)a.iw * a.c * 2, (cuuint64_t)a.ih * a.iw * a.c * 2};
  const cuuint32_t box[4] = {(cuuint32_t)CS, (cuuint32_t)IWt, (cuuint32_t)IHt, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<__half*>(a.x), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  static SmemAttr attr{};
  if (raise_smem_limit(attr, (const void*)dw_slide_kernel<ACT, K, RX, CPT, CS>, 120 * 1024,
                       "cudaFuncSetAttribute(dw_slide)"))
    return false;
  const int tiles_x = (a.ow + TW - 1) / TW, tiles_y = (a.oh + TH - 1) / TH;
  const int slabs = a.c / CS;
  const int64_t total = (int64_t)a.batch * slabs * tiles_x * tiles_y;
  if (total <= 0 || total > INT32_MAX) return false;
  int dev = 0, per_sm = 1;
  cudaGetDevice(&dev);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, dw_slide_kernel<ACT, K, RX, CPT, CS>, 256, smem);
  const int grid = (int)std::min<int64_t>(total, (int64_t)num_sms(dev) * std::max(1, per_sm));
  dw_slide_kernel<ACT, K, RX, CPT, CS><<<grid, 256, smem, st>>>(map, a, TH, tiles_x, tiles_y, slabs, (int)total);
  return true;
}

// ---- stride-2 sliding-window form: the same strips and ring, with input row iy feeding output
// rows (iy - ky) / 2 for the kernel rows ky of iy's parity. The ring holds R = ceil(K / 2) output
// rows; the row walk is unrolled by 2R so that every slot is compile-time (the tile's first input
// row is a multiple of 2R); rows outside the tile are skipped by warp-uniform range checks.
template <int ACT, int K, int RX, int CPT, int CS>
__global__ void __launch_bounds__(256, 2) dw_slide2_kernel(const __grid_constant__ CUtensorMap tmX, DwArgs a, int TH,
                                                           int tiles_x, int tiles_y, int slabs, int total) {
  constexpr int R = (K + 1) / 2;         // ring rows
  constexpr int P = 2 * R;               // unroll period of the input-row walk
  constexpr int NX = 2 * RX + K - 2;     // input pixels per strip row
  constexpr int TPP = CS / CPT;
  constexpr int TW = RX * (256 / TPP);
  constexpr int IWt = 2 * TW + K - 2;
  constexpr int PXB = CS * 2;
  constexpr int ROWB = IWt * PXB;
  extern __shared__ uint8_t dsm_raw[];
  uint8_t* dsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 127) & ~uintptr_t(127));
  const int IHt = 2 * TH + K - 2;
  const uint32_t tile_bytes = (uint32_t)IHt * ROWB;
  const uint32_t buf_bytes = (tile_bytes + 127u) & ~127u;
  uint64_t* full = reinterpret_cast<uint64_t*>(dsm + 2 * buf_bytes);
  __shared__ int abort_flag;
  const int tid = threadIdx.x;
  const int per = (total + gridDim.x - 1) / gridDim.x;
  const int t0 = blockIdx.x * per, t1 = min(total, t0 + per);
  if (t0 >= t1) return;
  const int tiles_per_img = tiles_x * tiles_y;
  auto decode = [&](int t, int& n, int& slab, int& oy0, int& ox0) {
    n = t / (slabs * tiles_per_img);
    const int r = t - n * slabs * tiles_per_img;
    slab = r / tiles_per_img;
    const int q = r - slab * tiles_per_img;
    const int ty = q / tiles_x;
    oy0 = ty * TH;
    ox0 = (q - ty * tiles_x) * TW;
  };
  // warp 0 issues the tile copies warp-uniformly from its elected lane
  uint32_t ld0 = 0;
  if (tid < 32) ld0 = elect_leader();
  auto issue = [&](int t, int b) {
    int n, slab, oy0, ox0;
    decode(t, n, slab, oy0, ox0);
    const uint32_t bar = smem_u32(&full[b]);
    mbar_arrive_expect_tx_p(ld0, bar, tile_bytes);
    tma_load_4d_p(ld0, smem_u32(dsm + b * buf_bytes), &tmX, bar, slab * CS, 2 * ox0 - a.pl, 2 * oy0 - a.pt, n);
  };
  uint32_t issued[2] = {0, 0};
  if (tid == 0) {
    abort_flag = 0;
    mbar_init(smem_u32(&full[0]), 1);
    mbar_init(smem_u32(&full[1]), 1);
    mbar_fence_init();
    tma_prefetch_desc(&tmX);
  }
  __syncthreads();
  if (tid < 32) {
    issue(t0, 0);
    issued[0] = 1;
  }
  const int cp = tid % TPP, strip = tid / TPP;
  const int lx0 = strip * RX;
  int key = -1;
  float w[K][K][CPT];
  float bias[CPT];
  int i = 0;
  for (int t = t0; t < t1; t++, i++) {
    const int b = i & 1;
    if (tid < 32 && t + 1 < t1) {
      issue(t + 1, b ^ 1);
      issued[b ^ 1]++;
    }
    int n, slab, oy0, ox0;
    decode(t, n, slab, oy0, ox0);
    const int c = slab * CS + CPT * cp;
    if (n * slabs + slab != key) {
      key = n * slabs + slab;
#pragma unroll
      for (int q = 0; q < CPT; q++) {
        const float sc = a.in_scale ? __ldg(a.in_scale + (int64_t)n * a.c + c + q) : 1.0f;
#pragma unroll
        for (int ky = 0; ky < K; ky++)
#pragma unroll
          for (int kx = 0; kx < K; kx++) w[ky][kx][q] = __ldg(a.w + (int64_t)(ky * K + kx) * a.c + c + q) * sc;
        bias[q] = __ldg(a.bias + c + q);
      }
    }
    const bool ok = mbar_wait(smem_u32(&full[b]), (uint32_t)(i >> 1) & 1u, a.err, SDX_DEV_WAIT_FULL, &abort_flag);
    if (__syncthreads_or(!ok)) break;
    const uint8_t* sp = dsm + (size_t)b * buf_bytes + (2 * lx0 * CS + CPT * cp) * 2;
    float acc[R][RX][CPT];
#pragma unroll
    for (int sl = 0; sl < R; sl++)
#pragma unroll
      for (int r = 0; r < RX; r++)
#pragma unroll
        for (int q = 0; q < CPT; q++) acc[sl][r][q] = bias[q];
    const int ncols = min(RX, a.ow - (ox0 + lx0));
    const int64_t row_step = (int64_t)a.ow * a.c;
    const int64_t base0 = (((int64_t)n * a.oh + oy0) * a.ow + ox0 + lx0) * a.c + c;
    for (int iy0 = 0; iy0 < IHt; iy0 += P) {
      static_for<0, P>([&](auto ic) {
        constexpr int u = decltype(ic)::value;
        const int iy = iy0 + u;
        if (iy < IHt) {
          float xf[NX][CPT];
          const uint8_t* rowp = sp + (size_t)iy * ROWB;
#pragma unroll
          for (int j = 0; j < NX; j++) dw_load_px<CPT>(rowp + j * PXB, xf[j]);
          static_for<0, K>([&](auto kc) {
            constexpr int ky = decltype(kc)::value;
            if constexpr (((u - ky) & 1) == 0) {
              const int o = (iy - ky) / 2;  // iy - ky is even here
              if (iy >= ky && o < TH) {
                constexpr int sl = (((u - ky) / 2) % R + R) % R;
#pragma unroll
                for (int r = 0; r < RX; r++)
#pragma unroll
                  for (int kx = 0; kx < K; kx++) fma_px<CPT>(acc[sl][r], xf[2 * r + kx], w[ky][kx]);
              }
            }
          });
          if constexpr (((u - (K - 1)) & 1) == 0) {
            // output row (iy - K + 1) / 2 has had its last input row
            if (iy >= K - 1) {
              const int o = (iy - (K - 1)) / 2;
              if (o < TH) {
                constexpr int sl = (((u - (K - 1)) / 2) % R + R) % R;
                dw_store_row<ACT, R, RX, CPT, sl>(a, acc, bias, oy0 + o, base0 + o * row_step, ncols);
              }
            }
          }
        }
      });
    }
    __syncthreads();
  }
  if (tid < 32) {
    for (int b = 0; b < 2; b++)
      if (issued[b] > 0) mbar_wait_drain(smem_u32(&full[b]), (issued[b] - 1) & 1u, a.err, SDX_DEV_WAIT_DRAIN);
  }
}

template <int ACT, int K, int CS>
static bool dw_slide2_launch_cs(const DwArgs& a, cudaStream_t st) {
  constexpr int RX = DW_SLIDE_RX, CPT = K <= 3 ? 2 : 1;
  constexpr int TPP = CS / CPT, TW = RX * (256 / TPP), IWt = 2 * TW + K - 2;
  if constexpr (IWt > 256) {
    return false;
  } else {
    const size_t row_bytes = (size_t)IWt * CS * 2;
    const size_t buf_cap = 54 * 1024;
    const int ih_max = (int)std::min<size_t>(buf_cap / row_bytes, 256);
    const int th_max = (ih_max - (K - 2)) / 2;
    if (th_max < 1) return false;
    int TH = th_max, best = INT32_MAX;
    for (int th = th_max; th >= 1; th--) {
      const int rows = (a.oh + th - 1) / th * (2 * th + K - 2);
      if (rows < best) {
        best = rows;
        TH = th;
      }
    }
    const int IHt = 2 * TH + K - 2;
    const size_t tile_bytes = (size_t)IHt * row_bytes;
    const size_t smem = 128 + 2 * ((tile_bytes + 127) & ~(size_t)127) + 16;
    PFN_encodeTiled enc = get_encode_tiled();
    if (!enc) return false;
    CUtensorMap map;
    const cuuint64_t dims[4] = {(cuuint64_t)a.c, (cuuint64_t)a.iw, (cuuint64_t)a.ih, (cuuint64_t)a.batch};
    const cuuint64_t strides[3] = {(cuuint64_t)a.c * 2, (cuuint64_t)a.iw * a.c * 2,
                                   (cuuint64_t)a.ih * a.iw * a.c * 2};
    const cuuint32_t box[4] = {(cuuint32_t)CS, (cuuint32_t)IWt, (cuuint32_t)IHt, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<__half*>(a.x), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return false;
    static SmemAttr attr{};
    if (raise_smem_limit(attr, (const void*)dw_slide2_kernel<ACT, K, RX, CPT, CS>, 120 * 1024,
                         "cudaFuncSetAttribute(dw_slide2)"))
      return false;
    const int tiles_x = (a.ow + TW - 1) / TW, tiles_y = (a.oh + TH - 1) / TH;
    const int slabs = a.c / CS;
    const int64_t total = (int64_t)a.batch * slabs * tiles_x * tiles_y;
    if (total <= 0 || total > INT32_MAX) return false;
    int dev = 0, per_sm = 1;
    cudaGetDevice(&dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, dw_slide2_kernel<ACT, K, RX, CPT, CS>, 256, smem);
    const int grid = (int)std::min<int64_t>(total, (int64_t)num_sms(dev) * std::max(1, per_sm));
    dw_slide2_kernel<ACT, K, RX, CPT, CS><<<grid, 256, smem, st>>>(map, a, TH, tiles_x, tiles_y, slabs, (int)total);
    return true;
  }
}

template <int ACT, int K>
static bool dw_slide2_launch_t(const DwArgs& a, cudaStream_t st) {
  if constexpr (K != 3 && K != 5) {
    return false;
  } else {
    if ((reinterpret_cast<uintptr_t>(a.x) & 15u) || (reinterpret_cast<uintptr_t>(a.y) & 3u)) return false;
    if (a.add && (reinterpret_cast<uintptr_t>(a.add) & 3u)) return false;
    if (a.c == 32) return dw_slide2_launch_cs<ACT, K, 32>(a, st);
    if (a.c % 64 == 0) return dw_slide2_launch_cs<ACT, K, 64>(a, st);
    return false;
  }
}

template <int ACT, int K>
static bool dw_slide_launch_t(const DwArgs& a, cudaStream_t st) {
  if constexpr (K != 3 && K != 5) {
    return false;
  } else {
    if ((reinterpret_cast<uintptr_t>(a.x) & 15u) || (reinterpret_cast<uintptr_t>(a.y) & 3u)) return false;
    if (a.add && (reinterpret_cast<uintptr_t>(a.add) & 3u)) return false;
    if (a.c == 16) return dw_slide_launch_cs<ACT, K, 16>(a, st);
    if (a.c == 32) return dw_slide_launch_cs<ACT, K, 32>(a, st);
    if (a.c % 64 == 0) return dw_slide_launch_cs<ACT, K, 64>(a, st);
    return false;
  }
}

// Strip length: 8 outputs per thread for stride-1 layers on maps of at least 64 x 64 (fewer
// shared-memory reads per output; measured 1.13-1.26x faster there), else 4 (taller tiles of the
// 8-output form waste rows on small maps, and stride 2 needs the registers).
template <int ACT, int K, int S>
static bool dw_tma_pick(const DwArgs& a, cudaStream_t st) {
  if constexpr (S == 1) {
    if (dw_slide_launch_t<ACT, K>(a, st)) return true;
    if (a.oh >= 64 && a.ow >= 64) return dw_tma_launch_t<ACT, K, S, 8>(a, st);
  } else if constexpr (S == 2) {
    if (dw_slide2_launch_t<ACT, K>(a, st)) return true;
  }
  return dw_tma_launch_t<ACT, K, S, 4>(a, st);
}

template <int ACT>
static bool dw_dispatch_ks(const DwArgs& a, cudaStream_t st) {
#define SDX_DW_CASE(KK, SS)                                   \
  if (a.kh == KK && a.kw == KK && a.sh == SS && a.sw == SS) { \
    return dw_tma_pick<ACT, KK, SS>(a, st) || dw_launch_t<ACT, KK, SS>(a, st); \
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
static bool stem_launch_t(const DirectArgs& a, cudaStream_t st) {
  const int TH = 8, TW = 32;
  const int IWt = (TW - 1) * S + K, IHt = (TH - 1) * S + K;
  const size_t smem = sizeof(float) * ((size_t)K * K * a.ic * a.oc + (size_t)a.ic * IHt * IWt);
  static SmemAttr attr{};
  if (raise_smem_limit(attr, (const void*)stem_tiled_kernel<ACT, K, S>, 96 * 1024, "cudaFuncSetAttribute(stem_tiled)"))
    return false;
  const int tiles_x = (a.ow + TW - 1) / TW, tiles_y = (a.oh + TH - 1) / TH;
  dim3 grid(tiles_x * tiles_y, a.batch);
  stem_tiled_kernel<ACT, K, S><<<grid, 256, smem, st>>>(a, TH, TW, tiles_x);
  return true;
}

// ---- persistent, TMA-fed stem for the graph-input conv: fp32 NCHW input, IC = 3, OC = 16, 3x3,
// stride 2 (the det model's first conv; the NCHW -> NHWC relayout and fp16 rounding of its output
// happen on the way out). Each CTA walks a contiguous range of 16 x 64 output tiles; thread 0
// prefetches the next tile's three input planes (+ halo, zero fill = padding) with one TMA load while
// all threads compute the current tile. Thread = 4 horizontally adjacent outputs x 16 channels:
// per input row it reads 9 floats once, per tap the 16 weights once (shared-memory broadcasts).
// The TMA box starts 3 columns left of the window (pad 1 + 3 = 4 floats) so its x coordinate stays
// 16-byte aligned; buffers are 1024-byte aligned.
constexpr int STEM_TH = 16, STEM_TW = 64, STEM_R = 4;
constexpr int STEM_IH = (STEM_TH - 1) * 2 + 3;           // 33 input rows
constexpr int STEM_IW = ((STEM_TW - 1) * 2 + 3 + 3 + 3) / 4 * 4;  // 132 columns (3 of alignment)

// One 16 x 64 stem output tile from the planar fp32 input tile in shared memory ([3][33][132];
// output column j's window starts at column 2j + 3). A warp covers 32 consecutive output columns of
// 4 output rows: thread = one column x 4 rows x 16 channels. Per (input channel, kernel row, output
// row) it reads its 3 window values with two 8-byte loads at even columns (2j + 2, 2j + 4), so a
// warp's load is 256 contiguous bytes (conflict-free; one thread per 4 adjacent outputs read with
// an 8-word stride, 4- to 8-way bank conflicts); the 16 weights of a tap are shared-memory
// broadcasts.
template <int ACT>
__device__ __forceinline__ void stem_tile_compute(const DirectArgs& a, const float* tile, const float* sw, const float* sb,
                                                  int n, int oy0, int ox0, int tid) {
  constexpr int IC = 3, OC = 16, K = 3, RY = 4;
  const int warp = tid >> 5, lane = tid & 31;
  const int j = (warp & 1) * 32 + lane;  // output column inside the tile
  const int r0 = (warp >> 1) * RY;       // first output row inside the tile
  float acc[RY][OC];
#pragma unroll
  for (int r = 0; r < RY; r++)
#pragma unroll
    for (int o = 0; o < OC; o++) acc[r][o] = sb[o];
#pragma unroll
  for (int c = 0; c < IC; c++) {
#pragma unroll
    for (int ky = 0; ky < K; ky++) {
      float xv[RY][K];
#pragma unroll
      for (int r = 0; r < RY; r++) {
        const float* rp = tile + (c * STEM_IH + 2 * (r0 + r) + ky) * STEM_IW + 2 * j + 2;
        const float2 p0 = *reinterpret_cast<const float2*>(rp);
        const float2 p1 = *reinterpret_cast<const float2*>(rp + 2);
        xv[r][0] = p0.y;
        xv[r][1] = p1.x;
        xv[r][2] = p1.y;
      }
#pragma unroll
      for (int kx = 0; kx < K; kx++) {
        const float4* wp = reinterpret_cast<const float4*>(sw + ((ky * K + kx) * IC + c) * OC);
        float wv[OC];
#pragma unroll
        for (int q = 0; q < OC / 4; q++) {
          const float4 w4 = wp[q];
          wv[4 * q] = w4.x; wv[4 * q + 1] = w4.y; wv[4 * q + 2] = w4.z; wv[4 * q + 3] = w4.w;
        }
#pragma unroll
        for (int r = 0; r < RY; r++)
#pragma unroll
          for (int o = 0; o < OC; o++) acc[r][o] = fmaf(xv[r][kx], wv[o], acc[r][o]);
      }
    }
  }
  const int ox = ox0 + j;
  if (ox >= a.ow) return;
#pragma unroll
  for (int r = 0; r < RY; r++) {
    const int oy = oy0 + r0 + r;
    if (oy >= a.oh) break;
    __half* yp = static_cast<__half*>(a.y) + (((int64_t)n * a.oh + oy) * a.ow + ox) * a.y_pix_stride + a.y_ch_off;
#pragma unroll
    for (int h8 = 0; h8 < OC / 8; h8++) {
      uint4 u;
      __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
      for (int q = 0; q < 4; q++)
        h[q] = __floats2half2_rn(act_t<ACT>(acc[r][h8 * 8 + 2 * q]), act_t<ACT>(acc[r][h8 * 8 + 2 * q + 1]));
      reinterpret_cast<uint4*>(yp)[h8] = u;
    }
  }
}

// ---- tensor-core form of the det stem, warp-specialised like the tensor-core conv: warp 0 streams
// the fp32 input tiles (TMA, a ring of buffers), BG groups of four warps build im2col rows of
// 128-pixel M blocks into a ring of shared-memory slots, warp 1 issues the MMAs of each block into a
// ring of TMEM accumulators, DG groups of four warps drain them (bias, activation, fp16 NHWC stores).
// Each group handles every BG-th (DG-th) block: one group per role left each block's work as a
// single latency chain per warp (N=256: 0.64 ms with one of each, 0.45 with two, 0.42 with two
// builder and three drain groups; four builder or four drain groups gain nothing). Every hand-off
// is an mbarrier, so building, MMAs, draining and loading overlap. A row = one output pixel, K = 27
// taps (k = (ky*3 + kx)*3 + c, padded to 32) of fp16-rounded inputs in 64-byte rows under the 64-byte
// swizzle; B = the 16 filters as fp16 hi and lo terms (the same layout), fp32 accumulation.
constexpr int STEM_TC_TH = 8;
constexpr int STEM_TC_IH = 2 * STEM_TC_TH + 1;                   // 17 input rows
constexpr int STEM_TC_NBUF = 5;                                   // input tiles in flight or in use
constexpr int STEM_TC_NB = STEM_TC_TH * STEM_TW / 128;           // 4 M blocks per tile
constexpr int STEM_TC_NA = 4;                                     // im2col slots
constexpr int STEM_TC_NACC = 4;                                   // TMEM accumulators (16 columns each)
constexpr uint32_t STEM_TC_A_BYTES = 128u * 64u;                  // one block's im2col rows
constexpr uint32_t STEM_TC_B_BYTES = 16u * 64u;                   // the filters
constexpr uint32_t STEM_TC_TMEM_COLS = 64u;
constexpr int STEM_TC_BG = 2;                                     // im2col builder groups (4 warps each)
constexpr int STEM_TC_DG = 3;                                     // drain groups (4 warps each)
constexpr int STEM_TC_THREADS = 64 + 128 * (STEM_TC_BG + STEM_TC_DG);
static_assert(STEM_TC_BG <= STEM_TC_NB, "every builder group takes a block of each tile");

// Builds the filter rows as fp16 hi and lo terms (w = hi + lo to ~22 bits; one term leaves a
// weight error common to every pixel, which the det network amplifies past the parity bound): row n,
// column k = tap * 3 + c, swizzled like the A rows; the lo term STEM_TC_B_BYTES after the hi term.
__device__ __forceinline__ void stem_tc_weights(const float* sw, uint32_t b0, int tid, int nthreads) {
  for (int e = tid; e < 16 * 32; e += nthreads) {
    const int n = e >> 5, k = e & 31;
    const float w = k < 27 ? sw[k * 16 + n] : 0.0f;
    const __half h = __float2half_rn(w);
    const __half l = __float2half_rn(w - __half2float(h));
    const uint32_t off = (uint32_t)n * 64u + ((((uint32_t)k >> 3) ^ (((uint32_t)n >> 1) & 3u)) << 4) + ((uint32_t)k & 7u) * 2u;
    asm volatile("st.shared.b16 [%0], %1;" ::"r"(b0 + off), "h"(__half_as_ushort(h)) : "memory");
    asm volatile("st.shared.b16 [%0], %1;" ::"r"(b0 + STEM_TC_B_BYTES + off), "h"(__half_as_ushort(l)) : "memory");
  }
}

// im2col row `row` (0 .. 127) of block `blk` of the staged tile ([3][IH][STEM_IW] fp32, column
// 2j + 3 + kx under tap kx) into the slot at `slot`.
__device__ __forceinline__ void stem_tc_row(const float* tile, uint32_t slot, int blk, int row) {
  const int p = blk * 128 + row;
  const int r = p >> 6, j = p & 63;
  float xs[32];
#pragma unroll
  for (int c = 0; c < 3; c++)
#pragma unroll
    for (int ky = 0; ky < 3; ky++) {
      const float* rp = tile + (c * STEM_TC_IH + 2 * r + ky) * STEM_IW + 2 * j + 2;
      const float2 p0 = *reinterpret_cast<const float2*>(rp);
      const float2 p1 = *reinterpret_cast<const float2*>(rp + 2);
      xs[(ky * 3 + 0) * 3 + c] = p0.y;
      xs[(ky * 3 + 1) * 3 + c] = p1.x;
      xs[(ky * 3 + 2) * 3 + c] = p1.y;
    }
#pragma unroll
  for (int k = 27; k < 32; k++) xs[k] = 0.0f;
  const uint32_t base = slot + (uint32_t)row * 64u;
  const uint32_t xr = ((uint32_t)row >> 1) & 3u;
#pragma unroll
  for (int u = 0; u < 4; u++) {
    uint4 q;
    __half2* h = reinterpret_cast<__half2*>(&q);
#pragma unroll
    for (int i = 0; i < 4; i++) h[i] = __floats2half2_rn(xs[8 * u + 2 * i], xs[8 * u + 2 * i + 1]);
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(base + (((uint32_t)u ^ xr) << 4)), "r"(q.x),
                 "r"(q.y), "r"(q.z), "r"(q.w)
                 : "memory");
  }
}

template <int ACT>
__global__ void __launch_bounds__(STEM_TC_THREADS, 1) stem_tc_kernel(const __grid_constant__ CUtensorMap tmX,
                                                                    DirectArgs a, int tiles_x, int tiles_per_img,
                                                                    int total) {
  constexpr int IC = 3, OC = 16, K = 3;
  constexpr uint32_t kTileBytes = IC * STEM_TC_IH * STEM_IW * 4;
  constexpr uint32_t kBufBytes = (kTileBytes + 1023u) & ~1023u;  // TMA destinations 1024-aligned
  extern __shared__ uint8_t ssm_raw[];
  uint8_t* ssm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ssm_raw) + 1023) & ~uintptr_t(1023));
  float* bufs = reinterpret_cast<float*>(ssm);                                  // [NBUF][IC][IH][IW]
  uint8_t* sA = ssm + STEM_TC_NBUF * kBufBytes;                                 // [NA][128][64 B]
  uint8_t* sB = sA + STEM_TC_NA * STEM_TC_A_BYTES;                              // [2 terms][16][64 B]
  float* sw = reinterpret_cast<float*>(sB + 2 * STEM_TC_B_BYTES);               // [K*K][IC][OC]
  float* sb = sw + K * K * IC * OC;                                             // [OC]
  uint64_t* tfull = reinterpret_cast<uint64_t*>(sb + OC);                       // [NBUF] tile landed
  uint64_t* tempty = tfull + STEM_TC_NBUF;                                      // [NBUF] tile consumed (128)
  uint64_t* afull = tempty + STEM_TC_NBUF;                                      // [NA] rows built (128)
  uint64_t* aempty = afull + STEM_TC_NA;                                        // [NA] rows read (commit)
  uint64_t* accf = aempty + STEM_TC_NA;                                         // [NACC] MMAs done (commit)
  uint64_t* acce = accf + STEM_TC_NACC;                                         // [NACC] drained (128)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce + STEM_TC_NACC);
  __shared__ int abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int per = (total + gridDim.x - 1) / gridDim.x;
  const int t0 = blockIdx.x * per, t1 = min(total, t0 + per);
  if (t0 >= t1) return;
  const int ntiles = t1 - t0;
  auto decode = [&](int t, int& n, int& oy0, int& ox0) {
    n = t / tiles_per_img;
    const int q = t - n * tiles_per_img;
    const int ty = q / tiles_x;
    oy0 = ty * STEM_TC_TH;
    ox0 = (q - ty * tiles_x) * STEM_TW;
  };
  for (int i = tid; i < K * K * IC * OC; i += blockDim.x) sw[i] = __ldg(a.w + i);
  for (int i = tid; i < OC; i += blockDim.x) sb[i] = a.bias ? __ldg(a.bias + i) : 0.0f;
  if (tid == 0) {
    abort_flag = 0;
    for (int i = 0; i < STEM_TC_NBUF; i++) {
      mbar_init(smem_u32(&tfull[i]), 1);
      mbar_init(smem_u32(&tempty[i]), 128 * STEM_TC_BG);
    }
    for (int i = 0; i < STEM_TC_NA; i++) {
      mbar_init(smem_u32(&afull[i]), 128);
      mbar_init(smem_u32(&aempty[i]), 1);
    }
    for (int i = 0; i < STEM_TC_NACC; i++) {
      mbar_init(smem_u32(&accf[i]), 1);
      mbar_init(smem_u32(&acce[i]), 128);
    }
    mbar_fence_init();
    tma_prefetch_desc(&tmX);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), STEM_TC_TMEM_COLS);
    tmem_relinquish();
  }
  __syncthreads();
  stem_tc_weights(sw, smem_u32(sB), tid, blockDim.x);
  fence_async_smem_cta();  // the filter rows are read by the tensor cores (async proxy)
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t ld = elect_leader();  // warp-uniform issue from the elected lane (warps 0 and 1)
  const int nblk = ntiles * STEM_TC_NB;
  uint32_t issued[STEM_TC_NBUF] = {};  // warp 0: copies per buffer
  int mma_done = 0;             // warp 1: blocks whose MMAs were committed

  if (warp == 0) {
    // ---- input tiles
    for (int i = 0; i < ntiles; i++) {
      const int b = i % STEM_TC_NBUF, use = i / STEM_TC_NBUF;
      if (use > 0 && !mbar_wait(smem_u32(&tempty[b]), (uint32_t)(use - 1) & 1u, a.err, SDX_DEV_WAIT_EMPTY,
                                &abort_flag))
        break;
      int n, oy0, ox0;
      decode(t0 + i, n, oy0, ox0);
      const uint32_t bar = smem_u32(&tfull[b]);
      mbar_arrive_expect_tx_p(ld, bar, kTileBytes);
      tma_load_4d_p(ld, smem_u32(bufs + b * (kBufBytes / 4)), &tmX, bar, ox0 * 2 - a.pl - 3, oy0 * 2 - a.pt, 0, n);
      issued[b]++;
    }
  } else if (warp == 1) {
    // ---- MMAs: two k-steps per block into accumulator g % NACC
    constexpr uint32_t idesc = umma_idesc_f16(128, 16);
    const uint64_t bd = umma_desc_kmajor(smem_u32(sB), 64);
    for (int g = 0; g < nblk; g++) {
      const int sl = g % STEM_TC_NA, ac = g % STEM_TC_NACC;
      bool ok = mbar_wait(smem_u32(&afull[sl]), (uint32_t)(g / STEM_TC_NA) & 1u, a.err, SDX_DEV_WAIT_FULL, &abort_flag);
      if (ok && g >= STEM_TC_NACC)
        ok = mbar_wait(smem_u32(&acce[ac]), (uint32_t)(g / STEM_TC_NACC - 1) & 1u, a.err, SDX_DEV_WAIT_ACC_EMPTY,
                       &abort_flag);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const uint64_t ad = umma_desc_kmajor(smem_u32(sA) + (uint32_t)sl * STEM_TC_A_BYTES, 64);
      const uint32_t d = tmem + (uint32_t)(16 * ac);
      const uint64_t bl = bd + (STEM_TC_B_BYTES >> 4);  // the lo term
      umma_f16_p(ld, d, ad, bd, idesc, 0u);
      umma_f16_p(ld, d, ad, bl, idesc, 1u);
      umma_f16_p(ld, d, ad + 2u, bd + 2u, idesc, 1u);
      umma_f16_p(ld, d, ad + 2u, bl + 2u, idesc, 1u);
      tc_commit_p(ld, smem_u32(&aempty[sl]));
      tc_commit_p(ld, smem_u32(&accf[ac]));
      mma_done = g + 1;
    }
  } else if (warp < 2 + 4 * STEM_TC_BG) {
    // ---- im2col rows: BG groups of four warps take the blocks of each tile round-robin; thread =
    // one row of its group's blocks
    const int bg = (warp - 2) >> 2, row = tid - 64 - 128 * bg;
    for (int i = 0; i < ntiles; i++) {
      const int b = i % STEM_TC_NBUF;
      bool ok = mbar_wait(smem_u32(&tfull[b]), (uint32_t)(i / STEM_TC_NBUF) & 1u, a.err, SDX_DEV_WAIT_FULL,
                          &abort_flag);
      if (!ok) break;
      const float* tile = bufs + b * (kBufBytes / 4);
      for (int blk = bg; blk < STEM_TC_NB && ok; blk += STEM_TC_BG) {
        const int g = i * STEM_TC_NB + blk, sl = g % STEM_TC_NA;
        if (g >= STEM_TC_NA)
          ok = mbar_wait(smem_u32(&aempty[sl]), (uint32_t)(g / STEM_TC_NA - 1) & 1u, a.err, SDX_DEV_WAIT_EMPTY,
                         &abort_flag);
        if (!ok) break;
        stem_tc_row(tile, smem_u32(sA) + (uint32_t)sl * STEM_TC_A_BYTES, blk, row);
        fence_async_smem_cta();
        mbar_arrive(smem_u32(&afull[sl]));
      }
      if (!ok) break;
      mbar_arrive(smem_u32(&tempty[b]));
    }
  } else {
    // ---- drain: DG groups of four warps take the blocks round-robin (each block's TMEM load, bias,
    // activation and stores are one latency chain per warp); warp w reads TMEM lanes 32 (w % 4) ..
    const int q = warp & 3, dg = (warp - 2 - 4 * STEM_TC_BG) >> 2;
    for (int g = dg; g < nblk; g += STEM_TC_DG) {
      const int ac = g % STEM_TC_NACC;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&accf[ac]), (uint32_t)(g / STEM_TC_NACC) & 1u, a.err,
                                                        SDX_DEV_WAIT_ACC_FULL, &abort_flag));
      if (!ok) break;
      tc_fence_after();
      float v[16];
      tmem_ld16_issue(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(16 * ac), v);
      tmem_wait_ld();
      tmem_ld_wait16(v);
      tc_fence_before();
      mbar_arrive(smem_u32(&acce[ac]));
      const int i = g / STEM_TC_NB, blk = g - i * STEM_TC_NB;
      int n, oy0, ox0;
      decode(t0 + i, n, oy0, ox0);
      const int p = blk * 128 + q * 32 + lane;
      const int oy = oy0 + (p >> 6), ox = ox0 + (p & 63);
      if (oy < a.oh && ox < a.ow) {
        __half* yp = static_cast<__half*>(a.y) + (((int64_t)n * a.oh + oy) * a.ow + ox) * a.y_pix_stride + a.y_ch_off;
#pragma unroll
        for (int h8 = 0; h8 < 2; h8++) {
          uint4 u;
          __half2* hh = reinterpret_cast<__half2*>(&u);
#pragma unroll
          for (int k = 0; k < 4; k++) {
            const int o = h8 * 8 + 2 * k;
            hh[k] = __floats2half2_rn(act_t<ACT>(v[o] + sb[o]), act_t<ACT>(v[o + 1] + sb[o + 1]));
          }
          reinterpret_cast<uint4*>(yp)[h8] = u;
        }
      }
    }
  }
  // wind-down: copies in flight must land and committed MMAs finish before smem and TMEM go away
  if (warp == 0) {
    for (int b = 0; b < STEM_TC_NBUF; b++)
      if (issued[b] > 0) mbar_wait_drain(smem_u32(&tfull[b]), (issued[b] - 1) & 1u, a.err, SDX_DEV_WAIT_DRAIN);
  }
  if (warp == 1 && mma_done > 0) {
    const int g = mma_done - 1;
    mbar_wait_drain(smem_u32(&accf[g % STEM_TC_NACC]), (uint32_t)(g / STEM_TC_NACC) & 1u, a.err, SDX_DEV_WAIT_DRAIN);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, STEM_TC_TMEM_COLS);
  }
}

template <int ACT>
__global__ void __launch_bounds__(256, 2) stem_tma_kernel(const __grid_constant__ CUtensorMap tmX, DirectArgs a,
                                                       int tiles_x, int tiles_per_img, int total) {
  constexpr int IC = 3, OC = 16, K = 3;
  constexpr uint32_t kTileBytes = IC * STEM_IH * STEM_IW * 4;
  constexpr uint32_t kBufBytes = (kTileBytes + 1023u) & ~1023u;  // TMA destinations 1024-aligned
  extern __shared__ uint8_t ssm_raw[];
  uint8_t* ssm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ssm_raw) + 1023) & ~uintptr_t(1023));
  float* bufs = reinterpret_cast<float*>(ssm);                                   // [2][IC][IH][IW]
  float* sw = reinterpret_cast<float*>(ssm + 2 * kBufBytes);                     // [K*K][IC][OC]
  float* sb = sw + K * K * IC * OC;                                              // [OC]
  uint64_t* full = reinterpret_cast<uint64_t*>(sb + OC);
  __shared__ int abort_flag;
  const int tid = threadIdx.x;
  const int per = (total + gridDim.x - 1) / gridDim.x;
  const int t0 = blockIdx.x * per, t1 = min(total, t0 + per);
  if (t0 >= t1) return;
  auto decode = [&](int t, int& n, int& oy0, int& ox0) {
    n = t / tiles_per_img;
    const int q = t - n * tiles_per_img;
    const int ty = q / tiles_x;
    oy0 = ty * STEM_TH;
    ox0 = (q - ty * tiles_x) * STEM_TW;
  };
  // warp 0 issues the tile copies warp-uniformly from its elected lane
  uint32_t ld0 = 0;
  if (tid < 32) ld0 = elect_leader();
  auto issue = [&](int t, int b) {
    int n, oy0, ox0;
    decode(t, n, oy0, ox0);
    const uint32_t bar = smem_u32(&full[b]);
    mbar_arrive_expect_tx_p(ld0, bar, kTileBytes);
    tma_load_4d_p(ld0, smem_u32(bufs + b * (kBufBytes / 4)), &tmX, bar, ox0 * 2 - a.pl - 3, oy0 * 2 - a.pt, 0, n);
  };
  uint32_t issued[2] = {0, 0};
  for (int i = tid; i < K * K * IC * OC; i += blockDim.x) sw[i] = __ldg(a.w + i);
  for (int i = tid; i < OC; i += blockDim.x) sb[i] = a.bias ? __ldg(a.bias + i) : 0.0f;
  if (tid == 0) {
    abort_flag = 0;
    mbar_init(smem_u32(&full[0]), 1);
    mbar_init(smem_u32(&full[1]), 1);
    mbar_fence_init();
    tma_prefetch_desc(&tmX);
  }
  __syncthreads();
  if (tid < 32) {
    issue(t0, 0);
    issued[0] = 1;
  }
  int i = 0;
  for (int t = t0; t < t1; t++, i++) {
    const int b = i & 1;
    if (tid < 32 && t + 1 < t1) {
      issue(t + 1, b ^ 1);
      issued[b ^ 1]++;
    }
    int n, oy0, ox0;
    decode(t, n, oy0, ox0);
    const bool ok = mbar_wait(smem_u32(&full[b]), (uint32_t)(i >> 1) & 1u, a.err, SDX_DEV_WAIT_FULL, &abort_flag);
    if (__syncthreads_or(!ok)) break;
    const float* tile = bufs + b * (kBufBytes / 4);
    stem_tile_compute<ACT>(a, tile, sw, sb, n, oy0, ox0, tid);
    __syncthreads();
  }
  if (tid < 32) {
    for (int b = 0; b < 2; b++)
      if (issued[b] > 0) mbar_wait_drain(smem_u32(&full[b]), (issued[b] - 1) & 1u, a.err, SDX_DEV_WAIT_DRAIN);
  }
}

template <int ACT>
static bool stem_tma_launch_t(const DirectArgs& a, cudaStream_t st) {
  PFN_encodeTiled enc = get_encode_tiled();
  if (!enc) return false;
  CUtensorMap map;
  const cuuint64_t dims[4] = {(cuuint64_t)a.iw, (cuuint64_t)a.ih, 3, (cuuint64_t)a.batch};
  const cuuint64_t strides[3] = {(cuuint64_t)a.iw * 4, (cuuint64_t)a.ih * a.iw * 4, (cuuint64_t)3 * a.ih * a.iw * 4};
  const cuuint32_t box[4] = {(cuuint32_t)STEM_IW, (cuuint32_t)STEM_IH, 3, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void*>(a.x), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  const size_t buf = ((size_t)3 * STEM_IH * STEM_IW * 4 + 1023) & ~(size_t)1023;
  const size_t smem = 1024 + 2 * buf + sizeof(float) * (9 * 3 * 16 + 16) + 16;
  static SmemAttr attr{};
  if (raise_smem_limit(attr, (const void*)stem_tma_kernel<ACT>, (int)smem, "cudaFuncSetAttribute(stem_tma)"))
    return false;
  const int tiles_x = (a.ow + STEM_TW - 1) / STEM_TW, tiles_y = (a.oh + STEM_TH - 1) / STEM_TH;
  const int64_t total = (int64_t)a.batch * tiles_x * tiles_y;
  if (total <= 0 || total > INT32_MAX) return false;
  int dev = 0, per_sm = 1;
  cudaGetDevice(&dev);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, stem_tma_kernel<ACT>, 256, smem);
  const int grid = (int)std::min<int64_t>(total, (int64_t)num_sms(dev) * std::max(1, per_sm));
  stem_tma_kernel<ACT><<<grid, 256, smem, st>>>(map, a, tiles_x, tiles_x * tiles_y, (int)total);
  return true;
}

// Shared memory of stem_tc_kernel and its launch: one persistent CTA per SM over contiguous tile
// ranges.
template <int ACT>
static bool stem_tc_run(const CUtensorMap& map, const DirectArgs& a, cudaStream_t st) {
  const size_t buf = ((size_t)3 * STEM_TC_IH * STEM_IW * 4 + 1023) & ~(size_t)1023;
  const size_t smem = 1024 + STEM_TC_NBUF * buf + (size_t)STEM_TC_NA * STEM_TC_A_BYTES + 2 * STEM_TC_B_BYTES +
                      sizeof(float) * (9 * 3 * 16 + 16) +
                      sizeof(uint64_t) * (2 * STEM_TC_NBUF + 2 * STEM_TC_NA + 2 * STEM_TC_NACC) + 16;
  static SmemAttr attr{};
  if (raise_smem_limit(attr, (const void*)stem_tc_kernel<ACT>, (int)smem, "cudaFuncSetAttribute(stem_tc)"))
    return false;
  const int tiles_x = (a.ow + STEM_TW - 1) / STEM_TW, tiles_y = (a.oh + STEM_TC_TH - 1) / STEM_TC_TH;
  const int64_t total = (int64_t)a.batch * tiles_x * tiles_y;
  if (total <= 0 || total > INT32_MAX) return false;
  int dev = 0;
  cudaGetDevice(&dev);
  const int grid = (int)std::min<int64_t>(total, (int64_t)num_sms(dev));  // one CTA per SM
  stem_tc_kernel<ACT><<<grid, STEM_TC_THREADS, smem, st>>>(map, a, tiles_x, tiles_x * tiles_y, (int)total);
  return true;
}

template <int ACT>
static bool stem_tc_launch_t(const DirectArgs& a, cudaStream_t st) {
  PFN_encodeTiled enc = get_encode_tiled();
  if (!enc) return false;
  CUtensorMap map;
  const cuuint64_t dims[4] = {(cuuint64_t)a.iw, (cuuint64_t)a.ih, 3, (cuuint64_t)a.batch};
  const cuuint64_t strides[3] = {(cuuint64_t)a.iw * 4, (cuuint64_t)a.ih * a.iw * 4, (cuuint64_t)3 * a.ih * a.iw * 4};
  const cuuint32_t box[4] = {(cuuint32_t)STEM_IW, (cuuint32_t)STEM_TC_IH, 3, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void*>(a.x), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  return stem_tc_run<ACT>(map, a, st);
}

// ---- the det stem fed straight from u8 images (image session): the ImageToTensor normalisation
// (lut, optional R/B swap, replicate placement of the image inside the tensor) runs while the tile
// is filled, so the fp32 NCHW tensor is never written or read. One CTA per 16 x 64 output tile;
// the fill reads 3 bytes per input pixel (plain loads: rows of 3-byte pixels do not meet TMA's
// 16-byte rules) and writes the same planar fp32 tile as the TMA-fed stem, whose compute follows.
template <int ACT>
__global__ void __launch_bounds__(256, 2) stem_image_kernel(ImageArgs im, DirectArgs a, int tiles_x, int tiles_per_img) {
  constexpr int IC = 3, OC = 16, K = 3;
  constexpr int NCOL = (STEM_TW - 1) * 2 + K;  // 129 input columns of a tile
  extern __shared__ float fsm[];
  float* tile = fsm;                              // [IC][STEM_IH][STEM_IW]
  float* sw = tile + IC * STEM_IH * STEM_IW;      // [K*K][IC][OC]
  float* sb = sw + K * K * IC * OC;               // [OC]
  float* lut = sb + OC;                           // [3][256]
  const int tid = threadIdx.x;
  const int t = blockIdx.x;
  const int n = t / tiles_per_img;
  const int q = t - n * tiles_per_img;
  const int ty = q / tiles_x;
  const int oy0 = ty * STEM_TH, ox0 = (q - ty * tiles_x) * STEM_TW;
  for (int i = tid; i < K * K * IC * OC; i += blockDim.x) sw[i] = __ldg(a.w + i);
  for (int i = tid; i < OC; i += blockDim.x) sb[i] = a.bias ? __ldg(a.bias + i) : 0.0f;
  for (int i = tid; i < 3 * 256; i += blockDim.x) lut[i] = __ldg(im.lut + i);
  __syncthreads();
  // tensor row y = oy0*2 - pt + r, column x = ox0*2 - pl + col (conv zero padding outside the
  // tensor); the tensor pixel is image pixel (clamp(y - image top), clamp(x - image left))
  const uint8_t* img = im.src + (int64_t)n * im.img_bytes;
  const int ob = im.swap ? 2 : 0;
  for (int i = tid; i < STEM_IH * NCOL; i += blockDim.x) {
    const int r = i / NCOL, col = i - r * NCOL;
    const int y = oy0 * 2 - a.pt + r, x = ox0 * 2 - a.pl + col;
    float v0 = 0.0f, v1 = 0.0f, v2 = 0.0f;
    if ((unsigned)y < (unsigned)a.ih && (unsigned)x < (unsigned)a.iw) {
      const int sy = min(max(y - im.pt, 0), im.ih - 1), sx = min(max(x - im.pl, 0), im.iw - 1);
      const uint8_t* px = img + (int64_t)sy * im.stride + (int64_t)sx * im.bpp;
      v0 = lut[px[ob]];
      v1 = lut[256 + px[1]];
      v2 = lut[512 + px[2 - ob]];
    }
    float* d = tile + r * STEM_IW + col + 3;
    d[0] = v0;
    d[STEM_IH * STEM_IW] = v1;
    d[2 * STEM_IH * STEM_IW] = v2;
  }
  __syncthreads();
  stem_tile_compute<ACT>(a, tile, sw, sb, n, oy0, ox0, tid);
}

template <int ACT>
static bool stem_image_launch_t(const ImageArgs& im, const DirectArgs& a, cudaStream_t st) {
  const size_t smem = sizeof(float) * ((size_t)3 * STEM_IH * STEM_IW + 9 * 3 * 16 + 16 + 3 * 256);
  static SmemAttr attr{};
  if (raise_smem_limit(attr, (const void*)stem_image_kernel<ACT>, (int)smem, "cudaFuncSetAttribute(stem_image)"))
    return false;
  const int tiles_x = (a.ow + STEM_TW - 1) / STEM_TW, tiles_y = (a.oh + STEM_TH - 1) / STEM_TH;
  stem_image_kernel<ACT><<<a.batch * tiles_x * tiles_y, 256, smem, st>>>(im, a, tiles_x, tiles_x * tiles_y);
  return true;
}

bool stem_image_launch(const ImageArgs& im, const DirectArgs& a, cudaStream_t st) {
  // the det stem shape on an image-session input: 3 -> 16 channels, 3x3 stride 2, fp16 NHWC out
  if (!(a.ic == 3 && a.oc == 16 && a.kh == 3 && a.kw == 3 && a.sh == 2 && a.sw == 2 && !a.add && !a.y_f32 &&
        !a.y_nchw && a.y_pix_stride % 8 == 0 && a.y_ch_off % 8 == 0 &&
        (reinterpret_cast<uintptr_t>(a.y) & 15u) == 0))
    return false;
  if (im.bpp != 3 && im.bpp != 4) return false;
  if (a.ih != im.oh || a.iw != im.ow) return false;  // the conv reads the image session's tensor
  const int64_t tiles = (int64_t)a.batch * ((a.ow + STEM_TW - 1) / STEM_TW) * ((a.oh + STEM_TH - 1) / STEM_TH);
  if (tiles <= 0 || tiles > INT32_MAX) return false;
  switch (a.act) {
    case ACT_HARDSWISH: return stem_image_launch_t<ACT_HARDSWISH>(im, a, st);
    case ACT_RELU: return stem_image_launch_t<ACT_RELU>(im, a, st);
    case ACT_NONE: return stem_image_launch_t<ACT_NONE>(im, a, st);
    default: return false;
  }
}

bool stem_tiled_launch(const DirectArgs& a, cudaStream_t st) {
  // the det stem: fp32 NCHW graph input, 3 -> 16 channels, 3x3 stride 2 (TMA-fed form)
  if (a.ic == 3 && a.oc == 16 && a.kh == 3 && a.kw == 3 && a.sh == 2 && a.sw == 2 && a.x_f32 && a.x_nchw && !a.add &&
      !a.y_f32 && !a.y_nchw && a.y_pix_stride % 8 == 0 && a.y_ch_off % 8 == 0 && a.pl == 1 &&
      (reinterpret_cast<uintptr_t>(a.x) & 15u) == 0 && (a.iw * 4) % 16 == 0 &&
      (reinterpret_cast<uintptr_t>(a.y) & 15u) == 0) {
    bool done = false;
    switch (a.act) {
      case ACT_HARDSWISH: done = stem_tc_launch_t<ACT_HARDSWISH>(a, st) || stem_tma_launch_t<ACT_HARDSWISH>(a, st); break;
      case ACT_RELU: done = stem_tc_launch_t<ACT_RELU>(a, st) || stem_tma_launch_t<ACT_RELU>(a, st); break;
      case ACT_NONE: done = stem_tc_launch_t<ACT_NONE>(a, st) || stem_tma_launch_t<ACT_NONE>(a, st); break;
      default: break;
    }
    if (done) return true;
  }
  if (a.ic > 4 || a.oc % 8 != 0 || a.oc > 64 || a.add || a.y_f32 || a.y_nchw || a.kh != 3 || a.kw != 3 ||
      a.sh != a.sw || (a.sh != 1 && a.sh != 2) || a.batch > 65535 || (a.y_pix_stride % 8) || (a.y_ch_off % 8))
    return false;
  const size_t smem = sizeof(float) * ((size_t)9 * a.ic * a.oc + (size_t)a.ic * (7 * a.sh + 3) * (31 * a.sh + 3));
  if (smem > 96 * 1024) return false;
  switch (a.act) {
#define SDX_STEM_CASE(ACTC)                                               \
  case ACTC:                                                              \
    return a.sh == 1 ? stem_launch_t<ACTC, 3, 1>(a, st) : stem_launch_t<ACTC, 3, 2>(a, st);
    SDX_STEM_CASE(ACT_HARDSWISH)
    SDX_STEM_CASE(ACT_RELU)
    SDX_STEM_CASE(ACT_NONE)
#undef SDX_STEM_CASE
    default: return false;
  }
}

}  // namespace sdx
