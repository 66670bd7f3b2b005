// Bandwidth kernels of the remaining ExecNode kinds and of the reference's built-in fused ops:
//   * elementwise binary with numpy broadcasting (Ops.Elementwise, src/Kernels/Ops.cs:388-441);
//   * SafeDiv: clamp(a / max(b, eps), lo, hi) (SafeDivOp, src/Engine/Fusions/SafeDivOp.cs:14-34,
//     FusedKernels.SafeDiv, src/Kernels/FusedKernels.cs:32-55);
//   * ChannelShift: per channel group a zero-filled shift along H or W (ChannelShiftOp,
//     src/Engine/Fusions/ChannelShiftOp.cs:9-66, FusedKernels.ChannelShift, src/Kernels/FusedKernels.cs:196-221);
//   * UpHead: bilinear resize + skip add + 1x1 conv (oc <= 8) in one pass (UpHeadOp,
//     src/Engine/Fusions/UpHeadOp.cs:9-30, FusedKernels.UpHead, src/Kernels/FusedKernels.cs:71-193);
//   * batched MatMul with numpy batch broadcast, non-constant B (Ops.MatMul, src/Kernels/Ops.Seq.cs:90-113);
//   * the cross-tile merge of the fused CTC projection + argmax (MatMul.TryArgMax and UpdateArgMax,
//     src/Decoding/Kernels/MatMul.ArgMax.cs:29-70, :246-268).
// Storage is fp16 (activations) or fp32 per operand; arithmetic is fp32.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>

#include "sdx_device.cuh"
#include "sdx_internal.h"

namespace sdx {

#define SDX_EXT_LAUNCH_CHECK(what)                                     \
  do {                                                                 \
    cudaError_t e_ = cudaGetLastError();                               \
    if (e_ != cudaSuccess) return set_cuda_error(e_, what " launch");   \
    count_launch();                                                    \
  } while (0)

static int ext_grid(int64_t work, int block) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int64_t blocks = (work + block - 1) / block;
  return (int)std::max<int64_t>(1, std::min<int64_t>(blocks, (int64_t)num_sms(dev) * 16));
}

__device__ __forceinline__ float ld_any(const void* p, int64_t i, int f32) {
  return f32 ? __ldg(static_cast<const float*>(p) + i) : __half2float(static_cast<const __half*>(p)[i]);
}
__device__ __forceinline__ void st_any(void* p, int64_t i, int f32, float v) {
  if (f32) static_cast<float*>(p)[i] = v;
  else static_cast<__half*>(p)[i] = __float2half_rn(v);
}

// The reference's EwOp on one element pair (Ew.Binary, src/Kernels/Ew.cs:75-84): IEEE fp32 add, sub,
// mul, div.
__device__ __forceinline__ float ew_apply(float x, float y, int op) {
  switch (op) {
    case 0: return x + y;
    case 1: return x - y;
    case 2: return x * y;
    default: return x / y;
  }
}

// ------------------------------------------------------------------ broadcast binary
template <int ACT>
__global__ void bcast_binary_kernel(BcastArgs p) {
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < p.n; idx += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = idx, ao = 0, bo = 0;
    for (int d = p.rank - 1; d >= 0; d--) {
      const int64_t i = r % p.shape[d];
      r /= p.shape[d];
      ao += i * p.sa[d];
      bo += i * p.sb[d];
    }
    const float v = ew_apply(ld_any(p.a, ao, p.a_f32), ld_any(p.b, bo, p.b_f32), p.op);
    st_any(p.y, idx, p.y_f32, act_t<ACT>(v));
  }
}

int bcast_binary_launch(const BcastArgs& p, cudaStream_t st) {
  if (p.n == 0) return SDX_OK;
  const int grid = ext_grid(p.n, 256);
  SDX_ACT_DISPATCH(p.act, ACTC, bcast_binary_kernel<ACTC><<<grid, 256, 0, st>>>(p));
  SDX_EXT_LAUNCH_CHECK("bcast_binary");
  return SDX_OK;
}

// ------------------------------------------------------------------ SafeDiv
// Eight fp16 elements per thread with 16-byte accesses when n % 8 == 0 and the pointers allow it.
__device__ __forceinline__ float safe_div1(float a, float b, float eps, float lo, float hi) {
  return fminf(fmaxf(a / fmaxf(b, eps), lo), hi);
}

__global__ void safediv_vec8_kernel(int64_t n8, float eps, float lo, float hi, const __half* a, const __half* b, __half* y) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 ua = __ldg(reinterpret_cast<const uint4*>(a) + i), ub = __ldg(reinterpret_cast<const uint4*>(b) + i);
    const __half2* ha = reinterpret_cast<const __half2*>(&ua);
    const __half2* hb = reinterpret_cast<const __half2*>(&ub);
    uint4 uy;
    __half2* hy = reinterpret_cast<__half2*>(&uy);
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const float2 fa = __half22float2(ha[j]), fb = __half22float2(hb[j]);
      hy[j] = __floats2half2_rn(safe_div1(fa.x, fb.x, eps, lo, hi), safe_div1(fa.y, fb.y, eps, lo, hi));
    }
    reinterpret_cast<uint4*>(y)[i] = uy;
  }
}

__global__ void safediv_kernel(int64_t n, float eps, float lo, float hi, int f32, const void* a, const void* b, void* y) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    st_any(y, i, f32, safe_div1(ld_any(a, i, f32), ld_any(b, i, f32), eps, lo, hi));
}

int safediv_launch(int64_t n, float eps, float lo, float hi, int f32, const void* a, const void* b, void* y,
                   cudaStream_t st) {
  if (n == 0) return SDX_OK;
  const bool vec = !f32 && n % 8 == 0 && ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                                           reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  if (vec) safediv_vec8_kernel<<<ext_grid(n / 8, 256), 256, 0, st>>>(n / 8, eps, lo, hi, static_cast<const __half*>(a),
                                                                     static_cast<const __half*>(b), static_cast<__half*>(y));
  else safediv_kernel<<<ext_grid(n, 256), 256, 0, st>>>(n, eps, lo, hi, f32, a, b, y);
  SDX_EXT_LAUNCH_CHECK("safediv");
  return SDX_OK;
}

// ------------------------------------------------------------------ ChannelShift (NHWC)
// out[n, y, x, ch] = in[n, y + off_g, x, ch] (axis 2) or in[n, y, x + off_g, ch] (axis 3) for the
// group g whose channel range holds ch, zero outside the image; channels past the last group end
// are copied. Thread = one pixel x VEC channels (VEC = 8: 16-byte fp16 accesses, when every group
// boundary and c are multiples of 8).
template <int VEC>
__global__ void channel_shift_kernel(ShiftArgs a) {
  const int cv = a.c / VEC;
  const int64_t total = (int64_t)a.batch * a.h * a.w * cv;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int chv = (int)(i % cv);
    int64_t pix = i / cv;
    const int x = (int)(pix % a.w);
    const int64_t t = pix / a.w;
    const int y = (int)(t % a.h);
    const int64_t n = t / a.h;
    const int ch = chv * VEC;
    int off = 0;
    bool grouped = false;
    for (int g = 0, g0 = 0; g < a.ng; g++) {
      if (ch >= g0 && ch < a.ends[g]) {
        off = a.offs[g];
        grouped = true;
        break;
      }
      g0 = a.ends[g];
    }
    const int sy = grouped && a.axis == 2 ? y + off : y, sx = grouped && a.axis == 3 ? x + off : x;
    const bool inside = (unsigned)sy < (unsigned)a.h && (unsigned)sx < (unsigned)a.w;
    const int64_t src = ((n * a.h + sy) * a.w + sx) * a.c + ch;
    const int64_t dst = pix * a.c + ch;
    if (VEC == 8) {
      uint4 v = make_uint4(0, 0, 0, 0);
      if (inside) v = __ldg(reinterpret_cast<const uint4*>(static_cast<const __half*>(a.x) + src));
      *reinterpret_cast<uint4*>(static_cast<__half*>(a.y) + dst) = v;
    } else {
      st_any(a.y, dst, a.f32, inside ? ld_any(a.x, src, a.f32) : 0.0f);
    }
  }
}

int channel_shift_launch(const ShiftArgs& a, cudaStream_t st) {
  bool vec = !a.f32 && a.c % 8 == 0 &&
             ((reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.y)) & 15) == 0;
  for (int g = 0; g < a.ng; g++) vec = vec && a.ends[g] % 8 == 0;
  const int64_t total = (int64_t)a.batch * a.h * a.w * (vec ? a.c / 8 : a.c);
  if (total == 0) return SDX_OK;
  if (vec) channel_shift_kernel<8><<<ext_grid(total, 256), 256, 0, st>>>(a);
  else channel_shift_kernel<1><<<ext_grid(total, 256), 256, 0, st>>>(a);
  SDX_EXT_LAUNCH_CHECK("channel_shift");
  return SDX_OK;
}

// ------------------------------------------------------------------ UpHead
// out[n, y, x, o] = act(bias[o] + sum_c w[o, c] * s[c]), s = [relu](bilinear(x)) + [relu](skip).
// Bilinear source coordinates follow Nhwc.ResizeAxis (src/Kernels/Nhwc.cs:773-783): f = (o + 0.5) /
// scale - 0.5, floor, both taps clamped, weight f - floor(f); the lerps are the reference's separate
// multiply and add (Nhwc.ResizePixel, src/Kernels/Nhwc.cs:788-815), the dot an FMA chain in
// ascending channel order from the bias. Thread = one output pixel; weights [oc][c] in shared memory.
__device__ __forceinline__ void resize_axis(int o, int in_len, float scale, int& i0, int& i1, float& wt) {
  const float f = __fsub_rn(__fdiv_rn(__fadd_rn((float)o, 0.5f), scale), 0.5f);
  const float fl = floorf(f);
  i0 = min(max((int)fl, 0), in_len - 1);
  i1 = min(max((int)fl + 1, 0), in_len - 1);
  wt = __fsub_rn(f, fl);
}

__device__ __forceinline__ float lerp_ref(float a, float b, float w) { return __fadd_rn(a, __fmul_rn(__fsub_rn(b, a), w)); }

template <int ACT>
__global__ void uphead_kernel(UpHeadArgs a) {
  extern __shared__ float usm[];
  float* sw = usm;                  // [oc][c]
  float* sb = usm + a.oc * a.c;     // [oc]
  for (int i = threadIdx.x; i < a.oc * a.c; i += blockDim.x) sw[i] = a.w[i];
  for (int i = threadIdx.x; i < a.oc; i += blockDim.x) sb[i] = a.bias ? a.bias[i] : 0.0f;
  __syncthreads();
  const int64_t total = (int64_t)a.batch * a.oh * a.ow;
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < total; p += (int64_t)gridDim.x * blockDim.x) {
    const int ox = (int)(p % a.ow);
    const int64_t t = p / a.ow;
    const int oy = (int)(t % a.oh);
    const int64_t n = t / a.oh;
    int y0, y1, x0, x1;
    float wy, wx;
    resize_axis(oy, a.ih, a.sy, y0, y1, wy);
    resize_axis(ox, a.iw, a.sx, x0, x1, wx);
    const int64_t r0 = (n * a.ih + y0) * a.iw, r1 = (n * a.ih + y1) * a.iw;
    const int64_t pa = (r0 + x0) * a.c, pb = (r0 + x1) * a.c, pe = (r1 + x0) * a.c, pf = (r1 + x1) * a.c;
    const int64_t ps = p * a.c;
    float acc[8];
#pragma unroll
    for (int o = 0; o < 8; o++) acc[o] = o < a.oc ? sb[o] : 0.0f;
    for (int ch = 0; ch < a.c; ch++) {
      const float top = lerp_ref(ld_any(a.x, pa + ch, a.x_f32), ld_any(a.x, pb + ch, a.x_f32), wx);
      const float bot = lerp_ref(ld_any(a.x, pe + ch, a.x_f32), ld_any(a.x, pf + ch, a.x_f32), wx);
      float v = lerp_ref(top, bot, wy);
      if (a.resize_relu) v = fmaxf(v, 0.0f);
      float sk = ld_any(a.skip, ps + ch, a.skip_f32);
      if (a.skip_relu) sk = fmaxf(sk, 0.0f);
      v = __fadd_rn(v, sk);
#pragma unroll
      for (int o = 0; o < 8; o++)
        if (o < a.oc) acc[o] = fmaf(v, sw[o * a.c + ch], acc[o]);
    }
#pragma unroll
    for (int o = 0; o < 8; o++)
      if (o < a.oc) st_any(a.y, p * a.oc + o, a.y_f32, act_t<ACT>(acc[o]));
  }
}

int uphead_launch(const UpHeadArgs& a, cudaStream_t st) {
  if (a.oc < 1 || a.oc > 8 || a.c < 1 || a.c > 128 || a.c % 4 != 0)
    return set_error(SDX_ERR_NOT_SUPPORTED, "uphead: needs 1 <= oc <= 8 and c % 4 == 0, c <= 128");
  if (a.act != ACT_NONE && a.act != ACT_RELU && a.act != ACT_SIGMOID)
    return set_error(SDX_ERR_NOT_SUPPORTED, "uphead: activation must be none, relu or sigmoid");
  const int64_t total = (int64_t)a.batch * a.oh * a.ow;
  if (total == 0) return SDX_OK;
  const size_t smem = sizeof(float) * ((size_t)a.oc * a.c + a.oc);
  const int grid = ext_grid(total, 128);
  if (a.act == ACT_RELU) uphead_kernel<ACT_RELU><<<grid, 128, smem, st>>>(a);
  else if (a.act == ACT_SIGMOID) uphead_kernel<ACT_SIGMOID><<<grid, 128, smem, st>>>(a);
  else uphead_kernel<ACT_NONE><<<grid, 128, smem, st>>>(a);
  SDX_EXT_LAUNCH_CHECK("uphead");
  return SDX_OK;
}

// ------------------------------------------------------------------ batched MatMul
// C[b] = A[b] @ B[b] with numpy batch broadcast (per-batch element offsets from the caller's batch
// strides, 0 on broadcast dims): 32 x 32 output tiles, 16-deep K slabs of A and B in shared memory,
// fp32 FMA accumulation in ascending k (GemmKN's order, src/Kernels/Ops.Seq.cs:108-111).
constexpr int MM_T = 32, MM_K = 16;

__global__ void __launch_bounds__(256) batched_matmul_kernel(MatMulArgs p) {
  __shared__ float As[MM_K][MM_T + 1];
  __shared__ float Bs[MM_K][MM_T + 1];
  const int tiles_n = (p.n + MM_T - 1) / MM_T;
  const int tiles_m = (p.m + MM_T - 1) / MM_T;
  const int64_t tiles = (int64_t)p.batch * tiles_m * tiles_n;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;  // each thread: 2 x 2 outputs
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const int64_t bi = tile / (tiles_m * tiles_n);
    const int rem = (int)(tile - bi * tiles_m * tiles_n);
    const int m0 = (rem / tiles_n) * MM_T, n0 = (rem % tiles_n) * MM_T;
    int64_t r = bi, ao = 0, bo = 0;
    for (int d = p.batch_rank - 1; d >= 0; d--) {
      const int64_t i = r % p.bshape[d];
      r /= p.bshape[d];
      ao += i * p.a_bstride[d];
      bo += i * p.b_bstride[d];
    }
    float acc[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};
    for (int k0 = 0; k0 < p.k; k0 += MM_K) {
      for (int e = threadIdx.x; e < MM_K * MM_T; e += blockDim.x) {
        const int kk = e % MM_K, mm = e / MM_K;
        const int gm = m0 + mm, gk = k0 + kk;
        As[kk][mm] = (gm < p.m && gk < p.k) ? ld_any(p.a, ao + (int64_t)gm * p.k + gk, p.a_f32) : 0.0f;
        const int nn = e % MM_T, kb = e / MM_T;
        const int gn = n0 + nn, gk2 = k0 + kb;
        Bs[kb][nn] = (gn < p.n && gk2 < p.k) ? ld_any(p.b, bo + (int64_t)gk2 * p.n + gn, p.b_f32) : 0.0f;
      }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < MM_K; kk++) {
        const float a0 = As[kk][ty * 2], a1 = As[kk][ty * 2 + 1];
        const float b0 = Bs[kk][tx * 2], b1 = Bs[kk][tx * 2 + 1];
        acc[0][0] = fmaf(a0, b0, acc[0][0]);
        acc[0][1] = fmaf(a0, b1, acc[0][1]);
        acc[1][0] = fmaf(a1, b0, acc[1][0]);
        acc[1][1] = fmaf(a1, b1, acc[1][1]);
      }
      __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 2; i++)
#pragma unroll
      for (int j = 0; j < 2; j++) {
        const int gm = m0 + ty * 2 + i, gn = n0 + tx * 2 + j;
        if (gm < p.m && gn < p.n) st_any(p.y, (bi * p.m + gm) * (int64_t)p.n + gn, p.y_f32, acc[i][j]);
      }
  }
}

int batched_matmul_launch(const MatMulArgs& p, cudaStream_t st) {
  const int64_t tiles = (int64_t)p.batch * ((p.m + MM_T - 1) / MM_T) * ((p.n + MM_T - 1) / MM_T);
  if (tiles == 0) return SDX_OK;
  int dev = 0;
  cudaGetDevice(&dev);
  const int grid = (int)std::min<int64_t>(tiles, (int64_t)num_sms(dev) * 8);
  batched_matmul_kernel<<<grid, 256, 0, st>>>(p);
  SDX_EXT_LAUNCH_CHECK("batched_matmul");
  return SDX_OK;
}

// ------------------------------------------------------------------ CTC argmax merge
// Per row, the column tiles' (max, first index of the max, online softmax denominator) states
// [tile][row] merged in column order: a tile whose maximum is strictly larger takes over (the first
// index wins ties, as in the sequential UpdateArgMax) and rescales the running denominator by
// exp(old max - new max); otherwise its denominator is added scaled by exp(its max - running max).
// The winner's probability is min(1, 1 / denominator) (SoftmaxProbability).
__global__ void ctc_argmax_merge_kernel(const float* pm, const int* pi, const float* ps, int rows, int ld, int tiles,
                                        int* indices, float* probs, unsigned int* err) {
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    float m = -INFINITY, s = 0.0f;
    int best = 0;
    for (int t = 0; t < tiles; t++) {
      const float tm = pm[(int64_t)t * ld + r], ts = ps[(int64_t)t * ld + r];
      if (tm > m) {
        s = s * expf(m - tm) + ts;
        m = tm;
        best = pi[(int64_t)t * ld + r];
      } else {
        s += ts * expf(tm - m);
      }
    }
    const bool ok = isfinite(m) && s > 0.0f && isfinite(s);
    if (!ok) record_error(err, SDX_DEV_NONFINITE);
    indices[r] = ok ? best : -1;
    probs[r] = ok ? fminf(1.0f, 1.0f / s) : NAN;
  }
}

int ctc_argmax_merge_launch(const float* pm, const int* pi, const float* ps, int rows, int ld, int tiles,
                            int* indices, float* probs, unsigned int* err, cudaStream_t st) {
  if (rows == 0) return SDX_OK;
  ctc_argmax_merge_kernel<<<ext_grid(rows, 128), 128, 0, st>>>(pm, pi, ps, rows, ld, tiles, indices, probs, err);
  SDX_EXT_LAUNCH_CHECK("ctc_argmax_merge");
  return SDX_OK;
}

}  // namespace sdx
