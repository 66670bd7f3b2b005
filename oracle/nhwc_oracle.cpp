// CPU restatement of SimdOnnx's NHWC CPU kernels. TEST INFRASTRUCTURE ONLY (parity checker and
// timed CPU baseline); the product never links or calls this file. See oracle.h for the contract.
//
// Build: -O3 -ffp-contract=off (no implicit contraction: every fused multiply-add below is an
// explicit fmaf/vfma where the reference uses Fma.MultiplyAdd / FusedMultiplyAdd, and every other
// expression rounds after each operation like the reference's Vector operators) -fopenmp.
#include "oracle.h"

#include <math.h>
#include <omp.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <vector>

#if defined(__AVX512F__) || defined(__AVX2__)
#include <immintrin.h>
#endif

typedef float v16f __attribute__((vector_size(64)));
typedef float v8f __attribute__((vector_size(32)));

static int g_threads = 0;

extern "C" void orc_set_threads(int threads) { g_threads = threads > 0 ? threads : 0; }
extern "C" int orc_get_threads(void) { return g_threads > 0 ? g_threads : omp_get_max_threads(); }
extern "C" int orc_isa_avx512(void) {
#if defined(__AVX512F__)
  return 1;
#else
  return 0;
#endif
}

static inline v16f vload(const float* p) { v16f v; memcpy(&v, p, 64); return v; }
static inline void vstore(float* p, v16f v) { memcpy(p, &v, 64); }
static inline v16f vsplat(float x) { return (v16f){x, x, x, x, x, x, x, x, x, x, x, x, x, x, x, x}; }

// a*b + c with one rounding per lane (Avx512F.FusedMultiplyAdd / Fma.MultiplyAdd).
static inline v16f vfma(v16f a, v16f b, v16f c) {
#if defined(__AVX512F__)
  return (v16f)_mm512_fmadd_ps((__m512)a, (__m512)b, (__m512)c);
#elif defined(__FMA__)
  __m256 a0, a1, b0, b1, c0, c1;
  memcpy(&a0, &a, 32); memcpy(&a1, (const char*)&a + 32, 32);
  memcpy(&b0, &b, 32); memcpy(&b1, (const char*)&b + 32, 32);
  memcpy(&c0, &c, 32); memcpy(&c1, (const char*)&c + 32, 32);
  __m256 r0 = _mm256_fmadd_ps(a0, b0, c0), r1 = _mm256_fmadd_ps(a1, b1, c1);
  v16f r; memcpy(&r, &r0, 32); memcpy((char*)&r + 32, &r1, 32);
  return r;
#else
  v16f r;
  for (int i = 0; i < 16; i++) r[i] = fmaf(a[i], b[i], c[i]);
  return r;
#endif
}

static inline int par_threads() { return orc_get_threads(); }

// =====================================================================================
// Math cores of the fused epilogues (src/Kernels/SimdMath.cs:120-170, the AVX2 cores that
// Nhwc.Act8 uses, src/Kernels/Nhwc.cs:90-99).
// =====================================================================================
extern "C" float orc_exp_core(float x) {
  // ExpCore: cephes-style 2^n * poly(r) (src/Kernels/SimdMath.cs:121-139)
  x = fmaxf(x, -87.3f);
  x = fminf(x, 88.7f);
  float fx = fmaf(x, 1.4426950408889634f, 0.5f);
  float nf = floorf(fx);
  float r = fmaf(nf, -0.693359375f, x);
  r = fmaf(nf, 0.00021219444005469058f, r);
  float p = 1.9875691500e-4f;
  p = fmaf(p, r, 1.3981999507e-3f);
  p = fmaf(p, r, 8.3334519073e-3f);
  p = fmaf(p, r, 4.1665795894e-2f);
  p = fmaf(p, r, 1.6666665459e-1f);
  p = fmaf(p, r, 5.0000001201e-1f);
  float y = fmaf(p, r * r, r) + 1.0f;
  int ni = (int)nf + 127;
  uint32_t bits = (uint32_t)ni << 23;
  float pow2n;
  memcpy(&pow2n, &bits, 4);
  return y * pow2n;
}

static inline float sigmoid_core(float x) { return 1.0f / (1.0f + orc_exp_core(-x)); }

extern "C" float orc_erf_core(float x) {
  // ErfCore: Abramowitz-Stegun 7.1.26 (src/Kernels/SimdMath.cs:146-161)
  float sign = signbit(x) ? -1.0f : 1.0f;
  float ax = fabsf(x);
  float t = 1.0f / (1.0f + 0.3275911f * ax);
  float p = 1.061405429f;
  p = fmaf(p, t, -1.453152027f);
  p = fmaf(p, t, 1.421413741f);
  p = fmaf(p, t, -0.284496736f);
  p = fmaf(p, t, 0.254829592f);
  float y = 1.0f - (p * t) * orc_exp_core(-(ax * ax));
  return y * sign;
}

static inline float gelu_core(float x) { return (0.5f * x) * (1.0f + orc_erf_core(x * 0.70710678118654752f)); }

// Nhwc.Act8 per lane (src/Kernels/Nhwc.cs:90-99): the activation of every fused conv / Gemm epilogue.
static inline float act8(float v, int act) {
  switch (act) {
    case ORC_ACT_RELU: return fmaxf(v, 0.0f);
    case ORC_ACT_SIGMOID: return sigmoid_core(v);
    case ORC_ACT_GELU: return gelu_core(v);
    case ORC_ACT_HARDSWISH: return v * fminf(fmaxf(fmaf(v, 1.0f / 6.0f, 0.5f), 0.0f), 1.0f);
    case ORC_ACT_SWISH: return v * sigmoid_core(v);
    default: return v;
  }
}

// ErfScalar (src/Kernels/SimdMath.cs:270-277).
static inline float erf_scalar(float x) {
  float ax = fabsf(x);
  float t = 1.0f / (1.0f + 0.3275911f * ax);
  float p = ((((1.061405429f * t - 1.453152027f) * t + 1.421413741f) * t - 0.284496736f) * t + 0.254829592f) * t;
  float y = 1.0f - p * expf(-ax * ax);
  return x < 0 ? -y : y;
}

// Nhwc.ActS (src/Kernels/Nhwc.cs:82-88): scalar channel tails.
extern "C" float orc_act_scalar(float v, int act) {
  switch (act) {
    case ORC_ACT_RELU: return fmaxf(v, 0.0f);
    case ORC_ACT_SIGMOID: return 1.0f / (1.0f + expf(-v));
    case ORC_ACT_GELU: return 0.5f * v * (1.0f + erf_scalar(v * 0.70710678f));
    case ORC_ACT_HARDSWISH: return v * fminf(fmaxf(v * (1.0f / 6.0f) + 0.5f, 0.0f), 1.0f);
    case ORC_ACT_SWISH: return v / (1.0f + expf(-v));
    default: return v;
  }
}

// Act.cs vector op per lane (src/Kernels/Act.cs:25-68): standalone activation nodes.
static inline float act_node(float v, int act) {
  switch (act) {
    case ORC_ACT_RELU: return fmaxf(v, 0.0f);
    case ORC_ACT_SIGMOID: return sigmoid_core(v);
    case ORC_ACT_GELU: return gelu_core(v);
    case ORC_ACT_HARDSWISH: return v * fminf(fmaxf(v * (1.0f / 6.0f) + 0.5f, 0.0f), 1.0f);
    case ORC_ACT_SWISH: return v * sigmoid_core(v);
    default: return v;
  }
}

// =====================================================================================
// Packing (src/Kernels/Nhwc.cs:102-138)
// =====================================================================================
static const int Ob = 16;     // oc lanes per packed block (src/Kernels/Nhwc.cs:37)
static const int Tile5 = 10;  // AVX-512 pixel tile (src/Kernels/Nhwc.Avx512.cs:22)

extern "C" int64_t orc_pack_conv_floats(int oc, int ic, int kh, int kw) {
  int64_t nb = (oc + Ob - 1) / Ob;
  return nb * kh * kw * ic * Ob;
}

extern "C" void orc_pack_conv(const float* w, const float* bias, int oc, int ic, int kh, int kw, float* pw, float* pb) {
  int taps = kh * kw, nb = (oc + Ob - 1) / Ob;
  memset(pw, 0, sizeof(float) * (size_t)orc_pack_conv_floats(oc, ic, kh, kw));
  for (int o = 0; o < oc; o++)
    for (int c = 0; c < ic; c++)
      for (int t = 0; t < taps; t++)
        pw[(((int64_t)(o / Ob) * taps + t) * ic + c) * Ob + o % Ob] = w[((int64_t)o * ic + c) * taps + t];
  memset(pb, 0, sizeof(float) * nb * Ob);
  if (bias) memcpy(pb, bias, sizeof(float) * oc);
}

extern "C" void orc_pack_depthwise(const float* w, const float* bias, int c, int kh, int kw, float* pw, float* pb) {
  int taps = kh * kw;
  for (int ch = 0; ch < c; ch++)
    for (int t = 0; t < taps; t++) pw[(int64_t)t * c + ch] = w[(int64_t)ch * taps + t];
  if (bias) memcpy(pb, bias, sizeof(float) * c);
  else memset(pb, 0, sizeof(float) * c);
}

extern "C" void orc_pack_gemm(const float* b, int k, int n, int trans_b, const float* bias, float* pw, float* pb) {
  int nb = (n + Ob - 1) / Ob;
  memset(pw, 0, sizeof(float) * (size_t)nb * k * Ob);
  for (int o = 0; o < n; o++)
    for (int c = 0; c < k; c++)
      pw[((int64_t)(o / Ob) * k + c) * Ob + o % Ob] = trans_b ? b[(int64_t)o * k + c] : b[(int64_t)c * n + o];
  memset(pb, 0, sizeof(float) * nb * Ob);
  if (bias) memcpy(pb, bias, sizeof(float) * n);
}

extern "C" int orc_winograd_eligible(int group, int kh, int kw, int sh, int sw, int ic) {
  return group == 1 && kh == 3 && kw == 3 && sh == 1 && sw == 1 && ic >= 16 && ic % 8 == 0;
}

// G of F(4,3) (src/Kernels/NhwcWinograd.cs:35-43)
static const double s_g[6][3] = {
    {1.0 / 4, 0, 0},
    {-1.0 / 6, -1.0 / 6, -1.0 / 6},
    {-1.0 / 6, 1.0 / 6, -1.0 / 6},
    {1.0 / 24, 1.0 / 12, 1.0 / 6},
    {1.0 / 24, -1.0 / 12, 1.0 / 6},
    {0, 0, 1},
};

extern "C" int64_t orc_pack_winograd_floats(int oc, int ic) {
  int64_t nb = (oc + Ob - 1) / Ob;
  return 36 * nb * ic * Ob;
}

extern "C" void orc_pack_winograd(const float* w, int oc, int ic, float* u) {
  // PackWinograd (src/Kernels/NhwcWinograd.cs:46-68): U = G g G^T in double, stored as float
  int nb = (oc + Ob - 1) / Ob;
  memset(u, 0, sizeof(float) * (size_t)orc_pack_winograd_floats(oc, ic));
  for (int o = 0; o < oc; o++)
    for (int c = 0; c < ic; c++) {
      const float* k = w + ((int64_t)o * ic + c) * 9;
      double gg[18];
      for (int i = 0; i < 6; i++)
        for (int j = 0; j < 3; j++) gg[i * 3 + j] = s_g[i][0] * k[j] + s_g[i][1] * k[3 + j] + s_g[i][2] * k[6 + j];
      for (int i = 0; i < 6; i++)
        for (int j = 0; j < 6; j++) {
          double v = gg[i * 3] * s_g[j][0] + gg[i * 3 + 1] * s_g[j][1] + gg[i * 3 + 2] * s_g[j][2];
          u[((((int64_t)(i * 6 + j) * nb + o / Ob) * ic + c) * Ob) + o % Ob] = (float)v;
        }
    }
}

// =====================================================================================
// Index maps (src/Kernels/Nhwc.cs:56-80)
// =====================================================================================
static inline int reflect_idx(int i, int dim) {
  if (dim <= 1) return 0;
  while (i < 0 || i >= dim) i = i < 0 ? -i : 2 * dim - 2 - i;
  return i;
}

static std::vector<int> make_map(int out_len, int k, int stride, int pad, int in_len, int mode) {
  std::vector<int> m((size_t)out_len * k);
  for (int o = 0; o < out_len; o++)
    for (int kk = 0; kk < k; kk++) {
      int s = o * stride + kk - pad;
      m[(size_t)o * k + kk] = (unsigned)s < (unsigned)in_len ? s : mode == ORC_PAD_REFLECT ? reflect_idx(s, in_len) : -1;
    }
  return m;
}

// =====================================================================================
// Dense direct conv: Dense512 / Dense512Row / Tile512x32 / Epilogue512
// (src/Kernels/Nhwc.Avx512.cs:33-239). Per element: bias, taps ascending, channels ascending,
// one FMA each; then + residual, then Act8.
// =====================================================================================
struct DenseArgs {
  const float* src;  // one image [ih, iw, ic]
  const float* w;
  const float* bias;
  const float* padvec;  // ic*kw + 16 floats of the pad value
  const int* rm;
  const int* cm;
  int iw, ic, ow, oc, kh, kw, nb, act;
};

// Tile5 pixels x (16 * nblk) oc: part[r*32 + 0..31]
static void tile512(const float* const* ptrs, int nblk, int taps, int ic, const float* wb, int64_t wstep,
                    const float* bb, float* part) {
  v16f a[Tile5], b[Tile5];
  v16f ba = vload(bb), bbv = nblk == 2 ? vload(bb + Ob) : vsplat(0.0f);
  for (int i = 0; i < Tile5; i++) { a[i] = ba; b[i] = bbv; }
  for (int tap = 0; tap < taps; tap++) {
    const float* const* pp = ptrs + tap * Tile5;
    const float* w = wb + (int64_t)tap * ic * Ob;
    if (nblk == 2) {
      const float* x = w + wstep;
      for (int c = 0; c < ic; c++, w += Ob, x += Ob) {
        v16f wa = vload(w), wx = vload(x);
        for (int i = 0; i < Tile5; i++) {
          v16f v = vsplat(pp[i][c]);
          a[i] = vfma(v, wa, a[i]);
          b[i] = vfma(v, wx, b[i]);
        }
      }
    } else {
      for (int c = 0; c < ic; c++, w += Ob) {
        v16f wa = vload(w);
        for (int i = 0; i < Tile5; i++) a[i] = vfma(vsplat(pp[i][c]), wa, a[i]);
      }
    }
  }
  for (int i = 0; i < Tile5; i++) {
    vstore(part + i * 2 * Ob, a[i]);
    vstore(part + i * 2 * Ob + Ob, b[i]);
  }
}

// Store16 / Epilogue512 (src/Kernels/Nhwc.cs:376-398, src/Kernels/Nhwc.Avx512.cs:129-152)
static inline void store_lanes(float* o, const float* add, const float* s, int lanes, int act) {
  for (int l = 0; l < lanes; l++) {
    float v = s[l];
    if (add) v = v + add[l];
    o[l] = act8(v, act);
  }
}

static void epilogue512(const float* part, int rows, int nblk, float* outp, const float* addp, int oc, int lanes0,
                        int lanes1, int act) {
  for (int r = 0; r < rows; r++, part += 2 * Ob) {
    float* o = outp + (int64_t)r * oc;
    const float* ad = addp ? addp + (int64_t)r * oc : nullptr;
    for (int h = 0; h < nblk; h++) {
      int lanes = h == 0 ? lanes0 : lanes1;
      store_lanes(o + h * Ob, ad ? ad + h * Ob : nullptr, part + h * Ob, lanes, act);
    }
  }
}

static void dense512_row(const DenseArgs& a, int y, int blk, float* orow, const float* arow) {
  int kh = a.kh, kw = a.kw, taps = kh * kw, ic = a.ic, ow = a.ow, oc = a.oc, nblk = std::min(2, a.nb - blk);
  int64_t wstep = (int64_t)taps * ic * Ob;
  const float* ptrs[Tile5 * 49 > 2000 ? 2000 : Tile5 * 49];
  std::vector<const float*> big;
  const float** pt = (const float**)ptrs;
  if (taps > 49) { big.resize((size_t)Tile5 * taps); pt = big.data(); }
  alignas(64) float part[Tile5 * 2 * Ob];
  const float* wb = a.w + blk * wstep;
  const float* bb = a.bias + blk * Ob;
  int lanes0 = std::min(Ob, oc - blk * Ob), lanes1 = nblk == 2 ? std::min(Ob, oc - (blk + 1) * Ob) : 0;
  for (int x0 = 0; x0 < ow; x0 += Tile5) {
    int rows = std::min(Tile5, ow - x0);
    bool merged = kw > 1;
    for (int i = 0; i < rows && merged; i++) {
      const int* cx = a.cm + (int64_t)(x0 + i) * kw;
      merged = cx[0] >= 0;
      for (int kx = 1; kx < kw; kx++) merged &= cx[kx] == cx[0] + kx;
    }
    if (merged) {
      for (int ky = 0; ky < kh; ky++) {
        int r = a.rm[y * kh + ky];
        for (int i = 0; i < Tile5; i++) {
          int c = a.cm[(int64_t)(x0 + std::min(i, rows - 1)) * kw];
          pt[ky * Tile5 + i] = r < 0 ? a.padvec : a.src + ((int64_t)r * a.iw + c) * ic;
        }
      }
      tile512(pt, nblk, kh, kw * ic, wb, wstep, bb, part);
    } else {
      for (int tap = 0; tap < taps; tap++) {
        int r = a.rm[y * kh + tap / kw];
        for (int i = 0; i < Tile5; i++) {
          int c = a.cm[(int64_t)(x0 + std::min(i, rows - 1)) * kw + tap % kw];
          pt[tap * Tile5 + i] = r < 0 || c < 0 ? a.padvec : a.src + ((int64_t)r * a.iw + c) * ic;
        }
      }
      tile512(pt, nblk, taps, ic, wb, wstep, bb, part);
    }
    int64_t o = (int64_t)x0 * oc + blk * Ob;
    epilogue512(part, rows, nblk, orow + o, arow ? arow + o : nullptr, oc, lanes0, lanes1, a.act);
  }
}

// =====================================================================================
// Winograd F(4x4,3x3): WinoTiles / WinoOutput / InputTransform / OutputTransform
// (src/Kernels/NhwcWinograd.cs:97-398). Transforms round after every operation (no FMA), the
// 36 GEMMs are FMA chains from zero over ascending channels, then tmp + bias + residual, Act8.
// =====================================================================================
static void input_transform(const float* const* d, int ic, float* v, int64_t vstride) {
  // V[xi] = (B^T d B)[xi] for one tile (src/Kernels/NhwcWinograd.cs:254-291)
  std::vector<float> tb(36);
  for (int c = 0; c < ic; c++) {
    float t[36];
    for (int j = 0; j < 6; j++) {
      float d0 = d[j][c], d1 = d[6 + j][c], d2 = d[12 + j][c], d3 = d[18 + j][c], d4 = d[24 + j][c], d5 = d[30 + j][c];
      t[j] = 4.0f * d0 - 5.0f * d2 + d4;
      t[6 + j] = d3 + d4 - 4.0f * (d1 + d2);
      t[12 + j] = d4 - d3 + 4.0f * (d1 - d2);
      t[18 + j] = d4 - d2 + 2.0f * (d3 - d1);
      t[24 + j] = d4 - d2 - 2.0f * (d3 - d1);
      t[30 + j] = 4.0f * d1 - 5.0f * d3 + d5;
    }
    for (int i = 0; i < 6; i++) {
      float r0 = t[i * 6], r1 = t[i * 6 + 1], r2 = t[i * 6 + 2], r3 = t[i * 6 + 3], r4 = t[i * 6 + 4], r5 = t[i * 6 + 5];
      float* o = v + c;
      int64_t b = (int64_t)(i * 6) * vstride;
      o[b] = 4.0f * r0 - 5.0f * r2 + r4;
      o[b + vstride] = r3 + r4 - 4.0f * (r1 + r2);
      o[b + 2 * vstride] = r4 - r3 + 4.0f * (r1 - r2);
      o[b + 3 * vstride] = r4 - r2 + 2.0f * (r3 - r1);
      o[b + 4 * vstride] = r4 - r2 - 2.0f * (r3 - r1);
      o[b + 5 * vstride] = 4.0f * r1 - 5.0f * r3 + r5;
    }
  }
}

static void output_transform(const float* m, int64_t mstride, float* tmp) {
  // tmp[(py*4+px)*16 + l] = (A^T m A)[py,px] (src/Kernels/NhwcWinograd.cs:295-329)
  for (int l = 0; l < Ob; l++) {
    float s[24];
    for (int j = 0; j < 6; j++) {
      float m0 = m[j * mstride + l], m1 = m[(6 + j) * mstride + l], m2 = m[(12 + j) * mstride + l];
      float m3 = m[(18 + j) * mstride + l], m4 = m[(24 + j) * mstride + l], m5 = m[(30 + j) * mstride + l];
      float a = m1 + m2, b = m1 - m2, c = m3 + m4, e = m3 - m4;
      s[j] = m0 + a + c;
      s[6 + j] = b + 2.0f * e;
      s[12 + j] = a + 4.0f * c;
      s[18 + j] = b + 8.0f * e + m5;
    }
    for (int i = 0; i < 4; i++) {
      float r0 = s[i * 6], r1 = s[i * 6 + 1], r2 = s[i * 6 + 2], r3 = s[i * 6 + 3], r4 = s[i * 6 + 4], r5 = s[i * 6 + 5];
      float a = r1 + r2, b = r1 - r2, c = r3 + r4, e = r3 - r4;
      float* o = tmp + i * 4 * Ob + l;
      o[0] = r0 + a + c;
      o[Ob] = b + 2.0f * e;
      o[2 * Ob] = a + 4.0f * c;
      o[3 * Ob] = b + 8.0f * e + r5;
    }
  }
}

struct WinoArgs {
  const float* src;  // one image
  const float* u;
  const float* bias;
  const float* padvec;
  int ih, iw, ic, oh, ow, oc, tw, nb, pad_t, pad_l, reflect, act;
};

static inline int src_idx(int i, int n, int reflect) {
  return (unsigned)i < (unsigned)n ? i : reflect ? reflect_idx(i, n) : -1;
}

// tiles [t0, t0+tn) of one image into dp (row 0 == output row row_base), residual ap (same base)
static void wino_tiles(const WinoArgs& a, int t0, int tn, float* dp, const float* ap, int row_base) {
  int ic = a.ic, tw = a.tw, nb = a.nb, oc = a.oc, ow = a.ow, oh = a.oh;
  std::vector<float> V((size_t)36 * tn * ic), M((size_t)36 * tn * Ob);
  const float* d[36];
  for (int t = 0; t < tn; t++) {
    int ty = (t0 + t) / tw, tx = (t0 + t) % tw;
    int iy0 = ty * 4 - a.pad_t, ix0 = tx * 4 - a.pad_l;
    for (int i = 0; i < 6; i++) {
      int r = src_idx(iy0 + i, a.ih, a.reflect);
      for (int j = 0; j < 6; j++) {
        int c = src_idx(ix0 + j, a.iw, a.reflect);
        d[i * 6 + j] = r < 0 || c < 0 ? a.padvec : a.src + ((int64_t)r * a.iw + c) * ic;
      }
    }
    input_transform(d, ic, V.data() + (int64_t)t * ic, (int64_t)tn * ic);
  }
  alignas(64) float tmp[16 * Ob];
  for (int blk = 0; blk < nb; blk++) {
    for (int xi = 0; xi < 36; xi++) {
      const float* wb = a.u + ((int64_t)xi * nb + blk) * ic * Ob;
      const float* vx = V.data() + (int64_t)xi * tn * ic;
      float* mx = M.data() + (int64_t)xi * tn * Ob;
      for (int t = 0; t < tn; t++) {
        v16f acc = vsplat(0.0f);
        const float* vr = vx + (int64_t)t * ic;
        for (int c = 0; c < ic; c++) acc = vfma(vsplat(vr[c]), vload(wb + (int64_t)c * Ob), acc);
        vstore(mx + (int64_t)t * Ob, acc);
      }
    }
    int oc_off = blk * Ob, lanes = std::min(Ob, oc - oc_off);
    const float* bb = a.bias + oc_off;
    for (int t = 0; t < tn; t++) {
      int ty = (t0 + t) / tw, tx = (t0 + t) % tw;
      output_transform(M.data() + (int64_t)t * Ob, (int64_t)tn * Ob, tmp);
      for (int py = 0; py < 4; py++) {
        int oy = ty * 4 + py;
        if (oy >= oh) break;
        for (int px = 0; px < 4; px++) {
          int ox = tx * 4 + px;
          if (ox >= ow) break;
          int64_t o = ((int64_t)(oy - row_base) * ow + ox) * oc + oc_off;
          const float* tp = tmp + (py * 4 + px) * Ob;
          for (int l = 0; l < lanes; l++) {
            float v = tp[l] + bb[l];
            if (ap) v = v + ap[o + l];
            dp[o + l] = act8(v, a.act);
          }
        }
      }
    }
  }
}

// =====================================================================================
// Depthwise: Nhwc.Depthwise / DwRow / DwRunAvx / DwBlockAvx (src/Kernels/Nhwc.cs:496-631,
// src/Kernels/Nhwc.Depthwise.cs:23-156). Vector channels (c - c%8): FMA chain from the bias over
// the kernel rows that are in range (constant pad 0: out-of-range rows skipped), pad columns read
// the pad value; scalar channel tail: separate multiply and add, ActS.
// =====================================================================================
static void dw_row(const float* sp, float* dp, const float* ap, const float* wp, const float* bp, const float* padvec,
                   const int* rm, const int* cm, int iw, int c, int ow, int kh, int kw, bool clip_rows, int act, int y) {
  const int* rmy = rm + y * kh;
  int kyb = 0, kye = kh;
  if (clip_rows) {
    while (kyb < kye && rmy[kyb] < 0) kyb++;
    while (kye > kyb && rmy[kye - 1] < 0) kye--;
  }
  int cvec = c - c % 8;
  std::vector<float> acc((size_t)c);
  for (int x = 0; x < ow; x++) {
    const int* cmx = cm + (int64_t)x * kw;
    for (int ch = 0; ch < c; ch++) acc[ch] = bp[ch];
    for (int ky = kyb; ky < kye; ky++) {
      int r = rmy[ky];
      for (int kx = 0; kx < kw; kx++) {
        int cc = cmx[kx];
        const float* s = r < 0 || cc < 0 ? padvec : sp + ((int64_t)r * iw + cc) * c;
        const float* w = wp + (int64_t)(ky * kw + kx) * c;
        for (int ch = 0; ch < cvec; ch++) acc[ch] = fmaf(s[ch], w[ch], acc[ch]);
        for (int ch = cvec; ch < c; ch++) acc[ch] = acc[ch] + s[ch] * w[ch];
      }
    }
    float* o = dp + (int64_t)x * c;
    const float* ad = ap ? ap + (int64_t)x * c : nullptr;
    for (int ch = 0; ch < cvec; ch++) {
      float v = acc[ch];
      if (ad) v = v + ad[ch];
      o[ch] = act8(v, act);
    }
    for (int ch = cvec; ch < c; ch++) {
      float v = acc[ch];
      if (ad) v += ad[ch];
      o[ch] = orc_act_scalar(v, act);
    }
  }
}

// =====================================================================================
// Conv entry (src/Kernels/Nhwc.cs:172-217)
// =====================================================================================
extern "C" void orc_conv(const float* src, int batch, int ih, int iw, int ic, float* dst, int oh, int ow, int oc,
                         int kh, int kw, int sh, int sw, int pt, int pl, int pad_mode, float pad_value,
                         const float* pw, const float* pb, const float* wino_u, int depthwise,
                         const float* add, int act) {
  int64_t in_img = (int64_t)ih * iw * ic, out_img = (int64_t)oh * ow * oc;
  int threads = par_threads();
  if (depthwise) {
    std::vector<int> rm = make_map(oh, kh, sh, pt, ih, pad_mode), cm = make_map(ow, kw, sw, pl, iw, pad_mode);
    std::vector<float> padvec((size_t)ic * kw + Ob, pad_value);
    bool clip = pad_value == 0.0f;
#pragma omp parallel for schedule(static) num_threads(threads)
    for (int64_t t = 0; t < (int64_t)batch * oh; t++) {
      int b = (int)(t / oh), y = (int)(t % oh);
      dw_row(src + b * in_img, dst + b * out_img + (int64_t)y * ow * oc, add ? add + b * out_img + (int64_t)y * ow * oc : nullptr,
             pw, pb, padvec.data(), rm.data(), cm.data(), iw, ic, ow, kh, kw, clip, act, y);
    }
    return;
  }
  if (wino_u) {
    // WinogradConv (src/Kernels/NhwcWinograd.cs:97-119): tiles in chunks; per-tile math is
    // independent of the grouping
    std::vector<float> padvec((size_t)ic, pad_value);
    int tw = (ow + 3) / 4, nt = (oh + 3) / 4 * tw, T = 10;
    int chunks = (nt + T - 1) / T;
#pragma omp parallel for schedule(dynamic) num_threads(threads)
    for (int64_t job = 0; job < (int64_t)batch * chunks; job++) {
      int b = (int)(job / chunks), ch = (int)(job % chunks);
      WinoArgs a{src + b * in_img, wino_u, pb, padvec.data(), ih, iw, ic, oh, ow, oc, tw, (oc + Ob - 1) / Ob,
                 pt, pl, pad_mode == ORC_PAD_REFLECT, act};
      int t0 = ch * T;
      wino_tiles(a, t0, std::min(T, nt - t0), dst + b * out_img, add ? add + b * out_img : nullptr, 0);
    }
    return;
  }
  std::vector<int> rm = make_map(oh, kh, sh, pt, ih, pad_mode), cm = make_map(ow, kw, sw, pl, iw, pad_mode);
  std::vector<float> padvec((size_t)ic * kw + Ob, pad_value);
  int nb = (oc + Ob - 1) / Ob, np = (nb + 1) / 2;
#pragma omp parallel for schedule(dynamic) num_threads(threads)
  for (int64_t t = 0; t < (int64_t)batch * oh * np; t++) {
    int b = (int)(t / ((int64_t)oh * np));
    int r = (int)(t % ((int64_t)oh * np)), y = r / np, blk = r % np * 2;
    DenseArgs a{src + b * in_img, pw, pb, padvec.data(), rm.data(), cm.data(), iw, ic, ow, oc, kh, kw, nb, act};
    int64_t o = b * out_img + (int64_t)y * ow * oc;
    dense512_row(a, y, blk, dst + o, add ? add + o : nullptr);
  }
}

// ConvPool (src/Kernels/Nhwc.cs:666-727): conv rows (no residual) into a band, then PoolBand:
// max(max(max(s0, s1), s2), s3), optional relu.
extern "C" void orc_conv_pool(const float* src, int batch, int ih, int iw, int ic, float* dst, int oh, int ow, int oc,
                              int kh, int kw, int sh, int sw, int pt, int pl, int pad_mode, float pad_value,
                              const float* pw, const float* pb, const float* wino_u, int act, int pool_relu) {
  int ph = oh / 2, pwd = ow / 2;
  int64_t in_img = (int64_t)ih * iw * ic;
  std::vector<float> full((size_t)oh * ow * oc);
  for (int b = 0; b < batch; b++) {
    orc_conv(src + b * in_img, 1, ih, iw, ic, full.data(), oh, ow, oc, kh, kw, sh, sw, pt, pl, pad_mode, pad_value, pw, pb,
             wino_u, 0, nullptr, act);
    float* d = dst + (int64_t)b * ph * pwd * oc;
    for (int y = 0; y < ph; y++)
      for (int x = 0; x < pwd; x++) {
        const float* s0 = full.data() + ((int64_t)(2 * y) * ow + 2 * x) * oc;
        const float* s1 = s0 + oc;
        const float* s2 = s0 + (int64_t)ow * oc;
        const float* s3 = s2 + oc;
        float* o = d + ((int64_t)y * pwd + x) * oc;
        for (int c = 0; c < oc; c++) {
          float v = fmaxf(fmaxf(fmaxf(s0[c], s1[c]), s2[c]), s3[c]);
          o[c] = pool_relu ? fmaxf(v, 0.0f) : v;
        }
      }
  }
}

extern "C" void orc_conv_ref64(const float* src, int batch, int ih, int iw, int ic, double* dst, int oh, int ow, int oc,
                               int kh, int kw, int sh, int sw, int pt, int pl, int group, int pad_mode, float pad_value,
                               const float* w, const float* bias, const float* add, int act) {
  int icg = ic / group, ocg = oc / group;
  int threads = par_threads();
#pragma omp parallel for schedule(static) num_threads(threads)
  for (int64_t t = 0; t < (int64_t)batch * oh; t++) {
    int b = (int)(t / oh), y = (int)(t % oh);
    for (int x = 0; x < ow; x++)
      for (int o = 0; o < oc; o++) {
        int g = o / ocg;
        double acc = bias ? bias[o] : 0.0;
        for (int ky = 0; ky < kh; ky++)
          for (int kx = 0; kx < kw; kx++) {
            int sy = y * sh + ky - pt, sx = x * sw + kx - pl;
            bool in = (unsigned)sy < (unsigned)ih && (unsigned)sx < (unsigned)iw;
            if (!in && pad_mode == ORC_PAD_REFLECT) {
              sy = reflect_idx(sy, ih);
              sx = reflect_idx(sx, iw);
              in = true;
            }
            for (int c = 0; c < icg; c++) {
              double xv = in ? src[(((int64_t)b * ih + sy) * iw + sx) * ic + g * icg + c] : pad_value;
              acc += xv * (double)w[(((int64_t)o * icg + c) * kh + ky) * kw + kx];
            }
          }
        int64_t oi = (((int64_t)b * oh + y) * ow + x) * oc + o;
        if (add) acc += add[oi];
        double v = acc;
        switch (act) {
          case ORC_ACT_RELU: v = v > 0 ? v : 0; break;
          case ORC_ACT_SIGMOID: v = 1.0 / (1.0 + exp(-v)); break;
          case ORC_ACT_GELU: v = 0.5 * v * (1.0 + erf(v / sqrt(2.0))); break;
          case ORC_ACT_HARDSWISH: v = v * std::min(std::max(v / 6.0 + 0.5, 0.0), 1.0); break;
          case ORC_ACT_SWISH: v = v / (1.0 + exp(-v)); break;
          default: break;
        }
        dst[oi] = v;
      }
  }
}

// =====================================================================================
// Gemm (Gemm512, src/Kernels/Nhwc.Avx512.cs:241-266) and MatMul (GemmKN,
// src/Kernels/Avx2Kernels.cs:504-560 / src/Kernels/Ops.cs:600-640)
// =====================================================================================
extern "C" void orc_gemm(const float* a, int m, int k, float* dst, int n, const float* pw, const float* pb, int act) {
  int nb = (n + Ob - 1) / Ob, np = (nb + 1) / 2, tiles = (m + Tile5 - 1) / Tile5;
  int64_t wstep = (int64_t)k * Ob;
  int threads = par_threads();
#pragma omp parallel for schedule(dynamic) num_threads(threads)
  for (int64_t t = 0; t < (int64_t)tiles * np; t++) {
    int tile = (int)(t / np), blk = (int)(t % np) * 2, nblk = std::min(2, nb - blk);
    const float* ptrs[Tile5];
    alignas(64) float part[Tile5 * 2 * Ob];
    int m0 = tile * Tile5, rows = std::min(Tile5, m - m0);
    for (int i = 0; i < Tile5; i++) ptrs[i] = a + (int64_t)(m0 + std::min(i, rows - 1)) * k;
    tile512(ptrs, nblk, 1, k, pw + blk * wstep, wstep, pb + blk * Ob, part);
    int lanes0 = std::min(Ob, n - blk * Ob), lanes1 = nblk == 2 ? std::min(Ob, n - (blk + 1) * Ob) : 0;
    epilogue512(part, rows, nblk, dst + (int64_t)m0 * n + blk * Ob, nullptr, n, lanes0, lanes1, act);
  }
}

extern "C" void orc_matmul(const float* a, const float* b, float* dst, int batch, int m, int k, int n) {
  bool fma_path = (int64_t)m * n * k >= 32768;
  int nv = n - n % 16;
  int threads = par_threads();
#pragma omp parallel for schedule(static) num_threads(threads)
  for (int64_t t = 0; t < (int64_t)batch * m; t++) {
    int bi = (int)(t / m), row = (int)(t % m);
    const float* ar = a + ((int64_t)bi * m + row) * k;
    const float* bb = b + (int64_t)bi * k * n;
    float* dr = dst + ((int64_t)bi * m + row) * n;
    for (int n0 = 0; n0 < (fma_path ? nv : n - n % 8); n0++) {
      float s = 0.0f;
      if (fma_path)
        for (int kk = 0; kk < k; kk++) s = fmaf(ar[kk], bb[(int64_t)kk * n + n0], s);
      else
        for (int kk = 0; kk < k; kk++) s = s + bb[(int64_t)kk * n + n0] * ar[kk];
      dr[n0] = s;
    }
    for (int n0 = fma_path ? nv : n - n % 8; n0 < n; n0++) {
      float s = 0.0f;
      for (int kk = 0; kk < k; kk++) s += ar[kk] * bb[(int64_t)kk * n + n0];
      dr[n0] = s;
    }
  }
}

// =====================================================================================
// ConvTranspose stride == kernel (src/Kernels/Nhwc.Det.cs:26-131)
// =====================================================================================
extern "C" void orc_convt(const float* src, int batch, int ih, int iw, int ic, float* dst, int oc, int kh, int kw,
                          const float* w, const float* bias, int act) {
  int taps = kh * kw, ow = iw * kw, oh = ih * kh;
  int threads = par_threads();
  if (oc > 4) {
    // per tap a [ic] x [oc] panel through TileAvx: bias-init, ic ascending FMA, Store16 (Act8)
#pragma omp parallel for schedule(static) num_threads(threads)
    for (int64_t t = 0; t < (int64_t)batch * ih; t++) {
      int b = (int)(t / ih), y = (int)(t % ih);
      std::vector<float> acc((size_t)oc);
      for (int x = 0; x < iw; x++) {
        const float* xp = src + (((int64_t)b * ih + y) * iw + x) * ic;
        for (int tap = 0; tap < taps; tap++) {
          int dy = tap / kw, dx = tap % kw;
          for (int o = 0; o < oc; o++) acc[o] = bias ? bias[o] : 0.0f;
          for (int c = 0; c < ic; c++) {
            float xv = xp[c];
            const float* wr = w + (int64_t)c * oc * taps + tap;
            for (int o = 0; o < oc; o++) acc[o] = fmaf(xv, wr[(int64_t)o * taps], acc[o]);
          }
          float* op = dst + ((((int64_t)b * oh + y * kh + dy) * ow) + x * kw + dx) * oc;
          for (int o = 0; o < oc; o++) op[o] = act8(acc[o], act);
        }
      }
    }
    return;
  }
  // ConvTDot: 4-lane partial products (multiply then add per lane), ((a0+a1)+(a2+a3)), scalar tail,
  // then ActRow over the output rows (Act8 on 8-float runs, ActS on the row tail)
#pragma omp parallel for schedule(static) num_threads(threads)
  for (int64_t t = 0; t < (int64_t)batch * ih; t++) {
    int b = (int)(t / ih), y = (int)(t % ih);
    for (int x = 0; x < iw; x++) {
      const float* xp = src + (((int64_t)b * ih + y) * iw + x) * ic;
      for (int tap = 0; tap < taps; tap++) {
        float* o = dst + ((((int64_t)b * oh + y * kh + tap / kw) * ow) + x * kw + tap % kw) * oc;
        for (int k = 0; k < oc; k++) {
          float s = bias ? bias[k] : 0.0f;
          float acc[4] = {0, 0, 0, 0};
          int c = 0;
          for (; c + 4 <= ic; c += 4)
            for (int l = 0; l < 4; l++) acc[l] = acc[l] + xp[c + l] * w[((int64_t)(c + l) * oc + k) * taps + tap];
          s += (acc[0] + acc[1]) + (acc[2] + acc[3]);
          for (; c < ic; c++) s += xp[c] * w[((int64_t)c * oc + k) * taps + tap];
          o[k] = s;
        }
      }
    }
    if (act != ORC_ACT_NONE) {
      float* row = dst + ((int64_t)b * oh + (int64_t)y * kh) * ow * oc;
      int64_t len = (int64_t)kh * ow * oc, nv = len - len % 8, i = 0;
      for (; i < nv; i++) row[i] = act8(row[i], act);
      for (; i < len; i++) row[i] = orc_act_scalar(row[i], act);
    }
  }
}

// =====================================================================================
// Pools
// =====================================================================================
extern "C" void orc_maxpool(const float* src, int batch, int ih, int iw, int c, float* dst, int oh, int ow,
                            int kh, int kw, int sh, int sw, int pt, int pl, int relu) {
  // Nhwc.MaxPool / MaxPool512 (src/Kernels/Nhwc.cs:730-770, src/Kernels/Nhwc.Avx512.cs:293-323)
  std::vector<int> rm = make_map(oh, kh, sh, pt, ih, ORC_PAD_CONSTANT), cm = make_map(ow, kw, sw, pl, iw, ORC_PAD_CONSTANT);
  int threads = par_threads();
#pragma omp parallel for schedule(static) num_threads(threads)
  for (int64_t t = 0; t < (int64_t)batch * oh; t++) {
    int b = (int)(t / oh), y = (int)(t % oh);
    const float* sp = src + (int64_t)b * ih * iw * c;
    for (int x = 0; x < ow; x++) {
      float* o = dst + (((int64_t)b * oh + y) * ow + x) * c;
      bool any = false;
      for (int ky = 0; ky < kh; ky++) {
        int r = rm[(size_t)y * kh + ky];
        if (r < 0) continue;
        for (int kx = 0; kx < kw; kx++) {
          int cc = cm[(size_t)x * kw + kx];
          if (cc < 0) continue;
          const float* s = sp + ((int64_t)r * iw + cc) * c;
          if (!any) { memcpy(o, s, sizeof(float) * c); any = true; continue; }
          for (int ch = 0; ch < c; ch++) o[ch] = fmaxf(o[ch], s[ch]);
        }
      }
      if (!any) memset(o, 0, sizeof(float) * c);
      else if (relu)
        for (int ch = 0; ch < c; ch++) o[ch] = fmaxf(o[ch], 0.0f);
    }
  }
}

extern "C" void orc_avgpool(const float* src, int batch, int ih, int iw, int c, float* dst, int oh, int ow,
                            int kh, int kw, int sh, int sw, int pt, int pl, int count_include_pad) {
  // Nhwc.AvgPool (src/Kernels/Ops.Seq.cs:180-225): sum in tap order, times 1/count
  std::vector<int> rm = make_map(oh, kh, sh, pt, ih, ORC_PAD_CONSTANT), cm = make_map(ow, kw, sw, pl, iw, ORC_PAD_CONSTANT);
  int threads = par_threads();
#pragma omp parallel for schedule(static) num_threads(threads)
  for (int64_t t = 0; t < (int64_t)batch * oh; t++) {
    int b = (int)(t / oh), y = (int)(t % oh);
    const float* sp = src + (int64_t)b * ih * iw * c;
    for (int x = 0; x < ow; x++) {
      float* o = dst + (((int64_t)b * oh + y) * ow + x) * c;
      for (int ch = 0; ch < c; ch++) o[ch] = 0.0f;
      int cnt = 0;
      for (int ky = 0; ky < kh; ky++) {
        int r = rm[(size_t)y * kh + ky];
        if (r < 0) continue;
        for (int kx = 0; kx < kw; kx++) {
          int cc = cm[(size_t)x * kw + kx];
          if (cc < 0) continue;
          const float* s = sp + ((int64_t)r * iw + cc) * c;
          for (int ch = 0; ch < c; ch++) o[ch] = o[ch] + s[ch];
          cnt++;
        }
      }
      float inv = 1.0f / (float)(count_include_pad ? kh * kw : std::max(cnt, 1));
      for (int ch = 0; ch < c; ch++) o[ch] = o[ch] * inv;
    }
  }
}

static void gap_image(const float* src, int hw, int c, float* dst, int threads) {
  // Nhwc.GlobalAvgPool (src/Kernels/Nhwc.Det.cs:134-164)
  int64_t want = (int64_t)hw * c / 65536;
  int chunks = (int)std::min<int64_t>(std::max<int64_t>(want, 1), threads);
  std::vector<float> part((size_t)chunks * c, 0.0f);
  for (int k = 0; k < chunks; k++) {
    int p0 = (int)((int64_t)k * hw / chunks), p1 = (int)((int64_t)(k + 1) * hw / chunks);
    float* acc = part.data() + (int64_t)k * c;
    for (int px = p0; px < p1; px++) {
      const float* s = src + (int64_t)px * c;
      for (int ch = 0; ch < c; ch++) acc[ch] = acc[ch] + s[ch];
    }
  }
  float inv = 1.0f / (float)hw;
  for (int ch = 0; ch < c; ch++) {
    float s = 0.0f;
    for (int k = 0; k < chunks; k++) s += part[(size_t)k * c + ch];
    dst[ch] = s * inv;
  }
}

extern "C" void orc_global_avg_pool(const float* src, int batch, int hw, int c, float* dst) {
  int threads = par_threads();
#pragma omp parallel for schedule(static) num_threads(threads)
  for (int b = 0; b < batch; b++) gap_image(src + (int64_t)b * hw * c, hw, c, dst + (int64_t)b * c, threads);
}

// =====================================================================================
// SE gate and the per-channel broadcast (src/Kernels/Nhwc.Det.cs:287-351)
// =====================================================================================
extern "C" void orc_channel_gate(const float* src, int batch, int hw, int c, const float* w1, const float* b1,
                                 const float* w2, const float* b2, int r, int act1_relu, int hard, float alpha, float beta,
                                 float offset, float* dst) {
  int threads = par_threads();
#pragma omp parallel for schedule(static) num_threads(threads)
  for (int b = 0; b < batch; b++) {
    std::vector<float> mean((size_t)c), hid((size_t)r);
    gap_image(src + (int64_t)b * hw * c, hw, c, mean.data(), threads);
    for (int j = 0; j < r; j++) {
      float s = b1 ? b1[j] : 0.0f;
      const float* row = w1 + (int64_t)j * c;
      for (int k = 0; k < c; k++) s += row[k] * mean[k];
      hid[j] = act1_relu ? fmaxf(s, 0.0f) : s;
    }
    for (int ch = 0; ch < c; ch++) {
      float z = b2 ? b2[ch] : 0.0f;
      const float* row = w2 + (int64_t)ch * r;
      for (int j = 0; j < r; j++) z += row[j] * hid[j];
      float g = hard ? std::min(std::max(z * alpha + beta, 0.0f), 1.0f) : 1.0f / (1.0f + expf(-z));
      dst[(int64_t)b * c + ch] = g + offset;
    }
  }
}

static inline float ew(float a, float b, int op) {
  switch (op) {
    case ORC_EW_ADD: return a + b;
    case ORC_EW_SUB: return a - b;
    case ORC_EW_MUL: return a * b;
    default: return a / b;
  }
}

extern "C" void orc_channel_broadcast(const float* full, const float* vec, float* dst, int batch, int64_t rows, int c,
                                      int op, int rev, int relu) {
  int threads = par_threads();
#pragma omp parallel for schedule(static) num_threads(threads)
  for (int64_t t = 0; t < (int64_t)batch * rows; t++) {
    int b = (int)(t / rows);
    const float* f = full + t * c;
    const float* v = vec + (int64_t)b * c;
    float* d = dst + t * c;
    for (int ch = 0; ch < c; ch++) {
      float s = rev ? ew(v[ch], f[ch], op) : ew(f[ch], v[ch], op);
      d[ch] = relu ? fmaxf(s, 0.0f) : s;
    }
  }
}

extern "C" void orc_resize_nearest(const float* src, int batch, int ih, int iw, int c, float* dst, int oh, int ow,
                                   float sy, float sx, const float* add, int add_relu) {
  std::vector<int> xs((size_t)ow);
  for (int x = 0; x < ow; x++) xs[x] = std::min((int)floorf((float)x / sx), iw - 1);
  int threads = par_threads();
#pragma omp parallel for schedule(static) num_threads(threads)
  for (int64_t t = 0; t < (int64_t)batch * oh; t++) {
    int b = (int)(t / oh), y = (int)(t % oh);
    int ys = std::min((int)floorf((float)y / sy), ih - 1);
    const float* srow = src + (((int64_t)b * ih + ys) * iw) * c;
    float* orow = dst + (((int64_t)b * oh + y) * ow) * c;
    const float* arow = add ? add + (((int64_t)b * oh + y) * ow) * c : nullptr;
    for (int x = 0; x < ow; x++) {
      const float* s = srow + (int64_t)xs[x] * c;
      float* o = orow + (int64_t)x * c;
      if (!arow) { memcpy(o, s, sizeof(float) * c); continue; }
      const float* a = arow + (int64_t)x * c;
      for (int ch = 0; ch < c; ch++) o[ch] = s[ch] + (add_relu ? fmaxf(a[ch], 0.0f) : a[ch]);
    }
  }
}

extern "C" void orc_concat_inner(const float* const* ins, const int* counts, int nin, int64_t outer, float* dst) {
  int total = 0;
  for (int i = 0; i < nin; i++) total += counts[i];
  int threads = par_threads();
#pragma omp parallel for schedule(static) num_threads(threads)
  for (int64_t o = 0; o < outer; o++) {
    float* d = dst + o * total;
    for (int i = 0; i < nin; i++) {
      memcpy(d, ins[i] + o * counts[i], sizeof(float) * counts[i]);
      d += counts[i];
    }
  }
}

// =====================================================================================
// Elementwise, activations, LayerNorm, Softmax
// =====================================================================================
extern "C" void orc_act(const float* src, float* dst, int64_t n, int act) {
  // Act.Apply (src/Kernels/Act.cs:70-110): 8-float vector runs with the vector op, scalar tail
  int threads = par_threads();
  int64_t nv = n - n % 8;
#pragma omp parallel for schedule(static) num_threads(threads)
  for (int64_t i = 0; i < nv; i++) dst[i] = act_node(src[i], act);
  for (int64_t i = nv; i < n; i++) {
    float x = src[i];
    switch (act) {
      case ORC_ACT_RELU: dst[i] = fmaxf(x, 0.0f); break;
      case ORC_ACT_SIGMOID: dst[i] = 1.0f / (1.0f + expf(-x)); break;
      case ORC_ACT_GELU: dst[i] = 0.5f * x * (1.0f + erf_scalar(x * 0.70710678118654752f)); break;
      case ORC_ACT_HARDSWISH: dst[i] = x * std::min(std::max(x * (1.0f / 6.0f) + 0.5f, 0.0f), 1.0f); break;
      case ORC_ACT_SWISH: dst[i] = x / (1.0f + expf(-x)); break;
      default: dst[i] = x; break;
    }
  }
}

extern "C" void orc_binary(const float* a, const float* b, float* dst, int64_t n, int op, int relu) {
  int threads = par_threads();
#pragma omp parallel for schedule(static) num_threads(threads)
  for (int64_t i = 0; i < n; i++) {
    float s = ew(a[i], b[i], op);
    dst[i] = relu ? fmaxf(s, 0.0f) : s;
  }
}

extern "C" void orc_hardsigmoid(const float* src, float* dst, int64_t n, float alpha, float beta) {
  for (int64_t i = 0; i < n; i++) dst[i] = std::min(std::max(src[i] * alpha + beta, 0.0f), 1.0f);
}

extern "C" void orc_layernorm(const float* x, int64_t rows, int c, const float* w, const float* b, float* dst, float eps) {
  // Avx2Kernels.LayerNorm (src/Kernels/Avx2Kernels.cs:563-600): 8-lane sums (squares by FMA),
  // lanes added in order, one-pass variance clamped at 0, out = fma(x - mean, inv*w, b)
  int threads = par_threads();
#pragma omp parallel for schedule(static) num_threads(threads)
  for (int64_t r = 0; r < rows; r++) {
    const float* xr = x + r * c;
    float* dr = dst + r * c;
    float sum[8] = {0}, sq[8] = {0};
    int i = 0;
    for (; i + 8 <= c; i += 8)
      for (int l = 0; l < 8; l++) {
        sum[l] = sum[l] + xr[i + l];
        sq[l] = fmaf(xr[i + l], xr[i + l], sq[l]);
      }
    float s = 0, ss = 0;
    for (int l = 0; l < 8; l++) { s += sum[l]; ss += sq[l]; }
    for (; i < c; i++) { float v = xr[i]; s += v; ss += v * v; }
    float mean = s / c;
    float inv = 1.0f / sqrtf(fmaxf(ss / c - mean * mean, 0.0f) + eps);
    for (i = 0; i + 8 <= c; i += 8)
      for (int l = 0; l < 8; l++) dr[i + l] = fmaf(xr[i + l] - mean, inv * w[i + l], b[i + l]);
    for (; i < c; i++) dr[i] = (xr[i] - mean) * inv * w[i] + b[i];
  }
}

extern "C" void orc_softmax(const float* src, float* dst, int64_t rows, int c) {
  // SoftmaxRow (src/Kernels/Ops.Seq.cs:40-75): 4-lane max, ExpCore on 4-lane runs, 4-lane sum
  // reduced ((s0+s1)+(s2+s3)), scalar tails, multiply by 1/sum
  int threads = par_threads();
#pragma omp parallel for schedule(static) num_threads(threads)
  for (int64_t r = 0; r < rows; r++) {
    const float* s = src + r * c;
    float* d = dst + r * c;
    float mx = -INFINITY;
    int i = 0;
    if (c >= 4) {
      float vm[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      for (; i + 4 <= c; i += 4)
        for (int l = 0; l < 4; l++) vm[l] = fmaxf(vm[l], s[i + l]);
      mx = fmaxf(fmaxf(vm[0], vm[1]), fmaxf(vm[2], vm[3]));
    }
    for (; i < c; i++) mx = fmaxf(mx, s[i]);
    float acc[4] = {0, 0, 0, 0};
    i = 0;
    for (; i + 4 <= c; i += 4)
      for (int l = 0; l < 4; l++) {
        float e = orc_exp_core(s[i + l] - mx);
        d[i + l] = e;
        acc[l] = acc[l] + e;
      }
    float sum = (acc[0] + acc[1]) + (acc[2] + acc[3]);
    for (; i < c; i++) { float e = expf(s[i] - mx); d[i] = e; sum += e; }
    float inv = 1.0f / sum;
    for (i = 0; i < c; i++) d[i] = d[i] * inv;
  }
}
