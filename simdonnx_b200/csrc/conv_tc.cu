// Dense conv / pointwise conv / Gemm / stride==kernel ConvTranspose on the sm_100a tensor cores.
//
// One persistent, warp-specialised kernel (320 threads, one CTA per SM):
//   warp 0      TMA producer: per 64-channel k-block one A box and the two B boxes (weight terms
//               hi, lo) into a smem ring (SWIZZLE_128B, no multicast), full/empty mbarriers;
//   warp 1      allocates TMEM, one lane issues tcgen05.mma (M=128, N=BN, K=16 per instruction,
//               f16 x f16 -> f32) into one of four TMEM accumulators and commits the stage back;
//   warps 2..9  epilogue, two groups of four warps taking alternate tiles. Warp q of a group owns
//               TMEM lanes (= tile rows) 32q..32q+31 and finishes them on its own: tcgen05.ld in
//               16-column chunks (double-buffered registers), bias -> + residual -> activation (the
//               reference's Store16 order, src/Kernels/Nhwc.cs:376-398), a swizzled staging slab
//               in shared memory, and a TMA tensor store of its 32 rows (coalesced, asynchronous,
//               clipped at the tensor edges). Its residual rows arrive by a TMA load issued one
//               tile ahead. No barrier spans more than one warp.
// Four accumulators (two when BN > 128) let the MMAs run ahead of each epilogue group, and the
// double-buffered staging lets the TMA store of tile i overlap the epilogue of tile i+1.
//
// A operand ("mode"):
//   TC_ROWS  A is a row-major [M, K] matrix (1x1 conv with the batch folded into rows,
//            src/Kernels/Nhwc.cs:177-183; Gemm, src/Kernels/Nhwc.Avx512.cs:241-266).
//   TC_CONV  implicit-GEMM k x k conv, stride 1. Halo mode (kh > 1): per column tap kx and channel
//            block cb ONE 4-D box {64 ch, BW, BH + kh - 1, 1} of the NHWC input at
//            (ox0+kx-pl, oy0-pt) serves all kh row taps: the A operand of tap (ky, kx) is that box
//            from row ky*BW on (BW >= 8, so the offset is a whole 1024-byte swizzle atom). That
//            loads each input row (BH + kh - 1) / BH times per kx instead of kh times. Otherwise
//            (kh = 1) one box {64 ch, BW, BH, 1} per tap. The TMA zero-fills out-of-range
//            rows/columns, which is the constant-0 padding. K is tap-major then channel, the order
//            of the reference's packed weights (src/Kernels/Nhwc.cs:102-125).
// B operand: packed weights [terms][taps][n_tiles*BN][Kpad] fp16 (K-major), K padded to the channel
// block (64, 32 or 16). With two terms every weight w is stored as hi + lo, hi = fp16(w),
// lo = fp16(w - hi), and both are multiplied into the same TMEM accumulator (two MMAs per k-step):
// the weights keep ~22 significant bits, so weight rounding does not shift coherent sums such as
// squeeze-excitation means. 1x1 convs, Gemm and ConvT use two terms (their MMAs hide under HBM
// time); k x k convs default to one (the MMA issue rate bounds them; one fp16 term is the weight
// type of the reference's GPU backends). The activations are one fp16 term.
// The weights sit in shared memory for the whole kernel when they fit beside the A ring, else they
// are streamed with each A stage.
//
// ConvT (stride == kernel, src/Kernels/Nhwc.Det.cs:46-93): a 1x1 TC_CONV over the input pixels with
// N = kh*kw*OC columns (tap-major); the epilogue stores column group (dy, dx*OC + o) of a BH x BW
// input tile as one box of the 5-D output view {kw*OC, W, kh, H, batch}, i.e. straight to output
// pixels (y*kh + dy, x*kw + dx).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>

#include "sdx_device.cuh"
#include "sdx_internal.h"

namespace sdx {

constexpr int TC_BM = 128;
// Epilogue warp groups (kernel template G): 2, or 4 for tiles of at most 64 columns (more warps
// hide the per-tile latency of thin tiles); a CTA is the producer warp, the MMA warp and G groups.
constexpr int TC_EPI_GROUPS_MAX = 4;
constexpr int tc_threads(int groups) { return 64 + 128 * groups; }
constexpr int TC_MAX_STAGES = 8;  // <= 32 (ring slots are tracked in 32-bit masks)
constexpr int TC_SMEM_LIMIT = 227 * 1024;
constexpr int TC_BIAS_SMEM_MAX = 4096;  // bias floats staged in shared memory

struct TcArgs {
  int mode;
  int M;
  int N;
  int BN;
  int n_tiles;
  int m_tiles;
  int kb_per_tap;
  int halo;             // TC_CONV: one A box per (kx, channel block) holds the BH + kh - 1 input rows
                        // of all kh row taps; the MMAs of tap (ky, kx) read it from row ky * BW on
  int b_taps;           // weight taps per stage (kh in halo mode, else 1)
  uint32_t a_stage_bytes;  // bytes of one A stage: cps boxes of a_blk_bytes
  uint32_t a_blk_bytes;    // one channel block's A box, rounded up to 1024 bytes
  int cps;              // channel blocks per pipeline stage (divides kb_per_tap)
  int kblk;             // channels per k-block: 64, 32 or 16 (rows of 128/64/32 B, same-span swizzle)
  int b_resident;       // 1: all weights are loaded into shared memory once per CTA
  int wterms;           // fp16 weight terms: 1 (w) or 2 (hi, lo: two MMAs per k-step)
  uint32_t b_total_bytes;  // bytes of all weights (both terms), resident mode
  int taps, kw;
  int pad_t, pad_l;
  int OH, OW, BH, BW, tiles_h, tiles_w;
  int BWs;              // tile step along x (BW, or BW - 2 in kx-in-N mode: the halo columns overlap)
  int kxn;              // 3x3 conv with the column taps as GEMM columns (kx * 32 + oc)
  int b_rows_per_tap;
  int stages;
  int acc_stride;
  int nacc;             // TMEM accumulators: 4 when 4 x BN fits the 512 columns, else 2
  int egroups;          // epilogue warp groups (the kernel's G): 2 or 4
  uint32_t tmem_cols;
  uint32_t a_box_bytes;
  // epilogue
  const float* bias;
  const void* res;
  int res_f32;
  int64_t res_pix_stride;
  int res_ch_off;
  int res_up;           // 2: residual on the half-size grid, read nearest-upsampled (per thread)
  void* out;
  int out_f32;
  int64_t out_pix_stride;
  int out_ch_off;
  int act;
  int vec_ok;
  int convt_kh, convt_kw, convt_oc, convt_H, convt_W;
  // TMA store epilogue
  int tma_out;          // 1: staging buffer + TMA stores; 0: per-thread stores (fallback)
  int tma_res;          // 1: residual tile by TMA load into the staging buffer
  int esz;              // output element bytes
  int G;                // columns per store group
  int ngroups;          // groups per tile
  int swz;              // staging rows (G * esz bytes = 32, 64 or 128) use the TMA swizzle of that span
  uint32_t group_bytes; // bytes of one group in the staging buffer (128 rows)
  uint32_t sbuf_bytes;  // bytes of one staging buffer
  int nsbuf;            // staging buffers per epilogue group (1 or 2)
  uint32_t slab_tx;     // bytes one residual box (one group, one warp's 32 rows) delivers
  int bias_smem;        // bias floats staged in shared memory (per accumulator column), 0 = none
  int log2G;            // log2 of G (fast epilogue: G is 16, 32 or 64)
  // ConvT chain epilogue (EPI = 4): the second ConvT's weights follow the bias in smem
  int chain_act2, chain_y_f32;
  void* chain_y;
  const float* chain_w2;
  const float* chain_b2;
  // channel sums of the activated output over each run of 32 rows (a warp's rows; rows mode, M a
  // multiple of 32): fp32 [M / 32][N], or null
  float* gap;
  unsigned int* err;
};

// ------------------------------------------------------------------ TMA store / bulk-group helpers
// Predicated on `p` (the warp's elected lane, elect_leader()): called by the whole converged warp,
// executed by one lane. Bulk groups belong to the issuing thread, so one warp always uses the same
// elected lane (the lowest, as the warp is converged) for its stores, commits and waits.
__device__ __forceinline__ void tma_store_2d(uint32_t p, const CUtensorMap* map, uint32_t src, int c0, int c1) {
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %4, 0;\n\t"
               "@q cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];\n\t}" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(c0), "r"(c1), "r"(p)
               : "memory");
}
__device__ __forceinline__ void tma_store_4d(uint32_t p, const CUtensorMap* map, uint32_t src, int c0, int c1, int c2,
                                             int c3) {
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %6, 0;\n\t"
               "@q cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];\n\t}" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(p)
               : "memory");
}
__device__ __forceinline__ void tma_store_5d(uint32_t p, const CUtensorMap* map, uint32_t src, int c0, int c1, int c2,
                                             int c3, int c4) {
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %7, 0;\n\t"
               "@q cp.async.bulk.tensor.5d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5, %6}], [%1];\n\t}" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(p)
               : "memory");
}
__device__ __forceinline__ void bulk_commit(uint32_t p) {
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %0, 0;\n\t@q cp.async.bulk.commit_group;\n\t}" ::"r"(p) : "memory");
}
__device__ __forceinline__ void bulk_wait_read0(uint32_t p) {
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %0, 0;\n\t@q cp.async.bulk.wait_group.read 0;\n\t}" ::"r"(p)
               : "memory");
}
__device__ __forceinline__ void bulk_wait_read1(uint32_t p) {
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %0, 0;\n\t@q cp.async.bulk.wait_group.read 1;\n\t}" ::"r"(p)
               : "memory");
}
__device__ __forceinline__ void bulk_wait_all(uint32_t p) {
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %0, 0;\n\t@q cp.async.bulk.wait_group 0;\n\t}" ::"r"(p) : "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
// ------------------------------------------------------------------ per-thread fallback helpers
__device__ __forceinline__ void load8_res(const TcArgs& a, int64_t off, float* r) {
  if (a.res_f32) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(a.res) + off);
    float4 x = __ldg(p), y = __ldg(p + 1);
    r[0] = x.x; r[1] = x.y; r[2] = x.z; r[3] = x.w; r[4] = y.x; r[5] = y.y; r[6] = y.z; r[7] = y.w;
  } else {
    uint4 u = __ldg(reinterpret_cast<const uint4*>(static_cast<const __half*>(a.res) + off));
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      float2 f = __half22float2(h[i]);
      r[2 * i] = f.x;
      r[2 * i + 1] = f.y;
    }
  }
}

__device__ __forceinline__ void store8(const TcArgs& a, int64_t off, const float* v) {
  if (a.out_f32) {
    float4* p = reinterpret_cast<float4*>(static_cast<float*>(a.out) + off);
    p[0] = make_float4(v[0], v[1], v[2], v[3]);
    p[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    uint4 u;
    __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; i++) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(static_cast<__half*>(a.out) + off) = u;
  }
}

// Output pixel / channel of accumulator column n for GEMM row `row` (ConvT scatter or plain).
__device__ __forceinline__ void out_coord(const TcArgs& a, int64_t row, int n, int64_t& opix, int& och) {
  if (a.convt_oc > 0) {
    int tap = n / a.convt_oc, o = n - tap * a.convt_oc;
    int dy = tap / a.convt_kw, dx = tap - dy * a.convt_kw;
    int64_t x = row % a.convt_W, t = row / a.convt_W;
    int64_t y = t % a.convt_H, img = t / a.convt_H;
    opix = ((img * a.convt_H + y) * a.convt_kh + dy) * ((int64_t)a.convt_W * a.convt_kw) + x * a.convt_kw + dx;
    och = o;
  } else {
    opix = row;
    och = n;
  }
}

__device__ __forceinline__ void lds16(uint32_t addr, uint4& v) {
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
}
__device__ __forceinline__ void sts16(uint32_t addr, const uint4& v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Bounded mbarrier wait by every lane of a converged warp; the result is made warp-uniform.
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity, unsigned int* err, unsigned int code,
                                               volatile int* abort_flag) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, err, code, abort_flag));
}

struct TileCoord {
  int img, oy0, ox0, m0, n0;
};

// TMA store (or residual load) of column group g of warp q's 32 tile rows. Tile pixel rows
// 32q..32q+31 form one box: BW >= 32 gives a run of 32 pixels inside one tile row, BW < 32 gives
// 32/BW whole tile rows (tile widths are powers of two, so BW divides 32 or 32 divides BW).
// A store whose box starts past the tensor's edge is skipped (it would write nothing); loads there
// read the zero fill.
__device__ __forceinline__ void warp_copy(uint32_t p, const TcArgs& a, const CUtensorMap* map, uint32_t src, int g,
                                          int q, const TileCoord& t, bool load, uint32_t bar) {
  const int n = t.n0 + g * a.G;
  if (a.mode == TC_CONV) {
    const int p0 = q * 32;
    const int x = t.ox0 + p0 % a.BW, y = t.oy0 + p0 / a.BW;
    if (!load && (x >= a.OW || y >= a.OH)) return;
    if (a.convt_oc > 0) {
      const int row = a.convt_kw * a.convt_oc;
      const int dy = n / row, c = n - dy * row;
      tma_store_5d(p, map, src, c, x, dy, y, t.img);
    } else if (load) {
      tma_load_4d_p(p, src, map, bar, a.out_ch_off + n, x, y, t.img);
    } else {
      tma_store_4d(p, map, src, a.out_ch_off + n, x, y, t.img);
    }
  } else {
    if (load) tma_load_2d_p(p, src, map, bar, a.out_ch_off + n, t.m0 + q * 32);
    else if (t.m0 + q * 32 < a.M) tma_store_2d(p, map, src, a.out_ch_off + n, t.m0 + q * 32);
  }
}

// The MMAs of one pipeline stage, fully unrolled (the issuing thread's scalar work between MMAs is
// its bottleneck for small N): BT taps x NK k-steps of 16 channels, each multiplying the A rows by
// the weight term (TWO: both terms, hi then lo). Descriptors advance by constant strides given in
// 16-byte units: A by `a_tap` per tap, B by `b_tap` per tap and `b_lo` to the lo term.
// `first` = 0 makes the first MMA of a tile overwrite the accumulator.
template <int BT, int NK, bool TWO>
__device__ __forceinline__ void umma_stage(uint32_t p, uint32_t d, uint64_t ad, uint64_t bd, uint32_t a_tap, uint32_t b_tap,
                                           uint32_t b_lo, uint32_t idesc, uint32_t first) {
#pragma unroll
  for (int j = 0; j < BT; j++) {
#pragma unroll
    for (int k = 0; k < NK; k++) {
      const uint64_t a = ad + (uint64_t)(j * a_tap + 2u * k), b = bd + (uint64_t)(j * b_tap + 2u * k);
      umma_f16_p(p, d, a, b, idesc, (j == 0 && k == 0) ? first : 1u);
      if (TWO) umma_f16_p(p, d, a, b + b_lo, idesc, 1u);
    }
  }
}

template <bool TWO>
__device__ __forceinline__ void umma_stage_dispatch(uint32_t p, int bt, int nk, uint32_t d, uint64_t ad, uint64_t bd, uint32_t a_tap,
                                                    uint32_t b_tap, uint32_t b_lo, uint32_t idesc, uint32_t first) {
  if (bt == 1) {
    if (nk == 4) umma_stage<1, 4, TWO>(p, d, ad, bd, a_tap, b_tap, b_lo, idesc, first);
    else if (nk == 2) umma_stage<1, 2, TWO>(p, d, ad, bd, a_tap, b_tap, b_lo, idesc, first);
    else umma_stage<1, 1, TWO>(p, d, ad, bd, a_tap, b_tap, b_lo, idesc, first);
  } else if (bt == 3) {
    if (nk == 4) umma_stage<3, 4, TWO>(p, d, ad, bd, a_tap, b_tap, b_lo, idesc, first);
    else if (nk == 2) umma_stage<3, 2, TWO>(p, d, ad, bd, a_tap, b_tap, b_lo, idesc, first);
    else umma_stage<3, 1, TWO>(p, d, ad, bd, a_tap, b_tap, b_lo, idesc, first);
  } else {
    for (int j = 0; j < bt; j++) {
      if (nk == 4) umma_stage<1, 4, TWO>(p, d, ad + (uint64_t)(j * a_tap), bd + (uint64_t)(j * b_tap), 0, 0, b_lo, idesc, j == 0 ? first : 1u);
      else if (nk == 2) umma_stage<1, 2, TWO>(p, d, ad + (uint64_t)(j * a_tap), bd + (uint64_t)(j * b_tap), 0, 0, b_lo, idesc, j == 0 ? first : 1u);
      else umma_stage<1, 1, TWO>(p, d, ad + (uint64_t)(j * a_tap), bd + (uint64_t)(j * b_tap), 0, 0, b_lo, idesc, j == 0 ? first : 1u);
    }
  }
}

// MMA issue loop for tiles that are one pipeline stage (kernel taps 1, weights resident, every
// channel block of the tile in one stage): per tile two waits, CPS x NK (x2 with TWO) MMAs and two
// commits, no runtime loop or dispatch between them (each costs the issuing warp far more than
// the MMA itself); ring slot, phases and the N tile advance without branches.
// Producer loop for the same single-stage tiles: per tile one empty wait, one expect_tx and CPS
// A copies (2-D row boxes, or the 4-D pixel box at (ox0 - pad_l, oy0 - pad_t)), without per-stage
// dispatch. Ring slots that received a copy and their last phase are reported for the wind-down.
struct ProdSingle {
  uint32_t sA, a_stage_bytes, a_blk_bytes, stage_tx;
  int S, n_tiles, tiles_h, tiles_w, BH, BWs, kblk, pad_l, pad_t;
};
template <int CONV, int CPS>
__device__ __noinline__ void producer_single_loop(uint32_t ld, const ProdSingle p, const CUtensorMap* tmA, int tile0,
                                                  int total_tiles, int tstep, uint64_t* full, uint64_t* empty,
                                                  unsigned int* err, volatile int* abort_flag, uint32_t& issued_mask,
                                                  uint32_t& last_phase) {
  int s = 0;
  uint32_t phase = 0;
  for (int tile = tile0; tile < total_tiles; tile += tstep) {
    const int m_tile = p.n_tiles == 1 ? tile : tile / p.n_tiles;
    if (!mbar_wait_warp(smem_u32(&empty[s]), phase ^ 1u, err, SDX_DEV_WAIT_EMPTY, abort_flag)) break;
    const uint32_t fb = smem_u32(&full[s]);
    mbar_arrive_expect_tx_p(ld, fb, p.stage_tx);
    const uint32_t dA0 = p.sA + (uint32_t)s * p.a_stage_bytes;
    if (CONV) {
      const int per_img = p.tiles_h * p.tiles_w;
      const int img = m_tile / per_img;
      const int r = m_tile - img * per_img;
      const int ty = r / p.tiles_w;
      const int oy0 = ty * p.BH, ox0 = (r - ty * p.tiles_w) * p.BWs;
#pragma unroll
      for (int ci = 0; ci < CPS; ci++)
        tma_load_4d_p(ld, dA0 + (uint32_t)ci * p.a_blk_bytes, tmA, fb, ci * p.kblk, ox0 - p.pad_l, oy0 - p.pad_t, img);
    } else {
#pragma unroll
      for (int ci = 0; ci < CPS; ci++)
        tma_load_2d_p(ld, dA0 + (uint32_t)ci * p.a_blk_bytes, tmA, fb, ci * p.kblk, m_tile * TC_BM);
    }
    issued_mask |= 1u << s;
    last_phase = (last_phase & ~(1u << s)) | (phase << s);
    s = s + 1 == p.S ? 0 : s + 1;
    phase ^= s == 0 ? 1u : 0u;
  }
}
template <int CONV>
__device__ __forceinline__ void producer_single_cps(int cps, uint32_t ld, const ProdSingle& p, const CUtensorMap* tmA,
                                                    int tile0, int total_tiles, int tstep, uint64_t* full,
                                                    uint64_t* empty, unsigned int* err, volatile int* abort_flag,
                                                    uint32_t& issued_mask, uint32_t& last_phase) {
  if (cps == 1) producer_single_loop<CONV, 1>(ld, p, tmA, tile0, total_tiles, tstep, full, empty, err, abort_flag, issued_mask, last_phase);
  else if (cps == 2) producer_single_loop<CONV, 2>(ld, p, tmA, tile0, total_tiles, tstep, full, empty, err, abort_flag, issued_mask, last_phase);
  else if (cps == 3) producer_single_loop<CONV, 3>(ld, p, tmA, tile0, total_tiles, tstep, full, empty, err, abort_flag, issued_mask, last_phase);
  else producer_single_loop<CONV, 4>(ld, p, tmA, tile0, total_tiles, tstep, full, empty, err, abort_flag, issued_mask, last_phase);
}

struct MmaSingle {
  uint32_t d0, acc_stride, sA, a_stage_bytes, a_blk16, b_cb16, b_nt16, b_lo16, idesc, a_tap16, b_tap16;
  uint64_t dconst, bd0;
  int S, nacc, n_tiles, nt_step, nt0;
};
template <int BT, int NK, bool TWO, int CPS>
__device__ __noinline__ void mma_single_loop(uint32_t ld, const MmaSingle m, int tile0, int total_tiles, int tstep,
                                             uint64_t* full, uint64_t* empty, uint64_t* accf, uint64_t* acce,
                                             unsigned int* err, volatile int* abort_flag) {
  int s = 0, nt = m.nt0;
  uint32_t phase = 0, acc = 0, accph = 0;
  for (int tile = tile0; tile < total_tiles; tile += tstep) {
    if (!mbar_wait_warp(smem_u32(&acce[acc]), accph ^ 1u, err, SDX_DEV_WAIT_ACC_EMPTY, abort_flag)) break;
    if (!mbar_wait_warp(smem_u32(&full[s]), phase, err, SDX_DEV_WAIT_FULL, abort_flag)) break;
    tc_fence_after();
    const uint32_t d = m.d0 + acc * m.acc_stride;
    const uint64_t ad = m.dconst | (uint64_t)(((m.sA + (uint32_t)s * m.a_stage_bytes) >> 4) & 0x3FFFu);
    const uint64_t bd = m.bd0 + (uint64_t)((uint32_t)nt * m.b_nt16);
#pragma unroll
    for (int ci = 0; ci < CPS; ci++)
      umma_stage<BT, NK, TWO>(ld, d, ad + (uint64_t)(ci * m.a_blk16), bd + (uint64_t)(ci * m.b_cb16), m.a_tap16,
                              m.b_tap16, m.b_lo16, m.idesc, ci == 0 ? 0u : 1u);
    tc_commit_p(ld, smem_u32(&empty[s]));
    tc_commit_p(ld, smem_u32(&accf[acc]));
    s = s + 1 == m.S ? 0 : s + 1;
    phase ^= s == 0 ? 1u : 0u;
    acc = acc + 1 == (uint32_t)m.nacc ? 0u : acc + 1;
    accph ^= acc == 0 ? 1u : 0u;
    nt += m.nt_step;
    nt = nt >= m.n_tiles ? nt - m.n_tiles : nt;
  }
}
template <int BT, int NK, bool TWO>
__device__ __forceinline__ void mma_single_cps(int cps, uint32_t ld, const MmaSingle& m, int tile0, int total_tiles,
                                               int tstep, uint64_t* full, uint64_t* empty, uint64_t* accf,
                                               uint64_t* acce, unsigned int* err, volatile int* abort_flag) {
  if (cps == 1) mma_single_loop<BT, NK, TWO, 1>(ld, m, tile0, total_tiles, tstep, full, empty, accf, acce, err, abort_flag);
  else if (cps == 2) mma_single_loop<BT, NK, TWO, 2>(ld, m, tile0, total_tiles, tstep, full, empty, accf, acce, err, abort_flag);
  else if (cps == 3) mma_single_loop<BT, NK, TWO, 3>(ld, m, tile0, total_tiles, tstep, full, empty, accf, acce, err, abort_flag);
  else mma_single_loop<BT, NK, TWO, 4>(ld, m, tile0, total_tiles, tstep, full, empty, accf, acce, err, abort_flag);
}

// One 16-column chunk (tile columns 16c..16c+15) of one accumulator row: bias -> + residual ->
// activation -> staging slab row `srow` (TMA store path) or global memory (fallback path).
// (g, cg) = column group of the chunk and its first column inside the group; advanced here.
template <int ACT>
__device__ __forceinline__ void epi_chunk(const TcArgs& a, float (&v)[16], int c, uint32_t srow, uint32_t xr,
                                          const float* sBias, const TileCoord& t, bool valid, int64_t pix, int& g,
                                          int& cg) {
  const int n = t.n0 + c * 16;
  if (a.bias_smem) {
    const float4* bp = reinterpret_cast<const float4*>(sBias + n);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float4 b = bp[i];
      v[4 * i] += b.x; v[4 * i + 1] += b.y; v[4 * i + 2] += b.z; v[4 * i + 3] += b.w;
    }
  } else if (a.bias) {
#pragma unroll
    for (int j = 0; j < 16; j++)
      if (n + j < a.N) v[j] += __ldg(a.bias + (a.convt_oc > 0 ? (n + j) % a.convt_oc : n + j));
  }
  if (a.tma_out) {
    const uint32_t row = srow + (uint32_t)g * a.group_bytes;
    const uint32_t k0 = ((uint32_t)cg * (uint32_t)a.esz) >> 4;  // first 16-byte unit of the chunk
    if (a.esz == 2) {
      const uint32_t ad0 = row + (((k0) ^ xr) << 4), ad1 = row + (((k0 + 1u) ^ xr) << 4);
      if (a.tma_res) {
        uint4 u0, u1;
        lds16(ad0, u0);
        lds16(ad1, u1);
        const __half2* h0 = reinterpret_cast<const __half2*>(&u0);
        const __half2* h1 = reinterpret_cast<const __half2*>(&u1);
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const float2 f0 = __half22float2(h0[i]), f1 = __half22float2(h1[i]);
          v[2 * i] += f0.x; v[2 * i + 1] += f0.y;
          v[8 + 2 * i] += f1.x; v[8 + 2 * i + 1] += f1.y;
        }
      } else if (a.res && valid && n + 16 <= a.N) {
        float r8[8];
        load8_res(a, pix * a.res_pix_stride + a.res_ch_off + n, r8);
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] += r8[j];
        load8_res(a, pix * a.res_pix_stride + a.res_ch_off + n + 8, r8);
#pragma unroll
        for (int j = 0; j < 8; j++) v[8 + j] += r8[j];
      }
      uint4 u0, u1;
      __half2* h0 = reinterpret_cast<__half2*>(&u0);
      __half2* h1 = reinterpret_cast<__half2*>(&u1);
#pragma unroll
      for (int i = 0; i < 4; i++) {
        h0[i] = __floats2half2_rn(act_t<ACT>(v[2 * i]), act_t<ACT>(v[2 * i + 1]));
        h1[i] = __floats2half2_rn(act_t<ACT>(v[8 + 2 * i]), act_t<ACT>(v[8 + 2 * i + 1]));
      }
      sts16(ad0, u0);
      sts16(ad1, u1);
    } else {
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const uint32_t ad = row + (((k0 + (uint32_t)k) ^ xr) << 4);
        float* w = v + 4 * k;
        if (a.tma_res) {
          uint4 u;
          lds16(ad, u);
          w[0] += __uint_as_float(u.x); w[1] += __uint_as_float(u.y);
          w[2] += __uint_as_float(u.z); w[3] += __uint_as_float(u.w);
        } else if (a.res && valid && n + 16 <= a.N) {
#pragma unroll
          for (int j = 0; j < 4; j++) {
            const int64_t ro = pix * a.res_pix_stride + a.res_ch_off + n + 4 * k + j;
            w[j] += a.res_f32 ? static_cast<const float*>(a.res)[ro] : __half2float(static_cast<const __half*>(a.res)[ro]);
          }
        }
        uint4 u;
        u.x = __float_as_uint(act_t<ACT>(w[0])); u.y = __float_as_uint(act_t<ACT>(w[1]));
        u.z = __float_as_uint(act_t<ACT>(w[2])); u.w = __float_as_uint(act_t<ACT>(w[3]));
        sts16(ad, u);
      }
    }
    cg += 16;
    if (cg >= a.G) {
      cg -= a.G;
      g++;
    }
    return;
  }
  // ---- fallback: per-thread global stores
  if (!valid) return;
#pragma unroll
  for (int j0 = 0; j0 < 16; j0 += 8) {
    const int nn = n + j0;
    if (nn >= a.N) continue;
    float* vg = v + j0;
    int64_t opix;
    int och;
    out_coord(a, pix, nn, opix, och);
    if (a.vec_ok && nn + 8 <= a.N) {
      if (a.res) {
        float r8[8];
        load8_res(a, opix * a.res_pix_stride + a.res_ch_off + och, r8);
#pragma unroll
        for (int j = 0; j < 8; j++) vg[j] += r8[j];
      }
#pragma unroll
      for (int j = 0; j < 8; j++) vg[j] = act_t<ACT>(vg[j]);
      store8(a, opix * a.out_pix_stride + a.out_ch_off + och, vg);
    } else {
#pragma unroll
      for (int j = 0; j < 8; j++) {
        if (nn + j >= a.N) continue;
        int64_t op;
        int oc;
        out_coord(a, pix, nn + j, op, oc);
        float x = vg[j];
        if (a.res) {
          const int64_t ro = op * a.res_pix_stride + a.res_ch_off + oc;
          x += a.res_f32 ? static_cast<const float*>(a.res)[ro] : __half2float(static_cast<const __half*>(a.res)[ro]);
        }
        x = act_t<ACT>(x);
        const int64_t oo = op * a.out_pix_stride + a.out_ch_off + oc;
        if (a.out_f32) static_cast<float*>(a.out)[oo] = x;
        else static_cast<__half*>(a.out)[oo] = __float2half_rn(x);
      }
    }
  }
}

// (a0, a1) += h * (w0, w1) as one packed f32x2 FMA (sm_100); each lane is the single-rounding fmaf.
__device__ __forceinline__ void ffma2_pair(float& a0, float& a1, float h, float w0, float w1) {
  asm("{\n\t.reg .b64 ra, rh, rw;\n\t"
      "mov.b64 ra, {%0, %1};\n\tmov.b64 rh, {%2, %2};\n\tmov.b64 rw, {%3, %4};\n\t"
      "fma.rn.f32x2 ra, rh, rw, ra;\n\tmov.b64 {%0, %1}, ra;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(h), "f"(w0), "f"(w1));
}

// Two-float packed add (sm_100 f32x2 pipe: one instruction for both lanes of the pair).
__device__ __forceinline__ float2 add_f32x2(float2 a, float2 b) {
  uint64_t x, y, d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(a.x), "f"(a.y));
  asm("mov.b64 %0, {%1, %2};" : "=l"(y) : "f"(b.x), "f"(b.y));
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(x), "l"(y));
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(d));
  return r;
}

// Channel sums of one warp's 32 staged output rows (fp16, the fast epilogue's swizzled staging: BN
// columns in groups of G = min(BN, 64), row pitch P = 2G bytes) into gp[0 .. nlim). Lane l sums the
// column pair j = l % NP over rows l / NP + R * i (NP = min(BN / 2, 32) pairs side by side, R = 32 /
// NP rows per step), 4-byte loads; the swizzle term of those rows is a compile-time function of i, so
// each load is one instruction off a per-lane base. Lanes that share a pair then combine (offsets
// NP .. 16). BN = 128: two pairs per lane (one per 64-column group).
template <int BN>
__device__ __forceinline__ void gap_warp_rows(uint32_t slab, uint32_t group_bytes, int lane, float* gp, int nlim) {
  constexpr int G = BN < 64 ? BN : 64;
  constexpr int P = 2 * G;
  constexpr int XM = P / 16 - 1;  // swizzle mask of the 16-byte unit index
  constexpr int NP = BN / 2 < 32 ? BN / 2 : 32;
  constexpr int R = 32 / NP;
  constexpr int NG = BN / 2 / NP;  // pairs per lane: 1, or 2 for BN = 128
  constexpr int IT = 32 / R;       // row steps
  const int j = lane % NP, r0 = lane / NP;
  const uint32_t byte = (uint32_t)(2 * j * 2) % (uint32_t)P;  // pair's byte offset inside its group row
  const uint32_t k = byte >> 4, inner = byte & 15u;
  // per-lane address of row r0 for each swizzle term c (the term of row r0 + R * i is c = ((r0 + R * i)
  // * P >> 7) & XM; with r0 < R it depends on i only)
  uint32_t base[XM + 1];
#pragma unroll
  for (int c = 0; c <= XM; c++) base[c] = slab + (uint32_t)r0 * P + (((k ^ (uint32_t)c) << 4) | inner);
  float2 acc[NG];
#pragma unroll
  for (int g = 0; g < NG; g++) acc[g] = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int i = 0; i < IT; i++) {
    const int c = (((R * i) * P) >> 7) & XM;
#pragma unroll
    for (int g = 0; g < NG; g++) {
      uint32_t w;
      asm volatile("ld.shared.b32 %0, [%1];" : "=r"(w) : "r"(base[c] + (uint32_t)g * group_bytes + (uint32_t)(R * i * P)));
      acc[g] = add_f32x2(acc[g], __half22float2(*reinterpret_cast<const __half2*>(&w)));
    }
  }
#pragma unroll
  for (int off = NP; off < 32; off *= 2)
#pragma unroll
    for (int g = 0; g < NG; g++) {
      acc[g].x += __shfl_xor_sync(0xffffffffu, acc[g].x, off);
      acc[g].y += __shfl_xor_sync(0xffffffffu, acc[g].y, off);
    }
  if (r0 == 0) {
#pragma unroll
    for (int g = 0; g < NG; g++) {
      const int col = 2 * (j + g * NP);
      if (col < nlim) *reinterpret_cast<float2*>(gp + col) = acc[g];
    }
  }
}

// Fast form of epi_chunk (kernel template EPI = 1): fp16 output through swizzled staging and TMA
// stores, the bias (zeros when absent) in shared memory, the residual (if any) TMA-staged. The code
// is straight-line, so the sixteen columns interleave; `sb` is the tile's bias (sBias + n0).
template <int ACT>
__device__ __forceinline__ void epi_chunk_fast(const TcArgs& a, float (&v)[16], int c, uint32_t srow, uint32_t xr,
                                               const float* sb, bool res_smem) {
  const int col = c * 16;
  const uint32_t row = srow + (uint32_t)(col >> a.log2G) * a.group_bytes;
  const uint32_t k0 = ((uint32_t)(col & (a.G - 1)) * 2u) >> 4;
  const uint32_t ad0 = row + ((k0 ^ xr) << 4), ad1 = row + (((k0 + 1u) ^ xr) << 4);
  const float4* bp = reinterpret_cast<const float4*>(sb + col);
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const float4 b = bp[i];
    v[4 * i] += b.x; v[4 * i + 1] += b.y; v[4 * i + 2] += b.z; v[4 * i + 3] += b.w;
  }
  if (res_smem) {
    uint4 u0, u1;
    lds16(ad0, u0);
    lds16(ad1, u1);
    const __half2* h0 = reinterpret_cast<const __half2*>(&u0);
    const __half2* h1 = reinterpret_cast<const __half2*>(&u1);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float2 f0 = __half22float2(h0[i]), f1 = __half22float2(h1[i]);
      v[2 * i] += f0.x; v[2 * i + 1] += f0.y;
      v[8 + 2 * i] += f1.x; v[8 + 2 * i + 1] += f1.y;
    }
  }
#pragma unroll
  for (int i = 0; i < 16; i++) v[i] = act_t<ACT>(v[i]);
  uint4 u0, u1;
  __half2* h0 = reinterpret_cast<__half2*>(&u0);
  __half2* h1 = reinterpret_cast<__half2*>(&u1);
#pragma unroll
  for (int i = 0; i < 4; i++) {
    h0[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    h1[i] = __floats2half2_rn(v[8 + 2 * i], v[8 + 2 * i + 1]);
  }
  sts16(ad0, u0);
  sts16(ad1, u1);
}

// ConvT chain epilogue for one accumulator row = input pixel (y, x): the 4 x OC1 columns (tap1, c)
// of the first 2x2 ConvT come out of TMEM under one wait; each channel c (+ bias, activation) of
// each tap1 feeds the second 2x2 ConvT (one output channel), so the row yields the 4 x 4 output
// block at (4y, 4x): 16 independent FMA chains over c, stored as four 16-byte rows (fp32) or 8-byte
// rows (fp16). smem: sBias[c] = first bias, then the second ConvT's raw weights [c][tap2] and bias.
template <int ACT, int OC1>  // OC1 in {8, 16, 24}: 2 x OC1 columns = whole 16-column TMEM loads
__device__ __forceinline__ void chain_row(const TcArgs& a, uint32_t tbase, const float* sBias, uint64_t* acce_bar,
                                          int img, int y, int x, bool ok) {
  const float4* w2 = reinterpret_cast<const float4*>(sBias + a.BN);
  const float b2 = sBias[a.BN + 4 * OC1];
  float blk[16];
#pragma unroll
  for (int i = 0; i < 16; i++) blk[i] = b2;
  // two halves of two taps each (48 registers of accumulator at a time, so four epilogue groups fit)
#pragma unroll
  for (int hf = 0; hf < 2; hf++) {
    float v[2 * OC1];
#pragma unroll
    for (int j = 0; j < 2 * OC1 / 16; j++) tmem_ld16_issue(tbase + (uint32_t)(hf * 2 * OC1 + 16 * j), v + 16 * j);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 2 * OC1 / 16; j++) tmem_ld_wait16(v + 16 * j);
    if (hf == 1) {
      tc_fence_before();
      mbar_arrive(smem_u32(acce_bar));
    }
#pragma unroll
    for (int c = 0; c < OC1; c++) {
      const float4 w = w2[c];
      const float bb = sBias[c];
#pragma unroll
      for (int dx1 = 0; dx1 < 2; dx1++) {
        const float h = act_t<ACT>(v[dx1 * OC1 + c] + bb);
        const int r0 = 2 * hf, c0 = 2 * dx1;  // tap1 = (hf, dx1)
        ffma2_pair(blk[r0 * 4 + c0], blk[r0 * 4 + c0 + 1], h, w.x, w.y);
        ffma2_pair(blk[(r0 + 1) * 4 + c0], blk[(r0 + 1) * 4 + c0 + 1], h, w.z, w.w);
      }
    }
  }
  if (!ok) return;
  if (a.chain_act2 == ACT_SIGMOID) {
    // the det probability map: hardware exp and reciprocal (a few ulp) instead of the IEEE forms
#pragma unroll
    for (int i = 0; i < 16; i++) blk[i] = __frcp_rn(1.0f + __expf(-blk[i]));
  } else {
#pragma unroll
    for (int i = 0; i < 16; i++) blk[i] = act_apply(blk[i], a.chain_act2);
  }
  const int64_t W4 = (int64_t)a.OW * 4;
  const int64_t base = ((int64_t)img * a.OH * 4 + (int64_t)y * 4) * W4 + (int64_t)x * 4;
#pragma unroll
  for (int r = 0; r < 4; r++) {
    if (a.chain_y_f32) {
      *reinterpret_cast<float4*>(static_cast<float*>(a.chain_y) + base + r * W4) =
          make_float4(blk[4 * r], blk[4 * r + 1], blk[4 * r + 2], blk[4 * r + 3]);
    } else {
      __half2 h0 = __floats2half2_rn(blk[4 * r], blk[4 * r + 1]);
      __half2 h1 = __floats2half2_rn(blk[4 * r + 2], blk[4 * r + 3]);
      uint2 u;
      u.x = *reinterpret_cast<uint32_t*>(&h0);
      u.y = *reinterpret_cast<uint32_t*>(&h1);
      *reinterpret_cast<uint2*>(static_cast<__half*>(a.chain_y) + base + r * W4) = u;
    }
  }
}

template <int ACT, int EPI, int G>
__global__ void __launch_bounds__(tc_threads(G), 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ CUtensorMap tmRes,
                   const TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.stages;
  const uint32_t kbytes = (uint32_t)a.kblk * 2;                          // operand row bytes
  const uint32_t b_tap_bytes = (uint32_t)a.BN * kbytes;                  // one tap, one weight term
  const uint32_t b_cb_bytes = b_tap_bytes * (uint32_t)a.b_taps;          // one channel block: its taps, one term
  const uint32_t b_half_bytes = b_cb_bytes * (uint32_t)a.cps;            // one term of a stage
  const uint32_t b_stage_bytes = a.b_resident ? 0u : (uint32_t)a.wterms * b_half_bytes;
  uint8_t* sA = smem;
  uint8_t* sB = smem + (size_t)S * a.a_stage_bytes;  // resident: all weights; else S weight stages
  uint8_t* sStage = sB + (a.b_resident ? (size_t)a.b_total_bytes : (size_t)S * b_stage_bytes);
  float* sBias = reinterpret_cast<float*>(sStage + (size_t)G * a.nsbuf * a.sbuf_bytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sStage + (size_t)G * a.nsbuf * a.sbuf_bytes +
                                               (((size_t)a.bias_smem * 4 + 15) & ~(size_t)15));
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* accf = bars + 2 * S;                  // [4] accumulator full (MMA commit)
  uint64_t* acce = accf + 4;                      // [4] accumulator drained (128 epilogue threads)
  uint64_t* drain = acce + 4;
  uint64_t* resb = drain + 1;                     // [group][buffer][warp] residual slab landed
  uint64_t* bres = resb + G * 2 * 4;  // resident weights landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bres + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int i = 0; i < 4; i++) {
      mbar_init(smem_u32(&accf[i]), 1);
      mbar_init(smem_u32(&acce[i]), 128);
    }
    for (int i = 0; i < G * 2 * 4; i++) mbar_init(smem_u32(&resb[i]), 1);
    mbar_init(smem_u32(drain), 1);
    mbar_init(smem_u32(bres), 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (a.tma_out) tma_prefetch_desc(&tmOut);
    if (a.tma_res) tma_prefetch_desc(&tmRes);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), a.tmem_cols);
    tmem_relinquish();
  }
  // per-column bias in shared memory (ConvT: expanded over its taps), read as broadcasts
  for (int i = threadIdx.x; i < (EPI == 4 ? a.BN : a.bias_smem); i += blockDim.x)
    sBias[i] = (a.bias && i < a.N) ? __ldg(a.bias + (a.convt_oc > 0 ? i % a.convt_oc : i)) : 0.0f;
  if (EPI == 4) {
    // second ConvT: raw weights [c][tap2] (float4 per channel), then its bias
    const int oc1 = a.convt_oc;
    for (int i = threadIdx.x; i <= 4 * oc1; i += blockDim.x)
      sBias[a.BN + i] = i < 4 * oc1 ? __ldg(a.chain_w2 + i) : __ldg(a.chain_b2);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total_tiles = a.m_tiles * a.n_tiles;
  // pipeline stages per tile: (tap, channel block), or (kx, channel block) in halo mode
  const int groups = a.kb_per_tap / a.cps;  // channel-block groups per tap
  const int kblocks = (a.halo ? a.kw : a.taps) * groups;

  // weight block (term, tap, channel block, n tile) in the resident layout
  auto b_res_off = [&](int term, int tap, int cb, int nt) -> uint32_t {
    return (uint32_t)((((term * a.taps + tap) * a.kb_per_tap + cb) * a.n_tiles + nt)) * b_tap_bytes;
  };
  // The producer and MMA loops sit on the critical path of every stage: no integer division inside
  // them (ring slot, phase, tap and channel block advance as counters). Each runs on a whole warp
  // (warp-uniform values, uniform registers) and issues its copies / MMAs from the elected lane.
  if (warp == 0) {
    const uint32_t ld = elect_leader();
    {
      uint32_t issued_mask = 0;  // ring slots that received at least one copy
      uint32_t last_phase = 0;   // bit s: phase of the last copy into slot s
      bool ok = true;
      if (a.b_resident) {
        // every weight block once, onto one barrier
        const uint32_t bb = smem_u32(bres);
        mbar_arrive_expect_tx_p(ld, bb, a.b_total_bytes);
        for (int term = 0; term < a.wterms; term++)
          for (int tap = 0; tap < a.taps; tap++)
            for (int cb = 0; cb < a.kb_per_tap; cb++)
              for (int nt = 0; nt < a.n_tiles; nt++)
                tma_load_2d_p(ld, smem_u32(sB) + b_res_off(term, tap, cb, nt), &tmB, bb, cb * a.kblk,
                            (term * a.taps + tap) * a.b_rows_per_tap + nt * a.BN);
      }
      int s = 0;
      uint32_t phase = 0;
      // single-stage tiles with resident weights (pointwise, kx-in-N 3x3, ConvT): the dispatch-free
      // loop; a 4-D box at (ox0 - pad_l, oy0 - pad_t) covers halo mode with one column tap and the
      // one-tap conv mode alike
      if (kblocks == 1 && a.b_resident && a.cps <= 4 && (a.mode != TC_CONV || a.halo || a.taps == 1)) {
        ProdSingle ps;
        ps.sA = smem_u32(sA);
        ps.a_stage_bytes = a.a_stage_bytes;
        ps.a_blk_bytes = a.a_blk_bytes;
        ps.stage_tx = (uint32_t)a.cps * a.a_box_bytes;
        ps.S = S;
        ps.n_tiles = a.n_tiles;
        ps.tiles_h = a.tiles_h;
        ps.tiles_w = a.tiles_w;
        ps.BH = a.BH;
        ps.BWs = a.BWs;
        ps.kblk = a.kblk;
        ps.pad_l = a.pad_l;
        ps.pad_t = a.pad_t;
        if (a.mode == TC_CONV)
          producer_single_cps<1>(a.cps, ld, ps, &tmA, blockIdx.x, total_tiles, gridDim.x, full, empty, a.err, abort_flag,
                                 issued_mask, last_phase);
        else
          producer_single_cps<0>(a.cps, ld, ps, &tmA, blockIdx.x, total_tiles, gridDim.x, full, empty, a.err, abort_flag,
                                 issued_mask, last_phase);
        ok = false;  // every tile issued above
      }
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        const int m_tile = a.n_tiles == 1 ? tile : tile / a.n_tiles;
        const int n_tile = tile - m_tile * a.n_tiles;
        int img = 0, oy0 = 0, ox0 = 0;
        if (a.mode == TC_CONV) {
          const int per_img = a.tiles_h * a.tiles_w;
          img = m_tile / per_img;
          const int r = m_tile - img * per_img;
          const int ty = r / a.tiles_w;
          oy0 = ty * a.BH;
          ox0 = (r - ty * a.tiles_w) * a.BWs;
        }
        int tk = 0, cg = 0;  // tk: tap, or kx in halo mode; cg: channel-block group
        for (int kb = 0; kb < kblocks; kb++) {
          if (!mbar_wait_warp(smem_u32(&empty[s]), phase ^ 1u, a.err, SDX_DEV_WAIT_EMPTY, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&full[s]);
          mbar_arrive_expect_tx_p(ld, fb, (uint32_t)a.cps * a.a_box_bytes + b_stage_bytes);
          const uint32_t dA0 = smem_u32(sA) + (uint32_t)s * a.a_stage_bytes;
          const uint32_t dB0 = smem_u32(sB) + (uint32_t)s * b_stage_bytes;
          for (int ci = 0; ci < a.cps; ci++) {
            const int cb = cg * a.cps + ci;
            const uint32_t dA = dA0 + (uint32_t)ci * a.a_blk_bytes;
            if (a.halo) {
              // rows oy0 - pt .. oy0 - pt + BH + kh - 2 of input column block kx (zero fill = padding)
              tma_load_4d_p(ld, dA, &tmA, fb, cb * a.kblk, ox0 + tk - a.pad_l, oy0 - a.pad_t, img);
            } else if (a.mode == TC_CONV) {
              const int ky = tk / a.kw, kx = tk - ky * a.kw;
              tma_load_4d_p(ld, dA, &tmA, fb, cb * a.kblk, ox0 + kx - a.pad_l, oy0 + ky - a.pad_t, img);
            } else {
              tma_load_2d_p(ld, dA, &tmA, fb, cb * a.kblk, m_tile * TC_BM);
            }
            if (!a.b_resident) {
              const uint32_t dB = dB0 + (uint32_t)ci * b_cb_bytes;
              for (int j = 0; j < a.b_taps; j++) {
                const int tap = a.halo ? j * a.kw + tk : tk;
                const int brow = tap * a.b_rows_per_tap + n_tile * a.BN;
                tma_load_2d_p(ld, dB + j * b_tap_bytes, &tmB, fb, cb * a.kblk, brow);
                if (a.wterms == 2)
                  tma_load_2d_p(ld, dB + b_half_bytes + j * b_tap_bytes, &tmB, fb, cb * a.kblk, a.taps * a.b_rows_per_tap + brow);
              }
            }
          }
          issued_mask |= 1u << s;
          last_phase = (last_phase & ~(1u << s)) | (phase << s);
          if (++cg == groups) {
            cg = 0;
            tk++;
          }
          if (++s == S) {
            s = 0;
            phase ^= 1u;
          }
        }
      }
      // wind-down: every issued copy must land before the CTA's shared memory goes away
      for (int q = 0; q < S; q++)
        if (issued_mask & (1u << q))
          mbar_wait_drain(smem_u32(&full[q]), (last_phase >> q) & 1u, a.err, SDX_DEV_WAIT_DRAIN);
      if (a.b_resident) mbar_wait_drain(smem_u32(bres), 0, a.err, SDX_DEV_WAIT_DRAIN);
    }
    __syncwarp();
  } else if (warp == 1) {
    const uint32_t ld = elect_leader();
    {
      const uint32_t idesc = umma_idesc_f16(TC_BM, a.BN);
      const int nk = a.kblk / 16;  // MMA k-steps per block
      // descriptor words: the high word (stride offset, version, swizzle) and the leading-offset
      // bits are the same for every operand; only the start address changes
      const uint64_t dconst = umma_desc_kmajor(0u, kbytes);
      const uint32_t sB_addr = smem_u32(sB);
      // strides in 16-byte descriptor units: A rows of the next row tap (halo), the next tap's
      // weights (resident: kw taps on in the [tap][cb][n_tile] layout; streamed: the next block),
      // and the lo weight term
      const uint32_t a_tap16 = ((uint32_t)a.BW * kbytes) >> 4;
      const uint32_t b_tap16 = a.b_resident ? (b_res_off(0, a.kw, 0, 0) >> 4) : (b_tap_bytes >> 4);
      const uint32_t b_cb = a.b_resident ? b_res_off(0, 0, 1, 0) : b_cb_bytes;  // next channel block
      const uint32_t b_lo16 = (a.b_resident ? b_res_off(1, 0, 0, 0) : b_half_bytes) >> 4;
      bool ok = !a.b_resident || mbar_wait_warp(smem_u32(bres), 0, a.err, SDX_DEV_WAIT_FULL, abort_flag);
      if (ok) tc_fence_after();
      int s = 0;
      uint32_t phase = 0;
      uint32_t acc = 0, accph = 0;
      // one-tap tiles (pointwise), and the kx-in-N 3x3 convs (three row taps, one weight term)
      const bool single = kblocks == 1 && a.b_resident && (a.b_taps == 1 || (a.b_taps == 3 && a.wterms == 1)) &&
                          a.cps <= 4 && (nk == 1 || nk == 2 || nk == 4);
      if (ok && single) {
        MmaSingle m;
        m.d0 = tmem_base;
        m.acc_stride = (uint32_t)a.acc_stride;
        m.sA = smem_u32(sA);
        m.a_stage_bytes = a.a_stage_bytes;
        m.a_blk16 = a.a_blk_bytes >> 4;
        m.b_cb16 = b_cb >> 4;
        m.b_nt16 = b_res_off(0, 0, 0, 1) >> 4;
        m.b_lo16 = b_lo16;
        m.a_tap16 = a_tap16;
        m.b_tap16 = b_tap16;
        m.idesc = idesc;
        m.dconst = dconst;
        m.bd0 = dconst | (uint64_t)((sB_addr >> 4) & 0x3FFFu);
        m.S = S;
        m.nacc = a.nacc;
        m.n_tiles = a.n_tiles;
        m.nt_step = (int)(gridDim.x % (unsigned)a.n_tiles);
        m.nt0 = (int)(blockIdx.x % (unsigned)a.n_tiles);
        const int tt = a.m_tiles * a.n_tiles;
        if (a.b_taps == 3) {
          if (nk == 1) mma_single_cps<3, 1, false>(a.cps, ld, m, blockIdx.x, tt, gridDim.x, full, empty, accf, acce, a.err, abort_flag);
          else if (nk == 2) mma_single_cps<3, 2, false>(a.cps, ld, m, blockIdx.x, tt, gridDim.x, full, empty, accf, acce, a.err, abort_flag);
          else mma_single_cps<3, 4, false>(a.cps, ld, m, blockIdx.x, tt, gridDim.x, full, empty, accf, acce, a.err, abort_flag);
        } else if (a.wterms == 2) {
          if (nk == 1) mma_single_cps<1, 1, true>(a.cps, ld, m, blockIdx.x, tt, gridDim.x, full, empty, accf, acce, a.err, abort_flag);
          else if (nk == 2) mma_single_cps<1, 2, true>(a.cps, ld, m, blockIdx.x, tt, gridDim.x, full, empty, accf, acce, a.err, abort_flag);
          else mma_single_cps<1, 4, true>(a.cps, ld, m, blockIdx.x, tt, gridDim.x, full, empty, accf, acce, a.err, abort_flag);
        } else {
          if (nk == 1) mma_single_cps<1, 1, false>(a.cps, ld, m, blockIdx.x, tt, gridDim.x, full, empty, accf, acce, a.err, abort_flag);
          else if (nk == 2) mma_single_cps<1, 2, false>(a.cps, ld, m, blockIdx.x, tt, gridDim.x, full, empty, accf, acce, a.err, abort_flag);
          else mma_single_cps<1, 4, false>(a.cps, ld, m, blockIdx.x, tt, gridDim.x, full, empty, accf, acce, a.err, abort_flag);
        }
        ok = false;  // the loop above ran every tile
      }
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        const int n_tile = a.n_tiles == 1 ? 0 : tile % a.n_tiles;
        if (!mbar_wait_warp(smem_u32(&acce[acc]), accph ^ 1u, a.err, SDX_DEV_WAIT_ACC_EMPTY, abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + acc * (uint32_t)a.acc_stride;
        int tk = 0, cg = 0;
        uint32_t first = 0;  // 0 until the tile's first MMA (overwrite), then 1 (accumulate)
        for (int kb = 0; kb < kblocks; kb++) {
          if (!mbar_wait_warp(smem_u32(&full[s]), phase, a.err, SDX_DEV_WAIT_FULL, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // per channel block: descriptors of its first tap; the other taps are constant strides away
          uint32_t sa = smem_u32(sA) + (uint32_t)s * a.a_stage_bytes;
          uint32_t b0 = a.b_resident ? sB_addr + b_res_off(0, tk, cg * a.cps, n_tile)
                                     : sB_addr + (uint32_t)s * b_stage_bytes;
          for (int ci = 0; ci < a.cps; ci++, sa += a.a_blk_bytes, b0 += b_cb) {
            const uint64_t ad = dconst | (uint64_t)((sa >> 4) & 0x3FFFu);
            const uint64_t bd = dconst | (uint64_t)((b0 >> 4) & 0x3FFFu);
            if (a.wterms == 2) umma_stage_dispatch<true>(ld, a.b_taps, nk, d, ad, bd, a_tap16, b_tap16, b_lo16, idesc, first);
            else umma_stage_dispatch<false>(ld, a.b_taps, nk, d, ad, bd, a_tap16, b_tap16, b_lo16, idesc, first);
            first = 1u;
          }
          tc_commit_p(ld, smem_u32(&empty[s]));
          if (++cg == groups) {
            cg = 0;
            tk++;
          }
          if (++s == S) {
            s = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit_p(ld, smem_u32(&accf[acc]));
        if (++acc == (uint32_t)a.nacc) {
          acc = 0;
          accph ^= 1u;
        }
      }
      // wind-down: all issued MMAs complete before TMEM / smem are released
      tc_commit_p(ld, smem_u32(drain));
      mbar_wait_drain(smem_u32(drain), 0, a.err, SDX_DEV_WAIT_DRAIN);
    }
    __syncwarp();
  } else {
    // epilogue: group e (warps 2+4e .. 5+4e) takes the tiles lt = e, e+G, ... of this CTA (G groups); warp q
    // reads TMEM lanes 32q..32q+31 (the lane quadrant it may access), i.e. tile rows 32q..32q+31
    const int e = (warp - 2) >> 2;
    const int q = warp & 3;
    const int row_in_tile = q * 32 + lane;
    const uint32_t P = (uint32_t)(a.G * a.esz);  // staging row pitch in bytes
    // 16-byte-unit XOR of this row under the 32/64/128-byte TMA swizzle (address bits 7.. of a
    // 1024-aligned slab); 0 when the staging rows are not swizzled
    const uint32_t xr = a.swz ? (((uint32_t)lane * P) >> 7) & (P / 16u - 1u) : 0u;
    const uint32_t stage0 = smem_u32(sStage) + (uint32_t)e * a.nsbuf * a.sbuf_bytes + (uint32_t)q * 32u * P;
    const int tile0 = blockIdx.x + e * gridDim.x, tstep = G * gridDim.x;
    uint32_t res_phase = 0;    // bit b: parity of the next wait on buffer b's residual barrier
    bool res_pending = false;  // a residual load is in flight into buffer (lc % nsbuf)
    const uint32_t eld = elect_leader();  // this warp's issuing lane for TMA copies and bulk groups

    auto coords = [&](int tile, TileCoord& t) {
      const int m_tile = a.n_tiles == 1 ? tile : tile / a.n_tiles;
      const int n_tile = tile - m_tile * a.n_tiles;
      t.n0 = n_tile * a.BN;
      t.img = 0;
      t.oy0 = 0;
      t.ox0 = 0;
      t.m0 = m_tile * TC_BM;
      if (a.mode == TC_CONV) {
        const int per_img = a.tiles_h * a.tiles_w;
        t.img = m_tile / per_img;
        const int r = m_tile - t.img * per_img;
        t.oy0 = (r / a.tiles_w) * a.BH;
        t.ox0 = (r % a.tiles_w) * a.BWs;
      }
    };
    // column groups of a tile that start inside the tensor (a group fully past N is skipped)
    auto groups_of = [&](const TileCoord& t) {
      return a.convt_oc > 0 ? a.ngroups : min(a.ngroups, (a.N - t.n0 + a.G - 1) / max(a.G, 1));
    };
    auto issue_res = [&](int tile, uint32_t buf) {
      TileCoord t;
      coords(tile, t);
      const int ng = groups_of(t);
      const uint32_t rb = smem_u32(&resb[(e * 2 + buf) * 4 + q]);
      const uint32_t slab = stage0 + buf * a.sbuf_bytes;
      mbar_arrive_expect_tx_p(eld, rb, (uint32_t)ng * a.slab_tx);
      for (int g = 0; g < ng; g++) warp_copy(eld, a, &tmRes, slab + g * a.group_bytes, g, q, t, true, rb);
    };
    if (a.tma_res && tile0 < total_tiles) {
      issue_res(tile0, 0);
      res_pending = true;
    }

    uint32_t lc = 0;  // this group's tile count
    for (int tile = tile0; tile < total_tiles; tile += tstep, lc++) {
      const uint32_t lt = G * lc + (uint32_t)e;
      const uint32_t acc = lt & (uint32_t)(a.nacc - 1), ar = lt >> (a.nacc == 4 ? 2 : 1);
      const uint32_t sbi = a.nsbuf == 2 ? (lc & 1u) : 0u;
      TileCoord tcd;
      coords(tile, tcd);
      const uint32_t slab = stage0 + sbi * a.sbuf_bytes;
      const uint32_t srow = slab + (uint32_t)lane * P;
      // fast epilogue, residual without a TMA map (e.g. the nearest-upsampled FPN tensor): each
      // thread copies its row's residual into its staging row (cp.async, the staging swizzle) before
      // waiting for the accumulator, so the loads overlap the wait; the chunks read it from smem
      bool res_smem = a.tma_res != 0;
      if (EPI == 1 && a.res && !a.tma_res) {
        int64_t rpix = -1;
        if (a.mode == TC_CONV) {
          const int oy = tcd.oy0 + row_in_tile / a.BW, ox = tcd.ox0 + row_in_tile % a.BW;
          if (oy < a.OH && ox < a.OW)
            rpix = a.res_up ? ((int64_t)tcd.img * (a.OH >> 1) + (oy >> 1)) * (a.OW >> 1) + (ox >> 1)
                            : ((int64_t)tcd.img * a.OH + oy) * a.OW + ox;
        } else {
          const int64_t pix = (int64_t)tcd.m0 + row_in_tile;
          if (pix < a.M) {
            if (a.res_up) {
              // 32-bit index math (a.M < 2^31 rows): 64-bit divisions cost the epilogue per tile
              const uint32_t hw = (uint32_t)a.OH * (uint32_t)a.OW, p32 = (uint32_t)pix;
              const uint32_t img = p32 / hw, rem = p32 - img * hw;
              const uint32_t y = rem / (uint32_t)a.OW, x = rem - y * (uint32_t)a.OW;
              rpix = ((int64_t)img * (a.OH >> 1) + (y >> 1)) * (a.OW >> 1) + (x >> 1);
            } else {
              rpix = pix;
            }
          }
        }
        if (rpix >= 0) {
          const __half* src = static_cast<const __half*>(a.res) + (rpix * a.res_pix_stride + a.res_ch_off + tcd.n0);
          const int units = min(a.BN, a.N - tcd.n0) >> 3;  // 16-byte units inside the tensor
          for (int u = 0; u < units; u++) {
            const uint32_t g = (uint32_t)(u >> (a.log2G - 3)), k = (uint32_t)(u & ((a.G >> 3) - 1));
            cp_async16(srow + g * a.group_bytes + ((k ^ xr) << 4), src + u * 8);
          }
        }
        cp_async_commit();
        res_smem = true;
      }
      bool ok = mbar_wait_warp(smem_u32(&accf[acc]), ar & 1u, a.err, SDX_DEV_WAIT_ACC_FULL, abort_flag);
      if (ok && a.tma_res) {
        ok = mbar_wait_warp(smem_u32(&resb[(e * 2 + sbi) * 4 + q]), (res_phase >> sbi) & 1u, a.err, SDX_DEV_WAIT_FULL,
                            abort_flag);
        if (ok) {
          res_phase ^= 1u << sbi;
          res_pending = false;
        }
      }
      if (EPI == 1 && a.res && !a.tma_res) cp_async_wait_all();
      if (!ok) break;
      __syncwarp();
      tc_fence_after();

      // output pixel of this row: only the per-thread paths (no TMA store, or a residual that TMA
      // cannot stage) need it
      bool valid = false;
      int64_t pix = 0;
      if (!a.tma_out || (a.res && !a.tma_res)) {
        if (a.mode == TC_CONV) {
          const int h = row_in_tile / a.BW, w = row_in_tile - h * a.BW;
          const int oy = tcd.oy0 + h, ox = tcd.ox0 + w;
          valid = oy < a.OH && ox < a.OW;
          pix = ((int64_t)tcd.img * a.OH + oy) * a.OW + ox;
        } else {
          pix = (int64_t)tcd.m0 + row_in_tile;
          valid = pix < a.M;
        }
      }
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + acc * (uint32_t)a.acc_stride;
      if (EPI == 4) {
        const int y = tcd.oy0 + row_in_tile / a.BW, x = tcd.ox0 + row_in_tile % a.BW;
        const bool ok_px = y < a.OH && x < a.OW;
        if (a.convt_oc == 24) chain_row<ACT, 24>(a, tbase, sBias, acce + acc, tcd.img, y, x, ok_px);
        else if (a.convt_oc == 16) chain_row<ACT, 16>(a, tbase, sBias, acce + acc, tcd.img, y, x, ok_px);
        else chain_row<ACT, 8>(a, tbase, sBias, acce + acc, tcd.img, y, x, ok_px);
        __syncwarp();
        continue;
      }
      if (EPI == 2) {
        // kx-in-N, straight-line form (fp16 out, 16-byte rows, no residual, bias or zeros in smem):
        // per 16 output channels, the three taps' columns are loaded with one wait, combined across
        // neighbouring lanes (rows x-1, x, x+1), biased, activated and stored as two 16-byte words
        const int x = row_in_tile & (a.BW - 1), h = row_in_tile >> (a.BW == 16 ? 4 : 5);
        const int oy = tcd.oy0 + h, ox = tcd.ox0 - 1 + x;
        const bool st_ok = x >= 1 && x <= a.BW - 2 && oy < a.OH && ox < a.OW;
        __half* outp = static_cast<__half*>(a.out) +
                       ((((int64_t)tcd.img * a.OH + oy) * a.OW + ox) * a.out_pix_stride + a.out_ch_off);
        const int halves = a.N > 16 ? 2 : 1;
#pragma unroll
        for (int hf = 0; hf < 2; hf++) {
          if (hf < halves) {
            float v0[16], v1[16], v2[16];
            tmem_ld16_issue(tbase + (uint32_t)(hf * 16), v0);
            tmem_ld16_issue(tbase + (uint32_t)(32 + hf * 16), v1);
            tmem_ld16_issue(tbase + (uint32_t)(64 + hf * 16), v2);
            tmem_wait_ld();
            tmem_ld_wait16(v0);
            tmem_ld_wait16(v1);
            tmem_ld_wait16(v2);
            if (hf == halves - 1) {
              tc_fence_before();
              mbar_arrive(smem_u32(&acce[acc]));
            }
            const float4* bp = reinterpret_cast<const float4*>(sBias + hf * 16);
            uint4 w2[2];
            __half2* hp = reinterpret_cast<__half2*>(w2);
#pragma unroll
            for (int i = 0; i < 16; i += 4) {
              const float4 b = bp[i / 4];
              const float bb[4] = {b.x, b.y, b.z, b.w};
              float y[4];
#pragma unroll
              for (int j = 0; j < 4; j++)
                y[j] = act_t<ACT>(__shfl_up_sync(0xffffffffu, v0[i + j], 1) + v1[i + j] +
                                  __shfl_down_sync(0xffffffffu, v2[i + j], 1) + bb[j]);
              hp[i / 2] = __floats2half2_rn(y[0], y[1]);
              hp[i / 2 + 1] = __floats2half2_rn(y[2], y[3]);
            }
            if (st_ok) {
              uint4* op = reinterpret_cast<uint4*>(outp + hf * 16);
              op[0] = w2[0];
              if (hf * 16 + 8 < a.N) op[1] = w2[1];
            }
          }
        }
        __syncwarp();
        continue;
      }
      if (a.kxn) {
        // kx-in-N: columns kx * 32 + oc; row x of the tile is input column ox0 - 1 + x, and the
        // output at that column is D[x - 1][kx 0] + D[x][kx 1] + D[x + 1][kx 2] (neighbouring
        // lanes: the 32 rows of a warp are consecutive columns of one or two tile rows)
        float sum[32];
#pragma unroll
        for (int i = 0; i < 32; i++) sum[i] = 0.0f;
#pragma unroll
        for (int kx = 0; kx < 3; kx++) {
          float v[32];
          tmem_ld16_issue(tbase + (uint32_t)(kx * 32), v);
          tmem_ld16_issue(tbase + (uint32_t)(kx * 32 + 16), v + 16);
          tmem_wait_ld();
          tmem_ld_wait16(v);
          tmem_ld_wait16(v + 16);
          if (kx == 2) {
            tc_fence_before();
            mbar_arrive(smem_u32(&acce[acc]));
          }
#pragma unroll
          for (int i = 0; i < 32; i++) {
            float u = v[i];
            if (kx == 0) u = __shfl_up_sync(0xffffffffu, u, 1);
            if (kx == 2) u = __shfl_down_sync(0xffffffffu, u, 1);
            sum[i] += u;
          }
        }
        const int h = row_in_tile / a.BW, x = row_in_tile - h * a.BW;
        const int oy = tcd.oy0 + h, ox = tcd.ox0 - 1 + x;
        if (x >= 1 && x <= a.BW - 2 && oy < a.OH && ox < a.OW) {
          const int64_t px = ((int64_t)tcd.img * a.OH + oy) * a.OW + ox;
#pragma unroll
          for (int o0 = 0; o0 < 32; o0 += 8) {
            if (o0 >= a.N) break;
            float r8[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
              const int o = o0 + j;
              r8[j] = sum[o0 + j] + (a.bias_smem ? sBias[o] : (a.bias && o < a.N ? __ldg(a.bias + o) : 0.0f));
            }
            if (a.vec_ok && o0 + 8 <= a.N) {
              if (a.res) {
                float q8[8];
                load8_res(a, px * a.res_pix_stride + a.res_ch_off + o0, q8);
#pragma unroll
                for (int j = 0; j < 8; j++) r8[j] += q8[j];
              }
#pragma unroll
              for (int j = 0; j < 8; j++) r8[j] = act_t<ACT>(r8[j]);
              store8(a, px * a.out_pix_stride + a.out_ch_off + o0, r8);
            } else {
#pragma unroll
              for (int j = 0; j < 8; j++) {
                const int o = o0 + j;
                if (o >= a.N) continue;
                float y = r8[j];
                if (a.res) {
                  const int64_t ro = px * a.res_pix_stride + a.res_ch_off + o;
                  y += a.res_f32 ? static_cast<const float*>(a.res)[ro]
                                 : __half2float(static_cast<const __half*>(a.res)[ro]);
                }
                y = act_t<ACT>(y);
                const int64_t oo = px * a.out_pix_stride + a.out_ch_off + o;
                if (a.out_f32) static_cast<float*>(a.out)[oo] = y;
                else static_cast<__half*>(a.out)[oo] = __float2half_rn(y);
              }
            }
          }
        }
        __syncwarp();
        continue;
      }
      const int nch = a.BN / 16;
      int g = 0, cg = 0;
      // channel sums of this warp's 32 rows (rows mode): its row of a.gap, warp-uniform
      float* gp = nullptr;
      int nlim = 0;
      if (EPI == 1 && a.gap) {
        const int64_t r0 = (int64_t)tcd.m0 + q * 32;
        if (r0 < a.M) {
          gp = a.gap + (r0 >> 5) * a.N + tcd.n0;
          nlim = a.N - tcd.n0;
        }
      }
      if (EPI == 1 && nch <= 2) {
        // thin tiles: both chunks' TMEM loads in flight under one wait, the accumulator handed
        // back before any arithmetic
        float v0[16], v1[16];
        tmem_ld16_issue(tbase, v0);
        if (nch == 2) tmem_ld16_issue(tbase + 16u, v1);
        tmem_wait_ld();
        tmem_ld_wait16(v0);
        if (nch == 2) tmem_ld_wait16(v1);
        tc_fence_before();
        mbar_arrive(smem_u32(&acce[acc]));
        epi_chunk_fast<ACT>(a, v0, 0, srow, xr, sBias + tcd.n0, res_smem);
        if (nch == 2) epi_chunk_fast<ACT>(a, v1, 1, srow, xr, sBias + tcd.n0, res_smem);
      } else {
      // 16-column chunks through two register buffers: the load of chunk c+1 is in flight while
      // chunk c is processed; the accumulator goes back to the MMA warp after its last load
      float va[16], vb[16];
      tmem_ld16_issue(tbase, va);
      for (int c = 0; c < nch; c += 2) {
        tmem_wait_ld();
        tmem_ld_wait16(va);
        if (c + 1 < nch) {
          tmem_ld16_issue(tbase + (uint32_t)(c + 1) * 16u, vb);
        } else {
          tc_fence_before();
          mbar_arrive(smem_u32(&acce[acc]));
        }
        if (EPI == 1) epi_chunk_fast<ACT>(a, va, c, srow, xr, sBias + tcd.n0, res_smem);
        else epi_chunk<ACT>(a, va, c, srow, xr, sBias, tcd, valid, pix, g, cg);
        if (c + 1 < nch) {
          tmem_wait_ld();
          tmem_ld_wait16(vb);
          if (c + 2 < nch) {
            tmem_ld16_issue(tbase + (uint32_t)(c + 2) * 16u, va);
          } else {
            tc_fence_before();
            mbar_arrive(smem_u32(&acce[acc]));
          }
          if (EPI == 1) epi_chunk_fast<ACT>(a, vb, c + 1, srow, xr, sBias + tcd.n0, res_smem);
          else epi_chunk<ACT>(a, vb, c + 1, srow, xr, sBias, tcd, valid, pix, g, cg);
        }
      }
      }
      if (a.tma_out) {
        // make this warp's generic-proxy staging writes visible to the TMA engine, store its rows
        fence_async_smem();
        __syncwarp();
        {
          const int ng = groups_of(tcd);
          for (int gg = 0; gg < ng; gg++) warp_copy(eld, a, &tmOut, slab + gg * a.group_bytes, gg, q, tcd, false, 0);
          bulk_commit(eld);
          // channel sums of the staged rows (read alongside the store's own reads of them)
          if (EPI == 1 && gp) {
            if (a.BN == 16) gap_warp_rows<16>(slab, a.group_bytes, lane, gp, nlim);
            else if (a.BN == 32) gap_warp_rows<32>(slab, a.group_bytes, lane, gp, nlim);
            else if (a.BN == 64) gap_warp_rows<64>(slab, a.group_bytes, lane, gp, nlim);
            else gap_warp_rows<128>(slab, a.group_bytes, lane, gp, nlim);
          }
          // the next tile's buffer is free once the store that last read it has read it; then its
          // residual rows can be fetched while this warp waits for the next accumulator
          if (tile + tstep < total_tiles) {
            if (a.nsbuf == 2) bulk_wait_read1(eld);
            else bulk_wait_read0(eld);
            if (a.tma_res) {
              issue_res(tile + tstep, a.nsbuf == 2 ? ((lc + 1) & 1u) : 0u);
              res_pending = true;
            }
          }
        }
      }
      __syncwarp();
    }
    {
      if (res_pending) {
        // wind-down after an abort: the residual copy in flight must land before smem goes away
        const uint32_t buf = a.nsbuf == 2 ? (lc & 1u) : 0u;
        mbar_wait_drain(smem_u32(&resb[(e * 2 + buf) * 4 + q]), (res_phase >> buf) & 1u, a.err, SDX_DEV_WAIT_DRAIN);
      }
      if (a.tma_out) bulk_wait_all(eld);
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, a.tmem_cols);
  }
}

// ------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------
// N tile: ceil(N / 128) tiles of equal width, each rounded up to 16 columns (96 -> one 96-column
// tile, 192 -> two of 96), so that no MMA column or epilogue chunk is spent past N when N is not a
// power of two.
void tc_plan_n(int N, int* BN, int* n_tiles) {
  const int nt = (N + 127) / 128;
  *n_tiles = nt;
  *BN = ((N + nt - 1) / nt + 15) / 16 * 16;
}

// ConvT columns (dy, dx, o), tap-major: one tile holds whole dy rows (kw*OC <= 64) or 128-column
// pieces of one dy row.
void tc_plan_n_convt(int kh, int kw, int OC, int* BN, int* n_tiles) {
  const int N = kh * kw * OC;
  const int row = kw * OC;
  if (row <= 64 && N <= 256 && N % 16 == 0) {
    *BN = N;
    *n_tiles = 1;
  } else if (row % 128 == 0) {
    *BN = 128;
    *n_tiles = N / 128;
  } else if (N <= 64) {
    *BN = (N + 15) / 16 * 16;
    *n_tiles = 1;
  } else {
    *BN = 128;
    *n_tiles = (N + 127) / 128;
  }
}

static uint32_t pow2_cols(int cols) {
  uint32_t c = 32;
  while ((int)c < cols) c <<= 1;
  return c;
}

// Conv output tile: BW x BH = 128 pixels with BW a power of two (so each epilogue warp's 32 rows
// form one TMA box) and BW >= min_w, the one that wastes the fewest MMA rows; among equals the one
// whose input box with `halo` extra rows re-reads the least, then the wider one.
static void pick_pixel_tile(int OH, int OW, int min_w, int halo, int* BH, int* BW) {
  double best = -1, best_over = 0;
  int bh = TC_BM / 128, bw = 128;
  for (int w = 128; w >= min_w; w >>= 1) {
    const int h = TC_BM / w;
    const int tw = (OW + w - 1) / w, th = (OH + h - 1) / h;
    const double util = (double)OH * OW / ((double)tw * th * TC_BM);
    const double over = (double)(h + halo) / h;
    if (util > best + 1e-9 || (util > best - 1e-9 && over < best_over - 1e-9)) {
      best = util;
      best_over = over;
      bh = h;
      bw = w;
    }
  }
  *BH = bh;
  *BW = bw;
}

static int encode_map(CUtensorMap* map, const void* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                      const uint32_t* box, CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                      CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  PFN_encodeTiled enc = get_encode_tiled();
  if (!enc) return set_error(SDX_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  uint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = enc(map, dt, (cuuint32_t)rank, const_cast<void*>(base), reinterpret_cast<const cuuint64_t*>(dims),
                   reinterpret_cast<const cuuint64_t*>(strides_bytes), reinterpret_cast<const cuuint32_t*>(box),
                   reinterpret_cast<const cuuint32_t*>(estr), CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(SDX_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return SDX_OK;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <int ACT, int EPI, int G>
static int launch_tc(int dev, int grid, size_t smem, cudaStream_t stream, const CUtensorMap& mA, const CUtensorMap& mB,
                     const CUtensorMap& mOut, const CUtensorMap& mRes, const TcArgs& a) {
  static SmemAttr attr{};
  const int rc = raise_smem_limit(attr, (const void*)conv_tc_kernel<ACT, EPI, G>, TC_SMEM_LIMIT,
                                  "cudaFuncSetAttribute(conv_tc)");
  if (rc) return rc;
  conv_tc_kernel<ACT, EPI, G><<<grid, tc_threads(G), smem, stream>>>(mA, mB, mOut, mRes, a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "conv_tc launch");
  return SDX_OK;
}

// Channel block of a K-long reduction: 64 channels (128-byte rows) when K pads to a multiple of 64,
// else 32 or 16, so at most 15 zero channels are padded in.
int tc_kblk(int K) {
  const int r = (K + 15) / 16 * 16;
  return r % 64 == 0 ? 64 : r % 32 == 0 ? 32 : 16;
}

static int tc_kpad(int K) {
  const int kb = tc_kblk(K);
  return (K + kb - 1) / kb * kb;
}

static CUtensorMapSwizzle swizzle_of(int row_bytes) {
  return row_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : row_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                                          : CU_TENSOR_MAP_SWIZZLE_32B;
}

static size_t b_stage_bytes_of(const TcArgs& a) {
  return a.b_resident ? 0 : (size_t)a.wterms * a.cps * a.b_taps * a.BN * a.kblk * 2;
}

static size_t smem_fixed(const TcArgs& a) {
  return 1024 + (size_t)a.egroups * a.nsbuf * a.sbuf_bytes + (((size_t)a.bias_smem * 4 + 15) & ~(size_t)15) +
         8 * (2 * TC_MAX_STAGES + 10 + 8 * TC_EPI_GROUPS_MAX) + 16 + (a.b_resident ? (size_t)a.b_total_bytes : 0);
}

static size_t smem_bytes(const TcArgs& a) {
  return smem_fixed(a) + (size_t)a.stages * (a.a_stage_bytes + b_stage_bytes_of(a));
}

int tc_launch(const TcProblem& p, cudaStream_t stream) {
  if (p.N <= 0 || p.K <= 0) return set_error(SDX_ERR_INVALID, "tc: empty problem");
  if (!aligned16(p.a) || !aligned16(p.w)) return set_error(SDX_ERR_INVALID, "tc: operands must be 16-byte aligned");
  const bool convt = p.convt_oc > 0;
  int BN, n_tiles;
  if (convt) tc_plan_n_convt(p.convt_kh, p.convt_kw, p.convt_oc, &BN, &n_tiles);
  else if (p.kxn) BN = 96, n_tiles = 1;
  else tc_plan_n(p.N, &BN, &n_tiles);
  const int kblk = tc_kblk(p.K), kpad = tc_kpad(p.K);
  const int kbytes = kblk * 2;
  TcArgs a;
  memset(&a, 0, sizeof(a));
  a.mode = p.mode;
  a.N = p.N;
  a.BN = BN;
  a.n_tiles = n_tiles;
  a.kblk = kblk;
  a.kb_per_tap = kpad / kblk;
  a.wterms = p.wterms == 1 ? 1 : 2;
  a.taps = p.mode == TC_CONV ? p.kh * p.kw : 1;
  a.kw = p.kw;
  a.pad_t = p.pad_t;
  a.pad_l = p.pad_l;
  a.b_rows_per_tap = BN * n_tiles;
  if (BN > 256) return set_error(SDX_ERR_INVALID, "tc: N tile above 256 columns");
  a.acc_stride = BN;
  a.nacc = 4 * BN <= 512 ? 4 : 2;
  a.tmem_cols = pow2_cols(a.nacc * BN);
  a.bias = p.bias;
  a.res = p.res;
  a.res_f32 = p.res_f32;
  a.res_pix_stride = p.res_pix_stride;
  a.res_ch_off = p.res_ch_off;
  a.res_up = p.res_up;
  a.gap = p.gap;
  a.out = p.out;
  a.out_f32 = p.out_f32;
  a.out_pix_stride = p.out_pix_stride;
  a.out_ch_off = p.out_ch_off;
  a.act = p.act;
  a.err = p.err;
  a.convt_kh = p.convt_kh;
  a.convt_kw = p.convt_kw;
  a.convt_oc = p.convt_oc;
  a.convt_H = p.convt_H;
  a.convt_W = p.convt_W;
  const bool chain = p.chain_w2 != nullptr;
  if (chain) {
    if (!convt || p.mode != TC_CONV || p.convt_kh != 2 || p.convt_kw != 2 ||
        (p.convt_oc != 8 && p.convt_oc != 16 && p.convt_oc != 24) || BN != 4 * p.convt_oc ||
        n_tiles != 1 || !p.chain_b2 || !p.chain_y)
      return set_error(SDX_ERR_NOT_SUPPORTED, "tc convt chain: first ConvT must be 2x2 with 8, 16 or 24 outputs");
    a.chain_w2 = p.chain_w2;
    a.chain_b2 = p.chain_b2;
    a.chain_act2 = p.chain_act2;
    a.chain_y = p.chain_y;
    a.chain_y_f32 = p.chain_y_f32;
  }
  a.esz = p.out_f32 ? 4 : 2;
  bool vec = (p.out_pix_stride % 8 == 0) && (p.out_ch_off % 8 == 0) && aligned16(p.out) && (p.N % 8 == 0);
  if (convt) vec = vec && p.convt_oc % 8 == 0;
  if (p.res) vec = vec && (p.res_pix_stride % 8 == 0) && (p.res_ch_off % 8 == 0) && aligned16(p.res);
  if (p.bias) vec = vec && aligned16(p.bias);
  a.vec_ok = vec ? 1 : 0;

  // ---- A operand and tile geometry
  CUtensorMap mA, mB, mOut, mRes;
  memset(&mOut, 0, sizeof(mOut));
  memset(&mRes, 0, sizeof(mRes));
  if (p.mode == TC_CONV && p.kxn) {
    // kx-in-N: a virtual conv with the 3 row taps as pipeline taps (halo mode, one column block)
    // and N = 3 x 32 columns (kx, oc); the A box is BW = BWs + 2 input columns wide, starting one
    // column left of the tile, so row x of the tile holds input column ox0 - 1 + x
    if (p.C % 8 != 0) return set_error(SDX_ERR_INVALID, "tc conv: input channels must be a multiple of 8");
    const int BW = (p.OW + 13) / 14 * 14 <= (p.OW + 29) / 30 * 30 ? 16 : 32;  // less column waste
    const int BH = TC_BM / BW;
    a.kxn = 1;
    a.halo = 1;
    a.taps = 3;
    a.kw = 1;
    a.b_taps = 3;
    a.b_rows_per_tap = BN * n_tiles;
    a.BH = BH;
    a.BW = BW;
    a.BWs = BW - 2;
    a.OH = p.OH;
    a.OW = p.OW;
    a.tiles_h = (p.OH + BH - 1) / BH;
    a.tiles_w = (p.OW + a.BWs - 1) / a.BWs;
    a.m_tiles = p.batch * a.tiles_h * a.tiles_w;
    a.pad_t = 1;
    a.pad_l = 1;
    const int box_h = BH + 2;
    a.a_box_bytes = (uint32_t)(box_h * BW * kbytes);
    a.a_blk_bytes = (a.a_box_bytes + 1023u) & ~1023u;
    uint64_t dims[4] = {(uint64_t)p.C, (uint64_t)p.W, (uint64_t)p.H, (uint64_t)p.batch};
    uint64_t strides[3] = {(uint64_t)p.C * 2, (uint64_t)p.W * p.C * 2, (uint64_t)p.H * p.W * p.C * 2};
    uint32_t box[4] = {(uint32_t)kblk, (uint32_t)BW, (uint32_t)box_h, 1};
    int rc = encode_map(&mA, p.a, 4, dims, strides, box, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, swizzle_of(kbytes));
    if (rc) return rc;
  } else if (p.mode == TC_CONV) {
    if (p.C % 8 != 0) return set_error(SDX_ERR_INVALID, "tc conv: input channels must be a multiple of 8");
    // halo mode for kh > 1: tile widths of at least 8 pixels make the row offsets whole swizzle
    // atoms; used when three stages of it (A box + kh weight taps, two terms) and the staging fit,
    // or the weights fit resident beside three A boxes
    int BH, BW;
    pick_pixel_tile(p.OH, p.OW, 8, p.kh - 1, &BH, &BW);
    const size_t halo_a = (size_t)(BH + p.kh - 1) * BW * kbytes;
    const size_t staging_max = (size_t)2 * TC_BM * BN * (p.out_f32 ? 4 : 2);
    const size_t b_all = (size_t)a.wterms * p.kh * p.kw * (kpad / kblk) * n_tiles * BN * kbytes;
    const bool halo = p.kh > 1 && BH + p.kh - 1 <= 256 &&
                      (3 * (halo_a + (size_t)a.wterms * p.kh * BN * kbytes) + staging_max + 4096 <= (size_t)TC_SMEM_LIMIT ||
                       b_all + 3 * halo_a + staging_max + 4096 <= (size_t)TC_SMEM_LIMIT);
    if (!halo) pick_pixel_tile(p.OH, p.OW, 1, 0, &BH, &BW);
    a.halo = halo ? 1 : 0;
    a.b_taps = halo ? p.kh : 1;
    a.BH = BH;
    a.BW = BW;
    a.BWs = BW;
    a.OH = p.OH;
    a.OW = p.OW;
    a.tiles_h = (p.OH + BH - 1) / BH;
    a.tiles_w = (p.OW + BW - 1) / BW;
    a.m_tiles = p.batch * a.tiles_h * a.tiles_w;
    const int box_h = halo ? BH + p.kh - 1 : BH;
    a.a_box_bytes = (uint32_t)(box_h * BW * kbytes);
    a.a_blk_bytes = (a.a_box_bytes + 1023u) & ~1023u;
    uint64_t dims[4] = {(uint64_t)p.C, (uint64_t)p.W, (uint64_t)p.H, (uint64_t)p.batch};
    uint64_t strides[3] = {(uint64_t)p.C * 2, (uint64_t)p.W * p.C * 2, (uint64_t)p.H * p.W * p.C * 2};
    uint32_t box[4] = {(uint32_t)kblk, (uint32_t)BW, (uint32_t)box_h, 1};
    int rc = encode_map(&mA, p.a, 4, dims, strides, box, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, swizzle_of(kbytes));
    if (rc) return rc;
  } else {
    if (p.lda % 8 != 0) return set_error(SDX_ERR_INVALID, "tc rows: A row stride must be a multiple of 8 halves");
    a.M = p.M;
    a.OH = p.OH;  // pixel grid of the rows (upsampled residual)
    a.OW = p.OW;
    a.m_tiles = (p.M + TC_BM - 1) / TC_BM;
    a.a_box_bytes = (uint32_t)(TC_BM * kbytes);
    a.a_blk_bytes = (a.a_box_bytes + 1023u) & ~1023u;
    a.b_taps = 1;
    uint64_t dims[2] = {(uint64_t)p.K, (uint64_t)p.M};
    uint64_t strides[1] = {(uint64_t)p.lda * 2};
    uint32_t box[2] = {(uint32_t)kblk, TC_BM};
    int rc = encode_map(&mA, p.a, 2, dims, strides, box, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, swizzle_of(kbytes));
    if (rc) return rc;
  }
  {
    uint64_t dims[2] = {(uint64_t)kpad, (uint64_t)a.wterms * a.taps * a.b_rows_per_tap};
    uint64_t strides[1] = {(uint64_t)kpad * 2};
    uint32_t box[2] = {(uint32_t)kblk, (uint32_t)BN};
    int rc = encode_map(&mB, p.w, 2, dims, strides, box, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, swizzle_of(kbytes));
    if (rc) return rc;
  }

  // ---- epilogue: TMA store groups. A group is G columns (G * esz bytes = one staging row, at most
  // 128 B); each epilogue warp stores its 32 tile rows of every group as one box.
  const int esz = a.esz;
  const int cw = 128 / esz;  // columns in one 128-byte row
  int G;
  if (convt) {
    const int row = p.convt_kw * p.convt_oc;
    G = std::min(cw, row);
    if (row % G != 0 || BN % G != 0) G = 0;
  } else {
    // the widest store group (at most one 128-byte row) that divides the tile
    G = BN * esz >= 128 ? cw : BN;
    while (G > 0 && BN % G != 0) G = G % 2 == 0 && G / 2 >= 16 / esz * 2 ? G / 2 : 0;
  }
  // 16-column epilogue chunks must not straddle groups
  bool tma_out = G > 0 && G % 16 == 0 && aligned16(p.out) && (p.out_pix_stride * esz) % 16 == 0 &&
                 (p.out_ch_off * esz) % 16 == 0;
  if (convt) tma_out = tma_out && p.mode == TC_CONV && !chain;
  if (p.kxn) tma_out = false;  // the kx-in-N epilogue stores per thread
  if (tma_out) {
    const int P = G * esz;
    a.G = G;
    a.ngroups = BN / G;
    a.swz = (P == 32 || P == 64 || P == 128) ? 1 : 0;
    a.group_bytes = (uint32_t)(TC_BM * P);
    a.sbuf_bytes = (a.group_bytes * a.ngroups + 1023u) & ~1023u;
    const CUtensorMapDataType dt = p.out_f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const CUtensorMapSwizzle sw = !a.swz ? CU_TENSOR_MAP_SWIZZLE_NONE
                                  : P == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                  : P == 64  ? CU_TENSOR_MAP_SWIZZLE_64B
                                             : CU_TENSOR_MAP_SWIZZLE_32B;
    // one warp's 32 tile rows: a run of 32 pixels (BW >= 32) or 32/BW whole tile rows (BW < 32)
    const uint32_t wbw = (uint32_t)std::min(a.BW, 32), wbh = (uint32_t)std::max(1, 32 / std::max(a.BW, 1));
    int rc;
    if (convt) {
      const uint64_t row = (uint64_t)p.convt_kw * p.convt_oc;
      uint64_t dims[5] = {row, (uint64_t)p.convt_W, (uint64_t)p.convt_kh, (uint64_t)p.convt_H, (uint64_t)p.batch};
      uint64_t strides[4] = {row * esz, row * p.convt_W * esz, row * p.convt_W * p.convt_kh * esz,
                             row * p.convt_W * p.convt_kh * p.convt_H * esz};
      uint32_t box[5] = {(uint32_t)G, wbw, 1, wbh, 1};
      rc = encode_map(&mOut, p.out, 5, dims, strides, box, dt, sw);
    } else if (p.mode == TC_CONV) {
      const uint64_t ps = (uint64_t)p.out_pix_stride;
      uint64_t dims[4] = {(uint64_t)(p.out_ch_off + p.N), (uint64_t)p.OW, (uint64_t)p.OH, (uint64_t)p.batch};
      uint64_t strides[3] = {ps * esz, ps * p.OW * esz, ps * p.OW * p.OH * esz};
      uint32_t box[4] = {(uint32_t)G, wbw, wbh, 1};
      rc = encode_map(&mOut, p.out, 4, dims, strides, box, dt, sw);
    } else {
      uint64_t dims[2] = {(uint64_t)(p.out_ch_off + p.N), (uint64_t)p.M};
      uint64_t strides[1] = {(uint64_t)p.out_pix_stride * esz};
      uint32_t box[2] = {(uint32_t)G, 32};
      rc = encode_map(&mOut, p.out, 2, dims, strides, box, dt, sw);
    }
    if (rc) return rc;
    // residual by TMA when it has the output's type, layout and channel geometry
    if (p.res && !convt && !p.res_up && p.res_f32 == p.out_f32 && p.res_pix_stride == p.out_pix_stride &&
        p.res_ch_off == p.out_ch_off && aligned16(p.res)) {
      if (p.mode == TC_CONV) {
        const uint64_t ps = (uint64_t)p.res_pix_stride;
        uint64_t dims[4] = {(uint64_t)(p.res_ch_off + p.N), (uint64_t)p.OW, (uint64_t)p.OH, (uint64_t)p.batch};
        uint64_t strides[3] = {ps * esz, ps * p.OW * esz, ps * p.OW * p.OH * esz};
        uint32_t box[4] = {(uint32_t)G, wbw, wbh, 1};
        rc = encode_map(&mRes, p.res, 4, dims, strides, box, dt, sw);
      } else {
        uint64_t dims[2] = {(uint64_t)(p.res_ch_off + p.N), (uint64_t)p.M};
        uint64_t strides[1] = {(uint64_t)p.res_pix_stride * esz};
        uint32_t box[2] = {(uint32_t)G, 32};
        rc = encode_map(&mRes, p.res, 2, dims, strides, box, dt, sw);
      }
      if (rc) return rc;
      a.tma_res = 1;
      a.slab_tx = (uint32_t)(P * 32);
    }
    a.tma_out = 1;
  } else if (convt && p.mode == TC_CONV && !chain) {
    return set_error(SDX_ERR_NOT_SUPPORTED, "tc convt: channel geometry has no TMA store layout");
  }

  if (p.bias && BN * n_tiles <= TC_BIAS_SMEM_MAX) a.bias_smem = BN * n_tiles;
  // fast epilogue: fp16 out by TMA through 32/64/128-byte swizzled rows, bias in smem (zeros when
  // there is none), residual TMA-staged or absent
  // residual read per thread in the fast epilogue: fp16, 16-byte aligned rows (N is a multiple of 8)
  const bool res_thread = p.res && !p.res_f32 && !convt && aligned16(p.res) && p.res_pix_stride % 8 == 0 &&
                          p.res_ch_off % 8 == 0 && p.N % 8 == 0;
  const bool fast = a.tma_out && a.esz == 2 && a.swz && !p.kxn && (!p.res || a.tma_res || res_thread) &&
                    BN * n_tiles <= TC_BIAS_SMEM_MAX && (a.G == 16 || a.G == 32 || a.G == 64);
  if (fast) {
    a.bias_smem = BN * n_tiles;
    a.log2G = a.G == 16 ? 4 : a.G == 32 ? 5 : 6;
  }
  // straight-line kx-in-N epilogue: fp16 out with 16-byte rows, no residual, N a multiple of 8
  const bool kxn_fast = p.kxn && !p.out_f32 && a.vec_ok && !p.res && p.N % 8 == 0 && p.N <= 32 &&
                        BN * n_tiles <= TC_BIAS_SMEM_MAX;
  if (kxn_fast) a.bias_smem = BN * n_tiles;
  // ---- shared-memory plan. Preference: weights resident (loaded once per CTA) with 2 staging
  // buffers and >= 3 A stages, resident with 1 staging buffer and >= 2 stages, then streamed
  // weights (per stage) likewise. 8 stages at most.
  if (!a.tma_out) a.sbuf_bytes = 0;
  a.b_total_bytes = (uint32_t)((size_t)a.wterms * a.taps * a.kb_per_tap * n_tiles * BN * kbytes);
  // stages of cps channel blocks each (fewer, larger stages amortise the per-stage waits and
  // commits of the two issuing threads): the largest cps with >= 3 stages, else cps = 1 with >= 2
  bool planned = false;
  // four epilogue groups for thin tiles, and for the per-thread epilogue (ConvT scatter and other
  // general cases) up to 128 columns; two when the staging of four would crowd out the A stages
  if (p.res_up && !fast)
    return set_error(SDX_ERR_NOT_SUPPORTED, "tc: upsampled residual needs the fp16 TMA-store epilogue");
  if (p.gap && (!fast || p.mode == TC_CONV || convt || p.M % 32 != 0 || p.N % 16 != 0 ||
                (BN != 16 && BN != 32 && BN != 64 && BN != 128) || a.G != (BN < 64 ? BN : 64) ||
                (reinterpret_cast<uintptr_t>(p.gap) & 7)))
    return set_error(SDX_ERR_NOT_SUPPORTED,
                     "tc: fused channel sums need a 1x1 conv with the fp16 TMA-store epilogue, rows % 32 == 0, "
                     "oc 16, 32, 64 or a multiple of 128 and an 8-byte aligned sums buffer");
  if (chain) a.bias_smem = BN + 4 * p.convt_oc + 4;  // first bias, second ConvT's weights and bias
  const bool eg4 = !p.kxn && 4 * BN <= 512 && (BN <= 64 || chain || (!fast && !kxn_fast));
  for (int eg = eg4 ? 4 : 2; eg >= 2 && !planned; eg -= 2) {
  a.egroups = eg;
  for (int res = 1; res >= 0 && !planned; res--) {
    for (int pass = 0; pass < 2 && !planned; pass++) {
      for (int cps = pass == 0 ? a.kb_per_tap : 1; cps >= 1 && !planned; cps--) {
        if (a.kb_per_tap % cps) continue;
        for (int nsb = a.tma_out ? 2 : 1; nsb >= 1 && !planned; nsb--) {
          a.b_resident = res;
          a.nsbuf = nsb;
          a.cps = cps;
          a.a_stage_bytes = (uint32_t)cps * a.a_blk_bytes;
          const size_t fixed = smem_fixed(a);
          const size_t per = a.a_stage_bytes + b_stage_bytes_of(a);
          if (fixed >= (size_t)TC_SMEM_LIMIT) continue;
          const int st = (int)std::min<size_t>(TC_MAX_STAGES, ((size_t)TC_SMEM_LIMIT - fixed) / per);
          if (st >= (pass == 0 ? 3 : (nsb == 2 ? 3 : 2))) {
            a.stages = st;
            planned = true;
          }
        }
      }
    }
  }
  }
  if (!planned) return set_error(SDX_ERR_NOT_SUPPORTED, "tc: shared memory plan too large");
  const size_t smem = smem_bytes(a);
  if (smem > (size_t)TC_SMEM_LIMIT) return set_error(SDX_ERR_NOT_SUPPORTED, "tc: shared memory plan too large");

  const int total = a.m_tiles * a.n_tiles;
  if (total == 0) return SDX_OK;
  int dev = 0;
  cudaGetDevice(&dev);
  const int grid = std::min(total, num_sms(dev));
  int rc = SDX_OK;
  if (chain && a.egroups == 4) {
    SDX_ACT_DISPATCH(a.act, ACTC, rc = (launch_tc<ACTC, 4, 4>(dev, grid, smem, stream, mA, mB, mOut, mRes, a)));
  } else if (chain) {
    SDX_ACT_DISPATCH(a.act, ACTC, rc = (launch_tc<ACTC, 4, 2>(dev, grid, smem, stream, mA, mB, mOut, mRes, a)));
  } else if (fast && a.egroups == 4) {
    SDX_ACT_DISPATCH(a.act, ACTC, rc = (launch_tc<ACTC, 1, 4>(dev, grid, smem, stream, mA, mB, mOut, mRes, a)));
  } else if (fast) {
    SDX_ACT_DISPATCH(a.act, ACTC, rc = (launch_tc<ACTC, 1, 2>(dev, grid, smem, stream, mA, mB, mOut, mRes, a)));
  } else if (kxn_fast && a.egroups == 2) {
    SDX_ACT_DISPATCH(a.act, ACTC, rc = (launch_tc<ACTC, 2, 2>(dev, grid, smem, stream, mA, mB, mOut, mRes, a)));
  } else if (a.egroups == 4) {
    SDX_ACT_DISPATCH(a.act, ACTC, rc = (launch_tc<ACTC, 0, 4>(dev, grid, smem, stream, mA, mB, mOut, mRes, a)));
  } else {
    SDX_ACT_DISPATCH(a.act, ACTC, rc = (launch_tc<ACTC, 0, 2>(dev, grid, smem, stream, mA, mB, mOut, mRes, a)));
  }
  if (rc) return rc;
  count_launch();
  return SDX_OK;
}

// Packs ONNX conv weights w [OC][IC][KH][KW] (fp32) into the B operand [2][taps][n_tiles*BN][ICpad]
// fp16 (hi terms, then lo terms), zero padded.
size_t tc_weights_halves(int N, int K, int taps, int terms) {
  int BN, nt;
  tc_plan_n(N, &BN, &nt);
  size_t kpad = (size_t)tc_kpad(K);
  return (size_t)(terms == 1 ? 1 : 2) * taps * BN * nt * kpad;
}

size_t tc_convt_weights_halves(int IC, int OC, int KH, int KW) {
  int BN, nt;
  tc_plan_n_convt(KH, KW, OC, &BN, &nt);
  size_t kpad = (size_t)tc_kpad(IC);
  return 2 * (size_t)BN * nt * kpad;
}

// hi = fp16(w) at `idx`, lo = fp16(w - hi) at `idx + lo_off`
static inline void put2(__half* out, size_t idx, size_t lo_off, float w) {
  const __half h = __float2half_rn(w);
  out[idx] = h;
  out[idx + lo_off] = __float2half_rn(w - __half2float(h));
}

// terms == 1: only the hi block (w rounded to fp16).
void tc_pack_conv(const float* w, int OC, int IC, int KH, int KW, int terms, __half* out) {
  int BN, nt;
  tc_plan_n(OC, &BN, &nt);
  const size_t rows = (size_t)BN * nt, kpad = (size_t)tc_kpad(IC);
  const int taps = KH * KW;
  const size_t lo = (size_t)taps * rows * kpad;
  memset(out, 0, sizeof(__half) * (terms == 1 ? 1 : 2) * lo);
  for (int o = 0; o < OC; o++)
    for (int c = 0; c < IC; c++)
      for (int t = 0; t < taps; t++) {
        const size_t idx = ((size_t)t * rows + o) * kpad + c;
        const float v = w[((size_t)o * IC + c) * taps + t];
        if (terms == 1) out[idx] = __float2half_rn(v);
        else put2(out, idx, lo, v);
      }
}

bool tc_conv_kxn(int kh, int kw, int sh, int sw, int pt, int pl, int pb, int pr, int oc) {
  return kh == 3 && kw == 3 && sh == 1 && sw == 1 && pt == 1 && pl == 1 && pb == 1 && pr == 1 && oc >= 8 && oc <= 32;
}

size_t tc_kxn_weights_halves(int K, int terms) {
  return (size_t)(terms == 1 ? 1 : 2) * 3 * 96 * (size_t)tc_kpad(K);
}

// kx-in-N weights: [terms][ky][kx * 32 + o][Kpad], rows o >= OC zero.
void tc_pack_conv_kxn(const float* w, int OC, int IC, int terms, __half* out) {
  const size_t kpad = (size_t)tc_kpad(IC), lo = (size_t)3 * 96 * kpad;
  memset(out, 0, sizeof(__half) * (terms == 1 ? 1 : 2) * lo);
  for (int o = 0; o < OC; o++)
    for (int c = 0; c < IC; c++)
      for (int ky = 0; ky < 3; ky++)
        for (int kx = 0; kx < 3; kx++) {
          const size_t idx = ((size_t)ky * 96 + kx * 32 + o) * kpad + c;
          const float v = w[((size_t)o * IC + c) * 9 + ky * 3 + kx];
          if (terms == 1) out[idx] = __float2half_rn(v);
          else put2(out, idx, lo, v);
        }
}

// ConvT weights [IC][OC][KH][KW] -> one GEMM panel whose row tap*OC + o is w[:, o, tap].
void tc_pack_convt(const float* w, int IC, int OC, int KH, int KW, __half* out) {
  const int taps = KH * KW;
  int BN, nt;
  tc_plan_n_convt(KH, KW, OC, &BN, &nt);
  const size_t rows = (size_t)BN * nt, kpad = (size_t)tc_kpad(IC);
  const size_t lo = rows * kpad;
  memset(out, 0, sizeof(__half) * 2 * lo);
  for (int c = 0; c < IC; c++)
    for (int o = 0; o < OC; o++)
      for (int t = 0; t < taps; t++) put2(out, ((size_t)t * OC + o) * kpad + c, lo, w[((size_t)c * OC + o) * taps + t]);
}

void tc_pack_gemm(const float* b, int K, int N, int trans_b, __half* out) {
  int BN, nt;
  tc_plan_n(N, &BN, &nt);
  const size_t rows = (size_t)BN * nt, kpad = (size_t)tc_kpad(K);
  const size_t lo = rows * kpad;
  memset(out, 0, sizeof(__half) * 2 * lo);
  for (int n = 0; n < N; n++)
    for (int k = 0; k < K; k++) put2(out, (size_t)n * kpad + k, lo, trans_b ? b[(size_t)n * K + k] : b[(size_t)k * N + n]);
}

}  // namespace sdx
