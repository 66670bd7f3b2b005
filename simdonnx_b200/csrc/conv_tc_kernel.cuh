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
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>

#include "sdx_device.cuh"
#include "sdx_internal.h"
#include "conv_tc_args.h"

namespace sdx {

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
// L1-allocating: the nearest-upsampled residual rows that use it read each source pixel twice
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
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

// Named barrier `id` over `n` threads (a whole number of warps) that also ORs a predicate across them.
__device__ __forceinline__ bool named_bar_or(int id, int n, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "barrier.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("barrier.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

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
// Tiles of ordinals w, w + nw, ... of the CTA's sequence (nw MMA-issuing warps, this one w < nw <= 2):
// ordinal o uses ring slot o mod S and accumulator o mod nacc (S >= nw, nacc a multiple of nw).
template <int BT, int NK, bool TWO, int CPS>
__device__ __noinline__ void mma_single_loop(uint32_t ld, const MmaSingle m, int tile0, int total_tiles, int tstep,
                                             int w, int nw, uint64_t* full, uint64_t* empty, uint64_t* accf,
                                             uint64_t* acce, unsigned int* err, volatile int* abort_flag) {
  int s = w, nt = (m.nt0 + w * m.nt_step) % m.n_tiles;
  const int nt_adv = (nw * m.nt_step) % m.n_tiles;
  uint32_t phase = 0, acc = (uint32_t)w, accph = 0;
  for (int tile = tile0 + w * tstep; tile < total_tiles; tile += nw * tstep) {
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
    s += nw;
    if (s >= m.S) {
      s -= m.S;
      phase ^= 1u;
    }
    acc += (uint32_t)nw;
    if (acc >= (uint32_t)m.nacc) {
      acc -= (uint32_t)m.nacc;
      accph ^= 1u;
    }
    nt += nt_adv;
    nt = nt >= m.n_tiles ? nt - m.n_tiles : nt;
  }
}
template <int BT, int NK, bool TWO>
__device__ __forceinline__ void mma_single_cps(int cps, uint32_t ld, const MmaSingle& m, int tile0, int total_tiles,
                                               int tstep, int w, int nw, uint64_t* full, uint64_t* empty,
                                               uint64_t* accf, uint64_t* acce, unsigned int* err,
                                               volatile int* abort_flag) {
  if (cps == 1) mma_single_loop<BT, NK, TWO, 1>(ld, m, tile0, total_tiles, tstep, w, nw, full, empty, accf, acce, err, abort_flag);
  else if (cps == 2) mma_single_loop<BT, NK, TWO, 2>(ld, m, tile0, total_tiles, tstep, w, nw, full, empty, accf, acce, err, abort_flag);
  else if (cps == 3) mma_single_loop<BT, NK, TWO, 3>(ld, m, tile0, total_tiles, tstep, w, nw, full, empty, accf, acce, err, abort_flag);
  else mma_single_loop<BT, NK, TWO, 4>(ld, m, tile0, total_tiles, tstep, w, nw, full, empty, accf, acce, err, abort_flag);
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

// (a0, a1) += (x0, x1) * (w0, w1) as one packed f32x2 FMA; each lane is the single-rounding fmaf.
__device__ __forceinline__ void ffma2_vec(float& a0, float& a1, float x0, float x1, float w0, float w1) {
  asm("{\n\t.reg .b64 ra, rx, rw;\n\t"
      "mov.b64 ra, {%0, %1};\n\tmov.b64 rx, {%2, %3};\n\tmov.b64 rw, {%4, %5};\n\t"
      "fma.rn.f32x2 ra, rx, rw, ra;\n\tmov.b64 {%0, %1}, ra;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(x0), "f"(x1), "f"(w0), "f"(w1));
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

__device__ __forceinline__ float2 mul_f32x2(float2 a, float2 b) {
  uint64_t x, y, d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(a.x), "f"(a.y));
  asm("mov.b64 %0, {%1, %2};" : "=l"(y) : "f"(b.x), "f"(b.y));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(x), "l"(y));
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

// Channel sums of one warp's 32 staged rows of a pixel-folded tile (F pixels of OC channels per
// row, F * OC = 64 * NG columns in NG 64-column groups of 128-byte swizzled rows): per run of 32
// pixels (32 / F rows) and channel, into gp[run * OC + channel] for the warp's F runs. Lane j sums
// the column pair j of every group over every row (4-byte loads; the swizzle term of row r is
// r & 7, one base address per term), per run; the lanes whose pairs hold the same channel in other
// pixel slots (j ^ OC/2, ...) then combine by shuffles, and lanes 0 .. OC/2 - 1 store.
template <int F, int OC, int NG>
__device__ __forceinline__ void gap_warp_rows_fold(uint32_t slab, uint32_t group_bytes, int lane, float* gp) {
  static_assert(F * OC == 64 * NG && OC % 16 == 0 && OC <= 64, "folded tile of whole 64-column groups");
  constexpr int RPR = 32 / F;  // rows per 32-pixel run
  const uint32_t byte = (uint32_t)lane * 4u;  // the pair's byte offset in its 128-byte group row
  const uint32_t k = byte >> 4, inner = byte & 15u;
  uint32_t base[8];
#pragma unroll
  for (int c = 0; c < 8; c++) base[c] = slab + (((k ^ (uint32_t)c) << 4) | inner);
  float2 acc[F];
#pragma unroll
  for (int r = 0; r < F; r++) acc[r] = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int g = 0; g < NG; g++) {
#pragma unroll
    for (int row = 0; row < 32; row++) {
      uint32_t w;
      asm volatile("ld.shared.b32 %0, [%1];" : "=r"(w) : "r"(base[row & 7] + (uint32_t)g * group_bytes + (uint32_t)(row * 128)));
      acc[row / RPR] = add_f32x2(acc[row / RPR], __half22float2(*reinterpret_cast<const __half2*>(&w)));
    }
  }
#pragma unroll
  for (int off = OC / 2; off < 32; off *= 2)
#pragma unroll
    for (int r = 0; r < F; r++) {
      acc[r].x += __shfl_xor_sync(0xffffffffu, acc[r].x, off);
      acc[r].y += __shfl_xor_sync(0xffffffffu, acc[r].y, off);
    }
  if (lane < OC / 2) {
#pragma unroll
    for (int r = 0; r < F; r++) *reinterpret_cast<float2*>(gp + r * OC + 2 * lane) = acc[r];
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
  // bias (and residual) adds as packed f32x2 instructions: each lane is the same fp32 add
  const float4* bp = reinterpret_cast<const float4*>(sb + col);
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const float4 b = bp[i];
    float2 lo = add_f32x2(make_float2(v[4 * i], v[4 * i + 1]), make_float2(b.x, b.y));
    float2 hi = add_f32x2(make_float2(v[4 * i + 2], v[4 * i + 3]), make_float2(b.z, b.w));
    v[4 * i] = lo.x; v[4 * i + 1] = lo.y; v[4 * i + 2] = hi.x; v[4 * i + 3] = hi.y;
  }
  if (res_smem) {
    uint4 u0, u1;
    lds16(ad0, u0);
    lds16(ad1, u1);
    const __half2* h0 = reinterpret_cast<const __half2*>(&u0);
    const __half2* h1 = reinterpret_cast<const __half2*>(&u1);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float2 f0 = add_f32x2(make_float2(v[2 * i], v[2 * i + 1]), __half22float2(h0[i]));
      const float2 f1 = add_f32x2(make_float2(v[8 + 2 * i], v[8 + 2 * i + 1]), __half22float2(h1[i]));
      v[2 * i] = f0.x; v[2 * i + 1] = f0.y;
      v[8 + 2 * i] = f1.x; v[8 + 2 * i + 1] = f1.y;
    }
  }
  if constexpr (ACT == ACT_HARDSWISH) {
    // x * clamp(x / 6 + 1/2, 0, 1): the clamped FMA per lane, the product packed
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
      const float t0 = __saturatef(fmaf(v[i], 1.0f / 6.0f, 0.5f)), t1 = __saturatef(fmaf(v[i + 1], 1.0f / 6.0f, 0.5f));
      const float2 y = mul_f32x2(make_float2(v[i], v[i + 1]), make_float2(t0, t1));
      v[i] = y.x;
      v[i + 1] = y.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = act_t<ACT>(v[i]);
  }
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
__global__ void __launch_bounds__(tc_threads_epi(G, EPI), 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ CUtensorMap tmRes,
                   const TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr bool DWF = EPI == 6;               // A tiles from the fused depthwise warps
  constexpr bool FAST = EPI == 1 || EPI == 6;  // the straight-line fp16 TMA-store epilogue
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
    mbar_init(smem_u32(drain), EPI == 2 ? 2 : 1);  // one commit per MMA-issuing warp
    mbar_init(smem_u32(bres), 1);
    if (DWF) {
      uint64_t* hb = reinterpret_cast<uint64_t*>(smem + a.dw_off + (size_t)a.dw_slots * a.dw_slot_bytes +
                                                 (size_t)10 * a.dw_c * 4);
      for (int i = 0; i < 4; i++) mbar_init(smem_u32(&hb[i]), 1);  // halo full [2], halo empty [2]
    }
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
    sBias[i] = (a.bias && i < a.N)
                   ? __ldg(a.bias + (a.convt_oc > 0 ? i % a.convt_oc : a.bias_mod > 0 ? i % a.bias_mod : i))
                   : 0.0f;
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
  // this CTA's tiles: strided by the grid, or a contiguous range (per-image weights)
  const bool imgw = a.img_tiles > 0;
  const bool contig = imgw || a.contig;
  const int t_begin = contig ? (int)blockIdx.x * a.per_cta : (int)blockIdx.x;
  const int t_end = contig ? min(total_tiles, t_begin + a.per_cta) : total_tiles;
  const int t_step = contig ? 1 : (int)gridDim.x;
  // pipeline stages per tile: (tap, channel block), or (kx, channel block) in halo mode
  const int groups = a.kb_per_tap / a.cps;  // channel-block groups per tap
  const int kblocks = (a.halo ? a.kw : a.taps) * groups;

  // weight block (term, tap, channel block, n tile) in the resident layout
  auto b_res_off = [&](int term, int tap, int cb, int nt) -> uint32_t {
    return a.b_nslice ? (uint32_t)((term * a.taps + tap) * a.kb_per_tap + cb) * b_tap_bytes
                      : (uint32_t)((((term * a.taps + tap) * a.kb_per_tap + cb) * a.n_tiles + nt)) * b_tap_bytes;
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
      // every weight block of weight set `img` once, onto one barrier
      auto load_b = [&](int img) {
        const uint32_t bb = smem_u32(bres);
        mbar_arrive_expect_tx_p(ld, bb, a.b_total_bytes);
        for (int term = 0; term < a.wterms; term++)
          for (int tap = 0; tap < a.taps; tap++)
            for (int cb = 0; cb < a.kb_per_tap; cb++)
              for (int nt = 0; nt < a.n_tiles; nt++) {
                if (a.b_nslice && nt != (int)(blockIdx.x % (unsigned)a.n_tiles)) continue;
                tma_load_2d_p(ld, smem_u32(sB) + b_res_off(term, tap, cb, nt), &tmB, bb, cb * a.kblk,
                              img * a.b_img_rows + (term * a.taps + tap) * a.b_rows_per_tap + nt * a.BN);
              }
      };
      int cur_img = imgw ? t_begin / a.img_tiles : 0;
      uint32_t b_loads = 0;
      if (a.b_resident) {
        load_b(cur_img);
        b_loads = 1;
      }
      int s = 0;
      uint32_t phase = 0;
      int s_last = -1;          // ring slot and phase of the most recent stage issued
      uint32_t ph_last = 0;
      uint32_t h_issued[2] = {0, 0};  // fused depthwise: halo boxes issued per slot
      if (DWF) {
        // the depthwise input's halo box of every tile (all channel blocks) into dw_slots slots, freed
        // by the depthwise warps once they have built the tile's A block from it
        uint64_t* hfull = reinterpret_cast<uint64_t*>(smem + a.dw_off + (size_t)a.dw_slots * a.dw_slot_bytes +
                                                      (size_t)10 * a.dw_c * 4);
        uint64_t* hempty = hfull + 2;
        const int per_img = a.tiles_h * a.tiles_w;
        int hs = 0;
        uint32_t hph = 0;
        for (int tile = t_begin; tile < t_end; tile += t_step) {
          const int img = tile / per_img;
          const int r = tile - img * per_img;
          const int ty = r / a.tiles_w;
          const int oy0 = ty * a.BH, ox0 = (r - ty * a.tiles_w) * a.BWs;
          if (!mbar_wait_warp(smem_u32(&hempty[hs]), hph ^ 1u, a.err, SDX_DEV_WAIT_EMPTY, abort_flag)) break;
          const uint32_t hb = smem_u32(&hfull[hs]);
          mbar_arrive_expect_tx_p(ld, hb, (uint32_t)a.kb_per_tap * a.dw_box_bytes);
          const uint32_t dst = smem_u32(smem + a.dw_off) + (uint32_t)hs * a.dw_slot_bytes;
          for (int cb = 0; cb < a.kb_per_tap; cb++)
            tma_load_4d_p(ld, dst + (uint32_t)cb * a.dw_blk_bytes, &tmA, hb, cb * a.kblk, ox0 - 1, oy0 - 1, img);
          h_issued[hs]++;
          if (++hs == a.dw_slots) {
            hs = 0;
            hph ^= 1u;
          }
        }
        for (int q = 0; q < a.dw_slots; q++)
          if (h_issued[q] > 0) mbar_wait_drain(smem_u32(&hfull[q]), (h_issued[q] - 1) & 1u, a.err, SDX_DEV_WAIT_DRAIN);
        ok = false;  // the A stages are the depthwise warps'
      }
      // single-stage tiles with resident weights (pointwise, kx-in-N 3x3, ConvT): the dispatch-free
      // loop; a 4-D box at (ox0 - pad_l, oy0 - pad_t) covers halo mode with one column tap and the
      // one-tap conv mode alike
      if (ok && kblocks == 1 && a.b_resident && a.cps <= 4 && (a.mode != TC_CONV || a.halo || a.taps == 1) && !imgw) {
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
      if (a.mpair) {
        // pixel-tile pairs: each stage holds both tiles' A boxes (halo mode) and one weight stage
        const int n_units = (a.m_tiles >> 1) * a.n_tiles;
        const int per_img = a.tiles_h * a.tiles_w;
        for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
          const int pi = u / a.n_tiles, n_tile = u - pi * a.n_tiles;
          int img[2], oy0[2], ox0[2];
#pragma unroll
          for (int j = 0; j < 2; j++) {
            const int m = 2 * pi + j;
            img[j] = m / per_img;
            const int r = m - img[j] * per_img;
            const int ty = r / a.tiles_w;
            oy0[j] = ty * a.BH;
            ox0[j] = (r - ty * a.tiles_w) * a.BWs;
          }
          int tk = 0, cg = 0;
          for (int kb = 0; kb < kblocks; kb++) {
            if (!mbar_wait_warp(smem_u32(&empty[s]), phase ^ 1u, a.err, SDX_DEV_WAIT_EMPTY, abort_flag)) {
              ok = false;
              break;
            }
            const uint32_t fb = smem_u32(&full[s]);
            mbar_arrive_expect_tx_p(ld, fb, (uint32_t)(2 * a.cps) * a.a_box_bytes + b_stage_bytes);
            const uint32_t dA0 = smem_u32(sA) + (uint32_t)s * a.a_stage_bytes;
            const uint32_t dB0 = smem_u32(sB) + (uint32_t)s * b_stage_bytes;
            for (int ci = 0; ci < a.cps; ci++) {
              const int cb = cg * a.cps + ci;
#pragma unroll
              for (int j = 0; j < 2; j++)
                tma_load_4d_p(ld, dA0 + (uint32_t)(j * a.cps + ci) * a.a_blk_bytes, &tmA, fb, cb * a.kblk,
                              ox0[j] + tk - a.pad_l, oy0[j] - a.pad_t, img[j]);
              const uint32_t dB = dB0 + (uint32_t)ci * b_cb_bytes;
              for (int jj = 0; jj < a.b_taps; jj++) {
                const int brow = (jj * a.kw + tk) * a.b_rows_per_tap + n_tile * a.BN;
                tma_load_2d_p(ld, dB + jj * b_tap_bytes, &tmB, fb, cb * a.kblk, brow);
                if (a.wterms == 2)
                  tma_load_2d_p(ld, dB + b_half_bytes + jj * b_tap_bytes, &tmB, fb, cb * a.kblk,
                                a.taps * a.b_rows_per_tap + brow);
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
        ok = false;  // every unit issued above
      }
      for (int tile = t_begin; tile < t_end && ok; tile += t_step) {
        const int m_tile = a.n_tiles == 1 ? tile : tile / a.n_tiles;
        const int n_tile = tile - m_tile * a.n_tiles;
        if (imgw && m_tile / a.img_tiles != cur_img) {
          // a new image's weights: every MMA that read the loaded set has completed once the last
          // stage issued has been released (tcgen05.commit tracks all earlier MMAs of its thread)
          if (s_last >= 0 &&
              !mbar_wait_warp(smem_u32(&empty[s_last]), ph_last, a.err, SDX_DEV_WAIT_EMPTY, abort_flag)) {
            ok = false;
            break;
          }
          cur_img = m_tile / a.img_tiles;
          load_b(cur_img);
          b_loads++;
        }
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
          s_last = s;
          ph_last = phase;
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
      if (b_loads > 0) mbar_wait_drain(smem_u32(bres), (b_loads - 1) & 1u, a.err, SDX_DEV_WAIT_DRAIN);
    }
    __syncwarp();
  } else if (warp == 1 || (EPI == 2 && warp == 2 + 4 * G)) {
    // MMA issue: warp 1, and for kx-in-N tiles a second warp taking every other tile of the
    // single-stage loop (mw = 1); every other path runs on warp 1 alone
    const int mw = warp == 1 ? 0 : 1;
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
                          a.cps <= 4 && (nk == 1 || nk == 2 || nk == 4) && !imgw;
      const int nmw = (EPI == 2 && single && S >= 2 && (a.nacc & 1) == 0) ? 2 : 1;
      if (mw >= nmw) ok = false;  // the second warp has no tiles: only its drain commit below
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
          if (nk == 1) mma_single_cps<3, 1, false>(a.cps, ld, m, t_begin, t_end, t_step, mw, nmw, full, empty, accf, acce, a.err, abort_flag);
          else if (nk == 2) mma_single_cps<3, 2, false>(a.cps, ld, m, t_begin, t_end, t_step, mw, nmw, full, empty, accf, acce, a.err, abort_flag);
          else mma_single_cps<3, 4, false>(a.cps, ld, m, t_begin, t_end, t_step, mw, nmw, full, empty, accf, acce, a.err, abort_flag);
        } else if (a.wterms == 2) {
          if (nk == 1) mma_single_cps<1, 1, true>(a.cps, ld, m, t_begin, t_end, t_step, mw, nmw, full, empty, accf, acce, a.err, abort_flag);
          else if (nk == 2) mma_single_cps<1, 2, true>(a.cps, ld, m, t_begin, t_end, t_step, mw, nmw, full, empty, accf, acce, a.err, abort_flag);
          else mma_single_cps<1, 4, true>(a.cps, ld, m, t_begin, t_end, t_step, mw, nmw, full, empty, accf, acce, a.err, abort_flag);
        } else {
          if (nk == 1) mma_single_cps<1, 1, false>(a.cps, ld, m, t_begin, t_end, t_step, mw, nmw, full, empty, accf, acce, a.err, abort_flag);
          else if (nk == 2) mma_single_cps<1, 2, false>(a.cps, ld, m, t_begin, t_end, t_step, mw, nmw, full, empty, accf, acce, a.err, abort_flag);
          else mma_single_cps<1, 4, false>(a.cps, ld, m, t_begin, t_end, t_step, mw, nmw, full, empty, accf, acce, a.err, abort_flag);
        }
        ok = false;  // the loop above ran every tile
      }
      if (ok && a.mpair) {
        // pixel-tile pairs: per stage and channel block, the same weight descriptor for both tiles'
        // A blocks into their two accumulators
        const int n_units = (a.m_tiles >> 1) * a.n_tiles;
        for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
          uint32_t dj[2], aj[2];
#pragma unroll
          for (int j = 0; j < 2; j++) {
            if (!mbar_wait_warp(smem_u32(&acce[acc]), accph ^ 1u, a.err, SDX_DEV_WAIT_ACC_EMPTY, abort_flag)) {
              ok = false;
              break;
            }
            aj[j] = acc;
            dj[j] = tmem_base + acc * (uint32_t)a.acc_stride;
            if (++acc == (uint32_t)a.nacc) {
              acc = 0;
              accph ^= 1u;
            }
          }
          if (!ok) break;
          tc_fence_after();
          uint32_t first = 0;
          for (int kb = 0; kb < kblocks; kb++) {
            if (!mbar_wait_warp(smem_u32(&full[s]), phase, a.err, SDX_DEV_WAIT_FULL, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t sa = smem_u32(sA) + (uint32_t)s * a.a_stage_bytes;
            uint32_t b0 = sB_addr + (uint32_t)s * b_stage_bytes;
            for (int ci = 0; ci < a.cps; ci++, b0 += b_cb) {
              const uint64_t bd = dconst | (uint64_t)((b0 >> 4) & 0x3FFFu);
#pragma unroll
              for (int j = 0; j < 2; j++) {
                const uint32_t saj = sa + (uint32_t)(j * a.cps + ci) * a.a_blk_bytes;
                const uint64_t ad = dconst | (uint64_t)((saj >> 4) & 0x3FFFu);
                if (a.wterms == 2) umma_stage_dispatch<true>(ld, a.b_taps, nk, dj[j], ad, bd, a_tap16, b_tap16, b_lo16, idesc, first);
                else umma_stage_dispatch<false>(ld, a.b_taps, nk, dj[j], ad, bd, a_tap16, b_tap16, b_lo16, idesc, first);
              }
              first = 1u;
            }
            tc_commit_p(ld, smem_u32(&empty[s]));
            if (++s == S) {
              s = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
          tc_commit_p(ld, smem_u32(&accf[aj[0]]));
          tc_commit_p(ld, smem_u32(&accf[aj[1]]));
        }
        ok = false;  // every unit ran above
      }
      int cur_img = imgw ? t_begin / a.img_tiles : 0;
      uint32_t b_waits = 1;  // weight sets waited for (the first one above)
      for (int tile = t_begin; tile < t_end && ok; tile += t_step) {
        const int n_tile = a.n_tiles == 1 ? 0 : tile % a.n_tiles;
        if (imgw && tile / a.img_tiles != cur_img) {
          // the producer loads the next image's weights once this warp's MMAs on the last set are done
          if (!mbar_wait_warp(smem_u32(bres), b_waits & 1u, a.err, SDX_DEV_WAIT_FULL, abort_flag)) break;
          tc_fence_after();
          cur_img = tile / a.img_tiles;
          b_waits++;
        }
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
  } else if (DWF && warp >= 2 + 4 * G) {
    // fused depthwise: thread t owns 8-channel group g = t % (C / 8) (its 72 per-image scaled weights
    // and 8 biases in registers) for GEMM rows r = t / (C / 8), + 128 / (C / 8), ... (tile pixel
    // (r / BW, r % BW)): bias, the nine taps in (ky, kx) order as one FMA each, the activation, fp16,
    // written into the 128-byte-swizzled A rows of the stage the MMA warp released. A warp reads whole
    // 128-byte halo rows (the box rows are 128-byte swizzled the same way).
    constexpr int NDW = 32 * TC_DW_WARPS;
    const int t = (int)threadIdx.x - tc_threads(G);
    const int C = a.dw_c, NG = C / 8, RS = NDW / NG;
    const int g = t % NG, r0 = t / NG;
    const int cb = g >> 3, ch = g & 7, c0 = g * 8;
    const int HW = a.BW + 2;
    uint64_t* hfull = reinterpret_cast<uint64_t*>(smem + a.dw_off + (size_t)a.dw_slots * a.dw_slot_bytes +
                                                  (size_t)10 * C * 4);
    uint64_t* hempty = hfull + 2;
    float w[9][8], bias[8];
#pragma unroll
    for (int j = 0; j < 8; j++) bias[j] = __ldg(a.dw_b + c0 + j);
    // activation without a per-value branch: v * sat(v * act_s + act_o) is hardswish (1/6, 1/2),
    // relu (+inf, 0: the factor is 1 for v > 0 and 0 otherwise, sat(NaN) being 0) or none (0, 1);
    // sdx_dw_pw admits only these three
    const float act_s = a.dw_act == ACT_HARDSWISH ? 1.0f / 6.0f : a.dw_act == ACT_RELU ? INFINITY : 0.0f;
    const float act_o = a.dw_act == ACT_HARDSWISH ? 0.5f : a.dw_act == ACT_RELU ? 0.0f : 1.0f;
    const int per_img = a.tiles_h * a.tiles_w;
    int s = 0, hs = 0, cur_img = -1;
    uint32_t phase = 0, hph = 0;
    for (int tile = t_begin; tile < t_end; tile += t_step) {
      const int img = tile / per_img;
      if (img != cur_img) {
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const float sc = a.dw_scale ? __ldg(a.dw_scale + (int64_t)img * C + c0 + j) : 1.0f;
#pragma unroll
          for (int k = 0; k < 9; k++) w[k][j] = __ldg(a.dw_w + k * C + c0 + j) * sc;
        }
        cur_img = img;
      }
      bool ok = mbar_wait(smem_u32(&hfull[hs]), hph, a.err, SDX_DEV_WAIT_FULL, abort_flag);
      ok = ok && mbar_wait(smem_u32(&empty[s]), phase ^ 1u, a.err, SDX_DEV_WAIT_EMPTY, abort_flag);
      if (named_bar_or(1, NDW, !ok)) break;
      const uint32_t hblk = smem_u32(smem + a.dw_off) + (uint32_t)hs * a.dw_slot_bytes + (uint32_t)cb * a.dw_blk_bytes;
      const uint32_t ablk = smem_u32(sA) + (uint32_t)s * a.a_stage_bytes + (uint32_t)cb * a.a_blk_bytes;
#pragma unroll 1
      for (int row = r0; row < TC_BM; row += RS) {
        const int py = row / a.BW, px = row - py * a.BW;
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; j++) acc[j] = bias[j];
#pragma unroll
        for (int ky = 0; ky < 3; ky++)
#pragma unroll
          for (int kx = 0; kx < 3; kx++) {
            const uint32_t pix = (uint32_t)((py + ky) * HW + px + kx);
            uint4 u;
            lds16(hblk + pix * 128u + (((uint32_t)ch ^ (pix & 7u)) << 4), u);
            const __half2* h2 = reinterpret_cast<const __half2*>(&u);
#pragma unroll
            for (int j = 0; j < 4; j++) {
              const float2 f = __half22float2(h2[j]);
              acc[2 * j] = fmaf(f.x, w[ky * 3 + kx][2 * j], acc[2 * j]);
              acc[2 * j + 1] = fmaf(f.y, w[ky * 3 + kx][2 * j + 1], acc[2 * j + 1]);
            }
          }
        uint4 o;
        __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const float v0 = acc[2 * j] * __saturatef(fmaf(acc[2 * j], act_s, act_o));
          const float v1 = acc[2 * j + 1] * __saturatef(fmaf(acc[2 * j + 1], act_s, act_o));
          oh[j] = __floats2half2_rn(v0, v1);
        }
        sts16(ablk + (uint32_t)row * 128u + (((uint32_t)ch ^ ((uint32_t)row & 7u)) << 4), o);
      }
      fence_async_smem();  // the generic-proxy A writes, before the MMAs (async proxy) read them
      named_bar_sync(1, NDW);
      if (t == 0) {
        mbar_arrive(smem_u32(&full[s]));
        mbar_arrive(smem_u32(&hempty[hs]));
      }
      if (++s == S) {
        s = 0;
        phase ^= 1u;
      }
      if (++hs == a.dw_slots) {
        hs = 0;
        hph ^= 1u;
      }
    }
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
    // tile of this CTA's ordinal o (the order in which the MMA warp fills the accumulators), or -1
    auto ord_tile = [&](int o) -> int {
      if (a.mpair) {
        const int u = (int)blockIdx.x + (o >> 1) * (int)gridDim.x;
        if (u >= (a.m_tiles >> 1) * a.n_tiles) return -1;
        const int pi = u / a.n_tiles;
        return (2 * pi + (o & 1)) * a.n_tiles + (u - pi * a.n_tiles);
      }
      const int t = t_begin + o * t_step;
      return t < t_end ? t : -1;
    };
    const int tile0 = ord_tile(e);
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
    if (a.tma_res && tile0 >= 0) {
      issue_res(tile0, 0);
      res_pending = true;
    }

    uint32_t lc = 0;  // this group's tile count
    for (int o = e;; o += G, lc++) {
      const int tile = ord_tile(o);
      if (tile < 0) break;
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
      if (FAST && a.res && !a.tma_res) {
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
      if (FAST && a.res && !a.tma_res) cp_async_wait_all();
      if (!ok) break;
      __syncwarp();
      tc_fence_after();

      // output pixel of this row: only the per-thread paths (no TMA store, or a residual that TMA
      // cannot stage) need it
      bool valid = false;
      int64_t pix = 0;
      if (!FAST && (!a.tma_out || (a.res && !a.tma_res))) {
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
      if (EPI == 5) {
        // fused CTC head: this row's logits over the tile's columns, bias added, folded column by
        // column into (max, first index of the max, online softmax denominator) exactly as the
        // reference's UpdateArgMax does (a new maximum rescales the denominator by exp(old - new) and
        // adds 1; any other value adds exp(value - max)); the logits are never stored
        const int64_t row = (int64_t)tcd.m0 + row_in_tile;
        float m = -INFINITY, s = 0.0f;
        int best = 0;
        bool bad = false;
        const int nch = a.BN / 16;
        for (int c = 0; c < nch; c++) {
          float v[16];
          tmem_ld16_issue(tbase + (uint32_t)(c * 16), v);
          tmem_wait_ld();
          tmem_ld_wait16(v);
          if (c == nch - 1) {
            tc_fence_before();
            mbar_arrive(smem_u32(&acce[acc]));
          }
#pragma unroll
          for (int j = 0; j < 16; j++) {
            const int col = tcd.n0 + c * 16 + j;
            if (col < a.N) {
              const float x = v[j] + (a.bias ? __ldg(a.bias + col) : 0.0f);
              bad |= !isfinite(x);
              if (x > m) {
                s = s * expf(m - x) + 1.0f;
                m = x;
                best = col;
              } else {
                s += expf(x - m);
              }
            }
          }
        }
        if (row < a.M) {
          const int64_t o = (int64_t)(tcd.n0 / a.BN) * a.arg_ld + row;
          a.arg_m[o] = m;
          a.arg_i[o] = best;
          a.arg_s[o] = s;
        }
        if (bad) record_error(a.err, SDX_DEV_NONFINITE);
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
        const int halves = (a.N + 15) >> 4;  // 16-channel chunks
        const uint32_t kb = (uint32_t)a.BN / 3u;  // columns per column tap (32 or 64)
#pragma unroll
        for (int hf = 0; hf < 4; hf++) {
          if (hf < halves) {
            float v0[16], v1[16], v2[16];
            tmem_ld16_issue(tbase + (uint32_t)(hf * 16), v0);
            tmem_ld16_issue(tbase + kb + (uint32_t)(hf * 16), v1);
            tmem_ld16_issue(tbase + 2u * kb + (uint32_t)(hf * 16), v2);
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
      if (!FAST && a.kxn) {
        // kx-in-N: columns kx * kb + oc (kb = 32 or 64); row x of the tile is input column ox0 - 1 + x,
        // and the output at that column is D[x - 1][kx 0] + D[x][kx 1] + D[x + 1][kx 2] (neighbouring
        // lanes: the 32 rows of a warp are consecutive columns of one or two tile rows); 32 output
        // channels per pass
        const int kb = a.BN / 3;
        for (int c0 = 0; c0 < kb; c0 += 32) {
          float sum[32];
#pragma unroll
          for (int i = 0; i < 32; i++) sum[i] = 0.0f;
#pragma unroll
          for (int kx = 0; kx < 3; kx++) {
            float v[32];
            tmem_ld16_issue(tbase + (uint32_t)(kx * kb + c0), v);
            tmem_ld16_issue(tbase + (uint32_t)(kx * kb + c0 + 16), v + 16);
            tmem_wait_ld();
            tmem_ld_wait16(v);
            tmem_ld_wait16(v + 16);
            if (kx == 2 && c0 + 32 >= kb) {
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
            for (int q0 = 0; q0 < 32; q0 += 8) {
              const int o0 = c0 + q0;
              if (o0 >= a.N) break;
              float r8[8];
#pragma unroll
              for (int j = 0; j < 8; j++) {
                const int o = o0 + j;
                r8[j] = sum[q0 + j] + (a.bias_smem ? sBias[o] : (a.bias && o < a.N ? __ldg(a.bias + o) : 0.0f));
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
        }
        __syncwarp();
        continue;
      }
      const int nch = a.BN / 16;
      int g = 0, cg = 0;
      // channel sums of this warp's 32 rows (rows mode): its row of a.gap, warp-uniform
      float* gp = nullptr;
      int nlim = 0;
      if (DWF && a.gap) {
        // 32-pixel tile rows (BW = 32, OW a multiple of 32): the warp's rows are one 32-pixel run
        const int oy = tcd.oy0 + q;
        if (oy < a.OH) {
          gp = a.gap + ((((int64_t)tcd.img * a.OH + oy) * a.OW + tcd.ox0) >> 5) * a.N + tcd.n0;
          nlim = a.N - tcd.n0;
        }
      } else if (FAST && a.gap) {
        const int64_t r0 = (int64_t)tcd.m0 + q * 32;
        if (r0 < a.M) {
          if (a.fold > 1) {
            gp = a.gap + ((r0 * a.fold) >> 5) * a.bias_mod;  // the warp's first 32-pixel run
            nlim = a.bias_mod;
          } else {
            gp = a.gap + (r0 >> 5) * a.N + tcd.n0;
            nlim = a.N - tcd.n0;
          }
        }
      }
      if (FAST) {
        // chunk pairs: both chunks' TMEM loads in flight under one wait, the accumulator handed back
        // after the last pair's loads, before its arithmetic (two 16-float buffers: no spills at the
        // 96-register cap of four epilogue groups)
        for (int c = 0; c < nch; c += 2) {
          float v0[16], v1[16];
          const bool two = c + 1 < nch;
          tmem_ld16_issue(tbase + (uint32_t)c * 16u, v0);
          if (two) tmem_ld16_issue(tbase + (uint32_t)(c + 1) * 16u, v1);
          tmem_wait_ld();
          tmem_ld_wait16(v0);
          if (two) tmem_ld_wait16(v1);
          if (c + 2 >= nch) {
            tc_fence_before();
            mbar_arrive(smem_u32(&acce[acc]));
          }
          epi_chunk_fast<ACT>(a, v0, c, srow, xr, sBias + tcd.n0, res_smem);
          if (two) epi_chunk_fast<ACT>(a, v1, c + 1, srow, xr, sBias + tcd.n0, res_smem);
        }
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
        epi_chunk<ACT>(a, va, c, srow, xr, sBias, tcd, valid, pix, g, cg);
        if (c + 1 < nch) {
          tmem_wait_ld();
          tmem_ld_wait16(vb);
          if (c + 2 < nch) {
            tmem_ld16_issue(tbase + (uint32_t)(c + 2) * 16u, va);
          } else {
            tc_fence_before();
            mbar_arrive(smem_u32(&acce[acc]));
          }
          epi_chunk<ACT>(a, vb, c + 1, srow, xr, sBias, tcd, valid, pix, g, cg);
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
          if (FAST && gp && a.fold > 1) {
            if (a.fold == 4) gap_warp_rows_fold<4, 16, 1>(slab, a.group_bytes, lane, gp);
            else gap_warp_rows_fold<2, 32, 1>(slab, a.group_bytes, lane, gp);
          } else if (FAST && gp) {
            if (a.BN == 16) gap_warp_rows<16>(slab, a.group_bytes, lane, gp, nlim);
            else if (a.BN == 32) gap_warp_rows<32>(slab, a.group_bytes, lane, gp, nlim);
            else if (a.BN == 64) gap_warp_rows<64>(slab, a.group_bytes, lane, gp, nlim);
            else gap_warp_rows<128>(slab, a.group_bytes, lane, gp, nlim);
          }
          // the next tile's buffer is free once the store that last read it has read it; then its
          // residual rows can be fetched while this warp waits for the next accumulator
          if (ord_tile(o + G) >= 0) {
            if (a.nsbuf == 2) bulk_wait_read1(eld);
            else bulk_wait_read0(eld);
            if (a.tma_res) {
              issue_res(ord_tile(o + G), a.nsbuf == 2 ? ((lc + 1) & 1u) : 0u);
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

template <int ACT, int EPI, int G>
int launch_tc(int dev, int grid, size_t smem, cudaStream_t stream, const CUtensorMap& mA, const CUtensorMap& mB,
                     const CUtensorMap& mOut, const CUtensorMap& mRes, const TcArgs& a) {
  static SmemAttr attr{};
  const int rc = raise_smem_limit(attr, (const void*)conv_tc_kernel<ACT, EPI, G>, TC_SMEM_LIMIT,
                                  "cudaFuncSetAttribute(conv_tc)");
  if (rc) return rc;
  conv_tc_kernel<ACT, EPI, G><<<grid, tc_threads_epi(G, EPI), smem, stream>>>(mA, mB, mOut, mRes, a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "conv_tc launch");
  return SDX_OK;
}

}  // namespace sdx
