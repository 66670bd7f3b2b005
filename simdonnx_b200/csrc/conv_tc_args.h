// Tile-level arguments of the tcgen05 conv / GEMM kernel (conv_tc_kernel.cuh) shared by the host
// planner (conv_tc.cu) and the per-activation kernel instantiation units (conv_tc_inst_*.cu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace sdx {

constexpr int TC_BM = 128;
// Epilogue warp groups (kernel template G): 2, or 4 for tiles of at most 64 columns (more warps
// hide the per-tile latency of thin tiles); a CTA is the producer warp, the MMA warp and G groups.
constexpr int TC_EPI_GROUPS_MAX = 4;
constexpr int tc_threads(int groups) { return 64 + 128 * groups; }
constexpr int TC_DW_WARPS = 4;  // depthwise warps of the fused depthwise -> pointwise form (EPI = 6): one
                                // per scheduler, so that the CTA stays within 128 registers a thread
// kx-in-N 3x3 convs (EPI = 2) add a second MMA-issuing warp: their thin N = 96 MMAs are issue
// bound from one warp; two warps take alternate tiles
constexpr int tc_threads_epi(int groups, int epi) {
  return tc_threads(groups) + (epi == 6 ? 32 * TC_DW_WARPS : epi == 2 ? 32 : 0);
}
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
  // pixel folding (rows mode): each GEMM row holds `fold` consecutive pixels (A = [M, fold * K]
  // over the same memory, block-diagonal weights, N = fold * OC columns); the bias repeats every
  // bias_mod columns and the channel sums are per 32 pixels, i.e. per 32 / fold rows: [M * fold / 32][OC]
  int fold;
  int bias_mod;
  // fused CTC head (kernel template EPI = 5): per row and N tile, the running (max, first index of
  // the max, online softmax denominator) over the tile's columns, stored [n_tile][M]; no output
  float* arg_m;
  int* arg_i;
  float* arg_s;
  int arg_ld;  // entries between two N tiles' states (>= M)
  // resident weights of this CTA's N tile only (compact [term][tap][cb] layout): with a grid that
  // is a multiple of n_tiles every CTA keeps one N tile (tile = m * n_tiles + n, strided by the grid)
  int b_nslice;
  // per-image weights (rows mode, one N tile): the B map holds one weight set per image, b_img_rows
  // rows apart, and m tile t belongs to image t / img_tiles. Each CTA then runs the contiguous m-tile
  // range [blockIdx.x * per_cta, + per_cta) and reloads its resident weights when the image changes.
  // img_tiles = 0: one weight set, tiles strided by the grid.
  int img_tiles;
  int per_cta;
  int b_img_rows;
  // pixel-tile pairs (halo mode, streamed weights, m_tiles even): unit u = (pair u / n_tiles, N tile
  // u % n_tiles) covers m tiles 2 * pair and 2 * pair + 1, whose A boxes share every weight stage
  // (half the weight traffic per MMA); units are strided by the grid, tiles of a unit consecutive
  int mpair;
  // fused depthwise 3x3 (stride 1, pad 1) in front of a 1x1 conv (kernel template EPI = 6): TC_DW_WARPS
  // extra warps compute each tile's A block from a TMA-loaded halo box of the depthwise input (tmA:
  // box {64, BW + 2, BH + 2, 1}, 128-byte swizzle) and write it, swizzled, into the A stage; the
  // depthwise output never leaves the SM. Shared memory at dw_off: dw_slots halo slots, the [9][C] scaled
  // weights and [C] bias, four mbarriers (halo full / empty).
  const float* dw_w;      // [9][C] fp32
  const float* dw_b;      // [C] fp32
  const float* dw_scale;  // [batch][C] per-image input scale (an SE gate), or null
  int dw_act;
  int dw_c;
  uint32_t dw_off, dw_slot_bytes, dw_blk_bytes, dw_box_bytes, dw_extra;
  int dw_slots;           // halo slots: 2, or 1 when two do not fit (128 channels)
  int contig;             // 1: each CTA runs the contiguous tile range [blockIdx.x * per_cta, + per_cta)
                          // (the fused depthwise form: per-image weights change rarely)
  unsigned int* err;
};

// Launches conv_tc_kernel<ACT, EPI, G>; one explicit instantiation per (ACT, EPI, G) the planner
// uses, spread over conv_tc_inst_*.cu so that the kernels compile in parallel.
template <int ACT, int EPI, int G>
int launch_tc(int dev, int grid, size_t smem, cudaStream_t stream, const CUtensorMap& mA, const CUtensorMap& mB,
              const CUtensorMap& mOut, const CUtensorMap& mRes, const TcArgs& a);

}  // namespace sdx
