// Host side of the tcgen05 conv / GEMM path: tile planning, tensor maps, shared-memory plan and
// kernel dispatch (the kernel itself is conv_tc_kernel.cuh, instantiated in conv_tc_inst_*.cu),
// and the B-operand weight packing.
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


// Channel block of a K-long reduction: 64 channels (128-byte rows) when K pads to a multiple of 64,
// else 32 or 16, so at most 15 zero channels are padded in.
// weight bytes above which a k x k conv streams 32-channel blocks (they do not stay resident)
static constexpr size_t TC_KBLK32_WEIGHTS = 96 * 1024;

int tc_kblk(int K) {
  const int r = (K + 15) / 16 * 16;
  return r % 64 == 0 ? 64 : r % 32 == 0 ? 32 : 16;
}

static int tc_kpad(int K) {
  const int kb = tc_kblk(K);
  return (K + kb - 1) / kb * kb;
}

int tc_kpad_of(int K) { return tc_kpad(K); }

static CUtensorMapSwizzle swizzle_of(int row_bytes) {
  return row_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : row_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                                          : CU_TENSOR_MAP_SWIZZLE_32B;
}

static size_t b_stage_bytes_of(const TcArgs& a) {
  return a.b_resident ? 0 : (size_t)a.wterms * a.cps * a.b_taps * a.BN * a.kblk * 2;
}

static size_t smem_fixed(const TcArgs& a) {
  return 1024 + (size_t)a.egroups * a.nsbuf * a.sbuf_bytes + (((size_t)a.bias_smem * 4 + 15) & ~(size_t)15) +
         8 * (2 * TC_MAX_STAGES + 10 + 8 * TC_EPI_GROUPS_MAX) + 16 + (a.b_resident ? (size_t)a.b_total_bytes : 0) +
         a.dw_extra;
}

static size_t smem_bytes(const TcArgs& a) {
  return smem_fixed(a) + (size_t)a.stages * (a.a_stage_bytes + b_stage_bytes_of(a));
}

// end (from the 1024-aligned base) of the kernel's regular shared-memory layout: A stages, weights,
// staging, bias, barriers; the fused depthwise area follows at the next 1024-byte boundary
static size_t smem_layout_end(const TcArgs& a) {
  return smem_bytes(a) - 1024 - a.dw_extra;
}

int tc_launch(const TcProblem& p, cudaStream_t stream) {
  if (p.N <= 0 || p.K <= 0) return set_error(SDX_ERR_INVALID, "tc: empty problem");
  if (!aligned16(p.a) || !aligned16(p.w)) return set_error(SDX_ERR_INVALID, "tc: operands must be 16-byte aligned");
  const bool convt = p.convt_oc > 0;
  int BN, n_tiles;
  if (convt) tc_plan_n_convt(p.convt_kh, p.convt_kw, p.convt_oc, &BN, &n_tiles);
  else if (p.kxn) BN = 3 * tc_kxn_block(p.N), n_tiles = 1;
  else tc_plan_n(p.N, &BN, &n_tiles);
  // 128 output columns of a short reduction (pointwise convs): two 64-column tiles, whose fast
  // epilogue runs four warp groups instead of two; the packed weights are the same 128 rows, and
  // the two tiles of one row block run on neighbouring CTAs, so A's second read hits L2
  if (p.mode == TC_ROWS && !convt && BN == 128 && n_tiles == 1 && p.N == 128 && p.K <= 128 && !p.out_f32 &&
      p.fold <= 1 && p.img_rows == 0) {
    BN = 64;
    n_tiles = 2;
  }
  const int kpad = tc_kpad(p.K);
  int kblk = tc_kblk(p.K);
  // k x k convs with 128-column tiles whose weights cannot stay resident stream them with every
  // stage: 32-channel blocks halve the stage (A box + kh weight taps), so that four or more stages
  // are in flight instead of two (3x3 128->128 at 128x128: 545 -> 764 TFLOP/s; 64->128: 467 -> 628;
  // 512->256 at 64x64: 609 -> 892). 64-column tiles lose with it (128->64: 570 -> 524).
  if (p.mode == TC_CONV && !p.kxn && p.kh > 1 && kblk == 64 && p.N >= 128 &&
      (size_t)(p.wterms == 1 ? 1 : 2) * p.kh * p.kw * kpad * ((p.N + 15) / 16 * 16) * 2 > TC_KBLK32_WEIGHTS)
    kblk = 32;
  const int kbytes = kblk * 2;
  const bool imgw = p.img_rows > 0;
  // per-image weights: rows mode when whole 128-row tiles fit an image, else the 1x1 conv in pixel-tile
  // mode (tiles never straddle two images)
  if (imgw && (convt || n_tiles != 1 || p.fold > 1 || p.arg_m || p.gap || p.wterms != 2 ||
               (p.mode == TC_ROWS && (p.img_rows % TC_BM != 0 || p.M % p.img_rows != 0)) ||
               (p.mode == TC_CONV && (p.kh != 1 || p.kw != 1 || p.kxn))))
    return set_error(SDX_ERR_NOT_SUPPORTED,
                     "tc: per-image weights need a 1x1 conv with one N tile, two terms and no fused sums");
  const bool dwf = p.dw_w != nullptr;
  if (dwf && (p.mode != TC_CONV || p.kh != 1 || p.kw != 1 || p.kxn || convt || p.chain_w2 || p.arg_m || p.res ||
              p.fold > 1 || imgw || p.K % 64 != 0 || p.K > 128 || n_tiles != 1 || BN > 128 || p.out_f32 || !p.dw_b))
    return set_error(SDX_ERR_NOT_SUPPORTED,
                     "tc: the fused depthwise form needs a 1x1 conv over 64 or 128 channels to at most 128 fp16 "
                     "outputs, no residual");
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
  const bool argmax = p.arg_m != nullptr;
  if (argmax && (p.mode != TC_ROWS || convt || p.fold > 1 || p.gap || p.res || p.act != ACT_NONE || !p.arg_i ||
                 !p.arg_s))
    return set_error(SDX_ERR_INVALID, "tc: the fused CTC head is a plain rows-mode GEMM (no residual, act, sums)");
  a.arg_m = p.arg_m;
  a.arg_i = p.arg_i;
  a.arg_s = p.arg_s;
  a.arg_ld = p.arg_ld;
  if (argmax && p.arg_ld < p.M) return set_error(SDX_ERR_INVALID, "tc: argmax state stride below M");
  a.fold = p.fold > 1 ? p.fold : 1;
  a.bias_mod = p.bias_mod;
  if (a.fold > 1 && (p.mode != TC_ROWS || convt || p.N != 64 || p.bias_mod * a.fold != p.N || BN != 64 ||
                     n_tiles != 1))
    return set_error(SDX_ERR_INVALID, "tc: pixel folding needs rows mode and 64 folded columns");
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
    // and N = 3 x kb columns (kx, oc), kb = 32 or 64; the A box is BW = BWs + 2 input columns wide, starting one
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
  } else if (dwf) {
    // fused depthwise: 32 x 4 pixel tiles (a warp's 32 rows are one 32-pixel run of an image row);
    // tmA is the depthwise input, one {64, 34, 6, 1} halo box per channel block (zero fill = the
    // depthwise padding); the A blocks are written by the depthwise warps, not by TMA
    const int BW = 32, BH = TC_BM / BW;
    a.halo = 0;
    a.taps = 1;
    a.kw = 1;
    a.b_taps = 1;
    a.BH = BH;
    a.BW = BW;
    a.BWs = BW;
    a.OH = p.OH;
    a.OW = p.OW;
    a.tiles_h = (p.OH + BH - 1) / BH;
    a.tiles_w = (p.OW + BW - 1) / BW;
    a.m_tiles = p.batch * a.tiles_h * a.tiles_w;
    a.a_box_bytes = (uint32_t)(TC_BM * kbytes);
    a.a_blk_bytes = (a.a_box_bytes + 1023u) & ~1023u;
    a.dw_box_bytes = (uint32_t)((BW + 2) * (BH + 2) * kbytes);
    a.dw_blk_bytes = (a.dw_box_bytes + 1023u) & ~1023u;
    a.dw_slot_bytes = a.dw_blk_bytes * (uint32_t)a.kb_per_tap;
    a.dw_c = p.K;
    a.dw_w = p.dw_w;
    a.dw_b = p.dw_b;
    a.dw_scale = p.dw_scale;
    a.dw_act = p.dw_act;
    uint64_t dims[4] = {(uint64_t)p.C, (uint64_t)p.W, (uint64_t)p.H, (uint64_t)p.batch};
    uint64_t strides[3] = {(uint64_t)p.C * 2, (uint64_t)p.W * p.C * 2, (uint64_t)p.H * p.W * p.C * 2};
    uint32_t box[4] = {(uint32_t)kblk, (uint32_t)(BW + 2), (uint32_t)(BH + 2), 1};
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
    const uint64_t sets = !imgw ? 1 : p.mode == TC_ROWS ? (uint64_t)(p.M / p.img_rows) : (uint64_t)p.batch;
    uint64_t dims[2] = {(uint64_t)kpad, (uint64_t)a.wterms * a.taps * a.b_rows_per_tap * sets};
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
  if (argmax) tma_out = false;  // the fused CTC head stores no tensor
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
  const bool kxn_fast = p.kxn && !p.out_f32 && a.vec_ok && !p.res && p.N % 8 == 0 && BN * n_tiles <= TC_BIAS_SMEM_MAX;
  if (kxn_fast) a.bias_smem = BN * n_tiles;
  // ---- shared-memory plan. Preference: weights resident (loaded once per CTA) with 2 staging
  // buffers and >= 3 A stages, resident with 1 staging buffer and >= 2 stages, then streamed
  // weights (per stage) likewise. 8 stages at most.
  if (!a.tma_out) a.sbuf_bytes = 0;
  // every CTA keeps a single N tile when the grid (one CTA per SM, or one per tile) is a multiple
  // of n_tiles: then only that tile's weights need to be resident
  int dev = 0;
  cudaGetDevice(&dev);
  const int total = a.m_tiles * a.n_tiles;
  int grid = std::min(total, num_sms(dev));
  // pixel-tile pairs for halo-mode convs whose weights are streamed (decided with the smem plan): the
  // two tiles' A boxes share each weight stage; only with whole pairs and a pair per SM at least
  const bool pair_ok = p.mode == TC_CONV && a.halo && !p.kxn && !convt && !chain && !imgw && BN <= 128 &&
                       a.m_tiles % 2 == 0 && (a.m_tiles / 2) * n_tiles >= num_sms(dev) && !argmax;
  if (imgw && total > 0) {
    // contiguous tile ranges: each CTA crosses few image boundaries (weight reloads)
    a.img_tiles = p.mode == TC_ROWS ? p.img_rows / TC_BM : a.tiles_h * a.tiles_w;
    a.b_img_rows = a.wterms * a.taps * a.b_rows_per_tap;
    a.per_cta = (total + grid - 1) / grid;
    grid = (total + a.per_cta - 1) / a.per_cta;
  }
  a.b_nslice = (n_tiles > 1 && grid % n_tiles == 0) ? 1 : 0;
  a.b_total_bytes =
      (uint32_t)((size_t)a.wterms * a.taps * a.kb_per_tap * (a.b_nslice ? 1 : n_tiles) * BN * kbytes);
  // stages of cps channel blocks each (fewer, larger stages amortise the per-stage waits and
  // commits of the two issuing threads): the largest cps with >= 3 stages, else cps = 1 with >= 2
  bool planned = false;
  // four epilogue groups for thin tiles, and for the per-thread epilogue (ConvT scatter and other
  // general cases) up to 128 columns; two when the staging of four would crowd out the A stages
  if (p.res_up && !fast)
    return set_error(SDX_ERR_NOT_SUPPORTED, "tc: upsampled residual needs the fp16 TMA-store epilogue");
  if (p.gap && a.fold > 1 && (!fast || BN != 64 || n_tiles != 1 || a.G != 64 || p.M % 32 != 0))
    return set_error(SDX_ERR_NOT_SUPPORTED, "tc: folded channel sums need one 128-column tile, fast epilogue");
  if (dwf && (!fast || (p.gap && (p.OW % 32 != 0 || p.OH % 4 != 0))))
    return set_error(SDX_ERR_NOT_SUPPORTED, "tc: the fused depthwise form needs the fp16 TMA-store epilogue "
                                            "(channel sums: width a multiple of 32, height of 4)");
  if (p.gap && a.fold == 1 && !dwf && (!fast || p.mode == TC_CONV || convt || p.M % 32 != 0 || p.N % 16 != 0 ||
                (BN != 16 && BN != 32 && BN != 64 && BN != 128) || a.G != (BN < 64 ? BN : 64) ||
                (reinterpret_cast<uintptr_t>(p.gap) & 7)))
    return set_error(SDX_ERR_NOT_SUPPORTED,
                     "tc: fused channel sums need a 1x1 conv with the fp16 TMA-store epilogue, rows % 32 == 0, "
                     "oc 16, 32, 64 or a multiple of 128 and an 8-byte aligned sums buffer");
  if (chain) a.bias_smem = BN + 4 * p.convt_oc + 4;  // first bias, second ConvT's weights and bias
  // (96-column tiles of a short reduction, e.g. the largest FPN lateral: 0.75 -> 0.70 ms; with longer
  // reductions the fewer A stages that four staging groups leave cost more than they save)
  const bool eg4 = !p.kxn && 4 * BN <= 512 &&
                   (BN <= 64 || chain || (!fast && !kxn_fast) || (fast && BN <= 96 && p.K <= 64));
  // fused depthwise: two halo slots (the next tile's box lands while this one is consumed), else one
  for (int slots = dwf ? 2 : 0; slots >= (dwf ? 1 : 0) && !planned; slots--) {
  if (dwf) {
    a.dw_slots = slots;
    a.dw_extra = 1024u + (uint32_t)slots * a.dw_slot_bytes + 40u * (uint32_t)p.K + 64u;
  }
  for (int eg = (eg4 && !dwf) ? 4 : 2; eg >= 2 && !planned; eg -= 2) {
  a.egroups = eg;
  for (int res = 1; res >= (imgw ? 1 : 0) && !planned; res--) {
    for (int pass = 0; pass < 2 && !planned; pass++) {
      for (int cps = pass == 0 ? a.kb_per_tap : 1; cps >= 1 && !planned; cps--) {
        if (a.kb_per_tap % cps) continue;
        if (dwf && (!res || cps != a.kb_per_tap)) continue;  // resident weights, one stage per tile
        for (int nsb = a.tma_out ? 2 : 1; nsb >= 1 && !planned; nsb--) {
          a.b_resident = res;
          a.mpair = (pair_ok && !res) ? 1 : 0;
          a.nsbuf = nsb;
          a.cps = cps;
          a.a_stage_bytes = (uint32_t)(a.mpair ? 2 : 1) * cps * a.a_blk_bytes;
          const size_t fixed = smem_fixed(a);
          const size_t per = a.a_stage_bytes + b_stage_bytes_of(a);
          if (fixed >= (size_t)TC_SMEM_LIMIT) continue;
          const int st = (int)std::min<size_t>(TC_MAX_STAGES, ((size_t)TC_SMEM_LIMIT - fixed) / per);
          if (st >= (dwf ? 2 : pass == 0 ? 3 : (nsb == 2 ? 3 : 2))) {
            a.stages = st;
            planned = true;
          }
        }
      }
    }
  }
  }
  }
  if (!planned) return set_error(SDX_ERR_NOT_SUPPORTED, "tc: shared memory plan too large");
  if (a.mpair) grid = std::min((a.m_tiles / 2) * n_tiles, num_sms(dev));
  if (dwf && total > 0) {
    a.contig = 1;
    a.per_cta = (total + grid - 1) / grid;
    grid = (total + a.per_cta - 1) / a.per_cta;
  }
  size_t smem = smem_bytes(a);
  if (dwf) {
    a.dw_off = (uint32_t)((smem_layout_end(a) + 1023) & ~(size_t)1023);
    smem = 1024 + (size_t)a.dw_off + (size_t)a.dw_slots * a.dw_slot_bytes + 40 * (size_t)p.K + 64;
  }
  if (smem > (size_t)TC_SMEM_LIMIT) return set_error(SDX_ERR_NOT_SUPPORTED, "tc: shared memory plan too large");

  if (total == 0) return SDX_OK;
  int rc = SDX_OK;
  if (dwf) {
    SDX_ACT_DISPATCH(a.act, ACTC, rc = (launch_tc<ACTC, 6, 2>(dev, grid, smem, stream, mA, mB, mOut, mRes, a)));
  } else if (argmax) {
    rc = a.egroups == 4 ? launch_tc<ACT_NONE, 5, 4>(dev, grid, smem, stream, mA, mB, mOut, mRes, a)
                        : launch_tc<ACT_NONE, 5, 2>(dev, grid, smem, stream, mA, mB, mOut, mRes, a);
  } else if (chain && a.egroups == 4) {
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

// columns of one column tap in the kx-in-N layout: 32, or 64 for 33..64 output channels
int tc_kxn_block(int oc) { return oc <= 32 ? 32 : 64; }

size_t tc_kxn_weights_halves(int K, int OC, int terms) {
  return (size_t)(terms == 1 ? 1 : 2) * 3 * 3 * tc_kxn_block(OC) * (size_t)tc_kpad(K);
}

// weight bytes up to which a 33..64-output 3x3 conv takes the kx-in-N form (resident weights)
static constexpr size_t TC_KXN64_WEIGHTS = 150 * 1024;

bool tc_conv_kxn(int kh, int kw, int sh, int sw, int pt, int pl, int pb, int pr, int oc, int ic, int terms) {
  if (!(kh == 3 && kw == 3 && sh == 1 && sw == 1 && pt == 1 && pl == 1 && pb == 1 && pr == 1 && oc >= 8 && oc <= 64))
    return false;
  // 192-column tiles only while their weights stay resident (a streamed 192-column weight stage
  // leaves no room for a pipeline)
  return oc <= 32 || tc_kxn_weights_halves(ic, oc, terms) * 2 <= (size_t)TC_KXN64_WEIGHTS;
}


// kx-in-N weights: [terms][ky][kx * kb + o][Kpad] (kb = tc_kxn_block(OC)), rows o >= OC zero.
void tc_pack_conv_kxn(const float* w, int OC, int IC, int terms, __half* out) {
  const int kb = tc_kxn_block(OC);
  const size_t kpad = (size_t)tc_kpad(IC), lo = (size_t)3 * 3 * kb * kpad;
  memset(out, 0, sizeof(__half) * (terms == 1 ? 1 : 2) * lo);
  for (int o = 0; o < OC; o++)
    for (int c = 0; c < IC; c++)
      for (int ky = 0; ky < 3; ky++)
        for (int kx = 0; kx < 3; kx++) {
          const size_t idx = ((size_t)ky * 3 * kb + kx * kb + o) * kpad + c;
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

int tc_fold_factor(int64_t pixels, int IC, int OC) {
  // folded to 64-column tiles (the width whose fast epilogue runs four warp groups); pixels %
  // (32 * f): the folded rows come in whole 32-row runs (fused channel sums per 32 pixels)
  for (int f = 4; f >= 2; f /= 2)
    if (OC * f == 64 && IC * f <= 128 && pixels % (32 * f) == 0) return f;
  return 1;
}

// One thread per (image, packed element): the scaled weight v = (hi + lo) * s[image, k] split into
// two fp16 terms again (the padding columns k >= K stay zero).
__global__ void scale_weights_kernel(const __half* __restrict__ w, int terms, int64_t set, int kpad, int K,
                                     const float* __restrict__ s, int64_t total, __half* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / set, j = i - n * set;
    const int k = (int)(j % kpad);
    float v = __half2float(w[j]);
    if (terms == 2) v += __half2float(w[set + j]);
    v *= k < K ? __ldg(s + n * K + k) : 0.0f;
    const __half h = __float2half_rn(v);
    out[n * 2 * set + j] = h;
    out[n * 2 * set + set + j] = __float2half_rn(v - __half2float(h));
  }
}

int tc_scale_weights_launch(const __half* w, int terms, int rows, int kpad, int K, const float* s, int batch,
                            __half* out, cudaStream_t st) {
  if (!aligned16(out) || !aligned16(w)) return set_error(SDX_ERR_INVALID, "scaled weights: 16-byte aligned buffers");
  const int64_t set = (int64_t)rows * kpad, total = set * batch;
  if (total <= 0) return SDX_OK;
  int dev = 0;
  cudaGetDevice(&dev);
  const int grid = (int)std::min<int64_t>((total + 255) / 256, (int64_t)num_sms(dev) * 8);
  scale_weights_kernel<<<grid, 256, 0, st>>>(w, terms, set, kpad, K, s, total, out);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "scale_weights launch");
  count_launch();
  return SDX_OK;
}

size_t tc_fold_weights_halves(int IC, int OC, int fold, int terms) {
  return tc_weights_halves(OC * fold, IC * fold, 1, terms);
}

void tc_pack_conv_fold(const float* w, int OC, int IC, int fold, int terms, __half* out) {
  const int N = OC * fold, K = IC * fold;
  int BN, nt;
  tc_plan_n(N, &BN, &nt);
  const size_t rows = (size_t)BN * nt, kpad = (size_t)tc_kpad(K);
  const size_t lo = rows * kpad;
  memset(out, 0, sizeof(__half) * (terms == 1 ? 1 : 2) * lo);
  for (int j = 0; j < fold; j++)
    for (int o = 0; o < OC; o++)
      for (int c = 0; c < IC; c++) {
        const size_t idx = (size_t)(j * OC + o) * kpad + (size_t)(j * IC + c);
        const float v = w[(size_t)o * IC + c];
        if (terms == 1) out[idx] = __float2half_rn(v);
        else put2(out, idx, lo, v);
      }
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
