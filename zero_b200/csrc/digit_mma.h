// digit_mma.h — batched Q4_0 / Q8_0 matvec on the tensor cores that gives,
// for every vector, the single-vector GEMV's result bit for bit
// (digit_mma.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "internal.h"

namespace zgpu {

constexpr uint32_t kDmVec = 16;                              // vectors per MMA (a vector group)
constexpr uint32_t kDmN = 3 * kDmVec;                        // MMA columns: 3 digits x 16 vectors
constexpr uint32_t kDmImgBlock = kDmN * 32 + kDmVec * 4;     // image bytes per (vector group, block)
constexpr uint32_t kDmMaxVec = 32;        // vectors of one segment of a grouped (tabled) launch
constexpr uint32_t kDmMaxVecPlain = 256;  // vectors of a launch without vector tables

// Digit image of up to 32 vectors of in_dim floats: for each vector group g
// (16 vectors) and 32-element block b, at img + (g * bpr + b) * kDmImgBlock,
// the 48 x 32-byte MMA operand (row d * 16 + v: digit d of vector v, the
// three bytes of the GEMV image's integers, the two low ones stored minus
// 128 so that every digit is signed) in the K-major canonical layout, then
// the 16 vectors' f32 block scales.  n_img images side by side (image i at
// img + i * img_bytes(in_dim, n_vec)); vector v of image i reads
// x + i * x_img_stride + v * x_stride, or, with x_rows, row
// x_rows[i * kDmMaxVec + v] of x (x + row * x_stride); vectors at or past
// n_vec (or n_vec_of[i]) are zero.  norm_w: RMSNorm first, as the GEMV's
// prologue (same thread layout, same order).
struct DigitImageParams {
  const float *x;
  uint64_t x_stride, x_img_stride;
  const uint32_t *x_rows;
  const uint32_t *n_vec_of;
  const float *norm_w;
  float eps;
  uint32_t in_dim, n_vec, n_img;
  uint8_t *img;
  uint32_t *status;
  // optional: only the (image, vector) pairs pairs[i] = image << 8 | vector
  // for i < *n_pairs (at most max_pairs); the columns of absent vectors are
  // then left as they are (the matvec never reads their sums)
  const uint32_t *pairs, *n_pairs;
  uint32_t max_pairs;
};
inline uint32_t dm_groups(uint32_t n_vec) { return (n_vec + kDmVec - 1) / kDmVec; }
inline uint64_t dm_img_bytes(uint32_t in_dim, uint32_t n_vec) {
  return static_cast<uint64_t>(dm_groups(n_vec)) * (in_dim / 32) * kDmImgBlock;
}
cudaError_t launch_digit_image(const DigitImageParams &p, const LaunchCfg &lc);

// Weight tiles of the batched matvec: for each 128-row tile t and 32-element
// block b, at (t * bpr + b) * kDmTileBlock, the 128 rows' int8 weights w_j
// (n_j - 8 for Q4_0, q_j for Q8_0) in the MMA's K-major layout (4 KB), the
// rows' f32 block scales, and the rows' int32 sums of w_j.  Rows past `rows`
// in the last tile are zero.  Built once per tensor from its group streams.
constexpr uint32_t kDmTileBlock = 4096 + 128 * 4 + 128 * 4;
inline uint64_t dm_tile_bytes(uint64_t rows, uint32_t bpr) {
  return (rows + 127) / 128 * static_cast<uint64_t>(bpr) * kDmTileBlock;
}
cudaError_t launch_build_dm_tiles(const uint8_t *w, uint64_t gstride, uint32_t quant, uint32_t rows, uint32_t bpr,
                                  uint8_t *tiles, cudaStream_t s);

// Partial sums of n_seg matvecs against digit images: segment s multiplies
// the weight tiles at wt + s * wt_seg_stride (or w_tab[s % w_tab_mod]),
// rows x in_dim, by image s * img_seg (img_seg 0: one image for all), and
// writes part[((s * ks + c) * n_vec + v) * rows + r]: chunk c's sum of
// vector v for row r (ks = ceil(in_dim / 1024) chunks of 32 blocks).  A
// zero table entry skips its segment.  n_vec_of (per segment, device):
// fewer vectors than n_vec for that segment.
struct DmGemmParams {
  const uint8_t *wt;
  uint64_t wt_seg_stride;
  const unsigned long long *w_tab;
  uint32_t w_tab_mod;
  uint32_t rows, in_dim;
  const uint8_t *img;
  uint32_t img_seg;          // 1: image s for segment s, 0: image 0 for every segment
  uint32_t n_vec, n_seg;
  const uint32_t *n_vec_of;
  float *part;
  uint32_t *status;
};
cudaError_t launch_dm_gemm(const DmGemmParams &p, const LaunchCfg &lc);

// y = the chunk partials added in chunk order (from 0), then the GEMV's
// epilogue (EPI_STORE / EPI_RESADD / EPI_SWIGLU: gate rows 8u..8u+3 and up
// rows 8u+4..8u+7 give output rows 4u..4u+3) into out + s * out_seg_stride +
// v * out_vec_stride + row, or, with out_rows, into out_rows[s * kDmMaxVec +
// v] + row.
struct DmCombineParams {
  const float *part;
  uint32_t rows, ks, n_vec, n_seg;
  const uint32_t *n_vec_of;
  float *out;
  uint64_t out_seg_stride, out_vec_stride;
  float *const *out_rows;
  uint32_t epi;
  // optional: the launch covers only the (segment, vector) pairs pairs[i] =
  // segment << 8 | vector for i < *n_pairs (at most max_pairs), instead of
  // every segment x n_vec (a grouped launch whose segments hold few vectors)
  const uint32_t *pairs, *n_pairs;
  uint32_t max_pairs;
};
cudaError_t launch_dm_combine(const DmCombineParams &p, const LaunchCfg &lc);
cudaError_t dm_setup();

}  // namespace zgpu
