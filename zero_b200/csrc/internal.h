// internal.h — host-side structures shared by the zero-b200 modules.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <map>
#include <string>
#include <vector>

#include "../../include/zgpu.h"

namespace zgpu {

// Device copy of one registered tensor.  Matmul tensors are always held in
// the plane-chunk group layout of layout.h on the device, whatever layout the
// caller registered (plain rows or the .smodel-v2 X4 groups): group g of 4
// output rows is one contiguous stream of gstride bytes (a multiple of 16).
struct DeviceTensor {
  uint8_t *d = nullptr;       // device bytes
  size_t bytes = 0;
  uint32_t dtype = 0;         // dtype as registered
  uint32_t quant = 0;         // ZGPU_Q4_0 / ZGPU_Q8_0 / ZGPU_F32
  uint32_t interleave = 1;    // what group_of reports (registered layout)
  uint64_t rows = 0, cols = 0;
  uint64_t groups = 0;        // ceil(rows / 4)
  uint64_t gstride = 0;       // bytes per group stream on the device
  // batched-matmul operand tiles (ops.h), built on first batched use (Q4_0)
  int8_t *w8 = nullptr;
  float *ws8 = nullptr;
  // tiles of the digit-image matvec (digit_mma.h), built on first use
  uint8_t *dmt = nullptr;
};

// Geometry of one GEMV launch over a device tensor in the layout.h format.
struct GemvDesc {
  const uint8_t *w;           // group streams
  uint64_t gstride;           // bytes between groups
  uint32_t quant;             // ZGPU_Q4_0 / ZGPU_Q8_0
  uint32_t rows;              // valid output rows
  uint32_t groups;            // groups in the launch
  uint32_t in_dim;
  uint64_t wbytes = 0;        // bytes of the weight buffer (bounds checks)
  // Segmented launch: seg_count segments of `groups` groups each.  Segment s
  // streams its groups from the device address seg_w[s] (wbytes bytes from
  // there), reads its input at x + s * seg_x_stride and writes out + s *
  // seg_out_stride (floats).  No CTA spans two segments.  seg_dynamic: the
  // table is written by the preceding kernel, so the weight prefetch waits
  // for it (programmatic dependent launch) instead of starting early.
  const unsigned long long *seg_w = nullptr;
  uint32_t seg_count = 0;
  uint32_t seg_x_stride = 0, seg_out_stride = 0;
  bool seg_dynamic = false;
  // Batches: with seg_count > 1 and no table every segment streams w (the
  // same matrix for every sequence); segment s reads its input at
  // x + (s / seg_x_group) * seg_x_stride (several segments on one input, e.g.
  // a token's experts), and with seg_w_mod != 0 takes table entry
  // s % seg_w_mod (one table for every sequence).
  uint32_t seg_x_group = 1;
  uint32_t seg_w_mod = 0;
};

// PRO_Q8ACT: the input is Q8_0 blocks (34 bytes each: fp16 d, 32 int8) and
// the weights Q4_0 (the Q4_0 x Q8_0 GEMV of BASELINE config 1); store only.
enum GemvPro { PRO_PLAIN = 0, PRO_RMSNORM = 1, PRO_Q8ACT = 2 };
enum GemvEpi { EPI_STORE = 0, EPI_RESADD = 1, EPI_SWIGLU = 2, EPI_ARGMAX = 3 };

struct GemvIo {
  const float *x = nullptr;        // input vector (the residual for PRO_RMSNORM; Q8_0 blocks for PRO_Q8ACT)
  const float *norm_w = nullptr;   // RMSNorm gain (PRO_RMSNORM)
  float eps = 0.f;
  float *out = nullptr;            // STORE / RESADD / SWIGLU / ARGMAX (logits)
  unsigned long long *argmax = nullptr;
  uint32_t *status = nullptr;
};

struct LaunchCfg {
  cudaStream_t stream = nullptr;
  bool pdl = false;
  int sm_count = 148;
  uint32_t *launch_counter = nullptr;   // host-side count of kernel launches
};

cudaError_t launch_gemv(const GemvDesc &g, GemvPro pro, GemvEpi epi, const GemvIo &io,
                        const LaunchCfg &lc);
cudaError_t gemv_setup();

}  // namespace zgpu

struct zgpu_ctx {
  int device = 0;
  int sm_count = 0;
  int cc_major = 0, cc_minor = 0;
  uint32_t flags = 0;
  cudaStream_t stream = nullptr;
  std::string last_error;
  // the first expired device wait of the last status read (words 4..7 of
  // the status block: site, three values; site 0 when none was recorded)
  uint32_t last_wait[4] = {0, 0, 0, 0};
  std::map<uintptr_t, zgpu::DeviceTensor> weights;
  // scratch for the host-buffer entry points (grown on demand)
  float *d_x = nullptr, *d_y = nullptr;
  size_t d_x_cap = 0, d_y_cap = 0;
  uint32_t *d_status = nullptr;
  uint32_t launches = 0;
  // split-attention partials / arrival counters of the attention entry points
  float *d_attn_part = nullptr;
  size_t d_attn_part_cap = 0;
  uint32_t *d_attn_counters = nullptr;
  uint32_t d_attn_counters_cap = 0;
  // arrival counter of the MoE router entry point (zero between calls)
  uint32_t *d_route_counter = nullptr;
  // planar Q8_0 activations of the batched entry points
  uint8_t *d_q8 = nullptr;
  size_t d_q8_cap = 0;
};

// KV cache: layer-major [L][K block | V block], block = max_tokens x n_kv x
// head_dim f32, token stride n_kv*head_dim (kv_cache.rs:100-126).
struct zgpu_kv {
  zgpu_ctx *ctx = nullptr;
  float *d = nullptr;
  uint32_t max_tokens = 0, n_layers = 0, n_kv = 0, head_dim = 0;
  uint64_t block = 0;   // max_tokens * n_kv * head_dim
};

// Record an error message on the context and return the status.
zgpu_status zgpu_fail(zgpu_ctx *ctx, zgpu_status s, const std::string &msg);
zgpu_status zgpu_cuda_fail(zgpu_ctx *ctx, cudaError_t e, const char *what);
const zgpu::DeviceTensor *zgpu_lookup(const zgpu_ctx *ctx, const void *key);
// Copy a device status block back (synchronising the context stream), clear
// it when set and report a failed device bounds check; then map its error
// bits to a zgpu_status.
zgpu_status zgpu_read_device_status(zgpu_ctx *ctx, uint32_t *d_status, uint32_t *st_out);
zgpu_status zgpu_map_device_status(zgpu_ctx *ctx, uint32_t st);
