// attention_static.cu — decode attention whose scratch needs no allocation.
//
// zgpu_gqa_attention_decode_noalloc runs the same split-attention kernel as
// zgpu_gqa_attention_decode_device, but takes the kernel's scratch (split
// partials and per-kv-head arrival counters) from a fixed array that is part
// of this library's device image instead of memory the context allocates.
// It is meant for callers that must not allocate device memory while they
// run: hosts that reserve all device memory up front and hand out fixed
// buffers, runtimes that forbid allocation on their per-token path because
// an allocation can synchronise the device and stall unrelated work, and
// plugins whose memory is owned by an allocator that must not see foreign
// cudaMalloc calls.  Those callers still own every input and output.
//
// Limits and sharing:
//   * the array is kScratchBytes (1 MiB) and every GPU that loads this library
//     holds it until the process exits;
//   * the first kMaxKvHeads words are the counters, the rest holds the
//     partials: n_q_heads x ceil(max_tokens / 256) x (head_dim + 2) floats
//     must fit in kPartFloats, or the call is rejected before any launch;
//   * every call on a device shares the one array and leaves its contents
//     behind, so the counters are cleared on the caller's stream before each
//     launch, and calls that overlap on the GPU (other streams, other
//     contexts on the same device) race with each other.
#include <mutex>
#include <string>

#include "common.cuh"
#include "internal.h"
#include "ops.h"

namespace {

constexpr size_t kScratchBytes = 1u << 20;
constexpr uint32_t kMaxKvHeads = 256;
constexpr size_t kScratchFloats = kScratchBytes / sizeof(float);
constexpr size_t kPartFloats = kScratchFloats - kMaxKvHeads;
constexpr int kMaxDevices = 64;

// In host code this name only stands for the array; its device address comes
// from cudaGetSymbolAddress below.
static __device__ __align__(256) float g_attn_scratch[kScratchFloats];

std::mutex g_mu;
void *g_addr[kMaxDevices] = {};

// Device address of g_attn_scratch on `device`, looked up once per device
// with that device current and kept until the process exits (a device reset
// after the first call is not supported: the module would reload elsewhere).
zgpu_status scratch_address(zgpu_ctx *ctx, int device, float **out) {
  if (device < 0 || device >= kMaxDevices)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "attention (no-alloc): device index above 63");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_addr[device]) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "attention (no-alloc): cudaGetSymbolAddress");
    g_addr[device] = p;
  }
  *out = static_cast<float *>(g_addr[device]);
  return ZGPU_OK;
}

}  // namespace

extern "C" {

zgpu_status zgpu_gqa_attention_decode_noalloc(zgpu_ctx *ctx, zgpu_kv *kv, uint32_t layer,
                                              uint32_t pos, uint32_t n_q_heads, const float *d_qkv,
                                              const float *d_q_norm, const float *d_k_norm,
                                              const float *d_inv_freqs, float eps, float *d_out,
                                              void *stream) {
  if (!ctx || !kv || !d_qkv || !d_q_norm || !d_k_norm || !d_inv_freqs || !d_out)
    return ZGPU_ERR_INVALID_ARG;
  if (kv->ctx != ctx)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "attention (no-alloc): kv cache belongs to another context");
  if (layer >= kv->n_layers)
    return zgpu_fail(ctx, ZGPU_ERR_KV_LAYER_OUT_OF_RANGE, "attention (no-alloc): layer out of range");
  if (pos >= kv->max_tokens)
    return zgpu_fail(ctx, ZGPU_ERR_KV_TOKEN_OUT_OF_RANGE, "attention (no-alloc): position outside the kv cache");
  if (kv->head_dim != 128)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "attention (no-alloc): decode kernel requires head_dim 128");
  if (n_q_heads == 0 || n_q_heads % kv->n_kv != 0 || n_q_heads / kv->n_kv > 4)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "attention (no-alloc): n_q_heads must be 1..4 x n_kv_heads");
  const uint32_t splits = zgpu::attention_max_splits(kv->max_tokens);
  const size_t part = static_cast<size_t>(n_q_heads) * splits * (kv->head_dim + 2);
  if (kv->n_kv > kMaxKvHeads || part > kPartFloats)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG,
                     "attention (no-alloc): needs " + std::to_string(part) + " partial floats and " +
                         std::to_string(kv->n_kv) + " counters; the static scratch holds " +
                         std::to_string(kPartFloats) + " and " + std::to_string(kMaxKvHeads) +
                         " (use zgpu_gqa_attention_decode_device for larger caches)");
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "attention (no-alloc): cudaSetDevice");
  float *base = nullptr;
  zgpu_status s = scratch_address(ctx, ctx->device, &base);
  if (s) return s;
  uint32_t *counters = reinterpret_cast<uint32_t *>(base);
  const cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  e = cudaMemsetAsync(counters, 0, kv->n_kv * sizeof(uint32_t), st);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "attention (no-alloc): clear counters");
  zgpu::AttnParams ap = {};
  ap.qkv = d_qkv;
  ap.q_norm = d_q_norm;
  ap.k_norm = d_k_norm;
  ap.inv_freqs = d_inv_freqs;
  ap.kv_layer = kv->d + static_cast<size_t>(layer) * 2 * kv->block;
  ap.kv_block = kv->block;
  ap.max_tokens = kv->max_tokens;
  ap.pos_ptr = nullptr;
  ap.pos_value = pos;
  ap.out = d_out;
  ap.part = base + kMaxKvHeads;
  ap.counters = counters;
  ap.status = ctx->d_status;
  ap.n_q = n_q_heads;
  ap.n_kv = kv->n_kv;
  ap.max_splits = splits;
  ap.eps = eps;
  ap.scale = 1.0f / sqrtf(static_cast<float>(kv->head_dim));
  zgpu::LaunchCfg lc;
  lc.stream = st;
  lc.sm_count = ctx->sm_count;
  lc.launch_counter = &ctx->launches;
  e = zgpu::launch_attention(ap, lc);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "attention (no-alloc): launch");
  return ZGPU_OK;
}

}  // extern "C"
