// ctx.cu — context, weight registry and the op-level C ABI entry points.
#include <cmath>
#include <cstring>
#include <new>
#include <thread>
#include <vector>

#include "common.cuh"
#include "digit_mma.h"
#include "internal.h"
#include "layout.h"
#include "ops.h"
#include "step.h"
#include "mla.h"
#include "moe.h"

using zgpu::DeviceTensor;

zgpu_status zgpu_fail(zgpu_ctx *ctx, zgpu_status s, const std::string &msg) {
  if (ctx) ctx->last_error = msg;
  return s;
}

zgpu_status zgpu_cuda_fail(zgpu_ctx *ctx, cudaError_t e, const char *what) {
  std::string m = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
  return zgpu_fail(ctx, e == cudaErrorMemoryAllocation ? ZGPU_ERR_OUT_OF_MEMORY : ZGPU_ERR_CUDA, m);
}

const DeviceTensor *zgpu_lookup(const zgpu_ctx *ctx, const void *key) {
  auto it = ctx->weights.find(reinterpret_cast<uintptr_t>(key));
  return it == ctx->weights.end() ? nullptr : &it->second;
}

#define ZCHECK(call, what)                                   \
  do {                                                       \
    cudaError_t e_ = (call);                                 \
    if (e_ != cudaSuccess) return zgpu_cuda_fail(ctx, e_, what); \
  } while (0)

extern "C" {

const char *zgpu_status_string(zgpu_status s) {
  switch (s) {
    case ZGPU_OK: return "ok";
    case ZGPU_ERR_INVALID_ARG: return "invalid argument";
    case ZGPU_ERR_UNSUPPORTED_QUANT: return "unsupported quant type";
    case ZGPU_ERR_UNREGISTERED_WEIGHT: return "weight key not registered";
    case ZGPU_ERR_KV_TOKEN_OUT_OF_RANGE: return "kv cache: token index out of range";
    case ZGPU_ERR_KV_LAYER_OUT_OF_RANGE: return "kv cache: layer out of range";
    case ZGPU_ERR_KV_INVALID_SLICE_LENGTH: return "kv cache: invalid slice length";
    case ZGPU_ERR_KV_TOKEN_COUNT_EXCEEDS_MAX: return "kv cache: token count exceeds max";
    case ZGPU_ERR_NUMERICAL_INSTABILITY: return "attention: numerical instability";
    case ZGPU_ERR_EMBED_UNSUPPORTED_QUANT: return "embedding: unsupported quant";
    case ZGPU_ERR_EMBED_DIM_MISALIGNMENT: return "embedding: dim misalignment";
    case ZGPU_ERR_LM_NON_FINITE_LOGITS: return "lm head: non-finite logits";
    case ZGPU_ERR_LM_ARGMAX_IN_PADDING: return "lm head: argmax in padding region";
    case ZGPU_ERR_MODEL_MAGIC: return "model file: magic mismatch";
    case ZGPU_ERR_MODEL_UNSUPPORTED: return "model file: unsupported format";
    case ZGPU_ERR_MODEL_INVALID: return "model file: invalid container";
    case ZGPU_ERR_MODEL_IO: return "model file: cannot open or map";
    case ZGPU_ERR_NO_DEVICE: return "no usable sm_100 device";
    case ZGPU_ERR_CUDA: return "cuda error";
    case ZGPU_ERR_OUT_OF_MEMORY: return "out of device memory";
    case ZGPU_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
  }
  return "unknown status";
}

zgpu_status zgpu_init(const zgpu_opts *opts, zgpu_ctx **out) {
  if (!out) return ZGPU_ERR_INVALID_ARG;
  *out = nullptr;
  if (opts && opts->abi_version != ZGPU_ABI_VERSION) return ZGPU_ERR_INVALID_ARG;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    cudaGetLastError();
    return ZGPU_ERR_NO_DEVICE;
  }
  const int dev = opts ? opts->device : 0;
  if (dev < 0 || dev >= n) return ZGPU_ERR_INVALID_ARG;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return ZGPU_ERR_NO_DEVICE;
  // The kernels are compiled for sm_100a only.
  if (prop.major != 10) return ZGPU_ERR_NO_DEVICE;
  zgpu_ctx *ctx = new (std::nothrow) zgpu_ctx();
  if (!ctx) return ZGPU_ERR_OUT_OF_MEMORY;
  ctx->device = dev;
  ctx->sm_count = prop.multiProcessorCount;
  ctx->cc_major = prop.major;
  ctx->cc_minor = prop.minor;
  ctx->flags = opts ? opts->flags : 0;
  if (cudaSetDevice(dev) != cudaSuccess ||
      cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&ctx->d_status, zgpu::kStatusWords * sizeof(uint32_t)) != cudaSuccess ||
      cudaMemset(ctx->d_status, 0, zgpu::kStatusWords * sizeof(uint32_t)) != cudaSuccess ||
      zgpu::gemv_setup() != cudaSuccess || zgpu::attention_setup() != cudaSuccess ||
      zgpu::ops_setup() != cudaSuccess || zgpu::step_setup() != cudaSuccess ||
      zgpu::moe_setup() != cudaSuccess || zgpu::mla_setup() != cudaSuccess ||
      zgpu::prefill_setup() != cudaSuccess || zgpu::mma_setup() != cudaSuccess || zgpu::dm_setup() != cudaSuccess ||
      cudaMalloc(&ctx->d_route_counter, sizeof(uint32_t)) != cudaSuccess ||
      cudaMemset(ctx->d_route_counter, 0, sizeof(uint32_t)) != cudaSuccess) {
    delete ctx;
    return ZGPU_ERR_CUDA;
  }
  *out = ctx;
  return ZGPU_OK;
}

zgpu_status zgpu_clear_weights(zgpu_ctx *ctx) {
  if (!ctx) return ZGPU_ERR_INVALID_ARG;
  cudaSetDevice(ctx->device);
  for (auto &kv : ctx->weights) {
    cudaFree(kv.second.d);
    cudaFree(kv.second.w8);
    cudaFree(kv.second.dmt);
  }
  ctx->weights.clear();
  return ZGPU_OK;
}

void zgpu_destroy(zgpu_ctx *ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->device);
  zgpu_clear_weights(ctx);
  cudaFree(ctx->d_x);
  cudaFree(ctx->d_y);
  cudaFree(ctx->d_attn_part);
  cudaFree(ctx->d_attn_counters);
  cudaFree(ctx->d_route_counter);
  cudaFree(ctx->d_q8);
  cudaFree(ctx->d_status);
  if (ctx->stream) cudaStreamDestroy(ctx->stream);
  delete ctx;
}

const char *zgpu_last_error(const zgpu_ctx *ctx) {
  return ctx ? ctx->last_error.c_str() : "null context";
}

zgpu_status zgpu_device_info(const zgpu_ctx *ctx, int32_t *sm_count, int32_t *cc_major,
                             int32_t *cc_minor) {
  if (!ctx) return ZGPU_ERR_INVALID_ARG;
  if (sm_count) *sm_count = ctx->sm_count;
  if (cc_major) *cc_major = ctx->cc_major;
  if (cc_minor) *cc_minor = ctx->cc_minor;
  return ZGPU_OK;
}

zgpu_status zgpu_synchronize(zgpu_ctx *ctx) {
  if (!ctx) return ZGPU_ERR_INVALID_ARG;
  ZCHECK(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
  return ZGPU_OK;
}

zgpu_status zgpu_register_weights(zgpu_ctx *ctx, const void *host_ptr, size_t len, uint32_t dtype,
                                  uint64_t rows, uint64_t cols) {
  if (!ctx || !host_ptr) return ZGPU_ERR_INVALID_ARG;
  cudaSetDevice(ctx->device);
  DeviceTensor t;
  t.dtype = dtype;
  t.rows = rows;
  t.cols = cols;
  if (dtype == ZGPU_F32) {
    if (len != rows * cols * 4) return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "f32 length mismatch");
    t.quant = ZGPU_F32;
    t.bytes = len;
    ZCHECK(cudaMalloc(&t.d, len), "cudaMalloc(weights)");
    ZCHECK(cudaMemcpy(t.d, host_ptr, len, cudaMemcpyHostToDevice), "upload");
  } else if (dtype == ZGPU_Q4_K || dtype == ZGPU_Q6_K) {
    // K-quants stay in their plain row layout
    if (cols == 0 || cols % 256 != 0 || rows == 0)
      return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "K-quant cols must be a positive multiple of 256");
    if (len != rows * (cols / 256) * (dtype == ZGPU_Q4_K ? 144 : 210))
      return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "byte length does not match rows x cols");
    if (cols > 65536) return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "K-quant cols above 65536");
    t.quant = dtype;
    if (dtype == ZGPU_Q4_K) {
      t.bytes = len;
      ZCHECK(cudaMalloc(&t.d, len), "cudaMalloc(weights)");
      ZCHECK(cudaMemcpy(t.d, host_ptr, len, cudaMemcpyHostToDevice), "upload");
    } else {
      // Q6_K: each 210-byte super-block padded to kQ6kStride bytes
      const size_t nb = len / 210;
      std::vector<uint8_t> pad(nb * zgpu::kQ6kStride, 0);
      const uint8_t *src = static_cast<const uint8_t *>(host_ptr);
      for (size_t b = 0; b < nb; ++b) std::memcpy(pad.data() + b * zgpu::kQ6kStride, src + b * 210, 210);
      t.bytes = pad.size();
      ZCHECK(cudaMalloc(&t.d, t.bytes), "cudaMalloc(weights)");
      ZCHECK(cudaMemcpy(t.d, pad.data(), t.bytes, cudaMemcpyHostToDevice), "upload");
    }
  } else {
    const bool x4 = (dtype == ZGPU_Q4_0X4 || dtype == ZGPU_Q8_0X4);
    const uint32_t quant = (dtype == ZGPU_Q4_0 || dtype == ZGPU_Q4_0X4)   ? ZGPU_Q4_0
                           : (dtype == ZGPU_Q8_0 || dtype == ZGPU_Q8_0X4) ? ZGPU_Q8_0
                                                                          : 0;
    if (!quant) return zgpu_fail(ctx, ZGPU_ERR_UNSUPPORTED_QUANT, "unsupported dtype");
    if (cols == 0 || cols % 32 != 0 || rows == 0)
      return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "cols must be a positive multiple of 32");
    if (x4 && rows % 4 != 0)
      return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "interleaved tensor rows must be a multiple of 4");
    const uint64_t bb = quant == ZGPU_Q4_0 ? 18 : 34;
    const uint64_t bpr = cols / 32;
    if (len != rows * bpr * bb)
      return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "byte length does not match rows x cols");
    t.quant = quant;
    t.interleave = x4 ? 4 : 1;
    // groups padded to an even count: the GEMV works on units of two groups
    t.groups = ((rows + 3) / 4 + 1) & ~uint64_t(1);
    t.gstride = zgpu::group_stream_bytes(quant, bpr);
    t.bytes = t.groups * t.gstride;
    // Re-lay the tensor out as plane chunks (layout.h) on the host, then
    // upload once.  Padded rows and groups stay zero blocks.
    std::vector<uint8_t> img;
    try {
      img.assign(t.bytes, 0);
    } catch (...) {
      return zgpu_fail(ctx, ZGPU_ERR_OUT_OF_MEMORY, "host staging allocation failed");
    }
    const uint8_t *src = static_cast<const uint8_t *>(host_ptr);
    const uint64_t gb = bpr * bb * 4;          // bytes of one X4 group stream
    const uint64_t body = bb - 2;              // quant bytes of one row-block
    const uint32_t P = zgpu::plane_count(quant);
    auto convert = [&](uint64_t g0, uint64_t g1) {
      for (uint64_t g = g0; g < g1; ++g) {
        uint8_t *dst = img.data() + g * t.gstride;
        for (uint64_t l = 0; l < 4; ++l) {
          const uint64_t r = g * 4 + l;
          if (r >= rows) break;
          for (uint64_t b = 0; b < bpr; ++b) {
            const uint8_t *d16, *q;
            if (x4) {
              const uint8_t *gbk = src + g * gb + b * bb * 4;   // [d0..d3][row0..row3 bodies]
              d16 = gbk + 2 * l;
              q = gbk + 8 + l * body;
            } else {
              const uint8_t *blk = src + (r * bpr + b) * bb;    // [d][body]
              d16 = blk;
              q = blk + 2;
            }
            std::memcpy(dst + zgpu::scale_entry(quant, bpr, b) + 2 * l, d16, 2);
            const uint32_t per_row = P / 4;                     // planes per row
            for (uint32_t h = 0; h < per_row; ++h)
              std::memcpy(dst + zgpu::plane_entry(quant, bpr, b, static_cast<uint32_t>(l) * per_row + h),
                          q + 16 * h, 16);
          }
        }
      }
    };
    const uint64_t ng = (rows + 3) / 4;
    const unsigned nt = ng >= 256 ? 8u : 1u;
    if (nt == 1) {
      convert(0, ng);
    } else {
      std::vector<std::thread> pool;
      for (unsigned i = 0; i < nt; ++i) pool.emplace_back(convert, ng * i / nt, ng * (i + 1) / nt);
      for (auto &th : pool) th.join();
    }
    src = img.data();
    ZCHECK(cudaMalloc(&t.d, t.bytes), "cudaMalloc(weights)");
    ZCHECK(cudaMemcpy(t.d, src, t.bytes, cudaMemcpyHostToDevice), "upload");
  }
  auto key = reinterpret_cast<uintptr_t>(host_ptr);
  auto it = ctx->weights.find(key);
  if (it != ctx->weights.end()) {
    cudaFree(it->second.d);
    cudaFree(it->second.w8);
    cudaFree(it->second.dmt);
  }
  ctx->weights[key] = t;
  return ZGPU_OK;
}

uint32_t zgpu_group_of(const zgpu_ctx *ctx, const void *host_ptr) {
  if (!ctx) return 1;
  const DeviceTensor *t = zgpu_lookup(ctx, host_ptr);
  return t ? t->interleave : 1;
}

}  // extern "C"

static zgpu_status ensure_scratch(zgpu_ctx *ctx, size_t nx, size_t ny) {
  if (nx > ctx->d_x_cap) {
    cudaFree(ctx->d_x);
    ctx->d_x = nullptr;
    ZCHECK(cudaMalloc(&ctx->d_x, nx * sizeof(float)), "cudaMalloc(scratch x)");
    ctx->d_x_cap = nx;
  }
  if (ny > ctx->d_y_cap) {
    cudaFree(ctx->d_y);
    ctx->d_y = nullptr;
    ZCHECK(cudaMalloc(&ctx->d_y, ny * sizeof(float)), "cudaMalloc(scratch y)");
    ctx->d_y_cap = ny;
  }
  return ZGPU_OK;
}

static zgpu_status check_status_word(zgpu_ctx *ctx) {
  uint32_t sw[zgpu::kStatusWords] = {0};
  ZCHECK(cudaMemcpyAsync(sw, ctx->d_status, sizeof(sw), cudaMemcpyDeviceToHost, ctx->stream), "status");
  ZCHECK(cudaStreamSynchronize(ctx->stream), "sync");
  const uint32_t st = sw[0];
  if (st) {
    cudaMemsetAsync(ctx->d_status, 0, sizeof(sw), ctx->stream);
    if (sw[1])
      return zgpu_fail(ctx, ZGPU_ERR_CUDA, "device bounds check " + std::to_string(sw[1]) + " failed (" +
                                               std::to_string(sw[2]) + ", " + std::to_string(sw[3]) + ")");
    if (st & zgpu::ZDEV_ERR_TIMEOUT)
      return zgpu_fail(ctx, ZGPU_ERR_DEVICE_TIMEOUT, "device wait timed out");
    if (st & zgpu::ZDEV_ERR_NUMERICAL)
      return zgpu_fail(ctx, ZGPU_ERR_NUMERICAL_INSTABILITY, "non-finite input or softmax state");
    return zgpu_fail(ctx, ZGPU_ERR_CUDA, "device status " + std::to_string(st));
  }
  return ZGPU_OK;
}

static zgpu_status linear_device(zgpu_ctx *ctx, const float *d_x, const void *w_key, float *d_out,
                                 uint64_t in_dim, uint64_t out_dim, uint32_t quant,
                                 cudaStream_t stream) {
  if (quant != ZGPU_Q4_0 && quant != ZGPU_Q8_0 && quant != ZGPU_Q4_K && quant != ZGPU_Q6_K)
    return zgpu_fail(ctx, ZGPU_ERR_UNSUPPORTED_QUANT,
                     "linear_dispatch: unsupported quant type " + std::to_string(quant));
  const DeviceTensor *t = zgpu_lookup(ctx, w_key);
  if (!t) return zgpu_fail(ctx, ZGPU_ERR_UNREGISTERED_WEIGHT, "linear_dispatch: unregistered weight");
  if (t->quant != quant || t->cols != in_dim || t->rows != out_dim)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "linear_dispatch: shape/quant mismatch with registration");
  if (quant == ZGPU_Q4_K || quant == ZGPU_Q6_K) {
    ZCHECK(zgpu::launch_gemv_kquant(t->d, quant, static_cast<uint32_t>(out_dim), static_cast<uint32_t>(in_dim), d_x,
                                    d_out, stream),
           "K-quant GEMV");
    ++ctx->launches;
    return ZGPU_OK;
  }
  zgpu::GemvDesc g;
  g.w = t->d;
  g.wbytes = t->bytes;
  g.gstride = t->gstride;
  g.quant = t->quant;
  g.rows = static_cast<uint32_t>(out_dim);
  g.groups = static_cast<uint32_t>(t->groups);
  g.in_dim = static_cast<uint32_t>(in_dim);
  zgpu::GemvIo io;
  io.x = d_x;
  io.out = d_out;
  io.status = ctx->d_status;
  zgpu::LaunchCfg lc;
  lc.stream = stream ? stream : ctx->stream;
  lc.pdl = true;   // the weight prefetch of back-to-back calls overlaps the previous call's tail
  lc.sm_count = ctx->sm_count;
  lc.launch_counter = &ctx->launches;
  cudaError_t e = zgpu::launch_gemv(g, zgpu::PRO_PLAIN, zgpu::EPI_STORE, io, lc);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "launch_gemv");
  return ZGPU_OK;
}

extern "C" {

zgpu_status zgpu_linear_dispatch_device(zgpu_ctx *ctx, const float *d_x, const void *w_key,
                                        float *d_out, uint64_t in_dim, uint64_t out_dim,
                                        uint32_t quant, void *stream) {
  if (!ctx || !d_x || !d_out) return ZGPU_ERR_INVALID_ARG;
  cudaSetDevice(ctx->device);
  return linear_device(ctx, d_x, w_key, d_out, in_dim, out_dim, quant,
                       static_cast<cudaStream_t>(stream));
}

zgpu_status zgpu_linear_dispatch(zgpu_ctx *ctx, const float *x, const void *w_key, float *out,
                                 uint64_t in_dim, uint64_t out_dim, uint32_t quant) {
  if (!ctx || !x || !out) return ZGPU_ERR_INVALID_ARG;
  cudaSetDevice(ctx->device);
  zgpu_status s = ensure_scratch(ctx, in_dim, out_dim);
  if (s) return s;
  ZCHECK(cudaMemcpyAsync(ctx->d_x, x, in_dim * 4, cudaMemcpyHostToDevice, ctx->stream), "h2d x");
  s = linear_device(ctx, ctx->d_x, w_key, ctx->d_y, in_dim, out_dim, quant, ctx->stream);
  if (s) return s;
  ZCHECK(cudaMemcpyAsync(out, ctx->d_y, out_dim * 4, cudaMemcpyDeviceToHost, ctx->stream), "d2h out");
  return check_status_word(ctx);
}

zgpu_status zgpu_rmsnorm(zgpu_ctx *ctx, const float *x, const float *w, float *out, uint64_t n,
                         float eps) {
  if (!ctx || !x || !w || !out || n == 0) return ZGPU_ERR_INVALID_ARG;
  cudaSetDevice(ctx->device);
  zgpu_status s = ensure_scratch(ctx, 2 * n, n);
  if (s) return s;
  ZCHECK(cudaMemcpyAsync(ctx->d_x, x, n * 4, cudaMemcpyHostToDevice, ctx->stream), "h2d");
  ZCHECK(cudaMemcpyAsync(ctx->d_x + n, w, n * 4, cudaMemcpyHostToDevice, ctx->stream), "h2d");
  ZCHECK(zgpu::launch_rmsnorm(ctx->d_x, ctx->d_x + n, ctx->d_y, static_cast<uint32_t>(n), eps,
                              ctx->stream), "rmsnorm");
  ++ctx->launches;
  ZCHECK(cudaMemcpyAsync(out, ctx->d_y, n * 4, cudaMemcpyDeviceToHost, ctx->stream), "d2h");
  ZCHECK(cudaStreamSynchronize(ctx->stream), "sync");
  return ZGPU_OK;
}

zgpu_status zgpu_rope(zgpu_ctx *ctx, float *qk, uint32_t n_heads, uint32_t head_dim, uint32_t pos,
                      float freq_base) {
  if (!ctx || !qk || n_heads == 0 || head_dim == 0 || head_dim % 2) return ZGPU_ERR_INVALID_ARG;
  cudaSetDevice(ctx->device);
  const uint32_t half = head_dim / 2;
  std::vector<float> inv(half);
  // RopeContext::new (ops.rs:79-93): powf(base, -2*i / head_dim) in f32.
  const float hdf = static_cast<float>(head_dim);
  for (uint32_t i = 0; i < half; ++i) {
    const float exponent = -2.0f * static_cast<float>(i) / hdf;
    inv[i] = powf(freq_base, exponent);
  }
  const size_t n = static_cast<size_t>(n_heads) * head_dim;
  zgpu_status s = ensure_scratch(ctx, n + half, 1);
  if (s) return s;
  ZCHECK(cudaMemcpyAsync(ctx->d_x, qk, n * 4, cudaMemcpyHostToDevice, ctx->stream), "h2d");
  ZCHECK(cudaMemcpyAsync(ctx->d_x + n, inv.data(), half * 4, cudaMemcpyHostToDevice, ctx->stream), "h2d");
  ZCHECK(zgpu::launch_rope(ctx->d_x, ctx->d_x + n, n_heads, head_dim, pos, ctx->stream), "rope");
  ++ctx->launches;
  ZCHECK(cudaMemcpyAsync(qk, ctx->d_x, n * 4, cudaMemcpyDeviceToHost, ctx->stream), "d2h");
  ZCHECK(cudaStreamSynchronize(ctx->stream), "sync");
  return ZGPU_OK;
}

zgpu_status zgpu_silu_mul(zgpu_ctx *ctx, const float *gate, const float *up, float *out, uint64_t n) {
  if (!ctx || !gate || !up || !out || n == 0) return ZGPU_ERR_INVALID_ARG;
  cudaSetDevice(ctx->device);
  zgpu_status s = ensure_scratch(ctx, 2 * n, n);
  if (s) return s;
  ZCHECK(cudaMemcpyAsync(ctx->d_x, gate, n * 4, cudaMemcpyHostToDevice, ctx->stream), "h2d");
  ZCHECK(cudaMemcpyAsync(ctx->d_x + n, up, n * 4, cudaMemcpyHostToDevice, ctx->stream), "h2d");
  ZCHECK(zgpu::launch_silu_mul(ctx->d_x, ctx->d_x + n, ctx->d_y, n, ctx->stream), "silu_mul");
  ++ctx->launches;
  ZCHECK(cudaMemcpyAsync(out, ctx->d_y, n * 4, cudaMemcpyDeviceToHost, ctx->stream), "d2h");
  ZCHECK(cudaStreamSynchronize(ctx->stream), "sync");
  return ZGPU_OK;
}

zgpu_status zgpu_quantize_q8_0(zgpu_ctx *ctx, const float *x, void *blocks_out, uint64_t n) {
  if (!ctx || !x || !blocks_out || n == 0 || n % 32) return ZGPU_ERR_INVALID_ARG;
  cudaSetDevice(ctx->device);
  const size_t nb = n / 32;
  // x in d_x, blocks in d_y (34 bytes per block fits in 32 floats per block)
  zgpu_status s = ensure_scratch(ctx, n, (nb * 34 + 3) / 4);
  if (s) return s;
  ZCHECK(cudaMemcpyAsync(ctx->d_x, x, n * 4, cudaMemcpyHostToDevice, ctx->stream), "h2d");
  ZCHECK(zgpu::launch_quantize_q8_0(ctx->d_x, reinterpret_cast<uint8_t *>(ctx->d_y), n,
                                    ctx->d_status, ctx->stream), "quantize_q8_0");
  ++ctx->launches;
  ZCHECK(cudaMemcpyAsync(blocks_out, ctx->d_y, nb * 34, cudaMemcpyDeviceToHost, ctx->stream), "d2h");
  return check_status_word(ctx);
}

// The Q4_0 x Q8_0 GEMV on the standalone GEMV kernel's
// streaming path with a one-digit activation image.
static cudaError_t q8act_launch(zgpu_ctx *ctx, const DeviceTensor *t, uint64_t in_dim, uint64_t out_dim,
                                const uint8_t *d_xq, float *d_out, cudaStream_t stream) {
  zgpu::GemvDesc g;
  g.w = t->d;
  g.wbytes = t->bytes;
  g.gstride = t->gstride;
  g.quant = t->quant;
  g.rows = static_cast<uint32_t>(out_dim);
  g.groups = static_cast<uint32_t>(t->groups);
  g.in_dim = static_cast<uint32_t>(in_dim);
  zgpu::GemvIo io;
  io.x = reinterpret_cast<const float *>(d_xq);
  io.out = d_out;
  io.status = ctx->d_status;
  zgpu::LaunchCfg lc;
  lc.stream = stream;
  lc.pdl = true;
  lc.sm_count = ctx->sm_count;
  return zgpu::launch_gemv(g, zgpu::PRO_Q8ACT, zgpu::EPI_STORE, io, lc);
}

zgpu_status zgpu_linear_q8act_device(zgpu_ctx *ctx, const void *d_xq, const void *w_key,
                                     float *d_out, uint64_t in_dim, uint64_t out_dim, void *stream) {
  if (!ctx || !d_xq || !d_out || in_dim == 0 || in_dim % 32) return ZGPU_ERR_INVALID_ARG;
  cudaSetDevice(ctx->device);
  const DeviceTensor *t = zgpu_lookup(ctx, w_key);
  if (!t) return zgpu_fail(ctx, ZGPU_ERR_UNREGISTERED_WEIGHT, "linear_q8act: unregistered weight");
  if (t->quant != ZGPU_Q4_0)
    return zgpu_fail(ctx, ZGPU_ERR_UNSUPPORTED_QUANT, "linear_q8act: weights must be Q4_0");
  if (t->cols != in_dim || t->rows != out_dim)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "linear_q8act: shape mismatch with registration");
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  ZCHECK(q8act_launch(ctx, t, in_dim, out_dim, static_cast<const uint8_t *>(d_xq), d_out, s), "q8act gemv");
  ++ctx->launches;
  return ZGPU_OK;
}

zgpu_status zgpu_linear_q8act(zgpu_ctx *ctx, const void *xq_blocks, const void *w_key, float *out,
                              uint64_t in_dim, uint64_t out_dim) {
  if (!ctx || !xq_blocks || !out || in_dim == 0 || in_dim % 32) return ZGPU_ERR_INVALID_ARG;
  cudaSetDevice(ctx->device);
  const DeviceTensor *t = zgpu_lookup(ctx, w_key);
  if (!t) return zgpu_fail(ctx, ZGPU_ERR_UNREGISTERED_WEIGHT, "linear_q8act: unregistered weight");
  if (t->quant != ZGPU_Q4_0)
    return zgpu_fail(ctx, ZGPU_ERR_UNSUPPORTED_QUANT, "linear_q8act: weights must be Q4_0");
  if (t->cols != in_dim || t->rows != out_dim)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "linear_q8act: shape mismatch with registration");
  const size_t xbytes = in_dim / 32 * 34;
  zgpu_status s = ensure_scratch(ctx, (xbytes + 3) / 4, out_dim);
  if (s) return s;
  ZCHECK(cudaMemcpyAsync(ctx->d_x, xq_blocks, xbytes, cudaMemcpyHostToDevice, ctx->stream), "h2d");
  ZCHECK(q8act_launch(ctx, t, in_dim, out_dim, reinterpret_cast<const uint8_t *>(ctx->d_x), ctx->d_y, ctx->stream), "q8act gemv");
  ++ctx->launches;
  ZCHECK(cudaMemcpyAsync(out, ctx->d_y, out_dim * 4, cudaMemcpyDeviceToHost, ctx->stream), "d2h");
  ZCHECK(cudaStreamSynchronize(ctx->stream), "sync");
  return ZGPU_OK;
}

// Batched form: T rows of f32 activations, quantised to Q8_0 per row on the
// device, times Q4_0 weights on the tcgen05 int8 path (mma_gemm.cu).
static zgpu_status q8act_batch(zgpu_ctx *ctx, const float *d_x, const void *w_key, float *d_out, uint64_t T,
                               uint64_t in_dim, uint64_t out_dim, cudaStream_t s) {
  const DeviceTensor *t = zgpu_lookup(ctx, w_key);
  if (!t) return zgpu_fail(ctx, ZGPU_ERR_UNREGISTERED_WEIGHT, "linear_q8act_batch: unregistered weight");
  if (t->quant != ZGPU_Q4_0 && t->quant != ZGPU_Q8_0)
    return zgpu_fail(ctx, ZGPU_ERR_UNSUPPORTED_QUANT, "linear_q8act_batch: weights must be Q4_0 or Q8_0");
  if (t->cols != in_dim || t->rows != out_dim)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "linear_q8act_batch: shape mismatch with registration");
  if (out_dim % 128 || T > 0xFFFFFFu || T * in_dim > (1ull << 34))
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "linear_q8act_batch: rows must be a multiple of 128");
  const uint32_t bpr = static_cast<uint32_t>(in_dim / 32);
  // the weights' operand tiles, once per tensor
  DeviceTensor *wt = const_cast<DeviceTensor *>(t);
  if (!wt->w8) {
    ZCHECK(cudaMalloc(&wt->w8, zgpu::mma_tile_bytes(out_dim, bpr)), "cudaMalloc(weight tiles)");
    wt->ws8 = reinterpret_cast<float *>(wt->w8);   // the scales sit beside each 4 KB tile
    ZCHECK(zgpu::launch_build_w8_tiles(wt->d, wt->gstride, static_cast<uint32_t>(out_dim), bpr, t->quant, wt->w8, wt->ws8, s),
           "weight tiles");
    ++ctx->launches;
  }
  // scratch: activation tiles with their scales
  const size_t qbytes = zgpu::mma_tile_bytes(T, bpr), dbytes = 0;
  if (qbytes + dbytes > ctx->d_q8_cap) {
    cudaFree(ctx->d_q8);
    ctx->d_q8 = nullptr;
    ctx->d_q8_cap = 0;
    ZCHECK(cudaMalloc(&ctx->d_q8, qbytes + dbytes), "cudaMalloc(q8 scratch)");
    ctx->d_q8_cap = qbytes + dbytes;
  }
  int8_t *q = reinterpret_cast<int8_t *>(ctx->d_q8);
  float *d = reinterpret_cast<float *>(ctx->d_q8);
  ZCHECK(zgpu::launch_quantize_q8_0_tiles(d_x, q, d, static_cast<uint32_t>(T), static_cast<uint32_t>(in_dim),
                                         ctx->d_status, s),
         "q8 tiles");
  zgpu::MmaGemmParams p = {};
  p.wt = wt->w8;
  p.ws = wt->ws8;
  p.xt = q;
  p.xs = d;
  p.rows = static_cast<uint32_t>(out_dim);
  p.bpr = bpr;
  p.T = static_cast<uint32_t>(T);
  p.ldy = static_cast<uint32_t>(out_dim);
  p.y = d_out;
  p.status = ctx->d_status;
  ZCHECK(zgpu::launch_q4q8_mma(p, s), "q4q8 mma");
  ctx->launches += 2;
  return ZGPU_OK;
}

zgpu_status zgpu_linear_q8act_batch_device(zgpu_ctx *ctx, const float *d_x, const void *w_key, float *d_out,
                                           uint64_t T, uint64_t in_dim, uint64_t out_dim, void *stream) {
  if (!ctx || !d_x || !d_out || T == 0 || in_dim == 0 || in_dim % 32) return ZGPU_ERR_INVALID_ARG;
  cudaSetDevice(ctx->device);
  return q8act_batch(ctx, d_x, w_key, d_out, T, in_dim, out_dim,
                     stream ? static_cast<cudaStream_t>(stream) : ctx->stream);
}

zgpu_status zgpu_linear_dispatch_batch(zgpu_ctx *ctx, const float *x, const void *w_key, float *out,
                                       uint64_t n_vec, uint64_t in_dim, uint64_t out_dim, uint32_t quant) {
  if (!ctx || !x || !out || n_vec == 0 || in_dim == 0 || in_dim % 32) return ZGPU_ERR_INVALID_ARG;
  if (n_vec > zgpu::kDmMaxVecPlain)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "linear_dispatch_batch: at most 256 vectors");
  if (quant != ZGPU_Q4_0 && quant != ZGPU_Q8_0)
    return zgpu_fail(ctx, ZGPU_ERR_UNSUPPORTED_QUANT, "linear_dispatch_batch: Q4_0 or Q8_0 weights");
  DeviceTensor *t = const_cast<DeviceTensor *>(zgpu_lookup(ctx, w_key));
  if (!t) return zgpu_fail(ctx, ZGPU_ERR_UNREGISTERED_WEIGHT, "linear_dispatch_batch: unregistered weight");
  if (t->quant != quant || t->cols != in_dim || t->rows != out_dim)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "linear_dispatch_batch: shape/quant mismatch with registration");
  cudaSetDevice(ctx->device);
  if (!t->dmt) {
    ZCHECK(cudaMalloc(&t->dmt, zgpu::dm_tile_bytes(out_dim, static_cast<uint32_t>(in_dim / 32))), "cudaMalloc(tiles)");
    ZCHECK(zgpu::launch_build_dm_tiles(t->d, t->gstride, quant, static_cast<uint32_t>(out_dim),
                                       static_cast<uint32_t>(in_dim / 32), t->dmt, ctx->stream),
           "weight tiles");
    ++ctx->launches;
  }
  zgpu_status s = ensure_scratch(ctx, n_vec * in_dim, n_vec * out_dim);
  if (s) return s;
  const uint32_t nv = static_cast<uint32_t>(n_vec), ind = static_cast<uint32_t>(in_dim),
                 rows = static_cast<uint32_t>(out_dim);
  const uint32_t ks = (ind / 32 + zgpu::kChunkBlocks - 1) / zgpu::kChunkBlocks;
  const size_t img = zgpu::dm_img_bytes(ind, nv), part = static_cast<size_t>(ks) * nv * rows * 4;
  if (img + part > ctx->d_q8_cap) {
    cudaFree(ctx->d_q8);
    ctx->d_q8 = nullptr;
    ctx->d_q8_cap = 0;
    ZCHECK(cudaMalloc(&ctx->d_q8, img + part), "cudaMalloc(digit image scratch)");
    ctx->d_q8_cap = img + part;
  }
  ZCHECK(cudaMemcpyAsync(ctx->d_x, x, n_vec * in_dim * 4, cudaMemcpyHostToDevice, ctx->stream), "h2d");
  zgpu::LaunchCfg lc;
  lc.stream = ctx->stream;
  lc.pdl = !(ctx->flags & ZGPU_FLAG_NO_PDL);
  lc.sm_count = ctx->sm_count;
  lc.launch_counter = &ctx->launches;
  zgpu::DigitImageParams ip = {};
  ip.x = ctx->d_x;
  ip.x_stride = ind;
  ip.in_dim = ind;
  ip.n_vec = nv;
  ip.n_img = 1;
  ip.img = ctx->d_q8;
  ip.status = ctx->d_status;
  ZCHECK(zgpu::launch_digit_image(ip, lc), "digit image");
  zgpu::DmGemmParams gp = {};
  gp.wt = t->dmt;
  gp.rows = rows;
  gp.in_dim = ind;
  gp.img = ctx->d_q8;
  gp.n_vec = nv;
  gp.n_seg = 1;
  gp.part = reinterpret_cast<float *>(ctx->d_q8 + img);
  gp.status = ctx->d_status;
  ZCHECK(zgpu::launch_dm_gemm(gp, lc), "digit mma");
  zgpu::DmCombineParams cp = {};
  cp.part = gp.part;
  cp.rows = rows;
  cp.ks = ks;
  cp.n_vec = nv;
  cp.n_seg = 1;
  cp.out = ctx->d_y;
  cp.out_vec_stride = rows;
  cp.epi = zgpu::EPI_STORE;
  ZCHECK(zgpu::launch_dm_combine(cp, lc), "digit combine");
  ZCHECK(cudaMemcpyAsync(out, ctx->d_y, n_vec * out_dim * 4, cudaMemcpyDeviceToHost, ctx->stream), "d2h");
  return check_status_word(ctx);
}

zgpu_status zgpu_linear_q8act_batch(zgpu_ctx *ctx, const float *x, const void *w_key, float *out, uint64_t T,
                                    uint64_t in_dim, uint64_t out_dim) {
  if (!ctx || !x || !out || T == 0 || in_dim == 0 || in_dim % 32) return ZGPU_ERR_INVALID_ARG;
  cudaSetDevice(ctx->device);
  zgpu_status s = ensure_scratch(ctx, T * in_dim, T * out_dim);
  if (s) return s;
  ZCHECK(cudaMemcpyAsync(ctx->d_x, x, T * in_dim * 4, cudaMemcpyHostToDevice, ctx->stream), "h2d");
  if ((s = q8act_batch(ctx, ctx->d_x, w_key, ctx->d_y, T, in_dim, out_dim, ctx->stream))) return s;
  ZCHECK(cudaMemcpyAsync(out, ctx->d_y, T * out_dim * 4, cudaMemcpyDeviceToHost, ctx->stream), "d2h");
  return check_status_word(ctx);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Single-layer GQA decode attention (steps 2-5 of
// gqa_attention_single_token_dispatch, crates/zero-llm-inference/src/
// attention.rs:344-425): per-head QK RMSNorm, RoPE at `pos`, store_kv, then
// softmax(q.k / sqrt(hd)) . V over tokens 0..pos.
// ---------------------------------------------------------------------------

// Argument checks shared by both attention entry points; the error codes are
// the ones the reference's KvCache / attention paths return.
static zgpu_status attention_check(zgpu_ctx *ctx, const zgpu_kv *kv, uint32_t layer, uint32_t pos,
                                   uint32_t n_q) {
  if (kv->ctx != ctx) return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "attention: kv cache belongs to another context");
  if (layer >= kv->n_layers) return zgpu_fail(ctx, ZGPU_ERR_KV_LAYER_OUT_OF_RANGE, "attention: layer out of range");
  if (pos >= kv->max_tokens)
    return zgpu_fail(ctx, ZGPU_ERR_KV_TOKEN_OUT_OF_RANGE, "attention: position outside the kv cache");
  if (kv->head_dim != 128)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "attention: decode kernel requires head_dim 128");
  if (n_q == 0 || n_q % kv->n_kv != 0 || n_q / kv->n_kv > 4)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "attention: n_q_heads must be 1..4 x n_kv_heads");
  return ZGPU_OK;
}

// Grow the context's split partials [n_q][splits][hd + 2] and per-kv-head
// arrival counters.  Counters start at zero; the kernel's merging CTA resets
// its counter, so they stay zero between launches.
static zgpu_status ensure_attn_scratch(zgpu_ctx *ctx, size_t part_floats, uint32_t n_counters) {
  if (part_floats > ctx->d_attn_part_cap) {
    cudaFree(ctx->d_attn_part);
    ctx->d_attn_part = nullptr;
    ctx->d_attn_part_cap = 0;
    ZCHECK(cudaMalloc(&ctx->d_attn_part, part_floats * sizeof(float)), "cudaMalloc(attention partials)");
    ctx->d_attn_part_cap = part_floats;
  }
  if (n_counters > ctx->d_attn_counters_cap) {
    cudaFree(ctx->d_attn_counters);
    ctx->d_attn_counters = nullptr;
    ctx->d_attn_counters_cap = 0;
    ZCHECK(cudaMalloc(&ctx->d_attn_counters, n_counters * sizeof(uint32_t)), "cudaMalloc(attention counters)");
    ZCHECK(cudaMemset(ctx->d_attn_counters, 0, n_counters * sizeof(uint32_t)), "zero attention counters");
    ctx->d_attn_counters_cap = n_counters;
  }
  return ZGPU_OK;
}

static zgpu_status attention_device(zgpu_ctx *ctx, zgpu_kv *kv, uint32_t layer, uint32_t pos,
                                    uint32_t n_q, const float *d_qkv, const float *d_q_norm,
                                    const float *d_k_norm, const float *d_inv_freqs, float eps,
                                    float *d_out, cudaStream_t stream) {
  const uint32_t splits = zgpu::attention_max_splits(kv->max_tokens);
  zgpu_status s = ensure_attn_scratch(ctx, static_cast<size_t>(n_q) * splits * (kv->head_dim + 2), kv->n_kv);
  if (s) return s;
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
  ap.part = ctx->d_attn_part;
  ap.counters = ctx->d_attn_counters;
  ap.status = ctx->d_status;
  ap.n_q = n_q;
  ap.n_kv = kv->n_kv;
  ap.max_splits = splits;
  ap.eps = eps;
  ap.scale = 1.0f / sqrtf(static_cast<float>(kv->head_dim));
  zgpu::LaunchCfg lc;
  lc.stream = stream;
  lc.sm_count = ctx->sm_count;
  lc.launch_counter = &ctx->launches;
  ZCHECK(zgpu::launch_attention(ap, lc), "launch_attention");
  return ZGPU_OK;
}

extern "C" {

zgpu_status zgpu_gqa_attention_decode_device(zgpu_ctx *ctx, zgpu_kv *kv, uint32_t layer,
                                             uint32_t pos, uint32_t n_q_heads, const float *d_qkv,
                                             const float *d_q_norm, const float *d_k_norm,
                                             const float *d_inv_freqs, float eps, float *d_out,
                                             void *stream) {
  if (!ctx || !kv || !d_qkv || !d_q_norm || !d_k_norm || !d_inv_freqs || !d_out)
    return ZGPU_ERR_INVALID_ARG;
  zgpu_status s = attention_check(ctx, kv, layer, pos, n_q_heads);
  if (s) return s;
  cudaSetDevice(ctx->device);
  return attention_device(ctx, kv, layer, pos, n_q_heads, d_qkv, d_q_norm, d_k_norm, d_inv_freqs,
                          eps, d_out, stream ? static_cast<cudaStream_t>(stream) : ctx->stream);
}

zgpu_status zgpu_sample_top_k(zgpu_ctx *ctx, const float *logits, uint32_t len, uint32_t vocab_real, float temperature,
                              uint64_t *rng_state, uint32_t *token_out) {
  if (!ctx || !logits || !rng_state || !token_out || len == 0 || vocab_real == 0) return ZGPU_ERR_INVALID_ARG;
  cudaSetDevice(ctx->device);
  zgpu_status s = ensure_scratch(ctx, len, 4);   // y: rng state (2 words) | token
  if (s) return s;
  unsigned long long *d_rng = reinterpret_cast<unsigned long long *>(ctx->d_y);
  uint32_t *d_tok = reinterpret_cast<uint32_t *>(ctx->d_y + 2);
  ZCHECK(cudaMemcpyAsync(ctx->d_x, logits, static_cast<size_t>(len) * 4, cudaMemcpyHostToDevice, ctx->stream),
         "h2d logits");
  ZCHECK(cudaMemcpyAsync(d_rng, rng_state, 8, cudaMemcpyHostToDevice, ctx->stream), "h2d rng");
  ZCHECK(zgpu::launch_sample_topk(ctx->d_x, len, vocab_real, temperature, d_rng, d_tok, ctx->stream), "sample");
  ++ctx->launches;
  ZCHECK(cudaMemcpyAsync(token_out, d_tok, 4, cudaMemcpyDeviceToHost, ctx->stream), "d2h token");
  ZCHECK(cudaMemcpyAsync(rng_state, d_rng, 8, cudaMemcpyDeviceToHost, ctx->stream), "d2h rng");
  ZCHECK(cudaStreamSynchronize(ctx->stream), "sync");
  return ZGPU_OK;
}

zgpu_status zgpu_causal_attention(zgpu_ctx *ctx, zgpu_kv *kv, uint32_t layer, uint32_t pos0, uint32_t T,
                                  uint32_t n_q_heads, const float *q, float *out) {
  if (!ctx || !kv || !q || !out || T == 0) return ZGPU_ERR_INVALID_ARG;
  if (layer >= kv->n_layers) return zgpu_fail(ctx, ZGPU_ERR_KV_LAYER_OUT_OF_RANGE, "layer out of range");
  if (static_cast<uint64_t>(pos0) + T > kv->max_tokens)
    return zgpu_fail(ctx, ZGPU_ERR_KV_TOKEN_OUT_OF_RANGE, "query positions beyond the cache");
  if (kv->head_dim != 128 || !n_q_heads || n_q_heads % kv->n_kv)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "causal attention requires head_dim 128 and n_q a multiple of n_kv");
  cudaSetDevice(ctx->device);
  const size_t n = static_cast<size_t>(T) * n_q_heads * kv->head_dim;
  zgpu_status s = ensure_scratch(ctx, n, n);
  if (s) return s;
  ZCHECK(cudaMemcpyAsync(ctx->d_x, q, n * 4, cudaMemcpyHostToDevice, ctx->stream), "h2d q");
  ZCHECK(zgpu::launch_causal_attn(ctx->d_x, kv->d + static_cast<size_t>(layer) * 2 * kv->block, kv->block, n_q_heads,
                                  kv->n_kv, pos0, T, 1.0f / sqrtf(static_cast<float>(kv->head_dim)), ctx->d_y,
                                  ctx->d_status, ctx->stream),
         "launch_causal_attn");
  ++ctx->launches;
  ZCHECK(cudaMemcpyAsync(out, ctx->d_y, n * 4, cudaMemcpyDeviceToHost, ctx->stream), "d2h out");
  return check_status_word(ctx);
}

zgpu_status zgpu_gqa_attention_decode(zgpu_ctx *ctx, zgpu_kv *kv, uint32_t layer, uint32_t pos,
                                      uint32_t n_q_heads, const float *qkv, const float *q_norm,
                                      const float *k_norm, float freq_base, float eps, float *out) {
  if (!ctx || !kv || !qkv || !q_norm || !k_norm || !out) return ZGPU_ERR_INVALID_ARG;
  zgpu_status s = attention_check(ctx, kv, layer, pos, n_q_heads);
  if (s) return s;
  cudaSetDevice(ctx->device);
  const uint32_t hd = kv->head_dim, half = hd / 2;
  // RopeContext::new (ops.rs:79-93): powf(base, -2*i / head_dim) in f32.
  std::vector<float> inv(half);
  for (uint32_t i = 0; i < half; ++i)
    inv[i] = powf(freq_base, -2.0f * static_cast<float>(i) / static_cast<float>(hd));
  const size_t nqkv = static_cast<size_t>(n_q_heads + 2 * kv->n_kv) * hd;
  const size_t nout = static_cast<size_t>(n_q_heads) * hd;
  s = ensure_scratch(ctx, nqkv + 2 * hd + half, nout);
  if (s) return s;
  float *d_qkv = ctx->d_x, *d_qn = d_qkv + nqkv, *d_kn = d_qn + hd, *d_inv = d_kn + hd;
  ZCHECK(cudaMemcpyAsync(d_qkv, qkv, nqkv * 4, cudaMemcpyHostToDevice, ctx->stream), "h2d qkv");
  ZCHECK(cudaMemcpyAsync(d_qn, q_norm, hd * 4, cudaMemcpyHostToDevice, ctx->stream), "h2d q_norm");
  ZCHECK(cudaMemcpyAsync(d_kn, k_norm, hd * 4, cudaMemcpyHostToDevice, ctx->stream), "h2d k_norm");
  ZCHECK(cudaMemcpyAsync(d_inv, inv.data(), half * 4, cudaMemcpyHostToDevice, ctx->stream), "h2d rope");
  s = attention_device(ctx, kv, layer, pos, n_q_heads, d_qkv, d_qn, d_kn, d_inv, eps, ctx->d_y,
                       ctx->stream);
  if (s) return s;
  ZCHECK(cudaMemcpyAsync(out, ctx->d_y, nout * 4, cudaMemcpyDeviceToHost, ctx->stream), "d2h out");
  return check_status_word(ctx);
}

}  // extern "C"
