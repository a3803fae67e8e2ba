// attention.cu — standalone launch of the single-token GQA decode attention
// (the kernel body, shared with the persistent step kernel, is in
// attn_body.cuh).  Grid: (n_kv_heads, max_splits), 256 threads.
#include "attn_body.cuh"
#include "common.cuh"
#include "internal.h"
#include "ops.h"

namespace zgpu {

namespace {

struct BlockBar {
  __device__ __forceinline__ void operator()() const { __syncthreads(); }
};

__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const AttnParams p) {
  __shared__ AttnSmem sm;
  pdl_launch_dependents();
  pdl_wait();
  const uint32_t pos = p.pos_ptr ? *p.pos_ptr : p.pos_value;
  attn_decode_block(p, blockIdx.x, blockIdx.y, pos, threadIdx.x, sm, BlockBar());
}

}  // namespace

uint32_t attention_max_splits(uint32_t max_tokens) {
  return (max_tokens + kAttnSplitTokens - 1) / kAttnSplitTokens;
}

cudaError_t attention_setup() {
  return cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                              cudaSharedmemCarveoutMaxShared);
}

cudaError_t launch_attention(const AttnParams &ap, const LaunchCfg &lc) {
  if (ap.n_q % ap.n_kv != 0 || ap.n_q / ap.n_kv > kAttnMaxGqa || ap.n_q / ap.n_kv + 2 > kAttnWarps)
    return cudaErrorInvalidValue;
  if (ap.max_splits < attention_max_splits(ap.max_tokens)) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ap.n_kv, ap.max_splits);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = lc.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = lc.pdl ? 1 : 0;
  if (lc.launch_counter) ++*lc.launch_counter;
  return cudaLaunchKernelEx(&cfg, attn_decode_kernel, ap);
}

}  // namespace zgpu
