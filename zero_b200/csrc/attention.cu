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

// Grid (n_kv_heads, max_splits, n_seq): the same block as above on
// sequence blockIdx.z's rows, cache and position.
__global__ void __launch_bounds__(kAttnThreads, 2)
    attn_decode_batch_kernel(const AttnParams p, const AttnBatchSeq *seqs, uint32_t layer, uint32_t qkv_stride,
                             uint32_t out_stride) {
  __shared__ AttnSmem sm;
  pdl_launch_dependents();
  pdl_wait();
  const uint32_t z = blockIdx.z;
  const AttnBatchSeq sq = seqs[z];
  AttnParams q = p;
  q.qkv = p.qkv + static_cast<size_t>(z) * qkv_stride;
  q.out = p.out + static_cast<size_t>(z) * out_stride;
  q.part = p.part + static_cast<size_t>(z) * p.n_q * p.max_splits * (kAttnHd + 2);
  q.counters = p.counters + static_cast<size_t>(z) * p.n_kv;
  q.kv_layer = sq.kv + static_cast<size_t>(layer) * 2 * sq.block;
  q.kv_block = sq.block;
  q.max_tokens = sq.max_tokens;
  attn_decode_block<BlockBar, false, 4, kAttnWarps, AttnNoMark, true>(q, blockIdx.x, blockIdx.y, sq.pos, threadIdx.x,
                                                                      sm, BlockBar());
}

}  // namespace

uint32_t attention_max_splits(uint32_t max_tokens) {
  return (max_tokens + kAttnSplitTokens - 1) / kAttnSplitTokens;
}

cudaError_t attention_setup() {
  cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                       cudaSharedmemCarveoutMaxShared);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attn_decode_batch_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
  return e;
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

cudaError_t launch_attention_batch(const AttnParams &ap, const AttnBatchSeq *seqs, uint32_t layer, uint32_t n_seq,
                                   uint32_t qkv_stride, uint32_t out_stride, const LaunchCfg &lc) {
  if (ap.n_q % ap.n_kv != 0 || ap.n_q / ap.n_kv > kAttnMaxGqa || ap.n_q / ap.n_kv + 2 > kAttnWarps)
    return cudaErrorInvalidValue;
  if (n_seq == 0 || n_seq > 65535 || ap.max_splits == 0 || !seqs) return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_launch_cfg(dim3(ap.n_kv, ap.max_splits, n_seq), dim3(kAttnThreads), 0, lc, attr);
  if (lc.launch_counter) ++*lc.launch_counter;
  return cudaLaunchKernelEx(&cfg, attn_decode_batch_kernel, ap, seqs, layer, qkv_stride, out_stride);
}

}  // namespace zgpu
