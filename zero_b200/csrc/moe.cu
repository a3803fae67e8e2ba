// moe.cu — MoE router (moe_route_f32) and the weighted combine of moe_ffn.
//
// Router (crates/zero-llm-inference/src/moe.rs:132-317).  Expert ids must be
// bit-identical to the reference's, so each expert's score is the
// reference's own sequential f32 dot product: one thread per expert walks
// the hidden vector in order with separately rounded multiplies and adds
// (no FMA contraction, no tree).  That chain is latency-bound (dim dependent
// adds), so the experts are spread over several CTAs that each stage their
// rows and the input in shared memory with coalesced loads first; the last
// CTA to finish (arrival counter) runs the replacement-min top-k, the
// softmax / normalisation over the selected k, the uniform fallbacks and
// the expert_weight_scale exactly as the reference orders them.  It then
// writes the dispatch tables of the grouped expert GEMVs: the device
// address of each selected expert's gate/up and down group streams, shared
// experts first, so the following launches need no host round trip.
//
// Combine (moe.rs:534-589 then forward_pass.rs:894-897): mlp_out = shared
// outputs (the first written, later ones added), then mlp_out[i] += w_k *
// expert_k[i] for k in selection order (multiply, then add), then
// hidden[i] += mlp_out[i].
#include <cfloat>
#include <cmath>

#include "common.cuh"
#include "internal.h"
#include "moe.h"
#include "ops.h"

namespace zgpu {

namespace {

constexpr int kRouteThreads = 256;
constexpr uint32_t kRouteRowFloats = 16384;   // staged router floats per CTA
constexpr uint32_t kRouteRowPad = 4;          // floats of padding per staged row

__device__ __forceinline__ float route_scale(float s) {
  return (isfinite(s) && s > 0.0f) ? s : 1.0f;
}

__device__ void route_uniform(float *w, uint32_t k, float scale) {
  const float u = __fdiv_rn(1.0f, static_cast<float>(k));
  const float s = route_scale(scale);
  for (uint32_t i = 0; i < k; ++i) w[i] = (s != 1.0f) ? __fmul_rn(u, s) : u;
}

// This CTA's token (grid dimension y) of a batch: the per-token vectors of
// RouteParams rebased on it.
__device__ __forceinline__ RouteParams route_seq(const RouteParams &p0) {
  RouteParams p = p0;
  const uint32_t b = blockIdx.y;
  if (b) {
    const uint32_t nseg = p.n_shared + p.top_k;
    p.x += static_cast<size_t>(b) * p.x_stride;
    p.scores += static_cast<size_t>(b) * p.n_experts;
    p.ids += static_cast<size_t>(b) * p.top_k;
    p.weights += static_cast<size_t>(b) * p.top_k;
    p.counter += b;
    if (p.seg_gu) {
      p.seg_gu += static_cast<size_t>(b) * nseg;
      p.seg_dn += static_cast<size_t>(b) * nseg;
    }
  }
  return p;
}

__global__ void __launch_bounds__(kRouteThreads) moe_route_kernel(const RouteParams p0) {
  const RouteParams p = route_seq(p0);
  extern __shared__ __align__(16) float rsm[];
  __shared__ float red[kRouteThreads / 32];
  __shared__ uint32_t s_last;
  pdl_launch_dependents();
  const uint32_t tid = threadIdx.x;
  const uint32_t e0 = blockIdx.x * p.experts_per_cta;
  const uint32_t e1 = min(e0 + p.experts_per_cta, p.n_experts);
  const uint32_t ne = e1 > e0 ? e1 - e0 : 0;
  float *xs = rsm;                       // [dim]
  float *ws = rsm + p.dim;               // [ne][dim + 4]: rows padded so that the ne
                                         // chain threads read distinct banks
  const uint32_t wstride = p.dim + kRouteRowPad;
  // the router rows do not depend on the previous kernel: stage them first,
  // one bulk copy per row into the padded layout
  __shared__ __align__(8) uint64_t rbar;
  const uint32_t rb = smem_addr(&rbar);
  if (tid == 0) {
    mbar_init(rb, 1);
    fence_barrier_init();
    if (ne) {
      mbar_arrive_expect_tx(rb, ne * p.dim * 4);
      for (uint32_t e = 0; e < ne; ++e)
        bulk_copy_g2s(smem_addr(ws + e * wstride), p.w + static_cast<size_t>(e0 + e) * p.dim, p.dim * 4, rb);
    } else {
      mbar_arrive(rb);
    }
  }
  pdl_wait();
  // the routed vector: x itself, or rmsnorm(x) * gain (the model's post-
  // attention residual) with the GEMV prologue's fixed-order reduction
  float inv = 1.0f;
  if (p.norm_w) {
    float ss = 0.f;
    for (uint32_t f = tid; f < p.dim / 4; f += kRouteThreads) {
      const float4 t = __ldcg(reinterpret_cast<const float4 *>(p.x) + f);
      ss = __fadd_rn(ss, __fadd_rn(__fadd_rn(__fmul_rn(t.x, t.x), __fmul_rn(t.y, t.y)),
                                   __fadd_rn(__fmul_rn(t.z, t.z), __fmul_rn(t.w, t.w))));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kRouteThreads / 32; ++w) tot = __fadd_rn(tot, red[w]);
    inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(p.dim)), p.eps)));
  }
  for (uint32_t i = tid; i < p.dim; i += kRouteThreads) {
    const float v = __ldcg(p.x + i);
    xs[i] = p.norm_w ? __fmul_rn(__fmul_rn(v, inv), p.norm_w[i]) : v;
  }
  __syncthreads();
  // every thread has passed the barrier init above; a failed (timed-out)
  // copy leaves the scores undefined and sets the status word
  const bool rows_ok = mbar_wait(rb, 0, p.status);
  // moe.rs:168-186: dot += hidden[i] * row[i], i ascending, unfused
  if (tid < ne && rows_ok) {
    const float *row = ws + tid * wstride;
    float dot = 0.0f;
    // dim % 4 == 0; the products do not depend on the chain, so loads and
    // multiplies of later steps issue while the adds retire one by one
    for (uint32_t i = 0; i < p.dim; i += 4) {
      const float4 xv = *reinterpret_cast<const float4 *>(xs + i);
      const float4 wv = *reinterpret_cast<const float4 *>(row + i);
      const float p0 = __fmul_rn(xv.x, wv.x);
      const float p1 = __fmul_rn(xv.y, wv.y);
      const float p2 = __fmul_rn(xv.z, wv.z);
      const float p3 = __fmul_rn(xv.w, wv.w);
      dot = __fadd_rn(dot, p0);
      dot = __fadd_rn(dot, p1);
      dot = __fadd_rn(dot, p2);
      dot = __fadd_rn(dot, p3);
    }
    const uint32_t e = e0 + tid;
    float s;
    if (p.mode == 0) {
      s = p.bias ? __fadd_rn(dot, p.bias[e]) : dot;
    } else {
      s = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-dot)));
    }
    p.scores[e] = s;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = (atomicAdd(p.counter, 1u) == gridDim.x - 1) ? 1u : 0u;
  __syncthreads();
  if (!s_last || tid != 0) return;
  __threadfence();
  *p.counter = 0;   // ready for the next launch (stream-ordered)
  const uint32_t K = p.top_k;
  uint32_t idx[kMoeMaxTopK];
  float wt[kMoeMaxTopK];
  const bool sel_bias = p.bias && p.mode == 1;
  // moe.rs:200-232: slots seeded with experts 0..k-1; an expert replaces
  // the first smallest slot when its key is strictly greater
  for (uint32_t i = 0; i < K; ++i) {
    idx[i] = i;
    wt[i] = sel_bias ? __fadd_rn(__ldcg(p.scores + i), p.bias[i]) : __ldcg(p.scores + i);
  }
  uint32_t min_i = 0;
  float min_v = wt[0];
  for (uint32_t i = 1; i < K; ++i)
    if (wt[i] < min_v) { min_v = wt[i]; min_i = i; }
  for (uint32_t e = K; e < p.n_experts; ++e) {
    const float key = sel_bias ? __fadd_rn(__ldcg(p.scores + e), p.bias[e]) : __ldcg(p.scores + e);
    if (key > min_v) {
      idx[min_i] = e;
      wt[min_i] = key;
      min_v = wt[0];
      min_i = 0;
      for (uint32_t i = 1; i < K; ++i)
        if (wt[i] < min_v) { min_v = wt[i]; min_i = i; }
    }
  }
  // moe.rs:238-300: weights from the raw scores of the selected experts
  for (uint32_t i = 0; i < K; ++i) wt[i] = __ldcg(p.scores + idx[i]);
  float mx = wt[0];
  for (uint32_t i = 1; i < K; ++i)
    if (wt[i] > mx) mx = wt[i];
  bool uniform = !isfinite(mx);
  if (!uniform) {
    float sum = 0.0f;
    if (p.mode == 0) {
      for (uint32_t i = 0; i < K; ++i) {
        wt[i] = expf(__fsub_rn(wt[i], mx));
        sum = __fadd_rn(sum, wt[i]);
      }
    } else {
      for (uint32_t i = 0; i < K; ++i) sum = __fadd_rn(sum, wt[i]);
    }
    if (!isfinite(sum) || sum <= 0.0f) {
      uniform = true;
    } else {
      const float invs = __fdiv_rn(1.0f, sum);
      for (uint32_t i = 0; i < K; ++i) wt[i] = __fmul_rn(wt[i], invs);
      const float sc = route_scale(p.scale);
      if (sc != 1.0f)
        for (uint32_t i = 0; i < K; ++i) wt[i] = __fmul_rn(wt[i], sc);
    }
  }
  if (uniform) route_uniform(wt, K, p.scale);
  for (uint32_t i = 0; i < K; ++i) {
    p.ids[i] = idx[i];
    p.weights[i] = wt[i];
  }
  // dispatch tables: shared experts, then the selected ones in slot order
  if (p.seg_gu) {
    for (uint32_t s = 0; s < p.n_shared; ++s) {
      p.seg_gu[s] = p.sh_gu_base + s * p.gu_bytes;
      p.seg_dn[s] = p.sh_dn_base + s * p.dn_bytes;
    }
    for (uint32_t i = 0; i < K; ++i) {
      const bool mine = p.ep_per_rank == 0 || idx[i] / p.ep_per_rank == p.ep_rank;
      p.seg_gu[p.n_shared + i] = mine ? p.gu_base + idx[i] * p.gu_bytes : 0ull;
      p.seg_dn[p.n_shared + i] = mine ? p.dn_base + idx[i] * p.dn_bytes : 0ull;
    }
  }
}

// Words another GPU writes and this one polls (or the reverse) are accessed
// with relaxed system-scope operations.  A weak load (ld.global.cg) carries
// no guarantee that it ever observes a store from another GPU: it may keep
// returning a copy of the word cached on this GPU while the peer's store has
// reached the word's home.  The tags make every word self-validating, so no
// acquire / release ordering is needed beyond that.
__device__ __forceinline__ unsigned long long ld_peer_u64(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_peer_u64(unsigned long long *p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Limit of a combine's waits for other ranks (arrival words, slots).  Each
// rank's kernels are launched by its own host thread, so a peer can start an
// invocation seconds late for legitimate reasons (graph builds, allocations,
// a process still mapping its peers); 5 s covers that and still bounds a
// dead peer.  The first expiry aborts the exchange, so a failing model pays
// this once.
constexpr uint64_t kEpWaitLimitNs = 5000000000ull;

// An expired combine wait: the timeout bit, and (first one only) the wait
// in words 4..7 of the status block.
__device__ void wait_expired(uint32_t *status, uint32_t site, uint32_t ver, uint32_t tag, uint32_t which) {
  if (atomicCAS(&status[4], 0u, site) == 0u) {
    status[5] = ver;
    status[6] = tag;
    status[7] = which;
  }
  atomicOr(status, ZDEV_ERR_TIMEOUT);
}

__global__ void moe_combine_kernel(const CombineParams p0) {
  pdl_launch_dependents();
  pdl_wait();
  // this token (grid dimension y) of a batch
  const uint32_t tb = blockIdx.y;
  CombineParams p = p0;
  p.exp_out += static_cast<size_t>(tb) * (p.n_shared + p.top_k) * p.dim;
  p.weights += static_cast<size_t>(tb) * p.top_k;
  if (p.mlp_out) p.mlp_out += static_cast<size_t>(tb) * p.dim;
  if (p.hidden) p.hidden += static_cast<size_t>(tb) * p.dim;
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= p.dim) return;
  float o = 0.0f;
  uint32_t s = 0;
  if (p.n_shared) {
    o = __ldcg(p.exp_out + i);
    for (s = 1; s < p.n_shared; ++s) o = __fadd_rn(o, __ldcg(p.exp_out + static_cast<size_t>(s) * p.dim + i));
  }
  const uint32_t ver = p.xslots ? __ldcg(p.ep_seq) + 1 : 0u;
  bool gave_up = false;   // after one expired wait the others are not waited for
  unsigned long long *abort_w = p.xslots ? p.xslots + ep_abort_word(p.slot_cap, p.dim) : nullptr;
  if (p.xslots) {
    // flow control: every rank has published this invocation (and so has
    // finished its combine of the previous one).  A rank may already have
    // published the next invocation (its arrival word then reads ver + 1),
    // so the test is "at least ver".
    const unsigned long long *arrive = p.xslots + ep_slot_words(p.slot_cap, p.dim);
    if (ld_peer_u64(abort_w) != 0ull) {
      wait_expired(p.status, ZDEV_WAIT_EP_ABORTED, ver, 0u, 0u);
      gave_up = true;
    }
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t r = 0; r < p.world && !gave_up; ++r) {
      uint32_t tag;
      while ((tag = static_cast<uint32_t>(ld_peer_u64(arrive + r) >> 32)) < ver) {
        if (globaltimer_ns() - t0 > kEpWaitLimitNs) {
          wait_expired(p.status, ZDEV_WAIT_EP_ARRIVAL, ver, tag, r);
          st_peer_u64(abort_w, 1ull);
          gave_up = true;
          break;
        }
      }
    }
  }
  for (uint32_t k = 0; k < p.top_k; ++k) {
    const float w = __ldcg(p.weights + k);
    float y;
    if (p.xslots) {
      // the slot's output from whichever rank ran its expert (bounded wait)
      const unsigned long long *src =
          p.xslots + (static_cast<size_t>(ver & 1u) * p.slot_cap + tb * p.top_k + k) * p.dim + i;
      unsigned long long t = ld_peer_u64(src);
      if (gave_up) {
        t = static_cast<unsigned long long>(0x7fc00000u);
      } else if (static_cast<uint32_t>(t >> 32) != ver) {
        const uint64_t t0 = globaltimer_ns();
        while (static_cast<uint32_t>(t >> 32) != ver) {
          if (globaltimer_ns() - t0 > kEpWaitLimitNs) {
            wait_expired(p.status, ZDEV_WAIT_EP_SLOT, ver, static_cast<uint32_t>(t >> 32), tb * p.top_k + k);
            st_peer_u64(abort_w, 1ull);
            t = static_cast<unsigned long long>(0x7fc00000u);
            gave_up = true;
            break;
          }
          t = ld_peer_u64(src);
        }
      }
      y = __uint_as_float(static_cast<uint32_t>(t));
    } else {
      y = __ldcg(p.exp_out + static_cast<size_t>(p.n_shared + k) * p.dim + i);
    }
    o = __fadd_rn(o, __fmul_rn(w, y));
  }
  if (p.mlp_out) p.mlp_out[i] = o;
  if (p.hidden) p.hidden[i] = __fadd_rn(p.hidden[i], o);
}

// grid (ceil(dim / 256), top_k, tokens): slot k's row of token z, when this
// rank ran its expert
__global__ void moe_ep_publish_kernel(const EpPublishParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const uint32_t k = blockIdx.y, tb = blockIdx.z, i = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t ver = __ldcg(p.ep_seq) + 1;
  if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && threadIdx.x == 0) {
    // this rank's arrival for invocation ver, in every rank's buffer
    const size_t a = ep_slot_words(p.slot_cap, p.dim) + p.ep_rank;
    for (uint32_t d = 0; d < p.world; ++d) st_peer_u64(p.dst[d] + a, tag_word(0.0f, ver));
  }
  if (i >= p.dim) return;
  const uint32_t e = __ldcg(p.ids + static_cast<size_t>(tb) * p.top_k + k);
  if (e / p.ep_per_rank != p.ep_rank) return;
  const float *eo = p.exp_out + static_cast<size_t>(tb) * (p.n_shared + p.top_k) * p.dim;
  const unsigned long long w = tag_word(__ldcg(eo + static_cast<size_t>(p.n_shared + k) * p.dim + i), ver);
  const size_t off = (static_cast<size_t>(ver & 1u) * p.slot_cap + tb * p.top_k + k) * p.dim + i;
  for (uint32_t d = 0; d < p.world; ++d) st_peer_u64(p.dst[d] + off, w);
}

__global__ void moe_ep_advance_kernel(uint32_t *ep_seq) {
  pdl_launch_dependents();
  pdl_wait();
  if (threadIdx.x == 0) *ep_seq += 1;
}

}  // namespace

uint32_t route_experts_per_cta(uint32_t dim) {
  uint32_t e = kRouteRowFloats / dim;
  return e < 1 ? 1 : (e > kRouteThreads ? kRouteThreads : e);
}

size_t route_smem_bytes(uint32_t dim) {
  const size_t e = route_experts_per_cta(dim);
  return (dim + e * (dim + kRouteRowPad)) * sizeof(float);
}

__global__ void __launch_bounds__(256) moe_dispatch_kernel(const MoeDispatchParams p) {
  __shared__ uint32_t cnt[kMoeMaxSegs];
  pdl_launch_dependents();
  pdl_wait();   // the router's selections
  const uint32_t n_segs = p.n_local + p.n_shared, n_slot = p.n_shared + p.top_k;
  for (uint32_t s = threadIdx.x; s < n_segs; s += blockDim.x) cnt[s] = s < p.n_local ? 0u : p.n_seq;
  __syncthreads();
  auto put = [&](uint32_t s, uint32_t j, uint32_t b, uint32_t slot) {
    const uint32_t pr = b * n_slot + slot, i = s * 32 + j;
    p.x_rows_gu[i] = b;
    p.x_rows_dn[i] = pr;
    p.out_gu[i] = p.act + static_cast<uint64_t>(pr) * p.act_row;
    p.out_dn[i] = p.exp_out + static_cast<uint64_t>(pr) * p.dim;
  };
  for (uint32_t t = threadIdx.x; t < p.n_seq * p.top_k; t += blockDim.x) {
    const uint32_t b = t / p.top_k, k = t % p.top_k, e = __ldcg(p.ids + t);
    uint32_t s = e;
    if (p.ep_per_rank) {
      if (e / p.ep_per_rank != p.ep_rank) continue;   // another rank's expert
      s = e - p.ep_rank * p.ep_per_rank;
    }
    if (s >= p.n_local) continue;
    put(s, atomicAdd(&cnt[s], 1u), b, p.n_shared + k);
  }
  for (uint32_t t = threadIdx.x; t < p.n_seq * p.n_shared; t += blockDim.x)
    put(p.n_local + t % p.n_shared, t / p.n_shared, t / p.n_shared, t % p.n_shared);
  __syncthreads();
  // the pair list: segment s's pairs after those of segments < s (a serial
  // prefix over at most kMoeMaxSegs counts, by thread 0)
  __shared__ uint32_t base[kMoeMaxSegs];
  if (threadIdx.x == 0) {
    uint32_t acc = 0;
    for (uint32_t s = 0; s < n_segs; ++s) {
      base[s] = acc;
      acc += cnt[s];
    }
    *p.n_pairs = acc;
  }
  __syncthreads();
  for (uint32_t s = threadIdx.x; s < n_segs; s += blockDim.x)
    for (uint32_t j = 0; j < cnt[s]; ++j) p.pairs[base[s] + j] = s << 8 | j;
  for (uint32_t s = threadIdx.x; s < n_segs; s += blockDim.x) {
    const uint32_t n = cnt[s];
    p.n_vec[s] = n;
    const bool sh = s >= p.n_local;
    const uint64_t o = sh ? s - p.n_local : s;
    p.tab_gu[s] = n ? reinterpret_cast<unsigned long long>((sh ? p.sh_tiles_gu : p.tiles_gu) + o * p.tiles_gu_stride) : 0ull;
    p.tab_dn[s] = n ? reinterpret_cast<unsigned long long>((sh ? p.sh_tiles_dn : p.tiles_dn) + o * p.tiles_dn_stride) : 0ull;
  }
}

cudaError_t moe_setup() {
  const size_t max_smem = route_smem_bytes(kMoeMaxDim);
  return cudaFuncSetAttribute(moe_route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(max_smem));
}

cudaError_t launch_moe_route(const RouteParams &rp, const LaunchCfg &lc) {
  if (rp.dim == 0 || rp.dim % 4 || rp.dim > kMoeMaxDim || rp.top_k == 0 ||
      rp.top_k > rp.n_experts || rp.top_k > kMoeMaxTopK)
    return cudaErrorInvalidValue;
  RouteParams p = rp;
  p.experts_per_cta = route_experts_per_cta(p.dim);
  const uint32_t grid = (p.n_experts + p.experts_per_cta - 1) / p.experts_per_cta;
  cudaLaunchAttribute attr[1];
  const uint32_t ns = p.n_seq > 1 ? p.n_seq : 1;
  if (ns > 1 && p.x_stride < p.dim) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg =
      make_launch_cfg(dim3(grid, ns), dim3(kRouteThreads), route_smem_bytes(p.dim), lc, attr);
  if (lc.launch_counter) ++*lc.launch_counter;
  return cudaLaunchKernelEx(&cfg, moe_route_kernel, p);
}

cudaError_t launch_moe_dispatch(const MoeDispatchParams &p, const LaunchCfg &lc) {
  if (p.n_seq == 0 || p.n_seq > 32 || p.top_k == 0 || p.n_local + p.n_shared == 0 ||
      p.n_local + p.n_shared > kMoeMaxSegs)
    return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_launch_cfg(dim3(1), dim3(256), 0, lc, attr);
  if (lc.launch_counter) ++*lc.launch_counter;
  return cudaLaunchKernelEx(&cfg, moe_dispatch_kernel, p);
}

cudaError_t launch_moe_combine(const CombineParams &p, const LaunchCfg &lc) {
  const uint32_t ns = p.n_seq > 1 ? p.n_seq : 1;
  if (p.xslots && ns * p.top_k > p.slot_cap) return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_launch_cfg(dim3((p.dim + 255) / 256, ns), dim3(256), 0, lc, attr);
  if (lc.launch_counter) ++*lc.launch_counter;
  return cudaLaunchKernelEx(&cfg, moe_combine_kernel, p);
}

cudaError_t launch_moe_ep_publish(const EpPublishParams &p, const LaunchCfg &lc) {
  const uint32_t ns = p.n_seq > 1 ? p.n_seq : 1;
  if (p.dim == 0 || p.top_k == 0 || p.world == 0 || p.world > kEpMaxRanks || p.ep_per_rank == 0 ||
      ns * p.top_k > p.slot_cap)
    return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_launch_cfg(dim3((p.dim + 255) / 256, p.top_k, ns), dim3(256), 0, lc, attr);
  if (lc.launch_counter) ++*lc.launch_counter;
  return cudaLaunchKernelEx(&cfg, moe_ep_publish_kernel, p);
}

cudaError_t launch_moe_ep_advance(uint32_t *ep_seq, const LaunchCfg &lc) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_launch_cfg(dim3(1), dim3(32), 0, lc, attr);
  if (lc.launch_counter) ++*lc.launch_counter;
  return cudaLaunchKernelEx(&cfg, moe_ep_advance_kernel, ep_seq);
}

}  // namespace zgpu
