// K4: paged causal attention over block tables, for verify (T = k+1), decode (T = 1) and
// prefill (T = prompt length), with grouped-query heads.
//
// Replaces cache/kv.py:108-112 (gather: a copy of every cached position per layer per step)
// and the SDPA call at lm/forward.py:62-63: keys are read in place from the paged pool
// [num_slots, Hkv, d] through block_table, never copied. The mask is the reference's
// (lm/forward.py:44-49): query at absolute position p sees key j iff j <= p and
// j < past + n_new; a padded query (p >= total) sees every existing key, so it never makes NaN.
//
// Three kernels by shape. bf16 with d = 64: decode / verify shapes (at most 16 query rows per
// KV head) run the cluster kernel (attn_cluster.cuh) or, past one cluster's keys, split-KV
// tensor-core items (attn_item_mma.cuh); prefill shapes run the tensor-core flash kernel
// (attn_prefill.cuh). fp32 models and other head dims: grid (splits, Hkv * qtiles, B); a CTA
// serves the G = Hq / Hkv query heads that share one KV head for up to 32 query rows, over
// one contiguous chunk of keys (flash-decoding style split-KV), stages 32-key blocks of K and
// V in shared memory (fp32), keeps an online softmax (max, sum) per row and accumulates P V.
// The last CTA of each (row, kv head, q tile), found with an atomic ticket, merges the partial
// results in split order, which keeps the output independent of CTA scheduling; there is no
// spin-wait.
#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <type_traits>

#include "attn_cluster.cuh"
#include "attn_core.cuh"
#include "attn_item_mma.cuh"
#include "attn_prefill.cuh"

namespace specb200 {
namespace {

template <typename T, int D>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(AttnKernelArgs ka) {
  __shared__ float smem[AttnSmem<D>::kFloats];
  pdl_launch_dependents();
  pdl_wait();
  attention_item<T, D>(ka, blockIdx.z, blockIdx.y / ka.p.qtiles, blockIdx.y % ka.p.qtiles, blockIdx.x, smem);
}

// Decode / verify shapes (bf16, d = 64, T x G <= 16): one tensor-core item per (split, kv
// head, sequence). The item itself waits on the previous kernel, after loading the cached keys.
__global__ void __launch_bounds__(kAttnThreads) attention_mma_kernel(AttnKernelArgs ka) {
  __shared__ __align__(128) uint8_t smem[kAmItemSmem];
  pdl_launch_dependents();
  attention_item_mma(ka, blockIdx.z, blockIdx.y, blockIdx.x, smem, true);
}

// Decode / verify shapes whose keys fit one cluster: one cluster of C CTAs per (kv head,
// sequence); loads the cached keys before waiting on the previous kernel.
__global__ void __launch_bounds__(kAcThreads) attention_cluster_kernel(AttnKernelArgs ka) {
  extern __shared__ __align__(16) uint8_t ac_smem[];
  pdl_launch_dependents();
  attention_cluster_cta(ka, blockIdx.z, blockIdx.y, ac_smem, true);
}

// Prefill shapes (bf16, d = 64, more than 16 query rows per KV head): 64 query rows per CTA on
// the tensor cores, keys streamed in 64-key blocks (attn_prefill.cuh).
__global__ void __launch_bounds__(kApThreads) attention_prefill_kernel(AttnArgs a) {
  __shared__ __align__(128) ApSmem sm;
  pdl_launch_dependents();
  pdl_wait();
  attention_prefill_cta(a, sm);
}

constexpr int kAcSmemLimit = 200 * 1024;

cudaError_t launch_cluster(const AttnArgs& a, const AttnPlan& p, cudaStream_t s, bool pdl) {
  AttnKernelArgs ka;
  ka.a = a;
  ka.p = p;
  ka.counters = nullptr;
  ka.part = nullptr;
  const int R = a.T * (a.Hq / a.Hkv);
  const AcLayout lay = ac_layout(p.chunk, R, p.splits_max, a.bs);
  if (lay.total > kAcSmemLimit) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.splits_max, a.Hkv, a.B);
  cfg.blockDim = dim3(kAcThreads);
  cfg.dynamicSmemBytes = lay.total;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.splits_max;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, attention_cluster_kernel, ka);
}

template <typename T, int D>
cudaError_t launch_d(const AttnArgs& a, const AttnPlan& p, int* counters, float* partials, cudaStream_t s, bool pdl) {
  AttnKernelArgs ka;
  ka.a = a;
  ka.p = p;
  ka.counters = counters;
  ka.part = partials;
  return launch_kernel(attention_kernel<T, D>, dim3(p.splits_max, a.Hkv * p.qtiles, a.B), dim3(kAttnThreads), 0, s, pdl,
                       ka);
}

}  // namespace

bool attention_prepare() {
  static std::once_flag once;
  static bool ok = false;
  std::call_once(once, [] {
    ok = cudaFuncSetAttribute(attention_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAcSmemLimit) ==
         cudaSuccess;
    // the largest carveout, as every kernel of a forward, so that consecutive kernels share SMs
    for (const void* f : {reinterpret_cast<const void*>(attention_cluster_kernel),
                          reinterpret_cast<const void*>(attention_mma_kernel),
                          reinterpret_cast<const void*>(attention_prefill_kernel),
                          reinterpret_cast<const void*>(attention_kernel<float, 16>),
                          reinterpret_cast<const void*>(attention_kernel<float, 32>),
                          reinterpret_cast<const void*>(attention_kernel<float, 64>),
                          reinterpret_cast<const void*>(attention_kernel<__nv_bfloat16, 16>),
                          reinterpret_cast<const void*>(attention_kernel<__nv_bfloat16, 32>),
                          reinterpret_cast<const void*>(attention_kernel<__nv_bfloat16, 64>)})
      ok = ok && cudaFuncSetAttribute(f, cudaFuncAttributePreferredSharedMemoryCarveout,
                                      cudaSharedmemCarveoutMaxShared) == cudaSuccess;
  });
  return ok;
}

// Few (sequence, KV head) pairs: the cluster kernel, whose CTAs load their keys before the wait
// and merge in distributed shared memory, while its clusters fit about two waves (2 CTAs per
// SM). Many pairs (large batches): the split-KV items, one or more CTAs per pair streaming
// 32-key blocks through a cp.async ring, since a wave of clusters loads, computes and merges
// without overlapping the next wave. Measured per 24-layer 1.7B verify at 644 keys, B = 64 x 32
// KV heads: clusters 16.5 ms, the 64-row prefill kernel 10.4 ms, the items 8.6 ms.
constexpr int kClusterCtaBudget = 4 * 148;

AttnPlan plan_attention(int B, int T, int Hq, int Hkv, int max_kv_len, bool tensor_items) {
  if (tensor_items && T * (Hq / Hkv) <= kAmRows && attention_prepare()) {
    AttnPlan p;
    const bool cluster =
        plan_attention_cluster(max_kv_len, &p) && ac_layout(p.chunk, T * (Hq / Hkv), p.splits_max, 1).total <= kAcSmemLimit;
    const long pairs = static_cast<long>(B) * Hkv;
    if (cluster && pairs * p.splits_max <= kClusterCtaBudget) return p;
    if (pairs >= 148) {
      AttnPlan q = plan_attention_mma(B, Hkv, max_kv_len);
      q.mma = 1;
      return q;
    }
    if (cluster) return p;
  }
  if (tensor_items && T * (Hq / Hkv) <= kAmRows) {
    AttnPlan p = plan_attention_mma(B, Hkv, max_kv_len);
    p.mma = 1;
    return p;
  }
  if (tensor_items) {  // prefill shapes
    AttnPlan p;
    p.qtiles = (T * (Hq / Hkv) + kApRows - 1) / kApRows;
    p.splits_max = 1;
    p.chunk = 0;
    p.mma = 3;
    return p;
  }
  AttnPlan p;
  const int G = Hq / Hkv;
  p.qtiles = (T * G + kRows - 1) / kRows;
  const int groups = B * Hkv * p.qtiles;
  int splits = std::max(1, (2 * 148 + groups - 1) / groups);
  if (groups > kAttnMaxCounters) splits = 1;
  const int max_len = std::max(1, max_kv_len);
  splits = std::min(splits, (max_len + kKeys - 1) / kKeys);
  p.chunk = (((max_len + splits - 1) / splits) + kKeys - 1) / kKeys * kKeys;
  p.splits_max = (max_len + p.chunk - 1) / p.chunk;
  return p;
}

size_t attention_partials_bytes(const AttnPlan& p, int B, int Hkv, int D) {
  if (p.mma >= 2) return 0;  // the cluster kernel merges in distributed shared memory; prefill does not split
  const size_t groups = static_cast<size_t>(B) * Hkv * p.qtiles;
  return p.splits_max > 1 ? groups * p.splits_max * kRows * (D + 2) * sizeof(float) : 0;
}

size_t attention_workspace_bytes(const AttnPlan& p, int B, int Hkv, int D) {
  return kAttnCounterBytes + attention_partials_bytes(p, B, Hkv, D);
}

template <typename T>
int launch_attention(const AttnArgs& a, const AttnPlan& p, int* counters, float* partials, cudaStream_t s, bool pdl) {
  cudaError_t e;
  if (p.mma == 2) {
    if (!std::is_same<T, __nv_bfloat16>::value || a.D != 64 || a.T * (a.Hq / a.Hkv) > kAcRowsMax)
      return SPECB200_ERR_UNSUPPORTED;
    e = launch_cluster(a, p, s, pdl);
    return e == cudaSuccess ? SPECB200_OK : SPECB200_ERR_CUDA;
  }
  if (p.mma == 3) {
    if (!std::is_same<T, __nv_bfloat16>::value || a.D != 64) return SPECB200_ERR_UNSUPPORTED;
    if (a.Hkv > 65535 || a.B > 65535) return SPECB200_ERR_ARG;
    e = launch_kernel(attention_prefill_kernel, dim3(p.qtiles, a.Hkv, a.B), dim3(kApThreads), 0, s, pdl, a);
    return e == cudaSuccess ? SPECB200_OK : SPECB200_ERR_CUDA;
  }
  if (p.mma) {
    if (!std::is_same<T, __nv_bfloat16>::value || a.D != 64 || a.T * (a.Hq / a.Hkv) > kAmRows)
      return SPECB200_ERR_UNSUPPORTED;
    AttnKernelArgs ka;
    ka.a = a;
    ka.p = p;
    ka.counters = counters;
    ka.part = partials;
    e = launch_kernel(attention_mma_kernel, dim3(p.splits_max, a.Hkv, a.B), dim3(kAttnThreads), 0, s, pdl, ka);
    return e == cudaSuccess ? SPECB200_OK : SPECB200_ERR_CUDA;
  }
  switch (a.D) {
    case 16: e = launch_d<T, 16>(a, p, counters, partials, s, pdl); break;
    case 32: e = launch_d<T, 32>(a, p, counters, partials, s, pdl); break;
    case 64: e = launch_d<T, 64>(a, p, counters, partials, s, pdl); break;
    default: return SPECB200_ERR_UNSUPPORTED;
  }
  return e == cudaSuccess ? SPECB200_OK : SPECB200_ERR_CUDA;
}
template int launch_attention<float>(const AttnArgs&, const AttnPlan&, int*, float*, cudaStream_t, bool);
template int launch_attention<__nv_bfloat16>(const AttnArgs&, const AttnPlan&, int*, float*, cudaStream_t, bool);

}  // namespace specb200

using namespace specb200;
extern "C" int specb200_set_error(int code, const char* msg);

extern "C" size_t specb200_attention_workspace_bytes(int B, int T, int n_heads, int n_kv_heads, int head_dim,
                                                     int max_kv_len) {
  if (B <= 0 || T <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads) return 0;
  // the tensor-core items apply to bf16 with d = 64; the workspace covers either plan
  const AttnPlan a = plan_attention(B, T, n_heads, n_kv_heads, max_kv_len, false);
  const AttnPlan b = plan_attention(B, T, n_heads, n_kv_heads, max_kv_len, head_dim == 64);
  return std::max(attention_workspace_bytes(a, B, n_kv_heads, head_dim), attention_workspace_bytes(b, B, n_kv_heads, head_dim));
}

extern "C" int specb200_attention(int dtype, const void* q, const void* k_pool, const void* v_pool,
                                  const int32_t* block_table, int table_stride, int block_size, const int32_t* past_len,
                                  const int32_t* n_new, int B, int T, int n_heads, int n_kv_heads, int head_dim,
                                  int max_kv_len, float scale, void* out, void* workspace, size_t workspace_bytes,
                                  int32_t* status, void* stream) {
  if (B <= 0 || T <= 0 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || block_size <= 0 || max_kv_len <= 0)
    return specb200_set_error(SPECB200_ERR_ARG, "attention: bad sizes");
  if (head_dim != 16 && head_dim != 32 && head_dim != 64)
    return specb200_set_error(SPECB200_ERR_UNSUPPORTED, "attention: head_dim must be 16, 32 or 64");
  if (!q || !k_pool || !v_pool || !block_table || !past_len || !n_new || !out || !workspace)
    return specb200_set_error(SPECB200_ERR_ARG, "attention: null pointer");
  AttnPlan p = plan_attention(B, T, n_heads, n_kv_heads, max_kv_len, dtype == SPECB200_BF16 && head_dim == 64);
  if (workspace_bytes < attention_workspace_bytes(p, B, n_kv_heads, head_dim))
    return specb200_set_error(SPECB200_ERR_WORKSPACE, "attention: workspace too small");
  AttnArgs a;
  a.q = q;
  a.k_pool = k_pool;
  a.v_pool = v_pool;
  a.table = block_table;
  a.table_stride = table_stride;
  a.bs = block_size;
  a.past = past_len;
  a.n_new = n_new;
  a.B = B;
  a.T = T;
  a.Hq = n_heads;
  a.Hkv = n_kv_heads;
  a.D = head_dim;
  a.scale = scale;
  a.out = out;
  a.status = status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (status) cudaMemsetAsync(status, 0, sizeof(int32_t), s);
  int* counters = static_cast<int*>(workspace);
  float* partials = reinterpret_cast<float*>(static_cast<char*>(workspace) + kAttnCounterBytes);
  int rc = dtype == SPECB200_BF16 ? launch_attention<__nv_bfloat16>(a, p, counters, partials, s, false)
                                  : launch_attention<float>(a, p, counters, partials, s, false);
  if (rc != SPECB200_OK) return specb200_set_error(rc, cudaGetErrorString(cudaGetLastError()));
  return SPECB200_OK;
}
