// K4: paged causal attention over block tables, for verify (T = k+1), decode (T = 1) and
// prefill (T = prompt length), with grouped-query heads.
//
// Replaces cache/kv.py:108-112 (gather: a copy of every cached position per layer per step)
// and the SDPA call at lm/forward.py:62-63: keys are read in place from the paged pool
// [num_slots, Hkv, d] through block_table, never copied. The mask is the reference's
// (lm/forward.py:44-49): query at absolute position p sees key j iff j <= p and
// j < past + n_new; a padded query (p >= total) sees every existing key, so it never makes NaN.
//
// Grid (splits, Hkv * qtiles, B). A CTA serves the G = Hq / Hkv query heads that share one
// KV head for up to 32 query rows, over one contiguous chunk of keys: flash-decoding style
// split-KV so that a batch-1 verify still puts ~300 CTAs on 148 SMs. Each CTA stages 32-key
// blocks of K and V in shared memory (fp32), keeps an online softmax (max, sum) per row and
// accumulates P V. The last CTA of each (row, kv head, q tile), found with an atomic ticket,
// merges the partial results in split order, which keeps the output independent of CTA
// scheduling; there is no spin-wait.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace specb200 {
namespace {

constexpr int kAttnThreads = 128;
constexpr int kRows = 32;  // query rows per CTA
constexpr int kKeys = 32;  // keys per shared-memory block

// Convert one 16-byte chunk of a K/V row to fp32 in shared memory.
template <typename T>
SPECB200_DEVINL void load_chunk16(const T* src, float* dst);
template <>
SPECB200_DEVINL void load_chunk16<float>(const float* src, float* dst) {
  const float4 v = *reinterpret_cast<const float4*>(src);
  dst[0] = v.x; dst[1] = v.y; dst[2] = v.z; dst[3] = v.w;
}
template <>
SPECB200_DEVINL void load_chunk16<__nv_bfloat16>(const __nv_bfloat16* src, float* dst) {
  const uint4 v = *reinterpret_cast<const uint4*>(src);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(h[j]);
    dst[2 * j] = f.x;
    dst[2 * j + 1] = f.y;
  }
}

struct AttnKernelArgs {
  AttnArgs a;
  AttnPlan p;
  float* part;     // [B, Hkv, qtiles, splits_max, kRows, D + 2]
  int* counters;   // [B, Hkv, qtiles]
};

template <typename T, int D>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(AttnKernelArgs ka) {
  pdl_launch_dependents();
  pdl_wait();
  const AttnArgs& a = ka.a;
  const int b = blockIdx.z;
  const int g = blockIdx.y / ka.p.qtiles, qt = blockIdx.y % ka.p.qtiles;
  const int split = blockIdx.x;
  const int G = a.Hq / a.Hkv;
  const int past = a.past[b], nn = a.n_new[b], total = past + nn;
  const int r0 = qt * kRows;
  const int R = min(kRows, a.T * G - r0);
  if (R <= 0 || nn <= 0) return;
  const int t_max = (r0 + R - 1) / G;
  const int kmax = min(total, past + t_max + 1);
  const int nsplit = min(ka.p.splits_max, (kmax + ka.p.chunk - 1) / ka.p.chunk);
  if (split >= nsplit) return;
  const int kbeg = split * ka.p.chunk;
  const int kend = (split == nsplit - 1) ? kmax : min(kmax, kbeg + ka.p.chunk);

  __shared__ float qs[kRows][D + 1];
  __shared__ float ks[kKeys][D + 1];
  __shared__ float vs[kKeys][D];
  __shared__ float sc[kRows][kKeys + 1];
  __shared__ float os[kRows][D];
  __shared__ float m_s[kRows], l_s[kRows], alpha_s[kRows];
  __shared__ int lim_s[kRows];
  __shared__ int slot_s[kKeys];
  __shared__ int sh_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const T* q = static_cast<const T*>(a.q);
  for (int r = warp; r < R; r += kAttnThreads / 32) {
    const int rr = r0 + r, t = rr / G, h = g * G + rr % G;
    const T* src = q + (static_cast<int64_t>(b * a.T + t) * a.Hq + h) * D;
    for (int c = lane; c < D; c += 32) qs[r][c] = to_f32<T>(src[c]);
  }
  for (int i = tid; i < kRows * D; i += kAttnThreads) os[i / D][i % D] = 0.f;
  if (tid < kRows) {
    m_s[tid] = -INFINITY;
    l_s[tid] = 0.f;
    const int t = (r0 + tid) / G;
    lim_s[tid] = min(past + t + 1, total);
  }
  __syncthreads();

  const T* kp = static_cast<const T*>(a.k_pool);
  const T* vp = static_cast<const T*>(a.v_pool);
  const int32_t* table = a.table + static_cast<int64_t>(b) * a.table_stride;
  for (int kb = kbeg; kb < kend; kb += kKeys) {
    const int nk = min(kKeys, kend - kb);
    if (tid < kKeys) {
      const int j = kb + tid;
      slot_s[tid] = tid < nk ? table[j / a.bs] * a.bs + j % a.bs : 0;
    }
    __syncthreads();
    // K and V rows, one 16-byte chunk per thread per step; rows past nk are zero (masked below)
    constexpr int kEl = 16 / sizeof(T);
    constexpr int kCpr = D / kEl;
    for (int i = tid; i < 2 * kKeys * kCpr; i += kAttnThreads) {
      const int row = i / kCpr, c = (i % kCpr) * kEl;
      const int j = row % kKeys;
      const bool isv = row >= kKeys;
      float* dst = (isv ? vs[j] : ks[j]) + c;
      if (j < nk) {
        load_chunk16<T>((isv ? vp : kp) + (static_cast<int64_t>(slot_s[j]) * a.Hkv + g) * D + c, dst);
      } else {
#pragma unroll
        for (int e = 0; e < kEl; ++e) dst[e] = 0.f;
      }
    }
    __syncthreads();
    for (int i = tid; i < R * kKeys; i += kAttnThreads) {
      const int r = i / kKeys, j = i % kKeys;
      float s = -INFINITY;
      if (j < nk && kb + j < lim_s[r]) {
        float acc = 0.f;
#pragma unroll 16
        for (int c = 0; c < D; ++c) acc = fmaf(qs[r][c], ks[j][c], acc);
        s = acc * a.scale;
      }
      sc[r][j] = s;
    }
    __syncthreads();
    for (int r = warp; r < R; r += kAttnThreads / 32) {
      const float s = sc[r][lane];
      const float mx = warp_max(s);
      const float m_old = m_s[r];
      const float m_new = fmaxf(m_old, mx);
      float p = 0.f, alpha = 1.f;
      if (m_new != -INFINITY) {
        p = expf(s - m_new);
        alpha = expf(m_old - m_new);
      }
      const float sum = warp_sum(p);
      sc[r][lane] = p;
      if (lane == 0) {
        l_s[r] = l_s[r] * alpha + sum;
        m_s[r] = m_new;
        alpha_s[r] = alpha;
      }
    }
    __syncthreads();
    for (int i = tid; i < R * D; i += kAttnThreads) {
      const int r = i / D, c = i % D;
      float acc = os[r][c] * alpha_s[r];
#pragma unroll 8
      for (int j = 0; j < kKeys; ++j) acc = fmaf(sc[r][j], vs[j][c], acc);
      os[r][c] = acc;
    }
    __syncthreads();
  }

  T* out = static_cast<T*>(a.out);
  auto write_out = [&](int r, int c, float v) {
    const int rr = r0 + r, t = rr / G, h = g * G + rr % G;
    out[(static_cast<int64_t>(b * a.T + t) * a.Hq + h) * D + c] = from_f32<T>(v);
  };
  if (nsplit == 1) {
    for (int i = tid; i < R * D; i += kAttnThreads) {
      const int r = i / D, c = i % D;
      write_out(r, c, os[r][c] / l_s[r]);
    }
    return;
  }
  const int group = (b * a.Hkv + g) * ka.p.qtiles + qt;
  const size_t part_elems = static_cast<size_t>(kRows) * (D + 2);
  float* mine = ka.part + (static_cast<size_t>(group) * ka.p.splits_max + split) * part_elems;
  for (int i = tid; i < R * D; i += kAttnThreads) mine[i] = os[i / D][i % D];
  if (tid < R) {
    mine[kRows * D + tid] = m_s[tid];
    mine[kRows * D + kRows + tid] = l_s[tid];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) sh_last = (atomicAdd(ka.counters + group, 1) == nsplit - 1);
  __syncthreads();
  if (!sh_last) return;
  __threadfence();
  const float* base = ka.part + static_cast<size_t>(group) * ka.p.splits_max * part_elems;
  for (int i = tid; i < R * D; i += kAttnThreads) {
    const int r = i / D, c = i % D;
    float M = -INFINITY;
    for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, __ldcg(base + sp * part_elems + kRows * D + r));
    float L = 0.f, O = 0.f;
    for (int sp = 0; sp < nsplit; ++sp) {
      const float* ps = base + sp * part_elems;
      const float ms = __ldcg(ps + kRows * D + r);
      const float w = (ms == -INFINITY) ? 0.f : expf(ms - M);
      L = fmaf(__ldcg(ps + kRows * D + kRows + r), w, L);
      O = fmaf(__ldcg(ps + r * D + c), w, O);
    }
    write_out(r, c, O / L);
  }
  if (tid == 0) ka.counters[group] = 0;
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

AttnPlan plan_attention(int B, int T, int Hq, int Hkv, int max_kv_len) {
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
  const size_t groups = static_cast<size_t>(B) * Hkv * p.qtiles;
  return p.splits_max > 1 ? groups * p.splits_max * kRows * (D + 2) * sizeof(float) : 0;
}

size_t attention_workspace_bytes(const AttnPlan& p, int B, int Hkv, int D) {
  return kAttnCounterBytes + attention_partials_bytes(p, B, Hkv, D);
}

template <typename T>
int launch_attention(const AttnArgs& a, const AttnPlan& p, int* counters, float* partials, cudaStream_t s, bool pdl) {
  cudaError_t e;
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
  return attention_workspace_bytes(plan_attention(B, T, n_heads, n_kv_heads, max_kv_len), B, n_kv_heads, head_dim);
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
  AttnPlan p = plan_attention(B, T, n_heads, n_kv_heads, max_kv_len);
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
