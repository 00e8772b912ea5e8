// Decode-step linear layers on CUDA cores.
//
// The Llama linears of lm/forward.py:21-84 (q/k/v, o, gate/up, down and the LM head: nn.Linear,
// y = x W^T in the model dtype with fp32 accumulation) for calls of at most four token rows,
// i.e. the draft model's decode steps. At one token each weight row is used once, so the
// product is one dot product per row and tensor cores add only issue latency; what bounds a
// decode step of a small model is the chain of dependent launches. This kernel shortens each
// link of that chain:
// - a CTA's weight rows reach shared memory by one or two bulk copies issued BEFORE
//   griddepcontrol.wait (weights never depend on the previous kernel), so under programmatic
//   dependent launch they stream in while the previous kernels still run;
// - the RMSNorm in front of q/k/v, gate/up and the LM head is recomputed by every CTA from the
//   residual stream (LlamaRMSNorm, transformers modeling_llama.py:62-67, with the rounding of
//   norm.cu), which removes a launch and a round trip per norm;
// - each CTA owns whole output features (no split-K), so the fused epilogue follows the dot
//   products directly.
// Epilogues and rounding match epilogue.cuh: EPI_QKV (RoPE, q out, k/v into the paged pool),
// EPI_RESID (residual add), EPI_SILU_MUL (gate/up rows in 64-row groups), EPI_STORE.
#include <algorithm>
#include <mutex>

#include "epilogue.cuh"
#include "gemv.cuh"
#include "kernels.cuh"

namespace specb200 {
namespace {

constexpr int kGvThreads = 256;
constexpr int kGvWarps = kGvThreads / 32;
constexpr int kGvXChunks = 4;                          // 16-byte input chunks per thread
constexpr int kGvMaxK = kGvThreads * 8 * kGvXChunks;   // 8192
constexpr uint32_t kGvChunkBudget = 32 * 1024;         // weight bytes per chunk
constexpr size_t kGvSmemBudget = 200 * 1024;           // ring + staged inputs + partials
constexpr int kGvSms = 148;
static_assert(2 * kGvSms <= kGemvTraceCtas, "trace rows must cover the largest grid");

SPECB200_DEVINL void gv_bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

SPECB200_DEVINL unsigned long long gv_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

SPECB200_DEVINL void unpack8(const uint4& v, float (&f)[8]) {
  const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(u[i] << 16);
    f[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
  }
}

SPECB200_DEVINL uint32_t pack2(float lo, float hi) {
  const uint32_t l = __bfloat16_as_ushort(__float2bfloat16_rn(lo));
  const uint32_t h = __bfloat16_as_ushort(__float2bfloat16_rn(hi));
  return l | (h << 16);
}

struct Chunk {
  int f0;    // first output feature
  int nf;    // features in this chunk
  int row0;  // first weight row of segment 0
  int row1;  // first weight row of segment 1 (two-segment chunks)
};

SPECB200_DEVINL Chunk chunk_at(const GemvPlan& p, int c) {
  Chunk k;
  k.f0 = c * p.f;
  k.nf = min(p.f, p.features - k.f0);
  if (p.segs == 1) {
    k.row0 = k.f0;
    k.row1 = 0;
  } else {
    const int g = k.f0 / p.group, j0 = k.f0 - g * p.group;
    k.row0 = g * p.group_rows + j0;
    k.row1 = k.row0 + p.seg1_off;
  }
  return k;
}

// Bulk copies of chunk c into one ring stage: segment 0 rows first, then segment 1 rows.
SPECB200_DEVINL void issue_chunk(const GemvArgs& a, int c, uint8_t* stage, uint64_t* bar, uint64_t pol) {
  const Chunk k = chunk_at(a.p, c);
  const uint32_t seg = static_cast<uint32_t>(k.nf) * static_cast<uint32_t>(a.K) * 2u;
  mbar_arrive_expect_tx(bar, seg * static_cast<uint32_t>(a.p.segs));
  gv_bulk_load(stage, a.w + static_cast<int64_t>(k.row0) * a.K, seg, bar, pol);
  if (a.p.segs == 2) gv_bulk_load(stage + seg, a.w + static_cast<int64_t>(k.row1) * a.K, seg, bar, pol);
}

// Input rows into shared memory as bf16 [MR][K] (rows >= M zero), RMS-normalised when a norm
// weight is given: y = round(w * round(x * rsqrt(mean(x^2) + eps))), as rmsnorm_kernel.
template <int MR, typename Sync>
SPECB200_DEVINL void stage_x(const GemvArgs& a, const uint4 (&nw)[kGvXChunks], __nv_bfloat16* xs, float (*red)[MR],
                             Sync sync) {
  const int K = a.K, nch = K >> 3, tid = threadIdx.x;
  const bool norm = a.norm_w != nullptr;
  uint4 xv[kGvXChunks][MR];
  float ss[MR];
#pragma unroll
  for (int m = 0; m < MR; ++m) ss[m] = 0.f;
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    int64_t src = m;
    if (a.sel_n_new && m < a.M) src = static_cast<int64_t>(m) * a.T_tokens + max(__ldcg(a.sel_n_new + m) - 1, 0);
    const uint4* row = reinterpret_cast<const uint4*>(a.x + src * K);
#pragma unroll
    for (int i = 0; i < kGvXChunks; ++i) {
      const int ch = tid + i * kGvThreads;
      xv[i][m] = (ch < nch && m < a.M) ? __ldcg(row + ch) : make_uint4(0, 0, 0, 0);
    }
  }
  if (norm) {
#pragma unroll
    for (int i = 0; i < kGvXChunks; ++i)
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        float f[8];
        unpack8(xv[i][m], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss[m] = fmaf(f[e], f[e], ss[m]);
      }
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      ss[m] = warp_sum(ss[m]);
      if ((tid & 31) == 0) red[tid >> 5][m] = ss[m];
    }
    sync();
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < kGvWarps; ++w) t += red[w][m];
      ss[m] = 1.0f / sqrtf(t / static_cast<float>(K) + a.eps);
    }
  }
#pragma unroll
  for (int i = 0; i < kGvXChunks; ++i) {
    const int ch = tid + i * kGvThreads;
    if (ch >= nch) break;
    float wf[8];
    if (norm) unpack8(nw[i], wf);
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      uint4 v = xv[i][m];
      if (norm && m < a.M) {
        float f[8];
        unpack8(v, f);
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = wf[e] * round_to<__nv_bfloat16>(f[e] * ss[m]);
        v = make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
      }
      reinterpret_cast<uint4*>(xs + m * K)[ch] = v;
    }
  }
}

// Dot products of one chunk; lane sums land in part[row][slice][m]. With at least 8 rows
// (ksplit == 1) each warp takes rows warp, warp + 8, ... up to four at a time, so the FMA chains
// of different rows and the two halves of each 16-byte chunk are independent and every input
// chunk is read from shared memory once for all of them; the warp reductions of those rows
// run interleaved. With fewer rows each warp takes one (row, K-slice) item.
template <int MR>
SPECB200_DEVINL void dot_chunk(const GemvPlan& p, int K, int nf, const uint8_t* stage, const __nv_bfloat16* xs,
                               float* part) {
  constexpr int RB = 4;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ks = p.ksplit, rows = p.segs * nf, nch = K >> 3;
  const uint32_t rb = static_cast<uint32_t>(K) * 2u;
  const uint4* x4 = reinterpret_cast<const uint4*>(xs);
  const int xstride = K >> 3;  // uint4 per input row
  if (ks > 1) {
    if (warp >= rows * ks) return;
    const int r = warp / ks, kq = warp - r * ks;
    const uint4* wr = reinterpret_cast<const uint4*>(stage + r * rb);
    float acc[MR][2];
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[m][0] = acc[m][1] = 0.f;
    for (int ch = kq * 32 + lane; ch < nch; ch += 32 * ks) {
      float wf[8];
      unpack8(wr[ch], wf);
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        float xf[8];
        unpack8(x4[m * xstride + ch], xf);
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          acc[m][0] = fmaf(wf[e], xf[e], acc[m][0]);
          acc[m][1] = fmaf(wf[e + 1], xf[e + 1], acc[m][1]);
        }
      }
    }
    float v[MR];
#pragma unroll
    for (int m = 0; m < MR; ++m) v[m] = acc[m][0] + acc[m][1];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int m = 0; m < MR; ++m) v[m] += __shfl_xor_sync(0xffffffffu, v[m], o);
    if (lane == 0) {
#pragma unroll
      for (int m = 0; m < MR; ++m) part[(r * ks + kq) * MR + m] = v[m];
    }
    return;
  }
  for (int base = warp; base < rows; base += kGvWarps * RB) {
    float acc[RB][MR][2];
#pragma unroll
    for (int u = 0; u < RB; ++u)
#pragma unroll
      for (int m = 0; m < MR; ++m) acc[u][m][0] = acc[u][m][1] = 0.f;
    const int nu = min(RB, (rows - base + kGvWarps - 1) / kGvWarps);  // rows base + 8u < rows
    for (int ch = lane; ch < nch; ch += 32) {
      float xf[MR][8];
#pragma unroll
      for (int m = 0; m < MR; ++m) unpack8(x4[m * xstride + ch], xf[m]);
#pragma unroll
      for (int u = 0; u < RB; ++u) {
        if (u < nu) {
          float wf[8];
          unpack8(reinterpret_cast<const uint4*>(stage + (base + kGvWarps * u) * rb)[ch], wf);
#pragma unroll
          for (int m = 0; m < MR; ++m)
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
              acc[u][m][0] = fmaf(wf[e], xf[m][e], acc[u][m][0]);
              acc[u][m][1] = fmaf(wf[e + 1], xf[m][e + 1], acc[u][m][1]);
            }
        }
      }
    }
    float v[RB][MR];
#pragma unroll
    for (int u = 0; u < RB; ++u)
#pragma unroll
      for (int m = 0; m < MR; ++m) v[u][m] = acc[u][m][0] + acc[u][m][1];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int u = 0; u < RB; ++u)
#pragma unroll
        for (int m = 0; m < MR; ++m) v[u][m] += __shfl_xor_sync(0xffffffffu, v[u][m], o);
    if (lane == 0) {
#pragma unroll
      for (int u = 0; u < RB; ++u)
        if (u < nu) {
#pragma unroll
          for (int m = 0; m < MR; ++m) part[(base + kGvWarps * u) * MR + m] = v[u][m];
        }
    }
  }
}

// Epilogue inputs of one (feature, token) pair that come from global memory, loaded ahead of
// the dot products for a CTA's first chunk.
struct Pre {
  float h;     // EPI_RESID: residual value
  float c, s;  // EPI_QKV on q / k rows: rotary cos / sin at the token's position
  int slot;    // EPI_QKV: pool slot of the token (-1 padding)
};

SPECB200_DEVINL Pre load_pre(const GemvArgs& a, const Chunk& k, int j, int m) {
  const Epilogue& e = a.e;
  Pre q = {0.f, 1.f, 0.f, -1};
  if (e.op == EPI_RESID) {
    q.h = __bfloat162float(__ldcg(static_cast<const __nv_bfloat16*>(e.out) + static_cast<int64_t>(m) * e.ldo + k.f0 + j));
  } else if (e.op == EPI_QKV) {
    const int d = e.head_dim, half = d / 2;
    const int n = k.row0 + j;
    const int qkd = (e.n_heads + e.n_kv_heads) * d;
    if (n >= e.n_heads * d) q.slot = __ldcg(e.slot + m);
    if (n < qkd) {
      const int pos = __ldcg(e.pos + m);
      const int64_t off = static_cast<int64_t>(pos) * half + (n % d);
      q.c = round_to<__nv_bfloat16>(__ldg(e.rope_cos + off));
      q.s = round_to<__nv_bfloat16>(__ldg(e.rope_sin + off));
    }
  }
  return q;
}

template <int MR>
SPECB200_DEVINL float part_sum(const float* part, int ks, int r, int m) {
  float v = 0.f;
  for (int kq = 0; kq < ks; ++kq) v += part[(r * ks + kq) * MR + m];
  return v;
}

// The fused epilogue for output feature j of chunk k and token m: `lo` is the dot product of
// the feature's (first) weight row, `hi` that of its second row (gate/up and rotary pairs).
SPECB200_DEVINL void apply_one(const GemvArgs& a, const Chunk& k, int j, int m, float lo, float hi, const Pre& q) {
  using T = __nv_bfloat16;
  const Epilogue& e = a.e;
  switch (e.op) {
    case EPI_STORE: {
      const int64_t o = static_cast<int64_t>(m) * e.ldo + k.f0 + j;
      if (e.out_f32) static_cast<float*>(e.out)[o] = lo;
      else static_cast<T*>(e.out)[o] = from_f32<T>(lo);
      break;
    }
    case EPI_RESID: {
      const float proj = round_to<T>(lo);
      static_cast<T*>(e.out)[static_cast<int64_t>(m) * e.ldo + k.f0 + j] = from_f32<T>(q.h + proj);
      break;
    }
    case EPI_SILU_MUL: {
      const float g = round_to<T>(lo);
      const float u = round_to<T>(hi);
      const float act = round_to<T>(g / (1.0f + expf(-g)));
      static_cast<T*>(e.out)[static_cast<int64_t>(m) * e.ldo + k.f0 + j] = from_f32<T>(act * u);
      break;
    }
    case EPI_QKV: {
      const int d = e.head_dim, half = d / 2;
      const int qd = e.n_heads * d, kd = e.n_kv_heads * d;
      const int n = k.row0 + j;  // the pair's low row; its partner is n + half
      const int region = n < qd ? 0 : (n < qd + kd ? 1 : 2);
      lo = round_to<T>(lo);
      hi = round_to<T>(hi);
      if (region < 2) {
        const float lo2 = round_to<T>(round_to<T>(lo * q.c) + round_to<T>(-hi * q.s));
        const float hi2 = round_to<T>(round_to<T>(hi * q.c) + round_to<T>(lo * q.s));
        lo = lo2;
        hi = hi2;
      }
      if (region == 0) {
        T* out = static_cast<T*>(e.out) + static_cast<int64_t>(m) * e.ldo;
        out[n] = from_f32<T>(lo);
        out[n + half] = from_f32<T>(hi);
      } else if (q.slot >= 0) {
        const int idx = n - (region == 1 ? qd : qd + kd);
        const int hh = idx / d, i = idx % d;
        T* pool = static_cast<T*>(region == 1 ? e.k_pool : e.v_pool) + (static_cast<int64_t>(q.slot) * e.n_kv_heads + hh) * d;
        pool[i] = from_f32<T>(lo);
        pool[i + half] = from_f32<T>(hi);
      }
      break;
    }
    default:
      break;
  }
}

template <int MR>
SPECB200_DEVINL void epilogue(const GemvArgs& a, const Chunk& k, const float* part, bool have_pre, const Pre& pre) {
  const int ks = a.p.ksplit, nf = k.nf;
  for (int t = threadIdx.x; t < nf * MR; t += kGvThreads) {
    const int j = t % nf, m = t / nf;
    if (m >= a.M) continue;
    const Pre q = (have_pre && t == static_cast<int>(threadIdx.x)) ? pre : load_pre(a, k, j, m);
    const float lo = part_sum<MR>(part, ks, j, m);
    const float hi = a.p.segs == 2 ? part_sum<MR>(part, ks, nf + j, m) : 0.f;
    apply_one(a, k, j, m, lo, hi, q);
  }
}

template <int MR>
__global__ void __launch_bounds__(kGvThreads, 2) gemv_kernel(const __grid_constant__ GemvArgs a) {
  extern __shared__ __align__(128) uint8_t gv_smem_raw[];
  uint8_t* gv_smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gv_smem_raw) + 127) & ~uintptr_t(127));
  __shared__ float red[kGvWarps][MR];
  __shared__ int abort_flag;
  const GemvPlan& p = a.p;
  const int tid = threadIdx.x;
  const uint32_t cb = static_cast<uint32_t>(p.rows) * static_cast<uint32_t>(a.K) * 2u;
  uint8_t* ring = gv_smem;
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(gv_smem + static_cast<size_t>(p.stages) * cb);
  float* part = reinterpret_cast<float*>(xs + MR * a.K);
  const int part_elems = p.rows * p.ksplit * MR;
  uint64_t* full = reinterpret_cast<uint64_t*>(part + 2 * part_elems);
  const int n_mine = (p.chunks - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1;
  const uint64_t pol = l2_policy_evict_first();  // each weight byte is read once per forward
  unsigned long long* tr =
      a.trace ? a.trace + (static_cast<size_t>(a.trace_slot) * kGemvTraceCtas + blockIdx.x) * kGemvTraceStamps : nullptr;
  if (tr && tid == 0) tr[0] = gv_now();

  if (tid == 0) {
    for (int s = 0; s < p.stages; ++s) mbar_init(&full[s], 1);
    abort_flag = 0;
    fence_mbar_init();
    const int pre_n = min(p.stages, n_mine);
    for (int i = 0; i < pre_n; ++i) issue_chunk(a, blockIdx.x + i * gridDim.x, ring + i * cb, &full[i], pol);
  }
  pdl_launch_dependents();
  uint4 nw[kGvXChunks];
  {
    const int nch = a.K >> 3;
#pragma unroll
    for (int i = 0; i < kGvXChunks; ++i) {
      const int ch = tid + i * kGvThreads;
      nw[i] = (a.norm_w && ch < nch) ? __ldg(reinterpret_cast<const uint4*>(a.norm_w) + ch) : make_uint4(0, 0, 0, 0);
    }
  }
  pdl_wait();
  if (tr && tid == 0) tr[1] = gv_now();

  // Everything below reads what earlier kernels wrote.
  Pre pre = {0.f, 1.f, 0.f, -1};
  bool have_pre = false;
  {
    const Chunk k0 = chunk_at(p, blockIdx.x);
    if (tid < k0.nf * MR && tid / k0.nf < a.M) {
      pre = load_pre(a, k0, tid % k0.nf, tid / k0.nf);
      have_pre = true;
    }
  }
  stage_x<MR>(a, nw, xs, red, [] { __syncthreads(); });
  __syncthreads();
  if (tr && tid == 0) tr[2] = gv_now();

  unsigned long long t_wait = 0, t_dot = 0;  // trace only: thread 0's time in waits / dot products
  for (int i = 0; i < n_mine; ++i) {
    const int c = blockIdx.x + i * gridDim.x, st = i % p.stages;
    const Chunk k = chunk_at(p, c);
    const unsigned long long t0 = tr ? gv_now() : 0;
    const bool ok = mbar_wait_bounded(&full[st], (i / p.stages) & 1, a.status, &abort_flag);
    const unsigned long long t1 = tr ? gv_now() : 0;
    if (tr && tid == 0 && i == 0) tr[3] = t1;
    float* pb = part + (i & 1) * part_elems;
    if (ok) dot_chunk<MR>(p, a.K, k.nf, ring + static_cast<size_t>(st) * cb, xs, pb);
    // Every thread is done with this stage (and the previous chunk's partials) past here.
    if (__syncthreads_or(!ok)) break;
    if (tr) {
      t_wait += t1 - t0;
      t_dot += gv_now() - t1;
    }
    if (tid == 0 && i + p.stages < n_mine)
      issue_chunk(a, c + p.stages * gridDim.x, ring + static_cast<size_t>(st) * cb, &full[st], pol);
    epilogue<MR>(a, k, pb, i == 0 && have_pre, pre);
  }
  if (tr) {
    __syncthreads();
    if (tid == 0) {
      tr[4] = gv_now();
      tr[5] = t_wait;
      tr[6] = t_dot;
      tr[7] = n_mine;
    }
  }
}

template <int MR>
int launch_mr(const GemvArgs& a, cudaStream_t s, bool pdl) {
  const cudaError_t e = launch_kernel(gemv_kernel<MR>, dim3(a.p.grid), dim3(kGvThreads), a.p.smem, s, pdl, a);
  return e == cudaSuccess ? SPECB200_OK : SPECB200_ERR_CUDA;
}

int rows_instance(int M) { return M <= 1 ? 1 : (M <= 2 ? 2 : 4); }

}  // namespace

bool gemv_prepare() {
  static std::once_flag once;
  static bool ok = false;
  std::call_once(once, [] {
    const int bytes = static_cast<int>(kGvSmemBudget + 1024);
    ok = cudaFuncSetAttribute(gemv_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess &&
         cudaFuncSetAttribute(gemv_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess &&
         cudaFuncSetAttribute(gemv_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess;
    // the largest carveout, as every kernel of a forward, so that consecutive kernels share SMs
    for (const void* f : {reinterpret_cast<const void*>(gemv_kernel<1>), reinterpret_cast<const void*>(gemv_kernel<2>),
                          reinterpret_cast<const void*>(gemv_kernel<4>)})
      ok = ok && cudaFuncSetAttribute(f, cudaFuncAttributePreferredSharedMemoryCarveout,
                                      cudaSharedmemCarveoutMaxShared) == cudaSuccess;
  });
  return ok;
}

bool plan_gemv(int op, int M, int N, int K, int head_dim, GemvPlan* out) {
  if (M < 1 || M > kGemvMaxRows || N < 1 || K < 8 || K % 8 != 0 || K > kGvMaxK) return false;
  GemvPlan p = {};
  p.op = op;
  if (op == EPI_QKV) {
    if (head_dim < 2 || head_dim % 2 != 0 || N % head_dim != 0) return false;
    p.segs = 2;
    p.group = head_dim / 2;
    p.group_rows = head_dim;
    p.seg1_off = head_dim / 2;
    p.features = N / 2;
  } else if (op == EPI_SILU_MUL) {
    if (N % 128 != 0) return false;
    p.segs = 2;
    p.group = 64;
    p.group_rows = 128;
    p.seg1_off = 64;
    p.features = N / 2;
  } else if (op == EPI_STORE || op == EPI_RESID) {
    p.segs = 1;
    p.features = N;
  } else {
    return false;
  }
  const size_t rb = static_cast<size_t>(K) * 2;
  const int fmax = static_cast<int>(kGvChunkBudget / (p.segs * rb));
  if (fmax < 1) return false;
  int f = std::min(fmax, std::max(1, (p.features + kGvSms - 1) / kGvSms));
  if (p.segs == 2) {  // a power of two that divides the group, so chunks never cross a group
    int g = 1;
    while (g * 2 <= f && p.group % (g * 2) == 0) g *= 2;
    f = g;
  }
  p.f = f;
  p.rows = p.segs * f;
  p.chunks = (p.features + f - 1) / f;
  const size_t cb = static_cast<size_t>(p.rows) * rb;
  p.ksplit = (p.rows < kGvWarps && kGvWarps % p.rows == 0) ? kGvWarps / p.rows : 1;
  const int MR = rows_instance(M);
  const size_t fixed = static_cast<size_t>(MR) * K * 2 + 2 * static_cast<size_t>(p.rows) * p.ksplit * MR * 4;
  if (fixed + cb + 8 > kGvSmemBudget) return false;
  if (p.chunks <= 2 * kGvSms) {
    p.grid = p.chunks;
    p.stages = 1;
  } else {
    p.grid = kGvSms;
    const int per = (p.chunks + kGvSms - 1) / kGvSms;
    p.stages = std::max(1, std::min({per, static_cast<int>((kGvSmemBudget - fixed) / (cb + 8)), 8}));
  }
  p.smem = static_cast<size_t>(p.stages) * (cb + 8) + fixed + 128;  // + alignment slack
  *out = p;
  return true;
}

int launch_gemv(const GemvArgs& a, cudaStream_t s, bool pdl) {
  if (!a.w || !a.x || (reinterpret_cast<uintptr_t>(a.w) & 15) || (reinterpret_cast<uintptr_t>(a.x) & 15) ||
      (a.norm_w && (reinterpret_cast<uintptr_t>(a.norm_w) & 15)) || a.M < 1 || a.M > kGemvMaxRows)
    return SPECB200_ERR_ARG;
  switch (rows_instance(a.M)) {
    case 1: return launch_mr<1>(a, s, pdl);
    case 2: return launch_mr<2>(a, s, pdl);
    default: return launch_mr<4>(a, s, pdl);
  }
}

}  // namespace specb200
