// The Llama layer stack for decode-sized calls (at most 8 token rows) as one kernel on ONE
// thread-block cluster (16 CTAs, one per SM of a GPC), for small models whose per-layer
// weights are a few MB: there the forward is bound by the latency of its dependency chain
// (5 dependent steps per layer), not by HBM, and a cluster can pass data between SMs in
// ~150 ns where a grid-wide barrier costs ~2 us.
//
// Same computation as the per-layer kernels (forward.cu) -- lm/forward.py:21-84 with the
// Hugging Face Llama pieces, the same bf16 rounding points -- with a dataflow schedule:
//   * Weights: each GEMM kind's units (128 x 64 packed 16 KB tiles) are cut into C contiguous
//     ranges (stream-K); warp 4 of every CTA streams its ranges for all layers through a ring
//     with bulk copies of up to 64 KB, never waiting for activations; warp 5 issues
//     tcgen05.mma (M = 128 weight rows, N = 16 token columns) into two TMEM accumulators.
//   * Split-K partials go point-to-point: a contributor st.async's its fp32 partial into the
//     tile owner's shared memory, completing bytes on the owner's mbarrier; the owner sums the
//     partials in contributor order (deterministic) and runs the epilogue.
//   * Epilogue outputs go straight to their consumers' shared memory: roped q rows and the new
//     k/v rows to the attention items of their KV head; attention outputs and SiLU(gate)*up
//     blocks into the X operand slots of the CTAs whose O / down units need them (already in
//     the 128-byte-swizzled K-major layout the MMA reads).
//   * The residual stream h lives in global memory (L2); the owner of each 128-column tile
//     writes it and arrives (release, cluster scope) on every CTA's h barrier; RMSNorm
//     operands are built locally from h after that barrier.
// There is no cluster-wide barrier on the hot path. Every wait is bounded: a timeout records
// SPECB200_ERR_TIMEOUT and raises an abort flag in every CTA of the cluster; all CTAs then
// meet at the final cluster barrier, so no CTA exits while a peer may still write to it.
#include <algorithm>
#include <mutex>

#include "attn_mma.cuh"
#include "chain.cuh"
#include "epilogue.cuh"

namespace specb200 {
namespace {

constexpr int kThreads = 192;
constexpr uint32_t kUnitBytes = 16384;
constexpr int kRun = 4;    // units per bulk copy (64 KB)
constexpr int kTP = 132;   // fp32 tile pitch
constexpr int kKvBlocks = 4;  // attention K/V ring: blocks of 32 keys (8 KB)
constexpr int kItemSlots = 1024;  // cached keys of an attention item whose pool slots are resolved once per call

// ---------------------------------------------------------------- cluster PTX
SPECB200_DEVINL uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
SPECB200_DEVINL uint32_t mapa_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
SPECB200_DEVINL void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
SPECB200_DEVINL void st_async_v4(uint32_t raddr, uint4 v, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(raddr),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w), "r"(rbar)
               : "memory");
}
SPECB200_DEVINL void st_async_f32(uint32_t raddr, float v, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(raddr),
               "r"(__float_as_uint(v)), "r"(rbar)
               : "memory");
}
SPECB200_DEVINL void remote_arrive(uint32_t rbar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(rbar) : "memory");
}
SPECB200_DEVINL void st_cluster_u32(uint32_t raddr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(raddr), "r"(v) : "memory");
}
SPECB200_DEVINL bool try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
SPECB200_DEVINL void bulk_copy(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
SPECB200_DEVINL unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- stream-K partition
// CTA c owns units [U c / C, U (c + 1) / C); with U >= C every CTA owns at least one, and the
// contributors of a tile are consecutive CTAs, the first of which (holding the tile's first
// unit) owns the tile.
__host__ __device__ inline int range_lo(int U, int C, int c) {
  return static_cast<int>(static_cast<int64_t>(U) * c / C);
}
__host__ __device__ inline int owner_of(int U, int C, int u) {
  return static_cast<int>((static_cast<int64_t>(u + 1) * C - 1) / U);
}
__host__ __device__ inline int first_owned_tile(const ChainPhase& P, int C, int c) {
  return (range_lo(P.U, C, c) + P.kb - 1) / P.kb;
}
__host__ __device__ inline int contributors(const ChainPhase& P, int C, int t) {
  return owner_of(P.U, C, (t + 1) * P.kb - 1) - owner_of(P.U, C, t * P.kb) + 1;
}

// Floats between consecutive split partials in the combiner's buffer: R x 64 outputs, then R
// row maxima and R row sums, padded to 16 bytes so every partial starts 16-byte aligned for
// the vector st.async.
__host__ __device__ inline int comb_stride(int R) { return (R * 66 + 3) & ~3; }

// Partition of one GEMM kind as shared-memory tables (built once per launch, so the hot loops
// need no integer division): lo[c] = first unit of CTA c (lo[C] = U), own[u] = CTA owning unit u.
struct Part {
  const int* lo;
  const uint8_t* own;
  int U, kb;
  __device__ int first_tile(int c) const { return (lo[c] + kb - 1) / kb; }
  __device__ int owner_of_tile(int t) const { return own[t * kb]; }
  __device__ int contributors(int t) const { return own[(t + 1) * kb - 1] - own[t * kb] + 1; }
};

// ---------------------------------------------------------------- shared-memory context
struct Ctx {
  uint8_t *ring, *xn, *xp, *kvring;
  float* x32;
  float *pa, *pb, *comb, *ostage, *tile, *red;
  __nv_bfloat16 *qrecv, *knew, *vnew, *stage;
  uint64_t *full, *empty, *x_full, *xp_full, *acc_full, *acc_empty, *h_ready, *pbar, *attn_in, *comb_bar;
  uint32_t* tmem_holder;
  volatile int* abort_s;
  int *pos, *slot, *ids;
  int* lo_tab;        // [4][kChainMaxCluster + 1]
  int* key_slot;      // [kItemSlots] pool slot of the item's cached keys kc0 + j
  uint8_t* own_tab;   // units of the 4 kinds, concatenated
  uint32_t rank;
};

__device__ Ctx make_ctx(uint8_t* base, const ChainLayout& L) {
  Ctx c;
  c.ring = base;
  c.xn = base + L.xn;
  c.xp = base + L.xp;
  c.kvring = base + L.kvring;
  c.x32 = reinterpret_cast<float*>(base + L.x32);
  c.pa = reinterpret_cast<float*>(base + L.pa);
  c.pb = reinterpret_cast<float*>(base + L.pb);
  c.qrecv = reinterpret_cast<__nv_bfloat16*>(base + L.qrecv);
  c.knew = reinterpret_cast<__nv_bfloat16*>(base + L.kvrecv);
  c.vnew = c.knew + 8 * 64;
  c.comb = reinterpret_cast<float*>(base + L.comb);
  c.ostage = reinterpret_cast<float*>(base + L.ostage);
  c.tile = reinterpret_cast<float*>(base + L.tile);
  c.stage = reinterpret_cast<__nv_bfloat16*>(base + L.stage);
  uint64_t* b = reinterpret_cast<uint64_t*>(base + L.misc);
  c.full = b; b += kChainMaxSlots;
  c.empty = b; b += kChainMaxSlots;
  c.x_full = b++;
  c.xp_full = b++;
  c.acc_full = b; b += 2;
  c.acc_empty = b; b += 2;
  c.h_ready = b++;
  c.pbar = b; b += 2 * kChainOwnMax;
  c.attn_in = b++;
  c.comb_bar = b++;
  uint32_t* w = reinterpret_cast<uint32_t*>(b);
  c.tmem_holder = w++;
  c.abort_s = reinterpret_cast<volatile int*>(w++);
  c.pos = reinterpret_cast<int*>(w); w += kChainMaxRows;
  c.slot = reinterpret_cast<int*>(w); w += kChainMaxRows;
  c.ids = reinterpret_cast<int*>(w); w += kChainMaxRows;
  c.red = reinterpret_cast<float*>(w);  // [4 warps][kChainMaxRows]
  c.lo_tab = reinterpret_cast<int*>(base + L.part);
  c.key_slot = reinterpret_cast<int*>(base + L.keyslot);
  c.own_tab = reinterpret_cast<uint8_t*>(c.lo_tab + 4 * (kChainMaxCluster + 1));
  c.rank = cluster_rank();
  return c;
}
__device__ Part part_of(const ChainArgs& a, const Ctx& c, int kind) {
  Part p;
  p.lo = c.lo_tab + kind * (kChainMaxCluster + 1);
  int off = 0;
  for (int k = 0; k < kind; ++k) off += a.ph[k].U;
  p.own = c.own_tab + off;
  p.U = a.ph[kind].U;
  p.kb = a.ph[kind].kb;
  return p;
}
constexpr int kMiscBytes = (2 * kChainMaxSlots + 8 + 2 * kChainOwnMax + 2) * 8 + (2 + 3 * kChainMaxRows) * 4 +
                           4 * kChainMaxRows * 4;

__device__ void chain_abort(const ChainArgs& a, const Ctx& c) {
  set_status(a.status, SPECB200_ERR_TIMEOUT);
  for (int r = 0; r < a.C; ++r) st_cluster_u32(mapa_rank(smem_u32(const_cast<int*>(c.abort_s)), r), 1u);
}
// Bounded wait (acquire, cluster scope) on phase `parity` of a local mbarrier.
__device__ bool cwait(const ChainArgs& a, const Ctx& c, uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  if (try_wait_cluster(addr, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (try_wait_cluster(addr, parity)) return true;
    if (*c.abort_s) return false;
    if (clock64() - t0 > SPECB200_SPIN_LIMIT_CYCLES) {
      chain_abort(a, c);
      return false;
    }
  }
}

// lwait / cwait for a warp that issues with elect.sync: lane 0 waits, every lane gets the result.
__device__ bool lwait(const ChainArgs& a, const Ctx& c, uint64_t* bar, uint32_t parity);
__device__ bool lwait_warp(const ChainArgs& a, const Ctx& c, uint64_t* bar, uint32_t parity) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = lwait(a, c, bar, parity) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}
__device__ bool cwait_warp(const ChainArgs& a, const Ctx& c, uint64_t* bar, uint32_t parity) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = cwait(a, c, bar, parity) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// Bounded wait (acquire, CTA scope) for barriers completed by this CTA's own async units
// (bulk copies, tcgen05.commit) or threads.
__device__ bool lwait(const ChainArgs& a, const Ctx& c, uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*c.abort_s) return false;
    if (clock64() - t0 > SPECB200_SPIN_LIMIT_CYCLES) {
      chain_abort(a, c);
      return false;
    }
  }
}

// Profiling record, [C][n_layers * 5 phases][16] (kTraceSlots): globaltimer stamps written by
// compute thread 0 -- [0] phase start, [1] operand ready (norm phases) / query arrived
// (attention), [2] own segments done, [3] phase end, [12] h barrier passed; by the MMA thread
// [4] operand observed, [5] last MMA issued; by the weight thread [6] last copy issued -- and
// cycle counts: [8] / [9] / [10] CUDA-core loop waiting for weights / computing / releasing
// slots, [11] MMA thread waiting for weights, [14] SM cycles over the attention phase.
constexpr int kTraceSlots = 16;
SPECB200_DEVINL void trace_put(const ChainArgs& a, const Ctx& c, int idx, int which, unsigned long long v) {
  if (a.trace) a.trace[(static_cast<size_t>(c.rank) * a.n_layers * 5 + idx) * kTraceSlots + which] = v;
}
SPECB200_DEVINL void stamp_at(const ChainArgs& a, const Ctx& c, int idx, int which) {
  if (a.trace) trace_put(a, c, idx, which, now_ns());
}
SPECB200_DEVINL void stamp(const ChainArgs& a, const Ctx& c, int idx, int which) {
  if (threadIdx.x == 0) stamp_at(a, c, idx, which);
}

// The residual stream tile just written to global memory is visible: arrive on every CTA's
// h barrier (the CTA barrier orders all 128 threads' stores before the release arrives).
__device__ void signal_h(const ChainArgs& a, const Ctx& c) {
  epi_bar_sync();
  if (threadIdx.x < a.C) remote_arrive(mapa_rank(smem_u32(c.h_ready), threadIdx.x));
}

struct Counters {
  uint32_t h, segs, ain, comb, g, xp;
  long long cy_wait, cy_fma, cy_rel;  // profiling: cycles in the CUDA-core unit loop
  uint32_t pb[2][kChainOwnMax];
};

// ---------------------------------------------------------------- X operand from RMSNorm(h)
// Slot i (1 KB, swizzled 128-byte rows, row m = token) holds the normalised 64-column block of
// unit u0 + i. Thread t keeps 16-byte chunk t of every row (H <= 1024).
__device__ void build_xn(const ChainArgs& a, const Ctx& c, uint4 wv, int u0, int u1, int kb) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int chunks = a.H / 8, M = a.M;
  uint4 hv[kChainMaxRows];
  float ss[kChainMaxRows];
#pragma unroll
  for (int m = 0; m < kChainMaxRows; ++m) {
    hv[m] = make_uint4(0, 0, 0, 0);
    if (m < M && tid < chunks) hv[m] = __ldcg(reinterpret_cast<const uint4*>(a.h + static_cast<size_t>(m) * a.H) + tid);
  }
#pragma unroll
  for (int m = 0; m < kChainMaxRows; ++m) {
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&hv[m]);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h2[j]);
      s = fmaf(f.x, f.x, s);
      s = fmaf(f.y, f.y, s);
    }
    ss[m] = warp_sum(s);
  }
  if (lane == 0) {
#pragma unroll
    for (int m = 0; m < kChainMaxRows; ++m) c.red[warp * kChainMaxRows + m] = ss[m];
  }
  epi_bar_sync();
  if (tid < chunks) {
    const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&wv);
    const int kbt = tid >> 3, cc = tid & 7;
#pragma unroll
    for (int m = 0; m < kChainMaxRows; ++m) {
      if (m >= M) break;
      const float sum = c.red[m] + c.red[kChainMaxRows + m] + c.red[2 * kChainMaxRows + m] + c.red[3 * kChainMaxRows + m];
      const float inv = 1.0f / sqrtf(sum / static_cast<float>(a.H) + a.eps);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&hv[m]);
      uint4 o;
      __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h2[j]);
        const float2 wf = __bfloat1622float2(w2[j]);
        const float nx = round_to<__nv_bfloat16>(f.x * inv), ny = round_to<__nv_bfloat16>(f.y * inv);
        o2[j] = __floats2bfloat162_rn(wf.x * nx, wf.y * ny);
      }
      if (a.fma) {
        float4 lo, hi;
        lo.x = __bfloat162float(o2[0].x); lo.y = __bfloat162float(o2[0].y);
        lo.z = __bfloat162float(o2[1].x); lo.w = __bfloat162float(o2[1].y);
        hi.x = __bfloat162float(o2[2].x); hi.y = __bfloat162float(o2[2].y);
        hi.z = __bfloat162float(o2[3].x); hi.w = __bfloat162float(o2[3].y);
        for (int u = u0; u < u1; ++u)
          if (u % kb == kbt) {
            float* d = c.x32 + ((u - u0) * M + m) * 64 + cc * 8;
            *reinterpret_cast<float4*>(d) = lo;
            *reinterpret_cast<float4*>(d + 4) = hi;
          }
      } else {
        for (int u = u0; u < u1; ++u)
          if (u % kb == kbt) *reinterpret_cast<uint4*>(c.xn + (u - u0) * 1024 + m * 128 + ((cc ^ (m & 7)) << 4)) = o;
      }
    }
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  epi_bar_sync();
}

// ---------------------------------------------------------------- epilogues of owned tiles
// tile: fp32 [M][kTP], column j = output feature t * 128 + j.

// cs / sn: rounded RoPE cos / sin of each row's position at this thread's rotary index
// (tid % 32: heads are 64-row aligned inside the 128-row tile), loaded at phase start.
__device__ void epi_qkv(const ChainArgs& a, const Ctx& c, int l, int t, const float (&cs)[kChainMaxRows],
                        const float (&sn)[kChainMaxRows]) {
  const int tid = threadIdx.x, M = a.M, D = 64;
  const int qd = a.Hq * D, kd = a.Hkv * D, N = qd + 2 * kd;
  const int n = t * 128 + tid;
  const size_t layer_pool = static_cast<size_t>(a.num_slots) * a.Hkv * D;
  if (n < N) {
    const int region = n < qd ? 0 : (n < qd + kd ? 1 : 2);
    const int idx = n - (region == 0 ? 0 : (region == 1 ? qd : qd + kd));
    const int hh = idx / D, i = idx % D;
    const int partner = i < 32 ? tid + 32 : tid - 32;
    __nv_bfloat16* pool = (region == 1 ? a.k_pool : a.v_pool) + l * layer_pool;
#pragma unroll
    for (int m = 0; m < kChainMaxRows; ++m) {
      if (m >= M) break;
      float y = round_to<__nv_bfloat16>(c.tile[m * kTP + tid]);
      if (region < 2) {
        const float xp = round_to<__nv_bfloat16>(c.tile[m * kTP + partner]);
        const float rot = i < 32 ? -xp : xp;
        y = round_to<__nv_bfloat16>(round_to<__nv_bfloat16>(y * cs[m]) + round_to<__nv_bfloat16>(rot * sn[m]));
      }
      const __nv_bfloat16 yb = __float2bfloat16_rn(y);
      c.stage[m * 128 + tid] = yb;
      if (region > 0 && c.slot[m] >= 0) pool[(static_cast<int64_t>(c.slot[m]) * a.Hkv + hh) * D + i] = yb;
    }
  }
  epi_bar_sync();
  // 16-byte chunks (8 features of one head) to the attention items of their KV head
  const int G = a.Hq / a.Hkv, S = a.splits;
  const int work = M * 16 * S;
  for (int w = tid; w < work; w += 128) {
    const int s = w % S, mk = w / S, m = mk >> 4, k = mk & 15;
    const int row0 = t * 128 + k * 8;
    if (row0 >= N) continue;
    const int region = row0 < qd ? 0 : (row0 < qd + kd ? 1 : 2);
    if (region > 0 && s != 0) continue;
    const int idx = row0 - (region == 0 ? 0 : (region == 1 ? qd : qd + kd));
    const int hh = idx / D, c8 = (idx % D) >> 3;
    const int b = m / a.T, tt = m % a.T;
    const uint4 v = *reinterpret_cast<const uint4*>(c.stage + m * 128 + k * 8);
    int dst;
    uint32_t addr;
    if (region == 0) {
      const int g = hh / G;
      dst = (b * a.Hkv + g) * S + s;
      addr = smem_u32(c.qrecv + am_swz(tt * G + hh % G, c8 * 8));
    } else {
      dst = (b * a.Hkv + hh) * S + (S - 1);
      addr = smem_u32((region == 1 ? c.knew : c.vnew) + am_swz(tt, c8 * 8));
    }
    st_async_v4(mapa_rank(addr, dst), v, mapa_rank(smem_u32(c.attn_in), dst));
  }
}

// h rows of output tile t (this thread's column), read before the tile's partials are awaited.
__device__ void load_h_tile(const ChainArgs& a, int t, float (&hold)[kChainMaxRows]) {
  const int n = t * 128 + threadIdx.x;
#pragma unroll
  for (int m = 0; m < kChainMaxRows; ++m)
    hold[m] = (m < a.M && n < a.H) ? __bfloat162float(__ldcg(a.h + static_cast<size_t>(m) * a.H + n)) : 0.f;
}

__device__ void epi_resid(const ChainArgs& a, const Ctx& c, int t, const float (&hold)[kChainMaxRows]) {
  const int tid = threadIdx.x, n = t * 128 + tid;
  if (n < a.H) {
#pragma unroll
    for (int m = 0; m < kChainMaxRows; ++m)
      if (m < a.M)
        a.h[static_cast<size_t>(m) * a.H + n] = __float2bfloat16_rn(hold[m] + round_to<__nv_bfloat16>(c.tile[m * kTP + tid]));
  }
  signal_h(a, c);
}

// Push a [rows][64] bf16 block (stage, row r -> token row tok(r)) as 64-column block `kblk` of
// phase P's operand to every CTA whose units need it.
template <typename TokOf>
__device__ void push_operand(const ChainArgs& a, const Ctx& c, int kind, int kblk, int rows, TokOf tok_of) {
  const ChainPhase& P = a.ph[kind];
  const Part pt = part_of(a, c, kind);
  const int work = P.n_tiles * rows * 8;
  for (int w = threadIdx.x; w < work; w += 128) {
    const int cc = w & 7, r = (w >> 3) % rows, tile = (w >> 3) / rows;
    const int u = tile * P.kb + kblk;
    const int cons = pt.own[u];
    const int sl = u - pt.lo[cons];
    const int m = tok_of(r);
    const uint4 v = *reinterpret_cast<const uint4*>(c.stage + r * 64 + cc * 8);
    const uint32_t addr = smem_u32(c.xp + sl * 1024 + m * 128 + ((cc ^ (m & 7)) << 4));
    st_async_v4(mapa_rank(addr, cons), v, mapa_rank(smem_u32(c.xp_full), cons));
  }
}

__device__ void epi_gu(const ChainArgs& a, const Ctx& c, int t) {
  const int tid = threadIdx.x;
  if (tid < 64) {
    for (int m = 0; m < a.M; ++m) {
      const float g = round_to<__nv_bfloat16>(c.tile[m * kTP + tid]);
      const float u = round_to<__nv_bfloat16>(c.tile[m * kTP + 64 + tid]);
      const float act = round_to<__nv_bfloat16>(g / (1.0f + expf(-g)));
      c.stage[m * 64 + tid] = __float2bfloat16_rn(act * u);
    }
  }
  epi_bar_sync();
  push_operand(a, c, CK_DOWN, t, a.M, [](int r) { return r; });
}

// ---------------------------------------------------------------- CUDA-core GEMM units
// For calls of one or two token rows the tensor cores would run at N = 16 with ~120 cycles
// per instruction; plain fp32 FMAs stream weights faster. Thread t takes weight row t of the
// packed tile (its 16-byte chunk c sits at c ^ (t & 7)), the activations come from x32
// ([slot][M][64] fp32) as broadcast loads, and four partial sums per row keep the FMA chains
// short; bf16 weights widen to fp32 exactly by a 16-bit shift.
template <int MM>
__device__ __forceinline__ void fma_unit(const uint8_t* tile, const float* x, float (&acc)[MM][8]) {
  const int r = threadIdx.x;
  const uint8_t* row = tile + r * 128;
  uint4 wv[8];
#pragma unroll
  for (int cidx = 0; cidx < 8; ++cidx) wv[cidx] = *reinterpret_cast<const uint4*>(row + ((cidx ^ (r & 7)) << 4));
#pragma unroll
  for (int cidx = 0; cidx < 8; ++cidx) {
    const uint32_t wd[4] = {wv[cidx].x, wv[cidx].y, wv[cidx].z, wv[cidx].w};
#pragma unroll
    for (int m = 0; m < MM; ++m) {
      const float4 xa = *reinterpret_cast<const float4*>(x + m * 64 + cidx * 8);
      const float4 xb = *reinterpret_cast<const float4*>(x + m * 64 + cidx * 8 + 4);
      const float xs[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[m][2 * j] = fmaf(__uint_as_float(wd[j] << 16), xs[2 * j], acc[m][2 * j]);
        acc[m][2 * j + 1] = fmaf(__uint_as_float(wd[j] & 0xffff0000u), xs[2 * j + 1], acc[m][2 * j + 1]);
      }
    }
  }
}

// The pushed bf16 operand blocks (swizzled rows) of this CTA's units as fp32 rows.
__device__ void xp_to_x32(const ChainArgs& a, const Ctx& c, int nunits) {
  const int M = a.M;
  for (int w = threadIdx.x; w < nunits * M * 8; w += 128) {
    const int cc = w & 7, m = (w >> 3) % M, sl = (w >> 3) / M;
    const uint4 v = *reinterpret_cast<const uint4*>(c.xp + sl * 1024 + m * 128 + ((cc ^ (m & 7)) << 4));
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&v);
    float* d = c.x32 + (sl * M + m) * 64 + cc * 8;
    float4 lo, hi;
    lo.x = __bfloat162float(h2[0].x); lo.y = __bfloat162float(h2[0].y);
    lo.z = __bfloat162float(h2[1].x); lo.w = __bfloat162float(h2[1].y);
    hi.x = __bfloat162float(h2[2].x); hi.y = __bfloat162float(h2[2].y);
    hi.z = __bfloat162float(h2[3].x); hi.w = __bfloat162float(h2[3].y);
    *reinterpret_cast<float4*>(d) = lo;
    *reinterpret_cast<float4*>(d + 4) = hi;
  }
}

// One segment (units [u, seg_end) of one tile) on the CUDA cores, consuming the weight ring
// in the producer's order; returns this thread's row sums in v[0..M).
template <int MM>
__device__ bool fma_segment(const ChainArgs& a, const Ctx& c, int u0, int u, int seg_end, int u1, Counters& k,
                            int& run_left, float (&v)[16]) {
  const int S = a.L.ring_slots;
  float acc[MM][8];
#pragma unroll
  for (int m = 0; m < MM; ++m)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[m][j] = 0.f;
  for (int uu = u; uu < seg_end; ++uu, ++k.g) {
    const int st = static_cast<int>(k.g % S);
    const long long c0 = clock64();
    if (run_left == 0) {
      run_left = min(min(kRun, u1 - uu), S - st);
      if (!lwait(a, c, &c.full[st], (k.g / S) & 1)) return false;
    }
    --run_left;
    const long long c1 = clock64();
    fma_unit<MM>(c.ring + st * kUnitBytes, c.x32 + (uu - u0) * MM * 64, acc);
    const long long c2 = clock64();
    epi_bar_sync();  // every thread is done with the slot
    if (threadIdx.x == 0) mbar_arrive(&c.empty[st]);
    const long long c3 = clock64();
    k.cy_wait += c1 - c0;
    k.cy_fma += c2 - c1;
    k.cy_rel += c3 - c2;
  }
#pragma unroll
  for (int m = 0; m < MM; ++m)
    v[m] = ((acc[m][0] + acc[m][1]) + (acc[m][2] + acc[m][3])) + ((acc[m][4] + acc[m][5]) + (acc[m][6] + acc[m][7]));
  return true;
}

// ---------------------------------------------------------------- one GEMM phase
__device__ bool gemm_phase(const ChainArgs& a, const Ctx& c, uint32_t tmem_base, int kind, int l, Counters& k) {
  const ChainPhase& P = a.ph[kind];
  const int C = a.C, rank = static_cast<int>(c.rank), tid = threadIdx.x, warp = tid >> 5;
  const Part pt = part_of(a, c, kind);
  const int u0 = pt.lo[rank], u1 = pt.lo[rank + 1];
  const int pidx = l * 5 + (kind == CK_QKV ? 0 : kind == CK_O ? 2 : kind == CK_GU ? 3 : 4);
  const int region = (kind == CK_QKV || kind == CK_GU) ? 0 : 1;
  float* preg = region ? c.pb : c.pa;
  const int ncR = region ? a.L.ncB : a.L.ncA;
  const int slot_floats = a.M * 128;
  const int t_first = pt.first_tile(rank);
  uint64_t* pbar = c.pbar + region * kChainOwnMax;
  if (tid == 0) {
    for (int t = t_first; t * P.kb < u1; ++t) {
      const int nc = pt.contributors(t);
      if (nc > 1) mbar_arrive_expect_tx(&pbar[t - t_first], static_cast<uint32_t>((nc - 1) * slot_floats * 4));
    }
  }
  // epilogue inputs that do not depend on this phase's results, loaded now
  float cs[kChainMaxRows], sn[kChainMaxRows], hold0[kChainMaxRows], hold1[kChainMaxRows];
  if (kind == CK_QKV) {
#pragma unroll
    for (int m = 0; m < kChainMaxRows; ++m) {
      const int64_t off = static_cast<int64_t>(m < a.M ? c.pos[m] : 0) * 32 + (tid & 31);
      cs[m] = round_to<__nv_bfloat16>(a.rope_cos[off]);
      sn[m] = round_to<__nv_bfloat16>(a.rope_sin[off]);
    }
  }
  if (region == 1) {
    // h is final for this phase: written before the h barrier this CTA passed in the phase
    // before (QKV for O, gate/up for down), and only this tile's owner rewrites its columns
    if (t_first * P.kb < u1) load_h_tile(a, t_first, hold0);
    if ((t_first + 1) * P.kb < u1) load_h_tile(a, t_first + 1, hold1);
  }
  if (region == 0) {
    const __nv_bfloat16* norm_w = kind == CK_QKV ? a.layers[l].attn_norm : a.layers[l].mlp_norm;
    const uint4 wv = tid < a.H / 8 ? reinterpret_cast<const uint4*>(norm_w)[tid] : make_uint4(0, 0, 0, 0);
    if (!cwait(a, c, c.h_ready, k.h & 1)) return false;
    ++k.h;
    stamp(a, c, pidx, 12);
    build_xn(a, c, wv, u0, u1, P.kb);
    if (tid == 0 && !a.fma) mbar_arrive(c.x_full);
    stamp(a, c, pidx, 1);
  } else {
    if (tid == 0) mbar_arrive_expect_tx(c.xp_full, static_cast<uint32_t>((u1 - u0) * a.M * 128));
    if (a.fma) {
      if (!cwait(a, c, c.xp_full, k.xp & 1)) return false;
      ++k.xp;
      xp_to_x32(a, c, u1 - u0);
      epi_bar_sync();
    }
  }
  int run_left = 0;
  // accumulators: keep the owner's own share, push the rest to the tile owners
  for (int u = u0; u < u1;) {
    const int t = u / P.kb;
    const int seg_end = min(u1, (t + 1) * P.kb);
    const uint32_t buf = k.segs & 1;
    float v[16];
    if (a.fma) {
      const bool fok = a.M == 1 ? fma_segment<1>(a, c, u0, u, seg_end, u1, k, run_left, v)
                                : fma_segment<2>(a, c, u0, u, seg_end, u1, k, run_left, v);
      if (!fok) return false;
    } else {
      if (!lwait(a, c, &c.acc_full[buf], (k.segs >> 1) & 1)) return false;
      tc_fence_after();
      tmem_ld16(tmem_base + (static_cast<uint32_t>(warp * 32) << 16) + buf * kStreamBN, v);
      tmem_ld_wait();
    }
    const int cown = pt.owner_of_tile(t);
    const int j = rank - cown;
    const int o = t - pt.first_tile(cown);
    if (j == 0) {
      float* dst = preg + (o * ncR) * slot_floats;
#pragma unroll
      for (int m = 0; m < kChainMaxRows; ++m)
        if (m < a.M) dst[m * 128 + tid] = v[m];
    } else {
      const uint32_t rdst = mapa_rank(smem_u32(preg + (o * ncR + j) * slot_floats), cown);
      const uint32_t rbar = mapa_rank(smem_u32(&pbar[o]), cown);
#pragma unroll
      for (int m = 0; m < kChainMaxRows; ++m)
        if (m < a.M) st_async_f32(rdst + (m * 128 + tid) * 4, v[m], rbar);
    }
    if (!a.fma) {
      tc_fence_before();
      epi_bar_sync();
      if (tid == 0) mbar_arrive(&c.acc_empty[buf]);
    }
    ++k.segs;
    u = seg_end;
  }
  stamp(a, c, pidx, 2);
  if (a.fma && tid == 0) {
    trace_put(a, c, pidx, 8, k.cy_wait);
    trace_put(a, c, pidx, 9, k.cy_fma);
    trace_put(a, c, pidx, 10, k.cy_rel);
    k.cy_wait = k.cy_fma = k.cy_rel = 0;
  }
  // owned tiles: sum the contributors in order, then the epilogue
  for (int t = t_first; t * P.kb < u1; ++t) {
    const int o = t - t_first;
    const int nc = pt.contributors(t);
    if (nc > 1) {
      if (!cwait(a, c, &pbar[o], k.pb[region][o] & 1)) return false;
      ++k.pb[region][o];
    }
    const float* src = preg + o * ncR * slot_floats;
    for (int m = 0; m < a.M; ++m) {
      float s = 0.f;
      for (int jj = 0; jj < nc; ++jj) s += src[jj * slot_floats + m * 128 + tid];
      c.tile[m * kTP + tid] = s;
    }
    epi_bar_sync();
    if (kind == CK_QKV) {
      epi_qkv(a, c, l, t, cs, sn);
    } else if (kind == CK_GU) {
      epi_gu(a, c, t);
    } else if (o < 2) {
      epi_resid(a, c, t, o == 0 ? hold0 : hold1);
    } else {
      float hold[kChainMaxRows];
      load_h_tile(a, t, hold);
      epi_resid(a, c, t, hold);
    }
    epi_bar_sync();
  }
  return true;
}

// ---------------------------------------------------------------- attention item
// Item rank = (b * Hkv + g) * S + s: sequence b, KV head g, key split s. Split s covers the
// cached keys [past * s / S, past * (s + 1) / S); the last split also takes the call's new
// keys, which arrive with q from the QKV tile owners. Cached keys do not depend on the layer's
// activations, so their first kKvBlocks blocks are requested at the start of the layer (before
// the QKV phase) into a ring of 32-key blocks and are resident when q arrives.
struct Item {
  int b, g, s, past, nn, kc0, kc1, nblk;
  bool active;
};

__device__ Item item_of(const ChainArgs& a, const Ctx& c) {
  Item it;
  const int S = a.splits, rank = static_cast<int>(c.rank);
  it.active = rank < a.B * a.Hkv * S;
  it.b = rank / (a.Hkv * S);
  it.g = (rank / S) % a.Hkv;
  it.s = rank % S;
  it.past = it.active ? a.past[it.b] : 0;
  it.nn = it.active ? a.n_new[it.b] : 0;
  it.kc0 = static_cast<int>(static_cast<int64_t>(it.past) * it.s / S);
  it.kc1 = static_cast<int>(static_cast<int64_t>(it.past) * (it.s + 1) / S);
  it.nblk = (it.kc1 - it.kc0 + 31) / 32;
  return it;
}

// Cached-key block j of the item into ring slot j % kKvBlocks ([K 32 x 64 | V 32 x 64], swizzled
// rows; keys past the split's end are zero). Commits one cp.async group.
__device__ void kv_load_block(const ChainArgs& a, const Ctx& c, const Item& it, int l, int j) {
  const size_t layer_pool = static_cast<size_t>(a.num_slots) * a.Hkv * 64;
  const __nv_bfloat16* kp = a.k_pool + l * layer_pool;
  const __nv_bfloat16* vp = a.v_pool + l * layer_pool;
  const int32_t* table = a.table + static_cast<int64_t>(it.b) * a.table_stride;
  __nv_bfloat16* blk = reinterpret_cast<__nv_bfloat16*>(c.kvring) + (j % kKvBlocks) * 4096;
  const int k0 = it.kc0 + j * 32;
  for (int idx = threadIdx.x; idx < 32 * 16; idx += 128) {
    const int r = idx >> 4, part = idx & 15, isv = part >> 3, cc = part & 7;
    __nv_bfloat16* dst = blk + isv * 2048 + am_swz(r, cc * 8);
    const int key = k0 + r;
    if (key < it.kc1) {
      const int j = key - it.kc0;
      const int64_t sl = j < kItemSlots ? c.key_slot[j] : static_cast<int64_t>(table[key / a.bs]) * a.bs + key % a.bs;
      cp_async_16(dst, (isv ? vp : kp) + (sl * a.Hkv + it.g) * 64 + cc * 8);
    } else {
      *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    }
  }
  cp_async_commit();
}

__device__ void attn_prefetch(const ChainArgs& a, const Ctx& c, int l) {
  const Item it = item_of(a, c);
  if (!it.active) return;
  for (int j = 0; j < min(kKvBlocks, it.nblk); ++j) kv_load_block(a, c, it, l, j);
}

static_assert(kKvBlocks <= 4, "cp_async_wait_upto covers up to 3 pending groups");

__device__ bool attention_phase(const ChainArgs& a, const Ctx& c, int l, Counters& k) {
  const Item it = item_of(a, c);
  if (!it.active) return true;
  const int S = a.splits, rank = static_cast<int>(c.rank), tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b = it.b, g = it.g, s = it.s;
  const int G = a.Hq / a.Hkv, R = a.T * G;
  const int past = it.past, nn = it.nn, total = past + nn;
  if (tid == 0) {
    mbar_arrive_expect_tx(c.attn_in, static_cast<uint32_t>(R * 128 + (s == S - 1 ? 2 * a.T * 128 : 0)));
    if (s == 0 && S > 1) mbar_arrive_expect_tx(c.comb_bar, static_cast<uint32_t>((S - 1) * R * 66 * 4));
  }
  if (!cwait(a, c, c.attn_in, k.ain & 1)) return false;
  ++k.ain;
  stamp(a, c, l * 5 + 1, 1);
  AmState st;
  am_init(st, c.qrecv);
  const int r0 = lane >> 2, r1 = r0 + 8;
  const int lim0 = r0 < R ? min(past + r0 / G + 1, total) : 0;
  const int lim1 = r1 < R ? min(past + r1 / G + 1, total) : 0;
  for (int j = 0; j < it.nblk; ++j) {
    cp_async_wait_upto(min(it.nblk, j + kKvBlocks) - (j + 1));  // block j has landed
    epi_bar_sync();
    const __nv_bfloat16* blk = reinterpret_cast<const __nv_bfloat16*>(c.kvring) + (j % kKvBlocks) * 4096;
    const int k0 = it.kc0 + j * 32 + warp * 8;
    const int nval = min(8, it.kc1 - k0);
    if (nval > 0) am_step(st, blk, blk + 2048, warp * 8, k0, nval, lim0, lim1, a.attn_scale);
    epi_bar_sync();
    if (j + kKvBlocks < it.nblk) kv_load_block(a, c, it, l, j + kKvBlocks);
  }
  if (s == S - 1 && nn > 0 && warp == 0) am_step(st, c.knew, c.vnew, 0, past, min(nn, 8), lim0, lim1, a.attn_scale);
  float* oo = c.ostage;
  float* om = oo + 16 * 64;
  float* ol = om + 16;
  am_merge(st, reinterpret_cast<float*>(c.kvring), R, oo, om, ol, [] { epi_bar_sync(); });
  const int pstride = comb_stride(R);
  if (S > 1 && s > 0) {
    const int comb_cta = rank - s;
    float* dst = c.comb + (s - 1) * pstride;
    const uint32_t rbar = mapa_rank(smem_u32(c.comb_bar), comb_cta);
    for (int i = tid; i < R * 16; i += 128)
      st_async_v4(mapa_rank(smem_u32(dst + i * 4), comb_cta), *reinterpret_cast<const uint4*>(oo + i * 4), rbar);
    for (int i = tid; i < 2 * R; i += 128)
      st_async_f32(mapa_rank(smem_u32(dst + R * 64 + i), comb_cta), i < R ? om[i] : ol[i - R], rbar);
    return true;
  }
  if (S > 1) {
    if (!cwait(a, c, c.comb_bar, k.comb & 1)) return false;
    ++k.comb;
  }
  for (int i = tid; i < R * 64; i += 128) {
    const int r = i >> 6;
    float Mx = om[r];
    for (int sp = 1; sp < S; ++sp) Mx = fmaxf(Mx, c.comb[(sp - 1) * pstride + R * 64 + r]);
    float O = 0.f, Ls = 0.f;
    for (int sp = 0; sp < S; ++sp) {
      const float* base = sp == 0 ? nullptr : c.comb + (sp - 1) * pstride;
      const float ms = sp == 0 ? om[r] : base[R * 64 + r];
      const float ls = sp == 0 ? ol[r] : base[R * 64 + R + r];
      const float ov = sp == 0 ? oo[i] : base[i];
      const float w = (ms == -INFINITY) ? 0.f : exp2f(ms - Mx);  // base-2 maxima (am_step)
      O = fmaf(ov, w, O);
      Ls = fmaf(ls, w, Ls);
    }
    c.stage[i] = __float2bfloat16_rn(O / Ls);
  }
  epi_bar_sync();
  // rows r = t * G + j (head g * G + j) go to 64-column block (head) of the O operand
  const ChainPhase& P = a.ph[CK_O];
  const Part pt = part_of(a, c, CK_O);
  const int work = P.n_tiles * R * 8;
  for (int w = tid; w < work; w += 128) {
    const int cc = w & 7, r = (w >> 3) % R, tile = (w >> 3) / R;
    const int head = g * G + r % G, m = b * a.T + r / G;
    const int u = tile * P.kb + head;
    const int cons = pt.own[u];
    const int sl = u - pt.lo[cons];
    const uint4 v = *reinterpret_cast<const uint4*>(c.stage + r * 64 + cc * 8);
    const uint32_t addr = smem_u32(c.xp + sl * 1024 + m * 128 + ((cc ^ (m & 7)) << 4));
    st_async_v4(mapa_rank(addr, cons), v, mapa_rank(smem_u32(c.xp_full), cons));
  }
  return true;
}

// ---------------------------------------------------------------- the kernel
SPECB200_DEVINL const uint8_t* phase_weights(const StreamLayer& L, int kind) {
  return kind == CK_QKV ? L.qkv : kind == CK_O ? L.o : kind == CK_GU ? L.gu : L.down;
}

__global__ void __launch_bounds__(kThreads, 1) chain_kernel(const __grid_constant__ ChainArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Ctx c = make_ctx(base, a.L);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = a.L.ring_slots;

  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&c.full[i], 1);
      mbar_init(&c.empty[i], 1);
    }
    mbar_init(c.x_full, 1);
    mbar_init(c.xp_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&c.acc_full[i], 1);
      mbar_init(&c.acc_empty[i], 1);
    }
    mbar_init(c.h_ready, a.ph[CK_O].n_tiles);
    for (int i = 0; i < 2 * kChainOwnMax; ++i) mbar_init(&c.pbar[i], 1);
    mbar_init(c.attn_in, 1);
    mbar_init(c.comb_bar, 1);
    *c.abort_s = 0;
    fence_mbar_init();
  }
  if (tid < a.M) {
    const int m = tid, b = m / a.T, t = m % a.T;
    const int pos = a.past[b] + t;
    int slot = -1;
    if (t < a.n_new[b]) {
      const int blk = pos / a.bs;
      if (pos >= a.max_positions || blk >= a.table_stride) {
        set_status(a.status, SPECB200_ERR_RANGE);
      } else {
        const int64_t s = static_cast<int64_t>(a.table[static_cast<int64_t>(b) * a.table_stride + blk]) * a.bs + pos % a.bs;
        if (s < 0 || s >= a.num_slots) set_status(a.status, SPECB200_ERR_RANGE);
        else slot = static_cast<int>(s);
      }
    }
    c.pos[m] = min(pos, a.max_positions - 1);
    c.slot[m] = slot;
    int id = a.ids[m];
    if (id < 0 || id >= a.V) {
      set_status(a.status, SPECB200_ERR_RANGE);
      id = 0;
    }
    c.ids[m] = id;
  }
  // query / new-key receive rows past the call's rows stay zero (finite MMA operands)
  for (int i = tid; i < (16 * 64 + 16 * 64) / 8; i += kThreads)
    reinterpret_cast<uint4*>(i < 128 ? static_cast<void*>(c.qrecv) : static_cast<void*>(c.knew))[i < 128 ? i : i - 128] =
        make_uint4(0, 0, 0, 0);
  // pool slots of this CTA's attention keys: the block table is fixed for the whole call
  {
    const Item it = item_of(a, c);
    if (it.active) {
      const int32_t* table = a.table + static_cast<int64_t>(it.b) * a.table_stride;
      for (int j = tid; j < min(it.kc1 - it.kc0, kItemSlots); j += kThreads) {
        const int key = it.kc0 + j;
        c.key_slot[j] = table[key / a.bs] * a.bs + key % a.bs;
      }
    }
  }
  // partition tables
  for (int kind = 0, off = 0; kind < 4; off += a.ph[kind].U, ++kind) {
    const int U = a.ph[kind].U;
    for (int i = tid; i <= a.C; i += kThreads) c.lo_tab[kind * (kChainMaxCluster + 1) + i] = range_lo(U, a.C, i);
    for (int u = tid; u < U; u += kThreads) c.own_tab[off + u] = static_cast<uint8_t>(owner_of(U, a.C, u));
  }
  if (warp == 5) {
    tmem_alloc(c.tmem_holder, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // every CTA's barriers are initialised before anyone signals them
  tc_fence_after();
  const uint32_t tmem_base = *c.tmem_holder;
  const int C = a.C, rank = static_cast<int>(c.rank);

  if (warp == 4) {
    // ------------------------------------------------------------ weight stream
    if (lane == 0) {
      const uint64_t pol = a.ring_evict_first ? l2_policy_evict_first() : l2_policy_evict_normal();
      uint32_t g = 0;
      bool ok = true;
      for (int l = 0; l < a.n_layers && ok; ++l) {
        for (int kind = 0; kind < 4 && ok; ++kind) {
          const Part pt = part_of(a, c, kind);
          const uint8_t* w = phase_weights(a.layers[l], kind);
          const int u1 = pt.lo[rank + 1];
          for (int u = pt.lo[rank]; u < u1 && ok;) {
            const int s0 = static_cast<int>(g % S);
            const int n = min(min(kRun, u1 - u), S - s0);
            for (int i = 0; i < n && ok; ++i)
              if (g + i >= static_cast<uint32_t>(S))
                ok = lwait(a, c, &c.empty[s0 + i], (((g + i) / S) - 1) & 1);
            if (!ok) break;
            mbar_arrive_expect_tx(&c.full[s0], n * kUnitBytes);
            for (int i = 1; i < n; ++i) mbar_arrive(&c.full[s0 + i]);
            bulk_copy(c.ring + s0 * kUnitBytes, w + static_cast<size_t>(u) * kUnitBytes, n * kUnitBytes, &c.full[s0], pol);
            g += n;
            u += n;
          }
          stamp_at(a, c, l * 5 + (kind == CK_QKV ? 0 : kind == CK_O ? 2 : kind == CK_GU ? 3 : 4), 6);
        }
      }
      // every issued copy has landed before the CTA may exit
      const uint32_t first = g > static_cast<uint32_t>(S) ? g - S : 0;
      for (uint32_t i = first; i < g; ++i) mbar_wait_bounded(&c.full[i % S], (i / S) & 1, a.status, nullptr);
    }
    __syncwarp();
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issue (warp-uniform;
    // one elected lane issues). A ring slot is released by one commit per copy run.
    if (!a.fma) {
      const uint32_t idesc = umma_idesc_bf16(128, kStreamBN);
      uint32_t g = 0, segs = 0, xn_n = 0, xp_n = 0;
      long long cy_acc = 0, cy_issue = 0;
      bool ok = true;
      for (int l = 0; l < a.n_layers && ok; ++l) {
        for (int kind = 0; kind < 4 && ok; ++kind) {
          const Part pt = part_of(a, c, kind);
          const int u0 = pt.lo[rank], u1 = pt.lo[rank + 1];
          const bool norm_x = (kind == CK_QKV || kind == CK_GU);
          ok = norm_x ? lwait_warp(a, c, c.x_full, (xn_n++) & 1) : cwait_warp(a, c, c.xp_full, (xp_n++) & 1);
          if (!ok) break;
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          tc_fence_after();
          const int pidx = l * 5 + (kind == CK_QKV ? 0 : kind == CK_O ? 2 : kind == CK_GU ? 3 : 4);
          if (lane == 0) stamp_at(a, c, pidx, 4);
          const uint8_t* xb = norm_x ? c.xn : c.xp;
          int run_left = 0, run_first = 0, run_n = 0;
          bool first = true;
          uint32_t buf = 0;
          unsigned long long waited = 0;
          for (int u = u0; u < u1 && ok; ++u, ++g) {
            if (run_left == 0) {
              run_first = static_cast<int>(g % S);
              run_n = run_left = min(min(kRun, u1 - u), S - run_first);
              const unsigned long long w0 = a.trace ? now_ns() : 0;
              ok = lwait_warp(a, c, &c.full[run_first], (g / S) & 1);
              if (a.trace) waited += now_ns() - w0;
              if (!ok) break;
              tc_fence_after();
            }
            --run_left;
            const long long q0 = clock64();
            if (first) {
              buf = segs & 1;
              if (segs >= 2) {
                ok = lwait_warp(a, c, &c.acc_empty[buf], ((segs >> 1) - 1) & 1);
                if (!ok) break;
              }
              tc_fence_after();
            }
            const long long q1 = clock64();
            cy_acc += q1 - q0;
            const int st = static_cast<int>(g % S);
            const uint64_t da = umma_desc_sw128(smem_u32(c.ring + st * kUnitBytes));
            const uint64_t db = umma_desc_sw128(smem_u32(xb + (u - u0) * 1024));
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_bf16_elect(tmem_base + buf * kStreamBN, da + kk * 2, db + kk * 2, idesc, (first && kk == 0) ? 0u : 1u);
            if (run_left == 0)  // the run's slots are free once its MMAs complete
              for (int i = 0; i < run_n; ++i) umma_commit_elect(&c.empty[run_first + i]);
            if (u + 1 == u1 || (u + 1) % pt.kb == 0) {
              umma_commit_elect(&c.acc_full[buf]);
              ++segs;
              first = true;
            } else {
              first = false;
            }
            cy_issue += clock64() - q1;
          }
          if (lane == 0) {
            stamp_at(a, c, pidx, 5);
            trace_put(a, c, pidx, 11, waited);
            trace_put(a, c, pidx, 8, static_cast<unsigned long long>(cy_acc));
            trace_put(a, c, pidx, 9, static_cast<unsigned long long>(cy_issue));
          }
          cy_acc = cy_issue = 0;
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ compute warps 0-3
    Counters k = {};
    bool ok = true;
    // h = embed rows, written by the owners of the O / down output tiles
    {
      const Part pt = part_of(a, c, CK_DOWN);
      const int u1 = pt.lo[rank + 1];
      for (int t = pt.first_tile(rank); t * pt.kb < u1; ++t) {
        const int n = t * 128 + tid;
        if (n < a.H)
          for (int m = 0; m < a.M; ++m)
            a.h[static_cast<size_t>(m) * a.H + n] = a.embed[static_cast<int64_t>(c.ids[m]) * a.H + n];
        signal_h(a, c);
      }
    }
    for (int l = 0; l < a.n_layers && ok; ++l) {
      stamp(a, c, l * 5 + 0, 0);
      attn_prefetch(a, c, l);
      ok = gemm_phase(a, c, tmem_base, CK_QKV, l, k);
      stamp(a, c, l * 5 + 0, 3);
      if (!ok) break;
      stamp(a, c, l * 5 + 1, 0);
      const long long ck0 = clock64();
      ok = attention_phase(a, c, l, k);
      stamp(a, c, l * 5 + 1, 3);
      if (tid == 0) trace_put(a, c, l * 5 + 1, 14, static_cast<unsigned long long>(clock64() - ck0));
      if (!ok) break;
      stamp(a, c, l * 5 + 2, 0);
      ok = gemm_phase(a, c, tmem_base, CK_O, l, k);
      stamp(a, c, l * 5 + 2, 3);
      if (!ok) break;
      stamp(a, c, l * 5 + 3, 0);
      ok = gemm_phase(a, c, tmem_base, CK_GU, l, k);
      stamp(a, c, l * 5 + 3, 3);
      if (!ok) break;
      stamp(a, c, l * 5 + 4, 0);
      ok = gemm_phase(a, c, tmem_base, CK_DOWN, l, k);
      stamp(a, c, l * 5 + 4, 3);
    }
    cp_async_wait<0>();  // no K/V prefetch left in flight when leaving early
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 32);
  }
  cluster_sync_all();  // no CTA leaves while a peer may still write to its shared memory
}

}  // namespace

// ---------------------------------------------------------------- host side
int chain_cluster_size() {
  static int C = -1;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (C >= 0) return C;
  C = 0;
  if (cudaFuncSetAttribute(chain_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess ||
      cudaFuncSetAttribute(chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess) {
    cudaGetLastError();
    return C;
  }
  for (int cs : {16, 8}) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cs);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = 227 * 1024;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = cs;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, chain_kernel, &cfg) == cudaSuccess && n >= 1) {
      C = cs;
      break;
    }
    cudaGetLastError();
  }
  return C;
}

bool chain_plan(int n_layers, int H, int Hq, int Hkv, int D, int I, int B, int T, int C, ChainPhase ph[4], int* splits,
                ChainLayout* L) {
  const int M = B * T;
  if (C <= 0 || D != 64 || M > kChainMaxRows || T > 8 || H % 64 || H > 1024 || I % 64 || Hq % Hkv) return false;
  if (n_layers > kStreamMaxLayers) return false;
  const int G = Hq / Hkv, R = T * G;
  if (R > kAmRows) return false;
  const int Ns[4] = {(Hq + 2 * Hkv) * D, H, 2 * I, H};
  const int Ks[4] = {H, Hq * D, H, I};
  int max_units[2] = {0, 0}, own[2] = {0, 0}, nc[2] = {0, 0};
  for (int kind = 0; kind < 4; ++kind) {
    ChainPhase& P = ph[kind];
    P.N = Ns[kind];
    P.K = Ks[kind];
    if (P.K % 64) return false;
    P.n_tiles = (P.N + 127) / 128;
    P.kb = P.K / 64;
    P.U = P.n_tiles * P.kb;
    if (P.U < C) return false;
    const int region = (kind == CK_QKV || kind == CK_GU) ? 0 : 1;
    for (int c = 0; c < C; ++c) {
      const int u0 = range_lo(P.U, C, c), u1 = range_lo(P.U, C, c + 1);
      max_units[region] = std::max(max_units[region], u1 - u0);
      int owned = 0;
      for (int t = first_owned_tile(P, C, c); t * P.kb < u1; ++t) ++owned;
      own[region] = std::max(own[region], owned);
    }
    for (int t = 0; t < P.n_tiles; ++t) nc[region] = std::max(nc[region], contributors(P, C, t));
  }
  if (ph[CK_O].n_tiles != ph[CK_DOWN].n_tiles) return false;
  if (max_units[0] > 32 || max_units[1] > 32 || own[0] > kChainOwnMax || own[1] > kChainOwnMax ||
      nc[0] > kChainContribMax || nc[1] > kChainContribMax)
    return false;
  int S = std::min(kChainMaxSplits, C / (B * Hkv));
  if (S < 1) return false;
  *splits = S;
  auto al = [](int x, int a) { return (x + a - 1) / a * a; };
  ChainLayout l = {};
  l.ownA = own[0];
  l.ncA = nc[0];
  l.ownB = own[1];
  l.ncB = nc[1];
  const int xn = (max_units[0] + 1) * 1024;
  const int x32 = M <= kChainFmaRows ? std::max(max_units[0], max_units[1]) * M * 64 * 4 : 0;
  const int kvring = kKvBlocks * 8192;  // also the attention merge scratch (4 x (16 x 64 + 32) floats)
  static_assert(kKvBlocks * 8192 >= 4 * (16 * 64 + 32) * 4, "merge scratch fits the K/V ring");
  const int xp = (max_units[1] + 1) * 1024;
  const int pa = al(own[0] * nc[0] * M * 512, 128);
  const int pb = al(own[1] * nc[1] * M * 512, 128);
  const int comb = al((S - 1) * comb_stride(R) * 4, 128);
  const int ostage = al((16 * 64 + 32) * 4, 128);
  const int tile = al(kChainMaxRows * kTP * 4, 128);
  const int stage = 2048;
  const int misc = al(kMiscBytes, 128);
  int sumU = 0;
  for (int kind = 0; kind < 4; ++kind) sumU += ph[kind].U;
  if (sumU > 8192 || C > kChainMaxCluster) return false;
  const int part = al(4 * (kChainMaxCluster + 1) * 4 + sumU, 128);
  const int keyslot = kItemSlots * 4;
  const int others = part + keyslot + xn + xp + al(x32, 128) + kvring + pa + pb + 2048 + 2048 + comb + ostage + tile + stage + misc;
  const int budget = 227 * 1024 - 1024;
  const int slots = std::min(kChainMaxSlots, (budget - others) / static_cast<int>(kUnitBytes));
  if (slots < 4) return false;
  l.ring_slots = slots;
  int off = slots * static_cast<int>(kUnitBytes);
  l.xn = off; off += xn;
  l.xp = off; off += xp;
  l.part = off; off += part;
  l.keyslot = off; off += keyslot;
  l.x32 = off; off += al(x32, 128);
  l.kvring = off; off += kvring;
  l.pa = off; off += pa;
  l.pb = off; off += pb;
  l.qrecv = off; off += 2048;
  l.kvrecv = off; off += 2048;
  l.comb = off; off += comb;
  l.ostage = off; off += ostage;
  l.tile = off; off += tile;
  l.stage = off; off += stage;
  l.misc = off; off += misc;
  l.total = off;
  *L = l;
  return true;
}

int launch_chain(const ChainArgs& a, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.C);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = a.L.total + 1024;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = a.C;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, chain_kernel, a) == cudaSuccess ? SPECB200_OK : SPECB200_ERR_CUDA;
}

}  // namespace specb200
