// Decode / verify attention (bf16, d = 64, at most 16 query rows per KV head) as one
// thread-block cluster per (sequence, KV head): the same computation and mask as
// attention_item_mma (the reference's SDPA over the gathered cache, lm/forward.py:44-49,62-63),
// organised for the latency of one decode step.
//
// - The cluster's C CTAs split the key range into contiguous chunks of at most
//   kAcMaxChunk keys, and each CTA holds its whole chunk of K and V in shared memory.
// - The cached keys (positions < past) were written before the forward call started (its
//   first kernel launches without programmatic overlap), so they are loaded BEFORE
//   griddepcontrol.wait; only the query rows and this call's new keys wait for the q/k/v
//   projection.
// - 8 warps each run 8-key mma.sync steps (attn_mma.cuh) over their share of the chunk. The
//   warps merge in shared memory, and the CTAs merge through distributed shared memory into
//   the cluster's first CTA. There are no global partials, tickets or second round trips.
#pragma once
#include "attn_core.cuh"
#include "attn_mma.cuh"

namespace specb200 {

constexpr int kAcThreads = 256;  // two CTAs per SM, so a batch-1 verify's clusters fit one wave
constexpr int kAcWarps = kAcThreads / 32;
constexpr int kAcMaxCluster = 8;
constexpr int kAcMaxChunk = 512;  // keys per CTA
constexpr int kAcRowsMax = 16;

// Dynamic shared memory of the cluster kernel for chunk keys per CTA, R query rows and C CTAs.
struct AcLayout {
  int kv, scratch, slots, tab, total;  // byte offsets (q rows at 0), total size
};
__host__ __device__ inline AcLayout ac_layout(int chunk, int R, int C, int bs) {
  AcLayout L;
  const int region = chunk * 256 > kAcWarps * (R * 64 + 32) * 4 ? chunk * 256 : kAcWarps * (R * 64 + 32) * 4;
  L.kv = 2048;
  L.scratch = L.kv;  // the K / V region is reused by the warp merge once the products are done
  L.slots = L.kv + ((region + 127) / 128) * 128;
  L.tab = L.slots + C * (R * 64 + 32) * 4;
  L.total = L.tab + ((chunk + bs - 1) / bs + 2) * 4 + 128;
  return L;
}

SPECB200_DEVINL uint32_t ac_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
SPECB200_DEVINL uint32_t ac_mapa(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
SPECB200_DEVINL void ac_st_remote(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
SPECB200_DEVINL void ac_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Split cluster barrier: arrive when the CTA starts, wait before its first remote store, so
// that every CTA of the cluster is known to be running when its memory is written.
SPECB200_DEVINL void ac_cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory"); }
SPECB200_DEVINL void ac_cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

// Merge of the warps' states into rows 0..R-1: out_o [R][64] (relative to out_m, base 2),
// out_m [R], out_l [R]; scratch holds kAcWarps * (R * 64 + 32) floats. Ends with __syncthreads.
SPECB200_DEVINL void ac_merge_warps(const AmState& st, float* scratch, int R, float* out_o, float* out_m, float* out_l) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tig = lane & 3;
  const int stride = R * 64 + 32;
  float* wo = scratch + warp * stride;
  float* wm = wo + R * 64;
  float* wl = wm + 16;
  float l0 = st.l[0], l1 = st.l[1];
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    const int c = nt * 8 + 2 * tig;
    if (g < R) {
      wo[g * 64 + c] = st.o[nt][0];
      wo[g * 64 + c + 1] = st.o[nt][1];
    }
    if (g + 8 < R) {
      wo[(g + 8) * 64 + c] = st.o[nt][2];
      wo[(g + 8) * 64 + c + 1] = st.o[nt][3];
    }
  }
  if (tig == 0) {
    wm[g] = st.m[0];
    wm[g + 8] = st.m[1];
    wl[g] = l0;
    wl[g + 8] = l1;
  }
  __syncthreads();
  for (int i = tid; i < R * 64; i += kAcThreads) {
    const int r = i >> 6, c = i & 63;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAcWarps; ++w) M = fmaxf(M, scratch[w * stride + R * 64 + r]);
    float O = 0.f, L = 0.f;
#pragma unroll
    for (int w = 0; w < kAcWarps; ++w) {
      const float* b = scratch + w * stride;
      const float mw = b[R * 64 + r];
      const float wgt = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
      O = fmaf(b[r * 64 + c], wgt, O);
      L = fmaf(b[R * 64 + 16 + r], wgt, L);
    }
    out_o[i] = O;
    if (c == 0) {
      out_m[r] = M;
      out_l[r] = L;
    }
  }
  __syncthreads();
}

// One CTA of the cluster for (sequence b, KV head g): keys [rank * chunk, ...) of the row.
// With `pdl` the cached keys are loaded before griddepcontrol.wait.
static __device__ void attention_cluster_cta(const AttnKernelArgs& ka, int b, int g, uint8_t* smem, bool pdl) {
  const AttnArgs& a = ka.a;
  constexpr int D = 64;
  const int C = ka.p.splits_max, chunk = ka.p.chunk;
  const int G = a.Hq / a.Hkv;
  const int R = a.T * G;
  const int rank = static_cast<int>(ac_rank());
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const AcLayout lay = ac_layout(chunk, R, C, a.bs);
  unsigned long long* tr = nullptr;  // optional record (AttnArgs::trace), thread 0
  if (a.trace && tid == 0) {
    const unsigned cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
    if (cta < kAttnTraceCtas) tr = a.trace + (static_cast<size_t>(a.trace_slot) * kAttnTraceCtas + cta) * 8;
  }
  auto stamp = [&](int k) {
    if (tr) {
      unsigned long long t;
      asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
      tr[k] = t;
    }
  };
  stamp(0);
  const int past = a.past[b], nn = a.n_new[b], total = past + nn;
  if (nn <= 0) return;  // the same for every CTA of the cluster: none of them synchronises
  ac_cluster_arrive_relaxed();
  const int kmax = min(total, past + (R - 1) / G + 1);
  const int kbeg = min(kmax, rank * chunk);
  const int kend = min(kmax, kbeg + chunk);
  __nv_bfloat16* q_s = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* k_s = reinterpret_cast<__nv_bfloat16*>(smem + lay.kv);
  __nv_bfloat16* v_s = k_s + chunk * 64;
  int* tab = reinterpret_cast<int*>(smem + lay.tab);
  const __nv_bfloat16* kp = static_cast<const __nv_bfloat16*>(a.k_pool);
  const __nv_bfloat16* vp = static_cast<const __nv_bfloat16*>(a.v_pool);
  const int32_t* table = a.table + static_cast<int64_t>(b) * a.table_stride;
  const int ngrp = (kend - kbeg + 7) / 8;  // 8-key groups of this CTA

  // block-table entries of the chunk, then keys [lo, hi) by cp.async; rows up to the next
  // multiple of 8 past kend are zero (masked in the scores, and 0 * V must stay finite)
  const int tb0 = kbeg / a.bs;
  const int ntab = kend > kbeg ? (kend - 1) / a.bs - tb0 + 1 : 0;
  for (int i = tid; i < ntab; i += kAcThreads) tab[i] = table[tb0 + i];
  __syncthreads();
  auto load_keys = [&](int lo, int hi) {
    for (int idx = tid; idx < (hi - lo) * 16; idx += kAcThreads) {
      const int key = lo + (idx >> 4), part = idx & 15, isv = part >> 3, cc = part & 7;
      const int r = key - kbeg;
      const int64_t sl = static_cast<int64_t>(tab[key / a.bs - tb0]) * a.bs + key % a.bs;
      cp_async_16((isv ? v_s : k_s) + am_swz(r, cc * 8), (isv ? vp : kp) + (sl * a.Hkv + g) * D + cc * 8);
    }
  };
  const int split_at = max(kbeg, min(kend, past));
  load_keys(kbeg, split_at);
  cp_async_commit();
  for (int idx = tid; idx < (ngrp * 8 - (kend - kbeg)) * 16; idx += kAcThreads) {
    const int r = (kend - kbeg) + (idx >> 4), part = idx & 15, isv = part >> 3, cc = part & 7;
    *reinterpret_cast<uint4*>((isv ? v_s : k_s) + am_swz(r, cc * 8)) = make_uint4(0, 0, 0, 0);
  }
  if (pdl) pdl_wait();
  stamp(1);
  // query rows (zero past R) and this call's keys
  const __nv_bfloat16* q = static_cast<const __nv_bfloat16*>(a.q);
  for (int i = tid; i < 16 * 8; i += kAcThreads) {
    const int r = i >> 3, c8 = i & 7;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < R) {
      const int t = r / G, h = g * G + r % G;
      v = *reinterpret_cast<const uint4*>(q + (static_cast<int64_t>(b * a.T + t) * a.Hq + h) * D + c8 * 8);
    }
    *reinterpret_cast<uint4*>(q_s + am_swz(r, c8 * 8)) = v;
  }
  load_keys(split_at, kend);
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  stamp(2);

  AmState st;
  am_init(st, q_s);
  const int r0 = lane >> 2, r1 = r0 + 8;
  const int lim0 = r0 < R ? min(past + r0 / G + 1, total) : 0;
  const int lim1 = r1 < R ? min(past + r1 / G + 1, total) : 0;
  for (int j = warp; j < ngrp; j += kAcWarps) {
    const int kabs = kbeg + 8 * j;
    am_step(st, k_s, v_s, 8 * j, kabs, min(8, kend - kabs), lim0, lim1, a.scale);
  }
  __syncthreads();  // K / V region becomes the merge scratch
  stamp(3);
  float* scratch = reinterpret_cast<float*>(smem + lay.scratch);
  float* slots = reinterpret_cast<float*>(smem + lay.slots);  // [C][R * 64 + 32] in the first CTA
  // This CTA's merged partial, [R][64] o then m at R * 64 and l at R * 64 + 16: built in its
  // own slot `rank`, then (other CTAs) copied to the same slot of the first CTA.
  const int slot_floats = R * 64 + 32;
  float* mo = slots + rank * slot_floats;
  ac_merge_warps(st, scratch, R, mo, mo + R * 64, mo + R * 64 + 16);
  stamp(4);
  ac_cluster_wait();
  if (rank != 0) {
    const uint32_t dst = ac_mapa(smem_u32(slots + rank * slot_floats), 0);
    for (int i = tid; i < slot_floats; i += kAcThreads) ac_st_remote(dst + 4 * i, mo[i]);
  }
  ac_cluster_sync();
  stamp(5);
  if (rank != 0) return;
  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out);
  for (int i = tid; i < R * D; i += kAcThreads) {
    const int r = i >> 6, c = i & 63;
    float M = -INFINITY;
    for (int cr = 0; cr < C; ++cr) M = fmaxf(M, slots[cr * slot_floats + R * 64 + r]);
    float O = 0.f, L = 0.f;
    for (int cr = 0; cr < C; ++cr) {
      const float* sp = slots + cr * slot_floats;
      const float ms = sp[R * 64 + r];
      const float w = (ms == -INFINITY) ? 0.f : exp2f(ms - M);
      O = fmaf(sp[i], w, O);
      L = fmaf(sp[R * 64 + 16 + r], w, L);
    }
    const int t = r / G, h = g * G + r % G;
    out[(static_cast<int64_t>(b * a.T + t) * a.Hq + h) * D + c] = __float2bfloat16_rn(O / L);
  }
  stamp(6);
}

// Cluster plan: C = ceil(max_kv_len / 64) CTAs (at most kAcMaxCluster), chunk a multiple of 8.
// Returns false when the keys do not fit C * kAcMaxChunk.
inline bool plan_attention_cluster(int max_kv_len, AttnPlan* p) {
  const int len = max_kv_len < 1 ? 1 : max_kv_len;
  int C = (len + 63) / 64;
  C = C > kAcMaxCluster ? kAcMaxCluster : C;
  const int chunk = ((len + C - 1) / C + 7) / 8 * 8;
  if (chunk > kAcMaxChunk) return false;
  p->qtiles = 1;
  p->splits_max = C;
  p->chunk = chunk;
  p->mma = 2;
  return true;
}

}  // namespace specb200
