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
constexpr int kQkvMaxSplits = 4;  // q/k/v partials summed by the attention (AttnArgs::qkv_parts)

// Dynamic shared memory of the cluster kernel for chunk keys per CTA, R query rows and S merge
// slots (CTAs per head).
struct AcLayout {
  int kv, scratch, slots, tab, bar, total;  // byte offsets (q rows at 0), total size
};
__host__ __device__ inline AcLayout ac_layout(int chunk, int R, int S, int bs) {
  AcLayout L;
  const int region = chunk * 256 > kAcWarps * (R * 64 + 32) * 4 ? chunk * 256 : kAcWarps * (R * 64 + 32) * 4;
  L.kv = 2048;
  L.scratch = L.kv;  // the K / V region is reused by the warp merge once the products are done
  L.slots = L.kv + ((region + 127) / 128) * 128;
  L.tab = L.slots + S * (R * 64 + 32) * 4;
  L.bar = L.tab + (((chunk + bs - 1) / bs + 2) * 4 + 127) / 128 * 128;
  L.total = L.bar + 16 + 128;
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

// 8 bf16 values of a 16-byte chunk as fp32 (exact), and back with round-to-nearest-even.
SPECB200_DEVINL void ac_unpack8(const uint4& v, float (&f)[8]) {
  const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(u[i] << 16);
    f[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
  }
}
SPECB200_DEVINL uint4 ac_pack8(const float (&f)[8]) {
  uint32_t u[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    u[i] = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(f[2 * i]))) |
           (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(f[2 * i + 1]))) << 16);
  return make_uint4(u[0], u[1], u[2], u[3]);
}

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

// One CTA of the cluster for (sequence b, KV head g): keys [rank * chunk, ...) of the row; the
// cluster's first CTA writes the output. With `pdl` the cached keys are loaded before
// griddepcontrol.wait.
static __device__ void attention_cluster_cta(const AttnKernelArgs& ka, int b, int g, uint8_t* smem, bool pdl) {
  const AttnArgs& a = ka.a;
  constexpr int D = 64;
  const int chunk = ka.p.chunk;
  const int G = a.Hq / a.Hkv;
  const int R = a.T * G;
  const int part = static_cast<int>(ac_rank());
  const int P = ka.p.splits_max;  // CTAs per KV head
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const AcLayout lay = ac_layout(chunk, R, P, a.bs);
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
  const int kbeg = min(kmax, part * chunk);
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
    // one task per (key, K or V, row half): one slot lookup per four 16-byte copies
    for (int idx = tid; idx < (hi - lo) * 4; idx += kAcThreads) {
      const int key = lo + (idx >> 2), isv = (idx >> 1) & 1, c0 = (idx & 1) * 4;
      const int r = key - kbeg;
      const int64_t sl = static_cast<int64_t>(tab[key / a.bs - tb0]) * a.bs + key % a.bs;
      const __nv_bfloat16* src = (isv ? vp : kp) + (sl * a.Hkv + g) * D;
      __nv_bfloat16* dst = isv ? v_s : k_s;
#pragma unroll
      for (int cc = c0; cc < c0 + 4; ++cc) cp_async_16(dst + am_swz(r, cc * 8), src + cc * 8);
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
  if (a.qkv_parts) {
    // q rows and the new keys / values from the q/k/v GEMM's partials: pair (c, c + 32) of a
    // head, summed over splits in order, rounded, rotated (q and k) as EPI_QKV does. Two pairs
    // per thread per pass with every partial load of the pass in flight together.
    using T16 = __nv_bfloat16;
    const int qd = a.Hq * D, kd = a.Hkv * D;
    const int nq = R * 32;        // (query row, pair)
    const int nkv = a.T * 2 * 32;  // (new token, k or v, pair)
    for (int i = tid; i < (16 - R) * 64; i += kAcThreads)  // query rows past R are zero
      q_s[am_swz(R + i / 64, i % 64)] = __float2bfloat16_rn(0.f);
    for (int i0 = 0; i0 < nq + nkv; i0 += 2 * kAcThreads) {
      int col[2], t[2], c[2], r[2];
      bool live[2], isq[2], isv[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int i = i0 + u * kAcThreads + tid;
        live[u] = i < nq + nkv;
        isq[u] = i < nq;
        isv[u] = false;
        r[u] = 0;
        if (isq[u]) {
          r[u] = i >> 5;
          c[u] = i & 31;
          t[u] = r[u] / G;
          col[u] = (g * G + r[u] % G) * D + c[u];
        } else {
          const int k = i - nq;
          t[u] = k >> 6;
          isv[u] = (k >> 5) & 1;
          c[u] = k & 31;
          col[u] = (isv[u] ? qd + kd : qd) + g * D + c[u];
          live[u] = live[u] && t[u] < nn;  // padding tokens have no key
        }
      }
      float v[kQkvMaxSplits][2][2];
#pragma unroll
      for (int sp = 0; sp < kQkvMaxSplits; ++sp)
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          v[sp][u][0] = v[sp][u][1] = 0.f;
          if (sp < a.qkv_splits && live[u]) {
            const float* row =
                a.qkv_parts + (static_cast<int64_t>(sp) * a.B * a.T + static_cast<int64_t>(b) * a.T + t[u]) * a.qkv_n;
            v[sp][u][0] = __ldcg(row + col[u]);
            v[sp][u][1] = __ldcg(row + col[u] + 32);
          }
        }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (!live[u]) continue;
        float lo = 0.f, hi = 0.f;
#pragma unroll
        for (int sp = 0; sp < kQkvMaxSplits; ++sp)
          if (sp < a.qkv_splits) {
            lo += v[sp][u][0];
            hi += v[sp][u][1];
          }
        lo = round_to<T16>(lo);
        hi = round_to<T16>(hi);
        if (!isv[u]) {  // q and k rotate
          const int pos = min(past + t[u], a.max_positions - 1);
          const float cs = round_to<T16>(a.rope_cos[static_cast<int64_t>(pos) * 32 + c[u]]);
          const float sn = round_to<T16>(a.rope_sin[static_cast<int64_t>(pos) * 32 + c[u]]);
          const float lo2 = round_to<T16>(round_to<T16>(lo * cs) + round_to<T16>(-hi * sn));
          const float hi2 = round_to<T16>(round_to<T16>(hi * cs) + round_to<T16>(lo * sn));
          lo = lo2;
          hi = hi2;
        }
        if (isq[u]) {
          q_s[am_swz(r[u], c[u])] = __float2bfloat16_rn(lo);
          q_s[am_swz(r[u], c[u] + 32)] = __float2bfloat16_rn(hi);
          continue;
        }
        const int kk = past + t[u];  // key index of the new token
        if (kk >= kbeg && kk < kend) {
          __nv_bfloat16* dst = isv[u] ? v_s : k_s;
          dst[am_swz(kk - kbeg, c[u])] = __float2bfloat16_rn(lo);
          dst[am_swz(kk - kbeg, c[u] + 32)] = __float2bfloat16_rn(hi);
        }
        if (part == 0) {  // the new key / value into the pool, once per cluster
          const int64_t sl = static_cast<int64_t>(table[kk / a.bs]) * a.bs + kk % a.bs;
          __nv_bfloat16* pool = const_cast<__nv_bfloat16*>(isv[u] ? vp : kp) + (sl * a.Hkv + g) * D;
          pool[c[u]] = __float2bfloat16_rn(lo);
          pool[c[u] + 32] = __float2bfloat16_rn(hi);
        }
      }
    }
  } else {
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
  }
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
  // own slot `part`, then (other CTAs) copied to the same slot of the head's first CTA.
  const int slot_floats = R * 64 + 32;
  float* mo = slots + part * slot_floats;
  ac_merge_warps(st, scratch, R, mo, mo + R * 64, mo + R * 64 + 16);
  stamp(4);
  ac_cluster_wait();
  if (part != 0) {
    const uint32_t dst = ac_mapa(smem_u32(slots + part * slot_floats), 0);
    for (int i = tid; i < slot_floats; i += kAcThreads) ac_st_remote(dst + 4 * i, mo[i]);
  }
  ac_cluster_sync();
  stamp(5);
  if (part == 0) {
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out);
    for (int i = tid; i < R * D; i += kAcThreads) {
      const int r = i >> 6, c = i & 63;
      float M = -INFINITY;
      for (int cr = 0; cr < P; ++cr) M = fmaxf(M, slots[cr * slot_floats + R * 64 + r]);
      float O = 0.f, L = 0.f;
      for (int cr = 0; cr < P; ++cr) {
        const float* sp = slots + cr * slot_floats;
        const float ms = sp[R * 64 + r];
        const float w = (ms == -INFINITY) ? 0.f : exp2f(ms - M);
        O = fmaf(sp[i], w, O);
        L = fmaf(sp[R * 64 + 16 + r], w, L);
      }
      const int t = r / G, h = g * G + r % G;
      out[(static_cast<int64_t>(b * a.T + t) * a.Hq + h) * D + c] = __float2bfloat16_rn(O / L);
    }
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
