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
constexpr int kAcQkvChunks = 2;   // fused projection: 16-byte input chunks per thread (H <= 4096)
constexpr int kAcQkvMaxT = 4;     // fused projection: token rows per sequence

// The o projection fused behind the attention (decode steps of small models): one cluster per
// sequence covers every KV head (P CTAs per head); after the heads' merges every CTA holds the
// whole attention output and computes `rows` rows of o = W_o attn with the residual add.
struct FuseO {
  const __nv_bfloat16* w;  // [H, Hq d] row-major
  __nv_bfloat16* hidden;   // residual stream [B T, H]
  int H;
  int P;     // CTAs per KV head
  int rows;  // o rows per CTA
};

// The q/k/v projection fused in front of the attention (decode steps of small models; the
// reference's input RMSNorm, q/k/v linears, RoPE and cache.write, lm/forward.py:55-60): the
// cluster of KV head g computes that head's rows of Y = RMSNorm(x) W_qkv^T itself. The head's
// (G + 2) * 32 rotary pairs (G query heads, the key head, the value head; pair c of a head is
// rows c and c + 32) are split into runs of `pairs` between the cluster's CTAs; each CTA brings
// its weight rows on chip by bulk copies issued before griddepcontrol.wait, normalises the
// input rows, computes its pairs, rotates them and sends each value where the attention reads
// it: q to every CTA, a new key or value to the CTA whose chunk holds its position (and to the
// pool), through distributed shared memory.
struct FuseQKV {
  const __nv_bfloat16* w;       // [Hq d + 2 Hkv d, H] q/k/v weight rows
  const __nv_bfloat16* x;       // residual stream [B T, H]
  const __nv_bfloat16* norm_w;  // [H] RMSNorm weight in front of the projection
  const int32_t* slot;          // [B T] pool slot of each token row, -1 for padding rows
  float eps;
  int H;
  int pairs;  // rotary pairs per CTA
};

// Regions of the fused projection, after the attention's own layout (`base` bytes): weight
// rows [2 pairs][H] bf16 (the pairs' first rows, then their second rows), the normalised
// input [T][H] bf16, the rounded products [T][2 pairs] fp32, the norm's warp sums and the
// weights' mbarrier.
struct AcQkvLayout {
  int w, x, res, red, bar, total;
};
__host__ __device__ inline AcQkvLayout ac_qkv_layout(int base, int T, int H, int pairs) {
  AcQkvLayout q;
  q.w = (base + 127) / 128 * 128;
  q.x = q.w + 2 * pairs * H * 2;
  q.res = q.x + (T * H * 2 + 15) / 16 * 16;
  q.red = q.res + T * 2 * pairs * 4;
  q.bar = (q.red + kAcWarps * 4 * 4 + 7) / 8 * 8;
  q.total = q.bar + 8;
  return q;
}

// Dynamic shared memory of the cluster kernel for chunk keys per CTA, R query rows, S merge
// slots (CTAs per head) and, when fused, T tokens of Hq heads and `orows` o rows of K = Hq d.
struct AcLayout {
  int kv, scratch, slots, tab, attn, wo, bar, total;  // byte offsets (q rows at 0), total size
};
__host__ __device__ inline AcLayout ac_layout(int chunk, int R, int S, int bs, int T = 0, int Hq = 0, int orows = 0) {
  AcLayout L;
  const int region = chunk * 256 > kAcWarps * (R * 64 + 32) * 4 ? chunk * 256 : kAcWarps * (R * 64 + 32) * 4;
  L.kv = 2048;
  L.scratch = L.kv;  // the K / V region is reused by the warp merge once the products are done
  L.slots = L.kv + ((region + 127) / 128) * 128;
  L.tab = L.slots + S * (R * 64 + 32) * 4;
  L.attn = L.tab + (((chunk + bs - 1) / bs + 2) * 4 + 127) / 128 * 128;
  L.wo = L.attn + (T * Hq * 64 * 2 + 127) / 128 * 128;
  L.bar = L.wo + orows * Hq * 64 * 2;
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

// One CTA of the cluster for (sequence b, KV head g): keys [part * chunk, ...) of the row. Without
// `fo` the cluster is one KV head (part = rank) and its first CTA writes the output; with `fo`
// the cluster is every KV head of the sequence (g = rank / P, part = rank % P), each head's first
// CTA sends the head's output to every CTA, and each CTA computes its o rows.
// With `pdl` the cached keys (and the o or q/k/v weights) are loaded before griddepcontrol.wait.
// With `fq` (never together with `fo`) the cluster computes its own q and new keys / values.
static __device__ void attention_cluster_cta(const AttnKernelArgs& ka, int b, int g, uint8_t* smem, bool pdl,
                                             const FuseO* fo = nullptr, const FuseQKV* fq = nullptr) {
  const AttnArgs& a = ka.a;
  constexpr int D = 64;
  const int chunk = ka.p.chunk;
  const int G = a.Hq / a.Hkv;
  const int R = a.T * G;
  const int rank = static_cast<int>(ac_rank());
  const int P = fo ? fo->P : ka.p.splits_max;  // CTAs per KV head
  if (fo) g = rank / P;
  const int part = fo ? rank % P : rank;
  const int lead = rank - part;  // the head's first CTA
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = a.Hq * D;  // o projection inputs
  const AcLayout lay = fo ? ac_layout(chunk, R, P, a.bs, a.T, a.Hq, fo->rows) : ac_layout(chunk, R, P, a.bs);
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
  // fused o projection: this CTA's weight rows [o0, o1) by one bulk copy, before the wait
  const int o0 = fo ? min(fo->H, rank * fo->rows) : 0, o1 = fo ? min(fo->H, o0 + fo->rows) : 0;
  uint64_t* obar = reinterpret_cast<uint64_t*>(smem + lay.bar);
  __nv_bfloat16* wo_s = reinterpret_cast<__nv_bfloat16*>(smem + lay.wo);
  __nv_bfloat16* attn_s = reinterpret_cast<__nv_bfloat16*>(smem + lay.attn);  // [T][Hq d]
  if (fo && tid == 0) {
    mbar_init(obar, 1);
    fence_mbar_init();
    if (o1 > o0) {
      const uint32_t bytes = static_cast<uint32_t>(o1 - o0) * K * 2;
      mbar_arrive_expect_tx(obar, bytes);
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                       smem_u32(wo_s)),
                   "l"(reinterpret_cast<uint64_t>(fo->w + static_cast<int64_t>(o0) * K)), "r"(bytes), "r"(smem_u32(obar))
                   : "memory");
    } else {
      mbar_arrive(obar);
    }
  }
  // fused q/k/v projection: this CTA's pairs [p0, p1) of the head's (G + 2) * 32, their weight
  // rows by bulk copies (one per run of first rows and one per run of second rows within each
  // head), and the norm weight into registers, all before the wait
  const AcQkvLayout ql = fq ? ac_qkv_layout(lay.total, a.T, fq->H, fq->pairs) : AcQkvLayout{};
  const int npairs_all = (G + 2) * 32;
  const int p0 = fq ? min(npairs_all, part * fq->pairs) : 0;
  const int np = fq ? min(npairs_all, p0 + fq->pairs) - p0 : 0;
  uint64_t* wbar = reinterpret_cast<uint64_t*>(smem + ql.bar);
  __nv_bfloat16* w_s = reinterpret_cast<__nv_bfloat16*>(smem + ql.w);
  uint4 nw[kAcQkvChunks];
  if (fq) {
    const int Hf = fq->H;
    if (tid == 0) {
      mbar_init(wbar, 1);
      fence_mbar_init();
      mbar_arrive_expect_tx(wbar, static_cast<uint32_t>(2 * np) * Hf * 2);
      for (int s0 = p0; s0 < p0 + np;) {  // one run per head
        const int hh = s0 / 32, s1 = min(p0 + np, (hh + 1) * 32), c0 = s0 % 32;
        const int base = hh < G ? (g * G + hh) * D : (hh == G ? a.Hq * D + g * D : (a.Hq + a.Hkv) * D + g * D);
        const uint32_t bytes = static_cast<uint32_t>(s1 - s0) * Hf * 2;
        const __nv_bfloat16* src = fq->w + static_cast<int64_t>(base + c0) * Hf;
        for (int half = 0; half < 2; ++half)
          asm volatile(
              "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                  smem_u32(w_s + static_cast<int64_t>(half * np + s0 - p0) * Hf)),
              "l"(reinterpret_cast<uint64_t>(src + static_cast<int64_t>(half * 32) * Hf)), "r"(bytes),
              "r"(smem_u32(wbar))
              : "memory");
        s0 = s1;
      }
    }
#pragma unroll
    for (int i = 0; i < kAcQkvChunks; ++i) {
      const int ch = tid + i * kAcThreads;
      nw[i] = ch * 8 < Hf ? __ldg(reinterpret_cast<const uint4*>(fq->norm_w) + ch) : make_uint4(0, 0, 0, 0);
    }
  }
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
  if (fq) {
    using T16 = __nv_bfloat16;
    const int Hf = fq->H, nch = Hf >> 3, Tn = a.T;
    __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem + ql.x);  // [T][H]
    float* red = reinterpret_cast<float*>(smem + ql.red);               // [warp][4]
    float* res = reinterpret_cast<float*>(smem + ql.res);               // [T][2 np]
    // input rows, RMS-normalised as rmsnorm_kernel rounds: y = round(w * round(x * rsqrt(..)))
    uint4 xv[kAcQkvChunks][4];
    float ss[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int t = 0; t < 4; ++t)
#pragma unroll
      for (int i = 0; i < kAcQkvChunks; ++i) {
        const int ch = tid + i * kAcThreads;
        xv[i][t] = (t < Tn && ch < nch)
                       ? __ldcg(reinterpret_cast<const uint4*>(fq->x + static_cast<int64_t>(b * Tn + t) * Hf) + ch)
                       : make_uint4(0, 0, 0, 0);
        float f[8];
        ac_unpack8(xv[i][t], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss[t] = fmaf(f[e], f[e], ss[t]);
      }
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      ss[t] = warp_sum(ss[t]);
      if (lane == 0) red[warp * 4 + t] = ss[t];
    }
    for (int i = tid; i < (16 - R) * 64; i += kAcThreads)  // query rows past R are zero
      q_s[am_swz(R + i / 64, i % 64)] = __float2bfloat16_rn(0.f);
    __syncthreads();
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < kAcWarps; ++w) tot += red[w * 4 + t];
      ss[t] = 1.0f / sqrtf(tot / static_cast<float>(Hf) + fq->eps);
    }
#pragma unroll
    for (int i = 0; i < kAcQkvChunks; ++i) {
      const int ch = tid + i * kAcThreads;
      if (ch >= nch) break;
      float wf[8];
      ac_unpack8(nw[i], wf);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        if (t >= Tn) break;
        float f[8];
        ac_unpack8(xv[i][t], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = wf[e] * round_to<T16>(f[e] * ss[t]);
        reinterpret_cast<uint4*>(xs + t * Hf)[ch] = ac_pack8(f);
      }
    }
    __syncthreads();
    // this CTA's 2 np weight rows: one row per warp at a time, lanes over 16-byte chunks; the
    // products are rounded to bf16 as the projection's output
    mbar_wait_bounded(wbar, 0, a.status, nullptr);
    const uint4* x4 = reinterpret_cast<const uint4*>(xs);
    for (int j = warp; j < 2 * np; j += kAcWarps) {
      const uint4* wr = reinterpret_cast<const uint4*>(w_s + static_cast<int64_t>(j) * Hf);
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      for (int ch = lane; ch < nch; ch += 32) {
        float wf[8];
        ac_unpack8(wr[ch], wf);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          if (t >= Tn) break;
          float f[8];
          ac_unpack8(x4[t * nch + ch], f);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[t] = fmaf(wf[e], f[e], acc[t]);
        }
      }
#pragma unroll
      for (int t = 0; t < 4; ++t) acc[t] = warp_sum(acc[t]);
      if (lane == 0) {
#pragma unroll
        for (int t = 0; t < 4; ++t)
          if (t < Tn) res[t * 2 * np + j] = round_to<T16>(acc[t]);
      }
    }
    __syncthreads();
    // rotate q and k (EPI_QKV's rounding), then send: q to every CTA of the cluster, a new key
    // or value to the CTA whose chunk holds its position, and to the pool
    const int C = ka.p.splits_max;
    ac_cluster_wait();  // every CTA of the cluster runs, so its shared memory can be written
    for (int i = tid; i < Tn * np; i += kAcThreads) {
      const int t = i / np, l = i - t * np;
      const int pr = p0 + l, hh = pr >> 5, c = pr & 31;
      float lo = res[t * 2 * np + l], hi = res[t * 2 * np + np + l];
      if (hh <= G) {
        const int pos = min(past + t, a.max_positions - 1);
        const float cs = round_to<T16>(a.rope_cos[static_cast<int64_t>(pos) * 32 + c]);
        const float sn = round_to<T16>(a.rope_sin[static_cast<int64_t>(pos) * 32 + c]);
        const float lo2 = round_to<T16>(round_to<T16>(lo * cs) + round_to<T16>(-hi * sn));
        const float hi2 = round_to<T16>(round_to<T16>(hi * cs) + round_to<T16>(lo * sn));
        lo = lo2;
        hi = hi2;
      }
      const unsigned short ulo = __bfloat16_as_ushort(__float2bfloat16_rn(lo));
      const unsigned short uhi = __bfloat16_as_ushort(__float2bfloat16_rn(hi));
      if (hh < G) {
        const int r = t * G + hh;
        const uint32_t olo = smem_u32(q_s + am_swz(r, c)), ohi = smem_u32(q_s + am_swz(r, c + 32));
        for (int cr = 0; cr < C; ++cr) {
          asm volatile("st.shared::cluster.u16 [%0], %1;" ::"r"(ac_mapa(olo, cr)), "h"(ulo) : "memory");
          asm volatile("st.shared::cluster.u16 [%0], %1;" ::"r"(ac_mapa(ohi, cr)), "h"(uhi) : "memory");
        }
      } else if (t < nn) {
        const int kk = past + t, tgt = kk / chunk;
        const bool isv = hh > G;
        if (tgt < C) {
          __nv_bfloat16* dst = isv ? v_s : k_s;
          const int rr = kk - tgt * chunk;
          asm volatile("st.shared::cluster.u16 [%0], %1;" ::"r"(ac_mapa(smem_u32(dst + am_swz(rr, c)), tgt)), "h"(ulo)
                       : "memory");
          asm volatile("st.shared::cluster.u16 [%0], %1;" ::"r"(ac_mapa(smem_u32(dst + am_swz(rr, c + 32)), tgt)),
                       "h"(uhi)
                       : "memory");
        }
        const int sl = fq->slot[b * Tn + t];
        if (sl >= 0) {
          __nv_bfloat16* pool = const_cast<__nv_bfloat16*>(isv ? vp : kp) + (static_cast<int64_t>(sl) * a.Hkv + g) * D;
          pool[c] = __ushort_as_bfloat16(ulo);
          pool[c + 32] = __ushort_as_bfloat16(uhi);
        }
      }
    }
    ac_cluster_sync();  // every CTA's q rows and new keys / values have landed
  } else if (a.qkv_parts) {
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
  if (!fq) ac_cluster_wait();  // (the fused projection waited on the start barrier already)
  if (part != 0) {
    const uint32_t dst = ac_mapa(smem_u32(slots + part * slot_floats), lead);
    for (int i = tid; i < slot_floats; i += kAcThreads) ac_st_remote(dst + 4 * i, mo[i]);
  }
  ac_cluster_sync();
  stamp(5);
  if (part == 0) {
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out);
    const int nc = fo ? static_cast<int>(gridDim.x) : 1;  // CTAs that receive the head's output
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
      const __nv_bfloat16 v = __float2bfloat16_rn(O / L);
      if (!fo) {
        out[(static_cast<int64_t>(b * a.T + t) * a.Hq + h) * D + c] = v;
      } else {
        const uint32_t off = smem_u32(attn_s + t * K + h * D + c);
        for (int cr = 0; cr < nc; ++cr)
          asm volatile("st.shared::cluster.u16 [%0], %1;" ::"r"(ac_mapa(off, cr)), "h"(__bfloat16_as_ushort(v)) : "memory");
      }
    }
  }
  if (!fo) {
    stamp(6);
    return;
  }
  ac_cluster_sync();  // every CTA holds the attention output of all heads
  // o = W_o attn for rows [o0, o1) and the residual add (the GEMM's EPI_RESID rounding)
  if (!mbar_wait_bounded(obar, 0, a.status, nullptr)) return;
  const uint4* a4 = reinterpret_cast<const uint4*>(attn_s);
  const int nch = K >> 3;
  for (int n = o0 + warp; n < o1; n += kAcWarps) {
    const uint4* wr = reinterpret_cast<const uint4*>(wo_s + static_cast<int64_t>(n - o0) * K);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int ch = lane; ch < nch; ch += 32) {
      const uint4 wv = wr[ch];
      const uint32_t wu[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        if (t >= a.T) break;
        const uint4 xv = a4[t * nch + ch];
        const uint32_t xu[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc[t] = fmaf(__uint_as_float(wu[q] << 16), __uint_as_float(xu[q] << 16), acc[t]);
          acc[t] = fmaf(__uint_as_float(wu[q] & 0xffff0000u), __uint_as_float(xu[q] & 0xffff0000u), acc[t]);
        }
      }
    }
#pragma unroll
    for (int t = 0; t < 4; ++t) acc[t] = warp_sum(acc[t]);
    if (lane < a.T) {
      float v = acc[0];
#pragma unroll
      for (int t = 1; t < 4; ++t)
        if (lane == t) v = acc[t];
      __nv_bfloat16* hp = fo->hidden + static_cast<int64_t>(b * a.T + lane) * fo->H + n;
      *hp = __float2bfloat16_rn(__bfloat162float(*hp) + round_to<__nv_bfloat16>(v));
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
