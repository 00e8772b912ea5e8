// Decode / verify attention work item on the tensor cores: bf16, d = 64, at most 16 query rows
// (T x G) per KV head, for the per-layer attention kernel (attention.cu) when the keys exceed
// one cluster. One item = (sequence b, KV head g, key chunk `split` of the plan).
//
// Same computation and mask as attention_item (attn_core.cuh) -- the reference's SDPA over the
// gathered cache, lm/forward.py:44-49,62-63 -- with the products on mma.sync (attn_mma.cuh).
// Memory round trips per item: (1) the query rows and the chunk's block-table entries
// together, (2) cp.async of up to kAmRing blocks of 32 keys at once into a ring, refilled as
// blocks are consumed. Splits merge as in attention_item: partials to the workspace, the last
// CTA of the (b, g) group (atomic ticket) combines them in split order.
//
// With `pdl` (a kernel launched with programmatic dependent launch) the item reads what
// precedes the forward call before griddepcontrol.wait: past / n_new, the block table and the
// keys and values of positions < past. The call's first kernel is launched without the
// overlap, so all of these were complete before any kernel of the call started; only the
// query rows and this call's new keys and values come from the q/k/v projection, after the
// wait. When the chunk fits the ring, its cached keys are therefore in shared memory by the
// time the projection finishes.
#pragma once
#include "attn_core.cuh"
#include "attn_mma.cuh"

namespace specb200 {

constexpr int kAmRing = 4;          // 32-key blocks in flight (8 KB each: K then V)
constexpr int kAmItemTab = 512;     // block-table entries staged per item
constexpr int kAmItemSmem = 2048 + kAmRing * 8192 + kAmItemTab * 4 + 64;
static_assert(kAmRing * 8192 >= 4 * (16 * 64 + 32) * 4 + (16 * 64 + 32) * 4, "merge scratch and outputs fit the ring");
constexpr int kAmMaxSplits = 148;  // the split merge keeps 2 floats per (split, row) + 1 per row in the ring
static_assert((2 * kAmMaxSplits * 16 + 16) * 4 <= kAmRing * 8192, "split weights fit the ring");

static __device__ void attention_item_mma(const AttnKernelArgs& ka, int b, int g, int split, uint8_t* smem,
                                          bool pdl = false) {
  const AttnArgs& a = ka.a;
  constexpr int D = 64;
  const int G = a.Hq / a.Hkv;
  const int R = a.T * G;
  const int past = a.past[b], nn = a.n_new[b], total = past + nn;
  if (nn <= 0) return;
  const int kmax = min(total, past + (R - 1) / G + 1);
  const int nsplit = min(ka.p.splits_max, (kmax + ka.p.chunk - 1) / ka.p.chunk);
  if (split >= nsplit) return;
  const int kbeg = split * ka.p.chunk;
  const int kend = (split == nsplit - 1) ? kmax : min(kmax, kbeg + ka.p.chunk);
  __nv_bfloat16* q_s = reinterpret_cast<__nv_bfloat16*>(smem);
  uint8_t* ring = smem + 2048;
  int* tab = reinterpret_cast<int*>(ring + kAmRing * 8192);
  int* last = tab + kAmItemTab;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const __nv_bfloat16* q = static_cast<const __nv_bfloat16*>(a.q);
  const __nv_bfloat16* kp = static_cast<const __nv_bfloat16*>(a.k_pool);
  const __nv_bfloat16* vp = static_cast<const __nv_bfloat16*>(a.v_pool);
  const int32_t* table = a.table + static_cast<int64_t>(b) * a.table_stride;
  unsigned long long* tr = nullptr;
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

  auto load_q = [&] {
    for (int i = tid; i < 16 * 8; i += kAttnThreads) {
      const int r = i >> 3, c8 = i & 7;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (r < R) {
        const int t = r / G, h = g * G + r % G;
        v = *reinterpret_cast<const uint4*>(q + (static_cast<int64_t>(b * a.T + t) * a.Hq + h) * D + c8 * 8);
      }
      *reinterpret_cast<uint4*>(q_s + am_swz(r, c8 * 8)) = v;
    }
  };
  const int nblk = (kend - kbeg + 31) / 32;
  const bool early = pdl && nblk <= kAmRing;  // the whole chunk is loaded before the wait
  if (pdl && !early) {
    pdl_wait();
    stamp(1);
  }

  // (1) query rows (zero past R) and the chunk's block-table entries
  if (!early) load_q();
  const int tb0 = kbeg / a.bs;
  const int ntab = (kend - 1) / a.bs - tb0 + 1;
  for (int i = tid; i < min(ntab, kAmItemTab); i += kAttnThreads) tab[i] = table[tb0 + i];
  attn_sync();

  // (2) K and V blocks through the ring: keys [lo, hi) of block j (zero past kend)
  // Thread t takes half (t & 1) of the K (or V, (t >> 1) & 1) row of key t >> 2: one slot
  // lookup per four 16-byte copies.
  static_assert(kAttnThreads == 32 * 4, "four (row half) tasks per key of a 32-key block");
  auto load_keys = [&](int j, int lo, int hi) {
    __nv_bfloat16* blk = reinterpret_cast<__nv_bfloat16*>(ring) + (j % kAmRing) * 4096;
    const int r = tid >> 2, isv = (tid >> 1) & 1, c0 = (tid & 1) * 4;
    const int key = kbeg + j * 32 + r;
    __nv_bfloat16* dst = blk + isv * 2048;
    if (key >= kend) {
      if (lo == kbeg) {
#pragma unroll
        for (int cc = c0; cc < c0 + 4; ++cc) *reinterpret_cast<uint4*>(dst + am_swz(r, cc * 8)) = make_uint4(0, 0, 0, 0);
      }
    } else if (key >= lo && key < hi) {
      const int e = key / a.bs - tb0;
      const int64_t blkid = e < kAmItemTab ? tab[e] : table[key / a.bs];
      const int64_t sl = blkid * a.bs + key % a.bs;
      const __nv_bfloat16* src = (isv ? vp : kp) + (sl * a.Hkv + g) * D;
#pragma unroll
      for (int cc = c0; cc < c0 + 4; ++cc) cp_async_16(dst + am_swz(r, cc * 8), src + cc * 8);
    }
  };
  auto load_block = [&](int j) {
    load_keys(j, kbeg, kend);
    cp_async_commit();
  };
  AmState st;
  const int r0 = lane >> 2, r1 = r0 + 8;
  const int lim0 = r0 < R ? min(past + r0 / G + 1, total) : 0;
  const int lim1 = r1 < R ? min(past + r1 / G + 1, total) : 0;
  if (early) {
    // cached keys now; the query rows and this call's keys once the projection is done
    const int split_at = max(kbeg, min(kend, past));
    for (int j = 0; j < nblk; ++j) load_keys(j, kbeg, split_at);
    cp_async_commit();
    pdl_wait();
    stamp(1);
    load_q();
    if (split_at < kend)
      for (int j = (split_at - kbeg) / 32; j < nblk; ++j) load_keys(j, split_at, kend);
    cp_async_commit();
    cp_async_wait<0>();
    attn_sync();
    stamp(2);
    am_init(st, q_s);
    for (int j = 0; j < nblk; ++j) {
      const __nv_bfloat16* blk = reinterpret_cast<const __nv_bfloat16*>(ring) + j * 4096;
      const int k0 = kbeg + j * 32 + warp * 8;
      const int nval = min(8, kend - k0);
      if (nval > 0) am_step(st, blk, blk + 2048, warp * 8, k0, nval, lim0, lim1, a.scale);
    }
    attn_sync();
  } else {
    for (int j = 0; j < min(kAmRing, nblk); ++j) load_block(j);
    am_init(st, q_s);
    for (int j = 0; j < nblk; ++j) {
      cp_async_wait_upto(min(nblk, j + kAmRing) - (j + 1));
      attn_sync();
      const __nv_bfloat16* blk = reinterpret_cast<const __nv_bfloat16*>(ring) + (j % kAmRing) * 4096;
      const int k0 = kbeg + j * 32 + warp * 8;
      const int nval = min(8, kend - k0);
      if (nval > 0) am_step(st, blk, blk + 2048, warp * 8, k0, nval, lim0, lim1, a.scale);
      attn_sync();
      if (j + kAmRing < nblk) load_block(j + kAmRing);
    }
  }
  float* scratch = reinterpret_cast<float*>(ring);
  float* oo = scratch + 4 * (16 * 64 + 32);
  float* om = oo + 16 * 64;
  float* ol = om + 16;
  am_merge(st, scratch, R, oo, om, ol, [] { attn_sync(); });
  stamp(3);

  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out);
  auto write_out = [&](int r, int c, float v) {
    const int t = r / G, h = g * G + r % G;
    out[(static_cast<int64_t>(b * a.T + t) * a.Hq + h) * D + c] = __float2bfloat16_rn(v);
  };
  if (nsplit == 1) {
    for (int i = tid; i < R * D; i += kAttnThreads) write_out(i / D, i % D, oo[i] / ol[i / D]);
    stamp(5);
    return;
  }
  const int group = b * a.Hkv + g;  // one query tile
  const size_t part_elems = static_cast<size_t>(kRows) * (D + 2);
  float* mine = ka.part + (static_cast<size_t>(group) * ka.p.splits_max + split) * part_elems;
  for (int i = tid; i < R * D; i += kAttnThreads) mine[i] = oo[i];
  if (tid < R) {
    mine[kRows * D + tid] = om[tid];
    mine[kRows * D + kRows + tid] = ol[tid];
  }
  __threadfence();
  attn_sync();
  if (tid == 0) *last = (atomicAdd(ka.counters + group, 1) == nsplit - 1);
  attn_sync();
  stamp(4);
  if (!*last) return;
  __threadfence();
  // Last CTA of the group: per-row weights of the splits (base-2 maxima) into shared memory
  // first, then each output element as the weighted sum over splits with its loads in flight
  // together.
  const float* base = ka.part + static_cast<size_t>(group) * ka.p.splits_max * part_elems;
  float* wsm = reinterpret_cast<float*>(ring);  // [nsplit][R] maxima -> weights, [nsplit][R] sums, [R] 1 / L
  float* lsm = wsm + nsplit * R;
  float* inv = lsm + nsplit * R;
  for (int i = tid; i < nsplit * R; i += kAttnThreads) {
    const int sp = i / R, r = i - sp * R;
    wsm[i] = __ldcg(base + sp * part_elems + kRows * D + r);
    lsm[i] = __ldcg(base + sp * part_elems + kRows * D + kRows + r);
  }
  attn_sync();
  for (int r = tid; r < R; r += kAttnThreads) {
    float M = -INFINITY;
    for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, wsm[sp * R + r]);
    float L = 0.f;
    for (int sp = 0; sp < nsplit; ++sp) {
      const float ms = wsm[sp * R + r];
      const float w = (ms == -INFINITY) ? 0.f : exp2f(ms - M);
      wsm[sp * R + r] = w;
      L = fmaf(lsm[sp * R + r], w, L);
    }
    inv[r] = L;
  }
  attn_sync();
  for (int i = tid; i < R * D; i += kAttnThreads) {
    const int r = i / D, c = i % D;
    float O = 0.f;
#pragma unroll 8
    for (int sp = 0; sp < nsplit; ++sp) O = fmaf(__ldcg(base + sp * part_elems + r * D + c), wsm[sp * R + r], O);
    write_out(r, c, O / inv[r]);
  }
  if (tid == 0) ka.counters[group] = 0;
  stamp(5);
}

// Split plan for the tensor-core item: enough (b, kv head, chunk) items for about four per SM,
// chunks of at least 64 keys (a multiple of 32).
inline AttnPlan plan_attention_mma(int B, int Hkv, int max_kv_len) {
  AttnPlan p;
  p.qtiles = 1;
  const int groups = B * Hkv;
  const int max_len = max_kv_len < 1 ? 1 : max_kv_len;
  int splits = (4 * 148 + groups - 1) / groups;  // about four per SM (config 5 verify 3.61 vs 4.77 ms at two)
  const int cap = (max_len + 63) / 64;
  splits = splits > cap ? cap : splits;
  splits = splits > kAmMaxSplits ? kAmMaxSplits : splits;
  splits = splits < 1 ? 1 : splits;
  if (groups > kAttnMaxCounters) splits = 1;
  p.chunk = (((max_len + splits - 1) / splits) + 31) / 32 * 32;
  p.splits_max = (max_len + p.chunk - 1) / p.chunk;
  return p;
}

}  // namespace specb200
