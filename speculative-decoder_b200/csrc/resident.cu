// Resident decode schedule: one decode step of a small bf16 Llama (the reference's forward,
// lm/forward.py:21-84, at one to four token rows: the draft model's steps) as ONE cooperative
// launch with one CTA per SM, instead of a chain of ~5 launches per layer.
//
// What bounds a decode step of a small model is latency, not bytes: the 135M draft streams
// 284 MB per step (43 us at HBM speed) but a chain of 153 dependent launches costs ~3.7 us
// per link. Here the links are flagged packets in global memory:
//
// - Every CTA owns fixed slices of every linear (rotary pairs of q/k/v, rows of o and down,
//   features of gate/up, rows of the LM head). A producer warp streams the CTA's slices, in the
//   order they will be used, through a ring of 16 KB shared-memory slots with bulk copies;
//   weights never depend on activations, so the stream runs ahead across layers while the
//   compute warps wait for activations.
// - A phase's outputs go to global memory as 16-byte packets of two (32-bit payload, 32-bit
//   epoch) words, stored and polled with volatile 16-byte accesses: a consumer knows a word has
//   arrived when its epoch matches, without fences, counters or barriers. Epochs are unique per
//   (launch, layer, phase): a launch-generation counter in the workspace is advanced by the
//   last CTA to finish, so stale packets of earlier launches never match.
// - Per layer: q/k/v (RMSNorm folded in, RoPE and the paged K/V write in the epilogue) ->
//   attention items (sequence, KV head, key chunk) on the tensor cores (mma.sync, the cluster
//   kernel's per-CTA math) -> o (every CTA merges the items' partials itself) with the residual
//   add -> gate/up (RMSNorm folded in) with SiLU*mul -> down with the residual add. Then the
//   final RMSNorm (last-token rows) and the LM head into fp32 logits.
//
// Roundings are those of the per-layer kernels and the GEMV schedule (bf16 activations as
// torch computes them: each linear's output, the residual sums, the norm output and SiLU*mul
// rounded to bf16; fp32 accumulation). Every wait is bounded: packet waits by the launch's
// wait limit (cycles, a runtime parameter), waits on the CTA's own bulk copies by the fixed
// limit; a wait that gives up records SPECB200_ERR_TIMEOUT, raises the launch's abort flag and
// every CTA then drains its copies in flight and leaves.
#include <algorithm>
#include <cstdio>
#include <mutex>

#include "attn_mma.cuh"
#include "kernels.cuh"
#include "resident.cuh"

extern "C" int specb200_set_error(int code, const char* msg);

namespace specb200 {
namespace {

using bf16 = __nv_bfloat16;

// ---------------------------------------------------------------- packets
SPECB200_DEVINL void pk_store(uint4* dst, uint32_t d0, uint32_t d1, uint32_t ep) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "r"(d0), "r"(ep), "r"(d1), "r"(ep)
               : "memory");
}
SPECB200_DEVINL uint4 pk_load(const uint4* src) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(src)
               : "memory");
  return v;
}
SPECB200_DEVINL int ld_volatile_i32(const unsigned* p) {
  int v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

SPECB200_DEVINL void cons_sync() { asm volatile("bar.sync 2, 256;" ::: "memory"); }

// Phase stamp j of this CTA (thread 0 of the compute warps) when the launch records a trace.
SPECB200_DEVINL void stamp(const ResArgs& a, int j) {
  if (a.trace && threadIdx.x == 0) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    a.trace[static_cast<size_t>(j) * gridDim.x + blockIdx.x] = t;
  }
}

SPECB200_DEVINL void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

SPECB200_DEVINL float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
SPECB200_DEVINL float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
SPECB200_DEVINL uint32_t bf_pack(float lo, float hi) {
  return static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(lo))) |
         (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(hi))) << 16);
}
SPECB200_DEVINL float rbf(float x) { return round_to<bf16>(x); }

// ---------------------------------------------------------------- static work split
// Contiguous share [lo, hi) of n units for part i of `parts`, in multiples of `align`.
__host__ __device__ inline void share(int n, int parts, int i, int align, int& lo, int& hi) {
  const int units = (n + align - 1) / align;
  lo = min(n, static_cast<int>(static_cast<long long>(units) * i / parts) * align);
  hi = min(n, static_cast<int>(static_cast<long long>(units) * (i + 1) / parts) * align);
}

enum { PH_QKV = 0, PH_O = 1, PH_GU = 2, PH_DOWN = 3, PH_HEAD = 4 };

// One ring piece: `n` units starting at unit `first` of the CTA's share; its weight rows are
// seg0 .. seg0 + n - 1, then (paired phases) seg1 .. seg1 + n - 1, each of K bf16.
struct Piece {
  int n, first, seg0, seg1, K;
  bool pair;
};

struct PhaseShape {
  const bf16* w;
  int units, K, align;
  bool pair;
};

SPECB200_DEVINL PhaseShape phase_shape(const ResArgs& a, int layer, int ph) {
  PhaseShape s;
  const int P = (a.Hq + 2 * a.Hkv) * 32;
  switch (ph) {
    case PH_QKV: s = {a.layers[layer].w_qkv, P, a.H, 2, true}; break;
    case PH_O: s = {a.layers[layer].w_o, a.H, a.Hq * 64, 4, false}; break;
    case PH_GU: s = {a.layers[layer].w_gu, a.I, a.H, 4, true}; break;
    case PH_DOWN: s = {a.layers[layer].w_down, a.H, a.I, 4, false}; break;
    default: s = {a.head, a.V, a.H, 1, false}; break;
  }
  return s;
}

// Iterates the pieces of one phase's share in order (the producer and the compute warps walk
// the same sequence). Pieces never cross a q/k/v head (32 pairs) or a gate/up group (64
// features), and fill at most one ring slot.
struct PieceWalk {
  int pos, hi, K, per, group;
  bool pair;
  int ph;
  __device__ PieceWalk(const ResArgs& a, int layer, int ph_, int cta) : ph(ph_) {
    const PhaseShape s = phase_shape(a, layer, ph_);
    int lo;
    share(s.units, a.p.grid, cta, s.align, lo, hi);
    pos = lo;
    K = s.K;
    pair = s.pair;
    per = min(kResSlot / ((pair ? 2 : 1) * K * 2), pair ? 32 : 64);  // rows of a piece <= 64 (s.res)
    group = ph_ == PH_QKV ? 32 : (ph_ == PH_GU ? 64 : 0);
  }
  __device__ bool next(Piece& pc) {
    if (pos >= hi) return false;
    const int g = group ? pos / group : 0, j = pos - g * group;
    const int end = group ? min(hi, (g + 1) * group) : hi;
    const int n = min(end - pos, per);
    pc.n = n;
    pc.first = pos;
    pc.K = K;
    pc.pair = pair;
    if (ph == PH_QKV) {
      pc.seg0 = g * 64 + j;
      pc.seg1 = pc.seg0 + 32;
    } else if (ph == PH_GU) {
      pc.seg0 = g * 128 + j;
      pc.seg1 = pc.seg0 + 64;
    } else {
      pc.seg0 = pos;
      pc.seg1 = 0;
    }
    pos += n;
    return true;
  }
};

// ---------------------------------------------------------------- shared state
struct ResShared {
  uint64_t* full;
  uint64_t* empty;
  volatile int* abort;  // CTA-local: stop waiting, drain and leave
  int* misc;            // [0] generation, [4..9] attention item table, [16..19] head rows
  float* h;             // [M][H] fp32: the residual stream rows
  bf16* x;              // [M][Kmax] bf16: the current phase's input
  float* res;           // [M][64]: dot products of one piece
  uint32_t* out;        // [M][kResMaxWords]: the phase's output words (bf16 pairs)
  uint8_t* att;         // attention region
  uint8_t* ring;
};

// Bounded wait for the launch's packets: returns false once the wait limit ran out or the
// launch was aborted (then the CTA-local abort flag is set).
SPECB200_DEVINL bool pk_wait(const ResArgs& a, const ResShared& s, const uint4* src, uint32_t ep, uint4& v,
                             unsigned* ctl) {
  v = pk_load(src);
  if (v.y == ep && v.w == ep) return true;
  const long long t0 = clock64();
  for (unsigned it = 1;; ++it) {
    v = pk_load(src);
    if (v.y == ep && v.w == ep) return true;
    if (*s.abort) return false;
    if ((it & 31) == 0 && ld_volatile_i32(ctl + 2)) {
      *s.abort = 1;
      return false;
    }
    if (clock64() - t0 > a.wait_limit) {
      set_status(a.status, SPECB200_ERR_TIMEOUT);
      atomicExch(ctl + 2, 1u);
      *s.abort = 1;
      return false;
    }
  }
}

// Packets i = tid, tid + 256, ... < n of the compute warps: the loads of up to two go out
// together (one round trip when they have all arrived), and only the ones whose epoch has not
// arrived yet are then waited for. use(i, v, ok) consumes packet i (ok false after a wait gave
// up or the launch was aborted).
template <class At, class Use>
SPECB200_DEVINL void pk_gather(const ResArgs& a, const ResShared& s, int n, uint32_t ep, unsigned* ctl, At&& at,
                               Use&& use) {
  constexpr int kBatch = 2;
  for (int base = threadIdx.x; base < n; base += kBatch * kResConsumers) {
    uint4 v[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int i = base + j * kResConsumers;
      if (i < n) v[j] = pk_load(at(i));
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int i = base + j * kResConsumers;
      if (i >= n) break;
      bool ok = v[j].y == ep && v[j].w == ep;
      if (!ok) ok = pk_wait(a, s, at(i), ep, v[j], ctl);
      use(i, v[j], ok);
    }
  }
}

// Region layout (fixed offsets inside kResRegionBytes): control words, then per layer parity
// the q/k/v, attention, h-after-attention, activation and h-after-MLP packet buffers.
struct Region {
  unsigned* ctl;  // [0] generation, [1] finished CTAs, [2] abort
  uint4 *qkv, *att, *hmid, *hout, *act;
  int qkv_n, att_n, h_n, act_n;  // uint4 per parity
};
__host__ __device__ inline size_t region_layout(int M, int P, int H, int I, int max_items, size_t offs[6]) {
  size_t off = 256;
  const size_t q = static_cast<size_t>(M) * P / 2, h = static_cast<size_t>(M) * H / 4,
               ac = static_cast<size_t>(M) * I / 4,
               at = static_cast<size_t>(max_items) * kResMaxQRows * kResAttRow;
  const size_t sizes[5] = {q, at, h, h, ac};
  for (int i = 0; i < 5; ++i) {
    offs[i] = off;
    off += 2 * sizes[i] * sizeof(uint4);
  }
  offs[5] = off;
  return off;
}
SPECB200_DEVINL Region region_of(const ResArgs& a) {
  size_t offs[6];
  const int P = (a.Hq + 2 * a.Hkv) * 32;
  region_layout(a.M, P, a.H, a.I, a.p.max_items, offs);
  Region r;
  r.ctl = reinterpret_cast<unsigned*>(a.region);
  r.qkv = reinterpret_cast<uint4*>(a.region + offs[0]);
  r.att = reinterpret_cast<uint4*>(a.region + offs[1]);
  r.hmid = reinterpret_cast<uint4*>(a.region + offs[2]);
  r.hout = reinterpret_cast<uint4*>(a.region + offs[3]);
  r.act = reinterpret_cast<uint4*>(a.region + offs[4]);
  r.qkv_n = a.M * P / 2;
  r.att_n = a.p.max_items * kResMaxQRows * kResAttRow;
  r.h_n = a.M * a.H / 4;
  r.act_n = a.M * a.I / 4;
  return r;
}

// ---------------------------------------------------------------- compute helpers
// RMSNorm of the M rows of s.h into s.x (bf16, row stride K = H), as rmsnorm_kernel rounds:
// y = round(w * round(x * rsqrt(mean(x^2) + eps))). rows_sel: for the final norm, output row
// o < rows reads residual row sel[o]. 256 threads; ends synchronised.
SPECB200_DEVINL void res_norm(const ResArgs& a, const ResShared& s, const bf16* w, int rows, const int* sel) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* red = s.res + kResMaxRows * 64;  // [8 warps][kResMaxRows]
  for (int o = 0; o < rows; ++o) {
    const float* hr = s.h + (sel ? sel[o] : o) * a.H;
    float ss = 0.f;
    for (int j = tid; j < a.H; j += kResConsumers) ss = fmaf(hr[j], hr[j], ss);
    ss = warp_sum(ss);
    if (lane == 0) red[warp * kResMaxRows + o] = ss;
  }
  cons_sync();
  for (int o = 0; o < rows; ++o) {
    float tot = 0.f;
#pragma unroll
    for (int wv = 0; wv < 8; ++wv) tot += red[wv * kResMaxRows + o];
    const float rs = 1.0f / sqrtf(tot / static_cast<float>(a.H) + a.eps);
    const float* hr = s.h + (sel ? sel[o] : o) * a.H;
    bf16* xr = s.x + o * a.H;
    for (int j = tid; j < a.H; j += kResConsumers)
      xr[j] = __float2bfloat16_rn(__bfloat162float(w[j]) * rbf(hr[j] * rs));
  }
  cons_sync();
}

// Dot products of one piece: rows r < nrows of the slot (K bf16 each) against the `rows` input
// rows of s.x (stride K); results to s.res[m * 64 + r]. 8 warps, a warp per row.
SPECB200_DEVINL void piece_dots(const ResShared& s, const uint8_t* slot, int nrows, int K, int rows) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nch = K >> 3;
  for (int r = warp; r < nrows; r += 8) {
    const uint4* wr = reinterpret_cast<const uint4*>(slot + static_cast<size_t>(r) * K * 2);
    float acc[kResMaxRows] = {0.f, 0.f, 0.f, 0.f};
    for (int c = lane; c < nch; c += 32) {
      const uint4 wv = wr[c];
      const uint32_t wu[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int m = 0; m < kResMaxRows; ++m) {
        if (m >= rows) break;
        const uint4 xv = reinterpret_cast<const uint4*>(s.x + m * K)[c];
        const uint32_t xu[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc[m] = fmaf(bf_lo(wu[q]), bf_lo(xu[q]), acc[m]);
          acc[m] = fmaf(bf_hi(wu[q]), bf_hi(xu[q]), acc[m]);
        }
      }
    }
#pragma unroll
    for (int m = 0; m < kResMaxRows; ++m) acc[m] = warp_sum(acc[m]);
    if (lane == 0) {
#pragma unroll
      for (int m = 0; m < kResMaxRows; ++m)
        if (m < rows) s.res[m * 64 + r] = acc[m];
    }
  }
  cons_sync();
}

// Position and pool slot of token row m (slot -1 for a padding token).
SPECB200_DEVINL void token_pos(const ResArgs& a, int m, int& pos, int& slot) {
  const int b = m / a.T, t = m - b * a.T;
  pos = a.past[b] + t;
  slot = -1;
  if (t < a.n_new[b]) {
    const int blk = pos / a.bs;
    if (blk < a.table_stride) {
      const int64_t sl = static_cast<int64_t>(a.table[static_cast<int64_t>(b) * a.table_stride + blk]) * a.bs + pos % a.bs;
      if (sl >= 0 && sl < a.num_slots) slot = static_cast<int>(sl);
    }
    if (slot < 0) set_status(a.status, SPECB200_ERR_RANGE);
  }
}

// ---------------------------------------------------------------- attention items
// Item i of a launch: (sequence b, KV head g, key chunk c), ordered by b, g, c; each sequence
// has ceil(kmax_b / chunk) chunks per head, kmax_b = past_b + n_new_b.
struct Item {
  int b, g, c, kbeg, kend;
};
// Key chunks per KV head of sequence b; a row with no new tokens this call (a finished row
// kept in a fixed-shape batch) has none.
SPECB200_DEVINL int chunks_of(const ResArgs& a, int b) {
  return a.n_new[b] > 0 ? (a.past[b] + a.n_new[b] + a.p.chunk - 1) / a.p.chunk : 0;
}
SPECB200_DEVINL int items_total(const ResArgs& a, const int* tab) { return tab[a.B]; }
SPECB200_DEVINL Item item_at(const ResArgs& a, const int* tab, int i) {
  Item it;
  int b = 0;
  while (b + 1 < a.B && tab[b + 1] <= i) ++b;
  const int total = a.past[b] + a.n_new[b];
  const int nck = chunks_of(a, b);
  const int local = i - tab[b];
  it.b = b;
  it.g = local / nck;
  it.c = local - it.g * nck;
  it.kbeg = it.c * a.p.chunk;
  it.kend = min(total, it.kbeg + a.p.chunk);
  return it;
}

// Attention region layout: q rows [16][64] bf16 (swizzled), K and V [chunk][64] bf16
// (swizzled), the merge scratch reusing K / V, and the partial [16][66] fp32.
constexpr int kResMergeScratch = 8 * (16 * 64 + 32) * 4;  // the 8 warps' states, reusing K / V
__host__ __device__ inline int att_kv_bytes(int chunk) { return chunk * 256 > kResMergeScratch ? chunk * 256 : kResMergeScratch; }
SPECB200_DEVINL void att_ptrs(const ResArgs& a, const ResShared& s, bf16*& q_s, bf16*& k_s, bf16*& v_s, float*& part) {
  q_s = reinterpret_cast<bf16*>(s.att);
  k_s = reinterpret_cast<bf16*>(s.att + 2048);
  v_s = k_s + a.p.chunk * 64;
  part = reinterpret_cast<float*>(s.att + 2048 + att_kv_bytes(a.p.chunk));
}

// Issue the cp.async loads of an item's cached keys (positions < past) and zero the rows
// past the chunk up to a multiple of 8; one commit group.
SPECB200_DEVINL void att_prefetch(const ResArgs& a, const ResShared& s, const Item& it, int layer) {
  bf16 *q_s, *k_s, *v_s;
  float* part;
  att_ptrs(a, s, q_s, k_s, v_s, part);
  const int tid = threadIdx.x;
  const int past = a.past[it.b];
  const int hi = max(it.kbeg, min(it.kend, past));
  const size_t lstride = static_cast<size_t>(a.num_slots) * a.Hkv * 64;
  const bf16* kp = a.k_pool + layer * lstride;
  const bf16* vp = a.v_pool + layer * lstride;
  const int32_t* table = a.table + static_cast<int64_t>(it.b) * a.table_stride;
  for (int idx = tid; idx < (hi - it.kbeg) * 16; idx += kResConsumers) {
    const int key = it.kbeg + (idx >> 4), part16 = idx & 15, isv = part16 >> 3, cc = part16 & 7;
    const int64_t sl = static_cast<int64_t>(table[key / a.bs]) * a.bs + key % a.bs;
    cp_async_16((isv ? v_s : k_s) + am_swz(key - it.kbeg, cc * 8), (isv ? vp : kp) + (sl * a.Hkv + it.g) * 64 + cc * 8);
  }
  cp_async_commit();
  const int nk = it.kend - it.kbeg, ngrp8 = (nk + 7) / 8;
  for (int idx = tid; idx < (ngrp8 * 8 - nk) * 16; idx += kResConsumers) {
    const int r = nk + (idx >> 4), part16 = idx & 15, isv = part16 >> 3, cc = part16 & 7;
    *reinterpret_cast<uint4*>((isv ? v_s : k_s) + am_swz(r, cc * 8)) = make_uint4(0, 0, 0, 0);
  }
}

// Merge of the 8 warps' online-softmax states into the partial [R][66] (o, m, l); the scratch
// reuses the K / V region. Ends synchronised.
SPECB200_DEVINL void att_merge_warps(const AmState& st, float* scratch, int R, float* part) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tig = lane & 3;
  const int stride = 16 * 64 + 32;
  float* wo = scratch + warp * stride;
  float* wm = wo + 16 * 64;
  float* wl = wm + 16;
  float l0 = st.l[0], l1 = st.l[1];
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    const int c = nt * 8 + 2 * tig;
    wo[g * 64 + c] = st.o[nt][0];
    wo[g * 64 + c + 1] = st.o[nt][1];
    wo[(g + 8) * 64 + c] = st.o[nt][2];
    wo[(g + 8) * 64 + c + 1] = st.o[nt][3];
  }
  if (tig == 0) {
    wm[g] = st.m[0];
    wm[g + 8] = st.m[1];
    wl[g] = l0;
    wl[g + 8] = l1;
  }
  cons_sync();
  for (int i = tid; i < R * 64; i += kResConsumers) {
    const int r = i >> 6, c = i & 63;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 8; ++w) M = fmaxf(M, scratch[w * stride + 16 * 64 + r]);
    float O = 0.f, L = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const float* b = scratch + w * stride;
      const float mw = b[16 * 64 + r];
      const float wgt = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
      O = fmaf(b[r * 64 + c], wgt, O);
      L = fmaf(b[16 * 64 + 16 + r], wgt, L);
    }
    part[r * 66 + c] = O;
    if (c == 0) {
      part[r * 66 + 64] = M;
      part[r * 66 + 65] = L;
    }
  }
  cons_sync();
}

// One attention item: wait for its q rows and new keys / values (q/k/v packets), compute the
// partial over its key chunk, publish it. The cached keys were prefetched (att_prefetch).
SPECB200_DEVINL void att_item(const ResArgs& a, const ResShared& s, const Region& rg, const Item& it, int par,
                              uint32_t ep_in, uint32_t ep_out, int item_index) {
  bf16 *q_s, *k_s, *v_s;
  float* part;
  att_ptrs(a, s, q_s, k_s, v_s, part);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int G = a.Hq / a.Hkv, R = a.T * G, P = (a.Hq + 2 * a.Hkv) * 32;
  const int past = a.past[it.b], nn = a.n_new[it.b], total = past + nn;
  const uint4* qkv = rg.qkv + static_cast<size_t>(par) * rg.qkv_n;
  // q rows (row r = token t, head g G + r % G; rows past R are zero) and this call's keys /
  // values inside the chunk, their packets requested together
  for (int i = R * 32 + tid; i < 16 * 32; i += kResConsumers) {
    const int r = i >> 5, c = i & 31;
    q_s[am_swz(r, c)] = __float2bfloat16_rn(0.f);
    q_s[am_swz(r, c + 32)] = __float2bfloat16_rn(0.f);
  }
  auto q_word = [&](int i) {
    const int r = i >> 5, c = i & 31, t = r / G, h = it.g * G + r % G;
    return (it.b * a.T + t) * P + h * 32 + c;
  };
  pk_gather(
      a, s, R * 32, ep_in, rg.ctl, [&](int i) { return qkv + (q_word(i) >> 1); },
      [&](int i, const uint4& v, bool ok) {
        const uint32_t w = ok ? ((q_word(i) & 1) ? v.z : v.x) : 0u;
        const int r = i >> 5, c = i & 31;
        q_s[am_swz(r, c)] = __ushort_as_bfloat16(static_cast<unsigned short>(w & 0xffffu));
        q_s[am_swz(r, c + 32)] = __ushort_as_bfloat16(static_cast<unsigned short>(w >> 16));
      });
  const int nlo = max(it.kbeg, past), nhi = it.kend;  // new keys inside the chunk
  auto kv_word = [&](int i) {
    const int key = nlo + (i >> 6), isv = (i >> 5) & 1, c = i & 31;
    return (it.b * a.T + (key - past)) * P + (a.Hq + (isv ? a.Hkv : 0) + it.g) * 32 + c;
  };
  pk_gather(
      a, s, max(0, nhi - nlo) * 64, ep_in, rg.ctl, [&](int i) { return qkv + (kv_word(i) >> 1); },
      [&](int i, const uint4& v, bool ok) {
        const uint32_t w = ok ? ((kv_word(i) & 1) ? v.z : v.x) : 0u;
        const int key = nlo + (i >> 6), isv = (i >> 5) & 1, c = i & 31;
        bf16* dst = isv ? v_s : k_s;
        dst[am_swz(key - it.kbeg, c)] = __ushort_as_bfloat16(static_cast<unsigned short>(w & 0xffffu));
        dst[am_swz(key - it.kbeg, c + 32)] = __ushort_as_bfloat16(static_cast<unsigned short>(w >> 16));
      });
  cp_async_wait<0>();
  cons_sync();
  AmState st;
  am_init(st, q_s);
  const int lane = tid & 31, r0 = lane >> 2, r1 = r0 + 8;
  const int lim0 = r0 < R ? min(past + r0 / G + 1, total) : 0;
  const int lim1 = r1 < R ? min(past + r1 / G + 1, total) : 0;
  const int ngrp = (it.kend - it.kbeg + 7) / 8;
  for (int j = warp; j < ngrp; j += 8) {
    const int kabs = it.kbeg + 8 * j;
    am_step(st, k_s, v_s, 8 * j, kabs, min(8, it.kend - kabs), lim0, lim1, a.scale);
  }
  cons_sync();  // K / V become the merge scratch
  att_merge_warps(st, reinterpret_cast<float*>(k_s), R, part);
  uint4* dst = rg.att + static_cast<size_t>(par) * rg.att_n + static_cast<size_t>(item_index) * kResMaxQRows * kResAttRow;
  for (int i = tid; i < R * kResAttRow; i += kResConsumers) {
    const int r = i / kResAttRow, q = i - r * kResAttRow;
    pk_store(dst + r * kResAttRow + q, __float_as_uint(part[r * 66 + 2 * q]), __float_as_uint(part[r * 66 + 2 * q + 1]),
             ep_out);
  }
  cons_sync();
}

// Every CTA: the attention output of all heads, merged from the items' partials, into s.x as
// bf16 [M][Hq 64]. The partials are staged in the attention region first.
SPECB200_DEVINL void att_gather(const ResArgs& a, const ResShared& s, const Region& rg, const int* tab, int par,
                                uint32_t ep) {
  const int tid = threadIdx.x;
  const int G = a.Hq / a.Hkv, R = a.T * G;
  const int n_items = items_total(a, tab);
  const bool valid = tab[kResMaxRows + 1] == 0;  // the item table fits the packet buffer
  float* stage = reinterpret_cast<float*>(s.att);  // [items][R][66]
  const uint4* src = rg.att + static_cast<size_t>(par) * rg.att_n;
  pk_gather(
      a, s, n_items * R * kResAttRow, ep, rg.ctl,
      [&](int i) {
        const int item = i / (R * kResAttRow), rem = i - item * R * kResAttRow;
        return src + static_cast<size_t>(item) * kResMaxQRows * kResAttRow + rem;
      },
      [&](int i, const uint4& v, bool ok) {
        const int item = i / (R * kResAttRow), rem = i - item * R * kResAttRow;
        const int r = rem / kResAttRow, q = rem - r * kResAttRow;
        stage[(item * R + r) * 66 + 2 * q] = ok ? __uint_as_float(v.x) : 0.f;
        stage[(item * R + r) * 66 + 2 * q + 1] = ok ? __uint_as_float(v.z) : 0.f;
      });
  cons_sync();
  const int QD = a.Hq * 64;
  for (int i = tid; valid && i < a.M * QD; i += kResConsumers) {
    const int m = i / QD, hd = i - m * QD, h = hd >> 6, d = hd & 63;
    const int b = m / a.T, t = m - b * a.T;
    const int g = h / G, r = t * G + (h - g * G);
    const int nck = chunks_of(a, b);
    const int base = tab[b] + g * nck;
    float M = -INFINITY;
    for (int c = 0; c < nck; ++c) M = fmaxf(M, stage[((base + c) * R + r) * 66 + 64]);
    float O = 0.f, L = 0.f;
    for (int c = 0; c < nck; ++c) {
      const float* p = stage + ((base + c) * R + r) * 66;
      const float wgt = (p[64] == -INFINITY) ? 0.f : exp2f(p[64] - M);
      O = fmaf(p[d], wgt, O);
      L = fmaf(p[65], wgt, L);
    }
    s.x[m * QD + hd] = __float2bfloat16_rn(L > 0.f ? O / L : 0.f);
  }
  cons_sync();
}

// Read M rows of bf16-pair packets (n words per row) into fp32 rows of s.h (stride H) or
// bf16 rows of s.x (stride n * 2).
SPECB200_DEVINL void read_rows(const ResArgs& a, const ResShared& s, const uint4* src, int words, uint32_t ep,
                               bool to_h, unsigned* ctl) {
  const int tid = threadIdx.x;
  const int per = words / 2;  // uint4 per row
  pk_gather(
      a, s, a.M * per, ep, ctl, [&](int i) { return src + i; },
      [&](int i, const uint4& v, bool ok) {
        const int m = i / per, q = i - m * per;
        const uint32_t w0 = ok ? v.x : 0u, w1 = ok ? v.z : 0u;
        if (to_h) {
          float* hr = s.h + m * a.H + 4 * q;
          hr[0] = bf_lo(w0);
          hr[1] = bf_hi(w0);
          hr[2] = bf_lo(w1);
          hr[3] = bf_hi(w1);
        } else {
          uint32_t* xr = reinterpret_cast<uint32_t*>(s.x) + m * words + 2 * q;
          xr[0] = w0;
          xr[1] = w1;
        }
      });
  cons_sync();
}

// Publish the CTA's output words [w0, w1) of each row (from s.out) as packets.
SPECB200_DEVINL void write_rows(const ResArgs& a, const ResShared& s, uint4* dst, int words, int w0, int w1,
                                uint32_t ep) {
  const int tid = threadIdx.x;
  const int per = (w1 - w0) / 2;
  for (int i = tid; i < a.M * per; i += kResConsumers) {
    const int m = i / per, q = i - m * per;
    const uint32_t* o = s.out + m * kResMaxWords + 2 * q;
    pk_store(dst + (m * words + w0) / 2 + q, o[0], o[1], ep);
  }
}

// ---------------------------------------------------------------- the kernel
// 288 threads (nine warps), one CTA per SM: at most 168 registers a thread, since three of the
// warps share one of the SM's four 16,384-register partitions.
__global__ void __launch_bounds__(kResThreads, 1) resident_kernel(const __grid_constant__ ResArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cta = blockIdx.x, S = a.p.slots;
  const Region rg = region_of(a);
  ResShared s;
  s.full = reinterpret_cast<uint64_t*>(smem + a.p.off_bar);
  s.empty = s.full + kResMaxSlots;
  s.abort = reinterpret_cast<volatile int*>(s.empty + kResMaxSlots);
  s.misc = reinterpret_cast<int*>(smem + a.p.off_misc);
  s.h = reinterpret_cast<float*>(smem + a.p.off_h);
  s.x = reinterpret_cast<bf16*>(smem + a.p.off_x);
  s.res = reinterpret_cast<float*>(smem + a.p.off_res);
  s.out = reinterpret_cast<uint32_t*>(smem + a.p.off_out);
  s.att = smem + a.p.off_att;
  s.ring = smem;
  int* tab = s.misc + 4;  // item base per sequence, [B + 1]
  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    *s.abort = 0;
    s.misc[0] = ld_volatile_i32(rg.ctl);
    int acc = 0;
    for (int b = 0; b < a.B; ++b) {
      tab[b] = acc;
      acc += a.Hkv * chunks_of(a, b);
    }
    tab[a.B] = acc;
    tab[kResMaxRows + 1] = 0;
    if (acc > a.p.max_items) {  // more items than the packet buffer holds: none run
      set_status(a.status, SPECB200_ERR_RANGE);
      *s.abort = 1;
      for (int b = 0; b <= a.B; ++b) tab[b] = 0;
      tab[kResMaxRows + 1] = 1;
    }
    fence_mbar_init();
  }
  __syncthreads();
  const uint32_t gen = static_cast<uint32_t>(s.misc[0]);
  const uint32_t ep_base = 1u + gen * static_cast<uint32_t>(5 * a.L + 4);
  auto ep = [&](int layer, int ph) { return ep_base + static_cast<uint32_t>(5 * layer + ph); };

  if (warp == 8) {
    // ------------------------------------------------------------ weight producer
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      long q = 0;
      for (int l = 0; l <= a.L && !*s.abort; ++l) {
        const int nph = l < a.L ? 4 : 1;
        for (int pi = 0; pi < nph && !*s.abort; ++pi) {
          const int ph = l < a.L ? (pi == 0 ? PH_QKV : pi == 1 ? PH_O : pi == 2 ? PH_GU : PH_DOWN) : PH_HEAD;
          const PhaseShape shp = phase_shape(a, l < a.L ? l : 0, ph);
          PieceWalk walk(a, l < a.L ? l : 0, ph, cta);
          Piece pc;
          while (walk.next(pc)) {
            const int slot = static_cast<int>(q % S);
            if (q >= S && !mbar_wait_bounded(&s.empty[slot], static_cast<uint32_t>(((q / S) - 1) & 1), a.status,
                                             s.abort))
              break;
            if (*s.abort) break;  // (the consumers release slots without waiting once aborted)
            const uint32_t seg = static_cast<uint32_t>(pc.n) * pc.K * 2u;
            mbar_arrive_expect_tx(&s.full[slot], seg * (pc.pair ? 2u : 1u));
            uint8_t* dst = s.ring + static_cast<size_t>(slot) * kResSlot;
            bulk_load(dst, shp.w + static_cast<int64_t>(pc.seg0) * pc.K, seg, &s.full[slot], pol);
            if (pc.pair) bulk_load(dst + seg, shp.w + static_cast<int64_t>(pc.seg1) * pc.K, seg, &s.full[slot], pol);
            ++q;
          }
        }
      }
      // drain: every copy issued must have landed before the CTA leaves
      for (long d = max(0L, q - S); d < q; ++d) {
        uint64_t* bar = &s.full[d % S];
        const uint32_t par = static_cast<uint32_t>((d / S) & 1);
        if (mbar_try_wait(bar, par)) continue;
        const long long t0 = clock64();
        while (!mbar_try_wait(bar, par) && clock64() - t0 < SPECB200_SPIN_LIMIT_CYCLES) {
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ compute warps
    long q = 0;  // ring pieces consumed
    // Every function below that synchronises the compute warps runs unconditionally: the abort
    // flag can change at any time (the producer and every wait may raise it), so it only
    // shortens waits and suppresses stores, never a barrier.
    auto consume = [&](int layer, int ph, auto&& epi) {
      PieceWalk walk(a, layer, ph, cta);
      Piece pc;
      while (walk.next(pc)) {
        const int slot = static_cast<int>(q % S);
        if (!*s.abort) {
          if (!mbar_wait_bounded(&s.full[slot], static_cast<uint32_t>((q / S) & 1), a.status, s.abort)) {
            *s.abort = 1;
            atomicExch(rg.ctl + 2, 1u);
          }
        }
        cons_sync();
        const int rows = ph == PH_HEAD ? (a.last_only ? a.B : a.M) : a.M;
        piece_dots(s, s.ring + static_cast<size_t>(slot) * kResSlot, pc.pair ? 2 * pc.n : pc.n, pc.K, rows);
        if (!*s.abort) epi(pc);
        cons_sync();
        if (tid == 0) mbar_arrive(&s.empty[slot]);
        ++q;
      }
    };
    const int P = (a.Hq + 2 * a.Hkv) * 32;
    const int n_items = items_total(a, tab);
    stamp(a, 9 * a.L + 2);
    for (int l = 0; l < a.L; ++l) {
      const int par = l & 1;
      const ResLayer& Lw = a.layers[l];
      // my first attention item's cached keys, early
      const bool has_item = cta < n_items;
      if (has_item) att_prefetch(a, s, item_at(a, tab, cta), l);
      // ---- the layer input: the embedding rows, or the previous layer's output packets
      if (l == 0) {
        for (int i = tid; i < a.M * a.H; i += kResConsumers) {
          const int m = i / a.H, j = i - m * a.H;
          int id = a.ids[m];
          if (id < 0 || id >= a.V) {
            if (j == 0) set_status(a.status, SPECB200_ERR_RANGE);
            id = 0;
          }
          s.h[i] = __bfloat162float(a.embed[static_cast<int64_t>(id) * a.H + j]);
        }
        cons_sync();
      } else {
        read_rows(a, s, rg.hout + static_cast<size_t>(par ^ 1) * rg.h_n, a.H / 2, ep(l - 1, 4), true, rg.ctl);
      }
      stamp(a, 9 * l);
      // ---- q / k / v with RoPE; k and v also into the pool
      res_norm(a, s, Lw.attn_norm, a.M, nullptr);
      int p0, p1;
      share(P, a.p.grid, cta, 2, p0, p1);
      const size_t lstride = static_cast<size_t>(a.num_slots) * a.Hkv * 64;
      consume(l, PH_QKV, [&](const Piece& pc) {
        for (int i = tid; i < a.M * pc.n; i += kResConsumers) {
          const int m = i / pc.n, u = i - m * pc.n;
          const int pr = pc.first + u, hh = pr >> 5, c = pr & 31;
          float lo = rbf(s.res[m * 64 + u]), hi = rbf(s.res[m * 64 + pc.n + u]);
          int pos, slot;
          token_pos(a, m, pos, slot);
          if (hh < a.Hq + a.Hkv) {
            const int pp = min(pos, a.max_positions - 1);
            const float cs = rbf(a.rope_cos[static_cast<int64_t>(pp) * 32 + c]);
            const float sn = rbf(a.rope_sin[static_cast<int64_t>(pp) * 32 + c]);
            const float lo2 = rbf(rbf(lo * cs) + rbf(-hi * sn));
            const float hi2 = rbf(rbf(hi * cs) + rbf(lo * sn));
            lo = lo2;
            hi = hi2;
          }
          s.out[m * kResMaxWords + (pr - p0)] = bf_pack(lo, hi);
          if (hh >= a.Hq && slot >= 0) {
            const bool isv = hh >= a.Hq + a.Hkv;
            const int g = hh - a.Hq - (isv ? a.Hkv : 0);
            bf16* pool = (isv ? a.v_pool : a.k_pool) + l * lstride + (static_cast<int64_t>(slot) * a.Hkv + g) * 64;
            pool[c] = __float2bfloat16_rn(lo);
            pool[c + 32] = __float2bfloat16_rn(hi);
          }
        }
      });
      if (!*s.abort) write_rows(a, s, rg.qkv + static_cast<size_t>(par) * rg.qkv_n, P, p0, p1, ep(l, 0));
      stamp(a, 9 * l + 1);
      // ---- attention items
      for (int it = cta; it < n_items; it += a.p.grid) {
        const Item item = item_at(a, tab, it);
        if (it != cta) {
          cons_sync();
          att_prefetch(a, s, item, l);
        }
        att_item(a, s, rg, item, par, ep(l, 0), ep(l, 1), it);
      }
      if (!has_item) cp_async_wait<0>();
      stamp(a, 9 * l + 2);
      // ---- o with the residual add
      att_gather(a, s, rg, tab, par, ep(l, 1));
      stamp(a, 9 * l + 3);
      int r0, r1;
      share(a.H, a.p.grid, cta, 4, r0, r1);
      consume(l, PH_O, [&](const Piece& pc) {
        bf16* ob = reinterpret_cast<bf16*>(s.out);
        for (int i = tid; i < a.M * pc.n; i += kResConsumers) {
          const int m = i / pc.n, u = i - m * pc.n, j = pc.first + u;
          ob[m * 2 * kResMaxWords + (j - r0)] = __float2bfloat16_rn(s.h[m * a.H + j] + rbf(s.res[m * 64 + u]));
        }
      });
      if (!*s.abort) write_rows(a, s, rg.hmid + static_cast<size_t>(par) * rg.h_n, a.H / 2, r0 / 2, r1 / 2, ep(l, 2));
      stamp(a, 9 * l + 4);
      // ---- gate / up with SiLU * mul
      read_rows(a, s, rg.hmid + static_cast<size_t>(par) * rg.h_n, a.H / 2, ep(l, 2), true, rg.ctl);
      res_norm(a, s, Lw.mlp_norm, a.M, nullptr);
      stamp(a, 9 * l + 5);
      int f0, f1;
      share(a.I, a.p.grid, cta, 4, f0, f1);
      consume(l, PH_GU, [&](const Piece& pc) {
        bf16* ob = reinterpret_cast<bf16*>(s.out);
        for (int i = tid; i < a.M * pc.n; i += kResConsumers) {
          const int m = i / pc.n, u = i - m * pc.n, f = pc.first + u;
          const float g = rbf(s.res[m * 64 + u]), up = rbf(s.res[m * 64 + pc.n + u]);
          const float act = rbf(g / (1.0f + expf(-g)));
          ob[m * 2 * kResMaxWords + (f - f0)] = __float2bfloat16_rn(act * up);
        }
      });
      if (!*s.abort) write_rows(a, s, rg.act + static_cast<size_t>(par) * rg.act_n, a.I / 2, f0 / 2, f1 / 2, ep(l, 3));
      stamp(a, 9 * l + 6);
      // ---- down with the residual add
      read_rows(a, s, rg.act + static_cast<size_t>(par) * rg.act_n, a.I / 2, ep(l, 3), false, rg.ctl);
      stamp(a, 9 * l + 7);
      consume(l, PH_DOWN, [&](const Piece& pc) {
        bf16* ob = reinterpret_cast<bf16*>(s.out);
        for (int i = tid; i < a.M * pc.n; i += kResConsumers) {
          const int m = i / pc.n, u = i - m * pc.n, j = pc.first + u;
          ob[m * 2 * kResMaxWords + (j - r0)] = __float2bfloat16_rn(s.h[m * a.H + j] + rbf(s.res[m * 64 + u]));
        }
      });
      if (!*s.abort) write_rows(a, s, rg.hout + static_cast<size_t>(par) * rg.h_n, a.H / 2, r0 / 2, r1 / 2, ep(l, 4));
      stamp(a, 9 * l + 8);
    }
    // ---- final norm (each sequence's last token row when last_only) and the LM head
    const int lp = (a.L - 1) & 1;
    read_rows(a, s, rg.hout + static_cast<size_t>(lp) * rg.h_n, a.H / 2, ep(a.L - 1, 4), true, rg.ctl);
    stamp(a, 9 * a.L);
    const int rows_out = a.last_only ? a.B : a.M;
    int* sel = s.misc + 16;
    if (tid < rows_out) sel[tid] = a.last_only ? tid * a.T + max(a.n_new[tid] - 1, 0) : tid;
    cons_sync();
    res_norm(a, s, a.final_norm, rows_out, sel);
    consume(0, PH_HEAD, [&](const Piece& pc) {
      for (int i = tid; i < rows_out * pc.n; i += kResConsumers) {
        const int o = i / pc.n, u = i - o * pc.n;
        a.logits[static_cast<int64_t>(o) * a.V + pc.first + u] = s.res[o * 64 + u];
      }
    });
    stamp(a, 9 * a.L + 1);
  }
  __syncthreads();
  // ---- the last CTA to finish advances the launch generation and clears the abort flag
  if (tid == 0) {
    __threadfence();
    const unsigned done = atomicAdd(rg.ctl + 1, 1u);
    if (done == static_cast<unsigned>(gridDim.x) - 1) {
      atomicExch(rg.ctl + 1, 0u);
      atomicExch(rg.ctl + 2, 0u);
      __threadfence();
      atomicAdd(rg.ctl, 1u);
    }
  }
}

int g_sms = 0;

}  // namespace

bool resident_prepare() {
  static std::once_flag once;
  static bool ok = false;
  std::call_once(once, [] {
    int dev = 0, blocks = 0;
    const char* step = "cudaGetDevice";
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) {
      step = "multiprocessor count";
      e = cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
    }
    if (e == cudaSuccess) {
      step = "shared-memory limit";
      e = cudaFuncSetAttribute(resident_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    }
    if (e == cudaSuccess) {
      step = "carveout";
      e = cudaFuncSetAttribute(resident_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                               cudaSharedmemCarveoutMaxShared);
    }
    if (e == cudaSuccess) {
      step = "occupancy";
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, resident_kernel, kResThreads, 200 * 1024);
    }
    ok = e == cudaSuccess && blocks >= 1;
    if (!ok) {
      char msg[256];
      std::snprintf(msg, sizeof(msg), "resident kernel unavailable (%s: %s, %d blocks per SM)", step,
                    cudaGetErrorString(e), blocks);
      specb200_set_error(SPECB200_ERR_CUDA, msg);
    }
  });
  return ok;
}

bool plan_resident(int L, int H, int Hq, int Hkv, int D, int I, int V, int B, int T, int max_kv_len, ResPlan* p) {
  if (D != 64 || L <= 0 || L > kResMaxLayers || B <= 0 || T <= 0 || B * T > kResMaxRows) return false;
  // Draft-class models only (hidden <= 1024). A target model's one-token decode must round
  // exactly as its (k+1)-token verify does -- the per-layer tensor-core kernels at both shapes --
  // so that speculative greedy output equals plain greedy output bit for bit.
  if (H > kResMaxHidden) return false;
  if (Hq % Hkv || T * (Hq / Hkv) > kResMaxQRows || H % 8 || I % 64 || H % 4) return false;
  if (!resident_prepare()) return false;
  const int grid = g_sms;
  const int M = B * T;
  const int P = (Hq + 2 * Hkv) * 32;
  // every CTA must own gate/up features (the phase that ties all CTAs together each layer)
  if (I / 4 < grid) return false;
  // per-CTA output words of a phase must fit the staging (q/k/v pairs, o / down rows, features)
  auto max_share = [&](int n, int align) { return ((n + align - 1) / align + grid - 1) / grid * align; };
  if (max_share(P, 2) > kResMaxWords || max_share(H, 4) / 2 > kResMaxWords || max_share(I, 4) / 2 > kResMaxWords)
    return false;
  // one ring slot must hold a row (or a row pair) of every phase
  const int kmax = std::max({H, Hq * 64, I});
  if (2 * H * 2 > kResSlot || Hq * 64 * 2 > kResSlot || I * 2 > kResSlot) return false;
  // attention items: chunks so that the partials of every item fit the attention region
  const int R = T * (Hq / Hkv);
  const int len = std::max(1, max_kv_len);
  int chunk = 0, items = 0, att = 0;
  for (int c : {128, 256, 512}) {
    const int nck = (len + c - 1) / c;
    const int it = B * Hkv * nck;
    const int item_bytes = 2048 + att_kv_bytes(c) + kResMaxQRows * 66 * 4;
    const int stage = it * R * 66 * 4;
    const int need = std::max(item_bytes, stage);
    if (need <= 96 * 1024) {
      chunk = c;
      items = it;
      att = (need + 1023) / 1024 * 1024;
      break;
    }
  }
  if (!chunk) return false;
  size_t offs[6];
  if (region_layout(M, P, H, I, items, offs) > kResRegionBytes) return false;
  // shared memory: ring slots, then h, x, attention, res, out, barriers, misc
  const int h_bytes = (M * H * 4 + 1023) / 1024 * 1024;
  const int x_bytes = (M * kmax * 2 + 1023) / 1024 * 1024;
  const int res_bytes = kResMaxRows * 64 * 4 + 8 * kResMaxRows * 4;  // piece results + norm scratch
  const int out_bytes = kResMaxRows * kResMaxWords * 4;
  const int tail = h_bytes + x_bytes + att + res_bytes + out_bytes + 2 * kResMaxSlots * 8 + 16 + 256;
  const int budget = 227 * 1024 - 1024;
  const int slots = std::min(kResMaxSlots, (budget - tail) / kResSlot);
  if (slots < 4) return false;
  p->grid = grid;
  p->slots = slots;
  p->chunk = chunk;
  p->max_items = items;
  p->att_bytes = att;
  int off = slots * kResSlot;
  p->off_h = off;
  off += h_bytes;
  p->off_x = off;
  off += x_bytes;
  p->off_att = off;
  off += att;
  p->off_res = off;
  off += (res_bytes + 15) / 16 * 16;
  p->off_out = off;
  off += out_bytes;
  p->off_bar = off;
  off += 2 * kResMaxSlots * 8 + 16;
  p->off_misc = off;
  off += 256;
  p->smem = static_cast<size_t>(off);
  (void)V;
  return p->smem <= static_cast<size_t>(227 * 1024);
}

int launch_resident(const ResArgs& a, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.p.grid);
  cfg.blockDim = dim3(kResThreads);
  cfg.dynamicSmemBytes = a.p.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, resident_kernel, a) == cudaSuccess ? SPECB200_OK : SPECB200_ERR_CUDA;
}

}  // namespace specb200
