// Paged causal attention for one work item (a batch row, a KV head, a tile of up to 32 query
// rows and a chunk of keys), for the per-layer attention kernel (attention.cu): fp32 models and
// the shapes the tensor-core kernels do not take. Runs on 128 threads (threadIdx.x 0..127) that
// synchronise with named barrier 1, over a caller-provided shared-memory buffer of
// AttnSmem<D>::kFloats floats.
#pragma once
#include "common.cuh"
#include "kernels.cuh"

namespace specb200 {

SPECB200_DEVINL void attn_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

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

// Shared-memory layout of one attention item, carved from a float buffer.
template <int D>
struct AttnSmem {
  static constexpr int kFloats = kRows * (D + 1) + kKeys * (D + 1) + kKeys * D + kRows * (kKeys + 1) + kRows * D +
                                 3 * kRows + kRows + kKeys + 1;
  float (*qs)[D + 1];
  float (*ks)[D + 1];
  float (*vs)[D];
  float (*sc)[kKeys + 1];
  float (*os)[D];
  float *m, *l, *alpha;
  int *lim, *slot, *last;
  __device__ explicit AttnSmem(float* p) {
    qs = reinterpret_cast<float(*)[D + 1]>(p); p += kRows * (D + 1);
    ks = reinterpret_cast<float(*)[D + 1]>(p); p += kKeys * (D + 1);
    vs = reinterpret_cast<float(*)[D]>(p); p += kKeys * D;
    sc = reinterpret_cast<float(*)[kKeys + 1]>(p); p += kRows * (kKeys + 1);
    os = reinterpret_cast<float(*)[D]>(p); p += kRows * D;
    m = p; p += kRows;
    l = p; p += kRows;
    alpha = p; p += kRows;
    lim = reinterpret_cast<int*>(p); p += kRows;
    slot = reinterpret_cast<int*>(p); p += kKeys;
    last = reinterpret_cast<int*>(p);
  }
};

struct AttnKernelArgs {
  AttnArgs a;
  AttnPlan p;
  float* part;     // [B, Hkv, qtiles, splits_max, kRows, D + 2]
  int* counters;   // [B, Hkv, qtiles]
};

template <typename T, int D>
__device__ void attention_item(const AttnKernelArgs& ka, int b, int g, int qt, int split, float* smem) {
  const AttnArgs& a = ka.a;
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

  AttnSmem<D> sm(smem);
  float(*qs)[D + 1] = sm.qs;
  float(*ks)[D + 1] = sm.ks;
  float(*vs)[D] = sm.vs;
  float(*sc)[kKeys + 1] = sm.sc;
  float(*os)[D] = sm.os;
  float* m_s = sm.m;
  float* l_s = sm.l;
  float* alpha_s = sm.alpha;
  int* lim_s = sm.lim;
  int* slot_s = sm.slot;
  int& sh_last = *sm.last;

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
  attn_sync();

  const T* kp = static_cast<const T*>(a.k_pool);
  const T* vp = static_cast<const T*>(a.v_pool);
  const int32_t* table = a.table + static_cast<int64_t>(b) * a.table_stride;
  for (int kb = kbeg; kb < kend; kb += kKeys) {
    const int nk = min(kKeys, kend - kb);
    if (tid < kKeys) {
      const int j = kb + tid;
      slot_s[tid] = tid < nk ? table[j / a.bs] * a.bs + j % a.bs : 0;
    }
    attn_sync();
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
    attn_sync();
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
    attn_sync();
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
    attn_sync();
    for (int i = tid; i < R * D; i += kAttnThreads) {
      const int r = i / D, c = i % D;
      float acc = os[r][c] * alpha_s[r];
#pragma unroll 8
      for (int j = 0; j < kKeys; ++j) acc = fmaf(sc[r][j], vs[j][c], acc);
      os[r][c] = acc;
    }
    attn_sync();
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
  attn_sync();
  if (tid == 0) sh_last = (atomicAdd(ka.counters + group, 1) == nsplit - 1);
  attn_sync();
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


}  // namespace specb200
