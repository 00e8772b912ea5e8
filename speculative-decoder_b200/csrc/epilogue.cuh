// Fused GEMM epilogues of the per-layer GEMM kernels (gemm.cu). Each runs on 128 or 256
// threads over an fp32 tile held in shared memory: tile[token][feature], pitch kEpiPitch,
// feature j = output column n0 + j; thread x works on feature x % 128.
#pragma once
#include "gemm.cuh"

namespace specb200 {

SPECB200_DEVINL void epi_bar_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// The epilogue threads of a kernel (128 or 256) on named barrier 1.
SPECB200_DEVINL void epi_bar_sync(int n) { asm volatile("bar.sync 1, %0;" ::"r"(n) : "memory"); }

constexpr int kEpiBatch = 8;

// Global inputs of one batch of kEpiBatch tokens for thread t's feature: the residual values
// (EPI_RESID), positions, pool slots and rotary factors (EPI_QKV). Loaded by load_epi_inputs,
// consumed by apply_epilogue_batch, so a split-K CTA can fetch them before its ticket and the
// CTA that finishes the tile does not wait for them.
struct EpiInputs {
  float h[kEpiBatch];
  float c[kEpiBatch], s[kEpiBatch];
  int slot[kEpiBatch];
};

template <typename T>
__device__ void load_epi_inputs(const Epilogue& e, int n0, int m0, int t0, int valid, int N, EpiInputs& in,
                                int t = threadIdx.x) {
  const int n = n0 + t;
  if (n >= N) return;
  if (e.op == EPI_RESID) {
    const T* out = static_cast<const T*>(e.out);
#pragma unroll
    for (int j = 0; j < kEpiBatch; ++j)
      in.h[j] = (t0 + j < valid) ? to_f32<T>(out[static_cast<int64_t>(m0 + t0 + j) * e.ldo + n]) : 0.f;
  } else if (e.op == EPI_QKV) {
    const int d = e.head_dim, half = d / 2;
    const int qd = e.n_heads * d, kd = e.n_kv_heads * d;
    const int region = n < qd ? 0 : (n < qd + kd ? 1 : 2);
    const int i = (n - (region == 0 ? 0 : (region == 1 ? qd : qd + kd))) % d;
    int pos[kEpiBatch];
#pragma unroll
    for (int j = 0; j < kEpiBatch; ++j) {
      const bool live = t0 + j < valid;
      pos[j] = live ? e.pos[m0 + t0 + j] : 0;
      in.slot[j] = (live && region > 0) ? e.slot[m0 + t0 + j] : -1;
    }
    if (region < 2) {
#pragma unroll
      for (int j = 0; j < kEpiBatch; ++j) {
        const int64_t off = static_cast<int64_t>(pos[j]) * half + (i % half);
        in.c[j] = round_to<T>(e.rope_cos[off]);
        in.s[j] = round_to<T>(e.rope_sin[off]);
      }
    }
  }
}

// Tokens t0 .. min(valid, t0 + kEpiBatch) - 1 of the tile, with inputs from load_epi_inputs.
template <typename T>
__device__ void apply_epilogue_batch(const Epilogue& e, const float* tile, int n0, int m0, int t0, int valid, int N,
                                     const EpiInputs& in, int t = threadIdx.x) {
  const int n = n0 + t;
  const int t1 = min(valid, t0 + kEpiBatch);
  switch (e.op) {
    case EPI_STORE: {
      if (n >= N) return;
      for (int tok = t0; tok < t1; ++tok) {
        const float v = tile[tok * kEpiPitch + t];
        const int64_t o = static_cast<int64_t>(m0 + tok) * e.ldo + n;
        if (e.out_f32) static_cast<float*>(e.out)[o] = v;
        else static_cast<T*>(e.out)[o] = from_f32<T>(v);
      }
      return;
    }
    case EPI_RESID: {
      if (n >= N) return;
      T* out = static_cast<T*>(e.out);
#pragma unroll
      for (int j = 0; j < kEpiBatch; ++j) {
        if (t0 + j >= t1) break;
        const float proj = round_to<T>(tile[(t0 + j) * kEpiPitch + t]);
        out[static_cast<int64_t>(m0 + t0 + j) * e.ldo + n] = from_f32<T>(in.h[j] + proj);
      }
      return;
    }
    case EPI_SILU_MUL: {
      if (t >= 64 || n >= N) return;
      T* out = static_cast<T*>(e.out);
      const int f = n0 / 2 + t;
      for (int tok = t0; tok < t1; ++tok) {
        const float g = round_to<T>(tile[tok * kEpiPitch + t]);
        const float u = round_to<T>(tile[tok * kEpiPitch + 64 + t]);
        const float act = round_to<T>(g / (1.0f + expf(-g)));
        out[static_cast<int64_t>(m0 + tok) * e.ldo + f] = from_f32<T>(act * u);
      }
      return;
    }
    case EPI_QKV: {
      if (n >= N) return;
      const int d = e.head_dim, half = d / 2;
      const int qd = e.n_heads * d, kd = e.n_kv_heads * d;
      const int region = n < qd ? 0 : (n < qd + kd ? 1 : 2);
      const int idx = n - (region == 0 ? 0 : (region == 1 ? qd : qd + kd));
      const int h = idx / d, i = idx % d;
      const int partner = i < half ? t + half : t - half;
#pragma unroll
      for (int j = 0; j < kEpiBatch; ++j) {
        const int tok = t0 + j;
        if (tok >= t1) break;
        const int m = m0 + tok;
        float y = round_to<T>(tile[tok * kEpiPitch + t]);
        if (region < 2) {
          const float xp = round_to<T>(tile[tok * kEpiPitch + partner]);
          const float rot = i < half ? -xp : xp;
          y = round_to<T>(round_to<T>(y * in.c[j]) + round_to<T>(rot * in.s[j]));
        }
        if (region == 0) {
          static_cast<T*>(e.out)[static_cast<int64_t>(m) * e.ldo + n] = from_f32<T>(y);
        } else if (in.slot[j] >= 0) {
          T* pool = static_cast<T*>(region == 1 ? e.k_pool : e.v_pool);
          pool[(static_cast<int64_t>(in.slot[j]) * e.n_kv_heads + h) * d + i] = from_f32<T>(y);
        }
      }
      return;
    }
    default:
      return;
  }
}

// tile: fp32 [BN][kEpiPitch] in shared memory, nthr threads; thread x owns feature column
// x % 128. Global inputs are loaded for 8 tokens at a time before any of them is used, so an
// epilogue over T tokens costs about T / 8 memory round trips instead of T.
template <typename T>
__device__ void apply_epilogue(const Epilogue& e, float* tile, int n0, int m0, int valid, int N, int nthr = 128) {
  // nthr threads (128 or 256): thread x takes feature x % 128 of the tile and, with 256, every
  // other 8-token batch (x / 128 picks which)
  const int x = threadIdx.x, t = x & 127, ph = x >> 7, nph = nthr >> 7;
  if (e.op == EPI_SILU_MUL) {
    // feature x % 64 of the tile's 64 gate/up pairs, tokens x / 64, + nthr / 64, ...
    const int j = x & 63, n = n0 + j;
    if (n >= N) return;
    T* out = static_cast<T*>(e.out);
    const int f = n0 / 2 + j;
    for (int tok = x >> 6; tok < valid; tok += nthr >> 6) {
      const float g = round_to<T>(tile[tok * kEpiPitch + j]);
      const float u = round_to<T>(tile[tok * kEpiPitch + 64 + j]);
      const float act = round_to<T>(g / (1.0f + expf(-g)));
      out[static_cast<int64_t>(m0 + tok) * e.ldo + f] = from_f32<T>(act * u);
    }
    return;
  }
  if (e.op == EPI_QKV && valid > kEpiBatch) {
    // the tile's positions and pool slots in one round trip, into rows the tile does not use
    // (rows valid .. of the staged tile); then each batch's rotary factors are requested before
    // the thread's previous batch is applied
    int* spos = reinterpret_cast<int*>(tile + static_cast<size_t>(valid) * kEpiPitch);
    int* sslot = spos + valid;
    for (int i = x; i < valid; i += nthr) {
      spos[i] = e.pos[m0 + i];
      sslot[i] = e.slot[m0 + i];
    }
    epi_bar_sync(nthr);
    const int n = n0 + t;
    const int d = e.head_dim, half = d / 2;
    const int qd = e.n_heads * d, kd = e.n_kv_heads * d;
    const int region = n < qd ? 0 : (n < qd + kd ? 1 : 2);
    const int i = (n - (region == 0 ? 0 : (region == 1 ? qd : qd + kd))) % d;
    auto load = [&](int t0, EpiInputs& in) {
#pragma unroll
      for (int j = 0; j < kEpiBatch; ++j) {
        const bool live = t0 + j < valid;
        in.slot[j] = (live && region > 0) ? sslot[t0 + j] : -1;
        in.c[j] = 1.f;
        in.s[j] = 0.f;
        if (live && region < 2) {
          const int64_t off = static_cast<int64_t>(spos[t0 + j]) * half + (i % half);
          in.c[j] = round_to<T>(e.rope_cos[off]);
          in.s[j] = round_to<T>(e.rope_sin[off]);
        }
      }
    };
    if (n >= N) return;
    EpiInputs cur;
    const int step = nph * kEpiBatch;
    if (ph * kEpiBatch < valid) load(ph * kEpiBatch, cur);
    for (int t0 = ph * kEpiBatch; t0 < valid; t0 += step) {
      EpiInputs nxt;
      if (t0 + step < valid) load(t0 + step, nxt);
      apply_epilogue_batch<T>(e, tile, n0, m0, t0, valid, N, cur, t);
      cur = nxt;
    }
    return;
  }
  for (int t0 = ph * kEpiBatch; t0 < valid; t0 += nph * kEpiBatch) {
    EpiInputs in;
    load_epi_inputs<T>(e, n0, m0, t0, valid, N, in, t);
    apply_epilogue_batch<T>(e, tile, n0, m0, t0, valid, N, in, t);
  }
}

}  // namespace specb200
