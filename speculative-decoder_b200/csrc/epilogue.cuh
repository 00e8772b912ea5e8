// Fused GEMM epilogues, shared by the per-layer GEMM kernels (gemm.cu) and the persistent
// layer-stream kernel (stream.cu). Each runs on 128 threads over an fp32 tile held in shared
// memory: tile[token][feature], pitch kEpiPitch, feature j = output column n0 + j.
#pragma once
#include "gemm.cuh"

namespace specb200 {

SPECB200_DEVINL void epi_bar_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// tile: fp32 [BN][kEpiPitch] in shared memory, column j = output feature n0 + j.
// 128 threads; thread t owns feature column t.
// Global loads are issued for 8 tokens at a time before any of them is used, so an
// epilogue over T tokens costs about T / 8 memory round trips instead of T.
constexpr int kEpiBatch = 8;

template <typename T>
__device__ void apply_epilogue(const Epilogue& e, const float* tile, int n0, int m0, int valid, int N) {
  const int t = threadIdx.x;
  const int n = n0 + t;
  switch (e.op) {
    case EPI_STORE: {
      if (n >= N) return;
      for (int tok = 0; tok < valid; ++tok) {
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
      for (int t0 = 0; t0 < valid; t0 += kEpiBatch) {
        float h[kEpiBatch];
#pragma unroll
        for (int j = 0; j < kEpiBatch; ++j)
          h[j] = (t0 + j < valid) ? to_f32<T>(out[static_cast<int64_t>(m0 + t0 + j) * e.ldo + n]) : 0.f;
#pragma unroll
        for (int j = 0; j < kEpiBatch; ++j) {
          if (t0 + j >= valid) break;
          const float proj = round_to<T>(tile[(t0 + j) * kEpiPitch + t]);
          out[static_cast<int64_t>(m0 + t0 + j) * e.ldo + n] = from_f32<T>(h[j] + proj);
        }
      }
      return;
    }
    case EPI_SILU_MUL: {
      if (t >= 64 || n >= N) return;
      T* out = static_cast<T*>(e.out);
      const int f = n0 / 2 + t;
      for (int tok = 0; tok < valid; ++tok) {
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
      for (int t0 = 0; t0 < valid; t0 += kEpiBatch) {
        int pos[kEpiBatch], slot[kEpiBatch];
        float c[kEpiBatch], s[kEpiBatch];
#pragma unroll
        for (int j = 0; j < kEpiBatch; ++j) {
          const bool in = t0 + j < valid;
          pos[j] = in ? e.pos[m0 + t0 + j] : 0;
          slot[j] = (in && region > 0) ? e.slot[m0 + t0 + j] : -1;
        }
        if (region < 2) {
#pragma unroll
          for (int j = 0; j < kEpiBatch; ++j) {
            const int64_t off = static_cast<int64_t>(pos[j]) * half + (i % half);
            c[j] = round_to<T>(e.rope_cos[off]);
            s[j] = round_to<T>(e.rope_sin[off]);
          }
        }
#pragma unroll
        for (int j = 0; j < kEpiBatch; ++j) {
          const int tok = t0 + j;
          if (tok >= valid) break;
          const int m = m0 + tok;
          float y = round_to<T>(tile[tok * kEpiPitch + t]);
          if (region < 2) {
            const float xp = round_to<T>(tile[tok * kEpiPitch + partner]);
            const float rot = i < half ? -xp : xp;
            y = round_to<T>(round_to<T>(y * c[j]) + round_to<T>(rot * s[j]));
          }
          if (region == 0) {
            static_cast<T*>(e.out)[static_cast<int64_t>(m) * e.ldo + n] = from_f32<T>(y);
          } else if (slot[j] >= 0) {
            T* pool = static_cast<T*>(region == 1 ? e.k_pool : e.v_pool);
            pool[(static_cast<int64_t>(slot[j]) * e.n_kv_heads + h) * d + i] = from_f32<T>(y);
          }
        }
      }
      return;
    }
    default:
      return;
  }
}

}  // namespace specb200
