// Causal paged attention for prefill shapes on the tensor cores (bf16, d = 64, more than 16
// query rows per KV head): the reference's SDPA over the gathered cache with its mask
// (lm/forward.py:44-49,62-63), flash-attention style.
//
// A CTA of 4 warps takes 64 query rows of one (sequence, KV head); row r is token r / G of
// query head g G + r % G. Each warp owns 16 rows and keeps their online softmax in registers
// (AmState of attn_mma.cuh). Keys stream through shared memory in blocks of 64 (K and V,
// cp.async, double buffered) straight from the paged pool. Per block a warp computes
// S = Q K^T for the block's 8-key groups that any of its rows may see (m16n8k16), rescales its
// running output once, and adds P V (m16n8k8 on a bf16 high part and remainder of P, as the
// decode kernels do). The CTA stops at the last key any of its rows may see. No split of the
// key range, so no partials and no merge: each warp writes its rows once.
#pragma once
#include "attn_core.cuh"
#include "attn_mma.cuh"

namespace specb200 {

constexpr int kApWarps = 4;
constexpr int kApThreads = kApWarps * 32;
constexpr int kApRows = kApWarps * kAmRows;  // 64 query rows per CTA
constexpr int kApKeys = 64;                  // keys per shared-memory block

struct ApSmem {
  __nv_bfloat16 q[kApWarps][kAmRows * 64];  // each warp's 16 rows, swizzled
  __nv_bfloat16 kv[2][2][kApKeys * 64];     // [buffer][K, V][key][64], swizzled
};

// One warp's pass over a 64-key block held in k_s / v_s (rows 0..63 = absolute keys kabs ..).
// Key kabs + j is visible to the warp's row g (g + 8) iff kabs + j < lim0 (lim1); 8-key groups
// at or past ngrp are skipped (no row of the warp sees them). sl = scale * log2(e).
SPECB200_DEVINL void ap_block(AmState& st, const __nv_bfloat16* k_s, const __nv_bfloat16* v_s, int kabs, int ngrp,
                              int lim0, int lim1, float sl) {
  const int lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
  float s[8][4];
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
    if (nt < ngrp) {
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const int c0 = ks * 16 + tig * 2;
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(k_s + am_swz(nt * 8 + g, c0));
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(k_s + am_swz(nt * 8 + g, c0 + 8));
        mma_bf16_16816(s[nt], st.qa[ks], b0, b1);
      }
    }
  }
  // mask, block maxima per row half, one rescale of the running state
  float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
  for (int nt = 0; nt < 8; ++nt)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int half = j >> 1, key = kabs + nt * 8 + 2 * tig + (j & 1);
      float x = s[nt][j] * sl;
      if (nt >= ngrp || key >= (half ? lim1 : lim0)) x = -INFINITY;
      s[nt][j] = x;
      mx[half] = fmaxf(mx[half], x);
    }
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    float m = mx[half];
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    const float m_old = st.m[half], m_new = fmaxf(m_old, m);
    const float alpha = (m_new == -INFINITY) ? 1.f : exp2f(m_old - m_new);
    float sum = 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float p0 = (m_new == -INFINITY) ? 0.f : exp2f(s[nt][2 * half] - m_new);
      const float p1 = (m_new == -INFINITY) ? 0.f : exp2f(s[nt][2 * half + 1] - m_new);
      s[nt][2 * half] = p0;
      s[nt][2 * half + 1] = p1;
      sum += p0 + p1;
    }
    st.l[half] = st.l[half] * alpha + sum;
    st.m[half] = m_new;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      st.o[nt][2 * half] *= alpha;
      st.o[nt][2 * half + 1] *= alpha;
    }
  }
  // O += P V per 8-key group: P (16 x 8) as the m16n8k8 A operand in a bf16 high part and
  // remainder, V's B fragments by ldmatrix.trans of the group's 8 rows
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    if (nt >= ngrp) break;
    const uint32_t a_hi0 = pack_bf16(s[nt][0], s[nt][1]), a_hi1 = pack_bf16(s[nt][2], s[nt][3]);
    const float2 f0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&a_hi0));
    const float2 f1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&a_hi1));
    const uint32_t a_lo0 = pack_bf16(s[nt][0] - f0.x, s[nt][1] - f0.y);
    const uint32_t a_lo1 = pack_bf16(s[nt][2] - f1.x, s[nt][3] - f1.y);
    const int vr = nt * 8 + (lane & 7);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int chunk = half * 4 + (lane >> 3);
      uint32_t b[4];
      ldmatrix_x4_trans(smem_u32(v_s + vr * 64 + ((chunk ^ (vr & 7)) << 3)), b[0], b[1], b[2], b[3]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        mma_bf16_1688(st.o[half * 4 + j], a_hi0, a_hi1, b[j]);
        mma_bf16_1688(st.o[half * 4 + j], a_lo0, a_lo1, b[j]);
      }
    }
  }
}

// Grid (ceil(T G / 64), Hkv, B), kApThreads threads.
static __device__ void attention_prefill_cta(const AttnArgs& a, ApSmem& sm) {
  constexpr int D = 64;
  const int b = blockIdx.z, g = blockIdx.y;
  const int G = a.Hq / a.Hkv, R = a.T * G;
  const int r0 = blockIdx.x * kApRows;
  const int past = a.past[b], nn = a.n_new[b], total = past + nn;
  if (nn <= 0 || r0 >= R) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rlast = min(R, r0 + kApRows) - 1;
  const int kmax = min(total, past + rlast / G + 1);  // keys any row of the CTA may see
  const __nv_bfloat16* q = static_cast<const __nv_bfloat16*>(a.q);
  const __nv_bfloat16* kp = static_cast<const __nv_bfloat16*>(a.k_pool);
  const __nv_bfloat16* vp = static_cast<const __nv_bfloat16*>(a.v_pool);
  const int32_t* table = a.table + static_cast<int64_t>(b) * a.table_stride;

  // keys [k0, k0 + 64) into buffer `buf` (one cp.async group); rows at or past kmax are zero
  auto load_block = [&](int k0, int buf) {
    const int nk = min(kApKeys, kmax - k0);
    // one task per (key, K or V, row half): one slot lookup per four 16-byte copies
    for (int idx = tid; idx < kApKeys * 4; idx += kApThreads) {
      const int kr = idx >> 2, isv = (idx >> 1) & 1, c0 = (idx & 1) * 4;
      __nv_bfloat16* dst = sm.kv[buf][isv];
      if (kr < nk) {
        const int key = k0 + kr;
        const int64_t sl = static_cast<int64_t>(__ldg(table + key / a.bs)) * a.bs + key % a.bs;
        const __nv_bfloat16* src = (isv ? vp : kp) + (sl * a.Hkv + g) * D;
#pragma unroll
        for (int cc = c0; cc < c0 + 4; ++cc) cp_async_16(dst + am_swz(kr, cc * 8), src + cc * 8);
      } else {
#pragma unroll
        for (int cc = c0; cc < c0 + 4; ++cc) *reinterpret_cast<uint4*>(dst + am_swz(kr, cc * 8)) = make_uint4(0, 0, 0, 0);
      }
    }
    cp_async_commit();
  };
  load_block(0, 0);
  // the CTA's query rows (zero past R)
  for (int i = tid; i < kApRows * 8; i += kApThreads) {
    const int rr = i >> 3, c8 = i & 7, r = r0 + rr;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < R) {
      const int t = r / G, h = g * G + r % G;
      v = *reinterpret_cast<const uint4*>(q + (static_cast<int64_t>(b * a.T + t) * a.Hq + h) * D + c8 * 8);
    }
    *reinterpret_cast<uint4*>(&sm.q[rr >> 4][am_swz(rr & 15, c8 * 8)]) = v;
  }
  __syncthreads();
  AmState st;
  am_init(st, sm.q[warp]);
  const int ra = r0 + warp * kAmRows + (lane >> 2), rb = ra + 8;
  const int lim0 = ra < R ? min(past + ra / G + 1, total) : 0;
  const int lim1 = rb < R ? min(past + rb / G + 1, total) : 0;
  const int wfirst = r0 + warp * kAmRows;
  const int wlim = wfirst < R ? min(total, past + (min(R, wfirst + kAmRows) - 1) / G + 1) : 0;  // warp's last key + 1
  const float sl = a.scale * 1.4426950408889634f;  // log2(e)
  const int nblk = (kmax + kApKeys - 1) / kApKeys;
  for (int i = 0; i < nblk; ++i) {
    const int buf = i & 1;
    if (i + 1 < nblk) {
      load_block((i + 1) * kApKeys, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // block i is in shared memory for every thread
    const int k0 = i * kApKeys;
    const int ngrp = min(8, max(0, (wlim - k0 + 7) / 8));  // warp-uniform
    if (ngrp > 0) ap_block(st, sm.kv[buf][0], sm.kv[buf][1], k0, ngrp, lim0, lim1, sl);
    __syncthreads();  // every warp is done with the buffer before it is refilled
  }
  // rows g and g + 8 of the warp's tile: O / l to bf16
  float l0 = st.l[0], l1 = st.l[1];
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out);
  const int tig = lane & 3;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int r = half ? rb : ra;
    if (r >= R) continue;
    const float l = half ? l1 : l0;
    const float inv = l > 0.f ? 1.0f / l : 0.f;
    const int t = r / G, h = g * G + r % G;
    __nv_bfloat16* orow = out + (static_cast<int64_t>(b * a.T + t) * a.Hq + h) * D;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int c = nt * 8 + 2 * tig;
      *reinterpret_cast<__nv_bfloat162*>(orow + c) =
          __floats2bfloat162_rn(st.o[nt][2 * half] * inv, st.o[nt][2 * half + 1] * inv);
    }
  }
}

}  // namespace specb200
