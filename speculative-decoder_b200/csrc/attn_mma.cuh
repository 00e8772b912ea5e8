// Decode / verify attention of up to 16 query rows against one KV head on the tensor cores
// (mma.sync bf16 -> fp32), for the few-row shapes of draft and verify steps.
//
// Same computation as the fp32 attention items (attn_core.cuh) -- softmax(q k^T * scale) v
// over the keys a row may see, lm/forward.py:21-84 via the Hugging Face Llama attention --
// with the two products on the tensor cores: S = Q K^T with m16n8k16 (bf16 Q and K are exact
// operands, fp32 accumulation), and O += P V with m16n8k8 where P is split into a bf16 high
// part and a bf16 remainder (two products), so P keeps about 16 bits of mantissa.
//
// Four warps each take 8 keys of every 32-key block and keep an online softmax (running row
// max m, row sum l, unnormalised O) in registers; at the end the four warps' states merge in
// a fixed order. Rows are the m16 tile's rows: row r of the caller's query buffer.
//
// Shared-memory operand layout ("swizzled row"): a [rows][64] bf16 matrix whose row r keeps its
// 16-byte chunk c at position c ^ (r & 7), so fragment loads and ldmatrix hit distinct banks.
#pragma once
#include "common.cuh"

namespace specb200 {

constexpr int kAmRows = 16;    // query rows (one m16 tile)
constexpr int kAmBlock = 32;   // keys per block (8 per warp)
constexpr int kAmD = 64;       // head dim

// Element offset of (row, col) in a swizzled [rows][64] bf16 matrix.
SPECB200_DEVINL int am_swz(int r, int c) { return r * 64 + ((((c >> 3) ^ (r & 7)) << 3) | (c & 7)); }

SPECB200_DEVINL void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
SPECB200_DEVINL void mma_bf16_1688(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
               : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
               : "r"(a0), "r"(a1), "r"(b0));
}
// Four 8x8 bf16 matrices, transposed: lanes 8j..8j+7 give the row addresses of matrix j.
SPECB200_DEVINL void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
SPECB200_DEVINL uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}
SPECB200_DEVINL void cp_async_16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
SPECB200_DEVINL void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
SPECB200_DEVINL void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
// Wait until at most n (0..3) of this thread's most recent cp.async groups are pending.
SPECB200_DEVINL void cp_async_wait_upto(int n) {
  if (n <= 0) cp_async_wait<0>();
  else if (n == 1) cp_async_wait<1>();
  else if (n == 2) cp_async_wait<2>();
  else cp_async_wait<3>();
}

// Per-warp online-softmax state for rows g = lane / 4 and g + 8 (replicated over the 4 lanes of
// the row group; l is this lane's partial sum, reduced at the end).
struct AmState {
  float o[8][4];   // dims 8 * nt + 2 * (lane % 4) + {0, 1}; [0..1] row g, [2..3] row g + 8
  float m[2], l[2];
  uint32_t qa[4][4];  // Q A-fragments for the 4 k-steps of 16 dims
};

SPECB200_DEVINL void am_init(AmState& st, const __nv_bfloat16* q_s) {
  const int lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
#pragma unroll
  for (int nt = 0; nt < 8; ++nt)
#pragma unroll
    for (int j = 0; j < 4; ++j) st.o[nt][j] = 0.f;
  st.m[0] = st.m[1] = -INFINITY;
  st.l[0] = st.l[1] = 0.f;
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    const int c0 = ks * 16 + tig * 2;
    st.qa[ks][0] = *reinterpret_cast<const uint32_t*>(q_s + am_swz(g, c0));
    st.qa[ks][1] = *reinterpret_cast<const uint32_t*>(q_s + am_swz(g + 8, c0));
    st.qa[ks][2] = *reinterpret_cast<const uint32_t*>(q_s + am_swz(g, c0 + 8));
    st.qa[ks][3] = *reinterpret_cast<const uint32_t*>(q_s + am_swz(g + 8, c0 + 8));
  }
}

// One warp's 8 keys: rows of k_s / v_s (swizzled [.][64] bf16) key0 .. key0 + 7 hold absolute
// keys kabs .. kabs + 7. Key kabs + j is visible to row r iff kabs + j < lim_r and j < nvalid.
// The softmax runs in base 2: logits are scaled by scale * log2(e), so the running maxima m
// (and every partial maximum derived from them) are in log2 units and weights are exp2f(x - m).
SPECB200_DEVINL void am_step(AmState& st, const __nv_bfloat16* k_s, const __nv_bfloat16* v_s, int key0, int kabs,
                             int nvalid, int lim0, int lim1, float scale) {
  const int lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
  float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    const int c0 = ks * 16 + tig * 2;
    const uint32_t b0 = *reinterpret_cast<const uint32_t*>(k_s + am_swz(key0 + g, c0));
    const uint32_t b1 = *reinterpret_cast<const uint32_t*>(k_s + am_swz(key0 + g, c0 + 8));
    mma_bf16_16816(s, st.qa[ks], b0, b1);
  }
  // s[0], s[1]: row g, keys 2 tig + {0, 1}; s[2], s[3]: row g + 8
  float p[4];
  const float sl = scale * 1.4426950408889634f;  // log2(e)
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int lim = half ? lim1 : lim0;
    float x0 = s[2 * half] * sl, x1 = s[2 * half + 1] * sl;
    const int j0 = 2 * tig, j1 = 2 * tig + 1;
    if (j0 >= nvalid || kabs + j0 >= lim) x0 = -INFINITY;
    if (j1 >= nvalid || kabs + j1 >= lim) x1 = -INFINITY;
    float mx = fmaxf(x0, x1);
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_old = st.m[half], m_new = fmaxf(m_old, mx);
    const float alpha = (m_new == -INFINITY) ? 1.f : exp2f(m_old - m_new);
    p[2 * half] = (m_new == -INFINITY) ? 0.f : exp2f(x0 - m_new);
    p[2 * half + 1] = (m_new == -INFINITY) ? 0.f : exp2f(x1 - m_new);
    st.l[half] = st.l[half] * alpha + p[2 * half] + p[2 * half + 1];
    st.m[half] = m_new;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      st.o[nt][2 * half] *= alpha;
      st.o[nt][2 * half + 1] *= alpha;
    }
  }
  // P (16 x 8 keys) as an m16n8k8 A operand, split into bf16 high part and remainder
  const uint32_t a_hi0 = pack_bf16(p[0], p[1]), a_hi1 = pack_bf16(p[2], p[3]);
  const __nv_bfloat162 h0 = *reinterpret_cast<const __nv_bfloat162*>(&a_hi0);
  const __nv_bfloat162 h1 = *reinterpret_cast<const __nv_bfloat162*>(&a_hi1);
  const float2 f0 = __bfloat1622float2(h0), f1 = __bfloat1622float2(h1);
  const uint32_t a_lo0 = pack_bf16(p[0] - f0.x, p[1] - f0.y), a_lo1 = pack_bf16(p[2] - f1.x, p[3] - f1.y);
  // V B-fragments: ldmatrix.trans of rows key0 .. key0 + 7, 16-byte chunk = dim tile
  const int vr = key0 + (lane & 7);
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int chunk = half * 4 + (lane >> 3);
    const uint32_t addr = smem_u32(v_s + vr * 64 + ((chunk ^ (vr & 7)) << 3));
    uint32_t b[4];
    ldmatrix_x4_trans(addr, b[0], b[1], b[2], b[3]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      mma_bf16_1688(st.o[half * 4 + j], a_hi0, a_hi1, b[j]);
      mma_bf16_1688(st.o[half * 4 + j], a_lo0, a_lo1, b[j]);
    }
  }
}

// Merge the four warps' states (fixed order) into rows 0..R-1 of out_o [R][64] (unnormalised,
// relative to out_m, a base-2 maximum) with out_m[R], out_l[R]. scratch: 4 * (16 * 64 + 32) floats. Runs on the
// 128 threads; ends with the caller's named barrier `sync`.
template <typename Sync>
__device__ void am_merge(const AmState& st, float* scratch, int R, float* out_o, float* out_m, float* out_l, Sync sync) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tig = lane & 3;
  float* wo = scratch + warp * (16 * 64 + 32);
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
  sync();
  for (int i = tid; i < R * 64; i += 128) {
    const int r = i >> 6, c = i & 63;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, scratch[w * (16 * 64 + 32) + 16 * 64 + r]);
    float O = 0.f, L = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float* b = scratch + w * (16 * 64 + 32);
      const float mw = b[16 * 64 + r];
      const float wgt = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
      O = fmaf(b[r * 64 + c], wgt, O);
      L = fmaf(b[16 * 64 + 16 + r], wgt, L);
    }
    out_o[r * 64 + c] = O;
    if (c == 0) {
      out_m[r] = M;
      out_l[r] = L;
    }
  }
  sync();
}

}  // namespace specb200
