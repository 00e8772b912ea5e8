// K1 embedding gather (+ per-token position and paged slot), K2 RMSNorm.
//
// prep: for token m = b*T + t, position = past[b] + t and, for real tokens (t < n_new[b]),
// the pool slot block_table[b][pos / bs] * bs + pos % bs: the slot arithmetic of
// cache/paged.py:73-76, computed on the device instead of the host SlotMap of
// cache/kv.py:79-99. Padded tokens get slot -1 (their K/V are never written, as
// write_index excludes them at cache/kv.py:104-106). The embedding row is copied into the
// residual stream (lm/forward.py:52).
//
// rmsnorm: LlamaRMSNorm (transformers/models/llama/modeling_llama.py:62-67): the mean of
// squares in fp32, x * rsqrt(var + eps) rounded to the activation dtype, then multiplied by
// the weight in that dtype. With a row selection it also does lm/forward.py:66-67 (keep each
// row's last real token) before the final norm.
#include "common.cuh"
#include "kernels.cuh"

namespace specb200 {

template <typename T>
__global__ void __launch_bounds__(128)
    prep_embed_kernel(const int32_t* __restrict__ ids, const int32_t* __restrict__ n_new,
                      const int32_t* __restrict__ past, const int32_t* __restrict__ table, int table_stride, int bs,
                      int num_slots, int max_positions, int Tt, int V, int H, const T* __restrict__ embed,
                      T* __restrict__ hidden, int32_t* __restrict__ pos_out, int32_t* __restrict__ slot_out,
                      int32_t* status) {
  pdl_launch_dependents();
  pdl_wait();
  const int m = blockIdx.x;
  const int b = m / Tt, t = m % Tt;
  __shared__ int sh_id;
  if (threadIdx.x == 0) {
    const int pos = past[b] + t;
    int slot = -1;
    if (t < n_new[b]) {
      const int blk = pos / bs;
      if (pos >= max_positions || blk >= table_stride) {
        set_status(status, SPECB200_ERR_RANGE);
      } else {
        const int64_t s = static_cast<int64_t>(table[static_cast<int64_t>(b) * table_stride + blk]) * bs + pos % bs;
        if (s < 0 || s >= num_slots) set_status(status, SPECB200_ERR_RANGE);
        else slot = static_cast<int>(s);
      }
    }
    pos_out[m] = min(pos, max_positions - 1);
    slot_out[m] = slot;
    int id = ids[m];
    if (id < 0 || id >= V) {
      set_status(status, SPECB200_ERR_RANGE);
      id = 0;
    }
    sh_id = id;
  }
  __syncthreads();
  const T* src = embed + static_cast<int64_t>(sh_id) * H;
  T* dst = hidden + static_cast<int64_t>(m) * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) dst[i] = src[i];
}

// One CTA per output row; each thread holds up to kNormChunks 16-byte chunks of the row in
// registers (H <= 256 * kNormChunks * 16 / sizeof(T)), so the row is read from memory once; the
// weight chunks are loaded before griddepcontrol.wait (parameters, not produced upstream).
constexpr int kNormThreads = 256;
constexpr int kNormChunks = 4;

template <typename T>
SPECB200_DEVINL void unpack_chunk(const uint4& v, float (&f)[16 / sizeof(T)]);
template <>
SPECB200_DEVINL void unpack_chunk<__nv_bfloat16>(const uint4& v, float (&f)[8]) {
  const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(u[i] << 16);
    f[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
  }
}
template <>
SPECB200_DEVINL void unpack_chunk<float>(const uint4& v, float (&f)[4]) {
  f[0] = __uint_as_float(v.x);
  f[1] = __uint_as_float(v.y);
  f[2] = __uint_as_float(v.z);
  f[3] = __uint_as_float(v.w);
}
template <typename T>
SPECB200_DEVINL uint4 pack_chunk(const float (&f)[16 / sizeof(T)]);
template <>
SPECB200_DEVINL uint4 pack_chunk<__nv_bfloat16>(const float (&f)[8]) {
  uint32_t u[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 p = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    u[i] = *reinterpret_cast<const uint32_t*>(&p);
  }
  return make_uint4(u[0], u[1], u[2], u[3]);
}
template <>
SPECB200_DEVINL uint4 pack_chunk<float>(const float (&f)[4]) {
  return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
}

template <typename T>
__global__ void __launch_bounds__(kNormThreads)
    rmsnorm_kernel(const T* __restrict__ x, const T* __restrict__ w, int H, float eps, T* __restrict__ y,
                   const int32_t* __restrict__ sel_n_new, int T_tokens) {
  constexpr int E = 16 / sizeof(T);  // elements per chunk
  pdl_launch_dependents();
  const int row = blockIdx.x, tid = threadIdx.x;
  const int nch = H / E;
  const bool vec = (H % E == 0) && nch <= kNormThreads * kNormChunks &&
                   ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  uint4 wv[kNormChunks];
  if (vec) {
#pragma unroll
    for (int i = 0; i < kNormChunks; ++i) {
      const int c = tid + i * kNormThreads;
      wv[i] = c < nch ? __ldg(reinterpret_cast<const uint4*>(w) + c) : make_uint4(0, 0, 0, 0);
    }
  }
  pdl_wait();
  // A masked-out row (n_new == 0) selects its first token: finite, and never read back.
  const int64_t src = sel_n_new ? static_cast<int64_t>(row) * T_tokens + max(sel_n_new[row] - 1, 0) : row;
  const T* xr = x + src * H;
  T* yr = y + static_cast<int64_t>(row) * H;
  __shared__ float sh[kNormThreads / 32];
  auto block_sum = [&](float v) {
    v = warp_sum(v);
    if ((tid & 31) == 0) sh[tid >> 5] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < kNormThreads / 32; ++i) t += sh[i];
    return t;
  };
  if (vec) {
    uint4 xv[kNormChunks];
#pragma unroll
    for (int i = 0; i < kNormChunks; ++i) {
      const int c = tid + i * kNormThreads;
      xv[i] = c < nch ? __ldcg(reinterpret_cast<const uint4*>(xr) + c) : make_uint4(0, 0, 0, 0);
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kNormChunks; ++i) {
      float f[E];
      unpack_chunk<T>(xv[i], f);
#pragma unroll
      for (int e = 0; e < E; ++e) ss = fmaf(f[e], f[e], ss);
    }
    const float r = 1.0f / sqrtf(block_sum(ss) / static_cast<float>(H) + eps);
#pragma unroll
    for (int i = 0; i < kNormChunks; ++i) {
      const int c = tid + i * kNormThreads;
      if (c >= nch) break;
      float f[E], g[E];
      unpack_chunk<T>(xv[i], f);
      unpack_chunk<T>(wv[i], g);
#pragma unroll
      for (int e = 0; e < E; ++e) f[e] = g[e] * round_to<T>(f[e] * r);
      reinterpret_cast<uint4*>(yr)[c] = pack_chunk<T>(f);
    }
    return;
  }
  float ss = 0.f;
  for (int i = tid; i < H; i += kNormThreads) {
    const float v = to_f32<T>(xr[i]);
    ss = fmaf(v, v, ss);
  }
  const float r = 1.0f / sqrtf(block_sum(ss) / static_cast<float>(H) + eps);
  for (int i = tid; i < H; i += kNormThreads) {
    const float nx = round_to<T>(to_f32<T>(xr[i]) * r);
    yr[i] = from_f32<T>(to_f32<T>(w[i]) * nx);
  }
}

// The residual update deferred by an EPI_PARTIAL GEMM, then RMSNorm: for each output row
//   h = round(h + round(sum over splits of the partials, in split order))   (EPI_RESID's rounding)
//   y = w * round(h * rsqrt(mean(h^2) + eps))                              (rmsnorm_kernel's)
// with h written back to the residual stream. One CTA per row, 8 elements per thread in
// registers (H <= 8 * kNormThreads); all partial loads of a thread are in flight together.
constexpr int kResidMaxSplits = 8;

__global__ void __launch_bounds__(kNormThreads)
    residual_norm_kernel(__nv_bfloat16* __restrict__ h, const float* __restrict__ parts, int splits, int M, int H,
                         const __nv_bfloat16* __restrict__ w, float eps, __nv_bfloat16* __restrict__ y,
                         const int32_t* __restrict__ sel_n_new, int T_tokens) {
  pdl_launch_dependents();
  const int row = blockIdx.x, tid = threadIdx.x;
  const int c = tid;  // 8-element chunk of the row
  const bool live = c * 8 < H;
  uint4 wv = live ? __ldg(reinterpret_cast<const uint4*>(w) + c) : make_uint4(0, 0, 0, 0);
  pdl_wait();
  const int64_t src = sel_n_new ? static_cast<int64_t>(row) * T_tokens + max(sel_n_new[row] - 1, 0) : row;
  float hv[8];
  float ss = 0.f;
  if (live) {
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    float4 pv[kResidMaxSplits][2];
#pragma unroll
    for (int sp = 0; sp < kResidMaxSplits; ++sp) {
      if (sp < splits) {
        const float4* p = reinterpret_cast<const float4*>(parts + (static_cast<size_t>(sp) * M + src) * H) + 2 * c;
        pv[sp][0] = __ldcg(p);
        pv[sp][1] = __ldcg(p + 1);
      }
    }
    const uint4 hb = __ldcg(reinterpret_cast<const uint4*>(h + src * H) + c);
#pragma unroll
    for (int sp = 0; sp < kResidMaxSplits; ++sp) {
      if (sp < splits) {
        acc[0] += pv[sp][0].x; acc[1] += pv[sp][0].y; acc[2] += pv[sp][0].z; acc[3] += pv[sp][0].w;
        acc[4] += pv[sp][1].x; acc[5] += pv[sp][1].y; acc[6] += pv[sp][1].z; acc[7] += pv[sp][1].w;
      }
    }
    float hf[8];
    unpack_chunk<__nv_bfloat16>(hb, hf);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      hv[e] = round_to<__nv_bfloat16>(hf[e] + round_to<__nv_bfloat16>(acc[e]));
      ss = fmaf(hv[e], hv[e], ss);
    }
    reinterpret_cast<uint4*>(h + src * H)[c] = pack_chunk<__nv_bfloat16>(hv);
  }
  __shared__ float sh[kNormThreads / 32];
  ss = warp_sum(ss);
  if ((tid & 31) == 0) sh[tid >> 5] = ss;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) t += sh[i];
  const float r = 1.0f / sqrtf(t / static_cast<float>(H) + eps);
  if (live) {
    float g[8];
    unpack_chunk<__nv_bfloat16>(wv, g);
#pragma unroll
    for (int e = 0; e < 8; ++e) hv[e] = g[e] * round_to<__nv_bfloat16>(hv[e] * r);
    reinterpret_cast<uint4*>(y + static_cast<int64_t>(row) * H)[c] = pack_chunk<__nv_bfloat16>(hv);
  }
}

int launch_residual_norm(__nv_bfloat16* h, const float* parts, int splits, int M, int rows, int H,
                         const __nv_bfloat16* w, float eps, __nv_bfloat16* y, const int32_t* sel_n_new, int T_tokens,
                         cudaStream_t s, bool pdl) {
  if (splits < 1 || splits > kResidMaxSplits || H % 8 != 0 || H > 8 * kNormThreads) return SPECB200_ERR_UNSUPPORTED;
  const cudaError_t e = launch_kernel(residual_norm_kernel, dim3(rows), dim3(kNormThreads), 0, s, pdl, h, parts, splits, M,
                                      H, w, eps, y, sel_n_new, T_tokens);
  return e == cudaSuccess ? SPECB200_OK : SPECB200_ERR_CUDA;
}

bool residual_norm_fits(int splits, int H) { return splits >= 1 && splits <= kResidMaxSplits && H % 8 == 0 && H <= 8 * kNormThreads; }

bool norm_prepare() {
  // the largest carveout, as every kernel of a forward, so that consecutive kernels share SMs
  bool ok = true;
  for (const void* f : {reinterpret_cast<const void*>(rmsnorm_kernel<float>),
                        reinterpret_cast<const void*>(rmsnorm_kernel<__nv_bfloat16>),
                        reinterpret_cast<const void*>(prep_embed_kernel<float>),
                        reinterpret_cast<const void*>(prep_embed_kernel<__nv_bfloat16>),
                        reinterpret_cast<const void*>(residual_norm_kernel)})
    ok = ok && cudaFuncSetAttribute(f, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared) ==
                   cudaSuccess;
  return ok;
}

template <typename T>
int launch_prep_embed(const PrepArgs& a, const T* embed, T* hidden, cudaStream_t s, bool pdl) {
  cudaError_t e = launch_kernel(prep_embed_kernel<T>, dim3(a.M), dim3(128), 0, s, pdl, a.ids, a.n_new, a.past, a.table,
                                a.table_stride, a.bs, a.num_slots, a.max_positions, a.T, a.V, a.H, embed, hidden,
                                a.pos_out, a.slot_out, a.status);
  return e == cudaSuccess ? SPECB200_OK : SPECB200_ERR_CUDA;
}

template <typename T>
int launch_rmsnorm(const T* x, const T* w, int rows, int H, float eps, T* y, const int32_t* sel_n_new, int T_tokens,
                   cudaStream_t s, bool pdl) {
  cudaError_t e =
      launch_kernel(rmsnorm_kernel<T>, dim3(rows), dim3(kNormThreads), 0, s, pdl, x, w, H, eps, y, sel_n_new, T_tokens);
  return e == cudaSuccess ? SPECB200_OK : SPECB200_ERR_CUDA;
}

template int launch_prep_embed<float>(const PrepArgs&, const float*, float*, cudaStream_t, bool);
template int launch_prep_embed<__nv_bfloat16>(const PrepArgs&, const __nv_bfloat16*, __nv_bfloat16*, cudaStream_t, bool);
template int launch_rmsnorm<float>(const float*, const float*, int, int, float, float*, const int32_t*, int, cudaStream_t,
                                   bool);
template int launch_rmsnorm<__nv_bfloat16>(const __nv_bfloat16*, const __nv_bfloat16*, int, int, float, __nv_bfloat16*,
                                           const int32_t*, int, cudaStream_t, bool);

}  // namespace specb200

using namespace specb200;
extern "C" int specb200_set_error(int code, const char* msg);

extern "C" int specb200_rmsnorm(int dtype, const void* x, const void* weight, int M, int H, float eps, void* y,
                                void* stream) {
  if (M <= 0 || H <= 0 || !x || !weight || !y) return specb200_set_error(SPECB200_ERR_ARG, "rmsnorm: bad arguments");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc;
  if (dtype == SPECB200_BF16)
    rc = launch_rmsnorm<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(weight), M,
                                       H, eps, static_cast<__nv_bfloat16*>(y), nullptr, 1, s, false);
  else if (dtype == SPECB200_F32)
    rc = launch_rmsnorm<float>(static_cast<const float*>(x), static_cast<const float*>(weight), M, H, eps,
                               static_cast<float*>(y), nullptr, 1, s, false);
  else
    return specb200_set_error(SPECB200_ERR_UNSUPPORTED, "rmsnorm: dtype");
  if (rc != SPECB200_OK) return specb200_set_error(rc, cudaGetErrorString(cudaGetLastError()));
  return SPECB200_OK;
}
