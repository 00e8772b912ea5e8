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

template <typename T>
__global__ void __launch_bounds__(256)
    rmsnorm_kernel(const T* __restrict__ x, const T* __restrict__ w, int H, float eps, T* __restrict__ y,
                   const int32_t* __restrict__ sel_n_new, int T_tokens) {
  pdl_launch_dependents();
  pdl_wait();
  const int row = blockIdx.x;
  // A masked-out row (n_new == 0) selects its first token: finite, and never read back.
  const int64_t src = sel_n_new ? static_cast<int64_t>(row) * T_tokens + max(sel_n_new[row] - 1, 0) : row;
  const T* xr = x + src * H;
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float v = to_f32<T>(xr[i]);
    ss = fmaf(v, v, ss);
  }
  __shared__ float sh[8];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) sh[0] = v;
  }
  __syncthreads();
  const float var = sh[0] / static_cast<float>(H);
  const float r = 1.0f / sqrtf(var + eps);
  T* yr = y + static_cast<int64_t>(row) * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float nx = round_to<T>(to_f32<T>(xr[i]) * r);
    yr[i] = from_f32<T>(to_f32<T>(w[i]) * nx);
  }
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
  cudaError_t e = launch_kernel(rmsnorm_kernel<T>, dim3(rows), dim3(256), 0, s, pdl, x, w, H, eps, y, sel_n_new, T_tokens);
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
