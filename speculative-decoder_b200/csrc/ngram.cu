// K9: n-gram prompt lookup, plus the device-side context bookkeeping of the round.
//
// lookup() at spec/ngram.py:32-45 scans, for n = min(max_n, L-1) down to 1, the starts
// L-n-1 .. 0 and returns the continuation of the first (most recent) start whose n tokens
// equal the last n. Written by the match's END index e = start + n - 1 (0 <= e <= L-2), a
// start is valid for n iff the tokens ending at e agree with the context's suffix for n
// steps. One pass therefore finds, for every e, the suffix-match length ml(e) (capped at
// nmax), and for every n the largest e with ml(e) >= n: a block-wide max per n. The winner is
// the largest n that has any e; the draft copies ctx[e+1 .. L-1] cyclically (the self-
// extending copy of spec/ngram.py:40-43 is out[i] = src[i mod len(src)]). With no match the
// last token repeats (spec/ngram.py:45). Bit-exact with the reference by construction: only
// integer comparisons.
#include "common.cuh"

namespace specb200 {
namespace {

constexpr int kNgramThreads = 256;
constexpr int kMaxN = 8;

__global__ void __launch_bounds__(kNgramThreads)
    ngram_kernel(const int32_t* __restrict__ ctx, int64_t stride, const int32_t* __restrict__ ctx_len, int k, int max_n,
                 int64_t* __restrict__ draft, int32_t* status) {
  pdl_wait();
  const int b = blockIdx.x;
  const int32_t* c = ctx + static_cast<int64_t>(b) * stride;
  const int L = ctx_len[b];
  __shared__ int sh_best[kMaxN + 1][kNgramThreads / 32];
  __shared__ int sh_e, sh_n;
  if (L <= 0 || L > stride) {
    if (threadIdx.x == 0) set_status(status, SPECB200_ERR_RANGE);
    if (threadIdx.x < k) draft[static_cast<int64_t>(b) * k + threadIdx.x] = 0;
    return;
  }
  const int nmax = min(max_n, L - 1);
  int suffix[kMaxN];
#pragma unroll
  for (int j = 0; j < kMaxN; ++j) suffix[j] = (j < nmax) ? c[L - 1 - j] : 0;
  int best[kMaxN + 1];
#pragma unroll
  for (int n = 0; n <= kMaxN; ++n) best[n] = -1;
  for (int e = threadIdx.x; e <= L - 2; e += kNgramThreads) {
    int ml = 0;
#pragma unroll
    for (int j = 0; j < kMaxN; ++j) {
      if (j >= nmax || j > e) break;
      if (c[e - j] != suffix[j]) break;
      ml = j + 1;
    }
#pragma unroll
    for (int n = 1; n <= kMaxN; ++n)
      if (ml >= n) best[n] = max(best[n], e);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int n = 1; n <= kMaxN; ++n) {
    int v = warp_max_i(best[n]);
    if (lane == 0) sh_best[n][warp] = v;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int e = -1, nn = 0;
    for (int n = nmax; n >= 1 && e < 0; --n) {
      int v = -1;
      for (int w = 0; w < kNgramThreads / 32; ++w) v = max(v, sh_best[n][w]);
      if (v >= 0) { e = v; nn = n; }
    }
    sh_e = e;
    sh_n = nn;
  }
  __syncthreads();
  const int e = sh_e;
  for (int i = threadIdx.x; i < k; i += kNgramThreads) {
    int64_t tok;
    if (e < 0) {
      tok = c[L - 1];
    } else {
      const int src_len = L - 1 - e;  // ctx[e+1 .. L-1]
      tok = c[e + 1 + (i % src_len)];
    }
    draft[static_cast<int64_t>(b) * k + i] = tok;
  }
}

__global__ void commit_kernel(int32_t* ctx, int64_t stride, int32_t* ctx_len, const int64_t* draft,
                              const int64_t* n_accepted, const int64_t* next_token, const int32_t* active, int B, int k) {
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  if (active && !active[b]) return;
  const int L = ctx_len[b];
  int n = static_cast<int>(n_accepted[b]);
  n = max(0, min(n, k));
  int32_t* c = ctx + static_cast<int64_t>(b) * stride;
  for (int j = 0; j < n && L + j < stride; ++j) c[L + j] = static_cast<int32_t>(draft[static_cast<int64_t>(b) * k + j]);
  if (L + n < stride) c[L + n] = static_cast<int32_t>(next_token[b]);
  ctx_len[b] = min(L + n + 1, static_cast<int>(stride));
}

__global__ void verify_ids_kernel(const int32_t* ctx, int64_t stride, const int32_t* ctx_len, const int64_t* draft,
                                  const int32_t* active, int B, int k, int32_t* ids, int32_t* past, int32_t* n_new) {
  pdl_wait();
  const int b = blockIdx.x;
  const int j = threadIdx.x;
  if (j == 0 && past) past[b] = max(ctx_len[b] - 1, 0);
  if (j == 0 && n_new) n_new[b] = (active == nullptr || active[b]) ? k + 1 : 0;
  if (j > k) return;
  int32_t v;
  if (j == 0) {
    const int L = ctx_len[b];
    v = L > 0 ? ctx[static_cast<int64_t>(b) * stride + L - 1] : 0;
  } else {
    v = static_cast<int32_t>(draft[static_cast<int64_t>(b) * k + j - 1]);
  }
  ids[static_cast<int64_t>(b) * (k + 1) + j] = v;
}

}  // namespace
}  // namespace specb200

using namespace specb200;
extern "C" int specb200_set_error(int code, const char* msg);

extern "C" int specb200_ngram(const int32_t* ctx, int64_t ctx_stride, const int32_t* ctx_len, int B, int k, int max_n,
                              int64_t* draft, int32_t* status, void* stream) {
  if (B <= 0 || k <= 0 || max_n < 1 || max_n > kMaxN || ctx_stride <= 0)
    return specb200_set_error(SPECB200_ERR_ARG, "ngram: bad B/k/max_n/stride (max_n must be 1..8)");
  if (!ctx || !ctx_len || !draft) return specb200_set_error(SPECB200_ERR_ARG, "ngram: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (status) cudaMemsetAsync(status, 0, sizeof(int32_t), s);
  ngram_kernel<<<B, kNgramThreads, 0, s>>>(ctx, ctx_stride, ctx_len, k, max_n, draft, status);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return specb200_set_error(SPECB200_ERR_CUDA, cudaGetErrorString(e));
  return SPECB200_OK;
}

extern "C" int specb200_commit_tokens(int32_t* ctx, int64_t ctx_stride, int32_t* ctx_len, const int64_t* draft,
                                      const int64_t* n_accepted, const int64_t* next_token, const int32_t* active, int B,
                                      int k, void* stream) {
  if (B <= 0 || k < 0 || ctx_stride <= 0) return specb200_set_error(SPECB200_ERR_ARG, "commit: bad sizes");
  if (!ctx || !ctx_len || !n_accepted || !next_token || (k > 0 && !draft))
    return specb200_set_error(SPECB200_ERR_ARG, "commit: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  commit_kernel<<<(B + 127) / 128, 128, 0, s>>>(ctx, ctx_stride, ctx_len, draft, n_accepted, next_token, active, B, k);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return specb200_set_error(SPECB200_ERR_CUDA, cudaGetErrorString(e));
  return SPECB200_OK;
}

extern "C" int specb200_verify_ids(const int32_t* ctx, int64_t ctx_stride, const int32_t* ctx_len, const int64_t* draft,
                                   const int32_t* active, int B, int k, int32_t* ids, int32_t* past, int32_t* n_new,
                                   void* stream) {
  if (B <= 0 || k < 0 || k > 1023 || ctx_stride <= 0) return specb200_set_error(SPECB200_ERR_ARG, "verify_ids: bad sizes");
  if (!ctx || !ctx_len || !ids || (k > 0 && !draft)) return specb200_set_error(SPECB200_ERR_ARG, "verify_ids: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  verify_ids_kernel<<<B, ((k + 1 + 31) / 32) * 32, 0, s>>>(ctx, ctx_stride, ctx_len, draft, active, B, k, ids, past,
                                                            n_new);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return specb200_set_error(SPECB200_ERR_CUDA, cudaGetErrorString(e));
  return SPECB200_OK;
}

namespace specb200 {
namespace {
__global__ void scatter_tokens_kernel(const int64_t* tok, int B, int k, int j, int64_t* draft, int32_t* ids) {
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int64_t t = tok[b];
  if (draft) draft[static_cast<int64_t>(b) * k + j] = t;
  if (ids) ids[b] = static_cast<int32_t>(t);
}
}  // namespace
}  // namespace specb200

extern "C" int specb200_scatter_tokens(const int64_t* tokens, int B, int k, int j, int64_t* draft, int32_t* ids,
                                       void* stream) {
  if (B <= 0 || !tokens || (draft && (k <= 0 || j < 0 || j >= k)))
    return specb200_set_error(SPECB200_ERR_ARG, "scatter_tokens: bad arguments");
  scatter_tokens_kernel<<<(B + 127) / 128, 128, 0, static_cast<cudaStream_t>(stream)>>>(tokens, B, k, j, draft, ids);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return specb200_set_error(SPECB200_ERR_CUDA, cudaGetErrorString(e));
  return SPECB200_OK;
}
