// Seeded Gaussian noise on draft logits: the noisy-copy drafter of BASELINE config 2's second
// variant (a draft that is the target itself with N(0, sigma^2) added to its final logits).
// The reference has no such drafter; the noise must come out the same in the CPU oracle, so it
// is a pure function of (seed, row id, position, vocabulary index):
//
//   (r0, r1, r2, r3) = Philox4x32-10(counter = (v, position, row_id, 0), key = (seed lo, seed hi))
//   u1 = ((r0 >> 8) + 0.5) * 2^-24,  u2 = (r1 >> 8) * 2^-24
//   z  = sqrt(-2 ln u1) * cos(2 pi u2)                       (Box-Muller)
//   logits[b, v] += sigma * z
//
// Philox4x32-10 is the counter-based generator of Salmon, Moraes, Dror and Shaw, "Parallel
// random numbers: as easy as 1, 2, 3" (SC 2011): ten rounds of two 32x32->64-bit multiplies
// with the multipliers 0xD2511F53 and 0xCD9E8D57, the key bumped by the Weyl constants
// 0x9E3779B9 and 0xBB67AE85 between rounds. `position` is the absolute position of the token
// the logits predict (past + n_new of the forward that produced them), so a row's noise at a
// position does not depend on how the positions were batched into forward calls.
#include "common.cuh"

namespace specb200 {
namespace {

constexpr int kNoiseThreads = 256;
constexpr int kNoisePerThread = 4;

SPECB200_DEVINL void mulhilo(uint32_t a, uint32_t b, uint32_t& hi, uint32_t& lo) {
  const uint64_t p = static_cast<uint64_t>(a) * b;
  hi = static_cast<uint32_t>(p >> 32);
  lo = static_cast<uint32_t>(p);
}

SPECB200_DEVINL uint4 philox4x32_10(uint4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    if (r > 0) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
    uint32_t hi0, lo0, hi1, lo1;
    mulhilo(0xD2511F53u, c.x, hi0, lo0);
    mulhilo(0xCD9E8D57u, c.z, hi1, lo1);
    c = make_uint4(hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0);
  }
  return c;
}

__global__ void __launch_bounds__(kNoiseThreads) logit_noise_kernel(float* __restrict__ logits, int V, int64_t ld,
                                                                    const int32_t* __restrict__ past,
                                                                    const int32_t* __restrict__ n_new,
                                                                    const int32_t* __restrict__ row_id, uint32_t k0,
                                                                    uint32_t k1, float sigma) {
  const int b = blockIdx.y;
  const int nn = n_new ? n_new[b] : 1;
  if (nn <= 0) return;  // a row with nothing new this call has no logits to perturb
  const uint32_t pos = static_cast<uint32_t>((past ? past[b] : 0) + nn);
  const uint32_t rid = static_cast<uint32_t>(row_id ? row_id[b] : b);
  float* row = logits + static_cast<int64_t>(b) * ld;
  const int v0 = (blockIdx.x * kNoiseThreads + threadIdx.x) * kNoisePerThread;
#pragma unroll
  for (int i = 0; i < kNoisePerThread; ++i) {
    const int v = v0 + i;
    if (v >= V) break;
    const uint4 r = philox4x32_10(make_uint4(static_cast<uint32_t>(v), pos, rid, 0u), k0, k1);
    const float u1 = (static_cast<float>(r.x >> 8) + 0.5f) * 5.9604644775390625e-8f;  // 2^-24
    const float u2 = static_cast<float>(r.y >> 8) * 5.9604644775390625e-8f;
    const float z = sqrtf(-2.0f * logf(u1)) * cosf(6.2831853071795864769f * u2);
    row[v] = fmaf(sigma, z, row[v]);
  }
}

}  // namespace
}  // namespace specb200

using namespace specb200;
extern "C" int specb200_set_error(int code, const char* msg);

extern "C" int specb200_logit_noise(float* logits, int B, int V, int64_t ld, const int32_t* past, const int32_t* n_new,
                                    const int32_t* row_id, uint64_t seed, float sigma, void* stream) {
  if (!logits || B <= 0 || V <= 0 || ld < V || !(sigma >= 0.f))
    return specb200_set_error(SPECB200_ERR_ARG, "logit_noise: bad arguments");
  if (B > 65535) return specb200_set_error(SPECB200_ERR_ARG, "logit_noise: at most 65535 rows");
  const int per_block = kNoiseThreads * kNoisePerThread;
  dim3 grid((V + per_block - 1) / per_block, B);
  logit_noise_kernel<<<grid, kNoiseThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      logits, V, ld, past, n_new, row_id, static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32), sigma);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return specb200_set_error(SPECB200_ERR_CUDA, cudaGetErrorString(e));
  return SPECB200_OK;
}
