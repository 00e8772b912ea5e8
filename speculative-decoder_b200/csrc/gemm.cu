// K3/K5/K6/K7: the linear layers of the Llama forward.
//
// bf16: a tcgen05 swap-AB GEMM. The weight tile (128 output features x 64 of K, TMA-loaded
// with the 128-byte swizzle) is the MMA's A operand (M = 128) and the token tile (BN tokens x
// 64, BN a multiple of 16 up to 256) is its B operand, so a verify step with 5 tokens costs
// one M=128,N=16 MMA per 64-wide K block while the weights stream from HBM at full rate.
// fp32 products of bf16 inputs are exact and accumulate in TMEM in fp32. Warp roles: warp 8
// issues TMA (weights for the first stages before griddepcontrol.wait, so a kernel launched
// with programmatic dependent launch streams its weights while the previous kernel drains),
// warp 9 issues tcgen05.mma from one thread and owns the TMEM allocation, warps 0-7 read the
// accumulator back (tcgen05.ld, warps w and w + 4 on TMEM lane quarter w, alternate 16-column
// chunks) and run the epilogue (feature x % 128 of the tile per thread, every other 8-token
// batch per warpgroup; a split tile of one 8-token batch is reduced on the first warpgroup,
// larger ones on all eight warps).
//
// fp32: an FFMA kernel with the same tiling and epilogue (tcgen05 has no fp32 inputs and
// TF32 would change results; this path serves fp32 models such as BASELINE config 1).
//
// K is split across CTAs when the output has too few 128-row tiles to fill 148 SMs. Each CTA
// writes its fp32 partial tile to the workspace; the last CTA of a tile (atomic ticket, no
// spin) sums the partials in split order, so results do not depend on scheduling, then runs
// the fused epilogue (RoPE + paged KV write, SiLU*mul, residual add or fp32 store).
#include <algorithm>
#include <mutex>

#include "epilogue.cuh"
#include "gemm.cuh"
#include "kernels.cuh"

namespace specb200 {

// Split-K reduction (when splits > 1) followed by the epilogue. Called by the nthr epilogue
// threads (128 or 256) that hold this CTA's partial tile in `tile`; returns early in every CTA
// but the last of a tile. The partials of each element are summed in split order (0, 1, ...)
// whichever threads do it, so the result does not depend on the path taken.
template <typename T>
__device__ void finish_tile(const GemmShape& s, const Epilogue& e, float* tile, GemmScratch scratch, int tile_id,
                            int split, int n0, int m0, int nthr, unsigned long long* tr = nullptr) {
  __shared__ int sh_last;
  const int x = threadIdx.x, t = x & 127;
  const bool lead = x < 128;
  auto stamp = [&](int k) {  // optional launch record (thread 0)
    if (tr && x == 0) {
      unsigned long long v;
      asm volatile("mov.u64 %0, %globaltimer;" : "=l"(v));
      tr[k] = v;
    }
  };
  const int valid = min(s.BN, s.M - m0);
  if (e.op == EPI_PARTIAL) {  // every split stores its own partial: no ticket, no reduction here
    float* out = static_cast<float*>(e.out) + static_cast<size_t>(split) * s.M * s.N;
    const int n = n0 + t;
    if (n < s.N)
      for (int tok = x >> 7; tok < valid; tok += nthr >> 7)
        out[static_cast<size_t>(m0 + tok) * s.N + n] = tile[tok * kEpiPitch + t];
    return;
  }
  if (s.splits > 1) {
    int* counters = scratch.counters;
    float* parts = scratch.partials;
    const size_t tile_elems = static_cast<size_t>(s.BN) * kTileN;
    float* mine = parts + (static_cast<size_t>(tile_id) * s.splits + split) * tile_elems;
    // Token tiles of more than one epilogue batch store, reduce and finish on all nthr threads
    // in 16-byte pieces (32 per token row); one batch's tile keeps the first 128 threads and
    // fetches its epilogue inputs before the ticket.
    const bool wide = valid > kEpiBatch;
    const int n4 = valid * (kTileN / 4);
    EpiInputs pre;
    if (wide) {
      for (int p = x; p < n4; p += nthr) {
        const int r = p >> 5, c = (p & 31) * 4;
        *reinterpret_cast<float4*>(mine + r * kTileN + c) = *reinterpret_cast<const float4*>(tile + r * kEpiPitch + c);
      }
      __threadfence();
    } else if (lead) {
      for (int tok = 0; tok < valid; ++tok) mine[tok * kTileN + t] = tile[tok * kEpiPitch + t];
      // The first batch's epilogue inputs now, in every split CTA: off the critical path of
      // the CTA that turns out to finish the tile.
      load_epi_inputs<T>(e, n0, m0, 0, valid, s.N, pre, t);
      __threadfence();
    }
    epi_bar_sync(nthr);
    stamp(5);
    if (x == 0) sh_last = (atomicAdd(counters + tile_id, 1) == s.splits - 1);
    epi_bar_sync(nthr);
    stamp(6);
    if (!sh_last) return;
    const float* base = parts + static_cast<size_t>(tile_id) * s.splits * tile_elems;
    constexpr int kSplitBatch = 4;  // splits whose partials are loaded together (summed in split order)
    if (wide) {
      __threadfence();
      constexpr int kRows = 3;  // 16-byte pieces per thread whose loads are in flight together (no spills at 3)
      for (int p0 = x; p0 < n4; p0 += kRows * nthr) {
        float4 acc[kRows];
#pragma unroll
        for (int u = 0; u < kRows; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int sp0 = 0; sp0 < s.splits; sp0 += kSplitBatch) {
          float4 v[kSplitBatch][kRows];
#pragma unroll
          for (int q = 0; q < kSplitBatch; ++q)
#pragma unroll
            for (int u = 0; u < kRows; ++u) {
              const int p = p0 + u * nthr;
              v[q][u] = (sp0 + q < s.splits && p < n4)
                            ? __ldcg(reinterpret_cast<const float4*>(base + (sp0 + q) * tile_elems + (p >> 5) * kTileN) +
                                     (p & 31))
                            : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
          for (int q = 0; q < kSplitBatch; ++q)
#pragma unroll
            for (int u = 0; u < kRows; ++u)
              if (sp0 + q < s.splits) {
                acc[u].x += v[q][u].x; acc[u].y += v[q][u].y; acc[u].z += v[q][u].z; acc[u].w += v[q][u].w;
              }
        }
#pragma unroll
        for (int u = 0; u < kRows; ++u) {
          const int p = p0 + u * nthr;
          if (p < n4) *reinterpret_cast<float4*>(tile + (p >> 5) * kEpiPitch + (p & 31) * 4) = acc[u];
        }
      }
      if (x == 0) counters[tile_id] = 0;
      epi_bar_sync(nthr);
      stamp(7);
      apply_epilogue<T>(e, tile, n0, m0, valid, s.N, nthr);
      return;
    }
    if (!lead) return;  // a one-batch tile is finished on the first 128 threads
    __threadfence();
    for (int t0 = 0; t0 < valid; t0 += kEpiBatch) {
      float acc[kEpiBatch];
#pragma unroll
      for (int j = 0; j < kEpiBatch; ++j) acc[j] = 0.f;
      for (int sp0 = 0; sp0 < s.splits; sp0 += kSplitBatch) {
        float v[kSplitBatch][kEpiBatch];
#pragma unroll
        for (int q = 0; q < kSplitBatch; ++q)
#pragma unroll
          for (int j = 0; j < kEpiBatch; ++j)
            v[q][j] = (sp0 + q < s.splits && t0 + j < valid)
                          ? __ldcg(base + (sp0 + q) * tile_elems + (t0 + j) * kTileN + t)
                          : 0.f;
#pragma unroll
        for (int q = 0; q < kSplitBatch; ++q)
#pragma unroll
          for (int j = 0; j < kEpiBatch; ++j)
            if (sp0 + q < s.splits) acc[j] += v[q][j];
      }
#pragma unroll
      for (int j = 0; j < kEpiBatch; ++j)
        if (t0 + j < valid) tile[(t0 + j) * kEpiPitch + t] = acc[j];
    }
    if (t == 0) counters[tile_id] = 0;
    epi_bar_sync();  // the first 128 threads only from here
    stamp(7);
    apply_epilogue_batch<T>(e, tile, n0, m0, 0, valid, s.N, pre, t);
    for (int t0 = kEpiBatch; t0 < valid; t0 += kEpiBatch) {
      EpiInputs in;
      load_epi_inputs<T>(e, n0, m0, t0, valid, s.N, in, t);
      apply_epilogue_batch<T>(e, tile, n0, m0, t0, valid, s.N, in, t);
    }
    return;
  }
  apply_epilogue<T>(e, tile, n0, m0, valid, s.N, nthr);
}

SPECB200_DEVINL void split_range(const GemmShape& s, int split, int& kb0, int& kb1) {
  kb0 = static_cast<int>(static_cast<int64_t>(s.kblocks) * split / s.splits);
  kb1 = static_cast<int>(static_cast<int64_t>(s.kblocks) * (split + 1) / s.splits);
}

// ------------------------------------------------------------------------------ tcgen05 kernel
constexpr int kTcThreads = 320;  // 8 epilogue warps (two per TMEM lane quarter), the TMA warp, the MMA warp
constexpr int kTcEpiThreads = 256;
constexpr uint32_t kWTileBytes = kTileN * kTileK * 2;  // 16 KB

SPECB200_DEVINL uint32_t tmem_cols_for(int BN) { return BN <= 32 ? 32u : BN <= 64 ? 64u : BN <= 128 ? 128u : 256u; }

__global__ void __launch_bounds__(kTcThreads, 2)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap w_map, const __grid_constant__ CUtensorMap x_map, GemmShape s,
                   Epilogue e, GemmScratch scratch, int32_t* status, int stages) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int BN = s.BN;
  const uint32_t x_bytes = static_cast<uint32_t>(BN) * kTileK * 2;
  const uint32_t stage_bytes = kWTileBytes + x_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + stages * stage_bytes);
  uint64_t* empty = full + stages;
  uint64_t* tmem_full = empty + stages;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tmem_full + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x, split = blockIdx.y, m_tile = blockIdx.z;
  unsigned long long* tr = nullptr;
  if (scratch.trace) {
    const unsigned cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
    if (cta < kGemmTraceCtas) tr = scratch.trace + (static_cast<size_t>(scratch.trace_slot) * kGemmTraceCtas + cta) * 8;
  }
  auto stamp = [&](int k) {
    if (tr) {
      unsigned long long t;
      asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
      tr[k] = t;
    }
  };
  if (threadIdx.x == 0) stamp(0);
  const int tile_id = m_tile * s.n_tiles + n_tile;
  int kb0, kb1;
  split_range(s, split, kb0, kb1);
  const int nkb = kb1 - kb0;
  const uint32_t tmem_cols = tmem_cols_for(BN);

  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(tmem_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_holder, tmem_cols);
    tmem_relinquish();
  }
  pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 8) {
    if (lane == 0) {
      tma_prefetch_desc(&w_map);
      tma_prefetch_desc(&x_map);
      const uint64_t pol_w = l2_policy_evict_first();
      const int pre = min(stages, nkb);
      // Weights do not depend on the previous kernel: start streaming them before the wait.
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], stage_bytes);
        tma_load_2d_hint(smem + i * stage_bytes, &w_map, &full[i], (kb0 + i) * kTileK, n_tile * kTileN, pol_w);
      }
      pdl_wait();
      stamp(1);
      for (int i = 0; i < pre; ++i)
        tma_load_2d(smem + i * stage_bytes + kWTileBytes, &x_map, &full[i], (kb0 + i) * kTileK, m_tile * BN);
      for (int i = pre; i < nkb; ++i) {
        const int st = i % stages;
        if (!mbar_wait_bounded(&empty[st], ((i / stages) - 1) & 1, status, abort_flag)) break;
        mbar_arrive_expect_tx(&full[st], stage_bytes);
        tma_load_2d_hint(smem + st * stage_bytes, &w_map, &full[st], (kb0 + i) * kTileK, n_tile * kTileN, pol_w);
        tma_load_2d(smem + st * stage_bytes + kWTileBytes, &x_map, &full[st], (kb0 + i) * kTileK, m_tile * BN);
      }
      // Tail: wait until the MMAs have released the last use of every stage, so that no
      // tcgen05.commit arrive lands on this CTA's shared memory after it has exited.
      for (int i = max(0, nkb - stages); i < nkb; ++i)
        if (!mbar_wait_bounded(&empty[i % stages], (i / stages) & 1, status, abort_flag)) break;
    }
    __syncwarp();
  } else if (warp == 9) {
    // The whole warp runs the loop and one elected lane issues each MMA: issuing from a lone
    // lane while the others wait diverged costs about a third more per instruction.
    const uint32_t idesc = umma_idesc_bf16(kTileN, BN);
    for (int i = 0; i < nkb; ++i) {
      const int st = i % stages;
      if (!mbar_wait_warp(&full[st], (i / stages) & 1, status, abort_flag)) break;
      if (i == 0 && lane == 0) stamp(2);
      tc_fence_after();
      const uint64_t da = umma_desc_sw128(smem_u32(smem + st * stage_bytes));
      const uint64_t dx = umma_desc_sw128(smem_u32(smem + st * stage_bytes + kWTileBytes));
#pragma unroll
      for (int kk = 0; kk < kTileK / 16; ++kk)
        umma_bf16_elect(tmem_base, da + kk * 2, dx + kk * 2, idesc, (i > 0 || kk > 0) ? 1u : 0u);
      umma_commit_elect(&empty[st]);  // frees the stage once these MMAs have read it
    }
    umma_commit_elect(tmem_full);
    __syncwarp();
  } else {
    pdl_wait();
    const bool ok = mbar_wait_bounded(tmem_full, 0, status, abort_flag);
    if (threadIdx.x == 0) stamp(3);
    tc_fence_after();
    float* tile = reinterpret_cast<float*>(smem);  // the pipeline stages are idle now
    if (ok) {
      // warps w and w + 4 read TMEM lane quarter w, alternate 16-column chunks
      const int q = warp & 3;
      for (int c = (warp >> 2) * 16; c < BN; c += 32) {
        float v[16];
        tmem_ld16(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + c, v);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) tile[(c + j) * kEpiPitch + q * 32 + lane] = v[j];
      }
    }
    epi_bar_sync(kTcEpiThreads);
    if (ok && !*reinterpret_cast<volatile int*>(abort_flag))
      finish_tile<__nv_bfloat16>(s, e, tile, scratch, tile_id, split, n_tile * kTileN, m_tile * BN, kTcEpiThreads, tr);
    if (threadIdx.x == 0) stamp(4);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tmem_cols);
  }
}

// ------------------------------------------------------------------------------ FFMA kernel
constexpr int kSimtThreads = 128;
constexpr int kSimtKC = 256;   // K chunk staged in shared memory
constexpr int kSimtMaxBN = 32;

template <typename T> SPECB200_DEVINL void load4(const T* p, float (&v)[4]);
template <> SPECB200_DEVINL void load4<float>(const float* p, float (&v)[4]) {
  float4 q = *reinterpret_cast<const float4*>(p);
  v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
}
template <> SPECB200_DEVINL void load4<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[4]) {
  uint2 q = *reinterpret_cast<const uint2*>(p);
  __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&q.x), b = *reinterpret_cast<__nv_bfloat162*>(&q.y);
  float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
  v[0] = fa.x; v[1] = fa.y; v[2] = fb.x; v[3] = fb.y;
}

template <typename T>
__global__ void __launch_bounds__(kSimtThreads)
    gemm_simt_kernel(const T* __restrict__ w, const T* __restrict__ x, GemmShape s, Epilogue e, GemmScratch scratch) {
  extern __shared__ float xs[];  // [BN][kSimtKC], reused as the epilogue tile
  pdl_launch_dependents();
  pdl_wait();
  const int n_tile = blockIdx.x, split = blockIdx.y, m_tile = blockIdx.z;
  const int tile_id = m_tile * s.n_tiles + n_tile;
  const int n0 = n_tile * kTileN, m0 = m_tile * s.BN;
  const int BN = s.BN;
  int kb0, kb1;
  split_range(s, split, kb0, kb1);
  const int kbeg = kb0 * kTileK, kend = min(s.K, kb1 * kTileK);
  const int row = n0 + threadIdx.x;
  float acc[kSimtMaxBN];
#pragma unroll
  for (int j = 0; j < kSimtMaxBN; ++j) acc[j] = 0.f;
  for (int k0 = kbeg; k0 < kend; k0 += kSimtKC) {
    const int kc = min(kSimtKC, kend - k0);
    __syncthreads();
    for (int idx = threadIdx.x; idx < BN * kSimtKC; idx += kSimtThreads) {
      const int tok = idx / kSimtKC, kk = idx % kSimtKC;
      float v = 0.f;
      if (m0 + tok < s.M && kk < kc) v = to_f32<T>(x[static_cast<int64_t>(m0 + tok) * s.K + k0 + kk]);
      xs[idx] = v;
    }
    __syncthreads();
    if (row < s.N) {
      const T* wr = w + static_cast<int64_t>(row) * s.K + k0;
      for (int kk = 0; kk < kc; kk += 4) {
        float wv[4];
        load4<T>(wr + kk, wv);
#pragma unroll
        for (int j = 0; j < kSimtMaxBN; ++j) {
          if (j < BN) {
            const float* xr = xs + j * kSimtKC + kk;
            acc[j] = fmaf(wv[0], xr[0], acc[j]);
            acc[j] = fmaf(wv[1], xr[1], acc[j]);
            acc[j] = fmaf(wv[2], xr[2], acc[j]);
            acc[j] = fmaf(wv[3], xr[3], acc[j]);
          }
        }
      }
    }
  }
  __syncthreads();
  float* tile = xs;
#pragma unroll
  for (int j = 0; j < kSimtMaxBN; ++j)
    if (j < BN) tile[j * kEpiPitch + threadIdx.x] = acc[j];
  __syncthreads();
  finish_tile<T>(s, e, tile, scratch, tile_id, split, n0, m0, kSimtThreads);
}

// ------------------------------------------------------------------------------ host side
GemmShape plan_gemm(int M, int N, int K, bool tensor_core, int min_split_kblocks) {
  GemmShape s;
  s.M = M;
  s.N = N;
  s.K = K;
  s.n_tiles = (N + kTileN - 1) / kTileN;
  const int kblocks = (K + kTileK - 1) / kTileK;
  bool split_fill = false;  // fill two CTAs per SM with K-splits rather than smaller token tiles
  if (tensor_core) {
    // The fewest token tiles of at most 256, split evenly (a multiple of 16, the MMA's N
    // granularity): 320 tokens run as 2 x 160, not 256 + 64 with a padded second tile.
    const int mt = (M + 255) / 256;
    s.BN = std::min(256, ((M + mt - 1) / mt + 15) / 16 * 16);
    // Prefill and large batches: halve the token tile (kept a multiple of 16) until the grid
    // covers the 148 SMs (a 512-token q/k/v projection gets 192 CTAs of 128 tokens instead of
    // 96 of 256). Token tiles of at most 160 (two CTAs per SM) with a long K split K instead,
    // once up to eight splits that fill two CTAs per SM leave every CTA at least
    // min_split_kblocks k-blocks (16 by default; 4 for the o projection, whose split partials
    // go to the next RMSNorm, not through a split-K epilogue):
    // each halving re-reads every weight tile once more, and at 32 tokens a CTA streams the
    // whole K (B = 64 down projection: 10 token tiles x 128 k-blocks per CTA).
    if (M > 16) {
      const bool two_per_sm = s.BN <= 160;
      while (s.BN > 32 && s.n_tiles * ((M + s.BN - 1) / s.BN) < 148) {
        if (two_per_sm) {
          const int ctas = s.n_tiles * ((M + s.BN - 1) / s.BN);
          const int want = std::min(8, (2 * 148 + ctas - 1) / ctas);
          if (kblocks / want >= min_split_kblocks) {
            split_fill = true;
            break;
          }
        }
        s.BN = (s.BN / 2 + 15) / 16 * 16;
      }
    }
  } else {
    s.BN = std::min(kSimtMaxBN, ((M + 3) / 4) * 4);
  }
  s.m_tiles = (M + s.BN - 1) / s.BN;
  s.kblocks = (K + kTileK - 1) / kTileK;
  const int ctas = s.n_tiles * s.m_tiles;
  int splits;
  if (tensor_core) {
    // The fewest K-splits that let every CTA's K-range fit its ring of weight stages (so the
    // whole share is prefetched before griddepcontrol.wait and the split-K reduction has few
    // contributors), but never more CTAs than fill the GPU once.
    const int per_stage = kTileN * kTileK * 2 + s.BN * kTileK * 2;
    const int stages = std::max(2, std::min(8, (200 * 1024) / per_stage));
    const int fit = (s.kblocks + stages - 1) / stages;
    const int fill = split_fill ? std::max(1, std::min(8, 2 * 148 / ctas)) : std::max(1, 148 / ctas);
    splits = std::max(1, std::min({fit, fill, 16, s.kblocks}));
  } else {
    splits = (148 + ctas / 2) / ctas;
    splits = std::max(1, std::min(splits, std::min(16, s.kblocks)));
  }
  if (ctas > kGemmMaxCounters) splits = 1;
  s.splits = splits;
  return s;
}

size_t gemm_partials_bytes(const GemmShape& s) {
  return s.splits > 1 ? static_cast<size_t>(s.n_tiles) * s.m_tiles * s.splits * s.BN * kTileN * 4 : 0;
}

size_t gemm_workspace_bytes(const GemmShape& s) { return kGemmCounterBytes + gemm_partials_bytes(s); }

namespace {
int tc_stages(int BN, size_t* smem_bytes) {
  const size_t stage = kWTileBytes + static_cast<size_t>(BN) * kTileK * 2;
  const size_t tile = static_cast<size_t>(BN) * kEpiPitch * 4;
  // Token tiles up to 160 get about 110 KB of ring, so two CTAs share an SM: for decode and
  // verify shapes a CTA of the next GEMM prefetches its weights beside the current one (1.343
  // vs 1.361 ms per B = 1 verify against a 200 KB ring); for large batches one CTA's epilogue
  // runs beside the other's mainloop and twice the tiles fit a wave (B = 64 verify 5.89 vs
  // 7.38 ms, B = 32 4.22 vs 4.81 ms). Larger tiles keep one CTA per SM with a deep ring.
  const size_t budget = BN <= 160 ? 110 * 1024 : 200 * 1024;
  int stages = static_cast<int>(std::min<size_t>(8, budget / stage));
  while (static_cast<size_t>(stages) * stage < tile) ++stages;
  stages = std::max(stages, 2);
  *smem_bytes = 1024 + stages * stage + 256;
  return stages;
}

}  // namespace

// Every kernel of a forward asks for the largest shared-memory carveout, so that CTAs of
// consecutive kernels can share an SM under programmatic dependent launch (an SM runs CTAs of
// one carveout configuration at a time).
bool gemm_prepare() {
  static std::once_flag once;
  static bool ok = false;
  std::call_once(once, [] {
    ok = cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                              cudaSharedmemCarveoutMaxShared) == cudaSuccess;
  });
  return ok;
}

int launch_gemm_tc(const GemmShape& s, const CUtensorMap& w_map, const CUtensorMap& x_map, const Epilogue& epi,
                   GemmScratch scratch, int32_t* status, cudaStream_t stream, bool pdl) {
  // the token tile is the MMA's N: a multiple of 16 from 16 to 256 for M = 128
  if (s.BN < 16 || s.BN > 256 || s.BN % 16) return SPECB200_ERR_ARG;
  size_t smem = 0;
  const int stages = tc_stages(s.BN, &smem);
  static std::mutex mu;
  static size_t smem_set = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (smem > smem_set) {
      if (cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
          cudaSuccess)
        return SPECB200_ERR_CUDA;
      smem_set = smem;
    }
  }
  const cudaError_t err = launch_kernel(gemm_tc_kernel, dim3(s.n_tiles, s.splits, s.m_tiles), dim3(kTcThreads), smem,
                                        stream, pdl, w_map, x_map, s, epi, scratch, status, stages);
  return err == cudaSuccess ? SPECB200_OK : SPECB200_ERR_CUDA;
}

template <typename T>
int launch_gemm_simt(const GemmShape& s, const T* w, const T* x, const Epilogue& epi, GemmScratch scratch,
                     int32_t* status, cudaStream_t stream, bool pdl) {
  (void)status;
  const size_t smem = std::max(static_cast<size_t>(s.BN) * kSimtKC, static_cast<size_t>(s.BN) * kEpiPitch) * 4;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(gemm_simt_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
  });
  if (attr_err != cudaSuccess) return SPECB200_ERR_CUDA;
  cudaError_t err = launch_kernel(gemm_simt_kernel<T>, dim3(s.n_tiles, s.splits, s.m_tiles), dim3(kSimtThreads), smem, stream,
                           pdl, w, x, s, epi, scratch);
  return err == cudaSuccess ? SPECB200_OK : SPECB200_ERR_CUDA;
}
template int launch_gemm_simt<float>(const GemmShape&, const float*, const float*, const Epilogue&, GemmScratch,
                                     int32_t*, cudaStream_t, bool);
template int launch_gemm_simt<__nv_bfloat16>(const GemmShape&, const __nv_bfloat16*, const __nv_bfloat16*,
                                             const Epilogue&, GemmScratch, int32_t*, cudaStream_t, bool);

// ------------------------------------------------------------------------------ TMA descriptors
namespace {
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}
}  // namespace

bool make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint32_t box_inner,
                       uint32_t box_outer) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (inner * 2) % 16) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace specb200

// ------------------------------------------------------------------------------ C ABI
using namespace specb200;
extern "C" int specb200_set_error(int code, const char* msg);

extern "C" size_t specb200_linear_workspace_bytes(int M, int N, int K) {
  GemmShape s = plan_gemm(M, N, K, true);
  GemmShape f = plan_gemm(M, N, K, false);
  return std::max(gemm_workspace_bytes(s), gemm_workspace_bytes(f));
}

extern "C" int specb200_linear(int dtype, const void* w, const void* x, int M, int N, int K, int out_f32, void* y,
                               void* workspace, size_t workspace_bytes, int32_t* status, void* stream) {
  if (M <= 0 || N <= 0 || K <= 0 || K % 8) return specb200_set_error(SPECB200_ERR_ARG, "linear: bad M/N/K (K % 8 == 0)");
  if (!w || !x || !y || !workspace) return specb200_set_error(SPECB200_ERR_ARG, "linear: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (status) cudaMemsetAsync(status, 0, sizeof(int32_t), s);
  Epilogue e = {};
  e.op = EPI_STORE;
  e.out_f32 = out_f32;
  e.out = y;
  e.ldo = N;
  GemmScratch scratch{static_cast<int*>(workspace),
                      reinterpret_cast<float*>(static_cast<char*>(workspace) + kGemmCounterBytes)};
  if (dtype == SPECB200_BF16) {
    GemmShape sh = plan_gemm(M, N, K, true);
    if (workspace_bytes < gemm_workspace_bytes(sh)) return specb200_set_error(SPECB200_ERR_WORKSPACE, "linear: workspace");
    CUtensorMap wm, xm;
    if (!make_tmap_bf16_2d(&wm, w, K, N, kTileK, kTileN) || !make_tmap_bf16_2d(&xm, x, K, M, kTileK, sh.BN))
      return specb200_set_error(SPECB200_ERR_ARG, "linear: TMA descriptor (16-byte alignment?)");
    if (launch_gemm_tc(sh, wm, xm, e, scratch, status, s, false) != SPECB200_OK)
      return specb200_set_error(SPECB200_ERR_CUDA, cudaGetErrorString(cudaGetLastError()));
  } else if (dtype == SPECB200_F32) {
    GemmShape sh = plan_gemm(M, N, K, false);
    if (workspace_bytes < gemm_workspace_bytes(sh)) return specb200_set_error(SPECB200_ERR_WORKSPACE, "linear: workspace");
    if (launch_gemm_simt<float>(sh, static_cast<const float*>(w), static_cast<const float*>(x), e, scratch, status, s,
                                false) != SPECB200_OK)
      return specb200_set_error(SPECB200_ERR_CUDA, cudaGetErrorString(cudaGetLastError()));
  } else {
    return specb200_set_error(SPECB200_ERR_UNSUPPORTED, "linear: dtype");
  }
  return SPECB200_OK;
}
