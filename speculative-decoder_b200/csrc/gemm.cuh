// Linear layers of the Llama forward: Y[M, N] = X[M, K] W[N, K]^T with fused epilogues.
#pragma once
#include "common.cuh"

namespace specb200 {

enum EpilogueOp : int {
  EPI_STORE = 0,     // out[m, n] = acc (fp32 or rounded to the model dtype)
  EPI_RESID = 1,     // out[m, n] = round(out[m, n] + round(acc)): `hidden + proj(x)` in the model dtype
  EPI_SILU_MUL = 2,  // tile rows 0-63 gate, 64-127 up: out[m, n/2 + j] = round(round(silu(round(g))) * round(u))
  EPI_QKV = 3,       // rows of q_proj | k_proj | v_proj: RoPE on q and k, q to out, k and v to the paged pool
  EPI_PARTIAL = 4,   // out (fp32) [split][M][N] = this K split's partial sums; the residual add is
                     // deferred to the following RMSNorm launch (launch_residual_norm)
};

struct Epilogue {
  int op;
  int out_f32;       // EPI_STORE: 1 = fp32 output
  void* out;         // EPI_STORE / EPI_RESID / EPI_SILU_MUL / EPI_QKV (q)
  int64_t ldo;       // row stride of out, in elements
  // EPI_QKV
  void* k_pool;      // this layer's [num_slots, Hkv, d]
  void* v_pool;
  const int32_t* slot;  // [M] pool slot of each token, -1 for padding
  const int32_t* pos;   // [M] absolute position of each token
  const float* rope_cos;  // [max_positions, d/2]
  const float* rope_sin;
  int n_heads, n_kv_heads, head_dim;
};

// Tile shape: 128 output features (one tcgen05 M=128 tile of W rows) x BN tokens.
constexpr int kTileN = 128;
constexpr int kTileK = 64;  // one 128-byte swizzle atom of bf16
constexpr int kEpiPitch = kTileN + 4;  // fp32 epilogue tile row pitch (floats)
// Split-K tickets live in a fixed region at the start of every GEMM workspace that nothing
// else writes; each ticket returns to zero when its tile is done, so the region stays zero
// across calls of any shape. Split-K is only planned when the tile count fits in it.
constexpr int kGemmMaxCounters = 1024;
constexpr size_t kGemmCounterBytes = kGemmMaxCounters * sizeof(int);

struct GemmShape {
  int M, N, K;
  int BN;       // token columns per CTA (multiple of 16, <= 256)
  int splits;   // K splits (deterministic reduction by the last CTA of each tile)
  int n_tiles, m_tiles, kblocks;
};

// Host-side choice of BN and split count for a weight-streaming GEMM on 148 SMs.
// min_split_kblocks: the fewest k-blocks per CTA at which a token tile of at most 160 keeps its
// size and K is split to fill two CTAs per SM, rather than the tile being halved.
GemmShape plan_gemm(int M, int N, int K, bool tensor_core, int min_split_kblocks = 16);
size_t gemm_workspace_bytes(const GemmShape& s);

// Launchers (gemm.cu). w_map is a tensor map over W [N, K] with box {64, 128}; x_map over
// X [M, K] with box {64, BN}. Both 128-byte swizzled bf16.
// counters: kGemmMaxCounters ints that start zero (the kernels leave them zero);
// partials: gemm_partials_bytes(s) of scratch.
struct GemmScratch {
  int* counters;
  float* partials;
  // Optional launch record (globaltimer ns): CTA c (linear block index < kGemmTraceCtas) of
  // launch trace_slot writes trace[(trace_slot * kGemmTraceCtas + c) * 8 + {0..7}] = entry,
  // wait return, first stage at the MMA warp, accumulator ready, end, then with split-K the
  // partial published (after the fence), the ticket taken, the partials summed.
  unsigned long long* trace = nullptr;
  int trace_slot = 0;
};
constexpr int kGemmTraceCtas = 512;
size_t gemm_partials_bytes(const GemmShape& s);
// Function attributes of the GEMM kernels (largest shared-memory carveout); call outside any
// stream capture.
bool gemm_prepare();
int launch_gemm_tc(const GemmShape& s, const CUtensorMap& w_map, const CUtensorMap& x_map, const Epilogue& epi,
                   GemmScratch scratch, int32_t* status, cudaStream_t stream, bool pdl);
template <typename T>
int launch_gemm_simt(const GemmShape& s, const T* w, const T* x, const Epilogue& epi, GemmScratch scratch,
                     int32_t* status, cudaStream_t stream, bool pdl);

// TMA descriptor helpers (forward.cu / gemm.cu).
bool make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint32_t box_inner,
                       uint32_t box_outer);

}  // namespace specb200
