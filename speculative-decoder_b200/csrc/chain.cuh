// Arguments of the cluster layer-chain forward (chain.cu), filled by forward.cu.
#pragma once
#include "stream.cuh"

namespace specb200 {

constexpr int kChainMaxRows = 8;      // token rows (B * T) per call
constexpr int kChainMaxCluster = 16;
constexpr int kChainOwnMax = 4;       // tiles one CTA finishes in one GEMM phase
constexpr int kChainContribMax = 8;   // CTAs contributing partial sums to one tile
constexpr int kChainMaxSplits = 5;    // attention key splits per (sequence, KV head)
constexpr int kChainMaxSlots = 24;    // weight-ring slots of 16 KB
constexpr int kChainFmaRows = 2;      // calls of at most this many rows run the GEMMs on CUDA cores

enum ChainKind { CK_QKV = 0, CK_O = 1, CK_GU = 2, CK_DOWN = 3 };

// One GEMM kind's shape: N output features in n_tiles tiles of 128, K in kb blocks of 64,
// U = n_tiles * kb units of one packed 16 KB weight tile each.
struct ChainPhase {
  int N, K, n_tiles, kb, U;
};

// Shared-memory carve (byte offsets from the 1024-byte-aligned base), fixed per call shape.
struct ChainLayout {
  int ring_slots;
  int part, keyslot, xn, xp, x32, kvring, pa, pb, qrecv, kvrecv, comb, ostage, tile, stage, misc, total;
  int ownA, ncA, ownB, ncB;   // partial-sum slot grid of the QKV/GU and O/down regions
};

struct ChainArgs {
  int n_layers, H, Hq, Hkv, D, I;
  float eps, attn_scale;
  int max_positions, V;
  const __nv_bfloat16* embed;
  const float* rope_cos;
  const float* rope_sin;
  StreamLayer layers[kStreamMaxLayers];
  int B, T, M;
  const int32_t* ids;
  const int32_t* n_new;
  const int32_t* past;
  const int32_t* table;
  int table_stride, bs, num_slots;
  __nv_bfloat16* k_pool;
  __nv_bfloat16* v_pool;
  __nv_bfloat16* h;           // [M, H] residual stream; holds the last layer's output at exit
  ChainPhase ph[4];           // indexed by ChainKind
  int splits;                 // attention key splits per (sequence, KV head)
  int C;                      // cluster size (CTAs)
  ChainLayout L;
  int ring_evict_first;
  int fma;                    // 1: GEMM units on the CUDA cores (calls of at most 2 token rows)
  int32_t* status;
  unsigned long long* trace;  // optional [C][n_layers * 5][16] profiling record (chain.cu)
};

// Cluster size the chain kernel runs with on this device (16, else 8; 0 if neither fits).
int chain_cluster_size();
// Plan a call: false if the shape is outside the kernel's limits.
bool chain_plan(int n_layers, int H, int Hq, int Hkv, int D, int I, int B, int T, int C, ChainPhase ph[4], int* splits,
                ChainLayout* L);
int launch_chain(const ChainArgs& a, cudaStream_t s);

}  // namespace specb200
