// Arguments of the persistent layer-stream forward (stream.cu), filled by forward.cu.
#pragma once
#include "gemm.cuh"
#include "kernels.cuh"

namespace specb200 {

constexpr int kStreamBN = 16;      // token rows per call (MMA N)
constexpr int kStreamMaxLayers = 64;

struct StreamLayer {
  const __nv_bfloat16* attn_norm;
  const __nv_bfloat16* mlp_norm;
  const uint8_t* qkv;   // packed 16 KB tiles: [tile][k-block][128 x 64], 128-byte swizzled
  const uint8_t* o;
  const uint8_t* gu;
  const uint8_t* down;
};

struct StreamArgs {
  int n_layers, H, Hq, Hkv, D, I, V;
  float eps, attn_scale;
  int max_positions;
  const __nv_bfloat16* embed;
  const __nv_bfloat16* final_norm;
  const uint8_t* head;
  const float* rope_cos;
  const float* rope_sin;
  StreamLayer layers[kStreamMaxLayers];
  int B, T, M, last_only;
  const int32_t* ids;
  const int32_t* n_new;
  const int32_t* past;
  const int32_t* table;
  int table_stride, bs, num_slots;
  __nv_bfloat16* k_pool;
  __nv_bfloat16* v_pool;
  float* logits;
  __nv_bfloat16* h;
  __nv_bfloat16* q;
  __nv_bfloat16* attn;
  __nv_bfloat16* act;
  int32_t* pos;
  int32_t* slot;
  int* tile_counters;   // kGemmMaxCounters, zero, left zero
  float* partials;
  int max_contrib;
  unsigned* barrier;    // [0] arrivals (zeroed per launch), [1] generation
  int* abort_flag;      // zeroed per launch
  AttnPlan ap;
  int* attn_counters;
  float* attn_partials;
  int32_t* status;
  unsigned long long* trace;  // optional [grid][phases][8] globaltimer stamps
  int prefetch_ahead;         // GEMM phases whose weights are pulled into L2 ahead of use
  int ring_evict_first;       // L2 eviction hint for the ring's weight copies
};

size_t stream_packed_bytes(int N, int K);
size_t stream_smem_bytes();
int stream_max_contrib(int N, int K, int G);
bool stream_units_fit(int N, int K, int G);
int stream_grid_size();
int launch_stream(const StreamArgs& a, const CUtensorMap& map_attn, const CUtensorMap& map_act, int grid,
                  cudaStream_t s);

}  // namespace specb200
