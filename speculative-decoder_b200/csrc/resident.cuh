// Resident decode schedule (resident.cu): the whole decode step of a small bf16 Llama -- every
// layer and the LM head -- as ONE cooperative launch with one CTA per SM.
#pragma once
#include "common.cuh"

namespace specb200 {

constexpr int kResConsumers = 256;                 // 8 compute warps
constexpr int kResThreads = kResConsumers + 32;    // + 1 weight-producer warp
constexpr int kResMaxRows = 4;                     // token rows per call (B * T)
constexpr int kResSlot = 16384;                    // bytes per weight-ring slot
constexpr int kResMaxSlots = 16;
constexpr int kResMaxLayers = 64;
constexpr int kResMaxHidden = 1024;              // draft-class models
constexpr int kResMaxWords = 256;                  // output words per CTA per phase per row
constexpr int kResAttRow = 33;                     // uint4 packets per attention partial row (64 o, m, l)
constexpr int kResMaxQRows = 16;                   // query rows per attention item (T * G)
constexpr size_t kResRegionBytes = 8u << 20;       // fixed workspace region (packets + control words)

struct ResLayer {
  const __nv_bfloat16* attn_norm;
  const __nv_bfloat16* w_qkv;   // [(Hq + 2 Hkv) 64, H]
  const __nv_bfloat16* w_o;     // [H, Hq 64]
  const __nv_bfloat16* mlp_norm;
  const __nv_bfloat16* w_gu;    // [2 I, H], 64-row groups: gate rows then up rows
  const __nv_bfloat16* w_down;  // [H, I]
};

struct ResPlan {
  int grid;           // CTAs (one per SM)
  int slots;          // weight-ring slots
  int chunk;          // keys per attention item (multiple of 8)
  int max_items;      // attention items the packet buffer holds
  int off_h, off_x, off_att, off_res, off_out, off_bar, off_misc;  // dynamic shared-memory offsets
  int att_bytes;      // size of the attention region
  size_t smem;        // dynamic shared memory
};

struct ResArgs {
  int L, H, Hq, Hkv, I, V, max_positions;
  float eps, scale;
  const __nv_bfloat16* embed;
  const __nv_bfloat16* final_norm;
  const __nv_bfloat16* head;
  const float* rope_cos;
  const float* rope_sin;
  ResLayer layers[kResMaxLayers];
  int B, T, M, last_only;
  const int32_t* ids;
  const int32_t* n_new;
  const int32_t* past;
  const int32_t* table;
  int table_stride, bs, num_slots;
  __nv_bfloat16* k_pool;  // [L, num_slots, Hkv, 64]
  __nv_bfloat16* v_pool;
  float* logits;          // [rows_out, V]
  uint8_t* region;        // kResRegionBytes of the workspace (zeroed once by the caller)
  int32_t* status;
  long long wait_limit;   // clock cycles a packet wait may spin before it gives up
  // Optional phase record (globaltimer ns): stamp j of CTA c at trace[j * grid + c]; per layer
  // l the stamps 9 l .. 9 l + 8 (input read, q/k/v published, attention items done, attention
  // gathered, o published, MLP input normalised, gate/up published, activation read, down
  // published), then 9 L (final rows read), 9 L + 1 (head done), 9 L + 2 (kernel entry).
  unsigned long long* trace;
  ResPlan p;
};

// Whether a call with B rows of T tokens of this model runs the resident schedule; fills the plan.
bool plan_resident(int L, int H, int Hq, int Hkv, int D, int I, int V, int B, int T, int max_kv_len, ResPlan* p);
// Function attributes (shared memory, carveout); call outside any stream capture.
bool resident_prepare();
int launch_resident(const ResArgs& a, cudaStream_t stream);

}  // namespace specb200
