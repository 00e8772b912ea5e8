// Host-side launchers shared by the forward orchestration (forward.cu) and the C ABI.
#pragma once
#include "common.cuh"

namespace specb200 {

// Launch with the programmatic-dependent-launch attribute when `pdl` is set: the kernel may
// start while the previous kernel on the stream drains, and orders itself after it with
// griddepcontrol.wait (every kernel here calls pdl_wait() before reading dependent data).
template <typename K, typename... Args>
cudaError_t launch_kernel(K kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

struct PrepArgs {
  const int32_t* ids;
  const int32_t* n_new;
  const int32_t* past;
  const int32_t* table;
  int table_stride, bs, num_slots, max_positions;
  int M, T, V, H;
  int32_t* pos_out;
  int32_t* slot_out;
  int32_t* status;
};

template <typename T>
int launch_prep_embed(const PrepArgs& a, const T* embed, T* hidden, cudaStream_t s, bool pdl);
// Function attributes of the prep / RMSNorm kernels; call outside any stream capture.
bool norm_prepare();
// Residual update of an EPI_PARTIAL GEMM (parts [splits][M][H] fp32) into h, then RMSNorm of
// `rows` rows into y (with the last-token selection when sel_n_new is given).
int launch_residual_norm(__nv_bfloat16* h, const float* parts, int splits, int M, int rows, int H,
                         const __nv_bfloat16* w, float eps, __nv_bfloat16* y, const int32_t* sel_n_new, int T_tokens,
                         cudaStream_t s, bool pdl);
bool residual_norm_fits(int splits, int H);
template <typename T>
int launch_rmsnorm(const T* x, const T* w, int rows, int H, float eps, T* y, const int32_t* sel_n_new, int T_tokens,
                   cudaStream_t s, bool pdl);

struct AttnArgs {
  const void* q;        // [B*T, Hq, D]
  const void* k_pool;   // [num_slots, Hkv, D] (one layer)
  const void* v_pool;
  const int32_t* table;
  int table_stride, bs;
  const int32_t* past;
  const int32_t* n_new;
  int B, T, Hq, Hkv, D;
  float scale;
  void* out;            // [B*T, Hq, D]
  int32_t* status;
  // Optional record (globaltimer ns); CTA c (linear block index, < kAttnTraceCtas) of launch
  // `trace_slot` writes trace[(trace_slot * kAttnTraceCtas + c) * 8 + k]. Tensor-core decode
  // items, k = 0..5: entry, wait return, keys landed, merged within the CTA, partial
  // published, end. Cluster kernel, k = 0..6: entry, wait return, keys landed, products done,
  // warps merged, cluster merged, end (first CTA).
  unsigned long long* trace = nullptr;
  int trace_slot = 0;
  // Optional (cluster kernel): q and the new keys / values come from the q/k/v GEMM's split
  // partials [qkv_splits][B T][qkv_n] (EPI_PARTIAL) instead of q and the pool; the kernel sums
  // them in split order, applies the EPI_QKV rounding and RoPE, and the first CTA of each
  // cluster writes the new keys and values to the pool.
  const float* qkv_parts = nullptr;
  int qkv_splits = 0, qkv_n = 0;
  const float* rope_cos = nullptr;
  const float* rope_sin = nullptr;
  int max_positions = 0;
};

constexpr int kAttnTraceCtas = 512;  // CTAs per launch in an attention trace record

// Split-KV merge tickets: a fixed region at the start of the attention workspace (see the
// GEMM's kGemmMaxCounters). Split-KV is only planned when the group count fits in it.
constexpr int kAttnMaxCounters = 65536;
constexpr size_t kAttnCounterBytes = kAttnMaxCounters * sizeof(int);

struct AttnPlan {
  int chunk, splits_max, qtiles;
  // 1: tensor-core decode items (bf16, d = 64, at most 16 query rows per KV head);
  // 2: the cluster kernel for the same shapes (splits_max = cluster size, chunk = keys per CTA);
  // 3: prefill shapes on the tensor cores (bf16, d = 64; qtiles = 64-row query tiles, no split)
  int mma = 0;
};
// Sets the cluster kernel's shared-memory limit; call outside any stream capture.
bool attention_prepare();
// tensor_items: the call is bf16 with d = 64, so decode / verify shapes (T x G <= 16) use the
// cluster kernel or the tensor-core items (attn_item_mma.cuh) and prefill shapes the
// tensor-core prefill kernel (attn_prefill.cuh).
AttnPlan plan_attention(int B, int T, int Hq, int Hkv, int max_kv_len, bool tensor_items);
size_t attention_partials_bytes(const AttnPlan& p, int B, int Hkv, int D);
size_t attention_workspace_bytes(const AttnPlan& p, int B, int Hkv, int D);  // counters + partials
// counters: kAttnMaxCounters ints that start zero (left zero); partials: attention_partials_bytes.
template <typename T>
int launch_attention(const AttnArgs& a, const AttnPlan& p, int* counters, float* partials, cudaStream_t s, bool pdl);

}  // namespace specb200
