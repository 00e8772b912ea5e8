// Decode-step linear layers on CUDA cores (gemv.cu): Y[M, N] = X[M, K] W[N, K]^T for M <= 4
// token rows, with the weight rows staged into shared memory by bulk copies that are issued
// before the kernel waits on its predecessor, an optional fused RMSNorm of the input rows, and
// the tensor-core GEMM's epilogues.
#pragma once
#include "gemm.cuh"

namespace specb200 {

constexpr int kGemvMaxRows = 4;  // token rows per call

struct GemvPlan {
  int op;        // EpilogueOp
  int f;         // output features per chunk (QKV: rotary pairs, SILU_MUL: activation columns)
  int segs;      // weight row segments per chunk: 1 (STORE, RESID) or 2 (the pair / gate-up halves)
  int group;     // features per group (segs == 2): a chunk never crosses a group
  int group_rows;  // weight rows per group (segs == 2)
  int seg1_off;  // row offset of the second segment from the first
  int features;  // output features in total
  int rows;      // weight rows per full chunk (segs * f)
  int chunks;    // chunks in total
  int grid;      // CTAs; CTA b takes chunks b, b + grid, ...
  int stages;    // ring depth in chunks
  int ksplit;    // warps per weight row (rows < 8)
  size_t smem;   // dynamic shared memory bytes
};

// Plans the kernel for an (M, N, K) product with epilogue `op`; head_dim is used by EPI_QKV.
// Returns false when the shape is outside the kernel's limits (then the tensor-core GEMM runs).
bool plan_gemv(int op, int M, int N, int K, int head_dim, GemvPlan* p);

struct GemvArgs {
  const __nv_bfloat16* w;       // [N, K] row-major, 16-byte aligned
  const __nv_bfloat16* x;       // input rows, [*, K]
  const __nv_bfloat16* norm_w;  // [K]: RMSNorm of each input row first; nullptr = none
  const int32_t* sel_n_new;     // with norm: input row of output row b is b * T + n_new[b] - 1
  int T_tokens;
  float eps;
  int M, N, K;
  GemvPlan p;
  Epilogue e;
  int32_t* status;
  // Optional launch record (globaltimer ns): CTA b of launch `trace_slot` writes
  // trace[(trace_slot * kGemvTraceCtas + b) * kGemvTraceStamps + {0..7}] = entry, return from
  // griddepcontrol.wait, inputs staged, first weight chunk landed, end, then the time spent
  // waiting for weight chunks, the time in dot products, and the chunk count.
  unsigned long long* trace;
  int trace_slot;
};
constexpr int kGemvTraceCtas = 296;  // the largest grid plan_gemv makes
constexpr int kGemvTraceStamps = 8;

int launch_gemv(const GemvArgs& a, cudaStream_t stream, bool pdl);
// Raises the kernels' dynamic shared-memory limit; call once outside any stream capture.
// Returns false when the device refuses (then the schedule is not used).
bool gemv_prepare();

}  // namespace specb200
