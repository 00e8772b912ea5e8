// The Llama forward as one persistent kernel per call, for decode and verify shapes (bf16,
// at most 16 token rows): every layer's weights stream through each SM continuously.
//
// Same computation as the per-layer kernels (forward.cu) -- lm/forward.py:21-84 with the
// Hugging Face Llama pieces -- with a different schedule. One CTA per SM (cooperative
// launch, so every CTA is resident) walks the phase list
//   prep, then per layer  QKV -> attention -> O -> gate/up -> down,  then the LM head,
// with a grid barrier between dependent phases. Warp roles:
//   warp 4 (weight stream): walks the CTA's share of every GEMM phase of every layer in
//     order and copies 16 KB weight tiles (pre-packed 128 x 64 bf16, already in the 128-byte
//     swizzle the MMA descriptors expect, so each is one contiguous 1-D bulk copy) into an
//     8-stage ring. It never waits for activations, so the ring refills during barriers,
//     attention and epilogues and HBM keeps streaming across phase boundaries.
//   warp 5 (MMA): one thread issues tcgen05.mma (M = 128 weight rows, N = 16 token columns,
//     K = 16) into two alternating TMEM accumulators.
//   warps 0-3 (compute): build the activation operand in shared memory (RMSNorm fused here;
//     the attention and MLP activations come by TMA), read accumulators back with
//     tcgen05.ld, reduce stream-K partials, run the fused epilogues (RoPE + paged KV write,
//     residual add, SiLU*mul, fp32 logits), run the attention work items, and the barriers.
// GEMM work is split stream-K: the n_tiles x k_blocks units of a phase are cut into 148 equal
// contiguous ranges (contiguous in the packed weight buffer, so each SM streams one range).
// A tile whose k-blocks span several CTAs is reduced by its last contributor in contributor
// order (atomic ticket, no spin), so results do not depend on timing. Every spin-wait is
// bounded; a timeout sets the status word and a global abort flag that ends all CTAs.
#include <algorithm>
#include <mutex>

#include "attn_core.cuh"
#include "attn_item_mma.cuh"
#include "epilogue.cuh"
#include "stream.cuh"

namespace specb200 {
namespace {

constexpr int kThreads = 192;
constexpr int kStages = 8;
constexpr uint32_t kUnitBytes = 128 * 64 * 2;
constexpr uint32_t kXBlockBytes = kStreamBN * 64 * 2;
constexpr int kXBlocks = 32;
constexpr size_t kSmemBytes = 1024 + kStages * kUnitBytes + kXBlocks * kXBlockBytes +
                              kStreamBN * kEpiPitch * sizeof(float) + 256;

enum Kind { K_PREP = 0, K_QKV, K_ATTN, K_O, K_GU, K_DOWN, K_HEAD };
enum XMode { X_NORM = 0, X_NORM_SELECT, X_TMA_ATTN, X_TMA_ACT };

struct GemmInfo {
  const uint8_t* w;
  int N, K, n_tiles, kb;
  int xmode;
  const __nv_bfloat16* norm_w;
  int per_unit;
  int rows;
  Epilogue epi;
};

SPECB200_DEVINL int phase_kind(const StreamArgs& a, int p) {
  if (p == 0) return K_PREP;
  if (p == 1 + 5 * a.n_layers) return K_HEAD;
  return K_QKV + (p - 1) % 5;
}
SPECB200_DEVINL int phase_layer(int p) { return (p - 1) / 5; }
SPECB200_DEVINL bool is_gemm(int kind) { return kind != K_PREP && kind != K_ATTN; }

__device__ GemmInfo gemm_info(const StreamArgs& a, int p) {
  const int kind = phase_kind(a, p);
  GemmInfo g = {};
  g.rows = a.M;
  g.epi = Epilogue{};
  if (kind == K_HEAD) {
    g.w = a.head;
    g.N = a.V;
    g.K = a.H;
    g.xmode = a.last_only ? X_NORM_SELECT : X_NORM;
    g.norm_w = a.final_norm;
    g.rows = a.last_only ? a.B : a.M;
    g.epi.op = EPI_STORE;
    g.epi.out_f32 = 1;
    g.epi.out = a.logits;
    g.epi.ldo = a.V;
  } else {
    const int l = phase_layer(p);
    const StreamLayer& L = a.layers[l];
    const size_t layer_pool = static_cast<size_t>(a.num_slots) * a.Hkv * a.D;
    switch (kind) {
      case K_QKV:
        g.w = L.qkv; g.N = (a.Hq + 2 * a.Hkv) * a.D; g.K = a.H; g.xmode = X_NORM; g.norm_w = L.attn_norm;
        g.epi.op = EPI_QKV; g.epi.out = a.q; g.epi.ldo = a.Hq * a.D;
        g.epi.k_pool = a.k_pool + l * layer_pool; g.epi.v_pool = a.v_pool + l * layer_pool;
        g.epi.slot = a.slot; g.epi.pos = a.pos; g.epi.rope_cos = a.rope_cos; g.epi.rope_sin = a.rope_sin;
        g.epi.n_heads = a.Hq; g.epi.n_kv_heads = a.Hkv; g.epi.head_dim = a.D;
        break;
      case K_O:
        g.w = L.o; g.N = a.H; g.K = a.Hq * a.D; g.xmode = X_TMA_ATTN;
        g.epi.op = EPI_RESID; g.epi.out = a.h; g.epi.ldo = a.H;
        break;
      case K_GU:
        g.w = L.gu; g.N = 2 * a.I; g.K = a.H; g.xmode = X_NORM; g.norm_w = L.mlp_norm;
        g.epi.op = EPI_SILU_MUL; g.epi.out = a.act; g.epi.ldo = a.I;
        break;
      default:  // K_DOWN
        g.w = L.down; g.N = a.H; g.K = a.I; g.xmode = X_TMA_ACT;
        g.epi.op = EPI_RESID; g.epi.out = a.h; g.epi.ldo = a.H;
        break;
    }
  }
  g.n_tiles = (g.N + 127) / 128;
  g.kb = (g.K + 63) / 64;
  g.per_unit = g.kb > kXBlocks;
  return g;
}

// Stream-K partition: CTA c owns units [c U / G, (c + 1) U / G); owner(u) inverts it.
SPECB200_DEVINL void unit_range(int U, int G, int c, int& u0, int& u1) {
  u0 = static_cast<int>(static_cast<int64_t>(U) * c / G);
  u1 = static_cast<int>(static_cast<int64_t>(U) * (c + 1) / G);
}
SPECB200_DEVINL int unit_owner(int U, int G, int u) {
  return static_cast<int>((static_cast<int64_t>(u + 1) * G - 1) / U);
}

SPECB200_DEVINL void bulk_copy(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
SPECB200_DEVINL void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(src)), "r"(bytes)
               : "memory");
}
SPECB200_DEVINL unsigned atom_add_release_u32(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.add.release.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
SPECB200_DEVINL int atom_add_acq_rel_i32(int* p, int v) {
  int old;
  asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
SPECB200_DEVINL unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
SPECB200_DEVINL int ld_volatile_i32(const int* p) {
  int v;
  asm volatile("ld.volatile.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
SPECB200_DEVINL unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Profiling stamps: compute thread 0 writes [0] phase entry, [1] after the barrier,
// [2] operand ready, [3] phase work done, [6] first accumulator ready; the MMA thread writes
// [4] operand observed, [5] last MMA issued; the weight thread [7] last copy issued.
SPECB200_DEVINL void stamp(const StreamArgs& a, int n_phases, int p, int i) {
  if (a.trace) a.trace[(static_cast<size_t>(blockIdx.x) * n_phases + p) * 8 + i] = now_ns();
}

SPECB200_DEVINL void abort_all(const StreamArgs& a, volatile int* abort_s, int code) {
  set_status(a.status, code);
  atomicExch(a.abort_flag, 1);
  *abort_s = 1;
}

// Grid-wide barrier among the compute warps of every CTA (sense by generation counter).
// Returns false if the run has been aborted.
__device__ bool grid_barrier(const StreamArgs& a, volatile int* abort_s, int* sh_flag) {
  epi_bar_sync();
  if (threadIdx.x == 0) {
    bool ok = !*abort_s && !ld_volatile_i32(a.abort_flag);
    if (ok) {
      // The CTA barrier above orders every compute thread's writes before this release.
      const unsigned g0 = ld_acquire_u32(a.barrier + 1);
      const unsigned arrived = atom_add_release_u32(a.barrier, 1u) + 1u;
      if (arrived == gridDim.x) {
        atomicExch(a.barrier, 0u);
        atom_add_release_u32(a.barrier + 1, 1u);
      } else {
        const long long t0 = clock64();
        while (ld_acquire_u32(a.barrier + 1) == g0) {
          if (ld_volatile_i32(a.abort_flag)) { ok = false; break; }
          if (clock64() - t0 > SPECB200_SPIN_LIMIT_CYCLES) {
            abort_all(a, abort_s, SPECB200_ERR_TIMEOUT);
            ok = false;
            break;
          }
        }
      }
    }
    if (!ok) *abort_s = 1;
    *sh_flag = ok;
  }
  epi_bar_sync();
  return *sh_flag;
}

// ---------------------------------------------------------------- compute-warp pieces
__device__ void prep_phase(const StreamArgs& a) {
  for (int m = blockIdx.x; m < a.M; m += gridDim.x) {
    const int b = m / a.T, t = m % a.T;
    __shared__ int sh_id;
    if (threadIdx.x == 0) {
      const int pos = a.past[b] + t;
      int slot = -1;
      if (t < a.n_new[b]) {
        const int blk = pos / a.bs;
        if (pos >= a.max_positions || blk >= a.table_stride) {
          set_status(a.status, SPECB200_ERR_RANGE);
        } else {
          const int64_t s = static_cast<int64_t>(a.table[static_cast<int64_t>(b) * a.table_stride + blk]) * a.bs + pos % a.bs;
          if (s < 0 || s >= a.num_slots) set_status(a.status, SPECB200_ERR_RANGE);
          else slot = static_cast<int>(s);
        }
      }
      a.pos[m] = min(pos, a.max_positions - 1);
      a.slot[m] = slot;
      int id = a.ids[m];
      if (id < 0 || id >= a.V) {
        set_status(a.status, SPECB200_ERR_RANGE);
        id = 0;
      }
      sh_id = id;
    }
    epi_bar_sync();
    const uint4* src = reinterpret_cast<const uint4*>(a.embed + static_cast<int64_t>(sh_id) * a.H);
    uint4* dst = reinterpret_cast<uint4*>(a.h + static_cast<int64_t>(m) * a.H);
    for (int i = threadIdx.x; i < a.H / 8; i += 128) dst[i] = src[i];
    epi_bar_sync();
  }
}

// X = RMSNorm(h rows) written straight into the swizzled K-major operand layout: row r of
// K-block kb at kb * 2 KB + r * 128 B, 16-byte chunk c stored at position c ^ (r % 8). All
// 128 threads load every row they need at once (one memory round trip), the per-row sums of
// squares meet in shared memory, and the normalised values go out from registers.
__device__ void build_x_norm(const StreamArgs& a, const GemmInfo& g, uint8_t* xreg, float* red) {
  constexpr int kCpt = 2;  // 16-byte chunks per thread: H <= 128 * 2 * 8 = 2048
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int chunks = a.H / 8;
  uint4 w[kCpt];
#pragma unroll
  for (int i = 0; i < kCpt; ++i) {
    const int c = t + 128 * i;
    w[i] = c < chunks ? reinterpret_cast<const uint4*>(g.norm_w)[c] : make_uint4(0, 0, 0, 0);
  }
  for (int r0 = 0; r0 < g.rows; r0 += 8) {
    uint4 v[8][kCpt];
    float ss[8];
#pragma unroll
    for (int rr = 0; rr < 8; ++rr) {
      const int r = r0 + rr;
      ss[rr] = 0.f;
      const int64_t src_row = r < g.rows ? ((g.xmode == X_NORM_SELECT)
                                                ? static_cast<int64_t>(r) * a.T + max(a.n_new[r] - 1, 0) : r)
                                         : 0;
      const uint4* src = reinterpret_cast<const uint4*>(a.h + src_row * a.H);
#pragma unroll
      for (int i = 0; i < kCpt; ++i) {
        const int c = t + 128 * i;
        v[rr][i] = (r < g.rows && c < chunks) ? src[c] : make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int rr = 0; rr < 8; ++rr) {
#pragma unroll
      for (int i = 0; i < kCpt; ++i) {
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&v[rr][i]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(h2[j]);
          ss[rr] = fmaf(f.x, f.x, ss[rr]);
          ss[rr] = fmaf(f.y, f.y, ss[rr]);
        }
      }
      const float tot = warp_sum(ss[rr]);
      if (lane == 0) red[warp * 8 + rr] = tot;
    }
    epi_bar_sync();
#pragma unroll
    for (int rr = 0; rr < 8; ++rr) {
      const int r = r0 + rr;
      if (r >= g.rows) break;
      const float sum = red[rr] + red[8 + rr] + red[16 + rr] + red[24 + rr];
      const float inv = 1.0f / sqrtf(sum / static_cast<float>(a.H) + a.eps);
#pragma unroll
      for (int i = 0; i < kCpt; ++i) {
        const int c = t + 128 * i;
        if (c >= chunks) continue;
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&v[rr][i]);
        const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&w[i]);
        uint4 o;
        __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(h2[j]);
          const float2 wf = __bfloat1622float2(w2[j]);
          const float nx = round_to<__nv_bfloat16>(f.x * inv), ny = round_to<__nv_bfloat16>(f.y * inv);
          o2[j] = __floats2bfloat162_rn(wf.x * nx, wf.y * ny);
        }
        const int kb = c >> 3, cc = c & 7;
        *reinterpret_cast<uint4*>(xreg + kb * kXBlockBytes + r * 128 + ((cc ^ (r & 7)) << 4)) = o;
      }
    }
    epi_bar_sync();
  }
}

// Contributors of a tile: with U >= G every CTA owns at least one unit, so they are the
// consecutive CTAs owner(first unit) .. owner(last unit); with U < G each CTA owns at most one
// unit and each of the tile's kb units has its own CTA. slot = this CTA's position among them.
SPECB200_DEVINL void tile_contributors(int U, int G, int kb, int tile, int cta, int seg_u0, int& nc, int& slot) {
  if (U >= G) {
    const int c0 = unit_owner(U, G, tile * kb);
    nc = unit_owner(U, G, (tile + 1) * kb - 1) - c0 + 1;
    slot = cta - c0;
  } else {
    nc = kb;
    slot = seg_u0 - tile * kb;
  }
}

__device__ void finish_segment(const StreamArgs& a, const GemmInfo& g, int tile, int U, int seg_u0, float* tile_smem,
                               int* sh_flag) {
  int nc, slot;
  tile_contributors(U, gridDim.x, g.kb, tile, blockIdx.x, seg_u0, nc, slot);
  const int t = threadIdx.x;
  if (nc > 1) {
    const size_t tile_elems = static_cast<size_t>(kStreamBN) * 128;
    float* base = a.partials + static_cast<size_t>(tile) * a.max_contrib * tile_elems;
    float* mine = base + slot * tile_elems;
    for (int tok = 0; tok < g.rows; ++tok) mine[tok * 128 + t] = tile_smem[tok * kEpiPitch + t];
    epi_bar_sync();  // orders every thread's partial before thread 0's release below
    if (t == 0) *sh_flag = (atom_add_acq_rel_i32(a.tile_counters + tile, 1) == nc - 1);
    epi_bar_sync();  // and thread 0's acquire before every thread's reads
    if (!*sh_flag) return;
    for (int t0 = 0; t0 < g.rows; t0 += kEpiBatch) {
      float acc[kEpiBatch];
#pragma unroll
      for (int j = 0; j < kEpiBatch; ++j) acc[j] = 0.f;
      for (int s = 0; s < nc; ++s) {
#pragma unroll
        for (int j = 0; j < kEpiBatch; ++j)
          if (t0 + j < g.rows) acc[j] += __ldcg(base + s * tile_elems + (t0 + j) * 128 + t);
      }
#pragma unroll
      for (int j = 0; j < kEpiBatch; ++j)
        if (t0 + j < g.rows) tile_smem[(t0 + j) * kEpiPitch + t] = acc[j];
    }
    if (t == 0) a.tile_counters[tile] = 0;
    epi_bar_sync();
  }
  apply_epilogue<__nv_bfloat16>(g.epi, tile_smem, tile * 128, 0, g.rows, g.N);
}

__global__ void __launch_bounds__(kThreads, 1)
    stream_kernel(const __grid_constant__ StreamArgs a, const __grid_constant__ CUtensorMap map_attn,
                  const __grid_constant__ CUtensorMap map_act) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint8_t* xreg = ring + kStages * kUnitBytes;
  float* tile_smem = reinterpret_cast<float*>(xreg + kXBlocks * kXBlockBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(tile_smem + kStreamBN * kEpiPitch);
  uint64_t* empty = full + kStages;
  uint64_t* x_full = empty + kStages;
  uint64_t* acc_full = x_full + 1;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_s = reinterpret_cast<volatile int*>(tmem_holder + 1);
  int* sh_flag = const_cast<int*>(abort_s) + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, cta = blockIdx.x;
  const int n_phases = 2 + 5 * a.n_layers;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(x_full, 1);
    mbar_init(&acc_full[0], 1);
    mbar_init(&acc_full[1], 1);
    mbar_init(&acc_empty[0], 1);
    mbar_init(&acc_empty[1], 1);
    *abort_s = 0;
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_holder, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 4) {
    // ------------------------------------------------------------ weight stream
    if (lane == 0) {
      const uint64_t pol = a.ring_evict_first ? l2_policy_evict_first() : l2_policy_evict_normal();
      uint32_t gu = 0;
      for (int p = 0; p < n_phases && !*abort_s; ++p) {
        if (!is_gemm(phase_kind(a, p))) continue;
        const GemmInfo g = gemm_info(a, p);
        const int U = g.n_tiles * g.kb;
        int u0, u1;
        unit_range(U, G, cta, u0, u1);
        // Pull this CTA's share of the GEMM phase `prefetch_ahead` phases later into L2 now (up
        // to 512 KB), so HBM keeps streaming while barriers, operand builds and epilogues run.
        // (With prefetch_ahead = k, the first k phases are requested here at the start.)
        for (int q = p + 1, seen = 0; q < n_phases && a.prefetch_ahead > 0; ++q) {
          if (!is_gemm(phase_kind(a, q))) continue;
          ++seen;
          const bool first_phase = (p == 1);
          if (seen < a.prefetch_ahead && !first_phase) continue;
          const GemmInfo gn = gemm_info(a, q);
          int v0, v1;
          unit_range(gn.n_tiles * gn.kb, G, cta, v0, v1);
          for (int v = v0; v < v1 && v < v0 + 32; ++v) prefetch_l2(gn.w + static_cast<size_t>(v) * kUnitBytes, kUnitBytes);
          if (seen >= a.prefetch_ahead) break;
        }
        for (int u = u0; u < u1; ++u, ++gu) {
          const int st = gu % kStages;
          if (gu >= kStages && !mbar_wait_bounded(&empty[st], ((gu / kStages) - 1) & 1, a.status, abort_s)) break;
          mbar_arrive_expect_tx(&full[st], kUnitBytes);
          bulk_copy(ring + st * kUnitBytes, g.w + static_cast<size_t>(u) * kUnitBytes, kUnitBytes, &full[st], pol);
        }
        if (u1 > u0) stamp(a, n_phases, p, 7);
      }
      if (!*abort_s) {
        const uint32_t first = gu > kStages ? gu - kStages : 0;
        for (uint32_t i = first; i < gu; ++i)
          if (!mbar_wait_bounded(&empty[i % kStages], (i / kStages) & 1, a.status, abort_s)) break;
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issue: the whole warp
    // runs the loop and one elected lane issues (a lone issuing lane with the other lanes
    // waiting diverged costs about a third more per instruction)
    {
      const uint32_t idesc = umma_idesc_bf16(128, kStreamBN);
      uint32_t gu = 0, xc = 0, segs = 0;
      bool ok = true;
      for (int p = 0; p < n_phases && ok; ++p) {
        ok = __shfl_sync(0xffffffffu, *abort_s ? 0 : 1, 0) != 0;
        if (!ok) break;
        if (!is_gemm(phase_kind(a, p))) continue;
        const GemmInfo g = gemm_info(a, p);
        const int U = g.n_tiles * g.kb;
        int u0, u1;
        unit_range(U, G, cta, u0, u1);
        if (u0 == u1) continue;
        if (!mbar_wait_warp(x_full, xc & 1, a.status, abort_s)) {
          ok = false;
          break;
        }
        ++xc;
        tc_fence_after();
        if (lane == 0) stamp(a, n_phases, p, 4);
        bool first = true;
        uint32_t buf = 0;
        for (int u = u0; u < u1; ++u, ++gu) {
          if (first) {
            buf = segs & 1;
            if (segs >= 2 && !mbar_wait_warp(&acc_empty[buf], ((segs >> 1) - 1) & 1, a.status, abort_s)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          const int st = gu % kStages;
          if (!mbar_wait_warp(&full[st], (gu / kStages) & 1, a.status, abort_s)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int xslot = g.per_unit ? (u - u0) : (u % g.kb);
          const uint64_t da = umma_desc_sw128(smem_u32(ring + st * kUnitBytes));
          const uint64_t dx = umma_desc_sw128(smem_u32(xreg + xslot * kXBlockBytes));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16_elect(tmem_base + buf * kStreamBN, da + kk * 2, dx + kk * 2, idesc, (first && kk == 0) ? 0u : 1u);
          umma_commit_elect(&empty[st]);
          const bool seg_end = (u + 1 == u1) || ((u + 1) % g.kb == 0);
          if (seg_end) {
            umma_commit_elect(&acc_full[buf]);
            ++segs;
            first = true;
          } else {
            first = false;
          }
        }
        if (lane == 0) stamp(a, n_phases, p, 5);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ compute warps 0-3
    uint32_t xc = 0, segs = 0;
    for (int p = 0; p < n_phases; ++p) {
      if (threadIdx.x == 0) stamp(a, n_phases, p, 0);
      if (p > 0 && !grid_barrier(a, abort_s, sh_flag)) break;
      if (threadIdx.x == 0) stamp(a, n_phases, p, 1);
      const int kind = phase_kind(a, p);
      if (kind == K_PREP) {
        prep_phase(a);
        if (threadIdx.x == 0) stamp(a, n_phases, p, 3);
        continue;
      }
      if (kind == K_ATTN) {
        const int l = phase_layer(p);
        const size_t layer_pool = static_cast<size_t>(a.num_slots) * a.Hkv * a.D;
        AttnKernelArgs ka;
        ka.a.q = a.q;
        ka.a.k_pool = a.k_pool + l * layer_pool;
        ka.a.v_pool = a.v_pool + l * layer_pool;
        ka.a.table = a.table;
        ka.a.table_stride = a.table_stride;
        ka.a.bs = a.bs;
        ka.a.past = a.past;
        ka.a.n_new = a.n_new;
        ka.a.B = a.B;
        ka.a.T = a.T;
        ka.a.Hq = a.Hq;
        ka.a.Hkv = a.Hkv;
        ka.a.D = a.D;
        ka.a.scale = a.attn_scale;
        ka.a.out = a.attn;
        ka.a.status = a.status;
        ka.p = a.ap;
        ka.counters = a.attn_counters;
        ka.part = a.attn_partials;
        const int per_b = a.Hkv * a.ap.splits_max;
        const int items = a.B * per_b;
        const bool tensor_items = a.T * (a.Hq / a.Hkv) <= kAmRows;
        for (int it = cta; it < items; it += G) {
          const int b = it / per_b, r = it % per_b;
          if (tensor_items) attention_item_mma(ka, b, r / a.ap.splits_max, r % a.ap.splits_max, xreg);
          else attention_item_decode(ka, b, r / a.ap.splits_max, r % a.ap.splits_max, xreg);
          epi_bar_sync();
        }
        if (threadIdx.x == 0) stamp(a, n_phases, p, 3);
        continue;
      }
      const GemmInfo g = gemm_info(a, p);
      const int U = g.n_tiles * g.kb;
      int u0, u1;
      unit_range(U, G, cta, u0, u1);
      if (u0 == u1) continue;
      // activation operand
      if (g.xmode == X_NORM || g.xmode == X_NORM_SELECT) {
        build_x_norm(a, g, xreg, tile_smem);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        epi_bar_sync();
        if (threadIdx.x == 0) mbar_arrive(x_full);
      } else if (threadIdx.x == 0) {
        const CUtensorMap* map = g.xmode == X_TMA_ATTN ? &map_attn : &map_act;
        // the activations were written by other CTAs' generic stores before the barrier, and
        // this region was last touched by generic accesses (attention scratch): order both
        // before the async-proxy copy
        asm volatile("fence.proxy.async.global;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        const int n = g.per_unit ? (u1 - u0) : min(u1 - u0, g.kb);
        mbar_arrive_expect_tx(x_full, n * kXBlockBytes);
        for (int i = 0; i < n; ++i) {
          const int kbi = (u0 + i) % g.kb;
          const int slot = g.per_unit ? i : kbi;
          tma_load_2d(xreg + slot * kXBlockBytes, map, x_full, kbi * 64, 0);
        }
      }
      ++xc;
      if (threadIdx.x == 0) stamp(a, n_phases, p, 2);
      // segments: one per tile touched by this CTA's unit range
      int u = u0;
      while (u < u1) {
        const int tile = u / g.kb;
        const int seg_end = min(u1, (tile + 1) * g.kb);
        const uint32_t buf = segs & 1;
        const bool ok = mbar_wait_bounded(&acc_full[buf], (segs >> 1) & 1, a.status, abort_s);
        tc_fence_after();
        if (threadIdx.x == 0 && u == u0) stamp(a, n_phases, p, 6);
        if (ok) {
          float v[16];
          tmem_ld16(tmem_base + (static_cast<uint32_t>(warp * 32) << 16) + buf * kStreamBN, v);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) tile_smem[j * kEpiPitch + warp * 32 + lane] = v[j];
        }
        tc_fence_before();
        epi_bar_sync();
        if (threadIdx.x == 0) mbar_arrive(&acc_empty[buf]);
        if (ok && !*abort_s) finish_segment(a, g, tile, U, u, tile_smem, sh_flag);
        epi_bar_sync();
        ++segs;
        u = seg_end;
        if (!ok) break;
      }
      if (threadIdx.x == 0) stamp(a, n_phases, p, 3);
      if (*abort_s) break;
    }
    (void)xc;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 32);
  }
}

// packed[(tile * KB + kb) * 8192 + r * 64 + ((c / 8) ^ (r % 8)) * 8 + c % 8] = W[tile*128 + r][kb*64 + c]
__global__ void pack_tiles_kernel(const __nv_bfloat16* __restrict__ w, int N, int K, __nv_bfloat16* __restrict__ out) {
  const int KB = (K + 63) / 64;
  const int64_t unit = blockIdx.x;  // (tile, kb)
  const int tile = static_cast<int>(unit / KB), kb = static_cast<int>(unit % KB);
  for (int i = threadIdx.x; i < 128 * 8; i += blockDim.x) {
    const int r = i / 8, c8 = i % 8;
    const int n = tile * 128 + r;
    uint4 v = make_uint4(0, 0, 0, 0);
    const int k0 = kb * 64 + c8 * 8;
    if (n < N && k0 + 8 <= K) v = *reinterpret_cast<const uint4*>(w + static_cast<int64_t>(n) * K + k0);
    *reinterpret_cast<uint4*>(out + unit * 8192 + r * 64 + ((c8 ^ (r & 7)) * 8)) = v;
  }
}

}  // namespace

size_t stream_packed_bytes(int N, int K) {
  return static_cast<size_t>((N + 127) / 128) * ((K + 63) / 64) * kUnitBytes;
}

size_t stream_smem_bytes() { return kSmemBytes; }

int stream_max_contrib(int N, int K, int G) {
  const int n_tiles = (N + 127) / 128, kb = (K + 63) / 64, U = n_tiles * kb;
  if (U < G) return kb;  // one unit per CTA: every unit of a tile is its own contributor
  int best = 1;
  for (int t = 0; t < n_tiles; ++t) {
    const int c0 = static_cast<int>((static_cast<int64_t>(t * kb + 1) * G - 1) / U);
    const int c1 = static_cast<int>((static_cast<int64_t>((t + 1) * kb) * G - 1) / U);
    best = std::max(best, c1 - c0 + 1);
  }
  return best;
}

bool stream_units_fit(int N, int K, int G) {
  const int kb = (K + 63) / 64;
  if (kb <= kXBlocks) return true;
  const int U = ((N + 127) / 128) * kb;
  return (U + G - 1) / G <= kXBlocks;
}

int launch_stream(const StreamArgs& a, const CUtensorMap& map_attn, const CUtensorMap& map_act, int grid,
                  cudaStream_t s) {
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] {
    attr = cudaFuncSetAttribute(stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBytes));
  });
  if (attr != cudaSuccess) return SPECB200_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, stream_kernel, a, map_attn, map_act) == cudaSuccess ? SPECB200_OK : SPECB200_ERR_CUDA;
}

int stream_grid_size() {
  static int g = 0;
  if (!g) {
    int dev = 0, sms = 0, per = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaFuncSetAttribute(stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBytes));
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, stream_kernel, kThreads, kSmemBytes);
    g = per >= 1 ? sms : -1;
  }
  return g;
}

}  // namespace specb200

using namespace specb200;
extern "C" int specb200_set_error(int code, const char* msg);

extern "C" size_t specb200_packed_tile_bytes(int N, int K) { return stream_packed_bytes(N, K); }

extern "C" int specb200_pack_tiles(const void* w, int N, int K, void* out, void* stream) {
  if (!w || !out || N <= 0 || K <= 0 || K % 8) return specb200_set_error(SPECB200_ERR_ARG, "pack_tiles: bad arguments");
  const int units = ((N + 127) / 128) * ((K + 63) / 64);
  pack_tiles_kernel<<<units, 256, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const __nv_bfloat16*>(w), N, K,
                                                                          static_cast<__nv_bfloat16*>(out));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return specb200_set_error(SPECB200_ERR_CUDA, cudaGetErrorString(e));
  return SPECB200_OK;
}
