// The Llama forward over the paged KV cache: lm/forward.py:21-68 + lm/forward.py:71-84.
//
// A model handle holds the weight pointers and one TMA descriptor per bf16 weight matrix;
// specb200_forward launches, per call: prep/embed, then per layer RMSNorm -> QKV GEMM
// (RoPE + paged KV write epilogue) -> paged attention -> O GEMM (+ residual) -> RMSNorm ->
// gate/up GEMM (SiLU*mul epilogue) -> down GEMM (+ residual), then the final RMSNorm (with
// the last-token row selection of lm/forward.py:66-67) and the fp32-accumulated LM head.
// Every kernel after the first is launched with programmatic dependent launch, so each GEMM
// starts streaming its weights while the kernel before it drains. The whole sequence is
// stream-ordered and allocation-free, so callers can capture it in a CUDA graph.
#include <algorithm>
#include <cstdlib>
#include <vector>

#include "attn_cluster.cuh"
#include "attn_core.cuh"
#include "gemm.cuh"
#include "gemv.cuh"
#include "kernels.cuh"
#include "chain.cuh"
#include "stream.cuh"

namespace specb200 {
namespace {

struct LayerMaps {
  CUtensorMap qkv, o, gu, down;
};

int env_int(const char* name, int def) {
  const char* v = std::getenv(name);
  return v && *v ? std::atoi(v) : def;
}

struct Model {
  int prefetch_ahead = 1, ring_evict_first = 1;
  specb200_model_config cfg;
  specb200_model_weights w;
  std::vector<specb200_layer_weights> layers;
  std::vector<LayerMaps> maps;
  CUtensorMap head;
  int qkv_n;
  bool stream_ok;  // packed weights present and shapes within the layer-stream kernel's limits
  int chain_C = 0;  // cluster size of the layer-chain kernel, 0 = not used for this model
  bool gemv_ok = false;  // bf16 weights usable by the decode-step GEMV kernels (gemv.cu)
  bool gemm_norm = false;  // RMSNorms folded into the tensor-core GEMMs that consume them
  bool defer_resid = true;  // residual adds of the o / down GEMMs deferred to the next RMSNorm
  bool defer_qkv = true;    // q/k/v GEMM partials summed by the cluster attention
  bool qkv_attn = false;    // GEMV schedule: each KV head's q/k/v projection inside its attention cluster
};

// Whether a call of this shape runs the cluster layer-chain kernel (small models, decode
// shapes); fills its plan.
bool use_chain(const Model& m, int B, int T, ChainPhase ph[4], int* splits, ChainLayout* L) {
  const specb200_model_config& c = m.cfg;
  if (m.chain_C <= 0) return false;
  return chain_plan(c.n_layers, c.hidden, c.n_heads, c.n_kv_heads, c.head_dim, c.intermediate, B, T, m.chain_C, ph,
                    splits, L);
}

// Whether a call of this shape runs the persistent layer-stream kernel; fills its grid size
// and the stream-K partial slots it needs.
bool use_stream(const Model& m, int B, int T, int* grid, int* max_contrib) {
  const specb200_model_config& c = m.cfg;
  if (!m.stream_ok || B * T > kStreamBN) return false;
  if (T * (m.cfg.n_heads / m.cfg.n_kv_heads) > 32) return false;  // one 32-row query tile per KV head
  const int G = stream_grid_size();
  if (G <= 0) return false;
  if (!stream_units_fit(c.hidden, c.intermediate, G)) return false;
  const int qd = c.n_heads * c.head_dim;
  int mc = 1;
  mc = std::max(mc, stream_max_contrib(m.qkv_n, c.hidden, G));
  mc = std::max(mc, stream_max_contrib(c.hidden, qd, G));
  mc = std::max(mc, stream_max_contrib(2 * c.intermediate, c.hidden, G));
  mc = std::max(mc, stream_max_contrib(c.hidden, c.intermediate, G));
  mc = std::max(mc, stream_max_contrib(c.vocab, c.hidden, G));
  *grid = G;
  *max_contrib = mc;
  return true;
}

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

struct Carve {
  size_t gemm_counters, attn_counters, stream_ctl, hidden, xbuf, qbuf, attn, act, pos, slot, gemm_parts, attn_parts,
      stream_parts, resid_parts, qkv_parts, total;
  // per-layer schedule: the o and down GEMMs store split partials (EPI_PARTIAL) and the RMSNorm
  // launch that follows each adds them to the residual stream (launch_residual_norm)
  bool defer;
  // ... and the q/k/v GEMM stores split partials that the cluster attention sums, rotates and
  // writes to the pool itself (no ticket, no epilogue tail in the GEMM)
  bool defer_qkv;
  bool stream, chain;
  int grid, max_contrib;
  ChainPhase cph[4];
  int csplits;
  ChainLayout cl;
  GemmShape g_qkv, g_o, g_gu, g_down, g_head;
  bool gemv;  // decode-step schedule: the per-layer order with GEMV kernels and fused norms
  bool gemv_head;  // ... and the LM head as a GEMV with the final norm folded in
  bool attn_o;     // ... and attention + o projection as one cluster kernel per sequence
  AttnPlan ap_o;
  int ao_P, ao_rows;
  bool qkv_attn;   // ... or the q/k/v projection inside the attention clusters
  AttnPlan ap_qkv;
  int qkv_pairs;
  bool norm_qkv, norm_gu, norm_head;  // per-layer schedule: norm folded into these GEMMs
  GemvPlan v_qkv, v_o, v_gu, v_down, v_head;
  AttnPlan ap;
};

// Whether a call of this shape runs the decode-step GEMV schedule: at most kGemvMaxRows token
// rows of a bf16 model whose every layer linear has its weights on chip at once (one chunk per
// CTA, at most two CTAs per SM). Fills the four layer plans and, in *head, the LM head's; the
// head runs as a GEMV (final norm folded in) only when *head_gemv, else as RMSNorm + the
// tensor-core GEMM, which streams a large vocabulary faster than the CUDA-core dot products.
bool use_gemv(const Model& m, int M, int rows_out, GemvPlan* qkv, GemvPlan* o, GemvPlan* gu, GemvPlan* down,
              GemvPlan* head, bool* head_gemv) {
  const specb200_model_config& c = m.cfg;
  if (!m.gemv_ok || M > kGemvMaxRows) return false;
  const int qd = c.n_heads * c.head_dim;
  const bool ok = plan_gemv(EPI_QKV, M, m.qkv_n, c.hidden, c.head_dim, qkv) && plan_gemv(EPI_RESID, M, c.hidden, qd, 0, o) &&
                  plan_gemv(EPI_SILU_MUL, M, 2 * c.intermediate, c.hidden, 0, gu) &&
                  plan_gemv(EPI_RESID, M, c.hidden, c.intermediate, 0, down);
  if (!ok || qkv->stages > 1 || o->stages > 1 || gu->stages > 1 || down->stages > 1) return false;
  static const int head_mode = env_int("SPECB200_GEMV_HEAD", 0);  // 1: GEMV head even when it streams
  *head_gemv = plan_gemv(EPI_STORE, rows_out, c.vocab, c.hidden, 0, head) && (head->stages == 1 || head_mode == 1);
  return true;
}

Carve carve(const Model& m, int B, int T, int max_kv_len, int last_only) {
  const specb200_model_config& c = m.cfg;
  const bool tc = c.dtype == SPECB200_BF16;
  const size_t el = tc ? 2 : 4;
  const int M = B * T;
  const int rows_out = last_only ? B : M;
  const int qd = c.n_heads * c.head_dim;
  Carve r;
  r.g_qkv = plan_gemm(M, m.qkv_n, c.hidden, tc);
  r.g_o = plan_gemm(M, c.hidden, qd, tc);
  r.g_gu = plan_gemm(M, 2 * c.intermediate, c.hidden, tc);
  r.g_down = plan_gemm(M, c.hidden, c.intermediate, tc);
  r.g_head = plan_gemm(rows_out, c.vocab, c.hidden, tc);
  r.chain = use_chain(m, B, T, r.cph, &r.csplits, &r.cl);
  r.stream = !r.chain && use_stream(m, B, T, &r.grid, &r.max_contrib);
  r.gemv_head = false;
  r.norm_qkv = m.gemm_norm && gemm_norm_fits(r.g_qkv);
  r.norm_gu = m.gemm_norm && gemm_norm_fits(r.g_gu);
  r.norm_head = m.gemm_norm && gemm_norm_fits(r.g_head);
  r.defer = tc && m.defer_resid && !r.norm_qkv && !r.norm_gu && !r.norm_head;
  if (r.defer) {  // the residual-norm kernel sums at most 8 partials per element
    r.g_o.splits = std::min(r.g_o.splits, 8);
    r.g_down.splits = std::min(r.g_down.splits, 8);
    r.defer = residual_norm_fits(r.g_o.splits, c.hidden) && residual_norm_fits(r.g_down.splits, c.hidden);
  }
  r.gemv = !r.chain && !r.stream &&
           use_gemv(m, M, rows_out, &r.v_qkv, &r.v_o, &r.v_gu, &r.v_down, &r.v_head, &r.gemv_head);
  r.defer = r.defer && !r.gemv && !r.stream && !r.chain;
  r.attn_o = r.gemv && plan_attention_o(B, T, c.n_heads, c.n_kv_heads, c.head_dim, c.hidden, max_kv_len, &r.ap_o,
                                        &r.ao_P, &r.ao_rows);
  r.qkv_attn = r.gemv && !r.attn_o && m.qkv_attn &&
               plan_attention_qkv(T, c.n_heads, c.n_kv_heads, c.head_dim, c.hidden, max_kv_len, &r.ap_qkv, &r.qkv_pairs);
  r.ap = r.stream ? plan_attention_decode(B, c.n_kv_heads, max_kv_len, r.grid)
                  : plan_attention(B, T, c.n_heads, c.n_kv_heads, max_kv_len, tc && c.head_dim == 64);
  r.defer_qkv = r.defer && r.ap.mma == 2 && c.head_dim == 64 && m.defer_qkv && r.g_qkv.splits <= kQkvMaxSplits;
  // The two ticket-counter regions sit at fixed offsets so that they stay zero across calls
  // of every shape; everything after them is rewritten before it is read.
  size_t off = 0;
  r.gemm_counters = off; off += align256(kGemmCounterBytes);
  r.attn_counters = off; off += align256(kAttnCounterBytes);
  r.stream_ctl = off; off += 256;
  r.hidden = off; off += align256(static_cast<size_t>(M) * c.hidden * el);
  r.xbuf = off; off += align256(static_cast<size_t>(M) * c.hidden * el);
  r.qbuf = off; off += align256(static_cast<size_t>(M) * qd * el);
  r.attn = off; off += align256(static_cast<size_t>(M) * qd * el);
  r.act = off; off += align256(static_cast<size_t>(M) * c.intermediate * el);
  r.pos = off; off += align256(static_cast<size_t>(M) * 4);
  r.slot = off; off += align256(static_cast<size_t>(M) * 4);
  size_t gws = 0;
  for (const GemmShape* s : {&r.g_qkv, &r.g_o, &r.g_gu, &r.g_down, &r.g_head}) gws = std::max(gws, gemm_partials_bytes(*s));
  r.gemm_parts = off; off += align256(gws);
  r.attn_parts = off; off += align256(attention_partials_bytes(r.ap, B, c.n_kv_heads, c.head_dim));
  r.resid_parts = off;
  if (r.defer)
    off += align256(static_cast<size_t>(std::max(r.g_o.splits, r.g_down.splits)) * M * c.hidden * sizeof(float));
  r.qkv_parts = off;
  if (r.defer_qkv) off += align256(static_cast<size_t>(r.g_qkv.splits) * M * m.qkv_n * sizeof(float));
  r.stream_parts = off;
  if (r.stream) {
    const int max_tiles = std::max({(m.qkv_n + 127) / 128, (c.hidden + 127) / 128, (2 * c.intermediate + 127) / 128,
                                    (c.vocab + 127) / 128});
    off += align256(static_cast<size_t>(max_tiles) * r.max_contrib * kStreamBN * 128 * sizeof(float));
  }
  r.total = off;
  return r;
}

int run_stream(const Model& m, const specb200_batch& bt, char* ws, const Carve& cv, cudaStream_t s) {
  const specb200_model_config& c = m.cfg;
  const int B = bt.B, Tt = bt.T, M = B * Tt;
  const int qd = c.n_heads * c.head_dim;
  StreamArgs a = {};
  a.n_layers = c.n_layers;
  a.H = c.hidden;
  a.Hq = c.n_heads;
  a.Hkv = c.n_kv_heads;
  a.D = c.head_dim;
  a.I = c.intermediate;
  a.V = c.vocab;
  a.eps = c.rms_eps;
  a.attn_scale = 1.0f / sqrtf(static_cast<float>(c.head_dim));
  a.max_positions = c.max_positions;
  a.embed = static_cast<const __nv_bfloat16*>(m.w.embed);
  a.final_norm = static_cast<const __nv_bfloat16*>(m.w.final_norm);
  a.head = static_cast<const uint8_t*>(m.w.p_lm_head);
  a.rope_cos = m.w.rope_cos;
  a.rope_sin = m.w.rope_sin;
  for (int l = 0; l < c.n_layers; ++l) {
    const specb200_layer_weights& L = m.layers[l];
    a.layers[l].attn_norm = static_cast<const __nv_bfloat16*>(L.attn_norm);
    a.layers[l].mlp_norm = static_cast<const __nv_bfloat16*>(L.mlp_norm);
    a.layers[l].qkv = static_cast<const uint8_t*>(L.p_qkv);
    a.layers[l].o = static_cast<const uint8_t*>(L.p_o);
    a.layers[l].gu = static_cast<const uint8_t*>(L.p_gate_up);
    a.layers[l].down = static_cast<const uint8_t*>(L.p_down);
  }
  a.B = B;
  a.T = Tt;
  a.M = M;
  a.last_only = bt.last_only;
  a.ids = bt.input_ids;
  a.n_new = bt.n_new;
  a.past = bt.past_len;
  a.table = bt.block_table;
  a.table_stride = bt.table_stride;
  a.bs = bt.block_size;
  a.num_slots = bt.num_slots;
  a.k_pool = static_cast<__nv_bfloat16*>(bt.k_pool);
  a.v_pool = static_cast<__nv_bfloat16*>(bt.v_pool);
  a.logits = bt.logits;
  a.h = reinterpret_cast<__nv_bfloat16*>(ws + cv.hidden);
  a.q = reinterpret_cast<__nv_bfloat16*>(ws + cv.qbuf);
  a.attn = reinterpret_cast<__nv_bfloat16*>(ws + cv.attn);
  a.act = reinterpret_cast<__nv_bfloat16*>(ws + cv.act);
  a.pos = reinterpret_cast<int32_t*>(ws + cv.pos);
  a.slot = reinterpret_cast<int32_t*>(ws + cv.slot);
  a.tile_counters = reinterpret_cast<int*>(ws + cv.gemm_counters);
  a.partials = reinterpret_cast<float*>(ws + cv.stream_parts);
  a.max_contrib = cv.max_contrib;
  a.barrier = reinterpret_cast<unsigned*>(ws + cv.stream_ctl);
  a.abort_flag = reinterpret_cast<int*>(ws + cv.stream_ctl + 64);
  a.ap = cv.ap;
  a.attn_counters = reinterpret_cast<int*>(ws + cv.attn_counters);
  a.attn_partials = reinterpret_cast<float*>(ws + cv.attn_parts);
  a.status = bt.status;
  a.trace = reinterpret_cast<unsigned long long*>(bt.trace);
  a.prefetch_ahead = m.prefetch_ahead;
  a.ring_evict_first = m.ring_evict_first;
  CUtensorMap map_attn{}, map_act{};
  if (!make_tmap_bf16_2d(&map_attn, a.attn, qd, M, kTileK, kStreamBN) ||
      !make_tmap_bf16_2d(&map_act, a.act, c.intermediate, M, kTileK, kStreamBN))
    return SPECB200_ERR_ARG;
  cudaMemsetAsync(ws + cv.stream_ctl, 0, 128, s);  // barrier arrivals/generation and the abort flag
  return launch_stream(a, map_attn, map_act, cv.grid, s);
}

template <typename T>
int run_head(const Model& m, const specb200_batch& bt, char* ws, const Carve& cv, cudaStream_t s,
             const CUtensorMap* x_final);

template <typename T>
int run_forward(const Model& m, const specb200_batch& bt, char* ws, const Carve& cv, cudaStream_t s) {
  const specb200_model_config& c = m.cfg;
  const bool tc = c.dtype == SPECB200_BF16;
  const int B = bt.B, Tt = bt.T, M = B * Tt;
  const int rows_out = bt.last_only ? B : M;
  const int qd = c.n_heads * c.head_dim;
  T* hidden = reinterpret_cast<T*>(ws + cv.hidden);
  T* xbuf = reinterpret_cast<T*>(ws + cv.xbuf);
  T* qbuf = reinterpret_cast<T*>(ws + cv.qbuf);
  T* attn = reinterpret_cast<T*>(ws + cv.attn);
  T* act = reinterpret_cast<T*>(ws + cv.act);
  int32_t* pos = reinterpret_cast<int32_t*>(ws + cv.pos);
  int32_t* slot = reinterpret_cast<int32_t*>(ws + cv.slot);
  float* resid_parts = reinterpret_cast<float*>(ws + cv.resid_parts);
  GemmScratch gscr{reinterpret_cast<int*>(ws + cv.gemm_counters), reinterpret_cast<float*>(ws + cv.gemm_parts)};
  int* attn_counters = reinterpret_cast<int*>(ws + cv.attn_counters);
  float* attn_parts = reinterpret_cast<float*>(ws + cv.attn_parts);
  int32_t* status = bt.status;

  CUtensorMap x_hidden{}, x_attn{}, x_act{}, x_final{};
  if (tc) {
    bool ok = make_tmap_bf16_2d(&x_hidden, xbuf, c.hidden, M, kTileK, cv.g_qkv.BN) &&
              make_tmap_bf16_2d(&x_attn, attn, qd, M, kTileK, cv.g_o.BN) &&
              make_tmap_bf16_2d(&x_act, act, c.intermediate, M, kTileK, cv.g_down.BN) &&
              make_tmap_bf16_2d(&x_final, xbuf, c.hidden, rows_out, kTileK, cv.g_head.BN);
    if (!ok) return SPECB200_ERR_ARG;
  }

  PrepArgs pa;
  pa.ids = bt.input_ids;
  pa.n_new = bt.n_new;
  pa.past = bt.past_len;
  pa.table = bt.block_table;
  pa.table_stride = bt.table_stride;
  pa.bs = bt.block_size;
  pa.num_slots = bt.num_slots;
  pa.max_positions = c.max_positions;
  pa.M = M;
  pa.T = Tt;
  pa.V = c.vocab;
  pa.H = c.hidden;
  pa.pos_out = pos;
  pa.slot_out = slot;
  pa.status = status;
  int rc = launch_prep_embed<T>(pa, static_cast<const T*>(m.w.embed), hidden, s, false);
  if (rc) return rc;

  const bool pdl = true;
  const size_t layer_pool = static_cast<size_t>(bt.num_slots) * c.n_kv_heads * c.head_dim;
  // With a trace buffer, tensor-core GEMM launch i (4 per layer, then the head) records its
  // CTAs' timing (GemmScratch::trace).
  int gemm_slot = 0;
  auto gemm = [&](const GemmShape& sh, const CUtensorMap* wmap, const CUtensorMap* xmap, const void* w, const T* x,
                  const Epilogue& e, const void* norm_w = nullptr) -> int {
    GemmScratch g = gscr;
    if (bt.trace) {
      g.trace = reinterpret_cast<unsigned long long*>(bt.trace);
      g.trace_slot = gemm_slot++;
    }
    if (tc && norm_w) {  // X = RMSNorm(hidden) built inside the GEMM
      GemmNorm nrm;
      nrm.x = reinterpret_cast<const __nv_bfloat16*>(hidden);
      nrm.w = static_cast<const __nv_bfloat16*>(norm_w);
      nrm.eps = c.rms_eps;
      return launch_gemm_tc(sh, *wmap, *xmap, e, g, status, s, pdl, &nrm);
    }
    if (tc) return launch_gemm_tc(sh, *wmap, *xmap, e, g, status, s, pdl);
    return launch_gemm_simt<T>(sh, static_cast<const T*>(w), x, e, gscr, status, s, pdl);
  };
  // Decode-step schedule (bf16 only): the GEMV kernels, with the two RMSNorms of each layer
  // folded into the q/k/v and gate/up kernels. With a trace buffer, launch i of the forward
  // (4 per layer, then the head) records its timing in trace[4 i .. 4 i + 3].
  int gemv_slot = 0;
  auto gemv = [&](const GemvPlan& p, const void* w, const T* x, const void* norm_w, const Epilogue& e, int N,
                  int K) -> int {
    GemvArgs g = {};
    g.w = static_cast<const __nv_bfloat16*>(w);
    g.x = reinterpret_cast<const __nv_bfloat16*>(x);
    g.norm_w = static_cast<const __nv_bfloat16*>(norm_w);
    g.eps = c.rms_eps;
    g.M = M;
    g.N = N;
    g.K = K;
    g.p = p;
    g.e = e;
    g.status = status;
    g.trace = reinterpret_cast<unsigned long long*>(bt.trace);
    g.trace_slot = gemv_slot++;
    return launch_gemv(g, s, pdl);
  };

  for (int l = 0; l < c.n_layers; ++l) {
    const specb200_layer_weights& L = m.layers[l];
    const LayerMaps* mp = tc ? &m.maps[l] : nullptr;
    if (cv.defer && l > 0) {  // the previous layer's down projection joins the residual stream here
      rc = launch_residual_norm(reinterpret_cast<__nv_bfloat16*>(hidden), resid_parts, cv.g_down.splits, M, M, c.hidden,
                                static_cast<const __nv_bfloat16*>(L.attn_norm), c.rms_eps,
                                reinterpret_cast<__nv_bfloat16*>(xbuf), nullptr, 1, s, pdl);
      if (rc) return rc;
    } else if (!cv.gemv && !cv.norm_qkv &&
               (rc = launch_rmsnorm<T>(hidden, static_cast<const T*>(L.attn_norm), M, c.hidden, c.rms_eps, xbuf, nullptr,
                                       1, s, pdl))) {
      return rc;
    }
    Epilogue eq = {};
    eq.op = EPI_QKV;
    eq.out = qbuf;
    eq.ldo = qd;
    eq.k_pool = static_cast<T*>(bt.k_pool) + l * layer_pool;
    eq.v_pool = static_cast<T*>(bt.v_pool) + l * layer_pool;
    eq.slot = slot;
    eq.pos = pos;
    eq.rope_cos = m.w.rope_cos;
    eq.rope_sin = m.w.rope_sin;
    eq.n_heads = c.n_heads;
    eq.n_kv_heads = c.n_kv_heads;
    eq.head_dim = c.head_dim;
    Epilogue eqp = {};  // deferred: partials for the cluster attention
    eqp.op = EPI_PARTIAL;
    eqp.out = ws + cv.qkv_parts;
    eqp.ldo = m.qkv_n;
    if (cv.qkv_attn) {
      ++gemv_slot;  // computed by the attention clusters; keep the trace slots in place
    } else {
      rc = cv.gemv ? gemv(cv.v_qkv, L.w_qkv, hidden, L.attn_norm, eq, m.qkv_n, c.hidden)
                   : gemm(cv.g_qkv, mp ? &mp->qkv : nullptr, &x_hidden, L.w_qkv, xbuf, cv.defer_qkv ? eqp : eq,
                          cv.norm_qkv ? L.attn_norm : nullptr);
      if (rc) return rc;
    }

    AttnArgs aa;
    aa.q = qbuf;
    aa.k_pool = eq.k_pool;
    aa.v_pool = eq.v_pool;
    aa.table = bt.block_table;
    aa.table_stride = bt.table_stride;
    aa.bs = bt.block_size;
    aa.past = bt.past_len;
    aa.n_new = bt.n_new;
    aa.B = B;
    aa.T = Tt;
    aa.Hq = c.n_heads;
    aa.Hkv = c.n_kv_heads;
    aa.D = c.head_dim;
    aa.scale = 1.0f / sqrtf(static_cast<float>(c.head_dim));
    aa.out = attn;
    aa.status = status;
    if (cv.defer_qkv) {
      aa.qkv_parts = reinterpret_cast<const float*>(ws + cv.qkv_parts);
      aa.qkv_splits = cv.g_qkv.splits;
      aa.qkv_n = m.qkv_n;
      aa.rope_cos = m.w.rope_cos;
      aa.rope_sin = m.w.rope_sin;
      aa.max_positions = c.max_positions;
    }
    if (bt.trace) {  // after the GEMV or GEMM launch records
      aa.trace = reinterpret_cast<unsigned long long*>(bt.trace) +
                 static_cast<size_t>(4 * c.n_layers + 1) * (cv.gemv ? kGemvTraceCtas * kGemvTraceStamps : kGemmTraceCtas * 8);
      aa.trace_slot = l;
    }
    if (cv.qkv_attn) {  // the q/k/v projection and the attention, one launch
      aa.rope_cos = m.w.rope_cos;
      aa.rope_sin = m.w.rope_sin;
      aa.max_positions = c.max_positions;
      rc = launch_attention_qkv(aa, cv.ap_qkv, cv.qkv_pairs, static_cast<const __nv_bfloat16*>(L.w_qkv),
                                reinterpret_cast<const __nv_bfloat16*>(hidden),
                                static_cast<const __nv_bfloat16*>(L.attn_norm), slot, c.rms_eps, c.hidden, s, pdl);
      if (rc) return rc;
    } else if (cv.attn_o) {  // attention and the o projection with the residual add, one launch
      rc = launch_attention_o(aa, cv.ap_o, cv.ao_P, cv.ao_rows, static_cast<const __nv_bfloat16*>(L.w_o),
                              reinterpret_cast<__nv_bfloat16*>(hidden), c.hidden, s, pdl);
      if (rc) return rc;
    } else if ((rc = launch_attention<T>(aa, cv.ap, attn_counters, attn_parts, s, pdl))) {
      return rc;
    }

    Epilogue er = {};
    er.op = EPI_RESID;
    er.out = hidden;
    er.ldo = c.hidden;
    Epilogue ep = {};  // deferred: partials for launch_residual_norm
    ep.op = EPI_PARTIAL;
    ep.out = resid_parts;
    ep.ldo = c.hidden;
    if (!cv.attn_o) {
      rc = cv.gemv ? gemv(cv.v_o, L.w_o, attn, nullptr, er, c.hidden, qd)
                   : gemm(cv.g_o, mp ? &mp->o : nullptr, &x_attn, L.w_o, attn, cv.defer ? ep : er);
      if (rc) return rc;
    } else {
      ++gemv_slot;  // keep the trace slots of the remaining launches in place
    }
    if (cv.defer) {
      rc = launch_residual_norm(reinterpret_cast<__nv_bfloat16*>(hidden), resid_parts, cv.g_o.splits, M, M, c.hidden,
                                static_cast<const __nv_bfloat16*>(L.mlp_norm), c.rms_eps,
                                reinterpret_cast<__nv_bfloat16*>(xbuf), nullptr, 1, s, pdl);
      if (rc) return rc;
    } else if (!cv.gemv && !cv.norm_gu &&
               (rc = launch_rmsnorm<T>(hidden, static_cast<const T*>(L.mlp_norm), M, c.hidden, c.rms_eps, xbuf, nullptr,
                                       1, s, pdl))) {
      return rc;
    }
    Epilogue eg = {};
    eg.op = EPI_SILU_MUL;
    eg.out = act;
    eg.ldo = c.intermediate;
    rc = cv.gemv ? gemv(cv.v_gu, L.w_gate_up, hidden, L.mlp_norm, eg, 2 * c.intermediate, c.hidden)
                 : gemm(cv.g_gu, mp ? &mp->gu : nullptr, &x_hidden, L.w_gate_up, xbuf, eg, cv.norm_gu ? L.mlp_norm : nullptr);
    if (rc) return rc;
    rc = cv.gemv ? gemv(cv.v_down, L.w_down, act, nullptr, er, c.hidden, c.intermediate)
                 : gemm(cv.g_down, mp ? &mp->down : nullptr, &x_act, L.w_down, act, cv.defer ? ep : er);
    if (rc) return rc;
  }
  return run_head<T>(m, bt, ws, cv, s, tc ? &x_final : nullptr);
}

// Final RMSNorm (of each sequence's last valid row when last_only) and the LM head GEMM into
// fp32 logits, reading the residual stream from the workspace's hidden buffer.
template <typename T>
int run_head(const Model& m, const specb200_batch& bt, char* ws, const Carve& cv, cudaStream_t s,
             const CUtensorMap* x_final) {
  const specb200_model_config& c = m.cfg;
  const int rows_out = bt.last_only ? bt.B : bt.B * bt.T;
  T* hidden = reinterpret_cast<T*>(ws + cv.hidden);
  T* xbuf = reinterpret_cast<T*>(ws + cv.xbuf);
  GemmScratch gscr{reinterpret_cast<int*>(ws + cv.gemm_counters), reinterpret_cast<float*>(ws + cv.gemm_parts)};
  Epilogue eh = {};
  eh.op = EPI_STORE;
  eh.out_f32 = 1;
  eh.out = bt.logits;
  eh.ldo = c.vocab;
  if (cv.gemv_head) {  // final norm (with the last-token selection) folded into the LM head
    GemvArgs g = {};
    g.w = static_cast<const __nv_bfloat16*>(m.w.lm_head);
    g.x = reinterpret_cast<const __nv_bfloat16*>(hidden);
    g.norm_w = static_cast<const __nv_bfloat16*>(m.w.final_norm);
    g.sel_n_new = bt.last_only ? bt.n_new : nullptr;
    g.T_tokens = bt.T;
    g.eps = c.rms_eps;
    g.M = rows_out;
    g.N = c.vocab;
    g.K = c.hidden;
    g.p = cv.v_head;
    g.e = eh;
    g.status = bt.status;
    g.trace = reinterpret_cast<unsigned long long*>(bt.trace);
    g.trace_slot = 4 * c.n_layers;
    return launch_gemv(g, s, true);
  }
  if (bt.trace && !cv.gemv) {
    gscr.trace = reinterpret_cast<unsigned long long*>(bt.trace);
    gscr.trace_slot = 4 * c.n_layers;
  }
  if (cv.norm_head) {  // the final norm and the last-token selection inside the LM head GEMM
    GemmNorm nrm;
    nrm.x = reinterpret_cast<const __nv_bfloat16*>(hidden);
    nrm.w = static_cast<const __nv_bfloat16*>(m.w.final_norm);
    nrm.sel_n_new = bt.last_only ? bt.n_new : nullptr;
    nrm.T_tokens = bt.T;
    nrm.eps = c.rms_eps;
    return launch_gemm_tc(cv.g_head, m.head, *x_final, eh, gscr, bt.status, s, true, &nrm);
  }
  int rc;
  if (cv.defer) {  // the last layer's down projection joins the residual stream with the final norm
    rc = launch_residual_norm(reinterpret_cast<__nv_bfloat16*>(hidden), reinterpret_cast<const float*>(ws + cv.resid_parts),
                              cv.g_down.splits, bt.B * bt.T, rows_out, c.hidden,
                              static_cast<const __nv_bfloat16*>(m.w.final_norm), c.rms_eps,
                              reinterpret_cast<__nv_bfloat16*>(xbuf), bt.last_only ? bt.n_new : nullptr, bt.T, s, true);
  } else {
    rc = launch_rmsnorm<T>(hidden, static_cast<const T*>(m.w.final_norm), rows_out, c.hidden, c.rms_eps, xbuf,
                           bt.last_only ? bt.n_new : nullptr, bt.T, s, true);
  }
  if (rc) return rc;
  if (c.dtype == SPECB200_BF16) return launch_gemm_tc(cv.g_head, m.head, *x_final, eh, gscr, bt.status, s, true);
  return launch_gemm_simt<T>(cv.g_head, static_cast<const T*>(m.w.lm_head), xbuf, eh, gscr, bt.status, s, true);
}

// Decode-shaped calls of small bf16 models: the layer stack on one thread-block cluster
// (chain.cu), then the final norm and the LM head on the whole GPU.
int run_chain(const Model& m, const specb200_batch& bt, char* ws, const Carve& cv, cudaStream_t s) {
  const specb200_model_config& c = m.cfg;
  ChainArgs a = {};
  a.n_layers = c.n_layers;
  a.H = c.hidden;
  a.Hq = c.n_heads;
  a.Hkv = c.n_kv_heads;
  a.D = c.head_dim;
  a.I = c.intermediate;
  a.eps = c.rms_eps;
  a.attn_scale = 1.0f / sqrtf(static_cast<float>(c.head_dim));
  a.max_positions = c.max_positions;
  a.V = c.vocab;
  a.embed = static_cast<const __nv_bfloat16*>(m.w.embed);
  a.rope_cos = m.w.rope_cos;
  a.rope_sin = m.w.rope_sin;
  for (int l = 0; l < c.n_layers; ++l) {
    const specb200_layer_weights& L = m.layers[l];
    a.layers[l].attn_norm = static_cast<const __nv_bfloat16*>(L.attn_norm);
    a.layers[l].mlp_norm = static_cast<const __nv_bfloat16*>(L.mlp_norm);
    a.layers[l].qkv = static_cast<const uint8_t*>(L.p_qkv);
    a.layers[l].o = static_cast<const uint8_t*>(L.p_o);
    a.layers[l].gu = static_cast<const uint8_t*>(L.p_gate_up);
    a.layers[l].down = static_cast<const uint8_t*>(L.p_down);
  }
  a.B = bt.B;
  a.T = bt.T;
  a.M = bt.B * bt.T;
  a.ids = bt.input_ids;
  a.n_new = bt.n_new;
  a.past = bt.past_len;
  a.table = bt.block_table;
  a.table_stride = bt.table_stride;
  a.bs = bt.block_size;
  a.num_slots = bt.num_slots;
  a.k_pool = static_cast<__nv_bfloat16*>(bt.k_pool);
  a.v_pool = static_cast<__nv_bfloat16*>(bt.v_pool);
  a.h = reinterpret_cast<__nv_bfloat16*>(ws + cv.hidden);
  for (int i = 0; i < 4; ++i) a.ph[i] = cv.cph[i];
  a.splits = cv.csplits;
  a.C = m.chain_C;
  a.L = cv.cl;
  a.ring_evict_first = m.ring_evict_first;
  // GEMM units on the tensor cores by default; SPECB200_CHAIN_FMA=1 runs calls of at most
  // kChainFmaRows rows on the CUDA cores instead (measured 1.24 vs 1.20 ms per draft step).
  a.fma = a.M <= kChainFmaRows && env_int("SPECB200_CHAIN_FMA", 0) == 1;
  a.status = bt.status;
  a.trace = reinterpret_cast<unsigned long long*>(bt.trace);
  int rc = launch_chain(a, s);
  if (rc) return rc;
  const int rows_out = bt.last_only ? bt.B : bt.B * bt.T;
  CUtensorMap x_final{};
  if (!make_tmap_bf16_2d(&x_final, ws + cv.xbuf, c.hidden, rows_out, kTileK, cv.g_head.BN)) return SPECB200_ERR_ARG;
  return run_head<__nv_bfloat16>(m, bt, ws, cv, s, &x_final);
}

}  // namespace
}  // namespace specb200

using namespace specb200;
extern "C" int specb200_set_error(int code, const char* msg);

extern "C" int specb200_model_create(const specb200_model_config* config, const specb200_model_weights* weights,
                                     void** handle) {
  if (!config || !weights || !handle || !weights->layers) return specb200_set_error(SPECB200_ERR_ARG, "model: null");
  const specb200_model_config& c = *config;
  if (c.n_layers <= 0 || c.hidden <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 || c.n_heads % c.n_kv_heads ||
      c.vocab <= 0 || c.intermediate <= 0 || c.max_positions <= 0)
    return specb200_set_error(SPECB200_ERR_ARG, "model: bad dimensions");
  if (c.head_dim != 16 && c.head_dim != 32 && c.head_dim != 64)
    return specb200_set_error(SPECB200_ERR_UNSUPPORTED, "model: head_dim must be 16, 32 or 64");
  if (c.intermediate % 64 || c.hidden % 8 || (c.n_heads * c.head_dim) % 8)
    return specb200_set_error(SPECB200_ERR_UNSUPPORTED, "model: intermediate % 64 and hidden % 8 required");
  if (c.dtype != SPECB200_F32 && c.dtype != SPECB200_BF16) return specb200_set_error(SPECB200_ERR_UNSUPPORTED, "model: dtype");
  Model* m = new Model();
  m->cfg = c;
  m->w = *weights;
  m->layers.assign(weights->layers, weights->layers + c.n_layers);
  m->w.layers = m->layers.data();
  m->qkv_n = (c.n_heads + 2 * c.n_kv_heads) * c.head_dim;
  m->stream_ok = c.dtype == SPECB200_BF16 && c.head_dim == 64 && c.n_layers <= kStreamMaxLayers &&
                 c.hidden <= 2048 && c.n_heads * c.head_dim <= 2048 && c.hidden % 64 == 0 && weights->p_lm_head;
  for (int l = 0; l < c.n_layers && m->stream_ok; ++l) {
    const specb200_layer_weights& L = weights->layers[l];
    m->stream_ok = L.p_qkv && L.p_o && L.p_gate_up && L.p_down;
  }
  // The layer-stream schedule is opt-in (SPECB200_STREAM=1): its per-phase latency chain (grid
  // barrier, operand build, split-K reduction, attention items) now costs more than the launch
  // gaps it removes (1.7B verify at 644 cached tokens: 2.16 ms vs 1.90 ms per step on the
  // per-layer kernels; 135M draft step: 1.62 vs 1.17 ms). Even when enabled, small models stay
  // on the per-layer kernels (layers under SPECB200_STREAM_MIN_LAYER_MB, default 32 MB).
  const size_t layer_bytes = 2ull * c.hidden *
                             (static_cast<size_t>(m->qkv_n) + static_cast<size_t>(c.n_heads) * c.head_dim + 3ull * c.intermediate);
  if (layer_bytes < (static_cast<size_t>(env_int("SPECB200_STREAM_MIN_LAYER_MB", 32)) << 20)) m->stream_ok = false;
  if (env_int("SPECB200_STREAM", 0) != 1) m->stream_ok = false;
  // Layer-stream schedule knobs (L2 prefetch distance in GEMM phases; ring eviction hint).
  m->prefetch_ahead = env_int("SPECB200_STREAM_PREFETCH", 0);  // measured: prefetching slows it
  m->ring_evict_first = env_int("SPECB200_STREAM_EVICT_FIRST", 1);
  // Size the persistent grid now, outside any stream capture (it sets a function attribute).
  if (m->stream_ok && stream_grid_size() <= 0) m->stream_ok = false;
  // The cluster layer-chain kernel: same packed weights, small models (hidden <= 1024) only.
  // Opt-in (SPECB200_CHAIN=1): on the 135M draft it is not yet faster than the per-layer
  // kernels (measured 1.20 vs 1.17-1.29 ms per decode step).
  const bool chain_weights = c.dtype == SPECB200_BF16 && c.head_dim == 64 && c.hidden <= 1024 &&
                             c.n_layers <= kStreamMaxLayers && env_int("SPECB200_CHAIN", 0) == 1;
  bool packed = chain_weights;
  for (int l = 0; l < c.n_layers && packed; ++l) {
    const specb200_layer_weights& L = weights->layers[l];
    packed = L.p_qkv && L.p_o && L.p_gate_up && L.p_down;
  }
  m->chain_C = packed ? chain_cluster_size() : 0;
  attention_prepare();  // function attributes are set here, outside any stream capture
  gemm_prepare();
  norm_prepare();
  // Folding the RMSNorms into the tensor-core GEMMs is opt-in (SPECB200_GEMM_NORM=1): the
  // operand build and its 64 KB of shared memory (which keeps the attention CTAs off the SMs
  // while the q/k/v GEMM runs) cost more than the norm launches (1.66 vs 1.58 ms per verify).
  m->gemm_norm = c.dtype == SPECB200_BF16 && env_int("SPECB200_GEMM_NORM", 0) == 1;
  m->defer_resid = env_int("SPECB200_DEFER_RESID", 1) == 1;
  m->defer_qkv = env_int("SPECB200_DEFER_QKV", 1) == 1;
  // q/k/v projection inside the attention clusters of the GEMV schedule: opt-in
  // (SPECB200_DRAFT_QKV=1). One launch fewer per layer, but 0.608 vs 0.578 ms per 1-token
  // draft step of the 135M model: its 80 KB CTAs do not fit beside the down GEMV's, so the
  // clusters start late and lose the early weight and key loads.
  m->qkv_attn = env_int("SPECB200_DRAFT_QKV", 0) == 1;
  // Decode-step GEMV schedule: bf16 weights, 16-byte aligned rows (SPECB200_GEMV=0 turns it off).
  auto al16 = [](const void* p) { return p && (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  m->gemv_ok = c.dtype == SPECB200_BF16 && env_int("SPECB200_GEMV", 1) == 1 && al16(weights->lm_head) &&
               al16(weights->final_norm) && gemv_prepare();
  for (int l = 0; l < c.n_layers && m->gemv_ok; ++l) {
    const specb200_layer_weights& L = weights->layers[l];
    m->gemv_ok = al16(L.w_qkv) && al16(L.w_o) && al16(L.w_gate_up) && al16(L.w_down) && al16(L.attn_norm) &&
                 al16(L.mlp_norm);
  }
  if (c.dtype == SPECB200_BF16) {
    const int qd = c.n_heads * c.head_dim;
    m->maps.resize(c.n_layers);
    bool ok = make_tmap_bf16_2d(&m->head, weights->lm_head, c.hidden, c.vocab, kTileK, kTileN);
    for (int l = 0; l < c.n_layers && ok; ++l) {
      const specb200_layer_weights& L = m->layers[l];
      ok = make_tmap_bf16_2d(&m->maps[l].qkv, L.w_qkv, c.hidden, m->qkv_n, kTileK, kTileN) &&
           make_tmap_bf16_2d(&m->maps[l].o, L.w_o, qd, c.hidden, kTileK, kTileN) &&
           make_tmap_bf16_2d(&m->maps[l].gu, L.w_gate_up, c.hidden, 2 * c.intermediate, kTileK, kTileN) &&
           make_tmap_bf16_2d(&m->maps[l].down, L.w_down, c.intermediate, c.hidden, kTileK, kTileN);
    }
    if (!ok) {
      delete m;
      return specb200_set_error(SPECB200_ERR_ARG, "model: TMA descriptor for a weight (16-byte alignment?)");
    }
  }
  *handle = m;
  return SPECB200_OK;
}

// Kernel launches of one forward call: 3 for the layer chain (chain kernel, final norm, LM head),
// 1 for the layer stream, 2 + 5 L for the GEMV schedule (prep, 5 per layer, head; 4 per layer
// when the o or the q/k/v projection runs inside the attention clusters), and for the
// per-layer kernels 2 + 5 L (prep, 5 per layer, head) plus one launch per RMSNorm that is not
// folded into its GEMM (at most 3 + 7 L).
extern "C" int specb200_forward_launches(void* model, int B, int T) {
  if (!model || B <= 0 || T <= 0) return 0;
  const Model& m = *static_cast<Model*>(model);
  ChainPhase ph[4];
  int splits = 0;
  ChainLayout L;
  if (use_chain(m, B, T, ph, &splits, &L)) return 3;
  int grid = 0, mc = 0;
  if (use_stream(m, B, T, &grid, &mc)) return 1;
  GemvPlan v[5];
  bool head_gemv = false;
  const int M = B * T;
  const bool tc = m.cfg.dtype == SPECB200_BF16;
  const bool head_norm = m.gemm_norm && gemm_norm_fits(plan_gemm(B, m.cfg.vocab, m.cfg.hidden, tc));
  if (use_gemv(m, M, B, &v[0], &v[1], &v[2], &v[3], &v[4], &head_gemv)) {
    AttnPlan ap;
    int P = 0, rows = 0;  // counted for contexts up to 1024 keys
    const specb200_model_config& c = m.cfg;
    const bool ao = plan_attention_o(B, T, c.n_heads, c.n_kv_heads, c.head_dim, c.hidden, 1024, &ap, &P, &rows);
    const bool fq = !ao && m.qkv_attn && plan_attention_qkv(T, c.n_heads, c.n_kv_heads, c.head_dim, c.hidden, 1024, &ap, &P);
    return (head_gemv || head_norm ? 2 : 3) + (ao || fq ? 4 : 5) * m.cfg.n_layers;
  }
  const int norms = (m.gemm_norm && gemm_norm_fits(plan_gemm(M, m.qkv_n, m.cfg.hidden, tc)) ? 0 : 1) +
                    (m.gemm_norm && gemm_norm_fits(plan_gemm(M, 2 * m.cfg.intermediate, m.cfg.hidden, tc)) ? 0 : 1);
  return 2 + (head_norm ? 0 : 1) + (5 + norms) * m.cfg.n_layers;
}

extern "C" int specb200_forward_uses_stream(void* model, int B, int T) {
  if (!model || B <= 0 || T <= 0) return 0;
  const Model& m = *static_cast<Model*>(model);
  ChainPhase ph[4];
  int splits = 0;
  ChainLayout L;
  if (use_chain(m, B, T, ph, &splits, &L)) return 2;
  int grid = 0, mc = 0;
  if (use_stream(m, B, T, &grid, &mc)) return 1;
  GemvPlan v[5];
  bool head_gemv = false;
  return use_gemv(m, B * T, B, &v[0], &v[1], &v[2], &v[3], &v[4], &head_gemv) ? 3 : 0;
}

extern "C" int specb200_model_destroy(void* handle) {
  delete static_cast<Model*>(handle);
  return SPECB200_OK;
}

extern "C" size_t specb200_forward_workspace_bytes(void* model, int B, int T, int max_kv_len) {
  if (!model || B <= 0 || T <= 0) return 0;
  const Model& m = *static_cast<Model*>(model);
  return std::max(carve(m, B, T, max_kv_len, 0).total, carve(m, B, T, max_kv_len, 1).total);
}

extern "C" int specb200_forward(void* model, const specb200_batch* batch, void* workspace, size_t workspace_bytes,
                                void* stream) {
  if (!model || !batch || !workspace) return specb200_set_error(SPECB200_ERR_ARG, "forward: null pointer");
  const Model& m = *static_cast<Model*>(model);
  const specb200_batch& bt = *batch;
  if (bt.B <= 0 || bt.T <= 0 || bt.block_size <= 0 || bt.table_stride <= 0 || bt.num_slots <= 0 || bt.max_kv_len <= 0)
    return specb200_set_error(SPECB200_ERR_ARG, "forward: bad batch sizes");
  if (!bt.input_ids || !bt.n_new || !bt.past_len || !bt.block_table || !bt.k_pool || !bt.v_pool || !bt.logits)
    return specb200_set_error(SPECB200_ERR_ARG, "forward: null batch pointer");
  Carve cv = carve(m, bt.B, bt.T, bt.max_kv_len, bt.last_only);
  if (workspace_bytes < cv.total) return specb200_set_error(SPECB200_ERR_WORKSPACE, "forward: workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (bt.status) cudaMemsetAsync(bt.status, 0, sizeof(int32_t), s);
  int rc = cv.chain  ? run_chain(m, bt, static_cast<char*>(workspace), cv, s)
           : cv.stream ? run_stream(m, bt, static_cast<char*>(workspace), cv, s)
           : m.cfg.dtype == SPECB200_BF16 ? run_forward<__nv_bfloat16>(m, bt, static_cast<char*>(workspace), cv, s)
                                          : run_forward<float>(m, bt, static_cast<char*>(workspace), cv, s);
  if (rc != SPECB200_OK) {
    cudaError_t e = cudaGetLastError();
    return specb200_set_error(rc, e != cudaSuccess ? cudaGetErrorString(e) : "forward: launch failed");
  }
  return SPECB200_OK;
}
