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
#include <atomic>
#include <cstdlib>
#include <vector>

#include "attn_cluster.cuh"
#include "attn_core.cuh"
#include "gemm.cuh"
#include "gemv.cuh"
#include "kernels.cuh"

namespace specb200 {
namespace {

struct LayerMaps {
  CUtensorMap qkv, o, gu, down;
};

struct Model {
  specb200_model_config cfg;
  specb200_model_weights w;
  std::vector<specb200_layer_weights> layers;
  std::vector<LayerMaps> maps;
  CUtensorMap head;
  int qkv_n;
  bool gemv_ok = false;  // bf16 weights usable by the decode-step GEMV kernels (gemv.cu)
};


size_t align256(size_t x) { return (x + 255) / 256 * 256; }

struct Carve {
  size_t gemm_counters, attn_counters, hidden, xbuf, qbuf, attn, act, pos, slot, gemm_parts, attn_parts, resid_parts,
      qkv_parts, total;
  // per-layer schedule: the o and down GEMMs store split partials (EPI_PARTIAL) and the RMSNorm
  // launch that follows each adds them to the residual stream (launch_residual_norm)
  bool defer;
  // ... and the q/k/v GEMM stores split partials that the cluster attention sums, rotates and
  // writes to the pool itself (no ticket, no epilogue tail in the GEMM)
  bool defer_qkv;
  GemmShape g_qkv, g_o, g_gu, g_down, g_head;
  bool gemv;  // decode-step schedule: the per-layer order with GEMV kernels and fused norms
  bool gemv_head;  // ... and the LM head as a GEMV with the final norm folded in
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
  *head_gemv = plan_gemv(EPI_STORE, rows_out, c.vocab, c.hidden, 0, head) && head->stages == 1;
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
  // o's partials are summed by the following residual RMSNorm: it may split K down to 4
  // k-blocks per CTA (B = 64 verify: 12.25 -> 8.75 us per o GEMM). q/k/v keeps 16: a split q/k/v
  // tile runs its RoPE epilogue after the reduction (30.5 -> 49.6 us per GEMM at B = 64).
  r.g_o = plan_gemm(M, c.hidden, qd, tc, 4);
  r.g_gu = plan_gemm(M, 2 * c.intermediate, c.hidden, tc);
  r.g_down = plan_gemm(M, c.hidden, c.intermediate, tc);
  r.g_head = plan_gemm(rows_out, c.vocab, c.hidden, tc);
  r.gemv_head = false;
  r.defer = tc;
  if (r.defer) {  // the residual-norm kernel sums at most 8 partials per element
    r.g_o.splits = std::min(r.g_o.splits, 8);
    r.g_down.splits = std::min(r.g_down.splits, 8);
    r.defer = residual_norm_fits(r.g_o.splits, c.hidden) && residual_norm_fits(r.g_down.splits, c.hidden);
  }
  r.gemv = use_gemv(m, M, rows_out, &r.v_qkv, &r.v_o, &r.v_gu, &r.v_down, &r.v_head, &r.gemv_head);
  r.defer = r.defer && !r.gemv;
  r.ap = plan_attention(B, T, c.n_heads, c.n_kv_heads, max_kv_len, tc && c.head_dim == 64);
  r.defer_qkv = r.defer && r.ap.mma == 2 && c.head_dim == 64 && r.g_qkv.splits <= kQkvMaxSplits;
  // The two ticket-counter regions sit at fixed offsets so that they stay zero across calls
  // of every shape; everything after them is rewritten before it is read.
  size_t off = 0;
  r.gemm_counters = off; off += align256(kGemmCounterBytes);
  r.attn_counters = off; off += align256(kAttnCounterBytes);
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
  r.total = off;
  return r;
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

  // One token-operand map per GEMM shape: the box height is that GEMM's token tile, which
  // the plan sizes per output width (q/k/v and gate/up both read xbuf, with their own tiles).
  CUtensorMap x_hidden{}, x_mlp{}, x_attn{}, x_act{}, x_final{};
  if (tc) {
    bool ok = make_tmap_bf16_2d(&x_hidden, xbuf, c.hidden, M, kTileK, cv.g_qkv.BN) &&
              make_tmap_bf16_2d(&x_mlp, xbuf, c.hidden, M, kTileK, cv.g_gu.BN) &&
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
                  const Epilogue& e) -> int {
    GemmScratch g = gscr;
    if (bt.trace) {
      g.trace = reinterpret_cast<unsigned long long*>(bt.trace);
      g.trace_slot = gemm_slot++;
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
    } else if (!cv.gemv &&
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
    rc = cv.gemv ? gemv(cv.v_qkv, L.w_qkv, hidden, L.attn_norm, eq, m.qkv_n, c.hidden)
                 : gemm(cv.g_qkv, mp ? &mp->qkv : nullptr, &x_hidden, L.w_qkv, xbuf, cv.defer_qkv ? eqp : eq);
    if (rc) return rc;

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
    if ((rc = launch_attention<T>(aa, cv.ap, attn_counters, attn_parts, s, pdl))) return rc;

    Epilogue er = {};
    er.op = EPI_RESID;
    er.out = hidden;
    er.ldo = c.hidden;
    Epilogue ep = {};  // deferred: partials for launch_residual_norm
    ep.op = EPI_PARTIAL;
    ep.out = resid_parts;
    ep.ldo = c.hidden;
    rc = cv.gemv ? gemv(cv.v_o, L.w_o, attn, nullptr, er, c.hidden, qd)
                 : gemm(cv.g_o, mp ? &mp->o : nullptr, &x_attn, L.w_o, attn, cv.defer ? ep : er);
    if (rc) return rc;
    if (cv.defer) {
      rc = launch_residual_norm(reinterpret_cast<__nv_bfloat16*>(hidden), resid_parts, cv.g_o.splits, M, M, c.hidden,
                                static_cast<const __nv_bfloat16*>(L.mlp_norm), c.rms_eps,
                                reinterpret_cast<__nv_bfloat16*>(xbuf), nullptr, 1, s, pdl);
      if (rc) return rc;
    } else if (!cv.gemv &&
               (rc = launch_rmsnorm<T>(hidden, static_cast<const T*>(L.mlp_norm), M, c.hidden, c.rms_eps, xbuf, nullptr,
                                       1, s, pdl))) {
      return rc;
    }
    Epilogue eg = {};
    eg.op = EPI_SILU_MUL;
    eg.out = act;
    eg.ldo = c.intermediate;
    rc = cv.gemv ? gemv(cv.v_gu, L.w_gate_up, hidden, L.mlp_norm, eg, 2 * c.intermediate, c.hidden)
                 : gemm(cv.g_gu, mp ? &mp->gu : nullptr, &x_mlp, L.w_gate_up, xbuf, eg);
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
  attention_prepare();  // function attributes are set here, outside any stream capture
  gemm_prepare();
  norm_prepare();
  // Decode-step GEMV schedule: bf16 weights, 16-byte aligned rows.
  auto al16 = [](const void* p) { return p && (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  m->gemv_ok = c.dtype == SPECB200_BF16 && al16(weights->lm_head) &&
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

// Kernel launches of one forward call: 2 + 5 L for the GEMV schedule
// (prep, 5 per layer, head; one more when the head is RMSNorm + the tensor-core GEMM), and for
// the per-layer kernels 3 + 7 L (prep, RMSNorm + 5 GEMM / attention launches + RMSNorm per
// layer, final norm, head). Counted for contexts of up to 1024 keys.
extern "C" int specb200_forward_launches(void* model, int B, int T) {
  if (!model || B <= 0 || T <= 0) return 0;
  const Model& m = *static_cast<Model*>(model);
  GemvPlan v[5];
  bool head_gemv = false;
  if (use_gemv(m, B * T, B, &v[0], &v[1], &v[2], &v[3], &v[4], &head_gemv))
    return (head_gemv ? 2 : 3) + 5 * m.cfg.n_layers;
  return 3 + 7 * m.cfg.n_layers;
}

// Which schedule a call runs: 3 = the decode-step GEMV kernels, 0 = one kernel per layer op.
extern "C" int specb200_forward_schedule(void* model, int B, int T) {
  if (!model || B <= 0 || T <= 0) return 0;
  const Model& m = *static_cast<Model*>(model);
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
  int rc = m.cfg.dtype == SPECB200_BF16 ? run_forward<__nv_bfloat16>(m, bt, static_cast<char*>(workspace), cv, s)
                                          : run_forward<float>(m, bt, static_cast<char*>(workspace), cv, s);
  if (rc != SPECB200_OK) {
    cudaError_t e = cudaGetLastError();
    return specb200_set_error(rc, e != cudaSuccess ? cudaGetErrorString(e) : "forward: launch failed");
  }
  return SPECB200_OK;
}

