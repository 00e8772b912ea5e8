// K8/K10: fused probabilities + accept-reject + residual sampling (one launch).
//
// Restates, as one kernel over logit or probability rows:
//   lm/sampling.py:13-18        probabilities(): T == 0 -> one-hot of the first maximum,
//                               else softmax(logits.float() / T)
//   spec/accept.py:44-79        accept_reject(): accept draft i iff u_i * q_i(x_i) < p_i(x_i),
//                               n = number of leading accepts, then one residual sample at row n
//   spec/accept.py:18-26        residual_distribution(): max(0, p - q) normalised, or p when it
//                               sums to 0; the bonus row (n == k) uses q = 0
//   spec/accept.py:29-35        sample_inverse_cdf(): first index whose cdf exceeds u * total,
//                               clamped to V - 1
//
// Grid (R, B): one CTA per input row (R = k+1 target rows, plus k draft rows when q is a
// real tensor). Each CTA streams its row once from HBM (128-bit loads) and leaves per-row
// statistics (max and sum of exp for the softmax, the value at the drafted token, the
// argmax) in the workspace. The last CTA of batch row b, found with an atomic ticket (no
// spin-wait), makes the accept decisions and draws the residual sample from row n, which
// it re-reads from L2. Decisions therefore cost one HBM pass over p and q.
#include "common.cuh"

namespace specb200 {
namespace {

constexpr int kAcceptThreads = 512;
constexpr int kAcceptWarps = kAcceptThreads / 32;

struct RowStat {
  float m;     // max of z = x / T (logit rows)
  float s;     // sum of exp(z - m)
  float zx;    // z (logit rows) or probability (probability rows) at the drafted token
  int amax;    // first index of the maximum (greedy rows)
};

struct AcceptArgs {
  const float* p;
  const float* q;
  const int64_t* draft;
  const float* u_accept;
  const float* u_residual;
  int B, k, V, R;
  int logits, greedy, q_onehot, q_present, decide_only, q_step_major;
  float temperature;
  int64_t* n_accepted;
  int64_t* next_token;
  int32_t* status;
  int* counters;   // [B]
  RowStat* stats;  // [B, R]
};

SPECB200_DEVINL const float* row_ptr(const AcceptArgs& a, int b, int r) {
  // rows 0..k: target positions; rows k+1..2k: draft positions 0..k-1
  if (r <= a.k) return a.p + (static_cast<int64_t>(b) * (a.k + 1) + r) * a.V;
  const int i = r - a.k - 1;
  if (a.q_step_major) return a.q + (static_cast<int64_t>(i) * a.B + b) * a.V;  // q [k, B, V]
  return a.q + (static_cast<int64_t>(b) * a.k + i) * a.V;                       // q [B, k, V]
}

// Block-wide combination of per-thread (max, sum-exp) pairs.
SPECB200_DEVINL void combine_ms(float& m, float& s, float m2, float s2) {
  float mx = fmaxf(m, m2);
  if (mx == -INFINITY) return;  // both empty
  s = s * expf(m - mx) + s2 * expf(m2 - mx);
  m = mx;
}

__device__ void row_statistics(const AcceptArgs& a, int b, int r, RowStat* out) {
  __shared__ float sh_m[kAcceptWarps], sh_s[kAcceptWarps];
  __shared__ int sh_i[kAcceptWarps];
  const float* row = row_ptr(a, b, r);
  const int i = r <= a.k ? r : r - a.k - 1;  // window position of this row
  const int64_t d = i < a.k ? a.draft[static_cast<int64_t>(b) * a.k + i] : -1;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool vec = (a.V % 4 == 0) && ((reinterpret_cast<uintptr_t>(row) & 15) == 0);

  if (!a.logits) {  // probability rows: only the value at the drafted token is needed
    if (tid == 0) {
      RowStat st{0.f, 1.f, 0.f, 0};
      if (d >= 0 && d < a.V) st.zx = row[d];
      *out = st;
    }
    return;
  }
  if (a.greedy) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
    if (vec) {
      const float4* r4 = reinterpret_cast<const float4*>(row);
      const int n4 = a.V / 4;
#pragma unroll 8
      for (int j = tid; j < n4; j += kAcceptThreads) {
        float4 v = __ldg(r4 + j);
        argmax_merge(best, bi, v.x, 4 * j);
        argmax_merge(best, bi, v.y, 4 * j + 1);
        argmax_merge(best, bi, v.z, 4 * j + 2);
        argmax_merge(best, bi, v.w, 4 * j + 3);
      }
    } else {
      for (int j = tid; j < a.V; j += kAcceptThreads) argmax_merge(best, bi, __ldg(row + j), j);
    }
    warp_argmax(best, bi);
    if (lane == 0) { sh_m[warp] = best; sh_i[warp] = bi; }
    __syncthreads();
    if (tid == 0) {
      for (int w = 1; w < kAcceptWarps; ++w) argmax_merge(best, bi, sh_m[w], sh_i[w]);
      RowStat st{best, 1.f, 0.f, bi == 0x7fffffff ? 0 : bi};
      *out = st;
    }
    return;
  }
  // softmax statistics of z = x / T, online per thread: 8 float4 (32 values) per chunk, one
  // rescale per chunk; at T == 1 the division is skipped (x / 1 is exact)
  const float T = a.temperature;
  const bool unit_t = (T == 1.f);
  float m = -INFINITY, s = 0.f;
  if (vec) {
    const float4* r4 = reinterpret_cast<const float4*>(row);
    const int n4 = a.V / 4;
    constexpr int kU = 8;
    for (int j0 = tid; j0 < n4; j0 += kU * kAcceptThreads) {
      float z[kU * 4];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int j = j0 + u * kAcceptThreads;
        float4 v = j < n4 ? __ldg(r4 + j) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        z[4 * u] = v.x; z[4 * u + 1] = v.y; z[4 * u + 2] = v.z; z[4 * u + 3] = v.w;
      }
      float mx = m;
#pragma unroll
      for (int i = 0; i < kU * 4; ++i) {
        if (!unit_t) z[i] = z[i] / T;
        mx = fmaxf(mx, z[i]);
      }
      if (mx != -INFINITY) {
        float acc = s * expf(m - mx);
#pragma unroll
        for (int i = 0; i < kU * 4; ++i) acc += expf(z[i] - mx);
        s = acc;
        m = mx;
      }
    }
  } else {
    for (int j = tid; j < a.V; j += kAcceptThreads) {
      float z = __ldg(row + j);
      if (!unit_t) z = z / T;
      float mx = fmaxf(z, m);
      if (mx != -INFINITY) {
        s = s * expf(m - mx) + expf(z - mx);
        m = mx;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    combine_ms(m, s, m2, s2);
  }
  if (lane == 0) { sh_m[warp] = m; sh_s[warp] = s; }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < kAcceptWarps; ++w) combine_ms(m, s, sh_m[w], sh_s[w]);
    RowStat st{m, s, 0.f, 0};
    if (d >= 0 && d < a.V) st.zx = row[d] / T;
    *out = st;
  }
}

// Probability of token x in target row pr (or draft row qr) for the finishing CTA.
SPECB200_DEVINL float prob_at(const AcceptArgs& a, const float* row, const RowStat& st, float inv_s, int x) {
  float v = row[x];
  if (!a.logits) return v;
  return expf(v / a.temperature - st.m) * inv_s;
}

// Residual sampling at row n: r = max(0, p_n - q_n); sample by inverse CDF with u.
// Pass A: the row is cut into 128-element segments (one warp x 4 consecutive elements per
// lane); every warp sums its segments (float4 loads, several segments in flight) into
// shared memory. The total gives the target u * total; warp 0 scans the segment sums to find
// the segment holding the crossing, then scans that segment element by element (pass B).
// Sums accumulate in double so both passes agree except within a few ulps of a boundary.
constexpr int kSeg = 128;
constexpr int kMaxSegs = 4096;  // V <= 524288
SPECB200_DEVINL void seg_values(const AcceptArgs& a, const float* prow, const RowStat& ps, float p_inv,
                                const float* qrow, const RowStat& qs, float q_inv, bool q_row, bool q_hot,
                                int64_t dn, int use_p, int x0, float (&v)[4]) {
  // 4 consecutive elements x0..x0+3 (x0 % 4 == 0); out-of-range elements are 0
  float pv[4], qv[4] = {0.f, 0.f, 0.f, 0.f};
  const bool full = x0 + 3 < a.V;
  const bool vec = full && (a.V % 4 == 0);
  if (vec) {
    const float4 t = *reinterpret_cast<const float4*>(prow + x0);
    pv[0] = t.x; pv[1] = t.y; pv[2] = t.z; pv[3] = t.w;
    if (q_row && !use_p) {
      const float4 u = *reinterpret_cast<const float4*>(qrow + x0);
      qv[0] = u.x; qv[1] = u.y; qv[2] = u.z; qv[3] = u.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      pv[j] = x0 + j < a.V ? prow[x0 + j] : -INFINITY;
      if (q_row && !use_p) qv[j] = x0 + j < a.V ? qrow[x0 + j] : -INFINITY;
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (x0 + j >= a.V) { v[j] = 0.f; continue; }
    float px = pv[j];
    if (a.logits) px = expf((a.temperature == 1.f ? px : px / a.temperature) - ps.m) * p_inv;
    if (use_p) { v[j] = px; continue; }
    float qx = 0.f;
    if (q_row) {
      qx = qv[j];
      if (a.logits) qx = expf((a.temperature == 1.f ? qx : qx / a.temperature) - qs.m) * q_inv;
    } else if (q_hot) {
      qx = (x0 + j == dn) ? 1.f : 0.f;
    }
    v[j] = fmaxf(px - qx, 0.f);  // torch.clamp(p - q, min=0)
  }
}

__device__ int64_t residual_sample(const AcceptArgs& a, int b, int n, const RowStat* st) {
  __shared__ double sh_seg[kMaxSegs];
  __shared__ double sh_part[kAcceptWarps];
  __shared__ double sh_total;
  __shared__ int64_t sh_token;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* prow = row_ptr(a, b, n);
  const RowStat ps = st[n];
  const float p_inv = 1.0f / ps.s;
  // q at row n: absent (k == 0 sampler), zero (bonus row), one-hot at the draft, or a row
  const bool bonus = n >= a.k;
  const bool q_row = a.q_present && !a.q_onehot && !bonus;
  const bool q_hot = a.q_present && a.q_onehot && !bonus;
  const int64_t dn = bonus ? -1 : a.draft[static_cast<int64_t>(b) * a.k + n];
  const float* qrow = q_row ? row_ptr(a, b, a.k + 1 + n) : nullptr;
  const RowStat qs = q_row ? st[a.k + 1 + n] : RowStat{0.f, 1.f, 0.f, 0};
  const float q_inv = 1.0f / qs.s;
  const int nseg = (a.V + kSeg - 1) / kSeg;

  auto segment_sums = [&](int use_p) {
    for (int s0 = warp; s0 < nseg; s0 += 4 * kAcceptWarps) {
      double acc[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int sg = s0 + u * kAcceptWarps;
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        if (sg < nseg) seg_values(a, prow, ps, p_inv, qrow, qs, q_inv, q_row, q_hot, dn, use_p, sg * kSeg + 4 * lane, v);
        acc[u] = static_cast<double>(v[0]) + v[1] + v[2] + v[3];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const double t = warp_sum_d(acc[u]);
        const int sg = s0 + u * kAcceptWarps;
        if (lane == 0 && sg < nseg) sh_seg[sg] = t;
      }
    }
    __syncthreads();
    double t = 0.0;
    for (int sg = tid; sg < nseg; sg += kAcceptThreads) t += sh_seg[sg];
    t = warp_sum_d(t);
    if (lane == 0) sh_part[warp] = t;
    __syncthreads();
    if (tid == 0) {
      double tot = 0.0;
      for (int w = 0; w < kAcceptWarps; ++w) tot += sh_part[w];
      sh_total = tot;
    }
    __syncthreads();
  };
  segment_sums(0);
  int use_p = 0;
  if (!(sh_total > 0.0)) {  // residual sums to 0: residual_distribution falls back to p
    use_p = 1;
    segment_sums(1);
  }
  const double target = static_cast<double>(a.u_residual[b]) * sh_total;
  if (tid == 0) sh_token = a.V - 1;  // searchsorted past the end, clamped
  __syncthreads();
  if (warp == 0) {
    // first segment whose running sum passes the target (warp scan over segment sums)
    double base = 0.0;
    int s_hit = nseg;
    for (int s0 = 0; s0 < nseg && s_hit == nseg; s0 += 32) {
      const int sg = s0 + lane;
      double v = sg < nseg ? sh_seg[sg] : 0.0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const double t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
      }
      const unsigned hit = __ballot_sync(0xffffffffu, sg < nseg && base + v > target);
      if (hit) {
        const int l = __ffs(hit) - 1;
        s_hit = s0 + l;
        const double before = __shfl_sync(0xffffffffu, v, l) - __shfl_sync(0xffffffffu, sg < nseg ? sh_seg[sg] : 0.0, l);
        base += before;
      } else {
        base += __shfl_sync(0xffffffffu, v, 31);
      }
    }
    // element scan from that segment on (continues if rounding put the crossing later)
    for (int sg = s_hit; sg < nseg; ++sg) {
      float v4[4];
      seg_values(a, prow, ps, p_inv, qrow, qs, q_inv, q_row, q_hot, dn, use_p, sg * kSeg + 4 * lane, v4);
      double e[4];
      e[0] = v4[0];
      e[1] = e[0] + v4[1];
      e[2] = e[1] + v4[2];
      e[3] = e[2] + v4[3];
      double lsum = e[3];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const double t = __shfl_up_sync(0xffffffffu, lsum, o);
        if (lane >= o) lsum += t;
      }
      const double excl = base + lsum - e[3];
      int first = 4;
#pragma unroll
      for (int j = 3; j >= 0; --j)
        if (sg * kSeg + 4 * lane + j < a.V && excl + e[j] > target) first = j;
      const unsigned hit = __ballot_sync(0xffffffffu, first < 4);
      if (hit) {
        const int l = __ffs(hit) - 1;
        const int fj = __shfl_sync(0xffffffffu, first, l);
        if (lane == 0) sh_token = sg * kSeg + 4 * l + fj;
        break;
      }
      base += __shfl_sync(0xffffffffu, lsum, 31);
    }
  }
  __syncthreads();
  return sh_token;
}

__global__ void __launch_bounds__(kAcceptThreads) accept_kernel(AcceptArgs a) {
  pdl_wait();
  const int r = blockIdx.x % a.R, b = blockIdx.x / a.R;  // b-major: a row's CTAs run together
  RowStat* st = a.stats + static_cast<int64_t>(b) * a.R;
  row_statistics(a, b, r, st + r);
  __shared__ int sh_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) sh_last = (atomicAdd(a.counters + b, 1) == a.R - 1);
  __syncthreads();
  if (!sh_last) return;
  __threadfence();
  // Last CTA of batch row b: decisions, then the residual/bonus sample.
  __shared__ RowStat sst[32];
  __shared__ int sh_n;
  if (threadIdx.x < a.R) {
    const RowStat* src = st + threadIdx.x;
    RowStat v;
    v.m = __ldcg(&src->m);
    v.s = __ldcg(&src->s);
    v.zx = __ldcg(&src->zx);
    v.amax = __ldcg(&src->amax);
    sst[threadIdx.x] = v;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    a.counters[b] = 0;  // ready for the next launch
    int n = 0;
    bool run = true;
    for (int i = 0; i < a.k; ++i) {
      const int64_t d = a.draft[static_cast<int64_t>(b) * a.k + i];
      if (d < 0 || d >= a.V) { set_status(a.status, SPECB200_ERR_RANGE); run = false; continue; }
      float px, qx = 1.f;
      if (a.greedy) {
        px = (sst[i].amax == d) ? 1.f : 0.f;
        if (a.q_present && !a.q_onehot) qx = (sst[a.k + 1 + i].amax == d) ? 1.f : 0.f;
      } else if (a.logits) {
        px = expf(sst[i].zx - sst[i].m) * (1.0f / sst[i].s);
        if (a.q_present && !a.q_onehot) {
          const RowStat& qs = sst[a.k + 1 + i];
          qx = expf(qs.zx - qs.m) * (1.0f / qs.s);
        }
      } else {
        px = sst[i].zx;
        if (a.q_present && !a.q_onehot) qx = sst[a.k + 1 + i].zx;
      }
      if (!(qx > 0.f)) set_status(a.status, SPECB200_ERR_ZERO_Q);
      const bool acc = a.u_accept[static_cast<int64_t>(b) * a.k + i] * qx < px;
      if (run && acc) ++n; else run = false;
    }
    sh_n = n;
    a.n_accepted[b] = n;
  }
  __syncthreads();
  if (a.decide_only) return;
  const int n = sh_n;
  if (a.greedy) {
    if (threadIdx.x == 0) a.next_token[b] = sst[n].amax;
    return;
  }
  const int64_t tok = residual_sample(a, b, n, sst);
  if (threadIdx.x == 0) a.next_token[b] = tok;
}

// probabilities() of lm/sampling.py:13-18, materialised: one-hot of the first maximum at
// T == 0, else softmax(x / T) = exp(z - max) * (1 / sum). One CTA per row.
__global__ void __launch_bounds__(kAcceptThreads)
    probabilities_kernel(const float* __restrict__ logits, int V, float T, float* __restrict__ out) {
  pdl_wait();
  __shared__ float sh_m[kAcceptWarps], sh_s[kAcceptWarps];
  __shared__ int sh_i[kAcceptWarps];
  __shared__ float sh_bm, sh_bs;
  __shared__ int sh_bi;
  const float* row = logits + static_cast<int64_t>(blockIdx.x) * V;
  float* o = out + static_cast<int64_t>(blockIdx.x) * V;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (T == 0.f) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int j = tid; j < V; j += kAcceptThreads) argmax_merge(best, bi, row[j], j);
    warp_argmax(best, bi);
    if (lane == 0) { sh_m[warp] = best; sh_i[warp] = bi; }
    __syncthreads();
    if (tid == 0) {
      for (int w = 1; w < kAcceptWarps; ++w) argmax_merge(best, bi, sh_m[w], sh_i[w]);
      sh_bi = bi == 0x7fffffff ? 0 : bi;
    }
    __syncthreads();
    for (int j = tid; j < V; j += kAcceptThreads) o[j] = (j == sh_bi) ? 1.f : 0.f;
    return;
  }
  float m = -INFINITY, s = 0.f;
  for (int j = tid; j < V; j += kAcceptThreads) {
    const float z = row[j] / T;
    const float mx = fmaxf(z, m);
    if (mx != -INFINITY) {
      s = s * expf(m - mx) + expf(z - mx);
      m = mx;
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, off);
    combine_ms(m, s, m2, s2);
  }
  if (lane == 0) { sh_m[warp] = m; sh_s[warp] = s; }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < kAcceptWarps; ++w) combine_ms(m, s, sh_m[w], sh_s[w]);
    sh_bm = m;
    sh_bs = 1.0f / s;
  }
  __syncthreads();
  for (int j = tid; j < V; j += kAcceptThreads) o[j] = expf(row[j] / T - sh_bm) * sh_bs;
}

}  // namespace
}  // namespace specb200

using namespace specb200;

extern "C" size_t specb200_accept_workspace_bytes(int B, int k) {
  const size_t R = 2 * static_cast<size_t>(k) + 1;
  return 256 + static_cast<size_t>(B) * sizeof(int) + 256 + static_cast<size_t>(B) * R * sizeof(RowStat);
}

extern "C" int specb200_set_error(int code, const char* msg);

extern "C" int specb200_accept(const float* p, const float* q, const int64_t* draft, const float* u_accept,
                               const float* u_residual, int B, int k, int V, int flags, float temperature,
                               int64_t* n_accepted, int64_t* next_token, int32_t* status, void* workspace,
                               size_t workspace_bytes, void* stream) {
  if (B <= 0 || k < 0 || V <= 0 || k > 15 || V > kMaxSegs * kSeg)
    return specb200_set_error(SPECB200_ERR_ARG, "accept: bad B/k/V (k must be 0..15, V <= 524288)");
  if (!p || !n_accepted || !workspace || !u_residual) return specb200_set_error(SPECB200_ERR_ARG, "accept: null pointer");
  if (k > 0 && (!draft || !u_accept)) return specb200_set_error(SPECB200_ERR_ARG, "accept: null draft/u_accept");
  if (!(flags & SPECB200_ACCEPT_DECIDE_ONLY) && !next_token) return specb200_set_error(SPECB200_ERR_ARG, "accept: null next_token");
  if (workspace_bytes < specb200_accept_workspace_bytes(B, k))
    return specb200_set_error(SPECB200_ERR_WORKSPACE, "accept: workspace too small");
  const bool logits = flags & SPECB200_ACCEPT_LOGITS;
  if (logits && !(temperature >= 0.f)) return specb200_set_error(SPECB200_ERR_ARG, "accept: temperature < 0");
  AcceptArgs a;
  a.p = p;
  a.q = q;
  a.draft = draft;
  a.u_accept = u_accept;
  a.u_residual = u_residual;
  a.B = B;
  a.k = k;
  a.V = V;
  a.q_onehot = (flags & SPECB200_ACCEPT_Q_ONEHOT) ? 1 : 0;
  a.q_present = (k > 0) && (q != nullptr || a.q_onehot);
  a.R = (k + 1) + ((a.q_present && !a.q_onehot) ? k : 0);
  a.logits = logits ? 1 : 0;
  a.greedy = (logits && temperature == 0.f) ? 1 : 0;
  a.decide_only = (flags & SPECB200_ACCEPT_DECIDE_ONLY) ? 1 : 0;
  a.q_step_major = (flags & SPECB200_ACCEPT_Q_STEP_MAJOR) ? 1 : 0;
  a.temperature = temperature;
  a.n_accepted = n_accepted;
  a.next_token = next_token;
  a.status = status;
  char* ws = static_cast<char*>(workspace);
  a.counters = reinterpret_cast<int*>(ws + 256);
  a.stats = reinterpret_cast<RowStat*>(ws + 256 + ((static_cast<size_t>(B) * sizeof(int) + 255) / 256) * 256);
  if (reinterpret_cast<char*>(a.stats + static_cast<size_t>(B) * a.R) > ws + workspace_bytes)
    return specb200_set_error(SPECB200_ERR_WORKSPACE, "accept: workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (status) cudaMemsetAsync(status, 0, sizeof(int32_t), s);
  // The ticket counters sit where a call with another B may have left statistics: clear them.
  cudaMemsetAsync(a.counters, 0, static_cast<size_t>(B) * sizeof(int), s);
  accept_kernel<<<static_cast<unsigned>(a.R) * B, kAcceptThreads, 0, s>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return specb200_set_error(SPECB200_ERR_CUDA, cudaGetErrorString(e));
  return SPECB200_OK;
}

extern "C" int specb200_probabilities(const float* logits, int rows, int V, float temperature, float* out, void* stream) {
  if (rows <= 0 || V <= 0 || !logits || !out || !(temperature >= 0.f))
    return specb200_set_error(SPECB200_ERR_ARG, "probabilities: bad arguments");
  probabilities_kernel<<<rows, kAcceptThreads, 0, static_cast<cudaStream_t>(stream)>>>(logits, V, temperature, out);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return specb200_set_error(SPECB200_ERR_CUDA, cudaGetErrorString(e));
  return SPECB200_OK;
}

// ---------------------------------------------------------------------------------------
// Allocation-free variant of specb200_accept.
//
// Some callers cannot hand this library a workspace: a serving runtime that reserves all of
// HBM for weights and KV pages at start-up and treats any later cudaMalloc as an error, or a
// plugin host whose operator interface passes only input and output buffers. For them the
// accept kernel's scratch (one ticket counter per row and the per-row statistics) lives in
// g_accept_scratch, a file-scope device array of fixed size that every GPU loading this
// library holds until the process exits. Limits: B <= kNoAllocMaxB rows and k <= 15.
//
// Host code cannot use g_accept_scratch as an address (on the host the name is only a
// stand-in for the device symbol), so the first call on each device, with that device
// current, looks the address up with cudaGetSymbolAddress and caches it; make that first call
// before any stream capture. All calls share the array and it keeps the last call's contents:
// the counters that must start at zero are cleared by every call, and two calls that overlap
// on the GPU (different streams, or different host threads) race on it.
// ---------------------------------------------------------------------------------------
#include <mutex>

namespace {
constexpr int kNoAllocMaxB = 512;
constexpr int kNoAllocMaxK = 15;
constexpr size_t kNoAllocCounterBytes = ((kNoAllocMaxB * sizeof(int) + 255) / 256) * 256;
constexpr size_t kNoAllocScratchBytes =
    kNoAllocCounterBytes + static_cast<size_t>(kNoAllocMaxB) * (2 * kNoAllocMaxK + 1) * sizeof(RowStat);

static __device__ __align__(256) unsigned char g_accept_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_accept_scratch on the current device, looked up once per device.
int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return specb200_set_error(SPECB200_ERR_CUDA, cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return specb200_set_error(SPECB200_ERR_ARG, "accept_noalloc: device index too large");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_accept_scratch);
    if (e != cudaSuccess || !p) return specb200_set_error(SPECB200_ERR_CUDA, "accept_noalloc: cudaGetSymbolAddress failed");
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return SPECB200_OK;
}
}  // namespace

extern "C" size_t specb200_accept_noalloc_max_rows(void) { return kNoAllocMaxB; }

extern "C" int specb200_accept_noalloc(const float* p, const float* q, const int64_t* draft, const float* u_accept,
                                       const float* u_residual, int B, int k, int V, int flags, float temperature,
                                       int64_t* n_accepted, int64_t* next_token, int32_t* status, void* stream) {
  if (B <= 0 || k < 0 || V <= 0 || V > kMaxSegs * kSeg)
    return specb200_set_error(SPECB200_ERR_ARG, "accept_noalloc: bad B/k/V (V <= 524288)");
  if (B > kNoAllocMaxB || k > kNoAllocMaxK)
    return specb200_set_error(SPECB200_ERR_ARG,
                              "accept_noalloc: B must be <= 512 and k <= 15 (fixed device scratch); "
                              "use specb200_accept with a caller workspace for larger batches");
  if (!p || !n_accepted || !u_residual) return specb200_set_error(SPECB200_ERR_ARG, "accept_noalloc: null pointer");
  if (k > 0 && (!draft || !u_accept)) return specb200_set_error(SPECB200_ERR_ARG, "accept_noalloc: null draft/u_accept");
  if (!(flags & SPECB200_ACCEPT_DECIDE_ONLY) && !next_token)
    return specb200_set_error(SPECB200_ERR_ARG, "accept_noalloc: null next_token");
  const bool logits = flags & SPECB200_ACCEPT_LOGITS;
  if (logits && !(temperature >= 0.f)) return specb200_set_error(SPECB200_ERR_ARG, "accept_noalloc: temperature < 0");
  void* scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc != SPECB200_OK) return rc;
  AcceptArgs a;
  a.p = p;
  a.q = q;
  a.draft = draft;
  a.u_accept = u_accept;
  a.u_residual = u_residual;
  a.B = B;
  a.k = k;
  a.V = V;
  a.q_onehot = (flags & SPECB200_ACCEPT_Q_ONEHOT) ? 1 : 0;
  a.q_present = (k > 0) && (q != nullptr || a.q_onehot);
  a.R = (k + 1) + ((a.q_present && !a.q_onehot) ? k : 0);
  a.logits = logits ? 1 : 0;
  a.greedy = (logits && temperature == 0.f) ? 1 : 0;
  a.decide_only = (flags & SPECB200_ACCEPT_DECIDE_ONLY) ? 1 : 0;
  a.q_step_major = (flags & SPECB200_ACCEPT_Q_STEP_MAJOR) ? 1 : 0;
  a.temperature = temperature;
  a.n_accepted = n_accepted;
  a.next_token = next_token;
  a.status = status;
  a.counters = static_cast<int*>(scratch);
  a.stats = reinterpret_cast<RowStat*>(static_cast<char*>(scratch) + kNoAllocCounterBytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (status) cudaMemsetAsync(status, 0, sizeof(int32_t), s);
  cudaMemsetAsync(a.counters, 0, static_cast<size_t>(B) * sizeof(int), s);  // the array keeps old tickets
  accept_kernel<<<static_cast<unsigned>(a.R) * B, kAcceptThreads, 0, s>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return specb200_set_error(SPECB200_ERR_CUDA, cudaGetErrorString(e));
  return SPECB200_OK;
}
