// K8/K10: fused probabilities + accept-reject + residual sampling (two launches).
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
// Two launches, the second chained with programmatic dependent launch:
//   accept_kernel: one CTA per statistics unit -- a whole input row (R = k+1 target rows, plus
//     k draft rows when q is a real tensor) when rows are many, else a column chunk of one --
//     streamed once from HBM with 128-bit loads: the softmax statistics (max and sum of exp),
//     the first argmax and, in the unit holding the drafted token, the value there. The last
//     chunk of a row (ticket) combines the chunks; the last row of a sequence (ticket) makes the
//     accept decisions: n, and for greedy rows the next token; sampling rows leave a 32-byte
//     record (n, the drafted token, the statistics of target and draft row n) for:
//   residual_kernel (sampling only): one CTA per chunk of the residual row max(0, p_n - q_n) of
//     each sequence (16 of 3072 elements at V = 49,152), each warp summing a 384-element
//     sub-chunk of it (and of p) in double; the sequence's last chunk (ticket) finds the
//     sub-chunk holding the crossing from those sums with a warp scan and scans its elements
//     with the same warp.
// Every word a call writes into the workspace is back to zero when its kernels end (tickets by
// their last arriver, partial and row statistics, decision records and sums once read), so one
// zero-filled workspace serves calls of any (B, k) with no clearing in between. Decisions
// therefore cost one HBM pass over p and q.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace specb200 {
namespace {

constexpr int kAcceptThreads = 256;
constexpr int kAcceptWarps = kAcceptThreads / 32;
constexpr int kStatCtas = 4 * 148;  // statistics CTAs aimed for when rows are few (one wave at 4 per SM)

struct RowStat {
  float m;     // max of z = x / T (logit rows)
  float s;     // sum of exp(z - m)
  float zx;    // z (logit rows) or probability (probability rows) at the drafted token
  int amax;    // first index of the maximum (greedy rows)
};

// Published by the decisions of a sampling sequence for its residual units (one 32-byte load):
// the accepted length n, the drafted token at n (-1 at the bonus row) and the softmax
// statistics of target row n and draft row n.
struct __align__(16) ResDesc {
  int n, dn;
  float p_m, p_s, q_m, q_s;
  int pad[2];
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
  int* row_tickets;    // [B, R]: chunks of the row done
  int* seq_tickets;    // [B]: rows of the sequence done
  int* res_tickets;    // [B]: residual chunks of the sequence done
  RowStat* stats;      // [B, R]
  RowStat* cstats;     // [B, R, nrc]: chunk statistics of chunked rows
  ResDesc* desc;       // [B]: what the residual units of b need from its decisions
  double* chunk_sums;  // [B, C, 8, 2]: residual and p sums of each residual sub-chunk (one per warp)
  int nrc, rclen;      // statistics chunks per row and their length (a multiple of 4)
  int C, chunk;        // residual chunks per sequence and their length (a multiple of 1024)
};

// Statistics units: whole rows when there are at least half as many rows as kStatCtas (config
// 3: 576 rows, one wave at 4 CTAs per SM); fewer rows are cut into column chunks of at least
// 2048 elements, about kStatCtas units in all (the draft sampler: one row in 24 chunks), at
// most kMaxStatParts partials. Probability rows need one load at the drafted token.
constexpr int kStatChunkMin = 2048;
constexpr int kMaxStatParts = 8192;
inline void stat_chunks(int rows, int V, bool logits, int* nrc, int* len) {
  int n = 1;
  if (logits && 2 * rows < kStatCtas) {
    n = (kStatCtas + rows - 1) / rows;
    const int by_len = V / kStatChunkMin;
    n = n < by_len ? n : by_len;
    if (n * rows > kMaxStatParts) n = kMaxStatParts / rows;
    n = n < 1 ? 1 : n;
  }
  const int l = n == 1 ? V : ((V + n - 1) / n + 3) / 4 * 4;
  *nrc = (V + l - 1) / l;
  *len = l;
}
// Residual chunks: at most 16 per sequence, at least 3072 elements (12 per thread: 8 warp
// sub-chunks of 384), 16 per sequence at V = 49,152.
constexpr int kResChunks = 16;
inline void residual_chunks(int V, int B, int* C, int* len) {
  (void)B;
  int c = (V + 3071) / 3072;
  c = c < kResChunks ? c : kResChunks;
  *len = ((V + c - 1) / c + 1023) / 1024 * 1024;
  *C = (V + *len - 1) / *len;
}

// Workspace carve, shared by the caller-workspace and the allocation-free entry points.
struct AcceptLayout {
  size_t row_tickets, seq_tickets, res_tickets, stats, cstats, desc, sums, total;
};
constexpr AcceptLayout accept_layout(int B, int k) {
  auto al = [](size_t x) { return (x + 255) / 256 * 256; };
  const size_t R = 2 * static_cast<size_t>(k) + 1;
  AcceptLayout l{};
  l.row_tickets = 0;
  l.seq_tickets = l.row_tickets + al(static_cast<size_t>(B) * R * sizeof(int));
  l.res_tickets = l.seq_tickets + al(static_cast<size_t>(B) * sizeof(int));
  l.stats = l.res_tickets + al(static_cast<size_t>(B) * sizeof(int));
  l.cstats = l.stats + al(static_cast<size_t>(B) * R * sizeof(RowStat));
  l.desc = l.cstats + al(static_cast<size_t>(kMaxStatParts) * sizeof(RowStat));
  l.sums = l.desc + al(static_cast<size_t>(B) * sizeof(ResDesc));
  l.total = l.sums + al(static_cast<size_t>(B) * kResChunks * 8 * 2 * sizeof(double));
  return l;
}

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

// Statistics of row r of sequence b over columns [x0, x1) (x0 % 4 == 0); thread 0 writes them
// to *out: max and sum of exp of z = x / T, the first argmax (greedy rows), and z at the
// drafted token when it lies in [x0, x1). Every thread of the CTA calls it.
__device__ void chunk_statistics(const AcceptArgs& a, int b, int r, int x0, int x1, RowStat* out) {
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
      if (d >= x0 && d < x1) st.zx = row[d];
      *out = st;
    }
    return;
  }
  if (a.greedy) {
    // First maximum (torch.argmax): per group of 4 values take the group's max; only a group
    // that can win (or holds a NaN) goes through the exact tie / NaN merge.
    float best = -INFINITY;
    int bi = 0x7fffffff;
    if (vec) {
      const float4* r4 = reinterpret_cast<const float4*>(row);
      const int n4 = x1 / 4;
      constexpr int kU = 8;  // the loads of 8 float4 per thread in flight together, then merged in order
      for (int j0 = x0 / 4 + tid; j0 < n4; j0 += kU * kAcceptThreads) {
        float4 v[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int j = j0 + u * kAcceptThreads;
          v[u] = j < n4 ? __ldg(r4 + j) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int j = j0 + u * kAcceptThreads;
          const float gm = fmaxf(fmaxf(v[u].x, v[u].y), fmaxf(v[u].z, v[u].w));
          const bool nan = (v[u].x != v[u].x) || (v[u].y != v[u].y) || (v[u].z != v[u].z) || (v[u].w != v[u].w);
          if (j < n4 && (gm >= best || nan || best != best)) {
            argmax_merge(best, bi, v[u].x, 4 * j);
            argmax_merge(best, bi, v[u].y, 4 * j + 1);
            argmax_merge(best, bi, v[u].z, 4 * j + 2);
            argmax_merge(best, bi, v[u].w, 4 * j + 3);
          }
        }
      }
    } else {
      for (int j = x0 + tid; j < x1; j += kAcceptThreads) argmax_merge(best, bi, __ldg(row + j), j);
    }
    warp_argmax(best, bi);
    if (lane == 0) { sh_m[warp] = best; sh_i[warp] = bi; }
    __syncthreads();
    if (tid == 0) {
      for (int w = 1; w < kAcceptWarps; ++w) argmax_merge(best, bi, sh_m[w], sh_i[w]);
      RowStat st{best, 1.f, 0.f, bi};  // 0x7fffffff: nothing seen (the combine turns it into 0)
      *out = st;
    }
    return;
  }
  // softmax statistics of z = x / T, online per thread: groups of kU float4 whose loads are all
  // in flight together, one rescale per group; at T == 1 the division is skipped (x / 1 is
  // exact). The per-element exponentials of these sums use the fast intrinsic (the decisions
  // use expf on the few values they need).
  const float T = a.temperature;
  const bool unit_t = (T == 1.f);
  float m = -INFINITY, s = 0.f;
  if (vec) {
    const float4* r4 = reinterpret_cast<const float4*>(row);
    const int n4 = x1 / 4;
    constexpr int kU = 8;  // 8 float4 per thread in flight: 32 KB per CTA, 128 KB per SM
    for (int j0 = x0 / 4 + tid; j0 < n4; j0 += kU * kAcceptThreads) {
      float z[kU * 4];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int j = j0 + u * kAcceptThreads;
        const float4 v = j < n4 ? __ldg(r4 + j) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        z[4 * u] = v.x; z[4 * u + 1] = v.y; z[4 * u + 2] = v.z; z[4 * u + 3] = v.w;
      }
      float mx = m;
#pragma unroll
      for (int i = 0; i < kU * 4; ++i) {
        if (!unit_t) z[i] = z[i] / T;
        mx = fmaxf(mx, z[i]);
      }
      if (mx != -INFINITY) {
        float acc = s * __expf(m - mx);
#pragma unroll
        for (int i = 0; i < kU * 4; ++i) acc += __expf(z[i] - mx);
        s = acc;
        m = mx;
      }
    }
  } else {
    for (int j = x0 + tid; j < x1; j += kAcceptThreads) {
      float z = __ldg(row + j);
      if (!unit_t) z = z / T;
      float mx = fmaxf(z, m);
      if (mx != -INFINITY) {
        s = s * __expf(m - mx) + __expf(z - mx);
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
    if (d >= x0 && d < x1) st.zx = row[d] / T;
    *out = st;
  }
}

// Residual sampling at row n: r = max(0, p_n - q_n); sample by inverse CDF with u. Elements
// go in groups of 4 (x % 4 == 0): res_load fetches a group's p and q words, res_values turns
// them into residual values (or p when use_p), 0 past V.
constexpr int kSeg = 128;
constexpr int kMaxSegs = 4096;  // V <= kMaxSegs * kSeg = 524288 (argument check)

// The residual row of sequence b at its accepted length n: row pointers, statistics and the
// q form of row n.
struct ResidualRow {
  const float* prow;
  const float* qrow;
  RowStat ps, qs;
  float p_inv, q_inv;
  bool q_row, q_hot;
  int64_t dn;
};
__device__ ResidualRow residual_row(const AcceptArgs& a, int b, const ResDesc& d) {
  ResidualRow r;
  const int n = d.n;
  r.prow = row_ptr(a, b, n);
  r.ps = RowStat{d.p_m, d.p_s, 0.f, 0};
  r.p_inv = 1.0f / r.ps.s;
  const bool bonus = n >= a.k;  // the bonus row uses q = 0
  r.q_row = a.q_present && !a.q_onehot && !bonus;
  r.q_hot = a.q_present && a.q_onehot && !bonus;
  r.dn = d.dn;
  r.qrow = r.q_row ? row_ptr(a, b, a.k + 1 + n) : nullptr;
  r.qs = RowStat{r.q_row ? d.q_m : 0.f, r.q_row ? d.q_s : 1.f, 0.f, 0};
  r.q_inv = 1.0f / r.qs.s;
  return r;
}

SPECB200_DEVINL ResDesc load_desc(const ResDesc* p) {
  ResDesc d;
  const int4 lo = __ldcg(reinterpret_cast<const int4*>(p));
  d.n = lo.x;
  d.dn = lo.y;
  d.p_m = __int_as_float(lo.z);
  d.p_s = __int_as_float(lo.w);
  const int4 hi = __ldcg(reinterpret_cast<const int4*>(p) + 1);
  d.q_m = __int_as_float(hi.x);
  d.q_s = __int_as_float(hi.y);
  return d;
}

SPECB200_DEVINL void res_load(const AcceptArgs& a, const ResidualRow& r, int x, float4& pv, float4& qv) {
  pv = qv = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
  if (x >= a.V) return;
  if (x + 3 < a.V && a.V % 4 == 0) {
    pv = *reinterpret_cast<const float4*>(r.prow + x);
    if (r.q_row) qv = *reinterpret_cast<const float4*>(r.qrow + x);
  } else {
    float* pp = &pv.x;
    float* qq = &qv.x;
    for (int j = 0; j < 4 && x + j < a.V; ++j) {
      pp[j] = r.prow[x + j];
      if (r.q_row) qq[j] = r.qrow[x + j];
    }
  }
}

// probabilities (lm/sampling.py:13-18) of the loaded words, then torch.clamp(p - q, min=0)
// (spec/accept.py:18-26) into v (p itself with use_p); p into w as well.
SPECB200_DEVINL void res_values(const AcceptArgs& a, const ResidualRow& r, int use_p, int x, const float4& pv,
                                const float4& qv, float (&v)[4], float (&w)[4]) {
  const float* pp = &pv.x;
  const float* qq = &qv.x;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (x + j >= a.V) { v[j] = w[j] = 0.f; continue; }
    float px = pp[j];
    if (a.logits) px = __expf((a.temperature == 1.f ? px : px / a.temperature) - r.ps.m) * r.p_inv;
    w[j] = px;
    if (use_p) { v[j] = px; continue; }
    float qx = 0.f;
    if (r.q_row) {
      qx = qq[j];
      if (a.logits) qx = __expf((a.temperature == 1.f ? qx : qx / a.temperature) - r.qs.m) * r.q_inv;
    } else if (r.q_hot) {
      qx = (x + j == r.dn) ? 1.f : 0.f;
    }
    v[j] = fmaxf(px - qx, 0.f);
  }
}

// A residual chunk is 8 sub-chunks of sub = chunk / 8 elements (a multiple of 128), one per
// warp; lane l of a warp takes elements sub_start + 128 i + 4 l .. + 3 for i = 0, 1, ... (the
// element order is i, then lane, then j). Per warp: the double sums of the residual and of p
// over its sub-chunk, loads of kResBatch steps in flight together.
constexpr int kResBatch = 3;  // a 384-element sub-chunk (3 steps) in one round trip
SPECB200_DEVINL void res_warp_sums(const AcceptArgs& a, const ResidualRow& r, int sub_start, int sub, double& res,
                                   double& pr) {
  const int lane = threadIdx.x & 31;
  const int steps = sub / 128;
  double acc = 0.0, accp = 0.0;
  for (int i0 = 0; i0 < steps; i0 += kResBatch) {
    float4 pv[kResBatch], qv[kResBatch];
#pragma unroll
    for (int i = 0; i < kResBatch; ++i)
      if (i0 + i < steps) res_load(a, r, sub_start + 128 * (i0 + i) + 4 * lane, pv[i], qv[i]);
    float bs = 0.f, bp = 0.f;  // the batch's at most 4 kResBatch values per lane in fp32, then one double add
#pragma unroll
    for (int i = 0; i < kResBatch; ++i) {
      if (i0 + i >= steps) break;
      const int x = sub_start + 128 * (i0 + i) + 4 * lane;
      float v[4], w[4];
      res_values(a, r, 0, x, pv[i], qv[i], v, w);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        bs += v[j];
        bp += w[j];
      }
    }
    acc += static_cast<double>(bs);
    accp += static_cast<double>(bp);
  }
  res = warp_sum_d(acc);
  pr = warp_sum_d(accp);
}

// First element x of sub-chunk [sub_start, sub_start + sub) where base + the running sum (in
// element order) passes target, or -1 with base advanced past the sub-chunk. One warp.
SPECB200_DEVINL int res_warp_find(const AcceptArgs& a, const ResidualRow& r, int use_p, int sub_start, int sub,
                                  double& base, double target) {
  const int lane = threadIdx.x & 31;
  const int steps = sub / 128;
  for (int i0 = 0; i0 < steps; i0 += kResBatch) {
    float4 pv[kResBatch], qv[kResBatch];
#pragma unroll
    for (int i = 0; i < kResBatch; ++i)  // the loads of the batch first, all in flight together
      if (i0 + i < steps) res_load(a, r, sub_start + 128 * (i0 + i) + 4 * lane, pv[i], qv[i]);
#pragma unroll
    for (int i = 0; i < kResBatch; ++i) {
      if (i0 + i >= steps) break;
      const int x = sub_start + 128 * (i0 + i) + 4 * lane;
      float v[4], w[4];
      res_values(a, r, use_p, x, pv[i], qv[i], v, w);
      const double mine = static_cast<double>(v[0]) + v[1] + v[2] + v[3];
      double incl = mine;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const double t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      const unsigned hit = __ballot_sync(0xffffffffu, base + incl > target);
      if (hit) {
        const int first = __ffs(hit) - 1;
        int found = -1;
        if (lane == first) {
          double c = base + incl - mine;  // running sum before this lane's four
          for (int j = 0; j < 4; ++j) {
            c += v[j];
            if (c > target) {
              found = x + j;
              break;
            }
          }
          if (found < 0) found = min(x + 3, a.V - 1);  // the lane's total passed it: its last element
        }
        return __shfl_sync(0xffffffffu, found, first);
      }
      base += __shfl_sync(0xffffffffu, incl, 31);
    }
  }
  return -1;
}

// Decisions for sequence b once all its row statistics are in the workspace (the caller is
// the CTA that finished its last row): n accepted drafts, then the greedy next token, or the
// record the residual kernel reads. All threads of the CTA call it.
__device__ void decide(const AcceptArgs& a, int b) {
  __shared__ RowStat sst[32];
  __shared__ int64_t sdraft[16];
  __shared__ float su[16];
  const RowStat* st = a.stats + static_cast<int64_t>(b) * a.R;
  if (threadIdx.x >= 32 && threadIdx.x < 32 + a.k) {
    const int i = threadIdx.x - 32;
    sdraft[i] = a.draft[static_cast<int64_t>(b) * a.k + i];
    su[i] = a.u_accept[static_cast<int64_t>(b) * a.k + i];
  }
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
  const bool sampling = !a.greedy && !a.decide_only;
  // the row statistics are read: back to zero (the residual units get theirs in a descriptor)
  if (threadIdx.x < a.R) a.stats[static_cast<int64_t>(b) * a.R + threadIdx.x] = RowStat{0.f, 0.f, 0.f, 0};
  if (threadIdx.x == 0) {
    a.seq_tickets[b] = 0;  // ready for the next call
    int n = 0;
    bool run = true;
    for (int i = 0; i < a.k; ++i) {
      const int64_t d = sdraft[i];
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
      const bool acc = su[i] * qx < px;
      if (run && acc) ++n; else run = false;
    }
    a.n_accepted[b] = n;
    if (a.greedy && !a.decide_only) a.next_token[b] = sst[n].amax;
    if (sampling) {
      const bool qr = a.q_present && !a.q_onehot && n < a.k;
      ResDesc d{};
      d.n = n;
      d.dn = n < a.k ? static_cast<int>(sdraft[n]) : -1;
      d.p_m = sst[n].m;
      d.p_s = sst[n].s;
      d.q_m = qr ? sst[a.k + 1 + n].m : 0.f;
      d.q_s = qr ? sst[a.k + 1 + n].s : 1.f;
      a.desc[b] = d;
    }
  }
  __syncthreads();
}

// Statistics unit u: chunk c of row r of sequence b. The row's last chunk combines the
// chunks (warp 0: chunk order within each lane, then a fixed xor tree); the sequence's last
// row decides.
__device__ void stat_unit(const AcceptArgs& a, int u) {
  __shared__ int sh_last;
  const int c = u % a.nrc, rb = u / a.nrc;
  const int r = rb % a.R, b = rb / a.R;
  RowStat* st = a.stats + static_cast<int64_t>(b) * a.R;
  if (a.nrc == 1) {
    chunk_statistics(a, b, r, 0, a.V, st + r);
  } else {
    RowStat* part = a.cstats + static_cast<int64_t>(rb) * a.nrc;
    chunk_statistics(a, b, r, c * a.rclen, min(a.V, (c + 1) * a.rclen), part + c);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) sh_last = (atomicAdd(a.row_tickets + rb, 1) == a.nrc - 1);
    __syncthreads();
    if (!sh_last) return;
    __threadfence();
    if (threadIdx.x < 32) {
      const int lane = threadIdx.x;
      RowStat t{-INFINITY, 0.f, 0.f, 0x7fffffff};
      for (int j = lane; j < a.nrc; j += 32) {
        const float m2 = __ldcg(&part[j].m), s2 = __ldcg(&part[j].s);
        const int i2 = __ldcg(&part[j].amax);
        if (a.greedy) argmax_merge(t.m, t.amax, m2, i2);
        else combine_ms(t.m, t.s, m2, s2);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, t.m, o), s2 = __shfl_xor_sync(0xffffffffu, t.s, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, t.amax, o);
        if (a.greedy) argmax_merge(t.m, t.amax, m2, i2);
        else combine_ms(t.m, t.s, m2, s2);
      }
      if (lane == 0) {
        if (a.greedy) {
          t.s = 1.f;
          t.amax = t.amax == 0x7fffffff ? 0 : t.amax;
        } else {
          const int i = r <= a.k ? r : r - a.k - 1;
          const int64_t d = i < a.k ? a.draft[static_cast<int64_t>(b) * a.k + i] : -1;
          if (d >= 0 && d < a.V) t.zx = __ldcg(&part[d / a.rclen].zx);
        }
        st[r] = t;
        a.row_tickets[rb] = 0;
      }
      __syncwarp();
      for (int j = lane; j < a.nrc; j += 32) part[j] = RowStat{0.f, 0.f, 0.f, 0};  // read: back to zero
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) sh_last = (atomicAdd(a.seq_tickets + b, 1) == a.R - 1);
  __syncthreads();
  if (!sh_last) return;
  __threadfence();
  decide(a, b);
}

// The last residual chunk of sequence b, after every chunk of b has read them: b's chunk sums
// and decision record go back to zero. All threads of the CTA call it.
__device__ void residual_clear(const AcceptArgs& a, int b, double* sums) {
  __syncthreads();
  const int tid = threadIdx.x;
  for (int i = tid; i < 16 * a.C; i += kAcceptThreads) sums[i] = 0.0;
  if (tid == 0) a.desc[b] = ResDesc{};
}

// Grid C * B (1-D, b-major): chunk c of the residual row of sequence b. The sequence's last
// chunk draws the sample.
__global__ void __launch_bounds__(kAcceptThreads, 4) residual_kernel(AcceptArgs a) {
  __shared__ int sh_ok, sh_last;
  __shared__ ResDesc sh_desc;
  const int b = blockIdx.x / a.C, c = blockIdx.x % a.C, tid = threadIdx.x;
  pdl_wait();
  if (tid == 0) {
    // the accepted length and token index rows and the vocabulary: values out of range (a
    // workspace that was not zero-filled before its first use) are reported, never used
    const ResDesc d = load_desc(a.desc + b);
    sh_ok = 1;
    if (d.n < 0 || d.n > a.k || d.dn < -1 || d.dn >= a.V) {
      set_status(a.status, SPECB200_ERR_WORKSPACE);
      sh_ok = 0;
    }
    sh_desc = d;
  }
  __syncthreads();
  const bool ok = sh_ok;
  double* sums = a.chunk_sums + static_cast<int64_t>(b) * a.C * 16;
  const int warp = tid >> 5, lane = tid & 31, sub = a.chunk / 8;
  ResidualRow r{};
  if (ok) {
    r = residual_row(a, b, sh_desc);
    double sr, sp;
    res_warp_sums(a, r, c * a.chunk + warp * sub, sub, sr, sp);
    if (lane == 0) {
      sums[(c * 8 + warp) * 2] = sr;
      sums[(c * 8 + warp) * 2 + 1] = sp;
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) sh_last = (atomicAdd(a.res_tickets + b, 1) == a.C - 1);
  __syncthreads();
  if (!sh_last) return;
  __threadfence();
  if (tid == 0) a.res_tickets[b] = 0;  // ready for the next call
  if (!ok) {
    if (tid == 0) a.next_token[b] = a.V - 1;
    residual_clear(a, b, sums);
    return;
  }
  // The sample: the residual total over the sub-chunks in element order (p when it is zero),
  // u times it, the first sub-chunk whose running sum passes that, then its elements (later
  // sub-chunks too, if rounding put the crossing past its end); past the end: V - 1
  // (searchsorted(right=True), clamped).
  __shared__ double sh_sub[2 * 8 * kResChunks];
  for (int i = tid; i < 16 * a.C; i += kAcceptThreads) sh_sub[i] = __ldcg(sums + i);
  __syncthreads();
  if (warp == 0) {
    // lane l holds sub-chunks 4 l .. 4 l + 3 (at most 128 = 8 x kResChunks); the total, the
    // choice of residual or p, the target and the crossing sub-chunk by a warp scan
    const int S = 8 * a.C;
    double rs[4], ps[4], lr = 0.0, lp = 0.0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = 4 * lane + j;
      rs[j] = i < S ? sh_sub[2 * i] : 0.0;
      ps[j] = i < S ? sh_sub[2 * i + 1] : 0.0;
      lr += rs[j];
      lp += ps[j];
    }
    const double total_r = warp_sum_d(lr);
    const int use_p = !(total_r > 0.0);  // residual sums to 0: residual_distribution falls back to p
    const double total = use_p ? warp_sum_d(lp) : total_r;
    const double target = static_cast<double>(a.u_residual[b]) * total;
    const double mine = use_p ? lp : lr;
    double incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    const unsigned hit = __ballot_sync(0xffffffffu, incl > target);
    int first = S;
    double base = 0.0;
    if (hit) {  // warp-uniform: every lane computes the same first / base
      const int hl = __ffs(hit) - 1;
      double c = __shfl_sync(0xffffffffu, incl - mine, hl);  // running sum before lane hl's four
      bool found = false;
      first = 4 * hl + 3;  // lane hl's total passed the target: its last sub-chunk at the latest
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        const double v = __shfl_sync(0xffffffffu, use_p ? ps[j] : rs[j], hl);
        if (!found) {
          if (c + v > target) {
            first = 4 * hl + j;
            found = true;
          } else {
            c += v;
          }
        }
      }
      base = c;
    }
    int64_t tok = a.V - 1;
    for (int i = first; i < S; ++i) {
      const int x = res_warp_find(a, r, use_p, (i / 8) * a.chunk + (i % 8) * sub, sub, base, target);
      if (x >= 0) {
        tok = x;
        break;
      }
    }
    if (lane == 0) a.next_token[b] = tok;
  }
  residual_clear(a, b, sums);
}

// One CTA per statistics unit (b-major, then row, then column chunk: a sequence's CTAs run
// together). The residual kernel may start its prologue; it waits for this grid.
__global__ void __launch_bounds__(kAcceptThreads, 4) accept_kernel(AcceptArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  stat_unit(a, blockIdx.x);
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

namespace specb200 {
namespace {
// Both kernels on `s` (after clearing the caller's status word); the residual kernel follows
// with programmatic dependent launch. The workspace's tickets are zero on entry and on exit.
// Returns the first CUDA error met.
cudaError_t launch_accept(AcceptArgs& a, char* ws, const AcceptLayout& l, cudaStream_t s) {
  a.row_tickets = reinterpret_cast<int*>(ws + l.row_tickets);
  a.seq_tickets = reinterpret_cast<int*>(ws + l.seq_tickets);
  a.res_tickets = reinterpret_cast<int*>(ws + l.res_tickets);
  a.stats = reinterpret_cast<RowStat*>(ws + l.stats);
  a.cstats = reinterpret_cast<RowStat*>(ws + l.cstats);
  a.desc = reinterpret_cast<ResDesc*>(ws + l.desc);
  a.chunk_sums = reinterpret_cast<double*>(ws + l.sums);
  stat_chunks(a.B * a.R, a.V, a.logits != 0, &a.nrc, &a.rclen);
  residual_chunks(a.V, a.B, &a.C, &a.chunk);
  cudaError_t e = cudaSuccess;
  if (a.status) e = cudaMemsetAsync(a.status, 0, sizeof(int32_t), s);
  if (e != cudaSuccess) return e;
  accept_kernel<<<static_cast<unsigned>(a.B) * a.R * a.nrc, kAcceptThreads, 0, s>>>(a);
  e = cudaGetLastError();
  if (e == cudaSuccess && !a.greedy && !a.decide_only)
    e = launch_kernel(residual_kernel, dim3(static_cast<unsigned>(a.C) * a.B), dim3(kAcceptThreads), 0, s, true, a);
  return e;
}
}  // namespace
}  // namespace specb200

// Workspace of a call with B sequences and k drafts (any V the kernel accepts).
extern "C" size_t specb200_accept_workspace_bytes(int B, int k) {
  if (B <= 0 || k < 0) return 0;
  return accept_layout(B, k).total;
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
  const AcceptLayout l = accept_layout(B, k);
  if (l.total > workspace_bytes) return specb200_set_error(SPECB200_ERR_WORKSPACE, "accept: workspace too small");
  const cudaError_t e = launch_accept(a, static_cast<char*>(workspace), l, static_cast<cudaStream_t>(stream));
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
// accept kernel's scratch (the work queue, tickets and flags, the per-row statistics and the
// residual chunk sums) lives in g_accept_scratch, a file-scope device array of fixed size
// (about 600 KB) that every GPU loading this library holds until the process exits. Limits:
// B <= kNoAllocMaxB rows and k <= 15.
//
// Host code cannot use g_accept_scratch as an address (on the host the name is only a
// stand-in for the device symbol), so the first call on each device, with that device
// current, looks the address up with cudaGetSymbolAddress and caches it; make that first call
// before any stream capture. All calls share the array and it keeps the last call's contents:
// the queue, tickets and flags that must start at zero are zero when the library is loaded
// and every call leaves them at zero when its kernel ends, and two calls that overlap on the
// GPU (different streams, or different host threads) race on it.
// ---------------------------------------------------------------------------------------
#include <mutex>

namespace {
constexpr int kNoAllocMaxB = 512;
constexpr int kNoAllocMaxK = 15;
// accept_layout(kNoAllocMaxB, kNoAllocMaxK): queue, tickets, flags, statistics, the chunked-row
// partials, the accepted lengths and 16 residual chunk sums per row (~575 KB)
constexpr size_t kNoAllocScratchBytes = accept_layout(kNoAllocMaxB, kNoAllocMaxK).total;

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
  const AcceptLayout l = accept_layout(B, k);
  if (l.total > kNoAllocScratchBytes) return specb200_set_error(SPECB200_ERR_ARG, "accept_noalloc: scratch too small");
  // the array holds zero tickets and flags: every call leaves them so
  const cudaError_t e = launch_accept(a, static_cast<char*>(scratch), l, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return specb200_set_error(SPECB200_ERR_CUDA, cudaGetErrorString(e));
  return SPECB200_OK;
}
