/* Oracle: n-gram prompt lookup, a literal C restatement of spec/ngram.py:32-45 of the
 * reference (test infrastructure only). For n = min(max_n, len-1) down to 1, scan starts
 * from len-n-1 down to 0 and take the first whose n tokens equal the last n; copy what
 * followed, reading the copy's own output once it runs past the end; with no match repeat
 * the last token. */
#include <stdint.h>

int oracle_ngram_lookup(const int32_t* ctx, int len, int k, int max_n, int64_t* out) {
  if (len <= 0) return -1;
  int nmax = max_n < len - 1 ? max_n : len - 1;
  for (int n = nmax; n >= 1; --n) {
    const int32_t* suffix = ctx + len - n;
    for (int start = len - n - 1; start >= 0; --start) {
      int eq = 1;
      for (int j = 0; j < n && eq; ++j) eq = ctx[start + j] == suffix[j];
      if (!eq) continue;
      const int32_t* src = ctx + start + n;
      int src_len = len - start - n;
      for (int i = 0; i < k; ++i) out[i] = i < src_len ? src[i] : out[i - src_len];
      return n;
    }
  }
  for (int i = 0; i < k; ++i) out[i] = ctx[len - 1];
  return 0;
}

/* B contexts, row b at ctx + b * stride with lens[b] tokens; out [B, k]. */
int oracle_ngram_batch(const int32_t* ctx, int64_t stride, const int32_t* lens, int B, int k, int max_n, int64_t* out) {
  for (int b = 0; b < B; ++b)
    if (oracle_ngram_lookup(ctx + b * stride, lens[b], k, max_n, out + (int64_t)b * k) < 0) return -1;
  return 0;
}
