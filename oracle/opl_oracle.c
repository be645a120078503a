/* CPU oracle for the operator library -- TEST INFRASTRUCTURE ONLY.
 *
 * Plain-C restatement of the reference project's CPU verification loops, used
 * by tests/ (as the checker), by __graft_entry__.smoke() and by bench.py's
 * cpu_baseline / --impl reference legs.  Nothing in the shipped library
 * calls, links or loads this file.
 *
 * Each function names the reference loop it restates.  Pinned against the
 * reference's own loops compiled from its sources (oracle/_ref, built by
 * oracle/build_oracle.py) and against the committed fixtures in tests/golden/.
 */
#include <float.h>
#include <math.h>
#include <stddef.h>
#include <stdint.h>

/* reduce/reduce_v3.cu:125-128 -- std::accumulate(..., 0.0): sequential double
 * sum in index order, returned as double (the reference then casts to float). */
double oracle_reduce_sum(const float* x, size_t n) {
  double s = 0.0;
  for (size_t i = 0; i < n; ++i) s += (double)x[i];
  return s;
}

/* softmax/softmax_v4.cu:253-268 -- float row max; double sum of
 * exp((double)(x - max)) where x - max is a float subtraction; output
 * (float)(exp(...) / sum). */
void oracle_softmax(const float* in, float* out, int rows, int cols) {
  for (int r = 0; r < rows; ++r) {
    const float* x = in + (size_t)r * cols;
    float* y = out + (size_t)r * cols;
    float m = -FLT_MAX;
    for (int c = 0; c < cols; ++c) m = x[c] > m ? x[c] : m;
    double s = 0.0;
    for (int c = 0; c < cols; ++c) s += exp((double)(x[c] - m));
    for (int c = 0; c < cols; ++c) y[c] = (float)(exp((double)(x[c] - m)) / s);
  }
}

/* transpose/transpose_v2.cu:104-113 -- out[c * rows + r] = in[r * cols + c]. */
void oracle_transpose(const float* in, float* out, int rows, int cols) {
  for (int r = 0; r < rows; ++r)
    for (int c = 0; c < cols; ++c)
      out[(size_t)c * rows + r] = in[(size_t)r * cols + c];
}

/* rmsnorm/rmsnorm_v3.cu:154-172 -- double sum of squares, inverse_rms =
 * 1 / sqrt(sum / hidden + (double)eps), y = (float)(x * inverse_rms * w)
 * evaluated in double. */
void oracle_rmsnorm(const float* in, const float* w, float* out, int tokens,
                    int hidden, float eps) {
  for (int t = 0; t < tokens; ++t) {
    const float* x = in + (size_t)t * hidden;
    float* y = out + (size_t)t * hidden;
    double sq = 0.0;
    for (int c = 0; c < hidden; ++c) sq += (double)x[c] * (double)x[c];
    const double inv = 1.0 / sqrt(sq / hidden + (double)eps);
    for (int c = 0; c < hidden; ++c) y[c] = (float)((double)x[c] * inv * (double)w[c]);
  }
}

/* attention/attention_common.h:123-156 (same loop as the reference's
 * tests/attention_smoke.cu:31-66) -- per (head, row): double scores
 * dot(q, k) * (1 / sqrt(d)), causal rows see keys 0..row, double max, exp,
 * denominator, then out = (float)(sum_j p_j v_j / denominator).
 * heads = batch * heads; tensors are contiguous [heads, s, d]. */
static void attention_row(const float* q, const float* k, const float* v,
                          float* out_row, int s, int d, int causal, int row,
                          double* scores) {
  const double scale = 1.0 / sqrt((double)d);
  const int visible = causal ? row + 1 : s;
  double m = -INFINITY;
  for (int col = 0; col < visible; ++col) {
    double dot = 0.0;
    for (int x = 0; x < d; ++x)
      dot += (double)q[(size_t)row * d + x] * k[(size_t)col * d + x];
    scores[col] = dot * scale;
    if (scores[col] > m) m = scores[col];
  }
  double den = 0.0;
  for (int col = 0; col < visible; ++col) {
    scores[col] = exp(scores[col] - m);
    den += scores[col];
  }
  for (int x = 0; x < d; ++x) {
    double acc = 0.0;
    for (int col = 0; col < visible; ++col)
      acc += scores[col] * v[(size_t)col * d + x];
    out_row[x] = (float)(acc / den);
  }
  (void)s;
}

void oracle_attention(const float* q, const float* k, const float* v,
                      float* out, int heads, int s, int d, int causal,
                      double* scores /* scratch of s doubles */) {
  for (int h = 0; h < heads; ++h) {
    const size_t base = (size_t)h * s * d;
    for (int row = 0; row < s; ++row)
      attention_row(q + base, k + base, v + base, out + base + (size_t)row * d, s,
                    d, causal, row, scores);
  }
}

/* The same per-row computation for selected query rows of ONE head
 * ([s, d] q/k/v): out[i] is the output row of query rows[i].  Lets callers
 * check sampled rows of heads too long for a full CPU pass. */
void oracle_attention_rows(const float* q, const float* k, const float* v,
                           float* out, int s, int d, int causal,
                           const int* rows, int nrows, double* scores) {
  for (int i = 0; i < nrows; ++i)
    attention_row(q, k, v, out + (size_t)i * d, s, d, causal, rows[i], scores);
}

/* GEMM: the reference's oracle is cuBLAS (gemm/gemm_common.h:80-86,153-160;
 * gemm/gemm_v8.cu:355-362), with no CPU loop.  Restated as the exact
 * mathematical product in double: C[i][j] = sum_p A[i][p] * B[p][j], rows
 * [row_begin, row_end) only so callers can sample or split rows. */
void oracle_gemm_rows(const float* a, const float* b, double* c, int m, int n,
                      int k, int row_begin, int row_end) {
  (void)m;
  for (int i = row_begin; i < row_end; ++i) {
    double* crow = c + (size_t)(i - row_begin) * n;
    for (int j = 0; j < n; ++j) crow[j] = 0.0;
    for (int p = 0; p < k; ++p) {
      const double av = a[(size_t)i * k + p];
      const float* brow = b + (size_t)p * n;
      for (int j = 0; j < n; ++j) crow[j] += av * (double)brow[j];
    }
  }
}

/* IEEE binary16 -> float (round-trip helper for FP16 inputs: the reference
 * quantises FP16 test inputs before its CPU loop,
 * attention/attention_fp16_common.h:15-22). */
float oracle_half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  const uint32_t exp = (h >> 10) & 0x1f;
  const uint32_t man = h & 0x3ff;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: value = man * 2^-24 */
      float f = (float)man * 5.9604644775390625e-8f;
      union { float f; uint32_t u; } cv = {f};
      bits = sign | cv.u;
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112) << 23) | (man << 13);
  }
  union { uint32_t u; float f; } out = {bits};
  return out.f;
}
