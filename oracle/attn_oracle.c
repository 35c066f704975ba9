/*
 * TEST INFRASTRUCTURE -- CPU oracle for the attention forward path.
 * Used only by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * reference legs as the checker; never by the product path.
 *
 * Restatement of the reference's CPU attention, `cpu_attn_forward` in
 * src/tests/attn_test.cpp:10-49 of JoursBleu/rocm_attn: for every query row,
 * (1) scores s_j = (q . k_j) * scale and their max, (2) the denominator
 * sum_j exp(s_j - max), (3) out_d = sum_j exp(s_j - max) / denom * v_jd.
 * Extended to the kernel contract of src/attn_kernel.h:9-20 and
 * src/attn_kernel_torch.cu: Skv != Sq (attn_kernel_torch.cu:28 via
 * attn_torch.cpp:28), causal masking of key j > query i
 * (attn_kernel_torch.cu:54), an explicit scale (the reference hard-wires
 * rsqrt(D), attn_kernel_torch.cu:49), and an empty denominator giving 0
 * (attn_kernel_torch.cu:335-336).  Products and sums accumulate in double.
 */
#include <math.h>
#include <stddef.h>
#include <stdlib.h>

#if defined(__GNUC__)
#define ORACLE_API __attribute__((visibility("default")))
#else
#define ORACLE_API
#endif

/* q [B,H,Sq,D], k/v [B,H,Skv,D], out [B,H,Sq,D], all fp32 row-major.
 * scale <= 0 selects 1/sqrt(D).  rows [row_begin, row_end) of the flattened
 * (B*H*Sq) query rows are computed, so callers can split work. */
ORACLE_API void attn_oracle_rows(const float* q, const float* k, const float* v, float* out, int B, int H,
                                 int Sq, int Skv, int D, int causal, float scale, long long row_begin,
                                 long long row_end) {
  const double sc = scale > 0.f ? (double)scale : 1.0 / sqrt((double)D);
  const long long total = (long long)B * H * Sq;
  double* scores = (double*)malloc(sizeof(double) * (size_t)(Skv > 0 ? Skv : 1));
  if (!scores) return;
  if (row_end > total) row_end = total;
  for (long long r = row_begin; r < row_end; ++r) {
    const long long bh = r / Sq;
    const int s = (int)(r % Sq);
    const float* qr = q + r * D;
    const float* kb = k + bh * (long long)Skv * D;
    const float* vb = v + bh * (long long)Skv * D;
    float* orow = out + r * D;
    double mx = -INFINITY;
    int any = 0;
    for (int j = 0; j < Skv; ++j) {
      if (causal && j > s) { scores[j] = -INFINITY; continue; }
      double acc = 0.0;
      for (int d = 0; d < D; ++d) acc += (double)qr[d] * (double)kb[(long long)j * D + d];
      scores[j] = acc * sc;
      if (scores[j] > mx) mx = scores[j];
      any = 1;
    }
    if (!any) {
      for (int d = 0; d < D; ++d) orow[d] = 0.f;
      continue;
    }
    double denom = 0.0;
    for (int j = 0; j < Skv; ++j) {
      const double w = (scores[j] == -INFINITY) ? 0.0 : exp(scores[j] - mx);
      scores[j] = w;
      denom += w;
    }
    for (int d = 0; d < D; ++d) {
      double acc = 0.0;
      for (int j = 0; j < Skv; ++j) acc += scores[j] * (double)vb[(long long)j * D + d];
      orow[d] = (float)(acc / denom);
    }
  }
  free(scores);
}

ORACLE_API void attn_oracle_forward(const float* q, const float* k, const float* v, float* out, int B, int H,
                                    int Sq, int Skv, int D, int causal, float scale) {
  attn_oracle_rows(q, k, v, out, B, H, Sq, Skv, D, causal, scale, 0, (long long)B * H * Sq);
}
