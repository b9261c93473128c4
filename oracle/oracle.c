/* oracle.c - CPU restatement of the reference algorithms on the hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This is the checker the parity tests compare the
 * CUDA kernels against, and the CPU baseline bench.py times; nothing in the
 * product (vkcuda_b200/) calls it.
 *
 * Each function restates the host-side reference loop of a junka/vkcuda demo
 * (file:line cited), generalised from the demo's compile-time shapes to
 * runtime arguments:
 *   oracle_fa_runif / oracle_fa_gaussian / oracle_fa_inputs
 *       examples/flash_attn.vc:178-188 (LCG + Box-Muller), :202-207 (seed,
 *       Q/K/V interleaved per element)
 *   oracle_attention
 *       examples/flash_attn.vc:129-165 (referenceAttn: fp64, two passes per
 *       row, dot product recomputed in pass 2, exp2 of scale*dot - max,
 *       O = float(acc / l), causal skips j > i)
 *   oracle_gemm
 *       examples/matmul_coopmat_bench.vc:168-184 (fp64 sum over k of
 *       A[n][k]*B[k][m]) and test/wmma_gemm.vc:71-79 (D = A*B + C)
 *   oracle_vadd       test/vadd.vc:40-43 (c = a + b in fp32)
 *   oracle_sum_f64    fp64 sum of the vadd output (the streaming pair's check)
 *   oracle_block_reduce
 *       test/reduce.vc:11-38 (per-block shared-memory tree, s = block/2 ...
 *       1, slot t += slot t+s) - the device kernel's pairing order.
 * Parallel loops use OpenMP over independent rows/chunks; every per-row
 * computation runs in the reference's order, so results do not depend on the
 * thread count (the fp64 sum uses fixed chunks combined in order).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static void set_threads(int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
}

int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* One uniform in (0, 1): 32-bit LCG, 16 bits of its state (flash_attn.vc:178-181). */
double oracle_fa_runif(uint32_t *st) {
  *st = *st * 1103515245u + 12345u;
  return ((double)((*st >> 8) & 0xffffu) + 0.5) / 65536.0;
}

/* Box-Muller normal from two uniforms, rounded to float (flash_attn.vc:183-188). */
float oracle_fa_gaussian(uint32_t *st) {
  const double u1 = oracle_fa_runif(st);
  const double u2 = oracle_fa_runif(st);
  return (float)(sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2));
}

/* Demo inputs: for each element i, Q[i], K[i], V[i] drawn in that order from
 * one stream seeded with `seed` (the demo uses 12345 + causal). */
void oracle_fa_inputs(uint32_t seed, int64_t elems, float *Q, float *K, float *V) {
  uint32_t st = seed;
  for (int64_t i = 0; i < elems; ++i) {
    Q[i] = oracle_fa_gaussian(&st);
    K[i] = oracle_fa_gaussian(&st);
    V[i] = oracle_fa_gaussian(&st);
  }
}

/* One query row of referenceAttn. `scale` is the exp2-domain scale (the demo
 * passes float(log2(e)/sqrt(d))), applied in fp64 as the reference does. */
static void attention_row(const float *Q, const float *K, const float *V, float *O, int N,
                          int d, double scale, int causal, int64_t base, int i, double *acc) {
  double m = -1.0e30;
  const int jend = causal ? i + 1 : N;
  for (int j = 0; j < jend; ++j) {
    double s = 0.0;
    for (int t = 0; t < d; ++t)
      s += (double)Q[base + (int64_t)i * d + t] * (double)K[base + (int64_t)j * d + t];
    s *= scale;
    if (s > m) m = s;
  }
  double l = 0.0;
  for (int t = 0; t < d; ++t) acc[t] = 0.0;
  for (int j = 0; j < jend; ++j) {
    double s = 0.0;
    for (int t = 0; t < d; ++t)
      s += (double)Q[base + (int64_t)i * d + t] * (double)K[base + (int64_t)j * d + t];
    s *= scale;
    const double p = exp2(s - m);
    l += p;
    for (int t = 0; t < d; ++t) acc[t] += p * (double)V[base + (int64_t)j * d + t];
  }
  for (int t = 0; t < d; ++t) O[base + (int64_t)i * d + t] = (float)(acc[t] / l);
}

/* referenceAttn over slices [bh_begin, bh_end) and query rows
 * [row_begin, row_end) of each, layout [BH][N][d]. Rows outside the range
 * are left untouched (used for sampled checks and the CPU baseline). */
void oracle_attention(const float *Q, const float *K, const float *V, float *O, int BH, int N,
                      int d, float scale_log2, int causal, int bh_begin, int bh_end,
                      int row_begin, int row_end, int threads) {
  (void)BH;
  set_threads(threads);
  const int rows = row_end - row_begin;
  const int64_t total = (int64_t)(bh_end - bh_begin) * rows;
#pragma omp parallel
  {
    double acc_local[1024];
#pragma omp for schedule(dynamic, 4)
    for (int64_t w = 0; w < total; ++w) {
      const int h = bh_begin + (int)(w / rows);
      const int i = row_begin + (int)(w % rows);
      attention_row(Q, K, V, O, N, d, (double)scale_log2, causal, (int64_t)h * N * d, i,
                    acc_local);
    }
  }
}

/* D[m][n] = sum_k A[m][k] * B(k, n) (+ Cin[m][n]) in fp64 over fp32 inputs
 * (fp16/bf16 values widened exactly), rows [row_begin, row_end).
 * B(k, n) = b_kn ? B[k*ldb + n] : B[n*ldb + k]. */
void oracle_gemm(const float *A, const float *B, double *D, const float *Cin, int M, int N,
                 int K, int64_t lda, int64_t ldb, int64_t ldd, int64_t ldc, int b_kn,
                 int row_begin, int row_end, int threads) {
  (void)M;
  set_threads(threads);
#pragma omp parallel for schedule(dynamic, 1)
  for (int m = row_begin; m < row_end; ++m) {
    double *drow = D + (int64_t)m * ldd;
    for (int n = 0; n < N; ++n) drow[n] = Cin ? (double)Cin[(int64_t)m * ldc + n] : 0.0;
    const float *arow = A + (int64_t)m * lda;
    if (b_kn) {
      /* k-outer: the same per-element sum order (k ascending), row-contiguous B. */
      for (int k = 0; k < K; ++k) {
        const double a = (double)arow[k];
        const float *brow = B + (int64_t)k * ldb;
        for (int n = 0; n < N; ++n) drow[n] += a * (double)brow[n];
      }
    } else {
      for (int n = 0; n < N; ++n) {
        const float *bcol = B + (int64_t)n * ldb;
        double s = drow[n];
        for (int k = 0; k < K; ++k) s += (double)arow[k] * (double)bcol[k];
        drow[n] = s;
      }
    }
  }
}

/* c = a + b in fp32 (round-to-nearest, no contraction). */
void oracle_vadd(const float *a, const float *b, float *c, int64_t n, int threads) {
  set_threads(threads);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) c[i] = a[i] + b[i];
}

/* fp64 sum; fixed 1 Mi-element chunks combined in index order, so the result
 * is independent of the thread count. */
double oracle_sum_f64(const float *x, int64_t n, int threads) {
  set_threads(threads);
  const int64_t chunk = 1 << 20;
  const int64_t nchunks = (n + chunk - 1) / chunk;
  double total = 0.0;
  if (nchunks == 0) return 0.0;
  double partial[1024];
  /* Chunks are summed 1024 at a time (in parallel), then folded in order. */
  for (int64_t c0 = 0; c0 < nchunks; c0 += 1024) {
    const int64_t c1 = c0 + 1024 < nchunks ? c0 + 1024 : nchunks;
#pragma omp parallel for schedule(static)
    for (int64_t c = c0; c < c1; ++c) {
      const int64_t lo = c * chunk, hi = lo + chunk < n ? lo + chunk : n;
      double s = 0.0;
      for (int64_t i = lo; i < hi; ++i) s += (double)x[i];
      partial[c - c0] = s;
    }
    for (int64_t c = c0; c < c1; ++c) total += partial[c - c0];
  }
  return total;
}

/* Per-block tree sum with the reference's pairing (test/reduce.vc:11-38):
 * slots hold in[g*block + t] (0 past n); for s = block/2, block/4, ..., 1,
 * slot t < s += slot t + s; out[g] = slot 0. fp32 throughout. */
void oracle_block_reduce(const float *in, float *out, int n, int block, int groups) {
  float slots[1024];
  for (int g = 0; g < groups; ++g) {
    for (int t = 0; t < block; ++t) {
      const int64_t i = (int64_t)g * block + t;
      slots[t] = i < n ? in[i] : 0.0f;
    }
    for (int s = block / 2; s > 0; s /= 2)
      for (int t = 0; t < s; ++t) slots[t] = slots[t] + slots[t + s];
    out[g] = slots[0];
  }
}
