/*
 * ORACLE (test infrastructure only).  Seeded synthetic topologies of the
 * benchmark networks, generated on the host with no dependency on the CUDA
 * library, so that the CPU legs (tests, bench.py's reference arm) build their
 * networks without loading it.  It restates the engine's generator draw for
 * draw: the same counter-based splitmix64 streams keyed (seed, stream id) and
 * (a, b), the same Box-Muller normal, the same weight rounding, so the edge
 * set equals the engine's exactly (tests/test_oracle_net.py checks it).
 *
 * Topologies (per the benchmark configurations; none is fixed by the
 * reference, whose simulator builds its own anatomy, neurogen/anatomy.py):
 *   Erdos-Renyi  -- each ordered pair pre != post with probability p, keyed
 *                   (pre, post); delay U{dmin..dmax}, weight keyed (pre, post).
 *   fixed fan-in -- post j draws `fanin` uniform presynaptic cells keyed
 *                   (j, k); a draw of j itself moves to (j + 1) mod n.
 *   16x16 blocks -- per block-row `blocks` distinct block-columns (Floyd's
 *                   sampling), per block `fill` distinct entries, one delay a
 *                   block keyed (block-row, block-column).
 * Weights: lognormal exp(mu + sigma z) rounded to the nearest multiple of
 * 2^-24 nS (at least 2^-24), or |sigma z| rounded to fp16 (at least the
 * smallest subnormal); negative for inhibitory presynaptic cells (Dale).  The
 * unrounded double value is also returned, for the fp64 mode of the oracle.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
  int32_t n, n_exc, topology; /* 0 Erdos-Renyi, 1 fixed fan-in, 2 16x16 blocks */
  float p_connect;
  int32_t fanin, bsr_blocks, bsr_fill;
  int32_t weight_kind; /* 0 lognormal fp32, 1 half-normal fp16 */
  float w_mu, w_sigma;
  int32_t delay_min, delay_max;
  uint64_t seed;
} ot_config;

enum { S_EDGE = 1, S_PRE, S_DELAY, S_W1, S_W2, S_BLOCK, S_FILL };

/* splitmix64 finaliser (S. Vigna, public domain). */
static uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
static uint64_t key_of(uint64_t seed, uint64_t id) { return mix64(seed ^ mix64(id)); }
static uint64_t bits(uint64_t key, uint64_t a, uint64_t b) { return mix64(((a << 32) | (b & 0xFFFFFFFFull)) ^ key); }
static double uniform(uint64_t key, uint64_t a, uint64_t b) { return (double)(bits(key, a, b) >> 11) * 0x1.0p-53; }
static uint64_t below(uint64_t key, uint64_t a, uint64_t b, uint64_t m) {
  return (uint64_t)(((unsigned __int128)bits(key, a, b) * m) >> 64);
}

typedef struct {
  const ot_config *c;
  uint64_t k1, k2;
} wdraw;

/* Signed weight keyed (a, b): fp32 value (fp16 value for fp16 weights) and the
 * unrounded double. */
static float draw_weight(const wdraw *wd, uint64_t a, uint64_t b, int inhibitory, double *exact) {
  const double u1 = (double)((bits(wd->k1, a, b) >> 11) + 1) * 0x1.0p-53; /* (0, 1] */
  const double u2 = uniform(wd->k2, a, b);
  const double z = sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
  if (wd->c->weight_kind == 0) {
    const double w = exp((double)wd->c->w_mu + (double)wd->c->w_sigma * z);
    float q = (float)(nearbyint(w * 16777216.0) * 0x1.0p-24);
    if (q == 0.f) q = 0x1.0p-24f;
    *exact = inhibitory ? -w : w;
    return inhibitory ? -q : q;
  }
  const float m = (float)fabs((double)wd->c->w_sigma * z);
  _Float16 h = (_Float16)m; /* round to nearest even */
  if ((float)h == 0.f) {
    uint16_t one = 1;
    memcpy(&h, &one, 2);
  }
  const float v = (float)h;
  *exact = inhibitory ? -(double)v : (double)v;
  return inhibitory ? -v : v;
}

/* Floyd's algorithm: m distinct values of [0, range), keyed (a, salt + j), sorted. */
static int cmp_int(const void *x, const void *y) { return *(const int *)x - *(const int *)y; }
static void floyd(uint64_t key, uint64_t a, uint64_t salt, int range, int m, int *out) {
  int k = 0;
  for (int j = range - m; j < range; ++j) {
    const int t = (int)below(key, a, salt + (uint64_t)j, (uint64_t)j + 1);
    int seen = 0;
    for (int q = 0; q < k; ++q)
      if (out[q] == t) seen = 1;
    out[k++] = seen ? j : t;
  }
  qsort(out, (size_t)m, sizeof(int), cmp_int);
}

/* Number of synapses of the configuration. */
int64_t ot_count(const ot_config *c) {
  if (c->topology == 1) return (int64_t)c->n * c->fanin;
  if (c->topology == 2) return (int64_t)(c->n / 16) * c->bsr_blocks * c->bsr_fill;
  const uint64_t ke = key_of(c->seed, S_EDGE);
  int64_t total = 0;
#pragma omp parallel for schedule(dynamic, 64) reduction(+ : total)
  for (int i = 0; i < c->n; ++i)
    for (int j = 0; j < c->n; ++j)
      if (j != i && uniform(ke, (uint64_t)i, (uint64_t)j) < (double)c->p_connect) ++total;
  return total;
}

/* Fills the ot_count(c) synapses (any order).  w64 may be NULL. */
void ot_fill(const ot_config *c, int32_t *pre, int32_t *post, int32_t *delay, float *w, double *w64) {
  const int n = c->n;
  const uint64_t dspan = (uint64_t)(c->delay_max - c->delay_min + 1);
  const uint64_t kd = key_of(c->seed, S_DELAY);
  const wdraw wd = {c, key_of(c->seed, S_W1), key_of(c->seed, S_W2)};
  if (c->topology == 1) {
    const uint64_t kp = key_of(c->seed, S_PRE);
    const int K = c->fanin;
#pragma omp parallel for schedule(static)
    for (int j = 0; j < n; ++j)
      for (int k = 0; k < K; ++k) {
        int p = (int)below(kp, (uint64_t)j, (uint64_t)k, (uint64_t)n);
        if (p == j) p = (p + 1) % n;
        const int64_t e = (int64_t)j * K + k;
        double x;
        pre[e] = p;
        post[e] = j;
        delay[e] = c->delay_min + (int)below(kd, (uint64_t)j, (uint64_t)k, dspan);
        w[e] = draw_weight(&wd, (uint64_t)j, (uint64_t)k, p >= c->n_exc, &x);
        if (w64) w64[e] = x;
      }
  } else if (c->topology == 2) {
    const int NB = n / 16, M = c->bsr_blocks, F = c->bsr_fill;
    const uint64_t kb = key_of(c->seed, S_BLOCK), kf = key_of(c->seed, S_FILL);
#pragma omp parallel
    {
      int *cols = malloc(sizeof(int) * (size_t)(M > 0 ? M : 1));
      int *pos = malloc(sizeof(int) * 256);
#pragma omp for schedule(dynamic, 16)
      for (int br = 0; br < NB; ++br) {
        floyd(kb, (uint64_t)br, 0, NB, M, cols);
        for (int m = 0; m < M; ++m) {
          const int bc = cols[m];
          const int d = c->delay_min + (int)below(kd, (uint64_t)br, (uint64_t)bc, dspan);
          floyd(kf, (uint64_t)br, (uint64_t)bc * 256, 256, F, pos);
          for (int q = 0; q < F; ++q) {
            const int r = pos[q] / 16, col = pos[q] % 16, p = bc * 16 + col;
            const int64_t e = ((int64_t)br * M + m) * F + q;
            double x;
            pre[e] = p;
            post[e] = br * 16 + r;
            delay[e] = d;
            w[e] = draw_weight(&wd, (uint64_t)br * 16 + (uint64_t)r, (uint64_t)p, p >= c->n_exc, &x);
            if (w64) w64[e] = x;
          }
        }
      }
      free(cols);
      free(pos);
    }
  } else {
    const uint64_t ke = key_of(c->seed, S_EDGE);
    int64_t *start = malloc(sizeof(int64_t) * ((size_t)n + 1));
    start[0] = 0;
#pragma omp parallel for schedule(dynamic, 64)
    for (int i = 0; i < n; ++i) {
      int64_t k = 0;
      for (int j = 0; j < n; ++j)
        if (j != i && uniform(ke, (uint64_t)i, (uint64_t)j) < (double)c->p_connect) ++k;
      start[i + 1] = k;
    }
    for (int i = 0; i < n; ++i) start[i + 1] += start[i];
#pragma omp parallel for schedule(dynamic, 64)
    for (int i = 0; i < n; ++i) {
      int64_t e = start[i];
      for (int j = 0; j < n; ++j) {
        if (j == i || !(uniform(ke, (uint64_t)i, (uint64_t)j) < (double)c->p_connect)) continue;
        double x;
        pre[e] = i;
        post[e] = j;
        delay[e] = c->delay_min + (int)below(kd, (uint64_t)i, (uint64_t)j, dspan);
        w[e] = draw_weight(&wd, (uint64_t)i, (uint64_t)j, i >= c->n_exc, &x);
        if (w64) w64[e] = x;
        ++e;
      }
    }
    free(start);
  }
}
