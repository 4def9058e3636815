/*
 * ORACLE (test infrastructure only).  Plain-C restatement of one tick of the
 * conductance-based adaptive LIF network with per-synapse integer delays, the
 * semantics of the reference's NumPy simulator with frozen synapses:
 *   neurogen/biology.py:132-180  BiologicalNetwork.step
 *     - arrivals read from delay slot t (biology.py:141-145, 175-176)
 *     - g_E *= exp(-dt/5), g_I *= exp(-dt/10), arrivals added by presynaptic
 *       sign (biology.py:147-150); adaptation *= exp(-dt/200) (:152)
 *     - exact constant-conductance membrane update toward
 *       (gL*EL + EI*gI - a + I)/(gL+gE+gI) with C = 200 pF (E) / 100 pF (I)
 *       (:153-159), refractory clamp to -65 mV for 2 ms (:160-163),
 *       spike at V >= -50 mV -> reset -65 mV, adaptation += 15 pA (E) (:161-166)
 *     - emissions scheduled into slot (t + d) after all cells advanced (:174-176)
 *   E/I split of arrivals by presynaptic sign as include/engine/SparseKernels.cuh:229-287.
 * Optional plasticity (on_set_plasticity): biology.py:182-218 BiologicalNetwork.learn
 * -- pair STDP with soft bounds on E contacts, Vogels-style inhibitory rule on
 * I->E contacts, multiplicative synaptic scaling toward the target rate, weight
 * clipping, and the pre/post/potential traces, coactivity and usage -- plus the
 * rate trace of step() (:167-168); learning runs after the membrane update and
 * before the tick's emissions, which carry the new weights (:169-176).
 * Rewiring and Poisson background (biology.py:151,171-173,220-) are out of
 * scope; an optional Bernoulli drive replaces the background.
 *
 * Two modes:
 *   fp32 -- the exact arithmetic contract of the CUDA engine: fp32 state, the
 *           delay ring holds integer multiples of 2^-24 nS (order-independent
 *           sums), exp() is the shared Cody-Waite + degree-7 Taylor scheme
 *           below, every operation rounded as written (-ffp-contract=off).
 *           The GPU must reproduce this bit for bit.
 *   fp64 -- the same equations in double with libm exp and a double ring,
 *           used to pin the restatement to biology.py itself.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define RING 16

typedef struct {
  int32_t n, n_exc;
  float dt, cap_e, cap_i, g_leak, e_leak, e_inh, v_th, v_reset, t_ref;
  float tau_e, tau_i, tau_a, adapt_inc, bias;
  int32_t drive_kind; /* 0 conductance, 1 imposed */
  float drive_p, drive_ns;
  uint64_t seed;
} on_params;

typedef struct {
  on_params p;
  int64_t nnz;
  int64_t *row;   /* [n+1] by presynaptic neuron */
  int32_t *post;  /* [nnz] */
  int32_t *delay; /* [nnz] */
  float *w;       /* [nnz] fp32 weights (multiples of 2^-24 for the fp32 mode) */
  double *w64;    /* [nnz] the same weights in double (fp64 mode) */
  /* fp32 state */
  float *v, *a, *ge, *gi;
  int32_t *ref;
  int32_t *ring; /* [RING][n][2] */
  /* fp64 state */
  double *v64, *a64, *ge64, *gi64, *ref64;
  double *ring64; /* [RING][n][2] */
  int64_t tick;
  /* plasticity (on_set_plasticity); per-synapse arrays in the stored order */
  int32_t plastic;
  float stdp_rate, inh_rate, target_hz, scaling_tau_ms;
  float *pre_tr, *pot_tr, *coact, *usage, *post_tr, *rate;            /* fp32 */
  double *pre_tr64, *pot_tr64, *coact64, *usage64, *post_tr64, *rate64; /* fp64 */
  uint8_t *hist;   /* [RING][n] spikes of the last RING ticks (fp32 mode) */
  uint8_t *hist64; /* the same for the fp64 mode */
} on_net;

/* splitmix64 finaliser (S. Vigna, public domain) used as a counter-based RNG. */
static uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
/* Drive draw for neuron i at tick t: stream constant 0xD41E. */
static int drive_event(const on_params *p, int64_t t, int32_t i) {
  uint64_t key = mix64(p->seed ^ 0xD41Eull);
  uint32_t u = (uint32_t)(mix64(((uint64_t)t << 32 | (uint32_t)i) ^ key) >> 32);
  double thr = (double)p->drive_p * 4294967296.0;
  uint32_t t32 = thr >= 4294967295.0 ? 0xFFFFFFFFu : (uint32_t)thr;
  return u < t32;
}

/* exp(x) for x <= 0: x = k ln2 + r with ln2 split into a 15-bit head and a
 * tail (Cody & Waite 1980), e^r by its Taylor polynomial to degree 7 in Horner
 * form (|r| <= ln2/2: truncation < 3e-9), scaled by 2^k. */
static float ng_expf(float x) {
  if (x < -87.f) return 0.f;
  const float kf = rintf(x * 1.44269504f);
  const float r = (x - kf * 0.693145751953125f) - kf * 1.42860682e-06f;
  float p = 0.000198412701f;
  p = p * r + 0.00138888892f;
  p = p * r + 0.00833333377f;
  p = p * r + 0.0416666679f;
  p = p * r + 0.166666672f;
  p = p * r + 0.5f;
  p = p * r + 1.0f;
  p = p * r + 1.0f;
  const int k = (int)kf;
  union { uint32_t u; float f; } s;
  if (k >= -126) {
    s.u = (uint32_t)(127 + k) << 23;
    return p * s.f;
  }
  s.u = (uint32_t)(127 + k + 64) << 23; /* two-step scaling into the subnormal range */
  return (p * s.f) * 5.42101086e-20f;  /* 2^-64 */
}

float on_exp_probe(float x) { return ng_expf(x); }

void on_destroy(void *h) {
  on_net *o = (on_net *)h;
  if (!o) return;
  free(o->row); free(o->post); free(o->delay); free(o->w); free(o->w64);
  free(o->v); free(o->a); free(o->ge); free(o->gi); free(o->ref); free(o->ring);
  free(o->v64); free(o->a64); free(o->ge64); free(o->gi64); free(o->ref64); free(o->ring64);
  free(o->pre_tr); free(o->pot_tr); free(o->coact); free(o->usage); free(o->post_tr); free(o->rate);
  free(o->pre_tr64); free(o->pot_tr64); free(o->coact64); free(o->usage64); free(o->post_tr64);
  free(o->rate64); free(o->hist); free(o->hist64);
  free(o);
}

/* Edges in any order; stored by presynaptic neuron, stable in input order.
 * Weights are given in double; the fp32 mode uses them rounded to float. */
/* Network from an edge list: fp32-contract weights w32 and, for the fp64
 * mode, w64 (the same values, or the unrounded draws they were rounded from). */
void *on_create_w(const on_params *p, int64_t nnz, const int32_t *pre, const int32_t *post,
                  const int32_t *delay, const float *w32, const double *w64);

void *on_create(const on_params *p, int64_t nnz, const int32_t *pre, const int32_t *post,
                const int32_t *delay, const double *w) {
  float *w32 = (float *)malloc((size_t)(nnz ? nnz : 1) * sizeof(float));
  for (int64_t e = 0; e < nnz; ++e) w32[e] = (float)w[e];
  void *o = on_create_w(p, nnz, pre, post, delay, w32, w);
  free(w32);
  return o;
}

void *on_create_w(const on_params *p, int64_t nnz, const int32_t *pre, const int32_t *post,
                  const int32_t *delay, const float *w32, const double *w64) {
  on_net *o = (on_net *)calloc(1, sizeof(on_net));
  o->p = *p;
  int32_t n = p->n;
  o->nnz = nnz;
  o->row = (int64_t *)calloc((size_t)n + 1, sizeof(int64_t));
  o->post = (int32_t *)malloc((size_t)(nnz ? nnz : 1) * sizeof(int32_t));
  o->delay = (int32_t *)malloc((size_t)(nnz ? nnz : 1) * sizeof(int32_t));
  o->w = (float *)malloc((size_t)(nnz ? nnz : 1) * sizeof(float));
  o->w64 = (double *)malloc((size_t)(nnz ? nnz : 1) * sizeof(double));
  for (int64_t e = 0; e < nnz; ++e) o->row[pre[e] + 1]++;
  for (int32_t i = 0; i < n; ++i) o->row[i + 1] += o->row[i];
  int64_t *fill = (int64_t *)malloc(((size_t)n + 1) * sizeof(int64_t));
  memcpy(fill, o->row, ((size_t)n + 1) * sizeof(int64_t));
  for (int64_t e = 0; e < nnz; ++e) {
    int64_t k = fill[pre[e]]++;
    o->post[k] = post[e];
    o->delay[k] = delay[e];
    o->w[k] = w32[e];
    o->w64[k] = w64[e];
  }
  free(fill);
  size_t N = (size_t)n;
  o->v = (float *)calloc(N, 4); o->a = (float *)calloc(N, 4);
  o->ge = (float *)calloc(N, 4); o->gi = (float *)calloc(N, 4);
  o->ref = (int32_t *)calloc(N, 4);
  o->ring = (int32_t *)calloc(RING * N * 2, 4);
  o->v64 = (double *)calloc(N, 8); o->a64 = (double *)calloc(N, 8);
  o->ge64 = (double *)calloc(N, 8); o->gi64 = (double *)calloc(N, 8);
  o->ref64 = (double *)calloc(N, 8);
  o->ring64 = (double *)calloc(RING * N * 2, 8);
  for (size_t i = 0; i < N; ++i) { o->v[i] = p->e_leak; o->v64[i] = p->e_leak; }
  return o;
}

void on_set_state(void *h, const float *v, const float *a, const float *ge, const float *gi,
                  const int32_t *ref, const int32_t *ring, int64_t tick) {
  on_net *o = (on_net *)h;
  size_t N = (size_t)o->p.n;
  if (v) memcpy(o->v, v, N * 4);
  if (a) memcpy(o->a, a, N * 4);
  if (ge) memcpy(o->ge, ge, N * 4);
  if (gi) memcpy(o->gi, gi, N * 4);
  if (ref) memcpy(o->ref, ref, N * 4);
  if (ring) memcpy(o->ring, ring, RING * N * 2 * 4);
  o->tick = tick;
}

void on_get_state(void *h, float *v, float *a, float *ge, float *gi, int32_t *ref, int32_t *ring,
                  int64_t *tick) {
  on_net *o = (on_net *)h;
  size_t N = (size_t)o->p.n;
  if (v) memcpy(v, o->v, N * 4);
  if (a) memcpy(a, o->a, N * 4);
  if (ge) memcpy(ge, o->ge, N * 4);
  if (gi) memcpy(gi, o->gi, N * 4);
  if (ref) memcpy(ref, o->ref, N * 4);
  if (ring) memcpy(ring, o->ring, RING * N * 2 * 4);
  if (tick) *tick = o->tick;
}


/* ---- plasticity: biology.py:182-218 (learn) and :167-168 (rate) ---- */

typedef struct {
  int32_t on;
  float stdp_rate, inh_rate, target_hz, scaling_tau_ms; /* .005, .002, 5, 100000 */
} on_plastic;

/* Switches learning on (traces start at zero) or off. */
void on_set_plasticity(void *h, const on_plastic *pl) {
  on_net *o = (on_net *)h;
  const size_t E = (size_t)(o->nnz ? o->nnz : 1), N = (size_t)o->p.n;
  o->plastic = pl->on;
  o->stdp_rate = pl->stdp_rate; o->inh_rate = pl->inh_rate;
  o->target_hz = pl->target_hz; o->scaling_tau_ms = pl->scaling_tau_ms;
  if (!o->pre_tr) {
    o->pre_tr = calloc(E, 4); o->pot_tr = calloc(E, 4); o->coact = calloc(E, 4); o->usage = calloc(E, 4);
    o->post_tr = calloc(N, 4); o->rate = calloc(N, 4);
    o->pre_tr64 = calloc(E, 8); o->pot_tr64 = calloc(E, 8); o->coact64 = calloc(E, 8);
    o->usage64 = calloc(E, 8); o->post_tr64 = calloc(N, 8); o->rate64 = calloc(N, 8);
    o->hist = calloc(RING * N, 1); o->hist64 = calloc(RING * N, 1);
  }
}

/* Constants of the fp32 contract: the reference's expressions in double,
 * rounded once to float. */
typedef struct {
  float decay, slow, one_minus_slow, rate_inc, per_ms, alpha, dt;
} on_lc;

static on_lc lc_of(const on_net *o) {
  const double dt = o->p.dt;
  on_lc c;
  c.decay = (float)exp(-dt / 20.0);
  c.slow = (float)exp(-dt / 1000.0);
  c.one_minus_slow = (float)(1.0 - exp(-dt / 1000.0));
  c.rate_inc = (float)((1.0 - exp(-dt / 1000.0)) * 1000.0 / dt);
  c.per_ms = (float)(1000.0 / dt);
  c.alpha = (float)(2.0 * (double)o->target_hz * .020);
  c.dt = (float)dt;
  return c;
}

/* One learning step in the fp32 contract, every operation rounded as written.
 * arr(e): the contact's presynaptic spike d ticks ago arrives now (biology.py:
 * arrivals = queued amplitude > 0, and potential arrivals: the same for every
 * stored contact); spk(i): this tick's spikes.  The weight's magnitude learns;
 * its sign stays the presynaptic cell's. */
static void learn32(on_net *o, const uint8_t *arr, const uint8_t *spk) {
  const on_params *p = &o->p;
  const on_lc c = lc_of(o);
  const float stdp = o->stdp_rate, inh = o->inh_rate, tgt = o->target_hz, tau_s = o->scaling_tau_ms;
  for (int32_t i = 0; i < p->n; ++i) {
    for (int64_t e = o->row[i]; e < o->row[i + 1]; ++e) {
      const float w0 = o->w[e];
      if (w0 == 0.f) continue; /* not a contact */
      const int32_t q = o->post[e];
      const float a = arr[e] ? 1.f : 0.f, post = spk[q] ? 1.f : 0.f;
      const float pt = o->pre_tr[e] * c.decay, pot = o->pot_tr[e] * c.decay, pq = o->post_tr[q] * c.decay;
      float w = fabsf(w0);
      const int exc = i < p->n_exc;
      if (o->plastic) {
        float delta;
        if (exc) {
          delta = stdp * ((pt * post) * (4.f - w) - ((1.05f * pq) * a) * w);
        } else {
          delta = inh * (a * (pq - c.alpha) + pt * post);
          delta = delta * (q < p->n_exc ? 1.f : 0.f);
        }
        w = w + delta;
        if (exc) {
          float x = (((tgt - o->rate[q]) / tgt) * c.dt) / tau_s;
          x = x < -.001f ? -.001f : (x > .001f ? .001f : x);
          w = w * ng_expf(x);
        }
        const float hi = exc ? 4.f : 12.f;
        w = w < .01f ? .01f : w;
        w = w > hi ? hi : w;
      }
      o->coact[e] = o->coact[e] * c.slow + (c.one_minus_slow * pot) * post;
      o->usage[e] = o->usage[e] * c.slow + ((c.one_minus_slow * a) * c.per_ms);
      o->pre_tr[e] = pt + a;
      o->pot_tr[e] = pot + a;
      o->w[e] = w0 < 0.f ? -w : w;
    }
  }
  for (int32_t i = 0; i < p->n; ++i) o->post_tr[i] = o->post_tr[i] * c.decay + (spk[i] ? 1.f : 0.f);
}

/* The same step in double, in biology.py's operation order (fp64 mode). */
static void learn64(on_net *o, const uint8_t *arr, const uint8_t *spk) {
  const on_params *p = &o->p;
  const double dt = p->dt, decay = exp(-dt / 20.0), slow = exp(-dt / 1000.0);
  const double stdp = o->stdp_rate, inh = o->inh_rate, tgt = o->target_hz, tau_s = o->scaling_tau_ms;
  const double alpha = 2.0 * tgt * .020;
  for (int32_t i = 0; i < p->n; ++i) {
    for (int64_t e = o->row[i]; e < o->row[i + 1]; ++e) {
      const double w0 = o->w64[e];
      if (w0 == 0.0) continue;
      const int32_t q = o->post[e];
      const double a = arr[e] ? 1.0 : 0.0, post = spk[q] ? 1.0 : 0.0;
      const double pt = o->pre_tr64[e] * decay, pot = o->pot_tr64[e] * decay, pq = o->post_tr64[q] * decay;
      double w = fabs(w0);
      const int exc = i < p->n_exc;
      if (o->plastic) {
        double delta;
        if (exc) {
          delta = stdp * (pt * post * (4 - w) - 1.05 * pq * a * w);
        } else {
          delta = inh * (a * (pq - alpha) + pt * post);
          delta *= q < p->n_exc ? 1.0 : 0.0;
        }
        w += delta;
        if (exc) {
          double x = (tgt - o->rate64[q]) / tgt * dt / tau_s;
          x = x < -.001 ? -.001 : (x > .001 ? .001 : x);
          w *= exp(x);
        }
        const double hi = exc ? 4.0 : 12.0;
        w = w < .01 ? .01 : w;
        w = w > hi ? hi : w;
      }
      o->coact64[e] = o->coact64[e] * slow + (1 - slow) * pot * post;
      o->usage64[e] = o->usage64[e] * slow + (1 - slow) * a * 1000 / dt;
      o->pre_tr64[e] = pt + a;
      o->pot_tr64[e] = pot + a;
      o->w64[e] = w0 < 0 ? -w : w;
    }
  }
  for (int32_t i = 0; i < p->n; ++i) o->post_tr64[i] = o->post_tr64[i] * decay + (spk[i] ? 1.0 : 0.0);
}

/* Arrival flags of this tick from the spike history (contact e: its
 * presynaptic cell's spike `delay` ticks ago). */
static void arrivals_of(const on_net *o, const uint8_t *hist, int64_t t, uint8_t *arr) {
  for (int32_t i = 0; i < o->p.n; ++i)
    for (int64_t e = o->row[i]; e < o->row[i + 1]; ++e)
      arr[e] = hist[(size_t)((t - o->delay[e]) & (RING - 1)) * o->p.n + i];
}

/* One learning step with caller-given arrivals (per stored contact) and
 * spikes (per cell), as biology.py's learn() probe; fp64 != 0 selects the
 * double state.  Test infrastructure for the reference's known-answer tests. */
void on_learn_probe(void *h, const uint8_t *arr, const uint8_t *spk, int fp64) {
  on_net *o = (on_net *)h;
  if (fp64) learn64(o, arr, spk);
  else learn32(o, arr, spk);
}

/* Plasticity state in the stored contact order (by presynaptic cell, stable
 * in input order): weights, traces; per cell the post trace and the rate.
 * Any pointer may be NULL. */
void on_get_plasticity(void *h, float *w, float *pre_tr, float *pot_tr, float *coact, float *usage,
                       float *post_tr, float *rate) {
  on_net *o = (on_net *)h;
  const size_t E = (size_t)o->nnz, N = (size_t)o->p.n;
  if (w) memcpy(w, o->w, E * 4);
  if (o->pre_tr) {
    if (pre_tr) memcpy(pre_tr, o->pre_tr, E * 4);
    if (pot_tr) memcpy(pot_tr, o->pot_tr, E * 4);
    if (coact) memcpy(coact, o->coact, E * 4);
    if (usage) memcpy(usage, o->usage, E * 4);
    if (post_tr) memcpy(post_tr, o->post_tr, N * 4);
    if (rate) memcpy(rate, o->rate, N * 4);
  }
}

void on_get_plasticity64(void *h, double *w, double *pre_tr, double *pot_tr, double *coact, double *usage,
                         double *post_tr, double *rate) {
  on_net *o = (on_net *)h;
  const size_t E = (size_t)o->nnz, N = (size_t)o->p.n;
  if (w) memcpy(w, o->w64, E * 8);
  if (o->pre_tr64) {
    if (pre_tr) memcpy(pre_tr, o->pre_tr64, E * 8);
    if (pot_tr) memcpy(pot_tr, o->pot_tr64, E * 8);
    if (coact) memcpy(coact, o->coact64, E * 8);
    if (usage) memcpy(usage, o->usage64, E * 8);
    if (post_tr) memcpy(post_tr, o->post_tr64, N * 8);
    if (rate) memcpy(rate, o->rate64, N * 8);
  }
}

static float decay_f(float dt, float tau) { return (float)exp(-(double)dt / (double)tau); }

/* fp32 ticks.  spikes: [ticks][ceil(n/32)] bit words (may be NULL);
 * counts: [ticks][2] = spikes, synaptic events (may be NULL). */
int on_run(void *h, int ticks, uint32_t *spikes, int64_t *counts) {
  on_net *o = (on_net *)h;
  const on_params *p = &o->p;
  const int32_t n = p->n;
  const size_t words = ((size_t)n + 31) / 32;
  const float dE = decay_f(p->dt, p->tau_e), dI = decay_f(p->dt, p->tau_i), dA = decay_f(p->dt, p->tau_a);
  const float Q = 5.9604644775390625e-08f; /* 2^-24 */
  const float gLEL = p->g_leak * p->e_leak, neg_dt = -p->dt;
  const int32_t ref_ticks = (int32_t)lround((double)p->t_ref / (double)p->dt);
  uint8_t *fired = (uint8_t *)malloc((size_t)n);
  for (int k = 0; k < ticks; ++k) {
    const int64_t t = o->tick;
    const int slot = (int)(t & (RING - 1));
    int64_t nspk = 0, events = 0;
    for (int32_t i = 0; i < n; ++i) {
      int32_t *rs = o->ring + ((size_t)slot * n + i) * 2;
      const int32_t re = rs[0], ri = rs[1];
      rs[0] = rs[1] = 0;
      const int exc = i < p->n_exc;
      float ge = o->ge[i] * dE + (float)re * Q;
      float gi = o->gi[i] * dI + (float)ri * Q;
      const int ev = drive_event(p, t, i);
      if (p->drive_kind == 0 && ev) ge = ge + p->drive_ns;
      float a = o->a[i] * dA;
      const float g = (p->g_leak + ge) + gi;
      const float vinf = (((gLEL + p->e_inh * gi) - a) + p->bias) / g;
      const int avail = o->ref[i] <= 0;
      const float cap = exc ? p->cap_e : p->cap_i;
      float v = vinf + (o->v[i] - vinf) * ng_expf((neg_dt * g) / cap);
      if (!avail) v = p->v_reset;
      const int s = p->drive_kind == 1 ? ev : (avail && v >= p->v_th);
      if (s) v = p->v_reset;
      int32_t ref = o->ref[i] > 0 ? o->ref[i] - 1 : 0;
      if (s) ref = ref_ticks;
      if (s && exc) a = a + p->adapt_inc;
      o->v[i] = v; o->a[i] = a; o->ge[i] = ge; o->gi[i] = gi; o->ref[i] = ref;
      fired[i] = (uint8_t)s;
    }
    if (o->pre_tr) { /* rate (biology.py:167-168), learn (:170), spike history (:174) */
      const on_lc c = lc_of(o);
      for (int32_t i = 0; i < n; ++i) {
        o->rate[i] = o->rate[i] * c.slow;
        if (fired[i]) o->rate[i] = o->rate[i] + c.rate_inc;
      }
      uint8_t *arr = (uint8_t *)malloc((size_t)(o->nnz ? o->nnz : 1));
      arrivals_of(o, o->hist, t, arr);
      learn32(o, arr, fired);
      free(arr);
      memcpy(o->hist + (size_t)(t & (RING - 1)) * n, fired, (size_t)n);
    }
    if (spikes) memset(spikes + (size_t)k * words, 0, words * 4);
    for (int32_t i = 0; i < n; ++i) {
      if (!fired[i]) continue;
      ++nspk;
      if (spikes) spikes[(size_t)k * words + i / 32] |= 1u << (i % 32);
      for (int64_t e = o->row[i]; e < o->row[i + 1]; ++e) {
        const float w = o->w[e];
        if (w == 0.f) continue;
        ++events;
        const int comp = w < 0.f;
        const int32_t q = (int32_t)lrintf(fabsf(w) * 16777216.f);
        const int dslot = (int)((t + o->delay[e]) & (RING - 1));
        o->ring[((size_t)dslot * n + o->post[e]) * 2 + comp] += q;
      }
    }
    if (counts) { counts[2 * k] = nspk; counts[2 * k + 1] = events; }
    o->tick++;
  }
  free(fired);
  return 0;
}

/* fp64 ticks with libm exp and a double ring; current: per-neuron injected
 * current in pA for every tick (NULL = p->bias).  v_out: [ticks][n] (may be
 * NULL).  Used only to pin the equations to biology.py. */
int on_run64(void *h, int ticks, const double *current, uint32_t *spikes, double *v_out,
             double *ge_out, double *gi_out) {
  on_net *o = (on_net *)h;
  const on_params *p = &o->p;
  const int32_t n = p->n;
  const size_t words = ((size_t)n + 31) / 32;
  const double dt = p->dt;
  const double dE = exp(-dt / p->tau_e), dI = exp(-dt / p->tau_i), dA = exp(-dt / p->tau_a);
  uint8_t *fired = (uint8_t *)malloc((size_t)n);
  for (int k = 0; k < ticks; ++k) {
    const int64_t t = o->tick;
    const int slot = (int)(t % RING);
    for (int32_t i = 0; i < n; ++i) {
      double *rs = o->ring64 + ((size_t)slot * n + i) * 2;
      const int exc = i < p->n_exc;
      double ge = o->ge64[i] * dE + rs[0];
      double gi = o->gi64[i] * dI + rs[1];
      rs[0] = rs[1] = 0;
      if (p->drive_kind == 0 && drive_event(p, t, i)) ge += p->drive_ns;
      double a = o->a64[i] * dA;
      const double drive = current ? current[i] : p->bias;
      const double g = p->g_leak + ge + gi;
      const double vinf = ((double)p->g_leak * p->e_leak + p->e_inh * gi - a + drive) / g;
      const int avail = o->ref64[i] <= 0;
      const double cap = exc ? p->cap_e : p->cap_i;
      double v = vinf + (o->v64[i] - vinf) * exp(-dt * g / cap);
      if (!avail) v = p->v_reset;
      const int s = avail && v >= p->v_th;
      if (s) v = p->v_reset;
      double ref = o->ref64[i] - dt;
      if (ref < 0) ref = 0;
      if (s) ref = p->t_ref;
      if (s && exc) a += p->adapt_inc;
      o->v64[i] = v; o->a64[i] = a; o->ge64[i] = ge; o->gi64[i] = gi; o->ref64[i] = ref;
      fired[i] = (uint8_t)s;
      if (v_out) v_out[(size_t)k * n + i] = v;
      if (ge_out) ge_out[(size_t)k * n + i] = ge;
      if (gi_out) gi_out[(size_t)k * n + i] = gi;
    }
    if (o->pre_tr64) {
      for (int32_t i = 0; i < n; ++i) {
        o->rate64[i] *= exp(-dt / 1000.0);
        o->rate64[i] += (1 - exp(-dt / 1000.0)) * (fired[i] ? 1.0 : 0.0) * 1000 / dt;
      }
      uint8_t *arr = (uint8_t *)malloc((size_t)(o->nnz ? o->nnz : 1));
      arrivals_of(o, o->hist64, t, arr);
      learn64(o, arr, fired);
      free(arr);
      memcpy(o->hist64 + (size_t)(t & (RING - 1)) * n, fired, (size_t)n);
    }
    if (spikes) memset(spikes + (size_t)k * words, 0, words * 4);
    for (int32_t i = 0; i < n; ++i) {
      if (!fired[i]) continue;
      if (spikes) spikes[(size_t)k * words + i / 32] |= 1u << (i % 32);
      for (int64_t e = o->row[i]; e < o->row[i + 1]; ++e) {
        const double w = o->w64[e];
        const int dslot = (int)((t + o->delay[e]) % RING);
        o->ring64[((size_t)dslot * n + o->post[e]) * 2 + (w < 0)] += fabs(w);
      }
    }
    o->tick++;
  }
  free(fired);
  return 0;
}

void on_set_state64(void *h, const double *v, const double *a, const double *ge, const double *gi,
                    const double *ref) {
  on_net *o = (on_net *)h;
  size_t N = (size_t)o->p.n;
  if (v) memcpy(o->v64, v, N * 8);
  if (a) memcpy(o->a64, a, N * 8);
  if (ge) memcpy(o->ge64, ge, N * 8);
  if (gi) memcpy(o->gi64, gi, N * 8);
  if (ref) memcpy(o->ref64, ref, N * 8);
}

/* on_run with OpenMP: neurons in parallel for the membrane update, spiking
 * neurons in parallel for delivery (integer atomics, so the ring -- and every
 * result -- is identical to on_run).  Used as the timed CPU baseline. */
int on_run_mt(void *h, int ticks, int64_t *counts) {
  on_net *o = (on_net *)h;
  if (o->pre_tr) return -1; /* plasticity runs in on_run */
  const on_params *p = &o->p;
  const int32_t n = p->n;
  const float dE = decay_f(p->dt, p->tau_e), dI = decay_f(p->dt, p->tau_i), dA = decay_f(p->dt, p->tau_a);
  const float Q = 5.9604644775390625e-08f;
  const float gLEL = p->g_leak * p->e_leak, neg_dt = -p->dt;
  const int32_t ref_ticks = (int32_t)lround((double)p->t_ref / (double)p->dt);
  uint8_t *fired = (uint8_t *)malloc((size_t)n);
  for (int k = 0; k < ticks; ++k) {
    const int64_t t = o->tick;
    const int slot = (int)(t & (RING - 1));
    int64_t nspk = 0, events = 0;
#pragma omp parallel for schedule(static) reduction(+ : nspk)
    for (int32_t i = 0; i < n; ++i) {
      int32_t *rs = o->ring + ((size_t)slot * n + i) * 2;
      const int32_t re = rs[0], ri = rs[1];
      rs[0] = rs[1] = 0;
      const int exc = i < p->n_exc;
      float ge = o->ge[i] * dE + (float)re * Q;
      float gi = o->gi[i] * dI + (float)ri * Q;
      const int ev = drive_event(p, t, i);
      if (p->drive_kind == 0 && ev) ge = ge + p->drive_ns;
      float a = o->a[i] * dA;
      const float g = (p->g_leak + ge) + gi;
      const float vinf = (((gLEL + p->e_inh * gi) - a) + p->bias) / g;
      const int avail = o->ref[i] <= 0;
      const float cap = exc ? p->cap_e : p->cap_i;
      float v = vinf + (o->v[i] - vinf) * ng_expf((neg_dt * g) / cap);
      if (!avail) v = p->v_reset;
      const int s = p->drive_kind == 1 ? ev : (avail && v >= p->v_th);
      if (s) v = p->v_reset;
      int32_t ref = o->ref[i] > 0 ? o->ref[i] - 1 : 0;
      if (s) ref = ref_ticks;
      if (s && exc) a = a + p->adapt_inc;
      o->v[i] = v; o->a[i] = a; o->ge[i] = ge; o->gi[i] = gi; o->ref[i] = ref;
      fired[i] = (uint8_t)s;
      nspk += s;
    }
#pragma omp parallel for schedule(dynamic, 256) reduction(+ : events)
    for (int32_t i = 0; i < n; ++i) {
      if (!fired[i]) continue;
      for (int64_t e = o->row[i]; e < o->row[i + 1]; ++e) {
        const float w = o->w[e];
        if (w == 0.f) continue;
        ++events;
        const int comp = w < 0.f;
        const int32_t q = (int32_t)lrintf(fabsf(w) * 16777216.f);
        const int dslot = (int)((t + o->delay[e]) & (RING - 1));
        int32_t *dst = &o->ring[((size_t)dslot * n + o->post[e]) * 2 + comp];
#pragma omp atomic
        *dst += q;
      }
    }
    if (counts) { counts[2 * k] = nspk; counts[2 * k + 1] = events; }
    o->tick++;
  }
  free(fired);
  return 0;
}
