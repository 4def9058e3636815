/*
 * ORACLE (test infrastructure only).  Plain-C restatement of the reference's
 * native spiking language core, used by tests/ and bench.py's CPU-baseline leg
 * to check the CUDA engine.  Nothing in the product links or calls this file.
 *
 * It follows, operation for operation and in the same fp32 evaluation order
 * (compiled with -ffp-contract=off, so a*b+c is never fused):
 *   - weight unpacking and transforms   src/native/NeuralEngine.cpp:38-67, 111-132
 *   - region step (current, LN, memory)  src/native/NeuralEngine.cpp:68-110
 *   - advance / step / activity          src/native/NeuralEngine.cpp:164-191
 *   - dense projection (mode 0)          src/native/CPUBackend.cpp:13-19
 *   - fused recurrent ALIF tick (mode 1) src/native/CPUBackend.cpp:20-42
 *   - tick loop and activity             src/native/PackedBackend.h:29-54
 *   - state layout                       src/native/NeuralEngine.cpp:137-163
 * and is checked bit-for-bit against the reference library built from those
 * sources (oracle/_ref).  Beyond the reference ABI it can record the spike
 * vector of every tick and the smallest |V - thr - a| margin seen, which the
 * parity tests use to state how far each spike decision was from flipping.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define VOCAB 264
#define UNITS 64

/* Laminar table: (layer, excitatory, inhibitory), include/engine/ALIFNeuron.h:14-15 */
static const int LAYER_TABLE[6][3] = {{1, 0, 2}, {2, 8, 2}, {3, 8, 2},
                                      {4, 12, 3}, {5, 12, 3}, {6, 10, 2}};

typedef struct {
  float *rec;      /* [c,64,64] transformed recurrent weights */
  float *in_w;     /* [c*12, w] */
  float *in_b;     /* [c*12] */
  float *fb_w;     /* [c*29, w] */
  float *out_w;    /* [w, c*100] */
  float *out_b;    /* [w] */
  float *norm_w;   /* [w] */
  float *norm_b;   /* [w] */
  float *decay;    /* [w] transformed memory decay */
} og_region;

typedef struct {
  int columns, width, regions, ticks, idle;
  float sign[UNITS];
  int layer[UNITS];
  int in_ids[UNITS], fb_ids[UNITS], out_ids[UNITS];
  int n_in, n_fb, n_out;
  float *embedding; /* [264, w] */
  float *head_w;    /* [264, w] */
  float *head_b;    /* [264] */
  og_region *reg;
  float *weights; /* owned copy of the packed stream */
  /* optional recording */
  uint8_t *spike_rec;   /* next free slot, advanced per tick */
  uint8_t *spike_end;
  double min_margin;
} og_engine;

static float sigmoidf_(float x) { return 1.f / (1.f + expf(-x)); }

static void build_tables(og_engine *e) {
  int id = 0;
  e->n_in = e->n_fb = e->n_out = 0;
  for (int l = 0; l < 6; ++l) {
    int layer = LAYER_TABLE[l][0], ne = LAYER_TABLE[l][1], ni = LAYER_TABLE[l][2];
    for (int i = 0; i < ne + ni; ++i, ++id) {
      int exc = i < ne;
      e->sign[id] = exc ? 1.f : -1.f;
      e->layer[id] = layer;
      if (layer == 4 && exc) e->in_ids[e->n_in++] = id;
      if (layer >= 5 || layer == 1) e->fb_ids[e->n_fb++] = id;
      if (exc) e->out_ids[e->n_out++] = id;
    }
  }
}

static size_t region_params(const og_engine *e) {
  size_t c = e->columns, w = e->width;
  return c * 4096 + c * e->n_in * (w + 1) + c * e->n_fb * w +
         w * (c * e->n_out * 2 + 1) + 3 * w;
}

size_t og_parameter_count(int columns, int width, int regions) {
  og_engine e;
  memset(&e, 0, sizeof e);
  e.columns = columns;
  e.width = width;
  build_tables(&e);
  return 528ull * width + 264 + (size_t)regions * region_params(&e);
}

size_t og_state_size(int columns, int width, int regions) {
  return (size_t)regions * (5ull * columns * UNITS + width);
}

static int allowed_pair(const og_engine *e, int post, int pre) {
  static const int preferred[6][2] = {{4, 2}, {4, 3}, {2, 3}, {3, 5}, {5, 6}, {6, 4}};
  int ok = e->layer[post] == e->layer[pre];
  for (int k = 0; k < 6; ++k)
    ok |= e->layer[pre] == preferred[k][0] && e->layer[post] == preferred[k][1];
  ok |= e->sign[pre] < 0 && abs(e->layer[post] - e->layer[pre]) <= 1;
  return ok && post != pre;
}

void og_destroy(void *p) {
  og_engine *e = (og_engine *)p;
  if (!e) return;
  free(e->weights);
  free(e->reg);
  free(e);
}

/* Returns NULL on invalid dimensions / count / non-finite weights. */
void *og_create(int columns, int width, int regions, int ticks, int idle,
                const float *weights, size_t count) {
  if (columns < 1 || columns > 4096 || width < 1 || width > 16384 || regions < 1 ||
      regions > 128 || ticks < 1 || ticks > 10000 || idle < 0 || idle > 16)
    return NULL;
  if (!weights || count != og_parameter_count(columns, width, regions)) return NULL;
  for (size_t i = 0; i < count; ++i)
    if (!isfinite(weights[i])) return NULL;
  og_engine *e = (og_engine *)calloc(1, sizeof(og_engine));
  e->columns = columns;
  e->width = width;
  e->regions = regions;
  e->ticks = ticks;
  e->idle = idle;
  build_tables(e);
  e->weights = (float *)malloc(count * sizeof(float));
  memcpy(e->weights, weights, count * sizeof(float));
  e->reg = (og_region *)calloc(regions, sizeof(og_region));
  size_t c = columns, w = width;
  float *p = e->weights;
  e->embedding = p;
  p += 264 * w;
  for (int r = 0; r < regions; ++r) {
    og_region *g = &e->reg[r];
    g->rec = p;
    p += c * 4096;
    for (size_t col = 0; col < c; ++col)
      for (int post = 0; post < UNITS; ++post)
        for (int pre = 0; pre < UNITS; ++pre) {
          float *raw = &g->rec[col * 4096 + post * 64 + pre];
          if (allowed_pair(e, post, pre)) {
            float pos = *raw < 0.f ? 0.f : *raw;
            *raw = (pos + log1pf(expf(-fabsf(*raw)))) * e->sign[pre];
          } else {
            *raw = 0.f;
          }
        }
    g->in_w = p;   p += c * e->n_in * w;
    g->in_b = p;   p += c * e->n_in;
    g->fb_w = p;   p += c * e->n_fb * w;
    g->out_w = p;  p += w * c * e->n_out * 2;
    g->out_b = p;  p += w;
    g->norm_w = p; p += w;
    g->norm_b = p; p += w;
    g->decay = p;  p += w;
    for (size_t i = 0; i < w; ++i) g->decay[i] = .5f + .499f * sigmoidf_(g->decay[i]);
  }
  e->head_w = p;
  p += 264 * w;
  e->head_b = p;
  return e;
}

/* y[i] = b[i] + sum_j W[i,j] x[j], sequential j (CPUBackend.cpp:13-19). */
static void matvec(const float *W, const float *x, const float *b, size_t rows,
                   size_t cols, float *y) {
  for (size_t i = 0; i < rows; ++i) {
    float v = b ? b[i] : 0.f;
    const float *row = W + i * cols;
    for (size_t j = 0; j < cols; ++j) v += row[j] * x[j];
    y[i] = v;
  }
}

/* Per-region state views inside the packed caller state. */
typedef struct {
  float *V, *trace, *adapt, *last, *mem, *counts;
} og_view;

static og_view view(const og_engine *e, float *s, int r) {
  size_t n = (size_t)e->columns * UNITS, w = e->width;
  float *b = s + (size_t)r * (5 * n + w);
  og_view v = {b, b + n, b + 2 * n, b + 3 * n, b + 4 * n, b + 4 * n + w};
  return v;
}

/* One synchronous recurrent ALIF tick (CPUBackend.cpp:20-42); returns spike count. */
static double tick(og_engine *e, const og_region *g, og_view s, const float *current,
                   float *scratch) {
  size_t n = (size_t)e->columns * UNITS;
  float *V = scratch, *tr = scratch + n, *a = scratch + 2 * n, *last = scratch + 3 * n,
        *cnt = scratch + 4 * n;
  double total = 0;
  for (size_t i = 0; i < n; ++i) {
    size_t col = i / UNITS, id = i % UNITS;
    int exc = e->sign[id] > 0;
    float rec = 0.f;
    for (size_t j = 0; j < UNITS; ++j) rec += g->rec[col * 4096 + id * 64 + j] * s.trace[col * 64 + j];
    float nb = 0.f;
    if (exc) {
      if (col > 0) nb += s.trace[i - UNITS];
      if (i + UNITS < n) nb += s.trace[i + UNITS];
    }
    float decay = exc ? .6f : .4f;
    float v = decay * s.V[i] + (1 - decay) * (current[i] + rec + .08f * nb);
    float margin = v - (exc ? 1.f : .6f) - s.adapt[i];
    if (s.last[i] == 0.f && fabs((double)margin) < e->min_margin) e->min_margin = fabs((double)margin);
    float spike = (margin >= 0 ? 1.f : 0.f) * (1 - s.last[i]);
    V[i] = v * (1 - spike);
    tr[i] = .8f * s.trace[i] + .2f * spike;
    a[i] = .98f * s.adapt[i] + (exc ? .03f : 0.f) * spike;
    last[i] = spike;
    cnt[i] = s.counts[i] + spike;
  }
  memcpy(s.V, V, n * sizeof(float));
  memcpy(s.trace, tr, n * sizeof(float));
  memcpy(s.adapt, a, n * sizeof(float));
  memcpy(s.last, last, n * sizeof(float));
  memcpy(s.counts, cnt, n * sizeof(float));
  for (size_t i = 0; i < n; ++i) total += last[i];
  if (e->spike_rec && e->spike_rec + n <= e->spike_end) {
    for (size_t i = 0; i < n; ++i) e->spike_rec[i] = last[i] != 0.f;
    e->spike_rec += n;
  }
  return total;
}

/* CorticalColumnV2::step restated (NeuralEngine.cpp:68-110). h is in/out [w]. */
static float region_step(og_engine *e, int r, float *h, og_view s, int sensory) {
  const og_region *g = &e->reg[r];
  size_t c = e->columns, w = e->width, n = c * UNITS;
  float *current = (float *)malloc(n * sizeof(float));
  float *scratch = (float *)malloc(5 * n * sizeof(float));
  float *tmp = (float *)malloc((c * (e->n_in + e->n_fb) + w) * sizeof(float));
  float *features = (float *)malloc(c * e->n_out * 2 * sizeof(float));
  for (size_t i = 0; i < n; ++i) current[i] = e->sign[i % UNITS] > 0 ? .15f : .35f;
  if (sensory) {
    matvec(g->in_w, h, g->in_b, c * e->n_in, w, tmp);
    for (size_t col = 0; col < c; ++col)
      for (int j = 0; j < e->n_in; ++j)
        current[col * UNITS + e->in_ids[j]] = 3 * sigmoidf_(tmp[col * e->n_in + j]);
  }
  matvec(g->fb_w, s.mem, NULL, c * e->n_fb, w, tmp);
  for (size_t col = 0; col < c; ++col)
    for (int j = 0; j < e->n_fb; ++j)
      current[col * UNITS + e->fb_ids[j]] += .5f * tanhf(tmp[col * e->n_fb + j]);
  double spikes = 0;
  for (int t = 0; t < e->ticks; ++t) spikes += tick(e, g, s, current, scratch);
  float activity = (float)(spikes / (double)(n * e->ticks));
  size_t k = 0;
  for (size_t col = 0; col < c; ++col)
    for (int j = 0; j < e->n_out; ++j) features[k++] = s.V[col * UNITS + e->out_ids[j]];
  for (size_t col = 0; col < c; ++col)
    for (int j = 0; j < e->n_out; ++j) features[k++] = s.trace[col * UNITS + e->out_ids[j]];
  matvec(g->out_w, features, g->out_b, w, c * e->n_out * 2, tmp);
  double mean = 0, var = 0;
  for (size_t i = 0; i < w; ++i) {
    tmp[i] += .25f * s.mem[i];
    mean += tmp[i];
  }
  mean /= (double)w;
  for (size_t i = 0; i < w; ++i) var += (tmp[i] - mean) * (tmp[i] - mean);
  float inv = (float)(1.f / sqrt(var / (double)w + 1e-5));
  for (size_t i = 0; i < w; ++i) {
    h[i] = (tmp[i] - (float)mean) * inv * g->norm_w[i] + g->norm_b[i];
    s.mem[i] = g->decay[i] * s.mem[i] + (1 - g->decay[i]) * h[i];
  }
  free(current);
  free(scratch);
  free(tmp);
  free(features);
  return activity;
}

static float advance(og_engine *e, float *h, float *state, int idle) {
  float activity = 0;
  for (int r = 0; r < e->regions; ++r) {
    float a = region_step(e, r, h, view(e, state, r), !idle || r > 0);
    activity += a;
  }
  return activity / e->regions;
}

static void set_recording(og_engine *e, uint8_t *spikes, size_t spike_bytes) {
  e->spike_rec = spikes;
  e->spike_end = spikes ? spikes + spike_bytes : NULL;
}

/* Token step (NeuralEngine.cpp:177-191).  Optional spikes buffer receives one
 * byte per neuron per tick, in order advance -> region -> tick -> neuron:
 * (1+idle)*regions*ticks*columns*64 bytes. */
int og_step(void *p, int token, const float *state, float *next, float *logits,
            float *hidden, float *activity, uint8_t *spikes, size_t spike_bytes) {
  og_engine *e = (og_engine *)p;
  if (!e || token < 0 || token >= VOCAB || !state || !next || !logits || !hidden || !activity)
    return -1;
  size_t ss = og_state_size(e->columns, e->width, e->regions), w = e->width;
  for (size_t i = 0; i < ss; ++i)
    if (!isfinite(state[i])) return -1;
  if (next != state) memcpy(next, state, ss * sizeof(float));
  set_recording(e, spikes, spike_bytes);
  float *h = (float *)malloc(w * sizeof(float));
  memcpy(h, e->embedding + (size_t)token * w, w * sizeof(float));
  float act = advance(e, h, next, 0);
  for (int i = 0; i < e->idle; ++i) {
    memset(h, 0, w * sizeof(float));
    act += advance(e, h, next, 1);
  }
  *activity = act / (1 + e->idle);
  matvec(e->head_w, h, e->head_b, VOCAB, w, logits);
  memcpy(hidden, h, w * sizeof(float));
  free(h);
  set_recording(e, NULL, 0);
  return 0;
}

/* ng_advance restated (NeuralEngine.cpp:247-267). */
int og_advance(void *p, const float *input, const float *state, int idle, float *next,
               float *hidden, float *activity, uint8_t *spikes, size_t spike_bytes) {
  og_engine *e = (og_engine *)p;
  if (!e || !input || !state || !next || !hidden || !activity) return -1;
  size_t ss = og_state_size(e->columns, e->width, e->regions), w = e->width;
  for (size_t i = 0; i < ss; ++i)
    if (!isfinite(state[i])) return -1;
  for (size_t i = 0; i < w; ++i)
    if (!isfinite(input[i])) return -1;
  if (next != state) memcpy(next, state, ss * sizeof(float));
  set_recording(e, spikes, spike_bytes);
  memcpy(hidden, input, w * sizeof(float));
  *activity = advance(e, hidden, next, idle != 0);
  set_recording(e, NULL, 0);
  return 0;
}

void og_reset_margin(void *p) { ((og_engine *)p)->min_margin = INFINITY; }
double og_min_margin(void *p) { return ((og_engine *)p)->min_margin; }
