/* C restatement of rngd-pd's CPU fp32 path, for full Llama-3.1-8B sizes.
 *
 * TEST INFRASTRUCTURE ONLY: loaded by tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py through oracle/corc.py.
 * It is the checker, never the product.
 *
 * Arithmetic follows the reference's numpy oracles, fp32 throughout:
 *   decode layer   src/rngd_pd/kernels/decode_batch.py:126-161 (cpu_layer)
 *   prefill layer  src/rngd_pd/kernels/prefill_full.py:97-128 (cpu_layer_p)
 *   rmsnorm/rope   src/rngd_pd/engines/model.py:53-66
 *   lm_head+argmax src/rngd_pd/engines/decode_batch.py:162-171 (first maximum)
 * with one modelling choice stated by the build: every k/v written to the
 * cache is rounded to bf16 (round-to-nearest-even) before attention reads it,
 * because the cache the device keeps is bf16.  oracle/ref_np.py holds the same
 * restatement in numpy; tests/test_oracle_c.py checks the two agree.
 *
 * Weights are bf16 (uint16 bits) in the HF [out, in] layout, generated here by
 * the integer-only recipe documented in oracle/synth_np.py.  Caches are bf16
 * bits: decode K and V [L][B][NKV][S][HD]; prefill output in the reference
 * layout K [L][NKV][HD][S], V [L][NKV][S][HD].
 */
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------ synthetic data */
static inline uint64_t mix64(uint64_t x) {
  uint64_t z = x + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
static inline uint64_t stream_key(uint64_t seed, uint64_t tid) { return mix64(mix64(seed) ^ tid); }
static inline uint16_t f2bf(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}
static inline float bf2f(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static inline uint16_t gauss_one(uint64_t key, uint64_t i, float scale) {
  uint64_t h = mix64(key + i);
  int64_t s = (int64_t)((h & 0xFFFF) + ((h >> 16) & 0xFFFF) + ((h >> 32) & 0xFFFF) + (h >> 48)) - 131070;
  return f2bf((float)s * scale);
}

void orc_gauss_bf16(uint16_t* out, uint64_t seed, uint64_t tid, uint64_t start, uint64_t n, float scale) {
  uint64_t key = stream_key(seed, tid);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < (int64_t)n; i++) out[i] = gauss_one(key, start + (uint64_t)i, scale);
}

void orc_uniform(int64_t* out, uint64_t seed, uint64_t tid, uint64_t start, uint64_t n, uint64_t hi) {
  uint64_t key = stream_key(seed, tid);
  for (uint64_t i = 0; i < n; i++) out[i] = (int64_t)((mix64(key + start + i) >> 32) % hi);
}

void orc_set_threads(int n) { if (n > 0) omp_set_num_threads(n); }
int orc_get_threads(void) { return omp_get_max_threads(); }

/* ------------------------------------------------------------------- model */
enum { K_Q, K_K, K_V, K_O, K_GATE, K_UP, K_DOWN, NKIND };
#define T_EMBED 0x7000
#define T_LMHEAD 0x7001
#define T_KCACHE 0x8000
#define T_VCACHE 0x8001

typedef struct {
  int H, M, NH, NKV, HD, L, V;
  float eps, theta;
  float inv[256];
  uint16_t** w;      /* [L * NKIND] */
  uint16_t* embed;   /* [V][H] */
  uint16_t* lm;      /* [V][H] */
} OrcModel;

static void kind_shape(const OrcModel* m, int k, int* rows, int* cols) {
  switch (k) {
    case K_Q: *rows = m->NH * m->HD; *cols = m->H; break;
    case K_K: case K_V: *rows = m->NKV * m->HD; *cols = m->H; break;
    case K_O: *rows = m->H; *cols = m->NH * m->HD; break;
    case K_GATE: case K_UP: *rows = m->M; *cols = m->H; break;
    default: *rows = m->H; *cols = m->M; break;
  }
}

/* inv: fp32 inverse frequencies computed by the caller (float64 power cast to fp32,
 * kernels/decode_batch.py:197).  Norm weights are 1.0 (HF initialisation). */
OrcModel* orc_model_create(int H, int M, int NH, int NKV, int HD, int L, int V, float eps,
                           const float* inv, uint64_t seed, float scale) {
  OrcModel* m = (OrcModel*)calloc(1, sizeof(OrcModel));
  m->H = H; m->M = M; m->NH = NH; m->NKV = NKV; m->HD = HD; m->L = L; m->V = V; m->eps = eps;
  memcpy(m->inv, inv, sizeof(float) * (size_t)(HD / 2));
  m->w = (uint16_t**)calloc((size_t)L * NKIND, sizeof(uint16_t*));
  for (int l = 0; l < L; l++)
    for (int k = 0; k < NKIND; k++) {
      int r, c;
      kind_shape(m, k, &r, &c);
      uint16_t* p = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)r * c);
      orc_gauss_bf16(p, seed, (uint64_t)(l * 16 + k), 0, (uint64_t)r * c, scale);
      m->w[l * NKIND + k] = p;
    }
  m->embed = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)V * H);
  m->lm = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)V * H);
  orc_gauss_bf16(m->embed, seed, T_EMBED, 0, (uint64_t)V * H, scale);
  orc_gauss_bf16(m->lm, seed, T_LMHEAD, 0, (uint64_t)V * H, scale);
  return m;
}

void orc_model_free(OrcModel* m) {
  if (!m) return;
  for (int i = 0; i < m->L * NKIND; i++) free(m->w[i]);
  free(m->w); free(m->embed); free(m->lm); free(m);
}

/* Y[b][n] = sum_k W[n][k] * X[b][k], fp32 accumulation (16 partial sums). */
static void gemv(const uint16_t* W, int N, int K, const float* X, int B, float* Y) {
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; n++) {
    const uint16_t* w = W + (size_t)n * K;
    for (int b0 = 0; b0 < B; b0 += 16) {
      int nb = B - b0 < 16 ? B - b0 : 16;
      float acc[16][16];
      memset(acc, 0, sizeof(acc));
      for (int k = 0; k < K; k += 16) {
        float wf[16];
        for (int j = 0; j < 16; j++) wf[j] = bf2f(w[k + j]);
        for (int b = 0; b < nb; b++) {
          const float* x = X + (size_t)(b0 + b) * K + k;
          for (int j = 0; j < 16; j++) acc[b][j] += wf[j] * x[j];
        }
      }
      for (int b = 0; b < nb; b++) {
        float s = 0.f;
        for (int j = 0; j < 16; j++) s += acc[b][j];
        Y[(size_t)(b0 + b) * N + n] = s;
      }
    }
  }
}

static void rmsnorm_rows(const float* x, int R, int H, float eps, float* out) {
  for (int r = 0; r < R; r++) {
    const float* xr = x + (size_t)r * H;
    float acc[16] = {0};
    for (int k = 0; k < H; k += 16)
      for (int j = 0; j < 16; j++) acc[j] += xr[k + j] * xr[k + j];
    float s = 0.f;
    for (int j = 0; j < 16; j++) s += acc[j];
    float inv = 1.0f / sqrtf(s / (float)H + eps);  /* norm weight = 1 */
    for (int k = 0; k < H; k++) out[(size_t)r * H + k] = xr[k] * inv;
  }
}

/* HF rotate-half RoPE at position pos over nh heads of HD (engines/model.py:57-66). */
static void rope(float* t, int nh, int HD, int pos, const float* inv) {
  int half = HD / 2;
  for (int h = 0; h < nh; h++) {
    float* r = t + (size_t)h * HD;
    for (int i = 0; i < half; i++) {
      float ang = (float)pos * inv[i];
      float c = cosf(ang), s = sinf(ang);
      float a = r[i], b = r[i + half];
      r[i] = a * c - b * s;
      r[i + half] = b * c + a * s;
    }
  }
}

static float silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

/* MLP block + residual for R rows: x2 (residual in) -> xout. */
static void mlp(const OrcModel* m, int l, const float* x2, int R, float* xout) {
  int H = m->H, Mi = m->M;
  float* h2 = (float*)malloc(sizeof(float) * (size_t)R * H);
  float* g = (float*)malloc(sizeof(float) * (size_t)R * Mi);
  float* u = (float*)malloc(sizeof(float) * (size_t)R * Mi);
  float* y = (float*)malloc(sizeof(float) * (size_t)R * H);
  rmsnorm_rows(x2, R, H, m->eps, h2);
  gemv(m->w[l * NKIND + K_GATE], Mi, H, h2, R, g);
  gemv(m->w[l * NKIND + K_UP], Mi, H, h2, R, u);
  for (size_t i = 0; i < (size_t)R * Mi; i++) g[i] = silu_mul(g[i], u[i]);
  gemv(m->w[l * NKIND + K_DOWN], H, Mi, g, R, y);
  for (size_t i = 0; i < (size_t)R * H; i++) xout[i] = y[i] + x2[i];
  free(h2); free(g); free(u); free(y);
}

static void logits_rows(const OrcModel* m, const float* x, int R, float* logits) {
  float* h = (float*)malloc(sizeof(float) * (size_t)R * m->H);
  rmsnorm_rows(x, R, m->H, m->eps, h);
  gemv(m->lm, m->V, m->H, h, R, logits);
  free(h);
}

static int argmax_first(const float* v, int n) {
  int best = 0;
  for (int i = 1; i < n; i++)
    if (v[i] > v[best]) best = i;
  return best;
}

/* One batched decode step for B streams (engines/decode_batch.py:427-442).
 * Kc, Vc: bf16 caches [L][B][NKV][S][HD], updated at pos[b].  Writes fp32 logits
 * [B][V] when logits != NULL, next tokens when next != NULL, final hidden [B][H]
 * when hidden != NULL. */
static void decode_impl(const OrcModel* m, int B, int S, const int64_t* toks, const int64_t* pos, uint16_t* Kc,
                        uint16_t* Vc, float* logits, int64_t* next, float* hidden, int keep_rows, uint16_t* own_k,
                        uint16_t* own_v);

void orc_decode_step(const OrcModel* m, int B, int S, const int64_t* toks, const int64_t* pos,
                     uint16_t* Kc, uint16_t* Vc, float* logits, int64_t* next, float* hidden) {
  decode_impl(m, B, S, toks, pos, Kc, Vc, logits, next, hidden, 0, NULL, NULL);
}

/* The same step for a per-step parity check: the cache rows at pos[b] are left as the caller
 * put them (keep_rows = 1: e.g. the device's rows of this step), and the rows this oracle
 * computes are written to own_k / own_v ([L][B][NKV*HD] bf16 bits) when those are non-NULL. */
void orc_decode_step_rows(const OrcModel* m, int B, int S, const int64_t* toks, const int64_t* pos,
                          uint16_t* Kc, uint16_t* Vc, float* logits, int64_t* next, float* hidden, int keep_rows,
                          uint16_t* own_k, uint16_t* own_v) {
  decode_impl(m, B, S, toks, pos, Kc, Vc, logits, next, hidden, keep_rows, own_k, own_v);
}

static void decode_impl(const OrcModel* m, int B, int S, const int64_t* toks, const int64_t* pos, uint16_t* Kc,
                        uint16_t* Vc, float* logits, int64_t* next, float* hidden, int keep_rows, uint16_t* own_k,
                        uint16_t* own_v) {
  int H = m->H, NH = m->NH, NKV = m->NKV, HD = m->HD, G = NH / NKV;
  int QN = NH * HD, KN = NKV * HD;
  float* x = (float*)malloc(sizeof(float) * (size_t)B * H);
  float* h = (float*)malloc(sizeof(float) * (size_t)B * H);
  float* q = (float*)malloc(sizeof(float) * (size_t)B * QN);
  float* k = (float*)malloc(sizeof(float) * (size_t)B * KN);
  float* v = (float*)malloc(sizeof(float) * (size_t)B * KN);
  float* ao = (float*)malloc(sizeof(float) * (size_t)B * QN);
  float* x2 = (float*)malloc(sizeof(float) * (size_t)B * H);
  float scale = 1.0f / sqrtf((float)HD);
  for (int b = 0; b < B; b++)
    for (int i = 0; i < H; i++) x[(size_t)b * H + i] = bf2f(m->embed[(size_t)toks[b] * H + i]);
  for (int l = 0; l < m->L; l++) {
    rmsnorm_rows(x, B, H, m->eps, h);
    gemv(m->w[l * NKIND + K_Q], QN, H, h, B, q);
    gemv(m->w[l * NKIND + K_K], KN, H, h, B, k);
    gemv(m->w[l * NKIND + K_V], KN, H, h, B, v);
    for (int b = 0; b < B; b++) {
      rope(q + (size_t)b * QN, NH, HD, (int)pos[b], m->inv);
      rope(k + (size_t)b * KN, NKV, HD, (int)pos[b], m->inv);
      for (int kh = 0; kh < NKV; kh++) {
        size_t base = ((((size_t)l * B + b) * NKV + kh) * S + (size_t)pos[b]) * HD;
        size_t own = (((size_t)l * B + b) * NKV + kh) * HD;
        for (int d = 0; d < HD; d++) {
          uint16_t kb = f2bf(k[(size_t)b * KN + kh * HD + d]), vb = f2bf(v[(size_t)b * KN + kh * HD + d]);
          if (own_k) own_k[own + d] = kb;
          if (own_v) own_v[own + d] = vb;
          if (!keep_rows) {
            Kc[base + d] = kb;
            Vc[base + d] = vb;
          }
        }
      }
    }
#pragma omp parallel for collapse(2) schedule(static)
    for (int b = 0; b < B; b++)
      for (int hh = 0; hh < NH; hh++) {
        int kh = hh / G, P = (int)pos[b] + 1;
        const float* qh = q + (size_t)b * QN + (size_t)hh * HD;
        size_t base = (((size_t)l * B + b) * NKV + kh) * (size_t)S * HD;
        float* sc = (float*)malloc(sizeof(float) * (size_t)P);
        float mx = -INFINITY;
        for (int s = 0; s < P; s++) {
          float acc = 0.f;
          for (int d = 0; d < HD; d++) acc += qh[d] * bf2f(Kc[base + (size_t)s * HD + d]);
          sc[s] = acc * scale;
          if (sc[s] > mx) mx = sc[s];
        }
        float sum = 0.f;
        for (int s = 0; s < P; s++) { sc[s] = expf(sc[s] - mx); sum += sc[s]; }
        float* o = ao + (size_t)b * QN + (size_t)hh * HD;
        for (int d = 0; d < HD; d++) o[d] = 0.f;
        for (int s = 0; s < P; s++) {
          float p = sc[s] / sum;
          for (int d = 0; d < HD; d++) o[d] += p * bf2f(Vc[base + (size_t)s * HD + d]);
        }
        free(sc);
      }
    gemv(m->w[l * NKIND + K_O], H, QN, ao, B, x2);
    for (size_t i = 0; i < (size_t)B * H; i++) x2[i] += x[i];
    mlp(m, l, x2, B, x);
  }
  if (hidden) memcpy(hidden, x, sizeof(float) * (size_t)B * H);
  if (logits || next) {
    float* lg = logits ? logits : (float*)malloc(sizeof(float) * (size_t)B * m->V);
    logits_rows(m, x, B, lg);
    if (next)
      for (int b = 0; b < B; b++) next[b] = argmax_first(lg + (size_t)b * m->V, m->V);
    if (!logits) free(lg);
  }
  free(x); free(h); free(q); free(k); free(v); free(ao); free(x2);
}

/* Whole-prompt prefill of P tokens (engines/prefill_full.py:337-388 for an exact-fit
 * bucket: causal attention within the prompt, cache zero past P).
 * Kout [L][NKV][HD][S], Vout [L][NKV][S][HD] bf16 bits (reference layout);
 * logits [V] of the last position and its first-max argmax. */
void orc_prefill(const OrcModel* m, int P, const int64_t* toks, int S, uint16_t* Kout, uint16_t* Vout,
                 float* logits, int64_t* next, float* hidden) {
  int H = m->H, NH = m->NH, NKV = m->NKV, HD = m->HD, G = NH / NKV;
  int QN = NH * HD, KN = NKV * HD;
  float* x = (float*)malloc(sizeof(float) * (size_t)P * H);
  float* h = (float*)malloc(sizeof(float) * (size_t)P * H);
  float* q = (float*)malloc(sizeof(float) * (size_t)P * QN);
  float* k = (float*)malloc(sizeof(float) * (size_t)P * KN);
  float* v = (float*)malloc(sizeof(float) * (size_t)P * KN);
  float* ao = (float*)malloc(sizeof(float) * (size_t)P * QN);
  float* x2 = (float*)malloc(sizeof(float) * (size_t)P * H);
  float scale = 1.0f / sqrtf((float)HD);
  memset(Kout, 0, sizeof(uint16_t) * (size_t)m->L * NKV * HD * S);
  memset(Vout, 0, sizeof(uint16_t) * (size_t)m->L * NKV * S * HD);
  for (int c = 0; c < P; c++)
    for (int i = 0; i < H; i++) x[(size_t)c * H + i] = bf2f(m->embed[(size_t)toks[c] * H + i]);
  for (int l = 0; l < m->L; l++) {
    rmsnorm_rows(x, P, H, m->eps, h);
    gemv(m->w[l * NKIND + K_Q], QN, H, h, P, q);
    gemv(m->w[l * NKIND + K_K], KN, H, h, P, k);
    gemv(m->w[l * NKIND + K_V], KN, H, h, P, v);
    for (int c = 0; c < P; c++) {
      rope(q + (size_t)c * QN, NH, HD, c, m->inv);
      rope(k + (size_t)c * KN, NKV, HD, c, m->inv);
      for (int i = 0; i < KN; i++) {   /* the cache is bf16: attention reads the rounded values */
        k[(size_t)c * KN + i] = bf2f(f2bf(k[(size_t)c * KN + i]));
        v[(size_t)c * KN + i] = bf2f(f2bf(v[(size_t)c * KN + i]));
      }
      for (int kh = 0; kh < NKV; kh++)
        for (int d = 0; d < HD; d++) {
          Kout[(((size_t)l * NKV + kh) * HD + d) * S + c] = f2bf(k[(size_t)c * KN + kh * HD + d]);
          Vout[(((size_t)l * NKV + kh) * S + c) * HD + d] = f2bf(v[(size_t)c * KN + kh * HD + d]);
        }
    }
#pragma omp parallel for collapse(2) schedule(dynamic, 4)
    for (int hh = 0; hh < NH; hh++)
      for (int c = 0; c < P; c++) {
        int kh = hh / G;
        const float* qh = q + (size_t)c * QN + (size_t)hh * HD;
        float* sc = (float*)malloc(sizeof(float) * (size_t)(c + 1));
        float mx = -INFINITY;
        for (int s = 0; s <= c; s++) {
          const float* ks = k + (size_t)s * KN + (size_t)kh * HD;
          float acc = 0.f;
          for (int d = 0; d < HD; d++) acc += qh[d] * ks[d];
          sc[s] = acc * scale;
          if (sc[s] > mx) mx = sc[s];
        }
        float sum = 0.f;
        for (int s = 0; s <= c; s++) { sc[s] = expf(sc[s] - mx); sum += sc[s]; }
        float* o = ao + (size_t)c * QN + (size_t)hh * HD;
        for (int d = 0; d < HD; d++) o[d] = 0.f;
        for (int s = 0; s <= c; s++) {
          float p = sc[s] / sum;
          const float* vs = v + (size_t)s * KN + (size_t)kh * HD;
          for (int d = 0; d < HD; d++) o[d] += p * vs[d];
        }
        free(sc);
      }
    gemv(m->w[l * NKIND + K_O], H, QN, ao, P, x2);
    for (size_t i = 0; i < (size_t)P * H; i++) x2[i] += x[i];
    mlp(m, l, x2, P, x);
  }
  if (hidden) memcpy(hidden, x, sizeof(float) * (size_t)P * H);
  float* lg = logits ? logits : (float*)malloc(sizeof(float) * (size_t)m->V);
  logits_rows(m, x + (size_t)(P - 1) * H, 1, lg);
  if (next) *next = argmax_first(lg, m->V);
  if (!logits) free(lg);
  free(x); free(h); free(q); free(k); free(v); free(ao); free(x2);
}

/* Seeded past KV of one request written into lane b of a decode cache
 * [L][B][NKV][S][HD]: positions < len drawn ~N(0, sigma) in [L][NKV][S][HD] order
 * (tids 0x8000 / 0x8001, the request's own seed), the tail zeroed. */
void orc_kv_fill_lane(uint16_t* Kc, uint16_t* Vc, int L, int B, int NKV, int S, int HD, int b,
                      uint64_t seed, int len, float scale) {
  uint64_t kk = stream_key(seed, T_KCACHE), vk = stream_key(seed, T_VCACHE);
#pragma omp parallel for collapse(2) schedule(static)
  for (int l = 0; l < L; l++)
    for (int kh = 0; kh < NKV; kh++)
      for (int s = 0; s < S; s++) {
        size_t dst = ((((size_t)l * B + b) * NKV + kh) * S + s) * HD;
        uint64_t src = (((uint64_t)l * NKV + kh) * S + s) * HD;
        for (int d = 0; d < HD; d++) {
          Kc[dst + d] = s < len ? gauss_one(kk, src + d, scale) : 0;
          Vc[dst + d] = s < len ? gauss_one(vk, src + d, scale) : 0;
        }
      }
}
