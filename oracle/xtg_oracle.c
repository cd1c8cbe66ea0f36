// TEST INFRASTRUCTURE ONLY: CPU restatement of the Dory verify step (see xtg_oracle.h for what is pinned and what
// is not). Every function names the reference code it restates. Built with -ffp-contract=off so that products and
// sums round one at a time, as the device generators do.
#include "xtg_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

// ---------------------------------------------------------------------------------------------------------------
// Number formats
// ---------------------------------------------------------------------------------------------------------------

// E4M3 (float8_e4m3fn) decode: bias 7, subnormals in steps of 2^-9, 0x7f / 0xff NaN (engine/src/fp.cpp:12-26).
float xo_e4m3_to_f32(uint8_t b) {
  const int e = (b >> 3) & 15, m = b & 7;
  float mag;
  if ((b & 0x7f) == 0x7f)
    mag = NAN;
  else if (e == 0)
    mag = ldexpf((float)m, -9);
  else
    mag = ldexpf((float)(8 + m), e - 10);
  return (b & 0x80) ? -mag : mag;
}

// FP32 -> E4M3, round to nearest even, saturating to 448 (engine/src/fp.cpp:30-49 and kv.cpp:20-40 give the same
// codes). Restated with frexp / rint instead of a table search or mantissa arithmetic.
uint8_t xo_f32_to_e4m3(float f) {
  const uint8_t sign = signbit(f) ? 0x80 : 0;
  if (isnan(f)) return (uint8_t)(sign | 0x7f);
  const float a = fabsf(f);
  if (a >= 448.f) return (uint8_t)(sign | 0x7e);
  if (a < 0x1p-6f) {   // subnormal: multiples of 2^-9 (8 * 2^-9 = 2^-6 is the first normal code, 0x08)
    return (uint8_t)(sign | (int)rintf(a * 512.f));
  }
  int e2;
  const float fr = frexpf(a, &e2);           // a = fr * 2^e2, fr in [0.5, 1)
  int mant = (int)rintf(ldexpf(fr, 4));      // 8 .. 16: the implicit bit and 3 mantissa bits
  int exp = e2 - 1 + 7;
  if (mant == 16) {
    mant = 8;
    ++exp;
  }
  int code = (exp << 3) | (mant - 8);
  if (code > 0x7e) code = 0x7e;
  return (uint8_t)(sign | code);
}

// FP32 -> BF16, round to nearest even, NaN kept quiet (engine/include/xtg/fp.h:18-24).
uint16_t xo_f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
  const uint32_t keep = (u >> 16) & 1u;
  return (uint16_t)((u + 0x7fffu + keep) >> 16);
}

float xo_bf16_to_f32(uint16_t h) {
  const uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

// E2M1 (engine/include/xtg/fp.h:36-39): bit 3 sign, magnitudes 0, 0.5, 1, 1.5, 2, 3, 4, 6.
float xo_e2m1_to_f32(uint8_t n) {
  static const float mag[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  const float v = mag[n & 7];
  return (n & 8) ? -v : v;
}

// ---------------------------------------------------------------------------------------------------------------
// Seeded generators (no reference counterpart). SplitMix64's finalizer over (seed, stream, index); normals are an
// Irwin-Hall sum of four 16-bit uniforms scaled to unit variance, so that every operation is exact or one IEEE
// rounding and the device generator reproduces the same bits.
// ---------------------------------------------------------------------------------------------------------------

static uint64_t mix64(uint64_t z) {
  z ^= z >> 30;
  z *= 0xbf58476d1ce4e5b9ull;
  z ^= z >> 27;
  z *= 0x94d049bb133111ebull;
  z ^= z >> 31;
  return z;
}

uint64_t xo_rand_bits(uint64_t seed, uint64_t stream, uint64_t index) {
  const uint64_t key = mix64(seed + 0x9e3779b97f4a7c15ull * (stream + 1));
  return mix64(key + 0x9e3779b97f4a7c15ull * (index + 1));
}

static float normal_from_bits(uint64_t b) {
  float s = 0.f;
  for (int j = 0; j < 4; ++j) s += (float)((b >> (16 * j)) & 0xffff) + 0.5f;   // exact: < 2^19
  const float c = s * (1.f / 65536.f) - 2.f;                                     // exact
  return c * 1.7320508f;                                                         // one rounding
}

void xo_gen_normal_bf16(uint64_t seed, uint64_t stream, float stddev, uint16_t* out, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const float z = normal_from_bits(xo_rand_bits(seed, stream, (uint64_t)i));
    out[i] = xo_f32_to_bf16(z * stddev);
  }
}

void xo_gen_uniform(uint64_t seed, uint64_t stream, float lo, float hi, float* out, int64_t n) {
  const float span = hi - lo;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const float u = (float)(xo_rand_bits(seed, stream, (uint64_t)i) >> 40) * 0x1p-24f;   // exact
    const float p = span * u;
    out[i] = lo + p;
  }
}

void xo_gen_int8(uint64_t seed, uint64_t stream, int8_t* out, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = (int8_t)((int)(xo_rand_bits(seed, stream, (uint64_t)i) % 255u) - 127);
}

// ---------------------------------------------------------------------------------------------------------------
// NVFP4
// ---------------------------------------------------------------------------------------------------------------

// Nearest E2M1 magnitude code, ties to the even code; above 6 saturates to code 7.
static uint8_t e2m1_code(float q) {
  const float a = fabsf(q);
  int c = (a > 0.25f) + (a >= 0.75f) + (a > 1.25f) + (a >= 1.75f) + (a > 2.5f) + (a >= 3.5f) + (a > 5.f);
  if (q < 0.f) c |= 8;
  return (uint8_t)c;
}

void xo_quantize_nvfp4(const uint16_t* w, int n_out, int k, uint8_t* codes, uint8_t* scales, float* global_out) {
  float amax = 0.f;
  for (int64_t i = 0; i < (int64_t)n_out * k; ++i) {
    const float a = fabsf(xo_bf16_to_f32(w[i]));
    if (a > amax) amax = a;
  }
  float global = amax / 2688.f;   // 6 * 448
  if (global == 0.f) global = 1.f;
  *global_out = global;
  const float six_g = 6.f * global;
  const int groups = k / 16;
#pragma omp parallel for schedule(static)
  for (int n = 0; n < n_out; ++n) {
    for (int g = 0; g < groups; ++g) {
      const uint16_t* src = w + (int64_t)n * k + g * 16;
      float bmax = 0.f;
      for (int j = 0; j < 16; ++j) {
        const float a = fabsf(xo_bf16_to_f32(src[j]));
        if (a > bmax) bmax = a;
      }
      float sc = bmax / six_g;
      if (sc == 0.f) sc = 1.f;
      const uint8_t sc_code = xo_f32_to_e4m3(sc);
      scales[(int64_t)n * groups + g] = sc_code;
      const float denom = xo_e4m3_to_f32(sc_code) * global;
      uint8_t* dst = codes + (int64_t)n * (k / 2) + g * 8;
      for (int j = 0; j < 8; ++j) {
        const uint8_t lo = e2m1_code(xo_bf16_to_f32(src[2 * j]) / denom);
        const uint8_t hi = e2m1_code(xo_bf16_to_f32(src[2 * j + 1]) / denom);
        dst[j] = (uint8_t)(lo | (hi << 4));
      }
    }
  }
}

// engine/src/kernels.cpp:34-45
void xo_nvfp4_row(const xo_nvfp4* w, int row, float* out) {
  const uint8_t* c = w->codes + (int64_t)row * (w->k / 2);
  const uint8_t* s = w->scales + (int64_t)row * (w->k / 16);
  for (int g = 0; g < w->k / 16; ++g) {
    const float sc = xo_e4m3_to_f32(s[g]) * w->global;
    for (int j = 0; j < 8; ++j) {
      out[g * 16 + 2 * j] = xo_e2m1_to_f32(c[g * 8 + j] & 15) * sc;
      out[g * 16 + 2 * j + 1] = xo_e2m1_to_f32(c[g * 8 + j] >> 4) * sc;
    }
  }
}

// One output: per 16-input group the E2M1 products are summed, then scaled; the sum over groups is scaled by the
// global (the order of engine/src/kernels.cpp:48-60).
static float nvfp4_dot(const xo_nvfp4* w, int n, const float* x) {
  const uint8_t* c = w->codes + (int64_t)n * (w->k / 2);
  const uint8_t* s = w->scales + (int64_t)n * (w->k / 16);
  float acc = 0.f;
  for (int g = 0; g < w->k / 16; ++g) {
    float part = 0.f;
    for (int j = 0; j < 8; ++j) {
      const uint8_t b = c[g * 8 + j];
      part += xo_e2m1_to_f32(b & 15) * x[g * 16 + 2 * j];
      part += xo_e2m1_to_f32(b >> 4) * x[g * 16 + 2 * j + 1];
    }
    acc += part * xo_e4m3_to_f32(s[g]);
  }
  return acc * w->global;
}

void xo_matmul_nvfp4(const xo_nvfp4* ws, int nw, const float* x, int m, float* const* ys) {
  int64_t total = 0;
  for (int i = 0; i < nw; ++i) total += ws[i].n_out;
#pragma omp parallel for schedule(dynamic, 16)
  for (int64_t r = 0; r < total; ++r) {
    int wi = 0;
    int64_t n = r;
    while (n >= ws[wi].n_out) n -= ws[wi++].n_out;
    for (int i = 0; i < m; ++i)
      ys[wi][(int64_t)i * ws[wi].n_out + n] = nvfp4_dot(&ws[wi], (int)n, x + (int64_t)i * ws[wi].k);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Elementwise (engine/src/kernels.cpp:162-234)
// ---------------------------------------------------------------------------------------------------------------

static float inv_norm(const float* x, int w) {
  float s = 0.f;
  for (int j = 0; j < w; ++j) s += x[j] * x[j];
  return 1.f / sqrtf(s + 1e-6f);
}

void xo_justnorm(float* x, int rows, int width) {
  for (int r = 0; r < rows; ++r) {
    float* v = x + (int64_t)r * width;
    const float f = inv_norm(v, width);
    for (int j = 0; j < width; ++j) v[j] *= f;
  }
}

void xo_slerp_residual(float* a, const float* b, const float* lr, int rows, int width) {
  for (int r = 0; r < rows; ++r) {
    float* va = a + (int64_t)r * width;
    const float* vb = b + (int64_t)r * width;
    const float fa = inv_norm(va, width), fb = inv_norm(vb, width);
    for (int j = 0; j < width; ++j) {
      const float ya = va[j] * fa, yb = vb[j] * fb;
      va[j] = ya + lr[j] * (yb - ya);
    }
    const float f = inv_norm(va, width);
    for (int j = 0; j < width; ++j) va[j] *= f;
  }
}

// NeoX rotation with vLLM's table: inv_freq = 1 / theta^(2i/d) in FP32, angle = FP32(pos) * inv_freq.
void xo_rope(float* x, int rows, int heads, int head_dim, int64_t pos0, float theta) {
  const int half = head_dim / 2;
  float* cs = (float*)malloc(sizeof(float) * (size_t)head_dim);
  for (int r = 0; r < rows; ++r) {
    const float pos = (float)(pos0 + r);
    for (int i = 0; i < half; ++i) {
      const float inv = 1.f / powf(theta, (float)(2 * i) / (float)head_dim);
      const float ang = pos * inv;
      cs[i] = cosf(ang);
      cs[half + i] = sinf(ang);
    }
    for (int h = 0; h < heads; ++h) {
      float* v = x + ((int64_t)r * heads + h) * head_dim;
      for (int i = 0; i < half; ++i) {
        const float x1 = v[i], x2 = v[i + half];
        v[i] = x1 * cs[i] - x2 * cs[half + i];
        v[i + half] = x2 * cs[i] + x1 * cs[half + i];
      }
    }
  }
  free(cs);
}

void xo_swiglu_scaled(float* g, const float* u, const float* sg, const float* su, int rows, int width) {
  for (int r = 0; r < rows; ++r)
    for (int j = 0; j < width; ++j) {
      const int64_t i = (int64_t)r * width + j;
      const float z = g[i] * sg[j];
      g[i] = z / (1.f + expf(-z)) * (u[i] * su[j]);
    }
}

// ---------------------------------------------------------------------------------------------------------------
// KV
// ---------------------------------------------------------------------------------------------------------------

void xo_kv_encode(int dtype, const float* x, int d, uint8_t* codes, float* scale) {
  float amax = 0.f;
  for (int j = 0; j < d; ++j)
    if (fabsf(x[j]) > amax) amax = fabsf(x[j]);
  const float top = dtype == XO_KV_FP8 ? 448.f : 127.f;
  const float s = amax > 0.f ? amax / top : 1.f;
  const float inv = 1.f / s;
  for (int j = 0; j < d; ++j) {
    const float t = x[j] * inv;
    if (dtype == XO_KV_FP8) {
      codes[j] = xo_f32_to_e4m3(t);
    } else {
      float r = rintf(t);
      if (r > 127.f) r = 127.f;
      if (r < -127.f) r = -127.f;
      codes[j] = (uint8_t)(int8_t)r;
    }
  }
  *scale = s;
}

float xo_kv_decode(int dtype, uint8_t code, float scale) {
  return (dtype == XO_KV_FP8 ? xo_e4m3_to_f32(code) : (float)(int8_t)code) * scale;
}

// ---------------------------------------------------------------------------------------------------------------
// Attention
// ---------------------------------------------------------------------------------------------------------------

enum { TILE = 64 };

typedef struct {
  float m, l;
} online_t;

// Fold a tile of `n` scores (already scaled) and their value rows into (st, acc): the reference's update
// (engine/src/kv.cpp:219-242).
static void fold_tile(online_t* st, float* acc, int d, const float* sc, const float* vals, int n) {
  if (n == 0) return;
  float mx = -INFINITY;
  for (int j = 0; j < n; ++j)
    if (sc[j] > mx) mx = sc[j];
  const float m_new = st->m > mx ? st->m : mx;
  const float corr = st->m == -INFINITY ? 0.f : expf(st->m - m_new);
  if (corr != 1.f)
    for (int e = 0; e < d; ++e) acc[e] *= corr;
  st->l *= corr;
  for (int j = 0; j < n; ++j) {
    const float w = expf(sc[j] - m_new);
    st->l += w;
    const float* vv = vals + (int64_t)j * d;
    for (int e = 0; e < d; ++e) acc[e] += w * vv[e];
  }
  st->m = m_new;
}

void xo_attention(const xo_attn* a) {
  const int group = a->heads / a->kv_heads, d = a->head_dim;
  const xo_cache* c = a->cache;
#pragma omp parallel for schedule(dynamic, 1)
  for (int pair = 0; pair < a->n_q * a->heads; ++pair) {
    const int i = pair / a->heads, h = pair % a->heads, kh = h / group;
    const int64_t t = a->pos0 + i;
    const float* q = a->q + ((int64_t)i * a->heads + h) * d;
    float* kt = (float*)malloc(sizeof(float) * TILE * d);
    float* vt = (float*)malloc(sizeof(float) * TILE * d);
    float* acc = (float*)calloc((size_t)d, sizeof(float));
    float sc[TILE];
    online_t st = {-INFINITY, 0.f};
    int n = 0;
    // cached keys: slots in order, a global cache's slot is its position
    for (int64_t s = 0; s < c->slots; ++s) {
      const int64_t p = c->ring ? a->ring_pos[s] : s;
      if (p < 0 || p >= a->pos0) continue;
      if (a->window > 0 && t - p >= a->window) continue;
      const int64_t idx = s * a->kv_heads + kh;
      const uint8_t* kc = c->k + idx * d;
      const uint8_t* vc = c->v + idx * d;
      float dot = 0.f;
      for (int e = 0; e < d; ++e) {
        kt[(int64_t)n * d + e] = xo_kv_decode(c->dtype, kc[e], c->ks[idx]);
        vt[(int64_t)n * d + e] = xo_kv_decode(c->dtype, vc[e], c->vs[idx]);
      }
      for (int e = 0; e < d; ++e) dot += q[e] * kt[(int64_t)n * d + e];
      sc[n++] = dot * a->scale;
      if (n == TILE) {
        fold_tile(&st, acc, d, sc, vt, n);
        n = 0;
      }
    }
    fold_tile(&st, acc, d, sc, vt, n);
    n = 0;
    // this call's own keys
    for (int j = 0; j <= i; ++j) {
      if (a->window > 0 && i - j >= a->window) continue;
      const float* kr = a->k + ((int64_t)j * a->kv_heads + kh) * d;
      const float* vr = a->v + ((int64_t)j * a->kv_heads + kh) * d;
      float dot = 0.f;
      for (int e = 0; e < d; ++e) dot += q[e] * kr[e];
      memcpy(vt + (int64_t)n * d, vr, sizeof(float) * (size_t)d);
      sc[n++] = dot * a->scale;
      if (n == TILE) {   // a prompt chunk of more than a tile of own keys: folded tile by tile as well
        fold_tile(&st, acc, d, sc, vt, n);
        n = 0;
      }
    }
    fold_tile(&st, acc, d, sc, vt, n);
    float* o = a->out + ((int64_t)i * a->heads + h) * d;
    const float inv = st.l > 0.f ? 1.f / st.l : 0.f;
    for (int e = 0; e < d; ++e) o[e] = acc[e] * inv;
    free(kt);
    free(vt);
    free(acc);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Ring / masks / rewind (npu/xtg_npu.cpp:236-258, 362-369)
// ---------------------------------------------------------------------------------------------------------------

void xo_fill_masks(int ar, int rows, int64_t n_past, int ctx, int ring, int window, const int64_t* ring_pos,
                   uint8_t* mask, uint8_t* wmask) {
  const int mc = ctx + ar, wc = ring + ar;
  memset(mask, 0, (size_t)ar * mc);
  memset(wmask, 0, (size_t)ar * wc);
  for (int i = 0; i < ar; ++i) {
    uint8_t* mr = mask + (int64_t)i * mc;
    uint8_t* wr = wmask + (int64_t)i * wc;
    if (i >= rows) {
      mr[ctx + i] = 1;
      wr[ring + i] = 1;
      continue;
    }
    const int64_t p = n_past + i;
    for (int64_t s = 0; s < n_past && s < ctx; ++s) mr[s] = 1;
    for (int j = 0; j <= i; ++j) mr[ctx + j] = 1;
    for (int s = 0; s < ring; ++s) {
      const int64_t q = ring_pos[s];
      if (q >= 0 && q < n_past && p - q < window) wr[s] = 1;
    }
    for (int j = i - window + 1 > 0 ? i - window + 1 : 0; j <= i; ++j) wr[ring + j] = 1;
  }
}

int xo_rewind_ok(int64_t to, int64_t n_past, int window, int ring, const int64_t* ring_pos) {
  if (to < 0 || to > n_past) return 0;
  for (int64_t q = to - window + 1 > 0 ? to - window + 1 : 0; q < to; ++q)
    if (ring_pos[q % ring] != q) return 0;
  return 1;
}

// ---------------------------------------------------------------------------------------------------------------
// The step (packs/dory/dory.cpp:467-544)
// ---------------------------------------------------------------------------------------------------------------

int64_t xo_step_work_floats(const xo_model* M, int m) {
  const int64_t H = M->hidden, F = M->ffn, Q = (int64_t)M->heads * M->head_dim, KV = (int64_t)M->kv_heads * M->head_dim;
  return (int64_t)m * (4 * H + 3 * Q + 2 * KV + 2 * F) + 2 * (int64_t)M->head_dim;
}

typedef struct {
  float *x, *input, *state, *q, *k, *v, *g, *att, *o, *mg, *mu;
} bufs_t;

static void sublayer(const xo_model* M, xo_state* S, const xo_layer* L, bufs_t* b, int m) {
  const int H = M->hidden, F = M->ffn, Q = M->heads * M->head_dim, KV = M->kv_heads * M->head_dim, d = M->head_dim;
  const int64_t pos0 = S->n_past;
  if (L->kind == 0) {
    float* ys[2] = {b->mg, b->mu};
    xo_matmul_nvfp4(L->w, 2, b->x, m, ys);
    xo_swiglu_scaled(b->mg, b->mu, L->sg, L->su, m, F);
    xo_justnorm(b->mg, m, F);
    float* yo[1] = {b->o};
    xo_matmul_nvfp4(&L->w[2], 1, b->mg, m, yo);
    xo_slerp_residual(b->x, b->o, L->lr, m, H);
    return;
  }
  float* ys[4] = {b->q, b->k, b->v, b->g};
  xo_matmul_nvfp4(L->w, 4, b->x, m, ys);
  xo_rope(b->q, m, M->heads, d, pos0, L->theta);
  xo_rope(b->k, m, M->kv_heads, d, pos0, L->theta);
  xo_justnorm(b->q, m * M->heads, d);
  for (int r = 0; r < m; ++r)
    for (int j = 0; j < Q; ++j) b->q[(int64_t)r * Q + j] *= L->qscale[j];
  xo_justnorm(b->k, m * M->kv_heads, d);
  xo_cache* c = &S->caches[L->cache];
  xo_attn a;
  a.n_q = m;
  a.pos0 = pos0;
  a.heads = M->heads;
  a.kv_heads = M->kv_heads;
  a.head_dim = d;
  a.window = L->kind == 1 ? M->window : 0;
  a.scale = 1.f / sqrtf((float)d);
  a.q = b->q;
  a.k = b->k;
  a.v = b->v;
  a.cache = c;
  a.ring_pos = S->ring_pos;
  a.out = b->att;
  xo_attention(&a);
  // the new rows into the cache (a ring slot is position % slots)
  for (int r = 0; r < m; ++r) {
    const int64_t p = pos0 + r, slot = c->ring ? p % c->slots : p;
    for (int h = 0; h < M->kv_heads; ++h) {
      const int64_t idx = slot * M->kv_heads + h;
      xo_kv_encode(c->dtype, b->k + ((int64_t)r * M->kv_heads + h) * d, d, c->k + idx * d, &c->ks[idx]);
      xo_kv_encode(c->dtype, b->v + ((int64_t)r * M->kv_heads + h) * d, d, c->v + idx * d, &c->vs[idx]);
    }
  }
  (void)KV;
  for (int r = 0; r < m; ++r)
    for (int j = 0; j < Q; ++j) {
      const int64_t i = (int64_t)r * Q + j;
      b->att[i] *= 1.f / (1.f + expf(-b->g[i] * L->gscale[j]));
    }
  xo_justnorm(b->att, m, Q);
  float* yo[1] = {b->o};
  xo_matmul_nvfp4(&L->w[4], 1, b->att, m, yo);
  xo_slerp_residual(b->x, b->o, L->lr, m, H);
}

void xo_step(const xo_model* M, xo_state* S, const int32_t* tokens, int m, float* logits, float* work) {
  const int H = M->hidden, F = M->ffn, Q = M->heads * M->head_dim, KV = M->kv_heads * M->head_dim;
  bufs_t b;
  float* p = work;
  b.x = p;      p += (int64_t)m * H;
  b.input = p;  p += (int64_t)m * H;
  b.state = p;  p += (int64_t)m * H;
  b.o = p;      p += (int64_t)m * H;
  b.q = p;      p += (int64_t)m * Q;
  b.g = p;      p += (int64_t)m * Q;
  b.att = p;    p += (int64_t)m * Q;
  b.k = p;      p += (int64_t)m * KV;
  b.v = p;      p += (int64_t)m * KV;
  b.mg = p;     p += (int64_t)m * F;
  b.mu = p;
  const int64_t n = (int64_t)m * H;
  for (int r = 0; r < m; ++r) {
    float* xr = b.x + (int64_t)r * H;
    if (M->embed_bf16) {   // bf16_row (engine/src/kernels.cpp:157-160)
      for (int j = 0; j < H; ++j) xr[j] = xo_bf16_to_f32(M->embed_bf16[(int64_t)tokens[r] * H + j]);
    } else {
      xo_nvfp4_row(&M->head, tokens[r], xr);
    }
  }
  int e = 0;
  for (int l = 0; l < M->n_in; ++l) sublayer(M, S, &M->layers[e++], &b, m);
  memcpy(b.input, b.x, sizeof(float) * (size_t)n);
  memcpy(b.state, b.x, sizeof(float) * (size_t)n);
  for (int i = 0; i < M->loops; ++i) {
    for (int64_t j = 0; j < n; ++j) b.x[j] = b.state[j] + b.input[j];
    xo_justnorm(b.x, m, H);
    for (int l = 0; l < M->n_rec; ++l) sublayer(M, S, &M->layers[e++], &b, m);
    memcpy(b.state, b.x, sizeof(float) * (size_t)n);
    xo_justnorm(b.state, m, H);
  }
  memcpy(b.x, b.state, sizeof(float) * (size_t)n);
  for (int l = 0; l < M->n_out; ++l) sublayer(M, S, &M->layers[e++], &b, m);
  if (M->head_bf16) {   // matmul_bf16 (engine/src/kernels.cpp:140-155): row n's f32 weights dotted with each row
    for (int n = 0; n < M->vocab; ++n) {
      const uint16_t* w = M->head_bf16 + (int64_t)n * H;
      for (int r = 0; r < m; ++r) {
        const float* xr = b.x + (int64_t)r * H;
        float acc = 0.f;
        for (int j = 0; j < H; ++j) acc += xo_bf16_to_f32(w[j]) * xr[j];
        logits[(int64_t)r * M->vocab + n] = acc;
      }
    }
  } else {
    float* yl[1] = {logits};
    xo_matmul_nvfp4(&M->head, 1, b.x, m, yl);
  }
  for (int r = 0; r < m; ++r)
    for (int j = 0; j < M->vocab; ++j) logits[(int64_t)r * M->vocab + j] *= M->logit_scale[j];
  for (int r = 0; r < m; ++r) S->ring_pos[(S->n_past + r) % S->ring] = S->n_past + r;
  S->n_past += m;
}

int xo_argmax(const float* x, int n) {
  int best = 0;
  for (int i = 1; i < n; ++i)
    if (x[i] > x[best]) best = i;
  return best;
}

// ---------------------------------------------------------------------------------------------------------------
// The seeded synthetic model and state (see xtg_oracle.h for the stream map)
// ---------------------------------------------------------------------------------------------------------------

int xo_synth_n_evals(const xo_synth_cfg* c) { return c->n_in + c->n_rec * c->loops + c->n_out; }

static int synth_phys(const xo_synth_cfg* c, int e) {
  if (e < c->n_in) return e;
  e -= c->n_in;
  if (e < c->n_rec * c->loops) return c->n_in + e % c->n_rec;
  return c->n_in + c->n_rec + (e - c->n_rec * c->loops);
}

int xo_synth_kind(const xo_synth_cfg* c, int e) {
  const int l = synth_phys(c, e);
  if (l % 2) return 0;
  const int a = l / 2;
  return (c->global_every > 0 && a % c->global_every == c->global_every - 1) ? 2 : 1;
}

static void synth_weight(const xo_synth_cfg* c, uint64_t stream, int n_out, int k, xo_nvfp4* w) {
  uint16_t* raw = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)n_out * (size_t)k);
  uint8_t* codes = (uint8_t*)malloc((size_t)n_out * (size_t)(k / 2));
  uint8_t* scales = (uint8_t*)malloc((size_t)n_out * (size_t)(k / 16));
  xo_gen_normal_bf16(c->seed, stream, c->weight_std, raw, (int64_t)n_out * k);
  float g;
  xo_quantize_nvfp4(raw, n_out, k, codes, scales, &g);
  free(raw);
  w->codes = codes;
  w->scales = scales;
  w->global = g;
  w->n_out = n_out;
  w->k = k;
}

static float* synth_vec(const xo_synth_cfg* c, uint64_t stream, float lo, float hi, int n) {
  float* v = (float*)malloc(sizeof(float) * (size_t)n);
  xo_gen_uniform(c->seed, stream, lo, hi, v, n);
  return v;
}

xo_model* xo_synth_model_new(const xo_synth_cfg* c) {
  const int H = c->hidden, F = c->ffn, Q = c->heads * c->head_dim, KV = c->kv_heads * c->head_dim;
  const int ne = xo_synth_n_evals(c);
  xo_model* m = (xo_model*)calloc(1, sizeof(xo_model));
  xo_layer* L = (xo_layer*)calloc((size_t)ne, sizeof(xo_layer));
  m->hidden = H;
  m->ffn = F;
  m->heads = c->heads;
  m->kv_heads = c->kv_heads;
  m->head_dim = c->head_dim;
  m->vocab = c->vocab;
  m->window = c->window;
  m->n_in = c->n_in;
  m->n_rec = c->n_rec;
  m->n_out = c->n_out;
  m->loops = c->loops;
  m->layers = L;
  int n_attn = 0;
  for (int e = 0; e < ne; ++e) {
    const uint64_t base = 1000 + 16 * (uint64_t)e;
    L[e].kind = xo_synth_kind(c, e);
    L[e].lr = synth_vec(c, base + 8, c->lr_lo, c->lr_hi, H);
    if (L[e].kind == 0) {
      synth_weight(c, base + 0, F, H, &L[e].w[0]);
      synth_weight(c, base + 1, F, H, &L[e].w[1]);
      synth_weight(c, base + 2, H, F, &L[e].w[2]);
      L[e].sg = synth_vec(c, base + 11, c->suv_lo, c->suv_hi, F);
      L[e].su = synth_vec(c, base + 12, c->suv_lo, c->suv_hi, F);
    } else {
      synth_weight(c, base + 0, Q, H, &L[e].w[0]);
      synth_weight(c, base + 1, KV, H, &L[e].w[1]);
      synth_weight(c, base + 2, KV, H, &L[e].w[2]);
      synth_weight(c, base + 3, Q, H, &L[e].w[3]);
      synth_weight(c, base + 4, H, Q, &L[e].w[4]);
      L[e].qscale = synth_vec(c, base + 9, c->qs_lo, c->qs_hi, Q);
      L[e].gscale = synth_vec(c, base + 10, c->gs_lo, c->gs_hi, Q);
      L[e].theta = L[e].kind == 2 ? c->theta_global : c->theta_sliding;
      L[e].cache = n_attn++;
    }
  }
  synth_weight(c, 1, c->vocab, H, &m->head);
  m->logit_scale = synth_vec(c, 2, c->ls_lo, c->ls_hi, c->vocab);
  return m;
}

static void free_w(xo_nvfp4* w) {
  free((void*)w->codes);
  free((void*)w->scales);
}

void xo_synth_model_free(xo_model* m) {
  const int ne = m->n_in + m->n_rec * m->loops + m->n_out;
  xo_layer* L = (xo_layer*)m->layers;
  for (int e = 0; e < ne; ++e) {
    for (int j = 0; j < 5; ++j)
      if (L[e].w[j].codes) free_w(&L[e].w[j]);
    free((void*)L[e].lr);
    free((void*)L[e].qscale);
    free((void*)L[e].gscale);
    free((void*)L[e].sg);
    free((void*)L[e].su);
  }
  free(L);
  free_w(&m->head);
  free((void*)m->logit_scale);
  free(m);
}

xo_state* xo_synth_state_new(const xo_model* m, const xo_synth_cfg* c, int64_t ctx, int kv_dtype, int64_t n_prefill) {
  const int ne = xo_synth_n_evals(c), d = c->head_dim, kvh = c->kv_heads;
  int n_attn = 0;
  for (int e = 0; e < ne; ++e) n_attn += m->layers[e].kind != 0;
  xo_state* s = (xo_state*)calloc(1, sizeof(xo_state));
  s->caches = (xo_cache*)calloc((size_t)n_attn, sizeof(xo_cache));
  s->n_caches = n_attn;
  s->ring = c->ring;
  s->ring_pos = (int64_t*)malloc(sizeof(int64_t) * (size_t)c->ring);
  for (int r = 0; r < c->ring; ++r) {
    // the largest prefilled position held by slot r
    int64_t p = -1;
    if (n_prefill > 0) {
      const int64_t last = n_prefill - 1;
      p = last - ((last - r) % c->ring + c->ring) % c->ring;
    }
    s->ring_pos[r] = p;
  }
  s->n_past = n_prefill;
  for (int e = 0; e < ne; ++e) {
    if (m->layers[e].kind == 0) continue;
    const int i = m->layers[e].cache;
    xo_cache* kc = &s->caches[i];
    kc->dtype = kv_dtype;
    kc->ring = m->layers[e].kind == 1;
    kc->slots = kc->ring ? c->ring : ctx;
    const int64_t rows = kc->slots * kvh;
    kc->k = (uint8_t*)calloc((size_t)(rows * d), 1);
    kc->v = (uint8_t*)calloc((size_t)(rows * d), 1);
    kc->ks = (float*)calloc((size_t)rows, sizeof(float));
    kc->vs = (float*)calloc((size_t)rows, sizeof(float));
    const uint64_t base = 500000 + 8 * (uint64_t)i;
    // filled slots: a ring's slots that hold a position, a global cache's first n_prefill
    const int64_t filled = kc->ring ? (n_prefill < kc->slots ? n_prefill : kc->slots) : n_prefill;
    if (filled > 0) {
      xo_gen_int8(c->seed, base + 0, (int8_t*)kc->k, filled * kvh * d);
      xo_gen_int8(c->seed, base + 1, (int8_t*)kc->v, filled * kvh * d);
      xo_gen_uniform(c->seed, base + 2, c->kvs_lo, c->kvs_hi, kc->ks, filled * kvh);
      xo_gen_uniform(c->seed, base + 3, c->kvs_lo, c->kvs_hi, kc->vs, filled * kvh);
    }
  }
  return s;
}

void xo_synth_state_free(xo_state* s) {
  for (int i = 0; i < s->n_caches; ++i) {
    free(s->caches[i].k);
    free(s->caches[i].v);
    free(s->caches[i].ks);
    free(s->caches[i].vs);
  }
  free(s->caches);
  free(s->ring_pos);
  free(s);
}
