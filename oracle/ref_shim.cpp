// TEST INFRASTRUCTURE ONLY (the checker, never the product): C entry points over XTier Go's own CPU kernels.
//
// oracle/Makefile compiles this file together with the reference's engine sources, unmodified and in place
// (engine/src/{kernels,fp,kv,threadpool,common,sampler}.cpp, and for whole checkpoints model.cpp, safetensors.cpp,
// opencl.cpp and packs/dory/{dory,npu}.cpp), into oracle/_ref/libxtgref.so. Tests call it through ctypes to
// pin the C restatement (xtg_oracle.c) against the reference's own arithmetic, and bench.py's reference arm times
// it as the reference's CPU implementation of the Dory verify step. Every function below forwards to the named
// reference function; the step harness at the end calls them in the order of DorySession::sublayer
// (packs/dory/dory.cpp:467-518) and DorySession::run_chunk (dory.cpp:520-544).
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <exception>
#include <limits>
#include <random>
#include <memory>
#include <mutex>
#include <vector>

#include "dory/dory.h"
#include "xtg/fp.h"
#include "xtg/kernels.h"
#include "xtg/kv.h"
#include "xtg/model.h"
#include "xtg/sampler.h"
#include "xtg/threadpool.h"

using namespace xtg;

namespace {
thread_local char g_err[512];

template <class F>
int guarded(F&& f) {
  try {
    f();
    return 0;
  } catch (const std::exception& e) {
    std::snprintf(g_err, sizeof(g_err), "%s", e.what());
    return -1;
  }
}
}  // namespace

extern "C" {

const char* xr_last_error() { return g_err; }

// ThreadPool (engine/include/xtg/threadpool.h:15-49)
void* xr_pool_new(int threads) { return new ThreadPool(threads); }
void xr_pool_free(void* p) { delete static_cast<ThreadPool*>(p); }
int xr_pool_size(void* p) { return static_cast<ThreadPool*>(p)->size(); }

// Number formats (engine/include/xtg/fp.h:10-41, engine/src/fp.cpp:30-49)
float xr_e4m3_to_f32(uint8_t b) { return e4m3_to_f32(b); }
uint8_t xr_f32_to_e4m3(float f) { return f32_to_e4m3(f); }
uint16_t xr_f32_to_bf16(float f) { return f32_to_bf16(f); }
float xr_bf16_to_f32(uint16_t h) { return bf16_to_f32(h); }

// nvfp4_row (engine/src/kernels.cpp:34-45)
void xr_nvfp4_row(const uint8_t* codes, const uint8_t* scales, float global, int n_out, int k, int row, float* out) {
  Nvfp4Weight w;
  w.codes = codes;
  w.scales = scales;
  w.global = global;
  w.n_out = n_out;
  w.k = k;
  nvfp4_row(w, row, out);
}

// matmul_nvfp4 over nw weights that read the same x (engine/src/kernels.cpp:84-138)
int xr_matmul_nvfp4(void* pool, int nw, const uint8_t* const* codes, const uint8_t* const* scales,
                    const float* globals, const int* n_out, int k, const float* x, int m, float* const* ys) {
  return guarded([&] {
    std::vector<Nvfp4Weight> ws(static_cast<size_t>(nw));
    std::vector<const Nvfp4Weight*> wp;
    std::vector<float*> yp;
    for (int i = 0; i < nw; ++i) {
      ws[size_t(i)].codes = codes[i];
      ws[size_t(i)].scales = scales[i];
      ws[size_t(i)].global = globals[i];
      ws[size_t(i)].n_out = n_out[i];
      ws[size_t(i)].k = k;
      wp.push_back(&ws[size_t(i)]);
      yp.push_back(ys[i]);
    }
    matmul_nvfp4(*static_cast<ThreadPool*>(pool), wp, x, m, yp);
  });
}

// justnorm / slerp_residual / rope / swiglu_scaled (engine/src/kernels.cpp:169-234)
void xr_justnorm(float* x, int rows, int width) { justnorm(x, rows, width); }
void xr_slerp_residual(float* a, const float* b, const float* lr, int rows, int width) {
  slerp_residual(a, b, lr, rows, width);
}
void xr_rope(float* x, int rows, int heads, int head_dim, int64_t pos0, float theta) {
  rope(x, rows, heads, head_dim, pos0, theta);
}
void xr_swiglu_scaled(float* g, const float* u, const float* sg, const float* su, int rows, int w) {
  swiglu_scaled(g, u, sg, su, rows, w);
}

// KvCache (engine/include/xtg/kv.h:21-62, engine/src/kv.cpp:42-149); fp8 = 0 keeps BF16 rows.
void* xr_kv_new(int kv_heads, int head_dim, int64_t slots, int ring, int fp8) {
  try {
    return new KvCache(kv_heads, head_dim, slots, ring, fp8 ? KvDtype::FP8 : KvDtype::BF16);
  } catch (const std::exception& e) {
    std::snprintf(g_err, sizeof(g_err), "%s", e.what());
    return nullptr;
  }
}
void xr_kv_free(void* c) { delete static_cast<KvCache*>(c); }
int xr_kv_store(void* c, int64_t pos, int n, const float* k, const float* v) {
  return guarded([&] { static_cast<KvCache*>(c)->store(pos, n, k, v); });
}
void xr_kv_load(void* c, int h, int64_t p0, int64_t p1, float* k, float* v) {
  static_cast<KvCache*>(c)->load(h, p0, p1, k, v);
}

// attention (engine/src/kv.cpp:166-286) with the arguments of AttnArgs (kv.h:67-78)
int xr_attention(void* pool, int n_q, int64_t pos0, int heads, int kv_heads, int head_dim, int window, float scale,
                 const float* q, const float* k, const float* v, const void* cache, float* out) {
  return guarded([&] {
    AttnArgs a;
    a.n_q = n_q;
    a.pos0 = pos0;
    a.heads = heads;
    a.kv_heads = kv_heads;
    a.head_dim = head_dim;
    a.window = window;
    a.scale = scale;
    a.q = q;
    a.k = k;
    a.v = v;
    a.cache = static_cast<const KvCache*>(cache);
    a.out = out;
    attention(*static_cast<ThreadPool*>(pool), a);
  });
}

// One Dory sublayer on m rows, in the order of DorySession::sublayer (packs/dory/dory.cpp:467-518), with the
// reference's kernels. Attention weights: q, k, v, g, o (5 NVFP4 weights); MLP weights: gate, up, down. Vectors are
// the folded ones (dory.cpp:326-364): lr; qscale, gscale (attention); sg, su (MLP). cache: an xr_kv_new cache; the
// new rows are stored after the attention, as the session does.
struct XrSublayer {
  int kind;   // 0 MLP, 1 sliding attention, 2 global attention
  const uint8_t* codes[5];
  const uint8_t* scales[5];
  float globals[5];
  const float* lr;
  const float* qscale;
  const float* gscale;
  const float* sg;
  const float* su;
  float theta;
  int window;
  void* cache;
};

struct XrShape {
  int hidden, ffn, heads, kv_heads, head_dim;
};

int xr_sublayer(void* pool_, const XrShape* c, const XrSublayer* L, float* x, int m, int64_t pos0, int store,
                float* work) {
  return guarded([&] {
    ThreadPool& pool = *static_cast<ThreadPool*>(pool_);
    const int H = c->hidden, F = c->ffn, Q = c->heads * c->head_dim, KV = c->kv_heads * c->head_dim;
    auto w = [&](int i, int n_out, int k) {
      Nvfp4Weight r;
      r.codes = L->codes[i];
      r.scales = L->scales[i];
      r.global = L->globals[i];
      r.n_out = n_out;
      r.k = k;
      return r;
    };
    if (L->kind == 0) {
      float* g = work;
      float* u = g + size_t(m) * F;
      float* o = u + size_t(m) * F;
      Nvfp4Weight wg = w(0, F, H), wu = w(1, F, H), wd = w(2, H, F);
      matmul_nvfp4(pool, {&wg, &wu}, x, m, {g, u});
      swiglu_scaled(g, u, L->sg, L->su, m, F);
      justnorm(g, m, F);
      matmul_nvfp4(pool, {&wd}, g, m, {o});
      slerp_residual(x, o, L->lr, m, H);
      return;
    }
    float* hq = work;
    float* hk = hq + size_t(m) * Q;
    float* hv = hk + size_t(m) * KV;
    float* hg = hv + size_t(m) * KV;
    float* ha = hg + size_t(m) * Q;
    float* ho = ha + size_t(m) * Q;
    Nvfp4Weight wq = w(0, Q, H), wk = w(1, KV, H), wv = w(2, KV, H), wgt = w(3, Q, H), wo = w(4, H, Q);
    matmul_nvfp4(pool, {&wq, &wk, &wv, &wgt}, x, m, {hq, hk, hv, hg});
    rope(hq, m, c->heads, c->head_dim, pos0, L->theta);
    rope(hk, m, c->kv_heads, c->head_dim, pos0, L->theta);
    justnorm(hq, m * c->heads, c->head_dim);
    for (int r = 0; r < m; ++r)
      for (int j = 0; j < Q; ++j) hq[size_t(r) * Q + j] *= L->qscale[j];
    justnorm(hk, m * c->kv_heads, c->head_dim);
    KvCache& cache = *static_cast<KvCache*>(L->cache);
    AttnArgs a;
    a.n_q = m;
    a.pos0 = pos0;
    a.heads = c->heads;
    a.kv_heads = c->kv_heads;
    a.head_dim = c->head_dim;
    a.window = L->window;
    a.scale = 1.f / std::sqrt(float(c->head_dim));
    a.q = hq;
    a.k = hk;
    a.v = hv;
    a.cache = &cache;
    a.out = ha;
    attention(pool, a);
    if (store) cache.store(pos0, m, hk, hv);
    for (int r = 0; r < m; ++r)
      for (int j = 0; j < Q; ++j) {
        float& e = ha[size_t(r) * Q + j];
        e *= 1.f / (1.f + std::exp(-hg[size_t(r) * Q + j] * L->gscale[j]));
      }
    justnorm(ha, m, Q);
    matmul_nvfp4(pool, {&wo}, ha, m, {ho});
    slerp_residual(x, ho, L->lr, m, H);
  });
}

// The NVFP4 head (a tied embedding): logits = x W^T, times the folded per-token logit scale (dory.cpp:566-576).
int xr_head(void* pool, const uint8_t* codes, const uint8_t* scales, float global, int vocab, int hidden,
            const float* x, int m, const float* logit_scale, float* logits) {
  return guarded([&] {
    Nvfp4Weight w;
    w.codes = codes;
    w.scales = scales;
    w.global = global;
    w.n_out = vocab;
    w.k = hidden;
    matmul_nvfp4(*static_cast<ThreadPool*>(pool), {&w}, x, m, {logits});
    for (int r = 0; r < m; ++r)
      for (int j = 0; j < vocab; ++j) logits[size_t(r) * vocab + j] *= logit_scale[j];
  });
}

// Sampler (engine/include/xtg/sampler.h, engine/src/sampler.cpp)
int xr_argmax(const float* logits, int n) { return argmax(logits, n); }

// top_logprobs (sampler.cpp:30-40): the k most likely (log probability, token) pairs, most likely first.
int xr_top_logprobs(const float* logits, int n, int k, float* lp, int32_t* idx) {
  return guarded([&] {
    std::vector<std::pair<float, int>> out;
    top_logprobs(logits, n, k, out);
    for (size_t i = 0; i < out.size(); ++i) {
      lp[i] = out[i].first;
      idx[i] = out[i].second;
    }
  });
}

// A fresh Sampler(seed)'s sample (sampler.cpp:41-94); *u = the first draw of an identically seeded engine in
// [0, 1), the value its uniform_real_distribution(0, total) scales by total.
int xr_sample(const float* logits, int n, float temperature, int top_k, float top_p, float min_p, uint64_t seed,
              double* u) {
  SamplingParams p;
  p.temperature = temperature;
  p.top_k = top_k;
  p.top_p = top_p;
  p.min_p = min_p;
  Sampler s(seed);
  std::mt19937_64 eng(seed);
  *u = std::generate_canonical<double, std::numeric_limits<double>::digits>(eng);
  return s.sample(logits, n, p);
}

// A Dory checkpoint through the reference's own pack (packs/dory/dory.cpp: DoryModel, DorySession) on its CPU
// backend: load_model (engine/src/model.cpp) with JSON launch options, sessions, forward with every row's logits.
void* xr_dory_load(const char* dir, const char* options, void* pool) {
  static std::once_flag once;
  std::unique_ptr<Model> m;
  const int rc = guarded([&] {
    std::call_once(once, [] { dory::register_pack(); });
    m = load_model(dir, json::parse(options ? options : "{}"), *static_cast<ThreadPool*>(pool));
  });
  return rc == 0 ? m.release() : nullptr;
}
void xr_dory_free(void* model) { delete static_cast<Model*>(model); }
int xr_dory_vocab(void* model) { return static_cast<Model*>(model)->info().vocab; }
void* xr_dory_session(void* model) {
  std::unique_ptr<Session> s;
  const int rc = guarded([&] { s = static_cast<Model*>(model)->new_session(); });
  return rc == 0 ? s.release() : nullptr;
}
void xr_dory_session_free(void* s) { delete static_cast<Session*>(s); }
int64_t xr_dory_n_past(void* s) { return static_cast<Session*>(s)->n_past(); }
int xr_dory_rewind(void* s, int64_t n) { return static_cast<Session*>(s)->rewind(n) ? 0 : -1; }
// logits [n][vocab]: every row of this call
int xr_dory_forward(void* s, const int32_t* tokens, int n, int vocab, float* logits) {
  return guarded([&] {
    static_cast<Session*>(s)->forward(tokens, n, Logits::All, [&](int row, const float* lg) {
      std::memcpy(logits + size_t(row) * size_t(vocab), lg, sizeof(float) * size_t(vocab));
    });
  });
}

}  // extern "C"
