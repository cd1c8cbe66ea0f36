// Kernel-level entry points of include/xtg_cuda.h: the device forms of the reference's CPU kernels on caller-owned
// device memory (matmul_nvfp4, attention, KvCache::store, the quantizer, the generators).
#include <algorithm>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/xtg_cuda.h"
#include "attention.h"
#include "common.cuh"
#include "elementwise.h"
#include "sampling.h"
#include "fp4mma.cuh"
#include "kernels.h"

using namespace xtg;

struct xtg_cuda_linear {
  int device = 0;
  int k = 0, nw = 0, tiles = 0, kblocks = 0;
  std::vector<int> n_out, tile0;
  std::vector<float> globals;
  uint8_t* w = nullptr;
  TileOut* outs = nullptr;          // device, rewritten per call (the ys pointers)
  std::vector<TileOut> outs_host;
  uint8_t* xb = nullptr;            // the input's B digits
  float* xb_pre = nullptr;
  GemvPlan plan;
  int64_t bytes = 0;
  int sms = 0;
  // GEMM path (m > 8): the activation units and row prescales, grown to the largest m seen
  uint8_t* act = nullptr;
  float* act_pre = nullptr;
  int act_rows = 0;

  ~xtg_cuda_linear() {
    cudaFree(w);
    cudaFree(outs);
    cudaFree(xb);
    cudaFree(xb_pre);
    cudaFree(act);
    cudaFree(act_pre);
  }
};

namespace {

void set_err(char* err, int len, const char* what) {
  if (err && len > 0) std::snprintf(err, (size_t)len, "%s", what);
}

template <class F>
int guarded(char* err, int err_len, F&& f) {
  try {
    f();
    return 0;
  } catch (const std::exception& e) {
    set_err(err, err_len, e.what());
    return -1;
  }
}

// The kernels read these operands 16 bytes at a time (vector loads, bulk copies): a caller's pointer must start on a
// 16-byte boundary, checked here so that a bad pointer is an error, not a GPU fault.
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

void require_attn_alignment(const xtg_cuda_attn_args* p) {
  XTG_REQUIRE(aligned16(p->q) && aligned16(p->k) && aligned16(p->v) && aligned16(p->out) && aligned16(p->k_codes) &&
                  aligned16(p->v_codes) && aligned16(p->k_scales) && aligned16(p->v_scales) &&
                  (p->ring == 0 || aligned16(p->ring_pos)),
              "attention: q, k, v, out, the cache codes and scales and the ring table must start on 16-byte boundaries");
}

}  // namespace

extern "C" {

xtg_cuda_linear* xtg_cuda_linear_new(int nw, const uint8_t* const* codes, const uint8_t* const* scales,
                                     const float* globals, const int* n_out, int k, char* err, int err_len) {
  std::unique_ptr<xtg_cuda_linear> L;
  try {
    XTG_REQUIRE(nw >= 1 && k >= 16 && k % 16 == 0, "linear: at least one weight, k a positive multiple of 16");
    L = std::make_unique<xtg_cuda_linear>();
    XTG_CUDA(cudaGetDevice(&L->device));
    int sms = 0;
    XTG_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, L->device));
    L->k = k;
    L->nw = nw;
    L->sms = sms;
    L->kblocks = packed_kblocks(k);
    for (int i = 0; i < nw; ++i) {
      XTG_REQUIRE(n_out[i] > 0, "linear: n_out must be positive");
      L->n_out.push_back(n_out[i]);
      L->globals.push_back(globals[i]);
      L->tile0.push_back(L->tiles);
      L->tiles += packed_tiles(n_out[i], false);
    }
    L->bytes = (int64_t)L->tiles * L->kblocks * kPackUnitBytes;
    XTG_CUDA(cudaMalloc(&L->w, L->bytes));
    for (int i = 0; i < nw; ++i)
      pack_nvfp4(codes[i], scales[i], nullptr, nullptr, n_out[i], k, false,
                 L->w + (int64_t)L->tile0[i] * L->kblocks * kPackUnitBytes, nullptr);
    XTG_CUDA(cudaMalloc(&L->outs, sizeof(TileOut) * L->tiles));
    L->outs_host.resize(L->tiles);
    L->plan = plan_gemv(L->tiles, L->kblocks, sms, 8, 1 << 20);
    XTG_CUDA(cudaMalloc(&L->xb, (size_t)digit_bytes(k)));
    XTG_CUDA(cudaMalloc(&L->xb_pre, (size_t)packed_kblocks(k) * 4 * kMaxRows * sizeof(float)));
    XTG_CUDA(cudaMemset(L->xb, 0, (size_t)digit_bytes(k)));
    {
      const std::vector<float> ones((size_t)packed_kblocks(k) * 4 * kMaxRows, kEmptyPrescale);
      XTG_CUDA(cudaMemcpy(L->xb_pre, ones.data(), ones.size() * sizeof(float), cudaMemcpyHostToDevice));
    }
    XTG_CUDA(cudaDeviceSynchronize());
  } catch (const std::exception& e) {
    set_err(err, err_len, e.what());
    return nullptr;
  }
  return L.release();
}

int xtg_cuda_linear_forward(xtg_cuda_linear* L, const float* x, int m, float* const* ys, void* stream, char* err,
                            int err_len) {
  return guarded(err, err_len, [&] {
    XTG_REQUIRE(m >= 1 && m <= kMaxGemmRows, "linear: 1..65536 rows");
    XTG_REQUIRE(aligned16(x), "linear: x must start on a 16-byte boundary");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    for (int i = 0; i < L->nw; ++i) {
      const int t0 = L->tile0[i], nt = packed_tiles(L->n_out[i], false);
      for (int t = 0; t < nt; ++t)
        L->outs_host[t0 + t] = TileOut{ys[i] + 128 * t, L->n_out[i], std::min(128, L->n_out[i] - 128 * t),
                                       L->globals[i], L->globals[i]};
    }
    XTG_CUDA(cudaMemcpyAsync(L->outs, L->outs_host.data(), sizeof(TileOut) * L->tiles, cudaMemcpyHostToDevice, s));
    if (m > kMaxRows) {
      // prefill chunk / batch: the tensor-core GEMM (matmul_nvfp4's m > 2 path)
      if (m > L->act_rows) {
        XTG_CUDA(cudaStreamSynchronize(s));
        cudaFree(L->act);
        cudaFree(L->act_pre);
        L->act = nullptr;
        L->act_pre = nullptr;
        L->act_rows = 0;
        const int rows = gemm_padded_rows(m);
        XTG_CUDA(cudaMalloc(&L->act, (size_t)gemm_act_bytes(rows, L->k)));
        XTG_CUDA(cudaMemset(L->act, 0, (size_t)gemm_act_bytes(rows, L->k)));   // K padding stays zero
        XTG_CUDA(cudaMalloc(&L->act_pre, (size_t)rows * sizeof(float)));
        L->act_rows = rows;
      }
      gemm_digitize(x, m, L->k, L->act, L->act_pre, s);
      launch_gemm(L->w, L->tiles, L->kblocks, L->act, L->act_pre, m, L->outs, L->sms, nullptr, s);
      XTG_CUDA(cudaStreamSynchronize(s));
      return;
    }
    digitize_rows(x, m, L->k, L->xb, L->xb_pre, s);
    GemvArgs a = {};
    a.w = L->w;
    a.tiles = L->tiles;
    a.kblocks = L->kblocks;
    a.xb = L->xb;
    a.xb_pre = L->xb_pre;
    a.m = m;
    a.err = nullptr;
    a.outs = L->outs;
    launch_gemv(kEpiStore, a, L->plan, s, false);
    // outs_host is read by the copy above before this call returns to the caller's next forward
    XTG_CUDA(cudaStreamSynchronize(s));
  });
}

int64_t xtg_cuda_linear_bytes(xtg_cuda_linear* L) { return L ? L->bytes : -1; }

void xtg_cuda_linear_free(xtg_cuda_linear* L) { delete L; }

int xtg_cuda_quantize_nvfp4(const uint16_t* w_bf16, int n_out, int k, uint8_t* codes, uint8_t* scales,
                            float* global, void* stream, char* err, int err_len) {
  return guarded(err, err_len, [&] {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned int* amax = nullptr;
    XTG_CUDA(cudaMalloc(&amax, sizeof(unsigned int)));
    try {
      quantize_nvfp4(w_bf16, n_out, k, codes, scales, global, amax, s);
      XTG_CUDA(cudaStreamSynchronize(s));
    } catch (...) {
      cudaFree(amax);
      throw;
    }
    cudaFree(amax);
  });
}

int xtg_cuda_attention(const xtg_cuda_attn_args* p, int splits, void* stream, char* err, int err_len) {
  return guarded(err, err_len, [&] {
    XTG_REQUIRE(p->head_dim == 128 || p->head_dim == 256, "attention: head_dim 128 or 256");
    require_attn_alignment(p);
    XTG_REQUIRE(p->n_q >= 1 && p->n_q <= kMaxRows, "attention: 1..8 query rows");
    XTG_REQUIRE(splits >= 1, "attention: at least one split");
    XTG_REQUIRE(p->kv_heads >= 1 && p->heads >= 1, "attention: at least one q head and one KV head");
    XTG_REQUIRE(p->ring == 0 || p->ring_pos != nullptr, "attention: a ring needs its slot -> position table");
    XTG_REQUIRE(p->ring != 0 || p->pos0 <= p->slots, "attention: pos0 beyond the cache");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float* part = nullptr;
    XTG_CUDA(cudaMalloc(&part, attention_part_floats(p->kv_heads, splits, p->head_dim) * sizeof(float)));
    try {
      AttnArgs a = {};
      a.q = p->q;
      a.k = p->k;
      a.v = p->v;
      a.kc = const_cast<uint8_t*>(p->k_codes);
      a.vc = const_cast<uint8_t*>(p->v_codes);
      a.ks = const_cast<float*>(p->k_scales);
      a.vs = const_cast<float*>(p->v_scales);
      a.slots = p->slots;
      a.ring = p->ring;
      a.ring_pos = p->ring_pos;
      a.dtype = p->dtype;
      a.window = p->window;
      a.scale = p->scale;
      a.m = p->n_q;
      a.pos0 = p->pos0;
      a.heads = p->heads;
      a.kv_heads = p->kv_heads;
      a.splits = splits;
      a.part = part;
      a.err = nullptr;
      a.head_dim = p->head_dim;
      launch_attention(a, s, false);
      CombineArgs cb = {};
      cb.part = part;
      cb.q = p->q;
      cb.k = p->k;
      cb.v = p->v;
      cb.scale = p->scale;
      cb.window = p->window;
      cb.splits = splits;
      cb.heads = p->heads;
      cb.kv_heads = p->kv_heads;
      cb.m = p->n_q;
      cb.out = p->out;
      cb.head_dim = p->head_dim;
      launch_attn_combine(cb, s, false);
      XTG_CUDA(cudaStreamSynchronize(s));
    } catch (...) {
      cudaFree(part);
      throw;
    }
    cudaFree(part);
  });
}

}  // extern "C"

// ---- attention without allocation ----
// Some callers cannot call cudaMalloc: a host runtime that reserved the GPU's memory for its own arena at start-up
// (a fresh allocation then fails, or fragments that arena), and code on a path where an allocation may not block
// or synchronise the device. xtg_cuda_attention allocates its split-KV partials per call; for those callers
// xtg_cuda_attention_noalloc keeps them in the fixed array below instead: 4,325,376 bytes, room for 256 KV-head x
// split pairs (32 query rows x 132 floats each). Every GPU that loads this library holds the array until the process
// exits. All calls share it, and it keeps the last call's contents.
namespace {
constexpr int kNoAllocPairs = 256;
constexpr int64_t kNoAllocFloats = (int64_t)kNoAllocPairs * 32 * 132;
}  // namespace

// In host code this name is only a host-side stand-in for the array; its device address comes from
// cudaGetSymbolAddress, once per device.
__device__ __align__(256) float g_noalloc_attn_part[kNoAllocFloats];

namespace {
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// The array's device address on the current device; the first call on a device looks it up with that device current.
float* noalloc_scratch() {
  int device = 0;
  XTG_CUDA(cudaGetDevice(&device));
  XTG_REQUIRE(device >= 0 && device < kNoAllocMaxDevices, "attention_noalloc: device index above 63");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[device]) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_attn_part);
    if (e != cudaSuccess)
      throw CudaError(std::string("attention_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    g_noalloc_ptr[device] = static_cast<float*>(ptr);
  }
  return g_noalloc_ptr[device];
}
}  // namespace

extern "C" {

int xtg_cuda_attention_noalloc(const xtg_cuda_attn_args* p, int splits, void* stream, char* err, int err_len) {
  return guarded(err, err_len, [&] {
    XTG_REQUIRE(p->head_dim == 128 || p->head_dim == 256, "attention: head_dim 128 or 256");
    require_attn_alignment(p);
    XTG_REQUIRE(p->n_q >= 1 && p->n_q <= kMaxRows, "attention: 1..8 query rows");
    XTG_REQUIRE(splits >= 1, "attention: at least one split");
    XTG_REQUIRE(p->ring == 0 || p->ring_pos != nullptr, "attention: a ring needs its slot -> position table");
    XTG_REQUIRE(p->ring != 0 || p->pos0 <= p->slots, "attention: pos0 beyond the cache");
    XTG_REQUIRE(p->kv_heads >= 1 && p->heads >= 1, "attention: at least one q head and one KV head");
    XTG_REQUIRE(attention_part_floats(p->kv_heads, splits, p->head_dim) <= kNoAllocFloats,
                "attention_noalloc: kv_heads x splits above 256 (128 at head_dim 256), the fixed scratch's limit "
                "(4,325,376 bytes)");
    float* part = noalloc_scratch();
    // every split writes the partial of every live query row that the combine reads: nothing needs clearing
    AttnArgs a = {};
    a.q = p->q;
    a.k = p->k;
    a.v = p->v;
    a.kc = const_cast<uint8_t*>(p->k_codes);
    a.vc = const_cast<uint8_t*>(p->v_codes);
    a.ks = const_cast<float*>(p->k_scales);
    a.vs = const_cast<float*>(p->v_scales);
    a.slots = p->slots;
    a.ring = p->ring;
    a.ring_pos = p->ring_pos;
    a.dtype = p->dtype;
    a.window = p->window;
    a.scale = p->scale;
    a.m = p->n_q;
    a.pos0 = p->pos0;
    a.heads = p->heads;
    a.kv_heads = p->kv_heads;
    a.splits = splits;
    a.part = part;
    a.err = nullptr;
    a.head_dim = p->head_dim;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    launch_attention(a, s, false);
    CombineArgs cb = {};
    cb.part = part;
    cb.q = p->q;
    cb.k = p->k;
    cb.v = p->v;
    cb.scale = p->scale;
    cb.window = p->window;
    cb.splits = splits;
    cb.heads = p->heads;
    cb.kv_heads = p->kv_heads;
    cb.m = p->n_q;
    cb.out = p->out;
    cb.head_dim = p->head_dim;
    launch_attn_combine(cb, s, false);
  });
}

int xtg_cuda_kv_store(const float* k, const float* v, int64_t pos, int n, int kv_heads, int64_t slots, int ring,
                      int dtype, uint8_t* k_codes, uint8_t* v_codes, float* k_scales, float* v_scales, void* stream,
                      char* err, int err_len) {
  return guarded(err, err_len, [&] {
    XTG_REQUIRE(ring || pos + n <= slots, "KV cache full");
    KvStoreArgs a = {};
    a.k = k;
    a.v = v;
    a.pos = pos;
    a.n = n;
    a.kv_heads = kv_heads;
    a.slots = slots;
    a.ring = ring;
    a.dtype = dtype;
    a.kc = k_codes;
    a.vc = v_codes;
    a.ks = k_scales;
    a.vs = v_scales;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    launch_kv_store(a, s);
    XTG_CUDA(cudaStreamSynchronize(s));
  });
}

int xtg_cuda_gen(int what, uint64_t seed, uint64_t stream_id, float a, float b, void* out, int64_t n, void* stream,
                 char* err, int err_len) {
  return guarded(err, err_len, [&] {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (what == 0)
      gen_normal_bf16(seed, stream_id, a, static_cast<uint16_t*>(out), n, s);
    else if (what == 1)
      gen_uniform(seed, stream_id, a, b, static_cast<float*>(out), n, s);
    else if (what == 2)
      gen_int8(seed, stream_id, static_cast<int8_t*>(out), n, s);
    else
      throw CudaError("gen: what must be 0, 1 or 2");
    XTG_CUDA(cudaStreamSynchronize(s));
  });
}

int xtg_cuda_head_bf16(const float* x, int m, const uint16_t* w, int vocab, int hidden, const float* logit_scale,
                       float* logits, int32_t* argmax, void* stream, char* err, int err_len) {
  return guarded(err, err_len, [&] {
    XTG_REQUIRE(x && w && logit_scale && (logits || argmax), "head_bf16: null pointer");
    XTG_REQUIRE(m >= 1 && m <= kMaxRows && vocab >= 1, "head_bf16: 1..8 rows, a vocabulary");
    XTG_REQUIRE(aligned16(x) && aligned16(w), "head_bf16: x and w must start on a 16-byte boundary");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int dev = 0, sms = 0;
    XTG_CUDA(cudaGetDevice(&dev));
    XTG_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int tiles = (vocab + 127) / 128;
    // the per-tile candidates and the rows for the argmax kernel (it reads m from a StepParams)
    void* scratch = nullptr;
    const size_t cand_bytes = (size_t)tiles * kMaxRows * sizeof(ArgCand);
    XTG_CUDA(cudaMalloc(&scratch, cand_bytes + sizeof(StepParams) + 16));
    struct Free {
      void* p;
      ~Free() { cudaFree(p); }
    } f{scratch};
    ArgCand* cand = static_cast<ArgCand*>(scratch);
    StepParams* params = reinterpret_cast<StepParams*>(static_cast<uint8_t*>(scratch) + cand_bytes);
    int* derr = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(params) + sizeof(StepParams));
    StepParams hp = {};
    hp.m = m;
    XTG_CUDA(cudaMemcpyAsync(params, &hp, sizeof(hp), cudaMemcpyHostToDevice, s));
    XTG_CUDA(cudaMemsetAsync(derr, 0, sizeof(int), s));
    HeadBf16Args h = {};
    h.x = x;
    h.m = m;
    h.w = w;
    h.vocab = vocab;
    h.hidden = hidden;
    h.logit_scale = logit_scale;
    h.logits = logits;
    h.cand = cand;
    h.err = derr;
    launch_head_bf16(h, sms, s, false);
    if (argmax) launch_argmax(cand, tiles, params, argmax, nullptr, nullptr, s, false);
    int e = 0;
    XTG_CUDA(cudaMemcpyAsync(&e, derr, sizeof(int), cudaMemcpyDeviceToHost, s));
    XTG_CUDA(cudaStreamSynchronize(s));   // the scratch is freed on return
    XTG_REQUIRE(e == 0, "head_bf16: a device wait timed out");
  });
}

int xtg_cuda_topk_rows(const float* logits, int rows, int vocab, int k, float temperature, int32_t* idx, float* logit,
                       float* row_max, double* total, void* stream, char* err, int err_len) {
  return guarded(err, err_len, [&] {
    XTG_REQUIRE(logits && idx && logit && row_max && total, "topk: null pointer");
    launch_topk(logits, rows, vocab, k, temperature, idx, logit, row_max, total, static_cast<cudaStream_t>(stream));
  });
}

}  // extern "C"
