// The session behind include/xtg_cuda.h: what npu/xtg_npu.cpp does for the Hexagon NPU (KV instances, the ring's
// slot -> position table, rewinds, snapshots, context tiers, logits out through a callback), done on one B200 with
// the step of packs/dory/dory.cpp:467-578 as a chain of sm_100a kernels captured once into a CUDA graph.
//
// HBM layout of a session:
//   weight arena   every NVFP4 weight in the GEMV streaming layout (weights.cu), in execution order: per attention
//                  evaluation the fused q|k|v|g weight then o; per MLP evaluation the interleaved gate/up weight then
//                  down; the tied head last. The step streams it front to back once.
//   KV instances   one per attention evaluation (loops unrolled, per_loop): global ones hold `context` slots (slot =
//                  position), sliding ones a ring of `ring` slots; layouts in attention.cu.
//   activations    the residual stream h (f32 [8][hidden]) and its fp16 fragments, the loop state and input, the
//                  projection rows, attention partials, the gated attention / SwiGLU fragments, logits.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "../../include/xtg_cuda.h"
#include "attention.h"
#include "common.cuh"
#include "elementwise.h"
#include "fp4mma.cuh"
#include "batch.h"
#include "checkpoint.h"
#include "json.h"
#include "nccl_rt.h"
#include "sampling.h"
#include "kernels.h"

namespace xtg {

namespace {

struct Config {
  int hidden = 3072, ffn = 9216, heads = 24, kv_heads = 6, head_dim = 128, vocab = 131072;
  int n_in = 4, n_rec = 40, n_out = 4, loops = 2;
  int window = 1024, ring = 1088, global_every = 4;
  float theta_sliding = 1e4f, theta_global = 1e7f, weight_std = 0.02f;
  float lr_lo = 0.05f, lr_hi = 0.2f, qs_lo = 48.f, qs_hi = 80.f, gs_lo = 25.f, gs_hi = 75.f;
  float suv_lo = 25.f, suv_hi = 75.f, ls_lo = 100.f, ls_hi = 200.f, kvs_lo = 0.0008f, kvs_hi = 0.0016f;
  uint64_t seed = 3;
  // session options
  int64_t context = 8192;
  int kv_dtype = kKvInt8;
  int snapshots = 2;
  int decode_rows = 8;
  int device = 0;
  bool graph = true, pdl = true, l2_first = true;
  bool batch = true;   // xtg_cuda_forward_batch steps sessions over one weight set together (batch.h)
  bool nvtx = false;   // NVTX ranges per sublayer while a step is enqueued (aligned with the kernels when graph = 0)
  int splits_global = 0, splits_ring = 0;   // 0: chosen from the SM count
  // batch-1 split-KV across processes (one GPU each): every process holds the whole model and every cache and runs
  // the whole step, but attends only its share of each global cache's chunks; the attention partials of the global
  // layers meet by an NCCL all-gather (kv_world processes, this one kv_rank, nccl_id the 128-byte unique id in hex)
  int kv_world = 1, kv_rank = 0;
  std::string nccl_id;
  // "peer": each combine kernel sends its merged partials to the peers' exchange slots over NVLink (CUDA IPC) and
  // waits for theirs, at most kv_wait_ms; "nccl": an ncclAllGather of every split's partial between the kernels
  std::string kv_exchange = "peer";
  int kv_wait_ms = 10000;
  // a checkpoint (path to a ModelOpt W4A16_NVFP4 Dory directory; "synthetic": the seeded synthetic model): the kind
  // of every physical sublayer, and the lm_head kept in BF16 (the reference's matmul_bf16) or quantized to NVFP4
  std::string path = "synthetic";
  std::vector<int> kinds;
  bool head_bf16 = false;

  int n_evals() const { return n_in + n_rec * loops + n_out; }
  int phys(int e) const {
    if (e < n_in) return e;
    e -= n_in;
    if (e < n_rec * loops) return n_in + e % n_rec;
    return n_in + n_rec + (e - n_rec * loops);
  }
  // 0 MLP, 1 sliding attention, 2 global attention (the oracle's xo_synth_kind)
  int kind(int e) const {
    const int l = phys(e);
    if (!kinds.empty()) return kinds[l];
    if (l % 2) return 0;
    const int a = l / 2;
    return (global_every > 0 && a % global_every == global_every - 1) ? 2 : 1;
  }
};

int64_t parse_tier(const std::string& s) {
  if (s.empty()) throw CudaError("tier: empty");
  char* end = nullptr;
  const long long v = std::strtoll(s.c_str(), &end, 10);
  if (end == s.c_str() || v <= 0) throw CudaError("tier: " + s + " is not a context length");
  int64_t n = v;
  if (*end == 'k' || *end == 'K') {
    n *= 1024;
    ++end;
  }
  if (*end) throw CudaError("tier: " + s + " is not a context length");
  return n;
}

// Session options (JSON) over the synthetic model's shape (options "model": {...}) or a checkpoint's (ck, its
// config.json; the options may then pick loops, kv_mode, ring and how the head is kept).
Config parse_config(const std::string& options, const DoryConfig* ck = nullptr) {
  Config c;
  Json o = options.empty() ? Json() : Json::parse(options);
  if (o.kind != Json::Null && o.kind != Json::Object) throw CudaError("options: not a JSON object");
  const Json& m = o.at("model");
  if (ck) {
    if (m.kind != Json::Null) throw CudaError("model: a checkpoint brings its own shape (no \"model\" option)");
    c.hidden = ck->hidden;
    c.ffn = ck->ffn;
    c.heads = ck->heads;
    c.kv_heads = ck->kv_heads;
    c.head_dim = ck->head_dim;
    c.vocab = ck->vocab;
    c.n_in = ck->n_in;
    c.n_rec = ck->n_rec;
    c.n_out = ck->n_out;
    c.kinds = ck->kind;
    c.global_every = 0;
    c.theta_sliding = ck->theta_sliding;
    c.theta_global = ck->theta_global;
    const bool sliding = std::count(c.kinds.begin(), c.kinds.end(), 1) > 0;
    c.window = sliding ? ck->window : 64;   // no sliding layer: a ring nothing reads
    c.ring = (int)o.number("ring", c.window + 64);
    c.loops = (int)o.number("loops", ck->default_loops);
    if (c.loops < 1 || c.loops > 4) throw CudaError("loops: 1..4");
    const std::string mode = o.string("kv_mode", ck->kv_mode);
    if (mode != "per_loop") throw CudaError("kv_mode: " + mode + " (only per_loop: a KV instance per loop)");
    const std::string head = o.string("head", "bf16");
    if (head != "bf16" && head != "nvfp4") throw CudaError("head: " + head + " (bf16 | nvfp4)");
    c.head_bf16 = head == "bf16";
  }
  if (!ck) {   // the synthetic model's shape and seeds
    auto I = [&](const char* k, int& v) { v = (int)m.number(k, v); };
    auto F = [&](const char* k, float& v) { v = (float)m.number(k, v); };
    I("hidden", c.hidden);
    I("ffn", c.ffn);
    I("heads", c.heads);
    I("kv_heads", c.kv_heads);
    I("head_dim", c.head_dim);
    I("vocab", c.vocab);
    I("n_in", c.n_in);
    I("n_rec", c.n_rec);
    I("n_out", c.n_out);
    I("loops", c.loops);
    I("window", c.window);
    c.ring = c.window + 64;
    I("ring", c.ring);
    I("global_every", c.global_every);
    F("theta_sliding", c.theta_sliding);
    F("theta_global", c.theta_global);
    F("weight_std", c.weight_std);
    F("lr_lo", c.lr_lo);
    F("lr_hi", c.lr_hi);
    F("qs_lo", c.qs_lo);
    F("qs_hi", c.qs_hi);
    F("gs_lo", c.gs_lo);
    F("gs_hi", c.gs_hi);
    F("suv_lo", c.suv_lo);
    F("suv_hi", c.suv_hi);
    F("ls_lo", c.ls_lo);
    F("ls_hi", c.ls_hi);
    F("kvs_lo", c.kvs_lo);
    F("kvs_hi", c.kvs_hi);
    c.seed = (uint64_t)m.number("seed", (double)c.seed);
  }
  const Json& ctx = o.at("context");
  if (ctx.kind == Json::String)
    c.context = parse_tier(ctx.str);
  else
    c.context = (int64_t)o.number("context", (double)c.context);
  const std::string dt = o.string("kv_dtype", "int8");
  if (dt != "int8" && dt != "fp8") throw CudaError("kv_dtype: " + dt + " (int8 | fp8)");
  c.kv_dtype = dt == "fp8" ? kKvFp8 : kKvInt8;
  c.snapshots = (int)o.number("snapshots", c.snapshots);
  c.decode_rows = (int)o.number("decode_rows", c.decode_rows);
  c.device = (int)o.number("device", c.device);
  c.graph = o.number("graph", 1) != 0;
  c.pdl = o.number("pdl", 1) != 0;
  c.l2_first = o.number("l2_evict_first", 1) != 0;
  c.batch = o.number("batch", 1) != 0;
  c.nvtx = o.number("nvtx", 0) != 0;
  c.splits_global = (int)o.number("splits_global", 0);
  c.splits_ring = (int)o.number("splits_ring", 0);
  c.kv_world = (int)o.number("kv_world", 1);
  c.kv_rank = (int)o.number("kv_rank", 0);
  c.nccl_id = o.string("nccl_id", "");
  c.kv_exchange = o.string("kv_exchange", "peer");
  c.kv_wait_ms = (int)o.number("kv_wait_ms", 10000);
  if (c.kv_exchange != "peer" && c.kv_exchange != "nccl") throw CudaError("kv_exchange: \"peer\" or \"nccl\"");
  if (c.kv_wait_ms < 1) throw CudaError("kv_wait_ms: at least 1");
  if (c.kv_world < 1 || c.kv_world > 8 || c.kv_rank < 0 || c.kv_rank >= c.kv_world)
    throw CudaError("kv_world: 1..8 processes, kv_rank below it");
  if (c.kv_world > 1 && c.nccl_id.size() != 2 * sizeof(ncclUniqueId))
    throw CudaError("nccl_id: the NCCL unique id as " + std::to_string(2 * sizeof(ncclUniqueId)) + " hex digits");
  if (c.head_dim != 128 && c.head_dim != 256) throw CudaError("model: head_dim must be 128 or 256");
  if (c.head_dim != 128 && c.kv_world > 1)
    throw CudaError("kv_world: split-KV across GPUs takes head_dim 128 (the exchange slots hold 128 dims)");
  if (c.heads % c.kv_heads || c.heads / c.kv_heads > 4) throw CudaError("model: at most 4 q heads per KV head");
  if (c.hidden % 64 || c.ffn % 64 || c.hidden > 8192) throw CudaError("model: hidden, ffn multiples of 64, hidden <= 8192");
  if (c.vocab <= 0 || c.n_in < 0 || c.n_rec < 0 || c.n_out < 0 || c.loops < 0 || c.n_evals() <= 0)
    throw CudaError("model: bad layer counts");
  if (c.window <= 0 || c.ring % 64 || c.ring < c.window + kMaxRows)
    throw CudaError("model: the ring needs window + 8 slots or more, a multiple of 64");
  if (c.context < 64 || c.context % 64) throw CudaError("context: a multiple of 64");
  if (c.decode_rows < 1 || c.decode_rows > kMaxRows) throw CudaError("decode_rows: 1..8");
  if (c.snapshots < 0 || c.snapshots > 8) throw CudaError("snapshots: 0..8");
  if (ck && c.context > ck->max_pos) throw CudaError("context: above the model's max_position_embeddings");
  if (c.head_bf16 && (c.hidden > kMaxHeadBf16Hidden || c.hidden % 64))
    throw CudaError("head: bf16 takes hidden <= 5120 (a multiple of 64); use \"nvfp4\"");
  return c;
}

// A packed weight (or fused set) and where its tiles go.
struct Linear {
  uint8_t* w = nullptr;   // inside the arena
  int tiles = 0, kblocks = 0;
  int64_t bytes = 0;
  int64_t alg_bytes = 0;  // codes + scales + globals of the NVFP4 weights
  int n_total = 0, k = 0;
  TileOut* outs = nullptr;   // device, kEpiStore
  float g0 = 1.f, g1 = 1.f;  // gate / up globals (kEpiSwiglu), head global
  GemvPlan plan;
};

struct Eval {
  int kind = 0;
  Linear qkvg, o, gu, down;   // o.g0 / down.g0: their global scales; gq: those of q, k, v, g
  float gq[4] = {1.f, 1.f, 1.f, 1.f};
  float *lr = nullptr, *qscale = nullptr, *gscale = nullptr, *sg = nullptr, *su = nullptr;
  int theta = 0;   // 0 sliding, 1 global
  int cache = -1;
};

struct KvInst {
  uint8_t *kc = nullptr, *vc = nullptr;
  float *ks = nullptr, *vs = nullptr;
  int64_t slots = 0;
  bool ring = false;
};

struct Snap {
  int64_t pos = -1;
  std::vector<KvInst> rings;   // device copies of the ring instances
  std::vector<int64_t> ring_pos;
};

enum KernelClass { kClsGemv = 0, kClsAttn = 1, kClsCombine = 2, kClsSmall = 3, kClasses = 4 };

// An NVTX range for as long as it lives (nothing when off; NVTX itself is inert without a tool attached).
struct NvtxRange {
  bool on;
  NvtxRange(bool enabled, const char* name) : on(enabled) {
    if (on) nvtxRangePushA(name);
  }
  ~NvtxRange() {
    if (on) nvtxRangePop();
  }
};

}  // namespace

}  // namespace xtg

using namespace xtg;

namespace {
// prompt chunks of more than decode_rows rows as one batched step (defined with BatchStep below)
int prefill_rows(const xtg_cuda* h);
void prefill_chunk(xtg_cuda* h, const int32_t* tokens, int m, int want, int off, int n, xtg_cuda_logits_fn fn,
                   void* user);
}  // namespace

struct xtg_cuda {
  Config c;
  cudaStream_t stream = nullptr;
  int num_sms = 148;
  std::vector<void*> allocs;   // freed at close
  // the model's weights (packed arena, per-layer vectors, RoPE frequencies): shared by the sessions opened from this
  // one with xtg_cuda_open_shared, freed with the last of them
  struct DeviceBlocks {
    std::vector<void*> p;
    ~DeviceBlocks() {
      for (void* q : p) cudaFree(q);
    }
  };
  std::shared_ptr<DeviceBlocks> wmem = std::make_shared<DeviceBlocks>();
  // model
  uint8_t* arena = nullptr;
  int64_t arena_bytes = 0;
  std::vector<Eval> evals;
  Linear head;
  float* logit_scale = nullptr;
  float* inv_freq = nullptr;   // [2][head_dim / 2]
  // a checkpoint's BF16 embedding table and (head "bf16") BF16 lm_head, [vocab][hidden]; null for the synthetic
  // model, whose tied NVFP4 head is also its embedding
  uint16_t* embed_bf16 = nullptr;
  uint16_t* head_w_bf16 = nullptr;
  // session
  std::vector<KvInst> kv;
  KvSeq* kv_seq_dev = nullptr;   // the instances as the q|k|v preparation kernel takes them (head dim 256)
  int32_t* ring_pos_dev = nullptr;
  std::vector<int64_t> ring_pos;
  int64_t n_past = 0;
  uint64_t generation = 0;   // advanced when the caches move (a tier change): a batched step built over them is stale
  std::vector<Snap> snaps;
  int last_rows = 0;
  // activations and scratch
  StepParams* params_dev = nullptr;
  StepParams* params_host = nullptr;
  float *h = nullptr, *state = nullptr, *input = nullptr, *o = nullptr, *proj = nullptr, *part = nullptr;
  // GEMV inputs as B digits with their per-group prescales: h (the residual's output), the gated attention output
  // (the O projection's input), v (the down projection's input)
  uint8_t *xb = nullptr, *ab = nullptr, *vb = nullptr;
  float *xb_pre = nullptr, *ab_pre = nullptr, *vb_pre = nullptr;
  float *q_prep = nullptr, *k_new = nullptr, *v_new = nullptr;   // this step's prepared q / k / v rows
  float *asum = nullptr, *vsum = nullptr, *rsum = nullptr, *logits = nullptr, *logits_host = nullptr, *argmax_val = nullptr;
  float *rope_cos = nullptr, *rope_sin = nullptr;
  int32_t* argmax = nullptr;
  // xtg_cuda_topk's results on the device (allocated at its first call)
  int32_t* tk_idx = nullptr;
  float* tk_val = nullptr;
  float* tk_max = nullptr;
  double* tk_total = nullptr;
  ArgCand* cand = nullptr;
  int* dev_err = nullptr;   // bounded device waits that gave up (never expected)
  int* err_host = nullptr;  // pinned copy of dev_err
  // forward(): the error word's copy and each logits row's, so that a row's callback runs while later rows copy
  cudaEvent_t err_ev = nullptr, row_ev[kMaxRows] = {};
  int splits_g = 1, splits_r = 1;
  int proj_ld = 0;
  ncclComm_t comm = nullptr;   // split-KV only
  // the peer exchange: this process's exchange slots (exported by CUDA IPC), the peers' (imported), the step
  // counter, the global layers per step
  void* xbuf = nullptr;
  void* peer_base[kMaxKvWorld] = {};
  PeerXchg xchg = {};
  uint32_t* epoch = nullptr;
  int n_glob = 0;
  // graph
  cudaGraphExec_t exec = nullptr;
  // profiling
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>>* prof = nullptr;
  std::vector<int>* prof_cls = nullptr;

  template <class T>
  T* walloc(size_t n) {
    void* p = nullptr;
    XTG_CUDA(cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)));
    wmem->p.push_back(p);
    return static_cast<T*>(p);
  }

  template <class T>
  T* dalloc(size_t n, bool zero = true) {
    void* p = nullptr;
    XTG_CUDA(cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)));
    allocs.push_back(p);
    if (zero) XTG_CUDA(cudaMemsetAsync(p, 0, std::max<size_t>(n, 1) * sizeof(T), stream));
    return static_cast<T*>(p);
  }

  ~xtg_cuda() {
    if (stream) cudaStreamSynchronize(stream);
    if (exec) cudaGraphExecDestroy(exec);
    for (void* p : peer_base)
      if (p) cudaIpcCloseMemHandle(p);
    if (xbuf) cudaFree(xbuf);
    if (comm) nccl_api().comm_destroy(comm);
    free_kv(kv);
    for (auto& s : snaps) free_kv(s.rings);
    for (void* p : allocs) cudaFree(p);
    if (params_host) cudaFreeHost(params_host);
    if (logits_host) cudaFreeHost(logits_host);
    if (err_host) cudaFreeHost(err_host);
    if (err_ev) cudaEventDestroy(err_ev);
    for (cudaEvent_t e : row_ev)
      if (e) cudaEventDestroy(e);
    if (stream) cudaStreamDestroy(stream);
  }

  static void free_kv(std::vector<KvInst>& v) {
    for (auto& k : v) {
      cudaFree(k.kc);
      cudaFree(k.vc);
      cudaFree(k.ks);
      cudaFree(k.vs);
    }
    v.clear();
  }

  static KvInst alloc_kv(int kv_heads, int hd, int64_t slots, bool ring, cudaStream_t s) {
    KvInst k;
    k.slots = slots;
    k.ring = ring;
    const size_t codes = (size_t)kv_heads * slots * hd, sc = (size_t)kv_heads * slots * sizeof(float);
    cudaError_t e = cudaMalloc(&k.kc, codes);
    if (e == cudaSuccess) e = cudaMalloc(&k.vc, codes);
    if (e == cudaSuccess) e = cudaMalloc(&k.ks, sc);
    if (e == cudaSuccess) e = cudaMalloc(&k.vs, sc);
    if (e != cudaSuccess) {
      cudaFree(k.kc);
      cudaFree(k.vc);
      cudaFree(k.ks);
      cudaFree(k.vs);
      cudaGetLastError();
      throw CudaError(std::string("KV cache allocation: ") + cudaGetErrorString(e));
    }
    // zero codes: no stale FP8 NaN pattern is ever read, even under a mask
    XTG_CUDA(cudaMemsetAsync(k.kc, 0, codes, s));
    XTG_CUDA(cudaMemsetAsync(k.vc, 0, codes, s));
    XTG_CUDA(cudaMemsetAsync(k.ks, 0, sc, s));
    XTG_CUDA(cudaMemsetAsync(k.vs, 0, sc, s));
    return k;
  }

  static void copy_kv(const KvInst& src, KvInst& dst, int kv_heads, int hd, int64_t used, cudaStream_t s) {
    if (used <= 0) return;
    // K [kv_heads][slots][hd]: rows of used * hd bytes
    XTG_CUDA(cudaMemcpy2DAsync(dst.kc, dst.slots * hd, src.kc, src.slots * hd, used * hd, kv_heads,
                               cudaMemcpyDeviceToDevice, s));
    // V [kv_heads][slots / 64][hd][64]: the whole 64-slot chunks that hold the first `used` slots
    const int64_t vbytes = (used + 63) / 64 * 64 * hd;
    XTG_CUDA(cudaMemcpy2DAsync(dst.vc, dst.slots * hd, src.vc, src.slots * hd, vbytes, kv_heads,
                               cudaMemcpyDeviceToDevice, s));
    XTG_CUDA(cudaMemcpy2DAsync(dst.ks, dst.slots * 4, src.ks, src.slots * 4, used * 4, kv_heads,
                               cudaMemcpyDeviceToDevice, s));
    XTG_CUDA(cudaMemcpy2DAsync(dst.vs, dst.slots * 4, src.vs, src.slots * 4, used * 4, kv_heads,
                               cudaMemcpyDeviceToDevice, s));
  }

  // ---- model construction (the seeded synthetic Dory; the oracle's stream map) ----

  void build_model() {
    if (c.path != "synthetic") {
      load_checkpoint();
      return;
    }
    const int H = c.hidden, F = c.ffn, Q = c.heads * c.head_dim, KV = c.kv_heads * c.head_dim;
    const int ne = c.n_evals();
    // arena size
    int64_t total = 0;
    for (int e = 0; e < ne; ++e) {
      if (c.kind(e) == 0)
        total += packed_bytes(F, H, true) + packed_bytes(H, F, false);
      else
        total += packed_bytes(2 * Q + 2 * KV, H, false) + packed_bytes(H, Q, false);
    }
    total += packed_bytes(c.vocab, H, false);
    // the fused q|k|v|g weight packs each projection in whole tiles
    for (int e = 0; e < ne; ++e)
      if (c.kind(e) != 0) {
        total -= packed_bytes(2 * Q + 2 * KV, H, false);
        total += (int64_t)(packed_tiles(Q, false) * 2 + packed_tiles(KV, false) * 2) * packed_kblocks(H) *
                 kPackUnitBytes;
      }
    arena_bytes = total;
    arena = walloc<uint8_t>((size_t)total);
    // temporaries: the largest weight (the head) in bf16, ModelOpt codes / scales for two weights
    const int64_t max_elems = std::max<int64_t>((int64_t)c.vocab * H, (int64_t)F * H);
    uint16_t* raw = nullptr;
    uint8_t *codes_a = nullptr, *scales_a = nullptr, *codes_b = nullptr, *scales_b = nullptr;
    float* gdev = nullptr;
    unsigned int* amax = nullptr;
    XTG_CUDA(cudaMalloc(&raw, max_elems * 2));
    XTG_CUDA(cudaMalloc(&codes_a, max_elems / 2));
    XTG_CUDA(cudaMalloc(&scales_a, max_elems / 16));
    XTG_CUDA(cudaMalloc(&codes_b, (int64_t)F * H / 2));
    XTG_CUDA(cudaMalloc(&scales_b, (int64_t)F * H / 16));
    XTG_CUDA(cudaMalloc(&gdev, 2 * sizeof(float)));
    XTG_CUDA(cudaMalloc(&amax, sizeof(unsigned int)));
    auto make = [&](uint64_t stream_id, int n_out, int k, uint8_t* codes, uint8_t* scales) {
      gen_normal_bf16(c.seed, stream_id, c.weight_std, raw, (int64_t)n_out * k, stream);
      quantize_nvfp4(raw, n_out, k, codes, scales, gdev, amax, stream);
      float g = 0.f;
      XTG_CUDA(cudaMemcpyAsync(&g, gdev, sizeof(float), cudaMemcpyDeviceToHost, stream));
      XTG_CUDA(cudaStreamSynchronize(stream));
      return g;
    };
    auto vec = [&](uint64_t stream_id, float lo, float hi, int n) {
      float* v = walloc<float>(n);
      gen_uniform(c.seed, stream_id, lo, hi, v, n, stream);
      return v;
    };
    uint8_t* cursor = arena;
    // the head takes whole tiles (its argmax candidates), SwiGLU one tile per CTA
    auto place = [&](Linear& L, int tiles, int kblocks, int max_split = 8, int max_tpc = 1 << 20) {
      L.w = cursor;
      L.tiles = tiles;
      L.kblocks = kblocks;
      L.bytes = (int64_t)tiles * kblocks * kPackUnitBytes;
      L.plan = plan_gemv(tiles, kblocks, num_sms, max_split, max_tpc);
      cursor += L.bytes;
    };
    auto alg = [](int n, int k) { return (int64_t)n * k / 2 + (int64_t)n * k / 16 + 4; };
    proj_ld = 2 * Q + 2 * KV;
    int n_attn = 0;
    evals.resize(ne);
    for (int e = 0; e < ne; ++e) {
      Eval& E = evals[e];
      E.kind = c.kind(e);
      const uint64_t base = 1000 + 16 * (uint64_t)e;
      E.lr = vec(base + 8, c.lr_lo, c.lr_hi, H);
      if (E.kind == 0) {
        E.sg = vec(base + 11, c.suv_lo, c.suv_hi, F);
        E.su = vec(base + 12, c.suv_lo, c.suv_hi, F);
        place(E.gu, packed_tiles(F, true), packed_kblocks(H), 8, 1);
        E.gu.g0 = make(base + 0, F, H, codes_a, scales_a);
        E.gu.g1 = make(base + 1, F, H, codes_b, scales_b);
        pack_nvfp4(codes_a, scales_a, codes_b, scales_b, F, H, true, E.gu.w, stream);
        E.gu.alg_bytes = 2 * alg(F, H);
        E.gu.n_total = 2 * F;
        E.gu.k = H;
        place(E.down, packed_tiles(H, false), packed_kblocks(F));
        const float gd = make(base + 2, H, F, codes_a, scales_a);
        pack_nvfp4(codes_a, scales_a, nullptr, nullptr, H, F, false, E.down.w, stream);
        E.down.alg_bytes = alg(H, F);
        E.down.n_total = H;
        E.down.k = F;
        E.down.g0 = gd;
      } else {
        E.qscale = vec(base + 9, c.qs_lo, c.qs_hi, Q);
        E.gscale = vec(base + 10, c.gs_lo, c.gs_hi, Q);
        E.theta = E.kind == 2 ? 1 : 0;
        E.cache = n_attn++;
        const int tq = packed_tiles(Q, false), tk = packed_tiles(KV, false), kblocks = packed_kblocks(H);
        place(E.qkvg, 2 * tq + 2 * tk, kblocks);
        const int n_out[4] = {Q, KV, KV, Q};
        int tile0 = 0;
        for (int j = 0; j < 4; ++j) {
          E.gq[j] = make(base + j, n_out[j], H, codes_a, scales_a);
          pack_nvfp4(codes_a, scales_a, nullptr, nullptr, n_out[j], H, false,
                     E.qkvg.w + (int64_t)tile0 * kblocks * kPackUnitBytes, stream);
          tile0 += packed_tiles(n_out[j], false);
          E.qkvg.alg_bytes += alg(n_out[j], H);
        }
        E.qkvg.n_total = 2 * Q + 2 * KV;
        E.qkvg.k = H;
        place(E.o, packed_tiles(H, false), packed_kblocks(Q));
        const float go = make(base + 4, H, Q, codes_a, scales_a);
        pack_nvfp4(codes_a, scales_a, nullptr, nullptr, H, Q, false, E.o.w, stream);
        E.o.alg_bytes = alg(H, Q);
        E.o.n_total = H;
        E.o.k = Q;
        E.o.g0 = go;
      }
    }
    place(head, packed_tiles(c.vocab, false), packed_kblocks(H), 1);
    head.g0 = make(1, c.vocab, H, codes_a, scales_a);
    pack_nvfp4(codes_a, scales_a, nullptr, nullptr, c.vocab, H, false, head.w, stream);
    head.alg_bytes = alg(c.vocab, H);
    head.n_total = c.vocab;
    head.k = H;
    logit_scale = vec(2, c.ls_lo, c.ls_hi, c.vocab);
    XTG_REQUIRE(cursor == arena + arena_bytes, "weight arena size mismatch");
    // RoPE inverse frequencies, computed as the reference does on the host: 1 / theta^(2i / d) in FP32
    const int half = c.head_dim / 2;
    std::vector<float> inv(2 * half);
    const float th[2] = {c.theta_sliding, c.theta_global};
    for (int t = 0; t < 2; ++t)
      for (int i = 0; i < half; ++i) inv[t * half + i] = 1.f / std::pow(th[t], float(2 * i) / float(c.head_dim));
    inv_freq = walloc<float>(inv.size());
    XTG_CUDA(cudaMemcpyAsync(inv_freq, inv.data(), inv.size() * sizeof(float), cudaMemcpyHostToDevice, stream));
    XTG_CUDA(cudaStreamSynchronize(stream));
    make_outs();
    cudaFree(raw);
    cudaFree(codes_a);
    cudaFree(scales_a);
    cudaFree(codes_b);
    cudaFree(scales_b);
    cudaFree(gdev);
    cudaFree(amax);
  }

  // ---- a Dory checkpoint (packs/dory/dory.cpp:316-439): ModelOpt NVFP4 rows repacked into tensor-core units ----
  // Weights of a recurrent sublayer are packed once and read by every loop's evaluation; each attention evaluation
  // keeps its own KV instance (per_loop). The stored scales are folded as the reference folds them: logit scale /
  // init_range, |alpha| * alpha_init / init_range, (sqk sqrt(head_dim) / init_range)^2, (s_gate sqrt(gate_init) /
  // init_range)^2, suv * sqrt(hidden).
  void load_checkpoint() {
    const DoryConfig dc = read_dory_config(c.path);
    SafeTensors st(c.path + "/model.safetensors");
    const int H = c.hidden, F = c.ffn, Q = c.heads * c.head_dim, KV = c.kv_heads * c.head_dim, V = c.vocab;
    const int ne = c.n_evals(), layers = (int)c.kinds.size();
    const int tq = packed_tiles(Q, false), tk = packed_tiles(KV, false);
    int64_t total = 0;
    for (int l = 0; l < layers; ++l)
      total += c.kinds[l] == 0 ? packed_bytes(F, H, true) + packed_bytes(H, F, false)
                               : (int64_t)(2 * tq + 2 * tk) * packed_kblocks(H) * kPackUnitBytes + packed_bytes(H, Q, false);
    if (!c.head_bf16) total += packed_bytes(V, H, false);
    arena_bytes = total;
    arena = walloc<uint8_t>((size_t)total);
    const int64_t max_elems = std::max<int64_t>({(int64_t)F * H, (int64_t)Q * H, c.head_bf16 ? 0 : (int64_t)V * H});
    uint8_t *codes_a = nullptr, *scales_a = nullptr, *codes_b = nullptr, *scales_b = nullptr;
    XTG_CUDA(cudaMalloc(&codes_a, max_elems / 2));
    XTG_CUDA(cudaMalloc(&scales_a, max_elems / 16));
    XTG_CUDA(cudaMalloc(&codes_b, (int64_t)F * H / 2));
    XTG_CUDA(cudaMalloc(&scales_b, (int64_t)F * H / 16));
    struct Temps {
      std::vector<void*> p;
      ~Temps() {
        for (void* q : p) cudaFree(q);
      }
    } temps;
    temps.p = {codes_a, scales_a, codes_b, scales_b};
    auto h2d = [&](void* dst, const TensorView& t) {
      XTG_CUDA(cudaMemcpyAsync(dst, t.data, t.bytes, cudaMemcpyHostToDevice, stream));
    };
    // an NVFP4 weight's codes and scales into (codes, scales); its global scale
    auto nvfp4 = [&](const std::string& name, int n_out, int k, uint8_t* codes, uint8_t* scales) {
      h2d(codes, st.get(name + ".weight", "U8", {n_out, k / 2}));
      h2d(scales, st.get(name + ".weight_scale", "F8_E4M3", {n_out, k / 16}));
      const TensorView& g = st.get(name + ".weight_scale_2", "F32", {});
      float v;
      std::memcpy(&v, g.data, 4);
      XTG_CUDA(cudaStreamSynchronize(stream));   // the temporaries are reused by the next weight
      return v;
    };
    auto bf16_vec = [&](const std::string& name, int n) {
      const TensorView& t = st.get(name, "BF16", {n});
      std::vector<float> v(n);
      for (int i = 0; i < n; ++i) {
        uint16_t hb;
        std::memcpy(&hb, t.data + 2 * i, 2);
        v[i] = bf16_bits_f32(hb);
      }
      return v;
    };
    auto wupload = [&](const std::vector<float>& v) {
      float* d = walloc<float>(v.size());
      XTG_CUDA(cudaMemcpyAsync(d, v.data(), v.size() * sizeof(float), cudaMemcpyHostToDevice, stream));
      XTG_CUDA(cudaStreamSynchronize(stream));
      return d;
    };
    uint8_t* cursor = arena;
    auto place = [&](Linear& L, int tiles, int kblocks, int max_split = 8, int max_tpc = 1 << 20) {
      L.w = cursor;
      L.tiles = tiles;
      L.kblocks = kblocks;
      L.bytes = (int64_t)tiles * kblocks * kPackUnitBytes;
      L.plan = plan_gemv(tiles, kblocks, num_sms, max_split, max_tpc);
      cursor += L.bytes;
    };
    auto alg = [](int n, int k) { return (int64_t)n * k / 2 + (int64_t)n * k / 16 + 4; };
    const float alpha_scale = dc.alpha_init / dc.init_range;
    const float sqk_factor = std::sqrt(float(c.head_dim)) / dc.init_range;
    const float gate_factor = std::sqrt(dc.gate_init) / dc.init_range;
    const float suv_factor = std::sqrt(float(H));
    proj_ld = 2 * Q + 2 * KV;
    evals.resize(ne);
    std::vector<int> first(layers, -1);
    int n_attn = 0;
    for (int e = 0; e < ne; ++e) {
      Eval& E = evals[e];
      const int l = c.phys(e);
      if (first[l] >= 0) {   // a later loop of a recurrent sublayer: the same weights
        E = evals[first[l]];
        if (E.kind != 0) E.cache = n_attn++;
        continue;
      }
      first[l] = e;
      E.kind = c.kinds[l];
      const std::string p = "backbone.layers." + std::to_string(l) + ".";
      std::vector<float> lr = bf16_vec(p + (E.kind == 0 ? "mlp_alpha" : "attn_alpha"), H);
      for (float& x : lr) x = std::fabs(x * alpha_scale);
      E.lr = wupload(lr);
      if (E.kind == 0) {
        std::vector<float> sg = bf16_vec(p + "mixer.suv_gate", F), su = bf16_vec(p + "mixer.suv_up", F);
        for (float& x : sg) x *= suv_factor;
        for (float& x : su) x *= suv_factor;
        E.sg = wupload(sg);
        E.su = wupload(su);
        place(E.gu, packed_tiles(F, true), packed_kblocks(H), 8, 1);
        E.gu.g0 = nvfp4(p + "mixer.gate_proj", F, H, codes_a, scales_a);
        E.gu.g1 = nvfp4(p + "mixer.up_proj", F, H, codes_b, scales_b);
        pack_nvfp4(codes_a, scales_a, codes_b, scales_b, F, H, true, E.gu.w, stream);
        E.gu.alg_bytes = 2 * alg(F, H);
        E.gu.n_total = 2 * F;
        E.gu.k = H;
        place(E.down, packed_tiles(H, false), packed_kblocks(F));
        E.down.g0 = nvfp4(p + "mixer.down_proj", H, F, codes_a, scales_a);
        pack_nvfp4(codes_a, scales_a, nullptr, nullptr, H, F, false, E.down.w, stream);
        E.down.alg_bytes = alg(H, F);
        E.down.n_total = H;
        E.down.k = F;
      } else {
        std::vector<float> qs = bf16_vec(p + "mixer.sqk", Q), gs = bf16_vec(p + "mixer.s_gate", Q);
        for (float& x : qs) x = (x * sqk_factor) * (x * sqk_factor);
        for (float& x : gs) x = (x * gate_factor) * (x * gate_factor);
        E.qscale = wupload(qs);
        E.gscale = wupload(gs);
        E.theta = E.kind == 2 ? 1 : 0;
        E.cache = n_attn++;
        const int kblocks = packed_kblocks(H);
        place(E.qkvg, 2 * tq + 2 * tk, kblocks);
        const int n_out[4] = {Q, KV, KV, Q};
        const char* names[4] = {"mixer.q_proj", "mixer.k_proj", "mixer.v_proj", "mixer.g_proj"};
        int tile0 = 0;
        for (int j = 0; j < 4; ++j) {
          E.gq[j] = nvfp4(p + names[j], n_out[j], H, codes_a, scales_a);
          pack_nvfp4(codes_a, scales_a, nullptr, nullptr, n_out[j], H, false,
                     E.qkvg.w + (int64_t)tile0 * kblocks * kPackUnitBytes, stream);
          tile0 += packed_tiles(n_out[j], false);
          E.qkvg.alg_bytes += alg(n_out[j], H);
        }
        E.qkvg.n_total = 2 * Q + 2 * KV;
        E.qkvg.k = H;
        place(E.o, packed_tiles(H, false), packed_kblocks(Q));
        E.o.g0 = nvfp4(p + "mixer.o_proj", H, Q, codes_a, scales_a);
        pack_nvfp4(codes_a, scales_a, nullptr, nullptr, H, Q, false, E.o.w, stream);
        E.o.alg_bytes = alg(H, Q);
        E.o.n_total = H;
        E.o.k = Q;
      }
    }
    // the embedding table and the head (untied, packs/dory/dory.cpp:322-327)
    embed_bf16 = walloc<uint16_t>((size_t)V * H);
    h2d(embed_bf16, st.get("backbone.embeddings.weight", "BF16", {V, H}));
    const TensorView& lm = st.get("lm_head.weight", "BF16", {V, H});
    head.tiles = packed_tiles(V, false);
    head.kblocks = packed_kblocks(H);
    head.n_total = V;
    head.k = H;
    if (c.head_bf16) {
      head_w_bf16 = walloc<uint16_t>((size_t)V * H);
      h2d(head_w_bf16, lm);
      head.alg_bytes = (int64_t)V * H * 2;
      head.g0 = 1.f;
    } else {   // quantized here, as the synthetic model's head is
      uint16_t* raw = nullptr;
      float* gdev = nullptr;
      unsigned int* amax = nullptr;
      XTG_CUDA(cudaMalloc(&raw, (size_t)V * H * 2));
      temps.p.push_back(raw);
      XTG_CUDA(cudaMalloc(&gdev, sizeof(float)));
      temps.p.push_back(gdev);
      XTG_CUDA(cudaMalloc(&amax, sizeof(unsigned int)));
      temps.p.push_back(amax);
      h2d(raw, lm);
      quantize_nvfp4(raw, V, H, codes_a, scales_a, gdev, amax, stream);
      place(head, head.tiles, head.kblocks, 1);
      pack_nvfp4(codes_a, scales_a, nullptr, nullptr, V, H, false, head.w, stream);
      XTG_CUDA(cudaMemcpyAsync(&head.g0, gdev, sizeof(float), cudaMemcpyDeviceToHost, stream));
      head.alg_bytes = alg(V, H);
    }
    std::vector<float> ls = bf16_vec("lm_head.logit_scale", V);
    for (float& x : ls) x /= dc.init_range;
    logit_scale = wupload(ls);
    XTG_REQUIRE(cursor == arena + arena_bytes, "weight arena size mismatch");
    const int half = c.head_dim / 2;
    std::vector<float> inv(2 * half);
    const float th[2] = {c.theta_sliding > 0 ? c.theta_sliding : 1e4f, c.theta_global > 0 ? c.theta_global : 1e4f};
    for (int t = 0; t < 2; ++t)
      for (int i = 0; i < half; ++i) inv[t * half + i] = 1.f / std::pow(th[t], float(2 * i) / float(c.head_dim));
    inv_freq = wupload(inv);
    XTG_CUDA(cudaStreamSynchronize(stream));
    make_outs();
  }

  // this session's output descriptors of the STORE / q|k|v GEMVs (they point into its own activation buffers)
  static std::vector<TileOut> tile_outs(float* y, int ld, int n, float g) {
    std::vector<TileOut> v(packed_tiles(n, false));
    for (int t = 0; t < (int)v.size(); ++t) v[t] = TileOut{y + 128 * t, ld, std::min(128, n - 128 * t), g, g};
    return v;
  }

  void make_outs() {
    const int H = c.hidden, Q = c.heads * c.head_dim, KV = c.kv_heads * c.head_dim;
    for (Eval& E : evals) {
      if (E.kind == 0) {
        E.down.outs = upload(tile_outs(o, H, H, E.down.g0));
        continue;
      }
      std::vector<TileOut> outs;
      const int n_out[4] = {Q, KV, KV, Q};
      const int col[4] = {0, Q, Q + KV, Q + 2 * KV};
      for (int j = 0; j < 4; ++j)
        for (const TileOut& t : tile_outs(proj + col[j], proj_ld, n_out[j], E.gq[j])) outs.push_back(t);
      E.qkvg.outs = upload(outs);
      E.o.outs = upload(tile_outs(o, H, H, E.o.g0));
    }
  }

  // A session over another's weights (xtg_cuda_open_shared): the model's device blocks are shared, the output
  // descriptors are this session's own.
  void share_model(const xtg_cuda& m) {
    wmem = m.wmem;
    arena = m.arena;
    arena_bytes = m.arena_bytes;
    evals = m.evals;
    head = m.head;
    logit_scale = m.logit_scale;
    embed_bf16 = m.embed_bf16;
    head_w_bf16 = m.head_w_bf16;
    inv_freq = m.inv_freq;
    proj_ld = m.proj_ld;
    make_outs();
  }

  template <class T>
  T* upload(const std::vector<T>& v) {
    T* p = dalloc<T>(v.size(), false);
    XTG_CUDA(cudaMemcpyAsync(p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice, stream));
    XTG_CUDA(cudaStreamSynchronize(stream));   // the host vector goes out of scope
    return p;
  }

  void alloc_activations() {
    const int H = c.hidden, F = c.ffn, Q = c.heads * c.head_dim, KV = c.kv_heads * c.head_dim;
    params_dev = dalloc<StepParams>(1);
    XTG_CUDA(cudaMallocHost(&params_host, sizeof(StepParams)));
    std::memset(params_host, 0, sizeof(StepParams));
    h = dalloc<float>((size_t)kMaxRows * H);
    state = dalloc<float>((size_t)kMaxRows * H);
    input = dalloc<float>((size_t)kMaxRows * H);
    o = dalloc<float>((size_t)kMaxRows * H);
    proj = dalloc<float>((size_t)kMaxRows * (2 * Q + 2 * KV));
    xb = dalloc<uint8_t>((size_t)digit_bytes(H));
    ab = dalloc<uint8_t>((size_t)digit_bytes(Q));
    vb = dalloc<uint8_t>((size_t)digit_bytes(F));
    auto empty_pre = [&](int k) {   // rows never written: all-zero digits that never set a slice's prescale
      const std::vector<float> v((size_t)packed_kblocks(k) * 4 * kMaxRows, kEmptyPrescale);
      return upload(v);
    };
    xb_pre = empty_pre(H);
    ab_pre = empty_pre(Q);
    vb_pre = empty_pre(F);
    q_prep = dalloc<float>((size_t)kMaxRows * Q);
    k_new = dalloc<float>((size_t)kMaxRows * KV);
    v_new = dalloc<float>((size_t)kMaxRows * KV);
    asum = dalloc<float>((size_t)c.heads * kMaxRows);
    vsum = dalloc<float>((size_t)packed_tiles(F, true) * 8 * kMaxRows);
    rsum = dalloc<float>((size_t)2 * num_sms * kMaxRows * 5);   // a split GEMV has at most 2 CTAs per SM
    logits = dalloc<float>((size_t)kMaxRows * c.vocab);
    XTG_CUDA(cudaMallocHost(&logits_host, (size_t)kMaxRows * c.vocab * sizeof(float)));
    cand = dalloc<ArgCand>((size_t)packed_tiles(c.vocab, false) * kMaxRows);
    argmax = dalloc<int32_t>(kMaxRows);
    argmax_val = dalloc<float>(kMaxRows);
    rope_cos = dalloc<float>((size_t)2 * kMaxRows * (c.head_dim / 2));
    rope_sin = dalloc<float>((size_t)2 * kMaxRows * (c.head_dim / 2));
    dev_err = dalloc<int>(1);
    XTG_CUDA(cudaMallocHost(&err_host, sizeof(int)));
    *err_host = 0;
    XTG_CUDA(cudaEventCreateWithFlags(&err_ev, cudaEventDisableTiming));
    for (cudaEvent_t& e : row_ev) XTG_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    // the attention runs 2 CTAs per SM (1 at head dim 256): a global cache over every CTA slot, a ring one 64-slot
    // chunk per CTA
    const int per_sm = attention_ctas_per_sm(c.head_dim);
    splits_g = c.splits_global > 0 ? c.splits_global : std::max(1, std::min(256, per_sm * num_sms / c.kv_heads));
    splits_g = std::min(splits_g, 256 / c.kv_world);   // the combine takes at most 256 parts
    splits_r = c.splits_ring > 0 ? c.splits_ring : std::max(1, std::min(256, (int)(c.ring / 64)));
    part = dalloc<float>(
        (size_t)attention_part_floats(c.kv_heads, std::max(splits_g * c.kv_world, splits_r), c.head_dim));
    ring_pos_dev = dalloc<int32_t>(c.ring);
    ring_pos.assign(c.ring, -1);
    std::vector<int32_t> neg(c.ring, -1);
    XTG_CUDA(cudaMemcpyAsync(ring_pos_dev, neg.data(), neg.size() * 4, cudaMemcpyHostToDevice, stream));
    XTG_CUDA(cudaStreamSynchronize(stream));
  }

  void alloc_caches() {
    for (int e = 0; e < c.n_evals(); ++e)
      if (evals[e].kind != 0)
        kv.push_back(alloc_kv(c.kv_heads, c.head_dim, evals[e].kind == 1 ? c.ring : c.context, evals[e].kind == 1,
                              stream));
    n_glob = 0;
    for (int e = 0; e < c.n_evals(); ++e) n_glob += evals[e].kind == 2;
    snaps.resize(c.snapshots);
    kv_seq_dev = dalloc<KvSeq>(kv.size());
    upload_kv_seq();
  }

  void upload_kv_seq() {
    std::vector<KvSeq> v(kv.size());
    for (size_t i = 0; i < kv.size(); ++i)
      v[i] = KvSeq{kv[i].kc, kv[i].vc, kv[i].ks, kv[i].vs, kv[i].ring ? ring_pos_dev : nullptr, kv[i].slots};
    if (v.empty()) return;
    XTG_CUDA(cudaMemcpyAsync(kv_seq_dev, v.data(), v.size() * sizeof(KvSeq), cudaMemcpyHostToDevice, stream));
    XTG_CUDA(cudaStreamSynchronize(stream));
  }

  // ---- the step ----

  void mark(int cls, bool begin) {
    if (!prof) return;
    if (begin) {
      cudaEvent_t a, b;
      XTG_CUDA(cudaEventCreate(&a));
      XTG_CUDA(cudaEventCreate(&b));
      prof->push_back({a, b});
      prof_cls->push_back(cls);
      XTG_CUDA(cudaEventRecord(a, stream));
    } else {
      XTG_CUDA(cudaEventRecord(prof->back().second, stream));
    }
  }

  GemvArgs gemv_args(const Linear& L) {
    GemvArgs a = {};
    a.w = L.w;
    a.tiles = L.tiles;
    a.kblocks = L.kblocks;
    a.m_dev = &params_dev->m;
    a.err = dev_err;
    a.outs = L.outs;
    return a;
  }

  // a GEMV of activation digits (xb, xb_pre), with an optional justnorm row scale from sumsq (STORE)
  // whether xb holds the digits of the residual stream (written by a residual update: one prescale for every group)
  // rather than the embedding's
  bool xb_unit = false;

  void gemv(const Linear& L, int epi, GemvArgs a, const uint8_t* in, const float* in_pre, bool pdl,
            const float* sumsq = nullptr, int nparts = 0) {
    a.xb = in;
    a.xb_pre = in_pre;
    a.xb_fixed = (in == xb && xb_unit) ? kUnitPrescale : 0.f;
    a.sumsq = sumsq;
    a.nparts = nparts;
    a.l2_first = c.l2_first ? 1 : 0;
    mark(kClsGemv, true);
    launch_gemv(epi, a, L.plan, stream, pdl);
    mark(kClsGemv, false);
  }

  void enqueue_step(bool pdl) {
    const int H = c.hidden, F = c.ffn, Q = c.heads * c.head_dim;
    int glob = 0;   // global layers enqueued so far
    mark(kClsSmall, true);
    EmbedArgs ea = {};
    ea.params = params_dev;
    ea.head = head.w;
    ea.kblocks = head.kblocks;
    ea.global = head.g0;
    ea.table = embed_bf16;
    ea.hidden = H;
    ea.h = h;
    ea.xb = xb;
    ea.xb_pre = xb_pre;
    ea.inv_freq = inv_freq;
    ea.n_thetas = 2;
    ea.rope_half = c.head_dim / 2;
    ea.rope_cos = rope_cos;
    ea.rope_sin = rope_sin;
    ea.ring_pos = ring_pos_dev;
    ea.ring = c.ring;
    launch_embed(ea, stream, false);
    xb_unit = false;
    mark(kClsSmall, false);
    // the O / down projection feeds the slerp update with per-CTA row sums when split 4 or 8 ways
    auto with_rsum = [&](const Linear& L, const float* lr) {
      GemvArgs a = gemv_args(L);
      if (L.plan.split == 4 || L.plan.split == 8) {
        a.rsum = rsum;
        a.rs_h = h;
        a.rs_lr = lr;
        a.rs_ld = H;
      }
      return a;
    };
    auto resid = [&](int mode, const float* lr, const Linear* producer = nullptr) {
      ResidArgs r = {};
      r.mode = mode;
      r.params = params_dev;
      r.hidden = H;
      r.h = h;
      r.o = o;
      r.lr = lr;
      r.state = state;
      r.input = input;
      r.xb = xb;
      r.xb_pre = xb_pre;
      if (producer && (producer->plan.split == 4 || producer->plan.split == 8)) {
        r.rsum = rsum;
        r.nparts = producer->plan.grid;
      }
      mark(kClsSmall, true);
      launch_resid(r, stream, pdl);
      mark(kClsSmall, false);
      xb_unit = true;
    };
    static const char* const kKindName[3] = {"mlp", "sliding attention", "global attention"};
    auto sublayer = [&](int e) {
      const Eval& E = evals[e];
      char label[64];
      if (c.nvtx) std::snprintf(label, sizeof(label), "eval %d: %s", e, kKindName[E.kind]);
      NvtxRange range(c.nvtx, label);
      if (E.kind == 0) {
        GemvArgs a = gemv_args(E.gu);
        a.g_gate = E.gu.g0;
        a.g_up = E.gu.g1;
        a.sg = E.sg;
        a.su = E.su;
        a.features = F;
        a.vb = vb;
        a.vb_pre = vb_pre;
        a.vsum = vsum;
        gemv(E.gu, kEpiSwiglu, a, xb, xb_pre, pdl);
        gemv(E.down, kEpiStore, with_rsum(E.down, E.lr), vb, vb_pre, pdl, vsum, E.gu.tiles * E.gu.plan.split);
        resid(kResidSlerp, E.lr, &E.down);
        return;
      }
      const KvInst& K = kv[E.cache];
      if (c.head_dim != 128) {
        // a head spans two 128-row tiles: the projection's outputs, then RoPE, the norms and the KV store per head
        gemv(E.qkvg, kEpiStore, gemv_args(E.qkvg), xb, xb_pre, pdl);
        QkvPrepArgs qa = {};
        qa.params = params_dev;
        qa.nseq = 1;
        qa.proj = proj;
        qa.proj_ld = proj_ld;
        qa.ksplit = 1;
        qa.heads = c.heads;
        qa.kv_heads = c.kv_heads;
        qa.rope_cos = rope_cos;
        qa.rope_sin = rope_sin;
        qa.theta = E.theta;
        qa.qscale = E.qscale;
        qa.q_out = q_prep;
        qa.k_out = k_new;
        qa.v_out = v_new;
        qa.seqs = kv_seq_dev + E.cache;
        qa.ring = K.ring ? 1 : 0;
        qa.dtype = c.kv_dtype;
        qa.err = dev_err;
        qa.pdl = pdl ? 1 : 0;
        qa.head_dim = c.head_dim;
        mark(kClsSmall, true);
        launch_qkv_prep(qa, stream);
        mark(kClsSmall, false);
      } else {
        GemvArgs g = gemv_args(E.qkvg);
        g.q_tiles = c.heads;
        g.kv_tiles = c.kv_heads;
        g.rope_cos = rope_cos + E.theta * kMaxRows * 64;
        g.rope_sin = rope_sin + E.theta * kMaxRows * 64;
        g.qscale = E.qscale;
        g.q_out = q_prep;
        g.k_out = k_new;
        g.v_out = v_new;
        g.kc = K.kc;
        g.vc = K.vc;
        g.ks = K.ks;
        g.vs = K.vs;
        g.slots = K.slots;
        g.ring = K.ring ? 1 : 0;
        g.dtype = c.kv_dtype;
        g.pos0_dev = &params_dev->pos0;
        gemv(E.qkvg, kEpiQkv, g, xb, xb_pre, pdl);
      }
      AttnArgs at = {};
      at.head_dim = c.head_dim;
      at.q = q_prep;
      at.k = k_new;
      at.v = v_new;
      at.kc = K.kc;
      at.vc = K.vc;
      at.ks = K.ks;
      at.vs = K.vs;
      at.slots = K.slots;
      at.ring = K.ring ? 1 : 0;
      at.ring_pos = ring_pos_dev;
      at.dtype = c.kv_dtype;
      at.window = K.ring ? c.window : 0;
      at.scale = 1.f / std::sqrt((float)c.head_dim);
      at.params = params_dev;
      at.heads = c.heads;
      at.kv_heads = c.kv_heads;
      at.splits = K.ring ? splits_r : splits_g;
      const bool shard = !K.ring && comm;   // this process attends its share of the global cache's chunks
      const bool peer = shard && xbuf;      // ... and merges its splits before the peers' partials come in
      at.split0 = shard ? c.kv_rank * splits_g : 0;
      at.splits_total = shard ? splits_g * c.kv_world : at.splits;
      at.part_local = peer ? 1 : 0;
      at.part = part;
      at.err = dev_err;
      at.l2_first = (!K.ring && c.l2_first) ? 1 : 0;
      mark(kClsAttn, true);
      launch_attention(at, stream, pdl);
      mark(kClsAttn, false);
      if (shard && !peer) {   // in place: this process's partials are the block at its split offset
        const size_t n = (size_t)attention_part_floats(c.kv_heads, splits_g);
        nccl_check(nccl_api().all_gather(part + c.kv_rank * n, part, n, ncclFloat32, comm, stream), "ncclAllGather");
      }
      CombineArgs cb = {};
      cb.part = part;
      cb.err = dev_err;
      cb.head_dim = c.head_dim;
      if (peer) {
        cb.x = xchg;
        cb.x.g = glob++;
      }
      cb.q = q_prep;
      cb.k = k_new;
      cb.v = v_new;
      cb.scale = at.scale;
      cb.window = at.window;
      cb.splits = peer ? at.splits : at.splits_total;
      cb.heads = c.heads;
      cb.kv_heads = c.kv_heads;
      cb.params = params_dev;
      cb.gate = proj + Q + 2 * c.kv_heads * c.head_dim;
      cb.gate_ld = proj_ld;
      cb.gscale = E.gscale;
      cb.ab = ab;
      cb.ab_pre = ab_pre;
      cb.asum = asum;
      mark(kClsCombine, true);
      launch_attn_combine(cb, stream, pdl);
      mark(kClsCombine, false);
      gemv(E.o, kEpiStore, with_rsum(E.o, E.lr), ab, ab_pre, pdl, asum, c.heads);
      resid(kResidSlerp, E.lr, &E.o);
    };
    int e = 0;
    for (int l = 0; l < c.n_in; ++l) sublayer(e++);
    if (c.loops > 0) {
      resid(kResidLoopBegin, nullptr);
      for (int i = 0; i < c.loops; ++i) {
        for (int r = 0; r < c.n_rec; ++r) sublayer(e++);
        resid(i + 1 < c.loops ? kResidLoopNext : kResidLoopEnd, nullptr);
      }
    }
    for (int l = 0; l < c.n_out; ++l) sublayer(e++);
    if (head_w_bf16) {   // a checkpoint's BF16 head over the f32 rows
      HeadBf16Args hb = {};
      hb.x = h;
      hb.m_dev = &params_dev->m;
      hb.w = head_w_bf16;
      hb.vocab = c.vocab;
      hb.hidden = H;
      hb.logit_scale = logit_scale;
      hb.logits = logits;
      hb.cand = cand;
      hb.err = dev_err;
      mark(kClsGemv, true);
      launch_head_bf16(hb, num_sms, stream, pdl);
      mark(kClsGemv, false);
    } else {
      GemvArgs a = gemv_args(head);
      a.outs = nullptr;
      a.g_head = head.g0;
      a.logit_scale = logit_scale;
      a.logits = logits;
      a.vocab = c.vocab;
      a.cand = cand;
      gemv(head, kEpiHead, a, xb, xb_pre, pdl);
    }
    mark(kClsSmall, true);
    launch_argmax(cand, head.tiles, params_dev, argmax, argmax_val, epoch, stream, pdl);
    mark(kClsSmall, false);
  }

  // The split-KV peer exchange: allocate this process's exchange slots, export them by CUDA IPC, and map the peers'
  // (the handles travel by an NCCL all-gather, which also checks that every process sized them alike).
  void open_peer_exchange() {
    struct Record {
      cudaIpcMemHandle_t handle;
      uint64_t bytes;
      int32_t n_glob, splits;
    };
    const int w = c.kv_world, r = c.kv_rank;
    if (w > kMaxKvWorld) throw CudaError("split-KV: at most 8 processes");
    const size_t bytes = (size_t)2 * w * kMaxRows * c.heads * 130 * sizeof(uint64_t);
    XTG_CUDA(cudaMalloc(&xbuf, bytes));
    XTG_CUDA(cudaMemset(xbuf, 0, bytes));
    epoch = dalloc<uint32_t>(1);
    XTG_CUDA(cudaDeviceSynchronize());   // zeroed before any peer can map it
    Record mine = {};
    XTG_CUDA(cudaIpcGetMemHandle(&mine.handle, xbuf));
    mine.bytes = bytes;
    mine.n_glob = n_glob;
    mine.splits = splits_g;
    std::vector<Record> all(w);
    Record* stage = dalloc<Record>((size_t)w, false);
    XTG_CUDA(cudaMemcpy(stage + r, &mine, sizeof(Record), cudaMemcpyHostToDevice));
    nccl_check(nccl_api().all_gather(stage + r, stage, sizeof(Record), ncclUint8, comm, stream), "ncclAllGather");
    XTG_CUDA(cudaStreamSynchronize(stream));
    XTG_CUDA(cudaMemcpy(all.data(), stage, sizeof(Record) * w, cudaMemcpyDeviceToHost));
    for (int t = 0; t < w; ++t) {
      if (all[t].bytes != bytes || all[t].n_glob != n_glob || all[t].splits != splits_g)
        throw CudaError("split-KV: process " + std::to_string(t) + " has another model, context or split count");
      void* base = xbuf;
      if (t != r) {
        XTG_CUDA(cudaIpcOpenMemHandle(&peer_base[t], all[t].handle, cudaIpcMemLazyEnablePeerAccess));
        base = peer_base[t];
      }
      xchg.slot[t] = static_cast<uint64_t*>(base);
    }
    xchg.epoch = epoch;
    xchg.wait_ns = (uint64_t)c.kv_wait_ms * 1000000ull;
    xchg.world = w;
    xchg.rank = r;
    xchg.n_g = n_glob;
  }

  void capture() {
    if (exec) return;
    cudaGraph_t g = nullptr;
    XTG_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
    try {
      XTG_CUDA(cudaMemcpyAsync(params_dev, params_host, sizeof(StepParams), cudaMemcpyHostToDevice, stream));
      enqueue_step(c.pdl);
    } catch (...) {
      cudaStreamEndCapture(stream, &g);
      if (g) cudaGraphDestroy(g);
      throw;
    }
    XTG_CUDA(cudaStreamEndCapture(stream, &g));
    cudaError_t e = cudaGraphInstantiate(&exec, g, 0);
    cudaGraphDestroy(g);
    XTG_CUDA(e);
  }

  // One step of m rows at n_past (params_host filled), without the host bookkeeping.
  void launch_step() {
    if (c.graph) {
      capture();
      XTG_CUDA(cudaGraphLaunch(exec, stream));
    } else {
      XTG_CUDA(cudaMemcpyAsync(params_dev, params_host, sizeof(StepParams), cudaMemcpyHostToDevice, stream));
      enqueue_step(c.pdl);
    }
  }

  void set_params(const int32_t* tokens, int m) {
    std::memset(params_host, 0, sizeof(StepParams));
    for (int i = 0; i < m; ++i) params_host->tokens[i] = tokens[i];
    params_host->m = m;
    params_host->pos0 = n_past;
  }

  void commit(int m) {
    for (int r = 0; r < m; ++r) ring_pos[(n_past + r) % c.ring] = n_past + r;
    n_past += m;
  }

  // forward() in three parts, so that several sessions' steps can be in flight at once (xtg_cuda_forward_batch):
  // check the call (nothing changes on failure), enqueue one step of up to decode_rows tokens without waiting, then
  // wait for it, commit it and hand its logits out.
  void check_tokens(const int32_t* tokens, int n) const {
    for (int i = 0; i < n; ++i)
      if (tokens[i] < 0 || tokens[i] >= c.vocab)
        throw CudaError("token " + std::to_string(tokens[i]) + " out of range");
    if (n_past + n > c.context)
      throw CudaError("context full: " + std::to_string(n_past) + " + " + std::to_string(n) + " tokens (" +
                      std::to_string(c.context) + ")");
  }

  void drop_snapshots_past() {
    for (Snap& s : snaps)   // a snapshot past this point no longer matches what the caches will hold
      if (s.pos > n_past) s.pos = -1;
  }

  struct Chunk {
    int off, m, r0;
  };

  Chunk enqueue_chunk(const int32_t* tokens, int n, int off, int want, bool copy) {
    const int m = std::min(c.decode_rows, n - off);
    set_params(tokens + off, m);
    launch_step();
    const int r0 = want == 2 ? 0 : (want == 1 && off + m == n ? m - 1 : m);
    // the error word first, then each row with its own event: the callback of a row runs while the next copies
    XTG_CUDA(cudaMemcpyAsync(err_host, dev_err, sizeof(int), cudaMemcpyDeviceToHost, stream));
    XTG_CUDA(cudaEventRecord(err_ev, stream));
    if (copy)
      for (int r = r0; r < m; ++r) {
        XTG_CUDA(cudaMemcpyAsync(logits_host + (size_t)r * c.vocab, logits + (size_t)r * c.vocab,
                                 (size_t)c.vocab * sizeof(float), cudaMemcpyDeviceToHost, stream));
        XTG_CUDA(cudaEventRecord(row_ev[r], stream));
      }
    return Chunk{off, m, r0};
  }

  // false: a bounded device wait gave up, the step's results are not to be trusted (not committed, no callback)
  bool finish_chunk(const Chunk& k, xtg_cuda_logits_fn fn, void* user, int row_base) {
    XTG_CUDA(cudaEventSynchronize(err_ev));
    if (*err_host) {
      XTG_CUDA(cudaStreamSynchronize(stream));   // the row copies in flight
      *err_host = 0;
      XTG_CUDA(cudaMemsetAsync(dev_err, 0, sizeof(int), stream));
      return false;
    }
    commit(k.m);
    last_rows = k.m;
    if (fn)
      for (int i = k.r0; i < k.m; ++i) {
        XTG_CUDA(cudaEventSynchronize(row_ev[i]));
        fn(row_base + k.off + i, logits_host + (size_t)i * c.vocab, user);
      }
    return true;
  }

  // Rows n <= decode_rows run the verify step; longer inputs go in prompt chunks of up to prefill_rows (64: the
  // ring's slack past the window) through the batched step, the rest in verify steps (xtg_npu.cpp:346-360).
  void forward(const int32_t* tokens, int n, int want, xtg_cuda_logits_fn fn, void* user) {
    if (n <= 0) return;
    check_tokens(tokens, n);
    drop_snapshots_past();
    const int pr = prefill_rows(this);
    for (int off = 0; off < n;) {
      const int left = n - off;
      if (pr > c.decode_rows && left > c.decode_rows) {
        const int m = std::min(pr, left);
        prefill_chunk(this, tokens + off, m, want, off, n, fn, user);
        off += m;
        continue;
      }
      const Chunk k = enqueue_chunk(tokens, n, off, want, fn != nullptr);
      if (!finish_chunk(k, fn, user, 0)) throw CudaError("a device wait timed out during the step (results discarded)");
      off += c.decode_rows;
    }
  }

  bool rewind(int64_t to) {
    if (to < 0 || to > n_past) return false;
    for (int64_t q = std::max<int64_t>(0, to - c.window + 1); q < to; ++q)
      if (ring_pos[q % c.ring] != q) return false;
    n_past = to;
    return true;
  }

  void snapshot(int slot) {
    if (slot < 0 || slot >= (int)snaps.size()) return;
    Snap& s = snaps[slot];
    if (s.rings.empty())
      for (const KvInst& k : kv)
        if (k.ring) s.rings.push_back(alloc_kv(c.kv_heads, c.head_dim, k.slots, true, stream));
    size_t i = 0;
    for (const KvInst& k : kv)
      if (k.ring) copy_kv(k, s.rings[i++], c.kv_heads, c.head_dim, k.slots, stream);
    XTG_CUDA(cudaStreamSynchronize(stream));
    s.ring_pos = ring_pos;
    s.pos = n_past;
  }

  bool restore(int slot) {
    if (slot < 0 || slot >= (int)snaps.size() || snaps[slot].pos < 0) return false;
    Snap& s = snaps[slot];
    size_t i = 0;
    for (KvInst& k : kv)
      if (k.ring) copy_kv(s.rings[i++], k, c.kv_heads, c.head_dim, k.slots, stream);
    ring_pos = s.ring_pos;
    upload_ring_pos();
    n_past = s.pos;
    return true;
  }

  void upload_ring_pos() {
    std::vector<int32_t> rp(ring_pos.begin(), ring_pos.end());
    XTG_CUDA(cudaMemcpyAsync(ring_pos_dev, rp.data(), rp.size() * 4, cudaMemcpyHostToDevice, stream));
    XTG_CUDA(cudaStreamSynchronize(stream));
  }

  void grow(int64_t ctx) {
    if (ctx < 64 || ctx % 64) throw CudaError("tier: a context of a multiple of 64 positions");
    if (ctx < n_past) throw CudaError("tier " + std::to_string(ctx) + " cannot hold " + std::to_string(n_past) +
                                      " positions");
    if (ctx == c.context) return;
    std::vector<KvInst> next;
    try {
      for (const KvInst& k : kv) {
        if (k.ring) continue;
        next.push_back(alloc_kv(c.kv_heads, c.head_dim, ctx, false, stream));
        copy_kv(k, next.back(), c.kv_heads, c.head_dim, n_past, stream);
      }
      XTG_CUDA(cudaStreamSynchronize(stream));
    } catch (...) {
      free_kv(next);
      throw;
    }
    size_t i = 0;
    for (KvInst& k : kv) {
      if (k.ring) continue;
      cudaFree(k.kc);
      cudaFree(k.vc);
      cudaFree(k.ks);
      cudaFree(k.vs);
      k = next[i++];
    }
    c.context = ctx;
    upload_kv_seq();
    ++generation;
    for (Snap& s : snaps)   // a smaller tier drops what it cannot hold
      if (s.pos > ctx) s.pos = -1;
    if (exec) {   // the graph holds the old caches' addresses
      cudaGraphExecDestroy(exec);
      exec = nullptr;
    }
  }

  void prefill_synthetic(int64_t n) {
    if (n < 0 || n > c.context) throw CudaError("prefill: " + std::to_string(n) + " positions do not fit the tier");
    for (size_t i = 0; i < kv.size(); ++i) {
      KvInst& k = kv[i];
      const int64_t filled = k.ring ? std::min<int64_t>(n, k.slots) : n;
      kv_prefill(c.seed, 500000 + 8 * (uint64_t)i, c.kvs_lo, c.kvs_hi, filled, c.kv_heads, c.head_dim, k.slots, k.kc,
                 k.vc, k.ks, k.vs, stream);
    }
    for (int r = 0; r < c.ring; ++r) {
      int64_t p = -1;
      if (n > 0) {
        const int64_t last = n - 1;
        p = last - ((last - r) % c.ring + c.ring) % c.ring;
      }
      ring_pos[r] = p;
    }
    upload_ring_pos();
    n_past = n;
    for (Snap& s : snaps) s.pos = -1;
  }

  int64_t kv_bytes() const {
    int64_t b = 0;
    for (const KvInst& k : kv) b += (int64_t)c.kv_heads * k.slots * (2 * c.head_dim + 8);
    return b;
  }

  int64_t step_bytes(int what, int m) const {
    const int H = c.hidden, Q = c.heads * c.head_dim;
    int64_t gemv = 0, attn = 0;
    auto act = [&](const Linear& L) { return (int64_t)m * L.k * 2 + (int64_t)m * L.n_total * 4; };
    for (const Eval& E : evals) {
      if (E.kind == 0) {
        gemv += E.gu.alg_bytes + act(E.gu) + E.down.alg_bytes + act(E.down);
      } else {
        gemv += E.qkvg.alg_bytes + act(E.qkvg) + E.o.alg_bytes + act(E.o);
        const int64_t keys = E.kind == 1 ? c.ring : n_past;
        attn += keys * c.kv_heads * (2 * c.head_dim + 8) + (int64_t)m * Q * 4 * 2;
      }
    }
    gemv += head.alg_bytes + act(head);
    (void)H;
    return what == 1 ? gemv : what == 2 ? attn : gemv + attn;
  }
};

// ---- the batched verify step (batch.h): S sessions over one weight set, one step for all of them ----
// Every projection is one tcgen05 GEMM over the S sessions' 8 S activation rows (the weights stream once per step for
// all of them; K split so that a GEMM of few weight tiles still spreads over the SMs); embedding, q / k / v
// preparation with the KV store, SwiGLU and the logit scale run as the batch kernels, the attention and its combine
// per sequence over that session's own caches (grid z = sequence), the nGPT residual updates per row. Each session
// keeps its caches, ring table, snapshots and position; its step is the same arithmetic as its own forward (the
// activations as the GEMM's 4 digits per value, one prescale per row). Captured once into a CUDA graph per set of
// sessions.
struct BatchStep {
  xtg_cuda* model = nullptr;   // the first session: the weights every session shares
  std::vector<xtg_cuda*> seqs;
  std::vector<uint64_t> gens;
  int S = 0, H = 0, F = 0, Q = 0, KV = 0, proj_ld = 0, splits_g = 1, splits_r = 1;
  cudaStream_t stream = nullptr;
  std::vector<void*> allocs;
  StepParams* params_dev = nullptr;
  StepParams* params_host = nullptr;
  float *h = nullptr, *state = nullptr, *input = nullptr, *o = nullptr, *proj = nullptr, *q_prep = nullptr;
  float *k_new = nullptr, *v_new = nullptr, *att = nullptr, *asum = nullptr, *gu = nullptr, *logits = nullptr;
  float *rope_cos = nullptr, *rope_sin = nullptr, *act_post = nullptr, *part = nullptr;
  uint8_t* act = nullptr;
  int32_t* argmax = nullptr;
  int32_t** ring_tab = nullptr;
  KvSeq* kvseq = nullptr;                    // [attention evaluations][S]
  std::vector<TileOut*> outs_a, outs_b;      // per evaluation: qkvg | gate/up, o | down
  TileOut* outs_head = nullptr;
  int* dev_err = nullptr;
  int* err_host = nullptr;
  cudaGraphExec_t exec = nullptr;
  static constexpr int kRows = 64;           // one GEMM activation tile
  bool distinct = true;                      // false: the row groups of one session's prompt chunk
  int ks_qkv = 2, ks_o = 6, ks_gu = 1, ks_down = 6;

  template <class T>
  T* alloc(size_t n) {
    void* p = nullptr;
    XTG_CUDA(cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)));
    allocs.push_back(p);
    XTG_CUDA(cudaMemsetAsync(p, 0, std::max<size_t>(n, 1) * sizeof(T), stream));
    return static_cast<T*>(p);
  }
  template <class T>
  T* upload(const std::vector<T>& v) {
    T* p = alloc<T>(v.size());
    XTG_CUDA(cudaMemcpyAsync(p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice, stream));
    XTG_CUDA(cudaStreamSynchronize(stream));
    return p;
  }

  ~BatchStep() {
    if (stream) cudaStreamSynchronize(stream);
    if (exec) cudaGraphExecDestroy(exec);
    for (void* p : allocs) cudaFree(p);
    if (params_host) cudaFreeHost(params_host);
    if (err_host) cudaFreeHost(err_host);
    if (stream) cudaStreamDestroy(stream);
  }

  // K parts of a GEMM over wtiles weight tiles: enough (weight tile, K part) pairs to cover the SMs
  static int ksplit_for(int wtiles, int kblocks, int sms) {
    return std::max(1, std::min(kblocks / 4, sms / std::max(1, wtiles)));
  }

  void build(const std::vector<xtg_cuda*>& sessions) {
    seqs = sessions;
    S = (int)seqs.size();
    model = seqs[0];
    const Config& c = model->c;
    H = c.hidden;
    F = c.ffn;
    Q = c.heads * c.head_dim;
    KV = c.kv_heads * c.head_dim;
    proj_ld = model->proj_ld;
    for (xtg_cuda* q : seqs) gens.push_back(q->generation);
    distinct = std::count(seqs.begin(), seqs.end(), seqs[0]) == 1;   // forward_batch never repeats a session
    XTG_CUDA(cudaSetDevice(c.device));
    XTG_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    const int sms = model->num_sms;
    const Eval* e_att = nullptr;
    const Eval* e_mlp = nullptr;
    for (const Eval& E : model->evals) (E.kind ? e_att : e_mlp) = &E;
    if (e_att) {
      ks_qkv = ksplit_for(e_att->qkvg.tiles, e_att->qkvg.kblocks, sms);
      ks_o = ksplit_for(e_att->o.tiles, e_att->o.kblocks, sms);
    }
    if (e_mlp) {
      ks_gu = ksplit_for(e_mlp->gu.tiles, e_mlp->gu.kblocks, sms);
      ks_down = ksplit_for(e_mlp->down.tiles, e_mlp->down.kblocks, sms);
    }
    XTG_CUDA(cudaMallocHost(&params_host, sizeof(StepParams) * S));
    std::memset(params_host, 0, sizeof(StepParams) * S);
    params_dev = alloc<StepParams>(S);
    const int R = kRows;
    h = alloc<float>((size_t)R * H);
    state = alloc<float>((size_t)R * H);
    input = alloc<float>((size_t)R * H);
    o = alloc<float>((size_t)std::max(ks_o, ks_down) * R * H);
    proj = alloc<float>((size_t)ks_qkv * R * proj_ld);
    q_prep = alloc<float>((size_t)R * Q);
    k_new = alloc<float>((size_t)R * KV);
    v_new = alloc<float>((size_t)R * KV);
    att = alloc<float>((size_t)R * Q);
    asum = alloc<float>((size_t)c.heads * R);
    gu = alloc<float>((size_t)ks_gu * R * 2 * F);
    logits = alloc<float>((size_t)R * c.vocab);
    rope_cos = alloc<float>((size_t)S * 2 * kMaxRows * (c.head_dim / 2));
    rope_sin = alloc<float>((size_t)S * 2 * kMaxRows * (c.head_dim / 2));
    act = alloc<uint8_t>((size_t)gemm_act_bytes(R, std::max(std::max(H, F), Q)));
    act_post = alloc<float>(R);
    argmax = alloc<int32_t>(R);
    dev_err = alloc<int>(1);
    XTG_CUDA(cudaMallocHost(&err_host, sizeof(int)));
    *err_host = 0;
    // one wave of attention CTAs (2 per SM, 1 at head dim 256) over every sequence's KV heads
    splits_g = std::max(1, std::min(256, attention_ctas_per_sm(c.head_dim) * sms / (c.kv_heads * S)));
    splits_r = std::max(1, std::min(splits_g, (int)(c.ring / 64)));
    part = alloc<float>((size_t)S * attention_part_floats(c.kv_heads, std::max(splits_g, splits_r), c.head_dim));
    std::vector<int32_t*> rt;
    for (xtg_cuda* q : seqs) rt.push_back(q->ring_pos_dev);
    ring_tab = upload(rt);
    std::vector<KvSeq> kt;
    for (size_t i = 0; i < model->kv.size(); ++i)
      for (xtg_cuda* q : seqs) {
        const KvInst& k = q->kv[i];
        kt.push_back(KvSeq{k.kc, k.vc, k.ks, k.vs, k.ring ? q->ring_pos_dev : nullptr, k.slots});
      }
    kvseq = upload(kt);
    // the GEMMs' output tiles (this batch's buffers, the model's global scales)
    auto tiles = [](float* y, int ld, int n, float g) {
      std::vector<TileOut> v(packed_tiles(n, false));
      for (int t = 0; t < (int)v.size(); ++t) v[t] = TileOut{y + 128 * t, ld, std::min(128, n - 128 * t), g, g};
      return v;
    };
    for (const Eval& E : model->evals) {
      if (E.kind == 0) {
        std::vector<TileOut> g(E.gu.tiles);
        for (int t = 0; t < E.gu.tiles; ++t) g[t] = TileOut{gu + 128 * t, 2 * F, 128, E.gu.g0, E.gu.g1};
        outs_a.push_back(upload(g));
        outs_b.push_back(upload(tiles(o, H, H, E.down.g0)));
      } else {
        std::vector<TileOut> v;
        const int n_out[4] = {Q, KV, KV, Q}, col[4] = {0, Q, Q + KV, Q + 2 * KV};
        for (int j = 0; j < 4; ++j)
          for (const TileOut& t : tiles(proj + col[j], proj_ld, n_out[j], E.gq[j])) v.push_back(t);
        outs_a.push_back(upload(v));
        outs_b.push_back(upload(tiles(o, H, H, E.o.g0)));
      }
    }
    outs_head = upload(tiles(logits, c.vocab, c.vocab, model->head.g0));
    XTG_CUDA(cudaStreamSynchronize(stream));
  }

  void gemm(const Linear& L, const TileOut* outs, int ksplit, int64_t stride, bool pdl) {
    launch_gemm(L.w, L.tiles, L.kblocks, act, act_post, kMaxRows * S, outs, model->num_sms, dev_err, stream, ksplit,
                stride, pdl);
  }

  void enqueue() {
    const Config& c = model->c;
    const int M = kMaxRows * S;
    const bool pdl = c.pdl;
    EmbedBatchArgs ea = {};
    ea.params = params_dev;
    ea.nseq = S;
    ea.head = model->head.w;
    ea.kblocks = model->head.kblocks;
    ea.global = model->head.g0;
    ea.table = model->embed_bf16;
    ea.hidden = H;
    ea.h = h;
    ea.inv_freq = model->inv_freq;
    ea.rope_half = c.head_dim / 2;
    ea.rope_cos = rope_cos;
    ea.rope_sin = rope_sin;
    ea.ring_pos = ring_tab;
    ea.ring = c.ring;
    ea.act = act;
    ea.act_post = act_post;
    launch_embed_batch(ea, stream);
    auto resid = [&](int mode, const float* lr, int oparts) {
      ResidArgs r = {};
      r.mode = mode;
      r.params = params_dev;
      r.hidden = H;
      r.h = h;
      r.o = o;
      r.lr = lr;
      r.state = state;
      r.input = input;
      r.nseq = S;
      r.o_parts = oparts;
      r.o_stride = (int64_t)kRows * H;
      r.gemm_act = act;   // the next GEMM's input: the new h
      r.gemm_post = act_post;
      launch_resid(r, stream, pdl);
    };
    auto slerp = [&](const float* lr, int oparts) {
      SlerpBatchArgs sb = {};
      sb.params = params_dev;
      sb.nseq = S;
      sb.hidden = H;
      sb.h = h;
      sb.o = o;
      sb.o_parts = oparts;
      sb.o_stride = (int64_t)kRows * H;
      sb.lr = lr;
      sb.act = act;
      sb.act_post = act_post;
      sb.pdl = pdl;
      launch_slerp_batch(sb, stream);
    };
    int e = 0, a_i = 0;
    auto sublayer = [&](int ei) {
      const Eval& E = model->evals[ei];
      if (E.kind == 0) {
        gemm(E.gu, outs_a[ei], ks_gu, (int64_t)kRows * 2 * F, pdl);
        SwigluBatchArgs sa = {};
        sa.params = params_dev;
        sa.nseq = S;
        sa.gu = gu;
        sa.ksplit = ks_gu;
        sa.split_stride = (int64_t)kRows * 2 * F;
        sa.features = F;
        sa.sg = E.sg;
        sa.su = E.su;
        sa.act = act;
        sa.act_post = act_post;
        sa.pdl = pdl;
        launch_swiglu_batch(sa, stream);
        gemm(E.down, outs_b[ei], ks_down, (int64_t)kRows * H, pdl);
        slerp(E.lr, ks_down);
        return;
      }
      gemm(E.qkvg, outs_a[ei], ks_qkv, (int64_t)kRows * proj_ld, pdl);
      QkvPrepArgs qa = {};
      qa.params = params_dev;
      qa.nseq = S;
      qa.proj = proj;
      qa.proj_ld = proj_ld;
      qa.ksplit = ks_qkv;
      qa.split_stride = (int64_t)kRows * proj_ld;
      qa.heads = c.heads;
      qa.kv_heads = c.kv_heads;
      qa.rope_cos = rope_cos;
      qa.rope_sin = rope_sin;
      qa.theta = E.theta;
      qa.qscale = E.qscale;
      qa.q_out = q_prep;
      qa.k_out = k_new;
      qa.v_out = v_new;
      qa.seqs = kvseq + (size_t)E.cache * S;
      qa.ring = E.kind == 1;
      qa.dtype = c.kv_dtype;
      qa.err = dev_err;
      qa.pdl = pdl;
      qa.head_dim = c.head_dim;
      launch_qkv_prep(qa, stream);
      const bool ring = E.kind == 1;
      AttnArgs at = {};
      at.q = q_prep;
      at.k = k_new;
      at.v = v_new;
      at.ring = ring ? 1 : 0;
      at.dtype = c.kv_dtype;
      at.window = ring ? c.window : 0;
      at.scale = 1.f / std::sqrt((float)c.head_dim);
      at.params = params_dev;
      at.heads = c.heads;
      at.kv_heads = c.kv_heads;
      at.splits = ring ? splits_r : splits_g;
      at.slots = 64;   // per sequence from seqs
      at.part = part;
      at.err = dev_err;
      at.seqs = kvseq + (size_t)E.cache * S;
      at.nseq = S;
      // a prompt chunk reads its cache below the chunk's first position only (own_rows): nothing this step writes,
      // so its copies go out before the dependency wait too
      at.late_copies = 0;
      at.l2_first = (!ring && c.l2_first) ? 1 : 0;
      at.part_seq_stride = attention_part_floats(c.kv_heads, std::max(splits_g, splits_r), c.head_dim);
      at.head_dim = c.head_dim;
      launch_attention(at, stream, pdl);
      CombineArgs cb = {};
      cb.part = part;
      cb.q = q_prep;
      cb.k = k_new;
      cb.v = v_new;
      cb.scale = at.scale;
      cb.window = at.window;
      cb.splits = at.splits;
      cb.heads = c.heads;
      cb.kv_heads = c.kv_heads;
      cb.params = params_dev;
      cb.gate = proj + Q + 2 * KV;   // the gate columns (K part 0; the parts are summed below)
      cb.gate_ld = proj_ld;
      cb.gscale = E.gscale;
      cb.asum = asum;
      cb.asum_ld = kRows;
      cb.gated_out = att;
      cb.nseq = S;
      cb.prompt = distinct ? 0 : 1;
      cb.part_seq_stride = at.part_seq_stride;
      cb.err = dev_err;
      cb.head_dim = c.head_dim;
      launch_attn_combine(cb, stream, pdl);
      gemm_digitize(att, M, Q, act, act_post, stream, asum, c.heads, kRows, pdl);
      gemm(E.o, outs_b[ei], ks_o, (int64_t)kRows * H, pdl);
      slerp(E.lr, ks_o);
      ++a_i;
    };
    for (int l = 0; l < c.n_in; ++l) sublayer(e++);
    if (c.loops > 0) {
      resid(kResidLoopBegin, nullptr, 1);
      for (int i = 0; i < c.loops; ++i) {
        for (int r = 0; r < c.n_rec; ++r) sublayer(e++);
        resid(i + 1 < c.loops ? kResidLoopNext : kResidLoopEnd, nullptr, 1);
      }
    }
    for (int l = 0; l < c.n_out; ++l) sublayer(e++);
    gemm(model->head, outs_head, 1, 0, pdl);
    ScaleArgmaxArgs sa = {};
    sa.params = params_dev;
    sa.nseq = S;
    sa.logits = logits;
    sa.vocab = c.vocab;
    sa.logit_scale = model->logit_scale;
    sa.argmax = argmax;
    sa.pdl = pdl;
    launch_scale_argmax(sa, stream);
    // each session's rows and argmax into its own buffers (xtg_cuda_argmax / xtg_cuda_topk read the last step there);
    // a prompt chunk (one session's row groups) copies its last group's after the step
    for (int i = 0; i < S && distinct; ++i) {
      XTG_CUDA(cudaMemcpyAsync(seqs[i]->logits, logits + (size_t)kMaxRows * i * c.vocab,
                               (size_t)kMaxRows * c.vocab * sizeof(float), cudaMemcpyDeviceToDevice, stream));
      XTG_CUDA(cudaMemcpyAsync(seqs[i]->argmax, argmax + kMaxRows * i, kMaxRows * sizeof(int32_t),
                               cudaMemcpyDeviceToDevice, stream));
    }
  }

  void capture() {
    if (exec) return;
    cudaGraph_t g = nullptr;
    XTG_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
    try {
      XTG_CUDA(cudaMemcpyAsync(params_dev, params_host, sizeof(StepParams) * S, cudaMemcpyHostToDevice, stream));
      enqueue();
    } catch (...) {
      cudaStreamEndCapture(stream, &g);
      if (g) cudaGraphDestroy(g);
      throw;
    }
    XTG_CUDA(cudaStreamEndCapture(stream, &g));
    cudaError_t e = cudaGraphInstantiate(&exec, g, 0);
    cudaGraphDestroy(g);
    XTG_CUDA(e);
  }

  bool stale() const {
    for (size_t i = 0; i < seqs.size(); ++i)
      if (seqs[i]->generation != gens[i]) return true;
    return false;
  }
};

namespace {

// The batched steps built so far, by their sessions (in call order). A session's close or tier change drops those it
// is in; one engine thread uses them at a time (the plugin's threading rule).
std::mutex g_batches_mu;
std::map<std::vector<xtg_cuda*>, std::unique_ptr<BatchStep>> g_batches;

void drop_batches_of(xtg_cuda* h) {
  std::lock_guard<std::mutex> lock(g_batches_mu);
  for (auto it = g_batches.begin(); it != g_batches.end();)
    if (std::find(it->first.begin(), it->first.end(), h) != it->first.end())
      it = g_batches.erase(it);
    else
      ++it;
}

BatchStep* batch_for(const std::vector<xtg_cuda*>& key) {
  std::lock_guard<std::mutex> lock(g_batches_mu);
  auto it = g_batches.find(key);
  if (it != g_batches.end() && it->second->stale()) {
    g_batches.erase(it);
    it = g_batches.end();
  }
  if (it == g_batches.end()) {
    auto b = std::make_unique<BatchStep>();
    b->build(key);
    it = g_batches.emplace(key, std::move(b)).first;
  }
  return it->second.get();
}

// Prompt chunks through the batched step: the chunk's rows as kMaxBatch groups of 8 of one session, group g at
// position n_past + 8 g, every group over the session's own caches. The projections of all the chunk's rows are one
// GEMM each. As attend_rows (packs/dory/dory.cpp:825-929) and the CPU path's multi-row attention (engine/src/kv.cpp:
// 166-286) do, every row attends the cache below the chunk's first position and the chunk's own rows up to itself,
// scored unquantized from the prepared rows: group g has own_rows = 8 g, and the combine folds the earlier groups'
// keys before its own. A ring holds the window plus its slack: the chunk's new rows overwrite only slots of
// positions the window has left, so a chunk is at most the slack (64 for the 1088-slot ring over a window of 1024).
int prefill_rows(const xtg_cuda* h) {
  const Config& c = h->c;
  if (!c.batch || !c.graph || c.kv_world != 1 || h->head_w_bf16) return 0;   // the batched step's head is NVFP4
  const int slack = c.ring - c.window;
  return std::min(kMaxBatch * kMaxRows, slack / kMaxRows * kMaxRows);
}

void prefill_chunk(xtg_cuda* h, const int32_t* tokens, int m, int want, int off, int n, xtg_cuda_logits_fn fn,
                   void* user) {
  BatchStep* b = batch_for(std::vector<xtg_cuda*>(kMaxBatch, h));
  const int vocab = h->c.vocab;
  for (int g = 0; g < kMaxBatch; ++g) {
    StepParams& p = b->params_host[g];
    std::memset(&p, 0, sizeof(p));
    const int mg = std::max(0, std::min(kMaxRows, m - kMaxRows * g));
    for (int r = 0; r < mg; ++r) p.tokens[r] = tokens[kMaxRows * g + r];
    p.m = mg;
    p.pos0 = h->n_past + kMaxRows * g;
    // the chunk's earlier rows are this group's own keys (packs/dory/dory.cpp:825-929, attend_rows: keys below the
    // chunk's first position from the cache, the chunk's own rows unquantized)
    p.own_rows = kMaxRows * g;
  }
  b->capture();
  XTG_CUDA(cudaGraphLaunch(b->exec, b->stream));
  // the session's last-step buffers get the chunk's last group (xtg_cuda_argmax / xtg_cuda_topk read them)
  const int G = (m - 1) / kMaxRows, mlast = m - kMaxRows * G;
  XTG_CUDA(cudaMemcpyAsync(h->logits, b->logits + (size_t)kMaxRows * G * vocab, (size_t)kMaxRows * vocab * sizeof(float),
                           cudaMemcpyDeviceToDevice, b->stream));
  XTG_CUDA(cudaMemcpyAsync(h->argmax, b->argmax + kMaxRows * G, kMaxRows * sizeof(int32_t), cudaMemcpyDeviceToDevice,
                           b->stream));
  XTG_CUDA(cudaMemcpyAsync(b->err_host, b->dev_err, sizeof(int), cudaMemcpyDeviceToHost, b->stream));
  XTG_CUDA(cudaStreamSynchronize(b->stream));
  if (*b->err_host) {
    *b->err_host = 0;
    XTG_CUDA(cudaMemsetAsync(b->dev_err, 0, sizeof(int), b->stream));
    throw CudaError("a device wait timed out during a prompt chunk (results discarded)");
  }
  h->commit(m);
  h->last_rows = mlast;
  const int r0 = want == 2 ? 0 : (want == 1 && off + m == n ? m - 1 : m);
  if (!fn) return;
  for (int g0 = r0; g0 < m; g0 += kMaxRows) {   // the rows through the session's 8-row host buffer
    const int cnt = std::min(kMaxRows, m - g0);
    XTG_CUDA(cudaMemcpyAsync(h->logits_host, b->logits + (size_t)g0 * vocab, (size_t)cnt * vocab * sizeof(float),
                             cudaMemcpyDeviceToHost, b->stream));
    XTG_CUDA(cudaStreamSynchronize(b->stream));
    for (int r = 0; r < cnt; ++r) fn(off + g0 + r, h->logits_host + (size_t)r * vocab, user);
  }
}

// sessions that can step as one: one weight set, one device, one KV format, graphs on, one process each
bool batchable(xtg_cuda* const* hs, int nh) {
  if (nh < 2) return false;
  for (int i = 0; i < nh; ++i) {
    const Config& c = hs[i]->c;
    if (!c.batch || !c.graph || c.kv_world != 1 || hs[i]->head_w_bf16 || hs[i]->wmem != hs[0]->wmem ||
        c.device != hs[0]->c.device ||
        c.kv_dtype != hs[0]->c.kv_dtype || c.decode_rows != hs[0]->c.decode_rows)
      return false;
  }
  return true;
}

}  // namespace

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

// xtg_cuda_forward_batch over sessions that step as one (batchable): groups of up to kMaxBatch sessions, in call
// order, each group one batched step per round on its own stream; every group's round is in flight before the first
// wait. A round's rows: session i's next min(decode_rows, what is left) tokens, none once it is done.
void run_batched(xtg_cuda* const* hs, int nh, const int32_t* const* tokens, const int* n, int want,
                 xtg_cuda_logits_fn fn, void* user, const std::vector<int>& base) {
  std::vector<BatchStep*> groups;
  for (int g0 = 0; g0 < nh; g0 += kMaxBatch) {
    const std::vector<xtg_cuda*> key(hs + g0, hs + std::min(nh, g0 + kMaxBatch));
    groups.push_back(batch_for(key));
  }
  XTG_CUDA(cudaSetDevice(hs[0]->c.device));
  const int rows = hs[0]->c.decode_rows;
  for (int off = 0;; off += rows) {
    bool any = false;
    for (size_t gi = 0; gi < groups.size(); ++gi) {
      BatchStep* b = groups[gi];
      bool live = false;
      for (int k = 0; k < b->S; ++k) {
        const int i = (int)gi * kMaxBatch + k;
        xtg_cuda* h = hs[i];
        StepParams& p = b->params_host[k];
        std::memset(&p, 0, sizeof(p));
        const int m = off < n[i] ? std::min(rows, n[i] - off) : 0;
        for (int r = 0; r < m; ++r) p.tokens[r] = tokens[i][off + r];
        p.m = m;
        p.pos0 = h->n_past;
        live |= m > 0;
      }
      if (!live) continue;
      any = true;
      b->capture();
      XTG_CUDA(cudaGraphLaunch(b->exec, b->stream));
      for (int k = 0; k < b->S; ++k) {
        const int i = (int)gi * kMaxBatch + k, m = b->params_host[k].m;
        const int r0 = want == 2 ? 0 : (want == 1 && off + m == n[i] ? m - 1 : m);
        xtg_cuda* h = hs[i];
        if (m > 0 && r0 < m && fn)
          XTG_CUDA(cudaMemcpyAsync(h->logits_host + (size_t)r0 * h->c.vocab, h->logits + (size_t)r0 * h->c.vocab,
                                   (size_t)(m - r0) * h->c.vocab * sizeof(float), cudaMemcpyDeviceToHost, b->stream));
      }
      XTG_CUDA(cudaMemcpyAsync(b->err_host, b->dev_err, sizeof(int), cudaMemcpyDeviceToHost, b->stream));
    }
    if (!any) break;
    std::string failed;
    for (size_t gi = 0; gi < groups.size(); ++gi) {
      BatchStep* b = groups[gi];
      XTG_CUDA(cudaStreamSynchronize(b->stream));
      if (*b->err_host) {
        *b->err_host = 0;
        XTG_CUDA(cudaMemsetAsync(b->dev_err, 0, sizeof(int), b->stream));
        if (failed.empty()) failed = "a device wait timed out during a batched step (results discarded)";
        continue;
      }
      for (int k = 0; k < b->S; ++k) {
        const int i = (int)gi * kMaxBatch + k, m = b->params_host[k].m;
        if (m == 0) continue;
        xtg_cuda* h = hs[i];
        h->commit(m);
        h->last_rows = m;
        const int r0 = want == 2 ? 0 : (want == 1 && off + m == n[i] ? m - 1 : m);
        if (fn)
          for (int r = r0; r < m; ++r) fn(base[(size_t)i] + off + r, h->logits_host + (size_t)r * h->c.vocab, user);
      }
    }
    if (!failed.empty()) throw CudaError(failed);
  }
}

}  // namespace

extern "C" {

xtg_cuda* xtg_cuda_open(const char* model_path, const char* options, char* err, int err_len) {
  std::unique_ptr<xtg_cuda> h;
  try {
    const std::string path = model_path ? model_path : "";
    if (path.empty()) throw CudaError("model: no path (a Dory checkpoint directory, or \"synthetic\")");
    h = std::make_unique<xtg_cuda>();
    if (path == "synthetic") {
      h->c = parse_config(options ? options : "");
    } else {   // read and checked before any device work
      const DoryConfig dc = read_dory_config(path);
      h->c = parse_config(options ? options : "", &dc);
      h->c.path = path;
      SafeTensors probe(path + "/model.safetensors");
    }
    int ndev = 0;
    XTG_CUDA(cudaGetDeviceCount(&ndev));
    XTG_REQUIRE(h->c.device >= 0 && h->c.device < ndev, "device: no CUDA device " + std::to_string(h->c.device));
    XTG_CUDA(cudaSetDevice(h->c.device));
    cudaDeviceProp prop;
    XTG_CUDA(cudaGetDeviceProperties(&prop, h->c.device));
    XTG_REQUIRE(prop.major == 10, std::string("libxtg_cuda is built for sm_100a; device is ") + prop.name);
    h->num_sms = prop.multiProcessorCount;
    XTG_CUDA(cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking));
    h->alloc_activations();
    h->build_model();
    h->alloc_caches();
    XTG_CUDA(cudaStreamSynchronize(h->stream));
    if (h->c.kv_world > 1) {   // every process opens its handle at the same time (a collective)
      ncclUniqueId id;
      auto hex = [](char ch) { return ch <= '9' ? ch - '0' : (ch | 0x20) - 'a' + 10; };
      for (size_t i = 0; i < sizeof(id); ++i)
        id.internal[i] = (char)(hex(h->c.nccl_id[2 * i]) * 16 + hex(h->c.nccl_id[2 * i + 1]));
      nccl_check(nccl_api().comm_init_rank(&h->comm, h->c.kv_world, id, h->c.kv_rank), "ncclCommInitRank");
      if (h->c.kv_exchange == "peer") h->open_peer_exchange();
    }
  } catch (const std::exception& e) {
    set_err(err, err_len, e.what());
    return nullptr;
  }
  return h.release();
}

xtg_cuda* xtg_cuda_open_shared(xtg_cuda* owner, const char* options, char* err, int err_len) {
  std::unique_ptr<xtg_cuda> h;
  try {
    XTG_REQUIRE(owner, "open_shared: no session to share weights with");
    const Config o = parse_config(options ? options : "");
    XTG_REQUIRE(o.kv_world == 1, "open_shared: a shared session runs in one process (kv_world 1)");
    h = std::make_unique<xtg_cuda>();
    // the owner's model and device; this session's own tier, KV format, snapshots, rows, graph and splits
    h->c = owner->c;
    h->c.context = o.context;
    h->c.kv_dtype = o.kv_dtype;
    h->c.snapshots = o.snapshots;
    h->c.decode_rows = o.decode_rows;
    h->c.graph = o.graph;
    h->c.pdl = o.pdl;
    h->c.l2_first = o.l2_first;
    h->c.batch = o.batch;
    h->c.nvtx = o.nvtx;
    h->c.splits_global = o.splits_global;
    h->c.splits_ring = o.splits_ring;
    h->c.kv_world = 1;
    h->c.kv_rank = 0;
    h->c.nccl_id.clear();
    XTG_CUDA(cudaSetDevice(h->c.device));
    h->num_sms = owner->num_sms;
    XTG_CUDA(cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking));
    h->alloc_activations();
    h->share_model(*owner);
    h->alloc_caches();
    XTG_CUDA(cudaStreamSynchronize(h->stream));
  } catch (const std::exception& e) {
    set_err(err, err_len, e.what());
    return nullptr;
  }
  return h.release();
}

int xtg_cuda_info(xtg_cuda* h, char* out, int out_len) {
  int rings = 0;
  for (const KvInst& k : h->kv) rings += k.ring;
  const int len = std::snprintf(
      out, (size_t)(out_len > 0 ? out_len : 0),
      "{\"vocab\":%d,\"context\":%lld,\"max_position\":%lld,\"prefill_ar\":%d,\"decode_ar\":%d,"
      "\"kv_instances\":%d,\"ring_instances\":%d,\"ring_slots\":%d,\"sliding_window\":%d,\"kv_bytes\":%lld,"
      "\"snapshots\":%d,\"kvmap\":false,\"kv_dtype\":\"%s\",\"weight_bytes\":%lld,\"hidden\":%d,\"evaluations\":%d,"
      "\"sm_count\":%d,\"graph\":%s,\"pdl\":%s,\"splits_global\":%d,\"splits_ring\":%d,"
      "\"kv_world\":%d,\"kv_rank\":%d,\"kv_exchange\":\"%s\",\"global_layers\":%d,\"source\":\"%s\","
      "\"head\":\"%s\",\"loops\":%d}",
      h->c.vocab, (long long)h->c.context, (long long)h->c.context - 1, std::max(h->c.decode_rows, prefill_rows(h)),
      h->c.decode_rows,
      (int)h->kv.size(), rings, h->c.ring, h->c.window, (long long)h->kv_bytes(), (int)h->snaps.size(),
      h->c.kv_dtype == kKvFp8 ? "fp8" : "int8", (long long)h->arena_bytes, h->c.hidden, h->c.n_evals(), h->num_sms,
      h->c.graph ? "true" : "false", h->c.pdl ? "true" : "false", h->splits_g, h->splits_r,
      h->c.kv_world, h->c.kv_rank, h->c.kv_world > 1 ? h->c.kv_exchange.c_str() : "none", h->n_glob,
      h->c.path == "synthetic" ? "synthetic" : "checkpoint", h->head_w_bf16 ? "bf16" : "nvfp4", h->c.loops);
  return len < out_len ? len : -1;
}

int xtg_cuda_forward(xtg_cuda* h, const int32_t* tokens, int n, int want, xtg_cuda_logits_fn fn, void* user,
                     char* err, int err_len) {
  return guarded(err, err_len, [&] {
    XTG_CUDA(cudaSetDevice(h->c.device));
    h->forward(tokens, n, want, fn, user);
  });
}

int xtg_cuda_forward_batch(xtg_cuda* const* hs, int nh, const int32_t* const* tokens, const int* n, int want,
                           xtg_cuda_logits_fn fn, void* user, char* err, int err_len) {
  // the caller's current device is restored on every exit (the steps switch to each session's device)
  int caller_device = -1;
  cudaGetDevice(&caller_device);
  struct RestoreDevice {
    int d;
    ~RestoreDevice() {
      if (d >= 0) cudaSetDevice(d);
    }
  } restore_device{caller_device};
  return guarded(err, err_len, [&] {
    XTG_REQUIRE(nh >= 0 && (nh == 0 || (hs && tokens && n)), "forward_batch: null arrays");
    std::vector<int> base((size_t)nh + 1, 0);
    for (int i = 0; i < nh; ++i) {   // every check before any step: a refused call changes nothing
      XTG_REQUIRE(hs[i], "forward_batch: null session");
      XTG_REQUIRE(n[i] >= 0, "forward_batch: negative token count");
      XTG_REQUIRE(n[i] == 0 || tokens[i], "forward_batch: null token list");
      for (int j = 0; j < i; ++j) XTG_REQUIRE(hs[j] != hs[i], "forward_batch: a session appears twice");
      hs[i]->check_tokens(tokens[i], n[i]);
      base[(size_t)i + 1] = base[(size_t)i] + n[i];
    }
    // as forward() does: a session given no tokens keeps its snapshots
    for (int i = 0; i < nh; ++i)
      if (n[i] > 0) hs[i]->drop_snapshots_past();
    if (batchable(hs, nh)) {
      run_batched(hs, nh, tokens, n, want, fn, user, base);
      return;
    }
    std::string failed;
    std::vector<xtg_cuda::Chunk> ks((size_t)nh);
    for (int step = 0;; ++step) {
      bool any = false;
      for (int i = 0; i < nh; ++i) {   // every session's next step goes out before the first wait
        xtg_cuda* h = hs[i];
        const int off = step * h->c.decode_rows;
        ks[(size_t)i].m = 0;
        if (off >= n[i]) continue;
        XTG_CUDA(cudaSetDevice(h->c.device));
        ks[(size_t)i] = h->enqueue_chunk(tokens[i], n[i], off, want, fn != nullptr);
        any = true;
      }
      if (!any) break;
      for (int i = 0; i < nh; ++i) {
        if (ks[(size_t)i].m == 0) continue;
        XTG_CUDA(cudaSetDevice(hs[i]->c.device));
        if (!hs[i]->finish_chunk(ks[(size_t)i], fn, user, base[(size_t)i]) && failed.empty())
          failed = "session " + std::to_string(i) + ": a device wait timed out during the step (results discarded)";
      }
      if (!failed.empty()) throw CudaError(failed);
    }
  });
}

int64_t xtg_cuda_pos(xtg_cuda* h) { return h->n_past; }

int xtg_cuda_rewind(xtg_cuda* h, int64_t n) { return h->rewind(n) ? 0 : -1; }

int xtg_cuda_snapshot_slots(xtg_cuda* h) { return (int)h->snaps.size(); }

int64_t xtg_cuda_snapshot_pos(xtg_cuda* h, int slot) {
  return slot >= 0 && slot < (int)h->snaps.size() ? h->snaps[slot].pos : -1;
}

void xtg_cuda_snapshot(xtg_cuda* h, int slot) {
  try {
    XTG_CUDA(cudaSetDevice(h->c.device));
    h->snapshot(slot);
  } catch (const std::exception&) {
    if (slot >= 0 && slot < (int)h->snaps.size()) h->snaps[slot].pos = -1;
  }
}

int xtg_cuda_restore(xtg_cuda* h, int slot) {
  try {
    XTG_CUDA(cudaSetDevice(h->c.device));
    return h->restore(slot) ? 0 : -1;
  } catch (const std::exception&) {
    return -1;
  }
}

int xtg_cuda_grow(xtg_cuda* h, const char* tier, char* err, int err_len) {
  return guarded(err, err_len, [&] {
    XTG_CUDA(cudaSetDevice(h->c.device));
    h->grow(parse_tier(tier ? tier : ""));
  });
}

int64_t xtg_cuda_debug_cache(xtg_cuda* h, int instance, int value, void* out, int64_t len) {
  if (instance < 0 || instance >= (int)h->kv.size() || value < 0 || value > 3) return -1;
  const KvInst& k = h->kv[instance];
  const int kvh = h->c.kv_heads;
  const int hd = h->c.head_dim;
  const int64_t codes = (int64_t)kvh * k.slots * hd, scales = (int64_t)kvh * k.slots * 4;
  const int64_t bytes = value < 2 ? codes : scales;
  if (!out || len < bytes) return bytes;
  try {
    XTG_CUDA(cudaSetDevice(h->c.device));
    if (value >= 2) {
      XTG_CUDA(cudaMemcpy(out, value == 2 ? k.ks : k.vs, bytes, cudaMemcpyDeviceToHost));
      return bytes;
    }
    std::vector<uint8_t> tmp(bytes);
    XTG_CUDA(cudaMemcpy(tmp.data(), value == 0 ? k.kc : k.vc, bytes, cudaMemcpyDeviceToHost));
    uint8_t* o = static_cast<uint8_t*>(out);
    // this library's layouts (attention.h) -> K [h][d][slot], V [h][slot][d]
    for (int hh = 0; hh < kvh; ++hh)
      for (int64_t s = 0; s < k.slots; ++s)
        for (int d = 0; d < hd; ++d) {
          if (value == 0)
            o[((int64_t)hh * hd + d) * k.slots + s] = tmp[k_offset(hh, s, d, k.slots, hd)];
          else
            o[((int64_t)hh * k.slots + s) * hd + d] = tmp[v_offset(hh, d, s, k.slots, hd)];
        }
  } catch (const std::exception&) {
    return -1;
  }
  return bytes;
}

void xtg_cuda_close(xtg_cuda* h) {
  if (!h) return;
  cudaSetDevice(h->c.device);
  drop_batches_of(h);
  delete h;
}

int xtg_cuda_argmax(xtg_cuda* h, int32_t* out, int n) {
  try {
    const int rows = std::min(n, h->last_rows);
    if (rows <= 0) return -1;
    XTG_CUDA(cudaMemcpy(out, h->argmax, rows * sizeof(int32_t), cudaMemcpyDeviceToHost));
    return rows;
  } catch (const std::exception&) {
    return -1;
  }
}

int xtg_cuda_topk(xtg_cuda* h, int k, float temperature, int32_t* idx, float* logit, float* row_max, double* total,
                  char* err, int err_len) {
  int rows = 0;
  const int rc = guarded(err, err_len, [&] {
    XTG_CUDA(cudaSetDevice(h->c.device));
    rows = h->last_rows;
    XTG_REQUIRE(rows > 0, "topk: no step yet");
    XTG_REQUIRE(k >= 1 && k <= kMaxTopK && k <= h->c.vocab, "topk: k in 1..min(1024, vocab)");
    XTG_REQUIRE(idx && logit && row_max && total, "topk: null output");
    if (!h->tk_idx) {
      h->tk_idx = h->dalloc<int32_t>((size_t)kMaxRows * kMaxTopK, false);
      h->tk_val = h->dalloc<float>((size_t)kMaxRows * kMaxTopK, false);
      h->tk_max = h->dalloc<float>(kMaxRows, false);
      h->tk_total = h->dalloc<double>(kMaxRows, false);
    }
    launch_topk(h->logits, rows, h->c.vocab, k, temperature, h->tk_idx, h->tk_val, h->tk_max, h->tk_total, h->stream);
    XTG_CUDA(cudaMemcpyAsync(idx, h->tk_idx, sizeof(int32_t) * rows * k, cudaMemcpyDeviceToHost, h->stream));
    XTG_CUDA(cudaMemcpyAsync(logit, h->tk_val, sizeof(float) * rows * k, cudaMemcpyDeviceToHost, h->stream));
    XTG_CUDA(cudaMemcpyAsync(row_max, h->tk_max, sizeof(float) * rows, cudaMemcpyDeviceToHost, h->stream));
    XTG_CUDA(cudaMemcpyAsync(total, h->tk_total, sizeof(double) * rows, cudaMemcpyDeviceToHost, h->stream));
    XTG_CUDA(cudaStreamSynchronize(h->stream));
  });
  return rc == 0 ? rows : -1;
}

int xtg_cuda_prefill_synthetic(xtg_cuda* h, int64_t n_past, char* err, int err_len) {
  return guarded(err, err_len, [&] {
    XTG_CUDA(cudaSetDevice(h->c.device));
    h->prefill_synthetic(n_past);
  });
}

int xtg_cuda_bench(xtg_cuda* h, const int32_t* tokens, int m, int steps, int profile, double* out_ms,
                   double* out_class_ms, int64_t* out_class_launches, char* err, int err_len) {
  return guarded(err, err_len, [&] {
    XTG_CUDA(cudaSetDevice(h->c.device));
    XTG_REQUIRE(m >= 1 && m <= h->c.decode_rows, "bench: 1..decode_rows rows");
    XTG_REQUIRE(steps >= 1, "bench: at least one step");
    for (int i = 0; i < m; ++i) XTG_REQUIRE(tokens[i] >= 0 && tokens[i] < h->c.vocab, "bench: token out of range");
    XTG_REQUIRE(h->n_past + m <= h->c.context, "bench: context full");
    h->set_params(tokens, m);
    if (!profile) {
      h->launch_step();   // capture / warm
      cudaEvent_t a, b;
      XTG_CUDA(cudaEventCreate(&a));
      XTG_CUDA(cudaEventCreate(&b));
      XTG_CUDA(cudaEventRecord(a, h->stream));
      for (int s = 0; s < steps; ++s) h->launch_step();
      XTG_CUDA(cudaEventRecord(b, h->stream));
      XTG_CUDA(cudaEventSynchronize(b));
      float ms = 0.f;
      XTG_CUDA(cudaEventElapsedTime(&ms, a, b));
      cudaEventDestroy(a);
      cudaEventDestroy(b);
      if (out_ms) *out_ms = ms / steps;
    } else {
      std::vector<std::pair<cudaEvent_t, cudaEvent_t>> ev;
      std::vector<int> cls;
      double cms[kClasses] = {0, 0, 0, 0};
      int64_t cl[kClasses] = {0, 0, 0, 0};
      double total = 0;
      for (int s = 0; s < steps; ++s) {
        h->prof = &ev;
        h->prof_cls = &cls;
        XTG_CUDA(cudaMemcpyAsync(h->params_dev, h->params_host, sizeof(StepParams), cudaMemcpyHostToDevice,
                                 h->stream));
        try {
          h->enqueue_step(false);
        } catch (...) {
          h->prof = nullptr;
          h->prof_cls = nullptr;
          throw;
        }
        h->prof = nullptr;
        h->prof_cls = nullptr;
        XTG_CUDA(cudaStreamSynchronize(h->stream));
        for (size_t i = 0; i < ev.size(); ++i) {
          float ms = 0.f;
          XTG_CUDA(cudaEventElapsedTime(&ms, ev[i].first, ev[i].second));
          cms[cls[i]] += ms;
          cl[cls[i]] += 1;
          total += ms;
          cudaEventDestroy(ev[i].first);
          cudaEventDestroy(ev[i].second);
        }
        ev.clear();
        cls.clear();
      }
      if (out_ms) *out_ms = total / steps;
      for (int c = 0; c < kClasses; ++c) {
        if (out_class_ms) out_class_ms[c] = cms[c] / steps;
        if (out_class_launches) out_class_launches[c] = cl[c] / steps;
      }
    }
    XTG_CUDA(cudaMemcpy(h->err_host, h->dev_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (*h->err_host) {
      *h->err_host = 0;
      XTG_CUDA(cudaMemset(h->dev_err, 0, sizeof(int)));
      throw CudaError("a device wait timed out during the timed steps");
    }
    // the steps wrote positions n_past .. n_past + m - 1 into the rings: the state of a forward rewound to n_past
    for (int r = 0; r < m; ++r) h->ring_pos[(h->n_past + r) % h->c.ring] = h->n_past + r;
    h->last_rows = m;
  });
}

int64_t xtg_cuda_step_bytes(xtg_cuda* h, int what, int m) { return h->step_bytes(what, m); }

}  // extern "C"
