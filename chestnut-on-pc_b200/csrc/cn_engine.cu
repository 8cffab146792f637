// Frame engine: random-init weights, device buffers, the per-frame launch
// plan, CUDA-graph replay and the C ABI (include/chestnut.h).
//
// Reference: run_pinned2.py:1346-1572 -- load, allocate queues, record the
// first frame's 497 launches and replay them as one CUDA graph per frame.
// Here the plan is built directly from the model description, captured once
// into a graph, and replayed with the recurrent state (queue rings, frame
// counter, optionally the hidden state) resident on the device.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/chestnut.h"
#include "cn_common.cuh"
#include "cn_gemm.cuh"
#include "cn_ops.cuh"
#include "cn_stem.cuh"
#include "cn_trunk.cuh"

namespace cn {

// ---------------------------------------------------------------- errors
static thread_local char g_err[512] = "";

void set_last_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}
const char* last_error_text() { return g_err; }

#define CN_CUDA(call)                                                                    \
  do {                                                                                   \
    cudaError_t _e = (call);                                                             \
    if (_e != cudaSuccess) {                                                             \
      set_last_error("%s failed: %s (%s:%d)", #call, cudaGetErrorString(_e), __FILE__, __LINE__); \
      return CN_ERR_CUDA;                                                                \
    }                                                                                    \
  } while (0)
#define CN_TRY(call)              \
  do {                            \
    int _r = (call);              \
    if (_r) return _r < 0 ? _r : CN_ERR_CUDA; \
  } while (0)

// ---------------------------------------------------------- model layout
struct ModelDims {
  int stem[5];
  int d, heads, layers, mlp;
};

static ModelDims dims_of(int model) {
  if (model == CN_MODEL_1B) return {{64, 128, 256, 512, 1024}, 2048, 16, 20, 8192};
  return {{32, 64, 128, 256, 512}, 512, 8, 4, 2048};
}

enum PKind { PK_W = 0, PK_B = 1, PK_POS = 2 };
struct ParamDesc {
  std::string name;
  int tid;
  long long rows, cols, valid;  // f16 weights: [rows][cols], columns >= valid are zero
  int fan_in;
  int kind;
};

// Same order / tensor ids as the oracle's spec.param_table.
static std::vector<ParamDesc> param_table(int model) {
  const ModelDims m = dims_of(model);
  std::vector<ParamDesc> P;
  int tid = 0;
  auto add = [&](std::string n, long long r, long long c, long long v, int fan, int kind) {
    P.push_back({n, tid++, r, c, v, fan, kind});
  };
  for (int cam = 0; cam < 2; ++cam) {
    int cin = 12;
    for (int s = 0; s < 5; ++s) {
      const int c = m.stem[s], k = 9 * cin;
      const std::string pre = "cam" + std::to_string(cam) + ".s" + std::to_string(s);
      add(pre + ".conv3.w", c, s == 0 ? kK0Pad : k, k, k, PK_W);
      add(pre + ".conv3.b", 1, c, c, k, PK_B);
      add(pre + ".conv1.w", c, c, c, c, PK_W);
      add(pre + ".conv1.b", 1, c, c, c, PK_B);
      cin = c;
    }
    add("cam" + std::to_string(cam) + ".vis.w", m.d, cin, cin, cin, PK_W);
    add("cam" + std::to_string(cam) + ".vis.b", 1, m.d, m.d, cin, PK_B);
  }
  add("temp.w", m.d, kFeat, kFeat, kFeat, PK_W);
  add("temp.b", 1, m.d, m.d, kFeat, PK_B);
  add("cond.w", m.d, kCondPad, kCond, kCond, PK_W);
  add("cond.b", 1, m.d, m.d, kCond, PK_B);
  add("pos", kT, m.d, m.d, 0, PK_POS);
  for (int l = 0; l < m.layers; ++l) {
    const std::string pre = "l" + std::to_string(l);
    add(pre + ".qkv.w", 3 * m.d, m.d, m.d, m.d, PK_W);
    add(pre + ".qkv.b", 1, 3 * m.d, 3 * m.d, m.d, PK_B);
    add(pre + ".o.w", m.d, m.d, m.d, m.d, PK_W);
    add(pre + ".o.b", 1, m.d, m.d, m.d, PK_B);
    add(pre + ".fc1.w", m.mlp, m.d, m.d, m.d, PK_W);
    add(pre + ".fc1.b", 1, m.mlp, m.mlp, m.d, PK_B);
    add(pre + ".fc2.w", m.d, m.mlp, m.mlp, m.mlp, PK_W);
    add(pre + ".fc2.b", 1, m.d, m.d, m.mlp, PK_B);
  }
  add("hid.w", kFeat, m.d, m.d, m.d, PK_W);
  add("hid.b", 1, kFeat, kFeat, m.d, PK_B);
  add("trunk.w", kTrunk, kFeat, kFeat, kFeat, PK_W);
  add("trunk.b", 1, kTrunk, kTrunk, kFeat, PK_B);
  add("heads.w", kNHeadsOut, kTrunk, kTrunk, kTrunk, PK_W);
  add("heads.b", 1, kNHeadsOut, kNHeadsOut, kTrunk, PK_B);
  return P;
}

static inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct Step {
  std::string name;
  std::function<int(cudaStream_t)> fn;
  cn_kernel_info info;
  bool side = false;  // runs on the side stream, forked from the main stream at the first side step
  bool join = false;  // main step that first waits for everything launched on the side stream
};

}  // namespace cn

using namespace cn;

struct cn_engine {
  cn_config cfg;
  ModelDims m;
  int B;
  cudaStream_t stream = nullptr;
  std::vector<ParamDesc> params;
  std::vector<size_t> poff;  // byte offset of each param in wblob
  uint8_t* wblob = nullptr;
  size_t wbytes = 0;
  uint8_t* ablob = nullptr;
  size_t abytes = 0;
  long long n_params = 0;
  // activations / state
  uint8_t* d_warped;
  float* d_packed;
  Rings rings;
  __half *a0, *gat[5], *y3[5], *act[5];
  __half *cond16, *feat16, *h, *qkv, *att, *u, *pooled, *hid16, *z;
  float *condv, *x, *out;
  // persistent trunk (single-clip frames): split-K partials + counter block
  bool use_trunk = false;
  bool tail_in_trunk = false;  // the trunk launch also computes hidden state, trunk head and heads
  int nsm = 0;
  TrunkPlan trunk;
  float* part = nullptr;
  __half* h2 = nullptr;  // LN2 output of the persistent trunk
  uint8_t* tctr = nullptr;
  size_t tctr_bytes = 0;
  // persistent conv stem: split-K partials + counters
  bool use_stem = false;
  StemPlan stem;
  float* spart = nullptr;
  uint8_t* sctr = nullptr;
  long long spart_floats = 0;
  std::vector<Step> steps;
  std::vector<GemmPlan> plans;
  // side branch of the frame (steps that depend only on the queues, not on the
  // conv stem) and its fork / join events
  cudaStream_t side = nullptr;
  cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t gexec = nullptr;
  // timed class (event nodes inside the graph)
  std::string timed_prefix;
  std::vector<cudaEvent_t> tev;  // pairs
  int pending = 0;               // a frame is in flight
  float* dec = nullptr;          // decoded outputs (cn_decode_frame), allocated on first use
  size_t dec_floats = 0;
  // double-buffered input (cn_stage_input / cn_run_staged), allocated on first use
  uint8_t* stage_buf = nullptr;  // [2][B][warped]
  cudaStream_t copy = nullptr;
  cudaEvent_t stage_ready[2] = {nullptr, nullptr}, stage_free[2] = {nullptr, nullptr};
  int stage_head = 0, stage_count = 0;
  // frames queued by cn_run_staged_async: output-copied events and the
  // device error word of each (pinned)
  cudaEvent_t out_ev[2] = {nullptr, nullptr};
  int* err_host = nullptr;
  int out_head = 0, out_count = 0;
};

namespace cn {

static void* wptr(cn_engine* e, const std::string& name) {
  for (size_t i = 0; i < e->params.size(); ++i)
    if (e->params[i].name == name) return e->wblob + e->poff[i];
  return nullptr;
}

static int gen_weights(cn_engine* e) {
  const uint64_t seed = e->cfg.seed;
  for (size_t i = 0; i < e->params.size(); ++i) {
    const ParamDesc& p = e->params[i];
    void* dst = e->wblob + e->poff[i];
    int r;
    if (p.kind == PK_W)
      r = launch_fill_f16_blocked((__half*)dst, p.rows, p.cols, p.valid, seed, (uint64_t)p.tid,
                                  sqrtf(6.0f / (float)p.fan_in), e->stream);
    else if (p.kind == PK_B)
      r = launch_fill_f32((float*)dst, p.rows * p.cols, seed, (uint64_t)p.tid, 1.0f / sqrtf((float)p.fan_in),
                          e->stream);
    else
      r = launch_fill_f32((float*)dst, p.rows * p.cols, seed, (uint64_t)p.tid, 0.5f, e->stream);
    if (r) {
      set_last_error("weight init launch failed: %s", cudaGetErrorString((cudaError_t)r));
      return CN_ERR_CUDA;
    }
  }
  CN_CUDA(cudaStreamSynchronize(e->stream));
  return 0;
}

// Layout: the two cameras' tensors of the same kind sit next to each other so
// a single grouped GEMM (group = camera) covers both.
static int layout_weights(cn_engine* e) {
  e->params = param_table(e->cfg.model);
  e->poff.assign(e->params.size(), 0);
  size_t off = 0;
  std::vector<bool> placed(e->params.size(), false);
  auto bytes_of = [](const ParamDesc& p) {
    return p.kind == PK_W ? (size_t)((p.cols + 63) / 64) * 64 * p.rows * 2 : (size_t)p.rows * p.cols * 4;
  };
  for (size_t i = 0; i < e->params.size(); ++i) {
    if (placed[i]) continue;
    const std::string& n = e->params[i].name;
    if (n.rfind("cam0.", 0) == 0) {
      // place cam0 and cam1 copies back to back with equal stride
      const std::string other = "cam1." + n.substr(5);
      size_t j = 0;
      for (; j < e->params.size(); ++j)
        if (e->params[j].name == other) break;
      const size_t b = align256(bytes_of(e->params[i]));
      e->poff[i] = off;
      e->poff[j] = off + b;
      placed[i] = placed[j] = true;
      off += 2 * b;
    } else {
      e->poff[i] = off;
      placed[i] = true;
      off += align256(bytes_of(e->params[i]));
    }
  }
  e->wbytes = off;
  e->n_params = 0;
  for (auto& p : e->params) e->n_params += p.rows * p.valid;
  return 0;
}

static size_t cam_stride_bytes(cn_engine* e, const std::string& cam0name) {
  const std::string other = "cam1." + cam0name.substr(5);
  return (size_t)((uint8_t*)wptr(e, other) - (uint8_t*)wptr(e, cam0name));
}

// The conv stem, the cond embedding and the token embeddings of a frame (one
// clip or a batch) as the phases of one persistent launch (cn_stem.cu).  Phase order:
// stage 0 (3x3 + fused 1x1), cond, temporal tokens, stage 1, then the other
// stages (the 1x1 fused while the stage has at most 256 channels), then the
// visual tokens.
// Returns 0, or -1 if a shape is not covered.
static int stem_build(cn_engine* e, StemPlan* sp) {
  const ModelDims& m = e->m;
  const int B = e->B;
  stem_plan_begin(sp, e->nsm);
  auto blank = [] {
    StemSpec s;
    memset(&s, 0, sizeof(s));
    s.dep0 = s.dep1 = -1;
    return s;
  };
  int prev = -1, ph_cond = -1;
  int cin = 12;
  for (int st = 0; st < 5; ++st) {
    const std::string pre = "cam0.s" + std::to_string(st);
    const int Ho = 64 >> st, Wo = 128 >> st, C = m.stem[st];
    const int Mg = B * Ho * Wo;
    StemSpec s = blank();
    s.G = 2;
    s.Mg = Mg;
    s.N = C;
    if (st == 0) {
      s.akind = SA_ROWS;
      s.A = e->a0;
      s.K = kK0Pad;
      s.lda = kK0Pad;
      s.a_gs = (long long)B * 8192 * kK0Pad;
    } else {
      s.akind = SA_GATHER;
      s.A = e->act[st - 1];
      s.K = 9 * cin;
      s.Hin = 2 * Ho;
      s.Win = 2 * Wo;
      s.Cin = cin;
      s.a_gs = (long long)B * s.Hin * s.Win * cin;
    }
    s.W = wptr(e, pre + ".conv3.w");
    s.w_gs = (long long)cam_stride_bytes(e, pre + ".conv3.w");
    s.epi = SE_RELU_F16;
    s.out = e->y3[st];
    s.ldo = C;
    s.o_gs = (long long)Mg * C;
    s.bias = (const float*)wptr(e, pre + ".conv3.b");
    s.b_gs = (long long)cam_stride_bytes(e, pre + ".conv3.b") / 4;
    const bool fuse = C <= 256;  // the 1x1 runs inside the 3x3 unit while a tile's channels fit one MMA
    if (fuse) {
      s.W1 = wptr(e, pre + ".conv1.w");
      s.w1_gs = (long long)cam_stride_bytes(e, pre + ".conv1.w");
      s.out1 = e->act[st];
      s.ldo1 = C;
      s.o1_gs = (long long)Mg * C;
      s.bias1 = (const float*)wptr(e, pre + ".conv1.b");
      s.b1_gs = (long long)cam_stride_bytes(e, pre + ".conv1.b") / 4;
    }
    s.dep0 = prev;
    const int p3 = stem_add(sp, s);
    if (p3 < 0) return -1;
    prev = p3;
    if (!fuse) {
      StemSpec c = blank();
      c.G = 2;
      c.Mg = Mg;
      c.N = C;
      c.K = C;
      c.akind = SA_ROWS;
      c.A = e->y3[st];
      c.lda = C;
      c.a_gs = (long long)Mg * C;
      c.W = wptr(e, pre + ".conv1.w");
      c.w_gs = (long long)cam_stride_bytes(e, pre + ".conv1.w");
      c.epi = SE_RELU_F16;
      c.out = e->act[st];
      c.ldo = C;
      c.o_gs = (long long)Mg * C;
      c.bias = (const float*)wptr(e, pre + ".conv1.b");
      c.b_gs = (long long)cam_stride_bytes(e, pre + ".conv1.b") / 4;
      c.dep0 = p3;
      if ((prev = stem_add(sp, c)) < 0) return -1;
    }
    if (st == 0) {
      // cond embedding (f32, read by both token phases) and the temporal tokens:
      // they read only what gather0 wrote
      StemSpec c = blank();
      c.G = 1;
      c.Mg = B;
      c.N = m.d;
      c.K = kCondPad;
      c.akind = SA_ROWS;
      c.A = e->cond16;
      c.lda = kCondPad;
      c.W = wptr(e, "cond.w");
      c.epi = SE_F32;
      c.out = e->condv;
      c.ldo = m.d;
      c.bias = (const float*)wptr(e, "cond.b");
      if ((ph_cond = stem_add(sp, c)) < 0) return -1;
      StemSpec t = blank();
      t.G = 1;
      t.Mg = B * kNTemp;
      t.N = m.d;
      t.K = kFeat;
      t.akind = SA_ROWS;
      t.A = e->feat16;
      t.lda = kFeat;
      t.W = wptr(e, "temp.w");
      t.epi = SE_TOKENS;
      t.out = e->x;
      t.ldo = m.d;
      t.bias = (const float*)wptr(e, "temp.b");
      t.pos = (const float*)wptr(e, "pos");
      t.cond = e->condv;
      t.cond_ld = m.d;
      t.rows_per_clip = kNTemp;
      t.tok_base = kNVis;
      t.tok_gstride = 0;
      t.T = kT;
      t.dep0 = ph_cond;
      if (stem_add(sp, t) < 0) return -1;
    }
    cin = C;
  }
  // visual token embeddings into rows [0, 64) of each clip of x
  StemSpec v = blank();
  const int C4 = m.stem[4];
  v.G = 2;
  v.Mg = B * kNVisCam;
  v.N = m.d;
  v.K = C4;
  v.akind = SA_ROWS;
  v.A = e->act[4];
  v.lda = C4;
  v.a_gs = (long long)B * kNVisCam * C4;
  v.W = wptr(e, "cam0.vis.w");
  v.w_gs = (long long)cam_stride_bytes(e, "cam0.vis.w");
  v.epi = SE_TOKENS;
  v.out = e->x;
  v.ldo = m.d;
  v.bias = (const float*)wptr(e, "cam0.vis.b");
  v.b_gs = (long long)cam_stride_bytes(e, "cam0.vis.b") / 4;
  v.pos = (const float*)wptr(e, "pos");
  v.cond = e->condv;
  v.cond_ld = m.d;
  v.rows_per_clip = kNVisCam;
  v.tok_base = 0;
  v.tok_gstride = kNVisCam;
  v.T = kT;
  v.dep0 = prev;
  v.dep1 = ph_cond;
  if (stem_add(sp, v) < 0) return -1;
  return 0;
}

static int layout_acts(cn_engine* e) {
  const int B = e->B;
  const ModelDims& m = e->m;
  size_t off = 0;
  std::vector<std::pair<void**, size_t>> req;
  auto want = [&](void** p, size_t bytes) { req.push_back({p, bytes}); };
  want((void**)&e->d_warped, (size_t)B * kWarpedBytes);
  want((void**)&e->d_packed, (size_t)B * kPacked * 4);
  want((void**)&e->rings.img, (size_t)B * 2 * kImgQ * kFrameBytes);
  want((void**)&e->rings.feat, (size_t)B * kFeatQ * kFeat * 4);
  want((void**)&e->rings.desire, (size_t)B * kDesireQ * kDesire * 4);
  want((void**)&e->rings.ctr, 256);
  want((void**)&e->a0, (size_t)2 * B * 8192 * kK0Pad * 2);
  if (e->use_stem) {
    // plan over the (not yet placed) activations: does the persistent stem
    // cover these shapes, and how large are its split-K partials?
    StemPlan* dry = new StemPlan;
    if (stem_build(e, dry) == 0) {
      e->spart_floats = dry->part_floats;
      want((void**)&e->spart, (size_t)e->spart_floats * 4 + 16);
      want((void**)&e->sctr, stem_counter_bytes());
    } else {
      e->use_stem = false;  // shapes the persistent stem does not cover: per-layer stem kernels
    }
    delete dry;
  }
  int cin = 12;
  for (int s = 0; s < 5; ++s) {
    const size_t P = (size_t)(64 >> s) * (128 >> s);
    // im2col matrices: per-layer stem only (the persistent stem gathers in its loads)
    e->gat[s] = nullptr;
    if (s > 0 && !e->use_stem) want((void**)&e->gat[s], 2 * B * P * 9 * cin * 2);
    want((void**)&e->y3[s], 2 * B * P * m.stem[s] * 2);
    want((void**)&e->act[s], 2 * B * P * m.stem[s] * 2);
    cin = m.stem[s];
  }
  const size_t R = (size_t)B * kT;
  want((void**)&e->cond16, (size_t)B * kCondPad * 2);
  want((void**)&e->feat16, (size_t)B * kNTemp * kFeat * 2);
  want((void**)&e->condv, (size_t)B * m.d * 4);
  want((void**)&e->x, R * m.d * 4);
  want((void**)&e->h, R * m.d * 2);
  want((void**)&e->qkv, R * 3 * m.d * 2);
  want((void**)&e->att, R * m.d * 2);
  want((void**)&e->u, R * m.mlp * 2);
  want((void**)&e->pooled, (size_t)B * m.d * 2);
  want((void**)&e->hid16, (size_t)B * kFeat * 2);
  want((void**)&e->z, (size_t)B * kTrunk * 2);
  want((void**)&e->out, (size_t)B * kNOut * 4);
  if (e->use_trunk) {
    want((void**)&e->part, trunk_part_floats((int)R, m.d, m.mlp, m.layers, e->nsm) * 4);
    want((void**)&e->h2, R * m.d * 2);
    e->tctr_bytes = trunk_counter_bytes(m.layers);
    want((void**)&e->tctr, e->tctr_bytes);
  }
  for (auto& r : req) off += align256(r.second);
  e->abytes = off;
  CN_CUDA(cudaMalloc((void**)&e->ablob, e->abytes));
  CN_CUDA(cudaMemsetAsync(e->ablob, 0, e->abytes, e->stream));
  off = 0;
  for (auto& r : req) {
    *r.first = e->ablob + off;
    off += align256(r.second);
  }
  return 0;
}

static cn_kernel_info kinfo(const char* name, dim3 g, dim3 b, dim3 cl, size_t smem) {
  cn_kernel_info k;
  memset(&k, 0, sizeof(k));
  snprintf(k.name, sizeof(k.name), "%s", name);
  k.grid[0] = g.x; k.grid[1] = g.y; k.grid[2] = g.z;
  k.block[0] = b.x; k.block[1] = b.y; k.block[2] = b.z;
  k.cluster[0] = cl.x; k.cluster[1] = cl.y; k.cluster[2] = cl.z;
  k.smem_bytes = (unsigned)smem;
  return k;
}

static int add_gemm(cn_engine* e, const std::string& name, const void* A, long long lda, long long a_gs,
                    const void* Bw, long long ldb, long long b_gs, int M, int N, int K, int G, const GemmParams& ep) {
  GemmPlan g;
  int r = gemm_plan(&g, A, lda, a_gs, Bw, ldb, b_gs, M, N, K, G, B_K_BLOCKED, 0, 0, ep);
  if (r) return r < 0 ? r : CN_ERR_CUDA;
  g.pdl = true;
  const size_t idx = e->plans.size();
  e->plans.push_back(g);
  char nm[64];
  snprintf(nm, sizeof(nm), "gemm_tc_bn%d_s%d:%s", g.bn, g.p.splits, name.c_str());
  e->steps.push_back({nm, [e, idx](cudaStream_t s) { return gemm_launch(e->plans[idx], s); },
                      kinfo(nm, g.grid, dim3(128), dim3(1, 1, g.p.splits), g.smem)});
  return 0;
}

static GemmParams epi_f16(void* out, long long ldo, long long ogs, const float* bias, long long bgs, int act) {
  GemmParams p;
  memset(&p, 0, sizeof(p));
  p.epi = EPI_F16;
  p.act = act;
  p.out = out;
  p.ldo = ldo;
  p.out_gstride = ogs;
  p.bias = bias;
  p.bias_gstride = bgs;
  return p;
}

static int build_plan(cn_engine* e) {
  const int B = e->B;
  const ModelDims& m = e->m;
  const int R = B * kT;
  e->steps.clear();
  e->plans.clear();
  e->plans.reserve(256);
  const float* carry = e->cfg.carry_hidden ? e->out + kNHeadsOut : nullptr;
  {
    const long long vecs = 2LL * kFrameBytes / 16;
    e->steps.push_back({"push", [e, carry](cudaStream_t s) {
                          return launch_push(e->d_warped, e->d_packed, carry, kNOut, e->rings, e->B, s, true);
                        },
                        kinfo("queue_push", dim3((unsigned)((vecs + 255) / 256), B), dim3(256), dim3(1, 1, 1), 0)});
    e->steps.push_back({"gather0", [e](cudaStream_t s) {
                          return launch_gather0(e->rings, e->d_packed, e->B, e->a0, e->cond16, e->feat16, s, true);
                        },
                        kinfo("border_gather0", dim3(64, 2 * B + 1), dim3(128), dim3(1, 1, 1), 0)});
  }
  if (e->use_stem) {
    // conv stem, cond embedding and token embeddings: one persistent launch
    if (stem_build(e, &e->stem) != 0) return CN_ERR_ARG;
    CN_TRY(stem_plan_end(&e->stem, e->spart, e->sctr));
    e->steps.push_back({"stem", [e](cudaStream_t s) { return stem_launch(e->stem, s); },
                        kinfo("conv_stem", dim3(e->stem.grid), dim3(256), dim3(1, 1, 1), e->stem.smem)});
  } else {
    // Side branch: the cond embedding and the temporal tokens read only what
    // gather0 wrote, so they run beside the conv stem instead of after it.
    {
      GemmParams ep;
      memset(&ep, 0, sizeof(ep));
      ep.epi = EPI_F32_OUT;
      ep.out = e->condv;
      ep.ldo = m.d;
      ep.bias = (const float*)wptr(e, "cond.b");
      CN_TRY(add_gemm(e, "cond", e->cond16, kCondPad, 0, wptr(e, "cond.w"), kCondPad, 0, B, m.d, kCondPad, 1, ep));
      e->steps.back().side = true;
      e->plans.back().pdl = false;  // first kernel of the branch: its dependency is the fork event
    }
    {
      // temporal token embeddings into rows [kNVis, kT) of each clip of x
      GemmParams ep;
      memset(&ep, 0, sizeof(ep));
      ep.epi = EPI_TOKENS;
      ep.out = e->x;
      ep.ldo = m.d;
      ep.bias = (const float*)wptr(e, "temp.b");
      ep.bias_gstride = 0;
      ep.pos = (const float*)wptr(e, "pos");
      ep.cond = e->condv;
      ep.cond_ld = m.d;
      ep.rows_per_clip = kNTemp;
      ep.tok_base = kNVis;
      ep.tok_gstride = 0;
      ep.T = kT;
      CN_TRY(add_gemm(e, "temp_tokens", e->feat16, kFeat, 0, wptr(e, "temp.w"), kFeat, 0, B * kNTemp, m.d, kFeat, 1,
                      ep));
      e->steps.back().side = true;
    }
    // conv stem, both cameras as one grouped GEMM per layer
    int cin = 12;
    for (int s = 0; s < 5; ++s) {
      const int Pp = (64 >> s) * (128 >> s);
      const int C = m.stem[s];
      const int Ho = 64 >> s, Wo = 128 >> s;
      const __half* A;
      int K;
      if (s == 0) {
        A = e->a0;
        K = kK0Pad;
      } else {
        K = 9 * cin;
        const __half* src = e->act[s - 1];
        __half* dst = e->gat[s];
        const int Hin = 2 * Ho, Win = 2 * Wo, Ci = cin;
        const long long total = 2LL * B * Ho * Wo * 9 * (Ci / 8);
        char nm[64];
        snprintf(nm, sizeof(nm), "border_gather_s2:s%d", s);
        e->steps.push_back({nm, [src, dst, B, Hin, Win, Ci](cudaStream_t st) {
                              return launch_gather_s2(src, 2, B, Hin, Win, Ci, dst, st, true);
                            },
                            kinfo(nm, dim3((unsigned)std::min<long long>((total + 255) / 256, 1LL << 20)), dim3(256),
                                  dim3(1, 1, 1), 0)});
        A = dst;
      }
      const std::string pre = "cam0.s" + std::to_string(s);
      const long long M = (long long)B * Pp;
      {
        const void* W = wptr(e, pre + ".conv3.w");
        const float* b = (const float*)wptr(e, pre + ".conv3.b");
        const long long wgs = cam_stride_bytes(e, pre + ".conv3.w") / 2;
        const long long bgs = cam_stride_bytes(e, pre + ".conv3.b") / 4;
        GemmParams ep = epi_f16(e->y3[s], C, M * C, b, bgs, ACT_RELU);
        CN_TRY(add_gemm(e, "s" + std::to_string(s) + ".conv3", A, K, M * K, W, K, wgs, (int)M, C, K, 2, ep));
      }
      {
        const void* W = wptr(e, pre + ".conv1.w");
        const float* b = (const float*)wptr(e, pre + ".conv1.b");
        const long long wgs = cam_stride_bytes(e, pre + ".conv1.w") / 2;
        const long long bgs = cam_stride_bytes(e, pre + ".conv1.b") / 4;
        GemmParams ep = epi_f16(e->act[s], C, M * C, b, bgs, ACT_RELU);
        CN_TRY(add_gemm(e, "s" + std::to_string(s) + ".conv1", e->y3[s], C, M * C, W, C, wgs, (int)M, C, C, 2, ep));
      }
      cin = C;
    }
    // visual token embeddings into the residual stream x [B*88][d]: rows of
    // the camera tokens; waits for the side branch (cond, temporal tokens)
    {
      GemmParams ep;
      memset(&ep, 0, sizeof(ep));
      ep.epi = EPI_TOKENS;
      ep.out = e->x;
      ep.ldo = m.d;
      ep.bias = (const float*)wptr(e, "cam0.vis.b");
      ep.bias_gstride = cam_stride_bytes(e, "cam0.vis.b") / 4;
      ep.pos = (const float*)wptr(e, "pos");
      ep.cond = e->condv;
      ep.cond_ld = m.d;
      ep.rows_per_clip = kNVisCam;
      ep.tok_base = 0;
      ep.tok_gstride = kNVisCam;
      ep.T = kT;
      const int C4 = m.stem[4];
      CN_TRY(add_gemm(e, "vis_tokens", e->act[4], C4, (long long)B * 32 * C4, wptr(e, "cam0.vis.w"), C4,
                      cam_stride_bytes(e, "cam0.vis.w") / 2, B * 32, m.d, C4, 2, ep));
      e->steps.back().join = true;
    }
  }
  // transformer
  if (e->use_trunk) {
    const char* wn[4] = {".qkv.w", ".o.w", ".fc1.w", ".fc2.w"};
    const char* bn[4] = {".qkv.b", ".o.b", ".fc1.b", ".fc2.b"};
    const void* w0[4];
    const float* b0[4];
    long long wstride = 0, bstride = 0;
    for (int g = 0; g < 4; ++g) {
      w0[g] = wptr(e, std::string("l0") + wn[g]);
      b0[g] = (const float*)wptr(e, std::string("l0") + bn[g]);
    }
    if (m.layers > 1) {
      wstride = (long long)((uint8_t*)wptr(e, std::string("l1") + wn[0]) - (uint8_t*)w0[0]);
      bstride = (long long)((const float*)wptr(e, std::string("l1") + bn[0]) - b0[0]);
    }
    for (int l = 0; l < m.layers; ++l)
      for (int g = 0; g < 4; ++g) {
        const std::string pre = "l" + std::to_string(l);
        if ((uint8_t*)wptr(e, pre + wn[g]) != (uint8_t*)w0[g] + l * wstride ||
            (const float*)wptr(e, pre + bn[g]) != b0[g] + l * bstride) {
          set_last_error("trunk: layer tensors are not equally strided");
          return CN_ERR_ARG;
        }
      }
    CN_TRY(trunk_plan(&e->trunk, B, kT, m.d, m.mlp, m.heads, m.layers, w0, wstride, b0, bstride, e->x, e->h, e->qkv,
                      e->att, e->u, e->h2, e->part, e->tctr, e->rings.ctr, e->nsm, e->h, e->pooled));
    {
      // the tail products of the frame run at the end of the trunk launch
      const void* tw[3] = {wptr(e, "hid.w"), wptr(e, "trunk.w"), wptr(e, "heads.w")};
      const float* tb[3] = {(const float*)wptr(e, "hid.b"), (const float*)wptr(e, "trunk.b"),
                            (const float*)wptr(e, "heads.b")};
      const int tn[3] = {kFeat, kTrunk, kNHeadsOut}, tk[3] = {m.d, kFeat, kTrunk};
      e->tail_in_trunk = trunk_set_tail(&e->trunk, tw, tb, tn, tk, e->hid16, e->z, e->out, kNHeadsOut);
    }
    e->steps.push_back({"trunk", [e](cudaStream_t s) { return trunk_launch(e->trunk, s); },
                        kinfo("transformer_trunk", dim3(e->trunk.grid), dim3(256), dim3(1, 1, 1), e->trunk.smem)});
  }
  for (int l = 0; l < (e->use_trunk ? 0 : m.layers); ++l) {
    const std::string pre = "l" + std::to_string(l);
    int* bump = l == 0 ? e->rings.ctr : nullptr;  // all readers of the frame counter ran before this
    {
      float* x = e->x;
      __half* h = e->h;
      const int d = m.d;
      e->steps.push_back({"ln1", [x, h, R, d, bump](cudaStream_t s) { return launch_layernorm(x, h, R, d, bump, s, true); },
                          kinfo(("layernorm:" + pre + ".ln1").c_str(), dim3((R + 7) / 8), dim3(256), dim3(1, 1, 1), 0)});
    }
    CN_TRY(add_gemm(e, pre + ".qkv", e->h, m.d, 0, wptr(e, pre + ".qkv.w"), m.d, 0, R, 3 * m.d, m.d, 1,
                    epi_f16(e->qkv, 3 * m.d, 0, (const float*)wptr(e, pre + ".qkv.b"), 0, ACT_NONE)));
    {
      const __half* q = e->qkv;
      __half* o = e->att;
      const int d = m.d, H = m.heads;
      const int hd = d / H;
      const size_t smem = attention_smem_bytes(hd);
      e->steps.push_back({"attn", [q, o, B, d, H](cudaStream_t s) { return launch_attention(q, o, B, kT, d, H, s, true); },
                          kinfo(("attention:" + pre).c_str(), dim3(B * H, (kT + 7) / 8), dim3(256), dim3(1, 1, 1), smem)});
    }
    {
      GemmParams ep;
      memset(&ep, 0, sizeof(ep));
      ep.epi = EPI_RESID;
      ep.out = e->x;
      ep.ldo = m.d;
      ep.bias = (const float*)wptr(e, pre + ".o.b");
      CN_TRY(add_gemm(e, pre + ".o", e->att, m.d, 0, wptr(e, pre + ".o.w"), m.d, 0, R, m.d, m.d, 1, ep));
    }
    {
      float* x = e->x;
      __half* h = e->h;
      const int d = m.d;
      e->steps.push_back({"ln2", [x, h, R, d](cudaStream_t s) { return launch_layernorm(x, h, R, d, nullptr, s, true); },
                          kinfo(("layernorm:" + pre + ".ln2").c_str(), dim3((R + 7) / 8), dim3(256), dim3(1, 1, 1), 0)});
    }
    CN_TRY(add_gemm(e, pre + ".fc1", e->h, m.d, 0, wptr(e, pre + ".fc1.w"), m.d, 0, R, m.mlp, m.d, 1,
                    epi_f16(e->u, m.mlp, 0, (const float*)wptr(e, pre + ".fc1.b"), 0, ACT_GELU)));
    {
      GemmParams ep;
      memset(&ep, 0, sizeof(ep));
      ep.epi = EPI_RESID;
      ep.out = e->x;
      ep.ldo = m.d;
      ep.bias = (const float*)wptr(e, pre + ".fc2.b");
      CN_TRY(add_gemm(e, pre + ".fc2", e->u, m.mlp, 0, wptr(e, pre + ".fc2.w"), m.mlp, 0, R, m.d, m.mlp, 1, ep));
    }
  }
  if (!e->use_trunk) {
    // final LayerNorm (into h) then the token mean of each clip (the
    // persistent trunk does both at its end)
    float* x = e->x;
    __half* h = e->h;
    __half* p = e->pooled;
    const int d = m.d;
    e->steps.push_back({"lnf", [x, h, R, d](cudaStream_t s) { return launch_layernorm(x, h, R, d, nullptr, s, true); },
                        kinfo("layernorm:final", dim3((R + 7) / 8), dim3(256), dim3(1, 1, 1), 0)});
    e->steps.push_back({"pool", [h, p, B, d](cudaStream_t s) { return launch_colmean(h, p, B, kT, d, s, true); },
                        kinfo("token_mean_pool", dim3(B, d / 256), dim3(256), dim3(1, 1, 1), 0)});
  }
  if (!e->tail_in_trunk) {
    // hidden state, trunk head and heads (the persistent trunk runs them at its end)
    {
      GemmParams ep = epi_f16(e->hid16, kFeat, 0, (const float*)wptr(e, "hid.b"), 0, ACT_TANH);
      ep.out32 = e->out + kNHeadsOut;
      ep.ld32 = kNOut;
      CN_TRY(add_gemm(e, "hidden_state", e->pooled, m.d, 0, wptr(e, "hid.w"), m.d, 0, B, kFeat, m.d, 1, ep));
    }
    CN_TRY(add_gemm(e, "trunk", e->hid16, kFeat, 0, wptr(e, "trunk.w"), kFeat, 0, B, kTrunk, kFeat, 1,
                    epi_f16(e->z, kTrunk, 0, (const float*)wptr(e, "trunk.b"), 0, ACT_RELU)));
    {
      GemmParams ep;
      memset(&ep, 0, sizeof(ep));
      ep.epi = EPI_F32_OUT;
      ep.out = e->out;
      ep.ldo = kNOut;
      ep.bias = (const float*)wptr(e, "heads.b");
      CN_TRY(add_gemm(e, "heads", e->z, kTrunk, 0, wptr(e, "heads.w"), kTrunk, 0, B, kNHeadsOut, kTrunk, 1, ep));
    }
  }
  return 0;
}

static bool timed(const cn_engine* e, const Step& st) {
  return !e->timed_prefix.empty() && std::string(st.info.name).find(e->timed_prefix) != std::string::npos;
}

static int run_steps(cn_engine* e, cudaStream_t s, bool with_events) {
  size_t ev = 0;
  bool forked = false;
  for (auto& st : e->steps) {
    if (st.side && !forked) {  // fork: the side stream starts after the main stream's work so far
      CN_CUDA(cudaEventRecord(e->ev_fork, s));
      CN_CUDA(cudaStreamWaitEvent(e->side, e->ev_fork, 0));
      forked = true;
    }
    if (st.join && forked) {  // join: everything on the side stream before this step
      CN_CUDA(cudaEventRecord(e->ev_join, e->side));
      CN_CUDA(cudaStreamWaitEvent(s, e->ev_join, 0));
      forked = false;
    }
    const cudaStream_t ss = st.side ? e->side : s;
    const bool t = with_events && timed(e, st);
    // External records become real event-record nodes when captured into the graph.
    if (t) CN_CUDA(cudaEventRecordWithFlags(e->tev[ev], ss, cudaEventRecordExternal));
    int r = st.fn(ss);
    if (r) {
      if (r > 0) set_last_error("launch of %s failed: %s", st.info.name, cudaGetErrorString((cudaError_t)r));
      return r < 0 ? r : CN_ERR_CUDA;
    }
    if (t) {
      CN_CUDA(cudaEventRecordWithFlags(e->tev[ev + 1], ss, cudaEventRecordExternal));
      ev += 2;
    }
  }
  if (forked) {  // a branch without a join step rejoins at the end
    CN_CUDA(cudaEventRecord(e->ev_join, e->side));
    CN_CUDA(cudaStreamWaitEvent(s, e->ev_join, 0));
  }
  return 0;
}

static int rebuild_graph(cn_engine* e) {
  if (e->gexec) cudaGraphExecDestroy(e->gexec);
  if (e->graph) cudaGraphDestroy(e->graph);
  e->gexec = nullptr;
  e->graph = nullptr;
  if (!e->cfg.use_graph) return 0;
  CN_CUDA(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
  int r = run_steps(e, e->stream, true);
  cudaGraph_t g = nullptr;
  cudaError_t ce = cudaStreamEndCapture(e->stream, &g);
  if (r) {
    if (g) cudaGraphDestroy(g);
    return r;
  }
  if (ce != cudaSuccess) {
    set_last_error("graph capture failed: %s", cudaGetErrorString(ce));
    return CN_ERR_CUDA;
  }
  e->graph = g;
  CN_CUDA(cudaGraphInstantiate(&e->gexec, g, 0));
  return 0;
}

static int check_device_error(cn_engine* e) {
  int code = 0;
  int r = device_error_read_and_clear(e->stream, &code);
  if (r) {
    set_last_error("device error read failed: %s", cudaGetErrorString((cudaError_t)r));
    return CN_ERR_CUDA;
  }
  if (code) {
    set_last_error("device-side error code %d (a bounded wait expired inside a kernel)", code);
    return CN_ERR_DEVICE;
  }
  return 0;
}

static int launch_frame(cn_engine* e) {
  if (e->gexec) {
    CN_CUDA(cudaGraphLaunch(e->gexec, e->stream));
  } else {
    CN_TRY(run_steps(e, e->stream, false));
  }
  return 0;
}

}  // namespace cn

// =================================================================== C ABI
extern "C" {

const char* cn_last_error(void) { return cn::last_error_text(); }
int cn_version(void) { return 1; }

int cn_engine_destroy(cn_engine* e) {
  if (!e) return 0;
  cudaSetDevice(e->cfg.device);
  if (e->stream) cudaStreamSynchronize(e->stream);
  if (e->gexec) cudaGraphExecDestroy(e->gexec);
  if (e->graph) cudaGraphDestroy(e->graph);
  for (auto ev : e->tev) cudaEventDestroy(ev);
  if (e->ev_fork) cudaEventDestroy(e->ev_fork);
  if (e->ev_join) cudaEventDestroy(e->ev_join);
  if (e->side) {
    cudaStreamSynchronize(e->side);
    cudaStreamDestroy(e->side);
  }
  if (e->wblob) cudaFree(e->wblob);
  if (e->ablob) cudaFree(e->ablob);
  if (e->dec) cudaFree(e->dec);
  if (e->copy) {
    cudaStreamSynchronize(e->copy);
    cudaStreamDestroy(e->copy);
  }
  for (int i = 0; i < 2; ++i) {
    if (e->stage_ready[i]) cudaEventDestroy(e->stage_ready[i]);
    if (e->stage_free[i]) cudaEventDestroy(e->stage_free[i]);
  }
  if (e->stage_buf) cudaFree(e->stage_buf);
  for (int i = 0; i < 2; ++i)
    if (e->out_ev[i]) cudaEventDestroy(e->out_ev[i]);
  if (e->err_host) cudaFreeHost(e->err_host);
  if (e->stream) cudaStreamDestroy(e->stream);
  delete e;
  return 0;
}

int cn_engine_create(const cn_config* cfg, cn_engine** out) {
  if (!cfg || !out) {
    set_last_error("cn_engine_create: null argument");
    return CN_ERR_ARG;
  }
  *out = nullptr;
  if ((cfg->model != CN_MODEL_39M && cfg->model != CN_MODEL_1B) || cfg->batch < 1 || cfg->batch > 64 ||
      cfg->seed >= (1ull << 16)) {
    set_last_error("cn_engine_create: bad config (model %d, batch %d, seed %llu)", cfg->model, cfg->batch,
                   (unsigned long long)cfg->seed);
    return CN_ERR_ARG;
  }
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || cfg->device < 0 || cfg->device >= ndev) {
    set_last_error("cn_engine_create: device %d not available (%d devices)", cfg->device, ndev);
    return CN_ERR_CUDA;
  }
  cn_engine* e = new cn_engine();
  e->cfg = *cfg;
  e->m = dims_of(cfg->model);
  e->B = cfg->batch;
  int r = 0;
  do {
    if (cudaSetDevice(cfg->device) != cudaSuccess) { set_last_error("cudaSetDevice failed"); r = CN_ERR_CUDA; break; }
    cudaDeviceProp prop;
    cudaGetDeviceProperties(&prop, cfg->device);
    if (prop.major != 10) {
      set_last_error("libchestnut is built for sm_100a; device %d is sm_%d%d", cfg->device, prop.major, prop.minor);
      r = CN_ERR_CUDA;
      break;
    }
    if (cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&e->side, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&e->ev_fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&e->ev_join, cudaEventDisableTiming) != cudaSuccess) {
      set_last_error("stream / event create failed"); r = CN_ERR_CUDA; break;
    }
    // Single-clip frames run the transformer as one persistent kernel;
    // CN_TRUNK=0 selects the per-layer kernels instead.
    e->nsm = prop.multiProcessorCount;
    {
      const char* tv = getenv("CN_TRUNK");
      e->use_trunk = trunk_supported(e->B * kT, e->m.d, e->m.heads) && !(tv && tv[0] == '0');
      // the conv stem as one persistent kernel (any number of clips; batched
      // clips then run the per-layer transformer kernels); CN_STEM=0 selects
      // the per-layer stem kernels
      const char* sv = getenv("CN_STEM");
      e->use_stem = !(sv && sv[0] == '0');
    }
    layout_weights(e);
    if (cudaMalloc((void**)&e->wblob, e->wbytes) != cudaSuccess) {
      set_last_error("cudaMalloc of %zu weight bytes failed", e->wbytes); r = CN_ERR_CUDA; break;
    }
    if ((r = gen_weights(e))) break;
    if ((r = layout_acts(e))) break;
    if ((r = build_plan(e))) break;
    if ((r = rebuild_graph(e))) break;
    if (cudaStreamSynchronize(e->stream) != cudaSuccess) { set_last_error("init sync failed"); r = CN_ERR_CUDA; break; }
  } while (0);
  if (r) {
    std::string msg = cn_last_error();
    cn_engine_destroy(e);
    set_last_error("%s", msg.c_str());
    return r;
  }
  *out = e;
  return 0;
}

int cn_run_frame_device(cn_engine* e, const void* d_warped, const void* d_packed) {
  if (!e) return CN_ERR_ARG;
  CN_CUDA(cudaSetDevice(e->cfg.device));
  if (d_warped)
    CN_CUDA(cudaMemcpyAsync(e->d_warped, d_warped, (size_t)e->B * kWarpedBytes, cudaMemcpyDeviceToDevice, e->stream));
  if (d_packed)
    CN_CUDA(cudaMemcpyAsync(e->d_packed, d_packed, (size_t)e->B * kPacked * 4, cudaMemcpyDeviceToDevice, e->stream));
  CN_TRY(launch_frame(e));
  e->pending = 1;
  return 0;
}

int cn_sync(cn_engine* e) {
  if (!e) return CN_ERR_ARG;
  CN_CUDA(cudaSetDevice(e->cfg.device));
  CN_CUDA(cudaStreamSynchronize(e->stream));
  e->pending = 0;
  return check_device_error(e);
}

int cn_read_output(cn_engine* e, float* out) {
  if (!e || !out) return CN_ERR_ARG;
  CN_CUDA(cudaSetDevice(e->cfg.device));
  CN_CUDA(cudaMemcpyAsync(out, e->out, (size_t)e->B * kNOut * 4, cudaMemcpyDeviceToHost, e->stream));
  return cn_sync(e);
}

int cn_decode_frame(cn_engine* e, const cn_decode_field* fields, int n_fields, float* host_out) {
  if (!e || !fields || !host_out || n_fields < 1 || n_fields > 32) {
    set_last_error("cn_decode_frame: bad arguments");
    return CN_ERR_ARG;
  }
  std::vector<cn_decode_field> f(fields, fields + n_fields);
  int len = 0;
  CN_TRY(cn_decode_layout(f.data(), n_fields, &len));
  CN_CUDA(cudaSetDevice(e->cfg.device));
  const size_t need = (size_t)e->B * len;
  if (need > e->dec_floats) {
    if (e->dec) CN_CUDA(cudaFree(e->dec));
    e->dec = nullptr;
    e->dec_floats = 0;
    CN_CUDA(cudaMalloc(&e->dec, need * 4));
    e->dec_floats = need;
  }
  CN_TRY(cn_decode_outputs(e->out, e->B, kNOut, f.data(), n_fields, e->dec, len, e->stream));
  CN_CUDA(cudaMemcpyAsync(host_out, e->dec, need * 4, cudaMemcpyDeviceToHost, e->stream));
  return cn_sync(e);
}

int cn_run_frame(cn_engine* e, const uint8_t* warped, const float* packed, float* out) {
  if (!e || !warped || !packed) {
    set_last_error("cn_run_frame: null argument");
    return CN_ERR_ARG;
  }
  CN_CUDA(cudaSetDevice(e->cfg.device));
  CN_CUDA(cudaMemcpyAsync(e->d_warped, warped, (size_t)e->B * kWarpedBytes, cudaMemcpyHostToDevice, e->stream));
  CN_CUDA(cudaMemcpyAsync(e->d_packed, packed, (size_t)e->B * kPacked * 4, cudaMemcpyHostToDevice, e->stream));
  CN_TRY(launch_frame(e));
  if (!out) {
    e->pending = 1;
    return 0;
  }
  return cn_read_output(e, out);
}

int cn_stage_input(cn_engine* e, const uint8_t* warped) {
  if (!e || !warped) {
    set_last_error("cn_stage_input: null argument");
    return CN_ERR_ARG;
  }
  if (e->stage_count >= 2) {
    set_last_error("cn_stage_input: two inputs are already staged (run one with cn_run_staged first)");
    return CN_ERR_ARG;
  }
  CN_CUDA(cudaSetDevice(e->cfg.device));
  const size_t bytes = (size_t)e->B * kWarpedBytes;
  if (!e->stage_buf) {
    CN_CUDA(cudaMalloc((void**)&e->stage_buf, 2 * bytes));
    CN_CUDA(cudaStreamCreateWithFlags(&e->copy, cudaStreamNonBlocking));
    for (int i = 0; i < 2; ++i) {
      CN_CUDA(cudaEventCreateWithFlags(&e->stage_ready[i], cudaEventDisableTiming));
      CN_CUDA(cudaEventCreateWithFlags(&e->stage_free[i], cudaEventDisableTiming));
      CN_CUDA(cudaEventRecord(e->stage_free[i], e->stream));
    }
  }
  const int slot = (e->stage_head + e->stage_count) & 1;
  // the slot's previous contents have been moved out by the frame that used them
  CN_CUDA(cudaStreamWaitEvent(e->copy, e->stage_free[slot], 0));
  CN_CUDA(cudaMemcpyAsync(e->stage_buf + slot * bytes, warped, bytes, cudaMemcpyHostToDevice, e->copy));
  CN_CUDA(cudaEventRecord(e->stage_ready[slot], e->copy));
  ++e->stage_count;
  return 0;
}

// The staged input of the oldest cn_stage_input -> the engine's input buffer
// on its stream, then the packed vector; the caller launches the frame.
static int take_staged(cn_engine* e, const float* packed) {
  const size_t bytes = (size_t)e->B * kWarpedBytes;
  const int slot = e->stage_head;
  CN_CUDA(cudaStreamWaitEvent(e->stream, e->stage_ready[slot], 0));
  CN_CUDA(cudaMemcpyAsync(e->d_warped, e->stage_buf + slot * bytes, bytes, cudaMemcpyDeviceToDevice, e->stream));
  CN_CUDA(cudaEventRecord(e->stage_free[slot], e->stream));
  e->stage_head ^= 1;
  --e->stage_count;
  CN_CUDA(cudaMemcpyAsync(e->d_packed, packed, (size_t)e->B * kPacked * 4, cudaMemcpyHostToDevice, e->stream));
  return 0;
}

int cn_run_staged_async(cn_engine* e, const float* packed, float* out) {
  if (!e || !packed || !out) {
    set_last_error("cn_run_staged_async: null argument");
    return CN_ERR_ARG;
  }
  if (e->stage_count == 0 || e->out_count >= 2) {
    set_last_error("cn_run_staged_async: %s", e->stage_count == 0 ? "no input staged (cn_stage_input first)"
                                                                  : "two frames already queued (cn_wait_output first)");
    return CN_ERR_ARG;
  }
  CN_CUDA(cudaSetDevice(e->cfg.device));
  if (!e->err_host) {
    CN_CUDA(cudaHostAlloc((void**)&e->err_host, 2 * sizeof(int), cudaHostAllocDefault));
    for (int i = 0; i < 2; ++i) CN_CUDA(cudaEventCreateWithFlags(&e->out_ev[i], cudaEventDisableTiming));
  }
  CN_TRY(take_staged(e, packed));
  CN_TRY(launch_frame(e));
  const int slot = (e->out_head + e->out_count) & 1;
  CN_CUDA(cudaMemcpyAsync(out, e->out, (size_t)e->B * kNOut * 4, cudaMemcpyDeviceToHost, e->stream));
  CN_CUDA(cudaMemcpyFromSymbolAsync(&e->err_host[slot], g_cn_dev_error, sizeof(int), 0, cudaMemcpyDeviceToHost,
                                    e->stream));
  CN_CUDA(cudaEventRecord(e->out_ev[slot], e->stream));
  ++e->out_count;
  return 0;
}

int cn_wait_output(cn_engine* e) {
  if (!e || e->out_count == 0) {
    set_last_error("cn_wait_output: no frame queued");
    return CN_ERR_ARG;
  }
  CN_CUDA(cudaSetDevice(e->cfg.device));
  const int slot = e->out_head;
  CN_CUDA(cudaEventSynchronize(e->out_ev[slot]));
  e->out_head ^= 1;
  --e->out_count;
  if (e->err_host[slot]) {
    set_last_error("device-side error code %d (a bounded wait expired inside a kernel)", e->err_host[slot]);
    return CN_ERR_DEVICE;
  }
  return 0;
}

int cn_run_staged(cn_engine* e, const float* packed, float* out) {
  if (!e || !packed) {
    set_last_error("cn_run_staged: null argument");
    return CN_ERR_ARG;
  }
  if (e->stage_count == 0) {
    set_last_error("cn_run_staged: no input staged (cn_stage_input first)");
    return CN_ERR_ARG;
  }
  CN_CUDA(cudaSetDevice(e->cfg.device));
  CN_TRY(take_staged(e, packed));
  CN_TRY(launch_frame(e));
  if (!out) {
    e->pending = 1;
    return 0;
  }
  return cn_read_output(e, out);
}

int cn_run_frames(cn_engine* e, int n, const uint8_t* warped, const float* packed0, float* outs) {
  if (!e || n < 0 || !warped || !packed0 || !outs) return CN_ERR_ARG;
  std::vector<float> pk(packed0, packed0 + (size_t)e->B * kPacked);
  for (int f = 0; f < n; ++f) {
    float* o = outs + (size_t)f * e->B * kNOut;
    CN_TRY(cn_run_frame(e, warped + (size_t)f * e->B * kWarpedBytes, pk.data(), o));
    for (int b = 0; b < e->B; ++b)
      memcpy(&pk[(size_t)b * kPacked + 12], o + (size_t)b * kNOut + kNHeadsOut, kFeat * 4);
  }
  return 0;
}

size_t cn_state_bytes(void) {
  return 2 * (size_t)kImgQ * kFrameBytes + (size_t)kFeatQ * kFeat * 4 + (size_t)kDesireQ * kDesire * 4 + kFeat * 4;
}

// Canonical row i of a ring with Q slots after `c` pushes sits in slot (c + i) % Q.
int cn_get_state(cn_engine* e, int clip, void* buf, size_t bytes) {
  if (!e || !buf || clip < 0 || clip >= e->B || bytes < cn_state_bytes()) return CN_ERR_ARG;
  CN_CUDA(cudaSetDevice(e->cfg.device));
  CN_CUDA(cudaStreamSynchronize(e->stream));
  int c = 0;
  CN_CUDA(cudaMemcpy(&c, e->rings.ctr, 4, cudaMemcpyDeviceToHost));
  uint8_t* p = (uint8_t*)buf;
  for (int cam = 0; cam < 2; ++cam)
    for (int i = 0; i < kImgQ; ++i) {
      const uint8_t* src = e->rings.img + (((size_t)clip * 2 + cam) * kImgQ + (c + i) % kImgQ) * kFrameBytes;
      CN_CUDA(cudaMemcpy(p, src, kFrameBytes, cudaMemcpyDeviceToHost));
      p += kFrameBytes;
    }
  for (int i = 0; i < kFeatQ; ++i) {
    CN_CUDA(cudaMemcpy(p, e->rings.feat + ((size_t)clip * kFeatQ + (c + i) % kFeatQ) * kFeat, kFeat * 4,
                       cudaMemcpyDeviceToHost));
    p += kFeat * 4;
  }
  for (int i = 0; i < kDesireQ; ++i) {
    CN_CUDA(cudaMemcpy(p, e->rings.desire + ((size_t)clip * kDesireQ + (c + i) % kDesireQ) * kDesire, kDesire * 4,
                       cudaMemcpyDeviceToHost));
    p += kDesire * 4;
  }
  CN_CUDA(cudaMemcpy(p, e->out + (size_t)clip * kNOut + kNHeadsOut, kFeat * 4, cudaMemcpyDeviceToHost));
  return 0;
}

int cn_set_state(cn_engine* e, int clip, const void* buf, size_t bytes) {
  if (!e || !buf || clip < 0 || clip >= e->B || bytes < cn_state_bytes()) return CN_ERR_ARG;
  CN_CUDA(cudaSetDevice(e->cfg.device));
  CN_CUDA(cudaStreamSynchronize(e->stream));
  int c = 0;
  CN_CUDA(cudaMemcpy(&c, e->rings.ctr, 4, cudaMemcpyDeviceToHost));
  const uint8_t* p = (const uint8_t*)buf;
  for (int cam = 0; cam < 2; ++cam)
    for (int i = 0; i < kImgQ; ++i) {
      uint8_t* dst = e->rings.img + (((size_t)clip * 2 + cam) * kImgQ + (c + i) % kImgQ) * kFrameBytes;
      CN_CUDA(cudaMemcpy(dst, p, kFrameBytes, cudaMemcpyHostToDevice));
      p += kFrameBytes;
    }
  for (int i = 0; i < kFeatQ; ++i) {
    CN_CUDA(cudaMemcpy(e->rings.feat + ((size_t)clip * kFeatQ + (c + i) % kFeatQ) * kFeat, p, kFeat * 4,
                       cudaMemcpyHostToDevice));
    p += kFeat * 4;
  }
  for (int i = 0; i < kDesireQ; ++i) {
    CN_CUDA(cudaMemcpy(e->rings.desire + ((size_t)clip * kDesireQ + (c + i) % kDesireQ) * kDesire, p, kDesire * 4,
                       cudaMemcpyHostToDevice));
    p += kDesire * 4;
  }
  CN_CUDA(cudaMemcpy(e->out + (size_t)clip * kNOut + kNHeadsOut, p, kFeat * 4, cudaMemcpyHostToDevice));
  return 0;
}

int cn_reset_state(cn_engine* e) {
  if (!e) return CN_ERR_ARG;
  CN_CUDA(cudaSetDevice(e->cfg.device));
  CN_CUDA(cudaMemsetAsync(e->rings.img, 0, (size_t)e->B * 2 * kImgQ * kFrameBytes, e->stream));
  CN_CUDA(cudaMemsetAsync(e->rings.feat, 0, (size_t)e->B * kFeatQ * kFeat * 4, e->stream));
  CN_CUDA(cudaMemsetAsync(e->rings.desire, 0, (size_t)e->B * kDesireQ * kDesire * 4, e->stream));
  CN_CUDA(cudaMemsetAsync(e->rings.ctr, 0, sizeof(int), e->stream));
  CN_CUDA(cudaMemsetAsync(e->out, 0, (size_t)e->B * kNOut * 4, e->stream));
  if (e->tctr) CN_CUDA(cudaMemsetAsync(e->tctr, 0, e->tctr_bytes, e->stream));
  if (e->sctr) CN_CUDA(cudaMemsetAsync(e->sctr, 0, stem_counter_bytes(), e->stream));
  CN_CUDA(cudaStreamSynchronize(e->stream));
  return 0;
}

int cn_kernel_list(cn_engine* e, cn_kernel_info* out, int* n_inout) {
  if (!e || !n_inout) return CN_ERR_ARG;
  const int n = (int)e->steps.size();
  if (out) {
    const int m = std::min(n, *n_inout);
    for (int i = 0; i < m; ++i) out[i] = e->steps[i].info;
  }
  *n_inout = n;
  return 0;
}

int cn_profile_frame(cn_engine* e, const uint8_t* warped, const float* packed, float* ms, int* n_inout) {
  if (!e || !warped || !packed || !n_inout) return CN_ERR_ARG;
  CN_CUDA(cudaSetDevice(e->cfg.device));
  const int n = (int)e->steps.size();
  if (!ms || *n_inout < n) {
    *n_inout = n;
    return ms ? CN_ERR_ARG : 0;
  }
  CN_CUDA(cudaMemcpyAsync(e->d_warped, warped, (size_t)e->B * kWarpedBytes, cudaMemcpyHostToDevice, e->stream));
  CN_CUDA(cudaMemcpyAsync(e->d_packed, packed, (size_t)e->B * kPacked * 4, cudaMemcpyHostToDevice, e->stream));
  std::vector<cudaEvent_t> ev(n + 1);
  for (auto& x : ev) CN_CUDA(cudaEventCreate(&x));
  int r = 0;
  CN_CUDA(cudaEventRecord(ev[0], e->stream));
  for (int i = 0; i < n && !r; ++i) {
    r = e->steps[i].fn(e->stream);
    if (!r) r = (int)cudaEventRecord(ev[i + 1], e->stream);
  }
  cudaStreamSynchronize(e->stream);
  for (int i = 0; i < n && !r; ++i) cudaEventElapsedTime(&ms[i], ev[i], ev[i + 1]);
  for (auto& x : ev) cudaEventDestroy(x);
  *n_inout = n;
  if (r) {
    set_last_error("profile frame launch failed (%d)", r);
    return CN_ERR_CUDA;
  }
  return check_device_error(e);
}

int cn_set_timed_class(cn_engine* e, const char* prefix) {
  if (!e) return CN_ERR_ARG;
  CN_CUDA(cudaSetDevice(e->cfg.device));
  CN_CUDA(cudaStreamSynchronize(e->stream));
  for (auto ev : e->tev) cudaEventDestroy(ev);
  e->tev.clear();
  e->timed_prefix = prefix ? prefix : "";
  int cnt = 0;
  for (auto& st : e->steps)
    if (timed(e, st)) ++cnt;
  e->tev.resize(2 * cnt);
  for (auto& ev : e->tev) CN_CUDA(cudaEventCreate(&ev));
  return rebuild_graph(e);
}

int cn_timed_class_ms(cn_engine* e, float* ms, int* n_inout) {
  if (!e || !n_inout) return CN_ERR_ARG;
  CN_CUDA(cudaSetDevice(e->cfg.device));
  const int n = (int)e->tev.size() / 2;
  if (ms) {
    const int m = std::min(n, *n_inout);
    for (int i = 0; i < m; ++i) CN_CUDA(cudaEventElapsedTime(&ms[i], e->tev[2 * i], e->tev[2 * i + 1]));
  }
  *n_inout = n;
  return 0;
}

int cn_engine_info(cn_engine* e, long long* n_params, long long* weight_bytes, int* n_kernels) {
  if (!e) return CN_ERR_ARG;
  if (n_params) *n_params = e->n_params;
  if (weight_bytes) *weight_bytes = (long long)e->wbytes;
  if (n_kernels) *n_kernels = (int)e->steps.size();
  return 0;
}

int cn_output_slices(cn_slice* out, int* n_inout) {
  static const cn_slice S[4] = {{"plan", 0, 2475}, {"lane_lines", 2475, 2739}, {"lead", 2739, 2811},
                                {"hidden_state", 2811, 3323}};
  if (!n_inout) return CN_ERR_ARG;
  if (out)
    for (int i = 0; i < std::min(4, *n_inout); ++i) out[i] = S[i];
  *n_inout = 4;
  return 0;
}

int cn_param_count(int model) {
  if (model != CN_MODEL_39M && model != CN_MODEL_1B) return -1;
  return (int)param_table(model).size();
}

int cn_param_info(int model, int index, char* name, int name_len, int* tensor_id, long long* rows, long long* cols,
                  long long* valid_cols, int* kind) {
  if (model != CN_MODEL_39M && model != CN_MODEL_1B) return CN_ERR_ARG;
  const auto P = param_table(model);
  if (index < 0 || index >= (int)P.size()) return CN_ERR_ARG;
  const ParamDesc& p = P[index];
  if (name && name_len > 0) snprintf(name, (size_t)name_len, "%s", p.name.c_str());
  if (tensor_id) *tensor_id = p.tid;
  if (rows) *rows = p.rows;
  if (cols) *cols = p.cols;
  if (valid_cols) *valid_cols = p.valid;
  if (kind) *kind = p.kind;
  return 0;
}

int cn_gemm_wmma_f16(const void* A, const void* B, float* C, int M, int N, int K, int b_kmajor, int bn, int splits,
                     void* stream) {
  if (!A || !B || !C) {
    set_last_error("cn_gemm_wmma_f16: null pointer");
    return CN_ERR_ARG;
  }
  struct Key {
    const void *a, *b;
    float* c;
    int m, n, k, kmaj, bn, s, dev;
    bool operator==(const Key& o) const {
      return a == o.a && b == o.b && c == o.c && m == o.m && n == o.n && k == o.k && kmaj == o.kmaj && bn == o.bn &&
             s == o.s && dev == o.dev;
    }
  };
  static std::mutex mu;
  static Key keys[16];
  static GemmPlan plans[16];
  static int used = 0, next = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  const Key key{A, B, C, M, N, K, b_kmajor, bn, splits, dev};
  GemmPlan g;
  bool hit = false;
  {
    std::lock_guard<std::mutex> lk(mu);
    for (int i = 0; i < used; ++i)
      if (keys[i] == key) {
        g = plans[i];
        hit = true;
        break;
      }
  }
  if (!hit) {
    GemmParams ep;
    memset(&ep, 0, sizeof(ep));
    ep.epi = EPI_F32_ACCUM;
    ep.out = C;
    ep.ldo = N;
    ep.b_dep = 1;  // a caller's B may come from the previous kernel on the stream
    const bool mn = !b_kmajor;
    int r = gemm_plan(&g, A, K, 0, B, mn ? N : K, 0, M, N, K, 1, mn ? B_MN_MAJOR : B_K_MAJOR, bn, splits, ep);
    if (r) return r < 0 ? r : CN_ERR_CUDA;
    // Programmatic dependent launch: back-to-back calls on one stream overlap
    // the next call's launch and set-up with this call's tail; every operand
    // is read only after griddepcontrol.wait.
    g.pdl = true;
    std::lock_guard<std::mutex> lk(mu);
    keys[next] = key;
    plans[next] = g;
    next = (next + 1) % 16;
    if (used < 16) ++used;
  }
  int r = gemm_launch(g, (cudaStream_t)stream);
  return r ? (r < 0 ? r : CN_ERR_CUDA) : 0;
}

int cn_reduce_rows_f16(const void* x, const void* w, float* out, long long rows, long long len, int cpr, void* stream) {
  if (!x || !w || !out || rows <= 0 || rows > 65535 || len <= 0 || (len % 8) ||
      (reinterpret_cast<uintptr_t>(x) % 16) || (reinterpret_cast<uintptr_t>(w) % 16)) {
    set_last_error("cn_reduce_rows_f16: need rows in [1, 65535], len %% 8 == 0 and 16-byte aligned x, w");
    return CN_ERR_ARG;
  }
  if (cpr <= 0) cpr = rows >= 1184 ? 1 : (rows >= 296 ? 4 : 8);  // enough rows alone fill the GPU
  if (cpr != 1 && cpr != 2 && cpr != 4 && cpr != 8) {
    set_last_error("cn_reduce_rows_f16: chunks_per_row must be 1, 2, 4 or 8");
    return CN_ERR_ARG;
  }
  int r = reduce_rows_launch(x, w, out, rows, len, cpr, (cudaStream_t)stream);
  if (r) {
    set_last_error("reduce launch failed: %s", cudaGetErrorString((cudaError_t)r));
    return CN_ERR_CUDA;
  }
  return 0;
}

int cn_border_gather_s2(const void* act, int G, int B, int H, int W, int C, void* out, void* stream) {
  if (!act || !out || G < 1 || B < 1 || H < 2 || W < 2 || (H % 2) || (W % 2) || C < 8 || (C % 8)) {
    set_last_error("cn_border_gather_s2: bad arguments");
    return CN_ERR_ARG;
  }
  int r = launch_gather_s2((const __half*)act, G, B, H, W, C, (__half*)out, (cudaStream_t)stream);
  if (r) {
    set_last_error("gather launch failed (%d)", r);
    return CN_ERR_CUDA;
  }
  return 0;
}

int cn_device_error(int* code) {
  if (!code) return CN_ERR_ARG;
  int r = device_error_read_and_clear(0, code);
  return r ? CN_ERR_CUDA : 0;
}

int cn_selftest_bounded_wait(int limit_ms, int* code) {
  if (!code || limit_ms < 1 || limit_ms > 10000) return CN_ERR_ARG;
  int r = launch_selftest_wait((unsigned long long)limit_ms * 1000000ull, 0);
  if (r) {
    set_last_error("selftest launch failed: %s", cudaGetErrorString((cudaError_t)r));
    return CN_ERR_CUDA;
  }
  CN_CUDA(cudaDeviceSynchronize());
  r = device_error_read_and_clear(0, code);
  return r ? CN_ERR_CUDA : 0;
}

int cn_dev_alloc(void** ptr, size_t bytes, int device) {
  if (!ptr) return CN_ERR_ARG;
  CN_CUDA(cudaSetDevice(device));
  CN_CUDA(cudaMalloc(ptr, bytes));
  return 0;
}
int cn_dev_free(void* ptr) {
  CN_CUDA(cudaFree(ptr));
  return 0;
}
int cn_host_alloc_pinned(void** ptr, size_t bytes) {
  if (!ptr) return CN_ERR_ARG;
  CN_CUDA(cudaMallocHost(ptr, bytes));
  return 0;
}
int cn_host_free_pinned(void* ptr) {
  CN_CUDA(cudaFreeHost(ptr));
  return 0;
}
int cn_memcpy(void* dst, const void* src, size_t bytes, int kind) {
  const cudaMemcpyKind k = kind == 0 ? cudaMemcpyHostToDevice : (kind == 1 ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice);
  CN_CUDA(cudaMemcpy(dst, src, bytes, k));
  return 0;
}
int cn_memset(void* dst, int value, size_t bytes) {
  CN_CUDA(cudaMemset(dst, value, bytes));
  return 0;
}
int cn_device_synchronize(int device) {
  CN_CUDA(cudaSetDevice(device));
  CN_CUDA(cudaDeviceSynchronize());
  return 0;
}
int cn_engine_stream(cn_engine* e, void** stream) {
  if (!e || !stream) return CN_ERR_ARG;
  *stream = (void*)e->stream;
  return 0;
}

}  // extern "C"
