// Persistent transformer trunk for single-clip frames (M <= 128 token rows).
//
// The 1B frame's transformer streams 100 MB of f16 weights per layer against
// 88 tokens of activations, so it is an HBM stream with small dependent steps
// in between.  Launched as separate kernels, every GEMM pays its launch,
// pipeline fill and split-K epilogue before its successor can touch HBM.  This
// kernel runs the whole trunk (layers x {LN1, QKV, attention, O, LN2, fc1 +
// GELU, fc2}) as one cooperative launch of one CTA per SM.  Steps meet on
// dataflow counters instead of grid barriers: a step waits only for the
// counters of the rows / feature tiles it reads and publishes its own
// completion with a release add.  The weight stream is decoupled from the
// steps:
//
//   warps 0, 1 (lane 0)  stream every weight stage this CTA will consume, over
//                        all layers, into a ring of shared-memory stages with
//                        TMA (alternate stages per warp: a thread's loads
//                        complete one after another).  They wait only for
//                        free stages, never for the steps.
//   warps 2..7           the compute group.  In a GEMM step warps 2 and 3
//                        (lane 0) load the activation k-blocks once their
//                        producers are done, warp 4 lane 0 issues tcgen05.mma
//                        and warps 4..7 run the epilogue (TMEM lane quadrants
//                        0..3); the QKV / fc1 split-K reduction and attention
//                        use all six warps, the row steps warps 4..7.
//
// GEMMs are computed transposed ("swap AB"): D[128 features][ntok tokens] =
// W[128 x 64k] (A, the k-blocked weight tile) x X[ntok x 64k]^T (B), M = 128,
// N = ntok (88 tokens -> 96), f32 accumulator in TMEM.  A GEMM slot is cut
// into units (128-feature tile, split-K part); a unit writes its partial tile
// to an L2-resident scratch.  QKV / fc1: the S units of a feature tile meet on
// an arrival counter, and unit s then reduces tokens [s*M/S, (s+1)*M/S) in
// split order 0..S-1 (deterministic) and applies bias / GELU, so that
// attention and fc2 can start on single heads / tiles.  O / fc2 feed the
// residual stream, whose next reader (LayerNorm) needs whole rows: there the
// CTA of row r sums the row's partials in split order, adds bias and residual
// and normalises in one row step, one hop instead of a reduction hop plus a
// LayerNorm hop.
//
// Every wait is bounded (%globaltimer); on timeout a code lands in the device
// error word and the kernel unwinds instead of hanging.  Counters are
// monotonic across launches (targets derive from a launch epoch), so nothing
// has to be reset between frames.  No TMA multicast.
#include <algorithm>

#include "cn_common.cuh"
#include "cn_gemm.cuh"
#include "cn_ops.cuh"
#include "cn_trunk.cuh"

namespace cn {

namespace {

constexpr int kTrThreads = 256;
constexpr int kComputeThreads = 192;       // warps 2..7
constexpr int kComputeT0 = 64;             // first compute thread
constexpr int kWTileBytes = 128 * 64 * 2;  // one k-block of 128 output features
constexpr int kKbPerStage = 2;              // k-blocks per ring stage (one TMA box each for W and X)
constexpr int kWStageBytes = kKbPerStage * kWTileBytes;
constexpr int kBarCompute = 1, kBarEpi = 2;
constexpr int kPhasesPerLayer = 7;
constexpr int kMaxTrunkSplit = 16;
constexpr int kMaxTiles = 64;  // feature tiles per GEMM slot (N <= 8192)
// Dataflow counters of one layer (u32, monotonic across launches; a step is
// complete for launch e once its counter reaches (e + 1) x contributions):
constexpr int kDepPerLayer = 256;
constexpr int kDepLn1 = 0;    // LN1 rows done (M per launch)
constexpr int kDepLn2 = 1;    // LN2 rows done (M)
constexpr int kDepOp = 2;     // O units whose split-K partials are stored (units_O)
constexpr int kDepFc2p = 3;   // fc2 units whose split-K partials are stored (units_fc2)
constexpr int kDepQkv = 64;   // [tile] QKV feature tile reduced (S_QKV units)
constexpr int kDepAtt = 128;  // [head] attention rows of a head done (clips x 16-row blocks)
constexpr int kDepFc1 = 192;  // [tile] fc1 feature tile reduced (S_fc1 units)
constexpr int kBarRegion = 512;  // barriers, flags, LayerNorm partials
constexpr int kRowChunk = 5;     // split-K slices a row step loads per round trip

__device__ __forceinline__ void named_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
// Generic-proxy global writes of this thread -> visible to async-proxy (TMA) reads.
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ void red_release_add(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ bool dev_error_set() { return *reinterpret_cast<volatile int*>(&g_cn_dev_error) != 0; }

// Phase-trace instrumentation, compiled only with -DCN_TRUNK_TRACE (a
// profiling build): %globaltimer stamps per (layer, phase, CTA, slot).
#ifdef CN_TRUNK_TRACE
__device__ unsigned long long* g_trunk_trace = nullptr;
__device__ unsigned long long* g_trunk_strace = nullptr;  // [layer][4 slots][16 stages][grid][8]
#define CN_TRS(l, gi, stg, k)                                                                                 \
  do {                                                                                                       \
    if (g_trunk_strace && (stg) < 16)                                                                        \
      g_trunk_strace[((((size_t)(l) * 4 + (gi)) * 16 + (stg)) * gridDim.x + blockIdx.x) * 8 + (k)] = global_ns(); \
  } while (0)
#define CN_TR(l, ph, k)                                                                                   \
  do {                                                                                                   \
    if (g_trunk_trace)                                                                                   \
      g_trunk_trace[((((size_t)(l)) * 8 + (ph)) * gridDim.x + blockIdx.x) * 8 + (k)] = global_ns();       \
  } while (0)
#else
#define CN_TR(l, ph, k) \
  do {                  \
  } while (0)
#define CN_TRS(l, gi, stg, k) \
  do {                        \
  } while (0)
#endif

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// The weights are read once per frame and are 16x the L2: their boxes are
// loaded with an evict-first L2 policy, so the stream does not push the
// split-K partials and activations (read again microseconds later) out to
// HBM.  Without it the trunk wrote ~0.5 GB of evicted partials back to DRAM
// per launch, and the frame took 2.7% longer.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void tma_load_4d_hint(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                                 int c2, int c3, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Request [p, p + bytes) into L2 (16-byte aligned address and size).
__device__ __forceinline__ void bulk_prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(p)), "r"(bytes)
               : "memory");
}

// Counters are monotonic across launches and their targets grow with a launch
// epoch, so both wrap around; a counter never trails its target by 2^31 or
// more (it trails by at most the units of one launch), so the signed
// difference orders them.
__device__ __forceinline__ bool ctr_reached(unsigned v, unsigned target) { return (int)(v - target) >= 0; }
__device__ __forceinline__ bool ctr_reached(unsigned long long v, unsigned long long target) {
  return (long long)(v - target) >= 0;
}

// Spin until *ctr has reached target (bounded).  false on timeout or a recorded error.
template <typename T, typename Ld>
__device__ __forceinline__ bool spin_until(const T* ctr, T target, int code, Ld ld) {
  if (ctr_reached(ld(ctr), target)) return true;
  const unsigned long long t0 = global_ns();
  while (!ctr_reached(ld(ctr), target)) {
    if (dev_error_set()) return false;
    if (global_ns() - t0 > kWaitLimitNs) {
      set_dev_error(code);
      return false;
    }
  }
  return true;
}

// Grid barrier of the compute groups (all compute threads call it).
__device__ __forceinline__ bool grid_sync(unsigned long long* ctr, unsigned long long target, volatile int* flag) {
  fence_proxy_async_global();
  named_sync(kBarCompute, kComputeThreads);
  if (threadIdx.x == kComputeT0) {
    // one release per CTA covers the group's writes (ordered by the barrier above)
    fence_acq_rel_gpu();
    red_release_add(ctr, 1ull);
    bool ok = spin_until(ctr, target, 10, ld_acquire_u64);
    fence_acq_rel_gpu();
    *flag = ok && !dev_error_set();
  }
  named_sync(kBarCompute, kComputeThreads);
  return *flag != 0;
}

__device__ __forceinline__ void unit_range(const TrunkArgs& a, int gi, int u, int* nt, int* s, int* kb0, int* kb1) {
  const int S = a.S[gi], KB = a.K[gi] / 64;
  *nt = u / S;
  *s = u % S;
  *kb0 = *s * KB / S;
  *kb1 = (*s + 1) * KB / S;
}

// Position in this CTA's weight stream: the stage starting at k-block kb of
// its unit (layer l, slot gi, feature tile nt) whose k-blocks end at kb1.
// The stream visits layers in order, slots 0..3, and each unit's k-blocks in
// steps of kKbPerStage: the order in which the MMA issuer consumes stages.
struct WPos {
  int l, gi, nt, kb, kb1;
};
__device__ __forceinline__ void wpos_seek(const TrunkArgs& a, WPos& p) {
  while (p.l < a.layers) {
    if ((int)blockIdx.x < a.units[p.gi]) {
      int s;
      unit_range(a, p.gi, blockIdx.x, &p.nt, &s, &p.kb, &p.kb1);
      return;
    }
    if (++p.gi == 4) {
      p.gi = 0;
      ++p.l;
    }
  }
}
__device__ __forceinline__ void wpos_next(const TrunkArgs& a, WPos& p) {
  p.kb += kKbPerStage;
  if (p.kb < p.kb1) return;
  if (++p.gi == 4) {
    p.gi = 0;
    ++p.l;
  }
  wpos_seek(a, p);
}

// TMEM columns [c0, c0 + 16 * NL) of this warp's 32 lanes -> partial rows
// [c0, c0 + 16 * NL) (rows >= M skipped), all NL loads in flight before one
// wait.  Lane i of the warp owns one feature, so every store instruction
// writes one whole 128-byte row segment of the tile-contiguous layout.
template <int NL>
__device__ __forceinline__ void store_cols(uint32_t taddr, int c0, float* dst, int M) {
  uint32_t r[NL][16];
#pragma unroll
  for (int q = 0; q < NL; ++q) tmem_ld16(taddr + c0 + 16 * q, r[q]);
  tmem_ld_wait();
#pragma unroll
  for (int q = 0; q < NL; ++q)
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int t = c0 + 16 * q + j;
      if (t < M) dst[(size_t)t * 128] = __uint_as_float(r[q][j]);
    }
}

// Final value of output (token t, feature n) of GEMM slot QKV or fc1.
__device__ __forceinline__ void store_out(const TrunkArgs& a, int gi, int t, int n, float v) {
  const size_t i = (size_t)t * a.N[gi] + n;
  if (gi == TG_QKV)
    a.qkv[i] = __float2half_rn(v);
  else
    a.u[i] = __float2half_rn(apply_act(v, ACT_GELU));
}


// Split-K reduction of tokens [t0, t1) of feature tile nt of slot QKV or fc1:
// the S slices (S x R rows of 128 features, split order 0..S-1) sit in shared
// memory; the slot's epilogue is compiled in.
// A thread always handles features 4 * (ct % 32) .. + 3 (the stride over
// items is a multiple of 32), so its bias quad b4 is loaded once, early.
static_assert(kComputeThreads % 32 == 0, "reduction items keep their feature quad");
template <int GI>
__device__ __forceinline__ void trunk_reduce(const TrunkArgs& a, const float* sl, float4 b4, int S, int R, int t0,
                                             int t1, int nt, int ct) {
  for (int i = ct; i < (t1 - t0) * 32; i += kComputeThreads) {
    const int tt = i >> 5, fq = i & 31;
    const float* row = sl + tt * 128 + 4 * fq;
    float4 acc = *reinterpret_cast<const float4*>(row);
    for (int q = 1; q < S; ++q) {
      const float4 v = *reinterpret_cast<const float4*>(row + (size_t)q * R * 128);
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    acc.x += b4.x; acc.y += b4.y; acc.z += b4.z; acc.w += b4.w;
    const size_t o = (size_t)(t0 + tt) * a.N[GI] + nt * 128 + 4 * fq;
    const bool g = GI == TG_FC1;
    __align__(8) __half hv[4] = {__float2half_rn(g ? apply_act(acc.x, ACT_GELU) : acc.x),
                                 __float2half_rn(g ? apply_act(acc.y, ACT_GELU) : acc.y),
                                 __float2half_rn(g ? apply_act(acc.z, ACT_GELU) : acc.z),
                                 __float2half_rn(g ? apply_act(acc.w, ACT_GELU) : acc.w)};
    *reinterpret_cast<uint2*>((g ? a.u : a.qkv) + o) = *reinterpret_cast<const uint2*>(hv);
  }
}

// Row step of the residual stream on warps 4..7 (named barrier kBarEpi), in
// ln_row's feature layout: warp q holds features q * d / 4 + 4 * (lane + 32 i).
// With a source slot (O or fc2 of layer sl) row r of x is first brought up to
// date: the split-K partials of its feature tiles are added in split order
// 0..S-1, then the bias, then the old row (the residual), and x is written
// back.  The partials are waited for as a whole (src_done >= target): a row
// needs every feature tile, and every tile every split.  With y the row is
// then normalised into y.  Returns false if the wait expired.
template <int NV>
__device__ __forceinline__ bool trunk_row(const TrunkArgs& a, int src, int sl, const unsigned* src_done,
                                          unsigned target, __half* y, int r, int q, int lane, volatile int* flags,
                                          float (*lnpart)[2], int trl = 0, int trph = 0) {
  constexpr int d = NV * 512;
  float* xr = a.x + (size_t)r * d + q * (d / 4) + 4 * lane;
  float4 v[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i)  // x row r is written only by this CTA's row steps (same threads) or before the launch
    v[i] = __ldcg(reinterpret_cast<const float4*>(xr + 128 * i));
  bool live = true;
  if (src >= 0) {
    float4 b[NV];
    const float* bias = a.bias[src] + (size_t)sl * a.bias_lstride + q * (d / 4) + 4 * lane;
#pragma unroll
    for (int i = 0; i < NV; ++i) b[i] = __ldg(reinterpret_cast<const float4*>(bias + 128 * i));
    if (threadIdx.x == 128) {
      flags[2] = spin_until(src_done, target, 18, ld_acquire_u32);
      CN_TR(trl, trph, 1);
    }
    named_sync(kBarEpi, 128);
    live = flags[2] != 0;
    if (live) {
      // partials [S][d / 128][M][128]: feature tile of v[i] is q * NV + i, column 4 * lane
      const size_t ss = (size_t)a.M * d, ts = (size_t)a.M * 128;
      const float* p = a.pslot[src] + (size_t)r * 128 + 4 * lane + (size_t)q * NV * ts;
      // kRowChunk slices per L2 round trip (a load-then-add loop over a runtime
      // S serialises one round trip per slice); sums stay in split order
      const int S = a.S[src];
      float4 acc[NV];
      for (int s0 = 0; s0 < S; s0 += kRowChunk) {
        float4 t[kRowChunk][NV];
#pragma unroll
        for (int j = 0; j < kRowChunk; ++j)
#pragma unroll
          for (int i = 0; i < NV; ++i)
            t[j][i] = s0 + j < S ? __ldcg(reinterpret_cast<const float4*>(p + (s0 + j) * ss + i * ts))
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < kRowChunk; ++j)
#pragma unroll
          for (int i = 0; i < NV; ++i) {
            if (s0 + j == 0) {
              acc[i] = t[j][i];
            } else if (s0 + j < S) {
              acc[i].x += t[j][i].x; acc[i].y += t[j][i].y; acc[i].z += t[j][i].z; acc[i].w += t[j][i].w;
            }
          }
      }
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        acc[i].x += b[i].x; acc[i].y += b[i].y; acc[i].z += b[i].z; acc[i].w += b[i].w;
        v[i] = make_float4(v[i].x + acc[i].x, v[i].y + acc[i].y, v[i].z + acc[i].z, v[i].w + acc[i].w);
        *reinterpret_cast<float4*>(xr + 128 * i) = v[i];
      }
    }
  }
  if (y) ln_vals<NV>(v, y, r, live, q, lane, lnpart, [] { named_sync(kBarEpi, 128); });
  return live;
}

// Attention of query rows [q0, q0 + 16) of (clip b, head h).  Shared layout
// (halves, row stride HD + 8): Q rows 0..15, K rows 16..111, V rows 112..207.
constexpr int kAttnKW = 16;                  // keys per warp
constexpr int kAttnWarpsT = kAttnRows / kAttnKW;  // all six compute warps split the keys
static_assert(kAttnWarpsT * 32 == kComputeThreads, "every compute warp takes a key block");

template <int HD>
__device__ __forceinline__ void attn16_stage(const __half* __restrict__ qkv, __half* base, int T, int d, int b, int h,
                                             int q0, int tid, int nthr) {
  constexpr int LD = HD + 8, CPR = HD / 8;
  const size_t ld = 3 * (size_t)d;
  const __half* src = qkv + (size_t)b * T * ld + (size_t)h * HD;
  for (int i = tid; i < (16 + 2 * kAttnRows) * CPR; i += nthr) {
    const int row = i / CPR, c = (i % CPR) * 8;
    const int mat = row < 16 ? 0 : (row < 16 + kAttnRows ? 1 : 2);
    const int r = mat == 0 ? q0 + row : row - 16 - (mat - 1) * kAttnRows;
    __half* dst = base + row * LD + c;
    if (r < T)
      cp_async16(dst, src + (size_t)r * ld + (size_t)mat * d + c);
    else
      *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
  }
}

// Warp w: scores of the 16 rows against keys [16w, 16w+16), their row max m
// and sum l of exp(s - m), and O_w = exp(S - m) V_w (P split f16 hi + lo).
// Results go to shared memory over the staging rows, which every warp is done
// with by then: float O[6][16][HD], then float ml[6][16][2].
template <int HD>
__device__ __forceinline__ void attn16_keys(__half* base, int T, int w, int lane) {
  constexpr int LD = HD + 8;
  const __half* Qs = base;
  const __half* Ks = base + 16 * LD;
  const __half* Vs = base + (16 + kAttnRows) * LD;
  constexpr int NJ = kAttnKW / 8;  // 8-key score tiles per warp
  const int g = lane >> 2, t4 = lane & 3;
  float s[NJ][4];
#pragma unroll
  for (int j = 0; j < NJ; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
  for (int kk = 0; kk < HD; kk += 16) {
    uint32_t a[4];
    {
      const int i = lane >> 3;
      ldsm_x4(a, Qs + ((i & 1) * 8 + (lane & 7)) * LD + kk + (i >> 1) * 8);
    }
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      uint32_t bb[2];
      ldsm_x2(bb, Ks + (kAttnKW * w + 8 * j + (lane & 7)) * LD + kk + ((lane >> 3) & 1) * 8);
      mma16816(s[j], a, bb[0], bb[1]);
    }
  }
  const float scale = 1.0f / sqrtf((float)HD);
  float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
  for (int j = 0; j < NJ; ++j)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const bool valid = kAttnKW * w + 8 * j + 2 * t4 + e < T;
      s[j][e] = valid ? s[j][e] * scale : -INFINITY;
      s[j][2 + e] = valid ? s[j][2 + e] * scale : -INFINITY;
      m0 = fmaxf(m0, s[j][e]);
      m1 = fmaxf(m1, s[j][2 + e]);
    }
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
    m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, o));
  }
  float l0 = 0.f, l1 = 0.f;
#pragma unroll
  for (int j = 0; j < NJ; ++j)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      s[j][e] = m0 == -INFINITY ? 0.f : expf(s[j][e] - m0);
      s[j][2 + e] = m1 == -INFINITY ? 0.f : expf(s[j][2 + e] - m1);
      l0 += s[j][e];
      l1 += s[j][2 + e];
    }
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, o);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o);
  }
  float o[HD / 8][4];
#pragma unroll
  for (int nb = 0; nb < HD / 8; ++nb) o[nb][0] = o[nb][1] = o[nb][2] = o[nb][3] = 0.f;
#pragma unroll
  for (int ks = 0; ks < kAttnKW / 16; ++ks) {
    uint32_t ahi[4], alo[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int j = 2 * ks + (q >> 1);
      const float x = s[j][(q & 1) * 2], y = s[j][(q & 1) * 2 + 1];
      const __half2 hi = __floats2half2_rn(x, y);
      const float2 hf = __half22float2(hi);
      ahi[q] = pack_h2(hi);
      alo[q] = pack_h2(__floats2half2_rn(x - hf.x, y - hf.y));
    }
#pragma unroll
    for (int nb = 0; nb < HD / 8; nb += 2) {
      uint32_t bv[4];
      const int i = lane >> 3;
      ldsm_x4_t(bv, Vs + (kAttnKW * w + 16 * ks + (i & 1) * 8 + (lane & 7)) * LD + 8 * nb + (i >> 1) * 8);
      mma16816(o[nb], ahi, bv[0], bv[1]);
      mma16816(o[nb], alo, bv[0], bv[1]);
      mma16816(o[nb + 1], ahi, bv[2], bv[3]);
      mma16816(o[nb + 1], alo, bv[2], bv[3]);
    }
  }
  // every warp is done with Q and K before they are overwritten
  named_sync(kBarCompute, kComputeThreads);
  float* O = reinterpret_cast<float*>(base) + (size_t)w * 16 * HD;
#pragma unroll
  for (int nb = 0; nb < HD / 8; ++nb) {
    const int col = 8 * nb + 2 * t4;
    *reinterpret_cast<float2*>(O + g * HD + col) = make_float2(o[nb][0], o[nb][1]);
    *reinterpret_cast<float2*>(O + (g + 8) * HD + col) = make_float2(o[nb][2], o[nb][3]);
  }
  float* ml = reinterpret_cast<float*>(base) + kAttnWarpsT * 16 * HD + w * 32;
  if (t4 == 0) {
    ml[2 * g] = m0;
    ml[2 * g + 1] = l0;
    ml[2 * (g + 8)] = m1;
    ml[2 * (g + 8) + 1] = l1;
  }
}

// Combine the key blocks and store rows [q0, q0+16) of out f16 [B*T][d].
template <int HD>
__device__ __forceinline__ void attn16_combine(const __half* base, __half* __restrict__ out, int T, int d, int b, int h,
                                               int q0, int tid, int nthr) {
  const float* O = reinterpret_cast<const float*>(base);
  const float* ml = O + kAttnWarpsT * 16 * HD;
  for (int i = tid; i < 16 * HD / 4; i += nthr) {
    const int r = i / (HD / 4), c = (i % (HD / 4)) * 4;
    if (q0 + r >= T) continue;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarpsT; ++w) M = fmaxf(M, ml[w * 32 + 2 * r]);
    float L = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < kAttnWarpsT; ++w) {
      const float mw = ml[w * 32 + 2 * r];
      const float f = mw == -INFINITY ? 0.f : expf(mw - M);
      L += f * ml[w * 32 + 2 * r + 1];
      const float4 v = *reinterpret_cast<const float4*>(O + ((size_t)w * 16 + r) * HD + c);
      acc.x += f * v.x; acc.y += f * v.y; acc.z += f * v.z; acc.w += f * v.w;
    }
    __align__(8) __half hv[4] = {__float2half_rn(acc.x / L), __float2half_rn(acc.y / L), __float2half_rn(acc.z / L),
                                 __float2half_rn(acc.w / L)};
    *reinterpret_cast<uint2*>(out + ((size_t)b * T + q0 + r) * d + (size_t)h * HD + c) = *reinterpret_cast<uint2*>(hv);
  }
}

// staging (Q 16 rows, K and V 96 rows, row stride hd + 8 halves), later
// reused for the per-warp partial outputs and row statistics
size_t attn16_smem_bytes(int hd) {
  const size_t stage = (size_t)(16 + 2 * kAttnRows) * (hd + 8) * 2;
  const size_t part = (size_t)kAttnWarpsT * 16 * hd * 4 + (size_t)kAttnWarpsT * 32 * 4;
  return stage > part ? stage : part;
}

template <int HD, int NV>
__global__ void __launch_bounds__(kTrThreads, 1)
    k_trunk(const __grid_constant__ TrunkMaps maps, const __grid_constant__ TrunkArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int ST = a.stages;
  uint64_t* fullW = reinterpret_cast<uint64_t*>(smem + a.bar_off);
  uint64_t* fullX = fullW + 8;
  uint64_t* empty = fullW + 16;
  uint64_t* done = fullW + 24;
  uint64_t* fixb = fullW + 25;  // reduction slices landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fullW + 27);
  volatile int* flags = reinterpret_cast<volatile int*>(fullW + 28);  // [0] grid barrier, [1] tile counter
  float(*lnpart)[2] = reinterpret_cast<float(*)[2]>(fullW + 30);     // 4 x 2 floats
  uint8_t* aux = smem + a.aux_off;  // attention staging / split-K reduction (phases never overlap)
  __half* attn = reinterpret_cast<__half*>(aux);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&fullW[s], 1);
      mbar_init(&fullX[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    mbar_init(fixb, 1);
    fence_barrier_init();
    for (int g = 0; g < 4; ++g) {
      tma_prefetch_desc(&maps.w[g]);
      tma_prefetch_desc(&maps.x[g]);
      tma_prefetch_desc(&maps.p[g]);
    }
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const unsigned epoch = *reinterpret_cast<volatile unsigned*>(a.epoch);
  if (blockIdx.x == 0 && threadIdx.x == 0 && a.bump) atomicAdd(a.bump, 1);

  if (warp < 2) {
    // ------------------------------------------------ weight stream
    // Two issuing warps (k-blocks alternate between them): a thread's TMA
    // loads complete one after another, so throughput scales with issuers.
    if (lane == 0) {
      uint32_t last = 0;
      bool ok = true;
      WPos cur = {0, 0, 0, 0, 0};
      wpos_seek(a, cur);
      const uint64_t wpol = l2_policy_evict_first();
      // one stage = k-blocks kb, kb+1 (a box past the unit's range loads
      // the neighbour's k-block, or zeros past K; the MMA skips it)
      for (uint32_t g = 0; cur.l < a.layers; ++g, wpos_next(a, cur)) {
        if ((int)(g & 1) != warp) continue;
        const int st = (int)(g % ST);
        const uint32_t ph = (g / ST) & 1;
        if (!mbar_wait(&empty[st], ph ^ 1, 14)) {
          ok = false;
          break;
        }
        {
          int nt_, s_, kb0_, kb1_;
          unit_range(a, cur.gi, blockIdx.x, &nt_, &s_, &kb0_, &kb1_);
          CN_TRS(cur.l, cur.gi, (cur.kb - kb0_) / kKbPerStage, 3);
        }
        mbar_arrive_expect_tx(&fullW[st], kWStageBytes);
        tma_load_4d_hint(smem + st * a.stage_bytes, &maps.w[cur.gi], &fullW[st], 0, cur.nt * 128, cur.kb, cur.l, wpol);
        last = g + 1;
      }
      if (!ok || dev_error_set()) {
        // do not leave a TMA write in flight into shared memory of an exiting CTA
        for (uint32_t i = last > (uint32_t)ST ? last - ST : 0; i < last; ++i)
          if ((int)(i & 1) == warp) mbar_wait(&fullW[i % ST], (i / ST) & 1, 0, 100000000ull);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------ compute group (warps 2..7)
    // Dataflow instead of phase barriers: every step waits only for the
    // counters of the data it reads (see the dependency table in dep_*), and
    // publishes its own completion with a release add.  A CTA runs its steps
    // in layer order, and each wait targets steps of earlier order, so the
    // waits cannot form a cycle.
    const int ct = threadIdx.x - kComputeT0;
    const unsigned ep1 = epoch + 1u;
    uint32_t gx = 0, gm = 0, ndone = 0, nfix = 0, x_last = 0;
    bool ok = true;
    const int QB = (a.T + 15) / 16;
    const int att_units = a.B * a.heads * QB;
    for (int l = 0; l < a.layers && ok; ++l) {
      unsigned* dep = a.dep + (size_t)l * kDepPerLayer;
      for (int ph = 0; ph < kPhasesPerLayer && ok; ++ph) {
        if (ph == 0 || ph == 4) {
          // ---------------- row step (fc2 of layer l-1 / O of layer l -> x, LayerNorm -> h / h2),
          // warps 4..7, one row at a time
          const bool first = ph == 0;
          int src = -1, sl = l;
          const unsigned* sd = dep + kDepOp;
          unsigned tgt = (unsigned)a.units[TG_O] * ep1;
          if (!first) {
            src = TG_O;
          } else if (l > 0) {
            src = TG_FC2;
            sl = l - 1;
            sd = a.dep + (size_t)(l - 1) * kDepPerLayer + kDepFc2p;
            tgt = (unsigned)a.units[TG_FC2] * ep1;
          }
          if (warp >= 4)
            for (int r = blockIdx.x; r < a.M; r += gridDim.x) {
              if (threadIdx.x == 128) CN_TR(l, ph, 0);
              trunk_row<NV>(a, src, sl, sd, tgt, first ? a.h : a.h2, r, warp & 3, lane, flags, lnpart, l, ph);
              fence_proxy_async_global();  // the normalised rows are read by TMA
              named_sync(kBarEpi, 128);
              if (threadIdx.x == 128) {
                red_release_add(dep + (first ? kDepLn1 : kDepLn2), 1u);
                CN_TR(l, ph, 2);
              }
            }
        } else if (ph == 2) {
          // ---------------- attention, one (clip, head, 16 query rows) per CTA
          for (int uu = blockIdx.x; uu < att_units; uu += gridDim.x) {
            const int qb = uu % QB, h = (uu / QB) % a.heads, b = uu / (QB * a.heads);
            if (threadIdx.x == kComputeT0) {
              CN_TR(l, ph, 0);
              // q, k and v of head h (a 128-feature QKV tile holds 128 / HD heads)
              const unsigned tgt = (unsigned)a.S[TG_QKV] * ep1;
              bool met = spin_until(dep + kDepQkv + (h * HD) / 128, tgt, 19, ld_acquire_u32);
              met = met && spin_until(dep + kDepQkv + (a.d + h * HD) / 128, tgt, 19, ld_acquire_u32);
              met = met && spin_until(dep + kDepQkv + (2 * a.d + h * HD) / 128, tgt, 19, ld_acquire_u32);
              fence_acq_rel_gpu();
              flags[2] = met;
              CN_TR(l, ph, 1);
            }
            named_sync(kBarCompute, kComputeThreads);
            if (flags[2] == 0) break;  // uniform: read after the barrier
            attn16_stage<HD>(a.qkv, attn, a.T, a.d, b, h, 16 * qb, ct, kComputeThreads);
            cp_async_wait_all();
            named_sync(kBarCompute, kComputeThreads);
            if (threadIdx.x == kComputeT0) CN_TR(l, ph, 2);
            attn16_keys<HD>(attn, a.T, warp - 2, lane);
            named_sync(kBarCompute, kComputeThreads);
            attn16_combine<HD>(attn, a.att, a.T, a.d, b, h, 16 * qb, ct, kComputeThreads);
            fence_proxy_async_global();  // the attention rows are read by TMA
            named_sync(kBarCompute, kComputeThreads);
            if (threadIdx.x == kComputeT0) {
              red_release_add(dep + kDepAtt + h, 1u);
              CN_TR(l, ph, 3);
            }
          }
        } else {
          // ---------------- GEMM slot
          const int gi = ph == 1 ? TG_QKV : (ph == 3 ? TG_O : (ph == 5 ? TG_FC1 : TG_FC2));
          if ((int)blockIdx.x < a.units[gi]) {
            if (threadIdx.x == kComputeT0) CN_TR(l, ph, 0);
            int nt, s, kb0, kb1;
            unit_range(a, gi, blockIdx.x, &nt, &s, &kb0, &kb1);
            const int nkb = kb1 - kb0;
            const int S = a.S[gi], M = a.M, R = a.R[gi];
            const int t0 = s * M / S, t1 = (s + 1) * M / S;
            // O and fc2 units only publish partials: the row steps reduce them
            const bool rowred = gi == TG_O || gi == TG_FC2;
            // bias quad of this thread's reduction features, in flight during the MMAs
            float4 b4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (S > 1 && !rowred)
              b4 = __ldg(reinterpret_cast<const float4*>(a.bias[gi] + (size_t)l * a.bias_lstride + nt * 128) +
                         (ct & 31));
            if (warp == 2 || warp == 3) {
              // activation k-blocks: warp 2 the even stages, warp 3 the odd
              // ones, each once the producers of its k-blocks are done: QKV /
              // fc1 read every row of h / h2; an O stage reads the heads, an
              // fc2 stage the fc1 feature tiles of its own k-blocks, so the
              // MMAs start on the first ready stage
              if (lane == 0) {
                bool met = true;
                if (gi == TG_QKV || gi == TG_FC1)
                  met = spin_until(dep + (gi == TG_QKV ? kDepLn1 : kDepLn2), (unsigned)M * ep1, 20, ld_acquire_u32);
                if (warp == 2) CN_TR(l, ph, 1);
                for (int i = 0; i < nkb && met; i += kKbPerStage, ++gx) {
                  if ((int)(gx & 1) != warp - 2) continue;
                  if (gi == TG_O || gi == TG_FC2) {
                    const int c0 = (kb0 + i) * 64, c1 = min(kb0 + i + kKbPerStage, kb1) * 64 - 1;
                    if (gi == TG_O) {
                      for (int h = c0 / HD; h <= c1 / HD && met; ++h)
                        met = spin_until(dep + kDepAtt + h, (unsigned)att_units / a.heads * ep1, 20, ld_acquire_u32);
                    } else {
                      for (int t = c0 / 128; t <= c1 / 128 && met; ++t)
                        met = spin_until(dep + kDepFc1 + t, (unsigned)a.S[TG_FC1] * ep1, 20, ld_acquire_u32);
                    }
                    if (!met) break;
                  }
                  fence_proxy_async_global();
                  const int st = (int)(gx % ST);
                  const uint32_t par = (gx / ST) & 1;
                  if (!mbar_wait(&empty[st], par ^ 1, 12)) break;
                  CN_TRS(l, gi, i / kKbPerStage, 4);
                  mbar_arrive_expect_tx(&fullX[st], (uint32_t)(kKbPerStage * a.x_bytes));
                  tma_load_3d(smem + st * a.stage_bytes + kWStageBytes, &maps.x[gi], &fullX[st], 0, 0, kb0 + i);
                  x_last = gx + 1;
                }
              }
              __syncwarp();
            }
            if (warp == 4 && lane == 0) {
              tc_fence_after();
              const uint32_t idesc = umma_idesc_f16(a.ntok, false);
              // kernel-parameter fields held in registers: the asm memory
              // clobbers of the waits and MMAs would otherwise reload them
              // per instruction
              const int stage_bytes = a.stage_bytes, x_bytes = a.x_bytes;
              for (int i = 0; i < nkb; i += kKbPerStage, ++gm) {
                const int st = (int)(gm % ST);
                const uint32_t par = (gm / ST) & 1;
                if (!mbar_wait(&fullW[st], par, 13)) break;
                CN_TRS(l, gi, i / kKbPerStage, 0);
                if (!mbar_wait(&fullX[st], par, 1)) break;
                CN_TRS(l, gi, i / kKbPerStage, 1);
                tc_fence_after();
                const uint32_t wa = smem_u32(smem + st * stage_bytes);
                const uint32_t xa = wa + kWStageBytes;
                for (int h = 0; h < kKbPerStage && i + h < nkb; ++h)
#pragma unroll
                  for (int k = 0; k < 4; ++k)
                    tc_mma_f16(tmem, umma_desc_sw128(wa + h * kWTileBytes + k * 32, 16, 1024),
                               umma_desc_sw128(xa + h * x_bytes + k * 32, 16, 1024), idesc,
                               (i > 0 || h > 0 || k > 0) ? 1u : 0u);
                tc_commit(&empty[st]);
                CN_TRS(l, gi, i / kKbPerStage, 2);
              }
              tc_commit(done);
            }
            __syncwarp();
            if (warp >= 4) {
              const int e = threadIdx.x - 128;  // == 32 * (warp & 3) + lane: TMEM lane / feature in tile
              const int n = nt * 128 + e;
              const uint32_t taddr = tmem + ((uint32_t)((warp & 3) * 32) << 16);
              const bool have = mbar_wait(done, ndone & 1, 15);
              if (threadIdx.x == 128) CN_TR(l, ph, 2);
              tc_fence_after();
              if (S == 1 && !rowred) {
                const float bv = a.bias[gi][(size_t)l * a.bias_lstride + n];
                if (have)
                  for (int c = 0; c < a.ntok; c += 16) {
                    uint32_t r[16];
                    tmem_ld16(taddr + c, r);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                      if (c + j < M) store_out(a, gi, c + j, n, __uint_as_float(r[j]) + bv);
                  }
                tc_fence_before();
              } else {
                // partial tile -> global, straight from the TMEM registers
                // (staging in shared memory and one TMA store per warp took
                // ~0.5 us longer per unit).  QKV / fc1: the S units of this
                // feature tile meet on an arrival counter; unit s then reduces
                // tokens [t0, t1) from one TMA box holding all S partials
                // (split order 0..S-1) on the whole compute group.  O / fc2:
                // the unit is done; the row steps reduce.
                float* dst = a.pslot[gi] + ((size_t)s * (a.N[gi] / 128) + nt) * (size_t)M * 128 + e;
                if (have) {
                  int c0 = 0;
                  for (; c0 + 64 <= a.ntok; c0 += 64) store_cols<4>(taddr, c0, dst, M);
                  if (c0 + 32 <= a.ntok) {
                    store_cols<2>(taddr, c0, dst, M);
                    c0 += 32;
                  }
                  if (c0 < a.ntok) store_cols<1>(taddr, c0, dst, M);
                }
                tc_fence_before();
                fence_proxy_async_global();  // QKV / fc1 partials are read by TMA
                named_sync(kBarEpi, 128);
                // the barrier orders every epilogue thread's stores before the
                // release add (TMA readers fence their loads)
                if (rowred) {
                  if (e == 0) {
                    red_release_add(dep + (gi == TG_O ? kDepOp : kDepFc2p), 1u);
                    CN_TR(l, ph, 3);
                  }
                } else if (e == 0) {
                  unsigned* ctr = a.tile_ctr + ((size_t)l * 4 + gi) * kMaxTiles + nt;
                  red_release_add(ctr, 1u);
                  const bool met = spin_until(ctr, (unsigned)S * ep1, 11, ld_acquire_u32);
                  fence_acq_rel_gpu();
                  fence_proxy_async_global();
                  flags[1] = met && have;
                  if (met && have) {
                    mbar_arrive_expect_tx(fixb, (uint32_t)(S * R) * 512u);
                    tma_load_4d(aux, &maps.p[gi], fixb, 0, t0, nt, 0);
                  }
                }
              }
            }
            // the whole compute group: reduce (split units), then publish
            named_sync(kBarCompute, kComputeThreads);
            if (!rowred) {
              if (S > 1) {
                bool landed = false;
                if (flags[1]) {
                  landed = mbar_wait(fixb, nfix & 1, 16);
                  ++nfix;
                }
                if (landed) {
                  const float* sl = reinterpret_cast<const float*>(aux);
                  if (gi == TG_QKV)
                    trunk_reduce<TG_QKV>(a, sl, b4, S, R, t0, t1, nt, ct);
                  else
                    trunk_reduce<TG_FC1>(a, sl, b4, S, R, t0, t1, nt, ct);
                }
              }
              fence_proxy_async_global();  // outputs read by cp.async (qkv, attention) and TMA (u, fc2)
              named_sync(kBarCompute, kComputeThreads);
              // feature tile nt gained one unit
              if (threadIdx.x == kComputeT0) {
                red_release_add(dep + (gi == TG_QKV ? kDepQkv : kDepFc1) + nt, 1u);
                CN_TR(l, ph, 3);
              }
            }
            ++ndone;
          }
        }
        // one uniform verdict per step for the whole compute group (loops
        // with named barriers must not diverge between warps)
        named_sync(kBarCompute, kComputeThreads);
        if (threadIdx.x == kComputeT0) flags[3] = !dev_error_set();
        named_sync(kBarCompute, kComputeThreads);
        ok = flags[3] != 0;
      }
    }
    // the last fc2 brought into x, and the final LayerNorm of each row into hf
    if (ok && warp >= 4)
      for (int r = blockIdx.x; r < a.M; r += gridDim.x)
        trunk_row<NV>(a, TG_FC2, a.layers - 1, a.dep + (size_t)(a.layers - 1) * kDepPerLayer + kDepFc2p,
                      (unsigned)a.units[TG_FC2] * ep1, a.hf, r, warp & 3, lane, flags, lnpart);
    // one grid barrier per launch: every CTA has read the epoch before it moves
    // on, and every row of hf is final after it
    if (!grid_sync(a.grid_ctr, (unsigned long long)ep1 * gridDim.x, &flags[0])) ok = false;
    if (ok && a.tw[0] && threadIdx.x == kComputeT0) {
      // this CTA's share of the tail weights into L2 while the pooling runs
      for (int i = 0; i < 3; ++i) {
        const size_t bytes = (size_t)a.tN[i] * a.tK[i] * 2, part = (bytes / gridDim.x + 15) & ~size_t(15);
        const size_t off = part * blockIdx.x;
        if (off < bytes)
          bulk_prefetch_l2(reinterpret_cast<const uint8_t*>(a.tw[i]) + off, (uint32_t)min(part, bytes - off));
      }
    }
    if (ok && a.pooled) {
      // token mean of each clip's final LayerNorm rows: a CTA owns 16 clip
      // columns, thread ct sums row chunk ct / 16 (of 12) of column ct % 16
      // (the loads of a chunk in flight together), and the 12 chunk sums are
      // added in chunk order: deterministic, one L2 round trip per chunk
      constexpr int kPoolCols = 16, kPoolChunks = kComputeThreads / kPoolCols;
      float* pp = reinterpret_cast<float*>(aux);
      const int j = ct / kPoolCols, q = ct % kPoolCols;
      const int t0 = j * a.T / kPoolChunks, t1 = (j + 1) * a.T / kPoolChunks;
      for (int c0 = blockIdx.x * kPoolCols; c0 < a.B * a.d; c0 += gridDim.x * kPoolCols) {
        const int b = (c0 + q) / a.d, c = (c0 + q) % a.d;
        const __half* y = a.hf + (size_t)b * a.T * a.d + c;
        float sum = 0.f;
#pragma unroll 8
        for (int t = t0; t < t1; ++t) sum += __half2float(__ldcg(y + (size_t)t * a.d));
        pp[j * kPoolCols + q] = sum;
        named_sync(kBarCompute, kComputeThreads);
        if (j == 0) {
          float tot = 0.f;
          for (int i = 0; i < kPoolChunks; ++i) tot += pp[i * kPoolCols + q];
          a.pooled[(size_t)b * a.d + c] = __float2half_rn(tot / (float)a.T);
        }
        named_sync(kBarCompute, kComputeThreads);
      }
      if (threadIdx.x == kComputeT0 && a.tw[0]) red_release_add(a.tail_ctr, 1u);
    }
    // tail products: one warp per output (two in flight), lane sums added in a
    // fixed shuffle tree; phase i starts once every CTA finished phase i - 1
    if (ok && a.pooled && a.tw[0]) {
      const int gw = blockIdx.x * (kComputeThreads / 32) + (warp - 2), nw = gridDim.x * (kComputeThreads / 32);
      for (int tp = 0; tp < 3 && ok; ++tp) {
        if (threadIdx.x == kComputeT0) flags[2] = spin_until(a.tail_ctr + tp, gridDim.x * ep1, 22, ld_acquire_u32);
        named_sync(kBarCompute, kComputeThreads);
        if (flags[2] == 0) {
          ok = false;
          break;
        }
        const __half* xv = tp == 0 ? a.pooled : (tp == 1 ? a.hid16 : a.z);
        // lane = (k-block group kq, 16-byte chunk c8): every load instruction of
        // the warp reads four whole 128-byte k-block rows of one output
        const int N = a.tN[tp], nv = a.tK[tp] / 256, c8 = lane & 7, kq = lane >> 3;
        const __half* wb = a.tw[tp] + (size_t)kq * N * 64 + c8 * 8;
        const size_t wstep = (size_t)4 * N * 64;  // four k-blocks further
        uint4 xq[8];
#pragma unroll
        for (int c = 0; c < 8; ++c)
          xq[c] = c < nv ? __ldcg(reinterpret_cast<const uint4*>(xv + (kq + 4 * c) * 64 + c8 * 8))
                         : make_uint4(0, 0, 0, 0);
        for (int n0 = gw; n0 < N; n0 += 2 * nw) {
          float acc[2] = {0.f, 0.f};
          uint4 wv[2][8];
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int n = n0 + j * nw;
            const __half* wr = wb + (size_t)(n < N ? n : 0) * 64;
#pragma unroll
            for (int c = 0; c < 8; ++c)
              wv[j][c] = c < nv && n < N ? __ldg(reinterpret_cast<const uint4*>(wr + c * wstep)) : make_uint4(0, 0, 0, 0);
          }
#pragma unroll
          for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const __half2* wh = reinterpret_cast<const __half2*>(&wv[j][c]);
              const __half2* xh = reinterpret_cast<const __half2*>(&xq[c]);
#pragma unroll
              for (int e2 = 0; e2 < 4; ++e2) {
                const float2 wf = __half22float2(wh[e2]), xf = __half22float2(xh[e2]);
                acc[j] = fmaf(wf.x, xf.x, acc[j]);
                acc[j] = fmaf(wf.y, xf.y, acc[j]);
              }
            }
#pragma unroll
          for (int j = 0; j < 2; ++j) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
          }
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int n = n0 + j * nw;
            if (lane == 0 && n < N) {
              const float v = acc[j] + a.tb[tp][n];
              if (tp == 0) {
                const __half hv = __float2half_rn(tanhf(v));
                a.hid16[n] = hv;
                a.out[a.out_hid + n] = __half2float(hv);
              } else if (tp == 1) {
                a.z[n] = __float2half_rn(fmaxf(v, 0.0f));
              } else {
                a.out[n] = v;
              }
            }
          }
        }
        if (tp < 2) {
          named_sync(kBarCompute, kComputeThreads);
          if (threadIdx.x == kComputeT0) red_release_add(a.tail_ctr + tp + 1, 1u);
        }
      }
    }
    if ((warp == 2 || warp == 3) && lane == 0 && !ok) {
      for (uint32_t i = x_last > (uint32_t)ST ? x_last - ST : 0; i < x_last; ++i)
        if ((int)(i & 1) == warp - 2) mbar_wait(&fullX[i % ST], (i / ST) & 1, 0, 100000000ull);
    }
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem, 128);
  if (blockIdx.x == 0 && threadIdx.x == 0) atomicAdd(a.epoch, 1u);
}

using TrunkFn = void (*)(TrunkMaps, TrunkArgs);

TrunkFn trunk_kernel(int hd, int d) {
  if (hd == 64 && d == 512) return reinterpret_cast<TrunkFn>(k_trunk<64, 1>);
  if (hd == 128 && d == 2048) return reinterpret_cast<TrunkFn>(k_trunk<128, 4>);
  if (hd == 64 && d == 1024) return reinterpret_cast<TrunkFn>(k_trunk<64, 2>);
  if (hd == 128 && d == 1024) return reinterpret_cast<TrunkFn>(k_trunk<128, 2>);
  return nullptr;
}

int trunk_split(int ntiles, int kb, int nsm) {
  int s = nsm / ntiles;
  if (s > kb) s = kb;
  if (s > kMaxTrunkSplit) s = kMaxTrunkSplit;
  return s < 1 ? 1 : s;
}

}  // namespace

bool trunk_supported(int M, int d, int heads) {
  return M > 0 && M <= 128 && heads > 0 && d % heads == 0 && trunk_kernel(d / heads, d) != nullptr;
}

size_t trunk_part_floats(int M, int d, int mlp, int layers, int nsm) {
  (void)layers;
  const int N[4] = {3 * d, d, mlp, d}, K[4] = {d, d, d, mlp};
  size_t mx = 0;
  for (int g = 0; g < 4; ++g) {
    const size_t s = (size_t)trunk_split(N[g] / 128, K[g] / 64, nsm);
    mx += s * M * N[g];  // one partial buffer per slot: steps of different slots overlap in time
  }
  return mx;
}

size_t trunk_counter_bytes(int layers) {
  return 256 + (size_t)layers * (4 * kMaxTiles + kDepPerLayer) * sizeof(unsigned);
}

int trunk_plan(TrunkPlan* tp, int B, int T, int d, int mlp, int heads, int layers, const void* const w0[4],
               long long w_lstride_bytes, const float* const b0[4], long long b_lstride, float* x, __half* h,
               __half* qkv, __half* att, __half* u, __half* h2, float* part, void* counters, int* bump, int nsm,
               __half* hf, __half* pooled) {
  const int M = B * T;
  if (!trunk_supported(M, d, heads) || T > 96 || (mlp % 128) || (d % 128) || mlp / 128 > kMaxTiles ||
      3 * d / 128 > kMaxTiles || (w_lstride_bytes % 16)) {
    set_last_error("trunk_plan: unsupported shape M=%d d=%d mlp=%d heads=%d", M, d, mlp, heads);
    return -2;
  }
  memset(tp, 0, sizeof(*tp));
  TrunkArgs& a = tp->a;
  a.M = M;
  a.ntok = (M + 15) / 16 * 16;
  a.T = T;
  a.B = B;
  a.d = d;
  a.mlp = mlp;
  a.heads = heads;
  a.layers = layers;
  const int N[4] = {3 * d, d, mlp, d}, K[4] = {d, d, d, mlp};
  for (int g = 0; g < 4; ++g) {
    a.N[g] = N[g];
    a.K[g] = K[g];
    a.S[g] = trunk_split(N[g] / 128, K[g] / 64, nsm);
    a.units[g] = N[g] / 128 * a.S[g];
    a.bias[g] = b0[g];
    if (a.units[g] > nsm) {  // every unit needs its own CTA (one CTA per SM)
      set_last_error("trunk_plan: %d feature tiles exceed %d SMs", N[g] / 128, nsm);
      return -2;
    }
    a.R[g] = (M + a.S[g] - 1) / a.S[g];
  }
  a.bias_lstride = b_lstride;
  a.x_bytes = a.ntok * 128;
  a.stage_bytes = kWStageBytes + kKbPerStage * a.x_bytes;  // all sub-tiles multiples of 1 KB (SW128 atoms)
  tp->hd = d / heads;
  // aux: attention staging, or the S reduction slices of a QKV or fc1 unit
  size_t aux_bytes = attn16_smem_bytes(tp->hd);
  for (int g : {TG_QKV, TG_FC1}) aux_bytes = std::max(aux_bytes, (size_t)a.S[g] * a.R[g] * 512);
  const size_t budget = 227 * 1024 - 1024 - kBarRegion;
  if (aux_bytes + 2 * (size_t)a.stage_bytes > budget) {
    set_last_error("trunk_plan: shared memory too small for the weight ring");
    return -2;
  }
  int st = (int)((budget - aux_bytes) / a.stage_bytes);
  if (st > 8) st = 8;
  if (st < 2) {
    set_last_error("trunk_plan: shared memory too small for the weight ring");
    return -2;
  }
  a.stages = st;
  a.aux_off = st * a.stage_bytes;
  a.bar_off = (int)((a.aux_off + aux_bytes + 63) / 64 * 64);
  a.phases = 1;  // grid barriers per launch (the closing one)
  tp->smem = (size_t)a.bar_off + kBarRegion + 1024;
  a.x = x;
  a.h = h;
  a.qkv = qkv;
  a.att = att;
  a.u = u;
  a.part = part;
  uint8_t* c = static_cast<uint8_t*>(counters);
  a.grid_ctr = reinterpret_cast<unsigned long long*>(c);
  a.epoch = reinterpret_cast<unsigned*>(c + 64);
  a.tile_ctr = reinterpret_cast<unsigned*>(c + 256);
  a.tail_ctr = reinterpret_cast<unsigned*>(c + 128);
  a.dep = a.tile_ctr + (size_t)layers * 4 * kMaxTiles;
  a.h2 = h2;
  a.hf = hf;
  a.pooled = pooled;
  a.bump = bump;
  tp->grid = nsm;
  // tensor maps
  for (int g = 0; g < 4; ++g) {
    const uint64_t dims[4] = {64, (uint64_t)N[g], (uint64_t)(K[g] / 64), (uint64_t)layers};
    const uint64_t strides[3] = {128, (uint64_t)N[g] * 128, (uint64_t)w_lstride_bytes};
    const uint32_t box[4] = {64, 128, (uint32_t)kKbPerStage, 1};
    if (encode(&tp->maps.w[g], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, w0[g], dims, strides, box,
               CU_TENSOR_MAP_SWIZZLE_128B))
      return -3;
  }
  const __half* xin[4] = {h, att, h2, u};
  for (int g = 0; g < 4; ++g) {
    // [M][K] viewed as (64-wide k, row, k-block): one box = kKbPerStage k-block tiles of ntok rows
    const uint64_t dims[3] = {64, (uint64_t)M, (uint64_t)(K[g] / 64)};
    const uint64_t strides[2] = {(uint64_t)K[g] * 2, 128};
    const uint32_t box[3] = {64, (uint32_t)a.ntok, (uint32_t)kKbPerStage};
    if (encode(&tp->maps.x[g], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, xin[g], dims, strides, box,
               CU_TENSOR_MAP_SWIZZLE_128B))
      return -3;
  }
  float* part_g = part;
  for (int g = 0; g < 4; ++g) {
    // partials [S][N/128][M][128]: every unit's tile is one contiguous block
    // (row-strided [S][M][N] tiles stored ~3.5x slower for N = 6144)
    const uint64_t dims[4] = {128, (uint64_t)M, (uint64_t)(N[g] / 128), (uint64_t)a.S[g]};
    const uint64_t strides[3] = {512, (uint64_t)M * 512, (uint64_t)M * N[g] * 4};
    const uint32_t box[4] = {128, (uint32_t)a.R[g], 1, (uint32_t)a.S[g]};  // all S slices in one load
    if (encode(&tp->maps.p[g], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, part_g, dims, strides, box,
               CU_TENSOR_MAP_SWIZZLE_NONE))
      return -3;
    a.pslot[g] = part_g;
    part_g += (size_t)a.S[g] * M * N[g];  // matches trunk_part_floats
  }
  TrunkFn fn = trunk_kernel(tp->hd, d);
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tp->smem) != cudaSuccess) {
    set_last_error("trunk_plan: cannot reserve %zu bytes of shared memory", tp->smem);
    return -3;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kTrThreads, tp->smem) != cudaSuccess || per_sm < 1) {
    set_last_error("trunk_plan: the trunk kernel does not fit on an SM");
    return -3;
  }
  return 0;
}

bool trunk_set_tail(TrunkPlan* tp, const void* const w[3], const float* const b[3], const int N[3], const int K[3],
                    __half* hid16, __half* z, float* out, int out_hid) {
  TrunkArgs& a = tp->a;
  if (a.B != 1 || !a.pooled) return false;
  for (int i = 0; i < 3; ++i)
    if (K[i] % 256 || K[i] > 2048 || N[i] < 1 || (reinterpret_cast<uintptr_t>(w[i]) & 15)) return false;
  if (K[0] != a.d || K[1] != N[0] || K[2] != N[1]) return false;
  for (int i = 0; i < 3; ++i) {
    a.tw[i] = static_cast<const __half*>(w[i]);
    a.tb[i] = b[i];
    a.tN[i] = N[i];
    a.tK[i] = K[i];
  }
  a.hid16 = hid16;
  a.z = z;
  a.out = out;
  a.out_hid = out_hid;
  return true;
}

#ifdef CN_TRUNK_TRACE
// Profiling builds only: point the phase trace at a device buffer of
// layers x 8 x grid x 8 u64 (null turns it off).
extern "C" int cn_trunk_trace_set(void* dev_buf) {
  unsigned long long* p = static_cast<unsigned long long*>(dev_buf);
  return (int)cudaMemcpyToSymbol(g_trunk_trace, &p, sizeof(p));
}
// [layers][4][16][grid][8] u64 per GEMM stage: 0 weight tile landed, 1 activation tile landed (both as seen
// by the MMA thread), 2 MMAs issued, 3 weight load issued, 4 activation load issued
extern "C" int cn_trunk_strace_set(void* dev_buf) {
  unsigned long long* p = static_cast<unsigned long long*>(dev_buf);
  return (int)cudaMemcpyToSymbol(g_trunk_strace, &p, sizeof(p));
}
#endif

int trunk_launch(const TrunkPlan& tp, cudaStream_t s) {
  TrunkFn fn = trunk_kernel(tp.hd, tp.a.d);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tp.grid);
  cfg.blockDim = dim3(kTrThreads);
  cfg.dynamicSmemBytes = tp.smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return (int)cudaLaunchKernelEx(&cfg, fn, tp.maps, tp.a);
}

}  // namespace cn
