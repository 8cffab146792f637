// Persistent conv stem and token embeddings (one clip or a batch of clips).
//
// The conv stem of a frame (compile_modeld.py's vision encoder as restated in
// the synthetic layer list: per camera five 3x3 / stride-2 convs, each with a
// 1x1 conv, ReLU) plus the conditioning and token-embedding GEMMs are ~3.6
// GFLOP over ~42 MB of weights: microseconds of work, but eleven dependent
// GEMMs.  As separate launches each paid its launch, pipeline fill, an
// im2col pass through HBM and a split-K cluster exchange (~120 us in all).
// This kernel runs them as one cooperative launch of one CTA per SM:
//
//   warp 0 (lane 0)  streams the weight k-blocks of every unit this CTA will
//                    run, over all phases, into a ring of three 32 KB stages
//                    with TMA (one box of 1-8 k-blocks per stage; the weights
//                    never depend on the frame, so they are in flight while
//                    earlier phases compute); each CTA also requests its
//                    1/grid share of every phase's weights into L2 at launch.
//   warp 1 (lane 0)  issues tcgen05.mma (M = 128 rows, N = the tile's
//                    features, f32 accumulators in TMEM, units alternating
//                    between the two 256-column halves).
//   warps 2, 3       load the activation k-blocks into a 4-slot ring in the
//                    128-byte-swizzled layout the MMA reads: TMA boxes for
//                    row operands and for a 3x3 conv over 64-channel input
//                    (a strided box over the previous stage's NHWC output,
//                    the zero border as its out-of-bounds fill), else 16-byte
//                    cp.async gathers with zero-fill at the border.  No im2col
//                    matrix is written.
//   warps 4..7       epilogue from TMEM (lane quadrant = warp & 3).
//   warps 2..7       the split-K reduction.
//
// A phase is one GEMM cut into units (group, 128-row tile, feature tile,
// split).  Phases meet on dataflow counters: a unit's activation loads wait
// only for the phases it reads, and completions are published with release
// adds.  Split-K units store their partials ([feature][row], so a warp's
// stores are whole 128-byte lines), meet on a per-tile arrival counter, and
// then each reduces a band of 8-feature column groups: its slices of all S
// partials arrive by bulk copies into shared memory and are added in split
// order 0..S-1 (deterministic).  Stages of at most 256 channels fuse the 1x1
// conv into the 3x3 unit: the ReLU output goes to shared memory as the next
// MMA's operand and never leaves the SM.
//
// Decoupled phases (unsplit units whose epilogue stages only in the Y buffer:
// a fused operand of one k-block, an output of at most two 64-column boxes,
// or f32 / token rows) let the loads run ahead of the epilogue; warps 2..3
// and 4..7 then meet once per phase and publish once per phase, and a unit's
// fused 1x1 is issued after the next unit's 3x3 where both weight streams fit
// in the ring together.  Batched clips (tens of units per CTA and phase) live
// on this; other phases run unit by unit in lock-step.
//
// Every wait is bounded (%globaltimer); on timeout a code lands in the device
// error word and the roles unwind (named barriers are always reached by every
// warp of their group).  Counters are monotonic across launches (compared
// wrap-safe).  No TMA multicast.
#include <algorithm>

#include "cn_common.cuh"
#include "cn_gemm.cuh"
#include "cn_ops.cuh"
#include "cn_stem.cuh"

namespace cn {

namespace {

constexpr int kStThreads = 256;
constexpr int kStWStages = 3, kStWBytes = 32768;  // 32768 / (BN * 128) weight k-blocks per stage
constexpr int kStAStages = 4, kStABytes = 16384;  // one k-block of 128 activation rows
constexpr int kStYBytes = 36864;                  // fused 1x1 operand / output staging
constexpr int kStAOff = kStWStages * kStWBytes;
constexpr int kStYOff = kStAOff + kStAStages * kStABytes;
constexpr int kStBarOff = kStYOff + kStYBytes;
constexpr int kStRedBytes = kStBarOff - kStAOff;  // the activation ring and Y hold the reduction slices
constexpr int kStBiasOff = kStBarOff + 256;           // the unit's bias columns (f32 x 512)
constexpr int kStPhOff = kStBiasOff + 2048;           // the phase table
constexpr size_t kStSmem = (size_t)kStPhOff + sizeof(StemPhase) * kStemMaxPhases + 1024;
constexpr int kStMaxSplit = 18;
constexpr int kStMaxUnsplitKb = 40;
constexpr int kStBarRed = 1, kStBarEpi = 2;  // named barriers: warps 2..7, warps 4..7
constexpr int kStCompute = 192;

// (no memory clobber: ordering against the copies comes from the wait_group /
// fence / mbarrier steps, and a clobber would force every value the loop
// reads from memory to be reloaded per copy)
__device__ __forceinline__ void cp_async16_zfill(void* smem, const void* gmem, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// TMA tile store from shared memory (no multicast; never at a negative
// coordinate), and its bulk-group bookkeeping.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* smem_src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// every store issued so far has read its shared-memory source
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

// Wait until at most n (< 4) copy groups of this thread are in flight.
__device__ __forceinline__ void cp_async_wait_pending(int n) {
  switch (n) {
    case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
  }
}
// Weight k-blocks one ring stage holds for tiles n rows wide (n <= 256).
__host__ __device__ __forceinline__ int st_kps(int n) { return n <= 256 ? kStWBytes / (n * 128) : 1; }
__device__ __forceinline__ void cp_async_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Phase-trace instrumentation, compiled only with -DCN_STEM_TRACE (a
// profiling build): %globaltimer stamps per (phase, CTA, event) of the
// CTA's last unit of the phase; row kStemMaxPhases holds the launch start.
#ifdef CN_STEM_TRACE
__device__ unsigned long long* g_stem_trace = nullptr;
#define CN_ST(p, k)                                                                                   \
  do {                                                                                                \
    unsigned long long* tp_ = g_stem_trace;                                                           \
    if (tp_) tp_[(((size_t)(p)) * gridDim.x + blockIdx.x) * 16 + (k)] = global_ns();                 \
  } while (0)
// Per-unit stamps of CTA 0 (its first 32 units of each phase), after the
// per-CTA rows: [phase][unit ordinal][8 events].
#define CN_SU(p, P, u, k)                                                                              \
  do {                                                                                                \
    unsigned long long* tp_ = g_stem_trace;                                                           \
    const int j_ = ((u) - st_first(P)) / (int)gridDim.x;                                              \
    if (tp_ && blockIdx.x == 0 && j_ < 32)                                                            \
      tp_[(size_t)(kStemMaxPhases + 1) * gridDim.x * 16 + ((size_t)(p) * 32 + j_) * 8 + (k)] = global_ns(); \
  } while (0)
#else
#define CN_ST(p, k) \
  do {              \
  } while (0)
#define CN_SU(p, P, u, k) \
  do {                    \
  } while (0)
#endif

struct SUnit {
  int g, tm, tn, s, kb0, kb1;
};
__device__ __forceinline__ SUnit st_unit(const StemPhase& P, int u) {
  SUnit r;
  r.s = u % P.S;
  int t = u / P.S;
  r.tn = t % P.tn;
  t /= P.tn;
  r.tm = t % P.tm;
  r.g = t / P.tm;
  r.kb0 = r.s * P.KB / P.S;
  r.kb1 = (r.s + 1) * P.KB / P.S;
  return r;
}
// First unit of phase P that this CTA runs (unit u on CTA (cta0 + u) mod grid).
__device__ __forceinline__ int st_first(const StemPhase& P) {
  return (int)((blockIdx.x + gridDim.x - (unsigned)P.cta0 % gridDim.x) % gridDim.x);
}
// Column band [c0, c0 + cw) of a BN-wide tile that split s of S reduces
// (8-feature groups).
__device__ __forceinline__ void st_band(int BN, int S, int s, int* c0, int* cw) {
  const int ng = BN / 8;
  const int g0 = s * ng / S, g1 = (s + 1) * ng / S;
  *c0 = 8 * g0;
  *cw = 8 * (g1 - g0);
}

__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

// Epilogue fields of a phase, held in registers by the threads that store.
struct StEmit {
  int epi, N;
  void* out;
  long long ldo, o_gs;
  const float* pos;
  const float* cond;
  long long cond_ld;
  int rows_per_clip, tok_base, tok_gstride, T;
};

__device__ __forceinline__ StEmit st_emit_of(const StemPhase& P) {
  StEmit E;
  E.epi = P.epi;
  E.N = P.N;
  E.out = P.out;
  E.ldo = P.ldo;
  E.o_gs = P.o_gs;
  E.pos = P.pos;
  E.cond = P.cond;
  E.cond_ld = P.cond_ld;
  E.rows_per_clip = P.rows_per_clip;
  E.tok_base = P.tok_base;
  E.tok_gstride = P.tok_gstride;
  E.T = P.T;
  return E;
}

// Final value -> output for 8 consecutive features n..n+7 of row m of group
// g; bp: their bias (shared memory).
__device__ __forceinline__ void st_emit8(const StEmit& E, int g, int m, int n, const float (&v)[8], const float* bp) {
  float b[8];
  {
    const float4 b0 = *reinterpret_cast<const float4*>(bp), b1 = *reinterpret_cast<const float4*>(bp + 4);
    b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
    b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
  }
  if (E.epi == SE_RELU_F16) {
    __align__(16) __half h[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) h[j] = __float2half_rn(fmaxf(v[j] + b[j], 0.0f));
    *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(E.out) + (long long)g * E.o_gs + (long long)m * E.ldo + n) =
        *reinterpret_cast<const uint4*>(h);
  } else if (E.epi == SE_F32) {
    float* o = reinterpret_cast<float*>(E.out) + (long long)g * E.o_gs + (long long)m * E.ldo + n;
    reinterpret_cast<float4*>(o)[0] = make_float4(v[0] + b[0], v[1] + b[1], v[2] + b[2], v[3] + b[3]);
    reinterpret_cast<float4*>(o)[1] = make_float4(v[4] + b[4], v[5] + b[5], v[6] + b[6], v[7] + b[7]);
  } else {  // SE_TOKENS
    const int clip = m / E.rows_per_clip;
    const int t = E.tok_base + g * E.tok_gstride + m % E.rows_per_clip;
    const float* ps = E.pos + (long long)t * E.N + n;
    const float* cs = E.cond + (long long)clip * E.cond_ld + n;
    float* o = reinterpret_cast<float*>(E.out) + ((long long)clip * E.T + t) * E.ldo + n;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float4 p4 = ldg4(ps + 4 * h);
      const float4 c4 = __ldcg(reinterpret_cast<const float4*>(cs + 4 * h));  // written in this launch
      reinterpret_cast<float4*>(o)[h] =
          make_float4(((v[4 * h] + b[4 * h]) + p4.x) + c4.x, ((v[4 * h + 1] + b[4 * h + 1]) + p4.y) + c4.y,
                      ((v[4 * h + 2] + b[4 * h + 2]) + p4.z) + c4.z, ((v[4 * h + 3] + b[4 * h + 3]) + p4.w) + c4.w);
    }
  }
}

// 16 accumulator columns of this thread's row -> 16 f16 values (+ bias from
// shared memory, ReLU).
__device__ __forceinline__ void st_relu16(const uint32_t (&r)[16], const float* bias, __half (&h)[16]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 b = *reinterpret_cast<const float4*>(bias + 4 * q);
    h[4 * q + 0] = __float2half_rn(fmaxf(__uint_as_float(r[4 * q + 0]) + b.x, 0.0f));
    h[4 * q + 1] = __float2half_rn(fmaxf(__uint_as_float(r[4 * q + 1]) + b.y, 0.0f));
    h[4 * q + 2] = __float2half_rn(fmaxf(__uint_as_float(r[4 * q + 2]) + b.z, 0.0f));
    h[4 * q + 3] = __float2half_rn(fmaxf(__uint_as_float(r[4 * q + 3]) + b.w, 0.0f));
  }
}

__global__ void __launch_bounds__(kStThreads, 1)
    k_stem(const __grid_constant__ StemMaps maps, const __grid_constant__ StemArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStBarOff);
  uint64_t* fullW = bars;        // [kStWStages]
  uint64_t* emptyW = bars + 4;   // [kStWStages]
  uint64_t* fullA = bars + 8;    // [kStAStages], two arrivals per phase
  uint64_t* emptyA = bars + 12;  // [kStAStages]
  uint64_t* yready = bars + 17;  // fused 1x1 operand written
  uint64_t* redbar = bars + 18;  // reduction slices landed
  uint64_t* tfree = bars + 19;   // [2] accumulator half read out by the epilogue
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 21);
  volatile int* flags = reinterpret_cast<volatile int*>(bars + 22);
  // Per accumulator half, one phase per unit: the unit's GEMM MMAs complete
  // (doneA), its fused 1x1 MMAs complete (doneB; right after doneA when the
  // unit has none).  A half is reused only after the epilogue released it
  // (tfree), so neither barrier can run two phases ahead of its waiter.
  uint64_t* doneA = bars + 24;
  uint64_t* doneB = bars + 26;
  uint8_t* ringA = smem + kStAOff;
  uint8_t* Y = smem + kStYOff;
  float* sbias = reinterpret_cast<float*>(smem + kStBiasOff);  // [0, 256) the GEMM's, [256, 384) the fused 1x1's
  // The phase table lives in shared memory: read from the kernel parameters
  // inside loops with asm memory clobbers, every field would be reloaded
  // through the generic path on every iteration.
  StemPhase* sph = reinterpret_cast<StemPhase*>(smem + kStPhOff);
  {
    static_assert(sizeof(StemPhase) % 4 == 0, "phase table copied as words");
    const uint32_t* src = reinterpret_cast<const uint32_t*>(a.ph);
    uint32_t* dst = reinterpret_cast<uint32_t*>(sph);
    for (int i = threadIdx.x; i < (int)(sizeof(StemPhase) / 4) * a.nph; i += blockDim.x) dst[i] = src[i];
  }
  const float* red = reinterpret_cast<const float*>(smem + kStAOff);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStWStages; ++i) {
      mbar_init(&fullW[i], 1);
      mbar_init(&emptyW[i], 1);
    }
    for (int i = 0; i < kStAStages; ++i) {
      mbar_init(&fullA[i], 2);  // two arrivals: the producer warps (cp.async) or the TMA issuer twice
      mbar_init(&emptyA[i], 1);
    }
    mbar_init(&doneA[0], 1);
    mbar_init(&doneA[1], 1);
    mbar_init(&doneB[0], 1);
    mbar_init(&doneB[1], 1);
    mbar_init(yready, 1);
    mbar_init(redbar, 1);
    mbar_init(&tfree[0], 1);
    mbar_init(&tfree[1], 1);
    fence_barrier_init();
    for (int p = 0; p < a.nph; ++p) {
      tma_prefetch_desc(&maps.w[p]);
      if (a.ph[p].atma) tma_prefetch_desc(&maps.x[p]);
      if (a.ph[p].S == 1 && (a.ph[p].fuse || a.ph[p].epi == SE_RELU_F16)) tma_prefetch_desc(&maps.o[p]);
      if (a.ph[p].fuse) tma_prefetch_desc(&maps.w1[p]);  // (before the table copy is visible)
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const unsigned ep1 = *reinterpret_cast<volatile unsigned*>(a.epoch) + 1u;
  if (threadIdx.x == 0) CN_ST(kStemMaxPhases, 0);

  if (warp == 0) {
    // ------------------------------------------------ weight stream
    if (lane == 0) {
      // Once the ring's first fill is in flight, every later weight k-block
      // of this CTA is requested into L2 (the ring then reloads it from L2
      // whenever its phase comes).
      auto prefetch_rest = [&]() {
        // every CTA requests its 1/grid share of each phase's weights (units
        // of many row tiles share theirs, so a per-unit walk would repeat)
        for (int p = 0; p < a.nph; ++p) {
          const StemPhase& P = sph[p];
          for (int f = 0; f < (P.fuse ? 2 : 1); ++f) {
            const long long R = (long long)(f ? P.KB1 : P.KB) * P.N * 128;  // one group's k-blocked tensor
            const long long chunk = ((R + gridDim.x - 1) / gridDim.x + 255) / 256 * 256;
            const long long off = (long long)blockIdx.x * chunk;
            if (off >= R) continue;
            const uint32_t bytes = (uint32_t)(R - off < chunk ? R - off : chunk);
            for (int g = 0; g < P.G; ++g)
              bulk_prefetch_l2((f ? P.w1 + g * P.w1_gs : P.w + g * P.w_gs) + off, bytes);
          }
        }
      };
      uint32_t gw = 0;
      bool ok = true;
      for (int p = 0; p < a.nph && ok; ++p) {
        const StemPhase& P = sph[p];
        const int BN = P.BN, N = P.N, KB1 = P.fuse ? P.KB1 : 0, units = P.units;
        const int kps = P.kps, kps1 = P.kps1;
        const CUtensorMap* mw = &maps.w[p];
        const CUtensorMap* mw1 = &maps.w1[p];
        for (int u = st_first(P); u < units && ok; u += gridDim.x) {
          const SUnit U = st_unit(P, u);
          // one box of kps k-blocks per stage (past the unit's range it loads
          // the neighbour's k-blocks, or zeros past K: the MMA skips them)
          const int n3 = (U.kb1 - U.kb0 + kps - 1) / kps, n1 = KB1 ? (KB1 + kps1 - 1) / kps1 : 0;
          for (int i = 0; i < n3 + n1; ++i, ++gw) {
            const int st = (int)(gw % kStWStages);
            if (!mbar_wait(&emptyW[st], ((gw / kStWStages) & 1) ^ 1, 41)) {
              ok = false;
              break;
            }
            if (i == 0) CN_ST(p, 12);
            if (i < n3) {
              mbar_arrive_expect_tx(&fullW[st], (uint32_t)(BN * 128 * kps));
              tma_load_4d(smem + st * kStWBytes, mw, &fullW[st], 0, U.tn * BN, U.kb0 + i * kps, U.g);
            } else {
              mbar_arrive_expect_tx(&fullW[st], (uint32_t)(N * 128 * kps1));
              tma_load_4d(smem + st * kStWBytes, mw1, &fullW[st], 0, 0, (i - n3) * kps1, U.g);
            }
            if (gw + 1 == (uint32_t)kStWStages) prefetch_rest();
          }
        }
      }
      if (!ok || dev_error_set()) {
        // no TMA write may still be in flight into this CTA's shared memory when it exits
        for (uint32_t i = gw > (uint32_t)kStWStages ? gw - kStWStages : 0; i < gw; ++i)
          mbar_wait(&fullW[i % kStWStages], (i / kStWStages) & 1, 0, 100000000ull);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issue
    if (lane == 0) {
      // Units alternate between the two 256-column halves of TMEM; a unit
      // starts only once the epilogue has read out the unit before last.
      uint32_t gw = 0, ga = 0, ny = 0, lu = 0;
      bool ok = true;
      const uint32_t ring_a = smem_u32(ringA), ring_w = smem_u32(smem);
      for (int p = 0; p < a.nph && ok; ++p) {
        const StemPhase& P = sph[p];
        const int units = P.units, KB1 = P.fuse ? P.KB1 : 0;
        const int kps = P.kps, kps1 = P.kps1, wsub = P.BN * 128, wsub1 = P.N * 128;
        const uint32_t yop = P.dec ? smem_u32(Y) : ring_a;  // the fused 1x1's operand
        const uint32_t idesc = umma_idesc_f16(P.BN, false), idesc1 = umma_idesc_f16(P.N, false);
        const int n1 = KB1 ? (KB1 + kps1 - 1) / kps1 : 0;  // weight stages of a fused 1x1
        const bool defer = P.defer != 0;
        // The fused 1x1 of a unit into accumulator acc, its weight stages
        // from ring index g1 on, once the epilogue has written its operand.
        auto issue_1x1 = [&](uint32_t acc, uint32_t g1) -> bool {
          if (!mbar_wait(yready, ny & 1, 44)) return false;
          ++ny;
          tc_fence_after();
          for (int kb = 0, sub = 0; kb < KB1; ++kb) {
            const int sw = (int)(g1 % kStWStages);
            if (sub == 0 && !mbar_wait(&fullW[sw], (g1 / kStWStages) & 1, 45)) return false;
            tc_fence_after();
            const uint32_t ya = yop + kb * kStABytes, wa = ring_w + sw * kStWBytes + sub * wsub1;
#pragma unroll
            for (int k = 0; k < 4; ++k)
              tc_mma_f16(acc, umma_desc_sw128(ya + 32 * k, 16, 1024), umma_desc_sw128(wa + 32 * k, 16, 1024), idesc1,
                         (kb > 0 || k > 0) ? 1u : 0u);
            if (++sub == kps1 || kb + 1 == KB1) {
              tc_commit(&emptyW[sw]);
              ++g1;
              sub = 0;
            }
          }
          return true;
        };
        bool pend1 = false;  // deferred: a unit whose 1x1 is still to be issued
        uint32_t pacc = 0, pg1 = 0, plu = 0;
        for (int u = st_first(P); u < units && ok; u += gridDim.x, ++lu) {
          const SUnit U = st_unit(P, u);
          const uint32_t acc = tmem + 256u * (lu & 1);
          if (lu >= 2) {
            if (!mbar_wait(&tfree[lu & 1], ((lu >> 1) - 1) & 1, 40)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          for (int kb = U.kb0, sub = 0; kb < U.kb1; ++kb, ++ga) {
            const int sw = (int)(gw % kStWStages), sa = (int)(ga % kStAStages);
            if ((sub == 0 && !mbar_wait(&fullW[sw], (gw / kStWStages) & 1, 42)) ||
                !mbar_wait(&fullA[sa], (ga / kStAStages) & 1, 43)) {
              ok = false;
              break;
            }
            if (kb == U.kb0) {
              CN_ST(p, 5);
              CN_SU(p, P, u, 2);
            }
            tc_fence_after();
            const uint32_t aa = ring_a + sa * kStABytes, wa = ring_w + sw * kStWBytes + sub * wsub;
#pragma unroll
            for (int k = 0; k < 4; ++k)
              tc_mma_f16(acc, umma_desc_sw128(aa + 32 * k, 16, 1024), umma_desc_sw128(wa + 32 * k, 16, 1024), idesc,
                         (kb > U.kb0 || k > 0) ? 1u : 0u);
            tc_commit(&emptyA[sa]);
            if (++sub == kps || kb + 1 == U.kb1) {
              tc_commit(&emptyW[sw]);
              ++gw;
              sub = 0;
            }
          }
          if (!ok) break;
          tc_commit(&doneA[lu & 1]);
          CN_ST(p, 6);
          CN_SU(p, P, u, 3);
          if (!KB1) {
            tc_commit(&doneB[lu & 1]);
          } else if (!defer) {
            if (!issue_1x1(acc, gw)) {
              ok = false;
              break;
            }
            gw += n1;
            tc_commit(&doneB[lu & 1]);
          } else {
            // this unit's 1x1 waits for its operand while the next unit's
            // GEMM is issued; the previous unit's 1x1 goes now
            const uint32_t g1 = gw;
            gw += n1;
            if (pend1) {
              if (!issue_1x1(pacc, pg1)) {
                ok = false;
                break;
              }
              tc_commit(&doneB[plu & 1]);
            }
            pend1 = true;
            pacc = acc;
            pg1 = g1;
            plu = lu;
          }
        }
        if (ok && pend1) {
          if (issue_1x1(pacc, pg1))
            tc_commit(&doneB[plu & 1]);
          else
            ok = false;
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------ activations, epilogue, reduction (warps 2..7)
    // Every phase field a loop uses is held in a register: the phase table is
    // in shared memory, which any global store could alias.
    const int ct = threadIdx.x - 64;
    uint32_t ga = 0, nred = 0, lu = 0;
    int bkey = -1;  // (phase, group, feature tile) whose bias columns are in sbias
    // Decoupled units check the device error word once per unit; it is read
    // one unit ahead, so the load's latency is hidden behind the unit's work.
    int err_ahead = 0;
    bool ok = true;  // uniform over warps 2..7 (set from one verdict per unit)
    for (int p = 0; p < a.nph && ok; ++p) {
      const StemPhase& P = sph[p];
      const int units = P.units, S = P.S, BN = P.BN, N = P.N, Mg = P.Mg, rows_pad = P.rows_pad;
      const int fuse = P.fuse, KB1 = P.KB1, epi = P.epi, dep0 = P.dep0, dep1 = P.dep1, dec = P.dec;
      // the epilogue's staging: Y for decoupled units (the fused operand
      // first, then the output), else the activation ring
      uint8_t* const yop = dec ? Y : ringA;
      uint8_t* const ystg = dec ? Y + (fuse ? kStABytes : 0) : ringA;
      uint32_t pend = 0;  // decoupled: units done but not yet published
      bool deps = false, edeps = false;
      for (int u = st_first(P); u < units && ok; u += gridDim.x, ++lu) {
        const SUnit U = st_unit(P, u);
        bool live = true;  // this thread's part of the unit proceeds (waits may expire)
        if (warp < 4) {
          // decoupled: the loads run ahead of the epilogue and stop at a
          // recorded error on their own (warp-uniform)
          if (dec) {
            if (__shfl_sync(0xffffffffu, err_ahead, 0)) break;
            if (lane == 0) err_ahead = *reinterpret_cast<volatile int*>(&g_cn_dev_error);
          }
          // ---------------- activation k-blocks: chunk i = (row i / 8, 16-byte column i % 8)
          if (!deps) {
            int met = 1;
            if (threadIdx.x == 64) CN_ST(p, 0);
            if (lane == 0) {
              if (dep0 >= 0) met = spin_until(a.pctr + dep0, (unsigned)sph[dep0].units * ep1, 46, ld_acquire_u32);
              if (met && dep1 >= 0) met = spin_until(a.pctr + dep1, (unsigned)sph[dep1].units * ep1, 46, ld_acquire_u32);
              fence_acq_rel_gpu();
              fence_proxy_async_global();  // TMA reads what other CTAs stored
            }
            live = __shfl_sync(0xffffffffu, met, 0) != 0;
            deps = live;
            if (threadIdx.x == 64) CN_ST(p, 1);
          }
          if (P.atma) {
            // ---- one TMA box per k-block, issued by warp 2 lane 0
            const int nkb = U.kb1 - U.kb0;
            if (warp == 2 && lane == 0 && live) {
              const CUtensorMap* mx = &maps.x[p];
              const uint32_t abytes = (uint32_t)P.abytes;
              const bool gth = P.akind == SA_GATHER;
              const int lCin = P.lCin, lWo = P.lWo, lHo = P.lHo;
              const int m0 = U.tm * 128;
              const int img = U.g * P.B + (m0 >> (lWo + lHo)), oy0 = (m0 >> lWo) & ((1 << lHo) - 1);
              for (int i = 0; i < nkb; ++i) {
                const uint32_t gi = ga + i;
                const int sa = (int)(gi % kStAStages);
                if (!mbar_wait(&emptyA[sa], ((gi / kStAStages) & 1) ^ 1, 47)) {
                  live = false;
                  break;
                }
                if (i == 0) {
                  CN_ST(p, 14);
                  CN_SU(p, P, u, 0);
                }
                const int k = (U.kb0 + i) * 64;
                mbar_arrive_expect_tx(&fullA[sa], abytes);
                mbar_arrive(&fullA[sa]);
                if (gth) {
                  const int tap = k >> lCin, c0 = k & ((1 << lCin) - 1);
                  const int ky = tap / 3, kx = tap - 3 * ky;
                  tma_load_4d(ringA + sa * kStABytes, mx, &fullA[sa], c0, kx - 1, 2 * oy0 + ky - 1, img);
                } else {
                  tma_load_3d(ringA + sa * kStABytes, mx, &fullA[sa], k, m0, U.g);
                }
              }
              CN_ST(p, 2);
              CN_SU(p, P, u, 1);
            }
            ga += nkb;
            __syncwarp();
          } else {
          // Thread ct copies column j = ct % 8 of rows ct / 8 + 8 q (q < 16) of
          // every k-block; the row-dependent part of the addressing is
          // computed once per unit: SA_ROWS the row index, SA_GATHER the
          // image and the top-left input pixel of the 3x3 window (packed
          // b << 20 | (2 oy) << 10 | 2 ox, all-ones for rows past Mg).
          const int j = ct & 7;
          const __half* gA = P.A + (long long)U.g * P.a_gs;  // any valid address serves when nothing is read
          const bool gather = P.akind == SA_GATHER;
          const int aK = P.K, aHin = P.Hin, aWin = P.Win;
          const int lHin = P.lHin, lWin = P.lWin, lCin = P.lCin, lHo = P.lHo, lWo = P.lWo;
          const long long alda = P.lda;
          uint32_t rinfo[16];
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const int m = U.tm * 128 + (ct >> 3) + 8 * q;
            if (m >= Mg) {
              rinfo[q] = 0xffffffffu;
            } else if (!gather) {
              rinfo[q] = (uint32_t)m;
            } else {
              const int ox = m & ((1 << lWo) - 1), oy = (m >> lWo) & ((1 << lHo) - 1), b = m >> (lWo + lHo);
              rinfo[q] = ((uint32_t)b << 20) | ((uint32_t)(2 * oy) << 10) | (uint32_t)(2 * ox);
            }
          }
          if (threadIdx.x == 64) CN_ST(p, 4);
          // Issue and announce are decoupled: k-blocks are issued into free
          // slots (up to kStAStages in flight) and each one is announced
          // (copies landed, fence, one arrival per warp) as soon as its own
          // copies have landed, so the MMAs never wait for later issues.
          const int nkb = U.kb1 - U.kb0;
          int issued = 0, announced = 0;
          while (live && announced < nkb) {
            // issue into every slot that is free now
            while (issued < nkb && issued - announced < kStAStages) {
              const uint32_t gi = ga + issued;
              const int sa = (int)(gi % kStAStages);
              const uint32_t par = ((gi / kStAStages) & 1) ^ 1;
              int free_now = 1;
              if (lane == 0) free_now = mbar_try_wait(&emptyA[sa], par) ? 1 : 0;
              free_now = __shfl_sync(0xffffffffu, free_now, 0);
              if (!free_now) {
                if (issued > announced) break;  // announce what is in flight first
                if (!__all_sync(0xffffffffu, mbar_wait(&emptyA[sa], par, 47))) {
                  live = false;
                  break;
                }
              }
              const int kb = U.kb0 + issued;
              if (kb == U.kb0 && threadIdx.x == 64) {
                CN_ST(p, 14);
                CN_SU(p, P, u, 0);
              }
              uint8_t* dst = ringA + sa * kStABytes;
              const int k = kb * 64 + j * 8;
              const bool kin = k < aK;
              if (gather) {
                const int tap = k >> lCin;
                const int c = k & ((1 << lCin) - 1);
                const int ky = tap / 3 - 1, kx = tap - 3 * (tap / 3) - 1;
                const __half* gk = gA + c;
#pragma unroll
                for (int q = 0; q < 16; ++q) {
                  const int row = (ct >> 3) + 8 * q;
                  const uint32_t ri = rinfo[q];
                  const int y = (int)((ri >> 10) & 1023) + ky, x = (int)(ri & 1023) + kx, b = (int)(ri >> 20);
                  const bool v = kin && ri != 0xffffffffu && (unsigned)y < (unsigned)aHin && (unsigned)x < (unsigned)aWin;
                  const long long pix = ((long long)((b << lHin) + y) << lWin) + x;
                  const __half* src = v ? gk + (pix << lCin) : gA;
                  cp_async16_zfill(dst + row * 128 + ((j ^ (row & 7)) << 4), src, v ? 16u : 0u);
                }
              } else {
                const __half* gk = gA + k;
#pragma unroll
                for (int q = 0; q < 16; ++q) {
                  const int row = (ct >> 3) + 8 * q;
                  const uint32_t ri = rinfo[q];
                  const bool v = kin && ri != 0xffffffffu;
                  const __half* src = v ? gk + (long long)ri * alda : gA;
                  cp_async16_zfill(dst + row * 128 + ((j ^ (row & 7)) << 4), src, v ? 16u : 0u);
                }
              }
              cp_async_commit();
              if (kb == U.kb0 && threadIdx.x == 64) CN_ST(p, 13);
              ++issued;
            }
            if (!live || issued == announced) continue;
            // the oldest k-block in flight: wait for its copies only (one
            // arrival per producer warp)
            cp_async_wait_pending(issued - announced - 1);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&fullA[(ga + announced) % kStAStages]);
            ++announced;
          }
          if (threadIdx.x == 64) {
            CN_ST(p, 2);
            CN_SU(p, P, u, 1);
          }
          cp_async_wait0();
          ga += nkb;
          }
          if (threadIdx.x == 64) CN_ST(p, 3);
          __syncwarp();
        } else {
          // ---------------- epilogue: TMEM lane quadrant q, one accumulator row per thread
          const int q = warp & 3, row = 32 * q + lane;
          const int rv = min(128, Mg - U.tm * 128);  // valid rows of the tile
          const uint32_t taddr = tmem + 256u * (lu & 1) + ((uint32_t)(32 * q) << 16);
          {
            // this unit's bias columns into shared memory while the MMAs run
            // (the previous unit's readers are past its last barrier); units
            // of the same group and feature tile keep what is there
            const int t = threadIdx.x - 128;
            const int key = ((p * 2 + U.g) << 8) + U.tn;
            if (key != bkey) {
              bkey = key;
              const float* b0 = P.bias + (long long)U.g * P.b_gs + U.tn * BN;
              for (int i = t; i < BN; i += 128) sbias[i] = __ldg(b0 + i);
              if (fuse) {
                const float* b1 = P.bias1 + (long long)U.g * P.b1_gs;
                for (int i = t; i < N; i += 128) sbias[256 + i] = __ldg(b1 + i);
              }
            }
            if (dec && threadIdx.x == 128) {
              flags[0] = err_ahead != 0 ? 1 : 0;
              err_ahead = *reinterpret_cast<volatile int*>(&g_cn_dev_error);
            }
            named_sync(kStBarEpi, 128);
            if (threadIdx.x == 128) {
              CN_ST(p, 15);
              CN_SU(p, P, u, 5);
            }
          }
          // decoupled: the epilogue stops at a recorded error on its own
          // (uniform over its four warps: the flag was set before the barrier)
          if (dec && flags[0]) break;
          const uint32_t hpar = (lu >> 1) & 1;  // this unit's phase of its half's barriers
          live = __all_sync(0xffffffffu, mbar_wait(&doneA[lu & 1], hpar, 48));  // warp-uniform: tcgen05.ld is .aligned
          if (threadIdx.x == 128) {
            CN_ST(p, 7);
            CN_SU(p, P, u, 4);
          }
          tc_fence_after();
          if (S == 1) {
            const int nout = fuse ? N : BN;
            if (fuse) {
              // 3x3 output (ReLU, f16) -> the 1x1 conv's operand in the
              // activation ring (idle once the 3x3 MMAs are done; the next
              // unit's loads wait for this unit's closing verdict), swizzled
              // k-blocks, columns past N in the last k-block zero.  The 1x1
              // then accumulates into the same TMEM columns.
              if (live) {
                for (int c0 = 0; c0 < N; c0 += 16) {
                  uint32_t r[16];
                  tmem_ld16(taddr + c0, r);
                  tmem_ld_wait();
                  __align__(16) __half h[16];
                  st_relu16(r, sbias + c0, h);
#pragma unroll
                  for (int hh = 0; hh < 2; ++hh) {
                    const int c = c0 + 8 * hh, kb = c >> 6, jc = (c & 63) >> 3;
                    *reinterpret_cast<uint4*>(yop + kb * kStABytes + row * 128 + ((jc ^ (row & 7)) << 4)) =
                        *reinterpret_cast<const uint4*>(h + 8 * hh);
                  }
                }
                for (int c = N; c < KB1 * 64; c += 8) {
                  const int kb = c >> 6, jc = (c & 63) >> 3;
                  *reinterpret_cast<uint4*>(yop + kb * kStABytes + row * 128 + ((jc ^ (row & 7)) << 4)) =
                      make_uint4(0, 0, 0, 0);
                }
              }
              fence_proxy_async_smem();
              tc_fence_before();
              named_sync(kStBarEpi, 128);
              if (threadIdx.x == 128) mbar_arrive(yready);
              live = __all_sync(0xffffffffu, mbar_wait(&doneB[lu & 1], hpar, 49)) && live;
              if (threadIdx.x == 128) {
                CN_ST(p, 8);
                CN_SU(p, P, u, 6);
              }
              tc_fence_after();
            }
            // final accumulator -> output
            const uint32_t acc = taddr;  // the fused 1x1 accumulates into the 3x3's columns
            const float* bias = fuse ? sbias + 256 : sbias;
            if (epi == SE_RELU_F16 || fuse) {
              // rows -> the activation ring as swizzled 64-column tiles (the
              // TMA layout), then one thread stores them with TMA, waits for
              // the writes and publishes (no copy loop, no proxy fence)
              if (live)
                for (int c0 = 0; c0 < nout; c0 += 16) {
                  uint32_t r[16];
                  tmem_ld16(acc + c0, r);
                  tmem_ld_wait();
                  __align__(16) __half h[16];
                  st_relu16(r, bias + c0, h);
#pragma unroll
                  for (int hh = 0; hh < 2; ++hh) {
                    const int c = c0 + 8 * hh, kb = c >> 6, jc = (c & 63) >> 3;
                    *reinterpret_cast<uint4*>(ystg + kb * kStABytes + row * 128 + ((jc ^ (row & 7)) << 4)) =
                        *reinterpret_cast<const uint4*>(h + 8 * hh);
                  }
                }
              fence_proxy_async_smem();
              tc_fence_before();
              named_sync(kStBarEpi, 128);
              if (threadIdx.x == 128) {
                mbar_arrive(&tfree[lu & 1]);
                if (live) {
                  const int col0 = fuse ? 0 : U.tn * BN;
                  for (int kb = 0; kb * 64 < nout; ++kb)
                    tma_store_3d(&maps.o[p], ystg + kb * kStABytes, col0 + kb * 64, U.tm * 128, U.g);
                  bulk_commit();
                }
                if (dec) {
                  // Y is free again once the store has read it; the rows are
                  // published with the CTA's other units of the phase at its
                  // end (the next phases wait for all units anyway)
                  bulk_wait_read_all();
                  ++pend;
                } else {
                  if (live) {
                    bulk_wait_all();
                    fence_proxy_async_global();
                  }
                  red_release_add(a.pctr + p, 1u);
                }
                CN_ST(p, 11);
                CN_SU(p, P, u, 7);
              }
            } else {
              // f32 / token tiles (at most 64 features wide): the warps
              // holding valid rows stage the accumulators in Y ([row][BN + 4]
              // f32), then all four warps emit 8-feature groups
              float* sacc = reinterpret_cast<float*>(Y);
              const int ld = BN + 4;
              if (live && 32 * q < rv)
                for (int c0 = 0; c0 < BN; c0 += 16) {
                  uint32_t r[16];
                  tmem_ld16(acc + c0, r);
                  tmem_ld_wait();
#pragma unroll
                  for (int h4 = 0; h4 < 4; ++h4)
                    *reinterpret_cast<float4*>(sacc + row * ld + c0 + 4 * h4) =
                        make_float4(__uint_as_float(r[4 * h4]), __uint_as_float(r[4 * h4 + 1]),
                                    __uint_as_float(r[4 * h4 + 2]), __uint_as_float(r[4 * h4 + 3]));
                }
              tc_fence_before();
              if (threadIdx.x == 128) {
                // token tiles read the cond vector of this launch (waited
                // for once per phase)
                int met = 1;
                if (!edeps) {
                  if (dep0 >= 0) met = spin_until(a.pctr + dep0, (unsigned)sph[dep0].units * ep1, 52, ld_acquire_u32);
                  if (met && dep1 >= 0)
                    met = spin_until(a.pctr + dep1, (unsigned)sph[dep1].units * ep1, 52, ld_acquire_u32);
                  fence_acq_rel_gpu();
                  edeps = met != 0;
                }
                flags[2] = met;
              }
              named_sync(kStBarEpi, 128);
              if (threadIdx.x == 128) mbar_arrive(&tfree[lu & 1]);
              const StEmit E = st_emit_of(P);
              const int ncg = BN / 8;
              if (live && flags[2])
                for (int i = threadIdx.x - 128; i < rv * ncg; i += 128) {
                  const int rr = i / ncg, cg = i % ncg;
                  float v[8];
                  const float4 v0 = *reinterpret_cast<const float4*>(sacc + rr * ld + 8 * cg);
                  const float4 v1 = *reinterpret_cast<const float4*>(sacc + rr * ld + 8 * cg + 4);
                  v[0] = v0.x; v[1] = v0.y; v[2] = v0.z; v[3] = v0.w;
                  v[4] = v1.x; v[5] = v1.y; v[6] = v1.z; v[7] = v1.w;
                  st_emit8(E, U.g, U.tm * 128 + rr, U.tn * BN + 8 * cg, v, sbias + 8 * cg);
                }
            }
            if (epi != SE_RELU_F16 && !fuse) {
              fence_proxy_async_global();  // the next phases read these rows by TMA
              named_sync(kStBarEpi, 128);
              if (threadIdx.x == 128) {
                if (dec)
                  ++pend;
                else
                  red_release_add(a.pctr + p, 1u);
                CN_ST(p, 11);
              }
            }
          } else {
            // partial tile [BN][rows_pad] -> global (lane = row: whole 128-byte lines per store)
            const long long tile = (long long)((U.g * P.tm + U.tm) * P.tn + U.tn);
            float* pt = P.part + (tile * S + U.s) * BN * rows_pad;
            if (live && 32 * q < rows_pad) {
              float* pr = pt + row;
              for (int c0 = 0; c0 < BN; c0 += 32) {
                uint32_t r[2][16];
#pragma unroll
                for (int h4 = 0; h4 < 2; ++h4) tmem_ld16(taddr + c0 + 16 * h4, r[h4]);
                tmem_ld_wait();
#pragma unroll
                for (int h4 = 0; h4 < 2; ++h4)
#pragma unroll
                  for (int jv = 0; jv < 16; ++jv) pr[(long long)(c0 + 16 * h4 + jv) * rows_pad] = __uint_as_float(r[h4][jv]);
              }
            }
            tc_fence_before();
            fence_proxy_async_global();  // the reducers read the partials with bulk copies
            named_sync(kStBarEpi, 128);
            if (threadIdx.x == 128) {
              mbar_arrive(&tfree[lu & 1]);
              CN_ST(p, 8);
              unsigned* ctr = a.tctr + p * kStemMaxTiles + tile;
              red_release_add(ctr, 1u);
              const bool met = live && spin_until(ctr, (unsigned)S * ep1, 50, ld_acquire_u32);
              fence_acq_rel_gpu();
              fence_proxy_async_global();
              CN_ST(p, 9);
              int c0, cw;
              st_band(BN, S, U.s, &c0, &cw);
              flags[1] = met ? 1 : 0;
              if (met && cw > 0) {
                const uint32_t bytes = (uint32_t)cw * rows_pad * 4;
                const float* tp = pt - (long long)U.s * BN * rows_pad;
                mbar_arrive_expect_tx(redbar, bytes * (uint32_t)S);
                for (int s2 = 0; s2 < S; ++s2)
                  bulk_g2s(smem_u32(smem + kStAOff) + s2 * bytes, tp + ((long long)s2 * BN + c0) * rows_pad, bytes,
                           smem_u32(redbar));
              }
            }
          }
        }
        if (S > 1) {
          // ---------------- split-K reduction of this unit's column band (warps 2..7)
          named_sync(kStBarRed, kStCompute);
          int c0, cw;
          st_band(BN, S, U.s, &c0, &cw);
          bool landed = false;
          if (flags[1] && cw > 0) {
            landed = mbar_wait(redbar, nred & 1, 51);
            ++nred;
          }
          if (threadIdx.x == 64) CN_ST(p, 10);
          if (landed) {
            const StEmit E = st_emit_of(P);
            const int rv = min(128, Mg - U.tm * 128), ncg = cw / 8, rp = rows_pad;
            for (int i = ct; i < rv * ncg; i += kStCompute) {
              const int r = i % rv, cg = i / rv;
              float v[8];
#pragma unroll
              for (int jv = 0; jv < 8; ++jv) v[jv] = red[(cg * 8 + jv) * rp + r];
              for (int s2 = 1; s2 < S; ++s2) {
                const float* sl = red + ((long long)s2 * cw + cg * 8) * rp + r;
#pragma unroll
                for (int jv = 0; jv < 8; ++jv) v[jv] += sl[jv * rp];
              }
              st_emit8(E, U.g, U.tm * 128 + r, U.tn * BN + c0 + 8 * cg, v, sbias + c0 + 8 * cg);
            }
          }
          fence_proxy_async_global();  // the next phases read these rows by TMA
          named_sync(kStBarRed, kStCompute);
          if (threadIdx.x == 64) {
            red_release_add(a.pctr + p, 1u);
            CN_ST(p, 11);
          }
        }
        (void)live;
        if (dec) continue;
        // one uniform verdict per unit for warps 2..7
        named_sync(kStBarRed, kStCompute);
        if (threadIdx.x == 64) flags[3] = !dev_error_set();
        named_sync(kStBarRed, kStCompute);
        ok = flags[3] != 0;
      }
      if (dec) {
        // publish the last unit's rows; before a phase whose units may stage
        // in the activation ring, one uniform verdict for warps 2..7 (that
        // phase's loads start after it)
        if (threadIdx.x == 128 && pend) {
          bulk_wait_all();  // (no stores in flight for f32 / token phases)
          fence_proxy_async_global();
          red_release_add(a.pctr + p, pend);
          pend = 0;
        }
        if (p + 1 < a.nph && !sph[p + 1].dec) {
          named_sync(kStBarRed, kStCompute);
          if (threadIdx.x == 64) flags[3] = !dev_error_set();
          named_sync(kStBarRed, kStCompute);
          ok = flags[3] != 0;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
  if (threadIdx.x == 0) {
    // the last CTA out advances the epoch: every CTA read it before counting itself out
    const unsigned prev = atomicAdd(a.exits, 1u);
    if (prev == gridDim.x * ep1 - 1u) atomicAdd(a.epoch, 1u);
  }
}

}  // namespace

size_t stem_counter_bytes() { return 256 + (size_t)kStemMaxPhases * (1 + kStemMaxTiles) * sizeof(unsigned); }

static bool pow2(int v) { return v > 0 && (v & (v - 1)) == 0; }

// Tiled f16 tensor map with traversal strides (128-byte swizzle, zero fill).
static int encode_strided(CUtensorMap* map, int rank, const void* base, const uint64_t* dims,
                          const uint64_t* strides_bytes, const uint32_t* box, const uint32_t* estr) {
  if (get_encoder()) {
    set_last_error("cuTensorMapEncodeTiled entry point unavailable");
    return -1;
  }
  cuuint64_t d[5];
  cuuint64_t st[4];
  cuuint32_t b[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = estr[i];
    if (i + 1 < rank) st[i] = strides_bytes[i];
  }
  const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, (cuuint32_t)rank, const_cast<void*>(base), d, st, b,
                              es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("cuTensorMapEncodeTiled (strided) failed (%d)", (int)r);
    return (int)r;
  }
  return 0;
}
static int ilog2(int v) {
  int l = 0;
  while (v > 1) {
    v >>= 1;
    ++l;
  }
  return l;
}

void stem_plan_begin(StemPlan* sp, int nsm) {
  memset(sp, 0, sizeof(*sp));
  sp->grid = nsm;
  sp->smem = kStSmem;
}

int stem_add(StemPlan* sp, const StemSpec& s) {
  StemArgs& a = sp->a;
  if (a.nph >= kStemMaxPhases) {
    set_last_error("stem_add: more than %d phases", kStemMaxPhases);
    return -1;
  }
  const bool fuse = s.W1 != nullptr;
  StemPhase P;
  memset(&P, 0, sizeof(P));
  P.G = s.G;
  P.Mg = s.Mg;
  P.N = s.N;
  P.K = s.K;
  P.KB = (s.K + 63) / 64;
  // Tiling: a unit of at most kStMaxUnsplitKb k-blocks runs whole (a split
  // costs a partial store, an arrival, a reduction and a second publish,
  // ~7 us, more than the MMAs it saves); tiles of a few rows are 64 wide,
  // so that more CTAs share the epilogue.
  const int KB = (s.K + 63) / 64;
  const bool split = !fuse && KB > kStMaxUnsplitKb;
  // f32 / token epilogues stage a whole tile in Y ([rows][BN + 4] f32): a
  // full 128-row tile is 64 features wide.
  if (fuse)
    P.BN = s.N;
  else if (!split)
    P.BN = std::min(s.N, s.Mg >= 128 && s.epi == SE_RELU_F16 ? 128 : 64);
  else
    P.BN = s.Mg >= 128 ? std::min(s.N, 128) : std::min(s.N, 256);
  P.tm = (s.Mg + 127) / 128;
  P.tn = s.N / P.BN;
  P.rows_pad = s.Mg >= 128 ? 128 : (s.Mg + 31) / 32 * 32;
  const int tiles = s.G * P.tm * P.tn;
  auto red_bytes = [&](int S) { return (long long)S * 8 * ((P.BN / 8 + S - 1) / S) * P.rows_pad * 4; };
  int S = 1;
  if (split) {
    S = std::min(std::min(P.KB, kStMaxSplit), std::max(1, sp->grid / tiles));
    while (S > 1 && red_bytes(S) > kStRedBytes) --S;
  }
  P.S = S;
  const bool ok_shape = s.G >= 1 && s.Mg >= 1 && s.N % 16 == 0 && s.N % P.BN == 0 && P.BN >= 16 && P.BN <= 256 &&
                        s.K % 8 == 0 && (s.akind == SA_ROWS || (s.akind == SA_GATHER && s.Cin % 8 == 0)) &&
                        (!fuse || (s.N <= 256 && s.epi == SE_RELU_F16)) &&
                        (S > 1 || s.epi != SE_RELU_F16 || ((fuse ? s.N : P.BN) + 63) / 64 <= kStAStages) &&
                        (S > 1 || fuse || s.epi == SE_RELU_F16 || P.rows_pad * (P.BN + 4) * 4 <= kStYBytes) &&
                        (s.akind != SA_GATHER || (pow2(s.Hin) && pow2(s.Win) && pow2(s.Cin) && s.Cin >= 8)) &&
                        (S == 1 || (tiles <= kStemMaxTiles && red_bytes(S) <= kStRedBytes)) &&
                        (s.G == 1 || (s.w_gs > 0 && s.w_gs % 16 == 0)) &&
                        (!fuse || s.G == 1 || (s.w1_gs > 0 && s.w1_gs % 16 == 0));
  if (!ok_shape) {
    set_last_error("stem_add: unsupported phase G=%d Mg=%d N=%d K=%d BN=%d S=%d", s.G, s.Mg, s.N, s.K, P.BN, S);
    return -1;
  }
  P.units = tiles * S;
  // A ring stage holds one weight box of up to 32 KB, but no more k-blocks
  // than the GEMM has (a short GEMM's box would be mostly zero fill).
  P.kps = std::min(st_kps(P.BN), P.KB);
  P.kps1 = fuse ? std::min(st_kps(s.N), (s.N + 63) / 64) : P.kps;
  // Decoupled units: the epilogue stages the fused operand and the output in
  // Y, off the activation ring, so the loads of the next units need not wait
  // for it (a split's reduction and a wide fused operand use the ring).
  P.dec = (S == 1 && (fuse ? s.N <= 64 : (s.epi != SE_RELU_F16 || P.BN <= 128))) ? 1 : 0;
  // Deferred fused 1x1 (decoupled units only: the next unit's loads must not
  // wait for this unit's epilogue): the MMA thread issues unit u + 1's GEMM
  // before unit u's 1x1, consuming weight stages out of order, which needs
  // both of a unit's weight streams in the ring at once.
  {
    const int KB1 = (s.N + 63) / 64;
    const int n3 = (P.KB + P.kps - 1) / P.kps, n1 = (KB1 + P.kps1 - 1) / P.kps1;
    P.defer = (P.dec && fuse && n3 + n1 <= kStWStages) ? 1 : 0;
  }
  P.cta0 = sp->next_cta % sp->grid;
  sp->next_cta += P.units;
  P.akind = s.akind;
  P.A = s.A;
  P.lda = s.lda;
  P.a_gs = s.a_gs;
  P.Hin = s.Hin;
  P.Win = s.Win;
  P.Cin = s.Cin;
  P.Ho = s.Hin / 2;
  P.Wo = s.Win / 2;
  P.lHin = ilog2(s.Hin);
  P.lWin = ilog2(s.Win);
  P.lCin = ilog2(s.Cin);
  P.lHo = ilog2(P.Ho);
  P.lWo = ilog2(P.Wo);
  // Activations by TMA: rows always; the 3x3 gather when a k-block is one tap
  // (Cin a multiple of 64) and a tile's rows are whole output rows of one
  // image.  Otherwise 16-byte cp.async copies build the tile.
  if (s.akind == SA_ROWS) {
    P.atma = 1;
    P.abytes = 64 * 128 * 2;
  } else {
    P.B = s.Mg / (P.Ho * P.Wo);
    const int rows = std::min(P.Ho, 128 / P.Wo);
    P.atma = (s.Cin % 64 == 0 && P.Wo <= 128 && ((P.Ho * P.Wo) % 128 == 0 || P.B == 1)) ? 1 : 0;
    P.abytes = 64 * P.Wo * rows * 2;
  }
  P.w = static_cast<const uint8_t*>(s.W);
  P.w_gs = s.w_gs;
  P.epi = s.epi;
  P.out = s.out;
  P.ldo = s.ldo;
  P.o_gs = s.o_gs;
  P.bias = s.bias;
  P.b_gs = s.b_gs;
  P.pos = s.pos;
  P.cond = s.cond;
  P.cond_ld = s.cond_ld;
  P.rows_per_clip = s.rows_per_clip;
  P.tok_base = s.tok_base;
  P.tok_gstride = s.tok_gstride;
  P.T = s.T;
  P.fuse = fuse ? 1 : 0;
  P.KB1 = fuse ? (s.N + 63) / 64 : 0;
  P.w1 = static_cast<const uint8_t*>(s.W1);
  P.w1_gs = s.w1_gs;
  P.out1 = s.out1;
  P.ldo1 = s.ldo1;
  P.o1_gs = s.o1_gs;
  P.bias1 = s.bias1;
  P.b1_gs = s.b1_gs;
  P.dep0 = s.dep0;
  P.dep1 = s.dep1;
  P.part_off = sp->part_floats;
  if (S > 1) sp->part_floats += (long long)tiles * S * P.BN * P.rows_pad;
  a.ph[a.nph] = P;
  return a.nph++;
}

int stem_plan_end(StemPlan* sp, float* part, void* counters) {
  StemArgs& a = sp->a;
  uint8_t* c = static_cast<uint8_t*>(counters);
  a.epoch = reinterpret_cast<unsigned*>(c);
  a.exits = reinterpret_cast<unsigned*>(c + 128);
  a.pctr = reinterpret_cast<unsigned*>(c + 256);
  a.tctr = a.pctr + kStemMaxPhases;
  for (int p = 0; p < a.nph; ++p) {
    StemPhase& P = a.ph[p];
    P.part = part + P.part_off;
    {
      const uint64_t d[4] = {64, (uint64_t)P.N, (uint64_t)P.KB, (uint64_t)P.G};
      const uint64_t st[3] = {128, (uint64_t)P.N * 128,
                              (uint64_t)(P.G > 1 ? P.w_gs : (long long)P.KB * P.N * 128)};
      const uint32_t box[4] = {64, (uint32_t)P.BN, (uint32_t)P.kps, 1};
      if (encode(&sp->maps.w[p], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, P.w, d, st, box, CU_TENSOR_MAP_SWIZZLE_128B))
        return -3;
    }
    if (P.atma && P.akind == SA_ROWS) {
      const uint64_t d[3] = {(uint64_t)P.K, (uint64_t)P.Mg, (uint64_t)P.G};
      const uint64_t st[2] = {(uint64_t)P.lda * 2, (uint64_t)(P.G > 1 ? P.a_gs : (long long)P.Mg * P.lda) * 2};
      const uint32_t box[3] = {64, 128, 1};
      if (encode(&sp->maps.x[p], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, P.A, d, st, box, CU_TENSOR_MAP_SWIZZLE_128B))
        return -3;
    } else if (P.atma) {
      // NHWC input of all images: (Cin, Win, Hin, G x B); every second
      // pixel along W and H (traversal strides 1, 2, 2, 1)
      const int rows = std::min(P.Ho, 128 / P.Wo);
      const uint64_t d[4] = {(uint64_t)P.Cin, (uint64_t)P.Win, (uint64_t)P.Hin, (uint64_t)P.G * P.B};
      const uint64_t st[3] = {(uint64_t)P.Cin * 2, (uint64_t)P.Win * P.Cin * 2, (uint64_t)P.Hin * P.Win * P.Cin * 2};
      const uint32_t box[4] = {64, (uint32_t)(2 * P.Wo), (uint32_t)(2 * rows), 1};
      const uint32_t es[4] = {1, 2, 2, 1};
      if (encode_strided(&sp->maps.x[p], 4, P.A, d, st, box, es)) return -3;
    }
    if (P.S == 1 && (P.fuse || P.epi == SE_RELU_F16)) {
      // f16 output rows (the fused 1x1's for fused phases), 64 x 128 boxes
      const void* o = P.fuse ? P.out1 : P.out;
      const long long ldo = P.fuse ? P.ldo1 : P.ldo, ogs = P.fuse ? P.o1_gs : P.o_gs;
      const uint64_t d[3] = {(uint64_t)P.N, (uint64_t)P.Mg, (uint64_t)P.G};
      const uint64_t st[2] = {(uint64_t)ldo * 2, (uint64_t)(P.G > 1 ? ogs : (long long)P.Mg * ldo) * 2};
      const uint32_t box[3] = {64, 128, 1};
      if (encode(&sp->maps.o[p], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, o, d, st, box, CU_TENSOR_MAP_SWIZZLE_128B))
        return -3;
    }
    if (P.fuse) {
      const uint64_t d[4] = {64, (uint64_t)P.N, (uint64_t)P.KB1, (uint64_t)P.G};
      const uint64_t st[3] = {128, (uint64_t)P.N * 128,
                              (uint64_t)(P.G > 1 ? P.w1_gs : (long long)P.KB1 * P.N * 128)};
      const uint32_t box[4] = {64, (uint32_t)P.N, (uint32_t)P.kps1, 1};
      if (encode(&sp->maps.w1[p], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, P.w1, d, st, box, CU_TENSOR_MAP_SWIZZLE_128B))
        return -3;
    }
  }
  if (cudaFuncSetAttribute(k_stem, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sp->smem) != cudaSuccess) {
    set_last_error("stem_plan: cannot reserve %zu bytes of shared memory", sp->smem);
    return -3;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_stem, kStThreads, sp->smem) != cudaSuccess ||
      per_sm < 1) {
    set_last_error("stem_plan: the stem kernel does not fit on an SM");
    return -3;
  }
  return 0;
}

#ifdef CN_STEM_TRACE
// Profiling builds only: point the phase trace at a device buffer of
// (kStemMaxPhases + 1) x grid x 16 u64 (null turns it off).  Events per
// phase: 0/1 activation producer before / after the dependency wait, 2/3 last
// k-block issued / landed, 5 first MMA, 6 last MMA committed, 7 epilogue saw
// the MMAs done, 8 fused 1x1 done / partial stored, 9 split arrivals met,
// 10 reduction slices landed, 11 completion published, 12 first weight load.
extern "C" int cn_stem_trace_set(void* dev_buf) {
  unsigned long long* p = static_cast<unsigned long long*>(dev_buf);
  return (int)cudaMemcpyToSymbol(g_stem_trace, &p, sizeof(p));
}
#endif

int stem_launch(const StemPlan& sp, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sp.grid);
  cfg.blockDim = dim3(kStThreads);
  cfg.dynamicSmemBytes = sp.smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return (int)cudaLaunchKernelEx(&cfg, k_stem, sp.maps, sp.a);
}

}  // namespace cn
