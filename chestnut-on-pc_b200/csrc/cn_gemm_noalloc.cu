// Split-K GEMM whose scratch lives in a static device array, for callers that
// cannot allocate device memory.
//
// Some hosts embed this library where they may not call cudaMalloc: a process
// whose GPU memory is owned by another allocator (a framework's caching
// allocator or a fixed arena), or code on a latency-critical path where an
// allocation, which can synchronise the device, is not allowed.  They still
// own their inputs and outputs; what they cannot provide is workspace.
//
// cn_gemm_wmma_f16_noalloc computes the same C[M][N] += A[M][K] * B^T (B given
// as [N][K]) as cn_gemm_wmma_f16.  Its split-K reduction goes through global
// memory like the persistent trunk's: every CTA of a 128 x 128 output tile
// writes its partial tile, counts itself on the tile's arrival counter, and
// the last CTA to arrive adds the S partials in split order 0..S-1 into C, so
// the result does not depend on which CTA arrives last.  The partial tiles and
// the counters live in g_noalloc_scratch below (kNoallocScratchBytes per
// device that loads the library, held until the process exits).
//
// Sharing: every call uses the same array, and it keeps the previous call's
// partial tiles.  Each call clears the counters it uses before its kernel
// runs; calls that overlap on the GPU (different streams, or graphs replayed
// concurrently) race on the array.
#include <mutex>

#include "cn_common.cuh"
#include "cn_gemm.cuh"

namespace cn {

constexpr size_t kNoallocScratchBytes = size_t(16) << 20;  // 16 MiB
constexpr size_t kNoallocCounterBytes = 4096;              // 1024 output tiles
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoallocScratchBytes];

namespace {

constexpr int kNaThreads = 128;
constexpr int kNaStages = 4;
constexpr int kNaTile = 128 * 64 * 2;  // one 128-row x 64-k f16 tile (A or B)
constexpr int kNaStage = 2 * kNaTile;
constexpr int kNaMaxSplits = 16;
// Barrier area after the stage buffers: full[kNaStages], empty[kNaStages],
// done (8 bytes each), then the TMEM slot and the last-arriver flag (4 each).
constexpr int kNaBarBytes = (2 * kNaStages + 1) * 8 + 2 * 4;
static_assert(kNaBarBytes <= 128, "barrier area of the no-alloc GEMM");

struct NoallocArgs {
  int M, N, K, S;
  int tiles_n, Mp, Np;  // Mp, Np: M, N rounded up to 128 (partial tile layout [S][Mp][Np])
  float* C;
  float* part;
  unsigned* ctr;
};

__global__ void __launch_bounds__(kNaThreads, 1)
    k_gemm_noalloc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const NoallocArgs g) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kNaStages * kNaStage);
  uint64_t* empty = full + kNaStages;
  uint64_t* done = empty + kNaStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* last = reinterpret_cast<volatile int*>(done + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = blockIdx.x, mt = blockIdx.y, s = blockIdx.z;
  const int KB = (g.K + 63) / 64;  // a partial last k-block is zero-filled by TMA
  const int kb0 = s * KB / g.S, kb1 = (s + 1) * KB / g.S;
  const int nkb = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNaStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(done, 1);
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  int issued = 0;
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < nkb; ++i) {
      const int st = i % kNaStages;
      if (!mbar_wait(&empty[st], ((i / kNaStages) & 1) ^ 1, 2)) break;
      mbar_arrive_expect_tx(&full[st], kNaStage);
      tma_load_3d(smem + st * kNaStage, &tmA, &full[st], (kb0 + i) * 64, mt * 128, 0);
      tma_load_3d(smem + st * kNaStage + kNaTile, &tmB, &full[st], (kb0 + i) * 64, nt * 128, 0);
      issued = i + 1;
    }
  } else if (warp == 1 && lane == 0) {
    const uint32_t idesc = umma_idesc_f16(128, false);
    for (int i = 0; i < nkb; ++i) {
      const int st = i % kNaStages;
      if (!mbar_wait(&full[st], (i / kNaStages) & 1, 1)) break;
      tc_fence_after();
      const uint32_t a = smem_u32(smem + st * kNaStage), b = a + kNaTile;
#pragma unroll
      for (int k = 0; k < 4; ++k)
        tc_mma_f16(tmem, umma_desc_sw128(a + k * 32, 16, 1024), umma_desc_sw128(b + k * 32, 16, 1024), idesc,
                   (i > 0 || k > 0) ? 1u : 0u);
      tc_commit(&empty[st]);
    }
    tc_commit(done);
  }
  __syncwarp();

  const bool have = mbar_wait(done, 0, 3);
  tc_fence_after();
  const int row = warp * 32 + lane;  // TMEM lane = tile row
  const int m = mt * 128 + row;
  const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);
  if (g.S == 1) {
    if (have)
      for (int c = 0; c < 128; c += 16) {
        uint32_t r[16];
        tmem_ld16(taddr + c, r);  // warp-collective: every lane loads, rows past M are dropped
        tmem_ld_wait();
        if (m < g.M)
          for (int j = 0; j < 16; ++j) {
            const int n = nt * 128 + c + j;
            if (n < g.N) g.C[(size_t)m * g.N + n] += __uint_as_float(r[j]);
          }
      }
  } else {
    float* P = g.part + ((size_t)s * g.Mp + m) * g.Np + nt * 128;
    if (have)
      for (int c = 0; c < 128; c += 16) {
        uint32_t r[16];
        tmem_ld16(taddr + c, r);
        tmem_ld_wait();
#pragma unroll
        for (int v = 0; v < 4; ++v)
          *reinterpret_cast<float4*>(P + c + 4 * v) =
              make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]), __uint_as_float(r[4 * v + 2]),
                          __uint_as_float(r[4 * v + 3]));
      }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned* ctr = g.ctr + mt * g.tiles_n + nt;
      const unsigned prev = atomicAdd(ctr, 1u);
      *last = have && prev == (unsigned)(g.S - 1);
      if (prev == (unsigned)(g.S - 1)) *ctr = 0u;  // every split has arrived: ready for the next call
    }
    __syncthreads();
    if (*last) {
      __threadfence();
      // rows r = warp + 4j, columns 4*lane..4*lane+3: each warp reads whole 512 B rows
      for (int r0 = warp; r0 < 128; r0 += 16) {
        float4 acc[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          acc[j] = __ldcg(reinterpret_cast<const float4*>(g.part + ((size_t)(mt * 128 + r0 + 4 * j)) * g.Np +
                                                          nt * 128 + 4 * lane));
        for (int q = 1; q < g.S; ++q)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(
                g.part + ((size_t)q * g.Mp + mt * 128 + r0 + 4 * j) * g.Np + nt * 128 + 4 * lane));
            acc[j].x += v.x; acc[j].y += v.y; acc[j].z += v.z; acc[j].w += v.w;
          }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int mm = mt * 128 + r0 + 4 * j, n = nt * 128 + 4 * lane;
          if (mm >= g.M) continue;
          const float t[4] = {acc[j].x, acc[j].y, acc[j].z, acc[j].w};
          for (int e = 0; e < 4 && n + e < g.N; ++e) g.C[(size_t)mm * g.N + n + e] += t[e];
        }
      }
    }
  }
  // Error path: no TMA write may still be in flight when the CTA exits.  Best
  // effort: if this bounded drain also runs out, the error is already recorded
  // and the CTA exits anyway (as in cn_gemm.cu).
  if (warp == 0 && lane == 0 && g_cn_dev_error != 0)
    for (int i = (issued > kNaStages ? issued - kNaStages : 0); i < issued; ++i)
      mbar_wait(&full[i % kNaStages], (i / kNaStages) & 1, 0, 100000000ull);
  tc_fence_before();
  __syncthreads();
  if (warp == 2) tmem_dealloc(tmem, 128);
}

// stage buffers + the barrier area rounded up to 128 bytes + 1024 bytes of alignment slack
size_t noalloc_smem_bytes() { return (size_t)kNaStages * kNaStage + 128 + 1024; }

}  // namespace

}  // namespace cn

extern "C" int cn_gemm_wmma_f16_noalloc(const void* A, const void* B, float* C, int M, int N, int K, int splits,
                                        void* stream) {
  using namespace cn;
  if (!A || !B || !C || M <= 0 || N <= 0 || K <= 0 || (K % 8) ||
      (reinterpret_cast<uintptr_t>(A) % 16) || (reinterpret_cast<uintptr_t>(B) % 16)) {
    set_last_error("cn_gemm_wmma_f16_noalloc: bad arguments (M=%d N=%d K=%d; K %% 8 == 0 and 16-byte aligned A, B "
                   "required)", M, N, K);
    return -2;
  }
  const int KB = (K + 63) / 64;
  if (splits < 1 || splits > kNaMaxSplits || splits > KB) {
    set_last_error("cn_gemm_wmma_f16_noalloc: splits=%d outside [1, min(16, ceil(K/64)=%d)]", splits, KB);
    return -2;
  }
  const int tm = (M + 127) / 128, tn = (N + 127) / 128;
  const size_t Mp = (size_t)tm * 128, Np = (size_t)tn * 128;
  // Scratch is used only with splits > 1: one arrival counter per output tile
  // (at most 1024 tiles) and S partial tiles.  splits == 1 needs none.
  const size_t part_bytes = splits > 1 ? (size_t)splits * Mp * Np * 4 : 0;
  if (splits > 1 && (size_t)tm * tn * 4 > kNoallocCounterBytes) {
    set_last_error("cn_gemm_wmma_f16_noalloc: %d x %d output tiles exceed the tile limit of the static scratch "
                   "(at most 1024 output tiles when splits > 1)", tm, tn);
    return -2;
  }
  if (splits > 1 && kNoallocCounterBytes + part_bytes > kNoallocScratchBytes) {
    set_last_error("cn_gemm_wmma_f16_noalloc: %d x %d tiles x %d splits need %zu bytes of scratch; the static "
                   "scratch holds %zu bytes", tm, tn, splits, kNoallocCounterBytes + part_bytes,
                   kNoallocScratchBytes);
    return -2;
  }
  // Set-up, once per device with that device current: the device address of
  // the static array (the host-side name is only a stand-in) and the kernel's
  // shared-memory limit.  The first call on a device does this, so it should
  // come before any stream capture.
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    set_last_error("cn_gemm_wmma_f16_noalloc: no current device");
    return -3;
  }
  static std::mutex mu;
  static void* scratch_addr[64] = {};
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!scratch_addr[dev]) {
      void* p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess || !p) {
        set_last_error("cn_gemm_wmma_f16_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
        return -3;
      }
      e = cudaFuncSetAttribute(k_gemm_noalloc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)noalloc_smem_bytes());
      if (e != cudaSuccess) {
        set_last_error("cn_gemm_wmma_f16_noalloc: %s", cudaGetErrorString(e));
        return -3;
      }
      scratch_addr[dev] = p;
    }
    base = scratch_addr[dev];
  }
  NoallocArgs g;
  g.M = M;
  g.N = N;
  g.K = K;
  g.S = splits;
  g.tiles_n = tn;
  g.Mp = (int)Mp;
  g.Np = (int)Np;
  g.C = C;
  g.ctr = static_cast<unsigned*>(base);
  g.part = reinterpret_cast<float*>(static_cast<uint8_t*>(base) + kNoallocCounterBytes);
  CUtensorMap ta, tb;
  {
    const uint64_t da[3] = {(uint64_t)K, (uint64_t)M, 1}, sa[2] = {(uint64_t)K * 2, (uint64_t)K * M * 2};
    const uint64_t db[3] = {(uint64_t)K, (uint64_t)N, 1}, sb[2] = {(uint64_t)K * 2, (uint64_t)K * N * 2};
    const uint32_t box[3] = {64, 128, 1};
    if (encode(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, A, da, sa, box, CU_TENSOR_MAP_SWIZZLE_128B) ||
        encode(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, B, db, sb, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return -3;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (splits > 1 && cudaMemsetAsync(g.ctr, 0, (size_t)tm * tn * 4, st) != cudaSuccess) {
    set_last_error("cn_gemm_wmma_f16_noalloc: clearing the tile counters failed");
    return -3;
  }
  k_gemm_noalloc<<<dim3(tn, tm, splits), kNaThreads, noalloc_smem_bytes(), st>>>(ta, tb, g);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error("cn_gemm_wmma_f16_noalloc: launch failed: %s", cudaGetErrorString(e));
    return -3;
  }
  return 0;
}
