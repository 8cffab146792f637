// tcgen05 / TMEM / TMA GEMM for sm_100a.
//
// Replaces the reference's RDNA4-WMMA attention GEMMs (r_6_2_32_4_2_2_2_4_4_384,
// r_2_24..., r_12_32_4..., r_48_32_4...; run_pinned2.py:100-269 lowers each
// WMMA to 4x mma.sync.m16n8k8 with 128 live f32 fragments per thread) and the
// model's projection / conv-as-GEMM contractions.
//
// One CTA = 4 warps computes a 128 x BN output tile over a K range:
//   warp 0 lane 0 : TMA producer (A 128x64 and B BNx64 f16 tiles, 128B swizzle)
//   warp 1 lane 0 : tcgen05.mma issuer (M=128, N=BN, K=16 per instruction),
//                   f32 accumulator lives in TMEM (BN columns)
//   warp 2        : TMEM allocator
//   all 4 warps   : epilogue (tcgen05.ld -> smem -> fused epilogue -> global)
// Split-K: the K range is divided over the CTAs of a cluster (dims 1x1xS).
// Each CTA stages its partial tile in its own shared memory; after a cluster
// barrier CTA r reduces rows [r*128/S, (r+1)*128/S) by reading the S partials
// over DSMEM in rank order 0..S-1, so the sum order is fixed (deterministic)
// and no global workspace is needed.  No TMA multicast is used.
#include <cstdarg>
#include <cstdio>
#include <cudaTypedefs.h>
#include <map>
#include <mutex>
#include <tuple>

#include "cn_common.cuh"
#include "cn_gemm.cuh"

namespace cn {

namespace {
constexpr int kThreads = 128;
constexpr int kA_Bytes = 128 * 64 * 2;

template <int BN>
struct Tile {
  static constexpr int B_Bytes = BN * 64 * 2;
  static constexpr int Stage = kA_Bytes + B_Bytes;
  static constexpr int MaxStages = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int Ld = BN + 4;  // f32 row stride of the split-K receive tiles (bank spread)
  static constexpr size_t MaxSmem = 1024 + (size_t)MaxStages * Stage + 8 * (2 * 8 + 1) + 64;
};

__device__ __forceinline__ float apply_act(float v, int act) {
  switch (act) {
    case ACT_RELU: return fmaxf(v, 0.0f);
    case ACT_GELU: return 0.5f * v * (1.0f + erff(v * 0.7071067811865476f));
    case ACT_TANH: return tanhf(v);
    default: return v;
  }
}

__device__ __forceinline__ void st_cluster_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

// First row owned by cluster rank r when 128 rows are split over S ranks:
// ranks own [ceil(r*128/S), ceil((r+1)*128/S)), i.e. owner(row) = row*S/128.
__device__ __forceinline__ int owner_row0(int r, int S) { return (r * 128 + S - 1) / S; }

// Vector access only when the address really is 16-byte aligned (row strides
// such as the 3323-wide output vector are not); otherwise element by element.
__device__ __forceinline__ bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

__device__ __forceinline__ float4 ld4(const float* p, int nv) {
  if (nv == 4 && aligned16(p)) return *reinterpret_cast<const float4*>(p);
  float t[4] = {0.f, 0.f, 0.f, 0.f};
  for (int j = 0; j < nv; ++j) t[j] = p[j];
  return make_float4(t[0], t[1], t[2], t[3]);
}
__device__ __forceinline__ void st4(float* p, float4 v, int nv) {
  if (nv == 4 && aligned16(p)) {
    *reinterpret_cast<float4*>(p) = v;
  } else {
    const float t[4] = {v.x, v.y, v.z, v.w};
    for (int j = 0; j < nv; ++j) p[j] = t[j];
  }
}

// Epilogue for one thread: fixed 4-column group n..n+3, rows lr = tid/(BN/4) +
// k*(128/(BN/4)) of this CTA's owned row range.  Rows are processed in
// batches of U so that the global reads of a batch (residual, C, pos, cond)
// are all in flight together; partial sums are added in rank order 0..S-1.
template <int BN, int EPI>
__device__ __forceinline__ void epilogue_rows(const GemmParams& p, const uint8_t* smem, int S, int rpo, int r0,
                                              int m_first, int rows, int n, int group) {
  constexpr int C4 = BN / 4;
  constexpr int RSTEP = kThreads / C4;
  constexpr int Ld = BN + 4;
  constexpr int U = 8;
  const int c4 = threadIdx.x % C4;
  const int nv = min(4, p.N - n);
  const float4* rb = reinterpret_cast<const float4*>(smem);
  float4 bias = make_float4(0.f, 0.f, 0.f, 0.f);
  if (p.bias) bias = ld4(p.bias + (long long)group * p.bias_gstride + n, nv);
  for (int lr0 = threadIdx.x / C4; lr0 < rows; lr0 += RSTEP * U) {
    float4 v[U], old[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int lr = lr0 + u * RSTEP;
      if (lr < rows) {
        float4 a = rb[(lr * Ld) / 4 + c4];
        for (int src = 1; src < S; ++src) {
          const float4 t = rb[((src * rpo + lr) * Ld) / 4 + c4];
          a.x += t.x; a.y += t.y; a.z += t.z; a.w += t.w;
        }
        a.x += bias.x; a.y += bias.y; a.z += bias.z; a.w += bias.w;
        v[u] = a;
      }
    }
    // batch the global reads the epilogue needs
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int lr = lr0 + u * RSTEP;
      if (lr >= rows) continue;
      const long long m = m_first + lr;
      if constexpr (EPI == EPI_F32_ACCUM || EPI == EPI_RESID) {
        old[u] = ld4(reinterpret_cast<const float*>(p.out) + (long long)group * p.out_gstride + m * p.ldo + n, nv);
      } else if constexpr (EPI == EPI_TOKENS) {
        const int clip = (int)(m / p.rows_per_clip);
        const int t = p.tok_base + group * p.tok_gstride + (int)(m % p.rows_per_clip);
        const float4 ps = ld4(p.pos + (long long)t * p.N + n, nv);
        const float4 cs = ld4(p.cond + (long long)clip * p.cond_ld + n, nv);
        v[u] = make_float4((v[u].x + ps.x) + cs.x, (v[u].y + ps.y) + cs.y, (v[u].z + ps.z) + cs.z,
                           (v[u].w + ps.w) + cs.w);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int lr = lr0 + u * RSTEP;
      if (lr >= rows) continue;
      const long long m = m_first + lr;
      if constexpr (EPI == EPI_F32_ACCUM || EPI == EPI_RESID) {
        float* o = reinterpret_cast<float*>(p.out) + (long long)group * p.out_gstride + m * p.ldo + n;
        st4(o, make_float4(old[u].x + v[u].x, old[u].y + v[u].y, old[u].z + v[u].z, old[u].w + v[u].w), nv);
      } else if constexpr (EPI == EPI_F16) {
        __half* o = reinterpret_cast<__half*>(p.out) + (long long)group * p.out_gstride + m * p.ldo + n;
        __align__(8) __half h[4] = {__float2half_rn(apply_act(v[u].x, p.act)), __float2half_rn(apply_act(v[u].y, p.act)),
                                    __float2half_rn(apply_act(v[u].z, p.act)), __float2half_rn(apply_act(v[u].w, p.act))};
        if (nv == 4 && (reinterpret_cast<uintptr_t>(o) & 7) == 0) {
          *reinterpret_cast<uint2*>(o) = *reinterpret_cast<const uint2*>(h);
        } else {
          for (int j = 0; j < nv; ++j) o[j] = h[j];
        }
        if (p.out32)
          st4(p.out32 + m * p.ld32 + n,
              make_float4(__half2float(h[0]), __half2float(h[1]), __half2float(h[2]), __half2float(h[3])), nv);
      } else if constexpr (EPI == EPI_TOKENS) {
        const int clip = (int)(m / p.rows_per_clip);
        const int t = p.tok_base + group * p.tok_gstride + (int)(m % p.rows_per_clip);
        st4(reinterpret_cast<float*>(p.out) + ((long long)clip * p.T + t) * p.ldo + n, v[u], nv);
      } else {  // EPI_F32_OUT
        st4(reinterpret_cast<float*>(p.out) + (long long)group * p.out_gstride + m * p.ldo + n, v[u], nv);
      }
    }
  }
}

template <int BN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const GemmParams p) {
  using TL = Tile<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int ST = p.stages;
  uint8_t* sA = smem;
  uint8_t* sB = smem + ST * kA_Bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.region);
  uint64_t* empty = full + 8;
  uint64_t* done = empty + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.splits;
  const int split = blockIdx.z % S;
  const int group = blockIdx.z / S;
  const int n_tile = blockIdx.x, m_tile = blockIdx.y;
  const int KB = (p.K + 63) >> 6;  // a partial last k-block is zero-filled by TMA
  const int kb0 = split * KB / S, kb1 = (split + 1) * KB / S;
  const int nkb = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  int issued = 0;
  if (warp == 0 && lane == 0) {
    int s = 0;
    uint32_t ph = 0;
    for (int i = 0; i < nkb; ++i) {
      if (i >= ST && !mbar_wait(&empty[s], ph ^ 1, 2)) break;
      mbar_arrive_expect_tx(&full[s], TL::Stage);
      const int kc = (kb0 + i) * 64;
      tma_load_3d(sA + s * kA_Bytes, &tmA, &full[s], kc, m_tile * 128, group);
      if (!B_MN) {
        tma_load_3d(sB + s * TL::B_Bytes, &tmB, &full[s], kc, n_tile * BN, group);
      } else {
#pragma unroll
        for (int j = 0; j < BN / 64; ++j)
          tma_load_3d(sB + s * TL::B_Bytes + j * 8192, &tmB, &full[s], n_tile * BN + j * 64, kc, group);
      }
      issued = i + 1;
      if (++s == ST) { s = 0; ph ^= 1; }
    }
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = umma_idesc_f16(BN, B_MN);
    int s = 0;
    uint32_t ph = 0;
    for (int i = 0; i < nkb; ++i) {
      if (!mbar_wait(&full[s], ph, 1)) break;
      tc_fence_after();
      const uint32_t a_addr = smem_u32(sA + s * kA_Bytes);
      const uint32_t b_addr = smem_u32(sB + s * TL::B_Bytes);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        // K-major SW128: a 16-element K step is +32 bytes inside the swizzle atom.
        const uint64_t ad = umma_desc_sw128(a_addr + k * 32, 16, 1024);
        // MN-major SW128: 8-row K groups are 1024 B apart, 64-wide N blocks 8 KB apart.
        const uint64_t bd = B_MN ? umma_desc_sw128(b_addr + k * 2048, 8192, 1024)
                                 : umma_desc_sw128(b_addr + k * 32, 16, 1024);
        tc_mma_f16(tmem, ad, bd, idesc, (i > 0 || k > 0) ? 1u : 0u);
      }
      tc_commit(&empty[s]);
      if (++s == ST) { s = 0; ph ^= 1; }
    }
    tc_commit(done);
  }
  __syncwarp();

  // ---- accumulator ready; every CTA of the cluster is done with its pipeline smem
  mbar_wait(done, 0, 3);
  tc_fence_after();
  tc_fence_before();
  if (S > 1) cluster_sync(); else __syncthreads();
  tc_fence_after();

  // ---- push: TMEM row -> the owner CTA's receive tile, slot = my split rank
  const int rpo = (128 + S - 1) / S;
  const uint32_t recv = smem_u32(smem);
  {
    const int row = warp * 32 + lane;
    const int owner = row * S / 128;
    const int lr = row - owner_row0(owner, S);
    const uint32_t local = recv + (uint32_t)((split * rpo + lr) * TL::Ld * 4);
    const uint32_t dst = S > 1 ? map_shared_rank(local, (uint32_t)owner) : local;
#pragma unroll 1
    for (int c = 0; c < BN; c += 64) {
      uint32_t r[4][16];
#pragma unroll
      for (int q = 0; q < 4; ++q) tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(c + 16 * q), r[q]);
      tmem_ld_wait();
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int v = 0; v < 4; ++v)
          st_cluster_v4(dst + (uint32_t)((c + 16 * q + 4 * v) * 4), r[q][4 * v], r[q][4 * v + 1], r[q][4 * v + 2],
                        r[q][4 * v + 3]);
    }
  }
  tc_fence_before();
  if (S > 1) cluster_sync(); else __syncthreads();

  // ---- owner rows: sum the S partials in rank order (deterministic) + fused epilogue
  {
    const int r0 = owner_row0(split, S), r1 = owner_row0(split + 1, S);
    const int m_first = m_tile * 128 + r0;
    const int rows = min(r1 - r0, p.M - m_first);
    const int c4 = threadIdx.x % (BN / 4);
    const int n = n_tile * BN + c4 * 4;
    if (rows > 0 && n < p.N) {
      switch (p.epi) {
        case EPI_F32_ACCUM: epilogue_rows<BN, EPI_F32_ACCUM>(p, smem, S, rpo, r0, m_first, rows, n, group); break;
        case EPI_F16: epilogue_rows<BN, EPI_F16>(p, smem, S, rpo, r0, m_first, rows, n, group); break;
        case EPI_RESID: epilogue_rows<BN, EPI_RESID>(p, smem, S, rpo, r0, m_first, rows, n, group); break;
        case EPI_TOKENS: epilogue_rows<BN, EPI_TOKENS>(p, smem, S, rpo, r0, m_first, rows, n, group); break;
        default: epilogue_rows<BN, EPI_F32_OUT>(p, smem, S, rpo, r0, m_first, rows, n, group); break;
      }
    }
  }

  // Error path: do not leave a TMA write in flight into freed shared memory.
  if (warp == 0 && lane == 0 && g_cn_dev_error != 0) {
    for (int i = (issued > ST ? issued - ST : 0); i < issued; ++i) mbar_wait(&full[i % ST], (i / ST) & 1, 0);
  }
  __syncwarp();
  if (warp == 2) tmem_dealloc(tmem, BN);
}

// ------------------------------------------------------------------ host
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

int get_encoder() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode ? 0 : -1;
}

int encode_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1_bytes,
              uint64_t s2_bytes, uint32_t b0, uint32_t b1) {
  if (get_encoder()) {
    set_last_error("cuTensorMapEncodeTiled entry point unavailable");
    return -1;
  }
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1_bytes, s2_bytes};
  cuuint32_t box[3] = {b0, b1, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("cuTensorMapEncodeTiled failed (%d): dims %llu,%llu,%llu strides %llu,%llu box %u,%u", (int)r,
                   (unsigned long long)d0, (unsigned long long)d1, (unsigned long long)d2,
                   (unsigned long long)s1_bytes, (unsigned long long)s2_bytes, b0, b1);
    return (int)r;
  }
  return 0;
}

template <int BN, bool B_MN>
int launch_bn(const GemmPlan& g, cudaStream_t stream) {
  using TL = Tile<BN>;
  static unsigned long long attr_set = 0;  // per instantiation, one bit per device
  auto kern = k_gemm_tc<BN, B_MN>;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set & (1ull << (dev & 63)))) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TL::MaxSmem);
    if (e != cudaSuccess) {
      set_last_error("cudaFuncSetAttribute(smem=%zu): %s", TL::MaxSmem, cudaGetErrorString(e));
      return (int)e;
    }
    attr_set |= 1ull << (dev & 63);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = g.grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = g.smem;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 1;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = (unsigned)g.p.splits;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, g.ta, g.tb, g.p);
  if (e != cudaSuccess) {
    set_last_error("gemm launch (bn=%d splits=%d grid=%u,%u,%u): %s", BN, g.p.splits, g.grid.x, g.grid.y,
                   g.grid.z, cudaGetErrorString(e));
    return (int)e;
  }
  return 0;
}
}  // namespace

// Pipeline depth follows the k-blocks a CTA actually streams (short-K GEMMs
// then fit several CTAs per SM); the split-K receive tiles reuse the same
// region once the main loop is over.
static void gemm_smem_layout(int bn, int K, int splits, int* stages, int* region, size_t* smem) {
  const int stage = kA_Bytes + bn * 128;
  const int maxst = bn == 256 ? 4 : (bn == 128 ? 6 : 8);
  const int kb = (K + 63) / 64;
  const int per = (kb + splits - 1) / splits;
  const int st = per < 2 ? 2 : (per > maxst ? maxst : per);
  const int rpo = (128 + splits - 1) / splits;
  const int recv = splits * rpo * (bn + 4) * 4;
  int reg = st * stage > recv ? st * stage : recv;
  reg = (reg + 63) & ~63;
  *stages = st;
  *region = reg;
  *smem = 1024 + (size_t)reg + 8 * (2 * 8 + 1) + 64;
}

// Clusters of `splits` CTAs (with this smem footprint) that fit on the GPU at
// once; a grid with more clusters runs in several waves.
static int max_active_clusters(int bn, int K, int splits) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  int st, reg;
  size_t smem;
  gemm_smem_layout(bn, K, splits, &st, &reg, &smem);
  const auto key = std::make_tuple(dev, bn, splits, (int)smem);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  int n = 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, 1, splits);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 1;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = (unsigned)splits;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  cudaError_t e = cudaErrorInvalidValue;
  switch (bn) {
    case 64:
      cudaFuncSetAttribute(k_gemm_tc<64, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Tile<64>::MaxSmem);
      e = cudaOccupancyMaxActiveClusters(&n, k_gemm_tc<64, false>, &cfg);
      break;
    case 128:
      cudaFuncSetAttribute(k_gemm_tc<128, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Tile<128>::MaxSmem);
      e = cudaOccupancyMaxActiveClusters(&n, k_gemm_tc<128, false>, &cfg);
      break;
    default:
      cudaFuncSetAttribute(k_gemm_tc<256, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Tile<256>::MaxSmem);
      e = cudaOccupancyMaxActiveClusters(&n, k_gemm_tc<256, false>, &cfg);
      break;
  }
  if (e != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = 148 / splits;
  }
  std::lock_guard<std::mutex> lk(mu);
  cache[key] = n;
  return n;
}

int gemm_choose(int M, int N, int K, int G, int* bn_out, int* s_out) {
  // Cost model per candidate (bn, splits): waves of co-resident clusters x
  // per-CTA time, where a CTA streams its k-blocks (A 16 KB + B bn*128 B each)
  // at ~110 GB/s and pays a fixed prologue / epilogue plus a split-K
  // exchange proportional to the tile.  Weight-streaming GEMMs (M <= 128)
  // therefore spread over all SMs; large-M GEMMs keep splits low.
  const int KB = (K + 63) / 64;
  double best = 1e300;
  int bb = 128, bs = 1;
  const int mt = (M + 127) / 128;
  for (int bn : {64, 128, 256}) {
    const int nt = (N + bn - 1) / bn;
    if (bn > 64 && N <= bn / 2) continue;
    for (int s = 1; s <= 8 && s <= KB; ++s) {
      const long long clusters = (long long)mt * nt * G;
      const int maxc = max_active_clusters(bn, K, s);
      const long long waves = (clusters + maxc - 1) / maxc;
      const double kbs = (double)((KB + s - 1) / s);
      const double t = waves * (kbs * (16384.0 + 128.0 * bn) / 110e3 + 2.0 + (s > 1 ? 0.25 * s * bn / 128.0 : 0.0));
      if (t < best * 0.98) {
        best = t;
        bb = bn;
        bs = s;
      }
    }
  }
  *bn_out = bb;
  *s_out = bs;
  return 0;
}

int gemm_plan(GemmPlan* g, const void* A, long long lda, long long a_gs, const void* B, long long ldb,
              long long b_gs, int M, int N, int K, int G, bool b_mn, int bn, int splits, const GemmParams& epi) {
  if (M <= 0 || N <= 0 || K <= 0 || G <= 0 || (K % 8) != 0) {
    set_last_error("gemm_plan: bad shape M=%d N=%d K=%d G=%d (K must be a positive multiple of 8)", M, N, K, G);
    return -2;
  }
  if ((lda % 8) || (ldb % 8) || (a_gs % 8) || (b_gs % 8) || (reinterpret_cast<uintptr_t>(A) % 16) ||
      (reinterpret_cast<uintptr_t>(B) % 16)) {
    set_last_error("gemm_plan: operands must be 16-byte aligned with row strides a multiple of 8 elements");
    return -2;
  }
  if (b_mn && (N % 8)) {
    set_last_error("gemm_plan: MN-major B needs N %% 8 == 0");
    return -2;
  }
  if (bn <= 0 || splits <= 0) gemm_choose(M, N, K, G, &bn, &splits);
  if (!(bn == 64 || bn == 128 || bn == 256) || splits < 1 || splits > 8 || splits > (K + 63) / 64) {
    set_last_error("gemm_plan: unsupported tiling bn=%d splits=%d", bn, splits);
    return -2;
  }
  g->p = epi;
  g->p.M = M;
  g->p.N = N;
  g->p.K = K;
  g->p.splits = splits;
  g->bn = bn;
  g->b_mn = b_mn;
  gemm_smem_layout(bn, K, splits, &g->p.stages, &g->p.region, &g->smem);
  g->grid = dim3((N + bn - 1) / bn, (M + 127) / 128, G * splits);
  int r = encode_3d(&g->ta, A, K, M, G, lda * 2, (G > 1 ? a_gs : lda * M) * 2, 64, 128);
  if (r) return r;
  if (!b_mn)
    r = encode_3d(&g->tb, B, K, N, G, ldb * 2, (G > 1 ? b_gs : ldb * N) * 2, 64, bn);
  else
    r = encode_3d(&g->tb, B, N, K, G, ldb * 2, (G > 1 ? b_gs : ldb * K) * 2, 64, 64);
  return r;
}

int gemm_launch(const GemmPlan& g, cudaStream_t stream) {
  switch (g.bn | (g.b_mn ? 1 : 0)) {
    case 64: return launch_bn<64, false>(g, stream);
    case 128: return launch_bn<128, false>(g, stream);
    case 256: return launch_bn<256, false>(g, stream);
    case 65: return launch_bn<64, true>(g, stream);
    case 129: return launch_bn<128, true>(g, stream);
    case 257: return launch_bn<256, true>(g, stream);
  }
  set_last_error("gemm_launch: bad plan");
  return -2;
}

int device_error_read_and_clear(cudaStream_t stream, int* code) {
  int v = 0, z = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_cn_dev_error, sizeof(int), 0, cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaMemcpyToSymbolAsync(g_cn_dev_error, &z, sizeof(int), 0, cudaMemcpyHostToDevice, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  *code = v;
  return (int)e;
}

}  // namespace cn
