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
#include <mutex>

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
  static constexpr int Stages = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int RedLd = BN + 4;  // f32 row stride of the staging tile (bank spread)
  static constexpr int Pipe = Stages * Stage;
  static constexpr size_t Smem = 1024 + (size_t)Pipe + 8 * (2 * Stages + 1) + 16;
  static_assert(128 * RedLd * 4 <= Pipe, "staging tile must fit in the pipeline buffers");
};

__device__ __forceinline__ float apply_act(float v, int act) {
  switch (act) {
    case ACT_RELU: return fmaxf(v, 0.0f);
    case ACT_GELU: return 0.5f * v * (1.0f + erff(v * 0.7071067811865476f));
    case ACT_TANH: return tanhf(v);
    default: return v;
  }
}

template <int BN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const GemmParams p) {
  using TL = Tile<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + TL::Stages * kA_Bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + TL::Pipe);
  uint64_t* empty = full + TL::Stages;
  uint64_t* done = empty + TL::Stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  float* red = reinterpret_cast<float*>(smem);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.splits;
  const int split = blockIdx.z % S;
  const int group = blockIdx.z / S;
  const int n_tile = blockIdx.x, m_tile = blockIdx.y;
  const int KB = p.K >> 6;
  const int kb0 = split * KB / S, kb1 = (split + 1) * KB / S;
  const int nkb = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TL::Stages; ++s) {
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
    for (int i = 0; i < nkb; ++i) {
      const int s = i % TL::Stages;
      if (i >= TL::Stages && !mbar_wait(&empty[s], ((i / TL::Stages) & 1) ^ 1, 2)) break;
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
    }
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = umma_idesc_f16(BN, B_MN);
    for (int i = 0; i < nkb; ++i) {
      const int s = i % TL::Stages;
      if (!mbar_wait(&full[s], (i / TL::Stages) & 1, 1)) break;
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
    }
    tc_commit(done);
  }
  __syncwarp();

  // ---- epilogue: TMEM -> staging tile in shared memory ----
  const bool ok = mbar_wait(done, 0, 3);
  tc_fence_after();
  {
    const int row = warp * 32 + lane;
    float* dst = red + row * TL::RedLd;
#pragma unroll 1
    for (int c = 0; c < BN; c += 16) {
      uint32_t r[16];
      tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c, r);
      tmem_ld_wait();
      float4* d4 = reinterpret_cast<float4*>(dst + c);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        d4[q] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                            __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
    }
  }
  (void)ok;
  tc_fence_before();
  if (S > 1) cluster_sync(); else __syncthreads();

  // ---- reduction over the cluster (fixed rank order) + fused epilogue ----
  const int r0 = split * 128 / S, r1 = (split + 1) * 128 / S;
  constexpr int C4 = BN / 4;
  const uint32_t red_s = smem_u32(red);
  const int n0 = n_tile * BN;
  const int m0 = m_tile * 128;
  for (int idx = threadIdx.x; idx < (r1 - r0) * C4; idx += kThreads) {
    const int rr = r0 + idx / C4, c4 = idx % C4;
    const int m = m0 + rr;
    const int n = n0 + c4 * 4;
    if (m >= p.M || n >= p.N) continue;
    const uint32_t off = (uint32_t)((rr * TL::RedLd + c4 * 4) * 4);
    float4 v;
    if (S == 1) {
      v = *reinterpret_cast<const float4*>(red + rr * TL::RedLd + c4 * 4);
    } else {
      v = ld_dsmem_f4(map_shared_rank(red_s + off, 0));
      for (int src = 1; src < S; ++src) {
        const float4 t = ld_dsmem_f4(map_shared_rank(red_s + off, (uint32_t)src));
        v.x += t.x; v.y += t.y; v.z += t.z; v.w += t.w;
      }
    }
    float a[4] = {v.x, v.y, v.z, v.w};
    const int nv = min(4, p.N - n);
    if (p.bias) {
      const float* b = p.bias + (long long)group * p.bias_gstride + n;
      for (int j = 0; j < nv; ++j) a[j] += b[j];
    }
    switch (p.epi) {
      case EPI_F32_ACCUM: {
        float* o = reinterpret_cast<float*>(p.out) + (long long)group * p.out_gstride + (long long)m * p.ldo + n;
        for (int j = 0; j < nv; ++j) o[j] += a[j];
        break;
      }
      case EPI_F16: {
        __half* o = reinterpret_cast<__half*>(p.out) + (long long)group * p.out_gstride + (long long)m * p.ldo + n;
        __half h[4];
        for (int j = 0; j < 4; ++j) h[j] = __float2half_rn(apply_act(a[j], p.act));
        if (nv == 4) {
          *reinterpret_cast<uint2*>(o) = *reinterpret_cast<const uint2*>(h);
        } else {
          for (int j = 0; j < nv; ++j) o[j] = h[j];
        }
        if (p.out32) {
          float* o32 = p.out32 + (long long)m * p.ld32 + n;
          for (int j = 0; j < nv; ++j) o32[j] = __half2float(h[j]);
        }
        break;
      }
      case EPI_RESID: {
        float* o = reinterpret_cast<float*>(p.out) + (long long)group * p.out_gstride + (long long)m * p.ldo + n;
        if (nv == 4) {
          float4 x = *reinterpret_cast<float4*>(o);
          x.x += a[0]; x.y += a[1]; x.z += a[2]; x.w += a[3];
          *reinterpret_cast<float4*>(o) = x;
        } else {
          for (int j = 0; j < nv; ++j) o[j] += a[j];
        }
        break;
      }
      case EPI_TOKENS: {
        const int clip = m / p.rows_per_clip;
        const int t = p.tok_base + group * p.tok_gstride + m % p.rows_per_clip;
        float* o = reinterpret_cast<float*>(p.out) + ((long long)clip * p.T + t) * p.ldo + n;
        const float* ps = p.pos + (long long)t * p.N + n;
        const float* cs = p.cond + (long long)clip * p.cond_ld + n;
        for (int j = 0; j < nv; ++j) o[j] = (a[j] + ps[j]) + cs[j];
        break;
      }
      default: {  // EPI_F32_OUT
        float* o = reinterpret_cast<float*>(p.out) + (long long)group * p.out_gstride + (long long)m * p.ldo + n;
        for (int j = 0; j < nv; ++j) o[j] = a[j];
        break;
      }
    }
  }

  // Peers may still be reading this CTA's staging tile.
  if (S > 1) cluster_sync(); else __syncthreads();

  // Error path: do not leave a TMA write in flight into freed shared memory.
  if (warp == 0 && lane == 0 && g_cn_dev_error != 0) {
    for (int i = (issued > TL::Stages ? issued - TL::Stages : 0); i < issued; ++i)
      mbar_wait(&full[i % TL::Stages], (i / TL::Stages) & 1, 0);
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
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TL::Smem);
    if (e != cudaSuccess) {
      set_last_error("cudaFuncSetAttribute(smem=%zu): %s", TL::Smem, cudaGetErrorString(e));
      return (int)e;
    }
    attr_set |= 1ull << (dev & 63);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = g.grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = TL::Smem;
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

size_t gemm_smem_bytes(int bn) {
  return bn == 256 ? Tile<256>::Smem : (bn == 128 ? Tile<128>::Smem : Tile<64>::Smem);
}

int gemm_choose(int M, int N, int K, int G, int* bn_out, int* s_out) {
  // Cost model: per-CTA time ~ bytes it streams (A tile + B tile per k-block)
  // times the number of waves over 148 SMs, plus a small cost per split for
  // the DSMEM reduction.  Batch-1 GEMMs (M <= 128) are weight-streaming and
  // want all SMs busy; large-M GEMMs want fat tiles.
  const int SMS = 148;
  const int KB = K / 64;
  double best = 1e300;
  int bb = 128, bs = 1;
  const int mt = (M + 127) / 128;
  for (int bn : {64, 128, 256}) {
    const int nt = (N + bn - 1) / bn;
    if (bn > 64 && N <= bn / 2) continue;
    for (int s = 1; s <= 8 && s <= KB; ++s) {
      const long long ctas = (long long)mt * nt * G * s;
      const long long waves = (ctas + SMS - 1) / SMS;
      const double kbs = (double)((KB + s - 1) / s);
      const double t = waves * (kbs * (128 + bn) * 128.0 + 4096.0) + (s > 1 ? 2.0e4 * bn / 128.0 : 0.0);
      if (t < best * 0.97) {
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
  if (M <= 0 || N <= 0 || K <= 0 || G <= 0 || (K % 64) != 0) {
    set_last_error("gemm_plan: bad shape M=%d N=%d K=%d G=%d (K must be a positive multiple of 64)", M, N, K, G);
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
  if (!(bn == 64 || bn == 128 || bn == 256) || splits < 1 || splits > 8 || splits > K / 64) {
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
  g->smem = gemm_smem_bytes(bn);
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
