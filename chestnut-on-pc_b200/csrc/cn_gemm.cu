// tcgen05 / TMEM / TMA GEMM for sm_100a.
//
// Replaces the reference's RDNA4-WMMA attention GEMMs (r_6_2_32_4_2_2_2_4_4_384,
// r_2_24..., r_12_32_4..., r_48_32_4...; run_pinned2.py:100-269 lowers each
// WMMA to 4x mma.sync.m16n8k8 with 128 live f32 fragments per thread) and the
// model's projection / conv-as-GEMM contractions.
//
// One CTA = 4 warps computes a 128 x BN output tile over a K range:
//   warp 0 lane 0 : TMA producer (A 128x64 and B BNx64 f16 tiles, 128B swizzle);
//                   weight tiles for the first stages are requested before
//                   griddepcontrol.wait, since weights never depend on an
//                   earlier kernel
//   warp 1 lane 0 : tcgen05.mma issuer (M=128, N=BN, K=16 per instruction),
//                   f32 accumulator in TMEM (BN columns)
//   warp 2        : TMEM allocator
//   all 4 warps   : epilogue (tcgen05.ld -> shared memory -> fused epilogue)
// Split-K: the K range is divided over the S CTAs of a cluster (dims 1x1xS).
// Every CTA owns 128/S accumulator rows.  In column chunks of up to 128, each
// CTA stages its partial rows grouped by owner, ships every peer its slice
// with one DSMEM bulk copy (cp.async.bulk shared::cluster, mbarrier
// complete_tx), and owners add the S partials in rank order 0..S-1, so the
// result is deterministic and needs no global workspace.  No TMA multicast.
// Each instantiation carries a single epilogue (template EPI): the kernel runs
// once per SM per launch, so compact code (few cold instruction-cache lines)
// matters as much as instruction count.
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
constexpr size_t kMaxDynSmem = 227 * 1024;
constexpr int kMaxSplits = 16;  // split-K cluster size (above 8 uses non-portable clusters)

template <int BN>
struct Tile {
  static constexpr int B_Bytes = BN * 64 * 2;
  static constexpr int Stage = kA_Bytes + B_Bytes;
  static constexpr int MaxStages = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int CH = BN < 128 ? BN : 128;  // split-K exchange chunk (columns)
  static constexpr int LdC = CH + 4;              // f32 row stride of staging / receive tiles
};

__device__ __forceinline__ float apply_act(float v, int act) {
  switch (act) {
    case ACT_RELU: return fmaxf(v, 0.0f);
    case ACT_GELU: return 0.5f * v * (1.0f + erff(v * 0.7071067811865476f));
    case ACT_TANH: return tanhf(v);
    default: return v;
  }
}

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

// First row owned by cluster rank r when 128 rows are split over S ranks:
// ranks own [ceil(r*128/S), ceil((r+1)*128/S)), i.e. owner(row) = row*S/128.
__device__ __forceinline__ int owner_row0(int r, int S) { return (r * 128 + S - 1) / S; }

// Epilogue of one column chunk: thread -> fixed 4-column group, rows
// lr = tid / (CH/4) + k * (128 / (CH/4)) of the owned rows.  The S partials are
// added in rank order (own partial from the staging tile, the others from the
// receive tile); xs holds the prefetched residual / C rows when non-null.
template <int BN, int EPI>
__device__ __forceinline__ void epilogue_chunk(const GemmParams& p, const float* stg, const float* rcv, const float* xs,
                                               int S, int split, int rpo, int m_first, int rows, int n0, int group) {
  constexpr int CH = Tile<BN>::CH, LdC = Tile<BN>::LdC;
  constexpr int C4 = CH / 4;
  constexpr int RSTEP = kThreads / C4;
  const int c4 = threadIdx.x % C4;
  const int n = n0 + c4 * 4;
  if (n >= p.N) return;
  const int nv = min(4, p.N - n);
  float4 bias = make_float4(0.f, 0.f, 0.f, 0.f);
  if (p.bias) bias = ld4(p.bias + (long long)group * p.bias_gstride + n, nv);
#pragma unroll 1
  for (int lr = threadIdx.x / C4; lr < rows; lr += RSTEP) {
    float4 a = *reinterpret_cast<const float4*>((split == 0 ? stg : rcv) + lr * LdC + c4 * 4);
    for (int src = 1; src < S; ++src) {
      const float4 t = *reinterpret_cast<const float4*>((src == split ? stg : rcv) + (src * rpo + lr) * LdC + c4 * 4);
      a.x += t.x; a.y += t.y; a.z += t.z; a.w += t.w;
    }
    a.x += bias.x; a.y += bias.y; a.z += bias.z; a.w += bias.w;
    const long long m = m_first + lr;
    if constexpr (EPI == EPI_F32_ACCUM || EPI == EPI_RESID) {
      float* o = reinterpret_cast<float*>(p.out) + (long long)group * p.out_gstride + m * p.ldo + n;
      const float4 old = xs ? *reinterpret_cast<const float4*>(xs + lr * CH + c4 * 4) : ld4(o, nv);
      st4(o, make_float4(old.x + a.x, old.y + a.y, old.z + a.z, old.w + a.w), nv);
    } else if constexpr (EPI == EPI_F16) {
      __half* o = reinterpret_cast<__half*>(p.out) + (long long)group * p.out_gstride + m * p.ldo + n;
      __align__(8) __half h[4] = {__float2half_rn(apply_act(a.x, p.act)), __float2half_rn(apply_act(a.y, p.act)),
                                  __float2half_rn(apply_act(a.z, p.act)), __float2half_rn(apply_act(a.w, p.act))};
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
      const float4 ps = ld4(p.pos + (long long)t * p.N + n, nv);
      const float4 cs = ld4(p.cond + (long long)clip * p.cond_ld + n, nv);
      st4(reinterpret_cast<float*>(p.out) + ((long long)clip * p.T + t) * p.ldo + n,
          make_float4((a.x + ps.x) + cs.x, (a.y + ps.y) + cs.y, (a.z + ps.z) + cs.z, (a.w + ps.w) + cs.w), nv);
    } else {  // EPI_F32_OUT
      st4(reinterpret_cast<float*>(p.out) + (long long)group * p.out_gstride + m * p.ldo + n, a, nv);
    }
  }
}

// f16 epilogue of an unsplit tile straight from the TMEM registers: thread =
// accumulator row (lane quadrant = warp), 16 columns per tcgen05.ld; bias and
// activation, then the row's 16-column segment as two 16-byte stores.  No
// staging through shared memory, no per-element bounds checks (the host
// enables it only for N % 16 == 0 and 16-byte aligned rows).  The arithmetic
// is the staged epilogue's: f16(act(acc + bias)).
template <int BN, int ACT>
__device__ __forceinline__ void epilogue_direct(const GemmParams& p, uint32_t tmem, int m_tile, int n_tile,
                                                int group) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long m = (long long)m_tile * 128 + warp * 32 + lane;
  const bool live = m < p.M;
  const float* bias = p.bias ? p.bias + (long long)group * p.bias_gstride : nullptr;
  __half* out = reinterpret_cast<__half*>(p.out) + (long long)group * p.out_gstride + m * p.ldo;
#pragma unroll 1
  for (int c = 0; c < BN; c += 16) {
    const int n = n_tile * BN + c;
    if (n >= p.N) break;  // warp-uniform: tcgen05.ld is .aligned
    uint32_t r[16];
    tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c, r);
    tmem_ld_wait();
    float v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
    if (bias) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 b = __ldg(reinterpret_cast<const float4*>(bias + n) + q);
        v[4 * q] += b.x; v[4 * q + 1] += b.y; v[4 * q + 2] += b.z; v[4 * q + 3] += b.w;
      }
    }
    if (!live) continue;
    __align__(16) __half h[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) h[j] = __float2half_rn(apply_act(v[j], ACT));
    reinterpret_cast<uint4*>(out + n)[0] = reinterpret_cast<const uint4*>(h)[0];
    reinterpret_cast<uint4*>(out + n)[1] = reinterpret_cast<const uint4*>(h)[1];
  }
}

// BM: layout of B -- 0 K-major [N][K], 1 MN-major [K][N], 2 k-blocked [KB][N][64].
template <int BN, int BM, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const __grid_constant__ CUtensorMap tmX, const GemmParams p) {
  using TL = Tile<BN>;
  constexpr int CH = TL::CH, LdC = TL::LdC, NCH = BN / CH;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int ST = p.stages;
  uint8_t* sA = smem;
  uint8_t* sB = smem + ST * kA_Bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.region);
  uint64_t* empty = full + 8;
  uint64_t* done = empty + 8;
  uint64_t* recv_bar = done + 1;  // split-K slices arriving from cluster peers (one phase per chunk)
  uint64_t* xbar = done + 2;      // prefetched residual rows (one phase per chunk)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 3);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.splits;
  const int split = blockIdx.z % S;
  const int group = blockIdx.z / S;
  const int n_tile = blockIdx.x, m_tile = blockIdx.y;
  const int KB = (p.K + 63) >> 6;  // a partial last k-block is zero-filled by TMA
  const int kb0 = split * KB / S, kb1 = (split + 1) * KB / S;
  const int nkb = kb1 - kb0;
  const int rpo = (128 + S - 1) / S;  // rows per owner (upper bound)
  const int own0 = owner_row0(split, S), own1 = owner_row0(split + 1, S);
  const uint32_t slice_bytes = (uint32_t)((own1 - own0) * LdC * 4);

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    mbar_init(recv_bar, 1);
    mbar_init(xbar, 1);
    // armed before the first cluster barrier, i.e. before any peer can send
    if (S > 1) mbar_arrive_expect_tx(recv_bar, (uint32_t)(S - 1) * slice_bytes);
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (p.prefetch) tma_prefetch_desc(&tmX);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Dependents may launch now; the TMEM allocation above is already held, so a
  // dependent CTA landing on this SM cannot starve it.
  pdl_trigger();

  int issued = 0;
  if (warp == 0 && lane == 0) {
    auto load_b = [&](int stage, int kb) {
      if constexpr (BM == 2) {
        tma_load_4d(sB + stage * TL::B_Bytes, &tmB, &full[stage], 0, n_tile * BN, kb, group);
      } else if constexpr (BM == 0) {
        tma_load_3d(sB + stage * TL::B_Bytes, &tmB, &full[stage], kb * 64, n_tile * BN, group);
      } else {
#pragma unroll
        for (int j = 0; j < BN / 64; ++j)
          tma_load_3d(sB + stage * TL::B_Bytes + j * 8192, &tmB, &full[stage], n_tile * BN + j * 64, kb * 64, group);
      }
    };
    auto load_a = [&](int stage, int kb) {
      tma_load_3d(sA + stage * kA_Bytes, &tmA, &full[stage], kb * 64, m_tile * 128, group);
    };
    // B (weights) never depends on an earlier kernel: fill the first stages
    // with it before waiting for the producer of A (unless the caller says B
    // may be produced by an earlier kernel).
    const int pre = nkb < ST ? nkb : ST;
    if (p.b_dep) pdl_wait();
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(&full[i], TL::Stage);
      load_b(i, kb0 + i);
    }
    pdl_wait();
    for (int i = 0; i < pre; ++i) load_a(i, kb0 + i);
    issued = pre;
    int s = pre == ST ? 0 : pre;
    uint32_t ph = pre == ST ? 1 : 0;
    for (int i = pre; i < nkb; ++i) {
      if (!mbar_wait(&empty[s], ph ^ 1, 2)) break;
      mbar_arrive_expect_tx(&full[s], TL::Stage);
      load_a(s, kb0 + i);
      load_b(s, kb0 + i);
      issued = i + 1;
      if (++s == ST) { s = 0; ph ^= 1; }
    }
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = umma_idesc_f16(BN, BM == 1);
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
        const uint64_t bd = BM == 1 ? umma_desc_sw128(b_addr + k * 2048, 8192, 1024)
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

  bool direct = false;
  if constexpr (EPI == EPI_F16) {
    direct = p.direct != 0;
    if (direct) {
      pdl_wait();  // the epilogue reads / writes activations of earlier kernels
      switch (p.act) {
        case ACT_RELU: epilogue_direct<BN, ACT_RELU>(p, tmem, m_tile, n_tile, group); break;
        case ACT_GELU: epilogue_direct<BN, ACT_GELU>(p, tmem, m_tile, n_tile, group); break;
        case ACT_TANH: epilogue_direct<BN, ACT_TANH>(p, tmem, m_tile, n_tile, group); break;
        default: epilogue_direct<BN, ACT_NONE>(p, tmem, m_tile, n_tile, group); break;
      }
    }
  }
  if (!direct) {
  // ---- post-MMA, per column chunk.  Shared memory (pipeline buffers are free
  // now): staging [S][rpo][LdC] f32 = this CTA's partial rows grouped by owner
  // rank; recv [S][rpo][LdC] = the peers' partials of the owned rows;
  // xs [rpo][CH] = the prefetched residual rows of the owned rows.
  float* stg = reinterpret_cast<float*>(smem);
  float* rcv = stg + S * rpo * LdC;
  // TMA destination: 1024-byte aligned offset (matches gemm_smem_layout)
  float* xs = p.prefetch
                  ? reinterpret_cast<float*>(smem + ((((S > 1 ? 2 : 1) * S * rpo * LdC * 4) + 1023) & ~1023))
                  : nullptr;
  const int m_first = m_tile * 128 + own0;
  const int rows = min(own1 - own0, p.M - m_first);
  const int row = warp * 32 + lane;
  const int my_owner = row * S / 128;
  float* my_dst = stg + (my_owner * rpo + row - owner_row0(my_owner, S)) * LdC;
#pragma unroll 1
  for (int ch = 0; ch < NCH; ++ch) {
    const int c0 = ch * CH;
    if (xs && threadIdx.x == 96 && rows > 0) {
      pdl_wait();  // the residual was written by an earlier kernel
      mbar_arrive_expect_tx(xbar, (uint32_t)(rpo * CH * 4));
      tma_load_3d(xs, &tmX, xbar, n_tile * BN + c0, m_first, group);
    }
    constexpr int W = 64 < CH ? 64 : CH;
#pragma unroll
    for (int c = 0; c < CH; c += W) {
      uint32_t r[W / 16][16];
#pragma unroll
      for (int q = 0; q < W / 16; ++q)
        tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(c0 + c + 16 * q), r[q]);
      tmem_ld_wait();
#pragma unroll
      for (int q = 0; q < W / 16; ++q)
#pragma unroll
        for (int v = 0; v < 4; ++v)
          *reinterpret_cast<uint4*>(my_dst + c + 16 * q + 4 * v) =
              make_uint4(r[q][4 * v], r[q][4 * v + 1], r[q][4 * v + 2], r[q][4 * v + 3]);
    }
    fence_proxy_async_smem();
    __syncthreads();
    if (S > 1) {
      // one slice per peer; a thread's bulk copies complete one after
      // another, so the four warps share them
      if (lane == 0) {
        for (int q = warp; q < S; q += kThreads / 32) {
          if (q == split) continue;
          const int rq = owner_row0(q + 1, S) - owner_row0(q, S);
          bulk_s2cluster(map_shared_rank(smem_u32(rcv + split * rpo * LdC), (uint32_t)q),
                         smem_u32(stg + q * rpo * LdC), (uint32_t)(rq * LdC * 4),
                         map_shared_rank(smem_u32(recv_bar), (uint32_t)q));
        }
      }
      mbar_wait(recv_bar, (uint32_t)(ch & 1), 6);
      // After the last chunk every copy into this CTA has landed: announce it
      // now and wait for the others only before exiting (a CTA's staging tile
      // is the source of its peers' copies).
      if (ch + 1 == NCH) cluster_arrive();
    }
    if (xs && rows > 0) mbar_wait(xbar, (uint32_t)(ch & 1), 7);
    pdl_wait();  // the epilogue reads / writes activations of earlier kernels
    if (rows > 0)
      epilogue_chunk<BN, EPI>(p, stg, rcv, xs, S, split, rpo, m_first, rows, n_tile * BN + c0, group);
    if (ch + 1 < NCH) {
      // everyone is done with this chunk's staging / receive tiles before the
      // next chunk overwrites them; re-arm the receive barrier first
      if (S > 1 && threadIdx.x == 0) mbar_arrive_expect_tx(recv_bar, (uint32_t)(S - 1) * slice_bytes);
      tc_fence_before();
      if (S > 1) cluster_sync(); else __syncthreads();
      tc_fence_after();
    }
  }
  // Peers' bulk copies out of this CTA's staging tile have landed once every
  // CTA of the cluster has received its last chunk.
  if (S > 1) cluster_wait();
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

int encode(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base, const uint64_t* dims,
           const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz) {
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
    es[i] = 1;
    if (i + 1 < rank) st[i] = strides_bytes[i];
  }
  CUresult r = g_encode(map, dt, (cuuint32_t)rank, const_cast<void*>(base), d, st, b, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("cuTensorMapEncodeTiled failed (%d): rank %d dims %llu,%llu,%llu box %u,%u", (int)r, rank,
                   (unsigned long long)dims[0], (unsigned long long)dims[1],
                   (unsigned long long)(rank > 2 ? dims[2] : 1), box[0], box[1]);
    return (int)r;
  }
  return 0;
}

using KernelFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, GemmParams);

template <int BN, int BM, int EPI>
KernelFn kernel_ptr() {
  return reinterpret_cast<KernelFn>(k_gemm_tc<BN, BM, EPI>);
}

// Instantiations: the engine's k-blocked weights with every frame epilogue,
// and the kernel-level entry point (K- or MN-major B, C += A*B).
KernelFn pick_kernel(int bn, int bm, int epi) {
#define CN_K(BN_)                                                                 \
  if (bn == BN_) {                                                                \
    if (bm == B_K_BLOCKED) {                                                      \
      switch (epi) {                                                              \
        case EPI_F16: return kernel_ptr<BN_, B_K_BLOCKED, EPI_F16>();             \
        case EPI_RESID: return kernel_ptr<BN_, B_K_BLOCKED, EPI_RESID>();         \
        case EPI_TOKENS: return kernel_ptr<BN_, B_K_BLOCKED, EPI_TOKENS>();       \
        case EPI_F32_OUT: return kernel_ptr<BN_, B_K_BLOCKED, EPI_F32_OUT>();     \
        case EPI_F32_ACCUM: return kernel_ptr<BN_, B_K_BLOCKED, EPI_F32_ACCUM>(); \
      }                                                                           \
    } else if (epi == EPI_F32_ACCUM) {                                            \
      return bm == B_K_MAJOR ? kernel_ptr<BN_, B_K_MAJOR, EPI_F32_ACCUM>()       \
                             : kernel_ptr<BN_, B_MN_MAJOR, EPI_F32_ACCUM>();      \
    }                                                                             \
  }
  CN_K(64)
  CN_K(128)
  CN_K(256)
#undef CN_K
  return nullptr;
}

int launch_plan(const GemmPlan& g, cudaStream_t stream) {
  static std::mutex mu;
  static std::map<std::pair<void*, int>, bool> attr_set;
  KernelFn kern = pick_kernel(g.bn, g.b_mode, g.p.epi);
  if (!kern) {
    set_last_error("gemm_launch: no kernel for bn=%d b_mode=%d epi=%d", g.bn, g.b_mode, g.p.epi);
    return -2;
  }
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto key = std::make_pair(reinterpret_cast<void*>(kern), dev);
    if (!attr_set.count(key)) {
      cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(kern),
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxDynSmem);
      if (e == cudaSuccess)  // split-K clusters of up to 16 CTAs
        e = cudaFuncSetAttribute(reinterpret_cast<const void*>(kern),
                                 cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (e != cudaSuccess) {
        set_last_error("cudaFuncSetAttribute(smem=%zu): %s", kMaxDynSmem, cudaGetErrorString(e));
        return (int)e;
      }
      attr_set[key] = true;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = g.grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = g.smem;
  cfg.stream = stream;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 1;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = (unsigned)g.p.splits;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = g.pdl ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, g.ta, g.tb, g.tx, g.p);
  if (e != cudaSuccess) {
    set_last_error("gemm launch (bn=%d splits=%d grid=%u,%u,%u): %s", g.bn, g.p.splits, g.grid.x, g.grid.y, g.grid.z,
                   cudaGetErrorString(e));
    return (int)e;
  }
  return 0;
}
}  // namespace

// Pipeline depth follows the k-blocks a CTA actually streams (short-K GEMMs
// then fit several CTAs per SM); after the main loop the same region holds the
// split-K staging / receive tiles and the prefetched residual rows.
static void gemm_smem_layout(int bn, int K, int splits, bool prefetch, int* stages, int* region, size_t* smem,
                             bool direct = false) {
  const int stage = kA_Bytes + bn * 128;
  const int kb = (K + 63) / 64;
  const int per = (kb + splits - 1) / splits;
  // Unsplit CTAs with a short K keep a short ring (~96 KB) so that two or
  // three share an SM: one CTA's epilogue then overlaps another's main loop.
  // Long-K CTAs and split-K clusters (weight-streaming GEMMs of a few rows)
  // keep deep rings.
  const bool shallow = splits == 1 && per <= 12;
  // (a direct epilogue stages nothing: two-stage rings of 64-wide and
  // 128-wide tiles let three CTAs share an SM)
  const int maxst = shallow ? (bn == 256 || direct ? 2 : 3) : (bn == 256 ? 4 : (bn == 128 ? 6 : 8));
  const int st = per < 2 ? 2 : (per > maxst ? maxst : per);
  const int ch = bn < 128 ? bn : 128;
  const int rpo = (128 + splits - 1) / splits;
  const int stg = splits * rpo * (ch + 4) * 4;
  const int post = direct ? 0 : ((stg * (splits > 1 ? 2 : 1) + 1023) & ~1023) + (prefetch ? rpo * ch * 4 : 0);
  int reg = st * stage > post ? st * stage : post;
  reg = (reg + 1023) & ~1023;
  *stages = st;
  *region = reg;
  *smem = 1024 + (size_t)reg + 8 * (2 * 8 + 3) + 64;
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
  gemm_smem_layout(bn, K, splits, false, &st, &reg, &smem);
  const auto key = std::make_tuple(dev, bn, splits, (int)smem);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  int n = 0;
  KernelFn kern = pick_kernel(bn, B_K_BLOCKED, EPI_F16);
  cudaFuncSetAttribute(reinterpret_cast<const void*>(kern), cudaFuncAttributeMaxDynamicSharedMemorySize,
                       (int)kMaxDynSmem);
  cudaFuncSetAttribute(reinterpret_cast<const void*>(kern), cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
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
  cudaError_t e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
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
  // per-CTA time.  A CTA streams its k-blocks (A 16 KB + B bn*128 B each) at
  // ~100 GB/s and pays ~2.5 us of prologue / first-tile latency, ~0.9 us per
  // cluster barrier and a per-chunk exchange.  Weight-streaming GEMMs
  // (M <= 128) therefore spread over the SMs with wide tiles; large-M GEMMs
  // keep splits low.
  const int KB = (K + 63) / 64;
  double best = 1e300;
  int bb = 128, bs = 1;
  const int mt = (M + 127) / 128;
  for (int bn : {64, 128, 256}) {
    const int nt = (N + bn - 1) / bn;
    if (bn > 64 && N <= bn / 2) continue;
    const int nch = bn / (bn < 128 ? bn : 128);
    for (int s = 1; s <= kMaxSplits && s <= KB; ++s) {
      int st_, reg_;
      size_t smem_;
      gemm_smem_layout(bn, K, s, false, &st_, &reg_, &smem_);
      if (smem_ > kMaxDynSmem) continue;
      const long long clusters = (long long)mt * nt * G;
      const int maxc = max_active_clusters(bn, K, s);
      const long long waves = (clusters + maxc - 1) / maxc;
      const double kbs = (double)((KB + s - 1) / s);
      const double post = nch * (0.6 + (s > 1 ? 1.0 + 0.9 : 0.0) + 1.5 * 128.0 / s / 32.0);
      const double t = waves * (kbs * (16384.0 + 128.0 * bn) / 100e3 + 2.5 + post);
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
              long long b_gs, int M, int N, int K, int G, int b_mode, int bn, int splits, const GemmParams& epi) {
  const bool b_mn = b_mode == B_MN_MAJOR;
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
  if (!(bn == 64 || bn == 128 || bn == 256) || splits < 1 || splits > kMaxSplits || splits > (K + 63) / 64) {
    set_last_error("gemm_plan: unsupported tiling bn=%d splits=%d", bn, splits);
    return -2;
  }
  if (!pick_kernel(bn, b_mode, epi.epi)) {
    set_last_error("gemm_plan: no kernel for b_mode %d with epilogue %d", b_mode, epi.epi);
    return -2;
  }
  memset(g, 0, sizeof(*g));
  g->p = epi;
  g->p.M = M;
  g->p.N = N;
  g->p.K = K;
  g->p.splits = splits;
  g->bn = bn;
  g->b_mode = b_mode;
  g->pdl = false;
  // Residual / C rows are prefetched into shared memory (one TMA tile per
  // chunk) when the output is a 16-byte-aligned f32 matrix.
  const int ch = bn < 128 ? bn : 128;
  const int rpo = (128 + splits - 1) / splits;
  // Unsplit f16 tiles whose output rows take whole 16-column, 16-byte aligned
  // segments write straight from the TMEM registers (no staging).
  {
    // (f16 outputs only: a residual read row by row costs more than the
    // staged epilogue's TMA prefetch of it)
    g->p.direct = splits == 1 && epi.epi == EPI_F16 && !epi.out32 && (N % 16) == 0 &&
                  (epi.ldo % 8) == 0 && (epi.out_gstride % 8) == 0 &&
                  (reinterpret_cast<uintptr_t>(epi.out) % 16) == 0 &&
                  (!epi.bias || ((reinterpret_cast<uintptr_t>(epi.bias) % 16) == 0 && (epi.bias_gstride % 4) == 0));
  }
  bool pf = !g->p.direct && (epi.epi == EPI_RESID || epi.epi == EPI_F32_ACCUM) && (epi.ldo % 4) == 0 &&
            (N % 4) == 0 && (reinterpret_cast<uintptr_t>(epi.out) % 16) == 0 && (epi.out_gstride % 4) == 0;
  gemm_smem_layout(bn, K, splits, pf, &g->p.stages, &g->p.region, &g->smem, g->p.direct != 0);
  if (pf && g->smem > kMaxDynSmem) {
    pf = false;
    gemm_smem_layout(bn, K, splits, pf, &g->p.stages, &g->p.region, &g->smem);
  }
  if (g->smem > kMaxDynSmem) {
    set_last_error("gemm_plan: bn=%d splits=%d needs %zu bytes of shared memory", bn, splits, g->smem);
    return -2;
  }
  g->grid = dim3((N + bn - 1) / bn, (M + 127) / 128, G * splits);
  {
    const uint64_t d[3] = {(uint64_t)K, (uint64_t)M, (uint64_t)G};
    const uint64_t s[2] = {(uint64_t)lda * 2, (uint64_t)(G > 1 ? a_gs : lda * M) * 2};
    const uint32_t b[3] = {64, 128, 1};
    int r = encode(&g->ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, A, d, s, b, CU_TENSOR_MAP_SWIZZLE_128B);
    if (r) return r;
  }
  const long long KB = (K + 63) / 64;
  if (b_mode == B_K_MAJOR) {
    const uint64_t d[3] = {(uint64_t)K, (uint64_t)N, (uint64_t)G};
    const uint64_t s[2] = {(uint64_t)ldb * 2, (uint64_t)(G > 1 ? b_gs : ldb * N) * 2};
    const uint32_t b[3] = {64, (uint32_t)bn, 1};
    int r = encode(&g->tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, B, d, s, b, CU_TENSOR_MAP_SWIZZLE_128B);
    if (r) return r;
  } else if (b_mode == B_MN_MAJOR) {
    const uint64_t d[3] = {(uint64_t)N, (uint64_t)K, (uint64_t)G};
    const uint64_t s[2] = {(uint64_t)ldb * 2, (uint64_t)(G > 1 ? b_gs : ldb * K) * 2};
    const uint32_t b[3] = {64, 64, 1};
    int r = encode(&g->tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, B, d, s, b, CU_TENSOR_MAP_SWIZZLE_128B);
    if (r) return r;
  } else {  // k-blocked [G][KB][N][64]: every box is one contiguous run of bn*128 bytes
    const uint64_t d[4] = {64, (uint64_t)N, (uint64_t)KB, (uint64_t)G};
    const uint64_t s[3] = {128, (uint64_t)N * 128, (uint64_t)(G > 1 ? b_gs * 2 : KB * N * 128)};
    const uint32_t b[4] = {64, (uint32_t)bn, 1, 1};
    int r = encode(&g->tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, B, d, s, b, CU_TENSOR_MAP_SWIZZLE_128B);
    if (r) return r;
  }
  g->p.prefetch = pf ? 1 : 0;
  if (pf) {  // f32 output rows, one [rpo][ch] box per chunk, no swizzle
    const uint64_t d[3] = {(uint64_t)N, (uint64_t)M, (uint64_t)G};
    const uint64_t s[2] = {(uint64_t)epi.ldo * 4, (uint64_t)(G > 1 ? epi.out_gstride : epi.ldo * M) * 4};
    const uint32_t b[3] = {(uint32_t)ch, (uint32_t)rpo, 1};
    int r = encode(&g->tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, epi.out, d, s, b, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (r) return r;
  } else {
    g->tx = g->ta;  // unused
  }
  return 0;
}

int gemm_launch(const GemmPlan& g, cudaStream_t stream) { return launch_plan(g, stream); }

int device_error_read_and_clear(cudaStream_t stream, int* code) {
  int v = 0, z = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_cn_dev_error, sizeof(int), 0, cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaMemcpyToSymbolAsync(g_cn_dev_error, &z, sizeof(int), 0, cudaMemcpyHostToDevice, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  *code = v;
  return (int)e;
}

}  // namespace cn
