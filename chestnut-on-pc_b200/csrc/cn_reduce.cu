// HBM-streaming row reduction for the r_32_32_3_12288_32 shape (config 2).
//
// Reference: run_pinned2.py:989-1066 (_warp_split_ptx) and alu_opt.py:1-117 --
// out[32*32*3] = sum_{i<12288, j<32} x[.., i, j] * w[i, j], one warp per
// output group on sm_75 (6.8 ms), split over 4 warps + shared reduce (2.1 ms).
// Flattened, each output row r is a dot product of x[r, :] (393,216 f16,
// contiguous) with the shared vector w (same length, L2-resident).
//
// B200 design: a cluster of CPR CTAs owns one row; CTA c of the cluster
// streams the c-th contiguous chunk with 16-byte non-allocating loads (four
// loads in flight per thread), reduces through warp shuffles and a fixed
// shared-memory tree, and CTA 0 sums the CPR partials over DSMEM in rank order.
// The result is bitwise deterministic and needs no global workspace.
#include "cn_common.cuh"

namespace cn {

namespace {
constexpr int kRedThreads = 256;

__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ float dot8(const uint4& a, const uint4& b, float acc) {
  const __half2* ha = reinterpret_cast<const __half2*>(&a);
  const __half2* hb = reinterpret_cast<const __half2*>(&b);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float2 fa = __half22float2(ha[q]);
    const float2 fb = __half22float2(hb[q]);
    acc = fmaf(fa.x, fb.x, acc);
    acc = fmaf(fa.y, fb.y, acc);
  }
  return acc;
}

// grid (CPR, rows), cluster (CPR, 1, 1).  len % 8 == 0.
template <int CPR>
__global__ void __launch_bounds__(kRedThreads)
    k_row_dot(const __half* __restrict__ x, const __half* __restrict__ w, float* __restrict__ out, long long len) {
  __shared__ float warp_part[kRedThreads / 32];
  __shared__ float cta_part;
  const int c = blockIdx.x;
  const long long row = blockIdx.y;
  const long long nv = len >> 3;  // 16-byte vectors per row
  const long long v0 = nv * c / CPR, v1 = nv * (c + 1) / CPR;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * len);
  const uint4* wv = reinterpret_cast<const uint4*>(w);

  float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
  long long i = v0 + threadIdx.x;
  for (; i + 3 * kRedThreads < v1; i += 4 * kRedThreads) {
    const uint4 a0 = ld_stream(xr + i);
    const uint4 a1 = ld_stream(xr + i + kRedThreads);
    const uint4 a2 = ld_stream(xr + i + 2 * kRedThreads);
    const uint4 a3 = ld_stream(xr + i + 3 * kRedThreads);
    acc0 = dot8(a0, __ldg(wv + i), acc0);
    acc1 = dot8(a1, __ldg(wv + i + kRedThreads), acc1);
    acc2 = dot8(a2, __ldg(wv + i + 2 * kRedThreads), acc2);
    acc3 = dot8(a3, __ldg(wv + i + 3 * kRedThreads), acc3);
  }
  for (; i < v1; i += kRedThreads) acc0 = dot8(ld_stream(xr + i), __ldg(wv + i), acc0);
  float acc = (acc0 + acc1) + (acc2 + acc3);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) warp_part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < kRedThreads / 32; ++q) s += warp_part[q];
    cta_part = s;
  }
  if constexpr (CPR > 1) {
    cluster_sync();
    if (c == 0 && threadIdx.x == 0) {
      const uint32_t a = smem_u32(&cta_part);
      float s = 0.f;
      for (int r = 0; r < CPR; ++r) {
        float t;
        asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(t) : "r"(map_shared_rank(a, (uint32_t)r)) : "memory");
        s += t;
      }
      out[row] = s;
    }
    cluster_sync();
  } else {
    if (threadIdx.x == 0) out[row] = cta_part;
  }
}
}  // namespace

int reduce_rows_launch(const void* x, const void* w, float* out, long long rows, long long len, int cpr,
                       cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)cpr, (unsigned)rows, 1);
  cfg.blockDim = dim3(kRedThreads);
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = (unsigned)cpr;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  const __half* xh = static_cast<const __half*>(x);
  const __half* wh = static_cast<const __half*>(w);
  cudaError_t e;
  switch (cpr) {
    case 1: e = cudaLaunchKernelEx(&cfg, k_row_dot<1>, xh, wh, out, len); break;
    case 2: e = cudaLaunchKernelEx(&cfg, k_row_dot<2>, xh, wh, out, len); break;
    case 4: e = cudaLaunchKernelEx(&cfg, k_row_dot<4>, xh, wh, out, len); break;
    case 8: e = cudaLaunchKernelEx(&cfg, k_row_dot<8>, xh, wh, out, len); break;
    default: return -2;
  }
  return (int)e;
}

}  // namespace cn
