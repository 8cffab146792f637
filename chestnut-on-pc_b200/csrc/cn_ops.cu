// Frame-path kernels other than the GEMM: weight init, queue push, the
// zero-border gathers that feed the conv GEMMs, LayerNorm, attention, pooling.
#include "cn_common.cuh"
#include "cn_ops.cuh"

namespace cn {

namespace {

inline unsigned blocks_for(long long n, int threads, long long cap = 148LL * 16) {
  long long b = (n + threads - 1) / threads;
  return (unsigned)(b < 1 ? 1 : (b > cap ? cap : b));
}

// ---------------------------------------------------------------- weights
__global__ void k_fill_f16(__half* dst, long long rows, long long cols, long long valid_cols, uint64_t seed,
                           uint64_t tid, float bound) {
  const long long n = rows * cols;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long c = i % cols;
    const float v = __fmul_rn(hash_uniform(seed, tid, (uint64_t)i), bound);
    dst[i] = c < valid_cols ? __float2half_rn(v) : __float2half_rn(0.0f);
  }
}

// Weights for the frame GEMMs in the k-blocked layout [ceil(cols/64)][rows][64];
// the hash index stays the logical row-major index r*cols + c.
__global__ void k_fill_f16_blocked(__half* dst, long long rows, long long cols, long long valid_cols, uint64_t seed,
                                   uint64_t tid, float bound) {
  const long long kb_n = (cols + 63) / 64;
  const long long n = kb_n * rows * 64;
  for (long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x; j < n; j += (long long)gridDim.x * blockDim.x) {
    const long long kb = j / (rows * 64);
    const long long r = (j / 64) % rows;
    const long long c = kb * 64 + (j % 64);
    float v = 0.0f;
    if (c < valid_cols) v = __fmul_rn(hash_uniform(seed, tid, (uint64_t)(r * cols + c)), bound);
    dst[j] = __float2half_rn(v);
  }
}

__global__ void k_fill_f32(float* dst, long long n, uint64_t seed, uint64_t tid, float bound) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    dst[i] = __fmul_rn(hash_uniform(seed, tid, (uint64_t)i), bound);
}

// ------------------------------------------------------------------ queues
// grid (ceil(2*frame/16/256), B).  Ring slot layout: img[b][cam][slot][6][128][256].
__global__ void k_push(const uint8_t* __restrict__ warped, const float* __restrict__ packed,
                       const float* __restrict__ carry, long long carry_ld, Rings r) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.y;
  const int c = *r.ctr;
  constexpr long long kVecPerCam = (long long)kFrameBytes / 16;
  const long long v = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (v < 2 * kVecPerCam) {
    const int cam = (int)(v / kVecPerCam);
    const long long o = v % kVecPerCam;
    const uint4* src = reinterpret_cast<const uint4*>(warped + ((size_t)b * 2 + cam) * kFrameBytes);
    uint4* dst = reinterpret_cast<uint4*>(r.img + (((size_t)b * 2 + cam) * kImgQ + (c % kImgQ)) * kFrameBytes);
    dst[o] = src[o];
  }
  if (blockIdx.x == 0) {
    const float* pk = packed + (size_t)b * kPacked;
    if (threadIdx.x < kDesire) r.desire[((size_t)b * kDesireQ + c % kDesireQ) * kDesire + threadIdx.x] = pk[threadIdx.x];
    const float* pf = carry ? carry + (size_t)b * carry_ld : pk + (kDesire + 2 + 2);
    float* fd = r.feat + ((size_t)b * kFeatQ + c % kFeatQ) * kFeat;
    for (int i = threadIdx.x; i < kFeat; i += blockDim.x) fd[i] = pf[i];
  }
}

__device__ __forceinline__ __half norm_u8(uint32_t u) {
  // (u - 128) / 64 is exact in f16 for u in [0, 255]
  return __float2half_rn(__fmul_rn(__int2float_rn((int)u - 128), 0.015625f));
}

// grid (64, 2B + 1), block 128.  y < 2B: camera (b, cam), output row oy =
// blockIdx.x: the three input rows 2oy-1..2oy+1 of the 12 sampled planes are
// staged in shared memory (coalesced), then thread ox builds its 128-wide
// im2col row.  Out-of-range texels read as 0 after normalisation (the image2d
// border rule); the address itself is clamped, so no read leaves the frame.
// y == 2B: cond vector + features_buffer for clip blockIdx.x.
__global__ void __launch_bounds__(128) k_gather0(Rings r, const float* __restrict__ packed, int B,
                                                 __half* __restrict__ a0, __half* __restrict__ cond16,
                                                 __half* __restrict__ feat16) {
  pdl_trigger();
  pdl_wait();
  __shared__ __align__(16) uint8_t rows_s[12][3][kW];
  const int c = *r.ctr;  // frames pushed before this one; this frame sits in slot c % 5
  if (blockIdx.y < 2 * B) {
    const int b = blockIdx.y >> 1, cam = blockIdx.y & 1;
    const int oy = blockIdx.x, ox = threadIdx.x;
    const uint8_t* base = r.img + ((size_t)b * 2 + cam) * kImgQ * kFrameBytes;
    // sample_skip over the 5-row queue after the push: rows 0 (oldest) and 4 (newest)
    const uint8_t* f_old = base + (size_t)((c + 1) % kImgQ) * kFrameBytes;
    const uint8_t* f_new = base + (size_t)(c % kImgQ) * kFrameBytes;
    for (int i = threadIdx.x; i < 12 * 3 * (kW / 16); i += 128) {
      const int ch = i / (3 * (kW / 16)), rr = (i / (kW / 16)) % 3, q = i % (kW / 16);
      const int y = min(max(2 * oy + rr - 1, 0), kH - 1);
      const uint8_t* plane = ch < 6 ? f_old + (size_t)ch * kH * kW : f_new + (size_t)(ch - 6) * kH * kW;
      *reinterpret_cast<uint4*>(&rows_s[ch][rr][q * 16]) = *reinterpret_cast<const uint4*>(plane + y * kW + q * 16);
    }
    __syncthreads();
    __align__(16) __half row[kK0Pad];
#pragma unroll
    for (int tap = 0; tap < 9; ++tap) {
      const int ky = tap / 3, kx = tap % 3;
      const int y = 2 * oy + ky - 1, x = 2 * ox + kx - 1;
      const bool valid = (unsigned)y < (unsigned)kH && (unsigned)x < (unsigned)kW;
      const int xc = min(max(x, 0), kW - 1);
#pragma unroll
      for (int ch = 0; ch < 12; ++ch) {
        const __half v = norm_u8(rows_s[ch][ky][xc]);
        row[tap * 12 + ch] = valid ? v : __float2half_rn(0.0f);
      }
    }
#pragma unroll
    for (int k = kK0; k < kK0Pad; ++k) row[k] = __float2half_rn(0.0f);
    uint4* dst = reinterpret_cast<uint4*>(a0 + ((size_t)cam * B * 8192 + (size_t)b * 8192 + oy * 128 + ox) * kK0Pad);
    const uint4* src = reinterpret_cast<const uint4*>(row);
#pragma unroll
    for (int q = 0; q < kK0Pad / 8; ++q) dst[q] = src[q];
  } else {
    // features_buffer = feat_q[::4] after the push -> rows 0, 4, ..., 92, spread
    // over every block of this grid row (one block alone took ~40 us)
    const int nthr = gridDim.x * blockDim.x, tid = blockIdx.x * blockDim.x + threadIdx.x;
    constexpr int kRow4 = kFeat / 4;
    for (int i = tid; i < B * kNTemp * kRow4; i += nthr) {
      const int b = i / (kNTemp * kRow4), j = (i / kRow4) % kNTemp, k4 = i % kRow4;
      const float4 v = *reinterpret_cast<const float4*>(
          r.feat + ((size_t)b * kFeatQ + (c + 1 + kFS * j) % kFeatQ) * kFeat + 4 * k4);
      __align__(8) __half h[4] = {__float2half_rn(v.x), __float2half_rn(v.y), __float2half_rn(v.z),
                                  __float2half_rn(v.w)};
      *reinterpret_cast<uint2*>(feat16 + ((size_t)b * kNTemp + j) * kFeat + 4 * k4) = *reinterpret_cast<uint2*>(h);
    }
    if ((int)blockIdx.x >= B) return;
    const int b = blockIdx.x;
    const float* pk = packed + (size_t)b * kPacked;
    // cond = desire_pulse (25x8, max over FS groups of the 100-row queue) | tc | action_t | zero pad
    for (int i = threadIdx.x; i < kCondPad; i += blockDim.x) {
      float v = 0.0f;
      if (i < kNDesire * kDesire) {
        const int j = i / kDesire, k = i % kDesire;
        const float* dq = r.desire + (size_t)b * kDesireQ * kDesire;
        float m = dq[((c + 1 + kFS * j) % kDesireQ) * kDesire + k];
#pragma unroll
        for (int q = 1; q < kFS; ++q) m = fmaxf(m, dq[((c + 1 + kFS * j + q) % kDesireQ) * kDesire + k]);
        v = m;
      } else if (i < kCond) {
        v = pk[kDesire + (i - kNDesire * kDesire)];  // traffic_convention then action_t
      }
      cond16[(size_t)b * kCondPad + i] = __float2half_rn(v);
    }
  }
}

// One thread per 16-byte output chunk.  act: [G][B][Hin][Win][C] NHWC f16.
__global__ void k_gather_s2(const __half* __restrict__ act, int G, int B, int Hin, int Win, int C,
                            __half* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int Ho = Hin >> 1, Wo = Win >> 1;
  const int C8 = C >> 3;
  const long long total = (long long)G * B * Ho * Wo * 9 * C8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int c8 = (int)(i % C8);
    const int tap = (int)((i / C8) % 9);
    const long long row = i / (9LL * C8);  // (g, b, oy, ox)
    const int ox = (int)(row % Wo), oy = (int)((row / Wo) % Ho);
    const long long img = row / ((long long)Ho * Wo);  // g * B + b
    const int y = 2 * oy + tap / 3 - 1, x = 2 * ox + tap % 3 - 1;
    const bool valid = (unsigned)y < (unsigned)Hin && (unsigned)x < (unsigned)Win;
    const int yc = min(max(y, 0), Hin - 1), xc = min(max(x, 0), Win - 1);
    const uint4 v = *reinterpret_cast<const uint4*>(act + ((img * Hin + yc) * Win + xc) * C + c8 * 8);
    const uint4 z = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(out + row * 9LL * C + tap * C + c8 * 8) = valid ? v : z;
  }
}

// ------------------------------------------------------------ layer norm
// One row (d = NV * 512) by 4 warps, warp q owning the q-th quarter; per-warp
// partial sums are combined in warp order, so the result is deterministic.
// part[4][2] is shared scratch of the 4 warps and sync() synchronises them.
// Rows with live == false take part in the synchronisation only.
// ln_vals normalises a row whose values the warps already hold: v[i] are
// features q * d / 4 + 4 * (lane + 32 * i) .. + 3 of the row.
template <int NV, typename Sync>
__device__ __forceinline__ void ln_vals(const float4 (&v)[NV], __half* __restrict__ y, int row, bool live, int q,
                                        int lane, float (*part)[2], Sync sync) {
  constexpr int d = NV * 512;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) part[q][0] = s;
  sync();
  const float mean = (((part[0][0] + part[1][0]) + part[2][0]) + part[3][0]) / (float)d;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, e = v[i].w - mean;
    ss += (a * a + b * b) + (c * c + e * e);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) part[q][1] = ss;
  sync();
  const float var = (((part[0][1] + part[1][1]) + part[2][1]) + part[3][1]) / (float)d;
  const float rstd = 1.0f / sqrtf(var + 1e-5f);
  if (!live) return;
  uint2* yr = reinterpret_cast<uint2*>(y + (size_t)row * d + q * (d / 4));
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    __half2 h0 = __floats2half2_rn((v[i].x - mean) * rstd, (v[i].y - mean) * rstd);
    __half2 h1 = __floats2half2_rn((v[i].z - mean) * rstd, (v[i].w - mean) * rstd);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&h0);
    u.y = *reinterpret_cast<uint32_t*>(&h1);
    yr[lane + 32 * i] = u;
  }
}

template <int NV, typename Sync>
__device__ __forceinline__ void ln_row(const float* __restrict__ x, __half* __restrict__ y, int row, bool live, int q,
                                       int lane, float (*part)[2], Sync sync) {
  constexpr int d = NV * 512;
  const float4* xr = reinterpret_cast<const float4*>(x + (size_t)(live ? row : 0) * d + q * (d / 4));
  float4 v[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i)
    v[i] = live ? __ldcg(xr + lane + 32 * i) : make_float4(0.f, 0.f, 0.f, 0.f);  // L2: rows written by other SMs
  ln_vals<NV>(v, y, row, live, q, lane, part, sync);
}

// 2 rows per 256-thread block.
template <int NV>
__global__ void __launch_bounds__(256) k_layernorm(const float* __restrict__ x, __half* __restrict__ y, int rows,
                                                   int* bump) {
  pdl_trigger();
  pdl_wait();
  __shared__ float part[2][4][2];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = warp >> 2, q = warp & 3;
  const int row = blockIdx.x * 2 + slot;
  if (bump && blockIdx.x == 0 && threadIdx.x == 0) atomicAdd(bump, 1);
  ln_row<NV>(x, y, row, row < rows, q, lane, part[slot], [] { __syncthreads(); });
}

constexpr int kTP = 96;  // max tokens per clip handled by the pooling kernels

// ------------------------------------------------------------------ pool
// Mean over the T tokens of each clip of the (already f16-rounded) final
// LayerNorm output y [B*T][d]; each thread owns one column and adds the rows
// in token order.  grid (B, d/256), 256 threads.
__global__ void __launch_bounds__(256) k_colmean(const __half* __restrict__ y, __half* __restrict__ pooled, int T,
                                                 int d) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x;
  const int i = blockIdx.y * 256 + threadIdx.x;
  const __half* yb = y + (size_t)b * T * d + i;
  float s = 0.f;
#pragma unroll 8
  for (int t = 0; t < T; ++t) s += __half2float(yb[(size_t)t * d]);
  pooled[(size_t)b * d + i] = __float2half_rn(s / (float)T);
}

// Failure-detection self-test: wait on a barrier nothing arrives on.
__global__ void k_selftest_wait(unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&bar, 0, 9, limit_ns);
}

}  // namespace

int launch_selftest_wait(unsigned long long limit_ns, cudaStream_t s) {
  k_selftest_wait<<<1, 32, 0, s>>>(limit_ns);
  return (int)cudaGetLastError();
}

int launch_fill_f16(__half* dst, long long rows, long long cols, long long valid_cols, uint64_t seed, uint64_t tid,
                    float bound, cudaStream_t s) {
  k_fill_f16<<<blocks_for(rows * cols, 256), 256, 0, s>>>(dst, rows, cols, valid_cols, seed, tid, bound);
  return (int)cudaGetLastError();
}

int launch_fill_f16_blocked(__half* dst, long long rows, long long cols, long long valid_cols, uint64_t seed,
                            uint64_t tid, float bound, cudaStream_t s) {
  k_fill_f16_blocked<<<blocks_for(((cols + 63) / 64) * 64 * rows, 256), 256, 0, s>>>(dst, rows, cols, valid_cols, seed,
                                                                                    tid, bound);
  return (int)cudaGetLastError();
}

int launch_fill_f32(float* dst, long long count, uint64_t seed, uint64_t tid, float bound, cudaStream_t s) {
  k_fill_f32<<<blocks_for(count, 256), 256, 0, s>>>(dst, count, seed, tid, bound);
  return (int)cudaGetLastError();
}

int launch_push(const uint8_t* warped, const float* packed, const float* carry, long long carry_ld, Rings r, int B,
                cudaStream_t s, bool pdl) {
  const long long vecs = 2LL * kFrameBytes / 16;
  return (int)launch_ex(k_push, dim3((unsigned)((vecs + 255) / 256), (unsigned)B), dim3(256), 0, s, pdl, warped, packed,
                        carry, carry_ld, r);
}

int launch_gather0(Rings r, const float* packed, int B, __half* a0, __half* cond16, __half* feat16, cudaStream_t s,
                   bool pdl) {
  return (int)launch_ex(k_gather0, dim3(64, 2 * B + 1), dim3(128), 0, s, pdl, r, packed, B, a0, cond16, feat16);
}

int launch_gather_s2(const __half* act, int G, int B, int Hin, int Win, int C, __half* out, cudaStream_t s, bool pdl) {
  if (C % 8) return -2;
  const long long total = (long long)G * B * (Hin / 2) * (Win / 2) * 9 * (C / 8);
  return (int)launch_ex(k_gather_s2, dim3(blocks_for(total, 256, 1LL << 20)), dim3(256), 0, s, pdl, act, G, B, Hin,
                        Win, C, out);
}

int launch_layernorm(const float* x, __half* y, int rows, int d, int* bump, cudaStream_t s, bool pdl) {
  const dim3 g((unsigned)((rows + 1) / 2));
  switch (d) {
    case 512: return (int)launch_ex(k_layernorm<1>, g, dim3(256), 0, s, pdl, x, y, rows, bump);
    case 1024: return (int)launch_ex(k_layernorm<2>, g, dim3(256), 0, s, pdl, x, y, rows, bump);
    case 2048: return (int)launch_ex(k_layernorm<4>, g, dim3(256), 0, s, pdl, x, y, rows, bump);
    default: return -2;
  }
}

int launch_colmean(const __half* y, __half* pooled, int B, int T, int d, cudaStream_t s, bool pdl) {
  if (d % 256) return -2;
  return (int)launch_ex(k_colmean, dim3(B, d / 256), dim3(256), 0, s, pdl, y, pooled, T, d);
}

}  // namespace cn
