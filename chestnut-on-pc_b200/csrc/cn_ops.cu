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

// grid (64, 2B + 1), block 128.  y < 2B: camera (b, cam) first-conv gather;
// y == 2B: cond vector + features_buffer for clip blockIdx.x.
__global__ void __launch_bounds__(128) k_gather0(Rings r, const float* __restrict__ packed, int B,
                                                 __half* __restrict__ a0, __half* __restrict__ cond16,
                                                 __half* __restrict__ feat16) {
  pdl_trigger();
  pdl_wait();
  const int c = *r.ctr;  // frames pushed before this one; this frame sits in slot c % 5
  if (blockIdx.y < 2 * B) {
    const int b = blockIdx.y >> 1, cam = blockIdx.y & 1;
    const int pos = blockIdx.x * 128 + threadIdx.x;  // 0..8191
    const int oy = pos >> 7, ox = pos & 127;
    const uint8_t* base = r.img + ((size_t)b * 2 + cam) * kImgQ * kFrameBytes;
    // sample_skip over the 5-row queue after the push: rows 0 (oldest) and 4 (newest)
    const uint8_t* f_old = base + (size_t)((c + 1) % kImgQ) * kFrameBytes;
    const uint8_t* f_new = base + (size_t)(c % kImgQ) * kFrameBytes;
    __align__(16) __half row[kK0Pad];
#pragma unroll
    for (int tap = 0; tap < 9; ++tap) {
      const int y = 2 * oy + tap / 3 - 1, x = 2 * ox + tap % 3 - 1;
      const bool valid = (unsigned)y < (unsigned)kH && (unsigned)x < (unsigned)kW;
      const int yc = min(max(y, 0), kH - 1), xc = min(max(x, 0), kW - 1);  // address stays in bounds
      const int off = yc * kW + xc;
#pragma unroll
      for (int ch = 0; ch < 12; ++ch) {
        const uint8_t* plane = (ch < 6 ? f_old + (size_t)ch * kH * kW : f_new + (size_t)(ch - 6) * kH * kW);
        const __half v = norm_u8(plane[off]);
        row[tap * 12 + ch] = valid ? v : __float2half_rn(0.0f);
      }
    }
#pragma unroll
    for (int k = kK0; k < kK0Pad; ++k) row[k] = __float2half_rn(0.0f);
    uint4* dst = reinterpret_cast<uint4*>(a0 + ((size_t)cam * B * 8192 + (size_t)b * 8192 + pos) * kK0Pad);
    const uint4* src = reinterpret_cast<const uint4*>(row);
#pragma unroll
    for (int q = 0; q < kK0Pad / 8; ++q) dst[q] = src[q];
  } else if ((int)blockIdx.x < B) {
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
    // features_buffer = feat_q[::4] after the push -> rows 0, 4, ..., 92
    for (int i = threadIdx.x; i < kNTemp * kFeat; i += blockDim.x) {
      const int j = i / kFeat, k = i % kFeat;
      const float v = r.feat[((size_t)b * kFeatQ + (c + 1 + kFS * j) % kFeatQ) * kFeat + k];
      feat16[((size_t)b * kNTemp + j) * kFeat + k] = __float2half_rn(v);
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
template <int NV>  // float4 per lane; d = NV * 128
__global__ void __launch_bounds__(256) k_layernorm(const float* __restrict__ x, __half* __restrict__ y, int rows,
                                                   int* bump) {
  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  if (bump && blockIdx.x == 0 && threadIdx.x == 0) atomicAdd(bump, 1);
  if (row >= rows) return;
  constexpr int d = NV * 128;
  const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * d);
  float4 v[NV];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    v[i] = xr[lane + 32 * i];
    s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / (float)d;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, e = v[i].w - mean;
    q += (a * a + b * b) + (c * c + e * e);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float rstd = 1.0f / sqrtf(q / (float)d + 1e-5f);
  uint2* yr = reinterpret_cast<uint2*>(y + (size_t)row * d);
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

// -------------------------------------------------------------- attention
// grid (clip*heads, ceil(T/8)); 8 warps, one query row each.
// smem: Kt[HD][kTP] f32 (keys transposed, lane j reads key j), V[kTP][HD+1]
// f32 (odd stride: conflict-free), q[8][HD] f32, P[8][kTP] f32.
constexpr int kTP = 96;
template <int HD>
__global__ void __launch_bounds__(256) k_attention(const __half* __restrict__ qkv, __half* __restrict__ out, int T,
                                                   int d, int heads) {
  extern __shared__ float sm[];
  pdl_trigger();
  pdl_wait();
  constexpr int VL = HD + 1;
  float* Kt = sm;
  float* V = Kt + HD * kTP;
  float* Q = V + kTP * VL;
  float* P = Q + 8 * HD;
  const int b = blockIdx.x / heads, h = blockIdx.x % heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t ld = 3 * (size_t)d;
  const __half* base = qkv + (size_t)b * T * ld + (size_t)h * HD;
  // stage K and V: consecutive threads take consecutive tokens of one 8-wide
  // column chunk, all loads of a thread issued before any store
  constexpr int NCH = kTP * (HD / 8);
  constexpr int PER = (NCH + 255) / 256;
  uint4 kv[PER], vv[PER];
#pragma unroll
  for (int it = 0; it < PER; ++it) {
    const int idx = threadIdx.x + it * 256;
    const int t = idx % kTP, c8 = (idx / kTP) * 8;
    kv[it] = make_uint4(0, 0, 0, 0);
    vv[it] = make_uint4(0, 0, 0, 0);
    if (idx < NCH && t < T) {
      kv[it] = *reinterpret_cast<const uint4*>(base + (size_t)t * ld + d + c8);
      vv[it] = *reinterpret_cast<const uint4*>(base + (size_t)t * ld + 2 * d + c8);
    }
  }
#pragma unroll
  for (int it = 0; it < PER; ++it) {
    const int idx = threadIdx.x + it * 256;
    if (idx >= NCH) continue;
    const int t = idx % kTP, c8 = (idx / kTP) * 8;
    const __half* kh = reinterpret_cast<const __half*>(&kv[it]);
    const __half* vh = reinterpret_cast<const __half*>(&vv[it]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      Kt[(c8 + j) * kTP + t] = __half2float(kh[j]);
      V[t * VL + c8 + j] = __half2float(vh[j]);
    }
  }
  __syncthreads();
  const int t = blockIdx.y * 8 + warp;
  if (t >= T) return;
  const float scale = 1.0f / sqrtf((float)HD);
  float* q = Q + warp * HD;
  float* p = P + warp * kTP;
  for (int i = lane; i < HD; i += 32) q[i] = __half2float(base[(size_t)t * ld + i]);
  __syncwarp();
  float s[3] = {0.f, 0.f, 0.f};
#pragma unroll 8
  for (int i = 0; i < HD; ++i) {
    const float qi = q[i];
#pragma unroll
    for (int u = 0; u < 3; ++u) s[u] = fmaf(qi, Kt[i * kTP + lane + 32 * u], s[u]);
  }
  float mx = -INFINITY;
#pragma unroll
  for (int u = 0; u < 3; ++u) {
    s[u] = (lane + 32 * u < T) ? s[u] * scale : -INFINITY;
    mx = fmaxf(mx, s[u]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float e[3], sum = 0.f;
#pragma unroll
  for (int u = 0; u < 3; ++u) {
    e[u] = (lane + 32 * u < T) ? expf(s[u] - mx) : 0.f;
    sum += e[u];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
#pragma unroll
  for (int u = 0; u < 3; ++u) p[lane + 32 * u] = e[u] / sum;
  __syncwarp();
  float acc[HD / 32];
#pragma unroll
  for (int i = 0; i < HD / 32; ++i) acc[i] = 0.f;
#pragma unroll 4
  for (int j = 0; j < T; ++j) {
    const float pj = p[j];
#pragma unroll
    for (int i = 0; i < HD / 32; ++i) acc[i] = fmaf(pj, V[j * VL + lane + 32 * i], acc[i]);
  }
  __half* o = out + ((size_t)b * T + t) * d + (size_t)h * HD;
#pragma unroll
  for (int i = 0; i < HD / 32; ++i) o[lane + 32 * i] = __float2half_rn(acc[i]);
}

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

}  // namespace

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
  const dim3 g((unsigned)((rows + 7) / 8));
  switch (d) {
    case 512: return (int)launch_ex(k_layernorm<4>, g, dim3(256), 0, s, pdl, x, y, rows, bump);
    case 1024: return (int)launch_ex(k_layernorm<8>, g, dim3(256), 0, s, pdl, x, y, rows, bump);
    case 2048: return (int)launch_ex(k_layernorm<16>, g, dim3(256), 0, s, pdl, x, y, rows, bump);
    default: return -2;
  }
}

int launch_attention(const __half* qkv, __half* out, int B, int T, int d, int heads, cudaStream_t s, bool pdl) {
  const int hd = d / heads;
  if (T > kTP || (hd != 64 && hd != 128)) return -2;
  const size_t smem = attention_smem_bytes(hd);
  static unsigned long long set64 = 0, set128 = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (hd == 64) {
    if (!(set64 & (1ull << dev))) {
      cudaFuncSetAttribute(k_attention<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      set64 |= 1ull << dev;
    }
    return (int)launch_ex(k_attention<64>, dim3(B * heads, (T + 7) / 8), dim3(256), smem, s, pdl, qkv, out, T, d, heads);
  }
  if (!(set128 & (1ull << dev))) {
    cudaFuncSetAttribute(k_attention<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    set128 |= 1ull << dev;
  }
  return (int)launch_ex(k_attention<128>, dim3(B * heads, (T + 7) / 8), dim3(256), smem, s, pdl, qkv, out, T, d,
                        heads);
}

size_t attention_smem_bytes(int hd) { return (size_t)(hd * kTP + kTP * (hd + 1) + 8 * hd + 8 * kTP) * sizeof(float); }

int launch_colmean(const __half* y, __half* pooled, int B, int T, int d, cudaStream_t s, bool pdl) {
  if (d % 256) return -2;
  return (int)launch_ex(k_colmean, dim3(B, d / 256), dim3(256), 0, s, pdl, y, pooled, T, d);
}

}  // namespace cn
