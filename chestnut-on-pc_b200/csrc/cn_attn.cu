// Small-sequence attention on the tensor cores (mma.sync m16n8k16, f16 in,
// f32 accumulate).  The temporal transformer attends over T <= 96 tokens
// (64 vision + 24 temporal = 88), so one CTA holds a whole (clip, head):
// Q, K, V are staged once in shared memory, each of 6 warps owns 16 query
// rows, S = Q K^T and the softmax stay in registers, and O = P V reuses the S
// accumulator layout as the A fragment.  P is split into f16 hi + lo parts
// (P = hi + lo to ~2^-22) so P V keeps f32-level accuracy.
#include "cn_common.cuh"
#include "cn_ops.cuh"

namespace cn {

namespace {

constexpr int kAttnRows = 96;   // padded token count (keys and queries)
constexpr int kAttnWarps = 6;   // 16 query rows each

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// Stage K, V (all kAttnRows rows) and Q rows [q0, q0 + nq) of (clip b, head h)
// into shared memory (rows >= T zeroed); nthr threads starting at thread index
// tid take part.  The caller waits (cp_async_wait_all) and synchronises its
// thread group afterwards.
template <int HD>
__device__ __forceinline__ void attention_stage(const __half* __restrict__ qkv, __half* Qs, int T, int d, int b, int h,
                                                int q0, int nq, int tid, int nthr) {
  constexpr int LD = HD + 8;  // halves; +16 B per row spreads ldmatrix rows over the banks
  constexpr int CPR = HD / 8;  // 16-byte chunks per row
  const size_t ld = 3 * (size_t)d;
  const __half* base = qkv + (size_t)b * T * ld + (size_t)h * HD;
  const int nkv = 2 * kAttnRows * CPR;
  for (int i = tid; i < nkv + nq * CPR; i += nthr) {
    const int mat = i < nkv ? 1 + i / (kAttnRows * CPR) : 0;
    const int rem = i < nkv ? i % (kAttnRows * CPR) : i - nkv + q0 * CPR;
    const int r = rem / CPR, c = (rem % CPR) * 8;
    __half* dst = Qs + mat * kAttnRows * LD + r * LD + c;
    if (r < T)
      cp_async16(dst, base + (size_t)r * ld + (size_t)mat * d + c);
    else
      *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
  }
}

// One warp (wid in [0, 6)) computes query rows [16*wid, 16*wid+16) of the
// staged (clip b, head h) and stores the valid rows of out f16 [B*T][d].
template <int HD>
__device__ __forceinline__ void attention_rows(const __half* Qs, __half* __restrict__ out, int T, int d, int b, int h,
                                               int wid, int lane) {
  constexpr int LD = HD + 8;
  constexpr int NB = kAttnRows / 8;
  const __half* Ks = Qs + kAttnRows * LD;
  const __half* Vs = Ks + kAttnRows * LD;
  const int g = lane >> 2, t4 = lane & 3;
  const int r0 = wid * 16;
  // ---- S = Q K^T (16 rows x 96 keys per warp)
  float s[NB][4];
#pragma unroll
  for (int j = 0; j < NB; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
  for (int kk = 0; kk < HD; kk += 16) {
    uint32_t a[4];
    {
      const int i = lane >> 3;
      ldsm_x4(a, Qs + (r0 + (i & 1) * 8 + (lane & 7)) * LD + kk + (i >> 1) * 8);
    }
#pragma unroll
    for (int j = 0; j < NB; ++j) {
      uint32_t bb[2];
      ldsm_x2(bb, Ks + (8 * j + (lane & 7)) * LD + kk + ((lane >> 3) & 1) * 8);
      mma16816(s[j], a, bb[0], bb[1]);
    }
  }
  // ---- softmax over the valid keys (rows g and g+8 of this warp's block)
  const float scale = 1.0f / sqrtf((float)HD);
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int j = 0; j < NB; ++j)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const bool valid = 8 * j + 2 * t4 + e < T;
      s[j][e] = valid ? s[j][e] * scale : -INFINITY;
      s[j][2 + e] = valid ? s[j][2 + e] * scale : -INFINITY;
      mx0 = fmaxf(mx0, s[j][e]);
      mx1 = fmaxf(mx1, s[j][2 + e]);
    }
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
  }
  float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
  for (int j = 0; j < NB; ++j)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      s[j][e] = expf(s[j][e] - mx0);  // exp(-inf) = 0 for masked keys
      s[j][2 + e] = expf(s[j][2 + e] - mx1);
      sum0 += s[j][e];
      sum1 += s[j][2 + e];
    }
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    sum0 += __shfl_xor_sync(0xffffffffu, sum0, o);
    sum1 += __shfl_xor_sync(0xffffffffu, sum1, o);
  }
#pragma unroll
  for (int j = 0; j < NB; ++j) {
    s[j][0] /= sum0;
    s[j][1] /= sum0;
    s[j][2] /= sum1;
    s[j][3] /= sum1;
  }
  // ---- O = P V, P = hi + lo (two f16 passes)
  float o[HD / 8][4];
#pragma unroll
  for (int nb = 0; nb < HD / 8; ++nb) o[nb][0] = o[nb][1] = o[nb][2] = o[nb][3] = 0.f;
#pragma unroll
  for (int ks = 0; ks < kAttnRows / 16; ++ks) {
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
      ldsm_x4_t(bv, Vs + (16 * ks + (i & 1) * 8 + (lane & 7)) * LD + 8 * nb + (i >> 1) * 8);
      mma16816(o[nb], ahi, bv[0], bv[1]);
      mma16816(o[nb], alo, bv[0], bv[1]);
      mma16816(o[nb + 1], ahi, bv[2], bv[3]);
      mma16816(o[nb + 1], alo, bv[2], bv[3]);
    }
  }
  // ---- store the valid rows
  const int ra = r0 + g, rb = r0 + g + 8;
  __half* oa = out + ((size_t)b * T + ra) * d + (size_t)h * HD;
  __half* ob = out + ((size_t)b * T + rb) * d + (size_t)h * HD;
#pragma unroll
  for (int nb = 0; nb < HD / 8; ++nb) {
    const int col = 8 * nb + 2 * t4;
    if (ra < T) *reinterpret_cast<__half2*>(oa + col) = __floats2half2_rn(o[nb][0], o[nb][1]);
    if (rb < T) *reinterpret_cast<__half2*>(ob + col) = __floats2half2_rn(o[nb][2], o[nb][3]);
  }
}

// grid (clips * heads), 192 threads.  qkv f16 [B*T][3d] (q | k | v), out f16 [B*T][d].
template <int HD>
__global__ void __launch_bounds__(kAttnWarps * 32) k_attention_mma(const __half* __restrict__ qkv,
                                                                    __half* __restrict__ out, int T, int d,
                                                                    int heads) {
  extern __shared__ __align__(16) uint8_t attn_smem[];
  __half* Qs = reinterpret_cast<__half*>(attn_smem);
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x / heads, h = blockIdx.x % heads;
  attention_stage<HD>(qkv, Qs, T, d, b, h, 0, kAttnRows, threadIdx.x, kAttnWarps * 32);
  cp_async_wait_all();
  __syncthreads();
  attention_rows<HD>(Qs, out, T, d, b, h, threadIdx.x >> 5, threadIdx.x & 31);
}

}  // namespace

size_t attention_smem_bytes(int hd) { return (size_t)3 * kAttnRows * (hd + 8) * sizeof(__half); }

int launch_attention(const __half* qkv, __half* out, int B, int T, int d, int heads, cudaStream_t s, bool pdl) {
  const int hd = d / heads;
  if (T > kAttnRows || (hd != 64 && hd != 128)) return -2;
  const size_t smem = attention_smem_bytes(hd);
  static unsigned long long set64 = 0, set128 = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (hd == 64) {
    if (!(set64 & (1ull << dev))) {
      cudaFuncSetAttribute(k_attention_mma<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      set64 |= 1ull << dev;
    }
    return (int)launch_ex(k_attention_mma<64>, dim3(B * heads), dim3(kAttnWarps * 32), smem, s, pdl, qkv, out, T, d,
                          heads);
  }
  if (!(set128 & (1ull << dev))) {
    cudaFuncSetAttribute(k_attention_mma<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    set128 |= 1ull << dev;
  }
  return (int)launch_ex(k_attention_mma<128>, dim3(B * heads), dim3(kAttnWarps * 32), smem, s, pdl, qkv, out, T, d,
                        heads);
}

}  // namespace cn
