// On-device output decode: the reference's host-side Parser
// (parse_model_outputs.py:1-120) applied to the raw frame output on the GPU.
//
// A decode layout is a list of fields of one frame's raw vector:
//   MDN     (Parser.parse_mdn, :42-87): max(in_n, 1) hypothesis rows, each
//           [mu n | log-std n | ... | out_n selection logits], n =
//           (row - out_n) / 2; std = safe_exp(log-std).  With in_n > 1 the
//           selection logits are softmaxed across hypotheses; for out_n == 1
//           the hypotheses are reordered by weight, descending; every output
//           column takes the hypothesis of largest weight.  Decoded order:
//           [weights in_n x out_n | mu in_n x n | std in_n x n] (in_n > 1
//           only), then [mu | std] of the selected hypothesis per column.
//   SIGMOID (parse_binary_crossentropy, :35-40): 1 / (1 + safe_exp(-x)).
//   SOFTMAX (parse_categorical_crossentropy, :27-33): softmax over
//           consecutive groups of `width` values.
// safe_exp(x) = exp(min(x, 11)) (:4-6).  Ties follow numpy's stable argsort
// followed by [::-1]: the reordering ranks the higher index first, and the
// selection takes the later position in output order.
// One CTA per (field, frame); a layout has at most kMaxDecodeFields fields
// and MDN fields at most kMaxHyp hypotheses and kMaxSel selection columns.
#include <cstring>

#include "../../include/chestnut.h"
#include "cn_common.cuh"
#include "cn_gemm.cuh"

namespace cn {
namespace {

constexpr int kMaxDecodeFields = 32;
constexpr int kMaxHyp = 64;
constexpr int kMaxSel = 8;
constexpr int kDecThreads = 128;

struct DecodeLayout {
  cn_decode_field f[kMaxDecodeFields];
  int n;
};

__device__ __forceinline__ float safe_exp(float x) { return expf(fminf(x, 11.0f)); }

// Decoded values of one field per frame.
__host__ __device__ inline int field_out_len(const cn_decode_field& f) {
  if (f.kind != CN_DECODE_MDN) return f.raw_len;
  const int rows = f.in_n > 1 ? f.in_n : 1;
  const int n = (f.raw_len / rows - f.out_n) / 2;
  if (f.in_n > 1) return f.in_n * f.out_n + 2 * f.in_n * n + 2 * f.out_n * n;
  return 2 * n;
}

__global__ void __launch_bounds__(kDecThreads)
    k_decode(const float* __restrict__ raw, int raw_stride, const __grid_constant__ DecodeLayout L,
             float* __restrict__ out, int out_stride) {
  const cn_decode_field f = L.f[blockIdx.x];
  const float* x = raw + (size_t)blockIdx.y * raw_stride + f.raw_off;
  float* y = out + (size_t)blockIdx.y * out_stride + f.out_off;
  const int t = threadIdx.x;
  if (f.kind == CN_DECODE_SIGMOID) {
    for (int i = t; i < f.raw_len; i += kDecThreads) y[i] = 1.0f / (1.0f + safe_exp(-x[i]));
    return;
  }
  if (f.kind == CN_DECODE_SOFTMAX) {
    for (int g = t; g < f.raw_len / f.width; g += kDecThreads) {
      const float* xg = x + g * f.width;
      float m = xg[0];
      for (int i = 1; i < f.width; ++i) m = fmaxf(m, xg[i]);
      float s = 0.f;
      for (int i = 0; i < f.width; ++i) s += safe_exp(xg[i] - m);
      for (int i = 0; i < f.width; ++i) y[g * f.width + i] = safe_exp(xg[i] - m) / s;
    }
    return;
  }
  // MDN
  const int rows = f.in_n > 1 ? f.in_n : 1;
  const int row = f.raw_len / rows;
  const int n = (row - f.out_n) / 2;
  if (f.in_n <= 1) {
    for (int i = t; i < n; i += kDecThreads) {
      y[i] = x[i];
      y[n + i] = safe_exp(x[n + i]);
    }
    return;
  }
  __shared__ float w[kMaxHyp][kMaxSel];
  __shared__ int order[kMaxHyp];
  __shared__ int best[kMaxSel];
  const int H = f.in_n, S = f.out_n;
  if (t < S) {
    // softmax across hypotheses of selection column t (the row's last S values)
    const int c = row - S + t;
    float m = x[c];
    for (int h = 1; h < H; ++h) m = fmaxf(m, x[h * row + c]);
    float s = 0.f;
    for (int h = 0; h < H; ++h) s += safe_exp(x[h * row + c] - m);
    for (int h = 0; h < H; ++h) w[h][t] = safe_exp(x[h * row + c] - m) / s;
  }
  __syncthreads();
  if (t == 0) {
    // out_n == 1: hypotheses by weight, descending, ties -> higher index first
    for (int h = 0; h < H; ++h) order[h] = h;
    if (S == 1) {
      for (int i = 1; i < H; ++i) {
        const int v = order[i];
        int j = i - 1;
        while (j >= 0 && (w[order[j]][0] < w[v][0] || (w[order[j]][0] == w[v][0] && order[j] < v))) {
          order[j + 1] = order[j];
          --j;
        }
        order[j + 1] = v;
      }
    }
    for (int c = 0; c < S; ++c) {
      // position (in output order) of the largest weight; ties -> the later
      // position (argsort(...)[::-1][0] over the output-ordered weights)
      int b = 0;
      for (int p = 1; p < H; ++p)
        if (w[order[p]][c] >= w[order[b]][c]) b = p;
      best[c] = order[b];
    }
  }
  __syncthreads();
  float* yw = y;
  float* ym = yw + H * S;
  float* ys = ym + H * n;
  float* fm = ys + H * n;
  float* fs = fm + S * n;
  for (int i = t; i < H * S; i += kDecThreads) yw[i] = w[order[i / S]][i % S];
  for (int i = t; i < H * n; i += kDecThreads) {
    const int h = order[i / n], j = i % n;
    ym[i] = x[h * row + j];
    ys[i] = safe_exp(x[h * row + n + j]);
  }
  for (int i = t; i < S * n; i += kDecThreads) {
    const int h = best[i / n], j = i % n;
    fm[i] = x[h * row + j];
    fs[i] = safe_exp(x[h * row + n + j]);
  }
}

}  // namespace
}  // namespace cn

extern "C" int cn_decode_layout(cn_decode_field* fields, int n_fields, int* out_len) {
  using namespace cn;
  if (!fields || !out_len || n_fields < 1 || n_fields > kMaxDecodeFields) {
    set_last_error("cn_decode_layout: 1..%d fields required", kMaxDecodeFields);
    return -2;
  }
  int off = 0;
  for (int i = 0; i < n_fields; ++i) {
    cn_decode_field& f = fields[i];
    bool ok = f.raw_off >= 0 && f.raw_len > 0;
    if (f.kind == CN_DECODE_MDN) {
      const int rows = f.in_n > 1 ? f.in_n : 1;
      ok = ok && f.in_n >= 0 && f.out_n >= 0 && f.in_n <= kMaxHyp && f.out_n <= kMaxSel &&
           f.raw_len % rows == 0 && (f.raw_len / rows - f.out_n) >= 2 &&
           (f.in_n > 1 ? f.out_n >= 1 : f.out_n == 0);
    } else if (f.kind == CN_DECODE_SOFTMAX) {
      ok = ok && f.width > 0 && f.raw_len % f.width == 0;
    } else {
      ok = ok && f.kind == CN_DECODE_SIGMOID;
    }
    if (!ok) {
      set_last_error("cn_decode_layout: field %d (kind %d, raw %d+%d, in_n %d, out_n %d, width %d) is not decodable",
                     i, f.kind, f.raw_off, f.raw_len, f.in_n, f.out_n, f.width);
      return -2;
    }
    f.out_off = off;
    off += field_out_len(f);
  }
  *out_len = off;
  return 0;
}

extern "C" int cn_decode_outputs(const float* raw, int batch, int raw_stride, const cn_decode_field* fields,
                                 int n_fields, float* out, int out_stride, void* stream) {
  using namespace cn;
  if (!raw || !out || !fields || batch < 1 || n_fields < 1 || n_fields > kMaxDecodeFields) {
    set_last_error("cn_decode_outputs: bad arguments");
    return -2;
  }
  DecodeLayout L;
  memset(&L, 0, sizeof(L));
  memcpy(L.f, fields, sizeof(cn_decode_field) * n_fields);
  L.n = n_fields;
  int len = 0;
  if (cn_decode_layout(L.f, n_fields, &len)) return -2;
  for (int i = 0; i < n_fields; ++i)
    if (L.f[i].raw_off + L.f[i].raw_len > raw_stride || fields[i].out_off != L.f[i].out_off) {
      set_last_error("cn_decode_outputs: field %d lies outside the raw row or its out_off is not the layout's "
                     "(call cn_decode_layout first)", i);
      return -2;
    }
  if (len > out_stride) {
    set_last_error("cn_decode_outputs: decoded length %d exceeds out_stride %d", len, out_stride);
    return -2;
  }
  k_decode<<<dim3(n_fields, batch), kDecThreads, 0, static_cast<cudaStream_t>(stream)>>>(raw, raw_stride, L, out,
                                                                                         out_stride);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error("cn_decode_outputs: launch failed: %s", cudaGetErrorString(e));
    return -3;
  }
  return 0;
}
