// tcgen05 GEMM: host-side plan / launch interface.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

namespace cn {

enum Epi : int {
  EPI_F32_ACCUM = 0,  // C[m][n] += acc                       (WMMA semantics D = C + A*B)
  EPI_F16 = 1,        // out16[m][n] = f16(act(acc + bias[n]))  (+ optional f32 copy)
  EPI_RESID = 2,      // x32[m][n] += acc + bias[n]
  EPI_TOKENS = 3,     // x32[row(m)][n] = ((acc + bias[n]) + pos[t][n]) + cond[clip][n]
  EPI_F32_OUT = 4,    // out32[m][n] = acc + bias[n]
};
enum Act : int { ACT_NONE = 0, ACT_RELU = 1, ACT_GELU = 2, ACT_TANH = 3 };
// Layouts of the B operand: row-major [N][K] (K contiguous), [K][N], or the
// engine's k-blocked weight layout [KB][N][64] (one 64-wide k-block of every
// row stored contiguously, so a weight tile is a single contiguous HBM run).
enum BMode : int { B_K_MAJOR = 0, B_MN_MAJOR = 1, B_K_BLOCKED = 2 };

struct GemmParams {
  int M, N, K;        // per group; K % 8 == 0 (partial 64-wide k-blocks are zero-filled)
  int splits;         // split-K factor == cluster size along z
  int stages;         // pipeline depth (host-chosen, <= 8)
  int region;         // bytes of the pipeline / receive region before the barriers
  int prefetch;       // 1: residual / C rows are bulk-copied into shared memory
  int epi, act;
  void* out;          // f16 (EPI_F16) or f32 base
  long long ldo;      // out row stride (elements)
  long long out_gstride;  // elements between groups
  const float* bias;  // [G][N] (group stride = bias_gstride) or nullptr
  long long bias_gstride;
  float* out32;       // EPI_F16: optional f32 copy of the rounded value
  long long ld32;
  // EPI_TOKENS row mapping: GEMM row m of group g -> clip = m / rows_per_clip,
  // token t = tok_base + g * tok_gstride + m % rows_per_clip,
  // residual row = clip * T + t.
  const float* pos;   // [T][N]
  const float* cond;  // [clips][cond_ld]
  long long cond_ld;
  int rows_per_clip, tok_base, tok_gstride, T;
  int b_dep;          // 1: B may be written by an earlier kernel, so it is loaded only after griddepcontrol.wait
  int direct;         // set by gemm_plan: unsplit tile, epilogue straight from the TMEM registers
};

struct GemmPlan {
  CUtensorMap ta, tb, tx;  // A, B, and (prefetch only) the f32 output rows
  GemmParams p;
  dim3 grid;
  int bn;
  int b_mode;
  bool pdl;  // launch with programmatic stream serialization (frame graph only)
  size_t smem;
};

// A: [G][M][K] f16, row stride lda (elements), group stride a_gs (elements).
// B: per b_mode, K-major [G][N][K] (row stride ldb), MN-major [G][K][N]
// (row stride ldb), or k-blocked [G][ceil(K/64)][N][64] (ldb unused).
// bn/splits <= 0 pick a tiling automatically.  Returns 0 or a cudaError_t /
// CUresult code (also recorded in the engine's last-error string).
int gemm_plan(GemmPlan* g, const void* A, long long lda, long long a_gs, const void* B, long long ldb,
              long long b_gs, int M, int N, int K, int G, int b_mode, int bn, int splits, const GemmParams& epi);
int gemm_launch(const GemmPlan& g, cudaStream_t stream);
int gemm_choose(int M, int N, int K, int G, int* bn, int* splits);

int device_error_read_and_clear(cudaStream_t stream, int* code);
const char* last_error_text();
void set_last_error(const char* fmt, ...);

}  // namespace cn
