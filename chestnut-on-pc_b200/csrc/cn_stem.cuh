// Persistent conv stem + token embeddings (host interface).  See cn_stem.cu.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace cn {

constexpr int kStemMaxPhases = 12;
constexpr int kStemMaxTiles = 64;  // feature tiles of a split-K phase (arrival counters)

enum StemA : int {
  SA_ROWS = 0,    // A[g][row][k] rows (row stride lda, group stride a_gs); k >= K reads zeros
  SA_GATHER = 1,  // 3x3 / stride 2 / pad 1 zero-border im2col of NHWC f16 [g][B][Hin][Win][Cin], k = tap * Cin + c
};
enum StemEpi : int {
  SE_RELU_F16 = 0,  // out16[g][row][n] = f16(relu(acc + bias[g][n]))
  SE_F32 = 1,       // out32[g][row][n] = acc + bias[g][n]
  SE_TOKENS = 2,    // x[clip * T + t][n] = ((acc + bias[g][n]) + pos[t][n]) + cond[clip][n]
};

// One GEMM of the stem as the engine describes it (the plan picks tiles and splits).
struct StemSpec {
  int G, Mg, N, K;  // groups (cameras), rows per group, output features, reduction length
  int akind;
  const __half* A;
  long long lda, a_gs;
  int Hin, Win, Cin;  // SA_GATHER geometry (rows per group = B * Hin/2 * Win/2)
  const void* W;      // k-blocked weights [G][ceil(K/64)][N][64] f16
  long long w_gs;     // bytes between groups
  int epi;
  void* out;
  long long ldo, o_gs;
  const float* bias;
  long long b_gs;
  const float* pos;  // SE_TOKENS: [T][N]
  const float* cond;  // SE_TOKENS: [clips][cond_ld]
  long long cond_ld;
  int rows_per_clip, tok_base, tok_gstride, T;
  // Optional fused 1x1 conv on this GEMM's ReLU output (N x N weights, same
  // rows): out1 = f16(relu(relu_out . W1^T + bias1)).  N <= 256.
  const void* W1;
  long long w1_gs;
  void* out1;
  long long ldo1, o1_gs;
  const float* bias1;
  long long b1_gs;
  int dep0, dep1;  // phases whose outputs this one reads (-1: none)
};

struct StemPhase {
  int G, Mg, N, K, KB, BN, S, tm, tn, units, cta0, rows_pad;
  int akind;
  const __half* A;
  long long lda, a_gs;
  int Hin, Win, Cin, Ho, Wo;
  int lHin, lWin, lCin, lHo, lWo;  // SA_GATHER: log2 of the (power-of-two) extents
  int kps, kps1;                   // weight k-blocks per ring stage (GEMM, fused 1x1)
  int dec;                         // 1: loads run ahead of the epilogue (it stages in Y only)
  int defer;                       // 1: a unit's fused 1x1 is issued after the next unit's GEMM
  int atma;                        // 1: activation k-blocks by TMA (else 16-byte cp.async)
  int abytes;                      // bytes one activation TMA box lands
  int B;                           // images per group (SA_GATHER)
  const uint8_t* w;
  long long w_gs;
  int epi;
  void* out;
  long long ldo, o_gs;
  const float* bias;
  long long b_gs;
  const float* pos;
  const float* cond;
  long long cond_ld;
  int rows_per_clip, tok_base, tok_gstride, T;
  int fuse, KB1;
  const uint8_t* w1;
  long long w1_gs;
  void* out1;
  long long ldo1, o1_gs;
  const float* bias1;
  long long b1_gs;
  float* part;  // split-K partials [G][tm][tn][S][BN][rows_pad] f32
  long long part_off;
  int dep0, dep1;
};

struct StemMaps {
  CUtensorMap w[kStemMaxPhases];   // box 64 x BN x (32 KB / (BN x 128)) k-blocks x 1 group
  CUtensorMap w1[kStemMaxPhases];  // fused 1x1 weights, box 64 x N x (32 KB / (N x 128)) x 1
  // Activations (atma phases).  SA_ROWS: (K, rows, G), box 64 x 128 x 1.
  // SA_GATHER: NHWC (Cin, Win, Hin, G x B) with traversal strides (1, 2, 2, 1),
  // box 64 x 2 Wo x 2 R x 1: the R x Wo output pixels of a tile for one tap.
  CUtensorMap x[kStemMaxPhases];
  // f16 outputs of whole-unit ReLU phases: (N, rows, G), box 64 x 128 x 1
  CUtensorMap o[kStemMaxPhases];
};

struct StemArgs {
  int nph;
  unsigned* pctr;   // [kStemMaxPhases] units done (monotonic across launches)
  unsigned* tctr;   // [kStemMaxPhases][kStemMaxTiles] split-K arrivals
  unsigned* epoch;  // completed launches
  unsigned* exits;  // CTAs finished (monotonic)
  StemPhase ph[kStemMaxPhases];
};

struct StemPlan {
  StemMaps maps;
  StemArgs a;
  int grid;
  size_t smem;
  long long part_floats;
  int next_cta;
};

size_t stem_counter_bytes();
void stem_plan_begin(StemPlan* sp, int nsm);
// Appends one phase; returns its index, or -1 (message in the last-error text).
int stem_add(StemPlan* sp, const StemSpec& s);
// Binds scratch (partials, counters) and encodes the weight tensor maps.
int stem_plan_end(StemPlan* sp, float* part, void* counters);
int stem_launch(const StemPlan& sp, cudaStream_t s);

}  // namespace cn
