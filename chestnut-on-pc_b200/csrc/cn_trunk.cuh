// Persistent transformer trunk (host interface).  See cn_trunk.cu.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace cn {

// GEMM slots of one layer, in execution order.
enum TrunkGemm : int { TG_QKV = 0, TG_O = 1, TG_FC1 = 2, TG_FC2 = 3 };

struct TrunkMaps {
  CUtensorMap w[4];  // weights of all layers: [L][KB][N][64] f16, box 64 x 128 x 2 k-blocks
  CUtensorMap x[4];  // GEMM inputs [M][K] f16 as (64, M, K/64), box 64 x ntok x 2 (rows >= M zero-filled)
  CUtensorMap p[4];  // split-K partials [S][N/128][M][128] f32, box 128 x R x 1 x S
};

struct TrunkArgs {
  int M;          // token rows (clips x tokens), <= 128
  int ntok;       // MMA N: M rounded up to 16
  int T, B;       // tokens per clip, clips
  int d, mlp, heads, layers;
  int N[4], K[4], S[4], units[4];  // per GEMM slot: features, reduction, split-K, CTAs with work
  int R[4];                        // token rows per split-K reduction slice: ceil(M / S)
  int stages, stage_bytes, x_bytes;
  int aux_off, bar_off;            // shared-memory layout: ring at 0, then attention / reduction slices
  int phases;                      // grid barriers per launch (1: the closing one)
  float* x;                        // residual stream f32 [M][d]
  __half *h, *qkv, *att, *u;       // LN1 out [M][d], qkv [M][3d], attention out [M][d], MLP hidden [M][mlp]
  __half* h2;                      // LN2 out [M][d] (its own buffer: LN2 rows overlap QKV steps still reading h)
  __half* hf;                      // final LayerNorm out [M][d] (may be h: its last reader is done by then)
  __half* pooled;                  // token mean of hf per clip [B][d], f16 (null: not computed)
  // Tail products of a single-clip frame, after the pooling: hidden state
  // (tanh, f16 + an f32 copy into out), trunk head (relu, f16), heads (f32
  // into out).  Weights k-blocked [K/64][N][64]; tw[0] null: not computed.
  const __half* tw[3];
  const float* tb[3];
  int tN[3], tK[3];
  __half *hid16, *z;
  float* out;
  int out_hid;          // column of out where the f32 copy of the hidden state starts
  unsigned* tail_ctr;   // [3] CTAs done with: pooling, hidden state, trunk head
  float* part;                     // split-K partials, one [S][N/128][M][128] buffer per GEMM slot
  float* pslot[4];                 // the buffer of each slot
  unsigned* tile_ctr;              // [layers][4][64] split-K arrival counters
  unsigned* dep;                   // [layers][256] dataflow completion counters
  unsigned long long* grid_ctr;    // grid barrier arrivals (monotonic)
  unsigned* epoch;                 // completed launches
  int* bump;                       // frame counter incremented once per launch (or null)
  const float* bias[4];            // layer-0 biases; layer l at + l * bias_lstride
  long long bias_lstride;
};

struct TrunkPlan {
  TrunkMaps maps;
  TrunkArgs a;
  int grid;
  size_t smem;
  int hd;
};

// Scratch the trunk needs besides the activations: partial floats and the
// counter block (zeroed once; cn_reset_state zeroes it again).
size_t trunk_part_floats(int M, int d, int mlp, int layers, int nsm);
size_t trunk_counter_bytes(int layers);
bool trunk_supported(int M, int d, int heads);

int trunk_plan(TrunkPlan* tp, int B, int T, int d, int mlp, int heads, int layers, const void* const w0[4],
               long long w_lstride_bytes, const float* const b0[4], long long b_lstride, float* x, __half* h,
               __half* qkv, __half* att, __half* u, __half* h2, float* part, void* counters, int* bump, int nsm,
               __half* hf, __half* pooled);
int trunk_launch(const TrunkPlan& tp, cudaStream_t s);
// Adds the tail products to the launch (batch 1).  Returns false (and leaves
// the plan unchanged) if a shape is unsupported: K a multiple of 256, <= 2048.
bool trunk_set_tail(TrunkPlan* tp, const void* const w[3], const float* const b[3], const int N[3], const int K[3],
                    __half* hid16, __half* z, float* out, int out_hid);

}  // namespace cn
