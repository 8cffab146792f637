// Frame-path element / gather / normalisation kernels (host launchers).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace cn {

// Image geometry of the frame contract (run_pinned2.py:1377, ish['img']).
constexpr int kH = 128, kW = 256, kCH = 6, kImgQ = 5, kFS = 4;
constexpr int kFeat = 512, kFeatQ = 96, kNTemp = 24;
constexpr int kDesire = 8, kDesireQ = 100, kNDesire = 25;
constexpr int kPacked = 524, kCond = 204, kCondPad = 256;
constexpr int kT = 88, kNVisCam = 32, kNVis = 64;
constexpr int kK0 = 108, kK0Pad = 128;
constexpr int kTrunk = 1024, kNHeadsOut = 2811, kNOut = 3323;
constexpr size_t kFrameBytes = (size_t)kCH * kH * kW;        // one camera frame, 196,608 B
constexpr size_t kWarpedBytes = 2 * kFrameBytes;             // warped u8[2,6,128,256]

struct Rings {
  uint8_t* img;      // [B][2 cams][5 slots][6][128][256]
  float* feat;       // [B][96][512]
  float* desire;     // [B][100][8]
  int* ctr;          // frames pushed so far (shared by all clips)
};

int launch_fill_f16(__half* dst, long long rows, long long cols, long long valid_cols, uint64_t seed, uint64_t tid,
                    float bound, cudaStream_t s);
int launch_fill_f16_blocked(__half* dst, long long rows, long long cols, long long valid_cols, uint64_t seed,
                            uint64_t tid, float bound, cudaStream_t s);
int launch_fill_f32(float* dst, long long count, uint64_t seed, uint64_t tid, float bound, cudaStream_t s);

// Queue push (compile_modeld.py:199-213): frame -> img rings, desire and
// prev_feat -> their rings.  prev_feat comes from packed[12:] or, with
// carry != nullptr, from the previous frame's hidden_state output.
int launch_push(const uint8_t* warped, const float* packed, const float* carry, long long carry_ld, Rings r, int B,
                cudaStream_t s, bool pdl = false);
// First conv's zero-border im2col from the sampled u8 frames + the cond
// vector and the f16 features_buffer.  a0: [2][B*8192][128] f16.
int launch_gather0(Rings r, const float* packed, int B, __half* a0, __half* cond16, __half* feat16, cudaStream_t s,
                   bool pdl = false);
// 3x3 / stride 2 / pad 1 zero-border im2col of NHWC f16 [G][B][Hin][Win][C].
int launch_gather_s2(const __half* act, int G, int B, int Hin, int Win, int C, __half* out, cudaStream_t s,
                     bool pdl = false);
// Row LayerNorm f32 [rows][d] -> f16; bump (optional) is incremented once.
int launch_layernorm(const float* x, __half* y, int rows, int d, int* bump, cudaStream_t s, bool pdl = false);
// Per (clip, head) attention over T tokens: qkv f16 [B*T][3d] -> out f16 [B*T][d].
int launch_attention(const __half* qkv, __half* out, int B, int T, int d, int heads, cudaStream_t s,
                     bool pdl = false);
// Mean over the T tokens of each clip of the final LayerNorm output -> f16 [B][d].
int launch_colmean(const __half* y, __half* pooled, int B, int T, int d, cudaStream_t s, bool pdl = false);
size_t attention_smem_bytes(int hd);

int launch_selftest_wait(unsigned long long limit_ns, cudaStream_t s);

int reduce_rows_launch(const void* x, const void* w, float* out, long long rows, long long len, int cpr,
                       cudaStream_t stream);

}  // namespace cn
