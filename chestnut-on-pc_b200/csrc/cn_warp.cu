// Frame preparation: NV12 camera frames -> the engine's 6-plane model input.
//
// The step before the frame path (compile_modeld.py:53-118 warp_perspective /
// frames_to_tensor / make_frame_prepare, :179-191 make_warp): for the road and
// the wide camera, every destination pixel (x, y) of the model image is mapped
// through the camera's 3x3 inverse transform, src = M_inv . (x, y, 1), read
// nearest-neighbour (round half to even, clipped into the source, no border
// fill) from the NV12 Y plane at model resolution and from the deinterleaved
// U / V planes at half resolution (transform scaled by [[1,1,.5],[1,1,.5],
// [2,2,1]]).  The warped Y is split into its four 2x2 phases and U, V are
// appended: out u8[2][6][model_h/2][model_w/2], the layout cn_run_frame takes.
//
// Float sequence (fixed, since the reference's code generator is absent):
// each product and sum rounded to f32 separately, left to right, no fused
// multiply-add; the division is a multiply by the correctly rounded f32
// reciprocal; a NaN coordinate clips to 0.  Every address is clipped into its
// plane, so no transform can make the kernel read outside the frame.
//
// One thread writes 4 consecutive bytes of one output row (one 32-bit store);
// the gathers are 1-byte read-only loads.  HBM traffic is the output plus the
// source sectors the transforms touch; a frame pair is latency-bound.
#include "cn_common.cuh"

namespace cn {

namespace {

struct WarpArgs {
  const uint8_t* frame[2];
  float m[2][9];    // Y transform per camera (row-major)
  float muv[2][9];  // U / V transform per camera
  int width, height, stride, uv_off;
  int out_w, out_h;  // output plane: model_w / 2 x model_h / 2
  uint8_t* out;
};

__device__ __forceinline__ int warp_index(const float* m, float x, float y, int w_src, int h_src, int* yi) {
  const float sx = __fadd_rn(__fadd_rn(__fmul_rn(m[0], x), __fmul_rn(m[1], y)), m[2]);
  const float sy = __fadd_rn(__fadd_rn(__fmul_rn(m[3], x), __fmul_rn(m[4], y)), m[5]);
  const float sw = __fadd_rn(__fadd_rn(__fmul_rn(m[6], x), __fmul_rn(m[7], y)), m[8]);
  const float r = __frcp_rn(sw);
  // fmaxf / fminf return the non-NaN operand: a NaN coordinate clips to 0
  const float xc = fminf(fmaxf(rintf(__fmul_rn(sx, r)), 0.0f), (float)(w_src - 1));
  const float yc = fminf(fmaxf(rintf(__fmul_rn(sy, r)), 0.0f), (float)(h_src - 1));
  *yi = (int)yc;
  return (int)xc;
}

// grid: (out_w / 4 * out_h / 256-ish blocks, 6 planes, 2 cameras)
__global__ void __launch_bounds__(256) k_warp_nv12(const __grid_constant__ WarpArgs a) {
  const int cam = blockIdx.z, p = blockIdx.y;
  const int q = blockIdx.x * blockDim.x + threadIdx.x;  // 4-byte group of the plane
  const int groups = a.out_w / 4;
  if (q >= groups * a.out_h) return;
  const int r = q / groups, c0 = (q % groups) * 4;
  const uint8_t* f = a.frame[cam];
  uint32_t word = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c = c0 + j;
    int xi, yi;
    uint8_t v;
    if (p < 4) {
      // Y phase p: model pixel (x, y) = (2c + p / 2, 2r + p % 2)
      xi = warp_index(a.m[cam], (float)(2 * c + (p >> 1)), (float)(2 * r + (p & 1)), a.width, a.height, &yi);
      v = __ldg(f + (size_t)yi * a.stride + xi);
    } else {
      // U (p = 4) / V (p = 5): even / odd bytes of the interleaved UV rows
      xi = warp_index(a.muv[cam], (float)c, (float)r, a.width / 2, a.height / 2, &yi);
      v = __ldg(f + a.uv_off + (size_t)yi * a.stride + 2 * xi + (p - 4));
    }
    word |= (uint32_t)v << (8 * j);
  }
  *reinterpret_cast<uint32_t*>(a.out + (((size_t)cam * 6 + p) * a.out_h + r) * a.out_w + c0) = word;
}

}  // namespace

}  // namespace cn

using namespace cn;

extern "C" int cn_warp_frames(const uint8_t* frame, const uint8_t* big_frame, const float* tfm, const float* big_tfm,
                              int width, int height, int stride, int y_height, int uv_height, int model_w,
                              int model_h, uint8_t* out, void* stream) {
  if (!frame || !big_frame || !tfm || !big_tfm || !out || width < 2 || height < 2 || (width % 2) || (height % 2) ||
      stride < width || y_height < height || uv_height < height / 2 || model_w < 8 || (model_w % 8) ||
      model_h < 2 || (model_h % 2) || (reinterpret_cast<uintptr_t>(out) & 3)) {
    set_last_error("cn_warp_frames: bad arguments");
    return CN_ERR_ARG;
  }
  WarpArgs a;
  a.frame[0] = frame;
  a.frame[1] = big_frame;
  static const float kUv[9] = {1.0f, 1.0f, 0.5f, 1.0f, 1.0f, 0.5f, 2.0f, 2.0f, 1.0f};
  for (int i = 0; i < 9; ++i) {
    a.m[0][i] = tfm[i];
    a.m[1][i] = big_tfm[i];
    a.muv[0][i] = tfm[i] * kUv[i];  // exact: powers of two
    a.muv[1][i] = big_tfm[i] * kUv[i];
  }
  a.width = width;
  a.height = height;
  a.stride = stride;
  a.uv_off = stride * y_height;
  a.out_w = model_w / 2;
  a.out_h = model_h / 2;
  a.out = out;
  const int groups = a.out_w / 4 * a.out_h;
  const dim3 grid((groups + 255) / 256, 6, 2);
  k_warp_nv12<<<grid, 256, 0, (cudaStream_t)stream>>>(a);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error("cn_warp_frames: launch failed: %s", cudaGetErrorString(e));
    return CN_ERR_CUDA;
  }
  return 0;
}
