/* chestnut.h -- C ABI of the B200 chestnut frame engine (libchestnut.so).
 *
 * Every entry point returns 0 on success or a nonzero status; it never aborts
 * and never throws.  cn_last_error() returns a thread-local description of the
 * last failure.  Host pointers are owned by the caller; device buffers are
 * owned by the engine.  An engine is bound to one device and must be driven by
 * one host thread at a time (the reference's run_frame is likewise not
 * re-entrant: run_pinned2.py:1462-1463 uses module globals).
 *
 * Reference interfaces replaced (Alice7371/chestnut-on-pc):
 *   cn_engine_create   <- model load + recompile + queue allocation,
 *                         run_pinned2.py:1346-1389
 *   cn_run_frame       <- run_frame(warped_np, packed), run_pinned2.py:1462-1565
 *   cn_run_frames      <- the video_check.py:50-66 loop with hidden-state carry
 *   cn_get_state /
 *   cn_set_state       <- the module-level queues dict, run_pinned2.py:1379-1386
 *   cn_kernel_list     <- _LIN_BY_NAME / the recorded 497-launch plan,
 *                         run_pinned2.py:1092, :1472-1474
 *   cn_output_slices   <- meta['output_slices'], run_pinned2.py:1355
 *   cn_gemm_wmma_f16   <- the RDNA4 WMMA attention GEMM r_6_2_32_4_2_2_2_4_4_384
 *                         (run_pinned2.py:100-269; bench_r62.py:13-15)
 *   cn_reduce_rows_f16 <- the serial reduce r_32_32_3_12288_32 and its warp
 *                         split (run_pinned2.py:989-1066; bench_alu.py:13-16)
 *   cn_border_gather_s2<- the image2d zero-border read (run_pinned2.py:56-92,
 *                         :690-716)
 *   cn_warp_frames     <- the frame warp warp(tfm, big_tfm, frame, big_frame),
 *                         compile_modeld.py:179-191 (make_frame_prepare :95-118,
 *                         warp_perspective_tinygrad :53-81, frames_to_tensor
 *                         :84-93)
 *   cn_decode_outputs /
 *   cn_decode_frame    <- the host-side output parser Parser.parse_outputs
 *                         (parse_model_outputs.py:1-120: parse_mdn,
 *                         parse_binary_crossentropy,
 *                         parse_categorical_crossentropy), on the GPU
 */
#ifndef CHESTNUT_H
#define CHESTNUT_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CN_OK 0
#define CN_ERR_ARG (-2)
#define CN_ERR_CUDA (-3)
#define CN_ERR_DEVICE (-4)  /* a kernel recorded a device-side error (bounded wait expired) */
#define CN_ERR_STATE (-5)

#define CN_MODEL_39M 0
#define CN_MODEL_1B 1

#define CN_FRAME_BYTES (2 * 6 * 128 * 256)  /* warped u8[2,6,128,256] per clip */
#define CN_PACKED 524                      /* desire8 | tc2 | action_t2 | prev_feat512 */
#define CN_N_OUT 3323                      /* plan 2475 | lane_lines 264 | lead 72 | hidden_state 512 */

typedef struct cn_engine cn_engine;

typedef struct cn_config {
  int model;          /* CN_MODEL_39M or CN_MODEL_1B */
  int device;         /* CUDA device ordinal */
  int batch;          /* clips per launch (independent recurrent states) */
  int use_graph;      /* 1: replay the frame as one CUDA graph; 0: eager launches */
  int carry_hidden;   /* 1: feed hidden_state back on the device (packed[12:] ignored) */
  uint64_t seed;      /* weight seed (hash RNG), < 2^16 */
} cn_config;

typedef struct cn_kernel_info {
  char name[64];
  unsigned grid[3];
  unsigned block[3];
  unsigned cluster[3];
  unsigned smem_bytes;
} cn_kernel_info;

typedef struct cn_slice {
  char name[16];
  int start, stop;
} cn_slice;

const char* cn_last_error(void);
int cn_version(void);

/* ---- frame engine ---------------------------------------------------- */
int cn_engine_create(const cn_config* cfg, cn_engine** out);
int cn_engine_destroy(cn_engine* e);
/* warped: host u8 [batch][2][6][128][256]; packed: host f32 [batch][524];
 * out: host f32 [batch][CN_N_OUT] or NULL (the frame is then left in flight
 * and its output on the device; read it with cn_read_output). */
int cn_run_frame(cn_engine* e, const uint8_t* warped, const float* packed, float* out);
/* Double-buffered input (no counterpart in the reference, whose run_frame is
 * the only entry): cn_stage_input starts copying the next frame's warped
 * bytes (host u8 [batch][2][6][128][256]; pinned memory, or the copy is not
 * asynchronous) to the engine on a copy stream and returns at once;
 * cn_run_staged runs a frame, exactly as cn_run_frame would, on the oldest
 * staged input.  So the upload of frame f+1 overlaps the compute of frame f.
 * At most two inputs are staged ahead (CN_ERR_ARG beyond that, and for
 * cn_run_staged with nothing staged); the host buffer must stay unchanged
 * until the cn_run_staged call that consumes it returns. */
int cn_stage_input(cn_engine* e, const uint8_t* warped);
int cn_run_staged(cn_engine* e, const float* packed, float* out);
/* cn_run_staged without waiting: the frame and the copy of its output into
 * `out` (pinned host memory, B x CN_N_OUT f32) are queued and the call
 * returns; cn_wait_output waits for the oldest queued frame (at most two
 * queued) and reports a device-side error of that frame.  With the hidden
 * state carried on the device (cn_config.carry_hidden) nothing the host does
 * between frames depends on the previous output, so frame f+1 runs while the
 * host consumes frame f. */
int cn_run_staged_async(cn_engine* e, const float* packed, float* out);
int cn_wait_output(cn_engine* e);
/* n frames back to back with the hidden state carried by the caller's rule
 * packed[12:] = out[hidden_state] (video_check.py:60); outs: [n][batch][N_OUT]. */
int cn_run_frames(cn_engine* e, int n, const uint8_t* warped, const float* packed0, float* outs);
/* Same frame with inputs already resident on the device (d_warped, d_packed
 * device pointers in the layouts above); output stays on the device. */
int cn_run_frame_device(cn_engine* e, const void* d_warped, const void* d_packed);
int cn_read_output(cn_engine* e, float* out);
int cn_sync(cn_engine* e);
/* Canonical queue state of one clip: img_q u8[5,6,128,256] | big_img_q
 * u8[5,6,128,256] | feat_q f32[96,512] | desire_q f32[100,8] |
 * hidden f32[512] (the device-carried prev_feat). */
size_t cn_state_bytes(void);
int cn_get_state(cn_engine* e, int clip, void* buf, size_t bytes);
int cn_set_state(cn_engine* e, int clip, const void* buf, size_t bytes);
/* Zero every clip's queues, carried hidden state and frame counter (a new clip). */
int cn_reset_state(cn_engine* e);
int cn_kernel_list(cn_engine* e, cn_kernel_info* out, int* n_inout);
/* Eager run of one frame with an event pair around every launch; ms[i] is
 * the duration of kernel i of cn_kernel_list. */
int cn_profile_frame(cn_engine* e, const uint8_t* warped, const float* packed, float* ms, int* n_inout);
/* Per-launch durations of the marked kernel class inside the last graph
 * replay (see cn_set_timed_class); returns the count in *n. */
int cn_set_timed_class(cn_engine* e, const char* name_prefix);
int cn_timed_class_ms(cn_engine* e, float* ms, int* n_inout);
int cn_engine_info(cn_engine* e, long long* n_params, long long* weight_bytes, int* n_kernels);

/* ---- model description (host only, no GPU needed) ---------------------- */
int cn_output_slices(cn_slice* out, int* n_inout);
int cn_param_count(int model);
int cn_param_info(int model, int index, char* name, int name_len, int* tensor_id, long long* rows,
                  long long* cols, long long* valid_cols, int* kind);

/* ---- kernel-level entry points (device pointers, caller's stream) ------ */
/* C[M][N] += A[M][K] * B, f16 inputs, f32 accumulate (WMMA D = C + A*B).
 * b_kmajor: 1 -> B is [N][K]; 0 -> B is [K][N].  K % 8 == 0, 16-byte aligned
 * operands; bn in {64,128,256}, splits in [1,16] (<= K/64); bn / splits <= 0
 * choose a tiling automatically.  The tensor-map
 * plan of the last 16 distinct argument sets is cached, so repeated calls on
 * the same buffers cost one launch. */
int cn_gemm_wmma_f16(const void* A, const void* B, float* C, int M, int N, int K, int b_kmajor, int bn,
                     int splits, void* stream);
/* Same result as cn_gemm_wmma_f16 with b_kmajor = 1 (B is [N][K]), for callers
 * that cannot allocate device memory (a host whose GPU memory belongs to
 * another allocator, or a path where an allocation's implicit device
 * synchronisation is not allowed).  No counterpart in the reference.  The
 * split-K partial tiles and tile counters live in a 16 MiB static device array
 * that every GPU loading the library holds until exit; calls needing more
 * (splits x M x N rounded up to 128, x 4 bytes, plus 4 KiB of counters) or, with
 * splits > 1, more than 1024 output tiles are rejected with CN_ERR_ARG
 * (splits = 1 uses no scratch).  splits in [1, 16] and
 * <= ceil(K/64).  The first call on a device looks up the array's device
 * address, so make it before any stream capture.  All calls share the array:
 * calls that overlap on the GPU race. */
int cn_gemm_wmma_f16_noalloc(const void* A, const void* B, float* C, int M, int N, int K, int splits,
                             void* stream);
/* out[r] = sum_i x[r][i] * w[i]; x f16 [rows][len], w f16 [len]; f32 out.
 * chunks_per_row in {1,2,4,8} (0 = automatic). */
int cn_reduce_rows_f16(const void* x, const void* w, float* out, long long rows, long long len, int chunks_per_row,
                       void* stream);
/* 3x3 / stride-2 / pad-1 zero-border gather of NHWC f16 [G][B][H][W][C] into
 * f16 [G][B*(H/2)*(W/2)][9*C], k = tap*C + c; C % 8 == 0. */
int cn_border_gather_s2(const void* act, int G, int B, int H, int W, int C, void* out, void* stream);
/* Frame preparation: the road (frame) and wide (big_frame) NV12 camera frames,
 * device u8, each warped with its 3x3 inverse transform (host f32, row-major:
 * source = M . (x, y, 1)) into the model input u8 [2][6][model_h/2][model_w/2]
 * on the device (the `warped` layout of cn_run_frame: four 2x2 phases of the
 * warped Y plane, then U and V at half resolution).  Nearest-neighbour, round
 * half to even, clipped into the source (no border fill).  NV12 geometry:
 * stride bytes per row, y_height rows of Y, then uv_height rows of
 * interleaved UV.  width, height, model_h even; model_w % 8 == 0; out 4-byte
 * aligned. */
int cn_warp_frames(const uint8_t* frame, const uint8_t* big_frame, const float* tfm, const float* big_tfm, int width,
                   int height, int stride, int y_height, int uv_height, int model_w, int model_h, uint8_t* out,
                   void* stream);
/* ---- output decode (parse_model_outputs.py:1-120 on the GPU) ----------
 * A layout lists fields of one frame's raw output vector.  MDN
 * (Parser.parse_mdn): max(in_n,1) hypothesis rows [mu n | log-std n | ... |
 * out_n selection logits], std = exp(min(x, 11)); in_n > 1 needs out_n >= 1
 * (weights = softmax across hypotheses per selection column; out_n == 1
 * reorders the hypotheses by weight, descending), in_n <= 1 needs out_n == 0.
 * Decoded per MDN field: [weights in_n*out_n | mu in_n*n | std in_n*n] (in_n
 * > 1 only), then [mu | std] of the best hypothesis per column (max(out_n,1)
 * x n each).  SIGMOID: 1 / (1 + exp(min(-x, 11))).  SOFTMAX: softmax over
 * consecutive groups of `width` values.  At most 32 fields, 64 hypotheses and
 * 8 selection columns. */
#define CN_DECODE_MDN 0
#define CN_DECODE_SIGMOID 1
#define CN_DECODE_SOFTMAX 2
typedef struct cn_decode_field {
  int kind;              /* CN_DECODE_* */
  int raw_off, raw_len;  /* the field's values in one frame's raw vector */
  int in_n, out_n;       /* MDN: parse_mdn's in_N (hypotheses) and out_N (selection columns) */
  int width;             /* SOFTMAX: values per group */
  int out_off;           /* set by cn_decode_layout: first decoded value in one frame's output */
} cn_decode_field;
/* Checks a layout, sets every field's out_off and the decoded floats per frame. */
int cn_decode_layout(cn_decode_field* fields, int n_fields, int* out_len);
/* raw: device f32 [batch][raw_stride]; out: device f32 [batch][out_stride]
 * (fields as returned by cn_decode_layout). */
int cn_decode_outputs(const float* raw, int batch, int raw_stride, const cn_decode_field* fields, int n_fields,
                      float* out, int out_stride, void* stream);
/* Decode the engine's last frame output on its stream (after cn_run_frame /
 * cn_run_frame_device) and copy the decoded values to host f32
 * [batch][out_len], out_len from cn_decode_layout.  Synchronous. */
int cn_decode_frame(cn_engine* e, const cn_decode_field* fields, int n_fields, float* host_out);

/* Read (and clear) the device error word. */
int cn_device_error(int* code);
/* Failure-detection self-test: launches one CTA that waits on an mbarrier no
 * one arrives on.  The bounded wait gives up after `limit_ms`, records error
 * code 9 and the kernel returns; *code receives the device error word. */
int cn_selftest_bounded_wait(int limit_ms, int* code);

/* ---- plumbing for hosts without a CUDA binding (ctypes callers) ------- */
int cn_dev_alloc(void** ptr, size_t bytes, int device);
int cn_dev_free(void* ptr);
int cn_host_alloc_pinned(void** ptr, size_t bytes);
int cn_host_free_pinned(void* ptr);
/* kind: 0 host->device, 1 device->host, 2 device->device (synchronous) */
int cn_memcpy(void* dst, const void* src, size_t bytes, int kind);
int cn_memset(void* dst, int value, size_t bytes);
int cn_device_synchronize(int device);
int cn_engine_stream(cn_engine* e, void** stream);

#ifdef __cplusplus
}
#endif
#endif /* CHESTNUT_H */
