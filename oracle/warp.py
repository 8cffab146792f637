"""NV12 frame warp -> 6-plane model input (oracle side, test infrastructure).

Restates the reference's frame preparation (``compile_modeld.py:53-118``
``warp_perspective_tinygrad`` / ``frames_to_tensor`` / ``make_frame_prepare``,
and ``:179-191`` ``make_warp``):

* every destination pixel (x, y) of the model image is mapped through the 3x3
  inverse transform ``M_inv``: src = M_inv . (x, y, 1), src_x / src_w,
  src_y / src_w; the source is read nearest-neighbour at the rounded
  coordinate (round half to even), clipped into the source image -- no
  border fill (``border_fill_val=None`` at every call site);
* Y is warped at the model resolution (W x H); U and V, deinterleaved from
  the NV12 UV plane (even / odd bytes of each UV row), at half resolution
  with ``M_inv * [[1, 1, .5], [1, 1, .5], [2, 2, 1]]`` (``compile_modeld.py:101``);
* ``frames_to_tensor`` splits the warped Y into its four 2x2 phases (rows
  even/odd x columns even/odd, in the order (0,0), (1,0), (0,1), (1,1)) and
  appends U and V: u8[6, H/2, W/2];
* ``make_warp`` does this for the road and the wide camera, each with its own
  transform: u8[2, 6, H/2, W/2], the engine's ``warped`` input.

Float arithmetic.  The reference builds these expressions in tinygrad, which
is absent here (and with it the pinned code generator), so its exact rounding
sequence cannot be reproduced by running it.  This restatement fixes one:
every product and sum is rounded to f32 separately, left to right
(``m0 * x + m1 * y + m2`` = ((m0*x) + (m1*y)) + m2, no fused multiply-add),
and the division is a multiply by the correctly rounded f32 reciprocal, the
form tinygrad lowers float division to.  A NaN coordinate (src_w = 0) clips
to 0.  The CUDA kernel follows the same sequence, so the two agree bit for
bit; agreement with the reference itself is unpinned.

NV12 geometry (``NV12Frame``, ``compile_modeld.py:39``): width, height,
stride (bytes per Y / UV row), y_height (rows of the Y plane in the buffer),
uv_height (rows of the UV plane); the UV plane starts at stride * y_height.
The reference computes stride / y_height / uv_height with openpilot's
``get_nv12_info`` (camerad, not part of this repository); callers here pass
them explicitly.
"""
import numpy as np

UV_SCALE = np.array([[1.0, 1.0, 0.5], [1.0, 1.0, 0.5], [2.0, 2.0, 1.0]], np.float32)


def _src_coords(M, w_dst, h_dst):
    """f32 source coordinates of every destination pixel, row-major (h, w)."""
    M = np.asarray(M, np.float32).reshape(3, 3)
    x = np.broadcast_to(np.arange(w_dst, dtype=np.float32)[None, :], (h_dst, w_dst))
    y = np.broadcast_to(np.arange(h_dst, dtype=np.float32)[:, None], (h_dst, w_dst))

    def row(i):
        return (M[i, 0] * x + M[i, 1] * y) + M[i, 2]   # each op rounded to f32

    sx, sy, sw = row(0), row(1), row(2)
    with np.errstate(divide="ignore", invalid="ignore"):
        r = (np.float32(1.0) / sw).astype(np.float32)
        return (sx * r).astype(np.float32), (sy * r).astype(np.float32)


def _nearest(v, hi):
    """round half to even, clip into [0, hi] (NaN -> 0), as integer index."""
    with np.errstate(invalid="ignore"):
        rv = np.rint(v).astype(np.float32)
    return np.fmin(np.fmax(rv, np.float32(0)), np.float32(hi)).astype(np.int64)


def warp_perspective(src, M, w_dst, h_dst):
    """Nearest-neighbour warp of a 2-D u8 image src[h_src, w_src] -> [h_dst, w_dst]
    (``warp_perspective_tinygrad`` with border_fill_val=None)."""
    h_src, w_src = src.shape
    sx, sy = _src_coords(M, w_dst, h_dst)
    xi, yi = _nearest(sx, w_src - 1), _nearest(sy, h_src - 1)
    return src[yi, xi]


def nv12_planes(frame, width, height, stride, y_height):
    """Y [height, width], U and V [height/2, width/2] views of a flat NV12 buffer."""
    frame = np.asarray(frame, np.uint8).reshape(-1)
    y = frame[:height * stride].reshape(height, stride)[:, :width]
    uv = frame[stride * y_height: stride * y_height + (height // 2) * stride].reshape(height // 2, stride)
    return y, uv[:, 0:width:2], uv[:, 1:width:2]


def frame_prepare(frame, M_inv, width, height, stride, y_height, model_w=512, model_h=256):
    """One camera: u8[6, model_h/2, model_w/2] (``make_frame_prepare`` + ``frames_to_tensor``)."""
    Y, U, V = nv12_planes(frame, width, height, stride, y_height)
    M = np.asarray(M_inv, np.float32).reshape(3, 3)
    Muv = (M * UV_SCALE).astype(np.float32)
    yw = warp_perspective(Y, M, model_w, model_h)
    uw = warp_perspective(U, Muv, model_w // 2, model_h // 2)
    vw = warp_perspective(V, Muv, model_w // 2, model_h // 2)
    return np.stack([yw[0::2, 0::2], yw[1::2, 0::2], yw[0::2, 1::2], yw[1::2, 1::2], uw, vw]).astype(np.uint8)


def make_warp(frame, big_frame, tfm, big_tfm, width, height, stride, y_height, model_w=512, model_h=256):
    """Both cameras: u8[2, 6, model_h/2, model_w/2] (``make_warp``)."""
    return np.stack([frame_prepare(frame, tfm, width, height, stride, y_height, model_w, model_h),
                     frame_prepare(big_frame, big_tfm, width, height, stride, y_height, model_w, model_h)])
