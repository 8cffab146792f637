"""image2d zero-border gather (oracle side, test infrastructure).

Restates the reference's image read semantics: a texel (y, x) of an (A, B, C)
image is read at the edge-clamped address and then masked to zero when the
ORIGINAL coordinate is out of range -- OpenCL ``CLK_ADDRESS_CLAMP`` with a zero
border colour (``run_pinned2.py:56-92`` register-level clamp + validity,
``:690-716`` LOAD masking, ``research/probe_sampler.py:12-23`` probe).

The conv stem reads its inputs through this rule; ``im2col_*`` below build the
exact f16 matrices the engine's gather kernels must produce (bit-exact).
K index convention: k = (ky*3 + kx) * C + c.
"""
import numpy as np

from . import spec as S


def read_texel(img, y, x):
    """img: (A, B, C) array; returns img[y, x, :] or zeros outside (A, B)."""
    A, B = img.shape[0], img.shape[1]
    flat = min(max(y * B + x, 0), A * B - 1)     # address stays in bounds
    valid = (0 <= x < B) and (0 <= y < A)
    v = img.reshape(A * B, -1)[flat]
    return v if valid else np.zeros_like(v)


def normalize_u8(u8):
    """u8 texel -> f16 model input: (v - 128) / 64, exact in f16."""
    return ((u8.astype(np.float32) - 128.0) * np.float32(1.0 / 64.0)).astype(np.float16)


def im2col_s2(act_hwc, k_pad=None):
    """3x3 / stride 2 / pad 1 zero-border gather of an (H, W, C) f16 image.

    Returns f16 [(H/2)*(W/2), 9*C (padded to k_pad)] with k = tap*C + c.
    """
    Hh, Ww, C = act_hwc.shape
    Ho, Wo = Hh // 2, Ww // 2
    padded = np.zeros((Hh + 2, Ww + 2, C), act_hwc.dtype)
    padded[1:-1, 1:-1] = act_hwc
    K = 9 * C
    out = np.zeros((Ho * Wo, k_pad or K), np.float16)
    for ky in range(3):
        for kx in range(3):
            tap = ky * 3 + kx
            # input y = 2*oy + ky - 1 -> padded index 2*oy + ky
            patch = padded[ky:ky + 2 * Ho:2, kx:kx + 2 * Wo:2, :]
            out[:, tap * C:(tap + 1) * C] = patch.reshape(Ho * Wo, C)
    return out


def im2col_frame(img12_u8):
    """First-stage gather from the sampled u8 image (12, 128, 256)."""
    hwc = normalize_u8(np.transpose(img12_u8, (1, 2, 0)))
    return im2col_s2(hwc, S.K0_PAD)
