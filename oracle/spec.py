"""Synthetic chestnut-class model specification (oracle side).

Test infrastructure: restates the model that the engine implements so the
engine can be checked against it.  Shapes follow the reference's frame
contract:

  * ``warped`` u8[2, 6, 128, 256] and ``packed`` f32[524] per frame
    (``run_pinned2.py:1385,1462``; packed = desire8 | traffic_convention2 |
    action_t2 | prev_feat512, ``compile_modeld.py:138-145``).
  * queues with frame skip FS=4 (``run_pinned2.py:1373-1389``).
  * output heads plan[5x33x15], lane_lines[4x33x2], lead[3x6x4] and
    hidden_state[512] (BASELINE configs 3/4).

The layer list itself is synthetic (the comma pickles are absent): a conv stem
of five stride-2 stages (3x3 conv + 1x1 conv, ReLU) per camera, 64 vision
tokens + 24 temporal tokens = 88 tokens through a pre-LN transformer.
"""
from dataclasses import dataclass

H, W = 128, 256            # per-plane image size (run_pinned2.py:1377 ish['img'][2:])
CH = 6                     # YUV planes per frame (Y00,Y10,Y01,Y11,U,V; video_check.py:27-32)
FS = 4                     # frame skip (run_pinned2.py:1373)
N_FRAMES = 2               # img = (1, 12, 128, 256) -> 2 frames of 6 planes
IMG_Q = FS * (N_FRAMES - 1) + 1   # 5 rows in img_q / big_img_q (run_pinned2.py:1376)
FEAT = 512                 # features_buffer width / hidden_state width
N_TEMP = 24                # past feature tokens (features_buffer (1,24,512))
FEAT_Q = FS * N_TEMP       # 96 rows in feat_q
N_DESIRE = 25              # desire_pulse (1,25,8)
DESIRE = 8
DESIRE_Q = FS * N_DESIRE   # 100 rows in desire_q
TC = 2
AT = 2
PACKED = DESIRE + TC + AT + FEAT   # 524
COND = N_DESIRE * DESIRE + TC + AT  # 204
COND_PAD = 256
N_CAM = 2
STEM_STAGES = 5
VIS_H, VIS_W = H >> STEM_STAGES, W >> STEM_STAGES   # 4 x 8
N_VIS_CAM = VIS_H * VIS_W  # 32 tokens per camera
N_VIS = N_CAM * N_VIS_CAM  # 64
T = N_VIS + N_TEMP         # 88 tokens
TRUNK = 1024
K0 = 9 * N_FRAMES * CH     # 108 taps*channels of the first conv
K0_PAD = 128
LN_EPS = 1e-5

HEADS = (("plan", 5 * 33 * 15), ("lane_lines", 4 * 33 * 2), ("lead", 3 * 6 * 4))
N_HEADS_OUT = sum(n for _, n in HEADS)   # 2811
N_OUT = N_HEADS_OUT + FEAT               # 3323


def out_slices():
    """name -> slice into the flat f32 output (reference: meta['output_slices'])."""
    s, o = {}, 0
    for name, n in HEADS:
        s[name] = slice(o, o + n)
        o += n
    s["hidden_state"] = slice(o, o + FEAT)
    return s


@dataclass(frozen=True)
class ModelCfg:
    name: str
    stem: tuple
    d: int
    heads: int
    layers: int
    mlp: int

    @property
    def hd(self):
        return self.d // self.heads


CONFIGS = {
    "39m": ModelCfg("39m", (32, 64, 128, 256, 512), 512, 8, 4, 2048),
    "1b": ModelCfg("1b", (64, 128, 256, 512, 1024), 2048, 16, 20, 8192),
}


def param_table(cfg: ModelCfg):
    """Ordered parameter list: (name, tensor_id, shape, fan_in, kind).

    kind: 'w' (He-uniform weight, f16), 'b' (bias, f32, U(+-1/sqrt(fan_in))),
    'pos' (f32 positional table, U(+-0.5)).  tensor_id feeds the hash RNG.
    Weights are stored GEMM-ready as [N_out, K] (K contiguous); the first
    conv's K=108 is stored padded to 128 with zero columns.
    """
    P = []
    tid = 0

    def add(name, shape, fan_in, kind):
        nonlocal tid
        P.append((name, tid, tuple(shape), fan_in, kind))
        tid += 1

    for cam in range(N_CAM):
        cin = N_FRAMES * CH
        for s, c in enumerate(cfg.stem):
            k = 9 * cin
            add(f"cam{cam}.s{s}.conv3.w", (c, K0_PAD if s == 0 else k), k, "w")
            add(f"cam{cam}.s{s}.conv3.b", (c,), k, "b")
            add(f"cam{cam}.s{s}.conv1.w", (c, c), c, "w")
            add(f"cam{cam}.s{s}.conv1.b", (c,), c, "b")
            cin = c
        add(f"cam{cam}.vis.w", (cfg.d, cin), cin, "w")
        add(f"cam{cam}.vis.b", (cfg.d,), cin, "b")
    add("temp.w", (cfg.d, FEAT), FEAT, "w")
    add("temp.b", (cfg.d,), FEAT, "b")
    add("cond.w", (cfg.d, COND_PAD), COND, "w")
    add("cond.b", (cfg.d,), COND, "b")
    add("pos", (T, cfg.d), 0, "pos")
    for l in range(cfg.layers):
        add(f"l{l}.qkv.w", (3 * cfg.d, cfg.d), cfg.d, "w")
        add(f"l{l}.qkv.b", (3 * cfg.d,), cfg.d, "b")
        add(f"l{l}.o.w", (cfg.d, cfg.d), cfg.d, "w")
        add(f"l{l}.o.b", (cfg.d,), cfg.d, "b")
        add(f"l{l}.fc1.w", (cfg.mlp, cfg.d), cfg.d, "w")
        add(f"l{l}.fc1.b", (cfg.mlp,), cfg.d, "b")
        add(f"l{l}.fc2.w", (cfg.d, cfg.mlp), cfg.mlp, "w")
        add(f"l{l}.fc2.b", (cfg.d,), cfg.mlp, "b")
    add("hid.w", (FEAT, cfg.d), cfg.d, "w")
    add("hid.b", (FEAT,), cfg.d, "b")
    add("trunk.w", (TRUNK, FEAT), FEAT, "w")
    add("trunk.b", (TRUNK,), FEAT, "b")
    add("heads.w", (N_HEADS_OUT, TRUNK), TRUNK, "w")
    add("heads.b", (N_HEADS_OUT,), TRUNK, "b")
    return P


def n_params(cfg: ModelCfg):
    """Parameter count excluding storage padding."""
    n = 0
    for name, _, shape, fan_in, kind in param_table(cfg):
        if name.endswith("s0.conv3.w"):
            n += shape[0] * K0
        elif name == "cond.w":
            n += shape[0] * COND
        else:
            c = 1
            for x in shape:
                c *= x
            n += c
    return n
