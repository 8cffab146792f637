"""Drop-in replacement for the reference's ``run_pinned2.py`` engine module.

Consumers (``video_check.py:16-19``, ``drive_gui.py:26-28``, ``video_demo.py:21-24``)
set ``sys.argv = [x, pkl]``, read this file from the working directory, split it
on the literal smoke-run marker and ``exec`` the prefix.  The prefix defines
the same names the reference's prefix defines (``run_pinned2.py:1346-1565``):

  run_frame(warped_np u8[2,6,128,256], packed f32[524]) -> f32[3323] (fresh array)
  out_slices, ish, img, PACKED, queues, make_warped, _LIN_BY_NAME, jit, cap,
  rewrite_uop_list

The model behind it is the B200 engine (libchestnut.so through ctypes): a
synthetic chestnut-class model chosen from the pickle name ("big" -> the 1B
config, else the 39M config) with seeded random-init weights, replayed as one
CUDA graph per frame.  The comma pickles themselves are not read.
Environment: CN_SEED (weight seed, default 0), CN_DEVICE (default 0),
CN_GRAPH (1 = CUDA graph replay, default; 0 = eager launches).
"""
import os
import sys
import time

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__)) if "__file__" in globals() else os.getcwd()
for _p in (_HERE, os.path.join(os.getcwd(), "chestnut-on-pc_b200")):
    if os.path.isdir(os.path.join(_p, "chestnut_b200")) and _p not in sys.path:
        sys.path.insert(0, _p)

from chestnut_b200 import Engine  # noqa: E402

PKL = sys.argv[1] if len(sys.argv) > 1 else 'models/driving.pkl'
_MODEL = '1b' if 'big' in os.path.basename(PKL) else '39m'
print(f'loading {PKL} -> synthetic {_MODEL} chestnut model on the B200 engine ...')
_t0 = time.perf_counter()
_eng = Engine(_MODEL, device=int(os.getenv('CN_DEVICE', '0')), batch=1, seed=int(os.getenv('CN_SEED', '0')),
              use_graph=os.getenv('CN_GRAPH', '1') == '1')
print(f'engine ready in {time.perf_counter() - _t0:.1f}s ({_eng.info()["n_params"] / 1e6:.1f}M params, '
      f'{_eng.info()["n_kernels"]} launches per frame)')

ish = {
    'img': (1, 12, 128, 256), 'big_img': (1, 12, 128, 256), 'features_buffer': (1, 24, 512),
    'desire_pulse': (1, 25, 8), 'traffic_convention': (1, 2), 'action_t': (1, 2),
}
out_slices = dict(_eng.out_slices)
img = ish['img']
PACKED = np.zeros(8 + 2 + 2 + ish['features_buffer'][2], np.float32)  # desire8 | tc2 | action_t2 | prev_feat512


class _Queues(dict):
    """Lazy view of the engine's device-resident queues in the reference's
    shapes (img_q u8[5,6,128,256], feat_q f32[96,1,512], desire_q f32[100,1,8])."""

    def __getitem__(self, k):
        if k == 'packed_npy_inputs':
            return PACKED
        st = _eng.get_state(0)
        return st[k]

    def keys(self):
        return ['img_q', 'big_img_q', 'feat_q', 'desire_q', 'packed_npy_inputs']


queues = _Queues()


def make_warped(val=128):
    return np.full((2, 6, img[2], img[3]), val, np.uint8)


_LIN_BY_NAME = {k['name']: (k, k['block']) for k in _eng.kernel_list()}
jit = cap = _eng


def rewrite_uop_list(*_a, **_k):
    raise NotImplementedError('the B200 engine has no tinygrad uop lists; its kernels are listed in _LIN_BY_NAME')


def run_frame(warped_np, packed):
    PACKED[:] = packed
    return _eng.run_frame(np.ascontiguousarray(warped_np, np.uint8), PACKED)


# --- smoke run + timing ---------------------------------------------------------------
print('--- run 1 (cold) ---')
t0 = time.perf_counter()
p0 = np.zeros(524, np.float32)
out = run_frame(np.full((2, 6, img[2], img[3]), 128, np.uint8), p0)
print(f'cold call {time.perf_counter()-t0:.2f}s, finite={np.isfinite(out).all()} absmax={np.abs(out).max():.4f}')
p0[12:] = out[out_slices['hidden_state']]

print('--- timing (10 iters) ---')
ts = []
for i in range(10):
    t0 = time.perf_counter()
    out = run_frame(np.full((2, 6, img[2], img[3]), 128, np.uint8), p0)
    p0[12:] = out[out_slices['hidden_state']]
    ts.append((time.perf_counter() - t0) * 1e3)
print('per-call ms:', [f'{t:.2f}' for t in ts])
for name in ('plan', 'lead', 'lane_lines', 'hidden_state'):
    seg = out[out_slices[name]]
    print(f'  {name:14} absmax={np.abs(seg).max():9.4f} mean={seg.mean():9.4f}')

print('--- A/B sensitivity (bright vs dark road) ---')


def frames(val, n=4):
    pk = np.zeros(524, np.float32)
    outs = []
    wf = np.full((2, 6, img[2], img[3]), val, np.uint8)
    for _ in range(n):
        o = run_frame(wf, pk)
        pk[12:] = o[out_slices['hidden_state']]
        outs.append(o)
    return outs


A = frames(40)
B = frames(220)
for name in ('plan', 'lead', 'hidden_state', 'lane_lines'):
    d = np.abs(A[-1][out_slices[name]] - B[-1][out_slices[name]]).max()
    print(f'  {name:14} A/B maxdiff = {d:.4f}')
