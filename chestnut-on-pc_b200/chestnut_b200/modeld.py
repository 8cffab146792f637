"""ModelState-compatible host class over the B200 engine.

Mirrors ``ModelState.run`` of the reference's openpilot-derived host
(``modeld.py:165-200``) for callers that already hold the warped frame
(the NV12 warp, ``compile_modeld.py:53-118``, is not part of this engine):

  * the desire input is a pulse on the rising edge (modeld.py:177-179):
    ``desire = where(desire_pulse - prev_desire > .99, desire_pulse, 0)`` with
    ``desire_pulse[0]`` forced to 0;
  * traffic_convention and action_t are copied into the packed vector;
  * a frame whose output is not finite is dropped (returns None,
    modeld.py:191-194) and does not update the carried features;
  * ``prev_feat`` is carried from ``out[hidden_state]`` (modeld.py:196).

Output decoding (``parse_model_outputs.Parser``) is not part of the hot path;
``run`` returns the sliced heads the way ``slice_outputs`` does
(``modeld.py:160-162``), each with a leading batch axis.
"""
import numpy as np

DESIRE_LEN = 8


class ModelState:
    def __init__(self, model="1b", device=0, seed=0, engine=None):
        if engine is None:
            from .engine import Engine
            engine = Engine(model, device=device, batch=1, seed=seed)
        self.engine = engine
        self.output_slices = dict(engine.out_slices)
        self.input_shapes = {
            'img': (1, 12, 128, 256), 'big_img': (1, 12, 128, 256), 'features_buffer': (1, 24, 512),
            'desire_pulse': (1, 25, 8), 'traffic_convention': (1, 2), 'action_t': (1, 2),
        }
        self.prev_desire = np.zeros(DESIRE_LEN, dtype=np.float32)
        self.packed = np.zeros(DESIRE_LEN + 2 + 2 + 512, np.float32)  # desire | tc | action_t | prev_feat

    def slice_outputs(self, model_outputs, output_slices):
        return {k: model_outputs[np.newaxis, v] for k, v in output_slices.items()}

    def run(self, warped, inputs):
        """warped u8[2,6,128,256]; inputs: desire_pulse f32[8], traffic_convention f32[2], action_t f32[2]."""
        desire_pulse = np.asarray(inputs['desire_pulse'], np.float32).reshape(-1).copy()
        desire_pulse[0] = 0
        desire = np.where(desire_pulse - self.prev_desire > .99, desire_pulse, 0)
        self.prev_desire[:] = desire_pulse
        p = self.packed.copy()
        p[0:8] = desire
        p[8:10] = np.asarray(inputs['traffic_convention'], np.float32).reshape(-1)
        p[10:12] = np.asarray(inputs['action_t'], np.float32).reshape(-1)
        out = np.asarray(self.engine.run_frame(warped, p)).reshape(-1)
        if not np.all(np.isfinite(out)):
            return None
        self.packed[:12] = p[:12]
        self.packed[12:] = out[self.output_slices['hidden_state']]
        return self.slice_outputs(out, self.output_slices)
