"""ModelState-compatible host class over the B200 engine.

Mirrors ``ModelState.run`` of the reference's openpilot-derived host
(``modeld.py:165-200``).  ``run(bufs, transforms, inputs)`` takes the road
and wide NV12 camera frames (``bufs['img']``, ``bufs['big_img']``: host
buffers, or device pointers as ints) and their 3x3 warp transforms, warps
them on the GPU (``cn_warp_frames``, the reference's ``compile_modeld.py``
frame warp) into the engine's input and runs the frame from device buffers;
the NV12 geometry (width, height, stride, y_height, uv_height -- what the
reference gets from openpilot's ``get_nv12_info``) is given at construction.
``run(warped, inputs)`` takes an already warped u8[2,6,128,256] frame.
Both follow the reference's host semantics:

  * the desire input is a pulse on the rising edge (modeld.py:177-179):
    ``desire = where(desire_pulse - prev_desire > .99, desire_pulse, 0)`` with
    ``desire_pulse[0]`` forced to 0;
  * traffic_convention and action_t are copied into the packed vector;
  * a frame whose output is not finite is dropped (returns None,
    modeld.py:191-194) and does not update the carried features;
  * ``prev_feat`` is carried from ``out[hidden_state]`` (modeld.py:196).

``run`` returns the sliced heads the way ``slice_outputs`` does
(``modeld.py:160-162``), each with a leading batch axis.  Given a decode
layout at construction (``decode=SYNTHETIC_LAYOUT`` or a real model's), the
frame output is also parsed on the GPU as ``parse_model_outputs.Parser``
would parse it on the host (``decode.py``), and the parsed keys are added to
the returned dict with the same leading batch axis.
"""
import numpy as np

DESIRE_LEN = 8


class ModelState:
    def __init__(self, model="1b", device=0, seed=0, engine=None, nv12=None, decode=None):
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
        # NV12 geometry of both cameras: (width, height, stride, y_height, uv_height)
        self.nv12 = tuple(int(v) for v in nv12) if nv12 is not None else None
        self._dev = None
        self.last_output = None
        self.decode_layout = decode

    def slice_outputs(self, model_outputs, output_slices):
        return {k: model_outputs[np.newaxis, v] for k, v in output_slices.items()}

    def run(self, bufs, transforms, inputs=None):
        """run(bufs, transforms, inputs): NV12 frames + warp transforms (modeld.py:165);
        run(warped, inputs): warped u8[2,6,128,256].  inputs: desire_pulse f32[8],
        traffic_convention f32[2], action_t f32[2]."""
        if inputs is None:
            warped, inputs = bufs, transforms
            return self._run(inputs, lambda p: self.engine.run_frame(warped, p))
        if self.nv12 is None:
            raise ValueError("ModelState: NV12 frames need the camera geometry (nv12=...) at construction")
        return self._run(inputs, lambda p: self._run_nv12(bufs, transforms, p))

    def _buffers(self):
        if self._dev is None:
            from ._lib import DeviceBuffer
            _, _, stride, y_height, uv_height = self.nv12
            size = stride * (y_height + uv_height)
            self._dev = {'img': DeviceBuffer(size), 'big_img': DeviceBuffer(size),
                         'warped': DeviceBuffer(2 * 6 * 128 * 256), 'packed': DeviceBuffer(self.packed.nbytes)}
        return self._dev

    def _run_nv12(self, bufs, transforms, packed):
        from . import kernels
        d = self._buffers()
        width, height, stride, y_height, uv_height = self.nv12
        size = stride * (y_height + uv_height)
        ptr = {}
        for k in ('img', 'big_img'):
            b = bufs[k]
            if isinstance(b, (int, np.integer)):
                ptr[k] = int(b)          # already on the device (the caller's frame buffer)
            else:
                a = np.frombuffer(memoryview(b).cast('B'), np.uint8) if not isinstance(b, np.ndarray) else b
                d[k].upload(np.ascontiguousarray(a.reshape(-1)[:size]))
                ptr[k] = d[k].ptr
        # warp on the engine's stream, then the frame from device buffers (same stream)
        kernels.warp_frames(ptr['img'], ptr['big_img'], transforms['img'], transforms['big_img'], width, height,
                            stride, y_height, uv_height, d['warped'].ptr, stream=self.engine.stream_handle())
        d['packed'].upload(packed)
        self.engine.run_frame_device(d['warped'].ptr, d['packed'].ptr)
        return self.engine.read_output()[0]

    def _run(self, inputs, frame):
        desire_pulse = np.asarray(inputs['desire_pulse'], np.float32).reshape(-1).copy()
        desire_pulse[0] = 0
        desire = np.where(desire_pulse - self.prev_desire > .99, desire_pulse, 0)
        self.prev_desire[:] = desire_pulse
        p = self.packed.copy()
        p[0:8] = desire
        p[8:10] = np.asarray(inputs['traffic_convention'], np.float32).reshape(-1)
        p[10:12] = np.asarray(inputs['action_t'], np.float32).reshape(-1)
        out = np.asarray(frame(p)).reshape(-1)
        self.last_output = out  # the flat output of the last frame (video_check-style harnesses read it)
        if not np.all(np.isfinite(out)):
            return None
        self.packed[:12] = p[:12]
        self.packed[12:] = out[self.output_slices['hidden_state']]
        res = self.slice_outputs(out, self.output_slices)
        if self.decode_layout is not None:
            from .decode import decode_frame
            for k, v in decode_frame(self.engine, self.decode_layout)[0].items():
                res[k] = v[np.newaxis]
        return res
