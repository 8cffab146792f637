"""Counter-based hash RNG for synthetic weights (oracle side, test infrastructure).

The engine generates its random-init weights on the device with the same
function, so both sides hold bit-identical f16 weights without shipping a
weight file.  The mixer is the published SplitMix64 finaliser (Steele, Lea &
Flood, "Fast splittable pseudorandom number generators", OOPSLA 2014).

  key = seed << 48 | tensor_id << 32 | index
  u   = (splitmix64(key) >> 40) * 2**-23 - 1      in [-1, 1), exact in f32
  w   = f16(f32(u) * f32(bound))                  (IEEE RNE at both steps)
"""
import numpy as np

_C0 = np.uint64(0x9E3779B97F4A7C15)
_C1 = np.uint64(0xBF58476D1CE4E5B9)
_C2 = np.uint64(0x94D049BB133111EB)


def splitmix64(z):
    z = z + _C0
    z = (z ^ (z >> np.uint64(30))) * _C1
    z = (z ^ (z >> np.uint64(27))) * _C2
    return z ^ (z >> np.uint64(31))


def uniform(seed, tid, start, count):
    """f32 uniforms in [-1, 1) for indices [start, start+count)."""
    with np.errstate(over="ignore"):
        idx = np.arange(start, start + count, dtype=np.uint64)
        key = (np.uint64(seed) << np.uint64(48)) | (np.uint64(tid) << np.uint64(32)) | idx
        h = splitmix64(key)
    m = (h >> np.uint64(40)).astype(np.int64).astype(np.float32)
    return m * np.float32(2.0 ** -23) - np.float32(1.0)


def fill(seed, tid, count, bound, out_dtype, chunk=1 << 24):
    out = np.empty(count, dtype=out_dtype)
    b = np.float32(bound)
    for s in range(0, count, chunk):
        n = min(chunk, count - s)
        out[s:s + n] = (uniform(seed, tid, s, n) * b).astype(out_dtype)
    return out
