"""The reference's f16 divide rule has no counterpart in the engine (CPU check).

The reference lowers a half-precision division a / b to
a * f16(rcp_f32(f32(b))) (run_pinned2.py:622-632).  The engine never divides
in f16: every half value is converted to f32 before arithmetic (softmax,
LayerNorm and the head products divide in f32).  Two facts make that
checkable without a GPU:

* the library is compiled with __CUDA_NO_HALF_OPERATORS__ and
  __CUDA_NO_HALF2_OPERATORS__, so `/` (or any arithmetic operator) on __half /
  __half2 values does not compile;
* no source uses the explicit half division / reciprocal intrinsics.
"""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "chestnut-on-pc_b200")


def test_half_operators_are_disabled_in_the_build():
    src = open(os.path.join(PKG, "build.py")).read()
    assert '"-D__CUDA_NO_HALF_OPERATORS__"' in src and '"-D__CUDA_NO_HALF2_OPERATORS__"' in src


def test_no_half_division_or_reciprocal_intrinsics_in_the_sources():
    pat = re.compile(r"\b(__hdiv|__h2div|h2div|hdiv|hrcp|h2rcp|__hrcp|__h2rcp)\s*\(")
    csrc = os.path.join(PKG, "csrc")
    hits = []
    for name in sorted(os.listdir(csrc)):
        if name.endswith((".cu", ".cuh")):
            for i, line in enumerate(open(os.path.join(csrc, name)), 1):
                if pat.search(line):
                    hits.append(f"{name}:{i}: {line.strip()}")
    assert not hits, hits
