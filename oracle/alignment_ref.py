"""Build recipe and ctypes binding for the reference's own host alignment
controller, compiled here from its source where it lies.

TEST INFRASTRUCTURE ONLY: used by ``tests/golden/make_alignment_golden.py``
(and the CPU tests when the library is present) to pin ``oracle/alignment.py``.
The recipe compiles the reference's ``src/runtime/alignment_controller.cpp``
(which needs only ``src/manifest/manifest.hpp``, a header of plain structs)
together with ``oracle/csrc/alignment_ref_shim.cpp`` into
``oracle/_ref/libalignment_ref.so``; nothing of the reference is copied into
this repository.  Only the container that holds the reference tree can build
it; elsewhere ``available()`` is False.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_ROOT = os.environ.get("MTT_REFERENCE_ROOT", os.path.join(os.sep, "root", "reference"))
REF_SOURCE = os.path.join(REF_ROOT, "src", "runtime", "alignment_controller.cpp")
SHIM = os.path.join(HERE, "csrc", "alignment_ref_shim.cpp")
OUT_DIR = os.path.join(HERE, "_ref")
LIBRARY = os.path.join(OUT_DIR, "libalignment_ref.so")


def build(force: bool = False) -> Optional[str]:
    """Compile the reference controller; None when the reference tree is absent."""
    if os.path.exists(LIBRARY) and not force and (
            not os.path.exists(REF_SOURCE)
            or os.path.getmtime(LIBRARY) >= max(os.path.getmtime(SHIM), os.path.getmtime(REF_SOURCE))):
        return LIBRARY
    if not os.path.exists(REF_SOURCE):
        return None
    os.makedirs(OUT_DIR, exist_ok=True)
    cmd = ["g++", "-std=c++20", "-O2", "-fPIC", "-shared", "-I" + os.path.join(REF_ROOT, "src"),
           "-o", LIBRARY, REF_SOURCE, SHIM]
    subprocess.run(cmd, check=True)
    return LIBRARY


def available() -> bool:
    return build() is not None


class RefController:
    """ctypes handle on one reference AlignmentControllerReference."""

    _lib = None

    @classmethod
    def lib(cls):
        if cls._lib is None:
            path = build()
            if path is None:
                raise FileNotFoundError("the reference alignment controller is not built here")
            L = ctypes.CDLL(path)
            P, U32 = ctypes.c_void_p, ctypes.c_uint32
            L.mtt_ref_alignment_create.restype = P
            L.mtt_ref_alignment_create.argtypes = [U32, ctypes.c_double, U32, U32, U32, U32, U32,
                                                   ctypes.POINTER(ctypes.c_int)]
            L.mtt_ref_alignment_advance.restype = ctypes.c_int
            L.mtt_ref_alignment_advance.argtypes = [P, P, U32, P, P, P, U32]
            L.mtt_ref_alignment_last_attended.restype = U32
            L.mtt_ref_alignment_last_attended.argtypes = [P]
            L.mtt_ref_alignment_counters.restype = None
            L.mtt_ref_alignment_counters.argtypes = [P, P]
            L.mtt_ref_alignment_destroy.restype = None
            L.mtt_ref_alignment_destroy.argtypes = [P]
            cls._lib = L
        return cls._lib

    def __init__(self, text_length, prior_epsilon=0.1, initial_attended=1, ignored_terminal_tokens=3,
                 short_text_no_prior_max_tokens=5, lookahead=6, sink_threshold=4):
        L = self.lib()
        st = ctypes.c_int(-1)
        self.T = int(text_length)
        self.h = L.mtt_ref_alignment_create(text_length, prior_epsilon, initial_attended,
                                            ignored_terminal_tokens, short_text_no_prior_max_tokens,
                                            lookahead, sink_threshold, ctypes.byref(st))
        self.status = st.value

    def advance(self, scores):
        """-> (status, attended, unfinished, prior[2T] float32); status 0 ok,
        else 1 + the reference's error code index."""
        s = np.ascontiguousarray(np.asarray(scores, np.float32))
        att = ctypes.c_uint32(0)
        unf = ctypes.c_int32(0)
        prior = np.zeros(2 * self.T, np.float32)
        rc = self.lib().mtt_ref_alignment_advance(self.h, s.ctypes.data, s.size, ctypes.byref(att),
                                                  ctypes.byref(unf), prior.ctypes.data, prior.size)
        return rc, att.value, bool(unf.value), prior

    def counters(self):
        out = np.zeros(self.T, np.uint32)
        self.lib().mtt_ref_alignment_counters(self.h, out.ctypes.data)
        return out

    def last_attended(self):
        return self.lib().mtt_ref_alignment_last_attended(self.h)

    def __del__(self):
        if getattr(self, "h", None):
            self.lib().mtt_ref_alignment_destroy(self.h)
            self.h = None
