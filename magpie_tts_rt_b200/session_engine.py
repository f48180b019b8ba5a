"""Python handle on the per-GPU session engine (C ABI section 6 of
include/magpie_tts_rt_b200.h): the C++ host side that owns every session's
device state on one GPU and runs one step for all of them as one CUDA graph
([Main Decoder step ->] alignment gate -> Local AR frame [-> position + 1]).

The engine keeps pointers to the weights of the LocalArEngine (and
MainDecoderEngine) it is built from; keep those objects alive while it runs.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np
import torch

from magpie_tts_rt_b200 import _lib as L
from magpie_tts_rt_b200.local_ar import AlignmentKernelContract, LocalArEngine
from magpie_tts_rt_b200.model import EMBED


class SessionEngine:
    def __init__(self, lar: LocalArEngine, max_sessions: int, token_stride: int = 128, decoder=None,
                 cache_capacity: int = 0, contract: Optional[AlignmentKernelContract] = None,
                 decoder_hidden: Optional[torch.Tensor] = None, alignment_scores: Optional[torch.Tensor] = None,
                 next_embedding: Optional[torch.Tensor] = None):
        contract = contract or AlignmentKernelContract(text_length=1)
        cfg = L.SessionEngineConfig()
        cfg.max_sessions = max_sessions
        cfg.token_stride = token_stride
        cfg.with_decoder = 1 if decoder is not None else 0
        cfg.cache_capacity = cache_capacity
        cfg.ignored_terminal_tokens = contract.ignored_terminal_tokens
        cfg.short_text_no_prior_max_tokens = contract.short_text_no_prior_max_tokens
        cfg.lookahead = contract.lookahead
        cfg.sink_threshold = contract.sink_threshold
        cfg.shape = lar._shape
        cfg.local_ar = lar._w
        cfg.sampling = lar._sampling
        if decoder is not None:
            cfg.decoder = decoder._w
        self._keep = (lar, decoder, decoder_hidden, alignment_scores, next_embedding)
        cfg.decoder_hidden = decoder_hidden.data_ptr() if decoder_hidden is not None else None
        cfg.alignment_scores = alignment_scores.data_ptr() if alignment_scores is not None else None
        cfg.next_embedding = next_embedding.data_ptr() if next_embedding is not None else None
        self._cfg = cfg
        self._handle = ctypes.c_void_p()
        rc = L.lib.mtt_b200_session_engine_create(ctypes.byref(cfg), ctypes.byref(self._handle))
        if rc != L.STATUS_OK:
            raise RuntimeError(f"mtt_b200_session_engine_create failed with status {rc}")
        self.max_sessions = max_sessions
        self.buffers = L.SessionEngineBuffers()
        L.lib.mtt_b200_session_engine_buffers(self._handle, ctypes.byref(self.buffers))

    @property
    def stream_handle(self) -> int:
        return int(self.buffers.stream)

    def open(self, slot: int, seed: int, text_length: int, cross_k: Optional[torch.Tensor] = None,
             cross_v: Optional[torch.Tensor] = None, cond_mask: Optional[torch.Tensor] = None,
             initial_embedding: Optional[torch.Tensor] = None) -> None:
        p = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None
        rc = L.lib.mtt_b200_session_engine_open(self._handle, slot, seed, text_length, p(cross_k), p(cross_v),
                                                p(cond_mask), p(initial_embedding))
        if rc != L.STATUS_OK:
            raise RuntimeError(f"mtt_b200_session_engine_open failed with status {rc}")

    def close(self, slot: int) -> None:
        rc = L.lib.mtt_b200_session_engine_close(self._handle, slot)
        if rc != L.STATUS_OK:
            raise RuntimeError(f"mtt_b200_session_engine_close failed with status {rc}")

    def step(self) -> None:
        rc = L.lib.mtt_b200_session_engine_step(self._handle)
        if rc != L.STATUS_OK:
            raise RuntimeError(f"mtt_b200_session_engine_step failed with status {rc}")

    def collect(self, n: Optional[int] = None):
        """(codec_tokens [n, 8, 2] int64, end_frame_index [n] int32, invalid_rows [n] int32) on the host."""
        n = self.max_sessions if n is None else n
        codes = np.zeros((n, 8, 2), np.int64)
        end = np.zeros(n, np.int32)
        inv = np.zeros(n, np.int32)
        rc = L.lib.mtt_b200_session_engine_collect(self._handle, n, codes.ctypes.data_as(ctypes.c_void_p),
                                                   end.ctypes.data_as(ctypes.c_void_p),
                                                   inv.ctypes.data_as(ctypes.c_void_p))
        if rc != L.STATUS_OK:
            raise RuntimeError(f"mtt_b200_session_engine_collect failed with status {rc}")
        return codes, end, inv

    def synchronize(self) -> None:
        torch.cuda.ExternalStream(self.stream_handle).synchronize()

    def close_engine(self) -> None:
        if self._handle:
            L.lib.mtt_b200_session_engine_destroy(self._handle)
            self._handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close_engine()
        except Exception:
            pass


__all__ = ["SessionEngine", "EMBED"]
