"""Host-side mirror of the reference's Local AR plugin/launcher interface.

* ``launch_local_ar_sampling`` / ``local_ar_eos_workspace_size`` /
  ``launch_local_ar_eos`` / ``launch_finalize_local_step`` /
  ``launch_layer_norm`` / ``launch_gelu_tanh`` / ``launch_softmax``: same names,
  arguments and 0 / -1 return convention as the reference's C++ launchers
  (``plugins/local_ar_plugins.hpp:29-55``,
  ``src/runtime/synthesis_kernels.cu:177-214``), taking CUDA tensors and
  calling the C ABI of ``libmagpie_tts_rt_b200.so``.
* ``plugin_api()`` / ``main_device_position_class_table()``: the plugin
  library ABI (``include/magpie_tts_rt/magpie_tts_rt_plugin.h``).
* ``LocalArEngine`` + ``StreamBatch``: the batched frame for N sessions with
  structure-of-arrays device state (seed, counter, flags, outputs), which is
  what a per-GPU serving loop calls once per decoder step.

PyTorch is used only for device memory and stream handles.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Optional

import torch

from magpie_tts_rt_b200 import _lib as L
from magpie_tts_rt_b200.model import (
    EMBED, POSITIONS, VOCAB, CFG_SCALE, TEMPERATURE, TOP_K, LocalArShape, LocalArWeights,
)


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream) -> ctypes.c_void_p:
    if stream is None:
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream)


# ---------------------------------------------------------------------------
# plugin library ABI
# ---------------------------------------------------------------------------

def plugin_api(struct_size: Optional[int] = None, abi_version: int = L.MTT_PLUGIN_ABI_VERSION_1):
    api = L.PluginApiV1()
    api.struct_size = ctypes.sizeof(L.PluginApiV1) if struct_size is None else struct_size
    api.abi_version = abi_version
    status = L.lib.mtt_plugin_get_api_v1(ctypes.byref(api))
    return status, api


def main_device_position_class_table(struct_size: Optional[int] = None,
                                     abi_version: int = L.MTT_PLUGIN_ABI_VERSION_1):
    table = L.MainDevicePositionClassTableV1()
    table.struct_size = ctypes.sizeof(table) if struct_size is None else struct_size
    table.abi_version = abi_version
    return L.lib.mtt_plugin_get_main_device_position_class_table_v1(ctypes.byref(table)), table


# ---------------------------------------------------------------------------
# launchers with the reference's signatures
# ---------------------------------------------------------------------------

def launch_local_ar_sampling(logits, unfinished, finished, forbid_eos, rng_seed, rng_counter,
                             embedding_weight, sampled_token, next_embedding, updated_rng_counter,
                             invalid_rows, stream=None) -> int:
    return L.lib.mtt_b200_launch_local_ar_sampling(
        _ptr(logits), _ptr(unfinished), _ptr(finished), _ptr(forbid_eos), _ptr(rng_seed),
        _ptr(rng_counter), _ptr(embedding_weight), _ptr(sampled_token), _ptr(next_embedding),
        _ptr(updated_rng_counter), _ptr(invalid_rows), _stream(stream))


def local_ar_eos_workspace_size() -> int:
    return int(L.lib.mtt_b200_local_ar_eos_workspace_size())


def launch_local_ar_eos(decoder_hidden, codec_tokens, unfinished, finished, forbid_eos,
                        final_weight, final_bias, workspace, end_frame_index, stream=None) -> int:
    return L.lib.mtt_b200_launch_local_ar_eos(
        _ptr(decoder_hidden), _ptr(codec_tokens), _ptr(unfinished), _ptr(finished),
        _ptr(forbid_eos), _ptr(final_weight), _ptr(final_bias), _ptr(workspace),
        _ptr(end_frame_index), _stream(stream))


def launch_finalize_local_step(step_codec_tokens, aggregate_codec_tokens, frame_offset: int,
                               canonical_invalid_rows, canonical_end_frame_index,
                               step_invalid_rows, step_end_frame_index, updated_rng_counter,
                               rng_counter, generation_finished, stream=None) -> int:
    return L.lib.mtt_b200_launch_finalize_local_step(
        _ptr(step_codec_tokens), _ptr(aggregate_codec_tokens), frame_offset,
        _ptr(canonical_invalid_rows), _ptr(canonical_end_frame_index), _ptr(step_invalid_rows),
        _ptr(step_end_frame_index), _ptr(updated_rng_counter), _ptr(rng_counter),
        _ptr(generation_finished), _stream(stream))


def launch_layer_norm(input, weight, output, row_count: int, stream=None) -> int:
    return L.lib.mtt_b200_launch_layer_norm(_ptr(input), _ptr(weight), _ptr(output), row_count, _stream(stream))


def launch_gelu_tanh(input, output, element_count: int, stream=None) -> int:
    return L.lib.mtt_b200_launch_gelu_tanh(_ptr(input), _ptr(output), element_count, _stream(stream))


def launch_softmax(input, output, batch_count: int, element_count: int, stream=None) -> int:
    return L.lib.mtt_b200_launch_softmax(_ptr(input), _ptr(output), batch_count, element_count, _stream(stream))


# ---------------------------------------------------------------------------
# batched frame
# ---------------------------------------------------------------------------

@dataclass
class StreamBatch:
    """SoA device state and I/O for n independent sessions."""

    decoder_hidden: torch.Tensor  # [n, rows, 768] bf16
    unfinished: torch.Tensor  # [n] bool
    finished: torch.Tensor
    forbid_eos: torch.Tensor
    rng_seed: torch.Tensor  # [n] int64
    rng_counter: torch.Tensor  # [n] int64 (in/out)
    codec_tokens: torch.Tensor  # [n, 8, 2] int64 (out), or the [n, 8, 8] aggregate
    invalid_rows: torch.Tensor  # [n] int32 (out)
    end_frame_index: torch.Tensor  # [n] int32 (out)
    next_embedding: torch.Tensor  # [n, 768] bf16 (out)
    active: Optional[torch.Tensor] = None  # [n] bool
    forced_tokens: Optional[torch.Tensor] = None  # [n, 16] int64
    logits_out: Optional[torch.Tensor] = None  # [n, 16, rows, 2024] bf16
    # finalize_local_step folded into the frame: codec_tokens may be the
    # [n, 8, 8] emission aggregate (stride 8, this frame at codec_frame_offset)
    codec_frame_offset: int = 0
    finished_latch: Optional[torch.Tensor] = None  # [n] bool, may be `finished`
    codec_frames: Optional[torch.Tensor] = None  # [n] int32: audio frames in the aggregate so far
    # [n, 32] int32 from the Main Decoder step that produced decoder_hidden
    # (MainDecoderBatch.eos_projection): the frame skips its own EOS projection
    eos_projection: Optional[torch.Tensor] = None

    @property
    def n(self) -> int:
        return int(self.rng_seed.shape[0])

    @staticmethod
    def allocate(n: int, cfg: bool = True, device="cuda") -> "StreamBatch":
        rows = 2 if cfg else 1
        z = lambda *s, dt: torch.zeros(*s, dtype=dt, device=device)
        return StreamBatch(
            decoder_hidden=z(n, rows, EMBED, dt=torch.bfloat16),
            unfinished=z(n, dt=torch.bool), finished=z(n, dt=torch.bool),
            forbid_eos=z(n, dt=torch.bool), rng_seed=z(n, dt=torch.int64),
            rng_counter=z(n, dt=torch.int64), codec_tokens=z(n, 8, 2, dt=torch.int64),
            invalid_rows=z(n, dt=torch.int32), end_frame_index=z(n, dt=torch.int32),
            next_embedding=z(n, EMBED, dt=torch.bfloat16),
        )

    def c_struct(self) -> L.StreamBatch:
        b = L.StreamBatch()
        b.n_streams = self.n
        b.decoder_hidden = self.decoder_hidden.data_ptr()
        for name in ("unfinished", "finished", "forbid_eos", "rng_seed", "rng_counter",
                     "codec_tokens", "invalid_rows", "end_frame_index", "next_embedding"):
            setattr(b, name, getattr(self, name).data_ptr())
        b.active = self.active.data_ptr() if self.active is not None else None
        b.forced_tokens = self.forced_tokens.data_ptr() if self.forced_tokens is not None else None
        b.logits_out = self.logits_out.data_ptr() if self.logits_out is not None else None
        b.codec_frames_stride = int(self.codec_tokens.shape[2])
        b.codec_frame_offset = self.codec_frame_offset
        b.finished_latch = self.finished_latch.data_ptr() if self.finished_latch is not None else None
        b.codec_frames = self.codec_frames.data_ptr() if self.codec_frames is not None else None
        b.eos_projection = self.eos_projection.data_ptr() if self.eos_projection is not None else None
        return b


class LocalArEngine:
    """Device-resident Local AR weights + workspace for up to ``max_streams``
    sessions on one GPU.  ``frame(batch)`` enqueues one 16-position frame on
    the current (or given) CUDA stream."""

    def __init__(self, weights: LocalArWeights, max_streams: int, device="cuda", cfg: bool = True,
                 top_k: int = TOP_K, temperature: float = TEMPERATURE, cfg_scale: float = CFG_SCALE,
                 argmax: bool = False, path: int = L.PATH_AUTO, fold_in_projection: bool = True):
        self.shape = weights.shape
        self.device = torch.device(device)
        self.cfg = cfg
        self.max_streams = max_streams
        dev = {}
        for name, t in weights.tensors():
            if t is None or t.numel() == 0:
                dev[name] = None
            else:
                dev[name] = t.to(device=self.device, dtype=torch.bfloat16).contiguous()
        self.dev = dev
        self._w = L.Weights()
        for name in L.Weights._fields_:
            t = dev.get(name[0])
            setattr(self._w, name[0], t.data_ptr() if t is not None else None)
        self._shape = L.Shape(self.shape.d_model, self.shape.n_layers, self.shape.n_heads,
                              self.shape.d_ffn)
        # fold the in-projection into the embedding tables once (weight transform)
        self.emb_proj = None
        if fold_in_projection and self.shape.in_projection:
            nbytes = L.lib.mtt_b200_fold_in_projection_bytes(ctypes.byref(self._shape))
            self.emb_proj = torch.empty(nbytes // 2, dtype=torch.bfloat16, device=self.device)
            status = L.lib.mtt_b200_launch_fold_in_projection(
                ctypes.byref(self._shape), ctypes.byref(self._w),
                ctypes.c_void_p(self.emb_proj.data_ptr()), _stream(None))
            if status != L.STATUS_OK:
                raise RuntimeError(f"mtt_b200_launch_fold_in_projection failed with status {status}")
            self._w.emb_proj = self.emb_proj.data_ptr()
        self._sampling = L.SamplingConfig(top_k, temperature, cfg_scale, int(argmax), int(cfg), int(path))
        size = L.lib.mtt_b200_local_ar_frame_workspace_size(ctypes.byref(self._shape), max_streams,
                                                           int(cfg))
        if size == 0:
            raise ValueError(f"unsupported shape {self.shape}")
        self.workspace = torch.empty(size, dtype=torch.uint8, device=self.device)

    @property
    def path(self) -> int:
        """Frame path for a full batch of ``max_streams`` on the current device
        (1 phase kernels, 2 fused cluster kernel, 3 tile kernel, 4 pair kernel)."""
        return self.path_for(self.max_streams)

    def path_for(self, n_streams: int) -> int:
        return int(L.lib.mtt_b200_local_ar_frame_path(ctypes.byref(self._shape), ctypes.byref(self._sampling),
                                                      n_streams))

    def launch_count(self, n_streams: int) -> int:
        return int(L.lib.mtt_b200_local_ar_frame_launch_count(ctypes.byref(self._shape),
                                                              ctypes.byref(self._sampling), n_streams))

    def frame(self, batch: StreamBatch, stream=None) -> None:
        if batch.n > self.max_streams:
            raise ValueError(f"{batch.n} streams > max_streams {self.max_streams}")
        cb = batch.c_struct()
        status = L.lib.mtt_b200_launch_local_ar_frame(
            ctypes.byref(self._shape), ctypes.byref(self._w), ctypes.byref(self._sampling),
            ctypes.byref(cb), ctypes.c_void_p(self.workspace.data_ptr()), self.workspace.numel(),
            _stream(stream))
        if status != L.STATUS_OK:
            raise RuntimeError(f"mtt_b200_launch_local_ar_frame failed with status {status}")


# ---------------------------------------------------------------------------
# alignment controller
# ---------------------------------------------------------------------------

@dataclass
class AlignmentKernelContract:
    """AlignmentKernelContract (src/runtime/alignment_kernel.hpp:9-15)."""

    text_length: int
    ignored_terminal_tokens: int = 3
    short_text_no_prior_max_tokens: int = 5
    lookahead: int = 6
    sink_threshold: int = 4

    def c_struct(self) -> L.AlignmentContract:
        return L.AlignmentContract(self.text_length, self.ignored_terminal_tokens,
                                   self.short_text_no_prior_max_tokens, self.lookahead, self.sink_threshold)


def launch_alignment_controller(alignment_scores, contract: AlignmentKernelContract, counters, last_attended,
                                next_prior, attended_token_index, unfinished_text, invalid_state,
                                stream=None) -> int:
    """launch_alignment_controller (src/runtime/alignment_kernel.hpp:20-29):
    returns the cudaError_t value (0 success, 1 cudaErrorInvalidValue for a
    missing buffer)."""
    c = contract.c_struct() if contract is not None else None
    return L.lib.mtt_b200_launch_alignment_controller(
        _ptr(alignment_scores), ctypes.byref(c) if c is not None else None, _ptr(counters),
        _ptr(last_attended), _ptr(next_prior), _ptr(attended_token_index), _ptr(unfinished_text),
        _ptr(invalid_state), _stream(stream))


@dataclass
class AlignmentBatch:
    """SoA alignment state for n sessions (one utterance each), rows padded to
    ``token_stride`` tokens.  ``gate(frame)`` runs one controller step for
    every active session and writes the frame batch's ``unfinished``,
    ``forbid_eos`` and ``finished`` inputs on the device."""

    text_length: torch.Tensor     # [n] uint32 (int32 storage)
    alignment_scores: torch.Tensor  # [n, 2, S] bf16 (written by the Main Decoder step)
    counters: torch.Tensor        # [n, S] uint32 (int32 storage)
    last_attended: torch.Tensor   # [n] uint32 (int32 storage)
    next_prior: torch.Tensor      # [n, 2, S] bf16
    attended_token_index: torch.Tensor  # [n] int64
    invalid_state: torch.Tensor   # [n] int32
    decoder_steps: torch.Tensor   # [n] int64
    ignored_terminal_tokens: int = 3
    short_text_no_prior_max_tokens: int = 5
    lookahead: int = 6
    sink_threshold: int = 4

    @property
    def n(self) -> int:
        return int(self.text_length.shape[0])

    @property
    def token_stride(self) -> int:
        return int(self.alignment_scores.shape[2])

    @staticmethod
    def allocate(text_lengths, token_stride: int = 512, initial_attended: int = 1, device="cuda",
                 **contract) -> "AlignmentBatch":
        n = len(text_lengths)
        z = lambda *s, dt: torch.zeros(*s, dtype=dt, device=device)
        return AlignmentBatch(
            text_length=torch.as_tensor(list(text_lengths), dtype=torch.int32, device=device),
            alignment_scores=z(n, 2, token_stride, dt=torch.bfloat16),
            counters=z(n, token_stride, dt=torch.int32),
            last_attended=torch.full((n,), initial_attended, dtype=torch.int32, device=device),
            next_prior=z(n, 2, token_stride, dt=torch.bfloat16),
            attended_token_index=z(n, dt=torch.int64), invalid_state=z(n, dt=torch.int32),
            decoder_steps=z(n, dt=torch.int64), **contract)

    def c_struct(self, frame: Optional[StreamBatch] = None, unfinished=None, forbid_eos=None,
                 finished=None, end_frame_index=None, active=None) -> L.AlignmentBatch:
        if frame is not None:
            unfinished = frame.unfinished if unfinished is None else unfinished
            forbid_eos = frame.forbid_eos if forbid_eos is None else forbid_eos
            finished = frame.finished if finished is None else finished
            end_frame_index = frame.end_frame_index if end_frame_index is None else end_frame_index
            active = frame.active if active is None else active
        b = L.AlignmentBatch()
        b.n_sessions = self.n
        b.token_stride = self.token_stride
        b.ignored_terminal_tokens = self.ignored_terminal_tokens
        b.short_text_no_prior_max_tokens = self.short_text_no_prior_max_tokens
        b.lookahead = self.lookahead
        b.sink_threshold = self.sink_threshold
        for name in ("text_length", "alignment_scores", "counters", "last_attended", "next_prior",
                     "attended_token_index", "invalid_state"):
            setattr(b, name, getattr(self, name).data_ptr())
        b.unfinished = unfinished.data_ptr() if unfinished is not None else None
        b.active = active.data_ptr() if active is not None else None
        if forbid_eos is not None:
            b.decoder_steps = self.decoder_steps.data_ptr()
            b.forbid_eos = forbid_eos.data_ptr()
        if finished is not None and end_frame_index is not None:
            b.end_frame_index = end_frame_index.data_ptr()
            b.finished = finished.data_ptr()
        return b

    def gate(self, frame: Optional[StreamBatch] = None, stream=None, **outputs) -> None:
        cb = self.c_struct(frame, **outputs)
        status = L.lib.mtt_b200_launch_alignment_batch(ctypes.byref(cb), _stream(stream))
        if status != L.STATUS_OK:
            raise RuntimeError(f"mtt_b200_launch_alignment_batch failed with status {status}")
