"""Main Decoder one-step: shapes, weight container, seeded synthetic weights
and the batched device engine.

One Main Decoder step advances every session by one decoder position
(``tools/export/main_decoder_wrapper.py:778-911``, MainDecoderStepWrapper):
the codec-token embedding sum of the previous frame pair (the Local AR frame's
``next_embedding``) plus the learnable position embedding, then 12 pre-LN
layers of

* LN -> qkv (768 -> 3 x 12 x 64, no bias) -> the new key/value written at the
  session's position -> attention over positions [0, position] of the
  session's cache (scale 1/8, key mask) -> o_net (no bias) -> +res;
* LN -> cross-attention query (768 -> 128, one head) -> attention over the
  session's text keys (scale 128^-1/2, condition mask), renormalised by the
  alignment prior on layers 2..10 -> context -> o_net (128 -> 768) -> +res;
  the probabilities of layers 4, 5, 8, 9 are averaged into the step's
  alignment scores;
* LN -> FFN (kernel-one convolutions 768 -> 3072 -> 768, GELU-tanh) -> +res;

then the output LayerNorm: the [2, 768] decoder hidden state the Local AR
frame consumes.  Shapes are the reference bundle's accepted ones
(``main_decoder_wrapper.py:28-42``).

All matrices use PyTorch's [out_features, in_features] layout.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, fields
from typing import Optional

import torch

WIDTH = 768
LAYERS = 12
HEADS = 12
HEAD_DIM = 64
CROSS_DIM = 128
FFN = 3072
ALIGNMENT_LAYERS = (4, 5, 8, 9)
PRIOR_LAYERS = frozenset(range(2, 11))
REFERENCE_CACHE = 467      # SELF_CACHE_CAPACITY of the reference bundle
REFERENCE_PREFIX = 218     # PREFILL_LENGTH: the first step position
MAX_TEXT = 512


@dataclass
class MainDecoderWeights:
    pos: torch.Tensor      # [P, 768] learnable position embeddings (P >= cache capacity)
    ln_self: torch.Tensor  # [L, 768]
    qkv: torch.Tensor      # [L, 2304, 768]: q rows, k rows, v rows (12 heads x 64 each)
    o: torch.Tensor        # [L, 768, 768]
    ln_xq: torch.Tensor    # [L, 768] cross-attention query norm
    xq: torch.Tensor       # [L, 128, 768]
    xo: torch.Tensor       # [L, 768, 128]
    ln_ff: torch.Tensor    # [L, 768]
    ffn1: torch.Tensor     # [L, 3072, 768]
    ffn2: torch.Tensor     # [L, 768, 3072]
    norm_out: torch.Tensor  # [768]

    def tensors(self):
        for f in fields(self):
            yield f.name, getattr(self, f.name)

    def to(self, **kw) -> "MainDecoderWeights":
        return MainDecoderWeights(**{n: t.to(**kw).contiguous() for n, t in self.tensors()})


def make_main_decoder_weights(seed: int = 0, positions: int = 1024, layers: int = LAYERS,
                              dtype=torch.bfloat16) -> MainDecoderWeights:
    """Seeded synthetic weights: matrices ~N(0, 0.02), LayerNorm weights
    ~1 + N(0, 0.1), position embeddings ~N(0, 0.1) (CPU generator, so the
    same seed gives the same weights everywhere)."""
    g = torch.Generator().manual_seed(seed)

    def mat(*s, std=0.02):
        return (torch.randn(*s, generator=g) * std).to(dtype)

    def ln(*s):
        return (1.0 + torch.randn(*s, generator=g) * 0.1).to(dtype)

    return MainDecoderWeights(
        pos=mat(positions, WIDTH, std=0.1), ln_self=ln(layers, WIDTH), qkv=mat(layers, 3 * WIDTH, WIDTH),
        o=mat(layers, WIDTH, WIDTH), ln_xq=ln(layers, WIDTH), xq=mat(layers, CROSS_DIM, WIDTH),
        xo=mat(layers, WIDTH, CROSS_DIM), ln_ff=ln(layers, WIDTH), ffn1=mat(layers, FFN, WIDTH),
        ffn2=mat(layers, WIDTH, FFN), norm_out=ln(WIDTH))


def step_weight_bytes(layers: int = LAYERS) -> int:
    """Weight bytes one step reads: every layer matrix and LayerNorm weight,
    the output norm and one position row (bf16)."""
    per_layer = 3 * WIDTH * WIDTH + WIDTH * WIDTH + 2 * CROSS_DIM * WIDTH + 2 * FFN * WIDTH + 3 * WIDTH
    return 2 * (layers * per_layer + 2 * WIDTH)


# ---------------------------------------------------------------------------
# batched device engine
# ---------------------------------------------------------------------------

@dataclass
class MainDecoderBatch:
    """SoA device state of n sessions (see mtt_b200_main_decoder_batch_t)."""

    embedded: torch.Tensor     # [n, 768] bf16 (the Local AR frame's next_embedding)
    position: torch.Tensor     # [n] int64
    text_length: torch.Tensor  # [n] int32 (uint32 storage)
    self_k: torch.Tensor       # [n, L, 2, 12, cap, 64] bf16
    self_v: torch.Tensor
    self_mask: torch.Tensor    # [n, 2, cap] bool
    cross_k: torch.Tensor      # [n, L, 2, S, 128] bf16
    cross_v: torch.Tensor
    cond_mask: torch.Tensor    # [n, 2, S] bool
    prior: torch.Tensor        # [n, 2, S] bf16
    hidden: torch.Tensor       # [n, 2, 768] bf16 out
    alignment: torch.Tensor    # [n, 2, S] bf16 out
    status: torch.Tensor       # [n] int32 out
    active: Optional[torch.Tensor] = None
    # optional [n, 32] int32 out: the Local AR's EOS projection of `hidden`
    # (needs the engine's final projection); hand it to the frame's
    # StreamBatch.eos_projection
    eos_projection: Optional[torch.Tensor] = None
    eos_cfg_scale: float = 2.5

    @property
    def n(self) -> int:
        return int(self.position.shape[0])

    @property
    def cap(self) -> int:
        return int(self.self_k.shape[4])

    @property
    def token_stride(self) -> int:
        return int(self.cond_mask.shape[2])

    @staticmethod
    def allocate(n: int, cap: int = REFERENCE_CACHE, token_stride: int = 128, layers: int = LAYERS,
                 device="cuda") -> "MainDecoderBatch":
        bf = torch.bfloat16
        z = lambda *s, dt: torch.zeros(*s, dtype=dt, device=device)
        return MainDecoderBatch(
            embedded=z(n, WIDTH, dt=bf), position=z(n, dt=torch.int64), text_length=z(n, dt=torch.int32),
            self_k=z(n, layers, 2, HEADS, cap, HEAD_DIM, dt=bf), self_v=z(n, layers, 2, HEADS, cap, HEAD_DIM, dt=bf),
            self_mask=z(n, 2, cap, dt=torch.bool), cross_k=z(n, layers, 2, token_stride, CROSS_DIM, dt=bf),
            cross_v=z(n, layers, 2, token_stride, CROSS_DIM, dt=bf), cond_mask=z(n, 2, token_stride, dt=torch.bool),
            prior=z(n, 2, token_stride, dt=bf), hidden=z(n, 2, WIDTH, dt=bf),
            alignment=z(n, 2, token_stride, dt=bf), status=z(n, dt=torch.int32))

    def c_struct(self):
        from magpie_tts_rt_b200 import _lib as L
        b = L.MainDecoderBatch()
        b.n_sessions = self.n
        b.cache_capacity = self.cap
        b.token_stride = self.token_stride
        for f in ("embedded", "position", "text_length", "self_k", "self_v", "self_mask", "cross_k", "cross_v",
                  "cond_mask", "prior", "hidden", "alignment", "status"):
            setattr(b, f, getattr(self, f).data_ptr())
        b.active = self.active.data_ptr() if self.active is not None else None
        b.eos_projection = self.eos_projection.data_ptr() if self.eos_projection is not None else None
        b.eos_cfg_scale = float(self.eos_cfg_scale)
        return b


class MainDecoderEngine:
    """Device-resident Main Decoder weights and workspace for up to
    ``max_sessions`` sessions; ``step(batch)`` enqueues one decoder position
    for every session on the current (or given) CUDA stream."""

    def __init__(self, weights: MainDecoderWeights, max_sessions: int, token_stride: int = 128, device="cuda",
                 final_w: Optional[torch.Tensor] = None, final_b: Optional[torch.Tensor] = None):
        """final_w / final_b ([16 x 2024, 768] / [16 x 2024] bf16): the final
        projection, needed only for batches that ask for eos_projection."""
        from magpie_tts_rt_b200 import _lib as L
        self.device = torch.device(device)
        self.dev = weights.to(device=self.device, dtype=torch.bfloat16)
        self._w = L.MainDecoderWeights()
        for name, t in self.dev.tensors():
            setattr(self._w, name, t.data_ptr())
        self.final_w = final_w.to(self.device, torch.bfloat16).contiguous() if final_w is not None else None
        self.final_b = final_b.to(self.device, torch.bfloat16).contiguous() if final_b is not None else None
        self._w.final_w = self.final_w.data_ptr() if self.final_w is not None else None
        self._w.final_b = self.final_b.data_ptr() if self.final_b is not None else None
        self._w.n_layers = int(self.dev.qkv.shape[0])
        self._w.pos_rows = int(self.dev.pos.shape[0])
        self.max_sessions = max_sessions
        self.token_stride = token_stride
        size = L.lib.mtt_b200_main_decoder_workspace_size(max_sessions, token_stride)
        if size == 0:
            raise ValueError("bad max_sessions / token_stride")
        self.workspace = torch.empty(size, dtype=torch.uint8, device=self.device)

    def step(self, batch: MainDecoderBatch, stream=None) -> None:
        from magpie_tts_rt_b200 import _lib as L
        if batch.n > self.max_sessions or batch.token_stride != self.token_stride:
            raise ValueError("batch does not fit this engine")
        if stream is None:
            stream = torch.cuda.current_stream(self.device)
        cb = batch.c_struct()
        status = L.lib.mtt_b200_launch_main_decoder_step(
            ctypes.byref(self._w), ctypes.byref(cb), ctypes.c_void_p(self.workspace.data_ptr()),
            self.workspace.numel(), ctypes.c_void_p(stream.cuda_stream))
        if status != L.STATUS_OK:
            raise RuntimeError(f"mtt_b200_launch_main_decoder_step failed with status {status}")
