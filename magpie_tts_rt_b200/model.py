"""Local AR model shapes, weight container and seeded synthetic weights.

The Local AR codebook predictor of MagpieTTS-RT is a small causal pre-LN
Transformer run for 16 positions per decoder step (8 codebooks x frame-stack 2):

* ``local_transformer_in_projection``: Linear 768 -> d (+bias), or Identity when
  d == 768 (``reference/nemo-oracle-overlay/nemo/collections/tts/models/
  magpietts.py:1347-1352``);
* learnable position embedding table [18, d] (``magpietts.py:1360-1361``,
  ``transformer_2501.py:1191``);
* L layers of LN(no bias) -> qkv(no bias) -> causal attention (head width 64,
  scale 1/8) -> o_net(no bias) -> +res -> LN -> FFN1 (kernel-1 conv, no bias)
  -> GELU-tanh -> FFN2 -> +res (``transformer_2501.py:405-442,761-851``,
  ``ffn_modules.py:187-290``);
* 16 per-position output heads Linear d -> 2024 (+bias)
  (``magpietts.py:1363-1369``);
* 16 audio embedding tables [2024, 768] shared with the Main Decoder
  (``magpietts.py:1305-1308``);
* the Main Decoder final projection [16*2024, 768] (+bias) used by EOS
  (``plugins/local_ar_plugins.cu:1372-1432``).

Two shapes are in play: the NeMo-default shape the benchmarks use
(``SHAPE_BASELINE``: d=256, 1 layer, 4 heads, FFN 1024, in-projection) and the
reference bundle's accepted shape (``SHAPE_SOFIA``: d=768, 2 layers, 12 heads,
FFN 3072, identity in-projection; ``tools/export/local_ar_wrapper.py:25-47``).

All tensors use PyTorch's [out_features, in_features] layout (K contiguous).
"""
from __future__ import annotations

from dataclasses import dataclass, fields
from typing import Optional

import torch

VOCAB = 2024
CODEBOOK = 2016
EOS_ID = 2017
EMBED = 768
POSITIONS = 16
CODEBOOKS = 8
FRAMES = 2
POSITION_TABLE_ROWS = 18
HEAD_DIM = 64
TOP_K = 80
TEMPERATURE = 0.6
CFG_SCALE = 2.5
FINAL_ROWS = POSITIONS * VOCAB  # 32384


@dataclass(frozen=True)
class LocalArShape:
    d_model: int
    n_layers: int
    n_heads: int
    d_ffn: int

    @property
    def in_projection(self) -> bool:
        return self.d_model != EMBED

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_heads

    def validate(self) -> None:
        if self.d_model % self.n_heads or self.head_dim != HEAD_DIM:
            raise ValueError(f"head width must be {HEAD_DIM}: {self}")
        if self.d_model % 64 or self.d_ffn % 64:
            raise ValueError(f"d_model and d_ffn must be multiples of 64: {self}")

    def layer_params(self) -> int:
        d, f = self.d_model, self.d_ffn
        return 2 * d + 3 * d * d + d * d + 2 * d * f

    def frame_weight_params(self) -> int:
        """Unique weight parameters read by one 16-position frame step."""
        d = self.d_model
        p = self.n_layers * self.layer_params() + POSITIONS * d
        p += POSITIONS * (VOCAB * d + VOCAB)
        if self.in_projection:
            p += EMBED * d + d
        return p

    def macs_per_row(self) -> int:
        """Multiply-accumulates per CFG row per frame (linear layers + attention)."""
        d, f = self.d_model, self.d_ffn
        per_pos = self.n_layers * (3 * d * d + d * d + 2 * d * f) + d * VOCAB
        if self.in_projection:
            per_pos += EMBED * d
        attn = self.n_layers * sum(2 * (p + 1) * d for p in range(POSITIONS))
        return POSITIONS * per_pos + attn


SHAPE_BASELINE = LocalArShape(d_model=256, n_layers=1, n_heads=4, d_ffn=1024)
SHAPE_SOFIA = LocalArShape(d_model=768, n_layers=2, n_heads=12, d_ffn=3072)


@dataclass
class LocalArWeights:
    shape: LocalArShape
    in_proj_w: Optional[torch.Tensor]  # [d, 768]
    in_proj_b: Optional[torch.Tensor]  # [d]
    pos: torch.Tensor  # [18, d]
    ln_self: torch.Tensor  # [L, d]
    qkv: torch.Tensor  # [L, 3d, d]; rows q | k | v, heads contiguous inside each
    o: torch.Tensor  # [L, d, d]
    ln_ff: torch.Tensor  # [L, d]
    ffn1: torch.Tensor  # [L, F, d]
    ffn2: torch.Tensor  # [L, d, F]
    head_w: torch.Tensor  # [16, 2024, d]
    head_b: torch.Tensor  # [16, 2024]
    emb: torch.Tensor  # [16, 2024, 768]
    final_w: torch.Tensor  # [32384, 768]
    final_b: torch.Tensor  # [32384]

    def tensors(self):
        for f in fields(self):
            if f.name == "shape":
                continue
            yield f.name, getattr(self, f.name)

    def to(self, dtype: torch.dtype) -> "LocalArWeights":
        kw = {n: (t.to(dtype) if t is not None else None) for n, t in self.tensors()}
        return LocalArWeights(shape=self.shape, **kw)


def make_weights(
    shape: LocalArShape = SHAPE_BASELINE,
    seed: int = 0,
    dtype: torch.dtype = torch.bfloat16,
    profile: str = "baseline",
    with_final: bool = True,
) -> LocalArWeights:
    """Seeded synthetic weights on the CPU.

    ``profile="baseline"`` draws every parameter from N(0, 0.02), as the
    benchmark configurations specify.  ``profile="parity"`` uses
    variance-preserving scales (LN weights 1 + N(0, 0.1), linear weights
    N(0, 1/fan_in)) so that every sub-layer moves the logits and a wrong
    attention or FFN cannot hide under the comparison tolerance.
    """
    shape.validate()
    g = torch.Generator().manual_seed(seed)
    d, f, L = shape.d_model, shape.d_ffn, shape.n_layers

    def normal(*size, std):
        return torch.empty(size, dtype=torch.float32).normal_(0.0, std, generator=g)

    if profile == "baseline":
        lin = lambda out_f, in_f, *lead: normal(*lead, out_f, in_f, std=0.02)
        vec = lambda *size: normal(*size, std=0.02)
        ln = lambda *size: normal(*size, std=0.02)
        table_std = 0.02
    elif profile == "parity":
        lin = lambda out_f, in_f, *lead: normal(*lead, out_f, in_f, std=in_f ** -0.5)
        vec = lambda *size: normal(*size, std=0.1)
        ln = lambda *size: 1.0 + normal(*size, std=0.1)
        table_std = 1.0
    else:
        raise ValueError(profile)

    w = dict(
        in_proj_w=lin(d, EMBED) if shape.in_projection else None,
        in_proj_b=vec(d) if shape.in_projection else None,
        pos=normal(POSITION_TABLE_ROWS, d, std=0.02 if profile == "baseline" else 0.5),
        ln_self=ln(L, d),
        qkv=lin(3 * d, d, L),
        o=lin(d, d, L),
        ln_ff=ln(L, d),
        ffn1=lin(f, d, L),
        ffn2=lin(d, f, L),
        head_w=lin(VOCAB, d, POSITIONS),
        head_b=vec(POSITIONS, VOCAB),
        emb=normal(POSITIONS, VOCAB, EMBED, std=table_std),
    )
    if with_final:
        w["final_w"] = lin(FINAL_ROWS, EMBED)
        w["final_b"] = vec(FINAL_ROWS)
    else:
        w["final_w"] = torch.zeros(0, EMBED)
        w["final_b"] = torch.zeros(0)
    out = LocalArWeights(shape=shape, **w)
    return out.to(dtype)
