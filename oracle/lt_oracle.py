"""PyTorch-CPU restatement of the reference's 16-position Local AR frame.

TEST INFRASTRUCTURE ONLY: the checker for the CUDA path, and the timed CPU
baseline in ``bench.py``.  The product library never imports this module.

The forward follows, op for op and in the same tensor shapes (so that
PyTorch's bf16 rounding points are the same):

* ``tools/export/local_ar_wrapper.py:609-645``  ``_local_layer_step``
* ``tools/export/local_ar_wrapper.py:672-751``  ``LocalARWrapper.forward``
* ``reference/nemo-oracle-overlay/.../transformer_2501.py:1153-1232``
  ``Transformer.forward_incremental`` (position-embedding add :1191)
* ``reference/nemo-oracle-overlay/.../ffn_modules.py:268-290``
  (kernel-1 convolutions)
* ``reference/nemo-oracle-overlay/.../magpietts_modules.py:642-680``
  ``_execute_fixed_shape`` (in-projection of the next embedding)

Sampling, EOS and the embedding sum use the C oracle (``oracle.sampler``).
Streams are independent sessions: stream s owns CFG rows 2s (conditional)
and 2s+1 (unconditional), its own seed and its own RNG counter.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch
import torch.nn.functional as F

from magpie_tts_rt_b200.model import (
    CODEBOOK, EMBED, EOS_ID, POSITIONS, VOCAB, LocalArWeights,
)
from oracle import sampler as S

LAYER_NORM_EPSILON = 1.0e-5


def _bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> uint16 bit pattern array."""
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def layer_step(w: LocalArWeights, layer: int, x: torch.Tensor, keys: list, values: list):
    """One pre-LN layer for one position; x is [R, 1, d].

    local_ar_wrapper.py:609-645; transformer_2501.py:761-851 (the all-true
    mask multiplies are the identity and are omitted).
    """
    shape = w.shape
    R = x.shape[0]
    H, dh, d = shape.n_heads, shape.head_dim, shape.d_model
    normalized = F.layer_norm(x, (d,), w.ln_self[layer], None, LAYER_NORM_EPSILON)
    qkv = F.linear(normalized, w.qkv[layer]).reshape(R, 1, 3, H, dh)
    query, key_step, value_step = qkv.unbind(dim=2)
    k_all = torch.cat((*keys, key_step), dim=1)
    v_all = torch.cat((*values, value_step), dim=1)
    scores = torch.matmul(query.transpose(1, 2), k_all.transpose(1, 2).transpose(2, 3)) * (dh ** -0.5)
    probabilities = F.softmax(scores, dim=-1)
    attended = torch.matmul(probabilities, v_all.transpose(1, 2))
    attended = attended.transpose(1, 2).contiguous().reshape(R, 1, d)
    x = x + F.linear(attended, w.o[layer])
    normalized_ff = F.layer_norm(x, (d,), w.ln_ff[layer], None, LAYER_NORM_EPSILON)
    projected = F.conv1d(normalized_ff.transpose(1, 2), w.ffn1[layer].unsqueeze(-1))
    projected = F.gelu(projected, approximate="tanh")
    ff_out = F.conv1d(projected, w.ffn2[layer].unsqueeze(-1)).transpose(1, 2)
    return x + ff_out, key_step, value_step


def in_projection(w: LocalArWeights, rows: torch.Tensor) -> torch.Tensor:
    """rows [R, 1, 768] -> [R, 1, d] (Identity when d == 768)."""
    if w.in_proj_w is None:
        return rows
    return F.linear(rows, w.in_proj_w, w.in_proj_b)


@dataclass
class FrameResult:
    tokens: np.ndarray  # int64 [S, 16] position-major
    codec_tokens: np.ndarray  # int64 [S, 8, 2]
    counter: np.ndarray  # int64 [S]
    invalid: np.ndarray  # int32 [S] (max over positions)
    end_frame: np.ndarray  # int32 [S]
    next_embedding: np.ndarray  # uint16 bf16 bits [S, 768] (or f32 in fp32 mode)
    logits: Optional[np.ndarray] = None  # [S, 16, rows_per_stream, V] (bf16 bits or f32)


def run_frame(
    w: LocalArWeights,
    hidden: torch.Tensor,
    unfinished,
    finished,
    forbid_eos,
    seed,
    counter,
    params: S.SamplingParams = S.SamplingParams(),
    teacher_tokens: Optional[np.ndarray] = None,
    record_logits: bool = False,
    eos: bool = True,
) -> FrameResult:
    """One Local AR frame for S independent streams.

    ``hidden`` is [S, 2, 768] (CFG pair) or [S, 768] (no CFG), in the weights'
    dtype.  ``teacher_tokens`` [S, 16], when given, replaces the sampled token
    as the next position's input (the sampled tokens are still returned); the
    GPU parity tests use it to compare logits on the GPU's own token history.
    """
    cfg = hidden.dim() == 3
    S_ = hidden.shape[0]
    rows_per = 2 if cfg else 1
    R = S_ * rows_per
    dtype = w.pos.dtype
    flags = [np.broadcast_to(np.asarray(v, dtype=bool), (S_,)) for v in (unfinished, finished, forbid_eos)]
    seed = np.broadcast_to(np.asarray(seed, dtype=np.int64), (S_,))
    ctr = np.array(np.broadcast_to(np.asarray(counter, dtype=np.int64), (S_,)))
    invalid = np.zeros(S_, np.int32)
    tokens = np.zeros((S_, POSITIONS), np.int64)
    logit_rec = [] if record_logits else None

    with torch.no_grad():
        x_step = in_projection(w, hidden.reshape(R, 1, EMBED).to(dtype))
        keys = [[] for _ in range(w.shape.n_layers)]
        values = [[] for _ in range(w.shape.n_layers)]
        for p in range(POSITIONS):
            x = x_step + w.pos[p : p + 1].unsqueeze(0)
            for layer in range(w.shape.n_layers):
                x, k, v = layer_step(w, layer, x, keys[layer], values[layer])
                keys[layer].append(k)
                values[layer].append(v)
            logits = F.linear(x[:, 0, :], w.head_w[p], w.head_b[p])  # [R, V]
            if dtype == torch.bfloat16:
                lg = _bits(logits).reshape(S_, rows_per, VOCAB)
                lg_in = lg if cfg else lg[:, 0, :]
            else:
                lg = logits.float().numpy().reshape(S_, rows_per, VOCAB)
                lg_in = np.ascontiguousarray(lg[:, 0, :])
            if record_logits:
                logit_rec.append(lg.copy())
            tok, ctr, inv = S.sample(lg_in, flags[0], flags[1], flags[2], seed, ctr, params)
            tokens[:, p] = tok
            invalid = np.maximum(invalid, inv)
            feed = tok if teacher_tokens is None else np.asarray(teacher_tokens)[:, p]
            if p + 1 < POSITIONS:
                e = w.emb[p][torch.from_numpy(np.asarray(feed, dtype=np.int64))]  # [S, 768]
                e_rows = e.repeat_interleave(rows_per, dim=0).reshape(R, 1, EMBED)
                x_step = in_projection(w, e_rows)

    codec = np.stack([S.codec_layout(tokens[s]) for s in range(S_)])
    end = np.full(S_, -1, np.int32)
    for s in range(S_):
        need = eos and not (flags[0][s] or flags[1][s] or flags[2][s])
        guided = None
        if need:
            hb = _bits(hidden[s].to(torch.bfloat16)) if cfg else None
            guided = S.eos_guided(hb, _bits(w.final_w.to(torch.bfloat16)),
                                  _bits(w.final_b.to(torch.bfloat16)), params.cfg_scale)
        end[s] = S.eos_end_frame(guided, codec[s], flags[0][s], flags[1][s], flags[2][s]) if (need or flags[1][s]) else -1

    if dtype == torch.bfloat16:
        emb_bits = _bits(w.emb)
        next_emb = np.stack([S.embedding_sum(emb_bits, tokens[s]) for s in range(S_)])
    else:
        rows = []
        for s in range(S_):
            acc = w.emb[0][int(tokens[s, 0])].float()
            for p in range(1, POSITIONS):
                acc = acc + w.emb[p][int(tokens[s, p])].float()
            rows.append((acc / 16.0).numpy())
        next_emb = np.stack(rows).astype(np.float32)
    return FrameResult(
        tokens=tokens, codec_tokens=codec, counter=ctr, invalid=invalid, end_frame=end,
        next_embedding=next_emb,
        logits=np.stack(logit_rec, axis=1) if record_logits else None,
    )


__all__ = ["run_frame", "layer_step", "in_projection", "FrameResult", "CODEBOOK", "EOS_ID"]
