"""CPU restatement of the reference's Main Decoder one-step.

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline leg as the checker.  The product library never
imports this module.

``step`` follows ``tools/export/main_decoder_wrapper.py:812-911``
(MainDecoderStepWrapper.forward) op for op in bf16 on the CPU, with the eager
forwards of the oracle functions it calls: ``_OracleLayerNorm``
(``text_encoder_wrapper.py:30-46``), the self-attention of
``_OracleMainSelfAttentionDevicePosition`` (``main_decoder_wrapper.py:
188-228``), ``_cross_attention`` (:559-603) with
``_OracleMainCrossAttentionSoftmax`` (:101-122) and
``_OracleMainAttentionPriorNormalization`` (:293-309),
``_pointwise_feed_forward`` (:606-620), ``_OracleMainAlignmentMean``
(:325-345).  The same PyTorch operations in the same order give the same bf16
bits as the reference wrapper itself, which ``tests/golden/
make_main_decoder_golden.py`` runs to pin this restatement.

Layouts are this library's (``magpie_tts_rt_b200.main_decoder``): one
session's self-attention cache per layer is [2 rows][12 heads][capacity][64]
(the reference's is [2][capacity][12][64]); one key mask per row [2][capacity]
serves all layers (the reference keeps twelve copies, updated identically);
the cross-attention keys and values per layer are [2][T][128].
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

WIDTH = 768
HEADS = 12
HEAD_DIM = 64
CROSS_DIM = 128
ALIGNMENT_LAYERS = (4, 5, 8, 9)
PRIOR_LAYERS = frozenset(range(2, 11))
EPS = 1e-5


@dataclass
class StepInputs:
    embedded: torch.Tensor     # [768] bf16: the codec-token embedding sum (Local AR next_embedding)
    position: int              # absolute decoder position written by this step
    prior: torch.Tensor        # [2, T] bf16 attention prior (alignment controller output)
    cond_mask: torch.Tensor    # [2, T] bool condition (text) mask
    self_k: torch.Tensor       # [L, 2, 12, cap, 64] bf16
    self_v: torch.Tensor       # [L, 2, 12, cap, 64] bf16
    self_mask: torch.Tensor    # [2, cap] bool
    cross_k: torch.Tensor      # [L, 2, T, 128] bf16
    cross_v: torch.Tensor      # [L, 2, T, 128] bf16


@dataclass
class StepOutputs:
    hidden: torch.Tensor       # [2, 768] bf16 decoder hidden state (the Local AR input)
    alignment: torch.Tensor    # [2, T] bf16 alignment scores (the alignment controller input)
    k_new: torch.Tensor        # [L, 2, 768] bf16: the keys written at `position`
    v_new: torch.Tensor        # [L, 2, 768] bf16


def make_step_inputs(seed: int, text_length: int, position: int, cap: int, layers: int = 12,
                     embedded_scale: float = 0.05) -> StepInputs:
    """Seeded synthetic state of one session: caches ~N(0, 1), keys masked in
    up to `position`, a two-level prior (0.1 / 1.0, as the controller writes
    it), the unconditional row's condition mask keeping only the first text
    token (``main_decoder_wrapper.py:954-957,984-985``)."""
    g = torch.Generator().manual_seed(seed)
    bf = torch.bfloat16
    T = text_length
    mask = torch.zeros(2, cap, dtype=torch.bool)
    mask[:, :position] = True
    cond = torch.ones(2, T, dtype=torch.bool)
    cond[1, 1:] = False
    prior = torch.full((2, T), 0.1)
    prior[0, (torch.rand(T, generator=g) > 0.6)] = 1.0
    return StepInputs(
        embedded=(torch.randn(WIDTH, generator=g) * embedded_scale).to(bf), position=position,
        prior=prior.to(bf), cond_mask=cond,
        self_k=torch.randn(layers, 2, HEADS, cap, HEAD_DIM, generator=g).to(bf),
        self_v=torch.randn(layers, 2, HEADS, cap, HEAD_DIM, generator=g).to(bf),
        self_mask=mask,
        cross_k=torch.randn(layers, 2, T, CROSS_DIM, generator=g).to(bf),
        cross_v=torch.randn(layers, 2, T, CROSS_DIM, generator=g).to(bf))


def _layer_norm(x, weight):
    return F.layer_norm(x, (WIDTH,), weight, None, EPS)


def _query_mask(x, mask):
    return torch.where(mask.unsqueeze(-1), x, torch.zeros_like(x))


def step(w, inp: StepInputs) -> StepOutputs:
    """One decoder position for one session (both CFG rows)."""
    p = int(inp.position)
    L = w.qkv.shape[0]
    x = inp.embedded.reshape(1, 1, WIDTH).expand(2, -1, -1)
    x = x + w.pos[p].reshape(1, 1, WIDTH)  # position_embeddings(position).unsqueeze(0)
    x_mask = torch.ones((2, 1), dtype=torch.bool)
    mask = inp.self_mask.clone()
    mask[:, p] = True  # updated_mask
    active = p + 1
    am = mask[:, None, None, :active]
    valid = inp.cond_mask[:, None, None, :]
    prior = inp.prior.reshape(2, 1, -1)  # [2, 1, T] as the wrapper's attention_prior input
    aligns, k_new, v_new = [], [], []
    with torch.no_grad():
        for l in range(L):
            x = _query_mask(x, x_mask)
            h = _layer_norm(x, w.ln_self[l])
            qkv = F.linear(h, w.qkv[l]).reshape(2, 1, 3, HEADS, HEAD_DIM)
            q, k_step, v_step = qkv.unbind(dim=2)
            k_new.append(k_step.reshape(2, WIDTH))
            v_new.append(v_step.reshape(2, WIDTH))
            key_heads = inp.self_k[l].clone()  # [2, 12, cap, 64]
            value_heads = inp.self_v[l].clone()
            key_heads[:, :, p] = k_step[:, 0]
            value_heads[:, :, p] = v_step[:, 0]
            query_heads = q.transpose(1, 2).contiguous()
            scores = torch.matmul(query_heads, key_heads[..., :active, :].transpose(-1, -2).contiguous())
            scores = scores * HEAD_DIM ** -0.5
            scores = scores.masked_fill(~am, float("-inf"))
            probs = torch.softmax(scores, dim=-1)
            probs = probs.masked_fill(~am, 0.0)
            o = torch.matmul(probs, value_heads[..., :active, :])
            o = o.transpose(1, 2).contiguous().view(2, 1, WIDTH)
            x = x + F.linear(o, w.o[l])
            # cross attention
            hq = _layer_norm(x, w.ln_xq[l])
            qx = F.linear(hq, w.xq[l]).reshape(2, 1, 1, CROSS_DIM).transpose(1, 2)
            key = inp.cross_k[l].reshape(2, -1, 1, CROSS_DIM)
            vheads = inp.cross_v[l].reshape(2, -1, 1, CROSS_DIM).transpose(1, 2)
            kh = key.transpose(1, 2)
            s = torch.matmul(qx, kh.transpose(2, 3)) * (CROSS_DIM ** -0.5)
            s = s.masked_fill(~valid, float("-inf"))
            pr = F.softmax(s, dim=-1).masked_fill(~valid, 0.0)
            if l in PRIOR_LAYERS:
                pri = prior[:, None] + torch.finfo(prior.dtype).tiny
                num = pr * pri
                pr = num / num.sum(dim=-1, keepdim=True)
            ctx = torch.matmul(pr, vheads).transpose(1, 2).contiguous().view(2, 1, CROSS_DIM)
            if l in ALIGNMENT_LAYERS:
                aligns.append(pr[:, :, -1, :].mean(dim=1))
            x = x + F.linear(ctx, w.xo[l])
            # feed-forward (kernel-one convolutions)
            hf = _layer_norm(x, w.ln_ff[l])
            f = F.conv1d(hf.transpose(1, 2), w.ffn1[l][:, :, None])
            f = F.gelu(f, approximate="tanh")
            f = F.conv1d(f, w.ffn2[l][:, :, None]).transpose(1, 2)
            x = x + f
            x = _query_mask(x, x_mask)
        x = _layer_norm(x, w.norm_out)
        alignment = torch.stack(aligns, dim=1).mean(dim=1)
    return StepOutputs(hidden=x[:, -1, :].contiguous(), alignment=alignment.contiguous(),
                       k_new=torch.stack(k_new), v_new=torch.stack(v_new))
