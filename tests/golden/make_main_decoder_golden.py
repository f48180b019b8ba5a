"""Generate ``tests/golden/main_decoder.npz``: Main Decoder steps computed by
the reference's own wrapper (``tools/export/main_decoder_wrapper.py``
MainDecoderStepWrapper.forward) on NeMo's ``transformer_2501.Transformer``
built with the accepted shape (12 layers, d 768, 12 heads, FFN 3072 with
kernel-one convolutions, one 128-wide cross-attention head, learnable
positions, output norm), in bf16 on the CPU.

Run where the reference tree is present:
    python tests/golden/make_main_decoder_golden.py

Weights come from ``make_main_decoder_weights(seed)`` and the per-session
state from ``oracle.main_decoder.make_step_inputs(seed, ...)`` (CPU
generators, reproducible anywhere), so the fixture stores only the case
parameters and the outputs: the hidden state [2, 768], the alignment scores
[2, T] and the key / value rows written at the step's position [12, 2, 768],
as bf16 bits.  The script also checks that ``oracle/main_decoder.py`` gives
the same bits.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, HERE)

import make_golden as MG  # noqa: E402  (imports the reference with its three stubs)
from magpie_tts_rt_b200.main_decoder import make_main_decoder_weights  # noqa: E402
from oracle import main_decoder as OMD  # noqa: E402

OUT = os.path.join(HERE, "main_decoder.npz")
WEIGHT_SEED = 7
CAP = 467  # the reference wrapper's SELF_CACHE_CAPACITY
# (state seed, text length, position)
CASES = [(1, 40, 300), (2, 128, 466), (3, 7, 218), (4, 512, 350)]


def bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def reference_wrapper(w):
    T2501, MDW = MG.T2501, MG.MDW
    dec = T2501.Transformer(n_layers=12, d_model=768, d_ffn=3072, sa_n_heads=12, kernel_size=1,
                            has_xattn=True, xa_d_memory=768, xa_n_heads=1, xa_d_head=128, is_causal=True,
                            apply_norm_to_cond=True, apply_norm_out=True, use_learnable_pos_emb=True,
                            max_length_causal_mask=w.pos.shape[0]).to(torch.bfloat16)
    with torch.no_grad():
        dec.position_embeddings.weight.copy_(w.pos)
        dec.norm_out.weight.copy_(w.norm_out)
        for l, layer in enumerate(dec.layers):
            layer.norm_self.weight.copy_(w.ln_self[l])
            layer.self_attention.qkv_net.weight.copy_(w.qkv[l])
            layer.self_attention.o_net.weight.copy_(w.o[l])
            layer.norm_xattn_query.weight.copy_(w.ln_xq[l])
            layer.cross_attention.q_net.weight.copy_(w.xq[l])
            layer.cross_attention.o_net.weight.copy_(w.xo[l])
            layer.norm_pos_ff.weight.copy_(w.ln_ff[l])
            layer.pos_ff.proj.conv.weight.copy_(w.ffn1[l][:, :, None])
            layer.pos_ff.o_net.conv.weight.copy_(w.ffn2[l][:, :, None])
    # the accepted-model check needs a full MagpieTTSModel; the forward uses
    # only the decoder, the audio embeddings and the cache positions
    wrapper = MDW.MainDecoderStepWrapper.__new__(MDW.MainDecoderStepWrapper)
    torch.nn.Module.__init__(wrapper)
    wrapper.decoder = dec
    wrapper.register_buffer("cache_positions", torch.arange(MDW.SELF_CACHE_CAPACITY, dtype=torch.long),
                            persistent=False)
    return wrapper, MDW


def run_reference(wrapper, MDW, inp):
    """MainDecoderStepWrapper.forward after its embedding sum (the step's
    embedded input is given)."""
    T = inp.prior.shape[1]
    wrapper._embed_codec_tokens = lambda tokens: inp.embedded.reshape(1, 1, -1)
    args = [torch.zeros((1, 8, 2), dtype=torch.long), torch.tensor(inp.position, dtype=torch.long),
            torch.zeros((), dtype=torch.int32), inp.prior.reshape(2, 1, T), inp.cond_mask]
    for l in range(12):
        args += [inp.self_k[l].permute(0, 2, 1, 3).contiguous(), inp.self_v[l].permute(0, 2, 1, 3).contiguous(),
                 inp.self_mask.clone(), inp.cross_k[l].reshape(2, T, 1, 128), inp.cross_v[l].reshape(2, T, 1, 128)]
    with torch.no_grad():
        out = wrapper(*args)
    p = inp.position
    k_new = torch.stack([out[3 + 3 * l][:, p].reshape(2, 768) for l in range(12)])
    v_new = torch.stack([out[4 + 3 * l][:, p].reshape(2, 768) for l in range(12)])
    return out[0], out[1], k_new, v_new


def main():
    w = make_main_decoder_weights(WEIGHT_SEED, positions=CAP)
    wrapper, MDW = reference_wrapper(w)
    out = {"n_cases": np.int32(len(CASES)), "weight_seed": np.int64(WEIGHT_SEED), "cap": np.int64(CAP)}
    for i, (seed, T, pos) in enumerate(CASES):
        inp = OMD.make_step_inputs(seed, T, pos, CAP)
        hidden, align, k_new, v_new = run_reference(wrapper, MDW, inp)
        mine = OMD.step(w, inp)
        for a, b, name in ((hidden, mine.hidden, "hidden"), (align, mine.alignment, "alignment"),
                           (k_new, mine.k_new, "k_new"), (v_new, mine.v_new, "v_new")):
            assert torch.equal(a, b), f"case {i}: oracle differs from the reference wrapper in {name}"
        out[f"c{i}_case"] = np.array([seed, T, pos], np.int64)
        out[f"c{i}_hidden"] = bits(hidden)
        out[f"c{i}_alignment"] = bits(align)
        out[f"c{i}_k_new"] = bits(k_new)
        out[f"c{i}_v_new"] = bits(v_new)
    np.savez_compressed(OUT, **out)
    print(OUT, os.path.getsize(OUT))


if __name__ == "__main__":
    main()
