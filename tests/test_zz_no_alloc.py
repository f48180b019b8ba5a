"""The allocation-free frame entry point (its scratch lives in a static device
array inside the library, for callers that cannot call cudaMalloc where frames
run: TensorRT enqueue, CUDA-graph capture, real-time threads) must produce
exactly what the workspace entry point produces, on two calls in a row, and
must refuse a batch whose scratch would not fit its 2 MiB array.

Called through the C ABI with ctypes.  This file is collected last on
purpose; it builds all of its own state so it also runs alone.
"""
import ctypes

import numpy as np
import pytest
import torch

from magpie_tts_rt_b200.model import EMBED, POSITIONS, SHAPE_BASELINE, VOCAB, make_weights

pytestmark = pytest.mark.gpu

STATIC_WORKSPACE_TOO_SMALL = -4


def _entry():
    from magpie_tts_rt_b200 import _lib as L
    fn = L.lib.mtt_b200_launch_local_ar_frame_static_workspace
    fn.restype = ctypes.c_int32
    fn.argtypes = [ctypes.POINTER(L.Shape), ctypes.POINTER(L.Weights), ctypes.POINTER(L.SamplingConfig),
                   ctypes.POINTER(L.StreamBatch), ctypes.c_void_p]
    return L, fn


def _batch(n, seed):
    from magpie_tts_rt_b200.local_ar import StreamBatch
    g = torch.Generator().manual_seed(seed)
    b = StreamBatch.allocate(n)
    b.decoder_hidden.copy_(torch.randn(n, 2, EMBED, generator=g).to(torch.bfloat16))
    b.unfinished.copy_(torch.tensor([i % 3 == 0 for i in range(n)]))
    b.forbid_eos.copy_(torch.tensor([i % 3 == 1 for i in range(n)]))
    b.rng_seed.copy_(torch.arange(n) * 7 + 1)
    b.rng_counter.copy_(torch.arange(n) * 16)
    b.logits_out = torch.zeros(n, POSITIONS, 2, VOCAB, dtype=torch.bfloat16, device="cuda")
    return b


def _outputs(b):
    return [t.clone() for t in (b.codec_tokens, b.rng_counter, b.invalid_rows, b.end_frame_index,
                                b.next_embedding, b.logits_out)]


def test_static_workspace_entry_matches_workspace_entry():
    from magpie_tts_rt_b200.local_ar import LocalArEngine
    L, fn = _entry()
    w = make_weights(SHAPE_BASELINE, seed=31, profile="parity")
    n = 6
    eng = LocalArEngine(w, max_streams=n)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    ref = _batch(n, 1)
    got = _batch(n, 1)
    for call in range(2):  # two calls in a row; counters carry over between them
        eng.frame(ref)
        cb = got.c_struct()
        status = fn(ctypes.byref(eng._shape), ctypes.byref(eng._w), ctypes.byref(eng._sampling),
                    ctypes.byref(cb), stream)
        assert status == 0, status
        torch.cuda.synchronize()
        for a, b in zip(_outputs(ref), _outputs(got)):
            assert torch.equal(a, b), call
        assert int(got.invalid_rows.abs().sum()) == 0
        np.testing.assert_array_equal(got.rng_counter.cpu().numpy(), (np.arange(n) * 16) + 16 * (call + 1))


def test_static_workspace_entry_rejects_oversized_batch():
    from magpie_tts_rt_b200.local_ar import LocalArEngine
    L, fn = _entry()
    w = make_weights(SHAPE_BASELINE, seed=32, profile="baseline", with_final=False)
    eng = LocalArEngine(w, max_streams=1)
    n = 64  # 64 sessions x CFG needs about 3.3 MB of scratch
    assert L.lib.mtt_b200_local_ar_frame_workspace_size(ctypes.byref(eng._shape), n, 1) > (2 << 20)
    b = _batch(n, 2)
    b.codec_tokens.fill_(-9)
    status = fn(ctypes.byref(eng._shape), ctypes.byref(eng._w), ctypes.byref(eng._sampling),
                ctypes.byref(b.c_struct()), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert status == STATIC_WORKSPACE_TOO_SMALL
    assert int((b.codec_tokens != -9).sum()) == 0
