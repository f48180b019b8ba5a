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

from magpie_tts_rt_b200.model import EMBED, POSITIONS, SHAPE_BASELINE, SHAPE_SOFIA, VOCAB, make_weights

pytestmark = pytest.mark.gpu

STATIC_WORKSPACE_TOO_SMALL = -4
STATIC_BYTES = 2 << 20


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


def _call(fn, eng, batch, stream=None):
    stream = torch.cuda.current_stream() if stream is None else stream
    return fn(ctypes.byref(eng._shape), ctypes.byref(eng._w), ctypes.byref(eng._sampling),
              ctypes.byref(batch.c_struct()), ctypes.c_void_p(stream.cuda_stream))


@pytest.mark.parametrize("shape,n", [(SHAPE_BASELINE, 6), (SHAPE_SOFIA, 5)])
def test_static_workspace_entry_matches_workspace_entry(shape, n):
    from magpie_tts_rt_b200.local_ar import LocalArEngine
    L, fn = _entry()
    w = make_weights(shape, seed=31, profile="parity")
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


def _largest_fitting(L, eng, cfg=1):
    size = lambda n: L.lib.mtt_b200_local_ar_frame_workspace_size(ctypes.byref(eng._shape), n, cfg)
    n = 1
    while size(n + 1) <= STATIC_BYTES:
        n += 1
    return n


def test_static_workspace_entry_boundary():
    """The largest batch whose workspace size fits the 2 MiB array runs (and
    matches the workspace entry); one session more is rejected untouched."""
    from magpie_tts_rt_b200.local_ar import LocalArEngine
    L, fn = _entry()
    w = make_weights(SHAPE_BASELINE, seed=33, profile="parity")
    probe = LocalArEngine(w, max_streams=1)
    n = _largest_fitting(L, probe)
    assert n >= 32
    eng = LocalArEngine(w, max_streams=n + 1)
    ref, got = _batch(n, 4), _batch(n, 4)
    eng.frame(ref)
    assert _call(fn, eng, got) == 0
    torch.cuda.synchronize()
    for a, b in zip(_outputs(ref), _outputs(got)):
        assert torch.equal(a, b)
    over = _batch(n + 1, 5)
    over.codec_tokens.fill_(-9)
    assert _call(fn, eng, over) == STATIC_WORKSPACE_TOO_SMALL
    torch.cuda.synchronize()
    assert int((over.codec_tokens != -9).sum()) == 0


def test_static_workspace_entry_in_a_cuda_graph():
    """The use the entry exists for: after a first call on the device (which
    resolves the array's address), the call is recorded into a CUDA graph in
    global capture mode (where an allocation would fail the capture) and
    replayed; each replay gives bit for bit what the workspace entry gives for
    the same frame."""
    from magpie_tts_rt_b200.local_ar import LocalArEngine
    L, fn = _entry()
    w = make_weights(SHAPE_BASELINE, seed=34, profile="parity")
    n = 6
    eng = LocalArEngine(w, max_streams=n)
    ref, got = _batch(n, 6), _batch(n, 6)
    assert _call(fn, eng, got) == 0  # the first call on this device, outside any capture
    eng.frame(ref)
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side, capture_error_mode="global"):
        status = _call(fn, eng, got, stream=side)
    assert status == 0
    for replay in range(2):
        graph.replay()
        eng.frame(ref)
        torch.cuda.synchronize()
        for a, b in zip(_outputs(ref), _outputs(got)):
            assert torch.equal(a, b), replay
    del graph
