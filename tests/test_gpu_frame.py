"""GPU parity of the batched Local AR frame against the oracle.

For every case:
* logits: the oracle is teacher-forced on the GPU's own tokens and its
  per-position logits must agree with the GPU's within the bf16 tolerance:
  every 2024-wide logits row within 1e-2 relative L2 error, and no single
  logit further than 5e-2 x the row RMS;
* tokens / RNG counter / invalid flag: the C oracle sampler applied to the
  GPU's logits must reproduce the GPU's tokens bit for bit;
* next-frame embedding: bit-exact sequential bf16 sum of the GPU tokens' rows;
* end_frame_index: the oracle EOS decision on the GPU tokens.
"""
import os

import numpy as np
import pytest
import torch

from magpie_tts_rt_b200.model import (
    EMBED, POSITIONS, SHAPE_BASELINE, SHAPE_SOFIA, VOCAB, LocalArShape, make_weights,
)
from oracle import lt_oracle
from oracle import sampler as S

pytestmark = pytest.mark.gpu

RTOL = 1e-2
PATH_AUTO, PHASE, FUSED, TILE, PAIR, SPLIT1, SPLIT2, SPLIT4, SPLIT8, SPLIT2X32, QUAD, OCTO = range(12)
SPLITS = [SPLIT1, SPLIT2, SPLIT4, SPLIT8, SPLIT2X32]
BOTH = [PHASE, FUSED, TILE, PAIR, QUAD, OCTO] + SPLITS
PATH_IDS = {PATH_AUTO: "auto", PHASE: "phase", FUSED: "cluster", TILE: "tile", PAIR: "pair", SPLIT1: "split1",
            SPLIT2: "split2", SPLIT4: "split4", SPLIT8: "split8", SPLIT2X32: "split2x32", QUAD: "quad",
            OCTO: "octo"}


def path_id(v):
    return PATH_IDS.get(v) if isinstance(v, int) and not isinstance(v, bool) and v in PATH_IDS else None


def bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def from_bits(b):
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16)


_weights_cache = {}


def weights(shape, seed, with_final=True):
    key = (shape, seed, with_final)
    if key not in _weights_cache:
        _weights_cache[key] = make_weights(shape, seed=seed, dtype=torch.bfloat16, profile="parity",
                                           with_final=with_final)
    return _weights_cache[key]


def run_gpu(engine, hidden, flags, seed, counter, forced=None, active=None, sentinel=False):
    from magpie_tts_rt_b200.local_ar import StreamBatch
    n = hidden.shape[0]
    cfg = hidden.dim() == 3
    rows = 2 if cfg else 1
    b = StreamBatch.allocate(n, cfg=cfg)
    b.decoder_hidden.copy_(hidden.reshape(n, rows, EMBED))
    uf, fi, fb = (torch.as_tensor(np.asarray(f, dtype=bool)).cuda() for f in flags)
    b.unfinished.copy_(uf); b.finished.copy_(fi); b.forbid_eos.copy_(fb)
    b.rng_seed.copy_(torch.as_tensor(np.asarray(seed, dtype=np.int64)))
    b.rng_counter.copy_(torch.as_tensor(np.asarray(counter, dtype=np.int64)))
    b.logits_out = torch.zeros(n, POSITIONS, rows, VOCAB, dtype=torch.bfloat16, device="cuda")
    if sentinel:
        b.codec_tokens.fill_(-7); b.invalid_rows.fill_(-7); b.end_frame_index.fill_(-7)
        b.next_embedding.fill_(7.0)
    if forced is not None:
        b.forced_tokens = torch.as_tensor(forced, dtype=torch.int64).cuda()
    if active is not None:
        b.active = torch.as_tensor(np.asarray(active, dtype=bool)).cuda()
    engine.frame(b)
    torch.cuda.synchronize()
    codec = b.codec_tokens.cpu().numpy()
    return dict(
        codec=codec,
        tokens=np.stack([codec[s].T.reshape(-1) for s in range(n)]),  # position-major
        counter=b.rng_counter.cpu().numpy(), invalid=b.invalid_rows.cpu().numpy(),
        end=b.end_frame_index.cpu().numpy(), next_emb=bits(b.next_embedding),
        logits=bits(b.logits_out),
    )


def logit_errors(gpu_bits, ref_bits):
    """Per logits row: relative L2 error and max element error / row RMS."""
    g = S.bf16_bits_to_f32(gpu_bits).astype(np.float64)
    r = S.bf16_bits_to_f32(ref_bits).astype(np.float64)
    rms = np.sqrt(np.mean(r * r, axis=-1))
    rel_l2 = np.linalg.norm(g - r, axis=-1) / np.linalg.norm(r, axis=-1)
    max_rel = np.max(np.abs(g - r), axis=-1) / rms
    return rel_l2, max_rel


def check_logits(gpu_bits, ref_bits, what):
    """bf16 tolerance: every logits row within 1e-2 relative (L2), and no
    single logit further than 5e-2 of the row RMS from the oracle."""
    rel_l2, max_rel = logit_errors(gpu_bits, ref_bits)
    assert rel_l2.max() <= RTOL, f"{what}: relative L2 error {rel_l2.max():.4g} > {RTOL}"
    assert max_rel.max() <= 5 * RTOL, f"{what}: max element error {max_rel.max():.4g} x row RMS"
    return float(rel_l2.max())


def check_frame(w, hidden, flags, seed, counter, gpu, params=S.SamplingParams(), streams=None):
    cfg = hidden.dim() == 3
    n = hidden.shape[0]
    streams = range(n) if streams is None else streams
    uf, fi, fb = (np.broadcast_to(np.asarray(f, dtype=bool), (n,)) for f in flags)
    seed = np.broadcast_to(np.asarray(seed, dtype=np.int64), (n,))
    counter = np.broadcast_to(np.asarray(counter, dtype=np.int64), (n,))
    sel = list(streams)
    r = lt_oracle.run_frame(w, hidden[sel], uf[sel], fi[sel], fb[sel], seed[sel], counter[sel], params,
                            teacher_tokens=gpu["tokens"][sel], record_logits=True, eos=False)
    rows = 2 if cfg else 1
    worst = check_logits(gpu["logits"][sel], r.logits.reshape(len(sel), POSITIONS, rows, VOCAB), "logits")
    emb_bits = bits(w.emb)
    fw, fbias = (bits(w.final_w), bits(w.final_b)) if w.final_w.numel() else (None, None)
    for j, s in enumerate(sel):
        ctr = int(counter[s])
        inv = 0
        for p in range(POSITIONS):
            lg = gpu["logits"][s, p]
            lg_in = lg[None] if cfg else lg[:1]
            tok, c2, iv = S.sample(lg_in, uf[s], fi[s], fb[s], seed[s], ctr, params)
            assert tok[0] == gpu["tokens"][s, p], (s, p)
            ctr = int(c2[0])
            inv = max(inv, int(iv[0]))
        assert gpu["counter"][s] == ctr, s
        assert gpu["invalid"][s] == inv, s
        np.testing.assert_array_equal(gpu["next_emb"][s], S.embedding_sum(emb_bits, gpu["tokens"][s]))
        enabled = not (uf[s] or fi[s] or fb[s])
        guided = None
        if enabled and fw is not None:
            hb = bits(hidden[s].reshape(rows, EMBED))
            if not cfg:
                hb = np.concatenate([hb, hb])
            guided = S.eos_guided(hb, fw, fbias, params.cfg_scale if cfg else 1.0)
        exp_end = S.eos_end_frame(guided, S.codec_layout(gpu["tokens"][s]), uf[s], fi[s], fb[s])
        assert gpu["end"][s] == exp_end, (s, gpu["end"][s], exp_end)
    return worst


@pytest.fixture(scope="module")
def engines():
    from magpie_tts_rt_b200.local_ar import LocalArEngine
    cache = {}

    def get(shape, seed, max_streams, cfg=True, argmax=False, with_final=True, path=PATH_AUTO, fold=True):
        key = (shape, seed, max_streams, cfg, argmax, with_final, path, fold)
        if key not in cache:
            cache[key] = LocalArEngine(weights(shape, seed, with_final), max_streams=max_streams, cfg=cfg,
                                       argmax=argmax, path=path, fold_in_projection=fold)
        return cache[key]
    return get


def _hidden(n, seed, cfg=True):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(n, 2 if cfg else 1, EMBED, generator=g).to(torch.bfloat16).reshape(
        (n, 2, EMBED) if cfg else (n, EMBED))


FLAGS6 = ([0, 1, 0, 0, 0, 1], [0, 0, 0, 1, 0, 1], [0, 0, 1, 0, 0, 0])  # incl. an invalid overlap


@pytest.mark.parametrize("shape,n,path,fold", [
    (SHAPE_BASELINE, 6, PHASE, True), (SHAPE_BASELINE, 6, FUSED, True), (SHAPE_BASELINE, 11, FUSED, True),
    (SHAPE_BASELINE, 6, TILE, True), (SHAPE_BASELINE, 11, TILE, True), (SHAPE_BASELINE, 11, TILE, False),
    (SHAPE_BASELINE, 11, FUSED, False), (SHAPE_BASELINE, 6, PAIR, True), (SHAPE_BASELINE, 11, PAIR, True),
    (SHAPE_BASELINE, 20, PAIR, True), (SHAPE_BASELINE, 11, PAIR, False), (SHAPE_SOFIA, 3, PHASE, True)] +
    [(SHAPE_BASELINE, n, sp, fold) for sp in SPLITS for n, fold in ((6, True), (11, True), (20, True), (11, False))] +
    [(SHAPE_BASELINE, 24, SPLIT2X32, True), (SHAPE_BASELINE, 17, SPLIT2X32, False)] +
    [(SHAPE_BASELINE, n, qp, fold) for qp in (QUAD, OCTO)
     for n, fold in ((6, True), (11, True), (20, True), (24, True), (17, False))])
def test_frame_matches_oracle(engines, shape, n, path, fold):
    w = weights(shape, 21)
    eng = engines(shape, 21, 24, path=path, fold=fold)
    assert eng.path == path
    hidden = _hidden(n, 5)
    flags = tuple(np.resize(np.asarray(f), n) for f in FLAGS6)
    seed = np.resize(np.array([1234, 0, 7, (1 << 32) - 1, 99, 5]), n)
    counter = np.resize(np.array([0, 16, 3200, 48, S.MAX_COUNTER - 3, 0]), n)
    gpu = run_gpu(eng, hidden, flags, seed, counter)
    check_frame(w, hidden, flags, seed, counter, gpu)


def test_auto_path_for_the_benchmark_shape(engines):
    """One wave of 16-CTA clusters: the cluster kernel (latency); then the
    split kernel with the widest cluster whose tiles fit in one wave (8, then
    4 CTAs per 8 sessions); the quad kernel while its 16-session tiles fit in
    one wave of 4-CTA clusters; split x2; the pair kernel while its
    16-session tiles fit in one wave; the tile kernel for the largest
    batches; other shapes: phase kernels."""
    from magpie_tts_rt_b200 import _lib as L
    eng = engines(SHAPE_BASELINE, 21, 16)
    assert eng.path == FUSED
    assert eng.path_for(1) == FUSED
    assert eng.path_for(56) == FUSED
    c8 = L.lib.mtt_b200_local_ar_frame_path_clusters(SPLIT8)
    c4 = L.lib.mtt_b200_local_ar_frame_path_clusters(SPLIT4)
    c2 = L.lib.mtt_b200_local_ar_frame_path_clusters(SPLIT2)
    assert L.lib.mtt_b200_local_ar_frame_path_clusters(FUSED) == 7
    assert 7 < c8 < c4 < c2 <= 148
    assert eng.path_for(8 * 7 + 1) == SPLIT8
    assert eng.path_for(8 * c8) == SPLIT8
    assert eng.path_for(8 * c8 + 1) == SPLIT4
    assert eng.path_for(8 * c4) == SPLIT4
    cq = L.lib.mtt_b200_local_ar_frame_path_clusters(QUAD)
    assert 8 * c4 < 16 * cq < 8 * c2
    assert eng.path_for(8 * c4 + 1) == QUAD
    assert eng.path_for(16 * cq) == QUAD
    assert eng.path_for(16 * cq + 1) == SPLIT2
    assert eng.path_for(8 * c2) == SPLIT2
    cp = L.lib.mtt_b200_local_ar_frame_path_clusters(PAIR)
    assert 8 * c2 < 16 * cp
    assert eng.path_for(8 * c2 + 1) == PAIR
    assert eng.path_for(16 * cp) == PAIR
    assert eng.path_for(16 * cp + 1) == TILE
    assert engines(SHAPE_SOFIA, 21, 1, with_final=False).path == PHASE


@pytest.mark.parametrize("path", BOTH, ids=path_id)
def test_frame_sequence_counters(engines, path):
    """Three consecutive frames of 4 sessions: the counter advances by 16 per
    frame and every frame matches the oracle (sequence_contract.py:95-160)."""
    shape = SHAPE_BASELINE
    w = weights(shape, 22)
    eng = engines(shape, 22, 4, path=path)
    seed = np.array([1234, 1, 2, 3])
    counter = np.zeros(4, np.int64)
    for f in range(3):
        hidden = _hidden(4, 100 + f)
        forbid = np.full(4, f < 2)
        flags = (np.zeros(4, bool), np.zeros(4, bool), forbid)
        gpu = run_gpu(eng, hidden, flags, seed, counter)
        check_frame(w, hidden, flags, seed, counter, gpu)
        np.testing.assert_array_equal(gpu["counter"], counter + 16)
        if f < 2:
            assert (gpu["end"] == -1).all()
        counter = gpu["counter"]


@pytest.mark.parametrize("path", BOTH, ids=path_id)
def test_inactive_streams_untouched(engines, path):
    shape = SHAPE_BASELINE
    w = weights(shape, 21)
    eng = engines(shape, 21, 8, path=path)
    n = 5
    hidden = _hidden(n, 9)
    flags = (np.zeros(n, bool), np.zeros(n, bool), np.ones(n, bool))
    seed = np.arange(n) + 10
    counter = np.arange(n) * 16
    active = np.array([1, 0, 1, 0, 1], bool)
    gpu = run_gpu(eng, hidden, flags, seed, counter, active=active, sentinel=True)
    for s in np.nonzero(~active)[0]:
        assert (gpu["codec"][s] == -7).all() and gpu["invalid"][s] == -7 and gpu["end"][s] == -7
        assert gpu["counter"][s] == counter[s]
    check_frame(w, hidden, flags, seed, counter, gpu, streams=np.nonzero(active)[0])


@pytest.mark.parametrize("path", BOTH, ids=path_id)
def test_frames_fill_the_emission_aggregate(path):
    """launch_finalize_local_step folded into the frame call
    (synthesis_kernels.cu:53-86): four frames write their [8][2] tokens
    straight into the [n][8][8] emission aggregate at frame offsets 0, 2, 4, 6
    (the same tokens, counters and EOS as the [n][8][2] layout), and
    finished_latch is set exactly where end_frame_index is 0 or 1, and
    codec_frames counts the aggregate's audio frames.  The EOS
    bias is raised so that every session with EOS enabled ends at frame 0."""
    from magpie_tts_rt_b200 import _lib as L
    from magpie_tts_rt_b200.local_ar import LocalArEngine, StreamBatch
    import ctypes
    w = make_weights(SHAPE_BASELINE, seed=21, dtype=torch.bfloat16, profile="parity", with_final=True)
    w.final_b.view(POSITIONS, VOCAB)[:, S.EOS_ID] = 50.0
    n = 8
    eng = LocalArEngine(w, max_streams=n, path=path)
    uf = torch.tensor([1, 0, 0, 0, 1, 0, 0, 0], dtype=torch.bool)
    fi = torch.tensor([0, 1, 0, 0, 0, 1, 0, 0], dtype=torch.bool)
    fb = torch.tensor([0, 0, 1, 0, 0, 0, 1, 0], dtype=torch.bool)
    agg, ref = StreamBatch.allocate(n), StreamBatch.allocate(n)
    agg.codec_tokens = torch.full((n, 8, 8), -7, dtype=torch.int64, device="cuda")
    agg.finished_latch = torch.zeros(n, dtype=torch.bool, device="cuda")
    agg.codec_frames = torch.full((n,), -1, dtype=torch.int32, device="cuda")
    for b in (agg, ref):
        b.unfinished.copy_(uf); b.finished.copy_(fi); b.forbid_eos.copy_(fb)
        b.rng_seed.copy_(torch.arange(n) + 3)
    latch = np.zeros(n, bool)
    for k, off in enumerate((0, 2, 4, 6)):
        hidden = _hidden(n, 40 + k).cuda()
        agg.decoder_hidden.copy_(hidden); ref.decoder_hidden.copy_(hidden)
        agg.codec_frame_offset = off
        eng.frame(agg)
        eng.frame(ref)
        torch.cuda.synchronize()
        assert torch.equal(agg.codec_tokens[:, :, off:off + 2], ref.codec_tokens)
        assert (agg.codec_tokens[:, :, off + 2:] == -7).all()
        for name in ("end_frame_index", "rng_counter", "invalid_rows", "next_embedding"):
            assert torch.equal(getattr(agg, name), getattr(ref, name)), name
        end = ref.end_frame_index.cpu().numpy()
        enabled = ~(uf | fi | fb).numpy()
        assert (end[enabled] == 0).all() and (end[fi.numpy()] == 0).all() and (end[(uf | fb).numpy() & ~fi.numpy()] == -1).all()
        latch |= (end == 0) | (end == 1)
        np.testing.assert_array_equal(agg.finished_latch.cpu().numpy(), latch)
        # audio frames of the aggregate (eos_contract.hpp:14-30): offset + 2, or offset + end at the
        # EOS frame, for sessions not finished on entry (those keep their count: -1 here)
        exp_frames = np.where(fi.numpy(), -1, np.where(end >= 0, off + end, off + 2))
        np.testing.assert_array_equal(agg.codec_frames.cpu().numpy(), exp_frames)
    # argument checks: stride below 2, odd offset, offset past the row
    for stride, off in ((1, 0), (8, 3), (8, 8), (2, 2), (-2, 0)):
        cb = agg.c_struct()
        cb.codec_frames_stride, cb.codec_frame_offset = stride, off
        rc = L.lib.mtt_b200_launch_local_ar_frame(
            ctypes.byref(eng._shape), ctypes.byref(eng._w), ctypes.byref(eng._sampling), ctypes.byref(cb),
            ctypes.c_void_p(eng.workspace.data_ptr()), eng.workspace.numel(), None)
        assert rc == L.STATUS_INVALID_ARGUMENT, (stride, off)


@pytest.mark.parametrize("path", BOTH, ids=path_id)
def test_argmax_without_cfg(engines, path):
    """Greedy decoding, one row per stream (config 1's mode, bf16 on the GPU):
    no RNG, counter unchanged (magpietts_fused_sampling.py:136-197)."""
    shape = SHAPE_BASELINE
    w = weights(shape, 23)
    eng = engines(shape, 23, 4, cfg=False, argmax=True, path=path)
    n = 3
    hidden = _hidden(n, 11, cfg=False)
    flags = (np.array([0, 1, 0], bool), np.zeros(n, bool), np.array([0, 0, 1], bool))
    seed = np.zeros(n, np.int64)
    counter = np.array([0, 5, 17])
    gpu = run_gpu(eng, hidden, flags, seed, counter)
    check_frame(w, hidden, flags, seed, counter, gpu, params=S.SamplingParams(argmax=True))
    np.testing.assert_array_equal(gpu["counter"], counter)


@pytest.mark.parametrize("name,path", [("A_bf16_cfg", PATH_AUTO), ("A_bf16_cfg", TILE), ("A_bf16_cfg", PAIR),
                                       ("R_bf16_cfg", PATH_AUTO), ("A_bf16_cfg", QUAD), ("A_bf16_cfg", OCTO)] +
                         [("A_bf16_cfg", sp) for sp in SPLITS], ids=path_id)
def test_frame_against_reference_golden(engines, golden, golden_dir, name, path):
    """Teacher-forced on the reference's tokens, the GPU logits match the NeMo
    oracle's recorded logits within tolerance."""
    meta = golden["lt_frames"][name]
    z = np.load(os.path.join(golden_dir, "lt_frames.npz"))
    shape = LocalArShape(meta["d_model"], meta["n_layers"], meta["n_heads"], meta["d_ffn"])
    # AUTO: fused cluster kernel for A, phase kernels for R
    eng = engines(shape, meta["weights_seed"], 1, with_final=False, path=path)
    for f, fr in enumerate(meta["frames"]):
        hidden = from_bits(z[f"{name}/f{f}/hidden"]).reshape(1, 2, EMBED)
        ref_tokens = z[f"{name}/f{f}/tokens"]
        flags = tuple(np.array([v], bool) for v in fr["flags"])
        gpu = run_gpu(eng, hidden, flags, [meta["seed"]], [fr["counter_in"]], forced=ref_tokens[None])
        check_logits(gpu["logits"][0], z[f"{name}/f{f}/logits"].reshape(POSITIONS, 2, VOCAB), name)


@pytest.mark.parametrize("path", BOTH, ids=path_id)
def test_batch_of_64_streams(engines, path):
    """Config 3's batch size: 64 sessions x CFG pair, seeds 0..63."""
    shape = SHAPE_BASELINE
    w = weights(shape, 24)
    eng = engines(shape, 24, 64, path=path)
    n = 64
    hidden = _hidden(n, 12)
    flags = (np.ones(n, bool), np.zeros(n, bool), np.zeros(n, bool))
    seed = np.arange(n)
    counter = np.full(n, 32)
    gpu = run_gpu(eng, hidden, flags, seed, counter)
    check_frame(w, hidden, flags, seed, counter, gpu, streams=range(0, 64, 7))


def test_gpu_no_further_from_exact_than_oracle(engines):
    """Both bf16 implementations drift from exact arithmetic by rounding; the
    GPU must be no further from an f32 evaluation of the same bf16 weights
    and inputs (same token history) than the PyTorch-CPU bf16 oracle is."""
    shape = SHAPE_SOFIA
    w = weights(shape, 21)
    eng = engines(shape, 21, 8)
    n = 3
    hidden = _hidden(n, 5)
    flags = (np.zeros(n, bool), np.zeros(n, bool), np.ones(n, bool))
    seed = np.array([1, 2, 3])
    counter = np.zeros(n, np.int64)
    gpu = run_gpu(eng, hidden, flags, seed, counter)
    r16 = lt_oracle.run_frame(w, hidden, *flags, seed, counter, teacher_tokens=gpu["tokens"],
                              record_logits=True, eos=False)
    w32 = w.to(torch.float32)
    r32 = lt_oracle.run_frame(w32, hidden.float(), *flags, seed, counter,
                              params=S.SamplingParams(), teacher_tokens=gpu["tokens"], record_logits=True,
                              eos=False)
    exact = S.f32_to_bf16_bits(r32.logits.reshape(n, POSITIONS, 2, VOCAB).astype(np.float32))
    gpu_err, _ = logit_errors(gpu["logits"], exact)
    cpu_err, _ = logit_errors(r16.logits.reshape(n, POSITIONS, 2, VOCAB), exact)
    assert gpu_err.mean() <= 1.5 * cpu_err.mean() + 1e-4, (gpu_err.mean(), cpu_err.mean())
    assert gpu_err.max() <= 2.0 * cpu_err.max() + 1e-4, (gpu_err.max(), cpu_err.max())


@pytest.mark.parametrize("path", [FUSED, TILE, PAIR, QUAD, OCTO] + SPLITS, ids=path_id)
@pytest.mark.parametrize("kind", ["flat", "sharp", "ties"])
def test_sampler_row_shapes(path, kind):
    """Logit rows that drive each top-k select path: flat rows (every token
    tied: the whole-row search), a few dominant tokens (the narrowest window)
    and a tie block straddling the k-th place; tokens must match the oracle
    sampler on the GPU's logits."""
    from magpie_tts_rt_b200.local_ar import LocalArEngine
    shape = SHAPE_BASELINE
    w = make_weights(shape, seed=26, dtype=torch.bfloat16, profile="parity", with_final=True)
    g = torch.Generator().manual_seed(9)
    if kind == "flat":
        w.head_w.zero_()
        w.head_b.fill_(0.5)
    elif kind == "sharp":
        w.head_w.mul_(0.25)
        for p in range(POSITIONS):
            w.head_b[p, torch.randperm(2016, generator=g)[:40]] = 6.0
    else:
        w.head_w.zero_()
        w.head_b.copy_(torch.randn(w.head_b.shape, generator=g).to(torch.bfloat16))
        for p in range(POSITIONS):
            w.head_b[p, torch.randperm(2016, generator=g)[:120]] = 3.0  # 120 ties around k = 80
    eng = LocalArEngine(w, max_streams=8, path=path)
    n = 5
    hidden = _hidden(n, 31)
    flags = (np.array([1, 1, 0, 1, 0], bool), np.array([0, 0, 0, 0, 1], bool), np.zeros(n, bool))
    seed = np.arange(n) + 40
    counter = np.arange(n) * 3
    gpu = run_gpu(eng, hidden, flags, seed, counter)
    check_frame(w, hidden, flags, seed, counter, gpu)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs in this process")
@pytest.mark.parametrize("path", [PATH_AUTO, FUSED, TILE, PAIR, SPLIT4, SPLIT8, QUAD, OCTO], ids=path_id)
def test_frames_on_two_devices_in_one_process(path):
    """One process drives frames on cuda:0 and then cuda:1 (the reference
    allows several runtimes per process, tests/c_api/multi_runtime_plugin_gpu_tests.cpp).
    Each device makes its own kernel set-up (the shared-memory opt-in is a
    per-device setting); each GPU uses only its own memory.  Both match the
    oracle and agree with each other bit for bit."""
    from magpie_tts_rt_b200.local_ar import LocalArEngine
    shape = SHAPE_BASELINE
    w = weights(shape, 21)
    n = 6
    hidden = _hidden(n, 5)
    flags = tuple(np.resize(np.asarray(f), n) for f in FLAGS6)
    seed = np.resize(np.array([1234, 0, 7, (1 << 32) - 1, 99, 5]), n)
    counter = np.resize(np.array([0, 16, 3200, 48, S.MAX_COUNTER - 3, 0]), n)
    out = []
    for dev in (0, 1):
        with torch.cuda.device(dev):
            eng = LocalArEngine(w, max_streams=n, device=f"cuda:{dev}", path=path)
            assert path == PATH_AUTO or eng.path == path
            gpu = run_gpu(eng, hidden, flags, seed, counter)
        check_frame(w, hidden, flags, seed, counter, gpu)
        out.append(gpu)
    for k in ("tokens", "counter", "invalid", "end", "next_emb", "logits"):
        np.testing.assert_array_equal(out[0][k], out[1][k], err_msg=k)
