"""C-ABI library checks that need no GPU: the library loads, exports every
symbol include/*.h declares (and nothing else), the plugin ABI structs are
byte-compatible with the reference's, and the host-only entry points follow
the reference's status conventions."""
import ctypes
import glob
import os
import re
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

from magpie_tts_rt_b200 import _lib as L  # noqa: E402  (raises if the .so is missing)
from magpie_tts_rt_b200 import local_ar  # noqa: E402


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(REPO, "include", "*.h")):
        text = open(h).read()
        for m in re.finditer(r"MTT_B200_API\s+[\w\s\*]+?\b(mtt_\w+)\s*\(", text):
            names.add(m.group(1))
    return names


def exported_symbols():
    out = subprocess.run(["nm", "-D", "--defined-only", L.LIBRARY], capture_output=True, text=True,
                         check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


def test_exports_match_header():
    declared = declared_symbols()
    assert len(declared) >= 11
    exported = exported_symbols()
    assert declared == exported, (declared ^ exported)
    for name in declared:
        assert hasattr(L.lib, name)


def test_struct_layout_matches_reference():
    # sizeof / offsetof measured with gcc on the reference's
    # include/magpie_tts_rt/magpie_tts_rt_plugin.h:70-146 (x86-64 / aarch64 LP64)
    assert ctypes.sizeof(L.PluginCreatorV1) == 152
    assert ctypes.sizeof(L.PluginApiV1) == 816
    assert L.PluginApiV1.register_plugins.offset == 776
    assert ctypes.sizeof(L.MainDevicePositionClassV1) == 344
    assert ctypes.sizeof(L.MainDevicePositionKV1) == 80
    assert ctypes.sizeof(L.MainDevicePositionClassTableV1) == 27192
    assert L.MainDevicePositionClassTableV1.k_records.offset == 7240


def test_plugin_api_negotiation():
    """plugins/local_ar_plugins.cu:4858-4900 semantics."""
    assert L.lib.mtt_plugin_get_api_v1(None) == 2  # INVALID_ARGUMENT
    status, _ = local_ar.plugin_api(struct_size=ctypes.sizeof(L.PluginApiV1) - 8)
    assert status == 3  # ABI_MISMATCH
    status, _ = local_ar.plugin_api(abi_version=2)
    assert status == 3
    status, api = local_ar.plugin_api()
    assert status == 0
    assert api.struct_size == 816 and api.abi_version == 1 and api.creator_count == 5
    names = [c.name.decode() for c in api.creators]
    assert names == ["MagpieLocalARSampling", "MagpieLocalAREos", "MagpieLayerNorm",
                     "MagpieGeluTanh", "MagpieSoftmax"]
    for c in api.creators:
        assert c.struct_size == 152 and c.abi_version == 1
        assert c.version.decode() == "1" and c.plugin_namespace.decode() == "magpie_tts_rt"
    # no TensorRT in this build: the registry is unavailable
    assert api.register_plugins() == 4


def test_class_table_never_ready():
    assert L.lib.mtt_plugin_get_main_device_position_class_table_v1(None) == 2
    status, _ = local_ar.main_device_position_class_table(struct_size=100)
    assert status == 3
    status, _ = local_ar.main_device_position_class_table()
    assert status == 7  # NOT_READY


def test_workspace_sizes():
    # aligned(16*2017*4, 256) + 2*4, the reference's local_ar_eos_workspace_size
    assert local_ar.local_ar_eos_workspace_size() == 129288
    ok = L.Shape(256, 1, 4, 1024)
    assert L.lib.mtt_b200_local_ar_frame_workspace_size(ctypes.byref(ok), 64, 1) > 0
    assert L.lib.mtt_b200_local_ar_frame_workspace_size(ctypes.byref(L.Shape(768, 2, 12, 3072)), 1, 1) > 0
    bad = L.Shape(256, 1, 3, 1024)  # head width must be 64
    assert L.lib.mtt_b200_local_ar_frame_workspace_size(ctypes.byref(bad), 64, 1) == 0
    assert L.lib.mtt_b200_local_ar_frame_workspace_size(ctypes.byref(ok), 0, 1) == 0
    phase = L.SamplingConfig(80, 0.6, 2.5, 0, 1, L.PATH_PHASE_KERNELS)
    # begin + 16 x (in-projection, LN rows, 6 layer launches, head, sampling) + EOS rows, EOS GEMM, end
    assert L.lib.mtt_b200_local_ar_frame_launch_count(ctypes.byref(ok), ctypes.byref(phase), 64) == 1 + 16 * 10 + 3
    # identity in-projection: the position add (position 0) or the previous position's sampling kernel
    # writes the rows and their LN
    sofia = L.Shape(768, 2, 12, 3072)
    assert L.lib.mtt_b200_local_ar_frame_launch_count(ctypes.byref(sofia), ctypes.byref(phase), 64) == 1 + 1 + 16 * 16 + 3
    assert L.lib.mtt_b200_local_ar_frame_path(ctypes.byref(ok), ctypes.byref(phase), 64) == L.PATH_PHASE_KERNELS
    assert L.lib.mtt_b200_local_ar_frame_path(ctypes.byref(ok), ctypes.byref(phase), 0) == -1
    bad_path = L.SamplingConfig(80, 0.6, 2.5, 0, 1, 99)
    assert L.lib.mtt_b200_local_ar_frame_path(ctypes.byref(ok), ctypes.byref(bad_path), 64) == -1
    # a fused path the device cannot run (here: no device at all) is UNSUPPORTED, not a fallback
    for path in (L.PATH_FUSED_TILE, L.PATH_SPLIT_1, L.PATH_SPLIT_2, L.PATH_SPLIT_4):
        cfg = L.SamplingConfig(80, 0.6, 2.5, 0, 1, path)
        if L.lib.mtt_b200_local_ar_frame_path_clusters(path) == 0:
            assert L.lib.mtt_b200_local_ar_frame_path(ctypes.byref(ok), ctypes.byref(cfg), 64) == -3


def test_null_arguments_rejected_without_launch():
    """Null pointers return -1 before any CUDA call (local_ar_plugins.cu:4141-4147)."""
    assert L.lib.mtt_b200_launch_local_ar_sampling(*([None] * 12)) == -1
    assert L.lib.mtt_b200_launch_local_ar_eos(*([None] * 10)) == -1
    assert L.lib.mtt_b200_launch_finalize_local_step(None, None, 0, *([None] * 8)) == -1
    assert L.lib.mtt_b200_launch_test_clamped_gumbel(None, None, 4, None) == -1
    assert L.lib.mtt_b200_launch_local_ar_frame(None, None, None, None, None, 0, None) == -1


def test_alignment_launchers_without_a_gpu():
    """launch_alignment_controller's null-pointer status (cudaErrorInvalidValue,
    alignment_kernel.cu:168-173) and the batch's argument checks, all decided
    before any CUDA call; the contract struct is layout-identical to
    AlignmentKernelContract (five uint32)."""
    assert ctypes.sizeof(L.AlignmentContract) == 20
    assert L.lib.mtt_b200_launch_alignment_controller(None, None, *([None] * 7)) == 1
    c = L.AlignmentContract(12, 3, 5, 6, 4)
    assert L.lib.mtt_b200_launch_alignment_controller(None, ctypes.byref(c), *([None] * 7)) == 1
    assert L.lib.mtt_b200_launch_alignment_batch(None, None) == -1
    b = L.AlignmentBatch()
    b.n_sessions = 0
    assert L.lib.mtt_b200_launch_alignment_batch(ctypes.byref(b), None) == 0
    b.n_sessions = 4
    b.token_stride = 16
    assert L.lib.mtt_b200_launch_alignment_batch(ctypes.byref(b), None) == -1
    b.n_sessions = -1
    assert L.lib.mtt_b200_launch_alignment_batch(ctypes.byref(b), None) == -1


def test_main_decoder_entry_without_a_gpu():
    """Argument checks decided before any CUDA call."""
    assert L.lib.mtt_b200_main_decoder_workspace_size(0, 128) == 0
    assert L.lib.mtt_b200_main_decoder_workspace_size(4, 513) == 0
    assert L.lib.mtt_b200_main_decoder_workspace_size(4, 100) == 0
    # activations + the FFN2 split-K partial sums (4 splits x 8 rows x 768 f32); no library workspace
    assert 4 * 8 * 768 * 4 < L.lib.mtt_b200_main_decoder_workspace_size(4, 128) < 1 << 20
    assert L.lib.mtt_b200_launch_main_decoder_step(None, None, None, 0, None) == -1
    w, b = L.MainDecoderWeights(), L.MainDecoderBatch()
    b.n_sessions, b.cache_capacity, b.token_stride, w.n_layers = 2, 467, 100, 12  # stride not a multiple of 8
    assert L.lib.mtt_b200_launch_main_decoder_step(ctypes.byref(w), ctypes.byref(b), None, 0, None) == -1


def test_session_engine_argument_checks_without_a_gpu():
    """Configuration checks decided before any CUDA call; without a device
    the engine cannot be created (CUDA error), never a crash."""
    h = ctypes.c_void_p()
    cfg = L.SessionEngineConfig()
    assert L.lib.mtt_b200_session_engine_create(ctypes.byref(cfg), ctypes.byref(h)) == -1  # no sessions
    cfg.max_sessions, cfg.token_stride, cfg.lookahead, cfg.sink_threshold = 4, 100, 6, 4
    assert L.lib.mtt_b200_session_engine_create(ctypes.byref(cfg), ctypes.byref(h)) == -1  # stride not x8
    cfg.token_stride, cfg.with_decoder = 64, 1
    assert L.lib.mtt_b200_session_engine_create(ctypes.byref(cfg), ctypes.byref(h)) == -1  # decoder w/o capacity
    assert L.lib.mtt_b200_session_engine_create(ctypes.byref(cfg), None) == -1
    assert L.lib.mtt_b200_session_engine_step(None) == -1
    assert L.lib.mtt_b200_session_engine_open(None, 0, 1, 1, None, None, None, None) == -1
    assert L.lib.mtt_b200_session_engine_collect(None, 0, None, None, None) == -1
    L.lib.mtt_b200_session_engine_destroy(None)


def test_struct_layouts_match_the_header(tmp_path):
    """sizeof and offsetof of this library's C structs, measured with gcc on
    include/magpie_tts_rt_b200.h, equal the ctypes mirrors'."""
    import shutil
    import subprocess
    if shutil.which("gcc") is None:
        pytest.skip("needs gcc")
    mirrors = {"mtt_b200_stream_batch_t": L.StreamBatch, "mtt_b200_local_ar_weights_t": L.Weights,
               "mtt_b200_sampling_config_t": L.SamplingConfig, "mtt_b200_alignment_batch_t": L.AlignmentBatch,
               "mtt_b200_main_decoder_weights_t": L.MainDecoderWeights,
               "mtt_b200_main_decoder_batch_t": L.MainDecoderBatch,
               "mtt_b200_session_engine_config_t": L.SessionEngineConfig,
               "mtt_b200_session_engine_buffers_t": L.SessionEngineBuffers}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "magpie_tts_rt_b200.h"', 'int main(void) {']
    for cname, py in mirrors.items():
        lines.append(f'  printf("{cname} %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'  printf("{cname}.{fname} %zu\\n", offsetof({cname}, {fname}));')
    lines += ['  return 0;', '}']
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    inc = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")
    subprocess.run(["gcc", "-I", inc, str(src), "-o", str(exe)], check=True)
    got = dict(line.rsplit(" ", 1) for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                               check=True).stdout.splitlines())
    for cname, py in mirrors.items():
        assert int(got[cname]) == ctypes.sizeof(py), cname
        for fname, _ in py._fields_:
            assert int(got[f"{cname}.{fname}"]) == getattr(py, fname).offset, (cname, fname)
