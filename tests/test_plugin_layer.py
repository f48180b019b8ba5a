"""The TensorRT plugin layer on the CPU (no TensorRT in this image).

magpie_tts_rt_b200/csrc/trt_plugins.cpp (one IPluginV3 class over the
contract table of plugin_contract.cpp) is compiled against the stand-in
header tests/trt_stub/NvInfer.h together with the plugin ABI
(plugin_abi.cpp built with MTT_B200_WITH_TENSORRT) and
tests/csrc/plugin_layer_test.cpp, which supplies a fake plugin registry and
expression builder.  The program checks the five creators' order, names,
version, namespace and fields, each plugin's tensor types, formats, output
types and shapes, accepted and rejected input shapes, workspace size and
enqueue argument check, and the registration statuses of register_plugins
(OK, ALREADY_REGISTERED, REGISTRATION_CONFLICT, REGISTRATION_FAILED with the
added creators taken back, REGISTRY_UNAVAILABLE), as
plugins/local_ar_plugins.cu:1805-2180, 3880-4104 define them."""
import os
import shutil
import subprocess
import tempfile

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "magpie_tts_rt_b200")
CUDA_INCLUDE = "/usr/local/cuda/include"


def _build_and_run(gpu: bool):
    from magpie_tts_rt_b200 import _lib  # noqa: F401  (the library is built and loads)
    with tempfile.TemporaryDirectory() as tmp:
        exe = os.path.join(tmp, "plugin_layer_test")
        cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-Werror", "-DMTT_B200_WITH_TENSORRT",
               "-I", os.path.join(REPO, "tests", "trt_stub"), "-I", os.path.join(REPO, "include"),
               "-I", CUDA_INCLUDE,
               os.path.join(REPO, "tests", "csrc", "plugin_layer_test.cpp"),
               os.path.join(PKG, "csrc", "plugin_contract.cpp"),
               os.path.join(PKG, "csrc", "trt_plugins.cpp"),
               os.path.join(PKG, "csrc", "plugin_abi.cpp"),
               "-L", PKG, "-lmagpie_tts_rt_b200", "-Wl,-rpath," + PKG,
               "-L/usr/local/cuda/lib64", "-lcudart", "-Wl,-rpath,/usr/local/cuda/lib64", "-o", exe]
        r = subprocess.run(cmd, capture_output=True, text=True)
        assert r.returncode == 0, r.stderr[-4000:]
        r = subprocess.run([exe] + (["--gpu"] if gpu else []), capture_output=True, text=True, timeout=120)
        assert r.returncode == 0 and r.stdout.strip().endswith("OK"), r.stdout[-4000:] + r.stderr[-2000:]


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_plugin_layer_against_a_fake_tensorrt():
    _build_and_run(gpu=False)


@pytest.mark.gpu
@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_plugin_enqueue_on_the_gpu_matches_the_launchers():
    """Each plugin's enqueue through the IPluginV3 layer, on device buffers,
    gives bit for bit what its launcher gives for the same inputs."""
    _build_and_run(gpu=True)
