"""Source rules every file that travels to a GPU box keeps (CPU only).

* No bulk or TMA tensor load with the cluster-multicast qualifier: the frame
  kernels read only this GPU's own weights and rows, and the multi-GPU runs
  must not reach such a load.  A tcgen05 commit to a cluster's barriers
  stays allowed.
* None of the batched memory-copy entry points of the CUDA runtime or driver.

The patterns are assembled from pieces, so this file itself names neither
form; the planted cases are assembled the same way.
"""
import pathlib
import re

import pytest

REPO = pathlib.Path(__file__).resolve().parents[1]
SOURCE_SUFFIXES = {".cu", ".cuh", ".cpp", ".hpp", ".h", ".c", ".py"}
SOURCE_DIRS = ["magpie_tts_rt_b200", "include", "oracle", "tests"]

_BULK = "cp" + r"\.async\.bulk"
_MCAST = r"\.multi" + "cast::cluster"
BULK_MULTICAST = re.compile(_BULK + r"[^\n\"]*" + _MCAST)
BATCH_COPY = re.compile("(cuda|cu)" + "Memcpy" + "(3D)?" + "Batch")


def _sources():
    files = [REPO / "bench.py", REPO / "__graft_entry__.py"]
    for d in SOURCE_DIRS:
        for p in (REPO / d).rglob("*"):
            if p.is_file() and p.suffix in SOURCE_SUFFIXES and "_ref" not in p.parts and "_build" not in p.parts:
                files.append(p)
    return sorted(files)


def test_sources_found():
    names = {p.name for p in _sources()}
    assert {"frame_pair.cu", "frame_split.cu", "ptx.cuh", "bench.py"} <= names


def test_patterns_catch_planted_cases():
    mc = ".multi" + "cast::cluster"
    assert BULK_MULTICAST.search("cp" + ".async.bulk.tensor.2d.shared::cluster.global" + mc + " [%0], [%1];")
    assert not BULK_MULTICAST.search("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster" + mc)
    assert not BULK_MULTICAST.search("// " + "cp" + ".async.bulk.tensor.2d, 128-byte swizzle, no multicast")
    assert BATCH_COPY.search("cuda" + "Memcpy" + "BatchAsync(")
    assert BATCH_COPY.search("cu" + "Memcpy3D" + "BatchAsync(")
    assert not BATCH_COPY.search("cudaMemcpyAsync(")


@pytest.mark.parametrize("pattern,what", [(BULK_MULTICAST, "bulk load with cluster multicast"),
                                          (BATCH_COPY, "batched memory copy")])
def test_no_forbidden_forms(pattern, what):
    hits = []
    for p in _sources():
        for n, line in enumerate(p.read_text(errors="replace").splitlines(), 1):
            if pattern.search(line):
                hits.append(f"{p.relative_to(REPO)}:{n}")
    assert not hits, f"{what}: {hits}"
