"""ctypes binding of the C oracle (``oracle/csrc/oracle.c``).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline leg as the checker.  The product library never
imports this module.

The functions mirror the reference's sampling contract:
``plugins/local_ar_plugins.cu:1149-1495`` (sampling + EOS kernels) and
``tools/export/local_ar_wrapper.py:153-286,424-476`` (pure-tensor statements).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from oracle import build as _build

VOCAB = 2024
CODEBOOK = 2016
EOS_ID = 2017
EMBED = 768
POSITIONS = 16
CODEBOOKS = 8
FRAMES = 2
TOP_K = 80
TEMPERATURE = 0.6
CFG_SCALE = 2.5
PHILOX_STRIDE = 2048
MAX_COUNTER = ((1 << 63) - 1 - (PHILOX_STRIDE - 1)) // PHILOX_STRIDE

LOGITS_BF16_CFG = 0
LOGITS_BF16 = 1
LOGITS_F32 = 2


class _Params(ctypes.Structure):
    _fields_ = [
        ("top_k", ctypes.c_int32),
        ("temperature", ctypes.c_float),
        ("cfg_scale", ctypes.c_float),
        ("argmax", ctypes.c_int32),
    ]


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = _build.build()
        handle = ctypes.CDLL(path)
        P = ctypes.c_void_p
        handle.orc_philox_word.restype = ctypes.c_uint32
        handle.orc_philox_word.argtypes = [ctypes.c_uint32, ctypes.c_uint64]
        handle.orc_philox_uniform.restype = ctypes.c_float
        handle.orc_philox_uniform.argtypes = [ctypes.c_uint32, ctypes.c_uint64]
        handle.orc_log_f32.restype = ctypes.c_float
        handle.orc_log_f32.argtypes = [ctypes.c_float]
        handle.orc_clamped_gumbel.restype = ctypes.c_float
        handle.orc_clamped_gumbel.argtypes = [ctypes.c_float]
        handle.orc_guided_logit.restype = ctypes.c_float
        handle.orc_guided_logit.argtypes = [ctypes.c_uint16, ctypes.c_uint16, ctypes.c_float]
        handle.orc_sample_batch.restype = None
        handle.orc_sample_batch.argtypes = [
            P, ctypes.c_int, ctypes.c_int64, ctypes.c_int, P, P, P, P, P,
            ctypes.POINTER(_Params), P, P, P,
        ]
        handle.orc_eos_guided.restype = None
        handle.orc_eos_guided.argtypes = [P, P, P, ctypes.c_float, P]
        handle.orc_eos_end_frame.restype = ctypes.c_int32
        handle.orc_eos_end_frame.argtypes = [P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        handle.orc_embedding_sum.restype = None
        handle.orc_embedding_sum.argtypes = [P, P, P]
        handle.orc_finalize_local_step.restype = None
        handle.orc_finalize_local_step.argtypes = [
            P, P, ctypes.c_uint32, ctypes.c_int32, ctypes.c_int32, P, P,
            ctypes.c_int64, P, P,
        ]
        _lib = handle
    return _lib


def _ptr(a: np.ndarray) -> ctypes.c_void_p:
    assert a.flags["C_CONTIGUOUS"]
    return ctypes.c_void_p(a.ctypes.data)


@dataclass(frozen=True)
class SamplingParams:
    top_k: int = TOP_K
    temperature: float = TEMPERATURE
    cfg_scale: float = CFG_SCALE
    argmax: bool = False

    def c(self) -> _Params:
        return _Params(self.top_k, self.temperature, self.cfg_scale, int(self.argmax))


def philox_word(seed: int, offset: int) -> int:
    return int(lib().orc_philox_word(seed, offset))


def philox_uniform(seed: int, offset: int) -> float:
    return float(lib().orc_philox_uniform(seed, offset))


def log_f32(x: float) -> float:
    return float(lib().orc_log_f32(x))


def clamped_gumbel(u: float) -> float:
    return float(lib().orc_clamped_gumbel(u))


def sample(
    logits: np.ndarray,
    unfinished,
    finished,
    forbid_eos,
    seed,
    counter,
    params: SamplingParams = SamplingParams(),
):
    """Sample n independent (stream, position) calls.

    ``logits`` is uint16 (bf16 bits) of shape [n, 2, V] (CFG pair) or [n, V]
    (no CFG), or float32 of shape [n, V] (no CFG).  Flags / seed / counter are
    length-n arrays.  Returns (token int64[n], counter_out int64[n],
    invalid int32[n]).
    """
    logits = np.ascontiguousarray(logits)
    if logits.dtype == np.uint16 and logits.ndim == 3:
        kind, stride = LOGITS_BF16_CFG, 2 * VOCAB
    elif logits.dtype == np.uint16 and logits.ndim == 2:
        kind, stride = LOGITS_BF16, VOCAB
    elif logits.dtype == np.float32 and logits.ndim == 2:
        kind, stride = LOGITS_F32, VOCAB
    else:
        raise ValueError(f"unsupported logits {logits.dtype} {logits.shape}")
    n = logits.shape[0]
    assert logits.shape[-1] == VOCAB
    as_u8 = lambda v: np.ascontiguousarray(np.broadcast_to(np.asarray(v, dtype=np.uint8), (n,)))
    as_i64 = lambda v: np.ascontiguousarray(np.broadcast_to(np.asarray(v, dtype=np.int64), (n,)))
    uf, fi, fb = as_u8(unfinished), as_u8(finished), as_u8(forbid_eos)
    sd, ct = as_i64(seed), as_i64(counter)
    token = np.empty(n, np.int64)
    counter_out = np.empty(n, np.int64)
    invalid = np.empty(n, np.int32)
    p = params.c()
    lib().orc_sample_batch(
        _ptr(logits), kind, stride, n, _ptr(uf), _ptr(fi), _ptr(fb), _ptr(sd), _ptr(ct),
        ctypes.byref(p), _ptr(token), _ptr(counter_out), _ptr(invalid),
    )
    return token, counter_out, invalid


def eos_guided(hidden: np.ndarray, weight: np.ndarray, bias: np.ndarray,
               cfg_scale: float = CFG_SCALE) -> np.ndarray:
    """Guided EOS logits [16, 2017] (f32) for one stream; bf16-bit inputs."""
    hidden = np.ascontiguousarray(hidden, dtype=np.uint16).reshape(2, EMBED)
    weight = np.ascontiguousarray(weight, dtype=np.uint16)
    bias = np.ascontiguousarray(bias, dtype=np.uint16)
    assert weight.size == POSITIONS * VOCAB * EMBED and bias.size == POSITIONS * VOCAB
    out = np.empty((POSITIONS, CODEBOOK + 1), np.float32)
    lib().orc_eos_guided(_ptr(hidden), _ptr(weight), _ptr(bias), cfg_scale, _ptr(out))
    return out


def eos_end_frame(guided, codec_tokens: np.ndarray, unfinished: bool, finished: bool,
                  forbid_eos: bool) -> int:
    codec_tokens = np.ascontiguousarray(codec_tokens, dtype=np.int64).reshape(CODEBOOKS, FRAMES)
    g = None
    if guided is not None:
        g = np.ascontiguousarray(guided, dtype=np.float32)
        assert g.shape == (POSITIONS, CODEBOOK + 1)
    return int(lib().orc_eos_end_frame(
        _ptr(g) if g is not None else None, _ptr(codec_tokens),
        int(unfinished), int(finished), int(forbid_eos)))


def embedding_sum(tables: np.ndarray, tokens: np.ndarray) -> np.ndarray:
    """bf16 bits [768]: sequential bf16 sum of table_p[token_p] over p, / 16."""
    tables = np.ascontiguousarray(tables, dtype=np.uint16)
    assert tables.shape == (POSITIONS, VOCAB, EMBED)
    tokens = np.ascontiguousarray(tokens, dtype=np.int64).reshape(POSITIONS)
    out = np.empty(EMBED, np.uint16)
    lib().orc_embedding_sum(_ptr(tables), _ptr(tokens), _ptr(out))
    return out


def codec_layout(position_major: np.ndarray) -> np.ndarray:
    """[16] position-major -> [8, 2] codec layout, p = frame * 8 + codebook."""
    pm = np.asarray(position_major, dtype=np.int64).reshape(FRAMES, CODEBOOKS)
    return np.ascontiguousarray(pm.T)


def finalize_local_step(step_codec_tokens, aggregate, frame_offset, invalid_rows,
                        end_frame_index, updated_counter):
    """Returns (aggregate, step_invalid, step_end, counter, finished_latched)."""
    step = np.ascontiguousarray(step_codec_tokens, dtype=np.int64).reshape(16)
    agg = np.array(aggregate, dtype=np.int64).reshape(8, 8).copy()
    si = np.zeros(1, np.int32)
    se = np.zeros(1, np.int32)
    cnt = np.zeros(1, np.int64)
    fin = np.zeros(1, np.uint8)
    lib().orc_finalize_local_step(_ptr(step), _ptr(agg), frame_offset, invalid_rows,
                                  end_frame_index, _ptr(si), _ptr(se), updated_counter,
                                  _ptr(cnt), _ptr(fin))
    return agg, int(si[0]), int(se[0]), int(cnt[0]), bool(fin[0])


# ---------------------------------------------------------------------------
# bf16 helpers shared by the oracle users
# ---------------------------------------------------------------------------

def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bits (NaN preserved)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
