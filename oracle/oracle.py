"""ctypes wrapper of the CPU checker (oracle/_build/liboracle.so).

TEST INFRASTRUCTURE ONLY.  This restates the Sullux/ai-research CPU path (quant.zig,
tensor.zig, kernels.zig, ring_buffer.zig, model/forward.zig, the Q4 dequant loop of
test_q4_exec.zig) and is used by tests/, __graft_entry__.smoke() and bench.py's CPU
baseline leg as the parity checker.  The product library never loads it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"

QUANT_NONE, QUANT_Q8, QUANT_Q4 = 0, 1, 2

_P = C.c_void_p
_U32 = C.c_uint32
_U64 = C.c_uint64
_SZ = C.c_size_t
_F = C.c_float
_I = C.c_int


class OrcConfig(C.Structure):
    _fields_ = [
        ("vocab_size", _U32), ("hidden_size", _U32), ("intermediate_size", _U32),
        ("num_layers", _U32), ("num_q_heads", _U32), ("num_kv_heads", _U32),
        ("num_global_kv_heads", _U32), ("head_dim", _U32), ("global_head_dim", _U32),
        ("num_anchors", _U32), ("window_size", _U32), ("num_recall", _U32),
        ("kv_bf16", _U32), ("has_post_norms", _U32), ("full_every", _U32),
        ("attention_k_eq_v", _U32),
        ("rms_norm_eps", _F), ("rope_theta", _F), ("rope_theta_full", _F), ("attn_scale", _F),
        ("layer_quant", _U32), ("quiescence_threshold", _F),
    ]


_SIGS = {
    "orc_bf16_from_f32": (C.c_uint16, [_F]),
    "orc_bf16_to_f32": (_F, [C.c_uint16]),
    "orc_f16_round": (_F, [_F]),
    "orc_quantize_row_q8_0": (None, [_P, _P, _SZ]),
    "orc_quantize_row_q4_0": (None, [_P, _P, _SZ]),
    "orc_quantize_matrix": (None, [_P, _P, _SZ, _SZ, _I, _I]),
    "orc_quantized_row_words": (_SZ, [_SZ, _I]),
    "orc_dequant_q4": (None, [_P, _P, _SZ, _SZ]),
    "orc_dequant_q8": (None, [_P, _P, _SZ, _SZ]),
    "orc_gemv_q4": (None, [_P, _P, _P, _SZ, _SZ, _I]),
    "orc_gemv_q8": (None, [_P, _P, _P, _SZ, _SZ, _I]),
    "orc_gate_up_geglu_q4": (None, [_P, _P, _P, _P, _SZ, _SZ, _I]),
    "orc_gemv_bf16": (None, [_P, _P, _P, _SZ, _SZ]),
    "orc_gemv_bf16_mt": (None, [_P, _P, _P, _SZ, _SZ, _I]),
    "orc_quiescence_gate": (_I, [_P, _P, _U32, _F, _P]),
    "orc_archive_create": (_P, [_P, _U32, _F, _F, _F, _F]),
    "orc_archive_destroy": (None, [_P]),
    "orc_archive_integrate": (_U32, [_P, _U64, _P]),
    "orc_archive_count": (_U32, [_P]),
    "orc_archive_entry": (None, [_P, _U32, _P, _P, _P, _P, _P]),
    "orc_archive_scan": (_U32, [_P, _P, _U64, _P, _U32]),
    "orc_archive_create_dim": (_P, [_U32, _U32, _F, _F, _F, _F]),
    "orc_archive_append": (None, [_P, _U64, _F, _P]),
    "orc_archive_write_head": (_U32, [_P]),
    "orc_model_gate_stats": (None, [_P, _P, _P]),
    "orc_gate_up_geglu_q8": (None, [_P, _P, _P, _P, _SZ, _SZ, _I]),
    "orc_rmsnorm": (None, [_P, _P, _P, _SZ, _F]),
    "orc_unit_rmsnorm": (None, [_P, _P, _SZ, _F]),
    "orc_add_rmsnorm": (None, [_P, _P, _P, _P, _SZ, _F, _F]),
    "orc_gelu_tanh": (_F, [_F]),
    "orc_rope_inv_freq": (None, [_P, _SZ, _F]),
    "orc_apply_rope_partial": (None, [_P, _SZ, _U64, _SZ, _SZ, _P]),
    "orc_softmax": (None, [_P, _SZ]),
    "orc_argmax": (_U32, [_P, _SZ]),
    "orc_qkv_rope": (None, [_P, _P, _P, _P, _P, _P, _P, _I, _U32, _U32, _U32, _U32, _U32, _P,
                            _F, _U64, _U32, _U32]),
    "orc_decode_attn": (None, [_P, _P, _P, _P, _P, _U32, _U32, _U32, _U32, _U32, _F]),
    "orc_ring_create": (_P, [_U32, _U32, _U32, _U32]),
    "orc_ring_destroy": (None, [_P]),
    "orc_ring_reset": (None, [_P]),
    "orc_ring_slot_index": (_U32, [_P, _U64]),
    "orc_ring_activate_slot": (_U32, [_P, _U32, _U64]),
    "orc_ring_prefill": (None, [_P, _U32, _U64]),
    "orc_ring_write_recall": (None, [_P, _U32, _U32, _U64]),
    "orc_ring_clear_recall": (None, [_P]),
    "orc_ring_active_slots": (_U32, [_P, _U32, _U64, _P]),
    "orc_ring_total_slots": (_U32, [_P]),
    "orc_hash": (_U64, [_U64, _U64, _U64]),
    "orc_synth_normal": (_F, [_U64, _U64, _U64]),
    "orc_synth_q4": (None, [_P, _SZ, _SZ, _U64, _U64]),
    "orc_synth_q8": (None, [_P, _SZ, _SZ, _U64, _U64]),
    "orc_synth_bf16_normal": (None, [_P, _SZ, _U64, _U64, _F, _F]),
    "orc_synth_gain_f32": (None, [_P, _SZ, _U64, _U64]),
    "orc_synth_embed_row": (None, [_P, _U32, _U32, _U64]),
    "orc_model_create": (_P, [C.POINTER(OrcConfig), _U64, _I]),
    "orc_model_destroy": (None, [_P]),
    "orc_model_ring": (_P, [_P]),
    "orc_model_forward": (_U32, [_P, _P, _U64, _I, _P, _P]),
    "orc_model_set_act_bf16": (None, [_P, _I]),
    "orc_model_fill_kv": (None, [_P, _U64]),
    "orc_model_synth_recall": (None, [_P, _U64, _U32, _U64]),
    "orc_model_kcache": (C.POINTER(_F), [_P, _U32]),
    "orc_model_vcache": (C.POINTER(_F), [_P, _U32]),
    "orc_model_kv_dim": (_U32, [_P, _U32]),
}

_lib = None


def build() -> Path:
    src = HERE / "sx_oracle.c"
    if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def threads() -> int:
    return int(os.environ.get("SX_ORACLE_THREADS", os.cpu_count() or 1))


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


# ---- elementwise / formats
def bf16_from_f32(v: float) -> int:
    return int(lib().orc_bf16_from_f32(v))


def bf16_to_f32(b: int) -> float:
    return float(lib().orc_bf16_to_f32(b))


def bf16_round(a: np.ndarray) -> np.ndarray:
    """tensor.zig:7-13 RNE (vectorised restatement, same integer formula)."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint32) << 16
    return r.astype(np.uint32).view(np.float32)


def quantized_row_words(cols: int, mode: int) -> int:
    return int(lib().orc_quantized_row_words(cols, mode))


def quantize_matrix(src_bf16: np.ndarray, rows: int, cols: int, mode: int) -> np.ndarray:
    src = np.ascontiguousarray(src_bf16, np.uint16)
    out = np.zeros(rows * quantized_row_words(cols, mode), np.uint32)
    lib().orc_quantize_matrix(_p(out), _p(src), rows, cols, mode, threads())
    return out


def dequant_q4(w: np.ndarray, rows: int, cols: int) -> np.ndarray:
    out = np.zeros(rows * cols, np.float32)
    lib().orc_dequant_q4(_p(out), _p(np.ascontiguousarray(w, np.uint32)), rows, cols)
    return out.reshape(rows, cols)


def dequant_q8(w: np.ndarray, rows: int, cols: int) -> np.ndarray:
    out = np.zeros(rows * cols, np.float32)
    lib().orc_dequant_q8(_p(out), _p(np.ascontiguousarray(w, np.uint32)), rows, cols)
    return out.reshape(rows, cols)


def gemv_q4(w, x, rows, cols):
    y = np.zeros(rows, np.float32)
    lib().orc_gemv_q4(_p(y), _p(np.ascontiguousarray(w, np.uint32)),
                      _p(np.ascontiguousarray(x, np.float32)), rows, cols, threads())
    return y


def gemv_q8(w, x, rows, cols):
    y = np.zeros(rows, np.float32)
    lib().orc_gemv_q8(_p(y), _p(np.ascontiguousarray(w, np.uint32)),
                      _p(np.ascontiguousarray(x, np.float32)), rows, cols, threads())
    return y


def gate_up_geglu_q4(wg, wu, x, rows, cols):
    y = np.zeros(rows, np.float32)
    lib().orc_gate_up_geglu_q4(_p(y), _p(np.ascontiguousarray(wg, np.uint32)),
                               _p(np.ascontiguousarray(wu, np.uint32)),
                               _p(np.ascontiguousarray(x, np.float32)), rows, cols, threads())
    return y


def gemv_bf16(w_bf16, x, rows, cols):
    y = np.zeros(rows, np.float32)
    lib().orc_gemv_bf16_mt(_p(y), _p(np.ascontiguousarray(x, np.float32)),
                           _p(np.ascontiguousarray(w_bf16, np.uint16)), rows, cols, threads())
    return y


def gate_up_geglu_q8(wg, wu, x, rows, cols):
    y = np.zeros(rows, np.float32)
    lib().orc_gate_up_geglu_q8(_p(y), _p(np.ascontiguousarray(wg, np.uint32)),
                               _p(np.ascontiguousarray(wu, np.uint32)),
                               _p(np.ascontiguousarray(x, np.float32)), rows, cols, threads())
    return y


def quiescence_gate(x, x_prev, threshold_sq):
    """quiescence_gate.wgsl on one vector: (runs, mean_sq); x_prev (float32 array) is updated."""
    ms = np.zeros(1, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    assert x_prev.dtype == np.float32 and x_prev.flags.c_contiguous
    r = lib().orc_quiescence_gate(_p(x), _p(x_prev), x.size, threshold_sq, _p(ms))
    return bool(r), float(ms[0])


def gate_up_geglu_bf16(wg, wu, x, rows, cols):
    """kernels.zig gatedMlp's product with bf16 weights: gelu_tanh(Wg x) * (Wu x)."""
    g = gemv_bf16(wg, x, rows, cols)
    u = gemv_bf16(wu, x, rows, cols)
    return np.array([gelu_tanh(float(a)) * b for a, b in zip(g, u)], np.float32)


def rmsnorm(x, w, eps=1e-6):
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros_like(x)
    lib().orc_rmsnorm(_p(out), _p(x), _p(np.ascontiguousarray(w, np.float32)), x.size, eps)
    return out


def unit_rmsnorm(x, eps=1e-6):
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros_like(x)
    lib().orc_unit_rmsnorm(_p(out), _p(x), x.size, eps)
    return out


def add_rmsnorm(x, r, w, eps=1e-6, scalar=1.0):
    x = np.array(x, np.float32, copy=True)
    y = np.zeros_like(x)
    lib().orc_add_rmsnorm(_p(x), _p(np.ascontiguousarray(r, np.float32)),
                          _p(np.ascontiguousarray(w, np.float32)), _p(y), x.size, eps, scalar)
    return x, y


def gelu_tanh(v: float) -> float:
    return float(lib().orc_gelu_tanh(v))


def rope_inv_freq(rot: int, theta: float) -> np.ndarray:
    out = np.zeros(max(rot // 2, 1), np.float32)
    lib().orc_rope_inv_freq(_p(out), rot, theta)
    return out[: rot // 2]


def softmax(v):
    v = np.array(v, np.float32, copy=True)
    lib().orc_softmax(_p(v), v.size)
    return v


def argmax(v) -> int:
    v = np.ascontiguousarray(v, np.float32)
    return int(lib().orc_argmax(_p(v), v.size))


def qkv_rope(q, k_in, v_in, q_norm_w, k_norm_w, k_cache, v_cache, cache_bf16, num_q, num_kv,
             head_dim, rot, k_eq_v, theta, eps, clock, slot, total_slots):
    """Returns the new q; k_cache / v_cache (f32 numpy, [slot][kv_head][D]) are updated."""
    q = np.array(q, np.float32, copy=True)
    freq = rope_inv_freq(rot, theta)
    if freq.size == 0:
        freq = np.zeros(1, np.float32)
    lib().orc_qkv_rope(_p(q), _p(np.ascontiguousarray(k_in, np.float32)),
                       _p(np.ascontiguousarray(v_in, np.float32)),
                       _p(np.ascontiguousarray(q_norm_w, np.float32)),
                       _p(np.ascontiguousarray(k_norm_w, np.float32)),
                       _p(k_cache), _p(v_cache), int(cache_bf16), num_q, num_kv, head_dim, rot,
                       int(k_eq_v), _p(freq), eps, clock, slot, total_slots)
    return q


def decode_attn(q, k_cache, v_cache, slots, num_q, num_kv, head_dim, total_slots, scale):
    out = np.zeros(num_q * head_dim, np.float32)
    sl = np.ascontiguousarray(slots, np.uint32)
    lib().orc_decode_attn(_p(out), _p(np.ascontiguousarray(q, np.float32)),
                          _p(np.ascontiguousarray(k_cache, np.float32)),
                          _p(np.ascontiguousarray(v_cache, np.float32)), _p(sl), len(sl), num_q,
                          num_kv, head_dim, total_slots, scale)
    return out


# ---- synthetic inputs (bit-identical to libsx's generator)
def synth_q4(rows, cols, seed, stream):
    out = np.zeros(rows * (cols // 32) * 5, np.uint32)
    lib().orc_synth_q4(_p(out), rows, cols, seed, stream)
    return out


def synth_q8(rows, cols, seed, stream):
    out = np.zeros(rows * (cols // 32) * 9, np.uint32)
    lib().orc_synth_q8(_p(out), rows, cols, seed, stream)
    return out


def synth_normal(seed, stream, idx) -> float:
    return float(lib().orc_synth_normal(seed, stream, idx))


def synth_bf16_normal(n, seed, stream, mean=0.0, std=1.0) -> np.ndarray:
    out = np.zeros(n, np.uint16)
    lib().orc_synth_bf16_normal(_p(out), n, seed, stream, mean, std)
    return out


def synth_gain(n, seed, stream) -> np.ndarray:
    out = np.zeros(n, np.float32)
    lib().orc_synth_gain_f32(_p(out), n, seed, stream)
    return out


def synth_embed_row(hidden, token, seed) -> np.ndarray:
    out = np.zeros(hidden, np.float32)
    lib().orc_synth_embed_row(_p(out), hidden, token, seed)
    return out


class Ring:
    """ring_buffer.zig restatement."""

    def __init__(self, num_layers, num_anchors, window_size, num_recall):
        self.h = lib().orc_ring_create(num_layers, num_anchors, window_size, num_recall)
        self.total_slots = int(lib().orc_ring_total_slots(self.h))
        self._own = True

    @classmethod
    def borrow(cls, handle):
        r = cls.__new__(cls)
        r.h = handle
        r.total_slots = int(lib().orc_ring_total_slots(handle))
        r._own = False
        return r

    def __del__(self):
        if getattr(self, "_own", False) and self.h:
            lib().orc_ring_destroy(self.h)
            self.h = None

    def get_slot_index(self, clock):
        return int(lib().orc_ring_slot_index(self.h, clock))

    def activate_slot(self, layer, clock):
        return int(lib().orc_ring_activate_slot(self.h, layer, clock))

    def prefill(self, layer, upto):
        lib().orc_ring_prefill(self.h, layer, upto)

    def write_recall(self, layer, rank, clock):
        lib().orc_ring_write_recall(self.h, layer, rank, clock)

    def clear_recall(self):
        lib().orc_ring_clear_recall(self.h)

    def get_active_slots(self, layer, clock) -> np.ndarray:
        out = np.zeros(self.total_slots, np.uint32)
        n = lib().orc_ring_active_slots(self.h, layer, clock, _p(out))
        return out[:n].copy()


class Model:
    """Whole-model decode in the GPU graph's op order (model_dispatch.zig)."""

    def __init__(self, cfg: dict, seed: int, nthreads: int | None = None):
        names = {f for f, _ in OrcConfig._fields_}
        kw = {k: v for k, v in cfg.items() if k in names}
        kw.setdefault("layer_quant", QUANT_Q4)
        c = OrcConfig(**kw)
        self.cfg = dict(cfg)
        self.h = lib().orc_model_create(C.byref(c), seed, nthreads or threads())
        self.ring = Ring.borrow(lib().orc_model_ring(self.h))

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_model_destroy(self.h)
            self.h = None

    def fill_kv(self, seed):
        lib().orc_model_fill_kv(self.h, seed)

    def set_act_bf16(self, on=True):
        """Round each projection's input to bf16 (the batched-prefill GEMM path)."""
        lib().orc_model_set_act_bf16(self.h, int(on))

    def synth_recall(self, clock, n_recall, seed):
        lib().orc_model_synth_recall(self.h, clock, n_recall, seed)

    def forward(self, x, clock, want_logits=True):
        x = np.ascontiguousarray(x, np.float32)
        logits = np.zeros(self.cfg["vocab_size"], np.float32)
        xo = np.zeros(self.cfg["hidden_size"], np.float32)
        tok = lib().orc_model_forward(self.h, _p(x), clock, int(want_logits), _p(logits), _p(xo))
        return int(tok), logits, xo

    def gate_stats(self):
        """(mean_sq[layers], active[layers]) of the last forward's quiescence gates."""
        n = self.cfg["num_layers"]
        ms = np.zeros(n, np.float32)
        act = np.zeros(n, np.uint32)
        lib().orc_model_gate_stats(self.h, _p(ms), _p(act))
        return ms, act

    def kv_dim(self, layer):
        return int(lib().orc_model_kv_dim(self.h, layer))

    def kcache(self, layer) -> np.ndarray:
        n = self.kv_dim(layer) * (self.cfg["num_anchors"] + self.cfg["window_size"] +
                                  self.cfg["num_recall"])
        return np.ctypeslib.as_array(lib().orc_model_kcache(self.h, layer), shape=(n,))

    def vcache(self, layer) -> np.ndarray:
        n = self.kv_dim(layer) * (self.cfg["num_anchors"] + self.cfg["window_size"] +
                                  self.cfg["num_recall"])
        return np.ctypeslib.as_array(lib().orc_model_vcache(self.h, layer), shape=(n,))


class Archive:
    """memory.zig DiffArchive with the recall injection of memory_inject.zig, on a checker
    model (its caches, ring and final normed state)."""

    def __init__(self, model: "Model | None", capacity: int, alpha=1.0, beta=0.5, gamma=1.0,
                 lam=1.0 / 2048.0, dim: int | None = None):
        self.model = model  # keeps the model alive
        if model is None:  # DiffArchive.init: vectors and metadata only
            self.h = lib().orc_archive_create_dim(dim, capacity, alpha, beta, gamma, lam)
            self.dim, self.recall = dim, 0
        else:
            self.h = lib().orc_archive_create(model.h, capacity, alpha, beta, gamma, lam)
            self.dim = model.cfg["hidden_size"]
            self.recall = model.cfg["num_recall"]

    def append(self, timestamp, salience, vector):
        lib().orc_archive_append(self.h, timestamp, salience,
                                 _p(np.ascontiguousarray(vector, np.float32)))

    @property
    def write_head(self) -> int:
        return int(lib().orc_archive_write_head(self.h))

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_archive_destroy(self.h)
            self.h = None

    def integrate(self, clock) -> np.ndarray:
        sel = np.zeros(max(self.recall, 1), np.uint32)
        n = lib().orc_archive_integrate(self.h, clock, _p(sel))
        return sel[:n]

    @property
    def count(self) -> int:
        return int(lib().orc_archive_count(self.h))

    def entry(self, i):
        v = np.zeros(self.dim, np.float32)
        ts, la, ac, sal = C.c_uint64(), C.c_uint64(), C.c_uint32(), C.c_float()
        lib().orc_archive_entry(self.h, i, _p(v), C.byref(ts), C.byref(la), C.byref(ac),
                                C.byref(sal))
        return v, ts.value, la.value, ac.value, sal.value

    def scan(self, query, now, top_k) -> np.ndarray:
        out = np.zeros(max(top_k, 1), np.uint32)
        n = lib().orc_archive_scan(self.h, _p(np.ascontiguousarray(query, np.float32)), now,
                                   _p(out), top_k)
        return out[:n]
