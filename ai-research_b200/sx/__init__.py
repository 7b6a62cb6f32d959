"""Python host binding of libsx (include/sx.h), the B200 decode hot path.

This is a thin ctypes layer over the C ABI; the names follow the reference's Zig GPU
dispatch API (src/gpu/kernels.zig ``GpuEngine.record*`` / ``submitPreRecorded``,
src/gpu/model_gpu.zig ``GpuModelContext``, src/ring_buffer.zig ``DynamicRingBuffer``) so
that tests read like the reference's own.  Every call goes to the CUDA library; there is
no CPU fallback: importing this module without a built libsx.so raises.
"""
from __future__ import annotations

import ctypes as C
import os
import weakref
from pathlib import Path

import numpy as np

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libsx.so"

SX_OK = 0
SX_ERR_INVALID = 1
SX_ERR_CUDA = 2
SX_ERR_LAUNCH = 3
SX_ERR_TIMEOUT = 4
SX_ERR_OOM = 5
SX_ERR_PEER = 6
SX_ERR_UNSUPPORTED = 7
SX_ERR_DEVICE = 8

QUANT_NONE = 0
QUANT_Q8 = 1
QUANT_Q4 = 2

ENGINE_KV_F32 = 1


class SxError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"sx status {status}: {message}")
        self.status = status
        self.message = message


class ModelConfig(C.Structure):
    """sx_model_config (mirrors ModelConfig, src/model/types.zig:44-61)."""

    _fields_ = [
        ("vocab_size", C.c_uint32),
        ("hidden_size", C.c_uint32),
        ("intermediate_size", C.c_uint32),
        ("num_layers", C.c_uint32),
        ("num_q_heads", C.c_uint32),
        ("num_kv_heads", C.c_uint32),
        ("num_global_kv_heads", C.c_uint32),
        ("head_dim", C.c_uint32),
        ("global_head_dim", C.c_uint32),
        ("num_anchors", C.c_uint32),
        ("window_size", C.c_uint32),
        ("num_recall", C.c_uint32),
        ("kv_bf16", C.c_uint32),
        ("has_post_norms", C.c_uint32),
        ("full_every", C.c_uint32),
        ("attention_k_eq_v", C.c_uint32),
        ("rms_norm_eps", C.c_float),
        ("rope_theta", C.c_float),
        ("rope_theta_full", C.c_float),
        ("attn_scale", C.c_float),
        ("reference_graph", C.c_uint32),
        ("tp_size", C.c_uint32),
        ("tp_rank", C.c_uint32),
        ("num_sessions", C.c_uint32),
        ("quiescence_threshold", C.c_float),
    ]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


class QuiescenceGatePC(C.Structure):
    """sx_quiescence_gate_pc (QuiescenceGatePushConstants, src/gpu/kernels.zig:10-16)."""

    _fields_ = [("hidden_size", C.c_uint32), ("threshold_sq", C.c_float),
                ("base_cmd_idx", C.c_uint32), ("num_cmds", C.c_uint32),
                ("targets", C.c_uint32 * 16)]


class TpShard(C.Structure):
    """sx_tp_shard: one rank's heads, intermediate rows and vocabulary rows."""

    _fields_ = [(n, C.c_uint32) for n in (
        "q_heads", "q_head0", "kv_heads", "kv_head0", "global_kv_heads", "global_kv_head0",
        "inter", "inter0", "vocab", "vocab0")]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


class ModelIO(C.Structure):
    _fields_ = [
        ("x", C.c_void_p),
        ("slots", C.c_void_p),
        ("step", C.c_void_p),
        ("token", C.c_void_p),
        ("logits", C.c_void_p),
        ("normed", C.c_void_p),
    ]


def model_config(**kw) -> ModelConfig:
    """A config with the reference defaults (types.zig:44-61, main.zig:34 ring sizes)."""
    base = dict(
        vocab_size=262144,
        hidden_size=1536,
        intermediate_size=12288,
        num_layers=35,
        num_q_heads=8,
        num_kv_heads=1,
        num_global_kv_heads=1,
        head_dim=256,
        global_head_dim=256,
        num_anchors=32,
        window_size=512,
        num_recall=96,
        kv_bf16=1,
        has_post_norms=1,
        full_every=5,
        attention_k_eq_v=0,
        rms_norm_eps=1e-6,
        rope_theta=10000.0,
        rope_theta_full=1000000.0,
        attn_scale=1.0,
        reference_graph=0,
        tp_size=1,
        tp_rank=0,
        num_sessions=1,
        quiescence_threshold=0.0,
    )
    base.update(kw)
    return ModelConfig(**base)


# 12B-shaped decode config
def config_12b(**kw) -> ModelConfig:
    d = dict(
        vocab_size=262144,
        hidden_size=3840,
        intermediate_size=15360,
        num_layers=48,
        num_q_heads=16,
        num_kv_heads=8,
        num_global_kv_heads=8,
        head_dim=256,
        global_head_dim=256,
    )
    d.update(kw)
    return model_config(**d)


_lib = None


def _quiet_close(obj):
    """__del__: release the handle; at interpreter exit the module may already be torn down."""
    try:
        obj.close()
    except Exception:
        pass

_P = C.c_void_p
_U32 = C.c_uint32
_U64 = C.c_uint64
_F = C.c_float
_I = C.c_int
_S = C.c_int32

_SIGS = {
    "sx_version": (C.c_char_p, []),
    "sx_last_error": (C.c_char_p, []),
    "sx_status_string": (C.c_char_p, [_S]),
    "sx_quantized_row_words": (_U64, [_U32, _I]),
    "sx_packed_bytes": (_U64, [_U32, _U32, _I]),
    "sx_rope_inv_freq": (None, [_P, _U32, _F]),
    "sx_synth_embed_row": (None, [_P, _U32, _U32, _U64]),
    "sx_ring_create": (_S, [_U32, _U32, _U32, _U32, C.POINTER(_P)]),
    "sx_ring_destroy": (None, [_P]),
    "sx_ring_reset": (None, [_P]),
    "sx_ring_total_slots": (_U32, [_P]),
    "sx_ring_slot_index": (_U32, [_P, _U64]),
    "sx_ring_activate_slot": (_U32, [_P, _U32, _U64]),
    "sx_ring_prefill": (None, [_P, _U32, _U64]),
    "sx_ring_write_recall": (None, [_P, _U32, _U32, _U64]),
    "sx_ring_clear_recall": (None, [_P]),
    "sx_ring_active_slots": (_U32, [_P, _U32, _U64, _P]),
    "sx_engine_create": (_S, [_I, _I, _U32, C.POINTER(_P)]),
    "sx_engine_destroy": (None, [_P]),
    "sx_engine_set_stream": (_S, [_P, _P]),
    "sx_engine_stream": (_P, [_P]),
    "sx_engine_sync": (_S, [_P]),
    "sx_buffer_create": (_S, [_P, _U64, C.POINTER(_P)]),
    "sx_buffer_wrap": (_S, [_P, _P, _U64, C.POINTER(_P)]),
    "sx_buffer_destroy": (None, [_P]),
    "sx_buffer_device_ptr": (_P, [_P]),
    "sx_buffer_size": (_U64, [_P]),
    "sx_buffer_write": (_S, [_P, _U64, _P, _U64]),
    "sx_buffer_read": (_S, [_P, _U64, _P, _U64]),
    "sx_buffer_upload_weights": (_S, [_P, _P, _U32, _U32, _I]),
    "sx_buffer_repack_device": (_S, [_P, _P, _U32, _U32, _I]),
    "sx_buffer_quantize_device": (_S, [_P, _P, _U32, _U32, _I]),
    "sx_dispatch_quantize": (_S, [_P, _I, _P, _P, _U32, _U32]),
    "sx_set_create": (_S, [_P, _P, _U32, C.POINTER(_P)]),
    "sx_set_destroy": (None, [_P]),
    "sx_cmd_create": (_S, [_P, C.POINTER(_P)]),
    "sx_cmd_destroy": (None, [_P]),
    "sx_cmd_begin": (_S, [_P]),
    "sx_cmd_end": (_S, [_P]),
    "sx_record_gemv": (None, [_P, _P, _P, _U32, _U32]),
    "sx_record_gemv_logits": (None, [_P, _P, _P, _U32, _U32]),
    "sx_record_gate_up": (None, [_P, _P, _P, _U32, _U32]),
    "sx_record_add_rmsnorm": (None, [_P, _P, _P, _U32, _F, _F]),
    "sx_record_rmsnorm": (None, [_P, _P, _P, _U32, _F]),
    "sx_record_decode_attn": (None, [_P, _P, _P, _U32, _U32, _U32, _F, _U32, _U32]),
    "sx_record_qkv_rope": (None, [_P, _P, _P, _U32, _U32, _U32, _U32, _U32, _F, _F, _U32]),
    "sx_record_argmax": (None, [_P, _P, _P, _U32]),
    "sx_record_quiescence_gate": (None, [_P, _P, _P, _P]),
    "sx_record_gemv_indirect": (None, [_P, _P, _P, _U32, _U32, _P, _U64]),
    "sx_record_gate_up_indirect": (None, [_P, _P, _P, _U32, _U32, _P, _U64]),
    "sx_record_add_rmsnorm_indirect": (None, [_P, _P, _P, _U32, _F, _F, _P, _U64]),
    "sx_record_rmsnorm_indirect": (None, [_P, _P, _P, _U32, _F, _P, _U64]),
    "sx_record_decode_attn_indirect": (None, [_P, _P, _P, _U32, _U32, _U32, _F, _U32, _U32, _P,
                                               _U64]),
    "sx_record_qkv_rope_indirect": (None, [_P, _P, _P, _U32, _U32, _U32, _U32, _U32, _F, _F,
                                            _U32, _P, _U64]),
    "sx_dispatch_quiescence_gate": (_S, [_P, _P, _P, _P, _P]),
    "sx_record_barrier": (None, [_P, _P]),
    "sx_submit": (_S, [_P, _P, _U64]),
    "sx_dispatch_gemv": (_S, [_P, _I, _P, _P, _P, _U32, _U32, _U32]),
    "sx_dispatch_gate_up": (_S, [_P, _P, _P, _P, _P, _U32, _U32, _U32]),
    "sx_dispatch_rmsnorm": (_S, [_P, _P, _P, _P, _U32, _U32, _F]),
    "sx_dispatch_add_rmsnorm": (_S, [_P, _P, _P, _P, _P, _U32, _U32, _F, _F]),
    "sx_dispatch_qkv_rope": (
        _S,
        [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _U32, _U32, _U32, _U32, _U32, _F, _F, _U32],
    ),
    "sx_dispatch_decode_attn": (
        _S,
        [_P, _P, _P, _P, _P, _P, _P, _U32, _U32, _U32, _F, _U32, _U32],
    ),
    "sx_dispatch_qkv_rope_attn": (
        _S,
        [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _U32, _U32, _U32, _U32, _U32, _F, _F, _F,
         _U32, _U32, _U32],
    ),
    "sx_dispatch_argmax": (_S, [_P, _P, _U32, _P]),
    "sx_decode_attn_noalloc": (
        _S,
        [_P, _P, _P, _P, _P, _P, _U32, _U32, _U32, _F, _U32, _U32, _U32, _P],
    ),
    "sx_dispatch_unpack_q4": (_S, [_P, _P, _P, _U32, _U32]),
    "sx_dispatch_synth_weights": (_S, [_P, _I, _P, _U32, _U32, _U32, _U64, _U64]),
    "sx_model_create": (_S, [_P, C.POINTER(ModelConfig), C.POINTER(_P)]),
    "sx_dispatch_prefill_gemm": (_S, [_P, _P, _P, _P, _U32, _U32, _U32]),
    "sx_model_create_tp": (_S, [_P, C.POINTER(ModelConfig), _P, C.POINTER(_P)]),
    "sx_tp_shard_plan": (_S, [C.POINTER(ModelConfig), C.POINTER(TpShard)]),
    "sx_comm_unique_id": (_S, [C.c_char_p]),
    "sx_comm_create": (_S, [_P, C.c_char_p, _U32, _U32, C.POINTER(_P)]),
    "sx_comm_destroy": (None, [_P]),
    "sx_comm_set_allreduce": (_S, [_P, _I]),
    "sx_comm_allreduce_is_nccl": (_I, [_P]),
    "sx_comm_allreduce": (_S, [_P, _P, _U32]),
    "sx_comm_set_wait_ns": (_S, [_P, _U64]),
    "sx_model_destroy": (None, [_P]),
    "sx_model_synth_weights": (_S, [_P, _U64]),
    "sx_model_fill_kv": (_S, [_P, _U64]),
    "sx_model_fill_kv_session": (_S, [_P, _U32, _U64]),
    "sx_model_config_bytes": (_U32, []),
    "sx_decode_batch": (_S, [_P, _U32, _P, _P, _P, _P, _P, _I, _P, _P]),
    "sx_prefill_batch": (_S, [_P, _U32, _P, _P, _P, _P, _P, _P, _U32, _P, _P, _P]),
    "sx_model_launch_batch": (_S, [_P, _U32, _I]),
    "sx_forward_token": (_S, [_P, _P, _U32, _U32, _P, _U32, _I, _P, _P]),
    "sx_model_launch": (_S, [_P, _I]),
    "sx_model_get_io": (_S, [_P, C.POINTER(ModelIO)]),
    "sx_model_kcache": (_P, [_P, _U32]),
    "sx_model_vcache": (_P, [_P, _U32]),
    "sx_model_weight_bytes": (_U64, [_P]),
    "sx_model_kernels_per_token": (_U32, [_P, _I]),
    "sx_archive_create": (_S, [_P, _U32, _P, C.POINTER(_P)]),
    "sx_archive_destroy": (None, [_P]),
    "sx_archive_integrate": (_S, [_P, _P, _U64, _P, _P]),
    "sx_archive_count": (_U32, [_P]),
    "sx_archive_entry": (_S, [_P, _U32, _P, _P, _P, _P, _P]),
}


def lib():
    """Load libsx.so (built by __graft_entry__.build()); raises when it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    path = os.environ.get("SX_LIB", str(LIB_PATH))
    if not os.path.exists(path):
        raise ImportError(
            f"libsx.so not found at {path}: build it with __graft_entry__.build(); "
            "the decode path has no CPU fallback"
        )
    L = C.CDLL(path)
    for name, (res, args) in _SIGS.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    if L.sx_model_config_bytes() != C.sizeof(ModelConfig):
        raise ImportError(f"{path}: sx_model_config is {L.sx_model_config_bytes()} bytes, this "
                          f"binding's mirror {C.sizeof(ModelConfig)}: rebuild the library")
    _lib = L
    return L


def declared_symbols() -> list[str]:
    return list(_SIGS)


def last_error() -> str:
    return lib().sx_last_error().decode()


def check(status: int) -> None:
    if status != SX_OK:
        raise SxError(status, last_error())


def _ptr(a) -> int | None:
    """Device or host address of a numpy array, torch tensor or raw int."""
    if a is None:
        return None
    if isinstance(a, int):
        return a
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    raise TypeError(f"cannot take the address of {type(a)}")


# ------------------------------------------------------------------------------------
def quantized_row_words(cols: int, mode: int) -> int:
    return int(lib().sx_quantized_row_words(cols, mode))


def packed_bytes(rows: int, cols: int, mode: int) -> int:
    return int(lib().sx_packed_bytes(rows, cols, mode))


def rope_inv_freq(rotary_dim: int, theta: float) -> np.ndarray:
    out = np.zeros(max(rotary_dim // 2, 1), np.float32)
    lib().sx_rope_inv_freq(out.ctypes.data, rotary_dim, theta)
    return out[: rotary_dim // 2]


def synth_embed_row(hidden: int, token: int, seed: int) -> np.ndarray:
    out = np.zeros(hidden, np.float32)
    lib().sx_synth_embed_row(out.ctypes.data, hidden, token, seed)
    return out


class Ring:
    """DynamicRingBuffer slot bookkeeping (src/ring_buffer.zig:8-146)."""

    def __init__(self, num_layers: int, num_anchors: int, window_size: int, num_recall: int):
        h = C.c_void_p()
        check(lib().sx_ring_create(num_layers, num_anchors, window_size, num_recall, C.byref(h)))
        self.h = h
        self.total_slots = int(lib().sx_ring_total_slots(h))

    def close(self):
        if getattr(self, "h", None):
            lib().sx_ring_destroy(self.h)
            self.h = None

    __del__ = _quiet_close

    def reset(self):
        lib().sx_ring_reset(self.h)

    def get_slot_index(self, clock: int) -> int:
        return int(lib().sx_ring_slot_index(self.h, clock))

    def activate_slot(self, layer: int, clock: int) -> int:
        return int(lib().sx_ring_activate_slot(self.h, layer, clock))

    def prefill(self, layer: int, upto: int) -> None:
        lib().sx_ring_prefill(self.h, layer, upto)

    def write_recall(self, layer: int, rank: int, clock: int) -> None:
        lib().sx_ring_write_recall(self.h, layer, rank, clock)

    def clear_recall(self) -> None:
        lib().sx_ring_clear_recall(self.h)

    def get_active_slots(self, layer: int, clock: int) -> np.ndarray:
        out = np.zeros(self.total_slots, np.uint32)
        n = lib().sx_ring_active_slots(self.h, layer, clock, out.ctypes.data)
        return out[:n].copy()


class Engine:
    """GpuEngine (src/gpu/kernels.zig:18-158) on one B200."""

    def __init__(self, device: int = 0, mode: int = QUANT_Q4, kv_f32: bool = False):
        h = C.c_void_p()
        flags = ENGINE_KV_F32 if kv_f32 else 0
        check(lib().sx_engine_create(device, mode, flags, C.byref(h)))
        self.h = h
        self.mode = mode
        self.kv_bf16 = not kv_f32
        self._models = weakref.WeakSet()  # closed before the engine they were made on

    def close(self):
        if getattr(self, "h", None):
            for m in list(getattr(self, "_models", ())):
                m.close()
            lib().sx_engine_destroy(self.h)
            self.h = None

    __del__ = _quiet_close

    @property
    def stream(self) -> int:
        return int(lib().sx_engine_stream(self.h) or 0)

    def set_stream(self, stream: int | None) -> None:
        check(lib().sx_engine_set_stream(self.h, stream))

    def sync(self) -> None:
        check(lib().sx_engine_sync(self.h))

    # --- buffers / sets / command buffers
    def buffer(self, nbytes: int) -> "Buffer":
        return Buffer.create(self, nbytes)

    def wrap(self, tensor_or_ptr, nbytes: int | None = None) -> "Buffer":
        if nbytes is None:
            nbytes = tensor_or_ptr.numel() * tensor_or_ptr.element_size()
        return Buffer.wrap(self, _ptr(tensor_or_ptr), nbytes)

    def set(self, *buffers: "Buffer") -> "DescriptorSet":
        return DescriptorSet(self, buffers)

    def command_buffer(self) -> "CommandBuffer":
        return CommandBuffer(self)

    # --- record API (kernels.zig:80-146)
    def record_gemv(self, cmd, s, m, k):
        lib().sx_record_gemv(self.h, cmd.h, s.h, m, k)

    def record_gemv_logits(self, cmd, s, m, k):
        lib().sx_record_gemv_logits(self.h, cmd.h, s.h, m, k)

    def record_gate_up(self, cmd, s, m, k):
        lib().sx_record_gate_up(self.h, cmd.h, s.h, m, k)

    def record_add_rmsnorm(self, cmd, s, h, eps, scalar):
        lib().sx_record_add_rmsnorm(self.h, cmd.h, s.h, h, eps, scalar)

    def record_rmsnorm(self, cmd, s, h, eps):
        lib().sx_record_rmsnorm(self.h, cmd.h, s.h, h, eps)

    def record_decode_attn(self, cmd, s, head_dim, kv_dim, gqa_ratio, inv_sqrt_dim, num_q_heads,
                           total_slots):
        lib().sx_record_decode_attn(self.h, cmd.h, s.h, head_dim, kv_dim, gqa_ratio,
                                    inv_sqrt_dim, num_q_heads, total_slots)

    def record_qkv_rope(self, cmd, s, num_q, num_kv, head_dim, rotary_dim, k_eq_v, theta, eps,
                        total_slots):
        lib().sx_record_qkv_rope(self.h, cmd.h, s.h, num_q, num_kv, head_dim, rotary_dim,
                                 int(k_eq_v), theta, eps, total_slots)

    def record_argmax(self, cmd, s, vocab):
        lib().sx_record_argmax(self.h, cmd.h, s.h, vocab)

    def record_quiescence_gate(self, cmd, s, pc: "QuiescenceGatePC"):
        lib().sx_record_quiescence_gate(self.h, cmd.h, s.h, C.byref(pc))

    def record_gemv_indirect(self, cmd, s, m, k, ind, offset):
        lib().sx_record_gemv_indirect(self.h, cmd.h, s.h, m, k, ind.h, offset)

    def record_gate_up_indirect(self, cmd, s, m, k, ind, offset):
        lib().sx_record_gate_up_indirect(self.h, cmd.h, s.h, m, k, ind.h, offset)

    def record_add_rmsnorm_indirect(self, cmd, s, h, eps, scalar, ind, offset):
        lib().sx_record_add_rmsnorm_indirect(self.h, cmd.h, s.h, h, eps, scalar, ind.h, offset)

    def record_rmsnorm_indirect(self, cmd, s, h, eps, ind, offset):
        lib().sx_record_rmsnorm_indirect(self.h, cmd.h, s.h, h, eps, ind.h, offset)

    def record_decode_attn_indirect(self, cmd, s, head_dim, kv_dim, gqa_ratio, inv_sqrt_dim,
                                    num_q_heads, total_slots, ind, offset):
        lib().sx_record_decode_attn_indirect(self.h, cmd.h, s.h, head_dim, kv_dim, gqa_ratio,
                                             inv_sqrt_dim, num_q_heads, total_slots, ind.h,
                                             offset)

    def record_qkv_rope_indirect(self, cmd, s, num_q, num_kv, head_dim, rotary_dim, k_eq_v,
                                 theta, eps, total_slots, ind, offset):
        lib().sx_record_qkv_rope_indirect(self.h, cmd.h, s.h, num_q, num_kv, head_dim,
                                          rotary_dim, int(k_eq_v), theta, eps, total_slots,
                                          ind.h, offset)

    def quiescence_gate(self, x_curr, x_prev, ind, pc: "QuiescenceGatePC"):
        check(lib().sx_dispatch_quiescence_gate(self.h, _ptr(x_curr), _ptr(x_prev), _ptr(ind),
                                                C.byref(pc)))

    def record_barrier(self, cmd):
        lib().sx_record_barrier(self.h, cmd.h)

    def submit_pre_recorded(self, cmd, timeout_ns: int = 0) -> None:
        check(lib().sx_submit(self.h, cmd.h, timeout_ns))

    # --- immediate mode (device pointers: torch tensors or ints)
    def quantize(self, mode, bf16, ref_out, rows, cols):
        """sx_dispatch_quantize: reference-layout Q4_0/Q8_0 block words of a device bf16 matrix."""
        check(lib().sx_dispatch_quantize(self.h, mode, _ptr(bf16), _ptr(ref_out), rows, cols))

    def gemv(self, mode, w_packed, x, y, m, k, batch=1):
        check(lib().sx_dispatch_gemv(self.h, mode, _ptr(w_packed), _ptr(x), _ptr(y), m, k, batch))

    def prefill_gemm(self, w_packed, x_bf16, y, t, n, k):
        """y[t][n] = x[t][:] . bf16(deq(w[n][:])) on the tcgen05 tensor cores (bf16 x, f32 y)."""
        check(lib().sx_dispatch_prefill_gemm(self.h, _ptr(w_packed), _ptr(x_bf16), _ptr(y), t, n,
                                             k))

    def gate_up(self, wg, wu, x, y, m, k, batch=1):
        check(lib().sx_dispatch_gate_up(self.h, _ptr(wg), _ptr(wu), _ptr(x), _ptr(y), m, k, batch))

    def rmsnorm(self, x, w, y, n, batch=1, eps=1e-6):
        check(lib().sx_dispatch_rmsnorm(self.h, _ptr(x), _ptr(w), _ptr(y), n, batch, eps))

    def add_rmsnorm(self, x, r, w, y, n, batch=1, eps=1e-6, scalar=1.0):
        check(lib().sx_dispatch_add_rmsnorm(self.h, _ptr(x), _ptr(r), _ptr(w), _ptr(y), n, batch,
                                            eps, scalar))

    def qkv_rope(self, q_in, k_in, v_in, q_norm_w, k_norm_w, q_out, k_cache, v_cache, step,
                 num_q, num_kv, head_dim, rotary_dim, k_eq_v, theta, eps, total_slots):
        check(lib().sx_dispatch_qkv_rope(
            self.h, _ptr(q_in), _ptr(k_in), _ptr(v_in), _ptr(q_norm_w), _ptr(k_norm_w),
            _ptr(q_out), _ptr(k_cache), _ptr(v_cache), _ptr(step), num_q, num_kv, head_dim,
            rotary_dim, int(k_eq_v), theta, eps, total_slots))

    def decode_attn(self, q, k_cache, v_cache, slots, step, out, head_dim, kv_dim, gqa_ratio,
                    scale, num_q_heads, total_slots):
        check(lib().sx_dispatch_decode_attn(
            self.h, _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(slots), _ptr(step), _ptr(out),
            head_dim, kv_dim, gqa_ratio, scale, num_q_heads, total_slots))

    def qkv_rope_attn(self, q_in, k_in, v_in, q_norm_w, k_norm_w, k_cache, v_cache, slots, step,
                      out, num_q, num_kv, head_dim, rotary_dim, k_eq_v, theta, eps, scale,
                      total_slots, instances=1, qkv_stride=0):
        """The decode graph's fused qkv_rope + decode attention kernel (sx_dispatch_qkv_rope_attn)."""
        check(lib().sx_dispatch_qkv_rope_attn(
            self.h, _ptr(q_in), _ptr(k_in), _ptr(v_in), _ptr(q_norm_w), _ptr(k_norm_w),
            _ptr(k_cache), _ptr(v_cache), _ptr(slots), _ptr(step), _ptr(out), num_q, num_kv,
            head_dim, rotary_dim, int(k_eq_v), theta, eps, scale, total_slots, instances,
            qkv_stride))

    def argmax(self, logits, n, out):
        check(lib().sx_dispatch_argmax(self.h, _ptr(logits), n, _ptr(out)))

    def unpack_q4(self, w_packed, out, m, k):
        check(lib().sx_dispatch_unpack_q4(self.h, _ptr(w_packed), _ptr(out), m, k))

    def synth_weights(self, mode, ref_out, row0, rows, cols, seed, stream_id):
        check(lib().sx_dispatch_synth_weights(self.h, mode, _ptr(ref_out), row0, rows, cols, seed,
                                              stream_id))


class Buffer:
    """GpuBuffer (src/gpu/buffer.zig)."""

    def __init__(self, engine: Engine, h, nbytes: int):
        self.engine = engine
        self.h = h
        self.nbytes = nbytes

    @classmethod
    def create(cls, engine: Engine, nbytes: int) -> "Buffer":
        h = C.c_void_p()
        check(lib().sx_buffer_create(engine.h, nbytes, C.byref(h)))
        return cls(engine, h, nbytes)

    @classmethod
    def wrap(cls, engine: Engine, ptr: int, nbytes: int) -> "Buffer":
        h = C.c_void_p()
        check(lib().sx_buffer_wrap(engine.h, ptr, nbytes, C.byref(h)))
        return cls(engine, h, nbytes)

    def close(self):
        if getattr(self, "h", None):
            lib().sx_buffer_destroy(self.h)
            self.h = None

    __del__ = _quiet_close

    @property
    def ptr(self) -> int:
        return int(lib().sx_buffer_device_ptr(self.h))

    def write(self, arr: np.ndarray, offset: int = 0) -> None:
        a = np.ascontiguousarray(arr)
        check(lib().sx_buffer_write(self.h, offset, a.ctypes.data, a.nbytes))

    def read(self, dtype, count: int, offset: int = 0) -> np.ndarray:
        out = np.empty(count, dtype)
        check(lib().sx_buffer_read(self.h, offset, out.ctypes.data, out.nbytes))
        return out

    def upload_weights(self, ref_words: np.ndarray, rows: int, cols: int, mode: int) -> None:
        w = np.ascontiguousarray(ref_words, dtype=np.uint32)
        check(lib().sx_buffer_upload_weights(self.h, w.ctypes.data, rows, cols, mode))

    def quantize_device(self, bf16_ptr, rows: int, cols: int, mode: int) -> None:
        """sx_buffer_quantize_device: quantise a device bf16 matrix into this buffer."""
        check(lib().sx_buffer_quantize_device(self.h, _ptr(bf16_ptr), rows, cols, mode))

    def repack_device(self, ref_ptr, rows: int, cols: int, mode: int) -> None:
        check(lib().sx_buffer_repack_device(self.h, _ptr(ref_ptr), rows, cols, mode))


class DescriptorSet:
    def __init__(self, engine: Engine, buffers):
        self.buffers = list(buffers)  # keep alive
        arr = (C.c_void_p * len(self.buffers))(*[b.h.value for b in self.buffers])
        h = C.c_void_p()
        check(lib().sx_set_create(engine.h, arr, len(self.buffers), C.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            lib().sx_set_destroy(self.h)
            self.h = None

    __del__ = _quiet_close


class CommandBuffer:
    def __init__(self, engine: Engine):
        h = C.c_void_p()
        check(lib().sx_cmd_create(engine.h, C.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            lib().sx_cmd_destroy(self.h)
            self.h = None

    __del__ = _quiet_close

    def begin(self):
        check(lib().sx_cmd_begin(self.h))

    def end(self):
        check(lib().sx_cmd_end(self.h))


def tp_shard_plan(cfg: ModelConfig) -> TpShard:
    """sx_tp_shard_plan: the shard of rank cfg.tp_rank of cfg.tp_size (host only)."""
    out = TpShard()
    check(lib().sx_tp_shard_plan(C.byref(cfg), C.byref(out)))
    return out


def comm_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    check(lib().sx_comm_unique_id(buf))
    return buf.raw


class Comm:
    """A tensor-parallel communicator (NCCL) of one rank, on the engine's GPU."""

    def __init__(self, engine: Engine, unique_id: bytes, nranks: int, rank: int):
        assert len(unique_id) == 128
        h = C.c_void_p()
        check(lib().sx_comm_create(engine.h, unique_id, nranks, rank, C.byref(h)))
        self.h = h
        self.engine = engine
        self.nranks, self.rank = nranks, rank

    def set_allreduce(self, use_nccl: bool) -> None:
        """NCCL or the one-shot peer kernel for the o / down all-reduces (before the model)."""
        check(lib().sx_comm_set_allreduce(self.h, int(use_nccl)))

    @property
    def allreduce_is_nccl(self) -> bool:
        return bool(lib().sx_comm_allreduce_is_nccl(self.h))

    def allreduce(self, buf, count: int) -> None:
        """sx_comm_allreduce: in-place sum of `count` floats at a device pointer over the ranks."""
        check(lib().sx_comm_allreduce(self.h, _ptr(buf), count))

    def set_wait_ns(self, wait_ns: int) -> None:
        """How long the peer all-reduce waits for the other ranks' flags."""
        check(lib().sx_comm_set_wait_ns(self.h, wait_ns))

    def close(self):
        if getattr(self, "h", None):
            lib().sx_comm_destroy(self.h)
            self.h = None

    __del__ = _quiet_close


class Model:
    """GpuModelContext (src/gpu/model_gpu.zig:35-197) + gpuDispatchForwardToken."""

    def __init__(self, engine: Engine, cfg: ModelConfig, comm: "Comm | None" = None):
        h = C.c_void_p()
        self.cfg = cfg
        if comm is None:
            check(lib().sx_model_create(engine.h, C.byref(cfg), C.byref(h)))
        else:
            check(lib().sx_model_create_tp(engine.h, C.byref(cfg), comm.h, C.byref(h)))
        self.h = h
        self.engine = engine
        self.comm = comm  # kept alive while the model's graphs reference it
        self.total_slots = cfg.num_anchors + cfg.window_size + cfg.num_recall
        self.sessions = max(1, cfg.num_sessions)
        engine._models.add(self)

    def close(self):
        if getattr(self, "h", None):
            lib().sx_model_destroy(self.h)
            self.h = None

    __del__ = _quiet_close

    def synth_weights(self, seed: int) -> None:
        check(lib().sx_model_synth_weights(self.h, seed))

    def fill_kv(self, seed: int) -> None:
        check(lib().sx_model_fill_kv(self.h, seed))

    def fill_kv_session(self, session: int, seed: int) -> None:
        check(lib().sx_model_fill_kv_session(self.h, session, seed))

    def decode_batch(self, xs: np.ndarray, clocks, slots, active_lists, want_logits: bool = True,
                     logits_out: np.ndarray | None = None) -> np.ndarray:
        """One token for each of sessions 0..n-1 (sx_decode_batch): xs [n][hidden], per-session
        clock, slot and active-slot list; returns the n greedy tokens."""
        x = np.ascontiguousarray(xs, np.float32)
        n = x.shape[0]
        act = np.zeros((n, self.total_slots), np.uint32)
        cnt = np.zeros(n, np.uint32)
        for i, a in enumerate(active_lists):
            a = np.asarray(a, np.uint32)
            act[i, : len(a)] = a
            cnt[i] = len(a)
        clk = np.ascontiguousarray(clocks, np.uint32)
        sl = np.ascontiguousarray(slots, np.uint32)
        toks = np.zeros(n, np.uint32)
        check(lib().sx_decode_batch(self.h, n, x.ctypes.data, clk.ctypes.data, sl.ctypes.data,
                                    act.ctypes.data, cnt.ctypes.data, int(want_logits),
                                    toks.ctypes.data,
                                    None if logits_out is None else logits_out.ctypes.data))
        return toks

    def forward_token(self, x: np.ndarray, clock: int, slot: int, active_slots: np.ndarray,
                      want_logits: bool = True, logits_out: np.ndarray | None = None) -> int:
        xs = np.ascontiguousarray(x, np.float32)
        sl = np.ascontiguousarray(active_slots, np.uint32)
        tok = C.c_uint32(0)
        check(lib().sx_forward_token(self.h, xs.ctypes.data, clock, slot, sl.ctypes.data,
                                     len(sl), int(want_logits), C.byref(tok),
                                     None if logits_out is None else logits_out.ctypes.data))
        return int(tok.value)

    def prefill_plan(self, prompts, rings, start_clocks, sessions=None) -> dict:
        """Per-token inputs of sx_prefill_batch for several sessions' prompts: prompts[i] are
        the embedding rows [L_i][hidden] of session sessions[i] (default i), whose ring
        (sx.Ring, advanced here) is at start_clocks[i]; token j gets clock start_clocks[i] + j
        and its slot and active list from the ring, as forwardToken would."""
        sessions = list(range(len(prompts))) if sessions is None else list(sessions)
        ts = self.total_slots
        T = sum(len(p) for p in prompts)
        x = np.empty((T, self.cfg.hidden_size), np.float32)
        sess, clk, slt, cnt = (np.empty(T, np.uint32) for _ in range(4))
        act = np.zeros((T, ts), np.uint32)
        out_rows = []
        t = 0
        for i, (xs, ring, c0) in enumerate(zip(prompts, rings, start_clocks)):
            for j in range(len(xs)):
                c = c0 + j
                slt[t] = ring.activate_slot(0, c)
                a = ring.get_active_slots(0, c)
                act[t, : len(a)] = a
                cnt[t] = len(a)
                x[t] = xs[j]
                sess[t] = sessions[i]
                clk[t] = c
                t += 1
            out_rows.append(t - 1)
        return dict(x=x, session=sess, clock=clk, slot=slt, active=act, n_active=cnt,
                    out_rows=np.asarray(out_rows, np.uint32))

    def prefill_run(self, plan: dict, logits_out: np.ndarray | None = None) -> np.ndarray:
        """sx_prefill_batch on a plan from prefill_plan; returns the greedy token after each
        prompt (logits_out, optional: [prompts][vocab])."""
        p = plan
        toks = np.zeros(len(p["out_rows"]), np.uint32)
        check(lib().sx_prefill_batch(self.h, len(p["x"]), p["x"].ctypes.data,
                                     p["session"].ctypes.data, p["clock"].ctypes.data,
                                     p["slot"].ctypes.data, p["active"].ctypes.data,
                                     p["n_active"].ctypes.data, len(p["out_rows"]),
                                     p["out_rows"].ctypes.data, toks.ctypes.data,
                                     None if logits_out is None else logits_out.ctypes.data))
        return toks

    def prefill_batch(self, prompts, rings, start_clocks, sessions=None,
                      logits_out: np.ndarray | None = None) -> np.ndarray:
        """Prefill the prompts of several sessions in one pass (sx_prefill_batch); see
        prefill_plan for the arguments."""
        return self.prefill_run(self.prefill_plan(prompts, rings, start_clocks, sessions),
                                logits_out)

    def launch(self, want_logits: bool = True) -> None:
        check(lib().sx_model_launch(self.h, int(want_logits)))

    def launch_batch(self, n: int, want_logits: bool = True) -> None:
        """Replay the n-session step of the last decode_batch on the engine stream."""
        check(lib().sx_model_launch_batch(self.h, n, int(want_logits)))

    def io(self) -> ModelIO:
        io = ModelIO()
        check(lib().sx_model_get_io(self.h, C.byref(io)))
        return io

    def kcache_ptr(self, layer: int) -> int:
        return int(lib().sx_model_kcache(self.h, layer))

    def vcache_ptr(self, layer: int) -> int:
        return int(lib().sx_model_vcache(self.h, layer))

    @property
    def weight_bytes(self) -> int:
        return int(lib().sx_model_weight_bytes(self.h))

    def kernels_per_token(self, want_logits: bool = True) -> int:
        return int(lib().sx_model_kernels_per_token(self.h, int(want_logits)))


class Archive:
    """The recall tier on the device (sx_archive_*): DiffArchive + integrateMemory over a model."""

    def __init__(self, model: "Model", capacity: int):
        h = C.c_void_p()
        check(lib().sx_archive_create(model.h, capacity, None, C.byref(h)))
        self.h = h
        self.model = model
        self.recall = model.cfg.num_recall
        self.dim = model.cfg.hidden_size

    def close(self):
        if getattr(self, "h", None):
            lib().sx_archive_destroy(self.h)
            self.h = None

    __del__ = _quiet_close

    def integrate(self, ring: "Ring", clock: int) -> np.ndarray:
        n = C.c_uint32()
        sel = np.zeros(max(self.recall, 1), np.uint32)
        check(lib().sx_archive_integrate(self.h, ring.h, clock, C.byref(n), sel.ctypes.data))
        return sel[: n.value]

    @property
    def count(self) -> int:
        return int(lib().sx_archive_count(self.h))

    def entry(self, i: int):
        v = np.zeros(self.dim, np.float32)
        ts, la, ac, sal = C.c_uint64(), C.c_uint64(), C.c_uint32(), C.c_float()
        check(lib().sx_archive_entry(self.h, i, v.ctypes.data, C.byref(ts), C.byref(la),
                                     C.byref(ac), C.byref(sal)))
        return v, ts.value, la.value, ac.value, sal.value
