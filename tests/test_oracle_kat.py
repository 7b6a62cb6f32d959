"""Pin the CPU checker against the reference's own known-answer tests.

The reference (Zig) cannot be built here, so its tests are restated: every case cites the
reference test it comes from.  The quantiser cases are hand-derived from quant.zig's
algorithm (round half away from zero, clamp, +8 offset, nibble order).
"""
import numpy as np
import pytest

from oracle import oracle as orc


def _bf16_trunc(f32: np.ndarray) -> np.ndarray:
    """The reference tests' `@truncate(bits >> 16)` bf16 conversion."""
    return (np.ascontiguousarray(f32, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def _bf16_bits(vals) -> np.ndarray:
    return _bf16_trunc(np.asarray(vals, np.float32))


# --- tensor.zig:30-41 ------------------------------------------------------------------
def test_bf16_roundtrip_tensor_zig():
    assert abs(orc.bf16_to_f32(orc.bf16_from_f32(3.1415926)) - 3.1415926) <= 0.02
    assert orc.bf16_to_f32(orc.bf16_from_f32(0.0)) == 0.0
    assert abs(orc.bf16_to_f32(orc.bf16_from_f32(-42.5)) + 42.5) <= 0.1


def test_bf16_round_to_nearest_even_ties():
    # 1 + 2^-8 is halfway between 1.0 (even) and 1.0078125: RNE keeps 1.0
    assert orc.bf16_to_f32(orc.bf16_from_f32(1.0 + 2.0**-8)) == 1.0
    # 1 + 3*2^-8 is halfway between 1.0078125 (odd) and 1.015625 (even): rounds up
    assert orc.bf16_to_f32(orc.bf16_from_f32(1.0 + 3 * 2.0**-8)) == 1.015625
    vals = np.random.default_rng(0).standard_normal(4096).astype(np.float32)
    assert np.array_equal(
        orc.bf16_round(vals), np.array([orc.bf16_to_f32(orc.bf16_from_f32(v)) for v in vals],
                                       np.float32))


# --- kernels.zig:176-183 ---------------------------------------------------------------
def test_gemv_known_answer_kernels_zig():
    w = _bf16_bits([1.0, 2.0, 3.0, 4.0])
    y = orc.gemv_bf16(w, np.array([1.0, 2.0], np.float32), 2, 2)
    assert abs(y[0] - 5.0) <= 0.01 and abs(y[1] - 11.0) <= 0.01


# --- ring_buffer.zig:149-166 -----------------------------------------------------------
def test_ring_tiers_and_window_eviction():
    ring = orc.Ring(2, 4, 8, 4)
    assert ring.total_slots == 16
    for c in range(20):
        ring.activate_slot(0, c)  # writeKV's slot bookkeeping
    slots = ring.get_active_slots(0, 19)
    assert len(slots) == 12
    assert slots[0] == 0 and slots[3] == 3


# --- ring_buffer.zig:168-187 -----------------------------------------------------------
def test_ring_recall_written_cleared_included():
    ring = orc.Ring(1, 2, 4, 3)
    ring.write_recall(0, 0, 100)
    ring.write_recall(0, 1, 50)
    assert len(ring.get_active_slots(0, 101)) == 2
    ring.clear_recall()
    assert len(ring.get_active_slots(0, 101)) == 0


def test_ring_slot_index_rule():
    ring = orc.Ring(1, 32, 512, 96)
    assert [ring.get_slot_index(c) for c in (0, 31, 32, 543, 544, 545)] == [0, 31, 32, 543, 32, 33]


# --- quant.zig:53-90 (hand-derived) ----------------------------------------------------
def test_q4_quantize_known_block():
    vals = np.zeros(32, np.float32)
    vals[:5] = [7.0, 2.5, -2.5, 0.5, -0.5]
    w = orc.quantize_matrix(_bf16_bits(vals), 1, 32, orc.QUANT_Q4)
    assert w.view(np.float32)[0] == 1.0  # d = amax / 7
    nib = [(int(w[1 + i // 8]) >> (4 * (i % 8))) & 0xF for i in range(32)]
    # q = round_half_away(v * 7 / amax): 7, 3, -3, 1, -1, then 0 -> stored q + 8
    assert nib[:5] == [15, 11, 5, 9, 7]
    assert nib[5:] == [8] * 27


def test_q4_zero_block():
    w = orc.quantize_matrix(np.zeros(32, np.uint16), 1, 32, orc.QUANT_Q4)
    assert w[0] == 0 and all(int(x) == 0x88888888 for x in w[1:5])


# --- quant.zig:18-51 (hand-derived) ----------------------------------------------------
def test_q8_quantize_known_block():
    vals = np.zeros(32, np.float32)
    vals[:4] = [127.0, 2.5, -2.5, 0.5]
    w = orc.quantize_matrix(_bf16_bits(vals), 1, 32, orc.QUANT_Q8)
    assert w.view(np.float32)[0] == 1.0
    q = np.frombuffer(w[1:9].tobytes(), np.int8)
    assert list(q[:4]) == [127, 3, -3, 1]  # half away from zero, not half even
    assert not q[4:].any()


def test_quantized_row_words_quant_zig():
    assert orc.quantized_row_words(3840, orc.QUANT_Q4) == 120 * 5
    assert orc.quantized_row_words(3840, orc.QUANT_Q8) == 120 * 9
    assert orc.quantized_row_words(40, orc.QUANT_Q4) == 2 * 5  # (cols + 31) / 32 blocks


# --- gpu.zig:30-59 (all-ones Q4 GEMV is positive) ---------------------------------------
def test_q4_all_ones_positive_gpu_zig():
    m, k = 64, 128
    raw = np.full(m * k, 0x3F80, np.uint16)
    w = orc.quantize_matrix(raw, m, k, orc.QUANT_Q4)
    x = (np.arange(k) % 5).astype(np.float32) * 0.25
    y = orc.gemv_q4(w, x, m, k)
    assert np.all(y > 0)
    assert np.allclose(y, x.sum(), rtol=1e-6)  # all weights dequantise to exactly 1.0


# --- test_q4_exec.zig:16-101 (3840 x 15360, max-abs < 1e-3) ------------------------------
def test_q4_gemv_down_proj_shape_test_q4_exec():
    m, k = 3840, 15360
    rng = np.random.default_rng(42)
    w_f = ((rng.random(m * k, dtype=np.float32) - 0.5) * 0.2).astype(np.float32)
    w = orc.quantize_matrix(_bf16_trunc(w_f), m, k, orc.QUANT_Q4)
    x = ((rng.random(k, dtype=np.float32) - 0.5) * 0.5).astype(np.float32)
    y = orc.gemv_q4(w, x, m, k)
    # independent float64 recomputation of the dequantised product
    words = w.reshape(m, k // 32, 5)
    d = words[:, :, 0].view(np.float32).astype(np.float64)
    shifts = np.arange(8, dtype=np.uint32) * 4
    nib = ((words[:, :, 1:, None] >> shifts) & 0xF).reshape(m, k // 32, 32).astype(np.float64)
    ref = (((nib - 8.0) * d[:, :, None]).reshape(m, k) @ x.astype(np.float64))
    assert np.max(np.abs(y - ref)) < 1e-3


# --- test_gpu_suite.zig:9-54 (bf16 GEMV 512 x 1024 < 1e-3) -------------------------------
def test_bf16_gemv_test_gpu_suite():
    m, k = 512, 1024
    rng = np.random.default_rng(101)
    w = _bf16_trunc((rng.random(m * k, dtype=np.float32) - 0.5) * 0.1)
    x = ((rng.random(k, dtype=np.float32) - 0.5) * 0.5).astype(np.float32)
    y = orc.gemv_bf16(w, x, m, k)
    wf = (w.astype(np.uint32) << 16).view(np.float32).astype(np.float64).reshape(m, k)
    assert np.max(np.abs(y - wf @ x.astype(np.float64))) < 1e-3


# --- test_gpu_suite.zig:56-102 (RMSNorm D=2048 < 1e-4) -----------------------------------
def test_rmsnorm_test_gpu_suite():
    d, eps = 2048, 1e-6
    rng = np.random.default_rng(202)
    x = ((rng.random(d, dtype=np.float32) - 0.5) * 2.0).astype(np.float32)
    wb = _bf16_trunc((1.0 + (rng.random(d, dtype=np.float32) - 0.5) * 0.1).astype(np.float32))
    w = (wb.astype(np.uint32) << 16).view(np.float32)
    y = orc.rmsnorm(x, w, eps)
    x64 = x.astype(np.float64)
    ref = x64 / np.sqrt(np.mean(x64 * x64) + eps) * w
    assert np.max(np.abs(y - ref)) < 1e-4


# --- kernels.zig:164-174 argmax: first index of the maximum -----------------------------
def test_argmax_first_index_of_max():
    v = np.array([1.0, 3.0, -2.0, 3.0, 0.5], np.float32)
    assert orc.argmax(v) == 1
    assert orc.argmax(np.full(7, -np.inf, np.float32)) == 0
    v2 = np.array([np.nan, 5.0, 6.0], np.float32)
    assert orc.argmax(v2) == 0  # max starts at logits[0]; NaN is never beaten


# --- kernels.zig:94-97 ------------------------------------------------------------------
@pytest.mark.parametrize("x", [-6.0, -1.0, -0.1, 0.0, 0.3, 1.0, 4.0])
def test_gelu_tanh(x):
    ref = 0.5 * x * (1.0 + np.tanh(0.7978845608 * (x + 0.044715 * x**3)))
    assert abs(orc.gelu_tanh(x) - ref) <= 1e-6 * max(1.0, abs(ref))


# --- kernels.zig:132-150 RoPE --------------------------------------------------------------
def test_rope_partial_rotates_prefix_only():
    d, rot = 256, 64
    v = np.random.default_rng(3).standard_normal(d).astype(np.float32)
    freq = orc.rope_inv_freq(rot, 1e6)
    out = v.copy()
    orc.lib().orc_apply_rope_partial(out.ctypes.data, d, 12345, d, rot, freq.ctypes.data)
    assert np.array_equal(out[rot:], v[rot:])
    half = rot // 2
    ang = np.float32(12345) * freq
    ref0 = v[:half] * np.cos(ang) - v[half:rot] * np.sin(ang)
    assert np.max(np.abs(out[:half] - ref0)) < 1e-5
    # rotation preserves pair norms
    n0 = v[:half] ** 2 + v[half:rot] ** 2
    n1 = out[:half] ** 2 + out[half:rot] ** 2
    assert np.allclose(n0, n1, rtol=1e-5)


# ---- memory.zig:153-175: the archive's own tests, on the checker's restatement
def test_archive_recall_ranks_cosine_match_above_recency():
    a = orc.Archive(None, 8, dim=4)
    a.append(0, 0.5, [1, 0, 0, 0])
    a.append(1, 0.5, [0, 1, 0, 0])
    idx = a.scan(np.array([1, 0, 0, 0], np.float32), 2, 2)
    assert len(idx) == 2 and idx[0] == 0


def test_archive_wraps_and_caps_count():
    a = orc.Archive(None, 3, dim=2)
    for t, v in enumerate(([1, 0], [0, 1], [1, 1], [-1, 0])):
        a.append(t, 0.0, v)
    assert a.count == 3 and a.write_head == 1


def test_archive_scan_is_selection_with_swaps():
    # equal scores resolve by position after the swaps of memory.zig:123-134, not by index:
    # scores [1, 1, 5] (salience only, zero vectors) select 2, then 1, then 0
    a = orc.Archive(None, 4, alpha=0.0, beta=0.0, gamma=1.0, dim=2)
    for sal in (1.0, 1.0, 5.0):
        a.append(0, sal, [0, 0])
    assert list(a.scan(np.zeros(2, np.float32), 0, 3)) == [2, 1, 0]
