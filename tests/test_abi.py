"""The C ABI: the library loads, exports every symbol include/sx.h declares, and its host-only
entry points (ring bookkeeping, formats, RoPE table, synthetic embeddings) agree bit for bit
with the CPU checker.  No GPU needed."""
import re
from pathlib import Path

import numpy as np
import pytest

import sx
from oracle import oracle as orc

HEADER = Path(__file__).resolve().parents[1] / "include" / "sx.h"


def header_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"SX_API\s+[\w\s\*]+?\b(sx_\w+)\s*\(", text)))


def test_header_declares_api():
    syms = header_symbols()
    assert len(syms) > 50
    assert "sx_record_gemv" in syms and "sx_submit" in syms and "sx_forward_token" in syms


def test_library_exports_every_declared_symbol():
    L = sx.lib()
    missing = [s for s in header_symbols() if not hasattr(L, s)]
    assert not missing, f"libsx.so lacks {missing}"


def test_binding_covers_header():
    assert sorted(sx.declared_symbols()) == header_symbols()


def test_status_strings():
    L = sx.lib()
    for code in range(9):
        assert L.sx_status_string(code)
    assert sx.lib().sx_version().decode().startswith("sx")


def test_quantized_row_words_matches_quant_zig():
    for cols in (32, 40, 1536, 3840, 15360):
        for mode in (sx.QUANT_Q4, sx.QUANT_Q8):
            assert sx.quantized_row_words(cols, mode) == orc.quantized_row_words(cols, mode)


def test_packed_bytes_equal_reference_bytes_on_aligned_shapes():
    # 16-row tiles x 64-column pairs: same 20 B / 36 B per 32-value block as the reference
    for rows, cols in ((6144, 1536), (3840, 15360), (262144, 3840)):
        assert sx.packed_bytes(rows, cols, sx.QUANT_Q4) == rows * cols // 32 * 20
        assert sx.packed_bytes(rows, cols, sx.QUANT_Q8) == rows * cols // 32 * 36
    # ragged shapes pad to whole tiles / pairs
    assert sx.packed_bytes(17, 96, sx.QUANT_Q4) == 2 * 2 * 640


@pytest.mark.parametrize("rot,theta", [(64, 1e6), (256, 1e4), (128, 5e5)])
def test_rope_table_bit_identical(rot, theta):
    assert np.array_equal(sx.rope_inv_freq(rot, theta), orc.rope_inv_freq(rot, theta))


def test_synth_embed_row_bit_identical():
    for tok in (0, 1, 262143):
        assert np.array_equal(sx.synth_embed_row(3840, tok, 99), orc.synth_embed_row(3840, tok, 99))


@pytest.mark.parametrize("anchors,window,recall", [(32, 512, 96), (4, 8, 4), (0, 16, 0), (2, 4, 3)])
def test_ring_bit_exact_against_checker(anchors, window, recall):
    rng = np.random.default_rng(anchors * 1000 + window)
    a = sx.Ring(1, anchors, window, recall)
    b = orc.Ring(1, anchors, window, recall)
    clock = 0
    for step in range(600):
        op = rng.integers(0, 10)
        if op < 7:
            clock += int(rng.integers(1, 3))
            assert a.activate_slot(0, clock) == b.activate_slot(0, clock)
        elif op < 9 and recall:
            rank = int(rng.integers(0, recall))
            c = int(rng.integers(0, clock + 2))
            a.write_recall(0, rank, c)
            b.write_recall(0, rank, c)
        else:
            a.clear_recall()
            b.clear_recall()
        q = clock + int(rng.integers(-2, 3))
        q = max(q, 0)
        assert np.array_equal(a.get_active_slots(0, q), b.get_active_slots(0, q))
        assert a.get_slot_index(q) == b.get_slot_index(q)


def test_ring_reference_cases_through_abi():
    ring = sx.Ring(2, 4, 8, 4)
    assert ring.total_slots == 16
    for c in range(20):
        ring.activate_slot(0, c)
    s = ring.get_active_slots(0, 19)
    assert len(s) == 12 and s[0] == 0 and s[3] == 3
    r2 = sx.Ring(1, 2, 4, 3)
    r2.write_recall(0, 0, 100)
    r2.write_recall(0, 1, 50)
    assert len(r2.get_active_slots(0, 101)) == 2
    r2.clear_recall()
    assert len(r2.get_active_slots(0, 101)) == 0


def test_ring_prefill_equals_activation_history():
    a = sx.Ring(1, 32, 512, 96)
    b = sx.Ring(1, 32, 512, 96)
    a.prefill(0, 3000)
    for c in range(3000):
        b.activate_slot(0, c)
    for q in (2999, 3000, 3100):
        assert np.array_equal(a.get_active_slots(0, q), b.get_active_slots(0, q))


def test_ring_rejects_bad_geometry():
    with pytest.raises(sx.SxError):
        sx.Ring(1, 4, 0, 4)


def test_engine_create_without_gpu_fails_cleanly():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(sx.SxError):
        sx.Engine(0)
