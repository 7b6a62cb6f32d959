"""The batch-prefill GEMM's dequantisation arithmetic, checked on the CPU for every input.

The tcgen05 prefill kernel (sx_prefill.cu, dequant_chunk_sw128) forms each weight as
fma(m, d, -C d) with m = 2^(23-p) + q built by one LOP3 from the nibble at bit position p
(p = 8: C = 2^15 + 8; p = 12: C = 2^11 + 8).  That equals the checker's f32 product (q - 8) * d
(oracle dequant_q4, following quant.zig's Q4_0 block rule) only if -C d is exact in f32 for
every scale the format can hold (f16 scales) and the fused product-sum then rounds once to the
exact value.  These tests enumerate all 16 nibbles x all finite f16 scales."""
import numpy as np
import pytest

MAGIC = {8: (0x47000000, 2.0**15), 12: (0x45000000, 2.0**11)}


def finite_f16_scales():
    h = np.arange(0, 65536, dtype=np.uint32).astype(np.uint16).view(np.float16)
    return h[np.isfinite(h)].astype(np.float32)


@pytest.mark.parametrize("p", [8, 12])
def test_negated_offset_times_scale_is_exact(p):
    d = finite_f16_scales()
    c = np.float32(MAGIC[p][1] + 8.0)
    assert np.array_equal((-c * d).astype(np.float64), -(float(c)) * d.astype(np.float64))


@pytest.mark.parametrize("p", [8, 12])
def test_lop3_magic_gives_offset_nibble(p):
    bits, base = MAGIC[p]
    for q in range(16):
        word = (q << p) | (0xA5A5A5A5 & ~(0xF << p))  # unrelated bits around the nibble
        m = np.uint32((word & (0xF << p)) | bits).view(np.float32)
        assert float(m) == base + q


@pytest.mark.parametrize("p", [8, 12])
def test_fused_form_equals_checker_product(p):
    d = finite_f16_scales()
    base = MAGIC[p][1]
    neg = (np.float32(-(base + 8.0)) * d).astype(np.float64)  # exact (previous test)
    for q in range(16):
        # fma: the exact m*d + (-C d), rounded once to f32 (the float64 sum is exact here:
        # both terms are multiples of d's last bit and the result has at most 15 bits)
        got = ((base + q) * d.astype(np.float64) + neg).astype(np.float32)
        want = np.float32(q - 8) * d
        assert np.array_equal(got, want), q
