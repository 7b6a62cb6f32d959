"""Weight ingest on the device: sx_dispatch_quantize / sx_buffer_quantize_device against the CPU
quantiser (quantizeMatrix, src/quant.zig:18-162, restated in the checker and pinned to the
reference's quantiser known-answer tests).  Bit-exact: the block words, and the packed buffer
against sx_buffer_upload_weights of the checker's words."""
import numpy as np
import pytest

import sx
from oracle import oracle as orc

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

MODES = [(sx.QUANT_Q4, orc.QUANT_Q4 if hasattr(orc, "QUANT_Q4") else 2),
         (sx.QUANT_Q8, orc.QUANT_Q8 if hasattr(orc, "QUANT_Q8") else 1)]


def bf16_matrix(rows, cols, seed):
    rng = np.random.default_rng(seed)
    v = (rng.standard_normal((rows, cols)) * rng.uniform(0.01, 3.0, (rows, 1))).astype(np.float32)
    v[0, :32] = 0.0                                   # an all-zero block: d = 0, q = 0
    if cols >= 64:
        v[0, 32:64] = np.linspace(-7.0, 7.0, 32)      # amax 7: many half-way products
        v[0, 40] = 0.5                                # 0.5 * 7 / 7 -> rounds away from zero
        v[0, 41] = -2.5
    bits = v.view(np.uint32)
    return ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16).astype(np.uint16)  # RNE to bf16


@pytest.mark.parametrize("rows,cols", [(16, 64), (37, 96), (256, 3840), (1000, 1536)])
@pytest.mark.parametrize("mode,omode", MODES)
def test_device_quantiser_bit_exact(engine, rows, cols, mode, omode):
    b = bf16_matrix(rows, cols, rows + cols)
    want = orc.quantize_matrix(b, rows, cols, omode)
    src = torch.from_numpy(b.view(np.int16)).cuda()
    out = torch.zeros(want.size, dtype=torch.int32, device="cuda")
    engine.quantize(mode, src, out, rows, cols)
    engine.sync()
    got = out.cpu().numpy().view(np.uint32)
    assert np.array_equal(got, want), f"{np.count_nonzero(got != want)} words differ"


@pytest.mark.parametrize("mode,omode", MODES)
def test_quantize_into_buffer_equals_upload(engine, mode, omode):
    rows, cols = 300, 2048
    b = bf16_matrix(rows, cols, 7)
    nb = sx.packed_bytes(rows, cols, mode)
    via_cpu = engine.buffer(nb)
    via_cpu.upload_weights(orc.quantize_matrix(b, rows, cols, omode), rows, cols, mode)
    via_gpu = engine.buffer(nb)
    via_gpu.quantize_device(torch.from_numpy(b.view(np.int16)).cuda(), rows, cols, mode)
    assert np.array_equal(via_gpu.read(np.uint8, nb), via_cpu.read(np.uint8, nb))


def test_quantize_rejects_bad_shapes(engine):
    src = torch.zeros(64, dtype=torch.int16, device="cuda")
    out = torch.zeros(64, dtype=torch.int32, device="cuda")
    with pytest.raises(sx.SxError):
        engine.quantize(sx.QUANT_Q4, src, out, 2, 48)  # cols not a multiple of 32
