"""Batch-prefill Q4_0 GEMM on the tcgen05 tensor cores (sx_dispatch_prefill_gemm).

Parity policy: the dequantised weight inside the GEMM equals the checker's f32 (q - 8) * d
rounded to bf16, bit for bit (checked through the whole path with x = identity rows, where
every output is one product with 1.0), and products of random bf16 activations stay within the
path's tolerance of a float64 product of the same bf16 operands."""
import numpy as np
import pytest

import sx
from oracle import oracle as orc
from tests.conftest import assert_close

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def upload_q4(engine, n, k, seed, stream):
    w = orc.synth_q4(n, k, seed, stream)
    buf = engine.buffer(sx.packed_bytes(n, k, sx.QUANT_Q4))
    buf.upload_weights(w, n, k, sx.QUANT_Q4)
    return w, buf


def deq_bf16(w, n, k):
    return orc.bf16_round(orc.dequant_q4(w, n, k).ravel()).reshape(n, k)


@pytest.mark.parametrize("n,k", [(160, 128), (256, 320), (128, 64)])
def test_dequant_is_bit_exact_through_the_gemm(engine, n, k):
    w, buf = upload_q4(engine, n, k, 3, n + k)
    t = k  # x = identity: y[t][n] = deq(w)[n][t] exactly
    x = torch.eye(t, k, dtype=torch.bfloat16, device="cuda")
    y = torch.full((t, n), float("nan"), dtype=torch.float32, device="cuda")
    engine.prefill_gemm(buf.ptr, x, y, t, n, k)
    engine.sync()
    got = y.cpu().numpy()
    want = deq_bf16(w, n, k).T
    assert np.array_equal(got.view(np.uint32), want.astype(np.float32).view(np.uint32)), (
        f"{np.sum(got != want)} of {got.size} dequantised values differ")


@pytest.mark.parametrize("t,n,k", [(300, 384, 512), (512, 2560, 1536), (1000, 640, 2048),
                                   (17, 128, 6144)])
def test_gemm_matches_float64_product(engine, t, n, k):
    w, buf = upload_q4(engine, n, k, 5, 7 * n + k)
    xs = orc.bf16_round(np.random.default_rng(t + n).standard_normal(t * k).astype(np.float32))
    x = torch.from_numpy(xs.reshape(t, k)).to(torch.bfloat16).cuda()
    y = torch.empty((t, n), dtype=torch.float32, device="cuda")
    engine.prefill_gemm(buf.ptr, x, y, t, n, k)
    engine.sync()
    ref = xs.reshape(t, k).astype(np.float64) @ deq_bf16(w, n, k).astype(np.float64).T
    assert_close(y.cpu().numpy().ravel(), ref.ravel(), what=f"prefill gemm {t}x{n}x{k}")


def test_gemm_rejects_bad_shapes(engine):
    buf = engine.buffer(sx.packed_bytes(128, 96, sx.QUANT_Q4))
    x = torch.zeros((4, 96), dtype=torch.bfloat16, device="cuda")
    y = torch.zeros((4, 128), dtype=torch.float32, device="cuda")
    with pytest.raises(sx.SxError):
        engine.prefill_gemm(buf.ptr, x, y, 4, 128, 96)  # k not a multiple of 64
    buf2 = engine.buffer(sx.packed_bytes(130, 128, sx.QUANT_Q4))
    x2 = torch.zeros((4, 128), dtype=torch.bfloat16, device="cuda")
    y2 = torch.zeros((4, 130), dtype=torch.float32, device="cuda")
    with pytest.raises(sx.SxError):
        engine.prefill_gemm(buf2.ptr, x2, y2, 4, 130, 128)  # rows of y not 16-byte multiples
