"""The engine's other layer formats (src/gpu/kernels.zig:36-41 GpuEngine.init by mode) on a B200:
mode q8 (Q8_0 layers: gemv_q8.wgsl, fused_mlp_q8.wgsl; Q8_0 LM head) and mode none (bf16 layers:
gemv_bf16.wgsl for every projection and the logits), kernel by kernel and as whole-token greedy
decode, against the CPU checker in the same layer format."""
import numpy as np
import pytest

import sx
from oracle import oracle as orc
from tests.conftest import assert_close
from tests.test_gpu_model import margin_top2, tiny_cfg

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.fixture(scope="module")
def eng_q8():
    e = sx.Engine(0, mode=sx.QUANT_Q8)
    yield e
    e.close()


@pytest.fixture(scope="module")
def eng_bf16():
    e = sx.Engine(0, mode=sx.QUANT_NONE)
    yield e
    e.close()


def bf16_bits(a):
    return (np.asarray(a, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def test_gemv_bf16_reference_test_inputs(eng_bf16):
    # test_gpu_suite.zig:9-54: M 512, K 1024, w = bf16-truncated U(-0.05, 0.05),
    # x = U(-0.25, 0.25), max-abs error against kernels.gemv below 1e-3
    m, k = 512, 1024
    rng = np.random.default_rng(101)
    w = bf16_bits((rng.random(m * k, dtype=np.float32) - 0.5) * 0.1)
    x = ((rng.random(k, dtype=np.float32) - 0.5) * 0.5).astype(np.float32)
    buf = eng_bf16.buffer(sx.packed_bytes(m, k, sx.QUANT_NONE))
    buf.upload_weights(w.view(np.uint32), m, k, sx.QUANT_NONE)
    y = torch.empty(m, dtype=torch.float32, device="cuda")
    eng_bf16.gemv(sx.QUANT_NONE, buf.ptr, dev(x), y, m, k, 1)
    assert np.max(np.abs(host(y) - orc.gemv_bf16(w, x, m, k))) < 1e-3


@pytest.mark.parametrize("m,k,batch", [(3840, 3840, 1), (2048, 1536, 8), (100, 264, 3),
                                       (262144, 64, 1)])
def test_gemv_bf16_matches_checker(eng_bf16, m, k, batch):
    rng = np.random.default_rng(m + k)
    w = bf16_bits(rng.standard_normal(m * k).astype(np.float32) * 0.02)
    x = rng.standard_normal((batch, k)).astype(np.float32)
    buf = eng_bf16.buffer(sx.packed_bytes(m, k, sx.QUANT_NONE))
    buf.upload_weights(w.view(np.uint32), m, k, sx.QUANT_NONE)
    y = torch.empty(batch, m, dtype=torch.float32, device="cuda")
    eng_bf16.gemv(sx.QUANT_NONE, buf.ptr, dev(x), y, m, k, batch)
    got = host(y)
    for b in range(batch):
        assert_close(got[b], orc.gemv_bf16(w, x[b], m, k), what=f"gemv_bf16 row {b}")


@pytest.mark.parametrize("i,h,batch", [(1536, 3840, 1), (640, 256, 4)])
def test_gate_up_bf16_matches_checker(eng_bf16, i, h, batch):
    rng = np.random.default_rng(i)
    wg = bf16_bits(rng.standard_normal(i * h).astype(np.float32) * 0.02)
    wu = bf16_bits(rng.standard_normal(i * h).astype(np.float32) * 0.02)
    x = rng.standard_normal((batch, h)).astype(np.float32)
    bg = eng_bf16.buffer(sx.packed_bytes(i, h, sx.QUANT_NONE))
    bu = eng_bf16.buffer(sx.packed_bytes(i, h, sx.QUANT_NONE))
    bg.upload_weights(wg.view(np.uint32), i, h, sx.QUANT_NONE)
    bu.upload_weights(wu.view(np.uint32), i, h, sx.QUANT_NONE)
    y = torch.empty(batch, i, dtype=torch.float32, device="cuda")
    eng_bf16.gate_up(bg.ptr, bu.ptr, dev(x), y, i, h, batch)
    got = host(y)
    for b in range(batch):
        assert_close(got[b], orc.gate_up_geglu_bf16(wg, wu, x[b], i, h), what=f"row {b}")


@pytest.mark.parametrize("i,h,batch", [(6144, 1536, 1), (6144, 1536, 8), (15360, 3840, 1),
                                       (96, 160, 3)])
def test_gate_up_q8_matches_checker(eng_q8, i, h, batch):
    # fused_mlp_q8.wgsl: gelu_tanh(Wg . x) * (Wu . x) with Q8_0 weights
    wg = orc.synth_q8(i, h, 23, 1)
    wu = orc.synth_q8(i, h, 23, 2)
    bg = eng_q8.buffer(sx.packed_bytes(i, h, sx.QUANT_Q8))
    bu = eng_q8.buffer(sx.packed_bytes(i, h, sx.QUANT_Q8))
    bg.upload_weights(wg, i, h, sx.QUANT_Q8)
    bu.upload_weights(wu, i, h, sx.QUANT_Q8)
    gain = orc.synth_gain(h, 23, 3)
    xs = np.stack([orc.rmsnorm(np.random.default_rng(b).standard_normal(h).astype(np.float32), gain)
                   for b in range(batch)])
    y = torch.empty(batch, i, dtype=torch.float32, device="cuda")
    eng_q8.gate_up(bg.ptr, bu.ptr, dev(xs), y, i, h, batch)
    got = host(y)
    # Against the exact (float64) product of the dequantised weights: with Q8 weights at this
    # scale the pre-activations reach ~100, and where the gate is near zero y = gelu(g) u
    # ~ g u / 2 turns the checker's own sequential-f32 rounding in g into a relative error of
    # the small product above 1e-2; the f64 product has no such error.
    dg = orc.dequant_q8(wg, i, h).astype(np.float64)
    du = orc.dequant_q8(wu, i, h).astype(np.float64)
    for b in range(batch):
        g, u = dg @ xs[b].astype(np.float64), du @ xs[b].astype(np.float64)
        want = 0.5 * g * (1.0 + np.tanh(0.7978845608 * (g + 0.044715 * g ** 3))) * u
        assert_close(got[b], want, what=f"geglu q8 row {b} vs f64")


def assert_close_few(got, want, what, frac=2e-3, scale_tol=1e-4):
    """Q8 layers: every GeGLU product with a gate near zero carries the checker's own f32
    summation error times a large up value (see test_gate_up_q8_matches_checker), which the
    following layers spread thinly: all but a fraction `frac` of the logits meet the
    elementwise bound, and every logit lies within scale_tol of the logit scale (a wrong row,
    block or scale moves logits by the order of the scale)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    err = np.abs(got - want)
    bad = int(np.count_nonzero(err > 1e-3 + 1e-2 * np.abs(want)))
    scale = float(np.abs(want).max())
    assert bad <= max(1, int(frac * err.size)), f"{what}: {bad} of {err.size} past the bound"
    assert err.max() <= scale_tol * scale, f"{what}: worst {err.max():.3e}, scale {scale:.3e}"


def run(engine, cfg, layer_quant, seed, steps, start_clock, n_recall=0):
    model = sx.Model(engine, sx.model_config(**cfg))
    model.synth_weights(seed)
    model.fill_kv(seed)
    ref = orc.Model(dict(cfg, layer_quant=layer_quant), seed)
    ref.fill_kv(seed)
    ring = sx.Ring(1, cfg["num_anchors"], cfg["window_size"], cfg["num_recall"])
    ring.prefill(0, start_clock)
    ref.ring.prefill(0, start_clock)
    rng = np.random.default_rng(seed)
    for r in range(n_recall):
        c = int(rng.integers(0, max(start_clock, 1)))
        ring.write_recall(0, r, c)
        ref.ring.write_recall(0, r, c)
    token = 5
    for i in range(steps):
        clock = start_clock + i
        x = sx.synth_embed_row(cfg["hidden_size"], token, seed)
        slot = ring.activate_slot(0, clock)
        logits = np.zeros(cfg["vocab_size"], np.float32)
        tok = model.forward_token(x, clock, slot, ring.get_active_slots(0, clock), True, logits)
        rtok, rlg, _ = ref.forward(x, clock, True)
        if layer_quant == orc.QUANT_Q8:
            assert_close_few(logits, rlg, what=f"logits step {i}")
        else:
            assert_close(logits, rlg, what=f"logits step {i}")
        if tok != rtok:
            assert margin_top2(rlg) < 1e-3, f"step {i}: token {tok} vs {rtok}"
        token = tok


@pytest.mark.parametrize("graph", [0, 1])
def test_q8_layer_model_decodes_like_checker(eng_q8, graph):
    # fused graph (Q8 GEMV / GeGLU kernels with the norm prologues) and the op-by-op graph
    run(eng_q8, tiny_cfg(reference_graph=graph), orc.QUANT_Q8, seed=7, steps=10, start_clock=3,
        n_recall=0)


def test_q8_layer_model_12b_width(eng_q8):
    cfg = tiny_cfg(vocab_size=16384, hidden_size=3840, intermediate_size=15360, num_layers=2,
                   num_q_heads=16, num_kv_heads=8, num_global_kv_heads=8, head_dim=256,
                   global_head_dim=256, num_anchors=32, window_size=512, num_recall=96,
                   full_every=2)
    run(eng_q8, cfg, orc.QUANT_Q8, seed=3, steps=2, start_clock=4000, n_recall=20)


def test_bf16_layer_model_decodes_like_checker(eng_bf16):
    # mode none: every projection and the logits through gemv_bf16 semantics
    run(eng_bf16, tiny_cfg(reference_graph=1), orc.QUANT_NONE, seed=11, steps=10, start_clock=6,
        n_recall=2)


def test_layer_modes_reject_what_they_do_not_run(eng_bf16, eng_q8):
    with pytest.raises(sx.SxError):  # bf16 layers only in the op-by-op graph
        sx.Model(eng_bf16, sx.model_config(**tiny_cfg(reference_graph=0)))
    m = sx.Model(eng_q8, sx.model_config(**tiny_cfg(num_sessions=1)))
    ring = sx.Ring(1, 4, 8, 4)
    with pytest.raises(sx.SxError):  # the batched prefill GEMM is Q4_0
        m.prefill_batch([np.zeros((2, 256), np.float32)], [ring], [0])
