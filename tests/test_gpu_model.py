"""Model-level parity on a B200: the record API replaying recordLayerDirect, and whole-token
greedy decode through sx_forward_token (gpuDispatchForwardToken), against the CPU checker's
decode in the GPU graph's op order."""
import ctypes
import math

import numpy as np
import pytest

import sx
from oracle import oracle as orc
from tests.conftest import assert_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

_libm = ctypes.CDLL("libm.so.6")
_libm.fmaf.restype = ctypes.c_float
_libm.fmaf.argtypes = [ctypes.c_float] * 3


def tiny_cfg(**kw):
    cfg = dict(
        vocab_size=4096, hidden_size=256, intermediate_size=640, num_layers=3,
        num_q_heads=4, num_kv_heads=2, num_global_kv_heads=2, head_dim=64, global_head_dim=64,
        num_anchors=4, window_size=8, num_recall=4, kv_bf16=1, has_post_norms=1, full_every=3,
        attention_k_eq_v=0, rms_norm_eps=1e-6, rope_theta=10000.0, rope_theta_full=1000000.0,
        attn_scale=1.0,
    )
    cfg.update(kw)
    return cfg


def margin_top2(logits):
    s = np.sort(logits)
    return float(s[-1] - s[-2])


def run_decode(engine, cfg, seed, steps, start_clock, n_recall=0):
    """Greedy decode on both sides, feeding the GPU's token back to both."""
    model = sx.Model(engine, sx.model_config(**cfg))
    model.synth_weights(seed)
    model.fill_kv(seed)
    ref = orc.Model(cfg, seed)
    ref.fill_kv(seed)
    ring = sx.Ring(1, cfg["num_anchors"], cfg["window_size"], cfg["num_recall"])
    ring.prefill(0, start_clock)
    ref.ring.prefill(0, start_clock)
    rng = np.random.default_rng(seed)
    for r in range(n_recall):
        c = int(rng.integers(0, max(start_clock, 1)))
        ring.write_recall(0, r, c)
        ref.ring.write_recall(0, r, c)
    token = 17
    results = []
    for t in range(steps):
        clock = start_clock + t
        x = sx.synth_embed_row(cfg["hidden_size"], token, seed)
        assert np.array_equal(x, orc.synth_embed_row(cfg["hidden_size"], token, seed))
        slot = ring.activate_slot(0, clock)
        slots = ring.get_active_slots(0, clock)
        logits = np.zeros(cfg["vocab_size"], np.float32)
        tok = model.forward_token(x, clock, slot, slots, True, logits)
        rtok, rlogits, _ = ref.forward(x, clock, True)
        assert np.array_equal(slots, ref.ring.get_active_slots(0, clock))
        results.append((tok, rtok, logits, rlogits))
        token = tok
    return results


# fused kernels, the reference's op-by-op graph, one persistent launch, fused kernels with the
# attention block (q|k|v, attention, o) as one kernel
GRAPHS = [0, 1, 2, 4]


@pytest.mark.parametrize("reference_graph", GRAPHS)
@pytest.mark.parametrize("kv_f32", [False, True])
def test_greedy_decode_matches_checker(engine, engine_f32kv, kv_f32, reference_graph):
    eng = engine_f32kv if kv_f32 else engine
    cfg = tiny_cfg(kv_bf16=0 if kv_f32 else 1, reference_graph=reference_graph)
    res = run_decode(eng, cfg, seed=3, steps=24, start_clock=0)  # window wraps twice
    from tests.conftest import assert_close_bf16_operands
    for i, (tok, rtok, lg, rlg) in enumerate(res):
        if kv_f32:
            assert_close(lg, rlg, what=f"logits step {i}")
        else:  # a cached element rounded from f32 values one ulp apart differs by 2^-8
            assert_close_bf16_operands(lg, rlg, what=f"logits step {i}")
        if tok != rtok:
            assert margin_top2(rlg) < 1e-3, f"step {i}: token {tok} vs {rtok}"


@pytest.mark.parametrize("reference_graph", GRAPHS)
def test_greedy_decode_with_recall_and_large_clock(engine, reference_graph):
    cfg = tiny_cfg(reference_graph=reference_graph)
    res = run_decode(engine, cfg, seed=9, steps=6, start_clock=90000, n_recall=3)
    for i, (tok, rtok, lg, rlg) in enumerate(res):
        assert_close(lg, rlg, what=f"logits step {i}")
        if tok != rtok:
            assert margin_top2(rlg) < 1e-3


def test_long_ring_uses_global_merge(engine):
    # 1108 live slots: more than 16 clusters of 64 slots, so the fused graph's attention
    # takes the global-merge form (one record per 32-slot chunk, last CTA merges)
    cfg = tiny_cfg(num_anchors=4, window_size=1100, num_recall=4, num_layers=2)
    res = run_decode(engine, cfg, seed=13, steps=3, start_clock=3000, n_recall=2)
    for i, (tok, rtok, lg, rlg) in enumerate(res):
        assert_close(lg, rlg, what=f"logits step {i}")
        if tok != rtok:
            assert margin_top2(rlg) < 1e-3


@pytest.mark.parametrize("reference_graph", [0, 2, 4])
def test_12b_width_two_layers_full_vocab(engine, reference_graph):
    # 12B layer shapes and full vocabulary with two layers (one sliding, one full attention)
    cfg = tiny_cfg(vocab_size=262144, hidden_size=3840, intermediate_size=15360, num_layers=2,
                   num_q_heads=16, num_kv_heads=8, num_global_kv_heads=8, head_dim=256,
                   global_head_dim=256, num_anchors=32, window_size=512, num_recall=96,
                   full_every=2, reference_graph=reference_graph)
    res = run_decode(engine, cfg, seed=5, steps=2, start_clock=5000, n_recall=96)
    for i, (tok, rtok, lg, rlg) in enumerate(res):
        assert_close(lg, rlg, what=f"logits step {i}")
        if tok != rtok:
            assert margin_top2(rlg) < 1e-3


@pytest.mark.parametrize("reference_graph", GRAPHS)
def test_prefill_graph_skips_logits(engine, reference_graph):
    cfg = tiny_cfg(reference_graph=reference_graph)
    model = sx.Model(engine, sx.model_config(**cfg))
    model.synth_weights(1)
    ring = sx.Ring(1, 4, 8, 4)
    x = sx.synth_embed_row(256, 3, 1)
    slot = ring.activate_slot(0, 0)
    tok = model.forward_token(x, 0, slot, ring.get_active_slots(0, 0), want_logits=False)
    assert tok == 0
    if reference_graph == 2:  # every phase, LM head included, is one launch
        assert model.kernels_per_token(False) == model.kernels_per_token(True) == 1
    else:
        assert model.kernels_per_token(False) < model.kernels_per_token(True)
        # op-by-op: 14; fused: q|k|v, attention with the o projection folded in, gate+up,
        # down; graph 4: attention block + gate+up + down
        per_layer = {1: 14, 0: 4, 4: 3}[reference_graph]
        L = cfg["num_layers"]
        gates = (L - L // 3) if reference_graph == 1 else 0  # recordLayerIndirect's gate
        assert model.kernels_per_token(False) == per_layer * L + gates


def mid_cfg(**kw):
    """The smallest shapes the streaming graph (reference_graph 3) accepts: every GEMV input at
    least 16 block pairs (K >= 1024)."""
    return tiny_cfg(vocab_size=8192, hidden_size=1024, intermediate_size=2048, num_q_heads=16,
                    num_kv_heads=8, num_global_kv_heads=8, head_dim=64, global_head_dim=64, **kw)


@pytest.mark.parametrize("kv_f32", [False, True])
def test_stream_graph_greedy_decode_matches_checker(engine, engine_f32kv, kv_f32):
    """Graph mode 3 (sx_stream.cu: one launch per token, producer-warp weight ring) against the
    checker, with the window wrapping twice."""
    from tests.conftest import assert_close_bf16_operands
    eng = engine_f32kv if kv_f32 else engine
    cfg = mid_cfg(kv_bf16=0 if kv_f32 else 1, reference_graph=3)
    res = run_decode(eng, cfg, seed=23, steps=20, start_clock=0)
    for i, (tok, rtok, lg, rlg) in enumerate(res):
        if kv_f32:
            assert_close(lg, rlg, what=f"logits step {i}")
        else:  # cached K/V rounded to bf16 on both sides: the double-rounding allowance
            assert_close_bf16_operands(lg, rlg, what=f"logits step {i}")
        if tok != rtok:
            assert margin_top2(rlg) < 1e-3, f"step {i}: token {tok} vs {rtok}"


def test_stream_graph_equals_fused_graph_bits(engine):
    """The streaming kernel sums each tile's chunk partials in a different order than the fused
    GEMV kernels, so the two graphs agree within the f32 tolerance; both against each other
    over a recall tier and a large clock."""
    outs = []
    for g in (0, 3):
        cfg = mid_cfg(reference_graph=g)
        res = run_decode(engine, cfg, seed=31, steps=4, start_clock=70000, n_recall=4)
        outs.append(res)
    for i, ((t0, r0, l0, _), (t3, r3, l3, rl)) in enumerate(zip(*outs)):
        assert_close(l3, l0, what=f"stream vs fused logits step {i}")
        assert_close(l3, rl, what=f"stream vs checker logits step {i}")


def test_stream_graph_12b_width_full_vocab(engine):
    cfg = tiny_cfg(vocab_size=262144, hidden_size=3840, intermediate_size=15360, num_layers=2,
                   num_q_heads=16, num_kv_heads=8, num_global_kv_heads=8, head_dim=256,
                   global_head_dim=256, num_anchors=32, window_size=512, num_recall=96,
                   full_every=2, reference_graph=3)
    res = run_decode(engine, cfg, seed=5, steps=3, start_clock=5000, n_recall=96)
    for i, (tok, rtok, lg, rlg) in enumerate(res):
        assert_close(lg, rlg, what=f"logits step {i}")
        if tok != rtok:
            assert margin_top2(rlg) < 1e-3


def test_stream_graph_is_one_launch_and_rejects_small_k(engine):
    model = sx.Model(engine, sx.model_config(**mid_cfg(reference_graph=3)))
    assert model.kernels_per_token(True) == model.kernels_per_token(False) == 1
    with pytest.raises(sx.SxError):  # K = 256: fewer than 16 block pairs per row
        sx.Model(engine, sx.model_config(**tiny_cfg(reference_graph=3)))


def test_forward_token_rejects_oversized_slot_list(engine):
    cfg = tiny_cfg()
    model = sx.Model(engine, sx.model_config(**cfg))
    with pytest.raises(sx.SxError):
        model.forward_token(np.zeros(256, np.float32), 0, 0, np.zeros(100, np.uint32))


def test_record_api_layer_matches_checker(engine):
    """recordLayerDirect (model_dispatch.zig:10-43) written with the record API directly,
    bound like model_gpu.zig:140-156, against one checker layer."""
    cfg = tiny_cfg(num_layers=1, full_every=0)
    seed, clock = 4, 30
    H, I, D, nq, nkv = 256, 640, 64, 4, 2
    qd, kvd, total = nq * D, nkv * D, 16
    eps = cfg["rms_norm_eps"]
    E = engine

    def stream(kind):
        return 64 + kind

    def buf_f32(arr):
        b = E.buffer(arr.nbytes)
        b.write(arr.astype(np.float32))
        return b

    def wbuf(rows, cols, kind):
        b = E.buffer(sx.packed_bytes(rows, cols, sx.QUANT_Q4))
        b.upload_weights(orc.synth_q4(rows, cols, seed, stream(kind)), rows, cols, sx.QUANT_Q4)
        return b

    x0 = sx.synth_embed_row(H, 21, seed)
    x = buf_f32(x0)
    normed, q = E.buffer(4 * H), E.buffer(4 * qd)
    k, v, attn = E.buffer(4 * kvd), E.buffer(4 * kvd), E.buffer(4 * qd)
    act, mlp = E.buffer(4 * I), E.buffer(4 * H)
    kc, vc = E.buffer(2 * total * kvd), E.buffer(2 * total * kvd)
    in_norm = buf_f32(orc.synth_gain(H, seed, stream(0)))
    qn, kn = buf_f32(orc.synth_gain(D, seed, stream(5))), buf_f32(orc.synth_gain(D, seed, stream(6)))
    post_attn = buf_f32(orc.synth_gain(H, seed, stream(7)))
    pre_ffn = buf_f32(orc.synth_gain(H, seed, stream(8)))
    post_ffn = buf_f32(orc.synth_gain(H, seed, stream(12)))
    wq, wk, wv = wbuf(qd, H, 1), wbuf(kvd, H, 2), wbuf(kvd, H, 3)
    wo, wg, wu, wd = wbuf(H, qd, 4), wbuf(I, H, 9), wbuf(I, H, 10), wbuf(H, I, 11)
    z = orc.synth_normal(seed, stream(13), 0)
    scalar = orc.bf16_round(np.array([_libm.fmaf(0.05, z, 1.0)], np.float32))[0]

    ring = sx.Ring(1, 4, 8, 4)
    ring.prefill(0, clock)
    slot = ring.activate_slot(0, clock)
    slots = ring.get_active_slots(0, clock)
    slot_buf = E.buffer(4 * total)
    slot_buf.write(np.concatenate([slots, np.zeros(total - len(slots), np.uint32)]))
    step = E.buffer(16)
    step.write(np.array([clock, slot, len(slots), 0], np.uint32))

    S = E.set
    cmd = E.command_buffer()
    cmd.begin()
    E.record_rmsnorm(cmd, S(x, in_norm, normed), H, eps)
    E.record_barrier(cmd)
    E.record_gemv(cmd, S(wq, normed, q), qd, H)
    E.record_gemv(cmd, S(wk, normed, k), kvd, H)
    E.record_gemv(cmd, S(wv, normed, v), kvd, H)
    E.record_barrier(cmd)
    E.record_qkv_rope(cmd, S(q, k, v, qn, kn, q, kc, vc, step), nq, nkv, D, D, 0,
                      cfg["rope_theta"], eps, total)
    E.record_barrier(cmd)
    E.record_decode_attn(cmd, S(q, kc, vc, slot_buf, attn, step), D, kvd, nq // nkv, 1.0, nq,
                         total)
    E.record_barrier(cmd)
    E.record_gemv(cmd, S(wo, attn, mlp), H, qd)
    E.record_rmsnorm(cmd, S(mlp, post_attn, mlp), H, eps)
    E.record_add_rmsnorm(cmd, S(x, mlp, pre_ffn, normed), H, eps, 1.0)
    E.record_gate_up(cmd, S(wg, wu, normed, act), I, H)
    E.record_gemv(cmd, S(wd, act, mlp), H, I)
    E.record_rmsnorm(cmd, S(mlp, post_ffn, mlp), H, eps)
    E.record_add_rmsnorm(cmd, S(x, mlp, in_norm, normed), H, eps, float(scalar))
    E.record_barrier(cmd)
    cmd.end()
    E.submit_pre_recorded(cmd)
    got = x.read(np.float32, H)

    ref = orc.Model(cfg, seed)
    ref.ring.prefill(0, clock)
    _, _, rx = ref.forward(x0, clock, want_logits=False)
    assert_close(got, rx, what="residual after one layer")


def test_record_on_unbegun_command_buffer_fails_at_end(engine):
    cmd = engine.command_buffer()
    b = engine.buffer(64)
    engine.record_rmsnorm(cmd, engine.set(b, b, b), 16, 1e-6)  # not recording yet
    cmd.begin()
    engine.record_rmsnorm(cmd, engine.set(b, b), 16, 1e-6)  # too few buffers
    with pytest.raises(sx.SxError):
        cmd.end()


def test_submit_deadline_returns_timeout_not_hang(engine):
    """submitPreRecorded's bounded fence wait (kernels.zig:151-156): a deadline that cannot be
    met returns SX_ERR_TIMEOUT instead of blocking; the work still completes afterwards."""
    m, k = 262144, 3840
    E = engine
    w = E.buffer(sx.packed_bytes(m, k, sx.QUANT_Q8))
    x, y = E.buffer(4 * k), E.buffer(4 * m)
    cmd = E.command_buffer()
    cmd.begin()
    for _ in range(8):
        E.record_gemv_logits(cmd, E.set(w, x, y), m, k)
    cmd.end()
    with pytest.raises(sx.SxError) as ei:
        E.submit_pre_recorded(cmd, timeout_ns=1000)
    assert ei.value.status == sx.SX_ERR_TIMEOUT
    E.sync()
    E.submit_pre_recorded(cmd)  # default 5 s deadline is met


def test_attention_block_config5_shape_matches_checker(engine):
    """Graph 4's attention-block kernel (q|k|v, norm + RoPE + cache write, attention and the o
    projection in one launch) on config 5's layer shape: one kv head read by 8 q heads, so all
    148 CTAs form one group; head_dim 256; a 640-slot ring with a young window, then a wrapped
    one with a recall tier.  Against the checker with the bf16-cache allowance (a cached element
    rounded from f32 values one ulp apart differs by 2^-8)."""
    from tests.conftest import assert_close_bf16_operands
    cfg = tiny_cfg(vocab_size=8192, hidden_size=1536, intermediate_size=6144, num_layers=2,
                   num_q_heads=8, num_kv_heads=1, num_global_kv_heads=1, head_dim=256,
                   global_head_dim=256, num_anchors=32, window_size=512, num_recall=96,
                   full_every=2, reference_graph=4)
    for start, n_recall in ((3, 0), (4000, 40)):
        res = run_decode(engine, cfg, seed=41, steps=3, start_clock=start, n_recall=n_recall)
        for i, (tok, rtok, lg, rlg) in enumerate(res):
            assert_close_bf16_operands(lg, rlg, what=f"start {start} logits step {i}")
            if tok != rtok:
                assert margin_top2(rlg) < 1e-3, f"start {start} step {i}: {tok} vs {rtok}"


@pytest.mark.parametrize("kv_f32", [False, True])
def test_attention_block_equals_separate_launches(engine, engine_f32kv, kv_f32):
    """The attention block (graph 4) and its three separate launches (graph 0) compute the same
    token: the block sums the o projection per kv-head group, so the logits agree within the f32
    tolerance, not bit for bit; both also against the checker."""
    eng = engine_f32kv if kv_f32 else engine
    outs = []
    for g in (4, 0):
        cfg = mid_cfg(kv_bf16=0 if kv_f32 else 1, reference_graph=g)
        outs.append(run_decode(eng, cfg, seed=37, steps=4, start_clock=900, n_recall=4))
    from tests.conftest import assert_close_bf16_operands
    for i, ((t0, _, l0, _), (t4, _, l4, rl)) in enumerate(zip(*outs)):
        if kv_f32:
            assert_close(l0, l4, what=f"block vs separate logits step {i}")
            assert_close(l0, rl, what=f"block vs checker logits step {i}")
        else:  # cached K/V rounded to bf16 from slightly different f32 values
            assert_close_bf16_operands(l0, l4, what=f"block vs separate logits step {i}")
        if t0 != t4:
            assert margin_top2(rl) < 1e-3, f"step {i}: {t0} vs {t4}"
