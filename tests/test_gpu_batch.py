"""Batch decode of independent sessions (sx_decode_batch) on a B200.

Each session has its own KV cache (synthetic past with its own seed), ring and clock; one
sx_decode_batch step equals one sx_forward_token step of each session on its own
(src/model/forward.zig:19-75 per session, src/ring_buffer.zig slot rules per ring).

Two claims, tested separately: (1) batching is exact -- every row of a batched step is bit
for bit the step of a one-session model holding that session (bf16 cache); (2) the path
matches the CPU checker (one single-session checker model per session) within the f32
tolerance.  (2) runs with the f32 KV cache: with a bf16 cache a 1-ulp f32 difference before
rounding can flip a cached element by 2^-8, which attention at scale 1.0 amplifies into
logit differences of ~1e-2 at logits of ~100 -- a property of rounding twice, not of the
batch path (the one-session path shows the same step)."""
import numpy as np
import pytest

import sx
from oracle import oracle as orc
from tests.conftest import assert_close
from tests.test_gpu_model import margin_top2, tiny_cfg

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def make_sessions(engine, cfg, seed, starts, n_recall=0):
    model = sx.Model(engine, sx.model_config(**cfg))
    model.synth_weights(seed)
    refs, rings = [], []
    rng = np.random.default_rng(seed)
    for s, start in enumerate(starts):
        model.fill_kv_session(s, seed + 101 * s)
        ref = orc.Model(cfg, seed)
        ref.fill_kv(seed + 101 * s)
        ring = sx.Ring(1, cfg["num_anchors"], cfg["window_size"], cfg["num_recall"])
        ring.prefill(0, start)
        ref.ring.prefill(0, start)
        for r in range(n_recall):
            c = int(rng.integers(0, max(start, 1)))
            ring.write_recall(0, r, c)
            ref.ring.write_recall(0, r, c)
        refs.append(ref)
        rings.append(ring)
    return model, refs, rings


def step_all(model, refs, rings, cfg, seed, clocks, tokens, n):
    xs = np.stack([sx.synth_embed_row(cfg["hidden_size"], int(tokens[i]), seed) for i in range(n)])
    slots = [rings[i].activate_slot(0, clocks[i]) for i in range(n)]
    lists = [rings[i].get_active_slots(0, clocks[i]) for i in range(n)]
    logits = np.zeros((n, cfg["vocab_size"]), np.float32)
    toks = model.decode_batch(xs, clocks[:n], slots, lists, True, logits)
    out = []
    for i in range(n):
        rtok, rlg, _ = refs[i].forward(xs[i], clocks[i], True)
        assert np.array_equal(lists[i], refs[i].ring.get_active_slots(0, clocks[i]))
        out.append((int(toks[i]), rtok, logits[i], rlg))
    return out


@pytest.mark.parametrize("n", [2, 5, 8])
def test_batch_decode_matches_checker_per_session(engine_f32kv, n):
    engine = engine_f32kv
    cfg = tiny_cfg(num_sessions=8, kv_bf16=0)
    starts = [3 + 7 * s for s in range(n)]  # different clocks; some windows wrap
    model, refs, rings = make_sessions(engine, cfg, seed=21, starts=starts, n_recall=0)
    clocks = list(starts)
    tokens = [11 + s for s in range(n)]
    for t in range(12):
        res = step_all(model, refs, rings, cfg, 21, clocks, tokens, n)
        for i, (tok, rtok, lg, rlg) in enumerate(res):
            assert_close(lg, rlg, what=f"session {i} step {t} logits")
            if tok != rtok:
                assert margin_top2(rlg) < 1e-3, f"session {i} step {t}: {tok} vs {rtok}"
            tokens[i] = tok
        clocks = [c + 1 for c in clocks]


def test_batch_with_recall_and_large_clocks(engine_f32kv):
    engine = engine_f32kv
    cfg = tiny_cfg(num_sessions=4, kv_bf16=0)
    starts = [90000, 5, 12345, 700]
    model, refs, rings = make_sessions(engine, cfg, seed=4, starts=starts, n_recall=3)
    clocks, tokens = list(starts), [1, 2, 3, 4]
    for t in range(4):
        for i, (tok, rtok, lg, rlg) in enumerate(step_all(model, refs, rings, cfg, 4, clocks,
                                                          tokens, 4)):
            assert_close(lg, rlg, what=f"session {i} step {t} logits")
            if tok != rtok:
                assert margin_top2(rlg) < 1e-3
            tokens[i] = tok
        clocks = [c + 1 for c in clocks]


@pytest.mark.parametrize("n", [2, 8])
def test_batched_rows_equal_one_session_models(engine, n):
    """A session's row of an n-session step is bit-identical to the same session stepped alone
    (n = 1) through the batched graph of a model of its own.  (The one-session graph of a
    num_sessions <= 1 model folds the o projection into the attention per kv head and agrees
    with these rows within the f32 tolerance, not bit for bit.)"""
    cfg = tiny_cfg(num_layers=2, num_sessions=8)
    cfg1 = tiny_cfg(num_layers=2, num_sessions=8)
    seed = 17
    model = sx.Model(engine, sx.model_config(**cfg))
    model.synth_weights(seed)
    singles = []
    for s in range(n):
        model.fill_kv_session(s, seed + 7 * s)
        m1 = sx.Model(engine, sx.model_config(**cfg1))
        m1.synth_weights(seed)
        m1.fill_kv_session(0, seed + 7 * s)
        singles.append(m1)
    mk = lambda: sx.Ring(1, cfg["num_anchors"], cfg["window_size"], cfg["num_recall"])
    rings, rings1 = [mk() for _ in range(n)], [mk() for _ in range(n)]
    clocks = [5 + 3 * s for s in range(n)]
    for r, r1, c in zip(rings, rings1, clocks):
        r.prefill(0, c)
        r1.prefill(0, c)
    tokens = [100 + s for s in range(n)]
    V = cfg["vocab_size"]
    for t in range(6):
        xs = np.stack([sx.synth_embed_row(cfg["hidden_size"], tokens[s], seed) for s in range(n)])
        slots = [rings[s].activate_slot(0, clocks[s]) for s in range(n)]
        lists = [rings[s].get_active_slots(0, clocks[s]) for s in range(n)]
        lg = np.zeros((n, V), np.float32)
        got = model.decode_batch(xs, clocks, slots, lists, True, lg)
        for s in range(n):
            l1 = np.zeros((1, V), np.float32)
            t1 = singles[s].decode_batch(xs[s:s + 1], [clocks[s]],
                                         [rings1[s].activate_slot(0, clocks[s])],
                                         [rings1[s].get_active_slots(0, clocks[s])], True, l1)
            assert int(got[s]) == int(t1[0]), f"session {s} step {t}"
            assert np.array_equal(lg[s].view(np.uint32), l1[0].view(np.uint32)), f"session {s} step {t}"
        tokens = [int(g) for g in got]
        clocks = [c + 1 for c in clocks]


def test_sessions_outside_the_step_are_untouched(engine):
    cfg = tiny_cfg(num_sessions=4, num_layers=2)
    model = sx.Model(engine, sx.model_config(**cfg))
    model.synth_weights(8)
    for s in range(4):
        model.fill_kv_session(s, 50 + s)
    ts = cfg["num_anchors"] + cfg["window_size"] + cfg["num_recall"]
    kv_dim = cfg["num_kv_heads"] * cfg["head_dim"]
    nbytes = ts * kv_dim * 2  # bf16 cache of one session, layer 0
    view = engine.wrap(model.kcache_ptr(0), 4 * nbytes)
    b = view.read(np.uint8, 4 * nbytes).reshape(4, nbytes)
    ring = sx.Ring(1, cfg["num_anchors"], cfg["window_size"], cfg["num_recall"])
    ring.prefill(0, 9)
    clocks = [9, 9]
    slots = [ring.activate_slot(0, 9)] * 2
    lists = [ring.get_active_slots(0, 9)] * 2
    xs = np.stack([sx.synth_embed_row(cfg["hidden_size"], 3, 8)] * 2)
    model.decode_batch(xs, clocks, slots, lists, True)
    a = view.read(np.uint8, 4 * nbytes).reshape(4, nbytes)
    assert not np.array_equal(a[0], b[0]) and not np.array_equal(a[1], b[1])  # slot 9 written
    assert np.array_equal(a[2], b[2]) and np.array_equal(a[3], b[3])


def test_batched_row_equals_single_session_model(engine):
    # session 0 of a two-session step against a one-session model's sx_forward_token
    cfg1 = tiny_cfg(num_layers=2)
    cfg2 = tiny_cfg(num_layers=2, num_sessions=2)
    m1 = sx.Model(engine, sx.model_config(**cfg1))
    m2 = sx.Model(engine, sx.model_config(**cfg2))
    for m in (m1, m2):
        m.synth_weights(6)
        m.fill_kv_session(0, 6)
    m2.fill_kv_session(1, 7)
    rings = [sx.Ring(1, cfg1["num_anchors"], cfg1["window_size"], cfg1["num_recall"])
             for _ in range(2)]
    for r, c in zip(rings, (20, 33)):
        r.prefill(0, c)
    slots = [rings[0].activate_slot(0, 20), rings[1].activate_slot(0, 33)]
    lists = [rings[0].get_active_slots(0, 20), rings[1].get_active_slots(0, 33)]
    xs = np.stack([sx.synth_embed_row(cfg1["hidden_size"], t, 6) for t in (9, 10)])
    l1 = np.zeros(cfg1["vocab_size"], np.float32)
    l2 = np.zeros((2, cfg1["vocab_size"]), np.float32)
    t1 = m1.forward_token(xs[0], 20, slots[0], lists[0], True, l1)
    t2 = m2.decode_batch(xs, [20, 33], slots, lists, True, l2)
    assert_close(l2[0], l1, what="batched row 0 vs one-session logits")
    if t1 != int(t2[0]):
        assert margin_top2(l1) < 1e-3


def test_batch_rejects_bad_requests(engine):
    cfg = tiny_cfg(num_sessions=2, num_layers=1)
    m = sx.Model(engine, sx.model_config(**cfg))
    x = np.zeros((3, cfg["hidden_size"]), np.float32)
    with pytest.raises(sx.SxError):
        m.decode_batch(x, [0, 0, 0], [0, 0, 0], [[0]] * 3)  # 3 sessions of 2
    with pytest.raises(sx.SxError):
        sx.Model(engine, sx.model_config(**tiny_cfg(num_sessions=9)))
    with pytest.raises(sx.SxError):
        sx.Model(engine, sx.model_config(**tiny_cfg(num_sessions=2, reference_graph=1)))


def c5_cfg(**kw):
    """BASELINE config 5's model shape: H 1536, 8 q / 1 kv heads x 256, I 6144, Q4_0 layers,
    Q8_0 LM head over the full 262144 vocabulary, 32 + 512 + 96 ring, bf16 KV cache (what
    bench.py --case sessions runs), with fewer layers so that the checker finishes in seconds
    (layer 4 is a full-attention layer: rot 64, theta 1e6)."""
    cfg = tiny_cfg(vocab_size=262144, hidden_size=1536, intermediate_size=6144, num_layers=5,
                   num_q_heads=8, num_kv_heads=1, num_global_kv_heads=1, head_dim=256,
                   global_head_dim=256, num_anchors=32, window_size=512, num_recall=96,
                   full_every=5, kv_bf16=1, num_sessions=8)
    cfg.update(kw)
    return cfg


def test_config5_shape_batch8_bf16_kv_matches_checker(engine):
    """sx_decode_batch at n = 8 on config 5's shape with the bf16 cache against one checker
    model per session in its bf16-cache mode (forward.zig:19-75 per session).  Logits use the
    double-rounding allowance of conftest.assert_close_bf16_operands: a cached element rounded
    from f32 values one ulp apart on the two sides differs by 2^-8."""
    from tests.conftest import assert_close_bf16_operands
    cfg = c5_cfg()
    starts = [700, 31, 5000, 12, 99999, 544, 2, 1234]  # wrapped windows, young rings
    model, refs, rings = make_sessions(engine, cfg, seed=55, starts=starts, n_recall=0)
    rng = np.random.default_rng(56)
    for i, s in enumerate(starts):  # recall tiers of different fill
        for r in range(int(rng.integers(0, 97)) if s > 600 else 0):
            c = int(rng.integers(0, s))
            rings[i].write_recall(0, r, c)
            refs[i].ring.write_recall(0, r, c)
    clocks, tokens = list(starts), [7 + 3 * s for s in range(8)]
    for t in range(3):
        for i, (tok, rtok, lg, rlg) in enumerate(step_all(model, refs, rings, cfg, 55, clocks,
                                                          tokens, 8)):
            assert_close_bf16_operands(lg, rlg, what=f"session {i} step {t} logits")
            if tok != rtok:
                assert margin_top2(rlg) < 1e-3, f"session {i} step {t}: {tok} vs {rtok}"
            tokens[i] = tok
        clocks = [c + 1 for c in clocks]
