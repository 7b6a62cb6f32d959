"""The recall tier on the device (sx_archive_*) on a B200: DiffArchive (src/memory.zig:19-151) and
integrateMemory (src/model/memory_inject.zig:17-46) over the model's own caches, against the CPU
checker's restatement on its caches and ring (pinned to memory.zig's own tests in
test_oracle_kat.py).  Each decode step: greedy token on both sides, then integrate -- the
selected archive indices must be identical (the scores agree to float rounding and the test
data keep their order well separated), the injected recall K/V must reproduce the checker's
next-step logits, and the archive's entries must match."""
import numpy as np
import pytest

import sx
from oracle import oracle as orc
from tests.conftest import assert_close, assert_close_bf16_operands
from tests.test_gpu_model import margin_top2, tiny_cfg

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def run(engine, cfg, seed, steps, start, capacity, bf16):
    model = sx.Model(engine, sx.model_config(**cfg))
    model.synth_weights(seed)
    model.fill_kv(seed)
    ref = orc.Model(cfg, seed)
    ref.fill_kv(seed)
    arch = sx.Archive(model, capacity)
    rarch = orc.Archive(ref, capacity)
    ring = sx.Ring(1, cfg["num_anchors"], cfg["window_size"], cfg["num_recall"])
    ring.prefill(0, start)
    ref.ring.prefill(0, start)
    token, recalled = 3, 0
    for i in range(steps):
        clock = start + i
        x = sx.synth_embed_row(cfg["hidden_size"], token, seed)
        slot = ring.activate_slot(0, clock)
        lists = ring.get_active_slots(0, clock)
        logits = np.zeros(cfg["vocab_size"], np.float32)
        tok = model.forward_token(x, clock, slot, lists, True, logits)
        rtok, rlg, _ = ref.forward(x, clock, True)
        assert np.array_equal(lists, ref.ring.get_active_slots(0, clock)), f"step {i} slot list"
        if bf16:
            assert_close_bf16_operands(logits, rlg, what=f"logits step {i}")
        else:
            assert_close(logits, rlg, what=f"logits step {i}")
        if tok != rtok:
            assert margin_top2(rlg) < 1e-3, f"step {i}: {tok} vs {rtok}"
        sel = arch.integrate(ring, clock)
        rsel = rarch.integrate(clock)
        assert list(sel) == list(rsel), f"step {i}: recalled {list(sel)} vs {list(rsel)}"
        assert arch.count == rarch.count
        recalled += len(sel)
        token = tok
    for e in range(arch.count):
        v, ts, la, ac, sal = arch.entry(e)
        rv, rts, rla, rac, rsal = rarch.entry(e)
        assert (ts, la, ac) == (rts, rla, rac), f"entry {e} metadata"
        assert abs(sal - rsal) <= 1e-5 * max(1.0, abs(rsal)), f"entry {e} salience"
        assert_close(v, rv, atol=1e-6, rtol=1e-5, what=f"entry {e} vector")
    assert recalled > 0
    arch.close()


def test_recall_tier_matches_checker_f32_cache(engine_f32kv):
    cfg = tiny_cfg(kv_bf16=0, num_recall=4)
    run(engine_f32kv, cfg, seed=13, steps=14, start=20, capacity=64, bf16=False)


def test_recall_tier_archive_wraps(engine_f32kv):
    # capacity 5 < the number of appended states: the write head wraps (memory.zig:103-110)
    cfg = tiny_cfg(kv_bf16=0, num_recall=4)
    run(engine_f32kv, cfg, seed=17, steps=9, start=5, capacity=5, bf16=False)


def test_recall_tier_12b_width_bf16_cache(engine):
    cfg = tiny_cfg(vocab_size=16384, hidden_size=3840, intermediate_size=15360, num_layers=2,
                   num_q_heads=16, num_kv_heads=8, num_global_kv_heads=8, head_dim=256,
                   global_head_dim=256, num_anchors=32, window_size=512, num_recall=96,
                   full_every=2)
    run(engine, cfg, seed=5, steps=4, start=700, capacity=128, bf16=True)


def test_archive_rejects_bad_capacity(engine):
    model = sx.Model(engine, sx.model_config(**tiny_cfg()))
    with pytest.raises(sx.SxError):
        sx.Archive(model, 0)
    with pytest.raises(sx.SxError):
        sx.Archive(model, 1 << 20)
