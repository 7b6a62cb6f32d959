"""The quiescence gate and indirect dispatch on a B200 (src/gpu/model_dispatch.zig:45-118,
shaders/quiescence_gate.wgsl:1-62, src/gpu/kernels.zig:84-138).

Layers l >= num_layers / 3 run behind a gate that compares the residual entering the layer with
its value at the previous token (mean square of the difference against the threshold, the
history updated every token) and writes the dispatch records of the layer's 13 commands: zeros
skip the layer.  Checked against the CPU checker's restatement of the shader, kernel by kernel
and as whole-token greedy decode with a positive threshold."""
import numpy as np
import pytest

import sx
from oracle import oracle as orc
from tests.conftest import assert_close
from tests.test_gpu_model import margin_top2, tiny_cfg

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def pc_for(h, thr, base=0, n=13):
    pc = sx.QuiescenceGatePC()
    pc.hidden_size, pc.threshold_sq, pc.base_cmd_idx, pc.num_cmds = h, thr, base, n
    for i in range(16):
        pc.targets[i] = 100 + i
    return pc


@pytest.mark.parametrize("h", [3840, 1536, 100])
def test_gate_kernel_matches_checker(engine, h):
    rng = np.random.default_rng(h)
    x = rng.standard_normal(h).astype(np.float32)
    prev = (x + 0.05 * rng.standard_normal(h)).astype(np.float32)
    ref_prev = prev.copy()
    _, ms = orc.quiescence_gate(x, ref_prev, 0.0)
    for thr, runs in ((0.0, True), (-1.0, True), (ms * 0.5, True), (ms * 2.0, False)):
        xp = torch.from_numpy(prev.copy()).cuda()
        ind = torch.full((16 * 3 * 2,), 7, dtype=torch.int32, device="cuda")
        engine.quiescence_gate(torch.from_numpy(x).cuda(), xp, ind, pc_for(h, thr, base=16))
        got = host(ind).view(np.uint32).reshape(-1, 3)
        assert np.array_equal(host(xp).view(np.uint32), x.view(np.uint32)), "x_prev = x_curr"
        want_run, _ = orc.quiescence_gate(x, prev.copy(), thr)
        assert want_run == runs
        for c in range(13):
            want = [100 + c, 1, 1] if runs else [0, 0, 0]
            assert list(got[16 + c]) == want, (thr, c)
        assert np.all(got[:16] == 7) and np.all(got[16 + 13:] == 7), "records outside untouched"


def test_indirect_records_skip_or_run(engine):
    """A GEMV and an RMSNorm recorded behind a dispatch record: zeros skip them (outputs
    untouched), a non-zero record runs them in full."""
    m, k = 64, 256
    w = orc.synth_q4(m, k, 3, 4)
    wb = engine.buffer(sx.packed_bytes(m, k, sx.QUANT_Q4))
    wb.upload_weights(w, m, k, sx.QUANT_Q4)
    xb, yb = engine.buffer(4 * k), engine.buffer(4 * m)
    nb, gb, ob = engine.buffer(4 * k), engine.buffer(4 * k), engine.buffer(4 * k)
    ind = engine.buffer(24)
    x = np.random.default_rng(1).standard_normal(k).astype(np.float32)
    g = orc.synth_gain(k, 3, 5)
    xb.write(x)
    nb.write(x)
    gb.write(g)
    cmd = engine.command_buffer()
    cmd.begin()
    engine.record_gemv_indirect(cmd, engine.set(wb, xb, yb), m, k, ind, 0)
    engine.record_rmsnorm_indirect(cmd, engine.set(nb, gb, ob), k, 1e-6, ind, 12)
    cmd.end()
    for rec, runs in (([0, 1, 1], False), ([5, 1, 1], True), ([5, 0, 1], False)):
        yb.write(np.full(m, 9.0, np.float32))
        ob.write(np.full(k, 9.0, np.float32))
        ind.write(np.array(rec + rec, np.uint32))
        engine.submit_pre_recorded(cmd)
        y, o = yb.read(np.float32, m), ob.read(np.float32, k)
        if runs:
            assert_close(y, orc.gemv_q4(w, x, m, k), what="gemv behind an open record")
            assert_close(o, orc.rmsnorm(x, g), atol=1e-5, rtol=1e-4, what="rmsnorm")
        else:
            assert np.all(y == 9.0) and np.all(o == 9.0), f"{rec} must skip"


def checker_run(cfg, seed, thr, steps, start):
    ref = orc.Model(dict(cfg, quiescence_threshold=thr), seed)
    ref.fill_kv(seed)
    ref.ring.prefill(0, start)
    token, stats = 5, []
    for i in range(steps):
        x = orc.synth_embed_row(cfg["hidden_size"], token, seed)
        token, _, _ = ref.forward(x, start + i, True)
        stats.append(ref.gate_stats())
    return stats


def test_gated_decode_matches_checker(engine):
    """Greedy decode through the op-by-op graph with a positive threshold: layers 2..5 of 6 are
    gated, some run and some are skipped; the threshold is picked (on the checker) at least 3%
    away from every gate statistic the decode produces (the GPU evaluates the statistic in the
    shader's order of operations on a residual that agrees to ~1e-6), so both sides take the
    same decisions; among such thresholds the one with the widest margin that still skips
    layers after the first token (whose history is zero) is used."""
    cfg = tiny_cfg(num_layers=6, reference_graph=1)
    seed, steps, start = 19, 8, 30
    base = checker_run(cfg, seed, 0.0, steps, start)
    vals = np.concatenate([ms[2:] for ms, _ in base[1:]])
    thr, best = None, 0.0
    for c in np.linspace(vals.min(), vals.max(), 25):
        st = checker_run(cfg, seed, float(c), steps, start)
        ms = np.concatenate([m[2:] for m, _ in st])
        act = np.concatenate([a[2:] for _, a in st[1:]])
        margin = float(np.min(np.abs(ms - c) / c))
        if margin > max(best, 0.01) and act.min() == 0 and act.max() == 1:
            thr, best = float(c), margin
    assert thr is not None, "no threshold with a clear margin"
    gcfg = dict(cfg, quiescence_threshold=thr)
    model = sx.Model(engine, sx.model_config(**gcfg))
    model.synth_weights(seed)
    model.fill_kv(seed)
    ref = orc.Model(gcfg, seed)
    ref.fill_kv(seed)
    ring = sx.Ring(1, cfg["num_anchors"], cfg["window_size"], cfg["num_recall"])
    ring.prefill(0, start)
    ref.ring.prefill(0, start)
    token, skipped = 5, 0
    for i in range(steps):
        clock = start + i
        x = sx.synth_embed_row(cfg["hidden_size"], token, seed)
        slot = ring.activate_slot(0, clock)
        logits = np.zeros(cfg["vocab_size"], np.float32)
        tok = model.forward_token(x, clock, slot, ring.get_active_slots(0, clock), True, logits)
        rtok, rlg, _ = ref.forward(x, clock, True)
        skipped += int((ref.gate_stats()[1] == 0).sum())
        assert_close(logits, rlg, what=f"gated logits step {i}")
        if tok != rtok:
            assert margin_top2(rlg) < 1e-3, f"step {i}: {tok} vs {rtok}"
        token = tok
    assert skipped > 0


def test_positive_threshold_needs_the_op_by_op_graph(engine):
    with pytest.raises(sx.SxError):
        sx.Model(engine, sx.model_config(**tiny_cfg(reference_graph=0, quiescence_threshold=0.5)))
