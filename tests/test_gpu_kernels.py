"""Kernel parity on a B200: each CUDA kernel of libsx against the CPU checker, through the
C ABI, on seeded inputs.  Bit-exact for dequantised weights, slot handling and argmax ids;
|a - b| <= 1e-3 + 1e-2 |b| for activations and logits."""
import zlib

import numpy as np
import pytest

import sx
from oracle import oracle as orc
from tests.conftest import assert_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def upload(engine, ref_words, rows, cols, mode):
    buf = engine.buffer(sx.packed_bytes(rows, cols, mode))
    buf.upload_weights(ref_words, rows, cols, mode)
    return buf


def bf16_normal(n, seed):
    return orc.bf16_round(np.random.default_rng(seed).standard_normal(n).astype(np.float32))


# ---------------------------------------------------------------------------------------
@pytest.mark.parametrize("rows,cols", [(64, 128), (17, 96), (6144, 1536), (3840, 15360)])
def test_q4_packed_layout_dequantises_bit_exact(engine, rows, cols):
    w = orc.synth_q4(rows, cols, 5, 77)
    buf = upload(engine, w, rows, cols, sx.QUANT_Q4)
    out = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
    engine.unpack_q4(buf.ptr, out, rows, cols)
    got = host(out).reshape(rows, cols)
    want = orc.dequant_q4(w, rows, cols)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("mode", [sx.QUANT_Q4, sx.QUANT_Q8])
def test_device_synth_matches_checker_bits(engine, mode):
    rows, cols = 200, 3840
    words_per_row = sx.quantized_row_words(cols, mode)
    out = torch.zeros(rows * words_per_row, dtype=torch.int32, device="cuda")
    engine.synth_weights(mode, out, 100, rows - 100, cols, 3, 9)
    got = host(out).view(np.uint32)[: (rows - 100) * words_per_row]
    ref = (orc.synth_q4 if mode == sx.QUANT_Q4 else orc.synth_q8)(rows, cols, 3, 9)
    assert np.array_equal(got, ref[100 * words_per_row:])


# ---------------------------------------------------------------------------------------
GEMV_Q4_CASES = [
    (6144, 1536, 1),
    (3840, 15360, 1),  # test_q4_exec.zig:16-17 shape
    (100, 96, 1),      # ragged rows, odd number of blocks
    (33, 64, 3),
    (6144, 1536, 2),
    (1536, 6144, 4),
    (6144, 1536, 8),   # BASELINE config 2 batch 8
    (1536, 6144, 8),
    (16, 15360, 1),    # one tile split across hundreds of stream-K workers
    (1, 4096, 1),      # a single row
    (262144, 64, 1),   # many tiles, one pair each
    (48, 1536, 5),
]


@pytest.mark.parametrize("m,k,batch", GEMV_Q4_CASES)
def test_gemv_q4_matches_checker(engine, m, k, batch):
    w = orc.synth_q4(m, k, 11, m + k)
    buf = upload(engine, w, m, k, sx.QUANT_Q4)
    x = bf16_normal(batch * k, m * 7 + batch).reshape(batch, k)
    y = torch.empty(batch, m, dtype=torch.float32, device="cuda")
    engine.gemv(sx.QUANT_Q4, buf.ptr, dev(x), y, m, k, batch)
    got = host(y)
    for b in range(batch):
        assert_close(got[b], orc.gemv_q4(w, x[b], m, k), what=f"gemv_q4 row {b}")


def test_gemv_q4_reference_test_inputs(engine):
    # test_q4_exec.zig:16-101: bf16-truncated U(-0.1, 0.1) weights quantised with
    # quantizeMatrix, x = U(-0.25, 0.25) f32, max-abs error < 1e-3
    m, k = 3840, 15360
    rng = np.random.default_rng(42)
    wf = ((rng.random(m * k, dtype=np.float32) - 0.5) * 0.2).astype(np.float32)
    w = orc.quantize_matrix((wf.view(np.uint32) >> 16).astype(np.uint16), m, k, orc.QUANT_Q4)
    x = ((rng.random(k, dtype=np.float32) - 0.5) * 0.5).astype(np.float32)
    buf = upload(engine, w, m, k, sx.QUANT_Q4)
    y = torch.empty(m, dtype=torch.float32, device="cuda")
    engine.gemv(sx.QUANT_Q4, buf.ptr, dev(x), y, m, k, 1)
    assert np.max(np.abs(host(y) - orc.gemv_q4(w, x, m, k))) < 1e-3


def test_gemv_q4_all_ones_positive(engine):
    # gpu.zig:30-59
    m, k = 64, 128
    w = orc.quantize_matrix(np.full(m * k, 0x3F80, np.uint16), m, k, orc.QUANT_Q4)
    x = (np.arange(k) % 5).astype(np.float32) * 0.25
    buf = upload(engine, w, m, k, sx.QUANT_Q4)
    y = torch.empty(m, dtype=torch.float32, device="cuda")
    engine.gemv(sx.QUANT_Q4, buf.ptr, dev(x), y, m, k, 1)
    got = host(y)
    assert np.all(got > 0)
    assert_close(got, orc.gemv_q4(w, x, m, k))


@pytest.mark.parametrize("m,k,batch", [(4096, 3840, 1), (262144, 3840, 1), (77, 160, 5),
                                       (2048, 1536, 8)])
def test_gemv_q8_matches_checker(engine, m, k, batch):
    w = orc.synth_q8(m, k, 13, m + 3)
    buf = upload(engine, w, m, k, sx.QUANT_Q8)
    x = np.random.default_rng(m).standard_normal((batch, k)).astype(np.float32)
    y = torch.empty(batch, m, dtype=torch.float32, device="cuda")
    engine.gemv(sx.QUANT_Q8, buf.ptr, dev(x), y, m, k, batch)
    got = host(y)
    for b in range(batch):
        assert_close(got[b], orc.gemv_q8(w, x[b], m, k), what=f"gemv_q8 row {b}")


def test_gemv_q8_wide_dynamic_range(engine):
    # activations far outside fp16 range still work: the kernel prescales by a power of two
    m, k = 256, 1024
    w = orc.synth_q8(m, k, 1, 2)
    buf = upload(engine, w, m, k, sx.QUANT_Q8)
    for scale in (1e-6, 1.0, 3e5):
        x = (np.random.default_rng(5).standard_normal(k) * scale).astype(np.float32)
        y = torch.empty(m, dtype=torch.float32, device="cuda")
        engine.gemv(sx.QUANT_Q8, buf.ptr, dev(x), y, m, k, 1)
        ref = orc.gemv_q8(w, x, m, k)
        assert_close(host(y), ref, atol=1e-3 * scale, what=f"scale {scale}")


@pytest.mark.parametrize("h,i,batch", [(1536, 6144, 1), (1536, 6144, 8), (3840, 15360, 1),
                                       (96, 160, 3)])
def test_gate_up_geglu_matches_checker(engine, h, i, batch):
    # x = RMSNorm(N(0,1)) with gain 1 + N(0, 0.1)
    wg = orc.synth_q4(i, h, 21, 1)
    wu = orc.synth_q4(i, h, 21, 2)
    bg = upload(engine, wg, i, h, sx.QUANT_Q4)
    bu = upload(engine, wu, i, h, sx.QUANT_Q4)
    gain = orc.synth_gain(h, 21, 3)
    xs = np.stack([orc.rmsnorm(bf16_normal(h, 30 + b), gain) for b in range(batch)])
    y = torch.empty(batch, i, dtype=torch.float32, device="cuda")
    engine.gate_up(bg.ptr, bu.ptr, dev(xs), y, i, h, batch)
    got = host(y)
    for b in range(batch):
        assert_close(got[b], orc.gate_up_geglu_q4(wg, wu, xs[b], i, h), what=f"geglu row {b}")


def test_gemv_rejects_bad_shapes(engine):
    y = torch.empty(16, dtype=torch.float32, device="cuda")
    x = torch.empty(48, dtype=torch.float32, device="cuda")
    with pytest.raises(sx.SxError):
        engine.gemv(sx.QUANT_Q4, x.data_ptr(), x, y, 16, 48, 1)  # k % 32 != 0
    with pytest.raises(sx.SxError):
        engine.gemv(sx.QUANT_Q4, x.data_ptr(), x, y, 16, 32, 9)  # batch > 8


# ---------------------------------------------------------------------------------------
def test_rmsnorm_reference_test(engine):
    # test_gpu_suite.zig:56-102: D=2048, x = U(-1,1), w = bf16(1 + U(-0.05, 0.05)), < 1e-4
    d, eps = 2048, 1e-6
    rng = np.random.default_rng(202)
    x = ((rng.random(d, dtype=np.float32) - 0.5) * 2.0).astype(np.float32)
    wb = ((1.0 + (rng.random(d, dtype=np.float32) - 0.5) * 0.1).astype(np.float32).view(np.uint32) >> 16)
    w = (wb << 16).astype(np.uint32).view(np.float32)
    y = torch.empty(d, dtype=torch.float32, device="cuda")
    engine.rmsnorm(dev(x), dev(w), y, d, 1, eps)
    assert np.max(np.abs(host(y) - orc.rmsnorm(x, w, eps))) < 1e-4


@pytest.mark.parametrize("n,batch,scalar", [(3840, 1, 1.0), (1536, 8, 0.97), (100, 3, 1.3)])
def test_add_rmsnorm_matches_checker(engine, n, batch, scalar):
    rng = np.random.default_rng(n)
    x = rng.standard_normal((batch, n)).astype(np.float32) * 3
    r = rng.standard_normal((batch, n)).astype(np.float32)
    w = orc.synth_gain(n, 1, 2)
    xd, yd = dev(x), torch.empty(batch, n, dtype=torch.float32, device="cuda")
    engine.add_rmsnorm(xd, dev(r), dev(w), yd, n, batch, 1e-6, scalar)
    gx, gy = host(xd), host(yd)
    for b in range(batch):
        rx, ry = orc.add_rmsnorm(x[b], r[b], w, 1e-6, scalar)
        assert np.max(np.abs(gx[b] - rx)) <= 1e-6 * np.max(np.abs(rx))
        assert_close(gy[b], ry, atol=1e-5, rtol=1e-4)


# ---------------------------------------------------------------------------------------
def cache_to_np(t, kv_bf16):
    a = host(t)
    if kv_bf16:
        return (a.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
    return a.view(np.float32)


@pytest.mark.parametrize("kv_f32", [False, True])
@pytest.mark.parametrize("num_q,num_kv,d,rot,theta,k_eq_v,clock", [
    (8, 1, 256, 64, 1e6, 0, 99999),   # BASELINE config 3 (full-attention style)
    (16, 8, 256, 256, 1e4, 0, 4321),  # 12B sliding layer
    (16, 8, 256, 64, 1e6, 1, 77),     # k_eq_v
    (4, 2, 64, 16, 1e4, 0, 0),
])
def test_qkv_rope_matches_checker(engine, engine_f32kv, kv_f32, num_q, num_kv, d, rot, theta,
                                  k_eq_v, clock):
    eng = engine_f32kv if kv_f32 else engine
    total, slot, eps = 40, 37, 1e-6
    rng = np.random.default_rng(clock + d)
    q = rng.standard_normal(num_q * d).astype(np.float32)
    k = rng.standard_normal(num_kv * d).astype(np.float32)
    v = rng.standard_normal(num_kv * d).astype(np.float32)
    qn, kn = orc.synth_gain(d, 4, 1), orc.synth_gain(d, 4, 2)
    dtype = torch.float32 if kv_f32 else torch.int16
    kc = torch.zeros(total * num_kv * d, dtype=dtype, device="cuda")
    vc = torch.zeros_like(kc)
    qd = dev(q)
    step = dev(np.array([clock, slot, 0, 0], np.uint32).view(np.int32))
    eng.qkv_rope(qd, dev(k), dev(v), dev(qn), dev(kn), qd, kc, vc, step, num_q, num_kv, d, rot,
                 k_eq_v, theta, eps, total)
    rkc = np.zeros(total * num_kv * d, np.float32)
    rvc = np.zeros_like(rkc)
    rq = orc.qkv_rope(q, k, v, qn, kn, rkc, rvc, not kv_f32, num_q, num_kv, d, rot, k_eq_v,
                      theta, eps, clock, slot, total)
    assert_close(host(qd), rq, atol=1e-5, rtol=1e-4, what="q")
    gk, gv = cache_to_np(kc, not kv_f32), cache_to_np(vc, not kv_f32)
    sl = slice(slot * num_kv * d, (slot + 1) * num_kv * d)
    tol = 2 ** -7 if not kv_f32 else 1e-4  # one bf16 ulp at worst across a rounding edge
    assert np.max(np.abs(gk[sl] - rkc[sl])) <= tol * max(1.0, np.max(np.abs(rkc[sl])))
    assert np.max(np.abs(gv[sl] - rvc[sl])) <= tol * max(1.0, np.max(np.abs(rvc[sl])))
    assert not np.any(gk[: slot * num_kv * d]) and not np.any(gv[: slot * num_kv * d])


def test_qkv_rope_bad_slot_reports_device_error(engine):
    num_q, num_kv, d, total = 2, 1, 64, 8
    z = torch.zeros(num_q * d, dtype=torch.float32, device="cuda")
    kc = torch.zeros(total * num_kv * d, dtype=torch.int16, device="cuda")
    step = dev(np.array([5, total + 3, 0, 0], np.int32))  # slot beyond the ring
    engine.qkv_rope(z, z, z, z, z, z, kc, kc, step, num_q, num_kv, d, d, 0, 1e4, 1e-6, total)
    with pytest.raises(sx.SxError) as ei:
        engine.sync()
    assert ei.value.status == sx.SX_ERR_DEVICE
    engine.sync()  # the error word is cleared and the context stays usable


# ---------------------------------------------------------------------------------------
def ring_case(anchors, window, recall, clock, n_recall, seed):
    ring = orc.Ring(1, anchors, window, recall)
    ring.prefill(0, clock)
    rng = np.random.default_rng(seed)
    for r in range(n_recall):
        ring.write_recall(0, r, int(rng.integers(0, clock)))
    slot = ring.activate_slot(0, clock)
    return ring.get_active_slots(0, clock), slot


@pytest.mark.parametrize("kv_f32", [False, True])
@pytest.mark.parametrize("num_q,num_kv,d,scale,clock,n_recall", [
    (8, 1, 256, 1 / 16, 99999, 96),   # BASELINE config 3, all recall live
    (8, 1, 256, 1 / 16, 5000, 0),     # no recall live
    (8, 1, 256, 1 / 16, 20, 0),       # young ring: 21 live slots (ragged)
    (16, 8, 256, 1.0, 7000, 40),      # 12B layer, reference scale 1.0
    (4, 4, 128, 0.3, 600, 3),
    (2, 1, 64, 1.0, 0, 0),            # single live slot
    (16, 2, 512, 0.05, 1000, 10),
])
def test_decode_attn_matches_checker(engine, engine_f32kv, kv_f32, num_q, num_kv, d, scale,
                                     clock, n_recall):
    eng = engine_f32kv if kv_f32 else engine
    anchors, window, recall = 32, 512, 96
    total = anchors + window + recall
    slots, _ = ring_case(anchors, window, recall, clock, n_recall, clock + 1)
    rng = np.random.default_rng(d + clock)
    kv_dim = num_kv * d
    k = orc.bf16_round(rng.standard_normal(total * kv_dim).astype(np.float32))
    v = orc.bf16_round(rng.standard_normal(total * kv_dim).astype(np.float32))
    q = rng.standard_normal(num_q * d).astype(np.float32)
    if kv_f32:
        kd, vd = dev(k), dev(v)
    else:
        kd = dev((k.view(np.uint32) >> 16).astype(np.uint16).view(np.int16))
        vd = dev((v.view(np.uint32) >> 16).astype(np.uint16).view(np.int16))
    out = torch.empty(num_q * d, dtype=torch.float32, device="cuda")
    step = dev(np.array([clock, 0, len(slots), 0], np.int32))
    sl = dev(np.concatenate([slots, np.zeros(total - len(slots), np.uint32)]).view(np.int32))
    eng.decode_attn(dev(q), kd, vd, sl, step, out, d, kv_dim, num_q // num_kv, scale, num_q, total)
    ref = orc.decode_attn(q, k, v, slots, num_q, num_kv, d, total, scale)
    assert_close(host(out), ref, atol=1e-4, rtol=1e-3, what="attn")


def c3_instance(rng, num_q, num_kv, d, clock, n_recall, seed, total=640):
    """One BASELINE config-3 problem: a 32 + 512 + 96 ring at `clock` (window written by
    getSlotIndex, n_recall live recall slots), K = bf16 N(0,1) and V unit-RMS per slot in the
    cache, raw q/k/v projections N(0,1)."""
    slots, slot = ring_case(32, 512, 96, clock, n_recall, seed)
    kv_dim = num_kv * d
    k = orc.bf16_round(rng.standard_normal(total * kv_dim).astype(np.float32))
    v = rng.standard_normal((total * num_kv, d)).astype(np.float32)
    v = orc.bf16_round(np.stack([orc.unit_rmsnorm(r) for r in v]).reshape(-1))
    q_in = rng.standard_normal(num_q * d).astype(np.float32)
    k_in = rng.standard_normal(kv_dim).astype(np.float32)
    v_in = rng.standard_normal(kv_dim).astype(np.float32)
    return slots, slot, k, v, q_in, k_in, v_in


def bf16_bits(a):
    return (orc.bf16_round(a).view(np.uint32) >> 16).astype(np.uint16).view(np.int16)


@pytest.mark.parametrize("num_q,num_kv,d,rot,theta,scale,clocks,n_recall", [
    (8, 1, 256, 64, 1e6, 1 / 16, [99999], [96]),   # BASELINE config 3, every recall slot live
    (8, 1, 256, 64, 1e6, 1 / 16, [99999], [0]),    # config 3, recall tier empty
    (8, 1, 256, 64, 1e6, 1 / 16, [600, 31, 54321], [5, 0, 96]),  # 3 instances in one launch
    (8, 1, 256, 64, 1e6, 1 / 16, [5, 70], [0, 3]),  # young rings: most CTAs hold no live slot
    (16, 8, 256, 256, 1e4, 1.0, [7000], [40]),     # 12B sliding layer, reference scale 1.0
    (4, 2, 128, 32, 1e4, 0.5, [3], [0]),           # young ring: 4 live slots
])
def test_qkv_rope_attn_fused_matches_checker(engine, num_q, num_kv, d, rot, theta, scale, clocks,
                                             n_recall):
    """The decode graph's fused kernel (attn_cluster_kernel) stand-alone against qkv_rope +
    decode_attn of the checker (qkv_rope.wgsl, decode_attn.wgsl; forward.zig:77-104), with the
    bf16 cache the model uses."""
    total, eps, n = 640, 1e-6, len(clocks)
    rng = np.random.default_rng(sum(clocks) + d)
    qn, kn = orc.synth_gain(d, 9, 1), orc.synth_gain(d, 9, 2)
    kv_dim = num_kv * d
    stride = (num_q + 2 * num_kv) * d
    qkv = np.zeros((n, stride), np.float32)
    kc = np.zeros((n, total * kv_dim), np.int16)
    vc = np.zeros_like(kc)
    sl = np.zeros((n, total), np.uint32)
    steps = np.zeros((n, 4), np.uint32)
    cases = []
    for i, (clock, nr) in enumerate(zip(clocks, n_recall)):
        slots, slot, k, v, q_in, k_in, v_in = c3_instance(rng, num_q, num_kv, d, clock, nr,
                                                          clock + i)
        qkv[i] = np.concatenate([q_in, k_in, v_in])
        kc[i], vc[i] = bf16_bits(k), bf16_bits(v)
        sl[i, :len(slots)] = slots
        steps[i] = [clock, slot, len(slots), 0]
        cases.append((slots, slot, k, v, q_in, k_in, v_in))
    qkv_d = dev(qkv.reshape(-1))
    kc_d, vc_d = dev(kc.reshape(-1)), dev(vc.reshape(-1))
    out = torch.zeros(n * num_q * d, dtype=torch.float32, device="cuda")
    q_ptr = qkv_d.data_ptr()
    engine.qkv_rope_attn(q_ptr, q_ptr + 4 * num_q * d, q_ptr + 4 * (num_q + num_kv) * d, dev(qn),
                         dev(kn), kc_d, vc_d, dev(sl.reshape(-1).view(np.int32)),
                         dev(steps.reshape(-1).view(np.int32)), out, num_q, num_kv, d, rot, 0,
                         theta, eps, scale, total, n, stride)
    got = host(out).reshape(n, num_q * d)
    gk = cache_to_np(kc_d, True).reshape(n, total * kv_dim)
    gv = cache_to_np(vc_d, True).reshape(n, total * kv_dim)
    assert np.array_equal(host(qkv_d).reshape(n, stride), qkv), "q|k|v input was modified"
    for i, (slots, slot, k, v, q_in, k_in, v_in) in enumerate(cases):
        rk, rv = k.copy(), v.copy()
        rq = orc.qkv_rope(q_in, k_in, v_in, qn, kn, rk, rv, True, num_q, num_kv, d, rot, 0, theta,
                          eps, clocks[i], slot, total)
        ref = orc.decode_attn(rq, rk, rv, slots, num_q, num_kv, d, total, scale)
        assert_close(got[i], ref, what=f"instance {i} attention output")
        row = slice(slot * kv_dim, (slot + 1) * kv_dim)
        for name, g, r in (("K", gk[i], rk), ("V", gv[i], rv)):
            assert np.max(np.abs(g[row] - r[row])) <= 2 ** -7 * max(1.0, np.max(np.abs(r[row]))), name
            rest = np.ones(total * kv_dim, bool)
            rest[row] = False
            assert np.array_equal(g[rest], r[rest]), f"{name} cache rows besides the slot changed"


def test_decode_attn_empty_list_gives_zeros(engine):
    num_q, d, total = 2, 64, 16
    kc = torch.zeros(total * d, dtype=torch.int16, device="cuda")
    out = torch.full((num_q * d,), 7.0, dtype=torch.float32, device="cuda")
    step = dev(np.array([0, 0, 0, 0], np.int32))
    sl = torch.zeros(total, dtype=torch.int32, device="cuda")
    engine.decode_attn(torch.ones(num_q * d, device="cuda"), kc, kc, sl, step, out, d, d,
                       num_q, 1.0, num_q, total)
    assert not np.any(host(out))


# ---------------------------------------------------------------------------------------
@pytest.mark.parametrize("case", ["random", "ties", "all_neg_inf", "nan_first", "nan_inside",
                                  "max_last", "small"])
def test_argmax_first_index_rule(engine, case):
    n = 262144 if case != "small" else 5
    # a fixed per-case seed (str hashes are randomised per process)
    rng = np.random.default_rng(zlib.crc32(case.encode()))
    v = rng.standard_normal(n).astype(np.float32)
    if case == "ties":
        v[[1000, 5, 200000]] = 50.0
    elif case == "all_neg_inf":
        v[:] = -np.inf
    elif case == "nan_first":
        v[0] = np.nan
    elif case == "nan_inside":
        v[123] = np.nan
        v[4567] = 9.0
    elif case == "max_last":
        v[-1] = 100.0
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    engine.argmax(dev(v), n, out)
    assert int(host(out)[0]) == orc.argmax(v)
