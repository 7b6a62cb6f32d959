"""The allocation-free decode attention entry point (sx_decode_attn_noalloc).

It serves callers that must not allocate device memory while decoding, for example a host
whose GPU memory belongs to another allocator's fixed arena.  The test calls it through the
C ABI twice in a row with different inputs (the shared scratch keeps the first call's
partials) and compares each result with the CPU checker's decode attention
(src/model/forward.zig:77-104) and with the engine-based sx_dispatch_decode_attn.  Its calls
come before it asks for the engine fixture, so when this file runs alone in a fresh process
they run with no engine in the process.  This file is collected last on purpose.
"""
import ctypes

import numpy as np
import pytest

import sx
from oracle import oracle as orc
from tests.conftest import assert_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _case(seed, num_q, num_kv, d, clock, n_recall):
    anchors, window, recall = 32, 512, 96
    total = anchors + window + recall
    ring = orc.Ring(1, anchors, window, recall)
    ring.prefill(0, clock)
    rng = np.random.default_rng(seed)
    for r in range(n_recall):
        ring.write_recall(0, r, int(rng.integers(0, clock)))
    ring.activate_slot(0, clock)
    slots = ring.get_active_slots(0, clock)
    kv = num_kv * d
    k = orc.bf16_round(rng.standard_normal(total * kv).astype(np.float32))
    v = orc.bf16_round(rng.standard_normal(total * kv).astype(np.float32))
    q = rng.standard_normal(num_q * d).astype(np.float32)

    def bf16_dev(a):
        return torch.from_numpy((a.view(np.uint32) >> 16).astype(np.uint16).view(np.int16)).cuda()

    slot_arr = np.concatenate([slots, np.zeros(total - len(slots), np.uint32)]).view(np.int32)
    return dict(
        q_host=q, k_host=k, v_host=v, slots_host=slots, num_kv=num_kv,
        q=torch.from_numpy(q).cuda(), k=bf16_dev(k), v=bf16_dev(v),
        slots=torch.from_numpy(slot_arr).cuda(),
        step=torch.from_numpy(np.array([clock, 0, len(slots), 0], np.int32)).cuda(),
        num_q=num_q, d=d, kv=kv, gqa=num_q // num_kv, total=total,
    )


def _noalloc(c, scale, out):
    st = sx.lib().sx_decode_attn_noalloc(
        c["q"].data_ptr(), c["k"].data_ptr(), c["v"].data_ptr(), c["slots"].data_ptr(),
        c["step"].data_ptr(), out.data_ptr(), c["d"], c["kv"], c["gqa"], scale, c["num_q"],
        c["total"], 1, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    sx.check(st)


def test_noalloc_attention_matches_checker_and_engine_path_twice(request):
    cases = [(_case(1, 16, 8, 256, 7000, 40), 1.0), (_case(2, 8, 1, 256, 99999, 96), 1 / 16)]
    outs = []
    for c, scale in cases:  # two calls in a row share the fixed scratch
        o = torch.full((c["num_q"] * c["d"],), float("nan"), device="cuda")
        _noalloc(c, scale, o)
        outs.append(o)
    torch.cuda.synchronize()
    for (c, scale), got in zip(cases, outs):
        ref = orc.decode_attn(c["q_host"], c["k_host"], c["v_host"], c["slots_host"], c["num_q"],
                              c["num_kv"], c["d"], c["total"], scale)
        assert_close(got.cpu().numpy(), ref, atol=1e-4, rtol=1e-3, what="noalloc vs checker")
    engine = request.getfixturevalue("engine")
    for (c, scale), got in zip(cases, outs):
        want = torch.empty_like(got)
        engine.decode_attn(c["q"], c["k"], c["v"], c["slots"], c["step"], want, c["d"], c["kv"],
                           c["gqa"], scale, c["num_q"], c["total"])
        engine.sync()
        assert_close(got.cpu().numpy(), want.cpu().numpy(), atol=1e-4, rtol=1e-3,
                     what="noalloc vs engine attention")


def test_noalloc_rejects_requests_above_the_fixed_scratch():
    z = torch.zeros(16, device="cuda")
    # 64 q heads x 32 chunks x 514 floats x 4 B > 1 MiB
    st = sx.lib().sx_decode_attn_noalloc(z.data_ptr(), z.data_ptr(), z.data_ptr(), z.data_ptr(),
                                         z.data_ptr(), z.data_ptr(), 512, 8 * 512, 8, 1.0, 64,
                                         1024, 1, None)
    assert st == sx.SX_ERR_INVALID
    assert "1 MiB" in sx.last_error()
