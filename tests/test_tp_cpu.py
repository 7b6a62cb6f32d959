"""Tensor-parallel decode, host logic on CPU: two gloo ranks run the CPU checker on the shards
that libsx's sx_tp_shard_plan assigns them (rows of q/k/v/gate/up/LM head, 32-column blocks of
o/down, the rank's kv heads of the cache), sum the row-parallel o / down outputs with an
all-reduce and merge the vocabulary-parallel argmax candidates exactly like the device merge.
The tokens must equal the one-process checker's and the logits stay within the path's
tolerance.  No GPU is used."""
import os
import socket

import numpy as np
import pytest

import sx
from oracle import oracle as orc
from tests.conftest import assert_close

torch = pytest.importorskip("torch")

T_INPUT_NORM, T_Q, T_K, T_V, T_O, T_QNORM, T_KNORM = 0, 1, 2, 3, 4, 5, 6
T_POST_ATTN, T_PRE_FFN, T_GATE, T_UP, T_DOWN, T_POST_FFN, T_SCALAR = 7, 8, 9, 10, 11, 12, 13

CFG = dict(vocab_size=4096, hidden_size=256, intermediate_size=640, num_layers=3,
           num_q_heads=4, num_kv_heads=2, num_global_kv_heads=2, head_dim=64, global_head_dim=64,
           num_anchors=4, window_size=8, num_recall=4, kv_bf16=1, has_post_norms=1,
           full_every=3, attention_k_eq_v=0, rms_norm_eps=1e-6, rope_theta=10000.0,
           rope_theta_full=1000000.0, attn_scale=1.0)
SEED, STEPS, START = 7, 5, 20


def stream(layer, kind):
    return (layer + 1) * 64 + kind


def layer_shape(c, l):
    """loader.zig:36-42: sliding vs full-attention layer geometry."""
    full = c["full_every"] and (l + 1) % c["full_every"] == 0
    hd = c["global_head_dim"] if full else c["head_dim"]
    return dict(full=full, hd=hd, rot=hd // 4 if full else hd,
                kv=c["num_global_kv_heads"] if full else c["num_kv_heads"],
                theta=c["rope_theta_full"] if full else c["rope_theta"],
                k_eq_v=bool(full and c["attention_k_eq_v"]))


def rows_of(w, rows, cols, r0, n):
    return np.ascontiguousarray(w.reshape(rows, cols // 32, 5)[r0:r0 + n]).ravel()


def blocks_of(w, rows, cols, b0, nb):
    return np.ascontiguousarray(w.reshape(rows, cols // 32, 5)[:, b0:b0 + nb]).ravel()


class ShardModel:
    """One rank's shard of the checker's model, built from the plan of libsx."""

    def __init__(self, c, plan, kv_src):
        self.c, self.p = c, plan
        H, I = c["hidden_size"], c["intermediate_size"]
        self.L = []
        for l in range(c["num_layers"]):
            g = layer_shape(c, l)
            hd, nkv = g["hd"], (plan.global_kv_heads if g["full"] else plan.kv_heads)
            kv0 = plan.global_kv_head0 if g["full"] else plan.kv_head0
            qd_glob, kvd_glob = c["num_q_heads"] * hd, g["kv"] * hd
            wq = synth(qd_glob, H, stream(l, T_Q))
            wk = synth(kvd_glob, H, stream(l, T_K))
            wv = synth(kvd_glob, H, stream(l, T_K if g["k_eq_v"] else T_V))
            wo = synth(H, qd_glob, stream(l, T_O))
            wg, wu = synth(I, H, stream(l, T_GATE)), synth(I, H, stream(l, T_UP))
            wd = synth(H, I, stream(l, T_DOWN))
            slots = c["num_anchors"] + c["window_size"] + c["num_recall"]
            kc = kv_src.kcache(l).reshape(slots, g["kv"], hd)[:, kv0:kv0 + nkv].copy().ravel()
            vc = kv_src.vcache(l).reshape(slots, g["kv"], hd)[:, kv0:kv0 + nkv].copy().ravel()
            z = orc.synth_normal(SEED, stream(l, T_SCALAR), 0)
            self.L.append(dict(
                g=g, nkv=nkv, hd=hd,
                wq=rows_of(wq, qd_glob, H, plan.q_head0 * hd, plan.q_heads * hd),
                wk=rows_of(wk, kvd_glob, H, kv0 * hd, nkv * hd),
                wv=rows_of(wv, kvd_glob, H, kv0 * hd, nkv * hd),
                wo=blocks_of(wo, H, qd_glob, plan.q_head0 * hd // 32, plan.q_heads * hd // 32),
                wg=rows_of(wg, I, H, plan.inter0, plan.inter),
                wu=rows_of(wu, I, H, plan.inter0, plan.inter),
                wd=blocks_of(wd, H, I, plan.inter0 // 32, plan.inter // 32),
                in_norm=orc.synth_gain(H, SEED, stream(l, T_INPUT_NORM)),
                post_attn=orc.synth_gain(H, SEED, stream(l, T_POST_ATTN)),
                pre_ffn=orc.synth_gain(H, SEED, stream(l, T_PRE_FFN)),
                post_ffn=orc.synth_gain(H, SEED, stream(l, T_POST_FFN)),
                q_norm=orc.synth_gain(hd, SEED, stream(l, T_QNORM)),
                k_norm=orc.synth_gain(hd, SEED, stream(l, T_KNORM)),
                scalar=float(orc.bf16_round(np.array([np.float32(0.05) * np.float32(z) + 1],
                                                     np.float32))[0]),
                kc=kc, vc=vc))
        head = orc.synth_q8(c["vocab_size"], H, SEED, 2)
        self.head = np.ascontiguousarray(
            head.reshape(c["vocab_size"], H // 32, 9)[plan.vocab0:plan.vocab0 + plan.vocab]).ravel()
        self.final_norm = orc.synth_gain(H, SEED, 3)

    def forward(self, x, clock, slot, slots, allreduce, allgather):
        """The fused graph's op order with the two all-reduces and the candidate merge."""
        c, p = self.c, self.p
        H, eps = c["hidden_size"], c["rms_norm_eps"]
        total = c["num_anchors"] + c["window_size"] + c["num_recall"]
        x = np.array(x, np.float32)
        for L in self.L:
            g, hd, nkv = L["g"], L["hd"], L["nkv"]
            normed = orc.rmsnorm(x, L["in_norm"], eps)
            q = orc.gemv_q4(L["wq"], normed, p.q_heads * hd, H)
            k = orc.gemv_q4(L["wk"], normed, nkv * hd, H)
            v = orc.gemv_q4(L["wv"], normed, nkv * hd, H)
            q = orc.qkv_rope(q, k, v, L["q_norm"], L["k_norm"], L["kc"], L["vc"], c["kv_bf16"],
                             p.q_heads, nkv, hd, g["rot"], g["k_eq_v"], g["theta"], eps, clock,
                             slot, total)
            attn = orc.decode_attn(q, L["kc"], L["vc"], slots, p.q_heads, nkv, hd, total,
                                   c["attn_scale"])
            mlp = allreduce(orc.gemv_q4(L["wo"], attn, H, p.q_heads * hd))
            mlp = orc.rmsnorm(mlp, L["post_attn"], eps)
            x, normed = orc.add_rmsnorm(x, mlp, L["pre_ffn"], eps, 1.0)
            act = orc.gate_up_geglu_q4(L["wg"], L["wu"], normed, p.inter, H)
            mlp = allreduce(orc.gemv_q4(L["wd"], act, H, p.inter))
            mlp = orc.rmsnorm(mlp, L["post_ffn"], eps)
            x, normed = orc.add_rmsnorm(x, mlp, L["in_norm"], eps, L["scalar"])
        logits = orc.gemv_q8(self.head, orc.rmsnorm(x, self.final_norm, eps), p.vocab, H)
        # local candidate {value, global index, logits[0] is NaN}; NaN logits never win
        v = np.where(np.isnan(logits), -np.inf, logits)
        i = int(np.argmax(v))
        nan0 = p.vocab0 == 0 and bool(np.isnan(logits[0]))
        cand = allgather(np.array([v[i], p.vocab0 + i, float(nan0)], np.float64))
        best = None
        for cv, ci, cn in cand:
            if cn:
                return 0, logits
            if best is None or cv > best[0] or (cv == best[0] and ci < best[1]):
                best = (cv, int(ci))
        return best[1], logits


def synth(rows, cols, st):
    return orc.synth_q4(rows, cols, SEED, st)


def _rank(rank, world, port):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        c = dict(CFG)
        plan = sx.tp_shard_plan(sx.model_config(**c, tp_size=world, tp_rank=rank))
        ref = orc.Model(c, SEED)
        ref.fill_kv(SEED)
        shard = ShardModel(c, plan, ref)
        ring = orc.Ring(1, c["num_anchors"], c["window_size"], c["num_recall"])
        ring.prefill(0, START)
        ref.ring.prefill(0, START)

        def allreduce(a):
            t = torch.from_numpy(np.ascontiguousarray(a, np.float32))
            dist.all_reduce(t)
            return t.numpy()

        def allgather(a):
            out = [torch.zeros(len(a), dtype=torch.float64) for _ in range(world)]
            dist.all_gather(out, torch.from_numpy(a))
            return [o.numpy() for o in out]

        token = 17
        for s in range(STEPS):
            clock = START + s
            x = orc.synth_embed_row(c["hidden_size"], token, SEED)
            slot = ring.activate_slot(0, clock)
            slots = ring.get_active_slots(0, clock)
            tok, logits = shard.forward(x, clock, slot, slots, allreduce, allgather)
            parts = [torch.zeros(plan.vocab, dtype=torch.float32) for _ in range(world)]
            dist.all_gather(parts, torch.from_numpy(logits))
            rtok, rlogits, _ = ref.forward(x, clock, True)
            if rank == 0:
                full = np.concatenate([p.numpy() for p in parts])
                assert_close(full, rlogits, what=f"tp logits step {s}")
                srt = np.sort(rlogits)
                assert tok == rtok or srt[-1] - srt[-2] < 1e-3, f"step {s}: {tok} vs {rtok}"
            token = rtok
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_plan_splits_evenly():
    c = sx.model_config(**CFG, tp_size=2, tp_rank=1)
    p = sx.tp_shard_plan(c)
    assert (p.q_heads, p.q_head0, p.kv_heads, p.kv_head0) == (2, 2, 1, 1)
    assert (p.inter, p.inter0, p.vocab, p.vocab0) == (320, 320, 2048, 2048)
    with pytest.raises(sx.SxError):
        sx.tp_shard_plan(sx.model_config(**CFG, tp_size=3, tp_rank=0))  # 4 q heads / 3


def test_tensor_parallel_two_ranks_match_one_process():
    import torch.multiprocessing as mp

    mp.spawn(_rank, args=(2, _free_port()), nprocs=2, join=True)
