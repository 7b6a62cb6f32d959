"""Tensor-parallel decode on 2 GPUs (skipped with fewer): two ranks, each with its engine,
communicator and model shard, decode greedily; both ranks agree on every token, which
matches the one-process CPU checker, and the concatenated logits shards stay within the
path's tolerance.  Run with NCCL and with the one-shot peer all-reduce."""
import os
import socket

import numpy as np
import pytest

import sx
from oracle import oracle as orc
from tests.conftest import assert_close
from tests.test_gpu_model import tiny_cfg

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

SEED, STEPS, START = 11, 6, 40


def _rank(rank, world, port, cfg, allreduce="nccl"):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.cuda.set_device(rank)
    eng = sx.Engine(rank)
    obj = [sx.comm_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    comm = sx.Comm(eng, obj[0], world, rank)
    comm.set_allreduce(allreduce == "nccl")
    assert comm.allreduce_is_nccl == (allreduce == "nccl")
    model = sx.Model(eng, sx.model_config(**cfg, tp_size=world, tp_rank=rank), comm)
    try:
        model.synth_weights(SEED)
        model.fill_kv(SEED)
        plan = sx.tp_shard_plan(sx.model_config(**cfg, tp_size=world, tp_rank=rank))
        ring = sx.Ring(1, cfg["num_anchors"], cfg["window_size"], cfg["num_recall"])
        ring.prefill(0, START)
        ref = orc.Model(cfg, SEED) if rank == 0 else None
        if ref is not None:
            ref.fill_kv(SEED)
            ref.ring.prefill(0, START)
        token = 3
        for s in range(STEPS):
            clock = START + s
            x = sx.synth_embed_row(cfg["hidden_size"], token, SEED)
            slot = ring.activate_slot(0, clock)
            logits = np.zeros(plan.vocab, np.float32)
            tok = model.forward_token(x, clock, slot, ring.get_active_slots(0, clock), True,
                                      logits)
            parts = [torch.zeros(plan.vocab) for _ in range(world)]
            dist.all_gather(parts, torch.from_numpy(logits))
            toks = [None] * world
            dist.all_gather_object(toks, tok)
            if rank == 0:
                assert len(set(toks)) == 1, f"ranks disagree on the token: {toks}"
                rtok, rlogits, _ = ref.forward(x, clock, True)
                assert_close(np.concatenate([p.numpy() for p in parts]), rlogits,
                             what=f"tp logits step {s}")
                srt = np.sort(rlogits)
                assert tok == rtok or srt[-1] - srt[-2] < 1e-3, f"step {s}: {tok} vs {rtok}"
            token = toks[0]
    finally:
        model.close()
        comm.close()
        eng.close()
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="tensor parallelism needs 2 GPUs")
@pytest.mark.parametrize("allreduce", ["nccl", "peer"])
@pytest.mark.parametrize("shape", ["tiny", "12b_width"])
def test_tensor_parallel_decode_two_gpus(shape, allreduce):
    import torch.multiprocessing as mp

    if shape == "tiny":
        cfg = tiny_cfg()
    else:
        cfg = tiny_cfg(vocab_size=262144, hidden_size=3840, intermediate_size=15360,
                       num_layers=2, num_q_heads=16, num_kv_heads=8, num_global_kv_heads=8,
                       head_dim=256, global_head_dim=256, num_anchors=32, window_size=512,
                       num_recall=96, full_every=2)
    cfg.pop("reference_graph", None)
    mp.spawn(_rank, args=(2, _free_port(), cfg, allreduce), nprocs=2, join=True)
