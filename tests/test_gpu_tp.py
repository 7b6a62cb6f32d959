"""Tensor-parallel decode on 2 and 4 GPUs (skipped with fewer): the ranks, each with its
engine, communicator and model shard, decode greedily; all ranks agree on every token, which
matches the one-process CPU checker, and the concatenated logits shards stay within the
path's tolerance.  Run with NCCL and with the one-shot peer all-reduce.  A last test has one
rank skip an all-reduce: the other rank's bounded flag wait runs out and reports a device
error instead of hanging (no GPU fault: a flag that nothing sets)."""
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


def _gpus():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("allreduce", ["nccl", "peer"])
@pytest.mark.parametrize("shape", ["tiny", "12b_width"])
def test_tensor_parallel_decode(world, shape, allreduce):
    import torch.multiprocessing as mp

    if _gpus() < world:
        pytest.skip(f"tensor parallelism over {world} ranks needs {world} GPUs")
    if shape == "tiny":
        cfg = tiny_cfg()
    else:
        cfg = tiny_cfg(vocab_size=262144, hidden_size=3840, intermediate_size=15360,
                       num_layers=2, num_q_heads=16, num_kv_heads=8, num_global_kv_heads=8,
                       head_dim=256, global_head_dim=256, num_anchors=32, window_size=512,
                       num_recall=96, full_every=2)
    cfg.pop("reference_graph", None)
    mp.spawn(_rank, args=(world, _free_port(), cfg, allreduce), nprocs=world, join=True)


def _skip_rank(rank, world, port):
    """Rank 1 leaves out the second of three all-reduce calls; rank 0 waits at most 50 ms for
    its flag and must report SX_ERR_DEVICE from the next sync, with its GPU still usable."""
    import torch.distributed as dist

    # a failure test: no NVLink multicast objects (NVLS) in NCCL
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.cuda.set_device(rank)
    eng = sx.Engine(rank)
    obj = [sx.comm_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    comm = sx.Comm(eng, obj[0], world, rank)
    try:
        comm.set_allreduce(False)
        comm.set_wait_ns(50_000_000)
        buf = torch.full((3840,), float(rank + 1), device="cuda")
        comm.allreduce(buf, 3840)  # call 1: both ranks
        eng.sync()
        assert torch.all(buf == 3.0).item()
        dist.barrier()
        if rank == 0:
            comm.allreduce(buf, 3840)  # call 2: rank 1 never arrives
            with pytest.raises(sx.SxError) as ei:
                eng.sync()
            assert ei.value.status == sx.SX_ERR_DEVICE
            eng.sync()  # the error word is cleared; the context still works
            z = torch.ones(8, device="cuda") * 2
            torch.cuda.synchronize()
            assert torch.all(z == 2).item()
        dist.barrier()
    finally:
        comm.close()
        eng.close()
        dist.destroy_process_group()


def test_peer_allreduce_wait_runs_out_when_a_rank_skips_a_call():
    import torch.multiprocessing as mp

    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    mp.spawn(_skip_rank, args=(2, _free_port()), nprocs=2, join=True)
