"""The multi-GPU harness on CPU: two ranks over gloo (world_size 2) exercise what every rank of a
`torchrun` bench job does apart from the GPU work — rank discovery, a seeded batch of its own
per rank, the job time as the maximum and the tokens as the sum over ranks — and the reference
arm's rank-0-only rule."""
import datetime
import importlib
import os
import socket
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    bench = importlib.import_module("bench")
    synth = importlib.import_module("gemma-embed-swift_b200.synthetic")
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    try:
        env = bench.dist_env()
        seqs = synth.config_sequences(2, seed=rank)
        ntok = sum(len(s) for s in seqs)
        ms = [3.0, 5.0][rank]
        result = bench.reduce_max_sum(dist, ms, ntok)
        q.put((rank, env, ntok, result, list(seqs[0][:8])))
    finally:
        dist.destroy_process_group()


def test_two_ranks_over_gloo():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(2):
        rank, env, ntok, result, head = q.get(timeout=120)
        out[rank] = (env, ntok, result, head)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert out[0][0] == (0, 2, 0) and out[1][0] == (1, 2, 1)
    total = out[0][1] + out[1][1]
    assert out[0][2] == (5.0, total) and out[1][2] == (5.0, total)  # max time, summed tokens
    assert out[0][3] != out[1][3]  # each rank embeds its own seeded batch (weak scaling)


def test_reference_arm_runs_on_rank_zero_only():
    sys.path.insert(0, ROOT)
    bench = importlib.import_module("bench")

    class Args:
        arch, config, steps, warmup = "gemma-embedding", 2, 1, 0

    assert bench.run_reference(Args(), rank=1, world=2) == 0  # returns at once, no oracle work
