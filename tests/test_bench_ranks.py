"""The N > 1 logic of bench.py on CPU: two gloo ranks on 127.0.0.1 (the
replicas of the scaling run; no data-path collective exists, only the
max-over-ranks timing, the whole-job value and the box run's sums of
frames), and the reference arm's rank handling (rank 0 alone runs it)."""
import os
import socket
import sys

import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    import datetime

    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    import bench
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    # rank r took 10 + r ms for the frames and 20 - r ms end to end
    ms, e2e = bench.max_over_ranks([10.0 + rank, 20.0 - rank], dist, "cpu")
    # the box run: rank r's frames and endings summed over the ranks
    frames, eos = bench.sum_over_ranks([1000 + rank, rank], dist)
    dist.barrier()
    dist.destroy_process_group()
    out.put((rank, ms, e2e, bench.job_value(world, 156, ms), frames, eos))


def test_max_over_ranks_and_job_value_gloo():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for _, ms, e2e, v, frames, eos in res:
        assert ms == 11.0 and e2e == 20.0  # the slowest rank's times
        assert abs(v - 2 * 156 / 0.011) < 1e-6  # frames of both ranks over that time
        assert frames == 2001.0 and eos == 1.0


def test_single_rank_keeps_its_values():
    import bench
    assert bench.max_over_ranks([3.5, 4.0], None, "cpu") == [3.5, 4.0]
    assert bench.job_value(1, 100, 250.0) == 400.0
    assert bench.sum_over_ranks([7, 2.5], None) == [7.0, 2.5]


def test_reference_arm_runs_on_rank_0_only():
    import bench

    class Args:
        config, warmup, steps, gpus = "q8_0", 0, 1, 2
        talker_layers, pred_layers = 28, 5

    # rank 1 of a torchrun job returns at once, without work or output
    assert bench.reference_arm(Args(), 1) is None
