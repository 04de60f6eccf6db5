"""Multi-rank plumbing of bench.py on the CPU: two gloo ranks (127.0.0.1) exercise the
max-over-ranks reduction and the whole-job aggregate that the GPU run uses over NCCL,
and the rule that both arms run one replica per rank."""
import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    import bench

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    local_ms = 100.0 + 50.0 * rank  # rank 1 is the slow one
    m = bench.reduce_max(local_ms, dist, "cpu")
    v = bench.aggregate_gbs(world, 10**9, 10, m)
    q.put((rank, m, v))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_max_and_aggregate():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, m, v in res:
        assert m == 150.0  # every rank sees the slowest rank's time
        assert v == pytest.approx(2 * 10**9 * 10 / 0.150 / 1e9)


def test_reference_arm_runs_on_every_rank(monkeypatch):
    """Both arms run one replica per rank (the reference's launchers act on the calling
    rank's own device), so rank 1 of the reference arm goes on to set up its GPU instead of
    returning early; here that set-up is intercepted before any CUDA call."""
    sys.path.insert(0, ROOT)
    import torch

    import bench

    class Reached(Exception):
        pass

    def fake_set_device(i):
        raise Reached(i)

    monkeypatch.setenv("RANK", "1")
    monkeypatch.setenv("WORLD_SIZE", "2")
    monkeypatch.setenv("LOCAL_RANK", "1")
    monkeypatch.setattr(sys, "argv", ["bench.py", "--impl", "reference", "--gpus", "2"])
    monkeypatch.setattr(torch.cuda, "set_device", fake_set_device)
    with pytest.raises(Reached) as e:
        bench.main()
    assert e.value.args == (1,)


def test_cfg1_byte_count_per_block():
    """BASELINE config 1 (512x512 image, 1024 tokens, batch 1): 134.5 MB per block."""
    sys.path.insert(0, ROOT)
    import bench

    total, _, _ = bench.chain_bytes(dict(bench.CFG, **bench.CFG1))
    assert abs(total / 28 / 1e6 - 134.5) < 1.0


def test_chain_byte_count_per_block():
    sys.path.insert(0, ROOT)
    import bench

    total, per_block, launches = bench.chain_bytes()
    assert abs(total / 28 / 1e6 - 1049.6) < 1.5  # MB per block at cfg2 (plus the tiny mod adds)
    assert sum(launches.values()) == 14


def test_cfg5_byte_count_per_image_pair():
    """BASELINE's throughput sweep: one image pair (9216 tokens x CFG 2 = 18432 rows) is
    2351 MB per block; --workload cfg5 gives each GPU 8/N pairs as batch rows."""
    sys.path.insert(0, ROOT)
    import bench

    cfg = dict(bench.CFG, pe=(1, 96, 96), batch=2)
    total, _, _ = bench.chain_bytes(cfg)
    assert abs(total / 28 / 1e6 - 2351) < 4
    four_pairs, _, _ = bench.chain_bytes(dict(cfg, batch=8))  # 2 GPUs: 4 pairs each
    assert abs(four_pairs / total - 4) < 0.01
