"""The N > 1 host path of bench.py on CPU: two ranks as spawned processes over the gloo backend.

Each GPU runs a replica on its own request stream (weak scaling, no data-path collective); the only
collectives are the timing barrier and the reduction of the per-rank job numbers.
"""
import datetime
import os
import socket
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "gsv.cpp_b200"))
    import torch.distributed as dist
    import bench
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        ms, tok, seqs = [1000.0, 1250.0][rank], [90000, 95000][rank], [115, 118][rank]
        out = bench.reduce_over_ranks(ms, tok, seqs, world, "cpu")
        dist.barrier()
        stream = bench.RequestStream(rank, 2000)
        first = [stream.next() for _ in range(3)]
        q.put((rank, out, [seed for _, seed in first], [r.phones.tolist() for r, _ in first]))
    finally:
        dist.destroy_process_group()


def test_two_ranks_reduce_and_shard():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            rank, out, seeds, phones = q.get(timeout=120)
            res[rank] = (out, seeds, phones)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    # the slowest rank's time, all ranks' tokens and sequences, on every rank
    for r in (0, 1):
        assert res[r][0] == (1250.0, 185000.0, 233.0)
    # each rank serves its own request stream: different requests and sampler seeds
    assert set(res[0][1]).isdisjoint(res[1][1])
    assert res[0][2] != res[1][2]


def test_request_stream_is_reproducible():
    sys.path.insert(0, ROOT)
    import bench
    a = bench.RequestStream(1, 2000)
    b = bench.RequestStream(1, 2000)
    for _ in range(3):
        (ra, sa), (rb, sb) = a.next(), b.next()
        assert sa == sb and ra.phones.tolist() == rb.phones.tolist() and ra.prompt.tolist() == rb.prompt.tolist()


def test_reference_arm_line():
    """`bench.py --impl reference` (the CPU reference arm the driver runs beside this library's arm) prints
    one JSON line with the bench contract's keys; here on a small job (4 slots, 32 iterations) split into
    2 timed steps. Its config is the one the GPU arm prints for the same arguments."""
    import json
    import subprocess
    sys.path.insert(0, ROOT)
    import bench
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "2",
                          "--warmup", "3", "--slots", "4", "--iters", "32"], capture_output=True, text=True,
                         timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr
    line = json.loads(out.stdout.strip().splitlines()[-1])
    for k in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in line, k
    assert line["impl"] == "reference" and line["value"] > 0 and line["ms_per_step"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["kind"] == "port"
    args = bench.argparse.Namespace(slots=4, iters=32, refill_every=16, format="q8_0")
    assert line["config"] == bench.serve_config(args, 1)
    assert line["steps"] == 2 and line["job"]["chunks"] == 2 and line["job"]["tokens"] > 0
