"""The multi-rank (N > 1) host path on CPU: world-size-2 `gloo` process
groups stand in for the NCCL ranks of `torchrun ... bench.py --gpus 2`.

Covered: the max-over-ranks reduction of timings, the batch partition of the
attention bench (16 rows) and of the end-to-end run (32 rows), the
rank-ordered all-gather of each step's logits, and the
reference arm under torchrun (rank 0 alone prints its line, every rank exits
0).  No GPU is touched."""

import json
import os
import socket
import subprocess
import sys

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    sys.path.insert(0, ROOT)
    import bench
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        dev = torch.device("cpu")
        mx = bench.max_over_ranks([float(rank), 5.0 - rank, 2.5], dev, world)
        rows = bench.rows_per_rank(32, world)
        rows16 = bench.rows_per_rank(bench.B, world)
        vocab = 7
        logits = torch.full((rows, vocab), float(rank)) + torch.arange(vocab).float() * (rank + 1)
        gathered = torch.empty(world * rows, vocab)
        g = bench.gather_logits(logits, gathered, world)
        mine = g[rank * rows:(rank + 1) * rows]
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
            json.dump({"max": mx, "rows": rows, "rows16": rows16, "gathered": g[:, 0].tolist(),
                       "mine_equal": bool(torch.equal(mine, logits))}, f)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_reduce_partition_and_gather_logits(tmp_path):
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    for rank in range(world):
        r = json.load(open(tmp_path / f"rank{rank}.json"))
        assert r["max"] == [1.0, 5.0, 2.5]          # slowest rank per timing, on every rank
        assert r["rows"] == 16 and r["rows16"] == 8  # disjoint halves of each batch
        assert r["gathered"] == [0.0] * 16 + [1.0] * 16  # rank order
        assert r["mine_equal"]                       # each rank's own rows come back unchanged


def test_reference_arm_under_torchrun_prints_one_line():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "3"]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [json.loads(l) for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1 and lines[0]["impl"] == "reference" and lines[0]["n_gpus"] == 2
    assert lines[0]["e2e"]["h2d_bytes_per_step"] == 0
