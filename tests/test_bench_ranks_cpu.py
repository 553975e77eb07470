"""The multi-rank plumbing of bench.py on the CPU: two `gloo` ranks, as torchrun launches them (RANK,
WORLD_SIZE, MASTER_ADDR=127.0.0.1). Checks the max over ranks (every rank gets the slowest rank's time), the
gather of per-rank figures in rank order (the decode's per-GPU and aggregate bytes/s), and that the
reference arm prints its line on rank 0 only while the other rank exits without work."""

from __future__ import annotations

import json
import os
import socket
import sys
from pathlib import Path

import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    sys.path.insert(0, str(ROOT))
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    import contextlib
    import io

    import torch.distributed as dist

    import bench

    bench.init_dist("gloo", timeout_s=60)
    res = {"max": bench.max_over_ranks(1.5 + rank), "gathered": bench.gather_over_ranks(10.0 * (rank + 1))}
    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
        res["ref_rc"] = bench.main(["--impl", "reference", "--gpus", str(world), "--steps", "1", "--warmup", "3"])
    res["ref_out"] = buf.getvalue()
    dist.barrier()
    dist.destroy_process_group()
    Path(out_dir, f"rank{rank}.json").write_text(json.dumps(res))


@pytest.mark.timeout(600)
def test_two_gloo_ranks_take_the_max_gather_in_order_and_print_once(tmp_path):
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    res = [json.loads((tmp_path / f"rank{r}.json").read_text()) for r in range(world)]
    assert all(r["max"] == 2.5 for r in res)
    assert all(r["gathered"] == [10.0, 20.0] for r in res)
    assert res[0]["ref_rc"] == 0 and res[1]["ref_rc"] == 0
    assert res[1]["ref_out"] == ""
    line = json.loads(res[0]["ref_out"].strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["n_gpus"] == world and line["steps"] == 1
    assert line["config"] == __import__("bench").workload_config(world)
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["kind"] == "port"
