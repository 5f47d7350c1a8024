"""The multi-GPU host logic on CPU: two gloo ranks (one process each, 127.0.0.1), as bench.py
runs one rank a GPU.  Pages are sharded by rank with no exchange on the data path; the job's
time is the maximum over ranks; the reference arm runs on rank 0 only."""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shard_lines(bench, rank: int, world: int, pages_total: int):
    """The rank's lines as bench.py lays them out, page indices made global (slot numbers)."""
    from carbon_rec import native
    _, boxes, bws = bench.content(lambda b: native.crop_region(b)[1])
    slots = bench.shard(rank, world, pages_total)
    page_of, allb, bw = bench.lines_of(slots, boxes, bws)
    return page_of + slots[0], allb, bw


def _rank_main(rank: int, world: int, port: int, pages_total: int, out_dir: str) -> None:
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "carbon-ocr_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist

    import bench

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        page_of, boxes, bws = _shard_lines(bench, rank, world, pages_total)
        # each rank's own step time; the job's is the slowest rank's
        t = bench.reduce_max(0.5 + rank, world, "cpu")
        total = bench.reduce_sum(10 + rank, world, "cpu")
        dist.barrier()
        np.savez(Path(out_dir) / f"rank{rank}.npz", page_of=page_of, boxes=boxes, bws=bws, t=t, total=total)
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_two_ranks_shard_pages_and_take_the_max(tmp_path):
    world, pages_total = 2, 6
    mp.start_processes(_rank_main, args=(world, _free_port(), pages_total, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "carbon-ocr_b200"))
    import bench

    page_of1, boxes1, bws1 = _shard_lines(bench, 0, 1, pages_total)
    parts = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    # every slot's lines exactly once, in slot order: rank 0 takes the first half of the slots
    assert np.array_equal(np.concatenate([p["page_of"] for p in parts]), page_of1)
    assert np.array_equal(np.concatenate([p["boxes"] for p in parts]), boxes1)
    assert np.array_equal(np.concatenate([p["bws"] for p in parts]), bws1)
    assert [len(p["page_of"]) for p in parts] == [pages_total // world * bench.LINES_PER_PAGE] * world
    assert all(float(p["t"]) == 0.5 + (world - 1) for p in parts)
    assert all(float(p["total"]) == 10 * world + world * (world - 1) // 2 for p in parts)


def test_reference_arm_leaves_the_cuda_library_unloaded():
    """The reference arm times the reference's own code: its process never maps this
    repository's CUDA library (crop widths come from the reference's crop_region)."""
    import subprocess
    sys.path.insert(0, str(ROOT))
    from oracle import oracle as O
    if not O.Reference.available():
        pytest.skip("the reference's compiled code (oracle/_ref) is not here")
    code = ("import sys, json; sys.argv = ['bench.py', '--impl', 'reference', '--steps', '1', '--warmup', '0']; "
            "import bench; bench.main(); maps = open('/proc/self/maps').read(); "
            "print('MAPS', 'libcarbon_rec' in maps, 'libcarbon_ref' in maps)")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("{")][0]
    out = __import__("json").loads(line)
    assert out["impl"] == "reference" and out["value"] > 0 and out["config"]["lines"] == 65536
    assert "MAPS False True" in r.stdout, r.stdout[-500:]


def test_reference_arm_runs_on_rank_zero_only():
    sys.path.insert(0, str(ROOT))
    import bench

    class Args:
        gpus, steps, warmup = 2, 1, 1

    assert bench.run_reference(Args(), 1, 2) == 0  # no work, no output, exit 0
