"""Multi-rank env sharding over gloo (world_size 2).

Each rank owns the global env range that ``bench.shard`` gives it and builds
its batch with ``env_offset``; snapshot levels, the frame-limit RNG and the
action stream are keyed by the global env index.  Gathered over ranks, the
sharded run must equal one batch over all envs, bit for bit -- the path has
no exchange step, so nothing else couples the ranks.  Where CUDA exists each
rank drives the product (libnesle_b200.so through its C ABI, on GPU
rank % device_count) and the checker is only the comparison; without CUDA the
ranks drive the checker, which still exercises the rank plumbing.  The timing
reduction ``bench.combine_over_ranks`` is checked on the same process group.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

ENVS_PER_RANK = 24
STEPS = 8
FIELDS = ("pc", "a", "x", "y", "sp", "p", "cycles", "ram", "oam", "frame", "last_reward", "last_done", "episode")


def _short_config4():
    from nesle_b200 import workloads as w

    wl = w.config4()
    wl.done_args = (6, 20)  # many auto-resets inside 8 env-steps
    return wl


def _run(wl, offset: int, n: int, device: int | None = None) -> dict:
    """The shard's state after STEPS env-steps: on the checker (device None) or
    on the product on CUDA device `device`."""
    env = np.arange(offset, offset + n)
    kw = dict(env_to_level=wl.env_to_level(env), done_mode=wl.done_mode, done_args=wl.done_args, seed=wl.seed,
              env_offset=offset)
    if device is None:
        from oracle import Oracle

        o = Oracle(n, wl.frameskip, wl.rom.image, wl.snapshots, **kw)
    else:
        from harness import GpuCore

        o = GpuCore(n, wl.frameskip, wl.rom.image, wl.snapshots, device=device, **kw)
    for s in range(STEPS):
        o.step(wl.actions(env, s))
    return {f: o.get(f) for f in FIELDS}


def _worker(rank: int, world: int, port: int, result_dir: str, product: bool = False) -> None:
    import torch
    import torch.distributed as dist

    import bench

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        wl = _short_config4()
        offset, env = bench.shard(rank, ENVS_PER_RANK)
        assert offset == rank * ENVS_PER_RANK and len(env) == ENVS_PER_RANK
        mine = _run(wl, offset, ENVS_PER_RANK, rank % torch.cuda.device_count() if product else None)
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        # rank r reports elapsed 10 + r ms, e2e 1 + r s, 100 * (r + 1) instructions
        t, e, i = bench.combine_over_ranks(10.0 + rank, 1.0 + rank, 100 * (rank + 1), torch.device("cpu"), world)
        if rank == 0:
            full = _run(wl, 0, ENVS_PER_RANK * world)
            for f in FIELDS:
                cat = np.concatenate([g[f] for g in gathered])
                np.testing.assert_array_equal(cat, full[f], err_msg=f)
            assert int(full["last_done"].sum()) + int((full["episode"] > 0).sum()) > 0
            assert (t, e, i) == (10.0 + world - 1, 1.0 + world - 1, sum(100 * (r + 1) for r in range(world)))
            with open(os.path.join(result_dir, "ok"), "w") as fh:
                fh.write("ok")
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_sharding_equals_one_batch(tmp_path):
    mp = pytest.importorskip("torch.multiprocessing")
    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    assert (tmp_path / "ok").read_text() == "ok"


@pytest.mark.gpu
def test_two_rank_sharding_on_the_product(tmp_path):
    """The same over gloo with each rank stepping its shard on the CUDA path."""
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from nesle_b200 import build

    build.build()
    mp = pytest.importorskip("torch.multiprocessing")
    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path), True), nprocs=2, join=True,
                       start_method="spawn")
    assert (tmp_path / "ok").read_text() == "ok"


def test_shard_ranges_tile_the_global_range():
    import bench

    ranges = [bench.shard(r, 65536)[1] for r in range(8)]
    cat = np.concatenate(ranges)
    np.testing.assert_array_equal(cat, np.arange(8 * 65536))


@pytest.mark.parametrize("summary", ["step_kernel_config4.txt", "gray84_kernel_config3.txt",
                                     "render_kernel_rgb_config3.txt"])
def test_bench_reads_traffic_from_profile_summaries(summary):
    """The bench line's roofline `traffic` comes from the committed ncu summaries."""
    import bench

    t = bench.profile_traffic(summary)
    assert t is not None and t > 1e8, summary


def test_reference_arm_prints_one_contract_line():
    """`bench.py --impl reference` (the reference CPU core on the host cores)
    prints exactly one JSON line with the bench contract's keys, on CPU."""
    import json
    import subprocess
    import sys
    from pathlib import Path

    from oracle import reference_available

    if not reference_available():
        pytest.skip("oracle/_ref not built")
    root = Path(__file__).resolve().parents[1]
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--envs", "64", "--steps", "1",
                          "--warmup", "1"], cwd=root, capture_output=True, text=True, timeout=300, check=True)
    lines = [ln for ln in out.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["value"] > 0 and d["unit"] == "env-steps/s" and d["higher_is_better"]
    assert d["metric"].startswith("env-steps/s") and d["n_gpus"] == 1 and d["steps"] == 1
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
