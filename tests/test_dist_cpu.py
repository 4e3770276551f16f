"""Block-row sharding across ranks, on CPU with the gloo backend.

Each of P ranks computes its block-row shard of a layer with the CPU oracle
(the GPU kernels are not needed to test the host logic), writes it into its
slot of the gather buffer, and ShardPlan.gather all-gathers and assembles y;
every rank must then hold exactly the single-process oracle output.  A
second test makes one rank fail before the collective and checks the other
sees an error (timeout) instead of hanging.
"""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, cfg: str, out_dir: str):
    sys.path.insert(0, str(REPO))
    sys.path.insert(0, str(REPO / "oracle"))
    import datetime

    import torch.distributed as dist

    import slr_oracle
    from s_salaad_b200 import workloads
    from s_salaad_b200.shard import ShardPlan

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    spec = workloads.layer_set(cfg)[0] if cfg != "small" else _small()
    t = spec.tensors("cpu", torch.float32)
    x = workloads.tokens(9, spec.in_features, seed=4)
    plan = ShardPlan(spec.crow, out_features=spec.out_features, block_p=spec.block_p, block_q=spec.block_q,
                     rank_r=spec.rank, rank=rank, world=world)
    p = plan.slice(t)
    buf = plan.gather_buffer(9, torch.float32, "cpu")
    buf.zero_()
    if plan.width:
        buf[rank][:, :plan.width] = slr_oracle.lrs_forward_f32(x, p["A"], p["B"], p["S_crow"], p["S_col"],
                                                                p["S_values"], p["S_active_rows"], p["bias"])
    y = plan.gather(buf)
    torch.save({"y": y, "bounds": torch.from_numpy(np.asarray(plan.bounds))}, os.path.join(out_dir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def _small():
    from s_salaad_b200 import workloads

    crow, col = workloads.zipf_structure(12, 10, 0.3, 1.1, seed=5)
    return workloads.LayerSpec("small", 12 * 16, 10 * 16, 24, 16, 16, crow, col, seed=6, bias_std=0.01)


@pytest.mark.parametrize("world,cfg", [(2, "small"), (3, "small"), (2, "cfg1")])
def test_sharded_layer_equals_single_process(tmp_path, oracle, world, cfg):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, cfg, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
        assert p.exitcode == 0
    from s_salaad_b200 import workloads

    spec = workloads.layer_set(cfg)[0] if cfg != "small" else _small()
    t = spec.tensors("cpu", torch.float32)
    x = workloads.tokens(9, spec.in_features, seed=4)
    ref = oracle.lrs_forward_f32(x, t["A"], t["B"], t["S_crow"], t["S_col"], t["S_values"], t["S_active_rows"],
                                 t["bias"])
    bounds = None
    for r in range(world):
        got = torch.load(tmp_path / f"rank{r}.pt")
        # each output element comes from exactly one rank with the same arithmetic
        torch.testing.assert_close(got["y"], ref, rtol=0, atol=0)
        if bounds is None:
            bounds = got["bounds"].numpy()
        assert np.array_equal(bounds, got["bounds"].numpy())
    assert bounds[0] == 0 and bounds[-1] == spec.nb


def _failing_worker(rank: int, world: int, port: int, out_dir: str):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        raise SystemExit(3)  # this rank fails before the collective
    buf = torch.zeros(2, 4)
    try:
        dist.all_gather_into_tensor(buf.view(-1), buf[0].view(-1))
        status = "completed"
    except Exception as exc:  # noqa: BLE001 - the point is that it raises
        status = f"error: {type(exc).__name__}"
    Path(out_dir, "status.txt").write_text(status)


def test_rank_failure_surfaces_as_an_error(tmp_path):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert procs[1].exitcode == 3
    status = (tmp_path / "status.txt").read_text()
    assert status.startswith("error"), status
