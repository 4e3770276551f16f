"""Run under torchrun (one process per GPU): every rank computes its
block-row shard of real-size layers with the CUDA kernels, NCCL all-gathers
y, and each rank compares the result with the single-GPU forward of the full
layer (computed on its own device).  Exit status 0 = all equal."""
from __future__ import annotations

import datetime
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
from s_salaad_b200 import ops, workloads  # noqa: E402
from s_salaad_b200.shard import ShardedLayer  # noqa: E402


def check_peer_outputs(rank: int, world: int, dev) -> int:
    """Outputs stored straight into every rank's y (peer memory) equal the
    all-gather path bit for bit, call after call, eagerly and from a CUDA graph."""
    import ctypes

    from s_salaad_b200 import _lib
    from s_salaad_b200.shard import PeerOutputs, all_ranks

    bad = 0
    for cfg, idx, T in [("cfg4", 0, 1024), ("cfg4", 6, 300)]:
        s = workloads.layer_set(cfg)[idx]
        t = s.tensors(dev, torch.bfloat16)
        x = workloads.tokens(T, s.in_features, seed=7, device=dev, dtype=torch.bfloat16)
        sh = ShardedLayer(t, s.crow, in_features=s.in_features, out_features=s.out_features,
                          block_p=s.block_p, block_q=s.block_q, rank=rank, world=world)
        if not all_ranks(sh.peers_supported(x), dev):
            print(f"rank {rank}/{world} peers {cfg}[{idx}] T={T} not supported on every rank", flush=True)
            bad += 1
            continue
        ref = sh.forward(x)
        po = PeerOutputs(sh, T, torch.bfloat16, dev)
        errs = []
        for _ in range(3):
            po.y.zero_()
            sh.start_peers(x, po)
            y = sh.finish_peers(po)
            errs.append(not torch.equal(y, ref))
        stream = torch.cuda.Stream(dev)
        stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(stream):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                sh.start_peers(x, po)
                sh.finish_peers(po)
        torch.cuda.current_stream(dev).wait_stream(stream)
        for _ in range(3):
            po.y.zero_()
            g.replay()
            errs.append(not torch.equal(po.y, ref))
        torch.cuda.synchronize()
        st = ctypes.c_int(-1)
        _lib.check(_lib.load().slr_device_status(ctypes.byref(st)), "device_status")
        ok = not any(errs) and st.value == 0
        bad += 0 if ok else 1
        print(f"rank {rank}/{world} peers {cfg}[{idx}] T={T} mismatching calls={sum(errs)} "
              f"status={st.value} {'ok' if ok else 'MISMATCH'}", flush=True)
        del g
        dist.barrier()
        po.close()
    return bad


def check_set_peers(rank: int, world: int, dev, x, grp, shards, refs) -> int:
    """q/k/v (one group, one H) and o_proj (its own input and H) of cfg4: the
    four combines as ONE launch storing into every rank's y, signals on the
    first layer's slot; three calls (the last with the four x*B^T products as
    one layer-set launch), each equal to the single-GPU forward bit for bit."""
    from s_salaad_b200.shard import PeerOutputs, ShardedLayer, all_ranks, finish_set_peers, start_set_peers

    T = x.shape[0]
    s_o = workloads.layer_set("cfg4")[3]
    t = s_o.tensors(dev, torch.bfloat16)
    x_o = workloads.tokens(T, s_o.in_features, seed=6, device=dev, dtype=torch.bfloat16)
    order = torch.from_numpy(ops.plan_row_order(s_o.crow.astype(np.int32))).to(dev)
    full = ops.LayerDesc(A=t["A"], B=t["B"], bias=t["bias"], crow=t["S_crow"], col=t["S_col"],
                         values=t["S_values"], row_order=order, in_features=s_o.in_features,
                         out_features=s_o.out_features, block_p=s_o.block_p, block_q=s_o.block_q)
    ref_o = full.forward(x_o)
    sh_o = ShardedLayer(t, s_o.crow, in_features=s_o.in_features, out_features=s_o.out_features,
                        block_p=s_o.block_p, block_q=s_o.block_q, rank=rank, world=world)
    layers = list(shards) + [sh_o]
    xs = [x, x, x, x_o]
    wants = list(refs) + [ref_o]
    if not all_ranks(all(L.peers_supported(xi) for L, xi in zip(layers, xs)), dev):
        print(f"rank {rank}/{world} set peers: not supported on every rank", flush=True)
        return 1
    pos = [PeerOutputs(L, T, torch.bfloat16, dev) for L in layers]
    bad = 0
    lset = ops.LayerSet([L.desc for L in layers])
    for call in range(3):
        for po in pos:
            po.y.fill_(float("nan"))
        if call < 2:
            grp.lowrank(x)
            sh_o._lowrank(x_o)
            hs = [grp.h_of(j, T) for j in range(3)] + [sh_o.h_address(T)]
        else:  # the four x*B^T products as one launch of the layer set
            lset.lowrank(xs)
            hs = lset.h_addresses(xs)
        launched = start_set_peers(layers, xs, pos, hs, pos[0])
        finish_set_peers(pos[0], launched)
        for j, (po, ref) in enumerate(zip(pos, wants)):
            err = float((po.y.float() - ref.float()).abs().nan_to_num(float("inf")).max())
            ok = err == 0.0
            bad += 0 if ok else 1
            print(f"rank {rank}/{world} set peers call {call} cfg4[{j}] T={T} max|diff|={err:.3e} "
                  f"{'ok' if ok else 'MISMATCH'}", flush=True)
    torch.cuda.synchronize()
    dist.barrier()
    for po in pos:
        po.close()
    return bad


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    bad = 0
    cases = [("cfg4", 0, 1024), ("cfg4", 6, 300), ("cfg3", 4, 16), ("cfg3", 0, 2048), ("cfg5", 0, 1)]
    for cfg, idx, T in cases:
        s = workloads.layer_set(cfg)[idx]
        t = s.tensors(dev, torch.bfloat16)
        x = workloads.tokens(T, s.in_features, seed=3, device=dev, dtype=torch.bfloat16)
        order = torch.from_numpy(ops.plan_row_order(s.crow.astype(np.int32))).to(dev)
        full = ops.LayerDesc(A=t["A"], B=t["B"], bias=t["bias"], crow=t["S_crow"], col=t["S_col"],
                             values=t["S_values"], row_order=order, in_features=s.in_features,
                             out_features=s.out_features, block_p=s.block_p, block_q=s.block_q)
        ref = full.forward(x)
        errs = []
        for split in (False, True):
            sh = ShardedLayer(t, s.crow, in_features=s.in_features, out_features=s.out_features,
                              block_p=s.block_p, block_q=s.block_q, rank=rank, world=world, split_lowrank=split)
            y = sh.forward(x)
            torch.cuda.synchronize()
            errs.append(float((y.float() - ref.float()).abs().max()))
        err = max(errs)
        scale = float(ref.float().pow(2).mean().sqrt())
        ok = err <= 1e-6 * max(scale, 1.0)
        bad += 0 if ok else 1
        print(f"rank {rank}/{world} {cfg}[{idx}] T={T} bounds={sh.bounds.tolist()} max|diff|={err:.3e} "
              f"{'ok' if ok else 'MISMATCH'}", flush=True)
    # q/k/v shards of cfg4 as one group per rank, x*B^T split by tokens + all-gather of H
    T = 1024
    specs = workloads.layer_set("cfg4")[:3]
    x = workloads.tokens(T, specs[0].in_features, seed=5, device=dev, dtype=torch.bfloat16)
    shards, refs = [], []
    for s in specs:
        t = s.tensors(dev, torch.bfloat16)
        order = torch.from_numpy(ops.plan_row_order(s.crow.astype(np.int32))).to(dev)
        full = ops.LayerDesc(A=t["A"], B=t["B"], bias=t["bias"], crow=t["S_crow"], col=t["S_col"],
                             values=t["S_values"], row_order=order, in_features=s.in_features,
                             out_features=s.out_features, block_p=s.block_p, block_q=s.block_q)
        refs.append(full.forward(x))
        shards.append(ShardedLayer(t, s.crow, in_features=s.in_features, out_features=s.out_features,
                                   block_p=s.block_p, block_q=s.block_q, rank=rank, world=world))
    grp = ops.LayerGroup([sh.desc for sh in shards])
    tp = T // world
    h = grp.lowrank_rows(x, rank * tp, tp)
    rb = tp * grp.h_row_bytes()
    dist.all_gather_into_tensor(h, h[rank * rb:(rank + 1) * rb])
    for j, (sh, ref) in enumerate(zip(shards, refs)):
        buf = sh.local_buffer(T)
        grp.combine(j, x, buf[rank][:, :sh.width])
        dist.all_gather_into_tensor(buf.view(-1), buf[rank].view(-1))
        y = sh.finish((None, buf))
        err = float((y.float() - ref.float()).abs().max())
        ok = err == 0.0
        bad += 0 if ok else 1
        print(f"rank {rank}/{world} grouped split-H cfg4[{j}] T={T} max|diff|={err:.3e} "
              f"{'ok' if ok else 'MISMATCH'}", flush=True)
    # the same group with every combine storing into all ranks' y (peer memory)
    from s_salaad_b200.shard import PeerOutputs, all_ranks
    if all_ranks(all(sh.peers_supported(x) for sh in shards), dev):
        pos = [PeerOutputs(sh, T, torch.bfloat16, dev) for sh in shards]
        grp.lowrank(x)
        for j, po in enumerate(pos):
            grp.combine_peers(j, x, po)
        for j, (sh, po, ref) in enumerate(zip(shards, pos, refs)):
            y = sh.finish_peers(po)
            err = float((y.float() - ref.float()).abs().max())
            ok = err == 0.0
            bad += 0 if ok else 1
            print(f"rank {rank}/{world} grouped peers cfg4[{j}] T={T} max|diff|={err:.3e} "
                  f"{'ok' if ok else 'MISMATCH'}", flush=True)
        torch.cuda.synchronize()
        dist.barrier()
        for po in pos:
            po.close()
    else:
        print(f"rank {rank}/{world} grouped peers: not supported on every rank", flush=True)
        bad += 1
    bad += check_set_peers(rank, world, dev, x, grp, shards, refs)
    bad += check_peer_outputs(rank, world, dev)
    flag = torch.tensor([bad], device=dev)
    dist.all_reduce(flag)
    dist.barrier()
    dist.destroy_process_group()
    return 0 if int(flag.item()) == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
