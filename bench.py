#!/usr/bin/env python
"""S+LR linear forward benchmark (B200).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg4|cfg3-T<T>|cfg5-T<T>|cfg1|cfg2|cfg2-model]

Prints ONE JSON line (rank 0).  A step is one forward of the workload's
layer set over one batch of T synthetic tokens:

* cfg4 (default): the seven projections of a LLaMA-7B-shaped decoder layer
  (q/k/v/o 4096x4096, gate/up 11008x4096, down 4096x11008), 64x64 blocks,
  20% of blocks with Zipf(1.1) skew over block-rows, rank 512, T = 4096
  tokens, bf16.  q/k/v read one input, gate/up another, as in the model.

`value` is whole-job tokens/s with inputs resident in HBM (device time from
CUDA events, L2 flushed between steps, max over ranks).  `e2e` is the same
through the public API with pinned host inputs copied in and every output
copied back inside the timed region.  At N > 1 every projection is
block-row sharded over the ranks and y is all-gathered (NCCL), so the total
work is fixed (strong scaling).  `--impl reference` times the reference's
CPU implementation of the path (its AVX2 BSR kernel, compiled from the
reference sources into oracle/_ref, plus the low-rank F.linear calls and the
bias, in fp32) on this host's cores over the same token batch.
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

_RESULT_FD = 1


def small_kernel_shape(s) -> tuple[int, int]:
    """Kernel instance of a layer's small-batch combine (x sub-tile width, rank
    chunk): layers of a group that agree run as one launch below 128 tokens."""
    bq = s.block_q if s.nnz > 0 else 16
    return min(bq, 64), (64 if s.rank >= 64 else 32 if s.rank >= 32 else 16)


def multi_launches(specs) -> int:
    """Launches of one multi-input call over `specs` below 128 tokens: one
    x*B^T launch, then one combine launch when every layer has a rank and the
    same small-batch kernel shape, else one per layer (a layer without rank
    sends every layer through its own forward)."""
    if any(s.rank <= 0 for s in specs):
        return sum(2 if s.rank > 0 else 1 for s in specs)
    return 1 + (1 if len({small_kernel_shape(s) for s in specs}) == 1 else len(specs))


def emit(line: dict) -> None:
    """Write the one JSON result line to the original stdout."""
    os.write(_RESULT_FD, (json.dumps(line) + "\n").encode())


METRIC = "S+LR linear tokens/s + %HBM/TC roofline at 1/2/4/8 B200 vs AVX2 CPU & cuBLAS"
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of the
# kernel the roofline covers, from one ncu capture of
# `bench.py --ncu --workload <w> --steps 1 --warmup 3` on a B200 with
# `--metrics dram__bytes_read.sum,dram__bytes_write.sum,gpu__time_duration.sum`:
# cfg4 and cfg3-T2048 = the one combine launch of the layer set (third launch
# of the process, `-k regex:tc2_rowblock -s 2 -c 1`); cfg3-T1 = the whole
# layer set of one step (its roofline covers the graph-replayed layer set).
NCU_TRAFFIC = {"cfg3-T1": 50881280.0, "cfg4": 1001.91e6, "cfg3-T2048": 144.76e6}
# SMs kept free of the persistent kernels at N > 1 (for the overlapping NCCL
# all-gathers); SLR_BENCH_NCCL_SMS overrides it.
SMS_FOR_NCCL = int(os.environ.get("SLR_BENCH_NCCL_SMS", "16"))
# N > 1: combine epilogues store y straight into every rank's y (peer memory)
# when every rank's kernels support it; 0 = NCCL all-gather of y instead
USE_PEERS = os.environ.get("SLR_BENCH_PEERS", "1") != "0"
# ... and then all projections' combines in one launch of the 2-SM kernel; 0 = one launch each
SET_PEERS = os.environ.get("SLR_BENCH_SET_PEERS", "1") != "0"
# N >= 4: x*B^T of a group split by tokens over the ranks + NCCL all-gather of H (1); the
# default computes it whole on every rank, which measured faster (cfg4, 4 x B200: 0.19 against
# 0.35 ms per step: the collective's latency exceeds the GEMM time it saves)
SPLIT_H = os.environ.get("SLR_BENCH_SPLIT_H", "0") == "1"
L2_FLUSH_BYTES = 256 << 20  # > 126 MB L2


def flush_l2(buf: torch.Tensor) -> None:
    """Evict L2 between timed steps: write a buffer twice the L2 size, then
    read it back, so every line the write left dirty is written back before
    the next step (a write alone leaves ~126 MB of dirty lines whose
    write-back would compete with the step's reads)."""
    buf.zero_()
    buf.sum(dtype=torch.int32)


# ------------------------------------------------------------ workloads --

def parse_workload(name: str) -> tuple[str, int]:
    from s_salaad_b200 import workloads

    if "-T" in name:
        cfg, t = name.split("-T")
        return cfg, int(t)
    return name, workloads.CFG_TOKENS[name][0]


def input_roles(specs) -> list[int]:
    """Index of the shared input each projection reads (q/k/v share one,
    gate/up share one, as in a decoder layer); singletons otherwise."""
    roles, seen = [], {}
    for s in specs:
        key = {"q_proj": "attn", "k_proj": "attn", "v_proj": "attn", "gate_proj": "mlp",
               "up_proj": "mlp"}.get(s.name.rsplit(".", 1)[-1], s.name)
        if key not in seen:
            seen[key] = len(seen)
        roles.append(seen[key])
    return roles


def peaks() -> tuple[dict, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.is_file():
        return json.loads(p.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# --------------------------------------------------------------- clocks --

class ClockSampler:
    """Polls the SM clock, max clock and clock-event (throttle) reasons in a
    thread while the timed region runs: through NVML, or `nvidia-smi` when
    NVML cannot be initialised; one sample is always taken as the region
    starts and one as it ends, so a short region still has a record."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, index: int):
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self.index = index
        self._stop = threading.Event()
        self._thread = None
        self.nv = None
        for _ in range(2):
            try:
                import pynvml

                pynvml.nvmlInit()
                self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
                self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
                self.nv = pynvml
                break
            except Exception:  # noqa: BLE001 - clocks are best effort
                time.sleep(0.05)
        self.smi = self.nv is None and shutil.which("nvidia-smi") is not None

    def _sample(self) -> None:
        try:
            if self.nv is not None:
                mhz = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                rs = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            elif self.smi:
                out = subprocess.run(["nvidia-smi", "-i", str(self.index), "--format=csv,noheader,nounits",
                                      "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active"],
                                     capture_output=True, text=True, timeout=5).stdout.strip().split(",")
                mhz, self.max_mhz, rs = int(out[0]), int(out[1]), int(out[2].strip(), 16)
            else:
                return
            self.samples.append((mhz, rs))
        except Exception:  # noqa: BLE001
            pass

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(0.002)

    def __enter__(self):
        self._sample()
        if self.nv is not None or self.smi:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join()
        self._sample()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        mhz = [m for m, _ in self.samples]
        bits = 0
        for _, r in self.samples:
            bits |= r
        return {"sm_mhz": float(statistics.median(mhz)), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(n for b, n in self.REASONS.items() if bits & b), "samples": len(mhz)}


# ---------------------------------------------------------- CPU leg --

def cpu_reference_run(specs, T_sample: int, steps: int, warmup: int, budget_s: float | None):
    """Time the reference CPU path (AVX2 kernel from oracle/_ref + MKL
    F.linear + bias, fp32) on T_sample tokens through the layer set.
    Returns (seconds per sample, kind, cores, CPU model name)."""
    sys.path.insert(0, str(REPO / "oracle"))
    import slr_oracle  # noqa: E402  (CPU baseline leg)

    cores = slr_oracle.max_threads()
    cpu_model = cpu_model_name()
    torch.set_num_threads(cores)
    mod = slr_oracle.ref_avx2_module()
    kind = "reference" if mod is not None else "port"
    from s_salaad_b200 import workloads

    layers = []
    for s in specs:
        t = s.tensors("cpu", torch.float32)
        x = workloads.tokens(T_sample, s.in_features, seed=7)
        layers.append((t, x))

    def one():
        for t, x in layers:
            if mod is not None:
                slr_oracle.lrs_forward_f32_ref_kernel(x, t["A"], t["B"], t["S_crow"], t["S_col"], t["S_values"],
                                                      t["S_active_rows"], t["bias"], mod=mod)
            else:
                slr_oracle.lrs_forward_f32(x, t["A"], t["B"], t["S_crow"], t["S_col"], t["S_values"],
                                           t["S_active_rows"], t["bias"])

    for _ in range(max(warmup, 1)):
        one()
    times = []
    t_end = None if budget_s is None else time.perf_counter() + budget_s
    while True:
        t0 = time.perf_counter()
        one()
        times.append(time.perf_counter() - t0)
        if budget_s is None and len(times) >= steps:
            break
        if budget_s is not None and (time.perf_counter() > t_end and len(times) >= 3):
            break
    if kind == "port":
        cores = 1
    return times, kind, cores, cpu_model


def cpu_model_name() -> str:
    """The host CPU's model name (what lscpu reports), from /proc/cpuinfo."""
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ---------------------------------------------------------------- main --

DECODE_POINTS = ("cfg3-T1", "cfg3-T16", "cfg5-T1", "cfg5-T32")


def graph_ms(fn, dev, steps: int, warmup: int, flush: torch.Tensor) -> float:
    """Mean device time of `fn` replayed from a CUDA graph, L2 flushed
    between replays (outside the events)."""
    side = torch.cuda.Stream(dev)
    cur = torch.cuda.current_stream(dev)
    side.wait_stream(cur)
    with torch.cuda.stream(side):
        for _ in range(max(warmup, 1)):
            fn()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            fn()
    cur.wait_stream(side)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize(dev)
    mk = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    ev = [(mk(), mk()) for _ in range(steps)]
    for a, b in ev:
        flush_l2(flush)
        a.record(cur)
        graph.replay()
        b.record(cur)
    torch.cuda.synchronize(dev)
    return sum(a.elapsed_time(b) for a, b in ev) / steps


def decode_points(dev, steps: int, warmup: int, flush: torch.Tensor, hbm_gbs: float) -> dict:
    """The decode-sized workloads (HBM-bound) on one GPU, each as
    * the whole projection set as one call (the inputs are independent in the
      layer set): x·Bᵀ of every layer in one launch, the combines in another;
    * `model_order`: per input group, in decoder order (q/k/v grouped, o,
      gate/up grouped, down), as a model that chains them would call them;
    * `single_launch_kernel`: both again on the opt-in single-launch decode
      kernel (x·Bᵀ and the combine of a call in one launch).
    Algorithmic bytes: weights and indices of every projection plus x and y
    (2 bytes per element); frac = achieved / measured HBM peak."""
    from s_salaad_b200 import ops, workloads

    out = {}
    for name in DECODE_POINTS:
        cfg, T = parse_workload(name)
        specs = workloads.layer_set(cfg)
        roles = input_roles(specs)
        layers = []
        for s in specs:
            t = s.tensors(dev, torch.bfloat16)
            order = torch.from_numpy(ops.plan_row_order(s.crow.astype(np.int32))).to(dev)
            layers.append(ops.LayerDesc(A=t["A"], B=t["B"], bias=t["bias"], crow=t["S_crow"], col=t["S_col"],
                                        values=t["S_values"], row_order=order, in_features=s.in_features,
                                        out_features=s.out_features, block_p=s.block_p, block_q=s.block_q))
        xin = {}
        for i, s in enumerate(specs):
            xin.setdefault(roles[i], workloads.tokens(T, s.in_features, seed=100 + roles[i], device=dev,
                                                      dtype=torch.bfloat16))
        xs = [xin[roles[i]] for i in range(len(specs))]
        ys = [torch.empty(T, s.out_features, dtype=torch.bfloat16, device=dev) for s in specs]
        lset = ops.LayerSet(layers)
        members: dict[int, list[int]] = {}
        for i, r in enumerate(roles):
            members.setdefault(r, []).append(i)
        groups = {r: ops.LayerGroup([layers[i] for i in idx]) for r, idx in members.items() if len(idx) > 1}

        def chained():
            for r, idx in members.items():
                if r in groups:
                    groups[r].forward(xs[idx[0]], [ys[i] for i in idx])
                else:
                    for i in idx:
                        layers[i].forward(xs[i], ys[i])

        nbytes = sum(s.weight_bytes(2) + 2 * T * (s.in_features + s.out_features) for s in specs)
        ms = graph_ms(lambda: lset.forward(xs, ys), dev, steps, warmup, flush)
        ms_chain = graph_ms(chained, dev, steps, warmup, flush)
        single = None
        if ops.decode_supported(layers, xs):
            with ops.single_launch_decode(True):
                ms_one = graph_ms(lambda: lset.forward(xs, ys), dev, steps, warmup, flush)
                ms_one_chain = graph_ms(chained, dev, steps, warmup, flush)
            single = {"ms_per_step": ms_one, "frac": nbytes / (ms_one / 1e3) / 1e9 / hbm_gbs, "launches": 1,
                      "model_order": {"ms_per_step": ms_one_chain,
                                      "frac": nbytes / (ms_one_chain / 1e3) / 1e9 / hbm_gbs,
                                      "launches": len(members)}}
        gbs, gbs_chain = nbytes / (ms / 1e3) / 1e9, nbytes / (ms_chain / 1e3) / 1e9
        out[name] = {"ms_per_step": ms, "tokens_per_s": T / (ms / 1e3), "algorithmic_bytes": nbytes,
                     "achieved_gbs": gbs, "frac": gbs / hbm_gbs, "launches": multi_launches(specs),
                     "model_order": {"ms_per_step": ms_chain, "achieved_gbs": gbs_chain, "frac": gbs_chain / hbm_gbs},
                     "single_launch_kernel": single}
        del layers, lset, groups, xs, ys, xin
        torch.cuda.empty_cache()
    return out


def generation_bench(model, dense, vocab: int, dev, batch: int = 8, prompt: int = 128, new: int = 64) -> dict:
    """Greedy generation tokens/s (new tokens per second over the batch),
    eager (the KV cache grows each step), timed with CUDA events around the
    whole call: the KV-cached loop on the S+LR model (decode kernels), the
    same loop on the dense bf16 model, and the reference's loop (the whole
    prefix recomputed each step) on the S+LR model over fewer tokens."""
    from s_salaad_b200.inference import generate, generate_no_cache

    g = torch.Generator(device="cpu").manual_seed(11)
    ids = torch.randint(0, vocab, (batch, prompt), generator=g).to(dev)

    def rate(fn, m, n) -> float:
        fn(m, ids, n)  # warm-up over the same lengths (attention set-up per KV length is paid here)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        fn(m, ids, n)
        b.record()
        torch.cuda.synchronize()
        return batch * n / (a.elapsed_time(b) / 1e3)

    return {"unit": "new tokens/s", "batch": batch, "prompt": prompt, "new_tokens": new,
            "kv_cache_slr": rate(generate, model, new), "kv_cache_dense_bf16": rate(generate, dense, new),
            "no_cache_slr_reference_loop": rate(generate_no_cache, model, 16),
            "what": "greedy decoding, eager steps; the reference loop recomputes the prefix each step "
                    "(measured over 16 new tokens)"}


def nm_points(dev, steps: int, warmup: int, flush: torch.Tensor, peaks_: dict) -> dict:
    """The N:M 2:4 + low-rank layer (the reference's other compressed-layer
    kind) on a LLaMA-7B-shaped MLP projection: 11008 x 4096, S 2:4 (the 2
    largest of N(0, 0.02) in every group of 4), rank 512, bf16, at a decode
    and a prefill token count (below 256 tokens the mma.sp kernel, from 256
    S unpacked into dense blocks on the tensor-core combine, the unpacking
    inside the timed call); each beside dense cuBLAS on W = A*B + S, both
    replayed from a CUDA graph with L2 flushed between replays.  Decode: HBM
    roofline on the algorithmic bytes (S values + metadata, A, B, bias, x, y).
    Prefill: FLOP rate on 2*T*(N*K/2 + r*(N+K)) against the measured dense
    bf16 peak."""
    from s_salaad_b200 import workloads
    from s_salaad_b200.efficient import LRSLinear

    n, k, r = 11008, 4096, 512
    g = torch.Generator(device="cpu").manual_seed(24)
    R = torch.randn(n, k, generator=g) * 0.02
    grp = R.view(n, k // 4, 4)
    keep = torch.zeros_like(grp, dtype=torch.bool).scatter_(-1, grp.abs().topk(2, dim=-1).indices, True)
    S = torch.where(keep, grp, torch.zeros_like(grp)).view(n, k).to(dev, torch.bfloat16)
    A = (torch.randn(n, r, generator=g) * (0.02 / 8)).to(dev, torch.bfloat16)
    B = (torch.randn(r, k, generator=g) * (0.02 / 8)).to(dev, torch.bfloat16)
    bias = (torch.randn(n, generator=g) * 0.01).to(dev, torch.bfloat16)
    layer = LRSLinear(A, B, S, in_features=k, out_features=n, bias=bias, nm_n=2, nm_m=4)
    W = (A.float() @ B.float() + S.float()).to(torch.bfloat16)
    out = {}
    for T in (1, 4096):
        x = workloads.tokens(T, k, seed=T, device=dev, dtype=torch.bfloat16)
        y = torch.empty(T, n, device=dev, dtype=torch.bfloat16)
        ms = graph_ms(lambda: layer(x), dev, steps, warmup, flush)
        ms_dense = graph_ms(lambda: torch.addmm(bias, x, W.t(), out=y), dev, steps, warmup, flush)
        point = {"ms": ms, "tokens_per_s": T / (ms / 1e3), "cublas_dense_ms": ms_dense}
        if T <= 16:
            nbytes = 2 * n * (k // 2) + 4 * n * (k // 32) + 2 * r * (n + k) + 2 * n + 2 * T * (k + n)
            point.update({"algorithmic_bytes": nbytes, "achieved_gbs": nbytes / (ms / 1e3) / 1e9,
                          "frac": nbytes / (ms / 1e3) / 1e9 / peaks_["hbm_gbs"], "bound": "hbm"})
        else:
            fl = 2 * T * (n * k // 2 + r * (n + k))
            point.update({"algorithmic_flops": fl, "achieved_tflops": fl / (ms / 1e3) / 1e12,
                          "frac": fl / (ms / 1e3) / 1e12 / peaks_["bf16_tflops"], "bound": "tensor (dense peak)"})
        out[f"T{T}"] = point
        del x, y
    return {"shape": [n, k], "rank": r, "sparsity": "2:4 along K",
            "kernel": {"T1": "mma.sp (m16n8k32) + mma.sync, one fused launch after x*B^T",
                       "T4096": "S unpacked per call into full-density 64x64 blocks, then x*B^T and the 2-SM "
                                "tcgen05 combine (the block-sparse layer's kernels)"},
            "points": out}


def model_bench(args) -> None:
    """cfg2 as a whole model: the 8-layer LLaMA-60M-shaped model of a
    synthetic bundle, loaded by build_efficient_model (every projection an
    S+LR layer, q/k/v and gate/up grouped), forward on batch 8 x 256 tokens
    replayed from a CUDA graph; the same model with dense bf16 weights
    (cuBLAS) beside it.  One GPU, no reference arm (the reference's CPU model
    forward is not a kernel comparison)."""
    import tempfile

    from s_salaad_b200 import workloads
    from s_salaad_b200.efficient import build_efficient_model, build_model_from_config, load_artifact

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    batch, seq = 8, 256
    with tempfile.TemporaryDirectory() as d:
        path = Path(d) / "cfg2.pt"
        dense = workloads.compressed_bundle(path, n_layers=8)
        model, config, _ = build_efficient_model(path, device=dev)
        payload = load_artifact(path)
        ref = build_model_from_config(payload["model_config"], attn_implementation="sdpa")
        ref.load_state_dict(payload["base_state_dict"], strict=False)
        with torch.no_grad():
            for name, W in dense.items():
                ref.get_submodule(name).weight.copy_(W)
        ref = ref.to(device=dev, dtype=torch.bfloat16).eval()
    g = torch.Generator(device="cpu").manual_seed(0)
    ids = torch.randint(0, config["vocab_size"], (batch, seq), generator=g).to(dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    mk = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731

    def timed(m) -> float:
        with torch.no_grad():
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                for _ in range(args.warmup):
                    m(ids)
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=side):
                    m(ids)
            torch.cuda.current_stream(dev).wait_stream(side)
            for _ in range(3):
                graph.replay()
            torch.cuda.synchronize()
            ev = [(mk(), mk()) for _ in range(args.steps)]
            for a, b in ev:
                flush_l2(flush)
                a.record()
                graph.replay()
                b.record()
            torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in ev) / args.steps

    with ClockSampler(0) as clocks:
        ms = timed(model)
    ms_dense = timed(ref)
    gen = generation_bench(model, ref, config["vocab_size"], dev)
    emit({"metric": "compressed LLaMA-60M-shaped model forward tokens/s (cfg2, whole model)",
          "value": batch * seq / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
          "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
          "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded bundle; random ids)",
          "config": {"workload": "cfg2-model: 8 decoder layers, 56 S+LR projections (16x16 blocks, 50 %, r 64), "
                                 "batch 8 x seq 256, forward replayed from a CUDA graph",
                     "l2": "flushed between timed steps (256 MB written, then read back)"},
          "dense_bf16": {"ms_per_step": ms_dense, "value": batch * seq / (ms_dense / 1e3),
                         "what": "the same model with dense W = A*B + S (torch/cuBLAS), same graph replay"},
          "generate": gen,
          "clocks": clocks.summary()})


def main() -> None:
    # Only the result line goes to stdout: libraries (NCCL, torch) may print
    # there, so fd 1 points at stderr for the run and the line is written to
    # the saved original stdout.
    out_fd = os.dup(1)
    os.dup2(2, 1)
    sys.stdout = os.fdopen(os.dup(2), "w")
    global _RESULT_FD
    _RESULT_FD = out_fd
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="cfg4")
    ap.add_argument("--cpu-sample-tokens", type=int, default=0)
    ap.add_argument("--cpu-budget-s", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-cublas", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="skip the decode points of the headline run")
    ap.add_argument("--decode-kernel", action="store_true",
                    help="calls of 1..32 tokens take the opt-in single-launch decode kernel")
    ap.add_argument("--ncu", action="store_true",
                    help="profiling mode: warm-up + timed steps only (no e2e, cuBLAS or CPU legs)")
    args = ap.parse_args()
    if args.ncu:
        args.no_cublas = args.no_cpu_baseline = args.no_decode = True
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3

    from s_salaad_b200 import ops, workloads

    if args.decode_kernel:
        ops._single_launch = True  # the process's calls of 1..32 tokens: ops.single_launch_decode(True)
    if args.workload == "cfg2-model":
        return model_bench(args)
    cfg, T = parse_workload(args.workload)
    specs = workloads.layer_set(cfg)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    # the CPU legs run the workload's full token batch unless a sample is asked for
    T_sample = args.cpu_sample_tokens or T
    config = {"workload": f"{cfg}: {len(specs)} S+LR projections, T={T}",
              "tokens_per_step": T, "projections": [[s.name, s.out_features, s.in_features] for s in specs],
              "block": [specs[0].block_p, specs[0].block_q], "rank": specs[0].rank,
              "nnz_blocks": sum(s.nnz for s in specs)}

    # ------------------------------------------------ reference (CPU) arm
    if args.impl == "reference":
        if rank != 0:
            return
        times, kind, cores, model = cpu_reference_run(specs, T_sample, args.steps, args.warmup, None)
        tok_s = T_sample * len(times) / sum(times)
        line = {"metric": METRIC, "impl": "reference", "value": tok_s, "unit": "tokens/s", "n_gpus": world,
                "steps": len(times), "warmup": args.warmup, "ms_per_step": 1e3 * statistics.mean(times),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded; no dataset)",
                "config": {**config, "parallelism": "host threads (CPU)"},
                "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": cores, "kind": kind, "cpu_model": model,
                                 "sample": f"{T_sample} of {T} tokens per step through all {len(specs)} projections"},
                "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        emit(line)
        return

    # ------------------------------------------------------------ our arm
    import torch.distributed as dist

    from s_salaad_b200 import ops
    from s_salaad_b200.shard import PeerOutputs, ShardedLayer, all_ranks

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
        # y all-gathers on their own communicator so they overlap the small H exchanges and kernels
        group_y = dist.new_group(list(range(world)))
    dtype = torch.float32 if cfg == "cfg1" else torch.bfloat16
    esize = 4 if dtype == torch.float32 else 2

    layers, tens = [], []
    for s in specs:
        t = s.tensors(dev, dtype)
        tens.append(t)
        if world > 1:
            layers.append(ShardedLayer(t, s.crow, in_features=s.in_features, out_features=s.out_features,
                                       block_p=s.block_p, block_q=s.block_q, rank=rank, world=world,
                                       group=group_y, group_h=None))
        else:
            order = torch.from_numpy(ops.plan_row_order(s.crow.astype(np.int32))).to(dev)
            layers.append(ops.LayerDesc(A=t["A"], B=t["B"], bias=t["bias"], crow=t["S_crow"], col=t["S_col"],
                                        values=t["S_values"], row_order=order, in_features=s.in_features,
                                        out_features=s.out_features, block_p=s.block_p, block_q=s.block_q))
    roles = input_roles(specs)
    xin = {}
    for i, s in enumerate(specs):
        if roles[i] not in xin:
            xin[roles[i]] = workloads.tokens(T, s.in_features, seed=100 + roles[i], device=dev, dtype=dtype)
    xs = [xin[roles[i]] for i in range(len(specs))]
    # projections that read one x (q/k/v, gate/up) run as one grouped call on
    # one GPU: their x*B^T products are a single GEMM
    members: dict[int, list[int]] = {}
    for i, r in enumerate(roles):
        members.setdefault(r, []).append(i)
    groups = {}
    if world == 1:
        groups = {r: ops.LayerGroup([layers[i] for i in idx]) for r, idx in members.items() if len(idx) > 1}
    else:
        # each rank's shards of q/k/v (gate/up) read the whole x and keep all of B: one grouped x*B^T,
        # computed for this rank's 1/world of the tokens and all-gathered (a few MB)
        groups = {r: ops.LayerGroup([layers[i].desc for i in idx]) for r, idx in members.items()
                  if all(layers[i].desc is not None for i in idx)}
    pos = None
    if world > 1 and USE_PEERS and all_ranks(all(L.peers_supported(xs[i]) for i, L in enumerate(layers)), dev):
        pos = [PeerOutputs(L, T, dtype, dev) for L in layers]
    elif world > 1:
        # leave SMs to the NCCL all-gathers that overlap the next projections' kernels
        from s_salaad_b200 import _lib
        _lib.load().slr_set_sm_limit(_lib.load_sm_count() - SMS_FOR_NCCL)
    # N > 1 with peer outputs: the combines of all projections in one launch of
    # the 2-SM kernel (one signal slot, one wait) when they share its shape
    set_peers = (pos is not None and SET_PEERS and T >= 256 and len(specs) <= 8
                 and all(s.nnz > 0 and s.block_p in (32, 64) and (s.block_p, s.block_q) ==
                         (specs[0].block_p, specs[0].block_q) for s in specs))
    if set_peers:
        from s_salaad_b200.shard import finish_set_peers, start_set_peers
    # ... and this rank's x*B^T of all projections in one launch (a layer set over its shards)
    mine = [i for i in range(len(specs)) if world > 1 and layers[i].desc is not None]
    pset = (ops.LayerSet([layers[i].desc for i in mine])
            if set_peers and not SPLIT_H and 1 <= len(mine) <= 8 else None)
    ys = ([po.y for po in pos] if pos is not None else
          [torch.empty(T, s.out_features, dtype=dtype, device=dev) for s in specs])
    # one GPU: the projections (independent inputs) run as one layer-set call
    # (slr_lrs_linear_forward_multi): below 128 tokens x*B^T of all of them in
    # one launch and the combines in another; from 128 tokens x*B^T per
    # projection and, on the pair kernel, the combines of all in one launch
    lset = ops.LayerSet(layers) if (world == 1 and dtype != torch.float32) else None
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step(ev=None):
        """One forward of the layer set; ev = per-projection event triples."""
        if world > 1 and pset is not None:
            xs_l = [xs[i] for i in mine]
            if ev is not None:
                ev[mine[0]][0].record(stream)
            pset.lowrank(xs_l)
            if ev is not None:
                # the set's x*B^T charged to its first projection, its combine to the same one
                for i in range(len(specs)):
                    if i != mine[0]:
                        ev[i][0].record(stream)
                    ev[i][1].record(stream)
                    if i != mine[0]:
                        ev[i][2].record(stream)
            hs = [None] * len(specs)
            for i, h in zip(mine, pset.h_addresses(xs_l)):
                hs[i] = h
            launched = start_set_peers(layers, xs, pos, hs, pos[0])
            if ev is not None:
                ev[mine[0]][2].record(stream)
            finish_set_peers(pos[0], launched)
            return
        if world > 1:
            handles = {}
            hs = [None] * len(specs)  # H of each projection (set_peers)
            tp = T // world
            for r, idx in members.items():
                grp = groups.get(r)
                if grp is not None:
                    if ev is not None:
                        ev[idx[0]][0].record(stream)
                    if SPLIT_H and world >= 4 and T % world == 0 and tp >= 128:
                        h = grp.lowrank_rows(xs[idx[0]], rank * tp, tp)
                        rb = tp * grp.h_row_bytes()
                        dist.all_gather_into_tensor(h, h[rank * rb:(rank + 1) * rb])
                    else:
                        grp.lowrank(xs[idx[0]])
                if set_peers:
                    # x*B^T only; the combines of all projections follow as one launch
                    for j, i in enumerate(idx):
                        L = layers[i]
                        if ev is not None and (grp is None or j):
                            ev[i][0].record(stream)
                        if grp is None and L.desc is not None:
                            L._lowrank(xs[i])
                        if ev is not None:
                            ev[i][1].record(stream)
                            ev[i][2].record(stream)
                        if L.desc is not None:
                            hs[i] = grp.h_of(j, T) if grp is not None else L.h_address(T)
                    continue
                for j, i in enumerate(idx):
                    L = layers[i]
                    if pos is not None:
                        # y tiles go straight into every rank's y; the waits end the step
                        if L.desc is None:
                            continue
                        if ev is not None and (grp is None or j):
                            ev[i][0].record(stream)
                        if grp is None:
                            L._lowrank(xs[i])
                        if ev is not None:
                            ev[i][1].record(stream)
                        if grp is None:
                            L.start_peers_combine(xs[i], pos[i])
                        else:
                            grp.combine_peers(j, xs[i], pos[i])
                        if ev is not None:
                            ev[i][2].record(stream)
                        continue
                    if L.desc is None:
                        handles[i] = L.start(xs[i])
                        continue
                    if ev is not None and (grp is None or j):
                        ev[i][0].record(stream)
                    if grp is None:
                        L._lowrank(xs[i])
                    if ev is not None:
                        ev[i][1].record(stream)
                    buf = L.local_buffer(T)
                    if grp is None:
                        L.desc.combine(xs[i], buf[rank][:, :L.width])
                    else:
                        grp.combine(j, xs[i], buf[rank][:, :L.width])
                    if ev is not None:
                        ev[i][2].record(stream)
                    work = dist.all_gather_into_tensor(buf.view(-1), buf[rank].view(-1), group=L.group,
                                                       async_op=True)
                    handles[i] = (work, buf)
            if set_peers:
                launched = start_set_peers(layers, xs, pos, hs, pos[0])
                if ev is not None:
                    # the set's combine, charged to the last projection (its x*B^T ended just before)
                    ev[len(specs) - 1][2].record(stream)
                finish_set_peers(pos[0], launched)
                return
            for i, L in enumerate(layers):
                if pos is not None:
                    L.finish_peers(pos[i])
                else:
                    L.finish(handles[i], ys[i])
            return
        if lset is not None:
            if ev is None:
                lset.forward(xs, ys)
            else:
                # the set's two phases, charged to its first projection
                ev[0][0].record(stream)
                lset.lowrank(xs)
                ev[0][1].record(stream)
                lset.combine(xs, ys)
                ev[0][2].record(stream)
            return
        step_roles(ev)

    def step_roles(ev=None):
        """One GPU: the projections per input, in a decoder's order (q/k/v
        grouped, o, gate/up grouped, down), as a model issues them."""
        for r, idx in members.items():
            grp = groups.get(r)
            if grp is None:
                for i in idx:
                    L = layers[i]
                    if ev is not None:
                        ev[i][0].record(stream)
                    L.lowrank(xs[i])
                    if ev is not None:
                        ev[i][1].record(stream)
                    L.combine(xs[i], ys[i])
                    if ev is not None:
                        ev[i][2].record(stream)
            elif ev is None:
                grp.forward(xs[idx[0]], [ys[i] for i in idx])
            else:
                # the group's x*B^T is charged to its first projection
                ev[idx[0]][0].record(stream)
                grp.lowrank(xs[idx[0]])
                for j, i in enumerate(idx):
                    if j:
                        ev[i][0].record(stream)
                    ev[i][1].record(stream)
                    grp.combine(j, xs[i], ys[i])
                    ev[i][2].record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    K = args.steps
    mk = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    # The step is captured once and replayed from a CUDA graph (NCCL
    # collectives included at N > 1), so host launch overhead (ctypes +
    # tensor-map encoding, ~15 us per call; ~30 us per NCCL call) is not timed.
    use_graph = True
    graph = None
    if use_graph:
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            step()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                step()
        stream.wait_stream(side)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    step_ev = [(mk(), mk()) for _ in range(K)]
    kern_ev = [[(mk(), mk(), mk()) for _ in specs] for _ in range(K)]
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        for k in range(K):
            flush_l2(flush)  # evict L2 between timed steps (outside the events)
            step_ev[k][0].record(stream)
            if graph is not None:
                graph.replay()
            else:
                step(kern_ev[k])
            step_ev[k][1].record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    step_ms = [a.elapsed_time(b) for a, b in step_ev]
    total_ms = sum(step_ms)
    has_local = [world == 1 or layers[i].desc is not None for i in range(len(specs))]
    if graph is not None and T >= 128:
        # Per-kernel durations for the roofline: the same steps once more,
        # eagerly, with events between the x*B^T and combine launches (these
        # kernels are long enough that the host stays ahead of the GPU).
        for k in range(K):
            flush_l2(flush)
            step(kern_ev[k])
        torch.cuda.synchronize()
    if lset is not None and T >= 128:
        h_ms = [sum(kern_ev[k][0][0].elapsed_time(kern_ev[k][0][1]) for k in range(K))] + [0.0] * (len(specs) - 1)
        c_ms = [sum(kern_ev[k][0][1].elapsed_time(kern_ev[k][0][2]) for k in range(K))] + [0.0] * (len(specs) - 1)
    elif graph is None or T >= 128:
        h_ms = [sum(kern_ev[k][i][0].elapsed_time(kern_ev[k][i][1]) for k in range(K)) if has_local[i] else 0.0
                for i in range(len(specs))]
        c_ms = [sum(kern_ev[k][i][1].elapsed_time(kern_ev[k][i][2]) for k in range(K)) if has_local[i] else 0.0
                for i in range(len(specs))]
    else:
        h_ms = [0.0] * len(specs)
        c_ms = [total_ms / len(specs)] * len(specs)
    t = torch.tensor([total_ms, sum(c_ms), sum(h_ms)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, comb_ms_max, low_ms_max = t.tolist()

    # combine launches of the layer-set call: one when every projection takes the
    # pair kernel (2-SM, block_p 32/64, 256+ tokens, column schedule, enough items)
    pair_set = lset is not None and T >= 256 and all(
        s.nnz > 0 and s.block_p in (32, 64)
        and -(-s.out_features // s.block_p // (256 // s.block_p)) * -(-T // 128) >= 16 for s in specs)
    comb_launches = 1 if (pair_set or set_peers) else len(specs)

    # ------------------------------------------------- roofline (combine)
    P, pk_src = peaks()
    comb_flops = comb_bytes = low_flops = 0
    for i, s in enumerate(specs):
        if world > 1:
            L = layers[i]
            if L.desc is None:
                continue
            crow = s.crow[L.bounds[rank]:L.bounds[rank + 1] + 1]
            nnz = int(crow[-1] - crow[0])
            N = L.width
        else:
            nnz, N = s.nnz, s.out_features
        NB = N // s.block_p
        comb_flops += 2 * T * (nnz * s.block_p * s.block_q + s.rank * N)
        comb_bytes += (esize * nnz * s.block_p * s.block_q + 4 * nnz + 8 * (NB + 1) + esize * s.rank * N
                       + esize * T * (s.in_features + s.rank + N))
        low_flops += 2 * T * s.rank * s.in_features
    tensor_bound = T >= 128
    comb_s = sum(c_ms) / 1e3
    if graph is not None and not tensor_bound:
        # whole layer set per graph replay: both kernels of every projection
        op_bytes = sum(s.weight_bytes(esize) + esize * T * (s.in_features + s.out_features) for s in specs)
        achieved = op_bytes * K / (total_ms / 1e3) / 1e9
        roof = {"bound": "hbm", "unit": "GB/s", "algorithmic_per_step": op_bytes,
                "kernel": "layer set from a CUDA graph: one multi-input call (x*B^T launch + combine launch) "
                          "over all projections"}
        peak = P["hbm_gbs"]
    elif tensor_bound:
        achieved = comb_flops * K / comb_s / 1e12
        peak = P["bf16_tflops"]
        roof = {"bound": "tensor", "unit": "TFLOP/s", "algorithmic_per_step": comb_flops,
                "kernel": ("combine (sparse + H*A^T + bias) of all projections of the set"
                           + (" in one launch of the 2-SM pair kernel" if (pair_set or set_peers)
                              else ", one launch each")
                           + (", tiles stored into every rank's y" if set_peers else ""))
                if (lset is not None or set_peers) else "combine (sparse + H*A^T + bias; one launch per projection)"}
    else:
        achieved = comb_bytes * K / comb_s / 1e9
        peak = P["hbm_gbs"]
        roof = {"bound": "hbm", "unit": "GB/s", "algorithmic_per_step": comb_bytes,
                "kernel": "combine (sparse + H*A^T + bias; one launch per projection)"}
    # captured on one GPU (full layers); a shard's launches move other byte counts
    traffic = NCU_TRAFFIC.get(args.workload) if world == 1 else None
    if tensor_bound:
        roof["step_tflops"] = (comb_flops + low_flops) * K / (total_ms / 1e3) / 1e12
    roof.update({"achieved": achieved, "peak": peak, "peak_source": pk_src,
                 "frac": achieved / peak, "traffic": traffic,
                 "combine_ms_per_step": sum(c_ms) / K, "combine_launches_per_step": comb_launches,
                 "lowrank_ms_per_step": sum(h_ms) / K,
                 "lowrank_tflops": low_flops * K / (sum(h_ms) / 1e3) / 1e12 if sum(h_ms) else None})

    value = T * K / (total_ms / 1e3)
    if args.ncu:
        if rank == 0:
            emit({"ncu_mode": True, "ms_per_step": total_ms / K, "roofline": roof})
        if world > 1:
            del graph  # a graph holding NCCL calls must go before the process group
            torch.cuda.synchronize()
            dist.barrier()
            for po in pos or []:
                po.close()
            dist.destroy_process_group()
        return
    launches_per_step = sum((1 if s.rank > 0 else 0) + 1 for i, s in enumerate(specs) if has_local[i])
    for r, grp in groups.items():  # one x*B^T launch per group
        launches_per_step -= len(members[r]) - 1
    if lset is not None:
        launches_per_step = multi_launches(specs) if T < 128 else len(members) + comb_launches
    if set_peers:
        launches_per_step += 1 - sum(1 for i in range(len(specs)) if has_local[i])  # one combine, not one each
    if pset is not None:
        launches_per_step = 2  # one x*B^T launch and one combine launch for the set
    if pos is not None:
        launches_per_step += 1 if set_peers else len(specs)  # the wait(s) that end the call(s)

    # ------------------------------------------------------------- e2e
    x_host = {r: xin[r].cpu().pin_memory() for r in xin}
    xin_dev = {r: torch.empty_like(xin[r]) for r in xin}
    y_host = [torch.empty(T, s.out_features, dtype=dtype).pin_memory() for s in specs]
    h2d = sum(v.numel() * v.element_size() for v in x_host.values())
    d2h = sum(v.numel() * v.element_size() for v in y_host) if rank == 0 else 0

    def e2e_step():
        if world > 1:
            # the timed step itself (shards, H exchange, y assembly), fed from host memory
            for r in xin:
                xin[r].copy_(x_host[r], non_blocking=True)
            step()
            if rank == 0:
                for i in range(len(specs)):
                    y_host[i].copy_(ys[i], non_blocking=True)
            return
        for r in xin:
            xin_dev[r].copy_(x_host[r], non_blocking=True)
        if lset is not None:
            lset.forward([xin_dev[roles[i]] for i in range(len(specs))], ys)
            if rank == 0:
                for i in range(len(specs)):
                    y_host[i].copy_(ys[i], non_blocking=True)
            return
        for r, idx in members.items():
            x_r = xin_dev[r]
            if r in groups:
                groups[r].forward(x_r, [ys[i] for i in idx])
            else:
                for i in idx:
                    layers[i].forward(x_r, ys[i])
            if rank == 0:
                for i in idx:
                    y_host[i].copy_(ys[i], non_blocking=True)

    if world == 1 and T >= 128:
        # Two steps in flight, as a server would run them: step k+1's inputs
        # cross PCIe on one copy stream while step k computes, and each
        # projection's y leaves on a second copy stream as soon as it is
        # written (H2D and D2H use separate copy engines).  Every step still
        # moves all of its inputs in and all of its outputs out; x and y are
        # larger than L2, so no flush is needed between steps.  (Decode-sized
        # steps are bound by host launch overhead, which the extra streams and
        # events would only add to: they run one after another below.)
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        xb = [{r: torch.empty_like(xin[r]) for r in xin} for _ in range(2)]
        yb = [[torch.empty_like(ys[i]) for i in range(len(specs))] for _ in range(2)]
        ev_in = [torch.cuda.Event() for _ in range(2)]    # inputs of buffer b landed
        ev_read = [torch.cuda.Event() for _ in range(2)]  # step on buffer b no longer reads x
        ev_out = [torch.cuda.Event() for _ in range(2)]   # outputs of buffer b copied out
        ev_y = [[torch.cuda.Event() for _ in specs] for _ in range(2)]

        def e2e_pipelined(k: int) -> None:
            b = k & 1
            if k >= 2:
                s_in.wait_event(ev_read[b])
            with torch.cuda.stream(s_in):
                for r in xin:
                    xb[b][r].copy_(x_host[r], non_blocking=True)
            ev_in[b].record(s_in)
            stream.wait_event(ev_in[b])
            if k >= 2:
                stream.wait_event(ev_out[b])
            for r, idx in members.items():
                if r in groups:
                    groups[r].forward(xb[b][r], [yb[b][i] for i in idx])
                else:
                    for i in idx:
                        layers[i].forward(xb[b][r], yb[b][i])
                for i in idx:
                    ev_y[b][i].record(stream)
            ev_read[b].record(stream)
            for i in range(len(specs)):
                s_out.wait_event(ev_y[b][i])
                with torch.cuda.stream(s_out):
                    y_host[i].copy_(yb[b][i], non_blocking=True)
            ev_out[b].record(s_out)

        for k in range(2):
            e2e_pipelined(k)
        torch.cuda.synchronize()
        t0, t1 = mk(), mk()
        t0.record(s_in)
        for k in range(K):
            e2e_pipelined(k)
        t1.record(s_out)
        torch.cuda.synchronize()
        e2e_ms = torch.tensor([t0.elapsed_time(t1)], device=dev, dtype=torch.float64)
    else:
        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        e2e_ev = [(mk(), mk()) for _ in range(K)]
        for k in range(K):
            flush_l2(flush)
            e2e_ev[k][0].record(stream)
            e2e_step()
            e2e_ev[k][1].record(stream)
        torch.cuda.synchronize()
        e2e_ms = torch.tensor([sum(a.elapsed_time(b) for a, b in e2e_ev)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_val = T * K / (e2e_ms.item() / 1e3)

    # ------------------------------------------------ cuBLAS dense (N=1)
    cublas = None
    if world == 1 and not args.no_cublas:
        Ws = []
        for s, tt in zip(specs, tens):
            W = (tt["A"].float() @ tt["B"].float())
            Wv = W.view(s.nb, s.block_p, s.in_features // s.block_q, s.block_q).permute(0, 2, 1, 3)
            rows = torch.from_numpy(np.repeat(np.arange(s.nb), np.diff(s.crow))).to(dev)
            cols = torch.from_numpy(s.col).to(dev)
            Wv[rows, cols] += tt["values_pq"].float()
            Ws.append(W.to(dtype))
            del W, Wv
        biases = [tt["bias"] for tt in tens]
        fl = torch.nn.functional.linear
        for _ in range(3):
            for i in range(len(specs)):
                fl(xs[i], Ws[i], biases[i])
        torch.cuda.synchronize()
        dev_ev = [(mk(), mk()) for _ in range(K)]
        for k in range(K):
            flush_l2(flush)
            dev_ev[k][0].record(stream)
            for i in range(len(specs)):
                torch.matmul(xs[i], Ws[i].T, out=ys[i]) if biases[i] is None else fl(xs[i], Ws[i], biases[i])
            dev_ev[k][1].record(stream)
        torch.cuda.synchronize()
        cb_ms = sum(a.elapsed_time(b) for a, b in dev_ev)
        dense_flops = sum(2 * T * s.out_features * s.in_features for s in specs)
        cublas = {"value": T * K / (cb_ms / 1e3), "unit": "tokens/s", "ms_per_step": cb_ms / K,
                  "tflops": dense_flops * K / (cb_ms / 1e3) / 1e12, "what": "torch F.linear (cuBLAS) on dense "
                  "W = A*B + S in bf16, same shapes and inputs"}
        del Ws

    # ------------------------------------- the same step in model order (N=1)
    model_order = None
    if world == 1 and lset is not None and T >= 128:
        mo_ms = graph_ms(step_roles, dev, K, args.warmup, flush)
        model_order = {"ms_per_step": mo_ms, "tokens_per_s": T / (mo_ms / 1e3),
                       "what": "the projections per input in a decoder's order (q/k/v grouped, o, gate/up grouped, "
                               "down), graph-replayed, L2 flushed between steps"}

    # ------------------------------------------- decode points (N=1 headline)
    decode = None
    nm24 = None
    if world == 1 and args.workload == "cfg4" and not args.no_decode:
        decode = decode_points(dev, max(K, 20), args.warmup, flush, P["hbm_gbs"])
        nm24 = nm_points(dev, max(K, 20), args.warmup, flush, P)

    # ------------------------------------------------------- CPU baseline
    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        times, kind, cores, model = cpu_reference_run(specs, T_sample, 0, 1, args.cpu_budget_s)
        cpu = {"value": T_sample * len(times) / sum(times), "unit": "tokens/s", "cores": cores, "kind": kind,
               "cpu_model": model,
               "sample": f"{T_sample} of {T} tokens x {len(times)} reps through all {len(specs)} projections, "
                         f"fp32 (reference AVX2 BSR kernel + MKL low-rank + bias)"}

    if rank == 0:
        all_flops = sum(s.flops_per_token() for s in specs) * T
        line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K,
                "warmup": args.warmup, "ms_per_step": total_ms / K, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "bf16" if dtype == torch.bfloat16 else "f32",
                "data": "synthetic (seeded generators; random-init weights; no dataset)",
                "config": {**config, "l2": "flushed between timed steps (256 MB written, then read back)",
                           "parallelism": (f"block-row shards x{world}, x*B^T "
                                           + ("split by tokens + NCCL all-gather of H" if (SPLIT_H and world >= 4)
                                              else "of all projections in one launch on every rank" if pset is not None
                                              else "on every rank")
                                           + ((", the combines of all projections in one launch whose epilogue "
                                               "stores y into every rank's y over NVLink (CUDA IPC)") if set_peers
                                              else ", combine epilogues store y into every rank's y over NVLink "
                                                   "(CUDA IPC)" if pos is not None else ", NCCL all-gather of y")
                                           + ", step replayed from a CUDA graph")
                           if world > 1 else ("1 GPU, the projections (independent inputs) as one layer-set call, "
                                              "step replayed from a CUDA graph"),
                           "algorithmic_tflop_per_step": all_flops / 1e12},
                "roofline": roof, "e2e": {"value": e2e_val, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                                          "d2h_bytes_per_step": d2h},
                "gpu_launches": launches_per_step * K, "clocks": clocks.summary(),
                "cpu_baseline": cpu, "cublas_dense": cublas}
        if model_order is not None:
            line["model_order"] = model_order
        if nm24 is not None:
            line["nm24"] = nm24
        if decode is not None:
            line["decode"] = {"what": "decode-sized layer sets on 1 GPU, each step replayed from a CUDA graph with L2 "
                                      "flushed between steps; roofline = algorithmic bytes (weights, indices, x, y) "
                                      "per step / time, against the measured HBM peak",
                              "peak_gbs": P["hbm_gbs"], "points": decode}
        emit(line)
    if world > 1:
        del graph  # a graph holding NCCL calls must go before the process group
        torch.cuda.synchronize()
        dist.barrier()
        for po in pos or []:
            po.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
