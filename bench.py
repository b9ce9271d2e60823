"""Benchmark of the FP8 hot path (BASELINE cfg3: per-block scaled FP8 BMM).

One step = quantize A (bf16 [b, 4096, 7168], 1x128 tiles) + quantize B (bf16
[b, 7168, 2048], 128x128 tiles) + the per-block scaled BMM -> bf16 C, for the
b = 32 / N batches this rank owns (the 32 batches are sharded across ranks,
no collective on the data path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Under torchrun (N > 1) every rank runs its shard; the timed region is
bracketed by a barrier and a device synchronize, and the max over ranks is
reported.  Rank 0 prints one JSON line.

* value      -- whole-job BMM TFLOP/s of the step (quant + BMM), inputs resident in HBM.
* e2e        -- the same metric through the public API (registry impls) with
                pinned HOST bf16 inputs copied in and bf16 C copied out every step.
* roofline   -- the BMM kernel: FLOPs per launch / its CUDA-event duration,
                against 2x the measured dense bf16 peak (FP8 dense).
* cpu_baseline -- the CPU oracle (reference's torch formulation) on one batch.
``--impl reference`` times that CPU path on all host cores (rank 0 only).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GLOBAL_B, M, K, N = 32, 4096, 7168, 2048
QA, QB = (1, 128), (128, 128)
FLOP_PER_BATCH = 2 * M * N * K
L2_BYTES = 126 * 1024 * 1024


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--batches", type=int, default=GLOBAL_B, help="global batch count (cfg3: 32)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["cfg3", "cfg5"], default="cfg3",
                    help="cfg3: per-block BMM step (default); cfg5: FSDP2 FP8 training step of the Llama decoder")
    ap.add_argument("--cfg5-linear", choices=["fp8_e8m0", "fp8", "bf16"], default="fp8_e8m0",
                    help="cfg5 only: per-block FP8 linears with power-of-two scales on the block-scaled "
                         "tensor-core GEMM (default), with the reference's fp32 scales (fp8), or the bf16 baseline")
    ap.add_argument("--layers", type=int, default=8, help="cfg5 only: decoder layers (BASELINE: 8)")
    ap.add_argument("--fp8-peak", action="store_true",
                    help="only measure the FP8 dense peak with torch._scaled_mm (cuBLASLt) at 8192^3")
    return ap.parse_args()


def measured_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def shard_range(total: int, rank: int, world: int) -> tuple[int, int]:
    from practice_cuda_b200.sharding import shard_range as sr

    return sr(total, rank, world)


# ------------------------------------------------------------------ clocks ---
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device_index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                smax.append(float(parts[1]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[3:7]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(smax) if smax else None,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


# ------------------------------------------------------------------ inputs ---
def make_inputs(b0: int, b1: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """Seeded synthetic cfg3 inputs for batches [b0, b1): A ~ N(0,1) with
    numel//1000 entries x100, B ~ N(0, 0.02), both bf16.  Generated per batch
    from seed (1000 + batch) on the device so every GPU count sees the same
    bytes for the same batch."""
    nb = b1 - b0
    a = torch.empty((nb, M, K), device=device, dtype=torch.bfloat16)
    b = torch.empty((nb, K, N), device=device, dtype=torch.bfloat16)
    for i in range(nb):
        g = torch.Generator(device=device).manual_seed(1000 + b0 + i)
        x = torch.randn((M, K), device=device, generator=g)
        flat = x.view(-1)
        idx = torch.randperm(flat.numel(), device=device, generator=g)[: flat.numel() // 1000]
        flat[idx] *= 100.0
        a[i].copy_(x)
        b[i].copy_(torch.randn((K, N), device=device, generator=g) * 0.02)
        del x, flat, idx
    return a, b


# ------------------------------------------------------------- CPU baseline ---
def cpu_sample_seconds() -> tuple[float, int, str]:
    """The oracle (reference's torch CPU formulation) on one cfg3 batch."""
    import oracle

    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    g = torch.Generator().manual_seed(1000)
    a = torch.randn((M, K), generator=g)
    flat = a.view(-1)
    idx = torch.randperm(flat.numel(), generator=g)[: flat.numel() // 1000]
    flat[idx] *= 100.0
    a = a.bfloat16()
    b = (torch.randn((K, N), generator=g) * 0.02).bfloat16()
    t0 = time.perf_counter()
    ya, sa = oracle.per_block_quant(a, block_m=QA[0], block_n=QA[1])
    yb, sb = oracle.per_block_quant(b, block_m=QB[0], block_n=QB[1])
    c = oracle.scaled_bmm_dequant_reference(
        ya.unsqueeze(0), sa.unsqueeze(0), "block", {"block_m": QA[0], "block_n": QA[1]},
        yb.unsqueeze(0), sb.unsqueeze(0), "block", {"block_m": QB[0], "block_n": QB[1]},
        out_dtype=torch.bfloat16)
    dt = time.perf_counter() - t0
    del c
    return dt, cores, "1 of 32 cfg3 batches: per-block quant A (1x128) + B (128x128), dequantize, fp32 bmm, bf16 cast"


def run_reference(args, rank: int) -> None:
    if rank != 0:
        return
    for _ in range(max(0, args.warmup)):
        cpu_sample_seconds()
    times = []
    cores, sample = 0, ""
    for _ in range(args.steps):
        dt, cores, sample = cpu_sample_seconds()
        times.append(dt)
    total = sum(times)
    value = FLOP_PER_BATCH * args.steps / total / 1e12
    line = {
        "impl": "reference",
        "metric": "fp8_bmm_tflops",
        "value": value,
        "unit": "TFLOP/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1000 * total / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "fp32",
        "data": "synthetic",
        "config": workload_config(args),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(args) -> dict:
    return {
        "workload": "cfg3 per-block scaled FP8 BMM: quant A 1x128 + quant B 128x128 + BMM, bf16 out",
        "batches": args.batches,
        "m": M, "k": K, "n": N,
        "a_block": list(QA), "b_block": list(QB),
        "b_layout": "a_k_b_n (B N-major, MN-major UMMA operand)",
        "parallelism": f"batch-sharded x{args.gpus}",
        "l2": "inputs larger than L2 (A bf16 is 1.9 GB/32 batches)",
    }


def measure_fp8_peak() -> None:
    """torch._scaled_mm e4m3 8192^3: best of 10 (burst) and back-to-back for
    4 s (sustained), the protocol of MEASURED_PEAKS.json's bf16 entry."""
    n = 8192
    dev = torch.device("cuda", 0)
    a = torch.randn((n, n), device=dev).to(torch.float8_e4m3fn)
    b = torch.randn((n, n), device=dev).to(torch.float8_e4m3fn).t()
    one = torch.ones((), device=dev)

    def mm():
        return torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)

    for _ in range(5):
        mm()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(10):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        mm()
        e.record()
        torch.cuda.synchronize()
        best = min(best, s.elapsed_time(e))
    flop = 2 * n ** 3
    clocks = ClockSampler(0)
    clocks.start()
    iters, t0 = 0, time.perf_counter()
    s = torch.cuda.Event(enable_timing=True)
    s.record()
    while time.perf_counter() - t0 < 4.0:
        for _ in range(20):
            mm()
        iters += 20
        torch.cuda.synchronize()
    e = torch.cuda.Event(enable_timing=True)
    e.record()
    torch.cuda.synchronize()
    sustained_ms = s.elapsed_time(e) / iters
    print(json.dumps({"fp8_e4m3_scaled_mm_tflops_burst": flop / (best * 1e-3) / 1e12,
                      "fp8_e4m3_scaled_mm_tflops_sustained": flop / (sustained_ms * 1e-3) / 1e12,
                      "shape": [n, n, n], "clocks": clocks.stop(), "how": "torch._scaled_mm (cuBLASLt) e4m3, bf16 out"}))


def run_cfg5(args, world: int, rank: int, local_rank: int) -> None:
    """BASELINE cfg5: one FSDP2 training step (forward, backward, AdamW) of the
    random-init Llama-style decoder on seq 4096 x batch 1 per GPU, synthetic
    token ids.  Linear layers are per-block FP8 (forward, dgrad, wgrad) with
    the FP8 weight + scale all-gather; ``--cfg5-linear bf16`` runs the same
    model with bf16 linears and bf16 all-gather as the comparison point.
    Reports model TFLOP/s per GPU as 6 * tokens * linear params / step time
    (the reference's estimate, bench_fsdp2.py:179-187) plus the causal
    attention FLOPs separately."""
    import torch.distributed as dist
    from torch.distributed.fsdp import MixedPrecisionPolicy, fully_shard

    from practice_cuda_b200.fp8_linear import FP8BlockLinear
    from practice_cuda_b200.fsdp_fp8 import enable_fp8_all_gather, precompute_fp8_block_weights
    from practice_cuda_b200.llama import Llama, LlamaConfig

    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29555")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    dist.init_process_group("nccl", device_id=device, rank=rank, world_size=world)
    cfg = LlamaConfig(n_layers=args.layers,
                      linear_scaling="e8m0" if args.cfg5_linear == "fp8_e8m0" else "fp32")
    with torch.device(device):
        model = Llama(cfg)
    model.init_weights(seed=0)
    if args.cfg5_linear == "bf16":
        for mod in list(model.modules()):
            for name, child in list(mod.named_children()):
                if isinstance(child, FP8BlockLinear):
                    lin = torch.nn.Linear(child.in_features, child.out_features, bias=False, device=device)
                    lin.weight = child.weight
                    setattr(mod, name, lin)
    else:
        enable_fp8_all_gather(model)
    mp = MixedPrecisionPolicy(param_dtype=torch.bfloat16, reduce_dtype=torch.float32)
    for layer in model.layers:
        fully_shard(layer, mp_policy=mp)
    fully_shard(model, mp_policy=mp)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4, fused=True)
    g = torch.Generator(device=device).manual_seed(1234 + rank)
    tokens = torch.randint(0, cfg.vocab, (1, cfg.seq_len + 1), device=device, generator=g)

    def step():
        logits = model(tokens[:, :-1])
        loss = torch.nn.functional.cross_entropy(logits.float().view(-1, cfg.vocab), tokens[:, 1:].reshape(-1))
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        if args.cfg5_linear != "bf16":
            precompute_fp8_block_weights(model)  # quantize each shard once per step
        return loss

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        loss = step()
    e.record()
    torch.cuda.synchronize()
    ms = torch.tensor([s.elapsed_time(e) / args.steps], device=device, dtype=torch.float64)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = ms.item()
    tokens_per_gpu = cfg.seq_len
    linear_flop = 6 * tokens_per_gpu * cfg.linear_params()
    attn_flop = 3 * cfg.n_layers * 2 * 2 * cfg.seq_len * cfg.seq_len * cfg.dim / 2  # causal, fwd + 2x bwd
    if rank == 0:
        print(json.dumps({
            "metric": "fsdp2_train_model_tflops_per_gpu",
            "value": linear_flop / (ms * 1e-3) / 1e12,
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "weak",
            "dtype": {"fp8": "per-block e4m3 linears (fp32 scales)",
                      "fp8_e8m0": "per-block e4m3 linears (power-of-two scales, block-scaled MMA)",
                      "bf16": "bf16 linears"}[args.cfg5_linear],
            "data": "synthetic token ids, random-init weights",
            "config": {"workload": "cfg5 FSDP2 training step", "layers": cfg.n_layers, "dim": cfg.dim,
                       "heads": cfg.n_heads, "ffn": cfg.ffn_dim, "vocab": cfg.vocab, "seq_len": cfg.seq_len,
                       "batch_per_gpu": 1, "parallelism": f"fsdp2 x{world}",
                       "all_gather": "per-block fp8 + fp32 scales" if args.cfg5_linear != "bf16" else "bf16",
                       "lm_head_and_embedding": "bf16"},
            "linear_tflop_per_gpu_step": linear_flop / 1e12,
            "attention_tflop_per_gpu_step": attn_flop / 1e12,
            "tokens_per_s": world * tokens_per_gpu / (ms * 1e-3),
            "final_loss": float(loss.item()),
        }), flush=True)
    dist.destroy_process_group()


# ------------------------------------------------------------------- main ---
def main() -> None:
    args = parse_args()
    if args.fp8_peak:
        measure_fp8_peak()
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.workload == "cfg5":
        run_cfg5(args, world, rank, local_rank)
        return

    import torch.distributed as dist

    from practice_cuda_b200 import _lib, get_bmm, get_quant

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", device_id=device)
    b0, b1 = shard_range(args.batches, rank, world)
    nb = b1 - b0
    a, b = make_inputs(b0, b1, device)

    quant = get_quant("b200_per_block_1x128_128x128").fn
    bmm = get_bmm("b200_per_block_1x128_128x128_a_k_b_n").fn
    out = torch.empty((nb, M, N), device=device, dtype=torch.bfloat16)
    stream = torch.cuda.current_stream(device)

    ev_bmm = []  # (start, end) CUDA events around each BMM launch

    def step(record=False):
        qa = quant(a, block_m=QA[0], block_n=QA[1])
        qb = quant(b, block_m=QB[0], block_n=QB[1])
        if record:
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            bmm(qa, qb, out=out)
            e.record(stream)
            ev_bmm.append((s, e))
        else:
            bmm(qa, qb, out=out)
        return qa, qb

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    _lib.device_error()

    clocks = None
    if rank == 0:
        visible = os.environ.get("CUDA_VISIBLE_DEVICES")
        smi_index = int(visible.split(",")[local_rank]) if visible else local_rank
        clocks = ClockSampler(smi_index)
        clocks.start()
        time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for _ in range(args.steps):
        step(record=True)
    t_end.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clock_info = clocks.stop() if clocks else None
    elapsed_ms = t_start.elapsed_time(t_end)
    bmm_ms = statistics.mean(s.elapsed_time(e) for s, e in ev_bmm)
    err = _lib.device_error()
    if err[0] != 0:
        raise RuntimeError(f"device error word set during the bench: {err}")

    stats = torch.tensor([elapsed_ms, bmm_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    elapsed_ms, bmm_ms = stats.tolist()
    ms_per_step = elapsed_ms / args.steps
    total_flop = FLOP_PER_BATCH * args.batches
    value = total_flop / (ms_per_step * 1e-3) / 1e12

    # Quant kernels alone (informational; HBM-bound).
    def time_fn(fn, reps=5):
        fn()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for _ in range(reps):
            fn()
        e.record(stream)
        torch.cuda.synchronize()
        return s.elapsed_time(e) / reps

    qa_ms = time_fn(lambda: quant(a, block_m=QA[0], block_n=QA[1]))
    qb_ms = time_fn(lambda: quant(b, block_m=QB[0], block_n=QB[1]))
    qa_bytes = nb * M * K * 3 + nb * M * (K // 128) * 4
    qb_bytes = nb * K * N * 3 + nb * (K // 128) * (N // 128) * 4

    # End to end through the public API from pinned host memory.
    e2e = None
    if not args.no_e2e:
        del a, b
        torch.cuda.empty_cache()
        a_h, b_h = (t.cpu().pin_memory() for t in make_inputs(b0, b1, device))
        c_h = torch.empty((nb, M, N), dtype=torch.bfloat16).pin_memory()
        a_d = torch.empty_like(a_h, device=device)
        b_d = torch.empty_like(b_h, device=device)

        c_d = torch.empty((nb, M, N), dtype=torch.bfloat16, device=device)
        # Batches move in chunks over three streams so the host->device copy
        # of chunk j+1, the kernels of chunk j and the device->host copy of
        # chunk j-1 overlap (PCIe is the bound, not the kernels).
        cb = max(1, min(4, nb))
        chunks = [(lo, min(nb, lo + cb)) for lo in range(0, nb, cb)]
        h2d, d2h = torch.cuda.Stream(device), torch.cuda.Stream(device)
        ev_in = [torch.cuda.Event() for _ in chunks]
        ev_done = [torch.cuda.Event() for _ in chunks]
        ev_out = [torch.cuda.Event() for _ in chunks]

        def e2e_step():
            h2d.wait_stream(stream)  # previous step's kernels are done with a_d / b_d
            for j, (lo, hi) in enumerate(chunks):
                with torch.cuda.stream(h2d):
                    a_d[lo:hi].copy_(a_h[lo:hi], non_blocking=True)
                    b_d[lo:hi].copy_(b_h[lo:hi], non_blocking=True)
                    ev_in[j].record(h2d)
                stream.wait_event(ev_in[j])
                stream.wait_event(ev_out[j])  # previous step's copy of this C chunk is out
                qa = quant(a_d[lo:hi], block_m=QA[0], block_n=QA[1])
                qb = quant(b_d[lo:hi], block_m=QB[0], block_n=QB[1])
                bmm(qa, qb, out=c_d[lo:hi])
                ev_done[j].record(stream)
                with torch.cuda.stream(d2h):
                    d2h.wait_event(ev_done[j])
                    c_h[lo:hi].copy_(c_d[lo:hi], non_blocking=True)
                    ev_out[j].record(d2h)
            stream.wait_stream(d2h)  # the step ends when C is in host memory

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e2e_steps = max(2, min(args.steps, 5))
        s.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        e.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / e2e_steps], dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = t.item()
        e2e = {
            "value": total_flop / (e2e_ms * 1e-3) / 1e12,
            "unit": "TFLOP/s",
            "ms_per_step": e2e_ms,
            "h2d_bytes_per_step": (a_h.numel() + b_h.numel()) * 2 * world,
            "d2h_bytes_per_step": c_h.numel() * 2 * world,
            "path": "registry impls (b200_per_block_1x128_128x128) from pinned host bf16, C copied back; "
                    f"{cb}-batch chunks, copies overlapped with the kernels on separate streams",
        }

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        dt, cores, sample = cpu_sample_seconds()
        cpu = {"value": FLOP_PER_BATCH / dt / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port",
               "sample": sample}

    peaks = measured_peaks()
    fp8_peak, fp8_src = 2 * peaks["bf16_tflops"], f"2 x {peaks['source']} bf16 burst"
    fp8_path = os.path.join(ROOT, "profiles", "fp8_peak.json")
    if os.path.exists(fp8_path):
        with open(fp8_path) as f:
            fp8_peak = json.load(f)["fp8_e4m3_dense_tflops_burst"]
        fp8_src = "measured cuBLASLt e4m3 burst (profiles/fp8_peak.json)"
    achieved = FLOP_PER_BATCH * nb / (bmm_ms * 1e-3) / 1e12
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "bmm_cfg3_traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            traffic = json.load(f).get("dram_bytes_per_launch_per_batch")
            if traffic is not None:
                traffic = traffic * nb

    if rank == 0:
        line = {
            "metric": "fp8_bmm_tflops",
            "value": value,
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_per_step,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "e4m3 (fp32 accumulate, bf16 out)",
            "data": "synthetic",
            "config": workload_config(args),
            "per_gpu_tflops": value / world,
            "bmm_kernel_ms": bmm_ms,
            "quant_a_gbs": qa_bytes / (qa_ms * 1e-3) / 1e9,
            "quant_b_gbs": qb_bytes / (qb_ms * 1e-3) / 1e9,
            "quant_hbm_peak_gbs": peaks["hbm_gbs"],
            "roofline": {
                "bound": "tensor",
                "achieved": achieved,
                "peak": fp8_peak,
                "unit": "TFLOP/s",
                "frac": achieved / fp8_peak,
                "traffic": traffic,
                "peak_note": f"FP8 dense peak: {fp8_src}; 2 x measured bf16 = {2 * peaks['bf16_tflops']:.0f}; "
                             f"vs 4500 spec: {achieved / 4500:.3f}",
            },
            "e2e": e2e,
            "cpu_baseline": cpu,
            "gpu_launches": 3 * args.steps,
            "clocks": clock_info,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
