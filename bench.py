#!/usr/bin/env python
"""Benchmark of the flash-mlm forward path on B200 (one JSON line on rank 0).

Default workload = BASELINE config 2 (the configuration the headline metric is
quoted on): flash_attn_mlm_compressed, B=32 sequences, H=16, N=512, D=64,
bf16, query lengths U[64, 512], block_n=64, one shared 1024-token context
prefilled into InferenceCache layer 0 by a prior prefill=True call,
scale = 1/sqrt(64).  Synthetic seeded N(0,1) data.

A step is one query call.  `value` is whole-job attention TFLOP/s with
inputs resident in HBM (L2 flushed between steps); `e2e` is the same call
through the public API with host (pinned) inputs and a read-back of the
output inside the timed region; `roofline` is the attention kernel alone
(re-issued through the C ABI) against the measured bf16 peak; `cpu_baseline`
is the CPU oracle (a numpy restatement of the reference's fp32 math) on a
bounded sample.  `--impl reference` times only that CPU path.

Multi-GPU (torchrun): one process per GPU, each rank runs its own batch of
32 sequences (weak scaling, no collective on the data path); the step time
is the max over ranks.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "flash-mlm_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import numpy as np  # noqa: E402
import torch  # noqa: E402

CFG2 = dict(B=32, H=16, N=512, D=64, ctx=1024, lo=64, hi=512, block_n=64, dtype="bf16")
WORKLOAD = ("config2: flash_attn_mlm_compressed packed varlen B=32 H=16 N=512 D=64 bf16, "
            "query lengths U[64,512], shared 1024-token context prefilled into layer 0")


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def make_workload(rank: int, device):
    c = CFG2
    g = torch.Generator().manual_seed(0 + 1000 * rank)
    lengths = torch.randint(c["lo"], c["hi"] + 1, (c["B"],), generator=g, dtype=torch.int32)
    shape = (c["B"], c["H"], c["N"], c["D"])
    dt = torch.bfloat16
    tens = []
    for i in range(3):
        gi = torch.Generator().manual_seed(1 + i + 1000 * rank)
        tens.append(torch.randn(shape, generator=gi).to(dt))
    gc = torch.Generator().manual_seed(4 + 1000 * rank)
    ctx_k = torch.randn((1, c["H"], c["ctx"], c["D"]), generator=gc).to(dt)
    ctx_v = torch.randn((1, c["H"], c["ctx"], c["D"]), generator=gc).to(dt)
    return lengths, tens, (ctx_k, ctx_v)


def flops_and_bytes(lengths: list[int]):
    c = CFG2
    H, D, ctx = c["H"], c["D"], c["ctx"]
    flops = 4.0 * H * D * sum(L * (ctx + L) for L in lengths)
    T = sum(lengths)
    nbytes = 2 * D * (2 * H * T + 2 * H * T + 2 * H * ctx)
    return flops, nbytes


class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons while the GPU is under load."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        self.f.flush()
        rows = []
        for line in Path(self.f.name).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(parts)
            except ValueError:
                pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows)}


def cpu_oracle_sample(lengths, tens, ctx, budget_s: float, max_seqs: int | None = None):
    """Run the CPU oracle on whole sequences until the time budget is used; returns (flops, seconds, nseq)."""
    import oracle

    c = CFG2
    q, k, v = (t.float().numpy() for t in tens)
    kc = ctx[0][0].float().numpy().reshape(c["H"] * c["ctx"], c["D"])
    vc = ctx[1][0].float().numpy().reshape(c["H"] * c["ctx"], c["D"])
    cu_kv = np.array([0, c["ctx"]])
    scale = 1.0 / math.sqrt(c["D"])
    done, flops, t0 = 0, 0.0, time.perf_counter()
    for b, L in enumerate(lengths):
        if max_seqs is not None and done >= max_seqs:
            break
        cu = np.array([0, L])
        oracle.attention_packed(q[b:b + 1], k[b:b + 1], v[b:b + 1], cu, scale, k_cache=kc, v_cache=vc, cu_kv=cu_kv,
                                context_batch_size=1, total_context_len=c["ctx"])
        flops += flops_and_bytes([L])[0]
        done += 1
        if time.perf_counter() - t0 > budget_s:
            break
    return flops, time.perf_counter() - t0, done


def cpu_threads() -> int:
    try:
        from threadpoolctl import threadpool_info

        n = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        if n:
            return int(max(n))
    except Exception:
        pass
    return os.cpu_count() or 1


def run_reference(args, rank, world):
    """--impl reference: the CPU oracle (numpy restatement of the reference's fp32 path)."""
    if rank != 0:
        return
    lengths, tens, ctx = make_workload(0, "cpu")
    L = lengths.tolist()
    per_step_seqs = 2
    for _ in range(args.warmup):
        cpu_oracle_sample(L, tens, ctx, budget_s=1e9, max_seqs=per_step_seqs)
    fl, sec = 0.0, 0.0
    for i in range(args.steps):
        off = (i * per_step_seqs) % len(L)
        sub = L[off:] + L[:off]
        f, s, _ = cpu_oracle_sample(sub, [t.roll(-off, 0) for t in tens], ctx, budget_s=1e9, max_seqs=per_step_seqs)
        fl += f
        sec += s
    value = fl / sec / 1e12
    line = {
        "impl": "reference", "metric": "attention TFLOP/s", "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample": f"{per_step_seqs} of 32 sequences (all 16 heads) per step"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": cpu_threads(), "kind": "port",
                         "sample": f"{per_step_seqs} sequences x 16 heads per step (numpy fp32 oracle)"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--cpu-budget", type=float, default=12.0, help="seconds of CPU-oracle work for cpu_baseline")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist_mod

        dist = dist_mod
        dist.init_process_group("nccl", device_id=device)

    import ctypes

    import flash_mlm
    from flash_mlm import _lib
    from flash_mlm.host import host as host_mod

    c = CFG2
    lengths, tens, ctx = make_workload(rank, device)
    L = lengths.tolist()
    flops, alg_bytes = flops_and_bytes(L)
    T = sum(L)
    q, k, v = (t.to(device) for t in tens)
    cache = flash_mlm.InferenceCache()
    # The shared context is prefilled into layer 0 by a prior prefill=True call (B=1, N=1024).
    pre_meta = flash_mlm.build_pack_metadata(torch.tensor([c["ctx"]], dtype=torch.int32, device=device), c["ctx"],
                                             c["block_n"])
    kc, vc = ctx[0].to(device), ctx[1].to(device)
    flash_mlm.flash_attn_mlm_compressed(kc, kc, vc, num_heads=c["H"], q_meta=pre_meta, scale=0.125,
                                        inference_cache=cache, layer_id=0, block_n=c["block_n"], prefill=True)
    meta = flash_mlm.build_pack_metadata(lengths.to(device), c["N"], c["block_n"])
    scale = 1.0 / math.sqrt(c["D"])

    def step():
        return flash_mlm.flash_attn_mlm_compressed(q, k, v, num_heads=c["H"], q_meta=meta, scale=scale,
                                                   inference_cache=cache, layer_id=0, block_n=c["block_n"])

    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)  # > 126 MB L2
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)

    K = args.steps
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    with ClockSampler(local_rank) as clk:
        # pre-roll so the clock samples cover a loaded GPU around the timed region
        t_end = time.perf_counter() + 1.5
        while time.perf_counter() < t_end:
            for _ in range(50):
                step()
            torch.cuda.synchronize(device)
        if dist:
            dist.barrier()
        torch.cuda.synchronize(device)
        for i in range(K):
            flush.fill_(float(i))
            ev[i][0].record()
            step()
            ev[i][1].record()
        torch.cuda.synchronize(device)
        if dist:
            dist.barrier()
        torch.cuda.synchronize(device)
    step_ms = [a.elapsed_time(b) for a, b in ev]
    total_ms = sum(step_ms)

    # attention kernel alone: re-issue the last launch through the C ABI with the schedule reused
    args_c, ws = host_mod.last_packed_launch
    kargs = _lib.PackedArgs.from_buffer_copy(args_c)
    kargs.reuse_schedule = 1
    lib = _lib.lib()
    stream = _lib.stream_ptr(device)
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    for i in range(K):
        flush.fill_(float(i))
        kev[i][0].record()
        _lib.check(lib.fmlm_attn_packed_fwd(ctypes.byref(kargs), stream), "attn kernel")
        kev[i][1].record()
    torch.cuda.synchronize(device)
    kernel_ms = sum(a.elapsed_time(b) for a, b in kev) / K

    # end to end: host (pinned) inputs -> device, API call, output -> host
    qh, kh, vh = (t.pin_memory() for t in tens)
    out_h = torch.empty((c["H"] * T, c["D"]), dtype=torch.bfloat16).pin_memory()
    qd, kd, vd = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    K_e2e = max(3, min(K, 50))
    e2e_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K_e2e)]
    for i in range(K_e2e + 2):
        if i >= 2:
            e2e_ev[i - 2][0].record()
        qd.copy_(qh, non_blocking=True)
        kd.copy_(kh, non_blocking=True)
        vd.copy_(vh, non_blocking=True)
        o = flash_mlm.flash_attn_mlm_compressed(qd, kd, vd, num_heads=c["H"], q_meta=meta, scale=scale,
                                                inference_cache=cache, layer_id=0, block_n=c["block_n"])
        out_h.copy_(o, non_blocking=True)
        if i >= 2:
            e2e_ev[i - 2][1].record()
    torch.cuda.synchronize(device)
    e2e_ms = sum(a.elapsed_time(b) for a, b in e2e_ev) / K_e2e
    flash_mlm.check_device_errors(device)

    t_max = torch.tensor([total_ms, kernel_ms, e2e_ms, flops, float(T)], dtype=torch.float64, device=device)
    if dist:
        mx = t_max.clone()
        dist.all_reduce(mx[:3], op=dist.ReduceOp.MAX)
        sm = t_max.clone()
        dist.all_reduce(sm[3:], op=dist.ReduceOp.SUM)
        total_ms, kernel_ms, e2e_ms = mx[0].item(), mx[1].item(), mx[2].item()
        all_flops, all_tokens = sm[3].item(), sm[4].item()
    else:
        all_flops, all_tokens = flops, float(T)

    if rank == 0:
        pk = peaks()
        ms_step = total_ms / K
        value = all_flops * K / (total_ms * 1e-3) / 1e12
        tok_s = all_tokens * K / (total_ms * 1e-3)
        k_tflops = flops / (kernel_ms * 1e-3) / 1e12
        traffic = None
        tf = ROOT / "profiles" / "attn_fwd_config2_traffic.txt"
        if tf.exists():
            for line in tf.read_text().splitlines():
                if line.startswith("dram_bytes_per_launch="):
                    traffic = float(line.split("=", 1)[1])
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            f, s, nseq = cpu_oracle_sample(L, tens, ctx, budget_s=args.cpu_budget)
            cpu = {"value": f / s / 1e12, "unit": "TFLOP/s", "cores": cpu_threads(), "kind": "port",
                   "sample": f"{nseq} of {c['B']} sequences x {c['H']} heads (numpy fp32 oracle), {s:.1f} s"}
        h2d = sum(t.numel() * t.element_size() for t in tens)
        d2h = out_h.numel() * out_h.element_size()
        line = {
            "metric": "attention TFLOP/s",
            "value": value,
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": K,
            "warmup": args.warmup,
            "ms_per_step": ms_step,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) q/k/v and context, lengths U[64,512])",
            "config": {"workload": WORKLOAD, "B_per_gpu": c["B"], "H": c["H"], "N": c["N"], "D": c["D"],
                       "context": c["ctx"], "block_n": c["block_n"], "tokens_per_gpu_step": T,
                       "l2": "flushed (256 MB write) between timed steps", "parallelism": f"dp{world} (batch shards)"},
            "tokens_per_s": tok_s,
            "tokens_per_s_per_gpu": tok_s / world,
            "tflops_per_gpu": value / world,
            "roofline": {
                "bound": "tensor",
                "achieved": k_tflops,
                "peak": pk["bf16_tflops"],
                "unit": "TFLOP/s",
                "frac": k_tflops / pk["bf16_tflops"],
                "traffic": traffic,
                "kernel": "attn_fwd_kernel<64,2,bf16>",
                "kernel_ms": kernel_ms,
                "alg_flops_per_launch": flops,
                "alg_bytes_per_launch": alg_bytes,
                "hbm_frac": alg_bytes / (kernel_ms * 1e-3) / 1e9 / pk["hbm_gbs"],
                "peak_source": pk["source"] + " (burst, kernel timed alone)",
            },
            "cpu_baseline": cpu,
            "e2e": {"value": all_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
            "gpu_launches": 2 * K,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
