#!/usr/bin/env python
"""Benchmark of the flash-mlm forward path on B200 (one JSON line on rank 0).

Headline workload = BASELINE config 2: flash_attn_mlm_compressed, B=32
sequences, H=16, N=512, D=64, bf16, query lengths U[64, 512], block_n=64,
one shared 1024-token context prefilled into InferenceCache layer 0 by a prior
prefill=True call, scale = 1/sqrt(64).  Synthetic seeded data of the
configured shapes and distributions.  `--config 1|3|4|5a|5b` makes another
BASELINE configuration the headline; by default every other configuration is
also measured once (a shorter run) and reported under `per_config`.

A step is one pass of the path through the public API (config 3: a prefill
call followed by the causal query call).  `value` is whole-job attention
TFLOP/s with inputs resident in HBM (L2 flushed between steps); `e2e` is the
same call with host (pinned) inputs copied in and the output read back inside
the timed region; `roofline` is the attention kernel alone (re-issued through
the C ABI) against the measured peak; `cpu_baseline` is the reference's CPU
path (its fp32 torch loop, restated in oracle/torch_ref.py) on the same
inputs, all host threads, on the longest sequences that fit a time budget,
and `parity` compares the GPU output with it on those sequences.
`--impl reference` times only that CPU path (the whole configuration per
step when it fits the time budget).

Multi-GPU (torchrun, one process per GPU, no collective on the data path):
the job is split with flash_mlm.parallel.plan_shards and each rank keeps its
own KV-cache shard.  `--scaling weak` (default): the job grows with N (N times
the sequences, split by cost-balanced sequence shards; a causal job, whose
sequences read all earlier sequences' keys, N times the heads, split by
heads).  `--scaling strong`: the configuration itself is split (heads, or
sequences for MLA).  Step time = max over ranks; value = all ranks' FLOPs /
that time.
"""

from __future__ import annotations

import argparse
import ctypes
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

import torch  # noqa: E402

TOL = {torch.float16: 2e-3, torch.bfloat16: 8e-3}
PER_CONFIG = ["1", "3", "4", "5a:1024", "5a:4096", "5a:32768", "5b:1", "5b:32", "5b:256"]


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def _lengths(g, B, lo, hi):
    return torch.randint(lo, hi + 1, (B,), generator=g, dtype=torch.int32).tolist()


def parse_config(label: str, args):
    """'5a:4096' -> ('5a', ctx=4096); '5b:32' -> ('5b', batch=32)."""
    name, _, val = label.partition(":")
    ctx, batch = args.ctx, args.batch
    if val:
        if name == "5a":
            ctx = int(val)
        elif name == "5b":
            batch = int(val)
    return name, ctx, batch


class Workload:
    """One BASELINE configuration (this rank's shard of it): synthetic inputs,
    a step through the public API, its work counts and the CPU reference."""

    def __init__(self, label: str, args, rank: int = 0, world: int = 1, scaling: str = "weak"):
        from flash_mlm.parallel import plan_shards

        config, ctx, batch = parse_config(label, args)
        self.config, self.label = config, label
        g = torch.Generator().manual_seed(0)
        self.is_mla = self.causal = self.dense = False
        self.shared_ctx = 0
        ctx_lengths = prefill_lengths = None
        if config == "1":
            B, H, N, D, dt, lengths, scale = 2, 8, 128, 64, torch.float16, [128, 128], 0.125
            self.dense = True
            desc = "config1: flash_attn_mlm dense [2,8,128,64] f16, scale 1/8, no cache"
        elif config == "2":
            B, H, N, D, dt, scale = 32, 16, 512, 64, torch.bfloat16, 1.0 / 8
            lengths = _lengths(g, B * (world if scaling == "weak" else 1), 64, 512)
            self.shared_ctx = 1024
            desc = ("config2: flash_attn_mlm_compressed packed varlen B=32 H=16 N=512 D=64 bf16, "
                    "query lengths U[64,512], shared 1024-token context prefilled into layer 0")
        elif config == "3":
            B, H, N, D, dt, scale = 64, 12, 256, 64, torch.float16, 0.125
            lengths = _lengths(g, B, 32, 256)
            ctx_lengths = prefill_lengths = _lengths(g, B, 256, 2048)
            self.causal = True
            if scaling == "weak":
                H *= world
            desc = ("config3: prefill call (per-sequence context U[256,2048]) then causal_query_seq_attn query "
                    "call, B=64 H=12 N=256 D=64 f16, query lengths U[32,256]")
        elif config == "4":
            B, H, N, D, dt, scale = 16, 128, 256, 512, torch.bfloat16, 1.0 / math.sqrt(512)
            lengths = _lengths(g, B * (world if scaling == "weak" else 1), 128, 256)
            ctx_lengths = [4096] * len(lengths)
            self.is_mla = True
            desc = ("config4: MLA, 128 query heads over one 512-wide latent KV head, B=16, query lengths "
                    "U[128,256], 4096 context tokens per sequence, bf16")
        elif config == "5a":
            B, H, N, D, dt, scale = 8, 16, 512, 128, torch.bfloat16, 1.0 / math.sqrt(128)
            lengths = _lengths(g, B * (world if scaling == "weak" else 1), 256, 512)
            ctx_lengths = [ctx] * len(lengths)
            desc = f"config5a: H=16 D=128 bf16 B=8, query lengths U[256,512], {ctx} context tokens per sequence"
        elif config == "5b":
            B, H, N, D, dt, scale = batch, 16, 512, 128, torch.bfloat16, 1.0 / math.sqrt(128)
            lengths = _lengths(g, B * (world if scaling == "weak" else 1), 256, 512)
            desc = f"config5b: H=16 D=128 bf16 N=512, query lengths U[256,512], B={batch}, no context"
        else:
            raise SystemExit(f"unknown --config {config}")
        self.desc = desc
        self.N, self.D, self.dtype, self.scale = N, D, dt, scale
        self.block_n = 64
        # ---- this rank's shard of the job (flash_mlm.parallel.plan_shards)
        self.plan = None
        self.H_job, self.B_job = H, len(lengths)
        if world > 1 and not self.dense:
            mode = "batch" if (scaling == "weak" and not self.causal) else "auto"
            plans = plan_shards(lengths, H, world, context_lengths=ctx_lengths, causal=self.causal,
                                is_mla=self.is_mla, mode=mode)
            self.plan = plans[rank]
            h0, h1 = self.plan.heads
            H = h1 - h0
            keep = self.plan.batches
            lengths = [lengths[b] for b in keep]
            if ctx_lengths is not None:
                ctx_lengths = [ctx_lengths[b] for b in keep]
            if prefill_lengths is not None:
                prefill_lengths = [prefill_lengths[b] for b in keep]
            g = torch.Generator().manual_seed(1000 * rank + 7)  # this rank's own data
        self.g = g
        self.B, self.H = len(lengths), H
        self.lengths, self.ctx_lengths, self.prefill_lengths = lengths, ctx_lengths, prefill_lengths
        self.T = sum(lengths)

    def parallelism(self, world):
        if self.plan is None:
            return f"dp{world} (replicas)" if world > 1 else "single GPU"
        return (f"{self.plan.mode} shards over {world} ranks (job: B={self.B_job} H={self.H_job}; this rank "
                f"B={self.B} H={self.H}; each rank its own KV-cache shard)")

    # ---------------------------------------------------------------- work counts
    def _kv_rows(self, b):
        kv = (sum(self.lengths[: b + 1]) if self.causal else self.lengths[b])
        if self.shared_ctx:
            kv += self.shared_ctx
        elif self.ctx_lengths is not None:
            kv += self.ctx_lengths[b]
        return kv

    def seq_flops(self, b):
        return 4.0 * self.H * self.D * self.lengths[b] * self._kv_rows(b)

    def flops(self, query_only=False):
        f = sum(self.seq_flops(b) for b in range(self.B))
        if self.prefill_lengths is not None and not query_only:
            f += 4.0 * self.H * self.D * sum(L * L for L in self.prefill_lengths)
        return f

    def alg_bytes(self):
        e, D, H, T = 2, self.D, self.H, self.T
        hkv, kv = (1, 1) if self.is_mla else (H, 2)
        ctx = self.shared_ctx if self.shared_ctx else (sum(self.ctx_lengths) if self.ctx_lengths else 0)
        return e * D * (2 * H * T + kv * hkv * T + kv * hkv * ctx)

    # ---------------------------------------------------------------- inputs and step
    def make_host(self):
        """Seeded host copies of every input: q/k/v, and the context in the
        head-major order the cache holds it (kc_h/vc_h, cu_kv, ctx_bs, tcl)."""
        g, dt = self.g, self.dtype
        B, H, N, D = self.B, self.H, self.N, self.D
        sc = 0.5 if self.is_mla else 1.0
        self.q_h = (torch.randn((B, H, N, D), generator=g) * sc).to(dt)
        if self.is_mla:
            self.k_h = (torch.randn((B, 1, N, D), generator=g) * sc).to(dt)
            self.v_h = self.k_h
        else:
            self.k_h = torch.randn((B, H, N, D), generator=g).to(dt)
            self.v_h = torch.randn((B, H, N, D), generator=g).to(dt)
        self.kc_h = self.vc_h = self.cu_kv = None
        self.ctx_bs, self.tcl = 1, 0
        if self.dense:
            return
        if self.shared_ctx:
            C = self.shared_ctx
            self.pk_h = torch.randn((1, H, C, D), generator=g).to(dt)
            self.pv_h = torch.randn((1, H, C, D), generator=g).to(dt)
            self.kc_h, self.vc_h = self.pk_h.reshape(H * C, D), self.pv_h.reshape(H * C, D)
            self.cu_kv, self.ctx_bs, self.tcl = [0, C], 1, C
        elif self.prefill_lengths is not None:
            Np = max(self.prefill_lengths)
            self.pq_h, self.pk_h, self.pv_h = (torch.randn((B, H, Np, D), generator=g).to(dt) for _ in range(3))
            cu = [0]
            for L in self.prefill_lengths:
                cu.append(cu[-1] + L)
            self.kc_h = torch.cat([self.pk_h[b, :, :L] for b, L in enumerate(self.prefill_lengths)], 1).reshape(-1, D)
            self.vc_h = torch.cat([self.pv_h[b, :, :L] for b, L in enumerate(self.prefill_lengths)], 1).reshape(-1, D)
            self.cu_kv, self.ctx_bs, self.tcl = cu, B, cu[-1]
        elif self.ctx_lengths is not None:
            cu = [0]
            for L in self.ctx_lengths:
                cu.append(cu[-1] + L)
            rows = cu[-1] if self.is_mla else H * cu[-1]
            self.kc_h = (torch.randn((rows, D), generator=g) * sc).to(dt)
            self.vc_h = None if self.is_mla else torch.randn((rows, D), generator=g).to(dt)
            self.cu_kv, self.ctx_bs, self.tcl = cu, B, cu[-1]

    def build(self, device):
        import flash_mlm

        self.fm = flash_mlm
        self.make_host()
        H, N, D = self.H, self.N, self.D
        self.q = self.q_h.to(device)
        self.k = self.k_h.to(device)
        self.v = self.v_h.to(device) if not self.is_mla else self.k
        self.cache = flash_mlm.InferenceCache()
        if self.dense:
            self.meta = None
            return
        self.meta = flash_mlm.build_pack_metadata(torch.tensor(self.lengths, dtype=torch.int32, device=device),
                                                  N, self.block_n)
        if self.shared_ctx:
            # one shared context, prefilled into layer 0 by a prior prefill=True call (B=1, N=ctx)
            C = self.shared_ctx
            pm = flash_mlm.build_pack_metadata(torch.tensor([C], dtype=torch.int32, device=device), C, self.block_n)
            kc, vc = self.pk_h.to(device), self.pv_h.to(device)
            flash_mlm.flash_attn_mlm_compressed(kc, kc, vc, num_heads=H, q_meta=pm, scale=self.scale,
                                                inference_cache=self.cache, layer_id=0, block_n=self.block_n,
                                                prefill=True)
        elif self.prefill_lengths is not None:
            self.pq, self.pk, self.pv = (x.to(device) for x in (self.pq_h, self.pk_h, self.pv_h))
            self.pmeta = flash_mlm.build_pack_metadata(
                torch.tensor(self.prefill_lengths, dtype=torch.int32, device=device), self.pq_h.shape[2],
                self.block_n)
        elif self.ctx_lengths is not None:
            self.cache.prefill_kv_cache(0, k_cache=self.kc_h.to(device),
                                        v_cache=None if self.is_mla else self.vc_h.to(device),
                                        total_context_len=self.tcl,
                                        cu_seqlens_kv=torch.tensor(self.cu_kv, dtype=torch.int32, device=device),
                                        context_batch_size=self.B, is_mla=self.is_mla, num_heads=H, head_dim=D)

    def step(self, q=None, k=None, v=None):
        fm = self.fm
        q = self.q if q is None else q
        k = self.k if k is None else k
        v = self.v if v is None else v
        if self.is_mla:
            k = k.expand(self.B, self.H, self.N, self.D)
            v = k
        if self.dense:
            return fm.flash_attn_mlm(q, k, v, scale=self.scale)
        if self.prefill_lengths is not None:
            fm.flash_attn_mlm_compressed(self.pq, self.pk, self.pv, num_heads=self.H, q_meta=self.pmeta,
                                         scale=self.scale, inference_cache=self.cache, layer_id=0,
                                         block_n=self.block_n, prefill=True)
        return fm.flash_attn_mlm_compressed(q, k, v, num_heads=self.H, q_meta=self.meta, scale=self.scale,
                                            inference_cache=self.cache, layer_id=0, block_n=self.block_n,
                                            is_mla=self.is_mla, causal_query_seq_attn=self.causal)

    def launches_per_step(self):
        if self.dense:
            return 1
        # The tile schedule is built on the first call with a given metadata
        # and memoised in the InferenceCache, so a timed step launches only:
        n = 1  # attention
        if self.causal:
            n += 2  # pack main K and V into the packed prefix
        if self.prefill_lengths is not None:
            n += 2 + 1  # prefill: pack K, V into the cache + attention
        return n

    # ---------------------------------------------------------------- the reference's CPU path
    def cpu_reference(self, only):
        """fp32 CPU reference (oracle/torch_ref.py) of sequences `only` (all heads); packed [H*T, D]."""
        from oracle import torch_ref

        f = lambda x: None if x is None else x.float()  # noqa: E731
        q, k, v = f(self.q_h), f(self.k_h), f(self.v_h)
        if self.dense:
            return torch_ref.dense_attention_with_cache(q, k, v, self.scale)
        cu = [0]
        for L in self.lengths:
            cu.append(cu[-1] + L)
        return torch_ref.varlen_attention_with_cache(
            q, k, v, cu, self.scale, k_cache=f(self.kc_h), v_cache=f(self.vc_h), cu_kv=self.cu_kv,
            context_batch_size=getattr(self, "ctx_bs", 1), total_context_len=getattr(self, "tcl", 0),
            is_mla=self.is_mla, causal_query_seq_attn=self.causal, only=only)

    def rows_of(self, packed, only):
        """Rows of sequences `only` (all heads) from a packed [H*T, D] output."""
        if self.dense:
            return packed.float().reshape(-1, self.D)
        cu = [0]
        for L in self.lengths:
            cu.append(cu[-1] + L)
        x = packed.float().reshape(self.H, self.T, self.D)
        return torch.cat([x[:, cu[b]:cu[b + 1]] for b in sorted(only)], dim=1).reshape(-1, self.D)

    def by_cost(self):
        return sorted(range(self.B), key=lambda b: -self.seq_flops(b)) if not self.dense else [0]


def cpu_leg(w: Workload, out_gpu, budget_s: float):
    """The cpu_baseline leg: the reference's CPU path on the most expensive
    sequences that fit `budget_s` (at least one), timed on all host threads,
    and the GPU output compared with it on those sequences."""
    torch.set_num_threads(os.cpu_count() or 1)
    done, fl, t_cpu, err = [], 0.0, 0.0, 0.0
    for b in w.by_cost():
        t0 = time.perf_counter()
        ref = w.cpu_reference([b])
        t_cpu += time.perf_counter() - t0
        done.append(b)
        fl += w.seq_flops(b) if not w.dense else w.flops()
        got = w.rows_of(out_gpu.cpu(), [b])
        err = max(err, (got - w.rows_of(ref, [b])).abs().max().item() if got.numel() else 0.0)
        if t_cpu > budget_s or w.dense:
            break
    tol = TOL[w.dtype]
    seqs = "all" if w.dense else f"{len(done)} of {w.B} sequences (longest first), all {w.H} heads"
    return ({"value": fl / t_cpu / 1e12, "unit": "TFLOP/s", "cores": torch.get_num_threads(), "kind": "port",
             "sample": f"{seqs}: torch fp32 loop of the reference's CPU path (oracle/torch_ref.py), "
                       f"{t_cpu:.1f} s"},
            {"max_abs_err": err, "tol": tol, "pass": err <= tol, "sequences": seqs})


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
        rows = [[x.strip() for x in line.split(",")] for line in Path(self.f.name).read_text().splitlines()]
        rows = [r for r in rows if len(r) >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [v for v in (num(r[1]) for r in rows) if v is not None]
        smax = [v for v in (num(r[2]) for r in rows) if v is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows)}


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU path (fp32 torch loop) on the host cores."""
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    w = Workload(args.config, args)
    w.make_host()  # the same seeded host inputs the native arm builds
    # per-step sample: the whole configuration when (steps + warmup) of it fit the budget
    order = w.by_cost()
    t0 = time.perf_counter()
    w.cpu_reference([order[0]])  # probe: the most expensive sequence
    probe = time.perf_counter() - t0
    est_full = probe if w.dense else probe * w.flops(query_only=True) / w.seq_flops(order[0])
    n_steps = args.steps + args.warmup
    per_step = len(order) if est_full * n_steps <= args.cpu_budget_total else \
        max(1, int(len(order) * args.cpu_budget_total / max(est_full * n_steps, 1e-9)))
    fl = sec = 0.0
    pos = 0
    for i in range(n_steps):
        only = [order[(pos + j) % len(order)] for j in range(per_step)]
        pos += per_step
        t0 = time.perf_counter()
        w.cpu_reference(only)
        dt_s = time.perf_counter() - t0
        if i >= args.warmup:
            sec += dt_s
            fl += sum(w.seq_flops(b) for b in set(only)) if not w.dense else w.flops()
    if w.prefill_lengths is not None:
        sample_note = " (query call of each step; its prefill call is the same loop without context)"
    else:
        sample_note = ""
    value = fl / sec / 1e12
    sample = ("the whole configuration each step" if per_step == len(order) else
              f"{per_step} of {w.B} sequences (all {w.H} heads) per step, rotating") + sample_note
    line = {
        "impl": "reference", "metric": "attention TFLOP/s", "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": w.desc, "sample": sample},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"{sample}; torch fp32 loop of the reference's CPU path (oracle/torch_ref.py)"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def time_steps(w, K, flush, device):
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    for i in range(K):
        flush.fill_(float(i))
        ev[i][0].record()
        w.step()
        ev[i][1].record()
    torch.cuda.synchronize(device)
    return sum(a.elapsed_time(b) for a, b in ev)


def time_kernel(w, K, flush, device, total_ms):
    """Attention kernel alone: the last packed launch re-issued through the C ABI with its schedule reused."""
    from flash_mlm import _lib
    from flash_mlm.host import host as host_mod

    if w.dense or host_mod.last_packed_launch is None:
        return total_ms / K, w.flops()
    kargs = _lib.PackedArgs.from_buffer_copy(host_mod.last_packed_launch[0])
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
    return sum(a.elapsed_time(b) for a, b in kev) / K, w.flops(query_only=True)


def roofline(w, kernel_ms, k_flops, pk, traffic=None):
    achieved = k_flops / (kernel_ms * 1e-3) / 1e12
    alg_bytes = w.alg_bytes()
    t_tensor = k_flops / (pk["bf16_tflops"] * 1e12)
    t_hbm = alg_bytes / (pk["hbm_gbs"] * 1e9)
    if t_tensor >= t_hbm:
        roof = {"bound": "tensor", "achieved": achieved, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                "frac": achieved / pk["bf16_tflops"]}
    else:
        gbs = alg_bytes / (kernel_ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": gbs, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": gbs / pk["hbm_gbs"]}
    nq = 1 if w.D >= 256 or w.D == 64 else 2
    roof.update({"traffic": traffic, "kernel": f"attn_fwd_kernel<{w.D},{nq},"
                 f"{'bf16' if w.dtype == torch.bfloat16 else 'f16'}>", "kernel_ms": kernel_ms,
                 "alg_flops_per_launch": k_flops, "alg_bytes_per_launch": alg_bytes,
                 "roofline_ms": max(t_tensor, t_hbm) * 1e3,
                 "frac_of_roofline_time": max(t_tensor, t_hbm) / (kernel_ms * 1e-3),
                 "peak_source": pk["source"] + " (burst, kernel timed alone)"})
    return roof


def measure_config(label, args, device, flush, pk):
    """A shorter run of another configuration: value, kernel time, roofline fraction, parity (rank 0, N=1)."""
    w = Workload(label, args)
    w.build(device)
    for _ in range(3):
        w.step()
    torch.cuda.synchronize(device)
    K = max(3, min(args.steps, args.per_config_steps))
    total_ms = time_steps(w, K, flush, device)
    kernel_ms, k_flops = time_kernel(w, K, flush, device, total_ms)
    out = w.step()
    torch.cuda.synchronize(device)
    w.fm.check_device_errors(device)
    roof = roofline(w, kernel_ms, k_flops, pk)
    _, parity = cpu_leg(w, out, args.per_config_cpu_budget)
    return {"workload": w.desc, "value_tflops": w.flops() * K / (total_ms * 1e-3) / 1e12,
            "ms_per_step": total_ms / K, "tokens_per_s": w.T * K / (total_ms * 1e-3), "kernel_ms": kernel_ms,
            "roofline_bound": roof["bound"], "achieved": roof["achieved"], "achieved_unit": roof["unit"],
            "frac": roof["frac"], "parity_max_abs_err": parity["max_abs_err"], "parity_tol": parity["tol"],
            "parity_sample": parity["sequences"], "steps": K}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--config", default="2", choices=["1", "2", "3", "4", "5a", "5b"])
    ap.add_argument("--ctx", type=int, default=4096, help="config 5a: context tokens per sequence")
    ap.add_argument("--batch", type=int, default=32, help="config 5b: batch size")
    ap.add_argument("--scaling", default="weak", choices=["weak", "strong"])
    ap.add_argument("--cpu-budget", type=float, default=12.0, help="seconds of CPU reference for cpu_baseline")
    ap.add_argument("--cpu-budget-total", type=float, default=150.0,
                    help="--impl reference: seconds of CPU work for the whole run")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-per-config", action="store_true")
    ap.add_argument("--per-config-steps", type=int, default=30)
    ap.add_argument("--per-config-cpu-budget", type=float, default=2.0)
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
        os.environ.setdefault("NCCL_DEBUG", "WARN")  # keep NCCL's version banner off stdout (one JSON line)
        import torch.distributed as dist_mod

        dist = dist_mod
        dist.init_process_group("nccl", device_id=device)

    import flash_mlm
    from flash_mlm.host import host as host_mod

    host_mod.record_packed_launches(True)  # the kernel-only timing re-issues the last launch
    w = Workload(args.config, args, rank, world, args.scaling)
    w.build(device)
    flops = w.flops()
    T = w.T

    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)  # > 126 MB L2
    for _ in range(args.warmup):
        w.step()
    torch.cuda.synchronize(device)

    K = args.steps
    with ClockSampler(local_rank) as clk:
        # pre-roll so the clock samples cover a loaded GPU around the timed region
        t_end = time.perf_counter() + 1.5
        while time.perf_counter() < t_end:
            for _ in range(20):
                w.step()
            torch.cuda.synchronize(device)
        if dist:
            dist.barrier()
        torch.cuda.synchronize(device)
        total_ms = time_steps(w, K, flush, device)
        if dist:
            dist.barrier()
        torch.cuda.synchronize(device)
    kernel_ms, k_flops = time_kernel(w, K, flush, device, total_ms)

    # end to end: host (pinned) inputs -> device, API call, output -> host
    hosts = [w.q_h.pin_memory(), w.k_h.pin_memory()] + ([] if w.is_mla else [w.v_h.pin_memory()])
    devs = [torch.empty_like(x, device=device) for x in hosts]
    out0 = w.step()
    out_h = torch.empty(out0.shape, dtype=out0.dtype).pin_memory()
    K_e2e = max(3, min(K, 50))
    e2e_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K_e2e)]
    for i in range(K_e2e + 2):
        if i >= 2:
            e2e_ev[i - 2][0].record()
        for d, h in zip(devs, hosts):
            d.copy_(h, non_blocking=True)
        o = w.step(devs[0], devs[1], devs[1] if w.is_mla else devs[2])
        out_h.copy_(o, non_blocking=True)
        if i >= 2:
            e2e_ev[i - 2][1].record()
    torch.cuda.synchronize(device)
    e2e_ms = sum(a.elapsed_time(b) for a, b in e2e_ev) / K_e2e
    flash_mlm.check_device_errors(device)

    t = torch.tensor([total_ms, kernel_ms, e2e_ms, flops, float(T)], dtype=torch.float64, device=device)
    if dist:
        mx = t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = t.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        total_ms, kernel_ms, e2e_ms = mx[0].item(), mx[1].item(), mx[2].item()
        all_flops, all_tokens = sm[3].item(), sm[4].item()
    else:
        all_flops, all_tokens = flops, float(T)

    if rank == 0:
        pk = peaks()
        value = all_flops * K / (total_ms * 1e-3) / 1e12
        tok_s = all_tokens * K / (total_ms * 1e-3)
        traffic = None
        tf = ROOT / "profiles" / f"attn_fwd_config{args.config}_traffic.txt"
        if tf.exists() and world == 1:
            for line in tf.read_text().splitlines():
                if line.startswith("dram_bytes_per_launch="):
                    traffic = float(line.split("=", 1)[1])
        roof = roofline(w, kernel_ms, k_flops, pk, traffic)
        cpu = parity = None
        if world == 1 and not args.no_cpu_baseline:
            cpu, parity = cpu_leg(w, out0, args.cpu_budget)
        h2d = sum(x.numel() * x.element_size() for x in hosts)
        d2h = out_h.numel() * out_h.element_size()
        line = {
            "metric": "attention TFLOP/s",
            "value": value,
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": K,
            "warmup": args.warmup,
            "ms_per_step": total_ms / K,
            "higher_is_better": True,
            "scaling": args.scaling,
            "vs_baseline": None,
            "dtype": "bf16" if w.dtype == torch.bfloat16 else "f16",
            "data": "synthetic (seeded N(0,1) inputs and context of the configured shapes)",
            "config": {"workload": w.desc, "B_per_gpu": w.B, "H_per_gpu": w.H, "N": w.N, "D": w.D,
                       "tokens_per_gpu_step": T, "l2": "flushed (256 MB write) between timed steps",
                       "parallelism": w.parallelism(world)},
            "tokens_per_s": tok_s,
            "tokens_per_s_per_gpu": tok_s / world,
            "tflops_per_gpu": value / world,
            "roofline": roof,
            "cpu_baseline": cpu,
            "parity": parity,
            "e2e": {"value": all_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
            "gpu_launches": w.launches_per_step() * K,
            "clocks": clk.summary(),
        }
        if world == 1 and not args.no_per_config:
            del w, hosts, devs, out0, out_h
            torch.cuda.empty_cache()
            per = {}
            for label in PER_CONFIG:
                if label.split(":")[0] == args.config:
                    continue
                per[label] = measure_config(label, args, device, flush, pk)
                torch.cuda.empty_cache()
            line["per_config"] = per
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
