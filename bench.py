"""bench.py -- LoRA fwd+bwd+AdamW step throughput of the 9B-class synthetic hybrid model on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config 5|4]
    python bench.py --case NAME      # one small kernel case to profile under ncu (profile_case)

One process per GPU (torchrun for N > 1, NCCL over NVLink). Each rank trains its own micro-batch of
seq 4096 x 2 (config 5) on the same frozen IQR base and the same adapter; the adapter gradient is
all-reduced (averaged) per layer bucket as the reverse walk finishes each layer, on a side stream, and
every rank applies the same AdamW update (data parallel, weak scaling). Rank 0 prints one JSON line.

`value` is the whole-job tokens/s with token ids already on the device; `e2e` is the same step driven
through the public API from pinned host token ids, with the H2D copy of the ids and the D2H read of the
loss inside the timed region. `roofline` is the dominant kernel -- the tcgen05 GEMM -- measured live:
algorithmic FLOPs of every GEMM launch in the timed steps over their CUDA-event durations, against the
measured sustained bf16 peak. `cpu_baseline` times the reference's own host rows (oracle/_ref) on a
bounded sample and extrapolates tokens/s.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "LoRA fwd+bwd step tokens/sec at 1/2/4/8 B200; per-kernel roofline %"


def _peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        return None


def _config(name):
    from r97training_b200.model import CONFIG4, CONFIG5
    return CONFIG5 if str(name) == "5" else CONFIG4


def _cfg_dict(cfg, model_groups, base_weights, adapter_params):
    return dict(hidden=cfg.hidden, ffn=cfg.ffn, rank=cfg.rank, alpha=cfg.alpha, vocab=cfg.vocab,
                gdn_heads=cfg.gdn_heads, gdn_qk_heads=cfg.gdn_qk_heads, seq=cfg.seq, micro_batch=cfg.micro_batch,
                kinds=cfg.kinds, groups=model_groups, base_weights=base_weights, adapter_params=adapter_params)


def _static_sizes(cfg):
    from r97training_b200.model import groups_of, has_lora
    groups = {k: groups_of(cfg, k) for k in ("gdn", "attn")}
    base = cfg.vocab * cfg.hidden
    adapter = 0
    for kind in cfg.kinds:
        for gname, k, projs in groups[kind]:
            for _, n in projs:
                base += n * k
                if has_lora(cfg, gname):
                    adapter += cfg.rank * (n + k)
    return groups, base, adapter


# The CPU sample's token count, the same for the cpu_baseline leg and (as the middle of its sweep) the
# reference arm; oracle.cpu_baseline fits each part between 8 tokens and this many, so the figure does not
# depend on it beyond timing noise.
CPU_SAMPLE_TOKENS = 64
CPU_SWEEP = (32, 64, 128)


def cpu_reference(cfg, sample_tokens=CPU_SAMPLE_TOKENS):
    """tokens/s of the reference's own host rows on a bounded sample (rank 0, N = 1 only)."""
    import oracle
    from oracle import cpu_baseline as CB
    if not oracle.ref_available():
        return None, None
    threads = CB.threads()
    os.environ.setdefault("R97_THREADS", str(threads))
    M = sample_tokens
    groups, base, adapter = _static_sizes(cfg)
    parts = CB.sample_step(_cfg_dict(cfg, groups, base, adapter), M)
    return 1.0 / parts["seconds_per_token"], dict(parts=parts, M=M, threads=threads)


def reference_arm(args):
    """--impl reference: the reference's CPU implementation of the path (its own host rows, compiled
    from its sources in oracle/_ref) on the host cores, K timed sample steps after W warm-ups."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cfg = _config(args.config)
    import oracle
    if not oracle.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "reference host library not built and reference tree absent"}))
        return 0
    from oracle import cpu_baseline as CB
    threads = CB.threads()
    os.environ.setdefault("R97_THREADS", str(threads))
    groups, base, adapter = _static_sizes(cfg)
    cd = _cfg_dict(cfg, groups, base, adapter)
    for _ in range(min(args.warmup, 1)):  # the rows are plain host code: one warm-up settles the caches
        CB.sample_step(cd, CPU_SAMPLE_TOKENS, seed=1)
    per_tok, sweep = [], {}
    t0 = time.perf_counter()
    for i in range(args.steps):
        M = CPU_SWEEP[i % len(CPU_SWEEP)]  # each step samples another token count of the sweep
        sp = CB.sample_step(cd, M, seed=2 + i)["seconds_per_token"]
        per_tok.append(sp)
        sweep.setdefault(str(M), []).append(sp)
    wall = time.perf_counter() - t0
    sec = sum(per_tok) / len(per_tok)
    value = 1.0 / sec
    M = "/".join(sorted(sweep, key=int))
    step_tokens = cfg.tokens
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": 0,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * step_tokens * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": f"config {args.config}: hybrid LoRA step, reference host rows on a {M}-token sample",
                   "model": "synthetic 9B-class hybrid (3 GDN : 1 gated attention)" if str(args.config) == "5" else
                   "synthetic small hybrid", "global_batch": cfg.micro_batch, "seq_len": cfg.seq,
                   "parallelism": "host threads"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "reference",
                         "sample": f"one GDN and one attention block's rows and the head fitted between 8 and {M} "
                                   "tokens (per-token slope + fixed per-call cost once a step), one 64-token GDN "
                                   "chunk, one 4096x4096 decode and a 16M AdamW, extrapolated per token",
                         "seconds_per_token_by_M": {k: sum(v) / len(v) for k, v in sweep.items()}},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": wall,
    }
    print(json.dumps(line), flush=True)
    return 0


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.proc, self.path = index, None, None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sms, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sms.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        if not sms:
            return None
        sms.sort()
        return {"sm_mhz": sms[len(sms) // 2], "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sms)}


def b200_arm(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    from r97training_b200 import ops
    from r97training_b200.model import Adapter, HybridModel, TrainStep, flops_per_token

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    cfg = _config(args.config)
    model = HybridModel(cfg, dev)
    adapter = Adapter(model, dev)
    step = TrainStep(model, adapter)

    buckets = None
    if world > 1:  # the adapter gradient's all-reduce: per layer while the walk goes on, or once at the end
        from r97training_b200.dp import GradBuckets
        buckets = GradBuckets(adapter.g, adapter.layer_ranges, overlap=args.dp_overlap)
        step.grad_hook = buckets.ready

    def one_step(ids):
        loss = step.run(ids)
        if buckets is not None:
            buckets.join()
        adapter.adamw()
        return loss

    gen = torch.Generator(device=dev)
    gen.manual_seed(1000 + rank)
    n_batches = args.warmup + args.steps
    ids_dev = [torch.randint(0, cfg.vocab, (cfg.micro_batch, cfg.seq), device=dev, generator=gen, dtype=torch.int32)
               for _ in range(min(n_batches, 4))]

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # warm-up: eager steps first (kernel attributes, encoders and buffers are set up on first use), then the
    # step is captured as one CUDA graph and the rest of the warm-up and every timed step replay it
    eager_warm = 1 if args.eager else min(2, max(1, args.warmup - 1))
    for i in range(eager_warm if not args.eager else args.warmup):
        one_step(ids_dev[i % len(ids_dev)])
    graph = None
    graph_launches = 0
    prof = []
    if not args.eager:
        from r97training_b200.model import GraphStep
        from r97training_b200._lib import lib as _lc
        barrier()
        ops.GEMM_PROFILE = prof  # the GEMMs' timing events become nodes of the graph
        c0 = int(_lc().r97b_launch_count())
        # the whole step in one graph; at N > 1 with the per-layer all-reduces captured on their side stream,
        # overlapping the rest of the backward, and AdamW after their join
        graph = GraphStep(step, ids_dev[0], update=True, buckets=buckets)
        graph_launches = int(_lc().r97b_launch_count()) - c0  # this library's kernels in the captured step
        ops.GEMM_PROFILE = None

        def one_step(ids):  # noqa: F811 -- the replayed step
            return graph.replay(ids)

        for i in range(eager_warm, args.warmup):
            one_step(ids_dev[i % len(ids_dev)])
    barrier()
    # ------------------------------------------------------------ timed: device-resident inputs
    sampler = ClockSampler(local)
    sampler.start()
    if graph is None:
        ops.GEMM_PROFILE = prof
    from r97training_b200._lib import lib as _l
    launches0 = int(_l().r97b_launch_count())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        loss = one_step(ids_dev[i % len(ids_dev)])
    e1.record()
    barrier()
    ops.GEMM_PROFILE = None
    # this library's kernels launched in the timed region: counted at launch from the host, or, when the
    # step is a replayed graph, the kernels captured in it times the replays
    own_launches = int(_l().r97b_launch_count()) - launches0 + graph_launches * (args.steps if graph else 0)
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    launches, gemm_ms, gemm_flops = ops.gemm_profile_summary(prof)
    if args.gemm_shapes and rank == 0:  # one step's GEMMs by shape, to stderr
        for shape, (n, gms, fl) in sorted(ops.gemm_profile_by_shape(prof).items(), key=lambda kv: -kv[1][1]):
            print(f"gemm {shape:48s} x{n:4d} {gms:8.3f} ms {fl / gms / 1e9 if gms else 0:7.0f} TFLOP/s",
                  file=sys.stderr)
    if graph is not None:  # the graph's events hold the last timed replay: one step's GEMMs
        launches, gemm_ms, gemm_flops = launches * args.steps, gemm_ms * args.steps, gemm_flops * args.steps
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    tokens = cfg.tokens * world * args.steps
    value = tokens / (ms / 1e3)
    # ------------------------------------------------------------ timed: e2e through the public API
    host_ids = [torch.randint(0, cfg.vocab, (cfg.micro_batch, cfg.seq), generator=torch.Generator().manual_seed(7 + i),
                              dtype=torch.int32).pin_memory() for i in range(2)]
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for i in range(args.steps):
        ids = host_ids[i % 2].to(dev, non_blocking=True)
        loss_host = float(one_step(ids).item())
    f1.record()
    barrier()
    ms_e2e = f0.elapsed_time(f1)
    t = torch.tensor([ms_e2e], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_e2e = float(t.item())
    e2e_value = tokens / (ms_e2e / 1e3)

    peaks = _peaks()
    if peaks:
        peak, peak_src = float(peaks.get("bf16_tflops_sustained") or peaks["bf16_tflops"]), "measured sustained"
    else:
        peak, peak_src = 1400.0, "fallback"
    gemm_tflops = gemm_flops / (gemm_ms / 1e3) / 1e12 if gemm_ms > 0 else 0.0
    traffic = None
    try:
        tr = json.load(open(os.path.join(ROOT, "profiles", "gemm_traffic.json")))
        traffic = tr.get("bytes_per_launch")
    except Exception:
        pass
    gpu_launches = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (uniform random token ids, seeded IQR base)",
            "config": {"workload": f"config {args.config}: full LoRA fwd+bwd+AdamW step of the random-init "
                                   f"{'9B-class' if str(args.config) == '5' else 'small'} hybrid",
                       "model": f"hybrid {cfg.layers}L d{cfg.hidden} 3xGDN:1xattn, IQR u4 base, LoRA r{cfg.rank}",
                       "global_batch": cfg.micro_batch * world, "seq_len": cfg.seq,
                       "parallelism": f"dp{world}", "l2": "inputs larger than L2 (about 60 GB of activations a step)",
                       "launch": "eager" if graph is None else
                       ("CUDA graph of the whole step" if world == 1 else
                        "CUDA graph of the whole step, per-layer gradient all-reduces captured on a side "
                        "stream overlapping the backward, AdamW after their join" if args.dp_overlap else
                        "CUDA graph of the whole step, one all-reduce of the gradient after the backward, "
                        "then AdamW"),
                       "flops_per_token": flops_per_token(cfg)},
            "roofline": {"bound": "tensor", "kernel": "gemm_kernel (tcgen05)", "achieved": gemm_tflops, "peak": peak,
                         "unit": "TFLOP/s", "frac": gemm_tflops / peak, "traffic": traffic,
                         "peak_source": peak_src, "launches_per_step": launches / max(args.steps, 1),
                         "gemm_ms_per_step": gemm_ms / max(args.steps, 1)},
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": cfg.tokens * 4,
                    "d2h_bytes_per_step": 4},
            "clocks": clocks,
            "loss": loss_host,
        }
        if world == 1 and not args.no_cpu_baseline:
            try:
                v, info = cpu_reference(cfg)
                if v is not None:
                    line["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": info["threads"],
                                            "kind": "reference",
                                            "sample": f"one GDN and one attention block's reference host rows and "
                                                      f"the head fitted between 8 and {info['M']} tokens (per-token "
                                                      "slope + fixed per-call cost once a step), one 64-token GDN "
                                                      "chunk, one 4096x4096 decode and a 16M AdamW, extrapolated "
                                                      "per token"}
            except Exception as e:  # the baseline is reported, not required
                line["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
        line["gpu_launches"] = own_launches
        line["gpu_launches_per_step"] = own_launches / max(args.steps, 1)
        print(json.dumps(line), flush=True)
    if graph is not None:
        graph.release()  # a graph holding NCCL calls goes before the process group
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def profile_case(case: str) -> None:
    """One small, self-contained case of a hot kernel, for profiling a few launches under ncu
    (`python bench.py --case NAME`): two or three launches of the kernel at a config-5 shape on operands
    larger than the 126 MB L2, then exit. NAME is one of

    gemm, gemm_dx   the config-5 gate_up forward GEMM (8192 x 24576 x 4096) / its input adjoint (B MN-major)
    gemm_swiglu     the gate_up forward as the step runs it: LoRA tail, SwiGLU in the epilogue
    gemm_swiglu_bwd the down projection's input adjoint with SwiGLU's adjoint in the epilogue (B MN-major)
    gemm_i8         the w8a8 trunk's int8 products at config-5 shapes: gemm_nt_q (8192 x 4096 x 4096) and the
                    gated fold with its Hadamard quantiser (8192 x 24576 x 4096), with CUDA-event timings
    gdn             one config-5 GDN layer, forward + backward
    decode          the IQR decode of a 24576 x 4096 weight
    norms / gnorm   rmsnorm fwd/bwd at 8192 x 4096 / gated rmsnorm at 8192 tokens x 32 heads x 128
    swiglu          SwiGLU fwd/bwd at 8192 x 12288
    loss            CE over 2048 x 151936 bf16 logits (one head chunk)
    adamw           AdamW over the config-5 adapter (160.4 M f32 params)
    conv            GDN conv prep fwd + bwd at 8192 tokens, 8192 channels
    attn            one config-5 attention core (B 2, 16 / 4 heads, S 4096, D 256), forward + backward, with
                    CUDA-event timings; attn_small the same at B 1, S 2048; attn_fwd the forward alone
    step            one config-5 training step after one warm-up step, inside an NVTX range "step"
    """
    import torch

    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    if case == "gemm_swiglu":
        from r97training_b200 import ops
        M, F, K, r = 8192, 12288, 4096, 128
        X = torch.randn(M, K, device=dev).bfloat16()
        W = (torch.randn(2 * F, K, device=dev) * 0.02).bfloat16()
        t = torch.randn(M, r, device=dev).bfloat16()
        Bb = (torch.randn(2 * F, r, device=dev) * 0.02).bfloat16()
        gu = torch.empty(M, 2 * F, device=dev, dtype=torch.bfloat16)
        a = torch.empty(M, F, device=dev, dtype=torch.bfloat16)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        for _ in range(3):
            ev[0].record()
            ops.gemm(X, W, gu, a2=t, b2=Bb, mode=ops.EPI_SWIGLU, out2=a)
            ev[1].record()
        torch.cuda.synchronize()
        ms = ev[0].elapsed_time(ev[1])
        print(f"gate_up + SwiGLU {M} x {2 * F} x {K + r}: {ms * 1e3:.1f} us, "
              f"{2 * M * 2 * F * (K + r) / ms / 1e9:.0f} TFLOP/s (third launch)")
    elif case == "gemm_swiglu_bwd":
        from r97training_b200 import ops
        M, F, K, r = 8192, 12288, 4096, 64
        dY = torch.randn(M, K, device=dev).bfloat16()
        W = (torch.randn(K, F, device=dev) * 0.02).bfloat16()  # the down projection [out K][in F]
        dt = torch.randn(M, r, device=dev).bfloat16()
        A = (torch.randn(r, F, device=dev) * 0.02).bfloat16()
        gu = torch.randn(M, 2 * F, device=dev).bfloat16()
        dgu = torch.empty(M, 2 * F, device=dev, dtype=torch.bfloat16)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        for _ in range(3):
            ev[0].record()
            ops.gemm(dY, W, dgu, b_mn=True, a2=dt, b2=A, N=F, mode=ops.EPI_SWIGLU_BWD, addend=gu)
            ev[1].record()
        torch.cuda.synchronize()
        ms = ev[0].elapsed_time(ev[1])
        print(f"down-projection dX + SwiGLU adjoint {M} x {F} x {K + r}: {ms * 1e3:.1f} us, "
              f"{2 * M * F * (K + r) / ms / 1e9:.0f} TFLOP/s (third launch)")
    elif case == "gemm_i8":
        from r97training_b200 import ops
        M, K = 8192, 4096
        a = torch.randint(-127, 128, (M, K), device=dev, dtype=torch.int8)
        sa = torch.rand(M, K // 128, device=dev) * 0.01
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        for N, gated in ((4096, False), (24576, True)):
            b = torch.randint(-127, 128, (N, K), device=dev, dtype=torch.int8)
            sb = torch.rand(N, K // 128, device=dev) * 0.002
            y = None if gated else torch.empty(M, N, device=dev, dtype=torch.bfloat16)
            for _ in range(3):
                ev[0].record()
                if gated:
                    ops.gemm_i8g_gated(a, sa, b, sb)
                else:
                    ops.gemm_i8g(a, sa, b, sb, y=y)
                ev[1].record()
            torch.cuda.synchronize()
            ms = ev[0].elapsed_time(ev[1])
            print(f"int8 {'gated fold' if gated else 'gemm_nt_q'} {M} x {N} x {K}: {ms * 1e3:.1f} us, "
                  f"{2 * M * N * K / ms / 1e9:.0f} TOP/s (third launch)")
    elif case in ("gemm", "gemm_dx"):
        from r97training_b200 import ops
        M, N, K = 8192, 24576, 4096
        X = torch.randn(M, K, device=dev).bfloat16()
        W = (torch.randn(N, K, device=dev) * 0.02).bfloat16()
        if case == "gemm":
            Y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
            for _ in range(3):
                ops.gemm(X, W, Y)
        else:
            dY = torch.randn(M, N, device=dev).bfloat16()
            dX = torch.empty(M, K, device=dev, dtype=torch.bfloat16)
            for _ in range(3):
                ops.gemm(dY, W, dX, b_mn=True, N=K)
    elif case == "gdn":
        from r97training_b200.gdn import GdnPlan
        T, H, Hg = 8192, 32, 16
        q = torch.nn.functional.normalize(torch.randn(T, Hg, 128, device=dev), dim=-1).bfloat16()
        k = torch.nn.functional.normalize(torch.randn(T, Hg, 128, device=dev), dim=-1).bfloat16()
        v = torch.randn(T, H, 128, device=dev).bfloat16()
        g = (-torch.nn.functional.softplus(torch.randn(T, H, device=dev))).view(-1, 64, H).cumsum(1).view(T, H)
        beta = torch.sigmoid(torch.randn(T, H, device=dev))
        do = (torch.randn(T, H, 128, device=dev) * 1e-2).bfloat16()
        plan = GdnPlan([0, 4096, 8192], H, Hg, dev)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        fwd = bwd = 0.0
        for it in range(2):
            ev[0].record()
            o, _, sv = plan.forward(q, k, v, g.contiguous(), beta)
            ev[1].record()
            plan.backward(sv, do)
            ev[2].record()
            torch.cuda.synchronize()
            fwd, bwd = ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])
        print(f"gdn layer T {T} H {H} Hg {Hg}: forward {fwd:.3f} ms, backward {bwd:.3f} ms (second pass)")
    elif case == "decode":
        from r97training_b200 import iqr as IQ
        w = IQ.synth_weight(24576, 4096, seed=1, device=dev)
        out = torch.empty(24576, 4096, dtype=torch.bfloat16, device=dev)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        for _ in range(3):
            ev[0].record()
            IQ.dequant_bf16(w, out=out)
            ev[1].record()
        torch.cuda.synchronize()
        print(f"iqr decode 24576 x 4096 -> bf16: {ev[0].elapsed_time(ev[1]) * 1e3:.1f} us (third launch)")
    elif case == "norms":
        from r97training_b200 import ops
        x = torch.randn(8192, 4096, device=dev).bfloat16()
        dy = torch.randn(8192, 4096, device=dev).bfloat16()
        w = torch.ones(4096, device=dev)
        for _ in range(3):
            ops.rmsnorm_fwd(x, w)
            ops.rmsnorm_bwd(x, w, dy, addend=dy)
    elif case == "gnorm":
        from r97training_b200 import ops
        T, H = 8192, 32
        x = torch.randn(T * H, 128, device=dev).bfloat16()
        z = torch.randn(T, H * 128, device=dev).bfloat16()
        do = torch.randn(T * H, 128, device=dev).bfloat16()
        w = torch.ones(128, device=dev)
        dx, dz = torch.empty_like(x), torch.empty_like(z)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        for _ in range(3):
            ev[0].record()
            ops.gated_rmsnorm_fwd(x, z, w)
            ev[1].record()
            ops.gated_rmsnorm_bwd(x, z, w, do, dx=dx, dz=dz)
            ev[2].record()
        torch.cuda.synchronize()
        print(f"gated rmsnorm {T * H} rows x 128: forward {ev[0].elapsed_time(ev[1]) * 1e3:.1f} us, "
              f"backward {ev[1].elapsed_time(ev[2]) * 1e3:.1f} us (third pass)")
    elif case == "swiglu":
        from r97training_b200 import ops
        T, F = 8192, 12288
        gu = torch.randn(T, 2 * F, device=dev).bfloat16()
        y = torch.empty(T, F, device=dev, dtype=torch.bfloat16)
        dy = torch.randn(T, F, device=dev).bfloat16()
        dgu = torch.empty_like(gu)
        for _ in range(3):
            ops.swiglu_fwd(gu, y)
            ops.swiglu_bwd(gu, dy, dgu)
    elif case == "loss":
        from r97training_b200 import ops
        rows, vocab = 2048, 151936
        logits = (torch.randn(rows, vocab, device=dev) * 2).bfloat16()
        tgt = torch.randint(0, vocab, (rows,), device=dev, dtype=torch.int32)
        loss = torch.empty(rows, device=dev)
        grad = torch.empty_like(logits)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        for _ in range(3):
            ev[0].record()
            ops.ce_kld(logits, tgt, loss_ce=loss, grad=grad, grad_scale=1.0 / rows)
            ev[1].record()
        torch.cuda.synchronize()
        us = ev[0].elapsed_time(ev[1]) * 1e3
        print(f"CE {rows} x {vocab} bf16 logits: {us:.1f} us, {2 * 2 * rows * vocab / us / 1e3:.0f} GB/s "
              "(logits read + gradient written, third launch)")
    elif case == "adamw":
        from r97training_b200 import ops
        n = 160_432_128
        w = torch.randn(n, device=dev) * 0.01
        m, v, g = torch.zeros_like(w), torch.zeros_like(w), torch.randn(n, device=dev) * 1e-3
        for i in range(3):
            ops.adamw_step(w, m, v, g, lr=1e-4, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.0,
                           bc1=1.0 - 0.9 ** (i + 1), bc2=1.0 - 0.999 ** (i + 1))
    elif case == "conv":
        from r97training_b200 import ops
        T, Hg, H = 8192, 16, 32
        C = (2 * Hg + H) * 128
        x = torch.randn(T, C + 8256, device=dev).bfloat16()
        cw = torch.randn(C, 4, device=dev) * 0.5
        cu = torch.tensor([0, 4096, 8192], dtype=torch.int32, device=dev)
        q = torch.empty(T, Hg, 128, device=dev, dtype=torch.bfloat16)
        k, v = torch.empty_like(q), torch.empty(T, H, 128, device=dev, dtype=torch.bfloat16)
        dq, dk, dv = (torch.randn(T, H, 128, device=dev) for _ in range(3))
        dx = torch.zeros_like(x)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        for _ in range(3):
            ev[0].record()
            ops.conv_prep_fwd(x, cw, cu, 2, Hg, H, q, k, v)
            ev[1].record()
            ops.conv_prep_bwd(x, cw, cu, 2, Hg, H, dq, dk, dv, dx)
            ev[2].record()
        torch.cuda.synchronize()
        print(f"conv prep {T} tokens x {C} channels: forward {ev[0].elapsed_time(ev[1]) * 1e3:.1f} us, "
              f"backward {ev[1].elapsed_time(ev[2]) * 1e3:.1f} us (third pass)")
    elif case == "attn_fwd":
        from r97training_b200 import ops
        B, Hq, Hkv, S, D = 2, 16, 4, 4096, 256
        q = torch.randn(B, Hq, S, D, device=dev).bfloat16()
        k = torch.randn(B, Hkv, S, D, device=dev).bfloat16()
        v = torch.randn(B, Hkv, S, D, device=dev).bfloat16()
        for _ in range(3):
            ops.attn_fwd(q, k, v, D ** -0.5)
    elif case in ("attn", "attn_small"):
        from r97training_b200 import ops
        B, Hq, Hkv, S, D = (2, 16, 4, 4096, 256) if case == "attn" else (1, 16, 4, 2048, 256)
        q = torch.randn(B, Hq, S, D, device=dev).bfloat16()
        k = torch.randn(B, Hkv, S, D, device=dev).bfloat16()
        v = torch.randn(B, Hkv, S, D, device=dev).bfloat16()
        do = (torch.randn(B, Hq, S, D, device=dev) * 0.1).bfloat16()
        ws = ops.attn_bwd_workspace(B, Hq, S, dev)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        fw, bw = [], []
        for _ in range(3):
            ev[0].record()
            o, lse = ops.attn_fwd(q, k, v, D ** -0.5)
            ev[1].record()
            ops.attn_bwd(q, k, v, o, do, lse, D ** -0.5, ws)
            ev[2].record()
            torch.cuda.synchronize()
            fw.append(ev[0].elapsed_time(ev[1]))
            bw.append(ev[1].elapsed_time(ev[2]))
        causal = 4.0 * B * Hq * (S * (S + 128) / 2) * D  # QK^T and PV over the causal tiles (128-row blocks)
        print(f"attention B{B} Hq{Hq} Hkv{Hkv} S{S} D{D}: forward {min(fw):.3f} ms "
              f"({causal / min(fw) / 1e9:.0f} TFLOP/s of the causal 2-product work), backward {min(bw):.3f} ms "
              f"({2.5 * causal / min(bw) / 1e9:.0f} TFLOP/s of 2.5 x that)")
    elif case == "step":
        from r97training_b200.model import CONFIG5, Adapter, HybridModel, TrainStep
        model = HybridModel(CONFIG5, dev)
        adapter = Adapter(model, dev)
        step = TrainStep(model, adapter)
        gen = torch.Generator(device=dev)
        gen.manual_seed(5)
        ids = torch.randint(0, CONFIG5.vocab, (CONFIG5.micro_batch, CONFIG5.seq), device=dev, generator=gen,
                            dtype=torch.int32)
        step.run(ids)
        adapter.adamw()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("step")
        step.run(ids)
        adapter.adamw()
        torch.cuda.nvtx.range_pop()
    else:
        raise SystemExit(f"unknown case {case}")
    torch.cuda.synchronize()



def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="5")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--gemm-shapes", action="store_true", help="print one step's GEMM time by shape to stderr")
    ap.add_argument("--dp-overlap", type=int, default=0,
                    help="N > 1: 1 = per-layer gradient all-reduces on a side stream during the backward, "
                         "0 = one all-reduce of the whole gradient after it (measured no slower at 8 GPUs: the "
                         "collective's kernels slow the backward's persistent kernels as much as they hide)")
    ap.add_argument("--eager", action="store_true", help="launch every kernel from the host each step "
                    "instead of replaying the step captured as a CUDA graph")
    ap.add_argument("--case", default=None, help="run one small kernel case for ncu instead of the bench "
                    "(see profile_case)")
    args = ap.parse_args()
    if args.case:
        profile_case(args.case)
        return 0
    if args.impl == "reference":
        return reference_arm(args)
    return b200_arm(args)


if __name__ == "__main__":
    sys.exit(main())
