"""Benchmark of the hybrid-attention hot path.

Workload ("step"): batched hybrid decode -- 64 sequences per GPU, each with a
ragged KV cache of L_i ~ U{512..32768} cached positions (seeded), advance one
token through one gated GQA layer (dz_gqa_decode) and one Gated DeltaNet layer
(dz_gdn_decode).  Inputs are synthetic N(0,1) activations (projections are out
of scope), KV contents N(0,1), DeltaNet state N(0, 0.02).  Sequence-sharded
across GPUs with no collective: every rank owns its own 64 sequences (weak
scaling).  The per-step KV + state traffic (~9 GB) is far above the 126 MB L2,
so no flush is needed between steps.

Metric: decode tokens/s (whole job), with the achieved HBM GB/s of the
dominant kernel group against the measured copy bandwidth.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
import argparse
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "hybrid-attn decode tok/s + % HBM BW; prefill attn TFLOP/s vs peak"
B_PER_RANK = 64
LEN_LO, LEN_HI = 512, 32768
SEED0 = 0xDA12A000 + 2      # config 2

HQ, HKV, GRP, HD = 24, 4, 6, 256
SSM_HV, SSM_D, QKV_LEN, INNER = 48, 128, 10240, 6144


def seq_lengths(rank):
    rng = np.random.default_rng(SEED0 + 7919 * rank)
    return rng.integers(LEN_LO, LEN_HI + 1, size=B_PER_RANK).astype(np.int64)


def layer_params(seed):
    """Seeded synthetic parameters: norm weights ~ U(0.5,1.5), conv w ~ N(0,0.5),
    ssm_a = -exp(U(0,2.7)), dt_bias = 0."""
    rng = np.random.default_rng(seed)
    f = np.float32
    q_norm = rng.uniform(0.5, 1.5, HD).astype(f)
    k_norm = rng.uniform(0.5, 1.5, HD).astype(f)
    conv_w = rng.normal(0.0, 0.5, (4, QKV_LEN)).astype(f)
    ssm_a = (-np.exp(rng.uniform(0.0, 2.7, SSM_HV))).astype(f)
    dt_bias = np.zeros(SSM_HV, f)
    norm_w = rng.uniform(0.5, 1.5, SSM_D).astype(f)
    return (q_norm, k_norm), (conv_w, ssm_a, dt_bias, norm_w)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


# algorithmic bytes (SURVEY 8d formulas, counted per step)
def gqa_bytes(lens_before):
    n = np.asarray(lens_before, np.int64) + 1
    kv_read = int(n.sum()) * HKV * HD * 4 * 2
    per_seq = HQ * 2 * HD * 4 + HKV * HD * 4 * 2 + HQ * HD * 4      # q_gate in, k/v append, out
    return kv_read + len(n) * per_seq + 2 * HD * 4


def gdn_bytes(B):
    per_seq = (2 * SSM_HV * SSM_D * SSM_D * 4            # state read + write
               + 3 * QKV_LEN * 4 + QKV_LEN * 4          # 3 history rows read, 1 written
               + QKV_LEN * 4 + 2 * SSM_HV * 4           # qkv, alpha, beta
               + INNER * 4 * 2)                         # z in, y out
    return B * per_seq + 4 * QKV_LEN * 4 + (2 * SSM_HV + SSM_D) * 4   # + conv weights and params once


class Clocks:
    """Samples nvidia-smi (clocks and throttle reasons) around the timed region.

    Sampling starts before the timed region and stops after it; samples whose
    timestamp falls inside [start, end] are reported.  When the timed region is
    shorter than the sampling interval, the nearest samples on either side are
    reported instead and "window" says so."""
    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id, period_ms=50):
        self.gpu_id = gpu_id          # nvidia-smi id (UUID), independent of CUDA_VISIBLE_DEVICES
        self.period_ms = period_ms
        self.proc = None
        self.raw = ""
        self.t0 = self.t1 = None

    def start(self):
        import datetime
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu_id}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", str(self.period_ms)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            time.sleep(1.0)           # let the sampler produce its first rows
        except (FileNotFoundError, OSError):
            self.proc = None
        self._now = datetime.datetime.now

    def mark_start(self):
        self.t0 = self._now() if self.proc else None

    def mark_end(self):
        self.t1 = self._now() if self.proc else None

    def stop(self):
        import datetime
        if self.proc is None:
            return None
        time.sleep(0.3)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        self.raw = out
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        rows = []
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f")
                rows.append((ts, float(f[2]), float(f[3]), [n for n, v in zip(names, f[6:10])
                                                          if v.lower().startswith("active")]))
            except ValueError:
                continue
        if not rows or self.t0 is None:
            return None
        inside = [r for r in rows if self.t0 <= r[0] <= self.t1]
        window = "timed region"
        if not inside:
            before = [r for r in rows if r[0] < self.t0][-1:]
            after = [r for r in rows if r[0] > self.t1][:1]
            inside = before + after
            window = "nearest samples around a timed region shorter than the sampling period"
        reasons = sorted({n for r in inside for n in r[3]})
        return {"sm_mhz": float(np.median([r[1] for r in inside])), "sm_max_mhz": inside[0][2],
                "reasons": reasons, "samples": len(inside), "window": window}


# ---------------------------------------------------------------------------
# reference arm / CPU baseline: the oracle (C++ restatement of the AVX2 path)
# ---------------------------------------------------------------------------
class CpuWorkload:
    """A bounded sample of config 2 for the oracle (C++ restatement of the
    reference's AVX2 path): n_seq of the 64 sequences (evenly spaced, their real
    lengths), built once; step() advances every sampled sequence by one token
    through both layers."""

    def __init__(self, n_seq, max_steps, rank=0):
        import oracle as O
        self.O = O
        lens = seq_lengths(rank)
        self.pick = lens[:: max(1, B_PER_RANK // n_seq)][:n_seq]
        (self.qn, self.kn), self.p = layer_params(SEED0)
        self.kvs, self.sts = [], []
        for i, n in enumerate(self.pick):
            kv = O.OracleKv(int(n) + max_steps)
            kv.k[:, :n] = O.normal(SEED0 + 500 + i, (HKV, int(n), HD))
            kv.v[:, :n] = O.normal(SEED0 + 600 + i, (HKV, int(n), HD))
            kv.len = int(n)
            self.kvs.append(kv)
            self.sts.append(O.OracleSsm(O.normal(SEED0 + 700 + i, (SSM_HV, SSM_D, SSM_D), 0.0, 0.02),
                                        O.normal(SEED0 + 800 + i, (4, QKV_LEN)), 0))
        Bs = len(self.pick)
        self.qg = O.normal(SEED0 + 1, (Bs, HQ * 2 * HD))
        self.k = O.normal(SEED0 + 2, (Bs, HKV * HD))
        self.v = O.normal(SEED0 + 3, (Bs, HKV * HD))
        self.qkv = O.normal(SEED0 + 4, (Bs, QKV_LEN))
        self.a = O.normal(SEED0 + 5, (Bs, SSM_HV))
        self.b = O.normal(SEED0 + 6, (Bs, SSM_HV))
        self.z = O.normal(SEED0 + 7, (Bs, INNER))

    def step(self, n_threads):
        t0 = time.perf_counter()
        self.O.gqa_decode_batch(self.qg, self.k, self.v, self.qn, self.kn, self.kvs, n_threads=n_threads)
        self.O.gdn_decode_batch(self.qkv, self.a, self.b, self.z, self.p, self.sts, n_threads=n_threads)
        return time.perf_counter() - t0


def cpu_baseline(n_seq_sample=8, steps=1, n_threads=1, rank=0):
    w = CpuWorkload(n_seq_sample, steps, rank)
    dt = sum(w.step(n_threads) for _ in range(steps))
    return len(w.pick) * steps / dt, dt, w.pick


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cores = os.cpu_count() or 1
    n_seq = min(cores, 32)
    w = CpuWorkload(n_seq, args.warmup + args.steps, rank)
    for _ in range(args.warmup):
        w.step(cores)
    dts = [w.step(cores) for _ in range(args.steps)]
    wall = sum(dts)
    value = len(w.pick) * args.steps / wall
    sample = (f"{len(w.pick)} of the 64 config-2 sequences (evenly spaced, real lengths, "
              f"{int(np.sum(w.pick))} cached tokens), one decode step of both layers per timed step; "
              f"one sequence per thread on {cores} host threads (harness parallelisation: the reference "
              "decodes one sequence at a time)")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * wall / max(1, args.steps),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": "config 2: batched hybrid decode, 64 seqs/GPU, "
                                                        "KV U{512..32768}, 1 GQA + 1 GDN layer"},
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args):
    import torch
    import daiza_b200 as dz

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)

    lens = seq_lengths(rank)[: args.seqs]
    total_steps = args.warmup + args.steps + args.e2e_steps + 2
    cfg = dz.default_config(n_layers=2, full_attention_interval=2)   # layer 0 GDN, layer 1 GQA
    ctx = dz.Context(local, cfg)
    (qn, kn), sp = layer_params(SEED0)
    ctx.set_attn_params(1, qn, kn)
    ctx.set_ssm_params(0, *sp)
    ctx.cache_create(lens + total_steps)
    g = torch.Generator(device=dev)
    g.manual_seed(SEED0 + rank)
    for s, n in enumerate(lens):
        kf = torch.randn(int(n), HKV, HD, device=dev, generator=g)
        vf = torch.randn(int(n), HKV, HD, device=dev, generator=g)
        ctx.kv_import(1, s, kf, vf)
        del kf, vf
        st = torch.randn(SSM_HV, SSM_D, SSM_D, device=dev, generator=g) * 0.02
        hist = torch.randn(4, QKV_LEN, device=dev, generator=g)
        ctx.ssm_import(0, s, st, hist, 0)
    torch.cuda.synchronize()
    B = len(lens)
    ids = np.arange(B, dtype=np.int32)
    qg = torch.randn(B, HQ * 2 * HD, device=dev, generator=g)
    kk = torch.randn(B, HKV * HD, device=dev, generator=g)
    vv = torch.randn(B, HKV * HD, device=dev, generator=g)
    qkv = torch.randn(B, QKV_LEN, device=dev, generator=g)
    al = torch.randn(B, SSM_HV, device=dev, generator=g)
    be = torch.randn(B, SSM_HV, device=dev, generator=g)
    z = torch.randn(B, INNER, device=dev, generator=g)
    out = torch.empty(B, HQ * HD, device=dev)
    y = torch.empty(B, INNER, device=dev)
    stream = torch.cuda.current_stream()

    def step():
        ctx.gqa_decode(1, ids, qg, kk, vv, out)
        n1 = ctx.last_launch_count
        ctx.gdn_decode(0, ids, qkv, al, be, z, y)
        return n1 + ctx.last_launch_count

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()

    lens_at = np.array([ctx.kv_len(1, s) for s in range(B)], np.int64)
    uuid = str(torch.cuda.get_device_properties(dev).uuid)
    clocks = Clocks(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
    clocks.start()
    clocks.mark_start()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    launches = 0
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(args.steps):
        ev[i][0].record(stream)
        ctx.gqa_decode(1, ids, qg, kk, vv, out)
        launches += ctx.last_launch_count
        ev[i][1].record(stream)
        ctx.gdn_decode(0, ids, qkv, al, be, z, y)
        launches += ctx.last_launch_count
        ev[i][2].record(stream)
    t_end.record(stream)
    torch.cuda.synchronize()
    clocks.mark_end()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = t_start.elapsed_time(t_end)
    gqa_ms = [ev[i][0].elapsed_time(ev[i][1]) for i in range(args.steps)]
    gdn_ms = [ev[i][1].elapsed_time(ev[i][2]) for i in range(args.steps)]
    if dist:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = world * B * args.steps / (ms / 1000.0)

    # bytes per step of the dominant kernel group (GQA decode: prep + split-K + combine)
    gqa_b = np.mean([gqa_bytes(lens_at + i) for i in range(args.steps)])
    gdn_b = gdn_bytes(B)
    hbm, bf16, peak_kind = peaks()
    gqa_gbs = gqa_b / (np.mean(gqa_ms) / 1000.0) / 1e9
    gdn_gbs = gdn_b / (np.mean(gdn_ms) / 1000.0) / 1e9
    step_gbs = (gqa_b + gdn_b) / (ms / args.steps / 1000.0) / 1e9

    # end-to-end through the public C ABI host entry points (pinned host buffers)
    e2e = None
    if args.e2e_steps > 0:
        hq = torch.empty(B, HQ * 2 * HD, pin_memory=True)
        hq.copy_(qg.cpu())
        hk = kk.cpu().pin_memory()
        hv = vv.cpu().pin_memory()
        hx = qkv.cpu().pin_memory()
        ha = al.cpu().pin_memory()
        hb = be.cpu().pin_memory()
        hz = z.cpu().pin_memory()
        ho = torch.empty(B, HQ * HD, pin_memory=True)
        hy = torch.empty(B, INNER, pin_memory=True)
        np_views = [t.numpy() for t in (hq, hk, hv, hx, ha, hb, hz, ho, hy)]
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.e2e_steps):
            ctx.gqa_decode_host(1, ids, np_views[0], np_views[1], np_views[2], np_views[7])
            ctx.gdn_decode_host(0, ids, np_views[3], np_views[4], np_views[5], np_views[6], np_views[8])
        e1.record(stream)
        torch.cuda.synchronize()
        ems = e0.elapsed_time(e1)
        if dist:
            t = torch.tensor([ems], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ems = float(t.item())
        h2d = B * (HQ * 2 * HD + 2 * HKV * HD + QKV_LEN + 2 * SSM_HV + INNER) * 4
        d2h = B * (HQ * HD + INNER) * 4
        e2e = {"value": world * B * args.e2e_steps / (ems / 1000.0), "unit": "tok/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "path": "dz_gqa_decode_host + dz_gdn_decode_host (pinned host buffers, copies inside the timed region)",
               "steps": args.e2e_steps}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        v, dt, pick = cpu_baseline(n_seq_sample=8, steps=args.cpu_steps, n_threads=1)
        cpu = {"value": v, "unit": "tok/s", "cores": 1, "kind": "port",
               "sample": f"8 of the 64 sequences (lengths {list(map(int, pick))}), {args.cpu_steps} decode step(s) "
                         f"of both layers, single thread like the reference's decode attention/scan; {dt:.2f} s"}

    prefill = None
    if not args.no_prefill:
        prefill = run_prefill(dz, torch, local, args)

    err = ctx.device_error()
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": "config 2: batched hybrid decode, 64 seqs/GPU, KV lengths U{512..32768} "
                                       "(seeded), 1 gated GQA + 1 Gated DeltaNet layer, f32 caches",
                           "seqs_per_gpu": B, "kv_tokens_per_gpu": int(lens_at.sum()),
                           "parallelism": f"sequence-sharded x{world}, no collective",
                           "l2": "no flush: per-step KV+state traffic ~9 GB >> 126 MB L2"},
                "hbm_gbs_step": step_gbs, "hbm_frac_step": step_gbs / hbm,
                "roofline": {"bound": "hbm", "kernel": "dz_gqa_decode (prep + split-K + combine)",
                             "achieved": gqa_gbs, "peak": hbm, "unit": "GB/s", "frac": gqa_gbs / hbm,
                             "traffic": None, "peak_kind": f"{peak_kind} hbm_gbs",
                             "bytes_per_launch": gqa_b, "ms_per_launch": float(np.mean(gqa_ms))},
                "gdn": {"achieved_gbs": gdn_gbs, "frac": gdn_gbs / hbm, "bytes": gdn_b,
                        "ms": float(np.mean(gdn_ms))},
                "gpu_launches": launches, "clocks": clk, "e2e": e2e, "cpu_baseline": cpu, "prefill": prefill,
                "device_error": err}
        if clk is None and clocks.raw:
            line["clocks_raw_head"] = clocks.raw[:300]
        print(json.dumps(line))
    ctx.close()
    if dist:
        dist.destroy_process_group()
    return 0


PF_T = 8192


def run_prefill(dz, torch, local, args):
    """Config 3 GQA prefill: one sequence, T=8192 bf16 tokens, positions 0..8191,
    through dz_gqa_prefill_bf16 (prep + tcgen05 attention).  FLOPs counted as
    4 * 24 * 256 * sum_{t<T}(t+1) (QK^T and PV over the causal range)."""
    dev = torch.device("cuda", local)
    cfg = dz.default_config(n_layers=2, full_attention_interval=2)
    ctx = dz.Context(local, cfg)
    (qn, kn), sp = layer_params(SEED0 + 3)
    ctx.set_attn_params(1, qn, kn)
    ctx.set_ssm_params(0, *sp)
    ctx.cache_create([PF_T])
    g = torch.Generator(device=dev)
    g.manual_seed(SEED0 + 3)
    qg = torch.randn(PF_T, HQ * 2 * HD, device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn(PF_T, HKV * HD, device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn(PF_T, HKV * HD, device=dev, generator=g).to(torch.bfloat16)
    out = torch.empty(PF_T, HQ * HD, device=dev)
    stream = torch.cuda.current_stream()
    iters = max(3, args.prefill_iters)
    for _ in range(3):
        ctx.kv_truncate(1, 0, 0)
        ctx.gqa_prefill(1, 0, qg, k, v, out)
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        ctx.kv_truncate(1, 0, 0)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        ctx.gqa_prefill(1, 0, qg, k, v, out)
        e1.record(stream)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    launches = ctx.last_launch_count
    # Gated DeltaNet prefill, same T: f32 qkv/alpha/beta/z, zero state and history
    qkv = torch.randn(PF_T, QKV_LEN, device=dev, generator=g)
    al = torch.randn(PF_T, SSM_HV, device=dev, generator=g)
    be = torch.randn(PF_T, SSM_HV, device=dev, generator=g)
    z = torch.randn(PF_T, INNER, device=dev, generator=g)
    y = torch.empty(PF_T, INNER, device=dev)
    zero_state = torch.zeros(SSM_HV, SSM_D, SSM_D, device=dev)
    zero_hist = torch.zeros(4, QKV_LEN, device=dev)
    gtimes = []
    for it in range(3 + iters):
        ctx.ssm_import(0, 0, zero_state, zero_hist, 0)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        ctx.gdn_prefill(0, 0, qkv, al, be, z, y)
        e1.record(stream)
        torch.cuda.synchronize()
        if it >= 3:
            gtimes.append(e0.elapsed_time(e1))
    glaunches = ctx.last_launch_count
    ctx.close()
    gms = float(np.median(gtimes))
    C, d = 64, SSM_D
    g_flops = (PF_T // C) * SSM_HV * (10 * C * C * d + 6 * C * d * d + (2 / 3) * C ** 3)
    g_bytes = PF_T * (QKV_LEN + 2 * SSM_HV + 2 * INNER) * 4 + SSM_HV * SSM_D * SSM_D * 4 * 2
    hbm, _, _ = peaks()
    gdn = {"workload": "config 3 Gated DeltaNet prefill, T=8192, f32, chunk 64, zero state",
           "ms": gms, "algorithmic_gflop": g_flops / 1e9, "tflops": g_flops / (gms / 1000.0) / 1e12,
           "bytes": g_bytes, "gbs": g_bytes / (gms / 1000.0) / 1e9, "hbm_frac": g_bytes / (gms / 1000.0) / 1e9 / hbm,
           "launches_per_call": glaunches,
           "note": "f32 CUDA-core WY/UT chunk kernels (intra-chunk parallel, inter-chunk sequential per head)"}
    flops = 4.0 * HQ * HD * (PF_T * (PF_T + 1) / 2)
    ms = float(np.median(times))
    tf = flops / (ms / 1000.0) / 1e12
    _, bf16, kind = peaks()
    return {"workload": "config 3 GQA prefill, T=8192, bf16 q/k/v, 24/4 heads, D=256, causal",
            "ms": ms, "tflops": tf, "peak_tflops": bf16, "frac": tf / bf16, "peak_kind": f"{kind} bf16_tflops (burst)",
            "flops": flops, "iters": iters, "launches_per_call": launches,
            "timed": "dz_gqa_prefill_bf16 = prep (norm/rope/cache append) + tcgen05 attention, median of iters",
            "gdn": gdn}


def run_stack(args):
    """Config 4: the 64-layer attention stack (48 Gated DeltaNet + 16 GQA layers),
    head-sharded over the ranks with an NCCL all-gather of head outputs after
    every layer.  Decode: batch 8 at context 131072 (KV rows are a synthetic byte
    pattern).  Prefill: one sequence of 32768 tokens."""
    import datetime
    import torch
    import torch.distributed as dist
    from daiza_b200 import parallel as P
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29555")
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=300),
                                device_id=dev)
    B, CTX, T = 8, args.stack_ctx, args.stack_prefill
    steps, warm = args.steps, args.warmup
    plan = P.head_plan(world, rank)
    rows = plan.decode_rows(B)
    caps = [(CTX + steps + warm + 2) if b in rows else 1 for b in range(B)] + [T]

    def params(layer, kind):
        a, s_ = layer_params(SEED0 + 4 * 1000 + layer)
        return a if kind == "attn" else s_

    stack = P.ShardedStack(local, B, caps, params)
    t0 = time.time()
    for layer in range(64):
        if stack.ctx.is_attention(layer):
            for b in rows:
                stack.ctx.kv_fill_pattern(layer, b, CTX, 0x3C)
    torch.cuda.synchronize()
    fill_s = time.time() - t0
    g = torch.Generator(device=dev)
    g.manual_seed(SEED0 + 4)
    qg = torch.randn(B, HQ * 2 * HD, device=dev, generator=g)
    k = torch.randn(B, HKV * HD, device=dev, generator=g)
    v = torch.randn(B, HKV * HD, device=dev, generator=g)
    gdn = tuple(torch.randn(B, n, device=dev, generator=g) for n in (QKV_LEN, SSM_HV, SSM_HV, INNER))
    sq, sk, sv = stack.slice_inputs(qg, k, v)
    gqa_in = tuple(x[rows[0]:rows[-1] + 1].contiguous() for x in (sq, sk, sv))
    stream = torch.cuda.current_stream()
    for _ in range(warm):
        stack.decode_step(gqa_in, gdn)
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        stack.decode_step(gqa_in, gdn)
    e1.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    dms = torch.tensor([e0.elapsed_time(e1) / steps], device=dev)
    dist.all_reduce(dms, op=dist.ReduceOp.MAX)
    dms = float(dms.item())
    # bytes per decode step on this rank: its KV rows (incl. new token) + its DeltaNet states
    ctx_now = CTX + warm + steps // 2
    kvc = plan.kv_heads[1] - plan.kv_heads[0]
    vc = plan.v_heads[1] - plan.v_heads[0]
    rank_bytes = 16 * len(rows) * (ctx_now + 1) * kvc * HD * 4 * 2 + 48 * B * vc * SSM_D * SSM_D * 4 * 2
    hbm, bf16, kind = peaks()
    # prefill
    pg = torch.randn(T, HQ * 2 * HD, device=dev, generator=g).to(torch.bfloat16)
    pk = torch.randn(T, HKV * HD, device=dev, generator=g).to(torch.bfloat16)
    pv = torch.randn(T, HKV * HD, device=dev, generator=g).to(torch.bfloat16)
    pgdn = tuple(torch.randn(T, n, device=dev, generator=g) for n in (QKV_LEN, SSM_HV, SSM_HV, INNER))
    pin = stack.slice_inputs(pg, pk, pv)
    ptimes = []
    for it in range(1 + args.stack_prefill_iters):
        stack.ctx.cache_reset(B)
        torch.cuda.synchronize()
        dist.barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        stack.prefill(B, pin, pgdn)
        a1.record(stream)
        torch.cuda.synchronize()
        if it > 0:
            ptimes.append(a0.elapsed_time(a1))
    pms = torch.tensor([float(np.median(ptimes))], device=dev)
    dist.all_reduce(pms, op=dist.ReduceOp.MAX)
    pms = float(pms.item())
    gqa_flops = 16 * 4.0 * HQ * HD * (T * (T + 1) / 2)
    err = stack.ctx.device_error()
    stack.close()
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "workload": "config 4: 64-layer stack (48 GDN + 16 GQA), head-sharded, NCCL all-gather "
                                          "of head outputs per layer",
            "n_gpus": world, "scaling": "strong",
            "decode": {"batch": B, "context": CTX, "ms_per_token_step": dms, "tok_s": B / (dms / 1000.0),
                       "hbm_gbs_per_gpu": rank_bytes / (dms / 1000.0) / 1e9,
                       "hbm_frac_per_gpu": rank_bytes / (dms / 1000.0) / 1e9 / hbm, "steps": steps, "warmup": warm,
                       "kv": "synthetic byte pattern (0x3C) for the cached rows"},
            "prefill": {"tokens": T, "ms": pms, "tok_s": T / (pms / 1000.0),
                        "gqa_tflops_whole_job": gqa_flops / (pms / 1000.0) / 1e12,
                        "note": "ms covers all 64 layers incl. per-layer all-gathers (GQA + GDN)"},
            "plan": {"kv_heads_per_rank": kvc, "v_heads_per_rank": vc, "pair_count": plan.pair_count},
            "kv_fill_s": fill_s, "device_error": err}))
    dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--cpu-steps", type=int, default=1)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--workload", default="decode", choices=["decode", "stack"],
                    help="decode = config 2 (the bench line); stack = config 4 (64 layers, head-sharded)")
    ap.add_argument("--stack-ctx", type=int, default=131072)
    ap.add_argument("--stack-prefill", type=int, default=32768)
    ap.add_argument("--stack-prefill-iters", type=int, default=2)
    ap.add_argument("--prefill-iters", type=int, default=5)
    ap.add_argument("--seqs", type=int, default=B_PER_RANK,
                    help="sequences per GPU (default 64 = config 2; smaller only for profiler captures)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "stack":
        return run_stack(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
