"""Benchmark of the hybrid-attention hot path.

Headline ("step", the JSON line's value): BASELINE config 2, batched hybrid
decode -- 64 sequences in total with ragged KV caches of L_i ~ U{512..32768}
cached positions (seeded), each advancing one token through one gated GQA layer
(dz_gqa_decode) and one Gated DeltaNet layer (dz_gdn_decode).  Sequence-sharded
across the GPUs with no collective: the 64 sequences are split by LPT on
L_i + 1 (strong scaling).  Inputs are synthetic N(0,1) activations (projections
are out of scope), KV contents N(0,1), DeltaNet state N(0, 0.02).  Per-step
KV + state traffic (~9 GB in total) is far above the 126 MB L2, so no flush is
needed between steps.

Extra keys on the same line:
  config0 / config1  single-layer decode (config 0: one GQA layer at position
                     2048; config 1: one Gated DeltaNet layer), many back-to-back
                     layer instances over buffers larger than L2, replayed from a
                     CUDA graph; N = 1 only
  prefill            config 3 (T = 8192): GQA prefill TFLOP/s against the bf16
                     peak, Gated DeltaNet prefill time, CPU baselines; N = 1 only
  stack              config 4: the 64-layer stack head-sharded over the ranks
                     with an NCCL all-gather per layer (decode B = 8 at context
                     131072, prefill T = 32768); every N
  q1_gemv            the Q1_0 input-projection GEMV that feeds the cores (hidden
                     5120, 1 and 4 tokens) and the block tail after them
                     (post-norm + SwiGLU MLP, d_ff 17408); N = 1 only
  block              whole decoder blocks for one sequence and one token (norm,
                     projections, core, output projection, MLP) and their
                     64-layer sum beside the reference's published per-token
                     decode times; N = 1 only

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
N_SEQ = 64
LEN_LO, LEN_HI = 512, 32768
SEED0 = 0xDA12A000 + 2      # config 2

HQ, HKV, GRP, HD = 24, 4, 6, 256
SSM_HV, SSM_D, QKV_LEN, INNER = 48, 128, 10240, 6144

# DRAM bytes (read + write) that one ncu capture counted for the split-K
# attention kernel, divided by the algorithmic bytes of that launch: the first
# 16 config-2 sequences (205,050 KV positions, 1.681 GB algorithmic, 1.692 GB
# counted).  Traffic grows with the KV positions read, so the roofline's
# `traffic` is this ratio times the algorithmic bytes of the timed launch.
GQA_SPLIT_TRAFFIC_RATIO = 1.0066


def seq_lengths():
    """The 64 config-2 cache lengths (seeded, identical on every rank)."""
    rng = np.random.default_rng(SEED0)
    return rng.integers(LEN_LO, LEN_HI + 1, size=N_SEQ).astype(np.int64)


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


# algorithmic bytes per step (K/V rows read once, inputs read once, outputs written once)
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


def gqa_prefill_flops(T, base=0):
    """QK^T and PV over the causal range: 4 * 24 * 256 * sum_t (base + t + 1)."""
    return 4.0 * HQ * HD * (T * base + T * (T + 1) / 2)


def gdn_prefill_flops(T, heads=SSM_HV, C=64):
    """Chunked form per (chunk, head): 10 C^2 d + 6 C d^2 + (2/3) C^3."""
    return (T // C) * heads * (10 * C * C * SSM_D + 6 * C * SSM_D * SSM_D + (2 / 3) * C ** 3)


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
# reference arm / CPU baselines: the oracle (C++ restatement of the AVX2 path)
# ---------------------------------------------------------------------------
class CpuWorkload:
    """Config 2 for the oracle: the sequences `pick` (indices into the 64), their
    real lengths, built once; step() advances every one of them by one token
    through both layers.  KV rows are tiled from one seeded random block of 4096
    positions (the attention's cost does not depend on the values)."""

    def __init__(self, pick, max_steps):
        import oracle as O
        self.O = O
        lens = seq_lengths()
        self.pick = np.asarray(pick)
        self.lens = lens[self.pick]
        (self.qn, self.kn), self.p = layer_params(SEED0)
        blk_k = O.normal(SEED0 + 500, (HKV, 4096, HD))
        blk_v = O.normal(SEED0 + 600, (HKV, 4096, HD))
        st0 = O.normal(SEED0 + 700, (SSM_HV, SSM_D, SSM_D), 0.0, 0.02)
        h0 = O.normal(SEED0 + 800, (4, QKV_LEN))
        self.kvs, self.sts = [], []
        for n in self.lens:
            n = int(n)
            kv = O.OracleKv(n + max_steps)
            reps = -(-n // 4096)
            kv.k[:, :n] = np.tile(blk_k, (1, reps, 1))[:, :n]
            kv.v[:, :n] = np.tile(blk_v, (1, reps, 1))[:, :n]
            kv.len = n
            self.kvs.append(kv)
            self.sts.append(O.OracleSsm(st0, h0, 0))
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


def cpu_baseline_decode(steps=1):
    """Config 2, 8 of the 64 sequences, one thread (the reference decodes one
    sequence at a time, attention and scan single-threaded)."""
    pick = np.arange(0, N_SEQ, N_SEQ // 8)
    w = CpuWorkload(pick, steps)
    dt = sum(w.step(1) for _ in range(steps))
    return {"value": len(pick) * steps / dt, "unit": "tok/s", "cores": 1, "kind": "port",
            "sample": f"8 of the 64 sequences (lengths {list(map(int, w.lens))}), {steps} decode step(s) of both "
                      f"layers, single thread like the reference's decode attention/scan; {dt:.2f} s"}


def cpu_baseline_prefill(T=1024):
    """Config 3 on the host cores: the oracle's parallel prefills (GQA over
    (token, kv head) units, Gated DeltaNet over v heads, as the reference's
    forward.rs:643,920,1025) at T tokens, all cores."""
    import oracle as O
    cores = os.cpu_count() or 1
    (qn, kn), p = layer_params(SEED0 + 3)
    qg, k, v = O.normal(SEED0 + 31, (T, HQ * 2 * HD)), O.normal(SEED0 + 32, (T, HKV * HD)), \
        O.normal(SEED0 + 33, (T, HKV * HD))
    t0 = time.perf_counter()
    O.gqa_prefill(qg, k, v, qn, kn, O.OracleKv(T), n_threads=cores)
    tg = time.perf_counter() - t0
    qkv, a, b, z = O.normal(SEED0 + 34, (T, QKV_LEN)), O.normal(SEED0 + 35, (T, SSM_HV)), \
        O.normal(SEED0 + 36, (T, SSM_HV)), O.normal(SEED0 + 37, (T, INNER))
    t0 = time.perf_counter()
    O.gdn_prefill(qkv, a, b, z, p, O.OracleSsm(), n_threads=cores)
    td = time.perf_counter() - t0
    return {"gqa": {"value": gqa_prefill_flops(T) / tg / 1e12, "unit": "TFLOP/s", "ms": tg * 1e3, "cores": cores,
                    "kind": "port", "sample": f"T={T} tokens (config 3 has 8192; work grows as T^2)"},
            "gdn": {"value": T / td, "unit": "tok/s", "ms": td * 1e3, "cores": cores, "kind": "port",
                    "sample": f"T={T} tokens, token-recurrent per v head like the reference"}}


def run_reference(args):
    """The reference's CPU path (the oracle port of its AVX2 code) on config 2:
    all 64 sequences, one decode step of both layers per timed step, one
    sequence per host thread."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cores = os.cpu_count() or 1
    w = CpuWorkload(np.arange(N_SEQ), args.warmup + args.steps)
    for _ in range(args.warmup):
        w.step(cores)
    dts = [w.step(cores) for _ in range(args.steps)]
    wall = sum(dts)
    value = N_SEQ * args.steps / wall
    sample = (f"all {N_SEQ} config-2 sequences ({int(np.sum(w.lens))} cached tokens), one decode step of both layers "
              f"per timed step; {cores} host threads, one sequence per thread (harness parallelisation: the reference "
              "decodes one sequence at a time)")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * wall / max(1, args.steps),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": "config 2: batched hybrid decode, 64 sequences, "
                                                        "KV U{512..32768}, 1 GQA + 1 GDN layer"},
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def _max_over_ranks(dist, dev, x):
    if dist is None:
        return x
    import torch
    t = torch.tensor([x], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def bench_config2(dz, torch, dist, dev, local, rank, world, args):
    """This rank's LPT share of the 64 sequences, timed with CUDA events; the
    headline value uses the max over ranks."""
    from daiza_b200 import parallel as P
    all_lens = seq_lengths()[:args.sample_seqs] if args.sample_seqs else seq_lengths()
    n_total = len(all_lens)
    mine = P.lpt_shard(all_lens, world)[rank]
    lens = all_lens[mine]
    B = len(lens)
    total_steps = args.warmup + args.steps + args.e2e_steps + 4
    cfg = dz.default_config(n_layers=2, full_attention_interval=2)   # layer 0 GDN, layer 1 GQA
    ctx = dz.Context(local, cfg)
    (qn, kn), sp = layer_params(SEED0)
    ctx.set_attn_params(1, qn, kn)
    ctx.set_ssm_params(0, *sp)
    ctx.cache_create(lens + total_steps)
    g = torch.Generator(device=dev)
    g.manual_seed(SEED0 + 1000 + rank)
    for s, n in enumerate(lens):
        kf = torch.randn(int(n), HKV, HD, device=dev, generator=g)
        vf = torch.randn(int(n), HKV, HD, device=dev, generator=g)
        ctx.kv_import(1, s, kf, vf)
        del kf, vf
        st = torch.randn(SSM_HV, SSM_D, SSM_D, device=dev, generator=g) * 0.02
        hist = torch.randn(4, QKV_LEN, device=dev, generator=g)
        ctx.ssm_import(0, s, st, hist, 0)
    torch.cuda.synchronize()
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

    for _ in range(args.warmup):
        ctx.gqa_decode(1, ids, qg, kk, vv, out)
        ctx.gdn_decode(0, ids, qkv, al, be, z, y)
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
    ms_rank = t_start.elapsed_time(t_end)
    ms = _max_over_ranks(dist, dev, ms_rank)
    gqa_ms = [ev[i][0].elapsed_time(ev[i][1]) for i in range(args.steps)]
    gdn_ms = [ev[i][1].elapsed_time(ev[i][2]) for i in range(args.steps)]

    gqa_b = np.mean([gqa_bytes(lens_at + i) for i in range(args.steps)])
    gdn_b = gdn_bytes(B)
    hbm, _, peak_kind = peaks()
    gqa_gbs = gqa_b / (np.mean(gqa_ms) / 1000.0) / 1e9
    gdn_gbs = gdn_b / (np.mean(gdn_ms) / 1000.0) / 1e9

    # end to end through the public C ABI host entry points (pinned host buffers)
    e2e = None
    if args.e2e_steps > 0:
        host = [t.cpu().pin_memory() for t in (qg, kk, vv, qkv, al, be, z)]
        ho = torch.empty(B, HQ * HD, pin_memory=True)
        hy = torch.empty(B, INNER, pin_memory=True)
        nv = [t.numpy() for t in host] + [ho.numpy(), hy.numpy()]
        for _ in range(2):                       # untimed: staging buffers, copy stream, events
            ctx.gqa_decode_host(1, ids, nv[0], nv[1], nv[2], nv[7], sync=False)
            ctx.gdn_decode_host(0, ids, nv[3], nv[4], nv[5], nv[6], nv[8], sync=False)
            stream.synchronize()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.e2e_steps):
            # the DeltaNet inputs go up while the GQA layer runs; one wait per step
            # for both results to be in host memory
            ctx.gqa_decode_host(1, ids, nv[0], nv[1], nv[2], nv[7], sync=False)
            ctx.gdn_decode_host(0, ids, nv[3], nv[4], nv[5], nv[6], nv[8], sync=False)
            stream.synchronize()
        e1.record(stream)
        torch.cuda.synchronize()
        ems = _max_over_ranks(dist, dev, e0.elapsed_time(e1))
        h2d = B * (HQ * 2 * HD + 2 * HKV * HD + QKV_LEN + 2 * SSM_HV + INNER) * 4
        d2h = B * (HQ * HD + INNER) * 4
        e2e = {"value": n_total * args.e2e_steps / (ems / 1000.0), "unit": "tok/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "path": "dz_gqa_decode_host_async + dz_gdn_decode_host_async (pinned host buffers, uploads on a copy "
                       "stream, copies inside the timed region, one stream synchronisation per step), max over ranks",
               "steps": args.e2e_steps}
    err = ctx.device_error()
    ctx.close()
    traffic = None if GQA_SPLIT_TRAFFIC_RATIO is None else GQA_SPLIT_TRAFFIC_RATIO * gqa_b
    return {"ms": ms, "ms_rank": ms_rank, "B": B, "n_total": n_total, "kv_tokens": int(lens_at.sum()), "clk": clk, "clocks": clocks,
            "launches": launches, "e2e": e2e, "device_error": err,
            "roofline": {"bound": "hbm", "kernel": "dz_gqa_decode (prep + split-K + combine)", "achieved": gqa_gbs,
                         "peak": hbm, "unit": "GB/s", "frac": gqa_gbs / hbm, "traffic": traffic,
                         "peak_kind": f"{peak_kind} hbm_gbs", "bytes_per_launch": gqa_b,
                         "traffic_source": "ncu dram bytes of gqa_split_kernel on the first 16 config-2 sequences, "
                                           "scaled by KV positions (ratio %.4f)" % GQA_SPLIT_TRAFFIC_RATIO,
                         "ms_per_launch": float(np.mean(gqa_ms)), "rank": rank},
            "gdn": {"achieved_gbs": gdn_gbs, "frac": gdn_gbs / hbm, "bytes": gdn_b, "ms": float(np.mean(gdn_ms))},
            "step_gbs": (gqa_b + gdn_b) / (ms_rank / args.steps / 1000.0) / 1e9}


def bench_single_layer(dz, torch, dev, local, kind, reps=20):
    """Configs 0 and 1: one decode step of one layer, measured over many
    back-to-back layer instances (16 GQA layers x 16.8 MB of KV, or 96 Gated
    DeltaNet layers x 3.1 MB of state: 269 MB and 302 MB, both above the 126 MB
    L2, so every instance reads its bytes from HBM), captured once into a CUDA graph and
    replayed (every replay rewrites the same cache slot / conv slot, which is
    the same work as a fresh step)."""
    g = torch.Generator(device=dev)
    g.manual_seed(SEED0 + 7 + (kind == "gdn"))
    if kind == "gqa":
        M, n_prior = 16, 2048
        cfg = dz.default_config(n_layers=4 * M, full_attention_interval=4)
        layers = [4 * i + 3 for i in range(M)]
    else:
        M = 96
        cfg = dz.default_config(n_layers=M, full_attention_interval=M + 1)
        layers = list(range(M))
    ctx = dz.Context(local, cfg)
    for layer in range(cfg.n_layers):
        a, s_ = layer_params(SEED0 + 100 + layer)
        if ctx.is_attention(layer):
            ctx.set_attn_params(layer, *a)
        else:
            ctx.set_ssm_params(layer, *s_)
    if kind == "gqa":
        ctx.cache_create([n_prior + 2])
        for layer in layers:
            kf = torch.randn(n_prior, HKV, HD, device=dev, generator=g)
            vf = torch.randn(n_prior, HKV, HD, device=dev, generator=g)
            ctx.kv_import(layer, 0, kf, vf)
        qg = torch.randn(1, HQ * 2 * HD, device=dev, generator=g)
        kk = torch.randn(1, HKV * HD, device=dev, generator=g)
        vv = torch.randn(1, HKV * HD, device=dev, generator=g)
        out = torch.empty(1, HQ * HD, device=dev)

        def one_round():
            for layer in layers:
                ctx.gqa_decode(layer, [0], qg, kk, vv, out)

        def rewind():
            for layer in layers:
                ctx.kv_truncate(layer, 0, n_prior)
        bytes_per = gqa_bytes([n_prior])
    else:
        ctx.cache_create([4])
        for layer in layers:
            st = torch.randn(SSM_HV, SSM_D, SSM_D, device=dev, generator=g) * 0.02
            hist = torch.randn(4, QKV_LEN, device=dev, generator=g)
            ctx.ssm_import(layer, 0, st, hist, 0)
        qkv = torch.randn(1, QKV_LEN, device=dev, generator=g)
        al = torch.randn(1, SSM_HV, device=dev, generator=g)
        be = torch.randn(1, SSM_HV, device=dev, generator=g)
        z = torch.randn(1, INNER, device=dev, generator=g)
        y = torch.empty(1, INNER, device=dev)

        def one_round():
            for layer in layers:
                ctx.gdn_decode(layer, [0], qkv, al, be, z, y)

        def rewind():
            pass
        bytes_per = gdn_bytes(1)
    for _ in range(2):
        one_round()
        rewind()
    torch.cuda.synchronize()
    graph = None
    try:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            one_round()
        rewind()
    except Exception as e:  # noqa: BLE001 -- fall back to eager issue and say so
        graph = None
        note = f"eager (graph capture failed: {type(e).__name__})"
        torch.cuda.synchronize()
        rewind()
    else:
        note = "CUDA graph of one round, replayed"
    stream = torch.cuda.current_stream()
    for _ in range(3):
        graph.replay() if graph is not None else one_round()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        if graph is not None:
            graph.replay()
        else:
            one_round()
            rewind()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    err = ctx.device_error()
    del graph
    ctx.close()
    us = ms * 1000.0 / (reps * len(layers))
    hbm, _, kind_p = peaks()
    gbs = bytes_per / (us * 1e-6) / 1e9
    return {"workload": ("config 0: one gated GQA decode step at position 2048 (2048 cached positions), 24/4 heads, "
                         "D=256" if kind == "gqa" else
                         "config 1: one Gated DeltaNet decode step, 16/48 heads, d=128, state N(0,0.02)"),
            "us_per_layer_step": us, "tok_s": 1e6 / us, "bytes": bytes_per, "achieved_gbs": gbs, "peak_gbs": hbm,
            "frac": gbs / hbm, "peak_kind": f"{kind_p} hbm_gbs", "instances": len(layers), "replays": reps,
            "issue": note, "device_error": err}


Q1_SETS = (("attention input projections attn_q/attn_k/attn_v (model/attention.rs:80-87)", (12288, 1024, 1024)),
           ("Gated DeltaNet input projections attn_qkv/ssm_alpha/ssm_beta/attn_gate (model/ssm.rs:451-463)",
            (10240, 48, 48, 6144)))
Q1_HIDDEN = 5120
Q1_FF = 17408


def bench_q1(dz, torch, local, tokens=(1, 4)):
    """Q1_0 projection GEMV (dz_q1_gemv) on the model's two input-projection
    sets from hidden 5120, for a few tokens: 24 calls over 24 distinct copies of
    the weights (10-12 MB each, ~250 MB in all > L2) captured in one CUDA graph
    and replayed.  Then the block tail (dz_block_mlp: RMSNorm, gate/up GEMV,
    SwiGLU, down GEMV added into h) over 12 copies of one block's MLP weights
    (d_ff 17408, 37.6 MB each); its roofline bytes are the Q1_0 bytes.  Synthetic Q1_0 weights (random signs, |N(0,0.02)| binary16
    scales); roofline bytes = the Q1_0 bytes + x + y."""
    import oracle as O
    dev = torch.device("cuda", local)
    ctx = dz.Context(local, dz.default_config(n_layers=2, full_attention_interval=2))
    hbm, _, kind = peaks()
    out = []
    for name, rows in Q1_SETS:
        base = [O.q1_random(SEED0 + 900 + i, r, Q1_HIDDEN) for i, r in enumerate(rows)]
        copies = [[torch.from_numpy(w).to(dev) for w in base] for _ in range(24)]
        wbytes = sum(w.nbytes for w in base)
        for T in tokens:
            x = torch.randn(T, Q1_HIDDEN, device=dev)
            ys = [torch.empty(T, r, device=dev) for r in rows]
            for _ in range(3):
                ctx.q1_gemv(copies[0], x, ys)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for i in range(24):
                    ctx.q1_gemv(copies[i], x, ys)
            for _ in range(2):
                graph.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(10):
                graph.replay()
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1000.0 / 240
            nbytes = wbytes + T * Q1_HIDDEN * 4 + T * sum(rows) * 4
            out.append({"set": name, "rows": sum(rows), "cols": Q1_HIDDEN, "tokens": T, "us": us,
                        "weight_mb": wbytes / 1e6, "gbs": nbytes / us / 1e3, "frac": nbytes / us / 1e3 / hbm,
                        "peak_kind": f"{kind} hbm_gbs"})
            del graph
        del copies
    # block tail (dz_block_mlp): post-norm + SwiGLU MLP of one block, 12 distinct weight copies (~450 MB)
    mlp_w = [O.q1_random(SEED0 + 960, Q1_FF, Q1_HIDDEN), O.q1_random(SEED0 + 961, Q1_FF, Q1_HIDDEN),
             O.q1_random(SEED0 + 962, Q1_HIDDEN, Q1_FF, 0.01)]
    mcopies = [[torch.from_numpy(w).to(dev) for w in mlp_w] for _ in range(12)]
    post = torch.ones(Q1_HIDDEN, device=dev)
    mbytes = sum(w.nbytes for w in mlp_w)
    for T in tokens:
        h = torch.randn(T, Q1_HIDDEN, device=dev)
        for _ in range(3):
            ctx.block_mlp(h, post, *mcopies[0])
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(12):
                ctx.block_mlp(h, post, *mcopies[i])
        for _ in range(2):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(10):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1000.0 / 120
        out.append({"set": "block_mlp", "rows": 2 * Q1_FF + Q1_HIDDEN, "cols": f"{Q1_HIDDEN}/{Q1_FF}", "tokens": T,
                    "us": us, "weight_mb": mbytes / 1e6, "gbs": mbytes / us / 1e3, "frac": mbytes / us / 1e3 / hbm,
                    "peak_kind": f"{kind} hbm_gbs"})
        del graph
    del mcopies
    # CPU baseline: the oracle's restatement of the reference matvec, all host cores, first set, 1 token
    cores = os.cpu_count() or 1
    base = [O.q1_random(SEED0 + 900 + i, r, Q1_HIDDEN) for i, r in enumerate(Q1_SETS[0][1])]
    xh = O.normal(SEED0 + 950, (1, Q1_HIDDEN))
    O.q1_gemv(base, xh, n_threads=cores)
    t0 = time.perf_counter()
    reps = 5
    for _ in range(reps):
        O.q1_gemv(base, xh, n_threads=cores)
    cpu_us = (time.perf_counter() - t0) / reps * 1e6
    err = ctx.device_error()
    ctx.close()
    return {"workload": "Q1_0 projection GEMV (dz_q1_gemv), hidden 5120, synthetic weights",
            "runs": out, "device_error": err,
            "cpu_baseline": {"us": cpu_us, "cores": cores, "kind": "port",
                             "sample": "attention input projection set, 1 token, dot_q1_0_row over all rows"}}


BLOCK_LAYERS = 16            # 8 gated GQA + 8 Gated DeltaNet layers, each with its own weights
BLOCK_POS = 2048             # KV positions cached in front of the timed tokens (config 0)
PUBLISHED_MS = {"attn16": 11.5, "gdn48": 38.5, "model": 143.0}   # reference README.md:431-439, per token


def bench_block(dz, torch, local):
    """Whole decoder blocks, one sequence, one token (the reference's decode
    step): rmsnorm -> Q1_0 input projections -> core -> Q1_0 output projection
    added into h -> post-norm SwiGLU MLP added into h, all through the public
    entry points.  8 layers of each kind with distinct synthetic weights (~52 MB
    per block, ~850 MB in all > L2), captured per kind in one CUDA graph and
    replayed; the GQA layers hold 2048 cached positions.  The 64-layer figure is
    16 x GQA block + 48 x DeltaNet block (embedding, final norm and LM head
    excluded), beside the reference's published per-token times on its CPU."""
    import oracle as O
    dev = torch.device("cuda", local)
    ctx = dz.Context(local, dz.default_config(n_layers=BLOCK_LAYERS, full_attention_interval=2))
    (qn, kn), sp = layer_params(SEED0 + 7)
    ctx.cache_create([BLOCK_POS + 64])
    hbm, _, kind = peaks()
    base = {
        "attn_norm": torch.ones(Q1_HIDDEN, device=dev), "post_norm": torch.ones(Q1_HIDDEN, device=dev),
        "gate": O.q1_random(SEED0 + 970, Q1_FF, Q1_HIDDEN), "up": O.q1_random(SEED0 + 971, Q1_FF, Q1_HIDDEN),
        "down": O.q1_random(SEED0 + 972, Q1_HIDDEN, Q1_FF, 0.01),
        "out": O.q1_random(SEED0 + 973, Q1_HIDDEN, HQ * HD, 0.01),
        "attn_proj": [O.q1_random(SEED0 + 974 + i, r, Q1_HIDDEN) for i, r in enumerate(Q1_SETS[0][1])],
        "gdn_proj": [O.q1_random(SEED0 + 978 + i, r, Q1_HIDDEN) for i, r in enumerate(Q1_SETS[1][1])],
    }
    layers = []
    for layer in range(BLOCK_LAYERS):
        attn = ctx.is_attention(layer)
        if attn:
            ctx.set_attn_params(layer, qn, kn)
            ctx.kv_fill_pattern(layer, 0, BLOCK_POS)
        else:
            ctx.set_ssm_params(layer, *sp)
        proj = base["attn_proj"] if attn else base["gdn_proj"]
        layers.append({"attn": attn,
                       "proj": [torch.from_numpy(x).to(dev) for x in proj],
                       "out": torch.from_numpy(base["out"]).to(dev),
                       "gate": torch.from_numpy(base["gate"]).to(dev), "up": torch.from_numpy(base["up"]).to(dev),
                       "down": torch.from_numpy(base["down"]).to(dev)})
    wbytes = {a: sum(x.nbytes for x in (base["attn_proj"] if a else base["gdn_proj"])) + base["out"].nbytes
              + base["gate"].nbytes + base["up"].nbytes + base["down"].nbytes for a in (True, False)}
    h = torch.randn(1, Q1_HIDDEN, device=dev)
    normed = torch.empty_like(h)
    core = torch.empty(1, HQ * HD, device=dev)
    bufs = {a: [torch.empty(1, r, device=dev) for r in (Q1_SETS[0][1] if a else Q1_SETS[1][1])] for a in (True, False)}

    def block(L, li):
        ctx.rmsnorm_rows(h, base["attn_norm"], normed)
        p = bufs[L["attn"]]
        ctx.q1_gemv(L["proj"], normed, p)
        if L["attn"]:
            ctx.gqa_decode(li, [0], p[0], p[1], p[2], core)
        else:
            ctx.gdn_decode(li, [0], p[0], p[1], p[2], p[3], core)
        ctx.q1_gemv_add([L["out"]], core, [h])
        ctx.block_mlp(h, base["post_norm"], L["gate"], L["up"], L["down"])

    out = {}
    for attn in (True, False):
        idx = [i for i in range(BLOCK_LAYERS) if layers[i]["attn"] == attn]
        block(layers[idx[0]], idx[0])            # warm-up outside the graph (scratch allocation)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in idx:
                block(layers[i], i)
        for _ in range(2):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 10
        e0.record()
        for _ in range(reps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1000.0 / (reps * len(idx))
        core_bytes = (gqa_bytes([BLOCK_POS + 8]) if attn else gdn_bytes(1))
        nbytes = wbytes[attn] + core_bytes
        out["gqa_block" if attn else "gdn_block"] = {
            "us": us, "weight_mb": wbytes[attn] / 1e6, "core_mb": core_bytes / 1e6, "gbs": nbytes / us / 1e3,
            "frac": nbytes / us / 1e3 / hbm, "peak_kind": f"{kind} hbm_gbs", "layers_timed": len(idx)}
        del graph
    a_us, g_us = out["gqa_block"]["us"], out["gdn_block"]["us"]
    out["per_token_ms"] = {"attn16": 16 * a_us / 1e3, "gdn48": 48 * g_us / 1e3, "blocks64": (16 * a_us + 48 * g_us) / 1e3}
    out["reference_published_ms"] = dict(PUBLISHED_MS,
                                         note="README.md:431-439, Core Ultra 5 225H CPU, whole model incl. LM head")
    out["device_error"] = ctx.device_error()
    ctx.close()
    return out


PF_T = 8192


def bench_prefill(dz, torch, local, args):
    """Config 3: one sequence, T=8192 tokens, positions 0..8191.  GQA prefill with
    bf16 q/k/v (prep + tcgen05 attention); Gated DeltaNet prefill with f32
    qkv/alpha/beta/z from a zero state (prep + ring + intra + chain)."""
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
    err = ctx.device_error()
    ctx.close()
    gms = float(np.median(gtimes))
    g_flops = gdn_prefill_flops(PF_T)
    g_bytes = PF_T * (QKV_LEN + 2 * SSM_HV + 2 * INNER) * 4 + SSM_HV * SSM_D * SSM_D * 4 * 2
    hbm, bf16, kind = peaks()
    gdn = {"workload": "config 3 Gated DeltaNet prefill, T=8192, f32 in/out, chunk 64, zero state",
           "ms": gms, "tok_s": PF_T / (gms / 1000.0), "algorithmic_gflop": g_flops / 1e9,
           "tflops": g_flops / (gms / 1000.0) / 1e12, "bytes": g_bytes, "gbs": g_bytes / (gms / 1000.0) / 1e9,
           "hbm_frac": g_bytes / (gms / 1000.0) / 1e9 / hbm, "launches_per_call": glaunches,
           "note": "tcgen05 bf16 hi/lo split products (3 per product, f32 accumulate in TMEM): persistent intra-chunk "
                   "WY kernel + one persistent chain CTA per v head with the state in TMEM"}
    flops = gqa_prefill_flops(PF_T)
    ms = float(np.median(times))
    tf = flops / (ms / 1000.0) / 1e12
    return {"workload": "config 3 GQA prefill, T=8192, bf16 q/k/v, 24/4 heads, D=256, causal",
            "ms": ms, "tok_s": PF_T / (ms / 1000.0), "tflops": tf, "peak_tflops": bf16, "frac": tf / bf16,
            "peak_kind": f"{kind} bf16_tflops (burst)", "flops": flops, "iters": iters,
            "launches_per_call": launches,
            "timed": "dz_gqa_prefill_bf16 = prep (norm/rope/cache append) + tcgen05 attention, median of iters",
            "gdn": gdn, "device_error": err}


def bench_stack(dz, torch, dist, dev, local, rank, world, args):
    """Config 4: the 64-layer attention stack (48 Gated DeltaNet + 16 GQA layers),
    head-sharded over the ranks with an NCCL all-gather of head outputs after
    every layer.  Decode: batch 8 at context 131072 (KV rows are a synthetic byte
    pattern).  Prefill: one sequence of 32768 tokens.  Times are the max over
    ranks; strong scaling (the whole problem is split over the ranks)."""
    from daiza_b200 import parallel as P
    B, CTX, T = 8, args.stack_ctx, args.stack_prefill
    steps, warm = args.stack_steps, 2
    plan = P.head_plan(world, rank)
    rows = plan.decode_rows(B)
    caps = [(CTX + steps + warm + 2) if b in rows else 1 for b in range(B)] + [T]

    def params(layer, kind):
        a, s_ = layer_params(SEED0 + 4 * 1000 + layer)
        return a if kind == "attn" else s_

    stack = P.ShardedStack(local, B, caps, params)
    t0 = time.time()
    for layer in range(64):
        if stack.attn[layer]:
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
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        stack.decode_step(gqa_in, gdn)
    e1.record(stream)
    torch.cuda.synchronize()
    dms = _max_over_ranks(dist, dev, e0.elapsed_time(e1) / steps)
    ctx_now = CTX + warm + steps // 2
    kvc = plan.kv_heads[1] - plan.kv_heads[0]
    vc = plan.v_heads[1] - plan.v_heads[0]
    rank_bytes = 16 * len(rows) * (ctx_now + 1) * kvc * HD * 4 * 2 + 48 * B * vc * SSM_D * SSM_D * 4 * 2
    hbm, bf16, kind = peaks()
    pg = torch.randn(T, HQ * 2 * HD, device=dev, generator=g).to(torch.bfloat16)
    pk = torch.randn(T, HKV * HD, device=dev, generator=g).to(torch.bfloat16)
    pv = torch.randn(T, HKV * HD, device=dev, generator=g).to(torch.bfloat16)
    pgdn = tuple(torch.randn(T, n, device=dev, generator=g) for n in (QKV_LEN, SSM_HV, SSM_HV, INNER))
    pin = stack.slice_inputs(pg, pk, pv)
    ptimes = []
    for it in range(1 + args.stack_prefill_iters):
        stack.ctx.cache_reset(B)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        stack.prefill(B, pin, pgdn)
        a1.record(stream)
        torch.cuda.synchronize()
        if it > 0:
            ptimes.append(a0.elapsed_time(a1))
    pms = _max_over_ranks(dist, dev, float(np.median(ptimes)))
    gqa_flops = 16 * gqa_prefill_flops(T)
    err = stack.ctx.device_error()
    stack.close()
    return {"workload": "config 4: 64-layer stack (48 Gated DeltaNet + 16 gated GQA), head-sharded, NCCL all-gather "
                        "of head outputs after every layer",
            "scaling": "strong",
            "decode": {"batch": B, "context": CTX, "ms_per_token_step": dms, "tok_s": B / (dms / 1000.0),
                       "hbm_gbs_per_gpu": rank_bytes / (dms / 1000.0) / 1e9,
                       "hbm_frac_per_gpu": rank_bytes / (dms / 1000.0) / 1e9 / hbm, "steps": steps, "warmup": warm,
                       "kv": "synthetic byte pattern (0x3C) for the cached rows"},
            "prefill": {"tokens": T, "ms": pms, "tok_s": T / (pms / 1000.0),
                        "gqa_tflops_whole_job": gqa_flops / (pms / 1000.0) / 1e12,
                        "note": "ms covers all 64 layers incl. per-layer all-gathers (GQA + GDN)"},
            "plan": {"kv_heads_per_rank": kvc, "v_heads_per_rank": vc, "pair_count": plan.pair_count},
            "kv_fill_s": fill_s, "device_error": err}


def run_ours(args):
    import torch
    import daiza_b200 as dz
    from daiza_b200 import parallel as P

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        P.init_process_group("nccl", device=dev)

    c2 = bench_config2(dz, torch, dist, dev, local, rank, world, args)
    extra = {}
    if world == 1 and not args.no_single:
        extra["config0"] = bench_single_layer(dz, torch, dev, local, "gqa")
        extra["config1"] = bench_single_layer(dz, torch, dev, local, "gdn")
    if world == 1 and not args.no_prefill:
        extra["prefill"] = bench_prefill(dz, torch, local, args)
    if world == 1 and not args.no_q1:
        extra["q1_gemv"] = bench_q1(dz, torch, local)
        torch.cuda.empty_cache()
        extra["block"] = bench_block(dz, torch, local)
    if not args.no_stack:
        torch.cuda.empty_cache()
        extra["stack"] = bench_stack(dz, torch, dist, dev, local, rank, world, args)
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline_decode(steps=args.cpu_steps)
        if "prefill" in extra:
            extra["prefill"]["cpu_baseline"] = cpu_baseline_prefill()
    else:
        cpu = None

    if rank == 0:
        ms = c2["ms"]
        line = {"metric": METRIC, "value": c2["n_total"] * args.steps / (ms / 1000.0), "unit": "tok/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic",
                "config": {"workload": "config 2: batched hybrid decode, 64 sequences in total, KV lengths "
                                       "U{512..32768} (seeded), 1 gated GQA + 1 Gated DeltaNet layer, f32 caches",
                           "sequences": c2["n_total"], "seqs_on_rank0": c2["B"], "kv_tokens_on_rank0": c2["kv_tokens"],
                           "parallelism": f"sequence-sharded x{world} (LPT on cached length), no collective",
                           "l2": "no flush: per-step KV+state traffic ~9 GB >> 126 MB L2"},
                "hbm_gbs_step_rank0": c2["step_gbs"], "roofline": c2["roofline"], "gdn": c2["gdn"],
                "gpu_launches": c2["launches"], "clocks": c2["clk"], "e2e": c2["e2e"], "cpu_baseline": cpu,
                "device_error": c2["device_error"]}
        if args.sample_seqs:
            line["config"]["workload"] = (f"PROFILING SAMPLE, not the benchmark: the first {c2['n_total']} of the 64 "
                                          "config-2 sequences")
        line.update(extra)
        if c2["clk"] is None and c2["clocks"].raw:
            line["clocks_raw_head"] = c2["clocks"].raw[:300]
        print(json.dumps(line))
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--cpu-steps", type=int, default=1)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-single", action="store_true", help="skip the config 0 / config 1 single-layer keys")
    ap.add_argument("--no-stack", action="store_true", help="skip the config 4 stack key")
    ap.add_argument("--no-q1", action="store_true", help="skip the Q1_0 projection GEMV key")
    ap.add_argument("--stack-ctx", type=int, default=131072)
    ap.add_argument("--stack-prefill", type=int, default=32768)
    ap.add_argument("--stack-steps", type=int, default=10)
    ap.add_argument("--stack-prefill-iters", type=int, default=2)
    ap.add_argument("--prefill-iters", type=int, default=5)
    ap.add_argument("--sample-seqs", type=int, default=0,
                    help="profiling only: run config 2 on the first N of its 64 sequences (a few GB instead of ~9)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
