"""Benchmark: single-query GQA decode over fp16 / INT8 / INT4-KIVI KV on B200.

    python bench.py [--gpus N --steps K --warmup W] [--impl ours|reference]

Headline workload (one step = one decode-attention launch over one batch):
BASELINE config 1 per GPU - batch 8, 32 query / 8 KV heads, head_dim 128,
seqlen 4096, fp16 KV [B, Hkv, S, D] contiguous, seeded N(0,1) synthetic data.
With N GPUs each rank runs its own config-1 batch (global batch 8N; units are
(batch, kv-head) pairs, disjoint per rank, no collective on the hot path):
"scaling": "weak". value = HBM bytes the step must move on all ranks (K + V
codes + scales/zeros + q + out) / the max over ranks of the device time per
step, in TB/s.

Also reported on the same line: INT8 per-token (config 2), INT4 KIVI
asymmetric g128 (config 3) and the reference's symmetric INT4 format at g128;
config 4 (batch 64, seqlen 32768, fp16 and INT4 asym) sharded over the ranks
by (batch, kv-head) (strong scaling of a fixed job); an end-to-end number
through the public op with pinned host buffers; the roofline of the fp16
kernel against the measured HBM peak; the KV quantize/pack (append side) and
fp16 materialize kernels at the config-1 cache shape ("kv_kernels": us, GB/s
and fraction of the HBM peak); and the CPU oracle timed on this host.

Timing: K steps are captured in one CUDA graph (each step reads a different
copy of the inputs; the copies together exceed 3x the L2 size, so every step
streams from HBM) and replayed once between CUDA events after a barrier and a
synchronize; the max over ranks is reported.

--impl reference times the reference's CPU path (the numpy port of
reference/attention_ref.py in oracle/) on this host with all cores, one
(batch, kv-head) unit of config 1 per step; rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "llm-inference-kernels_b200"))
sys.path.insert(0, ROOT)

HQ, HKV, D = 32, 8, 128
C1 = dict(batch=8, seqlen=4096)
C4 = dict(batch=64, seqlen=32768)
GS = 128
SCALE = 1.0 / math.sqrt(D)
METRIC = "GQA decode achieved HBM TB/s (fp16 KV, config 1 per GPU)"


def algo_bytes(fmt: str, batch: int, seqlen: int, gs: int = GS) -> int:
    """Bytes one decode step must move: codes + scales/zeros + q + out."""
    units = batch * HKV
    qo = 2 * batch * HQ * D * 2
    if fmt == "f16":
        return units * seqlen * D * 2 * 2 + qo
    if fmt == "int8":
        return units * seqlen * (D + 2) * 2 + qo
    ng = -(-seqlen // gs)
    kv = units * seqlen * (D // 2) * 2
    if fmt == "int4":
        return kv + units * ng * D * 2 + units * seqlen * 2 + qo
    if fmt == "int4_asym":
        return kv + 2 * units * ng * D * 2 + 2 * units * seqlen * 2 + qo
    raise ValueError(fmt)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-c4", action="store_true", help="skip the config-4 lines")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--profile", action="store_true",
                    help="profiler-friendly run: one warm replay, short e2e legs (timings not for reporting)")
    ap.add_argument("--case", choices=["f16", "int8", "int4", "int4_asym"] + list(QUANT_CASES),
                    help="profiling case: only `--launches` decode launches of this KV format at the config-1 "
                         "shape (one copy of the inputs, larger than L2), no timing, no JSON line")
    ap.add_argument("--launches", type=int, default=3, help="launches of --case")
    ap.add_argument("--batch", type=int, default=C1["batch"], help="batch of --case")
    ap.add_argument("--seqlen", type=int, default=C1["seqlen"], help="seqlen of --case")
    return ap.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# --------------------------------------------------------------- CPU side

def cpu_info():
    model = ""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return model


def cpu_unit_sample(steps: int, warmup: int):
    """Time the CPU oracle on one (batch, kv-head) unit of config 1 per step.

    Returns (seconds per unit, threads). numpy's BLAS uses all host cores.
    """
    import numpy as np
    from oracle import kv_oracle as O

    rng = np.random.default_rng(0)
    g = HQ // HKV
    q = rng.standard_normal((1, g, D)).astype(np.float16)
    k = rng.standard_normal((1, 1, C1["seqlen"], D)).astype(np.float16)
    v = rng.standard_normal((1, 1, C1["seqlen"], D)).astype(np.float16)
    for _ in range(max(1, warmup)):
        O.decode_attention(q, k, v, SCALE)
    times = []
    for _ in range(steps):
        t = time.perf_counter()
        O.decode_attention(q, k, v, SCALE)
        times.append(time.perf_counter() - t)
    return statistics.median(times), sum(times), os.cpu_count() or 1


def unit_bytes_c1() -> float:
    return algo_bytes("f16", C1["batch"], C1["seqlen"]) / (C1["batch"] * HKV)


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    steps = args.steps
    med, total, cores = cpu_unit_sample(steps, args.warmup)
    tbs = unit_bytes_c1() / med / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": tbs, "unit": "TB/s",
        "n_gpus": args.gpus, "steps": steps, "warmup": args.warmup,
        "ms_per_step": med * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1), fp16)",
        "config": {"workload": "config1 fp16 KV decode, 1 of 64 (batch, kv-head) units per step",
                   "batch": C1["batch"], "n_heads": HQ, "n_kv_heads": HKV, "head_dim": D,
                   "seqlen": C1["seqlen"]},
        "cpu_baseline": {"value": tbs, "unit": "TB/s", "cores": cores, "kind": "port",
                         "sample": "one (batch, kv-head) unit of config 1 (4 query heads, 4096 positions) "
                                   "per step; numpy port of reference/attention_ref.py; " + cpu_info()},
        "e2e": {"value": tbs, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling while the GPU is loaded."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------- GPU side

def make_slabs(torch, dev, batch, seqlen, slab0, seed, outliers=False):
    """K, V [batch, Hkv, seqlen, D] fp16, each (batch, kv-head) slab drawn from
    its own generator seeded with seed + global slab index, so any rank can
    regenerate any slab independently of the GPU count."""
    k = torch.empty(batch, HKV, seqlen, D, dtype=torch.float16, device=dev)
    v = torch.empty_like(k)
    g = torch.Generator(device=dev)
    for b in range(batch):
        for h in range(HKV):
            g.manual_seed(seed + slab0 + b * HKV + h)
            kk = torch.randn(seqlen, D, generator=g, device=dev)
            if outliers:   # config 3: 4 of 128 K channels scaled x10
                kk[:, [0, 37, 74, 111]] *= 10.0
            k[b, h] = kk.half()
            v[b, h] = torch.randn(seqlen, D, generator=g, device=dev).half()
    return k, v


class Workload:
    """R copies of one decode step's inputs for one KV format, and the op call."""

    def __init__(self, torch, L, dev, fmt, batch, seqlen, slab0, copies, seed=1000):
        self.fmt, self.batch, self.seqlen = fmt, batch, seqlen
        self.sets = []
        gq = torch.Generator(device=dev)
        for r in range(copies):
            base = seed + r * 1_000_003
            gq.manual_seed(base + 7 * 10**6 + slab0)
            q = torch.randn(batch, HQ, D, generator=gq, device=dev).half()
            k, v = make_slabs(torch, dev, batch, seqlen, slab0, base, outliers=fmt.startswith("int4"))
            if fmt == "f16":
                args = (q, k, v)
            elif fmt == "int8":
                kq, ks = L.quantize_per_token(k)
                vq, vs = L.quantize_per_token(v)
                args = (q, kq, ks, vq, vs)
            elif fmt == "int4":
                kq, ks = L.quantize_k_per_channel_groupwise_int4(k, GS)
                vq, vs = L.quantize_v_per_token_int4(v)
                args = (q, kq, ks, vq, vs)
            else:
                kq, ks, kz = L.quantize_k_per_channel_groupwise_int4_asym(k, GS)
                vq, vs, vz = L.quantize_v_per_token_int4_asym(v)
                args = (q, kq, ks, kz, vq, vs, vz)
            del k, v
            self.sets.append(args)
        self.L = L

    def step(self, i):
        a = self.sets[i % len(self.sets)]
        L = self.L
        if self.fmt == "f16":
            return L.decode_attention(a[0], a[1], a[2], SCALE)
        if self.fmt == "int8":
            return L.decode_attention_int8(*a, SCALE)
        if self.fmt == "int4":
            return L.decode_attention_int4(*a, GS, SCALE)
        return L.decode_attention_int4_asym(*a, GS, SCALE)

    def bytes(self):
        return algo_bytes(self.fmt, self.batch, self.seqlen)


def copies_for(nbytes, l2):
    return max(1, math.ceil(3 * l2 / nbytes))


def time_graph(torch, wl, steps, warmup, barrier, min_warm_s=1.0, max_warm=10000):
    """Capture `steps` steps in one CUDA graph; warm up; replay once timed.
    Returns device ms per step on this rank."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for i in range(max(3, warmup)):
            wl.step(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(steps):
            wl.step(i)
    # untimed replays: settle clocks and caches (at least min_warm_s)
    t0 = time.perf_counter()
    n = 0
    while n < max(1, warmup) or time.perf_counter() - t0 < min_warm_s:
        g.replay()
        torch.cuda.synchronize()
        n += 1
        if n >= max_warm:
            break
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        e0.record(s)
        g.replay()
        e1.record(s)
    torch.cuda.synchronize()
    barrier()
    del g
    return e0.elapsed_time(e1) / steps


def max_over_ranks(torch, x, world):
    from llmik_cuda.shard import max_over_ranks as _max
    return _max(x, device="cuda") if world > 1 else x


def physical_index(local: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        parts = [x.strip() for x in vis.split(",") if x.strip()]
        if local < len(parts) and parts[local].isdigit():
            return int(parts[local])
    return local


def measured_hbm_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def ncu_traffic():
    """Per-launch DRAM bytes (read + write) of the fp16 config-1 kernel, from the
    committed ncu summary profiles/decode_f16_config1.md, if present."""
    try:
        with open(os.path.join(ROOT, "profiles", "decode_f16_config1.md")) as f:
            for line in f:
                if line.startswith("dram_bytes_per_launch:"):
                    return int(line.split(":", 1)[1].strip())
    except (OSError, ValueError):
        pass
    return None


def check_against_oracle(out, q, k, v, units, what):
    """Compare a few (batch) rows of a step's output with the CPU oracle."""
    import numpy as np
    from oracle import kv_oracle as O
    for b in units:
        ref = O.decode_attention(q[b:b + 1].cpu().numpy(), k[b:b + 1].cpu().numpy(),
                                 v[b:b + 1].cpu().numpy(), SCALE)
        got = out[b:b + 1].float().cpu().numpy()
        err = np.abs(got - ref)
        if not (err <= 2e-3 + 1e-2 * np.abs(ref)).all():
            raise SystemExit(f"bench: {what} output mismatch vs oracle (max err {err.max():.3e})")


def check_c4_rows(out, args, fmt, rows, what):
    """Config-4 rows of one rank's shard vs the CPU oracle."""
    import numpy as np
    from oracle import kv_oracle as O
    for b in rows:
        a = [x[b:b + 1].cpu().numpy() for x in args]
        if fmt == "f16":
            kk, vv = a[1], a[2]
        else:   # (q, kq, ks, kz, vq, vs, vz), group size GS
            kk, vv = O.dequant_kivi_asym_exact(a[1], a[2], a[3], a[4], a[5], a[6], GS)
        ref = O.decode_attention(a[0], kk, vv, SCALE)
        got = out[b:b + 1].float().cpu().numpy()
        err = np.abs(got - ref)
        if not (err <= 2e-3 + 1e-2 * np.abs(ref)).all():
            raise SystemExit(f"bench: {what} row {b} mismatch vs oracle (max err {err.max():.3e})")


def e2e_host_buffers(torch, L, dev, steps):
    """Config-1 fp16 step through the public op with pinned host inputs:
    H2D q, k, v + decode + D2H out inside the timed region."""
    b, s = C1["batch"], C1["seqlen"]
    g = torch.Generator().manual_seed(5)
    qh = torch.randn(b, HQ, D, generator=g).half().pin_memory()
    kh = torch.randn(b, HKV, s, D, generator=g).half().pin_memory()
    vh = torch.randn(b, HKV, s, D, generator=g).half().pin_memory()
    oh = torch.empty(b, HQ, D, dtype=torch.float16).pin_memory()
    qd, kd, vd = (torch.empty_like(x, device=dev) for x in (qh, kh, vh))

    def step():
        qd.copy_(qh, non_blocking=True)
        kd.copy_(kh, non_blocking=True)
        vd.copy_(vh, non_blocking=True)
        out = L.decode_attention(qd, kd, vd, SCALE)
        oh.copy_(out, non_blocking=True)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    h2d = (qh.numel() + kh.numel() + vh.numel()) * 2
    return ms, h2d, oh.numel() * 2


def e2e_decode_step(torch, L, dev, steps):
    """A serving-style decode step at config 1: the fp16 cache stays resident
    in a preallocated [B, Hkv, S_max, D] buffer. Each step makes ONE pinned
    H2D upload of a packed record (q, the new token's K and V, and its cache
    slots), appends the token in place with the library's append kernel
    (paged_append, the contiguous cache viewed as B blocks of S_max rows),
    attends over the live length straight from the uploaded q, and reads the
    output back. Returns (device ms per step, h2d bytes, d2h bytes)."""
    b, s = C1["batch"], C1["seqlen"]
    buf = s + steps + 8
    g = torch.Generator(device=dev).manual_seed(6)
    kc = torch.randn(b, HKV, buf, D, generator=g, device=dev).half()
    vc = torch.randn(b, HKV, buf, D, generator=g, device=dev).half()
    nq, nkv = b * HQ * D * 2, b * HKV * D * 2
    rec = nq + 2 * nkv + b * 8                       # q | k_new | v_new | slots (int64)
    host = [torch.empty(rec, dtype=torch.uint8).pin_memory() for _ in range(2)]
    for h in host:
        h[:nq + 2 * nkv].view(torch.float16).copy_(torch.randn((nq + 2 * nkv) // 2).half())
    dev_rec = torch.empty(rec, dtype=torch.uint8, device=dev)
    q = dev_rec[:nq].view(torch.float16).view(b, HQ, D)
    kn = dev_rec[nq:nq + nkv].view(torch.float16).view(b, HKV, D)
    vn = dev_rec[nq + nkv:nq + 2 * nkv].view(torch.float16).view(b, HKV, D)
    slots = dev_rec[nq + 2 * nkv:].view(torch.int64)
    oh = torch.empty(b, HQ, D, dtype=torch.float16).pin_memory()
    base = torch.arange(b, dtype=torch.int64) * buf

    sent = [torch.cuda.Event(), torch.cuda.Event()]

    def step(p, i):
        # double-buffered host records: the host waits only until the upload
        # that last used this buffer (two steps back) has been consumed
        h = host[i & 1]
        sent[i & 1].synchronize()
        h[nq + 2 * nkv:].view(torch.int64).copy_(base + p)
        dev_rec.copy_(h, non_blocking=True)
        sent[i & 1].record()
        L.paged_append(kn, slots, kc.view(b, HKV, buf, D))
        L.paged_append(vn, slots, vc.view(b, HKV, buf, D))
        out = L.decode_attention(q, kc, vc, SCALE, p + 1)
        oh.copy_(out, non_blocking=True)

    p = s - 1
    for i in range(3):
        step(p, i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        step(p + i, i)
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps, rec, oh.numel() * 2


def time_kv_kernels(torch, L, dev, l2, peak_gbs, launches=50):
    """The KV quantize / pack (append side) and fp16 materialize kernels at the
    config-1/2/3 cache shape [8, 8, 4096, 128], each over freshly rotated
    copies whose total exceeds 3x L2. Bytes are algorithmic (inputs read once,
    outputs written once). `launches` calls are captured in a CUDA graph and
    the replay is timed with CUDA events."""
    b, s = C1["batch"], C1["seqlen"]
    E = b * HKV * s * D            # elements of one K (or V) tensor
    T = b * HKV * s                # tokens
    G = b * HKV * (-(-s // GS)) * D  # K group-scale elements at g128
    x_bytes = 2 * E
    reps = copies_for(x_bytes, l2)
    g = torch.Generator(device=dev).manual_seed(11)
    xs = [torch.randn(b, HKV, s, D, generator=g, device=dev).half() for _ in range(reps)]
    i8 = [L.quantize_per_token(x) for x in xs]
    i4 = [L.quantize_k_per_channel_groupwise_int4_asym(x, GS) + L.quantize_v_per_token_int4_asym(x) for x in xs]
    ops = [
        ("quantize_per_token (INT8, one tensor)", lambda r: L.quantize_per_token(xs[r]),
         x_bytes + E + 2 * T),
        ("quantize_k_per_channel_groupwise_int4 (g128)", lambda r: L.quantize_k_per_channel_groupwise_int4(xs[r], GS),
         x_bytes + E // 2 + 2 * G),
        ("quantize_v_per_token_int4", lambda r: L.quantize_v_per_token_int4(xs[r]),
         x_bytes + E // 2 + 2 * T),
        ("quantize_k_per_channel_groupwise_int4_asym (g128)",
         lambda r: L.quantize_k_per_channel_groupwise_int4_asym(xs[r], GS), x_bytes + E // 2 + 4 * G),
        ("quantize_v_per_token_int4_asym", lambda r: L.quantize_v_per_token_int4_asym(xs[r]),
         x_bytes + E // 2 + 4 * T),
        ("dequantize_int8 (K and V to fp16)",
         lambda r: L.dequantize_int8(i8[r][0], i8[r][1], i8[r][0], i8[r][1]), 2 * (E + 2 * T) + 2 * x_bytes),
        ("dequantize_int4 asym (K and V to fp16)",
         lambda r: L.dequantize_int4(i4[r][0], i4[r][1], i4[r][3], i4[r][4], GS, -1, i4[r][2], i4[r][5]),
         2 * (E // 2) + 4 * G + 4 * T + 2 * x_bytes),
    ]
    res = {}
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    for name, fn, nbytes in ops:
        # the calls are captured in one CUDA graph (the ops' host-side checks
        # and output allocations are not part of the device time) and replayed
        with torch.cuda.stream(st):
            for r in range(3):
                fn(r % reps)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=st):
            for i in range(launches):
                fn(i % reps)
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(st):
            e0.record(st)
            graph.replay()
            e1.record(st)
        torch.cuda.synchronize()
        del graph
        us = e0.elapsed_time(e1) * 1e3 / launches
        gbs = nbytes / (us * 1e-6) / 1e9
        res[name] = {"us": us, "GB_s": gbs, "bytes": nbytes, "frac_of_hbm_peak": gbs / peak_gbs}
    del xs, i8, i4
    torch.cuda.empty_cache()
    return res


def run_ours(args):
    import torch
    world, rank, local = dist_env()
    dist = None
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)
    import llmik_cuda as L

    def barrier():
        if dist is not None:
            dist.barrier()

    steps, warmup = args.steps, max(3, args.warmup)
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    sampler = ClockSampler(physical_index(local))
    sampler.start()

    # ---- config 1 per rank: fp16 (headline), INT8 (config 2), INT4 (config 3) ----
    b, s = C1["batch"], C1["seqlen"]
    slab0 = rank * b * HKV
    formats = {}
    head_ms = None
    for fmt, name in (("f16", "fp16"), ("int8", "int8_per_token"), ("int4_asym", "int4_kivi_asym_g128"),
                      ("int4", "int4_kivi_sym_g128")):
        nb = algo_bytes(fmt, b, s)
        wl = Workload(torch, L, dev, fmt, b, s, slab0, copies_for(nb, l2))
        if fmt == "f16":
            q, k, v = wl.sets[0]
            check_against_oracle(wl.step(0), q, k, v, [0, b - 1], "config-1 fp16")
        ms = max_over_ranks(torch, time_graph(torch, wl, steps, warmup, barrier,
                                              min_warm_s=0.0 if args.profile else 1.0,
                                              max_warm=1 if args.profile else 10000), world)
        formats[name] = {"us_per_step": ms * 1e3, "TB_s": world * nb / (ms * 1e-3) / 1e12,
                         "bytes_per_step_per_gpu": nb, "copies_rotated": len(wl.sets)}
        if fmt == "f16":
            head_ms = ms
        del wl
        torch.cuda.empty_cache()
    fp16_us = formats["fp16"]["us_per_step"]
    for f in formats.values():
        f["speedup_vs_fp16"] = fp16_us / f["us_per_step"]

    # ---- config 4: batch 64, seqlen 32768 sharded by (batch, kv-head) ----
    c4 = {}
    if not args.no_c4 and C4["batch"] % world == 0:
        bl = C4["batch"] // world
        c4steps = max(1, min(steps, 100))
        for fmt, name in (("f16", "fp16"), ("int4_asym", "int4_kivi_asym_g128")):
            nb = algo_bytes(fmt, bl, C4["seqlen"])
            wl = Workload(torch, L, dev, fmt, bl, C4["seqlen"], rank * bl * HKV, copies_for(nb, l2), seed=2000)
            ms = max_over_ranks(torch, time_graph(torch, wl, c4steps, warmup, barrier, min_warm_s=0.5), world)
            c4[name] = {"us_per_step": ms * 1e3, "TB_s": world * nb / (ms * 1e-3) / 1e12,
                        "steps": c4steps, "batch_per_gpu": bl}
            # every rank checks the first, middle and last sequence of its own
            # shard against the CPU oracle (INT4: on the exactly dequantized KV
            # the tensor-pipe kernel attends over)
            out0 = wl.step(0)
            rows = sorted({0, bl // 2, bl - 1})
            check_c4_rows(out0, wl.sets[0], fmt, rows, f"config-4 {name} rank {rank}")
            c4[name]["verified"] = (f"sequences {rows} of every rank's shard vs CPU oracle "
                                    f"(global batch rows {[rank * bl + r for r in rows]} on this rank)")
            if fmt == "f16" and world > 1:
                # the assembled output (NCCL all-gather, off the timed path)
                # equals the shards
                from llmik_cuda.shard import gather_shards
                full = gather_shards(out0)
                if not torch.equal(full[rank * bl:(rank + 1) * bl], out0):
                    raise SystemExit("bench: gathered config-4 output differs from the local shard")
            del wl
            torch.cuda.empty_cache()
    peak, peak_kind = measured_hbm_peak()
    kv_kernels = time_kv_kernels(torch, L, dev, l2, peak, launches=5 if args.profile else 50)
    clocks = sampler.stop()

    # ---- end to end through the public op (host buffers) ----
    e2e_steps = 3 if args.profile else max(3, min(steps, 20))
    e2e_ms, h2d, d2h = e2e_host_buffers(torch, L, dev, e2e_steps)
    e2e_ms = max_over_ranks(torch, e2e_ms, world)
    dec_ms, dec_h2d, dec_d2h = e2e_decode_step(torch, L, dev, 3 if args.profile else max(10, min(steps, 200)))
    dec_ms = max_over_ranks(torch, dec_ms, world)

    nb1 = algo_bytes("f16", b, s)
    value = world * nb1 / (head_ms * 1e-3) / 1e12
    achieved = nb1 / (head_ms * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": head_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16",
        "data": "synthetic: seeded N(0,1) per (batch, kv-head) slab, cast to fp16",
        "config": {"workload": "config1: fp16 KV GQA decode, batch 8 per GPU, 32 q / 8 kv heads, "
                               "head_dim 128, seqlen 4096",
                   "global_batch": b * world, "seq_len": s, "n_heads": HQ, "n_kv_heads": HKV,
                   "head_dim": D, "parallelism": f"shard(batch, kv_head) x{world}",
                   "l2": "inputs rotated over copies totalling > 3x L2 (every step streams from HBM)"},
        "us_per_step": head_ms * 1e3,
        "tokens_per_s": world * b / (head_ms * 1e-3),
        "formats": formats,
        "config4_sharded": c4,
        # config 4 is the strong-scaling workload: global batch 64 is split
        # over the N GPUs, so its per-N device time is the scaling curve
        "strong_scaling": {
            "workload": "config4: batch 64 (global) x seqlen 32768, 32 q / 8 kv heads, sharded by "
                        "(batch, kv-head), no collective on the timed path",
            "n_gpus": world,
            **{f"{k}_us_per_step": v["us_per_step"] for k, v in c4.items()},
            **{f"{k}_TB_s": v["TB_s"] for k, v in c4.items()}},
        "kv_kernels": kv_kernels,
        "e2e": {"value": world * nb1 / (e2e_ms * 1e-3) / 1e12, "unit": "TB/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
                "what": "llmik_cuda.decode_attention with q, k, v copied from pinned host memory "
                        "and the output copied back, every step"},
        "e2e_decode_step": {"us_per_step": dec_ms * 1e3, "overhead_us_vs_kernel": (dec_ms - head_ms) * 1e3,
                            "h2d_bytes_per_step": dec_h2d, "d2h_bytes_per_step": dec_d2h,
                            "what": "resident fp16 cache; per step one packed pinned H2D record (q, new "
                                    "K/V token, slots), paged_append of K and V in place, decode over the "
                                    "live length, D2H output"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": ncu_traffic(), "peak_source": peak_kind,
                     "kernel": "decode_kernel<fp16, 4 heads/unit>"},
        "clocks": clocks,
        "gpu_launches": steps,
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        med, _, cores = cpu_unit_sample(5, 1)
        n = max(5, min(20000, int(15.0 / max(med, 1e-4))))
        med, total, cores = cpu_unit_sample(n, 1)
        line["cpu_baseline"] = {"value": unit_bytes_c1() / med / 1e12, "unit": "TB/s", "cores": cores,
                                "kind": "port", "seconds": total,
                                "sample": f"{n} steps x one (batch, kv-head) unit of config 1 on the CPU "
                                          f"oracle (numpy port of reference/attention_ref.py); {cpu_info()}"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# the KV quantize / pack and materialize ops, for ncu captures of one kernel
QUANT_CASES = {
    "q_int8": lambda L, x, i8, i4: L.quantize_per_token(x),
    "q_k4": lambda L, x, i8, i4: L.quantize_k_per_channel_groupwise_int4(x, GS),
    "q_v4": lambda L, x, i8, i4: L.quantize_v_per_token_int4(x),
    "q_k4a": lambda L, x, i8, i4: L.quantize_k_per_channel_groupwise_int4_asym(x, GS),
    "q_v4a": lambda L, x, i8, i4: L.quantize_v_per_token_int4_asym(x),
    "dq_int8": lambda L, x, i8, i4: L.dequantize_int8(i8[0], i8[1], i8[0], i8[1]),
    "dq_int4a": lambda L, x, i8, i4: L.dequantize_int4(i4[0], i4[1], i4[3], i4[4], GS, -1, i4[2], i4[5]),
}


def run_case(args):
    """A few launches of one decode format or one KV quantize / materialize
    op at [batch, 8, seqlen, 128], for ncu captures (small, bounded)."""
    import torch
    import llmik_cuda as L
    dev = torch.device("cuda", 0)
    if args.case in QUANT_CASES:
        g = torch.Generator(device=dev).manual_seed(11)
        x = torch.randn(args.batch, HKV, args.seqlen, D, generator=g, device=dev).half()
        i8 = L.quantize_per_token(x)
        i4 = L.quantize_k_per_channel_groupwise_int4_asym(x, GS) + L.quantize_v_per_token_int4_asym(x)
        for i in range(args.launches):
            QUANT_CASES[args.case](L, x, i8, i4)
    else:
        wl = Workload(torch, L, dev, args.case, args.batch, args.seqlen, 0, 1)
        for i in range(args.launches):
            wl.step(i)
    torch.cuda.synchronize()
    print(f"case {args.case}: {args.launches} launches ok", flush=True)
    return 0


def main():
    args = parse()
    if args.case:
        return run_case(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
