"""Attention-forward benchmark (driver contract: one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config c5] [--dtype f16|bf16] [--scaling strong|weak]
                    [--no-extras] [--kvcache-only NAME|all] [--varlen-only NAME|all]
                    [--backward-only NAME|all]

Metric: attention-forward TFLOPS, FLOPs = 4*B*H*N^2*d (halved
for causal, the reference's convention).  `value` is the whole-job aggregate
over the N GPUs; `tflops_per_gpu` = value / N.
Default workload: configuration C5 full — B=4, H=32, N=8192, d=128, fp16,
1 % of K rows scaled x8 — the shape the north-star target is quoted on; it
fits one GPU.

Multi-GPU (torchrun, one rank per GPU), default `--scaling strong`: the global
C5 problem stays B=4 H=32 at every N and its independent (batch, KV-head
group) units are split into contiguous ranges (`sharding.shard_units`), so at
N=8 each rank owns 16 of the 128 (batch, head) units.  Every rank builds the
same seeded global inputs and runs its range as one launch; no collective
touches the timed data path.  After timing, an NCCL all-gather brings every
rank's O and LSE to rank 0, which checks sampled rows of the first and the
last (batch, head) unit against the CPU oracle.  `--scaling weak` gives each
rank its own B=4 batch instead.

A step is one attention forward over the rank's units, inputs resident in
HBM (1.07 GB per step read+written at N=1, larger than the 126 MB L2, so no
L2 flush is needed between steps).  `e2e` times the same forward through the
public Python API for host buffers (`flash_attention_forward_host`) on every
rank's units: the step's Q/K/V are copied from pinned host memory and O back
inside the timed region, with the copies of each (batch, KV-head group) chunk
overlapping the other chunks' computation.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(REPO, "flash-attention-sm75-register-fused_b200")
for _p in (REPO, PKG_DIR):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = ("attn fwd TFLOPS (causal-halved), whole-job aggregate over 1/2/4/8 B200 "
          "(per GPU: tflops_per_gpu); % of tensor peak")
FALLBACK_PEAK_TFLOPS = 1590.0
FALLBACK_HBM_GBS = 6650.0

CONFIG_TEXT = {
    "c1": "C1 full attention B=1 H=1 N=512 d=64",
    "c2": "C2 full attention B=4 H=12 N=1024 d=64",
    "c3": "C3 causal attention B=4 H=8 N=2048 d=64 (inputs x0.5)",
    "c4": "C4 GQA causal B=2 Hq=32 Hkv=8 N=4096 d=128",
    "c5": "C5 full attention B=4 H=32 N=8192 d=128 (1% K rows x8)",
    "c5c": "C5 causal attention B=4 H=32 N=8192 d=128 (1% K rows x8)",
}

# rows sampled per checked (batch, head) slice, besides the tile edges
PARITY_ROWS = 96


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="c5", choices=sorted(CONFIG_TEXT))
    ap.add_argument("--dtype", choices=["f16", "bf16"], default="f16")
    ap.add_argument("--scaling", choices=["strong", "weak"], default="strong",
                    help="strong: the global problem is fixed and split over the ranks "
                         "(default); weak: every rank runs its own full batch")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip e2e, cpu_baseline and the per-config tables (profiling runs)")
    ap.add_argument("--kvcache-only", default=None, metavar="NAME|all",
                    help="time only fa_fwd_kvcache workloads (decode / chunked prefill) and print "
                         "their table as one JSON line (profiling runs)")
    ap.add_argument("--varlen-only", default=None, metavar="NAME|all",
                    help="time only fa_fwd_varlen / fa_fwd_padded workloads and print their table "
                         "as one JSON line (profiling runs)")
    ap.add_argument("--backward-only", default=None, metavar="NAME|all",
                    help="time only fa_bwd workloads (attention backward) and print their table "
                         "as one JSON line (profiling runs)")
    ap.add_argument("--configs-only", default=None, metavar="NAME|all",
                    help="time only the forward of the BASELINE configurations (kernel time, "
                         "parity of sampled rows, SDPA beside it) as one JSON line")
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_PEAK_TFLOPS, FALLBACK_HBM_GBS, "fallback"


def load_traffic(config):
    """DRAM bytes per launch of the kernel for `config`, from the committed ncu
    summary (profiles/fa_fwd_traffic.txt, lines `config: bytes`), or None."""
    path = os.path.join(REPO, "profiles", "fa_fwd_traffic.txt")
    try:
        for line in open(path):
            line = line.strip()
            if line.startswith(config + ":"):
                return float(line.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return None


def config_dict(cfg, world, scaling):
    """The `config` object of both arms' JSON lines (same keys, same values)."""
    strong = scaling == "strong"
    return {
        "workload": CONFIG_TEXT[cfg.name], "B": cfg.B, "Hq": cfg.Hq, "Hkv": cfg.Hkv,
        "N": cfg.N, "d": cfg.d, "causal": cfg.causal,
        "global_batch": cfg.B if strong else cfg.B * world,
        "parallelism": (f"{world} rank(s), contiguous ranges of the B*Hkv (batch, KV-head "
                        f"group) units" if strong else f"{world} rank(s), one B={cfg.B} batch each"),
        "l2": ("inputs+outputs > 126 MB L2 per step; no flush needed" if cfg.min_bytes > 126e6
               else "L2 not flushed (inputs smaller than L2)"),
    }


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and throttle reasons of one GPU during the timed region
    (NVML; `nvidia-smi` as fallback)."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, index, period=0.02):
        self.index, self.period = index, period
        self.samples, self.reasons = [], 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            self._nvml = (pynvml, h)
        except Exception:
            self._nvml = None
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()

    def _sample(self):
        if self._nvml:
            pynvml, h = self._nvml
            mhz = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
            try:
                rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
            except Exception:
                rs = pynvml.nvmlDeviceGetCurrentClocksThrottleReasons(h)
            return mhz, rs
        out = subprocess.run(
            ["nvidia-smi", f"--id={self.index}", "--query-gpu=clocks.sm,clocks.max.sm,"
             "clocks_event_reasons.active", "--format=csv,noheader,nounits"],
            capture_output=True, text=True, timeout=5).stdout.strip().split(",")
        self.max_mhz = float(out[1])
        return float(out[0]), int(out[2].strip(), 16)

    def _run(self):
        while not self._stop.is_set():
            try:
                mhz, rs = self._sample()
                self.samples.append(mhz)
                self.reasons |= int(rs)
            except Exception:
                pass
            self._stop.wait(self.period)

    def stop(self):
        self._stop.set()
        if self._thread:
            self._thread.join(timeout=5)
        reasons = [n for bit, n in self.REASONS.items() if self.reasons & bit and bit != 0x1]
        return {
            "sm_mhz": statistics.median(self.samples) if self.samples else None,
            "sm_max_mhz": self.max_mhz,
            "samples": len(self.samples),
            "reasons": reasons,
        }


# ----------------------------------------------------------------- inputs
def make_device_inputs(cfg, b0, b1, dtype, device, seed=42):
    """Seeded synthetic inputs for global batch entries [b0, b1): per entry a
    CUDA generator seeded from (seed, b) draws Q, K, V ~ N(0,1) (times the
    config's input scale), then K rows ``randperm(N)[:frac*N]`` per head x8.
    Entry b's data do not depend on b0 / b1, so every rank that builds the
    global batch holds the same bits."""
    import torch
    qs, ks, vs = [], [], []
    for b in range(b0, b1):
        g = torch.Generator(device=device).manual_seed(seed * 1_000_003 + b)
        q = torch.randn(1, cfg.Hq, cfg.N, cfg.d, generator=g, device=device)
        k = torch.randn(1, cfg.Hkv, cfg.N, cfg.d, generator=g, device=device)
        v = torch.randn(1, cfg.Hkv, cfg.N, cfg.d, generator=g, device=device)
        if cfg.input_scale != 1.0:
            q *= cfg.input_scale
            k *= cfg.input_scale
            v *= cfg.input_scale
        n_out = int(cfg.N * cfg.k_outlier_frac)
        for h in range(cfg.Hkv if n_out else 0):
            idx = torch.randperm(cfg.N, generator=g, device=device)[:n_out]
            k[0, h, idx] *= cfg.k_outlier_scale
        qs.append(q.to(dtype))
        ks.append(k.to(dtype))
        vs.append(v.to(dtype))
    return torch.cat(qs).contiguous(), torch.cat(ks).contiguous(), torch.cat(vs).contiguous()


class RankShard:
    """The contiguous range of (batch, KV-head group) units rank r runs: views
    of the global [B, H, N, d] tensors flattened to [B*H, N, d] (one launch
    with batch 1 and the range's heads)."""

    def __init__(self, cfg, world, rank, scaling):
        from flash_attention_sm75.sharding import shard_units
        self.G = cfg.Hq // cfg.Hkv
        if scaling == "strong":
            s = shard_units(cfg.B, cfg.Hq, cfg.Hkv, world, rank)
            self.u0 = s.groups[0][0] * cfg.Hkv + s.groups[0][1] if s.groups else 0
            self.units = len(s.groups)
        else:  # weak: the rank's own batch is the whole problem
            self.u0, self.units = 0, cfg.B * cfg.Hkv
        self.q_heads = self.units * self.G

    def views(self, cfg, q, k, v, o, lse):
        G, u0, n = self.G, self.u0, self.units
        fl = lambda t: t.view(-1, cfg.N, cfg.d)
        return (fl(q)[u0 * G:(u0 + n) * G], fl(k)[u0:u0 + n], fl(v)[u0:u0 + n],
                fl(o)[u0 * G:(u0 + n) * G], lse.view(-1, cfg.N)[u0 * G:(u0 + n) * G])


# ----------------------------------------------------------------- parity
def parity_check(cfg, q, k, v, o, lse, units=None, n_rows=PARITY_ROWS):
    """Sampled-row parity of a computed O / LSE against the CPU oracle (the
    reference's fp32 attention restated): rows 0, N-1, every 128-row tile's
    edges and ``n_rows`` seeded random rows of the (batch, query head) units in
    ``units`` (default: the first and the last), each against all N keys.
    Tolerance: |err| <= 2e-3 + 1e-2*|ref| (bf16: 1.6e-2 + 2e-2*|ref|) on O,
    1e-4 on LSE."""
    from oracle import attention_oracle as orc
    import torch
    G = cfg.Hq // cfg.Hkv
    if units is None:
        units = [(0, 0), (cfg.B - 1, cfg.Hq - 1)]
    bf16 = q.dtype == torch.bfloat16
    atol, rtol = (1.6e-2, 2e-2) if bf16 else (orc.ATOL, orc.RTOL)
    rows = orc.sample_rows(cfg.N, n_rows, seed=0)
    res = {"max_abs_err": 0.0, "max_rel_err": 0.0, "max_err_over_bound": 0.0, "lse_err": 0.0}
    ok = True
    for b, h in units:
        qs = q[b:b + 1, h:h + 1].cpu()
        ks = k[b:b + 1, h // G:h // G + 1].cpu()
        vs = v[b:b + 1, h // G:h // G + 1].cpu()
        ref_o, ref_l = orc.attention_fp32(qs, ks, vs, causal=cfg.causal, rows=rows)
        got = o[b:b + 1, h:h + 1].cpu()[:, :, rows].float()
        err = (got - ref_o).abs()
        bound = atol + rtol * ref_o.abs()
        r = orc.check(got, ref_o, atol=atol, rtol=rtol)
        rl = orc.check_lse(lse[b:b + 1, h:h + 1].cpu()[:, :, rows], ref_l)
        res["max_abs_err"] = max(res["max_abs_err"], r["max_abs_err"])
        res["max_rel_err"] = max(res["max_rel_err"], r["max_rel_err"])
        res["max_err_over_bound"] = max(res["max_err_over_bound"], (err / bound).max().item())
        res["lse_err"] = max(res["lse_err"], rl["max_abs_err"])
        ok = ok and r["ok"] and rl["ok"]
    res["ok"] = ok
    res["checked"] = f"{len(rows)} rows x {len(units)} (b,h) units {units}"
    return res


# ----------------------------------------------------------------- CPU legs
def cpu_slice(cfg, g):
    """One (batch, head) slice of the workload's inputs on the CPU, drawn like
    oracle.make_inputs (N(0,1) x input scale, the K outlier rows) from the
    generator ``g``: Q, K, V [1, 1, N, d] fp16."""
    import torch
    q = torch.randn(1, 1, cfg.N, cfg.d, generator=g) * cfg.input_scale
    k = torch.randn(1, 1, cfg.N, cfg.d, generator=g) * cfg.input_scale
    v = torch.randn(1, 1, cfg.N, cfg.d, generator=g) * cfg.input_scale
    n_out = int(cfg.N * cfg.k_outlier_frac)
    if n_out:
        k[0, 0, torch.randperm(cfg.N, generator=g)[:n_out]] *= cfg.k_outlier_scale
    return q.half(), k.half(), v.half()


def cpu_time_slices(cfg, g, n_slices=None, budget_s=None, rows_n=512):
    """Times the CPU oracle (the reference's fp32 attention restated,
    oracle/attention_oracle.py) with all host threads on fresh (b, h) slices of
    the workload, each ``rows_n`` seeded query rows against all N keys, for
    ``n_slices`` slices or until ``budget_s`` seconds of oracle time.  Input
    generation is not timed.  Returns (flops, seconds, slices)."""
    import torch
    from oracle import attention_oracle as orc
    rows_n = min(rows_n, cfg.N)
    flops, secs, slices = 0.0, 0.0, 0
    while (n_slices is not None and slices < n_slices) or (budget_s is not None and secs < budget_s):
        q, k, v = cpu_slice(cfg, g)
        rows = torch.randperm(cfg.N, generator=g)[:rows_n].sort().values
        t1 = time.perf_counter()
        orc.attention_fp32(q, k, v, causal=cfg.causal, rows=rows)
        secs += time.perf_counter() - t1
        flops += (float(4.0 * cfg.d * (rows + 1).sum().item()) if cfg.causal
                  else 4.0 * rows_n * cfg.N * cfg.d)
        slices += 1
    return flops, secs, slices


def cpu_threads():
    import torch
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    return cores


def run_reference(args, cfg):
    """--impl reference: the reference's CPU path (the oracle port) on the host
    cores, on this arm's metric and config.  Each step is a bounded sample of
    the workload: enough fresh 512-row (b, h) slices (with the K outlier rows)
    for about 0.3 s of oracle time, the slice count fixed during warm-up — the
    same sampling as the GPU arm's `cpu_baseline` leg."""
    import torch
    cores = cpu_threads()
    g = torch.Generator().manual_seed(42)
    t_slice = min(cpu_time_slices(cfg, g, n_slices=1)[1] for _ in range(3))
    per_step = max(1, int(round(0.3 / max(t_slice, 1e-6))))
    for _ in range(args.warmup):
        cpu_time_slices(cfg, g, n_slices=per_step)
    flops, secs = 0.0, 0.0
    for _ in range(args.steps):
        f, s, n = cpu_time_slices(cfg, g, n_slices=per_step)
        flops += f
        secs += s
    tflops = flops / secs / 1e12
    sample = (f"per step: {per_step} fresh (b,h) slices of {cfg.name}, 512 query rows x "
              f"{cfg.N} keys each, d={cfg.d}, K outlier rows as the workload, fp32 torch CPU "
              f"oracle, {secs:.1f} s in total")
    line = {
        "metric": METRIC, "value": tflops, "unit": "TFLOPS", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": secs / args.steps * 1e3,
        "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "impl": "reference",
        "config": config_dict(cfg, args.gpus, args.scaling),
        "cpu_baseline": {"value": tflops, "unit": "TFLOPS", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": tflops, "unit": "TFLOPS", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- GPU arm
def time_steps(fn, steps, stream):
    import torch
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1)


def units_per_rank(cfg, world, scaling):
    """(batch, KV-head group) units each rank runs."""
    from flash_attention_sm75.sharding import shard_units
    if scaling != "strong":
        return [cfg.B * cfg.Hkv] * world
    return [len(shard_units(cfg.B, cfg.Hq, cfg.Hkv, world, r).groups) for r in range(world)]


def gather_to_rank0(dist, t, count, max_count, world, dev):
    """All-gather of each rank's first-dimension range (``count`` rows of
    ``t``, padded to ``max_count``) over NCCL; returns the [world, max_count,
    ...] result (used on rank 0)."""
    import torch
    pad = torch.zeros((max_count,) + tuple(t.shape[1:]), dtype=t.dtype, device=dev)
    if count:
        pad[:count].copy_(t[:count])
    out = torch.empty((world * max_count,) + tuple(t.shape[1:]), dtype=t.dtype, device=dev)
    dist.all_gather_into_tensor(out, pad)
    return out.view((world, max_count) + tuple(t.shape[1:]))


def main():
    args = parse_args()
    rank, world, local_rank = dist_env()
    from oracle import attention_oracle as orc  # config table, CPU legs and parity checks only
    cfg = orc.CONFIGS[args.config]

    if args.impl == "reference":
        if rank == 0:
            run_reference(args, cfg)
        return

    import torch
    import torch.distributed as dist
    import flash_attn_sm75_cuda as _C  # noqa: F401  (the pybind module must load)
    from flash_attention_sm75 import flash_attention_forward_host
    from flash_attention_sm75 import capi as abi

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dtype = torch.bfloat16 if args.dtype == "bf16" else torch.float16
    only = [("kvcache", args.kvcache_only, kvcache_configs),
            ("varlen", args.varlen_only, varlen_configs),
            ("backward", args.backward_only, backward_configs),
            ("configs", args.configs_only, other_configs)]
    for key, sel, fn in only:
        if sel:
            if rank == 0:
                names = None if sel == "all" else [sel]
                print(json.dumps({key: fn(abi.load(), abi, dtype, dev, names)}), flush=True)
            return
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    strong = args.scaling == "strong"
    shard = RankShard(cfg, world, rank, args.scaling)
    # every rank builds the same global inputs (strong) or its own batch (weak)
    b0 = 0 if strong else rank * cfg.B
    q, k, v = make_device_inputs(cfg, b0, b0 + cfg.B, dtype, dev)
    o = torch.zeros_like(q)
    lse = torch.zeros(q.shape[:3], dtype=torch.float32, device=dev)
    qs, ks, vs, os_, ls = shard.views(cfg, q, k, v, o, lse)
    stream = torch.cuda.current_stream(dev)
    scale = 1.0 / math.sqrt(cfg.d)
    dt_code = 1 if dtype == torch.bfloat16 else 0
    lib = abi.load()
    qp, kp, vp, op, lp, sp = (abi.ptr(qs), abi.ptr(ks), abi.ptr(vs), abi.ptr(os_), abi.ptr(ls),
                              abi.stream_ptr(stream))
    n_heads, n_kv = shard.q_heads, shard.units

    def step():
        if n_heads == 0:
            return
        rc = lib.fa_fwd(qp, kp, vp, op, lp, 1, n_heads, n_kv, cfg.N, cfg.d, scale,
                        int(cfg.causal), dt_code, sp)
        if rc != 0:
            raise RuntimeError(lib.fa_error_string(rc).decode())

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(local_rank)
    sampler.start()
    ms = time_steps(step, args.steps, stream)
    clocks = sampler.stop()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    status = lib.fa_device_status(0)
    if status != 0:
        raise RuntimeError(f"device watchdog fired: {lib.fa_error_string(status).decode()}")

    # ---- parity of this run's output (outside the timed region)
    if world > 1 and strong:
        max_heads = -(-cfg.B * cfg.Hkv // world) * shard.G
        go = gather_to_rank0(dist, os_, n_heads, max_heads, world, dev)
        gl = gather_to_rank0(dist, ls, n_heads, max_heads, world, dev)
        counts = torch.tensor([n_heads], device=dev, dtype=torch.int64)
        all_counts = torch.empty(world, device=dev, dtype=torch.int64)
        dist.all_gather_into_tensor(all_counts, counts)
        if rank == 0:
            o_full = torch.cat([go[r, :int(c)] for r, c in enumerate(all_counts.tolist())])
            l_full = torch.cat([gl[r, :int(c)] for r, c in enumerate(all_counts.tolist())])
            o_chk = o_full.view_as(o)
            l_chk = l_full.view_as(lse)
        del go, gl
    else:
        o_chk, l_chk = o, lse
    parity = parity_check(cfg, q, k, v, o_chk, l_chk) if rank == 0 else None

    ms_step = ms / args.steps
    total_flops = cfg.flops * (1 if strong else world)
    value = total_flops / (ms_step * 1e-3) / 1e12
    peak, hbm, peak_kind = load_peaks()
    per_gpu = value / world
    traffic = load_traffic(cfg.name)
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": world,
        "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
        "dtype": args.dtype, "data": "synthetic (seeded N(0,1), 1% K rows x8 for C5)",
        "config": config_dict(cfg, world, args.scaling),
        "tflops_per_gpu": per_gpu,
        "units_per_rank": units_per_rank(cfg, world, args.scaling),
        "gpu_launches": args.steps * world,
        "gpu_launches_per_rank": args.steps,
        "roofline": {"bound": "tensor", "achieved": per_gpu, "peak": peak, "unit": "TFLOP/s",
                     "frac": per_gpu / peak, "peak_kind": f"{peak_kind} bf16 dense (burst)",
                     "frac_of_spec_2250": per_gpu / 2250.0,
                     "traffic": traffic if world == 1 else None,
                     "algorithmic_bytes": cfg.min_bytes / (world if strong else 1)},
        "clocks": clocks,
        "parity": parity,
    }
    if not args.no_extras:
        line["e2e"] = e2e_leg(cfg, shard, qs, ks, vs, dev, flash_attention_forward_host,
                              dist if world > 1 else None, strong, world)
    if not args.no_extras and rank == 0 and world == 1:
        # the CPU baseline is taken at N = 1 only: with more ranks the other
        # processes share the host cores and the figure means nothing
        cores = cpu_threads()
        flops, cpu_s, slices = cpu_time_slices(cfg, torch.Generator().manual_seed(42),
                                               budget_s=8.0)
        line["cpu_baseline"] = {
            "value": flops / cpu_s / 1e12, "unit": "TFLOPS", "cores": cores, "kind": "port",
            "sample": f"{slices} fresh (b,h) slices of {cfg.name}, 512 query rows x {cfg.N} keys "
                      f"each, K outlier rows as the workload, fp32 torch CPU oracle, "
                      f"{cpu_s:.1f} s"}
        del q, k, v, o, lse, qs, ks, vs, os_, ls
        torch.cuda.empty_cache()
        line["configs"] = other_configs(lib, abi, dtype, dev)
        line["kvcache"] = kvcache_configs(lib, abi, dtype, dev)
        line["backward"] = backward_configs(lib, abi, dtype, dev)
        line["varlen"] = varlen_configs(lib, abi, dtype, dev)
    elif rank == 0:
        line["cpu_baseline"] = None
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
        if parity is not None and not parity["ok"]:
            sys.exit(f"parity check of the timed output failed: {parity}")


def e2e_leg(cfg, shard, qs, ks, vs, dev, fwd_host, dist, strong, world, steps=5):
    """Public API end to end: ``flash_attention_forward_host`` on pinned host
    copies of this rank's units (Q [1, heads, N, d], K/V [1, units, N, d]), O
    returned in pinned host memory (H2D, forward and D2H of each (batch,
    KV-head group) chunk overlap inside the call).  Multi-GPU: every rank runs
    its units; the step time is the max over ranks."""
    import torch
    hq = qs.unsqueeze(0).cpu().pin_memory()
    hk = ks.unsqueeze(0).cpu().pin_memory()
    hv = vs.unsqueeze(0).cpu().pin_memory()
    ho = torch.empty_like(hq).pin_memory()
    stream = torch.cuda.current_stream(dev)
    n = shard.q_heads

    def step():
        if n:
            fwd_host(hq, hk, hv, causal=cfg.causal, out=ho)

    step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    ms = time_steps(step, steps, stream) / steps
    h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv))
    d2h = ho.numel() * ho.element_size()
    if dist is not None:
        t = torch.tensor([ms, h2d, d2h], device=dev, dtype=torch.float64)
        tmax = t.clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        ms, h2d, d2h = float(tmax[0].item()), int(t[1].item()), int(t[2].item())
    flops = cfg.flops * (1 if strong else world)
    return {"value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOPS", "ms_per_step": ms,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}


def sdpa_time(q, k, v, causal, n):
    """PyTorch's scaled_dot_product_attention on the same inputs (its default
    backend choice), ms per call; a same-box comparison column only."""
    import torch
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel
    gqa = q.size(1) != k.size(1)
    # fused backends only: the math backend would materialise the N x N scores
    with sdpa_kernel([SDPBackend.CUDNN_ATTENTION, SDPBackend.FLASH_ATTENTION,
                      SDPBackend.EFFICIENT_ATTENTION]):
        fn = lambda: F.scaled_dot_product_attention(q, k, v, is_causal=causal, enable_gqa=gqa)
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        return time_steps(fn, n, torch.cuda.current_stream()) / n


def other_configs(lib, abi, dtype, dev, names=None):
    """Kernel-only TFLOPS of the BASELINE configurations (reported, not the
    headline), with the sampled-row parity of each timed output and PyTorch
    SDPA's time on the same inputs as a same-box comparison column."""
    import torch
    from oracle import attention_oracle as orc
    out = {}
    for name in ("c1", "c2", "c3", "c4", "c5", "c5c"):
        if names is not None and name not in names:
            continue
        c = orc.CONFIGS[name]
        q, k, v = make_device_inputs(c, 0, c.B, dtype, dev)
        o = torch.empty_like(q)
        lse = torch.empty(q.shape[:3], dtype=torch.float32, device=dev)
        s = torch.cuda.current_stream(dev)
        args = (abi.ptr(q), abi.ptr(k), abi.ptr(v), abi.ptr(o), abi.ptr(lse), c.B, c.Hq, c.Hkv,
                c.N, c.d, 1.0 / math.sqrt(c.d), int(c.causal), 1 if dtype == torch.bfloat16 else 0,
                abi.stream_ptr(s))
        fn = lambda: lib.fa_fwd(*args)
        for _ in range(10):
            fn()
        torch.cuda.synchronize()
        n = max(20, min(2000, int(2e12 / c.flops)))
        ms = time_steps(fn, n, s) / n
        par = parity_check(c, q, k, v, o, lse)
        try:
            ms_sdpa = sdpa_time(q, k, v, c.causal, n)
        except RuntimeError:  # no fused SDPA backend takes this shape
            ms_sdpa = float("nan")
        out[name] = {"tflops": round(c.flops / ms / 1e9, 1), "us": round(ms * 1e3, 2),
                     "gbs": round(c.min_bytes / (ms * 1e-3) / 1e9, 1),
                     "max_abs_err": par["max_abs_err"], "max_rel_err": par["max_rel_err"],
                     "max_err_over_bound": par["max_err_over_bound"], "lse_err": par["lse_err"],
                     "parity_ok": par["ok"],
                     "sdpa_tflops": round(c.flops / ms_sdpa / 1e9, 1),
                     "sdpa_us": round(ms_sdpa * 1e3, 2)}
        del q, k, v, o, lse
    return out


# fa_fwd_kvcache workloads (decode and chunked prefill; no reference counterpart):
# name -> (B, Hq, Hkv, Nq, Nk, d, causal mode)
KVCACHE_CONFIGS = {
    "decode_b8_gqa4_8k": (8, 32, 8, 1, 8192, 128, 0),
    "decode_b1_gqa4_64k": (1, 32, 8, 1, 65536, 128, 0),
    "decode_b8_gqa8_8k": (8, 64, 8, 1, 8192, 128, 0),
    "decode_b16_mha_4k_d64": (16, 16, 16, 1, 4096, 64, 0),
    "chunk_512_of_8k_causal": (1, 32, 8, 512, 8192, 128, 1),
    # speculative decoding: 4 draft tokens x GQA 4 = a 16-row block per KV head
    "spec4_b8_gqa4_8k": (8, 32, 8, 4, 8192, 128, 1),
}


def kvcache_configs(lib, abi, dtype, dev, names=None):
    """Kernel-only time of fa_fwd_kvcache on seeded N(0,1) inputs with a split
    workspace.  Decode is HBM-bound: GB/s counts Q, K, V, O and LSE once
    (K/V > L2, so no flush is needed) and ``hbm_frac`` divides by the measured
    copy bandwidth in MEASURED_PEAKS.json."""
    import torch
    peaks = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json"))) if os.path.exists(
        os.path.join(REPO, "MEASURED_PEAKS.json")) else {}
    hbm = peaks.get("hbm_gbs", 6650.0)
    out = {}
    el = 2
    # SM clocks while these workloads run (they follow the forward loop, so
    # the GPU is warm and may sit at its power cap)
    sampler = ClockSampler(dev.index if dev.index is not None else 0)
    sampler.start()
    for name, (B, Hq, Hkv, Nq, Nk, d, mode) in KVCACHE_CONFIGS.items():
        if names is not None and name not in names:
            continue
        g = torch.Generator(device=dev).manual_seed(7)
        q = torch.randn(B, Hq, Nq, d, device=dev, dtype=torch.float32, generator=g).to(dtype)
        k = torch.randn(B, Hkv, Nk, d, device=dev, dtype=torch.float32, generator=g).to(dtype)
        v = torch.randn(B, Hkv, Nk, d, device=dev, dtype=torch.float32, generator=g).to(dtype)
        o = torch.empty_like(q)
        lse = torch.empty(q.shape[:3], dtype=torch.float32, device=dev)
        nbytes = lib.fa_fwd_kvcache_workspace_bytes(B, Hq, Hkv, Nq, Nk, d)
        ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=dev)
        s = torch.cuda.current_stream(dev)
        args = (abi.ptr(q), abi.ptr(k), abi.ptr(v), abi.ptr(o), abi.ptr(lse), B, Hq, Hkv, Nq, Nk, d,
                1.0 / math.sqrt(d), mode, 1 if dtype == torch.bfloat16 else 0, abi.ptr(ws), nbytes,
                abi.stream_ptr(s))
        fn = lambda: lib.fa_fwd_kvcache(*args)
        assert fn() == 0
        for _ in range(10):
            fn()
        torch.cuda.synchronize()
        n = 200
        ms = time_steps(fn, n, s) / n
        byt = (2 * B * Hkv * Nk * d + 2 * B * Hq * Nq * d) * el + B * Hq * Nq * 4
        if mode:  # causal chunk: the keys a query row sees, averaged
            flops = 4.0 * B * Hq * d * sum(min(Nk, i + 1 + Nk - Nq) for i in range(Nq))
        else:
            flops = 4.0 * B * Hq * Nq * Nk * d
        out[name] = {"us": round(ms * 1e3, 2), "gbs": round(byt / (ms * 1e-3) / 1e9, 1),
                     "hbm_frac": round(byt / (ms * 1e-3) / 1e9 / hbm, 3),
                     "tflops": round(flops / ms / 1e9, 1), "splits_workspace_bytes": int(nbytes)}
        del q, k, v, o, lse, ws
    out["clocks"] = sampler.stop()
    return out


# fa_fwd_varlen / fa_fwd_padded workloads: a batch of sequences of mixed length
# (seeded, 512..8192 tokens) in the packed layout and the same batch padded to
# the longest sequence; name -> (n_seq, Hq, Hkv, d, causal)
VARLEN_CONFIGS = {
    "varlen_16seq_gqa4_causal": (16, 32, 8, 128, True),
    "varlen_16seq_mha_full": (16, 16, 16, 128, False),
}


def varlen_configs(lib, abi, dtype, dev, names=None):
    """Kernel-only time of fa_fwd_varlen (packed) and fa_fwd_padded (padded
    layout, valid ranges) on the same sequences; TFLOPS counts the attended
    (query, key) pairs of every sequence (4*d FLOPs each)."""
    import torch
    out = {}
    for name, (n_seq, Hq, Hkv, d, causal) in VARLEN_CONFIGS.items():
        if names is not None and name not in names:
            continue
        g = torch.Generator().manual_seed(5)
        lens = [int(x) for x in torch.randint(512, 8193, (n_seq,), generator=g)]
        total, nmax = sum(lens), max(lens)
        cu = [0]
        for n in lens:
            cu.append(cu[-1] + n)
        gd = torch.Generator(device=dev).manual_seed(6)
        mk = lambda *shape: torch.randn(*shape, device=dev, generator=gd).to(dtype)
        q, k, v = mk(total, Hq, d), mk(total, Hkv, d), mk(total, Hkv, d)
        o = torch.empty_like(q)
        cu_t = torch.tensor(cu, dtype=torch.int32, device=dev)
        s = torch.cuda.current_stream(dev)
        scale = 1.0 / math.sqrt(d)
        dt = 1 if dtype == torch.bfloat16 else 0
        mode = 1 if causal else 0
        pairs = sum(n * (n + 1) / 2 if causal else float(n) * n for n in lens)
        flops = 4.0 * d * Hq * pairs
        fn = lambda: lib.fa_fwd_varlen(abi.ptr(q), abi.ptr(k), abi.ptr(v), abi.ptr(o), None,
                                       abi.ptr(cu_t), abi.ptr(cu_t), n_seq, Hq, Hkv, total, total,
                                       nmax, nmax, d, scale, mode, dt, abi.stream_ptr(s))
        assert fn() == 0
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        n_it = 20
        ms = time_steps(fn, n_it, s) / n_it
        res = {"seqs": n_seq, "tokens": total, "max_len": nmax, "varlen_us": round(ms * 1e3, 1),
               "varlen_tflops": round(flops / ms / 1e9, 1)}
        # the same batch padded to the longest sequence
        qp = torch.zeros(n_seq, Hq, nmax, d, device=dev, dtype=dtype)
        kp = torch.zeros(n_seq, Hkv, nmax, d, device=dev, dtype=dtype)
        vp = torch.zeros_like(kp)
        for i, n in enumerate(lens):
            qp[i, :, :n] = q[cu[i]:cu[i + 1]].transpose(0, 1)
            kp[i, :, :n] = k[cu[i]:cu[i + 1]].transpose(0, 1)
            vp[i, :, :n] = v[cu[i]:cu[i + 1]].transpose(0, 1)
        op = torch.empty_like(qp)
        zeros = torch.zeros(n_seq, dtype=torch.int32, device=dev)
        ends = torch.tensor(lens, dtype=torch.int32, device=dev)
        fp = lambda: lib.fa_fwd_padded(abi.ptr(qp), abi.ptr(kp), abi.ptr(vp), abi.ptr(op), None,
                                       abi.ptr(zeros), abi.ptr(ends), abi.ptr(zeros), abi.ptr(ends),
                                       n_seq, Hq, Hkv, nmax, nmax, d, scale, mode, dt,
                                       abi.stream_ptr(s))
        assert fp() == 0
        for _ in range(3):
            fp()
        torch.cuda.synchronize()
        ms_p = time_steps(fp, n_it, s) / n_it
        res.update({"padded_us": round(ms_p * 1e3, 1), "padded_tflops": round(flops / ms_p / 1e9, 1)})
        out[name] = res
        del q, k, v, o, qp, kp, vp, op
    return out


# fa_bwd workloads (attention backward; no reference counterpart):
# name -> (B, Hq, Hkv, N, d, causal)
BACKWARD_CONFIGS = {
    "bwd_c5": (4, 32, 32, 8192, 128, False),
    "bwd_c5c": (4, 32, 32, 8192, 128, True),
    "bwd_c4_gqa": (2, 32, 8, 4096, 128, True),
    "bwd_c2_d64": (4, 12, 12, 1024, 64, False),
}


def backward_configs(lib, abi, dtype, dev, names=None):
    """Kernel-only time of fa_bwd (prep + dK/dV + dQ kernels) on seeded N(0,1)
    inputs, O and LSE from fa_fwd.  TFLOPS counts the five matrix products of
    the FlashAttention-2 backward, 10*B*Hq*N^2*d (causal: the visible pairs
    only); the kernels recompute S and dP in both passes (14*N^2*d executed)."""
    import torch
    out = {}
    for name, (B, Hq, Hkv, N, d, causal) in BACKWARD_CONFIGS.items():
        if names is not None and name not in names:
            continue
        g = torch.Generator(device=dev).manual_seed(11)
        mk = lambda h: torch.randn(B, h, N, d, device=dev, dtype=torch.float32,
                                   generator=g).to(dtype)
        q, k, v, do = mk(Hq), mk(Hkv), mk(Hkv), mk(Hq)
        o = torch.empty_like(q)
        lse = torch.empty(q.shape[:3], dtype=torch.float32, device=dev)
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        nbytes = lib.fa_bwd_workspace_bytes(B, Hq, N)
        ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=dev)
        s = torch.cuda.current_stream(dev)
        scale = 1.0 / math.sqrt(d)
        dt = 1 if dtype == torch.bfloat16 else 0
        assert lib.fa_fwd(abi.ptr(q), abi.ptr(k), abi.ptr(v), abi.ptr(o), abi.ptr(lse), B, Hq, Hkv,
                          N, d, scale, int(causal), dt, abi.stream_ptr(s)) == 0
        args = (abi.ptr(q), abi.ptr(k), abi.ptr(v), abi.ptr(o), abi.ptr(do), abi.ptr(lse),
                abi.ptr(dq), abi.ptr(dk), abi.ptr(dv), B, Hq, Hkv, N, d, scale, int(causal), dt,
                abi.ptr(ws), nbytes, abi.stream_ptr(s))
        fn = lambda: lib.fa_bwd(*args)
        assert fn() == 0
        for _ in range(5):
            fn()
        torch.cuda.synchronize()
        pairs = N * (N + 1) / 2 if causal else float(N) * N
        flops = 10.0 * B * Hq * d * pairs
        n = max(10, min(500, int(4e12 / flops)))
        ms = time_steps(fn, n, s) / n
        if lib.fa_device_status(0) != 0:
            raise RuntimeError("device watchdog fired in fa_bwd")
        out[name] = {"tflops": round(flops / ms / 1e9, 1), "us": round(ms * 1e3, 2),
                     "shape": f"B={B} Hq={Hq} Hkv={Hkv} N={N} d={d} causal={int(causal)}"}
        del q, k, v, do, o, lse, dq, dk, dv, ws
    return out


if __name__ == "__main__":
    main()
