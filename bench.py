#!/usr/bin/env python3
"""Benchmark of the B200 ChunkGatedDeltaRuleFwdH (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...        (N > 1)

Workload (default): the north-star configuration -- bf16, B=4, T=8192,
H=32, K=V=128, chunk 64, h0 ~ 0.1 randn (fp32), final_state stored -- per
rank, inputs generated on the device from seed + rank (weak scaling: the
(sequence, head) pairs are independent, so every rank runs its own shard and
there is no collective on the data path).  ``--config c5`` runs the
the benchmark's multi-GPU config instead (B=8, T=8192, H=64, K=128, V=256) with
its (b, h) pairs split evenly over the ranks (strong scaling).

Metric: fwd_h tokens/s (tokens = B*T per call), whole job.  ``value`` is
device time (CUDA events on the launching stream, max over ranks) with
inputs resident in HBM; inputs and outputs total ~1.9 GB per rank, far
beyond the 126 MB L2, so no flush is needed between steps.  ``e2e`` is the
same metric through the public Python API with pinned host buffers, the
host->device copy of every input and the device->host copy of every output
inside the timed region (through the host-memory front end, which overlaps
the two directions of copies with the kernels).  ``roofline`` relates the op's algorithmic HBM
bytes per launch to the measured HBM copy bandwidth.  ``cpu_baseline`` is
the reference's arithmetic (the CPU oracle, a restatement of the reference
PyTorch code) timed on this host's cores on a bounded sample.

``parity`` is the same CPU oracle used as the checker of the last timed output
(sequence 0, two heads; rank 0, untimed).  ``strong_scaling`` times the
multi-GPU configuration (B=8, T=8192, H=64, K=128, V=256) with its heads split
over the ranks, after the headline and outside its timed region; rank 0 also
times the unsplit configuration.  ``e2e.copy_only_ms_per_step`` moves the e2e
step's bytes with no kernel, which names what bounds the e2e number.

``--impl reference`` times that CPU implementation alone (rank 0; other
ranks exit), as the reference arm: the whole job per step where it fits a few
seconds.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIGS = {
    "ns": dict(B=4, T=8192, H=32, HK=32, K=128, V=128, scaling="weak"),
    "c5": dict(B=8, T=8192, H=64, HK=64, K=128, V=256, scaling="strong"),
    "c2": dict(B=2, T=4096, H=16, HK=16, K=128, V=128, scaling="weak"),
    "c3": dict(B=1, T=65536, H=32, HK=32, K=128, V=128, scaling="weak", h0=False),
    # a quarter of the north-star workload (one sequence per head): the small case of ncu captures
    "nsq": dict(B=1, T=8192, H=32, HK=32, K=128, V=128, scaling="weak"),
    # 16 sequences packed into T=32768 via cu_seqlens (lengths uniform in [64, 4096], multiples of 64)
    "c4": dict(B=1, T=32768, H=32, HK=32, K=128, V=128, scaling="weak", seqs=16),
    # the widest head the reference accepts (K = V = 256): 32 (sequence, head) pairs x 4 V tiles
    "w256": dict(B=4, T=8192, H=8, HK=8, K=256, V=256, scaling="weak"),
    # a quarter of it (one sequence per head): the small case of ncu captures
    "w256q": dict(B=1, T=8192, H=8, HK=8, K=256, V=256, scaling="weak"),
}


def varlen_lengths(n_seq, total, seed, lo=64, hi=4096):
    """Seeded lengths, uniform in [lo, hi], multiples of 64, rescaled to sum to `total`."""
    import numpy as np
    rng = np.random.default_rng(seed)
    lens = np.maximum(64, (rng.integers(lo, hi + 1, size=n_seq) // 64) * 64)
    lens = np.maximum(64, np.round(lens * (total / lens.sum()) / 64).astype(int) * 64)
    lens[-1] += total - lens.sum()
    return [int(x) for x in lens]


def algorithmic_bytes(B, T, H, HK, K, V, has_h0=True, store_final=True, save_v=True, final_bytes=4, h0_bytes=4,
                      N=None, NT=None):
    """Each tensor read or written once: k, w, u, g, v_new, h, h0, final.
    N sequences (default B) and NT chunks in h (default B's ceil(T/64))."""
    NT = (T + 63) // 64 if NT is None else NT
    N = B if N is None else N
    b = B * T * HK * K * 2 + B * T * H * K * 2 + B * T * H * V * 2 + B * T * H * 4
    if save_v:
        b += B * T * H * V * 2
    b += (B * NT if N == B else NT) * H * K * V * 2
    if has_h0:
        b += N * H * K * V * h0_bytes
    if store_final:
        b += N * H * K * V * final_bytes
    return b


def config_bytes(c, seed, has_h0=True):
    """Algorithmic bytes of one step of config `c` (its varlen lengths drawn
    with the same seed as the inputs)."""
    n_seq, n_chunks = c["B"], None
    if "seqs" in c:
        n_seq = c["seqs"]
        n_chunks = sum((L + 63) // 64 for L in varlen_lengths(c["seqs"], c["T"], seed))
    return algorithmic_bytes(c["B"], c["T"], c["H"], c["HK"], c["K"], c["V"], has_h0=has_h0, N=n_seq, NT=n_chunks)


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def load_traffic(config, kernel):
    """DRAM bytes per launch of `kernel` on `config`, from the committed ncu
    summary profiles/traffic.txt (lines "config kernel bytes"), or None."""
    p = ROOT / "profiles" / "traffic.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 3 and parts[0] == config and parts[1] == kernel:
            try:
                return float(parts[2])
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    QUERY = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None):
        self.uuid = uuid
        self.proc = None
        self.t_start = self.t_stop = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
            os.close(fd)
            cmd = ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "50"]
            if self.uuid:
                cmd.insert(1, f"--id={self.uuid}")
            self.proc = subprocess.Popen(cmd, stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def mark(self, which):
        setattr(self, which, time.time())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.12)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 10:
                continue
            rows.append(parts)
        os.unlink(self.path)
        sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        mx = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in rows:
            for name, val in zip(names, r[6:10]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows)}


def dist_setup():
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def gpu_numa_cpus(dev):
    """(NUMA node, CPUs of that node this process may use) of the GPU's PCI device,
    from sysfs; (None, None) where the platform does not say."""
    import torch
    try:
        pr = torch.cuda.get_device_properties(dev)
        bdf = f"{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        node = int(Path(f"/sys/bus/pci/devices/{bdf}/numa_node").read_text().strip())
        if node < 0:
            return None, None
        cpus = set()
        for part in Path(f"/sys/devices/system/node/node{node}/cpulist").read_text().strip().split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        cpus &= os.sched_getaffinity(0)
        return node, (cpus or None)
    except Exception:
        return None, None


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    """Largest value over all ranks (the device time of the slowest rank)."""
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def shard(cfg, world, rank):
    """Per-rank problem: weak scaling keeps the config per rank; strong
    scaling splits the (b, h) pairs by heads."""
    c = dict(cfg)
    if cfg["scaling"] == "strong" and world > 1:
        assert cfg["H"] % world == 0
        c["H"] = cfg["H"] // world
        c["HK"] = cfg["HK"] // world
    return c


def gen_inputs(c, seed, device):
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    B, T, H, HK, K, V = c["B"], c["T"], c["H"], c["HK"], c["K"], c["V"]
    k = torch.randn(B, T, HK, K, device=device, generator=g)
    k = (k / k.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    beta = torch.sigmoid(torch.randn(B, T, H, device=device, generator=g))
    w = (beta[..., None] * k.float().repeat_interleave(H // HK, dim=2)).to(torch.bfloat16)
    u = (0.5 * torch.randn(B, T, H, V, device=device, generator=g)).to(torch.bfloat16)
    gl = torch.nn.functional.logsigmoid(torch.randn(B, T, H, device=device, generator=g) + 2.0)
    pad = (-T) % 64
    gl = torch.nn.functional.pad(gl, (0, 0, 0, pad)).view(B, (T + pad) // 64, 64, H).cumsum(2).view(B, T + pad, H)
    gl = gl[:, :T].contiguous()
    N = c.get("seqs", B)
    h0 = (0.1 * torch.randn(N, H, K, V, device=device, generator=g)) if c.get("h0", True) else None
    out = dict(k=k, w=w, u=u, g=gl, initial_state=h0)
    if "seqs" in c:
        import cann_operator_challenge_august_b200 as cg
        lens = varlen_lengths(c["seqs"], T, seed)
        cu = [0]
        for L in lens:
            cu.append(cu[-1] + L)
        out["cu_seqlens"] = torch.tensor(cu, dtype=torch.int64, device=device)
        out["chunk_indices"] = cg.prepare_chunk_indices(out["cu_seqlens"])
    return out


def cpu_sample(c, P, chunks, seed=0):
    """Seeded inputs of P (sequence, head) pairs x `chunks` chunks of config c, in
    the oracle's layout (bf16 as uint16 bits), with the benchmark's distributions."""
    import numpy as np
    import torch
    gen = torch.Generator().manual_seed(seed)
    T = 64 * chunks
    k = torch.randn(1, T, P, c["K"], generator=gen)
    k = (k / k.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    w = (torch.sigmoid(torch.randn(1, T, P, 1, generator=gen)) * k.float()).to(torch.bfloat16)
    u = (0.5 * torch.randn(1, T, P, c["V"], generator=gen)).to(torch.bfloat16)
    g = torch.nn.functional.logsigmoid(torch.randn(1, T, P, generator=gen) + 2.0)
    g = g.view(1, chunks, 64, P).cumsum(2).view(1, T, P)
    h0 = 0.1 * torch.randn(1, P, c["K"], c["V"], generator=gen)
    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    return bits(k), bits(w), bits(u), g.numpy(), h0.numpy()


def cpu_time(sample, threads):
    """Seconds of one CPU-oracle run (reference arithmetic) over `sample`."""
    sys.path.insert(0, str(ROOT / "tests"))
    from oracle import oracle as o  # the reference arithmetic, restated (timed baseline)
    t0 = time.perf_counter()
    o.fwd_h(*sample, mode="reference", n_threads=threads)
    return time.perf_counter() - t0


def cpu_parity_check(c, inp, out, numerics, heads=None):
    """The CPU oracle as the checker of one timed output (outside every timed
    region): sequence 0 and two heads, against the arithmetic the bench ran and
    against the reference semantics, at the north-star rtol = atol = 2e-2."""
    import numpy as np
    import torch
    sys.path.insert(0, str(ROOT / "tests"))
    from oracle import oracle as o  # the checker

    H, HK = c["H"], c["HK"]
    heads = heads or [0, H - 1]
    kheads = [hh // (H // HK) for hh in heads]
    cu = inp.get("cu_seqlens")
    t0, t1 = (0, c["T"]) if cu is None else (int(cu[0]), int(cu[1]))
    nc = (t1 - t0 + 63) // 64
    bits = lambda t: t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    k = bits(inp["k"][0:1, t0:t1, kheads])
    w = bits(inp["w"][0:1, t0:t1, heads])
    u = bits(inp["u"][0:1, t0:t1, heads])
    g = inp["g"][0:1, t0:t1, heads].contiguous().cpu().numpy()
    h0 = None if inp["initial_state"] is None else inp["initial_state"][0:1, heads].contiguous().cpu().numpy()
    h, v, f = out
    got = {"h": h[0:1, 0:nc, heads].float().cpu().numpy(), "v_new": v[0:1, t0:t1, heads].float().cpu().numpy(),
           "final_state": f[0:1, heads].float().cpu().numpy()}

    def stats(mode):
        oh, ov, of = o.fwd_h(k, w, u, g, h0, None, mode=mode, final_dtype="f32")
        ref = {"h": oh, "v_new": ov, "final_state": of}
        bad = n = 0
        mx = 0.0
        for name in ref:
            r = ref[name]
            r = (r.astype(np.uint32) << 16).view(np.float32) if r.dtype == np.uint16 else r
            a = got[name].reshape(-1).astype(np.float64)
            r = r.reshape(-1).astype(np.float64)
            err = np.abs(a - r)
            bad += int((~(err <= 2e-2 + 2e-2 * np.abs(r))).sum())
            n += a.size
            mx = max(mx, float(err.max(initial=0.0)))
        return {"mode": mode, "bad": bad, "n": n, "max_abs": mx}

    res = {"sample": f"sequence 0 (tokens {t0}..{t1}), heads {heads}: h, v_new, final_state",
           "tolerance": "rtol = atol = 2e-2", "vs_oracle": stats(numerics)}
    res["bad"], res["n"], res["max_abs"] = res["vs_oracle"]["bad"], res["vs_oracle"]["n"], res["vs_oracle"]["max_abs"]
    if numerics != "reference":
        res["vs_reference_semantics"] = stats("reference")
    return res


def time_launches(step, steps, warmup, stream, world):
    """Device time of `steps` launches of `step` after `warmup`: the mean per
    launch (CUDA events on the launching stream), max over ranks."""
    import torch
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * steps)]
    for i in range(steps):
        ev[2 * i].record(stream)
        step()
        ev[2 * i + 1].record(stream)
    torch.cuda.synchronize()
    ms = sum(ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(steps)) / steps
    return max_over_ranks(ms, world)


def strong_scaling_leg(args, world, rank, dev, stream):
    """The benchmark's multi-GPU configuration (B=8, T=8192, H=64, K=128, V=256)
    with its value heads split over the ranks (no collective on the data path),
    timed after the headline and outside its timed region.  Rank 0 also times the
    whole configuration on its own GPU, so that one run gives both ends of the
    strong-scaling curve."""
    import torch
    import cann_operator_challenge_august_b200 as cg
    full = CONFIGS["c5"]
    c = shard(full, world, rank)
    opts = dict(numerics=args.numerics)

    def run(cfg, seed):
        inp = gen_inputs(cfg, seed=seed, device=dev)
        step = lambda: cg.chunk_gated_delta_rule_fwd_h(inp["k"], inp["w"], inp["u"], inp["g"],  # noqa: E731
                                                      inp["initial_state"], **opts)
        return inp, step

    inp, step = run(c, 2000 + rank)
    ms_n = time_launches(step, args.steps, args.warmup, stream, world)
    del inp, step
    torch.cuda.empty_cache()
    ms_1 = ms_n
    if world > 1:
        t = 0.0
        if rank == 0:
            inp, step = run(full, 2000)
            t = time_launches(step, args.steps, args.warmup, stream, 1)
            del inp, step
            torch.cuda.empty_cache()
        ms_1 = max_over_ranks(t, world)
    peak, _ = load_peaks()
    shard_bytes = config_bytes(c, 2000)
    full_bytes = config_bytes(full, 2000)
    tokens = full["B"] * full["T"]
    return {
        "config": (f"c5: B={full['B']} T={full['T']} H={full['H']} K={full['K']} V={full['V']}, "
                   f"{c['H']} value heads per rank, no collective on the data path"),
        "ranks": world,
        "ms_per_launch": ms_n,
        "tokens_per_s": tokens / (ms_n / 1000.0),
        "hbm_gbs_per_gpu": shard_bytes / (ms_n / 1000.0) / 1e9,
        "roofline_frac_per_gpu": shard_bytes / (ms_n / 1000.0) / 1e9 / peak,
        "one_gpu_ms_per_launch": ms_1,
        "one_gpu_roofline_frac": full_bytes / (ms_1 / 1000.0) / 1e9 / peak,
        "speedup_vs_one_gpu": ms_1 / ms_n,
        "efficiency_vs_one_gpu": ms_1 / ms_n / world,
    }


def copy_only_ms(host_in, host_out, dev, steps, world):
    """The e2e leg's host<->device traffic alone: every input copied in on one
    stream while every output is copied out on another, no kernel; CUDA events,
    mean per step, max over ranks.  Its ratio to the e2e time says whether the
    copies bound the end-to-end number."""
    import torch
    cur = torch.cuda.current_stream(dev)
    dev_in = [torch.empty(x.shape, dtype=x.dtype, device=dev) for x in host_in]
    dev_out = [torch.empty(x.shape, dtype=x.dtype, device=dev) for x in host_out]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def once():
        s_in.wait_stream(cur)
        s_out.wait_stream(cur)
        with torch.cuda.stream(s_in):
            for d, h in zip(dev_in, host_in):
                d.copy_(h, non_blocking=True)
        with torch.cuda.stream(s_out):
            for h, d in zip(host_out, dev_out):
                h.copy_(d, non_blocking=True)
        cur.wait_stream(s_in)
        cur.wait_stream(s_out)

    once()
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    for _ in range(steps):
        once()
    e1.record(cur)
    torch.cuda.synchronize()
    return max_over_ranks(e0.elapsed_time(e1) / steps, world)


def cpu_reference_steps(c, steps, warmup, per_step_s):
    """The CPU oracle (reference arithmetic) with every host thread, `steps` timed
    steps after `warmup`: each step runs the whole job (every (sequence, head)
    pair, every chunk) when that fits `per_step_s`, else a fixed subset of pairs
    (named in the description).  Returns (tokens/s, seconds per step, fraction of
    the job per step, description, threads)."""
    threads = len(os.sched_getaffinity(0))
    NT = (c["T"] + 63) // 64
    pairs = c["B"] * c["H"]
    probe = cpu_time(cpu_sample(c, min(threads, pairs), 1), threads)
    est_pair_chunk_s = probe / min(threads, pairs) * threads  # wall time of `threads` pair-chunks in parallel
    P = pairs
    while P > threads and est_pair_chunk_s * (P / threads) * NT > per_step_s:
        P = max(threads, P // 2)
    sample = cpu_sample(c, P, NT)
    times = []
    for i in range(warmup + steps):
        dt = cpu_time(sample, threads)
        if i >= warmup:
            times.append(dt)
    step_s = statistics.median(times)
    frac = P / pairs
    value = c["B"] * c["T"] * frac / step_s
    desc = (f"{P} of {pairs} (sequence, head) pairs x all {NT} chunks per step"
            + ("" if P == pairs else f" ({frac:.3f} of the job; tokens/s counts that fraction of B*T)")
            + f", median of {steps} steps after {warmup} warm-up steps, {threads} threads")
    return value, step_s, frac, desc, threads


def run_reference_arm(args, cfg_name, c, world, rank):
    """The reference arm: the CPU implementation of the path on this host's cores.
    Each step runs the whole job when that fits about 3 s, so ms_per_step is the
    measured time of a step; a larger job runs a fixed subset of pairs per step
    and says so."""
    if rank != 0:
        return 0
    K, W = args.steps, args.warmup
    value, step_s, frac, desc, threads = cpu_reference_steps(c, K, W, max(0.5, min(3.0, 150.0 / max(1, K + W))))
    line = {
        "impl": "reference",
        "metric": "fwd_h tokens/s",
        "value": value,
        "unit": "tokens/s",
        "n_gpus": args.gpus,
        "steps": K,
        "warmup": W,
        "ms_per_step": 1000.0 * step_s,
        "full_job_ms": 1000.0 * step_s / frac,
        "higher_is_better": True,
        "scaling": c["scaling"],
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": config_block(cfg_name, c, world, config_bytes(c, 1000 + rank)),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": desc},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def _plan_outputs(inp, c, dev):
    """Output tensors shaped for the phase-1 plan query (never launched)."""
    import torch
    B, T, H, K, V = c["B"], c["T"], c["H"], c["K"], c["V"]
    NT = inp["chunk_indices"].shape[0] if "chunk_indices" in inp else (T + 63) // 64
    N = c.get("seqs", B)
    return (torch.empty(B, NT, H, K, V, dtype=torch.bfloat16, device=dev),
            torch.empty(B, T, H, V, dtype=torch.bfloat16, device=dev),
            torch.empty(N, H, K, V, dtype=torch.float32, device=dev))


def config_block(name, c, world, nbytes):
    varlen = (f", varlen: {c['seqs']} sequences packed into T (lengths multiples of 64 in [64, 4096])"
              if "seqs" in c else "")
    block = {
        "workload": f"{name}: chunk_gated_delta_rule_fwd_h bf16 B={c['B']} T={c['T']} H={c['H']} "
                    f"K={c['K']} V={c['V']} chunk=64{varlen}, h0 fp32, final_state fp32, v_new stored"
                    + (" (per rank)" if c["scaling"] == "weak" else f" (heads split over {world} ranks)"),
        "B": c["B"], "T": c["T"], "H": c["H"], "K": c["K"], "V": c["V"], "chunk": 64,
        "tokens_per_step_per_rank": c["B"] * c["T"],
        "l2": f"inputs+outputs {nbytes / 1e9:.2f} GB per rank > 126 MB L2 (no flush needed)",
        "parallelism": (f"{world} independent rank(s), each with the whole workload, no collective"
                        if c["scaling"] == "weak" else
                        f"heads split over {world} rank(s), no collective on the data path"),
    }
    if "seqs" in c:
        block["sequences"] = c["seqs"]
    return block


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="ns")
    ap.add_argument("--numerics", choices=["fp32_state", "reference"], default="fp32_state")
    ap.add_argument("--v-tile", type=int, default=0)
    ap.add_argument("--chains", type=int, default=0, help="chains per CTA (0: the planner's choice)")
    ap.add_argument("--gdr-path", choices=["auto", "fused", "three_kernels"], default="auto",
                    help="--op gdr: the recurrence and output kernels (default: the planner's choice)")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the oracle check of the timed output")
    ap.add_argument("--no-strong-scaling", action="store_true",
                    help="skip the head-sharded multi-GPU configuration after the headline")
    ap.add_argument("--op", choices=["fwd_h", "chunk_o", "wy", "gdr"], default="fwd_h",
                    help="fwd_h: the recurrence (the headline); chunk_o: the chunk output that consumes it; "
                         "wy: the WY representation that feeds it; gdr: the whole forward operator")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    cfg = CONFIGS[args.config]
    if args.op == "chunk_o" and args.impl == "ours":
        return main_chunk_o(args)
    if args.op == "wy" and args.impl == "ours":
        return main_stage(args)
    if args.op == "gdr" and args.impl == "ours":
        return main_gdr(args)

    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        return run_reference_arm(args, args.config, shard(cfg, 1, 0), world, rank)

    import torch
    import cann_operator_challenge_august_b200 as cg

    world, rank, local = dist_setup()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    c = shard(cfg, world, rank)
    inp = gen_inputs(c, seed=1000 + rank, device=dev)
    stream = torch.cuda.current_stream(dev)
    opts = dict(numerics=args.numerics, v_tile=args.v_tile, chains=args.chains)

    def step():
        return cg.chunk_gated_delta_rule_fwd_h(inp["k"], inp["w"], inp["u"], inp["g"], inp["initial_state"],
                                               cu_seqlens=inp.get("cu_seqlens"), chunk_indices=inp.get("chunk_indices"),
                                               **opts)

    for _ in range(args.warmup):
        out = step()
    torch.cuda.synchronize()
    del out
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    clocks = ClockSampler(uuid)
    clocks.start()
    time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps)]
    t_start = torch.cuda.Event(enable_timing=True)
    t_stop = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(args.steps):
        ev[2 * i].record(stream)
        out = step()
        ev[2 * i + 1].record(stream)
    t_stop.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    elapsed_ms = t_start.elapsed_time(t_stop)
    per_launch_ms = sum(ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(args.steps)) / args.steps
    elapsed_ms = max_over_ranks(elapsed_ms, world)
    per_launch_ms = max_over_ranks(per_launch_ms, world)
    ms_per_step = elapsed_ms / args.steps
    tokens_per_step = c["B"] * c["T"] * world
    value = tokens_per_step / (ms_per_step / 1000.0)

    # ---- the last timed output, checked against the CPU oracle (rank 0, untimed)
    parity = None
    if rank == 0 and not args.no_parity:
        parity = cpu_parity_check(c, inp, out, args.numerics)

    # ---- e2e: public API with pinned host buffers, copies inside the timed region.  The
    # host side runs on the CPUs of the GPU's NUMA node (where the platform names one), so
    # that the pinned buffers are placed in that node's memory; restored afterwards.
    all_cpus = os.sched_getaffinity(0)
    numa_node, numa_cpus = gpu_numa_cpus(dev)
    if numa_cpus:
        os.sched_setaffinity(0, numa_cpus)
    host = {n: (x.cpu().pin_memory() if x is not None else None) for n, x in inp.items()}
    # bytes the front end copies to the device (cu_seqlens is read on the host; the chunk
    # list is derived from it)
    h2d = sum(x.numel() * x.element_size() for n, x in host.items()
              if x is not None and n not in ("cu_seqlens", "chunk_indices"))
    h_out, v_out, f_out = out
    host_out = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in (h_out, v_out, f_out)]
    d2h = sum(t.numel() * t.element_size() for t in host_out)
    del out, h_out, v_out, f_out

    def e2e_step():
        # the host-memory front end: pieces of the batch pipelined, copies in and out overlapped
        cg.chunk_gated_delta_rule_fwd_h_host(host["k"], host["w"], host["u"], host["g"], host["initial_state"],
                                             host.get("cu_seqlens"), device=dev, out=tuple(host_out), **opts)

    e2e_ms = e2e_value = None
    if args.e2e_steps > 0:
        e2e_step()
        torch.cuda.synchronize()
        barrier(world)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.e2e_steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1), world) / args.e2e_steps
        e2e_value = tokens_per_step / (e2e_ms / 1000.0)
    copy_ms = None
    if args.e2e_steps > 0:
        host_in = [x for n, x in host.items() if x is not None and n not in ("cu_seqlens", "chunk_indices")]
        copy_ms = copy_only_ms(host_in, host_out, dev, args.e2e_steps, world)
    os.sched_setaffinity(0, all_cpus)

    nbytes = config_bytes(c, 1000 + rank, has_h0=inp["initial_state"] is not None)
    if "chunk_indices" in inp:
        assert sum((L + 63) // 64 for L in varlen_lengths(c["seqs"], c["T"], 1000 + rank)) == inp["chunk_indices"].shape[0]
    peak, peak_kind = load_peaks()

    # ---- head-sharded multi-GPU configuration (strong scaling), after everything above
    strong = None
    if not args.no_strong_scaling and args.config == "ns" and CONFIGS["c5"]["H"] % world == 0:
        strong = strong_scaling_leg(args, world, rank, dev, stream)
    achieved = nbytes / (per_launch_ms / 1000.0) / 1e9
    plan = cg.ChunkGatedDeltaRuleFwdH(inp["k"], inp["w"], inp["u"], inp["g"], inp["initial_state"],
                                      inp.get("cu_seqlens"), inp.get("chunk_indices"), 64,
                                      *_plan_outputs(inp, c, dev), layout="token_major", **opts).plan
    kernel_name = {1: "tc", 2: "general", 3: "tc_fused"}.get(plan["kernel"], str(plan["kernel"]))
    traffic = load_traffic(args.config, kernel_name)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, _, _, desc, threads = cpu_reference_steps(c, 3, 1, 3.0)
        cpu = {"value": rate, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": desc}

    if rank == 0:
        line = {
            "metric": "fwd_h tokens/s",
            "value": value,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_per_step,
            "higher_is_better": True,
            "scaling": c["scaling"],
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded, generated on device per rank)",
            "numerics": args.numerics,
            "config": config_block(args.config, c, world, nbytes),
            "gpu_launches": args.steps * (2 if "cu_seqlens" in inp else 1),
            "roofline": {
                "bound": "hbm",
                "achieved": achieved,
                "peak": peak,
                "unit": "GB/s",
                "frac": achieved / peak,
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback",
                "algorithmic_bytes_per_launch": nbytes,
                "launch_ms": per_launch_ms,
                "traffic": traffic,
                "kernel": kernel_name,
            },
            "hbm_gbs_per_gpu": achieved,
            "clocks": clk,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms,
                    "copy_gbs_per_rank": None if e2e_ms is None else (h2d + d2h) / (e2e_ms / 1000.0) / 1e9,
                    "copy_gbs_total": None if e2e_ms is None else world * (h2d + d2h) / (e2e_ms / 1000.0) / 1e9,
                    "copy_only_ms_per_step": copy_ms,
                    "host_numa_node": numa_node,
                    "host_cpus": None if not numa_cpus else len(numa_cpus),
                    "e2e_over_copy_only": None if copy_ms is None else e2e_ms / copy_ms},
            "cpu_baseline": cpu,
            "parity": parity,
            "strong_scaling": strong,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def chunk_o_bytes(c, n_chunks=None):
    """Algorithmic bytes of one chunk-output launch: q, k, v_new, g, h read
    once, o written once."""
    B, T, H, HK, K, V = c["B"], c["T"], c["H"], c["HK"], c["K"], c["V"]
    NT = (T + 63) // 64 if n_chunks is None else n_chunks
    rows = B * NT if n_chunks is None else NT
    return B * T * (2 * HK * K * 2 + 2 * H * V * 2 + H * 4) + rows * H * K * V * 2


def cpu_chunk_o_rate(c, inp, q, h, v_new, budget_s):
    """The chunk-output oracle (numpy; BLAS threads as numpy configures them)
    on the first chunks of batch row 0, all heads, scaled to the whole job."""
    import numpy as np
    from oracle import gdr_stages as G

    def sample(nc):
        T = 64 * nc
        cvt = lambda t: t[:1, :T].float().cpu().numpy()  # noqa: E731
        return (cvt(q), cvt(inp["k"]), cvt(v_new), h[:1, :nc].float().cpu().numpy(), cvt(inp["g"]))

    def timed(nc):
        a = sample(nc)
        t0 = time.perf_counter()
        G.chunk_o(*a)
        return time.perf_counter() - t0

    t1 = timed(1)
    NT = (c["T"] + 63) // 64
    nc = int(max(1, min(NT, budget_s / max(t1, 1e-4))))
    dt = timed(nc)
    job_chunks = c["B"] * NT
    rate = c["B"] * c["T"] * (nc / dt) / job_chunks
    threads = int(os.environ.get("OMP_NUM_THREADS", "0") or 0) or len(os.sched_getaffinity(0))
    desc = (f"{nc} of {job_chunks} (batch row, chunk) tiles, all {c['H']} heads ({dt:.2f} s), scaled linearly "
            f"to the whole job")
    return rate, desc, threads


def main_chunk_o(args) -> int:
    """--op chunk_o: the chunk output that consumes fwd_h's h and v_new, on the
    same workload (h and v_new produced by the recurrence kernel once)."""
    import torch
    import cann_operator_challenge_august_b200 as cg

    world, rank, local = dist_setup()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    c = shard(CONFIGS[args.config], world, rank)
    if "seqs" in c:
        raise SystemExit("--op chunk_o runs the fixed-length configurations")
    inp = gen_inputs(c, seed=1000 + rank, device=dev)
    gen = torch.Generator(device=dev).manual_seed(2000 + rank)
    q = torch.randn(c["B"], c["T"], c["HK"], c["K"], device=dev, generator=gen)
    q = (q / q.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    h, v_new, _ = cg.chunk_gated_delta_rule_fwd_h(inp["k"], inp["w"], inp["u"], inp["g"], inp["initial_state"])
    del inp["w"], inp["u"]
    stream = torch.cuda.current_stream(dev)

    def step():
        return cg.chunk_fwd_o(q, inp["k"], v_new, h, inp["g"])

    for _ in range(args.warmup):
        out = step()
    torch.cuda.synchronize()
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    clocks = ClockSampler(uuid)
    clocks.start()
    time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps)]
    t_start = torch.cuda.Event(enable_timing=True)
    t_stop = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(args.steps):
        ev[2 * i].record(stream)
        out = step()
        ev[2 * i + 1].record(stream)
    t_stop.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    elapsed_ms = max_over_ranks(t_start.elapsed_time(t_stop), world)
    per_launch_ms = max_over_ranks(sum(ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(args.steps)) / args.steps,
                                   world)
    ms_per_step = elapsed_ms / args.steps
    tokens_per_step = c["B"] * c["T"] * world
    value = tokens_per_step / (ms_per_step / 1000.0)

    host = {n: t.cpu().pin_memory() for n, t in (("q", q), ("k", inp["k"]), ("v_new", v_new), ("h", h),
                                                  ("g", inp["g"]))}
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    host_o = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    d2h = host_o.numel() * host_o.element_size()

    def e2e_step():
        d = {n: t.to(dev, non_blocking=True) for n, t in host.items()}
        host_o.copy_(cg.chunk_fwd_o(d["q"], d["k"], d["v_new"], d["h"], d["g"]), non_blocking=True)

    e2e_ms = e2e_value = None
    if args.e2e_steps > 0:
        e2e_step()
        torch.cuda.synchronize()
        barrier(world)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.e2e_steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1), world) / args.e2e_steps
        e2e_value = tokens_per_step / (e2e_ms / 1000.0)

    nbytes = chunk_o_bytes(c)
    peak, peak_kind = load_peaks()
    achieved = nbytes / (per_launch_ms / 1000.0) / 1e9
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, desc, threads = cpu_chunk_o_rate(c, inp, q, h, v_new, 10.0)
        cpu = {"value": rate, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": desc}
    if rank == 0:
        line = {
            "metric": "chunk_o tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": c["scaling"], "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded, generated on device per rank; h and v_new from the recurrence kernel)",
            "config": dict(config_block(args.config, c, world, nbytes),
                           workload=f"{args.config}: chunk output bf16 B={c['B']} T={c['T']} H={c['H']} "
                                    f"K={c['K']} V={c['V']} chunk=64 (q, k, v_new, h, g in; o out)"),
            "gpu_launches": args.steps,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                         else "fallback",
                         "algorithmic_bytes_per_launch": nbytes, "launch_ms": per_launch_ms,
                         "traffic": load_traffic(args.config, "chunk_o"), "kernel": "chunk_o"},
            "clocks": clk,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms},
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def wy_bytes(c):
    """Algorithmic bytes of one WY launch: k, v, beta, g read once; w, u, g_c
    written once."""
    B, T, H, HK, K, V = c["B"], c["T"], c["H"], c["HK"], c["K"], c["V"]
    return B * T * (HK * K * 2 + H * V * 2 + H * 2 + H * 4 + H * K * 2 + H * V * 2 + H * 4)


def gen_wy_inputs(c, seed, device):
    """k L2-normalised, v ~ randn, beta ~ U(0, 1), g ~ U(-1, 0): the reference
    operator's input constraints (ref/chunk_gated_delta_rule/tests/assets/impl/inputs.py)."""
    import torch
    g0 = torch.Generator(device=device).manual_seed(seed)
    B, T, H, HK, K, V = c["B"], c["T"], c["H"], c["HK"], c["K"], c["V"]
    k = torch.nn.functional.normalize(torch.randn(B, T, HK, K, device=device, generator=g0), dim=-1).to(torch.bfloat16)
    v = torch.randn(B, T, H, V, device=device, generator=g0).to(torch.bfloat16)
    beta = torch.rand(B, T, H, device=device, generator=g0).clamp(1e-6, 1 - 1e-6).to(torch.bfloat16)
    g = -torch.rand(B, T, H, device=device, generator=g0)
    return k, v, beta, g


def cpu_wy_rate(c, k, v, beta, g, budget_s):
    """The WY oracle (numpy) on the first chunks of batch row 0, all heads,
    scaled to the whole job."""
    from oracle import gdr_stages as G

    def timed(nc):
        T = 64 * nc
        a = [t[:1, :T].float().cpu().numpy() for t in (k, v, beta, g)]
        t0 = time.perf_counter()
        G.wy(*a)
        return time.perf_counter() - t0

    t1 = timed(1)
    NT = (c["T"] + 63) // 64
    nc = int(max(1, min(NT, budget_s / max(t1, 1e-4))))
    dt = timed(nc)
    rate = c["B"] * c["T"] * (nc / dt) / (c["B"] * NT)
    threads = int(os.environ.get("OMP_NUM_THREADS", "0") or 0) or len(os.sched_getaffinity(0))
    desc = f"{nc} of {c['B'] * NT} (batch row, chunk) tiles, all {c['H']} heads ({dt:.2f} s), scaled to the whole job"
    return rate, desc, threads


def main_stage(args) -> int:
    """--op wy: the WY representation that produces fwd_h's w, u and
    cumulative gate, on the fixed-length configurations."""
    import torch
    import cann_operator_challenge_august_b200 as cg

    world, rank, local = dist_setup()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    c = shard(CONFIGS[args.config], world, rank)
    if "seqs" in c or c["K"] > 128 or c["V"] > 128:
        raise SystemExit("--op wy runs the fixed-length configurations with K, V <= 128")
    k, v, beta, g = gen_wy_inputs(c, 3000 + rank, dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        return cg.chunk_wy_fwd(k, v, beta, g)

    for _ in range(args.warmup):
        out = step()
    torch.cuda.synchronize()
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    clocks = ClockSampler(uuid)
    clocks.start()
    time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps)]
    t_start = torch.cuda.Event(enable_timing=True)
    t_stop = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(args.steps):
        ev[2 * i].record(stream)
        out = step()
        ev[2 * i + 1].record(stream)
    t_stop.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    elapsed_ms = max_over_ranks(t_start.elapsed_time(t_stop), world)
    per_launch_ms = max_over_ranks(sum(ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(args.steps)) / args.steps,
                                   world)
    ms_per_step = elapsed_ms / args.steps
    tokens_per_step = c["B"] * c["T"] * world
    value = tokens_per_step / (ms_per_step / 1000.0)

    host = [t.cpu().pin_memory() for t in (k, v, beta, g)]
    h2d = sum(t.numel() * t.element_size() for t in host)
    host_out = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in out]
    d2h = sum(t.numel() * t.element_size() for t in host_out)

    def e2e_step():
        d = [t.to(dev, non_blocking=True) for t in host]
        for dst, src in zip(host_out, cg.chunk_wy_fwd(*d)):
            dst.copy_(src, non_blocking=True)

    e2e_ms = e2e_value = None
    if args.e2e_steps > 0:
        e2e_step()
        torch.cuda.synchronize()
        barrier(world)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.e2e_steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1), world) / args.e2e_steps
        e2e_value = tokens_per_step / (e2e_ms / 1000.0)

    nbytes = wy_bytes(c)
    peak, peak_kind = load_peaks()
    achieved = nbytes / (per_launch_ms / 1000.0) / 1e9
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, desc, threads = cpu_wy_rate(c, k, v, beta, g, 10.0)
        cpu = {"value": rate, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": desc}
    if rank == 0:
        line = {
            "metric": "wy tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": c["scaling"], "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded, generated on device per rank, the reference operator's input ranges)",
            "config": dict(config_block(args.config, c, world, nbytes),
                           workload=f"{args.config}: WY representation bf16 B={c['B']} T={c['T']} H={c['H']} "
                                    f"K={c['K']} V={c['V']} chunk=64 (k, v, beta, g in; w, u, g_c out)"),
            "gpu_launches": args.steps,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                         else "fallback",
                         "algorithmic_bytes_per_launch": nbytes, "launch_ms": per_launch_ms,
                         "traffic": load_traffic(args.config, "wy"), "kernel": "wy"},
            "clocks": clk,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms},
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def gdr_bytes(c):
    """Operator-level bytes of one chunked Gated DeltaNet forward: query, key,
    value, beta, g and the initial state read once; out and the final state
    written once (a fully fused kernel's traffic)."""
    B, T, H, HK, K, V = c["B"], c["T"], c["H"], c["HK"], c["K"], c["V"]
    tot = B * T
    return tot * (2 * HK * K * 2 + H * V * 2 + H * 2 + H * 4 + H * V * 2) + 2 * B * H * K * V * 4


def main_gdr(args) -> int:
    """--op gdr: the whole chunked Gated DeltaNet forward (WY, recurrence,
    chunk output) through the reference operator's call, on B sequences of T
    tokens packed as one TND batch (actual_seq_lengths = [T] * B)."""
    import torch
    import cann_operator_challenge_august_b200 as cg

    world, rank, local = dist_setup()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    c = shard(CONFIGS[args.config], world, rank)
    if "seqs" in c or c["K"] > 128 or c["V"] > 128:
        raise SystemExit("--op gdr runs the fixed-length configurations with K, V <= 128")
    B, T, H, HK, K, V = c["B"], c["T"], c["H"], c["HK"], c["K"], c["V"]
    g0 = torch.Generator(device=dev).manual_seed(4000 + rank)
    tot = B * T
    q = torch.nn.functional.normalize(torch.randn(tot, HK, K, device=dev, generator=g0), dim=-1).to(torch.bfloat16)
    k = torch.nn.functional.normalize(torch.randn(tot, HK, K, device=dev, generator=g0), dim=-1).to(torch.bfloat16)
    v = torch.randn(tot, H, V, device=dev, generator=g0).to(torch.bfloat16)
    beta = torch.rand(tot, H, device=dev, generator=g0).clamp(1e-6, 1 - 1e-6).to(torch.bfloat16)
    g = -torch.rand(tot, H, device=dev, generator=g0)
    h0 = 0.1 * torch.randn(B, H, V, K, device=dev, generator=g0)
    asl = torch.full((B,), T, dtype=torch.int32, device=dev)
    out = torch.empty_like(v)
    fin = torch.empty_like(h0)
    gpath = args.gdr_path
    op0 = cg.ChunkGatedDeltaRule(q, k, v, beta, h0, asl, g, None, out, fin, path=gpath)
    ws = torch.empty(op0.workspace_size, dtype=torch.uint8, device=dev)
    path_taken = op0.path
    del op0
    stream = torch.cuda.current_stream(dev)

    def step():
        cg.ChunkGatedDeltaRule(q, k, v, beta, h0, asl, g, None, out, fin, path=gpath)(ws)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    clocks = ClockSampler(uuid)
    clocks.start()
    time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps)]
    t_start = torch.cuda.Event(enable_timing=True)
    t_stop = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(args.steps):
        ev[2 * i].record(stream)
        step()
        ev[2 * i + 1].record(stream)
    t_stop.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    elapsed_ms = max_over_ranks(t_start.elapsed_time(t_stop), world)
    per_launch_ms = max_over_ranks(sum(ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(args.steps)) / args.steps,
                                   world)
    ms_per_step = elapsed_ms / args.steps
    tokens_per_step = tot * world
    value = tokens_per_step / (ms_per_step / 1000.0)

    host = [t.cpu().pin_memory() for t in (q, k, v, beta, h0, asl, g)]
    h2d = sum(t.numel() * t.element_size() for t in host)
    host_out = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in (out, fin)]
    d2h = sum(t.numel() * t.element_size() for t in host_out)

    def e2e_step():
        d = [t.to(dev, non_blocking=True) for t in host]
        o, f = cg.chunk_gated_delta_rule(d[0], d[1], d[2], d[3], d[4], d[5], None, d[6], workspace=ws, path=gpath)
        host_out[0].copy_(o, non_blocking=True)
        host_out[1].copy_(f, non_blocking=True)

    e2e_ms = e2e_value = None
    if args.e2e_steps > 0:
        e2e_step()
        torch.cuda.synchronize()
        barrier(world)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.e2e_steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1), world) / args.e2e_steps
        e2e_value = tokens_per_step / (e2e_ms / 1000.0)

    nbytes = gdr_bytes(c)
    peak, peak_kind = load_peaks()
    achieved = nbytes / (per_launch_ms / 1000.0) / 1e9
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import gdr_stages as G
        f = lambda t, n: t[:n].float().cpu().numpy()  # noqa: E731
        n1 = 64
        t0 = time.perf_counter()
        G.benchmark_op(f(q, n1), f(k, n1), f(v, n1), f(beta, n1), K ** -0.5, h0[:1].float().cpu().numpy(), [n1],
                       f(g, n1))
        t1 = time.perf_counter() - t0
        n = int(max(64, min(T, 64 * (10.0 / max(t1, 1e-4)) // 64 * 1)))
        n = min(T, max(64, (n // 64) * 64))
        t0 = time.perf_counter()
        G.benchmark_op(f(q, n), f(k, n), f(v, n), f(beta, n), K ** -0.5, h0[:1].float().cpu().numpy(), [n], f(g, n))
        dt = time.perf_counter() - t0
        rate = n / dt
        threads = int(os.environ.get("OMP_NUM_THREADS", "0") or 0) or len(os.sched_getaffinity(0))
        cpu = {"value": rate, "unit": "tokens/s", "cores": threads, "kind": "port",
               "sample": f"the restated reference bf16 operator on the first {n} tokens of sequence 0, all {H} heads "
                         f"({dt:.2f} s), as tokens/s"}
    if rank == 0:
        line = {
            "metric": "gdr tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": c["scaling"], "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded, generated on device per rank, the reference operator's input ranges)",
            "config": dict(config_block(args.config, c, world, nbytes),
                           workload=f"{args.config}: chunked Gated DeltaNet forward (WY, recurrence, chunk output) bf16, "
                                    f"{B} sequences of T={T} packed as TND, Nk={HK} Nv={H} Dk={K} Dv={V}, "
                                    f"fp32 initial/final state",
                           path=path_taken),
            # per call: metadata, WY, the recurrence's sequence order, then the fused kernel
            # or the recurrence and the chunk output
            "gpu_launches": (4 if path_taken == "fused" else 5) * args.steps,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                         else "fallback",
                         "algorithmic_bytes_per_launch": nbytes, "launch_ms": per_launch_ms,
                         "bytes_basis": "operator inputs and outputs only (intermediates between kernels are "
                                        "not counted)",
                         "traffic": None,
                         "kernel": "wy+fwd_ho" if path_taken == "fused" else "wy+fwd_h+chunk_o"},
            "clocks": clk,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms},
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
