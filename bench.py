#!/usr/bin/env python
"""bench.py -- canvas-attention throughput on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c3]
                    [--impl ours|reference]

A step is one pass of the attention hot path over one synthetic batch of the
named config: for every layer of the config, the fused block entry point
(QK RMSNorm -> RoPE -> K/V cache store -> attention, src/model/forward.rs:
296-343) through the C ABI. Inputs are resident in HBM when timing starts.

Configs (seeded N(0,1) bf16 inputs):
  c1  B1  S128   H32/32  hd128  theta 5e5
  c2  B4  S1024  H28/4   hd128  theta 1e6
  c3  B8  S4096  H16/16  hd128  theta 5e4, QK RMSNorm (eps 1e-6, gains U(0.5,1.5))
  c4  B16 32 active queries at positions 2048..2079 over a 4128-position
      cache (4096 cached + 32 active), H32/8 hd128; the cache is reused and
      each step brings fresh active Q/K/V
  c5  B4  S8192  H16/8 hd256, 6 layers: 5 sliding (window 512, theta 1e4) +
      1 global (theta 1e6), soft-cap 50 (extension), scale 1/16
Default workload: c3, the 4k-token bidirectional case the north-star target
names. Multi-GPU is weak scaling: every rank runs its own full batch of the
config (sequences are independent, so no collective is on the data path).
Under torchrun the line also carries `head_sharded`: the same global batch
split by kv heads over the ranks plus one NCCL all-gather per layer of the
head slices (strong scaling, compute only and with the gather).

Metric: TFLOP/s = 4 * head_dim * visible (query, key) pairs * n_head summed
over the batch and layers, divided by time (softmax, RoPE and norms excluded).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "diffuse-rs_b200"))
sys.path.insert(0, ROOT)

L2_BYTES = 126 * 1024 * 1024

CONFIGS = {
    "c1": dict(B=1, na=128, n_total=128, start=0, H=32, Hkv=32, hd=128, qk_norm=False,
               layers=[(None, 5e5)], softcap=0.0, scale=128 ** -0.5,
               desc="LLaDA-8B single layer, B1 S128 H32/32 hd128"),
    "c2": dict(B=4, na=1024, n_total=1024, start=0, H=28, Hkv=4, hd=128, qk_norm=False,
               layers=[(None, 1e6)], softcap=0.0, scale=128 ** -0.5,
               desc="Dream-7B GQA, B4 S1024 H28/4 hd128"),
    "c3": dict(B=8, na=4096, n_total=4096, start=0, H=16, Hkv=16, hd=128, qk_norm=True,
               layers=[(None, 5e4)], softcap=0.0, scale=128 ** -0.5,
               desc="LLaDA-MoE + QK RMSNorm, B8 S4096 H16/16 hd128"),
    "c4": dict(B=16, na=32, n_total=4128, start=2048, H=32, Hkv=8, hd=128, qk_norm=False,
               layers=[(None, 5e5)], softcap=0.0, scale=128 ** -0.5,
               desc="KV-cache block decode, B16 x 32 queries over 4128 keys, H32/8 hd128"),
    "c5": dict(B=4, na=8192, n_total=8192, start=0, H=16, Hkv=8, hd=256, qk_norm=True,
               layers=[(512, 1e4)] * 5 + [(None, 1e6)], softcap=50.0, scale=256 ** -0.5,
               desc="DiffusionGemma hybrid, B4 S8192 H16/8 hd256, 5 sliding(512)+1 global"),
}


def visible_pairs(na, n_total, start, window):
    """Visible (query, key) pairs of one sequence: queries at positions
    start..start+na-1, keys at 0..n_total-1, visible iff |dq - dk| < window."""
    if window is None:
        return na * n_total
    tot = 0
    for qp in range(start, start + na):
        lo = max(0, qp - window + 1)
        hi = min(n_total - 1, qp + window - 1)
        tot += hi - lo + 1
    return tot


def layer_flops(cfg, window):
    return 4.0 * cfg["hd"] * cfg["H"] * cfg["B"] * visible_pairs(
        cfg["na"], cfg["n_total"], cfg["start"], window)


def step_flops(cfg):
    return sum(layer_flops(cfg, w) for w, _ in cfg["layers"])


def layer_bytes(cfg):
    """Algorithmic HBM bytes of one attention launch: Q read once, K and V read
    once per kv head (the whole cache for c4), O written once, all bf16."""
    B, H, Hkv, hd = cfg["B"], cfg["H"], cfg["Hkv"], cfg["hd"]
    return 2 * B * hd * (2 * cfg["na"] * H + 2 * cfg["n_total"] * Hkv)


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return dict(hbm=d["hbm_gbs"], tflops=d["bf16_tflops"],
                    tflops_sustained=d["bf16_tflops_sustained"], source="measured")
    return dict(hbm=6650.0, tflops=1590.0, tflops_sustained=1400.0, source="fallback")


def load_traffic(config):
    """Per-launch DRAM bytes of the attention kernel from a committed ncu
    summary (profiles/attn_fwd_dram_traffic.txt: '<config> <bytes>' lines)."""
    p = os.path.join(ROOT, "profiles", "attn_fwd_dram_traffic.txt")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        for line in f:
            parts = line.split()
            if len(parts) == 2 and parts[0] == config:
                return float(parts[1])
    return None


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu_index = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        import tempfile
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu_index), "-lms", "50"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.path is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        loaded = [s for s in sm if mx and s > 0.5 * max(mx)] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


class Workload:
    """Device tensors for one rank's batch of one config.

    heads=(q0, q1, kv0, kv1) keeps only that head range of a global batch
    generated from the same seed on every rank (the head-sharded form)."""

    def __init__(self, cfg, device, seed, heads=None):
        import torch
        import canvas_attn as ca
        self.ca, self.torch, self.cfg = ca, torch, cfg
        B, na, nt, H, Hkv, hd = (cfg[k] for k in ("B", "na", "n_total", "H", "Hkv", "hd"))
        g = torch.Generator(device=device).manual_seed(seed)
        bf = torch.bfloat16
        q0, q1, kv0, kv1 = heads if heads is not None else (0, H, 0, Hkv)
        self.H, self.Hkv = q1 - q0, kv1 - kv0

        def rnd(*shape, sl=None):
            t = torch.randn(*shape, generator=g, device=device, dtype=torch.float32).to(bf)
            if sl is None or (sl[0] == 0 and sl[1] == shape[2]):
                return t
            return t[:, :, sl[0]:sl[1]].contiguous()

        qs, kvs = (q0, q1), (kv0, kv1)
        self.n_sets = 2  # fresh active Q/K/V alternate between steps
        self.layers = []
        for (window, theta) in cfg["layers"]:
            rope = torch.from_numpy(ca.build_rope_cache(max(4096, nt), hd, theta)).to(device)
            L = dict(window=window, rope=rope, rope_len=max(4096, nt),
                     q=[rnd(B, na, H, hd, sl=qs) for _ in range(self.n_sets)],
                     k=[rnd(B, na, Hkv, hd, sl=kvs) for _ in range(self.n_sets)],
                     v=[rnd(B, na, Hkv, hd, sl=kvs) for _ in range(self.n_sets)],
                     cache_k=rnd(B, nt, Hkv, hd, sl=kvs), cache_v=rnd(B, nt, Hkv, hd, sl=kvs),
                     # Rotated Q for the attention-only timing; the fused
                     # block (head_dim 128, small grids) leaves it unwritten.
                     q_work=rnd(B, na, H, hd, sl=qs),
                     out=torch.empty(B, na, self.H, hd, dtype=bf, device=device))
            if cfg["qk_norm"]:
                L["wq"] = torch.rand(hd, generator=g, device=device) + 0.5
                L["wk"] = torch.rand(hd, generator=g, device=device) + 0.5
            self.layers.append(L)
        pos = torch.arange(cfg["start"], cfg["start"] + na, dtype=torch.int32, device=device)
        self.pos = pos.repeat(B, 1).contiguous()
        self.stream = torch.cuda.current_stream(device)

    def block_args(self, L, i, b0=0, b1=None):
        """Block arguments for sequences b0..b1-1 of input set i."""
        c = self.cfg
        b1 = c["B"] if b1 is None else b1
        sl = slice(b0, b1)
        return self.ca.make_block_args(
            L["q"][i][sl], L["k"][i][sl], L["v"][i][sl], batch=b1 - b0, n_active=c["na"],
            active_pos=self.pos[sl], rope=L["rope"], rope_len=L["rope_len"],
            rope_dim=c["hd"], cache_k=L["cache_k"][sl], cache_v=L["cache_v"][sl],
            n_total=c["n_total"], q_work=L["q_work"][sl], out=L["out"][sl], n_head=self.H,
            n_head_kv=self.Hkv, head_dim=c["hd"], q_norm_w=L.get("wq"),
            k_norm_w=L.get("wk"), rms_eps=1e-6, sliding_window=L["window"],
            scale=c["scale"], softcap=c["softcap"])

    def block(self, L, i, b0=0, b1=None, stream=None):
        import ctypes
        a = self.block_args(L, i % self.n_sets, b0, b1)
        sp = (stream or self.stream).cuda_stream
        rc = self.ca.lib.ca_attention_block_dev(ctypes.byref(a), sp)
        if rc != 0:
            raise self.ca.CaError(rc, "ca_attention_block_dev")

    def step(self, i):
        for L in self.layers:
            self.block(L, i)

    launches_per_step = property(lambda self: 2 * len(self.layers))

    def attn_args(self, L):
        c = self.cfg
        return self.ca.make_dev_args(
            L["q_work"], L["cache_k"], L["cache_v"], L["out"], batch=c["B"], sq=c["na"],
            sk=c["n_total"], n_head=self.H, n_head_kv=self.Hkv, head_dim=c["hd"],
            q_pos=self.pos, sliding_window=L["window"], scale=c["scale"],
            softcap=c["softcap"])

    def attn_only(self, L):
        import ctypes
        a = self.attn_args(L)
        rc = self.ca.lib.ca_attention_dev(ctypes.byref(a), self.stream.cuda_stream)
        if rc != 0:
            raise self.ca.CaError(rc, "ca_attention_dev")

    def input_bytes(self):
        return sum(t.numel() * t.element_size() for L in self.layers
                   for t in (L["q"][0], L["k"][0], L["v"][0], L["cache_k"], L["cache_v"]))


class CpuSample:
    """A bounded sample of one config's (head, query) rows for the CPU
    restatement of the reference's rayon/AVX2 attention (oracle/, the
    reference's own Rust cannot be built here). Rows are exact: each row's
    output is independent of the others, so a subset times the same code."""

    def __init__(self, cfg, seed=0):
        import numpy as np
        from oracle import oracle as orc
        self.np, self.orc, self.cfg = np, orc, cfg
        rng = np.random.default_rng(seed)
        c = cfg
        nk = c["n_total"]

        def rnd(n):
            return rng.standard_normal(n, dtype=np.float32)

        self.q = rnd(c["na"] * c["H"] * c["hd"])
        self.k = rnd(nk * c["Hkv"] * c["hd"])
        self.v = rnd(nk * c["Hkv"] * c["hd"])
        self.q_pos = np.arange(c["start"], c["start"] + c["na"], dtype=np.int64)
        self.k_pos = np.arange(nk, dtype=np.int64)
        # All host threads, whatever OMP_NUM_THREADS a launcher (torchrun
        # sets 1) put in the environment.
        try:
            self.threads = len(os.sched_getaffinity(0))
        except AttributeError:
            self.threads = os.cpu_count() or orc.max_threads()
        self.kind = orc.ROW_AVX2 if orc.have_avx2() else orc.ROW_SCALAR
        self.out = np.zeros(c["na"] * c["H"] * c["hd"], dtype=np.float32)

    def row_visible(self, qpos, window):
        if window is None:
            return self.cfg["n_total"]
        return min(self.cfg["n_total"] - 1, qpos + window - 1) - max(0, qpos - window + 1) + 1

    def run(self, n_rows):
        """Runs about n_rows rows spread over every layer, repeating whole
        layers when n_rows exceeds them; returns (flops, seconds, rows run)."""
        np, c = self.np, self.cfg
        n_tasks = c["H"] * c["na"]
        per_layer = max(1, n_rows // len(c["layers"]))
        reps = max(1, per_layer // n_tasks)
        flops, secs, rows = 0.0, 0.0, 0
        for window, _theta in c["layers"]:
            tasks = np.unique(np.linspace(0, n_tasks - 1, min(per_layer, n_tasks)).astype(np.int64))
            qrows = tasks % c["na"]
            flops += reps * 4.0 * c["hd"] * sum(self.row_visible(int(self.q_pos[r]), window)
                                                for r in qrows)
            rows += reps * len(tasks)
            t0 = time.perf_counter()
            for _ in range(reps):
                self.orc.attention(self.q, self.k, self.v, nq=c["na"], nk=c["n_total"],
                                   n_head=c["H"], n_head_kv=c["Hkv"], head_dim=c["hd"],
                                   q_pos=self.q_pos, k_pos=self.k_pos, sliding_window=window,
                                   scale=c["scale"], softcap=c["softcap"], kind=self.kind,
                                   threads=self.threads, tasks=tasks, out=self.out)
            secs += time.perf_counter() - t0
        return flops, secs, rows

    def calibrate(self, target_s):
        """Row count whose run takes about target_s seconds."""
        n = 64 * len(self.cfg["layers"])
        self.run(n)  # thread-pool start-up
        for _ in range(6):  # grow the probe until it takes ~1/4 of the target
            _f, s, rows = self.run(n)
            if s > min(0.5, target_s / 4):
                break
            n = int(rows * min(16.0, 0.6 / max(s, 1e-4)))
        return max(16, int(rows / max(s, 1e-6) * target_s))

    def describe(self, rows, config):
        return (f"{rows} (head, query) rows of the {config} config (one sequence, repeated "
                f"when the sample exceeds it) over {len(self.cfg['layers'])} layer(s), "
                f"{self.cfg['n_total']} keys each")


def cpu_baseline(cfg, config, seconds, repeats=3):
    """The oracle's AVX2 row kernel on all host threads: one fixed row sample
    (sized for about seconds / repeats), run `repeats` times; the median rate
    with the spread of the repeats."""
    cs = CpuSample(cfg)
    n_rows = cs.calibrate(seconds / repeats)
    rates, secs, rows = [], 0.0, 0
    for _ in range(repeats):
        f, s, rows = cs.run(n_rows)
        rates.append(f / s / 1e12)
        secs += s
    return dict(value=statistics.median(rates), unit="TFLOP/s", cores=cs.threads, kind="port",
                spread=[round(min(rates), 5), round(max(rates), 5)], repeats=repeats,
                sample=cs.describe(rows, config) + f", median of {repeats} repeats, "
                f"{secs:.1f} s in all")


class E2E:
    """The reference-facing call with HOST buffers: ca_attention_host_f32,
    i.e. attention(out, q, k, v, s, qr, kr) (src/model/attention.rs:106) on
    pinned fp32 host arrays, once per sequence and layer as the reference calls
    it. Host->device copies of Q/K/V and the device->host copy of out happen
    inside each call."""

    def __init__(self, cfg, seed=0):
        import numpy as np
        import torch
        import canvas_attn as ca
        self.ca, self.cfg = ca, cfg
        c = cfg
        g = torch.Generator().manual_seed(seed)

        def pinned(n):
            t = torch.randn(n, generator=g, dtype=torch.float32).pin_memory()
            return t, t.numpy()

        nk = c["n_total"]
        self._keep = []
        for name, n in (("q", c["na"] * c["H"] * c["hd"]), ("k", nk * c["Hkv"] * c["hd"]),
                        ("v", nk * c["Hkv"] * c["hd"]), ("out", c["na"] * c["H"] * c["hd"])):
            t, a = pinned(n)
            self._keep.append(t)
            setattr(self, name, a)
        # Key rows in the reference's cached order [cached asc | active asc]
        # (src/model/forward.rs:92-96); without a cache, keys = queries' positions.
        act = np.arange(c["start"], c["start"] + c["na"])
        if nk > c["na"]:
            cached = np.setdiff1d(np.arange(nk), act)
            self.k_pos = np.concatenate([cached, act])
        else:
            self.k_pos = act
        self.q_pos = act
        self.calls = len(c["layers"]) * c["B"]
        self.h2d = self.calls * 4 * (self.q.size + self.k.size + self.v.size)
        self.d2h = self.calls * 4 * self.out.size
        # Calls of at least 4 MiB of bf16 operands (or 16 MiB of fp32 Q, the
        # pipelined form), head_dim a multiple of 8, round Q/K/V to bf16 on
        # host threads before the copies (CA_HOST_ROUND=0 turns that off):
        # half the bytes cross PCIe.
        big = (self.q.size * 4 >= (16 << 20) or
               (self.q.size + self.k.size + self.v.size) * 2 >= (4 << 20))
        rounded = big and c["hd"] % 8 == 0 and nk > 0
        hround = os.environ.get("CA_HOST_ROUND", "1") != "0"
        self.pcie_h2d = self.h2d // 2 if rounded and hround else self.h2d

    def step(self):
        c = self.cfg
        for window, _theta in c["layers"]:
            s = self.ca.AttnShape(c["na"], c["n_total"], c["H"], c["Hkv"], c["hd"], window,
                                  None, c["scale"], c["softcap"])
            qr, kr = self.ca.Rows(self.q_pos), self.ca.Rows(self.k_pos)
            for _b in range(c["B"]):
                self.ca.attention(self.out, self.q, self.k, self.v, s, qr, kr)


def dist_setup(want_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(local)
        # NCCL prints a version banner on stdout while the communicator is
        # created (eagerly here, device_id given); keep stdout for the one
        # JSON line by pointing file descriptor 1 at stderr meanwhile.
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", device_id=torch.device("cuda", local))
            dist.barrier()
            torch.cuda.synchronize()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
    if want_gpus != world and rank == 0:
        print(f"note: --gpus {want_gpus} but WORLD_SIZE {world}; using {world}", file=sys.stderr)
    return world, rank, local


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def physical_gpu_index(local):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [x.strip() for x in vis.split(",") if x.strip()]
        if local < len(ids) and ids[local].isdigit():
            return int(ids[local])
    return local


def input_bytes_of(cfg):
    """Bytes of one step's inputs on one rank (Q/K/V of every layer plus the
    K/V cache), bf16; equals Workload.input_bytes()."""
    B, na, nt, H, Hkv, hd = (cfg[k] for k in ("B", "na", "n_total", "H", "Hkv", "hd"))
    return len(cfg["layers"]) * 2 * B * hd * (na * H + 2 * na * Hkv + 2 * nt * Hkv)


def config_dict(args, cfg, world):
    """The workload description both arms print (same keys and values)."""
    flush = input_bytes_of(cfg) < 2 * L2_BYTES
    return {"workload": args.config, "desc": cfg["desc"], "batch_per_gpu": cfg["B"],
            "global_batch": cfg["B"] * world, "seq_q": cfg["na"], "seq_k": cfg["n_total"],
            "layers": len(cfg["layers"]),
            "l2": "flushed between steps (working set < 2x L2)" if flush
            else "inputs larger than L2, no flush",
            "parallelism": f"dp{world} (independent sequences per rank)",
            **({"only_layer": args.only_layer} if args.only_layer is not None else {})}


def kernel_ms(wl, flush, scratch, reps):
    """Average device time (CUDA events on the launching stream) of the
    attention kernel alone, per layer, on the workload's prepared tensors."""
    import torch
    out = []
    for L in wl.layers:
        wl.attn_only(L)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(reps)]
        torch.cuda.synchronize()
        for a, b in ev:
            if flush:
                scratch.zero_()
            a.record(wl.stream)
            wl.attn_only(L)
            b.record(wl.stream)
        torch.cuda.synchronize()
        out.append(sum(a.elapsed_time(b) for a, b in ev) / reps)
    return out


def roofline(name, cfg, layers, ms, peaks, traffic_key=None):
    """Roofline of the attention kernel over `layers` of a config taking `ms`:
    c4 against HBM copy bandwidth (algorithmic bytes), the others against the
    burst bf16 tensor peak (algorithmic flops)."""
    if name == "c4":
        achieved = len(layers) * layer_bytes(cfg) / (ms * 1e-3) / 1e9
        r = dict(bound="hbm", achieved=round(achieved, 1), peak=peaks["hbm"], unit="GB/s",
                 peak_source=peaks["source"] + " copy")
    else:
        fl = sum(layer_flops(cfg, w) for w, _ in layers)
        r = dict(bound="tensor", achieved=round(fl / (ms * 1e-3) / 1e12, 1),
                 peak=peaks["tflops"], unit="TFLOP/s", peak_source=peaks["source"] + " burst")
    r["frac"] = round(r["achieved"] / r["peak"], 4)
    r["traffic"] = load_traffic(traffic_key or name)
    r["kernel_ms"] = round(ms, 4)
    return r


def _event_ms(fn, reps, flush=None):
    """Average device time of fn() over reps calls (CUDA events, current stream)."""
    import torch
    fn()
    torch.cuda.synchronize()
    tot = 0.0
    for _ in range(reps):
        if flush is not None:
            flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        tot += a.elapsed_time(b)
    return tot / reps


def run_extras(dev, peaks, scratch):
    """Kernel-alone rooflines of the projection and sampler rows (synthetic
    seeded data): Q4_K dequantisation of a 12288 x 4096 QKV weight
    (LLaDA-8B: n_embd 4096, Q, K and V of 32 heads x 128 each), the bf16 QKV GEMM of
    4096 tokens through it, and candidate statistics of 256 masked rows of a
    126464-entry vocabulary (LLaDA's)."""
    import numpy as np
    import torch
    from canvas_attn import denoise as dn
    from canvas_attn import projection as pj
    if scratch is None:
        scratch = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)
    out = {}
    rng = np.random.default_rng(11)
    rows, cols, n = 12288, 4096, 4096
    rb = pj.row_bytes(pj.Q4_K, cols)
    wq = rng.integers(0, 256, (rows, rb), dtype=np.uint8)
    blk = wq.reshape(-1, 144)
    blk[:, 0:2] = np.array([0.01], np.float16).view(np.uint8)  # moderate d / dmin in every block
    blk[:, 2:4] = np.array([0.005], np.float16).view(np.uint8)
    src = torch.from_numpy(wq).to(dev)
    w = torch.empty(rows, cols, dtype=torch.bfloat16, device=dev)
    ms = _event_ms(lambda: pj.dequantize(pj.Q4_K, src, rows, cols, w), 20, scratch)
    byt = rows * rb + rows * cols * 2
    out["dequant_q4k"] = dict(bound="hbm", achieved=round(byt / (ms * 1e-3) / 1e9, 1),
                              peak=peaks["hbm"], unit="GB/s", kernel_ms=round(ms, 4),
                              shape=f"{rows}x{cols} Q4_K -> bf16",
                              frac=round(byt / (ms * 1e-3) / 1e9 / peaks["hbm"], 4))
    act = torch.randn(n, cols, device=dev).to(torch.bfloat16)
    bias = torch.randn(rows, device=dev)
    o = torch.empty(n, rows, device=dev)
    ms = _event_ms(lambda: pj.linear(act, w, o, n=n, rows=rows, cols=cols, bias=bias), 20)
    tf = 2.0 * n * rows * cols / (ms * 1e-3) / 1e12
    out["linear_qkv"] = dict(bound="tensor", achieved=round(tf, 1), peak=peaks["tflops"],
                             unit="TFLOP/s", kernel_ms=round(ms, 4), frac=round(tf / peaks["tflops"], 4),
                             shape=f"[{n}, {cols}] x [{rows}, {cols}]^T + bias, fp32 out",
                             gemm="cuBLASLt (library GEMM)")
    del src, w, act, o
    n_cand, vocab = 256, 126464
    logits = torch.randn(n_cand + 8, vocab, device=dev) * 4
    rows_t = torch.arange(n_cand, dtype=torch.int32, device=dev)
    tok = torch.empty(n_cand, dtype=torch.int32, device=dev)
    vals = torch.empty(3, n_cand, device=dev)
    ms = _event_ms(lambda: dn.candidate_stats(logits, rows_t, tok, vals[0], vals[1], vals[2],
                                              n_vocab=vocab, mask_id=vocab - 1,
                                              want_entropy=True, want_prob=True), 20, scratch)
    byt = n_cand * vocab * 4
    out["candidate_stats"] = dict(bound="hbm", achieved=round(byt / (ms * 1e-3) / 1e9, 1),
                                  peak=peaks["hbm"], unit="GB/s", kernel_ms=round(ms, 4),
                                  frac=round(byt / (ms * 1e-3) / 1e9 / peaks["hbm"], 4),
                                  shape=f"{n_cand} rows x {vocab} fp32 logits (entropy + prob)")
    del logits
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return out


def run_head_sharded(args, cfg, world, rank, dev):
    """Head-sharded strong scaling of ONE global batch of the config: rank r
    computes kv heads [r * Hkv / N, (r + 1) * Hkv / N) and their query heads
    of every sequence, and the head slices are reassembled into full
    [tokens, n_head, head_dim] rows on every rank, the layout o_proj consumes
    (src/model/forward.rs:345). Three forms are timed:

    peer       the attention epilogue stores each finished tile into every
               rank's receive buffer over NVLink (CUDA IPC mappings,
               canvas_attn.sharding.PeerRows); one stream-ordered 4-byte
               all_reduce per step is the barrier after which all rows are
               in place.
    multicast  the same, but the epilogue writes each row once through an
               NVLS multicast address bound to every rank's buffer
               (MulticastRows; multimem stores), so a row crosses this GPU's
               NVLink once instead of once per peer. `value` is the faster
               of peer and multicast (`form` names it).
    nccl  per layer and chunk of sequences, one NCCL all_gather_into_tensor
          on a second stream overlapped with the next chunk's compute, then a
          copy into head order.

    Every rank generates the same global inputs from one seed; rank 0 then
    recomputes the whole batch on its own GPU and compares every form's
    gathered rows with it."""
    import torch
    import torch.distributed as dist
    from canvas_attn.sharding import MulticastRows, PeerRows, head_shard
    sh = head_shard(cfg["H"], cfg["Hkv"], world, rank)
    wl = Workload(cfg, dev, seed=4321, heads=(sh.q_begin, sh.q_end, sh.kv_begin, sh.kv_end))
    B, na, H, hd = cfg["B"], cfg["na"], cfg["H"], cfg["hd"]
    lh = wl.H
    tok = B * na
    ca = wl.ca

    # --- peer form
    recv = [PeerRows(tok, H, hd) for _ in wl.layers]
    flag = torch.zeros(1, dtype=torch.int32, device=dev)

    def step_peer(i):
        import ctypes
        for L, R in zip(wl.layers, recv):
            out, peers, ors = R.slice_args(sh)
            a = wl.block_args(L, i % wl.n_sets)
            a.out = out.data_ptr()
            a.out_row_stride = ors
            arr = (ctypes.c_void_p * len(peers))(*peers)
            a.peer_out = ctypes.cast(arr, ctypes.c_void_p)
            a.n_peer_out = len(peers)
            rc = ca.lib.ca_attention_block_dev(ctypes.byref(a), wl.stream.cuda_stream)
            if rc != 0:
                raise ca.CaError(rc, "ca_attention_block_dev (peer rows)")
        dist.all_reduce(flag)  # every rank's stores are in place after this

    # --- multicast form (NVLS): each row crosses this GPU's NVLink once
    mrecv = [MulticastRows(tok, H, hd) for _ in wl.layers]
    avail = [None] * world
    dist.all_gather_object(avail, (all(R.available for R in mrecv),
                                   next((R.why for R in mrecv if not R.available), "")))
    mc_ok = all(a for a, _ in avail)
    mc_why = next((w for a, w in avail if not a), "")

    def step_mc(i):
        import ctypes
        for L, R in zip(wl.layers, mrecv):
            out, mc, ors = R.slice_args(sh)
            a = wl.block_args(L, i % wl.n_sets)
            a.out = out.data_ptr()
            a.out_row_stride = ors
            a.out_multicast = mc
            rc = ca.lib.ca_attention_block_dev(ctypes.byref(a), wl.stream.cuda_stream)
            if rc != 0:
                raise ca.CaError(rc, "ca_attention_block_dev (multicast rows)")
        mrecv[0].barrier(wl.stream)  # every rank's multicast stores are in place after this

    # --- NCCL form
    n_chunks = max(1, min(args.hs_chunks, B))
    while B % n_chunks:
        n_chunks -= 1
    bc = B // n_chunks
    tok_c = bc * na
    comm = torch.cuda.Stream(dev)
    stage = torch.empty((n_chunks, world, tok_c, lh, hd), dtype=torch.bfloat16, device=dev)
    full = [torch.empty((tok, H, hd), dtype=torch.bfloat16, device=dev) for _ in wl.layers]
    done = [torch.cuda.Event() for _ in range(n_chunks)]

    def step_nccl(i, gather=True):
        for li, L in enumerate(wl.layers):
            for c in range(n_chunks):
                wl.block(L, i, c * bc, (c + 1) * bc)
                if not gather:
                    continue
                done[c].record(wl.stream)
                comm.wait_event(done[c])
                with torch.cuda.stream(comm):
                    src = L["out"][c * bc:(c + 1) * bc].view(-1)
                    dist.all_gather_into_tensor(stage[c].view(-1), src)
                    # [world, tok_c, lh, hd] -> rows of [tokens, H, hd]
                    full[li][c * tok_c:(c + 1) * tok_c].view(tok_c, world, lh, hd).copy_(
                        stage[c].permute(1, 0, 2, 3))
        if gather:
            fin = torch.cuda.Event()
            fin.record(comm)
            wl.stream.wait_event(fin)

    def timed(fn):
        for i in range(args.warmup):
            fn(i)
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
        barrier(world)
        torch.cuda.synchronize()
        for i in range(args.steps):
            ev[i][0].record(wl.stream)
            fn(i)
            ev[i][1].record(wl.stream)
        torch.cuda.synchronize()
        barrier(world)
        return max_over_ranks(sum(a.elapsed_time(b) for a, b in ev), world)

    comp = timed(wl.step)  # the peer form's launches (whole batch per layer), no gather
    t_peer = timed(step_peer)
    t_mc = timed(step_mc) if mc_ok else None
    t_nccl = timed(step_nccl)
    status = ca.device_status(wl.stream.cuda_stream)
    assert status == 0, f"device-side status {status}"

    # NCCL all-gather of the whole output payload alone (bus bandwidth).
    payload = torch.empty(tok * lh * hd, dtype=torch.bfloat16, device=dev)
    gbuf = torch.empty(world * payload.numel(), dtype=torch.bfloat16, device=dev)
    for _ in range(3):
        dist.all_gather_into_tensor(gbuf, payload)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(10):
        dist.all_gather_into_tensor(gbuf, payload)
    e1.record()
    torch.cuda.synchronize()
    ag_ms = max_over_ranks(e0.elapsed_time(e1) / 10, world)
    ag_bytes = gbuf.numel() * 2
    del payload, gbuf

    last = (args.steps - 1) % wl.n_sets
    parity = None
    if rank == 0:
        ref = Workload(cfg, dev, seed=4321)
        for L in ref.layers:
            ref.block(L, last)
        torch.cuda.synchronize()
        res = {}
        forms = [("peer", [R.buf for R in recv]), ("nccl", full)]
        if mc_ok:
            forms.append(("multicast", [R.buf for R in mrecv]))
        for form, bufs in forms:
            worst, exact = 0.0, True
            for li, L in enumerate(ref.layers):
                want = L["out"].view(tok, H, hd)
                exact = exact and torch.equal(bufs[li], want)
                worst = max(worst, (bufs[li].float() - want.float()).abs().max().item())
            res[form] = dict(max_abs_diff=worst, bit_identical=exact)
        parity = dict(res, rows_checked=tok * H,
                      against="all heads of the same global batch run on one GPU")
        del ref
        torch.cuda.synchronize()
    barrier(world)
    for R in recv:
        R.close()
    # Other ranks' multicast buffers were checked by the test suite; here
    # rank 0's copy stands for all (the same stores reach every rank).
    flops = step_flops(cfg) * args.steps
    tf = lambda ms: round(flops / (ms * 1e-3) / 1e12, 2)  # noqa: E731
    mc_line = (dict(value=tf(t_mc), ms_per_step=round(t_mc / args.steps, 4),
                    gather="attention epilogue writes each row once through an NVLS "
                           "multicast address (multimem.st); the switch delivers it to "
                           "every rank's buffer",
                    barrier="symmetric-memory signal-pad barrier on the stream")
               if mc_ok else dict(unavailable=mc_why))
    best = min(t for t in (t_peer, t_mc) if t is not None)
    return dict(value=tf(best), unit="TFLOP/s", compute_only=tf(comp),
                form="multicast" if best == t_mc else "peer",
                ms_per_step=round(best / args.steps, 4),
                peer=dict(value=tf(t_peer), ms_per_step=round(t_peer / args.steps, 4),
                          gather="attention epilogue stores its tiles into every rank's "
                                 "receive buffer over NVLink (CUDA IPC peer mappings)"),
                multicast=mc_line,
                barrier="peer and NCCL forms: one stream-ordered 4-byte all_reduce per step",
                compute_ms_per_step=round(comp / args.steps, 4),
                nccl=dict(value=tf(t_nccl), ms_per_step=round(t_nccl / args.steps, 4),
                          chunks=n_chunks,
                          collective="per layer and chunk of sequences, one NCCL "
                                     "all_gather_into_tensor on a second stream, then a "
                                     "copy into head order"),
                nccl_allgather_alone=dict(bytes_out=ag_bytes, ms=round(ag_ms, 4),
                                          busbw_gbs=round(ag_bytes * (world - 1) / world
                                                          / (ag_ms * 1e-3) / 1e9, 1)),
                heads_per_rank=lh, kv_heads_per_rank=wl.Hkv,
                global_batch=B, scaling="strong", parity=parity)


def run_ours(args, cfg):
    import torch
    world, rank, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    wl = Workload(cfg, dev, seed=1234 + rank)
    ws = wl.input_bytes()
    assert ws == input_bytes_of(cfg)
    flush = ws < 2 * L2_BYTES
    scratch = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev) if flush else None

    for i in range(args.warmup):
        wl.step(i)
    torch.cuda.synchronize()
    assert wl.ca.device_status(wl.stream.cuda_stream) == 0, "device-side timeout in warm-up"

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(physical_gpu_index(local)) as clk:
        for i in range(args.steps):
            if flush:
                scratch.zero_()
            starts[i].record(wl.stream)
            wl.step(i)
            ends[i].record(wl.stream)
        torch.cuda.synchronize()
    barrier(world)
    ms_local = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    ms_total = max_over_ranks(ms_local, world)
    status = wl.ca.device_status(wl.stream.cuda_stream)
    assert status == 0, f"device-side status {status}"
    clocks = clk.summary()

    flops = step_flops(cfg)
    value = world * flops * args.steps / (ms_total * 1e-3) / 1e12

    # Dominant kernel: the attention kernel alone, on the same prepared tensors.
    peaks = load_peaks()
    reps = max(3, min(args.steps, 50))
    attn_ms = sum(kernel_ms(wl, flush, scratch, reps))
    roof = roofline(args.config, cfg, cfg["layers"], attn_ms, peaks)

    # The attention kernel alone on the other tensor/HBM-bound configs, so
    # that one run records every config's roofline (1 GPU only).
    by_config = None
    if world == 1 and not args.no_by_config:
        by_config = {}
        for name in ("c2", "c4", "c5"):
            if name == args.config:
                continue
            c = CONFIGS[name]
            w2 = Workload(c, dev, seed=99)
            fl2 = w2.input_bytes() < 2 * L2_BYTES
            if fl2 and scratch is None:
                scratch = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)
            for i in range(3):
                w2.step(i)  # writes q_work (the rotated Q the kernel-alone run reads)
            ms = kernel_ms(w2, fl2, scratch, reps)
            if name == "c5":  # sliding-window layers and the global layer apart
                slide = [k for k, (w, _) in enumerate(c["layers"]) if w is not None]
                glob = [k for k, (w, _) in enumerate(c["layers"]) if w is None]
                by_config["c5_sliding"] = roofline(
                    name, c, [c["layers"][slide[0]]], statistics.mean(ms[k] for k in slide),
                    peaks, "c5_sliding")
                by_config["c5_global"] = roofline(name, c, [c["layers"][glob[0]]],
                                                  ms[glob[0]], peaks, "c5_global")
            else:
                by_config[name] = roofline(name, c, c["layers"], sum(ms), peaks)
            del w2
            torch.cuda.synchronize()
        torch.cuda.empty_cache()

    # The rows on either side of attention, on one GPU: weight dequantisation
    # (HBM), the QKV projection GEMM (tensor) and the denoising step's
    # per-candidate statistics (HBM).
    extras = None
    if world == 1 and not args.no_by_config:
        try:
            extras = run_extras(dev, peaks, scratch)
        except Exception as e:  # an optional leg must not lose the main line
            extras = {"error": f"{type(e).__name__}: {e}"}

    # Head sharding (N > 1): every rank computes its kv-head slice (and the
    # query heads of those groups) of ONE global batch of the config, then
    # one NCCL all-gather per layer reassembles full [tokens, n_head, hd]
    # rows for o_proj (src/model/forward.rs:345). Strong scaling; reported
    # compute-only and with the gather, both max over ranks.
    head_sharded = None
    if world > 1 and cfg["Hkv"] % world == 0 and not args.no_head_shard:
        head_sharded = run_head_sharded(args, cfg, world, rank, dev)

    # End to end through the host-buffer drop-in entry point.
    e2e = None
    if not args.no_e2e:
        ee = E2E(cfg)
        ee.step()
        torch.cuda.synchronize()
        n_e2e = max(1, min(args.steps, args.e2e_steps))
        barrier(world)
        t0 = time.perf_counter()
        for _ in range(n_e2e):
            ee.step()
        dt = max_over_ranks(time.perf_counter() - t0, world)
        e2e = dict(value=round(world * flops * n_e2e / dt / 1e12, 3), unit="TFLOP/s",
                   h2d_bytes_per_step=ee.h2d, d2h_bytes_per_step=ee.d2h, steps=n_e2e,
                   api="ca_attention_host_f32 (fp32 host buffers, precise weights)",
                   pcie_h2d_bytes_per_step=ee.pcie_h2d)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(cfg, args.config, args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": "canvas-attention TFLOP/s",
            "value": round(value, 2),
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_total / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded N(0,1), bf16)",
            "config": config_dict(args, cfg, world),
            "tokens_per_s": round(world * cfg["B"] * cfg["na"] * args.steps / (ms_total * 1e-3), 1),
            "roofline": roof,
            "roofline_by_config": by_config,
            "roofline_extras": extras,
            "head_sharded": head_sharded,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": wl.launches_per_step * args.steps,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_reference(args, cfg):
    """The reference's CPU implementation of the path (restated in C under
    oracle/, all host threads) on a bounded sample per step."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    cs = CpuSample(cfg)
    # Each step is the same bounded row sample, sized so that the whole run
    # stays within about two minutes of CPU time.
    n_rows = cs.calibrate(min(args.ref_step_seconds, 120.0 / max(1, args.steps)))
    for _ in range(args.warmup):
        cs.run(max(16, n_rows // 8))
    tf, ts, tr = 0.0, 0.0, 0
    rates = []
    for _ in range(args.steps):
        f, s, rows = cs.run(n_rows)
        tf += f
        ts += s
        tr += rows
        rates.append(f / s / 1e12)
    value = tf / ts / 1e12
    sample = cs.describe(tr // max(1, args.steps), args.config) + " per step"
    line = {
        "impl": "reference",
        "metric": "canvas-attention TFLOP/s",
        "value": value,
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ts / args.steps * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,1))",
        "config": config_dict(args, cfg, world),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": cs.threads, "kind": "port",
                         "sample": sample, "spread": [round(min(rates), 5), round(max(rates), 5)],
                         "median": round(statistics.median(rates), 5)},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[1])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c3", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-step-seconds", type=float, default=2.0)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-head-shard", action="store_true",
                    help="skip the head-sharded (all-gather) leg under torchrun")
    ap.add_argument("--no-by-config", action="store_true",
                    help="skip the kernel-alone rooflines of the other configs")
    ap.add_argument("--only-layer", type=int, default=None,
                    help="time only this layer of the config (e.g. c5: 0 sliding, 5 global)")
    ap.add_argument("--hs-chunks", type=int, default=4,
                    help="chunks of sequences the head-sharded leg pipelines")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    cfg = CONFIGS[args.config]
    if args.only_layer is not None:  # one layer of a multi-layer config (profiling)
        cfg = dict(cfg, layers=[cfg["layers"][args.only_layer]])
    if args.impl == "reference":
        run_reference(args, cfg)
    else:
        run_ours(args, cfg)


if __name__ == "__main__":
    main()
