"""MoE-layer throughput benchmark of the B200 MoE execution provider.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config c1|c2|c3|c4|c5] [--tokens T[,T...]] [--no-cpu]

A "step" is one com.microsoft MoE / QMoE layer call over one batch of synthetic tokens.
The default workload is benchmark config 2 of 5, the Mixtral-8x7B-shaped fp16 layer
(T=4096, H=4096, I=14336, E=8, k=2, SwiGLU via fc3, no bias); the other configs are
measured with --config for the kernel notes.  Inputs are generated on the device from
fixed seeds with the configs' distributions (no dataset is involved): x, logits ~ N(0,1),
weights ~ N(0, 0.02), biases ~ N(0, 0.01), int codes uniform with lognormal scales, and
for config 4 a Zipf(1.1) per-expert logit bias rescaled to [0, 3].

* ``value``: tokens/s with inputs resident in HBM, K timed steps bracketed by a
  barrier + synchronize, CUDA events on the launching stream, max over ranks.  Every
  config except the small fp32 one streams more than the 126 MB L2 per step.
* ``e2e``: the same metric through the kernel-object API (the call the plugin makes)
  with the step's input and router logits copied from pinned host memory and the
  output read back to host memory inside the timed region.
* ``roofline``: the dominant kernel, its algorithmic FLOPs (tensor-bound configs) or
  bytes (weight-streaming QMoE decode) per launch over its CUDA-event duration,
  against MEASURED_PEAKS.json.
* ``cpu_baseline``: the C restatement of the CPU path (oracle/moe_oracle.c, "port")
  on a bounded sample of the same layer on the host cores.
* ``--impl reference``: the same CPU restatement timed as the reference arm (the
  reference has no MoE kernel and ONNX Runtime is not installable here).

At N > 1 the layer runs expert-parallel: rank r owns experts [r*E/N, (r+1)*E/N), routes
its own T tokens and exchanges routed rows with NCCL all-to-alls (weak scaling: T
tokens per GPU; ``value`` counts the tokens of all ranks).
"""

from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import pathlib
import statistics
import subprocess
import sys
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "MoE-layer tokens/s"
UNIT = "tokens/s"

CONFIGS = {
    "c1": dict(kind="moe", T=256, H=512, I=1024, E=8, k=2, act="silu", gated=False,
               dtype="float32", bias=True,
               desc="configs[0]: com.microsoft.MoE fp32, T={T} H=512 I=1024 E=8 k=2 silu, "
                    "fc1/fc2 bias"),
    "c2": dict(kind="moe", T=4096, H=4096, I=14336, E=8, k=2, act="silu", gated=True,
               dtype="float16", bias=False,
               desc="configs[1]: Mixtral-8x7B-shaped com.microsoft.MoE fp16, T={T} H=4096 "
                    "I=14336 E=8 k=2 SwiGLU(fc3)"),
    "c3": dict(kind="qmoe", T=1, H=4096, I=14336, E=8, k=2, bits=4, block=128, mu=-5.0,
               sigma=0.3,
               desc="configs[2]: QMoE int4 block 128, fp16, Mixtral shape, T={T} E=8 k=2 "
                    "SwiGLU(fc3)"),
    "c4": dict(kind="moe", T=16384, H=2048, I=768, E=64, k=8, act="silu", gated=True,
               dtype="float16", bias=False, zipf=True,
               desc="configs[3]: fine-grained com.microsoft.MoE fp16, T={T} H=2048 I=768 "
                    "E=64 k=8 SwiGLU, Zipf expert bias"),
    "c5": dict(kind="qmoe", T=64, H=4096, I=6400, E=16, k=2, bits=8, block=0, mu=-6.0,
               sigma=0.25,
               desc="configs[4]: QMoE int8 per-row scales, fp16, T={T} H=4096 I=6400 E=16 "
                    "k=2 SwiGLU(fc3)"),
}

# DRAM bytes (read + write) of one fc1(+fc3) launch, keyed by (config, tokens), from the
# ncu captures summarised in profiles/tc_pair_grouped_gemm_c2.md and
# profiles/tc_pair_qgemm_kernel_c5_t4096.md.
FC1_TRAFFIC_BYTES = {("c2", 4096): 2_177_550_848, ("c5", 4096): 1_006_231_808}
# Routed rows (tokens x k) up to which QMoE prefill converts codes inside the GEMM
# (kQmoeFusedMaxRows in the library).
QMOE_FUSED_MAX_ROWS = 16384
# Routed rows from which a QMoE call with a prepack runs on the prepacked weights
# (kPrepackMinRows in the library; MOE_B200_PREPACK_MIN_ROWS overrides both).
PREPACK_MIN_ROWS = 0


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return dict(tflops=d["bf16_tflops"], tflops_sus=d.get("bf16_tflops_sustained"),
                    hbm=d["hbm_gbs"], src="measured")
    return dict(tflops=1590.0, tflops_sus=1400.0, hbm=6650.0, src="fallback")


class ClockSampler:
    """SM clocks and throttle reasons during the timed region: NVML queries from a thread
    every 2 ms (read-only), else nvidia-smi sampling.  The NVML handle is found by the CUDA
    device's PCI address, so it is the GPU being timed whatever the index order."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clocks-event reason bits (nvml.h): SwPowerCap, HwSlowdown, SwThermal, HwThermal.
    BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
            "hw_thermal_slowdown": 0x40}

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.rows = []      # nvidia-smi rows
        self.samples = []   # NVML: (sm_mhz, max_mhz, reasons bitmask)
        self._stop = None
        self._thread = None

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        pr = torch.cuda.get_device_properties(self.index)
        try:
            bus = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def __enter__(self):
        import threading
        try:
            nv, h = self._nvml_handle()
            mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            self._stop = threading.Event()

            def run():
                while not self._stop.is_set():
                    try:
                        self.samples.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM), mx,
                                             nv.nvmlDeviceGetCurrentClocksEventReasons(h)))
                    except Exception:
                        pass
                    self._stop.wait(0.002)

            self._thread = threading.Thread(target=run, daemon=True)
            self._thread.start()
            return self
        except Exception:
            self._thread = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.rows = [l.split(", ") for l in out.strip().splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        for clk, m, bits in self.samples:
            sm.append(float(clk))
            mx = max(mx, float(m))
            reasons.update(n for n, b in self.BITS.items() if bits & b)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            try:
                sm.append(float(r[1]))
                mx = max(mx, float(r[2]))
                for n, v in zip(names, r[5:9]):
                    if v.strip() == "Active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm),
                "source": "nvml" if self.samples else ("nvidia-smi" if self.rows else None)}


# ----------------------------------------------------------------- synthetic layer
def make_layer(cfg, dev, seed):
    """Device tensors of one layer with the config's distributions."""
    import torch
    g = torch.Generator(device=dev).manual_seed(seed)
    T, H, I, E = cfg["T"], cfg["H"], cfg["I"], cfg["E"]
    rn = lambda *s: torch.randn(*s, device=dev, generator=g)
    if cfg["kind"] == "moe":
        dt = getattr(torch, cfg["dtype"])
        logits = rn(T, E)
        if cfg.get("zipf"):
            import numpy as np
            z = np.random.default_rng(seed).zipf(1.1, E).astype(np.float64)
            span = z.max() - z.min()
            bias_e = 3.0 * (z - z.min()) / span if span > 0 else np.zeros(E)
            logits = logits + torch.tensor(bias_e, device=dev, dtype=torch.float32)[None, :]
        return dict(x=rn(T, H).to(dt), router_probs=logits.to(dt),
                    fc1_w=(rn(E, I, H) * 0.02).to(dt), fc2_w=(rn(E, H, I) * 0.02).to(dt),
                    fc3_w=(rn(E, I, H) * 0.02).to(dt) if cfg["gated"] else None,
                    fc1_b=(rn(E, I) * 0.01).to(dt) if cfg.get("bias") else None,
                    fc2_b=(rn(E, H) * 0.01).to(dt) if cfg.get("bias") else None)
    bits, bs = cfg["bits"], cfg["block"]
    lo, hi = (-8, 7) if bits == 4 else (-127, 127)

    def weights(N, K):
        codes = torch.randint(lo, hi + 1, (E, N, K), device=dev, generator=g, dtype=torch.int16)
        if bits == 4:
            q = (codes + 8).to(torch.uint8)
            packed = (q[..., 0::2] | (q[..., 1::2] << 4)).contiguous()
        else:
            packed = (codes + 128).to(torch.uint8)
        del codes
        shape = (E, N, (K + bs - 1) // bs) if bs else (E, N)
        sc = torch.exp(cfg["mu"] + cfg["sigma"] * torch.randn(*shape, device=dev, generator=g))
        return packed, sc.half()

    q1, s1 = weights(I, H)
    q3, s3 = weights(I, H)
    q2, s2 = weights(H, I)
    return dict(x=rn(T, H).half(), router_probs=rn(T, E).half(), fc1_q=q1, fc1_s=s1, fc2_q=q2,
                fc2_s=s2, fc3_q=q3, fc3_s=s3)


def problem_and_tensors(pkg, cfg, L, out):
    T, H, I, E, k = cfg["T"], cfg["H"], cfg["I"], cfg["E"], cfg["k"]
    if cfg["kind"] == "moe":
        dt = {"float32": pkg.FLOAT, "float16": pkg.FLOAT16, "bfloat16": pkg.BFLOAT16}[cfg["dtype"]]
        prob = pkg.make_problem(T, H, I, E, dt, has_fc3=cfg["gated"], activation_type=cfg["act"],
                                k=k, normalize_routing_weights=1)
        tens = dict(input=L["x"], router_probs=L["router_probs"], fc1_weights=L["fc1_w"],
                    fc1_bias=L["fc1_b"], fc2_weights=L["fc2_w"], fc2_bias=L["fc2_b"],
                    fc3_weights=L["fc3_w"], output=out)
        inputs = [L["x"], L["router_probs"], L["fc1_w"], L["fc1_b"], L["fc2_w"], L["fc2_b"],
                  L["fc3_w"], None]
        op_attrs = dict(activation_type=cfg["act"], k=k, normalize_routing_weights=1)
        return prob, tens, inputs, op_attrs, "MoE"
    prob = pkg.make_problem(T, H, I, E, pkg.FLOAT16, has_fc3=True, activation_type="silu", k=k,
                            normalize_routing_weights=1, expert_weight_bits=cfg["bits"],
                            block_size=cfg["block"])
    tens = dict(input=L["x"], router_probs=L["router_probs"], fc1_weights=L["fc1_q"],
                fc1_scales=L["fc1_s"], fc2_weights=L["fc2_q"], fc2_scales=L["fc2_s"],
                fc3_weights=L["fc3_q"], fc3_scales=L["fc3_s"], output=out)
    inputs = [L["x"], L["router_probs"], L["fc1_q"], L["fc1_s"], None, L["fc2_q"], L["fc2_s"],
              None, L["fc3_q"], L["fc3_s"], None]
    op_attrs = dict(activation_type="silu", k=k, normalize_routing_weights=1,
                    expert_weight_bits=cfg["bits"], block_size=cfg["block"])
    return prob, tens, inputs, op_attrs, "QMoE"


def algorithmic(cfg, L, pkg):
    """FLOPs and bytes of one layer call (bytes over the experts this routing touches)."""
    import torch
    T, H, I, E, k = cfg["T"], cfg["H"], cfg["I"], cfg["E"], cfg["k"]
    n_mat = 3 if (cfg["kind"] == "qmoe" or cfg["gated"]) else 2
    flops_fc1 = T * k * 2 * (n_mat - 1) * H * I
    flops_fc2 = T * k * 2 * H * I
    idx, _ = pkg.route(L["router_probs"], k, 1)
    touched = int(torch.unique(idx).numel())
    if cfg["kind"] == "moe":
        es = 4 if cfg["dtype"] == "float32" else 2
        per_expert = n_mat * H * I * es
        act_es = es
    else:
        per_w = H * I * cfg["bits"] // 8
        nb_h = (H + cfg["block"] - 1) // cfg["block"] if cfg["block"] else 1
        nb_i = (I + cfg["block"] - 1) // cfg["block"] if cfg["block"] else 1
        per_expert = 3 * per_w + (2 * I * nb_h + H * nb_i) * 2
        act_es = 2
    io = T * H * act_es * 2 + T * E * act_es
    return dict(flops=flops_fc1 + flops_fc2, flops_fc1=flops_fc1, flops_fc2=flops_fc2,
                bytes=touched * per_expert + io, touched=touched,
                bytes_fc1=touched * per_expert * (n_mat - 1) / n_mat,
                bytes_fc2=touched * per_expert / n_mat)


# ------------------------------------------------------------------ CPU baseline
def _oracle_lib():
    so = ROOT / "oracle" / "_build" / "libmoe_oracle.so"
    if not so.exists():
        subprocess.run(["make", "-s", "-C", str(ROOT / "oracle")], check=True)
    L = ctypes.CDLL(str(so))
    L.oracle_moe.restype = ctypes.c_int
    L.oracle_moe.argtypes = [ctypes.c_int64] * 4 + [ctypes.c_int] * 4 + [ctypes.c_float] * 3 + \
        [ctypes.c_int] * 2 + [ctypes.c_void_p] * 12
    L.oracle_get_threads.restype = ctypes.c_int
    return L


def cpu_baseline(cfg, L, budget_s=12.0):
    """The C restatement (oracle/moe_oracle.c) on a bounded token sample of the layer, all
    host cores.  MoE weights are handed over as fp32 copies (prepacked once, outside the
    timed call); QMoE weights stay packed and are dequantised inside the call."""
    import numpy as np
    lib = _oracle_lib()
    cores = lib.oracle_get_threads()
    f = lambda t: None if t is None else np.ascontiguousarray(t.float().cpu().numpy())
    u8 = lambda t: np.ascontiguousarray(t.cpu().numpy())
    P = lambda a: None if a is None else a.ctypes.data_as(ctypes.c_void_p)
    x_all, lg_all = f(L["x"]), f(L["router_probs"])
    T, H, I, E, k = cfg["T"], cfg["H"], cfg["I"], cfg["E"], cfg["k"]
    if cfg["kind"] == "moe":
        w1, w2, w3, b1, b2 = f(L["fc1_w"]), f(L["fc2_w"]), f(L["fc3_w"]), f(L["fc1_b"]), f(L["fc2_b"])
        act = {"silu": 2, "gelu": 1, "relu": 0, "identity": 3}[cfg["act"]]
        bits = bs = 0
        s1 = s2 = s3 = None
    else:
        w1, w2, w3 = u8(L["fc1_q"]), u8(L["fc2_q"]), u8(L["fc3_q"])
        s1, s2, s3 = f(L["fc1_s"]), f(L["fc2_s"]), f(L["fc3_s"])
        b1 = b2 = None
        act, bits, bs = 2, cfg["bits"], cfg["block"]

    def run(n):
        x, lg = np.ascontiguousarray(x_all[:n]), np.ascontiguousarray(lg_all[:n])
        out = np.zeros_like(x)
        t0 = time.perf_counter()
        rc = lib.oracle_moe(n, H, I, E, k, 1, act, 0, 1.0, 0.0, math.inf, bits, bs, P(x), P(lg),
                            P(w1), P(s1), P(b1), P(w2), P(s2), P(b2), P(w3), P(s3), None, P(out))
        if rc != 0:
            raise RuntimeError("oracle_moe failed")
        return time.perf_counter() - t0

    n = min(T, 32)
    dt = run(n)
    n2 = int(min(T, max(n, n * budget_s / max(dt, 1e-3) * 0.8)))
    if n2 > n:
        n, dt = n2, run(n2)
    return {"value": n / dt, "unit": UNIT, "cores": cores, "kind": "port",
            "label": f"C port of the CPU path (oracle/moe_oracle.c, cache-blocked fp32 FMA "
                     f"GEMM) on {cores} host cores; not the ONNX Runtime CPU EP, which is "
                     f"unavailable on this box",
            "sample": f"{n} of {T} tokens of the same layer, one call, {dt:.2f} s"}


# ------------------------------------------------------------------ our arm
def host_copy_ceiling(hx, hl, hout, dev, steps, warmup, world):
    """The host-copy part of an e2e step alone: per step the H2D copies of the step's
    tokens and logits (one stream) and the D2H copy of an output-sized buffer (another
    stream), back to back with no compute, on every rank at once (wall clock, max over
    ranks).  If the e2e step is not longer than this, the host copies bound it."""
    import torch
    import torch.distributed as dist
    dx = torch.empty(hx.shape, dtype=hx.dtype, device=dev)
    dl = torch.empty(hl.shape, dtype=hl.dtype, device=dev)
    dout = torch.zeros(hout.shape, dtype=hout.dtype, device=dev)
    cin, cout = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def step():
        with torch.cuda.stream(cin):
            dx.copy_(hx, non_blocking=True)
            dl.copy_(hl, non_blocking=True)
        with torch.cuda.stream(cout):
            hout.copy_(dout, non_blocking=True)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    torch.cuda.synchronize(dev)
    ms = (time.perf_counter() - t0) * 1e3 / steps
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    nbytes = (hx.numel() * hx.element_size() + hl.numel() * hl.element_size() +
              hout.numel() * hout.element_size())
    return {"copy_only_ms_per_step": round(ms, 4),
            "host_copy_gbs_per_gpu": round(nbytes / (ms / 1e3) / 1e9, 1),
            "host_copy_gbs_all_gpus": round(world * nbytes / (ms / 1e3) / 1e9, 1)}



def adjacent_ops(pkg, cfg, L, dev, stream, args, pk):
    """The pre-MoE rows of the same tokens (residual add + RMS norm + router MatMul,
    moe_b200_norm_router), timed with CUDA events against the HBM roofline."""
    import torch
    if cfg["kind"] != "moe" or cfg["dtype"] == "float32":
        return None
    x = L["x"]
    T, H = x.shape
    E = cfg["E"]
    g = torch.Generator(device=dev).manual_seed(99)
    skip = torch.randn(T, H, device=dev, generator=g).to(x.dtype)
    gamma = 1.0 + 0.1 * torch.randn(H, device=dev, generator=g)
    wr = (torch.randn(E, H, device=dev, generator=g) * 0.02).to(x.dtype)
    for _ in range(max(3, args.warmup)):
        pkg.norm_router(x, gamma, 1e-6, wr, skip=skip, stream=stream)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        pkg.norm_router(x, gamma, 1e-6, wr, skip=skip, stream=stream)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / args.steps
    es = x.element_size()
    # read x and skip once, write residual and normed, logits; gamma and the router weights
    alg = 4 * T * H * es + T * E * es + H * 4 + E * H * es
    gbs = alg / (ms / 1e3) / 1e9
    return {"norm_router": {"ms": round(ms, 4), "alg_bytes": alg, "achieved_gbs": round(gbs, 1),
                            "frac_of_hbm": round(gbs / pk["hbm"], 4),
                            "what": "h = x + skip; rms-normalised h * gamma; router logits [T, E]"}}


def bench_ours(args, cfg, rank, world, dev):
    import torch
    import __graft_entry__ as ge
    pkg = ge.load_package()
    L = make_layer(cfg, dev, 20261202 + rank)
    T = cfg["T"]
    out = torch.empty_like(L["x"])
    prob, tens, inputs, op_attrs, op_type = problem_and_tensors(pkg, cfg, L, out)
    # --prepack (QMoE): weights dequantised once before timing (moe_b200_prepack_create);
    # prefill-sized calls then run the fp16 GEMMs on them.
    wpk = pkg.Prepacked(prob, tens) if (args.prepack and cfg["kind"] == "qmoe") else None
    ws = torch.empty(pkg.workspace_size(prob, wpk), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def fwd(events=None):
        if wpk is None and events is None:
            return pkg.forward(prob, tens, ws, stream)
        return pkg.forward(prob, tens, ws, stream, prepacked=wpk, events=events)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    def timed(step, steps):
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize(dev)
        barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        return max_over_ranks(e0.elapsed_time(e1)) / steps

    # ---- device-resident throughput.  Inside the timed loop every call records CUDA
    # events at the fc1 and fc2 boundaries only (three events, a few us per call), so the
    # dominant kernel's roofline comes from the timed region itself.
    i_fc1, i_fc2 = pkg.STAGES.index("fc1"), pkg.STAGES.index("fc2")
    gemm_ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)]
               for _ in range(args.steps)]
    for row in gemm_ev:
        for ev in row:
            ev.record(stream)  # creates the event handle
    torch.cuda.synchronize(dev)
    it_ev = iter(gemm_ev)

    def timed_call():
        row = next(it_ev)
        evs = [None] * (len(pkg.STAGES) + 1)
        evs[i_fc1], evs[i_fc2], evs[i_fc2 + 1] = row
        return fwd(evs)

    warm_left = [args.warmup]  # timed() runs the warm-up calls first

    def step():
        if warm_left[0] > 0:
            warm_left[0] -= 1
            return fwd()
        return timed_call()

    with ClockSampler(dev.index) as clk:
        ms = timed(step, args.steps)
    value = world * T / (ms / 1e3)
    gemm_ms = {"fc1": statistics.median(r[0].elapsed_time(r[1]) for r in gemm_ev),
               "fc2": statistics.median(r[1].elapsed_time(r[2]) for r in gemm_ev)}

    # ---- per-stage times: the same number of back-to-back calls right after the timed
    # loop, with the stage boundaries recorded as CUDA events on the stream (no
    # synchronisation between calls; an event costs ~3 us of stream time, so the stage
    # sum slightly exceeds ms_per_step on small configs).
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(len(pkg.STAGES) + 1)]
           for _ in range(args.steps)]
    for row in evs:
        for ev in row:
            ev.record(stream)  # creates the event handle
    torch.cuda.synchronize(dev)
    for row in evs:
        fwd(row)
    torch.cuda.synchronize(dev)
    stage = {s: [row[i].elapsed_time(row[i + 1]) for row in evs]
             for i, s in enumerate(pkg.STAGES)}
    stage_ms = {s: statistics.median(v) for s, v in stage.items()}

    # ---- end to end through the kernel object with host buffers
    op = (pkg.QMoE if op_type == "QMoE" else pkg.MoE)(**op_attrs)
    hx, hl = L["x"].cpu().pin_memory(), L["router_probs"].cpu().pin_memory()
    hout = torch.empty_like(hx).pin_memory()
    dx, dl = torch.empty_like(L["x"]), torch.empty_like(L["router_probs"])
    e2e_inputs = [dx, dl] + inputs[2:]
    if wpk is not None:
        op.prepack(e2e_inputs)

    def e2e_step():
        dx.copy_(hx, non_blocking=True)
        dl.copy_(hl, non_blocking=True)
        op(e2e_inputs, out=out, stream=stream)
        hout.copy_(out, non_blocking=True)

    serial_ms = timed(e2e_step, args.steps)
    op.release()

    # ---- end to end through the host-buffer pipeline (moe_b200_pipeline_*): every step
    # copies its inputs from pinned host memory and its output back; the copies of
    # neighbouring steps overlap this step's compute.  Wall clock from the first submit
    # to the completion of the last D2H, max over ranks.
    with pkg.Pipeline(prob, tens, depth=args.pipeline_depth) as pl:
        if wpk is not None:
            pl.set_prepacked(wpk)
        for _ in range(args.warmup):
            pl.submit(hx, hl, hout)
        pl.synchronize()
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            pl.submit(hx, hl, hout)
        pl.synchronize()
        e2e_ms = max_over_ranks((time.perf_counter() - t0) * 1e3) / args.steps
        barrier()
    es = hx.element_size()
    e2e = {"value": world * T / (e2e_ms / 1e3), "unit": UNIT,
           "h2d_bytes_per_step": hx.numel() * es + hl.numel() * es,
           "d2h_bytes_per_step": hout.numel() * es,
           "api": "moe_b200_pipeline_submit (host buffers, copies overlapped across steps)",
           "serial_value": world * T / (serial_ms / 1e3),
           "serial_api": "moe_b200_kernel_compute, one call at a time (H2D, layer, D2H)",
           "host_copies_alone": host_copy_ceiling(hx, hl, hout, dev, args.steps, args.warmup,
                                                  world)}

    pk = peaks()
    adjacent = adjacent_ops(pkg, cfg, L, dev, stream, args, pk)
    alg = algorithmic(cfg, L, pkg)
    decode = cfg["kind"] == "qmoe" and T * cfg["k"] <= 512  # the library's decode threshold
    if decode:
        achieved = alg["bytes_fc1"] / (gemm_ms["fc1"] / 1e3) / 1e9
        roof = {"bound": "hbm", "kernel": "qmoe_decode_kernel (fc1+fc3 pass)",
                "achieved": round(achieved, 1), "peak": pk["hbm"], "unit": "GB/s",
                "frac": round(achieved / pk["hbm"], 4), "traffic": None,
                "peak_source": f"{pk['src']} HBM copy (MEASURED_PEAKS.json)",
                "alg_bytes_per_launch": int(alg["bytes_fc1"]),
                "fc2": {"achieved": round(alg["bytes_fc2"] / (gemm_ms["fc2"] / 1e3) / 1e9, 1)},
                "experts_touched": alg["touched"],
                "layer_frac": round((alg["bytes"] / pk["hbm"] / 1e9) / (ms / 1e3), 4)}
    else:
        prepacked = wpk is not None and not decode and T * cfg["k"] >= int(
            os.environ.get("MOE_B200_PREPACK_MIN_ROWS", PREPACK_MIN_ROWS))
        fused_q = (cfg["kind"] == "qmoe" and not prepacked
                   and T * cfg["k"] <= QMOE_FUSED_MAX_ROWS)
        if cfg["kind"] == "moe" and cfg["dtype"] == "float32":
            k_name = "simt_gemm_kernel (FFMA)"
        elif fused_q:
            k_name = "tc_pair_qgemm_kernel (codes converted in shared memory; fc1+fc3, SwiGLU epilogue)"
        else:
            k_name = "tc_pair_grouped_gemm_kernel (fc1+fc3, SwiGLU epilogue)"
        achieved = alg["flops_fc1"] / (gemm_ms["fc1"] / 1e3) / 1e12
        if cfg["kind"] == "moe" and cfg["dtype"] == "float32":
            # FFMA-bound: no tensor-core peak applies.  Derived peak = SMs x 128 fp32
            # lanes x 2 FLOP x the maximum SM clock (no measured FFMA figure exists).
            props = torch.cuda.get_device_properties(dev)
            mhz = float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text()).get(
                "sm_max_mhz", 1965.0)) if (ROOT / "MEASURED_PEAKS.json").exists() else 1965.0
            c_peak = props.multi_processor_count * 128 * 2 * mhz * 1e6 / 1e12
            bound, c_src, c_sus = "fp32 FFMA", (f"derived: {props.multi_processor_count} SMs x "
                                                f"128 lanes x 2 x {mhz:.0f} MHz"), None
        else:
            c_peak, bound = pk["tflops"], "tensor"
            c_src = f"{pk['src']} bf16 burst (MEASURED_PEAKS.json)"
            c_sus = round(achieved / pk["tflops_sus"], 4) if pk["tflops_sus"] else None
        roof_t = max(alg["flops"] / (c_peak * 1e12), alg["bytes"] / (pk["hbm"] * 1e9))
        roof = {"bound": bound, "kernel": k_name, "achieved": round(achieved, 1),
                "peak": round(c_peak, 1), "unit": "TFLOP/s", "frac": round(achieved / c_peak, 4),
                "peak_source": c_src,
                "frac_of_sustained": c_sus,
                "traffic": None if prepacked else FC1_TRAFFIC_BYTES.get((args.config, T)),
                "alg_flops_per_launch": alg["flops_fc1"],
                "fc2": {"achieved": round(alg["flops_fc2"] / (gemm_ms["fc2"] / 1e3) / 1e12, 1)},
                "layer_frac": round(roof_t / (ms / 1e3), 4)}
    # Launches per layer call: route, scan, permute, gather, fc1, fc2, combine.  QMoE
    # prefill with codes converted inside the GEMM adds two row-sum launches for int8
    # per-row scales (biased codes); beyond the fused limit it adds one dequantisation
    # launch per weight tensor.
    if decode:
        launches = 5
    elif cfg["kind"] != "qmoe":
        launches = 7
    elif prepacked:
        launches = 7
    elif not fused_q:
        launches = 10
    else:
        launches = 9 if (cfg["bits"] == 8 and cfg["block"] == 0) else 7
    result = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32" if cfg.get("dtype") == "float32" else "f16",
        "data": "synthetic (seeded, on-device; config distributions; random init)",
        "config": {"workload": cfg["desc"].format(T=T), "global_batch": T * world,
                   "tokens_per_gpu": T,
                   "parallelism": f"replicas{world}" if world > 1 else "single",
                   "l2": "inputs larger than L2 (weights streamed every step)"
                         if alg["bytes"] > 126e6 else "inputs smaller than L2 (not flushed)",
                   **({"weights": "prepacked: dequantised once before timing "
                                  "(moe_b200_prepack_create)"} if wpk is not None else {})},
        "e2e": e2e, "roofline": roof,
        "stage_ms": {s: round(v, 4) for s, v in stage_ms.items()},
        "adjacent_ops": adjacent,
        "gemm_ms_in_timed_loop": {s: round(v, 4) for s, v in gemm_ms.items()},
        "gpu_launches": launches * args.steps,
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        result["cpu_baseline"] = cpu_baseline(cfg, L)
    return result


def bench_ep(args, cfg, rank, world, dev):
    """Expert-parallel layer over ``world`` ranks (NCCL all-to-all dispatch/combine)."""
    import torch
    import torch.distributed as dist
    import __graft_entry__ as ge
    pkg = ge.load_package()
    from onnxruntime_musa_b200 import ep
    L = make_layer(cfg, dev, 20261202)          # the same weights on every rank
    g = torch.Generator(device=dev).manual_seed(7000 + rank)
    T, H, E = cfg["T"], cfg["H"], cfg["E"]
    L["x"] = torch.randn(T, H, device=dev, generator=g).to(L["x"].dtype)
    logits = torch.randn(T, E, device=dev, generator=g)
    if cfg.get("zipf"):  # the same per-expert bias on every rank (seeded as make_layer's)
        import numpy as np
        z = np.random.default_rng(20261202).zipf(1.1, E).astype(np.float64)
        span = z.max() - z.min()
        bias_e = 3.0 * (z - z.min()) / span if span > 0 else np.zeros(E)
        logits = logits + torch.tensor(bias_e, device=dev, dtype=torch.float32)[None, :]
    L["router_probs"] = logits.to(L["router_probs"].dtype)
    out = torch.empty_like(L["x"])
    # Load per rank: routed rows each rank's experts receive from all ranks (one routing
    # pass outside the timed region); imbalance = max over ranks / mean.
    ridx, _ = pkg.route(L["router_probs"], cfg["k"], 1)
    per_rank = torch.bincount((ridx.long() // (E // world)).flatten(), minlength=world)
    dist.all_reduce(per_rank)
    loads = [int(v) for v in per_rank.cpu()]
    imbalance = max(loads) / (sum(loads) / world)
    prob, tens, inputs, op_attrs, op_type = problem_and_tensors(pkg, cfg, L, out)
    names = ["fc1_weights", "fc1_scales", "fc1_bias", "fc2_weights", "fc2_scales", "fc2_bias",
             "fc3_weights", "fc3_scales", "fc3_bias"]
    local = ep.shard_experts({n: tens.get(n) for n in names}, rank, world)
    layer = ep.ExpertParallelMoE(pkg, num_experts=E, hidden_size=H, inter_size=cfg["I"],
                                 dtype=prob.dtype, has_fc3=bool(prob.has_fc3),
                                 local_weights=local, **op_attrs)
    stream = torch.cuda.current_stream(dev)

    def timed(step):
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize(dev)
        dist.barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        dist.barrier()
        t = torch.tensor([e0.elapsed_time(e1) / args.steps], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    x, lg = L["x"], L["router_probs"]
    chunks = args.ep_chunks or 1
    with ClockSampler(dev.index) as clk:
        ms = timed(lambda: layer.forward(x, lg, chunks=chunks))
    # Per-phase device times of the p2p exchange (a second run of `steps` calls with phase
    # events on the stream, no synchronisation between calls): median per rank, then the
    # max over ranks per phase.
    phase_ms = None
    if layer.transport == "p2p":
        n_ev = len(pkg.EP_PHASES) + 1
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(n_ev)]
               for _ in range(args.steps)]
        for row in evs:
            for ev in row:
                ev.record(stream)
        torch.cuda.synchronize(dev)
        dist.barrier()
        for row in evs:
            layer.forward(x, lg, events=row)
        torch.cuda.synchronize(dev)
        med = torch.tensor([statistics.median(row[i].elapsed_time(row[i + 1]) for row in evs)
                            for i in range(n_ev - 1)], dtype=torch.float64, device=dev)
        every = [torch.empty_like(med) for _ in range(world)]
        dist.all_gather(every, med)
        phase_ms = {name: {"max_over_ranks": round(max(float(e[i]) for e in every), 4),
                           "per_rank": [round(float(e[i]), 4) for e in every]}
                    for i, name in enumerate(pkg.EP_PHASES)}
    hx, hl = x.cpu().pin_memory(), lg.cpu().pin_memory()
    hout = torch.empty_like(hx).pin_memory()
    # End to end: every step copies its tokens and logits from pinned host memory and its
    # output back (ep.HostPipeline: the copies of neighbouring steps overlap this step's
    # layer); wall clock from the first submit to the last D2H, max over ranks.
    pipe = ep.HostPipeline(layer, T, x.dtype, dev)
    for _ in range(args.warmup):
        pipe.submit(hx, hl, hout)
    pipe.synchronize()
    dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        pipe.submit(hx, hl, hout)
    pipe.synchronize()
    tw = torch.tensor([(time.perf_counter() - t0) * 1e3 / args.steps], dtype=torch.float64,
                      device=dev)
    dist.all_reduce(tw, op=dist.ReduceOp.MAX)
    e2e_ms = float(tw.item())
    dist.barrier()
    copy_ceiling = host_copy_ceiling(hx, hl, hout, dev, args.steps, args.warmup, world)
    pk = peaks()
    alg = algorithmic(cfg, L, pkg)
    es = hx.element_size()
    achieved = alg["flops"] / (ms / 1e3) / 1e12
    return {
        "metric": METRIC, "value": round(world * T / (ms / 1e3), 1), "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32" if cfg.get("dtype") == "float32" else "f16",
        "data": "synthetic (seeded, on-device; config distributions; random init)",
        "config": {"workload": cfg["desc"].format(T=T), "global_batch": T * world,
                   "tokens_per_gpu": T, "parallelism": f"ep{world}", "ep_chunks": chunks,
                   "ep_transport": layer.transport,
                   "rows_per_rank": loads, "imbalance_max_over_mean": round(imbalance, 4),
                   "l2": "inputs larger than L2 (weights streamed every step)"},
        "e2e": {"value": world * T / (e2e_ms / 1e3), "unit": UNIT,
                "h2d_bytes_per_step": hx.numel() * es + hl.numel() * es,
                "d2h_bytes_per_step": hout.numel() * es,
                "api": "ep.HostPipeline over ExpertParallelMoE.forward (host buffers, copies "
                       "overlapped across steps)",
                "host_copies_alone": copy_ceiling},
        "roofline": {"bound": "tensor", "kernel": "expert-parallel layer (all stages, per rank)",
                     "achieved": round(achieved, 1), "peak": pk["tflops"], "unit": "TFLOP/s",
                     "frac": round(achieved / pk["tflops"], 4), "traffic": None,
                     "peak_source": f"{pk['src']} bf16 burst (MEASURED_PEAKS.json)"},
        # dispatch (route, scan, permute, gather) + expert FFN (fill, histogram, scan,
        # permute, gather, fc1, fc2, un-permute) + combine
        # p2p: route, scan, permute, counts, send, signal, wait, fc1, fc2, signal, wait,
        # combine; collective: 13 per chunk
        "ep_phase_ms": phase_ms,
        "gpu_launches": (12 if layer.transport == "p2p" else 13 * chunks) * args.steps,
        "clocks": clk.summary(),
    }


def bench_reference(args, cfg, rank, world):
    """Reference arm: the CPU restatement of the path on this host's cores."""
    import torch
    if rank != 0:
        return None
    if not torch.cuda.is_available():
        return {"impl": "reference", "unavailable": "no CUDA device to generate the layer on"}
    L = make_layer(cfg, torch.device("cuda:0"), 20261202)
    vals, base = [], None
    budget = max(2.0, 60.0 / (args.warmup + args.steps))
    for i in range(args.warmup + args.steps):
        base = cpu_baseline(cfg, L, budget_s=budget)
        if i >= args.warmup:
            vals.append(base["value"])
    v = statistics.median(vals)
    base["value"] = v
    return {"metric": METRIC, "value": round(v, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "impl": "reference", "dtype": "f32",
            "config": {"workload": cfg["desc"].format(T=cfg["T"]),
                       "engine": "C restatement of the CPU path (oracle/moe_oracle.c)"},
            "cpu_baseline": base,
            "e2e": {"value": round(v, 2), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c2")
    ap.add_argument("--tokens", default=None,
                    help="tokens per GPU (comma list for a sweep); default: the config's")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--prepack", action="store_true",
                    help="QMoE: dequantise the weights once before timing (weight prepack)")
    ap.add_argument("--pipeline-depth", type=int, default=2,
                    help="staging slots of the host-buffer pipeline (e2e)")
    ap.add_argument("--ep-chunks", type=int, default=None,
                    help="token chunks pipelined through the expert-parallel exchange "
                         "(default 1)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    base = CONFIGS[args.config]
    sweep = [int(t) for t in args.tokens.split(",")] if args.tokens else [base["T"]]
    if args.impl == "reference":
        for T in sweep:
            res = bench_reference(args, dict(base, T=T), rank, world)
            if res is not None:
                print(json.dumps(res), flush=True)
        return
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    if world > 1:
        torch.distributed.init_process_group("nccl", device_id=dev)
    for T in sweep:
        run = bench_ours if world == 1 else bench_ep
        res = run(args, dict(base, T=T), rank, world, dev)
        if rank == 0:
            print(json.dumps(res), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
