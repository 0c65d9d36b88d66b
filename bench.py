"""Benchmark of the hachiue attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2] [--impl ours|reference]
                    [--no-secondary] [--no-cpu-baseline]

Prints ONE JSON line (rank 0).

Headline (``value``): configuration 2 of the benchmark set, Qwen3-8B-shape
batched GQA decode attention (64 sequences, 32 query / 8 KV heads, head_dim
128, per-sequence contexts U[512, 8192] from seed 1, f16 KV cache, f32 q /
out).  A step is one decode-attention pass over the whole batch; ``value`` is
its algorithmic HBM GB/s with the inputs resident.  ``e2e`` is the same metric
through the public API with host buffers: every step copies its q and its new
K / V rows from pinned host memory, appends the rows, runs the attention and
reads the output back (hachiue_b200.pipeline.HostPipeline overlaps step i+1's
copies with step i's kernels, as a serving loop does).

``secondary`` (one GPU, default run): the other benchmark configurations in
the same run, each with its own value, roofline (algorithmic work per launch,
kernel time, fraction of MEASURED_PEAKS.json), clocks, e2e and CPU sample:
cfg1 (Qwen3-1.7B decode, f32 cache), cfg3 (PLaMo-3 SWA prefill, bf16, tensor
roofline), cfg4 (Qwen3.5 GDN decode step), cfg5 (Qwen3.5 GDN chunked prefill)
and cfg2_q8 (cfg2's shapes on the reference's own Q8_0 cache format).
``--config N`` (1-7, or 2q8) makes configuration N the headline instead.

Multi-GPU (torchrun, one process per GPU): the headline is weak scaling (each
rank owns its own 64-sequence batch; the per-head outputs of all ranks are
all-gathered every step through this library's NCCL communicator,
hcu_comm_init_rank / hcu_allgather, overlapped with the next step).  The
``strong`` block measures one configuration's fixed work split over the N
GPUs: cfg2 by KV head and cfg5 by QK head (V heads h and h + NK together),
with the all-gather's time and share measured by CUDA events.

Timing: CUDA events on the launching stream, W untimed warm-up steps, K timed
steps bracketed by barrier + synchronize, max over ranks.  cfg2, cfg2_q8, cfg3
and cfg5 read more than L2 (126 MB) per step; cfg1 and cfg4 rotate input
copies to exceed it.  Clocks are sampled (NVML, read-only) during each timed
region.

``--impl reference`` times the reference algorithm on the host cores: the
reference is TypeScript with no JS runtime on the box, so its JS-semantics C
restatement (oracle/) runs, multi-threaded over sequences, on a bounded
sample of the same workload, and also in the reference's own setting (one
thread over a Q8_0 cache), reported beside it.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    except Exception:
        return PEAKS_FALLBACK, "fallback"


def load_traffic(key: str):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu
    summary (profiles/dram_traffic.txt: '<key> <bytes>' lines), or None."""
    p = os.path.join(ROOT, "profiles", "dram_traffic.txt")
    try:
        for line in open(p):
            parts = line.split()
            if len(parts) >= 2 and parts[0] == key:
                return float(parts[1])
    except OSError:
        pass
    return None


class ClockSampler:
    """Samples SM clocks and clock-event (throttle) reasons while the timed
    region runs.  NVML is polled every ~2 ms from a thread (read-only queries),
    so even a timed region of a few milliseconds gets samples; `mark_start` /
    `mark_end` bracket the region and only samples inside it are reported.
    Falls back to `nvidia-smi -lms 100` when NVML is unavailable."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASON_NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.thread = None
        self.samples = []  # (perf_counter, sm_mhz, reasons)
        self.max_mhz = None
        self._stop = threading.Event()
        self.source = None

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:
            import torch
            prop = torch.cuda.get_device_properties(self.gpu)
            bus = f"{prop.pci_domain_id:08x}:{prop.pci_bus_id:02x}:{prop.pci_device_id:02x}.0"
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.gpu)

    def start(self):
        try:
            nv, h = self._nvml_handle()
            bits = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                    "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                    "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                    "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap}
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))

            def poll():
                while not self._stop.is_set():
                    t = time.perf_counter()
                    try:
                        sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                        r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    except Exception:
                        break
                    self.samples.append((t, sm, {n for n, b in bits.items() if r & b}))
                    time.sleep(0.002)

            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            self.source = "nvml"
            return
        except Exception:
            pass
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.source = "nvidia-smi"

        def read():
            for line in self.proc.stdout:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm, self.max_mhz = float(parts[1]), float(parts[2])
                except ValueError:
                    continue
                self.samples.append((time.perf_counter(), sm,
                                     {n for n, v in zip(self.REASON_NAMES, parts[5:9]) if v.lower() == "active"}))

        self.thread = threading.Thread(target=read, daemon=True)
        self.thread.start()

    def wait_ready(self, timeout: float = 10.0):
        """Returns once the first sample arrived (nvidia-smi starts slowly)."""
        t0 = time.perf_counter()
        while self.thread is not None and not self.samples and time.perf_counter() - t0 < timeout:
            time.sleep(0.01)

    def summary(self, t0: float, t1: float):
        """Median SM clock, max clock and the throttle reasons seen between
        perf_counter marks t0 and t1 (the samples just outside a window
        shorter than the polling period when none fall inside)."""
        if self.thread is None:
            return None
        inside = [x for x in self.samples if t0 <= x[0] <= t1]
        window = "timed region"
        if not inside:
            before = [x for x in self.samples if x[0] < t0]
            after = [x for x in self.samples if x[0] > t1]
            inside = before[-1:] + after[:1]
            window = "bracketing samples (timed region shorter than the polling period)"
        if not inside:
            return None
        reasons = set().union(*(x[2] for x in inside))
        return {"sm_mhz": statistics.median(x[1] for x in inside), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(inside), "source": self.source, "window": window}

    def stop(self):
        if self.thread is None:
            return
        self._stop.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        self.thread.join(timeout=5)


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local




# ---------------------------------------------------------------------------
# workload descriptions (no GPU: shared by both arms, so their `config` match)
# ---------------------------------------------------------------------------
def config_info(cfg: str) -> dict:
    from hachiue_b200 import workloads
    if cfg == "1":
        return dict(workload="cfg1 Qwen3-1.7B GQA decode attention", q_heads=16, kv_heads=8, head_dim=128,
                    context=1024, kv_dtype="f32", l2="rotates 32 cache copies (> L2)",
                    launch="device-resident warm-up and timed steps each run as one CUDA graph of the op calls; "
                           "e2e calls the API directly")
    if cfg in ("2", "2q8"):
        lens = workloads.cfg2_lens()
        return dict(workload="cfg2 Qwen3-8B batched GQA decode attention" + (" on a Q8_0 cache" if cfg == "2q8" else ""),
                    sequences=64, q_heads=32, kv_heads=8, head_dim=128,
                    kv_dtype="Q8_0 (int8 + f32 scale per 32, the reference's cache format)" if cfg == "2q8" else "f16",
                    context="U[512,8192] seed 1", sum_context=int(lens.sum()),
                    l2=("inputs (0.63 GB K/V) larger than L2" if cfg == "2q8" else "inputs (1.1 GB K/V) larger than L2"))
    if cfg == "3":
        return dict(workload="cfg3 PLaMo-3 sliding-window causal attention prefill", sequences=8, tokens=4096,
                    q_heads=16, kv_heads=4, head_dim=128, window=1024, io_dtype="bf16 in, bf16 out",
                    l2="inputs 201 MB > L2")
    if cfg == "4":
        return dict(workload="cfg4 Qwen3.5 Gated DeltaNet decode step", sequences=64, qk_heads=16, v_heads=32, d=128,
                    state="f32 [64,32,128,128]", l2="rotates 2 state copies (> L2)")
    if cfg == "5":
        return dict(workload="cfg5 Qwen3.5 Gated DeltaNet chunked prefill", sequences=8, tokens=8192, qk_heads=16,
                    v_heads=32, d=128, chunk=64, io_dtype="bf16 q/k/v, f32 g/beta, f32 out and final state",
                    l2="inputs 0.56 GB > L2")
    if cfg == "6":
        return dict(workload="cfg6 = cfg4 as a whole Qwen3.5 GDN layer step (conv1d K=4 + g/beta + recurrence + "
                             "gated RMSNorm, fused)", sequences=64, qk_heads=16, v_heads=32, d=128,
                    state="f32 [64,32,128,128] in place, conv state f32 [64,3,8192] ping-pong",
                    l2="rotates 2 state copies (> L2)")
    if cfg == "7":
        return dict(workload="cfg7 = cfg1 as a whole qwen3 attention layer step (q/k RMSNorm + RoPE + Q8_0 K/V "
                             "append + attention, fused prologue)", q_heads=16, kv_heads=8, head_dim=128,
                    context=1024, kv_dtype="Q8_0 (the reference's cache format)", l2="rotates 64 cache copies (> L2)",
                    launch="device-resident warm-up and timed steps (and the comparison arm's) each run as one CUDA "
                           "graph of the op calls; e2e calls the API directly")
    raise ValueError(cfg)


def metric_name(cfg: str) -> str:
    return {"1": "decode attn HBM GB/s", "2": "decode attn HBM GB/s", "2q8": "decode attn (Q8_0 cache) HBM GB/s",
            "3": "SWA prefill TFLOP/s", "4": "GDN decode HBM GB/s", "5": "GDN chunked prefill TFLOP/s",
            "6": "GDN layer step HBM GB/s", "7": "attention layer step HBM GB/s"}[cfg]


def metric_unit(cfg: str) -> str:
    return "TFLOP/s" if cfg in ("3", "5") else "GB/s"


def dtype_name(cfg: str) -> str:
    return {"1": "f32", "2": "f16", "2q8": "q8_0 cache, f32 math", "3": "bf16", "4": "f32", "5": "bf16",
            "6": "f32", "7": "q8_0 cache, f32 math"}[cfg]


# ---------------------------------------------------------------------------
# workloads (device side)
# ---------------------------------------------------------------------------
def _cfg2_device(torch, dev):
    """cfg2's inputs on the device: f16 K / V packed [sum T, 8, 128], q, the
    per-sequence positions and row offsets."""
    from hachiue_b200 import workloads
    w = workloads.decode_cfg2()
    return dict(w=w, k=torch.from_numpy(w["k"].view(np.int16)).to(dev).view(torch.float16),
                v=torch.from_numpy(w["v"].view(np.int16)).to(dev).view(torch.float16),
                q=torch.from_numpy(w["q"]).to(dev), pos=torch.from_numpy(w["pos_base"]).to(dev),
                off=torch.from_numpy(w["row_offset"]).to(dev), maxc=int(w["lens"].max()))


def _decode_e2e(torch, be, dev, cache, d, B=64, H=32, KV=8, Dh=128):
    """The user-facing decode step through the public API with host buffers:
    q and the step's new K / V rows (one per sequence, at its last position,
    already counted in its length) copied from pinned host memory, the rows
    appended in one launch, the attention over the whole context, and the
    output read back, pipelined over two slots (HostPipeline)."""
    from hachiue_b200.pipeline import HostPipeline
    w = d["w"]
    q_host = torch.from_numpy(w["q"]).pin_memory()
    kv_new_host = torch.from_numpy(
        np.random.default_rng(99).standard_normal((2, B, KV, Dh), dtype=np.float32)).pin_memory()
    out_host = torch.empty_like(q_host).pin_memory()
    last_rows = torch.from_numpy(w["row_offset"] + w["lens"] - 1).to(dev)
    pipe = HostPipeline(dev, [(tuple(q_host.shape), torch.float32), (tuple(kv_new_host.shape), torch.float32)],
                        [(tuple(out_host.shape), torch.float32)])

    def compute(ins, outs):
        be.kv_append_rows_kv(ins[1][0], ins[1][1], cache, last_rows)
        be.attention(ins[0], cache, outs[0], d["pos"], 0, kv_row_offset=d["off"], max_context=d["maxc"])

    def e2e_step(i):
        pipe.submit([q_host, kv_new_host], [out_host], compute)

    return dict(e2e_step=e2e_step, e2e_begin=pipe.begin, e2e_end=pipe.drain,
                h2d=q_host.numel() * 4 + kv_new_host.numel() * 4, d2h=out_host.numel() * 4, e2e_kernels_per_step=2,
                e2e_note="HostPipeline: two slots; step i+1's H2D and step i-1's D2H overlap step i's kernels")


def setup_cfg2(torch, be, dev, d=None):
    from hachiue_b200 import KV_F16, workloads
    from hachiue_b200.backend import KVCache
    d = d or _cfg2_device(torch, dev)
    cache = KVCache(KV_F16, d["k"], d["v"])
    outs = [torch.zeros_like(d["q"]) for _ in range(2)]  # step i writes outs[i % 2] (the gather reads it)

    def step(i):
        be.attention(d["q"], cache, outs[i & 1], d["pos"], 0, kv_row_offset=d["off"], max_context=d["maxc"])

    W = dict(step=step, bytes=workloads.cfg2_bytes(d["w"]["lens"]), tokens=64, info=config_info("2"),
             kernels_per_step=1, cpu=dict(w=d["w"], kind="cfg2"), outs=outs, traffic_key="cfg2", dev_inputs=d)
    W.update(_decode_e2e(torch, be, dev, cache, d))
    return W


def setup_cfg2q8(torch, be, dev, d=None):
    """cfg2's sequences, contexts and values on the reference's Q8_0 cache
    (appendKvQ8 of the same f16 values, done on the device)."""
    from hachiue_b200 import KV_Q8_0, workloads
    from hachiue_b200.backend import KVCache
    d = d or _cfg2_device(torch, dev)
    rows, KV, Dh = d["k"].shape
    cache = KVCache.allocate(rows, KV, Dh, KV_Q8_0, device=dev)
    for src, which in ((d["k"], "k"), (d["v"], "v")):
        be.kv_append(src.float(), cache, which, 0)
    torch.cuda.synchronize(dev)
    outs = [torch.zeros_like(d["q"]) for _ in range(2)]

    def step(i):
        be.attention(d["q"], cache, outs[i & 1], d["pos"], 0, kv_row_offset=d["off"], max_context=d["maxc"])

    W = dict(step=step, bytes=workloads.cfg2_q8_bytes(d["w"]["lens"]), tokens=64, info=config_info("2q8"),
             kernels_per_step=1, cpu=dict(w=d["w"], kind="cfg2q8", cache=cache), outs=outs, traffic_key="cfg2q8")
    W.update(_decode_e2e(torch, be, dev, cache, d))
    return W


def _pipelined_e2e(dev, host_in, host_out, compute):
    """End-to-end steps through the public API over HostPipeline: every step
    copies ``host_in`` (pinned) to the device, runs ``compute(i, device_inputs,
    device_outputs)`` and reads the outputs back into ``host_out`` (pinned),
    with step i+1's host-to-device copy and step i-1's device-to-host copy (the
    two PCIe directions) overlapping each other and step i's kernels."""
    from hachiue_b200.pipeline import HostPipeline
    pipe = HostPipeline(dev, [(tuple(x.shape), x.dtype) for x in host_in], [(tuple(x.shape), x.dtype) for x in host_out])

    def e2e_step(i):
        pipe.submit(host_in, host_out, lambda ins, outs: compute(i, ins, outs))

    return dict(e2e_step=e2e_step, e2e_begin=pipe.begin, e2e_end=pipe.drain,
                h2d=sum(x.numel() * x.element_size() for x in host_in),
                d2h=sum(x.numel() * x.element_size() for x in host_out),
                e2e_note="HostPipeline: two slots; step i+1's H2D and step i-1's D2H overlap step i's kernels")


def setup_cfg1(torch, be, dev):
    from hachiue_b200 import KV_F32, workloads
    from hachiue_b200.backend import KVCache
    w = workloads.decode_cfg1()
    copies = 32  # 32 x 8.4 MB > L2: each step reads a cold copy
    caches = [KVCache(KV_F32, torch.from_numpy(w["k"]).to(dev), torch.from_numpy(w["v"]).to(dev))
              for _ in range(copies)]
    q = torch.from_numpy(w["q"]).to(dev)
    out = torch.zeros_like(q)

    def step(i):
        be.attention(q, caches[i % copies], out, w["pos_base"])

    q_host = torch.from_numpy(w["q"]).pin_memory()
    out_host = torch.empty_like(q_host).pin_memory()
    q_dev = torch.empty_like(q)

    def e2e_step(i):
        q_dev.copy_(q_host, non_blocking=True)
        be.attention(q_dev, caches[i % copies], out, w["pos_base"])
        out_host.copy_(out, non_blocking=True)

    return dict(step=step, e2e_step=e2e_step, bytes=workloads.cfg1_bytes(), tokens=1, info=config_info("1"),
                h2d=q_host.numel() * 4, d2h=out_host.numel() * 4, kernels_per_step=1, e2e_kernels_per_step=1,
                cpu=dict(w=w, kind="cfg1"), out=out, traffic_key="cfg1", graph_period=copies)


def setup_cfg4(torch, be, dev):
    from hachiue_b200 import workloads
    w = workloads.gdn_decode_cfg4()
    NK, NV = w["NK"], w["NV"]
    copies = 2  # 2 x 268 MB of state > L2
    states = [torch.from_numpy(w["state"]).to(dev) for _ in range(copies)]
    qkv = torch.from_numpy(w["qkv"]).to(dev)
    a = torch.from_numpy(w["a"]).to(dev)
    b = torch.from_numpy(w["b"]).to(dev)
    an = torch.from_numpy(w["a_neg"]).to(dev)
    dtb = torch.from_numpy(w["dt_bias"]).to(dev)
    core = torch.zeros((64, 1, NV, 128), device=dev)

    def step(i):
        st = states[i % copies]
        be.deltanet_decode(qkv, a, b, an, dtb, st, core, st, NK, NV)

    hosts = [torch.from_numpy(w[k]).pin_memory() for k in ("qkv", "a", "b")]

    def compute(i, ins, outs):
        st = states[i % copies]
        be.deltanet_decode(ins[0], ins[1], ins[2], an, dtb, st, outs[0], st, NK, NV)

    W = dict(step=step, bytes=workloads.cfg4_bytes(), tokens=64, info=config_info("4"), kernels_per_step=1,
             e2e_kernels_per_step=1, cpu=dict(w=w, kind="cfg4"), out=core, traffic_key="cfg4")
    W.update(_pipelined_e2e(dev, hosts, [torch.empty(core.shape).pin_memory()], compute))
    return W


def setup_cfg3(torch, be, dev):
    from hachiue_b200 import workloads
    w = workloads.swa_cfg3()

    def bf(x):
        return torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).to(dev).view(torch.bfloat16)

    q, k, v = bf(w["q"]), bf(w["k"]), bf(w["v"])
    out = torch.empty((8, 4096, 16, 128), device=dev, dtype=torch.bfloat16)

    def step(i):
        be.swa_prefill(q, k, v, out, w["window"])

    hosts = [torch.from_numpy(np.ascontiguousarray(w[x]).view(np.int16)).pin_memory() for x in ("q", "k", "v")]
    out_h = torch.empty((8, 4096, 16, 128), dtype=torch.int16).pin_memory()

    def compute(i, ins, outs):
        qd, kd, vd = (x.view(torch.bfloat16) for x in ins)
        be.swa_prefill(qd, kd, vd, outs[0].view(torch.bfloat16), w["window"])

    W = dict(step=step, flops=workloads.swa_flops(), tokens=8 * 4096, info=config_info("3"), kernels_per_step=1,
             e2e_kernels_per_step=1, cpu=dict(w=w, kind="cfg3"), out=out, traffic_key="cfg3")
    W.update(_pipelined_e2e(dev, hosts, [out_h], compute))
    return W


# Prompt length of configuration 5 (8192 in the benchmark set; --cfg5-tokens
# shortens it for ncu captures of the same kernels on a smaller case).
CFG5_TOKENS = 8192


def setup_cfg5(torch, be, dev):
    from hachiue_b200 import workloads
    T = CFG5_TOKENS
    w = workloads.gdn_prefill_cfg5(T=T)

    def bf(x):
        return torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).to(dev).view(torch.bfloat16)

    q, k, v = bf(w["q"]), bf(w["k"]), bf(w["v"])
    g = torch.from_numpy(w["g"]).to(dev)
    beta = torch.from_numpy(w["beta"]).to(dev)
    core = torch.empty((8, T, 32, 128), device=dev)
    st = torch.empty((8, 32, 128, 128), device=dev)

    def step(i):
        be.deltanet_chunked_prefill(q, k, v, g, beta, core, st)

    hosts = [torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).pin_memory() for x in (w["q"], w["k"], w["v"])]
    hosts += [torch.from_numpy(w["g"]).pin_memory(), torch.from_numpy(w["beta"]).pin_memory()]

    def compute(i, ins, outs):
        qd, kd, vd = (x.view(torch.bfloat16) for x in ins[:3])
        be.deltanet_chunked_prefill(qd, kd, vd, ins[3], ins[4], outs[0], outs[1])

    info = config_info("5")
    if T != 8192:
        in_bytes = workloads.cfg5_bytes(T=T) - 8 * T * 32 * 128 * 4 - 8 * 32 * 128 * 128 * 4
        info.update(tokens=T, l2=f"inputs {in_bytes / 1e9:.2f} GB" + (" > L2" if in_bytes > 126e6 else ", within L2"))
    W = dict(step=step, flops=workloads.cfg5_flops(T=T), hbm_bytes=workloads.cfg5_bytes(T=T), tokens=8 * T,
             info=info, kernels_per_step=2, e2e_kernels_per_step=2, cpu=dict(w=w, kind="cfg5"), out=core,
             traffic_key="cfg5" if T == 8192 else None)
    W.update(_pipelined_e2e(dev, hosts, [torch.empty(core.shape).pin_memory(), torch.empty(st.shape).pin_memory()],
                            compute))
    return W


def setup_cfg6(torch, be, dev):
    """Configuration 4 as a whole GDN layer step (conv1d + g/beta + recurrence
    + gated RMSNorm in one kernel).  The unfused sequence of the reference's
    dispatches (conv1d_causal, the recurrence with g/beta fused, norm_gate:
    four launches) runs on the same inputs as the comparison arm."""
    from hachiue_b200 import workloads
    w = workloads.gdn_layer_cfg6()
    NK, NV, D = w["NK"], w["NV"], w["D"]
    B = w["qkv"].shape[0]
    copies = 2  # 2 x 268 MB of state > L2
    T = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    states = [T(w["state"]) for _ in range(copies)]
    conv = [T(w["conv_state"]), T(w["conv_state"])]  # ping-pong, as the engine
    qkv, conv_w, a, b, z, gamma = T(w["qkv"]), T(w["conv_w"]), T(w["a"]), T(w["b"]), T(w["z"]), T(w["gamma"])
    an, dtb = T(w["a_neg"]), T(w["dt_bias"])
    out = torch.zeros((B, NV * D), device=dev)
    qkv_conv = torch.zeros_like(qkv)
    core = torch.zeros((B, 1, NV, D), device=dev)

    def step(i):
        st = states[i % copies]
        be.gdn_layer_step(qkv, conv_w, conv[i & 1], conv[(i + 1) & 1], a, b, an, dtb, z, gamma, st, st, out, NK, NV,
                          w["eps"])

    def unfused(i):
        st = states[i % copies]
        be.conv1d_causal(qkv[:, None], conv_w, conv[i & 1], qkv_conv[:, None], conv[(i + 1) & 1])
        be.deltanet_decode(qkv_conv[:, None], a[:, None], b[:, None], an, dtb, st, core, st, NK, NV)
        be.deltanet_norm_gate(core, z, gamma, out, w["eps"])

    hosts = [torch.from_numpy(np.ascontiguousarray(w[k])).pin_memory() for k in ("qkv", "a", "b", "z")]

    def compute(i, ins, outs):
        st = states[i % copies]
        be.gdn_layer_step(ins[0], conv_w, conv[i & 1], conv[(i + 1) & 1], ins[1], ins[2], an, dtb, ins[3], gamma, st,
                          st, outs[0], NK, NV, w["eps"])

    info = config_info("6")
    W = dict(step=step, bytes=workloads.cfg6_bytes(), tokens=B, info=info, kernels_per_step=1, e2e_kernels_per_step=1,
             cpu=dict(w=w, kind="cfg6"), out=out, traffic_key="cfg6",
             alt=dict(name="unfused: conv1d_causal (2 kernels) + recurrence with g/beta + norm_gate",
                      step=unfused, kernels_per_step=4))
    W.update(_pipelined_e2e(dev, hosts, [torch.empty(out.shape).pin_memory()], compute))
    return W


def setup_cfg7(torch, be, dev):
    """Configuration 1 as a whole qwen3 attention layer step on the reference's
    Q8_0 cache: the fused prologue (q / k RMSNorm + RoPE + K / V append) and
    the attention, two launches.  The comparison arm is the engine's dispatch
    sequence (src/engine.ts:1419-1453) through the reference's op names:
    rmsnorm x2, rope x2, kv_append_q8 x2, attention_q8, seven launches."""
    from hachiue_b200 import KV_Q8_0, workloads
    from hachiue_b200.backend import KVCache, f32_word
    w = workloads.attn_layer_cfg7()
    H, KV, Dh, rot, pos, eps = w["H"], w["KV"], w["Dh"], w["rot"], w["pos"], w["eps"]
    T = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    half = rot // 2
    inv = 1.0 / np.power(w["theta"], 2.0 * np.arange(half) / rot)
    ang = np.arange(pos + 1)[:, None] * inv[None, :]
    cos, sin = T(np.cos(ang).astype(np.float32)), T(np.sin(ang).astype(np.float32))
    copies = 64  # 64 x 2.4 MB of cache > L2: each step reads a cold copy
    caches = [KVCache(KV_Q8_0, T(w["kq"]), T(w["vq"]), T(w["ks"]), T(w["vs"])) for _ in range(copies)]
    q, k, v, qn, kn = T(w["q"]), T(w["k"]), T(w["v"]), T(w["q_norm"]), T(w["k_norm"])
    q_out = torch.zeros_like(q)
    out = torch.zeros_like(q)
    qn_buf, kn_buf = torch.zeros_like(q), torch.zeros_like(k)

    def step(i):
        cache = caches[i % copies]
        be.attn_prologue(q, k, v, qn, kn, cos, sin, q_out, cache, pos, eps, rot)
        be.attention(q_out, cache, out, pos)

    def unfused(i):
        cache = caches[i % copies]
        be.dispatch("rmsnorm", [H, Dh, f32_word(eps), 0], [q, qn, qn_buf])
        be.dispatch("rmsnorm", [KV, Dh, f32_word(eps), 0], [k, kn, kn_buf])
        be.dispatch("rope", [1, H, Dh, rot, pos], [cos, sin, qn_buf])
        be.dispatch("rope", [1, KV, Dh, rot, pos], [cos, sin, kn_buf])
        be.dispatch("kv_append_q8", [1, KV, Dh, pos], [kn_buf, cache.k, cache.k_scale])
        be.dispatch("kv_append_q8", [1, KV, Dh, pos], [v, cache.v, cache.v_scale])
        be.dispatch("attention_q8", [1, H, KV, Dh, pos, 0], [qn_buf, cache.k, cache.k_scale, cache.v,
                                                             cache.v_scale, out])

    hs = {name: torch.from_numpy(np.ascontiguousarray(w[name])).pin_memory() for name in ("q", "k", "v")}
    dd = {name: torch.empty_like(t, device=dev) for name, t in hs.items()}
    out_h = torch.empty(out.shape).pin_memory()

    def e2e_step(i):
        for name in hs:
            dd[name].copy_(hs[name], non_blocking=True)
        cache = caches[i % copies]
        be.attn_prologue(dd["q"], dd["k"], dd["v"], qn, kn, cos, sin, q_out, cache, pos, eps, rot)
        be.attention(q_out, cache, out, pos)
        out_h.copy_(out, non_blocking=True)

    info = config_info("7")
    return dict(step=step, e2e_step=e2e_step, bytes=workloads.cfg7_bytes(), tokens=1, info=info,
                h2d=sum(t.numel() * 4 for t in hs.values()), d2h=out_h.numel() * 4, kernels_per_step=2,
                e2e_kernels_per_step=2, cpu=dict(w=w, kind="cfg7"), out=out, traffic_key="cfg7",
                alt=dict(name="unfused: the engine's dispatch sequence (rmsnorm x2, rope x2, kv_append_q8 x2, "
                              "attention_q8)", step=unfused, kernels_per_step=7), graph_period=copies)




SETUPS = {"1": setup_cfg1, "2": setup_cfg2, "2q8": setup_cfg2q8, "3": setup_cfg3, "4": setup_cfg4,
          "5": setup_cfg5, "6": setup_cfg6, "7": setup_cfg7}


# ---------------------------------------------------------------------------
# CPU baseline (the reference's algorithm on the host cores)
# ---------------------------------------------------------------------------
def cpu_sample(kind: str, w: dict, threads: int, budget_s: float = 12.0):
    """Times the oracle (JS-semantics C restatement) on a bounded sample of the
    workload; returns (GB/s, tokens/s, description)."""
    import oracle
    from hachiue_b200 import workloads
    if kind == "cfg2":
        lens = w["lens"]
        t0 = time.perf_counter()
        done_b, done_bytes, reps = 0, 0, 0
        k16, v16 = w["k"].view(np.uint16), w["v"].view(np.uint16)
        while time.perf_counter() - t0 < budget_s and reps < 4:
            oracle.attention_batch(w["q"], k16, v16, w["pos_base"], w["row_offset"], 0, oracle.KV_F16,
                                   threads=threads)
            done_b += 64
            done_bytes += workloads.cfg2_bytes(lens)
            reps += 1
        dt = time.perf_counter() - t0
        return done_bytes / dt / 1e9, done_b / dt, f"{reps} full passes of cfg2 (64 sequences, f16 KV) on {threads} threads", threads
    if kind == "cfg2q8":
        # The reference's own setting: runAttentionQ8 over a Q8_0 cache.  The
        # first sequences of cfg2 are quantised (appendKvQ8) and timed.
        nseq = w.get("_q8_nseq", 4)
        if "_q8" not in w:
            rows = int(w["lens"][:nseq].sum())
            kq, vq = np.zeros((rows, 8, 128), np.int8), np.zeros((rows, 8, 128), np.int8)
            ks, vs = np.zeros((rows, 8, 4), np.float32), np.zeros((rows, 8, 4), np.float32)
            oracle.append_kv_q8(w["k"][:rows].astype(np.float32), kq, ks, 0)
            oracle.append_kv_q8(w["v"][:rows].astype(np.float32), vq, vs, 0)
            w["_q8"] = (kq, ks, vq, vs)
        kq, ks, vq, vs = w["_q8"]
        lens = w["lens"][:nseq]
        t0 = time.perf_counter()
        reps = 0
        while True:
            oracle.attention_batch(np.ascontiguousarray(w["q"][:nseq]), kq, vq, w["pos_base"][:nseq],
                                   w["row_offset"][:nseq], 0, oracle.KV_Q8_0, ks, vs, threads=threads)
            reps += 1
            if time.perf_counter() - t0 > budget_s:
                break
        dt = time.perf_counter() - t0
        return (reps * workloads.cfg2_q8_bytes(lens) / dt / 1e9, reps * nseq / dt,
                f"{reps} passes over the first {nseq} sequences of cfg2 on a Q8_0 cache (appendKvQ8 of the same "
                f"values), {threads} thread(s)", threads)
    if kind == "cfg1":
        t0 = time.perf_counter()
        n = 0
        while time.perf_counter() - t0 < min(budget_s, 5.0):
            oracle.attention(w["q"], w["k"], w["v"], w["pos_base"])
            n += 1
        dt = time.perf_counter() - t0
        return n * workloads.cfg1_bytes() / dt / 1e9, n / dt, f"{n} cfg1 calls, 1 thread", 1
    if kind == "cfg4":
        B = 16
        gb = np.stack([oracle.deltanet_gbeta(w["a"][b], w["b"][b], w["a_neg"], w["dt_bias"]) for b in range(B)])
        t0 = time.perf_counter()
        oracle.deltanet_recur_batch(w["qkv"][:B], gb, w["state"][:B], w["NK"], w["NV"], True, threads=threads)
        dt = time.perf_counter() - t0
        return workloads.cfg4_bytes(B=B) / dt / 1e9, B / dt, f"{B} of 64 sequences of cfg4 on {threads} threads", threads
    if kind == "cfg6":
        B = 8
        t0 = time.perf_counter()
        oracle.gdn_layer_step(w["qkv"][:B], w["conv_w"], w["conv_state"][:B], w["a"][:B], w["b"][:B], w["a_neg"],
                              w["dt_bias"], w["z"][:B], w["gamma"], w["eps"], w["state"][:B], w["NK"], w["NV"], True)
        dt = time.perf_counter() - t0
        return workloads.cfg6_bytes(B=B) / dt / 1e9, B / dt, f"{B} of 64 sequences of cfg6, 1 thread", 1
    if kind == "cfg7":
        cos, sin = oracle.rope_tables(w["rot"], w["pos"] + 1, w["theta"])
        t0 = time.perf_counter()
        n = 0
        while time.perf_counter() - t0 < min(budget_s, 5.0):
            kq, ks, vq, vs = w["kq"].copy(), w["ks"].copy(), w["vq"].copy(), w["vs"].copy()
            oracle.attn_layer_step(w["q"], w["k"], w["v"], w["q_norm"], w["k_norm"], w["eps"], cos, sin, w["rot"],
                                   w["pos"], kq, ks, vq, vs)
            n += 1
        dt = time.perf_counter() - t0
        return n * workloads.cfg7_bytes() / dt / 1e9, n / dt, f"{n} cfg7 layer steps, 1 thread", 1
    if kind == "cfg3":
        from hachiue_b200 import workloads as wl
        qs, qe = 3000, 3064
        q = np.ascontiguousarray(wl.bf16_bits_to_f32(w["q"][0, qs:qe]))
        t0 = time.perf_counter()
        n = 0
        while True:
            oracle.attention(q, np.ascontiguousarray(w["k"][0]), np.ascontiguousarray(w["v"][0]), qs, w["window"],
                             oracle.KV_BF16)
            n += 1
            if time.perf_counter() - t0 > min(budget_s, 4.0):
                break
        dt = time.perf_counter() - t0
        flops = n * 4 * 128 * (qe - qs) * 16 * w["window"]
        return flops / dt / 1e12, n * (qe - qs) / dt, f"{n} x 64 queries x 16 heads of cfg3 sequence 0, 1 thread", 1
    if kind == "cfg5":
        from hachiue_b200 import workloads as wl
        T = 2048
        f = wl.bf16_bits_to_f32
        qkv = np.concatenate([f(w["q"][0, :T, 0]), f(w["k"][0, :T, 0]), f(w["v"][0, :T, 0])], 1).astype(np.float32)
        gb = np.stack([w["g"][0, :T, 0:1], w["beta"][0, :T, 0:1]]).astype(np.float32)
        t0 = time.perf_counter()
        n = 0
        while True:
            oracle.deltanet_recur(qkv, gb, np.zeros((1, 128, 128), np.float32), 1, 1, False)
            n += 1
            if time.perf_counter() - t0 > min(budget_s, 4.0):
                break
        dt = time.perf_counter() - t0
        flops = n * T * (10 * 64 * 128 + 6 * 128 * 128)
        return flops / dt / 1e12, n * T / dt, f"{n} x {T} tokens of one (sequence, head) of cfg5, 1 thread", 1
    raise ValueError(kind)


def run_reference(args, world, rank):
    """--impl reference: the reference's algorithm (its JS-semantics C
    restatement, oracle/) on the host cores, on the same workload and config
    as the GPU arm, plus the reference's own setting (one thread over a Q8_0
    cache) for the decode configurations."""
    if rank != 0:
        return 0
    from hachiue_b200 import workloads
    threads = os.cpu_count() or 1
    loaders = {"1": workloads.decode_cfg1, "2": workloads.decode_cfg2, "2q8": workloads.decode_cfg2,
               "3": workloads.swa_cfg3, "4": workloads.gdn_decode_cfg4, "5": workloads.gdn_prefill_cfg5,
               "6": workloads.gdn_layer_cfg6, "7": workloads.attn_layer_cfg7}
    w = loaders[args.config]()
    kind = "cfg" + args.config
    for _ in range(args.warmup):
        cpu_sample(kind, w, threads, budget_s=0.5)
    vals = []
    t_all = time.perf_counter()
    desc = ""
    cores = threads
    for _ in range(args.steps):
        v, _, desc, cores = cpu_sample(kind, w, threads, budget_s=2.0)
        vals.append(v)
    elapsed = time.perf_counter() - t_all
    value = statistics.median(vals)
    unit = metric_unit(args.config)
    line = {
        "impl": "reference", "metric": metric_name(args.config), "value": round(value, 4), "unit": unit,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1000 * elapsed / max(args.steps, 1), 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": dtype_name(args.config), "data": DATA,
        "config": config_info(args.config), "parallelism": f"{cores} host threads",
        "cpu_baseline": {"value": round(value, 4), "unit": unit, "cores": cores, "kind": "port",
                         "sample": desc + "; the reference is TypeScript with no runtime on this box, so its "
                                          "JS-semantics C restatement (oracle/) is timed"},
        "e2e": {"value": round(value, 4), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if args.config in ("1", "2"):
        # the reference's own setting: runAttentionQ8 is single-threaded JS over
        # the engine's Q8_0 cache (src/wasm-backend.ts:826-895)
        if args.config == "2":
            v1, _, d1, c1 = cpu_sample("cfg2q8", w, 1, budget_s=4.0)
            unit1 = "GB/s (Q8_0 algorithmic bytes)"
        else:
            v1, _, d1, c1 = cpu_sample("cfg1", w, 1, budget_s=3.0)
            unit1 = unit
        line["reference_setting"] = {"value": round(v1, 4), "unit": unit1, "cores": c1, "kind": "port",
                                     "sample": d1 + " (the reference's own setting: one JS thread"
                                     + (", Q8_0 KV cache)" if args.config == "2" else ")")}
    print(json.dumps(line), flush=True)
    return 0


DATA = "synthetic (seeded numpy PCG64, benchmark-config shapes)"


# ---------------------------------------------------------------------------
# measurement
# ---------------------------------------------------------------------------
def measure(torch, dist, W, args, world, dev, clocks, gather=None):
    """Times W's device-resident step (``value``: CUDA events around the
    whole timed region, and around each step's kernels for the roofline),
    then its end-to-end step, then its comparison arm.  Returns the times."""
    stream = torch.cuda.current_stream(dev)
    graph_mode = bool(W.get("graph_period")) and world == 1
    gather = gather or (lambda i, out: None)

    def out_of(i):
        return W["outs"][i & 1] if "outs" in W else W["out"]

    def capture(fn, n):
        for i in range(min(n, W["graph_period"])):  # every input variant once, outside capture
            fn(i)
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(n):
                fn(i)
        return g

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(ms):
        if world == 1:
            return ms
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident ----
    if graph_mode:
        g_warm, g_timed = capture(W["step"], args.warmup), capture(W["step"], args.steps)
        g_warm.replay()
    else:
        for i in range(args.warmup):
            W["step"](i)
            gather(i, out_of(i))
    gather(None, None)  # drain
    barrier()
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t0e, t1e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    c0 = time.perf_counter()
    t0e.record(stream)
    if graph_mode:
        g_timed.replay()
    else:
        for i in range(args.steps):
            kev[i][0].record(stream)
            W["step"](i)
            kev[i][1].record(stream)
            gather(i, out_of(i))
    gather(None, None)
    t1e.record(stream)
    barrier()
    c1 = time.perf_counter()
    total_ms = max_over_ranks(t0e.elapsed_time(t1e))
    kernel_ms = (t0e.elapsed_time(t1e) / args.steps if graph_mode
                 else statistics.mean(a.elapsed_time(b) for a, b in kev))
    clk = clocks.summary(c0, c1) if clocks else None

    # ---- end to end through the public API (host buffers) ----
    begin, end = W.get("e2e_begin", lambda: None), W.get("e2e_end", lambda: None)
    begin()
    for i in range(args.warmup):
        W["e2e_step"](i)
    end()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c2 = time.perf_counter()
    e0.record(stream)
    begin()
    for i in range(args.steps):
        W["e2e_step"](i)
    end()
    e1.record(stream)
    barrier()
    c3 = time.perf_counter()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    clk_e2e = clocks.summary(c2, c3) if clocks else None

    # ---- comparison arm of the same workload (device-resident, as `value`) ----
    alt = None
    if "alt" in W:
        if graph_mode:
            ga_warm, ga_timed = capture(W["alt"]["step"], args.warmup), capture(W["alt"]["step"], args.steps)
            ga_warm.replay()
        else:
            for i in range(args.warmup):
                W["alt"]["step"](i)
        barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        if graph_mode:
            ga_timed.replay()
        else:
            for i in range(args.steps):
                W["alt"]["step"](i)
        a1.record(stream)
        barrier()
        alt = {"name": W["alt"]["name"], "ms_per_step": round(a0.elapsed_time(a1) / args.steps, 5),
               "gpu_launches_per_step": W["alt"]["kernels_per_step"]}
    return dict(total_ms=total_ms, kernel_ms=kernel_ms, e2e_ms=e2e_ms, alt=alt, clocks=clk, clocks_e2e=clk_e2e)


def entry(cfg, W, res, peaks, peak_src, world, steps, cpu):
    """One configuration's measurement as a JSON object (the headline line's
    fields, or a ``secondary`` entry)."""
    tensor = "flops" in W
    work = W["flops"] if tensor else W["bytes"]
    scale = 1e12 if tensor else 1e9  # TFLOP/s or GB/s
    unit = metric_unit(cfg)
    ms = res["total_ms"] / steps
    value = world * work / (ms / 1e3) / scale
    kms = res["kernel_ms"]
    achieved = work / (kms / 1e3) / scale
    peak = peaks["bf16_tflops"] if tensor else peaks["hbm_gbs"]
    roof = {"bound": "tensor" if tensor else "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": unit,
            "frac": round(achieved / peak, 4), "peak_source": peak_src + (" bf16 burst" if tensor else " copy"),
            ("algorithmic_flops_per_launch" if tensor else "algorithmic_bytes_per_launch"): work,
            "kernel_ms": round(kms, 5), "traffic": load_traffic(W["traffic_key"]) if W["traffic_key"] else None}
    if "hbm_bytes" in W:  # tensor work at I/O dtypes whose bytes take longer than its flops: the HBM roof binds
        gbs = W["hbm_bytes"] / (kms / 1e3) / 1e9
        roof = {"bound": "hbm", "achieved": round(gbs, 2), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(gbs / peaks["hbm_gbs"], 4), "peak_source": peak_src + " copy",
                "algorithmic_bytes_per_launch": W["hbm_bytes"], "kernel_ms": round(kms, 5),
                "traffic": load_traffic(W["traffic_key"]) if W["traffic_key"] else None,
                "tensor_achieved_tflops": round(achieved, 2),
                "tensor_frac": round(achieved / peaks["bf16_tflops"], 4)}
    e2e_ms = res["e2e_ms"] / steps
    d = {"metric": metric_name(cfg), "value": round(value, 2), "unit": unit, "ms_per_step": round(ms, 5),
         "dtype": dtype_name(cfg), "config": W["info"],
         "tokens_per_s": round(world * W["tokens"] / (ms / 1e3), 1), "roofline": roof,
         "e2e": {"value": round(world * work / (e2e_ms / 1e3) / scale, 2), "unit": unit,
                 "h2d_bytes_per_step": W["h2d"], "d2h_bytes_per_step": W["d2h"], "ms_per_step": round(e2e_ms, 5),
                 "clocks": res["clocks_e2e"]},
         "gpu_launches": steps * W["kernels_per_step"], "e2e_gpu_launches": steps * W["e2e_kernels_per_step"],
         "clocks": res["clocks"], "cpu_baseline": cpu}
    if "e2e_note" in W:
        d["e2e"]["pipelining"] = W["e2e_note"]
    if res["alt"] is not None:
        alt = dict(res["alt"])
        alt["value"] = round(world * work / (alt["ms_per_step"] / 1e3) / scale, 2)
        alt["unit"] = unit
        d["comparison"] = alt
    return d


def cpu_entry(cfg, W, budget_s):
    threads = os.cpu_count() or 1
    v, _, desc, cores = cpu_sample(W["cpu"]["kind"], W["cpu"]["w"], threads, budget_s=budget_s)
    return {"value": round(v, 4), "unit": metric_unit(cfg), "cores": cores, "kind": "port",
            "sample": desc + " (the reference is TypeScript with no runtime here; its JS-semantics C restatement in "
                             "oracle/ is timed)"}


def strong_scaling(torch, dist, be, comm, comm_bulk, args, world, rank, dev, W2):
    """One configuration's fixed work split over the job's GPUs: cfg2 by KV
    head (reusing the headline's device inputs) and cfg5 by QK head.  Each
    step is the local kernels plus the all-gather of the per-head outputs
    (hcu_allgather); both are timed with CUDA events, max over ranks."""
    from hachiue_b200 import KV_F16, workloads
    from hachiue_b200 import dist as hdist
    from hachiue_b200.backend import KVCache
    stream = torch.cuda.current_stream(dev)

    def run(step, n_warm, n_steps):
        for _ in range(n_warm):
            step()
        dist.barrier()
        torch.cuda.synchronize(dev)
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(n_steps)]
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for e in ev:
            step(e)
        t1.record(stream)
        dist.barrier()
        torch.cuda.synchronize(dev)
        t = torch.tensor([t0.elapsed_time(t1) / n_steps, statistics.mean(a.elapsed_time(b) for a, b, _ in ev),
                          statistics.mean(b.elapsed_time(c) for _, b, c in ev)], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return [float(x) for x in t.tolist()]

    out = {}
    # cfg2 by KV head: KV heads [lo, hi) of all 64 sequences and their G query heads
    d = W2["dev_inputs"]
    lo, hi = hdist.kv_head_range(8, world, rank)
    G = 32 // 8
    cache = KVCache(KV_F16, d["k"][:, lo:hi].contiguous(), d["v"][:, lo:hi].contiguous())
    q_l = d["q"][:, :, lo * G:hi * G].contiguous()
    out_l = torch.empty_like(q_l)
    recv = torch.empty((world,) + tuple(out_l.shape), device=dev)

    def step2(ev=None):
        if ev:
            ev[0].record(stream)
        be.attention(q_l, cache, out_l, d["pos"], 0, kv_row_offset=d["off"], max_context=d["maxc"])
        if ev:
            ev[1].record(stream)
        comm_bulk.all_gather(out_l, recv)  # in line with the step: NCCL's full channel count
        if ev:
            ev[2].record(stream)

    ms, attn_ms, gather_ms = run(step2, args.warmup, args.steps)
    nbytes = workloads.cfg2_bytes(d["w"]["lens"])
    out["cfg2_by_kv_head"] = {
        "ms_per_step": round(ms, 5), "value": round(nbytes / (ms / 1e3) / 1e9, 2), "unit": "GB/s",
        "work": "one cfg2 step (64 sequences) in total, split over the ranks", "kv_heads_per_rank": hi - lo,
        "attention_ms": round(attn_ms, 5), "gather_ms": round(gather_ms, 5),
        "gather_share": round(gather_ms / ms, 4), "gather_bytes_per_rank": out_l.numel() * 4,
        "limiter": "all-gather latency" if gather_ms > attn_ms else "attention (HBM)"}
    del cache, q_l, out_l, recv

    # cfg5 by QK head: QK heads [lo, hi) and V heads {h : h % 16 in [lo, hi)}
    w = workloads.gdn_prefill_cfg5()
    ex = hdist.QKHeadShardedGDN(be, 16, 32)
    cpu = [torch.from_numpy(np.ascontiguousarray(w[n]).view(np.int16)).view(torch.bfloat16) for n in ("q", "k", "v")]
    cpu += [torch.from_numpy(w["g"]), torch.from_numpy(w["beta"])]
    ql, kl, vl, gl, bl = (x.to(dev) for x in ex.shard_prefill(*cpu))
    del cpu, w
    core_l = torch.empty((8, 8192, ex.nvl, 128), device=dev)
    st_l = torch.empty((8, ex.nvl, 128, 128), device=dev)
    recv5 = torch.empty((world,) + tuple(core_l.shape), device=dev)

    def step5(ev=None):
        if ev:
            ev[0].record(stream)
        be.deltanet_chunked_prefill(ql, kl, vl, gl, bl, core_l, st_l)
        if ev:
            ev[1].record(stream)
        comm_bulk.all_gather(core_l, recv5)
        if ev:
            ev[2].record(stream)

    ms, pre_ms, gather_ms = run(step5, 3, min(args.steps, 10))
    out["cfg5_by_qk_head"] = {
        "ms_per_step": round(ms, 5), "value": round(workloads.cfg5_flops() / (ms / 1e3) / 1e12, 2),
        "unit": "TFLOP/s", "work": "one cfg5 prefill (8 x 8192 tokens) in total, split over the ranks",
        "qk_heads_per_rank": ex.nkl, "v_heads_per_rank": ex.nvl, "prefill_ms": round(pre_ms, 5),
        "gather_ms": round(gather_ms, 5), "gather_share": round(gather_ms / ms, 4),
        "gather_bytes_per_rank": core_l.numel() * 4,
        "limiter": "all-gather of the f32 outputs over NVLink" if gather_ms > pre_ms else "prefill kernels"}
    return out


# ---------------------------------------------------------------------------
def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="2", choices=sorted(SETUPS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--cfg5-tokens", type=int, default=8192,
                    help="prompt length of configuration 5 (a multiple of 64; shorter only for profiling captures)")
    args = ap.parse_args(argv)
    global CFG5_TOKENS
    if args.cfg5_tokens != 8192 and (args.cfg5_tokens < 64 or args.cfg5_tokens % 64):
        ap.error("--cfg5-tokens must be a positive multiple of 64")
    CFG5_TOKENS = args.cfg5_tokens
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_setup(args)
    if args.impl == "reference":
        return run_reference(args, world, rank)

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    comm = None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
        from hachiue_b200.dist import RankComm
        comm = RankComm(local, max_ctas=4)  # per-step gathers of about 1 MB that overlap the next step
        comm_bulk = RankComm(local)  # the strong-scaling gathers of whole outputs

    from hachiue_b200 import CudaBackend
    be = CudaBackend(local)
    peaks, peak_src = load_peaks()
    clocks = ClockSampler(local)
    clocks.start()
    clocks.wait_ready()

    W = SETUPS[args.config](torch, be, dev)

    # Multi-GPU: each step's output is all-gathered (hcu_allgather) on a side
    # stream while the next step computes; a step's output buffer is reused
    # two steps later, after its gather.
    gather = None
    if world > 1:
        gstream = torch.cuda.Stream(dev)
        recv = [torch.empty((world,) + tuple((W["outs"][0] if "outs" in W else W["out"]).shape), device=dev,
                            dtype=(W["outs"][0] if "outs" in W else W["out"]).dtype) for _ in range(2)]
        stage = None if "outs" in W else [torch.empty_like(W["out"]) for _ in range(2)]
        done = [None, None]

        def gather(i, out):
            cur = torch.cuda.current_stream(dev)
            if i is None:  # drain
                for j in range(2):
                    if done[j] is not None:
                        cur.wait_event(done[j])
                        done[j] = None
                return
            j = i & 1
            if done[j] is not None:
                cur.wait_event(done[j])
            src = out
            if stage is not None:
                stage[j].copy_(out)
                src = stage[j]
            ready = torch.cuda.Event()
            ready.record(cur)
            gstream.wait_event(ready)
            with torch.cuda.stream(gstream):
                comm.all_gather(src, recv[j])
                done[j] = torch.cuda.Event()
                done[j].record(gstream)

    res = measure(torch, dist, W, args, world, dev, clocks, gather)
    status = be.device_status()
    if status:
        raise RuntimeError(f"device status {status} after the timed region")
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_entry(args.config, W, 12.0)
    head = entry(args.config, W, res, peaks, peak_src, world, args.steps, cpu)

    line = {"metric": head.pop("metric"), "value": head.pop("value"), "unit": head.pop("unit"), "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": head.pop("ms_per_step"),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": head.pop("dtype"),
            "data": DATA, "config": head.pop("config"),
            "parallelism": (f"dp{world}: each rank its own batch; per-head outputs all-gathered over NCCL "
                            "(hcu_allgather) overlapped with the next step" if world > 1 else "single GPU")}
    line.update(head)

    if world > 1:
        line["strong"] = (strong_scaling(torch, dist, be, comm, comm_bulk, args, world, rank, dev, W)
                          if args.config == "2" else None)
    del W
    torch.cuda.empty_cache()

    if world == 1 and args.config == "2" and not args.no_secondary:
        sec = {}
        for cfg in ("2q8", "1", "3", "4", "5"):
            Ws = SETUPS[cfg](torch, be, dev)
            r = measure(torch, dist, Ws, args, 1, dev, clocks)
            st = be.device_status()
            if st:
                raise RuntimeError(f"device status {st} after cfg{cfg}")
            c = None if args.no_cpu_baseline else cpu_entry(cfg, Ws, 3.0)
            sec["cfg" + cfg.replace("2q8", "2_q8")] = entry(cfg, Ws, r, peaks, peak_src, 1, args.steps, c)
            del Ws
            torch.cuda.empty_cache()
        line["secondary"] = sec
    clocks.stop()
    if rank == 0:
        print(json.dumps(line), flush=True)
    be.close()
    if world > 1:
        comm.close()
        comm_bulk.close()
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
