#!/usr/bin/env python
"""Benchmark of the B200 NPL backend on its headline workload.

Workload (one "step"): npl_conv2d_bn_activation on the ResNet-style 3x3 layer
N=32, C_in=64, H=W=56, C_out=64, stride 1, pad 1, no bias, inference BN
(gamma U[0.5,1.5], beta U[-0.1,0.1], mean N(0,0.1), var U[0.5,1.5], eps 1e-5),
ReLU; input U[0,1], weights N(0, sqrt(2/576)). Synthetic seeded inputs.
A step is the full operator: weight preparation (tf32 split + BN constants)
and the fused implicit-GEMM conv kernel the library picks for the geometry
(for this 3x3 stride-1 layer: shared im2col windows gathered from NCHW x,
two MMA pipelines per CTA). At N GPUs every rank runs its own
batch of 32 (batch-sharded data parallelism, no collective): weak scaling.

Reported (one JSON line on rank 0):
  value     whole-job TFLOP/s (2*N*Cout*Cin*Ho*Wo*9 per batch) with inputs
            resident in HBM, timed with CUDA events per step, L2 flushed
            between steps outside the timed events, max over ranks;
  e2e       the same metric through the public C ABI with pinned host
            buffers (host->device input copies and device->host output copy
            inside every step);
  roofline  the conv kernel against the 3xTF32 tensor-core roofline derived
            from the measured dense bf16 peak (TF32 runs at half the bf16
            rate and 3xTF32 issues three TF32 products per output product);
  cpu_baseline  the reference's own CPU code (oracle/_ref, built from the
            reference sources) on the same workload, all host threads;
  also      the other workloads on the GPU -- the large fp32 GEMM
            [8192x4096]@[4096x16384] (+bias via beta=1, then ReLU and layer
            norm), the 1024^3 GEMM, the 7x7/s2 stem conv + max pool, the
            bandwidth kernels and their depthwise->BN->ReLU->GAP->softmax
            chain -- and (cpu_reference_rows) the reference's CPU code on
            bounded samples of the same workloads, scaled to full size.

--impl reference runs only the reference CPU arm on the same workload.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "project-jcore_b200"))
import npl_b200 as nb  # noqa: E402
from npl_b200 import workloads  # noqa: E402

N_IMG, C_IN, HW_IN, C_OUT, KSZ = 32, 64, 56, 64, 3
CONV_FLOPS = 2.0 * N_IMG * C_OUT * C_IN * HW_IN * HW_IN * KSZ * KSZ
GEMM_M, GEMM_K, GEMM_N = 8192, 4096, 16384
GEMM_FLOPS = 2.0 * GEMM_M * GEMM_K * GEMM_N
WORKLOAD = ("npl_conv2d_bn_activation fp32 NCHW 3x3 s1 p1: N=32 C_in=64 56x56 C_out=64, "
            "inference BN + ReLU")


def conv_inputs(seed: int = 0):
    rng = np.random.default_rng(seed)
    x = rng.uniform(0, 1, (N_IMG, C_IN, HW_IN, HW_IN)).astype(np.float32)
    w = rng.normal(0, np.sqrt(2 / (9 * C_IN)), (C_OUT, C_IN, KSZ, KSZ)).astype(np.float32)
    gamma = rng.uniform(0.5, 1.5, C_OUT).astype(np.float32)
    beta = rng.uniform(-0.1, 0.1, C_OUT).astype(np.float32)
    mean = rng.normal(0, 0.1, C_OUT).astype(np.float32)
    var = rng.uniform(0.5, 1.5, C_OUT).astype(np.float32)
    return x, w, gamma, beta, mean, var


def make_l2_flush(dev):
    """L2 flush run between timed launches, outside the timed events: a
    256 MiB write (evicts every line of the working set) followed by a
    256 MiB read, whose clean lines replace the dirty ones the write left,
    so their write-back to HBM does not land in the next timed kernel."""
    import torch
    wbuf = torch.empty(64 * 1024 * 1024, device=dev)  # 256 MiB > 126 MB L2
    rbuf = torch.zeros(64 * 1024 * 1024, device=dev)
    acc = torch.empty((), device=dev)

    def flush():
        wbuf.zero_()
        torch.sum(rbuf, dim=0, out=acc)

    return flush


def measured_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle sampling while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.file = None
        # The NVML poll runs from construction on (its first samples take a
        # few milliseconds, longer than the timed region); start() marks the
        # window whose samples are reported.
        self.nvml = NvmlClockPoller(device_index)
        self.nvml.start()

    def start(self):
        self.nvml.mark()
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.dev), "-lms", "200"], stdout=self.file,
                stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        fine = self.nvml.stop()
        if not self.proc:
            return fine
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        rows = [r.split(",") for r in self.file.read().strip().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sm, reasons, mx = [], set(), None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [v.strip() for v in r]
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
            except ValueError:
                continue
            for name, flag in zip(names, r[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sm:
            return fine
        out = {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
               "samples": len(sm), "source": "nvidia-smi -lms 200"}
        if fine and fine["samples"] >= len(sm):
            # The timed region is only milliseconds long: the NVML poll sees
            # it at sub-millisecond intervals, nvidia-smi at most once or twice.
            out.update({"sm_mhz": fine["sm_mhz"], "sm_mhz_min": fine["sm_mhz_min"],
                        "samples": fine["samples"], "source": fine["source"],
                        "reasons": sorted(set(out["reasons"]) | set(fine["reasons"])),
                        "nvidia_smi": {"sm_mhz": statistics.median(sm), "samples": len(sm)}})
            if fine.get("sm_max_mhz"):
                out["sm_max_mhz"] = fine["sm_max_mhz"]
        return out


class NvmlClockPoller:
    """Reads the SM clock and the active clock-event (throttle) reasons through
    NVML in a background thread every ~0.5 ms while the timed region runs.
    Read-only: it changes no clock or other setting. The device is found by
    the PCI bus id torch reports for `device_index`."""

    # NVML clock-event reason bits (nvmlClocksEventReason*)
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device_index: int, interval_s: float = 0.0002):
        self.dev = device_index
        self.interval = interval_s
        self.thread = None
        self.samples = []  # (perf_counter time, MHz, reason bits)
        self.stop_flag = False
        self.handle = None
        self.max_mhz = None
        self.window = None

    def _open(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        pr = torch.cuda.get_device_properties(self.dev)
        try:
            bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except (AttributeError, pynvml.NVMLError):
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(self.dev)
        self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        return pynvml

    def start(self):
        import threading
        try:
            nv = self._open()
        except Exception:  # no NVML (or no device): nvidia-smi alone records clocks
            self.handle = None
            return

        def poll():
            get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            while not self.stop_flag:
                try:
                    mhz = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
                    rs = get_reasons(self.handle)
                except Exception:
                    break
                self.samples.append((time.perf_counter(), mhz, rs))
                time.sleep(self.interval)

        self.stop_flag = False
        # The timed region lasts milliseconds while the launching thread holds
        # the interpreter lock between its calls; a short switch interval lets
        # this thread take its samples meanwhile (restored in stop()).
        self.saved_switch = sys.getswitchinterval()
        sys.setswitchinterval(0.0001)
        self.thread = threading.Thread(target=poll, daemon=True)
        self.thread.start()

    def mark(self):
        """Start of the timed region: samples before it are not reported."""
        self.window = time.perf_counter()

    def stop(self):
        if self.thread is None:
            return None
        t_end = time.perf_counter()
        self.stop_flag = True
        self.thread.join(timeout=5)
        sys.setswitchinterval(self.saved_switch)
        t_start = self.window if self.window is not None else 0.0
        inside = [(m, rs) for t, m, rs in self.samples if t_start <= t <= t_end]
        if not inside:
            return None
        mhz = [m for m, _ in inside]
        reasons = set()
        for _, rs in inside:
            for bit, name in self.REASONS.items():
                if rs & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(mhz), "sm_mhz_min": min(mhz),
                "sm_max_mhz": self.max_mhz, "reasons": sorted(reasons),
                "samples": len(mhz), "source": "NVML poll every ~0.2 ms during the timed region"}


# ---------------------------------------------------------------------------
# reference CPU arm
# ---------------------------------------------------------------------------
def reference_cpu(steps: int, warmup: int, rows: bool = False):
    """Times the reference's own CPU implementation of the step (its
    npl_conv2d_bn_activation -- which runs the conv only -- followed by its
    npl_batch_norm and npl_relu) with all host threads. Returns
    (TFLOP/s, cores, sample, median seconds, rows) where rows (with
    rows=True) holds the reference's times on bounded samples of the other
    workloads (_reference_cpu_rows)."""
    ref_lib = REPO / "oracle" / "_ref" / "libnpl_ref.so"
    if not ref_lib.exists():
        return None
    sys.stdout.flush()
    devnull = os.open(os.devnull, os.O_WRONLY)
    saved = os.dup(1)
    os.dup2(devnull, 1)  # the reference prints on init and on every activation call
    try:
        return _reference_cpu_timed(ref_lib, steps, warmup, rows)
    finally:
        sys.stdout.flush()
        os.dup2(saved, 1)
        os.close(devnull)
        os.close(saved)


def _reference_cpu_rows(lib, cores):
    """The reference's CPU code on the other workloads, each on a bounded
    sample (median of 3 calls after one warm-up), scaled to the full workload
    by the sample's share of it: the 1024^3 GEMM in full; the stem on 2 of 128
    images (its conv -- conv only -- then its batch norm, ReLU and 3x3/s2 max
    pool); the depthwise -> BN -> ReLU -> GAP -> softmax chain on 16 of 256
    images; the 8192x4096x16384 GEMM (+ bias via beta=1) with ReLU and layer
    norm on 512 of 8192 rows."""
    rng = np.random.default_rng(0)
    keep = []

    def T(a):
        keep.append(a)
        return nb.tensor(lib, a.ctypes.data, a.shape)

    def timed(fn, reps=3):
        fn()
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return statistics.median(ts)

    def ok(rc):
        assert rc == 0, rc

    out = {}
    f32 = np.float32
    # d1: 1024^3
    a = rng.uniform(-1, 1, (1024, 1024)).astype(f32)
    b = rng.uniform(-1, 1, (1024, 1024)).astype(f32)
    ta, tb, tc = T(a), T(b), T(np.zeros((1024, 1024), f32))
    sec = timed(lambda: ok(lib.npl_matmul(C.byref(ta), C.byref(tb), C.byref(tc), C.c_float(1.0),
                                          C.c_float(0.0), None)))
    out["gemm_1024"] = {"us": round(sec * 1e6, 1), "TFLOP/s": round(2 * 1024 ** 3 / sec / 1e12, 5),
                        "sample": "full workload"}
    # d3: stem on 2 of 128 images
    ns = 2
    x = rng.uniform(-1, 1, (ns, 3, 224, 224)).astype(f32)
    w = rng.normal(0, np.sqrt(2 / 147), (64, 3, 7, 7)).astype(f32)
    g, be = rng.uniform(0.5, 1.5, 64).astype(f32), rng.uniform(-0.1, 0.1, 64).astype(f32)
    mu, va = rng.normal(0, 0.1, 64).astype(f32), rng.uniform(0.5, 1.5, 64).astype(f32)
    keep.extend([g, be, mu, va])
    tx, tw = T(x), T(w)
    tconv, tbn = T(np.zeros((ns, 64, 112, 112), f32)), T(np.zeros((ns, 64, 112, 112), f32))
    tpool = T(np.zeros((ns, 64, 56, 56), f32))
    cp = nb.conv_params(7, 7, 2, 3, padding=nb.NPL_PAD_EXPLICIT)
    bnp = nb.NplBatchnormParams(mu.ctypes.data, va.ctypes.data, g.ctypes.data, be.ctypes.data,
                                1e-5, 0, 0.1)
    pp = nb.NplPoolingParams(3, 3, 2, 2, 1, 1, nb.NPL_POOL_MAX, 0)

    def stem():
        ok(lib.npl_conv2d_bn_activation(C.byref(tx), C.byref(tw), None, C.byref(cp), C.byref(bnp),
                                        nb.NPL_ACT_RELU, C.byref(tconv), None))
        ok(lib.npl_batch_norm(C.byref(tconv), C.byref(bnp), C.byref(tbn), None))
        ok(lib.npl_relu(C.byref(tbn), C.byref(tbn), None))
        ok(lib.npl_pooling(C.byref(tbn), C.byref(pp), C.byref(tpool), None))

    sec = timed(stem) * (128 / ns)
    out["stem"] = {"ms_full_workload": round(sec * 1e3, 2),
                   "conv_TFLOP/s": round(2.0 * 128 * 64 * 3 * 112 * 112 * 49 / sec / 1e12, 5),
                   "sample": f"{ns} of 128 images, scaled"}
    # d4: chain on 16 of 256 images
    ns = 16
    x = rng.normal(0, 1, (ns, 512, 14, 14)).astype(f32)
    w = rng.normal(0, 0.3, (512, 1, 3, 3)).astype(f32)
    g, be = rng.uniform(0.5, 1.5, 512).astype(f32), rng.uniform(-0.1, 0.1, 512).astype(f32)
    mu, va = rng.normal(0, 0.1, 512).astype(f32), rng.uniform(0.5, 1.5, 512).astype(f32)
    keep.extend([g, be, mu, va])
    tx, tw = T(x), T(w)
    tdw, tb2 = T(np.zeros_like(x)), T(np.zeros_like(x))
    tgap, tsm = T(np.zeros((ns, 512), f32)), T(np.zeros((ns, 512), f32))
    dp = nb.conv_params(3, 3, 1, 1, padding=nb.NPL_PAD_EXPLICIT)
    bnp2 = nb.NplBatchnormParams(mu.ctypes.data, va.ctypes.data, g.ctypes.data, be.ctypes.data,
                                 1e-5, 0, 0.1)

    def chain():
        ok(lib.npl_depthwise_conv2d(C.byref(tx), C.byref(tw), None, C.byref(dp), C.byref(tdw),
                                    None))
        ok(lib.npl_batch_norm(C.byref(tdw), C.byref(bnp2), C.byref(tb2), None))
        ok(lib.npl_relu(C.byref(tb2), C.byref(tb2), None))
        ok(lib.npl_global_avg_pool(C.byref(tb2), C.byref(tgap), None))
        ok(lib.npl_softmax(C.byref(tgap), 1, C.byref(tsm), None))

    sec = timed(chain) * (256 / ns)
    out["bandwidth_chain"] = {"us_full_workload": round(sec * 1e6, 1),
                              "GB/s": round(720914432 / sec / 1e9, 2),
                              "sample": f"{ns} of 256 images, scaled"}
    # d5: GEMM + bias (beta=1) + ReLU + layer norm on 512 of 8192 rows
    ms_, k_, n_ = 512, 4096, 16384
    a = rng.normal(0, 1, (ms_, k_)).astype(f32)
    b = (rng.normal(0, 1, (k_, n_)) / 64.0).astype(f32)
    bias = rng.normal(0, 0.02, n_).astype(f32)
    c = np.empty((ms_, n_), f32)
    ta, tb, tcm, ty = T(a), T(b), T(c), T(np.zeros((ms_, n_), f32))
    lnp = nb.NplLayernormParams(None, None, 1e-5, n_)

    def big():
        c[:] = bias[None, :]
        ok(lib.npl_matmul(C.byref(ta), C.byref(tb), C.byref(tcm), C.c_float(1.0),
                          C.c_float(1.0), None))
        ok(lib.npl_relu(C.byref(tcm), C.byref(tcm), None))
        ok(lib.npl_layer_norm(C.byref(tcm), C.byref(lnp), C.byref(ty), None))

    sec = timed(big) * (8192 / ms_)
    out["gemm_relu_layer_norm"] = {
        "ms_full_workload": round(sec * 1e3, 2),
        "TFLOP/s (GEMM flops)": round(2.0 * 8192 * 4096 * 16384 / sec / 1e12, 5),
        "sample": f"{ms_} of 8192 rows, scaled"}
    out["cores"] = cores
    return out


def _reference_cpu_timed(ref_lib, steps, warmup, rows=False):
    lib = C.CDLL(str(ref_lib))
    nb.bind(lib, nb.NPL_SIGNATURES)
    cores = os.cpu_count() or 1
    cfg = nb.NplConfig()
    lib.npl_get_default_config(C.byref(cfg))
    cfg.num_threads = cores
    if lib.npl_init(C.byref(cfg)) != 0:
        return None
    x, w, gamma, beta, mean, var = conv_inputs(0)
    conv = np.zeros((N_IMG, C_OUT, HW_IN, HW_IN), np.float32)
    bnout = np.zeros_like(conv)
    y = np.zeros_like(conv)
    keep = [x, w, conv, bnout, y]
    tx, tw, tc, tb, ty = (nb.tensor(lib, a.ctypes.data, a.shape) for a in keep)
    p = nb.conv_params(KSZ, KSZ, 1, 1, padding=nb.NPL_PAD_EXPLICIT)
    bn = nb.NplBatchnormParams(mean.ctypes.data, var.ctypes.data, gamma.ctypes.data,
                               beta.ctypes.data, 1e-5, 0, 0.1)
    def step():
        assert lib.npl_conv2d_bn_activation(C.byref(tx), C.byref(tw), None, C.byref(p),
                                            C.byref(bn), nb.NPL_ACT_RELU, C.byref(tc),
                                            None) == 0
        assert lib.npl_batch_norm(C.byref(tc), C.byref(bn), C.byref(tb), None) == 0
        assert lib.npl_relu(C.byref(tb), C.byref(ty), None) == 0

    times = []
    for _ in range(max(1, warmup)):  # the warm-up count the line reports
        step()
    budget_end = time.perf_counter() + 30.0
    for _ in range(max(1, steps)):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > budget_end:
            break
    med = statistics.median(times)
    sample = (f"full workload (32 images), {len(times)} timed steps, median; reference "
              f"npl_conv2d_bn_activation (conv only) + npl_batch_norm + npl_relu, "
              f"num_threads={cores}, OpenBLAS {cores} threads")
    return (CONV_FLOPS / med / 1e12, cores, sample, med,
            _reference_cpu_rows(lib, cores) if rows else None)


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------
def bind_host_to_gpu(local_rank):
    """Restricts this process to the CPUs NVML reports as local to its GPU, so
    the e2e leg's pinned host buffers live on, and are copied from, the GPU's
    own socket. Returns the number of CPUs bound, or None when NVML or the
    affinity call is unavailable (the process is then left as it was)."""
    try:
        import pynvml
        import torch
        pr = torch.cuda.get_device_properties(local_rank)
        bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        pynvml.nvmlInit()
        try:
            h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            ncpu = os.cpu_count() or 1
            words = pynvml.nvmlDeviceGetCpuAffinity(h, (ncpu + 63) // 64)
        finally:
            pynvml.nvmlShutdown()
        cpus = {i * 64 + b for i, word in enumerate(words) for b in range(64)
                if (int(word) >> b) & 1 and i * 64 + b < ncpu}
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
        return len(cpus)
    except Exception:  # no NVML, no affinity support: leave the process as it is
        return None


def run_b200(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    lib = nb.load()
    rc = lib.npl_init(None)
    if rc != 0:
        raise RuntimeError(f"npl_init failed: {rc}")
    dev = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream()
    sptr = C.c_void_p(stream.cuda_stream)

    x, w, gamma, beta, mean, var = conv_inputs(0)
    tx = torch.from_numpy(x).to(dev)
    tw = torch.from_numpy(w).to(dev)
    tg, tb, tm, tv = (torch.from_numpy(a).to(dev) for a in (gamma, beta, mean, var))
    ty = torch.empty((N_IMG, C_OUT, HW_IN, HW_IN), device=dev)
    g = nb.conv_geom(N_IMG, C_IN, HW_IN, HW_IN, C_OUT, KSZ, KSZ, 1, 1)
    ws = lib.nplk_conv_workspace_size(C.byref(g))
    work = torch.empty(ws // 4 + 64, device=dev)
    flush = make_l2_flush(dev)
    p = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731

    def prepare():
        r = lib.nplk_conv2d_prepare(sptr, C.byref(g), p(tw), None, p(tm), p(tv), p(tg), p(tb),
                                    1e-5, p(work), ws)
        assert r == 0, r

    def run():
        r = lib.nplk_conv2d_run(sptr, C.byref(g), p(tx), nb.NPL_ACT_RELU, 0.0, p(ty), p(work),
                                ws, None)
        assert r == 0, r

    def fused():
        # weight preparation + conv in one call: the conv kernel overlaps the
        # preparation kernel (programmatic dependent launch)
        r = lib.nplk_conv2d_fused(sptr, C.byref(g), p(tx), p(tw), None, p(tm), p(tv), p(tg),
                                  p(tb), 1e-5, nb.NPL_ACT_RELU, 0.0, p(ty), p(work), ws, None)
        assert r == 0, r

    # clock sampling: the NVML poll starts before the warm-up and reports the
    # samples taken inside the timed region
    sampler = ClockSampler(local_rank) if rank == 0 else None
    for _ in range(args.warmup):
        flush()
        fused()
    torch.cuda.synchronize()
    if lib.nplk_read_status(sptr) != 0:
        raise RuntimeError("conv kernel reported a pipeline timeout")

    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    if sampler:
        sampler.start()
    lib.nplk_take_launch_count()
    for i in range(args.steps):
        flush()  # outside the timed events
        ev[i][0].record(stream)
        fused()
        ev[i][1].record(stream)
    torch.cuda.synchronize()
    launches = int(lib.nplk_take_launch_count())
    if world > 1:
        dist.barrier()
    clocks = sampler.stop() if sampler else None
    if lib.nplk_read_status(sptr) != 0:
        raise RuntimeError("conv kernel reported a pipeline timeout")
    step_ms = [e[0].elapsed_time(e[1]) for e in ev]
    # The conv kernel alone (for the roofline): the same loop on prepared
    # weights, one nplk_conv2d_run per step.
    prepare()
    kev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    for i in range(args.steps):
        flush()
        kev[i][0].record(stream)
        run()
        kev[i][1].record(stream)
    torch.cuda.synchronize()
    conv_ms = [e[0].elapsed_time(e[1]) for e in kev]
    stats = torch.tensor([sum(step_ms) / len(step_ms), statistics.mean(conv_ms)],
                         device=dev, dtype=torch.float64)
    tot_launch = torch.tensor([launches], device=dev, dtype=torch.int64)
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
        dist.all_reduce(tot_launch, op=dist.ReduceOp.SUM)
    ms_per_step, conv_kernel_ms = stats.tolist()

    # ---- e2e through the public C ABI with pinned host buffers ----
    # The process first moves to its GPU's local CPUs so its pinned buffers
    # sit on that socket; the affinity is restored after this leg (the CPU
    # baseline below uses every host thread).
    saved_affinity = os.sched_getaffinity(0)
    cpus_bound = bind_host_to_gpu(local_rank)
    hx = torch.from_numpy(x).pin_memory()
    hw_ = torch.from_numpy(w).pin_memory()
    hy = torch.empty((N_IMG, C_OUT, HW_IN, HW_IN)).pin_memory()
    hg, hb, hm, hv = (torch.from_numpy(a).pin_memory() for a in (gamma, beta, mean, var))
    t_x = nb.tensor(lib, hx.data_ptr(), hx.shape)
    t_w = nb.tensor(lib, hw_.data_ptr(), hw_.shape)
    t_y = nb.tensor(lib, hy.data_ptr(), hy.shape)
    cp = nb.conv_params(KSZ, KSZ, 1, 1, padding=nb.NPL_PAD_EXPLICIT)
    bnp = nb.NplBatchnormParams(hm.data_ptr(), hv.data_ptr(), hg.data_ptr(), hb.data_ptr(),
                                1e-5, 0, 0.1)

    def api_step():
        r = lib.npl_conv2d_bn_activation(C.byref(t_x), C.byref(t_w), None, C.byref(cp),
                                         C.byref(bnp), nb.NPL_ACT_RELU, C.byref(t_y), None)
        assert r == 0, r

    for _ in range(args.warmup):
        api_step()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        api_step()  # synchronous: copies in, kernels, copy out
    e2e_s = torch.tensor([(time.perf_counter() - t0) / args.steps], device=dev,
                         dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e2e_s, op=dist.ReduceOp.MAX)
    e2e_step = float(e2e_s.item())
    h2d = hx.numel() * 4 + hw_.numel() * 4 + 4 * C_OUT * 4
    d2h = hy.numel() * 4

    # ---- parity spot check of the timed output (device result vs host API result) ----
    torch.cuda.synchronize()
    same = torch.allclose(ty.cpu(), hy, rtol=0, atol=0)
    # The host link alone: the same bytes copied host->device and back from
    # the same pinned buffers, all ranks at once, no kernels.
    dx, dy = torch.empty_like(tx), torch.empty_like(ty)
    for _ in range(2):
        dx.copy_(hx, non_blocking=True)
        hy.copy_(dy, non_blocking=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        dx.copy_(hx, non_blocking=True)
        hy.copy_(dy, non_blocking=True)
        torch.cuda.synchronize()
    link_s = torch.tensor([(time.perf_counter() - t0) / args.steps], device=dev,
                          dtype=torch.float64)
    if world > 1:
        dist.all_reduce(link_s, op=dist.ReduceOp.MAX)
    link_step = float(link_s.item())
    del dx, dy
    os.sched_setaffinity(0, saved_affinity)

    result = None
    if rank == 0:
        hbm_peak, bf16_peak, peak_src = measured_peaks()
        tf32x3_peak = bf16_peak / 2.0 / 3.0
        achieved = (CONV_FLOPS / 1e12) / (conv_kernel_ms / 1e3)
        traffic = None
        tp = REPO / "profiles" / "conv_window_traffic.json"
        if tp.exists():
            traffic = json.loads(tp.read_text()).get("dram_bytes_per_launch")
        value = world * CONV_FLOPS / (ms_per_step / 1e3) / 1e12
        result = {
            "metric": "fused conv2d+BN+ReLU TFLOP/s (npl_conv2d_bn_activation, 3xTF32)",
            "value": round(value, 3),
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 5),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f32 (3xTF32 tensor-core products, fp32 accumulate)",
            "data": "synthetic (seeded; the benchmark workload's shapes and value distributions)",
            "config": {
                "workload": WORKLOAD,
                "per_gpu_batch": N_IMG,
                "global_batch": N_IMG * world,
                "parallelism": f"dp{world} (batch-sharded, no collective)",
                "l2": "flushed between steps (256 MiB write, then 256 MiB read so no dirty lines remain; outside the timed events)",
                "step": "nplk_conv2d_fused (weight split + BN constants, then the conv kernel "
                        "overlapping it)",
            },
            "e2e": {
                "value": round(world * CONV_FLOPS / e2e_step / 1e12, 3),
                "unit": "TFLOP/s",
                "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "api": "npl_conv2d_bn_activation on pinned host tensors (library stages)",
                "host_link": {
                    "copy_ms_per_step": round(link_step * 1e3, 4),
                    "GB/s_per_rank": round((hx.numel() + hy.numel()) * 4 / link_step / 1e9, 2),
                    "what": "the step's input and output bytes copied host->device and back "
                            "from the same pinned buffers, no kernels, all ranks at once "
                            "(max over ranks)",
                    "cpus_bound_per_rank": cpus_bound,
                },
            },
            "roofline": {
                "bound": "tensor",
                "achieved": round(achieved, 2),
                "peak": round(tf32x3_peak, 1),
                "unit": "TFLOP/s",
                "frac": round(achieved / tf32x3_peak, 4),
                "traffic": traffic,
                "kernel": "conv_window_3xtf32_kernel<64, relu, gather>",
                "kernel_ms": round(conv_kernel_ms, 5),
                "kernel_timing": "CUDA events around nplk_conv2d_run (prepared weights, same "
                                 "inputs and L2 flush), a second loop of --steps launches",
                "peak_basis": f"{peak_src} bf16 {bf16_peak} TFLOP/s / 2 (TF32) / 3 (3xTF32)",
            },
            "gpu_launches": int(tot_launch.item()),
            "output_matches_api_path": bool(same),
        }
        if clocks:
            result["clocks"] = clocks
    return lib, result


def bandwidth_also(lib, local_rank, reps=10):
    """The bandwidth-bound primitives on one GPU at the workload's size
    (N=256, C=512, 14x14 NCHW = 103 MB; layer norm on 8192 x 4096; softmax
    over 102400 rows of 1000) and at four times that size: median CUDA-event
    time of `reps` launches with L2 flushed before each, algorithmic bytes
    (each input read once, each output written once) per second, and the
    fraction of the measured HBM copy bandwidth.

    At the workload's size an output of ~100 MB is still largely dirty in the
    126 MB L2 when the end event fires, so write-heavy kernels read high
    (an upper bound) and read-only ones low; the 4x figures (outputs well
    beyond L2, ramp-up amortised) are the steady-state DRAM rates. Two
    size-matched references are timed the same way: a device copy and a pure
    read (a sum) of the same tensor."""
    import torch
    dev = torch.device("cuda", local_rank)
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    flush = make_l2_flush(dev)
    hbm, _, src = measured_peaks()

    def cases_at(scale):
        gen = torch.Generator(device=dev).manual_seed(0)
        n, c, hw = 256 * scale, 512, 14
        x = torch.randn(n, c, hw, hw, device=dev, generator=gen)
        y = torch.empty_like(x)
        w = torch.randn(c, 1, 3, 3, device=dev, generator=gen) * 0.3
        bn = [torch.rand(c, device=dev, generator=gen) + 0.5 for _ in range(4)]
        gap = torch.empty(n * c, device=dev)
        pooled = torch.empty(n, c, 7, 7, device=dev)
        rows = torch.randn(8192 * scale, 4096, device=dev, generator=gen)
        rows_y = torch.empty_like(rows)
        logits = torch.randn(102400 * scale, 1000, device=dev, generator=gen)
        probs = torch.empty_like(logits)
        g = nb.conv_geom(n, c, hw, hw, c, 3, 3, 1, 1)
        nx = x.numel()
        acc = torch.empty((), device=dev)
        cases = [
            ("depthwise 3x3", nx * 8 + w.numel() * 4,
             lambda: lib.nplk_depthwise_conv2d(s, C.byref(g), p(x), p(w), None, p(y))),
            ("batch_norm inference", nx * 8,
             lambda: lib.nplk_batch_norm_infer(s, n, c, hw * hw, p(x), p(y), p(bn[0]), p(bn[1]),
                                               p(bn[2]), p(bn[3]), 1e-5)),
            ("relu", nx * 8, lambda: lib.nplk_activation(s, nx, p(x), p(y), 1, 0.0, 0)),
            ("max pool 3x3/s2", nx * 4 + pooled.numel() * 4,
             lambda: lib.nplk_pool2d(s, n, c, hw, hw, 3, 3, 2, 2, 1, 1, 7, 7, 0, 0, p(x),
                                     p(pooled))),
            ("global avg pool", nx * 4 + gap.numel() * 4,
             lambda: lib.nplk_global_avg_pool(s, n * c, hw * hw, p(x), p(gap))),
            ("softmax rows of 1000", logits.numel() * 8,
             lambda: lib.nplk_softmax(s, logits.shape[0], 1000, 1, p(logits), p(probs))),
            ("layer_norm 8192x4096", rows.numel() * 8,
             lambda: lib.nplk_layer_norm(s, rows.shape[0], 4096, p(rows), p(rows_y), None, None,
                                         1e-5)),
        ]
        if scale == 1:
            # The depthwise -> BN -> ReLU -> GAP -> softmax chain on
            # [256,512,14,14] (BN into a second tensor, ReLU in place, softmax
            # over the 512 channels of each image), back to back after one L2
            # flush; bytes: each kernel's input read once, output written once.
            y2 = torch.empty_like(x)
            sm_out = torch.empty(n * c, device=dev)
            chain_bytes = (nx * 8 + w.numel() * 4) + nx * 8 + nx * 8 + (nx * 4 + n * c * 4) + \
                n * c * 8

            def chain():
                # the same function tests/test_gpu_workloads.py checks against
                # the reference's CPU chain
                return abs(workloads.bandwidth_chain(lib, s, x, w, bn[0], bn[1], bn[2], bn[3], y,
                                                     y2, gap, sm_out))

            cases.append(("chain depthwise->BN->ReLU->GAP->softmax [256,512,14,14]", chain_bytes,
                          chain))
        # The same chain with its first four calls in one pass
        # (nplk_depthwise_bn_act_gap, no intermediate map written), then the
        # softmax; bytes: x and the filters read once, the pooled [N,C] written,
        # the softmax's read and write.
        fgap = torch.empty(n * c, device=dev)
        fsm = torch.empty(n * c, device=dev)
        fused_bytes = nx * 4 + w.numel() * 4 + n * c * 4 + n * c * 8

        def chain_fused():
            return abs(workloads.bandwidth_chain_fused(lib, s, x, w, bn[0], bn[1], bn[2], bn[3],
                                                       fgap.view(n, c), fsm.view(n, c)))

        cases.append(("chain fused: depthwise+BN+ReLU+GAP in one pass, then softmax "
                      "[256,512,14,14]", fused_bytes, chain_fused))
        cases += [
            ("device copy of the same tensor (reference)", nx * 8, lambda: (y.copy_(x), 0)[1]),
            ("read (sum) of the same tensor (reference)", nx * 4,
             lambda: (torch.sum(x.view(-1), dim=0, out=acc), 0)[1]),
        ]
        res = {}
        for name, nbytes, fn in cases:
            assert fn() == 0
            ts = []
            for _ in range(reps):
                flush()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record()
                assert fn() == 0
                e1.record()
                torch.cuda.synchronize()
                ts.append(e0.elapsed_time(e1))
            ms = statistics.median(ts)
            res[name] = (ms, nbytes)
        return res

    out = {}
    base = cases_at(1)
    big = cases_at(4)
    torch.cuda.empty_cache()
    ref_gbs = None
    for name, (ms, nbytes) in base.items():
        gbs = nbytes / (ms / 1e3) / 1e9
        if name.startswith("device copy"):
            ref_gbs = gbs
        out[name] = {"us": round(ms * 1e3, 1), "bytes": int(nbytes), "GB/s": round(gbs, 1),
                     "frac_of_hbm": round(gbs / hbm, 3)}
        if name in big:
            ms4, nb4 = big[name]
            g4 = nb4 / (ms4 / 1e3) / 1e9
            out[name].update({"us_4x": round(ms4 * 1e3, 1), "GB/s_4x": round(g4, 1),
                              "frac_of_hbm_4x": round(g4 / hbm, 3)})
    for name, v in out.items():
        v["frac_of_copy_at_size"] = round(v["GB/s"] / ref_gbs, 3)
    out["peak"] = f"{src} HBM copy {hbm} GB/s (>= 1 GB transfers)"
    out["sizes"] = ("at size: the workload's tensors; _4x: batch (rows) x4, outputs beyond L2 "
                    "so their write-back falls inside the timed region")
    return out


def gemm_also(lib, args, local_rank):
    """Large-GEMM figure on one GPU: C = A@B + C (C pre-filled with the bias row)."""
    import torch
    dev = torch.device("cuda", local_rank)
    gen = torch.Generator(device=dev).manual_seed(0)
    A = torch.randn(GEMM_M, GEMM_K, device=dev, generator=gen)
    B = torch.randn(GEMM_K, GEMM_N, device=dev, generator=gen) / 64.0
    bias = torch.randn(GEMM_N, device=dev, generator=gen) * 0.02
    Cm = torch.empty(GEMM_M, GEMM_N, device=dev)
    ws = lib.nplk_gemm_workspace_size(GEMM_M, GEMM_N, GEMM_K)
    work = torch.empty(ws // 4 + 64, device=dev)
    stream = torch.cuda.current_stream()
    sptr = C.c_void_p(stream.cuda_stream)
    p = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731

    def step():
        Cm.copy_(bias.expand(GEMM_M, GEMM_N))
        r = lib.nplk_gemm(sptr, GEMM_M, GEMM_N, GEMM_K, 1.0, p(A), GEMM_K, p(B), GEMM_N, 1.0,
                          p(Cm), GEMM_N, None, 0, 0.0, 0, p(work), ws, None)
        assert r == 0, r

    for _ in range(2):
        step()
    torch.cuda.synchronize()
    n = max(3, min(args.steps, 10))
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(n)]
    for e0, e1 in evs:
        Cm.copy_(bias.expand(GEMM_M, GEMM_N))
        e0.record(stream)
        r = lib.nplk_gemm(sptr, GEMM_M, GEMM_N, GEMM_K, 1.0, p(A), GEMM_K, p(B), GEMM_N, 1.0,
                          p(Cm), GEMM_N, None, 0, 0.0, 0, p(work), ws, None)
        assert r == 0, r
        e1.record(stream)
    torch.cuda.synchronize()
    if lib.nplk_read_status(sptr) != 0:
        raise RuntimeError("GEMM kernel reported a pipeline timeout")
    ms = statistics.mean(e0.elapsed_time(e1) for e0, e1 in evs)
    # spot parity on a few rows against fp64
    rows = torch.arange(0, GEMM_M, GEMM_M // 8, device=dev)
    ref = A[rows].double() @ B.double() + bias.double()
    err = ((Cm[rows].double() - ref).abs().max() / ref.abs().max()).item()
    # The whole large-GEMM workload: bias (beta = 1) and ReLU in the GEMM
    # epilogue, then layer norm over rows of 16384.
    Y = torch.empty_like(Cm)
    pipe_ms, ln_ms = [], []
    for _ in range(n):
        workloads.fill_bias_rows(Cm, bias)
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record(stream)
        # the same function tests/test_gpu_workloads.py checks against the
        # reference's npl_matmul (beta 1) -> npl_relu -> npl_layer_norm
        r = workloads.gemm_bias_relu_layer_norm(lib, sptr, A, B, Cm, Y, work, ws,
                                                between=lambda: e1.record(stream))
        assert r == 0, r
        e2.record(stream)
        torch.cuda.synchronize()
        pipe_ms.append(e0.elapsed_time(e2))
        ln_ms.append(e1.elapsed_time(e2))
    pm, lm = statistics.mean(pipe_ms), statistics.mean(ln_ms)
    del A, B, Cm, Y, work
    torch.cuda.empty_cache()
    return {"workload": "npl_matmul fp32 [8192x4096]@[4096x16384] + bias (beta=1), 1 GPU",
            "value": round(GEMM_FLOPS / (ms / 1e3) / 1e12, 2), "unit": "TFLOP/s",
            "ms_per_step": round(ms, 4), "normwise_err_sampled_rows": err,
            "step": "split A and B^T into tf32 hi/lo + tcgen05 GEMM",
            "with_relu_and_layer_norm": {
                "ms": round(pm, 4), "TFLOP/s (GEMM flops)": round(GEMM_FLOPS / (pm / 1e3) / 1e12, 2),
                "layer_norm_ms": round(lm, 4),
                "layer_norm_GB/s": round(2 * GEMM_M * GEMM_N * 4 / (lm / 1e3) / 1e9, 1),
                "step": "GEMM with bias (beta=1) and ReLU in the epilogue, then layer norm "
                        "over rows of 16384 (gamma 1, beta 0, eps 1e-5)"}}


def stem_also(lib, local_rank, reps=5):
    """The stem layer on one GPU: conv 7x7/s2/p3 3->64 on [128,3,224,224]
    (C_in = 3: the direct-gather kernel) with BN + ReLU, then max pool
    3x3/s2/p1 -> [128,64,56,56]; inputs U[-1,1], w N(0, sqrt(2/147))."""
    import torch
    dev = torch.device("cuda", local_rank)
    gen = torch.Generator(device=dev).manual_seed(0)
    n = 128
    x = torch.rand(n, 3, 224, 224, device=dev, generator=gen) * 2 - 1
    w = torch.randn(64, 3, 7, 7, device=dev, generator=gen) * (2.0 / 147) ** 0.5
    bn = [torch.rand(64, device=dev, generator=gen) + 0.5 for _ in range(4)]
    y = torch.empty(n, 64, 112, 112, device=dev)
    pooled = torch.empty(n, 64, 56, 56, device=dev)
    g = nb.conv_geom(n, 3, 224, 224, 64, 7, 7, 2, 3)
    ws = lib.nplk_conv_workspace_size(C.byref(g))
    work = torch.empty(ws // 4 + 64, device=dev)
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    flush = make_l2_flush(dev)

    def conv():
        r = lib.nplk_conv2d_fused(s, C.byref(g), p(x), p(w), None, p(bn[0]), p(bn[1]), p(bn[2]),
                                  p(bn[3]), 1e-5, nb.NPL_ACT_RELU, 0.0, p(y), p(work), ws, None)
        assert r == 0, r

    def pool():
        r = lib.nplk_pool2d(s, n, 64, 112, 112, 3, 3, 2, 2, 1, 1, 56, 56, 0, 0, p(y), p(pooled))
        assert r == 0, r

    # The fused form: the conv epilogue writes the horizontal maxima of the
    # pool windows (half the conv output) and a vertical pass finishes the
    # pool (nplk_conv2d_maxpool_fused; bit-identical to conv then pool).
    fws = lib.nplk_conv2d_maxpool_workspace_size(C.byref(g))
    fwork = torch.empty(fws // 4 + 64, device=dev)
    fused_out = torch.empty_like(pooled)

    def fused():
        r = lib.nplk_conv2d_maxpool_fused(s, C.byref(g), p(x), p(w), None, p(bn[0]), p(bn[1]),
                                          p(bn[2]), p(bn[3]), 1e-5, nb.NPL_ACT_RELU, 0.0,
                                          p(fused_out), p(fwork), fws, None)
        assert r == 0, r

    conv(), pool(), fused()
    cms, pms, fms = [], [], []
    for _ in range(reps):
        flush()
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record()
        conv()
        e1.record()
        pool()
        e2.record()
        torch.cuda.synchronize()
        cms.append(e0.elapsed_time(e1))
        pms.append(e1.elapsed_time(e2))
        flush()
        e3, e4 = (torch.cuda.Event(enable_timing=True) for _ in range(2))
        e3.record()
        fused()
        e4.record()
        torch.cuda.synchronize()
        fms.append(e3.elapsed_time(e4))
    if lib.nplk_read_status(s) != 0:
        raise RuntimeError("conv kernel reported a pipeline timeout")
    same = bool(torch.equal(fused_out, pooled))
    flops = 2.0 * n * 64 * 3 * 112 * 112 * 49
    cm, pm, fm = statistics.median(cms), statistics.median(pms), statistics.median(fms)
    return {"workload": "conv 7x7/s2/p3 3->64 [128,3,224,224] + BN + ReLU, then max pool "
                        "3x3/s2/p1", "conv_ms": round(cm, 4),
            "conv_TFLOP/s": round(flops / (cm / 1e3) / 1e12, 2), "pool_ms": round(pm, 4),
            "pool_GB/s": round((y.numel() + pooled.numel()) * 4 / (pm / 1e3) / 1e9, 1),
            "conv_plus_pool_ms": round(cm + pm, 4),
            "fused_conv_maxpool_ms": round(fm, 4),
            "fused_TFLOP/s (conv flops)": round(flops / (fm / 1e3) / 1e12, 2),
            "fused_output_identical": same}


def gemm1024_also(lib, local_rank, reps=20):
    """npl_matmul 1024 x 1024 x 1024 (A, B ~ U[-1,1], beta 0) on device
    pointers: median CUDA-event time of nplk_gemm (split + GEMM). The inputs
    (12 MB) fit in L2, so L2 is flushed before every timed call, outside the
    events; the flush also keeps the GPU busy while the host launches the
    call, so the events time the device work."""
    import torch
    dev = torch.device("cuda", local_rank)
    gen = torch.Generator(device=dev).manual_seed(0)
    m = 1024
    a = torch.rand(m, m, device=dev, generator=gen) * 2 - 1
    b = torch.rand(m, m, device=dev, generator=gen) * 2 - 1
    c = torch.empty(m, m, device=dev)
    ws = lib.nplk_gemm_workspace_size(m, m, m)
    work = torch.empty(ws // 4 + 64, device=dev)
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    flush = make_l2_flush(dev)
    ts = []
    for i in range(reps + 3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        flush()
        e0.record()
        r = lib.nplk_gemm(s, m, m, m, 1.0, p(a), m, p(b), m, 0.0, p(c), m, None, 0, 0.0, 0,
                          p(work), ws, None)
        assert r == 0, r
        e1.record()
        torch.cuda.synchronize()
        if i >= 3:
            ts.append(e0.elapsed_time(e1))
    ms = statistics.median(ts)
    err = ((c.double() - a.double() @ b.double()).abs().max() /
           (a.double() @ b.double()).abs().max()).item()
    return {"workload": "npl_matmul 1024^3", "l2": "flushed before each call", "us": round(ms * 1e3, 2),
            "TFLOP/s": round(2 * m ** 3 / (ms / 1e3) / 1e12, 2), "normwise_err": err}


def strong_scaling_also(lib, rank, world, local_rank, reps=10):
    """The stated batches split over the ranks (strong scaling, no collective):
    the 3x3 layer's 32 images, the stem's 128 and the bandwidth chain's 256,
    each rank taking a contiguous block of batch_shard(N, world, rank) images
    (inputs resident on its GPU, weights replicated). Per rank: median CUDA-
    event time of `reps` runs with L2 flushed before each; the line's time is
    the max over ranks and its throughput the whole batch's work over that
    time. With more than one rank, rank 0 also times the whole batch on its
    own GPU, so each line carries its speed-up and efficiency against one GPU.
    The loop each rank runs is ExecuteConvDirect's ParallelFor over N*Cout
    (npl_convolution.cpp:267-342) cut along N."""
    import torch
    import torch.distributed as dist
    from npl_b200 import dist as nd

    dev = torch.device("cuda", local_rank)
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    flush = make_l2_flush(dev)

    def timed(fn):
        fn()
        ts = []
        for _ in range(reps):
            flush()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        if lib.nplk_read_status(s) != 0:
            raise RuntimeError("a kernel reported a pipeline timeout")
        return statistics.median(ts)

    def conv_case(n, c, hw, cout, k, stride, pad, x_lo, x_hi, pool):
        gen = torch.Generator(device=dev).manual_seed(1000 + rank)
        x = torch.rand(n, c, hw, hw, device=dev, generator=gen) * (x_hi - x_lo) + x_lo
        wgen = torch.Generator(device=dev).manual_seed(7)  # replicated weights
        w = torch.randn(cout, c, k, k, device=dev, generator=wgen) * (2.0 / (c * k * k)) ** 0.5
        bn = [torch.rand(cout, device=dev, generator=wgen) + 0.5 for _ in range(4)]
        g = nb.conv_geom(n, c, hw, hw, cout, k, k, stride, pad)
        y = torch.empty(n, cout, g.h_out, g.w_out, device=dev)
        ws = lib.nplk_conv_workspace_size(C.byref(g))
        work = torch.empty(ws // 4 + 64, device=dev)
        ho = g.h_out
        pooled = torch.empty(n, cout, (ho + 2 - 3) // 2 + 1, (ho + 2 - 3) // 2 + 1,
                             device=dev) if pool else None

        def fn():
            r = lib.nplk_conv2d_fused(s, C.byref(g), p(x), p(w), None, p(bn[0]), p(bn[1]),
                                      p(bn[2]), p(bn[3]), 1e-5, nb.NPL_ACT_RELU, 0.0, p(y),
                                      p(work), ws, None)
            assert r == 0, r
            if pool:
                po = pooled.shape[-1]
                r = lib.nplk_pool2d(s, n, cout, ho, ho, 3, 3, 2, 2, 1, 1, po, po, 0, 0, p(y),
                                    p(pooled))
                assert r == 0, r
        return fn

    def chain_fused_case(n):
        gen = torch.Generator(device=dev).manual_seed(2000 + rank)
        x = torch.randn(n, 512, 14, 14, device=dev, generator=gen)
        wgen = torch.Generator(device=dev).manual_seed(8)
        w = torch.randn(512, 1, 3, 3, device=dev, generator=wgen) * 0.3
        bn = [torch.rand(512, device=dev, generator=wgen) + 0.5 for _ in range(4)]
        gap, probs = torch.empty(n, 512, device=dev), torch.empty(n, 512, device=dev)

        def fn():
            r = workloads.bandwidth_chain_fused(lib, s, x, w, bn[0], bn[1], bn[2], bn[3], gap,
                                                probs)
            assert r == 0, r
        return fn

    def chain_case(n):
        gen = torch.Generator(device=dev).manual_seed(2000 + rank)
        x = torch.randn(n, 512, 14, 14, device=dev, generator=gen)
        wgen = torch.Generator(device=dev).manual_seed(8)
        w = torch.randn(512, 1, 3, 3, device=dev, generator=wgen) * 0.3
        bn = [torch.rand(512, device=dev, generator=wgen) + 0.5 for _ in range(4)]
        y, y2 = torch.empty_like(x), torch.empty_like(x)
        gap, probs = torch.empty(n, 512, device=dev), torch.empty(n, 512, device=dev)

        def fn():
            r = workloads.bandwidth_chain(lib, s, x, w, bn[0], bn[1], bn[2], bn[3], y, y2, gap,
                                          probs)
            assert r == 0, r
        return fn

    cases = [
        ("conv3x3 N=32 C=64 56x56 (+BN+ReLU)", 32, "TFLOP/s",
         lambda n: 2.0 * n * 64 * 64 * 56 * 56 * 9 / 1e12,
         lambda n: conv_case(n, 64, 56, 64, 3, 1, 1, 0.0, 1.0, False)),
        ("stem conv7x7/s2 N=128 (+BN+ReLU) + max pool 3x3/s2", 128, "TFLOP/s (conv flops)",
         lambda n: 2.0 * n * 64 * 3 * 112 * 112 * 49 / 1e12,
         lambda n: conv_case(n, 3, 224, 64, 7, 2, 3, -1.0, 1.0, True)),
        ("depthwise->BN->ReLU->GAP->softmax N=256 C=512 14x14", 256, "GB/s",
         lambda n: n * 720914432 / 256 / 1e9,
         lambda n: chain_case(n)),
        ("the same chain fused (depthwise+BN+ReLU+GAP in one pass, then softmax)", 256,
         "images/s", lambda n: n, lambda n: chain_fused_case(n)),
    ]
    out = {}
    for name, n_total, unit, work_of, make in cases:
        b0, b1 = nd.batch_shard(n_total, world, rank)
        ms = timed(make(b1 - b0))
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = float(t.item())
        entry = {"global_batch": n_total, "per_gpu_batch": b1 - b0, "ms": round(ms_max, 4),
                 "value": round(work_of(n_total) / (ms_max / 1e3), 2), "unit": unit}
        if world > 1 and rank == 0:
            ms1 = timed(make(n_total))
            entry["one_gpu_ms"] = round(ms1, 4)
            entry["speedup"] = round(ms1 / ms_max, 3)
            entry["efficiency"] = round(ms1 / ms_max / world, 3)
        if world > 1:
            dist.barrier()
        out[name] = entry
        torch.cuda.empty_cache()
    return {"scaling": "strong (the stated batch split over the GPUs, no collective)",
            "time": "per-rank median CUDA-event time, L2 flushed before each run, max over "
                    "ranks", "cases": out}


def gemm_dist(args, rank, world, local_rank):
    """Column-sharded large GEMM on `world` GPUs: each rank computes its block
    of C = A @ B + bias (A replicated) and every rank ends with the whole
    row-major C, either through the fused GEMM whose epilogue stores each tile
    into all ranks' C over NVLink (peer stores from its threads or the TMA
    unit, or one store through an NVLink multicast object where the fabric
    offers multicast; the faster bit-identical fused form is the end-to-end
    value) or through the GEMM followed by an NCCL all-gather and the relayout
    kernel. Device time per step, max over ranks, for the GEMM alone and for
    each form."""
    import torch
    import torch.distributed as dist
    from npl_b200 import dist as nd

    dev = torch.device("cuda", local_rank)
    gen = torch.Generator(device=dev).manual_seed(0)
    A = torch.randn(GEMM_M, GEMM_K, device=dev, generator=gen)
    B = torch.randn(GEMM_K, GEMM_N, device=dev, generator=gen) / 64.0
    bias = torch.randn(GEMM_N, device=dev, generator=gen) * 0.02
    lib = nb.load()
    w = GEMM_N // world
    ws = lib.nplk_gemm_workspace_size(GEMM_M, w, GEMM_K)
    work = torch.empty(ws // 4 + 64, device=dev)
    stream = torch.cuda.current_stream()

    def step():
        local = nd.column_sharded_gemm(A, B, bias, world, rank, workspace=work, gather=False)
        e_mid.record(stream)
        return nd.gather_column_blocks(local, world)

    for _ in range(2):
        e_mid = torch.cuda.Event(enable_timing=True)
        step()
    torch.cuda.synchronize()
    n = max(3, min(args.steps, 10))
    g_ms, t_ms = [], []
    dist.barrier()
    for _ in range(n):
        e0 = torch.cuda.Event(enable_timing=True)
        e_mid = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        full = step()
        e1.record(stream)
        torch.cuda.synchronize()
        g_ms.append(e0.elapsed_time(e_mid))
        t_ms.append(e0.elapsed_time(e1))
    dist.barrier()
    if lib.nplk_read_status(C.c_void_p(stream.cuda_stream)) != 0:
        raise RuntimeError("GEMM kernel reported a pipeline timeout")
    t = torch.tensor([statistics.mean(g_ms), statistics.mean(t_ms)], device=dev,
                     dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    rows = torch.arange(0, GEMM_M, GEMM_M // 4, device=dev)
    ref = A[rows].double() @ B.double() + bias.double()
    err = ((full[rows].double() - ref).abs().max() / ref.abs().max()).item()
    gm, tm = t.tolist()

    # Fused form: every rank's GEMM epilogue stores its blocks into all ranks'
    # C over NVLink (CUDA IPC peer pointers); C is complete on every rank when
    # all ranks' kernels have finished, i.e. after the max over ranks of the
    # per-rank device time.
    # The peers are written by 16-byte stores from the epilogue threads (the
    # default) and, for comparison, through the TMA unit; C is checked after
    # the default form, which runs last.
    full_f = torch.empty(GEMM_M, GEMM_N, device=dev)
    peers = nd.PeerBuffers(full_f, world, rank)

    def fused_ms(flags, dst=None):
        dst = peers if dst is None else dst
        for _ in range(2):
            nd.column_sharded_gemm_fused(A, B, dst, bias, workspace=work, flags=flags)
        torch.cuda.synchronize()
        dist.barrier()
        f_ms = []
        for _ in range(n):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            nd.column_sharded_gemm_fused(A, B, dst, bias, workspace=work, flags=flags)
            e1.record(stream)
            torch.cuda.synchronize()
            dist.barrier()
            f_ms.append(e0.elapsed_time(e1))
        tf = torch.tensor([statistics.mean(f_ms)], device=dev, dtype=torch.float64)
        dist.all_reduce(tf, op=dist.ReduceOp.MAX)
        return tf.item()

    try:
        tma_ms = fused_ms(nb.NPLK_GEMM_PEER_TMA_STORES)
        fm = fused_ms(0)
        ferr = ((full_f[rows].double() - ref).abs().max() / ref.abs().max()).item()
    finally:
        peers.close()
    # Multicast form: every rank's C bound to one NVLink multicast object; the
    # epilogue stores each tile once and NVSwitch delivers it to all ranks.
    mc, mc_ms, mc_why = None, None, None
    if os.environ.get("NPL_BENCH_NO_MULTICAST", "0") != "1":
        try:
            mc = nd.MulticastBuffers((GEMM_M, GEMM_N), world, rank)
        except RuntimeError as e:
            mc_why = str(e)[:200]
    else:
        mc_why = "skipped (NPL_BENCH_NO_MULTICAST=1)"
    if mc is not None:
        try:
            mc_ms = fused_ms(0, mc)
            full_mc = mc.tensor.clone()
        finally:
            mc.close()
        mc = None
    # Every rank's whole C against a one-GPU GEMM of the same inputs on this
    # rank (same k order and epilogue, so bit-identical is expected), for
    # both exchange forms.
    ws_full = lib.nplk_gemm_workspace_size(GEMM_M, GEMM_N, GEMM_K)
    work_full = torch.empty(ws_full // 4 + 64, device=dev)
    c_ref = torch.empty(GEMM_M, GEMM_N, device=dev)
    r = lib.nplk_gemm(C.c_void_p(stream.cuda_stream), GEMM_M, GEMM_N, GEMM_K, 1.0,
                      C.c_void_p(A.data_ptr()), GEMM_K, C.c_void_p(B.data_ptr()), GEMM_N, 0.0,
                      C.c_void_p(c_ref.data_ptr()), GEMM_N, C.c_void_p(bias.data_ptr()), 0, 0.0,
                      0, C.c_void_p(work_full.data_ptr()), ws_full, None)
    assert r == 0, r
    torch.cuda.synchronize()
    same = torch.tensor([int(torch.equal(full_f, c_ref)), int(torch.equal(full, c_ref)),
                         int(torch.equal(full_mc, c_ref)) if mc_ms is not None else 1],
                        device=dev, dtype=torch.int64)
    diff = torch.tensor([((full_f - c_ref).abs().max() / c_ref.abs().max()).item()],
                        device=dev, dtype=torch.float64)
    dist.all_reduce(same, op=dist.ReduceOp.MIN)
    dist.all_reduce(diff, op=dist.ReduceOp.MAX)
    del work_full, c_ref
    torch.cuda.empty_cache()
    egress = (world - 1) * GEMM_M * (GEMM_N // world) * 4  # bytes each rank stores to peers
    if mc_ms is not None:
        multimem = {"ms": round(mc_ms, 4), "value": round(GEMM_FLOPS / (mc_ms / 1e3) / 1e12, 2),
                    "c_identical_all_ranks": bool(same[2].item()),
                    "multicast_store_bytes_per_rank": GEMM_M * (GEMM_N // world) * 4,
                    "ingress_GB/s_per_rank": round(egress / (mc_ms / 1e3) / 1e9, 1),
                    "step": "nplk_gemm_allgather with NPLK_GEMM_MULTIMEM_STORES: every rank's C "
                            "bound to one NVLink multicast object (symmetric memory); the "
                            "epilogue stores each tile once (multimem.st) and NVSwitch delivers "
                            "it to all ranks"}
    else:
        multimem = {"unavailable": mc_why}
    # The end-to-end value: the faster fused form whose C is bit-identical on
    # every rank.
    best_ms, best_form = fm, "fused (below): every rank holds the whole row-major C"
    if mc_ms is not None and bool(same[2].item()) and mc_ms < fm:
        best_ms = mc_ms
        best_form = "fused.multimem (below): every rank holds the whole row-major C"
    return {"workload": f"npl_matmul fp32 [8192x4096]@[4096x16384] + bias, B/C column-sharded "
                        f"over {world} GPUs",
            "gemm_only_value": round(GEMM_FLOPS / (gm / 1e3) / 1e12, 2),
            "end_to_end_value": round(GEMM_FLOPS / (best_ms / 1e3) / 1e12, 2), "unit": "TFLOP/s",
            "end_to_end": best_form,
            "gemm_ms": round(gm, 4),
            "nccl": {"gemm_allgather_relayout_ms": round(tm, 4),
                     "c_identical_all_ranks": bool(same[1].item()),
                     "value": round(GEMM_FLOPS / (tm / 1e3) / 1e12, 2),
                     "step": "GEMM, then NCCL all-gather of the [g][M][N/g] blocks, then the "
                             "relayout kernel"},
            "fused": {"ms": round(fm, 4), "value": round(GEMM_FLOPS / (fm / 1e3) / 1e12, 2),
                      "normwise_err_sampled_rows": ferr,
                      "c_identical_all_ranks": bool(same[0].item()),
                      "c_max_normwise_diff_all_ranks": float(diff.item()),
                      "peer_egress_bytes_per_rank": egress,
                      "peer_egress_GB/s_per_rank": round(egress / (fm / 1e3) / 1e9, 1),
                      "step": "nplk_gemm_allgather: the GEMM epilogue stores every tile into "
                              "all ranks' C over NVLink (CUDA IPC peer pointers) with 16-byte "
                              "stores from its threads",
                      "multimem": multimem,
                      "tma_stores": {"ms": round(tma_ms, 4),
                                     "value": round(GEMM_FLOPS / (tma_ms / 1e3) / 1e12, 2),
                                     "step": "the same with one TMA tensor store per 32x32 piece "
                                             "and destination (NPLK_GEMM_PEER_TMA_STORES)"}},
            "normwise_err_sampled_rows": err}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-gemm", action="store_true")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        r = reference_cpu(args.steps, args.warmup)
        if r is None:
            print(json.dumps({"impl": "reference",
                              "unavailable": "oracle/_ref/libnpl_ref.so was not built"}))
            return
        tflops, cores, sample, med, _ = r
        print(json.dumps({
            "impl": "reference",
            "metric": "fused conv2d+BN+ReLU TFLOP/s (npl_conv2d_bn_activation, 3xTF32)",
            "value": round(tflops, 5), "unit": "TFLOP/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(med * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded; the benchmark workload's shapes and value distributions)",
            "config": {"workload": WORKLOAD, "per_gpu_batch": N_IMG,
                       "global_batch": N_IMG, "parallelism": "host CPU (reference build)"},
            "cpu_baseline": {"value": round(tflops, 5), "unit": "TFLOP/s", "cores": cores,
                             "kind": "reference", "sample": sample},
            "e2e": {"value": round(tflops, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
        }))
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        lib, result = run_b200(args, rank, world, local_rank)
        if world > 1 and not args.no_gemm:
            gd = gemm_dist(args, rank, world, local_rank)
            if rank == 0:
                result["also"] = {"gemm_column_sharded": gd}
        strong = strong_scaling_also(lib, rank, world, local_rank)
        if rank == 0:
            result.setdefault("also", {})["conv_strong_scaling"] = strong
        if rank == 0:
            if world == 1 and not args.no_gemm:
                result["also"].update({"gemm": gemm_also(lib, args, local_rank),
                                       "gemm_1024": gemm1024_also(lib, local_rank),
                                       "stem": stem_also(lib, local_rank),
                                       "bandwidth": bandwidth_also(lib, local_rank)})
            if world == 1:
                r = reference_cpu(3, 1, rows=not args.no_gemm)
                if r is not None:
                    tflops, cores, sample, _, ref_rows = r
                    result["cpu_baseline"] = {"value": round(tflops, 5), "unit": "TFLOP/s",
                                              "cores": cores, "kind": "reference",
                                              "sample": sample}
                    if ref_rows is not None and "also" in result:
                        result["also"]["cpu_reference_rows"] = ref_rows
            print(json.dumps(result))
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
