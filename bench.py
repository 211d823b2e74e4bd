#!/usr/bin/env python
"""KVForge codec benchmark on B200.

Workload (default): Aggressive preset (INT4 KIVI, SVD projection at 75%
variance, rANS, calibration) compress + decompress of a Llama-3-8B-shaped KV
cache: 32 layers x keys and values [8 heads, 32768 tokens, 128] fp16, layer
seed 100 + l, low-rank (rank 24) + 0.1 N(0,1) noise, 4 outlier key channels per
head at U[8, 16]. Layers are sharded across ranks (one process per GPU); the
total work is fixed, so scaling is strong. The calibrated projection bases are
computed once per layer before timing (the basis step may stay outside the
timed path); the timed step is everything else, on the device, issued as one
replay of a CUDA graph that captured the step's library calls (--no-graph
issues them from the host every step).

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]

Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import ctypes as C
import datetime
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "KV compress+decompress GB/s (fp16 K+V input bytes per second), Aggressive preset"
UNIT = "GB/s"
GB = 1e9


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def _traffic(kernel: str):
    """Per-launch DRAM traffic (read + write bytes) of `kernel` from the committed
    ncu summary (profiles/kernel_traffic.json); None when absent."""
    path = os.path.join(ROOT, "profiles", "kernel_traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(kernel)
    except Exception:
        return None


def kernel_rooflines(lib, L, K, torch, lay, dev, cfg, reps=20):
    """Isolated launches of the step's bandwidth-bound kernels on layer 0, timed
    with CUDA events on their own stream: value/key projection (+ per-token INT4
    quantization for values), standalone calibration of the keys, and value/key
    reconstruction on both engines. (The rANS coders return their container
    length to the host, so they are timed per stage by stage_rooflines.)
    Algorithmic bytes per launch: inputs read once plus outputs written once."""
    _, k, v, kb, vb = lay
    H, T, D = k.shape
    st = torch.cuda.Stream(device=dev)
    sp = C.c_void_p(st.cuda_stream)
    ctx = L.context(dev)
    P = lambda t: C.c_void_p(t.data_ptr())
    res = []

    def timed(fn):
        with torch.cuda.stream(st):
            for _ in range(3):
                fn()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            for _ in range(reps):
                fn()
            e1.record(st)
        e1.synchronize()
        return e0.elapsed_time(e1) / reps

    if kb is None:  # no projection (Conservative): KIVI quantize and dequantize of the raw tensors
        in_code = L.IN_F16 if k.dtype == torch.float16 else L.IN_F32
        dt = cfg.key_data_type
        n = H * T * D
        plen = (n + 1) // 2 if dt == L.INT4 else n
        packed = torch.empty(plen, dtype=torch.uint8, device=k.device)
        out = torch.empty((H, T, D), dtype=torch.float32, device=k.device)
        for name, x, axis in (("quantize_keys_per_channel", k, L.PER_CHANNEL), ("quantize_values_per_token", v, L.PER_TOKEN)):
            npar = H * D if axis == L.PER_CHANNEL else H * T
            sc = torch.empty(npar, device=k.device)
            mn = torch.empty(npar, device=k.device)
            ms = timed(lambda: L.check(lib.kvf_quantize(ctx, P(x), in_code, H, T, D, dt, axis, P(packed), P(sc), P(mn),
                                                        sp)))
            res.append({"name": name, "kernel": "kvf_quantize (KIVI codes + params)", "R": None,
                        "bytes": x.numel() * x.element_size() + plen + 8 * npar, "ms": ms, "in_step": True})
            ms = timed(lambda: L.check(lib.kvf_dequantize(ctx, P(packed), plen, P(sc), P(mn), dt, axis, H, T, D,
                                                          P(out), sp)))
            res.append({"name": name.replace("quantize", "dequantize"), "kernel": "kvf_dequantize (f32 out)",
                        "R": None, "bytes": plen + 8 * npar + 4 * n, "ms": ms, "in_step": True})
        return res

    # the value projection on the tensor-core engines as well (exact codes, and
    # the approximate engine), timed beside the default CUDA-core kernel
    tc_engines = ((L.PROJ_TENSOR_CORE, "_tcgen05_exact", "k_project_tc<RG, true> (tcgen05 + exact min/max chains)"),
                  (L.PROJ_TENSOR_CORE_APPROX, "_tcgen05_approx",
                   "k_project_tc<RG, false> (tcgen05, approximate codes)"))
    for eng, suffix, kern_name in (tc_engines if v.dtype == torch.float16 and D == 128 and vb.R <= 64 else ()):
        R = vb.R
        n = H * T * R
        packed = torch.empty((n + 1) // 2, dtype=torch.uint8, device=v.device)
        sc = torch.empty(H * T, device=v.device)
        mn = torch.empty(H * T, device=v.device)
        L.check(lib.kvf_set_projection_engine(ctx, eng))
        try:
            ms = timed(lambda: L.check(lib.kvf_fused_project_quantize(
                ctx, P(v), 1, H, T, D, C.c_void_p(vb.device_vt()), C.c_void_p(vb.device_ranks()), R, 0, 1,
                P(packed), P(sc), P(mn), sp)))
        finally:
            L.check(lib.kvf_set_projection_engine(ctx, L.PROJ_AUTO))
        res.append({"name": "project_values_int4_per_token" + suffix, "kernel": kern_name,
                    "bytes": v.numel() * 2 + (n + 1) // 2 + 8 * H * T, "ms": ms, "R": R, "in_step": False})
    for name, x, b, per_token in (("project_values_int4_per_token", v, vb, True), ("project_keys", k, kb, False)):
        R = b.R
        if per_token:
            n = H * T * R
            packed = torch.empty((n + 1) // 2, dtype=torch.uint8, device=x.device)
            sc = torch.empty(H * T, device=x.device)
            mn = torch.empty(H * T, device=x.device)
            ms = timed(lambda: L.check(lib.kvf_fused_project_quantize(
                ctx, P(x), 1, H, T, D, C.c_void_p(b.device_vt()), C.c_void_p(b.device_ranks()), R, 0, 1, P(packed),
                P(sc), P(mn), sp)))
            nbytes = x.numel() * 2 + (n + 1) // 2 + 8 * H * T
            kern = "k_project (MODE 2: per-token INT4 epilogue)"
        else:
            Pk = torch.empty((H, T, R), dtype=torch.float32, device=x.device)
            ms = timed(lambda: L.check(lib.kvf_project(ctx, P(x), 1, H, T, D, C.c_void_p(b.device_vt()),
                                                       C.c_void_p(b.device_ranks()), R, P(Pk), sp)))
            nbytes = x.numel() * 2 + 4 * H * T * R
            kern = "k_project (MODE 0: coefficients)"
        res.append({"name": name, "kernel": kern, "bytes": nbytes, "ms": ms, "R": R, "in_step": True})
    # calibration on its own (the step fuses its sums into the key projection):
    # per-head fp64 sums of the key tensor, then the scores
    scores = torch.empty(H, dtype=torch.float32, device=k.device)
    ms = timed(lambda: L.check(lib.kvf_calibrate(ctx, P(k), L.IN_F16 if k.dtype == torch.float16 else L.IN_F32, H, T, D, 64,
                                                 P(scores), sp)))
    res.append({"name": "calibrate_keys", "kernel": "k_calib_partials + k_calib_finalize", "R": None,
                "bytes": k.numel() * k.element_size() + 4 * H, "ms": ms, "in_step": False})
    # both reconstruction engines; the step uses the default choice (CUDA cores
    # up to 16 coefficients, tensor cores above), the other is timed beside it
    for engine, eng_name in ((L.RECON_CUDA_CORE, "cuda_core"), (L.RECON_TENSOR_CORE, "tcgen05")):
        L.check(lib.kvf_set_reconstruct_engine(ctx, engine))
        try:
            for name, b in (("reconstruct_values", vb), ("reconstruct_keys", kb)):
                R = b.R
                in_step = (engine == L.RECON_TENSOR_CORE) == (R > 16)
                kern = ("k_reconstruct_tc (tcgen05 split-tf32)" if engine == L.RECON_TENSOR_CORE else
                        "k_reconstruct_reg (basis in registers)" if R <= 16 else
                        "k_dequant_reconstruct (basis in shared memory)")
                Pc = torch.zeros((H, T, R), dtype=torch.float32, device=k.device)
                out = torch.empty((H, T, D), dtype=torch.float32, device=k.device)
                ms = timed(lambda: L.check(lib.kvf_reconstruct(ctx, P(Pc), H, T, R, D, C.c_void_p(b.device_vt()),
                                                               C.c_void_p(b.device_ranks()), P(out), sp)))
                res.append({"name": name + ("" if in_step else f"_{eng_name}"), "kernel": kern + ", f32 coefficients",
                            "bytes": 4 * H * T * R + 4 * H * T * D, "ms": ms, "R": R, "in_step": in_step})
        finally:
            L.check(lib.kvf_set_reconstruct_engine(ctx, L.RECON_AUTO))
    return res


def stage_rooflines(lib, L, torch, lay, dev, cfg, in_code, H, T, D, reps=10):
    """Per-stage device time of one layer's compress + decompress (layer 0,
    one caller stream; the library runs the value tensor on a side stream),
    from the library's stage events, against each stage's algorithmic bytes:
    the rANS coders read the packed codes and write the container (encode) or
    the reverse (decode); the other stages use the library's own byte counts."""
    l, k, v, kb, vb = lay
    st = torch.cuda.Stream(device=dev)
    sp = C.c_void_p(st.cuda_stream)
    ctx = L.context(dev)

    def compress():
        h = C.c_void_p()
        L.check(lib.kvf_compress_layer(ctx, C.c_void_p(k.data_ptr()), C.c_void_p(v.data_ptr()), in_code, H, T, D, l,
                                       C.byref(cfg), kb.handle if kb else None, vb.handle if vb else None,
                                       C.byref(h), sp))
        return h

    ko = torch.empty((H, T, D), dtype=torch.float32, device=f"cuda:{dev}")
    vo = torch.empty_like(ko)
    h = compress()
    ent_bytes = 0
    for which in (0, 1):
        R, pl, dl, he = C.c_size_t(), C.c_size_t(), C.c_size_t(), C.c_int32()
        L.check(lib.kvf_compressed_tensor_info(h, which, C.byref(R), C.byref(pl), C.byref(dl), C.byref(he)))
        if he.value:
            ent_bytes += pl.value + dl.value
    lib.kvf_compressed_free(h)
    L.check(lib.kvf_sync(ctx, sp))
    L.check(lib.kvf_profile_enable(ctx, 1))
    L.profile_read(dev)
    try:
        for _ in range(reps):
            h = compress()
            L.check(lib.kvf_decompress_layer(ctx, h, C.c_void_p(ko.data_ptr()), C.c_void_p(vo.data_ptr()), sp))
            lib.kvf_compressed_free(h)
        st.synchronize()
        prof = L.profile_read(dev)
    finally:
        L.check(lib.kvf_profile_enable(ctx, 0))
    L.check(lib.kvf_sync(ctx, sp))
    peak, _ = _peaks()
    out = []
    for name, (ms, cnt, nbytes) in prof.items():
        if not cnt:
            continue
        ms /= reps
        nb = ent_bytes if name.startswith("entropy") else nbytes / reps
        out.append({"stage": name, "ms_per_layer": ms, "launch_groups_per_layer": cnt / reps, "bytes": nb,
                    "achieved_gbs": nb / (ms / 1e3) / GB if ms > 0 else None,
                    "frac": nb / (ms / 1e3) / GB / peak if ms > 0 else None})
    return out


def decode_attention_leg(lib, L, torch, lay, dev, cfg, in_code, H, T, D, reps=20):
    """Decode attention of one query row per head on compressed layer 0
    (kvf_compressed_attention: rANS decode of both tensors into scratch, then
    attention on the codes), against decompress + f32 attention in torch on
    the reconstructed layer; error against fp64 attention on the exactly
    reconstructed layer. CUDA events on the launching stream."""
    l, k, v, kb, vb = lay
    st = torch.cuda.current_stream(dev)
    sp = C.c_void_p(st.cuda_stream)
    ctx = L.context(dev)
    h = C.c_void_p()
    L.check(lib.kvf_compress_layer(ctx, C.c_void_p(k.data_ptr()), C.c_void_p(v.data_ptr()), in_code, H, T, D, l,
                                   C.byref(cfg), kb.handle if kb else None, vb.handle if vb else None, C.byref(h), sp))
    q = torch.randn((H, D), generator=torch.Generator(device=f"cuda:{dev}").manual_seed(7), device=f"cuda:{dev}")
    out = torch.empty((H, D), dtype=torch.float32, device=f"cuda:{dev}")
    ko = torch.empty((H, T, D), dtype=torch.float32, device=f"cuda:{dev}")
    vo = torch.empty_like(ko)
    scale = 1.0 / float(np.sqrt(D))

    def fused():
        L.check(lib.kvf_compressed_attention(ctx, h, C.c_void_p(q.data_ptr()), C.c_float(scale),
                                             C.c_void_p(out.data_ptr()), sp))

    def unfused():
        L.check(lib.kvf_decompress_layer(ctx, h, C.c_void_p(ko.data_ptr()), C.c_void_p(vo.data_ptr()), sp))
        p = torch.softmax(torch.einsum("htd,hd->ht", ko, q) * scale, dim=1)
        return torch.einsum("ht,htd->hd", p, vo)

    res = {}
    for name, f in (("fused_ms", fused), ("decompress_then_attention_ms", unfused)):
        for _ in range(3):
            f()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        for _ in range(reps):
            f()
        b.record(st)
        torch.cuda.synchronize()
        res[name] = a.elapsed_time(b) / reps
    fused()
    L.check(lib.kvf_set_exact_reconstruct(ctx, 1))
    try:
        L.check(lib.kvf_decompress_layer(ctx, h, C.c_void_p(ko.data_ptr()), C.c_void_p(vo.data_ptr()), sp))
    finally:
        L.check(lib.kvf_set_exact_reconstruct(ctx, 0))
    s = torch.einsum("htd,hd->ht", ko.double(), q.double()) * scale
    ref = torch.einsum("ht,htd->hd", torch.softmax(s, dim=1), vo.double())
    unf = unfused().double()
    torch.cuda.synchronize()
    res["rel_err_fused_vs_fp64"] = float((out.double() - ref).norm() / ref.norm())
    res["rel_err_decompress_then_f32_attention_vs_fp64"] = float((unf - ref).norm() / ref.norm())
    n = C.c_size_t()
    L.check(lib.kvf_compressed_size_bytes(h, C.byref(n)))
    res["compressed_bytes_read"] = int(n.value)
    res["f32_kv_bytes_avoided"] = int(2 * H * T * D * 4)
    res["query_rows"] = H
    lib.kvf_compressed_free(h)
    L.check(lib.kvf_sync(ctx, sp))
    return res


class ClockSampler:
    """SM clock, power and clock-event (throttle) reasons of one GPU, sampled
    in-process with read-only NVML queries every `period` seconds on a
    background thread; nvidia-smi polling (200 ms) when NVML is not importable.
    The device is matched to the CUDA ordinal by UUID."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"),
               ("hw_power_brake_slowdown", "nvmlClocksEventReasonHwPowerBrakeSlowdown"))
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int, period: float = 0.01):
        self.device = device
        self.period = period
        self.samples = []  # (sm_mhz, power_w, reasons bitmask)
        self.lines = []
        self.proc = None
        self.nv = None
        self.handle = None
        self.max_mhz = None
        self.stop_flag = threading.Event()
        self.t = None
        self.source = None

    def _open_nvml(self):
        import pynvml as nv
        import torch
        nv.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(self.device).uuid)
        uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
        try:
            h = nv.nvmlDeviceGetHandleByUUID(uuid)
        except Exception:
            h = nv.nvmlDeviceGetHandleByIndex(self.device)
        self.nv, self.handle = nv, h
        self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))

    def _sample_nvml(self):
        nv, h = self.nv, self.handle
        while not self.stop_flag.is_set():
            try:
                self.samples.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                                     nv.nvmlDeviceGetPowerUsage(h) / 1000.0,
                                     int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))))
            except Exception:
                pass
            self.stop_flag.wait(self.period)

    def start(self):
        try:
            self._open_nvml()
            self.source = f"NVML in-process, every {self.period * 1e3:.0f} ms"
            self.t = threading.Thread(target=self._sample_nvml, daemon=True)
            self.t.start()
            return
        except Exception:
            self.nv = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.device)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.source = "nvidia-smi, every 200 ms"
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.time()
            while not self.lines and time.time() - t0 < 5.0 and self.proc.poll() is None:
                time.sleep(0.01)  # sampling is live before the timed region starts
            self.lines.clear()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.nv is not None:
            self.stop_flag.set()
            self.t.join(timeout=2)
            sm = [a for a, _, _ in self.samples]
            pw = [b for _, b, _ in self.samples]
            reasons = set()
            for _, _, bits in self.samples:
                for name, attr in self.REASONS:
                    if bits & int(getattr(self.nv, attr, 0)):
                        reasons.add(name)
            try:
                self.nv.nvmlShutdown()
            except Exception:
                pass
            return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": self.max_mhz,
                    "power_w_max": max(pw) if pw else None, "samples": len(sm), "reasons": sorted(reasons),
                    "source": self.source}
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock sampling unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, mx, pw, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
                pw.append(float(parts[3]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(pw) if pw else None, "samples": len(sm), "reasons": sorted(reasons),
                "source": self.source}


def entropy_accounting(lib, L, K, h, dev) -> dict:
    """Bytes of the entropy-coded data of one compressed layer (both tensors):
    this library's chunked multi-lane container (KVR2) as written, against
    what the reference's one serial rANS stream would take for the same codes
    (crates/kvforge-cpu/src/entropy.rs:24-86): the cross-entropy of the codes
    under the reference's model p_s = (f_s + 1) / sum(f + 1) in whole 32-bit
    words plus the coder's 64-bit final state (an estimate: constriction 0.4,
    which the reference calls, is not available to run), and the codes'
    empirical entropy (the Shannon bound of any order-0 coder)."""
    out = {"kvr2": 0, "single_stream": 0, "shannon": 0.0}
    for which in (0, 1):
        R, pl, dl, he = C.c_size_t(), C.c_size_t(), C.c_size_t(), C.c_int32()
        L.check(lib.kvf_compressed_tensor_info(h, which, C.byref(R), C.byref(pl), C.byref(dl), C.byref(he)))
        ptrs = [C.c_void_p() for _ in range(6)]
        L.check(lib.kvf_compressed_tensor_views(h, which, *[C.byref(p) for p in ptrs]))
        if not he.value or not ptrs[3].value:
            continue
        f = K._view(ptrs[3].value, (256,), "<u4", dev).cpu().numpy().astype(np.float64)
        n = f.sum()
        p_ref = (f + 1.0) / (f.sum() + 256.0)
        xent = float(-(f * np.log2(p_ref)).sum())
        nz = f > 0
        shannon = float(-(f[nz] * np.log2(f[nz] / n)).sum())
        out["kvr2"] += dl.value
        out["single_stream"] += 4 * int(np.ceil(xent / 32.0)) + 8
        out["shannon"] += shannon / 8.0
    return out


def _dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


# ---------------------------------------------------------------------------
# CPU legs (the oracle: a C restatement of the reference CPU crate)
# ---------------------------------------------------------------------------
def _oracle_time(O, keys, values, bases, preset, threads, min_seconds, max_reps):
    """Times oracle compress + decompress of one layer (basis given)."""
    reps, t0 = 0, time.perf_counter()
    while True:
        c = O.compress(keys, values, preset, 0, bases, threads=threads)
        O.decompress(c, threads=threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= min_seconds or reps >= max_reps:
            return el / reps, O.ratio(c)


def cpu_baseline(workload, k16, v16, bases, threads=1, min_seconds=10.0):
    from oracle import oracle as O
    O.build()
    k = k16.astype(np.float32)
    v = v16.astype(np.float32)
    w = workload
    sec, ratio = _oracle_time(O, k, v, bases, w["preset"], threads, min_seconds, 5)
    nbytes = k16.nbytes + v16.nbytes
    return {"value": nbytes / sec / GB, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"1 layer [{k.shape[0]},{k.shape[1]},{k.shape[2]}] fp16 K+V ({nbytes / 2**20:.0f} MiB), "
                      f"compress+decompress with the calibrated basis, {threads} thread(s), "
                      f"{sec:.2f} s per layer", "ratio": ratio}


def reference_arm(args):
    rank, world, _ = _dist_env()
    if rank != 0:
        return 0
    from kvforge_b200 import synth
    from oracle import oracle as O
    O.build()
    w = dict(synth.WORKLOADS[args.workload])
    threads = os.cpu_count() or 1
    k16, v16 = synth.workload_layer(args.workload, 0, backend="numpy")
    k, v = k16.astype(np.float32), v16.astype(np.float32)
    thr = O.PRESETS[w["preset"]]["thr"]
    bases = None
    if O.PRESETS[w["preset"]]["proj"]:
        bases = (O.basis_for(k, thr, threads=threads), O.basis_for(v, thr, threads=threads))
    for _ in range(args.warmup):
        c = O.compress(k, v, w["preset"], 0, bases, threads=threads)
        O.decompress(c, threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        c = O.compress(k, v, w["preset"], 0, bases, threads=threads)
        O.decompress(c, threads=threads)
    sec = (time.perf_counter() - t0) / args.steps
    nbytes = k16.nbytes + v16.nbytes
    val = nbytes / sec / GB
    line = {
        "impl": "reference", "metric": METRIC, "value": val, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": _config(args, w),
        "ratio": O.ratio(c),
        "cpu_baseline": {"value": val, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"layer 0 of the workload ([{k.shape[0]},{k.shape[1]},{k.shape[2]}] fp16 K+V, "
                                   f"{nbytes / 2**20:.0f} MiB) per step, CPU oracle (C restatement of the "
                                   f"reference crate; Rust is not installed) with {threads} OpenMP threads, "
                                   f"calibrated basis precomputed"},
        "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def _config(args, w):
    return {"workload": args.workload, "preset": w["preset"], "layers": args.layers or w.get("layers", 1),
            "heads": w["H"], "tokens": w["T"], "head_dim": w["D"], "input_dtype": w["dtype"],
            "output_dtype": "f32", "basis": "calibrated per layer, computed before the timed region",
            "l2": "inputs larger than L2 (no flush)", "parallelism": f"layer-sharded x{args.gpus}",
            "streams_per_gpu": getattr(args, "streams", 1), "order": getattr(args, "order", "interleaved"),
            "cuda_graph": bool(getattr(args, "graph", False))}


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def gpu_arm(args):
    import torch
    rank, world, local = _dist_env()
    torch.cuda.set_device(local)
    dev = local
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device(f"cuda:{dev}"))
    import kvforge_b200 as K
    from kvforge_b200 import _lib as L
    from kvforge_b200 import synth
    from kvforge_b200.dist import gather_stats, layer_shard, reduce_stats

    w = dict(synth.WORKLOADS[args.workload])
    n_layers = args.layers or w.get("layers", 1)
    mine = list(layer_shard(n_layers, world, rank))
    lib = L.lib()
    ctx = L.context(dev)
    cfg = K.config_from_preset(w["preset"])
    H, T, D = w["H"], w["T"], w["D"]
    in_code = L.IN_F16 if w["dtype"] == "float16" else L.IN_F32

    # inputs (device-resident, generated on the GPU) and calibrated bases
    layers = []
    t_basis = 0.0
    for l in mine:
        k, v = synth.workload_layer(args.workload, l, backend="torch", device=f"cuda:{dev}")
        kb = vb = None
        if cfg.enable_projection:
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            kb = K.Basis.compute(k, cfg.projection_variance_threshold, device=dev)
            vb = K.Basis.compute(v, cfg.projection_variance_threshold, device=dev)
            t_basis += time.perf_counter() - t0
        layers.append((l, k, v, kb, vb))
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    sptr = C.c_void_p(stream.cuda_stream)
    # layers are issued round-robin on several streams, each with its own output
    # buffers, so one layer's latency-bound entropy coding overlaps another
    # layer's bandwidth-bound projection and reconstruction
    nstreams = max(1, min(args.streams, len(layers)))
    workers = [torch.cuda.Stream(device=dev) for _ in range(nstreams)]
    wptr = [C.c_void_p(s.cuda_stream) for s in workers]
    outs = [(torch.empty((H, T, D), dtype=torch.float32, device=f"cuda:{dev}"),
             torch.empty((H, T, D), dtype=torch.float32, device=f"cuda:{dev}")) for _ in range(nstreams)]
    ko, vo = outs[0]

    def compress(l, k, v, kb, vb, wi=0):
        h = C.c_void_p()
        L.check(lib.kvf_compress_layer(ctx, C.c_void_p(k.data_ptr()), C.c_void_p(v.data_ptr()), in_code, H, T, D, l,
                                       C.byref(cfg), kb.handle if kb else None, vb.handle if vb else None,
                                       C.byref(h), wptr[wi]))
        return h

    def decompress(h, wi=0):
        L.check(lib.kvf_decompress_layer(ctx, h, C.c_void_p(outs[wi][0].data_ptr()),
                                         C.c_void_p(outs[wi][1].data_ptr()), wptr[wi]))

    def run_layer(l, k, v, kb, vb, keep=False, wi=0):
        h = compress(l, k, v, kb, vb, wi)
        decompress(h, wi)
        if keep:
            return h
        lib.kvf_compressed_free(h)
        return None

    start_ev = torch.cuda.Event()
    done_ev = [torch.cuda.Event() for _ in workers]

    # the issuing stream is looked up at call time: inside a CUDA graph
    # capture it is the capture stream
    def fork():
        cur = torch.cuda.current_stream(dev)
        start_ev.record(cur)
        for w in workers:
            w.wait_event(start_ev)

    def join():
        cur = torch.cuda.current_stream(dev)
        for w, e in zip(workers, done_ev):
            e.record(w)
            cur.wait_event(e)

    def step():
        fork()
        if args.order == "phased":
            # every layer's compression is issued before any decompression:
            # with few layers per stream the rANS coders of one layer no longer
            # wait behind another layer's reconstruction
            hs = [compress(*lay, wi=i % nstreams) for i, lay in enumerate(layers)]
            for i, h in enumerate(hs):
                decompress(h, wi=i % nstreams)
            for h in hs:
                lib.kvf_compressed_free(h)
        else:
            for i, lay in enumerate(layers):
                run_layer(*lay, wi=i % nstreams)
        join()

    for _ in range(args.warmup):
        step()
    L.check(lib.kvf_sync(ctx, sptr))

    # ratio, sizes and reconstruction error of this rank's layers (untimed)
    comp_bytes = 0
    err = {"err2_k": 0.0, "ref2_k": 0.0, "err2_v": 0.0, "ref2_v": 0.0}
    ent = {"kvr2": 0, "single_stream": 0, "shannon": 0.0}
    for lay in layers:
        h = run_layer(*lay, keep=True)
        torch.cuda.synchronize()
        n = C.c_size_t()
        L.check(lib.kvf_compressed_size_bytes(h, C.byref(n)))
        comp_bytes += n.value
        for k2, v2 in entropy_accounting(lib, L, K, h, dev).items():
            ent[k2] += v2
        kf, vf = lay[1].float(), lay[2].float()
        err["err2_k"] += float(((ko - kf) ** 2).sum())
        err["ref2_k"] += float((kf ** 2).sum())
        err["err2_v"] += float(((vo - vf) ** 2).sum())
        err["ref2_v"] += float((vf ** 2).sum())
        lib.kvf_compressed_free(h)
    torch.cuda.synchronize()
    L.check(lib.kvf_sync(ctx, sptr))
    in_bytes = sum(lay[1].numel() * lay[1].element_size() * 2 for lay in layers)
    orig_bytes = len(layers) * 2 * H * T * D * 4

    # by default one step (every library call of every layer, all streams) is
    # captured once as a CUDA graph and each warm-up and timed step replays it:
    # the GPU runs the same kernels, with one host launch per step instead of
    # hundreds of API calls (with 8 ranks on one host the per-call issue cost
    # had left each GPU waiting); --no-graph issues every call from the host
    # clocks are sampled from here (the graph's warm-up replays) to the end of
    # the timed region, so short timed regions still carry samples under load
    clocks = ClockSampler(dev)
    clocks.start()
    graph, graph_launches, graph_err = None, None, None
    if args.graph:
        torch.cuda.synchronize()
        na = lib.kvf_launch_count()
        g = torch.cuda.CUDAGraph()
        try:
            with torch.cuda.graph(g, capture_error_mode="relaxed"):
                step()
            graph, graph_launches = g, lib.kvf_launch_count() - na
            for _ in range(args.warmup):
                graph.replay()
        except Exception as ex:  # capture refused: eager steps, reported in the line
            graph_err = str(ex).splitlines()[0][:200]
            graph = None
        torch.cuda.synchronize()
        L.check(lib.kvf_sync(ctx, sptr))

    def run_step():
        if graph is not None:
            graph.replay()
        else:
            step()

    # timed region
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()
    n0 = lib.kvf_launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    h0 = time.perf_counter()
    for _ in range(args.steps):
        run_step()
    host_issue_ms = 1e3 * (time.perf_counter() - h0) / args.steps
    e1.record(stream)
    torch.cuda.synchronize()
    n1 = lib.kvf_launch_count()
    if graph is not None:  # the library counts launches when they are issued: once, at capture
        n1 = n0 + graph_launches * args.steps
    ms = e0.elapsed_time(e1) / args.steps
    clk = clocks.stop()
    L.check(lib.kvf_sync(ctx, sptr))

    # per-stage device times from the library's stage profiler, on separate
    # untimed steps (its events would perturb the timed ones)
    L.check(lib.kvf_profile_enable(ctx, 1))
    L.profile_read(dev)
    prof_steps = max(1, min(args.steps, 5))
    for _ in range(prof_steps):
        step()
    torch.cuda.synchronize()
    prof = L.profile_read(dev)
    L.check(lib.kvf_profile_enable(ctx, 0))
    L.check(lib.kvf_sync(ctx, sptr))
    if world > 1:
        import torch.distributed as dist
        dist.barrier()

    # compress-only and decompress-only passes over the same layers and streams
    # (untimed warm-up pass first); the handles of all layers stay alive between them
    def split_pass():
        handles = [None] * len(layers)

        def comp():
            fork()
            for i, lay in enumerate(layers):
                handles[i] = compress(*lay, wi=i % nstreams)
            join()

        def decomp():
            fork()
            for i in range(len(layers)):
                decompress(handles[i], wi=i % nstreams)
            join()

        t = []
        for f in (comp, decomp):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            f()
            b.record(stream)
            t.append((a, b))
        torch.cuda.synchronize()
        for h in handles:
            lib.kvf_compressed_free(h)
        return [a.elapsed_time(b) for a, b in t]

    split_pass()
    split_ms = np.mean([split_pass() for _ in range(max(1, min(args.steps, 10)))], axis=0)

    # end-to-end through the host-buffer C-ABI entry points: pinned host inputs
    # in, f32 host outputs back, every step. The entry points return only when
    # their host buffers are complete, so layers are spread over a few host
    # threads, each with its own stream and output buffers: one layer's
    # host->device copy overlaps another's device->host copy and compute.
    e2e = None
    if args.e2e_steps > 0:
        kh = [torch.empty((H, T, D), dtype=lay[1].dtype, pin_memory=True) for lay in layers]
        vh = [torch.empty((H, T, D), dtype=lay[2].dtype, pin_memory=True) for lay in layers]
        for i, lay in enumerate(layers):
            kh[i].copy_(lay[1])
            vh[i].copy_(lay[2])
        nthr = max(1, min(args.e2e_threads, len(layers)))
        estreams = [torch.cuda.Stream(device=dev) for _ in range(nthr)]
        eouts = [(torch.empty((H, T, D), dtype=torch.float32, pin_memory=True),
                  torch.empty((H, T, D), dtype=torch.float32, pin_memory=True)) for _ in range(nthr)]
        errs = []

        def e2e_worker(j):
            try:
                sp = C.c_void_p(estreams[j].cuda_stream)
                koh, voh = eouts[j]
                for i in range(j, len(layers), nthr):
                    l, _, _, kb, vb = layers[i]
                    h = C.c_void_p()
                    L.check(lib.kvf_compress_layer_host(ctx, C.c_void_p(kh[i].data_ptr()), C.c_void_p(vh[i].data_ptr()),
                                                        in_code, H, T, D, l, C.byref(cfg), kb.handle if kb else None,
                                                        vb.handle if vb else None, C.byref(h), sp))
                    L.check(lib.kvf_decompress_layer_host(ctx, h, C.c_void_p(koh.data_ptr()),
                                                          C.c_void_p(voh.data_ptr()), sp))
                    lib.kvf_compressed_free(h)
            except Exception as ex:  # reported after the join
                errs.append(ex)

        def e2e_step():
            ts = [threading.Thread(target=e2e_worker, args=(j,)) for j in range(nthr)]
            for t in ts:
                t.start()
            for t in ts:
                t.join()
            if errs:
                raise errs[0]

        e2e_step()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        e0.record(stream)
        for es in estreams:
            es.wait_event(e0)
        for _ in range(args.e2e_steps):
            e2e_step()
        for es in estreams:
            ev = torch.cuda.Event()
            ev.record(es)
            stream.wait_event(ev)
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1) / args.e2e_steps
        e2e_wall_ms = (time.perf_counter() - t0) * 1e3 / args.e2e_steps
        e2e = {"ms": e2e_ms, "h2d": in_bytes, "d2h": orig_bytes}
    else:
        e2e_ms = float("nan")
        e2e_wall_ms = float("nan")

    stats = {"layers": len(layers), "input_bytes": in_bytes, "compressed_bytes": comp_bytes,
             "original_bytes": orig_bytes, "ms": ms, "compress_ms": float(split_ms[0]),
             "decompress_ms": float(split_ms[1]), **err, "ent_kvr2": ent["kvr2"],
             "ent_single": ent["single_stream"], "ent_shannon": ent["shannon"]}
    per = gather_stats(stats, device=f"cuda:{dev}" if world > 1 else None)
    tot = reduce_stats(per)
    e2e_per = gather_stats({"ms": e2e_ms, "input_bytes": in_bytes, "original_bytes": orig_bytes},
                           device=f"cuda:{dev}" if world > 1 else None)
    e2e_tot = reduce_stats(e2e_per)

    kr = kernel_rooflines(lib, L, K, torch, layers[0], dev, cfg) if rank == 0 else []
    sr = stage_rooflines(lib, L, torch, layers[0], dev, cfg, in_code, H, T, D) if rank == 0 else []
    attn = decode_attention_leg(lib, L, torch, layers[0], dev, cfg, in_code, H, T, D) if rank == 0 else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        lay = layers[0]
        bases = None
        if lay[3] is not None:
            kbh, vbh = lay[3].host(), lay[4].host()
            bases = ((kbh[0], kbh[1]), (vbh[0], vbh[1]))
        cpu = cpu_baseline(w, lay[1].cpu().numpy(), lay[2].cpu().numpy(), bases, threads=1,
                           min_seconds=args.cpu_seconds)

    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0

    peak, peak_kind = _peaks()
    step_ms = tot["ms"]
    value = tot["input_bytes"] / (step_ms / 1e3) / GB
    # algorithmic bytes per step: inputs + compressed (written) + compressed (read) + f32 outputs
    alg = tot["input_bytes"] + 2 * tot["compressed_bytes"] + tot["original_bytes"]
    for r in kr:
        r["achieved_gbs"] = r["bytes"] / (r["ms"] / 1e3) / GB
        r["frac"] = r["achieved_gbs"] / peak
    in_step = [r for r in kr if r["in_step"]]
    dom = max(in_step, key=lambda r: r["ms"]) if in_step else None
    roof = None
    if dom is not None:
        traffic = _traffic(dom["name"])
        roof = {"kernel": f'{dom["name"]}: {dom["kernel"]}', "bound": "hbm", "achieved": dom["achieved_gbs"],
                "peak": peak, "unit": "GB/s", "frac": dom["frac"],
                "traffic": traffic["bytes_per_launch"] if traffic else None,
                "algorithmic_bytes_per_launch": dom["bytes"], "avg_launch_ms": dom["ms"], "peak_kind": peak_kind,
                "timing": "isolated launches on layer 0 inside bench.py, CUDA events on the launching stream"}
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded low-rank + noise + outlier channels)",
        "config": _config(args, w),
        "ratio": tot["original_bytes"] / tot["compressed_bytes"],
        "rel_err": {"keys": (tot["err2_k"] / tot["ref2_k"]) ** 0.5, "values": (tot["err2_v"] / tot["ref2_v"]) ** 0.5},
        "entropy_coder": None if not tot["ent_kvr2"] else {
            "kvr2_bytes": int(tot["ent_kvr2"]),
            "single_stream_estimate_bytes": int(tot["ent_single"]),
            "shannon_bound_bytes": float(tot["ent_shannon"]),
            "ratio_single_stream": tot["original_bytes"] / (tot["compressed_bytes"] - tot["ent_kvr2"]
                                                             + tot["ent_single"]),
            "ratio_shannon_bound": tot["original_bytes"] / (tot["compressed_bytes"] - tot["ent_kvr2"]
                                                             + tot["ent_shannon"]),
            "note": "ratio with this library's chunked 32-lane rANS container (ratio) against the same layers with "
                    "the codes in the reference's single serial stream (estimated from the codes' cross-entropy "
                    "under its (f+1)-smoothed model) and at the order-0 Shannon bound"},
        # the job's bytes over the job's peak: one GPU's measured peak times the GPU count
        "step_roofline": {"algorithmic_bytes": alg, "achieved_gbs": alg / (step_ms / 1e3) / GB, "peak": peak * world,
                          "peak_per_gpu": peak, "frac": alg / (step_ms / 1e3) / GB / (peak * world),
                          "peak_kind": peak_kind},
        "roofline": roof,
        "kernel_rooflines": [{k2: r[k2] for k2 in ("name", "kernel", "R", "bytes", "ms", "achieved_gbs", "frac",
                                                   "in_step")} for r in kr],
        "stage_rooflines_layer0": sr,
        "compress_only": {"ms_per_step": tot["compress_ms"],
                          "gbs": tot["input_bytes"] / (tot["compress_ms"] / 1e3) / GB},
        "decompress_only": {"ms_per_step": tot["decompress_ms"],
                            "gbs": tot["input_bytes"] / (tot["decompress_ms"] / 1e3) / GB,
                            "output_gbs": tot["original_bytes"] / (tot["decompress_ms"] / 1e3) / GB},
        "decode_attention_layer0": attn,
        "stages_ms_per_step_overlapped": {k: v[0] / prof_steps for k, v in prof.items() if v[1]},
        "basis_ms_per_layer_untimed": 1e3 * t_basis / max(len(layers), 1),
        "host_issue_ms_per_step_rank0": host_issue_ms,
        "cuda_graph": None if not args.graph else {"replayed": graph is not None,
                                                   "launches_per_step": graph_launches, "capture_error": graph_err},
        "gpu_launches": int(n1 - n0),
        "clocks": clk,
    }
    if e2e is not None:
        e2e_val = e2e_tot["input_bytes"] / (e2e_tot["ms"] / 1e3) / GB
        line["e2e"] = {"value": e2e_val, "unit": UNIT, "h2d_bytes_per_step": int(e2e_tot["input_bytes"]),
                       "d2h_bytes_per_step": int(e2e_tot["original_bytes"]), "ms_per_step": e2e_tot["ms"],
                       "wall_ms_per_step_rank0": e2e_wall_ms,
                       "api": "kvf_compress_layer_host + kvf_decompress_layer_host (pinned host buffers), "
                              f"{args.e2e_threads} host threads with one stream each"}
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# Streaming append workload
# ---------------------------------------------------------------------------
STREAM_METRIC = ("KV append compress+decompress GB/s (fp16 K+V bytes of the appended chunks per second), "
                 "Balanced preset")


def stream_arm(args):
    """Llama-3-70B-shaped streaming cache, Balanced preset: 80 layers, each a
    16384-token prefix of keys and values [8, T, 128] fp16 (compressed before
    the timed region, which calibrates the layer's bases), then appends of 64
    tokens to every layer. Each chunk is compressed as its own CompressedKV and
    decompressed at once. A timed step is one append to every layer of this
    rank, projected onto the prefix's bases (basis reuse); the reference's
    semantics (a fresh eigen-basis per chunk, a synchronising host solve each)
    are timed beside it on a few steps. Layers are spread over host threads,
    each with its own stream: a 64-token chunk is launch-bound."""
    import torch
    rank, world, local = _dist_env()
    torch.cuda.set_device(local)
    dev = local
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device(f"cuda:{dev}"))
    import kvforge_b200 as K
    from kvforge_b200 import _lib as L
    from kvforge_b200 import synth
    from kvforge_b200.dist import gather_stats, layer_shard, reduce_stats

    w = dict(synth.WORKLOADS[args.workload])
    n_layers = args.layers or w.get("layers", 1)
    mine = list(layer_shard(n_layers, world, rank))
    lib, ctx = L.lib(), L.context(dev)
    cfg = K.config_from_preset(w["preset"])
    H, P, D, A = w["H"], w["T"], w["D"], w["append"]
    in_code = L.IN_F16 if w["dtype"] == "float16" else L.IN_F32
    n_chunks = max(1, min(w["appends"], args.warmup + args.steps))
    fresh_steps = max(1, min(args.steps, 3))

    # per layer: prefix compressed once (its bases kept), then a pool of chunks
    # [n_chunks, H, A, D] drawn from the same generator as the prefix
    layers = []
    t_prefix = 0.0
    for l in mine:
        x = synth.workload_layer(args.workload, l, backend="torch", device=f"cuda:{dev}", T=P + A * n_chunks)
        k, v = x
        kp, vp = k[:, :P].contiguous(), v[:, :P].contiguous()
        kc = k[:, P:].reshape(H, n_chunks, A, D).permute(1, 0, 2, 3).contiguous()
        vc = v[:, P:].reshape(H, n_chunks, A, D).permute(1, 0, 2, 3).contiguous()
        del x, k, v
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        h = C.c_void_p()
        L.check(lib.kvf_compress_layer(ctx, C.c_void_p(kp.data_ptr()), C.c_void_p(vp.data_ptr()), in_code, H, P, D,
                                       l, C.byref(cfg), None, None, C.byref(h), None))
        kb, vb = C.c_void_p(), C.c_void_p()
        L.check(lib.kvf_compressed_basis(h, 0, C.byref(kb)))
        L.check(lib.kvf_compressed_basis(h, 1, C.byref(vb)))
        L.check(lib.kvf_sync(ctx, None))
        lib.kvf_compressed_free(h)
        t_prefix += time.perf_counter() - t0
        del kp, vp
        layers.append((l, kc, vc, kb if kb.value else None, vb if vb.value else None))
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    nthr = max(1, min(args.streams, len(layers)))
    tstreams = [torch.cuda.Stream(device=dev) for _ in range(nthr)]
    touts = [(torch.empty((H, A, D), dtype=torch.float32, device=f"cuda:{dev}"),
              torch.empty((H, A, D), dtype=torch.float32, device=f"cuda:{dev}")) for _ in range(nthr)]
    errs = []

    def worker(j, a, reuse, keep):
        try:
            sp = C.c_void_p(tstreams[j].cuda_stream)
            ko, vo = touts[j]
            for i in range(j, len(layers), nthr):
                l, kc, vc, kb, vb = layers[i]
                h = C.c_void_p()
                L.check(lib.kvf_compress_layer(ctx, C.c_void_p(kc[a].data_ptr()), C.c_void_p(vc[a].data_ptr()),
                                               in_code, H, A, D, l, C.byref(cfg), kb if reuse else None,
                                               vb if reuse else None, C.byref(h), sp))
                L.check(lib.kvf_decompress_layer(ctx, h, C.c_void_p(ko.data_ptr()), C.c_void_p(vo.data_ptr()), sp))
                if keep is not None:
                    keep(i, h, ko, vo, sp)
                lib.kvf_compressed_free(h)
        except Exception as ex:  # reported after the join
            errs.append(ex)

    def append_step(a, reuse, keep=None):
        ts = [threading.Thread(target=worker, args=(j, a, reuse, keep)) for j in range(nthr)]
        for t_ in ts:
            t_.start()
        for t_ in ts:
            t_.join()
        if errs:
            raise errs[0]

    # batched: one kvf_compress_layers call per step for all layers of this
    # rank (one kernel launch), outputs per layer
    nl = len(layers)
    bouts = [(torch.empty((H, A, D), dtype=torch.float32, device=f"cuda:{dev}"),
              torch.empty((H, A, D), dtype=torch.float32, device=f"cuda:{dev}")) for _ in range(nl)]
    PA = C.c_void_p * max(nl, 1)
    b_idx = (C.c_size_t * max(nl, 1))(*[lay[0] for lay in layers])
    b_kb = PA(*[lay[3].value if lay[3] is not None else None for lay in layers])
    b_vb = PA(*[lay[4].value if lay[4] is not None else None for lay in layers])
    b_ko = PA(*[o[0].data_ptr() for o in bouts])
    b_vo = PA(*[o[1].data_ptr() for o in bouts])
    b_keys = [PA(*[lay[1][a].data_ptr() for lay in layers]) for a in range(n_chunks)]
    b_vals = [PA(*[lay[2][a].data_ptr() for lay in layers]) for a in range(n_chunks)]
    b_out = PA()
    sp_main = C.c_void_p(stream.cuda_stream)

    def batched_step(a, keep=None):
        L.check(lib.kvf_compress_layers(ctx, nl, b_keys[a], b_vals[a], in_code, H, A, D, b_idx, C.byref(cfg), b_kb,
                                        b_vb, b_out, b_ko, b_vo, sp_main))
        if keep is not None:
            for i in range(nl):
                keep(i, C.c_void_p(b_out[i]), bouts[i][0], bouts[i][1], sp_main)
        L.check(lib.kvf_compressed_free_many(b_out, nl))

    batched = args.stream_mode == "batched"

    host_ms = {}

    def timed(reuse, steps, a0, use_batch=False):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        if use_batch:
            h0 = time.perf_counter()
            for s in range(steps):
                batched_step((a0 + s) % n_chunks)
            host_ms["batched"] = 1e3 * (time.perf_counter() - h0) / steps
        else:
            for s_ in tstreams:
                s_.wait_event(e0)
            for s in range(steps):
                append_step((a0 + s) % n_chunks, reuse)
            for s_ in tstreams:
                ev = torch.cuda.Event()
                ev.record(s_)
                stream.wait_event(ev)
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    # sizes and reconstruction error of one append (untimed), both modes
    def measure(reuse):
        per_layer = []  # one tuple per layer from the worker threads (list.append is atomic)

        def keep(i, h, ko, vo, sp):
            L.check(lib.kvf_sync(ctx, sp))
            n, b = C.c_size_t(), C.c_size_t()
            L.check(lib.kvf_compressed_size_bytes(h, C.byref(n)))
            L.check(lib.kvf_compressed_basis_bytes(h, C.byref(b)))
            kf, vf = layers[i][1][0].float(), layers[i][2][0].float()
            per_layer.append((i, n.value - (b.value if reuse else 0), float(((ko - kf) ** 2).sum()),
                              float((kf ** 2).sum()), float(((vo - vf) ** 2).sum()), float((vf ** 2).sum())))

        if reuse and batched:
            batched_step(0, keep)
        else:
            append_step(0, reuse, keep)
        torch.cuda.synchronize()
        per_layer.sort()
        keys_ = ("comp", "err2_k", "ref2_k", "err2_v", "ref2_v")
        return {k2: sum(r[j + 1] for r in per_layer) for j, k2 in enumerate(keys_)}

    engines = {"auto": L.RECON_AUTO, "cuda": L.RECON_CUDA_CORE, "tc": L.RECON_TENSOR_CORE}
    L.check(lib.kvf_set_reconstruct_engine(ctx, engines[args.recon_engine]))
    meas = {r: measure(r) for r in (True, False)}
    for s in range(args.warmup):
        if batched:
            batched_step(s % n_chunks)
        else:
            append_step(s % n_chunks, True)
    L.check(lib.kvf_sync(ctx, None))
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(dev)
    clocks.start()
    n0 = lib.kvf_launch_count()
    ms = timed(True, args.steps, args.warmup, use_batch=batched)
    n1 = lib.kvf_launch_count()
    clk = clocks.stop()
    if world > 1:
        dist.barrier()
    # the same appends through the per-layer entry point (host threads, one
    # stream each), for comparison with the batched call
    ms_layers = None
    if batched:
        for s in range(2):
            append_step(s % n_chunks, True)
        L.check(lib.kvf_sync(ctx, None))
        if world > 1:
            dist.barrier()
        ms_layers = timed(True, max(3, min(args.steps, 20)), 0)
        if world > 1:
            t_ = torch.tensor([ms_layers], device=f"cuda:{dev}")
            dist.all_reduce(t_, op=dist.ReduceOp.MAX)
            ms_layers = float(t_.item())
    append_step(0, False)  # warm the fresh-basis path
    ms_fresh = timed(False, fresh_steps, 0)
    L.check(lib.kvf_sync(ctx, None))

    in_bytes = len(layers) * 2 * H * A * D * (2 if w["dtype"] == "float16" else 4)
    orig_bytes = len(layers) * 2 * H * A * D * 4
    per = {}
    for name, m, t_ms in (("reuse", meas[True], ms), ("fresh", meas[False], ms_fresh)):
        st = {"layers": len(layers), "input_bytes": in_bytes, "compressed_bytes": m["comp"],
              "original_bytes": orig_bytes, "ms": t_ms, **{k2: m[k2] for k2 in ("err2_k", "ref2_k", "err2_v",
                                                                               "ref2_v")}}
        per[name] = reduce_stats(gather_stats(st, device=f"cuda:{dev}" if world > 1 else None))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle as O
        O.build()
        k32 = layers[0][1][0].float().cpu().numpy()
        v32 = layers[0][2][0].float().cpu().numpy()
        sec, _ = _oracle_time(O, k32, v32, None, w["preset"], 1, min(args.cpu_seconds, 10.0), 2000)
        nb = 2 * H * A * D * 2
        cpu = {"value": nb / sec / GB, "unit": UNIT, "cores": 1, "kind": "port",
               "sample": f"one {A}-token chunk [{H},{A},{D}] fp16 K+V, compress+decompress with a fresh basis "
                         f"per chunk (the reference's semantics), 1 thread, {sec * 1e3:.2f} ms per chunk"}
    L.check(lib.kvf_set_reconstruct_engine(ctx, L.RECON_AUTO))
    for lay in layers:
        for b in lay[3:]:
            if b is not None:
                lib.kvf_basis_free(b)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    peak, peak_kind = _peaks()
    r, f = per["reuse"], per["fresh"]
    value = r["input_bytes"] / (r["ms"] / 1e3) / GB
    alg = r["input_bytes"] + 2 * r["compressed_bytes"] + r["original_bytes"]
    line = {
        "metric": STREAM_METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": r["ms"], "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded low-rank + noise + outlier channels)",
        "config": {"workload": args.workload, "preset": w["preset"], "layers": n_layers, "heads": H,
                   "prefix_tokens": P, "append_tokens": A, "head_dim": D, "input_dtype": w["dtype"],
                   "output_dtype": "f32", "basis": "the prefix's calibrated basis, reused by every chunk",
                   "step": "one append to every layer", "chunk_pool": n_chunks,
                   "l2": "chunks are L2-resident (256 KiB each); the step is latency-bound",
                   "parallelism": f"layer-sharded x{world}", "host_threads_per_gpu": 1 if batched else nthr,
                   "entry_point": "kvf_compress_layers (all layers of the rank in one call)" if batched
                   else "kvf_compress_layer + kvf_decompress_layer per layer",
                   "reconstruct_engine": "cuda (inside the batched kernel)" if batched else args.recon_engine},
        "tokens_per_s": A * r["layers"] / (r["ms"] / 1e3),
        "us_per_layer_append": 1e3 * r["ms"] / max(len(mine), 1),
        "ratio_amortized": r["original_bytes"] / r["compressed_bytes"],
        "rel_err": {"keys": (r["err2_k"] / r["ref2_k"]) ** 0.5, "values": (r["err2_v"] / r["ref2_v"]) ** 0.5},
        "fresh_basis": {"ms_per_step": f["ms"], "value": f["input_bytes"] / (f["ms"] / 1e3) / GB,
                        "ratio": f["original_bytes"] / f["compressed_bytes"],
                        "rel_err": {"keys": (f["err2_k"] / f["ref2_k"]) ** 0.5,
                                    "values": (f["err2_v"] / f["ref2_v"]) ** 0.5}, "steps": fresh_steps},
        "step_roofline": {"algorithmic_bytes": alg, "achieved_gbs": alg / (r["ms"] / 1e3) / GB,
                          "peak": peak * world, "frac": alg / (r["ms"] / 1e3) / GB / (peak * world),
                          "peak_kind": peak_kind},
        "host_issue_ms_per_step": host_ms.get("batched"),
        "per_layer_entry_point": None if ms_layers is None else {
            "ms_per_step": ms_layers, "host_threads_per_gpu": nthr, "reconstruct_engine": args.recon_engine,
            "batched_speedup": ms_layers / r["ms"]},
        "prefix_ms_per_layer_untimed": 1e3 * t_prefix / max(len(layers), 1),
        "gpu_launches": int(n1 - n0),
        "clocks": clk,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="llama3_8b_32k")
    ap.add_argument("--layers", type=int, default=0, help="number of layers (default: the workload's)")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--e2e-threads", type=int, default=4, help="host threads (one stream each) for the e2e leg")
    ap.add_argument("--streams", type=int, default=4, help="streams layers are issued on")
    ap.add_argument("--no-graph", dest="graph", action="store_false",
                    help="issue every step's library calls from the host instead of replaying one captured CUDA graph")
    ap.add_argument("--stream-mode", default="batched", choices=["batched", "threads"],
                    help="streaming workloads: one kvf_compress_layers call per step, or per-layer calls on threads")
    ap.add_argument("--order", default="interleaved", choices=["interleaved", "phased"],
                    help="per layer compress then decompress, or all compressions then all decompressions")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--recon-engine", default="auto", choices=["auto", "cuda", "tc"],
                    help="reconstruction engine of the streaming workload")
    args = ap.parse_args()
    if args.impl == "reference":
        return reference_arm(args)
    from kvforge_b200 import synth
    if "append" in synth.WORKLOADS.get(args.workload, {}):
        return stream_arm(args)
    return gpu_arm(args)


if __name__ == "__main__":
    sys.exit(main())
