"""Throughput of the fused joint + sequence-loss path, forward + backward.

Default workload (the TDT BPE-1024 configuration batch-sharded
over 1/2/4/8 B200s): a global batch of 512 synthetic utterances, T ~ U[200, 500]
frames, U ~ U[20, 120] labels, joint dim 640, V = 1024 tokens + 5 durations
{0..4}, sigma = 0.05, activations ~N(0, 1/640), Xavier-uniform joint weights
(seeded; no dataset is available offline). Utterances are balanced over the
ranks by lattice size; every step each rank runs the fused TDT forward +
backward on its shard (public API: asr_b200.loss.tdt.tdt_loss) and the ranks
all-reduce the joint-weight gradients and the loss sum in one NCCL call.

  python bench.py [--gpus N --steps K --warmup W] [--impl reference]

Rank 0 prints one JSON line. `value` is device-timed (CUDA events, max over
ranks) with inputs resident in HBM; `e2e` adds, every step, the host->device
copy of the step's inputs from pinned memory and the device->host read of the
loss, with the next step's copy overlapping the current step's compute as a
training loop's input pipeline does (`e2e.serial`: without that overlap). The reference arm (--impl reference) times the CPU restatement of the
reference's algorithm (oracle/, the only implementation of the path that runs
on a host) on all host threads.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

D_MODEL = 640
VOCAB = 1024
DURATIONS = [0, 1, 2, 3, 4]
SIGMA = 0.05
GLOBAL_B = 512
T_RANGE = (200, 500)
U_RANGE = (20, 120)
SEED = 0


# ------------------------------------------------------------------ workload


def workload_lengths(seed=SEED):
    rng = np.random.default_rng(seed + 1)
    in_lens = rng.integers(T_RANGE[0], T_RANGE[1] + 1, size=GLOBAL_B).astype(np.int32)
    tgt_lens = rng.integers(U_RANGE[0], U_RANGE[1] + 1, size=GLOBAL_B).astype(np.int32)
    return in_lens, tgt_lens


def joint_weights(seed=SEED):
    rng = np.random.default_rng(seed + 2)

    def xavier(r, c):
        b = np.sqrt(6.0 / (r + c))
        return rng.uniform(-b, b, size=(r, c)).astype(np.float32)

    return xavier(VOCAB, D_MODEL), xavier(len(DURATIONS), D_MODEL)


def utterance(i, T, U, seed=SEED):
    """Activations and labels of utterance i (its own seeded stream)."""
    rng = np.random.default_rng([seed, 1000 + i])
    std = 1.0 / np.sqrt(D_MODEL)
    enc = (rng.standard_normal((T, D_MODEL)) * std).astype(np.float32)
    dec = (rng.standard_normal((U + 1, D_MODEL)) * std).astype(np.float32)
    y = rng.integers(1, VOCAB, size=U).astype(np.int32)
    return enc, dec, y


def make_batch(idx, in_lens, tgt_lens, seed=SEED):
    """Padded numpy batch of the utterances in idx (the shard of one rank)."""
    Bl = len(idx)
    T = int(in_lens[idx].max())
    U = int(tgt_lens[idx].max())
    enc = np.zeros((Bl, T, D_MODEL), np.float32)
    dec = np.zeros((Bl, U + 1, D_MODEL), np.float32)
    tg = np.ones((Bl, max(U, 1)), np.int32)
    for j, i in enumerate(idx):
        e, d, y = utterance(int(i), int(in_lens[i]), int(tgt_lens[i]), seed)
        enc[j, : len(e)] = e
        dec[j, : len(d)] = d
        tg[j, : len(y)] = y
    return {"enc": enc, "dec": dec, "targets": tg, "in_lens": in_lens[idx].copy(), "tgt_lens": tgt_lens[idx].copy()}


# ------------------------------------------------------------------- clocks


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap,uuid")

    def __init__(self, out_path=None, devices=1):
        """Samples every GPU of the box; the summary covers the CUDA devices
        0 .. devices - 1 of this process (matched by UUID), the GPUs the run uses."""
        self.proc = None
        self.out_path = out_path
        self.uuids = None
        try:
            import torch

            self.uuids = {str(torch.cuda.get_device_properties(i).uuid).lower() for i in range(devices)}
        except Exception:  # noqa: BLE001 - no torch / CUDA: summarise every GPU
            self.uuids = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self, gpu_indices=None):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        if self.out_path:
            Path(self.out_path).write_text(out)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            if gpu_indices is not None and int(f[0]) not in gpu_indices:
                continue
            if self.uuids and len(f) >= 10 and f[9].lower().removeprefix("gpu-") not in self.uuids:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() in ("active", "1"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------- roofline

def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


GEMM_KERNELS = ("joint_fwd_tc", "joint_dlogits_tc", "joint_dhidden_tc", "joint_dweight_tc",
                "joint_fwd_simt", "joint_dlogits_simt", "joint_dhidden_simt", "joint_dweight_simt")


def kernel_work(name, N, d, Vf, n_dur, frames=0, labels=0, stash_nodes=0, stash_per_node=0, g_width=0):
    """Algorithmic work of one step of kernel `name`: ('tensor', flops) or ('hbm', bytes).
    Joint GEMMs: 2 * N * d * Vf each (forward, backward recompute, d_hidden, dW);
    the recompute covers only the nodes past the logit stash, whose G rows the
    stash kernel forms from the stashed row (stash_per_node bytes) and the node's
    lse, cb, ct and duration grads, writing the 2 * g_width-byte G row.
    Hidden rows (forward and backward): bf16 H written (2 * ceil64(d) bytes per
    node) plus the fp32 enc / dec rows read once (frames + labels rows of d floats).
    Recursions: per node, the 4-byte lattice weights read plus the float64 alpha
    written (forward); the backward reads the weights and alpha and writes beta
    (TDT) and the 4-byte posteriors / duration gradients."""
    if name == "joint_dlogits_tc":
        return "tensor", 2.0 * max(N - stash_nodes, 0) * d * Vf
    if name in GEMM_KERNELS:
        return "tensor", 2.0 * N * d * Vf
    if name == "joint_dlogits_stash":
        return "hbm", min(stash_nodes, N) * (stash_per_node + 12.0 + 4.0 * n_dur + 2.0 * g_width)
    if name == "joint_hidden":
        kpad = (d + 63) // 64 * 64
        return "hbm", 2.0 * (N * 2.0 * kpad + (frames + labels) * d * 4.0)
    if name == "tdt_alpha":
        return "hbm", N * (4.0 * (2 + n_dur) + 8.0)
    if name == "tdt_beta_posteriors":  # weights and alpha read; beta, posteriors, duration grads written
        return "hbm", N * (8.0 * (2 + n_dur) + 16.0)
    if name == "rnnt_alpha":
        return "hbm", N * (8.0 + 8.0)
    if name == "rnnt_beta_posteriors":
        return "hbm", N * (8.0 + 8.0 + 8.0)
    return None, 0.0


def joint_path_name(tc, tf32):
    if not tc:
        return "SIMT fp32"
    return "tcgen05 bf16" if tf32 else "tcgen05 fp32 (three bf16 products of split operands)"


def parse_profile(text):
    rows = {}
    for line in text.strip().splitlines():
        name, n, ms = line.split()
        rows[name] = (int(n), float(ms))
    return rows


def profiler_report(clear=True):
    import ctypes

    from asr_b200 import _lib

    lib = _lib.capi_ops()
    n = lib.asr_profiler_report(None, 0, 0)
    buf = ctypes.create_string_buffer(max(n, 0) + 1)
    lib.asr_profiler_report(buf, len(buf), int(clear))
    return parse_profile(buf.value.decode())


# ------------------------------------------------------------ reference arm


CPU_SAMPLE = 8  # utterances in the fixed seeded CPU sample of the workload
CPU_PER_STEP = 2  # of them per step of the reference arm (cycled)


def cpu_sample(in_lens):
    """The fixed seeded subsample of the workload that both CPU timings use."""
    rng = np.random.default_rng([SEED, 99])
    return np.sort(rng.choice(len(in_lens), size=min(CPU_SAMPLE, len(in_lens)), replace=False))


def _oracle_utterances(idx, in_lens, tgt_lens, W, Wd, threads):
    from oracle import oracle

    b = make_batch(np.asarray(idx), in_lens, tgt_lens)
    oracle.tdt(b["enc"], b["dec"], W, Wd, b["targets"], b["in_lens"], b["tgt_lens"], np.array(DURATIONS, np.int32),
               sigma=SIGMA, grad_loss=np.ones(len(idx), np.float32), nthreads=threads)


def _cpu_sample_text(idx, in_lens, tgt_lens, threads, per_step=None):
    what = f"{per_step} of them per step, cycled" if per_step else "all of them once"
    return (f"fixed seeded sample of {len(idx)} utterances of the workload (indices {list(map(int, idx))}, "
            f"T={list(map(int, in_lens[idx]))}, U={list(map(int, tgt_lens[idx]))}), {what}; fwd+bwd, float64 C "
            f"restatement of the reference's float64 oracles (tests/loss/tdt_reference.py), {threads} threads")


def run_reference(args, rank):
    """CPU restatement of the reference path (oracle/) on all host threads, over
    the same fixed sample of utterances as the cpu_baseline leg of our arm."""
    if rank != 0:
        return
    from oracle import oracle

    oracle.build()
    in_lens, tgt_lens = workload_lengths()
    W, Wd = joint_weights()
    threads = os.cpu_count() or 1
    idx = cpu_sample(in_lens)
    k = 0

    def one():
        nonlocal k
        _oracle_utterances([idx[(k + j) % len(idx)] for j in range(CPU_PER_STEP)], in_lens, tgt_lens, W, Wd, threads)
        k += CPU_PER_STEP

    for _ in range(args.warmup):
        one()
    k = 0
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one()
    dt = time.perf_counter() - t0
    value = args.steps * CPU_PER_STEP / dt
    line = {
        "impl": "reference", "metric": "fused joint+loss fwd+bwd utterances/s", "value": round(value, 4),
        "unit": "utterances/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1000 * dt / args.steps, 3), "higher_is_better": True, "dtype": "f64",
        "data": "synthetic", "scaling": "strong",
        "config": {"workload": "tdt_bpe1024_sharded", "global_batch": GLOBAL_B, "vocab": VOCAB,
                   "durations": DURATIONS, "d_model": D_MODEL,
                   "sample": f"{CPU_PER_STEP} utterances per step from a fixed sample of {len(idx)}"},
        "cpu_baseline": {"value": round(value, 4), "unit": "utterances/s", "cores": threads, "kind": "port",
                         "sample": _cpu_sample_text(idx, in_lens, tgt_lens, threads, CPU_PER_STEP)},
        "e2e": {"value": round(value, 4), "unit": "utterances/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- our arm


def cpu_baseline_leg(in_lens, tgt_lens, W, Wd):
    from oracle import oracle

    oracle.build()
    threads = os.cpu_count() or 1
    idx = cpu_sample(in_lens)
    t0 = time.perf_counter()
    _oracle_utterances(idx, in_lens, tgt_lens, W, Wd, threads)
    dt = time.perf_counter() - t0
    return {"value": round(len(idx) / dt, 4), "unit": "utterances/s", "cores": threads, "kind": "port",
            "sample": _cpu_sample_text(idx, in_lens, tgt_lens, threads)}


# ------------------------------------------- the reference's own CUDA op, same GPU
#
# The reference installed by its own build into baseline/_ref (its CUDA loss op
# for sm_100a; cuBLAS joint GEMMs: fp32 with tf32 = 0, TF32 tensor cores with
# tf32 = 1) is timed on the same workload and GPU, fwd+bwd with inputs resident
# on the device, in a child process (its op library and ours both register the
# asr:: namespace). A secondary baseline beside the reference arm.

REF_ROOT = ROOT / "baseline" / "_ref"


def reference_workload(name):
    """Numpy inputs of a workload in the reference functional API's terms."""
    if name == "c5":
        in_lens, tgt_lens = workload_lengths()
        W, Wd = joint_weights()
        b = make_batch(np.arange(GLOBAL_B), in_lens, tgt_lens)
        return dict(b, kind="tdt", W=W, W_dur=Wd, durations=np.array(DURATIONS, np.int32), sigma=SIGMA,
                    grad_loss=np.full(GLOBAL_B, 1.0 / GLOBAL_B, np.float32))
    cfg = CONFIGS[name]
    x = config_inputs(cfg)
    x["kind"] = cfg["kind"]
    x["grad_loss"] = np.full(cfg["B"], 1.0 / cfg["B"], np.float32)
    if cfg["kind"] == "tdt":
        x.update(durations=np.array(DURATIONS, np.int32), sigma=SIGMA)
    return x


def reference_cuda_leg(workload, ours_value, steps=3, warmup=1, modes=(1, 0)):
    if not any((REF_ROOT / "asr" / "loss").glob("_C*.so")):
        return {"unavailable": "reference not installed in baseline/_ref (baseline/install_reference.py)"}
    import tempfile

    with tempfile.TemporaryDirectory() as tmp:
        spec = Path(tmp) / "spec.json"
        spec.write_text(json.dumps({"bench_dir": str(ROOT), "workload": workload, "tf32": list(modes),
                                    "steps": steps, "warmup": warmup}))
        r = subprocess.run([sys.executable, str(ROOT / "baseline" / "ref_worker.py"), "time", str(REF_ROOT),
                            str(spec)], capture_output=True, text=True, timeout=900)
    if r.returncode != 0:
        return {"unavailable": "reference worker failed: " + (r.stderr.strip().splitlines() or ["?"])[-1][:200]}
    out = json.loads(r.stdout.strip().splitlines()[-1])
    for v in out.values():
        v["ours_over_reference"] = round(ours_value / v["utt_per_s"], 3)
    out["what"] = ("the reference's own CUDA op (asr.loss._C built by its own setup.py for sm_100a), fwd+bwd on the "
                   "same workload and GPU, inputs resident, CUDA events, median of the timed steps; tf32_1: TF32 "
                   "cuBLAS joint GEMMs (the systems' setting), tf32_0: fp32")
    return out


# ------------------------------------------------ other BASELINE configurations
#
# `--workload c1..c4` times the other four BASELINE configurations on one GPU
# through the same public loss API (seeded synthetic inputs with the configs'
# shapes and distributions). They are secondary lines for the per-config
# table; the default workload (c5) is the headline.

CONFIGS = {
    "c1": {"name": "c1_ctc_char", "kind": "ctc", "B": 8, "T": (150, 200), "U": (20, 60), "V": 29},
    "c2": {"name": "c2_rnnt_char", "kind": "rnnt", "B": 32, "T": (100, 400), "U": (30, 150), "V": 30, "d": 640},
    "c3": {"name": "c3_tdt_bpe1024", "kind": "tdt", "B": 32, "T": (100, 400), "U": (10, 80), "V": 1024, "d": 640},
    "c4": {"name": "c4_rnnt_bpe1024_stress", "kind": "rnnt", "B": 128, "T": (400, 400), "U": (40, 100), "V": 1024,
           "d": 1024},
}


def config_inputs(cfg, seed=SEED):
    rng = np.random.default_rng([seed, 77])
    B = cfg["B"]
    in_lens = rng.integers(cfg["T"][0], cfg["T"][1] + 1, size=B).astype(np.int32)
    tgt_lens = rng.integers(cfg["U"][0], cfg["U"][1] + 1, size=B).astype(np.int32)
    T, U, V = int(in_lens.max()), int(tgt_lens.max()), cfg["V"]
    x = {"in_lens": in_lens, "tgt_lens": tgt_lens, "targets": rng.integers(1, V, size=(B, U)).astype(np.int32)}
    if cfg["kind"] == "ctc":
        x["logits"] = rng.standard_normal((B, T, V)).astype(np.float32)
        return x
    d = cfg["d"]

    def xavier(r, c):
        b = np.sqrt(6.0 / (r + c))
        return rng.uniform(-b, b, size=(r, c)).astype(np.float32)

    x["enc"] = (rng.standard_normal((B, T, d)) / np.sqrt(d)).astype(np.float32)
    x["dec"] = (rng.standard_normal((B, U + 1, d)) / np.sqrt(d)).astype(np.float32)
    x["W"] = xavier(V, d)
    if cfg["kind"] == "tdt":
        x["W_dur"] = xavier(len(DURATIONS), d)
    return x


def run_config(args):
    import torch

    from asr_b200 import _lib

    cfg = CONFIGS[args.workload]
    dev = torch.device("cuda", 0)
    host = config_inputs(cfg)
    kind = cfg["kind"]
    tf32 = bool(args.tf32)
    B = cfg["B"]
    float_keys = ["logits"] if kind == "ctc" else (["enc", "dec", "W"] + (["W_dur"] if kind == "tdt" else []))
    dev_in = {k: torch.tensor(v, device=dev) for k, v in host.items()}

    def step(t):
        leaves = [t[k].requires_grad_(True) if k in ("logits", "enc", "dec") else t[k] for k in float_keys]
        for v in leaves:
            v.grad = None
        if kind == "ctc":
            from asr_b200.loss.ctc import CTCLoss

            loss = CTCLoss()(leaves[0], t["targets"], t["in_lens"], t["tgt_lens"])
        elif kind == "rnnt":
            from asr_b200.loss.rnnt import rnnt_loss

            loss = rnnt_loss(*leaves, t["targets"], t["in_lens"], t["tgt_lens"], 0, tf32) / t["tgt_lens"].clamp_min(1)
        else:
            from asr_b200.loss.tdt import tdt_loss

            loss = tdt_loss(*leaves, t["targets"], t["in_lens"], t["tgt_lens"], DURATIONS, 0, SIGMA, tf32)
            loss = loss / t["tgt_lens"].clamp_min(1)
        total = loss.mean()
        total.backward()
        return total.detach()

    for k in ("W", "W_dur"):
        if k in dev_in:
            dev_in[k].requires_grad_(True)
    stream = torch.cuda.current_stream()
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)

    def timed(run, k):
        times = []
        for _ in range(k):
            flush.fill_(1)
            s0 = torch.cuda.Event(enable_timing=True)
            s1 = torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            run()
            s1.record(stream)
            times.append((s0, s1))
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in times)

    for _ in range(args.warmup):
        step(dev_in)
    torch.cuda.synchronize()
    lib = _lib.capi_ops()
    lib.asr_profiler_report(None, 0, 1)
    clocks = ClockSampler(args.clocks_log)
    clocks.start()
    time.sleep(0.3)
    lib.asr_profiler_enable(1)
    ms = timed(lambda: step(dev_in), args.steps) / args.steps
    lib.asr_profiler_enable(0)
    clock_info = clocks.stop()
    prof = profiler_report(clear=True)

    pinned = {k: torch.from_numpy(v).pin_memory() for k, v in host.items()}
    res = torch.empty(1, dtype=torch.float32).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in pinned.values())

    def e2e():
        t = {k: v.to(dev, non_blocking=True) for k, v in pinned.items()}
        res.copy_(step(t).reshape(1), non_blocking=True)

    e2e()
    torch.cuda.synchronize()
    e2e_ms = timed(e2e, args.steps) / args.steps

    N = int((host["in_lens"].astype(np.int64) * (host["tgt_lens"] + 1)).sum())
    d = cfg.get("d", 0)
    Vf = cfg["V"] + (len(DURATIONS) if kind == "tdt" else 0)
    n_dur = len(DURATIONS) if kind == "tdt" else 0
    peaks = measured_peaks()
    kernels, roof = {}, None
    total_ms = max(sum(v[1] for v in prof.values()), 1e-9)
    stash_nodes, stash_per = (0, 0)
    if kind != "ctc":
        stash_nodes, stash_per = _lib.logit_stash_layout(B, host["enc"].shape[1], host["dec"].shape[1], cfg["V"],
                                                         n_dur, d, tf32)
    g_width = (Vf + 15) // 16 * 16 * (1 if tf32 else 3)
    for name, (launches, kms) in prof.items():
        bound, work = kernel_work(name, N, d, Vf, n_dur, frames=int(host["in_lens"].sum()),
                                  labels=int((host["tgt_lens"] + 1).sum()), stash_nodes=stash_nodes,
                                  stash_per_node=stash_per, g_width=g_width)
        if name.startswith("ctc_"):
            tv = int(host["in_lens"].sum()) * cfg["V"] * 4.0
            states = int((host["in_lens"].astype(np.int64) * (2 * host["tgt_lens"] + 1)).sum()) * 8.0
            bound, work = "hbm", (tv + states) if name == "ctc_alpha" else (2 * tv + states)
        e = {"launches_per_step": launches / args.steps, "ms_per_step": round(kms / args.steps, 4),
             "share": round(kms / total_ms, 4)}
        if bound:
            sec = kms / args.steps / 1000.0
            ach = work / sec / (1e12 if bound == "tensor" else 1e9)
            pk = peaks["bf16_tflops_sustained"] if bound == "tensor" else peaks["hbm_gbs"]
            e.update({"bound": bound, "achieved": round(ach, 2), "unit": "TFLOP/s" if bound == "tensor" else "GB/s",
                      "frac": round(ach / pk, 4)})
        kernels[name] = e
    if prof:
        top = max(prof.items(), key=lambda kv: kv[1][1])[0]
        k = kernels[top]
        roof = {"kernel": top, "bound": k.get("bound"), "achieved": k.get("achieved"),
                "peak": peaks["bf16_tflops_sustained"] if k.get("bound") == "tensor" else peaks["hbm_gbs"],
                "unit": k.get("unit"), "frac": k.get("frac"), "traffic": None, "share": k["share"]}
    tc = kind != "ctc" and _lib.joint_uses_tensor_cores(cfg["V"], n_dur, d, tf32=tf32)
    line = {
        "metric": "fused joint+loss fwd+bwd utterances/s" if kind != "ctc" else "CTC loss fwd+bwd utterances/s",
        "value": round(B / (ms / 1000.0), 3), "unit": "utterances/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16" if tc and tf32 else "f32", "data": "synthetic",
        "config": {"workload": cfg["name"], "batch": B, "T": list(cfg["T"]), "U": list(cfg["U"]), "vocab": cfg["V"],
                   "d_model": d or None, "lattice_nodes": N if kind != "ctc" else None,
                   "l2": "flushed between timed steps (256 MB write)",
                   "joint_path": None if kind == "ctc" else joint_path_name(tc, tf32),
                   "logit_stash_nodes": min(stash_nodes, N)},
        "roofline": roof, "cpu_baseline": None,
        "e2e": {"value": round(B / (e2e_ms / 1000.0), 3), "unit": "utterances/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": 4, "ms_per_step": round(e2e_ms, 4)},
        "gpu_launches": int(sum(v[0] for v in prof.values())), "kernels": kernels, "clocks": clock_info,
        "reference_cuda": None if args.no_reference_cuda else reference_cuda_leg(args.workload, B / (ms / 1000.0)),
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------- greedy decoding
#
# `--workload decode-tdt | decode-rnnt` times batched greedy decoding
# (asr_b200.decode.{tdt,rnnt}.greedy_decode) on one GPU: decode-tdt on the
# config-5 shapes (B=512, T ~ U[200, 500], d=640, V=1024, durations 0..4),
# decode-rnnt on the config-4 shapes (B=128, T=400, d=1024, V=1024). The encoder
# output is synthetic, N(0, 0.8^2) with a constant component the blank row of
# the joint weight reads, so that blank wins most steps (about 0.2 tokens per
# frame, as a trained BPE model emits); the predictor is the reference system's
# Embedding + 2-layer LSTM(batch_first=False), random-initialised. Predictor
# calls (--decode-predict):
#   last-token (default): one call per scan for all utterances that emitted,
#     through asr_b200.decode.last_token_predictor, which gives this predictor's
#     outputs exactly (its (1, L) prefix input is read as L one-step sequences);
#   per-utterance: one call per emitted token and utterance on the whole prefix,
#     as the reference decoder calls it;
#   batched: a batch_first LSTM (another model) on the padded prefixes.

DECODE = {
    "decode-tdt": {"name": "decode_tdt_bpe1024", "B": 512, "T": T_RANGE, "d": 640, "V": 1024, "n_dur": 5,
                   "blank_bias": 7.5},
    "decode-rnnt": {"name": "decode_rnnt_bpe1024", "B": 128, "T": (400, 400), "d": 1024, "V": 1024, "n_dur": 0,
                    "blank_bias": 9.5},
}


def decode_inputs(cfg, seed=SEED):
    rng = np.random.default_rng([seed, 91])
    B, d, V = cfg["B"], cfg["d"], cfg["V"]
    in_lens = rng.integers(cfg["T"][0], cfg["T"][1] + 1, size=B).astype(np.int32)
    T = int(in_lens.max())
    enc = (rng.standard_normal((B, T, d), dtype=np.float32) * 0.8).astype(np.float32)
    enc[..., 0] = 2.0
    W = (rng.standard_normal((V, d)) * (3.0 / np.sqrt(d))).astype(np.float32)
    W[0, 0] += cfg["blank_bias"]
    Wd = None
    if cfg["n_dur"]:
        Wd = (rng.standard_normal((cfg["n_dur"], d)) * (3.0 / np.sqrt(d))).astype(np.float32)
        Wd[1, 0] += 0.5
    return {"enc": enc, "in_lens": in_lens, "W": W, "W_dur": Wd}


def decode_predictor(cfg, device, batch_first=False, seed=SEED):
    import torch

    g = torch.Generator().manual_seed(seed + 5)
    d, V = cfg["d"], cfg["V"]
    emb = torch.nn.Embedding(V, d, padding_idx=0)
    lstm = torch.nn.LSTM(input_size=d, hidden_size=d, num_layers=2, batch_first=batch_first)
    with torch.no_grad():
        for p in list(emb.parameters()) + list(lstm.parameters()):
            p.copy_(torch.randn(p.shape, generator=g) * (1.0 / np.sqrt(d)))
    emb, lstm = emb.to(device).eval(), lstm.to(device).eval()

    def predict(tokens):
        return lstm(emb(tokens))[0]

    return predict


def decode_cpu_sample(cfg, host, sample):
    """The reference greedy algorithm restated in numpy (oracle/greedy.py) with the
    same predictor on the CPU, on the first `sample` utterances."""
    import torch

    from oracle import greedy

    predict_t = decode_predictor(cfg, "cpu")

    def predict(prefix):
        with torch.no_grad():
            return predict_t(torch.as_tensor(np.asarray(prefix), dtype=torch.int64)[None])[0, -1].numpy()

    enc, lens = host["enc"][:sample], host["in_lens"][:sample]
    t0 = time.perf_counter()
    if cfg["n_dur"]:
        greedy.greedy_tdt(enc, lens, predict, host["W"], host["W_dur"], cfg["n_dur"] - 1)
    else:
        greedy.greedy_rnnt(enc, lens, predict, host["W"])
    return time.perf_counter() - t0


def run_decode(args):
    import ctypes

    import torch

    from asr_b200 import _lib
    from asr_b200.decode import last_token_predictor
    from asr_b200.decode import rnnt as dec_rnnt
    from asr_b200.decode import tdt as dec_tdt

    cfg = dict(DECODE[args.workload])
    host = decode_inputs(cfg)
    if args.batch:  # profiling aid: the first BATCH utterances
        cfg["B"] = min(args.batch, cfg["B"])
        host["enc"], host["in_lens"] = host["enc"][: cfg["B"]], host["in_lens"][: cfg["B"]]
    sample = 1  # ~10-30 s of CPU work: the reference re-runs the predictor on the whole prefix per token
    if args.impl == "reference":
        torch.set_num_threads(os.cpu_count() or 1)
        decode_cpu_sample(cfg, host, 1)  # warm-up
        dt = sum(decode_cpu_sample(cfg, host, sample) for _ in range(max(1, args.steps // 5)))
        value = sample * max(1, args.steps // 5) / dt
        base = {"value": round(value, 4), "unit": "utterances/s", "cores": torch.get_num_threads(), "kind": "port",
                "sample": f"utterances 0..{sample - 1} per step, numpy restatement of the reference greedy decoder "
                          "with the same LSTM predictor on the CPU (torch, float32)"}
        print(json.dumps({"impl": "reference", "metric": "greedy decode utterances/s", "value": base["value"],
                          "unit": "utterances/s", "n_gpus": 1, "steps": max(1, args.steps // 5), "warmup": 1,
                          "higher_is_better": True, "dtype": "f32", "data": "synthetic",
                          "config": {"workload": cfg["name"]}, "cpu_baseline": base,
                          "e2e": {"value": base["value"], "unit": "utterances/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return

    dev = torch.device("cuda", 0)
    batched = args.decode_predict == "batched"
    predict = decode_predictor(cfg, dev, batch_first=batched)
    mode = {"per-utterance": False, "batched": True,
            "last-token": last_token_predictor(predict)}[args.decode_predict]
    enc = torch.tensor(host["enc"], device=dev)
    lens = torch.tensor(host["in_lens"], device=dev)
    W = torch.tensor(host["W"], device=dev)
    Wd = torch.tensor(host["W_dur"], device=dev) if cfg["n_dur"] else None
    B = cfg["B"]

    def decode(e, ln):
        if cfg["n_dur"]:
            return dec_tdt.greedy_decode(e, ln, predict, W, Wd, cfg["n_dur"] - 1, batch_predict=mode)
        return dec_rnnt.greedy_decode(e, ln, predict, W, batch_predict=mode), None

    stream = torch.cuda.current_stream()
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    out = {}

    def timed(run, k):
        times = []
        for _ in range(k):
            flush.fill_(1)
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            run()
            s1.record(stream)
            times.append((s0, s1))
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in times)

    with torch.no_grad():
        for _ in range(args.warmup):
            out["r"] = decode(enc, lens)
        torch.cuda.synchronize()
        lib = _lib.capi()
        lib.asr_profiler_report(None, 0, 1)
        clocks = ClockSampler(args.clocks_log)
        clocks.start()
        time.sleep(0.3)
        lib.asr_profiler_enable(1)
        ms = timed(lambda: out.__setitem__("r", decode(enc, lens)), args.steps) / args.steps
        lib.asr_profiler_enable(0)
        clock_info = clocks.stop()
        n = lib.asr_profiler_report(None, 0, 0)
        buf = ctypes.create_string_buffer(max(n, 0) + 1)
        lib.asr_profiler_report(buf, len(buf), 1)
        prof = parse_profile(buf.value.decode())

        pinned = {"enc": torch.from_numpy(host["enc"]).pin_memory(), "in_lens": torch.from_numpy(host["in_lens"])}
        h2d = pinned["enc"].numel() * 4

        def e2e():
            out["r"] = decode(pinned["enc"].to(dev, non_blocking=True), pinned["in_lens"])

        e2e()
        e2e_ms = timed(e2e, args.steps) / args.steps

    hyps, durs = out["r"]
    n_tok = sum(map(len, hyps))
    frames = int(host["in_lens"].sum())
    # Joint evaluations the reference decoder makes: one per TDT step (the recorded
    # durations); for RNN-T one per emitted token plus one blank per frame.
    steps = sum(map(len, durs)) if durs is not None else n_tok + frames
    d2h = 8 * (n_tok + (steps if durs is not None else 0)) + 16 * B
    Vf = cfg["V"] + cfg["n_dur"]
    kernels = {}
    total_ms = max(sum(v[1] for v in prof.values()), 1e-9)
    sm_mhz = (clock_info or {}).get("sm_mhz") or 1965.0
    fp32_peak = 148 * 128 * 2 * sm_mhz * 1e6 / 1e12  # FFMA lanes x 2 flops x SM clock
    for name, (launches, kms) in prof.items():
        e = {"launches_per_step": launches / args.steps, "ms_per_step": round(kms / args.steps, 4),
             "share": round(kms / total_ms, 4)}
        if name == "greedy_scan":
            flops = 2.0 * steps * cfg["d"] * Vf
            ach = flops / (kms / args.steps / 1000.0) / 1e12
            e.update({"bound": "fp32", "achieved": round(ach, 2), "unit": "TFLOP/s", "frac": round(ach / fp32_peak, 4)})
        kernels[name] = e
    scan = kernels.get("greedy_scan", {})
    roof = {"kernel": "greedy_scan", "bound": "fp32", "achieved": scan.get("achieved"),
            "peak": round(fp32_peak, 2), "unit": "TFLOP/s", "frac": scan.get("frac"), "traffic": None,
            "peak_source": f"nominal FP32 FFMA rate of 148 SMs at the sampled SM clock ({sm_mhz:.0f} MHz)",
            "work": "2 * d * (V + n_dur) flops per reference decoding step"}
    cpu = None
    if not args.no_cpu_baseline:
        torch.set_num_threads(os.cpu_count() or 1)
        dt = decode_cpu_sample(cfg, host, sample)
        cpu = {"value": round(sample / dt, 4), "unit": "utterances/s", "cores": torch.get_num_threads(),
               "kind": "port", "sample": f"utterances 0..{sample - 1}: numpy restatement of the reference greedy "
                                         "decoder with the same LSTM predictor on the CPU"}
    line = {
        "metric": "greedy decode utterances/s", "value": round(B / (ms / 1000.0), 3), "unit": "utterances/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": cfg["name"], "batch": B, "T": list(cfg["T"]), "d_model": cfg["d"], "vocab": cfg["V"],
                   "n_dur": cfg["n_dur"], "predictor": {
                       "per-utterance": "Embedding + LSTM(2 layers, batch_first=False), one call per token",
                       "last-token": "Embedding + LSTM(2 layers, batch_first=False), one call per scan "
                                     "(last_token_predictor)",
                       "batched": "Embedding + LSTM(2 layers, batch_first=True), one call per scan on padded "
                                  "prefixes"}[args.decode_predict],
                   "tokens": n_tok, "frames": frames, "decoding_steps": steps,
                   "l2": "flushed between timed steps (256 MB write)"},
        "roofline": roof, "cpu_baseline": cpu,
        "e2e": {"value": round(B / (e2e_ms / 1000.0), 3), "unit": "utterances/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h), "ms_per_step": round(e2e_ms, 4)},
        "gpu_launches": int(sum(v[0] for v in prof.values()) / args.steps), "kernels": kernels, "clocks": clock_info,
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------ fused CTC head
#
# `--workload ctc-head` times the CTC system's head + loss fused into one op
# (asr_b200.loss.ctc_head.FusedCTCHead, forward + backward) on one GPU: B = 64
# utterances, T ~ U[200, 500] frames, S ~ U[20, 120] labels, d = 512 (the reference
# encoder width), V = 1024 (BPE), zero_infinity (the reference ctc.yaml), bf16
# encoder output as the system's autocast produces it. Beside it, in the same run,
# the unfused path of the reference system: Sequential(RMSNorm, Linear) under bf16
# autocast, fp32 log_softmax and the CTC loss module (asr_b200.loss.CTCLoss, the
# drop-in of the reference's), which writes the (B, T, V) logits, log-probs and
# their gradient to HBM.

CTC_HEAD = {"name": "ctc_head_bpe1024", "B": 64, "T": (200, 500), "S": (20, 120), "d": 512, "V": 1024}


def ctc_head_inputs(cfg, seed=SEED):
    rng = np.random.default_rng([seed, 53])
    B, d, V = cfg["B"], cfg["d"], cfg["V"]
    il = rng.integers(cfg["T"][0], cfg["T"][1] + 1, size=B).astype(np.int32)
    tl = rng.integers(cfg["S"][0], cfg["S"][1] + 1, size=B).astype(np.int32)
    T, S = int(il.max()), int(tl.max())
    return {"enc": rng.standard_normal((B, T, d), dtype=np.float32), "in_lens": il, "tgt_lens": tl,
            "targets": rng.integers(1, V, size=(B, S)).astype(np.int32)}


def run_ctc_head(args):
    import ctypes

    import torch

    from asr_b200 import _lib
    from asr_b200.loss import CTCLoss
    from asr_b200.loss.ctc_head import FusedCTCHead

    cfg = CTC_HEAD
    host = ctc_head_inputs(cfg)
    B, d, V = cfg["B"], cfg["d"], cfg["V"]
    if args.impl == "reference":
        from oracle import ctc_head as oracle_head

        torch.manual_seed(SEED)
        ref = torch.nn.Sequential(torch.nn.RMSNorm(d), torch.nn.Linear(d, V))
        g, W, b = (p.detach().numpy() for p in (ref[0].weight, ref[1].weight, ref[1].bias))
        sample = 2

        def one():
            oracle_head.ctc_head(host["enc"][:sample], g, W, b, host["targets"][:sample], host["in_lens"][:sample],
                                 host["tgt_lens"][:sample], zero_infinity=True)

        one()
        steps = max(1, args.steps // 2)
        t0 = time.perf_counter()
        for _ in range(steps):
            one()
        value = sample * steps / (time.perf_counter() - t0)
        base = {"value": round(value, 4), "unit": "utterances/s", "cores": os.cpu_count() or 1, "kind": "port",
                "sample": f"utterances 0..{sample - 1} per step: float64 numpy head + the C CTC oracle"}
        print(json.dumps({"impl": "reference", "metric": "fused CTC head + loss fwd+bwd utterances/s",
                          "value": base["value"], "unit": "utterances/s", "n_gpus": 1, "steps": steps, "warmup": 1,
                          "higher_is_better": True, "dtype": "f64", "data": "synthetic",
                          "config": {"workload": cfg["name"]}, "cpu_baseline": base,
                          "e2e": {"value": base["value"], "unit": "utterances/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return

    dev = torch.device("cuda", 0)
    torch.manual_seed(SEED)
    head = FusedCTCHead(d, V, zero_infinity=True).to(dev)
    ref = torch.nn.Sequential(torch.nn.RMSNorm(d), torch.nn.Linear(d, V)).to(dev)
    ref.load_state_dict(head.state_dict())
    ctc = CTCLoss(zero_infinity=True)
    enc = torch.tensor(host["enc"], device=dev).bfloat16()
    tg = torch.tensor(host["targets"], device=dev)
    il = torch.tensor(host["in_lens"], device=dev)
    tl = torch.tensor(host["tgt_lens"], device=dev)

    def fused(e, t, i, l):
        e = e.detach().requires_grad_(True)
        for p in head.parameters():
            p.grad = None
        loss = head(e, t, i, l).mean()
        loss.backward()
        return loss.detach()

    def unfused(e, t, i, l):
        e = e.detach().requires_grad_(True)
        for p in ref.parameters():
            p.grad = None
        with torch.autocast("cuda", dtype=torch.bfloat16):
            logits = ref(e)
        loss = ctc(logits, t, i, l).mean()
        loss.backward()
        return loss.detach()

    stream = torch.cuda.current_stream()
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)

    def timed(run, k):
        times = []
        for _ in range(k):
            flush.fill_(1)
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            run()
            s1.record(stream)
            times.append((s0, s1))
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in times) / k

    for _ in range(args.warmup):
        fused(enc, tg, il, tl)
        unfused(enc, tg, il, tl)
    torch.cuda.synchronize()
    lib = _lib.capi()
    lib.asr_profiler_report(None, 0, 1)
    clocks = ClockSampler(args.clocks_log)
    clocks.start()
    time.sleep(0.3)
    lib.asr_profiler_enable(1)
    ms = timed(lambda: fused(enc, tg, il, tl), args.steps)
    lib.asr_profiler_enable(0)
    clock_info = clocks.stop()
    n = lib.asr_profiler_report(None, 0, 0)
    buf = ctypes.create_string_buffer(max(n, 0) + 1)
    lib.asr_profiler_report(buf, len(buf), 1)
    prof = parse_profile(buf.value.decode())
    ms_unfused = timed(lambda: unfused(enc, tg, il, tl), args.steps)
    peak_mem = {}
    for name, fn in (("fused", fused), ("unfused", unfused)):
        torch.cuda.synchronize()
        torch.cuda.reset_peak_memory_stats(dev)
        base_mem = torch.cuda.memory_allocated(dev)
        fn(enc, tg, il, tl)
        torch.cuda.synchronize()
        peak_mem[name] = int(torch.cuda.max_memory_allocated(dev) - base_mem)

    pinned = {"enc": torch.from_numpy(host["enc"]).bfloat16().pin_memory(),
              "targets": torch.from_numpy(host["targets"]).pin_memory(),
              "in_lens": torch.from_numpy(host["in_lens"]).pin_memory(),
              "tgt_lens": torch.from_numpy(host["tgt_lens"]).pin_memory()}
    res = torch.empty(1, dtype=torch.float32).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in pinned.values())

    def e2e():
        t = {k: v.to(dev, non_blocking=True) for k, v in pinned.items()}
        res.copy_(fused(t["enc"], t["targets"], t["in_lens"], t["tgt_lens"]).reshape(1), non_blocking=True)

    e2e()
    e2e_ms = timed(e2e, args.steps)

    N = int(host["in_lens"].sum())
    kd = (d + 1 + 63) // 64 * 64
    peaks = measured_peaks()
    kernels = {}
    total_ms = max(sum(v[1] for v in prof.values()), 1e-9)
    for name, (launches, kms) in prof.items():
        e = {"launches_per_step": launches / args.steps, "ms_per_step": round(kms / args.steps, 4),
             "share": round(kms / total_ms, 4)}
        if name in GEMM_KERNELS:
            fl = 2.0 * N * kd * V
            ach = fl / (kms / args.steps / 1000.0) / 1e12
            e.update({"bound": "tensor", "achieved": round(ach, 2), "unit": "TFLOP/s",
                      "frac": round(ach / peaks["bf16_tflops_sustained"], 4)})
        kernels[name] = e
    top = max(prof.items(), key=lambda kv: kv[1][1])[0] if prof else None
    gem = [k for k in kernels if k in GEMM_KERNELS]
    gem_ms = sum(kernels[k]["ms_per_step"] for k in gem)
    gem_ach = 4 * 2.0 * N * kd * V / (gem_ms / 1000.0) / 1e12 if gem_ms else None
    roof = {"kernel": "joint GEMMs (fwd, dlogits, dhidden, dweight)", "bound": "tensor",
            "achieved": round(gem_ach, 2) if gem_ach else None, "peak": peaks["bf16_tflops_sustained"],
            "unit": "TFLOP/s", "frac": round(gem_ach / peaks["bf16_tflops_sustained"], 4) if gem_ach else None,
            "traffic": None, "top_kernel": top, "top_share": kernels[top]["share"] if top else None,
            "work": "2 * frames * ceil64(d + 1) * V flops per GEMM, 4 GEMMs per step"}
    cpu = None
    if not args.no_cpu_baseline:
        from oracle import ctc_head as oracle_head

        g, W, b = (p.detach().float().cpu().numpy() for p in (head[0].weight, head[1].weight, head[1].bias))
        t0 = time.perf_counter()
        oracle_head.ctc_head(host["enc"][:2], g, W, b, host["targets"][:2], host["in_lens"][:2],
                             host["tgt_lens"][:2], zero_infinity=True)
        cpu = {"value": round(2 / (time.perf_counter() - t0), 4), "unit": "utterances/s", "cores": 1,
               "kind": "port", "sample": "utterances 0..1: float64 numpy head + the C CTC oracle"}
    line = {
        "metric": "fused CTC head + loss fwd+bwd utterances/s", "value": round(B / (ms / 1000.0), 3),
        "unit": "utterances/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": cfg["name"], "batch": B, "T": list(cfg["T"]), "S": list(cfg["S"]), "d_model": d,
                   "vocab": V, "frames": N, "encoder_dtype": "bf16", "zero_infinity": True,
                   "l2": "flushed between timed steps (256 MB write)"},
        "unfused": {"value": round(B / (ms_unfused / 1000.0), 3), "unit": "utterances/s",
                    "ms_per_step": round(ms_unfused, 4),
                    "path": "Sequential(RMSNorm, Linear) under bf16 autocast + fp32 log_softmax + CTCLoss"},
        "peak_memory_bytes": peak_mem,
        "roofline": roof, "cpu_baseline": cpu,
        "e2e": {"value": round(B / (e2e_ms / 1000.0), 3), "unit": "utterances/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": 4, "ms_per_step": round(e2e_ms, 4)},
        "gpu_launches": int(sum(v[0] for v in prof.values()) / args.steps), "kernels": kernels, "clocks": clock_info,
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------ CTC prefix beam search
#
# `--workload ctc-beam` times CTC prefix beam search (asr_b200.decode.ctc.
# beam_decode, beam 32 as the reference's default) on one GPU over log-probs of
# B = 64 utterances, T ~ U[200, 500] frames, V = 1024 (BPE): log_softmax of
# N(0, 4^2) logits with the blank raised by 6, peaked frames as a trained model
# gives. The CPU baseline / reference arm is the reference's own op
# (src/asr/decode/csrc/ctc.cpp) compiled into oracle/_ref by `make -C oracle ref`
# (without OpenMP, so one thread; its own build parallelises over the batch).

CTC_BEAM = {"name": "ctc_beam_bpe1024", "B": 64, "T": (200, 500), "V": 1024, "beam": 32}


def ctc_beam_inputs(cfg, seed=SEED):
    import torch

    rng = np.random.default_rng([seed, 71])
    il = rng.integers(cfg["T"][0], cfg["T"][1] + 1, size=cfg["B"]).astype(np.int32)
    logits = rng.standard_normal((cfg["B"], int(il.max()), cfg["V"]), dtype=np.float32) * 4.0
    logits[..., 0] += 6.0
    return {"log_probs": torch.log_softmax(torch.from_numpy(logits), -1).numpy(), "in_lens": il}


def run_ctc_beam(args):
    import ctypes

    import torch

    from asr_b200 import _lib
    from asr_b200.decode import ctc as ctc_dec
    from oracle import ctc_beam as ref_beam

    cfg = CTC_BEAM
    host = ctc_beam_inputs(cfg)
    B, W = cfg["B"], cfg["beam"]
    sample = 2

    def cpu_ref():
        if not ref_beam.reference_available():
            return None
        lp, il = host["log_probs"][:sample], host["in_lens"][:sample]
        ref_beam.reference_beam_decode(lp[:, :20], il * 0 + 20, W)  # load + warm
        t0 = time.perf_counter()
        out = ref_beam.reference_beam_decode(lp, il, W)
        return sample / (time.perf_counter() - t0), out

    if args.impl == "reference":
        r = cpu_ref()
        if r is None:
            print(json.dumps({"impl": "reference", "unavailable": "reference beam-search op not built into "
                              "oracle/_ref (make -C oracle ref REF=<reference checkout>)"}), flush=True)
            return
        base = {"value": round(r[0], 4), "unit": "utterances/s", "cores": 1, "kind": "reference",
                "sample": f"utterances 0..{sample - 1}, the reference op built without OpenMP (one thread)"}
        print(json.dumps({"impl": "reference", "metric": "CTC beam decode utterances/s", "value": base["value"],
                          "unit": "utterances/s", "n_gpus": 1, "steps": 1, "warmup": 1, "higher_is_better": True,
                          "dtype": "f32", "data": "synthetic", "config": {"workload": cfg["name"], "beam": W},
                          "cpu_baseline": base, "e2e": {"value": base["value"], "unit": "utterances/s",
                                                         "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
              flush=True)
        return

    dev = torch.device("cuda", 0)
    lp = torch.tensor(host["log_probs"], device=dev)
    il = torch.tensor(host["in_lens"], device=dev)
    stream = torch.cuda.current_stream()
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    out = {}

    def timed(run, k):
        times = []
        for _ in range(k):
            flush.fill_(1)
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            run()
            s1.record(stream)
            times.append((s0, s1))
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in times) / k

    for _ in range(args.warmup):
        out["h"] = ctc_dec.beam_decode(lp, il, W)
    torch.cuda.synchronize()
    lib = _lib.capi()
    lib.asr_profiler_report(None, 0, 1)
    clocks = ClockSampler(args.clocks_log)
    clocks.start()
    time.sleep(0.3)
    lib.asr_profiler_enable(1)
    ms = timed(lambda: out.__setitem__("h", ctc_dec.beam_decode(lp, il, W)), args.steps)
    lib.asr_profiler_enable(0)
    clock_info = clocks.stop()
    n = lib.asr_profiler_report(None, 0, 0)
    buf = ctypes.create_string_buffer(max(n, 0) + 1)
    lib.asr_profiler_report(buf, len(buf), 1)
    prof = parse_profile(buf.value.decode())
    pinned = torch.from_numpy(host["log_probs"]).pin_memory()
    e2e_ms = timed(lambda: ctc_dec.beam_decode(pinned.to(dev, non_blocking=True), il, W), args.steps)
    frames = int(host["in_lens"].sum())
    kms = prof.get("ctc_beam", (0, 0.0))[1] / args.steps
    bytes_read = frames * cfg["V"] * 4.0
    peaks = measured_peaks()
    ach = bytes_read / (kms / 1000.0) / 1e9 if kms else None
    roof = {"kernel": "ctc_beam", "bound": "hbm", "achieved": round(ach, 2) if ach else None,
            "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(ach / peaks["hbm_gbs"], 5) if ach else None,
            "traffic": None, "work": "the log-prob rows read once (frames x V x 4 bytes)",
            "note": "latency-bound: two block-wide bitonic sorts per frame and utterance"}
    cpu = None
    r = None if args.no_cpu_baseline else cpu_ref()
    agree = None
    if r is not None:
        cpu = {"value": round(r[0], 4), "unit": "utterances/s", "cores": 1, "kind": "reference",
               "sample": f"utterances 0..{sample - 1}: the reference op (oracle/_ref, one thread)"}
        agree = r[1] == out["h"][:sample]
    kernels = {k: {"launches_per_step": v[0] / args.steps, "ms_per_step": round(v[1] / args.steps, 4)}
               for k, v in prof.items()}
    line = {
        "metric": "CTC beam decode utterances/s", "value": round(B / (ms / 1000.0), 3), "unit": "utterances/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": cfg["name"], "batch": B, "T": list(cfg["T"]), "vocab": cfg["V"], "beam": W,
                   "frames": frames, "l2": "flushed between timed steps (256 MB write)",
                   "sample_matches_reference": agree},
        "roofline": roof, "cpu_baseline": cpu,
        "e2e": {"value": round(B / (e2e_ms / 1000.0), 3), "unit": "utterances/s",
                "h2d_bytes_per_step": int(pinned.numel() * 4), "d2h_bytes_per_step": int(B * (lp.shape[1] + 1) * 4),
                "ms_per_step": round(e2e_ms, 4)},
        "gpu_launches": int(sum(v[0] for v in prof.values()) / args.steps), "kernels": kernels, "clocks": clock_info,
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--tf32", type=int, default=1, help="1: bf16 tensor-core joint (the systems' setting)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-reference-cuda", action="store_true",
                    help="skip timing the reference's own CUDA op (baseline/_ref) on the same workload")
    ap.add_argument("--clocks-log", default=None)
    ap.add_argument("--batch", type=int, default=None,
                    help="profiling aid: run only the first BATCH utterances of the workload")
    ap.add_argument("--act-dtype", default="f32", choices=["f32", "bf16"],
                    help="encoder / decoder activation dtype (bf16: a system's autocast activations, no float32 copies)")
    ap.add_argument("--workload", default="c5",
                    choices=["c1", "c2", "c3", "c4", "c5", *DECODE, "ctc-head", "ctc-beam"],
                    help="c5 (default): the headline config-5 workload; c1..c4: the other BASELINE configs, 1 GPU; "
                         "decode-tdt / decode-rnnt: batched greedy decoding; ctc-head: the fused CTC head; "
                         "ctc-beam: CTC prefix beam search (1 GPU each)")
    ap.add_argument("--decode-predict", default="last-token", choices=["last-token", "per-utterance", "batched"])
    args = ap.parse_args()
    if args.workload in DECODE or args.workload in ("ctc-head", "ctc-beam"):
        if int(os.environ.get("WORLD_SIZE", "1")) > 1:
            raise SystemExit("--workload decode-* / ctc-head / ctc-beam runs on one GPU")
        {"ctc-head": run_ctc_head, "ctc-beam": run_ctc_beam}.get(args.workload, run_decode)(args)
        return
    if args.workload != "c5":
        if args.impl == "reference" or int(os.environ.get("WORLD_SIZE", "1")) > 1:
            raise SystemExit("--workload c1..c4 runs our implementation on one GPU only")
        run_config(args)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))

    import ctypes  # noqa: F401

    from asr_b200 import _lib
    from asr_b200.loss.tdt import tdt_loss
    from asr_b200.shard import allreduce_joint, balance_shards, shard_imbalance

    in_lens, tgt_lens = workload_lengths()
    global GLOBAL_B
    if args.batch:
        GLOBAL_B = min(args.batch, GLOBAL_B)
        in_lens, tgt_lens = in_lens[:GLOBAL_B], tgt_lens[:GLOBAL_B]
    shards = balance_shards(in_lens, tgt_lens, world)
    mine = shards[rank]
    host = make_batch(mine, in_lens, tgt_lens)
    W_np, Wd_np = joint_weights()
    N_local = int((host["in_lens"].astype(np.int64) * (host["tgt_lens"] + 1)).sum())
    N_global = int((in_lens.astype(np.int64) * (tgt_lens + 1)).sum())

    act_dt = torch.bfloat16 if args.act_dtype == "bf16" else torch.float32
    enc = torch.tensor(host["enc"], device=dev).to(act_dt).requires_grad_(True)
    dec = torch.tensor(host["dec"], device=dev).to(act_dt).requires_grad_(True)
    W = torch.tensor(W_np, device=dev, requires_grad=True)
    Wd = torch.tensor(Wd_np, device=dev, requires_grad=True)
    targets = torch.tensor(host["targets"], device=dev)
    il = torch.tensor(host["in_lens"], device=dev)
    tl = torch.tensor(host["tgt_lens"], device=dev)
    stream = torch.cuda.current_stream()

    ar_events = []  # (start, end) of each all-reduce while timing it is on

    def step(e, d, tg, ilen, tlen):
        for p in (e, d, W, Wd):
            p.grad = None
        loss = tdt_loss(e, d, W, Wd, tg, ilen, tlen, DURATIONS, 0, SIGMA, bool(args.tf32))
        per = loss / tlen.clamp_min(1)
        total = per.sum() / GLOBAL_B  # global mean, as the systems' loss_per.mean()
        total.backward()
        if world > 1 and timing_ar[0]:
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a0.record(stream)
            out = allreduce_joint([W.grad, Wd.grad, total.detach().reshape(1)])
            a1.record(stream)
            ar_events.append((a0, a1))
            return out
        return allreduce_joint([W.grad, Wd.grad, total.detach().reshape(1)])

    timing_ar = [False]

    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)  # > L2 (126 MB)

    def timed_loop(run, k):
        times = []
        for _ in range(k):
            flush.fill_(1)  # evict L2 between timed iterations (not timed)
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record(stream)
            run()
            e.record(stream)
            times.append((s, e))
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in times)

    # ---- device-resident inputs
    for _ in range(args.warmup):
        step(enc, dec, targets, il, tl)
    torch.cuda.synchronize()
    lib = _lib.capi_ops()
    lib.asr_profiler_report(None, 0, 1)
    clocks = ClockSampler(args.clocks_log, devices=world) if rank == 0 else None
    if clocks:  # before the barrier: no rank may start timing while rank 0 waits for the sampler
        clocks.start()
        time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    lib.asr_profiler_enable(1)
    timing_ar[0] = True
    ms_total = timed_loop(lambda: step(enc, dec, targets, il, tl), args.steps)
    timing_ar[0] = False
    lib.asr_profiler_enable(0)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clock_info = clocks.stop() if clocks else None
    prof = profiler_report(clear=True)

    # ---- end to end: pinned host inputs copied in, loss read back, every step
    pinned = {k: torch.from_numpy(v).pin_memory() for k, v in host.items()}
    pinned["enc"] = pinned["enc"].to(act_dt).pin_memory()
    pinned["dec"] = pinned["dec"].to(act_dt).pin_memory()
    res_host = torch.empty(1, dtype=torch.float32).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in pinned.values())

    def e2e_step():
        e = pinned["enc"].to(dev, non_blocking=True).requires_grad_(True)
        d = pinned["dec"].to(dev, non_blocking=True).requires_grad_(True)
        tg = pinned["targets"].to(dev, non_blocking=True)
        ilen = pinned["in_lens"].to(dev, non_blocking=True)
        tlen = pinned["tgt_lens"].to(dev, non_blocking=True)
        flat = step(e, d, tg, ilen, tlen)
        res_host.copy_(flat[-1:], non_blocking=True)

    for _ in range(max(1, args.warmup // 2)):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e2e_serial_total = timed_loop(e2e_step, args.steps)

    # ---- end to end, pipelined as a training loop feeds batches: step i+1's inputs
    # are copied on a second stream into the other of two device buffers while step
    # i computes. Every step's copy and loss read-back is inside the timed region
    # (from the first copy to the last step); the inputs exceed L2, so no flush.
    copy_stream = torch.cuda.Stream(device=dev)
    keys = ("enc", "dec", "targets", "in_lens", "tgt_lens")
    bufs = [{k: torch.empty(pinned[k].shape, dtype=pinned[k].dtype, device=dev) for k in keys} for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    freed = [torch.cuda.Event() for _ in range(2)]

    def issue_copy(slot):
        copy_stream.wait_event(freed[slot])  # the step that last read this buffer has finished
        with torch.cuda.stream(copy_stream), torch.no_grad():
            for k in keys:
                bufs[slot][k].copy_(pinned[k], non_blocking=True)
        copied[slot].record(copy_stream)

    def pipeline(k_steps):
        for f in freed:
            f.record(stream)
        issue_copy(0)
        for i in range(k_steps):
            slot = i % 2
            if i + 1 < k_steps:
                issue_copy((i + 1) % 2)
            stream.wait_event(copied[slot])
            bt = bufs[slot]
            flat = step(bt["enc"].requires_grad_(True), bt["dec"].requires_grad_(True), bt["targets"],
                        bt["in_lens"], bt["tgt_lens"])
            res_host.copy_(flat[-1:], non_blocking=True)
            freed[slot].record(stream)

    pipeline(max(2, args.warmup // 2))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    pipeline(args.steps)
    p1.record(stream)
    torch.cuda.synchronize()
    e2e_total = p0.elapsed_time(p1)

    # the gradient all-reduce on its own, every rank already there (after a
    # barrier and a device sync): its transfer time, against the in-step window
    # above, which also holds the wait for the slowest rank
    ar_alone_ms = 0.0
    if world > 1:
        reps = 5
        for _ in range(2):
            allreduce_joint([W.grad, Wd.grad, torch.zeros(1, device=dev)])
        torch.cuda.synchronize()
        dist.barrier()
        q0, q1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        q0.record(stream)
        for _ in range(reps):
            allreduce_joint([W.grad, Wd.grad, torch.zeros(1, device=dev)])
        q1.record(stream)
        torch.cuda.synchronize()
        ar_alone_ms = q0.elapsed_time(q1) / reps

    # ---- max over ranks
    # per-rank device times of the timed steps (the imbalance the LPT split leaves)
    # and of the all-reduce alone
    ar_ms = sum(a.elapsed_time(b) for a, b in ar_events) / max(args.steps, 1) if ar_events else 0.0
    mine = torch.tensor([ms_total / args.steps, ar_ms, ar_alone_ms], device=dev, dtype=torch.float64)
    per_rank = [mine.clone() for _ in range(world)]
    if world > 1:
        dist.all_gather(per_rank, mine)
    rank_ms = [round(float(x[0]), 3) for x in per_rank]
    allreduce_ms = round(max(float(x[1]) for x in per_rank), 4)
    allreduce_alone_ms = round(max(float(x[2]) for x in per_rank), 4)
    t = torch.tensor([ms_total, e2e_total, e2e_serial_total], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_step = float(t[0]) / args.steps
    e2e_ms = float(t[1]) / args.steps
    e2e_serial_ms = float(t[2]) / args.steps
    value = GLOBAL_B / (ms_step / 1000.0)
    e2e_value = GLOBAL_B / (e2e_ms / 1000.0)

    # ---- roofline of the dominant kernel (rank 0's live event timings)
    peaks = measured_peaks()
    Vf = VOCAB + len(DURATIONS)
    roof = None
    per_kernel = {}
    total_ms = max(sum(v[1] for v in prof.values()), 1e-9)
    stash_nodes, stash_per = _lib.logit_stash_layout(len(host["in_lens"]), host["enc"].shape[1],
                                                     host["dec"].shape[1], VOCAB, len(DURATIONS), D_MODEL,
                                                     bool(args.tf32))
    g_width = (Vf + 15) // 16 * 16 * (1 if args.tf32 else 3)
    for name, (launches, kms) in prof.items():
        bound, work = kernel_work(name, N_local, D_MODEL, Vf, len(DURATIONS), frames=int(host["in_lens"].sum()),
                                  labels=int((host["tgt_lens"] + 1).sum()), stash_nodes=stash_nodes,
                                  stash_per_node=stash_per, g_width=g_width)
        per_launch_ms = kms / max(launches, 1)
        steps_launches = launches / args.steps
        work_per_launch = work / max(steps_launches, 1)
        entry = {"launches_per_step": steps_launches, "ms_per_step": round(kms / args.steps, 4),
                 "share": round(kms / total_ms, 4)}
        if bound == "tensor":
            achieved = work_per_launch / (per_launch_ms / 1000.0) / 1e12
            peak, unit = peaks["bf16_tflops_sustained"], "TFLOP/s"
        elif bound == "hbm":
            achieved = work_per_launch / (per_launch_ms / 1000.0) / 1e9
            peak, unit = peaks["hbm_gbs"], "GB/s"
        if bound:
            entry.update({"bound": bound, "achieved": round(achieved, 2), "unit": unit,
                          "frac": round(achieved / peak, 4)})
        per_kernel[name] = entry
    if prof:
        name, (launches, kms) = max(prof.items(), key=lambda kv: kv[1][1])
        k = per_kernel[name]
        steps_launches = launches / args.steps
        bound = k.get("bound")
        peak = peaks["bf16_tflops_sustained"] if bound == "tensor" else peaks["hbm_gbs"]
        traffic = None
        tfile = ROOT / "profiles" / "traffic.json"
        if tfile.exists():
            tj = json.loads(tfile.read_text()).get(name)
            if tj:  # bytes per node measured by ncu on a smaller case, scaled to this launch
                traffic = int(tj["bytes_per_node"] * N_local / max(steps_launches, 1))
        roof = {"kernel": name, "bound": bound, "achieved": k.get("achieved"), "peak": peak, "unit": k.get("unit"),
                "frac": k.get("frac"), "traffic": traffic,
                "peak_source": f"{peaks['source']} ({'bf16 sustained' if bound == 'tensor' else 'hbm copy'})",
                "launch_ms": round(kms / max(launches, 1), 4), "share": k["share"]}
    launches_total = int(sum(v[0] for v in prof.values()))

    if world > 1:
        dist.barrier()
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline_leg(in_lens, tgt_lens, W_np, Wd_np)
        ref_cuda = None
        if world == 1 and not args.no_reference_cuda and not args.batch:
            ref_cuda = reference_cuda_leg("c5", value)
        tc = _lib.joint_uses_tensor_cores(VOCAB, len(DURATIONS), D_MODEL, tf32=bool(args.tf32))
        line = {
            "metric": "fused joint+loss fwd+bwd utterances/s", "value": round(value, 3), "unit": "utterances/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16" if args.tf32 and tc else "f32", "data": "synthetic",
            "config": {"workload": "tdt_bpe1024_sharded", "global_batch": GLOBAL_B, "per_gpu_batch": len(mine),
                       "T": list(T_RANGE), "U": list(U_RANGE), "d_model": D_MODEL, "vocab": VOCAB,
                       "durations": DURATIONS, "sigma": SIGMA, "lattice_nodes_global": N_global,
                       "lattice_nodes_rank0": N_local, "rank_ms_per_step": rank_ms,
                       "allreduce_ms_per_step": allreduce_ms if world > 1 else None,
                       "allreduce_alone_ms": allreduce_alone_ms if world > 1 else None,
                       "shard_imbalance": round(shard_imbalance(
                           in_lens, tgt_lens, shards), 4), "parallelism": f"dp{world}",
                       "l2": "flushed between timed steps (256 MB write)",
                       "joint_path": joint_path_name(tc, args.tf32), "activations": args.act_dtype,
                       "logit_stash": {"nodes_rank0": min(stash_nodes, N_local), "bytes_per_node": stash_per,
                                       "budget_bytes": _lib.logit_stash_budget()}},
            "roofline": roof, "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 3), "unit": "utterances/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": 4, "ms_per_step": round(e2e_ms, 4),
                    "pipelining": "step i+1's host->device copy on a second stream overlaps step i",
                    "serial": {"value": round(GLOBAL_B / (e2e_serial_ms / 1000.0), 3),
                               "ms_per_step": round(e2e_serial_ms, 4)}},
            "gpu_launches": launches_total, "kernels": per_kernel,
            "clocks": clock_info, "reference_cuda": ref_cuda,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
