#!/usr/bin/env python
"""Throughput of the int8 ModernBERT encoder + decision heads on B200.

Workload: ModernBERT vocab 16384, hidden 256, 6 layers,
4 heads of 64, GeGLU 384, local window 128 with every 3rd layer global,
seeded random-init weights, 128-token sequences with ids uniform in
[4, 16384), heads noul / choice(5) / score(5 levels) / spans(9 tags).
A step is one call of the encoder + heads over `--seqs-per-step` sequences
(a stream of 32-sequence batches laid end to end); the metric is sequences
per second. Multi-GPU: one process per GPU, each encoding its own shard of
sequences (weak scaling, no data-path collective); the time is the max over
ranks.

  python bench.py [--gpus N --steps K --warmup W]   # this implementation
  python bench.py --impl reference ...               # the reference's CPU path
  python bench.py --workload c5 ...                  # config 5: the SigLIP vision tower (images/s)
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

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

METRIC = "int8 encoder seq/s (128 tok)"
METRIC_F32 = "float32 encoder seq/s (128 tok)"
F32_PATH_KERNELS = {"f32_gemm_qkv", "f32_gemm_wo", "f32_gemm_wi", "f32_gemm_womlp", "f32_attend_blocks"}
SEQ_LEN = 128
BATCH = 32


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--seqs-per-step", type=int, default=2048)
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="target length of the CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gemm", action="store_true")
    ap.add_argument("--workload", default="c1", choices=["c1", "c1-f32", "c3", "c3-varlen", "c4", "c5"],
                    help="c1: the ModernBERT headline (default); c1-f32: the same model on the float32 path "
                         "(SetInt8(false)); c3: 8 x 4096-token sequences; c3-varlen: 256 sequences of U[8,512] "
                         "tokens; c4: the base-size model on 256 x 512 tokens; c5: the SigLIP ViT-B/16 vision tower")
    ap.add_argument("--images-per-step", type=int, default=512, help="c5: images per step, shared by all ranks")
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return dict(hbm=float(p["hbm_gbs"]), bf16=float(p["bf16_tflops"]), src="measured")
    except Exception:
        return dict(hbm=6650.0, bf16=1590.0, src="fallback")


_JSON_FD = 1  # where the result line goes


def dist_setup():
    global _JSON_FD
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        # Rank 0's stdout carries one JSON line: libraries that print to fd 1
        # (NCCL's version banner at communicator creation) go to stderr.
        sys.stdout.flush()
        _JSON_FD = os.dup(1)
        os.dup2(2, 1)
    return world, rank, local


def emit(line: dict):
    """The result line, on the process's original stdout."""
    os.write(_JSON_FD, (json.dumps(line) + "\n").encode())


class Clocks:
    """Clock samples of one GPU during the timed region: NVML read every 20 ms
    from a thread (so short timed regions get samples too), else nvidia-smi
    every 100 ms. Reads only; no setting of the GPU is changed."""
    # NVML clock-event reason bits (nvml.h: nvmlClocksEventReason*)
    NVML_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.p = None
        self.thread = None

    def _nvml_loop(self, h, nv):
        while not self.halt.is_set():
            try:
                self.samples.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM),
                                     nv.nvmlDeviceGetCurrentClocksEventReasons(h)))
            except Exception:
                pass
            self.halt.wait(0.02)

    def start(self):
        try:
            import threading
            import pynvml as nv
            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByIndex(self.gpu)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            self.samples, self.halt = [], threading.Event()
            self.thread = threading.Thread(target=self._nvml_loop, args=(h, nv), daemon=True)
            self.thread.start()
            return
        except Exception:
            self.thread = None
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "100", "-i", str(self.gpu)], stdout=subprocess.PIPE,
                                      stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.p = None

    def stop(self):
        if self.thread is not None:
            self.halt.set()
            self.thread.join()
            if not self.samples:
                return None
            reasons = sorted({n for _, r in self.samples for n, b in self.NVML_BITS.items() if r & b})
            return {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": self.max_mhz,
                    "reasons": reasons, "samples": len(self.samples), "source": "nvml"}
        if self.p is None:
            return None
        self.p.terminate()
        try:
            out, _ = self.p.communicate(timeout=5)
        except Exception:
            self.p.kill()
            out, _ = self.p.communicate()
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
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def physical_gpu(local: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        try:
            return int(vis.split(",")[local])
        except (ValueError, IndexError):
            pass
    return local


def workload(seqs: int, seed: int):
    from indecis_b200 import synthetic as S
    return S.ids_fixed(seqs, SEQ_LEN, S.C1["vocab"], seed=seed)


# The encoder workloads. `per_gpu` sequences per GPU per step (the global
# batch is per_gpu x N, cut into one contiguous cost-balanced range per rank);
# `make(nseq)` draws the global batch with the config's seed.
def encoder_spec(args):
    from indecis_b200 import synthetic as S
    w = args.workload
    if w in ("c1", "c1-f32"):
        return dict(name=w, cfg=S.C1, per_gpu=args.seqs_per_step, heads=True,
                    make=lambda n: S.ids_fixed(n, SEQ_LEN, S.C1["vocab"], seed=1),
                    metric=METRIC_F32 if w == "c1-f32" else METRIC,
                    desc="C1 ModernBERT int8 forward + heads (vocab 16384, hidden 256, 6 layers, 4x64 heads, GeGLU "
                         "384, local 128 / global every 3rd), noul+choice5+score5+spans9 heads",
                    shape={"seq_len": SEQ_LEN, "batch": BATCH})
    if w == "c3":
        return dict(name=w, cfg=S.C1, per_gpu=8, heads=False,
                    make=lambda n: S.ids_fixed(n, 4096, S.C1["vocab"], seed=31),
                    metric="int8 encoder seq/s (4096 tok)",
                    desc="C3 long inputs: the C1 model (6 layers, layers 0 and 3 global over all 4096 tokens, the "
                         "others local 128), 8 x 4096 tokens, mean-pooled output",
                    shape={"seq_len": 4096, "batch": 8})
    if w == "c3-varlen":
        return dict(name=w, cfg=S.C1, per_gpu=256, heads=False,
                    make=lambda n: S.ids_varlen(n, 8, 512, S.C1["vocab"], seed=3),
                    metric="int8 encoder seq/s (varlen U[8,512])",
                    desc="C3 variable-length unpadded batch: the C1 model, 256 sequences of U[8,512] tokens (seed 3), "
                         "mean-pooled output",
                    shape={"seq_len": "U[8,512]", "batch": 256})
    if w == "c4":
        return dict(name=w, cfg=S.C4, per_gpu=256, heads=False,
                    make=lambda n: S.ids_fixed(n, 512, S.C4["vocab"], seed=41),
                    metric="int8 encoder seq/s (512 tok, base)",
                    desc="C4 base ModernBERT int8 encoder (vocab 262144, hidden 768, 22 layers, 12x64 heads, GeGLU "
                         "1152, local 128 / global every 3rd), 256 x 512 tokens, mean-pooled embedding output",
                    shape={"seq_len": 512, "batch": 256})
    raise ValueError(w)


def config_obj(args, world, spec=None):
    spec = spec or encoder_spec(args)
    per = spec["per_gpu"]
    c = {"workload": spec["desc"], **spec["shape"], "seqs_per_step_per_gpu": per, "global_batch": per * world,
         "parallelism": f"sequence shard x{world} (contiguous cost-balanced ranges of one global batch), no collective",
         "weights": "random-init seed 42"}
    if spec["name"] in ("c1", "c1-f32"):
        c["batches_per_step_per_gpu"] = per // BATCH
        c["l2"] = "inputs and activations larger than L2 (x alone is seqs*128*1 KiB)"
    elif spec["name"] == "c4":
        c["l2"] = "inputs and activations larger than L2 (x alone is 256*512*3 KiB = 384 MiB)"
    else:
        c["l2"] = "L2 flushed (256 MiB write, untimed) before every timed step"
    return c


# ---------------------------------------------------------------------------
# CPU legs (the oracle port of the reference path; test/bench infrastructure)
# ---------------------------------------------------------------------------

def cpu_model(spec):
    import oracle
    from indecis_b200 import synthetic as S
    oracle.build()
    model = oracle.Model(spec["cfg"], S.weights(spec["cfg"], seed=42))
    model.heads = S.heads(spec["cfg"]["hidden"]) if spec["heads"] else []
    return model, oracle


# Sequences per CPU call: C1 goes in the reference's batches of 32
# (forEachPooled, model.go:391-415); a long or base-size sequence alone.
CPU_UNIT = {"c1": BATCH, "c1-f32": BATCH, "c3": 1, "c3-varlen": 16, "c4": 1}


def cpu_sample(model, spec, ids, offs, units: int, threads: int, f32: bool = False):
    """The oracle port over the first `units` CPU calls of the batch: for the
    heads workloads token states, float64 mean pooling in token order and
    every head's float64 logits; otherwise the pooled encoder output.
    Returns (seconds, sequences)."""
    import oracle
    u = CPU_UNIT[spec["name"]]
    t0 = time.perf_counter()
    done = 0
    for b in range(units):
        lo, hi = b * u, min((b + 1) * u, len(offs) - 1)
        if lo >= hi:
            break
        o = offs[lo:hi + 1] - offs[lo]
        x = ids[offs[lo]:offs[hi]]
        if f32:
            model.encode_f32(x, o, threads=threads)
        elif model.heads:
            tokens = model.encode(x, o, mode=1, threads=threads, fast=True)
            pooled = np.stack([tokens[o[i]:o[i + 1]].astype(np.float64).mean(0)
                               for i in range(hi - lo)]).astype(np.float32)
            for h in model.heads:
                oracle.head_logits(h["w"], h["b"], tokens if h["kind"] == "spans" else pooled)
        else:
            model.encode(x, o, mode=0, threads=threads, fast=True)
        done += hi - lo
    return time.perf_counter() - t0, done


def encoder_gop(cfg, lens) -> float:
    """Algorithmic int8 operations (2 per multiply-add) of the encoder over
    sequences of the given lengths: the four projections per token and layer,
    and S = QK^T plus O = PV over each query's keys (the local window on
    local layers)."""
    H, I, L, nh = cfg["hidden"], cfg["intermediate"], cfg["layers"], cfg["heads"]
    D, w = H // nh, cfg["local_attention"] // 2
    proj = H * 3 * H + H * H + H * 2 * I + I * H
    macs = 0
    for n in lens:
        n = int(n)
        i = np.arange(n)
        local = int((np.minimum(n, i + w + 1) - np.maximum(0, i - w)).sum())
        for l in range(L):
            keys = n * n if l % cfg["global_every"] == 0 else local
            macs += proj * n + 2 * D * nh * keys
    return 2.0 * macs / 1e9


def cpu_isa(oracle):
    feats = oracle.lib().or_cpu_features()
    return "AVX-VNNI" if feats & 1 else ("AVX512-VNNI" if feats & 2 else "scalar int")


def cpu_baseline(spec, target_s: float, f32: bool = False):
    """The oracle port on all host threads, a bounded sample (about target_s)
    of the workload's own sequences."""
    model, oracle = cpu_model(spec)
    threads = os.cpu_count() or 1
    ids, offs = spec["make"](max(spec["per_gpu"], 200 * CPU_UNIT[spec["name"]]))
    t1, _ = cpu_sample(model, spec, ids, offs, 1, threads, f32)  # warm-up, and the size of one call
    units = int(max(1, min(200, target_s / max(t1, 1e-3))))
    oracle.phase_seconds(reset=True)
    t, n = cpu_sample(model, spec, ids, offs, units, threads, f32)
    ph = oracle.phase_seconds(reset=True)
    path = ("float32 path (scalar FMA chains)" if f32 else
            f"int8 path: {cpu_isa(oracle)} 6x16 tiles for the projections and for attention's S = QK^T and "
            f"O = PV, AVX2 (8 float32 lanes) LayerNorm, row quantization, RoPE, ExpShift and GeluMul")
    out = {"value": n / t, "unit": "seq/s", "cores": threads, "kind": "port",
           "sample": f"{n} sequences of the workload in calls of {CPU_UNIT[spec['name']]}, oracle C++ port of the "
                     f"reference {path}, {threads} threads, {t:.1f} s"}
    if not f32:
        gop = encoder_gop(spec["cfg"], np.diff(offs[:n + 1]))
        tot = sum(ph) or 1.0
        out["gop_per_s"] = gop / t
        out["gop_per_s_per_thread"] = gop / t / threads
        out["phase_share"] = {"norms_qkv_rope": ph[0] / tot, "attention": ph[1] / tot,
                              "out_proj_norm_mlp": ph[2] / tot}
    return out


def run_reference(args, world, rank):
    """The reference's CPU implementation of the path (the oracle port, since
    the Go reference cannot run on this image), on all host threads; each
    step one CPU call of the workload (a bounded sample)."""
    if rank != 0:
        return
    spec = encoder_spec(args)
    f32 = args.workload == "c1-f32"
    model, oracle = cpu_model(spec)
    threads = os.cpu_count() or 1
    u = CPU_UNIT[spec["name"]]
    ids, offs = spec["make"](max(spec["per_gpu"], (args.steps + args.warmup) * u))
    for k in range(args.warmup):
        cpu_sample(model, spec, *shift(ids, offs, k * u), 1, threads, f32)
    total, n = 0.0, 0
    for k in range(args.steps):
        t, m = cpu_sample(model, spec, *shift(ids, offs, (args.warmup + k) * u), 1, threads, f32)
        total, n = total + t, n + m
    v = n / total
    path = "float32 path" if f32 else f"int8 path, {cpu_isa(oracle)}"
    line = {"metric": spec["metric"], "value": v, "unit": "seq/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32" if f32 else "int8",
            "data": "synthetic", "config": config_obj(args, args.gpus, spec),
            "cpu_baseline": {"value": v, "unit": "seq/s", "cores": threads, "kind": "port",
                             "sample": f"each step one CPU call of {u} sequence(s) of the workload (bounded sample), "
                                       f"oracle C++ port of the reference {path} (Go reference not runnable: no Go "
                                       f"toolchain), {threads} threads"
                                       + ("" if f32 else ": VNNI 6x16 tiles for the projections and attention, AVX2 "
                                                         "8-lane LayerNorm, quantization, RoPE, ExpShift, GeluMul")},
            "e2e": {"value": v, "unit": "seq/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(line)


def shift(ids, offs, s0):
    """The batch from sequence s0 on (offsets rebased)."""
    t0 = int(offs[s0])
    return ids[t0:], offs[s0:] - t0


# ---------------------------------------------------------------------------
# GPU leg
# ---------------------------------------------------------------------------

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch
# per sequence, from one ncu capture of the C1 workload at 512 sequences
# (profiles/attn_qkv_c1_512seq.txt, profiles/attn_short_c1_512seq.txt,
# profiles/gemm_rows_c1_512seq.txt); a
# launch processes the whole step's sequences, so the per-launch traffic is
# this times the sequences per step (traffic grows with the sequences).
NCU_BYTES_PER_SEQ = {
    "attn_qkv_quant": (21564416 + 2816000) / 512,
    "attn_short": (201441536 + 38391040) / 512,
    "attn_short_quant": (201448192 + 11332864) / 512,
    "gemm_qkv": (21466368 + 145374976) / 512,
    "gemm_wo_residual": (88436736 + 11129856) / 512,
    "gemm_wi_geglu": (21517824 + 42096384) / 512,
    "ln_quant": (67132672 + 3182080) / 512,
}


# Warp instructions of one launch per sequence (smsp__inst_executed.sum of the
# capture in profiles/attn_qkv_c1_512seq.txt).
NCU_INST_PER_SEQ = {"attn_qkv_quant": 66996374 / 512}
B200_SMS = 148


def roofline(report, pk, nseq, workload="c1", sm_mhz=None, step_ms=None):
    """The dominant kernel's roofline entry from the timed region's events
    (around that kernel's launches only: its share is of the timed steps'
    device time, step_ms in all)."""
    ks = [k for k in report["kernels"] if k["records"] > 0 and k["ms"] > 0]
    top = max(ks, key=lambda k: k["ms"])
    total_ms = step_ms if step_ms else sum(k["ms"] for k in ks)
    per_ms = top["ms"] / top["records"]
    bytes_ = top["bytes"] / top["records"]
    ops = top["ops"] / top["records"]
    int8_peak = 2.0 * pk["bf16"]  # TOP/s: int8 dense = 2x bf16 dense on B200
    t_hbm = bytes_ / (pk["hbm"] * 1e9)
    t_ops = ops / (int8_peak * 1e12) if ops else 0.0
    if t_ops > t_hbm:
        ach = ops / (per_ms * 1e-3) / 1e12
        rf = {"bound": "tensor", "achieved": ach, "peak": int8_peak, "unit": "TFLOP/s", "frac": ach / int8_peak}
        peak_note = f"int8 dense = 2 x {pk['src']} bf16 burst {pk['bf16']} TFLOP/s (no int8 entry)"
    else:
        ach = bytes_ / (per_ms * 1e-3) / 1e9
        rf = {"bound": "hbm", "achieved": ach, "peak": pk["hbm"], "unit": "GB/s", "frac": ach / pk["hbm"]}
        peak_note = f"{pk['src']} HBM copy bandwidth"
    rf.update({"kernel": top["name"], "share": top["ms"] / total_ms, "ms_per_launch": per_ms,
               "algorithmic_bytes": bytes_, "algorithmic_ops": ops, "peak_source": peak_note})
    per_seq = NCU_BYTES_PER_SEQ.get(top["name"]) if workload == "c1" else None
    rf["traffic"] = per_seq * nseq if per_seq else None
    rf["traffic_source"] = "ncu dram bytes at 512 sequences, scaled" if per_seq else None
    # The bound these kernels meet first: instruction issue. Warp instructions
    # per launch from the same ncu capture, scaled by the sequences, over the
    # SMs' issue capacity (4 schedulers x the clock seen) in the launch's time.
    inst = NCU_INST_PER_SEQ.get(top["name"]) if workload == "c1" else None
    if inst and sm_mhz:
        cap = B200_SMS * 4 * sm_mhz * 1e6 * per_ms * 1e-3
        rf["issue"] = {"warp_instructions": inst * nseq, "frac": inst * nseq / cap, "sm_mhz": sm_mhz,
                       "source": "smsp__inst_executed.sum at 512 sequences (ncu), scaled; 148 SMs x 4 issue slots"}
    return rf


C2_SHAPES = [(768, 256), (256, 384), (2304, 768), (768, 1152)]  # (N, K) of config 2
C2_ROWS = [128, 4096, 65536]


def gemm_point(M, N, K, pk, flush, reps=10):
    """One config-2 point: u8 x s8 -> s32 -> f32 C = ((acc - zc) * sb) * sa
    through the library's GEMM, scales log-uniform in [1e-3, 1e-1]. Each rep
    is timed alone with CUDA events after a write of a buffer larger than L2,
    so small operands are read from HBM as at the large sizes."""
    import torch
    from indecis_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(0)
    A = torch.randint(1, 256, (M, K), dtype=torch.uint8, device="cuda", generator=g)
    B = torch.randint(-127, 128, (N, K), dtype=torch.int8, device="cuda", generator=g)
    sa = torch.exp(torch.empty(M, device="cuda").uniform_(math.log(1e-3), math.log(1e-1), generator=g))
    sb = torch.exp(torch.empty(N, device="cuda").uniform_(math.log(1e-3), math.log(1e-1), generator=g))
    zc = 128.0 * B.to(torch.float32).sum(1)
    C = torch.empty((M, N), dtype=torch.float32, device="cuda")
    for _ in range(3):
        ops.gemm_u8s8(A, B, sa=sa, sb=sb, zc=zc, C=C)
    st = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    torch.cuda.synchronize()
    torch.cuda._sleep(100_000_000)  # the device idles while the host queues every rep: no launch gaps timed
    for e0, e1 in ev:
        flush.fill_(1)
        e0.record(st)
        ops.gemm_u8s8(A, B, sa=sa, sb=sb, zc=zc, C=C)
        e1.record(st)
    torch.cuda.synchronize()
    ms = statistics.median(e0.elapsed_time(e1) for e0, e1 in ev)
    tops = 2.0 * M * N * K / (ms * 1e-3) / 1e12
    byts = M * K + N * K + 4 * M + 8 * N + 4 * M * N
    int8_peak = 2.0 * pk["bf16"]
    bound = min(int8_peak, (2.0 * M * N * K / byts) * pk["hbm"] / 1e3)
    return {"M": M, "N": N, "K": K, "us": round(ms * 1e3, 2), "tops": round(tops, 1),
            "frac_of_int8_peak": round(tops / int8_peak, 4), "frac_of_roofline": round(tops / bound, 4),
            "bound": "tensor" if bound >= int8_peak else "hbm", "out": "f32"}


def int8_dense_probe(reps=10):
    """The library's own tcgen05 int8 product on a shape bound by the tensor
    cores (M = N = 8192, K = 8192, int32 out: 1.1 TOP against 0.4 GB of
    traffic), median of reps launches with CUDA events: a measured int8
    dense rate to set beside 2 x the bf16 burst."""
    import torch
    from indecis_b200 import ops
    M = N = K = 8192
    g = torch.Generator(device="cuda").manual_seed(0)
    A = torch.randint(1, 256, (M, K), dtype=torch.uint8, device="cuda", generator=g)
    B = torch.randint(-127, 128, (N, K), dtype=torch.int8, device="cuda", generator=g)
    for _ in range(3):
        ops.gemm_u8s8(A, B, int32_out=True)
    st = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    torch.cuda.synchronize()
    for e0, e1 in ev:
        e0.record(st)
        ops.gemm_u8s8(A, B, int32_out=True)
        e1.record(st)
    torch.cuda.synchronize()
    ms = statistics.median(e0.elapsed_time(e1) for e0, e1 in ev)
    del A, B
    torch.cuda.empty_cache()
    return {"M": M, "N": N, "K": K, "us": round(ms * 1e3, 1), "tops": round(2.0 * M * N * K / (ms * 1e-3) / 1e12, 1),
            "kernel": "library GEMM (tcgen05 kind::i8, CTA pair for K >= 1024), int32 out"}


def gemm_sweep(pk):
    """Config 2: M in {128, 4096, 65536} x (N, K) in its four shapes."""
    import torch
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")  # 256 MiB > the 126 MB L2
    pts = [gemm_point(M, N, K, pk, flush) for M in C2_ROWS for N, K in C2_SHAPES]
    del flush
    probe = int8_dense_probe()
    for p in pts:
        p["frac_of_measured_int8"] = round(p["tops"] / probe["tops"], 4)
    return {"points": pts, "timing": "median of 10 reps, each after an L2 flush (256 MiB write), CUDA events; all reps "
                                      "queued behind a device sleep, so host launch time is not timed",
            "int8_peak_tops": 2.0 * pk["bf16"], "int8_peak_source": "2 x measured bf16 burst (no int8 entry)",
            "int8_dense_measured": probe}


def dist_init(world, local):
    import datetime
    import torch
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(world, v):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def batch32_calls(model, spec, heads):
    """The literal call shape of the reference's callers: EncodeSeqs / Decide
    batches of 32 sequences (forEachPooled, model.go:391-415), each one host
    call of ig_logits (ids from host memory, float64 logits back). Sequential
    calls from one thread, then 8 threads calling concurrently."""
    import threading
    ids, offs = spec["make"](32 * 64)
    batches = [shift(ids, offs, 32 * k) for k in range(64)]
    batches = [(x[:int(o[32])], o[:33]) for x, o in batches]
    for b in batches[:4]:
        model.Logits(b)
    t0 = time.perf_counter()
    for b in batches:
        model.Logits(b)
    seq_s = time.perf_counter() - t0

    def client(k):
        for b in batches[k::8]:
            model.Logits(b)

    ts = [threading.Thread(target=client, args=(k,)) for k in range(8)]
    t0 = time.perf_counter()
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    par_s = time.perf_counter() - t0
    n = 32 * len(batches)
    return {"seqs_per_call": 32, "calls": len(batches), "ms_per_call": 1000 * seq_s / len(batches),
            "seq_s_one_caller": n / seq_s, "seq_s_8_callers": n / par_s,
            "api": "ig_logits, host buffers, one 32x128 batch per call"}


def run_ours(args, world, rank, local):
    import torch
    from indecis_b200 import _capi, build, shard
    from indecis_b200 import synthetic as S
    from indecis_b200.model import Config, Head, Model

    spec = encoder_spec(args)
    dist_init(world, local)
    build.build()
    pk = peaks()
    cfg = Config.from_dict(spec["cfg"])
    model = Model.from_arrays(cfg, S.weights(spec["cfg"], seed=42), device=local)
    heads = [Head(h["name"], h["kind"], h["w"], h["b"]) for h in S.heads(cfg.hidden_size)] if spec["heads"] else []
    if heads:
        model.SetHeads(heads)
    f32 = args.workload == "c1-f32"
    if f32:
        model.SetInt8(False)
    L = _capi.load()

    # The global batch, cut into one contiguous cost-balanced range per rank
    # (every rank derives the same cut from the same offsets).
    gids, goffs = spec["make"](spec["per_gpu"] * world)
    costs = shard.seq_costs(goffs, cfg.num_hidden_layers, cfg.global_attn_every_n_layers, cfg.local_attention,
                            cfg.hidden_size)
    s0, s1 = shard.shard_ranges(goffs, world, costs)[rank]
    ids, offs = shard.local_batch(gids, goffs, s0, s1)
    nseq = s1 - s0
    N = int(offs[-1])
    H = cfg.hidden_size
    pooled_rows = sum(h.rows for h in heads if h.kind != "spans")
    token_rows = sum(h.rows for h in heads if h.kind == "spans")
    d_ids = torch.from_numpy(ids).cuda()
    stream = torch.cuda.current_stream()
    if heads:
        d_logits = torch.empty((nseq, pooled_rows), dtype=torch.float64, device="cuda")
        d_tlog = torch.empty((N, token_rows), dtype=torch.float64, device="cuda")

        def step():
            _capi.check(L.ig_logits_device(model._h, d_ids.data_ptr(), offs.ctypes.data, nseq, d_logits.data_ptr(),
                                           d_tlog.data_ptr(), stream.cuda_stream))
    else:
        d_out = torch.empty((nseq, H), dtype=torch.float32, device="cuda")

        def step():
            _capi.check(L.ig_encode_device(model._h, d_ids.data_ptr(), offs.ctypes.data, nseq, _capi.IG_MODE_POOLED,
                                           d_out.data_ptr(), stream.cuda_stream))

    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda") if spec["name"] in ("c3", "c3-varlen") else None
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # One more, untimed, step with CUDA events around every launch: the
    # per-kernel breakdown and the dominant kernel. The timed region then
    # carries events around that kernel's launches only (events between all
    # ~50 launches of a step cost about 3% of its time and keep each kernel
    # from being scheduled during the previous one's last wave).
    if flush is not None:
        flush.fill_(1)
    _capi.profile(True)
    step()
    breakdown = _capi.profile_report()
    _capi.profile(False)
    top_name = None
    if not f32:
        top_name = max((k for k in breakdown["kernels"] if k["records"] > 0), key=lambda k: k["ms"])["name"]
        _capi.profile_only(top_name)

    # ---- timed region: device events on the launching stream -------------
    clocks = Clocks(physical_gpu(local))
    _capi.profile(True)
    barrier(world)
    torch.cuda.synchronize()
    clocks.start()
    if flush is None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        ms_local = e0.elapsed_time(e1)
    else:
        # the L2 is flushed before every step, outside the timed events
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for e0, e1 in ev:
            flush.fill_(1)
            e0.record(stream)
            step()
            e1.record(stream)
        torch.cuda.synchronize()
        ms_local = sum(e0.elapsed_time(e1) for e0, e1 in ev)
    barrier(world)
    clk = clocks.stop()
    ms = max_over_ranks(world, ms_local)
    report = _capi.profile_report()
    _capi.profile(False)
    _capi.profile_only(None)
    gseq = spec["per_gpu"] * world
    value = gseq * args.steps / (ms / 1e3)
    dev_err = L.ig_device_error(1)
    if dev_err:
        raise RuntimeError(f"device error {dev_err}")
    del flush

    # ---- end to end: the host API (ids from host memory, results back) ----
    e2e_steps = max(3, min(args.steps, 20))
    seqs = (ids, offs)
    run_host = (lambda: model.Logits(seqs)) if heads else (lambda: model.EncodeSeqs(seqs))
    # Warm-up calls as for the device steps: the first host calls also pay for
    # the host allocator settling (fresh output pages, pinned staging).
    for _ in range(max(3, args.warmup)):
        run_host()
    barrier(world)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        run_host()
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(world, time.perf_counter() - t0)
    # ids + offsets + the plan's block lists: per sequence one 16-byte
    # tensor-core entry per 128 queries and attention kind, and one 8-byte
    # entry per 64 queries (row tables are filled on the device)
    blocks = sum(2 * 16 * ((n + 127) // 128) + 8 * ((n + 63) // 64) for n in np.diff(offs).tolist())
    h2d = 4 * N + 4 * (nseq + 1) + blocks
    d2h = 8 * nseq * pooled_rows + 8 * N * token_rows if heads else 4 * nseq * H
    e2e = {"value": gseq * e2e_steps / e2e_s, "unit": "seq/s", "h2d_bytes_per_step": h2d,
           "d2h_bytes_per_step": d2h,
           "api": ("ig_logits" if heads else "ig_encode (pooled)") + " (host buffers, synchronous), host clock around "
                  "device-synchronized calls; each rank's call covers its range of the global batch"}

    extra = {}
    if rank == 0 and spec["name"] == "c1":
        extra["c1_batch32"] = batch32_calls(model, spec, heads)
    gemm = None
    if rank == 0 and not args.no_gemm and spec["name"] == "c1":
        gemm = gemm_sweep(pk)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(spec, args.cpu_seconds, f32)

    if rank == 0:
        cfg_obj = config_obj(args, world, spec)
        if f32:
            cfg_obj["path"] = "float32 (SetInt8(false)): float products in the reference's FMA-chain order"
            rf = c5_roofline(report, pk, clk["sm_mhz"] if clk else None, fp32_names=F32_PATH_KERNELS)[0]
        else:
            rf = roofline(report, pk, nseq, spec["name"], clk["sm_mhz"] if clk else None, step_ms=ms_local)
        line = {"metric": spec["metric"], "value": value, "unit": "seq/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32" if f32 else "int8", "data": "synthetic",
                "config": cfg_obj, "e2e": e2e, "gpu_launches": report["launches"], "roofline": rf,
                "kernels": {k["name"]: {"ms": round(k["ms"], 3), "launches": k["launches"]}
                            for k in (report if f32 else breakdown)["kernels"]},
                "kernels_source": "the timed steps" if f32 else
                                  "one untimed step with events around every launch, just before the timed region",
                "clocks": clk, "cpu_baseline": cpu, **extra, "gemm_sweep": gemm}
        emit(line)
    model.close()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# C5: the SigLIP ViT-B/16 vision tower
# ---------------------------------------------------------------------------

C5_METRIC = "SigLIP ViT-B/16 int8 vision tower images/s (224 px, 196 patches)"
FP32_KERNELS = {"vis_attn_f32", "vis_patch_embed", "vis_head_kv", "vis_head_mlp", "vis_head_attn"}


def c5_config(args, world, per_rank):
    return {"workload": "C5 SigLIP ViT-B/16 vision tower, int8 layers (hidden 768, 12 layers, 12x64 heads, MLP 3072 "
                        "GELU-tanh, biases, LLM.int8 outlier split on fc2), float32 patch embedding, attention and "
                        "attention-pooling head; pixels uniform in [-1, 1]",
            "images_per_step": args.images_per_step, "images_per_step_per_gpu": per_rank, "image_size": 224,
            "patches": 196, "parallelism": f"image shard x{world}, no collective",
            "l2": "inputs and activations larger than L2 (fc1 output alone is images*196*12 KiB)",
            "weights": "random-init seed 42, 4 massive fc1 channels per layer"}


def c5_cpu(n_images: int, threads: int):
    import oracle
    from indecis_b200 import synthetic as S
    oracle.build()
    om = oracle.SigLIP(S.C5, S.siglip_weights(S.C5, seed=42))
    px = S.pixels(n_images, 224, seed=5)
    om.forward(px[:1], patches=False, threads=threads, fast=True)
    t0 = time.perf_counter()
    om.forward(px, patches=False, threads=threads, fast=True)
    return time.perf_counter() - t0, oracle


def run_reference_c5(args, world, rank):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    n = max(1, min(threads, 16))
    ts = []
    oracle = None
    for _ in range(max(1, args.steps)):
        t, oracle = c5_cpu(n, threads)
        ts.append(t)
    total = sum(ts)
    v = n * len(ts) / total
    line = {"metric": C5_METRIC, "value": v, "unit": "img/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": len(ts), "warmup": 1, "ms_per_step": 1000 * total / len(ts), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8+f32", "data": "synthetic",
            "config": {**c5_config(args, 1, n), "images_per_step": n, "note": "bounded CPU sample per step"},
            "cpu_baseline": {"value": v, "unit": "img/s", "cores": threads, "kind": "port",
                             "sample": f"{n} images per step, oracle C++ port of internal/siglip (images over "
                                       f"{threads} threads, VNNI integer products)"},
            "e2e": {"value": v, "unit": "img/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(line)


def c5_roofline(report, pk, sm_mhz, fp32_names=None):
    ks = [k for k in report["kernels"] if k["records"] > 0 and k["ms"] > 0]
    total = sum(k["ms"] for k in ks)
    fp32_peak = 148 * 128 * 2 * (sm_mhz or 1965.0) * 1e6 / 1e12  # CUDA-core FMA rate at the SM clock
    int8_peak = 2.0 * pk["bf16"]
    out = []
    for k in sorted(ks, key=lambda k: -k["ms"])[:4]:
        per_ms = k["ms"] / k["records"]
        ops, byts = k["ops"] / k["records"], k["bytes"] / k["records"]
        if k["name"] in (fp32_names or FP32_KERNELS) and ops:
            ach = ops / (per_ms * 1e-3) / 1e12
            r = {"bound": "fp32", "achieved": ach, "peak": fp32_peak, "unit": "TFLOP/s", "frac": ach / fp32_peak,
                 "peak_source": f"148 SMs x 128 FP32 FMA/clk at the sampled {sm_mhz or 1965.0:.0f} MHz (nominal)"}
        elif ops and ops / (int8_peak * 1e12) > byts / (pk["hbm"] * 1e9):
            ach = ops / (per_ms * 1e-3) / 1e12
            r = {"bound": "tensor", "achieved": ach, "peak": int8_peak, "unit": "TOP/s", "frac": ach / int8_peak,
                 "peak_source": f"int8 dense = 2 x {pk['src']} bf16 burst"}
        else:
            ach = byts / (per_ms * 1e-3) / 1e9
            r = {"bound": "hbm", "achieved": ach, "peak": pk["hbm"], "unit": "GB/s", "frac": ach / pk["hbm"],
                 "peak_source": f"{pk['src']} HBM copy bandwidth"}
        r.update({"kernel": k["name"], "share": k["ms"] / total, "ms_per_launch": per_ms, "traffic": None})
        out.append(r)
    return out


def run_ours_c5(args, world, rank, local):
    import torch
    from indecis_b200 import _capi, build
    from indecis_b200 import synthetic as S
    from indecis_b200.siglip import Vision, VisionConfig

    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    build.build()
    pk = peaks()
    vis = Vision.from_arrays(VisionConfig.from_dict(S.C5), S.siglip_weights(S.C5, seed=42), device=local)
    L = _capi.load()
    total = args.images_per_step
    lo, hi = rank * total // world, (rank + 1) * total // world
    n = hi - lo
    px_host = S.pixels(total, 224, seed=5)[lo:hi]
    d_px = torch.from_numpy(px_host).cuda()
    d_out = torch.empty((n, 768), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()

    def step():
        _capi.check(L.ig_vision_forward_device(vis._h, d_px.data_ptr(), n, 0, None, d_out.data_ptr(),
                                               stream.cuda_stream))

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        import torch.distributed as dist
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    clocks = Clocks(physical_gpu(local))
    _capi.profile(True)
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1))
    report = _capi.profile_report()
    _capi.profile(False)
    value = total * args.steps / (ms / 1e3)

    # End to end through the host API: pixels from host memory, embeddings back.
    e2e_steps = max(3, min(args.steps, 10))
    for _ in range(3):
        vis.Embed(px_host)
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        vis.Embed(px_host)
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    e2e = {"value": total * e2e_steps / e2e_s, "unit": "img/s", "h2d_bytes_per_step": int(px_host.nbytes),
           "d2h_bytes_per_step": int(n * 768 * 4),
           "api": "ig_vision_forward (host pixels, synchronous), host clock around device-synchronized calls"}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        k = max(1, min(threads, 16))
        t, _ = c5_cpu(k, threads)
        cpu = {"value": k / t, "unit": "img/s", "cores": threads, "kind": "port",
               "sample": f"{k} C5 images, oracle C++ port of internal/siglip (images over {threads} threads, VNNI "
                         f"integer products, scalar float32 chains), {t:.1f} s"}
    if rank == 0:
        rl = c5_roofline(report, pk, clk["sm_mhz"] if clk else None)
        line = {"metric": C5_METRIC, "value": value, "unit": "img/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "int8+f32", "data": "synthetic", "config": c5_config(args, world, n),
                "e2e": e2e, "gpu_launches": report["launches"], "roofline": rl[0], "roofline_top4": rl,
                "kernels": {k["name"]: {"ms": round(k["ms"], 3), "launches": k["launches"]}
                            for k in report["kernels"]},
                "clocks": clk, "cpu_baseline": cpu}
        emit(line)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse()
    world, rank, local = dist_setup()
    if args.workload == "c5":
        if args.impl == "reference":
            run_reference_c5(args, world, rank)
        else:
            run_ours_c5(args, world, rank, local)
        return
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    run_ours(args, world, rank, local)  # c1 and c1-f32


if __name__ == "__main__":
    main()
