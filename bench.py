#!/usr/bin/env python3
"""Benchmark of the B200 causal-attention engine (one JSON line on rank 0).

With no --config, one run measures every BASELINE configuration: the line's
top-level figures are the headline, c3-bf16 (causal prefill at the 343M
trainer shape, B=8 H=16 T=1024 d=64, bf16 in/out -- the configuration the
north-star tensor-core target is quoted on), and `configs` carries the same
measurements for every config:
  c1       16-layer KV-cached decode, fp32 cache           (HBM GB/s)
  c2       causal prefill fp32, d=32                       (TFLOP/s)
  c3-f32   causal prefill fp32, d=64  / c3-bf16 in bf16    (TFLOP/s)
  c4-f32   ragged decode, fp32 cache / c4-int8 INT8 cache  (HBM GB/s)
  c5-f32   causal backward fp32 / c5-bf16 in bf16          (TFLOP/s)
  trainer  the reference GPU trainer's attn_fwd + attn_bwd   (TFLOP/s)
  qkv      its fused Q, K, V projection (one launch)        (TFLOP/s)
--config <key> runs one of them alone.

A step is one call of the path over one batch of synthetic input that is
already resident in HBM.  The K timed steps run back to back on the launching
stream between two CUDA events, queued behind a device sleep long enough for
the host to enqueue them all, so the interval holds the steps and the gaps
between their kernels but not the host's enqueue.  No step starts L2-warm: when one step's
working set is below 2 x L2, the step's device tensors are rotated over
enough copies that together they exceed it.

Multi-GPU (torchrun, one process per GPU) is STRONG scaling: the fixed
workload of each config is split across the ranks -- prefill and backward
by (batch x head) units (attn_split_plan), the 16-layer decode by layers,
the ragged decode by sequences dealt longest-first (attn_shard_lpt).
`value` is the whole workload over the slowest rank's device time.  The
gather of a whole output over the library's own NCCL group (attn_gather_split,
attn_gather_rows) is timed separately (`gather`) and is part of `e2e`.

`e2e` times the same call through the C ABI with the step's inputs copied in
from pinned host memory and its result copied back inside the timed region.

--impl reference times the reference's own CPU attention (compiled from its
sources into oracle/_ref/) on a bounded sample of each workload.
"""
import argparse
import ctypes
import hashlib
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "pure-c-llm_b200")
sys.path.insert(0, PKG)
sys.path.insert(0, ROOT)

# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------
CONFIGS = {
    "c1": dict(kind="decode", L=16, H=16, d=32, prior=512, steps=128, kv="f32",
               workload="C1 KV-cached decode fp32, d_model 512 = 16 x 32, 16 layers, 512 prior rows, 128 steps"),
    "c2": dict(kind="fwd", B=8, H=16, T=1024, d=32, dtype="f32",
               workload="C2 causal prefill fp32 B8 H16 T1024 d32"),
    "c3-f32": dict(kind="fwd", B=8, H=16, T=1024, d=64, dtype="f32",
                   workload="C3 causal prefill fp32 B8 H16 T1024 d64 (343M shape)"),
    "c3-bf16": dict(kind="fwd", B=8, H=16, T=1024, d=64, dtype="bf16",
                    workload="C3 causal prefill bf16 B8 H16 T1024 d64 (343M shape)"),
    "c4-f32": dict(kind="ragged", n_seq=64, H=16, d=64, max_len=8192, kv="f32",
                   workload="C4 ragged decode fp32 cache, 64 seqs H16 d64 len~U[1,8192]"),
    "c4-int8": dict(kind="ragged", n_seq=64, H=16, d=64, max_len=8192, kv="int8",
                    workload="C4 ragged decode INT8 cache (per-token-head scale), 64 seqs H16 d64 len~U[1,8192]"),
    "c5-f32": dict(kind="bwd", B=4, H=16, T=4096, d=64, dtype="f32",
                   workload="C5 causal backward fp32 B4 H16 T4096 d64"),
    "c5-bf16": dict(kind="bwd", B=4, H=16, T=4096, d=64, dtype="bf16",
                    workload="C5 causal backward bf16 B4 H16 T4096 d64"),
    # not a BASELINE config: the reference GPU trainer's own attention call pair
    # (gpu_kernels.h:17-31 shape) through the drop-in symbols, beside the
    # reference's own cuBLAS attention at that shape
    "trainer": dict(kind="train", B=4, H=12, T=1024, d=128, dtype="f32",
                    workload="the reference GPU trainer's attention: attn_fwd + attn_bwd drop-ins at "
                             "gpu_kernels.h's shape B4 H12 T1024 d128, fp32"),
    # not a BASELINE config: the fused QKV projection that feeds attn_fwd in the
    # reference GPU trainer (train_kaggle.cu:152-154, three gemm_nn calls) at its
    # shape, M = B*T = 4096 rows, DIM 1536
    "qkv": dict(kind="qkv", M=4096, K=1536, N=1536, dtype="f32",
                workload="the reference GPU trainer's Q, K, V projections (train_kaggle.cu:152-154) in one "
                         "launch: X (4096 x 1536) times Wq, Wk, Wv (1536 x 1536) plus biases, fp32"),
}
ORDER = ["c3-bf16", "c1", "c2", "c3-f32", "c4-f32", "c4-int8", "c5-f32", "c5-bf16", "trainer", "qkv"]
DENSE = ("fwd", "bwd", "train", "qkv")     # kinds measured in TFLOP/s
HEADLINE = "c3-bf16"
METRIC = "causal-attn prefill TFLOP/s & KV-decode HBM GB/s per B200 at 1/2/4/8 GPUs"
L2_BYTES = 126 * 2 ** 20
TRAFFIC_FILE = os.path.join(ROOT, "profiles", "traffic.json")


def causal_flops(B, H, T, d):
    """QK^T and PV over the causal triangle: 4 d flops per (i, j<=i) pair."""
    return 4.0 * B * H * d * T * (T + 1) / 2


def qkv_flops(M, K, N):
    """Three (M x K) @ (K x N) products."""
    return 3 * 2.0 * M * K * N


def metric_of(cfg):
    return {"fwd": "causal-attn prefill TFLOP/s", "bwd": "causal-attn backward TFLOP/s",
            "train": "causal-attn forward+backward TFLOP/s",
            "qkv": "fused QKV projection TFLOP/s"}.get(cfg["kind"], "KV-decode HBM GB/s")


def unit_of(cfg):
    return "TFLOP/s" if cfg["kind"] in DENSE else "GB/s"


def dtype_of(cfg):
    if cfg["kind"] in DENSE:
        return cfg["dtype"]
    return "f32 (int8 cache)" if cfg.get("kv") == "int8" else "f32"


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        p = json.load(open(path))
        return dict(hbm=p["hbm_gbs"], bf16=p["bf16_tflops"], bf16_sus=p.get("bf16_tflops_sustained"),
                    src="measured")
    return dict(hbm=6650.0, bf16=1590.0, bf16_sus=1400.0, src="fallback")


def traffic_of(key):
    """DRAM bytes per launch of the config's dominant kernel(s) from the ncu
    capture recorded in profiles/traffic.json, with whether the kernel sources
    are still the ones captured (sha1 of the listed files)."""
    if not os.path.exists(TRAFFIC_FILE):
        return None, None
    ent = json.load(open(TRAFFIC_FILE)).get(key)
    if not ent:
        return None, None
    return ent["dram_bytes_per_launch"], {"kernels": ent["kernels"], "capture": ent.get("capture"),
                                          "sources_unchanged": sources_sha(ent["sources"]) == ent.get("source_sha1")}


def sources_sha(files):
    h = hashlib.sha1()
    for f in files:
        with open(os.path.join(ROOT, f), "rb") as fh:
            h.update(fh.read())
    return h.hexdigest()


# ---------------------------------------------------------------------------
# clocks sampler (nvidia-smi during the timed region)
# ---------------------------------------------------------------------------
class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = f"/tmp/attn_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            self.proc.wait()
            self.f.close()

    def summary(self):
        if not self.proc or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        rows = [r.split(", ") for r in open(self.path).read().strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows]
        mx = max(float(r[2]) for r in rows)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        loaded = [s for s, r in zip(sm, rows) if float(r[3]) > 200] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(rows)}


# ---------------------------------------------------------------------------
# CPU baseline: the reference's own attention (oracle/_ref), bounded sample
# ---------------------------------------------------------------------------
def _host_threads():
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    # all host threads for the reference's OpenMP loops (torchrun exports
    # OMP_NUM_THREADS=1, which would otherwise leave it single-threaded)
    os.environ["OMP_NUM_THREADS"] = str(cores)
    try:
        ctypes.CDLL("libgomp.so.1").omp_set_num_threads(cores)
    except OSError:
        pass
    return cores


class CpuSample:
    """One bounded sample of a config's workload for the reference's CPU code:
    one batch row (prefill), one batch row at T=1024 (backward), or a few
    caches (decode).  call() runs it once and returns the seconds taken."""

    def __init__(self, cfg):
        import synth
        from oracle import oracle as O
        self.O, self.cfg = O, cfg
        self.cores = _host_threads()
        kind = cfg["kind"]
        if kind == "qkv":
            M, K, N = 256, cfg["K"], cfg["N"]
            self.x = synth.normal(1, (M, K))
            self.ws = [synth.normal(2 + i, (K, N), 0, 0.02) for i in range(3)]
            self.bs = [synth.normal(5 + i, (N,), 0, 0.1) for i in range(3)]
            self.work = qkv_flops(M, K, N) / 1e12
            self.unit = "TFLOP/s"
            self.sample = (f"reference train.c matmul_forward x3 (the Q, K, V projections of train.c:517-519), "
                           f"{M} of {cfg['M']} rows")
            return
        if kind in ("fwd", "bwd", "train"):
            B, H, T, d = 1, cfg["H"], cfg["T"], cfg["d"]
            if kind == "bwd":
                T = min(T, 1024)
            self.args = (B, T, H, d)
            self.q, self.k, self.v = (synth.normal(s, (B * T, H * d), 0, 0.5) for s in (1, 2, 3))
            if kind in ("bwd", "train"):
                self.do = synth.normal(4, (B * T, H * d))
                _, self.probs = O.ref_attention_forward(self.q, self.k, self.v, B, T, H, d)
            self.work = causal_flops(B, H, T, d) * {"fwd": 1, "bwd": 2, "train": 3}[kind] / 1e12
            self.unit = "TFLOP/s"
            what = {"fwd": "attention_forward", "bwd": "attention_backward",
                    "train": "attention_forward + attention_backward"}[kind]
            self.sample = f"reference train.c {what} B={B} H={H} T={T} d={d} (one batch row of the workload)"
            return
        H, d = cfg["H"], cfg["d"]
        if kind == "decode":
            self.lens = [cfg["prior"] + cfg["steps"] // 2] * 16
            self.t_max = 1024
        else:
            self.lens = [int(x) for x in synth.uniform_int(2024, cfg["n_seq"], 1, cfg["max_len"])[:8]]
            self.t_max = 8192
        self.kc = synth.normal(5, (self.t_max, H * d))
        self.vc = synth.normal(6, (self.t_max, H * d))
        self.qv = synth.normal(7, (H * d,))
        int8 = cfg.get("kv") == "int8"
        if int8:
            self.kc = O.dequantize_kv_int8(*O.quantize_kv_int8(self.kc, H, d), H, d)
            self.vc = O.dequantize_kv_int8(*O.quantize_kv_int8(self.vc, H, d), H, d)
        bpe, sbytes = (1, 4) if int8 else (4, 0)
        self.work = (sum(n * H * (2 * d * bpe + 2 * sbytes) for n in self.lens) + len(self.lens) * 2 * H * d * 4) / 1e9
        self.unit = "GB/s"
        self.sample = (f"reference transformer.c cached_attention over {len(self.lens)} caches "
                       f"(H={H} d={d}{', dequantised INT8' if int8 else ''})")

    def call(self):
        O, c = self.O, self.cfg
        t0 = time.perf_counter()
        if c["kind"] == "qkv":
            for w, b in zip(self.ws, self.bs):
                O.ref_matmul_forward(self.x, w, b)
        elif c["kind"] == "fwd":
            B, T, H, d = self.args
            O.ref_attention_forward(self.q, self.k, self.v, B, T, H, d)
        elif c["kind"] == "bwd":
            B, T, H, d = self.args
            O.ref_attention_backward(self.do, self.q, self.k, self.v, self.probs, B, T, H, d)
        elif c["kind"] == "train":
            B, T, H, d = self.args
            _, probs = O.ref_attention_forward(self.q, self.k, self.v, B, T, H, d)
            O.ref_attention_backward(self.do, self.q, self.k, self.v, probs, B, T, H, d)
        else:
            for n in self.lens:
                O.ref_cached_attention(self.qv, self.kc, self.vc, n - 1, c["H"], c["d"], self.t_max)
        return time.perf_counter() - t0


def cpu_reference(cfg, budget_s=3.0, max_samples=30):
    s = CpuSample(cfg)
    times, t_end = [], time.time() + budget_s
    while True:
        times.append(s.call())
        if time.time() > t_end or len(times) >= max_samples:
            break
    return dict(value=s.work / min(times), unit=s.unit, cores=s.cores, kind="reference",
                sample=f"{s.sample}, best of {len(times)}")


# ---------------------------------------------------------------------------
# GPU workloads
# ---------------------------------------------------------------------------
class Workload:
    """Device-resident inputs of this rank's share of a config; step()
    enqueues one call on `stream`, gather() assembles the whole output."""

    def __init__(self, cfg, A, torch, dev, rank, world):
        self.cfg, self.A, self.torch, self.dev = cfg, A, torch, dev
        self.rank, self.world = rank, world
        kind = cfg["kind"]
        g = torch.Generator(device=dev).manual_seed(1234 + rank)
        self.gather_ok = world > 1 and kind in ("fwd", "decode", "ragged")
        self.gather_launches = 0
        if kind == "qkv":
            M, K, N = cfg["M"], cfg["K"], cfg["N"]
            r0, r1 = A.shard_range(M, world, rank)           # token rows: no exchange needed
            Ml = r1 - r0
            self.x = torch.randn((Ml, K), generator=g, device=dev)
            self.wq, self.wk, self.wv = (torch.randn((K, N), generator=g, device=dev) * 0.02 for _ in range(3))
            self.bq, self.bk, self.bv = (torch.randn((N,), generator=g, device=dev) * 0.1 for _ in range(3))
            self.q, self.k, self.v = (torch.empty((Ml, N), device=dev) for _ in range(3))
            self.shape = A.QKVShape(Ml, K, N, 0, 0)
            self.ws_bytes = A.lib.attn_qkv_workspace_bytes(ctypes.byref(self.shape))
            self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device=dev)
            self.work = qkv_flops(Ml, K, N)
            self.total_work = qkv_flops(M, K, N)
            self.launches = 2                        # weight split, then the projection
            self.in_names, self.out_names = ["x"], ["q", "k", "v"]
            self.local_desc = f"rows [{r0}, {r1}) of {M}"
        elif kind in ("fwd", "bwd", "train"):
            B, H, T, d = cfg["B"], cfg["H"], cfg["T"], cfg["d"]
            self.sp = sp = A.split_plan(B, H, world, rank)
            Bl, Hl = sp.batch, sp.heads
            dt = torch.bfloat16 if cfg["dtype"] == "bf16" else torch.float32
            self.dtype_code = A.BF16 if dt == torch.bfloat16 else A.F32
            self.esz = 2 if dt == torch.bfloat16 else 4
            mk = lambda s: (torch.randn((Bl * T, Hl * d), generator=g, device=dev) * s).to(dt)
            self.q, self.k, self.v = mk(0.5), mk(0.5), mk(0.5)
            self.o = torch.empty_like(self.q)
            self.lse = torch.empty(Bl * Hl * T, device=dev)
            self.shape = A.Shape(Bl, Hl, T, d, 0, 0)
            self.full_shape = A.Shape(B, H, T, d, 0, 0)
            self.work = causal_flops(Bl, Hl, T, d)
            self.total_work = causal_flops(B, H, T, d)
            self.launches = 1
            self.in_names, self.out_names = ["q", "k", "v"], ["o"]
            if kind == "train":
                # the drop-ins take their shape from the macro-shape setting and run
                # on the legacy default stream; probs and scratch are the trainer's
                # B*H*T*T-float buffers (train_kaggle.cu:128, 138)
                A.check(A.lib.attn_set_macro_shape(Bl, Hl, T, d))
                self.do = mk(1.0)
                self.dq, self.dk, self.dv = (torch.empty_like(self.q) for _ in range(3))
                self.probs = torch.empty(Bl * Hl * T * T, device=dev)
                self.scratch = torch.empty(Bl * Hl * T * T, device=dev)
                self.work *= 3
                self.total_work *= 3
                # forward; backward at d 96/128 on the tensor cores: row statistics, the
                # operand splits, 2 score GEMMs, P/dS, dQ/dV/dK GEMMs
                self.launches = 9 if d in (96, 128) and T % 4 == 0 else 4
                self.in_names = ["q", "k", "v", "do"]
                self.out_names = ["o", "dq", "dk", "dv"]
            if kind == "bwd":
                self.do = mk(1.0)
                A.fwd_ex(self.shape, self.dtype_code, self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(),
                         self.o.data_ptr(), self.lse.data_ptr(), 0)
                self.dq, self.dk, self.dv = (torch.empty_like(self.q) for _ in range(3))
                self.ws_bytes = A.bwd_workspace_bytes(self.shape, self.dtype_code)
                self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device=dev)
                self.work *= 2
                self.total_work *= 2
                self.launches = 3                    # row-dot pre-pass, dK/dV kernel, dQ kernel
                self.in_names = ["q", "k", "v", "do", "o", "lse"]
                self.out_names = ["dq", "dk", "dv"]
            if self.gather_ok and kind == "fwd":
                self.full = torch.empty((B * T, H * d), dtype=dt, device=dev)
                self.g_bytes = A.lib.attn_gather_workspace_bytes(ctypes.byref(self.full_shape), self.dtype_code, world)
                self.g_ws = torch.empty(max(self.g_bytes, 256), dtype=torch.uint8, device=dev)
                self.gather_launches = 1 if sp.nh > 1 else 0
            self.local_desc = f"batches [{sp.batch0}, {sp.batch0 + Bl}) x heads [{sp.head0}, {sp.head0 + Hl})"
        elif kind == "decode":
            L, H, d, prior, steps = cfg["L"], cfg["H"], cfg["d"], cfg["prior"], cfg["steps"]
            if L % world:
                raise SystemExit(f"c1: {world} ranks do not split {L} layers evenly")
            Ll = L // world
            cap = prior + steps
            self.kc = [torch.randn((cap, H * d), generator=g, device=dev) for _ in range(Ll)]
            self.vc = [torch.randn((cap, H * d), generator=g, device=dev) for _ in range(Ll)]
            self.kp = torch.tensor([t.data_ptr() for t in self.kc], dtype=torch.int64, device=dev)
            self.vp = torch.tensor([t.data_ptr() for t in self.vc], dtype=torch.int64, device=dev)
            self.qs = torch.randn((steps, Ll, H * d), generator=g, device=dev)
            self.outs = torch.empty_like(self.qs)
            self.lens = torch.tensor([[prior + s + 1] * Ll for s in range(steps)], dtype=torch.int32, device=dev)
            self.shape = A.DecodeShape(Ll, H, d, A.F32, 0, cap, cap)
            self.ws_bytes = A.decode_workspace_bytes(self.shape)
            self.ws = torch.zeros(self.ws_bytes, dtype=torch.uint8, device=dev)
            self.step_idx = 0
            per_layer = sum((prior + s + 1) * H * d * 4 * 2 + 2 * H * d * 4 for s in range(steps)) / steps
            self.work = per_layer * Ll                 # bytes of one step (mean over the 128 steps)
            self.total_work = per_layer * L
            self.launches = 1
            self.row_bytes, self.max_local, self.n_out, self.order = H * d * 4, Ll, L, None
            if self.gather_ok:
                self.full = torch.empty((L, H * d), device=dev)
            self.local_desc = f"layers [{rank * Ll}, {(rank + 1) * Ll})"
        else:  # ragged
            import synth
            import shard
            n, H, d, max_len = cfg["n_seq"], cfg["H"], cfg["d"], cfg["max_len"]
            lens_all = synth.uniform_int(2024, n, 1, max_len)
            seqs, _ = shard.lpt_sequences(lens_all, world)
            mine = seqs[rank]
            lens_h = lens_all[mine]
            cap = int(lens_h.max()) if len(mine) else 1
            nl = len(mine)
            kc = torch.randn((nl * cap, H * d), generator=g, device=dev)
            vc = torch.randn((nl * cap, H * d), generator=g, device=dev)
            self.int8 = cfg["kv"] == "int8"
            if self.int8:
                self.kc, self.ks = A.quantize_int8_t(kc, H)
                self.vc, self.vs = A.quantize_int8_t(vc, H)
                del kc, vc
            else:
                self.kc, self.vc, self.ks, self.vs = kc, vc, None, None
            self.max_local = max(len(s) for s in seqs)
            self.q = torch.randn((nl, H * d), generator=g, device=dev)
            self.o = torch.zeros((self.max_local, H * d), device=dev)
            self.lens = torch.from_numpy(lens_h.astype(np.int32)).to(dev)
            self.shape = A.DecodeShape(nl, H, d, A.I8 if self.int8 else A.F32, 0, cap, cap)
            self.ws_bytes = A.decode_workspace_bytes(self.shape)
            self.ws = torch.zeros(max(self.ws_bytes, 256), dtype=torch.uint8, device=dev)
            per_row = H * (2 * d + 2 * 4) if self.int8 else H * d * 4 * 2
            self.work = float(lens_h.sum()) * per_row + 2 * nl * H * d * 4
            self.total_work = float(lens_all.sum()) * per_row + 2 * n * H * d * 4
            self.launches = 2 if self.int8 else 1        # INT8: the decode kernel and the merge of split sequences
            self.row_bytes, self.n_out = H * d * 4, n
            if self.gather_ok:
                order = np.full((world, self.max_local), -1, np.int32)
                for r, s in enumerate(seqs):
                    order[r, :len(s)] = s
                self.order = torch.from_numpy(order.reshape(-1)).to(dev)
                self.full = torch.empty((n, H * d), device=dev)
            self.local_desc = f"{nl} of {n} sequences (LPT by length), {int(lens_h.sum())} of {int(lens_all.sum())} rows"
        if self.gather_ok and kind in ("decode", "ragged"):
            self.g_bytes = A.lib.attn_gather_rows_workspace_bytes(self.max_local, self.row_bytes, world)
            self.g_ws = torch.empty(max(self.g_bytes, 256), dtype=torch.uint8, device=dev)
            self.gather_launches = 1 if kind == "ragged" else 0
        self.working_set = self.work if kind in ("decode", "ragged") else \
            sum(getattr(self, a).numel() * getattr(self, a).element_size() for a in self.in_names + self.out_names)
        if kind == "qkv":
            self.working_set += 3 * self.wq.numel() * 4
        self.legacy_stream = kind == "train"     # the drop-ins run on the legacy default stream

    def unit_is_tflops(self):
        return self.cfg["kind"] in DENSE

    # device tensors a step reads or writes, per kind (the rotated input sets)
    _ROT = {"fwd": ("q", "k", "v", "o", "lse"), "bwd": ("q", "k", "v", "o", "lse", "do", "dq", "dk", "dv"),
            "train": ("q", "k", "v", "o", "do", "dq", "dk", "dv"), "decode": ("kc", "vc", "kp", "vp"), "ragged": (),
            "qkv": ("x", "q", "k", "v")}

    def rotate_inputs(self, n):
        """Keeps n copies of the step's device tensors and cycles through them,
        so that with n x working set > 2 x L2 every step starts from inputs that
        are not L2-resident (instead of flushing the L2 between steps)."""
        names = self._ROT[self.cfg["kind"]]
        base = {k: getattr(self, k) for k in names}
        self.sets = [base]
        for _ in range(n - 1):
            cp = {k: (v.clone() if not isinstance(v, list) else [t.clone() for t in v]) for k, v in base.items()}
            if "kp" in cp:   # the decode pointer tables point at this copy's caches
                cp["kp"] = self.torch.tensor([t.data_ptr() for t in cp["kc"]], dtype=self.torch.int64, device=self.dev)
                cp["vp"] = self.torch.tensor([t.data_ptr() for t in cp["vc"]], dtype=self.torch.int64, device=self.dev)
            self.sets.append(cp)
        self.rot = 0

    def step(self, stream):
        A, c = self.A, self.cfg
        kind = c["kind"]
        if getattr(self, "sets", None) and len(self.sets) > 1:
            for k_, v_ in self.sets[self.rot % len(self.sets)].items():
                setattr(self, k_, v_)
            self.rot += 1
        if kind == "fwd":
            A.fwd_ex(self.shape, self.dtype_code, self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(),
                     self.o.data_ptr(), self.lse.data_ptr(), stream)
        elif kind == "qkv":
            A.check(A.lib.attn_qkv_proj_ex(ctypes.byref(self.shape), self.x.data_ptr(), self.wq.data_ptr(),
                                           self.wk.data_ptr(), self.wv.data_ptr(), self.bq.data_ptr(),
                                           self.bk.data_ptr(), self.bv.data_ptr(), self.q.data_ptr(),
                                           self.k.data_ptr(), self.v.data_ptr(), self.ws.data_ptr(),
                                           self.ws_bytes, stream))
        elif kind == "bwd":
            A.bwd_ex(self.shape, self.dtype_code, self.do.data_ptr(), self.q.data_ptr(), self.k.data_ptr(),
                     self.v.data_ptr(), self.o.data_ptr(), self.lse.data_ptr(), self.dq.data_ptr(),
                     self.dk.data_ptr(), self.dv.data_ptr(), 0, self.ws.data_ptr(), self.ws_bytes, stream)
        elif kind == "train":
            P = ctypes.c_void_p
            A.lib.attn_fwd(P(self.q.data_ptr()), P(self.k.data_ptr()), P(self.v.data_ptr()), P(self.o.data_ptr()),
                           P(self.probs.data_ptr()))
            A.lib.attn_bwd(P(self.dq.data_ptr()), P(self.dk.data_ptr()), P(self.dv.data_ptr()),
                           P(self.scratch.data_ptr()), P(self.do.data_ptr()), P(self.q.data_ptr()),
                           P(self.k.data_ptr()), P(self.v.data_ptr()), P(self.probs.data_ptr()))
        elif kind == "decode":
            s = self.step_idx % c["steps"]
            self.step_idx += 1
            self.o = self.outs[s]
            A.check(A.lib.attn_decode_ptrs_ex(ctypes.byref(self.shape), self.qs[s].data_ptr(), self.kp.data_ptr(),
                                              self.vp.data_ptr(), None, None, self.lens[s].data_ptr(),
                                              self.outs[s].data_ptr(), self.ws.data_ptr(), self.ws_bytes, stream))
        elif self.shape.n_seq:
            A.decode_ex(self.shape, self.q.data_ptr(), self.kc.data_ptr(), self.vc.data_ptr(),
                        self.ks.data_ptr() if self.int8 else None, self.vs.data_ptr() if self.int8 else None,
                        self.lens.data_ptr(), self.o.data_ptr(), self.ws.data_ptr(), self.ws_bytes, stream)

    def gather(self, stream):
        """The whole output on every rank, over the library's NCCL group."""
        A, kind = self.A, self.cfg["kind"]
        if kind == "fwd":
            A.check(A.lib.attn_gather_split(ctypes.byref(self.full_shape), self.dtype_code, self.o.data_ptr(),
                                            self.full.data_ptr(), self.g_ws.data_ptr(), self.g_bytes, stream))
        else:
            order = self.order.data_ptr() if self.order is not None else None
            A.check(A.lib.attn_gather_rows(self.o.data_ptr(), self.max_local, self.row_bytes, order, self.n_out,
                                           self.full.data_ptr(), self.g_ws.data_ptr(), self.g_bytes, stream))

    # --- end to end: host inputs -> device -> call (-> gather) -> host output --
    def setup_e2e(self):
        torch = self.torch
        kind = self.cfg["kind"]
        self.e2e_pipe = kind in ("fwd", "bwd", "train", "ragged", "qkv")
        gather = self.gather_ok
        if self.e2e_pipe:
            # Every step copies its inputs in from pinned host memory and its
            # results out; consecutive steps overlap (H2D, the call and D2H on
            # three streams) over two sets of device and host buffers.  With a
            # gather, rank 0 reads the whole output back and the other ranks
            # read nothing.
            if kind == "ragged":                     # the query rows in, the outputs back
                self.e2e_in, self.e2e_out = ["q"], ["o"]
            else:
                self.e2e_in, self.e2e_out = list(self.in_names), list(self.out_names)
            if gather:
                self.e2e_out = ["full"] if self.rank == 0 else []
            names = self.e2e_in + (["o"] if gather else []) + self.e2e_out
            base = {a: getattr(self, a) for a in dict.fromkeys(names)}
            self.e2e_sets = [base, {a: torch.empty_like(t) for a, t in base.items()}]
            for a in self.e2e_in:                    # both sets hold the same input values
                self.e2e_sets[1][a].copy_(base[a])
            self.h_in = [base[a].cpu().pin_memory() for a in self.e2e_in]
            self.h_outs = [[torch.empty(base[a].shape, dtype=base[a].dtype).pin_memory() for a in self.e2e_out]
                           for _ in range(2)]
            self.h2d_bytes = sum(t.numel() * t.element_size() for t in self.h_in)
            self.d2h_bytes = sum(t.numel() * t.element_size() for t in self.h_outs[0])
            self.s_h2d, self.s_d2h = torch.cuda.Stream(), torch.cuda.Stream()
            self.ev = {n: [torch.cuda.Event(), torch.cuda.Event()] for n in ("h2d", "comp", "d2h")}
            self.e2e_i = 0
            return
        # c1: one step's query rows in, its outputs out, on the call's stream
        self.h_in = [self.qs[0].cpu().pin_memory()]
        self.d_in = [self.qs[0]]
        src = self.full if gather else self.outs[0]
        self.h_out = [torch.empty(src.shape).pin_memory()] if (self.rank == 0 or not gather) else []
        self.d_out = [src] if self.h_out else []
        self.h2d_bytes = sum(t.numel() * t.element_size() for t in self.h_in)
        self.d2h_bytes = sum(t.numel() * t.element_size() for t in self.h_out)

    def e2e_step(self, stream_obj):
        if not self.e2e_pipe:
            for h, d in zip(self.h_in, self.d_in):
                d.copy_(h, non_blocking=True)
            self.step(stream_obj.cuda_stream)
            if self.gather_ok:
                self.gather(stream_obj.cuda_stream)
            for h, d in zip(self.h_out, self.d_out):
                h.copy_(d, non_blocking=True)
            return
        torch = self.torch
        b = self.e2e_i % 2
        self.e2e_i += 1
        S, ev = self.e2e_sets[b], self.ev
        self.s_h2d.wait_event(ev["comp"][b])     # the call that last read set b is done
        with torch.cuda.stream(self.s_h2d):
            for h, a in zip(self.h_in, self.e2e_in):
                S[a].copy_(h, non_blocking=True)
        ev["h2d"][b].record(self.s_h2d)
        stream_obj.wait_event(ev["h2d"][b])
        stream_obj.wait_event(ev["d2h"][b])      # set b's previous results have been read out
        for a, t in S.items():
            setattr(self, a, t)
        self.step(stream_obj.cuda_stream)
        if self.gather_ok:
            self.gather(stream_obj.cuda_stream)
        ev["comp"][b].record(stream_obj)
        self.s_d2h.wait_event(ev["comp"][b])
        with torch.cuda.stream(self.s_d2h):
            for h, a in zip(self.h_outs[b], self.e2e_out):
                h.copy_(S[a], non_blocking=True)
        ev["d2h"][b].record(self.s_d2h)

    def e2e_begin(self, stream_obj, ev0):
        """Orders the copy streams after `ev0` (recorded on the call's stream)."""
        if self.e2e_pipe:
            self.s_h2d.wait_event(ev0)
            self.s_d2h.wait_event(ev0)

    def e2e_end(self, stream_obj):
        """Makes the call's stream wait for every copy issued so far."""
        if self.e2e_pipe:
            for b in range(2):
                stream_obj.wait_event(self.ev["d2h"][b])
                stream_obj.wait_event(self.ev["h2d"][b])


def gpu_baseline(key, args, ctx, wl):
    """The reference's own GPU attention (gpu_kernels.cu's cuBLAS path, built
    from its sources into baseline/_ref/) timed on the same device at the
    same shape: fp32 prefill and backward configs only, one GPU."""
    torch, A = ctx["torch"], ctx["A"]
    cfg = CONFIGS[key]
    if cfg["kind"] == "qkv":
        return gpu_baseline_qkv(args, ctx, wl)
    B, H, T, d = cfg["B"], cfg["H"], cfg["T"], cfg["d"]
    path = os.path.join(ROOT, "baseline", "_ref", f"libref_gpu_{B}x{H}x{T}x{d}.so")
    if not os.path.exists(path):
        return {"unavailable": "baseline/_ref not built (reference sources absent at build time)"}
    L = ctypes.CDLL(path)
    for f in ("refgpu_attn_fwd", "refgpu_attn_bwd"):
        getattr(L, f).restype = None
    L.refgpu_init()
    P = ctypes.c_void_p
    dev = ctx["dev"]
    s0 = torch.cuda.default_stream(dev)           # the reference runs on the legacy default stream
    q, k, v = wl.q, wl.k, wl.v
    att = torch.empty_like(q)
    probs = torch.empty(B * H * T * T, device=dev)
    fwd = lambda: L.refgpu_attn_fwd(P(q.data_ptr()), P(k.data_ptr()), P(v.data_ptr()), P(att.data_ptr()),
                                    P(probs.data_ptr()))
    with torch.cuda.stream(s0):
        if cfg["kind"] == "fwd":
            call = fwd
            ours = torch.empty_like(q)
            A.fwd_ex(wl.shape, A.F32, q.data_ptr(), k.data_ptr(), v.data_ptr(), ours.data_ptr(), None, 0)
            got, theirs = [ours], [att]
            flops = causal_flops(B, H, T, d)
        else:
            fwd()
            dq, dk, dv = (torch.empty_like(q) for _ in range(3))
            scratch = torch.empty_like(probs)
            bwd = lambda: L.refgpu_attn_bwd(P(dq.data_ptr()), P(dk.data_ptr()), P(dv.data_ptr()),
                                            P(scratch.data_ptr()), P(wl.do.data_ptr()), P(q.data_ptr()),
                                            P(k.data_ptr()), P(v.data_ptr()), P(probs.data_ptr()))
            if cfg["kind"] == "train":                # the trainer's call pair
                call = lambda: (fwd(), bwd())
            else:
                call = bwd
            saved, wl.sets = getattr(wl, "sets", None), None
            wl.step(0)                                 # ours on the same inputs (default stream)
            wl.sets = saved
            got, theirs = [wl.dq, wl.dk, wl.dv], [dq, dk, dv]
            if cfg["kind"] == "train":
                got, theirs = got + [wl.o], theirs + [att]
            flops = (3 if cfg["kind"] == "train" else 2) * causal_flops(B, H, T, d)
        for _ in range(args.warmup):
            call()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s0)
        for _ in range(args.steps):
            call()
        e1.record(s0)
        torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / args.steps
    diff = max(float(((a - b).abs().max() / b.abs().max().clamp_min(1e-6)).item()) for a, b in zip(got, theirs))
    return {"value": round(flops / (ms / 1e3) / 1e12, 3), "unit": "TFLOP/s", "ms_per_step": round(ms, 4),
            "kind": "reference GPU path: gpu_kernels.cu %s (cuBLAS SGEMM over the full T x T scores + its "
                    "softmax kernels), built from its sources for sm_100a"
                    % {"fwd": "attn_fwd", "bwd": "attn_bwd", "train": "attn_fwd + attn_bwd"}[cfg["kind"]],
            "max_rel_diff_vs_ours": diff}


def gpu_baseline_qkv(args, ctx, wl):
    """The reference GPU trainer's three gemm_nn calls (gpu_kernels.cu:112-120:
    cuBLAS SGEMM + its bias kernel each, built from its sources into
    baseline/_ref/) on the same inputs, same device."""
    torch, A = ctx["torch"], ctx["A"]
    path = os.path.join(ROOT, "baseline", "_ref", "libref_gpu_4x12x1024x128.so")
    if not os.path.exists(path):
        return {"unavailable": "baseline/_ref not built (reference sources absent at build time)"}
    L = ctypes.CDLL(path)
    L.refgpu_gemm_nn.restype = None
    L.refgpu_init()
    P, I = ctypes.c_void_p, ctypes.c_int
    dev = ctx["dev"]
    s0 = torch.cuda.default_stream(dev)           # the reference runs on the legacy default stream
    M, K, N = wl.shape.rows, wl.shape.in_features, wl.shape.out_features
    outs = [torch.empty_like(wl.q) for _ in range(3)]
    pairs = [(wl.wq, wl.bq), (wl.wk, wl.bk), (wl.wv, wl.bv)]

    def call():
        for (w, b), o in zip(pairs, outs):
            L.refgpu_gemm_nn(P(wl.x.data_ptr()), P(w.data_ptr()), P(b.data_ptr()), P(o.data_ptr()), I(M), I(K), I(N))

    with torch.cuda.stream(s0):
        saved, wl.sets = getattr(wl, "sets", None), None
        wl.step(0)
        wl.sets = saved
        for _ in range(args.warmup):
            call()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s0)
        for _ in range(args.steps):
            call()
        e1.record(s0)
        torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / args.steps
    diff = max(float(((a - b).abs().max() / b.abs().max().clamp_min(1e-6)).item())
               for a, b in zip((wl.q, wl.k, wl.v), outs))
    return {"value": round(qkv_flops(M, K, N) / (ms / 1e3) / 1e12, 3), "unit": "TFLOP/s",
            "ms_per_step": round(ms, 4),
            "kind": "reference GPU path: gpu_kernels.cu gemm_nn x3 (cuBLAS SGEMM + its bias kernel), built from "
                    "its sources for sm_100a",
            "max_rel_diff_vs_ours": diff}


def measure(key, args, ctx):
    """Times one config on every rank; returns the result dict on rank 0."""
    torch, dist, A = ctx["torch"], ctx["dist"], ctx["A"]
    world, rank, local, dev = ctx["world"], ctx["rank"], ctx["local"], ctx["dev"]
    cfg = CONFIGS[key]
    wl = Workload(cfg, A, torch, dev, rank, world)
    stream = torch.cuda.default_stream(dev) if wl.legacy_stream else torch.cuda.Stream(device=dev)
    # Inputs larger than L2 between timed steps: when one step's working set is
    # below 2 x L2, the step's tensors are rotated over enough copies.
    ws = max(1, int(wl.working_set))
    n_sets = 1 if ws >= 2 * L2_BYTES else max(2, -(-5 * L2_BYTES // (2 * ws)))
    if n_sets > 1:
        wl.rotate_inputs(n_sets)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    with torch.cuda.stream(stream):
        t_host = time.perf_counter()
        for _ in range(args.warmup):
            wl.step(stream.cuda_stream)
        t_host = (time.perf_counter() - t_host) / args.warmup     # host seconds to enqueue one step
        stream.synchronize()
        e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        # The K steps run back to back behind one device sleep long enough for
        # the host to enqueue all of them, so that the timed interval holds the
        # steps and the gaps between their kernels, not the host's enqueue.
        sleep_s = min(0.05, 2e-4 + 4.0 * t_host * args.steps)
        with Clocks(local) as clk:
            t_wall = time.perf_counter()
            torch.cuda._sleep(int(sleep_s * 2.0e9))               # cycles at up to 2 GHz
            e_start.record(stream)
            for i in range(args.steps):
                wl.step(stream.cuda_stream)
            e_end.record(stream)
            t_enq = time.perf_counter() - t_wall
            stream.synchronize()
            barrier()
            torch.cuda.synchronize()
            t_wall = time.perf_counter() - t_wall
        total_ms = e_start.elapsed_time(e_end)
        # the gather alone (every rank takes the same collective steps)
        gather_ms = 0.0
        if wl.gather_ok:
            for _ in range(args.warmup):
                wl.gather(stream.cuda_stream)
            stream.synchronize()
            barrier()
            g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            g0.record(stream)
            for _ in range(args.steps):
                wl.gather(stream.cuda_stream)
            g1.record(stream)
            stream.synchronize()
            gather_ms = g0.elapsed_time(g1)
        # end to end through the C ABI with host buffers
        saved_sets = getattr(wl, "sets", None)
        wl.sets = None                               # the e2e leg picks its own buffers
        wl.setup_e2e()
        for _ in range(max(1, args.warmup // 2)):
            wl.e2e_step(stream)
        wl.e2e_end(stream)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        e0.record(stream)
        wl.e2e_begin(stream, e0)
        for _ in range(args.steps):
            wl.e2e_step(stream)
        wl.e2e_end(stream)
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1)
        wl.sets = saved_sets

    h2d_all = wl.h2d_bytes
    gpu_base = None
    if world == 1 and cfg["kind"] in DENSE and cfg["dtype"] == "f32" and not args.no_gpu_baseline:
        gpu_base = gpu_baseline(key, args, ctx, wl)
    if world > 1:
        t = torch.tensor([total_ms, e2e_ms, gather_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, e2e_ms, gather_ms = t.tolist()
        hb = torch.tensor([h2d_all], dtype=torch.float64, device=dev)
        dist.all_reduce(hb)
        h2d_all = int(hb.item())
    clocks = clk.summary()
    res = None
    if rank == 0:
        pk = peaks()
        ms = total_ms / args.steps
        scale = 1e12 if wl.unit_is_tflops() else 1e9
        value = wl.total_work * args.steps / (total_ms / 1e3) / scale
        achieved = wl.work / (ms / 1e3) / scale                 # rank 0's kernel, per launch
        if scale == 1e12:
            peak, bound, punit = pk["bf16"], "tensor", "TFLOP/s"
        else:
            peak, bound, punit = pk["hbm"], "hbm", "GB/s"
        e2e_val = wl.total_work * args.steps / (e2e_ms / 1e3) / scale
        traffic, tinfo = traffic_of(key) if world == 1 else (None, None)
        res = {
            "metric": metric_of(cfg), "value": round(value, 3), "unit": unit_of(cfg), "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
            "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
            "dtype": dtype_of(cfg),
            "config": config_block(key, world),
            "measurement": {"parallelism": ("one GPU" if world == 1 else
                                            f"{world} GPUs, the fixed workload split: rank 0 runs {wl.local_desc}"),
                            "l2": (f"inputs larger than L2: {n_sets} rotated copies of the step's tensors "
                                   f"({n_sets} x {wl.working_set / 2**20:.0f} MiB)") if n_sets > 1
                                  else "inputs larger than L2 (working set > 2 x L2)",
                            "wall_s_timed": round(t_wall, 4),
                            "timing": (f"{args.steps} steps back to back between two CUDA events, queued behind a "
                                       f"{sleep_s * 1e3:.2f} ms device sleep; the host enqueued them in "
                                       f"{t_enq * 1e3:.2f} ms"),
                            "host_ahead_of_device": bool(t_enq < sleep_s)},
            "roofline": {"bound": bound, "achieved": round(achieved, 2), "peak": peak, "unit": punit,
                         "frac": round(achieved / peak, 4), "traffic": traffic, "traffic_capture": tinfo,
                         "peak_source": f"{pk['src']} ({'bf16_tflops burst' if bound == 'tensor' else 'hbm_gbs'})",
                         "algorithmic_work_per_launch": wl.work},
            "e2e": {"value": round(e2e_val, 4), "unit": unit_of(cfg),
                    "h2d_bytes_per_step": h2d_all, "d2h_bytes_per_step": wl.d2h_bytes,
                    "overlap": ("H2D, the call and D2H of consecutive steps overlap on three streams over two "
                                "sets of device and pinned host buffers") if wl.e2e_pipe else "none (one stream)",
                    "includes_gather": bool(wl.gather_ok)},
            "gpu_launches": wl.launches * args.steps,
            "clocks": clocks,
        }
        if gpu_base is not None:
            res["gpu_baseline"] = gpu_base
        if world > 1:
            res["gather"] = ({"ms_per_step": round(gather_ms / args.steps, 5),
                              "what": ("attn_gather_split: NCCL all-gather of every rank's compact split"
                                       + (" + permute kernel" if wl.gather_launches else " (in place)"))
                              if cfg["kind"] == "fwd" else
                              ("attn_gather_rows: NCCL all-gather of every rank's rows"
                               + (" + scatter kernel" if wl.gather_launches else "")),
                              "bytes_received_per_rank": int(wl.full.numel() * wl.full.element_size())}
                             if wl.gather_ok else
                             {"ms_per_step": None, "what": "none: each rank's dQ/dK/dV stay with its heads"})
    del wl
    torch.cuda.empty_cache()
    return res


def run_ours(args, keys):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    import attn_b200 as A
    if world > 1:
        import shard
        shard.init_group(rank, world, local)
    ctx = dict(torch=torch, dist=dist, A=A, world=world, rank=rank, local=local, dev=dev)
    results = {}
    for key in keys:
        results[key] = measure(key, args, ctx)
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier(device_ids=[local])
        A.check(A.lib.attn_finalize())
        dist.destroy_process_group()
    return results if rank == 0 else None


def reference_config(key, args):
    """The reference's CPU attention over a bounded sample of the workload:
    W untimed samples, then K timed ones; the value is their median."""
    cfg = CONFIGS[key]
    s = CpuSample(cfg)
    for _ in range(args.warmup):
        s.call()
    vals = [s.work / s.call() for _ in range(args.steps)]
    value = statistics.median(vals)
    cb = dict(value=value, unit=s.unit, cores=s.cores, kind="reference",
              sample=f"{s.sample}, median of {args.steps}")
    return {"metric": metric_of(cfg), "value": round(value, 6), "unit": s.unit, "dtype": "f32",
            "config": {"workload": cfg["workload"], "config_key": key},
            "cpu_baseline": cb,
            "e2e": {"value": round(value, 6), "unit": s.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def json_stream():
    """Rank 0's stdout carries the JSON line and nothing else.  Native code
    prints on file descriptor 1 too (NCCL its version line when a communicator
    is set up, with NCCL_DEBUG set), so descriptor 1 is pointed at stderr for
    the whole run and the line goes to a duplicate of the original stdout."""
    sys.stdout.flush()
    out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    return out


def emit(out, line):
    out.write(json.dumps(line) + "\n")
    out.flush()


def main():
    out = json_stream()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=["all"] + sorted(CONFIGS), default="all")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    keys = ORDER if args.config == "all" else [args.config]
    head = HEADLINE if args.config == "all" else args.config
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        try:
            from oracle import oracle as O
            if not O.ref_available():
                emit(out, {"impl": "reference", "unavailable": "oracle/_ref not built (reference sources "
                                "absent at build time)"})
                return
        except Exception as e:  # pragma: no cover
            emit(out, {"impl": "reference", "unavailable": f"oracle import failed: {e}"})
            return
        per = {k: reference_config(k, args) for k in keys}
        top = dict(per[head])
        line = {"impl": "reference", "metric": top["metric"] if args.config != "all" else METRIC,
                "value": top["value"], "unit": top["unit"], "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded normal inputs of the config's shape)",
                "config": config_block(head, world), "cpu_baseline": top["cpu_baseline"], "e2e": top["e2e"]}
        if args.config == "all":
            line["headline"] = f"{head}: {top['metric']}"
            line["configs"] = {k: {kk: vv for kk, vv in v.items() if kk != "config"} | {"config": config_block(k, world)}
                               for k, v in per.items()}
        emit(out, line)
        return

    res = run_ours(args, keys)
    if res is None:
        return
    if world == 1 and not args.no_cpu_baseline:
        budget = 12.0 if len(keys) == 1 else 2.5
        for k in keys:
            res[k]["cpu_baseline"] = cpu_reference(CONFIGS[k], budget_s=budget)
    line = dict(res[head])
    line["data"] = "synthetic (seeded normal inputs of the config's shape)"
    if args.config == "all":
        line["headline"] = f"{head}: {line['metric']}"
        line["metric"] = METRIC
        line["gpu_launches"] = sum(r["gpu_launches"] for r in res.values())
        line["configs"] = {k: {kk: vv for kk, vv in r.items()
                               if kk not in ("steps", "warmup", "n_gpus", "higher_is_better", "vs_baseline")}
                           for k, r in res.items()}
    emit(out, line)


def config_block(key, world):
    """The config dict both arms print for a workload (the identical part)."""
    cfg = CONFIGS[key]
    return {"workload": cfg["workload"], "config_key": key,
            "split": "none (one GPU)" if world == 1 else
            {"fwd": "(batch x head) units, attn_split_plan", "bwd": "(batch x head) units, attn_split_plan",
             "train": "(batch x head) units, attn_split_plan", "decode": "layers", "qkv": "token rows",
             "ragged": "sequences, LPT by length"}[cfg["kind"]]}


if __name__ == "__main__":
    main()
