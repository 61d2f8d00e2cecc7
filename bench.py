#!/usr/bin/env python
"""Benchmark of the fused layer-op hot path on B200 (one process per GPU).

Workload (benchmark config 4, the Llama-3-8B-shaped prefill layer ops, bf16):
batch 8 x seq 4096 = 32768 token rows per GPU, hidden 4096, 32 query / 8 KV
heads of 128, intermediate 14336, vocabulary 128256. One step is one pass of
the hot path over that batch:
  1. embedding gather  x = table[ids]                  (xn_index_select)
  2. RMSNorm           y1 = rms_norm(x)                  (xn_rms_norm)
  3. RoPE on Q and K   theta = 500000, positions 0..4095 (xn_rope_qk)
  4. residual+RMSNorm  h = x + attn_out; y2 = rms_norm(h) (xn_rms_norm, fused)
  5. SwiGLU            act = silu(gate) * up              (xn_swiglu)
Inputs are seeded synthetic tensors already resident in HBM; every tensor is
larger than the 126 MB L2 except the weights and cos/sin tables, so no L2
flush is needed between steps.

The metric is algorithmic HBM bytes per second (GB/s) over the whole job:
each op's bytes are its compulsory reads and writes (formulas in
op_bytes()), summed over the step and over all ranks (weak scaling: every rank
runs the full per-GPU batch, with no collective on the data path).

`--impl reference` times the reference CPU backend's algorithm (the oracle
restatement of mimi-rs/src/cpu_backend.rs) on the host cores for the same
workload and metric, on a bounded sample of rows.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
for _p in (REPO / "random-things_b200", REPO / "oracle"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

METRIC = "fused-op HBM GB/s (% of B200 peak) & Mimi decode frames/s, 1–8 GPUs"
UNIT = "GB/s"
FALLBACK_HBM_GBS = 6650.0

CFG = dict(batch=8, seq=4096, hidden=4096, heads_q=32, heads_kv=8, head_dim=128, inter=14336,
           vocab=128256, theta=500000.0, eps=1e-5)
OPS = ["embedding_gather", "rms_norm", "rope_qk", "rms_norm_residual", "swiglu"]
# Kernel-name fragments of each op (ncu launch list and roofline traffic).
KERNELS = {"embedding_gather": "gather_rows_kernel", "rms_norm": "norm_vec_kernel",
           "rope_qk": "rope_kernel", "rms_norm_residual": "norm_vec_kernel", "swiglu": "swiglu_kernel"}


def op_bytes(cfg: dict, rows: int, s: int = 2, id_bytes: int = 4) -> dict:
    """Algorithmic HBM bytes per op for `rows` token rows (1-D weights once)."""
    H, I, D = cfg["hidden"], cfg["inter"], cfg["head_dim"]
    seq = cfg["seq"]
    b = rows // seq
    q_el = b * cfg["heads_q"] * seq * D
    k_el = b * cfg["heads_kv"] * seq * D
    return {
        "embedding_gather": rows * id_bytes + 2 * rows * H * s,
        "rms_norm": 2 * rows * H * s + H * s,
        "rope_qk": 2 * (q_el + k_el) * s + 2 * seq * (D // 2) * s,
        "rms_norm_residual": 4 * rows * H * s + H * s,
        "swiglu": 3 * rows * I * s,
    }


def measured_peak() -> tuple[float, str]:
    p = REPO / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback (6.65 TB/s earlier pool measurement)"


def load_traffic() -> dict:
    """Per-launch DRAM bytes from the committed ncu summary, if present."""
    p = REPO / "profiles" / "traffic.json"
    try:
        return json.loads(p.read_text())
    except Exception:
        return {}


# ---------------------------------------------------------------------------
# Clock sampling during the timed region (nvidia-smi, 200 ms).
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None):
        self.uuid = uuid
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 8:
                continue
            if self.uuid and parts[0] != self.uuid:
                continue
            rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        try:
            sm = [float(r[1]) for r in rows]
            mx = max(float(r[2]) for r in rows)
        except ValueError:
            return None
        loaded = [r for r in rows if float(r[1]) > 0.5 * mx] or rows
        reasons = sorted({names[i] for r in rows for i in range(4) if r[4 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(float(r[1]) for r in loaded), "sm_max_mhz": mx,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# The GPU workload.
# ---------------------------------------------------------------------------
class LlamaPrefillOps:
    """The per-GPU workload: `batch` sequences of `seq` tokens (rows = batch*seq)."""

    def __init__(self, torch, xn, device, cfg: dict, seed: int = 0, ops=OPS):
        self.torch, self.xn, self.dev, self.cfg, self.ops = torch, xn, device, cfg, list(ops)
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        bf = torch.bfloat16
        B, S, H, I, D = cfg["batch"], cfg["seq"], cfg["hidden"], cfg["inter"], cfg["head_dim"]
        R = B * S
        self.rows = R

        def randn(shape, std=1.0, mean=0.0):
            t = torch.empty(shape, dtype=torch.float32, device=device)
            t.normal_(mean, std, generator=g)
            return t.to(bf)

        def need(*names):
            return any(n in self.ops for n in names)

        if need("embedding_gather"):
            self.table = randn((cfg["vocab"], H), 0.02)
            self.ids = torch.randint(0, cfg["vocab"], (R,), dtype=torch.int32, device=device, generator=g)
        if need("embedding_gather", "rms_norm", "rms_norm_residual"):
            self.x = randn((R, H))
        if need("rms_norm"):
            self.alpha1 = randn((H,), 0.02, 1.0)
            self.y1 = torch.empty_like(self.x)
        if need("rms_norm_residual"):
            self.alpha2 = randn((H,), 0.02, 1.0)
            self.attn_out = randn((R, H))
            self.h = torch.empty_like(self.x)
            self.y2 = torch.empty_like(self.x)
        if need("rope_qk"):
            self.q = randn((B, cfg["heads_q"], S, D))
            self.k = randn((B, cfg["heads_kv"], S, D))
            half = D // 2
            inv = 1.0 / (cfg["theta"] ** (torch.arange(half, dtype=torch.float32) * 2.0 / D))
            ang = torch.arange(S, dtype=torch.float32)[:, None] * inv[None, :]
            self.cos = ang.cos().to(bf).to(device)
            self.sin = ang.sin().to(bf).to(device)
            self.qo = torch.empty_like(self.q)
            self.ko = torch.empty_like(self.k)
        if need("swiglu"):
            self.gate = randn((R, I))
            self.up = randn((R, I))
            self.act = torch.empty_like(self.gate)
        allb = op_bytes(cfg, R)
        self.bytes = {n: allb[n] for n in self.ops}

    def run_op(self, name: str, b0: int = 0, b1: int | None = None):
        """One op on batch elements [b0, b1) (token rows [b0*seq, b1*seq))."""
        xn, c = self.xn, self.cfg
        b1 = self.cfg["batch"] if b1 is None else b1
        r0, r1 = b0 * c["seq"], b1 * c["seq"]
        if name == "embedding_gather":
            xn.index_select(self.table, self.ids[r0:r1], 0, out=self.x[r0:r1])
        elif name == "rms_norm":
            xn.rms_norm_(self.y1[r0:r1], self.x[r0:r1], self.alpha1, c["eps"])
        elif name == "rope_qk":
            xn.rope_qk(self.q[b0:b1], self.k[b0:b1], self.cos, self.sin, 0, out=(self.qo[b0:b1], self.ko[b0:b1]))
        elif name == "rms_norm_residual":
            xn.rms_norm_(self.y2[r0:r1], self.x[r0:r1], self.alpha2, c["eps"], branch=self.attn_out[r0:r1],
                         residual_out=self.h[r0:r1])
        elif name == "swiglu":
            xn.swiglu_(self.act[r0:r1], self.gate[r0:r1], self.up[r0:r1])

    def step(self, events=None):
        for i, name in enumerate(self.ops):
            if events is not None:
                events[i][0].record()
            self.run_op(name)
            if events is not None:
                events[i][1].record()

    # -- End to end through the public API with host buffers ------------------
    # Every step copies its inputs from pinned host memory and all of its
    # outputs back. The step is cut into per-sequence chunks on three streams
    # (H2D, compute, D2H) so both PCIe directions and the kernels overlap.
    IN_NAMES = ("ids", "attn_out", "q", "k", "gate", "up")
    OUT_NAMES = ("x", "y1", "h", "y2", "qo", "ko", "act")

    def host_buffers(self):
        t = self.torch
        self.h_in = {k: t.empty(getattr(self, k).shape, dtype=getattr(self, k).dtype, pin_memory=True)
                     .copy_(getattr(self, k)) for k in self.IN_NAMES if hasattr(self, k)}
        self.h_out = {k: t.empty(getattr(self, k).shape, dtype=getattr(self, k).dtype, pin_memory=True)
                      for k in self.OUT_NAMES if hasattr(self, k)}
        self.h2d_bytes = sum(v.numel() * v.element_size() for v in self.h_in.values())
        self.d2h_bytes = sum(v.numel() * v.element_size() for v in self.h_out.values())
        self.s_h2d, self.s_d2h = t.cuda.Stream(), t.cuda.Stream()
        self.s_comp = t.cuda.current_stream()

    def _chunk(self, name: str, b0: int, b1: int):
        seq = self.cfg["seq"]
        t = getattr(self, name)
        return t[b0:b1] if name in ("q", "k", "qo", "ko") else t[b0 * seq:b1 * seq]

    def transfer_step(self, chunk: int = 1):
        """The copies of e2e_step alone (same bytes, chunks and streams, no
        kernels): the host-link bound of the end-to-end step."""
        t = self.torch
        B, seq = self.cfg["batch"], self.cfg["seq"]
        for b0 in range(0, B, chunk):
            b1 = min(B, b0 + chunk)
            with t.cuda.stream(self.s_h2d):
                for k, v in self.h_in.items():
                    self._chunk(k, b0, b1).copy_(v[b0:b1] if k in ("q", "k") else v[b0 * seq:b1 * seq],
                                                 non_blocking=True)
            with t.cuda.stream(self.s_d2h):
                for k, v in self.h_out.items():
                    dst = v[b0:b1] if k in ("qo", "ko") else v[b0 * seq:b1 * seq]
                    dst.copy_(self._chunk(k, b0, b1), non_blocking=True)
        self.s_comp.wait_stream(self.s_h2d)
        self.s_comp.wait_stream(self.s_d2h)

    def e2e_step(self, chunk: int = 1):
        """Chunk c's H2D waits for the previous step's kernels on chunk c (its
        inputs are being overwritten) and chunk c's kernels wait for the
        previous step's D2H of chunk c (its outputs are being overwritten)."""
        t = self.torch
        B = self.cfg["batch"]
        prev = getattr(self, "_prev_events", {})
        cur = {}
        for b0 in range(0, B, chunk):
            b1 = min(B, b0 + chunk)
            with t.cuda.stream(self.s_h2d):
                if b0 in prev:
                    self.s_h2d.wait_event(prev[b0][0])
                for k, v in self.h_in.items():
                    dev = self._chunk(k, b0, b1)
                    dev.copy_(v[b0:b1] if k in ("q", "k") else v[b0 * self.cfg["seq"]:b1 * self.cfg["seq"]],
                              non_blocking=True)
                ev_in = t.cuda.Event()
                ev_in.record(self.s_h2d)
            self.s_comp.wait_event(ev_in)
            if b0 in prev:
                self.s_comp.wait_event(prev[b0][1])
            for name in self.ops:
                self.run_op(name, b0, b1)
            ev_out = t.cuda.Event()
            ev_out.record(self.s_comp)
            with t.cuda.stream(self.s_d2h):
                self.s_d2h.wait_event(ev_out)
                for k, v in self.h_out.items():
                    src = self._chunk(k, b0, b1)
                    dst = v[b0:b1] if k in ("qo", "ko") else v[b0 * self.cfg["seq"]:b1 * self.cfg["seq"]]
                    dst.copy_(src, non_blocking=True)
                ev_d2h = t.cuda.Event()
                ev_d2h.record(self.s_d2h)
            cur[b0] = (ev_out, ev_d2h)
        self._prev_events = cur
        # The step ends when its last output is on the host.
        self.s_comp.wait_stream(self.s_d2h)


# ---------------------------------------------------------------------------
# Mimi decode frames/s (benchmark config 2): RVQ decode + 8-layer decoder
# transformer on the fused ops, replayed as one CUDA graph.
# ---------------------------------------------------------------------------
def mimi_rate(torch, device, steps: int, batch: int = 4, frames: int = 250) -> dict:
    import mimi_chain as mc

    cfg = mc.MimiChainConfig()
    w = mc.synthetic_weights(cfg, torch.bfloat16, device, seed=7)
    cos, sin = mc.rope_tables(cfg, torch.bfloat16, device)
    chain = mc.MimiDecoderChain(cfg, w, cos, sin)
    g = torch.Generator().manual_seed(8)
    codes_h = torch.randint(0, cfg.bins, (batch, cfg.n_q, frames), generator=g, dtype=torch.int64).pin_memory()
    codes = codes_h.to(device)
    for _ in range(3):
        out = chain.decode(codes)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = chain.decode(codes)
    out_h = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    # End to end: codes H2D, decode, output D2H, every step.
    e0.record()
    for _ in range(steps):
        codes.copy_(codes_h, non_blocking=True)
        graph.replay()
        out_h.copy_(out, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    ms_e2e = e0.elapsed_time(e1) / steps
    del graph
    n = batch * frames
    return {"frames_per_s": round(n / (ms * 1e-3), 1), "ms_per_decode": round(ms, 4),
            "e2e_frames_per_s": round(n / (ms_e2e * 1e-3), 1), "batch": batch, "frames": frames,
            "dtype": "bf16", "layers": cfg.num_layers, "d_model": cfg.d_model, "codebooks": cfg.n_q,
            "what": "whole-sequence (non-streaming) decode, Mimi::decode's path without the conv stages: RVQ decode "
                    "(8 x 2048 x 256) + 8-layer decoder transformer over all 250 frames at once (LN, RoPE, causal "
                    "softmax, GELU fused ops; GEMMs on cuBLAS), one CUDA graph; not the reference's streaming "
                    "realtime loop, which is mimi_stream_decode; seeded synthetic weights"}


def gather_context(torch, xn, device, reps: int = 7) -> list:
    """The config-4 embedding gather (32768 ids into the 128256 x 4096 table)
    timed alone after different predecessors: a write flush or the step's
    SwiGLU (both leave ~126 MB of dirty lines in L2, written back during the
    gather) and the same followed by a clean 256 MB read (L2 left clean).
    Shows how much of the gather's in-step time is its predecessor's
    write-back."""
    g = torch.Generator(device=device).manual_seed(0)
    table = (torch.randn((CFG["vocab"], CFG["hidden"]), device=device, generator=g) * 0.02).to(torch.bfloat16)
    rows = CFG["batch"] * CFG["seq"]
    ids = torch.randint(0, CFG["vocab"], (rows,), dtype=torch.int32, device=device, generator=g)
    out = torch.empty((rows, CFG["hidden"]), dtype=torch.bfloat16, device=device)
    gate = torch.randn((rows, CFG["inter"]), device=device, generator=g).to(torch.bfloat16)
    up = torch.randn((rows, CFG["inter"]), device=device, generator=g).to(torch.bfloat16)
    act = torch.empty_like(gate)
    wflush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=device)
    rflush = torch.zeros(64 * 1024 * 1024, dtype=torch.float32, device=device)
    nbytes = rows * 4 + 2 * rows * CFG["hidden"] * 2
    peak, _ = measured_peak()

    def timed(pre):
        ts = []
        for _ in range(reps):
            pre()
            torch.cuda._sleep(1_000_000)  # host enqueues the events and the op while the GPU is busy
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            xn.index_select(table, ids, 0, out=out)
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        ms = statistics.median(ts)
        return {"ms": round(ms, 4), "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1),
                "frac": round(nbytes / (ms * 1e-3) / 1e9 / peak, 3)}

    return [dict(after="write flush (256 MB)", **timed(lambda: wflush.zero_())),
            dict(after="write flush + clean read", **timed(lambda: (wflush.zero_(), rflush.sum()))),
            dict(after="swiglu (the step's last op)", **timed(lambda: xn.swiglu_(act, gate, up))),
            dict(after="swiglu + clean read", **timed(lambda: (xn.swiglu_(act, gate, up), rflush.sum())))]


# ---------------------------------------------------------------------------
# Benchmark config 1: the CPU-runnable f32 micro-pipeline, timed on the GPU.
# ---------------------------------------------------------------------------
C1 = dict(tokens=512, hidden=2048, heads=16, head_dim=128, inter=5632, theta=10000.0, eps=1e-5)


def l2_flusher(torch, device):
    """Returns flush(): writes 256 MB (> the 126 MB L2), then reads another
    256 MB buffer, so the L2 holds only clean lines of the second buffer and a
    launch timed after it pays for no write-back of the flush."""
    wbuf = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)
    rbuf = torch.zeros(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)

    def flush():
        wbuf.zero_()
        rbuf.sum()
    return flush


def time_flushed(torch, fn, flush, reps: int) -> float:
    """Median CUDA-event time (ms) of fn() over `reps` launches, each after an
    L2 flush and a fixed GPU spin (so host launch latency never falls between
    the two events)."""
    times = []
    for _ in range(reps):
        flush()
        torch.cuda._sleep(1_000_000)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    return statistics.median(times)


def config1_rate(torch, xn, device, reps: int = 20) -> dict:
    """Benchmark config 1 (f32, seeded): x ~ N(0,1) [1, 512, 2048] -> RMSNorm
    (eps 1e-5, weight ~ N(1, 0.02)); RoPE (theta 1e4, half-split) on Q / K
    [1, 512, 16, 128] ~ N(0,1) at positions 0..511 ([B, T, H, D], no
    transposes); SwiGLU on gate / up [1, 512, 5632] ~ N(0,1); causal softmax
    over [1, 16, 512, 512] logits ~ N(0, 4). Each op is timed alone after an
    L2 flush (every input is smaller than the L2), then the four ops as one
    CUDA graph after a flush. The reference CPU backend's own path for these
    ops is cpu_backend.rs:359-392, 667-709."""
    c = C1
    g = torch.Generator(device=device).manual_seed(11)
    T, H, NH, D, I = c["tokens"], c["hidden"], c["heads"], c["head_dim"], c["inter"]

    def rnd(*shape, std=1.0, mean=0.0):
        t = torch.empty(shape, dtype=torch.float32, device=device)
        return t.normal_(mean, std, generator=g)

    x, w = rnd(1, T, H), rnd(H, std=0.02, mean=1.0)
    y = torch.empty_like(x)
    q, k = rnd(1, T, NH, D), rnd(1, T, NH, D)
    qo, ko = torch.empty_like(q), torch.empty_like(k)
    half = D // 2
    inv = 1.0 / (c["theta"] ** (torch.arange(half, dtype=torch.float32) * 2.0 / D))
    ang = torch.arange(T, dtype=torch.float32)[:, None] * inv[None, :]
    cos, sin = ang.cos().to(device), ang.sin().to(device)
    gate, up = rnd(1, T, I), rnd(1, T, I)
    act = torch.empty_like(gate)
    logits = rnd(1, NH, T, T, std=2.0)
    probs = torch.empty_like(logits)
    s = 4
    live = NH * T * (T + 1) // 2  # unmasked logits: row i reads i + 1 of them
    ops = {
        "rms_norm": (lambda: xn.rms_norm_(y, x, w, c["eps"]), 2 * T * H * s + H * s),
        "rope_qk": (lambda: xn.rope_qk(q, k, cos, sin, 0, layout="bthd", out=(qo, ko)),
                    2 * 2 * T * NH * D * s + 2 * T * half * s),
        "swiglu": (lambda: xn.swiglu_(act, gate, up), 3 * T * I * s),
        "softmax_causal": (lambda: xn.softmax_causal_(probs, logits, 0), (live + NH * T * T) * s),
    }
    flush = l2_flusher(torch, device)
    peak, _ = measured_peak()
    for fn, _ in ops.values():
        fn()
    out = {}
    for name, (fn, nbytes) in ops.items():
        ms = time_flushed(torch, fn, flush, reps)
        gbs = nbytes / (ms * 1e-3) / 1e9
        # The size reference: torch's device copy moving the same bytes (half read, half written).
        a = torch.empty(nbytes // 8, dtype=torch.float32, device=device)
        b = torch.empty_like(a)
        copy_ms = time_flushed(torch, lambda: b.copy_(a), flush, reps)
        out[name] = {"us": round(ms * 1e3, 2), "bytes": nbytes, "gbs": round(gbs, 1), "frac": round(gbs / peak, 3),
                     "copy_same_bytes_us": round(copy_ms * 1e3, 2)}
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(stream):
        for fn, _ in ops.values():
            fn()
    torch.cuda.current_stream(device).wait_stream(stream)
    torch.cuda.synchronize()
    with torch.cuda.graph(graph, stream=stream):
        for fn, _ in ops.values():
            fn()
    ms = time_flushed(torch, graph.replay, flush, reps)
    total = sum(b for _, b in ops.values())
    del graph
    return {"per_op": out, "pipeline_us": round(ms * 1e3, 2), "pipeline_bytes": total,
            "pipeline_gbs": round(total / (ms * 1e-3) / 1e9, 1),
            "pipeline_frac": round(total / (ms * 1e-3) / 1e9 / peak, 3),
            "what": "benchmark config 1, f32: RMSNorm [512, 2048], RoPE half-split on Q/K [1, 512, 16, 128] (BTHD), "
                    "SwiGLU [512, 5632], causal softmax [1, 16, 512, 512]; each op after an L2 flush (inputs are "
                    "smaller than L2), median of launches; pipeline = the four ops as one CUDA graph after a flush; "
                    "causal softmax bytes = unmasked reads + all writes; copy_same_bytes_us = torch's device copy "
                    "of the same bytes, timed the same way (what a launch of that size takes at all)"}


# ---------------------------------------------------------------------------
# Mimi streaming decode (benchmark config 2 shapes, frame by frame).
# ---------------------------------------------------------------------------
def mimi_stream_rate(torch, device, steps: int, batch: int = 4) -> dict:
    """Mimi::decode_step without its conv stages (mimi_chain.MimiStreamingDecoder):
    per step the codes of one frame [B, 8, 1] -> RVQ decode (8 x 2048 x 256)
    -> one step of the 8-layer decoder transformer (context-250 ring KV
    caches, offset = min(frames seen, 250)), one captured CUDA graph per step.
    `steps` frames from an empty cache (past 250, so the steady state with a
    full context is included); frames/s = batch x steps / time. End to end:
    each step's codes copied from pinned host memory and its output read back."""
    import mimi_chain as mc

    cfg = mc.MimiChainConfig()
    w = mc.synthetic_weights(cfg, torch.bfloat16, device, seed=7)
    cos, sin = mc.rope_tables(cfg, torch.bfloat16, device)
    dec = mc.MimiStreamingDecoder(cfg, w, cos, sin, batch, context=cfg.context)
    g = torch.Generator(device=device).manual_seed(12)
    codes = torch.randint(0, cfg.bins, (steps, batch, cfg.n_q, 1), dtype=torch.int64, device=device, generator=g)
    dec.capture(1)
    for s in range(3):
        dec.step_graph(codes[s])
    torch.cuda.synchronize()
    dec.reset()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for s in range(steps):
        dec.step_graph(codes[s])
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / steps
    codes_h = codes.cpu().pin_memory()
    out_h = torch.empty(dec.out_static.shape, dtype=torch.bfloat16, pin_memory=True)
    dec.reset()
    torch.cuda.synchronize()
    e0.record()
    for s in range(steps):
        dec.x_static.copy_(codes_h[s], non_blocking=True)
        dec.graph.replay()
        out_h.copy_(dec.out_static, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    us_e2e = e0.elapsed_time(e1) * 1e3 / steps
    del dec
    return {"us_per_step": round(us, 2), "frames_per_s": round(batch / (us * 1e-6), 1),
            "e2e_us_per_step": round(us_e2e, 2), "e2e_frames_per_s": round(batch / (us_e2e * 1e-6), 1),
            "batch": batch, "steps": steps, "context": cfg.context, "dtype": "bf16", "layers": cfg.num_layers,
            "h2d_bytes_per_step": batch * cfg.n_q * 8, "d2h_bytes_per_step": batch * cfg.d_model * 2,
            "what": "Mimi::decode_step without the conv upsample / SEANet decoder: RVQ decode of one frame + one "
                    "step of the 8-layer decoder transformer with context-250 ring KV caches (fused LN/residual, "
                    "KV append + RoPE + decode attention, GELU; GEMMs on cuBLAS), one CUDA graph per step; the "
                    "reference's streaming realtime loop (mimi-rs/examples/mimi.rs:220-235) at batch 4; seeded "
                    "synthetic weights"}


def cpu_mimi_stream_rate(steps: int = 3, batch: int = 4) -> dict:
    """The reference streaming op sequence of mimi_stream_rate on the CPU oracle
    (oracle ops single-threaded, numpy f32 GEMMs rounded to bf16): mean time
    per step of the steps after a warm-up step."""
    import numpy as np

    import mimi_chain as mc
    import mimi_oracle
    import xn_oracle
    import torch

    cfg = mc.MimiChainConfig()
    w = {k: mimi_oracle.to_storage(v.float().numpy(), "bf16")
         for k, v in mc.synthetic_weights(cfg, torch.float32, "cpu", seed=7).items()}
    cos, sin = (mimi_oracle.to_storage(t.float().numpy(), "bf16") for t in mc.rope_tables(cfg, torch.float32, "cpu"))
    r = np.random.default_rng(12)
    codes = [r.integers(0, cfg.bins, size=(batch, cfg.n_q, 1), dtype=np.int64) for _ in range(steps + 1)]
    with _oracle_threads(xn_oracle, 1):
        t0 = time.perf_counter()
        mimi_oracle.stream_ref(xn_oracle, cfg, w, cos, sin, codes[:1], "bf16", 0.125, cfg.context,
                               mask="cache_len", codes=True)
        t1 = time.perf_counter()
        mimi_oracle.stream_ref(xn_oracle, cfg, w, cos, sin, codes, "bf16", 0.125, cfg.context, mask="cache_len",
                               codes=True)
        t2 = time.perf_counter()
    us = ((t2 - t1) - (t1 - t0)) / steps * 1e6
    return {"us_per_step": round(us, 1), "frames_per_s": round(batch / (us * 1e-6), 1),
            "sample": f"steps 2..{steps + 1} of a stream at batch {batch}, bf16, oracle ops single-threaded + "
                      f"numpy f32 GEMMs on {os.cpu_count()} BLAS threads"}


def cpu_config1_rate(reps: int = 3) -> dict:
    """Benchmark config 1 on the CPU oracle (row-parallel ops on every host
    core, unary/binary single-threaded as the reference): per-op and
    pipeline time."""
    import numpy as np

    import xn_oracle as o

    o.build()
    threads = os.cpu_count() or 1
    c = C1
    r = np.random.default_rng(11)
    T, H, NH, D, I = c["tokens"], c["hidden"], c["heads"], c["head_dim"], c["inter"]
    f = lambda *shape, std=1.0, mean=0.0: (r.standard_normal(shape, dtype=np.float32) * np.float32(std)  # noqa: E731
                                          + np.float32(mean)).astype(np.float32)
    x, w = f(1, T, H), f(H, std=0.02, mean=1.0)
    q = np.ascontiguousarray(np.transpose(f(1, T, NH, D), (0, 2, 1, 3)))  # the reference rotates [B, H, T, D]
    k = np.ascontiguousarray(np.transpose(f(1, T, NH, D), (0, 2, 1, 3)))
    cos, sin = o.rope_tables(D, T, c["theta"], "f32", "llama")
    gate, up, logits = f(1, T, I), f(1, T, I), f(1, NH, T, T, std=2.0)
    ops = {"rms_norm": lambda: o.rms_norm(x, w, c["eps"], "f32"),
           "rope_qk": lambda: (o.rope(q, cos, sin, 0, "f32"), o.rope(k, cos, sin, 0, "f32")),
           "swiglu": lambda: o.swiglu(gate, up, "f32"),
           "softmax_causal": lambda: o.softmax_causal(logits, 0, "f32")}
    o.set_num_threads(threads)
    out = {}
    for name, fn in ops.items():
        fn()
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        out[name] = {"us": round(statistics.median(ts) * 1e6, 1)}
    return {"per_op": out, "pipeline_us": round(sum(v["us"] for v in out.values()), 1), "cores": threads,
            "sample": "the whole config-1 pipeline (it is CPU-sized), median of 3 runs per op"}


DECODE_CFG = dict(d_model=1024, num_heads=16, num_layers=6, dim_feedforward=4096)


def decode_rate(torch, device, steps: int, act: str, batch: int = 16) -> dict:
    """Benchmark config 3: streaming decode, B=16, D=1024, 16 heads of 64, 6
    layers, MLP 4096, one frame per step for steps t = 1..`steps` (the cache
    grows to `steps` positions). One captured CUDA graph per step (all
    layers, the position read from device memory) replayed for every step.
    Reports the mean time per step over the whole stream, inputs resident in
    HBM, and end to end with each step's input copied from pinned host memory
    and its output read back."""
    import mimi_chain as mc

    cfg = mc.MimiChainConfig(**DECODE_CFG)
    w = mc.synthetic_weights(cfg, torch.bfloat16, device, seed=9)
    cos, sin = mc.rope_tables(cfg, torch.bfloat16, device)
    chain = mc.StreamingDecoderChain(cfg, w, cos, sin, batch, act=act, context=steps)
    g = torch.Generator(device=device).manual_seed(10)
    xs = torch.randn((steps, batch, 1, cfg.d_model), device=device, generator=g).to(torch.bfloat16)
    chain.capture(1)
    for s in range(3):
        chain.step_graph(xs[s])
    torch.cuda.synchronize()
    chain.reset()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for s in range(steps):
        chain.step_graph(xs[s])
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / steps
    xs_h = xs.cpu().pin_memory()
    out_h = torch.empty(chain.out_static.shape, dtype=torch.bfloat16, pin_memory=True)
    chain.reset()
    torch.cuda.synchronize()
    e0.record()
    for s in range(steps):
        chain.x_static.copy_(xs_h[s], non_blocking=True)
        chain.graph.replay()
        out_h.copy_(chain.out_static, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    us_e2e = e0.elapsed_time(e1) * 1e3 / steps
    weight_bytes = sum(v.numel() * v.element_size() for k, v in w.items() if k.startswith("layers."))
    del chain
    return {"us_per_step": round(us, 2), "frames_per_s": round(batch / (us * 1e-6), 1),
            "e2e_us_per_step": round(us_e2e, 2), "e2e_frames_per_s": round(batch / (us_e2e * 1e-6), 1),
            "weight_gbs": round(weight_bytes / (us * 1e-6) / 1e9, 1),
            "batch": batch, "steps": steps, "dtype": "bf16", "mlp_activation": act, **DECODE_CFG,
            "h2d_bytes_per_step": batch * cfg.d_model * 2, "d2h_bytes_per_step": batch * cfg.d_model * 2,
            "what": "streaming decoder transformer, one frame per step (benchmark config 3): fused LN/residual, "
                    "KV-cache append + RoPE, decode attention, activation; GEMMs on cuBLAS; one CUDA graph "
                    "per step; seeded synthetic weights"}


def cpu_decode_rate(act: str, steps: int = 3, batch: int = 16) -> dict:
    """The reference streaming op sequence (oracle ops, numpy f32 GEMMs rounded
    to bf16) at config 3, mean time per step over the first steps after one
    warm-up step."""
    import numpy as np
    import torch

    import mimi_chain as mc
    import mimi_oracle
    import xn_oracle

    cfg = mc.MimiChainConfig(**DECODE_CFG)
    w = {k: mimi_oracle.to_storage(v.float().numpy(), "bf16")
         for k, v in mc.synthetic_weights(cfg, torch.float32, "cpu", seed=9).items() if k.startswith("layers.")}
    cos, sin = (mimi_oracle.to_storage(t.float().numpy(), "bf16") for t in mc.rope_tables(cfg, torch.float32, "cpu"))
    r = np.random.default_rng(10)
    xs = [mimi_oracle.to_storage(r.standard_normal((batch, 1, cfg.d_model), dtype=np.float32), "bf16")
          for _ in range(steps + 1)]
    with _oracle_threads(xn_oracle, 1):
        t0 = time.perf_counter()
        mimi_oracle.stream_ref(xn_oracle, cfg, w, cos, sin, xs[:1], "bf16", 0.125, 256, act=act)
        t1 = time.perf_counter()
        mimi_oracle.stream_ref(xn_oracle, cfg, w, cos, sin, xs, "bf16", 0.125, 256, act=act)
        t2 = time.perf_counter()
    us = ((t2 - t1) - (t1 - t0)) / steps * 1e6
    return {"us_per_step": round(us, 1), "frames_per_s": round(batch / (us * 1e-6), 1),
            "sample": f"steps 2..{steps + 1} of a stream at batch {batch}, bf16, oracle ops single-threaded + "
                      f"numpy f32 GEMMs on {os.cpu_count()} BLAS threads"}


# ---------------------------------------------------------------------------
# Bandwidth sweep (benchmark config 5): each op over row widths and row counts,
# f32 and bf16, L2 flushed before every timed launch. Points whose tensors
# exceed the memory cap are skipped (listed with the reason).
# ---------------------------------------------------------------------------
SWEEP_OPS = ["rms_norm_residual", "layer_norm", "rope", "swiglu", "softmax", "embedding_gather"]
# Further ops the sweep can run (--sweep-ops), outside benchmark config 5's list.
SWEEP_EXTRA_OPS = ["silu", "gelu_erf", "residual_add", "softmax_causal", "causal_mask", "rvq_decode", "copy"]
RVQ_BINS, RVQ_BOOKS = 2048, 8


def sweep(torch, xn, device, widths, rows_list, dtypes, reps: int, mem_cap_gb: float, ops=SWEEP_OPS,
          world: int = 1, rank: int = 0) -> list[dict]:
    """Each point: `rows` x `cols` of one op. With world > 1 (torchrun), the
    rows are sharded across the ranks (xn_shard_rows; causal ops by whole
    1024-query slices), every rank times its shard after a barrier, and a
    point's time is the max over ranks of each launch (strong scaling: the
    GB/s are the whole point's bytes over that time)."""
    import torch.distributed as dist

    flush = l2_flusher(torch, device)
    out = []
    for dname in dtypes:
        dt = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[dname]
        s = 4 if dname == "f32" else 2
        for op in ops:
            for cols in widths:
                for rows in rows_list:
                    n_tensors = {"rms_norm_residual": 4, "layer_norm": 2, "rope": 2, "swiglu": 3, "softmax": 2,
                                 "embedding_gather": 1, "silu": 2, "gelu_erf": 2, "residual_add": 3,
                                 "softmax_causal": 2, "causal_mask": 1, "rvq_decode": 1, "copy": 2}[op]
                    point = {"op": op, "dtype": dname, "rows": rows, "cols": cols, "n_gpus": world}
                    # Causal ops: prefill-shaped scores, slices of t1 = 1024 queries over `cols`
                    # keys, the last query seeing every key (offset = cols - t1).
                    t1 = min(1024, rows)
                    unit = t1 if op in ("softmax_causal", "causal_mask") else 1
                    if rows % unit:
                        point["skipped"] = "rows must be a multiple of the 1024-query slice"
                        out.append(point)
                        continue
                    _, cnt = xn.shard_rows(rows // unit, world, rank)
                    lrows = cnt * unit  # this rank's rows
                    need = n_tensors * lrows * cols * s + (32768 * cols * s if op == "embedding_gather" else 0) + \
                        (RVQ_BOOKS * (RVQ_BINS * cols * s + lrows * 8) if op == "rvq_decode" else 0)
                    if need > mem_cap_gb * 1e9:
                        point["skipped"] = f"needs {need / 1e9:.1f} GB > cap {mem_cap_gb} GB"
                        out.append(point)
                        continue
                    if op == "rope" and cols % 128:
                        point["skipped"] = "rope needs width = heads x 128"
                        out.append(point)
                        continue
                    g = torch.Generator(device=device)
                    g.manual_seed(rows + cols + rank)

                    def rnd(*shape):
                        t = torch.empty(shape, dtype=torch.float32, device=device)
                        t.normal_(generator=g)
                        return t.to(dt)

                    w = rnd(cols) * 0.02 + 1
                    extra = {}
                    if op == "rms_norm_residual":
                        x, br, y, h = rnd(lrows, cols), rnd(lrows, cols), torch.empty(lrows, cols, dtype=dt, device=device), \
                            torch.empty(lrows, cols, dtype=dt, device=device)
                        fn = lambda: xn.rms_norm_(y, x, w, 1e-5, branch=br, residual_out=h)  # noqa: E731
                        nbytes = 4 * rows * cols * s + cols * s
                    elif op == "layer_norm":
                        x, y, b = rnd(lrows, cols), torch.empty(lrows, cols, dtype=dt, device=device), rnd(cols)
                        fn = lambda: xn.layer_norm_(y, x, w, b, 1e-5)  # noqa: E731
                        nbytes = 2 * rows * cols * s + 2 * cols * s
                    elif op == "rope":
                        heads, d = cols // 128, 128
                        x, y = rnd(1, lrows, heads, d), torch.empty(1, lrows, heads, d, dtype=dt, device=device)
                        cos, sin = rnd(lrows, d // 2), rnd(lrows, d // 2)
                        fn = lambda: xn.rope_(y, x, cos, sin, 0, layout="bthd")  # noqa: E731
                        nbytes = 2 * rows * cols * s + 2 * rows * (d // 2) * s
                    elif op == "swiglu":
                        a, b2, y = rnd(lrows, cols), rnd(lrows, cols), torch.empty(lrows, cols, dtype=dt, device=device)
                        fn = lambda: xn.swiglu_(y, a, b2)  # noqa: E731
                        nbytes = 3 * rows * cols * s
                    elif op == "softmax":
                        x, y = rnd(lrows, cols), torch.empty(lrows, cols, dtype=dt, device=device)
                        fn = lambda: xn.softmax_(y, x)  # noqa: E731
                        nbytes = 2 * rows * cols * s
                    elif op == "copy":
                        # Not a library op: torch's device copy of the same bytes, the
                        # reference for what a launch of this size reaches at all.
                        x, y = rnd(lrows, cols), torch.empty(lrows, cols, dtype=dt, device=device)
                        fn = lambda: y.copy_(x)  # noqa: E731
                        nbytes = 2 * rows * cols * s
                    elif op in ("silu", "gelu_erf"):
                        x, y = rnd(lrows, cols), torch.empty(lrows, cols, dtype=dt, device=device)
                        fn = lambda: xn.unary_(y, x, op)  # noqa: E731
                        nbytes = 2 * rows * cols * s
                    elif op == "residual_add":
                        x, br, y = rnd(lrows, cols), rnd(lrows, cols), torch.empty(lrows, cols, dtype=dt, device=device)
                        ls = (rnd(cols).abs() * 0.05).to(dt)
                        fn = lambda: xn.residual_add_(y, x, br, ls)  # noqa: E731
                        nbytes = 3 * rows * cols * s + cols * s
                    elif op in ("softmax_causal", "causal_mask"):
                        offset = max(cols - t1, 0)
                        live = sum(min(offset + i + 1, cols) for i in range(t1)) * (rows // t1)
                        x = rnd(lrows // t1, t1, cols)
                        if op == "softmax_causal":
                            y = torch.empty_like(x)
                            fn = lambda: xn.softmax_causal_(y, x, offset)  # noqa: E731
                            nbytes = (live + rows * cols) * s  # unmasked reads, every element written
                        else:
                            fn = lambda: xn.apply_causality_mask_(x, offset)  # noqa: E731
                            nbytes = (rows * cols - live) * s  # the masked elements, written
                    elif op == "rvq_decode":
                        books = [rnd(RVQ_BINS, cols) for _ in range(RVQ_BOOKS)]
                        codes = torch.randint(0, RVQ_BINS, (1, RVQ_BOOKS, lrows), dtype=torch.int64, device=device,
                                              generator=g)
                        y = torch.empty(1, lrows, cols, dtype=dt, device=device)
                        fn = lambda: xn.rvq_decode_sum(books, codes, out_layout="btd", out=y)  # noqa: E731
                        # Compulsory bytes: the codes, each codebook once (per GPU) and the output.
                        # The rows gathered (8 per frame) mostly come from L2 while the codebooks fit
                        # there; their count is reported beside it.
                        nbytes = rows * (RVQ_BOOKS * 8 + cols * s) + world * RVQ_BOOKS * RVQ_BINS * cols * s
                        extra["gathered_bytes"] = rows * (RVQ_BOOKS * 8 + RVQ_BOOKS * cols * s + cols * s)
                    else:
                        table = rnd(32768, cols)
                        ids = torch.randint(0, 32768, (lrows,), dtype=torch.int32, device=device, generator=g)
                        y = torch.empty(lrows, cols, dtype=dt, device=device)
                        fn = lambda: xn.index_select(table, ids, 0, out=y)  # noqa: E731
                        nbytes = rows * 4 + 2 * rows * cols * s
                    fn()
                    times = []
                    for _ in range(reps):
                        flush()
                        if world > 1:
                            dist.barrier()
                        # Keep the GPU busy (a fixed ~0.5 ms spin) while the host enqueues the
                        # start event, the op and the stop event, so host launch latency never
                        # shows up between the two events of a short launch.
                        torch.cuda._sleep(1_000_000)
                        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        e0.record()
                        fn()
                        e1.record()
                        torch.cuda.synchronize()
                        times.append(e0.elapsed_time(e1))
                    if world > 1:
                        tt = torch.tensor(times, dtype=torch.float64, device=device)
                        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
                        times = tt.tolist()
                    ms = statistics.median(times)
                    point.update(ms=round(ms, 5), gbs=round(nbytes / (ms * 1e-3) / 1e9, 1))
                    for k, v in extra.items():
                        point[k.replace("_bytes", "_gbs")] = round(v / (ms * 1e-3) / 1e9, 1)
                    out.append(point)
                    del fn
                    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------
# CPU side: the oracle restatement of the reference CPU backend on a sample.
# ---------------------------------------------------------------------------
class CpuSample:
    """The same five ops on `rows` token rows (and 1 batch element of Q/K
    restricted to rows // heads... see __init__), run by the oracle."""

    def __init__(self, cfg: dict, rows: int, seed: int = 0):
        import numpy as np

        import xn_oracle as oracle

        self.o, self.np = oracle, np
        r = np.random.default_rng(seed)
        H, I, D = cfg["hidden"], cfg["inter"], cfg["head_dim"]
        self.cfg, self.rows = cfg, rows

        def bf(shape, std=1.0, mean=0.0):
            a = (r.standard_normal(shape, dtype=np.float32) * np.float32(std) + np.float32(mean))
            u = a.view(np.uint32)
            return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)

        # The embedding table sample keeps the full vocabulary row count small
        # enough for host memory: ids index a 16384-row slice.
        self.vocab = min(cfg["vocab"], 16384)
        self.table = bf((self.vocab, H), 0.02)
        self.ids = r.integers(0, self.vocab, size=rows).astype(np.uint32)
        self.alpha1, self.alpha2 = bf(H, 0.02, 1.0), bf(H, 0.02, 1.0)
        self.attn_out = bf((rows, H))
        # RoPE sample: the same number of (head, position) rows per token row
        # as the full workload: t positions of all heads of one batch element.
        self.t = max(1, rows)
        self.q = bf((1, cfg["heads_q"], min(self.t, cfg["seq"]), D))
        self.k = bf((1, cfg["heads_kv"], min(self.t, cfg["seq"]), D))
        self.cos, self.sin = oracle.rope_tables(D, cfg["seq"], cfg["theta"], "bf16", "llama")
        self.gate, self.up = bf((rows, I)), bf((rows, I))
        qk_rows_el = (self.q.size + self.k.size)
        self.bytes = {
            "embedding_gather": rows * 4 + 2 * rows * H * 2,
            "rms_norm": 2 * rows * H * 2 + H * 2,
            "rope_qk": 2 * qk_rows_el * 2 + 2 * self.q.shape[2] * (D // 2) * 2,
            "rms_norm_residual": 4 * rows * H * 2 + H * 2,
            "swiglu": 3 * rows * I * 2,
        }

    def step(self):
        o, eps = self.o, self.cfg["eps"]
        x = o.index_select(self.table, self.ids, 0)
        o.rms_norm(x, self.alpha1, eps, "bf16")
        o.rope(self.q, self.cos, self.sin, 0, "bf16")
        o.rope(self.k, self.cos, self.sin, 0, "bf16")
        o.rms_norm_residual(x, self.attn_out, self.alpha2, eps, "bf16")
        o.swiglu(self.gate, self.up, "bf16")

    def total_bytes(self) -> int:
        return sum(self.bytes.values())


def cpu_mimi_rate(batch: int = 1, frames: int = 250) -> dict:
    """The reference op sequence of the Mimi decoder chain on the CPU oracle
    (numpy f32 GEMMs rounded to bf16), one decode timed after a warm-up."""
    import numpy as np
    import torch

    import mimi_chain as mc
    import mimi_oracle
    import xn_oracle

    cfg = mc.MimiChainConfig()
    w = {k: mimi_oracle.to_storage(v.float().numpy(), "bf16")
         for k, v in mc.synthetic_weights(cfg, torch.float32, "cpu", seed=7).items()}
    cos, sin = (mimi_oracle.to_storage(t.float().numpy(), "bf16") for t in mc.rope_tables(cfg, torch.float32, "cpu"))
    codes = np.random.default_rng(8).integers(0, cfg.bins, size=(batch, cfg.n_q, frames), dtype=np.int64)
    scale = 0.125
    with _oracle_threads(xn_oracle, 1):
        mimi_oracle.chain_ref(xn_oracle, cfg, w, cos, sin, codes[:, :, :8], "bf16", scale)
        t0 = time.perf_counter()
        mimi_oracle.chain_ref(xn_oracle, cfg, w, cos, sin, codes, "bf16", scale)
        dt = time.perf_counter() - t0
    return {"frames_per_s": round(batch * frames / dt, 1),
            "sample": f"{batch} x {frames} frames, bf16, oracle ops single-threaded + numpy f32 GEMMs on "
                      f"{os.cpu_count()} BLAS threads (faster than OpenMP oracle ops beside the BLAS threads)"}


class _oracle_threads:
    """Temporarily sets the oracle's OpenMP thread count."""

    def __init__(self, oracle, n: int):
        self.oracle, self.n = oracle, n

    def __enter__(self):
        self.saved = self.oracle.get_num_threads()
        self.oracle.set_num_threads(self.n)

    def __exit__(self, *exc):
        self.oracle.set_num_threads(self.saved)


def cpu_rate(rows: int, steps: int, warmup: int) -> dict:
    import xn_oracle

    xn_oracle.build()
    threads = os.cpu_count() or 1
    xn_oracle.set_num_threads(threads)
    s = CpuSample(CFG, rows)
    for _ in range(warmup):
        s.step()
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        s.step()
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {"value": s.total_bytes() / med / 1e9, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{rows} of 32768 token rows per step (ids into a {s.vocab}-row table slice; Q/K: 1 batch "
                      f"element x {s.q.shape[2]} positions); median of {steps} steps; row-parallel ops use "
                      f"{threads} OpenMP threads, unary/binary ops are single-threaded as in the reference "
                      f"(cpu_backend.rs:1088-1106)",
            "ms_per_step": med * 1e3}


# ---------------------------------------------------------------------------
def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    rows = args.cpu_rows
    r = cpu_rate(rows, args.steps, args.warmup)
    line = {"impl": "reference", "metric": METRIC, "value": r["value"], "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.02) table, N(1,0.02) gains, uniform ids)",
            "config": config_block(args.gpus),
            "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": r["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def config_block(n: int, cfg: dict = CFG, ops=OPS) -> dict:
    return {"workload": "llama3-8b-shaped prefill layer ops (benchmark config 4): " + ", ".join(ops),
            "batch_per_gpu": cfg["batch"], "seq_len": cfg["seq"], "hidden": cfg["hidden"],
            "heads": "32q/8kv x 128", "intermediate": cfg["inter"], "vocab": cfg["vocab"],
            "rows_per_gpu": cfg["batch"] * cfg["seq"], "global_batch": cfg["batch"] * n,
            "parallelism": f"row-sharded x{n}, no collective", "l2": "inputs larger than L2 (126 MB), no flush"}


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["xn", "reference"], default="xn")
    ap.add_argument("--cpu-rows", type=int, default=1024, help="token rows in the CPU sample step")
    ap.add_argument("--e2e-steps", type=int, default=5, help="0 skips the end-to-end measurement")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--decode-steps", type=int, default=256,
                    help="streaming-decode stream length (benchmark config 3); 0 skips it")
    ap.add_argument("--decode-only", action="store_true",
                    help="run only the config-3 streaming-decode measurement")
    ap.add_argument("--decode-acts", default="silu,gelu_erf", help="MLP activations for --decode-only")
    ap.add_argument("--mimi-stream-only", action="store_true",
                    help="run only the Mimi streaming-decode measurement (--mimi-stream-steps frames)")
    ap.add_argument("--gather-context", action="store_true",
                    help="time the config-4 gather after dirty-L2 and clean-L2 predecessors")
    ap.add_argument("--rows", type=int, default=CFG["batch"] * CFG["seq"],
                    help="token rows per GPU (a multiple of 4096; smaller values for profiling captures)")
    ap.add_argument("--ops", default=",".join(OPS), help="comma-separated subset of " + ",".join(OPS))
    ap.add_argument("--mimi-steps", type=int, default=20, help="Mimi decode replays to time (0 skips it)")
    ap.add_argument("--mimi-stream-steps", type=int, default=300,
                    help="frames of the Mimi streaming decode to time (0 skips it)")
    ap.add_argument("--config1-reps", type=int, default=20,
                    help="flushed launches per op of the config-1 f32 micro-pipeline (0 skips it)")
    ap.add_argument("--sweep", action="store_true", help="run the per-op bandwidth sweep instead (JSON per point)")
    # Benchmark config 5's grid: power-of-two widths 256-16384 x rows 1K-1M.
    ap.add_argument("--sweep-widths", default="256,512,1024,2048,4096,8192,16384")
    ap.add_argument("--sweep-rows", default="1024,4096,16384,65536,262144,1048576")
    ap.add_argument("--sweep-dtypes", default="f32,bf16", help="comma-separated subset of f32, bf16, f16")
    ap.add_argument("--sweep-mem-gb", type=float, default=48.0)
    ap.add_argument("--sweep-ops", default=",".join(SWEEP_OPS),
                    help="comma-separated subset of " + ",".join(SWEEP_OPS + SWEEP_EXTRA_OPS))
    args = ap.parse_args()

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return 0

    import torch
    import torch.distributed as dist

    import xn_fused as xn

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if args.sweep:
        sweep_ops = [o for o in args.sweep_ops.split(",") if o]
        unknown = [o for o in sweep_ops if o not in SWEEP_OPS + SWEEP_EXTRA_OPS]
        if unknown:
            ap.error(f"--sweep-ops: unknown op(s) {unknown}")
        xn.lib()
        if world > 1:
            from datetime import timedelta

            dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
        peak, _ = measured_peak()
        pts = sweep(torch, xn, dev, [int(v) for v in args.sweep_widths.split(",")],
                    [int(v) for v in args.sweep_rows.split(",")], args.sweep_dtypes.split(","), max(3, args.steps),
                    args.sweep_mem_gb, sweep_ops, world=world, rank=rank)
        for pt in pts:
            if "gbs" in pt:
                pt["frac"] = round(pt["gbs"] / peak, 3)  # of one GPU's peak
                pt["frac_per_gpu"] = round(pt["gbs"] / world / peak, 3)
            if rank == 0:
                print(json.dumps(pt), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return 0
    if args.gather_context:
        xn.lib()
        for pt in gather_context(torch, xn, dev):
            print(json.dumps({"op": "embedding_gather", **pt}), flush=True)
        return 0
    if args.mimi_stream_only:
        xn.lib()
        print(json.dumps({"mimi_stream_decode": mimi_stream_rate(torch, dev, args.mimi_stream_steps)}), flush=True)
        return 0
    if args.decode_only:
        xn.lib()
        acts = [a for a in args.decode_acts.split(",") if a]
        print(json.dumps({"streaming_decode": {a: decode_rate(torch, dev, args.decode_steps, a) for a in acts}}),
              flush=True)
        return 0
    distributed = world > 1
    if distributed:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    xn.lib()
    ops = [o for o in args.ops.split(",") if o]
    for o in ops:
        if o not in OPS:
            raise SystemExit(f"unknown op {o}")
    if args.rows <= 0 or args.rows % CFG["seq"]:
        raise SystemExit(f"--rows must be a positive multiple of {CFG['seq']}")
    cfg = dict(CFG, batch=args.rows // CFG["seq"])
    wl = LlamaPrefillOps(torch, xn, dev, cfg, seed=1234 + rank, ops=ops)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()

    for _ in range(max(3, args.warmup)):
        wl.step()
    torch.cuda.synchronize()

    events = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in ops]
              for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
        uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
    except Exception:
        pass
    sampler = ClockSampler(uuid)
    sampler.start()
    time.sleep(0.3)
    if distributed:
        dist.barrier()
    torch.cuda.synchronize()
    start.record(stream)
    for k in range(args.steps):
        wl.step(events[k])
    stop.record(stream)
    torch.cuda.synchronize()
    if distributed:
        dist.barrier()
    clocks = sampler.stop()
    elapsed_ms = start.elapsed_time(stop)
    per_op_ms = {name: statistics.mean(events[k][i][0].elapsed_time(events[k][i][1]) for k in range(args.steps))
                 for i, name in enumerate(ops)}

    # End-to-end with host buffers (timed on the compute stream, which waits
    # for the last D2H copy of each step).
    e2e_ms = xfer_ms = float("nan")
    if args.e2e_steps > 0:
        wl.host_buffers()
        torch.cuda.synchronize()
        for _ in range(2):
            wl.e2e_step()
        torch.cuda.synchronize()
        if distributed:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.e2e_steps):
            wl.e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1) / args.e2e_steps
        # The same transfers without kernels: the PCIe bound the e2e step is measured against.
        wl.transfer_step()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.e2e_steps):
            wl.transfer_step()
        e1.record(stream)
        torch.cuda.synchronize()
        xfer_ms = e0.elapsed_time(e1) / args.e2e_steps

    # The optional output all-gather (not on the data path): the residual-RMSNorm
    # output of every rank gathered into the full tensor on every rank, timed
    # separately through the public API (NCCL over NVLink).
    gather_ms = float("nan")
    if distributed and hasattr(wl, "y2"):
        for _ in range(3):
            xn.all_gather_rows(wl.y2, wl.rows * world)
        torch.cuda.synchronize()
        dist.barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for _ in range(5):
            xn.all_gather_rows(wl.y2, wl.rows * world)
        g1.record(stream)
        torch.cuda.synchronize()
        gather_ms = g0.elapsed_time(g1) / 5

    # The same NCCL all-gather on preallocated buffers with nothing else
    # running: the library's own bound for the optional gather.
    raw_gather_ms = float("nan")
    if distributed and hasattr(wl, "y2"):
        src = wl.y2.contiguous()
        full = torch.empty((src.shape[0] * world, *src.shape[1:]), dtype=src.dtype, device=dev)
        for _ in range(3):
            dist.all_gather_into_tensor(full, src)
        torch.cuda.synchronize()
        dist.barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for _ in range(5):
            dist.all_gather_into_tensor(full, src)
        g1.record(stream)
        torch.cuda.synchronize()
        raw_gather_ms = g0.elapsed_time(g1) / 5
        del full

    mimi = None
    if args.mimi_steps > 0:
        mimi = mimi_rate(torch, dev, args.mimi_steps)
    mimi_stream = None
    if args.mimi_stream_steps > 0:
        mimi_stream = mimi_stream_rate(torch, dev, args.mimi_stream_steps)
    decode = None
    if args.decode_steps > 0:
        decode = {act: decode_rate(torch, dev, args.decode_steps, act) for act in ("silu", "gelu_erf")}
    config1 = None
    if args.config1_reps > 0:
        config1 = config1_rate(torch, xn, dev, args.config1_reps)

    if distributed:
        vals = [elapsed_ms, e2e_ms, mimi["ms_per_decode"] if mimi else 0.0, gather_ms if gather_ms == gather_ms else 0.0,
                raw_gather_ms if raw_gather_ms == raw_gather_ms else 0.0,
                mimi_stream["us_per_step"] if mimi_stream else 0.0, mimi_stream["e2e_us_per_step"] if mimi_stream else 0.0,
                config1["pipeline_us"] if config1 else 0.0,
                mimi["e2e_frames_per_s"] if mimi else 0.0]
        t = torch.tensor(vals, dtype=torch.float64, device=dev)
        dist.all_reduce(t[:8], op=dist.ReduceOp.MAX)
        dist.all_reduce(t[8:], op=dist.ReduceOp.MIN)
        elapsed_ms, e2e_ms = float(t[0]), float(t[1])
        if gather_ms == gather_ms:
            gather_ms = float(t[3])
        if raw_gather_ms == raw_gather_ms:
            raw_gather_ms = float(t[4])
        if mimi_stream:
            # Whole job: every rank streams its own batch; the slowest rank sets the step time.
            b = mimi_stream["batch"]
            mimi_stream["us_per_step"], mimi_stream["e2e_us_per_step"] = round(float(t[5]), 2), round(float(t[6]), 2)
            mimi_stream["frames_per_s"] = round(world * b / (float(t[5]) * 1e-6), 1)
            mimi_stream["e2e_frames_per_s"] = round(world * b / (float(t[6]) * 1e-6), 1)
            mimi_stream["ranks"] = world
        if config1:
            config1["pipeline_us"] = round(float(t[7]), 2)
            config1["pipeline_gbs"] = round(world * config1["pipeline_bytes"] / (float(t[7]) * 1e-6) / 1e9, 1)
            config1["ranks"] = world
            config1["per_op_note"] = "per_op: rank 0's launches; pipeline: max over ranks, bytes of all ranks"
        if mimi:
            # Whole-job rate: every rank decodes its own batch; the slowest rank sets the time.
            n = mimi["batch"] * mimi["frames"]
            mimi["ms_per_decode"] = round(float(t[2]), 4)
            mimi["frames_per_s"] = round(world * n / (float(t[2]) * 1e-3), 1)
            mimi["e2e_frames_per_s"] = round(world * float(t[8]), 1)

    if rank == 0:
        step_bytes = sum(wl.bytes.values())
        ms_per_step = elapsed_ms / args.steps
        value = world * step_bytes / (ms_per_step * 1e-3) / 1e9
        peak, peak_src = measured_peak()
        dom = max(per_op_ms, key=per_op_ms.get)
        achieved = wl.bytes[dom] / (per_op_ms[dom] * 1e-3) / 1e9
        traffic_all = load_traffic()
        traffic = traffic_all.get(dom)
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.02) table, N(1,0.02) gains, uniform ids)",
            "config": config_block(world, cfg, ops),
            "pct_of_hbm_peak": round(100.0 * value / world / peak, 1),
            "roofline": {"bound": "hbm", "kernel": dom, "kernel_fn": KERNELS[dom], "achieved": round(achieved, 1),
                         "peak": peak,
                         "peak_source": peak_src, "unit": "GB/s", "frac": round(achieved / peak, 3),
                         "traffic": traffic, "algorithmic_bytes": wl.bytes[dom],
                         "dram_gbs": None if traffic is None else round(traffic / (per_op_ms[dom] * 1e-3) / 1e9, 1),
                         "dram_frac": None if traffic is None else round(traffic / (per_op_ms[dom] * 1e-3) / 1e9 / peak, 3)},
            "per_op": {n: {"ms": round(per_op_ms[n], 4), "bytes": wl.bytes[n],
                           "gbs": round(wl.bytes[n] / (per_op_ms[n] * 1e-3) / 1e9, 1),
                           "frac": round(wl.bytes[n] / (per_op_ms[n] * 1e-3) / 1e9 / peak, 3),
                           # DRAM bytes actually moved (ncu, profiles/traffic.json), per launch
                           "dram_bytes": traffic_all.get(n),
                           "dram_frac": None if traffic_all.get(n) is None else
                           round(traffic_all[n] / (per_op_ms[n] * 1e-3) / 1e9 / peak, 3)} for n in ops},
            "step_dram_frac": None if not all(n in traffic_all for n in ops) else
            round(sum(traffic_all[n] for n in ops) / (ms_per_step * 1e-3) / 1e9 / peak, 3),
            "e2e": None if args.e2e_steps <= 0 else {
                "value": round(world * step_bytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": UNIT,
                "h2d_bytes_per_step": wl.h2d_bytes, "d2h_bytes_per_step": wl.d2h_bytes,
                "ms_per_step": round(e2e_ms, 3),
                "transfer_only_ms_per_step": round(xfer_ms, 3),
                "frac_of_transfer_bound": round(xfer_ms / e2e_ms, 3),
                "method": "per-sequence chunks; H2D, kernels and D2H on three streams; the transfer bound is "
                          "the same copies with no kernels"},
            "gpu_launches": len(ops) * args.steps,
            "all_gather": None if gather_ms != gather_ms else {
                "what": "optional output all-gather (xn_fused.all_gather_rows) of the residual-RMSNorm output, "
                        f"[{wl.rows}, {cfg['hidden']}] bf16 per rank, into the full tensor on every rank; NCCL over "
                        "NVLink; not on the data path",
                "bytes_out": wl.rows * world * cfg["hidden"] * 2, "ms": round(gather_ms, 4),
                "algbw_gbs": round(wl.rows * world * cfg["hidden"] * 2 / (gather_ms * 1e-3) / 1e9, 1),
                "busbw_gbs": round(wl.rows * (world - 1) * cfg["hidden"] * 2 / (gather_ms * 1e-3) / 1e9, 1),
                "raw_nccl_ms": None if raw_gather_ms != raw_gather_ms else round(raw_gather_ms, 4),
                "raw_nccl_busbw_gbs": None if raw_gather_ms != raw_gather_ms else
                round(wl.rows * (world - 1) * cfg["hidden"] * 2 / (raw_gather_ms * 1e-3) / 1e9, 1)},
            "mimi_decode": mimi,
            "mimi_stream_decode": mimi_stream,
            "streaming_decode": decode,
            "config1": config1,
            "clocks": clocks,
        }
        if not args.no_cpu_baseline and world == 1:
            cb = cpu_rate(args.cpu_rows, 3, 1)
            line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
            if mimi is not None:
                line["cpu_baseline"]["mimi_decode"] = cpu_mimi_rate()
            if decode is not None:
                line["cpu_baseline"]["streaming_decode"] = {act: cpu_decode_rate(act) for act in decode}
            if mimi_stream is not None:
                line["cpu_baseline"]["mimi_stream_decode"] = cpu_mimi_stream_rate()
            if config1 is not None:
                line["cpu_baseline"]["config1"] = cpu_config1_rate()
        print(json.dumps(line), flush=True)
    if distributed:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
