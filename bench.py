"""bench.py -- decode-path throughput on B200 (driver contract: one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Workloads (the benchmark configs, synthetic seeded inputs of the stated shapes):
  ragged9b  config 5 (default): 9B-shape ragged batch of 64 sequences, sharded by sequence
            over the ranks; at N = 1 the line also carries compact records of configs 1-4
            ("other_configs", skipped with --no-other-configs)
  decode2b  config 4: 2B-shape hybrid decoder, batch 1, greedy decode tokens/s
            (--kv packet keeps the history as the reference's Q4_K/Q6_K packets)
  mlp       config 1: SwiGLU MLP 2048 -> 6144 -> 2048, Q4_K, batch 1
  attention config 2: GQA decode 16q/4kv, head_dim 256, fp16 KV, history --history (default 32768)
  lmhead    config 3: vocabulary readout 151936 x 2048 Q6_K, batch 1, logits + argmax
  gemm      the tensor-core batched product alone (--rows --cols --batch --format)
  mlp_tp    the MLP split over the ranks (tensor parallel; --hidden --middle --batch)
  lmhead_tp config 3's readout split over the ranks (tensor parallel; --batch)
  cache     the decode caches on config 4's model: prefill computed / restored /
            extended, decode with state digests, the reply replayed (one GPU)
At N > 1 (torchrun, one process per GPU, NCCL) every rank runs the same
workload on its own GPU (replicas: the decode of one sequence does not shard),
except ragged9b (sequences sharded) and the *_tp workloads (one job split over
the ranks, strong scaling); the time is the max over ranks and `value` is the
whole-job aggregate.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "ray-tracing-attention_b200"))
sys.path.insert(0, str(ROOT))

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
L2_BYTES = 126 * 2 ** 20


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
    return dict(PEAKS_FALLBACK, source="fallback")


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons during the timed region
    (written to a file by nvidia-smi itself: a pipe would be block-buffered)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"rta_clocks_{os.getpid()}_{gpu_index}.csv"

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50", "-f", str(self.path)],
                                         stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
            time.sleep(0.3)  # let the first sample land before the timed region starts
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            try:
                self.lines = self.path.read_text().splitlines()
                self.path.unlink()
            except OSError:
                self.lines = []

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------ distributed
def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    import torch
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------- workloads
class Workload:
    """One step of the hot path over one batch of synthetic input."""
    name = ""
    metric = ""
    unit = ""
    dtype = ""
    launches_per_step = 0
    dominant = ""

    def step(self, i: int): ...
    def dominant_launch(self, i: int): ...
    def dominant_bytes(self) -> float: ...
    def units_per_step(self) -> float: ...
    def e2e_step(self, i: int): ...
    def e2e_bytes(self): ...
    def config(self) -> dict: ...
    def cpu_baseline(self, budget_s: float) -> dict: ...


def _rotations(footprint: int) -> int:
    return max(1, -(-2 * L2_BYTES // max(footprint, 1)))


class MLPWorkload(Workload):
    name, metric, unit, dtype, dominant = ("mlp", "SwiGLU MLP decode steps/s (Q4_K, 2048-6144-2048)", "steps/s",
                                           "q4k-int8mma-f32acc", "gemv_tiled_kernel<Q4_K> gate+up (SwiGLU)")
    D, F = 2048, 6144
    launches_per_step = 2
    # dram__bytes_read.sum + dram__bytes_write.sum of one gate+up launch, from one
    # ncu capture (profiles/gemv_tiled_q4k_mlp_2048_6144.md)
    traffic = 14.23e6

    def __init__(self, seed=20261110):
        import torch
        from rta_b200 import ops
        self.ops, self.torch = ops, torch
        per = 3 * self.F * self.D // 256 * 144
        self.copies = _rotations(per)
        # weights re-laid once into the tiled GEMV order, as the engine does at load
        tile = lambda w, r, c: ops.tile_weights(12, w, r, c)[1]
        self.w = [[tile(ops.synthetic_blocks(12, self.F, self.D, seed + 3 * c + j), self.F, self.D) for j in range(2)] +
                  [tile(ops.synthetic_blocks(12, self.D, self.F, seed + 3 * c + 2), self.D, self.F)]
                  for c in range(self.copies)]
        self.fmt = ops.TILED[12]
        self.x = ops.synthetic_normal(self.D, seed + 999)
        self.act = torch.empty(1, self.F, device="cuda")
        self.y = torch.empty(1, self.D, device="cuda")
        self.hx = torch.empty(self.D, dtype=torch.float32).pin_memory()
        self.hx.copy_(self.x.cpu())
        self.hy = torch.empty(self.D, dtype=torch.float32).pin_memory()

    def step(self, i):
        w = self.w[i % self.copies]
        self.ops.mlp_swiglu(self.fmt, w[0], w[1], w[2], self.D, self.F, self.x, y=self.y, act=self.act)

    def dominant_launch(self, i):
        w = self.w[i % self.copies]
        self.ops.gemv_swiglu(self.fmt, w[0], w[1], self.F, self.D, self.x, act=self.act)  # gate+up, 2 x 6144x2048

    def dominant_bytes(self):
        return 2 * self.F * self.D // 256 * 144 + self.D * 4 + self.F * 4

    def units_per_step(self):
        return 1.0

    def e2e_step(self, i):
        x = self.x
        x.copy_(self.hx, non_blocking=True)
        self.step(i)
        self.hy.copy_(self.y.view(-1), non_blocking=True)

    def e2e_bytes(self):
        return self.D * 4, self.D * 4

    def algorithmic_bytes_step(self):
        return 3 * self.F * self.D // 256 * 144 + 2 * self.D * 4 + 2 * self.F * 4

    def config(self):
        return {"workload": "config1_swiglu_mlp_b1", "hidden": self.D, "intermediate": self.F, "format": "Q4_K",
                "layout": "tiled (rta_tile_weights, once before timing)", "batch": 1,
                "l2": f"rotating {self.copies} weight copies (> L2 per pass)"}

    def cpu_baseline(self, budget_s):
        from oracle import oracle
        rng = np.random.default_rng(0)
        mats = [oracle.quantize(12, rng.normal(0, 0.02, n).astype(np.float32))
                for n in (self.F * self.D, self.F * self.D, self.D * self.F)]
        x = rng.normal(0, 1, (1, self.D)).astype(np.float32)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < budget_s or n == 0:
            oracle.mlp(12, *mats, self.D, self.F, x)
            n += 1
        dt = time.perf_counter() - t0
        return {"value": n / dt, "unit": self.unit, "cores": oracle.threads(), "kind": "port",
                "sample": f"{n} full config-1 MLP steps (C restatement of resident_math.comp op 2, OpenMP)"}


class GemmWorkload(Workload):
    """The tensor-core batched product alone (rta_gemm_tc): one 9B-shape projection
    (default: the 12288 x 4096 Q4_K gate) at a decode batch, weights in panel order,
    rotating weight copies larger than L2.  Kernel-level measurement for the ragged
    batch (benchmark config 5) projections; not a benchmark config of its own."""
    name, metric, unit, dtype = ("gemm", "tensor-core batched product rows/s (Q4_K/Q6_K panel x fp16 batch)",
                                 "batch-rows/s", "fp16-tcgen05-f32acc")
    launches_per_step = 3  # memset, prep, tcgen05 kernel

    def __init__(self, seed=20261207, batch=64, rows=12288, cols=4096, fmt=12):
        import torch
        from rta_b200 import ops
        self.ops, self.torch = ops, torch
        self.B, self.R, self.K, self.gf = batch, rows, cols, fmt
        self.wbytes = rows * cols // 256 * (144 if fmt == 12 else 210)
        self.copies = _rotations(self.wbytes)
        self.w = []
        for c in range(self.copies):
            code, w = ops.panel_weights(fmt, ops.synthetic_blocks(fmt, rows, cols, seed + c), rows, cols)
            self.w.append(w)
        self.fmt = code
        tile_n = 16 if batch <= 16 else 32 if batch <= 32 else 64
        self.dominant = f"tc_gemm_kernel<{'Q4_K' if fmt == 12 else 'Q6_K'},{tile_n}>"
        self.x = ops.synthetic_normal(batch * cols, seed + 99).reshape(batch, cols)
        self.y = torch.empty(batch, rows, device="cuda")
        self.ws = torch.empty(ops._lib.load().rta_gemm_tc_workspace_bytes(code, batch, cols), dtype=torch.uint8,
                              device="cuda")
        self.hx = torch.empty(batch * cols, dtype=torch.float32).pin_memory()
        self.hx.copy_(self.x.reshape(-1).cpu())
        self.hy = torch.empty(batch * rows, dtype=torch.float32).pin_memory()

    def step(self, i):
        self.ops.gemm_tc(self.fmt, self.w[i % self.copies], self.R, self.K, self.x, y=self.y, workspace=self.ws)

    dominant_launch = step

    def dominant_bytes(self):
        return self.wbytes + self.B * (self.K + self.R) * 4

    def units_per_step(self):
        return float(self.B)

    def e2e_step(self, i):
        self.x.view(-1).copy_(self.hx, non_blocking=True)
        self.step(i)
        self.hy.copy_(self.y.view(-1), non_blocking=True)

    def e2e_bytes(self):
        return self.B * self.K * 4, self.B * self.R * 4

    def algorithmic_bytes_step(self):
        return self.dominant_bytes()

    def config(self):
        return {"workload": f"gemm_{'q4k' if self.gf == 12 else 'q6k'}_{self.R}x{self.K}_b{self.B}", "rows": self.R,
                "cols": self.K, "batch": self.B, "format": "Q4_K" if self.gf == 12 else "Q6_K",
                "layout": "panel (rta_panel_weights, once before timing)",
                "l2": f"rotating {self.copies} weight copies (> L2 per pass)"}

    def cpu_baseline(self, budget_s):
        from oracle import oracle
        rng = np.random.default_rng(0)
        W = oracle.quantize(self.gf, rng.normal(0, 0.02, self.R * self.K).astype(np.float32))
        x = rng.normal(0, 1, (self.B, self.K)).astype(np.float32)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < budget_s or n == 0:
            oracle.gemv(self.gf, W, self.R, self.K, x)
            n += 1
        dt = time.perf_counter() - t0
        return {"value": n * self.B / dt, "unit": self.unit, "cores": oracle.threads(), "kind": "port",
                "sample": f"{n} full products of {self.B} rows (C restatement of resident_math.comp op 2, OpenMP)"}


class LMHeadWorkload(Workload):
    """benchmark config 3: LM head 151936 x 2048 Q6_K, logits + per-row argmax, batch 1 or 64."""
    name, metric, unit, dtype, dominant = ("lmhead", "vocabulary readout tokens/s (151936x2048 Q6_K, logits+argmax)",
                                           "tokens/s", "q6k-int8mma-f32acc", "gemv_tiled_kernel<Q6_K> readout + argmax")
    V, D = 151936, 2048
    # dram read + write of one batch-1 readout launch with logits, from one ncu
    # capture (profiles/gemv_tiled_q6k_readout_151936x2048.md)
    traffic = 255.36e6 + 3.69e6

    def __init__(self, seed=31, batch=1):
        import torch
        from rta_b200 import ops
        self.ops, self.torch = ops, torch
        self.B = batch
        # batches of 16 rows or more run on the tensor cores (rta_gemm_tc, panel layout)
        self.tc = batch >= 16
        raw = ops.synthetic_blocks(14, self.V, self.D, seed)
        if self.tc:
            self.launches_per_step = 3 + (batch + 63) // 64 * 2  # memset, (prep, tcgen05 kernel) per 64 rows, finish
            self.traffic = None
            self.dtype = "q6k-fp16-tcgen05-f32acc"
            self.dominant = f"tc_gemm_kernel<Q6_K,{min(64, batch)}> readout + argmax, {batch} rows"
            self.fmt, self.w = ops.panel_weights(14, raw, self.V, self.D)
            self.ws = torch.empty(ops._lib.load().rta_gemm_tc_workspace_bytes(self.fmt, batch, self.D),
                                  dtype=torch.uint8, device="cuda")
            self.y = torch.empty(batch, self.V, dtype=torch.float32, device="cuda")
        else:
            self.launches_per_step = 2 + (batch + 15) // 16  # memset, readout launches of <= 16 rows, finish
            if batch != 1:
                self.traffic = None
                self.dominant = f"gemv_tiled_kernel<Q6_K> readout + argmax, {batch} rows (launches of <= 16 rows)"
            self.fmt, self.w = ops.tile_weights(14, raw, self.V, self.D)
            self.ws = torch.empty(4096, dtype=torch.uint8, device="cuda")
        del raw
        self.x = ops.synthetic_normal(batch * self.D, seed + 1).reshape(batch, self.D)
        self.hx = torch.empty(batch * self.D, dtype=torch.float32).pin_memory()
        self.hx.copy_(self.x.reshape(-1).cpu())
        self.harg = torch.empty(batch, dtype=torch.int32).pin_memory()

    def step(self, i):
        if self.tc:
            y, ids, best = self.ops.gemm_tc(self.fmt, self.w, self.V, self.D, self.x, y=self.y, argmax=True,
                                            workspace=self.ws)
            self.last = (y, ids, best)
        else:
            self.last = self.ops.readout(self.fmt, self.w, self.V, self.D, self.x, logits=True, workspace=self.ws)

    dominant_launch = step

    def dominant_bytes(self):
        return self.V * self.D // 256 * 210 + self.B * (self.D * 4 + self.V * 4)

    def units_per_step(self):
        return float(self.B)

    def e2e_step(self, i):
        self.x.view(-1).copy_(self.hx, non_blocking=True)
        self.step(i)
        self.harg.copy_(self.last[1].view(-1), non_blocking=True)

    def e2e_bytes(self):
        return self.B * self.D * 4, self.B * 4

    def algorithmic_bytes_step(self):
        return self.dominant_bytes()

    def config(self):
        layout = ("panel (rta_panel_weights, once before timing); tcgen05 tensor cores" if self.tc
                  else "tiled (rta_tile_weights, once before timing)")
        return {"workload": f"config3_lmhead_b{self.B}", "vocab": self.V, "hidden": self.D, "format": "Q6_K",
                "layout": layout, "batch": self.B, "l2": "weights 255 MB > L2"}

    def cpu_baseline(self, budget_s):
        from oracle import oracle
        rng = np.random.default_rng(0)
        W = oracle.quantize(14, rng.normal(0, 0.02, self.V * self.D).astype(np.float32))
        x = rng.normal(0, 1, (self.B, self.D)).astype(np.float32)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < budget_s or n == 0:
            oracle.lmhead(14, W, self.V, self.D, x, want_logits=True)
            n += 1
        dt = time.perf_counter() - t0
        return {"value": n * self.B / dt, "unit": self.unit, "cores": oracle.threads(), "kind": "port",
                "sample": f"{n} full readouts of {self.B} rows (C restatement of resident_math.comp ops 16/17/23, "
                          "OpenMP)"}


class AttentionWorkload(Workload):
    name, metric, unit, dtype, dominant = ("attention", "GQA decode attention steps/s (16q/4kv, d 256, fp16 KV)",
                                           "steps/s", "f16-mma-f32acc", "attention_split_kernel")
    launches_per_step = 2

    def __init__(self, history=32768, seed=5):
        import torch
        from rta_b200 import ops
        self.ops, self.torch = ops, torch
        self.L = history
        kv_bytes = 2 * self.L * 4 * 256 * 2
        self.copies = _rotations(kv_bytes)
        g = torch.Generator(device="cuda").manual_seed(seed)
        self.k = [torch.randn(self.L, 4, 256, device="cuda", generator=g).half() for _ in range(self.copies)]
        self.v = [torch.randn(self.L, 4, 256, device="cuda", generator=g).half() for _ in range(self.copies)]
        self.q = torch.randn(16, 256, device="cuda", generator=g)
        self.splits = ops._lib.load().rta_attention_default_splits(self.L, 4)
        self.ws = ops.attention_workspace(16, 4, 256, self.splits)
        self.hq = torch.empty(16 * 256, dtype=torch.float32).pin_memory()
        self.hq.copy_(self.q.view(-1).cpu())
        self.hout = torch.empty(16 * 256, dtype=torch.float32).pin_memory()

    def step(self, i):
        c = i % self.copies
        self.last = self.ops.attention_decode_f16(self.q, self.k[c], self.v[c], self.L - 1, self.L, 4, 1,
                                                  splits=self.splits, workspace=self.ws, phys=False)

    dominant_launch = step

    def dominant_bytes(self):
        return 2 * self.L * 4 * 256 * 2 + 2 * 16 * 256 * 4

    def units_per_step(self):
        return 1.0

    def e2e_step(self, i):
        self.q.view(-1).copy_(self.hq, non_blocking=True)
        self.step(i)
        self.hout.copy_(self.last[0].view(-1), non_blocking=True)

    def e2e_bytes(self):
        return 16 * 256 * 4, 16 * 256 * 4

    def algorithmic_bytes_step(self):
        return self.dominant_bytes()

    def config(self):
        return {"workload": f"config2_gqa_decode_L{self.L}", "history": self.L, "q_heads": 16, "kv_heads": 4,
                "head_dim": 256, "kv": "fp16", "splits": self.splits,
                "l2": f"rotating {self.copies} KV copies (> L2 per pass)" if self.copies > 1 else "KV > L2"}

    def cpu_baseline(self, budget_s):
        from oracle import oracle
        rng = np.random.default_rng(0)
        L = min(self.L, 8192)
        q = rng.normal(0, 1, (1, 16, 256)).astype(np.float32)
        k = rng.normal(0, 1, (L, 4, 256)).astype(np.float16).astype(np.float32)
        v = rng.normal(0, 1, (L, 4, 256)).astype(np.float16).astype(np.float32)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < budget_s or n == 0:
            oracle.attention(q, k, v, None, L - 1, 0, L, False)
            n += 1
        dt = time.perf_counter() - t0
        return {"value": n / dt * (L / self.L), "unit": self.unit, "cores": oracle.threads(), "kind": "port",
                "sample": f"{n} decode steps at L={L}, scaled to L={self.L} by history length "
                          "(C restatement of the S_t/R_t detector, OpenMP over heads)"}


def decode_workload_name(kv):
    return "config4_2b_hybrid_decode_b1" + ("" if kv == "fp16" else "_packet_history")


class DecodeWorkload(Workload):
    """benchmark config 4: 2B-shape hybrid (24 layers, 3:1 recurrent:full), batch 1,
    prompt 512 random ids, then greedy decode.  A step is one decode token."""
    name, metric, unit, dtype, dominant = ("decode2b", "decode tokens/s (2B-shape hybrid, batch 1)", "tokens/s",
                                           "q4k/q6k-int8mma, f16-kv, f32 state",
                                           "gemv_tiled_kernel<Q4_K,1> -- every Q4_K matrix product of the step: "
                                           "QKV(+gate) / in-projections, o / out projections, gate+up, down")
    def __init__(self, seed=20261201, prompt_len=512, kv="fp16"):
        self.prompt_len = prompt_len
        self.kv = kv
        if kv == "packet":
            self.dtype = "q4k/q6k-int8mma, q4k/q6k-packet-kv (f32 decode), f32 state"
        import torch
        from rta_b200 import assets, ops
        from rta_b200.model import ResidentModel
        self.ops, self.torch, self.assets = ops, torch, assets
        self.spec = assets.spec_2b()
        self.seed = seed
        self.model = ResidentModel.synthetic(self.spec, seed, capacity=2048, history=kv)
        self.prompt = np.random.default_rng(seed).integers(0, self.spec.vocabulary_size, self.prompt_len)
        self.prefill_ms = self.model.prefill(self.prompt)  # 64-position chunks on the tensor cores
        self.launches_per_step = self.model.resources()["kernels_per_decode_step"]

    def decode(self, k):
        ids = self.model.generate(k)
        return self.model.last_gpu_ms, ids

    def step_bytes(self, position):
        """Algorithmic HBM bytes of one decode token at `position` (weights once, the visible
        history -- fp16 K and V, or one 1416-byte packet per position at 4 x 256 --, recurrent state)."""
        lay = self.model.layout
        weights = sum(t.nbytes for t in lay.matrices) + lay.basis[1].nbytes + self.spec.hidden_size * 210 // 256
        per_pos = self.spec.kv_width * 2 * 2 if self.kv == "fp16" else self.spec.kv_width // 256 * (144 + 210)
        kv = len(self.spec.full_layers) * min(position + 1, 2048) * per_pos
        rec = len(self.spec.recurrent_layers) * self.spec.state_heads * 128 * 128 * 4 * 2
        return weights + kv + rec

    def units_per_step(self):
        return 1.0

    def config(self):
        return {"workload": decode_workload_name(self.kv), "layers": self.spec.depth, "pattern": "rec,rec,rec,full",
                "hidden": self.spec.hidden_size, "intermediate": self.spec.middle_size,
                "vocab": self.spec.vocabulary_size, "q_heads": 16, "kv_heads": 4, "head_dim": 256,
                "rotary_dim": self.spec.rotary_dim, "state_heads": self.spec.state_heads,
                "state_key_heads": self.spec.state_key_heads, "formats": "Q4_K matrices, Q6_K embedding + LM head",
                "kv_cache": "fp16" if self.kv == "fp16" else "packets: 4 Q4_K key + 4 Q6_K value blocks, 1416 B",
                "prompt": self.prompt_len, "prefill_ms": getattr(self, "prefill_ms", None),
                "prefill": "64-position chunks (tcgen05 products, per-row attention, sequential recurrent rows)",
                "batch": 1, "tied_embeddings": False,
                "l2": "per-token weight stream 1.1 GB > L2"}

    def cpu_baseline(self, budget_s):
        from oracle import oracle
        from oracle.model import OracleModel
        from rta_b200 import assets
        spec = assets.spec_2b()
        lay = assets.plan(spec, self.seed)
        params, mats, basis = host_payloads(lay, self.seed)
        ref = OracleModel(spec, params, mats, basis, 2048, kv=self.kv)
        t0 = time.perf_counter()
        ref.prefill(np.random.default_rng(self.seed).integers(0, spec.vocabulary_size, 4))
        n = 0
        while time.perf_counter() - t0 < budget_s or n == 0:
            tok, _ = ref.readout()
            ref.forward(tok)
            n += 1
        dt = time.perf_counter() - t0
        return {"value": (n + 4) / dt, "unit": self.unit, "cores": oracle.threads(), "kind": "port",
                "sample": f"4 prompt + {n} greedy tokens of a 2B-shape model (random valid Q4_K/Q6_K blocks, "
                          f"{self.kv} history) through the model oracle (C restatement of the reference shader "
                          "math, OpenMP)"}


class MLPTPWorkload(Workload):
    """The SwiGLU MLP split over the GPUs of one box (tensor parallel, strong
    scaling): gate / up rows and down columns divided among the ranks
    (rta_b200.tensor_parallel.ShardedMLP), the partial products and the residual
    summed on every rank by one peer-memory exchange kernel
    (rta_team_allreduce_f32).  Default shape: benchmark config 1 (2048-6144-2048
    Q4_K, batch 1); --hidden 4096 --middle 12288 --batch 64 is config 5's MLP."""
    name, unit, strong = "mlp_tp", "steps/s", True

    def __init__(self, seed=20261110, batch=1, hidden=2048, middle=6144):
        import torch
        from rta_b200 import ops
        from rta_b200 import tensor_parallel as tp
        self.ops, self.torch, self.tp = ops, torch, tp
        self.B, self.D, self.F = batch, hidden, middle
        self.team = tp.Team(capacity_bytes=batch * hidden * 4)
        world = self.team.world
        self.local_cols = tp.split_units(middle, tp.MIDDLE_UNIT, world)[self.team.rank][1]
        self.local_bytes = 3 * self.local_cols * hidden // 256 * 144
        self.copies = _rotations(self.local_bytes)
        self.mlps = []
        for c in range(self.copies):
            full = [ops.synthetic_blocks(12, middle, hidden, seed + 3 * c + j) for j in range(2)]
            full.append(ops.synthetic_blocks(12, hidden, middle, seed + 3 * c + 2))
            self.mlps.append(tp.ShardedMLP(self.team, 12, *full, hidden, middle, batch))
            del full
        self.tc = self.mlps[0].tc
        self.metric = (f"SwiGLU MLP steps/s, tensor parallel (Q4_K, {hidden}-{middle}-{hidden}, batch {batch})")
        self.dtype = "q4k-fp16-tcgen05-f32acc" if self.tc else "q4k-int8mma-f32acc"
        # ours per step: (prep, tcgen05 kernel) x 2 per 64 rows (gate+up, down) or 2 GEMVs, plus the exchange
        self.launches_per_step = (4 * ((batch + 63) // 64) if self.tc else 2) + 1
        self.dominant = (f"local MLP slice ({self.local_cols} middle rows): "
                         + ("tc_gemm_kernel<Q4_K> gate+up, down" if self.tc else "gemv_tiled_kernel<Q4_K> gate+up, down"))
        self.x = ops.synthetic_normal(batch * hidden, seed + 999).reshape(batch, hidden)
        self.res = ops.synthetic_normal(batch * hidden, seed + 998).reshape(batch, hidden)
        self.y = torch.empty(batch, hidden, device="cuda")
        self.hx = torch.empty(batch * hidden, dtype=torch.float32).pin_memory()
        self.hx.copy_(self.x.reshape(-1).cpu())
        self.hy = torch.empty(batch * hidden, dtype=torch.float32).pin_memory()

    def step(self, i):
        self.mlps[i % self.copies](self.x, residual=self.res, out=self.y)

    def dominant_launch(self, i):
        m = self.mlps[i % self.copies]
        if m.tc:
            self.ops.mlp_tc(m.code, m.wg, m.wu, m.wd, self.D, m.count, self.x, y=m.partial, workspace=m.workspace)
        else:
            self.ops.mlp_swiglu(m.code, m.wg, m.wu, m.wd, self.D, m.count, self.x, y=m.partial, act=m.act)

    def dominant_bytes(self):
        return self.local_bytes + self.B * (2 * self.D + 2 * self.local_cols) * 4

    def units_per_step(self):
        return 1.0

    def e2e_step(self, i):
        self.x.view(-1).copy_(self.hx, non_blocking=True)
        self.step(i)
        self.hy.copy_(self.y.view(-1), non_blocking=True)

    def e2e_bytes(self):
        return self.B * self.D * 4, self.B * self.D * 4

    def config(self):
        return {"workload": f"mlp_tp_{self.D}x{self.F}_b{self.B}", "hidden": self.D, "intermediate": self.F,
                "format": "Q4_K", "batch": self.B, "split": f"{self.local_cols} middle rows on rank {self.team.rank}",
                "layout": ("panel (tensor cores)" if self.tc else "tiled (GEMV)") + ", relaid once before timing",
                "exchange": "rta_team_allreduce_f32: one kernel, NVLink peer stores, rank-order sum",
                "l2": f"rotating {self.copies} weight copies (> L2 per pass)"}

    def cpu_baseline(self, budget_s):
        from oracle import oracle
        rng = np.random.default_rng(0)
        mats = [oracle.quantize(12, rng.normal(0, 0.02, self.F * self.D).astype(np.float32)) for _ in range(3)]
        x = rng.normal(0, 1, (self.B, self.D)).astype(np.float32)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < budget_s or n == 0:
            oracle.mlp(12, *mats, self.D, self.F, x)
            n += 1
        dt = time.perf_counter() - t0
        return {"value": n / dt, "unit": self.unit, "cores": oracle.threads(), "kind": "port",
                "sample": f"{n} whole MLP steps of {self.B} rows, one process (the reference has no split; C "
                          "restatement of resident_math.comp op 2, OpenMP)"}

    def close(self):
        self.team.close()


class LMHeadTPWorkload(Workload):
    """benchmark config 3's readout split over the GPUs of one box (tensor
    parallel, strong scaling): vocabulary rows divided among the ranks
    (rta_b200.tensor_parallel.ShardedReadout), each rank's best row merged by one
    peer-memory exchange kernel (rta_team_argmax).  Argmax only (no logits)."""
    name, unit, strong = "lmhead_tp", "tokens/s", True
    V, D = 151936, 2048

    def __init__(self, seed=31, batch=1):
        import torch
        from rta_b200 import ops
        from rta_b200 import tensor_parallel as tp
        self.ops, self.torch = ops, torch
        self.B = batch
        self.team = tp.Team(capacity_bytes=max(batch * 8, 16))
        raw = ops.synthetic_blocks(14, self.V, self.D, seed)
        self.head = tp.ShardedReadout(self.team, 14, raw, self.V, self.D, batch)
        del raw
        self.tc = self.head.tc
        self.local_rows = self.head.count
        self.metric = f"vocabulary readout tokens/s, tensor parallel (151936x2048 Q6_K, argmax, batch {batch})"
        self.dtype = "q6k-fp16-tcgen05-f32acc" if self.tc else "q6k-int8mma-f32acc"
        self.launches_per_step = ((batch + 63) // 64 * 2 + 1 if self.tc else (batch + 15) // 16 + 1) + 1
        self.dominant = (f"local readout slice ({self.local_rows} rows): "
                         + ("tc_gemm_kernel<Q6_K> + argmax" if self.tc else "gemv_tiled_kernel<Q6_K> + argmax"))
        self.x = ops.synthetic_normal(batch * self.D, seed + 1).reshape(batch, self.D)
        self.hx = torch.empty(batch * self.D, dtype=torch.float32).pin_memory()
        self.hx.copy_(self.x.reshape(-1).cpu())
        self.harg = torch.empty(batch, dtype=torch.int32).pin_memory()

    def step(self, i):
        self.last = self.head(self.x)

    def dominant_launch(self, i):
        self.head.local(self.x)

    def dominant_bytes(self):
        return self.local_rows * self.D // 256 * 210 + self.B * self.D * 4

    def units_per_step(self):
        return float(self.B)

    def e2e_step(self, i):
        self.x.view(-1).copy_(self.hx, non_blocking=True)
        self.step(i)
        self.harg.copy_(self.last[0].view(-1), non_blocking=True)

    def e2e_bytes(self):
        return self.B * self.D * 4, self.B * 4

    def config(self):
        return {"workload": f"lmhead_tp_b{self.B}", "vocab": self.V, "hidden": self.D, "format": "Q6_K",
                "batch": self.B, "split": f"{self.local_rows} vocabulary rows on rank {self.team.rank}",
                "layout": ("panel (tensor cores)" if self.tc else "tiled (GEMV)") + ", relaid once before timing",
                "exchange": "rta_team_argmax: one kernel, NVLink peer stores", "l2": "weights 255 MB > L2"}

    def cpu_baseline(self, budget_s):
        from oracle import oracle
        rng = np.random.default_rng(0)
        W = oracle.quantize(14, rng.normal(0, 0.02, self.V * self.D).astype(np.float32))
        x = rng.normal(0, 1, (self.B, self.D)).astype(np.float32)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < budget_s or n == 0:
            oracle.lmhead(14, W, self.V, self.D, x, want_logits=False)
            n += 1
        dt = time.perf_counter() - t0
        return {"value": n * self.B / dt, "unit": self.unit, "cores": oracle.threads(), "kind": "port",
                "sample": f"{n} whole readouts (argmax) of {self.B} rows, one process (C restatement of "
                          "resident_math.comp ops 16/17, OpenMP)"}

    def close(self):
        self.team.close()


def host_payloads(layout, seed):
    """Host-side payloads of the layout's shapes with random valid packed blocks
    (no GPU kernels involved: the CPU arms time the reference's CPU path only)."""
    from rta_b200 import assets
    return assets.generate_host(layout, seed)


class RaggedBatchWorkload:
    """benchmark config 5: 9B-shape hybrid (32 layers 3:1, D 4096, F 12288), a ragged batch of
    64 sequences with seeded histories U[128, 8192], sharded by sequence over the ranks
    (weights replicated, no collective on the data path).  A step is one decode token
    for every sequence of the job."""
    name, metric, unit, dtype = ("ragged9b", "decode tokens/s (9B-shape hybrid, ragged batch of 64 sequences)",
                                 "tokens/s", "q4k/q6k fp16 tcgen05 (16+ seqs per rank) or int8 mma, f16-kv, f32 state")
    dominant = "vocabulary readout + argmax at the rank batch"
    seed = 20261205


WORKLOADS = {"mlp": MLPWorkload, "lmhead": LMHeadWorkload, "attention": AttentionWorkload,
             "decode2b": DecodeWorkload, "ragged9b": RaggedBatchWorkload, "gemm": GemmWorkload,
             "mlp_tp": MLPTPWorkload, "lmhead_tp": LMHeadTPWorkload}


def ragged_step_bytes(spec, layout, lengths, capacity, tp_world: int = 1, all_sequences: int | None = None):
    """Algorithmic HBM bytes of one ragged-batch step on one rank: weights once
    (with tensor parallelism: the attention / recurrent projections whole, a
    1/tp_world share of the MLP and vocabulary rows), one embedding row per
    sequence it embeds, every visible fp16 K/V position of its sequences, and
    their recurrent state read and written."""
    seqs = len(lengths)
    mlp = sum(t.nbytes for t in layout.matrices if ".ffn_" in t.name)
    other = sum(t.nbytes for t in layout.matrices) - mlp
    weights = other + (mlp + layout.basis[1].nbytes) / tp_world
    emb = (all_sequences or seqs) * spec.hidden_size * 210 // 256
    kv = sum(min(int(n) + 1, capacity) for n in lengths) * len(spec.full_layers) * spec.kv_width * 2 * 2
    rec = seqs * len(spec.recurrent_layers) * spec.state_heads * 128 * 128 * 4 * 2
    return weights + emb + kv + rec


def ragged_uses_hybrid(world: int, shard_sizes, force_tp: bool = False, force_no_tp: bool = False) -> bool:
    """Config 5's multi-GPU mode: sequence sharding while every rank keeps 16 or
    more sequences (all its products on the tensor cores, no exchange: 12215 vs
    11520 tokens/s for the hybrid at N = 2, 14720 vs 13333 at N = 4), the
    tensor-parallel hybrid below that (8 sequences per rank: the hybrid 11489,
    sequence sharding 7401 at N = 8, where sharded ranks fall to the batched GEMV
    over the full weights).  --tp / --no-tp force one or the other; one GPU never
    takes the hybrid."""
    if world <= 1:
        return False
    if force_tp:
        return True
    if force_no_tp:
        return False
    return min(shard_sizes) < 16


def run_ragged(args, world, rank, local):
    """Config 5 on `world` GPUs: every rank decodes its shard of the 64 sequences;
    `value` = 64 tokens per step / the slowest rank's step time (CUDA events around
    K graph replays); `e2e` = K public-API calls of one step each."""
    import torch
    from rta_b200 import assets, ops, sharding
    from rta_b200.model import ResidentModel
    wl = RaggedBatchWorkload
    spec = assets.spec_9b()
    lengths = sharding.config5_histories(wl.seed)
    small = bool(args.layers or args.max_history)  # profiling case: the 9B layer shapes, fewer layers / shorter histories
    if args.layers:
        import dataclasses
        spec = dataclasses.replace(spec, layer_types=spec.layer_types[:args.layers])
    if args.max_history:
        lengths = np.minimum(lengths, args.max_history).astype(lengths.dtype)
    shards = sharding.shard_sequences(lengths, world)
    mine = lengths[shards[rank]]
    capacity = (int(lengths.max()) + 256 + 255) // 256 * 256
    tp = ragged_uses_hybrid(world, [len(sh) for sh in shards], args.tp, args.no_tp)
    team = None
    if tp:
        # hybrid: every rank keeps the residual rows of all 64 sequences (its shard
        # contiguous), runs the attention / recurrent layers of its own shard, and a
        # 1/world slice of every MLP and of the vocabulary readout for all of them
        from rta_b200 import tensor_parallel
        order = np.concatenate([np.asarray(sh, np.int64) for sh in shards])
        starts = np.concatenate([[0], np.cumsum([len(sh) for sh in shards])]).astype(np.uint32)
        team = tensor_parallel.Team(capacity_bytes=len(lengths) * spec.hidden_size * 4)
        model = ResidentModel.synthetic_team(spec, wl.seed, capacity, starts, team, device=local)
        model.seed_history(lengths[order], seed=wl.seed + 1)
    else:
        model = ResidentModel.synthetic(spec, wl.seed, capacity=capacity, device=local, sequences=len(mine))
        model.seed_history(mine, seed=wl.seed + 1)
    torch.cuda.synchronize()
    barrier(world)  # the ranks' step graphs wait for each other (bounded): start them together
    model.generate_batch(args.warmup)
    torch.cuda.synchronize()
    barrier(world)
    with ClockSampler(local) as clk:
        reps, ms_total, t0 = 0, 0.0, time.perf_counter()
        while True:
            model.generate_batch(args.steps)
            ms_total += model.last_gpu_ms
            reps += 1
            if time.perf_counter() - t0 >= args.min_seconds or reps >= 64:
                break
    ms_step = max_over_ranks(ms_total / reps, world) / args.steps
    res = model.resources()
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        model.generate_batch(1)
    e2e_s = max_over_ranks((time.perf_counter() - t0) * 1e3, world) / 1e3 / args.steps
    positions = mine + args.warmup + args.steps * (reps + 1)
    step_bytes = ragged_step_bytes(spec, model.layout, positions, capacity, world if tp else 1,
                                   len(lengths) if tp else None)
    tc = res["tensor_core_matrices"] > 0
    tile = 16 if len(mine) <= 16 else 32 if len(mine) <= 32 else 64
    kernel = (f"tc_gemm_kernel<Q4_K,{tile}> (tcgen05)" if tc else "gemv_tiled_kernel<Q4_K> (batched rows)") + \
        " -- every Q4_K matrix product of the step: QKV(+gate) / in-projections, o / out projections, gate+up, down"
    roof = step_roofline(profile_summary(model), kernel, "tc_gemm" if tc else "gemv_tiled")
    pk = peaks()
    step_gbs = step_bytes / (ms_step / 1e3) / 1e9
    roof.update({"step_algorithmic_bytes_rank": step_bytes, "step_achieved_gbs_rank": step_gbs,
                 "step_frac": step_gbs / pk["hbm_gbs"], "profiled_rank": rank})
    model.close()
    if team is not None:
        team.close()
    torch.cuda.empty_cache()
    total = int(lengths.size)
    line = {
        "metric": wl.metric, "value": total / (ms_step / 1e3), "unit": wl.unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": wl.dtype,
        "data": "synthetic (seeded random init; seeded K/V, recurrent state and residual histories)",
        "config": {"workload": "config5_9b_ragged_batch64" if not small else
                   f"ragged9b_profile_case_{spec.depth}_layers_history_le_{int(lengths.max())}",
                   "layers": spec.depth, "pattern": "rec,rec,rec,full",
                   "hidden": spec.hidden_size, "intermediate": spec.middle_size, "vocab": spec.vocabulary_size,
                   "q_heads": 16, "kv_heads": 4, "head_dim": 256, "state_heads": spec.state_heads,
                   "state_key_heads": spec.state_key_heads, "sequences": total,
                   "history": "U[128, 8192] seeded", "sequences_per_rank": [len(x) for x in shards],
                   "capacity": capacity, "kv_cache": "fp16",
                   "parallelism": (f"hybrid x{world}: attention / recurrent layers sharded by sequence, MLP "
                                   "(gate/up rows, down columns) and vocabulary rows tensor-parallel, peer-memory "
                                   "exchanges after every block" if tp else
                                   f"sequence-sharded x{world}, weights replicated") if world > 1 else "single GPU",
                   "l2": "per-step weight stream 4 GB > L2"},
        "roofline": roof,
        "e2e": {"value": total / e2e_s, "unit": wl.unit,
                "h2d_bytes_per_step": 48 * (len(lengths) if tp else len(mine)),
                "d2h_bytes_per_step": 52 * (len(lengths) if tp else len(mine)),
                "api": "ResidentModel.generate_batch(1) -> rta_model_generate_batch (C-ABI)"},
        "gpu_launches": res["kernels_per_decode_step"] * args.steps,
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle
        oracle.use_all_cores()
        line["cpu_baseline"] = ragged_cpu_baseline(args.cpu_budget)
    if world == 1 and not args.no_other_configs and not small:
        line["other_configs"] = other_configs(args)
    return line


def ragged_cpu_baseline(budget_s, tokens=None):
    """The 9B model oracle on the host cores: one sequence, a 2-token prompt, then
    greedy tokens until the budget is spent (at least one).  The CPU port decodes
    the 64 sequences one after another, so its aggregate rate equals this rate."""
    from oracle import oracle
    from oracle.model import OracleModel
    from rta_b200 import assets
    spec = assets.spec_9b()
    lay = assets.plan(spec, RaggedBatchWorkload.seed)
    params, mats, basis = host_payloads(lay, RaggedBatchWorkload.seed)
    ref = OracleModel(spec, params, mats, basis, 256)
    ref.prefill(np.random.default_rng(3).integers(0, spec.vocabulary_size, 2))
    n, t0 = 0, time.perf_counter()
    while n == 0 or (time.perf_counter() - t0 < budget_s and (tokens is None or n < tokens)):
        ref.forward(ref.readout()[0])
        n += 1
    v = n / (time.perf_counter() - t0)
    return {"value": v, "unit": "tokens/s", "cores": oracle.threads(), "kind": "port",
            "sample": f"{n} greedy tokens of one sequence after a 2-token prompt, 9B-shape model (random valid "
                      "Q4_K/Q6_K blocks), model oracle = C restatement of the reference shader math (OpenMP); "
                      "sequences are decoded one after another on the CPU"}


def run_decode(args, world, rank, local):
    """Decode: `value` = K tokens generated in one public-API call (device-side
    graph replays, GPU time by CUDA events on the engine stream); `e2e` = K calls
    of generate(1) (host round trip per token: control H2D, ids D2H)."""
    import torch
    wl = DecodeWorkload(prompt_len=args.prompt, kv=args.kv)
    wl.decode(args.warmup)                       # warm-up tokens
    torch.cuda.synchronize()
    barrier(world)
    with ClockSampler(local) as clk:
        reps, ms_total, t0 = 0, 0.0, time.perf_counter()
        while True:
            ms, ids = wl.decode(args.steps)
            ms_total += ms
            reps += 1
            if time.perf_counter() - t0 >= args.min_seconds or reps >= 64:
                break
    ms_step = max_over_ranks(ms_total / reps, world) / args.steps
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        wl.model.generate(1)
    e2e_s = (time.perf_counter() - t0) / args.steps
    e2e_s = max_over_ranks(e2e_s * 1e3, world) / 1e3
    pos = wl.model.state()[1]
    roof = step_roofline(profile_summary(wl.model), wl.dominant, "gemv_tiled")
    pk = peaks()
    step_gbs = wl.step_bytes(pos) / (ms_step / 1e3) / 1e9
    roof.update({"step_algorithmic_bytes": wl.step_bytes(pos), "step_achieved_gbs": step_gbs,
                 "step_frac": step_gbs / pk["hbm_gbs"]})
    line = {
        "metric": wl.metric, "value": world / (ms_step / 1e3), "unit": wl.unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic (seeded random init, prompt ids)",
        "config": dict(wl.config(), parallelism=f"replicas x{world}" if world > 1 else "single GPU"),
        "roofline": roof,
        "e2e": {"value": world / e2e_s, "unit": wl.unit, "h2d_bytes_per_step": 48, "d2h_bytes_per_step": 52,
                "api": "ResidentModel.generate(1) -> rta_model_generate (C-ABI)"},
        "gpu_launches": wl.launches_per_step * args.steps,
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle
        oracle.use_all_cores()
        line["cpu_baseline"] = wl.cpu_baseline(args.cpu_budget)
    if hasattr(wl, "close"):
        wl.close()
    return line


# ----------------------------------------------------------------- timing
def time_steps(fn, steps, warmup, world, graph=True, min_seconds=0.0):
    """W warm-up steps, then EXACTLY `steps` steps timed with CUDA events on the
    launching stream between barrier + synchronize, max over ranks.  With
    graph=True the K steps are captured once into a CUDA graph and the timed
    region is one replay (device throughput without host launch overhead);
    graph=False times eager public-API calls.  min_seconds repeats the timed
    region (same K steps each time) and reports the per-replay mean, so the
    clock sampler sees the load."""
    import torch
    torch.cuda.synchronize()
    barrier(world)  # ranks that exchange data start together (their peer waits are bounded)
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    g = None
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(steps):
                fn(warmup + i)
        g.replay()  # untimed: first replay uploads the graph
        torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps, t0 = 0, time.perf_counter()
    start.record()
    while True:
        if g is not None:
            g.replay()
        else:
            for i in range(steps):
                fn(warmup + i)
        reps += 1
        if time.perf_counter() - t0 >= min_seconds:
            break
    stop.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(stop) / reps
    barrier(world)
    return max_over_ranks(ms, world)


# ------------------------------------------------------- step profile roofline
STEP_PRODUCTS = ("qkv", "o_proj", "in_proj", "out_proj", "gate_up", "down")
# One ncu capture of a representative launch of each step's dominant kernel
# (dram__bytes_read.sum + dram__bytes_write.sum against that launch's
# algorithmic bytes; the summaries under profiles/ give the commands).
TRAFFIC = {
    "tc_gemm": {"launch": "tc_gemm_kernel<Q4_K,64> 12288x4096, batch 64", "dram_bytes": 32.10e6,
                "algorithmic_bytes": 32.5e6, "source": "profiles/tc_gemm_q4k_12288x4096_b64.md"},
    "gemv_tiled": {"launch": "gemv_tiled_kernel<Q4_K,1> gate+up 2 x 6144x2048, batch 1", "dram_bytes": 14.23e6,
                   "algorithmic_bytes": 14.2e6, "source": "profiles/gemv_tiled_q4k_mlp_2048_6144.md"},
}


def profile_summary(model, reps: int = 3) -> dict:
    """Per launch-group kind of one decode step (rta_model_profile_step: CUDA events
    between the groups of a graph replay): device ms (median over `reps` steps),
    algorithmic bytes and groups per step."""
    runs = []
    for _ in range(reps):
        agg = {}
        for kind, ms, nbytes in model.profile_step():
            a = agg.setdefault(kind, [0.0, 0.0, 0])
            a[0] += ms
            a[1] += nbytes
            a[2] += 1
        runs.append(agg)
    return {k: {"ms": float(np.median([r[k][0] for r in runs])), "bytes": runs[-1][k][1],
                "launch_groups": runs[-1][k][2]} for k in runs[-1]}


def step_roofline(prof: dict, kernel: str, traffic_key: str) -> dict:
    """Roofline of the step's dominant kernel class -- its matrix products -- from a
    step profile: achieved = their algorithmic bytes / their summed device time;
    share = their time / the profiled step's time.  Every other launch group is
    listed under per_kind with its own bandwidth and share."""
    pk = peaks()
    total = sum(v["ms"] for v in prof.values())
    ms = sum(prof[k]["ms"] for k in STEP_PRODUCTS if k in prof)
    nbytes = sum(prof[k]["bytes"] for k in STEP_PRODUCTS if k in prof)
    groups = sum(prof[k]["launch_groups"] for k in STEP_PRODUCTS if k in prof)
    achieved = nbytes / (ms / 1e3) / 1e9
    per_kind = {}
    for k, v in prof.items():
        gbs = v["bytes"] / (v["ms"] / 1e3) / 1e9 if v["ms"] > 0 else None
        per_kind[k] = {"ms": v["ms"], "algorithmic_bytes": v["bytes"], "launch_groups": v["launch_groups"],
                       "achieved_gbs": gbs, "frac": gbs / pk["hbm_gbs"] if gbs is not None else None,
                       "share": v["ms"] / total if total > 0 else None}
    t = TRAFFIC[traffic_key]
    return {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
            "frac": achieved / pk["hbm_gbs"], "traffic": t["dram_bytes"], "kernel": kernel,
            "share": ms / total if total > 0 else None, "kernel_ms_per_step": ms,
            "algorithmic_bytes_per_step": nbytes, "launch_groups_per_step": groups,
            "traffic_launch": t["launch"], "traffic_launch_algorithmic_bytes": t["algorithmic_bytes"],
            "traffic_source": t["source"],
            "peak_source": f"{pk['source']} hbm_gbs (burst copy)",
            "method": "rta_model_profile_step: one decode step replayed as a graph with a CUDA event after every "
                      "launch group (median of 3 steps); the events remove the overlap of consecutive kernels, "
                      "so each group is timed on its own and the shares are of that serialised step",
            "per_kind": per_kind}


def other_configs(args) -> list:
    """The benchmark's other configurations on this GPU, measured in the same run
    (N = 1 only): config 1 (MLP), config 2 (attention at L = 32768), config 3 (LM
    head at batch 1 and 64) -- each with its dominant kernel timed alone by CUDA
    events and its public-API e2e -- and config 4 (2B decode, 512-token prompt)
    with its step-profile roofline.  A compact record per configuration."""
    import torch
    pk = peaks()
    out = []
    for name, kw in (("mlp", {}), ("attention", {"history": 32768}), ("lmhead", {"batch": 1}),
                     ("lmhead", {"batch": 64})):
        wl = WORKLOADS[name](**kw)
        steps = max(10, args.steps // 2)
        ms = time_steps(wl.step, steps, args.warmup, 1, min_seconds=0.3) / steps
        dom_ms = time_steps(wl.dominant_launch, steps, args.warmup, 1) / steps
        e2e_ms = time_steps(wl.e2e_step, steps, args.warmup, 1, graph=False) / steps
        achieved = wl.dominant_bytes() / (dom_ms / 1e3) / 1e9
        h2d, d2h = wl.e2e_bytes()
        out.append({"config": wl.config(), "metric": wl.metric, "value": wl.units_per_step() / (ms / 1e3),
                    "unit": wl.unit, "ms_per_step": ms,
                    "roofline": {"kernel": wl.dominant, "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                                 "frac": achieved / pk["hbm_gbs"], "kernel_ms": dom_ms,
                                 "algorithmic_bytes": wl.dominant_bytes(), "traffic": getattr(wl, "traffic", None)},
                    "e2e": {"value": wl.units_per_step() / (e2e_ms / 1e3), "unit": wl.unit,
                            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}})
        del wl
        torch.cuda.empty_cache()
    wl = DecodeWorkload(prompt_len=512)
    wl.decode(args.warmup)
    ms_total, reps = 0.0, 0
    for _ in range(3):
        ms, _ = wl.decode(args.steps)
        ms_total += ms
        reps += 1
    ms_step = ms_total / reps / args.steps
    t0 = time.perf_counter()
    for _ in range(args.steps):
        wl.model.generate(1)
    e2e_s = (time.perf_counter() - t0) / args.steps
    roof = step_roofline(profile_summary(wl.model), wl.dominant, "gemv_tiled")
    out.append({"config": wl.config(), "metric": wl.metric, "value": 1e3 / ms_step, "unit": wl.unit,
                "ms_per_step": ms_step, "roofline": roof,
                "e2e": {"value": 1.0 / e2e_s, "unit": wl.unit, "h2d_bytes_per_step": 48, "d2h_bytes_per_step": 52}})
    wl.model.close()
    torch.cuda.empty_cache()
    return out


def run_ours(args, world, rank, local):
    import torch
    kw = {"history": args.history} if args.workload == "attention" else \
        {"batch": args.batch} if args.workload in ("lmhead", "lmhead_tp") else \
        {"batch": args.batch, "hidden": args.hidden, "middle": args.middle} if args.workload == "mlp_tp" else \
        {"batch": args.batch, "rows": args.rows, "cols": args.cols, "fmt": {"q4k": 12, "q6k": 14}[args.format]} \
        if args.workload == "gemm" else {}
    wl = WORKLOADS[args.workload](**kw)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        ms = time_steps(wl.step, args.steps, args.warmup, world, min_seconds=args.min_seconds)
    ms_step = ms / args.steps
    strong = getattr(wl, "strong", False)  # tensor parallel: the job's work is fixed, split over the ranks
    jobs = 1 if strong else world
    value = wl.units_per_step() * jobs / (ms_step / 1e3)
    # dominant kernel alone, CUDA events on the launching (current) stream
    dom_ms = time_steps(wl.dominant_launch, args.steps, args.warmup, world) / args.steps
    pk = peaks()
    achieved = wl.dominant_bytes() / (dom_ms / 1e3) / 1e9
    e2e_ms = time_steps(wl.e2e_step, args.steps, args.warmup, world, graph=False) / args.steps
    h2d, d2h = wl.e2e_bytes()
    line = {
        "metric": wl.metric, "value": value, "unit": wl.unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": wl.dtype,
        "data": "synthetic (seeded, benchmark shapes)",
        "config": dict(wl.config(), parallelism=(f"tensor parallel x{world}" if strong else f"replicas x{world}")
                       if world > 1 else "single GPU"),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / pk["hbm_gbs"], "traffic": getattr(wl, "traffic", None), "kernel": wl.dominant,
                     "algorithmic_bytes": wl.dominant_bytes(), "kernel_ms": dom_ms,
                     "peak_source": f"{pk['source']} hbm_gbs (burst copy)"},
        "e2e": {"value": wl.units_per_step() * jobs / (e2e_ms / 1e3), "unit": wl.unit,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "api": "rta_b200.ops -> librta_cuda.so C-ABI"},
        "gpu_launches": wl.launches_per_step * args.steps,
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle
        oracle.use_all_cores()
        line["cpu_baseline"] = wl.cpu_baseline(args.cpu_budget)
    if hasattr(wl, "close"):
        wl.close()
    return line


def run_reference(args, world, rank):
    """Reference arm: the reference's CPU path for this workload (the oracle port of
    its shader math; the Vulkan path cannot run here), rank 0 only."""
    if rank != 0:
        return None
    if args.workload == "decode2b":
        return run_reference_decode(args, world)
    if args.workload == "ragged9b":
        base = ragged_cpu_baseline(args.cpu_budget, tokens=max(1, args.steps))
        v = base["value"]
        return {"impl": "reference", "metric": RaggedBatchWorkload.metric, "value": v, "unit": "tokens/s",
                "n_gpus": world, "steps": args.steps, "warmup": 0, "higher_is_better": True, "dtype": "f32",
                "data": "synthetic (seeded random init)", "config": {"workload": "config5_9b_ragged_batch64"},
                "cpu_baseline": base, "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                                              "d2h_bytes_per_step": 0},
                "note": "reference Vulkan ray-query worker unavailable on this box (no graphics stack, no RT "
                        "cores); timed its CPU path: the C restatement of its shader math"}
    cls = WORKLOADS[args.workload]
    wl = cls.__new__(cls)
    if args.workload == "attention":
        wl.L = args.history
    if args.workload == "decode2b":
        wl.seed = 20261201
    if args.workload in ("lmhead", "lmhead_tp"):
        wl.B = args.batch
    if args.workload == "mlp_tp":
        wl.B, wl.D, wl.F = args.batch, args.hidden, args.middle
    if args.workload == "gemm":
        wl.B, wl.R, wl.K, wl.gf = args.batch, args.rows, args.cols, {"q4k": 12, "q6k": 14}[args.format]
    budget = max(1.0, args.cpu_budget / max(args.steps, 1))
    vals = []
    for _ in range(args.warmup + args.steps):
        vals.append(wl.cpu_baseline(budget))
    vals = vals[args.warmup:]
    v = float(np.median([b["value"] for b in vals]))
    base = dict(vals[-1], value=v)
    cfg = {"mlp": {"workload": "config1_swiglu_mlp_b1"}, "lmhead": {"workload": f"config3_lmhead_b{args.batch}"},
           "attention": {"workload": f"config2_gqa_decode_L{args.history}"},
           "decode2b": {"workload": "config4_2b_hybrid_decode_b1"},
           "gemm": {"workload": f"gemm_{args.format}_{args.rows}x{args.cols}_b{args.batch}"},
           "mlp_tp": {"workload": f"mlp_tp_{args.hidden}x{args.middle}_b{args.batch}"},
           "lmhead_tp": {"workload": f"lmhead_tp_b{args.batch}"}}[args.workload]
    metric = {"mlp_tp": f"SwiGLU MLP steps/s, tensor parallel (Q4_K, {args.hidden}-{args.middle}-{args.hidden}, "
                        f"batch {args.batch})",
              "lmhead_tp": f"vocabulary readout tokens/s, tensor parallel (151936x2048 Q6_K, argmax, batch "
                           f"{args.batch})"}.get(args.workload, getattr(cls, "metric", ""))
    return {"impl": "reference", "metric": metric, "value": v, "unit": cls.unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "dtype": "f32",
            "data": "synthetic (seeded, benchmark shapes)", "config": cfg,
            "cpu_baseline": base, "e2e": {"value": v, "unit": cls.unit, "h2d_bytes_per_step": 0,
                                          "d2h_bytes_per_step": 0},
            "note": "reference Vulkan ray-query worker unavailable on this box (no graphics stack, no RT cores); "
                    "timed its CPU path: the C restatement of its shader math"}


def run_cache(args):
    """The decode caches (RTA_MODEL_CACHE) on config 4's model: a 512-position
    prompt prefilled and 256 tokens decoded with a state digest after every
    step (the reply tree records them), the same prompt prefilled again (its
    boundary restored: state words and 32 history blocks), the 256 tokens replayed
    from the reply tree, and a prompt that extends the boundary by 64 positions.
    Every figure comes through the public API (ResidentModel -> C-ABI) with host
    buffers; the value is the replayed reply's tokens per second of wall time.
    The uncached handle of the same weights gives the decode rate without digests."""
    from rta_b200 import assets
    from rta_b200.model import ResidentModel
    spec = assets.spec_2b()
    seed, n, k = 20261201, args.prompt, 256
    prompt = np.random.default_rng(seed).integers(0, spec.vocabulary_size, n)
    c = ResidentModel.synthetic(spec, seed, capacity=2048, history=args.kv, cache=True)
    u = ResidentModel.synthetic(spec, seed, capacity=2048, history=args.kv)
    wall = lambda f: (lambda t0: (f(), (time.perf_counter() - t0) * 1e3))(time.perf_counter())
    warm = np.random.default_rng(seed + 2).integers(0, spec.vocabulary_size, 64)  # shares no prefix
    for _ in range(max(1, args.warmup - 2)):  # graphs, allocator pools, the reply tree's nodes
        c.prefill(warm)
        c.generate(8)
    _, miss_ms = wall(lambda: c.prefill(prompt))
    miss = c.cache_info()
    first, _ = wall(lambda: c.generate(k))
    decode_cached_ms = c.last_gpu_ms
    u.prefill(prompt)
    plain = u.generate(k)
    decode_plain_ms = u.last_gpu_ms
    _, hit_ms = wall(lambda: c.prefill(prompt))
    hit = c.cache_info()
    replay, replay_ms = wall(lambda: c.generate(k))
    rep_info = c.cache_info()
    ext = np.concatenate([prompt, np.random.default_rng(seed + 1).integers(0, spec.vocabulary_size, 64)])
    _, ext_ms = wall(lambda: c.prefill(ext))
    ext_info = c.cache_info()
    same = bool(np.array_equal(first, plain) and np.array_equal(replay, first))
    c.close()
    u.close()
    value = len(replay) / (replay_ms / 1e3)
    return {"metric": "reply-tree replay tokens/s (2B shape, 512 prompt + 256 tokens, cache hit)", "value": value,
            "unit": "tokens/s", "n_gpus": 1, "steps": 1, "warmup": args.warmup, "higher_is_better": True,
            "dtype": "u32 (256-bit state keys)", "data": "synthetic (seeded random init, prompt ids)",
            "config": {"workload": "config4_2b_cache_replay", "prompt": n, "tokens": k, "history": args.kv},
            "tokens_identical_to_uncached": same, "replayed_tokens": rep_info["replayed_tokens"],
            "prefill_computed_ms": miss_ms, "prefill_restored_ms": hit_ms,
            "prefill_restored": {"reused": hit["reused_tokens"], "computed": hit["computed_tokens"],
                                 "address_hit": hit["address_hit"], "blocks": hit["shared_blocks"]},
            "prefill_extended_ms": ext_ms,
            "prefill_extended": {"reused": ext_info["reused_tokens"], "computed": ext_info["computed_tokens"]},
            "boundary_bytes": miss["bytes"],
            "decode_tok_s_with_digests": k / (decode_cached_ms / 1e3),
            "decode_tok_s_uncached": k / (decode_plain_ms / 1e3),
            "digest_us_per_token": (decode_cached_ms - decode_plain_ms) / k * 1e3,
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 4 * k}}


def run_reference_decode(args, world):
    """The 2B decode through the model oracle on all host cores: one model build,
    W warm-up tokens, then min(K, 16) timed tokens (a bounded sample)."""
    from oracle import oracle
    from oracle.model import OracleModel
    from rta_b200 import assets
    spec = assets.spec_2b()
    lay = assets.plan(spec, 20261201)
    params, mats, basis = host_payloads(lay, 20261201)
    ref = OracleModel(spec, params, mats, basis, 2048, kv=args.kv)
    ref.prefill(np.random.default_rng(1).integers(0, spec.vocabulary_size, 4))
    for _ in range(min(args.warmup, 3)):
        ref.forward(ref.readout()[0])
    n = max(1, min(args.steps, 16))
    t0 = time.perf_counter()
    for _ in range(n):
        ref.forward(ref.readout()[0])
    v = n / (time.perf_counter() - t0)
    base = {"value": v, "unit": "tokens/s", "cores": oracle.threads(), "kind": "port",
            "sample": f"{n} greedy tokens after a 4-token prompt of a 2B-shape model (random valid Q4_K/Q6_K "
                      f"blocks, {args.kv} history) through the model oracle, the C restatement of the reference "
                      "shader math (OpenMP)"}
    return {"impl": "reference", "metric": DecodeWorkload.metric, "value": v, "unit": "tokens/s", "n_gpus": world,
            "steps": n, "warmup": min(args.warmup, 3), "higher_is_better": True, "dtype": "f32",
            "data": "synthetic (seeded random init, prompt ids)",
            "config": {"workload": decode_workload_name(args.kv)}, "cpu_baseline": base,
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "reference Vulkan ray-query worker unavailable on this box (no graphics stack, no RT cores); "
                    "timed its CPU path: the C restatement of its shader math"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + ["cache"], default="ragged9b")
    ap.add_argument("--history", type=int, default=32768)
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--min-seconds", type=float, default=1.0,
                    help="repeat the timed K-step region for at least this long (clock sampling)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-tp", action="store_true",
                    help="ragged9b at N > 1: shard by sequence only (weights replicated, no exchanges)")
    ap.add_argument("--tp", action="store_true",
                    help="ragged9b at N > 1: the tensor-parallel hybrid whatever the sequences per rank "
                         "(default: the hybrid only below 16 sequences per rank)")
    ap.add_argument("--no-other-configs", action="store_true",
                    help="ragged9b at N=1: skip the compact lines of benchmark configs 1-4")
    ap.add_argument("--batch", type=int, default=1,
                    help="lmhead: hidden rows per readout (config 3: 1 or 64); gemm: batch rows")
    ap.add_argument("--rows", type=int, default=12288, help="gemm: weight rows (multiple of 128)")
    ap.add_argument("--hidden", type=int, default=2048, help="mlp_tp: hidden size (multiple of 256)")
    ap.add_argument("--middle", type=int, default=6144, help="mlp_tp: intermediate size (multiple of 256 x ranks)")
    ap.add_argument("--cols", type=int, default=4096, help="gemm: weight columns (multiple of 256)")
    ap.add_argument("--format", choices=("q4k", "q6k"), default="q4k", help="gemm: weight format")
    ap.add_argument("--layers", type=int, default=0,
                    help="ragged9b: first N layers of the 9B pattern only (profiling case; 0 = all 32)")
    ap.add_argument("--max-history", type=int, default=0,
                    help="ragged9b: cap the seeded histories (profiling case; 0 = config 5's U[128, 8192])")
    ap.add_argument("--kv", choices=("fp16", "packet"), default="fp16",
                    help="decode2b: attention history format (packet: the reference's Q4_K key / Q6_K value "
                         "packets, the worker's default)")
    ap.add_argument("--prompt", type=int, default=512,
                    help="decode2b: prompt length before the timed tokens (short prompts keep profiler runs small)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.workload == "cache":
        if args.impl == "reference":
            line = {"impl": "reference", "unavailable": "the reference's caches live in its Vulkan ray-query worker "
                                                        "(no graphics stack or RT cores on this box)"}
        else:
            line = run_cache(args)
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps(line), flush=True)
        return
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        if rank == 0:
            from oracle import oracle
            oracle.use_all_cores()  # torch.distributed.run sets OMP_NUM_THREADS=1 for every rank
        line = run_reference(args, world, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    world, rank, local = dist_setup(args.gpus)
    if args.workload == "decode2b":
        line = run_decode(args, world, rank, local)
    elif args.workload == "ragged9b":
        line = run_ragged(args, world, rank, local)
    else:
        line = run_ours(args, world, rank, local)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
