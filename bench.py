"""Benchmark of the FP32 operator path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload chain|gemm|layernorm|affine|add|softmax|reduce|attention|block]

Workloads (synthetic seeded inputs with the shapes and distributions of the
benchmark configurations; one "step" is one pass of the path over one batch):
  chain      Y = LayerNorm(X W), X[65536 x 4096] ~ N(0,1), W[4096 x 4096] ~ N(0,1/4096),
             gamma = 1, beta = 0, eps 1e-5, seed 4; rows sharded over the ranks (the
             default: the configuration that drives GEMM TFLOP/s, LayerNorm and scaling)
  gemm       C = A B, M = N = K = 4096, A, B ~ U[-1,1), seed 3; rows sharded
  layernorm  X[16384 x 4096] ~ N(0,1), gamma ~ N(1,.02), beta ~ N(0,.02), seed 2; rows sharded
  affine     y = 1.5 x - 0.25, n = 2^26, x ~ U[-4,4), seed 1 (replica per rank)
  add        c = a + b, n = 2^20, a, b ~ U[-1,1), seed 0 (replica per rank, 16 rotating sets)
  softmax    causal row softmax of x [32, 1024, 1024] ~ U[-8,8), scale 1/8, seed 5 (replica per rank)
  reduce     row sums of x [65536 x 1024] ~ U[-4,4), seed 6 (replica per rank)
  attention  batched Q K^T: Q, K [32 heads, 2048, 128] ~ U[-1,1), seed 7, K^T as a strided view
             (replica per rank)
  block      the reference example's pre-LN encoder block at T = 2048 tokens, d = 1024, 16 heads,
             d_ff = 4096, causal, in 11 commands (bias and GELU fused into the GEMMs; the four
             projection weights prepared once unless --split-w-per-step); value = the block's
             GEMM flops per second (replica per rank)
`value` is device time (CUDA events on the library's context stream between two
queue markers, max over ranks); `e2e` times the same steps through the public API
with pinned host inputs copied in and results copied out every step. Under
torchrun every rank drives cuda:LOCAL_RANK; a gloo process group carries only the
barrier and the max-over-ranks reduction (the path itself has no exchange).
`--impl reference` times the reference's CPU computation of the path (the
oracle's restatement of its verifier, all host threads) on a bounded sample.
"""
import argparse
import json
import math
import os
from pathlib import Path
import subprocess
import sys
import threading
import time

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "FP32 GEMM TFLOP/s; LayerNorm & affine HBM GB/s at 1/2/4/8 B200"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="chain",
                    choices=("chain", "gemm", "layernorm", "affine", "add", "softmax", "reduce", "attention", "block"))
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end leg")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true",
                    help="chain: skip the other benchmark configurations measured beside the headline")
    ap.add_argument("--matmul-mode", default="auto", choices=("auto", "reference", "ffma", "tf32x3"),
                    help="summation mode of the GEMM workloads (default auto: the 3xTF32 tensor-core kernel)")
    ap.add_argument("--split-w-per-step", action="store_true",
                    help="chain and block: split the weights in every step (pr_matmul_f32, "
                         "pr_b200_matmul_bias_activation_f32) instead of preparing them once "
                         "(pr_b200_matmul_prepare_f32) before the timed steps")
    ap.add_argument("--gather", action="store_true",
                    help="chain: also gather Y on every GPU (LayerNorm writes its rows to all ranks over NVLink); "
                         "gemm: gather C on every GPU after the GEMM (peer-store kernel)")
    return ap.parse_args()


# Sized so the timed region lasts about a second (the clock sampler needs several
# 200 ms samples inside it).
DEFAULT_STEPS = {"chain": 100, "gemm": 1500, "layernorm": 8000, "affine": 8000, "add": 20000, "softmax": 20000,
                 "reduce": 20000, "attention": 5000, "block": 1500}
METRICS = {"chain": "FP32 GEMM+LayerNorm chain throughput (GEMM TFLOP/s)",
           "gemm": "FP32 GEMM TFLOP/s (4096^3, rows sharded)",
           "layernorm": "FP32 row LayerNorm HBM GB/s (16384x4096, rows sharded)",
           "affine": "FP32 affine y = 1.5x - 0.25 HBM GB/s (n = 2^26)",
           "add": "FP32 vector add HBM GB/s (n = 2^20)",
           "softmax": "FP32 causal row softmax HBM GB/s ([32, 1024, 1024])",
           "reduce": "FP32 row sum HBM GB/s (65536 x 1024)",
           "attention": "FP32 batched matmul TFLOP/s (32 x 2048x2048x128, Q K^T)",
           "block": "FP32 encoder block GEMM TFLOP/s (T=2048, d=1024, 16 heads, d_ff=4096, causal)"}


# ---------------------------------------------------------------- distributed plumbing
class Group:
    def __init__(self, world):
        self.world = world
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", str(self.rank)))
        self.dist = None
        if world > 1 or (int(os.environ.get("WORLD_SIZE", "1")) > 1 and world != 1):
            import datetime
            import torch.distributed as dist
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=180))
            self.dist = dist
            self.world = dist.get_world_size()
            self.rank = dist.get_rank()

    def barrier(self):
        if self.dist:
            self.dist.barrier()

    def max(self, value):
        if not self.dist:
            return value
        import torch
        t = torch.tensor([float(value)], dtype=torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return t.item()

    def exchange(self, value):
        """Every rank's `value` (host objects over the gloo control plane)."""
        if not self.dist:
            return [value]
        out = [None] * self.world
        self.dist.all_gather_object(out, value)
        return out

    def close(self):
        if self.dist:
            self.dist.barrier()
            self.dist.destroy_process_group()


# ---------------------------------------------------------------- clocks during the timed region
class Clocks:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device, self.lines, self.proc = device, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.device)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            time.sleep(0.4)  # nvidia-smi's first sample arrives before the timed work starts
            self.lines.clear()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *_):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=2)

    def summary(self):
        mhz, max_mhz, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                mhz.append(float(f[1]))
                max_mhz = float(f[2])
            except ValueError:
                continue
            for name, flag in zip(names, f[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not mhz:
            return {"sm_mhz": None, "sm_max_mhz": max_mhz, "reasons": sorted(reasons), "samples": 0}
        mhz.sort()
        return {"sm_mhz": mhz[len(mhz) // 2], "sm_max_mhz": max_mhz, "reasons": sorted(reasons),
                "samples": len(mhz)}


# ---------------------------------------------------------------- workload descriptions (no device needed)
def describe(name, world, rank, gather=False):
    """(metric, unit, scaling, config) of a workload for `rank` of `world`; the same
    dict for both arms, so the two lines name one configuration."""
    from paralyn_b200 import shard
    if name == "chain":
        r0, r1 = shard.row_range(65536, world, rank)
        config = {"workload": "chain: Y = LayerNorm(X W), X[65536x4096] ~ N(0,1), W[4096x4096] ~ N(0,1/4096), "
                              "gamma=1, beta=0, eps=1e-5, seed 4",
                  "rows": 65536, "k": 4096, "n": 4096, "rows_per_gpu": r1 - r0, "parallelism": f"rows{world}",
                  "l2": "inputs larger than L2 (X shard >= 128 MiB)"}
        if gather:
            config["gathered_output"] = "Y gathered on every GPU by the fused LayerNorm (NVLink stores)"
        return METRICS[name], "TFLOP/s", "strong", config
    if name == "gemm":
        r0, r1 = shard.row_range(4096, world, rank)
        config = {"workload": "gemm: C = A B, M=N=K=4096, A,B ~ U[-1,1), seed 3", "m": 4096, "n": 4096, "k": 4096,
                  "rows_per_gpu": r1 - r0, "parallelism": f"rows{world}",
                  "l2": "operands are 64 MiB each; A/B re-reads are part of the GEMM"}
        if gather:
            config["gathered_output"] = "C gathered on every GPU (pr_b200_gather_rows_f32: peer stores over NVLink)"
        return METRICS[name], "TFLOP/s", "strong", config
    if name == "layernorm":
        r0, r1 = shard.row_range(16384, world, rank)
        return METRICS[name], "GB/s", "strong", {
            "workload": "layernorm: X[16384x4096] ~ N(0,1), gamma ~ N(1,.02), beta ~ N(0,.02), eps 1e-5, seed 2",
            "rows_per_gpu": r1 - r0, "cols": 4096, "parallelism": f"rows{world}",
            "l2": "inputs larger than L2 (256 MiB)"}
    if name == "affine":
        return METRICS[name], "GB/s", "weak", {
            "workload": "affine: y = alpha x + beta, n = 2^26, x ~ U[-4,4), alpha 1.5, beta -0.25, seed 1",
            "bytes_per_element": 8, "parallelism": f"replica{world}", "l2": "inputs larger than L2 (256 MiB)"}
    if name == "add":
        return METRICS[name], "GB/s", "weak", {
            "workload": "add: c = a + b, n = 1,048,576, a,b ~ U[-1,1), seed 0", "bytes_per_element": 12,
            "parallelism": f"replica{world}", "l2": "16 rotating buffer sets (192 MiB) exceed L2"}
    if name == "softmax":
        return METRICS[name], "GB/s", "weak", {
            "workload": "softmax: causal row softmax of x [32, 1024, 1024] ~ U[-8,8), scale 1/8, seed 5",
            "parallelism": f"replica{world}", "l2": "inputs larger than L2 (128 MiB)"}
    if name == "reduce":
        return METRICS[name], "GB/s", "weak", {
            "workload": "reduce: row sums of x [65536 x 1024] ~ U[-4,4), seed 6", "parallelism": f"replica{world}",
            "l2": "inputs larger than L2 (256 MiB)"}
    if name == "block":
        return METRICS[name], "TFLOP/s", "weak", {
            "workload": "block: pre-LN encoder block (reference examples/native/transformer_block), T=2048, d=1024, "
                        "16 heads of 64, d_ff=4096, causal, seeded weights; 11 commands per block (bias/GELU fused "
                        "into the GEMM epilogues; how the weights are read: the line's w_operand)",
            "tokens": 2048, "d_model": 1024, "heads": 16, "d_ff": 4096, "parallelism": f"replica{world}",
            "l2": "scores and probabilities 256 MiB each exceed L2"}
    if name == "attention":
        return METRICS[name], "TFLOP/s", "weak", {
            "workload": "attention: S = Q K^T per head, Q, K [32, 2048, 128] ~ U[-1,1), seed 7; K^T is a strided "
                        "view (no copy)", "batch": 32, "m": 2048, "n": 2048, "k": 128,
            "parallelism": f"replica{world}", "l2": "output 512 MiB exceeds L2"}
    raise ValueError(name)


# ---------------------------------------------------------------- workloads (our implementation)
class Workload:
    """Holds device inputs/outputs for one rank and runs steps through the public API."""

    def __init__(self, name, ctx, group, gather=False, prepare_w=True):
        import numpy as np
        import importlib
        import paralyn_b200 as p
        from paralyn_b200 import b200, shard, synthetic
        self.p, self.np, self.b200, self.shard = p, np, b200, shard
        self.T = importlib.import_module("paralyn_b200.tensor")
        self.name, self.ctx, self.group = name, ctx, group
        self.res = self.T.operators_of(ctx)
        self.queue = self.res.queue
        world, rank = group.world, group.rank
        if name == "chain":
            self.rows, self.k, self.n = 65536, 4096, 4096
            self.chain = shard.ChainShard(ctx, self.rows, self.k, self.n, world, rank, seed=4, w_std=1.0 / 64.0)
            self.chain.fill_synthetic()
            if prepare_w:  # W is the same in every step: its TF32 pair is made once
                self.chain.prepare_weights()
            self.gather = None
            if gather:
                self.gather = shard.GatheredOutput(ctx, self.rows, self.n, group.exchange, rank)
            self.units_total = 2 * self.rows * self.n * self.k
            self.units_local = self.chain.flops()
            self.h2d = 4 * self.chain.local_rows * self.k
            self.d2h = 4 * self.chain.local_rows * self.n
        elif name == "gemm":
            m = n = k = 4096
            r0, r1 = shard.row_range(m, world, rank)
            self.m_local, self.n, self.k = r1 - r0, n, k
            self.a = ctx.buffer(4 * self.m_local * k)
            self.b = ctx.buffer(4 * k * n)
            self.c = ctx.buffer(4 * self.m_local * n)
            fill = b200.fill_synthetic_into
            for e in (fill(self.queue, self.T.TensorDescriptor(self.a, (self.m_local, k)), seed=3, first_draw=r0 * k),
                      fill(self.queue, self.T.TensorDescriptor(self.b, (k, n)), seed=3, first_draw=m * k)):
                e.wait()
                e.close()
            self.units_total, self.units_local = 2 * m * n * k, 2 * self.m_local * n * k
            self.h2d, self.d2h = 4 * self.m_local * k, 4 * self.m_local * n
            self.r0, self.gather = r0, None
            if gather:  # C gathered on every GPU by a peer-store kernel after the GEMM
                self.gather = shard.GatheredOutput(ctx, m, n, group.exchange, rank)
        elif name == "layernorm":
            rows, cols = 16384, 4096
            r0, r1 = shard.row_range(rows, world, rank)
            self.rows_local, self.cols = r1 - r0, cols
            self.x = ctx.buffer(4 * self.rows_local * cols)
            self.g, self.bt = ctx.buffer(4 * cols), ctx.buffer(4 * cols)
            self.y = ctx.buffer(4 * self.rows_local * cols)
            fill = b200.fill_synthetic_into
            D = self.T.TensorDescriptor
            for e in (fill(self.queue, D(self.x, (self.rows_local, cols)), seed=2, first_draw=2 * r0 * cols,
                           distribution=b200.NORMAL, p0=0.0, p1=1.0),
                      fill(self.queue, D(self.g, (cols,)), seed=2, first_draw=2 * rows * cols,
                           distribution=b200.NORMAL, p0=1.0, p1=0.02),
                      fill(self.queue, D(self.bt, (cols,)), seed=2, first_draw=2 * rows * cols + 2 * cols,
                           distribution=b200.NORMAL, p0=0.0, p1=0.02)):
                e.wait()
                e.close()
            self.units_total = 2 * rows * cols * 4 + 2 * cols * 4 * world
            self.units_local = 2 * self.rows_local * cols * 4 + 2 * cols * 4
            self.h2d = self.d2h = 4 * self.rows_local * cols
        elif name == "affine":
            self.count = 1 << 26
            self.x = ctx.buffer(4 * self.count)
            self.y = ctx.buffer(4 * self.count)
            e = b200.fill_synthetic_into(self.queue, self.T.TensorDescriptor(self.x, (self.count,)), seed=1, p0=4.0)
            e.wait()
            e.close()
            self.module = p.Module.load_file(ctx, p.array.operators_path())
            self.kernel = self.module.kernel("array_affine_scalar")
            self.xv, self.yv = self.x.view(access=p.Access.READ), self.y.view(access=p.Access.WRITE)
            self.units_local = 8 * self.count
            self.units_total = self.units_local * world
            self.h2d = self.d2h = 4 * self.count
        elif name == "add":
            self.count, self.sets = 1 << 20, 16
            self.module = p.Module.load_file(ctx, p.array.operators_path())
            self.kernel = self.module.kernel("array_add")
            self.bufs = []
            for s in range(self.sets):
                a, b, c = (ctx.buffer(4 * self.count) for _ in range(3))
                for buf, first in ((a, 0), (b, self.count)):
                    e = b200.fill_synthetic_into(self.queue, self.T.TensorDescriptor(buf, (self.count,)), seed=0,
                                                 first_draw=first)
                    e.wait()
                    e.close()
                self.bufs.append((a, b, c, a.view(access=p.Access.READ), b.view(access=p.Access.READ),
                                  c.view(access=p.Access.WRITE)))
            self.units_local = 12 * self.count
            self.units_total = self.units_local * world
            self.h2d, self.d2h = 8 * self.count, 4 * self.count
            self.turn = 0
        elif name in ("softmax", "reduce"):
            D = self.T.TensorDescriptor
            if name == "softmax":
                self.shape = (32, 1024, 1024)
                count = 32 * 1024 * 1024
                self.units_local = 8 * count
                self.h2d = self.d2h = 4 * count
            else:
                self.shape = (65536, 1024)
                count = 65536 * 1024
                self.units_local = 4 * count + 4 * 65536
                self.h2d, self.d2h = 4 * count, 4 * 65536
            self.x = ctx.buffer(4 * count)
            self.y = ctx.buffer(self.d2h)
            e = b200.fill_synthetic_into(self.queue, D(self.x, (count,)), seed=5 if name == "softmax" else 6,
                                         p0=8.0 if name == "softmax" else 4.0)
            e.wait()
            e.close()
            self.units_total = self.units_local * world
        elif name == "block":
            from paralyn_b200.block import EncoderBlock
            self.block = EncoderBlock(ctx, 2048, 1024, 16, 4096, causal=True, seed=2026)
            if prepare_w:  # the weights are the same in every block: their TF32 pairs are made once
                self.block.prepare_weights()
            self.units_local = self.block.flops()
            self.units_total = self.units_local * world
            self.h2d = self.d2h = 4 * 2048 * 1024
        elif name == "attention":
            D = self.T.TensorDescriptor
            self.heads, self.seq, self.dh = 32, 2048, 128
            count = self.heads * self.seq * self.dh
            self.q, self.kmat = ctx.buffer(4 * count), ctx.buffer(4 * count)
            self.c = ctx.buffer(4 * self.heads * self.seq * self.seq)
            for buf, first in ((self.q, 0), (self.kmat, count)):
                e = b200.fill_synthetic_into(self.queue, D(buf, (count,)), seed=7, first_draw=first)
                e.wait()
                e.close()
            self.units_local = 2 * self.heads * self.seq * self.seq * self.dh
            self.units_total = self.units_local * world
            self.h2d, self.d2h = 8 * count, 4 * self.heads * self.seq * self.seq
        self.metric, self.unit, self.scaling, self.config = describe(name, world, rank, gather)
        self.scale = 1e-12 if self.unit == "TFLOP/s" else 1e-9
        if name == "block":
            self.config["gemm_flops_per_block"] = self.units_local
        self.ctx.synchronize()

    def step(self):
        """Enqueue one step; returns (events, dominant-kernel event)."""
        p = self.p
        if self.name == "chain":
            mm, ln = self.chain.step(self.gather)
            return [mm, ln], mm
        if self.name == "gemm":
            D = self.T.TensorDescriptor
            c = D(self.c, (self.m_local, self.n))
            e = self.T.matmul_into(self.queue, self.res.module, D(self.a, (self.m_local, self.k)), D(self.b, (self.k, self.n)),
                                   c, m=self.m_local, n=self.n, k=self.k)
            if self.gather is None:
                return [e], e
            g = self.b200.gather_rows_into(self.queue, c, self.gather.targets, row_offset=self.r0)
            return [e, g], e
        if self.name == "layernorm":
            D = self.T.TensorDescriptor
            e = self.T.layer_norm_into(self.queue, self.res.module, D(self.x, (self.rows_local, self.cols)),
                                       D(self.g, (self.cols,)), D(self.bt, (self.cols,)),
                                       D(self.y, (self.rows_local, self.cols)), epsilon=1e-5)
            return [e], e
        if self.name == "affine":
            e = self.queue.launch(self.kernel, [self.xv, self.yv, p.u32(self.count), p.f32(1.5), p.f32(-0.25)],
                                  grid=((self.count + 255) // 256, 1, 1), block=(256, 1, 1))
            return [e], e
        if self.name in ("softmax", "reduce"):
            D = self.T.TensorDescriptor
            if self.name == "softmax":
                e = self.T.softmax_rows_into(self.queue, self.res.module, D(self.x, self.shape), D(self.y, self.shape),
                                             scale=0.125, causal=True)
            else:
                e = self.T.reduce_rows_into(self.queue, self.res.module, D(self.x, self.shape),
                                            D(self.y, (self.shape[0],)))
            return [e], e
        if self.name == "block":
            events = self.block.run(fused=True)
            return events, events[8]  # the MLP up-projection (+ bias + GELU), the largest GEMM
        if self.name == "attention":
            D = self.T.TensorDescriptor
            H, S, K = self.heads, self.seq, self.dh
            e = self.T.batched_matmul_into(self.queue, self.res.module, D(self.q, (H, S, K)),
                                           D(self.kmat, (H, K, S), 0, (S * K, 1, K)), D(self.c, (H, S, S)),
                                           batch=H, m=S, n=S, k=K)
            return [e], e
        a, b, c, av, bv, cv = self.bufs[self.turn % self.sets]
        self.turn += 1
        e = self.queue.launch(self.kernel, [av, bv, cv, p.u32(self.count)], grid=((self.count + 255) // 256, 1, 1),
                              block=(256, 1, 1))
        return [e], e

    def streamed_step(self, host_in, host_out):
        """One step with inputs and result in host memory, pipelined over slices:
        per slice an upload, the step's kernels on that slice and a download, all
        enqueued at once (stream-ordered copies overlap the other slices' kernels).
        host_in: addresses matching io_buffers()[0]; host_out: address for the result.
        Returns the events."""
        p, b200, D = self.p, self.b200, self.T.TensorDescriptor
        if self.name == "chain":
            slices = max(1, min(8, self.chain.local_rows // 1024))
            return self.chain.step_from_host(host_in[0], host_out, slices=slices, gathered=self.gather)
        events = []

        def cuts(total, parts, align):
            return sorted({min(total, -(-total * i // parts) // align * align) for i in range(1, parts)} | {0, total})

        if self.name in ("gemm", "layernorm"):
            rows, width_in, width_out = ((self.m_local, self.k, self.n) if self.name == "gemm"
                                         else (self.rows_local, self.cols, self.cols))
            src, dst = (self.a, self.c) if self.name == "gemm" else (self.x, self.y)
            c = cuts(rows, 4, 128)
            for lo, hi in zip(c, c[1:]):
                n_rows, io, oo = hi - lo, 4 * lo * width_in, 4 * lo * width_out
                events.append(b200.write_async(self.queue, src, host_in[0] + io, offset=io, nbytes=4 * n_rows * width_in))
                if self.name == "gemm":
                    events.append(self.T.matmul_into(self.queue, self.res.module, D(self.a, (n_rows, self.k), io),
                                                     D(self.b, (self.k, self.n)), D(self.c, (n_rows, self.n), oo),
                                                     m=n_rows, n=self.n, k=self.k))
                else:
                    events.append(self.T.layer_norm_into(self.queue, self.res.module, D(self.x, (n_rows, self.cols), io),
                                                         D(self.g, (self.cols,)), D(self.bt, (self.cols,)),
                                                         D(self.y, (n_rows, self.cols), oo), epsilon=1e-5))
                events.append(b200.read_async(self.queue, dst, host_out + oo, offset=oo, nbytes=4 * n_rows * width_out))
            return events
        if self.name in ("softmax", "reduce", "attention", "block"):  # one slice: upload, step, download
            ins, (out, out_bytes) = self.io_buffers()
            for (buf, nbytes), host in zip(ins, host_in):
                events.append(b200.write_async(self.queue, buf, host, nbytes=nbytes))
            events += self.step()[0]
            events.append(b200.read_async(self.queue, out, host_out, nbytes=out_bytes))
            return events
        if self.name == "affine":
            ins, out = [self.x], self.y
        else:
            a, b, c_buf = self.bufs[0][:3]
            ins, out = [a, b], c_buf
        c = cuts(self.count, 8 if self.name == "affine" else 1, 1024)  # 12 MiB add: one slice
        for lo, hi in zip(c, c[1:]):
            n_el, off = hi - lo, 4 * lo
            for buf, host in zip(ins, host_in):
                events.append(b200.write_async(self.queue, buf, host + off, offset=off, nbytes=4 * n_el))
            views = [buf.view(offset=off, size=4 * n_el, access=p.Access.READ) for buf in ins]
            views.append(out.view(offset=off, size=4 * n_el, access=p.Access.WRITE))
            scalars = [p.u32(n_el)] + ([p.f32(1.5), p.f32(-0.25)] if self.name == "affine" else [])
            events.append(self.queue.launch(self.kernel, views + scalars, grid=((n_el + 255) // 256, 1, 1),
                                            block=(256, 1, 1)))
            events.append(b200.read_async(self.queue, out, host_out + off, offset=off, nbytes=4 * n_el))
            events += views  # closed with the events once the step is done
        return events

    def io_buffers(self):
        """(device buffer written from host, device buffer read back) for the e2e leg."""
        if self.name == "chain":
            return [(self.chain.x, self.h2d)], (self.chain.y, self.d2h)
        if self.name == "gemm":
            return [(self.a, self.h2d)], (self.c, self.d2h)
        if self.name == "layernorm":
            return [(self.x, self.h2d)], (self.y, self.d2h)
        if self.name == "affine":
            return [(self.x, self.h2d)], (self.y, self.d2h)
        if self.name in ("softmax", "reduce"):
            return [(self.x, self.h2d)], (self.y, self.d2h)
        if self.name == "attention":
            return [(self.q, self.h2d // 2), (self.kmat, self.h2d // 2)], (self.c, self.d2h)
        if self.name == "block":
            return [(self.block.buf["x"], self.h2d)], (self.block.buf["out"], self.d2h)
        a, b, c = self.bufs[0][:3]
        return [(a, 4 * self.count), (b, 4 * self.count)], (c, self.d2h)


def time_steps(w, ctx, group, steps, warmup):
    """W untimed warm-up steps, then `steps` steps between two queue markers (device
    time, max over ranks) with the clock sampler running. Returns the timed region."""
    import paralyn_b200 as p
    from paralyn_b200 import b200
    warm = []
    for _ in range(warmup):
        warm += w.step()[0]
    w.ctx.synchronize()
    for e in warm:
        e.close()
    kernels_before = p.device_kernel_count(ctx)
    group.barrier()
    ctx.synchronize()
    timed, dominant = [], []
    with Clocks(group.local_rank) as clocks:
        start = b200.marker(w.queue)
        for _ in range(steps):
            events, main = w.step()
            timed += events
            dominant.append(main)
        stop = b200.marker(w.queue)
        seconds = b200.elapsed(start, stop)
    ctx.synchronize()
    group.barrier()
    kernels = p.device_kernel_count(ctx) - kernels_before  # markers launch no kernel
    durations = [e.timing().duration_seconds for e in dominant]
    variant = last_variant(ctx, w.name)
    for e in timed + [start, stop]:
        e.close()
    worst = group.max(seconds)
    return {"seconds": worst, "steps": steps, "value": w.units_total * steps / worst * w.scale,
            "ms_per_step": worst / steps * 1e3, "gpu_launches": int(group.max(kernels)),
            "clocks": clocks.summary(), "variant": variant, "dominant_seconds": sum(durations) / len(durations)}


# Steps whose device work is a few microseconds (the 2^20 add: about 2 us of HBM time)
# finish faster than the host enqueues them (about 14 us per command through the
# binding, the checks and the launch), so a host-paced loop times the host. These
# workloads are timed as the reference times them (the GPU duration of its command
# buffers): in windows of this many steps, each enqueued behind a queue hold
# (pr_b200_queue_hold) long enough for the host to enqueue the whole window, so the
# steps run back to back on the device; `value` is the steps' device time between
# the markers around each window, summed. The host-paced figure is reported beside
# it (`host_paced`).
QUEUE_AHEAD = {"add": 1000}
HOLD_PER_STEP_S = 40e-6


def time_steps_queued(w, ctx, group, steps, warmup, per_window):
    """time_steps with the device held while each window of steps is enqueued."""
    import paralyn_b200 as p
    from paralyn_b200 import b200
    warm = []
    for _ in range(warmup):
        warm += w.step()[0]
    w.ctx.synchronize()
    for e in warm:
        e.close()
    kernels_before = p.device_kernel_count(ctx)
    group.barrier()
    ctx.synchronize()
    timed, dominant, windows, holds = [], [], [], []
    hold_s = min(1.0, 2e-3 + HOLD_PER_STEP_S * per_window)
    with Clocks(group.local_rank) as clocks:
        done = 0
        while done < steps:
            n = min(per_window, steps - done)
            holds.append(b200.queue_hold(w.queue, hold_s))
            start = b200.marker(w.queue)
            for _ in range(n):
                events, main = w.step()
                timed += events
                dominant.append(main)
            windows.append((start, b200.marker(w.queue)))
            done += n
        ctx.synchronize()
    group.barrier()
    seconds = sum(b200.elapsed(a, b) for a, b in windows)
    kernels = p.device_kernel_count(ctx) - kernels_before - len(holds)  # the holds are not steps
    durations = [e.timing().duration_seconds for e in dominant]
    variant = last_variant(ctx, w.name)
    for e in timed + holds + [x for pair in windows for x in pair]:
        e.close()
    worst = group.max(seconds)
    return {"seconds": worst, "steps": steps, "value": w.units_total * steps / worst * w.scale,
            "ms_per_step": worst / steps * 1e3, "gpu_launches": int(group.max(kernels)),
            "clocks": clocks.summary(), "variant": variant, "dominant_seconds": sum(durations) / len(durations),
            "queued": {"steps_per_window": per_window, "windows": len(windows), "hold_s": hold_s,
                       "busy_fraction": round(sum(durations) / seconds, 4),
                       "timing": "device time between markers around windows of steps enqueued behind a "
                                 "queue hold (pr_b200_queue_hold), summed; the holds are outside the windows"}}


def timed_region(w, ctx, group, steps, warmup):
    """The workload's timed region: queued-ahead windows for the microsecond-scale
    steps (with the host-paced figure beside them), else time_steps."""
    if w.name not in QUEUE_AHEAD:
        return time_steps(w, ctx, group, steps, warmup)
    t = time_steps_queued(w, ctx, group, steps, warmup, QUEUE_AHEAD[w.name])
    paced = time_steps(w, ctx, group, steps, warmup)
    t["host_paced"] = {"value": round(paced["value"], 3), "ms_per_step": round(paced["ms_per_step"], 5),
                       "steps": steps, "timing": "device time between two markers around steps enqueued one by "
                                                 "one by the host (bound by the host's enqueue rate)"}
    return t


def sm_count():
    """Streaming multiprocessors of the GPU in use, queried at run time."""
    import torch
    if torch.cuda.is_available():
        return torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    return 148  # a B200, for device-free calls


def with_clock_fraction(roofline, clocks):
    mhz = clocks.get("sm_mhz")
    if roofline.get("bound") == "fp32_ffma" and mhz:  # the FFMA peak scales with the clock actually run
        roofline["frac_at_median_sm_clock"] = round(
            roofline["achieved"] / (sm_count() * 128 * 2 * mhz * 1e6 / 1e12), 4)
    return roofline


def steps_for(args, name, w, world):
    # Sharded workloads shrink per GPU as N grows; keep the timed region near a second.
    return args.steps or DEFAULT_STEPS[name] * (world if w.scaling == "strong" else 1)


# The benchmark configurations measured beside the chain headline, each in its own
# timed region of the same process (the metric's GEMM TFLOP/s and LayerNorm / affine /
# add HBM GB/s at the configurations' sizes).
SIDE_CONFIGS = ("gemm", "layernorm", "affine", "add")


def side_configs(args, ctx, group):
    out = {}
    for name in SIDE_CONFIGS:
        w = Workload(name, ctx, group)
        if args.matmul_mode != "auto" and name == "gemm":
            w.config["matmul_mode"] = args.matmul_mode
        t = timed_region(w, ctx, group, DEFAULT_STEPS[name] * (group.world if w.scaling == "strong" else 1),
                         args.warmup)
        roofline = with_clock_fraction(roofline_for(w, t["dominant_seconds"], t["variant"], t["seconds"]),
                                       t["clocks"])
        out[name] = {"metric": w.metric, "value": round(t["value"], 3), "unit": w.unit, "steps": t["steps"],
                     "warmup": args.warmup, "ms_per_step": round(t["ms_per_step"], 5), "scaling": w.scaling,
                     "config": w.config, "roofline": roofline, "clocks": t["clocks"],
                     "gpu_launches": t["gpu_launches"], "dominant_kernel_variant": t["variant"]}
        for key in ("queued", "host_paced"):
            if key in t:
                out[name][key] = t[key]
        del w
        ctx.synchronize()
    return out


def run_ours(args, group):
    import paralyn_b200 as p
    world = group.world
    ctx = p.Context(f"cuda:{group.local_rank}")
    p.set_matmul_mode(ctx, {"auto": p.MatmulMode.AUTO, "reference": p.MatmulMode.REFERENCE,
                            "ffma": p.MatmulMode.FFMA, "tf32x3": p.MatmulMode.TF32X3}[args.matmul_mode])
    w = Workload(args.workload, ctx, group, gather=args.gather, prepare_w=not args.split_w_per_step)
    if args.matmul_mode != "auto":
        w.config["matmul_mode"] = args.matmul_mode
    t = timed_region(w, ctx, group, steps_for(args, args.workload, w, world), args.warmup)
    steps = t["steps"]

    e2e = None
    if not args.no_e2e:
        # About 24 GB of host<->device traffic per e2e measurement (PCIe-bound): the
        # pipeline's fill and drain, one slice each, weigh less over more steps (chain:
        # 11 steps, 92-94 TFLOP/s against 90 with 3).
        e2e_steps = max(2, min(steps, int(24e9 // (w.h2d + w.d2h))))
        e2e = end_to_end(w, ctx, group, steps=e2e_steps)

    roofline = with_clock_fraction(roofline_for(w, t["dominant_seconds"], t["variant"], t["seconds"]), t["clocks"])
    line = {"metric": w.metric, "value": round(t["value"], 3), "unit": w.unit, "n_gpus": world, "steps": steps,
            "warmup": args.warmup, "ms_per_step": round(t["ms_per_step"], 4), "higher_is_better": True,
            "scaling": w.scaling, "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded SplitMix64 stream generated on device)", "config": w.config, "e2e": e2e,
            "gpu_launches": t["gpu_launches"], "roofline": roofline, "clocks": t["clocks"],
            "dominant_kernel_variant": t["variant"], "headline_metric": METRIC}
    for key in ("queued", "host_paced"):
        if key in t:
            line[key] = t[key]
    if args.workload == "chain":
        line["w_operand"] = ("split in every step (pr_matmul_f32)" if args.split_w_per_step else
                             "prepared once before the timed steps (pr_b200_matmul_prepare_f32); every step "
                             "splits X, multiplies (pr_b200_matmul_prepared_f32) and normalizes")
    if args.workload == "block":
        line["w_operand"] = ("split in every block (pr_b200_matmul_bias_activation_f32)" if args.split_w_per_step
                             else "the four projection weights prepared once before the timed steps "
                             "(pr_b200_matmul_prepare_f32); every block runs its 11 commands with the projections "
                             "reading them (pr_b200_matmul_prepared_bias_activation_f32)")
    if args.workload == "chain" and not args.no_configs:
        line["configs"] = side_configs(args, ctx, group)
    if group.rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.workload)
    ctx.close()
    return line


DOMINANT_ENTRY = {"chain": ("b200_matmul_prepared_f32", "paralyn_matmul_f32"), "gemm": "paralyn_matmul_f32",
                  "layernorm": "paralyn_layer_norm_f32", "affine": "array_affine_scalar", "add": "array_add",
                  "softmax": "paralyn_softmax_rows_f32", "reduce": "paralyn_reduce_rows_f32",
                  "attention": "paralyn_batched_matmul_f32",
                  "block": ("b200_matmul_prepared_bias_activation_f32", "b200_matmul_bias_activation_f32")}


def last_variant(ctx, workload):
    """Implementation the library chose for the dominant entry (from the evidence log)."""
    from paralyn_b200 import b200
    entries = DOMINANT_ENTRY[workload]
    for entry in (entries,) if isinstance(entries, str) else entries:
        variant = b200.last_variant(ctx, entry)
        if variant is not None:
            return variant
    return None


def end_to_end(w, ctx, group, steps):
    """The same steps with host buffers, through the public API: every step copies its
    inputs in from pinned host memory and its result out to pinned host memory.

    The headline leg pipelines each step over slices with the stream-ordered copies
    (pr_b200_buffer_write_async / read_async), so PCIe traffic in both directions
    overlaps the kernels; `blocking` repeats it with the reference's blocking
    pr_buffer_write / pr_buffer_read around whole-step launches."""
    import torch
    torch.cuda.set_device(group.local_rank)  # pinned host memory comes from this rank's GPU context
    ins, (out_buf, out_bytes) = w.io_buffers()
    pinned_in = [(buf, torch.empty(nbytes, dtype=torch.uint8, pin_memory=True), nbytes) for buf, nbytes in ins]
    for buf, host, nbytes in pinned_in:  # the device's current inputs become the host copy
        buf.read_into(host.data_ptr(), nbytes)
    pinned_out = torch.empty(out_bytes, dtype=torch.uint8, pin_memory=True)
    host_in = [host.data_ptr() for _, host, _ in pinned_in]

    def close(events):
        for e in events:
            e.close()

    close(w.streamed_step(host_in, pinned_out.data_ptr()))  # warm-up (first-use costs)
    ctx.synchronize()
    group.barrier()
    t0 = time.perf_counter()
    pending = []
    for _ in range(steps):
        pending.append(w.streamed_step(host_in, pinned_out.data_ptr()))
        if len(pending) > 2:  # keep at most two steps in flight; release older events
            close(pending.pop(0))
    for events in pending:
        close(events)
    ctx.synchronize()
    seconds = time.perf_counter() - t0
    group.barrier()
    worst = group.max(seconds)

    group.barrier()
    t0 = time.perf_counter()
    for buf, host, nbytes in pinned_in:
        buf.write_from(host.data_ptr(), nbytes)
    events, _ = w.step()
    out_buf.read_into(pinned_out.data_ptr(), out_bytes)
    close(events)
    ctx.synchronize()
    blocking = group.max(time.perf_counter() - t0)
    group.barrier()

    # The reference binding's usual case: pageable (numpy) host arrays, blocking calls.
    import numpy as np
    pageable_in = [(buf, host.numpy().copy(), nbytes) for buf, host, nbytes in pinned_in]
    pageable_out = np.empty(out_bytes, np.uint8)

    def pageable_step():
        for buf, arr, nbytes in pageable_in:
            buf.write_from(arr.ctypes.data, nbytes)
        events, _ = w.step()
        out_buf.read_into(pageable_out.ctypes.data, out_bytes)
        close(events)
        ctx.synchronize()

    pageable_step()  # first use allocates the library's pinned staging ring
    group.barrier()
    t0 = time.perf_counter()
    pageable_step()
    pageable = group.max(time.perf_counter() - t0)
    group.barrier()
    return {"value": round(w.units_total * steps / worst * w.scale, 3), "unit": w.unit,
            "h2d_bytes_per_step": sum(n for _, _, n in pinned_in), "d2h_bytes_per_step": out_bytes,
            "timing": "host wall clock over the steps (inputs uploaded from and results downloaded to pinned host "
                      "memory every step, pipelined over row/element slices with stream-ordered copies), max over ranks",
            "steps": steps,
            "blocking": {"value": round(w.units_total / blocking * w.scale, 3), "unit": w.unit, "steps": 1,
                         "timing": "one step between blocking pr_buffer_write and pr_buffer_read"},
            "blocking_pageable": {"value": round(w.units_total / pageable * w.scale, 3), "unit": w.unit, "steps": 1,
                                  "timing": "the same with pageable (numpy) host arrays"}}


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "sm_max_mhz": 1965.0}, "fallback"


def roofline_for(w, seconds, variant, region_seconds):
    """Dominant kernel vs its roofline. Tensor-bound kernels timed inside a region of
    half a second or more are compared with the sustained (power-capped) GEMM figure,
    shorter ones with the burst figure."""
    peaks, basis = measured_peaks()
    simt = bool(variant) and "simt" in variant
    traffic = load_traffic().get(w.name + ("_ffma" if simt and "ffma" in variant else ""))
    if simt and "ffma" not in variant:
        traffic = None  # no capture of the reference-order kernel
    if w.name in ("layernorm", "affine", "add", "softmax", "reduce"):
        per_launch = w.units_local
        achieved = per_launch / seconds / 1e9
        return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": traffic,
                "peak_basis": f"{basis} STREAM-style copy"}
    if w.name == "block":
        flops = 2 * w.block.T * w.block.D * w.block.F  # the up-projection launch
    elif w.name == "attention":
        flops = w.units_local
    else:
        flops = 2 * (w.chain.local_rows if w.name == "chain" else w.m_local) * w.n * w.k
    achieved = flops / seconds / 1e12
    if variant and "tf32x3" in variant:
        sustained = region_seconds >= 0.5 and "bf16_tflops_sustained" in peaks
        peak = peaks["bf16_tflops_sustained" if sustained else "bf16_tflops"] / 2 / 3
        which = "sustained" if sustained else "burst"
        return {"bound": "tensor", "achieved": round(achieved, 2), "peak": round(peak, 1), "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4), "traffic": traffic,
                "peak_basis": f"{basis} bf16 cuBLAS {which} / 2 (TF32 rate) / 3 (three TF32 products per "
                              "FP32 product)"}
    sms = sm_count()
    peak = sms * 128 * 2 * peaks.get("sm_max_mhz", 1965.0) * 1e6 / 1e12
    if variant and "reference_order" in variant:
        # A rounded multiply and a rounded add per product: two FP32 pipe operations
        # for the two flops an FFMA does in one.
        return {"bound": "fp32_mul_add", "achieved": round(achieved, 2), "peak": round(peak / 2, 1),
                "unit": "TFLOP/s", "frac": round(achieved / (peak / 2), 4), "traffic": traffic,
                "frac_of_ffma_peak": round(achieved / peak, 4),
                "peak_basis": f"{sms} SMs x 128 FP32 lanes x 1 flop (FMUL then FADD per product) x {basis} max "
                              "SM clock"}
    return {"bound": "fp32_ffma", "achieved": round(achieved, 2), "peak": round(peak, 1), "unit": "TFLOP/s",
            "frac": round(achieved / peak, 4), "traffic": traffic,
            "peak_basis": f"{sms} SMs x 128 FP32 lanes x 2 flop x {basis} max SM clock"}


def load_traffic():
    path = ROOT / "profiles" / "traffic.json"
    if path.exists():
        return json.loads(path.read_text())
    return {}


# ---------------------------------------------------------------- CPU side (oracle)
def cpu_sample(workload, budget_seconds, threaded=True):
    """Runs the oracle (all host threads, or one with threaded=False) on a bounded sample;
    returns (units/s, unit, sample text)."""
    import numpy as np
    import oracle
    from paralyn_b200 import synthetic
    oracle.use_all_cores()
    if workload in ("chain", "gemm"):
        k = n = 4096
        b = synthetic.normal(4, 0, k * n, 0.0, 1.0 / 64) if workload == "chain" else synthetic.uniform(3, 0, k * n)
        rows = max(8, oracle.threads()) if threaded else 1
        block = synthetic.uniform(3, 1, 64 * k)  # timing does not depend on the values
        a = np.tile(block, (rows + 63) // 64)[:rows * k]
        t0 = time.perf_counter()
        z = oracle.matmul(a, b, rows, n, k, threaded=threaded)
        if workload == "chain":
            oracle.layer_norm(z, np.ones(n, np.float32), np.zeros(n, np.float32), 1e-5, threaded=threaded)
        t = time.perf_counter() - t0
        scale = max(1, int(budget_seconds / max(t, 1e-3)))
        rows2 = min(rows * scale, 65536)
        a = np.tile(block, (rows2 + 63) // 64)[:rows2 * k]
        t0 = time.perf_counter()
        z = oracle.matmul(a, b, rows2, n, k, threaded=threaded)
        if workload == "chain":
            oracle.layer_norm(z, np.ones(n, np.float32), np.zeros(n, np.float32), 1e-5, threaded=threaded)
        t = time.perf_counter() - t0
        return 2 * rows2 * n * k / t * 1e-12, "TFLOP/s", f"{rows2} of the rows x 4096 x 4096 (reference-order sequential GEMM" + (
            " + reference-order LayerNorm)" if workload == "chain" else ")")
    if workload == "layernorm":
        cols = 4096
        rows = 4096
        x = synthetic.normal(2, 0, rows * cols).reshape(rows, cols)
        g, bt = np.ones(cols, np.float32), np.zeros(cols, np.float32)
        t0 = time.perf_counter()
        reps = 0
        while time.perf_counter() - t0 < budget_seconds or reps == 0:
            oracle.layer_norm(x, g, bt, 1e-5, threaded=threaded)
            reps += 1
        t = time.perf_counter() - t0
        return reps * (2 * rows * cols * 4 + 2 * cols * 4) / t * 1e-9, "GB/s", f"{reps} x 4096 rows x 4096"
    if workload in ("softmax", "reduce"):
        shape = (8, 1024, 1024) if workload == "softmax" else (16384, 1024)
        x = synthetic.uniform(5, 0, int(np.prod(shape)), 8.0).reshape(shape)
        t0 = time.perf_counter()
        reps = 0
        while time.perf_counter() - t0 < budget_seconds or reps == 0:
            if workload == "softmax":
                oracle.softmax_rows(x, np.float32(0.125), causal=True, threaded=threaded)
            else:
                oracle.reduce_rows(x, 0, threaded=threaded)
            reps += 1
        t = time.perf_counter() - t0
        per = 8 * x.size if workload == "softmax" else 4 * x.size + 4 * shape[0]
        return reps * per / t * 1e-9, "GB/s", f"{reps} passes over x {list(shape)}"
    if workload == "block":  # the up-projection GEMM [T, 1024] x [1024, 4096] on a row sample
        k, n = 1024, 4096
        b = synthetic.uniform(7, 0, k * n, 0.125)
        rows = max(8, oracle.threads()) if threaded else 1
        while True:
            a = synthetic.uniform(7, 1 << 30, rows * k)
            t0 = time.perf_counter()
            oracle.matmul(a, b, rows, n, k, threaded=threaded)
            t = time.perf_counter() - t0
            if t >= budget_seconds / 4 or rows >= 2048:
                break
            rows = min(2048, rows * 2)
        return 2 * rows * n * k / t * 1e-12, "TFLOP/s", (f"{rows} rows of the MLP up-projection "
                                                          "[T,1024]x[1024,4096] (sequential reference order)")
    if workload == "attention":
        S, K = 2048, 128
        q, kk = synthetic.uniform(7, 0, S * K), synthetic.uniform(7, 1, S * K)
        rows = max(8, oracle.threads()) if threaded else 1
        while True:  # grow the sample (at most one head's 2048 query rows) to about a quarter of the budget
            c = np.zeros(rows * S, np.float32)
            t0 = time.perf_counter()
            (oracle.batched_matmul_threaded if threaded else oracle.batched_matmul)(q, (0, (0, K, 1)), kk, (0, (0, 1, K)), c,
                                                                                  (0, (0, S, 1)), 1, rows, S, K)
            t = time.perf_counter() - t0
            if t >= budget_seconds / 4 or rows == S:
                break
            rows = min(S, rows * 2)
        return 2 * rows * S * K / t * 1e-12, "TFLOP/s", f"{rows} query rows of one head x 2048 keys x 128"
    count = 1 << 26 if workload == "affine" else 1 << 20
    x = synthetic.uniform(1, 0, count, 4.0)
    y = synthetic.uniform(0, count, count)
    t0 = time.perf_counter()
    reps = 0
    while time.perf_counter() - t0 < budget_seconds or reps == 0:
        if workload == "affine":
            oracle.affine_scalar(x, np.float32(1.5), np.float32(-0.25), threaded=threaded)
        else:
            oracle.add(x, y, threaded=threaded)
        reps += 1
    t = time.perf_counter() - t0
    per = 8 * count if workload == "affine" else 12 * count
    return reps * per / t * 1e-9, "GB/s", f"{reps} passes over n = {count}"


def host_cpu():
    """(model name, logical CPUs) of the host, from /proc/cpuinfo and os.cpu_count()."""
    model = None
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return model, os.cpu_count()


def cpu_baseline(workload, budget=10.0):
    """The oracle port timed on the host: all host threads (OpenMP, the headline
    value) and one thread as the reference's verifier is written."""
    import oracle
    value, unit, sample = cpu_sample(workload, budget)
    one, _, one_sample = cpu_sample(workload, budget / 2, threaded=False)
    model, nproc = host_cpu()
    return {"value": round(value, 6), "unit": unit, "cores": oracle.threads(), "kind": "port",
            "sample": sample + "; oracle restatement of the reference's CPU verifier, -O2 -ffp-contract=off, OpenMP",
            "single_thread": {"value": round(one, 6), "unit": unit, "cores": 1, "sample": one_sample},
            "cpu_model": model, "nproc": nproc}


def run_reference(args, group):
    """The reference's CPU computation of the path (oracle port), rank 0 only, on the
    same configuration (metric, unit and config dict) as our arm."""
    if group.rank != 0:
        return None
    import oracle
    steps = args.steps or 2
    budget = 8.0
    for _ in range(args.warmup):
        cpu_sample(args.workload, 0.5)
    values = []
    unit = sample = None
    for _ in range(steps):
        v, unit, sample = cpu_sample(args.workload, budget)
        values.append(v)
    value = sorted(values)[len(values) // 2]
    world = int(os.environ.get("WORLD_SIZE", args.gpus))
    metric, unit_ours, scaling, config = describe(args.workload, world, 0, args.gather)
    assert unit == unit_ours
    if args.matmul_mode != "auto":
        config["matmul_mode"] = args.matmul_mode
    model, nproc = host_cpu()
    return {"impl": "reference", "metric": metric, "value": round(value, 6), "unit": unit, "n_gpus": world,
            "steps": steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": scaling, "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config,
            "cpu_baseline": {"value": round(value, 6), "unit": unit, "cores": oracle.threads(), "kind": "port",
                             "sample": sample, "cpu_model": model, "nproc": nproc},
            "e2e": {"value": round(value, 6), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    args = parse()
    if args.impl == "reference" and int(os.environ.get("RANK", "0")) != 0:
        return  # the CPU reference runs on rank 0 alone
    group = Group(1) if args.impl == "reference" else Group(args.gpus)
    try:
        line = run_reference(args, group) if args.impl == "reference" else run_ours(args, group)
        if group.rank == 0 and line is not None:
            print(json.dumps(line), flush=True)
    finally:
        group.close()


if __name__ == "__main__":
    main()
