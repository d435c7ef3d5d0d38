"""Benchmark of the causal linear-attention hot path (forward + backward).

Workload (per GPU): B=8, H=8, N=8192, d_head=64, bfloat16 inputs with float32
accumulation; Q, K, V, dO ~ N(0,1) from a seed; a key-padding mask with
per-sequence valid lengths drawn uniform in [N/2, N]; gamma == 1 (the plain
normaliser form phi(q)S/(phi(q)z), clamp 1e-5). One step = one forward and
one backward scan over the batch, the forward handing its segment-start
states to the backward as a training step does. Inputs (268 MB) exceed the
126 MB L2.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Multi-GPU (torchrun, one rank per GPU): every rank runs the full per-GPU
workload on its own batch (batch x head sharding, no collective in the
path): weak scaling; time = max over ranks of the device-timed region.
--scaling strong splits the one B=8 batch over the ranks instead (rank r
takes its slice; with 8 ranks one sequence of H=8 heads each, which the
kernels spread over clusters of up to 8 CTAs per head).

  python bench.py --impl reference [--steps K] [--warmup W]

times the reference's own C++ engine (its float32 CPU build, oracle/_ref) on
the host's cores: each step is one rank's batch, B x H head-sequences each
run at the live length the GPU step masks it to, forward + backward; step i
takes rank (i mod N)'s lengths; the time is the wall clock of each step.

  python bench.py --workload encoder [--seq-len 16384] [--batch 4]

prints a second kind of line (not the default): one training step of the
surgered audio encoder the model path runs (12 pre-LayerNorm blocks, d_model
768, 12 heads, FFN 3072 GELU, linear attention with data-dependent decay
gating, input Linear(80, 768), MSE loss, bf16 autocast, AdamW step), random
init and seeded N(0,1) frames; under torchrun the model is wrapped in DDP
(NCCL gradient all-reduce), per-GPU batch fixed (weak scaling).

  python bench.py --workload stream   long-context streaming inference: B=1, H=4,
      d=64, N=131072 fp16 fed as 32 calls of 4096 tokens with the float32
      state carried between calls (one step = the whole stream)
  python bench.py --workload engine   the C++ engine's forward (SubQEngine): B=1,
      N=1024, D=256 float32 U[0,1), decay 0.99, through the numpy API (host
      buffers) and forward_raw (device buffers); --impl reference times the
      reference's own C++ engine (CPU build) on the same call
  python bench.py --workload headnorm the module's per-head RMSNorm epilogue
      (subq_head_rmsnorm_fwd + _bwd with dweight) at the encoder layer's shape:
      [B=4, H=12, N=16384, D=64] bf16 in the projections' [B, N, H, D] memory
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

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "sub-quadratic-audio-transformer-engine_b200"))

B, H, N, D = 8, 8, 8192, 64
METRIC = "linear-attn fwd+bwd tokens/sec (B=8,H=8,N=8192,d=64 per GPU)"
UNIT = "tokens/s"
CONFIG = {"workload": "causal ELU+1 linear attention fwd+bwd, B=8 H=8 N=8192 d_head=64, "
                      "key-padding mask lengths U[N/2,N], gamma=1",
          "batch_per_gpu": B, "heads": H, "seq_len": N, "head_dim": D,
          "l2": "inputs 268 MB > 126 MB L2 (no flush needed)"}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--path", default="auto", choices=["auto", "exact", "tensorcore"])
    p.add_argument("--workload", default="scan", choices=["scan", "encoder", "stream", "engine", "headnorm"])
    p.add_argument("--scaling", default="weak", choices=["weak", "strong"],
                   help="scan workload: weak = the full batch on every rank; strong = the B=8 batch split "
                        "over the ranks (one slice each)")
    p.add_argument("--seq-len", type=int, default=16384)
    p.add_argument("--batch", type=int, default=4)
    p.add_argument("--scan-batch", type=int, default=8,
                   help="scan workload: sequences per GPU (the headline case is 8; a smaller batch is "
                        "the small case of the kernel profiles)")
    return p.parse_args()


def _device_timer(fn, steps, warmup):
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = clocks_sampler(torch.cuda.current_device())
    time.sleep(0.3)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps, clocks_summary(sampler)


def headnorm_main(args):
    """The per-head RMSNorm kernels at the encoder layer's shape; one step =
    forward + backward (with dweight). Algorithmic bytes: the forward reads x
    and writes y, the backward reads x and dy and writes dx (5 x 100.7 MB)."""
    import torch

    from subq_audio import ops

    B, H, N, D = 4, 12, 16384, 64
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(B, N, H, D, device="cuda", dtype=torch.bfloat16, generator=g).transpose(1, 2)
    dy = torch.randn(B, N, H, D, device="cuda", dtype=torch.bfloat16, generator=g).transpose(1, 2)
    w = torch.rand(D, device="cuda", generator=g) + 0.5

    def step():
        ops.head_rmsnorm(x, w)
        ops.head_rmsnorm_backward(dy, x, w)

    ms, clk = _device_timer(step, max(3, args.steps), max(3, args.warmup))
    nbytes = 5 * x.numel() * x.element_size()
    peak, _, peak_kind = peaks()
    gbs = nbytes / (ms / 1e3) / 1e9
    print(json.dumps({
        "metric": "head RMSNorm fwd+bwd rows/s (B=4,H=12,N=16384,D=64 bf16)", "value": B * H * N / (ms / 1e3),
        "unit": "rows/s", "n_gpus": 1, "steps": max(3, args.steps), "warmup": max(3, args.warmup),
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": "subq_head_rmsnorm_fwd + _bwd (dweight), [4, 12, 16384, 64] bf16, [B, N, H, D] memory",
                   "l2": "503 MB moved per step, above the 126 MB L2"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                     "frac": gbs / peak},
        "gpu_launches": 3 * max(3, args.steps), "clocks": clk}))
    return 0


def stream_main(args):
    """Long-context streaming inference (see the module docstring)."""
    import torch

    from subq_audio import ops

    Bs, Hs, Ns, Ls = 1, 4, 131072, 4096
    g = torch.Generator().manual_seed(77)
    hq, hk, hv = (torch.randn(Bs, Hs, Ns, D, generator=g).to(torch.float16).pin_memory() for _ in range(3))
    q, k, v = (x.cuda() for x in (hq, hk, hv))
    o = torch.empty_like(q)
    ho = torch.empty_like(hq).pin_memory()

    # the streaming API: one DecodeStep bound per 4096-token block (its q, k, v
    # and output slices), all sharing the float32 state, which each call
    # updates in place; a stream starts from a zero state
    S = torch.zeros(Bs, Hs, D, D, device="cuda")
    z = torch.zeros(Bs, Hs, D, device="cuda")
    calls = [ops.DecodeStep(q[:, :, s0:s0 + Ls], k[:, :, s0:s0 + Ls], v[:, :, s0:s0 + Ls], o[:, :, s0:s0 + Ls],
                            S, z) for s0 in range(0, Ns, Ls)]

    def run():
        S.zero_(), z.zero_()
        for c in calls:
            c.step()

    ms_eager, _ = _device_timer(run, args.steps, args.warmup)
    path = ops.last_path()
    o_eager = o.clone()
    # the serving form: the whole stream (state reset + 32 calls) captured once
    # in a CUDA graph and replayed, so no per-call host work sits between the
    # kernels; the steps allocate nothing and do not synchronise
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        run()  # launch attributes and occupancy queries happen outside the capture
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        run()
    ms, clk = _device_timer(graph.replay, args.steps, args.warmup)
    torch.cuda.synchronize()
    if not torch.equal(o, o_eager):
        raise SystemExit("graph replay of the stream differs from the eager calls")

    def e2e():  # inputs from pinned host memory, outputs back to it, every step
        q.copy_(hq, non_blocking=True), k.copy_(hk, non_blocking=True), v.copy_(hv, non_blocking=True)
        graph.replay()
        ho.copy_(o, non_blocking=True)

    e2e_ms, _ = _device_timer(e2e, max(3, args.steps // 2), 1)
    tokens = Bs * Ns
    line = {"metric": "streaming linear-attn forward tokens/sec (B=1,H=4,N=131072 as 32x4096 calls, d=64)",
            "value": tokens / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "ms_per_call": ms / (Ns // Ls),
            "ms_per_step_eager": ms_eager, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": "causal ELU+1 linear attention forward, B=1 H=4 d=64, N=131072 fed as 32 "
                                   "calls of 4096 tokens with the float32 (S, z) state carried (ops.DecodeStep), "
                                   "the stream replayed from one CUDA graph",
                       "path": path,
                       "l2": "inputs 201 MB > 126 MB L2"},
            "e2e": {"value": tokens / (e2e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": 3 * hq.numel() * 2, "d2h_bytes_per_step": ho.numel() * 2},
            "gpu_launches": (Ns // Ls) * args.steps, "clocks": clk}  # (plus two state memsets per stream)
    print(json.dumps(line))
    return 0


def engine_main(args):
    """The C++ engine's forward at B=1, N=1024, D=256 float32 (see the module docstring)."""
    import numpy as np

    Be, Ne, De = 1, 1024, 256
    rng = np.random.default_rng(0)
    q, k, v = (rng.random((Be, Ne, De), dtype=np.float32) for _ in range(3))
    reps = max(3, args.steps)
    if args.impl == "reference":
        sys.path.insert(0, os.path.join(REPO, "oracle", "_ref"))
        try:
            import _C as ref_C  # the reference engine built from its sources (CPU)
        except ImportError as exc:
            print(json.dumps({"impl": "reference", "unavailable": f"reference engine not built: {exc}"}))
            return 0
        eng = ref_C.SubQEngine(256 * 1024 * 1024)
        eng.forward(q, k, v, 0.99)
        t0 = time.perf_counter()
        n = 0
        while n < reps and (n == 0 or time.perf_counter() - t0 < 20.0):
            eng.forward(q, k, v, 0.99)
            n += 1
        ms = (time.perf_counter() - t0) / n * 1e3
        val = Be * Ne / (ms / 1e3)
        print(json.dumps({"impl": "reference", "metric": "engine forward tokens/sec (B=1,N=1024,D=256 fp32)",
                          "value": val, "unit": "tokens/s", "n_gpus": 0, "steps": n, "warmup": 1,
                          "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                          "dtype": "f32", "data": "synthetic",
                          "config": {"workload": "SubQEngine.forward B=1 N=1024 D=256 decay 0.99"},
                          "cpu_baseline": {"value": val, "unit": "tokens/s", "cores": 1, "kind": "reference",
                                           "sample": "the whole call (the engine's forward is single-threaded)"},
                          "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}))
        return 0
    import torch

    from subq_audio import SubQEngine

    eng = SubQEngine(256 * 1024 * 1024)
    # through the numpy API: host buffers, copies inside each call
    for _ in range(args.warmup):
        eng.forward(q, k, v, decay_factor=0.99)
    t0 = time.perf_counter()
    for _ in range(reps):
        eng.forward(q, k, v, decay_factor=0.99)
    e2e_ms = (time.perf_counter() - t0) / reps * 1e3
    # forward_raw on device buffers (the engine's state stays in its arena)
    dq, dk, dv = (torch.from_numpy(x).cuda() for x in (q, k, v))
    do = torch.empty_like(dq)
    raw = lambda: eng.forward_raw(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), do.data_ptr(), Be, Ne, De, 0.99)  # noqa: E731
    ms, clk = _device_timer(raw, reps, args.warmup)
    from subq_audio import _capi, ops

    raw()
    torch.cuda.synchronize()
    launches, path = _capi.last_launches(), ops.last_path()
    line = {"metric": "engine forward tokens/sec (B=1,N=1024,D=256 fp32)", "value": Be * Ne / (ms / 1e3),
            "unit": "tokens/s", "n_gpus": 1, "steps": reps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"SubQEngine.forward_raw B=1 N=1024 D=256 decay 0.99 ({path} kernels)",
                       "l2": "3 MB of inputs fit in L2: a latency-bound single-sequence scan"},
            "e2e": {"value": Be * Ne / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": 3 * q.nbytes,
                    "d2h_bytes_per_step": q.nbytes},
            "gpu_launches": reps * launches, "clocks": clk}
    print(json.dumps(line))
    return 0


def encoder_main(args, rank, world, local_rank):
    """One training step of the surgered encoder (see the module docstring)."""
    import datetime

    import torch
    import torch.distributed as dist
    import torch.nn as nn
    import torch.nn.functional as F

    from subq_audio import ops
    from subq_audio.autograd import SubQLinearAttention

    if world > 1:
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    dev = torch.device("cuda", local_rank if world > 1 else 0)
    torch.cuda.set_device(dev)
    Bb, L, Dm, Hh = args.batch, args.seq_len, 768, 12

    class Block(nn.Module):  # pre-LN block of the reference's audio model (model.py:97-135)
        def __init__(self):
            super().__init__()
            self.ln1, self.ln2 = nn.LayerNorm(Dm), nn.LayerNorm(Dm)
            self.attn = SubQLinearAttention(Dm, Hh, use_data_dependent_gating=True)
            self.ff = nn.Sequential(nn.Linear(Dm, 3072), nn.GELU(), nn.Linear(3072, Dm))

        def forward(self, x):
            x = x + self.attn(self.ln1(x))[0]
            return x + self.ff(self.ln2(x))

    torch.manual_seed(0)
    model = nn.Sequential(nn.Linear(80, Dm), *[Block() for _ in range(12)]).to(dev)
    if world > 1:
        model = nn.parallel.DistributedDataParallel(model, device_ids=[dev.index], bucket_cap_mb=25,
                                                    gradient_as_bucket_view=True)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4, fused=True)
    g = torch.Generator().manual_seed(4321 + rank)
    x_h = torch.randn(Bb, L, 80, generator=g).pin_memory()
    y = torch.randn(Bb, L, Dm, generator=g).to(dev)
    x_d = torch.empty(x_h.shape, device=dev)
    loss_h = torch.empty((), dtype=torch.float32).pin_memory()

    def train_step():
        x_d.copy_(x_h, non_blocking=True)  # the step's input frames from pinned host memory
        opt.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = model(x_d)
            loss = F.mse_loss(out.float(), y)
        loss.backward()
        opt.step()
        loss_h.copy_(loss.detach(), non_blocking=True)  # the step's loss back to the host

    for _ in range(args.warmup):
        train_step()
    # the clock sampler starts (rank 0) and every rank waits for its first
    # samples before the barrier, so that all ranks enter the timed steps
    # together (a rank that starts late stalls the others' gradient all-reduce)
    sampler = clocks_sampler(dev.index) if rank == 0 else None
    time.sleep(0.3)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        train_step()
    e1.record()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    clk = clocks_summary(sampler)
    t = torch.tensor([e0.elapsed_time(e1) / args.steps], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    tokens = Bb * L * world
    if rank == 0:
        line = {"metric": f"surgered encoder training step tokens/sec (B={Bb}/GPU, N={L}, 12x768)",
                "value": tokens / (ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": f"12-layer surgered audio encoder training step (pre-LN, d_model 768, "
                                       f"12 heads, FFN 3072, gated decay), B={Bb}/GPU, N={L}, AdamW",
                           "parallelism": f"ddp{world}" if world > 1 else "single", "scan_path": ops.last_path(),
                           "l2": "activations far above the 126 MB L2"},
                "e2e": {"value": tokens / (ms / 1e3), "unit": "tokens/s",
                        "h2d_bytes_per_step": x_h.numel() * 4, "d2h_bytes_per_step": 4},
                "gpu_launches": 7 * 12 * args.steps, "clocks": clk}
        print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()
    return 0


# --------------------------------------------------------------------------
# Reference CPU arm: the reference's own C++ engine (built from its sources
# into oracle/_ref, float32). A step is one rank's batch as the GPU step sees
# it: B x H head-sequences, each run at its live length (the key-padding
# length the GPU step masks with), forward + backward through
# SubQEngine.forward / .backward, one process per host core, longest first.
# --------------------------------------------------------------------------
_REF = {}


def live_lengths(rank, strong=False):
    """Key-padding lengths U[N/2, N] of one rank's B sequences (weak scaling:
    seed 4321 + rank; strong scaling: the shared batch, seed 4321)."""
    import torch

    g = torch.Generator(device="cpu").manual_seed(4321 if strong else 4321 + rank)
    return torch.randint(N // 2, N + 1, (B,), generator=g)


def _ref_init():
    import numpy as np

    sys.path.insert(0, os.path.join(REPO, "oracle", "_ref"))
    import _C  # the reference's pybind module (CPU build)

    rng = np.random.default_rng(os.getpid())
    _REF["eng"] = _C.SubQEngine(64 * 1024 * 1024)  # forward/backward reset its arena per call
    _REF["x"] = [rng.standard_normal((1, N, D)).astype(np.float32) for _ in range(4)]


def _ref_task(n):
    q, k, v, do = (x[:, :n] for x in _REF["x"])
    _REF["eng"].forward(q, k, v, 1.0)
    _REF["eng"].backward(do, q, k, v, 1.0)
    return n


class RefPool:
    """The reference engine on every host core (spawned workers, started
    before this process makes its first CUDA call)."""

    def __init__(self):
        import multiprocessing as mp

        self.cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
        self.pool = mp.get_context("spawn").Pool(self.cores, initializer=_ref_init)
        self.pool.map(_ref_task, [256] * self.cores, chunksize=1)

    def step(self, lens):
        """Seconds of wall time for one batch at these live lengths."""
        tasks = sorted((int(n) for n in lens for _ in range(H)), reverse=True)
        t0 = time.perf_counter()
        self.pool.map(_ref_task, tasks, chunksize=1)
        return time.perf_counter() - t0

    def close(self):
        self.pool.close()
        self.pool.join()


def ref_unavailable():
    d = os.path.join(REPO, "oracle", "_ref")
    if not os.path.isdir(d) or not any(f.startswith("_C") for f in os.listdir(d)):
        return "oracle/_ref was not built"
    return None


def ref_sample_text(cores, steps, lens_note):
    return (f"{steps} steps, each one rank's batch: {B}x{H} head-sequences (d={D}) at their live lengths "
            f"({lens_note}), through the reference C++ SubQEngine.forward+backward (float32), "
            f"{cores} processes, one per core")


def cpu_reference(steps=2):
    """The reference CPU path on rank 0's batch (a bounded sample: two steps);
    returns (tokens/s, info)."""
    why = ref_unavailable()
    if why:
        return None, {"unavailable": why}
    pool = RefPool()
    lens = live_lengths(0).tolist()
    walls = [pool.step(lens) for _ in range(steps)]
    pool.close()
    wall = sum(walls)
    return B * N * steps / wall, {"kind": "reference", "cores": pool.cores,
                                  "sample": ref_sample_text(pool.cores, steps, "rank 0's lengths"),
                                  "wall_s": round(wall, 3)}


# --------------------------------------------------------------------------
def clocks_sampler(dev_index):
    q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    try:
        return subprocess.Popen(["nvidia-smi", "-i", str(dev_index), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
    except OSError:
        return None


def clocks_summary(proc):
    if proc is None:
        return None
    proc.terminate()
    try:
        out, _ = proc.communicate(timeout=5)
    except subprocess.TimeoutExpired:
        proc.kill()
        out, _ = proc.communicate()
    sms, mx, reasons = [], None, set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for line in out.strip().splitlines():
        f = [x.strip() for x in line.split(",")]
        if len(f) < 9:
            continue
        try:
            sms.append(float(f[1]))
            mx = float(f[2])
        except ValueError:
            continue
        for n_, val in zip(names, f[5:9]):
            if val.lower() == "active":
                reasons.add(n_)
    if not sms:
        return None
    return {"sm_mhz": statistics.median(sms), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sms)}


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        return pk["hbm_gbs"], pk["bf16_tflops"], "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


def profile_traffic():
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary."""
    try:
        with open(os.path.join(REPO, "profiles", "traffic.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


def main():
    global B, METRIC, CONFIG
    args = parse()
    if args.scan_batch != B:
        B = args.scan_batch
        METRIC = METRIC.replace("B=8", f"B={B}")
        CONFIG = {**CONFIG, "batch_per_gpu": B}
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))

    if args.workload == "engine":
        return engine_main(args) if rank == 0 else 0
    if args.workload == "headnorm":
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the RMSNorm epilogue is timed on the GPU "
                                  "path only; the reference arm times the scan and engine workloads"}))
            return 0
        return headnorm_main(args) if rank == 0 else 0
    if args.workload == "stream":
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the streaming workload is timed on the "
                                  "GPU path only; the reference arm times the scan and engine workloads"}))
            return 0
        return stream_main(args) if rank == 0 else 0
    if args.workload == "encoder":
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the encoder workload is timed on the "
                                  "tensor-core path only; the reference arm times the scan workload"}))
            return 0
        return encoder_main(args, rank, world, local_rank)

    if args.impl == "reference":
        if rank != 0:  # rank 0 alone times the reference; the others exit without work
            return 0
        why = ref_unavailable()
        if why:
            print(json.dumps({"impl": "reference", "unavailable": why}))
            return 0
        strong = args.scaling == "strong"
        # step i runs rank (i mod world)'s batch at that rank's live lengths (strong
        # scaling: the one shared batch); a step is the work one GPU does in one step
        batches = [live_lengths(0, strong=True).tolist()] if strong else \
            [live_lengths(r).tolist() for r in range(world)]
        pool = RefPool()
        for i in range(args.warmup):
            pool.step(batches[i % len(batches)])
        walls = [pool.step(batches[i % len(batches)]) for i in range(args.steps)]
        pool.close()
        ms = 1e3 * sum(walls) / len(walls)
        val = B * N / (ms / 1e3)  # tokens of one step's batch (B sequences of N positions)
        note = "the shared batch's lengths" if strong else \
            ("rank 0's lengths" if world == 1 else f"ranks 0..{world - 1}'s lengths in turn")
        line = {"impl": "reference", "metric": METRIC, "value": val, "unit": UNIT, "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                "ms_per_step_min": 1e3 * min(walls), "ms_per_step_max": 1e3 * max(walls),
                "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None, "dtype": "f32",
                "data": "synthetic", "config": CONFIG,
                "cpu_baseline": {"value": val, "unit": UNIT, "kind": "reference", "cores": pool.cores,
                                 "sample": ref_sample_text(pool.cores, args.steps, note)},
                "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return 0

    import torch
    import torch.distributed as dist

    # The CPU-baseline pool starts (spawn) before the first GPU call.
    cpu_val, cpu_info = (None, None)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu_val, cpu_info = cpu_reference()

    if world > 1:
        torch.cuda.set_device(local_rank)
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    dev = torch.device("cuda", local_rank if world > 1 else 0)
    torch.cuda.set_device(dev)
    from subq_audio import ops

    strong = args.scaling == "strong"
    if strong and B % world:
        raise SystemExit(f"--scaling strong needs a rank count dividing B={B}")
    Bl = B // world if strong else B  # this rank's sequences
    g = torch.Generator(device="cpu").manual_seed(1234 if strong else 1234 + rank)
    q, k, v, do = (torch.randn(B, H, N, D, generator=g).to(torch.bfloat16) for _ in range(4))
    lens = live_lengths(rank, strong)
    if strong:  # one slice of the shared batch per rank
        sl = slice(rank * Bl, (rank + 1) * Bl)
        q, k, v, do, lens = (x[sl].contiguous() for x in (q, k, v, do, lens))
    mask = torch.arange(N)[None, :] < lens[:, None]
    qd, kd, vd, dod, md = (x.to(dev) for x in (q, k, v, do, mask))
    stream = torch.cuda.current_stream(dev)

    def step(qq, kk, vv, dd, mm):
        # as in training: the forward hands its segment-start states to the backward
        seg = ops.SegmentStates()
        o, _ = ops.scan_forward(qq, kk, vv, mask=mm, normalize=True, path=args.path, segments=seg)
        n_f = ops.last_launches()
        dq, dk, dv, _ = ops.scan_backward(qq, kk, vv, dd, mask=mm, normalize=True, path=args.path, segments=seg)
        return (o, dq, dk, dv), n_f + ops.last_launches()

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- device-resident timing ----
    for _ in range(args.warmup):
        step(qd, kd, vd, dod, md)
    sampler = clocks_sampler(dev.index) if rank == 0 else None
    time.sleep(0.3)  # every rank, before the barrier: the ranks start the timed steps together
    torch.cuda.synchronize(dev)
    barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches = 0
    e0.record(stream)
    for _ in range(args.steps):
        _, n_l = step(qd, kd, vd, dod, md)
        launches += n_l
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    torch.cuda.synchronize(dev)
    clk = clocks_summary(sampler)
    ms = e0.elapsed_time(e1) / args.steps
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    tokens = B * N * (1 if strong else world)
    value = tokens / (ms_max / 1e3)

    # ---- per-kernel launch timing (forward and backward separately) ----
    # back-to-back launches of one kind, so that host-side argument set-up
    # overlaps the previous launch and the events see device time only
    fe = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    reps = max(3, min(args.steps, 10))
    seg = ops.SegmentStates()
    # one launch already in flight when the first event is recorded, so that the
    # events do not count the host's set-up of the first timed launch
    ops.scan_forward(qd, kd, vd, mask=md, normalize=True, path=args.path, segments=seg)
    fe[0].record(stream)
    for _ in range(reps):
        ops.scan_forward(qd, kd, vd, mask=md, normalize=True, path=args.path, segments=seg)
    fe[1].record(stream)
    for _ in range(reps):
        ops.scan_backward(qd, kd, vd, dod, mask=md, normalize=True, path=args.path, segments=seg)
    fe[2].record(stream)
    torch.cuda.synchronize(dev)
    fwd_ms = fe[0].elapsed_time(fe[1]) / reps
    bwd_ms = fe[1].elapsed_time(fe[2]) / reps
    path_used = ops.last_path()

    # ---- end-to-end through the public API with host buffers ----
    # Each step copies its inputs from pinned host memory, runs the forward and
    # backward scans and copies o, dq, dk, dv back. The copies in, the compute
    # and the copies out run on three streams, double-buffered, so step k's
    # outputs travel back while step k+1's inputs arrive (PCIe is full duplex);
    # the timed region spans from before the first input copy to after the
    # last output copy.
    hq, hk, hv, hdo, hm = (x.pin_memory() for x in (q, k, v, do, mask))
    h_in = (hq, hk, hv, hdo, hm)
    outs_h = [[torch.empty((Bl, H, N, D), dtype=torch.bfloat16).pin_memory() for _ in range(4)] for _ in range(2)]
    h2d = sum(x.numel() * x.element_size() for x in h_in)
    d2h = sum(x.numel() * x.element_size() for x in outs_h[0])
    s_in, s_cmp, s_out = (torch.cuda.Stream(dev) for _ in range(3))
    d_in = [[torch.empty_like(x, device=dev) for x in h_in] for _ in range(2)]

    def e2e_run(nsteps):
        ev_c = []
        for kk in range(nsteps):
            buf = kk % 2
            with torch.cuda.stream(s_in):
                if kk >= 2:
                    s_in.wait_event(ev_c[kk - 2])  # step kk-2 has finished reading this buffer set
                for src, dst in zip(h_in, d_in[buf]):
                    dst.copy_(src, non_blocking=True)
                ev_in = torch.cuda.Event()
                ev_in.record(s_in)
            s_cmp.wait_event(ev_in)
            with torch.cuda.stream(s_cmp):
                res, _ = step(*d_in[buf])
                ev = torch.cuda.Event()
                ev.record(s_cmp)
                ev_c.append(ev)
            s_out.wait_event(ev)
            with torch.cuda.stream(s_out):
                for src, dst in zip(res, outs_h[buf]):
                    dst.copy_(src, non_blocking=True)
                    src.record_stream(s_out)

    e2e_run(max(2, args.warmup // 2))
    torch.cuda.synchronize(dev)
    barrier()
    torch.cuda.synchronize(dev)
    e2e_steps = max(6, args.steps)
    e0.record(s_in)
    e2e_run(e2e_steps)
    e1.record(s_out)
    torch.cuda.synchronize(dev)
    barrier()
    t2 = torch.tensor([e0.elapsed_time(e1) / e2e_steps], device=dev)
    if world > 1:
        dist.all_reduce(t2, op=dist.ReduceOp.MAX)
    e2e_val = tokens / (float(t2.item()) / 1e3)

    if rank == 0:
        hbm, tflops, src = peaks()
        valid = float(lens.sum())  # live tokens per head across the batch
        # algorithmic bytes (bf16, d=64): backward reads q,k,v,dO of live tokens and writes dq,dk,dv of all
        bwd_bytes = H * (valid * 4 * D * 2 + Bl * N * 3 * D * 2)
        fwd_bytes = H * (valid * 3 * D * 2 + Bl * N * D * 2)
        dom = "bwd" if bwd_ms >= fwd_ms else "fwd"
        dom_bytes, dom_ms = (bwd_bytes, bwd_ms) if dom == "bwd" else (fwd_bytes, fwd_ms)
        achieved = dom_bytes / (dom_ms / 1e3) / 1e9
        tr = profile_traffic().get(f"{path_used}_{dom}")
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True, "scaling": args.scaling,
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {**CONFIG, "kernel_path": path_used, "batch_this_gpu": Bl},
            "gpu_launches": launches,
            "roofline": {"bound": "hbm", "kernel": dom + (" (pre-pass + one-pass launches)" if dom == "bwd" else ""),
                         "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "peak_source": src,
                         "traffic": (tr * 1.0 if tr is not None else None),
                         "algorithmic_bytes": dom_bytes, "launch_ms": dom_ms},
            "kernels_ms": {"fwd": fwd_ms, "bwd": bwd_ms},
            "tc_frac": (12 * D * D * Bl * H * N) / (ms_max / 1e3) / (tflops * 1e12),
            "e2e": {"value": e2e_val, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "clocks": clk,
        }
        if cpu_val is not None:
            line["cpu_baseline"] = {"value": cpu_val, "unit": UNIT, **cpu_info}
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
