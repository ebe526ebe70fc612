"""Benchmark of the BlockFHT hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...           (N > 1)

Workload (configuration 2 of the baseline, headline point): bf16 latent of
32768 values ~N(0,1), padded block size 32768, layers=3, seed=123, 2^28
generated coordinates per GPU (8192 blocks).  One step = forward of all 2^28
coordinates + backward of an upstream gradient of the same size to the
latent.  value = generated coordinates (all ranks) / step time, Gcoords/s.

Multi-GPU: blocks are independent, so rank r owns blocks
[r*8192, (r+1)*8192) of one generator (weak scaling); the only exchange is
the NCCL all-reduce of the [32768] latent-gradient partials.

The reference arm (--impl reference) times the reference algorithm's CPU
restatement (oracle/, OpenMP over all host cores, fp32 math) on a bounded
sample of the same workload.
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

REPO = Path(__file__).resolve().parent
# NCCL's own banner would otherwise share stdout with the JSON line
os.environ.setdefault("NCCL_DEBUG", "WARN")
sys.path.insert(0, str(REPO / "latent-weight-lab_b200"))
sys.path.insert(0, str(REPO))

METRIC = "BlockFHT Gcoords/s (bf16, bs=32768)"
BLOCK = 32768
LAYERS = 3
SEED = 123
COORDS_PER_GPU = 1 << 28


def _peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clock / throttle sampling while the timed region runs.

    The GPU is named by its UUID (the CUDA ordinal inside a container need not
    match nvidia-smi's index).  A reader thread collects the lines; entering
    waits (at most 5 s) for the first sample so that sampling covers the whole
    timed region, which the caller starts after entering."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None
        self.error = None

    def _gpu_id(self) -> str:
        try:
            import torch

            uuid = str(torch.cuda.get_device_properties(self.gpu).uuid)
            if uuid:
                return uuid if uuid.startswith("GPU-") else "GPU-" + uuid
        except Exception:  # older torch or no device: fall back to the ordinal
            pass
        return str(self.gpu)

    def _reader(self):
        for ln in self.proc.stdout:
            if ln.strip():
                self.lines.append(ln)

    def __enter__(self):
        import threading

        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self._gpu_id()}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
            self.thread = threading.Thread(target=self._reader, daemon=True)
            self.thread.start()
            t0 = time.time()
            while not self.lines and self.proc.poll() is None and time.time() - t0 < 5.0:
                time.sleep(0.01)
        except OSError as exc:
            self.proc, self.error = None, str(exc)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                _, err = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                _, err = self.proc.communicate()
            if self.thread is not None:
                self.thread.join(timeout=2)
            if err and not self.lines:
                self.error = err.strip().splitlines()[-1][:200]

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[4:8]):
                if val.lower() == "active":
                    reasons.add(name)
        out = {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
               "reasons": sorted(reasons), "samples": len(sm)}
        if not sm and self.error:
            out["error"] = self.error
        return out


def _dist_env():
    return int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), \
        int(os.environ.get("LOCAL_RANK", "0"))


def host_threads() -> int:
    """Host cores this process may use (OMP_NUM_THREADS, which torchrun sets to 1, is ignored)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_sample(threads: int, seconds: float = 10.0, chunk_blocks: int = 64) -> dict:
    """Reference algorithm on host cores (fp32, OpenMP): fwd+bwd over chunks of the
    workload's blocks until about `seconds` have elapsed."""
    import numpy as np

    from oracle import oracle as orc

    rng = np.random.default_rng(0)
    z = rng.standard_normal(BLOCK).astype(np.float32)
    size = chunk_blocks * BLOCK
    g = rng.standard_normal(size).astype(np.float32)
    orc.fht_forward(z, 2 * BLOCK, LAYERS, SEED, 0, 2 * BLOCK, threads=threads)  # warm the library
    done, t0 = 0, time.perf_counter()
    while True:
        orc.fht_forward(z, size, LAYERS, SEED, 0, size, threads=threads)
        orc.fht_backward(g, BLOCK, size, LAYERS, SEED, 0, size, threads=threads)
        done += 1
        dt = time.perf_counter() - t0
        if dt >= seconds:
            break
    coords = done * size
    return {"value": coords / dt / 1e9, "unit": "Gcoords/s", "cores": threads, "kind": "port",
            "elapsed_s": dt, "coords": coords,
            "sample": f"{done} x {chunk_blocks} blocks of {BLOCK} (fwd+bwd, fp32 math, layers={LAYERS}) "
                      f"of the bench workload in {dt:.1f}s"}


def _config(n: int) -> dict:
    return {"workload": "C2 headline: BlockFHT fwd+bwd, bf16, block_size=32768, layers=3, 2^28 coords/GPU",
            "block_size": BLOCK, "layers": LAYERS, "seed": SEED, "coords_per_gpu": COORDS_PER_GPU,
            "parallelism": f"block-sharded x{n}", "l2": "no flush: per-step output and upstream gradient "
                                                        "(512 MiB each) exceed the 126 MB L2"}


def run_reference(args) -> None:
    """The reference algorithm on the host cores (oracle/ C port, OpenMP over every
    core this process may use).  The reference has no multi-GPU path, so under
    torchrun rank 0 alone runs it, with all host cores, and its value does not
    grow with N.  Each step is a timed, bounded sample of the workload."""
    _, rank, _ = _dist_env()
    if rank != 0:
        return
    threads = host_threads()
    for _ in range(max(args.warmup, 0)):
        cpu_sample(threads, seconds=0.2)
    per_step = max(0.2, min(4.0, 100.0 / max(args.steps, 1)))  # whole run stays within a couple of minutes
    samples = [cpu_sample(threads, seconds=per_step) for _ in range(args.steps)]
    value = statistics.median(x["value"] for x in samples)
    ms_step = statistics.median(1e3 * x["elapsed_s"] for x in samples)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "Gcoords/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": _config(args.gpus),
        "cpu_baseline": {"value": value, "unit": "Gcoords/s", "cores": threads, "kind": "port",
                         "sample": f"per step: {samples[0]['coords']} coordinates (~{per_step:.2f} s) of fwd+bwd over "
                                   "64-block chunks of the workload, fp32 math (oracle/ C restatement of the "
                                   "reference algorithm, OpenMP); one process on all host cores at every N, since "
                                   "the reference has no multi-GPU path"},
        "e2e": {"value": value, "unit": "Gcoords/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _traffic_from_profiles(which: str):
    """DRAM bytes per launch measured with ncu, recorded in profiles/traffic.json (None if absent)."""
    p = REPO / "profiles" / "traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text()).get(which)
        except (ValueError, OSError):
            return None
    return None


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    from latent_weight_lab import BlockFHT, _native

    world, rank, local = _dist_env()
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl")
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)
    lib = _native.load()

    size_total = COORDS_PER_GPU * world
    start, stop = rank * COORDS_PER_GPU, (rank + 1) * COORDS_PER_GPU
    gen = torch.Generator(device="cpu").manual_seed(0)
    z_host = torch.randn(BLOCK, generator=gen).to(torch.bfloat16).pin_memory()
    z = z_host.to(dev)
    g = torch.randn(COORDS_PER_GPU, device=dev, dtype=torch.bfloat16)
    y = torch.empty(COORDS_PER_GPU, device=dev, dtype=torch.bfloat16)
    code = _native.LWL_BF16
    ws_f = lib.lwl_fht_forward_workspace_bytes(code, BLOCK, size_total, LAYERS, start, stop, 0)
    ws_b = lib.lwl_fht_backward_workspace_bytes(code, BLOCK, size_total, LAYERS, start, stop, 0)
    ws = torch.empty(max(ws_f, ws_b, 1), dtype=torch.uint8, device=dev)
    grad = torch.empty(BLOCK, device=dev, dtype=torch.bfloat16)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream

    def fwd():
        if lib.lwl_fht_forward(code, z.data_ptr(), BLOCK, size_total, LAYERS, SEED, start, stop, y.data_ptr(),
                               ws.data_ptr(), ws.numel(), 0, sp):
            raise RuntimeError(lib.lwl_last_error().decode())

    def bwd():
        if lib.lwl_fht_backward(code, g.data_ptr(), BLOCK, size_total, LAYERS, SEED, start, stop, grad.data_ptr(),
                                ws.data_ptr(), ws.numel(), 0, sp):
            raise RuntimeError(lib.lwl_last_error().decode())
        if world > 1:
            dist.all_reduce(grad)

    nf = lib.lwl_fht_launch_count(code, BLOCK, size_total, LAYERS, start, stop, 0, 0)
    nb = lib.lwl_fht_launch_count(code, BLOCK, size_total, LAYERS, start, stop, 1, 0)

    for _ in range(args.warmup):
        fwd()
        bwd()
    torch.cuda.synchronize()
    ev = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(3)) for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # the clock sampler starts first; the barrier then lines all ranks up
    # right before the timed region
    with ClockSampler(dev.index) as clk:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t0.record(stream)
        for a, b, c in ev:
            a.record(stream)
            fwd()
            b.record(stream)
            bwd()
            c.record(stream)
        t1.record(stream)
        torch.cuda.synchronize()
    total_ms = t0.elapsed_time(t1)
    f_ms = [a.elapsed_time(b) for a, b, _ in ev]
    b_ms = [b.elapsed_time(c) for _, b, c in ev]
    if world > 1:
        tt = torch.tensor([total_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        total_ms = float(tt.item())
    ms_step = total_ms / args.steps
    value = size_total / (ms_step * 1e-3) / 1e9

    # End to end through the public module API: latent copied from pinned host
    # memory, forward, backward of a device-resident upstream gradient, latent
    # gradient read back to pinned host memory.
    mod = BlockFHT(torch.nn.Parameter(z.clone()), size=size_total, layers=LAYERS, seed=SEED)
    grad_host = torch.empty(BLOCK, dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        with torch.no_grad():
            mod.latent.copy_(z_host, non_blocking=True)
        mod.latent.grad = None
        out = mod.slice(start, stop)
        out.backward(g)
        if world > 1:
            dist.all_reduce(mod.latent.grad)
        grad_host.copy_(mod.latent.grad, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        tt = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_ms = float(tt.item())

    mlp = None if args.no_mlp else measure_mlp_pair(dev, world, max(args.steps, 10), args.warmup)
    # the GPT-shaped configurations on the same line: C5 training (data parallel
    # under torchrun) and, on one GPU, C4 inference; the headline's buffers go first
    del g, y, ws, mod, grad_host
    torch.cuda.empty_cache()
    gpt = {}
    if not args.no_gpt:
        for key, fn in (("gpt2xl", lambda: measure_gpt2xl(dev, world, rank, 3, 2)),
                        ("gpt2", (lambda: measure_gpt2(dev, 10, 3)) if world == 1 else None)):
            if fn is None:
                continue
            try:
                gpt[key] = fn()
            except Exception as exc:  # reported on the line; the headline stands on its own
                gpt[key] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
                torch.cuda.empty_cache()

    if rank == 0:
        peaks = _peaks()
        fm, bm = statistics.median(f_ms), statistics.median(b_ms)
        # algorithmic HBM bytes: forward writes 2 B/coord (+ latent read); backward reads 2 B/coord.
        f_bytes = COORDS_PER_GPU * 2 + BLOCK * 2
        b_bytes = COORDS_PER_GPU * 2 + BLOCK * 2
        dom_is_f = fm >= bm
        dom_ms, dom_bytes = (fm, f_bytes) if dom_is_f else (bm, b_bytes)
        achieved = dom_bytes / (dom_ms * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": value, "unit": "Gcoords/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (latent ~N(0,1), upstream grad ~N(0,1))",
            "config": _config(world),
            "forward_gcoords_s": COORDS_PER_GPU / (fm * 1e-3) / 1e9,
            "backward_gcoords_s": COORDS_PER_GPU / (bm * 1e-3) / 1e9,
            "roofline": {"bound": "hbm", "kernel": "forward" if dom_is_f else "backward", "achieved": achieved,
                         "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                         "traffic": _traffic_from_profiles("fwd" if dom_is_f else "bwd")
                         if COORDS_PER_GPU == 1 << 28 else None,
                         "peak_source": peaks["source"], "bytes_per_launch": dom_bytes,
                         "ms_per_launch": dom_ms},
            "e2e": {"value": size_total / (e2e_ms * 1e-3) / 1e9, "unit": "Gcoords/s",
                    "h2d_bytes_per_step": BLOCK * 2, "d2h_bytes_per_step": BLOCK * 2,
                    "ms_per_step": e2e_ms, "api": "BlockFHT.slice + backward(upstream grad)"},
            "gpu_launches": (nf + nb) * args.steps,
            "clocks": clk.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_sample(host_threads())
            if mlp is not None:
                mlp["cpu_baseline"] = cpu_mlp_sample(host_threads())
        if mlp is not None:
            line["mlp_pair"] = mlp
        line.update(gpt)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


MLP_T, MLP_D, MLP_F = 8 * 1024, 768, 3072


def measure_mlp_pair(dev, world: int, steps: int, warmup: int) -> dict:
    """C3: GPT-2-small MLP pair y = W2 GELU(W1 x) (W1 [3072,768], W2 [768,3072],
    each a BlockFHTLinear with its own seed, latent 32768, layers 3, bf16),
    forward + backward to both latents and x, 8192 tokens per GPU.  Device
    time of the step replayed as one CUDA graph, then end to end through the
    public module API: x copied in from pinned host memory and the latent and
    input gradients read back every step.  Under torchrun each rank runs its
    own tokens and the latent gradients are all-reduced (data parallel)."""
    import torch
    import torch.distributed as dist

    from latent_weight_lab import BlockFHTLinear

    torch.manual_seed(0)
    up = BlockFHTLinear(MLP_D, MLP_F, latent_dim=32768, layers=3, seed=11).to(dev, torch.bfloat16)
    down = BlockFHTLinear(MLP_F, MLP_D, latent_dim=32768, layers=3, seed=12).to(dev, torch.bfloat16)
    x = torch.randn(MLP_T, MLP_D, device=dev, dtype=torch.bfloat16, requires_grad=True)
    gy = torch.randn(MLP_T, MLP_D, device=dev, dtype=torch.bfloat16)
    lat = [up.generator.latent, down.generator.latent]

    def step():
        up.generator.latent.grad = down.generator.latent.grad = x.grad = None
        down(torch.nn.functional.gelu(up(x))).backward(gy)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream(dev).wait_stream(side)
    up.generator.latent.grad = down.generator.latent.grad = x.grad = None
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        down(torch.nn.functional.gelu(up(x))).backward(gy)
    flat = torch.cat([p.grad.reshape(-1) for p in lat]) if world > 1 else None

    def dev_step():
        graph.replay()
        if world > 1:
            torch.cat([p.grad.reshape(-1) for p in lat], out=flat)
            dist.all_reduce(flat)

    def timed(fn, n):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(n):
            fn()
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / n
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    ms = timed(dev_step, steps)
    x_host = x.detach().cpu().pin_memory()
    out_host = [torch.empty(p.numel(), dtype=p.dtype).pin_memory() for p in lat] + \
        [torch.empty(x.shape, dtype=x.dtype).pin_memory()]

    def e2e_step():
        with torch.no_grad():
            x.copy_(x_host, non_blocking=True)
        step()
        if world > 1:
            for p in lat:
                dist.all_reduce(p.grad)
        for h, d in zip(out_host, [p.grad.reshape(-1) for p in lat] + [x.grad]):
            h.copy_(d, non_blocking=True)

    ms_e2e = timed(e2e_step, max(3, steps // 2))

    # the same step on the reference's training path (block_fht.py:560-569):
    # both weights generated by one grouped launch, both latent projections by
    # one grouped launch (prepare_ / flush_block_fht_weight_cache), one CUDA graph
    from latent_weight_lab import flush_block_fht_weight_cache, prepare_block_fht_weight_cache

    pair = torch.nn.ModuleList([up, down])

    def cache_step():
        prepare_block_fht_weight_cache(pair)
        down(torch.nn.functional.gelu(up(x))).backward(gy)
        flush_block_fht_weight_cache(pair)

    for _ in range(warmup):
        up.generator.latent.grad = down.generator.latent.grad = x.grad = None
        cache_step()
    torch.cuda.synchronize()
    up.generator.latent.grad = down.generator.latent.grad = x.grad = None
    graph_c = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph_c):
        cache_step()

    def cache_dev_step():
        graph_c.replay()
        if world > 1:
            torch.cat([p.grad.reshape(-1) for p in lat], out=flat)
            dist.all_reduce(flat)

    ms_cache = timed(cache_dev_step, steps)
    flops = 6.0 * 2 * MLP_D * MLP_F * MLP_T  # per GPU: fwd 2*in*out, bwd 4*in*out, two matrices
    peaks = _peaks()
    achieved = flops / (ms * 1e-3) / 1e12
    return {
        "metric": "fused BlockFHTLinear tokens/s (C3 MLP pair fwd+bwd)",
        "value": world * MLP_T / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms, "n_gpus": world,
        "config": {"workload": "C3 MLP pair 768->3072->768, 8192 tokens/GPU, latents 32768 (block 32768), layers 3",
                   "path": "weights generated by liblwl_b200 (one launch per matrix), GEMMs by cuBLAS, latent "
                           "projection by liblwl_b200; the whole step replayed as one CUDA graph",
                   "parallelism": f"data parallel x{world}" + (" (NCCL all-reduce of the latent gradients)"
                                                                 if world > 1 else "")},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": achieved / peaks["bf16_tflops"], "traffic": None, "peak_source": peaks["source"],
                     "flops_per_step": flops},
        "e2e": {"value": world * MLP_T / (ms_e2e * 1e-3), "unit": "tokens/s", "ms_per_step": ms_e2e,
                "h2d_bytes_per_step": MLP_T * MLP_D * 2,
                "d2h_bytes_per_step": 2 * 32768 * 2 + MLP_T * MLP_D * 2,
                "api": "BlockFHTLinear modules, eager (x in, latent and input gradients out)"},
        "weight_cache_path": {"value": world * MLP_T / (ms_cache * 1e-3), "unit": "tokens/s", "ms_per_step": ms_cache,
                              "tensor_frac": flops / (ms_cache * 1e-3) / 1e12 / peaks["bf16_tflops"],
                              "path": "prepare_/flush_block_fht_weight_cache around the same fwd+bwd: one grouped "
                                      "generation and one grouped latent projection per step, one CUDA graph"},
    }


def cpu_mlp_sample(threads: int, tokens: int = 512) -> dict:
    """The C3 step with the reference algorithm on host cores at reduced tokens:
    both weights generated by the oracle port (fp32, OpenMP), the GEMMs and GELU
    in numpy fp32, the latent projections by the oracle port.  tokens/s."""
    import numpy as np

    from oracle import oracle as orc

    rng = np.random.default_rng(0)
    z1 = (0.02 * rng.standard_normal(32768)).astype(np.float32)
    z2 = (0.02 * rng.standard_normal(32768)).astype(np.float32)
    x = rng.standard_normal((tokens, MLP_D)).astype(np.float32)
    gy = rng.standard_normal((tokens, MLP_D)).astype(np.float32)
    n = MLP_D * MLP_F

    def gelu(v):
        return 0.5 * v * (1.0 + np.tanh(0.7978845608 * (v + 0.044715 * v ** 3)))

    def dgelu(v):
        t = np.tanh(0.7978845608 * (v + 0.044715 * v ** 3))
        return 0.5 * (1 + t) + 0.5 * v * (1 - t * t) * 0.7978845608 * (1 + 3 * 0.044715 * v * v)

    def generate():
        w1 = orc.fht_forward(z1, n, 3, 11, 0, n, threads=threads).reshape(MLP_F, MLP_D)
        w2 = orc.fht_forward(z2, n, 3, 12, 0, n, threads=threads).reshape(MLP_D, MLP_F)
        return w1, w2

    def gemms(w1, w2):
        h = x @ w1.T
        a = gelu(h)
        gh = (gy @ w2) * dgelu(h)
        gw2 = gy.T @ a
        gw1 = gh.T @ x
        gx = gh @ w1
        return gw1, gw2, gx

    def project(gw1, gw2):
        orc.fht_backward(np.ascontiguousarray(gw1).reshape(-1), 32768, n, 3, 11, 0, n, threads=threads)
        orc.fht_backward(np.ascontiguousarray(gw2).reshape(-1), 32768, n, 3, 12, 0, n, threads=threads)

    def timed(fn, *a):
        fn(*a)
        t0, k = time.perf_counter(), 0
        while True:
            out = fn(*a)
            k += 1
            if time.perf_counter() - t0 > 2.0:
                return out, (time.perf_counter() - t0) / k

    (w1, w2), t_gen = timed(generate)
    (gw1, gw2, _), t_gemm = timed(gemms, w1, w2)
    _, t_proj = timed(project, gw1, gw2)
    # the generation and projection are per step; the GEMMs scale with tokens
    dt = t_gen + t_proj + t_gemm * (MLP_T / tokens)
    return {"value": MLP_T / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"C3 fwd+bwd timed in parts on host cores: weight generation {t_gen * 1e3:.0f} ms and latent "
                      f"projection {t_proj * 1e3:.0f} ms per step (oracle/ C port, fp32), GEMMs + GELU in numpy fp32 "
                      f"{t_gemm * 1e3:.0f} ms at {tokens} tokens, scaled to {MLP_T} tokens: {dt * 1e3:.0f} ms per step"}



def run_mlp(args) -> None:
    """C3: GPT-2-small MLP pair y = W2 GELU(W1 x) with both weights generated by
    BlockFHT (layers=3), forward + backward to both latents and x; tokens/s.

    --latent 32768 (default) gives block size 32768; --latent 65536 is the
    configuration's literal latent size (block size 65536 under the reference's
    next_pow2 rule)."""
    import torch

    from latent_weight_lab import (BlockFHTLinear, _native, flush_block_fht_weight_cache,
                                   prepare_block_fht_weight_cache)

    _native.load()
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    T, D, F4 = 8 * 1024, 768, 3072
    up = BlockFHTLinear(D, F4, latent_dim=args.latent, layers=3, seed=11).to(dev, torch.bfloat16)
    down = BlockFHTLinear(F4, D, latent_dim=args.latent, layers=3, seed=12).to(dev, torch.bfloat16)
    x = torch.randn(T, D, device=dev, dtype=torch.bfloat16, requires_grad=True)
    gy = torch.randn(T, D, device=dev, dtype=torch.bfloat16)
    pair = torch.nn.ModuleList([up, down])

    def step():
        up.generator.latent.grad = down.generator.latent.grad = x.grad = None
        if args.cache:
            # the reference's training path (block_fht.py:560-569): both weights
            # generated by one grouped launch, both latent projections by one
            prepare_block_fht_weight_cache(pair)
        y = down(torch.nn.functional.gelu(up(x)))
        y.backward(gy)
        if args.cache:
            flush_block_fht_weight_cache(pair)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    run = step
    if not args.eager:
        # the whole fwd+bwd step (generation, GEMMs, GELU, latent projections)
        # replays as one CUDA graph; gradients are unset at capture, so every
        # replay assigns fresh ones
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            step()
        torch.cuda.current_stream(dev).wait_stream(side)
        up.generator.latent.grad = down.generator.latent.grad = x.grad = None
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            if args.cache:
                prepare_block_fht_weight_cache(pair)
            y = down(torch.nn.functional.gelu(up(x)))
            y.backward(gy)
            if args.cache:
                flush_block_fht_weight_cache(pair)
        for _ in range(args.warmup):
            graph.replay()
        torch.cuda.synchronize()
        run = graph.replay
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        a.record()
        for _ in range(args.steps):
            run()
        b.record()
        torch.cuda.synchronize()
    ms = a.elapsed_time(b) / args.steps
    flops = 6 * 2 * D * F4 * T  # fwd 2*in*out + bwd 4*in*out, two matrices
    peaks = _peaks()
    achieved = flops / (ms * 1e-3) / 1e12
    line = {
        "metric": "fused BlockFHTLinear tokens/s (C3 MLP pair fwd+bwd)", "value": T / (ms * 1e-3),
        "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (x ~N(0,1), latents ~N(0,0.02))",
        "config": {"workload": f"C3 MLP pair 768->3072->768, 8192 tokens, latent {args.latent}, layers=3",
                   "path": ("weight cache: one grouped generation and one grouped latent projection per step"
                            if args.cache else "weights generated per module by liblwl_b200")
                           + ", GEMMs by cuBLAS (F.linear)",
                   "execution": "eager" if args.eager else "one CUDA graph per fwd+bwd step"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": achieved / peaks["bf16_tflops"], "traffic": None, "peak_source": peaks["source"]},
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def run_sweep(args) -> None:
    """C2 sweep: every padded block size 2^5..2^23, layers 1 and 3, bf16 and fp32,
    2^28 coordinates per call (--log-coords) (latent length = block size); forward and backward
    Gcoords/s, one JSON line per point."""
    import torch

    from latent_weight_lab import _native

    lib = _native.load()
    dev = torch.device("cuda", 0)
    N = COORDS_PER_GPU
    stream = torch.cuda.current_stream(dev).cuda_stream
    kinds = (("bf16", torch.bfloat16, _native.LWL_BF16), ("fp32", torch.float32, _native.LWL_F32))
    flags = args.sweep_flags
    for dt_name, dt, code in (k for k in kinds if k[0] in args.sweep_dtypes.split(",")):
        y = torch.empty(N, device=dev, dtype=dt)
        g = torch.randn(N, device=dev, dtype=dt)
        for layers in (1, 3):
            for k in range(args.min_log, args.max_log + 1):
                B = 1 << k
                z = torch.randn(B, device=dev, dtype=dt)
                grad = torch.empty(B, device=dev, dtype=dt)
                wsb = max(lib.lwl_fht_forward_workspace_bytes(code, B, N, layers, 0, N, flags),
                          lib.lwl_fht_backward_workspace_bytes(code, B, N, layers, 0, N, flags), 1)
                ws = torch.empty(wsb, dtype=torch.uint8, device=dev)

                def fwd():
                    assert lib.lwl_fht_forward(code, z.data_ptr(), B, N, layers, SEED, 0, N, y.data_ptr(),
                                               ws.data_ptr(), wsb, flags, stream) == 0

                def bwd():
                    assert lib.lwl_fht_backward(code, g.data_ptr(), B, N, layers, SEED, 0, N, grad.data_ptr(),
                                                ws.data_ptr(), wsb, flags, stream) == 0

                res = {}
                for name, fn in (("forward", fwd), ("backward", bwd)):
                    for _ in range(2):
                        fn()
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    reps = 3
                    a.record()
                    for _ in range(reps):
                        fn()
                    b.record()
                    torch.cuda.synchronize()
                    ms = a.elapsed_time(b) / reps
                    res[name] = N / (ms * 1e-3) / 1e9
                print(json.dumps({"sweep": "C2", "dtype": dt_name, "flags": flags, "layers": layers, "block_size": B,
                                  "coords": N, "forward_gcoords_s": res["forward"],
                                  "backward_gcoords_s": res["backward"],
                                  "forward_hbm_frac": res["forward"] * 1e9 * y.element_size() / 1e9
                                  / _peaks()["hbm_gbs"]}), flush=True)
                del ws


def run_linear(args) -> None:
    """Fused BlockFHTLinear forward (inference): y = x @ (scale * W)^T with W
    regenerated on chip by the tcgen05 kernel (lwl_linear_forward), GPT-2
    fc shape 768 -> 3072, latent 32768 (block size 32768), layers=3, bf16.
    The same public call is timed against the unfused path of the same
    function (grouped-capable generation into HBM + cuBLAS), and against the
    kernel's dense-weight variant (same MMA pipeline, W read from HBM)."""
    import torch
    import torch.nn.functional as F

    from latent_weight_lab import BlockFHTLinear, _native, block_fht_linear_forward

    _native.load()
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    T, K, N = args.tokens, 768, 3072
    layer = BlockFHTLinear(K, N, bias=False, latent_dim=32768, layers=3, seed=7).to(dev, torch.bfloat16)
    lat = layer.generator.latent.detach()
    x = torch.randn(T, K, device=dev, dtype=torch.bfloat16)

    def fused():
        return block_fht_linear_forward(x, lat, N, 3, 7)

    def unfused():
        w = _native.fht_forward(lat, K * N, 3, 7, 0, K * N).view(N, K)
        return F.linear(x, w)

    w_dense = _native.fht_forward(lat, K * N, 3, 7, 0, K * N).view(N, K)

    def dense():
        return _native.tc_linear_dense(x, w_dense)[0]

    def timed(fn, steps):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / steps

    with torch.no_grad():
        with ClockSampler(0) as clk:
            ms = timed(fused, args.steps)
        ms_unfused = timed(unfused, args.steps)
        ms_dense = timed(dense, args.steps)
        # end to end: x from pinned host memory in, y back to pinned host memory, every step
        x_host = x.cpu().pin_memory()
        y_host = torch.empty(T, N, dtype=torch.bfloat16).pin_memory()

        def e2e():
            x.copy_(x_host, non_blocking=True)
            y_host.copy_(fused(), non_blocking=True)

        ms_e2e = timed(e2e, max(3, args.steps // 4))
    flops = 2.0 * T * K * N
    peaks = _peaks()
    achieved = flops / (ms * 1e-3) / 1e12
    line = {
        "metric": "fused BlockFHTLinear forward TFLOP/s (768->3072, latent 32768, layers 3)",
        "value": achieved, "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (x ~N(0,1), latent ~N(0,0.02) reference init)",
        "config": {"workload": f"fused BlockFHTLinear forward, {T} tokens x 768 -> 3072", "tokens": T,
                   "generated_weight_bytes_in_hbm": 0,
                   "l2": "y (T x 3072 bf16) exceeds L2 for T >= 32768; x is re-read from L2 by every panel"},
        "tokens_per_s": T / (ms * 1e-3),
        "unfused_ms": ms_unfused, "unfused_tflops": flops / (ms_unfused * 1e-3) / 1e12,
        "dense_weight_variant_ms": ms_dense,
        "e2e": {"value": flops / (ms_e2e * 1e-3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": T * K * 2, "d2h_bytes_per_step": T * N * 2},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": achieved / peaks["bf16_tflops"], "traffic": None, "peak_source": peaks["source"]},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def run_mix(args) -> None:
    """FixedFHTMix (reference examples/nanogpt/model.py:200-218) on activations:
    rows x features bf16 through lwl_fixed_fht_mix; HBM-bound (one read and
    one write per element).  Default: GPT-2-small c_fc output mix, 65536
    tokens x 3072 features (P = 4096)."""
    import torch

    from latent_weight_lab import _native
    from latent_weight_lab.fht_mix import FixedFHTMix

    _native.load()
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    T, Fe = args.tokens * 2, args.features
    mix = FixedFHTMix(Fe, 98).to(dev)
    x = torch.randn(T, Fe, device=dev, dtype=torch.bfloat16)
    for _ in range(args.warmup):
        _native.fixed_fht_mix(x, mix.signs)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        a.record()
        for _ in range(args.steps):
            _native.fixed_fht_mix(x, mix.signs)
        b.record()
        torch.cuda.synchronize()
    ms = a.elapsed_time(b) / args.steps
    nbytes = 2 * T * Fe * 2
    peaks = _peaks()
    gbs = nbytes / (ms * 1e-3) / 1e9
    line = {
        "metric": "FixedFHTMix GB/s (bf16 activations, read + write)", "value": gbs, "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic x ~N(0,1)",
        "config": {"workload": f"FixedFHTMix {T} rows x {Fe} features (P = {_native_pow2(Fe)})",
                   "l2": "input and output each exceed L2"},
        "rows_per_s": T / (ms * 1e-3),
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": gbs / peaks["hbm_gbs"], "traffic": None, "peak_source": peaks["source"]},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def _native_pow2(v: int) -> int:
    return 1 << (int(v) - 1).bit_length()


def measure_gpt2xl(dev, world: int, rank: int, steps: int, warmup: int, n_layer: int = 48,
                   latent_mode: str = "ratio") -> dict:
    """C5: GPT-2-XL-shaped training step (48 layers, d=1600, 25 heads, MLP 6400,
    seq 1024, batch 32 = 32768 tokens per GPU, vocab 50257 padded to 50304)
    with every qkv / attn-proj / fc / fc-proj weight generated by BlockFHT
    (bf16, layers=3, per-matrix seeds): forward, cross-entropy on random
    targets, backward to the latents, LayerNorms and embeddings, and a fused
    AdamW step.  N GPUs: data parallel (25 heads admit no 2/4/8-way tensor
    split); the trainable state is the latents, so the only exchange is one
    NCCL all-reduce of all gradients (98 M bf16 values at ratio latents, one
    flat buffer that the gradients are views of) per step.

    --latent-mode ratio: latent = 1% of each weight (block sizes
    131072 / 32768 / 131072 / 131072); literal: 1/16 (524288 / 262144 /
    1048576 / 1048576)."""
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F

    from latent_weight_lab import BlockFHTLinear

    torch.manual_seed(0)
    d, n_head, T, Bsz, vocab = 1600, 25, 1024, 32, 50304

    def lin(i, o, seed):
        lat = max(1, round(i * o * (0.01 if latent_mode == "ratio" else 1 / 16)))
        return BlockFHTLinear(i, o, bias=True, latent_dim=lat, layers=3, seed=seed)

    class Block(torch.nn.Module):
        def __init__(self, k):
            super().__init__()
            self.ln1, self.ln2 = torch.nn.LayerNorm(d), torch.nn.LayerNorm(d)
            self.qkv, self.proj = lin(d, 3 * d, 4 * k), lin(d, d, 4 * k + 1)
            self.fc, self.fcp = lin(d, 4 * d, 4 * k + 2), lin(4 * d, d, 4 * k + 3)

        def forward(self, x):
            b, t, _ = x.shape
            q, k_, v = self.qkv(self.ln1(x)).split(d, dim=2)
            q, k_, v = (u.view(b, t, n_head, d // n_head).transpose(1, 2) for u in (q, k_, v))
            a = F.scaled_dot_product_attention(q, k_, v, is_causal=True).transpose(1, 2).reshape(b, t, d)
            x = x + self.proj(a)
            return x + self.fcp(F.gelu(self.fc(self.ln2(x))))

    class GPT(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.wte = torch.nn.Parameter(torch.randn(vocab, d) * 0.02)
            self.wpe = torch.nn.Parameter(torch.randn(T, d) * 0.01)
            self.blocks = torch.nn.ModuleList([Block(k) for k in range(n_layer)])
            self.lnf = torch.nn.LayerNorm(d)

        def forward(self, idx, tgt):
            x = self.wte[idx] + self.wpe
            for blk in self.blocks:
                x = blk(x)
            logits = F.linear(self.lnf(x), self.wte)
            return F.cross_entropy(logits.view(-1, vocab).float(), tgt.view(-1))

    model = GPT().to(dev, torch.bfloat16)
    params = [q for q in model.parameters() if q.requires_grad]
    # every gradient is a view of one flat buffer: backward accumulates into
    # it in place and the data-parallel exchange is a single in-place all-reduce
    flat_grad = torch.zeros(sum(q.numel() for q in params), device=dev, dtype=torch.bfloat16)
    off = 0
    for q in params:
        q.grad = flat_grad[off:off + q.numel()].view_as(q)
        off += q.numel()
    opt = torch.optim.AdamW(params, lr=1e-4, fused=True)
    g = torch.Generator(device="cpu").manual_seed(1234 + rank)
    idx_host = torch.randint(0, 50257, (Bsz, T), generator=g).pin_memory()
    tgt_host = torch.randint(0, 50257, (Bsz, T), generator=g).pin_memory()
    idx = torch.empty(Bsz, T, dtype=torch.long, device=dev)
    tgt = torch.empty_like(idx)
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()
    n_grad = sum(q.numel() for q in params)

    def step():
        idx.copy_(idx_host, non_blocking=True)
        tgt.copy_(tgt_host, non_blocking=True)
        flat_grad.zero_()
        loss = model(idx, tgt)
        loss.backward()
        if world > 1:
            dist.all_reduce(flat_grad)
            flat_grad.div_(world)
        opt.step()
        loss_host.copy_(loss.detach(), non_blocking=True)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clk:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a.record()
        for _ in range(steps):
            step()
        b.record()
        torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    lin_flops_tok = 6 * n_layer * (d * 3 * d + d * d + 2 * d * 4 * d)
    tokens = Bsz * T * world
    peaks = _peaks()
    achieved = tokens / world * lin_flops_tok / (ms * 1e-3) / 1e12
    out = {
        "metric": "GPT-2-XL training tokens/s, BlockFHT-generated linears (C5)",
        "value": tokens / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic token ids and targets (uniform, seed 1234 + rank), random-init weights",
        "config": {"workload": f"C5 GPT-2-XL training step, latent mode {latent_mode}", "batch": Bsz,
                   "seq_len": T, "layers": n_layer, "d_model": d, "heads": n_head, "vocab_padded": vocab,
                   "parallelism": f"dp{world} (latent-gradient all-reduce, NCCL)",
                   "step": "forward + cross-entropy + backward + gradient all-reduce + fused AdamW",
                   "trainable_params_per_rank": n_grad},
        "e2e": {"value": tokens / (ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": 2 * Bsz * T * 8,
                "d2h_bytes_per_step": 4, "note": "token ids in and the loss out are inside every timed step"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": achieved / peaks["bf16_tflops"], "traffic": None, "peak_source": peaks["source"],
                     "counted": "6 * linear FLOPs per token (fwd + grad_x + grad_W); generation, attention "
                                "and the LM head not counted"},
        "clocks": clk.summary(),
    }
    del model, opt, params, flat_grad
    torch.cuda.empty_cache()
    return out


def run_gpt2xl(args) -> None:
    """C5 on its own line (see measure_gpt2xl); under torchrun, data parallel."""
    import torch
    import torch.distributed as dist

    from latent_weight_lab import _native

    world, rank, local = _dist_env()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    _native.load()
    line = measure_gpt2xl(dev, world, rank, args.steps, args.warmup, args.xl_layers, args.latent_mode)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def measure_gpt2(dev, steps: int, warmup: int, latent_mode: str = "ratio") -> dict:
    """C4: GPT-2-small-shaped decoder inference (12 layers, d=768, 12 heads, seq 1024,
    batch 8, vocab 50257 padded to 50304) with every qkv / attn-proj / fc / fc-proj
    weight regenerated from its own BlockFHT latent on each forward (bf16, layers=3,
    per-matrix seeds).  Embeddings and LayerNorms are dense random-init; the LM head
    is tied to the token embedding.  Reports logits tokens/s on 1 GPU.

    --latent-mode ratio: latent = 1% of the weight (the reference default
    latent_ratio=0.01; block sizes 32768/8192/32768/32768); --latent-mode literal:
    latent = 1/16 of the weight (block sizes 131072/65536/262144/262144)."""
    import torch
    import torch.nn.functional as F

    from latent_weight_lab import BlockFHTLinear

    torch.manual_seed(0)
    n_layer, d, n_head, T, Bsz, vocab = 12, 768, 12, 1024, 8, 50304

    def lin(i, o, seed):
        lat = max(1, round(i * o * (0.01 if latent_mode == "ratio" else 1 / 16)))
        return BlockFHTLinear(i, o, bias=True, latent_dim=lat, layers=3, seed=seed).to(dev, torch.bfloat16)

    class Block(torch.nn.Module):
        def __init__(self, k):
            super().__init__()
            self.ln1 = torch.nn.LayerNorm(d).to(dev, torch.bfloat16)
            self.ln2 = torch.nn.LayerNorm(d).to(dev, torch.bfloat16)
            self.qkv, self.proj = lin(d, 3 * d, 4 * k), lin(d, d, 4 * k + 1)
            self.fc, self.fcp = lin(d, 4 * d, 4 * k + 2), lin(4 * d, d, 4 * k + 3)

        def forward(self, x):
            b, t, _ = x.shape
            q, k_, v = self.qkv(self.ln1(x)).split(d, dim=2)
            q, k_, v = (u.view(b, t, n_head, d // n_head).transpose(1, 2) for u in (q, k_, v))
            a = F.scaled_dot_product_attention(q, k_, v, is_causal=True).transpose(1, 2).reshape(b, t, d)
            x = x + self.proj(a)
            return x + self.fcp(F.gelu(self.fc(self.ln2(x))))

    wte = (torch.randn(vocab, d, device=dev) * 0.02).bfloat16()
    wpe = (torch.randn(T, d, device=dev) * 0.01).bfloat16()
    blocks = [Block(k) for k in range(n_layer)]
    lnf = torch.nn.LayerNorm(d).to(dev, torch.bfloat16)
    g = torch.Generator(device="cpu").manual_seed(0)
    idx_host = torch.randint(0, 50257, (Bsz, T), generator=g).pin_memory()

    model = torch.nn.ModuleList(blocks)
    from latent_weight_lab import prepare_block_fht_weight_cache

    def forward(idx):
        # every generated weight of the model in one grouped library launch, then the dense compute
        prepare_block_fht_weight_cache(model)
        x = wte[idx] + wpe
        for blk in blocks:
            x = blk(x)
        for m in model.modules():
            if hasattr(m, "_cached_weight"):
                m._cached_weight = None
        return F.linear(lnf(x), wte)

    with torch.no_grad():
        idx = idx_host.to(dev)
        for _ in range(warmup):
            forward(idx)
        torch.cuda.synchronize()
        # the whole forward (generation + dense compute) replays as one CUDA graph
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            forward(idx)
        torch.cuda.current_stream(dev).wait_stream(side)
        with torch.cuda.graph(graph):
            logits = forward(idx)
            last_dev = logits[:, -1, :].argmax(-1)
        last = torch.empty_like(last_dev, device="cpu").pin_memory()
        for _ in range(warmup):
            graph.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(dev.index) as clk:
            a.record()
            for _ in range(steps):
                idx.copy_(idx_host, non_blocking=True)  # token ids from pinned host memory
                graph.replay()
                last.copy_(last_dev, non_blocking=True)  # next-token ids read back every step
            b.record()
            torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    lin_flops = 2 * Bsz * T * n_layer * (d * 3 * d + d * d + 2 * d * 4 * d)
    line = {
        "metric": "GPT-2-small inference logits tokens/s, BlockFHT-generated linears (C4)",
        "value": Bsz * T / (ms * 1e-3), "unit": "tokens/s", "n_gpus": 1, "steps": steps,
        "warmup": warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic token ids (uniform, seed 0), random-init weights",
        "config": {"workload": f"C4 GPT-2-small inference, latent mode {latent_mode}", "batch": Bsz,
                   "seq_len": T, "layers": n_layer, "d_model": d, "vocab_padded": vocab,
                   "e2e": "token ids copied from pinned host memory and next-token argmax read back each step",
                   "execution": "one CUDA graph per forward (grouped weight generation + dense compute)"},
        "linear_tflops": lin_flops / (ms * 1e-3) / 1e12,
        "clocks": clk.summary(),
    }
    del graph, blocks, model, wte
    torch.cuda.empty_cache()
    return line


def run_gpt2(args) -> None:
    """C4 on its own line (see measure_gpt2), one GPU."""
    import torch

    from latent_weight_lab import _native

    _native.load()
    print(json.dumps(measure_gpt2(torch.device("cuda", 0), args.steps, args.warmup, args.latent_mode)), flush=True)


def run_tp(args) -> None:
    """Tensor-parallel BlockFHTLinear MLP blocks under torchrun (N GPUs, one node):
    ColumnParallelBlockFHTLinear (up-projection, output features split, each rank
    generates only its contiguous rows of W) -> GELU -> RowParallelBlockFHTLinear
    (down-projection, input features split; every rank generates all of W and keeps
    its columns; partial outputs all-reduced over NCCL).  Forward + backward to
    both latents and x, bf16, layers 3.  Strong scaling: every rank sees the same
    tokens.  Two shapes: C3 (768 -> 3072 -> 768, 8192 tokens, latents 32768) and the
    C5 MLP (1600 -> 6400 -> 1600, 32768 tokens, latents at ratio 0.01 -> block 2^17).
    Prints one JSON line per shape on rank 0."""
    import torch
    import torch.distributed as dist

    from latent_weight_lab import _native
    from latent_weight_lab.distributed import ColumnParallelBlockFHTLinear, RowParallelBlockFHTLinear

    world, rank, local = _dist_env()
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl")
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)
    _native.load()
    shapes = [("C3 MLP pair", 768, 3072, 8192, 32768), ("C5 MLP (GPT-2-XL)", 1600, 6400, 32768, 102400)]
    for name, d, f, tokens, latent in shapes:
        torch.manual_seed(0)
        up = ColumnParallelBlockFHTLinear(d, f, latent_dim=latent, layers=3, seed=21).to(dev, torch.bfloat16)
        down = RowParallelBlockFHTLinear(f, d, latent_dim=latent, layers=3, seed=22).to(dev, torch.bfloat16)
        x = torch.randn(tokens, d, device=dev, dtype=torch.bfloat16, requires_grad=True)
        gy = torch.randn(tokens, d, device=dev, dtype=torch.bfloat16)

        def step():
            up.generator.latent.grad = down.generator.latent.grad = x.grad = None
            down(torch.nn.functional.gelu(up(x))).backward(gy)

        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        # the whole step (generation, GEMMs, NCCL collectives, latent projections)
        # replayed as one CUDA graph when capture works, else eager
        run, mode, graph = step, "eager", None
        if not args.eager:
            try:
                side = torch.cuda.Stream(dev)
                side.wait_stream(torch.cuda.current_stream(dev))
                with torch.cuda.stream(side):
                    step()
                torch.cuda.current_stream(dev).wait_stream(side)
                torch.cuda.synchronize()
                up.generator.latent.grad = down.generator.latent.grad = x.grad = None
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    down(torch.nn.functional.gelu(up(x))).backward(gy)
                for _ in range(args.warmup):
                    graph.replay()
                torch.cuda.synchronize()
                run, mode = graph.replay, "one CUDA graph per step"
            except Exception as exc:  # capture unsupported here: time the eager step
                mode = f"eager (graph capture failed: {type(exc).__name__})"
                torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            run()
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / args.steps
        # the collectives of one step on their own: forward all-reduce of the
        # [tokens, d] partial output plus the two latent-gradient all-reduces
        ar_ms = 0.0
        if world > 1:
            buf = torch.randn(tokens, d, device=dev, dtype=torch.bfloat16)
            lat = torch.randn(2, latent, device=dev, dtype=torch.bfloat16)
            for _ in range(3):
                dist.all_reduce(buf)
                dist.all_reduce(lat)
            torch.cuda.synchronize()
            dist.barrier()
            c, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            c.record()
            for _ in range(args.steps):
                dist.all_reduce(buf)
                dist.all_reduce(lat)
            e.record()
            torch.cuda.synchronize()
            ar_ms = c.elapsed_time(e) / args.steps
            t = torch.tensor([ms, ar_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms, ar_ms = (float(v) for v in t.tolist())
        flops = 6.0 * 2 * d * f * tokens
        peaks = _peaks()
        achieved = flops / (ms * 1e-3) / 1e12
        rows = up.rows[1] - up.rows[0]
        gen_local = rows * d + d * f  # coordinates generated per rank per forward: own rows of W_up, all of W_down
        if rank == 0:
            print(json.dumps({
                "metric": f"tensor-parallel BlockFHTLinear tokens/s ({name} fwd+bwd)",
                "value": tokens / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic (x ~N(0,1), latents ~N(0,0.02))",
                "config": {"workload": f"{name}: {d} -> {f} -> {d}, {tokens} tokens, latents {latent}, layers 3",
                           "parallelism": f"tp{world}: column-split up-projection, row-split down-projection",
                           "execution": mode},
                "allreduce_ms_per_step": ar_ms,
                "generated_coords_per_rank": gen_local, "generated_coords_total": 2 * d * f,
                "generation_redundancy": gen_local * world / (2 * d * f),
                "roofline": {"bound": "tensor", "achieved": achieved / world, "peak": peaks["bf16_tflops"],
                             "unit": "TFLOP/s per GPU", "frac": achieved / world / peaks["bf16_tflops"],
                             "traffic": None, "peak_source": peaks["source"]},
            }), flush=True)
        run = graph = None  # release the captured graph (and its NCCL work) before the next shape
        torch.cuda.synchronize()
        del up, down, x, gy
        torch.cuda.empty_cache()
    if world > 1:
        dist.barrier()
        # a process group whose collectives were captured in CUDA graphs can
        # block in destroy_process_group; process exit releases NCCL instead
        sys.stdout.flush()
        os._exit(0)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-mlp", action="store_true", help="skip the C3 MLP-pair keys of the default line")
    ap.add_argument("--no-gpt", action="store_true", help="skip the C4 / C5 keys of the default line")
    ap.add_argument("--log-coords", type=int, default=28,
                    help="default workload: log2 of the generated coordinates per GPU (28 = the benchmark; "
                         "smaller values give the reduced cases that ncu captures run on)")
    ap.add_argument("--workload", choices=["fht", "mlp", "sweep", "gpt2", "gpt2xl", "linear", "mix", "tp"], default="fht")
    ap.add_argument("--latent-mode", choices=["ratio", "literal"], default="ratio")
    ap.add_argument("--min-log", type=int, default=5)
    ap.add_argument("--max-log", type=int, default=23)
    ap.add_argument("--sweep-dtypes", default="bf16,fp32", help="--workload sweep: comma-separated bf16,fp32")
    ap.add_argument("--sweep-flags", type=int, default=0, help="--workload sweep: transform flags (1 = LWL_FLAG_EXACT)")
    ap.add_argument("--latent", type=int, default=32768, help="latent size for --workload mlp")
    ap.add_argument("--tokens", type=int, default=32768, help="tokens for --workload linear (mix: rows / 2)")
    ap.add_argument("--features", type=int, default=3072, help="features for --workload mix")
    ap.add_argument("--xl-layers", type=int, default=48, help="layers for --workload gpt2xl")
    ap.add_argument("--eager", action="store_true", help="--workload mlp without CUDA-graph capture")
    ap.add_argument("--cache", action="store_true",
                    help="--workload mlp through prepare_/flush_block_fht_weight_cache (grouped launches)")
    args = ap.parse_args()
    global COORDS_PER_GPU
    COORDS_PER_GPU = 1 << args.log_coords
    if args.workload == "mlp":
        run_mlp(args)
    elif args.workload == "sweep":
        run_sweep(args)
    elif args.workload == "gpt2":
        run_gpt2(args)
    elif args.workload == "gpt2xl":
        run_gpt2xl(args)
    elif args.workload == "linear":
        run_linear(args)
    elif args.workload == "mix":
        run_mix(args)
    elif args.workload == "tp":
        run_tp(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
