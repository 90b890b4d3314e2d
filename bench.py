#!/usr/bin/env python3
"""GLINT hot-path benchmark on B200 (one process per GPU).

Headline: encode of a synthetic Llama-3-8B-shaped
model, 225 BF16 tensors / 7,504,658,432 weights (N(0, 0.02), 0.1% x20
outliers), blocksize 64, in GB/s of BF16 input.  Weak scaling: every rank
converts its own copy of the model (the job is N models; tensors are placed per
rank by LPT with no collective), value = BF16 bytes of all ranks / max-rank time.

Sub-results in the same JSON line: expand of the same model to BF16, decode GEMV
(configs[2]: M in {1,4,16}, K=4096/N=14336 and K=14336/N=4096) and prefill GEMM
(configs[3]: M in {512,2048,8192}, K=4096, N in {4096,14336}), each with its
roofline fraction against MEASURED_PEAKS.json.

--impl reference times the reference's CPU path (the oracle/ restatement of
glint_np.encode_f32, all host cores) on bounded samples of the same workload.
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

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

BS = 64
ENC_BYTES_PER_W = 2 + 0.5 + 0.5 + 4 / 64        # 3.0625: BF16 in, hole + plug out, absmax out
# DRAM read+write bytes per weight of encode_stream_kernel from one ncu capture of
# `bench.py --profile encode` (4 x 14336x4096 tensors, one launch): 686.1 MB for
# 234,881,024 weights; scaled to the bench's launches by their weights
ENC_DRAM_BYTES_PER_W = 2.92
EXP_BYTES_PER_W = 0.5 + 0.5 + 4 / 64 + 2        # 3.0625: planes + absmax in, BF16 out


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.is_file():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class Clocks:
    """nvidia-smi sampling during the timed region (SM clock, throttle reasons)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = Path(f"/tmp/glint_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[4:8]):
                if v.lower() in ("active", "1", "yes"):
                    reasons.add(nm)
        self.path.unlink(missing_ok=True)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_init(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
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


def max_over_ranks(world, v: float) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def synth_model(specs, seed):
    """BF16 N(0,0.02) with floor(0.001 n) entries x20 per tensor, generated on the GPU."""
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    out = []
    for s in specs:
        n = s.numel
        w = torch.empty(n, dtype=torch.bfloat16, device="cuda")
        step = 1 << 27
        for i in range(0, n, step):
            j = min(n, i + step)
            w[i:j] = (torch.randn(j - i, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
        k = n // 1000
        if k:
            idx = torch.randint(0, n, (k,), generator=g, device="cuda")
            w[idx] = (w[idx].float() * 20).to(torch.bfloat16)
        out.append(w)
    return out


def batches(items, size=32):
    return [items[i:i + size] for i in range(0, len(items), size)]


def bench_glint(args):
    import torch
    from glint_b200 import device as D
    from glint_b200 import shard

    world, rank, local = dist_init(args)
    pk = peaks()
    specs = shard.llama3_8b_tensors()
    # weak scaling: the job is `world` copies of the model, LPT-placed (each rank gets one copy's worth)
    job = [s for _ in range(world) for s in specs]
    plan = shard.lpt_assign([s.numel for s in job], world)
    mine = [job[i] for i in plan[rank]]
    weights = sum(s.numel for s in mine)
    total_weights = sum(s.numel for s in job)

    ws = synth_model(mine, seed=1234 + rank)
    planes = [D.alloc_planes(w.numel(), BS, w.device) for w in ws]
    groups = batches(list(range(len(ws))))
    torch.cuda.synchronize()

    def encode_step(events=None):
        for gi, grp in enumerate(groups):
            if events is not None:
                events[gi][0].record()
            D.encode_batch([ws[i] for i in grp], BS, outs=[planes[i] for i in grp])
            if events is not None:
                events[gi][1].record()

    for _ in range(args.warmup):
        encode_step()
    torch.cuda.synchronize()
    barrier(world)
    ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in groups]
          for _ in range(args.steps)]
    clocks = Clocks(local)
    clocks.start()
    time.sleep(0.3)  # let the sampler come up before the timed region
    torch.cuda.synchronize()
    barrier(world)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("encode_timed")  # ncu --nvtx-include "encode_timed/" selects these launches
    t0.record()
    for k in range(args.steps):
        encode_step(ev[k])
    t1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    ms_local = t0.elapsed_time(t1)
    ms = max_over_ranks(world, ms_local)
    kern_ms = sum(a.elapsed_time(b) for step in ev for (a, b) in step)
    value = total_weights * 2 / (ms / args.steps / 1e3) / 1e9
    achieved = weights * ENC_BYTES_PER_W * args.steps / (kern_ms / 1e3) / 1e9

    result = {
        "metric": "GLINT encode throughput, Llama-3-8B-shaped model (GB/s of BF16 input)",
        "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16->u4+u4+f32 (f32 arithmetic)", "data": "synthetic",
        "config": {"workload": "encode_llama3_8b (BASELINE configs[1])", "tensors_per_rank": len(mine),
                   "weights_per_rank": weights, "blocksize": BS, "parallelism": f"per-tensor LPT x{world}, no collective",
                   "l2": "inputs (15 GB per rank) far larger than L2; no flush needed"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / pk["hbm_gbs"], 4),
                     "traffic": round(weights / len(groups) * ENC_DRAM_BYTES_PER_W),
                     "traffic_note": "DRAM bytes per launch: ncu bytes/weight of the profile case x mean weights per launch",
                     "peak_source": pk["source"], "bytes_per_weight": ENC_BYTES_PER_W},
        "clocks": clk,
        "gpu_launches": args.steps * len(groups),
    }

    # ---- expand the same model back to BF16 (sub-result)
    outs = [torch.empty_like(w) for w in ws]

    def expand_step():
        for grp in groups:
            D.expand_batch([planes[i] for i in grp], [outs[i] for i in grp], BS)
    for _ in range(args.warmup):
        expand_step()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("expand_timed")
    a.record()
    for _ in range(args.steps):
        expand_step()
    b.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    ems = max_over_ranks(world, a.elapsed_time(b)) / args.steps
    eg = weights * EXP_BYTES_PER_W / (ems / 1e3) / 1e9
    result["expand"] = {"ms_per_step": round(ems, 4), "bf16_out_gbs_all_ranks": round(total_weights * 2 / (ems / 1e3) / 1e9, 2),
                        "hbm_gbs_per_gpu": round(eg, 1), "frac": round(eg / pk["hbm_gbs"], 4),
                        "bytes_per_weight": EXP_BYTES_PER_W}
    del outs

    # ---- e2e through the reference-facing host ABI (pinned host buffers, PCIe inside the timing)
    result["e2e"] = e2e_encode(ws, args, world)
    # host copies for the pin-pipeline sub-result: the 8 linears after the embedding (one
    # layer's 7 and the next q_proj, 235 M weights, 0.47 GB BF16)
    ws_pin = [(mine[i].name, mine[i].rows, mine[i].cols, ws[i].view(torch.int16).cpu().numpy())
              for i in range(1, min(len(ws), 9))] if world == 1 else []
    del ws, planes
    torch.cuda.empty_cache()

    # ---- decode GEMV and prefill GEMM (per GPU)
    result["htile"] = bench_htile(args, pk)
    # ---- column-parallel decode of a 70B layer over the ranks (NCCL all-gathers when world > 1)
    result["tp_decode"] = bench_tp_decode(args, world, rank, pk)
    # ---- plugs in host memory, streamed through the two-slot ring (one GPU's PCIe link)
    if world == 1:
        result["plug_stream"] = bench_plug_stream(pk)
        # ---- the pin pipeline: safetensors on disk -> GLINT pin files (file IO, PCIe, encode, rmse)
        try:
            result["pin_pipeline"] = bench_pin(ws_pin)
        except Exception as e:  # a sub-result; the headline stands without it
            result["pin_pipeline"] = {"error": f"{type(e).__name__}: {e}"}
        del ws_pin
    # gpu_launches counts the headline's timed region (encode); the sub-results carry their own counts
    result["expand"]["launches"] = args.steps * len(groups)
    barrier(world)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return rank, result


def bench_pin(tensors):
    """glint_b200.pin.convert of a two-shard BF16 model written to a temporary
    directory: wall clock of the second of two conversions (so the source is in the
    page cache and the pipeline's staging exists), which covers reading the shards,
    host->device and device->host copies, the GPU encode and rmse, and writing the pin;
    then glint_b200.unpin.unpin of that pin back to BF16, timed the same way."""
    import shutil
    import tempfile
    from glint_b200 import pin, st_io, unpin
    root = Path(tempfile.mkdtemp(prefix="glint_pin_bench_"))
    try:
        src = root / "src"
        src.mkdir()
        half = (len(tensors) + 1) // 2
        names = ["model-00001-of-00002.safetensors", "model-00002-of-00002.safetensors"]
        weight_map = {}
        for name, part in zip(names, (tensors[:half], tensors[half:])):
            st_io.write_file(str(src / name), [(n, "BF16", (r, c), a) for n, r, c, a in part], {"format": "pt"})
            weight_map.update({n: name for n, _r, _c, _a in part})
        (src / pin.INDEX_NAME).write_text(json.dumps({"metadata": {}, "weight_map": weight_map}))
        n_in = sum(a.nbytes for _n, _r, _c, a in tensors)
        times = []
        for k in range(2):
            out = root / f"pin{k}"
            t = time.perf_counter()
            got = pin.convert(src, out, BS)
            times.append(time.perf_counter() - t)
        out_bytes = sum(p.stat().st_size for p in (root / "pin1").iterdir())
        utimes = []
        for k in range(2):
            t = time.perf_counter()
            unpin.unpin(root / "pin1", root / f"dense{k}", "BF16")
            utimes.append(time.perf_counter() - t)
        return {"gbs_bf16_in": round(n_in / times[-1] / 1e9, 2), "seconds": round(times[-1], 3),
                "unpin_gbs_bf16_out": round(n_in / utimes[-1] / 1e9, 2), "unpin_seconds": round(utimes[-1], 3),
                "first_run_seconds": round(times[0], 3), "bf16_in_bytes": n_in, "pin_bytes": out_bytes,
                "linears": got["pin"]["n_converted"], "rmse_max": got["pin"]["rmse_max"],
                "sample": f"{len(tensors)} BF16 linears in 2 shards on local disk",
                "timing": "wall clock of convert() (and of unpin() of its pin), second of two runs each "
                          "(inputs in the page cache)"}
    finally:
        shutil.rmtree(root, ignore_errors=True)


def e2e_encode(ws, args, world):
    """glint_encode_bf16_host on pinned host copies of the first layers' tensors:
    H2D of the BF16 input and D2H of the planes are inside the timed region."""
    import torch
    from glint_b200 import glint_cuda
    L = glint_cuda.load()
    sample = ws[: min(len(ws), 1 + 7 * 4)]  # the embedding + 4 layers
    hosts = []
    for w in sample:
        n = w.numel()
        hosts.append((w.view(torch.int16).cpu().pin_memory(), torch.empty((n + 1) // 2, dtype=torch.uint8).pin_memory(),
                      torch.empty((n + 1) // 2, dtype=torch.uint8).pin_memory(),
                      torch.empty((n + BS - 1) // BS, dtype=torch.float32).pin_memory()))
    nbytes = sum(h[0].numel() * 2 for h in hosts)
    outbytes = sum(h[1].numel() * 2 + h[3].numel() * 4 for h in hosts)
    steps = max(1, min(args.steps, 3))

    def step():
        for src, h, p, a in hosts:
            rc = L.glint_encode_bf16_host(src.data_ptr(), src.numel(), BS, h.data_ptr(), p.data_ptr(), a.data_ptr())
            if rc != 0:
                raise RuntimeError(f"glint_encode_bf16_host rc={rc}")
    step()
    barrier(world)
    t = time.perf_counter()
    for _ in range(steps):
        step()
    dt = max_over_ranks(world, (time.perf_counter() - t) / steps)
    return {"value": round(nbytes * world / dt / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": nbytes,
            "d2h_bytes_per_step": outbytes, "api": "glint_encode_bf16_host (pinned host buffers)",
            "sample": f"{len(hosts)} tensors ({nbytes / 1e9:.2f} GB BF16) per rank"}


def graph_time_us(fn, n_launch: int, reps: int = 5) -> float:
    """Median device time of one launch: `n_launch` calls captured back to back in
    a CUDA graph (no host gaps inside the timed region), replayed `reps` times."""
    import torch
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):  # first calls on the capture stream allocate its workspace
        for i in range(n_launch):
            fn(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for i in range(n_launch):
                fn(i)
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ts = []
    for _ in range(reps):
        a.record()
        g.replay()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b) * 1e3 / n_launch)
    del g
    return statistics.median(ts)


def bench_htile(args, pk):
    """Decode GEMV and prefill GEMM on one GPU, fast mode.
    Every launch reads a different copy of the GLINT planes (4 copies for the
    GEMV: 250 MB > L2, so each launch streams its weights from HBM; 2 for the
    GEMM), and launches run back to back in a CUDA graph, so the numbers are
    device time with no host gaps.  The decode kernel uses programmatic
    dependent launch: in the graph a launch's weight stream starts while the
    previous one drains, as in a decode step of consecutive linears."""
    import torch
    from glint_b200 import device as D
    res = {}
    cases = [(m, 4096, 14336) for m in (1, 4, 16)] + [(m, 14336, 4096) for m in (1, 4, 16)]
    gemm = [(m, 4096, n) for m in (512, 2048, 8192) for n in (4096, 14336)]
    g = torch.Generator(device="cuda")
    g.manual_seed(7)
    launches = 0
    for (M, K, N) in cases + gemm:
        w = (torch.randn(N * K, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
        base = D.encode(w, BS)
        del w
        ncopy = 4 if M <= 16 else 2
        copies = [base] + [tuple(t.clone() for t in base) for _ in range(ncopy - 1)]
        x = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
        y = torch.empty((M, N), dtype=torch.float32, device="cuda")
        n_launch = 16 if M <= 16 else 6
        t = graph_time_us(lambda i: D.htile(x, *copies[i % ncopy], N, BS, mode="fast", out=y), n_launch) / 1e6
        launches += n_launch * (5 + 2)
        if M <= 16:
            byt = N * K * (1 + 4 / 64) + M * K * 2 + M * N * 4
            gbs = byt / t / 1e9
            res[f"gemv_m{M}_k{K}_n{N}"] = {"us": round(t * 1e6, 2), "hbm_gbs": round(gbs, 1),
                                            "frac": round(gbs / pk["hbm_gbs"], 4), "mode": "fast"}
        else:
            tf = 2.0 * M * N * K / t / 1e12
            res[f"gemm_m{M}_k{K}_n{N}"] = {"us": round(t * 1e6, 1), "tflops": round(tf, 1),
                                            "frac": round(tf / pk["bf16_tflops"], 4), "mode": "fast"}
        del copies, base, x, y
    torch.cuda.empty_cache()
    res["timing"] = ("CUDA graph of back-to-back launches over rotating plane copies; median of 5 replays; "
                     "fractions of MEASURED_PEAKS hbm_gbs / bf16_tflops")
    res["launches"] = launches
    return res


def bench_tp_decode(args, world, rank, pk, M: int = 1):
    """configs[4]-style decode step of one Llama-3-70B layer, column-parallel over
    the ranks (glint_b200/tp.py): every rank holds 1/world of each linear's packed
    rows and runs the decode kernel on them.  Where a consumer needs whole rows the
    output is gathered: with `fused`, inside the decode kernel (tp.PeerGather: each
    rank stores its rows into every rank's buffer over NVLink) for o_proj, gate/up
    (so every rank forms the whole down_proj input) and down_proj, with one NCCL
    all-gather left for the attention output that feeds o_proj; without it, NCCL
    all-gathers of the o_proj and down_proj inputs and outputs.  The layer is
    captured once in a CUDA graph (kernels and collectives), replayed, timed with
    CUDA events, max over ranks; tokens/s assumes the 80 identical layers."""
    import torch
    import torch.nn.functional as F
    from glint_b200 import device as D
    from glint_b200 import shard as SH
    from glint_b200 import tp
    g = torch.Generator(device="cuda")
    g.manual_seed(99 + rank)
    lin = {nm: (N, K) for nm, N, K in SH.LLAMA3_70B_LAYER}
    shards = {}
    local_bytes = 0
    for nm, (N, K) in lin.items():
        n0, n1 = SH.column_shard(N, world, rank)
        w = (torch.randn((n1 - n0) * K, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
        h, p, a = D.encode(w, BS)
        del w
        shards[nm] = tp.ColumnShard(n0, n1, N, K, BS, h, p, a)
        local_bytes += (n1 - n0) * K * (1 + 4 / 64)
    gx = torch.Generator(device="cuda")
    gx.manual_seed(7)  # activations replicated: the same on every rank
    x = torch.randn((M, 8192), generator=gx, device="cuda").to(torch.bfloat16)
    attn = torch.randn((M, 8192), generator=gx, device="cuda").to(torch.bfloat16)
    act_full = torch.randn((M, 28672), generator=gx, device="cuda").to(torch.bfloat16)
    pg = None
    if world > 1:
        pg = tp.PeerGather({"o": (M, 8192, torch.float32), "gate": (M, 28672, torch.float32),
                            "up": (M, 28672, torch.float32), "down": (M, 8192, torch.float32)}, world, rank)

    def layer_nccl():
        outs = []
        for nm in ("q_proj", "k_proj", "v_proj", "gate_proj", "up_proj"):
            outs.append(tp.column_parallel(x, shards[nm], world, rank, gather=False))
        if world == 1:  # nothing to gather: the seven decode calls back to back
            return outs, tp.column_parallel(attn, shards["o_proj"], 1, 0), \
                tp.column_parallel(act_full, shards["down_proj"], 1, 0)
        # o_proj: gather its input shard (the attention output), then its output
        o_in = tp.gather_columns(attn[:, shards["o_proj"].n0:shards["o_proj"].n1].float(), 8192, world, rank)
        o = tp.column_parallel(o_in.to(torch.bfloat16), shards["o_proj"], world, rank)
        # down_proj: gather the activation shard, then the output
        n0, n1 = SH.column_shard(28672, world, rank)
        d_in = tp.gather_columns(act_full[:, n0:n1].float(), 28672, world, rank)
        d = tp.column_parallel(d_in.to(torch.bfloat16), shards["down_proj"], world, rank)
        return outs, o, d

    def layer_fused():
        outs = [tp.column_parallel(x, shards[nm], world, rank, gather=False) for nm in ("q_proj", "k_proj", "v_proj")]
        o_in = tp.gather_columns(attn[:, shards["o_proj"].n0:shards["o_proj"].n1].float(), 8192, world, rank)
        o = pg.linear(o_in.to(torch.bfloat16), shards["o_proj"], "o")
        gate = pg.linear(x, shards["gate_proj"], "gate")
        up = pg.linear(x, shards["up_proj"], "up")
        act = (F.silu(gate) * up).to(torch.bfloat16)
        d = pg.linear(act, shards["down_proj"], "down")
        return outs, o, d

    def timed(layer):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(3):
                layer()
        torch.cuda.synchronize()
        barrier(world)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(gr, stream=s):
                layer()
        torch.cuda.synchronize()
        barrier(world)
        reps = 50
        for _ in range(3):
            gr.replay()
        torch.cuda.synchronize()
        barrier(world)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            gr.replay()
        b.record()
        torch.cuda.synchronize()
        us = max_over_ranks(world, a.elapsed_time(b) * 1e3 / reps)
        barrier(world)
        del gr  # graphs holding NCCL calls go before the process group does
        torch.cuda.synchronize()
        return us

    res = {"model": "Llama-3-70B layer (configs[4] shapes)", "tp": world, "batch": M,
           "weight_bytes_per_gpu_per_layer": int(local_bytes), "kernels_per_layer": 7,
           "timing": "one layer in a CUDA graph (decode kernels + gathers), replayed; max over ranks"}
    if pg is not None:
        us = timed(layer_fused)  # first: the fused layer is not measured behind the all-NCCL graph
        pg.close()
        us_nccl = timed(layer_nccl)
        res.update({"us_per_layer": round(us, 2), "gathers": "fused into o/gate/up/down decode (peer stores) + 1 NCCL",
                    "us_per_layer_nccl_gathers": round(us_nccl, 2)})
    else:
        us = timed(layer_nccl)
        res.update({"us_per_layer": round(us, 2), "gathers": "none (one GPU)"})
    from glint_b200 import glint_cuda
    res.update({"tokens_per_s_80_layers": round(M / (80 * us * 1e-6), 1),
                "hbm_frac_per_gpu": round(local_bytes / (us * 1e-6) / 1e9 / pk["hbm_gbs"], 4),
                # nonzero if any bounded wait (pipeline barrier or gather arrival) ran out
                "kernel_error": int(max_over_ranks(world, float(glint_cuda.load().glint_kernel_error(1))))})
    return res


def bench_plug_stream(pk, passes: int = 3):
    """System-RAM residency (include/glint_plug_streamer.h): a Llama-3-8B decode
    pass (32 layers x 7 linears, M = 1) with hole planes and absmax resident and
    each layer's plug planes (109 MB) streamed from pinned host memory through the
    two-slot ring while the previous layer computes.  Reported beside the same
    pass with plugs resident and a plain pinned host->device copy of one layer's
    plugs (the PCIe ceiling the streamed pass is bound by)."""
    import torch
    from glint_b200 import device as D
    from glint_b200 import shard as SH
    from glint_b200.streamer import PlugStreamer, device_bytes
    g = torch.Generator(device="cuda")
    g.manual_seed(7)
    lins = []
    off = 0
    for nm, N, K in SH.LLAMA3_8B_LAYER:
        w = (torch.randn(N * K, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
        h, p, a = D.encode(w, BS)
        del w
        lins.append((N, K, h, p, a, off))
        off += p.numel()
    layer_plug = off
    n_layers = SH.LLAMA3_8B_LAYERS
    plug_cat = torch.cat([l[3] for l in lins]).cpu()
    xs = {K: torch.randn((1, K), generator=g, device="cuda").to(torch.bfloat16) for K in (4096, 14336)}
    ys = [torch.empty((1, N), dtype=torch.float32, device="cuda") for N, *_ in lins]
    copy_s, comp_s = torch.cuda.Stream(), torch.cuda.Stream()
    copy_s.wait_stream(torch.cuda.current_stream())
    comp_s.wait_stream(torch.cuda.current_stream())
    torch.cuda.synchronize()

    def layer_calls(plug_of):
        for i, (N, K, h, p, a, o) in enumerate(lins):
            D.htile(xs[K], h, plug_of(i), a, N, BS, mode="fast", out=ys[i], stream=comp_s)

    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    # plugs resident: the same 224 decode calls
    for _ in range(2):
        for _l in range(n_layers):
            layer_calls(lambda i: lins[i][3])
    ev[0].record(comp_s)
    for _l in range(n_layers):
        layer_calls(lambda i: lins[i][3])
    ev[1].record(comp_s)
    torch.cuda.synchronize()
    resident_ms = ev[0].elapsed_time(ev[1])
    with PlugStreamer([layer_plug] * n_layers, copy_s.cuda_stream, comp_s.cuda_stream) as st:
        for l in range(n_layers):
            st.set_host_data(l, plug_cat.numpy())

        def timed_pass(compute: bool) -> float:
            st.reset_stats()
            ev[0].record(comp_s)
            if st.start() != 0:
                raise RuntimeError("plug streamer start failed")
            for l in range(n_layers):
                rc, ptr = st.acquire(l)
                if rc != 0:
                    raise RuntimeError(f"plug streamer acquire rc={rc}")
                if compute:
                    layer_calls(lambda i: device_bytes(ptr + lins[i][5], lins[i][3].numel()))
                if st.release(l) != 0:
                    raise RuntimeError("plug streamer release failed")
            ev[1].record(comp_s)
            torch.cuda.synchronize()
            return ev[0].elapsed_time(ev[1])

        # the ring's copy rate alone (no reads between acquire and release): the PCIe ceiling
        copy_ms = statistics.median([timed_pass(False) for _ in range(passes + 1)][1:])
        pass_ms = statistics.median([timed_pass(True) for _ in range(passes + 1)][1:])
        stats = st.stats()
    streamed = n_layers * layer_plug
    return {"model": "Llama-3-8B decode pass, M=1, 32 layers x 7 linears, fast mode",
            "plug_bytes_per_layer": layer_plug, "layers": n_layers,
            "pass_ms": round(pass_ms, 3), "h2d_gbs": round(streamed / (pass_ms * 1e-3) / 1e9, 2),
            "copy_only_pass_ms": round(copy_ms, 3), "copy_only_h2d_gbs": round(streamed / (copy_ms * 1e-3) / 1e9, 2),
            "frac_of_copy_only": round(copy_ms / pass_ms, 4),
            "resident_pass_ms": round(resident_ms, 3), "stall_ms_last_pass": round(stats["total_stall_ms"], 3),
            "timing": "CUDA events on the compute stream around start() .. last release, median of 3 passes"}


# ------------------------------------------------------------------ CPU baselines
_CPU_SAMPLE = None


def _cpu_sample():
    """One 4096x4096 BF16 tensor of config 2's distribution, built once per process."""
    global _CPU_SAMPLE
    if _CPU_SAMPLE is None:
        import numpy as np
        sys.path.insert(0, str(ROOT / "oracle"))
        import glint_oracle as O
        threads = O.set_threads()
        rng = np.random.default_rng(0)
        n = 4096 * 4096
        w = rng.normal(0, 0.02, n).astype(np.float32)
        w[rng.choice(n, size=n // 1000, replace=False)] *= np.float32(20)
        bits = O.f32_to_bf16(w)
        O.encode_bf16(bits, BS)  # first call: thread pool and pages warm
        _CPU_SAMPLE = (O, bits, threads)
    return _CPU_SAMPLE


def cpu_encode_sample(seconds: float = 10.0):
    """The oracle's C restatement of glint_np.encode_f32 on all host cores, over a
    bounded sample of config 2's tensors (the 4096x4096 sample encoded repeatedly
    until ~`seconds` of wall time, at least once)."""
    O, bits, threads = _cpu_sample()
    n = bits.size
    done, t0 = 0, time.perf_counter()
    while True:
        O.encode_bf16(bits, BS)
        done += n
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": round(done * 2 / dt / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{done // n} x one 4096x4096 BF16 tensor of config 2 ({done / 1e6:.0f} M weights, {dt:.1f} s)"}


def cpu_other_paths(seconds: float = 3.0):
    """The reference's host paths for the other kernels, on the same sample tensor and
    host cores: expand to BF16 (the oracle's C restatement of glint_np.expand +
    f32_to_bf16_bytes, all cores) and the host GEMV, numpy x @ W.T on the expanded
    f32 weights (numpy's BLAS threads), each repeated for about `seconds`."""
    import numpy as np
    O, bits, threads = _cpu_sample()
    n = bits.size
    ho, po, ao = O.encode_bf16(bits, BS)
    done, t0 = 0, time.perf_counter()
    while True:
        O.expand_bf16(ho, po, ao, n, BS)
        done += n
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    W = O.expand_f32(ho, po, ao, n, BS).reshape(4096, 4096)
    x = np.random.default_rng(1).normal(0, 1, (1, 4096)).astype(np.float32)
    x @ W.T
    calls, t1 = 0, time.perf_counter()
    while True:
        x @ W.T
        calls += 1
        if time.perf_counter() - t1 >= seconds:
            break
    dg = time.perf_counter() - t1
    return {"expand_bf16": {"value": round(done * 2 / dt / 1e9, 4), "unit": "GB/s of BF16 output", "cores": threads,
                            "kind": "port", "sample": f"{done // n} x the 4096x4096 sample ({dt:.1f} s)"},
            "gemv_m1": {"us_per_call": round(dg / calls * 1e6, 1), "gweights_per_s": round(n * calls / dg / 1e9, 3),
                        "kind": "numpy", "sample": f"{calls} x x[1,4096] @ W.T, W the expanded f32 4096x4096 "
                                                   f"(64 MB), numpy's BLAS threads ({dg:.1f} s)"}}


def bench_reference(args):
    """The reference arm: the CPU encode (oracle port on all host cores), W warm-up
    and K timed steps, each step a bounded sample of the workload; the whole run
    is held to about a minute of CPU work whatever K is."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    per_step = min(2.0, max(0.05, 60.0 / max(1, args.steps + args.warmup)))
    vals = []
    cb = None
    for _ in range(args.warmup):
        cpu_encode_sample(seconds=per_step)
    done, secs = 0, 0.0
    for _ in range(max(1, args.steps)):
        cb = cpu_encode_sample(seconds=per_step)
        vals.append(cb["value"])
        done += int(cb["sample"].split(" x ")[0])
        secs += float(cb["sample"].rsplit(", ", 1)[1].split(" s")[0])
    v = round(statistics.median(vals), 4)
    cb["value"] = v
    cb["sample"] = (f"{max(1, args.steps)} steps of >= {per_step:.2f} s, each encoding one 4096x4096 BF16 tensor "
                    f"of config 2 at least once ({done} tensors, {secs:.1f} s in all); value = median step")
    line = {
        "impl": "reference",
        "metric": "GLINT encode throughput, Llama-3-8B-shaped model (GB/s of BF16 input)",
        "value": v, "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16->u4+u4+f32 (f32 arithmetic)", "data": "synthetic",
        "config": {"workload": "encode_llama3_8b (BASELINE configs[1])", "blocksize": BS,
                   "what": "reference CPU encode (glint_np.encode_f32 semantics) restated in oracle/glint_oracle.c"},
        "cpu_baseline": cb,
        "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def profile_case(case: str, iters: int = 5):
    """A small, fixed workload of one kernel family for ncu captures (a few
    launches, a few hundred MB on the device, inputs larger than L2)."""
    import torch
    from glint_b200 import device as D
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    shapes = [(14336, 4096)] * 4  # 235 M weights, 470 MB BF16
    ws = [(torch.randn(r * c, generator=g, device="cuda") * 0.02).to(torch.bfloat16) for r, c in shapes]
    planes = D.encode_batch(ws, BS)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = sum(w.numel() for w in ws)
    if case == "encode":
        fn = lambda: D.encode_batch(ws, BS, outs=planes)  # noqa: E731
    elif case == "expand":
        outs = [torch.empty_like(w) for w in ws]
        fn = lambda: D.expand_batch(planes, outs, BS)  # noqa: E731
    elif case.startswith("gemm"):
        M = int(case[4:] or 2048)
        x = torch.randn((M, 4096), generator=g, device="cuda").to(torch.bfloat16)
        y = torch.empty((M, 14336), dtype=torch.float32, device="cuda")
        n = 14336 * 4096
        fn = lambda: D.htile(x, *planes[0], 14336, BS, mode="fast", out=y)  # noqa: E731
    elif case.startswith("gemvt"):
        # the down_proj shape, K = 14336, N = 4096: the same planes read as [4096, 14336]
        M = int(case[5:] or 1)
        x = torch.randn((M, 14336), generator=g, device="cuda").to(torch.bfloat16)
        y = torch.empty((M, 4096), dtype=torch.float32, device="cuda")
        n = 14336 * 4096
        fn = lambda: D.htile(x, *planes[0], 4096, BS, mode="fast", out=y)  # noqa: E731
    elif case.startswith("gemv"):
        M = int(case[4:] or 1)
        x = torch.randn((M, 4096), generator=g, device="cuda").to(torch.bfloat16)
        y = torch.empty((M, 14336), dtype=torch.float32, device="cuda")
        n = 14336 * 4096
        fn = lambda: D.htile(x, *planes[0], 14336, BS, mode="fast", out=y)  # noqa: E731
    else:
        raise SystemExit(f"unknown case {case}")
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / iters
    print(json.dumps({"case": case, "ms": round(ms, 4), "weights": n, "gweights_per_s": round(n / ms / 1e6, 2)}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="glint_b200", choices=["glint_b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", default=None, help="run one small kernel case (encode|expand|gemv<M>|gemm<M>) for ncu")
    args = ap.parse_args()
    if args.profile:
        profile_case(args.profile)
        return
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        bench_reference(args)
        return
    cb = None
    if not args.no_cpu_baseline and int(os.environ.get("RANK", "0")) == 0 and int(os.environ.get("WORLD_SIZE", "1")) == 1:
        # the CPU baseline runs first, before this process creates a CUDA context
        cb = cpu_encode_sample()
        cb["other_paths"] = cpu_other_paths()
    rank, result = bench_glint(args)
    if rank == 0:
        result["cpu_baseline"] = cb
        print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
