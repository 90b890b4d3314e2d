#!/usr/bin/env python3
"""GLINT hot-path benchmark on B200 (one process per GPU).

Headline: encode of ONE synthetic Llama-3-8B-shaped
model, 225 BF16 tensors / 7,504,658,432 weights (N(0, 0.02), exactly
floor(0.001 n) entries x20 per tensor, drawn without replacement), blocksize 64,
in GB/s of BF16 input.  The model's tensors are placed on the N ranks by LPT on
their weight counts with no collective (strong scaling: the job is one model
whatever N is); value = the model's BF16 bytes / the max-rank time of a step.  At
N > 1 a weak-scaling figure (every rank converts a whole model) is reported beside
it.

Sub-results in the same JSON line (kept short, so the whole line survives in a
driver's output tail): expand of the same tensors back to BF16 (in
roofline.others), decode GEMV and prefill GEMM on one
GPU, the reference's own H-TILE entry point at the prefill shapes, the prefill GEMM
column-parallel over the ranks with its output all-gathered, the 80-layer
Llama-3-70B decode linear stack column-parallel over the ranks at
batch 1 / 8 / 32, plug streaming and the pin pipeline (one GPU).  After each timed
region its outputs are checked against the CPU oracle (`checks`).

--impl reference times the reference's CPU path (the oracle/ restatement of
glint_np.encode_f32, all host cores) on bounded samples of the same workload, and
the reference's own CUDA kernels (built for sm_100a into oracle/_ref) on the same
B200 beside it.
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
# 234,881,024 weights; scaled to the bench's launches by their weights.  A lower
# bound: writes still dirty in L2 when the kernel ends are not counted.
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


def cpu_model() -> str:
    """The host CPU's model name (the `lscpu` model name, read from /proc/cpuinfo)."""
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.lower().startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


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


def sum_over_ranks(world, v: float) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def synth_tensor(n: int, seed: int):
    """n BF16 weights N(0, 0.02) with exactly floor(0.001 n) of them x20 (indices drawn
    without replacement), generated on the GPU from `seed` (the tensor's index in the
    model, so a tensor has the same values on whichever rank holds it)."""
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    w = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    step = 1 << 27
    for i in range(0, n, step):
        j = min(n, i + step)
        w[i:j] = (torch.randn(j - i, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    k = n // 1000
    if k:
        idx = torch.randperm(n, generator=g, device="cuda")[:k]
        w[idx] = (w[idx].float() * 20).to(torch.bfloat16)
        del idx
    return w


def batches(items, size=32):
    return [items[i:i + size] for i in range(0, len(items), size)]


def _oracle():
    """The CPU oracle (test infrastructure): only the CPU-baseline leg and the output
    checks after the timed regions load it, never a timed region."""
    if str(ROOT / "oracle") not in sys.path:
        sys.path.insert(0, str(ROOT / "oracle"))
    import glint_oracle as O
    O.set_threads()
    return O


def check_encode_expand(w, planes, out_bf16):
    """One encoded tensor's hole / plug / absmax bytes and its expanded BF16 against the
    oracle's (bit-exact)."""
    import numpy as np
    import torch
    O = _oracle()
    bits = w.view(torch.int16).cpu().numpy().view(np.uint16)
    ho, po, ao = O.encode_bf16(bits, BS)
    enc_ok = (planes[0].cpu().numpy().tobytes() == ho.tobytes() and planes[1].cpu().numpy().tobytes() == po.tobytes()
              and planes[2].cpu().numpy().tobytes() == ao.tobytes())
    exp_ok = out_bf16.view(torch.int16).cpu().numpy().tobytes() == O.expand_bf16(ho, po, ao, bits.size, BS).tobytes()
    return enc_ok, exp_ok


def check_htile_rows(x, planes, y, N, rows):
    """max |y - y_ref| / max(1, max |y_ref|) of the given y rows against the oracle's f32
    dequant-then-matmul of the same x rows."""
    import numpy as np
    import torch
    O = _oracle()
    K = x.shape[1]
    xr = x[rows].contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    ref = O.htile(planes[0].cpu().numpy(), planes[1].cpu().numpy(), planes[2].cpu().numpy(), xr, len(rows), N, K,
                  BS).astype(np.float64)
    got = y[rows].float().cpu().numpy().astype(np.float64)
    return float(np.max(np.abs(got - ref)) / max(1.0, float(np.max(np.abs(ref)))))


def time_encode(ws, planes, groups, steps, warmup, world, nvtx=None):
    """W untimed and K timed steps of the batched encode; returns (max-rank ms for the K
    steps, this rank's summed launch ms, launches per step)."""
    import torch
    from glint_b200 import device as D

    def step(events=None):
        for gi, grp in enumerate(groups):
            if events is not None:
                events[gi][0].record()
            D.encode_batch([ws[i] for i in grp], BS, outs=[planes[i] for i in grp])
            if events is not None:
                events[gi][1].record()

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in groups]
          for _ in range(steps)]
    barrier(world)
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if nvtx:
        torch.cuda.nvtx.range_push(nvtx)  # ncu --nvtx-include "encode_timed/" selects these launches
    t0.record()
    for k in range(steps):
        step(ev[k])
    t1.record()
    if nvtx:
        torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(world, t0.elapsed_time(t1))
    kern_ms = sum(a.elapsed_time(b) for st in ev for (a, b) in st)
    return ms, kern_ms, len(groups)


def bench_glint(args):
    import torch
    from glint_b200 import device as D
    from glint_b200 import shard

    world, rank, local = dist_init(args)
    pk = peaks()
    specs = shard.llama3_8b_tensors()
    total_weights = sum(s.numel for s in specs)
    # strong scaling: the job is one model; its tensors are LPT-placed over the ranks
    plan = shard.lpt_assign([s.numel for s in specs], world)
    mine = plan[rank]
    weights = sum(specs[i].numel for i in mine)
    ws = [synth_tensor(specs[i].numel, 1234 + i) for i in mine]
    planes = [D.alloc_planes(w.numel(), BS, w.device) for w in ws]
    groups = batches(list(range(len(ws))))
    torch.cuda.synchronize()

    clocks = Clocks(local)
    clocks.start()
    time.sleep(0.3)  # let the sampler come up before the timed region
    ms, kern_ms, per_step = time_encode(ws, planes, groups, args.steps, args.warmup, world, nvtx="encode_timed")
    clk = clocks.stop()
    value = total_weights * 2 / (ms / args.steps / 1e3) / 1e9
    achieved = weights * ENC_BYTES_PER_W * args.steps / (kern_ms / 1e3) / 1e9

    result = {
        "metric": "GLINT encode throughput, Llama-3-8B-shaped model (GB/s of BF16 input)",
        "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16->u4+u4+f32 (f32 arithmetic)", "data": "synthetic",
        "config": {"workload": "encode_llama3_8b (BASELINE configs[1]): one model, 225 tensors LPT-sharded over "
                               "the ranks, no collective", "weights": total_weights, "weights_rank0": weights,
                   "tensors_rank0": len(mine), "blocksize": BS, "parallelism": f"per-tensor LPT x{world}",
                   "lpt_imbalance": round(shard.imbalance([s.numel for s in specs], plan), 4),
                   "l2": "inputs (15 GB) far larger than L2; no flush needed"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / pk["hbm_gbs"], 4),
                     "traffic": round(weights / per_step * ENC_DRAM_BYTES_PER_W),
                     "traffic_note": "lower bound: ncu DRAM bytes/weight of the profile case x mean weights per "
                                     "launch; writes still dirty in L2 at kernel end are not counted",
                     "peak_source": pk["source"], "bytes_per_weight": ENC_BYTES_PER_W},
        "clocks": clk,
        "gpu_launches": args.steps * per_step,
    }

    # ---- expand the same tensors back to BF16
    outs = [torch.empty_like(w) for w in ws]

    def expand_step():
        for grp in groups:
            D.expand_batch([planes[i] for i in grp], [outs[i] for i in grp], BS)
    for _ in range(args.warmup):
        expand_step()
    torch.cuda.synchronize()
    barrier(world)
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
    result["roofline"]["others"] = {
        "expand": {"achieved": round(eg, 1), "frac": round(eg / pk["hbm_gbs"], 4), "ms_per_step": round(ems, 4),
                   "bf16_out_gbs": round(total_weights * 2 / (ems / 1e3) / 1e9, 1), "bytes_per_weight": EXP_BYTES_PER_W}}

    # ---- outputs of both timed regions against the oracle: this rank's smallest tensor
    ci = min(range(len(ws)), key=lambda i: (ws[i].numel(), i))
    enc_ok, exp_ok = check_encode_expand(ws[ci], planes[ci], outs[ci])
    bad = max_over_ranks(world, 0.0 if (enc_ok and exp_ok) else 1.0)
    checks = {"encode_expand_bits": bad == 0.0, "tensor": specs[mine[ci]].name}
    del outs

    # ---- weak scaling beside the headline (N > 1): every rank converts a whole model
    if world > 1:
        rest = [i for i in range(len(specs)) if i not in set(mine)]
        ws_all = ws + [synth_tensor(specs[i].numel, 1234 + i) for i in rest]
        planes_all = planes + [D.alloc_planes(specs[i].numel, BS, "cuda") for i in rest]
        wsteps = max(1, min(args.steps, 5))
        wms, _k, wper = time_encode(ws_all, planes_all, batches(list(range(len(ws_all)))), wsteps, 2, world)
        result["weak"] = {"value": round(world * total_weights * 2 / (wms / wsteps / 1e3) / 1e9, 2),
                          "ms_per_step": round(wms / wsteps, 4), "steps": wsteps}
        del ws_all, planes_all

    # ---- e2e through the reference-facing host ABI (pinned host buffers, PCIe inside the timing)
    result["e2e"] = e2e_encode(ws, args, world)
    # host copies for the pin-pipeline sub-result: 8 linears of one layer and the next q_proj
    ws_pin = []
    if world == 1:
        for i in range(1, min(len(ws), 9)):
            s = specs[mine[i]]
            ws_pin.append((s.name, s.rows, s.cols, ws[i].view(torch.int16).cpu().numpy()))
    del ws, planes
    torch.cuda.empty_cache()

    # ---- decode GEMV and prefill GEMM (per GPU)
    result["htile"] = bench_htile(args, pk, checks)
    # ---- the prefill GEMM column-parallel over the ranks with the output all-gathered
    result["prefill_tp"] = bench_prefill_tp(args, world, rank, pk)
    # ---- the 80-layer Llama-3-70B decode linear stack, column-parallel over the ranks
    result["decode_stack"] = bench_decode_stack(args, world, rank, pk, checks)
    if world == 1:
        # ---- K-major decode: parent-only GEMV + activation-selected plug correction
        result["kmajor"] = bench_kmajor(pk, checks)
        # ---- INT8 W8A8 GEMM with the res4 late plug, beside the reference's own kernel
        result["int8"] = bench_int8(pk, checks)
        # ---- plugs in host memory, streamed through the two-slot ring (one GPU's PCIe link)
        result["plug_stream"] = bench_plug_stream(pk)
        # ---- the pin pipeline: safetensors on disk -> GLINT pin files (file IO, PCIe, encode, rmse)
        try:
            result["pin_pipeline"] = bench_pin(ws_pin)
        except Exception as e:  # a sub-result; the headline stands without it
            result["pin_pipeline"] = {"error": f"{type(e).__name__}: {e}"}
        del ws_pin
    checks["ok"] = bool(checks["encode_expand_bits"] and checks.get("htile_max_rel_err", 1.0) <= 1e-2
                        and checks.get("int8_bits_equal_reference", True)
                        and checks.get("decode_stack_ok", True) and checks.get("kmajor_max_rel_err", 0.0) <= 3e-5)
    result["checks"] = checks
    barrier(world)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return rank, result


def e2e_encode(ws, args, world):
    """glint_encode_bf16_host on pinned host copies of up to 29 of this rank's tensors:
    the H2D of the BF16 input and the D2H of the planes are inside the timed region."""
    import torch
    from glint_b200 import glint_cuda
    L = glint_cuda.load()
    sample = ws[: min(len(ws), 29)]
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
    dt = max_over_ranks(world, time.perf_counter() - t) / steps
    tin, tout = sum_over_ranks(world, nbytes), sum_over_ranks(world, outbytes)
    return {"value": round(tin / dt / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": int(tin),
            "d2h_bytes_per_step": int(tout), "api": "glint_encode_bf16_host (pinned host buffers)",
            "sample": f"{len(hosts)} tensors on rank 0 ({nbytes / 1e9:.2f} GB BF16), all ranks' bytes counted"}


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


def bench_htile(args, pk, checks):
    """Decode GEMV (configs[2], plus M = 32 for the decode stack's batch) and prefill
    GEMM on one GPU, fast mode, and the reference's own entry point
    (launch_glint_htile_s3_f32_stream, f32-class precise arithmetic) at the prefill
    shapes.  Weights are drawn as the configs draw them (synth_tensor: N(0, 0.02) with
    0.1 % x20 outliers).  Every launch reads a different copy of the GLINT planes (4
    copies for the GEMV: 250 MB > L2, so each launch streams its weights from HBM; 2 for
    the GEMM) and launches run back to back in a CUDA graph, median of 5 replays: device
    time with no host gaps.  The decode kernels use programmatic dependent launch, so in
    the graph a launch's weight stream starts while the previous one drains, as in a
    decode step of consecutive linears.  After each shape, rows 0 and M-1 of y are
    checked against the oracle (checks.htile_max_rel_err, bound 1e-2)."""
    import torch
    from glint_b200 import device as D
    gemv = [(m, 4096, 14336) for m in (1, 4, 16, 32)] + [(m, 14336, 4096) for m in (1, 4, 16, 32)]
    gemm = [(m, 4096, n) for m in (512, 2048, 8192) for n in (4096, 14336)]
    res = {"gemv": {}, "gemm": {}, "ref_abi": {}}
    g = torch.Generator(device="cuda")
    g.manual_seed(7)
    launches, worst = 0, 0.0
    for ci, (M, K, N) in enumerate(gemv + gemm):
        base = D.encode(synth_tensor(N * K, 77 + ci), BS)
        ncopy = 4 if M <= 32 else 2
        copies = [base] + [tuple(t.clone() for t in base) for _ in range(ncopy - 1)]
        x = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
        y = torch.empty((M, N), dtype=torch.float32, device="cuda")
        n_launch = 16 if M <= 32 else 6
        t = graph_time_us(lambda i: D.htile(x, *copies[i % ncopy], N, BS, mode="fast", out=y), n_launch) / 1e6
        launches += n_launch * 6
        key = f"m{M}_k{K}_n{N}"
        if M <= 32:
            byt = N * K * (1 + 4 / 64) + M * K * 2 + M * N * 4
            res["gemv"][key] = [round(t * 1e6, 2), round(byt / t / 1e9 / pk["hbm_gbs"], 4)]
        else:
            tf = 2.0 * M * N * K / t / 1e12
            res["gemm"][key] = [round(t * 1e6, 1), round(tf, 1), round(tf / pk["bf16_tflops"], 4),
                                round(tf / pk["bf16_tflops_sustained"], 4)]
            if M == 2048 or (M == 512 and N == 4096):
                tr = graph_time_us(lambda i: D.htile_reference_abi(x, *copies[i % ncopy], N, BS, out=y), 2, reps=3) / 1e6
                launches += 2 * 4
                res["ref_abi"][key] = [round(tr * 1e6, 1), round(2.0 * M * N * K / tr / 1e12, 1)]
        D.htile(x, *copies[0], N, BS, mode="fast", out=y)
        worst = max(worst, check_htile_rows(x, copies[0], y, N, [0, M - 1]))
        del copies, base, x, y
    torch.cuda.empty_cache()
    checks["htile_max_rel_err"] = round(worst, 6)
    res["launches"] = launches
    return res


def bench_prefill_tp(args, world, rank, pk, M: int = 2048, K: int = 4096, N: int = 14336):
    """configs[3] column-parallel: every rank holds rows shard.column_shard(N, world,
    rank) of one GLINT-packed [N, K] weight (0.1 % x20 outliers), runs the fast
    prefill GEMM on them for the replicated x [M, K], and every rank ends with the
    whole row-major y [M, N] f32.  Two ways: the gather fused into the GEMM
    (tp.PeerGather: the epilogue stores each tile into every rank's y over NVLink;
    `us_step`), and the GEMM followed by NCCL all_gather_into_tensor of the f32
    shards plus the column interleave (`us_step_nccl`, with `us_gemm` and
    `us_gather_nccl` alone).  Each is a CUDA graph, replayed; device time, max over
    ranks.  At one GPU the step is the GEMM."""
    import torch
    from glint_b200 import device as D
    from glint_b200 import shard as SH
    from glint_b200 import tp
    n0, n1 = SH.column_shard(N, world, rank)
    w = synth_tensor(N * K, 9090)  # the same weight on every rank; each keeps its rows
    h, p, a = D.encode(w[n0 * K:n1 * K].contiguous(), BS)
    del w
    sh = tp.ColumnShard(n0, n1, N, K, BS, h, p, a)
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    x = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
    y_loc = torch.empty((M, n1 - n0), dtype=torch.float32, device="cuda")

    def gemm():
        D.htile(x, sh.hole, sh.plug, sh.absmax, sh.rows, BS, mode="fast", out=y_loc)

    def gather():
        return tp.gather_columns(y_loc, N, world, rank)

    def step():
        gemm()
        return gather()

    pg = tp.PeerGather({"y": (M, N, torch.float32)}, world, rank) if world > 1 else None

    def fused():
        return pg.linear(x, sh, "y", mode="fast")

    def timed(fn, reps=10):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fn()
        torch.cuda.synchronize()
        barrier(world)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(gr, stream=s):
                fn()
        gr.replay()
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            gr.replay()
        e1.record()
        torch.cuda.synchronize()
        us = max_over_ranks(world, e0.elapsed_time(e1) * 1e3 / reps)
        barrier(world)
        del gr  # graphs holding NCCL calls go before the process group does
        torch.cuda.synchronize()
        return us
    us_gemm = timed(gemm)
    if world > 1:
        us_step = timed(fused)
        us_nccl = timed(step)
        us_gather = timed(gather)
        pg.close()
    else:
        us_step = us_nccl = us_gemm
        us_gather = 0.0
    flop = 2.0 * M * N * K
    return {"shape": f"M{M} K{K} N{N}", "tp": world, "us_step": round(us_step, 1),
            "tflops_all_ranks": round(flop / (us_step * 1e-6) / 1e12, 1), "us_gemm": round(us_gemm, 1),
            "us_step_nccl": round(us_nccl, 1), "us_gather_nccl": round(us_gather, 1), "y_bytes": M * N * 4,
            "gather": "fused into the GEMM epilogue (peer stores); NCCL all-gather + interleave beside it"}


def bench_decode_stack(args, world, rank, pk, checks, batches_m=(1, 8, 32)):
    """the linear path of a decode step through all 80 layers of a
    synthetic Llama-3-70B (q/k/v/o 8192x8192 / 1024x8192, gate/up 28672x8192, down
    8192x28672; random-init BF16 N(0, 0.02), GLINT-packed: 68.4 G weights, 72.7 GB of
    planes), column-parallel over the ranks (glint_b200/tp.py; 72.7 GB / world per
    GPU).  The linears that read the same input are one weight each, as serving
    stacks store them: q|k|v (10240 x 8192) and gate|up (57344 x 8192), the same
    weights and bytes in four decode calls per layer instead of seven.  Per layer:
    q|k|v on the hidden state; o_proj on a fixed attention output (attention itself
    is not on the path); gate|up, silu(gate) * up, down_proj, whose output is the next
    layer's hidden state.  At world > 1 the outputs a consumer needs whole (o,
    gate|up, down) are gathered inside their decode kernels (tp.PeerGather: peer
    stores over NVLink), and each rank's heads of the attention output that feeds
    o_proj with the same peer-store protocol (PeerGather.gather), no NCCL call on the
    path.  The whole 80-layer step is one CUDA graph, replayed; device time
    with CUDA events, max over ranks."""
    import torch
    import torch.nn.functional as F
    from glint_b200 import device as D
    from glint_b200 import glint_cuda
    from glint_b200 import shard as SH
    from glint_b200 import tp
    L = glint_cuda.load()
    layers = SH.LLAMA3_70B_LAYERS
    dims = {nm: (N, K) for nm, N, K in SH.LLAMA3_70B_LAYER}
    hid, inter = dims["o_proj"][0], dims["gate_proj"][0]
    fused = {"qkv": (dims["q_proj"][0] + dims["k_proj"][0] + dims["v_proj"][0], hid), "o": (hid, hid),
             "gu": (2 * inter, hid), "down": (hid, inter)}
    g = torch.Generator(device="cuda")
    stack, local_bytes = [], 0
    for l in range(layers):
        lay = {}
        for j, (nm, (N, K)) in enumerate(fused.items()):
            n0, n1 = SH.column_shard(N, world, rank)
            g.manual_seed(100000 + 16 * l + j * 2 + 1000003 * rank)
            w = (torch.randn((n1 - n0) * K, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
            h, p, a = D.encode(w, BS)
            del w
            lay[nm] = tp.ColumnShard(n0, n1, N, K, BS, h, p, a)
            local_bytes += h.numel() + p.numel() + a.numel() * 4
        stack.append(lay)
    torch.cuda.synchronize()
    out = {"model": "Llama-3-70B linear stack, 80 layers, q|k|v, o, gate|up, down GLINT decode linears (configs[4])",
           "tp": world, "weight_bytes_per_gpu": int(local_bytes), "batches": {}}
    gx = torch.Generator(device="cuda")
    gx.manual_seed(7)  # activations replicated: the same on every rank
    for M in batches_m:
        x0 = torch.randn((M, hid), generator=gx, device="cuda").to(torch.bfloat16)
        attn = torch.randn((M, hid), generator=gx, device="cuda").to(torch.bfloat16)
        pg = None
        if world > 1:
            pg = tp.PeerGather({"attn": (M, hid, torch.bfloat16), "o": (M, hid, torch.float32),
                                "gu": (M, 2 * inter, torch.float32), "down": (M, hid, torch.bfloat16)}, world, rank)
        hidden = torch.empty((M, hid), dtype=torch.bfloat16, device="cuda")
        act = torch.empty((M, inter), dtype=torch.bfloat16, device="cuda")
        downs = [torch.empty((M, hid), dtype=torch.bfloat16, device="cuda") for _ in range(2)]

        def step():
            hidden.copy_(x0)
            h = hidden
            for li, lay in enumerate(stack):
                tp.column_parallel(h, lay["qkv"], world, rank, gather=False)
                if pg is None:
                    tp.column_parallel(attn, lay["o"], 1, 0)
                    gu = tp.column_parallel(h, lay["gu"], 1, 0)
                    torch.mul(F.silu(gu[:, :inter]), gu[:, inter:], out=act)  # silu(gate) * up, stored BF16
                    sd = lay["down"]
                    # down writes the next layer's BF16 hidden state itself
                    h = D.htile(act, sd.hole, sd.plug, sd.absmax, sd.rows, BS, mode="fast", out=downs[li & 1])
                else:
                    sh_o = lay["o"]
                    o_in = pg.gather(attn[:, sh_o.n0:sh_o.n1], "attn", sh_o.n0)  # this rank's heads
                    pg.linear(o_in, sh_o, "o")
                    gu = pg.linear(h, lay["gu"], "gu")
                    torch.mul(F.silu(gu[:, :inter]), gu[:, inter:], out=act)
                    h = pg.linear(act, lay["down"], "down")  # BF16, gathered: the next layer's hidden state

        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            step()  # first calls on the capture stream set up its workspaces
        torch.cuda.synchronize()
        barrier(world)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(gr, stream=s):
                step()
        torch.cuda.synchronize()
        barrier(world)
        for _ in range(2):
            gr.replay()
        torch.cuda.synchronize()
        barrier(world)
        reps = 5
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            gr.replay()
        b.record()
        torch.cuda.synchronize()
        ms = max_over_ranks(world, a.elapsed_time(b) / reps)
        barrier(world)
        del gr  # graphs holding NCCL calls go before the process group does
        torch.cuda.synchronize()
        if pg is not None:
            pg.close()
        out["batches"][str(M)] = {"ms_per_step": round(ms, 3), "tokens_per_s": round(M / (ms * 1e-3), 1),
                                  "hbm_gbs_per_gpu": round(local_bytes / (ms * 1e-3) / 1e9, 1),
                                  "hbm_frac_per_gpu": round(local_bytes / (ms * 1e-3) / 1e9 / pk["hbm_gbs"], 4)}
    kerr = int(max_over_ranks(world, float(L.glint_kernel_error(1))))
    out["kernel_error"] = kerr
    # the four decode kernels per layer, and at world > 1 the attention-output gather
    out["launches_per_step"] = layers * (len(fused) + (1 if world > 1 else 0))
    checks["decode_stack_ok"] = kerr == 0
    del stack
    torch.cuda.empty_cache()
    return out


def bench_kmajor(pk, checks, shapes=((14336, 4096), (4096, 14336)), pcts=(1, 10, 25)):
    """The K-major decode (include/glint_km.h) at configs[2]'s decode shapes, M = 1:
    the parent-only GEMV (roofline: N*K/2 hole + N*K/16 scales + 2K + 4N bytes), and
    the decode step (channel selection beside the parent GEMV, plug correction,
    closing sums) at a few selected fractions, with the plug rows in device memory
    and, at 10 %, read in place from pinned host memory.  Device time of back-to-back
    launches in a CUDA graph over 4 rotating copies (> L2).  The 10 % step's output
    is checked against the oracle's f32 restatement of the reference's sequential
    order (3e-5 normwise: each of the two sums is within 1e-5 of an f64 one)."""
    import torch
    from glint_b200 import device as D
    out = {}
    g = torch.Generator(device="cuda")
    g.manual_seed(77)
    for si, (N, K) in enumerate(shapes):
        w = synth_tensor(N * K, 4242 + si)
        h, p, a = D.encode(w, BS)
        del w
        base = D.to_kmajor(h, p, a, N, K)
        copies = [base] + [tuple(t.clone() for t in base) for _ in range(3)]
        x = torch.randn(K, generator=g, device="cuda").to(torch.bfloat16)
        y = torch.empty(N, dtype=torch.float32, device="cuda")
        idx = torch.empty(K, dtype=torch.int32, device="cuda")
        cnt = torch.empty(1, dtype=torch.int32, device="cuda")
        t = graph_time_us(lambda i: D.gemv_km(x, copies[i % 4][0], copies[i % 4][2], N, out=y), 16)
        byt = N * K / 2 + N * K / 16 + 2 * K + 4 * N
        r = {"gemv_parent_us": round(t, 2), "frac": round(byt / (t * 1e-6) / 1e9 / pk["hbm_gbs"], 4)}
        for pct in pcts:
            nsel = (pct * K + 99) // 100
            r[f"step_{pct}pct_us"] = round(graph_time_us(
                lambda i: D.gemv_select(x, copies[i % 4][0], copies[i % 4][1], copies[i % 4][2], N, nsel, out=y,
                                        idx=idx, cnt=cnt), 16), 2)
        plug_host = torch.empty(K * N // 2, dtype=torch.uint8).pin_memory()
        plug_host.copy_(base[1].cpu())
        nsel = (10 * K + 99) // 100
        r["step_10pct_host_plugs_us"] = round(graph_time_us(
            lambda i: D.gemv_select(x, copies[i % 4][0], plug_host, copies[i % 4][2], N, nsel, out=y, idx=idx,
                                    cnt=cnt), 16), 2)
        if si == 0:
            D.gemv_select(x, base[0], base[1], base[2], N, nsel, out=y, idx=idx, cnt=cnt)
            hk, pkk, sk = (t_.cpu().numpy() for t_ in base)
            xb = x.view(torch.int16).cpu().numpy().view("uint16")
            O = _oracle()
            sel = O.select_topk(xb, nsel)
            want = O.apply_corr_k(O.gemv_km(hk, sk, xb, N, K), hk, pkk, sk, xb, sel, N, K).astype("float64")
            got = y.cpu().numpy().astype("float64")
            err = float(abs(got - want).max() / max(1.0, float(abs(want).max())))
            checks["kmajor_max_rel_err"] = round(err, 9)
            checks["kmajor_selected"] = [int(cnt.item()), len(sel)]
        out[f"n{N}_k{K}"] = r
        del copies, base, h, p, a, plug_host
    torch.cuda.empty_cache()
    out["timing"] = "CUDA graph of back-to-back steps over 4 rotating copies; median of 5 replays"
    return out


def bench_int8(pk, checks, shapes=((1, 14336, 4096), (32, 14336, 4096), (2048, 14336, 4096))):
    """The INT8 W8A8 GEMM (include/int8_mma_gemm.h) at configs[2]/[3]-shaped linears
    (M x N x K), plain and with the fused res4 plug, each call including its activation
    quantization; beside it the reference's cuda/int8_mma_gemm.cu built unchanged for
    sm_100a (oracle/_ref/libp7_int8.so) on the same GPU and inputs.  Device time of
    back-to-back calls in a CUDA graph over 2 rotating weight copies; int8 TOPS =
    2 M N K / time.  The reference's outputs are compared bit for bit."""
    import ctypes
    import torch
    from glint_b200 import int8 as I8
    ref_so = ROOT / "oracle" / "_ref" / "libp7_int8.so"
    ref = I8.bind(ctypes.CDLL(str(ref_so))) if ref_so.is_file() else None
    g = torch.Generator(device="cuda")
    g.manual_seed(91)
    out, same = {}, True
    for (M, N, K) in shapes:
        x = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
        ws = [(torch.randint(-127, 128, (N, K), generator=g, device="cuda", dtype=torch.int8),
               torch.rand(N * K // 64, generator=g, device="cuda") * 2e-4 + 1e-5) for _ in range(2)]
        q4 = torch.randint(0, 256, (N * K // 2,), generator=g, device="cuda", dtype=torch.uint8)
        ps = torch.rand(N * K // 64, generator=g, device="cuda") * 2e-5
        y = torch.empty((M, N), dtype=torch.float32, device="cuda")
        sc = {}
        r = {}
        for kind, plug in (("gemm", None), ("fused", (q4, ps))):
            for who, lib in (("", None), ("ref_", ref)):
                if who and lib is None:
                    continue
                t = graph_time_us(lambda i: I8.gemm(x, ws[i % 2][0], ws[i % 2][1], plug=plug, kind=kind, out=y,
                                                    scratch=sc, lib=lib), 8)
                r[f"{who}{kind}_us"] = round(t, 2)
                r[f"{who}{kind}_tops"] = round(2.0 * M * N * K / (t * 1e-6) / 1e12, 1)
            if ref is not None:
                a, _ = I8.gemm(x, ws[0][0], ws[0][1], plug=plug, kind=kind)
                b, _ = I8.gemm(x, ws[0][0], ws[0][1], plug=plug, kind=kind, lib=ref)
                torch.cuda.synchronize()
                same = same and bool(torch.equal(a.view(torch.int32), b.view(torch.int32)))
        out[f"m{M}_n{N}_k{K}"] = r
        del ws, q4, ps, x, y, sc
    torch.cuda.empty_cache()
    if ref is not None:
        checks["int8_bits_equal_reference"] = same
    out["timing"] = "CUDA graph of back-to-back calls (quantization + GEMM) over 2 weight copies; median of 5 replays"
    return out


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
    return {"pass_ms": round(pass_ms, 3), "h2d_gbs": round(streamed / (pass_ms * 1e-3) / 1e9, 2),
            "copy_only_h2d_gbs": round(streamed / (copy_ms * 1e-3) / 1e9, 2), "resident_pass_ms": round(resident_ms, 3),
            "stall_ms": round(stats["total_stall_ms"], 3)}


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
        return {"gbs_bf16_in": round(n_in / times[-1] / 1e9, 2), "unpin_gbs_bf16_out": round(n_in / utimes[-1] / 1e9, 2),
                "first_run_s": round(times[0], 3), "linears": got["pin"]["n_converted"],
                "rmse_max": round(got["pin"]["rmse_max"], 8)}
    finally:
        shutil.rmtree(root, ignore_errors=True)


# ------------------------------------------------------------------ CPU baselines
_CPU_SAMPLE = None


def _cpu_sample():
    """One 4096x4096 BF16 tensor of config 2's distribution, built once per process."""
    global _CPU_SAMPLE
    if _CPU_SAMPLE is None:
        import numpy as np
        O = _oracle()
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
            "cpu_model": cpu_model(),
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
    return {"expand_bf16_gbs": round(done * 2 / dt / 1e9, 3), "gemv_m1_us": round(dg / calls * 1e6, 1)}


def ref_gpu_kernels():
    """The reference's own CUDA code, built unchanged for sm_100a into oracle/_ref by
    oracle/Makefile, timed on this B200: its host encode API (glint_encode_bf16_host:
    one synchronous call with its own allocations and PCIe copies, as glint_cuda.py
    calls it), its device expand (glint_expand_packed_to_f32_device) and its H-TILE
    (launch_glint_htile_s3_f32_stream) at the configs' shapes.  Device times with CUDA
    events on the launching stream, median of a few launches."""
    import ctypes
    import numpy as np
    import torch
    from glint_b200 import device as D
    O = _oracle()
    enc_so, ht_so = O.ref_lib_path("libglint_encode.so"), O.ref_lib_path("libglint_htile.so")
    if enc_so is None or ht_so is None:
        return {"unavailable": "oracle/_ref not built"}
    RE, RH = ctypes.CDLL(str(enc_so)), ctypes.CDLL(str(ht_so))
    vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    RE.glint_encode_bf16_host.argtypes = [vp, i64, i32, vp, vp, vp]
    RE.glint_expand_packed_to_f32_device.argtypes = [vp, vp, vp, i64, i32, vp, vp]
    RH.launch_glint_htile_s3_f32_stream.argtypes = [vp, vp, vp, vp, vp, i32, i32, i32, i32, vp]
    torch.cuda.set_device(0)
    out = {}
    N, K = 14336, 4096
    n = N * K
    w = synth_tensor(n, 4242)
    h, p, a = D.encode(w, BS)
    # host encode API: pinned host buffers in and out, wall clock of the synchronous call
    src = w.view(torch.int16).cpu().pin_memory()
    hh, hp = torch.empty(n // 2, dtype=torch.uint8).pin_memory(), torch.empty(n // 2, dtype=torch.uint8).pin_memory()
    ha = torch.empty(n // BS, dtype=torch.float32).pin_memory()
    ts = []
    for _ in range(3):
        t = time.perf_counter()
        rc = RE.glint_encode_bf16_host(src.data_ptr(), n, BS, hh.data_ptr(), hp.data_ptr(), ha.data_ptr())
        ts.append(time.perf_counter() - t)
        if rc != 0:
            return {"unavailable": f"reference glint_encode_bf16_host rc={rc}"}
    out["encode_host_api_gbs"] = round(n * 2 / min(ts) / 1e9, 2)
    st = torch.cuda.current_stream()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]

    def dev_us(fn, reps):
        fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(reps):
            ev[0].record()
            fn()
            ev[1].record()
            torch.cuda.synchronize()
            ts.append(ev[0].elapsed_time(ev[1]) * 1e3)
        return statistics.median(ts)

    yf = torch.empty(n, dtype=torch.float32, device="cuda")
    us = dev_us(lambda: RE.glint_expand_packed_to_f32_device(h.data_ptr(), p.data_ptr(), a.data_ptr(), n, BS,
                                                             yf.data_ptr(), ctypes.c_void_p(st.cuda_stream)), 5)
    out["expand_f32_device_gbs"] = round(n * 5.0625 / (us * 1e-6) / 1e9, 1)
    del yf
    g = torch.Generator(device="cuda")
    g.manual_seed(9)
    ht = {}
    for (M, KK, NN) in [(1, 4096, 14336), (16, 4096, 14336), (1, 14336, 4096), (512, 4096, 4096),
                        (2048, 4096, 14336)]:
        x = torch.randn((M, KK), generator=g, device="cuda").to(torch.bfloat16)
        y = torch.empty((M, NN), dtype=torch.float32, device="cuda")
        us = dev_us(lambda: RH.launch_glint_htile_s3_f32_stream(h.data_ptr(), p.data_ptr(), a.data_ptr(), x.data_ptr(),
                                                                y.data_ptr(), M, NN, KK, BS,
                                                                ctypes.c_void_p(st.cuda_stream)), 3 if M < 512 else 1)
        key = f"m{M}_k{KK}_n{NN}"
        if M <= 32:
            ht[key] = [round(us, 1), round((NN * KK * 1.0625 + M * KK * 2 + M * NN * 4) / (us * 1e-6) / 1e9, 1)]
        else:
            ht[key] = [round(us, 1), round(2.0 * M * NN * KK / (us * 1e-6) / 1e12, 2)]
    out["htile_us_and_gbs_or_tflops"] = ht
    return out


def bench_reference(args):
    """The reference arm: the CPU encode (oracle port on all host cores), W warm-up
    and K timed steps, each step a bounded sample of the workload; the whole run
    is held to about a minute of CPU work whatever K is.  Beside it, the reference's
    own CUDA kernels on this GPU (`reference_gpu`), where a GPU is present."""
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
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16->u4+u4+f32 (f32 arithmetic)", "data": "synthetic",
        "config": {"workload": "encode_llama3_8b (BASELINE configs[1]): one model, 225 tensors LPT-sharded over "
                               "the ranks, no collective", "blocksize": BS,
                   "what": "reference CPU encode (glint_np.encode_f32 semantics) restated in oracle/glint_oracle.c"},
        "cpu_baseline": cb,
        "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    try:
        import torch
        if torch.cuda.is_available():
            line["reference_gpu"] = ref_gpu_kernels()
    except Exception as e:  # informational beside the CPU line; the line stands without it
        line["reference_gpu"] = {"error": f"{type(e).__name__}: {e}"}
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
    elif case.startswith("gemmp"):
        # precise mode at prefill shapes (the reference symbols' path)
        M = int(case[5:] or 2048)
        x = torch.randn((M, 4096), generator=g, device="cuda").to(torch.bfloat16)
        y = torch.empty((M, 14336), dtype=torch.float32, device="cuda")
        n = 14336 * 4096
        fn = lambda: D.htile_reference_abi(x, *planes[0], 14336, BS, out=y)  # noqa: E731
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
    elif case in ("int8", "int8d"):
        # INT8 W8A8 GEMM on a 14336 x 4096 int8 linear: M = 2048 plain, or M = 1 with the fused plug
        from glint_b200 import int8 as I8
        N, K = 14336, 4096
        M = 2048 if case == "int8" else 1
        q = torch.randint(-127, 128, (N, K), generator=g, device="cuda", dtype=torch.int8)
        sc_w = torch.rand(N * K // 64, generator=g, device="cuda") * 2e-4 + 1e-5
        q4 = torch.randint(0, 256, (N * K // 2,), generator=g, device="cuda", dtype=torch.uint8)
        ps = torch.rand(N * K // 64, generator=g, device="cuda") * 2e-5
        x = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
        y = torch.empty((M, N), dtype=torch.float32, device="cuda")
        scr = {}
        n = N * K
        if case == "int8":
            fn = lambda: I8.gemm(x, q, sc_w, out=y, scratch=scr)  # noqa: E731
        else:
            fn = lambda: I8.gemm(x, q, sc_w, plug=(q4, ps), kind="fused", out=y, scratch=scr)  # noqa: E731
    elif case in ("km", "kmstep"):
        # K-major decode at N = 14336, K = 4096: the parent-only GEMV, or the whole
        # step at 10 % of the channels selected
        N, K = 14336, 4096
        hk, pk_, sk = D.to_kmajor(*planes[0], N, K)
        x = torch.randn(K, generator=g, device="cuda").to(torch.bfloat16)
        y = torch.empty(N, dtype=torch.float32, device="cuda")
        n = N * K
        if case == "km":
            fn = lambda: D.gemv_km(x, hk, sk, N, out=y)  # noqa: E731
        else:
            fn = lambda: D.gemv_select(x, hk, pk_, sk, N, K // 10, out=y)  # noqa: E731
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
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="glint_b200", choices=["glint_b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", default=None,
                    help="run one small kernel case (encode|expand|gemv<M>|gemvt<M>|gemm<M>|gemmp<M>|km|kmstep|int8|int8d) "
                         "for ncu")
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
        print(json.dumps(result, separators=(",", ":")), flush=True)


if __name__ == "__main__":
    main()
