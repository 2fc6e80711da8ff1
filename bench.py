"""ZipGEMM benchmark: compressed-byte HBM throughput on the Llama-3-8B decode sweep.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: the four Llama-3-8B linears, qkv 6144x4096,
o 4096x4096, gate_up 28672x4096 and down 4096x14336, weights ~N(0, 0.02) BF16
packed to TCA-TBE, activations ~N(0, 1) BF16 with N in {1, 8, 16, 32, 64, 128}
tokens. One step = the 24 fused ZipGEMM calls (4 linears x 6 token counts).
The metric: ZipGEMM HBM GB/s on compressed bytes, i.e.
algorithmic bytes (packed weight + activations + BF16 output) / time.

Timing: every call has its own device copy of its weight, so one step
streams ~1.9 GB of packed weights (inputs far larger than the 126 MB L2) and
the 24 calls run back to back with no flush between them, as consecutive
layers do in a decode step. One pair of CUDA events brackets each step;
value = total bytes / step time (max over ranks for N > 1). A separate pass
brackets every call with its own events for the per-shape table. e2e repeats
the step through the public API (runtime.linear) with the activations copied
from pinned host memory and the outputs copied back inside the timed region
(the copies run on side streams, overlapping the kernels).
cuBLAS BF16 on the dense weights is timed the same way. With --gpus N
(torchrun), every linear is split Megatron-style: qkv/gate_up by output rows
(no collective), o/down by K with an NCCL all-reduce of the BF16 partial
outputs inside the timed region.

--impl reference times the reference's CPU implementation of the path on the
same metric and config: each step runs all 24 calls of the sweep, each on a
bounded sample of its weight (the first 256 rows, packed by the reference's
own encoder built from its sources into oracle/_ref, then decoded and
multiplied in FP32 by oracle/'s restatement of the reference's CPU decoder
and GEMM, all host threads). The same sample, plus the encoder's own time,
is the `cpu_baseline` of the default line. When oracle/_ref also holds the
reference's CUDA bridge recompiled for sm_100a, the per-shape table gains
`reference_gpu_us`: the reference's own fused kernel (mma.sync, its Split-K
reduction kernel) on the same packed weights, best of split_k 1/2/4/8.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

LAYERS = (  # name, M (out features), K (in features), tensor-parallel split
    ("qkv", 6144, 4096, "col"),
    ("o", 4096, 4096, "row"),
    ("gate_up", 28672, 4096, "col"),
    ("down", 4096, 14336, "row"),
)
TOKENS = (1, 8, 16, 32, 64, 128)
METRIC = "zipgemm_hbm_gbs_compressed_llama3_8b_decode_sweep"


CPU_SAMPLE_ROWS = 256  # rows of each weight in the CPU arms' bounded sample
REF_DIR = ROOT / "oracle" / "_ref"


def _config(args, world: int) -> dict:
    """The workload description both arms print (identical by construction)."""
    return {
        "workload": "llama3-8b linears qkv/o/gate_up/down x tokens {1,8,16,32,64,128}",
        "tokens": list(args.tokens),
        "split_k": "persistent stream-K schedule, K ranges summed in-kernel (FP32)",
        "l2": "no flush: every call reads its own weight copy, ~1.9 GB packed per step "
              "(inputs larger than the 126 MB L2); calls run back to back between one "
              "pair of events per step",
        "parallelism": f"tp{world}" if world > 1 else "single",
        **({"row_parallel_sum": "o and down split on K; their outputs summed inside the "
                                "fused kernel up to 32 tokens, by the GEMM + an NCCL "
                                "all-reduce above"} if world > 1 else {}),
    }


def _reference_bridge(name: str):
    """The reference's own bridge library from oracle/_ref (built from its
    sources by oracle/Makefile), bound with this package's ABI-2 signature
    table, or None when it was not built."""
    import ctypes

    path = REF_DIR / name
    if not path.is_file():
        return None
    from zipserv_asplos26_b200 import runtime

    lib = ctypes.CDLL(str(path))
    for sym in runtime._SIGNATURES:
        if hasattr(lib, sym):
            runtime._bind(lib, sym)
    return lib if lib.zipserv_abi_version() == 2 else None


def _peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.is_file():
        data = json.loads(path.read_text())
        return {"hbm_gbs": float(data["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_id: str | None):
        self.device_id = device_id
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
               "-lms", "50"]
        if self.device_id:
            cmd += ["-i", self.device_id]
        self.started = threading.Event()
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            # The timed region starts only once nvidia-smi is producing samples.
            self.started.wait(timeout=10)
            self.lines.clear()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())
            self.started.set()

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=2)

    def summary(self) -> dict:
        sm, sm_max, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                sm_max.append(float(parts[2]))
            except ValueError:
                continue
            for name, value in zip(names, parts[5:9]):
                if value.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(sm_max),
                "reasons": sorted(reasons), "samples": len(sm)}


def _pci_id(torch, dev) -> str | None:
    try:
        p = torch.cuda.get_device_properties(dev)
        return f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
    except Exception:
        return None


def _shard(name, m, k, split, world, rank):
    if world == 1:
        return m, k, (0, m), (0, k)
    if split == "col":
        mm = m // world
        return mm, k, (rank * mm, (rank + 1) * mm), (0, k)
    kk = k // world
    return m, kk, (0, m), (rank * kk, (rank + 1) * kk)


def run_ours(args, world: int, rank: int) -> dict | None:
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F

    from zipserv_asplos26_b200 import runtime

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    runtime._cuda_library()  # fail loudly without the native library
    gen = torch.Generator().manual_seed(0)
    layers = []
    for li, (name, m, k, split) in enumerate(LAYERS):
        g = torch.Generator().manual_seed(1000 + li)
        full = (torch.randn(m, k, generator=g) * 0.02).to(torch.bfloat16)
        mm, kk, (r0, r1), (c0, c1) = _shard(name, m, k, split, world, rank)
        local = full[r0:r1, c0:c1].contiguous()
        packed = runtime.compress(local)
        layers.append({"name": name, "m": mm, "k": kk, "split": split, "packed": packed,
                       "dense": local.to(dev), "storage": packed.storage_bytes})
        del full
    # Every call gets its own device copy of its weight (packed and dense), so
    # one step streams ~1.9 GB of packed weights (~2.6 GB dense): far more
    # than the 126 MB L2. Back-to-back calls therefore read their weights
    # from HBM with no flush between them.
    calls = []
    for lay in layers:
        for n in args.tokens:
            calls.append({
                "lay": lay, "n": n, "packed": lay["packed"].to(dev), "dense": lay["dense"].clone(),
                "x": torch.randn(n, lay["k"], generator=gen).to(torch.bfloat16).to(dev),
                "out": torch.empty(n, lay["m"], dtype=torch.bfloat16, device=dev),
            })
    for lay in layers:
        del lay["packed"], lay["dense"]
    torch.cuda.empty_cache()
    stream = torch.cuda.current_stream(dev)
    need_reduce = world > 1

    def call_bytes(c):
        return c["lay"]["storage"] + 2 * c["n"] * c["lay"]["k"] + 2 * c["n"] * c["lay"]["m"]

    total_bytes = sum(call_bytes(c) for c in calls)

    # Row-parallel layers sum their outputs across ranks through
    # tp.PeerExchange: inside the fused kernel up to its token limit, else
    # the GEMM and an NCCL all-reduce. The per-shape table also times both
    # routes at every token count.
    exchange = None
    if need_reduce:
        from zipserv_asplos26_b200 import tp as tpmod

        exchange = tpmod.PeerExchange(max(l["m"] for l in layers if l["split"] == "row"),
                                      max(args.tokens), device=dev)

    def zip_call(c):
        if need_reduce and c["lay"]["split"] == "row":
            return exchange.linear(c["x"], c["packed"], out=c["out"])
        return runtime.linear_kparts(c["x"], c["packed"], 0, out=c["out"])

    def fused_call(c):
        if need_reduce and c["lay"]["split"] == "row":
            return exchange.linear(c["x"], c["packed"], out=c["out"], fused=True)
        return runtime.linear_kparts(c["x"], c["packed"], 0, out=c["out"])

    def zip_nccl_call(c):
        y = runtime.linear_kparts(c["x"], c["packed"], 0, out=c["out"])
        if need_reduce and c["lay"]["split"] == "row":
            dist.all_reduce(y)
        return y

    def dense_call(c):
        y = F.linear(c["x"], c["dense"])
        if need_reduce and c["lay"]["split"] == "row":
            dist.all_reduce(y)
        return y

    align = torch.zeros(1, device=dev)

    def settle():
        """Keep the GPU busy while the host enqueues the step (so the timed
        region measures the device, not host launch latency); with several
        ranks, end with a tiny all-reduce so every rank's timed region starts
        together instead of absorbing the other ranks' enqueue skew."""
        torch.cuda._sleep(8_000_000)
        if world > 1:
            dist.all_reduce(align)

    def timed_step(fn) -> float:
        """One step (every call once, back to back) between two events."""
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        settle()
        start.record(stream)
        for c in calls:
            fn(c)
        end.record(stream)
        torch.cuda.synchronize(dev)
        return start.elapsed_time(end)

    def per_call_pass(fn, per_call: dict) -> None:
        """Every call between its own pair of events (for the per-shape table)."""
        events = []
        settle()
        for c in calls:
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            fn(c)
            e.record(stream)
            events.append((c, s, e))
        torch.cuda.synchronize(dev)
        for c, s, e in events:
            per_call.setdefault((c["lay"]["name"], c["n"]), []).append(s.elapsed_time(e))

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    # Warm-up (also primes the planner and tensor-map encoder).
    for _ in range(args.warmup):
        timed_step(zip_call)
        timed_step(dense_call)
    barrier()
    sampler = ClockSampler(_pci_id(torch, dev) if rank == 0 else None)
    wall0 = time.time()
    with sampler if rank == 0 else _Null():
        barrier()
        zip_ms = [timed_step(zip_call) for _ in range(args.steps)]
        barrier()
    wall = time.time() - wall0
    dense_ms = [timed_step(dense_call) for _ in range(args.steps)]
    barrier()
    per_call: dict = {}
    dense_per_call: dict = {}
    nccl_per_call: dict = {}
    fused_per_call: dict = {}
    for _ in range(max(3, min(args.steps, 10))):
        per_call_pass(zip_call, per_call)
        per_call_pass(dense_call, dense_per_call)
        if need_reduce:
            per_call_pass(zip_nccl_call, nccl_per_call)
            per_call_pass(fused_call, fused_per_call)
    barrier()
    ref_gpu, ref_gpu_note = (_reference_gpu_per_call(calls, stream, dev, settle)
                             if world == 1 else ({}, "single-GPU runs only"))

    # End to end through the public API: H2D of activations, GEMM, D2H of
    # outputs, every step. The step's input copies run on one side stream and
    # the outputs are read back on another as soon as their GEMMs are done (in
    # groups of calls), so the PCIe transfers overlap the kernels; the step
    # ends when the last output has reached the host.
    host_x = [c["x"].cpu().pin_memory() for c in calls]
    host_y = [torch.empty(c["out"].shape, dtype=c["out"].dtype).pin_memory() for c in calls]
    dev_x = [torch.empty_like(c["x"]) for c in calls]
    h2d = sum(x.numel() * 2 for x in host_x)
    d2h = sum(y.numel() * 2 for y in host_y)
    copy_in = torch.cuda.Stream(dev)
    copy_out = torch.cuda.Stream(dev)

    group = 4  # calls per input wait and per output read-back (measured best of 1, 4, 6, 24)

    def e2e_step() -> float:
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        settle()
        start.record(stream)
        copy_in.wait_stream(stream)
        landed = []
        with torch.cuda.stream(copy_in):
            for i in range(len(calls)):
                dev_x[i].copy_(host_x[i], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(copy_in)
                landed.append(ev)
        pending = []
        for i, c in enumerate(calls):
            if i % group == 0:  # this group's inputs are on the device
                stream.wait_event(landed[min(len(calls), i + group) - 1])
            if need_reduce and c["lay"]["split"] == "row":
                y = exchange.linear(dev_x[i], c["packed"])
            else:
                y = runtime.linear(dev_x[i], c["packed"])
            pending.append((i, y))
            if len(pending) == group or i == len(calls) - 1:
                done = torch.cuda.Event()
                done.record(stream)
                copy_out.wait_event(done)
                with torch.cuda.stream(copy_out):
                    for j, yj in pending:
                        host_y[j].copy_(yj, non_blocking=True)
                        yj.record_stream(copy_out)
                pending = []
        stream.wait_stream(copy_out)
        end.record(stream)
        torch.cuda.synchronize(dev)
        return start.elapsed_time(end)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    barrier()
    e2e_ms = [e2e_step() for _ in range(args.steps)]
    barrier()
    # The outputs read back are the GEMM results (the kernel is deterministic).
    if not need_reduce:
        for i, c in enumerate(calls):
            if not torch.equal(host_y[i], runtime.linear(dev_x[i], c["packed"]).cpu()):
                raise SystemExit(f"e2e output {i} differs from the device result")

    def agg(values):
        t = torch.tensor([sum(values)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # A kernel wait that gave up (bounded waits raise a device flag) makes the
    # numbers meaningless: fail loudly instead of printing them.
    flags = runtime.device_flags()
    if flags:
        raise SystemExit(f"device failure flags {flags:#x} set during the benchmark")
    zip_total, dense_total, e2e_total = agg(zip_ms), agg(dense_ms), agg(e2e_ms)
    bytes_all = torch.tensor([float(total_bytes)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(bytes_all)
    step_bytes = float(bytes_all.item())
    extras = {}
    if exchange is not None:
        exchange.close()
    if not args.no_extras:
        # Every rank takes part (the extras' collectives and max-over-ranks).
        for c in calls:  # free the sweep's device copies (shapes and sizes stay)
            for key in ("packed", "dense", "x", "out"):
                c.pop(key, None)
        torch.cuda.empty_cache()
        extras["llama70b_tp"] = tp70b_case(args, world, rank, dev)
        extras["decode_step"] = decode_step_case(args, world, rank, dev)
    if rank != 0:
        return None
    steps = args.steps
    value = step_bytes * steps / (zip_total * 1e-3) / 1e9
    peaks = _peaks()
    per_shape = []
    ours_sum = ref_sum = 0.0
    for c in calls:
        lay, n = c["lay"], c["n"]
        key = (lay["name"], n)
        us = statistics.median(per_call[key]) * 1e3
        dus = statistics.median(dense_per_call[key]) * 1e3
        row = {"layer": lay["name"], "m": lay["m"], "k": lay["k"], "n": n,
               "zipgemm_us": round(us, 2), "cublas_bf16_us": round(dus, 2),
               "gbs": round(call_bytes(c) / (us * 1e-6) / 1e9, 1),
               "speedup_vs_cublas": round(dus / us, 3)}
        if key in nccl_per_call and lay["split"] == "row":
            row["zipgemm_then_nccl_allreduce_us"] = round(
                statistics.median(nccl_per_call[key]) * 1e3, 2)
            row["fused_allreduce_us"] = round(statistics.median(fused_per_call[key]) * 1e3, 2)
        if key in ref_gpu:
            rus, rsplit = ref_gpu[key]
            row.update({"reference_gpu_us": round(rus, 2), "reference_split_k": rsplit,
                        "speedup_vs_reference_gpu": round(rus / us, 3)})
            ours_sum += us
            ref_sum += rus
        per_shape.append(row)
    traffic = _traffic_record()
    launches = len(calls) * steps
    # Per GPU: every rank launches the same calls on its own shards.
    avg_launch_bytes = step_bytes / world / len(calls)
    per_gpu = value / world
    line = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": args.warmup,
        "ms_per_step": round(zip_total / steps, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)",
        "config": _config(args, world),
        "bytes_per_step": int(step_bytes),
        "roofline": {
            "bound": "hbm",
            "achieved": round(per_gpu, 1),
            "peak": peaks["hbm_gbs"],
            "unit": "GB/s",
            "frac": round(per_gpu / peaks["hbm_gbs"], 4),
            "per": "one GPU (the job's algorithmic bytes per GPU over the step time)",
            "peak_source": peaks["source"],
            "traffic": (round(traffic["ratio"] * avg_launch_bytes)
                        if traffic.get("ratio") else None),
            "algorithmic_bytes_per_launch": round(avg_launch_bytes),
            "traffic_note": traffic.get("note"),
        },
        "cublas_bf16": {
            "ms_per_step": round(dense_total / steps, 4),
            "zipgemm_speedup": round(dense_total / zip_total, 3),
        },
        "reference_gpu": ({
            "what": "the reference's fused kernel (csrc/L_Kernel.cuh via its CUDA bridge, "
                    "recompiled for sm_100a) on the same packed weights, best split_k per call",
            "sum_of_calls_us": round(ref_sum, 1),
            "zipgemm_sum_of_calls_us": round(ours_sum, 1),
            "zipgemm_speedup": round(ref_sum / ours_sum, 3),
        } if ref_gpu else {"unavailable": ref_gpu_note}),
        "e2e": {
            "value": round(step_bytes * steps / (e2e_total * 1e-3) / 1e9, 1),
            "unit": "GB/s",
            "ms_per_step": round(e2e_total / steps, 4),
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
        },
        "gpu_launches": launches,
        "wall_s_timed_region": round(wall, 3),
        "per_shape": per_shape,
    }
    line["clocks"] = sampler.summary()
    line.update(extras)
    if args.stress and rank == 0:
        line["stress"] = stress_case(args)
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args)
    return line


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


def _traffic_record() -> dict:
    """DRAM bytes / algorithmic bytes of one ncu-captured ZipGEMM launch
    (profiles/zipgemm_gate_up16_traffic.txt, ``key: value`` lines: the
    largest bench shape, whose packed weight exceeds L2)."""
    path = ROOT / "profiles" / "zipgemm_gate_up16_traffic.txt"
    rec = {}
    if path.is_file():
        for line in path.read_text().splitlines():
            key, sep, value = line.partition(":")
            if sep:
                rec[key.strip()] = value.strip()
    try:
        ratio = float(rec["dram_bytes_per_launch"]) / float(rec["algorithmic_bytes_per_launch"])
    except (KeyError, ValueError, ZeroDivisionError):
        return {"ratio": None, "note": "no ncu capture recorded"}
    return {"ratio": ratio,
            "note": f"dram__bytes_read+write / algorithmic bytes = {ratio:.4f} on "
                    f"{rec.get('launch', 'one launch')}; scaled to the average launch"}


def _reference_gpu_per_call(calls, stream, dev, settle) -> tuple[dict, str]:
    """Per-call device time of the reference's own fused kernel on the same
    packed weights: {(layer, n): (best us, its split_k)}. Every split_k in
    {1, 2, 4, 8} that divides K/64 is timed in passes over all calls back to
    back (each call reading its own weight copy, as in the other per-call
    passes); the reference's outputs are checked against ours."""
    import torch

    from zipserv_asplos26_b200 import runtime

    lib = _reference_bridge("libzipserv_ref_cuda.so")
    if lib is None or not hasattr(lib, "zipserv_mm"):
        return {}, "the reference CUDA bridge is not built (make -C oracle ref-cuda REF=<reference checkout>)"
    ws = torch.empty(max(8 * c["n"] * c["lay"]["m"] for c in calls), dtype=torch.bfloat16,
                     device=dev)
    outs = [torch.empty_like(c["out"]) for c in calls]
    handle = stream.cuda_stream

    def launch(i, c, split):
        pk = c["packed"]
        status = lib.zipserv_mm(handle, *(b.data_ptr() for b in pk.buffers), pk.max_common,
                                pk.max_rare, pk.start_exp, c["x"].data_ptr(), outs[i].data_ptr(),
                                c["lay"]["m"], c["n"], c["lay"]["k"],
                                ws.data_ptr() if split > 1 else None, split)
        if status:
            raise SystemExit(f"reference zipserv_mm failed ({status}) on {c['lay']['name']}")

    times: dict = {}
    for split in (1, 2, 4, 8):
        todo = [(i, c) for i, c in enumerate(calls) if (c["lay"]["k"] // 64) % split == 0]
        for i, c in todo:  # warm-up
            launch(i, c, split)
        for _ in range(3):
            events = []
            settle()
            for i, c in todo:
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record(stream)
                launch(i, c, split)
                e.record(stream)
                events.append((c, s, e))
            torch.cuda.synchronize(dev)
            for c, s, e in events:
                times.setdefault((c["lay"]["name"], c["n"], split), []).append(s.elapsed_time(e))
        # The reference's result must agree with ours (FP32 sums, BF16 output).
        for i, c in todo:
            ours = runtime.linear_kparts(c["x"], c["packed"], 0).float()
            err = (outs[i].float() - ours).abs().max().item() / max(ours.abs().max().item(), 1e-30)
            if err > 2e-2:
                raise SystemExit(f"reference kernel disagrees on {c['lay']['name']} n={c['n']}")
    best = {}
    for (name, n, split), ts in times.items():
        us = statistics.median(ts) * 1e3
        if (name, n) not in best or us < best[(name, n)][0]:
            best[(name, n)] = (us, split)
    return best, ""


def _cpu_sweep(args, threads: int):
    """The sweep's bounded CPU sample: for every layer the first
    CPU_SAMPLE_ROWS rows of its weight, packed by the reference's own encoder
    (oracle/_ref; the oracle restatement when it was not built here), and for
    every token count one decode + FP32 GEMM of that sample (oracle/, the
    restated reference CPU decoder and GEMM loop). Returns (run_step,
    bytes_per_step, pack_seconds, pack_kind)."""
    import ctypes

    import numpy as np
    import torch

    from oracle import oracle
    from zipserv_asplos26_b200 import runtime

    ref = _reference_bridge("libzipserv_ref_cpu.so")
    samples, pack_s = [], 0.0
    for li, (name, m, k, _split) in enumerate(LAYERS):
        g = torch.Generator().manual_seed(1000 + li)
        full = (torch.randn(m, k, generator=g) * 0.02).to(torch.bfloat16)
        w = full[:CPU_SAMPLE_ROWS].contiguous().view(torch.int16).numpy().view(np.uint16)
        del full
        t0 = time.perf_counter()
        if ref is not None:
            desc = runtime._Descriptor()
            runtime._check(0 if ref.zipserv_compress(w.ctypes.data, w.shape[0], k,
                                                     ctypes.byref(desc)) == 0 else -1)
            bufs = [np.ctypeslib.as_array(ctypes.cast(desc.buffers[i], ctypes.POINTER(
                ctypes.c_uint8)), shape=(int(desc.lengths[i]),)).copy() if desc.lengths[i]
                else np.zeros(0, np.uint8) for i in range(7)]
            start_exp = desc.start_exp
            ref.zipserv_free(ctypes.byref(desc))
        else:
            packed = oracle.pack(w)
            bufs, start_exp = packed.abi_buffers(), packed.start_exp
        pack_s += time.perf_counter() - t0
        for n in args.tokens:
            x = torch.randn(n, k, generator=torch.Generator().manual_seed(7 + n)).to(
                torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
            nbytes = sum(b.nbytes for b in bufs) + 2 * n * k + 2 * n * w.shape[0]
            samples.append((bufs, w.shape[0], k, start_exp, x, nbytes))

    def run_step():
        for bufs, m, k, start_exp, x, _ in samples:
            dec = oracle.decode(bufs, m, k, start_exp, threads=threads)
            oracle.gemm(dec, x, threads=threads)

    kind = "reference" if ref is not None else "port"
    return run_step, sum(s[-1] for s in samples), pack_s, kind


def _sample_text(pack_kind: str) -> str:
    packer = ("the reference's own encoder built from its sources (oracle/_ref)"
              if pack_kind == "reference" else "the oracle restatement of the encoder")
    return (f"per step all 24 calls of the sweep, each on the first {CPU_SAMPLE_ROWS} rows of "
            f"its weight: packed once by {packer}, then decoded and multiplied in FP32 by "
            f"oracle/'s restatement of the reference CPU decoder and GEMM loop")


def cpu_baseline(args) -> dict:
    threads = os.cpu_count() or 1
    run_step, nbytes, pack_s, pack_kind = _cpu_sweep(args, threads)
    run_step()
    t0 = time.perf_counter()
    reps = 0
    while reps < 2 or time.perf_counter() - t0 < 10.0:
        run_step()
        reps += 1
        if time.perf_counter() - t0 > 30.0:
            break
    dt = time.perf_counter() - t0
    sample_weights = CPU_SAMPLE_ROWS * sum(lay[2] for lay in LAYERS)
    return {"value": round(nbytes * reps / dt / 1e9, 3), "unit": "GB/s", "cores": threads,
            "kind": "port",
            "pack": {"kind": pack_kind, "seconds_for_4_samples": round(pack_s, 4),
                     "weights_per_s": round(sample_weights / pack_s, 1)},
            "sample": _sample_text(pack_kind) + f"; {reps} steps in {dt:.1f} s"}


def run_reference(args, world: int, rank: int) -> dict | None:
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    run_step, nbytes, pack_s, pack_kind = _cpu_sweep(args, threads)
    for _ in range(args.warmup):
        run_step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        run_step()
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = nbytes * len(times) / total / 1e9
    return {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total / len(times) * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)",
        "impl": "reference",
        "config": _config(args, world),
        "bytes_per_step": nbytes,
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads,
                         "kind": "port",
                         "pack": {"kind": pack_kind, "seconds_for_4_samples": round(pack_s, 4)},
                         "sample": _sample_text(pack_kind)},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def decode_step_case(args, world: int, rank: int, dev) -> dict:
    """The Llama-3-8B decode step: one greedy decode step of a random-init
    Llama-3-8B (32 layers, 2048 cached positions per sequence, untied
    compressed lm_head) at TP = world, every linear through ZipGEMM, against
    the same step with the dense BF16 weights (cuBLAS). Each step is a CUDA
    graph replay (NCCL all-reduces of o and down inside it); the time is the
    max over ranks of the median of per-replay CUDA events."""
    import torch
    import torch.distributed as dist

    from zipserv_asplos26_b200.llama_decode import LLAMA3_8B, DecodeStep

    batches = [b for b in (1, 16, 64) if b <= args.max_step_batch]
    t0 = time.time()
    dense = DecodeStep(LLAMA3_8B, max(batches), dev, mode="dense", world=world, rank=rank)
    exchange = None
    if world > 1:
        from zipserv_asplos26_b200 import tp as tpmod

        exchange = tpmod.PeerExchange(LLAMA3_8B.hidden, max(batches), device=dev)
    zipm = DecodeStep.packed_from(dense, exchange=exchange)
    setup_s = time.time() - t0
    out = {"model": "llama3-8b random init, 32 layers, context 2048, greedy step",
           "row_parallel_reduction": ("fused in the ZipGEMM kernel (peer stores over NVLink); "
                                      "dense cuBLAS arm uses an NCCL all-reduce")
           if world > 1 else "none (one GPU)",
           "tp": world, "packed_weight_bytes_per_rank": zipm.weight_bytes(),
           "dense_weight_bytes_per_rank": dense.weight_bytes(),
           "setup_s": round(setup_s, 1), "batches": []}
    stream = torch.cuda.Stream(dev)
    for b in batches:
        tokens = torch.arange(b, device=dev, dtype=torch.int64) * 977 % 128256
        row = {"batch": b}
        for name, model in (("zipgemm", zipm), ("dense_cublas", dense)):
            graph, nxt = model.capture(tokens, stream)
            for _ in range(3):
                graph.replay()
            torch.cuda.synchronize(dev)
            times = []
            for _ in range(max(5, args.steps)):
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                graph.replay()
                e.record()
                torch.cuda.synchronize(dev)
                times.append(s.elapsed_time(e))
            t = torch.tensor([statistics.median(times)], dtype=torch.float64, device=dev)
            if world > 1:
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
            row[f"{name}_ms"] = round(float(t.item()), 3)
            del graph
        row["tokens_per_s_zipgemm"] = round(b / row["zipgemm_ms"] * 1e3, 1)
        row["zipgemm_speedup_vs_cublas"] = round(row["dense_cublas_ms"] / row["zipgemm_ms"], 3)
        out["batches"].append(row)
    del zipm, dense
    if exchange is not None:
        exchange.close()
    torch.cuda.empty_cache()
    return out


LLAMA70B = (  # name, M, K, tensor-parallel split
    ("qkv", 10240, 8192, "col"),
    ("o", 8192, 8192, "row"),
    ("gate_up", 57344, 8192, "col"),
    ("down", 8192, 28672, "row"),
)


def tp70b_case(args, world: int, rank: int, dev) -> dict:
    """The Llama-3-70B shape table: the Llama-3-70B linears split over `world` GPUs
    (qkv and gate_up on output rows, o and down on K), N in {1, 16, 64, 256}.
    Per call, after a 256 MiB L2 flush: ZipGEMM and cuBLAS BF16 on this
    rank's shard, and for the row-parallel layers the NCCL all-reduce of the
    [N, M] BF16 partial output timed separately; max over ranks."""
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F

    from zipserv_asplos26_b200 import runtime

    flush = torch.empty(64 * 2**20, dtype=torch.int32, device=dev)
    rows = []
    exchange = None
    if world > 1:
        from zipserv_asplos26_b200 import tp as tpmod

        exchange = tpmod.PeerExchange(8192, 256, device=dev)

    def timed(fn):
        for _ in range(2):
            fn()
        ts = []
        for _ in range(5):
            flush.zero_()
            torch.cuda._sleep(1_000_000)  # the host enqueues fn meanwhile: device time only
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize(dev)
            ts.append(s.elapsed_time(e) * 1e3)
        t = torch.tensor([statistics.median(ts)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for li, (name, m, k, split) in enumerate(LLAMA70B):
        mm, kk, (r0, r1), (c0, c1) = _shard(name, m, k, split, world, rank)
        g = torch.Generator(device=dev).manual_seed(7000 + li)
        w = (torch.randn(m, k, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        local = w[r0:r1, c0:c1].contiguous()
        del w
        packed = runtime.compress_device(local)
        for n in (1, 16, 64, 256):
            x = torch.randn(n, kk, generator=g, device=dev).to(torch.bfloat16)
            zus = timed(lambda: runtime.linear(x, packed))
            dus = timed(lambda: F.linear(x, local))
            row = {"layer": name, "m": mm, "k": kk, "n": n, "zipgemm_us": round(zus, 2),
                   "cublas_bf16_us": round(dus, 2),
                   "gbs": round((packed.storage_bytes + 2 * n * (kk + mm)) / (zus * 1e-6) / 1e9, 1),
                   "speedup_vs_cublas": round(dus / zus, 3)}
            if split == "row" and world > 1:
                y = torch.empty(n, mm, dtype=torch.bfloat16, device=dev)
                row["nccl_allreduce_us"] = round(timed(lambda: dist.all_reduce(y)), 2)
                row["zipgemm_fused_allreduce_us"] = round(
                    timed(lambda: exchange.linear(x, packed, out=y, fused=True)), 2)
            rows.append(row)
        del packed, local
    if exchange is not None:
        exchange.close()
    flags = runtime.device_flags()
    if flags:
        raise SystemExit(f"device failure flags {flags:#x} set during the 70B case")
    return {"workload": "llama3-70b linears, tp%d shards, N in {1,16,64,256}" % world,
            "timing": "median of 5 per-call CUDA events after a 256 MiB L2 flush (the call enqueued behind a GPU sleep, so host launch time is excluded), max over ranks",
            "per_shape": rows}


def threshold_sweep(args) -> None:
    """Per-shape crossover between the fused kernel and decompression + cuBLAS
    BF16 (the planner's large-batch route), one B200, per-call CUDA events
    after a 256 MiB L2 flush. Prints one JSON line."""
    import torch
    import torch.nn.functional as F

    from zipserv_asplos26_b200 import runtime

    dev = torch.device("cuda", 0)
    flush = torch.empty(64 * 2**20, dtype=torch.int32, device=dev)

    def timed(fn):
        for _ in range(2):
            fn()
        ts = []
        for _ in range(7):
            flush.zero_()
            torch.cuda._sleep(1_000_000)  # the host enqueues fn meanwhile: device time only
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize(dev)
            ts.append(s.elapsed_time(e) * 1e3)
        return statistics.median(ts)

    out = []
    for li, (name, m, k, _split) in enumerate(LAYERS + LLAMA70B):
        g = torch.Generator(device=dev).manual_seed(9000 + li)
        w = (torch.randn(m, k, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        packed = runtime.compress_device(w)
        dense = torch.empty_like(w)
        row = {"layer": name, "m": m, "k": k, "points": []}
        cross = None
        for n in (16, 32, 64, 96, 128, 192, 256, 384, 512, 768):
            x = torch.randn(n, k, generator=g, device=dev).to(torch.bfloat16)
            fused = timed(lambda: runtime.linear(x, packed))
            route = timed(lambda: F.linear(x, runtime.decompress(packed, out=dense)))
            row["points"].append([n, round(fused, 1), round(route, 1)])
            if cross is None and route < fused:
                cross = n
        row["first_n_where_decode_route_wins"] = cross
        out.append(row)
        del w, packed, dense
    print(json.dumps({"threshold_sweep": out}), flush=True)


def stress_case(args) -> dict:
    """The exception-stress configuration on this GPU: a 28672x8192 weight with 5 % N(0, 1)
    outliers. Standalone decompression (algorithmic bytes = packed + dense
    output), the fused path at N = 16, and prefill at N = 4096 as
    decompression + cuBLAS BF16 against cuBLAS on the dense weight. Every
    timed call runs between its own events after a 256 MiB L2 flush."""
    import torch
    import torch.nn.functional as F

    from zipserv_asplos26_b200 import runtime

    m, k = 28672, 8192
    g = torch.Generator().manual_seed(0)
    w = torch.randn(m, k, generator=g) * 0.02
    mask = torch.rand(m, k, generator=g) < 0.05
    w = torch.where(mask, torch.randn(m, k, generator=g), w).to(torch.bfloat16)
    packed_host = runtime.compress(w)
    packed = packed_host.to("cuda")
    dense = w.cuda()
    del w, mask
    x16 = torch.randn(16, k, generator=g).to(torch.bfloat16).cuda()
    x4k = torch.randn(4096, k, generator=g).to(torch.bfloat16).cuda()
    out = torch.empty(m, k, dtype=torch.bfloat16, device="cuda")
    flush = torch.empty(64 * 2**20, dtype=torch.int32, device="cuda")

    def timed(fn, reps=max(5, args.steps // 4)):
        for _ in range(3):
            fn()
        times = []
        for _ in range(reps):
            flush.zero_()
            torch.cuda._sleep(1_000_000)  # the host enqueues fn meanwhile: device time only
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
            times.append(s.elapsed_time(e) * 1e3)
        return statistics.median(times)

    storage = packed_host.storage_bytes
    t_dec = timed(lambda: runtime.decompress(packed, out=out))
    t_fused = timed(lambda: runtime.linear(x16, packed))
    t_prefill = timed(lambda: F.linear(x4k, runtime.decompress(packed, out=out)))
    t_dense = timed(lambda: F.linear(x4k, dense))
    flags = runtime.device_flags()
    if flags:
        raise SystemExit(f"device failure flags {flags:#x} set during the stress case")
    return {
        "workload": "28672x8192, 95 % N(0,0.02) + 5 % N(0,1) outliers (seeded)",
        "ratio_of_dense": round(storage / (m * k * 2), 4),
        "max_rare": packed_host.max_rare,
        "decompress_us": round(t_dec, 1),
        "decompress_gbs": round((storage + 2 * m * k) / (t_dec * 1e-6) / 1e9, 1),
        "fused_n16_us": round(t_fused, 1),
        "fused_n16_gbs": round((storage + 2 * 16 * (k + m)) / (t_fused * 1e-6) / 1e9, 1),
        "prefill_n4096_decompress_plus_cublas_us": round(t_prefill, 1),
        "prefill_n4096_cublas_dense_us": round(t_dense, 1),
        "prefill_tflops": round(2 * m * k * 4096 / (t_prefill * 1e-6) / 1e12, 1),
        "timing": "median of per-call CUDA events after a 256 MiB L2 flush (the call enqueued behind a GPU sleep, so host launch time is excluded)",
    }


def run_profile_case(spec: str, repeats: int) -> None:
    """Run one linear `repeats` times (for ncu captures; prints nothing timed)."""
    import torch

    from zipserv_asplos26_b200 import runtime

    name, n = spec.split(":")
    if name == "decompress":  # decompress:<layer>: the standalone decode kernel
        name, n = n, 0
    n = int(n)
    lay = {l[0]: l for l in LAYERS}[name]
    _, m, k, _ = lay
    g = torch.Generator().manual_seed(1000 + [l[0] for l in LAYERS].index(name))
    w = (torch.randn(m, k, generator=g) * 0.02).to(torch.bfloat16)
    packed = runtime.compress(w).to("cuda")
    if n == 0:
        out = torch.empty(m, k, dtype=torch.bfloat16, device="cuda")
        for _ in range(repeats):
            runtime.decompress(packed, out=out)
        torch.cuda.synchronize()
        if not torch.equal(out.cpu().view(torch.int16), w.view(torch.int16)):
            raise SystemExit("decompression is not bit-exact")
        print(json.dumps({"profile_case": spec, "m": m, "k": k, "repeats": repeats,
                          "algorithmic_bytes_per_launch": packed.storage_bytes + 2 * m * k}))
        return
    x = torch.randn(n, k, generator=torch.Generator().manual_seed(7)).to(torch.bfloat16).cuda()
    for _ in range(repeats):
        runtime.linear(x, packed)
    torch.cuda.synchronize()
    if runtime.device_flags() != 0:
        raise SystemExit("device wait timeout flag set")
    print(json.dumps({"profile_case": spec, "m": m, "k": k, "n": n, "repeats": repeats,
                      "algorithmic_bytes_per_launch": packed.storage_bytes + 2 * n * k + 2 * n * m,
                      "kparts": runtime.plan_kparts(m, n, k)}))


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=50)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument("--tokens", type=int, nargs="*", default=list(TOKENS))
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--profile", metavar="LAYER:N",
                        help="run one linear for ncu, e.g. o:16 (decompress:gate_up: the "
                             "standalone decompression of that weight)")
    parser.add_argument("--repeats", type=int, default=4)
    parser.add_argument("--no-extras", action="store_true",
                        help="skip the Llama-3-70B TP shapes and the Llama-3-8B decode step")
    parser.add_argument("--max-step-batch", type=int, default=64)
    parser.add_argument("--threshold-sweep", action="store_true",
                        help="measure the fused vs decompress + cuBLAS crossover per shape")
    parser.add_argument("--stress", action="store_true",
                        help="also measure the 28672x8192 outlier-stress weight")
    args = parser.parse_args()
    if args.profile:
        run_profile_case(args.profile, args.repeats)
        return
    if args.threshold_sweep:
        threshold_sweep(args)
        return
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1 and args.impl == "ours":
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    try:
        line = run_reference(args, world, rank) if args.impl == "reference" else run_ours(args, world, rank)
    finally:
        if world > 1 and args.impl == "ours":
            import torch.distributed as dist

            dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
