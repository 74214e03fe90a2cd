"""Benchmark of the B200 tensor-parallel INT8 linear path: the DiT MLP block.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (TP = N)

Workload (MLP part, M = 32768 tokens, hidden 3072, MLP 8192):
one step is FC1 (ColumnParallel, [gate|up]) -> FP32 SwiGLU -> ConvRot256 -> global
per-row INT8 quant -> FC2 (RowParallel) -> partial-sum reduction -> fp16 residual add,
i.e. TPDiTMLPINT8.forward, on seeded synthetic inputs and random-init INT8 weights of
that shape (no checkpoint or dataset is involved).

value: whole-job INT8 TOPS = 2*M*(2*ffn*hidden + hidden*ffn) / device time per block
       (max over ranks, CUDA events, inputs resident in HBM; h alone is 201 MB, larger
       than the 126 MB L2, so no flush is needed between steps).
e2e:   the same through the public module API with every step's inputs (h, residual)
       copied host->device from pinned memory and the updated residual copied back,
       inside the timed region (copies on two streams, overlapped with compute; at
       TP > 1 each rank uploads 1/t of the rows and NCCL all-gathers them).
roofline: the dominant kernel (the FC1 tcgen05 GEMM with the SwiGLU epilogue) timed
       with CUDA events inside the timed steps, against the INT8 tensor peak measured in
       the same run (the larger of cuBLAS int8 via torch._int_mm and this library's own
       INT32 GEMM at 8192^3, best of 10).
parity: after the timed region, one more step on a copy of the residual; sampled rows
       (two from every 256-row tile, plus the first and the last) are recomputed by the
       CPU checker (the oracle's composition of the same sharded arithmetic) and compared
       bit for bit, on every rank at every TP size; the e2e output likewise.
cpu_baseline / --impl reference: the reference's CPU path (torch._int_mm, the CPU
       INT32 GEMM of patches/parallel_int8.int_mm, plus the oracle's C restatement of
       the rotation / quantisation / epilogues) on a bounded row sample, host cores.
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
sys.path.insert(0, str(ROOT / "minimax-h3-2xt4_b200"))

METRIC = "INT8 TOPS/GPU and µs per DiT MLP block at M=32k, TP 1/2/4/8; % of INT8 TC peak"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=32768)
    ap.add_argument("--hidden", type=int, default=3072)
    ap.add_argument("--ffn", type=int, default=8192)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--sweep", action="store_true",
                    help="BASELINE config 5 shape sweep on one GPU: one JSON line per point")
    ap.add_argument("--sweep-producers", action="store_true",
                    help="only the activation-producer lines of the sweep")
    ap.add_argument("--sweep-only", default="",
                    help="comma-separated producer lines to run (column_quantize, "
                         "fc2_producer_tp1, fc2_producer_tp1_gateup, norm_producer, "
                         "fc2_producer_tp); all when empty")
    ap.add_argument("--fc1-epilogue", choices=["swiglu", "fp16"], default="swiglu",
                    help="FC1 writes the FP32 SwiGLU activation, or fp16 [gate|up] with the "
                         "SwiGLU applied in the FC2 producer (the reference's form)")
    ap.add_argument("--max-exchange", choices=["peer", "nccl"], default="peer",
                    help="FC2 row maxima at TP > 1: in-kernel over peer memory, or NCCL MAX")
    ap.add_argument("--payload", choices=["fp16", "int8_gather"], default="fp16",
                    help="row partial payload at TP > 1 (scaled fp16, or the packed INT8 scheme)")
    ap.add_argument("--transport", choices=["p2p", "nvls", "rowblock", "allreduce"], default="p2p",
                    help="row partial exchange at TP > 1 (peer memory, in-switch NVLS reduction, "
                         "NCCL row blocks or NCCL all-reduce)")
    ap.add_argument("--workload", choices=["dit_mlp_block", "dit_linear_block"],
                    default="dit_mlp_block",
                    help="dit_linear_block: BASELINE config 4's whole linear set (QKV, O, FC1, FC2)")
    ap.add_argument("--chunks", type=int, default=1,
                    help="TP > 1: row chunks of the pipelined MLP forward (1 = off, the policy "
                         "default; 0 = by size)")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the sampled-row bit-exactness check after the timed region")
    ap.add_argument("--int8-peak", action="store_true",
                    help="only measure the INT8 tensor peak on one GPU and print it")
    ap.add_argument("--ref-rows", type=int, default=4096,
                    help="--impl reference: rows of the block computed per step")
    return ap.parse_args()


def workload_config(args, world):
    """The `config` object both arms print for this workload."""
    return {"workload": "dit_mlp_block", "M": args.tokens, "hidden": args.hidden,
            "ffn": args.ffn, "tp": world, "parallelism": f"tp{world}",
            "fc2_quantizer": "fused_stored",
            "row_transport": args.transport, "row_payload": args.payload,
            "fc2_max_exchange": args.max_exchange, "fc1_epilogue": args.fc1_epilogue,
            "l2": "inputs larger than L2 (h = 201 MB per step), no flush"}


def cpu_info():
    model = None
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"cpu_model": model, "os_cpu_count": os.cpu_count()}


def block_ops(M, hidden, ffn):
    return 2 * M * (2 * ffn) * hidden + 2 * M * hidden * ffn


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d.get("hbm_gbs", 6650.0), "bf16": d.get("bf16_tflops", 1590.0),
                "bf16_sustained": d.get("bf16_tflops_sustained", 1400.0), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


# ----------------------------------------------------------------------------
# synthetic workload (identical bytes on every rank: generated on the CPU)
# ----------------------------------------------------------------------------
def make_weights(hidden, ffn, seed=0):
    import torch
    g = torch.Generator().manual_seed(seed)
    w1 = torch.randint(-127, 128, (2 * ffn, hidden), generator=g, dtype=torch.int8)
    s1 = (torch.rand((2 * ffn, 1), generator=g) * 9e-3 + 1e-3).float()
    w2 = torch.randint(-127, 128, (hidden, ffn), generator=g, dtype=torch.int8)
    s2 = ((torch.rand((hidden, 1), generator=g) * 9e-3 + 1e-3) / 512).float()  # /512 fold
    return w1, s1, w2, s2


def make_inputs(M, hidden, seed=1):
    import torch
    g = torch.Generator().manual_seed(seed)
    h = torch.randn((M, hidden), generator=g)
    cols = torch.randperm(hidden, generator=g)[: max(1, hidden // 100)]
    h[:, cols] *= 20.0  # 1% outlier columns
    x = torch.randn((M, hidden), generator=g) * 0.25
    return h.half(), x.half()


# ----------------------------------------------------------------------------
# clocks
# ----------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi clock / throttle-reason samples taken while the timed region runs.

    The sampler is started, and its first sample awaited, before the region begins;
    on exit it waits for one sample taken after the region ended, so even a short
    region is covered.  Only samples taken inside the region are summarised."""
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    PERIOD_MS = 20

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.samples = []  # (monotonic time, line)
        self.t0 = self.t1 = None

    def _read(self):
        for line in self.proc.stdout:
            if line.strip():
                self.samples.append((time.monotonic(), line))

    def _wait_for(self, pred, timeout):
        end = time.monotonic() + timeout
        while time.monotonic() < end and not pred():
            time.sleep(0.005)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.QUERY,
                 "--format=csv,noheader,nounits", "-lms", str(self.PERIOD_MS)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
            self._wait_for(lambda: len(self.samples) > 0, 15.0)
        except OSError:
            self.proc = None
        self.t0 = time.monotonic()
        return self

    def __exit__(self, *exc):
        self.t1 = time.monotonic()
        if self.proc is not None:
            self._wait_for(lambda: self.samples and self.samples[-1][0] > self.t1, 2.0)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        inside = [l for t, l in self.samples if self.t0 <= t <= self.t1 + 0.001 * self.PERIOD_MS]
        if not inside and self.samples:  # region shorter than one period: nearest sample
            inside = [min(self.samples, key=lambda s: abs(s[0] - self.t1))[1]]
        self.lines = inside

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in getattr(self, "lines", []):
            f = [v.strip() for v in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------
# CPU baseline (the reference's CPU path on host cores; oracle = checker code)
# ----------------------------------------------------------------------------
def cpu_block_sample(rows, w1, s1, w2, s2, h, x, threads, start=0):
    """One MLP block over rows [start, start + rows) on the CPU in the reference's
    order; returns (seconds, ops)."""
    import torch
    from oracle import oracle as O
    torch.set_num_threads(threads)
    hs = h[start:start + rows].numpy()
    t0 = time.perf_counter()
    q, a = O.column_quantize(hs, True)
    C1 = torch._int_mm(torch.from_numpy(q), w1.t().contiguous()).numpy()  # parallel_int8.int_mm
    act = O.swiglu_epilogue(C1, a, s1.numpy().ravel())
    R, m = O.fc2_rotate(act, "act_f32")
    q2, a2 = O.row_quantize(R, m)
    C2 = torch._int_mm(torch.from_numpy(q2), w2.t().contiguous()).numpy()
    res = x[start:start + rows].numpy().copy()
    O.dequantize_i32(C2, a2, s2.numpy().ravel(), out="residual", residual=res)
    dt = time.perf_counter() - t0
    return dt, block_ops(rows, w2.shape[0], w2.shape[1])


def cpu_baseline(w1, s1, w2, s2, h, x, budget_s=12.0, rows=4096):
    import torch
    threads = os.cpu_count() or 1
    cpu_block_sample(64, w1, s1, w2, s2, h, x, threads)  # warm-up
    total_t = total_ops = 0.0
    n = 0
    M = h.shape[0]
    while total_t < budget_s and n < 200:
        dt, ops = cpu_block_sample(rows, w1, s1, w2, s2, h, x, threads, (n * rows) % (M - rows + 1))
        total_t += dt
        total_ops += ops
        n += 1
    line = {"value": round(total_ops / total_t / 1e12, 4), "unit": "TOPS", "cores": threads,
            "kind": "port", "torch_threads": torch.get_num_threads(),
            "sample": f"{n} x {rows}-row slices of the M={M} MLP block (oracle C "
                      f"rotation/quant/epilogues + torch._int_mm), {total_t:.1f} s"}
    line.update(cpu_info())
    return line


def run_reference(args):
    """--impl reference: the reference's CPU path on the host cores; every step computes
    a bounded sample of the block (args.ref_rows consecutive rows, a different slice per
    step), so the rate is the workload's and the run stays short.  Rank 0 alone."""
    import torch
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    w1, s1, w2, s2 = make_weights(args.hidden, args.ffn)
    h, x = make_inputs(args.tokens, args.hidden)
    rows = min(args.ref_rows, args.tokens)
    threads = os.cpu_count() or 1
    M = args.tokens

    def at(i):
        return (i * rows) % (M - rows + 1)

    for i in range(args.warmup):
        cpu_block_sample(rows, w1, s1, w2, s2, h, x, threads, at(i))
    times = []
    for i in range(args.steps):
        dt, _ = cpu_block_sample(rows, w1, s1, w2, s2, h, x, threads, at(args.warmup + i))
        times.append(dt)
    total = sum(times)
    value = block_ops(rows, args.hidden, args.ffn) * args.steps / total / 1e12
    sample = (f"{rows} of the {M} rows of the MLP block per step (a different slice each "
              f"step; oracle C rotation/quant/epilogues + torch._int_mm, {threads} threads)")
    cpu = {"value": round(value, 4), "unit": "TOPS", "cores": threads, "kind": "port",
           "torch_threads": torch.get_num_threads(), "sample": sample}
    cpu.update(cpu_info())
    line = {
        "metric": METRIC, "value": round(value, 4), "unit": "TOPS", "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (seeded N(0,1) input with 1% x20 outlier columns, random int8 weights)",
        "config": workload_config(args, args.gpus),
        "cpu_baseline": cpu,
        "e2e": {"value": round(value, 4), "unit": "TOPS", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------
# sampled-row parity (checker: the oracle's composition of the sharded arithmetic)
# ----------------------------------------------------------------------------
def sample_rows(lo, hi, salt, tile=256):
    """Two rows of every `tile`-row block of [lo, hi) (offsets depend on `salt`, so
    different ranks check different rows), plus the first and the last row."""
    import numpy as np
    rows = {lo, hi - 1}
    o1, o2 = (37 * salt + 11) % tile, (101 * salt + 200) % tile
    for t in range(lo - lo % tile, hi, tile):
        for o in (o1, o2):
            if lo <= t + o < hi:
                rows.add(t + o)
    return np.array(sorted(rows), dtype=np.int64)


def oracle_block_rows(rows, h, x, w1, s1, w2, s2, world, payload):
    """The MLP block's residual output for the given rows, computed by the CPU checker
    exactly as `world` ranks shard it (FC1 rows per patches/parallel_int8.packed_rows,
    FC2 contiguous K blocks, rank-order partial reduction)."""
    import torch
    from oracle import oracle as O
    idx = torch.from_numpy(rows)
    return O.mlp_block(x[idx].numpy(), h[idx].numpy(), w1.numpy(), s1.numpy(), w2.numpy(),
                       s2.numpy(), world, payload=payload)


def rows_bit_exact(got, ref):
    """(number of rows compared, number of rows with any differing bit)."""
    import numpy as np
    bad = (got.view(np.uint16) != ref.view(np.uint16)).any(axis=1)
    return int(got.shape[0]), int(bad.sum())


def measure_int8_peak(dev):
    """INT8 dense tensor throughput measured on this GPU now: cuBLAS int8 through
    torch._int_mm (8192^3 and an FC1-shaped 8192 x 16384 x 3072) and this library's own
    exact INT32 GEMM (tcgen05 kind::i8) at 8192^3; best of 10 launches each, CUDA events
    on the launching stream.  Returns TOPS per case and the larger as the peak."""
    import torch
    from h3tp import ops
    g = torch.Generator(device=dev).manual_seed(7)
    out = {}

    def best(fn, ops_count):
        for _ in range(3):
            fn()
        ts = []
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize(dev)
            ts.append(e0.elapsed_time(e1))
        return round(ops_count / (min(ts) * 1e-3) / 1e12, 1)

    for name, (m, n, k) in {"8192^3": (8192, 8192, 8192), "fc1_8192x16384x3072": (8192, 16384, 3072)}.items():
        a = torch.randint(-128, 128, (m, k), generator=g, device=dev, dtype=torch.int8)
        b = torch.randint(-127, 128, (n, k), generator=g, device=dev, dtype=torch.int8)
        out[f"cublas_int_mm_{name}"] = best(lambda: torch._int_mm(a, b.t()), 2.0 * m * n * k)
        if name == "8192^3":
            out[f"ours_i32_{name}"] = best(lambda: ops.int8_gemm_i32(a, b), 2.0 * m * n * k)
        del a, b
    torch.cuda.empty_cache()
    out["peak"] = max(v for v in out.values())
    return out


def kernel_clock_mhz(dev, fn, probe_ns=8_000_000):
    """SM clock (MHz) while fn() runs back to back: the library's clock probe (one
    sleeping 32-thread CTA, which fits beside a GEMM CTA) runs on a second stream from
    the end of the second launch for probe_ns, and reports SM cycles / elapsed ns.  The
    nvidia-smi samples of `clocks` are taken every 200 ms, mostly between kernels; this
    is the clock inside the kernels."""
    import math
    import torch
    from h3tp import ops
    main = torch.cuda.current_stream(dev)
    side = torch.cuda.Stream(device=dev)
    out = torch.zeros(2, dtype=torch.int64, device=dev)
    for _ in range(3):
        fn()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(main)
    fn()
    e1.record(main)
    torch.cuda.synchronize(dev)
    n = 4 + math.ceil(2.0 * probe_ns * 1e-6 / max(e0.elapsed_time(e1), 1e-3))
    ev = torch.cuda.Event()
    for i in range(n):
        fn()
        if i == 1:
            ev.record(main)
            side.wait_event(ev)
            ops.sm_clock_probe(out, probe_ns, side)
    torch.cuda.synchronize(dev)
    ns, cycles = out.tolist()
    return round(cycles / ns * 1e3, 1) if ns else None


def run_int8_peak(args):
    import torch
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    with ClockSampler(0) as clocks:
        res = measure_int8_peak(dev)
    res["spec_dense_tops"] = 4500.0
    res["clocks"] = clocks.summary()
    print(json.dumps({"int8_peak": res}), flush=True)
    return 0


# ----------------------------------------------------------------------------
# GPU arm
# ----------------------------------------------------------------------------
def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    comm = None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
        comm = dist

    from h3tp import _native, ops
    from h3tp.tp_dit import TPDiTMLPINT8
    from h3tp import dit_column_linear as col, swiglu_quant as sq

    M, hidden, ffn = args.tokens, args.hidden, args.ffn
    w1, s1, w2, s2 = make_weights(hidden, ffn)
    h_cpu, x_cpu = make_inputs(M, hidden)
    from h3tp.h3_operator_policy import H3OperatorPolicy
    mlp = TPDiTMLPINT8(hidden, ffn, rank, world, device=dev, comm=comm,
                       policy=H3OperatorPolicy(row_payload=args.payload,
                                               row_transport=args.transport,
                                               fc2_max_exchange=args.max_exchange,
                                               fc1_swiglu_epilogue=args.fc1_epilogue == "swiglu",
                                               mlp_pipeline_chunks=args.chunks))
    mlp.fc1.load_shard_from_full(w1, s1)
    mlp.fc2.load_shard_from_full(w2, s2)
    h = h_cpu.to(dev)
    x = x_cpu.to(dev)
    stream = torch.cuda.current_stream(dev)
    pol = mlp.fc2.operator_policy

    fc1_events = []
    fc2_events = []
    sub_events = []  # TP > 1 peer route: (producer, FC2 GEMM, reduce, gather) boundaries
    from h3tp import peer as P, transport as T
    peer_route = (world > 1 and args.transport in ("p2p", "nvls") and args.payload == "fp16"
                  and args.max_exchange == "peer")

    def row_chain_peer(act, xres, record):
        # sq.row_linear's peer route, unrolled so each launch can be bracketed by events
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)] if record else None
        ws = P.workspace(comm, dev, hidden, M)
        q, scale = ws.quantize_rows(act, sq.input_kind(act, ffn // world)[0], "rn")
        if record:
            ev[0].record(stream)
        shift = T.shift_for(ffn // world, world)
        # the route row_linear takes
        form = P.exchange_form(world) if args.transport == "p2p" else "pull"
        push = form == "push"
        if push:
            ws.encode_push(q, mlp.fc2.weight, shift)
        else:
            ops.int8_gemm_row_encode(q, mlp.fc2.weight, shift, out=ws.partial(M))
        if record:
            ev[1].record(stream)
        if form == "dma":
            ws.reduce_and_gather_dma(M, shift, scale, mlp.fc2.weight_scale.reshape(-1), xres)
            if record:
                ev[2].record(stream)
                ev[3].record(stream)
                sub_events.append(ev)
            return
        ws.epoch = P.next_epoch(ws.epoch)
        ops.peer_reduce(ws.bases, ws.world, ws.rank, 0, ws.partial_off, ws.final_off, M, hidden,
                        shift, scale, mlp.fc2.weight_scale.reshape(-1), xres, None, None, ws.epoch,
                        multicast=ws.multicast if args.transport == "nvls" else 0, pushed=push)
        if record:
            ev[2].record(stream)
        ops.peer_gather(ws.bases, ws.world, ws.rank, 0, ws.final_off, M, hidden, xres, ws.epoch)
        if record:
            ev[3].record(stream)
            sub_events.append(ev)

    with torch.no_grad():  # the forward's own choice under inference
        chunks = mlp.pipeline_chunks(x, h)
    nvls_active = False
    if peer_route and args.transport == "nvls":
        nvls_active = P.workspace(comm, dev, hidden, M).multicast != 0
    pipe_events = []  # per step: {name: [(start, end) per chunk]}

    def step(xres, record=False):
        if chunks > 1:
            # the pipelined TP forward (TPDiTMLPINT8.forward_pipelined) with events
            # around every launch on the stream it runs on
            marks = {}

            def timer(name, c, edge):
                if edge == 0:
                    e = torch.cuda.Event(enable_timing=True)
                    e.record()
                    marks.setdefault(name, []).append([e, None])
                else:
                    e = torch.cuda.Event(enable_timing=True)
                    e.record()
                    marks[name][-1][1] = e

            mlp.forward_pipelined(xres, h, None, None, chunks, timer if record else None)
            if record:
                pipe_events.append(marks)
            return
        # TPDiTMLPINT8.forward, unrolled so the FC1 GEMM can be bracketed by events.
        codes, row_scale = col._prepare_activation(h, True, 256)
        if record:
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        if args.fc1_epilogue == "swiglu":
            act = ops.int8_gemm_swiglu(codes, mlp.fc1.weight, row_scale,
                                       mlp.fc1.weight_scale.reshape(-1), None, torch.float32)
        else:
            act = ops.int8_gemm_column(codes, mlp.fc1.weight, row_scale,
                                       mlp.fc1.weight_scale.reshape(-1))
        if record:
            e1.record(stream)
            fc1_events.append((e0, e1))
        if peer_route:
            row_chain_peer(act, xres, record)
        else:
            sq.row_linear(act, mlp.fc2.weight, mlp.fc2.weight_scale, comm,
                          mode=pol.fc2_quantizer, scaled_transport=True, residual=xres,
                          transport=pol.row_transport, payload=pol.row_payload,
                          peer_max=pol.fc2_max_exchange == "peer")
        if record:
            e2 = torch.cuda.Event(enable_timing=True)
            e2.record(stream)
            fc2_events.append((e1, e2))

    with torch.no_grad():
        for _ in range(max(3, args.warmup)):
            step(x)
        torch.cuda.synchronize()
        if comm:
            dist.barrier()
        calls0 = ops.launch_count()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clocks:
            if comm:
                dist.barrier()
            torch.cuda.synchronize()
            start.record(stream)
            for _ in range(args.steps):
                step(x, record=True)
            end.record(stream)
            torch.cuda.synchronize()
            if comm:
                dist.barrier()
        launches = ops.launch_count() - calls0
        elapsed_ms = start.elapsed_time(end)
        if pipe_events:
            # per step, the summed launch times of each phase (they overlap in time)
            def phase(name):
                return statistics.mean(sum(a.elapsed_time(b) for a, b in m[name])
                                       for m in pipe_events)
            fc1_ms = phase("fc1_gemm")
            fc2_ms = phase("peer_producer") + phase("fc2_gemm") + phase("reduce_gather")
            pipe_phases = {k: phase(k) for k in ("column_quantize", "fc1_gemm", "peer_producer",
                                                 "fc2_gemm", "reduce_gather")}
        else:
            fc1_ms = statistics.mean(a.elapsed_time(b) for a, b in fc1_events)
            fc2_ms = statistics.mean(a.elapsed_time(b) for a, b in fc2_events)
            pipe_phases = None
        sub = [0.0] * 4
        if sub_events:
            starts = [b for _, b in fc1_events]
            for k in range(4):
                sub[k] = statistics.mean((ev[k - 1] if k else s0).elapsed_time(ev[k])
                                         for s0, ev in zip(starts, sub_events))
        t = torch.tensor([elapsed_ms, fc1_ms, fc2_ms] + sub, device=dev, dtype=torch.float64)
        t_min = t.clone()
        if comm:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            dist.all_reduce(t_min, op=dist.ReduceOp.MIN)
        elapsed_ms, fc1_ms, fc2_ms = float(t[0]), float(t[1]), float(t[2])
        sub_max, sub_min = [float(v) for v in t[3:]], [float(v) for v in t_min[3:]]
        ms_per_step = elapsed_ms / args.steps

        # Parity of the timed code path: one more step on a copy of the residual.
        x_before = x.clone()
        x_after = x.clone()
        step(x_after)
        torch.cuda.synchronize()

        # e2e through the public module API with host buffers: every step uploads its
        # inputs from pinned host memory and reads the updated residual back.  Copies
        # run on two copy streams (host->device, device->host) with double buffers, so
        # they overlap each other and the previous / next step's compute.  At TP > 1
        # each rank uploads its 1/t row block, the blocks are all-gathered over NVLink
        # (NCCL), and each rank reads back its own 1/t of the (replicated) result into a
        # disjoint slice of the host output.
        e2e = None
        per = M // world if M % world == 0 else M
        a0, a1 = (rank * per, (rank + 1) * per) if per != M else (0, M)
        if not args.no_e2e:
            h_pin = h_cpu.pin_memory()
            x_pin = x_cpu.pin_memory()
            out_pin = [torch.empty_like(x_cpu).pin_memory() for _ in range(2)]
            hd = [torch.empty_like(h) for _ in range(2)]
            xd = [torch.empty_like(x) for _ in range(2)]
            up_s, down_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
            ev = lambda: torch.cuda.Event()  # noqa: E731
            ev_up = [ev(), ev()]
            ev_comp = [ev(), ev()]
            ev_down = [ev(), ev()]
            for e in ev_down:
                e.record(down_s)

            def upload(j):
                with torch.cuda.stream(up_s):
                    up_s.wait_event(ev_down[j])  # the buffer's previous result was read
                    hd[j][a0:a1].copy_(h_pin[a0:a1], non_blocking=True)
                    xd[j][a0:a1].copy_(x_pin[a0:a1], non_blocking=True)
                    ev_up[j].record(up_s)

            def compute(j):
                stream.wait_event(ev_up[j])
                if per != M:
                    dist.all_gather_into_tensor(hd[j], hd[j][a0:a1])
                    dist.all_gather_into_tensor(xd[j], xd[j][a0:a1])
                y = mlp(xd[j], hd[j])
                ev_comp[j].record(stream)
                return y

            def download(j, y):
                with torch.cuda.stream(down_s):
                    down_s.wait_event(ev_comp[j])
                    out_pin[j][a0:a1].copy_(y[a0:a1], non_blocking=True)
                    ev_down[j].record(down_s)

            def run_e2e(n):
                upload(0)
                for i in range(n):
                    if i + 1 < n:
                        upload((i + 1) % 2)
                    download(i % 2, compute(i % 2))
                stream.wait_event(ev_down[(n - 1) % 2])

            run_e2e(3)
            torch.cuda.synchronize()
            if comm:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            up_s.wait_event(e0)
            n_e2e = max(4, args.steps // 2)
            run_e2e(n_e2e)
            e1.record(stream)
            torch.cuda.synchronize()
            te = torch.tensor([e0.elapsed_time(e1) / n_e2e], device=dev, dtype=torch.float64)
            if comm:
                dist.all_reduce(te, op=dist.ReduceOp.MAX)
            e2e_ms = float(te[0])
            e2e_out = out_pin[(n_e2e - 1) % 2]
            e2e = {"value": round(block_ops(M, hidden, ffn) / (e2e_ms * 1e-3) / 1e12, 3),
                   "unit": "TOPS", "ms_per_step": round(e2e_ms, 4),
                   "h2d_bytes_per_step": h_cpu.numel() * 2 + x_cpu.numel() * 2,
                   "d2h_bytes_per_step": x_cpu.numel() * 2,
                   "api": "TPDiTMLPINT8.forward (h3tp.tp_dit) per step, inputs uploaded from "
                          "pinned host memory (1/t per rank, all-gathered over NVLink at t > 1) "
                          "and each rank's 1/t of the residual read back into a disjoint slice "
                          "of the host output; copies overlapped on two streams; bytes are per "
                          "step for the whole job"}

        err = _native.device_error(local)
        if comm:
            e = torch.tensor([err], device=dev)
            dist.all_reduce(e, op=dist.ReduceOp.MAX)
            err = int(e.item())

        # INT8 tensor peak, measured on this GPU now (rank 0; the others wait)
        int8 = measure_int8_peak(dev) if rank == 0 else None
        # the SM clock inside FC1 and inside cuBLAS's INT8 GEMM at the FC1 shape (rank 0)
        sm_clock = None
        if rank == 0:
            codes1, rs1 = col._prepare_activation(h, True, 256)
            act1 = torch.empty((M, ffn // world), dtype=torch.float32, device=dev)
            w1s = mlp.fc1.weight_scale.reshape(-1)
            sm_clock = {"fc1_gemm_mhz": kernel_clock_mhz(dev, lambda: ops.int8_gemm_swiglu(
                codes1, mlp.fc1.weight, rs1, w1s, None, torch.float32, out=act1))}
            del act1
            qa = torch.randint(-128, 128, (8192, 3072), device=dev, dtype=torch.int8)
            qb = torch.randint(-127, 128, (16384, 3072), device=dev, dtype=torch.int8)
            sm_clock["cublas_int8_8192x16384x3072_mhz"] = kernel_clock_mhz(
                dev, lambda: torch._int_mm(qa, qb.t()))
            del qa, qb
            sm_clock["method"] = ("h3_sm_clock_probe beside back-to-back launches: SM cycles / "
                                  "globaltimer ns over 8 ms")

    # Sampled-row bit-exactness of the device step and of the e2e output, checked on
    # every rank by the CPU checker (outside every timed region).
    parity = None
    if not args.no_parity:
        import torch as _t
        _t.set_num_threads(max(1, (os.cpu_count() or 1) // world))
        rows = sample_rows(0, M, rank)
        ref = oracle_block_rows(rows, h_cpu, x_before.cpu(), w1, s1, w2, s2, world, args.payload)
        n_rows, n_bad = rows_bit_exact(x_after[torch.from_numpy(rows).to(dev)].cpu().numpy(), ref)
        e_rows = e_bad = 0
        if e2e is not None:
            rows_e = sample_rows(a0, a1, rank + 7)
            ref_e = oracle_block_rows(rows_e, h_cpu, x_cpu, w1, s1, w2, s2, world, args.payload)
            e_rows, e_bad = rows_bit_exact(e2e_out[torch.from_numpy(rows_e)].numpy(), ref_e)
        c = torch.tensor([n_rows, n_bad, e_rows, e_bad], device=dev, dtype=torch.int64)
        if comm:
            dist.all_reduce(c, op=dist.ReduceOp.SUM)
        n_rows, n_bad, e_rows, e_bad = (int(v) for v in c.tolist())
        parity = {"rows": n_rows, "mismatched_rows": n_bad, "bit_exact": n_bad == 0,
                  "e2e_rows": e_rows, "e2e_bit_exact": e_bad == 0 if e_rows else None,
                  "tp": world, "checker": "CPU oracle composition of the sharded arithmetic",
                  "sampling": "per rank: 2 rows of every 256-row tile + first and last row "
                              "(rank-dependent offsets); e2e: the same over the rank's own slice"}

    if comm:
        dist.barrier()
    total_ops = block_ops(M, hidden, ffn)
    value = total_ops / (ms_per_step * 1e-3) / 1e12
    fc1_ops = 2 * M * (2 * ffn // world) * hidden
    achieved = fc1_ops / (fc1_ms * 1e-3) / 1e12
    traffic = None
    tfile = ROOT / "profiles" / "roofline_traffic.json"
    if tfile.exists():
        try:
            traffic = json.loads(tfile.read_text()).get(f"fc1_swiglu_gemm_tp{world}") \
                if args.fc1_epilogue == "swiglu" else None
        except ValueError:
            traffic = None
    peak = int8["peak"] if int8 else None
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "TOPS", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "us_per_block": round(ms_per_step * 1e3, 1), "tops_per_gpu": round(value / world, 3),
        "frac_of_int8_peak_per_gpu": round(value / world / peak, 4) if peak else None,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (seeded N(0,1) input with 1% x20 outlier columns, random int8 weights)",
        "config": {**workload_config(args, world), "pipeline_chunks": chunks,
                   **({"nvls_multicast": nvls_active} if args.transport == "nvls" else {})},
        "roofline": {"kernel": ("gemm_i8_pair_kernel<EPI_SWIGLU> (FC1)" if args.fc1_epilogue == "swiglu"
                               else "gemm_i8_pair_kernel<EPI_COLUMN> (FC1)"), "bound": "tensor",
                     "achieved": round(achieved, 2), "peak": peak, "unit": "TOPS",
                     "frac": round(achieved / peak, 4) if peak else None, "traffic": traffic,
                     "frac_of_spec": round(achieved / 4500.0, 4),
                     "ms_per_launch": round(fc1_ms, 4), "ops_per_launch": fc1_ops,
                     "peak_source": "measured in this run on this GPU: max of cuBLAS int8 "
                                    "(torch._int_mm) and this library's INT32 GEMM, best of 10",
                     "peak_cases": int8},
        "gpu_launches": int(launches),
        "phases_ms": ({"fc1_gemm": round(fc1_ms, 4), "fc2_chain": round(fc2_ms, 4),
                       "column_quantize_and_rest": round(ms_per_step - fc1_ms - fc2_ms, 4)}
                      if pipe_phases is None else
                      {**{k: round(v, 4) for k, v in pipe_phases.items()},
                       "note": f"pipelined over {chunks} row chunks: summed launch times per "
                               "step on this rank; they overlap, so they add up to more than "
                               "the step"}),
        **({"fc2_chain_ms": {k: [round(sub_min[i], 4), round(sub_max[i], 4)] for i, k in
                             enumerate(("peer_producer", "gemm_encode", "reduce_incl_ready_wait",
                                        "gather"))},
            "fc2_chain_note": "[min, max] over ranks of the mean per step; the reduce includes "
                              "the wait for the slowest rank's ready flag",
            "fc2_exchange": {"push": "push: the row GEMM stores each partial row into its "
                                     "owner's buffer over NVLink, the owner reduces from local "
                                     "memory",
                             "dma": "dma: copy engines pull the peers' rows of the owned block "
                                    "and, after the reduce, the peers' finished rows (the "
                                    "reduce column holds the whole exchange)",
                             "pull": "pull: the row GEMM writes locally, each owner loads its "
                                     "rows from every peer"}[
                P.exchange_form(world) if args.transport == "p2p" else "pull"]}
           if sub_events else {}),
        "device_error": err,
        **({"sm_clock_in_kernel": sm_clock} if sm_clock else {}),
    }
    if parity is not None:
        line["parity"] = parity
    clk = clocks.summary()
    line["clocks"] = {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"],
                      "reasons": clk["reasons"], "samples": clk["samples"]}
    if e2e is not None:
        line["e2e"] = e2e
    if world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(w1, s1, w2, s2, h_cpu, x_cpu, rows=min(args.ref_rows, M))
    if comm:
        from h3tp import peer
        peer.release()
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def linear_block_ops(M, hidden, ffn):
    """QKV [hidden -> 3 hidden] + O [hidden -> hidden] + FC1 [hidden -> 2 ffn] +
    FC2 [ffn -> hidden], 2 M N K each."""
    return 2 * M * hidden * (3 * hidden + hidden + 2 * ffn) + 2 * M * ffn * hidden


def make_linear_weights(hidden, ffn, seed=2):
    import torch
    g = torch.Generator().manual_seed(seed)
    wqkv = torch.randint(-127, 128, (3 * hidden, hidden), generator=g, dtype=torch.int8)
    sqkv = (torch.rand((3 * hidden, 1), generator=g) * 9e-3 + 1e-3).float()
    wo = torch.randint(-127, 128, (hidden, hidden), generator=g, dtype=torch.int8)
    so = ((torch.rand((hidden, 1), generator=g) * 9e-3 + 1e-3) / 512).float()  # /512 fold
    return wqkv, sqkv, wo, so


def run_linear_block(args):
    """BASELINE config 4, the whole DiT block linear set at M tokens: QKV (column) ->
    attention stand-in (the V third) -> O (row, gated residual) -> FC1 (column, SwiGLU)
    -> FC2 (row, gated residual), through TPDiTLinearBlockINT8.forward; same timing,
    e2e, parity and clock rules as the MLP block."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    comm = None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
        comm = dist
    from h3tp import _native, ops
    from h3tp.h3_operator_policy import H3OperatorPolicy
    from h3tp.tp_dit import TPDiTLinearBlockINT8

    M, hidden, ffn = args.tokens, args.hidden, args.ffn
    w1, s1, w2, s2 = make_weights(hidden, ffn)
    wqkv, sqkv, wo, so = make_linear_weights(hidden, ffn)
    _, x_cpu = make_inputs(M, hidden)
    x_cpu = (x_cpu.float() * 4).half()  # the block input and residual, ~N(0, 1)
    block = TPDiTLinearBlockINT8(hidden, ffn, rank, world, device=dev, comm=comm,
                                 policy=H3OperatorPolicy(row_transport=args.transport,
                                                         fc1_swiglu_epilogue=True,
                                                         mlp_pipeline_chunks=args.chunks))
    block.qkv_proj.load_shard_from_full(wqkv, sqkv)
    block.out_proj.load_shard_from_full(wo, so)
    block.fc1.load_shard_from_full(w1, s1)
    block.fc2.load_shard_from_full(w2, s2)
    x = x_cpu.to(dev)
    stream = torch.cuda.current_stream(dev)
    with torch.no_grad():
        for _ in range(max(3, args.warmup)):
            block(x)
        torch.cuda.synchronize()
        if comm:
            dist.barrier()
        calls0 = ops.launch_count()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clocks:
            if comm:
                dist.barrier()
            torch.cuda.synchronize()
            start.record(stream)
            for _ in range(args.steps):
                block(x)
            end.record(stream)
            torch.cuda.synchronize()
            if comm:
                dist.barrier()
        launches = ops.launch_count() - calls0
        t = torch.tensor([start.elapsed_time(end)], device=dev, dtype=torch.float64)
        if comm:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_per_step = float(t[0]) / args.steps
        x_before = x.clone()
        x_after = x.clone()
        block(x_after)
        torch.cuda.synchronize()

        e2e = None
        per = M // world if M % world == 0 else M
        a0, a1 = (rank * per, (rank + 1) * per) if per != M else (0, M)
        if not args.no_e2e:
            x_pin = x_cpu.pin_memory()
            out_pin = torch.empty_like(x_cpu).pin_memory()
            xd = torch.empty_like(x)
            n_e2e = max(4, args.steps // 2)

            def run_e2e(n):
                for _ in range(n):
                    xd[a0:a1].copy_(x_pin[a0:a1], non_blocking=True)
                    if per != M:
                        dist.all_gather_into_tensor(xd, xd[a0:a1])
                    y = block(xd)
                    out_pin[a0:a1].copy_(y[a0:a1], non_blocking=True)

            run_e2e(2)
            torch.cuda.synchronize()
            if comm:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            run_e2e(n_e2e)
            e1.record(stream)
            torch.cuda.synchronize()
            te = torch.tensor([e0.elapsed_time(e1) / n_e2e], device=dev, dtype=torch.float64)
            if comm:
                dist.all_reduce(te, op=dist.ReduceOp.MAX)
            e2e_ms = float(te[0])
            e2e = {"value": round(linear_block_ops(M, hidden, ffn) / (e2e_ms * 1e-3) / 1e12, 3),
                   "unit": "TOPS", "ms_per_step": round(e2e_ms, 4),
                   "h2d_bytes_per_step": x_cpu.numel() * 2, "d2h_bytes_per_step": x_cpu.numel() * 2,
                   "api": "TPDiTLinearBlockINT8.forward per step: the residual uploaded from pinned "
                          "host memory (1/t per rank, all-gathered at t > 1) and each rank's 1/t "
                          "of the result read back; copies in the stream order of the step"}
        err = _native.device_error(local)
        if comm:
            e = torch.tensor([err], device=dev)
            dist.all_reduce(e, op=dist.ReduceOp.MAX)
            err = int(e.item())
        int8 = measure_int8_peak(dev) if rank == 0 else None

    parity = None
    if not args.no_parity:
        from oracle import oracle as O
        torch.set_num_threads(max(1, (os.cpu_count() or 1) // world))
        rows = sample_rows(0, M, rank)
        idx = torch.from_numpy(rows)
        ref = O.linear_block(x_before.cpu()[idx].numpy(), wqkv.numpy(), sqkv.numpy(), wo.numpy(),
                             so.numpy(), w1.numpy(), s1.numpy(), w2.numpy(), s2.numpy(), world)
        n_rows, n_bad = rows_bit_exact(x_after[idx.to(dev)].cpu().numpy(), ref)
        c = torch.tensor([n_rows, n_bad], device=dev, dtype=torch.int64)
        if comm:
            dist.all_reduce(c, op=dist.ReduceOp.SUM)
        n_rows, n_bad = (int(v) for v in c.tolist())
        parity = {"rows": n_rows, "mismatched_rows": n_bad, "bit_exact": n_bad == 0, "tp": world,
                  "checker": "CPU oracle composition (oracle.linear_block)"}
    if comm:
        dist.barrier()
    ops_step = linear_block_ops(M, hidden, ffn)
    value = ops_step / (ms_per_step * 1e-3) / 1e12
    peak = int8["peak"] if int8 else None
    cfg = workload_config(args, world)
    cfg["workload"] = "dit_linear_block"
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "TOPS", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "us_per_block": round(ms_per_step * 1e3, 1), "tops_per_gpu": round(value / world, 3),
        "frac_of_int8_peak_per_gpu": round(value / world / peak, 4) if peak else None,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (seeded N(0,1) residual, random int8 weights)", "config": cfg,
        "roofline": {"kernel": "the whole block (four tcgen05 GEMMs with their producers and "
                               "transports)", "bound": "tensor",
                     "achieved": round(value / world, 2), "peak": peak, "unit": "TOPS",
                     "frac": round(value / world / peak, 4) if peak else None, "traffic": None,
                     "peak_source": "measured in this run (see the MLP block line)"},
        "gpu_launches": int(launches), "device_error": err,
    }
    if parity is not None:
        line["parity"] = parity
    clk = clocks.summary()
    line["clocks"] = {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"],
                      "reasons": clk["reasons"], "samples": clk["samples"]}
    if e2e is not None:
        line["e2e"] = e2e
    if comm:
        from h3tp import peer
        peer.release()
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def run_sweep(args):
    """M x (K, N) through the column linear (rotation + row quant +
    GEMM + ordered fp16 epilogue) and the TP1 row linear (post-SwiGLU fp16 input:
    ConvRot + row quant + GEMM + FP32 dequant), TOPS and fraction of the INT8 estimate.
    The (5120, 13824) point is the TE (Qwen3-VL) MLP shape."""
    import torch
    from h3tp import swiglu_quant as sq
    from h3tp.dit_column_linear import column_linear
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peak = 2.0 * peaks()["bf16"]
    g = torch.Generator(device=dev).manual_seed(0)

    def timed(fn):
        for _ in range(3):
            fn()
        ts = []
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        return statistics.median(ts)

    with torch.no_grad():
        for K, N in (() if args.sweep_producers else
                     ((3072, 3072), (3072, 16384), (8192, 3072), (5120, 13824))):
            w = torch.randint(-127, 128, (N, K), generator=g, device=dev, dtype=torch.int8)
            s = torch.rand((N, 1), generator=g, device=dev) * 9e-3 + 1e-3
            for M in (256, 1024, 4096, 16384, 65536):
                x = torch.randn((M, K), generator=g, device=dev).half()
                for variant in ("column", "row"):
                    if variant == "column":
                        ms = timed(lambda: column_linear(x, w, s))
                    else:
                        ms = timed(lambda: sq.row_linear(x, w, s, None, mode="fused_recompute"))
                    tops = 2.0 * M * N * K / (ms * 1e-3) / 1e12
                    print(json.dumps({"sweep": variant, "M": M, "K": K, "N": N,
                                      "ms": round(ms, 4), "tops": round(tops, 2),
                                      "frac_of_int8_estimate": round(tops / peak, 4)}), flush=True)
                del x
        # the activation producers of the MLP block at M = 32768 (HBM-bound): the column
        # quantiser of FC1's input and the TP1 FC2 producer (SwiGLU output -> ConvRot ->
        # row maximum -> codes in one pass)
        from h3tp import ops
        M = args.tokens
        hbm = peaks()["hbm_gbs"]
        staging = os.environ.get("H3_ROW_STAGING", "0") == "1"
        only = set(filter(None, args.sweep_only.split(",")))

        def sizes(line, values):
            return values if not only or line in only else ()

        for K in sizes("column_quantize", (3072, 5120)):
            hq = torch.randn((M, K), generator=g, device=dev).half()
            ms = timed(lambda: ops.column_quantize(hq, True))
            nbytes = M * K * 2 + M * K + 4 * M
            print(json.dumps({"sweep": "column_quantize", "M": M, "K": K, "ms": round(ms, 4),
                              "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1),
                              "frac_of_hbm": round(nbytes / (ms * 1e-3) / 1e9 / hbm, 4),
                              "row_staging": staging}), flush=True)
            del hq
        for kl in sizes("fc2_producer_tp1", (8192, 4096)):
            act = torch.randn((M, kl), generator=g, device=dev) * 0.7
            ms = timed(lambda: ops.swiglu_rotate_quantize_local(act, "act_f32"))
            nbytes = M * kl * 4 + M * kl + 8 * M
            print(json.dumps({"sweep": "fc2_producer_tp1", "M": M, "Kl": kl, "ms": round(ms, 4),
                              "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1),
                              "frac_of_hbm": round(nbytes / (ms * 1e-3) / 1e9 / hbm, 4),
                              "row_staging": staging}), flush=True)
            del act
        # the same with the reference's default FC1 output: fp16 [gate | up], the FP32
        # SwiGLU computed in the producer
        for kl in sizes("fc2_producer_tp1_gateup", (8192, 4096)):
            gu = torch.randn((M, 2 * kl), generator=g, device=dev).half()
            ms = timed(lambda: ops.swiglu_rotate_quantize_local(gu, "gateup_f16"))
            nbytes = M * 2 * kl * 2 + M * kl + 8 * M
            print(json.dumps({"sweep": "fc2_producer_tp1_gateup", "M": M, "Kl": kl,
                              "ms": round(ms, 4),
                              "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1),
                              "frac_of_hbm": round(nbytes / (ms * 1e-3) / 1e9 / hbm, 4),
                              "row_staging": staging}), flush=True)
            del gu
        # row 2 of the scope table: the column input producer, fused modulated RMSNorm ->
        # ConvRot -> quant, against the unfused route (norm -> fp16 h -> quantiser)
        for K in sizes("norm_producer", (3072, 5120, 5376)):
            x = torch.randn((M, K), generator=g, device=dev).half()
            w = torch.rand((K,), generator=g, device=dev) + 0.5
            sh = torch.randn((3, K), generator=g, device=dev) * 0.1
            sc = torch.randn((3, K), generator=g, device=dev) * 0.1
            lab = (torch.arange(M, device=dev) % 3).to(torch.int32)
            fused = timed(lambda: ops.modulated_norm_quantize(x, w, 1e-6, sh, sc, lab))

            def unfused():
                _, _, h = ops.modulated_norm_quantize(x, w, 1e-6, sh, sc, lab, quantize=False)
                ops.column_quantize(h, True)

            sep = timed(unfused)
            nbytes = M * K * 2 + M * K + 4 * M  # read x, write codes and scales
            print(json.dumps({"sweep": "norm_producer", "M": M, "K": K, "ms_fused": round(fused, 4),
                              "ms_unfused": round(sep, 4),
                              "gbs_fused": round(nbytes / (fused * 1e-3) / 1e9, 1),
                              "frac_of_hbm": round(nbytes / (fused * 1e-3) / 1e9 / hbm, 4)}),
                  flush=True)
            del x
        # TP > 1 FC2 producer (BASELINE config 4 at TP 2/4/8, Kl = 8192 / t): the
        # in-kernel row-maximum exchange against the two passes of the NCCL route (the
        # MAX all-reduce between them not included) and the TP1 single pass, one GPU
        # emulating `world` ranks whose slots are all published before the launch.
        for world in sizes("fc2_producer_tp", (2, 4, 8)):
            kl = 8192 // world
            act = torch.randn((M, kl), generator=g, device=dev) * 0.7
            _, mx = ops.swiglu_rotate_max(act, "act_f32", store=False)
            bits = mx.reshape(-1).view(torch.int32).to(torch.int64) & 0xFFFFFFFF
            slots = ((1 << 32) | bits).reshape(M, 1).expand(M, world).contiguous()
            bufs = [torch.zeros(256 + M * world * 8, dtype=torch.uint8, device=dev)
                    for _ in range(world)]
            for b in bufs:
                b[256:].view(torch.int64).view(M, world).copy_(slots)
            bases = [b.data_ptr() for b in bufs]
            peer = timed(lambda: ops.swiglu_rotate_quantize_peer(act, bases, world, 0, 256, 1,
                                                                 "act_f32"))

            def two_pass():
                _, m = ops.swiglu_rotate_max(act, "act_f32", store=False)
                ops.swiglu_rotate_quantize(act, m, "act_f32")

            two = timed(two_pass)
            local = timed(lambda: ops.swiglu_rotate_quantize_local(act, "act_f32"))
            nbytes = M * kl * 4 + M * kl + 4 * M  # read the activation, write codes, scales
            print(json.dumps({"sweep": "fc2_producer_tp", "tp": world, "M": M, "Kl": kl,
                              "ms_peer": round(peer, 4), "ms_two_pass": round(two, 4),
                              "ms_tp1_single_pass": round(local, 4),
                              "frac_of_hbm_peer": round(nbytes / (peer * 1e-3) / 1e9 / hbm, 4)}),
                  flush=True)
            del act, bufs
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.int8_peak:
        return run_int8_peak(args)
    if args.workload == "dit_linear_block":
        return run_linear_block(args)
    if args.sweep or args.sweep_producers:
        return run_sweep(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
