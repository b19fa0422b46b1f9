"""Benchmark of the B200 QuantLinear+LoRA hot path (one JSON line on rank 0).

Workload (the decode GEMV sweep): Llama-2-7B-shaped
projections W[N, K] in {4096x4096, 11008x4096, 4096x11008}, bf16 N(0, 0.02)
weights quantized to NF4 with double-quantized scales (block 64, fp8
second level over 256 blocks), X in {1, 4, 16} x K bf16 N(0, 1), LoRA r=16
alpha=32 with B ~ N(0, 0.01).  One step = the nine LoRALinear forwards of
the sweep.  Metric: HBM GB/s of algorithmic bytes per call:
N*K/2 (codes) + nb (fp8 second-level codes, nb = N*K/64 blocks) +
4*ceil(nb/256) (second-level scales) + 2MK (X) + 2MN (Y) + 2r(K+N) (A, B).

The weight set is replicated over >= 512 MB of distinct copies and each step
reads the next copy, so every call streams its weights from HBM (the 126 MB
L2 cannot hold the rotation).  Steps are replayed from CUDA graphs (one per
copy) and timed with CUDA events; multi-GPU runs time the max over ranks.

Arms:
  python bench.py [--gpus N] [--steps K] [--warmup W]   the B200 kernels
  python bench.py --impl reference ...                  the reference's CPU
      path (its eager torch ops, restated in oracle/torch_port.py) on this
      host's cores, over a bounded sample of the same workload.
The clock sampler (nvidia-smi, 100 ms) runs over untimed load steps right
before the timed region as well as during it, so short timed regions still
get samples under load.
With N > 1 (torchrun), each rank holds a column shard: the sweep's layers
have N times the output features, every rank runs its [N_shape, K] shard,
and Y is gathered on every rank (weak scaling): by default inside the GEMV
(each rank's epilogue stores its columns into every rank's full output over
NVLink and the ranks meet at the end of the kernel), with --gather nccl by
an NCCL all-gather after the layer.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "rocm-qlora_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

SHAPES = [(4096, 4096), (11008, 4096), (4096, 11008)]
MS = [1, 4, 16]
R, ALPHA = 16, 32
ROTATE_BYTES = 512 << 20
METRIC = "NF4 QuantLinear+LoRA decode HBM GB/s (configs[1] sweep)"


def algo_bytes(N, K, M, r, lora=True):
    nb = N * K // 64
    b = N * K // 2 + nb + 4 * ((nb + 255) // 256) + 2 * M * K + 2 * M * N
    return b + (2 * r * (K + N) if lora else 0)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ----------------------------------------------------------- clock sampler
class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region.  The
    raw samples go to bench_out/clocks_gpu<i>.csv (directory overridable
    with RQ_BENCH_OUT); the JSON line carries their summary."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        out = os.environ.get("RQ_BENCH_OUT", os.path.join(ROOT, "bench_out"))
        self.path = os.path.join(out, f"clocks_gpu{index}.csv")

    def __enter__(self):
        os.makedirs(os.path.dirname(self.path), exist_ok=True)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        try:
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                    rows.append(parts)
        except Exception:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows)}


# -------------------------------------------------------------- B200 arm
def build_layers(world: int, rank: int, device):
    """Quantized LoRA layers of the sweep (this rank's shard) and copies."""
    import torch.nn as nn
    from rocm_qlora import LoRALinear, QuantLinear
    from tests.inputs import layer_inputs
    layers = []
    for si, (N, K) in enumerate(SHAPES):
        inp = layer_inputs(N, K, 1, sigma=0.02, r=R, alpha=ALPHA, seed=100 + si + 17 * rank)
        lin = nn.Linear(K, N, bias=False, dtype=torch.bfloat16, device=device)
        with torch.no_grad():
            lin.weight.copy_(inp.W.to(device))
        ql = QuantLinear.from_linear(lin, bits=4)
        ql.enable_double_quant()
        lora = LoRALinear(ql, r=R, lora_alpha=ALPHA).to(device).eval()
        with torch.no_grad():
            lora.lora_A.copy_(inp.A)
            lora.lora_B.copy_(inp.B)
        layers.append(lora)
    return layers


def clone_weights(layers, copies):
    """`copies` independent copies of each layer's quantized buffers."""
    from rocm_qlora.quantization.layer_ops import weight_view
    sets = []
    for _ in range(copies):
        views = []
        for lora in layers:
            w = weight_view(lora.base_layer)
            views.append(type(w)(w.fmt, w.q.clone(), None, w.c2.clone(), w.c2_scales.clone(), w.N, w.K,
                                 w.block_size))
        sets.append(views)
    return sets


def run_ours(args, rank, world, device):
    import torch.distributed as dist
    from rocm_qlora.quantization import layer_ops
    hbm_peak, peak_kind = peaks()
    layers = build_layers(world, rank, device)
    per_set = sum(lo.base_layer.weight_quant.numel() + lo.base_layer.c2.numel() for lo in layers)
    copies = max(2, -(-ROTATE_BYTES // per_set))
    wsets = clone_weights(layers, copies)
    g = torch.Generator().manual_seed(7)
    xs = {(si, M): torch.randn(M, K, generator=g).to(torch.bfloat16).to(device)
          for si, (N, K) in enumerate(SHAPES) for M in MS}
    A = [lo.lora_A.detach().to(torch.bfloat16).contiguous() for lo in layers]
    B = [lo.lora_B.detach().to(torch.bfloat16).contiguous() for lo in layers]
    calls = [(si, M) for si in range(len(SHAPES)) for M in MS]

    gather_out, peers = {}, {}
    fused = world > 1 and args.gather == "fused"
    if fused:
        # the shared output buffers; if any rank cannot set them up, every
        # rank gathers with NCCL instead (the ranks must take the same path)
        from rocm_qlora.distributed.peer_gather import PeerGather
        ok = 1
        try:
            for si, (N, K) in enumerate(SHAPES):
                for M in MS:  # this rank's N columns of the full [M, world*N] output, on every rank
                    peers[(si, M)] = PeerGather(None, M, world * N, rank * N, torch.bfloat16, device)
        except Exception as e:  # reported in the JSON line
            ok = 0
            print(f"rank {rank}: fused gather unavailable ({e!r}); using NCCL", file=sys.stderr, flush=True)
        t = torch.tensor([ok], device=device, dtype=torch.int32)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        fused = bool(t.item())
    if world > 1 and not fused:
        for si, (N, K) in enumerate(SHAPES):
            for M in MS:
                gather_out[(si, M)] = torch.empty(world * M, N, dtype=torch.bfloat16, device=device)

    def step(c, lora=True):
        """One sweep pass.  lora=True is the measured step (adapter, and the
        all-gather of Y when sharded); lora=False is the roofline leg: the
        dequant GEMV kernels alone, no adapter and no collective."""
        for si, M in calls:
            w = wsets[c][si]
            if lora and fused:  # the GEMV writes Y into every rank's output (NVLink), no collective
                rc = layer_ops.forward_gather(w, xs[(si, M)], None, A[si], B[si], ALPHA / R, peers[(si, M)].descriptor)
                assert rc == 0, "the fused gather refused a decode call"
            elif lora:
                y = layer_ops.forward(w, xs[(si, M)], None, A[si], B[si], ALPHA / R)
                if world > 1:
                    dist.all_gather_into_tensor(gather_out[(si, M)], y)
            else:
                layer_ops.forward(w, xs[(si, M)], None, None, None, 1.0)

    def capture(lora):
        graphs = []
        s = torch.cuda.Stream(device)
        s.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(s):
            for c in range(copies):
                step(c, lora)
        torch.cuda.current_stream(device).wait_stream(s)
        torch.cuda.synchronize(device)
        for c in range(copies):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                step(c, lora)
            graphs.append(gr)
        return graphs

    if fused:
        # probe the fused gather once, eagerly, before anything is captured:
        # if any rank's calls gave up waiting for a peer (bounded wait in the
        # kernel), every rank switches to the NCCL all-gather
        step(0, True)
        torch.cuda.synchronize(device)
        t = torch.tensor([1 if any(pg.error() for pg in peers.values()) else 0], device=device, dtype=torch.int32)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if t.item():
            print(f"rank {rank}: fused gather probe failed; using NCCL", file=sys.stderr, flush=True)
            for pg in peers.values():
                pg.close()
            peers.clear()
            fused = False
            for si, (N, K) in enumerate(SHAPES):
                for M in MS:
                    gather_out[(si, M)] = torch.empty(world * M, N, dtype=torch.bfloat16, device=device)

    use_graphs = True
    graphs = capture(True)

    def run_steps(n, start, lora=True, gr=None):
        for i in range(n):
            c = (start + i) % copies
            if gr is not None:
                gr[c].replay()
            else:
                step(c, lora)

    def timed(n, lora=True, gr=None):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)
        st = torch.cuda.current_stream(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        run_steps(n, 0, lora, gr)
        e1.record(st)
        torch.cuda.synchronize(device)
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
            dist.barrier()
        return ms

    def all_done(flag: bool) -> bool:
        """True once any rank is done: every rank then takes the same number
        of load batches (each replay holds collectives when world > 1)."""
        if world == 1:
            return flag
        t = torch.tensor([1 if flag else 0], device=device, dtype=torch.int32)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return bool(t.item())

    run_steps(args.warmup, 0, True, graphs)
    with ClockSampler(device.index) as clk:
        # untimed load for the sampler (about 0.4 s), then the timed steps
        t_end = time.perf_counter() + 0.4
        done = False
        while not done:
            run_steps(50, 0, True, graphs)
            torch.cuda.synchronize(device)
            done = all_done(time.perf_counter() >= t_end)
        ms = timed(args.steps, True, graphs)
    clocks = clk.summary()
    step_bytes = sum(algo_bytes(SHAPES[si][0], SHAPES[si][1], M, R) for si, M in calls)
    value = step_bytes * args.steps * world / (ms / 1e3) / 1e9

    # roofline of the dominant kernel: the fused GEMV alone (no adapter)
    gemv_graphs = capture(False)
    run_steps(max(3, args.warmup), 0, False, gemv_graphs)
    ms_g = timed(args.steps, False, gemv_graphs)
    gemv_bytes = sum(algo_bytes(SHAPES[si][0], SHAPES[si][1], M, R, lora=False) for si, M in calls)
    n_launch = args.steps * len(calls)
    achieved = gemv_bytes * args.steps / (ms_g / 1e3) / 1e9
    traffic = None
    tfile = os.path.join(ROOT, "profiles", "gemv_decode_traffic.json")
    if os.path.exists(tfile):
        try:
            traffic = json.load(open(tfile)).get("bytes_per_launch_avg")
        except Exception:
            traffic = None

    # this library's kernels in one step (counted by the profiler, outside
    # the timed region)
    launches_per_step = count_rq_kernels(lambda: run_steps(1, 0, True, graphs), device)

    # graphs that hold NCCL calls are released before the process group goes
    del graphs, gemv_graphs
    torch.cuda.synchronize(device)
    gather_error = any(pg.error() for pg in peers.values())
    for pg in peers.values():
        pg.close()

    # end to end through the public API with host buffers
    e2e = run_e2e(args, rotated_modules(layers, wsets), device, world)

    # CPU baseline on rank 0 (bounded sample of the same workload)
    cpu_layers = _cpu_layers() if (rank == 0 and world == 1 and not args.no_cpu) else None
    cpu = cpu_baseline(args, cpu_layers) if cpu_layers is not None else None
    # configs[2] (prefill / training GEMM), single GPU, with the reference's
    # CPU path timed beside it
    prefill = prefill_leg(device) if (world == 1 and not args.no_prefill) else None
    if prefill is not None and cpu_layers is not None:
        prefill["cpu_baseline"] = prefill_cpu_baseline(cpu_layers)
    c5 = c5_leg(device) if (world == 1 and not args.no_prefill) else None
    if world > 1 and not args.no_prefill:
        c5 = c5_sharded_leg(device, rank, world)
    quant = quant_leg(device, no_cpu=args.no_cpu) if (world == 1 and not args.no_prefill) else None
    c4 = c4_leg(device) if (world == 1 and not args.no_prefill and not args.no_model) else None

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,.) tensors)",
            "config": {"workload": "configs[1]: decode GEMV sweep, W in 4096x4096 / 11008x4096 / 4096x11008 "
                                   "NF4 + double-quant, M in {1,4,16}, LoRA r16 a32",
                       "model": "Llama-2-7B-shaped projections", "global_batch": MS, "seq_len": 1,
                       "parallelism": f"column-shard x{world}" if world > 1 else "single GPU",
                       "gather": (("fused GEMV epilogue peer stores over NVLink" if fused else "NCCL all-gather")
                                  if world > 1 else None),
                       "gather_error": gather_error if world > 1 else None,
                       "l2": f"{copies} rotating weight copies ({copies * per_set / 2**20:.0f} MiB) > 126 MB L2",
                       "graphs": use_graphs},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(achieved / hbm_peak, 4), "traffic": traffic, "peak_kind": peak_kind,
                         "kernel": "gemv_nf4_k (fused NF4-DQ dequant GEMV, no adapter)",
                         "launches": n_launch, "us_per_launch": round(ms_g * 1e3 / n_launch, 3)},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": args.steps * launches_per_step,
            "clocks": clocks,
            "prefill": prefill,
            "c5": c5,
            "quant": quant,
            "c4": c4,
        }
        print(json.dumps(line), flush=True)


PREFILL_MS = [512, 2048, 8192]
PREFILL_R, PREFILL_ALPHA = 64, 128


def prefill_leg(device, iters=5):
    """the tcgen05 dequant GEMM on the three 7B shapes at
    M in {512, 2048, 8192}, forward Y and backward dX, LoRA r=64 alpha=128,
    timed with CUDA events (mean of `iters` calls after 2 warm-up calls).
    FLOPs per call: 2MNK + 2Mr(K+N)."""
    import torch.nn as nn
    from rocm_qlora import LoRALinear, QuantLinear
    from rocm_qlora.quantization import layer_ops
    from tests.inputs import layer_inputs
    peak = None
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        peak = float(pk["bf16_tflops"])  # burst: these calls are timed in isolation
    except Exception:
        peak = 1590.0
    out = {"fwd": {}, "dx": {}}
    flops_all, t_all = 0.0, 0.0
    for si, (N, K) in enumerate(SHAPES):
        inp = layer_inputs(N, K, 1, sigma=0.02, r=PREFILL_R, alpha=PREFILL_ALPHA, seed=200 + si)
        lin = nn.Linear(K, N, bias=False, dtype=torch.bfloat16, device=device)
        with torch.no_grad():
            lin.weight.copy_(inp.W.to(device))
        ql = QuantLinear.from_linear(lin, bits=4)
        ql.enable_double_quant()
        lora = LoRALinear(ql, r=PREFILL_R, lora_alpha=PREFILL_ALPHA).to(device).eval()
        with torch.no_grad():
            lora.lora_A.copy_(inp.A)
            lora.lora_B.copy_(inp.B)
        w = ql.weight_view()
        A = lora.lora_A.detach().bfloat16().contiguous()
        B = lora.lora_B.detach().bfloat16().contiguous()
        g = torch.Generator(device=device).manual_seed(si)
        for M in PREFILL_MS:
            x = torch.randn(M, K, generator=g, device=device).to(torch.bfloat16)
            dy = torch.randn(M, N, generator=g, device=device).to(torch.bfloat16)
            fl = 2.0 * M * N * K + 2.0 * M * PREFILL_R * (K + N)
            for kind, fn in (("fwd", lambda: layer_ops.forward(w, x, None, A, B, lora.scaling)),
                             ("dx", lambda: layer_ops.dx(w, dy, A, B, lora.scaling))):
                for _ in range(2):
                    fn()
                torch.cuda.synchronize(device)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(iters):
                    fn()
                e1.record()
                torch.cuda.synchronize(device)
                us = e0.elapsed_time(e1) * 1e3 / iters
                out[kind][f"{N}x{K}/M{M}"] = round(fl / us / 1e6, 1)
                flops_all += fl
                t_all += us
            del x, dy
        del lora, ql, lin
    tf = flops_all / t_all / 1e6
    return {"metric": "prefill TFLOP/s (2MNK + 2Mr(K+N) per call, incl. the LoRA down product)",
            "unit": "TFLOP/s", "value": round(tf, 1), "peak": peak,
            "peak_kind": "measured burst" if peak != 1590.0 else "fallback", "frac": round(tf / peak, 4),
            "config": "configs[2]: 7B shapes x M in {512,2048,8192}, forward and dX, NF4 double quant, r64 a128",
            "per_call_tflops": out}


QUANT_SHAPES = [(4096, 4096), (8192, 28672)]


def quant_leg(device, iters=5, cpu_seconds=4.0, no_cpu=False):
    """North-star kernel (1): the quantize / dequantize streaming kernels on
    bf16 weights [N, K] in {4096x4096, 8192x28672} (the second is 470 MB,
    larger than L2), timed with CUDA events through the C ABI (mean of
    `iters` calls after 2 warm-up calls).  Algorithmic bytes per call,
    n = N*K, nb = n/64, ng = ceil(nb/256):
      nf4_quantize      2n read + n/2 + 2nb written (codes, bf16 scales)
      nf4_dequantize    n/2 + 2nb read + 4n written (fp32, the reference's output)
      dq_quantize       4nb read (fp32 first-level scales) + nb + 4ng written
      dq_dequantize     n/2 + nb + 4ng read + 4n written (fp32)
      int8_quantize_rows 2n read + n + 2N written
      int8_dequantize   n + 2N read + 4n written (fp32, per-row scales)
    The reference's quantize_int4 (torch CPU ops, oracle/torch_port.py) is
    timed beside it on a bounded sample of the 4096x4096 weight."""
    from rocm_qlora import _native as nat
    L = nat.lib()
    hbm_peak, peak_kind = peaks()
    st = torch.cuda.current_stream(device).cuda_stream
    out = {}
    for (N, K) in QUANT_SHAPES:
        g = torch.Generator(device=device).manual_seed(N + K)
        W = (torch.randn(N, K, generator=g, device=device) * 0.02).to(torch.bfloat16)
        n, nb = N * K, N * K // 64
        ng = (nb + 255) // 256
        packed = torch.empty(n // 2, dtype=torch.uint8, device=device)
        sc = torch.empty(nb, dtype=torch.bfloat16, device=device)
        c1 = torch.empty(nb, dtype=torch.float32, device=device)
        c2 = torch.empty(ng * 256, dtype=torch.uint8, device=device)
        c2s = torch.empty(ng, dtype=torch.float32, device=device)
        fout = torch.empty(n, dtype=torch.float32, device=device)
        q8 = torch.empty(n, dtype=torch.int8, device=device)
        s8 = torch.empty(N, dtype=torch.bfloat16, device=device)
        ops = {
            "nf4_quantize": (lambda: L.rq_nf4_quantize(W.data_ptr(), nat.BF16, n, 64, packed.data_ptr(),
                                                       sc.data_ptr(), st), 2 * n + n // 2 + 2 * nb),
            "nf4_dequantize": (lambda: L.rq_nf4_dequantize(packed.data_ptr(), n // 2, sc.data_ptr(), nat.BF16, 64,
                                                           fout.data_ptr(), nat.F32, st), n // 2 + 2 * nb + 4 * n),
            "dq_quantize": (lambda: L.rq_dq_quantize_scales(c1.data_ptr(), nb, 256, 1, c2.data_ptr(), c2s.data_ptr(),
                                                            st), 4 * nb + nb + 4 * ng),
            "dq_dequantize": (lambda: L.rq_dq_dequantize(packed.data_ptr(), n, c2.data_ptr(), c2s.data_ptr(), 1, 64,
                                                         256, fout.data_ptr(), nat.F32, st),
                              n // 2 + nb + 4 * ng + 4 * n),
            "int8_quantize_rows": (lambda: L.rq_int8_quantize_rows(W.data_ptr(), nat.BF16, N, K, q8.data_ptr(),
                                                                   s8.data_ptr(), st), 2 * n + n + 2 * N),
            "int8_dequantize": (lambda: L.rq_int8_dequantize(q8.data_ptr(), n, s8.data_ptr(), nat.BF16, 64, K,
                                                             fout.data_ptr(), nat.F32, st), n + 2 * N + 4 * n),
        }
        res = {}
        for name, (fn, byts) in ops.items():
            if name == "dq_quantize":  # fp32 first-level scales of this weight
                c1.copy_(sc.float())
            for _ in range(2):
                assert fn() == 0, name
            torch.cuda.synchronize(device)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(iters):
                fn()
            e1.record()
            torch.cuda.synchronize(device)
            us = e0.elapsed_time(e1) * 1e3 / iters
            res[name] = {"GB/s": round(byts / us / 1e3, 1), "us": round(us, 2),
                         "frac": round(byts / us / 1e3 / hbm_peak, 4)}
        out[f"{N}x{K}"] = res
        del W, packed, sc, c1, c2, c2s, fout, q8, s8
    cpu = None
    if not no_cpu:
        from oracle import torch_port
        torch.set_num_threads(os.cpu_count() or 1)
        gc = torch.Generator().manual_seed(1)
        Wc = (torch.randn(4096, 4096, generator=gc) * 0.02).to(torch.bfloat16)
        rows, done, t_total = 256, 0, 0.0
        while t_total < cpu_seconds or done == 0:
            r0 = (done * rows) % 4096
            t0 = time.perf_counter()
            torch_port.nf4_quantize(Wc[r0:r0 + rows])
            t_total += time.perf_counter() - t0
            done += 1
        n = done * rows * 4096
        cpu = {"value": round((2 * n + n // 2 + 2 * n // 64) / t_total / 1e9, 4), "unit": "GB/s",
               "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"{done} quantize_int4 calls on 256-row slices of a 4096x4096 bf16 weight "
                         f"({t_total:.1f} s)"}
    return {"metric": "quantize / dequantize HBM GB/s of algorithmic bytes", "peak": hbm_peak,
            "peak_kind": peak_kind, "calls": out, "cpu_quantize_int4": cpu}


C5_SHAPES = [(8192, 28672), (28672, 8192)]


def c5_leg(device, iters=3):
    """The 70B-shaped projections on one GPU: W[N, K] in
    {8192x28672, 28672x8192}, bf16 N(0, 0.015) weights as NF4 + double quant
    and as INT8 with per-row scales, LoRA r=16 alpha=32; decode M=16 (HBM
    GB/s of algorithmic bytes) and prefill M=4096 (TFLOP/s), forward calls
    through the public layer op, CUDA-event timed (mean of `iters` calls
    after 2 warm-up calls)."""
    import torch.nn as nn
    from rocm_qlora import LoRALinear, QuantLinear
    from rocm_qlora.quantization import layer_ops, quantize_int8
    out = {"nf4_dq": {}, "int8_row": {}}
    for (N, K) in C5_SHAPES:
        g = torch.Generator(device=device).manual_seed(N)
        W = (torch.randn(N, K, generator=g, device=device) * 0.015).to(torch.bfloat16)
        A = ((torch.rand(16, K, generator=g, device=device) * 2 - 1) / K ** 0.5).to(torch.bfloat16).contiguous()
        B = (torch.randn(N, 16, generator=g, device=device) * 0.01).to(torch.bfloat16).contiguous()
        for fmt in ("nf4_dq", "int8_row"):
            if fmt == "nf4_dq":
                lin = nn.Linear(K, N, bias=False, dtype=torch.bfloat16, device=device)
                with torch.no_grad():
                    lin.weight.copy_(W)
                ql = QuantLinear.from_linear(lin, bits=4)
                ql.enable_double_quant()
                wbytes = N * K // 2 + N * K // 64 + 4 * (N * K // 64 // 256 + 1)
                del lin
            else:
                ql = QuantLinear(K, N, bits=8, bias=False).to(device)
                q, s = quantize_int8(W, per_channel=True)
                ql.weight_quant, ql.weight_scales = q, s
                wbytes = N * K + 2 * N
            w = ql.weight_view()
            for M in (16, 4096):
                x = torch.randn(M, K, generator=g, device=device).to(torch.bfloat16)
                fn = lambda: layer_ops.forward(w, x, None, A, B, 2.0)  # noqa: E731
                for _ in range(2):
                    fn()
                torch.cuda.synchronize(device)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(iters):
                    fn()
                e1.record()
                torch.cuda.synchronize(device)
                us = e0.elapsed_time(e1) * 1e3 / iters
                if M == 16:
                    byts = wbytes + 2 * M * (K + N) + 2 * 16 * (K + N)
                    out[fmt][f"{N}x{K}/M{M}"] = {"GB/s": round(byts / us / 1e3, 1), "us": round(us, 2)}
                else:
                    fl = 2.0 * M * N * K + 2.0 * M * 16 * (K + N)
                    out[fmt][f"{N}x{K}/M{M}"] = {"TFLOP/s": round(fl / us / 1e6, 1), "us": round(us, 2)}
                del x
            del ql, w
        del W
    return {"config": "70B-shaped projections on one GPU, NF4+DQ and INT8 per-row, LoRA r16 a32, forward",
            "calls": out}


C4_TARGETS = ["q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"]


def c4_leg(device, steps=4, warmup=2, batch=4, seq=2048):
    """one QLoRA training step of a random-init Llama-2-7B
    (32 layers, d 4096, 32 heads, SwiGLU FFN 11008, vocab 32000) in bf16,
    every q/k/v/o/gate/up/down projection replaced by quantize_model with
    NF4 + LoRA r16 alpha 32 (dropout 0.05, train mode), on batch x seq
    uniform random token ids: forward, causal-LM loss, backward to the
    LoRA parameters and an AdamW step on them.  Timed with CUDA events
    (mean of `steps` steps after `warmup`).  The share of the device time
    spent in this library's kernels (QuantLinear + LoRA forward / dX and the
    LoRA down products) comes from one profiled step (torch.profiler)."""
    from transformers import LlamaConfig, LlamaForCausalLM
    from rocm_qlora import enable_all_kernels, quantize_model
    cfg = LlamaConfig(hidden_size=4096, intermediate_size=11008, num_attention_heads=32, num_key_value_heads=32,
                      num_hidden_layers=32, vocab_size=32000, max_position_embeddings=seq)
    torch.manual_seed(0)
    with torch.device(device):
        model = LlamaForCausalLM._from_config(cfg, dtype=torch.bfloat16, attn_implementation="sdpa")
    import contextlib
    import io
    with contextlib.redirect_stdout(io.StringIO()):
        model = quantize_model(model, bits=4, lora_r=16, lora_alpha=32, lora_dropout=0.05,
                               target_modules=C4_TARGETS)
    enable_all_kernels(model)
    from rocm_qlora import QuantLinear
    n_quant = sum(isinstance(m, QuantLinear) for m in model.modules())
    model.to(device)
    torch.cuda.empty_cache()
    model.train()
    params = [p for p in model.parameters() if p.requires_grad]
    opt = torch.optim.AdamW(params, lr=1e-4)
    g = torch.Generator(device=device).manual_seed(1)
    ids = torch.randint(0, cfg.vocab_size, (batch, seq), generator=g, device=device)

    def step():
        out = model(input_ids=ids, labels=ids)
        out.loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        return out.loss

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        loss = step()
    e1.record()
    torch.cuda.synchronize(device)
    ms = e0.elapsed_time(e1) / steps
    share = None
    try:
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA], acc_events=True) as prof:
            step()
            torch.cuda.synchronize(device)
        tot = ours = 0.0
        for ev in prof.key_averages():
            t = getattr(ev, "device_time_total", None) or getattr(ev, "cuda_time_total", 0.0)
            if ev.key.startswith("void rq::") or ev.key.startswith("rq::"):
                ours += t
            if getattr(ev, "device_type", None) is not None and "CUDA" in str(ev.device_type):
                tot += t
        share = round(ours / tot, 4) if tot > 0 else None
    except Exception as e:  # profiler unavailable: reported, not fatal
        share = f"unavailable: {type(e).__name__}"
    peak_gb = torch.cuda.max_memory_allocated(device) / 2**30
    flops_quant = 0.0
    for m in model.modules():
        if hasattr(m, "in_features") and hasattr(m, "weight_quant"):
            flops_quant += 2.0 * batch * seq * m.in_features * m.out_features * 2  # forward + dX
    out = {"config": "configs[3]: random-init Llama-2-7B, NF4 + LoRA r16 a32 on q/k/v/o/gate/up/down, bf16, "
                     f"batch {batch} x seq {seq} random ids, forward + backward + AdamW on the LoRA parameters",
           "tok_per_s": round(batch * seq / (ms / 1e3), 1), "ms_per_step": round(ms, 2),
           "loss": round(float(loss.detach()), 4), "quantized_layers": n_quant,
           "rq_kernel_time_share": share,
           "quantlinear_tflops_in_step": round(flops_quant / (ms / 1e3) / 1e12, 1),
           "peak_mem_gib": round(peak_gb, 1)}
    del model, opt, params, ids
    torch.cuda.empty_cache()
    return out


def c5_sharded_leg(device, rank, world, iters=20):
    """configs[4] across the node (strong scaling): each 70B-shaped layer
    W[N, K] in {8192x28672, 28672x8192}, NF4 + double quant, LoRA r16 a32,
    built whole on every rank (same seed) and column-sharded without
    re-quantizing (ColumnParallelLinear.from_quant_linear: N/p rows a rank).
    Decode M in {1, 16} gathers Y inside the GEMV (fused, NVLink stores);
    prefill M = 4096 runs the tensor-core GEMM on the shard and an NCCL
    all-gather of Y, whose time is reported on its own.  Per call: the max
    over ranks of the CUDA-event time (graph replays for decode, eager calls
    for prefill), and the same layer unsharded on rank 0 alone (t1), so that
    efficiency = t1 / (p * tp)."""
    import torch.distributed as dist
    import torch.nn as nn
    from rocm_qlora import LoRALinear, QuantLinear
    from rocm_qlora.distributed import ColumnParallelLinear

    def tmax(ms):
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def event_time(fn, n):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dist.barrier()
        torch.cuda.synchronize(device)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize(device)
        return e0.elapsed_time(e1) / n

    out = {}
    for (N, K) in C5_SHAPES:
        g = torch.Generator(device=device).manual_seed(N)
        W = (torch.randn(N, K, generator=g, device=device) * 0.015).to(torch.bfloat16)
        lin = nn.Linear(K, N, bias=False, dtype=torch.bfloat16, device=device)
        with torch.no_grad():
            lin.weight.copy_(W)
        del W
        ql = QuantLinear.from_linear(lin, bits=4)
        ql.enable_double_quant()
        full = LoRALinear(ql, r=16, lora_alpha=32).to(device).eval()
        with torch.no_grad():
            full.lora_A.copy_((torch.rand(16, K, generator=g, device=device) * 2 - 1) / K ** 0.5)
            full.lora_B.copy_(torch.randn(N, 16, generator=g, device=device) * 0.01)
        del lin
        cp = ColumnParallelLinear.from_quant_linear(full, gather_tokens=16).eval()
        wbytes = N * K // 2 + N * K // 64 + 4 * (N * K // 64 // 256 + 1)
        for M in (1, 16, 4096):
            x = torch.randn(M, K, generator=g, device=device).to(torch.bfloat16)
            with torch.no_grad():
                if M <= 16:  # fused gather, graph-replayed
                    s = torch.cuda.Stream(device)
                    s.wait_stream(torch.cuda.current_stream(device))
                    with torch.cuda.stream(s):
                        for _ in range(3):
                            cp(x)
                    torch.cuda.current_stream(device).wait_stream(s)
                    gr = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(gr):
                        cp(x)
                    tp = tmax(event_time(gr.replay, iters))
                    del gr
                    coll = None
                else:  # GEMM on the shard + NCCL all-gather of Y
                    for _ in range(2):
                        cp(x)
                    tp = tmax(event_time(lambda: cp(x), 5))
                    y_loc = cp.local(x)
                    buf = torch.empty(world * M, max(cp.sizes), dtype=y_loc.dtype, device=device)
                    yl = torch.nn.functional.pad(y_loc, (0, max(cp.sizes) - y_loc.shape[1])).contiguous()
                    coll = tmax(event_time(lambda: dist.all_gather_into_tensor(buf, yl), 5))
                t1 = torch.zeros(1, device=device, dtype=torch.float64)
                if rank == 0:  # the unsharded layer alone
                    if M <= 16:
                        s = torch.cuda.Stream(device)
                        s.wait_stream(torch.cuda.current_stream(device))
                        with torch.cuda.stream(s):
                            for _ in range(3):
                                full(x)
                        torch.cuda.current_stream(device).wait_stream(s)
                        gr = torch.cuda.CUDAGraph()
                        with torch.cuda.graph(gr):
                            full(x)
                        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        torch.cuda.synchronize(device)
                        e0.record()
                        for _ in range(iters):
                            gr.replay()
                        e1.record()
                        torch.cuda.synchronize(device)
                        t1[0] = e0.elapsed_time(e1) / iters
                        del gr
                    else:
                        for _ in range(2):
                            full(x)
                        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        torch.cuda.synchronize(device)
                        e0.record()
                        for _ in range(5):
                            full(x)
                        e1.record()
                        torch.cuda.synchronize(device)
                        t1[0] = e0.elapsed_time(e1) / 5
                dist.broadcast(t1, src=0)
            t1 = float(t1.item())
            rec = {"us": round(tp * 1e3, 2), "us_1gpu": round(t1 * 1e3, 2),
                   "efficiency": round(t1 / (world * tp), 4)}
            if M <= 16:
                rec["GB/s"] = round((wbytes + 2 * M * (K + N)) / (tp * 1e-3) / 1e9, 1)
            else:
                rec["TFLOP/s"] = round(2.0 * M * N * K / (tp * 1e-3) / 1e12, 1)
                rec["allgather_us"] = round(coll * 1e3, 2)
            out[f"{N}x{K}/M{M}"] = rec
            del x
        cp.close()
        del cp, full, ql
        torch.cuda.empty_cache()
    return {"config": f"configs[4]: 70B-shaped NF4+DQ layers, LoRA r16 a32, column-sharded over {world} GPUs "
                      "(strong scaling; decode gathers Y in the GEMV, prefill with an NCCL all-gather)",
            "calls": out}


def count_rq_kernels(fn, device):
    """Kernels of this library (namespace rq) that one call of fn launches."""
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize(device)
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize(device)
    return sum(1 for e in prof.events()
               if e.device_type == torch.autograd.DeviceType.CUDA and "rq::" in e.name)


def rotated_modules(layers, wsets):
    """LoRALinear modules sharing the adapters of `layers` but reading the
    rotated weight copies, so the public-API leg streams from HBM too."""
    import copy
    mods = []
    for views in wsets:
        row = []
        for lora, w in zip(layers, views):
            ql = copy.copy(lora.base_layer)
            ql._buffers = dict(lora.base_layer._buffers)
            ql._buffers["weight_quant"] = w.q
            ql._buffers["c2"] = w.c2.view(lora.base_layer.c2.dtype)
            ql._buffers["c2_scales"] = w.c2_scales
            lo = copy.copy(lora)
            lo._modules = dict(lora._modules)
            lo._modules["base_layer"] = ql
            row.append(lo)
        mods.append(row)
    return mods


def run_e2e(args, mods, device, world):
    """Public-API timing: pinned host X -> device, LoRALinear.forward, Y -> host.

    A step's nine inputs sit in one pinned host buffer and go to the device
    in one copy; its nine outputs are gathered into one device buffer and
    come back in one copy (one H2D and one D2H transfer a step)."""
    g = torch.Generator().manual_seed(9)
    calls = [(si, M) for si in range(len(SHAPES)) for M in MS]
    xo, yo, off_x, off_y = {}, {}, 0, 0
    for si, M in calls:
        N, K = SHAPES[si]
        xo[(si, M)], yo[(si, M)] = off_x, off_y
        off_x += M * K
        off_y += M * N
    hx_all = torch.randn(off_x, generator=g).to(torch.bfloat16).pin_memory()
    hy_all = torch.empty(off_y, dtype=torch.bfloat16).pin_memory()
    xd_all = torch.empty(off_x, dtype=torch.bfloat16, device=device)
    yd_all = torch.empty(off_y, dtype=torch.bfloat16, device=device)
    xv = {(si, M): xd_all[xo[(si, M)]:xo[(si, M)] + M * SHAPES[si][1]].view(M, SHAPES[si][1]) for si, M in calls}

    def one(c):
        with torch.no_grad():
            xd_all.copy_(hx_all, non_blocking=True)
            ys = [mods[c % len(mods)][si](xv[(si, M)]).view(-1) for si, M in calls]
            torch.cat(ys, out=yd_all)
            hy_all.copy_(yd_all, non_blocking=True)

    for i in range(max(3, args.warmup)):
        one(i)
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    for i in range(args.steps):
        one(i)
    torch.cuda.synchronize(device)
    dt = time.perf_counter() - t0
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([dt], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = float(t.item())
    step_bytes = sum(algo_bytes(SHAPES[si][0], SHAPES[si][1], M, R) for si, M in calls)
    h2d = sum(M * SHAPES[si][1] * 2 for si, M in calls)
    d2h = sum(M * SHAPES[si][0] * 2 for si, M in calls)
    eager = step_bytes * args.steps * world / dt / 1e9

    # The same step captured once per weight copy in a CUDA graph, each step
    # still copying its inputs from pinned host memory and its outputs back
    # (a decode loop's usual form): replayed and wall-clocked.
    graphs = []
    with torch.no_grad():
        s = torch.cuda.Stream(device)
        s.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(s):
            for c in range(len(mods)):
                one(c)
        torch.cuda.current_stream(device).wait_stream(s)
        torch.cuda.synchronize(device)
        for c in range(len(mods)):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                one(c)
            graphs.append(gr)
    for i in range(max(3, args.warmup)):
        graphs[i % len(graphs)].replay()
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    for i in range(args.steps):
        graphs[i % len(graphs)].replay()
    torch.cuda.synchronize(device)
    dtg = time.perf_counter() - t0
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([dtg], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dtg = float(t.item())
    del graphs
    return {"value": round(step_bytes * args.steps * world / dtg / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "eager_value": round(eager, 2),
            "note": "LoRALinear.forward (each rank its shard) on pinned host inputs: every step copies the nine "
                    "calls' X in (one H2D copy from a pinned buffer) and their Y out (gathered on the device, one "
                    "D2H copy); value = the step captured in CUDA graphs and replayed, eager_value = plain "
                    "Python calls; wall clock, max over ranks"}


# --------------------------------------------------------- CPU reference
def _cpu_layers():
    """The sweep's quantized layers on the host: codes and double-quant
    scales from the C oracle (bit-exact with the reference), adapters."""
    import numpy as np
    from oracle import oracle as orc
    from tests.inputs import layer_inputs
    out = []
    for si, (N, K) in enumerate(SHAPES):
        inp = layer_inputs(N, K, 1, sigma=0.02, r=R, alpha=ALPHA, seed=100 + si)
        wb = inp.W.view(torch.int16).numpy().view(np.uint16).reshape(-1)
        packed, scales = orc.nf4_quantize(wb, orc.BF16, 64)
        c2, c2s = orc.enable_double_quant(packed, scales, orc.BF16, N * K)
        out.append((N, K, torch.from_numpy(packed), torch.from_numpy(c2), torch.from_numpy(c2s), inp.A, inp.B))
    return out


def cpu_baseline(args, layers=None, seconds=12.0):
    """The reference's eager CPU path (torch ops restated in
    oracle/torch_port.py) timed on this host with all its threads."""
    from oracle import torch_port
    torch.set_num_threads(os.cpu_count() or 1)
    layers = layers or _cpu_layers()
    g = torch.Generator().manual_seed(3)
    calls = [(si, M) for si in range(len(SHAPES)) for M in MS]
    done_bytes, t_total, n = 0, 0.0, 0
    while t_total < seconds or n < len(calls):
        si, M = calls[n % len(calls)]
        N, K, packed, c2, c2s, A, B = layers[si]
        x = torch.randn(M, K, generator=g).to(torch.bfloat16)
        t0 = time.perf_counter()
        with torch.no_grad():
            torch_port.loralinear_forward_dq(x, packed, c2, c2s, N, K, A, B, ALPHA / R)
        t_total += time.perf_counter() - t0
        done_bytes += algo_bytes(N, K, M, R)
        n += 1
    return {"value": round(done_bytes / t_total / 1e9, 4), "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{n} LoRALinear forwards of the sweep (torch CPU eager ops of the reference, "
                      f"{t_total:.1f} s)"}


def prefill_cpu_baseline(layers, seconds=6.0):
    """The reference's eager CPU path for the prefill metric (torch ops
    restated in oracle/torch_port.py), timed on this host with all its
    threads on a bounded sample of configs[2]: forward calls of the
    4096x4096 NF4 + double-quant layer at M = 512 with an r = 64 adapter
    (the smallest of the leg's calls), TFLOP/s counted as in prefill_leg."""
    from oracle import torch_port
    from tests.inputs import layer_inputs
    torch.set_num_threads(os.cpu_count() or 1)
    N, K, packed, c2, c2s, _, _ = layers[0]
    inp = layer_inputs(N, K, 1, sigma=0.02, r=PREFILL_R, alpha=PREFILL_ALPHA, seed=200)
    M = PREFILL_MS[0]
    fl = 2.0 * M * N * K + 2.0 * M * PREFILL_R * (K + N)
    g = torch.Generator().manual_seed(5)
    n, t_total = 0, 0.0
    while t_total < seconds or n == 0:
        x = torch.randn(M, K, generator=g).to(torch.bfloat16)
        t0 = time.perf_counter()
        with torch.no_grad():
            torch_port.loralinear_forward_dq(x, packed, c2, c2s, N, K, inp.A, inp.B, PREFILL_ALPHA / PREFILL_R)
        t_total += time.perf_counter() - t0
        n += 1
    return {"value": round(fl * n / t_total / 1e12, 5), "unit": "TFLOP/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{n} LoRALinear forwards of the {N}x{K} layer at M={M}, r={PREFILL_R} "
                      f"(torch CPU eager ops of the reference, {t_total:.1f} s)"}


def run_reference(args, rank, world):
    """--impl reference: the CPU port on rank 0; other ranks exit."""
    if rank != 0:
        return
    layers = _cpu_layers()
    for _ in range(args.warmup):
        cpu_baseline(args, layers, seconds=0.0)
    t0 = time.perf_counter()
    vals = [cpu_baseline(args, layers, seconds=0.0) for _ in range(args.steps)]
    wall = time.perf_counter() - t0
    v = statistics.median(x["value"] for x in vals)
    line = {"metric": METRIC, "value": v, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(wall * 1e3 / args.steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,.) tensors)",
            "impl": "reference",
            "config": {"workload": "configs[1]: decode GEMV sweep (one step = one pass of the 9 calls)",
                       "model": "Llama-2-7B-shaped projections", "global_batch": MS, "seq_len": 1,
                       "parallelism": "host CPU"},
            "cpu_baseline": {**vals[-1], "value": v},
            "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_case(args, device):
    """--case decode:N:K:M[:r] / decode8:... / decode8row:... (int8 blockwise / per-row) or prefill:N:K:M[:r] -- one layer call repeated
    (for profilers; prints the mean CUDA-event time per call)."""
    import torch.nn as nn
    from rocm_qlora import LoRALinear, QuantLinear
    from tests.inputs import layer_inputs
    parts = args.case.split(":")
    if parts[0] == "quant":  # quant:N:K -- rq_nf4_quantize of a bf16 [N, K] weight, repeated
        from rocm_qlora import _native as nat
        N, K = int(parts[1]), int(parts[2])
        L = nat.lib()
        W = (torch.randn(N, K, device=device) * 0.02).to(torch.bfloat16)
        packed = torch.empty(N * K // 2, dtype=torch.uint8, device=device)
        sc = torch.empty(N * K // 64, dtype=torch.bfloat16, device=device)
        st = torch.cuda.current_stream(device).cuda_stream
        fn = lambda: L.rq_nf4_quantize(W.data_ptr(), nat.BF16, N * K, 64, packed.data_ptr(), sc.data_ptr(), st)  # noqa: E731
        for _ in range(3):
            assert fn() == 0
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / args.steps
        n = N * K
        print(json.dumps({"case": args.case, "us_per_call": round(us, 3),
                          "gbs": round((2 * n + n // 2 + 2 * n // 64) / us / 1e3, 1)}))
        return
    kind, N, K, M = parts[0], int(parts[1]), int(parts[2]), int(parts[3])
    r = int(parts[4]) if len(parts) > 4 else R
    inp = layer_inputs(N, K, M, sigma=0.02, r=max(r, 1), alpha=2 * max(r, 1), seed=1, with_dy=kind == "dx")
    lin = nn.Linear(K, N, bias=False, dtype=torch.bfloat16, device=device)
    with torch.no_grad():
        lin.weight.copy_(inp.W.to(device))
    if kind in ("decode8", "decode8row"):  # int8 blockwise / per-row weights
        ql = QuantLinear(K, N, bits=8, bias=False).to(device)
        from rocm_qlora.quantization import quantize_int8
        wq, ws_ = quantize_int8(lin.weight.detach(), per_channel=kind == "decode8row")
        ql.weight_quant, ql.weight_scales = wq, ws_
        kind = "decode"
    else:
        ql = QuantLinear.from_linear(lin, bits=4)
        ql.enable_double_quant()
    lora = LoRALinear(ql, r=max(r, 1), lora_alpha=2 * max(r, 1)).to(device).eval()
    with torch.no_grad():
        lora.lora_A.copy_(inp.A)
        lora.lora_B.copy_(inp.B)
    from rocm_qlora.quantization import layer_ops
    w = ql.weight_view()
    x = inp.X.to(device)
    A = lora.lora_A.detach().bfloat16() if r > 0 else None
    B = lora.lora_B.detach().bfloat16() if r > 0 else None
    # weight copies over >= 512 MB so graph-replayed calls stream from HBM
    per = w.q.numel() + (w.c2.numel() if w.c2 is not None else 0)
    copies = max(1, -(-ROTATE_BYTES // per))
    views = [w] + [type(w)(w.fmt, w.q.clone(), None if w.scales is None else w.scales.clone(),
                           None if w.c2 is None else w.c2.clone(),
                           None if w.c2_scales is None else w.c2_scales.clone(), w.N, w.K, w.block_size)
                   for _ in range(copies - 1)]
    if kind == "dx":
        dy = inp.dY.to(device)
        fn = lambda v: layer_ops.dx(v, dy, A, B, 2.0)  # noqa: E731
    else:
        fn = lambda v: layer_ops.forward(v, x, None, A, B, 2.0)  # noqa: E731
    for _ in range(3):
        fn(w)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        fn(w)
    e1.record()
    torch.cuda.synchronize()
    eager = e0.elapsed_time(e1) * 1e3 / args.steps
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for v in views:
            fn(v)
    torch.cuda.current_stream().wait_stream(s)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        for v in views:
            fn(v)
    gr.replay()
    torch.cuda.synchronize()
    reps = max(1, args.steps // len(views))
    e0.record()
    for _ in range(reps):
        gr.replay()
    e1.record()
    torch.cuda.synchronize()
    graphed = e0.elapsed_time(e1) * 1e3 / (reps * len(views))
    nbytes = algo_bytes(N, K, M, r, lora=r > 0)
    print(json.dumps({"case": args.case, "us_per_call_eager": round(eager, 3), "us_per_call": round(graphed, 3),
                      "gbs": round(nbytes / graphed / 1e3, 1), "copies": len(views)}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default=None, help="single-layer run for profiling, e.g. decode:11008:4096:16")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-prefill", action="store_true", help="skip the configs[2] prefill GEMM leg")
    ap.add_argument("--no-model", action="store_true", help="skip the configs[3] whole-model training step leg")
    ap.add_argument("--gather", choices=["fused", "nccl"], default="fused",
                    help="N > 1: gather Y in the GEMV epilogue over NVLink (fused) or with NCCL all-gather")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if args.case:
        run_case(args, device)
        return
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    try:
        run_ours(args, rank, world, device)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
