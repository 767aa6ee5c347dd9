"""Benchmark: Qwen3-30B-A3B-shaped decode throughput with 4-bit g64 weights
and an 8-bit g64 paged KV cache on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch 64] [--ctx 2048]
    python bench.py --impl reference ...     # the CPU oracle port, same metric

A step is one decode step of all ``--batch`` sequences through all 48 layers
(attention over a ``--ctx``-token quantized context, routed SwiGLU experts,
lm_head, greedy argmax), captured once in a CUDA graph.  ``value`` is device
time with inputs resident in HBM; ``e2e`` adds, every step, the pinned-host
->device copy of the step's token ids and the device->host read of the next
tokens, with the host waiting for each step's tokens before it sends the next
(``pipelined_value``: the same copies queued without that wait).  Weights (~17 GB) and KV (~7 GB) exceed the 126 MB L2, so no flush
is needed between steps.  Under torchrun (N > 1) every rank runs its own
batch of sequences and holds 1/N of every layer's experts (expert parallel,
weak scaling); the slowest rank's time is used.

One JSON line on rank 0.
"""

import argparse
import json
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "mlx-flash_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "decode tok/s (Qwen3-30B-A3B shape, 4-bit)"
PEAKS_FILE = os.path.join(ROOT, "MEASURED_PEAKS.json")


def load_peaks():
    try:
        with open(PEAKS_FILE) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def workload_name(args):
    return (f"Qwen3-30B-A3B-shaped decoder decode step: {args.layers} layers, 32q/4kv heads d128, 128 experts top-8 "
            f"(H 2048, I 768), 4-bit g64 weights, 8-bit g64 KV, batch {args.batch}, context {args.ctx}")


def config_dict(args, world):
    return {"workload": workload_name(args), "batch_per_gpu": args.batch, "global_batch": args.batch * world,
            "context": args.ctx, "layers": args.layers, "weights": "4-bit affine g64 (N(0,0.02) random init)",
            "kv_cache": "8-bit sym g64, paged (64-token pages)", "routing": ("softmax top-8 over x.Wr + a fitted per-expert bias: each token's experts as if "
                        "drawn without replacement from Zipf(1.1) popularity (see routing_fit)"),
            "l2_policy": "inputs larger than L2 (weights ~17 GB, KV ~7 GB), no flush",
            "parallelism": (f"ep{world} experts ("
                            + ("dispatch / combine by the library's NVLink peer-memory kernels"
                               if getattr(args, "ep_exchange", "p2p") == "p2p"
                               else "NCCL all-gather dispatch / reduce-scatter combine")
                            + f"), dp{world} attention") if world > 1 else "1 GPU",
            "expert_placement": (("balanced: each layer's experts relabelled so the ExpertShard blocks carry even "
                                  "expected routing load (greedy longest-first)")
                                 if getattr(args, "ep_placement", "balanced") == "balanced"
                                 else "ExpertShard id blocks over the shuffled popularity") if world > 1 else None}


# ---------------------------------------------------------------------------
class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled while the timed
    region runs: NVML read every 10 ms from a thread (read-only queries), or
    ``nvidia-smi -lms 100`` when NVML is not importable."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.thread = None
        self.samples = []  # (sm_mhz, max_mhz, set of reasons)

    def _bus_id(self):
        """PCI bus id of the CUDA device (NVML and nvidia-smi number devices
        without regard to CUDA_VISIBLE_DEVICES, so the ordinal is not used)."""
        import torch
        pr = torch.cuda.get_device_properties(self.device)
        return f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(self._bus_id())

    def __enter__(self):
        import threading
        try:
            nv, h = self._nvml_handle()
            self.stop = threading.Event()
            mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)

            def run():
                while not self.stop.is_set():
                    sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                    bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    rs = {name for name, attr in self.REASONS if bits & getattr(nv, attr, 0)}
                    self.samples.append((float(sm), float(mx), rs))
                    self.stop.wait(0.01)

            self.thread = threading.Thread(target=run, daemon=True)
            self.thread.start()
        except Exception:
            self.thread = None
            try:
                self.proc = subprocess.Popen(["nvidia-smi", f"--id={self._bus_id()}",
                                              f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                              "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                             text=True)
            except Exception:
                self.proc = None
        return self

    def __exit__(self, *a):
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=5)
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out, _ = self.proc.communicate()
            names = [n for n, _ in self.REASONS]
            for l in out.splitlines():
                f = [x.strip() for x in l.split(",")]
                try:
                    self.samples.append((float(f[1]), float(f[2]),
                                         {n for n, v in zip(names, f[5:9]) if v.lower() == "active"}))
                except (ValueError, IndexError):
                    continue

    def summary(self):
        sm = sorted(x[0] for x in self.samples)
        reasons = set()
        for x in self.samples:
            reasons |= x[2]
        return {"sm_mhz": sm[len(sm) // 2] if sm else None,
                "sm_max_mhz": self.samples[-1][1] if self.samples else None, "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvml" if self.thread is not None else "nvidia-smi"}


# ---------------------------------------------------------------------------
def moe_bytes_per_expert(shape):
    H, I, gs = shape.hidden, shape.moe_inter, shape.group_size
    packed = I * H * shape.bits // 8
    sb = 2 * I * (H // gs) * 2
    return packed + sb  # one [I, H] or [H, I] matrix with its scales and biases


def profile_kernels(dec, torch):
    """One eager step with CUDA events around every launch of the two MoE
    grouped-GEMV kernels and the attention kernel (on the launching stream)."""
    from b200flash import _capi

    st = torch.cuda.current_stream(dec.dev)
    timings = {"moe_gate_up": [], "moe_down": [], "attention": [], "qkv_proj": []}
    orig_call = _capi.call
    pending = []
    state = {"gather": 0}

    def timed_call(name, *args):
        tag = None
        if name in ("b2f_gather_qgemm_affine_mma", "b2f_gather_qgemm_affine_mma_packed") and args[6] == 1:
            # one-expert plan: the dense q/k/v (or o) projection of the batch
            tag = "qkv_proj" if args[13] == dec.qkv_rows else None
        elif name in ("b2f_gather_qgemv_affine", "b2f_gather_qgemm_affine_tcgen05", "b2f_sorted_qgemm_affine_tcgen05",
                      "b2f_gather_qgemm_affine_mma", "b2f_gather_qgemm_affine_mma_packed"):
            tag = "moe_gate_up" if state["gather"] % 2 == 0 else "moe_down"
            state["gather"] += 1
        elif name == "b2f_qkv_decode_attn":
            tag = "attention"
        elif name in ("b2f_qgemv_affine", "b2f_qgemm_affine_tcgen05_splitk", "b2f_qgemm_affine_tcgen05_partials") \
                and args[6] == dec.qkv_rows:
            tag = "qkv_proj"
        if tag is None:
            return orig_call(name, *args)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(st)
        rc = orig_call(name, *args)
        e1.record(st)
        pending.append((tag, e0, e1))
        return rc

    import b200flash.decoder as dmod

    routed = []
    chosen = []
    dmod.call = timed_call
    try:
        # record the routing of every layer for the algorithmic byte count
        orig_route = timed_call

        def route_and_keep(name, *args):
            rc = orig_route(name, *args)
            if name in ("b2f_moe_route_topk", "b2f_moe_route_plan"):
                chosen.append(dec.inds.clone())
            if name in ("b2f_moe_route_topk", "b2f_moe_route_plan") and dec.ep is None:
                routed.append(dec.inds.clone())
            elif name == "b2f_ep_plan":
                loc = dec.ep.local.clone()
                routed.append(loc[loc >= 0])
            return rc

        import b200flash.ep as epmod

        dmod.call = route_and_keep
        epmod.call = route_and_keep
        dec.step()
    finally:
        dmod.call = orig_call
        epmod.call = orig_call
    torch.cuda.synchronize()
    for tag, e0, e1 in pending:
        timings[tag].append(e0.elapsed_time(e1) * 1e-3)
    # per layer: distinct experts this rank computes, and its assignments
    distinct = [(int(torch.unique(r).numel()), int(r.numel())) for r in routed]
    return timings, distinct, chosen


def routing_fit(dec, chosen):
    """Realised routing of one step against the Zipf(s) target: per layer the
    distinct experts the batch hit and the selection frequency of each
    popularity rank; mean over layers."""
    import numpy as np

    from b200flash.decoder import expected_distinct_experts, zipf_selection_frequency

    s = dec.s
    target = zipf_selection_frequency(s.n_experts, s.top_k, s.zipf_s)
    freq = np.zeros(s.n_experts)
    distinct = []
    for ly, inds in zip(dec.layers, chosen):
        rank = ly["zipf_rank"].to(inds.device)[inds.long()].reshape(-1)
        freq += np.bincount(rank.cpu().numpy(), minlength=s.n_experts) / inds.shape[0]
        distinct.append(int(torch_unique_count(inds)))
    freq /= max(1, len(chosen))
    B = chosen[0].shape[0] if chosen else 0
    return {"target": f"each token's top-{s.top_k} drawn without replacement from p_r ~ r^-{s.zipf_s} "
                      f"over {s.n_experts} experts",
            "tokens_per_layer": B,
            "distinct_experts_per_layer": round(float(np.mean(distinct)), 1) if distinct else None,
            "distinct_experts_expected": round(expected_distinct_experts(target, B), 1),
            "freq_max_abs_dev": round(float(np.abs(freq - target).max()), 4),
            "freq_top4": [round(float(v), 3) for v in freq[:4]],
            "freq_top4_target": [round(float(v), 3) for v in target[:4]],
            "layers": len(chosen)}


def torch_unique_count(t):
    import torch

    return torch.unique(t).numel()


# DRAM bytes moved per algorithmic byte, from ncu captures of the kernels the
# step runs, on the 2-layer copy of this decode step (dram__bytes_read.sum +
# dram__bytes_write.sum over the launch's algorithmic bytes; see
# profiles/qgemm_mma_packed_moe_b64_2layer_zipf_ncu.txt and
# profiles/qkv_decode_attn_b64_ctx2048.txt).  The per-layer shapes are those of
# the 48-layer step, so traffic scales with the units a launch processes.  The
# expert GEMMs' algorithmic bytes are the 2-layer run's mean per launch (the
# capture is layer 0's launch).
NCU_TRAFFIC_RATIO = {"attention": (147.63648 + 4.275712) / 144.142336,
                     "moe_gate_up": (168.513024 + 4.78976) / 178.946048,
                     "moe_down": (84.907008 + 2.450176) / 90.914816}


def attention_bytes(dec, ctx):
    s = dec.s
    per_tok = s.n_kv_heads * 2 * (dec.rb + 4 * (s.head_dim // 64))
    return dec.B * ctx * per_tok + 2 * dec.B * s.n_heads * s.head_dim * 2


# ---------------------------------------------------------------------------
def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))

    from b200flash.decoder import Qwen3MoeDecoder, Qwen3MoeShape
    from b200flash.ep import EPExchange, PeerExchange

    shape = Qwen3MoeShape()
    max_ctx = args.ctx + args.warmup * 3 + args.steps * 3 + 8
    # N > 1: experts sharded expert-parallel (ExpertShard blocks), attention,
    # router and lm_head data-parallel over each rank's own batch
    # N > 1: the decode exchange runs on the library's peer-memory kernels
    # (--ep-exchange p2p) or on NCCL all-gather / reduce-scatter (nccl)
    exchange = (PeerExchange() if args.ep_exchange == "p2p" else EPExchange()) if world > 1 else None
    dec = Qwen3MoeDecoder(shape, max_batch=args.batch, max_context=max_ctx, page_size=64, device=dev,
                          seed=1234, layers=args.layers, exchange=exchange, moe_engine=args.moe_engine,
                          dense_engine=args.dense_engine, moe_tile=args.moe_tile,
                          moe_packed=not args.moe_unpacked, pdl=not args.no_pdl,
                          moe_streamk=args.streamk, expert_placement=args.ep_placement)
    dec.fill_random_context(args.ctx)
    torch.cuda.synchronize()

    # eager warm-up then graph capture
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        dec.step()
    torch.cuda.current_stream(dev).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        dec.step()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clk:
        if args.profile_window:
            torch.cuda.profiler.start()
        e0.record()
        for _ in range(args.steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        if args.profile_window:
            torch.cuda.profiler.stop()
    barrier()
    t = e0.elapsed_time(e1) * 1e-3
    t_max = t
    if world > 1:
        tt = torch.tensor([t], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_max = float(tt.item())
    tokens_total = args.batch * world * args.steps
    value = tokens_total / t_max

    # end to end: token ids from pinned host memory in, next tokens out, every step
    host_in = torch.empty(args.batch, dtype=torch.int32).pin_memory()
    host_out = torch.empty(args.batch, dtype=torch.int32).pin_memory()
    host_in.copy_(dec.next_tokens.cpu())
    barrier()
    torch.cuda.synchronize()
    f0 = torch.cuda.Event(enable_timing=True)
    f1 = torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream(dev)
    # a decode loop: every step's next tokens are on the host (sampling, EOS
    # checks) before the next step's ids go up, so the host waits each step
    f0.record()
    for _ in range(args.steps):
        dec.tokens.copy_(host_in, non_blocking=True)
        graph.replay()
        host_out.copy_(dec.next_tokens, non_blocking=True)
        stream.synchronize()
        host_in.copy_(host_out)
    f1.record()
    torch.cuda.synchronize()
    te = f0.elapsed_time(f1) * 1e-3
    # the same copies queued back to back (no host wait between steps)
    f0.record()
    for _ in range(args.steps):
        dec.tokens.copy_(host_in, non_blocking=True)
        graph.replay()
        host_out.copy_(dec.next_tokens, non_blocking=True)
    f1.record()
    torch.cuda.synchronize()
    tp = f0.elapsed_time(f1) * 1e-3
    if world > 1:
        tt = torch.tensor([te, tp], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        te, tp = float(tt[0].item()), float(tt[1].item())
    e2e = tokens_total / te
    e2e_pipelined = tokens_total / tp

    # live per-kernel timing (eager step, events on the launching stream)
    timings, distinct, chosen = profile_kernels(dec, torch)
    rfit = routing_fit(dec, chosen)
    peak, peak_kind = load_peaks()
    per_exp = moe_bytes_per_expert(shape)
    gu_bytes = [2 * u * per_exp + a * shape.hidden * 2 + a * shape.moe_inter * 2 for u, a in distinct]
    dn_bytes = [u * per_exp + a * shape.moe_inter * 2 + a * shape.hidden * 2 for u, a in distinct]
    ctx_now = int(dec.positions[0].item())
    at_bytes = attention_bytes(dec, ctx_now)
    kernels = {}
    for tag, byts in (("moe_gate_up", gu_bytes), ("moe_down", dn_bytes), ("attention", [at_bytes] * dec.L)):
        ts = timings[tag]
        if ts:
            tot_b = sum(byts[: len(ts)])
            kernels[tag] = {"launches": len(ts), "avg_us": 1e6 * sum(ts) / len(ts),
                            "total_ms": 1e3 * sum(ts), "bytes_per_launch": tot_b / len(ts),
                            "gbs": tot_b / sum(ts) / 1e9}
    dom = max(kernels, key=lambda k: kernels[k]["total_ms"])
    d = kernels[dom]
    roofline = {"kernel": dom, "bound": "hbm", "achieved": round(d["gbs"], 1), "peak": peak,
                "peak_kind": peak_kind, "unit": "GB/s", "frac": round(d["gbs"] / peak, 4),
                "traffic": (int(d["bytes_per_launch"] * NCU_TRAFFIC_RATIO[dom]) if dom in NCU_TRAFFIC_RATIO
                            else None),
                "traffic_source": ("ncu DRAM read + write bytes / algorithmic bytes on the 2-layer capture, times this "
                                   "launch's algorithmic bytes" if dom in NCU_TRAFFIC_RATIO
                                   else "no ncu capture with read and write bytes"),
                "bytes_per_launch": int(d["bytes_per_launch"]),
                "avg_launch_us": round(d["avg_us"], 2),
                "distinct_experts_per_layer": round(sum(u for u, _ in distinct) / max(1, len(distinct)), 1)}
    result = {
        "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(1e3 * t_max / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random weights, random context, seeded)",
        "config": config_dict(args, world),
        "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": args.batch * 4,
                "d2h_bytes_per_step": args.batch * 4, "host_sync_per_step": True,
                "pipelined_value": round(e2e_pipelined, 2)},
        "gpu_launches": dec.launches_per_step() * args.steps,
        "roofline": roofline,
        "kernels": {k: {kk: (round(vv, 2) if isinstance(vv, float) else vv) for kk, vv in v.items()}
                    for k, v in kernels.items()},
        "clocks": clk.summary(),
        "routing_fit": rfit,
        "weight_bytes": dec.weight_bytes(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(args, shape)
    del graph
    if world > 1 and args.strong_batch:
        # strong scaling: the same global batch spread over the N ranks
        del dec
        torch.cuda.empty_cache()
        result["strong_scaling"] = strong_scaling(args, shape, world, dev, exchange, max_ctx)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


# ---------------------------------------------------------------------------
# Per-op workloads (single linear, quantized-KV decode attention, one MoE
# layer): each prints its own JSON line; the default run is the decode step.
def _graph_time(launch, reps, iters, dev):
    """Seconds per call of ``launch(i)``: ``reps`` calls on rotating buffers
    captured in one CUDA graph, replayed ``iters`` times after 3 warm-ups
    (CUDA events on the replaying stream)."""
    import torch

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for i in range(reps):
            launch(i)
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(reps):
            launch(i)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        g.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    del g
    return e0.elapsed_time(e1) * 1e-3 / (iters * reps)


def _op_line(args, metric, value, unit, config, extra, peak, peak_kind, kernels, cpu=None, higher=True):
    line = {"metric": metric, "value": round(value, 2), "unit": unit, "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": higher, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded random weights / activations)", "config": config,
            "kernels": kernels, "peak": {"hbm_gbs": peak, "kind": peak_kind}}
    line.update(extra)
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


def run_linear(args):
    """Single 4-bit affine linear W[4096, 4096], x[8, 4096]: quantize (the
    workload's min/max rule), quantized_matmul, dequantize."""
    import numpy as np
    import torch

    from b200flash import _capi
    from b200flash._capi import call, ptr
    from b200flash.mx_compat import tc_ksplit

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    N = K = 4096
    M, gs, bits = 8, 64, 4
    gen = torch.Generator(device=dev)
    gen.manual_seed(0)
    peak, peak_kind = load_peaks()
    nq = 8  # 8 x 32 MB of bf16 weights per rotation: beyond the 126 MB L2
    Ws = [(torch.randn(N, K, device=dev, generator=gen) * 0.02).to(torch.bfloat16) for _ in range(nq)]
    wq = [torch.empty(N, K * bits // 32, dtype=torch.uint32, device=dev) for _ in range(16)]
    sc = [torch.empty(N, K // gs, dtype=torch.bfloat16, device=dev) for _ in range(16)]
    bi = [torch.empty(N, K // gs, dtype=torch.bfloat16, device=dev) for _ in range(16)]
    for i in range(16):
        call("b2f_quantize_affine_minmax", ptr(Ws[i % nq]), 0, N, K, bits, gs, ptr(wq[i]), ptr(sc[i]), ptr(bi[i]), _capi.stream_of(dev))
    x = torch.randn(M, K, device=dev, generator=gen).to(torch.bfloat16)
    y = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    deq = [torch.empty(N, K, dtype=torch.bfloat16, device=dev) for _ in range(nq)]
    q_bytes = N * K * 2 + N * K * bits // 8 + 2 * N * (K // gs) * 2
    mm_bytes = N * K * bits // 8 + 2 * N * (K // gs) * 2 + M * K * 2 + M * N * 2
    it = max(args.steps, 20)

    def quant(i):
        call("b2f_quantize_affine_minmax", ptr(Ws[i]), 0, N, K, bits, gs, ptr(wq[i]), ptr(sc[i]), ptr(bi[i]), _capi.stream_of(dev))

    def quant_mlx(i):
        call("b2f_quantize_affine", ptr(Ws[i]), 0, N, K, bits, gs, ptr(wq[i]), ptr(sc[i]), ptr(bi[i]), _capi.stream_of(dev))

    def dequant(i):
        call("b2f_dequantize_affine", ptr(wq[i]), ptr(sc[i]), ptr(bi[i]), 0, N, K, bits, gs, 0, ptr(deq[i]), _capi.stream_of(dev))

    def gemv(i):
        call("b2f_qgemv_affine", ptr(x), K, M, ptr(wq[i]), ptr(sc[i]), ptr(bi[i]), N, K, bits, gs, 0, ptr(y), N, _capi.stream_of(dev))

    ks = tc_ksplit(N, K, torch.cuda.get_device_properties(dev).multi_processor_count)
    wsb = int(_capi.lib().b2f_qgemm_splitk_workspace_bytes(M, N, ks))
    tws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=dev)

    def tcsplit(i):
        call("b2f_qgemm_affine_tcgen05_splitk", ptr(x), K, M, ptr(wq[i]), ptr(sc[i]), ptr(bi[i]), N, K, bits, gs, 0,
             ptr(y), N, 16, ks, ptr(tws), wsb, _capi.stream_of(dev))

    t = {"quantize_minmax": _graph_time(quant, nq, it, dev), "quantize_mlx": _graph_time(quant_mlx, nq, it, dev),
         "dequantize": _graph_time(dequant, nq, it, dev), "qmm_gemv": _graph_time(gemv, 16, it * 4, dev),
         "qmm_tc_splitk": _graph_time(tcsplit, 16, it * 4, dev)}
    byts = {"quantize_minmax": q_bytes, "quantize_mlx": q_bytes, "dequantize": q_bytes, "qmm_gemv": mm_bytes,
            "qmm_tc_splitk": mm_bytes}
    kernels = {k: {"us": round(v * 1e6, 2), "bytes": byts[k], "gbs": round(byts[k] / v / 1e9, 1),
                   "frac": round(byts[k] / v / 1e9 / peak, 4)} for k, v in t.items()}
    best = min(("qmm_gemv", "qmm_tc_splitk"), key=lambda k: t[k])
    cpu = None
    if not args.no_cpu_baseline:
        from oracle import affine
        from oracle.fp import round_bf16

        w = round_bf16(np.random.default_rng(0).normal(0, 0.02, (N, K)).astype(np.float32))
        xx = round_bf16(np.random.default_rng(1).standard_normal((M, K)).astype(np.float32))
        c0 = time.perf_counter()
        owq, osc, obi = affine.quantize(w, gs, bits, rule="minmax")
        c1 = time.perf_counter()
        affine.quantized_matmul(xx, owq, osc, obi, True, gs, bits)
        c2 = time.perf_counter()
        affine.dequantize(owq, osc, obi, gs, bits)
        c3 = time.perf_counter()
        cpu = {"value": round(mm_bytes / (c2 - c1) / 1e9, 3), "unit": "GB/s", "cores": cpu_threads(), "kind": "port",
               "sample": (f"NumPy oracle on the full shape: quantize {c1 - c0:.2f} s, quantized_matmul "
                          f"{c2 - c1:.2f} s, dequantize {c3 - c2:.2f} s")}
    _op_line(args, "single 4-bit linear: quantized_matmul HBM GB/s (W 4096x4096 g64, x[8,4096])",
             kernels[best]["gbs"], "GB/s",
             {"workload": "single 4-bit affine linear W[4096,4096] ~N(0,0.02) bf16, group 64, x[8,4096] ~N(0,1)",
              "l2_policy": "8 weight copies (quantize / dequantize) and 16 packed copies (qmm) rotated per graph"},
             {"roofline": {"kernel": best, "bound": "hbm", "achieved": kernels[best]["gbs"], "peak": peak,
                           "unit": "GB/s", "frac": kernels[best]["frac"], "traffic": None},
              "ms_per_step": round(t[best] * 1e3, 5)}, peak, peak_kind, kernels, cpu)


def run_kv_attention(args):
    """Quantized-KV decode attention, Llama-3-8B heads (32q / 8kv, d 128),
    batch 16 x context 8192, 8- and 4-bit KV in 64-token head-major pages;
    plus the pack of a 512-token prefill chunk of all 16 sequences."""
    import torch

    from b200flash import _capi
    from b200flash._capi import call, ptr
    from b200flash.quantized_kv_cache import packed_len, pick_splits

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, ctx, Hq, Hkv, D, page = 16, 8192, 32, 8, 128, 64
    peak, peak_kind = load_peaks()
    gen = torch.Generator(device=dev)
    gen.manual_seed(0)
    npg = ctx // page
    bt = torch.arange(B * npg, dtype=torch.int32, device=dev).reshape(B, npg)
    sl = torch.full((B,), ctx, dtype=torch.int32, device=dev)
    q = torch.randn(B, Hq, D, device=dev, generator=gen).to(torch.bfloat16)
    out = torch.empty(B, Hq, D, dtype=torch.bfloat16, device=dev)
    ns = pick_splits(B, Hkv, ctx)
    wsb = int(_capi.lib().b2f_qkv_decode_attn_workspace_bytes(B, Hq, D, ns))
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=dev)
    kernels = {}
    it = max(args.steps, 20)
    for bits in (8, 4):
        rb = packed_len(D, bits, 64)
        pools = []
        for _ in range(2):  # two pools alternate: each step reads KV the previous step did not
            kc = torch.randint(0, 256, (B * npg, Hkv, page, rb), dtype=torch.uint8, device=dev, generator=gen)
            vc = torch.randint(0, 256, (B * npg, Hkv, page, rb), dtype=torch.uint8, device=dev, generator=gen)
            ks = torch.empty(B * npg, Hkv, page, D // 64, device=dev).uniform_(0.015, 0.03, generator=gen)
            vs = torch.empty_like(ks).uniform_(0.015, 0.03, generator=gen)
            pools.append((kc, ks, vc, vs))

        def attn(i, bits=bits, pools=pools):
            kc, ks, vc, vs = pools[i]
            call("b2f_qkv_decode_attn", ptr(q), ptr(kc), ptr(ks), ptr(vc), ptr(vs), ptr(bt), npg, ptr(sl), B, Hq, Hkv,
                 D, page, page, 1, bits, 64, D ** -0.5, ns, ptr(ws), wsb, ptr(out), _capi.stream_of(dev))

        tt = _graph_time(attn, 2, it, dev)
        byts = B * ctx * Hkv * 2 * (rb + 4 * (D // 64)) + 2 * B * Hq * D * 2
        kernels[f"attention_{bits}bit"] = {"us": round(tt * 1e6, 2), "bytes": byts, "gbs": round(byts / tt / 1e9, 1),
                                           "frac": round(byts / tt / 1e9 / peak, 4),
                                           "frac_of_8tbs": round(byts / tt / 8e12, 4)}
        del pools
        # the pack of a 512-token chunk of K and V (16 sequences x 8 heads rows)
        rows = B * 512 * Hkv
        xs = [torch.randn(rows, D, device=dev, generator=gen).to(torch.bfloat16) for _ in range(8)]
        pk = torch.empty(rows, rb, dtype=torch.uint8, device=dev)
        psc = torch.empty(rows, D // 64, dtype=torch.float32, device=dev)

        def pack(i, bits=bits, rb=rb):
            call("b2f_kv_quantize_sym", ptr(xs[i]), 0, rows, D, bits, 64, 0, ptr(pk), rb, ptr(psc), 0, D // 64, _capi.stream_of(dev))

        tp = _graph_time(pack, 8, it, dev) * 2  # K and V
        pb = 2 * (rows * D * 2 + rows * rb + rows * (D // 64) * 4)
        kernels[f"pack512_{bits}bit"] = {"us": round(tp * 1e6, 2), "bytes": pb, "gbs": round(pb / tp / 1e9, 1),
                                         "frac": round(pb / tp / 1e9 / peak, 4)}
        del xs
    cpu = None
    if not args.no_cpu_baseline:
        import numpy as np

        from oracle import attn as oattn
        from oracle import kv_sym

        rng = np.random.default_rng(0)
        kc = rng.integers(0, 255, (ctx, Hkv, D), dtype=np.uint8)
        ks = rng.uniform(0.015, 0.03, (ctx, Hkv, 2)).astype(np.float32)
        qq = rng.standard_normal((1, Hq, D)).astype(np.float32)
        c0 = time.perf_counter()
        kd = kv_sym.dequantize_tensor(kc, ks, 0 * ks, 8, (ctx, Hkv, D), 64)
        vd = kv_sym.dequantize_tensor(kc[::-1].copy(), ks, 0 * ks, 8, (ctx, Hkv, D), 64)
        oattn.decode_attention(qq, [kd], [vd])
        c1 = time.perf_counter()
        byts8 = kernels["attention_8bit"]["bytes"]
        cpu = {"value": round(byts8 / (16 * (c1 - c0)) / 1e9, 3), "unit": "GB/s", "cores": cpu_threads(),
               "kind": "port", "sample": f"NumPy oracle, 8-bit, 1 of 16 sequences at context {ctx}: {c1 - c0:.2f} s, x16"}
    k8 = kernels["attention_8bit"]
    _op_line(args, "quantized-KV decode attention HBM GB/s (8-bit KV, B16 x ctx 8192, 32q/8kv d128)", k8["gbs"], "GB/s",
             {"workload": "decode attention over 8-bit (and 4-bit) g64 KV, batch 16, context 8192, 32 query / 8 KV "
                          "heads, head_dim 128, 64-token pages; pack of a 512-token chunk",
              "l2_policy": "two KV pools alternate (each > 126 MB); 8 pack inputs rotate"},
             {"roofline": {"kernel": "attention_8bit", "bound": "hbm", "achieved": k8["gbs"], "peak": peak,
                           "unit": "GB/s", "frac": k8["frac"], "traffic": None},
              "ms_per_step": round(k8["us"] / 1e3, 5), "context_splits": ns}, peak, peak_kind, kernels, cpu)


def run_moe_layer(args):
    """One Qwen3-30B-A3B-shaped MoE layer (128 experts, top-8, H 2048, I 768,
    4-bit g64) with Zipf(1.1) routing at 1, 32 and 512 tokens: router + plan,
    SwiGLU gate/up, down, weighted combine."""
    import numpy as np
    import torch

    from b200flash import _capi
    from b200flash._capi import call, ptr
    from b200flash.decoder import random_qweight, zipf_router_bias

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    E, k, H, I, bits, gs = 128, 8, 2048, 768, 4, 64
    tau = 1.3
    peak, peak_kind = load_peaks()
    gen = torch.Generator(device=dev)
    gen.manual_seed(0)
    L = 8  # layer copies rotated per graph: 8 x 340 MB of experts
    beta = torch.from_numpy(np.array(zipf_router_bias(E, k, 1.1, tau))).to(dev)
    layers = []
    for _ in range(L):
        perm = torch.randperm(E, device=dev, generator=gen)
        layers.append({"g": random_qweight((E, I, H), bits, gs, dev, gen), "u": random_qweight((E, I, H), bits, gs, dev, gen),
                       "d": random_qweight((E, H, I), bits, gs, dev, gen),
                       "wr": (torch.randn(E, H, device=dev, generator=gen) * (tau / H ** 0.5)).to(torch.bfloat16),
                       "rb": beta[perm].contiguous()})
        ly = layers[-1]
        for name, mat in (("g", 2), ("u", 2), ("d", 1)):
            w = ly[name]
            nbytes = int(_capi.lib().b2f_mma_packed_bytes(E, w.N, w.K, mat))
            ly[name + "_packed"] = torch.empty(nbytes, dtype=torch.uint8, device=dev)
            call("b2f_mma_repack", ptr(w.wq), ptr(w.scales), ptr(w.biases), E, w.N, w.K, mat,
                 ptr(ly[name + "_packed"]), nbytes, _capi.stream_of(dev))
    per_exp = 3 * (I * H * bits // 8 + 2 * I * (H // gs) * 2)
    ones = torch.ones(H, dtype=torch.bfloat16, device=dev)
    results = {}
    lib = _capi.lib()
    # stream-K workspace of the packed expert GEMM (zeroed once; left zeroed)
    skb = int(lib.b2f_mma_streamk_workspace_bytes())
    skw_t = torch.zeros(skb, dtype=torch.uint8, device=dev)
    skw = ptr(skw_t) if args.streamk else 0
    for T in (1, 32, 512):
        A = T * k
        x = torch.randn(T, H, device=dev, generator=gen).to(torch.bfloat16)
        zeros = torch.zeros(T, H, dtype=torch.bfloat16, device=dev)
        gates = torch.empty(T, E, dtype=torch.float32, device=dev)
        inds = [torch.empty(T, k, dtype=torch.int32, device=dev) for _ in range(L)]
        scores = torch.empty(T, k, dtype=torch.float32, device=dev)
        hh = torch.empty(A, I, dtype=torch.bfloat16, device=dev)
        xs = torch.empty(A, H, dtype=torch.bfloat16, device=dev)
        y = torch.empty(A, H, dtype=torch.bfloat16, device=dev)
        out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        scratch = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        engines = ["mma", "mma_mlx"] + (["tc_sorted"] if T >= 32 else []) + (["gemv"] if T <= 32 else [])
        for eng in engines:
            tile = 16 if eng in ("mma", "mma_mlx", "gemv") else (64 if A >= 64 * E else 32)
            pb = int(lib.b2f_moe_plan_workspace_bytes(A, E, tile))
            pws = torch.empty(pb, dtype=torch.uint8, device=dev)

            def layer(i, eng=eng, tile=tile, pws=pws, pb=pb):
                ly = layers[i]
                g, u, d = ly["g"], ly["u"], ly["d"]
                call("b2f_moe_route_plan", ptr(x), T, H, ptr(ly["wr"]), ptr(ly["rb"]), E, k, 1, ptr(gates),
                     ptr(inds[i]), ptr(scores), tile, ptr(pws), pb, ptr(status), _capi.stream_of(dev))
                if eng == "gemv":
                    call("b2f_gather_qgemv_affine", ptr(x), H, 0, k, A, E, ptr(g.wq), ptr(g.scales), ptr(g.biases),
                         ptr(u.wq), ptr(u.scales), ptr(u.biases), I, H, bits, gs, tile, ptr(pws), pb, ptr(hh), I,
                         _capi.stream_of(dev))
                    call("b2f_gather_qgemv_affine", ptr(hh), I, 0, 1, A, E, ptr(d.wq), ptr(d.scales), ptr(d.biases),
                         0, 0, 0, H, I, bits, gs, tile, ptr(pws), pb, ptr(y), H, _capi.stream_of(dev))
                elif eng == "mma":
                    # packed tiles (the decoder's layout): codes + scales in one copy per tile
                    call("b2f_gather_qgemm_affine_mma_packed", ptr(x), H, 0, k, 0, A, E, ptr(ly["g_packed"]),
                         ptr(ly["u_packed"]), I, H, bits, gs, tile, ptr(pws), pb, ptr(hh), I, 1, skw, skb, 0,
                         _capi.stream_of(dev))
                    call("b2f_gather_qgemm_affine_mma_packed", ptr(hh), I, 0, 1, 1, A, E, ptr(ly["d_packed"]), 0, H,
                         I, bits, gs, tile, ptr(pws), pb, ptr(y), H, 0, skw, skb, 0, _capi.stream_of(dev))
                elif eng == "mma_mlx":
                    call("b2f_gather_qgemm_affine_mma", ptr(x), H, 0, k, 0, A, E, ptr(g.wq), ptr(g.scales),
                         ptr(g.biases), ptr(u.wq), ptr(u.scales), ptr(u.biases), I, H, bits, gs, tile, ptr(pws), pb,
                         ptr(hh), I, 1, _capi.stream_of(dev))
                    call("b2f_gather_qgemm_affine_mma", ptr(hh), I, 0, 1, 1, A, E, ptr(d.wq), ptr(d.scales),
                         ptr(d.biases), 0, 0, 0, H, I, bits, gs, tile, ptr(pws), pb, ptr(y), H, 0, _capi.stream_of(dev))
                else:
                    call("b2f_moe_gather_rows", ptr(x), H, 0, k, A, E, tile, ptr(pws), pb, H, ptr(xs), H, _capi.stream_of(dev))
                    call("b2f_sorted_qgemm_affine_tcgen05", ptr(xs), H, A, E, ptr(g.wq), ptr(g.scales), ptr(g.biases),
                         ptr(u.wq), ptr(u.scales), ptr(u.biases), I, H, bits, gs, tile, ptr(pws), pb, ptr(hh), I, 1,
                         _capi.stream_of(dev))
                    call("b2f_sorted_qgemm_affine_tcgen05", ptr(hh), I, A, E, ptr(d.wq), ptr(d.scales),
                         ptr(d.biases), 0, 0, 0, H, I, bits, gs, tile, ptr(pws), pb, ptr(y), H, 0, _capi.stream_of(dev))
                call("b2f_combine_rmsnorm", ptr(zeros), ptr(y), ptr(scores), T, k, ptr(ones), 1e-6, H, ptr(out),
                     ptr(scratch), _capi.stream_of(dev))

            tt = _graph_time(layer, L, max(args.steps, 10), dev)
            U = float(np.mean([torch.unique(inds[i]).numel() for i in range(L)]))
            byts = U * per_exp + E * H * 2 + 2 * T * H * 2
            flops = 2.0 * A * 3 * H * I
            results[f"T{T}_{eng}"] = {"us": round(tt * 1e6, 2), "distinct_experts": round(U, 1),
                                      "bytes": int(byts), "gbs": round(byts / tt / 1e9, 1),
                                      "frac": round(byts / tt / 1e9 / peak, 4), "tflops": round(flops / tt / 1e12, 2)}
    best = {T: min((v for kk, v in results.items() if kk.startswith(f"T{T}_")), key=lambda v: v["us"])
            for T in (1, 32, 512)}
    cpu = None
    if not args.no_cpu_baseline:
        from oracle import affine
        from oracle import moe as omoe

        rng = np.random.default_rng(0)
        xx = rng.standard_normal((32, H)).astype(np.float32)
        wrn = rng.normal(0, tau / H ** 0.5, (E, H)).astype(np.float32)
        oi, os_ = omoe.route(xx, wrn.T, k, bias=np.array(zipf_router_bias(E, k, 1.1, tau)))
        used = sorted(set(oi.ravel().tolist()))
        mk = {e: tuple(affine.quantize(rng.normal(0, 0.02, shp).astype(np.float32), gs, bits)
                       for shp in ((I, H), (I, H), (H, I))) for e in used}
        c0 = time.perf_counter()
        dq = {e: tuple(affine.dequantize_f32(*m, gs, bits).astype(np.float64) for m in mk[e]) for e in used}
        for t in range(32):
            for j in range(k):
                g_, u_, d_ = dq[int(oi[t, j])]
                hv = omoe.silu(g_ @ xx[t]) * (u_ @ xx[t])
                _ = d_ @ hv
        c1 = time.perf_counter()
        cpu = {"value": round(32 / (c1 - c0), 3), "unit": "tokens/s", "cores": cpu_threads(), "kind": "port",
               "sample": f"NumPy oracle MoE layer at 32 tokens ({len(used)} experts): {c1 - c0:.2f} s"}
    b32 = best[32]
    _op_line(args, "Qwen3-30B-A3B-shaped MoE layer (4-bit g64, Zipf(1.1) top-8): HBM GB/s at 32 tokens",
             b32["gbs"], "GB/s",
             {"workload": "one MoE layer: 128 experts top-8, H 2048, I 768, SwiGLU, 4-bit g64 N(0,0.02); router "
                          "x.Wr + fitted Zipf(1.1) bias; 1 / 32 / 512 tokens x ~N(0,1)",
              "l2_policy": f"{L} layer copies (340 MB of experts each) rotated per graph"},
             {"roofline": {"kernel": "moe_layer_T32", "bound": "hbm", "achieved": b32["gbs"], "peak": peak,
                           "unit": "GB/s", "frac": b32["frac"], "traffic": None},
              "ms_per_step": round(b32["us"] / 1e3, 5), "per_tokens": results}, peak, peak_kind, results, cpu)


def run_ds_prefill(args):
    """DeepSeek-V3-shaped MoE layer at prefill: 256 routed experts (top-8,
    sigmoid gates, the hottest 10% taking 40% of assignments) + 1 shared
    expert, H 7168, I 2048, SwiGLU, 4-bit g64; 4096 tokens over N ranks
    (4096/N each), experts sharded in ExpertShard blocks, tokens moved by the
    counts-then-rows NCCL all-to-all (b200flash.ep_a2a).  One step = router,
    dispatch, local experts, return, combine and the shared expert."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from b200flash import _capi
    from b200flash._capi import call, ptr
    from b200flash.decoder import fit_router_bias, hot_set_frequency, random_qweight
    from b200flash.distributed_experts import ExpertShard
    from b200flash.ep import EPExchange
    from b200flash.ep_a2a import ExpertParallelA2A

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    E, k, H, I, bits, gs = args.experts, 8, 7168, 2048, 4, 64
    T_all = args.tokens
    T = T_all // world
    tau = 1.3
    gen = torch.Generator(device=dev)
    gen.manual_seed(100 + rank)
    shard = ExpertShard(rank=rank, world_size=world, total_experts=E)
    E_loc = len(shard.owned_experts)
    g = random_qweight((E_loc, I, H), bits, gs, dev, gen)
    u = random_qweight((E_loc, I, H), bits, gs, dev, gen)
    dn = random_qweight((E_loc, H, I), bits, gs, dev, gen)
    sg = random_qweight((1, I, H), bits, gs, dev, gen)
    su = random_qweight((1, I, H), bits, gs, dev, gen)
    sd = random_qweight((1, H, I), bits, gs, dev, gen)
    rgen = torch.Generator(device=dev)
    rgen.manual_seed(7)  # the router is the same on every rank
    perm = torch.randperm(E, device=dev, generator=rgen)
    beta = torch.from_numpy(np.array(fit_router_bias(hot_set_frequency(E, k, 0.1, 0.4), k, tau))).to(dev)
    rbias = torch.empty_like(beta)
    rbias[perm] = beta  # expert perm[i] takes the i-th frequency (the hot set first)
    wr = (torch.randn(E, H, device=dev, generator=rgen) * (tau / H ** 0.5)).to(torch.bfloat16)
    x = torch.randn(T, H, device=dev, generator=gen).to(torch.bfloat16)
    gates = torch.empty(T, E, dtype=torch.float32, device=dev)
    inds = torch.empty(T, k, dtype=torch.int32, device=dev)
    scores = torch.empty(T, k, dtype=torch.float32, device=dev)
    ex = EPExchange() if world > 1 else None
    ep = ExpertParallelA2A(shard, T, H, I, k, dev, bits, gs, exchange=ex, engine="tc", tile=args.ds_tile)
    # shared expert: a one-expert plan over this rank's tokens, rows gathered
    # into the sorted GEMM's layout, SwiGLU fused, then down
    lib = _capi.lib()
    sp_bytes = int(lib.b2f_moe_plan_workspace_bytes(T, 1, 128))
    sp_ws = torch.empty(sp_bytes, dtype=torch.uint8, device=dev)
    call("b2f_moe_plan", ptr(torch.zeros(T, dtype=torch.int32, device=dev)), T, 1, 128, ptr(sp_ws), sp_bytes, 0,
         _capi.stream_of(dev))
    sxs = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    shh = torch.empty(T, I, dtype=torch.bfloat16, device=dev)
    sy = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    routed = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    scratch = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    ones_h = torch.ones(H, dtype=torch.bfloat16, device=dev)
    ones_t = torch.ones(T, 1, dtype=torch.float32, device=dev)
    ev = {n: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for n in ("route", "dispatch", "experts", "return", "shared")}

    def step(record=False):
        st = _capi.stream_of(dev)

        def mark(n, i):
            if record:
                ev[n][i].record()

        mark("route", 0)
        call("b2f_moe_route_topk_ex", ptr(x), T, H, ptr(wr), ptr(rbias), E, k, 1, 1, 0.0, ptr(gates), ptr(inds),
             ptr(scores), st)
        mark("route", 1)
        mark("dispatch", 0)
        sc, rc = ep.dispatch(x, inds, scores)
        mark("dispatch", 1)
        mark("experts", 0)
        ep.compute(sum(rc), (g.wq, g.scales, g.biases), (u.wq, u.scales, u.biases), (dn.wq, dn.scales, dn.biases))
        mark("experts", 1)
        mark("return", 0)
        ep.combine(T, sc, rc, out=routed)
        mark("return", 1)
        mark("shared", 0)
        call("b2f_moe_gather_rows", ptr(x), H, 0, 1, T, 1, 128, ptr(sp_ws), sp_bytes, H, ptr(sxs), H, st)
        call("b2f_sorted_qgemm_affine_tcgen05", ptr(sxs), H, T, 1, ptr(sg.wq), ptr(sg.scales), ptr(sg.biases),
             ptr(su.wq), ptr(su.scales), ptr(su.biases), I, H, bits, gs, 128, ptr(sp_ws), sp_bytes, ptr(shh), I, 1, st)
        call("b2f_sorted_qgemm_affine_tcgen05", ptr(shh), I, T, 1, ptr(sd.wq), ptr(sd.scales), ptr(sd.biases), 0, 0, 0,
             H, I, bits, gs, 128, ptr(sp_ws), sp_bytes, ptr(sy), H, 0, st)
        call("b2f_combine_rmsnorm", ptr(routed), ptr(sy), ptr(ones_t), T, 1, ptr(ones_h), 1e-6, H, ptr(out),
             ptr(scratch), st)
        mark("shared", 1)
        return sc, rc

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    ep.check()
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clk:
        e0.record()
        for _ in range(args.steps):
            sc, rc = step()
        e1.record()
        torch.cuda.synchronize()
    barrier()
    t = e0.elapsed_time(e1) * 1e-3 / args.steps
    sc, rc = step(record=True)
    torch.cuda.synchronize()
    phases = {n: ev[n][0].elapsed_time(ev[n][1]) * 1e3 for n in ev}
    A_here = int((ep.local[: sum(rc) * k] >= 0).sum().item()) if sum(rc) else 0
    routed_ids = inds.reshape(-1)
    hot_ids = perm[: max(1, int(round(0.1 * E)))]
    hot = float(torch.isin(routed_ids, hot_ids).float().mean().item())
    vals = torch.tensor([t, float(A_here), hot] + [phases[n] for n in ev], device=dev, dtype=torch.float64)
    if world > 1:
        tmax = vals[:1].clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        allv = [torch.empty_like(vals) for _ in range(world)]
        dist.all_gather(allv, vals)
        t = float(tmax.item())
        per_rank = [v.tolist() for v in allv]
    else:
        per_rank = [vals.tolist()]
    flops = 2.0 * T_all * k * 3 * H * I + 2.0 * T_all * 3 * H * I
    peak = None
    try:
        with open(PEAKS_FILE) as f:
            pk = json.load(f)
        peak = float(pk["bf16_tflops"])
    except Exception:
        peak = 1590.0
    if rank == 0:
        line = {"metric": "DeepSeek-V3-shaped prefill MoE layer TFLOP/s (4-bit g64, 256 experts top-8 + shared)",
                "value": round(flops / t / 1e12, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
                "warmup": max(args.warmup, 3), "ms_per_step": round(t * 1e3, 4), "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded random)",
                "config": {"workload": f"MoE layer, {E} routed experts top-{k} (sigmoid gates, hottest 10% take 40% "
                                       f"of assignments) + 1 shared, H {H}, I {I}, 4-bit g64, {T_all} tokens "
                                       f"({T} per rank)", "parallelism": f"ep{world} (NCCL all-to-all)",
                           "expert_tile": args.ds_tile},
                "roofline": {"kernel": "whole MoE layer", "bound": "tensor", "achieved": round(flops / t / 1e12, 2),
                             "peak": peak, "unit": "TFLOP/s", "frac": round(flops / t / 1e12 / peak / world, 4),
                             "traffic": None},
                "phases_us_rank0": {n: round(phases[n], 1) for n in ev},
                "per_rank": [{"ms": round(v[0] * 1e3, 3), "assignments": int(v[1]), "hot_share": round(v[2], 3),
                              "experts_us": round(v[3 + list(ev).index("experts")], 1)} for v in per_rank],
                "clocks": clk.summary()}
        print(json.dumps(line), flush=True)
    del ep
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def strong_scaling(args, shape, world, dev, exchange, max_ctx):
    """Decode step with ``--strong-batch`` sequences in total (that number / N
    per rank), timed like the main line (max over ranks)."""
    import torch
    import torch.distributed as dist

    from b200flash.decoder import Qwen3MoeDecoder

    b = max(1, args.strong_batch // world)
    dec = Qwen3MoeDecoder(shape, max_batch=b, max_context=max_ctx, page_size=64, device=dev, seed=1234,
                          layers=args.layers, exchange=exchange, moe_engine=args.moe_engine,
                          dense_engine=args.dense_engine, moe_tile=args.moe_tile, moe_packed=not args.moe_unpacked,
                          pdl=not args.no_pdl, moe_streamk=args.streamk, expert_placement=args.ep_placement)
    dec.fill_random_context(args.ctx)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        dec.step()
    torch.cuda.current_stream(dev).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        dec.step()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    dist.barrier()
    tt = torch.tensor([e0.elapsed_time(e1) * 1e-3], device=dev)
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    t = float(tt.item())
    del graph
    del dec
    torch.cuda.empty_cache()
    return {"global_batch": b * world, "batch_per_gpu": b, "value": round(b * world * args.steps / t, 2),
            "unit": "tok/s", "ms_per_step": round(1e3 * t / args.steps, 4)}


# ---------------------------------------------------------------------------
def _oracle_sample(args, shape, n_seq, layers_sampled, seed=0):
    """Time the CPU oracle on a bounded sample of the decode step and scale it
    to tok/s: ``layers_sampled`` decoder layers for ``n_seq`` sequences at
    ``--ctx`` context, plus 1/32 of the lm_head rows."""
    import numpy as np

    from oracle import affine, attn, kv_sym, moe
    from oracle.decoder import rmsnorm
    from oracle.fp import round_bf16

    rng = np.random.default_rng(seed)
    H, D, Hq, Hkv, I, E, k = (shape.hidden, shape.head_dim, shape.n_heads, shape.n_kv_heads, shape.moe_inter,
                               shape.n_experts, shape.top_k)

    def qw(N, K):
        w = round_bf16(rng.normal(0, 0.02, (N, K)).astype(np.float32))
        return affine.quantize(w, 64, 4)

    wqkv, wo = qw((Hq + 2 * Hkv) * D, H), qw(H, Hq * D)
    wr = rng.normal(0, 0.02, (E, H)).astype(np.float32)
    experts = {}
    ctx = args.ctx
    kv = []
    for _ in range(n_seq):
        kc = rng.integers(0, 255, (ctx, Hkv, D), dtype=np.uint8)
        sc = rng.uniform(0.015, 0.03, (ctx, Hkv, 2)).astype(np.float32)
        kv.append((kc, sc, kc[::-1].copy(), sc[::-1].copy()))
    lm = qw(shape.vocab // 32, H)
    x = round_bf16(rng.standard_normal((n_seq, H)).astype(np.float32))
    t0 = time.perf_counter()
    t_setup = 0.0  # weight creation inside the loop is excluded from the timing
    for _ in range(layers_sampled):
        xn = rmsnorm(x, np.ones(H), 1e-6).astype(np.float64)
        qkv = np.asarray(xn) @ affine.dequantize_f32(*wqkv, 64, 4).astype(np.float64).T
        q = qkv[:, : Hq * D].reshape(n_seq, Hq, D)
        keys = [kv_sym.dequantize_tensor(c[0], c[1], 0 * c[1], 8, (ctx, Hkv, D), 64) for c in kv]
        vals = [kv_sym.dequantize_tensor(c[2], c[3], 0 * c[3], 8, (ctx, Hkv, D), 64) for c in kv]
        a, _ = attn.decode_attention(q, keys, vals)
        h = xn + a.reshape(n_seq, -1) @ affine.dequantize_f32(*wo, 64, 4).astype(np.float64).T
        inds, scores = moe.route(h, wr.T, k)
        y = np.zeros_like(h)
        for b in range(n_seq):
            for j in range(k):
                e = int(inds[b, j])
                if e not in experts:
                    ts = time.perf_counter()
                    experts[e] = (qw(I, H), qw(I, H), qw(H, I))
                    t_setup += time.perf_counter() - ts
                g, u, dn = experts[e]
                gg = affine.dequantize_f32(*g, 64, 4).astype(np.float64) @ h[b]
                uu = affine.dequantize_f32(*u, 64, 4).astype(np.float64) @ h[b]
                y[b] += scores[b, j] * (affine.dequantize_f32(*dn, 64, 4).astype(np.float64) @ (moe.silu(gg) * uu))
        x = round_bf16((h + y).astype(np.float32))
    t_layers = time.perf_counter() - t0 - t_setup
    t1 = time.perf_counter()
    _ = np.asarray(x, np.float64) @ affine.dequantize_f32(*lm, 64, 4).astype(np.float64).T
    t_lm = (time.perf_counter() - t1) * 32
    t_step = t_layers / layers_sampled * 48 + t_lm
    return n_seq / t_step, t_layers + t_lm / 32, t_step, t_layers / layers_sampled, t_lm / 32


def cpu_threads():
    try:
        from threadpoolctl import threadpool_info

        return max([int(i.get("num_threads", 1)) for i in threadpool_info()] + [1])
    except Exception:
        return os.cpu_count() or 1


def cpu_baseline(args, shape):
    n_seq = 4
    tps, wall, t_step, t_layer, t_lm32 = _oracle_sample(args, shape, n_seq=n_seq, layers_sampled=1)
    return {"value": round(tps, 4), "unit": "tok/s", "cores": cpu_threads(), "kind": "port",
            "sample": (f"NumPy oracle (fp64) decode of {n_seq} sequences at context {args.ctx} (not the GPU's "
                       f"{args.batch}): 1 of 48 layers (qkv, 8-bit KV attention, o_proj, router, routed experts) "
                       f"measured at {t_layer:.2f} s, 1/32 of lm_head at {t_lm32:.2f} s; step = 48 x layer + "
                       f"32 x lm slice = {t_step:.1f} s (extrapolated), tok/s = {n_seq} / step"),
            "measured_s": round(wall, 2), "host_cpus": os.cpu_count()}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from b200flash.decoder import Qwen3MoeShape

    shape = Qwen3MoeShape()
    per_step = []
    per_layer = []
    walls = []
    n_seq = 2
    t_start = time.perf_counter()
    for i in range(args.warmup + args.steps):
        tps, wall, t_step, t_layer, t_lm32 = _oracle_sample(args, shape, n_seq=n_seq, layers_sampled=1, seed=i)
        if i >= args.warmup:
            per_step.append(t_step)
            per_layer.append(t_layer)
            walls.append(wall)
    t = sum(per_step)
    value = n_seq * len(per_step) / t
    world = int(os.environ.get("WORLD_SIZE", "1"))
    cb = {"value": round(value, 4), "unit": "tok/s", "kind": "port", "cores": cpu_threads(),
          "sample": (f"NumPy oracle (fp64) decode, {n_seq} sequences at context {args.ctx}; each step times 1 of 48 "
                     f"layers (mean {sum(per_layer) / len(per_layer):.2f} s measured) + 1/32 of lm_head and "
                     f"extrapolates to 48 layers + the whole lm_head; ms_per_step is that extrapolated step, "
                     f"measured_s the CPU time actually spent in the timed steps"),
          "measured_s": round(sum(walls), 2), "wall_s": round(time.perf_counter() - t_start, 2)}
    print(json.dumps({"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "tok/s",
                      "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                      "ms_per_step": round(1e3 * t / len(per_step), 2), "higher_is_better": True,
                      "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
                      "config": config_dict(args, world), "cpu_baseline": cb,
                      "e2e": {"value": round(value, 4), "unit": "tok/s", "h2d_bytes_per_step": 0,
                              "d2h_bytes_per_step": 0}}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--strong-batch", type=int, default=64,
                    help="N > 1: also time this global batch spread over the N ranks (0: skip)")
    ap.add_argument("--experts", type=int, default=256, help="ds-prefill: routed experts")
    ap.add_argument("--tokens", type=int, default=4096, help="ds-prefill: tokens over all ranks")
    ap.add_argument("--ds-tile", type=int, default=256,
                    help="ds-prefill: tokens per expert tile (measured 64 / 128 / 256: 185 / 300 / 336 TFLOP/s)")
    ap.add_argument("--workload", default="decode",
                    choices=["decode", "linear", "kv-attention", "moe-layer", "ds-prefill"],
                    help="decode: the 48-layer decode step (the benchmark line); linear / kv-attention / "
                         "moe-layer: the single-op workloads, one JSON line each")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--moe-engine", default="auto", choices=["auto", "mma", "tc_gather", "tc", "gemv"],
                    help="routed-expert GEMM engine (auto: the decoder's choice for this batch)")
    ap.add_argument("--dense-engine", default="auto", choices=["auto", "mma", "tc", "gemv", "dec"],
                    help="q/k/v and o projection engine (auto: the decoder's choice for this batch)")
    ap.add_argument("--moe-tile", type=int, default=16, choices=[16, 32],
                    help="tokens per expert tile of the warp-MMA expert GEMM")
    ap.add_argument("--no-pdl", action="store_true",
                    help="launch the decode-step kernels in plain stream order (no programmatic dependent launch)")
    ap.add_argument("--streamk", action="store_true",
                    help="stream-K ranges in the packed expert GEMM instead of one CTA per (slot, row block) item")
    ap.add_argument("--moe-unpacked", action="store_true",
                    help="stream the experts' MLX-layout codes by 2-D TMA instead of the packed tiles")
    ap.add_argument("--ep-exchange", default="p2p", choices=["p2p", "nccl"],
                    help="decode expert-parallel exchange for N > 1: peer-memory kernels or NCCL collectives")
    ap.add_argument("--ep-placement", default="balanced", choices=["balanced", "contiguous"],
                    help="N > 1: relabel each layer's experts so the rank blocks carry even expected load, "
                         "or keep the id blocks")
    ap.add_argument("--layers", type=int, default=48,
                    help="decoder depth; anything but 48 is a profiling case, not a bench line")
    ap.add_argument("--profile-window", action="store_true",
                    help="bracket the timed replays with cudaProfilerStart/Stop "
                         "(for ncu --profile-from-start off)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "linear":
        run_linear(args)
    elif args.workload == "kv-attention":
        run_kv_attention(args)
    elif args.workload == "moe-layer":
        run_moe_layer(args)
    elif args.workload == "ds-prefill":
        run_ds_prefill(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
