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
            "parallelism": (f"ep{world} experts (NCCL all-gather dispatch / reduce-scatter combine), "
                            f"dp{world} attention") if world > 1 else "1 GPU"}


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
        if name == "b2f_gather_qgemm_affine_mma" and args[6] == 1:
            # one-expert plan: the dense q/k/v (or o) projection of the batch
            tag = "qkv_proj" if args[13] == dec.qkv_rows else None
        elif name in ("b2f_gather_qgemv_affine", "b2f_gather_qgemm_affine_tcgen05", "b2f_sorted_qgemm_affine_tcgen05",
                      "b2f_gather_qgemm_affine_mma"):
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


# DRAM bytes moved per algorithmic byte, from an ncu capture of the kernel the
# step runs, on the 2-layer copy of this decode step (dram__bytes_read.sum +
# dram__bytes_write.sum over the launch's algorithmic bytes; see
# profiles/qkv_decode_attn_b64_ctx2048.txt).  The per-layer shapes are those
# of the 48-layer step, so traffic scales with the units a launch processes.
# The warp-MMA expert GEMMs have no capture with both counters (their summary,
# profiles/qgemm_mma_moe_b64_2layer_ncu.txt, holds DRAM reads only), so their
# traffic is reported as null.
NCU_TRAFFIC_RATIO = {"attention": (147.63648 + 4.275712) / 144.142336}


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
    from b200flash.ep import EPExchange

    shape = Qwen3MoeShape()
    max_ctx = args.ctx + args.warmup * 3 + args.steps * 3 + 8
    # N > 1: experts sharded expert-parallel (ExpertShard blocks), attention,
    # router and lm_head data-parallel over each rank's own batch
    exchange = EPExchange() if world > 1 else None
    dec = Qwen3MoeDecoder(shape, max_batch=args.batch, max_context=max_ctx, page_size=64, device=dev,
                          seed=1234, layers=args.layers, exchange=exchange, moe_engine=args.moe_engine,
                          dense_engine=args.dense_engine, moe_tile=args.moe_tile)
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
                "traffic_source": ("ncu DRAM bytes / algorithmic bytes on the 2-layer capture, times this launch's bytes"
                                   if dom in NCU_TRAFFIC_RATIO else "no ncu capture with read and write bytes"),
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
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


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
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--moe-engine", default="auto", choices=["auto", "mma", "tc_gather", "tc", "gemv"],
                    help="routed-expert GEMM engine (auto: the decoder's choice for this batch)")
    ap.add_argument("--dense-engine", default="auto", choices=["auto", "mma", "tc", "gemv"],
                    help="q/k/v and o projection engine (auto: the decoder's choice for this batch)")
    ap.add_argument("--moe-tile", type=int, default=16, choices=[16, 32],
                    help="tokens per expert tile of the warp-MMA expert GEMM")
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
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
