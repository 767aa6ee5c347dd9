"""Qwen3-MoE-shaped decoder driven entirely by libb200flash kernels.

This is the decode loop the reference runs through mlx-lm
(``serve.py:347-353`` -> model forward -> ``CachedSwitchLinear`` /
``QuantizedKVCacheManager``), rebuilt around the quantized hot path:

per layer (B sequences, one new token each)
  qkv   = quantized_matmul(xn, Wqkv)                    b2f_qgemv_affine
  q     = RoPE(RMSNorm(q)); K,V -> 8-bit pages          b2f_qk_norm_rope_kv_append
  a     = attention over packed K/V                     b2f_qkv_decode_attn
  h    += quantized_matmul(a, Wo)                       b2f_qgemv_affine (residual fused)
  xn    = RMSNorm(h)                                    b2f_combine_rmsnorm
  top-k = softmax router                                b2f_moe_route_topk
  plan  = group assignments by expert                   b2f_moe_plan
  hh    = silu(gather_qmm(xn, Wg)) * gather_qmm(xn, Wu) b2f_gather_qgemv_affine (fused)
  y     = gather_qmm(hh, Wd)                            b2f_gather_qgemv_affine
  h    += sum_k score_k y_k ; xn = RMSNorm(h)           b2f_combine_rmsnorm
then logits = quantized_matmul(xn, lm_head), next = argmax.

With an ``EPExchange`` over W > 1 ranks the routed experts are sharded
expert-parallel (``b200flash.ep``): each rank holds the ExpertShard block of
every layer's experts, runs attention, router and lm_head for its own B
sequences, and the plan/experts/combine lines above become all-gather of
the routing segments -> b2f_ep_plan -> local experts ->
b2f_ep_combine_partial -> reduce-scatter -> b2f_combine_rmsnorm (k = 1).

Every buffer is allocated once, so ``step()`` can be captured in a CUDA graph.
Weights are random (N(0, 0.02) before 4-bit quantization) with the model's
shapes.  Expert popularity follows Zipf(s): the router weight is Gaussian,
so for a unit-RMS hidden row the logits x.Wr are iid N(0, tau^2) over the
experts, and a per-expert logit bias (``zipf_router_bias``) is fitted so that
the top-k of ``x.Wr + bias`` picks each expert as often as drawing k experts
per token without replacement from p_r ~ r^-s does.
"""

import functools
import math
from dataclasses import dataclass

import numpy as np

import torch

from . import _capi
from ._capi import call, ptr
from .distributed_experts import ExpertShard, balanced_placement
from .ep import ExpertParallelMoE
from .quantized_kv_cache import packed_len, pick_splits


@dataclass
class Qwen3MoeShape:
    hidden: int = 2048
    layers: int = 48
    n_heads: int = 32
    n_kv_heads: int = 4
    head_dim: int = 128
    moe_inter: int = 768
    n_experts: int = 128
    top_k: int = 8
    vocab: int = 151936
    rope_theta: float = 1e6
    rms_eps: float = 1e-6
    bits: int = 4
    group_size: int = 64
    kv_bits: int = 8
    norm_topk: bool = True
    zipf_s: float = 1.1
    # std of the router logits x.Wr for a unit-RMS hidden row (sets Wr's std)
    router_tau: float = 1.3


@functools.lru_cache(maxsize=8)
def zipf_selection_frequency(E: int, k: int, s: float, samples: int = 100_000, seed: int = 0) -> np.ndarray:
    """Per-token probability that the expert of popularity rank r (0-based) is
    among a token's k experts when the k are drawn without replacement from
    p_r ~ (r+1)^-s (Gumbel top-k sampling), estimated from ``samples`` draws
    with a fixed seed.  For E=128, k=8, s=1.1: 0.90, 0.68, 0.52, ... 0.011."""
    p = np.arange(1, E + 1, dtype=np.float64) ** (-s)
    lp = np.log(p / p.sum())
    g = np.random.default_rng(seed)
    f = np.zeros(E)
    chunk = 10_000
    for i in range(0, samples, chunk):
        n = min(chunk, samples - i)
        top = np.argpartition(-(lp[None] + g.gumbel(size=(n, E))), k, axis=1)[:, :k]
        f += np.bincount(top.ravel(), minlength=E)
    f /= samples
    f.setflags(write=False)
    return f


@functools.lru_cache(maxsize=8)
def zipf_router_bias(E: int, k: int, s: float, tau: float, samples: int = 16384, iters: int = 60,
                     seed: int = 1) -> np.ndarray:
    """Per-rank logit bias beta (float32 [E]) such that the top-k of
    ``beta + tau * z`` (z iid N(0, 1) per expert, the router logits of a
    Gaussian Wr) selects rank r with frequency ``zipf_selection_frequency``."""
    return fit_router_bias(tuple(zipf_selection_frequency(E, k, s)), k, tau, samples, iters, seed)


def hot_set_frequency(E: int, k: int, hot_frac: float, hot_share: float) -> tuple:
    """Per-token selection frequency when the hottest ``round(hot_frac * E)``
    experts take ``hot_share`` of the T*k assignments, evenly within the hot
    and the cold set (hot first)."""
    nh = max(1, int(round(hot_frac * E)))
    fh = hot_share * k / nh
    fc = (1.0 - hot_share) * k / (E - nh)
    return tuple([fh] * nh + [fc] * (E - nh))


@functools.lru_cache(maxsize=8)
def fit_router_bias(freq: tuple, k: int, tau: float, samples: int = 16384, iters: int = 60,
                    seed: int = 1) -> np.ndarray:
    """Per-expert logit bias beta (float32 [E]) such that the top-k of
    ``beta + tau * z`` (z iid N(0, 1)) selects expert e with per-token
    frequency ``freq[e]`` (sum k).  Fixed-point fit on ``samples`` fixed
    noise draws: beta += 0.7 log(f / h)."""
    f = np.asarray(freq, np.float64)
    E = f.size
    z = (tau * np.random.default_rng(seed).standard_normal((samples, E))).astype(np.float32)
    beta = np.log(f).astype(np.float32)
    for _ in range(iters):
        top = np.argpartition(-(beta[None] + z), k, axis=1)[:, :k]
        h = np.bincount(top.ravel(), minlength=E) / samples
        beta += (0.7 * np.log(np.maximum(f, 1e-6) / np.maximum(h, 1e-6))).astype(np.float32)
        beta -= beta.max()
    beta.setflags(write=False)
    return beta


def expected_distinct_experts(freq: np.ndarray, tokens: int) -> float:
    """Expected number of distinct experts hit by ``tokens`` independent
    tokens whose per-token selection frequencies are ``freq``."""
    return float(np.sum(1.0 - (1.0 - np.asarray(freq, np.float64)) ** tokens))


class QWeight:
    """An affine-quantized weight ``[*lead, N, K]`` (wq uint32, bf16 scales/biases)."""

    def __init__(self, wq, scales, biases, bits, group_size):
        self.wq, self.scales, self.biases = wq, scales, biases
        self.bits, self.group_size = bits, group_size
        self.N = wq.shape[-2]
        self.K = wq.shape[-1] * 32 // bits

    @property
    def nbytes(self):
        return sum(t.numel() * t.element_size() for t in (self.wq, self.scales, self.biases))


def random_qweight(shape, bits, gs, dev, gen, std=0.02, chunk_rows=1 << 16):
    """N(0, std) bf16 weights quantized on the device in row chunks (bounded temp memory)."""
    *lead, N, K = shape
    rows = N
    for d in lead:
        rows *= d
    wq = torch.empty(rows, K * bits // 32, dtype=torch.uint32, device=dev)
    sc = torch.empty(rows, K // gs, dtype=torch.bfloat16, device=dev)
    bi = torch.empty_like(sc)
    st = _capi.stream_of(dev)
    for r0 in range(0, rows, chunk_rows):
        r1 = min(rows, r0 + chunk_rows)
        w = (torch.randn(r1 - r0, K, device=dev, generator=gen) * std).to(torch.bfloat16)
        call("b2f_quantize_affine", ptr(w), 0, r1 - r0, K, bits, gs, ptr(wq[r0]), ptr(sc[r0]), ptr(bi[r0]), st)
        del w
    return QWeight(wq.reshape(*lead, N, -1), sc.reshape(*lead, N, -1), bi.reshape(*lead, N, -1), bits, gs)


class Qwen3MoeDecoder:
    """Random-weight Qwen3-MoE-shaped decoder with a paged 8-bit KV cache."""

    def __init__(self, shape: Qwen3MoeShape, max_batch: int, max_context: int, page_size: int = 64,
                 device="cuda:0", seed: int = 0, layers=None, moe_engine: str = "auto", exchange=None,
                 dense_engine: str = "auto", moe_tile: int = 16, moe_packed: bool = True, pdl: bool = True,
                 moe_streamk: bool = False, expert_placement: str = "balanced"):
        self.s = s = shape
        self.pdl = bool(pdl)
        self.dev = dev = torch.device(device)
        self.B = max_batch
        self.page = page_size
        self.L = s.layers if layers is None else layers
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed)
        H, D, Hq, Hkv, E, I = s.hidden, s.head_dim, s.n_heads, s.n_kv_heads, s.n_experts, s.moe_inter
        # expert parallelism: this rank's block of every layer's experts
        self.world = 1 if exchange is None else exchange.world
        self.shard = ExpertShard(rank=0 if exchange is None else exchange.rank, world_size=self.world,
                                 total_experts=E)
        E_loc = len(self.shard.owned_experts)
        egen = gen
        if self.world > 1:
            egen = torch.Generator(device=dev)
            egen.manual_seed(seed + 1000003 * (self.shard.rank + 1))
        bits, gs = s.bits, s.group_size
        self.qkv_rows = (Hq + 2 * Hkv) * D

        def norm_w(n):
            return (1.0 + 0.1 * torch.randn(n, device=dev, generator=gen)).to(torch.bfloat16)

        self.embed = random_qweight((s.vocab, H), bits, gs, dev, gen, std=1.0)
        self.layers = []
        # router: x.Wr has std router_tau for a unit-RMS row scaled by the
        # post-attention norm weight (mean square 1.01); the fitted bias gives
        # the Zipf(s) selection frequencies, rank perm[e] for expert e
        zbias = torch.from_numpy(np.array(zipf_router_bias(E, s.top_k, s.zipf_s, s.router_tau))).to(dev)
        wr_std = s.router_tau / math.sqrt(H * 1.01)
        if expert_placement not in ("balanced", "contiguous"):
            raise ValueError("expert_placement is 'balanced' or 'contiguous'")
        # expert parallelism: "balanced" relabels each layer's experts so the
        # ExpertShard blocks carry even expected loads (balanced_placement over
        # the experts' selection frequencies); "contiguous" keeps the shuffled
        # popularity of the single-GPU model on the id blocks as they are
        self.expert_placement = expert_placement if self.world > 1 else "contiguous"
        sel_freq = np.array(zipf_selection_frequency(E, s.top_k, s.zipf_s))
        for _ in range(self.L):
            perm = torch.randperm(E, device=dev, generator=gen)
            if self.expert_placement == "balanced":
                order = balanced_placement(sel_freq[perm.cpu().numpy()], self.world)
                perm = perm[torch.tensor(order, device=dev)]
            self.layers.append({
                "in_norm": norm_w(H), "post_norm": norm_w(H), "q_norm": norm_w(D), "k_norm": norm_w(D),
                "wqkv": random_qweight((self.qkv_rows, H), bits, gs, dev, gen),
                "wo": random_qweight((H, Hq * D), bits, gs, dev, gen),
                "wr": (torch.randn(E, H, device=dev, generator=gen) * wr_std).to(torch.bfloat16),
                "rbias": zbias[perm].contiguous(), "zipf_rank": perm,
                "gate": random_qweight((E_loc, I, H), bits, gs, dev, egen),
                "up": random_qweight((E_loc, I, H), bits, gs, dev, egen),
                "down": random_qweight((E_loc, H, I), bits, gs, dev, egen),
            })
        self.final_norm = norm_w(H)
        self.lm_head = random_qweight((s.vocab, H), bits, gs, dev, gen)

        # paged KV pool (head-major pages), one block table row per sequence
        self.max_pages = (max_context + page_size - 1) // page_size + 1
        self.num_pages = self.B * self.max_pages
        self.rb = packed_len(D, s.kv_bits, 64)
        self.kv = []
        for _ in range(self.L):
            self.kv.append({
                "kc": torch.zeros(self.num_pages, Hkv, page_size, self.rb, dtype=torch.uint8, device=dev),
                "ks": torch.zeros(self.num_pages, Hkv, page_size, D // 64, dtype=torch.float32, device=dev),
                "vc": torch.zeros(self.num_pages, Hkv, page_size, self.rb, dtype=torch.uint8, device=dev),
                "vs": torch.zeros(self.num_pages, Hkv, page_size, D // 64, dtype=torch.float32, device=dev),
            })
        self.block_table = torch.arange(self.num_pages, dtype=torch.int32, device=dev).reshape(self.B, self.max_pages)

        # step buffers
        B, A = self.B, self.B * s.top_k
        self.tokens = torch.zeros(B, dtype=torch.int32, device=dev)
        self.positions = torch.zeros(B, dtype=torch.int32, device=dev)
        self.seq_lens = torch.zeros(B, dtype=torch.int32, device=dev)
        self.h = torch.empty(B, H, dtype=torch.bfloat16, device=dev)
        self.ep = None
        if self.world > 1:
            self.ep = ExpertParallelMoE(self.shard, B, H, I, s.top_k, dev, bits, gs, exchange,
                                        engine=moe_engine)
            self.moe_engine = self.ep.engine
        self.xn = torch.empty(B, H, dtype=torch.bfloat16, device=dev) if self.ep is None else self.ep.x
        self.qkv = torch.empty(B, self.qkv_rows, dtype=torch.bfloat16, device=dev)
        self.q = torch.empty(B, Hq, D, dtype=torch.bfloat16, device=dev)
        self.attn = torch.empty(B, Hq, D, dtype=torch.bfloat16, device=dev)
        if self.ep is None:
            self.inds = torch.empty(B, s.top_k, dtype=torch.int32, device=dev)
            self.scores = torch.empty(B, s.top_k, dtype=torch.float32, device=dev)
        else:
            self.inds, self.scores = self.ep.inds, self.ep.scores
        self.gates = torch.empty(B, E, dtype=torch.float32, device=dev)
        if self.ep is None:
            if moe_engine == "auto":
                # 4-bit / group 64 / 128-wide K: register-unpack warp MMA (decode
                # tiles of <= 16 tokens); else tcgen05 once experts see >= 1 token
                # on average, the register GEMV below that
                mma_ok = bits == 4 and gs == 64 and H % 128 == 0 and I % 128 == 0
                moe_engine = "mma" if mma_ok else ("tc_gather" if A >= E else "gemv")
            if moe_engine not in ("tc", "tc_gather", "gemv", "mma"):
                raise ValueError(f"unknown expert engine {moe_engine!r}")
            if moe_engine == "tc" and ((H // 64) % 2 or (I // 64) % 2):
                moe_engine = "tc_gather"  # the sorted-row kernel copies scales two groups at a time
            if moe_engine == "mma" and (bits != 4 or gs != 64 or H % 128 or I % 128):
                moe_engine = "tc_gather"  # register-dequant MMA: 4-bit, group 64, 128-wide K chunks
            self.moe_engine = moe_engine
            # per-slot tcgen05 kernel: 32-token tiles measured best from 16 to 512
            # tokens (two CTAs per SM fit; hot experts take several slots)
            if moe_engine == "tc_gather":
                self.tile = 32
            elif moe_engine == "mma":
                if moe_tile not in (16, 32):
                    raise ValueError("the warp-MMA expert GEMM takes 16- or 32-token tiles")
                self.tile = moe_tile
            else:
                self.tile = min(256, max(16, (B + 15) // 16 * 16)) if moe_engine != "gemv" else 16
            self.plan_bytes = int(_capi.lib().b2f_moe_plan_workspace_bytes(A, E, self.tile))
            self.plan_ws = torch.empty(self.plan_bytes, dtype=torch.uint8, device=dev)
            self.plan_status = torch.zeros(1, dtype=torch.int32, device=dev)
            self.hh = torch.empty(A, I, dtype=torch.bfloat16, device=dev)
            self.y = torch.empty(A, H, dtype=torch.bfloat16, device=dev)
            # "tc": activations gathered into expert-sorted rows once per layer
            self.xs = torch.empty(A, H, dtype=torch.bfloat16, device=dev) if moe_engine == "tc" else None
        else:
            self.tile = self.ep.tile
        # warp-MMA experts read their codes as packed tiles (b2f_mma_repack:
        # one contiguous bulk copy per staged tile); the MLX-layout codes stay
        # for export
        self.moe_packed = bool(moe_packed) and self.moe_engine == "mma" and self.tile == 16
        if self.moe_packed:
            lib = _capi.lib()
            st = _capi.stream_of(dev)
            for ly in self.layers:
                for name, mat in (("gate", 2), ("up", 2), ("down", 1)):
                    w = ly[name]
                    nbytes = int(lib.b2f_mma_packed_bytes(E_loc, w.N, w.K, mat))
                    pk = torch.empty(nbytes, dtype=torch.uint8, device=dev)
                    call("b2f_mma_repack", ptr(w.wq), ptr(w.scales), ptr(w.biases), E_loc, w.N, w.K, mat, ptr(pk),
                         nbytes, st)
                    ly[name + "_packed"] = pk
            # stream-K: every SM streams the same number of weight tiles (the
            # counters and partials start zeroed; each launch leaves them zeroed)
            if self.ep is None:
                self.sk_bytes = int(lib.b2f_mma_streamk_workspace_bytes()) if moe_streamk else 0
                self.sk_ws = torch.zeros(max(self.sk_bytes, 256), dtype=torch.uint8, device=dev)
            elif not moe_streamk:
                self.ep.sk_bytes = 0
        self.logits = torch.empty(B, s.vocab, dtype=torch.bfloat16, device=dev)
        self.next_tokens = torch.empty(B, dtype=torch.int32, device=dev)
        self.n_splits = pick_splits(B, Hkv, max_context)
        wsb = int(_capi.lib().b2f_qkv_decode_attn_workspace_bytes(B, Hq, D, self.n_splits))
        self.attn_ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=dev)
        self.attn_ws_bytes = wsb
        self.softmax_scale = 1.0 / math.sqrt(D)
        # dense projections: register GEMV for a few tokens, tcgen05 (split-K
        # where the matrix has few 128-row blocks) for larger batches; "mma":
        # the warp-MMA GEMM over the batch as 16-token slots of one expert,
        # split-K into fp32 planes summed by the RoPE/KV-append and
        # residual+RMSNorm kernels.
        mma_dense = bits == 4 and gs == 64 and H % 128 == 0 and (Hq * D) % 128 == 0
        dec_dense = mma_dense and B <= 64 and H % 8 == 0
        if dense_engine == "auto":
            # 32-64 tokens: the stream-K decode GEMM (every SM streams the same
            # weight bytes; measured ahead of tcgen05 split-K at batch 64:
            # 7244 against 6960 tok/s for the whole step)
            if dec_dense and B >= 32:
                dense_engine = "dec"
            else:
                dense_engine = "tc" if B >= 32 and s.group_size == 64 else "gemv"
        if dense_engine not in ("tc", "gemv", "mma", "dec"):
            raise ValueError(f"unknown dense engine {dense_engine!r}")
        if dense_engine == "mma" and not mma_dense:
            dense_engine = "tc" if s.group_size == 64 else "gemv"
        if dense_engine == "dec" and not dec_dense:
            dense_engine = "tc" if s.group_size == 64 else "gemv"
        self.dense_engine = dense_engine
        # lm_head: warp MMA over a one-expert plan for small batches (measured
        # ahead of the register GEMV at 8 tokens); tcgen05 from 32 tokens on
        self.lm_mma = bits == 4 and gs == 64 and H % 128 == 0 and s.vocab % 8 == 0 and B < 32
        if self.lm_mma:
            self.lmplan_bytes = int(_capi.lib().b2f_moe_plan_workspace_bytes(B, 1, 16))
            self.lmplan_ws = torch.empty(self.lmplan_bytes, dtype=torch.uint8, device=dev)
            call("b2f_moe_plan", ptr(torch.zeros(B, dtype=torch.int32, device=dev)), B, 1, 16, ptr(self.lmplan_ws),
                 self.lmplan_bytes, 0, _capi.stream_of(dev))
        if dense_engine == "mma":
            # the batch as 16-token slots of one "expert" (a plan over all-zero
            # expert ids); 64-token slots measured slower at batch 64
            self.dmma_tile = 16
            self.dplan_bytes = int(_capi.lib().b2f_moe_plan_workspace_bytes(B, 1, self.dmma_tile))
            self.dplan_ws = torch.empty(self.dplan_bytes, dtype=torch.uint8, device=dev)
            zeros = torch.zeros(B, dtype=torch.int32, device=dev)
            call("b2f_moe_plan", ptr(zeros), B, 1, self.dmma_tile, ptr(self.dplan_ws), self.dplan_bytes, 0,
                 _capi.stream_of(dev))
        self.dense_tile = min(256, max(16, (B + 15) // 16 * 16))
        sms = torch.cuda.get_device_properties(dev).multi_processor_count

        def ksplit_for(N, K):
            blocks = (N + 127) // 128
            chunks = K // 64
            ks = 1
            while blocks * ks * 2 <= 2 * sms and ks * 2 <= chunks // 4:
                ks *= 2
            return ks

        def mma_ksplit_for(N, K):
            # about three CTAs per SM: 256-row blocks x 16-token slots x K ranges
            ctas = ((N + 255) // 256) * ((B + 15) // 16)
            return max(1, min(K // 256, (3 * sms + ctas - 1) // ctas))

        lib = _capi.lib()
        # K ranges actually used (every range non-empty); 1 = no split
        if dense_engine == "dec":
            # stream-K decode GEMM: its plane counts
            self.ks_qkv = int(lib.b2f_qgemm_decode_planes(B, self.qkv_rows, H))
            self.ks_o = int(lib.b2f_qgemm_decode_planes(B, H, Hq * D))
        elif dense_engine == "mma":
            self.ks_qkv = int(lib.b2f_mma_splitk_ranges(H, mma_ksplit_for(self.qkv_rows, H)))
            self.ks_o = int(lib.b2f_mma_splitk_ranges(Hq * D, mma_ksplit_for(H, Hq * D)))
        else:
            self.ks_qkv = int(lib.b2f_qgemm_splitk_ranges(H, ksplit_for(self.qkv_rows, H)))
            self.ks_o = int(lib.b2f_qgemm_splitk_ranges(Hq * D, ksplit_for(H, Hq * D)))
        ws = 0
        if dense_engine == "dec":
            ws = 4 * B * max(self.ks_qkv * self.qkv_rows, self.ks_o * H)
        if dense_engine == "mma":
            ws = max(int(lib.b2f_mma_splitk_workspace_bytes(B, self.qkv_rows, H, self.ks_qkv)),
                     int(lib.b2f_mma_splitk_workspace_bytes(B, H, Hq * D, self.ks_o)))
        if dense_engine == "tc":
            ws = max(int(lib.b2f_qgemm_splitk_workspace_bytes(B, self.qkv_rows, self.ks_qkv)) if self.ks_qkv > 1 else 0,
                     int(lib.b2f_qgemm_splitk_workspace_bytes(B, H, self.ks_o)) if self.ks_o > 1 else 0)
        # fp32 split-K partials, consumed by the RoPE/KV-append and residual+norm kernels
        self.dense_ws = torch.empty(max(ws, 16), dtype=torch.uint8, device=dev)
        self.dense_ws_bytes = ws

    # ------------------------------------------------------------------
    def weight_bytes(self) -> int:
        n = self.embed.nbytes + self.lm_head.nbytes
        for ly in self.layers:
            n += sum(ly[k].nbytes for k in ("wqkv", "wo", "gate", "up", "down"))
            n += ly["wr"].numel() * 2
        return n

    def fill_random_context(self, ctx_len: int, seed: int = 1):
        """Synthetic prefilled context: every sequence holds ctx_len random
        8-bit KV rows (codes uniform, scales like N(0,1) data) in every layer."""
        g = torch.Generator(device=self.dev)
        g.manual_seed(seed)
        npg = (ctx_len + self.page - 1) // self.page
        for kv in self.kv:
            for key in ("kc", "vc"):
                kv[key].random_(0, 255, generator=g)
            for key in ("ks", "vs"):
                kv[key].uniform_(0.015, 0.03, generator=g)
        assert npg < self.max_pages
        self.positions.fill_(ctx_len)
        self.tokens.random_(0, self.s.vocab, generator=g)

    # ------------------------------------------------------------------
    def step(self):
        """One decode step for all B sequences (graph-capturable).  With
        `pdl` the library kernels are programmatic dependent launches: each is
        scheduled while its predecessor finishes (identical results)."""
        # NCCL's kernels take no part in programmatic dependent launch; with
        # the peer exchange every kernel of the step is this library's
        with _capi.dependent_launches(self.pdl and (self.ep is None or self.ep.p2p)):
            self._step()

    def _step(self):
        s, B = self.s, self.B
        H, D, Hq, Hkv, E, I = s.hidden, s.head_dim, s.n_heads, s.n_kv_heads, s.n_experts, s.moe_inter
        A = B * s.top_k
        st = _capi.stream_of(self.dev)
        # embedding gather (dequantize selected rows) and first norm
        e = self.embed
        torch.add(self.positions, 1, out=self.seq_lens)
        call("b2f_dequantize_affine", ptr(e.wq), ptr(e.scales), ptr(e.biases), 0, B, H, e.bits, e.group_size,
             ptr(self.tokens), ptr(self.h), st)
        call("b2f_combine_rmsnorm", ptr(self.h), 0, 0, B, 0, ptr(self.layers[0]["in_norm"]), s.rms_eps, H,
             0, ptr(self.xn), st)
        for li, (ly, kv) in enumerate(zip(self.layers, self.kv)):
            w = ly["wqkv"]
            if self.dense_engine in ("mma", "dec") or (self.dense_engine == "tc" and self.ks_qkv > 1):
                self._partials(self.xn, H, w, self.ks_qkv, st)
                call("b2f_qk_norm_rope_kv_append_partials", ptr(self.dense_ws), self.ks_qkv, B, Hq, Hkv, D,
                     ptr(ly["q_norm"]), ptr(ly["k_norm"]), s.rms_eps, s.rope_theta, ptr(self.positions), ptr(self.q),
                     ptr(kv["kc"]), ptr(kv["ks"]), ptr(kv["vc"]), ptr(kv["vs"]), ptr(self.block_table),
                     self.max_pages, self.page, s.kv_bits, st)
            else:
                self._dense(self.xn, H, w, 0, self.qkv, self.ks_qkv, st)
                call("b2f_qk_norm_rope_kv_append", ptr(self.qkv), B, Hq, Hkv, D, ptr(ly["q_norm"]),
                     ptr(ly["k_norm"]), s.rms_eps, s.rope_theta, ptr(self.positions), ptr(self.q), ptr(kv["kc"]),
                     ptr(kv["ks"]), ptr(kv["vc"]), ptr(kv["vs"]), ptr(self.block_table), self.max_pages, self.page,
                     s.kv_bits, st)
            call("b2f_qkv_decode_attn", ptr(self.q), ptr(kv["kc"]), ptr(kv["ks"]), ptr(kv["vc"]), ptr(kv["vs"]),
                 ptr(self.block_table), self.max_pages, ptr(self.seq_lens), B, Hq, Hkv, D, self.page, self.page, 1,
                 s.kv_bits, 64, self.softmax_scale, self.n_splits, ptr(self.attn_ws), self.attn_ws_bytes,
                 ptr(self.attn), st)
            w = ly["wo"]
            if self.dense_engine in ("mma", "dec") or (self.dense_engine == "tc" and self.ks_o > 1):
                self._partials(self.attn, Hq * D, w, self.ks_o, st)
                call("b2f_combine_rmsnorm_partials", ptr(self.h), ptr(self.dense_ws), self.ks_o, B,
                     ptr(ly["post_norm"]), s.rms_eps, H, ptr(self.h), ptr(self.xn), st)
            else:
                self._dense(self.attn, Hq * D, w, self.h, self.h, self.ks_o, st)
                call("b2f_combine_rmsnorm", ptr(self.h), 0, 0, B, 0, ptr(ly["post_norm"]), s.rms_eps, H, 0,
                     ptr(self.xn), st)
            nxt = self.layers[li + 1]["in_norm"] if li + 1 < self.L else self.final_norm
            g, u, d = ly["gate"], ly["up"], ly["down"]
            if self.ep is not None:
                self.ep.route(ly["wr"], ly["rbias"], s.norm_topk)
                self.ep.forward((g.wq, g.scales, g.biases), (u.wq, u.scales, u.biases), (d.wq, d.scales, d.biases),
                                (ly["gate_packed"], ly["up_packed"], ly["down_packed"]) if self.moe_packed else None,
                                wait_combine=False)
                self.ep.combine_rmsnorm(self.h, nxt, s.rms_eps, self.h, self.xn)
                continue
            call("b2f_moe_route_plan", ptr(self.xn), B, H, ptr(ly["wr"]), ptr(ly["rbias"]), E, s.top_k,
                 int(s.norm_topk), ptr(self.gates), ptr(self.inds), ptr(self.scores), self.tile, ptr(self.plan_ws),
                 self.plan_bytes, ptr(self.plan_status), st)
            if self.moe_packed:
                # gate/up rows land in plan order (the down GEMM's input layout);
                # the down GEMM's first weight tiles stream while the gate/up
                # GEMM's last wave finishes (its plan is two launches old)
                pdl = 1 if self.pdl else 0
                call("b2f_gather_qgemm_affine_mma_packed", ptr(self.xn), H, 0, s.top_k, 0, A, E, ptr(ly["gate_packed"]),
                     ptr(ly["up_packed"]), I, H, g.bits, g.group_size, self.tile, ptr(self.plan_ws), self.plan_bytes,
                     ptr(self.hh), I, 1, ptr(self.sk_ws) if self.sk_bytes else 0, self.sk_bytes, 2 * pdl, st)
                call("b2f_gather_qgemm_affine_mma_packed", ptr(self.hh), I, 0, 1, 1, A, E, ptr(ly["down_packed"]), 0,
                     H, I, d.bits, d.group_size, self.tile, ptr(self.plan_ws), self.plan_bytes, ptr(self.y), H, 0,
                     ptr(self.sk_ws) if self.sk_bytes else 0, self.sk_bytes, pdl, st)
            elif self.moe_engine == "mma":
                # gate/up rows land in plan order (the down GEMM's input layout)
                call("b2f_gather_qgemm_affine_mma", ptr(self.xn), H, 0, s.top_k, 0, A, E, ptr(g.wq), ptr(g.scales),
                     ptr(g.biases), ptr(u.wq), ptr(u.scales), ptr(u.biases), I, H, g.bits, g.group_size, self.tile,
                     ptr(self.plan_ws), self.plan_bytes, ptr(self.hh), I, 1, st)
                call("b2f_gather_qgemm_affine_mma", ptr(self.hh), I, 0, 1, 1, A, E, ptr(d.wq), ptr(d.scales),
                     ptr(d.biases), 0, 0, 0, H, I, d.bits, d.group_size, self.tile, ptr(self.plan_ws),
                     self.plan_bytes, ptr(self.y), H, 0, st)
            elif self.moe_engine == "tc":
                call("b2f_moe_gather_rows", ptr(self.xn), H, 0, s.top_k, A, E, self.tile, ptr(self.plan_ws),
                     self.plan_bytes, H, ptr(self.xs), H, st)
                call("b2f_sorted_qgemm_affine_tcgen05", ptr(self.xs), H, A, E, ptr(g.wq), ptr(g.scales),
                     ptr(g.biases), ptr(u.wq), ptr(u.scales), ptr(u.biases), I, H, g.bits, g.group_size, self.tile,
                     ptr(self.plan_ws), self.plan_bytes, ptr(self.hh), I, 1, st)
                call("b2f_sorted_qgemm_affine_tcgen05", ptr(self.hh), I, A, E, ptr(d.wq), ptr(d.scales),
                     ptr(d.biases), 0, 0, 0, H, I, d.bits, d.group_size, self.tile, ptr(self.plan_ws),
                     self.plan_bytes, ptr(self.y), H, 0, st)
            else:
                fn = "b2f_gather_qgemm_affine_tcgen05" if self.moe_engine == "tc_gather" else "b2f_gather_qgemv_affine"
                call(fn, ptr(self.xn), H, 0, s.top_k, A, E, ptr(g.wq), ptr(g.scales),
                     ptr(g.biases), ptr(u.wq), ptr(u.scales), ptr(u.biases), I, H, g.bits, g.group_size, self.tile,
                     ptr(self.plan_ws), self.plan_bytes, ptr(self.hh), I, st)
                call(fn, ptr(self.hh), I, 0, 1, A, E, ptr(d.wq), ptr(d.scales), ptr(d.biases),
                     0, 0, 0, H, I, d.bits, d.group_size, self.tile, ptr(self.plan_ws), self.plan_bytes,
                     ptr(self.y), H, st)
            call("b2f_combine_rmsnorm", ptr(self.h), ptr(self.y), ptr(self.scores), B, s.top_k, ptr(nxt),
                 s.rms_eps, H, ptr(self.h), ptr(self.xn), st)
        if self.lm_mma:
            # the vocabulary projection on warp MMA: the batch as 16-token slots
            # of a one-expert plan, each 64-row block read once from HBM
            w = self.lm_head
            call("b2f_gather_qgemm_affine_mma", ptr(self.xn), H, 0, 1, 0, B, 1, ptr(w.wq), ptr(w.scales),
                 ptr(w.biases), 0, 0, 0, w.N, w.K, w.bits, w.group_size, 16, ptr(self.lmplan_ws), self.lmplan_bytes,
                 ptr(self.logits), w.N, 0, st)
        else:
            self._dense(self.xn, H, self.lm_head, 0, self.logits, 1, st)
        call("b2f_argmax_rows", ptr(self.logits), B, s.vocab, ptr(self.next_tokens), st)
        # feed back: next input token and position
        self.tokens.copy_(self.next_tokens)
        self.positions.add_(1)

    def _dense(self, x, ldx, w, residual, out, ksplit, st):
        """out = x . W^T (+ residual): register GEMV or tcgen05 (split-K)."""
        B = self.B
        if self.dense_engine == "gemv":
            call("b2f_qgemv_affine", ptr(x), ldx, B, ptr(w.wq), ptr(w.scales), ptr(w.biases), w.N, w.K, w.bits,
                 w.group_size, ptr(residual) if isinstance(residual, torch.Tensor) else 0, ptr(out), w.N, st)
        else:
            call("b2f_qgemm_affine_tcgen05_splitk", ptr(x), ldx, B, ptr(w.wq), ptr(w.scales), ptr(w.biases), w.N, w.K,
                 w.bits, w.group_size, ptr(residual) if isinstance(residual, torch.Tensor) else 0, ptr(out), w.N,
                 self.dense_tile, ksplit, ptr(self.dense_ws), self.dense_ws_bytes, st)

    def _partials(self, x, ldx, w, ksplit, st):
        """fp32 split-K partials of x . W^T into the dense workspace."""
        if self.dense_engine == "dec":
            call("b2f_qgemm_affine_decode_partials", ptr(x), ldx, self.B, ptr(w.wq), ptr(w.scales), ptr(w.biases),
                 w.N, w.K, w.bits, w.group_size, ptr(self.dense_ws), self.dense_ws_bytes, st)
            return
        if self.dense_engine == "mma":
            call("b2f_gather_qgemm_affine_mma_partials", ptr(x), ldx, 0, 1, self.B, 1, ptr(w.wq), ptr(w.scales),
                 ptr(w.biases), w.N, w.K, w.bits, w.group_size, self.dmma_tile, ptr(self.dplan_ws), self.dplan_bytes,
                 ksplit, ptr(self.dense_ws), self.dense_ws_bytes, st)
            return
        call("b2f_qgemm_affine_tcgen05_partials", ptr(x), ldx, self.B, ptr(w.wq), ptr(w.scales), ptr(w.biases), w.N,
             w.K, w.bits, w.group_size, self.dense_tile, ksplit, ptr(self.dense_ws), self.dense_ws_bytes, st)

    def launches_per_step(self) -> int:
        """libb200flash kernel launches in one step (attention counts its combine pass)."""
        attn = 2 if self.n_splits > 1 else 1
        # qkv, rope+append, attention, o_proj, norm, router (logits + top-k/plan), gate/up, down, combine
        per_layer = 1 + 1 + attn + 1 + 1 + 2 + 2 + 1

        if self.moe_engine == "tc":
            per_layer += 1  # the row gather into expert-sorted order
        if self.ep is not None:
            per_layer += 1  # the partial-sum kernel before the reduce-scatter (or the peer combine)
            if self.ep.p2p:
                per_layer += 1  # the peer dispatch
        return 2 + self.L * per_layer + 2
