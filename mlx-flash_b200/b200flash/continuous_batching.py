"""Batched continuous decoding with chunked prefill over the quantized decode step.

The reference engine (``mlx_flash_compress/continuous_batching.py:337-668``:
``InferenceRequest``, ``BatchScheduler``, ``ContinuousBatchingEngine``) runs
every request on its own forward pass (``_batch_step`` loops over the batch,
``:532-554``; ``_prefill_step`` pushes a prompt chunk with a causal mask,
``:556-580``).  Here all active requests share one step of the B-row decoder
(``decoder.Qwen3MoeDecoder``, one CUDA graph per step).  A row is one query
token with its own position and its own block-table row, so rows of one step
can belong to different requests or to the same one:

* a generating request takes one row (its last sampled token);
* a prompting request takes up to ``prefill_chunk`` rows for its next prompt
  tokens, all pointing at its pages with consecutive positions.  Within a
  layer the KV rows of every row are appended before attention runs, and the
  attention of row i reads positions 0..i of its sequence, which is the
  causal mask of a chunked prefill, with no separate prefill kernel.

Each request owns one region of ``max_pages`` pages (region r = the block
table row r of the decoder's initial layout) from admission to completion;
idle rows point at a region no request owns.  Sampling is greedy (the step's
fused argmax); ``temperature`` other than 0 is rejected.

Per-token results do not depend on the other rows (the MoE plan only groups
tokens by expert; attention, projections and sampling are per token), so a
request's tokens are the same alone or batched, and with any prefill chunk.
"""

import itertools
import time
from collections import deque
from dataclasses import dataclass, field
from enum import Enum
from typing import Optional

import torch


class RequestStatus(Enum):
    WAITING = "waiting"
    PREFILLING = "prefilling"
    GENERATING = "generating"
    COMPLETED = "completed"
    CANCELLED = "cancelled"


_ids = itertools.count()


@dataclass
class InferenceRequest:
    prompt_tokens: list
    max_tokens: int = 256
    temperature: float = 0.0
    eos_token_id: Optional[int] = None
    request_id: str = field(default_factory=lambda: f"req-{next(_ids)}")
    generated_tokens: list = field(default_factory=list)
    status: RequestStatus = RequestStatus.WAITING
    created_at: float = field(default_factory=time.time)
    first_token_at: Optional[float] = None
    completed_at: Optional[float] = None
    _slot: int = -1  # page region owned while active
    _prefill_pos: int = 0
    _last: int = 0  # token to feed when generating

    @property
    def ttft_ms(self) -> float:
        if self.first_token_at is None:
            return 0.0
        return (self.first_token_at - self.created_at) * 1000.0

    @property
    def tokens_per_second(self) -> float:
        if self.first_token_at is None or not self.generated_tokens:
            return 0.0
        end = self.completed_at or time.time()
        dt = end - self.first_token_at
        return len(self.generated_tokens) / dt if dt > 0 else 0.0

    @property
    def is_prefill_done(self) -> bool:
        return self._prefill_pos >= len(self.prompt_tokens)


@dataclass
class BatchSchedulerConfig:
    max_batch_size: int = 64
    max_queue_size: int = 1024
    prefill_chunk_size: int = 16  # prompt tokens a request may push through one step


class BatchScheduler:
    """FIFO admission of waiting requests into free decoder slots."""

    def __init__(self, config: Optional[BatchSchedulerConfig] = None):
        self.config = config or BatchSchedulerConfig()
        self._waiting = deque()
        self._requests = {}
        self._completed = 0
        self._cancelled = 0

    def add_request(self, request: InferenceRequest):
        if len(self._waiting) >= self.config.max_queue_size:
            raise RuntimeError("request queue is full")
        self._requests[request.request_id] = request
        self._waiting.append(request)

    def cancel_request(self, request_id: str):
        req = self._requests.get(request_id)
        if req is not None and req.status not in (RequestStatus.COMPLETED, RequestStatus.CANCELLED):
            req.status = RequestStatus.CANCELLED
            self._cancelled += 1

    def next_waiting(self) -> Optional[InferenceRequest]:
        while self._waiting:
            req = self._waiting.popleft()
            if req.status == RequestStatus.WAITING:
                return req
        return None

    def mark_completed(self, request_id: str):
        req = self._requests.get(request_id)
        if req is not None and req.status != RequestStatus.COMPLETED:
            req.status = RequestStatus.COMPLETED
            req.completed_at = time.time()
            self._completed += 1

    def get_request(self, request_id: str) -> Optional[InferenceRequest]:
        return self._requests.get(request_id)

    def get_stats(self) -> dict:
        return {"waiting": sum(1 for r in self._waiting if r.status == RequestStatus.WAITING),
                "completed": self._completed, "cancelled": self._cancelled, "total": len(self._requests)}


class ContinuousBatchingEngine:
    """Continuous batching with chunked prefill over a ``Qwen3MoeDecoder`` (greedy decoding)."""

    def __init__(self, decoder, config: Optional[BatchSchedulerConfig] = None, use_graph: bool = True):
        self.dec = decoder
        self.B = decoder.B
        self.config = config or BatchSchedulerConfig(max_batch_size=decoder.B)
        self.scheduler = BatchScheduler(self.config)
        self.slots = [None] * self.B  # page region -> request
        self.max_context = (decoder.max_pages - 1) * decoder.page
        mp = decoder.max_pages
        self._regions = torch.arange(self.B * mp, dtype=torch.int32).reshape(self.B, mp)
        self._bt = torch.zeros(self.B, mp, dtype=torch.int32).pin_memory()
        self._tok = torch.zeros(self.B, dtype=torch.int32).pin_memory()
        self._pos = torch.zeros(self.B, dtype=torch.int32).pin_memory()
        self._next = torch.zeros(self.B, dtype=torch.int32).pin_memory()
        self._graph = None
        self._use_graph = use_graph
        self.steps = 0
        self._total_generated = 0

    # -- requests -----------------------------------------------------------
    def submit(self, prompt_tokens, max_tokens: int = 256, temperature: float = 0.0,
               eos_token_id: Optional[int] = None, request_id: Optional[str] = None) -> InferenceRequest:
        if temperature != 0.0:
            raise ValueError("only greedy decoding (temperature 0) is supported on this path")
        prompt = [int(t) for t in prompt_tokens]
        if not prompt:
            raise ValueError("empty prompt")
        if len(prompt) + max_tokens > self.max_context:
            raise ValueError(f"prompt + max_tokens exceeds the slot context ({self.max_context})")
        kw = {} if request_id is None else {"request_id": request_id}
        req = InferenceRequest(prompt_tokens=prompt, max_tokens=max_tokens, eos_token_id=eos_token_id, **kw)
        self.scheduler.add_request(req)
        return req

    def cancel(self, request_id: str):
        self.scheduler.cancel_request(request_id)

    # -- stepping -----------------------------------------------------------
    def _admit(self):
        for b in range(self.B):
            if self.slots[b] is None:
                req = self.scheduler.next_waiting()
                if req is None:
                    return
                req._slot = b
                req.status = RequestStatus.PREFILLING
                req._prefill_pos = 0
                self.slots[b] = req

    def _run_step(self):
        dec = self.dec
        dec.tokens.copy_(self._tok, non_blocking=True)
        dec.positions.copy_(self._pos, non_blocking=True)
        dec.block_table.copy_(self._bt, non_blocking=True)
        if self._use_graph:
            if self._graph is None:
                side = torch.cuda.Stream(dec.dev)
                side.wait_stream(torch.cuda.current_stream(dec.dev))
                with torch.cuda.stream(side):
                    dec.step()  # warm-up (also captures the libraries' lazy setup)
                torch.cuda.current_stream(dec.dev).wait_stream(side)
                dec.tokens.copy_(self._tok, non_blocking=True)
                dec.positions.copy_(self._pos, non_blocking=True)
                dec.block_table.copy_(self._bt, non_blocking=True)
                self._graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(self._graph):
                    dec.step()
            self._graph.replay()
        else:
            dec.step()
        self._next.copy_(dec.next_tokens, non_blocking=True)
        torch.cuda.current_stream(dec.dev).synchronize()

    def step(self) -> int:
        """Admit waiting requests, assign this step's rows (one per generating
        request, then prompt chunks), run one batched step, advance every
        request that had rows.  Returns the number of rows used."""
        for b, req in enumerate(self.slots):
            if req is not None and req.status == RequestStatus.CANCELLED:
                req._slot = -1
                self.slots[b] = None
        self._admit()
        active = [r for r in self.slots if r is not None]
        if not active:
            return 0
        rows = []  # (request, first prompt index or -1, count)
        for req in active:
            if req.is_prefill_done:
                rows.append((req, -1, 1))
        free = self.B - len(rows)
        for req in active:
            if not req.is_prefill_done and free > 0:
                n = min(self.config.prefill_chunk_size, len(req.prompt_tokens) - req._prefill_pos, free)
                rows.append((req, req._prefill_pos, n))
                free -= n
        idle_region = next((b for b in range(self.B) if self.slots[b] is None), None)
        row = 0
        owner = []
        for req, p0, n in rows:
            for i in range(n):
                if p0 < 0:
                    self._tok[row] = req._last
                    self._pos[row] = len(req.prompt_tokens) + len(req.generated_tokens) - 1
                else:
                    self._tok[row] = req.prompt_tokens[p0 + i]
                    self._pos[row] = p0 + i
                self._bt[row] = self._regions[req._slot]
                owner.append(req)
                row += 1
        used = row
        for r in range(used, self.B):  # idle rows: position 0 of a region no request owns
            self._tok[r] = 0
            self._pos[r] = 0
            self._bt[r] = self._regions[idle_region]
        self._run_step()
        self.steps += 1
        now = time.time()
        row = 0
        for req, p0, n in rows:
            last_row = row + n - 1
            row += n
            if p0 >= 0:
                req._prefill_pos = p0 + n
                if not req.is_prefill_done:
                    continue
                req.status = RequestStatus.GENERATING
                req.first_token_at = now
            tok = int(self._next[last_row])
            req.generated_tokens.append(tok)
            req._last = tok
            self._total_generated += 1
            if len(req.generated_tokens) >= req.max_tokens or (req.eos_token_id is not None and
                                                                 tok == req.eos_token_id):
                self.scheduler.mark_completed(req.request_id)
                self.slots[req._slot] = None
                req._slot = -1
        return used

    def run_until_idle(self, max_steps: int = 1 << 30):
        n = 0
        while n < max_steps and self.step():
            n += 1
        return n

    def get_stats(self) -> dict:
        st = self.scheduler.get_stats()
        st.update({"slots": self.B, "active": sum(1 for r in self.slots if r is not None), "steps": self.steps,
                   "total_generated": self._total_generated})
        return st
