"""GPU: continuous batching over the decode step -- requests joining and
leaving, prompts pushed through the batched step in chunks (rows of one
request share its pages with consecutive positions), greedy tokens identical
to each request decoded alone and for every chunk size."""

import pytest

from b200flash.continuous_batching import BatchSchedulerConfig, ContinuousBatchingEngine, RequestStatus
from b200flash.decoder import Qwen3MoeDecoder, Qwen3MoeShape

pytestmark = pytest.mark.gpu


def _decoder(dev):
    shape = Qwen3MoeShape(hidden=256, layers=2, n_heads=8, n_kv_heads=2, head_dim=128, moe_inter=128,
                          n_experts=8, top_k=2, vocab=1000, kv_bits=8)
    return Qwen3MoeDecoder(shape, max_batch=4, max_context=96, page_size=16, device=dev, seed=3)


@pytest.mark.parametrize("use_graph,chunk", [(True, 16), (False, 1), (True, 3)])
def test_batched_equals_alone(dev, use_graph, chunk):
    dec = _decoder(dev)
    prompts = [[3, 14, 15], [9, 2, 6, 5, 3, 5, 8], [7], [1, 4, 1, 4, 2, 1, 3, 5, 6, 2, 3, 7], [27, 18, 28, 18, 28],
               [31, 41, 59, 26, 53, 58, 97, 93, 23]]
    max_toks = [5, 3, 8, 4, 6, 2]
    cfg = BatchSchedulerConfig(max_batch_size=4, prefill_chunk_size=chunk)
    eng = ContinuousBatchingEngine(dec, cfg, use_graph=use_graph)
    reqs = [eng.submit(p, max_tokens=m) for p, m in zip(prompts, max_toks)]
    eng.run_until_idle()
    assert all(r.status == RequestStatus.COMPLETED for r in reqs)
    assert [len(r.generated_tokens) for r in reqs] == max_toks
    st = eng.get_stats()
    assert st["completed"] == 6 and st["active"] == 0 and st["total_generated"] == sum(max_toks)
    # six requests through four slots: later requests reused finished slots
    for p, m, r in zip(prompts, max_toks, reqs):
        alone = ContinuousBatchingEngine(dec, BatchSchedulerConfig(max_batch_size=4, prefill_chunk_size=1),
                                         use_graph=False)
        a = alone.submit(p, max_tokens=m)
        alone.run_until_idle()
        assert a.generated_tokens == r.generated_tokens, (p, a.generated_tokens, r.generated_tokens)


def test_eos_and_cancel(dev):
    dec = _decoder(dev)
    eng = ContinuousBatchingEngine(dec, use_graph=False)
    probe = eng.submit([5, 6, 7], max_tokens=4)
    eng.run_until_idle()
    eos = probe.generated_tokens[1]
    r = eng.submit([5, 6, 7], max_tokens=10, eos_token_id=eos)
    c = eng.submit([8, 9], max_tokens=10)
    eng.step()
    eng.cancel(c.request_id)
    eng.run_until_idle()
    stop = probe.generated_tokens.index(eos) + 1
    assert r.generated_tokens == probe.generated_tokens[:stop]  # stopped at the eos token
    assert c.status == RequestStatus.CANCELLED
    with pytest.raises(ValueError):
        eng.submit([1], temperature=0.7)
    with pytest.raises(ValueError):
        eng.submit([1] * 90, max_tokens=10)


@pytest.mark.parametrize("chunk", [1, 5, 16])
def test_chunked_prefill_matches_oracle(dev, chunk):
    """Prompts pushed through the batched step in chunks of `chunk` rows (the
    rows of one request attend causally over pages they fill in the same
    step), then greedy decoding: the oracle runs each request alone, one token
    per step from an empty cache, on the engine's own token sequence (prompt,
    then the engine's generated tokens as inputs).  Every generated token must
    carry the oracle's largest logit up to 0.05 (a near tie), and the oracle's
    clear winners must be the engine's tokens."""
    import numpy as np

    from oracle import decoder as odec
    from test_gpu_decoder import _export

    dec = _decoder(dev)
    model = _export(dec)
    s = dec.s
    prompts = [[3, 14, 15, 92, 65, 35, 89, 79], [9, 2, 6, 5, 3, 5, 8, 9, 7, 9, 3, 2, 3, 8, 4, 6, 2, 6], [7],
               [1, 4, 1, 4, 2, 1, 3, 5, 6, 2, 3, 7]]
    max_toks = [6, 4, 7, 5]
    eng = ContinuousBatchingEngine(dec, BatchSchedulerConfig(max_batch_size=4, prefill_chunk_size=chunk),
                                   use_graph=True)
    reqs = [eng.submit(p, max_tokens=m) for p, m in zip(prompts, max_toks)]
    eng.run_until_idle()
    exact = 0
    for p, r in zip(prompts, reqs):
        assert r.status == RequestStatus.COMPLETED
        seq = list(p) + list(r.generated_tokens)
        cache = [[{"k": np.zeros((0, s.n_kv_heads, s.head_dim), np.float32),
                   "v": np.zeros((0, s.n_kv_heads, s.head_dim), np.float32)}] for _ in range(dec.L)]
        for i in range(len(seq) - 1):
            logits, _, _ = odec.decode_step(model, cache, np.array([seq[i]], np.int64), np.array([i], np.int32))
            if i < len(p) - 1:
                continue  # prompt positions: the engine keeps no token there
            got = seq[i + 1]
            row = logits[0]
            top = float(row.max())
            assert row[got] >= top - 0.05, (p, i, got, int(row.argmax()), top - float(row[got]))
            second = float(np.sort(row)[-2])
            if top - second > 0.05:
                assert got == int(row.argmax())
            exact += int(got == int(row.argmax()))
    assert exact >= sum(max_toks) - 2
