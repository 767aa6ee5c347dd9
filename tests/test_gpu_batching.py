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
