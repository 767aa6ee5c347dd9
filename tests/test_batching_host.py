"""Host logic of the continuous-batching engine: FIFO admission, cancel, completion bookkeeping."""

import pytest

from b200flash.continuous_batching import BatchScheduler, BatchSchedulerConfig, InferenceRequest, RequestStatus


def test_fifo_admission_skips_cancelled():
    sch = BatchScheduler(BatchSchedulerConfig(max_batch_size=2))
    reqs = [InferenceRequest(prompt_tokens=[1, 2], request_id=f"r{i}") for i in range(4)]
    for r in reqs:
        sch.add_request(r)
    sch.cancel_request("r1")
    assert sch.next_waiting().request_id == "r0"
    assert sch.next_waiting().request_id == "r2"
    sch.mark_completed("r0")
    st = sch.get_stats()
    assert st == {"waiting": 1, "completed": 1, "cancelled": 1, "total": 4}
    assert reqs[0].status == RequestStatus.COMPLETED and reqs[0].completed_at is not None


def test_queue_limit_and_request_properties():
    sch = BatchScheduler(BatchSchedulerConfig(max_queue_size=1))
    sch.add_request(InferenceRequest(prompt_tokens=[5]))
    with pytest.raises(RuntimeError, match="queue is full"):
        sch.add_request(InferenceRequest(prompt_tokens=[6]))
    r = InferenceRequest(prompt_tokens=[1, 2, 3])
    assert not r.is_prefill_done and r.ttft_ms == 0.0 and r.tokens_per_second == 0.0
    r._prefill_pos = 3
    assert r.is_prefill_done
