"""The resident expert store keeps the expert cache's provider interface
(expert_cache.py:828, 990-1213): current_batched, get_many, iter_ready,
prefetch_layer, batched_layer, record_gather_qmm, with the same argument
checks.  Host logic only (CPU tensors stand in for the resident weights)."""
import pytest
import torch

import whallm_b200 as W


def _store():
    E, I, H = 4, 64, 64
    b = W.BatchedExperts(None, None, torch.zeros(E, H, I // 2, dtype=torch.uint8),
                         torch.zeros(E, H, I // 32, dtype=torch.uint8), None, None,
                         torch.arange(E, dtype=torch.uint8).view(E, 1, 1).expand(E, 2 * I, H // 2).contiguous(),
                         torch.zeros(E, 2 * I, H // 32, dtype=torch.uint8))
    return W.ResidentExpertStore({3: b}), b


def test_provider_interface():
    s, b = _store()
    assert s.current_batched(3) is b and s.current_batched(0) is None
    got = list(s.iter_ready(3, [2, 0, 2]))
    assert [e for e, _ in got] == [0, 2]
    assert int(got[1][1].w13[0, 0]) == 2
    r = s.get_many(3, [1, 1, 3])
    assert r.slots == {1: 0, 3: 1}
    with s.batched_layer(3) as bl:
        assert bl is b
    with s.batched_layer(3, enabled=False) as bl:
        assert bl is None
    s.prefetch_layer(7)                                   # out of range: nothing to do
    s.record_gather_qmm(3)
    assert s.metrics.gather_qmm_calls == 3


@pytest.mark.parametrize("call,msg", [
    (lambda s: list(s.iter_ready(0, [1])), "invalid layer"),
    (lambda s: list(s.iter_ready(3, [9])), "invalid expert"),
    (lambda s: s.get_many(3, [-1]), "invalid expert"),
    (lambda s: s.prefetch_layer(3, []), "cannot be empty"),
])
def test_provider_rejects(call, msg):
    s, _ = _store()
    with pytest.raises(ValueError, match=msg):
        call(s)


def test_unfused_experts_are_fused_once():
    # a store that supplies w1 and w3 separately gets [w3; w1] built on the first call and reused afterwards
    w1 = torch.arange(2 * 4 * 8, dtype=torch.uint8).view(2, 4, 8)
    w3 = w1 + 100
    s1 = torch.ones(2, 4, 1, dtype=torch.uint8)
    s3 = s1 * 2
    b = W.BatchedExperts(w1, s1, w1, s1, w3, s3)
    a13, a_s, calls = b.fused()
    b13, b_s, _ = b.fused()
    assert calls == 3
    assert a13 is b13 and a_s is b_s
    assert torch.equal(a13, torch.cat([w3, w1], dim=-2))
    assert torch.equal(a_s, torch.cat([s3, s1], dim=-2))
