"""GrowingKVCache's host logic, as the reference's own cache tests check it
(tests/test_kv_cache.py): the growth rule, the hard capacity, the order of
the history and the failed append that changes nothing.  The buffers live on
the CPU here; the GPU tests use the same class on the device."""

from __future__ import annotations

import pytest
import torch

from gdn_b200 import GrowingKVCache

HEADS, DIM = 2, 3


def _cache(max_context):
    return GrowingKVCache(max_context, HEADS, DIM, dtype=torch.float16, device="cpu")


def _token(value):
    return torch.full((HEADS, DIM), value, dtype=torch.float16)


def _values(cache):
    keys, _ = cache.state()
    return [float(keys[0, i, 0]) for i in range(keys.shape[1])]


def test_rejects_nonpositive_context():
    with pytest.raises(ValueError):
        GrowingKVCache(0, 1, 1, device="cpu")


def test_matches_full_history():
    cache = _cache(16)
    for v in range(7):
        cache.append(_token(float(v)), _token(float(v)))
    assert cache.size == 7
    assert _values(cache) == [float(v) for v in range(7)]


def test_raises_once_context_is_exceeded():
    cache = _cache(3)
    for v in (1.0, 2.0, 3.0):
        cache.append(_token(v), _token(v))
    with pytest.raises(IndexError):
        cache.append(_token(4.0), _token(4.0))


def test_allocation_follows_used_context():
    cache = GrowingKVCache(32768, HEADS, DIM, dtype=torch.float16, device="cpu")
    assert cache.allocated_size == 0
    cache.append(_token(1.0), _token(2.0))
    assert cache.allocated_size == 256 and cache.capacity == 32768


def test_batch_append_crosses_growth_boundaries_and_preserves_history():
    cache = GrowingKVCache(600, HEADS, DIM, dtype=torch.float32, device="cpu")
    keys = torch.arange(600, dtype=torch.float32)[None, :, None].expand(HEADS, 600, DIM).contiguous()
    values = -keys
    for start, end in ((0, 255), (255, 258), (258, 599), (599, 600)):
        cache.append_many(keys[:, start:end], values[:, start:end])
        k, v = cache.state()
        assert torch.equal(k, keys[:, :end]) and torch.equal(v, values[:, :end])
        assert end <= cache.allocated_size <= min(end + 255, cache.capacity)


def test_failed_batch_append_leaves_history_unchanged():
    cache = _cache(3)
    cache.append(_token(1.0), _token(2.0))
    with pytest.raises(IndexError):
        cache.append_many(torch.zeros(HEADS, 3, DIM, dtype=torch.float16),
                          torch.zeros(HEADS, 3, DIM, dtype=torch.float16))
    assert cache.size == 1
    keys, values = cache.state()
    assert torch.equal(keys[:, 0], _token(1.0)) and torch.equal(values[:, 0], _token(2.0))


def test_shape_checks():
    cache = _cache(8)
    with pytest.raises(ValueError):
        cache.append_many(torch.zeros(HEADS, 2, DIM), torch.zeros(HEADS, 3, DIM))
    with pytest.raises(ValueError):
        cache.append_many(torch.zeros(HEADS + 1, 2, DIM), torch.zeros(HEADS + 1, 2, DIM))
    assert cache.size == 0
