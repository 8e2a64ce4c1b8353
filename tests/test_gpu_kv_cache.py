"""The batch-aware KV cache (bm_kv_cache_*) on the GPU.

Each sequence keeps its own length; append() hands out per-sequence positions
for a batch of tokens from interleaved sequences, and bm_rope_kv_store writes
those tokens into the cache exactly where the oracle puts them. With one
sequence the positions are the reference KVCache's single running position
(src/kv_cache.cu:38-47).
"""
import numpy as np
import pytest
import torch

from baremetalinferenceengine_b200 import ops
from baremetalinferenceengine_b200._lib import BMError
from oracle import oracle as orc
from tests.helpers import TOL, bits_equal, from_np, gen, randn, to_np

pytestmark = pytest.mark.gpu


def device_ints(ptr, n, device):
    return torch.as_tensor(ops._DeviceArray(ptr, (n,), "<i4"), device=device).clone().cpu()


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def test_interleaved_sequences_get_their_own_positions(cuda, dt):
    layers, seqs, hkv, max_seq, hd, hq = 2, 3, 2, 16, 64, 4
    cache = ops.KVCache(layers, seqs, hkv, max_seq, hd, max_tokens=32, dtype=dt, device=cuda)
    table = ops.RopeTable(max_seq, hd, 1e4, cuda)
    want_k = [np.zeros((seqs, hkv, max_seq, hd), np.float32 if dt == torch.float32 else np.uint16)
              for _ in range(layers)]
    want_v = [w.copy() for w in want_k]
    batches = [[0, 1, 0, 2, 2, 0], [1, 1], [2, 0, 1, 2]]
    counters = [0] * seqs
    g = gen(5)
    for batch in batches:
        appended = cache.append(batch)
        pos = device_ints(appended[0], len(batch), cuda)
        seq = device_ints(appended[1], len(batch), cuda)
        expect = []
        for s in batch:
            expect.append(counters[s])
            counters[s] += 1
        assert pos.tolist() == expect and seq.tolist() == batch
        for layer in range(layers):
            q, k, v = randn((len(batch), hq, hd), dt, g), randn((len(batch), hkv, hd), dt, g), \
                randn((len(batch), hkv, hd), dt, g)
            qd = q.to(cuda)
            cache.rope_kv_store(layer, qd, k.to(cuda), v.to(cuda), appended, table=table, theta=1e4)
            wq, want_k[layer], want_v[layer], bad = orc.rope_kv_store(
                to_np(q), to_np(k), to_np(v), pos.numpy(), want_k[layer], want_v[layer], 1e4, seq_ids=seq.numpy())
            assert bad == 0
            assert orc.worst_error(to_np(qd), wq) <= TOL[dt]
    for s in range(seqs):
        assert cache.seq_len(s) == counters[s]
    for layer in range(layers):
        kc, vc = cache.views(layer)
        assert orc.worst_error(to_np(kc), want_k[layer]) <= TOL[dt]
        assert bits_equal(vc, from_np(want_v[layer]))
    cache.close()


def test_overflow_changes_nothing_and_reset(cuda):
    cache = ops.KVCache(1, 2, 1, 4, 8, max_tokens=8, dtype=torch.float32, device=cuda)
    cache.append([0, 0, 0])
    with pytest.raises(BMError):
        cache.append([1, 0, 0])  # sequence 0 would pass max_seq 4
    assert cache.seq_len(0) == 3 and cache.seq_len(1) == 0
    with pytest.raises(BMError):
        cache.append([0] * 9)  # more than max_tokens
    with pytest.raises(BMError):
        cache.append([2])  # no such sequence
    cache.reset(0)
    assert cache.seq_len(0) == 0
    cache.append([1, 1])
    cache.reset()
    assert cache.seq_len(1) == 0
    pos, _, n = cache.append([])
    assert n == 0
    cache.close()


def test_one_sequence_matches_the_reference_running_position(cuda):
    """num_seqs = 1: positions continue across calls like KVCache::increment_seq_pos."""
    cache = ops.KVCache(1, 1, 1, 64, 8, max_tokens=16, dtype=torch.float32, device=cuda)
    seen = []
    for n in (1, 5, 3, 1):
        appended = cache.append([0] * n)
        seen += device_ints(appended[0], n, cuda).tolist()
    assert seen == list(range(10))
    cache.close()
