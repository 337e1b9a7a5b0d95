"""Chunked prefill on the CPU: the chunker's behaviour (the reference's
tests/unit/test_scheduler.py TestChunkedPrefillScheduler cases) and the causal
prefill oracle's own properties."""
import numpy as np
import pytest

from mlxz_b200.engine.prefill import ChunkedPrefillScheduler
from oracle import paged as opaged
from oracle import rng


def test_short_prompt_single_chunk():
    c = ChunkedPrefillScheduler(chunk_size=256)
    tokens = list(range(100))
    assert not c.needs_chunking(tokens)
    chunk = c.get_next_chunk("r", tokens)
    assert chunk.is_last and len(chunk.tokens) == 100 and chunk.start_pos == 0
    assert chunk.total_prompt_tokens == 100


def test_long_prompt_multiple_chunks():
    c = ChunkedPrefillScheduler(chunk_size=4)
    tokens = list(range(10))
    assert c.needs_chunking(tokens)
    got = [c.get_next_chunk("r", tokens) for _ in range(3)]
    assert [ch.tokens for ch in got] == [[0, 1, 2, 3], [4, 5, 6, 7], [8, 9]]
    assert [ch.start_pos for ch in got] == [0, 4, 8]
    assert [ch.is_last for ch in got] == [False, False, True]


def test_exact_boundary_and_reset():
    c = ChunkedPrefillScheduler(chunk_size=4)
    tokens = list(range(8))
    c.get_next_chunk("r", tokens)
    last = c.get_next_chunk("r", tokens)
    assert last.is_last and len(last.tokens) == 4
    assert c.get_progress("r") == 8
    c.reset("r")
    assert c.get_progress("r") == 0
    assert c.chunk_size == 4


def test_invalid_chunk_size():
    with pytest.raises(ValueError):
        ChunkedPrefillScheduler(chunk_size=0)


def _f(shape, stream):
    return rng.to_f32(rng.normal(11, shape, "bf16", stream=stream), "bf16").astype(np.float64)


@pytest.mark.parametrize("G", [1, 4])
def test_prefill_rows_are_decodes_over_their_prefix(G):
    """Row i of a chunk at offset `start` is plain (unmasked) attention of that
    query over keys [0, start + i]."""
    Hkv, D, start, n = 2, 64, 37, 9
    q = _f((Hkv * G, n, D), 1)
    k, v = _f((Hkv, start + n, D), 2), _f((Hkv, start + n, D), 3)
    out = opaged.prefill_attention(q, k, v, start)
    for i in range(n):
        ref = opaged.attention(q[:, i:i + 1], k[:, :start + i + 1], v[:, :start + i + 1])
        np.testing.assert_allclose(out[:, i:i + 1], ref, rtol=1e-12, atol=1e-12)


def test_chunked_prefill_equals_whole_prompt():
    """Chunks of 5 at growing offsets give the whole prompt's causal attention."""
    H, D, T = 2, 32, 23
    q, k, v = _f((H, T, D), 4), _f((H, T, D), 5), _f((H, T, D), 6)
    whole = opaged.prefill_attention(q, k, v, 0)
    parts = [opaged.prefill_attention(q[:, a:a + 5], k[:, :min(a + 5, T)], v[:, :min(a + 5, T)], a)
             for a in range(0, T, 5)]
    np.testing.assert_allclose(np.concatenate(parts, axis=1), whole, rtol=1e-12, atol=1e-12)


def test_paged_prefill_oracle_matches_contiguous():
    """The batched pool form equals prefill_attention on the gathered KV."""
    bs, Hkv, D, G = 16, 2, 64, 2
    ctx, qlen = [40, 16, 5], [7, 16, 0]
    nb = 8
    kp = rng.normal(3, (nb, Hkv, bs, D), "f16", stream=1)
    vp = rng.normal(3, (nb, Hkv, bs, D), "f16", stream=2)
    tables = np.array([[5, 1, 3], [0, -1, -1], [7, -1, -1]], dtype=np.int32)
    T = sum(qlen)
    q = rng.normal(3, (T, Hkv * G, D), "f16", stream=3)
    qs = np.array([0, 7, 23], dtype=np.int32)
    out = opaged.paged_prefill(q, kp, vp, tables, qs, np.array(qlen), np.array(ctx), "f16")
    kb, vb = opaged.gather(kp, vp, [5, 1, 3], 40, bs)
    ref = opaged.prefill_attention(rng.to_f32(q[:7], "f16").transpose(1, 0, 2),
                                   rng.to_f32(kb, "f16"), rng.to_f32(vb, "f16"), 33)
    np.testing.assert_allclose(out[:7], ref.transpose(1, 0, 2), rtol=1e-12, atol=1e-12)


def test_prefill_step_host_metadata():
    """PagedPrefillStep's host side on a CPU store (no kernel runs): tables grow
    for the chunks, slots follow the tables from each sequence's offset, the
    chunks stack in order, and finish() advances the offsets once."""
    import torch

    from mlxz_b200.engine import PagedKVStore, PagedPrefillStep

    bs = 16
    store = PagedKVStore(1, 32, 2, 64, bs, torch.float16, device="cpu")
    store.add_sequence("a", 0)
    store.add_sequence("b", 20)
    store.add_sequence("c", 5)
    step = PagedPrefillStep(store, [("a", 40), ("b", 12), ("c", 0)], n_heads=8)
    assert step.T == 52 and step.max_q_len == 40
    assert step.q_start.tolist() == [0, 40, 52]
    assert step.q_len.tolist() == [40, 12, 0]
    assert step.ctx_lens.tolist() == [40, 32, 5]
    ta, tb = store.tables["a"], store.tables["b"]
    assert len(ta) == 3 and len(tb) == 2
    want = [ta[p // bs] * bs + p % bs for p in range(40)] + \
           [tb[p // bs] * bs + p % bs for p in range(20, 32)]
    assert step.slots.tolist() == want
    assert step.tables.shape == (3, 3)
    assert step.tables[1, :2].tolist() == tb and step.tables[1, 2].item() == -1
    step.finish()
    step.finish()
    assert [store.offsets[s] for s in "abc"] == [40, 32, 5]
    with pytest.raises(ValueError):
        PagedPrefillStep(store, [("a", 1)], n_heads=7)
