"""Loader invariants (every rank exactly T+1 tokens, documents start at BOS, caps), shard IO,
bigram hash and prefix table."""
import numpy as np
import pytest
import torch

from modded_nanogpt_b200.data import shards
from modded_nanogpt_b200.data.loader import Shard, TokenLoader, bigram_hash, distributed_data_generator
from modded_nanogpt_b200.data.prefix import build_prefix_table, synthetic_ranks


def test_shard_roundtrip(tmp_path):
    toks = shards.synth_tokens(10_000, seed=3)
    assert toks[0] == shards.BOS_ID and toks.dtype == np.uint16 and toks.size == 10_000
    p = tmp_path / "a.bin"
    shards.write_shard(p, toks)
    hdr = np.fromfile(p, dtype=np.int32, count=256)
    assert hdr[0] == 20240520 and hdr[1] == 1 and hdr[2] == 10_000
    back = shards.read_shard(p, pin=False)
    assert np.array_equal(back.numpy(), toks)


def test_shard_bad_magic(tmp_path):
    p = tmp_path / "bad.bin"
    p.write_bytes(b"\0" * 2048)
    with pytest.raises(ValueError):
        shards.read_shard(p, pin=False)


def test_synth_statistics():
    toks = shards.synth_tokens(400_000, seed=0)
    bos = np.flatnonzero(toks == shards.BOS_ID)
    lens = np.diff(bos)
    assert 350 < np.median(lens) < 900                      # lognormal, median ~600
    assert lens.max() <= 4096
    body = toks[toks != shards.BOS_ID]
    assert body.max() < 50256
    assert (body == 0).mean() > (body == 10).mean() > (body == 1000).mean()   # Zipf ordering
    assert np.array_equal(toks, shards.synth_tokens(400_000, seed=0))            # deterministic


def test_next_batch_invariants():
    toks = torch.from_numpy(shards.synth_tokens(200_000, seed=1, doc_len="geometric", mean_len=150.0))
    for world in (1, 2, 4):
        sh = Shard(toks, world)
        for T, cap in ((1024, 256), (4096, 896)):
            starts, ends = sh.next_batch(T, cap)
            for r in range(world):
                total = sum(e - s for s, e in zip(starts[r], ends[r]))
                assert total == T + 1
                for s, e in zip(starts[r], ends[r]):
                    assert toks[s] == shards.BOS_ID and 0 < e - s <= cap
                    assert not (toks[s + 1:e] == shards.BOS_ID).any()
    sh = Shard(toks[:5000], 1)
    with pytest.raises(StopIteration):
        for _ in range(100):
            sh.next_batch(1024, 256)


def test_ranks_get_disjoint_consecutive_docs(tiny_corpus):
    pat = tiny_corpus + "/data/fineweb10B/fineweb_train_*.bin"
    whole = TokenLoader(pat, 2048, 256, 2, True, 0, 1)        # 1 rank, 2 micro-batches
    a, b = whole.next_batch(), whole.next_batch()
    r0 = TokenLoader(pat, 2048, 256, 1, True, 0, 2).next_batch()
    r1 = TokenLoader(pat, 2048, 256, 1, True, 1, 2).next_batch()
    assert torch.equal(a.inputs, r0.inputs) and torch.equal(b.inputs, r1.inputs)
    assert torch.equal(a.targets, r0.targets) and torch.equal(b.cum_seqlens, r1.cum_seqlens)


def test_batch_layout(tiny_corpus):
    pat = tiny_corpus + "/data/fineweb10B/fineweb_train_*.bin"
    ld = TokenLoader(pat, 4096, 512, 1, True, 0, 1, bigram_vocab_size=3072)
    b = ld.next_batch()
    T = 4096
    assert b.inputs.dtype == torch.int32 and b.targets.dtype == torch.int64 and b.cum_seqlens.dtype == torch.int32
    assert b.inputs.shape == (T,) and torch.equal(b.inputs[1:].long(), b.targets[:-1])
    cu = b.cum_seqlens
    assert cu[0] == 0 and cu[-1] == T and (cu[1:] >= cu[:-1]).all() and cu.numel() % 128 == 0
    real = cu[cu < T]
    assert (b.inputs[real.long()] == shards.BOS_ID).all()       # every document starts with BOS
    assert (torch.diff(torch.cat([real, torch.tensor([T], dtype=torch.int32)])) <= 512).all()
    assert np.array_equal(b.bigram_cpu, b.bigram_inputs.numpy())
    # reparameterise like the reference generator's .send()
    b2 = ld.next_batch((8192, 256, 2))
    assert b2.inputs.shape == (4096,)


def test_generator_facade_and_val(tiny_corpus):
    pat = tiny_corpus + "/data/fineweb10B/fineweb_val_*.bin"
    g = distributed_data_generator(pat, 4096, -1, 2, align_to_bos=False, rank=1, world_size=2)
    inp, tgt, cu, bg, bg_cpu = next(g)
    raw = shards.read_shard(tiny_corpus + "/data/fineweb10B/fineweb_val_000000.bin", pin=False)
    assert torch.equal(inp, raw[1024:2048].to(torch.int32))
    assert torch.equal(tgt, raw[1025:2049].to(torch.int64))
    inp2, *_ = g.send((4096, -1, 2))
    assert torch.equal(inp2, raw[2048 + 1024:2048 + 2048].to(torch.int32))


def test_loader_resume(tiny_corpus):
    pat = tiny_corpus + "/data/fineweb10B/fineweb_train_*.bin"
    a = TokenLoader(pat, 2048, 256, 1, True, 0, 1)
    for _ in range(3):
        a.next_batch()
    st = a.state_dict()
    want = a.next_batch().inputs
    b = TokenLoader(pat, 2048, 256, 1, True, 0, 1)
    b.load_state_dict(st)
    assert torch.equal(b.next_batch().inputs, want)


def test_loader_crosses_shards(tiny_corpus):
    pat = tiny_corpus + "/data/fineweb10B/fineweb_train_*.bin"
    ld = TokenLoader(pat, 16384, 1024, 1, True, 0, 1)
    n = 0
    with pytest.raises(StopIteration):
        while True:
            ld.next_batch()
            n += 1
    assert n >= 15 and ld.file_idx == 1


def test_bigram_hash():
    x = torch.tensor([5, 7, 50256, 3], dtype=torch.int32)
    h = bigram_hash(x, 1000)
    mod = 999
    assert h[0] == mod and h.dtype == torch.int32
    for i in range(1, 4):
        assert h[i] == ((36313 * int(x[i])) ^ (27191 * int(x[i - 1]))) % mod
    big = torch.full((8,), 50303, dtype=torch.int32)
    assert (bigram_hash(big, 50304 * 15 // 2) >= 0).all()


def test_prefix_table_toy_vocab():
    vocab = {b"a": 0, b"ab": 1, b"abc": 2, b"b": 3, b"abd": 4, b"x": 5, b"abcde": 6}
    t = build_prefix_table(8, vocab)
    assert t.tolist() == [-1, 0, 1, -1, 1, -1, 2, -1]
    syn = synthetic_ranks(2000)
    t2 = build_prefix_table(2048, syn)
    inv = {i: b for b, i in syn.items()}
    for tid in range(256, 1999, 97):
        p = int(t2[tid])
        assert p >= 0 and inv[tid].startswith(inv[p]) and len(inv[p]) < len(inv[tid])
