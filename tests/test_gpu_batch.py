"""Batched decode (csrc/batch.cu, q3_batch_*) against the oracle model.

Several sequences of different lengths decode together, each teacher-checked
on its own: the oracle consumes the sequence's tokens one by one
(Model::forward, qwen3.hpp:131-166) and at every generated position the
batch's greedy token is the oracle's argmax unless the two are a near-tie
(the oracle's logits of the two picks within 2 x 3e-2); the last step's BF16
logits match the oracle's within 3e-2 + 1 BF16 ulp with cosine >= 0.9999.
A 4-layer Qwen3-0.6B-shaped model with an 8192-token vocabulary keeps the
oracle fast."""
import numpy as np
import pytest

from gpu_util import bf, bf16_ulp

pytestmark = pytest.mark.gpu
CAP = 320


def _cfg():
    from inference_b200 import Qwen3Config

    return Qwen3Config("qwen3-batch", hidden=1024, inter=3072, layers=4, q_heads=16, kv_heads=8, vocab=8192, tied=True)


def _check_against_oracle(oracle, cfg, toks, n_forced_until, last_logits):
    """toks: the sequence's tokens, of which the first n_forced_until were given
    (not checked); last_logits: the batch's logits at the last consumed position."""
    from oracle import ModelConfig

    om = oracle.model(ModelConfig.make(cfg.hidden, cfg.inter, cfg.layers, cfg.q_heads, cfg.kv_heads, 128, cfg.vocab,
                                       CAP, tied=True), seed=0)
    try:
        for p in range(len(toks) - 1):
            om.forward(int(toks[p]))
            if p + 1 < n_forced_until:
                continue
            ref = bf(om.logits()).astype(np.float64)
            pick, best = int(toks[p + 1]), int(np.argmax(ref))
            assert pick == best or ref[best] - ref[pick] <= 2 * 3e-2, f"position {p}: {pick} vs oracle {best}"
        ref = bf(om.logits()).astype(np.float64)
        mine = bf(last_logits).astype(np.float64)
        d = np.abs(mine - ref)
        assert (d <= 3e-2 + bf16_ulp(ref)).all(), f"max |d| {d.max():.4g}"
        cos = mine @ ref / (np.linalg.norm(mine) * np.linalg.norm(ref))
        assert cos >= 0.9999
    finally:
        om.close()


def test_batch_sequences_match_oracle(oracle):
    from inference_b200 import Batch, Engine, prompt_ids

    cfg = _cfg()
    prompts = [prompt_ids(n, seed=10 + n, vocab=cfg.vocab) for n in (5, 70, 130)]
    with Engine(cfg, capacity=CAP) as e:
        e.init_synthetic(0)
        with Batch(e, max_seqs=4, pool_pages=16) as b:
            ids = [b.add(p, max_len=200) for p in prompts]
            b.step(60)
            for sid, p in zip(ids, prompts):
                assert b.position(sid) == len(p) - 1 + 60
                toks = b.tokens(sid)
                assert len(toks) == len(p) + 60
                np.testing.assert_array_equal(toks[: len(p)], p)
                _check_against_oracle(oracle, cfg, toks, len(p), b.logits(sid))


def test_batch_fork_shares_full_pages(oracle):
    """A fork references the full pages of its source and copies the partial
    one; both continue correctly, the fork on a forced continuation of its own,
    and releasing them returns every page."""
    from inference_b200 import Batch, Engine, prompt_ids

    cfg = _cfg()
    prompt = prompt_ids(100, seed=7, vocab=cfg.vocab)
    with Engine(cfg, capacity=CAP) as e:
        e.init_synthetic(0)
        with Batch(e, max_seqs=4, pool_pages=12) as b:
            free0 = b.free_pages
            a = b.add(prompt, max_len=256)  # 4 pages
            assert b.free_pages == free0 - 4
            b.step(30)  # position 129: pages 0 and 1 are full
            f = b.fork(a)
            assert b.free_pages == free0 - 4 - 2  # the fork takes fresh pages 2 and 3 only
            head = b.tokens(a)
            np.testing.assert_array_equal(b.tokens(f), head)
            forced = [11, 22, 33]
            b.append(f, forced)
            b.step(20)
            ta, tf = b.tokens(a), b.tokens(f)
            np.testing.assert_array_equal(tf[: len(head)], head)
            np.testing.assert_array_equal(tf[len(head): len(head) + 3], forced)
            _check_against_oracle(oracle, cfg, ta, len(prompt), b.logits(a))
            _check_against_oracle(oracle, cfg, tf, len(head) + 3, b.logits(f))
            b.release(f)
            assert b.free_pages == free0 - 4
            b.release(a)
            assert b.free_pages == free0


def test_batch_sequences_stop_at_their_length():
    from inference_b200 import Batch, Engine, Q3Error, prompt_ids

    cfg = _cfg()
    with Engine(cfg, capacity=CAP) as e:
        e.init_synthetic(0)
        with Batch(e, max_seqs=3, pool_pages=5) as b:
            short = b.add(prompt_ids(10, seed=1, vocab=cfg.vocab), max_len=16)
            long_ = b.add(prompt_ids(10, seed=2, vocab=cfg.vocab), max_len=64)
            b.step(30)
            assert b.position(short) == 15 and len(b.tokens(short)) == 16
            assert b.position(long_) == 9 + 30
            with pytest.raises(Q3Error, match="does not fit"):
                b.add(prompt_ids(16, seed=3, vocab=cfg.vocab), max_len=16)
            with pytest.raises(Q3Error, match="exhausted"):
                b.add(prompt_ids(8, seed=4, vocab=cfg.vocab), max_len=300)  # 5 pages; 3 are left
