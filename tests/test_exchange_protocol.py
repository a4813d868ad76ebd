"""Model check, on host threads, of the two tensor-parallel exchange protocols.

Python restatements of the device protocols, run by W rank threads that are
randomly delayed at every step.  Each reader asserts that it saw exactly the
data of the exchange it waits for: a stale slot, or one that a faster rank
has already overwritten, would be caught.  No GPU is involved: this checks the
protocol logic -- slot counts, tags, flag order -- not the CUDA code.

* Decode exchange (gemv.cu, EPI_PARTIAL / PRO_RESID_NORM): exchange x of step s
  stores every partial element as one (value, tag) pair, tag = 256 s + x, into
  slot (x - 1) & 1 of every rank; the reader re-reads each pair until it
  carries its tag.  Two slots suffice because producing exchange x + 1 needs
  every rank's exchange x.
* Prefill exchange (prefill.cu, tp_signal / tp_resid_rows): exchange seq writes
  the rank's own slot seq & 1, then raises flags[j][slot][rank] = seq on every
  rank j; a reader waits for all flags of its own buffer, then reads every
  rank's slot.  A rank rewrites a slot only two exchanges later, after every
  rank raised its flag for the exchange in between -- which each does only
  after reading the slot.
"""
import random
import threading
import time

import numpy as np
import pytest

N_ELEM = 16


def _jitter(rng):
    if rng.random() < 0.3:
        time.sleep(rng.random() * 2e-4)


def _partial(rank, x):
    return (np.arange(N_ELEM, dtype=np.float64) + 1.0) * (rank + 1) * 1000.0 + x


def _expected(world, x):
    return sum(_partial(r, x) for r in range(world))


def _run(world, target):
    errors = []
    threads = [threading.Thread(target=target, args=(r, errors)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    assert not any(t.is_alive() for t in threads), "a rank is stuck: the protocol deadlocked"
    assert not errors, errors[:3]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_decode_tagged_pairs_two_slots(world):
    steps, per_step = 3, 6  # xtag 1 .. per_step per step (2 per layer)
    # recv[j][slot][r][e] = (value, tag) as rank j's buffer
    recv = [[[[(0.0, 0)] * N_ELEM for _ in range(world)] for _ in range(2)] for _ in range(world)]

    def rank_main(me, errors):
        rng = random.Random(1000 + me)
        for s in range(1, steps + 1):
            for x in range(1, per_step + 1):
                tag = 256 * s + x
                slot = (x - 1) & 1
                vals = _partial(me, tag)
                # producer: one (value, tag) store per element into every rank, any order
                order = [(j, e) for j in range(world) for e in range(N_ELEM)]
                rng.shuffle(order)
                for j, e in order:
                    recv[j][slot][me][e] = (float(vals[e]), tag)
                    _jitter(rng) if rng.random() < 0.05 else None
                # consumer: every rank's pairs, each re-read until it carries the tag
                total = np.zeros(N_ELEM)
                for r in range(world):
                    for e in range(N_ELEM):
                        t0 = time.time()
                        while True:
                            v, t = recv[me][slot][r][e]
                            if t == tag:
                                break
                            if t > tag:
                                errors.append(f"rank {me} step {s} x {x}: slot overwritten by tag {t}")
                                return
                            if time.time() - t0 > 60:
                                errors.append(f"rank {me}: wait for tag {tag} timed out")
                                return
                            time.sleep(0)
                        total[e] += v
                if not np.array_equal(total, _expected(world, tag)):
                    errors.append(f"rank {me} step {s} x {x}: wrong sum")
                    return
                _jitter(rng)

    _run(world, rank_main)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_prefill_flags_two_slots(world):
    n_exchanges = 12
    part = [[np.zeros(N_ELEM) for _ in range(2)] for _ in range(world)]  # rank j's own slots
    flags = [[[0] * world for _ in range(2)] for _ in range(world)]      # flags[j][slot][rank]

    def rank_main(me, errors):
        rng = random.Random(2000 + me)
        for seq in range(1, n_exchanges + 1):
            slot = seq & 1
            # GEMM_F32: this rank's partial rows into its own slot
            vals = _partial(me, seq)
            for e in rng.sample(range(N_ELEM), N_ELEM):
                part[me][slot][e] = vals[e]
                _jitter(rng) if rng.random() < 0.05 else None
            # tp_signal: flags of every rank, after the data
            for j in rng.sample(range(world), world):
                flags[j][slot][me] = seq
            # tp_resid_rows: wait for every flag of this rank's buffer, then read every slot
            t0 = time.time()
            while any(flags[me][slot][r] != seq for r in range(world)):
                if any(flags[me][slot][r] > seq for r in range(world)):
                    errors.append(f"rank {me} seq {seq}: a flag ran ahead")
                    return
                if time.time() - t0 > 60:
                    errors.append(f"rank {me}: flag wait for {seq} timed out")
                    return
                time.sleep(0)
            total = np.zeros(N_ELEM)
            for r in range(world):
                _jitter(rng)
                total += part[r][slot]
            if not np.array_equal(total, _expected(world, seq)):
                errors.append(f"rank {me} seq {seq}: read a slot another rank had already rewritten")
                return
            _jitter(rng)

    _run(world, rank_main)
