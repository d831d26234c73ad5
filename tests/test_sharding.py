"""Multi-rank host logic on CPU: two gloo ranks run the sequence-sharded decode
bookkeeping that bench.py runs over NCCL (sequence ownership, max-over-ranks timing,
gathered output checksums, one batch split over the ranks with its outputs gathered to
rank 0 and proven by exact per-rank checksums), and a rank that dies is reported to its
peer as an error instead of a hang.
"""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

from bgtq import sharding

D, T, R = 16, 40, 3
TOTAL = 7        # one batch split over two ranks: 4 + 3 sequences


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _sequence_output(seq):
    """Attention of R query rows over T keys/values of one sequence, drawn from the
    sequence id alone, so the result does not depend on which rank computes it."""
    rng = np.random.default_rng(1000 + seq)
    q, k, v = rng.standard_normal((R, D)), rng.standard_normal((T, D)), rng.standard_normal((T, D))
    s = q @ k.T / np.sqrt(D)
    p = np.exp(s - s.max(1, keepdims=True))
    return (p / p.sum(1, keepdims=True)) @ v


def _rank_main(rank, world, port, per_rank, mode, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank))
    import torch
    dist = sharding.init_from_env("gloo", timeout_s=10.0)
    try:
        if mode == "die" and rank == 1:
            os._exit(3)  # leaves between steps: nothing of it is in flight
        outs = [torch.from_numpy(_sequence_output(s)) for s in sharding.sequence_range(per_rank, rank)]
        timing = sharding.max_over_ranks([0.25 * (rank + 1), -float(rank)], dist, "cpu")
        sums = sharding.gather_checksums(outs, dist, "cpu")
        # one batch of TOTAL sequences split over the ranks, outputs gathered to rank 0
        mine = sharding.split_range(TOTAL, world, rank)
        share = torch.stack([torch.from_numpy(_sequence_output(s)).float() for s in mine])
        counts = [len(sharding.split_range(TOTAL, world, r)) for r in range(world)]
        gathered = sharding.gather_to_root(share, counts, dist, "cpu")
        bits = sharding.gather_ints([sharding.bit_checksum(share)], dist, "cpu")
        sharding.barrier(dist)
        np.save(os.path.join(out_dir, f"rank{rank}.npy"), np.array(timing + sums))
        if rank == 0:
            np.save(os.path.join(out_dir, "gathered.npy"), gathered.numpy())
            np.save(os.path.join(out_dir, "bits.npy"), np.array([b[0] for b in bits] +
                                                                [sharding.bit_checksum(gathered[:counts[0]]),
                                                                 sharding.bit_checksum(gathered[counts[0]:])]))
    except Exception as e:  # the peer's death surfaces here
        with open(os.path.join(out_dir, f"rank{rank}.err"), "w") as f:
            f.write(type(e).__name__ + ": " + str(e)[:200])
    finally:
        if mode != "die":
            dist.destroy_process_group()


def _run(world, mode, tmp_path, per_rank=3, timeout=120):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, per_rank, mode, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung"
    return procs


def test_sequence_ownership_partitions_the_batch():
    assert list(sharding.sequence_range(4, 2)) == [8, 9, 10, 11]
    for total in (0, 1, 7, 256):
        for world in (1, 2, 3, 8):
            got = [i for r in range(world) for i in sharding.split_range(total, world, r)]
            assert got == list(range(total))
            sizes = [len(sharding.split_range(total, world, r)) for r in range(world)]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        sharding.split_range(4, 2, 2)


def test_single_process_needs_no_group(monkeypatch):
    import torch
    monkeypatch.delenv("WORLD_SIZE", raising=False)
    assert sharding.init_from_env("gloo") is None
    assert sharding.max_over_ranks([1.5, 2.0], None, "cpu") == [1.5, 2.0]
    x = torch.arange(6, dtype=torch.float32)
    assert sharding.gather_checksums([x, x], None, "cpu") == [30.0]


def test_two_gloo_ranks_max_timing_and_checksums(tmp_path):
    procs = _run(2, "ok", tmp_path)
    assert all(p.exitcode == 0 for p in procs)
    per_rank = 3
    expect = [sum(float(_sequence_output(s).sum()) for s in sharding.sequence_range(per_rank, r)) for r in range(2)]
    for r in range(2):
        got = np.load(tmp_path / f"rank{r}.npy")
        np.testing.assert_allclose(got[:2], [0.5, 0.0])          # max over ranks, element-wise
        np.testing.assert_allclose(got[2:], expect, rtol=1e-12)  # rank-ordered checksums
    # the split batch gathered to rank 0 equals the single-process outputs, bit for bit
    gathered = np.load(tmp_path / "gathered.npy")
    single = np.stack([_sequence_output(s).astype(np.float32) for s in range(TOTAL)])
    assert np.array_equal(gathered, single)
    bits = np.load(tmp_path / "bits.npy")
    assert bits[0] == bits[2] and bits[1] == bits[3]                # per-rank checksums prove the copy


def test_dead_rank_is_reported_not_waited_for(tmp_path):
    procs = _run(2, "die", tmp_path)
    assert procs[1].exitcode == 3
    err = (tmp_path / "rank0.err")
    assert err.exists(), "the surviving rank should see an error from its collective"
    assert not (tmp_path / "rank0.npy").exists()
