"""Sentence sharding over ranks: planner properties and a 2-rank gloo run.

The ranks run the CPU oracle on their shards (no GPU here); the test checks
the host logic around the attention path: every sentence computed exactly
once, by the rank the deterministic plan names, gathered into the same
results a single process produces.
"""
import os
import socket

import numpy as np
import pytest

from nllb_attn import sharding


def test_plan_covers_each_sentence_once():
    rng = np.random.default_rng(4)
    lengths = rng.integers(18, 131, size=1024)
    for world in (1, 2, 4, 8):
        shards = sharding.plan_shards(lengths, world)
        flat = sorted(i for s in shards for i in s)
        assert flat == list(range(len(lengths)))
        loads = sharding.shard_loads(lengths, shards)
        # LPT bound: max load <= mean + largest single cost
        biggest = max(sharding.sentence_cost(int(n), 132) for n in lengths)
        assert max(loads) <= sum(loads) / world + biggest
        assert max(loads) / (sum(loads) / world) < 1.01


def test_plan_is_deterministic_and_handles_few_sentences():
    assert sharding.plan_shards([20, 30, 40], 8) == sharding.plan_shards([20, 30, 40], 8)
    shards = sharding.plan_shards([20, 30, 40], 8)
    assert sum(len(s) for s in shards) == 3 and sum(1 for s in shards if not s) == 5
    with pytest.raises(ValueError):
        sharding.plan_shards([1], 0)


def test_decode_steps_follows_reference_rule():
    assert sharding.decode_steps(18, 36) == 32      # config 0: 32 target tokens
    assert sharding.decode_steps(18, 132) == 64     # 3*18+10
    assert sharding.decode_steps(130, 132) == 128   # capped by max_gen - 4


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _sentence_result(i, n_src):
    import pyoracle as po
    K = po.det_uniform(1000 + i, (n_src, 1024))
    V = po.det_uniform(2000 + i, (n_src, 1024))
    q = po.det_uniform(3000 + i, (4, 1024))
    return po.cross(K, V, q)


def _worker(rank, world, port, lengths, outdir):
    import sys
    import torch.distributed as dist
    here = os.path.dirname(os.path.abspath(__file__))
    repo = os.path.dirname(here)
    sys.path[:0] = [os.path.join(repo, "bare-metal-nllb_b200"), os.path.join(repo, "oracle")]
    from nllb_attn import sharding as sh
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = sh.plan_shards(lengths, world)[rank]
        local = {i: _sentence_result(i, lengths[i]) for i in mine}
        merged = sh.gather_results(local)
        if rank == 0:
            np.savez(os.path.join(outdir, "merged.npz"),
                     **{str(k): v for k, v in merged.items()})
            np.save(os.path.join(outdir, "owners.npy"),
                    np.array([r for i in range(len(lengths))
                              for r, s in enumerate(sh.plan_shards(lengths, world)) if i in s]))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_run_matches_single_process(tmp_path):
    import torch.multiprocessing as mp
    lengths = [18, 130, 44, 77, 19, 101, 64, 23]
    port = _free_port()
    mp.start_processes(_worker, args=(2, port, lengths, str(tmp_path)), nprocs=2,
                       start_method="spawn", join=True)
    merged = np.load(tmp_path / "merged.npz")
    assert sorted(int(k) for k in merged.files) == list(range(len(lengths)))
    for i, n in enumerate(lengths):
        np.testing.assert_array_equal(merged[str(i)], _sentence_result(i, n))
    owners = np.load(tmp_path / "owners.npy")
    assert set(owners.tolist()) == {0, 1}
