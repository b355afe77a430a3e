"""Batch sharding (tosa_b200.parallel): shard arithmetic, split/concat, and the
one-process-per-rank path as two gloo ranks on the CPU, with the oracle standing
in for each rank's GPU run (the per-shard results must concatenate to the
whole-batch result, since every operator of the path is per sample)."""

import os
import socket

import numpy as np
import pytest

from oracle import oracle as O
from tosa_b200 import graphs
from tosa_b200 import interpreter as I
from tosa_b200 import parallel as P


@pytest.mark.parametrize("batch", [0, 1, 7, 64, 513])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shard_bounds_cover_the_batch(batch, world):
    spans = [P.shard_bounds(batch, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == batch
    for (lo0, hi0), (lo1, hi1) in zip(spans, spans[1:]):
        assert hi0 == lo1
    sizes = [hi - lo for lo, hi in spans]
    assert max(sizes) - min(sizes) <= 1


def test_shard_bounds_rejects_bad_requests():
    with pytest.raises(ValueError):
        P.shard_bounds(4, 0, 0)
    with pytest.raises(ValueError):
        P.shard_bounds(4, 2, 2)


def test_batch_axis_rule():
    assert P.batch_axis([2, 14, 14, 64], 2) == 0
    assert P.batch_axis([1, 64, 1000], 64) == 1
    with pytest.raises(ValueError):
        P.batch_axis([1, 1000], 64)


def test_split_concat_round_trip():
    rng = np.random.default_rng(1)
    x = rng.integers(-128, 128, (6, 3, 4, 2)).astype(np.int8)
    t = {"x": I.Tensor.from_numpy("x", x, 3)}
    parts = P.split_batch(t, 3)
    assert [p["x"].shape for p in parts] == [[2, 3, 4, 2]] * 3
    back = P.concat_batch(parts)
    assert back["x"].shape == [6, 3, 4, 2] and np.array_equal(back["x"].data, x)
    with pytest.raises(ValueError):
        P.split_batch(t, 4)


def _oracle_outputs(data, images):
    block = O.read_graph(data).main_block
    name = block.inputs[0]
    res = O.run_block(block, {name: O.T(3, list(images.shape), images.astype(np.int64).reshape(-1))})
    return {k: v.values.reshape(v.shape) for k, v in res.items()}, block.outputs


def _rank_main(rank, world, port, images, result_path):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lo, hi = P.shard_bounds(images.shape[0], world, rank)
        data, _ = graphs.residual_block_int8(batch=hi - lo)
        outs, names = _oracle_outputs(data, images[lo:hi])
        local = {nm: I.Tensor(nm, list(outs[nm].shape), 3, outs[nm]) for nm in names}
        axes = {nm: P.batch_axis(outs[nm].shape, hi - lo) for nm in names}  # logits [1, batch, 16]: axis 1
        gathered = P.gather_to_rank0(local, axes)
        slowest = P.max_over_ranks(float(rank + 1))
        if rank == 0:
            np.savez(result_path, slowest=slowest, **{k: np.asarray(v.data) for k, v in gathered.items()})
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_shard_and_gather(tmp_path):
    import torch.multiprocessing as mp

    world, batch = 2, 4
    images = np.random.default_rng(5).integers(-128, 128, (batch, 14, 14, 64)).astype(np.int8)
    path = str(tmp_path / "gathered.npz")
    mp.start_processes(_rank_main, args=(world, _free_port(), images, path), nprocs=world, start_method="spawn",
                       join=True)
    got = np.load(path)
    assert float(got["slowest"]) == float(world)
    whole, names = _oracle_outputs(graphs.residual_block_int8(batch=batch)[0], images)
    for nm in names:
        assert np.array_equal(got[nm], whole[nm]), nm


def _failing_rank_main(rank, world, port, images, result_path):
    """One rank of a sharded step in which TB_FAULT_SHARD makes shard 1 fail: every rank
    must end the step with ShardError naming shard 1, and the process group must stay
    consistent afterwards (a barrier completes)."""
    import json

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        lo, hi = P.shard_bounds(images.shape[0], world, rank)
        data, _ = graphs.residual_block_int8(batch=hi - lo)
        outcome = {"rank": rank}
        try:
            P.sharded_step(lambda: _oracle_outputs(data, images[lo:hi]), rank)
            outcome["error"] = None
        except P.ShardError as e:
            outcome["error"] = e.shard
            outcome["injected"] = isinstance(e.__cause__, P.InjectedFault)
        dist.barrier()
        with open(f"{result_path}.{rank}", "w") as f:
            json.dump(outcome, f)
    finally:
        dist.destroy_process_group()


def test_failed_shard_ends_the_step_on_every_rank(tmp_path, monkeypatch):
    import json

    import torch.multiprocessing as mp

    world = 2
    images = np.random.default_rng(6).integers(-128, 128, (2, 14, 14, 64)).astype(np.int8)
    path = str(tmp_path / "outcome")
    monkeypatch.setenv("TB_FAULT_SHARD", "1")  # inherited by the spawned ranks
    ctx = mp.start_processes(_failing_rank_main, args=(world, _free_port(), images, path), nprocs=world,
                             start_method="spawn", join=False)
    import time
    deadline = time.time() + 120
    while not ctx.join(timeout=5):
        assert time.time() < deadline, "ranks did not finish: a rank is waiting on the failed one"
    outcomes = [json.load(open(f"{path}.{r}")) for r in range(world)]
    assert [o["error"] for o in outcomes] == [1, 1]   # every rank reports shard 1
    assert outcomes[1]["injected"] and not outcomes[0]["injected"]


def test_sharded_step_without_a_process_group(monkeypatch):
    monkeypatch.delenv("TB_FAULT_SHARD", raising=False)
    assert P.sharded_step(lambda: 7, 0) == 7
    monkeypatch.setenv("TB_FAULT_SHARD", "0")
    with pytest.raises(P.ShardError) as ei:
        P.sharded_step(lambda: 7, 0)
    assert ei.value.shard == 0 and isinstance(ei.value.__cause__, P.InjectedFault)
