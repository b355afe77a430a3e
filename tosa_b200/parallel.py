"""Batch sharding over the GPUs of one box.

Every operator of the accelerated path works per sample (CONV2D, DEPTHWISE,
pools, RESCALE, CLAMP and ADD on NHWC batches; MATMUL row by row), so a graph
run over a batch is the concatenation of runs over slices of it: the batch
dimension shards across GPUs with no exchange step and no collective on the
data path. Outputs are gathered back to the host in shard order.

Two ways to use it:

* ``ShardedInterpreter`` -- one process drives several GPUs: one host thread,
  stream and Interpreter (graph runner) per device, so the shards run
  concurrently.
* one process per GPU (``torchrun``): each rank takes ``shard_bounds`` of the
  global batch and runs its own Interpreter; ``max_over_ranks`` combines the
  ranks' timings (the only collective, outside the data path) and
  ``gather_to_rank0`` brings outputs to rank 0 over the process group.
"""

from __future__ import annotations

import os

import numpy as np

from . import interpreter as I


class ShardError(RuntimeError):
    """A shard of a data-parallel run failed. `shard` is its index (the rank, or the
    device slot of a ShardedInterpreter); the run as a whole returns this error (the
    reference's run_graph returns Err for the batch), after every other shard has
    finished its own work."""

    def __init__(self, shard: int, msg: str):
        super().__init__(f"shard {shard}: {msg}")
        self.shard = shard


class InjectedFault(RuntimeError):
    """The failure TB_FAULT_SHARD asked for."""


def injected_shards() -> set:
    """Shards told to fail by TB_FAULT_SHARD (a comma-separated list of shard indices):
    host-side fault injection for the failure-handling tests. Nothing on the device is
    made to fail: the shard raises before its work starts."""
    spec = os.environ.get("TB_FAULT_SHARD", "").strip()
    return {int(v) for v in spec.split(",") if v.strip()} if spec else set()


def sharded_step(work, rank: int = 0):
    """Run this rank's share of a one-process-per-GPU step, `work()`, and agree on the
    outcome: every rank joins one all-reduce of a failure flag whether its work succeeded
    or not, so a failed shard ends the step on every rank with ShardError and no rank is
    left waiting in a later collective (every rank takes the same collective steps in the
    same order). Returns work()'s result."""
    import torch
    import torch.distributed as dist

    err = None
    res = None
    try:
        if rank in injected_shards():
            raise InjectedFault(f"TB_FAULT_SHARD: shard {rank} fails before its run")
        res = work()
    except Exception as e:  # the error is this shard's; report it after the agreement
        err = e
    failed = rank + 1 if err is not None else 0
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
        t = torch.tensor([failed], dtype=torch.int64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        failed = int(t.item())
    if err is not None:
        raise ShardError(rank, str(err)) from err
    if failed:
        raise ShardError(failed - 1, "failed; this shard's own work finished and was discarded")
    return res


def shard_bounds(batch: int, world: int, rank: int) -> tuple[int, int]:
    """[lo, hi) of `rank`'s contiguous slice of `batch` items over `world` ranks;
    the first batch % world ranks take one item more."""
    if world < 1 or not 0 <= rank < world or batch < 0:
        raise ValueError(f"bad shard request: batch={batch} world={world} rank={rank}")
    base, extra = divmod(batch, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def split_batch(inputs: dict, parts: int) -> list[dict]:
    """Split every input Tensor along its leading (batch) dimension into
    `parts` equal slices (the per-device graph has a fixed batch)."""
    out = [dict() for _ in range(parts)]
    for name, t in inputs.items():
        n = t.shape[0]
        if n % parts:
            raise ValueError(f"input {name}: batch {n} does not split into {parts} equal shards")
        step = n // parts
        for k in range(parts):
            out[k][name] = I.Tensor(name, [step] + list(t.shape[1:]), t.dtype,
                                    np.ascontiguousarray(t.data[k * step:(k + 1) * step]))
    return out


def batch_axis(shape, per_shard: int) -> int:
    """The axis of an output that carries the batch: the first whose extent is the
    per-shard batch (a flattened classifier output [1, batch, classes] carries it
    on axis 1). Pass explicit axes where that rule is ambiguous."""
    for ax, n in enumerate(shape):
        if n == per_shard:
            return ax
    raise ValueError(f"no axis of {list(shape)} has the per-shard batch {per_shard}")


def concat_batch(parts: list[dict], axes: dict | None = None) -> dict:
    """Concatenate per-shard output Tensors along each one's batch axis
    (`axes[name]`, default 0)."""
    out = {}
    for name in parts[0]:
        ts = [p[name] for p in parts]
        ax = (axes or {}).get(name, 0)
        data = np.concatenate([np.asarray(t.data) for t in ts], axis=ax)
        out[name] = I.Tensor(name, list(data.shape), ts[0].dtype, data)
    return out


class ShardedInterpreter:
    """Data-parallel replicas of one graph on several GPUs of one process.

    `data` is a graph whose batch is the per-device batch; ``run`` takes inputs
    with len(devices) times that batch, runs shard k on devices[k] and returns
    the outputs concatenated in shard order along each output's batch axis
    (``batch_axes`` {name: axis}, else ``batch_axis``'s rule).

    Each device has its own host thread (which creates and alone uses that
    device's context and Interpreter) and its own stream, so the shards run
    concurrently: a graph run blocks its thread until its device finishes."""

    def __init__(self, data: bytes, devices, batch_axes: dict | None = None, **kw):
        from concurrent.futures import ThreadPoolExecutor

        self.devices = list(devices)
        if not self.devices:
            raise ValueError("no devices")
        self._pools = [ThreadPoolExecutor(max_workers=1) for _ in self.devices]

        def make(dev):
            import torch

            it = I.Interpreter(data, device=dev, **kw)
            with torch.cuda.device(dev):
                st = torch.cuda.Stream(device=dev)
            return it, st

        made = [pool.submit(make, d) for pool, d in zip(self._pools, self.devices)]
        self._its, self._streams = zip(*[f.result() for f in made])
        self._per = {name: shape[0] for name, _, shape in self._its[0].inputs() if shape}
        per = next(iter(self._per.values()), 1)
        self._axes = {name: (batch_axes or {}).get(name, batch_axis(shape, per) if shape else 0)
                      for name, _, shape in self._its[0].outputs()}

    def close(self):
        for pool, it in zip(self._pools, self._its):
            pool.submit(it.close).result()
            pool.shutdown()
        self._its, self._pools = (), []

    def run(self, inputs: dict) -> dict:
        for name, t in inputs.items():
            want = self._per.get(name)
            if want is not None and t.shape[0] != want * len(self.devices):
                raise ValueError(f"input {name}: batch {t.shape[0]}, expected {want} x {len(self.devices)} devices")
        shards = split_batch(inputs, len(self.devices))

        fail = injected_shards()

        def work(k, it, st, shard):
            if k in fail:
                raise InjectedFault(f"TB_FAULT_SHARD: shard {k} fails before its run")
            it.bind(shard, stream=st)
            it.execute(stream=st)
            return {name: it.output(name) for name, _, _ in it.outputs()}

        futs = [pool.submit(work, k, it, st, sh)
                for k, (pool, it, st, sh) in enumerate(zip(self._pools, self._its, self._streams, shards))]
        # every shard drains before a failure is reported: no device is left running a shard
        results, errors = [], []
        for k, f in enumerate(futs):
            try:
                results.append(f.result())
            except Exception as e:
                errors.append((k, e))
        if errors:
            k, e = errors[0]
            raise ShardError(k, str(e)) from e
        return concat_batch(results, self._axes)


def run_graph_sharded(data: bytes, inputs: dict, devices, **kw) -> dict:
    """run_graph over several GPUs: the inputs' batch is split evenly across `devices`."""
    si = ShardedInterpreter(data, devices, **kw)
    try:
        return si.run(inputs)
    finally:
        si.close()


def max_over_ranks(value: float) -> float:
    """The maximum of `value` over the ranks of the default process group (the
    value itself without one): wall-clock of a data-parallel step is the
    slowest rank's."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_to_rank0(outputs: dict, axes: dict | None = None):
    """Gather every rank's host output Tensors to rank 0 (concatenated in rank
    order along `axes`, as concat_batch); other ranks get None. Host-side
    (object) gather: the data path itself never crosses devices."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return outputs
    got = [None] * dist.get_world_size() if dist.get_rank() == 0 else None
    dist.gather_object(outputs, got, dst=0)
    return concat_batch(got, axes) if dist.get_rank() == 0 else None
