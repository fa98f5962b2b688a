"""CPU-only checks of the data-parallel layer (omnimatchdeeplearningtool_b200.distributed):

  * the batch slicing follows the reference DataParallel (om.engine.distributed.ixx:80-110);
  * the gradient buckets cover the flat gradient exactly once, from its end;
  * the rendezvous hands rank 0's communicator id to every rank, and gives up with CommError
    when a rank never shows up (failure made on the host: a missing rank);
  * DataParallel starts each bucket's all-reduce when the backward pass reports its last
    parameter, starts the rest and joins before the update, and scales the update by 1/world;
  * with `gloo` ranks (world size 2) carrying the bucket all-reduces, every rank ends with the
    mean of the per-rank gradients (the oracle's training step stands in for the device);
  * an NCCL failure reported by the C ABI (a fake library returning OM_ERR_COMM: an error code
    injected on the host) surfaces as CommError and leaves the communicator closed.
"""
import os
import socket
import threading

import numpy as np
import pytest


def test_local_slice_matches_reference_chunking():
    from omnimatchdeeplearningtool_b200.distributed import local_slice
    assert [local_slice(10, 3, r) for r in range(3)] == [(0, 4), (4, 7), (7, 10)]
    assert [local_slice(8, 2, r) for r in range(2)] == [(0, 4), (4, 8)]
    assert local_slice(5, 1, 0) == (0, 5)
    with pytest.raises(ValueError):
        local_slice(4, 2, 2)


def _offsets(net):
    off, out = 0, {}
    for name, shape in net.params:
        n = int(np.prod(shape))
        out[name] = (off, n, shape)
        off += n
    return out, off


@pytest.mark.parametrize("bucket_mb", [1, 8, 25, 1000])
def test_gradient_buckets_cover_the_flat_gradient(bucket_mb):
    from omnimatchdeeplearningtool_b200 import synth
    from omnimatchdeeplearningtool_b200.distributed import gradient_buckets
    offsets, total = _offsets(synth.resnet_spec(18, 1000))
    buckets = gradient_buckets(offsets, bucket_mb << 20)
    seen = np.zeros(total, np.int32)
    end = total
    for i, b in enumerate(buckets):
        assert b.start + b.count == end            # contiguous, walking from the end
        end = b.start
        seen[b.start:b.start + b.count] += 1
        for n in b.names:
            off, cnt, _ = offsets[n]
            assert b.start <= off and off + cnt <= b.start + b.count
        if i < len(buckets) - 1:
            assert b.count * 4 >= bucket_mb << 20
    assert end == 0 and (seen == 1).all()
    assert sorted(n for b in buckets for n in b.names) == sorted(offsets)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_rendezvous_shares_rank0_payload():
    from omnimatchdeeplearningtool_b200.distributed import Rendezvous
    port, world = _free_port(), 4
    payload = bytes(range(128))
    got = [None] * world

    def run(r):
        got[r] = Rendezvous("127.0.0.1", port, r, world, timeout_s=20).share(
            payload if r == 0 else None)

    ts = [threading.Thread(target=run, args=(r,)) for r in range(world)]
    for t in ts[::-1]:  # the other ranks start first and retry until rank 0 listens
        t.start()
    for t in ts:
        t.join(30)
    assert got == [payload] * world


def test_rendezvous_missing_rank_times_out():
    from omnimatchdeeplearningtool_b200.distributed import CommError, Rendezvous
    port = _free_port()
    with pytest.raises(CommError):  # rank 0 never starts
        Rendezvous("127.0.0.1", port, 1, 2, timeout_s=0.5).share(None)
    with pytest.raises(CommError):  # rank 1 never connects
        Rendezvous("127.0.0.1", port, 0, 2, timeout_s=0.5).share(bytes(128))


class _FakeNet:
    """The part of plan.Fp32Net that DataParallel uses: offsets, the flat gradient pointer,
    the gradient hook and step(). Gradients live in host memory."""

    def __init__(self, net, grads):
        self.offsets, self.n_params = _offsets(net)
        self.flat = np.ascontiguousarray(grads, np.float32)
        self.grad_flat = self.flat.ctypes.data
        self.grad_hook = None
        self.steps = []

    def backward(self, order):
        for n in order:
            if self.grad_hook:
                self.grad_hook(n)

    def step(self, lr, momentum, grad_scale=1.0):
        self.steps.append(grad_scale)


class _RecordingComm:
    def __init__(self):
        self.calls = []

    def allreduce_async(self, ptr, count, op=0):
        self.calls.append(("ar", ptr, count))

    def join(self):
        self.calls.append(("join",))

    def poll(self, timeout_ms=None):
        self.calls.append(("poll",))


def test_data_parallel_starts_buckets_as_the_backward_completes_them():
    from omnimatchdeeplearningtool_b200 import synth
    from omnimatchdeeplearningtool_b200.distributed import DataParallel, DistributedConfig
    net = synth.resnet_spec(18, 1000)
    fake = _FakeNet(net, np.zeros(sum(int(np.prod(s)) for _, s in net.params)))
    comm = _RecordingComm()
    dp = DataParallel(fake, DistributedConfig(2, 1), comm, bucket_bytes=8 << 20)
    assert len(dp.buckets) >= 3
    names = [n for n, _ in net.params]
    # the backward reports the last parameters first; stop before the first bucket completes
    first = dp.buckets[0]
    order = [n for n in reversed(names) if n in first.names]
    fake.backward(order[:-1])
    assert comm.calls == []
    fake.backward(order[-1:])
    assert comm.calls == [("ar", fake.grad_flat + first.start * 4, first.count)]
    # the remaining buckets start at the synchronisation, then the update waits for them all
    dp.step(0.01, 0.9)
    ar = [c for c in comm.calls if c[0] == "ar"]
    assert sorted((c[1] - fake.grad_flat) // 4 for c in ar) == sorted(b.start for b in dp.buckets)
    assert comm.calls[-1] == ("join",)
    assert fake.steps == [0.5]
    # a full backward in order fires every bucket before the step
    comm.calls.clear()
    fake.backward(list(reversed(names)))
    assert len([c for c in comm.calls if c[0] == "ar"]) == len(dp.buckets)
    dp.step()
    assert comm.calls[-1] == ("join",) and len(comm.calls) == len(dp.buckets) + 1


def _rank_grads(rank, world):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    sys.path.insert(0, os.path.join(root, "oracle"))
    import oracle as orc
    from omnimatchdeeplearningtool_b200 import synth
    from omnimatchdeeplearningtool_b200.distributed import local_slice
    net = synth.resnet_spec(18, 10)
    w = synth.make_weights(net)
    x = synth.normal_input(4, 3, 32, 32, seed=21)
    y = synth.onehot_labels(4, 10, seed=22)
    s, e = local_slice(4, world, rank)
    _, grads = orc.train_step(net, w, x[s:e], y[s:e])
    return np.concatenate([grads[n].reshape(-1) for n, _ in net.params]).astype(np.float32)


def _worker(rank, world, port, out_dir):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import torch
    import torch.distributed as dist
    from omnimatchdeeplearningtool_b200 import synth
    from omnimatchdeeplearningtool_b200.distributed import DataParallel, DistributedConfig
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    net = synth.resnet_spec(18, 10)
    fake = _FakeNet(net, _rank_grads(rank, world))

    class _GlooComm:  # the bucket all-reduces over gloo, on the host gradient
        def allreduce_async(self, ptr, count, op=0):
            t = torch.from_numpy(fake.flat[(ptr - fake.grad_flat) // 4:][:count])
            dist.all_reduce(t)

        def join(self):
            pass

    dp = DataParallel(fake, DistributedConfig(world, rank), _GlooComm(), bucket_bytes=1 << 18)
    fake.backward([n for n, _ in reversed(net.params)])
    dp.step()
    np.save(os.path.join(out_dir, f"rank{rank}.npy"), fake.flat * fake.steps[-1])
    dist.barrier()
    dist.destroy_process_group()


def test_bucketed_allreduce_gives_every_rank_the_mean_gradient(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn")
    per_rank = [_rank_grads(r, world) for r in range(world)]
    mean = np.mean(per_rank, axis=0)
    for r in range(world):
        got = np.load(tmp_path / f"rank{r}.npy")
        assert np.allclose(got, mean, rtol=1e-6, atol=1e-7)


class _FakeLib:
    """Stands in for libomcuda.so's NCCL entry points; `fail` names the call that reports
    OM_ERR_COMM (-9)."""

    def __init__(self, fail=None):
        self.fail = fail
        self.aborted = False

    def _ret(self, name):
        return -9 if name == self.fail else 0

    def omNcclGetUniqueId(self, buf):
        return self._ret("omNcclGetUniqueId")

    def omNcclInit(self, rank, world, uid, timeout_ms):
        return self._ret("omNcclInit")

    def omCudaAllreduceAsync(self, ptr, count, op):
        return self._ret("omCudaAllreduceAsync")

    def omCudaAllreduceJoin(self):
        return self._ret("omCudaAllreduceJoin")

    def omCudaAllreduce(self, ptr, count, op):
        return self._ret("omCudaAllreduce")

    def omNcclPoll(self, timeout_ms):
        return self._ret("omNcclPoll")

    def omNcclAbort(self):
        self.aborted = True
        return 0

    def omNcclDestroy(self):
        return 0


@pytest.mark.parametrize("fail", ["omNcclInit", "omCudaAllreduceAsync", "omNcclPoll"])
def test_comm_failure_surfaces_as_comm_error(fail):
    from omnimatchdeeplearningtool_b200.distributed import (CommError, DataParallel,
                                                            DistributedConfig, NcclCommunicator,
                                                            Rendezvous)
    from omnimatchdeeplearningtool_b200 import synth
    lib = _FakeLib(fail)
    rv = Rendezvous("127.0.0.1", _free_port(), 0, 1)
    if fail == "omNcclInit":
        with pytest.raises(CommError):
            NcclCommunicator(0, 1, rv, timeout_ms=100, lib=lib)
        return
    comm = NcclCommunicator(0, 1, rv, timeout_ms=100, lib=lib)
    net = synth.resnet_spec(18, 10)
    fake = _FakeNet(net, np.zeros(_offsets(net)[1]))
    dp = DataParallel(fake, DistributedConfig(2, 0), comm, bucket_bytes=1 << 18)
    with pytest.raises(CommError):
        fake.backward([n for n, _ in reversed(net.params)])
        dp.step()
        dp.check(100)
    assert comm.closed
