"""Data parallelism on two GPUs over NCCL through the backend's C ABI (one process per GPU; no
PyTorch on the path: the communicator id goes through distributed.Rendezvous, the all-reduces
through omCudaAllreduceAsync / omCudaAllreduceJoin).

Each rank runs the fp32 training step of a small ResNet-18 on its own seeded batch. Checked:
  * the all-reduced flat gradient equals the sum of the ranks' local gradients (read before the
    all-reduce), to fp32 summation-order rounding (max|a-b|/max|b| <= 1e-6);
  * after two SGD steps with the mean gradient (the second with the bucket all-reduces started
    from the backward pass's gradient hook), every parameter is bit-identical on both ranks (the
    replicas stay in step, as the reference DataParallel intends,
    om.engine.distributed.ixx:132-188).
NVLS is off (NCCL_NVLS_ENABLE=0). Skipped when fewer than two GPUs are visible.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out_dir):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from omnimatchdeeplearningtool_b200 import backend, synth
    from omnimatchdeeplearningtool_b200._lib import call
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    from omnimatchdeeplearningtool_b200.distributed import (DataParallel, DistributedConfig,
                                                            NcclCommunicator, Rendezvous)
    from omnimatchdeeplearningtool_b200.plan import Fp32Net

    backend.init(rank)
    comm = NcclCommunicator(rank, world, Rendezvous("127.0.0.1", port, rank, world, 60),
                            timeout_ms=60000)
    net = synth.resnet_spec(18, 10)
    w = synth.make_weights(net)
    fnet = Fp32Net(net, w, 4, 64, 64)
    dp = DataParallel(fnet, DistributedConfig(world, rank), comm, bucket_bytes=4 << 20)
    x = DeviceBuffer.from_numpy(synth.normal_input(4, 3, 64, 64, seed=30 + rank))
    y = DeviceBuffer.from_numpy(synth.onehot_labels(4, 10, seed=40 + rank))
    loss = DeviceBuffer.zeros(4)
    try:
        # step 1: local gradients first (no hook), then the bucket all-reduces and the update
        hook, fnet.grad_hook = fnet.grad_hook, None
        fnet.forward_backward(x.ptr, y.ptr, loss.ptr)
        call("omCudaSynchronize")
        local = np.concatenate([g.reshape(-1) for g in fnet.read_grads().values()])
        np.save(os.path.join(out_dir, f"local_{rank}.npy"), local)
        fnet.grad_hook = hook
        dp.synchronize_gradients()
        dp.check(60000)
        call("omCudaSynchronize")
        red = np.concatenate([g.reshape(-1) for g in fnet.read_grads().values()])
        np.save(os.path.join(out_dir, f"red_{rank}.npy"), red)
        dp.step(0.01, 0.9)
        # step 2: the buckets start from the backward pass itself and overlap it
        fnet.forward_backward(x.ptr, y.ptr, loss.ptr)
        dp.step(0.01, 0.9)
        dp.check(60000)
        call("omCudaSynchronize")
        params = np.concatenate([fnet.read_param(n).reshape(-1) for n, _ in net.params])
        np.save(os.path.join(out_dir, f"param_{rank}.npy"), params)
        assert backend.kernel_error() == 0
    finally:
        comm.close()
        fnet.close()


def test_two_gpu_data_parallel_step(tmp_path):
    from omnimatchdeeplearningtool_b200._lib import lib
    if lib.omCudaGetDeviceCount() < 2:
        pytest.skip("needs two GPUs")
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    summed = np.load(tmp_path / "local_0.npy") + np.load(tmp_path / "local_1.npy")
    for r in range(2):
        red = np.load(tmp_path / f"red_{r}.npy")
        assert np.abs(red - summed).max() <= 1e-6 * np.abs(summed).max()
    assert np.array_equal(np.load(tmp_path / "param_0.npy"), np.load(tmp_path / "param_1.npy"))
