"""Data parallelism on two GPUs over NCCL (one process per GPU, torch.distributed plumbing).

Each rank runs the fp32 training step of a small ResNet-18 on its own seeded batch. Checked:
  * the all-reduced flat gradient equals the sum of the ranks' local gradients (gathered
    before the all-reduce), to fp32 summation-order rounding (max|a-b|/max|b| <= 1e-6);
  * after two SGD steps with the mean gradient, every parameter is bit-identical on both ranks
    (the replicas stay in step, as the reference DataParallel intends,
    om.engine.distributed.ixx:132-188).
Skipped when fewer than two GPUs are visible.
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
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch
    import torch.distributed as dist
    from omnimatchdeeplearningtool_b200 import backend, synth
    from omnimatchdeeplearningtool_b200._lib import call
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    from omnimatchdeeplearningtool_b200.distributed import DataParallel, DistributedConfig
    from omnimatchdeeplearningtool_b200.plan import Fp32Net

    backend.init(rank)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device(f"cuda:{rank}"))
    stream = torch.cuda.ExternalStream(backend.stream_handle(), device=rank)
    net = synth.resnet_spec(18, 10)
    w = synth.make_weights(net)
    n_params = sum(int(np.prod(s)) for _, s in net.params)
    grad = torch.zeros(n_params, dtype=torch.float32, device=f"cuda:{rank}")
    fnet = Fp32Net(net, w, 4, 64, 64, grad_ptr=grad.data_ptr())
    dp = DataParallel(fnet, DistributedConfig(world, rank))
    x = DeviceBuffer.from_numpy(synth.normal_input(4, 3, 64, 64, seed=30 + rank))
    y = DeviceBuffer.from_numpy(synth.onehot_labels(4, 10, seed=40 + rank))
    loss = DeviceBuffer.zeros(4)
    try:
        for step in range(2):
            fnet.forward_backward(x.ptr, y.ptr, loss.ptr)
            call("omCudaSynchronize")
            local = grad.detach().clone()
            with torch.cuda.stream(stream):
                dp.synchronize_gradients(grad)
            torch.cuda.synchronize()
            if step == 0:
                parts = [torch.empty_like(local) for _ in range(world)]
                dist.all_gather(parts, local)
                summed = torch.stack(parts).sum(0)
                np.save(os.path.join(out_dir, f"sum_{rank}.npy"), summed.cpu().numpy())
                np.save(os.path.join(out_dir, f"red_{rank}.npy"), grad.cpu().numpy())
            dp.step(0.01, 0.9)
        call("omCudaSynchronize")
        params = np.concatenate([fnet.read_param(n).reshape(-1) for n, _ in net.params])
        np.save(os.path.join(out_dir, f"param_{rank}.npy"), params)
        assert backend.kernel_error() == 0
    finally:
        fnet.close()
        dist.destroy_process_group()


def test_two_gpu_data_parallel_step(tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    for r in range(2):
        summed = np.load(tmp_path / f"sum_{r}.npy")
        red = np.load(tmp_path / f"red_{r}.npy")
        assert np.abs(red - summed).max() <= 1e-6 * np.abs(summed).max()
    assert np.array_equal(np.load(tmp_path / "param_0.npy"), np.load(tmp_path / "param_1.npy"))
