"""CPU-only checks of the data-parallel row with `gloo` ranks (world size 2): the batch slicing
follows the reference DataParallel (om.engine.distributed.ixx:80-110) and the summed-then-scaled
all-reduce that DataParallel.synchronize_gradients/step perform gives every rank the mean of
the per-rank gradients. The per-rank gradients come from the CPU oracle's training step, which
stands in for the device here."""
import os
import socket

import numpy as np
import pytest


def test_local_slice_matches_reference_chunking():
    from omnimatchdeeplearningtool_b200.distributed import local_slice
    assert [local_slice(10, 3, r) for r in range(3)] == [(0, 4), (4, 7), (7, 10)]
    assert [local_slice(8, 2, r) for r in range(2)] == [(0, 4), (4, 8)]
    assert local_slice(5, 1, 0) == (0, 5)
    with pytest.raises(ValueError):
        local_slice(4, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


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
    import torch
    import torch.distributed as dist
    from omnimatchdeeplearningtool_b200.distributed import DataParallel, DistributedConfig
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    flat = torch.from_numpy(_rank_grads(rank, world))

    class _Net:  # the step's scale is what DataParallel.step passes to the net
        def step(self, lr, momentum, grad_scale):
            flat.mul_(grad_scale)

    dp = DataParallel(_Net(), DistributedConfig(world, rank))
    dp.synchronize_gradients(flat)
    dp.step()
    np.save(os.path.join(out_dir, f"rank{rank}.npy"), flat.numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_allreduce_gives_every_rank_the_mean_gradient(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn")
    per_rank = [_rank_grads(r, world) for r in range(world)]
    mean = np.mean(per_rank, axis=0)
    for r in range(world):
        got = np.load(tmp_path / f"rank{r}.npy")
        assert np.allclose(got, mean, rtol=1e-6, atol=1e-7)
