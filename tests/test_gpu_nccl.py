"""The backend's NCCL entry points on one GPU (a one-rank communicator), and the failure path.

  * omCudaAllreduce / omCudaAllreduceAsync + omCudaAllreduceJoin / omNcclPoll on a one-rank
    communicator: the sum and max of one rank are the data itself, exactly, and the ordering
    against the compute stream holds (an all-reduce of data a kernel has just written sees it);
  * a rank that never joins: rank 0 of a two-rank communicator whose second rank never starts
    gets OM_ERR_COMM (CommError) once the set-up time limit passes, instead of waiting for good.
    This runs in a child process (host-side failure; no GPU kernel is involved) with NVLS off.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu


def test_one_rank_allreduce_and_ordering(gpu):
    import socket
    from omnimatchdeeplearningtool_b200._lib import call
    from omnimatchdeeplearningtool_b200.backend import DeviceBuffer
    from omnimatchdeeplearningtool_b200.distributed import (REDUCE_MAX, NcclCommunicator,
                                                            Rendezvous)
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    comm = NcclCommunicator(0, 1, Rendezvous("127.0.0.1", port, 0, 1), timeout_ms=30000)
    try:
        rng = np.random.Generator(np.random.PCG64(5))
        a = rng.standard_normal(1 << 20).astype(np.float32)
        buf = DeviceBuffer.from_numpy(a)
        comm.allreduce(buf.ptr, a.size)
        assert np.array_equal(buf.to_numpy(a.shape), a)
        comm.allreduce(buf.ptr, a.size, REDUCE_MAX)
        assert np.array_equal(buf.to_numpy(a.shape), a)
        # a kernel on the compute stream writes, the async all-reduce must see its result
        call("omCudaMulScalar", buf.ptr, 2.0, buf.ptr, a.size)
        comm.allreduce_async(buf.ptr, a.size)
        comm.join()
        comm.poll(30000)
        assert np.array_equal(buf.to_numpy(a.shape), 2 * a)
    finally:
        comm.close()


_MISSING_PEER = r"""
import os, sys, time
sys.path.insert(0, sys.argv[1])
os.environ["NCCL_NVLS_ENABLE"] = "0"
from omnimatchdeeplearningtool_b200 import backend
from omnimatchdeeplearningtool_b200._lib import lib
import ctypes
backend.init(0)
uid = ctypes.create_string_buffer(128)
assert lib.omNcclGetUniqueId(uid) == 0
t0 = time.time()
st = lib.omNcclInit(0, 2, uid, 3000)   # rank 1 never starts
dt = time.time() - t0
print("status", st, "seconds", round(dt, 2))
sys.exit(0 if st == -9 and dt < 60 else 1)
"""


def test_missing_rank_fails_setup_with_comm_error():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-c", _MISSING_PEER, ROOT], capture_output=True,
                       text=True, timeout=180, env=env)
    assert r.returncode == 0, r.stdout + r.stderr
