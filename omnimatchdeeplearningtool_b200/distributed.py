"""Data parallelism for the training step: the working version of the reference's DataParallel
(om.engine.distributed.ixx:49-188), whose gradient all-reduce is a no-op (:132-161).

One process per GPU. Each rank takes its slice of the global batch (the reference's slicing,
distributed.ixx:80-110: chunk = B // world, the first B % world ranks take one more), runs the
forward/backward on its own GPU, and the gradients are summed across ranks over NCCL through the
backend's C ABI (omNcclInit / omCudaAllreduceAsync / omCudaAllreduceJoin / omNcclPoll); the
SGD step applies them scaled by 1/world inside the update (omCudaSgdStepScaled), so every rank
applies the mean gradient. BatchNorm statistics stay per rank (the reference's bSyncBatchNorm
flag, distributed.ixx:35, is not implemented there either).

Overlap. The flat gradient is cut into buckets of about `bucket_bytes`, contiguous ranges of the
flat buffer taken from its end, because the backward pass finishes the gradients of the last
layers first. The net reports each parameter whose gradient kernels have all been issued; when
a bucket's last parameter is reported, its all-reduce is enqueued on the communication stream
behind the compute work issued so far, and runs while the rest of the backward pass computes.
The optimiser step waits for all of them on the device.

Failures. Rank 0's communicator id reaches the other ranks through a small TCP exchange
(:class:`Rendezvous`; no PyTorch is involved), bounded by a time limit. A rank that never
joins, an NCCL error, or a collective that does not finish within the poll's time limit aborts
the communicator and raises :class:`CommError` on the host, so no rank waits for good on a peer.
"""
from __future__ import annotations

import ctypes
import os
import socket
import time
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

NCCL_ID_BYTES = 128  # OM_NCCL_ID_BYTES
REDUCE_SUM, REDUCE_MAX = 0, 1


class CommError(RuntimeError):
    """A collective, the communicator's set-up or the id exchange failed or ran out of time."""


@dataclass
class DistributedConfig:
    """distributed.ixx:26-30"""
    nWorldSize: int = 1
    nLocalRank: int = 0
    bSyncBatchNorm: bool = False


def local_slice(batch: int, world: int, rank: int) -> Tuple[int, int]:
    """[start, end) of this rank's samples (distributed.ixx:80-110)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank out of range")
    chunk, rem = divmod(batch, world)
    start = sum(chunk + (1 if r < rem else 0) for r in range(rank))
    return start, start + chunk + (1 if rank < rem else 0)


# ---------------------------------------------------------------------------- id exchange
def _recv_exact(conn: socket.socket, n: int) -> bytes:
    buf = b""
    while len(buf) < n:
        part = conn.recv(n - len(buf))
        if not part:
            raise CommError("rendezvous: peer closed the connection")
        buf += part
    return buf


class Rendezvous:
    """Hands rank 0's payload (the communicator id) to every other rank over TCP.

    Rank 0 listens on (addr, port) and sends the payload to each of the world - 1 ranks that
    connect; the others connect (retrying while rank 0 starts up) and read it. Every wait is
    bounded by `timeout_s`; running out raises CommError."""

    def __init__(self, addr: str, port: int, rank: int, world: int, timeout_s: float = 60.0):
        if world < 1 or not 0 <= rank < world:
            raise ValueError("Rendezvous: bad rank or world size")
        self.addr, self.port, self.rank, self.world = addr, int(port), rank, world
        self.timeout_s = timeout_s

    @classmethod
    def from_env(cls, rank: int, world: int, timeout_s: float = 60.0) -> "Rendezvous":
        """MASTER_ADDR and OM_DP_PORT (default: MASTER_PORT + 1, next to the launcher's own
        store), as torchrun exports them."""
        addr = os.environ.get("MASTER_ADDR", "127.0.0.1")
        port = os.environ.get("OM_DP_PORT")
        if port is None:
            port = int(os.environ.get("MASTER_PORT", "29500")) + 1
        return cls(addr, int(port), rank, world, timeout_s)

    def share(self, payload: Optional[bytes], size: int = NCCL_ID_BYTES) -> bytes:
        if self.world == 1:
            return payload
        deadline = time.monotonic() + self.timeout_s
        if self.rank == 0:
            if payload is None or len(payload) != size:
                raise ValueError("Rendezvous: rank 0 must provide the payload")
            srv = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
            srv.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
            try:
                srv.bind((self.addr, self.port))
                srv.listen(self.world)
                served = 0
                while served < self.world - 1:
                    left = deadline - time.monotonic()
                    if left <= 0:
                        raise CommError(f"rendezvous: {self.world - 1 - served} rank(s) never "
                                        f"connected within {self.timeout_s:.0f} s")
                    srv.settimeout(left)
                    try:
                        conn, _ = srv.accept()
                    except socket.timeout:
                        continue
                    with conn:
                        conn.sendall(payload)
                    served += 1
            finally:
                srv.close()
            return payload
        while True:
            try:
                with socket.create_connection((self.addr, self.port), timeout=2.0) as conn:
                    conn.settimeout(max(0.1, deadline - time.monotonic()))
                    return _recv_exact(conn, size)
            except OSError as e:  # refused while rank 0 starts, or timed out
                if time.monotonic() >= deadline:
                    raise CommError(f"rendezvous: rank 0 not reachable at {self.addr}:"
                                    f"{self.port} within {self.timeout_s:.0f} s") from e
                time.sleep(0.05)


# ---------------------------------------------------------------------------- communicator
class NcclCommunicator:
    """The calling thread's device joins an NCCL communicator through the backend's C ABI."""

    def __init__(self, rank: int, world: int, rendezvous: Optional[Rendezvous] = None,
                 timeout_ms: int = 60000, lib=None):
        from . import _lib
        self._lib = lib if lib is not None else _lib.lib
        self.rank, self.world, self.timeout_ms = rank, world, timeout_ms
        self.closed = False
        rv = rendezvous or Rendezvous.from_env(rank, world, timeout_ms / 1e3)
        uid = ctypes.create_string_buffer(NCCL_ID_BYTES)
        if rank == 0:
            self._check(self._lib.omNcclGetUniqueId(uid), "omNcclGetUniqueId")
            payload = uid.raw
        else:
            payload = None
        got = rv.share(payload)
        uid = ctypes.create_string_buffer(got, NCCL_ID_BYTES)
        self._check(self._lib.omNcclInit(rank, world, uid, int(timeout_ms)), "omNcclInit")

    def _check(self, st: int, what: str) -> None:
        if st == -9:  # OM_ERR_COMM: the communicator has been aborted
            self.closed = True
            raise CommError(f"{what}: collective failed or timed out; communicator aborted")
        if st != 0:
            raise CommError(f"{what} failed with status {st}")

    def allreduce_async(self, ptr: int, count: int, op: int = REDUCE_SUM) -> None:
        self._check(self._lib.omCudaAllreduceAsync(ptr, count, op), "omCudaAllreduceAsync")

    def join(self) -> None:
        self._check(self._lib.omCudaAllreduceJoin(), "omCudaAllreduceJoin")

    def allreduce(self, ptr: int, count: int, op: int = REDUCE_SUM) -> None:
        self._check(self._lib.omCudaAllreduce(ptr, count, op), "omCudaAllreduce")

    def poll(self, timeout_ms: Optional[int] = None) -> None:
        """Wait on the host until the issued all-reduces finish; CommError (after an abort) on
        an NCCL error or when they do not finish within the limit."""
        self._check(self._lib.omNcclPoll(int(timeout_ms or self.timeout_ms)), "omNcclPoll")

    def abort(self) -> None:
        self._lib.omNcclAbort()
        self.closed = True

    def close(self) -> None:
        if not self.closed:
            st = self._lib.omNcclDestroy()
            self.closed = True
            if st != 0:
                raise CommError(f"omNcclDestroy failed with status {st}")


# ---------------------------------------------------------------------------- buckets
@dataclass
class Bucket:
    names: List[str]
    start: int   # first element of the bucket's range of the flat gradient
    count: int   # elements


def gradient_buckets(offsets: Dict[str, Tuple[int, int, tuple]], bucket_bytes: int) -> List[Bucket]:
    """Contiguous ranges of the flat gradient, from its end to its start, of at least
    `bucket_bytes` each (the last one takes what is left). offsets: name -> (offset, count, shape)
    in elements. Parameters are never split."""
    order = sorted(offsets.items(), key=lambda kv: kv[1][0], reverse=True)
    buckets: List[Bucket] = []
    cur: List[str] = []
    lo = hi = None
    for name, (off, n, _) in order:
        cur.append(name)
        hi = off + n if hi is None else hi
        lo = off
        if (hi - lo) * 4 >= bucket_bytes:
            buckets.append(Bucket(cur, lo, hi - lo))
            cur, hi = [], None
    if cur:
        buckets.append(Bucket(cur, lo, hi - lo))
    return buckets


class DataParallel:
    """Wraps a per-rank training net (plan.Fp32Net) and a communicator.

    Per step: ``begin_step()``, the net's forward/backward (its gradient hook starts bucket
    all-reduces), then ``step(lr, momentum)``, which makes the update wait for every bucket and
    applies the mean gradient. ``check()`` watches the collectives from the host."""

    def __init__(self, net, config: DistributedConfig, comm=None, bucket_bytes: int = 25 << 20):
        if config.nWorldSize < 1 or not 0 <= config.nLocalRank < config.nWorldSize:
            raise ValueError("DataParallel: bad world size or rank")
        if config.nWorldSize > 1 and comm is None:
            raise ValueError("DataParallel: a communicator is needed for more than one rank")
        self.net = net
        self.config = config
        self.comm = comm
        self.buckets = gradient_buckets(net.offsets, bucket_bytes)
        self._bucket_of = {n: i for i, b in enumerate(self.buckets) for n in b.names}
        self._left: List[int] = []
        self._fired: List[bool] = []
        self.begin_step()
        if config.nWorldSize > 1:
            net.grad_hook = self._grad_ready

    def begin_step(self) -> None:
        self._left = [len(b.names) for b in self.buckets]
        self._fired = [False] * len(self.buckets)

    def _fire(self, i: int) -> None:
        b = self.buckets[i]
        self._fired[i] = True
        self.comm.allreduce_async(self.net.grad_flat + b.start * 4, b.count, REDUCE_SUM)

    def _grad_ready(self, name: str) -> None:
        i = self._bucket_of.get(name)
        if i is None or self._fired[i]:
            return
        self._left[i] -= 1
        if self._left[i] == 0:
            self._fire(i)

    def synchronize_gradients(self) -> None:
        """Sum the flat gradient across ranks: start the buckets the backward pass has not
        completed (parameters without a gradient this step), then make later compute work wait
        for all of them."""
        if self.config.nWorldSize <= 1:
            return
        for i, fired in enumerate(self._fired):
            if not fired:
                self._fire(i)
        self.comm.join()

    def step(self, lr: float = 0.01, momentum: float = 0.9) -> None:
        self.synchronize_gradients()
        self.net.step(lr, momentum, grad_scale=1.0 / self.config.nWorldSize)
        self.begin_step()

    def check(self, timeout_ms: Optional[int] = None) -> None:
        """Host-side watch of this step's collectives (raises CommError after an abort)."""
        if self.comm is not None:
            self.comm.poll(timeout_ms)

    def is_master_rank(self) -> bool:
        return self.config.nLocalRank == 0
