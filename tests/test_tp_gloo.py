"""Host logic of the tensor-parallel path on the CPU: the shard geometry, the argument checks
of sx_model_create_tp that run before any device work, and the IPC-handle exchange across a
gloo world of two processes (each rank receives every rank's handle, in rank order)."""
import ctypes as C
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import syrinx_b200 as sx
from syrinx_b200 import _lib, tp
from syrinx_b200.configs import SX_DTYPE_Q8_0, shrink


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class FakeSession:
    """Stands in for a B200DualAr: a handle that names its rank, and a record of connect()."""

    def __init__(self, rank):
        self.rank = rank
        self.got = None

    def tp_handle(self):
        return bytes([self.rank]) * sx.dualar.TP_HANDLE_BYTES

    def tp_connect(self, handles):
        self.got = handles


def worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        s = FakeSession(rank)
        tp.connect(s, dist)
        q.put((rank, s.got))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_handle_exchange_in_rank_order(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, got in out:
        assert [h[0] for h in got] == list(range(world))
        assert all(len(h) == sx.dualar.TP_HANDLE_BYTES for h in got)


def test_shard_dims_config5():
    d = tp.shard_dims(sx.QWEN3_4B, 8)
    assert d == {"n_head": 4, "n_local_heads": 1, "intermediate_size": 1216, "qkv_rows": 768,
                 "wo_cols": 512, "w2_cols": 1216}
    # the shards tile the full matrices
    for n in (1, 2, 4, 8):
        d = tp.shard_dims(sx.QWEN3_4B, n)
        assert d["qkv_rows"] * n == sx.QWEN3_4B.slow.qkv_rows
        assert d["w2_cols"] * n == sx.QWEN3_4B.slow.intermediate_size
    with pytest.raises(ValueError):
        tp.shard_dims(sx.QWEN3_4B, 3)


def test_model_create_tp_rejects_bad_arguments_before_device():
    L = _lib.lib()
    cfg = shrink(sx.QWEN3_4B, 1, 1)
    desc = cfg.to_c()
    junk = np.zeros(64, np.uint8)
    h = C.c_void_p()
    for rank, size in ((0, 0), (2, 2), (-1, 2), (0, 9)):
        rc = L.sx_model_create_tp(C.byref(desc), junk.ctypes.data, junk.nbytes, 0, rank, size, C.byref(h))
        assert rc == -1 and not h.value, (rank, size, rc)
    # 32 heads do not split over 3 ranks
    rc = L.sx_model_create_tp(C.byref(desc), junk.ctypes.data, junk.nbytes, 0, 0, 3, C.byref(h))
    assert rc == -6 and b"split evenly" in L.sx_last_error()
