"""Host logic of the column-sharded linear on CPU ranks (gloo, world size 2): each rank
quantises and multiplies its own row shard with the CPU oracle, the shards are
all-gathered, and the library's [world, m, n_local] -> [m, n] index map (sdq.unshard)
reassembles exactly the unsharded product.  Also covers the shard plan's error path."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
import sdq


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, m, k, n, bits, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        xb, w = O.synthetic_linear(21, m, k, n, 0.02)
        lo, hi = sdq.shard_rows(n, world, rank)
        wq, s, b = O.quantize(np.ascontiguousarray(w[lo:hi]), bits)
        y_local = torch.from_numpy(O.qmatmul(xb, wq, s, b, hi - lo, bits))
        gathered = [torch.empty_like(y_local) for _ in range(world)]
        dist.all_gather(gathered, y_local)
        y = sdq.unshard(torch.stack(gathered)).numpy()
        np.save(os.path.join(out_dir, f"y{rank}.npy"), y)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("bits", [4, 8])
def test_two_rank_shard_gather_reassembles_the_full_product(tmp_path, bits):
    m, k, n, world = 24, 256, 96, 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, m, k, n, bits, str(tmp_path)))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    xb, w = O.synthetic_linear(21, m, k, n, 0.02)
    full = O.qmatmul(xb, *O.quantize(w, bits), n, bits)
    for r in range(world):
        y = np.load(tmp_path / f"y{r}.npy")
        # per-group quantisation is row-local, so sharding rows changes no bit
        assert (y == full).all()


def test_shard_plan():
    assert sdq.shard_rows(12288, 8, 3) == (4608, 6144)
    with pytest.raises(sdq.SdqError):
        sdq.shard_rows(100, 8, 0)
    ys = np.arange(2 * 3 * 4).reshape(2, 3, 4)
    u = sdq.unshard(ys)
    assert u.shape == (3, 8) and u[1, 5] == ys[1, 1, 1]
