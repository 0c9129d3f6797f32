"""GPU tests of the column-sharded linear (sdq_quantized_matmul_sharded over NCCL).

Each rank holds the rows [rank * n_local, (rank + 1) * n_local) of the packed weight; the
library runs the single-GPU kernel on them, all-gathers the [m, n_local] results and
permutes [world, m, n_local] into [m, n].  Quantisation is row-local, so a row shard of
the packed words, scales and biases of the full weight is exactly the quantisation of the
weight's row shard, and for M > 8 (the tensor-core kernel, whose per-element sum does not
depend on N) the sharded output equals the unsharded one bit for bit.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch

import sdq
from conftest import gpu_available

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not gpu_available(), reason="needs an sm_100 device")]


def _weights(n, k, bits, device, seed=7):
    g = torch.Generator(device).manual_seed(seed)
    w = torch.randn(n, k, device=device, generator=g) * 0.02
    return sdq.quantize(w, 64, bits)


def _x(m, k, device, seed=8):
    g = torch.Generator(device).manual_seed(seed)
    return torch.randn(m, k, device=device, generator=g).to(torch.bfloat16)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("m,n", [(64, 256), (300, 1000), (40, 200), (17, 36)])
def test_single_rank_sharded_call_equals_the_unsharded_one(bits, m, n):
    """World size 1: the all-gather is the identity and the permute copies y_shards into y
    (the 16-byte path when n % 8 == 0, the element path otherwise)."""
    k = 256
    wq, s, b = _weights(n, k, bits, "cuda")
    x = _x(m, k, "cuda")
    bias = (torch.randn(n, device="cuda") * 0.5).to(torch.bfloat16)
    want = sdq.quantized_matmul(x, wq, s, b, 64, bits, bias=bias)
    comm = sdq.Comm(sdq.Comm.unique_id(), 1, 0)
    try:
        out, shards = sdq.quantized_matmul_sharded(x, wq, s, b, comm, 64, bits, bias=bias)
        blocked, shards2 = sdq.quantized_matmul_sharded(x, wq, s, b, comm, 64, bits, bias=bias,
                                                         permute=False)
        sdq.device_status()
    finally:
        comm.destroy()
    assert torch.equal(out.view(torch.int16), want.view(torch.int16))
    assert blocked is None
    assert torch.equal(shards2[0].view(torch.int16), want.view(torch.int16))


def _free_port() -> int:
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _rank_main(rank, world, port, m, k, n, bits, q, into_comm_output=False, ms=None):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        uid = [sdq.Comm.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = sdq.Comm(uid[0], world, rank)
        try:
            wq, s, b = _weights(n, k, bits, "cuda")             # the full weight, on every rank
            lo, hi = sdq.shard_rows(n, world, rank)
            same, rel = True, 0.0
            for mi in (ms or [m]):      # several sizes: the exchange buffer grows between them
                x = _x(mi, k, "cuda")
                full = sdq.quantized_matmul(x, wq, s, b, 64, bits)
                args = (x, wq[lo:hi].contiguous(), s[lo:hi].contiguous(), b[lo:hi].contiguous(), comm, 64, bits)
                target = comm.output(mi, n) if into_comm_output else None
                for call in range(2):       # the second call reuses the exchange state
                    out, _ = sdq.quantized_matmul_sharded(*args, out=target)
                    torch.cuda.synchronize()
                    sdq.device_status()
                    same = same and torch.equal(out.view(torch.int16), full.view(torch.int16))
                    rel = max(rel, float((out.float() - full.float()).abs().max() / full.float().abs().max()))
                    if target is not None:
                        assert out.data_ptr() == target.data_ptr()
            q.put((rank, same, rel))
        finally:
            comm.destroy()
            dist.destroy_process_group()
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, None, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("into_comm_output", [False, True], ids=["caller_y", "comm_output"])
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("m", [4, 256, 1000])
def test_two_gpu_sharded_linear_reassembles_the_full_product(bits, m, into_comm_output):
    """m = 4: the plain path (kernel, ncclAllGather, permute); m = 256 / 1000: the overlapped
    path, its result assembled in the communicator's output and copied to the caller's y, or
    left in place when y is that output."""
    import torch.multiprocessing as mp
    world, k, n = 2, 512, 1024
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, m, k, n, bits, q, into_comm_output))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, same, rel in sorted(results):
        assert same is not None, f"rank {rank}: {rel}"
        if m > 8:
            assert same, f"rank {rank}: sharded product differs (max-abs-rel {rel:.3e})"
        else:
            # M <= 8 runs the weight-stream kernel, whose k-split follows N: tolerance only
            assert rel <= 1e-2, f"rank {rank}: max-abs-rel {rel:.3e}"


def _run_ranks(world, *args, **kw):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, *args, q), kwargs=kw) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return sorted(results)


@pytest.mark.parametrize("world", [4, 8])
@pytest.mark.parametrize("bits", [4, 8])
def test_sharded_linear_with_several_peers(world, bits):
    """Four and eight ranks: each kernel stores its tiles into three / seven peers' outputs
    and every rank's assembled output equals the unsharded product bit for bit, over
    several sizes (the exchange buffer grows between them, and shrinks back into use)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    k, n = 512, 256 * world
    for rank, same, rel in _run_ranks(world, 300, k, n, bits, ms=[300, 1000, 17, 300]):
        assert same is not None, f"rank {rank}: {rel}"
        assert same, f"rank {rank}: sharded product differs (max-abs-rel {rel:.3e})"


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_exchange_buffer_grows_between_sizes():
    for rank, same, rel in _run_ranks(2, 64, 512, 1024, 4, into_comm_output=True, ms=[64, 2048, 100]):
        assert same is not None, f"rank {rank}: {rel}"
        assert same, f"rank {rank}: sharded product differs (max-abs-rel {rel:.3e})"


def _static_rank_main(rank, world, port, m, k, n, bits, q):
    """Both ranks call the no-allocation entry point twice; each result must equal what the
    caller-buffer entry point gives for the same shard, bit for bit."""
    import ctypes
    import datetime
    import torch.distributed as dist
    from sdq import _abi
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        uid = [sdq.Comm.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = sdq.Comm(uid[0], world, rank)
        try:
            wq, s, b = _weights(n, k, bits, "cuda")
            lo, hi = sdq.shard_rows(n, world, rank)
            wl, sl, bl = wq[lo:hi].contiguous(), s[lo:hi].contiguous(), b[lo:hi].contiguous()
            same = True
            for call in range(2):       # the second call finds the first call's contents in the array
                x = _x(m, k, "cuda", seed=8 + call)
                want, _ = sdq.quantized_matmul_sharded(x, wl, sl, bl, comm, 64, bits)
                y = torch.full((m, n), float("nan"), device="cuda", dtype=torch.bfloat16)
                _abi.check(_abi.lib().sdq_quantized_matmul_sharded_static(
                    ctypes.c_void_p(x.data_ptr()), _abi.SDQ_BF16, m, k, ctypes.c_void_p(wl.data_ptr()),
                    ctypes.c_void_p(sl.data_ptr()), ctypes.c_void_p(bl.data_ptr()), _abi.SDQ_BF16, hi - lo,
                    64, bits, None, ctypes.c_void_p(y.data_ptr()), _abi.SDQ_BF16, comm.handle,
                    ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
                torch.cuda.synchronize()
                sdq.device_status()
                same = same and torch.equal(y.view(torch.int16), want.view(torch.int16))
            q.put((rank, same, 0.0))
        finally:
            comm.destroy()
            dist.destroy_process_group()
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, None, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("m", [4, 300])
def test_two_gpu_static_scratch_entry_point(bits, m):
    """The no-allocation sharded entry point on two ranks: NCCL all-gathers the peers' blocks
    into each rank's static array and the permute reads them back out of it."""
    import torch.multiprocessing as mp
    world, k, n = 2, 512, 1024
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_static_rank_main, args=(r, world, port, m, k, n, bits, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, same, err in sorted(results):
        assert same is not None, f"rank {rank}: {err}"
        assert same, f"rank {rank}: static-scratch result differs from the caller-buffer one"
