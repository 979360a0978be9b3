"""Host-side multi-rank paths on CPU (gloo, world size 2): the bench's shard
pieces and their point-to-point gather into rank 0, and concurrent creation
of one synthetic model file by several processes."""

import importlib.util
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("s3t_bench", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_pieces():
    b = _bench()
    assert b.shard_pieces(64, 1) == [(0, 64)]
    assert b.shard_pieces(32, 2) == [(0, 8), (8, 16), (16, 24), (24, 32)]
    assert b.shard_pieces(16, 4) == [(0, 8), (8, 16)]
    assert b.shard_pieces(8, 8) == [(0, 8)]
    assert b.shard_pieces(1, 8) == [(0, 1)]
    assert b.shard_pieces(20, 2, pieces=4) == [(0, 10), (10, 20)]
    for per in range(1, 40):
        pieces = b.shard_pieces(per, 4)
        assert pieces[0][0] == 0 and pieces[-1][1] == per
        assert all(p[1] == q[0] for p, q in zip(pieces, pieces[1:]))


def _gather_worker(rank, world, port, per, q, pieces):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        b = _bench()
        shape = (per, 3, 5, 7)
        out = torch.arange(np.prod(shape), dtype=torch.float32).reshape(shape) + 1000.0 * rank
        gathered = torch.full((world,) + shape, -1.0) if rank == 0 else None
        reqs = []
        for i0, i1 in b.shard_pieces(per, world, pieces):
            reqs += b.gather_piece_to_rank0(rank, world, out, gathered, i0, i1)
        for r in reqs:
            r.wait()
        if rank == 0:
            gathered[0].copy_(out)
            expect = torch.stack([torch.arange(np.prod(shape), dtype=torch.float32).reshape(shape) + 1000.0 * r
                                  for r in range(world)])
            q.put(bool(torch.equal(gathered, expect)))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("per,pieces", [(5, 1), (16, 2), (32, 4)])
def test_chunked_gather_gloo_world2(per, pieces):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, per, q, pieces)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) is True


def _write_worker(cache, barrier):
    os.environ["S3T_CACHE"] = cache
    sys.path.insert(0, str(ROOT))
    from sam3cpp_b200 import synthetic as syn

    w = syn.make_f32_weights(3, 1, False)
    barrier.wait(timeout=60)
    syn.write_gguf(Path(cache) / "same.gguf", w, "q8_0")


def test_concurrent_synthetic_file_creation(tmp_path):
    """Several ranks creating the same cached model file at once: each writes
    its own partial file and renames it, so every writer succeeds and the
    file left behind is whole."""
    import multiprocessing as mp

    from sam3cpp_b200 import synthetic as syn

    ctx = mp.get_context("spawn")
    barrier = ctx.Barrier(3)
    procs = [ctx.Process(target=_write_worker, args=(str(tmp_path), barrier)) for _ in range(3)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert not list(tmp_path.glob("*.partial"))
    ref = tmp_path / "ref.gguf"
    syn.write_gguf(ref, syn.make_f32_weights(3, 1, False), "q8_0")
    assert (tmp_path / "same.gguf").read_bytes() == ref.read_bytes()
    assert (tmp_path / "same.gguf.tensor_map.json").read_text() == (tmp_path / "ref.gguf.tensor_map.json").read_text()
