"""Ulysses sequence parallelism on CPU gloo ranks: the all-to-all re-shards are exact inverses, and
attention of a sequence-sharded prompt equals single-process causal attention (GQA, windows)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist

    from fak_b200.models.reference import attention
    from fak_b200.parallel.ulysses import head_to_seq, seq_to_head, ulysses_attention
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        g = torch.Generator().manual_seed(0)
        T, H, Hk, D = 12 * world, 8, 4, 16
        Q, K, V = (torch.randn(T, n, D, generator=g) for n in (H, Hk, Hk))
        sl = slice(rank * T // world, (rank + 1) * T // world)
        # the re-shard round trip is the identity, and seq_to_head gathers the whole sequence
        hs = seq_to_head(Q[sl], None)
        ok_shape = hs.shape == (T, H // world, D)
        ok_heads = torch.equal(hs, Q[:, rank * H // world:(rank + 1) * H // world])
        ok_back = torch.equal(head_to_seq(hs, None), Q[sl])
        errs = []
        for window in (0, 5):
            got = ulysses_attention(Q[sl], K[sl], V[sl], None, window=window)
            want = attention(Q, K, V, 0, window)[sl]
            errs.append(float((got - want).abs().max()))
        q.put((rank, ok_shape, ok_heads, ok_back, errs))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_ulysses_matches_single_process_attention(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    for rank, ok_shape, ok_heads, ok_back, errs in res:
        assert ok_shape and ok_heads and ok_back, rank
        assert max(errs) < 1e-5, (rank, errs)
