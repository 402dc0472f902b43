"""Multi-process host-side paths on CPU (gloo ranks, 127.0.0.1): pipeline parallelism against the
single-process oracle, and failure detection by a short process-group timeout."""
import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

from fak_b200.config import preset


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tiny_ref(path):
    from fak_b200.models.reference import ReferenceModel
    return ReferenceModel.from_gguf(path, "cpu")


@pytest.fixture(scope="module")
def tiny_gguf(tmp_path_factory):
    from fak_b200.gguf.synth import write_synthetic_gguf
    path = str(tmp_path_factory.mktemp("pp") / "tiny.gguf")
    write_synthetic_gguf(path, preset("tiny-llama").replace(n_layers=4), "q8_0", seed=3, std=0.05)
    return path


def _pp_worker(rank, world, port, path, prompt, n_new, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from fak_b200.parallel import dist as pdist
    from fak_b200.parallel.pp import PipelineGreedy, ReferenceStageModel
    torch.manual_seed(0)
    pdist.init(world, rank, 0, timeout_s=60, backend="gloo")
    try:
        pipe = PipelineGreedy(ReferenceStageModel(_tiny_ref(path)), rank, world)
        out = pipe.generate(prompt, n_new)
        q.put((rank, out, pipe.band))
    finally:
        pdist.shutdown()


@pytest.mark.parametrize("world", [2, 3])
def test_pipeline_parallel_greedy_matches_single_process(world, tiny_gguf):
    from fak_b200.parallel.pp import partition_layers
    prompt = [5, 17, 99, 3, 42, 7, 250, 11]
    want = _tiny_ref(tiny_gguf).generate_greedy(prompt, 6)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_pp_worker, args=(r, world, port, tiny_gguf, prompt, 6, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, out, band = q.get(timeout=120)
        res[r] = (out, band)
    for p in procs:
        p.join(timeout=60)
    assert all(res[r][0] == want for r in range(world)), (res, want)
    assert [res[r][1] for r in range(world)] == partition_layers(4, world)


def test_partition_layers():
    from fak_b200.parallel.pp import partition_layers
    assert partition_layers(28, 3) == [(0, 10), (10, 19), (19, 28)]
    assert partition_layers(4, 4) == [(0, 1), (1, 2), (2, 3), (3, 4)]
    with pytest.raises(ValueError):
        partition_layers(2, 3)


def _timeout_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from fak_b200.parallel import dist as pdist
    pdist.init(world, rank, 0, timeout_s=3, backend="gloo")
    if rank == 1:
        q.put((rank, "left"))  # the dead peer: never enters the collective
        time.sleep(8)
        return
    t0 = time.time()
    try:
        dist.all_reduce(torch.ones(4))
        q.put((rank, "no error"))
    except Exception as e:  # the process-group timeout surfaces as an error, not a hang
        q.put((rank, f"error after {time.time() - t0:.1f}s: {type(e).__name__}"))


def test_dead_rank_is_detected_by_the_group_timeout():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_timeout_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    msgs = dict(q.get(timeout=60) for _ in range(2))
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert msgs[1] == "left"
    assert msgs[0].startswith("error after"), msgs


def _handoff_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from fak_b200.engine.disagg import KVHandoff, recv_handoff, send_handoff
    from fak_b200.parallel import dist as pdist
    pdist.init(world, rank, 0, timeout_s=60, backend="gloo")
    try:
        if rank == 0:
            g = torch.Generator().manual_seed(7)
            h = KVHandoff([5, 6, 7, 8], 42, torch.randn(3, 2, 2, 16, 8, generator=g).bfloat16(),
                          torch.randn(3, 2, 2, 16, 8, generator=g).bfloat16(), 16)
            send_handoff(h, 1)
            q.put((0, h.prompt, h.first_token, h.k.float().sum().item(), h.v.float().sum().item()))
        else:
            h = recv_handoff(0, "cpu")
            q.put((1, h.prompt, h.first_token, h.k.float().sum().item(), h.v.float().sum().item()))
    finally:
        pdist.shutdown()


def test_kv_handoff_transport_between_processes():
    """A prefill-side KV handoff crosses processes (gloo point-to-point) intact."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_handoff_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((m[0], m[1:]) for m in (q.get(timeout=120) for _ in range(2)))
    for p in procs:
        p.join(timeout=60)
    assert res[0] == res[1] and res[1][0] == [5, 6, 7, 8] and res[1][1] == 42
