"""Tensor-parallel decode/prefill agreement with TP=1 (needs >= 2 GPUs)."""
import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("model", ["tiny-qwen2", "tiny-llama"])
@pytest.mark.parametrize("fused", [1, 0])
def test_tp2_matches_tp1(model, fused):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29533", "-m", "fak_b200.benchmarks.tpcheck",
           "--model", model, "--mix", "q8_0" if model == "tiny-llama" else "q4_k_m", "--fused", str(fused)]
    p = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=400)
    assert p.returncode == 0, p.stderr[-3000:]
    line = [l for l in p.stdout.splitlines() if l.startswith("{")][-1]
    res = json.loads(line)
    assert res["ok"], json.dumps({k: res.get(k) for k in ("teacher_forced", "greedy", "kernel_error",
                                                         "collective_error")})


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", ["p2p", "sp"])
def test_tp2_fused_prefill_matches_tp1(mode):
    """The opt-in in-kernel prefill all-reduce (reduce-scatter in the GEMM epilogue, owner reduce and
    broadcast) and the sequence-parallel prefill on top of it agree with TP=1."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT, FAK_PREFILL_P2P="1",
               FAK_PREFILL_SP="1" if mode == "sp" else "0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29536", "-m", "fak_b200.benchmarks.tpcheck",
           "--model", "tiny-qwen2", "--mix", "q4_k_m", "--fused", "1"]
    p = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=400)
    assert p.returncode == 0, p.stderr[-3000:]
    res = json.loads([l for l in p.stdout.splitlines() if l.startswith("{")][-1])
    assert res["ok"], json.dumps({k: res.get(k) for k in ("teacher_forced", "greedy", "kernel_error",
                                                         "collective_error")})


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep2_moe_matches_ep1():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29534", "-m", "fak_b200.benchmarks.tpcheck",
           "--model", "tiny-qwen3moe", "--mix", "q8_0"]
    p = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=400)
    assert p.returncode == 0, p.stderr[-3000:]
    res = json.loads([l for l in p.stdout.splitlines() if l.startswith("{")][-1])
    assert res["ok"], json.dumps({k: res.get(k) for k in ("teacher_forced", "greedy", "kernel_error",
                                                         "collective_error")})


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_that_never_arrives_fails_the_step():
    """Rank 1 stops launching between steps; rank 0's fused all-reduce wait runs out under a short
    spin limit, returns with error 4 in the step's kernel word, and the engine raises DeviceStepError
    (no GPU is faulted or hung: the waits are bounded; NVLS off, peer buffers through CUDA IPC)."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT, FAK_P2P_MEM="ipc")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29535", "-m",
           "fak_b200.benchmarks.faultcheck"]
    p = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stderr[-3000:]
    res = json.loads([l for l in p.stdout.splitlines() if l.startswith("{")][-1])
    assert res["ok"], res
    assert res["ranks"][0]["seconds_to_error"] < 60, res
