"""Peer-memory collectives. Multi-GPU cases run as child processes (one per GPU) and compare
against exact integer-valued expectations; the bounded-wait case runs on one GPU: a "peer" that
never signals must make the kernel give up with an error status instead of hanging."""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_peer_wait_times_out_and_context_survives():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from minisgl._native import cuda

    c = cuda()
    c.get_error()
    cap = 1 << 16
    a = c.peer_alloc(c.peer_flag_bytes() + 2 * cap)
    b = c.peer_alloc(c.peer_flag_bytes() + 2 * cap)  # plays rank 1, which never arrives
    try:
        state = torch.zeros(2 * c.peer_grid(), dtype=torch.int32, device="cuda")
        x = torch.ones(1024, dtype=torch.bfloat16, device="cuda")
        out = torch.empty_like(x)
        c.peer_collective(0, out, x, [a, b], 0, cap, state, 50_000_000)  # 50 ms limit
        torch.cuda.synchronize()
        code, _ = c.get_error()
        assert code == 2  # kErrPeerTimeout
        # the context is still usable
        y = torch.randn(256, 256, device="cuda")
        assert torch.isfinite((y @ y).sum()).item()
    finally:
        c.peer_free(a)
        c.peer_free(b)


WORKER = r"""
import os, sys
sys.path.insert(0, {root!r})
import torch, torch.distributed as dist
from datetime import timedelta
os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("gloo", timeout=timedelta(seconds=60))
from minisgl.parallel.comm import TorchDistributedImpl
from minisgl.parallel.peer import PeerCommImpl
from minisgl._native import cuda
dev = torch.device("cuda", rank)
impl = PeerCommImpl(dist.group.WORLD, dev, 8 << 20, TorchDistributedImpl())
for it in range(20):
    for n in (8, 1000, 4096 * 16, 300_000, 2 * 1024 * 1024):
        x = torch.full((n,), float(rank + 1 + it % 3), dtype=torch.bfloat16, device=dev)
        if it % 5 == 0 and rank == 0:
            torch.cuda._sleep(2_000_000)  # a lagging rank
        y = impl.all_reduce(x)
        exp = sum(r + 1 + it % 3 for r in range(world))
        assert torch.all(y == exp).item(), (it, n, y[:4])
    g = impl.all_gather(torch.full((3, 8), float(rank), dtype=torch.float32, device=dev))
    assert torch.equal(g[:, 0].cpu(), torch.arange(world, dtype=torch.float32).repeat_interleave(3))
torch.cuda.synchronize()
assert cuda().get_error()[0] == 0
impl.close()
dist.barrier()
print("OK", rank, flush=True)
"""


@pytest.mark.multigpu
def test_peer_collectives_multi_gpu(tmp_path, free_port):
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if n < 2:
        pytest.skip("needs 2+ GPUs")
    world = min(n, 8)
    script = tmp_path / "w.py"
    script.write_text(WORKER.format(root=ROOT))
    procs = [subprocess.Popen([sys.executable, str(script)], env=dict(
        os.environ, RANK=str(r), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(free_port),
        NCCL_NVLS_ENABLE="0"), stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True) for r in range(world)]
    outs = [p.communicate(timeout=300)[0] for p in procs]
    assert all(p.returncode == 0 for p in procs), outs


NVLS_WORKER = r"""
import os, sys
sys.path.insert(0, {root!r})
import torch, torch.distributed as dist
from datetime import timedelta
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dev = torch.device("cuda", rank)
dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
cpu = dist.new_group(backend="gloo", timeout=timedelta(seconds=60))
from minisgl import ops
from minisgl._native import cuda
from minisgl.parallel.nvls import NvlsNormComm
try:
    impl = NvlsNormComm(dist.group.WORLD, cpu, dev, 8 << 20)
except RuntimeError as e:
    print("SKIP", e, flush=True)
    dist.barrier(group=cpu)
    dist.destroy_process_group()
    sys.exit(0)
H, eps = 5120, 1e-6
g = torch.Generator(device="cpu").manual_seed(1234)
w = (torch.rand(H, generator=g) + 0.5).to(dev, torch.bfloat16)


def expected(x, res0):
    parts = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(parts, x)
    s = torch.stack([p.float() for p in parts]).sum(0)
    if res0 is not None:
        s = s + res0.float()
    r = s.to(torch.bfloat16)
    r32 = r.float()
    return r, (r32 * torch.rsqrt(r32.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(torch.bfloat16)


def check(T, res, out, exp_res, exp_out):
    # the RS form keeps only this rank's residual rows (i % world == rank); LL keeps them all
    rows = torch.arange(T, device=dev)
    mine = rows if impl.is_ll(T, H) else rows[rows % world == rank]
    torch.testing.assert_close(res[mine].float(), exp_res[mine].float(), atol=3e-2, rtol=2e-2)
    torch.testing.assert_close(out.float(), exp_out.float(), atol=3e-2, rtol=2e-2)


# LL for T x world x H x 4 <= 2 MiB (T <= 51 at 2 ranks, 12 at 8), RS above; alternate them
for it, T in enumerate([1, 7, 128, 256, 129, 800, 3, 256, 1, 400, 2, 64]):
    gp = torch.Generator(device="cpu").manual_seed(100 * it + rank)
    x = torch.randn(T, H, generator=gp).to(dev, torch.bfloat16)
    gr = torch.Generator(device="cpu").manual_seed(100 * it + 77)
    first = it % 4 == 0
    res0 = None if first else torch.randn(T, H, generator=gr).to(dev, torch.bfloat16)
    exp_res, exp_out = expected(x, res0)
    if it == 2 and rank == 0:
        torch.cuda._sleep(5_000_000)  # a lagging rank
    res = None if first else res0.clone()
    out, res = impl.all_reduce_add_rmsnorm(x, res, w, eps)
    torch.cuda.synchronize()
    check(T, res, out, exp_res, exp_out)

# GEMM fused with the collective: the row-parallel GEMM writes this rank's staging region and
# signals arrival itself; the partial sums are the same GEMM's output through the plain path
for it, (T, K) in enumerate([(64, 640), (256, 2560), (200, 640), (96, 4352), (256, 5120)]):
    gp = torch.Generator(device="cpu").manual_seed(500 + 10 * it + rank)
    xin = (torch.randn(T, K, generator=gp) * 0.5).to(dev, torch.bfloat16)
    wt = (torch.randn(H, K, generator=gp) * 0.02).to(dev, torch.bfloat16)
    gr = torch.Generator(device="cpu").manual_seed(900 + it)
    res0 = torch.randn(T, H, generator=gr).to(dev, torch.bfloat16)
    partial = ops.linear(xin, wt)
    exp_res, exp_out = expected(partial, res0)
    if it == 1 and rank == world - 1:
        torch.cuda._sleep(5_000_000)
    y = impl.linear_into_staging(xin, wt, None)
    assert y is not None and not impl.is_ll(T, H)
    res = res0.clone()
    out, res = impl.all_reduce_add_rmsnorm(y, res, w, eps)
    torch.cuda.synchronize()
    check(T, res, out, exp_res, exp_out)

# CUDA-graph replays: the per-CTA call counters keep advancing across replays of one captured
# sequence (LL, RS and GEMM-fused RS calls interleaved); a different rank lags before each replay.
# An RS call's output is a view of the gather region, overwritten by the next RS call, so each
# result is copied out right after its call (as the GEMM that consumes it would read it).
Ts = [4, 300, 8, 300, 128]
xs, res0, exp = [], [], []
for i, T in enumerate(Ts):
    gp = torch.Generator(device="cpu").manual_seed(1000 + 10 * i + rank)
    if i == 4:  # GEMM-fused call: K = 640, the input is [T, K]
        xin = (torch.randn(T, 640, generator=gp) * 0.5).to(dev, torch.bfloat16)
        wt = (torch.randn(H, 640, generator=gp) * 0.02).to(dev, torch.bfloat16)
        xs.append((xin, wt))
        part = ops.linear(xin, wt)
    else:
        xs.append(torch.randn(T, H, generator=gp).to(dev, torch.bfloat16))
        part = xs[i]
    gr = torch.Generator(device="cpu").manual_seed(2000 + i)
    res0.append(torch.randn(T, H, generator=gr).to(dev, torch.bfloat16))
    exp.append(expected(part, res0[i])[1])
res = [r.clone() for r in res0]
saved = [torch.empty(T, H, dtype=torch.bfloat16, device=dev) for T in Ts]


def sequence():
    for i in range(len(Ts)):
        res[i].copy_(res0[i])
        if i == 4:
            y = impl.linear_into_staging(xs[i][0], xs[i][1], None)
        else:
            y = xs[i]
        out, _ = impl.all_reduce_add_rmsnorm(y, res[i], w, eps)
        saved[i].copy_(out)


side = torch.cuda.Stream()
with torch.cuda.stream(side):
    sequence()
torch.cuda.synchronize()
graph = torch.cuda.CUDAGraph()
with torch.cuda.graph(graph, stream=side):
    sequence()
for rep in range(6):
    if rank == rep % world:
        torch.cuda._sleep(3_000_000)
    graph.replay()
    torch.cuda.synchronize()
    for i in range(len(Ts)):
        torch.testing.assert_close(saved[i].float(), exp[i].float(), atol=3e-2, rtol=2e-2)
del graph
assert cuda().get_error()[0] == 0
dist.barrier(group=cpu)
impl.close()
dist.destroy_process_group()
print("OK", rank, flush=True)
"""


@pytest.mark.multigpu
def test_nvls_allreduce_rmsnorm_multi_gpu(tmp_path, free_port):
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if n < 2:
        pytest.skip("needs 2+ GPUs")
    world = min(n, 8)
    script = tmp_path / "nvls.py"
    script.write_text(NVLS_WORKER.format(root=ROOT))
    procs = [subprocess.Popen([sys.executable, str(script)], env=dict(
        os.environ, RANK=str(r), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(free_port),
        LOCAL_RANK=str(r)), stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True) for r in range(world)]
    outs = [p.communicate(timeout=300)[0] for p in procs]
    assert all(p.returncode == 0 for p in procs), outs
    assert all(("OK" in o) or ("SKIP" in o) for o in outs), outs
