"""Data-parallel step logic on CPU with world_size 2 (gloo): gradient
accumulation with no_sync + DDP averaging give the same gradients as one
process over the union of the micro-batches; a failing rank surfaces as an
error on the other rank instead of a hang."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup(rank, world, port, timeout_s=60):
    import datetime

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _tiny_setup(world, ddp):
    from hackable_lm_b200 import train as tr

    torch.set_num_threads(1)
    return tr.build(torch.device("cpu"), depth=2, vocab=64, seq_len=16, micro_batch=2,
                    global_tokens=2 * 16 * 4, world=world, backend="torch", seed=0, ddp=ddp)


def _worker_dp(rank, world, port, out_path):
    from hackable_lm_b200 import train as tr

    _setup(rank, world, port)
    try:
        s = _tiny_setup(world, ddp=True)
        batches = tr.synthetic_batches(4, 2, 16, 64, rank=0, device="cpu")
        mine = batches[rank * s.accum:(rank + 1) * s.accum]
        loss = tr.train_step(s, mine, optimizer_step=False)
        if rank == 0:
            torch.save({n: p.grad.detach().float().clone() for n, p in s.model.named_parameters()}, out_path)
            torch.save(loss.float(), out_path + ".loss")
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_ddp_step_matches_single_process(tmp_path):
    from hackable_lm_b200 import train as tr

    out = str(tmp_path / "params.pt")
    port = _free_port()
    mp.start_processes(_worker_dp, args=(2, port, out), nprocs=2, join=True, start_method="spawn")
    ddp_grads = torch.load(out)

    s = _tiny_setup(1, ddp=False)
    assert s.accum == 4
    batches = tr.synthetic_batches(4, 2, 16, 64, rank=0, device="cpu")
    tr.train_step(s, batches, optimizer_step=False)
    for n, p in s.model.named_parameters():
        g = p.grad.detach().float()
        scale = g.abs().max().item() + 1e-12
        # bf16 gradients: summation order differs (per-rank accumulation + all-reduce)
        torch.testing.assert_close(ddp_grads[n] / scale, g / scale, atol=3e-2, rtol=0, msg=n)


def _worker_fail(rank, world, port, flag_path):
    _setup(rank, world, port, timeout_s=10)
    try:
        if rank == 1:
            raise RuntimeError("rank 1 fails before the collective")
        t = torch.ones(4)
        try:
            dist.all_reduce(t)
            open(flag_path, "w").write("completed")
        except Exception as exc:  # noqa: BLE001
            open(flag_path, "w").write(f"error: {type(exc).__name__}")
    finally:
        if rank == 0:
            try:
                dist.destroy_process_group()
            except Exception:  # noqa: BLE001
                pass


@pytest.mark.timeout(300)
def test_failed_rank_surfaces_as_error(tmp_path):
    flag = str(tmp_path / "flag.txt")
    port = _free_port()
    ctx = mp.start_processes(_worker_fail, args=(2, port, flag), nprocs=2, join=False, start_method="spawn")
    procs = ctx.processes
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung instead of failing"
    assert procs[1].exitcode != 0
    assert os.path.exists(flag) and open(flag).read().startswith("error"), "rank 0 did not see the failure"
