"""Host logic of the data-parallel gradient averaging (xdna_train.ddp) on
world_size-2 gloo process groups on the CPU, plus a rank-failure case made on
the host (a rank that raises before joining the collective): the survivor's
collective ends with an error within the process-group timeout, nothing hangs.
Gradient accumulation: two backward passes, the first inside no_sync(), give
the average of the accumulated gradients; two backward passes without
synchronize() between them raise instead of overwriting a bucket whose
all-reduce is in flight.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q):
    import datetime
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "..", "pytorch-xdna2_b200"))
    import torch.distributed as dist
    from xdna_train.ddp import GradAllReduce
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    # the timeout bounds both the rendezvous (a spawned rank's first torch
    # import can take a while on a loaded machine) and the failure case's wait
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        torch.manual_seed(0)
        model = torch.nn.Sequential(torch.nn.Linear(8, 16), torch.nn.ReLU(), torch.nn.Linear(16, 4))
        ar = GradAllReduce(model, bucket_cap_mb=0.0001, overlap=(mode != "after"))
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected rank failure before the collective")
        x = torch.randn(5, 8, generator=torch.Generator().manual_seed(100 + rank))
        if mode == "accumulate":
            with ar.no_sync():
                model(x).square().sum().backward()
            model(x * 0.5).square().sum().backward()
        elif mode == "double":
            model(x).square().sum().backward()
            model(x).square().sum().backward()  # no synchronize() between: must raise
        else:
            model(x).square().sum().backward()
        # numpy copies travel by value: a tensor put on the queue is shared
        # through a handle that dies with this process, which may exit before
        # the parent reads it
        local = [p.grad.numpy().copy() for p in model.parameters()]
        ar.synchronize()
        q.put((rank, "ok", [p.grad.numpy().copy() for p in model.parameters()], local, len(ar.buckets)))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", repr(e), None, None))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(2):
        r = q.get(timeout=120)
        out[r[0]] = r
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


@pytest.mark.parametrize("mode", ["overlap", "after", "accumulate"])
def test_grads_are_averaged(mode):
    out = _run(mode)
    assert out[0][1] == "ok" and out[1][1] == "ok"
    g0, l0, nb = out[0][2], out[0][3], out[0][4]
    g1, l1 = out[1][2], out[1][3]
    assert nb > 1  # tiny cap: several buckets
    for a, b, x, y in zip(g0, g1, l0, l1):
        a, b, x, y = (torch.from_numpy(t) for t in (a, b, x, y))
        assert torch.allclose(a, b)
        assert torch.allclose(a, (x + y) / 2, atol=1e-6)


def test_rank_failure_surfaces_as_error():
    out = _run("fail")
    assert out[1][1] == "error" and "injected" in out[1][2]
    assert out[0][1] == "error"  # the survivor's collective failed instead of hanging


def test_second_backward_before_synchronize_raises():
    out = _run("double")
    for r in (0, 1):
        assert out[r][1] == "error" and "in flight" in out[r][2]
