"""The N>1 path on CPU: two gloo ranks shard a batch by work, produce per-sequence rows and gather
them to rank 0 in the global order (the bench's gather step); a rank that fails is seen by the
other through a short process-group timeout instead of a hang."""
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, fail_rank):
    sys.path.insert(0, ROOT)
    import datetime
    import torch
    import torch.distributed as dist
    from tenzor_b200 import synthetic as S
    from tenzor_b200.shard import RankGather, gather_to_rank0, shard_by_tokens
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        ids, lens = S.token_batch(37, 64, 1, 64, seed=5)
        mine = shard_by_tokens(lens, world)[rank]
        local = torch.stack([torch.full((4,), float(i)) for i in mine]) if len(mine) else torch.zeros((0, 4))
        if rank == fail_rank:
            raise RuntimeError("injected rank failure")
        out = gather_to_rank0(local, mine, len(lens))
        # the bench's per-step gather: sizes exchanged once, padded buffer, reorder on rank 0
        rg = RankGather(mine, len(lens), 4, torch.device("cpu"),
                        lambda table, ids, o: o.copy_(table[ids.long()]))
        pad = torch.zeros((rg.cap, 4))
        pad[: len(mine)] = local
        out2 = rg.step(pad)
        out3 = rg.step(pad)  # a second step reuses the buffers
        if rank == 0:
            assert torch.equal(out2, out) and torch.equal(out3, out)
            q.put(("ok", out[:, 0].numpy().tolist()))
    except Exception as e:  # noqa: BLE001
        q.put(("err", f"rank {rank}: {type(e).__name__}: {e}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q, fail_rank)) for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=90)
        if p.is_alive():
            p.kill()
    res = []
    while not q.empty():
        res.append(q.get())
    return res


def test_two_rank_gather_order():
    res = _run(2)
    oks = [r for r in res if r[0] == "ok"]
    assert oks, res
    assert oks[0][1] == [float(i) for i in range(37)]


def test_rank_failure_is_detected_not_hung():
    res = _run(2, fail_rank=1)
    kinds = sorted(r[0] for r in res)
    assert "err" in kinds and "ok" not in kinds, res
