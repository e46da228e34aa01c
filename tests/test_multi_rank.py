"""Batch-row sharding host logic with two gloo ranks on the CPU: row blocks,
the row gather (even and uneven), max-over-ranks timing, a sharded greedy
decode equal to the single-process one, and a rank that fails before a
collective being seen by its peer as an error rather than a hang."""

import datetime
import multiprocessing as mp
import os
import socket
import sys
import traceback

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "dispatcher-hybrid-2_b200")

VOCAB = 97


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class CountingDecoder:
    """Stand-in for a decoder (same prefill/step contract): the next-token
    logits of a row are one-hot at (31 * running token sum + 7 * row) % VOCAB,
    so every row's output depends on its own history and on its global row
    index only."""

    def __init__(self, row0):
        self.row0 = row0

    def _onehot(self, s, rows):
        k = (31 * s + 7 * rows) % VOCAB
        return torch.nn.functional.one_hot(k, VOCAB).float()

    def prefill(self, idx):
        B, T = idx.shape
        rows = torch.arange(self.row0, self.row0 + B).view(B, 1)
        csum = idx.cumsum(1)
        self.sum = csum[:, -1].clone()
        return self._onehot(csum, rows.expand(B, T))

    def step(self, tok):
        self.sum = self.sum + tok
        rows = torch.arange(self.row0, self.row0 + tok.shape[0])
        return self._onehot(self.sum, rows)


def _worker(rank, world, port, mode, q):
    try:
        sys.path.insert(0, PKG)
        import torch.distributed as dist
        from dispatcher_b200 import sharding
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=20))
        out = {}
        if mode == "ok":
            assert sharding.world_info() == (world, rank)
            # blocks cover every row exactly once
            for n in (2, 5, 8, 17):
                got = sharding.gather_rows(torch.arange(n)[sharding.shard_rows(n, world, rank)], n)
                out[f"cover{n}"] = got.tolist()
            # rows with trailing dims
            n = 7
            blk = sharding.shard_rows(n, world, rank)
            full = torch.arange(n * 3 * 2, dtype=torch.float32).view(n, 3, 2)
            out["gather3d"] = bool(torch.equal(sharding.gather_rows(full[blk], n), full))
            out["max"] = sharding.max_over_ranks(1.5 + rank)
            sharding.barrier()
            # sharded greedy decode == single process
            n_rows, T, steps = 6, 9, 5
            g = torch.Generator().manual_seed(3)
            prompt = torch.randint(0, VOCAB, (n_rows, T), generator=g)
            blk = sharding.shard_rows(n_rows, world, rank)
            dec = sharding.ShardedGreedyDecode(CountingDecoder(blk.start), n_rows)
            out["decode"] = dec.run(prompt[blk], steps).tolist()
        elif mode == "fail":
            if rank == 1:
                raise RuntimeError("planted failure before the collective")
            try:
                sharding.gather_rows(torch.zeros(1), 2)
                out["peer_failure_seen"] = False
            except Exception as e:  # noqa: BLE001 - any error is the expected outcome
                out["peer_failure_seen"] = True
                out["error"] = type(e).__name__
        q.put((rank, out, None))
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        q.put((rank, None, traceback.format_exc()))


def _run(mode, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, out, err = q.get(timeout=timeout)
        results[rank] = (out, err)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return results


def _single_process_decode():
    sys.path.insert(0, PKG)
    from dispatcher_b200 import sharding
    n_rows, T, steps = 6, 9, 5
    g = torch.Generator().manual_seed(3)
    prompt = torch.randint(0, VOCAB, (n_rows, T), generator=g)
    return sharding.ShardedGreedyDecode(CountingDecoder(0), n_rows).run(prompt, steps).tolist()


def test_two_gloo_ranks_shard_gather_and_decode():
    res = _run("ok")
    want = _single_process_decode()
    for rank in (0, 1):
        out, err = res[rank]
        assert err is None, err
        for n in (2, 5, 8, 17):
            assert out[f"cover{n}"] == list(range(n))
        assert out["gather3d"]
        assert out["max"] == 2.5
        assert out["decode"] == want


def test_failed_rank_is_an_error_not_a_hang():
    res = _run("fail")
    assert res[1][1] is not None and "planted failure" in res[1][1]
    out, err = res[0]
    assert err is None, err
    assert out["peer_failure_seen"]


def test_shard_rows_rejects_bad_arguments():
    sys.path.insert(0, PKG)
    from dispatcher_b200 import sharding
    with pytest.raises(ValueError):
        sharding.shard_rows(1, 2, 0)
    with pytest.raises(ValueError):
        sharding.shard_rows(8, 2, 2)
    assert sharding.shard_sizes(17, 4) == [4, 4, 4, 5]
