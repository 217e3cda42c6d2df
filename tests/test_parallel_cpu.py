"""CPU tests of the multi-GPU host layer (flashnext/parallel.py) with world_size-2 `gloo` process groups: the row and
expert partitions, the lm_head key protocol (each rank's slice -> its winning key, keys gathered, combined by max)
against the oracle argmax of the whole vocabulary, and the peer-group handle exchange with a fake engine."""

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from oracle.argmax import argmax_fast, slice_key
from parallel import PeerGroup, combine_keys, expert_range, row_range

NAN = np.float32("nan")


def test_row_and_expert_ranges_partition():
    for rows in (1, 7, 512, 151936, 12288):
        for n in (1, 2, 3, 4, 8):
            parts = [row_range(rows, n, g) for g in range(n)]
            assert parts[0][0] == 0 and parts[-1][1] == rows
            assert all(parts[g][1] == parts[g + 1][0] for g in range(n - 1))
            sizes = [b - a for a, b in parts]
            assert max(sizes) - min(sizes) <= 1
    assert [expert_range(512, 8, g) for g in (0, 7)] == [(0, 64), (448, 512)]
    with pytest.raises(ValueError):
        row_range(10, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _logit_cases():
    rng = np.random.default_rng(0)
    V = 10007
    cases = []
    lg = rng.standard_normal((3, V)).astype(np.float32)
    cases.append(lg)
    t = lg.copy()
    m = np.float32(t.max() + 1)
    t[:, [V // 2 + 5, V // 2 - 5, V - 1]] = m  # ties on both sides of the two-rank boundary
    cases.append(t)
    t = lg.copy()
    t[:, :V // 2] = NAN  # rank 0's slice all NaN
    cases.append(t)
    t = -np.abs(lg) - 1
    t[:, V - 3] = np.float32(0.0)
    t[:, 17] = np.float32(-0.0)  # -0 on rank 0 ties +0 on rank 1: rank 0's lower index wins
    cases.append(t)
    cases.append(np.full((2, V), -np.inf, np.float32))
    return cases


def _keys_worker(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        res = []
        for lg in _logit_cases():
            r0, r1 = row_range(lg.shape[1], world, rank)
            k = slice_key(lg[:, r0:r1], r0)
            allk = [torch.zeros(len(k), dtype=torch.int64) for _ in range(world)]
            dist.all_gather(allk, torch.from_numpy(k.view(np.int64)))
            res.append(combine_keys([a.numpy().view(np.uint64) for a in allk]))
        np.save(os.path.join(out_dir, f"r{rank}.npy"), np.array(res, dtype=object), allow_pickle=True)
    finally:
        dist.destroy_process_group()


def test_lm_head_key_protocol_two_ranks(tmp_path):
    port = _free_port()
    mp.start_processes(_keys_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    want = [argmax_fast(lg) for lg in _logit_cases()]
    for rank in range(2):
        got = np.load(tmp_path / f"r{rank}.npy", allow_pickle=True)
        for g, w in zip(got, want):
            assert np.array_equal(g, w), (rank, g, w)


class _FakeFN:
    """Records the engine calls a PeerGroup makes (no GPU)."""

    def __init__(self, rank):
        self.rank, self.calls = rank, []

    def ipc_alloc(self, nbytes):
        self.calls.append(("alloc", nbytes))
        return 0x1000 * (self.rank + 1), bytes([self.rank]) * 64

    def ipc_open(self, h):
        self.calls.append(("open", h[0]))
        return 0x100000 * (h[0] + 1)

    def group_create(self, rank, n, bases, nbytes):
        self.calls.append(("group", rank, n, tuple(bases)))
        return 7

    def group_free(self, g):
        self.calls.append(("group_free", g))

    def ipc_close(self, p):
        self.calls.append(("close", p))

    def ipc_free(self, p):
        self.calls.append(("free", p))


def _group_worker(rank, world, port, out_dir):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        f = _FakeFN(rank)

        def gather(obj):
            out = [None] * world
            dist.all_gather_object(out, obj)
            return out

        g = PeerGroup(f, rank, world, gather, dist.barrier, nbytes=4096)
        assert g.id == 7
        g.close()
        np.save(os.path.join(out_dir, f"g{rank}.npy"), np.array(f.calls, dtype=object), allow_pickle=True)
    finally:
        dist.destroy_process_group()


def test_peer_group_handle_exchange_two_ranks(tmp_path):
    port = _free_port()
    mp.start_processes(_group_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    for rank in range(2):
        calls = list(np.load(tmp_path / f"g{rank}.npy", allow_pickle=True))
        peer = 1 - rank
        own, mapped = 0x1000 * (rank + 1), 0x100000 * (peer + 1)
        bases = [own, mapped] if rank == 0 else [mapped, own]
        assert calls == [("alloc", 4096), ("open", peer), ("group", rank, 2, tuple(bases)), ("group_free", 7),
                         ("close", mapped), ("free", own)]
