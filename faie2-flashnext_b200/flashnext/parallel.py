"""Multi-GPU host layer: one process per GPU, torch.distributed for the plumbing (handle exchange, barriers), the
engine's peer-memory groups for the data path.

The reference runs on at most two GPUs by splitting the layer stack and copying activations through the host; it
has no expert or row partition. This module partitions the decode hot path where it shards naturally:

* row split of a dense GEMV / the lm_head: rank g owns rows [g R / n, (g + 1) R / n); a row's sum order does not
  depend on the split, so every logit is bit-identical to the one-GPU result, and the lm_head's argmax is combined
  from the ranks' (value, index) keys, in-kernel over NVLink (PeerGroup + fn_w_gemv_argmax_group);
* expert parallel MoE: rank g owns experts [g E / n, (g + 1) E / n) (expert_range).

Every rank must issue the same group calls in the same order.
"""

from __future__ import annotations

from typing import Callable, List, Sequence

import numpy as np


def row_range(rows: int, n: int, g: int):
    """Rows [r0, r1) of rank g when `rows` are split over n ranks (contiguous, sizes differ by at most one)."""
    if not (0 <= g < n):
        raise ValueError("rank out of range")
    return g * rows // n, (g + 1) * rows // n


def expert_range(ne: int, n: int, g: int):
    """Experts [e0, e1) owned by rank g (same split as row_range)."""
    return row_range(ne, n, g)


class PeerGroup:
    """This rank's member of a peer-memory group: its own exported buffer, every peer's buffer mapped here, and the
    engine's group id. `all_gather(obj) -> list` exchanges a picklable object between the ranks (e.g.
    torch.distributed.all_gather_object) and `barrier()` synchronises them; both are host-side plumbing only."""

    BYTES = 8 << 20  # key area, MoE slot outputs for k <= 16, d <= 4096, 8 tokens, two parities

    def __init__(self, fn, rank: int, n: int, all_gather: Callable[[object], List[object]],
                 barrier: Callable[[], None], nbytes: int = BYTES):
        self.fn, self.rank, self.n, self.barrier = fn, rank, n, barrier
        self.nbytes = nbytes
        self.own, handle = fn.ipc_alloc(nbytes)
        handles = all_gather(handle)
        if len(handles) != n:
            raise RuntimeError("handle exchange returned the wrong number of ranks")
        self.bases: List[int] = []
        self.opened: List[int] = []
        try:
            for r, h in enumerate(handles):
                if r == rank:
                    self.bases.append(self.own)
                else:
                    p = fn.ipc_open(h)
                    self.opened.append(p)
                    self.bases.append(p)
            self.id = fn.group_create(rank, n, self.bases, nbytes)
        except Exception:
            self._release()
            raise
        barrier()

    def _release(self):
        for p in self.opened:
            self.fn.ipc_close(p)
        self.opened = []
        if self.own:
            self.fn.ipc_free(self.own)
            self.own = 0

    def close(self):
        """Free the group: every rank first stops using it, then the mappings of the peers go, then the own buffer
        (after a barrier, so no peer still maps it)."""
        if getattr(self, "id", 0):
            self.fn.group_free(self.id)
            self.id = 0
        self.barrier()
        for p in self.opened:
            self.fn.ipc_close(p)
        self.opened = []
        self.barrier()
        if self.own:
            self.fn.ipc_free(self.own)
            self.own = 0


class LmHeadSplit:
    """The lm_head split by vocabulary rows over a PeerGroup: this rank uploads rows row_range(V, n, rank) of the GGUF
    rows and runs the GEMV with the fused argmax whose keys every rank combines (fn_w_gemv_argmax_group)."""

    def __init__(self, fn, group: PeerGroup, qtype: int, raw_rows: np.ndarray, vocab: int, cols: int):
        self.fn, self.group = fn, group
        self.r0, self.r1 = row_range(vocab, group.n, group.rank)
        part = np.ascontiguousarray(raw_rows[self.r0:self.r1]) if raw_rows.shape[0] == vocab else raw_rows
        if part.shape[0] != self.r1 - self.r0:
            raise ValueError("raw_rows must be the whole vocabulary or exactly this rank's slice")
        self.h = fn.w_create(qtype, part, self.r1 - self.r0, cols)
        self.cols = cols

    def run(self, x_ptr: int, xs: int, index_ptr: int, nt: int = 1, y_ptr: int = 0, flags: int = 0, stream: int = 0):
        """index[t] (device int32, on every rank) = the vocabulary-wide argmax of W . x[t]; y (device, nullable)
        receives this rank's logit slice [nt][r1 - r0]."""
        self.fn.w_gemv_argmax_group(self.h, self.group.id, x_ptr, xs, y_ptr, self.r1 - self.r0, nt, flags, self.r0,
                                    index_ptr, stream)

    def close(self):
        if self.h:
            self.fn.w_free(self.h)
            self.h = 0


def combine_keys(keys: Sequence[np.ndarray]) -> np.ndarray:
    """Host restatement of the key combine (for tests of the partition logic): the index of the largest key over the
    ranks' key arrays [nt] (uint64), 0 when every key is 0."""
    k = np.max(np.stack([np.asarray(a, np.uint64) for a in keys]), axis=0)
    return np.where(k == 0, 0, (np.uint64(0xFFFFFFFF) - (k & np.uint64(0xFFFFFFFF))).astype(np.int64))
