"""Worker of the multi-GPU lm_head test (launched by tests/test_mgpu.py under torchrun, one process per GPU).

Row-split Q6_K lm_head 151936 x 2048 over the ranks with the argmax combined over NVLink in-kernel
(fn_w_gemv_argmax_group). Checks on every rank: the logit slice is bit-identical to the one-GPU GEMV's rows; the
index equals the oracle argmax of the one-GPU logits (nt 1 and 3, repeated calls, CUDA-graph replays); the NCCL
all-gather of the ranks' keys gives the same index. Then times both (device events, max over ranks) and, with
--fail-test, checks that a rank that skips a call makes the others' bounded wait give up with an error instead of
hanging. Prints one JSON line on rank 0.
"""

import datetime
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path[:0] = [ROOT, os.path.join(ROOT, "faie2-flashnext_b200", "flashnext"), os.path.join(ROOT, "faie2-flashnext_b200")]

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from fn import FN  # noqa: E402
from oracle.argmax import argmax_fast  # noqa: E402
from parallel import LmHeadSplit, PeerGroup, row_range  # noqa: E402
from synth import BY_NAME, random_blocks  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    fn = FN()
    fn.set_device(local)
    V, cols, q = 151936, 2048, BY_NAME["Q6_K"]
    rng = np.random.default_rng(11)
    raw = random_blocks(q, V, cols, rng)
    xs = rng.standard_normal((12, cols), dtype=np.float32)

    def gather(obj):
        out = [None] * world
        dist.all_gather_object(out, obj)
        return out

    group = PeerGroup(fn, rank, world, gather, dist.barrier)
    head = LmHeadSplit(fn, group, q, raw, V, cols)
    r0, r1 = head.r0, head.r1
    st = torch.cuda.Stream()
    torch.cuda.set_stream(st)
    s = st.cuda_stream
    x_d = torch.from_numpy(xs).cuda()
    y_d = torch.empty((8, r1 - r0), device="cuda")
    idx_d = torch.full((8,), -2, dtype=torch.int32, device="cuda")
    fails = []

    def check(cond, what):
        if not cond:
            fails.append(what)

    # the one-GPU reference: the whole lm_head on this rank's GPU (the engine's own GEMV, checked against the
    # float64 oracle by the single-GPU tests), in batches of 3 tokens
    y_full = np.concatenate([fn.gemv(q, raw, V, cols, xs[i:i + 3]) for i in range(0, 12, 3)])
    want = argmax_fast(y_full)

    # nt = 1, repeated calls with different tokens; nt = 3
    for i in range(6):
        head.run(x_d[i].data_ptr(), cols, idx_d.data_ptr(), 1, y_d.data_ptr(), 0, s)
        fn.sync(s)
        check(int(idx_d[0]) == int(want[i]), f"nt=1 call {i}: {int(idx_d[0])} != {int(want[i])}")
        check(np.array_equal(y_d[0].cpu().numpy().view(np.uint32), y_full[i, r0:r1].view(np.uint32)), f"slice {i}")
    head.run(x_d[6].data_ptr(), cols, idx_d.data_ptr(), 3, y_d.data_ptr(), 0, s)
    fn.sync(s)
    check(np.array_equal(idx_d[:3].cpu().numpy(), want[6:9]), "nt=3")

    # CUDA graph of 4 calls (tokens 8..11), replayed twice
    g = torch.cuda.CUDAGraph()
    outs = torch.full((4, 8), -2, dtype=torch.int32, device="cuda")
    with torch.cuda.graph(g, stream=st):
        for i in range(4):
            head.run(x_d[8 + i].data_ptr(), cols, outs[i].data_ptr(), 1, 0, 0, torch.cuda.current_stream().cuda_stream)
    for rep in range(2):
        outs.fill_(-2)
        g.replay()
        fn.sync(s)
        check(np.array_equal(outs[:, 0].cpu().numpy(), want[8:12]), f"graph replay {rep}")

    # NCCL baseline: each rank's key, all-gathered, combined
    keys = torch.zeros(8, dtype=torch.int64, device="cuda")
    allk = torch.zeros((world, 1), dtype=torch.int64, device="cuda")
    nidx = torch.zeros(8, dtype=torch.int32, device="cuda")

    def nccl_call(i):
        fn.w_gemv_argmax(head.h, x_d[i].data_ptr(), cols, 0, r1 - r0, 1, 0, r0, 0, keys.data_ptr(), s)
        dist.all_gather_into_tensor(allk, keys[:1])
        fn.argmax_keys(allk.data_ptr(), world, 1, nidx.data_ptr(), s)

    for i in range(3):
        nccl_call(i)
        fn.sync(s)
        check(int(nidx[0]) == int(want[i]), f"nccl combine {i}")

    # timing: device events around K calls, max over ranks
    K = 200
    gt = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gt, stream=st):
        for i in range(K):
            head.run(x_d[i % 12].data_ptr(), cols, idx_d.data_ptr(), 1, 0, 0, torch.cuda.current_stream().cuda_stream)

    def timed(fn_step, reps):
        dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        fn_step()
        b.record(st)
        torch.cuda.synchronize()
        t = torch.tensor([a.elapsed_time(b) / reps * 1e3], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    gt.replay()
    fn.sync(s)
    us_p2p = timed(gt.replay, K)

    def nccl_loop():
        for i in range(50):
            nccl_call(i % 12)

    nccl_loop()
    us_nccl = timed(nccl_loop, 50)
    fn.sync(s)
    check(int(idx_d[0]) == int(want[(K - 1) % 12]), "after timed graph")
    del g, gt

    failure = None
    if "--fail-test" in sys.argv and world > 1:
        # rank 1 skips one call: the others' combine must give up (bounded wait) with an error, index -1
        dist.barrier()
        if rank != 1:
            head.run(x_d[0].data_ptr(), cols, idx_d.data_ptr(), 1, 0, 0, s)
            try:
                fn.sync(s)
                failure = "no error"
            except RuntimeError as e:
                failure = "ok" if "peer" in str(e) and int(idx_d[0]) == -1 else f"unexpected: {e}"
            check(failure == "ok", f"failure test: {failure}")
        dist.barrier()

    head.close()
    group.close()
    nf = torch.tensor([len(fails)], device="cuda")
    dist.all_reduce(nf)
    if fails:
        print(f"rank {rank} FAIL: {fails}", flush=True)
    if rank == 0:
        print(json.dumps({"test": "lm_head row split + argmax", "n_gpus": world, "vocab": V, "cols": cols,
                          "format": "Q6_K", "us_per_call_p2p": round(us_p2p, 2), "us_per_call_nccl": round(us_nccl, 2),
                          "weight_bytes_per_rank": int(raw.nbytes // world), "failure_test": failure,
                          "failures": int(nf.item())}), flush=True)
    dist.destroy_process_group()
    sys.exit(1 if int(nf.item()) else 0)


if __name__ == "__main__":
    main()
