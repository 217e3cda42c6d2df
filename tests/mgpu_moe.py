"""Worker of the multi-GPU expert-parallel MoE test (launched by tests/test_mgpu.py under torchrun, one process per
GPU).

BASELINE config 3 (512 experts, top-10, width 512, hidden 2048, IQ3_XXS gate/up, Q4_K down, shared expert) split by
experts over the ranks (fn_moe_ep_*). Checks on every rank: y is bit-identical to the one-GPU layer (fn_moe_run on
the full weights, itself checked against the float64 oracle by the single-GPU tests) for nt 1 and 3, over repeated
calls with different routings and over CUDA-graph replays. Then times the expert-parallel and the one-GPU layer
(device events, max over ranks) and, with --fail-test, checks that a rank that skips a call makes the others'
bounded wait give up with an error. Prints one JSON line on rank 0.
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
from parallel import PeerGroup, expert_range  # noqa: E402
from synth import BY_NAME, random_blocks  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    fn = FN()
    fn.set_device(local)
    gu, dn, ne, k, ffe, d = BY_NAME["IQ3_XXS"], BY_NAME["Q4_K"], 512, 10, 512, 2048
    rng = np.random.default_rng(3)
    Wg = random_blocks(gu, ne * ffe, d, rng)
    Wu = random_blocks(gu, ne * ffe, d, rng)
    Wd = random_blocks(dn, ne * d, ffe, rng)
    Wsg, Wsu = random_blocks(gu, ffe, d, rng), random_blocks(gu, ffe, d, rng)
    Wsd = random_blocks(dn, d, ffe, rng)
    NX = 12
    xs = rng.standard_normal((NX, d), dtype=np.float32)
    logits = (rng.standard_normal((NX, ne + 1)) * 2.0).astype(np.float32)

    def gather(obj):
        out = [None] * world
        dist.all_gather_object(out, obj)
        return out

    group = PeerGroup(fn, rank, world, gather, dist.barrier)
    e0, e1 = expert_range(ne, world, rank)
    h_ep = fn.moe_ep_create(gu, dn, ne, k, ffe, d, group.id, Wg[e0 * ffe:e1 * ffe], Wu[e0 * ffe:e1 * ffe],
                            Wd[e0 * d:e1 * d], Wsg, Wsu, Wsd)
    h_one = fn.moe_create(gu, dn, ne, k, ffe, d, Wg, Wu, Wd, Wsg, Wsu, Wsd)
    del Wg, Wu, Wd
    st = torch.cuda.Stream()
    torch.cuda.set_stream(st)
    s = st.cuda_stream
    x_d = torch.from_numpy(xs).cuda()
    l_d = torch.from_numpy(logits).cuda()
    y_ep = torch.zeros((8, d), device="cuda")
    y_one = torch.zeros((8, d), device="cuda")
    fails = []

    def check(cond, what):
        if not cond:
            fails.append(what)

    def same(a, b):
        return np.array_equal(a.cpu().numpy().view(np.uint32), b.cpu().numpy().view(np.uint32))

    for i in range(5):
        fn.moe_ep_run(h_ep, l_d[i].data_ptr(), ne + 1, x_d[i].data_ptr(), y_ep.data_ptr(), 1, 0, s)
        fn.moe_run(h_one, l_d[i].data_ptr(), ne + 1, x_d[i].data_ptr(), y_one.data_ptr(), 1, 0, s)
        fn.sync(s)
        check(same(y_ep[0], y_one[0]), f"nt=1 call {i}")
    fn.moe_ep_run(h_ep, l_d[5].data_ptr(), ne + 1, x_d[5].data_ptr(), y_ep.data_ptr(), 3, 0, s)
    fn.moe_run(h_one, l_d[5].data_ptr(), ne + 1, x_d[5].data_ptr(), y_one.data_ptr(), 3, 0, s)
    fn.sync(s)
    check(same(y_ep[:3], y_one[:3]), "nt=3")

    # CUDA graph: 4 layers (tokens 8..11) into 4 outputs, replayed twice
    outs = torch.zeros((4, d), device="cuda")
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        cs = torch.cuda.current_stream().cuda_stream
        for i in range(4):
            fn.moe_ep_run(h_ep, l_d[8 + i].data_ptr(), ne + 1, x_d[8 + i].data_ptr(), outs[i].data_ptr(), 1, 0, cs)
    ref = torch.zeros((4, d), device="cuda")
    for i in range(4):
        fn.moe_run(h_one, l_d[8 + i].data_ptr(), ne + 1, x_d[8 + i].data_ptr(), ref[i].data_ptr(), 1, 0, s)
    for rep in range(2):
        outs.zero_()
        g.replay()
        fn.sync(s)
        check(same(outs, ref), f"graph replay {rep}")

    K = 200
    g_ep, g_one = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_ep, stream=st):
        cs = torch.cuda.current_stream().cuda_stream
        for i in range(K):
            fn.moe_ep_run(h_ep, l_d[i % NX].data_ptr(), ne + 1, x_d[i % NX].data_ptr(), y_ep.data_ptr(), 1, 0, cs)
    with torch.cuda.graph(g_one, stream=st):
        cs = torch.cuda.current_stream().cuda_stream
        for i in range(K):
            fn.moe_run(h_one, l_d[i % NX].data_ptr(), ne + 1, x_d[i % NX].data_ptr(), y_one.data_ptr(), 1, 0, cs)

    def timed(graph):
        graph.replay()
        fn.sync(s)
        dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        graph.replay()
        b.record(st)
        torch.cuda.synchronize()
        t = torch.tensor([a.elapsed_time(b) / K * 1e3], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    us_ep = timed(g_ep)
    us_one = timed(g_one)
    fn.sync(s)
    check(same(y_ep[0], y_one[0]), "after timed graphs")
    del g, g_ep, g_one

    failure = None
    if "--fail-test" in sys.argv and world > 1:
        dist.barrier()
        if rank != 1:
            fn.moe_ep_run(h_ep, l_d[0].data_ptr(), ne + 1, x_d[0].data_ptr(), y_ep.data_ptr(), 1, 0, s)
            try:
                fn.sync(s)
                failure = "no error"
            except RuntimeError as e:
                failure = "ok" if "peer" in str(e) else f"unexpected: {e}"
            check(failure == "ok", f"failure test: {failure}")
        dist.barrier()

    fn.moe_free(h_ep)
    fn.moe_free(h_one)
    group.close()
    nf = torch.tensor([len(fails)], device="cuda")
    dist.all_reduce(nf)
    if fails:
        print(f"rank {rank} FAIL: {fails}", flush=True)
    if rank == 0:
        print(json.dumps({"test": "MoE expert parallel (config 3)", "n_gpus": world, "experts": ne, "top_k": k,
                          "us_per_layer_ep": round(us_ep, 2), "us_per_layer_one_gpu": round(us_one, 2),
                          "failure_test": failure, "failures": int(nf.item())}), flush=True)
    dist.destroy_process_group()
    sys.exit(1 if int(nf.item()) else 0)


if __name__ == "__main__":
    main()
