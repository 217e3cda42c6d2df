"""GPU: the allocation-free MoE entry point (fn_moe_layer_static) gives the results of the allocating one.

fn_moe_layer_static serves callers that cannot call cudaMalloc (a host whose device memory all belongs to its own
pool, or a decode loop that must not pay cudaFree's device synchronisation): it takes only device pointers the caller
owns and keeps its scratch in a static device array of the library. This file is named to be collected last, so a
run that stops at its first failure has already run every other test; it also passes alone in a fresh process.
"""

import numpy as np
import pytest

from synth import BY_NAME, random_blocks, random_x

pytestmark = pytest.mark.gpu
MOE_TOL = 1e-5  # the MoE layer's bar in the rest of the suite


def test_static_moe_matches_allocating_entry_point_on_two_calls(fn):
    import torch
    gu, dn, ne, k, ffe, d = BY_NAME["IQ3_XXS"], BY_NAME["Q4_K"], 64, 10, 512, 2048
    rng = np.random.default_rng(42)
    W = [random_blocks(gu, ne * ffe, d, rng), random_blocks(gu, ne * ffe, d, rng), random_blocks(dn, ne * d, ffe, rng),
         random_blocks(gu, ffe, d, rng), random_blocks(gu, ffe, d, rng), random_blocks(dn, d, ffe, rng)]
    # these row sizes (784 and 288 bytes) are 16-byte multiples, so GGUF rows are already at the required stride
    dev = torch.device("cuda", 0)
    wd = [torch.from_numpy(np.ascontiguousarray(w).reshape(-1)).to(dev) for w in W]
    h = fn.moe_create(gu, dn, ne, k, ffe, d, *W)
    stream = torch.cuda.current_stream().cuda_stream
    try:
        for call, nt in enumerate((1, 3)):  # two calls in a row, different inputs and token counts
            x = torch.from_numpy(random_x(nt, d, rng)).to(dev)
            logits = torch.from_numpy((rng.standard_normal((nt, ne + 1)) * 2).astype(np.float32)).to(dev)
            y_ref = torch.zeros(nt, d, device=dev)
            y_static = torch.full((nt, d), float("nan"), device=dev)
            fn.moe_run(h, logits.data_ptr(), ne + 1, x.data_ptr(), y_ref.data_ptr(), nt, 0, stream)
            fn.moe_layer_static(gu, dn, ne, k, ffe, d, [t.data_ptr() for t in wd], logits.data_ptr(), ne + 1,
                                x.data_ptr(), y_static.data_ptr(), nt, stream)
            fn.sync(stream)
            a, b = y_static.cpu().numpy(), y_ref.cpu().numpy()
            assert np.isfinite(a).all(), f"call {call}"
            assert np.abs(a - b).max() <= MOE_TOL * np.abs(b).max(), f"call {call}"
        # the defining property: after the first call, more calls take no device memory at all
        nt = 5  # 5 x 11 x 512 = 28160 floats of the 65536
        x = torch.from_numpy(random_x(nt, d, rng)).to(dev)
        logits = torch.from_numpy((rng.standard_normal((nt, ne + 1)) * 2).astype(np.float32)).to(dev)
        y = torch.zeros(nt, d, device=dev)
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info(0)[0]
        for _ in range(3):
            fn.moe_layer_static(gu, dn, ne, k, ffe, d, [t.data_ptr() for t in wd], logits.data_ptr(), ne + 1,
                                x.data_ptr(), y.data_ptr(), nt, stream)
        fn.sync(stream)
        assert torch.cuda.mem_get_info(0)[0] == free0
    finally:
        fn.moe_free(h)


def test_static_moe_rejects_oversize_and_misaligned(fn):
    import torch
    dev = torch.device("cuda", 0)
    buf = torch.zeros(1 << 20, dtype=torch.uint8, device=dev)
    f = torch.zeros(1 << 16, device=dev)
    p = buf.data_ptr()
    # 8 tokens x 17 slots x 1024 = 139264 floats > 65536: rejected before any launch
    with pytest.raises(RuntimeError, match="static scratch"):
        fn.moe_layer_static(12, 12, 32, 16, 1024, 256, [p] * 6, f.data_ptr(), 33, f.data_ptr(), f.data_ptr(), 8, 0)
    with pytest.raises(RuntimeError, match="16-byte aligned"):
        fn.moe_layer_static(12, 12, 32, 4, 256, 256, [p + 1] + [p] * 5, f.data_ptr(), 33, f.data_ptr(), f.data_ptr(), 1, 0)


def test_static_moe_accepts_up_to_32_tokens(fn):
    """The token limit is the routing words' 32 tokens, with the scratch limit on top: 12 tokens of a small layer run
    (12 x 5 x 256 floats), and the results match the allocating entry point. (Q4_K rows of 512 and 256 columns are
    288 and 144 bytes, 16-byte multiples, so the GGUF rows are already at the entry point's stride.)"""
    import torch
    gu, dn, ne, k, ffe, d = BY_NAME["Q4_K"], BY_NAME["Q4_K"], 16, 4, 256, 512
    rng = np.random.default_rng(43)
    W = [random_blocks(gu, ne * ffe, d, rng), random_blocks(gu, ne * ffe, d, rng), random_blocks(dn, ne * d, ffe, rng),
         random_blocks(gu, ffe, d, rng), random_blocks(gu, ffe, d, rng), random_blocks(dn, d, ffe, rng)]
    dev = torch.device("cuda", 0)
    wd = [torch.from_numpy(np.ascontiguousarray(w).reshape(-1)).to(dev) for w in W]
    h = fn.moe_create(gu, dn, ne, k, ffe, d, *W)
    stream = torch.cuda.current_stream().cuda_stream
    try:
        nt = 12
        x = torch.from_numpy(random_x(nt, d, rng)).to(dev)
        logits = torch.from_numpy((rng.standard_normal((nt, ne + 1)) * 2).astype(np.float32)).to(dev)
        y_ref, y_static = torch.zeros(nt, d, device=dev), torch.zeros(nt, d, device=dev)
        fn.moe_run(h, logits.data_ptr(), ne + 1, x.data_ptr(), y_ref.data_ptr(), nt, 0, stream)
        fn.moe_layer_static(gu, dn, ne, k, ffe, d, [t.data_ptr() for t in wd], logits.data_ptr(), ne + 1,
                            x.data_ptr(), y_static.data_ptr(), nt, stream)
        fn.sync(stream)
        a, b = y_static.cpu().numpy(), y_ref.cpu().numpy()
        assert np.abs(a - b).max() <= MOE_TOL * np.abs(b).max()
    finally:
        fn.moe_free(h)
