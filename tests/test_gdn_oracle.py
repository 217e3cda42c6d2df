"""CPU: the gated-DeltaNet oracle is pinned against transformers' reference recurrence.

transformers 5.5.0 torch_causal_conv1d_update + torch_recurrent_gated_delta_rule (modeling_qwen3_next.py:350-366,
454-495) compute the same conv + delta rule; they group value heads as h // (nv / nk) and this engine (like the
reference's GGUF order, engine/faie2fn.cu:1374) as h % nk, so the test feeds transformers the key heads repeated in
the engine's order. transformers casts the recurrence to float32, hence the 1e-5 tolerance.
"""

import numpy as np
import pytest

from oracle import gdn as G

torch = pytest.importorskip("torch")


def test_gdn_oracle_matches_transformers_recurrence():
    from transformers.models.qwen3_next.modeling_qwen3_next import (torch_causal_conv1d_update,
                                                                    torch_recurrent_gated_delta_rule)
    rng = np.random.default_rng(0)
    nkh, nvh, ds, nt = 2, 4, 128, 5
    convch = 2 * nkh * ds + nvh * ds
    qkv = rng.standard_normal((nt, convch))
    z = rng.standard_normal((nt, nvh * ds))
    ab = rng.standard_normal((nt, 2 * nvh))
    conv_w = rng.standard_normal((convch, 4)) * 0.5
    dt_bias = rng.standard_normal(nvh)
    ssm_a = -np.exp(rng.standard_normal(nvh) * 0.5)
    norm_w = 1 + 0.1 * rng.standard_normal(ds)
    S0 = rng.standard_normal((nvh, ds, ds)) * 0.02
    c0 = rng.standard_normal((3, convch))
    out, S, cs = G.gdn_run(qkv, z, ab, conv_w, dt_bias, ssm_a, norm_w, S0, c0, nkh, nvh, ds)

    # transformers: conv on all channels, token by token
    state = torch.tensor(c0.T[None].copy())  # [1][CONVCH][3]
    xs = []
    for t in range(nt):
        y = torch_causal_conv1d_update(torch.tensor(qkv[t][None, :, None]), state, torch.tensor(conv_w), None, "silu")
        xs.append(y[0, :, 0].numpy())
    xs = np.array(xs)
    q = xs[:, :nkh * ds].reshape(nt, nkh, ds)
    k = xs[:, nkh * ds:2 * nkh * ds].reshape(nt, nkh, ds)
    v = xs[:, 2 * nkh * ds:].reshape(nt, nvh, ds)
    hmap = [h % nkh for h in range(nvh)]  # the engine's value-head -> key-head map
    qh, kh = q[:, hmap], k[:, hmap]
    beta = 1 / (1 + np.exp(-ab[:, nvh:]))
    g = ssm_a * np.where(ab[:, :nvh] + dt_bias > 20, ab[:, :nvh] + dt_bias, np.log1p(np.exp(ab[:, :nvh] + dt_bias)))
    o, Sf = torch_recurrent_gated_delta_rule(torch.tensor(qh[None]), torch.tensor(kh[None]), torch.tensor(v[None]),
                                             torch.tensor(g[None]), torch.tensor(beta[None]),
                                             torch.tensor(S0[None]), True, use_qk_l2norm_in_kernel=True)
    o = o[0].double().numpy()  # [nt][nvh][ds]
    want = o / np.sqrt((o * o).mean(-1, keepdims=True) + 1e-6) * norm_w / (1 + np.exp(-z.reshape(nt, nvh, ds)))
    assert np.allclose(out.reshape(nt, nvh, ds), want, rtol=1e-5, atol=1e-5)
    assert np.allclose(S, Sf[0].double().numpy(), rtol=1e-5, atol=1e-6)
    assert np.allclose(cs, state[0].numpy().T)
