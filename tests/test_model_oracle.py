"""CPU: the float64 model oracle (oracle/model.py) is pinned against transformers 5.5.0 Qwen3NextForCausalLM in float64.

The reference's own oracle is a float64 transformers forward over its dequantised GGUF weights (flashnext/ref_fn.py:
123-215); here a small Qwen3-Next of the config-5 structure (3 gated-DeltaNet layers then 1 gated-attention layer,
head sizes 128 and 256, partial RoPE on 64 of 256 dims with theta 1e7, a top-k MoE with a sigmoid-gated shared expert)
runs a token sequence in transformers, its weights are mapped into the oracle's layout, and the oracle steps the same
tokens one at a time. The mapping states the conventions where the two differ, each explicitly:
  * RMSNorm weights: transformers scales by (1 + w) (Qwen3NextRMSNorm, modeling_qwen3_next.py:158-176); the oracle by
    w, so it gets 1 + w (the gated norm of the DeltaNet output scales by w in both).
  * DeltaNet head order: transformers groups the projection rows per key head ([q k v z] of key head g, then its
    value heads; fix_query_key_value_ordering, :563-590) and maps value head i to key head i // (nv / nk); the engine
    (like the reference's GGUF order, engine/faie2fn.cu:1374) stacks [q | k | v | z] and maps value head j to key
    head j % nk, so the oracle's value head j is transformers' head (j % nk) (nv / nk) + j // nk.
  * The DeltaNet output gate: silu(z) in transformers (Qwen3NextRMSNormGated, :67-82), sigmoid(z) in the reference
    (engine/faie2fn.cu:1424). The test runs transformers with its gated norm using sigmoid(z), the reference's
    convention, so everything else is compared as is.
transformers keeps the DeltaNet recurrence, the RoPE tables and the router softmax in float32, hence the tolerance:
logits within 1e-5 of max |logit|.
"""

import numpy as np
import pytest

from oracle.model import OracleModel

torch = pytest.importorskip("torch")
TOL = 1e-5


def _tiny_config():
    from transformers import Qwen3NextConfig
    cfg = Qwen3NextConfig(
        vocab_size=96, hidden_size=64, num_hidden_layers=4, num_attention_heads=4, num_key_value_heads=1,
        head_dim=256, linear_num_key_heads=2, linear_num_value_heads=4, linear_key_head_dim=128,
        linear_value_head_dim=128, linear_conv_kernel_dim=4, num_experts=8, num_experts_per_tok=3,
        moe_intermediate_size=32, shared_expert_intermediate_size=32, norm_topk_prob=True, rms_norm_eps=1e-6,
        full_attention_interval=4, tie_word_embeddings=False, hidden_act="silu",
        rope_parameters={"rope_type": "default", "rope_theta": 1e7, "partial_rotary_factor": 0.25})
    cfg._attn_implementation = "eager"
    cfg._experts_implementation = "eager"
    return cfg


def _map_weights(model, c):
    """transformers' parameters -> the oracle's dense layout (see the module docstring for the conventions)."""
    P = {k: v.detach().double().numpy() for k, v in model.named_parameters()}
    nk, nv, dk, dv = c.linear_num_key_heads, c.linear_num_value_heads, c.linear_key_head_dim, c.linear_value_head_dim
    r = nv // nk
    hf = [(j % nk) * r + j // nk for j in range(nv)]  # the oracle's value head j -> transformers' value head
    nh, nkv, D = c.num_attention_heads, c.num_key_value_heads, c.hidden_size
    layers = []
    for l in range(c.num_hidden_layers):
        p = f"model.layers.{l}."
        L = dict(norm1=1.0 + P[p + "input_layernorm.weight"], norm2=1.0 + P[p + "post_attention_layernorm.weight"])
        if c.layer_types[l] == "linear_attention":
            L["kind"] = "G"
            W = P[p + "linear_attn.in_proj_qkvz.weight"]  # per key head g: q_g, k_g, v of its r value heads, z of them
            blk = 2 * dk + 2 * r * dv
            q = np.concatenate([W[g * blk:g * blk + dk] for g in range(nk)])
            k = np.concatenate([W[g * blk + dk:g * blk + 2 * dk] for g in range(nk)])
            vrow = lambda i: W[(i // r) * blk + 2 * dk + (i % r) * dv:][:dv]  # noqa: E731
            zrow = lambda i: W[(i // r) * blk + 2 * dk + r * dv + (i % r) * dv:][:dv]  # noqa: E731
            v = np.concatenate([vrow(hf[j]) for j in range(nv)])
            z = np.concatenate([zrow(hf[j]) for j in range(nv)])
            BA = P[p + "linear_attn.in_proj_ba.weight"]  # per key head g: b of its r value heads, then a
            b = np.stack([BA[(hf[j] // r) * 2 * r + hf[j] % r] for j in range(nv)])
            a = np.stack([BA[(hf[j] // r) * 2 * r + r + hf[j] % r] for j in range(nv)])
            conv = P[p + "linear_attn.conv1d.weight"][:, 0, :]  # [channels][4], channels q | k | v (transformers order)
            cv = conv[2 * nk * dk:]
            conv_w = np.concatenate([conv[:2 * nk * dk]] + [cv[hf[j] * dv:(hf[j] + 1) * dv] for j in range(nv)])
            out = P[p + "linear_attn.out_proj.weight"]
            L.update(w_in=np.concatenate([q, k, v, z]), w_ab=np.concatenate([a, b]),
                     w_out=np.concatenate([out[:, hf[j] * dv:(hf[j] + 1) * dv] for j in range(nv)], axis=1),
                     conv_w=conv_w, dt_bias=P[p + "linear_attn.dt_bias"][hf],
                     ssm_a=-np.exp(P[p + "linear_attn.A_log"][hf]), gnorm=P[p + "linear_attn.norm.weight"])
        else:
            L["kind"] = "A"
            L.update(w_q=P[p + "self_attn.q_proj.weight"], w_k=P[p + "self_attn.k_proj.weight"],
                     w_v=P[p + "self_attn.v_proj.weight"], w_o=P[p + "self_attn.o_proj.weight"],
                     q_norm=1.0 + P[p + "self_attn.q_norm.weight"], k_norm=1.0 + P[p + "self_attn.k_norm.weight"])
        gu = P[p + "mlp.experts.gate_up_proj"]  # [ne][2 ffe][D]
        ffe = c.moe_intermediate_size
        L["router"] = np.concatenate([P[p + "mlp.gate.weight"], P[p + "mlp.shared_expert_gate.weight"]])
        L["experts"] = (gu[:, :ffe], gu[:, ffe:], P[p + "mlp.experts.down_proj"],
                        P[p + "mlp.shared_expert.gate_proj.weight"], P[p + "mlp.shared_expert.up_proj.weight"],
                        P[p + "mlp.shared_expert.down_proj.weight"])
        layers.append(L)
    dense = dict(E=P["model.embed_tokens.weight"], Hd=P["lm_head.weight"], final_norm=1.0 + P["model.norm.weight"],
                 layers=layers)
    ocfg = dict(D=D, vocab=c.vocab_size, eps=c.rms_norm_eps, nkh=nk, nvh=nv, nh=nh, nkv=nkv, k=c.num_experts_per_tok,
                ne=c.num_experts, ffe=ffe)
    return ocfg, dense


def test_model_oracle_matches_transformers_qwen3next(monkeypatch):
    from transformers.models.qwen3_next import modeling_qwen3_next as Q
    c = _tiny_config()
    torch.manual_seed(0)
    model = Q.Qwen3NextForCausalLM(c).double().eval()
    with torch.no_grad():
        for name, prm in model.named_parameters():
            if name.endswith("A_log"):
                prm.copy_(torch.log(torch.rand(prm.shape, dtype=torch.float64) * 4 + 0.5))
            elif name.endswith("dt_bias"):
                prm.copy_(torch.randn(prm.shape, dtype=torch.float64) * 0.5)
            elif "norm" in name:
                prm.copy_(torch.randn(prm.shape, dtype=torch.float64) * 0.1)
            else:
                prm.copy_(torch.randn(prm.shape, dtype=torch.float64) * 0.2)

    def gated_norm_sigmoid(self, hidden_states, gate=None):  # the reference's sigmoid(z) output gate
        x = hidden_states.to(torch.float32)
        x = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.variance_epsilon)
        x = self.weight * x.to(hidden_states.dtype)
        return (x * torch.sigmoid(gate.to(torch.float32))).to(hidden_states.dtype)

    monkeypatch.setattr(Q.Qwen3NextRMSNormGated, "forward", gated_norm_sigmoid)
    tokens = np.random.default_rng(1).integers(0, c.vocab_size, 7)
    with torch.no_grad():
        want = model(torch.tensor(tokens[None])).logits[0].double().numpy()
    ocfg, dense = _map_weights(model, c)
    inv_freq = model.model.rotary_emb.inv_freq.double().numpy()
    o = OracleModel.from_dense(ocfg, dense, inv_freq)
    for i, t in enumerate(tokens):
        got = o.step(int(t))
        err = np.abs(got - want[i]).max() / np.abs(want[i]).max()
        assert err <= TOL, f"position {i}: {err:.3e}"
        assert int(np.argmax(got)) == int(np.argmax(want[i]))
