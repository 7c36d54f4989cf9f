"""Pins the model oracles' float skeletons to an independent implementation.

oracle/qwen3_ref.py and oracle/siglip_ref.py restate the reference's layer
math (src/qwen3_embedding/model.rs:261-606; the SigLIP-style pre-LN encoder of
the config). With quantisation off (quant=False: f32 weights as they are, f64
arithmetic, no f16 stores) they must equal random-init transformers modules
given the same weights: Qwen3Model (causal, the reference's own mask) and a
SiglipEncoder + post LayerNorm with zero biases. This is the target the
reference's own parity tooling uses (tools/clef_reference.py builds its
expected values from HF layers). CPU only.

Tolerance: transformers keeps RMSNorm, the RoPE angles and the softmax in f32
even in an f64 model, so agreement is at f32 rounding level: max |err| <=
1e-6 * max |ref| and cosine >= 1 - 1e-12 (measured: 1.5e-7 for Qwen3, 2e-9
for SigLIP).
"""
from dataclasses import replace

import numpy as np
import pytest

transformers = pytest.importorskip("transformers")
torch = pytest.importorskip("torch")

COS_MIN = 1.0 - 1e-12
MAX_REL = 1e-6


def cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def max_rel(got, want):
    return float(np.abs(np.asarray(got) - np.asarray(want)).max() / np.abs(want).max())


def _t(a):
    return torch.from_numpy(np.asarray(a, np.float64))


@pytest.mark.parametrize("seq", [1, 37, 96])
def test_qwen3_oracle_matches_transformers(seq):
    from transformers import Qwen3Config as HFConfig, Qwen3Model
    from burn_rocket_b200.qwen3 import Qwen3Config
    from oracle import qwen3_ref
    cfg = replace(Qwen3Config(), layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, inter=384, vocab=300)
    hw = qwen3_ref.make_host_weights(cfg, seed=3, norm_ones=False)
    hc = HFConfig(vocab_size=cfg.vocab, hidden_size=cfg.hidden, intermediate_size=cfg.inter,
                  num_hidden_layers=cfg.layers, num_attention_heads=cfg.heads, num_key_value_heads=cfg.kv_heads,
                  head_dim=cfg.head_dim, rms_norm_eps=cfg.eps, rope_theta=cfg.theta,
                  max_position_embeddings=max(seq, 128), attention_bias=False, tie_word_embeddings=False)
    hc._attn_implementation = "eager"
    model = Qwen3Model(hc).double().eval()
    with torch.no_grad():
        model.embed_tokens.weight.copy_(_t(hw["embed"]))
        model.norm.weight.copy_(_t(hw["final_norm"]))
        for lay, W in zip(model.layers, hw["layers"]):
            a, m = lay.self_attn, lay.mlp
            for mod, key in ((a.q_proj, "wq"), (a.k_proj, "wk"), (a.v_proj, "wv"), (a.o_proj, "wo"),
                             (m.gate_proj, "wg"), (m.up_proj, "wu"), (m.down_proj, "wd"),
                             (a.q_norm, "q_norm"), (a.k_norm, "k_norm"), (lay.input_layernorm, "in_norm"),
                             (lay.post_attention_layernorm, "post_norm")):
                mod.weight.copy_(_t(W[key]))
    ids = np.random.default_rng(seq).integers(0, cfg.vocab, size=seq, dtype=np.int64)
    with torch.no_grad():
        last = model(input_ids=torch.from_numpy(ids)[None]).last_hidden_state[0, -1].numpy()
    want = last / np.linalg.norm(last)
    got = qwen3_ref.forward(hw, cfg, ids, 1, seq, causal=True, quant=False)[0]
    assert cosine(got, want) >= COS_MIN, cosine(got, want)
    assert max_rel(got, want) <= MAX_REL, max_rel(got, want)


@pytest.mark.parametrize("patches", [1, 50])
def test_siglip_oracle_matches_transformers(patches):
    from transformers import SiglipVisionConfig
    from transformers.models.siglip.modeling_siglip import SiglipEncoder
    from burn_rocket_b200.siglip import SiglipConfig
    from oracle import siglip_ref
    cfg = replace(SiglipConfig(), layers=2, hidden=288, heads=4, head_dim=72, inter=400, patches=patches)
    hw = siglip_ref.make_host_weights(cfg, seed=5)
    sc = SiglipVisionConfig(hidden_size=cfg.hidden, intermediate_size=cfg.inter, num_attention_heads=cfg.heads,
                            num_hidden_layers=cfg.layers, layer_norm_eps=cfg.eps, hidden_act="gelu_pytorch_tanh",
                            attention_dropout=0.0)
    sc._attn_implementation = "eager"
    enc = SiglipEncoder(sc).double().eval()
    post = torch.nn.LayerNorm(cfg.hidden, eps=cfg.eps).double()
    with torch.no_grad():
        for lay, W in zip(enc.layers, hw["layers"]):
            a = lay.self_attn
            for mod, key in ((a.q_proj, "wq"), (a.k_proj, "wk"), (a.v_proj, "wv"), (a.out_proj, "wo"),
                             (lay.mlp.fc1, "w1"), (lay.mlp.fc2, "w2")):
                mod.weight.copy_(_t(W[key]))
                mod.bias.zero_()  # the tower's projections carry no bias
            lay.layer_norm1.weight.copy_(_t(W["ln1_g"]))
            lay.layer_norm1.bias.copy_(_t(W["ln1_b"]))
            lay.layer_norm2.weight.copy_(_t(W["ln2_g"]))
            lay.layer_norm2.bias.copy_(_t(W["ln2_b"]))
        post.weight.copy_(_t(hw["post_g"]))
        post.bias.copy_(_t(hw["post_b"]))
    x = np.random.default_rng(patches).standard_normal((patches, cfg.hidden)).astype(np.float32)
    with torch.no_grad():
        want = post(enc(inputs_embeds=_t(x)[None]).last_hidden_state)[0].numpy()
    got = siglip_ref.forward(hw, cfg, x, 1, quant=False)
    assert cosine(got, want) >= COS_MIN, cosine(got, want)
    assert max_rel(got, want) <= MAX_REL, max_rel(got, want)
