"""The decoder stack (``dsalt_b200.model``): the reference's module names and state-dict
keys (CPU; checked against the reference's recorded layout), and a GPU
prefill of a small Qwen-shaped model (grouped kv heads, head_dim 128, q/k/v bias,
block-causal selection) that is deterministic, finite and whose last-token logits equal
the full computation's."""
import json
import os

import pytest
import torch

from dsalt_b200.model import DSALTConfig, DSALTLMHeadModel

SMALL = dict(vocab_size=1000, d_model=256, n_layers=2, n_heads=4, n_min=16, n_max=128, k_lmk=32, max_seq_len=4096)


def test_state_dict_keys_follow_the_reference_layout():
    m = DSALTLMHeadModel.from_config(DSALTConfig(**SMALL, n_kv_heads=2, qkv_bias=True))
    keys = set(m.state_dict())
    for k in ("embed_tokens.weight", "lm_head.weight", "final_norm.weight", "layers.1.attn_norm.weight",
              "layers.1.ffn_norm.weight", "layers.1.attn.q_proj.weight", "layers.1.attn.q_proj.bias",
              "layers.1.attn.k_proj.weight", "layers.1.attn.v_proj.weight", "layers.1.attn.out_proj.weight",
              "layers.1.attn.win_gate.weight", "layers.1.attn.win_gate.bias", "layers.1.attn.alpha_w",
              "layers.1.ffn.gate_proj.weight", "layers.1.ffn.up_proj.weight", "layers.1.ffn.down_proj.weight"):
        assert k in keys, k
    # the reference's own layout for this configuration (tests/golden/make_lm_keys.py)
    with open(os.path.join(os.path.dirname(__file__), "golden", "lm_state_dict_small.json")) as f:
        ref = json.load(f)
    assert ref["config"] == dict(SMALL, n_kv_heads=2, qkv_bias=True)
    ms = {k: list(v.shape) for k, v in m.state_dict().items()}
    assert ms == ref["state_dict"]


@pytest.mark.gpu
def test_prefill_qwen_shaped_small():
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    cfg = DSALTConfig(vocab_size=1000, d_model=512, n_layers=2, n_heads=4, n_min=16, n_max=512, k_lmk=64,
                      max_seq_len=4096, d_ff=1024, n_kv_heads=2, qkv_bias=True, rope_base=1e6,
                      selection="block_causal", block=512, tie_weights=False)
    m = DSALTLMHeadModel.from_config(cfg).to(dev).to(torch.bfloat16).eval()
    g = torch.Generator(device=dev).manual_seed(1)
    cu = [0, 1500, 3000]
    ids = torch.randint(0, cfg.vocab_size, (cu[-1],), device=dev, generator=g)
    cu_t = torch.tensor(cu, dtype=torch.int32, device=dev)
    a = m(ids, cu_t, cu_list=cu)["logits"]
    b = m(ids, cu_t, cu_list=cu)["logits"]
    last = m(ids, cu_t, cu_list=cu, logits_to_keep=7)["logits"]
    from dsalt_b200 import ops
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert a.shape == (cu[-1], cfg.vocab_size)
    assert torch.isfinite(a.float()).all()
    assert torch.equal(a, b)
    assert torch.equal(last, a[-7:])
