"""The fp32 oracle decoder against Hugging Face transformers (tiny Llama / Mixtral)."""
import torch

from gollek_b200.config import preset
from gollek_b200.models.reference import ReferenceDecoder, init_random_weights


def _hf_model(cfg, weights, cls_name):
    import transformers
    hf_cfg = getattr(transformers, cls_name.replace("ForCausalLM", "Config"))(**{
        k: v for k, v in cfg.to_hf().items() if k not in ("architectures", "model_type", "torch_dtype")})
    model = getattr(transformers, cls_name)(hf_cfg).eval()
    missing, unexpected = model.load_state_dict(weights, strict=False)
    assert not [m for m in missing if "rotary" not in m], missing
    return model


def test_reference_llama_matches_hf(tiny_cfg, tiny_weights):
    ids = torch.randint(0, tiny_cfg.vocab_size, (32,), generator=torch.Generator().manual_seed(0))
    ours = ReferenceDecoder(tiny_cfg, tiny_weights).forward(ids)
    hf = _hf_model(tiny_cfg, tiny_weights, "LlamaForCausalLM")
    with torch.no_grad():
        theirs = hf(ids[None]).logits[0]
    torch.testing.assert_close(ours, theirs, rtol=1e-4, atol=1e-4)


def test_reference_llama3_rope_theta():
    cfg = preset("tiny-llama", rope_theta=500000.0)
    w = init_random_weights(cfg, seed=1)
    ids = torch.randint(0, cfg.vocab_size, (24,), generator=torch.Generator().manual_seed(1))
    ours = ReferenceDecoder(cfg, w).forward(ids)
    hf = _hf_model(cfg, w, "LlamaForCausalLM")
    with torch.no_grad():
        theirs = hf(ids[None]).logits[0]
    torch.testing.assert_close(ours, theirs, rtol=1e-4, atol=1e-4)


def test_reference_mixtral_matches_hf():
    cfg = preset("tiny-mixtral")
    w = init_random_weights(cfg, seed=2)
    ids = torch.randint(0, cfg.vocab_size, (20,), generator=torch.Generator().manual_seed(2))
    ours = ReferenceDecoder(cfg, w).forward(ids)
    import transformers
    hf_cfg = transformers.MixtralConfig(**{k: v for k, v in cfg.to_hf().items()
                                           if k not in ("architectures", "model_type", "torch_dtype")})
    model = transformers.MixtralForCausalLM(hf_cfg).eval()
    sd = model.state_dict()
    # transformers >= 5 fuses expert weights; map ours onto whatever layout it uses
    new = {}
    for k in sd:
        if k in w:
            new[k] = w[k]
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        for k in sd:
            if not k.startswith(p):
                continue
            if k.endswith("experts.gate_up_proj"):
                new[k] = torch.stack([torch.cat([w[p + f"block_sparse_moe.experts.{e}.w1.weight"],
                                                 w[p + f"block_sparse_moe.experts.{e}.w3.weight"]], 0)
                                      for e in range(cfg.num_local_experts)])
                if new[k].shape != sd[k].shape:
                    new[k] = new[k].transpose(1, 2)
            elif k.endswith("experts.down_proj"):
                new[k] = torch.stack([w[p + f"block_sparse_moe.experts.{e}.w2.weight"]
                                      for e in range(cfg.num_local_experts)])
                if new[k].shape != sd[k].shape:
                    new[k] = new[k].transpose(1, 2)
            elif k.endswith("mlp.gate.weight") or k.endswith("block_sparse_moe.gate.weight"):
                new[k] = w[p + "block_sparse_moe.gate.weight"]
            elif ".experts." in k and k not in new:
                parts = k.split(".")
                e = int(parts[parts.index("experts") + 1])
                wn = parts[parts.index("experts") + 2]
                new[k] = w[p + f"block_sparse_moe.experts.{e}.{wn}.weight"]
    model.load_state_dict(new, strict=False)
    with torch.no_grad():
        theirs = model(ids[None]).logits[0]
    torch.testing.assert_close(ours, theirs, rtol=1e-4, atol=1e-4)


import pytest  # noqa: E402


def _hf_family_model(cfg, weights):
    import transformers
    d = cfg.to_hf()
    mt = d.pop("model_type")
    arch = d.pop("architectures")[0]
    d.pop("torch_dtype", None)
    hf_cfg = transformers.AutoConfig.for_model(mt, **d)
    hf_cfg._attn_implementation = "eager"
    model = getattr(transformers, arch)(hf_cfg).eval()
    missing, unexpected = model.load_state_dict(weights, strict=False)
    assert not [m for m in missing if "rotary" not in m and not m.endswith("lm_head.weight")], missing
    assert not unexpected, unexpected
    if cfg.tie_word_embeddings:
        model.tie_weights()
    return model


@pytest.mark.parametrize("name,S", [("tiny-qwen2", 30), ("tiny-qwen3", 30), ("tiny-mistral", 48),
                                    ("tiny-gemma", 30), ("tiny-gemma2", 40), ("tiny-gemma3", 40),
                                    ("tiny-phi3", 56), ("tiny-cohere2", 40)])
def test_reference_family_matches_hf(name, S):
    """Each family's oracle forward (biases, QK-norm, windows longer than the sequence window,
    softcaps, sandwich norms, GeGLU, (1 + w) norms, per-layer RoPE bases) equals transformers'."""
    cfg = preset(name)
    w = init_random_weights(cfg, seed=3)
    ids = torch.randint(0, cfg.vocab_size, (S,), generator=torch.Generator().manual_seed(3))
    ours = ReferenceDecoder(cfg, w).forward(ids)
    hf = _hf_family_model(cfg, w)
    with torch.no_grad():
        theirs = hf(ids[None]).logits[0]
    torch.testing.assert_close(ours, theirs, rtol=1e-4, atol=2e-4)


def test_family_configs_parse_from_hf():
    import transformers
    from gollek_b200.config import ModelConfig
    for name in ("tiny-qwen2", "tiny-qwen3", "tiny-mistral", "tiny-gemma", "tiny-gemma2", "tiny-gemma3", "tiny-phi3",
                 "tiny-cohere2"):
        cfg = preset(name)
        d = cfg.to_hf()
        mt = d.pop("model_type")
        d.pop("architectures")
        d.pop("torch_dtype", None)
        hf_cfg = transformers.AutoConfig.for_model(mt, **d)
        back = ModelConfig.from_hf(hf_cfg.to_dict())
        for f in ("architecture", "head_dim", "sliding_window", "layer_types", "qk_norm", "attention_bias",
                  "sandwich_norm", "norm_unit_offset", "hidden_act", "query_pre_attn_scalar",
                  "attn_logit_softcapping", "final_logit_softcapping", "tie_word_embeddings", "norm_center",
                  "parallel_block", "rope_interleaved", "rope_sliding_only", "logit_scale"):
            assert getattr(back, f) == getattr(cfg, f), (name, f, getattr(back, f), getattr(cfg, f))
        assert abs(back.rope_theta - cfg.rope_theta) < 1e-3 and abs(back.embed_scale - cfg.embed_scale) < 1e-6
