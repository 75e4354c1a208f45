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
