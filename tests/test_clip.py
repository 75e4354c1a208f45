"""CLIP text encoder against transformers' CLIPTextModelWithProjection (tiny random config): last
hidden states, the end-of-text pooled state and the projected embedding, on CPU (fp32) and with
the GPU kernels (bf16)."""
import pytest
import torch

from gollek_b200.models.clip import CLIPTextConfig, CLIPTextEncoder


def _hf(eos=999):
    import transformers
    hc = transformers.CLIPTextConfig(vocab_size=1000, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                                     num_attention_heads=4, max_position_embeddings=77, projection_dim=32,
                                     eos_token_id=eos, hidden_act="quick_gelu")
    torch.manual_seed(0)
    m = transformers.CLIPTextModelWithProjection(hc).eval()
    return hc, m


def _ids(eos, lens=(9, 14)):
    g = torch.Generator().manual_seed(1)
    S = max(lens)
    ids = torch.randint(0, 990, (len(lens), S), generator=g)
    for b, n in enumerate(lens):
        ids[b, n - 1] = eos
        ids[b, n:] = eos  # padded with the end-of-text id, as CLIP tokenizers do
    return ids


@pytest.mark.parametrize("eos", [999, 2])
def test_clip_text_encoder_matches_hf(eos):
    hc, m = _hf(eos)
    ids = _ids(eos if eos != 2 else 999)  # legacy id 2: the pooled token is the largest id (999 here)
    sd = m.state_dict()
    enc = CLIPTextEncoder(CLIPTextConfig.from_hf(hc.to_dict()), sd.__getitem__, device="cpu", dtype=torch.float32)
    ours = enc.encode(ids)
    with torch.no_grad():
        ref = m(input_ids=ids)
    torch.testing.assert_close(ours["last_hidden_state"], ref.last_hidden_state, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(ours["text_embeds"], ref.text_embeds, rtol=1e-4, atol=1e-5)


@pytest.mark.gpu
def test_clip_text_encoder_gpu():
    hc, m = _hf()
    ids = _ids(999)
    sd = m.state_dict()
    enc = CLIPTextEncoder(CLIPTextConfig.from_hf(hc.to_dict()), sd.__getitem__, device="cuda")
    ours = enc.encode(ids)
    with torch.no_grad():
        ref = m(input_ids=ids)
    torch.testing.assert_close(ours["last_hidden_state"].float().cpu(), ref.last_hidden_state, rtol=5e-2, atol=5e-2)
    torch.testing.assert_close(ours["text_embeds"].float().cpu(), ref.text_embeds, rtol=5e-2, atol=5e-2)


def _hf_vision():
    import transformers
    vc = transformers.CLIPVisionConfig(hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                                       num_attention_heads=4, image_size=28, patch_size=7, projection_dim=32,
                                       hidden_act="quick_gelu")
    torch.manual_seed(0)
    return vc, transformers.CLIPVisionModelWithProjection(vc).eval()


def test_clip_vision_encoder_matches_hf():
    from gollek_b200.models.clip import CLIPVisionConfig, CLIPVisionEncoder
    vc, m = _hf_vision()
    px = torch.randn(2, 3, 28, 28, generator=torch.Generator().manual_seed(2))
    enc = CLIPVisionEncoder(CLIPVisionConfig.from_hf(vc.to_dict()), m.state_dict().__getitem__, device="cpu",
                            dtype=torch.float32)
    ours = enc.encode(px)
    with torch.no_grad():
        ref = m(pixel_values=px)
    torch.testing.assert_close(ours["last_hidden_state"], ref.last_hidden_state, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(ours["image_embeds"], ref.image_embeds, rtol=1e-4, atol=1e-5)


@pytest.mark.gpu
def test_clip_vision_encoder_gpu():
    from gollek_b200.models.clip import CLIPVisionConfig, CLIPVisionEncoder
    vc, m = _hf_vision()
    px = torch.randn(2, 3, 28, 28, generator=torch.Generator().manual_seed(2))
    enc = CLIPVisionEncoder(CLIPVisionConfig.from_hf(vc.to_dict()), m.state_dict().__getitem__, device="cuda")
    ours = enc.encode(px)
    with torch.no_grad():
        ref = m(pixel_values=px)
    torch.testing.assert_close(ours["image_embeds"].float().cpu(), ref.image_embeds, rtol=5e-2, atol=5e-2)
