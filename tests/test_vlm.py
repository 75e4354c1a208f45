"""Vision-language serving (LLaVA layout) against transformers' LlavaForConditionalGeneration: a
tiny random checkpoint saved to disk, loaded by the engine, greedy tokens for a prompt with an image
placeholder; image preprocessing against CLIPImageProcessor; image-salted prefix cache."""
import numpy as np
import pytest
import torch


def _tiny_llava(tmp_path):
    from transformers import CLIPVisionConfig, LlamaConfig, LlavaConfig, LlavaForConditionalGeneration
    vc = CLIPVisionConfig(hidden_size=64, intermediate_size=128, num_hidden_layers=3, num_attention_heads=4,
                          image_size=56, patch_size=14, projection_dim=32)
    tc = LlamaConfig(vocab_size=320, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                     num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=512, rms_norm_eps=1e-5)
    cfg = LlavaConfig(vision_config=vc, text_config=tc, image_token_index=319, vision_feature_layer=-2,
                      vision_feature_select_strategy="default", projector_hidden_act="gelu")
    torch.manual_seed(0)
    m = LlavaForConditionalGeneration(cfg).eval()
    with torch.no_grad():
        for p in m.parameters():
            p.mul_(3.0)  # larger random weights: decisive logits
    d = str(tmp_path / "llava")
    m.save_pretrained(d, safe_serialization=True)
    return m, d


def test_llava_engine_matches_transformers(tmp_path):
    from gollek_b200.config import EngineConfig
    from gollek_b200.engine.engine import LLMEngine
    from gollek_b200.engine.sequence import SamplingParams
    m, d = _tiny_llava(tmp_path)
    g = torch.Generator().manual_seed(1)
    pixel = torch.randn(3, 56, 56, generator=g)
    prompt = [5, 17, 319, 42, 99, 7]  # one image placeholder
    ec = EngineConfig(model=d, device="cpu", dtype="float32", max_num_seqs=2, max_num_batched_tokens=64,
                      max_model_len=256, use_cuda_graphs=False)
    eng = LLMEngine(ec, num_blocks=32)
    assert eng.vision is not None and eng.vision.tokens_per_image == 16
    out = eng.generate([prompt], SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True),
                       images=[[pixel]])[0].output_token_ids
    # transformers with the same pixels: the processor would expand <image> to 16 tokens
    ids = torch.tensor([[5, 17] + [319] * 16 + [42, 99, 7]])
    with torch.no_grad():
        ref = m.generate(input_ids=ids, pixel_values=pixel[None], max_new_tokens=6, do_sample=False,
                         attention_mask=torch.ones_like(ids))[0, ids.shape[1]:].tolist()
    assert out == ref


def test_image_preprocessing_matches_clip_processor():
    from PIL import Image
    from transformers import CLIPImageProcessor
    from gollek_b200.models.vlm import preprocess_image
    yy, xx = np.mgrid[0:90, 0:130]  # smooth content: bicubic implementations agree to rounding
    img = Image.fromarray(np.stack([127 + 100 * np.sin(xx / 9.0), 127 + 100 * np.cos(yy / 7.0),
                                    127 + 80 * np.sin((xx + yy) / 11.0)], -1).astype(np.uint8))
    ours = preprocess_image(img, 56)
    theirs = CLIPImageProcessor(size={"shortest_edge": 56}, crop_size={"height": 56, "width": 56})(
        img, return_tensors="pt")["pixel_values"][0]
    assert ours.shape == theirs.shape
    assert float((ours - theirs).abs().max()) < 0.03  # resampling rounding only
    assert float((ours - theirs).abs().mean()) < 1e-3
    portrait = preprocess_image(img.transpose(Image.Transpose.ROTATE_90), 56)
    theirs_p = CLIPImageProcessor(size={"shortest_edge": 56}, crop_size={"height": 56, "width": 56})(
        img.transpose(Image.Transpose.ROTATE_90), return_tensors="pt")["pixel_values"][0]
    assert float((portrait - theirs_p).abs().mean()) < 1e-3


def test_image_content_salts_the_prefix_cache(tmp_path):
    """Two requests with identical token ids but different images must not share KV blocks."""
    from gollek_b200.config import EngineConfig
    from gollek_b200.engine.engine import LLMEngine
    from gollek_b200.engine.sequence import SamplingParams
    _, d = _tiny_llava(tmp_path)
    ec = EngineConfig(model=d, device="cpu", dtype="float32", max_num_seqs=2, max_num_batched_tokens=64,
                      max_model_len=256, use_cuda_graphs=False, enable_prefix_caching=True)
    eng = LLMEngine(ec, num_blocks=64)
    prompt = [5, 319] + list(range(20, 60))
    sp = SamplingParams(temperature=0.0, max_tokens=3, ignore_eos=True)
    a = torch.randn(3, 56, 56, generator=torch.Generator().manual_seed(2))
    b = torch.randn(3, 56, 56, generator=torch.Generator().manual_seed(3))
    ra = eng.generate([prompt], sp, images=[[a]])[0].output_token_ids
    hits0 = eng.kv.prefix_hits
    rb = eng.generate([prompt], sp, images=[[b]])[0].output_token_ids
    assert eng.kv.prefix_hits == hits0  # no block of the first image reused for the second
    ra2 = eng.generate([prompt], sp, images=[[a]])[0].output_token_ids
    assert eng.kv.prefix_hits > hits0 and ra2 == ra  # same image: its blocks are reused
    fresh = LLMEngine(EngineConfig(model=d, device="cpu", dtype="float32", max_num_seqs=2, max_num_batched_tokens=64,
                                   max_model_len=256, use_cuda_graphs=False, enable_prefix_caching=False),
                      num_blocks=64)
    assert fresh.generate([prompt], sp, images=[[b]])[0].output_token_ids == rb


def test_chat_completions_with_image_url(tmp_path):
    """OpenAI content parts: an ``image_url`` data URL becomes the image placeholder in the prompt and
    its pixels feed the vision tower; the reply equals the engine's own generate() on the same input.
    Unsupported URL schemes and undecodable data are 400s."""
    import base64
    import io
    from fastapi.testclient import TestClient
    from PIL import Image
    from gollek_b200.config import EngineConfig
    from gollek_b200.engine.engine import LLMEngine
    from gollek_b200.engine.sequence import SamplingParams
    from gollek_b200.server.app import create_app
    from gollek_b200.server.async_engine import AsyncEngine
    from gollek_b200.utils.tokenizer import ByteTokenizer

    class ImageByteTokenizer(ByteTokenizer):  # bytes + "<image>" -> 319
        def token_text(self, i):
            return "<image>" if i == 319 else None

        def encode(self, text):
            ids = []
            for k, part in enumerate(text.split("<image>")):
                ids += ([319] if k else []) + super().encode(part)
            return ids

    _, d = _tiny_llava(tmp_path)
    tok = ImageByteTokenizer(320)
    ec = EngineConfig(model=d, device="cpu", dtype="float32", max_num_seqs=2, max_num_batched_tokens=256,
                      max_model_len=512, use_cuda_graphs=False)
    eng = LLMEngine(ec, tokenizer=tok, num_blocks=64)
    yy, xx = np.mgrid[0:64, 0:80]
    img = Image.fromarray(np.stack([xx * 3, yy * 4, (xx + yy) * 2], -1).astype(np.uint8))
    buf = io.BytesIO()
    img.save(buf, format="PNG")
    url = "data:image/png;base64," + base64.b64encode(buf.getvalue()).decode()
    prompt = tok.apply_chat_template([{"role": "user", "content": "what is <image> this"}])
    sp = SamplingParams(temperature=0.0, max_tokens=5, ignore_eos=True)
    want = eng.generate([prompt], sp, images=[[img]])[0].output_token_ids

    ae = AsyncEngine(eng).start()
    try:
        with TestClient(create_app(ae, model_name="llava")) as c:
            parts = [{"type": "text", "text": "what is "}, {"type": "image_url", "image_url": {"url": url}},
                     {"type": "text", "text": " this"}]
            body = {"model": "llava", "messages": [{"role": "user", "content": parts}], "max_tokens": 5,
                    "temperature": 0, "ignore_eos": True}
            j = c.post("/v1/chat/completions", json=body).json()
            assert j["usage"]["completion_tokens"] == 5
            assert j["choices"][0]["message"]["content"] == tok.decode(want)
            assert j["usage"]["prompt_tokens"] == len(tok.encode(prompt)) - 1 + eng.vision.tokens_per_image
            bad = [{"type": "image_url", "image_url": {"url": "file:///etc/hostname"}}]
            r = c.post("/v1/chat/completions", json={**body, "messages": [{"role": "user", "content": bad}]})
            assert r.status_code == 400
            bad = [{"type": "image_url", "image_url": {"url": "data:image/png;base64,AAAA"}}]
            r = c.post("/v1/chat/completions", json={**body, "messages": [{"role": "user", "content": bad}]})
            assert r.status_code == 400
    finally:
        ae.shutdown()


@pytest.mark.gpu
def test_llava_engine_gpu(tmp_path):
    """bf16 engine on the GPU: image features close to transformers' fp32 ones; the first greedy
    token is (within bf16 rounding of) transformers' argmax."""
    from gollek_b200.config import EngineConfig
    from gollek_b200.engine.engine import LLMEngine
    from gollek_b200.engine.sequence import SamplingParams
    m, d = _tiny_llava(tmp_path)
    pixel = torch.randn(3, 56, 56, generator=torch.Generator().manual_seed(1))
    ec = EngineConfig(model=d, device="cuda", dtype="bfloat16", max_num_seqs=2, max_num_batched_tokens=64,
                      max_model_len=256)
    eng = LLMEngine(ec, num_blocks=32)
    feats = eng.vision.encode(pixel[None].cuda()).float().cpu()
    with torch.no_grad():
        ref_feats = m.model.get_image_features(pixel_values=pixel[None], vision_feature_layer=-2,
                                               vision_feature_select_strategy="default")
    if hasattr(ref_feats, "pooler_output"):  # transformers 5: projected rows per image in pooler_output
        ref_feats = ref_feats.pooler_output
    ref_feats = torch.cat(list(ref_feats)) if isinstance(ref_feats, (list, tuple)) else ref_feats
    # bf16 through a CLIP tower with 3x-scaled random weights: a few percent relative error
    assert float((feats.reshape(-1) - ref_feats.reshape(-1)).norm() / ref_feats.norm()) < 0.1
    out = eng.generate([[5, 17, 319, 42, 99, 7]], SamplingParams(temperature=0.0, max_tokens=2, ignore_eos=True),
                       images=[[pixel]])[0].output_token_ids
    ids = torch.tensor([[5, 17] + [319] * 16 + [42, 99, 7]])
    with torch.no_grad():
        lg = m(input_ids=ids, pixel_values=pixel[None]).logits[0, -1]
    assert float(lg[out[0]]) >= float(lg.max()) - 0.02 * float(lg.max() - lg.min())
