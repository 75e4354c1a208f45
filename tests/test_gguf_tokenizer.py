"""GGUF tokenizers against their oracles on the same vocabularies: SentencePiece BPE (the
sentencepiece library) and byte-level BPE with merges (HF ``tokenizers``), plus special tokens and
the GGUF chat template."""
import pytest

from gollek_b200.utils.tokenizer import GGUFTokenizer

CORPUS = [
    "The quick brown fox jumps over the lazy dog.",
    "Tensor parallel inference on Blackwell GPUs uses NVLink and NVSwitch.",
    "Paged attention stores the KV cache in blocks of 16 tokens; prefix caching reuses them.",
    "Numbers like 12345 and 3.14159 appear, as do emails such as someone@example.com!",
    "Unicode: naïve café, façade, Zürich, 東京, Москва, emoji 🙂 and tabs\tand  double  spaces.",
    "def forward(self, x):\n    return self.linear(x) + 1\n",
] * 40

TESTS = [
    "The lazy fox paged over 16 KV blocks.",
    "Zürich naïve café 東京 🙂 — new words: Blackwellish NVSwitching!",
    "  leading spaces and trailing   ",
    "line one\nline two\n\n  indented 42 and 1234567",
    "someone@example.com costs $3.14",
]


@pytest.fixture(scope="module")
def spm_model(tmp_path_factory):
    spm = pytest.importorskip("sentencepiece")
    d = tmp_path_factory.mktemp("spm")
    corpus = d / "corpus.txt"
    corpus.write_text("\n".join(CORPUS))
    prefix = str(d / "m")
    spm.SentencePieceTrainer.train(input=str(corpus), model_prefix=prefix, model_type="bpe", vocab_size=400,
                                   byte_fallback=True, normalization_rule_name="identity",
                                   remove_extra_whitespaces=False, character_coverage=1.0,
                                   split_digits=False, allow_whitespace_only_pieces=True, minloglevel=2)
    return spm.SentencePieceProcessor(model_file=prefix + ".model")


def test_spm_bpe_matches_sentencepiece(spm_model):
    sp = spm_model
    n = sp.get_piece_size()
    tokens = [sp.id_to_piece(i) for i in range(n)]
    scores = [sp.get_score(i) for i in range(n)]
    types = [3 if sp.is_control(i) else 2 if sp.is_unknown(i) else 6 if sp.is_byte(i) else 1 for i in range(n)]
    tok = GGUFTokenizer(tokens, scores, bos=sp.bos_id(), eos=sp.eos_id(), model="llama", token_types=types,
                        add_bos=False)
    for text in TESTS + CORPUS[:6]:
        assert tok.encode(text) == sp.encode(text), text
        assert tok.decode(tok.encode(text)) == sp.decode(sp.encode(text))
    assert tok.encode("hi", add_special=True)[:1] != [sp.bos_id()]  # add_bos=False
    tok_b = GGUFTokenizer(tokens, scores, bos=sp.bos_id(), eos=sp.eos_id(), model="llama", token_types=types)
    assert tok_b.encode("hi")[0] == sp.bos_id()


def _hf_bpe(pattern):
    tk = pytest.importorskip("tokenizers")
    from tokenizers import Regex, Tokenizer, decoders, models, pre_tokenizers, trainers
    t = Tokenizer(models.BPE())
    if pattern is None:
        t.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=True)
    else:
        t.pre_tokenizer = pre_tokenizers.Sequence([
            pre_tokenizers.Split(Regex(pattern), behavior="isolated"),
            pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)])
    t.decoder = decoders.ByteLevel()
    tr = trainers.BpeTrainer(vocab_size=600, initial_alphabet=pre_tokenizers.ByteLevel.alphabet(),
                             special_tokens=["<|begin_of_text|>", "<|eot_id|>"], show_progress=False)
    t.train_from_iterator(CORPUS, tr)
    del tk
    return t


@pytest.mark.parametrize("pre", ["default", "llama-bpe"])
def test_byte_level_bpe_matches_hf_tokenizers(pre):
    import json
    from gollek_b200.utils.tokenizer import _PRE_PATTERNS
    hf = _hf_bpe(None if pre == "default" else _PRE_PATTERNS[pre])
    model = json.loads(hf.to_str())["model"]
    vocab = model["vocab"]
    merges = [m if isinstance(m, str) else " ".join(m) for m in model["merges"]]
    tokens = [None] * len(vocab)
    for piece, i in vocab.items():
        tokens[i] = piece
    types = [3 if p in ("<|begin_of_text|>", "<|eot_id|>") else 1 for p in tokens]
    tok = GGUFTokenizer(tokens, None, bos=vocab["<|begin_of_text|>"], eos=vocab["<|eot_id|>"], model="gpt2",
                        merges=merges, token_types=types, pre=pre, add_bos=False)
    for text in TESTS + CORPUS[:6]:
        assert tok.encode(text) == hf.encode(text).ids, (pre, text)
        assert tok.decode(tok.encode(text)) == text
    # a control token written in the text is one id, and decoding drops it
    ids = tok.encode("hello<|eot_id|>world")
    assert vocab["<|eot_id|>"] in ids and tok.decode(ids) == "helloworld"


def test_gguf_metadata_tokenizer_and_chat_template(tmp_path):
    from gollek_b200.loaders import gguf as G
    tmpl = ("{{ bos_token }}{% for m in messages %}<|{{ m['role'] }}|>{{ m['content'] }}<|end|>{% endfor %}"
            "{% if add_generation_prompt %}<|assistant|>{% endif %}")
    w = G.GGUFWriter(str(tmp_path / "t.gguf"))
    w.add("general.architecture", "llama")
    toks = ["<unk>", "<s>", "</s>"] + [f"<0x{b:02X}>" for b in range(256)] + ["▁h", "▁hi", "i"]
    w.add("tokenizer.ggml.model", "llama")
    w.add("tokenizer.ggml.tokens", toks, G.T_ARR, G.T_STR)
    w.add("tokenizer.ggml.scores", [0.0] * 259 + [-1.0, 0.0, -2.0], G.T_ARR, G.T_F32)
    w.add("tokenizer.ggml.token_type", [2, 3, 3] + [6] * 256 + [1, 1, 1], G.T_ARR, G.T_I32)
    w.add("tokenizer.ggml.bos_token_id", 1)
    w.add("tokenizer.ggml.eos_token_id", 2)
    w.add("tokenizer.chat_template", tmpl)
    w.write()
    f = G.GGUFFile(str(tmp_path / "t.gguf"))
    tok = GGUFTokenizer.from_metadata(f.metadata)
    f.close()
    assert tok.encode("hi") == [1, 260]  # BOS, then "▁hi" (merged by score over "▁h" + "i")
    assert tok.decode([1, 260]) == "hi"
    text = tok.apply_chat_template([{"role": "user", "content": "yo"}])
    assert text == "<|user|>yo<|end|><|assistant|>"  # the rendered BOS is left to encode()


def test_wordpiece_matches_hf_bert_tokenizer():
    """GGUF ``bert`` vocabularies (phantom-space form, as GGUF stores them) and the ``##`` form both
    tokenize like HF tokenizers' BERT WordPiece (uncased), with [CLS] / [SEP] around the ids."""
    from tokenizers import BertWordPieceTokenizer
    from gollek_b200.utils.tokenizer import GGUFTokenizer
    words = ["the", "run", "##ning", "##s", "un", "##believ", "##able", "thing", "hello", "world", "na", "##ive",
             "cafe", "token", "##izer", "a", "b", "c", "x", "##x", "test", "##ed", "中", "文", "don", "'", "t"]
    punct = list(",.!?-()'\"") + [";", ":"]
    vocab = ["[PAD]", "[UNK]", "[CLS]", "[SEP]", "[MASK]"] + words + [p for p in punct if p not in words]
    hf = BertWordPieceTokenizer({t: i for i, t in enumerate(vocab)}, lowercase=True)
    phantom = [t if (t.startswith("[") and t.endswith("]")) else (t[2:] if t.startswith("##") else "▁" + t)
               for t in vocab]
    types = [3 if (t.startswith("[") and t.endswith("]")) else 1 for t in vocab]
    texts = ["Hello, world!", "The running things... Unbelievable!", "naïve Café; TESTED tokenizers",
             "don't stop", "中文 mixed\twith\ncontrol\x07 chars", "zzz qqq", "x" * 150, "xxxx", "(a) [MASK] b",
             "  leading and trailing  ", ""]
    for form in (phantom, vocab):
        tok = GGUFTokenizer(form, None, bos=2, eos=3, model="bert", token_types=types)
        for text in texts:
            assert tok.encode(text) == hf.encode(text).ids, (form is phantom, text)
        assert tok.decode(tok.encode("the running things")) == "the running things"
    meta = {"tokenizer.ggml.model": "bert", "tokenizer.ggml.tokens": phantom, "tokenizer.ggml.token_type": types,
            "tokenizer.ggml.bos_token_id": 2, "tokenizer.ggml.eos_token_id": 3, "tokenizer.ggml.unknown_token_id": 1}
    t2 = GGUFTokenizer.from_metadata(meta)
    assert t2.encode("Hello, world!") == hf.encode("Hello, world!").ids
    assert t2.encode("hello", add_special=False) == [vocab.index("hello")]
